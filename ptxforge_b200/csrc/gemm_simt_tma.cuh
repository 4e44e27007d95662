// gemm_simt_tma.cuh -- fp32 fused C = gelu_tanh(A.B + bias) on the CUDA cores (FFMA), operands fed by TMA.
//
// The same products and order as the SIMT kernel of gemm_simt.cuh (and the reference kernel,
// kernels/gemm_bias_gelu.cu:62-97): every C[r,c] is the fp32 fmaf chain over k = 0, 1, ..., K-1 from 0, then
// gelu_tanh(acc + bias[c]) in the reference's expression form with tanhf -- bit for bit.  What differs is how
// the operands reach the FFMAs, chosen so that nearly every instruction a thread issues is an FFMA:
//   * one thread per CTA loads each k step's A tile (BM rows x BK k, row-major as in global memory) and B tile
//     (BK rows x BN columns) with two TMA copies into a STAGES-deep ring of shared memory, completion counted
//     on an mbarrier per slot; out-of-range rows, columns and k read as zeros, so the k loop has no bounds
//     checks and no per-element copy instructions;
//   * the A tile lands with the 64-byte (BK = 16) or 128-byte (BK = 32) TMA swizzle, and a thread owns rows
//     ty, ty + TY, ..., ty + (TM-1) TY (TY = BM / TM, a multiple of 8), so for every row it reads the same
//     swizzle term; its 16-byte reads of four consecutive k of a row fall on different banks across the warp;
//   * per group of four k a thread reads its TM rows x 4 k of A (TM 16-byte loads) and, per k, its TN columns
//     of B (TN / 4 16-byte loads, in 4-column groups BN / (TN / 4) apart: a warp's reads cover 128 contiguous
//     bytes), then issues TM x TN FMAs per k, two columns per packed fma.rn.f32x2 (micro_fma);
//   * no CTA-wide barrier in the k loop: each warp arrives on its slot's `empty` mbarrier when done with it, and
//     the copying thread waits for all warps there before refilling the slot, so a warp may run up to
//     STAGES - 1 k steps ahead of another.  Every wait is bounded: one that runs out sets a bit in the status
//     word and a CTA-wide abort flag, the CTA's threads leave the loop, and it exits after its copies in flight
//     have landed (also bounded).
// Needs 16-byte row strides (K and N multiples of 4) and 16-byte aligned operands; the library launches the
// cp.async kernel of gemm_simt.cuh elsewhere.
#pragma once

#include <cstdint>

#include "gemm_simt.cuh"
#include "sm100.cuh"

namespace pf {

template <int BM, int BN, int BK, int TM, int TN, int STAGES>
struct SimtTmaConfig {
  static constexpr int THREADS = (BM / TM) * (BN / TN);
  static constexpr int TX = BN / TN;
  static constexpr int TY = BM / TM;
  static constexpr int SWIZZLE_BYTES = BK * 4;              // one A row: 64 or 128 bytes
  static constexpr int A_BYTES = BM * BK * 4;
  static constexpr int B_BYTES = BK * BN * 4;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int WARPS = THREADS / 32;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 2 * STAGES * 8 + 16;
  // Registers per thread: 128 for micro-tiles up to 8 x 4 (then 65,536 / (128 * THREADS) CTAs fit an SM), 168
  // for 8 x 8, whose 64 accumulators, operand pairs and addresses need about 140 (at 128 they spilled).
  static constexpr int REG_TARGET = TM * TN >= 64 ? 168 : 128;
  static constexpr int MIN_BLOCKS = THREADS * REG_TARGET <= 65536 ? 65536 / (THREADS * REG_TARGET) : 1;
  static_assert(BK == 16 || BK == 32, "A rows are one 64- or 128-byte swizzle span");
  static_assert(TY % 8 == 0, "a thread's rows share one swizzle term: TY a multiple of 8");
  static_assert(TN % 4 == 0 && BN % 4 == 0, "B is read in 4-column groups");
  static_assert(B_BYTES % 1024 == 0 || STAGES == 1, "slots stay 1024-byte aligned");
  static_assert(A_BYTES % 1024 == 0, "slots stay 1024-byte aligned");
};

template <int BM, int BN, int BK, int TM, int TN, int STAGES>
__global__ void __launch_bounds__(SimtTmaConfig<BM, BN, BK, TM, TN, STAGES>::THREADS,
                                  SimtTmaConfig<BM, BN, BK, TM, TN, STAGES>::MIN_BLOCKS)
    gemm_bias_gelu_simt_tma(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const float *__restrict__ bias, float *__restrict__ C, int M, int N, int K,
                            unsigned *status, unsigned long long timeout_ns) {
  using Cfg = SimtTmaConfig<BM, BN, BK, TM, TN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t *sA = smem;                                 // [STAGES][BM][BK], swizzled rows
  uint8_t *sB = smem + STAGES * Cfg::A_BYTES;         // [STAGES][BK][BN]
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * Cfg::STAGE_BYTES);  // [STAGES] copies landed
  uint64_t *empty = full + STAGES;                                                   // [STAGES] warps done
  volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + STAGES);

  const int tid = threadIdx.x;
  const int tx = tid % Cfg::TX;
  const int ty = tid / Cfg::TX;
  const int row0 = blockIdx.y * BM;
  const int col0 = blockIdx.x * BN;
  const int ktiles = (K + BK - 1) / BK;

  if (tid == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], Cfg::WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  __syncthreads();

  int issued = 0;
  auto issue = [&](int kt) {
    const int s = kt % STAGES;
    mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
    tma_load_2d(sA + s * Cfg::A_BYTES, &tmA, &full[s], kt * BK, row0);
    tma_load_2d(sB + s * Cfg::B_BYTES, &tmB, &full[s], col0, kt * BK);
    ++issued;
  };
  if (tid == 0)
    for (int kt = 0; kt < STAGES - 1 && kt < ktiles; ++kt) issue(kt);

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  // This thread's A rows ty + TY * i share the swizzle term: a row of 64 bytes has its 16-byte chunk c at
  // c ^ ((row >> 1) & 3), a row of 128 bytes at c ^ (row & 7).
  const int xr = Cfg::SWIZZLE_BYTES == 64 ? ((ty >> 1) & 3) : (ty & 7);
  const uint8_t *a_thread = sA + ty * Cfg::SWIZZLE_BYTES;
  const uint8_t *b_thread = sB + tx * 16;
  volatile int no_abort = 0;
  const int lane = tid & 31;

  for (int kt = 0; kt < ktiles; ++kt) {
    bool bad = false;
    if (tid == 0 && kt + STAGES - 1 < ktiles) {
      // Refill the slot of step kt-1 once every warp is done with it.
      const int next = kt + STAGES - 1;
      if (next >= STAGES &&
          !mbar_wait(&empty[next % STAGES], static_cast<uint32_t>((next / STAGES - 1) & 1), timeout_ns, abort_flag))
        bad = true;
      else
        issue(next);
    }
    const int s = kt % STAGES;
    if (!bad && !mbar_wait(&full[s], static_cast<uint32_t>((kt / STAGES) & 1), timeout_ns, abort_flag)) bad = true;
    if (bad && !*abort_flag) {
      atomicOr(status, 1u);  // bit 0: a wait of the fp32 kernel ran out
      *abort_flag = 1;
    }
    if (__any_sync(0xffffffffu, bad)) break;  // the whole warp leaves together
    const uint8_t *a_slot = a_thread + s * Cfg::A_BYTES;
    const uint8_t *b_slot = b_thread + s * Cfg::B_BYTES;
#pragma unroll
    for (int k4 = 0; k4 < BK / 4; ++k4) {
      float a[TM][4];
      const int chunk = (k4 ^ xr) * 16;
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        const float4 v = *reinterpret_cast<const float4 *>(a_slot + i * Cfg::TY * Cfg::SWIZZLE_BYTES + chunk);
        a[i][0] = v.x;
        a[i][1] = v.y;
        a[i][2] = v.z;
        a[i][3] = v.w;
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        float b[TN], ak[TM];
#pragma unroll
        for (int i = 0; i < TM; ++i) ak[i] = a[i][kk];
#pragma unroll
        for (int j4 = 0; j4 < TN / 4; ++j4) {
          const float4 v =
              *reinterpret_cast<const float4 *>(b_slot + ((k4 * 4 + kk) * BN + j4 * (BN / (TN / 4))) * 4);
          b[j4 * 4 + 0] = v.x;
          b[j4 * 4 + 1] = v.y;
          b[j4 * 4 + 2] = v.z;
          b[j4 * 4 + 3] = v.w;
        }
        micro_fma<TM, TN>(acc, ak, b);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with the slot
  }
  __syncthreads();  // every thread has left the loop (finished, or stopped by the abort flag)
  if (*abort_flag) {
    if (tid == 0) {
      // Let copies still in flight land before the CTA's shared memory goes away (bounded).
      for (int kt = issued - STAGES > 0 ? issued - STAGES : 0; kt < issued; ++kt)
        (void)mbar_wait(&full[kt % STAGES], static_cast<uint32_t>((kt / STAGES) & 1), timeout_ns, &no_abort);
    }
    return;
  }

  // Fused epilogue: bias + GELU in registers, straight to C (16-byte stores of 4-column groups).
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int r = row0 + ty + i * Cfg::TY;
    if (r >= M) continue;
#pragma unroll
    for (int j4 = 0; j4 < TN / 4; ++j4) {
      const int c = col0 + j4 * (BN / (TN / 4)) + tx * 4;
      if (c < N) {
        const float4 bb = __ldg(reinterpret_cast<const float4 *>(bias + c));
        float4 o;
        o.x = gelu_tanh_ref_f32(acc[i][j4 * 4 + 0] + bb.x);
        o.y = gelu_tanh_ref_f32(acc[i][j4 * 4 + 1] + bb.y);
        o.z = gelu_tanh_ref_f32(acc[i][j4 * 4 + 2] + bb.z);
        o.w = gelu_tanh_ref_f32(acc[i][j4 * 4 + 3] + bb.w);
        *reinterpret_cast<float4 *>(C + static_cast<size_t>(r) * N + c) = o;
      }
    }
  }
}

}  // namespace pf
