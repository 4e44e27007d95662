// gemm_simt.cuh -- fp32 fused C = gelu_tanh(A.B + bias) on the CUDA cores (FFMA), sm_100a.
//
// Same tile parameters as the reference's tunable kernel (kernels/gemm_bias_gelu.cu:16-33): a BM x BN block
// tile, K walked in steps of BK, a TM x TN register micro-tile per thread and PAD floats of padding per row of
// the transposed A tile in shared memory.  How the data moves is this file's own:
//   * a STAGES-deep ring of shared-memory tiles filled by cp.async (LDGSTS), so global loads of the next
//     STAGES - 1 k steps are in flight while a step is computed and no registers stage them; one barrier per
//     k step.  A is transposed on its way in (one 4-byte copy per element into As[k][m], lanes along k so a
//     warp's reads are coalesced and, with BM + PAD = 4 mod 32 and BK = 8, its shared-memory writes
//     conflict-free); B rows go in 16 bytes at a time;
//   * out-of-range elements are zero-filled by the copies themselves (src-size 0), so ragged M / N / K need
//     no other branches in the k loop; stores are guarded;
//   * the micro-tile's A and B fragments of the next k are loaded while the current k's FFMAs issue; when TM
//     and TN are multiples of 4 (and BM + PAD too, for A) a thread owns 4 x 4 sub-blocks spread BM/(TM/4) rows
//     and BN/(TN/4) columns apart, so those loads are conflict-free 16-byte reads;
//   * the ring depth follows the tile: up to 4 stages within the shared memory a CTA gets when as many CTAs
//     as the register file allows share the SM (at most 48 KB, static, so the standalone image loads
//     anywhere); __launch_bounds__ asks for 128 registers per thread where the micro-tile fits them.
// Numerics match the reference kernel element for element: every C[r,c] is accumulated in fp32 by fmaf over
// k = 0, 1, ..., K-1 from 0, then gelu_tanh(acc + bias[c]) is evaluated in the same expression form with
// tanhf (kernels/gemm_bias_gelu.cu:37-40, 75-84, 89-97).  The tiling changes which thread computes an output
// and when its operands arrive, never the order of its fmaf chain.
#pragma once

#include <cstdint>

namespace pf {

// acc[i][j] = fmaf(a[i], b[j], acc[i][j]) for the TM x TN micro-tile.  When TN is even, column pairs (j, j + 1)
// go through one packed FMA (fma.rn.f32x2, sm_100): each half rounds exactly as fmaf, so every output's chain
// and bits are unchanged, but the FMA pipe takes two columns per issued instruction and is no longer starved
// by the loads and address arithmetic that share its issue slots (2048^3: 44.0 -> 48.5 TFLOP/s, same bits).
template <int TM, int TN>
__device__ __forceinline__ void micro_fma(float (&acc)[TM][TN], const float (&a)[TM], const float (&b)[TN]) {
  if constexpr (TN % 2 == 0) {
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const float2 aa = make_float2(a[i], a[i]);
#pragma unroll
      for (int j = 0; j < TN; j += 2) {
        const float2 r = __ffma2_rn(aa, make_float2(b[j], b[j + 1]), make_float2(acc[i][j], acc[i][j + 1]));
        acc[i][j] = r.x;
        acc[i][j + 1] = r.y;
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
}

__device__ __forceinline__ float gelu_tanh_ref_f32(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x * x * x)));
}

__device__ __forceinline__ uint32_t simt_smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Asynchronous global -> shared copies; `src_bytes` < size zero-fills the rest (0: nothing is read).
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int BM, int BN, int BK, int TM, int TN, int PAD>
struct SimtConfig {
  static constexpr int THREADS = (BM / TM) * (BN / TN);
  static constexpr int TX = BN / TN;  // threads along N
  static constexpr int TY = BM / TM;  // threads along M
  // 16-byte reads of the transposed A tile need 16-byte rows: BM + PAD a multiple of 4 floats.
  static constexpr bool SPLIT_M = (TM % 4 == 0) && ((BM + PAD) % 4 == 0);
  static constexpr bool SPLIT_N = (TN % 4 == 0);
  static constexpr int A_ELEMS = BM * BK;                    // 4-byte copies of the A tile
  static constexpr int A_PER = (A_ELEMS + THREADS - 1) / THREADS;
  static constexpr int B_VEC = BK * BN / 4;                  // 16-byte copies of the B tile
  static constexpr int B_VEC_PER = (B_VEC + THREADS - 1) / THREADS;
  static constexpr int B_ELEMS = BK * BN;                    // 4-byte copies when rows are not 16-byte aligned
  static constexpr int B_PER = (B_ELEMS + THREADS - 1) / THREADS;
  static constexpr int A_STAGE_FLOATS = BK * (BM + PAD);
  static constexpr int B_STAGE_FLOATS = BK * BN;
  static constexpr int STAGE_BYTES = 4 * (A_STAGE_FLOATS + B_STAGE_FLOATS);
  // Registers: 128 per thread for micro-tiles up to 8 x 4 (then 65,536 / (128 * THREADS) CTAs fit an SM), 168
  // for 8 x 8 (64 accumulators and the packed-FMA operand pairs spilled at 128), else the compiler's choice.
  static constexpr bool REG_CAP = (TM * TN <= 64) && (THREADS <= 512);
  static constexpr int REG_TARGET = TM * TN >= 64 ? 168 : 128;
  static constexpr int MIN_BLOCKS =
      REG_CAP ? (THREADS * REG_TARGET <= 65536 ? 65536 / (THREADS * REG_TARGET) : 1) : 1;
  // Shared memory per CTA when MIN_BLOCKS of them share the SM's 227 KB (1 KB per CTA is reserved), capped
  // at the 48 KB of static shared memory.
  static constexpr int SMEM_SHARE = 227 * 1024 / MIN_BLOCKS - 1024;
  static constexpr int SMEM_BUDGET = SMEM_SHARE < 48 * 1024 ? SMEM_SHARE : 48 * 1024;
  static constexpr int STAGES_FIT = SMEM_BUDGET / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT >= 4 ? 4 : (STAGES_FIT >= 2 ? STAGES_FIT : 1);
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES;
  static_assert(BM % TM == 0 && BN % TN == 0, "tile not divisible by micro-tile");
  static_assert(BK % 4 == 0 && BN % 4 == 0, "BK and BN must be multiples of 4");
  static_assert(SMEM_BYTES <= 48 * 1024, "static shared memory above 48 KB");
};

// Row of micro-tile element i for thread row ty (and likewise columns).
template <int BM, int TM, bool SPLIT>
__device__ __forceinline__ int micro_index(int ty, int i) {
  if constexpr (SPLIT) {
    return (i >> 2) * (BM / (TM / 4)) + ty * 4 + (i & 3);
  } else {
    return ty * TM + i;
  }
}

// The kernel body, shared by the templated kernel below and by the standalone image with the reference ABI
// (simt_image.cu).  VEC: B's rows, C and bias are 16-byte aligned (N % 4 == 0, aligned pointers), so B is
// copied and C stored 16 bytes at a time.
template <int BM, int BN, int BK, int TM, int TN, int PAD, bool VEC>
__device__ __forceinline__ void gemm_bias_gelu_simt_body(const float *__restrict__ A, const float *__restrict__ B,
                                                         const float *__restrict__ bias, float *__restrict__ C,
                                                         int M, int N, int K) {
  using Cfg = SimtConfig<BM, BN, BK, TM, TN, PAD>;
  constexpr int S = Cfg::STAGES;
  constexpr int LDA = BM + PAD;
  __shared__ __align__(16) float As[S][BK][LDA];  // transposed: As[k][m]
  __shared__ __align__(16) float Bs[S][BK][BN];

  const int tid = threadIdx.x;
  const int tx = tid % Cfg::TX;
  const int ty = tid / Cfg::TX;
  const int row0 = blockIdx.y * BM;
  const int col0 = blockIdx.x * BN;

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  const uint32_t as_base = simt_smem_u32(&As[0][0][0]);
  const uint32_t bs_base = simt_smem_u32(&Bs[0][0][0]);

  // Queue the copies of k step kt into ring slot `slot` (one commit group per call).
  auto issue = [&](int kt, int slot) {
    const int k0 = kt * BK;
#pragma unroll
    for (int l = 0; l < Cfg::A_PER; ++l) {
      const int idx = tid + l * Cfg::THREADS;
      if (Cfg::A_ELEMS % Cfg::THREADS == 0 || idx < Cfg::A_ELEMS) {
        const int r = idx / BK, c = idx % BK;  // lanes along k: coalesced reads
        const int gr = row0 + r, gk = k0 + c;
        const bool ok = gr < M && gk < K;
        const float *src = ok ? A + static_cast<size_t>(gr) * K + gk : A;
        cp_async_4(as_base + 4u * static_cast<uint32_t>((slot * BK + c) * LDA + r), src, ok ? 4u : 0u);
      }
    }
    if constexpr (VEC) {
#pragma unroll
      for (int l = 0; l < Cfg::B_VEC_PER; ++l) {
        const int idx = tid + l * Cfg::THREADS;
        if (Cfg::B_VEC % Cfg::THREADS == 0 || idx < Cfg::B_VEC) {
          const int r = idx / (BN / 4), cq = idx % (BN / 4);
          const int gk = k0 + r, gc = col0 + cq * 4;
          const bool ok = gk < K && gc < N;  // N % 4 == 0: a 16-byte piece is wholly in or out
          const float *src = ok ? B + static_cast<size_t>(gk) * N + gc : B;
          cp_async_16(bs_base + 4u * static_cast<uint32_t>((slot * BK + r) * BN + cq * 4), src, ok ? 16u : 0u);
        }
      }
    } else {
#pragma unroll
      for (int l = 0; l < Cfg::B_PER; ++l) {
        const int idx = tid + l * Cfg::THREADS;
        if (Cfg::B_ELEMS % Cfg::THREADS == 0 || idx < Cfg::B_ELEMS) {
          const int r = idx / BN, c = idx % BN;
          const int gk = k0 + r, gc = col0 + c;
          const bool ok = gk < K && gc < N;
          const float *src = ok ? B + static_cast<size_t>(gk) * N + gc : B;
          cp_async_4(bs_base + 4u * static_cast<uint32_t>((slot * BK + r) * BN + c), src, ok ? 4u : 0u);
        }
      }
    }
    cp_async_commit();
  };

  // One k step's FFMAs from ring slot `slot`, the next k's fragments loaded while this k's issue.
  auto compute = [&](int slot) {
    float a[2][TM], b[2][TN];
    auto load = [&](int k, float(&av)[TM], float(&bv)[TN]) {
      if constexpr (Cfg::SPLIT_M) {
#pragma unroll
        for (int i4 = 0; i4 < TM / 4; ++i4) {
          const float4 v = *reinterpret_cast<const float4 *>(&As[slot][k][i4 * (BM / (TM / 4)) + ty * 4]);
          av[i4 * 4 + 0] = v.x;
          av[i4 * 4 + 1] = v.y;
          av[i4 * 4 + 2] = v.z;
          av[i4 * 4 + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < TM; ++i) av[i] = As[slot][k][ty * TM + i];
      }
      if constexpr (Cfg::SPLIT_N) {
#pragma unroll
        for (int j4 = 0; j4 < TN / 4; ++j4) {
          const float4 v = *reinterpret_cast<const float4 *>(&Bs[slot][k][j4 * (BN / (TN / 4)) + tx * 4]);
          bv[j4 * 4 + 0] = v.x;
          bv[j4 * 4 + 1] = v.y;
          bv[j4 * 4 + 2] = v.z;
          bv[j4 * 4 + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < TN; ++j) bv[j] = Bs[slot][k][tx * TN + j];
      }
    };
    load(0, a[0], b[0]);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      if (k + 1 < BK) load(k + 1, a[(k + 1) & 1], b[(k + 1) & 1]);
      micro_fma<TM, TN>(acc, a[k & 1], b[k & 1]);
    }
  };

  const int ktiles = (K + BK - 1) / BK;
  if constexpr (S == 1) {
    // One slot (tiles whose two stages pass 48 KB): copy, wait, compute, and a barrier before the next copy.
    for (int kt = 0; kt < ktiles; ++kt) {
      issue(kt, 0);
      cp_async_wait<0>();
      __syncthreads();
      compute(0);
      __syncthreads();
    }
  } else {
    // Prologue: k steps 0 .. S-2 in flight (empty groups past the end keep the group count uniform).
#pragma unroll
    for (int s = 0; s < S - 1; ++s) {
      if (s < ktiles)
        issue(s, s);
      else
        cp_async_commit();
    }
    for (int kt = 0; kt < ktiles; ++kt) {
      cp_async_wait<S - 2>();  // this thread's copies of step kt landed
      __syncthreads();         // everyone's did, and everyone finished step kt-1 (its slot is free again)
      const int next = kt + S - 1;
      if (next < ktiles)
        issue(next, next % S);
      else
        cp_async_commit();
      compute(kt % S);
    }
    cp_async_wait<0>();
  }

  // Fused epilogue: bias + GELU in registers, straight to C.
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int r = row0 + micro_index<BM, TM, Cfg::SPLIT_M>(ty, i);
    if (r >= M) continue;
    if constexpr (Cfg::SPLIT_N && VEC) {
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
    } else {
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int c = col0 + micro_index<BN, TN, Cfg::SPLIT_N>(tx, j);
        if (c < N) C[static_cast<size_t>(r) * N + c] = gelu_tanh_ref_f32(acc[i][j] + bias[c]);
      }
    }
  }
}

template <int BM, int BN, int BK, int TM, int TN, int PAD, bool VEC>
__global__ void __launch_bounds__(SimtConfig<BM, BN, BK, TM, TN, PAD>::THREADS,
                                  SimtConfig<BM, BN, BK, TM, TN, PAD>::MIN_BLOCKS)
    gemm_bias_gelu_simt(const float *__restrict__ A, const float *__restrict__ B, const float *__restrict__ bias,
                        float *__restrict__ C, int M, int N, int K) {
  gemm_bias_gelu_simt_body<BM, BN, BK, TM, TN, PAD, VEC>(A, B, bias, C, M, N, K);
}

}  // namespace pf
