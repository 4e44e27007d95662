// gemm_tf32x3.cuh -- the fp32 fused GEMM + bias + GELU on the tensor cores: 3xTF32 on CTA pairs.
//
// The reference kernel is fp32 FFMA (kernels/gemm_bias_gelu.cu:42-98).  This kernel keeps fp32 inputs
// and an fp32 result but does the contraction on the TF32 tensor cores with the split-precision
// ("3xTF32") method (Ootomo & Yokota, "Recovering single precision accuracy from Tensor Cores while
// surpassing the FP32 theoretical peak performance", IJHPCA 2022; CUTLASS's tfloat32x3 GEMMs):
// every element is split in shared memory into
//     hi = x with its 13 low mantissa bits cleared   (exactly a TF32 value)
//     lo = x - hi                                     (exact in fp32, |lo| < 2^-10 |x|)
// and a*b is accumulated as lo_a*hi_b + hi_a*lo_b + hi_a*hi_b (tcgen05.mma kind::tf32, fp32 in TMEM).
// The dropped lo_a*lo_b term is below 2^-20 |a*b| and the TF32 reading of lo loses at most 2^-21 |x|,
// so each product is good to ~2^-19 relative -- inside the fp32 path's 1e-5 tolerance.  The epilogue's
// GELU is the reference's function evaluated through 1 + tanh(u) = 2 / (1 + e^-2u) (see gelu_tanh_exp).
//
// CTA pairs (cluster of 2, tcgen05 .cta_group::2, M = 256, N = 256), persistent, 448 threads per CTA, and
// two shared-memory rings per CTA:
//   raw ring   (RAW_STAGES x 32 KB): what TMA brings in -- A rows [m0 + 128*rank, +128) K-major and B
//              columns [n0 + 128*rank, +128) N-major, one 32-k block each;
//   split ring (SPLIT_STAGES x 64 KB): the MMA operands -- A hi | A lo | B^T hi | B^T lo, all K-major.
// Roles:
//   warp 0      TMA producer (both CTAs): fills the raw ring, counted on its own `raw_full` barrier (no
//               multicast), as soon as the split warps have taken a slot's data into registers;
//   warps 6-13  split (both CTAs): raw slot -> registers (A 16-byte runs; B in 4 x 4 blocks) -> release the
//               raw slot -> hi / lo -> split slot, B written back transposed (K-major); fence to the async
//               proxy; arrive on the leader's `ready` barrier (8 warps x 2 CTAs).  B must be transposed:
//               with an MN-major B operand kind::tf32 MMAs contributed nothing on this B200 (measured),
//               K-major operands on both sides are exact;
//   warp 1      leader lane: waits `ready`, issues the three MMAs per 8-k step, commits the split slot free
//               (multicast to both CTAs) and the finished accumulator to both epilogues;
//   warps 2-5   epilogue (both CTAs): tcgen05.ld 32 columns at a time, + bias[c], GELU, fp32 through a
//               128-byte-swizzled 32 x 32 box and a TMA store; the accumulator (double-buffered, 2 x 256
//               TMEM columns) goes back to the MMA lane right after its last load.
// Separate rings let TMA run ahead of the MMAs (a raw slot is free once split, not once multiplied) and
// let the split write without waiting for its own reads of the slot to finish elsewhere in the block.
// Work units are those of the CTA-pair kernel (sk_unit, gemm_tc2.cuh): whole tiles, then, with a stream-K
// tail, contiguous k ranges of the last tiles spread over every pair; a tail tile's head pair adds the other
// pairs' fp32 partial sums in its epilogue.  k always ascends inside a unit.
// Periodic promotion (p.promote_kb > 0): the tensor cores accumulate fp32 with truncation (round toward zero),
// so a long k range drifts toward zero -- by about 6.4e-9 x K relative on U(-0.5, 0.5) inputs, past 1e-5 from
// K ~ 2048.  A unit's k range is therefore cut into chunks of promote_kb k-blocks that alternate between the two
// TMEM accumulators; when a chunk is done the epilogue adds it, round to nearest, into this CTA's fp32 running
// sum in p.promote_ws (L2-resident, each lane reading back only what it wrote), while the MMAs fill the other
// accumulator; the last chunk is added to the running sum in the final epilogue.  The truncation then spans
// one chunk, and the drift falls to roughly 6.4e-9 x sqrt(K x 32 promote_kb).
#pragma once

#include "gemm_tc2.cuh"

namespace pf {

template <int kRawStages, int kSplitStages>
struct Tf32x3Config {
  static constexpr int BM = 256;                             // pair tile rows
  static constexpr int BM_CTA = 128;
  static constexpr int BN = 256;                             // pair tile columns (UMMA N)
  static constexpr int BN_CTA = 128;                         // B columns loaded by each CTA
  static constexpr int RAW_STAGES = kRawStages;
  static constexpr int SPLIT_STAGES = kSplitStages;
  static constexpr int STAGES = kRawStages + kSplitStages;   // pipeline depth reported to the host
  static constexpr int ELEM = 4;
  static constexpr int ATOM_K = 32;                          // fp32 elements in one 128-byte row
  static constexpr int BK = ATOM_K;                          // k per stage
  static constexpr int UMMA_K = 8;                           // k per kind::tf32 MMA (32 bytes)
  static constexpr int A_BYTES = BM_CTA * 128;               // 128 rows x 128 B
  static constexpr int B_CHUNK_N = 32;                       // N elements per 128-byte row of B
  static constexpr int B_CHUNKS = BN_CTA / B_CHUNK_N;
  static constexpr int B_CHUNK_BYTES = BK * 128;
  static constexpr int B_BYTES = B_CHUNKS * B_CHUNK_BYTES;   // = BN_CTA rows x 128 B once transposed
  static constexpr int RAW_BYTES = A_BYTES + B_BYTES;        // one raw slot
  static constexpr int SPLIT_BYTES = 2 * RAW_BYTES;          // one split slot: A hi, A lo, B^T hi, B^T lo
  static constexpr int EPI_WARPS = 4;
  static constexpr int SPLIT_WARPS = 8;
  static constexpr int EPI_COLS = 32;                        // fp32 columns per TMA store box (128 B)
  static constexpr int EPI_BUF_BYTES = 32 * EPI_COLS * 4;    // 32 rows x 128 B
  static constexpr int EPI_BUFS = 2;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUFS * EPI_BUF_BYTES;
  static constexpr int NUM_BARS = 2 * RAW_STAGES + 2 * SPLIT_STAGES + 4 + 1 + 1;
  static constexpr int PARTIAL_FLOATS = BM_CTA * BN;         // one CTA's share of a tile, fp32
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM_BYTES =
      1024 + SPLIT_STAGES * SPLIT_BYTES + RAW_STAGES * RAW_BYTES + EPI_BYTES + NUM_BARS * 8 + 16;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS + SPLIT_WARPS);
  static constexpr uint32_t IDESC = instr_desc(2u, 2u, /*A K-major*/ 0u, /*B K-major*/ 0u, 256, 256);
  static_assert(SMEM_BYTES <= 232448, "shared memory per block exceeds the sm_100 opt-in limit");
};

enum : unsigned { kErrSplitWait = 16u };

// The reference's GELU, 0.5*x*(1 + tanh(u)) with u = k0*(x + k1*x^3) (kernels/gemm_bias_gelu.cu:37-40),
// rewritten with 1 + tanh(u) = 2 / (1 + e^-2u) as x / (1 + e^-2u).  __expf and __fdividef (the hardware
// exponential and reciprocal) keep it within ~1e-6 relative of the fp64 function over the whole range
// (e^-2u overflowing to +inf for very negative x gives the right limit, -0), inside the fp32 path's 1e-5
// and far cheaper than tanhf in an epilogue that a single-tile-per-pair launch cannot hide.
__device__ __forceinline__ float gelu_tanh_exp(float x) {
  const float k0 = 0.7978845608028654f, k0k1 = 0.7978845608028654f * 0.044715f;
  const float u = x * fmaf(k0k1, x * x, k0);
  return __fdividef(x, 1.0f + __expf(-2.0f * u));
}

__device__ __forceinline__ void ld_shared_v4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

// hi (TF32: low 13 mantissa bits cleared) and lo = x - hi of four fp32 words, stored at hi_addr / lo_addr.
__device__ __forceinline__ void store_split4(uint32_t hi_addr, uint32_t lo_addr, uint32_t x0, uint32_t x1, uint32_t x2,
                                             uint32_t x3) {
  const uint32_t h0 = x0 & 0xFFFFE000u, h1 = x1 & 0xFFFFE000u, h2 = x2 & 0xFFFFE000u, h3 = x3 & 0xFFFFE000u;
  st_shared_v4(hi_addr, h0, h1, h2, h3);
  st_shared_v4(lo_addr, __float_as_uint(__uint_as_float(x0) - __uint_as_float(h0)),
               __float_as_uint(__uint_as_float(x1) - __uint_as_float(h1)),
               __float_as_uint(__uint_as_float(x2) - __uint_as_float(h2)),
               __float_as_uint(__uint_as_float(x3) - __uint_as_float(h3)));
}

// The running sum's 32 values of this lane's row for one 32-column piece: src[j4 * 32], j4 = 0..7 (float4 each;
// the partial-slot layout).
__device__ __forceinline__ void load_running_sum(float4 (&s)[8], const float4 *src) {
#pragma unroll
  for (int j4 = 0; j4 < 8; ++j4) s[j4] = __ldcg(src + j4 * 32);
}

// v[0..31] (fp32 bits of 32 accumulator columns) += s, rounding to nearest.
__device__ __forceinline__ void add_running_sum(uint32_t (&v)[32], const float4 (&s)[8]) {
#pragma unroll
  for (int j4 = 0; j4 < 8; ++j4) {
    v[j4 * 4 + 0] = __float_as_uint(s[j4].x + __uint_as_float(v[j4 * 4 + 0]));
    v[j4 * 4 + 1] = __float_as_uint(s[j4].y + __uint_as_float(v[j4 * 4 + 1]));
    v[j4 * 4 + 2] = __float_as_uint(s[j4].z + __uint_as_float(v[j4 * 4 + 2]));
    v[j4 * 4 + 3] = __float_as_uint(s[j4].w + __uint_as_float(v[j4 * 4 + 3]));
  }
}

template <class Cfg>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg::THREADS, 1)
    gemm_bias_gelu_tf32x3(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

  // split slot s: [A hi | A lo | B^T hi | B^T lo] (16 KB each); raw slot r: [A | B]; all 1024-byte aligned
  uint8_t *sSplit = smem;
  uint8_t *sRaw = smem + Cfg::SPLIT_STAGES * Cfg::SPLIT_BYTES;
  uint8_t *sEpi = sRaw + Cfg::RAW_STAGES * Cfg::RAW_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sEpi + Cfg::EPI_BYTES);
  uint64_t *raw_full = bars;                              // [RAW] own: TMA bytes landed
  uint64_t *raw_empty = raw_full + Cfg::RAW_STAGES;       // [RAW] own: the split warps took the data
  uint64_t *ready = raw_empty + Cfg::RAW_STAGES;          // [SPLIT] leader: both CTAs' split slot written
  uint64_t *split_empty = ready + Cfg::SPLIT_STAGES;      // [SPLIT] both: the MMAs reading the slot finished
  uint64_t *tfull = split_empty + Cfg::SPLIT_STAGES;      // [2] both: accumulator ready
  uint64_t *tempty = tfull + 2;                           // [2] leader: both CTAs drained the accumulator
  uint64_t *drain = tempty + 2;                           // [1] leader: all MMAs complete
  uint64_t *epi_sync = drain + 1;                         // [1] the 4 epilogue warps wrote this worker's partial
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(epi_sync + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();      // 0 = leader, 1 = follower
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    for (int r = 0; r < Cfg::RAW_STAGES; ++r) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], Cfg::SPLIT_WARPS);
    }
    for (int s = 0; s < Cfg::SPLIT_STAGES; ++s) {
      mbar_init(&ready[s], 2 * Cfg::SPLIT_WARPS);
      mbar_init(&split_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * Cfg::EPI_WARPS);
    }
    mbar_init(drain, 1);
    mbar_init(epi_sync, Cfg::EPI_WARPS);        // completes at most once: a worker has at most one partial
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
    tc_fence_before();
  }
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // Under a programmatic launch the set-up above overlapped the previous kernel's tail.  The roles that touch
  // global memory wait for that kernel to be done (griddepcontrol.wait) before their first access: the producer
  // before its first load (its first unit's coordinates are worked out before), the epilogue on entry.  The split
  // warps and the MMA issuer touch only shared memory and TMEM.

  auto fail = [&](unsigned bit) {
    atomicOr(p.status, bit);
    *abort_flag = 1;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      int slot = 0;
      uint32_t phase = 0;
      bool ok = true;
      int issued = 0;
      SkUnit un;
    int umb, unb;  // the unit's tile (this kernel reads it through tile_coords)
      for (int u = 0; ok && sk_unit(pair, num_pairs, u, p, un, umb, unb); ++u) {
        int mb, nb;
        tile_coords(un.tile, p, mb, nb);
        const int m0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::BM_CTA;
        const int n0 = nb * Cfg::BN + static_cast<int>(rank) * Cfg::BN_CTA;
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait(&raw_empty[slot], phase ^ 1u, p.timeout_ns, abort_flag)) {
            fail(kErrProducerWait);
            ok = false;
            break;
          }
          uint8_t *dst = sRaw + slot * Cfg::RAW_BYTES;
          mbar_arrive_expect_tx(&raw_full[slot], Cfg::RAW_BYTES);
          if (issued == 0) grid_dependency_wait();
          tma_load_2d(dst, &tmA, &raw_full[slot], kb * Cfg::BK, m0);
#pragma unroll
          for (int j = 0; j < Cfg::B_CHUNKS; ++j)
            tma_load_2d(dst + Cfg::A_BYTES + j * Cfg::B_CHUNK_BYTES, &tmB, &raw_full[slot], n0 + j * Cfg::B_CHUNK_N,
                        kb * Cfg::BK);
          ++issued;
          if (++slot == Cfg::RAW_STAGES) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Loads already issued land before the block may exit (bounded).
        for (int r = 0; r < Cfg::RAW_STAGES && r < issued; ++r) {
          const uint32_t ph = (r < slot) ? phase : (phase ^ 1u);
          volatile int no_abort = 0;
          if (!mbar_wait(&raw_full[r], ph, p.timeout_ns, &no_abort)) atomicOr(p.status, kErrTeardownWait);
        }
      }
    }
    grid_launch_dependents();  // this CTA's loads are all issued
  } else if (warp >= 2 + Cfg::EPI_WARPS) {
    // ---------------------------------------------------------------- split hi / lo (warps 6..13)
    grid_launch_dependents();  // a dependent launch waits for the producer and MMA warps, which signal last
    constexpr int SPLIT_THREADS = 32 * Cfg::SPLIT_WARPS;
    constexpr int A_VEC = Cfg::A_BYTES / 16 / SPLIT_THREADS;   // 16-byte runs of A per thread
    constexpr int BLOCKS = 256 / SPLIT_THREADS;                // 4 x 4 blocks of B per thread
    static_assert(A_VEC * SPLIT_THREADS * 16 == Cfg::A_BYTES && BLOCKS * SPLIT_THREADS == 256,
                  "split threads must divide the A runs and the 256 transpose blocks");
    const int tid = threadIdx.x - 32 * (2 + Cfg::EPI_WARPS);
    const uint32_t ready_leader0 = mapa_shared(smem_u32(&ready[0]), 0);
    // B transpose: block beta -> k-block a = x ^ c, n-block b = 8m + x (c = beta / 32, m = beta / 8 % 4,
    // x = beta % 8): in every quarter-warp the eight 16-byte reads (N-major rows) and the eight 16-byte
    // writes (K-major rows) hit eight distinct bank groups of the 128-byte swizzle.
    int blk_k[BLOCKS], blk_n[BLOCKS];
#pragma unroll
    for (int it = 0; it < BLOCKS; ++it) {
      const int beta = it * SPLIT_THREADS + tid;
      const int x = beta & 7;
      blk_k[it] = 4 * (x ^ (beta >> 5));
      blk_n[it] = 4 * (8 * ((beta >> 3) & 3) + x);
    }
    int rslot = 0, sslot = 0;
    uint32_t rphase = 0, sphase = 0;
    bool ok = true;
    SkUnit un;
    int umb, unb;  // the unit's tile (this kernel reads it through tile_coords)
    for (int u = 0; ok && sk_unit(pair, num_pairs, u, p, un, umb, unb); ++u) {
      for (int kb = un.kb0; kb < un.kb1; ++kb) {
        // 1. the raw slot's bytes, into registers
        bool waited = mbar_wait(&raw_full[rslot], rphase, p.timeout_ns, abort_flag);
        if (!__all_sync(0xffffffffu, waited)) {
          if (lane == 0) fail(kErrSplitWait);
          ok = false;
          break;
        }
        const uint32_t ra = smem_u32(sRaw + rslot * Cfg::RAW_BYTES), rb = ra + Cfg::A_BYTES;
        uint32_t a[A_VEC][4];
#pragma unroll
        for (int i = 0; i < A_VEC; ++i) ld_shared_v4(ra + (tid + i * SPLIT_THREADS) * 16, a[i]);
        uint32_t v[BLOCKS][4][4];  // N-major: chunk n/32, row k, 16-byte group (n%32/4) ^ (k%8)
#pragma unroll
        for (int it = 0; it < BLOCKS; ++it)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int k = blk_k[it] + i, n = blk_n[it];
            ld_shared_v4(rb + (n >> 5) * Cfg::B_CHUNK_BYTES + k * 128 + ((((n & 31) >> 2) ^ (k & 7)) << 4), v[it][i]);
          }
        // 2. the raw slot goes back to the producer once every lane of the warp holds its data
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rslot]);
        if (++rslot == Cfg::RAW_STAGES) {
          rslot = 0;
          rphase ^= 1u;
        }
        // 3. hi / lo into the split slot, once the MMAs have released it
        waited = mbar_wait(&split_empty[sslot], sphase ^ 1u, p.timeout_ns, abort_flag);
        if (!__all_sync(0xffffffffu, waited)) {
          if (lane == 0) fail(kErrSplitWait);
          ok = false;
          break;
        }
        const uint32_t s0 = smem_u32(sSplit + sslot * Cfg::SPLIT_BYTES);
        const uint32_t a_hi = s0, a_lo = s0 + Cfg::A_BYTES, b_hi = s0 + 2 * Cfg::A_BYTES,
                       b_lo = b_hi + Cfg::B_BYTES;
#pragma unroll
        for (int i = 0; i < A_VEC; ++i) {
          const uint32_t off = (tid + i * SPLIT_THREADS) * 16;
          store_split4(a_hi + off, a_lo + off, a[i][0], a[i][1], a[i][2], a[i][3]);
        }
        // B^T: K-major rows n of 32 k, 16-byte group (k/4) ^ (n%8)
#pragma unroll
        for (int it = 0; it < BLOCKS; ++it)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int n = blk_n[it] + j;
            const uint32_t off = n * 128 + (((blk_k[it] >> 2) ^ (n & 7)) << 4);
            store_split4(b_hi + off, b_lo + off, v[it][0][j], v[it][1][j], v[it][2][j], v[it][3][j]);
          }
        // The tensor cores read shared memory through the async proxy.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(ready_leader0 + sslot * 8);
        if (++sslot == Cfg::SPLIT_STAGES) {
          sslot = 0;
          sphase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader only)
    if (lane == 0 && rank == 0) {
      int sslot = 0;
      uint32_t sphase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      SkUnit un;
    int umb, unb;  // the unit's tile (this kernel reads it through tile_coords)
      for (int u = 0; ok && sk_unit(pair, num_pairs, u, p, un, umb, unb); ++u) {
        const int steps = un.kb1 - un.kb0;
        const int G = (p.promote_kb > 0 && p.promote_ws != nullptr) ? p.promote_kb : (steps > 0 ? steps : 1);
        // chunk [c0, c1) of the unit's k steps, into accumulator `acc` (the epilogue counts the same chunks)
        for (int c0 = 0; ok && (c0 < steps || c0 == 0); c0 += G) {
          const int c1 = min(c0 + G, steps);
          if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, p.timeout_ns, abort_flag)) {
            fail(kErrMmaWait);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::BN);
          for (int i = c0; i < c1; ++i) {
            if (!mbar_wait_cluster(&ready[sslot], sphase, p.timeout_ns, abort_flag)) {
              fail(kErrMmaWait);
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_hi = smem_u32(sSplit + sslot * Cfg::SPLIT_BYTES), a_lo = a_hi + Cfg::A_BYTES;
            const uint32_t b_hi = a_hi + 2 * Cfg::A_BYTES, b_lo = b_hi + Cfg::B_BYTES;
#pragma unroll
            for (int k = 0; k < Cfg::BK / Cfg::UMMA_K; ++k) {
              // A and B^T: K-major 128-byte swizzled rows; k advances 32 bytes inside the row.
              const uint64_t ah = smem_desc(a_hi + k * 32, 16, 1024, kSwizzle128B);
              const uint64_t al = smem_desc(a_lo + k * 32, 16, 1024, kSwizzle128B);
              const uint64_t bh = smem_desc(b_hi + k * 32, 16, 1024, kSwizzle128B);
              const uint64_t bl = smem_desc(b_lo + k * 32, 16, 1024, kSwizzle128B);
              // small terms first
              tc_mma_tf32_pair(d_tmem, al, bh, Cfg::IDESC, ((i - c0) | k) != 0 ? 1u : 0u);
              tc_mma_tf32_pair(d_tmem, ah, bl, Cfg::IDESC, 1u);
              tc_mma_tf32_pair(d_tmem, ah, bh, Cfg::IDESC, 1u);
            }
            tc_commit_pair_mc(&split_empty[sslot], 0x3);
            if (++sslot == Cfg::SPLIT_STAGES) {
              sslot = 0;
              sphase ^= 1u;
            }
          }
          if (!ok) break;
          tc_commit_pair_mc(&tfull[acc], 0x3);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
      }
      tc_commit_pair(drain);
      volatile int no_abort = 0;
      if (!mbar_wait(drain, 0, p.timeout_ns, &no_abort)) atomicOr(p.status, kErrTeardownWait);
    }
    grid_launch_dependents();  // this CTA's MMAs are all issued (and, on the leader, complete)
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5, both CTAs)
    grid_launch_dependents();
    grid_dependency_wait();
    const int q = warp & 3;
    const int ew = warp - 2;
    uint8_t *ebuf = sEpi + ew * Cfg::EPI_BUFS * Cfg::EPI_BUF_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    int buf = 0;
    SkUnit un;
    int umb, unb;  // the unit's tile (this kernel reads it through tile_coords)
    // This CTA's partial-sum slot (its 128 rows of a tile) in worker `w`'s workspace; a warp's 32 rows are
    // stored quad-of-columns-major so one warp-wide 16-byte access covers 512 contiguous bytes.
    auto slot = [&](int w) -> float4 * {
      return reinterpret_cast<float4 *>(p.sk_partials + (static_cast<size_t>(w) * 2 + rank) * Cfg::PARTIAL_FLOATS +
                                        static_cast<size_t>(q) * 32 * Cfg::BN);
    };
    // This CTA's running sum of a unit's finished chunks (periodic promotion), laid out as the partial slots.
    float4 *const run = p.promote_ws == nullptr
                            ? nullptr
                            : reinterpret_cast<float4 *>(p.promote_ws +
                                                         (static_cast<size_t>(pair) * 2 + rank) * Cfg::PARTIAL_FLOATS +
                                                         static_cast<size_t>(q) * 32 * Cfg::BN);
    bool stop = false;
    for (int u = 0; !stop && sk_unit(pair, num_pairs, u, p, un, umb, unb); ++u) {
      int mb, nb;
      tile_coords(un.tile, p, mb, nb);
      const int steps = un.kb1 - un.kb0;
      const int G = (p.promote_kb > 0 && p.promote_ws != nullptr) ? p.promote_kb : (steps > 0 ? steps : 1);
      const int chunks = steps > G ? (steps + G - 1) / G : 1;
      // Every chunk but the last: add it, round to nearest, into the running sum and hand the accumulator back.
      for (int ch = 0; ch + 1 < chunks; ++ch) {
        const bool waited = mbar_wait(&tfull[acc], acc_phase, p.timeout_ns, abort_flag);
        if (!__all_sync(0xffffffffu, waited)) {
          if (lane == 0) fail(kErrEpilogueWait);
          stop = true;
          break;
        }
        tc_fence_after();
        const uint32_t t_acc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * Cfg::BN);
        const uint32_t tempty_acc = mapa_shared(smem_u32(&tempty[acc]), 0);
        // 32 columns at a time; the piece's running sum is read from L2 while its TMEM load is in flight.
#pragma unroll 1
        for (int c = 0; c < Cfg::BN / 32; ++c) {
          float4 s_cur[8];
          if (ch > 0) load_running_sum(s_cur, run + c * 8 * 32 + lane);
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_acc + c * 32, v);
          tmem_ld_wait();
          if (c == Cfg::BN / 32 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_acc);
          }
          if (ch > 0) add_running_sum(v, s_cur);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            __stcg(run + (c * 8 + j4) * 32 + lane,
                   make_float4(__uint_as_float(v[j4 * 4 + 0]), __uint_as_float(v[j4 * 4 + 1]),
                               __uint_as_float(v[j4 * 4 + 2]), __uint_as_float(v[j4 * 4 + 3])));
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (stop) break;
      const bool waited = mbar_wait(&tfull[acc], acc_phase, p.timeout_ns, abort_flag);
      if (!__all_sync(0xffffffffu, waited)) {
        if (lane == 0) fail(kErrEpilogueWait);
        break;
      }
      tc_fence_after();
      const int m0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::BM_CTA + q * 32;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * Cfg::BN);
      const uint32_t tempty_leader = mapa_shared(smem_u32(&tempty[acc]), 0);
      if (un.kind == kUnitPartial) {
        // Write this worker's fp32 partial (its k range of the tile) and raise its flag.
        float4 *dst = slot(pair);
#pragma unroll 1
        for (int c = 0; c < Cfg::BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + c * 32, v);
          tmem_ld_wait();
          if (chunks > 1) {
            float4 s4[8];
            load_running_sum(s4, run + c * 8 * 32 + lane);
            add_running_sum(v, s4);
          }
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            __stcg(dst + (c * 8 + j4) * 32 + lane,
                   make_float4(__uint_as_float(v[j4 * 4 + 0]), __uint_as_float(v[j4 * 4 + 1]),
                               __uint_as_float(v[j4 * 4 + 2]), __uint_as_float(v[j4 * 4 + 3])));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader);
        // Every warp's stores are visible device-wide before it arrives; one lane publishes the flag once all
        // four have arrived (bounded wait, never a hardware barrier a departed warp could block).
        __threadfence();
        __syncwarp();
        if (lane == 0) mbar_arrive(epi_sync);
        if (warp == 2 && lane == 0) {
          if (mbar_wait(epi_sync, 0, p.timeout_ns, abort_flag))
            st_release_gpu(p.sk_flags + pair * 2 + rank, p.epoch);
          else
            fail(kErrEpilogueWait);
        }
      } else {
        // Whole tile, or the head of a tail tile: add the later workers' partials (bounded waits).
        int first = 0, last = -1;
        if (un.kind == kUnitHead) {
          const long long tile_end = static_cast<long long>(un.tile - p.dp_tiles + 1) * p.k_blocks;
          first = pair + 1;
          last = pair;
          while (last + 1 < num_pairs && sk_start(last + 1, num_pairs, p) < tile_end) ++last;
          bool ok = true;
          if (lane == 0) {
            for (int w = first; w <= last && ok; ++w) {
              const unsigned *flag = p.sk_flags + w * 2 + rank;
              if (ld_acquire_gpu(flag) != p.epoch) {
                const uint64_t t0 = globaltimer_ns();
                while (ld_acquire_gpu(flag) != p.epoch) {
                  if (*abort_flag || globaltimer_ns() - t0 > p.timeout_ns) {
                    ok = false;
                    break;
                  }
                  __nanosleep(256);
                }
              }
            }
            if (!ok) fail(kErrEpilogueWait);
          }
          if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
        }
#pragma unroll 1
        for (int c = 0; c < Cfg::BN / Cfg::EPI_COLS; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + c * Cfg::EPI_COLS, v);
          tmem_ld_wait();
          if (chunks > 1) {
            float4 s4[8];
            load_running_sum(s4, run + c * 8 * 32 + lane);
            add_running_sum(v, s4);
          }
          if (c == Cfg::BN / Cfg::EPI_COLS - 1) {
            // Last TMEM read of this accumulator: hand it back to the MMA issuer.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader);
          }
          for (int w = first; w <= last; ++w) {
            const float4 *src = slot(w) + c * 8 * 32 + lane;
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 s4 = __ldcg(src + j4 * 32);
              v[j4 * 4 + 0] = __float_as_uint(__uint_as_float(v[j4 * 4 + 0]) + s4.x);
              v[j4 * 4 + 1] = __float_as_uint(__uint_as_float(v[j4 * 4 + 1]) + s4.y);
              v[j4 * 4 + 2] = __float_as_uint(__uint_as_float(v[j4 * 4 + 2]) + s4.z);
              v[j4 * 4 + 3] = __float_as_uint(__uint_as_float(v[j4 * 4 + 3]) + s4.w);
            }
          }
          const int n0 = nb * Cfg::BN + c * Cfg::EPI_COLS;
          const uint32_t sbuf = smem_u32(ebuf + buf * Cfg::EPI_BUF_BYTES) + lane * 128;
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (n0 + j4 * 4 < p.N) b4 = __ldg(reinterpret_cast<const float4 *>(p.bias + n0 + j4 * 4));
            const float y0 = gelu_tanh_exp(__uint_as_float(v[j4 * 4 + 0]) + b4.x);
            const float y1 = gelu_tanh_exp(__uint_as_float(v[j4 * 4 + 1]) + b4.y);
            const float y2 = gelu_tanh_exp(__uint_as_float(v[j4 * 4 + 2]) + b4.z);
            const float y3 = gelu_tanh_exp(__uint_as_float(v[j4 * 4 + 3]) + b4.w);
            // row `lane` of the 32 x 32 fp32 box: 16-byte chunk j4 goes to chunk j4 ^ (row % 8)
            st_shared_v4(sbuf + static_cast<uint32_t>((j4 ^ (lane & 7)) * 16), __float_as_uint(y0),
                         __float_as_uint(y1), __float_as_uint(y2), __float_as_uint(y3));
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, ebuf + buf * Cfg::EPI_BUF_BYTES, n0, m0);
            tma_store_commit();
            tma_store_wait_read<1>();
          }
          __syncwarp();
          buf ^= 1;
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) tma_store_wait_all<0>();
    __syncwarp();
  }

  __syncwarp();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace pf
