// gemm_tc2.cuh -- the fused GEMM + bias + GELU on CTA pairs (tcgen05 .cta_group::2), 256 x 256 tiles.
//
// Same roles and math as gemm_tc.cuh, but two CTAs on two SMs (a cluster of 2) cooperate on each
// 256 x 256 output tile:
//   * each CTA TMA-loads its own operand halves -- A rows [m0 + 128*rank, +128) and B columns
//     [n0 + 128*rank, +128) -- into its own shared memory (no multicast); the loads of both CTAs
//     are counted on the even (leader) CTA's `full` barrier;
//   * the leader's MMA lane issues tcgen05.mma.cta_group::2 with M = 256, N = 256: the tensor cores
//     of both SMs read A from their own SM and B from both, and each SM's TMEM receives its 128
//     accumulator rows x 256 columns;
//   * tcgen05.commit multicasts the stage-free and accumulator-ready signals to both CTAs;
//   * each CTA's four epilogue warps drain its own TMEM rows and signal the leader's `tempty`.
// Per SM this halves the shared-memory B traffic of the 1-CTA 128 x 256 kernel; at 32 KB per k-atom
// and stage, 3 stages of two k-atoms (or 6 of one) fit.
//
// Work units.  A pair ("worker") walks a list of units that all three roles enumerate identically
// (sk_unit): first whole tiles, round-robin over the workers (data-parallel), then, when the launch
// enables the stream-K tail (p.sk_iters > 0), a contiguous share of the k-iterations of the last
// tiles, so a partial last wave does not leave SMs idle.  Or, with p.sk_band_workers = P > 0 (row-band
// stream-K), each row block of tiles is a band of P workers, each taking an equal contiguous share of the
// band's k-iterations (band_unit); workers at the same position of different bands then read the same
// B panel at the same k at the same time, so B comes from DRAM once for all bands.  A tail tile is split between consecutive
// workers: the one holding the tile's first k-block ("head") finishes it; the others ("partials")
// write their fp32 accumulators to a workspace and raise a flag tagged with the launch's epoch; the
// head adds them in its epilogue.  A worker's partial is its first tail unit and its head its last,
// so heads rarely wait; every wait is bounded.
#pragma once

#include "gemm_tc.cuh"

namespace pf {

// kBN: pair tile columns (UMMA N), 256 or 224.  A 224-wide tile gives 37 column tiles for N = 8192, so
// row shards whose 256-wide tiles would leave a partial last wave fill whole waves of pairs instead.
template <int kDtype, int kStages, int kKAtoms = 1, int kBN = 256>
struct Tc2Config {
  static constexpr int BM = 256;                             // pair tile rows
  static constexpr int BM_CTA = 128;
  static constexpr int BN = kBN;                             // pair tile columns (UMMA N)
  static constexpr int BN_CTA = kBN / 2;                     // B columns each CTA supplies to the MMA
  static constexpr int STAGES = kStages;
  static constexpr int ELEM = (kDtype == 0) ? 2 : 1;
  static constexpr int KATOMS = kKAtoms;                     // 128-byte k-atoms per stage
  static constexpr int ATOM_K = 128 / ELEM;
  static constexpr int BK = KATOMS * ATOM_K;
  static constexpr int UMMA_K = 32 / ELEM;
  static constexpr int A_ATOM_BYTES = BM_CTA * 128;
  static constexpr int A_BYTES = KATOMS * A_ATOM_BYTES;
  static constexpr int B_CHUNK_N = 128 / ELEM;
  static constexpr int B_CHUNKS = (BN_CTA + B_CHUNK_N - 1) / B_CHUNK_N;  // boxes loaded (the last may overhang)
  static constexpr int B_CHUNK_BYTES = BK * 128;
  static constexpr int B_BYTES = B_CHUNKS * B_CHUNK_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;      // per CTA
  static constexpr int EPI_WARPS = 4;
  static constexpr int EPI_BUF_BYTES = 32 * 64 * 2;
  static constexpr int EPI_BUFS = 2;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUFS * EPI_BUF_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 4 + 1 + 1;
  static constexpr int TMEM_COLS = 512;                      // 2 accumulators, 256 columns apart
  static constexpr int ACC_STRIDE = 256;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + NUM_BARS * 8 + 16;
  static constexpr int THREADS = 192;
  static constexpr int PARTIAL_FLOATS = BM_CTA * BN;         // one CTA's share of a tile, fp32
  static constexpr uint32_t IDESC =
      instr_desc(kDtype == 0 ? 1u : 0u, kDtype == 0 ? 1u : 0u, 0u, 1u, /*M*/ 256, /*N*/ BN);
  static_assert(SMEM_BYTES <= 232448, "shared memory per block exceeds the sm_100 opt-in limit");
  static_assert(BN == 256 || BN == 224, "pair tiles are 256 or 224 columns wide");
};

enum : int { kUnitWhole = 0, kUnitHead = 1, kUnitPartial = 2 };

struct SkUnit {
  int tile;      // global tile index (tile_coords order); -1 in row-band mode
  int kb0, kb1;  // k-block range [kb0, kb1)
  int kind;      // kUnitWhole / kUnitHead / kUnitPartial
};

// First k-iteration of band position j (of P) in a band of S k-iterations, floor(j * S / P), in 32-bit
// arithmetic (S = q * P + r: j * q + j * r / P; the host keeps S * P below 2^31 in band mode).
__device__ __forceinline__ int band_start(int j, int P, int S) { return j * (S / P) + (j * (S % P)) / P; }

// Row-band stream-K (p.sk_band_workers = P > 0): worker w is position j = w % P of band (row block) g = w / P
// and takes the band's k-iterations [band_start(j), band_start(j + 1)) -- its tiles left to right, k ascending.
// Unit `u` of worker w, its tile (mb, nb); false past the worker's last unit.
__device__ __forceinline__ bool band_unit(int w, int u, const TcParams &p, SkUnit &out, int &mb, int &nb) {
  const int P = p.sk_band_workers;
  const int g = w / P, j = w % P;
  if (g >= p.num_m_blocks) return false;
  const int KB = p.k_blocks;
  const int S = p.num_n_blocks * KB;
  const int e = band_start(j + 1, P, S);
  int pos = band_start(j, P, S);
  for (int i = 0; pos < e; ++i) {
    const int t = pos / KB;
    const int seg_end = min(e, (t + 1) * KB);
    if (i == u) {
      mb = g;
      nb = t;
      out.tile = -1;
      out.kb0 = pos - t * KB;
      out.kb1 = seg_end - t * KB;
      out.kind = out.kb0 == 0 ? (out.kb1 == KB ? kUnitWhole : kUnitHead) : kUnitPartial;
      return true;
    }
    pos = seg_end;
  }
  return false;
}

// The last worker whose partial a band-mode head at tile column nb adds: the band positions j' > j whose share
// starts inside the tile, floor(j' S / P) < tile_end, i.e. j' < tile_end P / S.
__device__ __forceinline__ int band_last_contributor(int w, int nb, const TcParams &p) {
  const int P = p.sk_band_workers;
  const int j = w % P;
  const int S = p.num_n_blocks * p.k_blocks;
  const int tile_end = (nb + 1) * p.k_blocks;
  return w + min(P - 1, (tile_end * P + S - 1) / S - 1) - j;
}

// Folds the fp32 partials of `n_contrib` consecutive workers (slots `stride` float4 apart from `first`, this
// lane's column-major layout: float4 index (col / 4) * 32 + lane) into this warp's 32 TMEM lanes: PIECES runs
// of NCOLS columns, `piece_stride` apart from col_first, of the accumulator at t_row.  64 columns at a time:
// both 32-column TMEM loads and all 16 partial loads of the first contributor in flight together, added in
// worker order, stored back.
template <int NCOLS, int PIECES = 1>
__device__ __forceinline__ void fold_partials(uint32_t t_row, int col_first, int piece_stride, const float4 *first,
                                              size_t stride, int n_contrib) {
  static_assert(NCOLS % 64 == 0, "64-column steps");
#pragma unroll 1
  for (int c = 0; c < PIECES * (NCOLS / 64); ++c) {
    const int col = col_first + (c / (NCOLS / 64)) * piece_stride + (c % (NCOLS / 64)) * 64;
    uint32_t v[2][32];
    tmem_ld_32x32b_x32(t_row + col, v[0]);
    tmem_ld_32x32b_x32(t_row + col + 32, v[1]);
    const float4 *src = first + (col / 4) * 32;
#pragma unroll 1
    for (int w = 0; w < n_contrib; ++w, src += stride) {
      float4 s4[16];
#pragma unroll
      for (int j4 = 0; j4 < 16; ++j4) s4[j4] = __ldcg(src + j4 * 32);
      if (w == 0) tmem_ld_wait();
#pragma unroll
      for (int j4 = 0; j4 < 16; ++j4) {
        uint32_t *d = &v[j4 / 8][(j4 % 8) * 4];
        d[0] = __float_as_uint(__uint_as_float(d[0]) + s4[j4].x);
        d[1] = __float_as_uint(__uint_as_float(d[1]) + s4[j4].y);
        d[2] = __float_as_uint(__uint_as_float(d[2]) + s4[j4].z);
        d[3] = __float_as_uint(__uint_as_float(d[3]) + s4[j4].w);
      }
    }
    if (n_contrib <= 0) tmem_ld_wait();
    tmem_st_32x32b_x32(t_row + col, v[0]);
    tmem_st_32x32b_x32(t_row + col + 32, v[1]);
  }
  tmem_st_wait();  // the folded sums are in TMEM before anything reads them back
}

// Unit `u` of worker `w` of `W` and its tile (mb, nb); false past the worker's last unit.
__device__ __forceinline__ bool sk_unit(int w, int W, int u, const TcParams &p, SkUnit &out, int &mb, int &nb) {
  if (p.sk_band_workers > 0) return band_unit(w, u, p, out, mb, nb);
  const int dp = p.sk_iters > 0 ? p.dp_tiles : p.num_tiles;
  const int n_dp = w < dp ? (dp - 1 - w) / W + 1 : 0;
  if (u < n_dp) {
    out = {w + u * W, 0, p.k_blocks, kUnitWhole};
    tile_coords(out.tile, p, mb, nb);
    return true;
  }
  if (p.sk_iters <= 0) return false;
  u -= n_dp;
  const long long KB = p.k_blocks;
  const long long s = static_cast<long long>(w) * p.sk_iters / W;
  const long long e = static_cast<long long>(w + 1) * p.sk_iters / W;
  long long pos = s;
  for (int i = 0; pos < e; ++i) {
    const long long local = pos / KB;
    const long long seg_end = min(e, (local + 1) * KB);
    if (i == u) {
      out.tile = dp + static_cast<int>(local);
      out.kb0 = static_cast<int>(pos - local * KB);
      out.kb1 = static_cast<int>(seg_end - local * KB);
      out.kind = out.kb0 == 0 ? (out.kb1 == KB ? kUnitWhole : kUnitHead) : kUnitPartial;
      tile_coords(out.tile, p, mb, nb);
      return true;
    }
    pos = seg_end;
  }
  return false;
}

// The k-block visited at step i of a unit.  Whole tiles of every other wave walk k downwards
// (tile_k_reversed): the pairs run a wave's tiles at about the same time, so each wave's A panels (shared
// with the previous wave inside a raster group) are then first read where the previous wave read them last,
// while they are still in L2, instead of after a whole wave's worth of other traffic.  Stream-K pieces keep
// ascending order (their partial sums are indexed by k range, not by order).
__device__ __forceinline__ int unit_kb(const SkUnit &un, bool reversed, int i) {
  return (un.kind == kUnitWhole && reversed) ? un.kb1 - 1 - i : un.kb0 + i;
}

// First k-iteration (in the tail's linear k space) owned by worker w.
__device__ __forceinline__ long long sk_start(int w, int W, const TcParams &p) {
  return static_cast<long long>(w) * p.sk_iters / W;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_gpu(unsigned *p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <class Cfg>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg::THREADS, 1)
    gemm_bias_gelu_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC_tail,
                       const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

  uint8_t *sA = smem;
  uint8_t *sB = smem + Cfg::STAGES * Cfg::A_BYTES;
  uint8_t *sEpi = smem + Cfg::STAGES * Cfg::STAGE_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sEpi + Cfg::EPI_BYTES);
  uint64_t *full = bars;                        // [STAGES] leader: TMA bytes of both CTAs landed
  uint64_t *empty = bars + Cfg::STAGES;         // [STAGES] both: MMAs reading the stage finished
  uint64_t *tfull = bars + 2 * Cfg::STAGES;     // [2] both: accumulator ready
  uint64_t *tempty = tfull + 2;                 // [2] leader: both CTAs drained the accumulator
  uint64_t *drain = tempty + 2;                 // [1] leader: all MMAs complete
  uint64_t *epi_sync = drain + 1;               // [1] the 4 epilogue warps wrote this worker's partial
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
    if (Cfg::BN % 64 != 0) tma_prefetch_desc(&tmC_tail);
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);                   // the leader's producer arrives (with both CTAs' bytes)
      mbar_init(&empty[s], 1);                  // one multicast commit
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
  // Both CTAs' barriers are initialised before any remote arrive or TMA completion targets them.
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // Under a programmatic launch the set-up above overlapped the previous kernel's tail.  The roles that touch
  // global memory wait for that kernel to be done (griddepcontrol.wait) before their first access: the producer
  // before its first load (its first unit's coordinates are worked out before), the epilogue on entry.  The MMA
  // issuer touches only shared memory and TMEM.

  auto fail = [&](unsigned bit) {
    atomicOr(p.status, bit);
    *abort_flag = 1;
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int issued = 0;
      SkUnit un;
      int mb, nb;
      for (int u = 0; ok && sk_unit(pair, num_pairs, u, p, un, mb, nb); ++u) {
        const int m0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::BM_CTA;
        const int n0 = nb * Cfg::BN + static_cast<int>(rank) * Cfg::BN_CTA;
        const bool reversed = p.sk_band_workers == 0 && tile_k_reversed(p, mb, nb, num_pairs);
        for (int i = 0; i < un.kb1 - un.kb0; ++i) {
          const int kb = unit_kb(un, reversed, i);
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.timeout_ns, abort_flag)) {
            fail(kErrProducerWait);
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
          if (issued == 0) grid_dependency_wait();
          const uint32_t bar = pair_leader_addr(smem_u32(&full[stage]));
#pragma unroll
          for (int a = 0; a < Cfg::KATOMS; ++a)
            tma_load_2d_pair(sA + stage * Cfg::A_BYTES + a * Cfg::A_ATOM_BYTES, &tmA, bar,
                             kb * Cfg::BK + a * Cfg::ATOM_K, m0);
          uint8_t *b_dst = sB + stage * Cfg::B_BYTES;
#pragma unroll
          for (int j = 0; j < Cfg::B_CHUNKS; ++j)
            tma_load_2d_pair(b_dst + j * Cfg::B_CHUNK_BYTES, &tmB, bar, n0 + j * Cfg::B_CHUNK_N, kb * Cfg::BK);
          ++issued;
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && rank == 0) {
        // Let loads already in flight land before the pair may exit (bounded).
        for (int s = 0; s < Cfg::STAGES && s < issued; ++s) {
          const uint32_t ph = (s < stage) ? phase : (phase ^ 1u);
          volatile int no_abort = 0;
          if (!mbar_wait(&full[s], ph, p.timeout_ns, &no_abort)) atomicOr(p.status, kErrTeardownWait);
        }
      }
    }
    grid_launch_dependents();  // this CTA's loads are all issued
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader only)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      SkUnit un;
      int mb, nb;
      for (int u = 0; ok && sk_unit(pair, num_pairs, u, p, un, mb, nb); ++u) {
        if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, p.timeout_ns, abort_flag)) {
          fail(kErrMmaWait);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::ACC_STRIDE);
        for (int i = 0; i < un.kb1 - un.kb0; ++i) {
          if (!mbar_wait(&full[stage], phase, p.timeout_ns, abort_flag)) {
            fail(kErrMmaWait);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < Cfg::BK / Cfg::UMMA_K; ++k) {
            constexpr int PER_ATOM = Cfg::ATOM_K / Cfg::UMMA_K;
            const uint64_t ad =
                smem_desc(a_addr + (k / PER_ATOM) * Cfg::A_ATOM_BYTES + (k % PER_ATOM) * 32, 16, 1024, kSwizzle128B);
            const uint64_t bd = smem_desc(b_addr + k * Cfg::UMMA_K * 128, Cfg::B_CHUNK_BYTES, 1024, kSwizzle128B);
            const uint32_t accumulate = (i != 0 || k != 0) ? 1u : 0u;
            if constexpr (Cfg::ELEM == 2)
              tc_mma_f16_pair(d_tmem, ad, bd, Cfg::IDESC, accumulate);
            else
              tc_mma_f8_pair(d_tmem, ad, bd, Cfg::IDESC, accumulate);
          }
          tc_commit_pair_mc(&empty[stage], 0x3);
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair_mc(&tfull[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      tc_commit_pair(drain);
      volatile int no_abort = 0;
      if (!mbar_wait(drain, 0, p.timeout_ns, &no_abort)) atomicOr(p.status, kErrTeardownWait);
    }
    grid_launch_dependents();  // this CTA's MMAs are all issued (and, on the leader, complete)
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5, both CTAs)
    // A dependent launch may be scheduled once the producer and MMA warps are done (they signal last); its
    // CTAs find SMs as this grid's CTAs exit, overlapping its launch and set-up with this tail.
    grid_launch_dependents();
    grid_dependency_wait();
    const int q = warp & 3;
    const int ew = warp - 2;
    uint8_t *ebuf = sEpi + ew * Cfg::EPI_BUFS * Cfg::EPI_BUF_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    int buf = 0;
    SkUnit un;
    // This CTA's partial-sum slot (its 128 rows of a tile) in worker `w`'s workspace; a warp's 32 rows
    // are stored quad-of-columns-major so one warp-wide 16-byte access covers 512 contiguous bytes.
    auto slot = [&](int w) -> float4 * {
      return reinterpret_cast<float4 *>(p.sk_partials + (static_cast<size_t>(w) * 2 + rank) * Cfg::PARTIAL_FLOATS +
                                        static_cast<size_t>(q) * 32 * Cfg::BN);
    };
    int mb, nb;
    for (int u = 0; sk_unit(pair, num_pairs, u, p, un, mb, nb); ++u) {
      const float2 bias_first = lane_bias64(p, nb * Cfg::BN, lane);  // loaded while the accumulator fills
      const bool waited = mbar_wait(&tfull[acc], acc_phase, p.timeout_ns, abort_flag);
      if (!__all_sync(0xffffffffu, waited)) {
        if (lane == 0) fail(kErrEpilogueWait);
        break;
      }
      tc_fence_after();
      const int m0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::BM_CTA + q * 32;
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * Cfg::ACC_STRIDE);
      const uint32_t tempty_leader = mapa_shared(smem_u32(&tempty[acc]), 0);
      if (un.kind == kUnitPartial) {
        // Write this worker's fp32 partial (its k-range of the tile) and raise its flag.
        float4 *dst = slot(pair);
#pragma unroll 1
        for (int c = 0; c < Cfg::BN / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(t_row + c * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            __stcg(dst + (c * 8 + j4) * 32 + lane,
                   make_float4(__uint_as_float(v[j4 * 4 + 0]), __uint_as_float(v[j4 * 4 + 1]),
                               __uint_as_float(v[j4 * 4 + 2]), __uint_as_float(v[j4 * 4 + 3])));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader);
        // Every warp's stores are visible device-wide before it arrives; one lane publishes the flag
        // once all four have arrived (bounded wait, never a hardware barrier a departed warp could block).
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
          first = pair + 1;
          if (p.sk_band_workers > 0) {
            last = band_last_contributor(pair, nb, p);
          } else {
            const long long tile_end = static_cast<long long>(un.tile - p.dp_tiles + 1) * p.k_blocks;
            last = pair;
            while (last + 1 < num_pairs && sk_start(last + 1, num_pairs, p) < tile_end) ++last;
          }
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
          for (int w = first; w <= last; ++w) (void)ld_acquire_gpu(p.sk_flags + w * 2 + rank);  // every lane
          if constexpr (Cfg::BN % 64 == 0) {
            if (p.sk_band_workers > 0) {
              // Row-band mode: fold the partials into TMEM first (loads batched 64 columns at a time), then drain
              // the tile as a whole one.
              fold_partials<Cfg::BN>(t_row, 0, 0, slot(first) + lane, 2 * Cfg::PARTIAL_FLOATS / 4, last - pair);
              first = last + 1;
            }
          }
        }
        auto addend = [&](uint32_t(&v)[32], int c0) {
          for (int w = first; w <= last; ++w) {
            const float4 *src = slot(w) + (c0 / 4) * 32 + lane;
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 s = __ldcg(src + j4 * 32);
              v[j4 * 4 + 0] = __float_as_uint(__uint_as_float(v[j4 * 4 + 0]) + s.x);
              v[j4 * 4 + 1] = __float_as_uint(__uint_as_float(v[j4 * 4 + 1]) + s.y);
              v[j4 * 4 + 2] = __float_as_uint(__uint_as_float(v[j4 * 4 + 2]) + s.z);
              v[j4 * 4 + 3] = __float_as_uint(__uint_as_float(v[j4 * 4 + 3]) + s.w);
            }
          }
        };
        epilogue_rows<Cfg::BN>(
            t_row, m0, nb * Cfg::BN, p, &tmC, &tmC_tail, ebuf, buf, lane, bias_first,
            [&] {
              if (lane == 0) mbar_arrive_cluster(tempty_leader);
            },
            addend);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) tma_store_wait_all<0>();
    __syncwarp();
  }

  // Neither CTA releases TMEM or exits while its peer may still address it.
  __syncwarp();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace pf
