// gemm_tc2w.cuh -- the fused GEMM + bias + GELU on CTA pairs with 256 x 512 tiles.
//
// Per k step a pair of the 256 x 256 kernel (gemm_tc2.cuh) loads 256 rows of A and 256 columns of B for
// 65,536 outputs; a pair here loads 256 rows of A and 512 columns of B for 131,072 outputs: a quarter
// fewer operand bytes through L2 per output.  Under back-to-back launches the B200 runs at its power
// cap, so those bytes cost clock, not just bandwidth.
//
// Each CTA's 128 accumulator rows x 512 fp32 columns fill its TMEM, so there is one accumulator per CTA,
// handed back in two halves: the epilogue drains columns [0, 256) and releases them, and the next
// unit's MMAs into that half start while it drains [256, 512).  The MMA issuer runs a stage's second-half
// MMAs as soon as that half is free; until then it holds at most STAGES stages whose second half is
// still to do (their shared memory stays loaded), and waits only when all of them are held.
//   * TMA (both CTAs): per stage, A rows [m0 + 128*rank, +128) and, for each half h, B columns
//     [n0 + 256*h + 128*rank, +128), counted on the leader's `full` barrier (no multicast);
//   * MMA (leader lane): per stage and half h, tcgen05.mma.cta_group::2 with M = 256, N = 256 into TMEM
//     columns [256*h, 256*h + 256); tcgen05.commit multicasts stage-free and accumulator-ready;
//   * epilogue (kEpiWarps warps from warp 2, both CTAs): the 256-wide kernel's epilogue, one half at a time,
//     each half released to the leader's `tempty[h]` right after its last TMEM load.  With 8 warps two
//     share each 32-lane quarter of TMEM and split a half's 256 columns, so a half drains in about half the
//     time: the tensor pipe waits on that drain at every tile boundary.
//   * tail split: a pair's last tile has no next tile to hide its epilogue behind, and a 128 x 512 drain per
//     CTA takes ~8 us.  So its last L k steps (p.tail_split) run half 0 first, then half 1 (A is loaded a
//     second time for those steps); `tfull[0]` fires after half 0's last MMA and the epilogue drains half 0
//     while the tensor pipe finishes half 1.  Every output still sums its k blocks in the same order.
//
// Work units.  Whole tiles round-robin over the pairs (k direction alternating by wave as in the other
// kernels), or -- when p.sk_band_workers > 0 -- row-band stream-K: each row block of tiles is a band
// shared by P pairs, pair j of a band taking k-iterations [j*S/P, (j+1)*S/P) of the band's S = tiles x k
// blocks (tiles left to right, k ascending).  A row shard of 1,024 x 8,192 has 64 tiles for 74 pairs:
// whole tiles leave 10 pairs idle, 4 bands of 18 pairs keep 72 busy.  Bands rather than one stream over all
// tiles because pairs j of every band then work on the same B panel at the same k at the same time, so each
// B slab comes from DRAM once and from L2 for the other bands; a stream-K order that does not line the tiles
// of a B panel up in time re-reads B from DRAM per row block.  A tile split between pairs is finished by the
// pair holding its first k-block (the "head", always a pair's last unit); the others ("partials", always a
// pair's first unit) write their fp32 sums to a workspace and raise a flag tagged with the launch's epoch;
// the head adds them before its epilogue.  Every wait is bounded.
#pragma once

#include "gemm_tc2.cuh"

namespace pf {

template <int kDtype, int kStages, int kEpiWarps = 4, int kEpiBufs = 2>
struct Tc2wConfig {
  static constexpr int BM = 256;                             // pair tile rows
  static constexpr int BM_CTA = 128;
  static constexpr int BN = 512;                             // pair tile columns
  static constexpr int HALF_N = 256;                         // UMMA N of each half
  static constexpr int STAGES = kStages;
  static constexpr int ELEM = (kDtype == 0) ? 2 : 1;
  static constexpr int KATOMS = 1;                           // one 128-byte k-atom per stage
  static constexpr int ATOM_K = 128 / ELEM;
  static constexpr int BK = ATOM_K;
  static constexpr int UMMA_K = 32 / ELEM;
  static constexpr int A_BYTES = BM_CTA * 128;
  static constexpr int B_CHUNK_N = 128 / ELEM;               // N elements per 128-byte row of B
  static constexpr int B_CHUNKS_HALF = (HALF_N / 2) / B_CHUNK_N;  // boxes per CTA and half
  static constexpr int B_CHUNK_BYTES = BK * 128;
  static constexpr int B_HALF_BYTES = B_CHUNKS_HALF * B_CHUNK_BYTES;
  static constexpr int B_BYTES = 2 * B_HALF_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;      // per CTA
  static constexpr int EPI_WARPS = kEpiWarps;                // 4 or 8: 1 or 2 per 32-lane quarter of TMEM
  static constexpr int EPI_SPLIT = kEpiWarps / 4;            // warps sharing a quarter split its columns
  static constexpr int EPI_COLS_WARP = HALF_N / EPI_SPLIT;   // columns of a half each epilogue warp drains
  static constexpr int EPI_BUF_BYTES = 32 * 64 * 2;
  static constexpr int EPI_BUFS = kEpiBufs;                  // staging boxes per epilogue warp (1: 4 stages fit)
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUFS * EPI_BUF_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 2 + 2 + 1 + 1;
  static constexpr int TMEM_COLS = 512;                      // one accumulator: two halves of 256 columns
  static constexpr int PARTIAL_FLOATS = BM_CTA * BN;         // one CTA's share of a tile, fp32
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + NUM_BARS * 8 + 16;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  static constexpr uint32_t IDESC =
      instr_desc(kDtype == 0 ? 1u : 0u, kDtype == 0 ? 1u : 0u, 0u, 1u, /*M*/ 256, /*N*/ HALF_N);
  static_assert(kEpiWarps == 4 || kEpiWarps == 8, "4 or 8 epilogue warps");
  static_assert(kEpiBufs == 2 || (kEpiBufs == 1 && kEpiWarps == 8), "one staging box only with 8 epilogue warps");
  // Only the 128-column epilogue (8 warps) takes the staging-box count; the other one (epilogue_rows) alternates
  // between two boxes per warp, and a single box would let it write into the next warp's box or the barriers.
  static_assert(EPI_COLS_WARP == 128 || kEpiBufs == 2, "epilogue_rows needs two staging boxes per warp");
  static_assert(SMEM_BYTES <= 232448, "shared memory per block exceeds the sm_100 opt-in limit");
  static_assert(B_CHUNKS_HALF >= 1, "each CTA supplies at least one 128-byte box of B per half");
};

// One unit of a pair's work: tile (mb, nb), k-blocks [kb0, kb1), whole / head / partial (kUnit*).
struct WideUnit {
  int mb, nb, kb0, kb1, kind;
  bool reversed;  // whole tiles of odd waves walk k downwards (data-parallel schedule only)
};


// Unit `u` of pair `w` of `W`; false past the pair's last unit.
__device__ __forceinline__ bool wide_unit(int w, int W, int u, const TcParams &p, WideUnit &out) {
  if (p.sk_band_workers <= 0) {
    const int t = w + u * W;
    if (t >= p.num_tiles) return false;
    int mb, nb;
    tile_coords(t, p, mb, nb);
    out = {mb, nb, 0, p.k_blocks, kUnitWhole, tile_k_reversed(p, mb, nb, W)};
    return true;
  }
  const int P = p.sk_band_workers;
  const int g = w / P, j = w % P;
  if (g >= p.num_m_blocks) return false;
  const int KB = p.k_blocks;
  const int S = p.num_n_blocks * KB;
  const int e = band_start(j + 1, P, S);
  int pos = band_start(j, P, S);
  for (int i = 0; pos < e; ++i) {
    const int nb = pos / KB;
    const int seg_end = min(e, (nb + 1) * KB);
    if (i == u) {
      out.mb = g;
      out.nb = nb;
      out.kb0 = pos - nb * KB;
      out.kb1 = seg_end - nb * KB;
      out.kind = out.kb0 == 0 ? (out.kb1 == KB ? kUnitWhole : kUnitHead) : kUnitPartial;
      out.reversed = false;
      return true;
    }
    pos = seg_end;
  }
  return false;
}

// k steps at the end of unit `u` (= un) of pair `w` whose half-1 MMAs follow all of half 0's (0: interleaved
// throughout): only the pair's last whole tile, and at most half of its k steps.
__device__ __forceinline__ int wide_tail_split(int w, int W, int u, const TcParams &p, const WideUnit &un) {
  if (p.tail_split <= 0 || p.sk_band_workers > 0 || un.kind != kUnitWhole) return 0;
  WideUnit next;
  if (wide_unit(w, W, u + 1, p, next)) return 0;
  return min(p.tail_split, (un.kb1 - un.kb0) / 2);
}

// The step order of a unit of S k steps with tail split L: steps j < S - L load and run both halves of k step
// j; then S - L <= j < S half 0 only of k step j; then S <= j < S + L half 1 only of k step j - L.
struct WideStep {
  int i;       // the unit's k step (0 .. S-1, in the unit's k direction)
  int halves;  // bit h: half h's B columns are loaded and its MMAs run
};
__device__ __forceinline__ WideStep wide_step(int j, int S, int L) {
  if (j < S - L) return {j, 3};
  if (j < S) return {j, 1};
  return {j - L, 2};
}

// One epilogue warp's 32 rows x 128 columns of one accumulator half: the four 32-column TMEM loads first,
// then the half is handed back (`release`) before any epilogue math, which runs from registers while the
// next tile's MMAs already write that half; then x*scale + bias, GELU, bf16, two 32 x 64 boxes through the
// double-buffered (BUFS = 2) or single (1) swizzled staging area and TMA stores, as epilogue_rows.
// The bias travels one value per lane: `bias_lane` holds this lane's of column n0 + lane (loaded before the
// accumulator was ready); each 32-column step loads the next step's, the last one that of column
// next_col + lane (the next half's first step; none if next_col < 0), which is what `bias_lane` holds on return.
template <int BUFS = 2, class Release>
__device__ __forceinline__ void epilogue_rows128_early(uint32_t t_col, int m0, int n0, const TcParams &p,
                                                       float &bias_lane, int next_col, const CUtensorMap *tmC,
                                                       uint8_t *ebuf, int &buf, int lane, Release release) {
  constexpr int BUF_BYTES = 32 * 64 * 2;
  uint32_t v[4][32];
#pragma unroll
  for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_col + c * 32, v[c]);
  tmem_ld_wait();
  tc_fence_before();
  __syncwarp();
  release();
#pragma unroll
  for (int b = 0; b < 2; ++b) {
    const uint32_t sbuf = smem_u32(ebuf + buf * BUF_BYTES) + lane * 128;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int col = (b * 2 + h < 3) ? n0 + (b * 2 + h + 1) * 32 + lane : (next_col < 0 ? p.N : next_col + lane);
      const float bias_next = col < p.N ? __ldg(p.bias + col) : 0.f;
      uint32_t packed[16];
      epilogue_math32_lane_bias<false>(v[b * 2 + h], bias_lane, p.scale, packed);
      bias_lane = bias_next;
      // Row `lane` of the 32 x 64 box: 16-byte chunk j goes to chunk j ^ (row % 8) (128-B swizzle).
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t chunk = static_cast<uint32_t>((h * 4 + i) ^ (lane & 7));
        st_shared_v4(sbuf + chunk * 16, packed[i * 4 + 0], packed[i * 4 + 1], packed[i * 4 + 2], packed[i * 4 + 3]);
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (n0 + b * 64 < p.N) tma_store_2d(tmC, ebuf + buf * BUF_BYTES, n0 + b * 64, m0);
      tma_store_commit();
      tma_store_wait_read<BUFS - 1>();  // the buffer written next is free again
    }
    __syncwarp();
    if constexpr (BUFS == 2) buf ^= 1;
  }
}

// A split tile's fp32 partial sums: one epilogue warp's 32 rows x COLS columns of a half, from TMEM to its
// slot (float4 index ((col / 4) * 32 + lane) from `dst`: each warp-wide store covers 512 contiguous bytes).
// 64 columns at a time are loaded, then stored; the half is released after its last load.
template <int COLS, class Release>
__device__ __forceinline__ void partial_rows(uint32_t t_col, float4 *dst, int lane, Release release) {
  static_assert(COLS % 64 == 0, "64-column steps");
#pragma unroll 1
  for (int s = 0; s < COLS / 64; ++s) {
    uint32_t v[2][32];
#pragma unroll
    for (int c = 0; c < 2; ++c) tmem_ld_32x32b_x32(t_col + s * 64 + c * 32, v[c]);
    tmem_ld_wait();
    if (s == COLS / 64 - 1) {
      tc_fence_before();
      __syncwarp();
      release();
    }
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4)
        __stcg(dst + ((s * 64 + c * 32) / 4 + j4) * 32 + lane,
               make_float4(__uint_as_float(v[c][j4 * 4 + 0]), __uint_as_float(v[c][j4 * 4 + 1]),
                           __uint_as_float(v[c][j4 * 4 + 2]), __uint_as_float(v[c][j4 * 4 + 3])));
  }
}

template <class Cfg>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg::THREADS, 1)
    gemm_bias_gelu_tc2w(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

  uint8_t *sA = smem;
  uint8_t *sB = smem + Cfg::STAGES * Cfg::A_BYTES;
  uint8_t *sEpi = smem + Cfg::STAGES * Cfg::STAGE_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sEpi + Cfg::EPI_BYTES);
  uint64_t *full = bars;                        // [STAGES] leader: TMA bytes of both CTAs landed
  uint64_t *empty = bars + Cfg::STAGES;         // [STAGES] both: MMAs reading the stage finished
  uint64_t *tfull = bars + 2 * Cfg::STAGES;     // [2] both: accumulator half h ready
  uint64_t *tempty = tfull + 2;                 // [2] leader: both CTAs drained half h
  uint64_t *drain = tempty + 2;                 // [1] leader: all MMAs complete
  uint64_t *epi_sync = drain + 1;               // [1] the epilogue warps wrote this pair's partial
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
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);                   // the leader's producer arrives (with both CTAs' bytes)
      mbar_init(&empty[s], 1);                  // one multicast commit
    }
    mbar_init(&tfull[0], 1);
    mbar_init(&tfull[1], 1);
    mbar_init(&tempty[0], 2 * Cfg::EPI_WARPS);
    mbar_init(&tempty[1], 2 * Cfg::EPI_WARPS);
    mbar_init(drain, 1);
    mbar_init(epi_sync, Cfg::EPI_WARPS);        // completes at most once: a pair has at most one partial
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
      WideUnit un;
      for (int u = 0; ok && wide_unit(pair, num_pairs, u, p, un); ++u) {
        const int m0 = un.mb * Cfg::BM + static_cast<int>(rank) * Cfg::BM_CTA;
        const int n0 = un.nb * Cfg::BN + static_cast<int>(rank) * (Cfg::HALF_N / 2);
        const int S = un.kb1 - un.kb0;
        const int L = wide_tail_split(pair, num_pairs, u, p, un);
        for (int j = 0; j < S + L; ++j) {
          const WideStep st = wide_step(j, S, L);
          const int kb = un.reversed ? un.kb1 - 1 - st.i : un.kb0 + st.i;
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.timeout_ns, abort_flag)) {
            fail(kErrProducerWait);
            ok = false;
            break;
          }
          if (rank == 0)
            mbar_arrive_expect_tx(&full[stage],
                                  2 * (Cfg::A_BYTES + (st.halves == 3 ? 2 : 1) * Cfg::B_HALF_BYTES));
          if (issued == 0) grid_dependency_wait();
          const uint32_t bar = pair_leader_addr(smem_u32(&full[stage]));
          tma_load_2d_pair(sA + stage * Cfg::A_BYTES, &tmA, bar, kb * Cfg::BK, m0);
          uint8_t *b_dst = sB + stage * Cfg::B_BYTES;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (!((st.halves >> h) & 1)) continue;
#pragma unroll
            for (int c = 0; c < Cfg::B_CHUNKS_HALF; ++c)
              tma_load_2d_pair(b_dst + h * Cfg::B_HALF_BYTES + c * Cfg::B_CHUNK_BYTES, &tmB, bar,
                               n0 + h * Cfg::HALF_N + c * Cfg::B_CHUNK_N, kb * Cfg::BK);
          }
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
      uint32_t tphase = 0;  // parity of this pair's unit count: the halves are released once per unit
      bool ok = true;
      const uint32_t tempty1_addr = smem_u32(&tempty[1]);
      // Half h's MMAs of the stage in ring slot s, the unit's i-th k step.
      auto issue_half = [&](int s, int h, int i) {
        const uint32_t a_addr = smem_u32(sA + s * Cfg::A_BYTES);
        const uint32_t b_addr = smem_u32(sB + s * Cfg::B_BYTES + h * Cfg::B_HALF_BYTES);
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(h * Cfg::HALF_N);
#pragma unroll
        for (int k = 0; k < Cfg::BK / Cfg::UMMA_K; ++k) {
          const uint64_t ad = smem_desc(a_addr + k * 32, 16, 1024, kSwizzle128B);
          const uint64_t bd = smem_desc(b_addr + k * Cfg::UMMA_K * 128, Cfg::B_CHUNK_BYTES, 1024, kSwizzle128B);
          const uint32_t accumulate = (i != 0 || k != 0) ? 1u : 0u;
          if constexpr (Cfg::ELEM == 2)
            tc_mma_f16_pair(d_tmem, ad, bd, Cfg::IDESC, accumulate);
          else
            tc_mma_f8_pair(d_tmem, ad, bd, Cfg::IDESC, accumulate);
        }
      };
      // The second half of the `pending` most recent stages (the last in slot `last`, k step i_last),
      // oldest first, each stage handed back to the producers once its second half is issued.
      auto flush = [&](int pending, int last, int i_last) {
        for (int j = pending - 1; j >= 0; --j) {
          const int s = (last - j + Cfg::STAGES) % Cfg::STAGES;
          issue_half(s, 1, i_last - j);
          tc_commit_pair_mc(&empty[s], 0x3);
        }
      };
      WideUnit un;
      for (int u = 0; ok && wide_unit(pair, num_pairs, u, p, un); ++u) {
        const int S = un.kb1 - un.kb0;
        const int L = wide_tail_split(pair, num_pairs, u, p, un);
        // The first half of the accumulator must be drained of the previous unit.
        if (!mbar_wait_cluster(&tempty[0], tphase ^ 1u, p.timeout_ns, abort_flag)) {
          fail(kErrMmaWait);
          ok = false;
          break;
        }
        tc_fence_after();
        bool second_free = false;
        int pending = 0;  // stages whose second-half MMAs wait for the second half of TMEM
        int last = 0;
        for (int j = 0; j < S + L; ++j) {
          const WideStep st = wide_step(j, S, L);
          if (st.halves != 3 && (pending > 0 || !second_free)) {
            // Entering the split tail: the second half is needed from here on, and stages held for it go first.
            if (!second_free) {
              if (!mbar_wait_cluster(&tempty[1], tphase ^ 1u, p.timeout_ns, abort_flag)) {
                fail(kErrMmaWait);
                ok = false;
                break;
              }
              second_free = true;
              tc_fence_after();
            }
            flush(pending, last, S - L - 1);
            pending = 0;
          }
          if (!mbar_wait(&full[stage], phase, p.timeout_ns, abort_flag)) {
            fail(kErrMmaWait);
            ok = false;
            break;
          }
          tc_fence_after();
          if (st.halves == 3) {
            issue_half(stage, 0, st.i);
            ++pending;
            last = stage;
            if (!second_free && mbar_test_wait_acq_cluster(tempty1_addr, tphase ^ 1u)) {
              second_free = true;
              tc_fence_after();
            }
            if (!second_free && pending == Cfg::STAGES) {
              // Every stage is held: nothing more can load until the second half is free.
              if (!mbar_wait_cluster(&tempty[1], tphase ^ 1u, p.timeout_ns, abort_flag)) {
                fail(kErrMmaWait);
                ok = false;
                break;
              }
              second_free = true;
              tc_fence_after();
            }
            if (second_free) {
              flush(pending, last, st.i);
              pending = 0;
            }
          } else {
            // The split tail: one half per stage, the stage handed back right after it.
            issue_half(stage, st.halves == 1 ? 0 : 1, st.i);
            tc_commit_pair_mc(&empty[stage], 0x3);
          }
          if (j == S - 1) tc_commit_pair_mc(&tfull[0], 0x3);  // every MMA of half 0 is issued
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (pending > 0) {
          // A unit of fewer k steps than stages: its second half waits here.
          if (!mbar_wait_cluster(&tempty[1], tphase ^ 1u, p.timeout_ns, abort_flag)) {
            fail(kErrMmaWait);
            ok = false;
            break;
          }
          tc_fence_after();
          flush(pending, last, S - 1);
        }
        tc_commit_pair_mc(&tfull[1], 0x3);
        tphase ^= 1u;
      }
      tc_commit_pair(drain);
      volatile int no_abort = 0;
      if (!mbar_wait(drain, 0, p.timeout_ns, &no_abort)) atomicOr(p.status, kErrTeardownWait);
    }
    grid_launch_dependents();  // this CTA's MMAs are all issued (and, on the leader, complete)
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2.., both CTAs)
    // A dependent launch may be scheduled once the producer and MMA warps are done (they signal last); its
    // CTAs find SMs as this grid's CTAs exit, overlapping its launch and set-up with this tail.
    grid_launch_dependents();
    grid_dependency_wait();
    const int q = warp & 3;                     // the TMEM lane quarter this warp may read
    const int ew = warp - 2;
    const int col0 = (ew / 4) * Cfg::EPI_COLS_WARP;  // its columns within each half
    uint8_t *ebuf = sEpi + ew * Cfg::EPI_BUFS * Cfg::EPI_BUF_BYTES;
    uint32_t tphase = 0;
    int buf = 0;
    const uint32_t tempty0_leader = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint32_t tempty1_leader = mapa_shared(smem_u32(&tempty[1]), 0);
    // This warp's share of pair w's partial slot: its 32 rows (TMEM quarter q) of this CTA's 128, stored
    // columns-of-4 major so a warp-wide 16-byte access covers 512 contiguous bytes.
    auto slot = [&](int w) -> float4 * {
      return reinterpret_cast<float4 *>(p.sk_partials +
                                        (static_cast<size_t>(w) * 2 + rank) * Cfg::PARTIAL_FLOATS +
                                        static_cast<size_t>(q) * 32 * Cfg::BN);
    };
    // Whether accumulator half h of the current unit is complete (bounded wait, the whole warp agrees).
    auto half_ready = [&](int h) -> bool {
      const bool waited = mbar_wait(&tfull[h], tphase, p.timeout_ns, abort_flag);
      if (!__all_sync(0xffffffffu, waited)) {
        if (lane == 0) fail(kErrEpilogueWait);
        return false;
      }
      tc_fence_after();
      return true;
    };
    WideUnit un;
    for (int u = 0; wide_unit(pair, num_pairs, u, p, un); ++u) {
      // This lane's bias of the warp's first column of the unit's tile, loaded while the accumulator fills.
      const int first_col = un.nb * Cfg::BN + col0 + lane;
      float bias_lane = (Cfg::EPI_COLS_WARP == 128 && first_col < p.N) ? __ldg(p.bias + first_col) : 0.f;
      if (!half_ready(0)) break;
      bool second_ready = false;
      const int m0 = un.mb * Cfg::BM + static_cast<int>(rank) * Cfg::BM_CTA + q * 32;
      const int n_tile = un.nb * Cfg::BN;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      auto release0 = [&] {
        if (lane == 0) mbar_arrive_cluster(tempty0_leader);
      };
      auto release1 = [&] {
        if (lane == 0) mbar_arrive_cluster(tempty1_leader);
      };
      if (un.kind == kUnitPartial) {
        // This pair's first k-blocks of a tile another pair finishes: fp32 sums to the workspace, then the flag.
        float4 *dst = slot(pair);
        partial_rows<Cfg::EPI_COLS_WARP>(t_row + col0, dst + (col0 / 4) * 32, lane, release0);
        if (!half_ready(1)) break;
        partial_rows<Cfg::EPI_COLS_WARP>(t_row + Cfg::HALF_N + col0, dst + ((Cfg::HALF_N + col0) / 4) * 32, lane,
                                         release1);
        // Every warp's stores are visible device-wide before it arrives; one lane publishes the flag once
        // all of them have (a bounded wait, never a hardware barrier a departed warp could block).
        __threadfence();
        __syncwarp();
        if (lane == 0) mbar_arrive(epi_sync);
        if (ew == 0 && lane == 0) {
          if (mbar_wait(epi_sync, 0, p.timeout_ns, abort_flag))
            st_release_gpu(p.sk_flags + pair * 2 + rank, p.epoch);
          else
            fail(kErrEpilogueWait);
        }
      } else if (un.kind == kUnitHead) {
        // The first k-blocks of a tile whose later k-blocks the next pairs of this band summed: wait for their
        // flags (bounded), then fold their partials into the accumulator (both halves).
        if (!half_ready(1)) break;
        second_ready = true;
        const int last = band_last_contributor(pair, un.nb, p);
        bool ok = true;
        if (lane == 0) {
          for (int w = pair + 1; w <= last && ok; ++w) {
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
        for (int w = pair + 1; w <= last; ++w) (void)ld_acquire_gpu(p.sk_flags + w * 2 + rank);  // every lane
        // Fold the partials of pairs [pair + 1, last] into this warp's accumulator rows in TMEM (both of its
        // 128-column pieces); the tile then drains through the whole-tile epilogue below.
        fold_partials<Cfg::EPI_COLS_WARP, 2>(t_row, col0, Cfg::HALF_N, slot(pair + 1) + lane,
                                             2 * Cfg::PARTIAL_FLOATS / 4, last - pair);
      }
      if (un.kind != kUnitPartial) {
        if constexpr (Cfg::EPI_COLS_WARP == 128) {
          // 128 columns fit in registers: each half goes back to the MMA issuer as soon as it is loaded.
          epilogue_rows128_early<Cfg::EPI_BUFS>(t_row + col0, m0, n_tile + col0, p, bias_lane,
                                                n_tile + Cfg::HALF_N + col0, &tmC, ebuf, buf, lane, release0);
          if (!second_ready && !half_ready(1)) break;
          epilogue_rows128_early<Cfg::EPI_BUFS>(t_row + Cfg::HALF_N + col0, m0, n_tile + Cfg::HALF_N + col0, p,
                                                bias_lane, -1, &tmC, ebuf, buf, lane, release1);
        } else {
          epilogue_rows<Cfg::EPI_COLS_WARP>(t_row + col0, m0, n_tile + col0, p, &tmC, nullptr, ebuf, buf, lane,
                                            lane_bias64(p, n_tile + col0, lane), release0);
          if (!second_ready && !half_ready(1)) break;
          epilogue_rows<Cfg::EPI_COLS_WARP>(t_row + Cfg::HALF_N + col0, m0, n_tile + Cfg::HALF_N + col0, p, &tmC,
                                            nullptr, ebuf, buf, lane, lane_bias64(p, n_tile + Cfg::HALF_N + col0, lane),
                                            release1);
        }
      }
      tphase ^= 1u;
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
