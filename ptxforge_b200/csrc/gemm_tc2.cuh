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
// Per SM this halves the shared-memory B traffic of the 1-CTA 128 x 256 kernel and, at 32 KB per
// stage, leaves room for 6 pipeline stages.
#pragma once

#include "gemm_tc.cuh"

namespace pf {

template <int kDtype, int kStages, int kKAtoms = 1>
struct Tc2Config {
  static constexpr int BM = 256;                             // pair tile rows
  static constexpr int BM_CTA = 128;
  static constexpr int BN = 256;                             // pair tile columns (UMMA N)
  static constexpr int BN_CTA = 128;                         // B columns loaded by each CTA
  static constexpr int STAGES = kStages;
  static constexpr int ELEM = (kDtype == 0) ? 2 : 1;
  static constexpr int KATOMS = kKAtoms;                     // 128-byte k-atoms per stage
  static constexpr int ATOM_K = 128 / ELEM;
  static constexpr int BK = KATOMS * ATOM_K;
  static constexpr int UMMA_K = 32 / ELEM;
  static constexpr int A_ATOM_BYTES = BM_CTA * 128;
  static constexpr int A_BYTES = KATOMS * A_ATOM_BYTES;
  static constexpr int B_CHUNK_N = 128 / ELEM;
  static constexpr int B_CHUNKS = BN_CTA / B_CHUNK_N;
  static constexpr int B_CHUNK_BYTES = BK * 128;
  static constexpr int B_BYTES = B_CHUNKS * B_CHUNK_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;      // per CTA
  static constexpr int EPI_WARPS = 4;
  static constexpr int EPI_BUF_BYTES = 32 * 64 * 2;
  static constexpr int EPI_BUFS = 2;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUFS * EPI_BUF_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 4 + 1;
  static constexpr int TMEM_COLS = 512;                      // 2 accumulators x 256 columns
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + NUM_BARS * 8 + 16;
  static constexpr int THREADS = 192;
  static constexpr uint32_t IDESC =
      instr_desc(kDtype == 0 ? 1u : 0u, kDtype == 0 ? 1u : 0u, 0u, 1u, /*M*/ 256, /*N*/ 256);
  static_assert(SMEM_BYTES <= 232448, "shared memory per block exceeds the sm_100 opt-in limit");
};

template <class Cfg>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg::THREADS, 1)
    gemm_bias_gelu_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
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
  uint64_t *tfull = bars + 2 * Cfg::STAGES;     // [2] both: accumulator ready
  uint64_t *tempty = tfull + 2;                 // [2] leader: both CTAs drained the accumulator
  uint64_t *drain = tempty + 2;                 // [1] leader: all MMAs complete
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);
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
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * Cfg::EPI_WARPS);
    }
    mbar_init(drain, 1);
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
      for (int t = pair; t < p.num_tiles && ok; t += num_pairs) {
        int mb, nb;
        tile_coords(t, p, mb, nb);
        const int m0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::BM_CTA;
        const int n0 = nb * Cfg::BN + static_cast<int>(rank) * Cfg::BN_CTA;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.timeout_ns, abort_flag)) {
            fail(kErrProducerWait);
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
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
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader only)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < p.num_tiles && ok; t += num_pairs) {
        if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, p.timeout_ns, abort_flag)) {
          fail(kErrMmaWait);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
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
            if constexpr (Cfg::ELEM == 2)
              tc_mma_f16_pair(d_tmem, ad, bd, Cfg::IDESC, (kb | k) != 0);
            else
              tc_mma_f8_pair(d_tmem, ad, bd, Cfg::IDESC, (kb | k) != 0);
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
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5, both CTAs)
    const int q = warp & 3;
    const int ew = warp - 2;
    uint8_t *ebuf = sEpi + ew * Cfg::EPI_BUFS * Cfg::EPI_BUF_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    int buf = 0;
    for (int t = pair; t < p.num_tiles; t += num_pairs) {
      int mb, nb;
      tile_coords(t, p, mb, nb);
      const bool waited = mbar_wait(&tfull[acc], acc_phase, p.timeout_ns, abort_flag);
      if (!__all_sync(0xffffffffu, waited)) {
        if (lane == 0) fail(kErrEpilogueWait);
        break;
      }
      tc_fence_after();
      const int m0 = mb * Cfg::BM + static_cast<int>(rank) * Cfg::BM_CTA + q * 32;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * Cfg::BN);
      const uint32_t tempty_leader = mapa_shared(smem_u32(&tempty[acc]), 0);
      epilogue_rows<Cfg::BN>(t_row, m0, nb * Cfg::BN, p, &tmC, ebuf, buf, lane, [&] {
        if (lane == 0) mbar_arrive_cluster(tempty_leader);
      });
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
