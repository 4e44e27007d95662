// gemm_tc.cuh -- fused C = gelu_tanh(scale * A.B + bias) on the 5th-generation tensor cores.
//
// Persistent, warp-specialised kernel for sm_100a (one CTA per SM, 192 threads):
//   warp 0      TMA producer: one elected lane streams A (K-major) and B (N-major) k-blocks into a
//               STAGES-deep ring of 128-byte-swizzled shared-memory tiles (full/empty mbarriers); every
//               other wave of tiles walks k downwards (tile_k_reversed), so the next wave starts on the A
//               and B slabs the previous wave read last (still in L2).
//   warp 1      MMA issuer: allocates TMEM, one lane issues tcgen05.mma (M=128, N=BN, K=16 bf16 /
//               32 e4m3) into a double-buffered fp32 accumulator (2 x BN TMEM columns) and
//               tcgen05.commit's the smem stage back to the producer and the finished accumulator
//               to the epilogue.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time, x*scale + bias[c], GELU(tanh form) with
//               MUFU tanh, round to bf16, stage through swizzled shared memory and TMA-store; the
//               pre-activation never touches HBM.  The accumulator buffer is handed back to the
//               MMA warp right after its last TMEM load, so tile i's epilogue overlaps tile i+1's
//               mainloop.
//
// Math is that of the reference kernel (kernels/gemm_bias_gelu.cu:37-40, 89-97): a row-major
// GEMM over K followed by +bias[c] and gelu_tanh with k0 = 0.7978845608028654, k1 = 0.044715.
// Inputs here are bf16 or e4m3 (the reference is fp32 only), accumulation is fp32 in TMEM.
//
// Shapes: any M >= 1; N and K as required by TMA row strides (multiples of 16 bytes).  Partial
// tiles are handled by TMA: loads outside the tensor are zero-filled (contribute 0 to the dot
// product) and stores outside it are clipped.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "sm100.cuh"

namespace pf {

struct TcParams {
  const float *bias;
  float scale;             // scale_a * scale_b (1 for bf16)
  int M, N, K;
  int num_m_blocks, num_n_blocks, num_tiles, k_blocks;
  int group_m;             // raster: tiles walk `group_m` M-blocks before moving to the next N-block
  unsigned *status;        // device status word (bounded-wait timeouts)
  unsigned long long timeout_ns;
  // Stream-K tail (CTA-pair kernel only; dp_tiles == num_tiles turns it off): tiles [0, dp_tiles) are
  // processed whole; the k-iterations of tiles [dp_tiles, num_tiles) are spread evenly over the workers.
  int dp_tiles = 0;
  long long sk_iters = 0;  // (num_tiles - dp_tiles) * k_blocks
  unsigned epoch = 0;      // this launch's tag for the partial-ready flags
  float *sk_partials = nullptr;    // [workers][2 CTAs][128 x 256] fp32
  unsigned *sk_flags = nullptr;    // [workers][2 CTAs]
  // The schedule that sets each tile's k direction (tile_k_reversed): 0 = this launch's own.  A launch over a
  // window of rows of a larger bound problem passes the whole problem's, so its tiles are summed in the same
  // order -- and give the same bits -- as in one launch over the whole problem.
  int dir_m0 = 0;             // first row block of this launch within the whole problem
  int dir_num_m_blocks = 0;   // row blocks of the whole problem
  int dir_group_m = 0;        // raster group of the whole problem's launch
  int dir_workers = 0;        // workers (CTAs or CTA pairs) of the whole problem's launch
  // Row-band stream-K (256 x 512 pair kernel only; 0 = off): each row block of tiles is a band worked by this
  // many pairs, each taking an equal contiguous share of the band's k-iterations (tiles left to right, k
  // ascending).  Pairs at the same position in different bands read the same B panel at the same time.
  // Partials go to sk_partials as [workers][2 CTAs][128 x 512] fp32; flags and epoch as above.
  int sk_band_workers = 0;
  // Tail split (256 x 512 pair kernel only; 0 = off): in a pair's last whole tile, the second half's MMAs of the
  // last min(tail_split, k_blocks / 2) k steps run after all of the first half's, so the epilogue drains the
  // first half while the tensor pipe still works on the second.  Same k order per output: same bits.
  int tail_split = 0;
  // Periodic promotion (3xTF32 kernel only; 0 = off): a unit's k range is summed in chunks of promote_kb k-blocks
  // that alternate between the two TMEM accumulators, and the epilogue adds each finished chunk into an fp32
  // running sum (round to nearest) in promote_ws ([workers][2 CTAs][128 x 256] fp32), so the tensor cores'
  // round-toward-zero accumulation spans promote_kb k-blocks, not the whole k range.
  int promote_kb = 0;
  float *promote_ws = nullptr;
};

// kDtype: 0 = bf16 (kind::f16), 1 = e4m3 (kind::f8f6f4).
template <int kDtype, int kBN, int kStages, int kKAtoms = 1>
struct TcConfig {
  static constexpr int BM = 128;
  static constexpr int BN = kBN;
  static constexpr int STAGES = kStages;
  static constexpr int ELEM = (kDtype == 0) ? 2 : 1;        // bytes per A/B element
  static constexpr int KATOMS = kKAtoms;                     // 128-byte k-atoms per stage
  static constexpr int ATOM_K = 128 / ELEM;                  // k elements in one 128-B swizzle row
  static constexpr int BK = KATOMS * ATOM_K;                 // k elements per stage
  static constexpr int UMMA_K = 32 / ELEM;                   // k per tcgen05.mma
  static constexpr int A_ATOM_BYTES = BM * 128;              // 128 rows x 128 B
  static constexpr int A_BYTES = KATOMS * A_ATOM_BYTES;
  static constexpr int B_CHUNK_N = 128 / ELEM;               // N elements per 128-B row of B
  static constexpr int B_CHUNKS = BN / B_CHUNK_N;            // TMA boxes of B per stage
  static constexpr int B_CHUNK_BYTES = BK * 128;             // BK rows x 128 B
  static constexpr int B_BYTES = B_CHUNKS * B_CHUNK_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_WARPS = 4;
  static constexpr int EPI_COLS = 64;                        // bf16 output columns per TMA store box
  static constexpr int EPI_BUF_BYTES = 32 * EPI_COLS * 2;   // 32 rows x 128 B
  static constexpr int EPI_BUFS = 2;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUFS * EPI_BUF_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 4 + 1;
  static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int SMEM_BYTES = 1024 /*alignment slack*/ + STAGES * STAGE_BYTES + EPI_BYTES + NUM_BARS * 8 + 16;
  static constexpr int THREADS = 192;
  static constexpr uint32_t IDESC =
      instr_desc(kDtype == 0 ? 1u : 0u, kDtype == 0 ? 1u : 0u, /*A K-major*/ 0u, /*B MN-major*/ 1u, BM, BN);

  static_assert(BN % B_CHUNK_N == 0, "BN must be a multiple of one 128-byte row of B");
  static_assert(BN % EPI_COLS == 0, "BN must be a multiple of the epilogue store width");
  static_assert(BN >= 16 && BN <= 256 && BN % 16 == 0, "UMMA N for M=128 is 16..256 in steps of 16");
  static_assert(SMEM_BYTES <= 232448, "shared memory per block exceeds the sm_100 opt-in limit");
};

// Tile order: consecutive tile ids walk down `group_m` M-blocks, then across N, so the CTAs that
// run at the same time share A row panels and B column panels in L2.
__device__ __forceinline__ void tile_coords(int t, const TcParams &p, int &mb, int &nb) {
  const int per_group = p.group_m * p.num_n_blocks;
  const int g = t / per_group;
  const int first_m = g * p.group_m;
  const int rows = min(p.num_m_blocks - first_m, p.group_m);
  const int r = t - g * per_group;
  mb = first_m + r % rows;
  nb = r / rows;
}

// Whether tile (mb, nb) walks k downwards: every other wave of the whole problem's schedule does (tile t of
// the raster order is a worker's (t / workers)-th tile), so each wave starts on the k slabs of its raster
// group's A (and B) panels that the previous wave read last, while they are still in L2.
__device__ __forceinline__ bool tile_k_reversed(const TcParams &p, int mb, int nb, int launch_workers) {
  const int num_m = p.dir_num_m_blocks ? p.dir_num_m_blocks : p.num_m_blocks;
  const int group = p.dir_group_m ? p.dir_group_m : p.group_m;
  const int workers = p.dir_workers ? p.dir_workers : launch_workers;
  const int m = mb + p.dir_m0;
  const int g = m / group, first_m = g * group;
  const int rows = min(num_m - first_m, group);
  const long long t = static_cast<long long>(g) * group * p.num_n_blocks + static_cast<long long>(nb) * rows + (m - first_m);
  return ((t / workers) & 1) != 0;
}

__device__ __forceinline__ float gelu_tanh_fast(float x) {
  // 0.5*x*(1 + tanh(k0*(x + k1*x^3))) with k0 = 0.7978845608028654, k1 = 0.044715.
  const float k0 = 0.7978845608028654f, k0k1 = 0.7978845608028654f * 0.044715f;
  const float x2 = x * x;
  const float u = x * fmaf(k0k1, x2, k0);
  const float hx = 0.5f * x;
  return fmaf(hx, tanh_approx(u), hx);
}

enum : unsigned {
  kErrProducerWait = 1u,
  kErrMmaWait = 2u,
  kErrEpilogueWait = 4u,
  kErrTeardownWait = 8u,
};

struct NoAddend {
  __device__ __forceinline__ void operator()(uint32_t (&)[32], int) const {}
};

// 32 accumulator columns of one row (this lane's) -> x*scale + bias[c], GELU -> 16 packed bf16 pairs.  The
// 32 columns' bias is held one per lane (lane j: column j) and broadcast by shuffles, so it is loaded ahead
// (while the warp waits for the accumulator, or during the previous box), not between TMEM loads and stores.
// Two columns go through each FP32 instruction: sm_100's packed mul / fma (mul.rn.f32x2, fma.rn.f32x2) round
// each half exactly as the scalar mul / fmaf of gelu_tanh_fast, so the bits are those of the scalar form with
// fewer instructions.  kPairAll = false keeps the scale-and-bias step and 0.5*x scalar (their constants are then
// immediates, not register pairs): the choice of the 8-warp epilogue, whose 128 loaded columns leave few
// registers (measured on an epilogue-bound 1,024 x 8,192 x 128 launch: 12.1 -> 11.3 us there, and 13.6 -> 12.8 us
// with kPairAll in the 4-warp epilogue of the 256 x 256 kernel).
template <bool kPairAll = true>
__device__ __forceinline__ void epilogue_math32_lane_bias(const uint32_t (&v)[32], float bias_lane, float scale,
                                                          uint32_t (&packed)[16]) {
  const float2 k0 = make_float2(0.7978845608028654f, 0.7978845608028654f);
  const float2 k0k1 = make_float2(0.7978845608028654f * 0.044715f, 0.7978845608028654f * 0.044715f);
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float b0 = __shfl_sync(0xffffffffu, bias_lane, j), b1 = __shfl_sync(0xffffffffu, bias_lane, j + 1);
    const float v0 = __uint_as_float(v[j]), v1 = __uint_as_float(v[j + 1]);
    float2 x, hx;
    if constexpr (kPairAll) {
      x = __ffma2_rn(make_float2(v0, v1), make_float2(scale, scale), make_float2(b0, b1));
    } else {
      x = make_float2(fmaf(v0, scale, b0), fmaf(v1, scale, b1));
    }
    // gelu_tanh_fast on both: u = x * (k0 + k0 k1 x^2), 0.5 x (1 + tanh u) = fma(0.5 x, tanh u, 0.5 x).
    const float2 u = __fmul2_rn(x, __ffma2_rn(k0k1, __fmul2_rn(x, x), k0));
    if constexpr (kPairAll) {
      hx = __fmul2_rn(make_float2(0.5f, 0.5f), x);
    } else {
      hx = make_float2(0.5f * x.x, 0.5f * x.y);
    }
    const float2 g = __ffma2_rn(hx, make_float2(tanh_approx(u.x), tanh_approx(u.y)), hx);
    packed[j / 2] = pack_bf16x2(g.x, g.y);
  }
}

// This lane's bias of columns col + lane and col + 32 + lane (0 past N): one 64-column box of a tile.
__device__ __forceinline__ float2 lane_bias64(const TcParams &p, int col, int lane) {
  const int c0 = col + lane, c1 = col + 32 + lane;
  return make_float2(c0 < p.N ? __ldg(p.bias + c0) : 0.f, c1 < p.N ? __ldg(p.bias + c1) : 0.f);
}

// One epilogue warp turns its 32 accumulator rows x BN columns (TMEM lanes q*32.., columns from
// `t_row`) into C rows [m0, m0+32) x columns [n_tile, n_tile+BN): x*scale + bias[c], GELU, bf16,
// staged through a double-buffered 32 x 64 swizzled shared-memory box and TMA-stored (`tmC`, 64 x 32
// boxes, 128-byte swizzle).  A BN that is 32 past a multiple of 64 ends with one 32-column box through
// `tmC_tail` (32 x 32 boxes, 64-byte swizzle), so a tile never writes into its neighbour's columns.
// `release()` is called by the whole warp right after the last TMEM load of the tile; `addend(v, c0)`
// may add other fp32 contributions to accumulator columns [c0, c0+32) before the epilogue math.
// The bias travels one per lane (lane_bias64): the caller loads the first box's before the accumulator is
// ready, and each box loads the next one's before its own TMEM loads.
template <int BN, class Release, class Addend = NoAddend>
__device__ __forceinline__ void epilogue_rows(uint32_t t_row, int m0, int n_tile, const TcParams &p,
                                              const CUtensorMap *tmC, const CUtensorMap *tmC_tail, uint8_t *ebuf,
                                              int &buf, int lane, float2 bias_first, Release release,
                                              Addend addend = Addend()) {
  constexpr int EPI_COLS = 64;
  constexpr int BUF_BYTES = 32 * EPI_COLS * 2;
  constexpr int FULL = BN / EPI_COLS;
  constexpr bool TAIL = (BN % EPI_COLS) != 0;
  static_assert(BN % 32 == 0, "the epilogue works in 32-column steps");
  float2 bias_next = bias_first;
#pragma unroll 1
  for (int c = 0; c < FULL; ++c) {
    const uint32_t sbuf = smem_u32(ebuf + buf * BUF_BYTES) + lane * 128;
    const float2 bias_box = bias_next;
    if (c + 1 < FULL || TAIL) bias_next = lane_bias64(p, n_tile + (c + 1) * EPI_COLS, lane);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(t_row + c * EPI_COLS + h * 32, v);
      tmem_ld_wait();
      addend(v, c * EPI_COLS + h * 32);
      uint32_t packed[16];
      epilogue_math32_lane_bias(v, h == 0 ? bias_box.x : bias_box.y, p.scale, packed);
      // Row `lane` of the 32 x 64 box: 16-byte chunk j goes to chunk j ^ (row % 8) (128-B swizzle).
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t chunk = static_cast<uint32_t>((h * 4 + i) ^ (lane & 7));
        st_shared_v4(sbuf + chunk * 16, packed[i * 4 + 0], packed[i * 4 + 1], packed[i * 4 + 2], packed[i * 4 + 3]);
      }
    }
    if (!TAIL && c == FULL - 1) {
      // Last TMEM read of this accumulator: hand it back to the MMA issuer.
      tc_fence_before();
      __syncwarp();
      release();
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      // A box wholly right of C (a 512-wide tile's columns past a ragged N) stores nothing.
      if (n_tile + c * EPI_COLS < p.N) tma_store_2d(tmC, ebuf + buf * BUF_BYTES, n_tile + c * EPI_COLS, m0);
      tma_store_commit();
      tma_store_wait_read<1>();  // the other buffer is free again
    }
    __syncwarp();
    buf ^= 1;
  }
  if constexpr (TAIL) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(t_row + FULL * EPI_COLS, v);
    tmem_ld_wait();
    tc_fence_before();
    __syncwarp();
    release();
    addend(v, FULL * EPI_COLS);
    uint32_t packed[16];
    epilogue_math32_lane_bias(v, bias_next.x, p.scale, packed);
    // Row `lane` of the 32 x 32 box is 64 bytes; under the 64-byte swizzle its 16-byte chunk i lands at
    // chunk i ^ ((row / 2) % 4), which also spreads a quarter-warp's stores over all eight bank groups.
    const uint32_t sbuf = smem_u32(ebuf + buf * BUF_BYTES) + lane * 64;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t chunk = static_cast<uint32_t>(i ^ ((lane >> 1) & 3));
      st_shared_v4(sbuf + chunk * 16, packed[i * 4 + 0], packed[i * 4 + 1], packed[i * 4 + 2], packed[i * 4 + 3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmC_tail, ebuf + buf * BUF_BYTES, n_tile + FULL * EPI_COLS, m0);
      tma_store_commit();
      tma_store_wait_read<1>();
    }
    __syncwarp();
    buf ^= 1;
  }
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
    gemm_bias_gelu_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmC, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzled tiles need 1024-byte aligned shared addresses.
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);

  uint8_t *sA = smem;
  uint8_t *sB = smem + Cfg::STAGES * Cfg::A_BYTES;
  uint8_t *sEpi = smem + Cfg::STAGES * Cfg::STAGE_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sEpi + Cfg::EPI_BYTES);
  uint64_t *full = bars;                        // [STAGES] TMA bytes landed
  uint64_t *empty = bars + Cfg::STAGES;         // [STAGES] MMAs reading the stage finished
  uint64_t *tfull = bars + 2 * Cfg::STAGES;     // [2] accumulator ready for the epilogue
  uint64_t *tempty = tfull + 2;                 // [2] accumulator drained by the epilogue
  uint64_t *drain = tempty + 2;                 // [1] teardown: all MMAs complete
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], Cfg::EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
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
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool dep_waited = false;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, p, mb, nb);
        const bool reversed = tile_k_reversed(p, mb, nb, gridDim.x);
        for (int i = 0; i < p.k_blocks; ++i) {
          const int kb = reversed ? p.k_blocks - 1 - i : i;
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.timeout_ns, abort_flag)) {
            fail(kErrProducerWait);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          if (!dep_waited) {
            grid_dependency_wait();
            dep_waited = true;
          }
#pragma unroll
          for (int a = 0; a < Cfg::KATOMS; ++a)
            tma_load_2d(sA + stage * Cfg::A_BYTES + a * Cfg::A_ATOM_BYTES, &tmA, &full[stage],
                        kb * Cfg::BK + a * Cfg::ATOM_K, mb * Cfg::BM);
          uint8_t *b_dst = sB + stage * Cfg::B_BYTES;
#pragma unroll
          for (int j = 0; j < Cfg::B_CHUNKS; ++j)
            tma_load_2d(b_dst + j * Cfg::B_CHUNK_BYTES, &tmB, &full[stage], nb * Cfg::BN + j * Cfg::B_CHUNK_N,
                        kb * Cfg::BK);
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Loads already issued must land before the block may exit: wait for each stage's last
        // issued phase (bounded; the stage that failed was never issued).
        for (int s = 0; s < Cfg::STAGES; ++s) {
          // stage s was last issued in phase (phase if s < stage else phase^1) -- only if issued.
          const uint32_t ph = (s < stage) ? phase : (phase ^ 1u);
          volatile int no_abort = 0;
          if (!mbar_wait(&full[s], ph, p.timeout_ns, &no_abort)) atomicOr(p.status, kErrTeardownWait);
        }
      }
    }
    grid_launch_dependents();  // this CTA's loads are all issued
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.timeout_ns, abort_flag)) {
          fail(kErrMmaWait);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Cfg::BN);
        for (int i = 0; i < p.k_blocks; ++i) {
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
            // A: K-major, 128-B swizzle; k advances 32 bytes inside a swizzle row, then to the next atom.
            constexpr int PER_ATOM = Cfg::ATOM_K / Cfg::UMMA_K;
            const uint64_t ad =
                smem_desc(a_addr + (k / PER_ATOM) * Cfg::A_ATOM_BYTES + (k % PER_ATOM) * 32, 16, 1024, kSwizzle128B);
            // B: N-major, 128-B swizzle; k advances UMMA_K rows of 128 B; LBO = next 128-B column chunk.
            const uint64_t bd = smem_desc(b_addr + k * Cfg::UMMA_K * 128, Cfg::B_CHUNK_BYTES, 1024, kSwizzle128B);
            if constexpr (Cfg::ELEM == 2)
              tc_mma_f16(d_tmem, ad, bd, Cfg::IDESC, (i | k) != 0);
            else
              tc_mma_f8(d_tmem, ad, bd, Cfg::IDESC, (i | k) != 0);
          }
          tc_commit(&empty[stage]);
          if (++stage == Cfg::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA issued must complete before TMEM is released.
      tc_commit(drain);
      volatile int no_abort = 0;
      if (!mbar_wait(drain, 0, p.timeout_ns, &no_abort)) atomicOr(p.status, kErrTeardownWait);
    }
    grid_launch_dependents();  // this CTA's MMAs are all issued and complete
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    grid_launch_dependents();  // a dependent launch waits for the producer and MMA warps, which signal last
    grid_dependency_wait();
    const int q = warp & 3;                  // TMEM lane quarter this warp may access
    const int ew = warp - 2;
    uint8_t *ebuf = sEpi + ew * Cfg::EPI_BUFS * Cfg::EPI_BUF_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    int buf = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, p, mb, nb);
      const float2 bias_first = lane_bias64(p, nb * Cfg::BN, lane);  // loaded while the accumulator fills
      // The TMEM loads below are warp-collective (.sync.aligned): the whole warp proceeds or leaves.
      const bool waited = mbar_wait(&tfull[acc], acc_phase, p.timeout_ns, abort_flag);
      if (!__all_sync(0xffffffffu, waited)) {
        if (lane == 0) fail(kErrEpilogueWait);
        break;
      }
      tc_fence_after();
      const int m0 = mb * Cfg::BM + q * 32;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * Cfg::BN);
      uint64_t *tempty_acc = &tempty[acc];
      epilogue_rows<Cfg::BN>(t_row, m0, nb * Cfg::BN, p, &tmC, nullptr, ebuf, buf, lane, bias_first, [&] {
        if (lane == 0) mbar_arrive(tempty_acc);
      });
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) tma_store_wait_all<0>();
    __syncwarp();
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace pf
