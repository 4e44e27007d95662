// pf_b200.cu -- the C ABI declared in include/pf_b200.h.
//
// One pf_ctx per (host thread, GPU).  pf_prepare picks a kernel variant for (dtype, tile, M, N, K),
// pf_bind records caller-owned device operands and encodes the TMA tensor maps, pf_launch launches,
// pf_time applies the reference timing protocol (core/src/cuda_runner.cpp:110-130).
//
// The CUDA driver is reached only through the runtime (cudaGetDriverEntryPoint for
// cuTensorMapEncodeTiled), so the library loads on a machine without a GPU driver; every entry
// point then reports PF_ENODEV instead of failing to load.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "pf_b200.h"
#include "gemm_simt.cuh"
#include "gemm_simt_tma.cuh"
#include "gemm_tc.cuh"
#include "gemm_tc2.cuh"
#include "gemm_tc2w.cuh"
#include "gemm_tf32x3.cuh"

#ifndef PF_VERSION_STR
#define PF_VERSION_STR "0.1.0"
#endif

namespace {

using pf::TcConfig;
using pf::TcParams;

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

enum class Path { kNone, kSimt, kTensor, kImage };

// Launch description of one compiled variant.
struct Variant {
  Path path = Path::kNone;
  const void *func = nullptr;  // kernel symbol (for attributes / occupancy)
  int threads = 0;
  int smem = 0;                // dynamic shared memory
  // tensor path
  int bm = 0, bn = 0, bk_elems = 0, stages = 0, elem = 0;
  int a_box_rows = 0;           // rows of A per TMA box (the CTA's share of BM)
  int a_box_k = 0;              // k elements per TMA box of A (one 128-byte swizzle row)
  int katoms = 1;               // 128-byte k-atoms per pipeline stage
  int cta_per_tile = 1;         // 2 = CTA-pair (cluster) kernel
  bool stream_k = false;        // the kernel can run a stream-K tail
  // Auto stream-K (pf_set_stream_k -1): at least this many waves of tiles (with a partial last one), or whole
  // tiles keeping fewer than this fraction of the workers busy; and at least this many of the leftover tiles'
  // k-blocks per worker.
  double sk_min_waves = 3.0;
  double sk_low_util = 0.0;
  int sk_min_share = 1;
  bool sk_band = false;         // the kernel can run row-band stream-K (p.sk_band_workers)
  int partial_cols = 256;       // fp32 columns of one CTA's stream-K partial (x 128 rows)
  int b_chunk_n = 0;
  // (grid, stream, A map, B map, C map, C tail map -- used by tiles whose width is not a multiple of 64)
  void (*launch_tc)(dim3, cudaStream_t, const CUtensorMap &, const CUtensorMap &, const CUtensorMap &, const CUtensorMap &,
                    const TcParams &) = nullptr;
  // image path (pf_prepare_image): a loaded kernel with the reference ABI
  CUfunction img_fn = nullptr;
  int img_gx = 0, img_gy = 0;
  // simt path
  int sbm = 0, sbn = 0;
  void (*launch_simt)(dim3, cudaStream_t, const float *, const float *, const float *, float *, int, int, int,
                      bool vec) = nullptr;
  // simt path fed by TMA (gemm_simt_tma.cuh), where the operands allow it: kernel, its dynamic shared memory,
  // BK, and launcher (grid, stream, A map, B map, bias, C, M, N, K, status word, wait bound)
  const void *tma_func = nullptr;
  int tma_smem = 0, tma_bk = 0;
  void (*launch_simt_tma)(dim3, cudaStream_t, const CUtensorMap &, const CUtensorMap &, const float *, float *, int,
                          int, int, unsigned *, unsigned long long) = nullptr;
};

// Programmatic dependent launch for the tensor-core kernels: each launch may be scheduled while the previous
// kernel in the stream finishes; the kernel sets up its barriers and TMEM, then waits (griddepcontrol.wait)
// for that kernel's completion before any global memory access, so the result is the same as a plain launch.
// PF_PDL=0 in the environment turns it off (plain launches).
bool pdl_enabled() {
  static const bool on = [] {
    const char *e = std::getenv("PF_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Tail split of the 256 x 512 pair kernel (TcParams::tail_split): k steps at the end of each pair's last tile
// whose second-half MMAs run after the first half's, so that the first half's epilogue overlaps them.
// PF_TAIL_SPLIT=<steps> in the environment overrides the default (0 turns it off).
int tail_split_steps() {
  static const int steps = [] {
    const char *e = std::getenv("PF_TAIL_SPLIT");
    return e ? std::max(0, std::atoi(e)) : 8;
  }();
  return steps;
}

// Periodic promotion of the 3xTF32 kernel (TcParams::promote_kb): k-blocks (32 k each) per chunk of tensor-core
// accumulation before the epilogue adds the chunk, round to nearest, into an fp32 running sum.  Measured on the
// reference runner's U(-0.5, 0.5) inputs, 1024^2 x K, max |ref - C| / (1 + |ref|) against fp64 at K = 512 / 1024 /
// 2048 / 4096: off 1.1e-5 / 6.9e-6 / 2.0e-5 / 5.0e-5; 8 k-blocks 6.2e-6 / 6.9e-6 / 1.2e-5 / 1.3e-5; 4 k-blocks (the
// default) 3.6e-6 / 4.1e-6 / 6.0e-6 / 8.6e-6 -- inside 1e-5 and below the fp32 fmaf chain's own 1.2e-5 / 1.8e-5
// at 2048 / 4096.  The running sums cost L2 bandwidth: 2048^3 184 (off) / 159 (8) / 144 (4) TFLOP/s.
// PF_PROMOTE_KB=<k-blocks> in the environment overrides the default (0 turns it off).
int promote_kb_default() {
  static const int kb = [] {
    const char *e = std::getenv("PF_PROMOTE_KB");
    return e ? std::max(0, std::atoi(e)) : 4;
  }();
  return kb;
}

template <class... Params, class... Args>
void launch_pdl(void (*kernel)(Params...), dim3 grid, int threads, int smem, cudaStream_t s, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  cfg.numAttrs = 0;
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  cfg.attrs = attr;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);  // errors surface through cudaGetLastError
}

template <int DT, int BN, int ST, int KA>
void launch_tc_impl(dim3 grid, cudaStream_t s, const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &c,
                    const CUtensorMap &,
                    const TcParams &p) {
  using Cfg = TcConfig<DT, BN, ST, KA>;
  launch_pdl(&pf::gemm_bias_gelu_tc<Cfg>, grid, Cfg::THREADS, Cfg::SMEM_BYTES, s, a, b, c, p);
}

template <int DT, int BN, int ST, int KA = 1>
Variant make_tc_variant() {
  using Cfg = TcConfig<DT, BN, ST, KA>;
  Variant v;
  v.path = Path::kTensor;
  v.func = reinterpret_cast<const void *>(&pf::gemm_bias_gelu_tc<Cfg>);
  v.threads = Cfg::THREADS;
  v.smem = Cfg::SMEM_BYTES;
  v.bm = Cfg::BM;
  v.bn = Cfg::BN;
  v.bk_elems = Cfg::BK;
  v.stages = Cfg::STAGES;
  v.elem = Cfg::ELEM;
  v.b_chunk_n = Cfg::B_CHUNK_N;
  v.a_box_rows = Cfg::BM;
  v.a_box_k = Cfg::ATOM_K;
  v.katoms = Cfg::KATOMS;
  v.cta_per_tile = 1;
  v.launch_tc = &launch_tc_impl<DT, BN, ST, KA>;
  return v;
}

template <int DT, int ST, int KA, int BN>
void launch_tc2_impl(dim3 grid, cudaStream_t s, const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &c,
                     const CUtensorMap &ct, const TcParams &p) {
  using Cfg = pf::Tc2Config<DT, ST, KA, BN>;
  launch_pdl(&pf::gemm_bias_gelu_tc2<Cfg>, grid, Cfg::THREADS, Cfg::SMEM_BYTES, s, a, b, c, ct, p);
}

template <int DT, int ST, int KA = 1, int BN = 256>
Variant make_tc2_variant() {
  using Cfg = pf::Tc2Config<DT, ST, KA, BN>;
  Variant v;
  v.path = Path::kTensor;
  v.func = reinterpret_cast<const void *>(&pf::gemm_bias_gelu_tc2<Cfg>);
  v.threads = Cfg::THREADS;
  v.smem = Cfg::SMEM_BYTES;
  v.bm = Cfg::BM;
  v.bn = Cfg::BN;
  v.bk_elems = Cfg::BK;
  v.stages = Cfg::STAGES;
  v.elem = Cfg::ELEM;
  v.b_chunk_n = Cfg::B_CHUNK_N;
  v.a_box_rows = Cfg::BM_CTA;
  v.a_box_k = Cfg::ATOM_K;
  v.katoms = Cfg::KATOMS;
  v.cta_per_tile = 2;
  v.stream_k = true;
  v.sk_band = BN % 64 == 0;  // row-band stream-K on 256-wide tiles (partials fold 64 columns at a time)
  v.launch_tc = &launch_tc2_impl<DT, ST, KA, BN>;
  return v;
}

template <int DT, int ST, int EW, int EB = 2>
void launch_tc2w_impl(dim3 grid, cudaStream_t s, const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &c,
                      const CUtensorMap &, const TcParams &p) {
  using Cfg = pf::Tc2wConfig<DT, ST, EW, EB>;
  launch_pdl(&pf::gemm_bias_gelu_tc2w<Cfg>, grid, Cfg::THREADS, Cfg::SMEM_BYTES, s, a, b, c, p);
}

// CTA pairs with 256 x 512 tiles (gemm_tc2w.cuh): whole tiles, one k-atom per stage.
template <int DT, int ST, int EW, int EB = 2>
Variant make_tc2w_variant() {
  using Cfg = pf::Tc2wConfig<DT, ST, EW, EB>;
  Variant v;
  v.path = Path::kTensor;
  v.func = reinterpret_cast<const void *>(&pf::gemm_bias_gelu_tc2w<Cfg>);
  v.threads = Cfg::THREADS;
  v.smem = Cfg::SMEM_BYTES;
  v.bm = Cfg::BM;
  v.bn = Cfg::BN;
  v.bk_elems = Cfg::BK;
  v.stages = Cfg::STAGES;
  v.elem = Cfg::ELEM;
  v.b_chunk_n = Cfg::B_CHUNK_N;
  v.a_box_rows = Cfg::BM_CTA;
  v.a_box_k = Cfg::ATOM_K;
  v.katoms = Cfg::KATOMS;
  v.cta_per_tile = 2;
  v.sk_band = true;
  v.partial_cols = Cfg::BN;
  v.launch_tc = &launch_tc2w_impl<DT, ST, EW, EB>;
  return v;
}

template <int RAW, int SPLIT>
void launch_tf32x3_impl(dim3 grid, cudaStream_t s, const CUtensorMap &a, const CUtensorMap &b, const CUtensorMap &c,
                        const CUtensorMap &,
                        const TcParams &p) {
  using Cfg = pf::Tf32x3Config<RAW, SPLIT>;
  launch_pdl(&pf::gemm_bias_gelu_tf32x3<Cfg>, grid, Cfg::THREADS, Cfg::SMEM_BYTES, s, a, b, c, p);
}

// 3xTF32: depth = raw TMA slots + split (hi / lo) slots.
template <int RAW, int SPLIT>
Variant make_tf32x3_variant() {
  using Cfg = pf::Tf32x3Config<RAW, SPLIT>;
  Variant v;
  v.path = Path::kTensor;
  v.func = reinterpret_cast<const void *>(&pf::gemm_bias_gelu_tf32x3<Cfg>);
  v.threads = Cfg::THREADS;
  v.smem = Cfg::SMEM_BYTES;
  v.bm = Cfg::BM;
  v.bn = Cfg::BN;
  v.bk_elems = Cfg::BK;
  v.stages = Cfg::STAGES;
  v.elem = Cfg::ELEM;
  v.b_chunk_n = Cfg::B_CHUNK_N;
  v.a_box_rows = Cfg::BM_CTA;
  v.a_box_k = Cfg::ATOM_K;
  v.katoms = 1;
  v.cta_per_tile = 2;
  // Below 3 waves the tail pays once whole tiles would leave a quarter of the pairs idle: measured (us, off ->
  // on) 16 tiles 86.3 -> 50.1, 32 tiles 86.5 -> 60.5, 36 tiles 76.2 -> 60.6, but 64 tiles 87.6 -> 89.9 (the
  // partial writes, the head's wait and its reads cost ~12 us per launch).
  v.stream_k = true;
  v.sk_low_util = 0.75;
  v.sk_min_share = 4;
  v.launch_tc = &launch_tf32x3_impl<RAW, SPLIT>;
  return v;
}

template <int BM, int BN, int BK, int TM, int TN, int PAD>
void launch_simt_impl(dim3 grid, cudaStream_t s, const float *A, const float *B, const float *bias, float *C, int M,
                      int N, int K, bool vec) {
  using Cfg = pf::SimtConfig<BM, BN, BK, TM, TN, PAD>;
  if (vec)
    pf::gemm_bias_gelu_simt<BM, BN, BK, TM, TN, PAD, true><<<grid, Cfg::THREADS, 0, s>>>(A, B, bias, C, M, N, K);
  else
    pf::gemm_bias_gelu_simt<BM, BN, BK, TM, TN, PAD, false><<<grid, Cfg::THREADS, 0, s>>>(A, B, bias, C, M, N, K);
}

template <int BM, int BN, int BK, int TM, int TN, int PAD>
Variant make_simt_variant() {
  using Cfg = pf::SimtConfig<BM, BN, BK, TM, TN, PAD>;
  Variant v;
  v.path = Path::kSimt;
  v.func = reinterpret_cast<const void *>(&pf::gemm_bias_gelu_simt<BM, BN, BK, TM, TN, PAD, true>);
  v.threads = Cfg::THREADS;
  v.smem = 0;
  v.sbm = BM;
  v.sbn = BN;
  v.launch_simt = &launch_simt_impl<BM, BN, BK, TM, TN, PAD>;
  return v;
}

template <int BM, int BN, int BK, int TM, int TN, int STAGES>
void launch_simt_tma_impl(dim3 grid, cudaStream_t s, const CUtensorMap &a, const CUtensorMap &b, const float *bias,
                          float *C, int M, int N, int K, unsigned *status, unsigned long long timeout_ns) {
  using Cfg = pf::SimtTmaConfig<BM, BN, BK, TM, TN, STAGES>;
  pf::gemm_bias_gelu_simt_tma<BM, BN, BK, TM, TN, STAGES>
      <<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, s>>>(a, b, bias, C, M, N, K, status, timeout_ns);
}

// The TMA-fed SIMT kernel for a tile, with the cp.async kernel of the same tile for operands TMA cannot
// address (rows not 16-byte multiples, unaligned pointers) and for row-window launches; both give the same
// bits.
template <int BM, int BN, int BK, int TM, int TN, int PAD, int STAGES>
Variant make_simt_tma_variant() {
  using Cfg = pf::SimtTmaConfig<BM, BN, BK, TM, TN, STAGES>;
  Variant v = make_simt_variant<BM, BN, BK, TM, TN, PAD>();
  v.tma_func = reinterpret_cast<const void *>(&pf::gemm_bias_gelu_simt_tma<BM, BN, BK, TM, TN, STAGES>);
  v.tma_smem = Cfg::SMEM_BYTES;
  v.tma_bk = BK;
  v.launch_simt_tma = &launch_simt_tma_impl<BM, BN, BK, TM, TN, STAGES>;
  return v;
}

struct SimtEntry {
  pf_tile tile;
  Variant (*make)();
};

// fp32 tile configs compiled into the library (the reference compiles one per trial with nvcc -D).
const SimtEntry kSimtTable[] = {
    {{128, 128, 8, 8, 8, 4}, &make_simt_variant<128, 128, 8, 8, 8, 4>},
    {{128, 128, 8, 8, 8, 0}, &make_simt_variant<128, 128, 8, 8, 8, 0>},
    {{128, 128, 16, 8, 8, 4}, &make_simt_variant<128, 128, 16, 8, 8, 4>},
    {{128, 64, 8, 8, 4, 4}, &make_simt_variant<128, 64, 8, 8, 4, 4>},
    {{64, 128, 8, 4, 8, 4}, &make_simt_variant<64, 128, 8, 4, 8, 4>},
    {{64, 64, 8, 4, 4, 0}, &make_simt_variant<64, 64, 8, 4, 4, 0>},
    {{64, 64, 8, 4, 4, 4}, &make_simt_variant<64, 64, 8, 4, 4, 4>},
    {{64, 64, 16, 4, 4, 4}, &make_simt_variant<64, 64, 16, 4, 4, 4>},
    {{32, 64, 8, 2, 4, 4}, &make_simt_variant<32, 64, 8, 2, 4, 4>},
    {{32, 32, 8, 2, 2, 0}, &make_simt_variant<32, 32, 8, 2, 2, 0>},
    // small problems (fewer 128 x 128 tiles than SMs): the best of a 160-trial tune at 512^3 on B200
    {{32, 32, 32, 4, 2, 2}, &make_simt_variant<32, 32, 32, 4, 2, 2>},
    {{64, 32, 32, 4, 2, 2}, &make_simt_variant<64, 32, 32, 4, 2, 2>},
    {{32, 64, 32, 4, 2, 2}, &make_simt_variant<32, 64, 32, 4, 2, 2>},
    // 64-thread CTAs with 8 x 8 micro-tiles: eight share an SM at 128 registers, so small block tiles fill
    // the SMs evenly (2048^2 outputs: 1,024 tiles of 64 x 64 for 148 x 8 slots)
    {{64, 64, 8, 8, 8, 4}, &make_simt_variant<64, 64, 8, 8, 8, 4>},
    {{64, 64, 16, 8, 8, 4}, &make_simt_variant<64, 64, 16, 8, 8, 4>},
    {{128, 64, 8, 8, 8, 4}, &make_simt_variant<128, 64, 8, 8, 8, 4>},
    {{64, 128, 8, 8, 8, 4}, &make_simt_variant<64, 128, 8, 8, 8, 4>},
    {{64, 32, 8, 8, 4, 4}, &make_simt_variant<64, 32, 8, 8, 4, 4>},
    {{32, 64, 8, 4, 8, 4}, &make_simt_variant<32, 64, 8, 4, 8, 4>},
    {{32, 32, 8, 4, 4, 4}, &make_simt_variant<32, 32, 8, 4, 4, 4>},
    {{32, 32, 16, 4, 4, 4}, &make_simt_variant<32, 32, 16, 4, 4, 4>},
    {{32, 32, 32, 4, 4, 4}, &make_simt_variant<32, 32, 32, 4, 4, 4>},
    // TMA-fed (gemm_simt_tma.cuh; PAD 0: A is not transposed, the TMA swizzle spreads its reads over the banks).
    // The ring depth fits the shared memory a CTA gets at its register-limited occupancy.
    {{64, 64, 16, 8, 8, 0}, &make_simt_tma_variant<64, 64, 16, 8, 8, 0, 3>},
    {{64, 64, 32, 8, 8, 0}, &make_simt_tma_variant<64, 64, 32, 8, 8, 0, 2>},
    {{128, 128, 16, 8, 8, 0}, &make_simt_tma_variant<128, 128, 16, 8, 8, 0, 4>},
    {{128, 64, 16, 8, 8, 0}, &make_simt_tma_variant<128, 64, 16, 8, 8, 0, 4>},
    {{64, 128, 16, 8, 8, 0}, &make_simt_tma_variant<64, 128, 16, 8, 8, 0, 4>},
    {{64, 32, 16, 8, 4, 0}, &make_simt_tma_variant<64, 32, 16, 8, 4, 0, 3>},
    {{32, 64, 16, 4, 8, 0}, &make_simt_tma_variant<32, 64, 16, 4, 8, 0, 3>},
    {{32, 32, 16, 4, 4, 0}, &make_simt_tma_variant<32, 32, 16, 4, 4, 0, 6>},
};

bool same_tile(const pf_tile &a, const pf_tile &b) {
  return a.BM == b.BM && a.BN == b.BN && a.BK == b.BK && a.TM == b.TM && a.TN == b.TN && a.PAD == b.PAD;
}

// Tensor-path variant for (dtype, BM, BN, requested pipeline depth TM, k-atoms per stage).  The depth is
// clamped to the deepest compiled variant that fits in shared memory (TM=8 asks for "as deep as fits").
bool find_tc_variant(pf_dtype dt, int bm, int bn, int depth, int katoms, Variant *out) {
  struct Entry {
    int dt, bm, bn, stages, katoms;
    Variant (*make)();
  };
  static const Entry table[] = {
      {PF_BF16, 128, 256, 2, 1, &make_tc_variant<0, 256, 2>},     {PF_BF16, 128, 256, 4, 1, &make_tc_variant<0, 256, 4>},
      {PF_BF16, 128, 256, 2, 2, &make_tc_variant<0, 256, 2, 2>},  {PF_BF16, 128, 128, 2, 1, &make_tc_variant<0, 128, 2>},
      {PF_BF16, 128, 128, 4, 1, &make_tc_variant<0, 128, 4>},     {PF_BF16, 128, 128, 6, 1, &make_tc_variant<0, 128, 6>},
      {PF_BF16, 128, 128, 3, 2, &make_tc_variant<0, 128, 3, 2>},  {PF_BF16, 128, 64, 4, 1, &make_tc_variant<0, 64, 4>},
      {PF_BF16, 128, 64, 8, 1, &make_tc_variant<0, 64, 8>},       {PF_BF16, 256, 256, 2, 1, &make_tc2_variant<0, 2>},
      {PF_BF16, 256, 256, 4, 1, &make_tc2_variant<0, 4>},         {PF_BF16, 256, 256, 6, 1, &make_tc2_variant<0, 6>},
      {PF_BF16, 256, 256, 3, 2, &make_tc2_variant<0, 3, 2>},      {PF_E4M3, 128, 256, 2, 1, &make_tc_variant<1, 256, 2>},
      {PF_E4M3, 128, 256, 4, 1, &make_tc_variant<1, 256, 4>},     {PF_E4M3, 128, 256, 2, 2, &make_tc_variant<1, 256, 2, 2>},
      {PF_E4M3, 128, 128, 2, 1, &make_tc_variant<1, 128, 2>},     {PF_E4M3, 128, 128, 4, 1, &make_tc_variant<1, 128, 4>},
      {PF_E4M3, 128, 128, 6, 1, &make_tc_variant<1, 128, 6>},     {PF_E4M3, 256, 256, 2, 1, &make_tc2_variant<1, 2>},
      {PF_E4M3, 256, 256, 4, 1, &make_tc2_variant<1, 4>},         {PF_E4M3, 256, 256, 6, 1, &make_tc2_variant<1, 6>},
      {PF_E4M3, 256, 256, 3, 2, &make_tc2_variant<1, 3, 2>},
      {PF_BF16, 256, 224, 3, 2, &make_tc2_variant<0, 3, 2, 224>}, {PF_E4M3, 256, 224, 3, 2, &make_tc2_variant<1, 3, 2, 224>},
      // 256 x 512, 8 epilogue warps: 3 stages with two staging boxes per warp, or 4 stages with one (shared memory
      // holds one or the other; measured, bursts of 20: 8192^3 685.0 / 686.4 us, 1,024-row shards 97.6 / 96.2 us)
      {PF_BF16, 256, 512, 3, 1, &make_tc2w_variant<0, 3, 8>},      {PF_E4M3, 256, 512, 3, 1, &make_tc2w_variant<1, 3, 8>},
      {PF_BF16, 256, 512, 4, 1, &make_tc2w_variant<0, 4, 8, 1>},   {PF_E4M3, 256, 512, 4, 1, &make_tc2w_variant<1, 4, 8, 1>},
      {PF_F32_3XTF32, 256, 256, 2, 1, &make_tf32x3_variant<1, 1>},
      {PF_F32_3XTF32, 256, 256, 3, 1, &make_tf32x3_variant<1, 2>},
      {PF_F32_3XTF32, 256, 256, 4, 1, &make_tf32x3_variant<2, 2>},
  };
  const Entry *best = nullptr;
  for (const Entry &e : table)
    if (e.dt == dt && e.bm == bm && e.bn == bn && e.katoms == katoms && e.stages <= depth &&
        (!best || e.stages > best->stages))
      best = &e;
  if (!best) return false;
  *out = best->make();
  return true;
}

// Driver entry points of the image path, fetched through the runtime (no link-time libcuda).
struct DriverApi {
  CUresult (*moduleLoadData)(CUmodule *, const void *) = nullptr;
  CUresult (*moduleUnload)(CUmodule) = nullptr;
  CUresult (*moduleGetFunction)(CUfunction *, CUmodule, const char *) = nullptr;
  CUresult (*launchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream,
                           void **, void **) = nullptr;
  CUresult (*funcGetAttribute)(int *, CUfunction_attribute, CUfunction) = nullptr;
  CUresult (*occupancy)(int *, CUfunction, int, size_t) = nullptr;
  CUresult (*getErrorString)(CUresult, const char **) = nullptr;
  bool ok = false;
};

const DriverApi &driver_api() {
  static DriverApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char *name, void **fn) {
      cudaDriverEntryPointQueryResult q;
      return cudaGetDriverEntryPointByVersion(name, fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
             q == cudaDriverEntryPointSuccess;
    };
    api.ok = get("cuModuleLoadData", reinterpret_cast<void **>(&api.moduleLoadData)) &&
             get("cuModuleUnload", reinterpret_cast<void **>(&api.moduleUnload)) &&
             get("cuModuleGetFunction", reinterpret_cast<void **>(&api.moduleGetFunction)) &&
             get("cuLaunchKernel", reinterpret_cast<void **>(&api.launchKernel)) &&
             get("cuFuncGetAttribute", reinterpret_cast<void **>(&api.funcGetAttribute)) &&
             get("cuOccupancyMaxActiveBlocksPerMultiprocessor", reinterpret_cast<void **>(&api.occupancy)) &&
             get("cuGetErrorString", reinterpret_cast<void **>(&api.getErrorString));
  });
  return api;
}

const char *cu_err(CUresult r) {
  const char *s = nullptr;
  if (driver_api().getErrorString) driver_api().getErrorString(r, &s);
  return s ? s : "unknown CUDA driver error";
}

// The driver's cuTensorMapEncodeTiled.  A function-local static is initialised exactly once, and threads
// whose first calls race all wait for that one initialisation (C++11 guarantees it), so none can see a
// half-initialised value.
EncodeTiledFn get_encode_fn() {
  static const EncodeTiledFn fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    return static_cast<EncodeTiledFn>(nullptr);
  }();
  return fn;
}

}  // namespace

struct pf_ctx {
  int device = -1;
  int num_sms = 0;
  cudaStream_t stream = nullptr;
  unsigned *d_status = nullptr;
  unsigned long long timeout_ns = 4000000000ull;
  std::string err;

  bool prepared = false, bound = false;
  pf_dtype dtype = PF_F32;
  pf_tile tile{};
  int M = 0, N = 0, K = 0;
  Variant var;
  int group_m = 16;
  int max_units = 0;  // persistent grid: co-resident CTAs (1-CTA) or CTA pairs (2-CTA)

  const void *A = nullptr, *B = nullptr;
  const float *bias = nullptr;
  void *C = nullptr;
  float sa = 1.f, sb = 1.f;
  CUtensorMap tmA{}, tmB{}, tmC{}, tmCt{};  // tmCt: 32-column C boxes for the last columns of 224-wide tiles
  bool simt_vec = false;
  bool simt_tma = false;  // the bound fp32 operands go through the TMA-fed kernel (maps in tmA / tmB)
  CUmodule module = nullptr;  // image loaded by pf_prepare_image

  // cuBLAS comparator state (pf_time_cublas): handle, workspace, GEMM output, transposed fp8 B, scales
  void *lt_handle = nullptr, *lt_ws = nullptr, *lt_D = nullptr, *lt_Bt = nullptr;
  float *lt_scales = nullptr;
  size_t lt_ws_cap = 0, lt_D_cap = 0, lt_Bt_cap = 0;

  // pf_run_host buffers
  void *hbufA = nullptr, *hbufB = nullptr, *hbufC = nullptr;
  float *hbufBias = nullptr;
  size_t capA = 0, capB = 0, capC = 0, capBias = 0;

  cudaEvent_t ev0 = nullptr, ev1 = nullptr;

  // stream-K tail of the CTA-pair kernel: mode (-1 auto, 0 off, 1 on), launch epoch, workspace, flags
  int stream_k = -1;
  int host_chunks = 0;   // pf_set_host_chunks: 0 = default
  unsigned epoch = 0;
  float *sk_ws = nullptr;
  float *promo_ws = nullptr;  // 3xTF32 periodic promotion: running sums, [pairs][2 CTAs][128 x 256] fp32
  size_t promo_ws_cap = 0;
  unsigned *sk_flags = nullptr;
  size_t sk_ws_cap = 0, sk_flags_cap = 0;

  // pf_run_host pipeline: compute and device-to-host streams, and per-chunk ordering events
  cudaStream_t s_comp = nullptr, s_out = nullptr;
  std::vector<cudaEvent_t> ev_pool;
};

namespace {

int set_err(pf_ctx *c, int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  return code;
}

#define PF_CUDA(ctx, call)                                                                               \
  do {                                                                                                   \
    cudaError_t _e = (call);                                                                             \
    if (_e != cudaSuccess) return set_err(ctx, PF_ECUDA, "%s -> %s", #call, cudaGetErrorString(_e));    \
  } while (0)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// A 2-D tiled TMA map; on failure a message goes to msg[0..len) (no heap: the no-allocation entry point
// uses it too).
int encode_2d_msg(char *msg, size_t len, CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t inner,
                  uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) {
    if (msg && len) snprintf(msg, len, "cuTensorMapEncodeTiled unavailable from the CUDA driver");
    return PF_ECUDA;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (msg && len)
      snprintf(msg, len, "cuTensorMapEncodeTiled failed (%d) for a %llux%llu tensor, box %ux%u", (int)r,
               (unsigned long long)outer, (unsigned long long)inner, box_outer, box_inner);
    return PF_ECUDA;
  }
  return PF_OK;
}

int encode_2d(pf_ctx *c, CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  char msg[200];
  const int rc = encode_2d_msg(msg, sizeof msg, map, dt, base, inner, outer, row_bytes, box_inner, box_outer, swz);
  return rc ? set_err(c, rc, "%s", msg) : PF_OK;
}

// Element types of the tensor path's TMA maps: A and B in the dtype's encoding; C is bf16 except on the
// 3xTF32 path (fp32).  A C box is one 128-byte row of columns by 32 rows (one epilogue warp).
CUtensorMapDataType in_map_type(pf_dtype dt) {
  return dt == PF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                       : dt == PF_E4M3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
}
CUtensorMapDataType out_map_type(pf_dtype dt) {
  return dt == PF_F32_3XTF32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

int encode_c_map(pf_ctx *c, CUtensorMap *map, void *C, int rows) {
  const uint64_t o = pf_out_bytes(c->dtype);
  return encode_2d(c, map, out_map_type(c->dtype), C, c->N, rows, c->N * o, static_cast<uint32_t>(128 / o), 32,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

// The C map for a tile's last 32 columns when its width is not a multiple of 64 (bf16 C: 64-byte rows,
// 64-byte swizzle); otherwise a copy of the main C map (never used).
int encode_c_tail_map(pf_ctx *c, CUtensorMap *map, const CUtensorMap &main, void *C, int rows) {
  if (c->var.bn % 64 == 0) {
    *map = main;
    return PF_OK;
  }
  return encode_2d(c, map, out_map_type(c->dtype), C, c->N, rows, c->N * pf_out_bytes(c->dtype), 32, 32,
                   CU_TENSOR_MAP_SWIZZLE_64B);
}

int encode_maps(pf_ctx *c) {
  const Variant &v = c->var;
  const CUtensorMapDataType in_t = in_map_type(c->dtype);
  const uint64_t e = static_cast<uint64_t>(v.elem);
  int rc;
  // A: [M x K], K contiguous; box = BK elements (128 B) x BM rows.
  rc = encode_2d(c, &c->tmA, in_t, c->A, c->K, c->M, c->K * e, v.a_box_k, v.a_box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // B: [K x N], N contiguous; box = 128 B of N x BK rows.
  rc = encode_2d(c, &c->tmB, in_t, c->B, c->N, c->K, c->N * e, v.b_chunk_n, v.bk_elems, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // C: [M x N]; box = 128 B of columns x 32 rows.
  if ((rc = encode_c_map(c, &c->tmC, c->C, c->M))) return rc;
  return encode_c_tail_map(c, &c->tmCt, c->tmC, c->C, c->M);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The 3xTF32 kernel's running-sum workspace for `workers` pairs, and the promotion parameters of a launch.
int set_promotion(pf_ctx *c, int workers, TcParams &p) {
  if (c->dtype != PF_F32_3XTF32 || promote_kb_default() <= 0) return PF_OK;
  const size_t ws = static_cast<size_t>(workers) * 2 * 128 * 256 * sizeof(float);
  if (c->promo_ws_cap < ws) {
    if (c->promo_ws) cudaFree(c->promo_ws);
    c->promo_ws = nullptr;
    c->promo_ws_cap = 0;
    if (cudaMalloc(&c->promo_ws, ws) != cudaSuccess) {
      cudaGetLastError();
      return set_err(c, PF_ENOMEM, "cudaMalloc(%zu) for the 3xTF32 running sums failed", ws);
    }
    c->promo_ws_cap = ws;
  }
  p.promote_kb = promote_kb_default();
  p.promote_ws = c->promo_ws;
  return PF_OK;
}

// Tiles of the stream-K tail for a CTA-pair launch of `tiles` tiles (0 = pure data-parallel).  With
// W resident pairs the tail is the partial last wave, R = tiles mod W (all tiles if fewer than W), so a
// pair's share of the tail is below one tile.  Auto mode uses it only where it measured faster on B200:
// at least 3 waves and a partial wave wasting more than 3 % (8192 x 8192 x 2048-row shards: 196 -> 194
// us).  Below 2 waves the per-pair fixed costs (pipeline fill, the head's wait and partial reads, the
// last epilogue) outweigh the rebalancing (1024-row shards: 105 -> 111 us), so auto stays data-parallel.
int sk_tail_tiles(const pf_ctx *c, int tiles, int k_blocks) {
  if (!c->var.stream_k || c->stream_k == 0 || c->stream_k == 2) return 0;
  const int W = c->max_units;
  const int R = tiles % W;
  if (R == 0 || static_cast<long long>(R) * k_blocks < W) return 0;
  if (c->stream_k < 0) {
    const double waves = static_cast<double>(tiles) / W;
    const bool many_waves = waves >= c->var.sk_min_waves && std::ceil(waves) / waves >= 1.03;
    const bool idle_workers = tiles / (std::ceil(waves) * W) < c->var.sk_low_util;
    if (!many_waves && !idle_workers) return 0;
    if (static_cast<long long>(R) * k_blocks < static_cast<long long>(c->var.sk_min_share) * W) return 0;
  }
  return R;
}

// Pairs per band of a row-band stream-K launch of a CTA-pair kernel (0 = whole tiles), used only when asked for
// (pf_set_stream_k 2).  Each of the launch's row blocks gets P = W / (row blocks) pairs, which share its
// k-iterations evenly, so the busiest pair does ceil(S / P) k-blocks of the band's S instead of ceil(tiles /
// W) whole tiles' worth: on the 8- and 4-GPU row shards of 8192^3 (4 and 8 bands of 18 and 9 pairs) 114 / 228
// 512-wide k-blocks per pair instead of 128 / 256.  Measured on B200 (CUDA events, bursts of 20 launches,
// us, whole tiles -> bands): 256 x 512 tiles 1,024 rows 100.7 -> 106.6, 2,048 rows 192.0 -> 193.3; 256 x 256
// tiles 105.2 -> 106.2 and 196.6 -> 192.2.  With more SMs busy each runs its MMAs less often (ncu, 256 x 512 at
// 1,024 rows: the busy SMs' tensor pipes 78.9 -> 68.1 % of cycles) and the split tiles add partial writes and
// reads, so the whole-tile schedule stays the default.
int band_workers(const pf_ctx *c, int num_m_blocks, int num_n_blocks, int k_blocks) {
  if (!c->var.sk_band || c->stream_k != 2) return 0;
  const int W = c->max_units;
  const int P = W / num_m_blocks;
  if (P < 2) return 0;
  // the kernels' band arithmetic is 32-bit: S * P < 2^31
  const long long S = static_cast<long long>(num_n_blocks) * k_blocks;
  if (S * P >= (1ll << 31)) return 0;
  return P;
}

int ensure_sk_workspace(pf_ctx *c, int workers) {
  const size_t ws = static_cast<size_t>(workers) * 2 * 128 * c->var.partial_cols * sizeof(float);
  const size_t fl = static_cast<size_t>(workers) * 2 * sizeof(unsigned);
  if (c->sk_ws_cap < ws) {
    if (c->sk_ws) cudaFree(c->sk_ws);
    c->sk_ws = nullptr;
    c->sk_ws_cap = 0;
    if (cudaMalloc(&c->sk_ws, ws) != cudaSuccess) {
      cudaGetLastError();
      return set_err(c, PF_ENOMEM, "cudaMalloc(%zu) for the stream-K workspace failed", ws);
    }
    c->sk_ws_cap = ws;
  }
  if (c->sk_flags_cap < fl) {
    if (c->sk_flags) cudaFree(c->sk_flags);
    c->sk_flags = nullptr;
    c->sk_flags_cap = 0;
    if (cudaMalloc(&c->sk_flags, fl) != cudaSuccess) {
      cudaGetLastError();
      return set_err(c, PF_ENOMEM, "cudaMalloc(%zu) for the stream-K flags failed", fl);
    }
    PF_CUDA(c, cudaMemset(c->sk_flags, 0, fl));  // epochs start at 1: no flag is set
    c->sk_flags_cap = fl;
    c->epoch = 0;
  }
  return PF_OK;
}

int do_launch(pf_ctx *c, cudaStream_t s) {
  if (!c->prepared) return set_err(c, PF_ESTATE, "pf_launch before pf_prepare");
  if (!c->bound) return set_err(c, PF_ESTATE, "pf_launch before pf_bind");
  const Variant &v = c->var;
  if (v.path == Path::kTensor) {
    TcParams p;
    p.bias = c->bias;
    p.scale = c->sa * c->sb;
    p.M = c->M;
    p.N = c->N;
    p.K = c->K;
    p.num_m_blocks = (c->M + v.bm - 1) / v.bm;
    p.num_n_blocks = (c->N + v.bn - 1) / v.bn;
    p.num_tiles = p.num_m_blocks * p.num_n_blocks;
    p.k_blocks = (c->K + v.bk_elems - 1) / v.bk_elems;
    p.group_m = std::max(1, std::min(c->group_m, p.num_m_blocks));
    p.status = c->d_status;
    p.timeout_ns = c->timeout_ns;
    p.tail_split = tail_split_steps();
    int workers = std::min(p.num_tiles, c->max_units);
    const int sk_tiles = sk_tail_tiles(c, p.num_tiles, p.k_blocks);
    const int band_p = band_workers(c, p.num_m_blocks, p.num_n_blocks, p.k_blocks);
    if (band_p > 0) {
      // Row-band stream-K: P pairs per row block; one partial per pair (two CTAs x 128 x 512 fp32).
      workers = p.num_m_blocks * band_p;
      int rc;
      if ((rc = ensure_sk_workspace(c, workers))) return rc;
      if (++c->epoch == 0) c->epoch = 1;
      p.sk_band_workers = band_p;
      p.epoch = c->epoch;
      p.sk_partials = c->sk_ws;
      p.sk_flags = c->sk_flags;
    } else if (sk_tiles > 0) {
      // Stream-K tail: whole waves stay data-parallel, the last sk_tiles tiles' k-iterations are
      // shared by every resident pair.  Workspace: one 256 KB partial per pair (two CTAs x 128 x 256 fp32).
      workers = c->max_units;
      int rc;
      if ((rc = ensure_sk_workspace(c, workers))) return rc;
      if (++c->epoch == 0) c->epoch = 1;
      p.dp_tiles = p.num_tiles - sk_tiles;
      p.sk_iters = static_cast<long long>(sk_tiles) * p.k_blocks;
      p.epoch = c->epoch;
      p.sk_partials = c->sk_ws;
      p.sk_flags = c->sk_flags;
    }
    dim3 grid(workers * v.cta_per_tile);
    int prc;
    if ((prc = set_promotion(c, workers, p))) return prc;
    v.launch_tc(grid, s, c->tmA, c->tmB, c->tmC, c->tmCt, p);
  } else if (v.path == Path::kImage) {
    // The reference's parameter block {&dA,&dB,&dBias,&dC,&M,&N,&K} (cuda_runner.cpp:182).
    const void *a = c->A, *b = c->B, *bias = c->bias;
    void *cc = c->C;
    int M = c->M, N = c->N, K = c->K;
    void *params[] = {&a, &b, &bias, &cc, &M, &N, &K};
    CUresult r = driver_api().launchKernel(v.img_fn, static_cast<unsigned>(v.img_gx), static_cast<unsigned>(v.img_gy),
                                           1, static_cast<unsigned>(v.threads), 1, 1, 0,
                                           reinterpret_cast<CUstream>(s), params, nullptr);
    if (r != CUDA_SUCCESS) return set_err(c, PF_ECUDA, "cuLaunchKernel -> %s", cu_err(r));
  } else {
    dim3 grid((c->N + v.sbn - 1) / v.sbn, (c->M + v.sbm - 1) / v.sbm);
    if (c->simt_tma)
      v.launch_simt_tma(grid, s, c->tmA, c->tmB, c->bias, static_cast<float *>(c->C), c->M, c->N, c->K, c->d_status,
                        c->timeout_ns);
    else
      v.launch_simt(grid, s, static_cast<const float *>(c->A), static_cast<const float *>(c->B), c->bias,
                    static_cast<float *>(c->C), c->M, c->N, c->K, c->simt_vec);
  }
  PF_CUDA(c, cudaGetLastError());
  return PF_OK;
}

}  // namespace

extern "C" {

const char *pf_version(void) { return "ptxforge_b200 " PF_VERSION_STR " (sm_100a)"; }

size_t pf_elem_bytes(pf_dtype dt) {
  switch (dt) {
    case PF_F32:
    case PF_F32_3XTF32: return 4;
    case PF_BF16: return 2;
    case PF_E4M3: return 1;
  }
  return 0;
}

size_t pf_out_bytes(pf_dtype dt) {
  switch (dt) {
    case PF_F32:
    case PF_F32_3XTF32: return 4;
    case PF_BF16:
    case PF_E4M3: return 2;
  }
  return 0;
}

int pf_open(int device, pf_ctx **out) {
  if (!out) return PF_EINVAL;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return PF_ENODEV;
  }
  if (device < 0 || device >= n) return PF_ENODEV;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return PF_ENODEV;
  if (prop.major != 10) return PF_ENODEV;  // kernels are sm_100a only
  pf_ctx *c = new pf_ctx();
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  DeviceGuard g(device);
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&c->d_status, sizeof(unsigned)) != cudaSuccess ||
      cudaMemset(c->d_status, 0, sizeof(unsigned)) != cudaSuccess || cudaEventCreate(&c->ev0) != cudaSuccess ||
      cudaEventCreate(&c->ev1) != cudaSuccess) {
    pf_close(c);
    return PF_ECUDA;
  }
  *out = c;
  return PF_OK;
}

}  // extern "C"

void cublas_cmp_release(pf_ctx *c);  // cublas_cmp.cuh

extern "C" {

int pf_close(pf_ctx *c) {
  if (!c) return PF_EINVAL;
  if (c->device >= 0) {
    DeviceGuard g(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    cublas_cmp_release(c);
    if (c->sk_ws) cudaFree(c->sk_ws);
    if (c->promo_ws) cudaFree(c->promo_ws);
    if (c->sk_flags) cudaFree(c->sk_flags);
    if (c->d_status) cudaFree(c->d_status);
    if (c->hbufA) cudaFree(c->hbufA);
    if (c->hbufB) cudaFree(c->hbufB);
    if (c->hbufC) cudaFree(c->hbufC);
    if (c->hbufBias) cudaFree(c->hbufBias);
    if (c->ev0) cudaEventDestroy(c->ev0);
    if (c->ev1) cudaEventDestroy(c->ev1);
    for (cudaEvent_t e : c->ev_pool) cudaEventDestroy(e);
    if (c->s_comp) cudaStreamDestroy(c->s_comp);
    if (c->s_out) cudaStreamDestroy(c->s_out);
    if (c->stream) cudaStreamDestroy(c->stream);
    if (c->module) driver_api().moduleUnload(c->module);
  }
  delete c;
  return PF_OK;
}

int pf_prepare_image(pf_ctx *c, const void *image, size_t image_bytes, const char *kernel, int grid_x, int grid_y,
                     int block, int M, int N, int K) {
  if (!c || !image || !image_bytes || !kernel) return set_err(c, PF_EINVAL, "null argument");
  c->prepared = false;
  c->bound = false;
  c->simt_tma = false;
  if (M <= 0 || N <= 0 || K <= 0 || grid_x <= 0 || grid_y <= 0 || block <= 0)
    return set_err(c, PF_EINVAL, "sizes and launch shape must be positive");
  const DriverApi &api = driver_api();
  if (!api.ok) return set_err(c, PF_ECUDA, "CUDA driver entry points unavailable");
  DeviceGuard g(c->device);
  if (c->module) {
    api.moduleUnload(c->module);
    c->module = nullptr;
  }
  // PTX must be NUL-terminated; a cubin is unaffected by a trailing byte (cuda_runner.cpp:157).
  std::string img(static_cast<const char *>(image), image_bytes);
  img.push_back('\0');
  CUresult r = api.moduleLoadData(&c->module, img.data());
  if (r != CUDA_SUCCESS) {
    c->module = nullptr;
    return set_err(c, PF_ECUDA, "cuModuleLoadData -> %s", cu_err(r));
  }
  CUfunction fn = nullptr;
  if ((r = api.moduleGetFunction(&fn, c->module, kernel)) != CUDA_SUCCESS)
    return set_err(c, PF_ECUDA, "cuModuleGetFunction(%s) -> %s", kernel, cu_err(r));
  int max_block = 0;
  if ((r = api.funcGetAttribute(&max_block, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, fn)) != CUDA_SUCCESS)
    return set_err(c, PF_ECUDA, "cuFuncGetAttribute -> %s", cu_err(r));
  if (block > max_block)
    return set_err(c, PF_ETILE, "block %d exceeds kernel max %d (register pressure)", block, max_block);
  Variant v;
  v.path = Path::kImage;
  v.img_fn = fn;
  v.img_gx = grid_x;
  v.img_gy = grid_y;
  v.threads = block;
  c->var = v;
  c->dtype = PF_F32;
  c->tile = pf_tile{0, 0, 0, 0, 0, 0};
  c->M = M;
  c->N = N;
  c->K = K;
  c->prepared = true;
  c->err.clear();
  return PF_OK;
}

const char *pf_last_error(const pf_ctx *c) { return c ? c->err.c_str() : "null context"; }

int pf_set_stream_k(pf_ctx *c, int mode) {
  if (!c || mode < -1 || mode > 2) return set_err(c, PF_EINVAL, "stream-K mode must be -1, 0, 1 or 2");
  c->stream_k = mode;
  return PF_OK;
}

int pf_set_host_chunks(pf_ctx *c, int chunks) {
  if (!c || chunks < 0 || chunks > 64) return set_err(c, PF_EINVAL, "host chunks must be 0 (default) or 1..64");
  c->host_chunks = chunks;
  return PF_OK;
}

int pf_set_wait_timeout(pf_ctx *c, unsigned long long ns) {
  if (!c || ns == 0) return set_err(c, PF_EINVAL, "timeout must be positive");
  c->timeout_ns = ns;
  return PF_OK;
}

int pf_prepare(pf_ctx *c, pf_dtype dt, const pf_tile *t, int M, int N, int K) {
  if (!c || !t) return set_err(c, PF_EINVAL, "null argument");
  c->prepared = false;
  c->bound = false;
  c->simt_tma = false;  // decided again when operands are bound
  if (M <= 0 || N <= 0 || K <= 0) return set_err(c, PF_EINVAL, "M, N, K must be positive (got %d, %d, %d)", M, N, K);
  DeviceGuard g(c->device);
  Variant v;
  if (dt == PF_F32) {
    bool found = false;
    for (const SimtEntry &e : kSimtTable)
      if (same_tile(e.tile, *t)) {
        v = e.make();
        found = true;
        break;
      }
    if (!found)
      return set_err(c, PF_ETILE, "fp32 tile %dx%dx%d t%dx%d p%d is not compiled into this library", t->BM, t->BN,
                     t->BK, t->TM, t->TN, t->PAD);
  } else if (dt == PF_BF16 || dt == PF_E4M3) {
    if (t->BM != 128 && t->BM != 256)
      return set_err(c, PF_ETILE, "tensor path: BM must be 128 (one CTA) or 256 (CTA pair), got %d", t->BM);
    if (t->BK != 32)
      return set_err(c, PF_ETILE, "tensor path: BK must be 32 words (one 128-byte swizzle row), got %d", t->BK);
    if (t->PAD != 0 && t->PAD != 1)
      return set_err(c, PF_ETILE, "tensor path: PAD (extra 128-byte k-atoms per stage) must be 0 or 1, got %d", t->PAD);
    if (t->TN < 1 || t->TN > 64) return set_err(c, PF_ETILE, "tensor path: TN (raster group) out of range: %d", t->TN);
    if (!find_tc_variant(dt, t->BM, t->BN, t->TM, t->PAD + 1, &v))
      return set_err(c, PF_ETILE, "tensor path: no %s kernel with BM=%d, BN=%d and at most %d stages",
                     dt == PF_BF16 ? "bf16" : "e4m3", t->BM, t->BN, t->TM);
    const int e = (int)pf_elem_bytes(dt);
    if ((static_cast<long long>(K) * e) % 16 != 0)
      return set_err(c, PF_ESHAPE, "tensor path: rows of A must be a multiple of 16 bytes (K=%d)", K);
    if ((static_cast<long long>(N) * e) % 16 != 0 || (N * 2) % 16 != 0)
      return set_err(c, PF_ESHAPE, "tensor path: rows of B and C must be multiples of 16 bytes (N=%d)", N);
    c->group_m = t->TN;
  } else if (dt == PF_F32_3XTF32) {
    if (t->BM != 256 || t->BN != 256)
      return set_err(c, PF_ETILE, "3xTF32 path: the tile is 256x256 (CTA pair), got BM=%d BN=%d", t->BM, t->BN);
    if (t->BK != 32)
      return set_err(c, PF_ETILE, "3xTF32 path: BK must be 32 words (one 128-byte swizzle row), got %d", t->BK);
    if (t->PAD != 0) return set_err(c, PF_ETILE, "3xTF32 path: PAD must be 0, got %d", t->PAD);
    if (t->TN < 1 || t->TN > 64) return set_err(c, PF_ETILE, "3xTF32 path: TN (raster group) out of range: %d", t->TN);
    if (!find_tc_variant(dt, t->BM, t->BN, t->TM, 1, &v))
      return set_err(c, PF_ETILE, "3xTF32 path: no kernel with at most %d stages (2 to 4)", t->TM);
    if (K % 4 != 0 || N % 4 != 0)
      return set_err(c, PF_ESHAPE, "3xTF32 path: rows of A, B and C must be multiples of 16 bytes (N=%d, K=%d)", N, K);
    c->group_m = t->TN;
  } else {
    return set_err(c, PF_ETILE, "dtype %d is not built in this library", (int)dt);
  }
  if (v.path == Path::kSimt && v.tma_func) {
    cudaError_t e = cudaFuncSetAttribute(v.tma_func, cudaFuncAttributeMaxDynamicSharedMemorySize, v.tma_smem);
    if (e != cudaSuccess) return set_err(c, PF_ECUDA, "cudaFuncSetAttribute -> %s", cudaGetErrorString(e));
  }
  if (v.path == Path::kTensor) {
    cudaError_t e = cudaFuncSetAttribute(v.func, cudaFuncAttributeMaxDynamicSharedMemorySize, v.smem);
    if (e != cudaSuccess) return set_err(c, PF_ECUDA, "cudaFuncSetAttribute -> %s", cudaGetErrorString(e));
    // Persistent grid: as many CTAs (or CTA pairs) as can be resident at once.
    c->max_units = c->num_sms;
    if (v.cta_per_tile == 2) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 2;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.gridDim = dim3(2 * (c->num_sms / 2));
      cfg.blockDim = dim3(v.threads);
      cfg.dynamicSmemBytes = v.smem;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      e = cudaOccupancyMaxActiveClusters(&clusters, v.func, &cfg);
      if (e != cudaSuccess || clusters <= 0) {
        cudaGetLastError();
        clusters = c->num_sms / 2;
      }
      c->max_units = clusters;
    }
  }
  c->var = v;
  c->dtype = dt;
  c->tile = *t;
  c->M = M;
  c->N = N;
  c->K = K;
  c->prepared = true;
  c->err.clear();
  return PF_OK;
}

int pf_bind(pf_ctx *c, const void *A, const void *B, const float *bias, void *C, float sa, float sb) {
  if (!c) return PF_EINVAL;
  if (!c->prepared) return set_err(c, PF_ESTATE, "pf_bind before pf_prepare");
  if (!A || !B || !bias || !C) return set_err(c, PF_EINVAL, "null operand");
  if (c->dtype != PF_E4M3 && (sa != 1.f || sb != 1.f))
    return set_err(c, PF_EINVAL, "scales apply to e4m3 operands only (got %g, %g)", sa, sb);
  DeviceGuard g(c->device);
  c->bound = false;
  c->A = A;
  c->B = B;
  c->bias = bias;
  c->C = C;
  c->sa = sa;
  c->sb = sb;
  if (c->var.path == Path::kTensor) {
    if (!aligned16(A) || !aligned16(B) || !aligned16(C) || !aligned16(bias))
      return set_err(c, PF_EINVAL, "tensor path: operands must be 16-byte aligned");
    int rc = encode_maps(c);
    if (rc) return rc;
  } else {
    c->simt_vec = aligned16(A) && aligned16(B) && aligned16(C) && aligned16(bias) && (c->K % 4 == 0) &&
                  (c->N % 4 == 0);
    c->simt_tma = false;
    if (c->simt_vec && c->var.tma_func) {
      // A: [M x K] fp32, box BK x BM with the swizzle of one BK-float row; B: [K x N], box BN x BK, unswizzled.
      const int bk = c->var.tma_bk;
      int rc = encode_2d(c, &c->tmA, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, A, c->K, c->M, c->K * 4ull, bk, c->var.sbm,
                         bk == 16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      rc = encode_2d(c, &c->tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, B, c->N, c->K, c->N * 4ull, c->var.sbn, bk,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
      c->simt_tma = true;
    }
  }
  c->bound = true;
  return PF_OK;
}

int pf_launch(pf_ctx *c, void *stream) {
  if (!c) return PF_EINVAL;
  DeviceGuard g(c->device);
  return do_launch(c, static_cast<cudaStream_t>(stream));
}

int pf_time(pf_ctx *c, int warmup, int iters, int reps, double *median_ms) {
  if (!c || !median_ms || warmup < 0 || iters <= 0 || reps <= 0) return set_err(c, PF_EINVAL, "bad timing arguments");
  DeviceGuard g(c->device);
  int rc;
  for (int i = 0; i < warmup; ++i)
    if ((rc = do_launch(c, c->stream))) return rc;
  PF_CUDA(c, cudaStreamSynchronize(c->stream));
  std::vector<double> per;
  for (int r = 0; r < reps; ++r) {
    PF_CUDA(c, cudaEventRecord(c->ev0, c->stream));
    for (int i = 0; i < iters; ++i)
      if ((rc = do_launch(c, c->stream))) return rc;
    PF_CUDA(c, cudaEventRecord(c->ev1, c->stream));
    PF_CUDA(c, cudaEventSynchronize(c->ev1));
    float ms = 0.f;
    PF_CUDA(c, cudaEventElapsedTime(&ms, c->ev0, c->ev1));
    per.push_back(static_cast<double>(ms) / iters);
  }
  std::sort(per.begin(), per.end());
  *median_ms = per[per.size() / 2];
  unsigned st = 0;
  PF_CUDA(c, cudaMemcpy(&st, c->d_status, sizeof st, cudaMemcpyDeviceToHost));
  if (st) return set_err(c, PF_ETIMEOUT, "a bounded device wait ran out during timing (status 0x%x)", st);
  return PF_OK;
}

int pf_attrs(pf_ctx *c, pf_attr *out) {
  if (!c || !out) return PF_EINVAL;
  if (!c->prepared) return set_err(c, PF_ESTATE, "pf_attrs before pf_prepare");
  DeviceGuard g(c->device);
  if (c->var.path == Path::kImage) {
    const DriverApi &api = driver_api();
    int regs = 0, local = 0, smem = 0, bps = 0;
    CUresult r;
    if ((r = api.funcGetAttribute(&regs, CU_FUNC_ATTRIBUTE_NUM_REGS, c->var.img_fn)) != CUDA_SUCCESS ||
        (r = api.funcGetAttribute(&local, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, c->var.img_fn)) != CUDA_SUCCESS ||
        (r = api.funcGetAttribute(&smem, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, c->var.img_fn)) != CUDA_SUCCESS ||
        (r = api.occupancy(&bps, c->var.img_fn, c->var.threads, 0)) != CUDA_SUCCESS)
      return set_err(c, PF_ECUDA, "kernel attributes -> %s", cu_err(r));
    out->regs = regs;
    out->local_bytes = local;
    out->smem_bytes = smem;
    out->blocks_per_sm = bps;
    out->threads = c->var.threads;
    out->num_sms = c->num_sms;
    out->grid = c->var.img_gx * c->var.img_gy;
    return PF_OK;
  }
  cudaFuncAttributes fa;
  // the fp32 kernel that runs the bound operands (the TMA-fed one where they allow it)
  const bool tma = c->simt_tma && c->var.tma_func && c->bound;
  const void *fn = tma ? c->var.tma_func : c->var.func;
  const int dyn_smem = tma ? c->var.tma_smem : c->var.smem;
  PF_CUDA(c, cudaFuncGetAttributes(&fa, fn));
  int bps = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, fn, c->var.threads, dyn_smem) != cudaSuccess) {
    cudaGetLastError();  // cluster kernels: the per-SM query may be refused; one CTA per SM by construction
    bps = 1;
  }
  out->regs = fa.numRegs;
  out->local_bytes = static_cast<int>(fa.localSizeBytes);
  out->smem_bytes = static_cast<int>(fa.sharedSizeBytes) + dyn_smem;
  out->blocks_per_sm = bps;
  out->threads = c->var.threads;
  out->num_sms = c->num_sms;
  if (c->var.path == Path::kTensor) {
    const int mblocks = (c->M + c->var.bm - 1) / c->var.bm, nblocks = (c->N + c->var.bn - 1) / c->var.bn;
    const int tiles = mblocks * nblocks;
    const int kb = (c->K + c->var.bk_elems - 1) / c->var.bk_elems;
    const int band_p = band_workers(c, mblocks, nblocks, kb);
    const int workers = band_p > 0 ? mblocks * band_p
                                   : (sk_tail_tiles(c, tiles, kb) > 0 ? c->max_units : std::min(tiles, c->max_units));
    out->grid = workers * c->var.cta_per_tile;
  } else {
    out->grid = ((c->N + c->var.sbn - 1) / c->var.sbn) * ((c->M + c->var.sbm - 1) / c->var.sbm);
  }
  return PF_OK;
}

int pf_device_status(pf_ctx *c, unsigned *err_word) {
  if (!c || !err_word) return PF_EINVAL;
  DeviceGuard g(c->device);
  PF_CUDA(c, cudaDeviceSynchronize());  // launches may be on any stream of this device
  PF_CUDA(c, cudaMemcpy(err_word, c->d_status, sizeof(unsigned), cudaMemcpyDeviceToHost));
  PF_CUDA(c, cudaMemset(c->d_status, 0, sizeof(unsigned)));
  return PF_OK;
}

}  // extern "C"

namespace {
// Context-owned device operands sized for the prepared problem, bound to the context.
int ensure_host_bufs(pf_ctx *c, float sa, float sb) {
  const size_t e = pf_elem_bytes(c->dtype), o = pf_out_bytes(c->dtype);
  const size_t nA = static_cast<size_t>(c->M) * c->K * e, nB = static_cast<size_t>(c->K) * c->N * e;
  const size_t nC = static_cast<size_t>(c->M) * c->N * o, nBias = static_cast<size_t>(c->N) * sizeof(float);
  auto ensure = [&](void **buf, size_t *cap, size_t need) -> int {
    if (*cap >= need) return PF_OK;
    if (*buf) cudaFree(*buf);
    *buf = nullptr;
    *cap = 0;
    if (cudaMalloc(buf, need) != cudaSuccess) {
      cudaGetLastError();
      return set_err(c, PF_ENOMEM, "cudaMalloc(%zu) failed", need);
    }
    *cap = need;
    return PF_OK;
  };
  int rc;
  if ((rc = ensure(&c->hbufA, &c->capA, nA)) || (rc = ensure(&c->hbufB, &c->capB, nB)) ||
      (rc = ensure(&c->hbufC, &c->capC, nC)) ||
      (rc = ensure(reinterpret_cast<void **>(&c->hbufBias), &c->capBias, nBias)))
    return rc;
  if (!c->bound || c->A != c->hbufA || c->B != c->hbufB || c->C != c->hbufC || c->bias != c->hbufBias ||
      c->sa != sa || c->sb != sb) {
    if ((rc = pf_bind(c, c->hbufA, c->hbufB, c->hbufBias, c->hbufC, sa, sb))) return rc;
  }
  return PF_OK;
}

// Row chunks of the host-buffer pipelines.
int host_chunk_cap(const pf_ctx *c) { return c->host_chunks > 0 ? c->host_chunks : 8; }

// Launch the bound problem restricted to output rows [r0, r0 + rows) on stream s: the same kernel
// variant on row windows of A and C (TMA maps re-encoded for the window on the tensor path).
int launch_rows(pf_ctx *c, cudaStream_t s, int r0, int rows) {
  const Variant &v = c->var;
  const size_t e = pf_elem_bytes(c->dtype), o = pf_out_bytes(c->dtype);
  const void *A = static_cast<const char *>(c->A) + static_cast<size_t>(r0) * c->K * e;
  void *C = static_cast<char *>(c->C) + static_cast<size_t>(r0) * c->N * o;
  if (v.path == Path::kTensor) {
    CUtensorMap tmA, tmC, tmCt;
    int rc;
    if ((rc = encode_2d(c, &tmA, in_map_type(c->dtype), A, c->K, rows, c->K * e, v.a_box_k, v.a_box_rows,
                        CU_TENSOR_MAP_SWIZZLE_128B)) ||
        (rc = encode_c_map(c, &tmC, C, rows)) || (rc = encode_c_tail_map(c, &tmCt, tmC, C, rows)))
      return rc;
    TcParams p;
    p.bias = c->bias;
    p.scale = c->sa * c->sb;
    p.M = rows;
    p.N = c->N;
    p.K = c->K;
    p.num_m_blocks = (rows + v.bm - 1) / v.bm;
    p.num_n_blocks = (c->N + v.bn - 1) / v.bn;
    p.num_tiles = p.num_m_blocks * p.num_n_blocks;
    p.k_blocks = (c->K + v.bk_elems - 1) / v.bk_elems;
    p.group_m = std::max(1, std::min(c->group_m, p.num_m_blocks));
    p.status = c->d_status;
    p.timeout_ns = c->timeout_ns;
    p.tail_split = tail_split_steps();
    // k directions as in one launch over the whole bound problem (the same bits as do_launch)
    const int full_m_blocks = (c->M + v.bm - 1) / v.bm;
    const int full_tiles = full_m_blocks * p.num_n_blocks;
    p.dir_m0 = r0 / v.bm;
    p.dir_num_m_blocks = full_m_blocks;
    p.dir_group_m = std::max(1, std::min(c->group_m, full_m_blocks));
    p.dir_workers = sk_tail_tiles(c, full_tiles, p.k_blocks) > 0 ? c->max_units : std::min(full_tiles, c->max_units);
    if ((rc = set_promotion(c, std::min(p.num_tiles, c->max_units), p))) return rc;
    v.launch_tc(dim3(std::min(p.num_tiles, c->max_units) * v.cta_per_tile), s, tmA, c->tmB, tmC, tmCt, p);
  } else if (v.path == Path::kSimt) {
    dim3 grid((c->N + v.sbn - 1) / v.sbn, (rows + v.sbm - 1) / v.sbm);
    v.launch_simt(grid, s, static_cast<const float *>(A), static_cast<const float *>(c->B), c->bias,
                  static_cast<float *>(C), rows, c->N, c->K, c->simt_vec);
  } else {
    return set_err(c, PF_ESTATE, "row-window launch on an image");
  }
  PF_CUDA(c, cudaGetLastError());
  return PF_OK;
}

// Context-owned device operands sized for the prepared problem; async H2D copies on the context's
// stream; bind.  Used by pf_upload.
int stage_inputs(pf_ctx *c, const void *hA, const void *hB, const float *hbias, float sa, float sb) {
  const size_t e = pf_elem_bytes(c->dtype);
  int rc;
  if ((rc = ensure_host_bufs(c, sa, sb))) return rc;
  PF_CUDA(c, cudaMemcpyAsync(c->hbufA, hA, static_cast<size_t>(c->M) * c->K * e, cudaMemcpyHostToDevice, c->stream));
  PF_CUDA(c, cudaMemcpyAsync(c->hbufB, hB, static_cast<size_t>(c->K) * c->N * e, cudaMemcpyHostToDevice, c->stream));
  PF_CUDA(c, cudaMemcpyAsync(c->hbufBias, hbias, static_cast<size_t>(c->N) * sizeof(float), cudaMemcpyHostToDevice,
                             c->stream));
  return PF_OK;
}
}  // namespace

extern "C" {

int pf_run_host(pf_ctx *c, const void *hA, const void *hB, const float *hbias, void *hC, float sa, float sb) {
  if (!c) return PF_EINVAL;
  if (!c->prepared) return set_err(c, PF_ESTATE, "pf_run_host before pf_prepare");
  if (!hA || !hB || !hbias || !hC) return set_err(c, PF_EINVAL, "null host operand");
  DeviceGuard g(c->device);
  int rc;
  if ((rc = ensure_host_bufs(c, sa, sb))) return rc;
  const size_t e = pf_elem_bytes(c->dtype), o = pf_out_bytes(c->dtype);
  const size_t rowA = static_cast<size_t>(c->K) * e, rowC = static_cast<size_t>(c->N) * o;
  // Row chunks (whole kernel tiles), at most 8: chunk i's GEMM starts as soon as B and its rows of A are
  // in; its rows of C go back while later chunks are still arriving (copies in both directions and the
  // kernels overlap).  An image keeps its fixed launch shape: one chunk.
  const int align = c->var.path == Path::kTensor ? c->var.bm : c->var.path == Path::kSimt ? c->var.sbm : c->M;
  const int units = (c->M + align - 1) / align;
  const int P = c->var.path == Path::kImage ? 1 : std::max(1, std::min(host_chunk_cap(c), units));
  if (!c->s_comp) PF_CUDA(c, cudaStreamCreateWithFlags(&c->s_comp, cudaStreamNonBlocking));
  if (!c->s_out) PF_CUDA(c, cudaStreamCreateWithFlags(&c->s_out, cudaStreamNonBlocking));
  while (c->ev_pool.size() < static_cast<size_t>(2 * P + 1)) {
    cudaEvent_t ev;
    PF_CUDA(c, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    c->ev_pool.push_back(ev);
  }
  cudaEvent_t evB = c->ev_pool[0];
  PF_CUDA(c, cudaMemcpyAsync(c->hbufB, hB, static_cast<size_t>(c->K) * c->N * e, cudaMemcpyHostToDevice, c->stream));
  PF_CUDA(c, cudaMemcpyAsync(c->hbufBias, hbias, static_cast<size_t>(c->N) * sizeof(float), cudaMemcpyHostToDevice,
                             c->stream));
  PF_CUDA(c, cudaEventRecord(evB, c->stream));
  PF_CUDA(c, cudaStreamWaitEvent(c->s_comp, evB, 0));
  for (int i = 0; i < P; ++i) {
    const int r0 = static_cast<int>(static_cast<long long>(units) * i / P) * align;
    const int r1 = std::min(c->M, static_cast<int>(static_cast<long long>(units) * (i + 1) / P) * align);
    if (r1 <= r0) continue;
    cudaEvent_t evA = c->ev_pool[1 + 2 * i], evC = c->ev_pool[2 + 2 * i];
    PF_CUDA(c, cudaMemcpyAsync(static_cast<char *>(c->hbufA) + r0 * rowA, static_cast<const char *>(hA) + r0 * rowA,
                               (r1 - r0) * rowA, cudaMemcpyHostToDevice, c->stream));
    PF_CUDA(c, cudaEventRecord(evA, c->stream));
    PF_CUDA(c, cudaStreamWaitEvent(c->s_comp, evA, 0));
    if ((rc = P == 1 ? do_launch(c, c->s_comp) : launch_rows(c, c->s_comp, r0, r1 - r0))) return rc;
    PF_CUDA(c, cudaEventRecord(evC, c->s_comp));
    PF_CUDA(c, cudaStreamWaitEvent(c->s_out, evC, 0));
    PF_CUDA(c, cudaMemcpyAsync(static_cast<char *>(hC) + r0 * rowC, static_cast<char *>(c->hbufC) + r0 * rowC,
                               (r1 - r0) * rowC, cudaMemcpyDeviceToHost, c->s_out));
  }
  PF_CUDA(c, cudaStreamSynchronize(c->s_out));
  PF_CUDA(c, cudaStreamSynchronize(c->s_comp));
  PF_CUDA(c, cudaStreamSynchronize(c->stream));
  return PF_OK;
}

int pf_run_host_rows(pf_ctx *c, const void *hA, void *hC, void *after_stream, void *copies_after_stream) {
  if (!c) return PF_EINVAL;
  if (!c->prepared || !c->bound) return set_err(c, PF_ESTATE, "pf_run_host_rows before pf_prepare / pf_bind");
  if (!hA || !hC) return set_err(c, PF_EINVAL, "null host operand");
  if (c->var.path == Path::kImage) return set_err(c, PF_ESTATE, "pf_run_host_rows on a loaded image");
  DeviceGuard g(c->device);
  const size_t e = pf_elem_bytes(c->dtype), o = pf_out_bytes(c->dtype);
  const size_t rowA = static_cast<size_t>(c->K) * e, rowC = static_cast<size_t>(c->N) * o;
  const int align = c->var.path == Path::kTensor ? c->var.bm : c->var.sbm;
  const int units = (c->M + align - 1) / align;
  const int P = std::max(1, std::min(host_chunk_cap(c), units));
  if (!c->s_comp) PF_CUDA(c, cudaStreamCreateWithFlags(&c->s_comp, cudaStreamNonBlocking));
  if (!c->s_out) PF_CUDA(c, cudaStreamCreateWithFlags(&c->s_out, cudaStreamNonBlocking));
  while (c->ev_pool.size() < static_cast<size_t>(2 * P + 1)) {
    cudaEvent_t ev;
    PF_CUDA(c, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    c->ev_pool.push_back(ev);
  }
  // B and bias are produced on `after_stream` (an upload, an all-gather): the kernels wait for it.  The
  // copies of A wait only for `copies_after_stream` -- e.g. the copy of this rank's slice of B, so that the
  // host link carries B first and then A while the all-gather runs over NVLink.
  cudaEvent_t evB = c->ev_pool[0];
  PF_CUDA(c, cudaEventRecord(evB, static_cast<cudaStream_t>(after_stream)));
  PF_CUDA(c, cudaStreamWaitEvent(c->s_comp, evB, 0));
  if (copies_after_stream != after_stream) {
    if (c->ev_pool.size() < static_cast<size_t>(2 * P + 2)) {
      cudaEvent_t ev;
      PF_CUDA(c, cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
      c->ev_pool.push_back(ev);
    }
    cudaEvent_t evCopy = c->ev_pool[2 * P + 1];
    PF_CUDA(c, cudaEventRecord(evCopy, static_cast<cudaStream_t>(copies_after_stream)));
    PF_CUDA(c, cudaStreamWaitEvent(c->stream, evCopy, 0));
  } else {
    PF_CUDA(c, cudaStreamWaitEvent(c->stream, evB, 0));
  }
  for (int i = 0; i < P; ++i) {
    const int r0 = static_cast<int>(static_cast<long long>(units) * i / P) * align;
    const int r1 = std::min(c->M, static_cast<int>(static_cast<long long>(units) * (i + 1) / P) * align);
    if (r1 <= r0) continue;
    cudaEvent_t evA = c->ev_pool[1 + 2 * i], evC = c->ev_pool[2 + 2 * i];
    PF_CUDA(c, cudaMemcpyAsync(static_cast<char *>(const_cast<void *>(c->A)) + r0 * rowA,
                               static_cast<const char *>(hA) + r0 * rowA, (r1 - r0) * rowA, cudaMemcpyHostToDevice,
                               c->stream));
    PF_CUDA(c, cudaEventRecord(evA, c->stream));
    PF_CUDA(c, cudaStreamWaitEvent(c->s_comp, evA, 0));
    int rc;
    if ((rc = P == 1 ? do_launch(c, c->s_comp) : launch_rows(c, c->s_comp, r0, r1 - r0))) return rc;
    PF_CUDA(c, cudaEventRecord(evC, c->s_comp));
    PF_CUDA(c, cudaStreamWaitEvent(c->s_out, evC, 0));
    PF_CUDA(c, cudaMemcpyAsync(static_cast<char *>(hC) + r0 * rowC, static_cast<char *>(c->C) + r0 * rowC,
                               (r1 - r0) * rowC, cudaMemcpyDeviceToHost, c->s_out));
  }
  PF_CUDA(c, cudaStreamSynchronize(c->s_out));
  PF_CUDA(c, cudaStreamSynchronize(c->s_comp));
  PF_CUDA(c, cudaStreamSynchronize(c->stream));
  return PF_OK;
}

int pf_upload(pf_ctx *c, const void *hA, const void *hB, const float *hbias, float sa, float sb) {
  if (!c) return PF_EINVAL;
  if (!c->prepared) return set_err(c, PF_ESTATE, "pf_upload before pf_prepare");
  if (!hA || !hB || !hbias) return set_err(c, PF_EINVAL, "null host operand");
  DeviceGuard g(c->device);
  int rc;
  if ((rc = stage_inputs(c, hA, hB, hbias, sa, sb))) return rc;
  PF_CUDA(c, cudaMemsetAsync(c->hbufC, 0, static_cast<size_t>(c->M) * c->N * pf_out_bytes(c->dtype), c->stream));
  PF_CUDA(c, cudaStreamSynchronize(c->stream));
  return PF_OK;
}

int pf_download(pf_ctx *c, void *hC) {
  if (!c || !hC) return PF_EINVAL;
  if (!c->prepared || !c->hbufC || c->C != c->hbufC)
    return set_err(c, PF_ESTATE, "pf_download without context-owned operands (call pf_upload first)");
  DeviceGuard g(c->device);
  PF_CUDA(c, cudaDeviceSynchronize());
  const size_t nC = static_cast<size_t>(c->M) * c->N * pf_out_bytes(c->dtype);
  PF_CUDA(c, cudaMemcpy(hC, c->hbufC, nC, cudaMemcpyDeviceToHost));
  return PF_OK;
}

int pf_shard_rows(int M, int G, int g, int align, int *row0, int *rows) {
  if (M <= 0 || G <= 0 || g < 0 || g >= G || align <= 0 || !row0 || !rows) return PF_EINVAL;
  // Split M into ceil(M / align) units of `align` rows (the last one partial for a ragged M) and give
  // shard g units [units*g/G, units*(g+1)/G): shard sizes differ by at most one unit.
  const long long units = (static_cast<long long>(M) + align - 1) / align;
  const long long lo = units * g / G, hi = units * (g + 1) / G;
  const long long r0 = std::min<long long>(lo * align, M), r1 = std::min<long long>(hi * align, M);
  *row0 = static_cast<int>(r0);
  *rows = static_cast<int>(r1 - r0);
  return PF_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Bounded-wait self-test: one block waits on an mbarrier that nothing arrives at.
// ------------------------------------------------------------------------------------------------
namespace {
__global__ void selftest_wait_kernel(unsigned *status, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    pf::mbar_init(&bar, 1);
    abort_flag = 0;
    pf::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!pf::mbar_wait(&bar, 0, timeout_ns, &abort_flag)) atomicOr(status, pf::kErrEpilogueWait);
  }
  __syncthreads();
}
}  // namespace

extern "C" int pf_selftest_wait_timeout(pf_ctx *c, unsigned long long timeout_ns, unsigned *err_word) {
  if (!c || !err_word || timeout_ns == 0 || timeout_ns > 10000000000ull)
    return set_err(c, PF_EINVAL, "bad self-test arguments");
  DeviceGuard g(c->device);
  PF_CUDA(c, cudaMemsetAsync(c->d_status, 0, sizeof(unsigned), c->stream));
  selftest_wait_kernel<<<1, 32, 0, c->stream>>>(c->d_status, timeout_ns);
  PF_CUDA(c, cudaGetLastError());
  return pf_device_status(c, err_word);
}

// ------------------------------------------------------------------------------------------------
// No-allocation entry point (no counterpart in the reference).  For callers that cannot allocate
// GPU memory at call time: the tensor-core kernel's scratch (its device status word) lives in this
// fixed, file-scope array instead of a cudaMalloc'ed word of a pf_ctx.  Every GPU that loads the
// library holds the array until the process exits.
// ------------------------------------------------------------------------------------------------
static __device__ __align__(256) unsigned char pf_noalloc_scratch[PF_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoallocMaxDevices = 64;
constexpr int kNoallocMaxKernels = 32;                       // kernel variants whose launch set-up is cached
constexpr unsigned long long kNoallocWaitNs = 4000000000ull;  // bound of each device wait (pf_ctx's default)

// Per-device set-up, done with that device current: the array's device address (host code cannot use
// the symbol itself -- on the host it names a stand-in, not device memory), the SM count and compute
// capability, and per kernel variant its shared-memory attribute and co-resident CTA pairs.  `ready` is set
// only when the look-ups succeeded, so a failed set-up (for instance a first call made during a stream
// capture) is tried again by the next call instead of failing every later call.  Fixed-size tables: the
// entry point allocates nothing, on the host either.
struct NoallocKernel {
  const void *func = nullptr;
  int units = 0;
};
struct NoallocDevice {
  std::mutex mu;
  bool ready = false;
  unsigned *scratch = nullptr;
  int num_sms = 0;
  int cc_major = 0;
  NoallocKernel kernels[kNoallocMaxKernels];
  int n_kernels = 0;
};
NoallocDevice g_noalloc_dev[kNoallocMaxDevices];

int noalloc_fail(char *err, size_t len, int code, const char *fmt, ...) {
  if (err && len) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, len, fmt, ap);
    va_end(ap);
  }
  return code;
}

// The device's scratch address and properties (first successful call per device does the look-ups).
cudaError_t noalloc_device_setup(NoallocDevice &d, int device) {
  std::lock_guard<std::mutex> lk(d.mu);
  if (d.ready) return cudaSuccess;
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, pf_noalloc_scratch);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, device);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return e;
  }
  d.scratch = static_cast<unsigned *>(p);
  d.ready = p != nullptr;
  return d.ready ? cudaSuccess : cudaErrorInvalidSymbol;
}

// Persistent-grid size for a variant: its co-resident CTAs (1-CTA kernels) or CTA pairs, after raising its
// dynamic shared-memory limit; cached per (device, variant) once both calls succeeded.
cudaError_t noalloc_kernel_units(NoallocDevice &d, const Variant &v, int *units) {
  std::lock_guard<std::mutex> lk(d.mu);
  for (int i = 0; i < d.n_kernels; ++i)
    if (d.kernels[i].func == v.func) {
      *units = d.kernels[i].units;
      return cudaSuccess;
    }
  cudaError_t ce = cudaFuncSetAttribute(v.func, cudaFuncAttributeMaxDynamicSharedMemorySize, v.smem);
  if (ce != cudaSuccess) return ce;
  int u = d.num_sms;
  if (v.cta_per_tile == 2) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (d.num_sms / 2));
    cfg.blockDim = dim3(v.threads);
    cfg.dynamicSmemBytes = v.smem;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, v.func, &cfg) != cudaSuccess || clusters <= 0) {
      cudaGetLastError();
      *units = d.num_sms / 2;  // not cached: the next call asks again
      return cudaSuccess;
    }
    u = clusters;
  }
  if (d.n_kernels < kNoallocMaxKernels) d.kernels[d.n_kernels++] = {v.func, u};
  *units = u;
  return cudaSuccess;
}

}  // namespace

extern "C" int pf_gemm_bias_gelu_noalloc(int device, pf_dtype dtype, const pf_tile *t, int M, int N, int K,
                                         const void *A, const void *B, const float *bias, void *C, float sa,
                                         float sb, void *stream, unsigned *status_out, char *err,
                                         size_t err_len) {
  if (err && err_len) err[0] = '\0';
  if (!t || !A || !B || !bias || !C) return noalloc_fail(err, err_len, PF_EINVAL, "null argument");
  if (M <= 0 || N <= 0 || K <= 0)
    return noalloc_fail(err, err_len, PF_EINVAL, "M, N, K must be positive (got %d, %d, %d)", M, N, K);
  if (dtype != PF_BF16 && dtype != PF_E4M3)
    return noalloc_fail(err, err_len, PF_EINVAL, "only the bf16 / e4m3 tensor-core kernels run without allocation");
  if (dtype == PF_BF16 && (sa != 1.f || sb != 1.f))
    return noalloc_fail(err, err_len, PF_EINVAL, "scales apply to e4m3 operands only");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev || device >= kNoallocMaxDevices) {
    cudaGetLastError();
    return noalloc_fail(err, err_len, PF_ENODEV, "no CUDA device %d", device);
  }
  DeviceGuard g(device);
  NoallocDevice &d = g_noalloc_dev[device];
  cudaError_t ce = noalloc_device_setup(d, device);
  if (ce != cudaSuccess)
    return noalloc_fail(err, err_len, PF_ECUDA, "scratch set-up on device %d failed: %s", device,
                        cudaGetErrorString(ce));
  if (d.cc_major != 10) return noalloc_fail(err, err_len, PF_ENODEV, "device %d is not an sm_100 GPU", device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int stream_dev = -1;
  ce = cudaStreamGetDevice(s, &stream_dev);
  if (ce != cudaSuccess) {
    cudaGetLastError();
    return noalloc_fail(err, err_len, PF_EINVAL, "stream is not a valid CUDA stream: %s", cudaGetErrorString(ce));
  }
  if (stream_dev != device)
    return noalloc_fail(err, err_len, PF_EINVAL, "stream belongs to device %d, not device %d", stream_dev, device);

  // Kernel variant and layout rules: those of pf_prepare / pf_bind.
  if ((t->BM != 128 && t->BM != 256) || t->BK != 32 || (t->PAD != 0 && t->PAD != 1) || t->TN < 1 || t->TN > 64)
    return noalloc_fail(err, err_len, PF_ETILE, "tile %dx%dx%d t%dx%d p%d has no tensor-core kernel", t->BM, t->BN,
                        t->BK, t->TM, t->TN, t->PAD);
  Variant v;
  if (!find_tc_variant(dtype, t->BM, t->BN, t->TM, t->PAD + 1, &v))
    return noalloc_fail(err, err_len, PF_ETILE, "no kernel with BM=%d, BN=%d and at most %d stages", t->BM, t->BN,
                        t->TM);
  const long long e = static_cast<long long>(pf_elem_bytes(dtype));
  if ((K * e) % 16 != 0 || (N * e) % 16 != 0 || (N * 2LL) % 16 != 0)
    return noalloc_fail(err, err_len, PF_ESHAPE, "rows of A, B and C must be multiples of 16 bytes (N=%d, K=%d)", N, K);
  if (!aligned16(A) || !aligned16(B) || !aligned16(C) || !aligned16(bias))
    return noalloc_fail(err, err_len, PF_EINVAL, "operands must be 16-byte aligned");
  // Scratch this kernel needs: one 32-bit status word.  Whole tiles only: the stream-K tail, which needs a
  // workspace of partial sums, is never used here.
  constexpr size_t kScratchNeeded = sizeof(unsigned);
  if (kScratchNeeded > sizeof(pf_noalloc_scratch))
    return noalloc_fail(err, err_len, PF_EINVAL, "the kernel needs %zu bytes of scratch; the fixed area holds %zu",
                        kScratchNeeded, sizeof(pf_noalloc_scratch));

  int units = 0;
  ce = noalloc_kernel_units(d, v, &units);
  if (ce != cudaSuccess) {
    cudaGetLastError();
    return noalloc_fail(err, err_len, PF_ECUDA, "kernel set-up: %s", cudaGetErrorString(ce));
  }

  const CUtensorMapDataType in_t =
      dtype == PF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  CUtensorMap tmA, tmB, tmC, tmCt;
  char msg[200];
  if (encode_2d_msg(msg, sizeof msg, &tmA, in_t, A, K, M, K * e, v.a_box_k, v.a_box_rows,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      encode_2d_msg(msg, sizeof msg, &tmB, in_t, B, N, K, N * e, v.b_chunk_n, v.bk_elems,
                    CU_TENSOR_MAP_SWIZZLE_128B) ||
      encode_2d_msg(msg, sizeof msg, &tmC, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, C, N, M, N * 2ull, 64, 32,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return noalloc_fail(err, err_len, PF_ECUDA, "TMA tensor-map encoding: %s", msg);
  tmCt = tmC;
  if (v.bn % 64 != 0 && encode_2d_msg(msg, sizeof msg, &tmCt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, C, N, M, N * 2ull,
                                      32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
    return noalloc_fail(err, err_len, PF_ECUDA, "TMA tensor-map encoding: %s", msg);

  TcParams p;
  p.bias = bias;
  p.scale = sa * sb;
  p.M = M;
  p.N = N;
  p.K = K;
  p.num_m_blocks = (M + v.bm - 1) / v.bm;
  p.num_n_blocks = (N + v.bn - 1) / v.bn;
  p.num_tiles = p.num_m_blocks * p.num_n_blocks;
  p.k_blocks = (K + v.bk_elems - 1) / v.bk_elems;
  p.group_m = std::max(1, std::min(t->TN, p.num_m_blocks));
  p.status = d.scratch;  // word 0 of the fixed scratch area
  p.timeout_ns = kNoallocWaitNs;
  p.tail_split = tail_split_steps();

  ce = cudaMemsetAsync(d.scratch, 0, sizeof(unsigned), s);  // the last call's status must not leak in
  if (ce != cudaSuccess) return noalloc_fail(err, err_len, PF_ECUDA, "cudaMemsetAsync: %s", cudaGetErrorString(ce));
  v.launch_tc(dim3(std::min(p.num_tiles, units) * v.cta_per_tile), s, tmA, tmB, tmC, tmCt, p);
  ce = cudaGetLastError();
  if (ce != cudaSuccess) return noalloc_fail(err, err_len, PF_ECUDA, "launch: %s", cudaGetErrorString(ce));
  if (status_out) {
    unsigned w = 0;
    ce = cudaMemcpyAsync(&w, d.scratch, sizeof w, cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) return noalloc_fail(err, err_len, PF_ECUDA, "status read: %s", cudaGetErrorString(ce));
    *status_out = w;
    if (w) return noalloc_fail(err, err_len, PF_ETIMEOUT, "a bounded device wait ran out (status 0x%x)", w);
  }
  return PF_OK;
}

// ------------------------------------------------------------------------------------------------
// cuBLAS comparator (pf_time_cublas)
// ------------------------------------------------------------------------------------------------
#include "cublas_cmp.cuh"
