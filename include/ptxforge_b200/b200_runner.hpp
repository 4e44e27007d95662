// b200_runner.hpp -- B200Runner: PTXForge's Runner interface (core/include/ptxforge/runner.hpp:39-45)
// backed by the sm_100a C ABI of pf_b200.h.  Header-only C++20; compile inside the PTXForge tree
// (it includes "ptxforge/runner.hpp") and link libpf_b200.so.
//
// What measure() does per trial, mirroring CudaRunner (core/src/cuda_runner.cpp:152-217, 255-285):
//   1. maps the tuner's Config onto a pf_tile (same six fields; see pf_b200.h for their meaning on
//      each path) -- an unmappable config is a failed trial, never a crash (cuda_runner.cpp:171-175);
//   2. owns seeded host inputs per problem (CudaRunner::Impl::ensure, cuda_runner.cpp:91-108) in the
//      chosen dtype: fp32 U(-1,1)/sqrt(K); bf16 N(0,1)/sqrt(K) rounded to nearest even; e4m3 N(0,1)
//      quantised with a per-tensor scale amax/448; bias N(0, 0.1);
//   3. with `gpus` > 1 splits rows of M across GPUs (pf_shard_rows), one host thread and pf_ctx per
//      GPU, B and bias replicated, no collective;
//   4. correctness gate FIRST (cuda_runner.cpp:185-203): one launch, C back to the host, `samples`
//      positions from mt19937(99) as r = pick() % M, c = pick() % N, fp64 reference on the
//      (dequantised) inputs, err = |ref - C| / (1 + |ref|), fail unless max_err < tolerance;
//   5. times with the reference protocol (median_ms, cuda_runner.cpp:110-130) via pf_time on every
//      GPU at once behind a barrier; the trial's time is the max over GPUs;
//   6. fills Measurement{ok, gflops, ms, profile{regs, local_bytes, static_smem, blocks_per_sm,
//      occupancy, max_err}, error} (runner.hpp:20-25).
// measure_many() runs up to Options::fanout such trials at once, each on its own group of GPUs; the
// batched search that feeds it is tune_fanout() (ptxforge_b200/tune_fanout.hpp).
#pragma once

#include <algorithm>
#include <barrier>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <mutex>
#include <random>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "pf_b200.h"
#include "ptxforge/runner.hpp"

namespace ptxforge {

// hw.hpp has no B200 row (core/include/ptxforge/hw.hpp:36-49).  peak_gflops is the dense rate of the
// dtype the runner measures (3xTF32: the tf32 rate over its three products per fp32 product);
// smem_per_block is the sm_100 opt-in limit (232,448 B).
inline GPU b200_gpu(pf_dtype dtype = PF_BF16) {
  const double peak = dtype == PF_E4M3          ? 4.5e6
                      : dtype == PF_BF16        ? 2.25e6
                      : dtype == PF_F32_3XTF32  ? 1.125e6 / 3
                                                : 74.4e3;
  return GPU{"b200", "NVIDIA B200", "sm_100a", 148, peak, 8000, 65536, 2048, 32, 233472, 232448, 0.75};
}

inline const char *pf_dtype_name(pf_dtype d) {
  switch (d) {
    case PF_F32: return "f32";
    case PF_F32_3XTF32: return "f32_3xtf32";
    case PF_BF16: return "bf16";
    case PF_E4M3: return "e4m3";
  }
  return "?";
}

inline double pf_default_tolerance(pf_dtype d) { return d == PF_E4M3 ? 5e-2 : d == PF_BF16 ? 2e-2 : 1e-5; }

class B200Runner : public Runner {
 public:
  struct Options {
    pf_dtype dtype = PF_BF16;
    int device = 0;            // first CUDA device used
    int gpus = 1;              // M-row shards, one per device [device, device + gpus)
    int warmup = 5, iters = 20, reps = 5, samples = 512;  // cuda_runner.hpp:29 defaults
    uint64_t seed = 0;
    double tolerance = 0;      // 0: 1e-5 fp32, 2e-2 bf16, 5e-2 e4m3
    std::string root = ".";    // repository root: kernel sources for stages() and the fp32 JIT
    // fp32 tiles that libpf_b200.so does not carry precompiled are compiled per trial with nvcc and
    // loaded through pf_prepare_image, cached on disk (cuda_runner.hpp:28, cuda_runner.cpp:219-237).
    bool jit = true;
    std::string nvcc = "nvcc";
    std::string workdir = "build/kernels";
    // cuBLAS comparator once per problem (cuda_runner.hpp:28 `cublas`, cuda_runner.cpp:132-149):
    // Measurement.cublas_gflops = cuBLAS GEMM alone; cuBLAS + separate bias/GELU via cublas_unfused_gflops().
    bool cublas = true;
    // Trial slots for measure_many(): slot s owns devices [device + s*gpus, device + (s+1)*gpus), so up
    // to `fanout` candidate configs are gated and timed at once, each on its own GPU(s).  measure() uses
    // slot 0 only.
    int fanout = 1;
  };

  explicit B200Runner(Options o) : opt_(std::move(o)) {
    if (opt_.gpus < 1) throw std::runtime_error("B200Runner: gpus must be >= 1");
    if (opt_.fanout < 1) throw std::runtime_error("B200Runner: fanout must be >= 1");
    if (opt_.tolerance <= 0) opt_.tolerance = pf_default_tolerance(opt_.dtype);
    hC_.resize(static_cast<size_t>(opt_.fanout));
    for (int g = 0; g < opt_.gpus * opt_.fanout; ++g) {
      pf_ctx *c = nullptr;
      int rc = pf_open(opt_.device + g, &c);
      if (rc) {
        close_all();
        throw std::runtime_error("pf_open(device " + std::to_string(opt_.device + g) + ") failed with code " +
                                 std::to_string(rc) + " (an sm_100 GPU is required; there is no CPU fallback)");
      }
      ctx_.push_back(c);
    }
  }
  ~B200Runner() override { close_all(); }
  B200Runner(const B200Runner &) = delete;
  B200Runner &operator=(const B200Runner &) = delete;

  std::string source() const override { return "harness"; }

  // Whether a tensor-path Config asks for the 256 x 512 pair tiles (see to_tile).
  static bool wide(const Config &c) { return c.BM == 256 && c.BN == 256 && (c.PAD == 2 || c.PAD == 4); }

  // The tuner's Config onto a pf_tile.  On the tensor-core path the k-block is made of 128-byte swizzle
  // atoms, so BK has no counterpart and is set to 32, and PAD (shared-memory padding in the SIMT kernel)
  // selects the stage layout: PAD=0 one k-atom per stage, PAD=1 or 8 two.  The search domain's columns
  // stop at 256 (space.hpp: BN in {32, 64, 128, 256}), so the 256 x 512 pair tiles are reached through
  // BM=256, BN=256 with PAD=2 (3 stages, two staging boxes per epilogue warp) or PAD=4 (4 stages, one); every
  // (BM, BN, TM, TN) the search proposes then reaches a kernel when one exists.  BM, BN, TM and TN keep the
  // meaning pf_b200.h gives them otherwise.  The fp32 path takes the Config as it is.
  pf_tile to_tile(const Config &c) const {
    pf_tile t{c.BM, c.BN, c.BK, c.TM, c.TN, c.PAD};
    if (opt_.dtype == PF_BF16 || opt_.dtype == PF_E4M3) {
      t.BK = 32;
      if (wide(c)) {
        t.BN = 512;
        t.TM = c.PAD == 2 ? 3 : 4;
        t.PAD = 0;
      } else {
        t.PAD = c.PAD >= 1 ? 1 : 0;
      }
    } else if (opt_.dtype == PF_F32_3XTF32) {
      t.BK = 32;
      t.PAD = 0;
    }
    return t;
  }

  Measurement measure(const Config &cfg, const Problem &p, const GPU &) override {
    try {
      ensure(p);
    } catch (const std::exception &ex) {
      Measurement m;
      m.error = ex.what();
      return m;
    }
    return measure_on(0, cfg, p);
  }

  // Gate and time several configs at once, one per trial slot (Options::fanout); results come back in
  // the order of `cfgs`.  With fanout 1 this is measure() on each config in turn.  Trials that share a
  // batch run on different GPUs of the box at the same time; each is timed on its own GPU(s) only.
  std::vector<Measurement> measure_many(const std::vector<Config> &cfgs, const Problem &p, const GPU &hw) {
    std::vector<Measurement> out(cfgs.size());
    if (opt_.fanout == 1) {
      for (size_t i = 0; i < cfgs.size(); ++i) out[i] = measure(cfgs[i], p, hw);
      return out;
    }
    try {
      ensure(p);  // host inputs are generated once, then only read by the slots
    } catch (const std::exception &ex) {
      for (auto &m : out) m.error = ex.what();
      return out;
    }
    for (size_t b = 0; b < cfgs.size(); b += static_cast<size_t>(opt_.fanout)) {
      const int n = static_cast<int>(std::min(cfgs.size() - b, static_cast<size_t>(opt_.fanout)));
      std::vector<std::thread> th;
      th.reserve(static_cast<size_t>(n));
      for (int s = 0; s < n; ++s) th.emplace_back([&, s] { out[b + s] = measure_on(s, cfgs[b + s], p); });
      for (auto &t : th) t.join();
    }
    // the comparator is measured once per problem, by the first slot to pass; every passing trial reports it
    for (auto &m : out)
      if (m.ok) m.cublas_gflops = cublas_gflops_;
    return out;
  }

  int fanout() const { return opt_.fanout; }

 private:
  // One trial on the contexts of trial slot `slot` (ctx_[slot*gpus .. slot*gpus + gpus)); ensure(p) has run.
  Measurement measure_on(int slot, const Config &cfg, const Problem &p) {
    Measurement m;
    try {
      const pf_tile tile = to_tile(cfg);
      const int G = opt_.gpus;
      pf_ctx *const *cx = ctx_.data() + static_cast<size_t>(slot) * G;
      std::vector<uint8_t> &hc = hC_[static_cast<size_t>(slot)];
      hc.resize(static_cast<size_t>(p.M) * p.N * pf_out_bytes(opt_.dtype));
      const int device0 = opt_.device + slot * G;
      const size_t e = pf_elem_bytes(opt_.dtype), o = pf_out_bytes(opt_.dtype);
      std::vector<int> row0(G), rows(G), rc(G, PF_OK);
      std::vector<std::string> err(G);
      std::vector<double> ms(G, 0.0);
      std::vector<pf_attr> attr(G);
      const int align = cfg.BM;
      for (int g = 0; g < G; ++g)
        if (pf_shard_rows(p.M, G, g, align, &row0[g], &rows[g])) throw std::runtime_error("pf_shard_rows failed");

      // prepare + upload + one gated launch per shard, each on its own host thread
      auto fail = [&](int g, int code) {
        rc[g] = code;
        err[g] = pf_last_error(cx[g]);
      };
      run_shards(G, [&](int g) {
        if (rows[g] == 0) return;
        pf_ctx *c = cx[g];
        int r = pf_prepare(c, opt_.dtype, &tile, rows[g], p.N, p.K);
        if (r == PF_ETILE && opt_.dtype == PF_F32 && opt_.jit) {
          std::string jerr;
          r = prepare_jit(c, cfg, rows[g], p, jerr);
          if (r && !jerr.empty()) {
            rc[g] = r;
            err[g] = jerr;
            return;
          }
        }
        if (r) return fail(g, r);
        if ((r = pf_upload(c, hA_.data() + static_cast<size_t>(row0[g]) * p.K * e, hB_.data(), hbias_.data(), sa_,
                           sb_)))
          return fail(g, r);
        if ((r = pf_attrs(c, &attr[g]))) return fail(g, r);
        if ((r = pf_launch(c, nullptr))) return fail(g, r);
        if ((r = pf_download(c, hc.data() + static_cast<size_t>(row0[g]) * p.N * o))) return fail(g, r);
        unsigned st = 0;
        if ((r = pf_device_status(c, &st))) return fail(g, r);
        if (st) {
          rc[g] = PF_ETIMEOUT;
          err[g] = "bounded device wait ran out (status 0x" + hex(st) + ")";
        }
      });
      for (int g = 0; g < G; ++g)
        if (rc[g]) {
          m.error = (G > 1 ? "gpu " + std::to_string(device0 + g) + ": " : std::string()) + err[g];
          return m;
        }
      const pf_attr &a0 = attr[first_nonempty(rows)];
      m.profile.regs = a0.regs;
      m.profile.local_bytes = a0.local_bytes;
      m.profile.static_smem = a0.smem_bytes;
      m.profile.blocks_per_sm = a0.blocks_per_sm;
      m.profile.occupancy = std::round(1e4 * a0.blocks_per_sm * a0.threads / 2048.0) / 1e4;

      // correctness gate first: never report speed for a wrong kernel
      const double max_err = gate(p, hc);
      m.profile.max_err = max_err;
      if (!(max_err < opt_.tolerance)) {
        m.error = "incorrect result (max_err=" + std::to_string(max_err) + ", tolerance " +
                  std::to_string(opt_.tolerance) + ")";
        return m;
      }

      // timing: every shard at once, behind a barrier; the trial's time is the slowest shard's
      std::barrier sync(G);
      run_shards(G, [&](int g) {
        sync.arrive_and_wait();
        if (rows[g] == 0) return;
        int r = pf_time(cx[g], opt_.warmup, opt_.iters, opt_.reps, &ms[g]);
        if (r) fail(g, r);
      });
      for (int g = 0; g < G; ++g)
        if (rc[g]) {
          m.error = "timing: " + err[g];
          return m;
        }
      const double t = *std::max_element(ms.begin(), ms.end());
      m.ok = true;
      m.ms = t;
      m.gflops = p.flops() / (t * 1e6);

      // cuBLAS comparator, once per problem, on the same shards at once (failures leave it unset, as
      // the reference's measure_cublas does when cuBLAS cannot be created); the first trial slot to pass
      // measures it while the others wait
      std::unique_lock<std::mutex> cmp_lock(cmp_mutex_);
      if (opt_.cublas && !cublas_gflops_) {
        std::vector<double> g_ms(G, 0.0), u_ms(G, 0.0);
        std::vector<int> crc(G, PF_OK);
        std::barrier sync2(G);
        run_shards(G, [&](int g) {
          sync2.arrive_and_wait();
          if (rows[g] == 0) return;
          crc[g] = pf_time_cublas(cx[g], opt_.warmup, opt_.iters, opt_.reps, &g_ms[g], &u_ms[g]);
        });
        if (std::all_of(crc.begin(), crc.end(), [](int r) { return r == PF_OK; })) {
          cublas_gflops_ = p.flops() / (*std::max_element(g_ms.begin(), g_ms.end()) * 1e6);
          cublas_unfused_gflops_ = p.flops() / (*std::max_element(u_ms.begin(), u_ms.end()) * 1e6);
        }
      }
      m.cublas_gflops = cublas_gflops_;
    } catch (const std::exception &ex) {
      m.ok = false;
      m.error = ex.what();
    }
    return m;
  }

 public:
  std::vector<Stage> stages(const Config &c, const Problem &, const GPU &) override {
    // Source only.  Compiler-written PTX/SASS of this build is never embedded in a trace.
    const std::string dir = opt_.root + "/ptxforge_b200/csrc/";
    const bool tensor = opt_.dtype == PF_BF16 || opt_.dtype == PF_E4M3;
    const std::string file = opt_.dtype == PF_F32_3XTF32 ? "gemm_tf32x3.cuh"
                             : !tensor                   ? "gemm_simt.cuh"
                             : wide(c)                   ? "gemm_tc2w.cuh"
                             : (c.BM == 256 ? "gemm_tc2.cuh" : "gemm_tc.cuh");
    std::string src;
    try {
      src = read_file(dir + file);
    } catch (const std::exception &) {
      src = "// " + dir + file + " not found";
    }
    std::string note = "// tile " + c.short_name() + ", dtype " + pf_dtype_name(opt_.dtype) +
                       ": kernels are built ahead of time for sm_100a (python -m ptxforge_b200.build); "
                       "compiler-written PTX and SASS are not embedded in traces.";
    return {{"CUDA C++ source", "cuda", "// " + file + "\n" + src},
            {"LLVM IR", "llvm", "// nvcc does not expose LLVM IR for this backend."},
            {"PTX", "ptx", note}};
  }

  const Options &options() const { return opt_; }

  // cuBLAS GEMM followed by a separate bias + GELU kernel on the current problem (GFLOP/s), if measured.
  std::optional<double> cublas_unfused_gflops() const { return cublas_unfused_gflops_; }

 private:
  // nvcc the fp32 SIMT kernel (ptxforge_b200/csrc/simt_image.cu, reference kernel ABI) for this tile
  // into workdir (cached; serialised across shard threads) and load it with pf_prepare_image on the
  // reference launch shape: grid (ceil(N/BN), ceil(rows/BM)), block (BM/TM)*(BN/TN).
  int prepare_jit(pf_ctx *c, const Config &cfg, int rows, const Problem &p, std::string &err) {
    const std::string name = "simt_" + std::to_string(cfg.BM) + "_" + std::to_string(cfg.BN) + "_" +
                             std::to_string(cfg.BK) + "_" + std::to_string(cfg.TM) + "_" + std::to_string(cfg.TN) +
                             "_" + std::to_string(cfg.PAD) + ".cubin";
    const std::string path = opt_.workdir + "/" + name;
    std::string image;
    {
      std::lock_guard<std::mutex> lock(jit_mutex_);
      std::ifstream probe(path, std::ios::binary);
      if (!probe) {
        std::string mk = "mkdir -p '" + opt_.workdir + "'";
        if (std::system(mk.c_str()) != 0) {
          err = "cannot create " + opt_.workdir;
          return PF_ETILE;
        }
        const std::string src = opt_.root + "/ptxforge_b200/csrc/simt_image.cu";
        std::string cmd = opt_.nvcc + " -cubin -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo";
        for (const auto &d : cfg.defines()) cmd += " " + d;
        cmd += " -I '" + opt_.root + "/ptxforge_b200/csrc' '" + src + "' -o '" + path + ".tmp' 2>&1";
        std::string log;
        FILE *pipe = popen(cmd.c_str(), "r");
        if (!pipe) {
          err = "cannot run nvcc";
          return PF_ETILE;
        }
        char buf[4096];
        size_t n;
        while ((n = fread(buf, 1, sizeof buf, pipe)) > 0) log.append(buf, n);
        if (pclose(pipe) != 0) {
          std::remove((path + ".tmp").c_str());
          err = "nvcc failed: " + log.substr(log.size() > 800 ? log.size() - 800 : 0);
          return PF_ETILE;
        }
        std::rename((path + ".tmp").c_str(), path.c_str());
      }
      image = read_file(path);
    }
    const int gx = (p.N + cfg.BN - 1) / cfg.BN, gy = (rows + cfg.BM - 1) / cfg.BM;
    return pf_prepare_image(c, image.data(), image.size(), "gemm_bias_gelu", gx, gy, cfg.threads(), rows, p.N, p.K);
  }

  static std::string hex(unsigned v) {
    std::ostringstream s;
    s << std::hex << v;
    return s.str();
  }
  static int first_nonempty(const std::vector<int> &rows) {
    for (size_t g = 0; g < rows.size(); ++g)
      if (rows[g] > 0) return static_cast<int>(g);
    return 0;
  }

  template <class F>
  static void run_shards(int G, F &&f) {
    if (G == 1) {
      f(0);
      return;
    }
    std::vector<std::thread> th;
    th.reserve(G);
    for (int g = 0; g < G; ++g) th.emplace_back([&f, g] { f(g); });
    for (auto &t : th) t.join();
  }

  void close_all() {
    for (pf_ctx *c : ctx_) pf_close(c);
    ctx_.clear();
  }

  static uint16_t bf16_rne(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(u >> 16);
  }

  // e4m3 value of a code: sign, 4 exponent bits (bias 7), 3 mantissa bits; 0x7f / 0xff are NaN.
  static float e4m3_value(uint8_t v) {
    const int s = v >> 7, ex = (v >> 3) & 15, mt = v & 7;
    if (ex == 15 && mt == 7) return NAN;
    const float mag = ex == 0 ? std::ldexp(static_cast<float>(mt), -9) : std::ldexp(1.0f + mt / 8.0f, ex - 7);
    return s ? -mag : mag;
  }

  // Round to the nearest e4m3 code (ties to even mantissa), saturating at +-448.
  static uint8_t e4m3_rne(float x) {
    const uint8_t sign = std::signbit(x) ? 0x80 : 0x00;
    float a = std::fabs(x);
    if (!(a < 448.0f)) return sign | 0x7e;
    int lo = 0, hi = 0x7e;
    while (lo < hi) {
      const int mid = (lo + hi + 1) / 2;
      if (e4m3_value(static_cast<uint8_t>(mid)) <= a) lo = mid; else hi = mid - 1;
    }
    if (lo < 0x7e) {
      const float d0 = a - e4m3_value(static_cast<uint8_t>(lo)), d1 = e4m3_value(static_cast<uint8_t>(lo + 1)) - a;
      if (d1 < d0 || (d1 == d0 && (lo & 1))) ++lo;
    }
    return sign | static_cast<uint8_t>(lo);
  }

  // Seeded inputs for problem p in the runner's dtype (host copies in the kernel's encoding plus the
  // exact values as doubles-to-be for the gate).
  void ensure(const Problem &p) {
    if (p.M == prob_.M && p.N == prob_.N && p.K == prob_.K && !hA_.empty()) return;
    prob_ = p;
    cublas_gflops_.reset();
    cublas_unfused_gflops_.reset();
    const size_t nA = static_cast<size_t>(p.M) * p.K, nB = static_cast<size_t>(p.K) * p.N;
    const size_t e = pf_elem_bytes(opt_.dtype), o = pf_out_bytes(opt_.dtype);
    std::vector<float> A(nA), B(nB);
    vbias_.assign(static_cast<size_t>(p.N), 0.f);
    std::mt19937_64 ra(opt_.seed * 3 + 1), rb(opt_.seed * 3 + 2), rbias(opt_.seed * 3 + 3);
    const float inv_sqrt_k = 1.0f / std::sqrt(static_cast<float>(p.K));
    if (opt_.dtype == PF_F32 || opt_.dtype == PF_F32_3XTF32) {
      std::uniform_real_distribution<float> U(-1.f, 1.f);
      for (auto &v : A) v = U(ra) * inv_sqrt_k;
      for (auto &v : B) v = U(rb) * inv_sqrt_k;
    } else {
      std::normal_distribution<float> Nd(0.f, 1.f);
      const float s = opt_.dtype == PF_BF16 ? inv_sqrt_k : 1.0f;
      for (auto &v : A) v = Nd(ra) * s;
      for (auto &v : B) v = Nd(rb) * s;
    }
    std::normal_distribution<float> Nb(0.f, 0.1f);
    for (auto &v : vbias_) v = Nb(rbias);
    hbias_ = vbias_;
    hA_.assign(nA * e, 0);
    hB_.assign(nB * e, 0);
    vA_.resize(nA);
    vB_.resize(nB);
    sa_ = sb_ = 1.f;
    if (e == 4) {
      std::memcpy(hA_.data(), A.data(), nA * 4);
      std::memcpy(hB_.data(), B.data(), nB * 4);
      vA_ = A;
      vB_ = B;
    } else if (opt_.dtype == PF_BF16) {
      auto *a16 = reinterpret_cast<uint16_t *>(hA_.data());
      auto *b16 = reinterpret_cast<uint16_t *>(hB_.data());
      for (size_t i = 0; i < nA; ++i) {
        a16[i] = bf16_rne(A[i]);
        uint32_t u = static_cast<uint32_t>(a16[i]) << 16;
        std::memcpy(&vA_[i], &u, 4);
      }
      for (size_t i = 0; i < nB; ++i) {
        b16[i] = bf16_rne(B[i]);
        uint32_t u = static_cast<uint32_t>(b16[i]) << 16;
        std::memcpy(&vB_[i], &u, 4);
      }
    } else {
      auto quant = [&](const std::vector<float> &x, uint8_t *q, std::vector<float> &v, float &scale) {
        float amax = 0.f;
        for (float f : x) amax = std::max(amax, std::fabs(f));
        scale = amax > 0 ? amax / 448.0f : 1.0f;
        float lut[256];
        for (int c = 0; c < 256; ++c) lut[c] = e4m3_value(static_cast<uint8_t>(c));
        for (size_t i = 0; i < x.size(); ++i) {
          q[i] = e4m3_rne(x[i] / scale);
          v[i] = lut[q[i]];
        }
      };
      quant(A, hA_.data(), vA_, sa_);
      quant(B, hB_.data(), vB_, sb_);
    }
  }

  // The reference gate (cuda_runner.cpp:189-197) over the gathered C.  A NaN at a sampled position
  // fails the trial.
  double gate(const Problem &p, const std::vector<uint8_t> &hc) const {
    const size_t o = pf_out_bytes(opt_.dtype);
    const double scale = static_cast<double>(sa_) * sb_;
    std::mt19937 pick(99);
    double max_err = 0;
    for (int s = 0; s < opt_.samples; ++s) {
      const int r = static_cast<int>(pick() % static_cast<unsigned>(p.M));
      const int c = static_cast<int>(pick() % static_cast<unsigned>(p.N));
      double acc = 0;
      for (int k = 0; k < p.K; ++k)
        acc += static_cast<double>(vA_[static_cast<size_t>(r) * p.K + k]) * vB_[static_cast<size_t>(k) * p.N + c];
      const double x = acc * scale + vbias_[static_cast<size_t>(c)];
      const double ref = 0.5 * x * (1.0 + std::tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)));
      const size_t idx = static_cast<size_t>(r) * p.N + c;
      float got;
      if (o == 4) {
        std::memcpy(&got, hc.data() + idx * 4, 4);
      } else {
        uint16_t h;
        std::memcpy(&h, hc.data() + idx * 2, 2);
        const uint32_t u = static_cast<uint32_t>(h) << 16;
        std::memcpy(&got, &u, 4);
      }
      const double err = std::fabs(ref - got) / (1.0 + std::fabs(ref));
      if (std::isnan(err)) return NAN;
      max_err = std::max(max_err, err);
    }
    return max_err;
  }

  Options opt_;
  std::vector<pf_ctx *> ctx_;
  Problem prob_{0, 0, 0};
  std::vector<uint8_t> hA_, hB_;
  std::vector<std::vector<uint8_t>> hC_;  // C on the host, one per trial slot
  std::vector<float> hbias_, vbias_, vA_, vB_;
  float sa_ = 1.f, sb_ = 1.f;
  std::mutex jit_mutex_, cmp_mutex_;
  std::optional<double> cublas_gflops_, cublas_unfused_gflops_;
};

}  // namespace ptxforge
