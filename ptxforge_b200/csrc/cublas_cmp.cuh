// cublas_cmp.cuh -- pf_time_cublas: the cuBLAS comparator (included at the end of pf_b200.cu, which
// defines pf_ctx).  cublasLt is opened with dlopen on first use, so libpf_b200.so has no link-time
// dependency on it and still loads where it is absent.
//
//   gemm alone      cublasLt GEMM of the bound operands into a scratch D (CudaRunner::Impl::measure_cublas,
//                   core/src/cuda_runner.cpp:132-149, times cublasSgemm the same way: row-major C = A.B as
//                   column-major C^T = B^T.A^T)
//   unfused         the same GEMM, then a separate kernel C = gelu_tanh(D + bias) -- what a framework without
//                   the fused kernel runs (scripts/run_ptx_on_gpu.py:88-90)
#pragma once

#include <cublasLt.h>
#include <dlfcn.h>

namespace {

struct LtApi {
  decltype(&cublasLtCreate) create = nullptr;
  decltype(&cublasLtDestroy) destroy = nullptr;
  decltype(&cublasLtMatmulDescCreate) desc_create = nullptr;
  decltype(&cublasLtMatmulDescDestroy) desc_destroy = nullptr;
  decltype(&cublasLtMatmulDescSetAttribute) desc_set = nullptr;
  decltype(&cublasLtMatrixLayoutCreate) layout_create = nullptr;
  decltype(&cublasLtMatrixLayoutDestroy) layout_destroy = nullptr;
  decltype(&cublasLtMatmulPreferenceCreate) pref_create = nullptr;
  decltype(&cublasLtMatmulPreferenceDestroy) pref_destroy = nullptr;
  decltype(&cublasLtMatmulPreferenceSetAttribute) pref_set = nullptr;
  decltype(&cublasLtMatmulAlgoGetHeuristic) heuristic = nullptr;
  decltype(&cublasLtMatmul) matmul = nullptr;
  bool ok = false;
  std::string err;
};

const LtApi &lt_api() {
  static LtApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = nullptr;
    for (const char *name : {"libcublasLt.so.12", "/usr/local/cuda/lib64/libcublasLt.so.12", "libcublasLt.so"})
      if ((h = dlopen(name, RTLD_NOW | RTLD_GLOBAL)) != nullptr) break;
    if (!h) {
      api.err = "cannot open libcublasLt";
      return;
    }
    auto sym = [&](auto &field, const char *name) {
      field = reinterpret_cast<std::remove_reference_t<decltype(field)>>(dlsym(h, name));
      if (!field && api.err.empty()) api.err = std::string("libcublasLt lacks ") + name;
    };
    sym(api.create, "cublasLtCreate");
    sym(api.destroy, "cublasLtDestroy");
    sym(api.desc_create, "cublasLtMatmulDescCreate");
    sym(api.desc_destroy, "cublasLtMatmulDescDestroy");
    sym(api.desc_set, "cublasLtMatmulDescSetAttribute");
    sym(api.layout_create, "cublasLtMatrixLayoutCreate");
    sym(api.layout_destroy, "cublasLtMatrixLayoutDestroy");
    sym(api.pref_create, "cublasLtMatmulPreferenceCreate");
    sym(api.pref_destroy, "cublasLtMatmulPreferenceDestroy");
    sym(api.pref_set, "cublasLtMatmulPreferenceSetAttribute");
    sym(api.heuristic, "cublasLtMatmulAlgoGetHeuristic");
    sym(api.matmul, "cublasLtMatmul");
    api.ok = api.err.empty();
  });
  return api;
}

template <typename T>
__device__ __forceinline__ float to_f32(T v) {
  return static_cast<float>(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T>
__device__ __forceinline__ T from_f32(float v) {
  return static_cast<T>(v);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// The separate epilogue pass: C[r,c] = gelu_tanh(D[r,c] + bias[c]), grid-stride, one element per step.
template <typename T>
__global__ void bias_gelu_pass(const T *__restrict__ D, const float *__restrict__ bias, T *__restrict__ C, int M,
                               int N) {
  const size_t total = static_cast<size_t>(M) * N;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float x = to_f32(D[i]) + bias[i % N];
    C[i] = from_f32<T>(pf::gelu_tanh_ref_f32(x));
  }
}

// B [K x N] bytes -> Bt [N x K] (untimed set-up of the fp8 comparator).
__global__ void transpose_bytes(const uint8_t *__restrict__ in, uint8_t *__restrict__ out, int K, int N) {
  __shared__ uint8_t tile[32][33];
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int k = k0 + i, n = n0 + threadIdx.x;
    if (k < K && n < N) tile[i][threadIdx.x] = in[static_cast<size_t>(k) * N + n];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int n = n0 + i, k = k0 + threadIdx.x;
    if (k < K && n < N) out[static_cast<size_t>(n) * K + k] = tile[threadIdx.x][i];
  }
}

int grow(pf_ctx *c, void **buf, size_t *cap, size_t need) {
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
}

// Median per-launch time of `fn` with the reference protocol on the context's stream.
template <class F>
int median_time(pf_ctx *c, F &&fn, int warmup, int iters, int reps, double *out) {
  for (int i = 0; i < warmup; ++i)
    if (int rc = fn()) return rc;
  PF_CUDA(c, cudaStreamSynchronize(c->stream));
  std::vector<double> per;
  for (int r = 0; r < reps; ++r) {
    PF_CUDA(c, cudaEventRecord(c->ev0, c->stream));
    for (int i = 0; i < iters; ++i)
      if (int rc = fn()) return rc;
    PF_CUDA(c, cudaEventRecord(c->ev1, c->stream));
    PF_CUDA(c, cudaEventSynchronize(c->ev1));
    float ms = 0.f;
    PF_CUDA(c, cudaEventElapsedTime(&ms, c->ev0, c->ev1));
    per.push_back(static_cast<double>(ms) / iters);
  }
  std::sort(per.begin(), per.end());
  *out = per[per.size() / 2];
  return PF_OK;
}

}  // namespace

void cublas_cmp_release(pf_ctx *c) {
  if (c->lt_handle && lt_api().ok) lt_api().destroy(static_cast<cublasLtHandle_t>(c->lt_handle));
  for (void *p : {c->lt_ws, c->lt_D, c->lt_Bt, static_cast<void *>(c->lt_scales)})
    if (p) cudaFree(p);
  c->lt_handle = c->lt_ws = c->lt_D = c->lt_Bt = nullptr;
  c->lt_scales = nullptr;
}

extern "C" int pf_time_cublas(pf_ctx *c, int warmup, int iters, int reps, double *gemm_ms, double *unfused_ms) {
  if (!c || !gemm_ms || !unfused_ms || warmup < 0 || iters <= 0 || reps <= 0)
    return set_err(c, PF_EINVAL, "bad arguments");
  if (!c->prepared || !c->bound) return set_err(c, PF_ESTATE, "pf_time_cublas before pf_prepare / pf_bind");
  const LtApi &lt = lt_api();
  if (!lt.ok) return set_err(c, PF_ECUDA, "cuBLAS comparator unavailable: %s", lt.err.c_str());
  DeviceGuard g(c->device);
  const int M = c->M, N = c->N, K = c->K;
  const bool f8 = c->dtype == PF_E4M3, f32 = c->dtype == PF_F32 || c->dtype == PF_F32_3XTF32;
  const size_t ob = pf_out_bytes(c->dtype);
  int rc;
  if (!c->lt_handle) {
    cublasLtHandle_t h;
    if (lt.create(&h) != CUBLAS_STATUS_SUCCESS) return set_err(c, PF_ECUDA, "cublasLtCreate failed");
    c->lt_handle = h;
  }
  const size_t ws_bytes = 64u << 20;
  if ((rc = grow(c, &c->lt_ws, &c->lt_ws_cap, ws_bytes)) ||
      (rc = grow(c, &c->lt_D, &c->lt_D_cap, static_cast<size_t>(M) * N * ob)))
    return rc;
  const void *cubA = c->B;  // column-major view: C^T (N x M) = B^T (N x K) . A^T (K x M)
  if (f8) {
    if ((rc = grow(c, &c->lt_Bt, &c->lt_Bt_cap, static_cast<size_t>(K) * N))) return rc;
    transpose_bytes<<<dim3((N + 31) / 32, (K + 31) / 32), dim3(32, 8), 0, c->stream>>>(
        static_cast<const uint8_t *>(c->B), static_cast<uint8_t *>(c->lt_Bt), K, N);
    PF_CUDA(c, cudaGetLastError());
    if (!c->lt_scales) {
      void *p = nullptr;
      PF_CUDA(c, cudaMalloc(&p, 2 * sizeof(float)));
      c->lt_scales = static_cast<float *>(p);
    }
    const float sc[2] = {c->sb, c->sa};  // cuBLAS's A is our B, its B is our A
    PF_CUDA(c, cudaMemcpyAsync(c->lt_scales, sc, sizeof sc, cudaMemcpyHostToDevice, c->stream));
    cubA = c->lt_Bt;
  }
  const cudaDataType_t in_t = f32 ? CUDA_R_32F : f8 ? CUDA_R_8F_E4M3 : CUDA_R_16BF;
  const cudaDataType_t out_t = f32 ? CUDA_R_32F : CUDA_R_16BF;
  cublasLtMatmulDesc_t desc = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, ld = nullptr;
  cublasLtMatmulPreference_t pref = nullptr;
  auto cleanup = [&] {
    if (pref) lt.pref_destroy(pref);
    if (ld) lt.layout_destroy(ld);
    if (lb) lt.layout_destroy(lb);
    if (la) lt.layout_destroy(la);
    if (desc) lt.desc_destroy(desc);
  };
  const cublasOperation_t opA = f8 ? CUBLAS_OP_T : CUBLAS_OP_N, opB = CUBLAS_OP_N;
  bool ok = lt.desc_create(&desc, CUBLAS_COMPUTE_32F, CUDA_R_32F) == CUBLAS_STATUS_SUCCESS &&
            lt.desc_set(desc, CUBLASLT_MATMUL_DESC_TRANSA, &opA, sizeof opA) == CUBLAS_STATUS_SUCCESS &&
            lt.desc_set(desc, CUBLASLT_MATMUL_DESC_TRANSB, &opB, sizeof opB) == CUBLAS_STATUS_SUCCESS;
  if (ok && f8) {
    const float *sa_ptr = c->lt_scales, *sb_ptr = c->lt_scales + 1;
    ok = lt.desc_set(desc, CUBLASLT_MATMUL_DESC_A_SCALE_POINTER, &sa_ptr, sizeof sa_ptr) == CUBLAS_STATUS_SUCCESS &&
         lt.desc_set(desc, CUBLASLT_MATMUL_DESC_B_SCALE_POINTER, &sb_ptr, sizeof sb_ptr) == CUBLAS_STATUS_SUCCESS;
  }
  // cuBLAS A: N x K (ld N), or for fp8 the K x N stored Bt transposed (ld K); cuBLAS B: K x M (ld K).
  ok = ok &&
       (f8 ? lt.layout_create(&la, in_t, K, N, K) : lt.layout_create(&la, in_t, N, K, N)) == CUBLAS_STATUS_SUCCESS &&
       lt.layout_create(&lb, in_t, K, M, K) == CUBLAS_STATUS_SUCCESS &&
       lt.layout_create(&ld, out_t, N, M, N) == CUBLAS_STATUS_SUCCESS &&
       lt.pref_create(&pref) == CUBLAS_STATUS_SUCCESS &&
       lt.pref_set(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws_bytes, sizeof ws_bytes) == CUBLAS_STATUS_SUCCESS;
  cublasLtMatmulHeuristicResult_t heur = {};
  int found = 0;
  ok = ok && lt.heuristic(static_cast<cublasLtHandle_t>(c->lt_handle), desc, la, lb, ld, ld, pref, 1, &heur, &found) ==
                 CUBLAS_STATUS_SUCCESS &&
       found > 0;
  if (!ok) {
    cleanup();
    return set_err(c, PF_ECUDA, "cublasLt set-up or heuristic failed for %dx%dx%d", M, N, K);
  }
  const float alpha = 1.f, beta = 0.f;
  auto gemm = [&]() -> int {
    if (lt.matmul(static_cast<cublasLtHandle_t>(c->lt_handle), desc, &alpha, cubA, la, c->A, lb, &beta, c->lt_D, ld,
                  c->lt_D, ld, &heur.algo, c->lt_ws, ws_bytes, c->stream) != CUBLAS_STATUS_SUCCESS)
      return set_err(c, PF_ECUDA, "cublasLtMatmul failed");
    return PF_OK;
  };
  const int blocks = 4 * c->num_sms;
  auto unfused = [&]() -> int {
    if (int r = gemm()) return r;
    if (f32)
      bias_gelu_pass<float><<<blocks, 256, 0, c->stream>>>(static_cast<const float *>(c->lt_D), c->bias,
                                                           static_cast<float *>(c->C), M, N);
    else
      bias_gelu_pass<__nv_bfloat16><<<blocks, 256, 0, c->stream>>>(
          static_cast<const __nv_bfloat16 *>(c->lt_D), c->bias, static_cast<__nv_bfloat16 *>(c->C), M, N);
    PF_CUDA(c, cudaGetLastError());
    return PF_OK;
  };
  rc = median_time(c, gemm, warmup, iters, reps, gemm_ms);
  if (!rc) rc = median_time(c, unfused, warmup, iters, reps, unfused_ms);
  cleanup();
  if (!rc) {
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return set_err(c, PF_ECUDA, "cuBLAS comparator: %s", cudaGetErrorString(e));
  }
  return rc;
}
