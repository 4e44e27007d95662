// ref_kernel_launch.cu -- TEST INFRASTRUCTURE ONLY: a launcher around the reference's own fp32
// kernel, so the GPU parity tests can run the unmodified reference kernel (kernels/gemm_bias_gelu.cu,
// compiled for sm_100a with its -D tile macros as core/src/cuda_runner.cpp:228-230 does) on the same
// inputs as this backend.  oracle/build.py compiles it with -include <reference kernel path>; the
// reference source is read where it lies and never copied.  Output goes to oracle/_ref/.
//
// The reference kernel (kernels/gemm_bias_gelu.cu:42-44) is
//   extern "C" __global__ gemm_bias_gelu(const float *A, const float *B, const float *bias, float *C,
//                                        int M, int N, int K)
// launched on grid (N/BN, M/BM), block (BM/TM)*(BN/TN) (kernels/gemm_bias_gelu.cu:15).
#include <cuda_runtime.h>

#ifndef THREADS
#error "compile with -include <reference>/kernels/gemm_bias_gelu.cu"
#endif

extern "C" int ref_tile(int *bm, int *bn, int *bk, int *tm, int *tn, int *pad) {
  *bm = BM;
  *bn = BN;
  *bk = BK;
  *tm = TM;
  *tn = TN;
  *pad = PAD;
  return 0;
}

// Returns 0, or a cudaError_t.  The reference kernel has no bounds checks, so sizes must be
// multiples of the tile (kernels/gemm_bias_gelu.cu:12-13); -1 if they are not.
extern "C" int ref_launch(const float *A, const float *B, const float *bias, float *C, int M, int N, int K,
                          void *stream) {
  if (M % BM || N % BN || K % BK) return -1;
  dim3 grid(N / BN, M / BM);
  gemm_bias_gelu<<<grid, THREADS, 0, static_cast<cudaStream_t>(stream)>>>(A, B, bias, C, M, N, K);
  return static_cast<int>(cudaGetLastError());
}
