// simt_image.cu -- the fp32 SIMT kernel as a standalone image with the reference kernel ABI,
//
//   extern "C" __global__ void gemm_bias_gelu(const float *A, const float *B, const float *bias, float *C,
//                                             int M, int N, int K)          (kernels/gemm_bias_gelu.cu:42-44)
//
// compiled per tile config with -D BM BN BK TM TN PAD (the reference's tunables and flag names,
// kernels/gemm_bias_gelu.cu:16-33, core/include/ptxforge/space.hpp:97-101) and launched on grid
// (ceil(N/BN), ceil(M/BM)), block (BM/TM)*(BN/TN) -- so any image-driven harness (PTXForge's
// `CudaRunner::run_ptx`, or pf_prepare_image) can load, gate and time it.  The B200 runner JIT-compiles
// it for fp32 tiles that libpf_b200.so does not carry precompiled:
//
//   nvcc -cubin -gencode arch=compute_100a,code=sm_100a -O3 -DBM=.. -DBN=.. -DBK=.. -DTM=.. -DTN=.. -DPAD=..
//        -I ptxforge_b200/csrc ptxforge_b200/csrc/simt_image.cu -o k.cubin
//
// 16-byte vector loads: the reference's divisibility rules (M%BM, N%BN, K%BK == 0) and cudaMalloc'd
// operands make every row 16-byte aligned when BN and BK are multiples of 4.
#ifndef BM
#define BM 64
#endif
#ifndef BN
#define BN 64
#endif
#ifndef BK
#define BK 8
#endif
#ifndef TM
#define TM 4
#endif
#ifndef TN
#define TN 4
#endif
#ifndef PAD
#define PAD 0
#endif

// The tile as constants; the macro names are released before the kernel header, whose template
// parameters use the same names.
constexpr int kImgBM = BM, kImgBN = BN, kImgBK = BK, kImgTM = TM, kImgTN = TN, kImgPAD = PAD;
#undef BM
#undef BN
#undef BK
#undef TM
#undef TN
#undef PAD

#include "gemm_simt.cuh"

extern "C" __global__ void __launch_bounds__((kImgBM / kImgTM) * (kImgBN / kImgTN))
    gemm_bias_gelu(const float *__restrict__ A, const float *__restrict__ B, const float *__restrict__ bias,
                   float *__restrict__ C, int M, int N, int K) {
  pf::gemm_bias_gelu_simt_body<kImgBM, kImgBN, kImgBK, kImgTM, kImgTN, kImgPAD, true>(A, B, bias, C, M, N, K);
}
