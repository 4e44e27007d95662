// gemm_simt.cuh -- fp32 fused C = gelu_tanh(A.B + bias) on the CUDA cores (FFMA), sm_100a.
//
// Same tile parameters as the reference's tunable kernel (kernels/gemm_bias_gelu.cu:16-33):
// a BM x BN block tile, K walked in steps of BK, a TM x TN register micro-tile per thread and
// PAD floats of padding per row of the transposed A tile in shared memory.  Differences, for speed
// on B200:
//   * double-buffered shared memory with a register-staged prefetch of the next K step, so one
//     barrier per K step instead of two (tiles whose two stages exceed 48 KB keep one stage);
//   * 16-byte global loads and stores; A is transposed on its way into shared memory;
//   * when TM and TN are multiples of 4 (and BM + PAD too, for A) a thread owns 4 x 4 sub-blocks spread BM/(TM/4) rows and
//     BN/(TN/4) columns apart, so its shared-memory reads are conflict-free float4 loads;
//   * ragged M / N / K are allowed (out-of-range loads read 0, stores are guarded).
// Numerics match the reference kernel element for element: every C[r,c] is accumulated in fp32 by
// fmaf over k = 0, 1, ..., K-1 from 0, then gelu_tanh(acc + bias[c]) is evaluated in the same
// expression form with tanhf (kernels/gemm_bias_gelu.cu:37-40, 75-84, 89-97).
#pragma once

#include <cstdint>

namespace pf {

__device__ __forceinline__ float gelu_tanh_ref_f32(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x * x * x)));
}

template <int BM, int BN, int BK, int TM, int TN, int PAD>
struct SimtConfig {
  static constexpr int THREADS = (BM / TM) * (BN / TN);
  static constexpr int TX = BN / TN;  // threads along N
  static constexpr int TY = BM / TM;  // threads along M
  // float4 reads of the transposed A tile need 16-byte rows: BM + PAD a multiple of 4 floats.
  static constexpr bool SPLIT_M = (TM % 4 == 0) && ((BM + PAD) % 4 == 0);
  static constexpr bool SPLIT_N = (TN % 4 == 0);
  static constexpr int A_VEC = BM * BK / 4;  // float4 pieces of the A tile
  static constexpr int B_VEC = BK * BN / 4;  // float4 pieces of the B tile
  static constexpr int A_PER = (A_VEC + THREADS - 1) / THREADS;
  static constexpr int B_PER = (B_VEC + THREADS - 1) / THREADS;
  static constexpr int STAGE_BYTES = 4 * (BK * (BM + PAD) + BK * BN);
  // Double-buffered when two stages fit the 48 KB of static shared memory, else one stage with two
  // barriers per K step (as the reference kernel).  Either way every output is the same fmaf chain.
  static constexpr int STAGES = 2 * STAGE_BYTES <= 48 * 1024 ? 2 : 1;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES;
  static_assert(BM % TM == 0 && BN % TN == 0, "tile not divisible by micro-tile");
  static_assert(BK % 4 == 0 && BN % 4 == 0, "BK and BN must be multiples of 4");
  static_assert(SMEM_BYTES <= 48 * 1024, "static shared memory above 48 KB");
};

// Row of micro-tile element i for thread row ty (and likewise columns).
template <int BM, int TM, bool SPLIT>
__device__ __forceinline__ int micro_index(int ty, int i) {
  if constexpr (SPLIT) {
    return (i >> 2) * (BM / (TM / 4)) + ty * 4 + (i & 3);
  } else {
    return ty * TM + i;
  }
}

// The kernel body, shared by the templated kernel below and by the standalone image with the
// reference ABI (simt_image.cu).
template <int BM, int BN, int BK, int TM, int TN, int PAD, bool VEC>
__device__ __forceinline__ void gemm_bias_gelu_simt_body(const float *__restrict__ A, const float *__restrict__ B,
                                                         const float *__restrict__ bias, float *__restrict__ C,
                                                         int M, int N, int K) {
  using Cfg = SimtConfig<BM, BN, BK, TM, TN, PAD>;
  __shared__ __align__(16) float As[Cfg::STAGES][BK][BM + PAD];  // transposed: As[k][m]
  __shared__ __align__(16) float Bs[Cfg::STAGES][BK][BN];

  const int tid = threadIdx.x;
  const int tx = tid % Cfg::TX;
  const int ty = tid / Cfg::TX;
  const int row0 = blockIdx.y * BM;
  const int col0 = blockIdx.x * BN;

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  float4 ra[Cfg::A_PER], rb[Cfg::B_PER];

  auto load_tiles = [&](int k0) {
#pragma unroll
    for (int l = 0; l < Cfg::A_PER; ++l) {
      const int idx = tid + l * Cfg::THREADS;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (idx < Cfg::A_VEC) {
        const int r = idx / (BK / 4), kq = idx % (BK / 4);
        const int gr = row0 + r, gk = k0 + kq * 4;
        if (gr < M) {
          const float *src = A + static_cast<size_t>(gr) * K + gk;
          if constexpr (VEC) {
            if (gk < K) v = __ldg(reinterpret_cast<const float4 *>(src));
          } else {
            if (gk + 0 < K) v.x = __ldg(src + 0);
            if (gk + 1 < K) v.y = __ldg(src + 1);
            if (gk + 2 < K) v.z = __ldg(src + 2);
            if (gk + 3 < K) v.w = __ldg(src + 3);
          }
        }
      }
      ra[l] = v;
    }
#pragma unroll
    for (int l = 0; l < Cfg::B_PER; ++l) {
      const int idx = tid + l * Cfg::THREADS;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (idx < Cfg::B_VEC) {
        const int r = idx / (BN / 4), cq = idx % (BN / 4);
        const int gk = k0 + r, gc = col0 + cq * 4;
        if (gk < K) {
          const float *src = B + static_cast<size_t>(gk) * N + gc;
          if constexpr (VEC) {
            if (gc < N) v = __ldg(reinterpret_cast<const float4 *>(src));
          } else {
            if (gc + 0 < N) v.x = __ldg(src + 0);
            if (gc + 1 < N) v.y = __ldg(src + 1);
            if (gc + 2 < N) v.z = __ldg(src + 2);
            if (gc + 3 < N) v.w = __ldg(src + 3);
          }
        }
      }
      rb[l] = v;
    }
  };

  auto store_tiles = [&](int buf) {
#pragma unroll
    for (int l = 0; l < Cfg::A_PER; ++l) {
      const int idx = tid + l * Cfg::THREADS;
      if (idx < Cfg::A_VEC) {
        const int r = idx / (BK / 4), kq = idx % (BK / 4);
        As[buf][kq * 4 + 0][r] = ra[l].x;
        As[buf][kq * 4 + 1][r] = ra[l].y;
        As[buf][kq * 4 + 2][r] = ra[l].z;
        As[buf][kq * 4 + 3][r] = ra[l].w;
      }
    }
#pragma unroll
    for (int l = 0; l < Cfg::B_PER; ++l) {
      const int idx = tid + l * Cfg::THREADS;
      if (idx < Cfg::B_VEC) {
        const int r = idx / (BN / 4), cq = idx % (BN / 4);
        *reinterpret_cast<float4 *>(&Bs[buf][r][cq * 4]) = rb[l];
      }
    }
  };

  const int ktiles = (K + BK - 1) / BK;
  load_tiles(0);
  store_tiles(0);
  __syncthreads();

  for (int kt = 0; kt < ktiles; ++kt) {
    const int buf = Cfg::STAGES == 2 ? (kt & 1) : 0;
    if (kt + 1 < ktiles) load_tiles((kt + 1) * BK);

#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[TM], b[TN];
      if constexpr (Cfg::SPLIT_M) {
#pragma unroll
        for (int i4 = 0; i4 < TM / 4; ++i4) {
          const float4 v = *reinterpret_cast<const float4 *>(&As[buf][k][i4 * (BM / (TM / 4)) + ty * 4]);
          a[i4 * 4 + 0] = v.x;
          a[i4 * 4 + 1] = v.y;
          a[i4 * 4 + 2] = v.z;
          a[i4 * 4 + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < TM; ++i) a[i] = As[buf][k][ty * TM + i];
      }
      if constexpr (Cfg::SPLIT_N) {
#pragma unroll
        for (int j4 = 0; j4 < TN / 4; ++j4) {
          const float4 v = *reinterpret_cast<const float4 *>(&Bs[buf][k][j4 * (BN / (TN / 4)) + tx * 4]);
          b[j4 * 4 + 0] = v.x;
          b[j4 * 4 + 1] = v.y;
          b[j4 * 4 + 2] = v.z;
          b[j4 * 4 + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < TN; ++j) b[j] = Bs[buf][k][tx * TN + j];
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }

    if (kt + 1 < ktiles) {
      if constexpr (Cfg::STAGES == 1) __syncthreads();  // every thread is done reading the one stage
      store_tiles(Cfg::STAGES == 2 ? (buf ^ 1) : 0);
    }
    __syncthreads();
  }

  // Fused epilogue: bias + GELU in registers, straight to C.
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int r = row0 + micro_index<BM, TM, Cfg::SPLIT_M>(ty, i);
    if (r >= M) continue;
    if constexpr (Cfg::SPLIT_N && VEC) {
#pragma unroll
      for (int j4 = 0; j4 < TN / 4; ++j4) {
        const int c = col0 + j4 * (BN / (TN / 4)) + tx * 4;
        if (c < N) {
          const float4 bb = __ldg(reinterpret_cast<const float4 *>(bias + c));
          float4 o;
          o.x = gelu_tanh_ref_f32(acc[i][j4 * 4 + 0] + bb.x);
          o.y = gelu_tanh_ref_f32(acc[i][j4 * 4 + 1] + bb.y);
          o.z = gelu_tanh_ref_f32(acc[i][j4 * 4 + 2] + bb.z);
          o.w = gelu_tanh_ref_f32(acc[i][j4 * 4 + 3] + bb.w);
          *reinterpret_cast<float4 *>(C + static_cast<size_t>(r) * N + c) = o;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int c = col0 + micro_index<BN, TN, Cfg::SPLIT_N>(tx, j);
        if (c < N) C[static_cast<size_t>(r) * N + c] = gelu_tanh_ref_f32(acc[i][j] + bias[c]);
      }
    }
  }
}

template <int BM, int BN, int BK, int TM, int TN, int PAD, bool VEC>
__global__ void __launch_bounds__(SimtConfig<BM, BN, BK, TM, TN, PAD>::THREADS)
    gemm_bias_gelu_simt(const float *__restrict__ A, const float *__restrict__ B, const float *__restrict__ bias,
                        float *__restrict__ C, int M, int N, int K) {
  gemm_bias_gelu_simt_body<BM, BN, BK, TM, TN, PAD, VEC>(A, B, bias, C, M, N, K);
}

}  // namespace pf
