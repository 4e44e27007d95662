/*
 * oracle.c -- CPU restatement of the reference's algorithm for the fused GEMM + bias + GELU path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * may load this library, and only as the checker (or as the timed CPU baseline), never as the
 * thing measured or shipped.  The product path (libpf_b200.so) never calls it.
 *
 * What it restates (file:line in the reference project):
 *   - gelu_ref: fp64 GELU, tanh form, k0 = 0.7978845608028654, k1 = 0.044715
 *       core/src/cuda_runner.cpp:32-34
 *   - the sampled correctness gate: positions drawn from mt19937(seed) as r = pick() % M,
 *     c = pick() % N; fp64 dot product over k ascending; err = |ref - C| / (1 + |ref|); the max
 *       core/src/cuda_runner.cpp:189-197
 *   - the fake driver's full fp64 launch (what the reference's own tests accept as correct)
 *       tests/fake_cuda/fake_cuda.cpp:45-50
 *   - the CPU-lowered MLIR schedule (tests/check_lowering_cpu.py): BM x BN block tiles, K walked
 *     in steps of BK with the A and B slices staged in buffers, fp32 accumulators updated by
 *     outer products (fused multiply-add, k ascending), then + bias and GELU per element in the
 *     order of compiler/samples/gemm_bias_gelu.mlir:40-53 (k0 = 0.7978845608, ten digits)
 *       scripts/schedule_template.mlir:33-124, compiler/samples/gemm_bias_gelu.mlir:25-56
 *     tanh here is the C library's tanhf: the reference lowers math.tanh to upstream MLIR 19's
 *     polynomial approximation (compiler/lib/ApproximateMath.cpp:48-56), whose source is not in
 *     the reference tree, so bit-level parity with that polynomial is unpinned; the reference's
 *     own pin at that boundary is allclose(rtol=1e-4, atol=1e-5) against fp64
 *     (tests/check_lowering_cpu.py:115).
 *   - MT19937 (the generator behind std::mt19937 used by the gate): the published algorithm of
 *     Matsumoto & Nishimura (1998), init_genrand seeding.
 *   - bf16 round-to-nearest-even and OCP fp8 e4m3 (bias 7, no infinities, max 448, satfinite)
 *     encode/decode, used to check the quantised inputs of the bf16 / e4m3 configs.
 *
 * Build: oracle/build.py (gcc -O3 -march=x86-64-v3 -ffp-contract=off -fopenmp -shared).
 * -ffp-contract=off keeps every multiply and add separately rounded except where fmaf() is
 * written, matching the reference's arithmetic.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------------------ */
/* MT19937                                                                                    */
/* ------------------------------------------------------------------------------------------ */
typedef struct {
  uint32_t mt[624];
  int mti;
} oracle_mt19937;

void oracle_mt_seed(oracle_mt19937 *s, uint32_t seed) {
  s->mt[0] = seed;
  for (int i = 1; i < 624; ++i) s->mt[i] = 1812433253u * (s->mt[i - 1] ^ (s->mt[i - 1] >> 30)) + (uint32_t)i;
  s->mti = 624;
}

uint32_t oracle_mt_next(oracle_mt19937 *s) {
  if (s->mti >= 624) {
    for (int i = 0; i < 624; ++i) {
      uint32_t y = (s->mt[i] & 0x80000000u) | (s->mt[(i + 1) % 624] & 0x7fffffffu);
      uint32_t v = s->mt[(i + 397) % 624] ^ (y >> 1);
      if (y & 1u) v ^= 0x9908b0dfu;
      s->mt[i] = v;
    }
    s->mti = 0;
  }
  uint32_t y = s->mt[s->mti++];
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}

/* First n outputs of mt19937(seed). */
void oracle_mt_stream(uint32_t seed, uint32_t *out, int n) {
  oracle_mt19937 s;
  oracle_mt_seed(&s, seed);
  for (int i = 0; i < n; ++i) out[i] = oracle_mt_next(&s);
}

/* ------------------------------------------------------------------------------------------ */
/* GELU                                                                                       */
/* ------------------------------------------------------------------------------------------ */
double oracle_gelu_f64(double x) { return 0.5 * x * (1.0 + tanh(0.7978845608028654 * (x + 0.044715 * x * x * x))); }

/* The MLIR epilogue (gemm_bias_gelu.mlir:40-53), one rounding per arith op, tanh = tanhf. */
float oracle_gelu_f32_mlir(float x) {
  const float half = 0.5f, one = 1.0f, k0 = 0.7978845608f, k1 = 0.044715f;
  float x2 = x * x;
  float x3 = x2 * x;
  float t1 = k1 * x3;
  float t2 = x + t1;
  float t3 = k0 * t2;
  float th = tanhf(t3);
  float p = one + th;
  float hx = half * x;
  return hx * p;
}

/* ------------------------------------------------------------------------------------------ */
/* fp64 references                                                                            */
/* ------------------------------------------------------------------------------------------ */
/* One output in fp64: gelu(scale * sum_k A[r,k]*B[k,c] + bias[c]), k ascending. */
static double ref_one(const float *A, const float *B, const float *bias, int N, int K, double scale, int r, int c) {
  double acc = 0.0;
  const float *a = A + (size_t)r * K;
  for (int k = 0; k < K; ++k) acc += (double)a[k] * (double)B[(size_t)k * N + c];
  if (scale != 1.0) acc *= scale;
  return oracle_gelu_f64(acc + (double)bias[c]);
}

/* Full fp64 reference (the fake driver's launch, generalised with a dequantisation scale).
 * out is M x N doubles.  OpenMP over rows. */
void oracle_full_f64(const float *A, const float *B, const float *bias, int M, int N, int K, double scale,
                     double *out) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int r = 0; r < M; ++r) {
    double *acc = (double *)calloc((size_t)N, sizeof(double));
    const float *a = A + (size_t)r * K;
    for (int k = 0; k < K; ++k) {
      const double av = (double)a[k];
      const float *b = B + (size_t)k * N;
      for (int c = 0; c < N; ++c) acc[c] += av * (double)b[c];
    }
    for (int c = 0; c < N; ++c) {
      double x = acc[c];
      if (scale != 1.0) x *= scale;
      out[(size_t)r * N + c] = oracle_gelu_f64(x + (double)bias[c]);
    }
    free(acc);
  }
}

/* The reference gate (cuda_runner.cpp:189-197) against a candidate C given as floats.
 * Writes the sampled positions to rows/cols (may be NULL) and returns the max error. */
double oracle_sampled_gate(const float *A, const float *B, const float *bias, const float *C, int M, int N, int K,
                           double scale, int samples, uint32_t seed, int *rows, int *cols) {
  oracle_mt19937 pick;
  oracle_mt_seed(&pick, seed);
  double max_err = 0.0;
  int nan_seen = 0;
  for (int s = 0; s < samples; ++s) {
    int r = (int)(oracle_mt_next(&pick) % (uint32_t)M);
    int c = (int)(oracle_mt_next(&pick) % (uint32_t)N);
    if (rows) rows[s] = r;
    if (cols) cols[s] = c;
    const double ref = ref_one(A, B, bias, N, K, scale, r, c);
    const double err = fabs(ref - (double)C[(size_t)r * N + c]) / (1.0 + fabs(ref));
    if (isnan(err)) nan_seen = 1;
    else if (err > max_err) max_err = err;
  }
  /* A NaN at a sampled position fails the gate.  (The reference's std::max(max_err, err) keeps the
   * old maximum when err is NaN; this checker is stricter on purpose.) */
  return nan_seen ? NAN : max_err;
}

/* Reference values at given positions (for sampled checks of huge problems). */
void oracle_ref_at(const float *A, const float *B, const float *bias, int N, int K, double scale, const int *rows,
                   const int *cols, int n, double *out) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) out[i] = ref_one(A, B, bias, N, K, scale, rows[i], cols[i]);
}

/* Same, for row-sharded operands: A_rows holds only the `rows` listed (row i of A_rows = the
 * i-th distinct requested row, index given by row_slot[i]). */
void oracle_ref_at_rowpack(const float *A_pack, const int *row_slot, const float *B, const float *bias, int N, int K,
                           double scale, const int *cols, int n, double *out) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; ++i) out[i] = ref_one(A_pack, B, bias, N, K, scale, row_slot[i], cols[i]);
}

/* ------------------------------------------------------------------------------------------ */
/* CPU-lowered schedule (fp32)                                                                */
/* ------------------------------------------------------------------------------------------ */
/* Computes output rows [row0, row0 + rows) of C = gelu(A.B + bias) the way the reference's
 * CPU-compiled schedule does: for each BM x BN block tile, zero the fp32 accumulators, walk K in
 * steps of BK copying the A (BM x BK) and B (BK x BN) slices into staging buffers, and update
 * every accumulator by fused multiply-adds in k order; then apply bias + GELU (MLIR op order).
 * Partial tiles at the edges are clipped.  Block tiles are distributed over `threads` OpenMP
 * threads (1 = the reference's serial execution, check_lowering_cpu.py:70-72,94). */
void oracle_cpu_schedule(const float *A, const float *B, const float *bias, float *C, int M, int N, int K, int BM,
                         int BN, int BK, int row0, int rows, int threads) {
  const int r_end = row0 + rows;
  const int mb0 = row0 / BM, mb1 = (r_end + BM - 1) / BM;
  const int nblocks = (N + BN - 1) / BN;
  const int ntiles = (mb1 - mb0) * nblocks;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#endif
#pragma omp parallel num_threads(threads)
  {
    float *acc = (float *)malloc(sizeof(float) * (size_t)BM * BN);
    float *As = (float *)malloc(sizeof(float) * (size_t)BM * BK);
    float *Bs = (float *)malloc(sizeof(float) * (size_t)BK * BN);
#pragma omp for schedule(dynamic, 1)
    for (int t = 0; t < ntiles; ++t) {
      const int mb = mb0 + t / nblocks, nb = t % nblocks;
      const int r0 = mb * BM > row0 ? mb * BM : row0;
      const int r1 = (mb + 1) * BM < r_end ? (mb + 1) * BM : r_end;
      const int c0 = nb * BN, c1 = (nb + 1) * BN < N ? (nb + 1) * BN : N;
      const int tm = r1 - r0, tn = c1 - c0;
      memset(acc, 0, sizeof(float) * (size_t)BM * BN);
      for (int k0 = 0; k0 < K; k0 += BK) {
        const int tk = (k0 + BK < K ? k0 + BK : K) - k0;
        for (int i = 0; i < tm; ++i) memcpy(As + (size_t)i * BK, A + (size_t)(r0 + i) * K + k0, sizeof(float) * tk);
        for (int k = 0; k < tk; ++k) memcpy(Bs + (size_t)k * BN, B + (size_t)(k0 + k) * N + c0, sizeof(float) * tn);
        for (int k = 0; k < tk; ++k) {
          const float *b = Bs + (size_t)k * BN;
          for (int i = 0; i < tm; ++i) {
            const float a = As[(size_t)i * BK + k];
            float *ac = acc + (size_t)i * BN;
            for (int j = 0; j < tn; ++j) ac[j] = fmaf(a, b[j], ac[j]);
          }
        }
      }
      for (int i = 0; i < tm; ++i)
        for (int j = 0; j < tn; ++j)
          C[(size_t)(r0 + i) * N + c0 + j] = oracle_gelu_f32_mlir(acc[(size_t)i * BN + j] + bias[c0 + j]);
    }
    free(acc);
    free(As);
    free(Bs);
  }
}

/* ------------------------------------------------------------------------------------------ */
/* number formats                                                                             */
/* ------------------------------------------------------------------------------------------ */
static uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* float -> bf16 bits, round to nearest even (NaN stays NaN). */
uint16_t oracle_bf16_rne(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

void oracle_bf16_to_f32_array(const uint16_t *h, float *out, size_t n) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; ++i) out[i] = u2f((uint32_t)h[i] << 16);
}

/* e4m3 (OCP FP8, "fn"): 1 sign, 4 exponent (bias 7), 3 mantissa; 0x7f/0xff are NaN; max 448. */
float oracle_e4m3_to_f32(uint8_t v) {
  const int s = v >> 7, e = (v >> 3) & 15, m = v & 7;
  float mag;
  if (e == 15 && m == 7) return NAN;
  if (e == 0)
    mag = ldexpf((float)m, -9); /* subnormal: m/8 * 2^-6 */
  else
    mag = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -mag : mag;
}

void oracle_e4m3_to_f32_array(const uint8_t *q, float *out, size_t n) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; ++i) out[i] = oracle_e4m3_to_f32(q[i]);
}

/* float -> e4m3 with round to nearest even and saturation to +-448 (satfinite). */
uint8_t oracle_e4m3_rne_sat(float f) {
  if (isnan(f)) return 0x7f;
  const uint8_t sign = signbit(f) ? 0x80 : 0x00;
  float a = fabsf(f);
  if (a >= 448.0f) return sign | 0x7e;
  /* Enumerate: the 127 finite non-negative codes are monotone in value. Pick nearest, ties to
   * the even code (even mantissa). */
  int lo = 0, hi = 0x7e;
  while (lo < hi) { /* largest code with value <= a */
    int mid = (lo + hi + 1) / 2;
    if (oracle_e4m3_to_f32((uint8_t)mid) <= a)
      lo = mid;
    else
      hi = mid - 1;
  }
  int code = lo;
  if (code < 0x7e) {
    const float v0 = oracle_e4m3_to_f32((uint8_t)code), v1 = oracle_e4m3_to_f32((uint8_t)(code + 1));
    const float d0 = a - v0, d1 = v1 - a;
    if (d1 < d0 || (d1 == d0 && (code & 1))) code += 1;
  }
  return sign | (uint8_t)code;
}

void oracle_e4m3_quantize_array(const float *x, float inv_scale, uint8_t *out, size_t n) {
#pragma omp parallel for schedule(static)
  for (size_t i = 0; i < n; ++i) out[i] = oracle_e4m3_rne_sat(x[i] * inv_scale);
}

/* Max of |ref - C| / (1 + |ref|) over n pairs (NaN in C counts as an infinite error). */
double oracle_max_rel_err(const double *ref, const float *C, size_t n) {
  double m = 0.0;
  for (size_t i = 0; i < n; ++i) {
    double e = fabs(ref[i] - (double)C[i]) / (1.0 + fabs(ref[i]));
    if (!(e <= m)) m = isnan(e) ? INFINITY : e;
  }
  return m;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
