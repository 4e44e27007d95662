/*
 * fake_pf.c -- a CPU stand-in for libpf_b200.so (the C ABI of include/pf_b200.h), so the C++ runner
 * and the tuner driving it can be tested without a GPU, following the reference's fake CUDA driver
 * (tests/fake_cuda/fake_cuda.cpp): "device" memory is host memory and a launch computes
 * C = gelu_tanh(scale * A.B + bias) in fp64 on the CPU, so the runner's correctness gate sees a
 * correct kernel.  Tile and shape rules are the real library's.  TEST INFRASTRUCTURE ONLY.
 *
 * Fault injection (environment):
 *   FAKE_PF_DEVICES=n        devices present (default 8)
 *   FAKE_PF_FAIL_OPEN=g      pf_open(g) fails with PF_ENODEV
 *   FAKE_PF_NOMEM=1          pf_upload fails with PF_ENOMEM
 *   FAKE_PF_FAIL_LAUNCH=1    pf_launch fails with PF_ECUDA
 *   FAKE_PF_WRONG=1          launches produce wrong results (every output + 0.5)
 *   FAKE_PF_TIMEOUT_DEV=g    launches on device g record a bounded-wait timeout in the status word
 *   FAKE_PF_LOG=path         append one line per call kind ("prepare", "launch", "time") to path
 */
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "pf_b200.h"

struct pf_ctx {
  int device;
  char err[256];
  int prepared, bound;
  pf_dtype dtype;
  pf_tile tile;
  int M, N, K;
  const void *A, *B;
  const float *bias;
  void *C;
  float sa, sb;
  void *own_A, *own_B, *own_C;
  float *own_bias;
  unsigned status;
};

static int env_int(const char *name, int dflt) {
  const char *v = getenv(name);
  return v ? atoi(v) : dflt;
}

static void flog(const char *what, int dev) {
  const char *p = getenv("FAKE_PF_LOG");
  if (!p) return;
  FILE *f = fopen(p, "a");
  if (!f) return;
  fprintf(f, "%s %d\n", what, dev);
  fclose(f);
}

static int set_err(pf_ctx *c, int code, const char *fmt, ...) {
  if (c) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(c->err, sizeof c->err, fmt, ap);
    va_end(ap);
  }
  return code;
}

const char *pf_version(void) { return "ptxforge_b200 fake (cpu)"; }
size_t pf_elem_bytes(pf_dtype d) { return d == PF_F32 || d == PF_F32_3XTF32 ? 4 : d == PF_BF16 ? 2 : d == PF_E4M3 ? 1 : 0; }
size_t pf_out_bytes(pf_dtype d) { return d == PF_F32 || d == PF_F32_3XTF32 ? 4 : (d == PF_BF16 || d == PF_E4M3) ? 2 : 0; }

int pf_open(int device, pf_ctx **out) {
  if (!out) return PF_EINVAL;
  *out = NULL;
  if (device < 0 || device >= env_int("FAKE_PF_DEVICES", 8) || device == env_int("FAKE_PF_FAIL_OPEN", -1))
    return PF_ENODEV;
  pf_ctx *c = (pf_ctx *)calloc(1, sizeof *c);
  c->device = device;
  *out = c;
  return PF_OK;
}

int pf_close(pf_ctx *c) {
  if (!c) return PF_EINVAL;
  free(c->own_A);
  free(c->own_B);
  free(c->own_C);
  free(c->own_bias);
  free(c);
  return PF_OK;
}

const char *pf_last_error(const pf_ctx *c) { return c ? c->err : "null context"; }

int pf_set_wait_timeout(pf_ctx *c, unsigned long long ns) { return (!c || !ns) ? PF_EINVAL : PF_OK; }

int pf_set_stream_k(pf_ctx *c, int mode) { return (!c || mode < -1 || mode > 1) ? PF_EINVAL : PF_OK; }

int pf_set_host_chunks(pf_ctx *c, int chunks) { return (!c || chunks < 0 || chunks > 64) ? PF_EINVAL : PF_OK; }

int pf_prepare(pf_ctx *c, pf_dtype dt, const pf_tile *t, int M, int N, int K) {
  if (!c || !t) return PF_EINVAL;
  flog(t->BN == 512 ? "prepare_bn512" : "prepare", c->device);
  c->prepared = c->bound = 0;
  if (M <= 0 || N <= 0 || K <= 0) return set_err(c, PF_EINVAL, "M, N, K must be positive");
  if (dt == PF_BF16 || dt == PF_E4M3) {
    if (t->BM != 128 && t->BM != 256) return set_err(c, PF_ETILE, "tensor path: BM must be 128 or 256, got %d", t->BM);
    if (t->BK != 32) return set_err(c, PF_ETILE, "tensor path: BK must be 32 words, got %d", t->BK);
    if (t->PAD != 0 && t->PAD != 1) return set_err(c, PF_ETILE, "tensor path: PAD must be 0 or 1, got %d", t->PAD);
    if (!(t->BN == 256 || t->BN == 128 || (t->BN == 64 && dt == PF_BF16) || ((t->BN == 224 || t->BN == 512) && t->BM == 256)) ||
        (t->BM == 256 && t->BN != 256 && t->BN != 224 && t->BN != 512))
      return set_err(c, PF_ETILE, "tensor path: no kernel with BM=%d BN=%d", t->BM, t->BN);
    if (t->TM < (t->BN == 512 ? 3 : 2)) return set_err(c, PF_ETILE, "tensor path: no kernel with %d stages", t->TM);
    if (t->BN == 512 && t->PAD != 0) return set_err(c, PF_ETILE, "tensor path: 512-column tiles take one k-atom");
    const int e = (int)pf_elem_bytes(dt);
    if ((K * e) % 16 || (N * e) % 16 || (N * 2) % 16) return set_err(c, PF_ESHAPE, "rows must be multiples of 16 bytes");
  } else if (dt == PF_F32) {
    /* the fp32 tiles the real library carries precompiled */
    static const int known[][6] = {{128, 128, 8, 8, 8, 4}, {128, 128, 8, 8, 8, 0}, {128, 128, 16, 8, 8, 4},
                                   {128, 64, 8, 8, 4, 4},  {64, 128, 8, 4, 8, 4},  {64, 64, 8, 4, 4, 0},
                                   {64, 64, 8, 4, 4, 4},   {64, 64, 16, 4, 4, 4},  {32, 64, 8, 2, 4, 4},
                                   {32, 32, 8, 2, 2, 0},   {32, 32, 32, 4, 2, 2},  {64, 32, 32, 4, 2, 2},
                                   {32, 64, 32, 4, 2, 2}};
    int found = 0;
    for (size_t i = 0; i < sizeof known / sizeof known[0]; ++i)
      found |= known[i][0] == t->BM && known[i][1] == t->BN && known[i][2] == t->BK && known[i][3] == t->TM &&
               known[i][4] == t->TN && known[i][5] == t->PAD;
    if (!found) return set_err(c, PF_ETILE, "fp32 tile is not compiled into this library");
  } else if (dt == PF_F32_3XTF32) {
    if (t->BM != 256 || t->BN != 256 || t->BK != 32 || t->PAD != 0 || t->TM < 2)
      return set_err(c, PF_ETILE, "3xTF32 path: no kernel for this tile");
    if (K % 4 || N % 4) return set_err(c, PF_ESHAPE, "rows must be multiples of 16 bytes");
  } else {
    return set_err(c, PF_ETILE, "dtype %d not built", (int)dt);
  }
  c->dtype = dt;
  c->tile = *t;
  c->M = M;
  c->N = N;
  c->K = K;
  c->prepared = 1;
  c->err[0] = 0;
  return PF_OK;
}

int pf_prepare_image(pf_ctx *c, const void *image, size_t image_bytes, const char *kernel, int gx, int gy, int block,
                     int M, int N, int K) {
  if (!c || !image || !image_bytes || !kernel) return PF_EINVAL;
  flog("prepare_image", c->device);
  c->prepared = c->bound = 0;
  if (M <= 0 || N <= 0 || K <= 0 || gx <= 0 || gy <= 0 || block <= 0) return set_err(c, PF_EINVAL, "bad sizes");
  if (block > 1024) return set_err(c, PF_ETILE, "block %d exceeds kernel max 1024 (register pressure)", block);
  c->dtype = PF_F32;
  memset(&c->tile, 0, sizeof c->tile);
  c->M = M;
  c->N = N;
  c->K = K;
  c->prepared = 1;
  return PF_OK;
}

int pf_bind(pf_ctx *c, const void *A, const void *B, const float *bias, void *C, float sa, float sb) {
  if (!c) return PF_EINVAL;
  if (!c->prepared) return set_err(c, PF_ESTATE, "pf_bind before pf_prepare");
  if (!A || !B || !bias || !C) return set_err(c, PF_EINVAL, "null operand");
  c->A = A;
  c->B = B;
  c->bias = bias;
  c->C = C;
  c->sa = sa;
  c->sb = sb;
  c->bound = 1;
  return PF_OK;
}

static double elem(pf_dtype dt, const void *p, size_t i) {
  if (dt == PF_F32 || dt == PF_F32_3XTF32) return ((const float *)p)[i];
  if (dt == PF_BF16) {
    unsigned u = (unsigned)((const unsigned short *)p)[i] << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
  }
  const unsigned char v = ((const unsigned char *)p)[i];
  const int s = v >> 7, e = (v >> 3) & 15, m = v & 7;
  double mag = e == 0 ? ldexp((double)m, -9) : ldexp(1.0 + m / 8.0, e - 7);
  return s ? -mag : mag;
}

static unsigned short to_bf16(float f) {
  unsigned u;
  memcpy(&u, &f, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (unsigned short)(u >> 16);
}

int pf_launch(pf_ctx *c, void *stream) {
  (void)stream;
  if (!c) return PF_EINVAL;
  flog("launch", c->device);
  if (!c->prepared) return set_err(c, PF_ESTATE, "pf_launch before pf_prepare");
  if (!c->bound) return set_err(c, PF_ESTATE, "pf_launch before pf_bind");
  if (env_int("FAKE_PF_FAIL_LAUNCH", 0)) return set_err(c, PF_ECUDA, "cudaLaunchKernel -> fake launch failure");
  if (c->device == env_int("FAKE_PF_TIMEOUT_DEV", -1)) c->status |= 2u;
  const double scale = (double)c->sa * c->sb, wrong = env_int("FAKE_PF_WRONG", 0) ? 0.5 : 0.0;
  for (int r = 0; r < c->M; ++r)
    for (int j = 0; j < c->N; ++j) {
      double a = 0;
      for (int k = 0; k < c->K; ++k)
        a += elem(c->dtype, c->A, (size_t)r * c->K + k) * elem(c->dtype, c->B, (size_t)k * c->N + j);
      const double x = a * scale + c->bias[j];
      const double y = 0.5 * x * (1.0 + tanh(0.7978845608028654 * (x + 0.044715 * x * x * x))) + wrong;
      if (c->dtype == PF_F32 || c->dtype == PF_F32_3XTF32)
        ((float *)c->C)[(size_t)r * c->N + j] = (float)y;
      else
        ((unsigned short *)c->C)[(size_t)r * c->N + j] = to_bf16((float)y);
    }
  return PF_OK;
}

int pf_time(pf_ctx *c, int warmup, int iters, int reps, double *median_ms) {
  if (!c || !median_ms || warmup < 0 || iters <= 0 || reps <= 0) return PF_EINVAL;
  flog("time", c->device);
  if (!c->bound) return set_err(c, PF_ESTATE, "pf_time before pf_bind");
  /* Timings are meaningless; make them depend on the config so the tuner has something to rank. */
  *median_ms = 1.0 + 0.001 * (c->tile.BN + 2 * c->tile.TM + c->tile.TN) + 0.01 * c->device;
  return PF_OK;
}

int pf_time_cublas(pf_ctx *c, int warmup, int iters, int reps, double *gemm_ms, double *unfused_ms) {
  if (!c || !gemm_ms || !unfused_ms || warmup < 0 || iters <= 0 || reps <= 0) return PF_EINVAL;
  flog("cublas", c->device);
  if (!c->bound) return set_err(c, PF_ESTATE, "pf_time_cublas before pf_bind");
  *gemm_ms = 0.9;
  *unfused_ms = 1.4;
  return PF_OK;
}

int pf_attrs(pf_ctx *c, pf_attr *a) {
  if (!c || !a) return PF_EINVAL;
  if (!c->prepared) return set_err(c, PF_ESTATE, "pf_attrs before pf_prepare");
  a->regs = 149;
  a->local_bytes = 0;
  a->smem_bytes = 230520;
  a->blocks_per_sm = 1;
  a->threads = 192;
  a->grid = 148;
  a->num_sms = 148;
  return PF_OK;
}

int pf_device_status(pf_ctx *c, unsigned *w) {
  if (!c || !w) return PF_EINVAL;
  *w = c->status;
  c->status = 0;
  return PF_OK;
}

static int ensure(void **buf, size_t n) {
  free(*buf);
  *buf = calloc(1, n ? n : 1);
  return *buf ? PF_OK : PF_ENOMEM;
}

int pf_run_host_rows(pf_ctx *c, const void *hA, void *hC, void *after_stream, void *copies_after_stream) {
  (void)after_stream;
  (void)copies_after_stream;
  if (!c) return PF_EINVAL;
  if (!c->prepared || !c->bound) return set_err(c, PF_ESTATE, "pf_run_host_rows before pf_prepare / pf_bind");
  if (!hA || !hC) return set_err(c, PF_EINVAL, "null host operand");
  /* "device" memory is host memory here: rows of A into the bound A, launch, C back */
  memcpy((void *)c->A, hA, (size_t)c->M * c->K * pf_elem_bytes(c->dtype));
  int rc = pf_launch(c, NULL);
  if (rc) return rc;
  memcpy(hC, c->C, (size_t)c->M * c->N * pf_out_bytes(c->dtype));
  return PF_OK;
}

int pf_upload(pf_ctx *c, const void *hA, const void *hB, const float *hbias, float sa, float sb) {
  if (!c) return PF_EINVAL;
  if (!c->prepared) return set_err(c, PF_ESTATE, "pf_upload before pf_prepare");
  if (env_int("FAKE_PF_NOMEM", 0)) return set_err(c, PF_ENOMEM, "cudaMalloc(...) failed (fake)");
  const size_t e = pf_elem_bytes(c->dtype), o = pf_out_bytes(c->dtype);
  const size_t nA = (size_t)c->M * c->K * e, nB = (size_t)c->K * c->N * e, nC = (size_t)c->M * c->N * o;
  if (ensure(&c->own_A, nA) || ensure(&c->own_B, nB) || ensure(&c->own_C, nC) ||
      ensure((void **)&c->own_bias, (size_t)c->N * 4))
    return set_err(c, PF_ENOMEM, "host allocation failed");
  memcpy(c->own_A, hA, nA);
  memcpy(c->own_B, hB, nB);
  memcpy(c->own_bias, hbias, (size_t)c->N * 4);
  return pf_bind(c, c->own_A, c->own_B, c->own_bias, c->own_C, sa, sb);
}

int pf_download(pf_ctx *c, void *hC) {
  if (!c || !hC) return PF_EINVAL;
  if (!c->own_C || c->C != c->own_C) return set_err(c, PF_ESTATE, "pf_download without pf_upload");
  memcpy(hC, c->own_C, (size_t)c->M * c->N * pf_out_bytes(c->dtype));
  return PF_OK;
}

int pf_run_host(pf_ctx *c, const void *hA, const void *hB, const float *hbias, void *hC, float sa, float sb) {
  int rc;
  if ((rc = pf_upload(c, hA, hB, hbias, sa, sb)) || (rc = pf_launch(c, NULL))) return rc;
  return pf_download(c, hC);
}

int pf_shard_rows(int M, int G, int g, int align, int *row0, int *rows) {
  if (M <= 0 || G <= 0 || g < 0 || g >= G || align <= 0 || !row0 || !rows) return PF_EINVAL;
  const long long units = ((long long)M + align - 1) / align;
  long long r0 = units * g / G * align, r1 = units * (g + 1) / G * align;
  if (r0 > M) r0 = M;
  if (r1 > M) r1 = M;
  *row0 = (int)r0;
  *rows = (int)(r1 - r0);
  return PF_OK;
}

int pf_selftest_wait_timeout(pf_ctx *c, unsigned long long ns, unsigned *w) {
  if (!c || !w || !ns) return PF_EINVAL;
  *w = 4u;
  return PF_OK;
}
