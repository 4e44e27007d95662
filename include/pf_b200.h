/*
 * pf_b200.h -- C ABI of the sm_100a backend for PTXForge's one hot path:
 *
 *     C[r,c] = gelu_tanh( scale_a*scale_b * sum_k A[r,k]*B[k,c] + bias[c] )
 *
 * with A row-major [M x K], B row-major [K x N], bias fp32 [N], C row-major [M x N].
 *
 * This library replaces, for PTXForge's `Runner` boundary
 * (core/include/ptxforge/runner.hpp:39-45), what `CudaRunner` does per trial
 * (core/src/cuda_runner.cpp:152-217): select and load a kernel for a tile config,
 * launch it, time it with the reference protocol and report kernel attributes.
 * The reference's kernel ABI (kernels/gemm_bias_gelu.cu:42-44) is kept by the fp32 path:
 * same operand order, same row-major layout, same GELU (tanh form, k0=0.7978845608028654,
 * k1=0.044715, kernels/gemm_bias_gelu.cu:37-40).
 *
 * Conventions
 *   - Every function returns PF_OK (0) on success or a nonzero PF_E* code.  Nothing here throws,
 *     aborts or exits; the text of the last failure is available from pf_last_error().
 *   - A pf_ctx belongs to one host thread and one GPU.  It is not thread-safe; use one context per
 *     (thread, device), as the multi-GPU row-sharded runner does.
 *   - Device pointers passed to pf_bind are owned by the caller.  Buffers used by pf_run_host are
 *     owned by the context and freed by pf_close.
 *   - Kernel-side waits are bounded: a wait that runs out sets a bit in the context's device status
 *     word (read it with pf_device_status) and the kernel returns instead of hanging.
 */
#ifndef PF_B200_H
#define PF_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------------- */
enum {
  PF_OK = 0,
  PF_EINVAL = 1,       /* bad argument (null pointer, non-positive size, ...)                   */
  PF_ENODEV = 2,       /* no such CUDA device, or not an sm_100 part                            */
  PF_ECUDA = 3,        /* a CUDA runtime / driver call failed                                   */
  PF_ETILE = 4,        /* the tile config does not map onto a kernel of this backend            */
  PF_ESHAPE = 5,       /* M/N/K violate a layout rule of the chosen path (e.g. TMA 16-B rows)   */
  PF_ESTATE = 6,       /* call out of order (launch before prepare/bind, ...)                   */
  PF_ETIMEOUT = 7,     /* a bounded device-side wait ran out; see pf_device_status              */
  PF_ENOMEM = 8        /* device or pinned-host allocation failed                               */
};

/* ---- data types --------------------------------------------------------------------------- */
typedef enum {
  PF_F32 = 0,          /* fp32 A/B/C, fp32 FFMA (SIMT) accumulate, tanhf epilogue               */
  PF_F32_3XTF32 = 1,   /* fp32 A/B/C; each operand split into tf32 hi + lo, three tf32
                        * tensor-core products per step (lo*hi + hi*lo + hi*hi), fp32 accumulate
                        * in TMEM in chunks of a few k-blocks, each chunk added round-to-nearest
                        * into an fp32 running sum (the context's workspace), exp-form GELU:
                        * fp32-path tolerance at tensor-core speed                              */
  PF_BF16 = 2,         /* bf16 A/B, fp32 accumulate in TMEM, bf16 C                             */
  PF_E4M3 = 3          /* fp8 e4m3 A/B with per-tensor fp32 scales, fp32 accumulate, bf16 C     */
} pf_dtype;

/* The tuner's tile config: exactly the fields of ptxforge::Config (core/include/ptxforge/space.hpp:58).
 *   fp32 path   : the reference meaning (block tile BM x BN, K step BK, TM x TN per thread, PAD).
 *   tensor path : BM = tile rows: 128 (one CTA, UMMA M=128) or 256 (a CTA pair, cta_group::2);
 *                 BN = UMMA N (64/128/256) for BM=128; for BM=256 the pair tile's columns: 256, 224, or
 *                 512 (two N=256 halves in one TMEM accumulator: TM=3 gives 8 epilogue warps, TM>=4 four,
 *                 PAD=0); BK = 32 (4-byte words of one 128-byte
 *                 swizzle row); TM = requested pipeline depth in stages (clamped to the deepest
 *                 compiled variant that fits shared memory); TN = tile-raster group height in M
 *                 blocks (consecutive tiles walk TN row blocks before moving along N); PAD = extra
 *                 128-byte k-atoms per stage (0: one atom = 64 bf16 / 128 e4m3 k, 1: two atoms).
 *   3xTF32 path : BM = BN = 256 (a CTA pair), BK = 32 (one 128-byte row of fp32 k), TM = depth
 *                 (raw TMA slots + split hi/lo slots: 2, 3 or 4, clamped), TN = raster group, PAD = 0. */
typedef struct {
  int BM, BN, BK, TM, TN, PAD;
} pf_tile;

/* Opaque per-(thread, GPU) state: device, stream, selected kernel, tensor maps, status word. */
typedef struct pf_ctx pf_ctx;

/* Kernel attributes of the prepared variant (what CudaRunner reads with cuFuncGetAttribute and
 * cuOccupancyMaxActiveBlocksPerMultiprocessor, core/src/cuda_runner.cpp:163-179). */
typedef struct {
  int regs;            /* registers per thread                                                   */
  int local_bytes;     /* local (spill) bytes per thread                                        */
  int smem_bytes;      /* static + dynamic shared memory per block                              */
  int blocks_per_sm;   /* occupancy: resident blocks per SM                                     */
  int threads;         /* threads per block                                                     */
  int grid;            /* blocks launched (persistent kernels: min(tiles, SMs))                 */
  int num_sms;         /* SMs on the device                                                     */
} pf_attr;

/* ---- lifecycle ---------------------------------------------------------------------------- */

/* Open device `device` (CUDA ordinal).  Replaces CudaRunner::Impl's constructor
 * (core/src/cuda_runner.cpp:65-79: cuInit, device, primary context). */
int pf_open(int device, pf_ctx **out);

/* Release everything the context owns.  Replaces CudaRunner::Impl::~Impl (cuda_runner.cpp:81-88). */
int pf_close(pf_ctx *ctx);

/* Select the kernel variant for (dtype, tile, M, N, K) and build its TMA tensor maps once the
 * operands are bound.  Rejects configs this backend cannot run with PF_ETILE / PF_ESHAPE (an
 * invalid config is a failed trial, never a crash: cuda_runner.cpp:171-175).  Replaces the
 * per-trial compile + module load (cuda_runner.cpp:159-161, 219-237). */
int pf_prepare(pf_ctx *ctx, pf_dtype dtype, const pf_tile *tile, int M, int N, int K);

/* Load a kernel image -- PTX text (NUL-terminated or not) or an sm_100a cubin -- whose entry point
 * `kernel` has the reference kernel ABI
 *     extern "C" __global__ void kernel(const float *A, const float *B, const float *bias, float *C,
 *                                       int M, int N, int K)        (kernels/gemm_bias_gelu.cu:42-44)
 * and prepare it for an fp32 M x N x K problem launched on grid (grid_x, grid_y) with `block` threads.
 * Afterwards pf_bind / pf_upload / pf_launch / pf_time / pf_attrs / pf_download work as for a
 * prepared fp32 tile.  A block larger than the kernel allows is refused (PF_ETILE), as in
 * cuda_runner.cpp:171-175.  Replaces CudaRunner::run_ptx (core/include/ptxforge/cuda_runner.hpp:41-42,
 * core/src/cuda_runner.cpp:152-217, 251-253): any image -- the reference's own kernel, an
 * MLIR-generated one, or this library's fp32 kernel JIT-compiled for a tile (simt_image.cu) -- goes
 * through the same launch, gate and timing. */
int pf_prepare_image(pf_ctx *ctx, const void *image, size_t image_bytes, const char *kernel, int grid_x,
                     int grid_y, int block, int M, int N, int K);

/* Bind caller-owned device operands (row-major).  A/B are float, bf16 or e4m3 bytes according to
 * the prepared dtype; C is float for PF_F32 and PF_F32_3XTF32 and bf16 otherwise.  scale_a/scale_b are the
 * per-tensor dequantisation scales (used by PF_E4M3, must be 1 otherwise).  Replaces the
 * parameter block {&dA,&dB,&dBias,&dC,&M,&N,&K} of cuda_runner.cpp:182. */
int pf_bind(pf_ctx *ctx, const void *A, const void *B, const float *bias, void *C, float scale_a,
            float scale_b);

/* Launch once on `stream` (a cudaStream_t; NULL = the CUDA default stream, where the reference
 * launches, cuda_runner.cpp:183).  Asynchronous.  pf_time and pf_run_host use the context's own
 * stream instead. */
int pf_launch(pf_ctx *ctx, void *stream);

/* Reference timing protocol (CudaRunner::Impl::median_ms, cuda_runner.cpp:110-130): `warmup`
 * launches, then `reps` repetitions of `iters` back-to-back launches between two events on the
 * context's stream; per-launch time = elapsed/iters; returns the median over reps in ms. */
int pf_time(pf_ctx *ctx, int warmup, int iters, int reps, double *median_ms);

/* cuBLAS comparator on the bound operands and shape, timed with the pf_time protocol on the context's
 * stream: `gemm_ms` = cublasLt GEMM alone (what CudaRunner::Impl::measure_cublas times with
 * cublasSgemm, cuda_runner.cpp:132-149), `unfused_ms` = the same GEMM followed by a separate bias +
 * GELU kernel (the "cuBLAS + separate epilogue" of scripts/run_ptx_on_gpu.py:88-90).  bf16: bf16 GEMM,
 * fp32 accumulate; e4m3: fp8 GEMM with the bound per-tensor scales (B is transposed once, untimed,
 * as cublasLt's fp8 GEMM wants K-major operands); fp32: fp32 GEMM, no TF32.  C is overwritten with the
 * unfused result.  cublasLt is loaded at run time; PF_ECUDA if it cannot be. */
int pf_time_cublas(pf_ctx *ctx, int warmup, int iters, int reps, double *gemm_ms, double *unfused_ms);

/* Kernel attributes of the prepared variant. */
int pf_attrs(pf_ctx *ctx, pf_attr *out);

/* Synchronise the device and read (then clear) the context's device status word: 0 = clean,
 * nonzero = a bounded device-side wait ran out (bit 0: TMA-producer wait, bit 1: MMA wait,
 * bit 2: epilogue wait, bit 3: teardown wait, bit 4: 3xTF32 split wait). */
int pf_device_status(pf_ctx *ctx, unsigned *err_word);

/* Stream-K of the CTA-pair (BM=256) kernels: -1 auto (default), 0 off (every tile whole: results
 * independent of the launch shape, bit for bit), 1 the stream-K tail wherever there is a partial wave,
 * 2 row-band stream-K wherever a row block gets at least two pairs.
 *   - Stream-K tail (256 x 256 pair tiles, PF_F32_3XTF32): the leftover tiles' k-iterations of a partial last
 *     wave are spread over all resident CTA pairs.  Auto: with at least 3 waves of tiles when the last partial
 *     wave would waste more than 3 % of the launch; PF_F32_3XTF32 also below that when whole tiles would
 *     leave a quarter of the CTA pairs idle, given 4 leftover k-blocks per pair.  Workspace: 256 KB per pair.
 *   - Row-band stream-K (256 x 256 and 256 x 512 pair tiles, mode 2 only): each row block of tiles is shared
 *     by P = pairs / row blocks pairs, each taking an equal contiguous share of its k-iterations (pairs at the
 *     same position of every band read the same B panel at the same time).  Measured no faster than whole
 *     tiles on the row shards it was built for, so auto mode does not use it.  Workspace: 256 / 512 KB per
 *     pair.
 * Split tiles' fp32 partial sums are added in a fixed order (deterministic for a given shape), but in a
 * different rounding from whole tiles. */
int pf_set_stream_k(pf_ctx *ctx, int mode);

/* Row chunks of the host-buffer pipelines (pf_run_host, pf_run_host_rows): 0 = default (8), else at most
 * `chunks` (1..64) chunks of whole kernel tiles, each one's copy of A in, kernel and copy of C out
 * overlapping the others'.  More chunks shorten the pipeline's fill and drain (the first kernel starts
 * after a smaller piece of A, the last copy of C is smaller) at the price of smaller launches.  The
 * results do not depend on it: every chunk's tiles keep the whole problem's k order. */
int pf_set_host_chunks(pf_ctx *ctx, int chunks);

/* Bound, in nanoseconds, on every device-side wait of subsequent launches (default 4e9). */
int pf_set_wait_timeout(pf_ctx *ctx, unsigned long long ns);

/* Text of the most recent failure on this context ("" if none).  Valid until the next call. */
const char *pf_last_error(const pf_ctx *ctx);

/* ---- host-buffer path (the end-to-end call a host-side caller makes) ---------------------- */

/* Copy host operands in (pinned or pageable), launch the prepared kernel, copy C back, and
 * synchronise.  Device buffers are owned by the context and re-used while the problem size is
 * unchanged.  This is the one-call form of CudaRunner::Impl::ensure + launch + cuMemcpyDtoH
 * (cuda_runner.cpp:91-108, 183-188). */
int pf_run_host(pf_ctx *ctx, const void *hA, const void *hB, const float *hbias, void *hC,
                float scale_a, float scale_b);

/* The two halves of pf_run_host for callers that launch and time in between: pf_upload copies host
 * operands into context-owned device buffers (allocated on first use, re-used while the problem
 * size is unchanged), binds them and synchronises -- CudaRunner::Impl::ensure
 * (cuda_runner.cpp:91-108).  pf_download copies the context-owned C back after synchronising the
 * device -- the gate's cuMemcpyDtoH (cuda_runner.cpp:188). */
int pf_upload(pf_ctx *ctx, const void *hA, const void *hB, const float *hbias, float scale_a,
              float scale_b);
int pf_download(pf_ctx *ctx, void *hC);

/* pf_run_host for a row shard whose B and bias are already on the device (e.g. all-gathered over
 * NVLink): copies the host rows hA into the bound A buffer, launches, and copies C (the bound C buffer)
 * back to hC, in up to 8 row chunks whose H2D copies, kernels and D2H copies overlap, then synchronises.
 * Requires pf_prepare + pf_bind with caller-owned device A, B, bias and C; the bound A and C buffers are
 * overwritten, so no work that reads them may still be in flight.  The kernels start after everything
 * queued on `after_stream` (where the caller produced B and bias), the copies of A after everything queued
 * on `copies_after_stream` (e.g. the copy of this rank's slice of B, so the host link carries B first and
 * then A while B is all-gathered); pass the same stream twice to order everything after it (cudaStream_t
 * handles, NULL = the CUDA default stream).  The row-shard counterpart of pf_run_host (same reference call
 * sites, cuda_runner.cpp:91-108, 183-188); one launch over the shard gives the same bits. */
int pf_run_host_rows(pf_ctx *ctx, const void *hA, void *hC, void *after_stream, void *copies_after_stream);

/* ---- row sharding (no collective on the hot path) ----------------------------------------- */

/* Rows [*row0, *row0 + *rows) of A and C that shard `g` of `G` owns for an M-row problem.  Shard
 * boundaries are multiples of `align` rows (the CTA tile height) except for the last shard. */
int pf_shard_rows(int M, int G, int g, int align, int *row0, int *rows);

/* ---- no-allocation entry point ------------------------------------------------------------ */

/* Size of the library's fixed per-GPU scratch area used by pf_gemm_bias_gelu_noalloc, in bytes. */
#define PF_NOALLOC_SCRATCH_BYTES 256

/* No counterpart in the reference: an extra entry point for callers that cannot allocate GPU memory
 * when they call us -- for example a serving process that reserved nearly all of HBM for its own
 * pool at start-up (a cudaMalloc then fails or forces the pool to shrink), or a pipeline that cannot
 * afford the device-wide synchronisation cudaFree implies.  It runs the bf16 / e4m3 tensor-core
 * kernel (the kernels of pf_launch, chosen by `tile` as in pf_prepare) on caller-owned device
 * operands without a pf_ctx and without allocating anything: no cudaMalloc, no cudaFree, no host
 * heap.  The kernel's scratch -- its device status word, 4 bytes -- lives in a fixed array of
 * PF_NOALLOC_SCRATCH_BYTES bytes compiled into the library, which every GPU that loads the library
 * keeps until the process exits; a kernel needing more scratch than that is refused (PF_EINVAL).
 *   - Whole tiles only: the stream-K tail, whose partial sums need a workspace, never runs here.  Where
 *     pf_launch's automatic mode turns that tail on (long multi-wave problems), the two entry points
 *     round the tail tiles differently (both within the dtype's tolerance); elsewhere they give the
 *     same bits.
 *   - The first successful call on a device looks the array's device address up (with that device
 *     made current) and caches each kernel's launch set-up; a failed look-up is retried by the next
 *     call.  Make that first call before any stream capture.
 *   - The array is shared by every call on a device and keeps the last call's contents; each call
 *     clears the status word on `stream` before its launch.  Calls that overlap on the GPU (different
 *     streams, no ordering between them) race on it: order them, or use pf_ctx contexts instead.
 *   - `stream` NULL = the CUDA default stream; a stream of another device is refused (PF_EINVAL).
 *     With `status_out` NULL the call returns after queueing the work; with `status_out` non-NULL it
 *     synchronises `stream`, stores the status word there and returns PF_ETIMEOUT if a bounded device
 *     wait ran out.  Each device wait is bounded by 4 s (pf_ctx's default, pf_set_wait_timeout).
 *   - `err` (may be NULL) receives a short message of at most `err_len` bytes on failure.
 * fp32 (PF_F32) is not accepted: its kernel uses no scratch, call pf_launch instead. */
int pf_gemm_bias_gelu_noalloc(int device, pf_dtype dtype, const pf_tile *tile, int M, int N, int K,
                              const void *A, const void *B, const float *bias, void *C, float scale_a,
                              float scale_b, void *stream, unsigned *status_out, char *err,
                              size_t err_len);

/* ---- utilities ---------------------------------------------------------------------------- */

/* Bytes of one element of A/B and of C for a dtype (0 for an unknown dtype). */
size_t pf_elem_bytes(pf_dtype dtype);
size_t pf_out_bytes(pf_dtype dtype);

/* Library version string, and the architecture the kernels were compiled for ("sm_100a"). */
const char *pf_version(void);

/* Self-test of the bounded wait: launches one block that waits on an mbarrier nothing arrives at,
 * with a bound of `timeout_ns`.  Returns PF_OK and sets *err_word to the bit the kernel recorded
 * (expected nonzero) -- the kernel returns on its own, the context stays usable. */
int pf_selftest_wait_timeout(pf_ctx *ctx, unsigned long long timeout_ns, unsigned *err_word);

#ifdef __cplusplus
}
#endif

#endif /* PF_B200_H */
