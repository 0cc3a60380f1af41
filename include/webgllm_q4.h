/*
 * webgllm_q4.h: the C ABI of the B200 Q4 matmul library (libwebgllm_b200.so).
 *
 * It replaces, for webgllm's 4-bit matmul path, the engine's WebGL2 calls:
 * the weight upload (Engine.matrix -> allocateMatrix -> writeMatrix), the
 * loader's repack (packQ4_0 / packMatMulNBits) and the matmul passes
 * (Engine.project -> splitPartials / matmul -> Gpu.run). Each declaration
 * names the reference interface it stands in for, as a path inside the
 * webgllm package (packages/webgllm/) with its line.
 *
 * Conventions
 * - Every entry point returns a status (WG_OK = 0, else a WG_* code);
 *   wg_error_string() names it and wg_last_error() gives the detail of the
 *   last failure on a context. The reference throws GpuError with a message
 *   (src/gpu/types.ts:14), classified by text in src/worker-errors.ts:14-24;
 *   WG_OUT_OF_MEMORY and WG_DEVICE_LOST are the "out-of-memory" and
 *   "gpu-context-lost" classes there.
 * - A context is one device and one CUDA stream, used from one host thread
 *   at a time, as the reference's engine owns one GL context in one worker
 *   (src/client.ts:64). Work is enqueued on the context's stream and returns
 *   without waiting, like Gpu.run (src/gpu/gl.ts:501); wg_read and wg_sync
 *   wait.
 * - Device pointers come from wg_alloc (or any cudaMalloc'd memory of the
 *   context's device). Host pointers stay owned by the caller; they are
 *   copied before the call returns.
 * - Shapes follow the reference's QuantMatrix rules (src/repack.ts:21-24):
 *   N (output rows) a multiple of 4, K (inputs per row) a multiple of 32.
 *   WG_INVALID_SHAPE otherwise.
 */
#ifndef WEBGLLM_Q4_H
#define WEBGLLM_Q4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum wg_status {
  WG_OK = 0,
  WG_INVALID_ARGUMENT = 1,
  WG_INVALID_SHAPE = 2,  /* N % 4 or K % 32 (src/repack.ts:21-24) */
  WG_OUT_OF_RANGE = 3,   /* rows outside the matrix (src/repack.ts:52-53) */
  WG_DATA_TOO_SHORT = 4, /* "Q4_0 data is too short" (src/repack.ts:69) */
  WG_OUT_OF_MEMORY = 5,  /* worker-errors.ts:20 "out-of-memory" */
  WG_CUDA_ERROR = 6,
  WG_TIMEOUT = 7,        /* a bounded device-side wait ran out */
  WG_DEVICE_LOST = 8,    /* worker-errors.ts:19 "gpu-context-lost" */
  WG_UNSUPPORTED = 9,
  WG_NO_DEVICE = 10      /* worker-errors.ts:21 "webgl2-unavailable" */
};

/* Element types of activations and outputs. */
enum wg_dtype { WG_F32 = 0, WG_F16 = 1, WG_BF16 = 2 };

typedef struct wg_ctx wg_ctx;
/* A 4-bit matrix resident on the device in the library's tiled layout. */
typedef struct wg_q4mat wg_q4mat;

/* ---- context, memory, transfers (the Gpu object, src/gpu/gl.ts) ---------- */

/* Gpu constructor (src/gpu/gl.ts:108): a context on CUDA device `device`. */
int wg_init(int device, wg_ctx **out);
/* Gpu.dispose (src/gpu/gl.ts:316). Frees the context's own buffers. */
int wg_destroy(wg_ctx *ctx);
/* Run the context's work on `stream` (a cudaStream_t; NULL: the context's
 * own non-blocking stream, which is not ordered with the legacy default
 * stream: to share that one, pass cudaStreamLegacy). No reference
 * counterpart: WebGL has one implicit queue. */
int wg_set_stream(wg_ctx *ctx, void *stream);

/* Context options (wg_set_option). */
/* Matmuls of up to this many rows (default 16; 0 .. 256) run on the decode
 * GEMV, in launches of up to 32 rows: exact weights, fp32 block scaling —
 * the reference's split-path arithmetic, which serves its decode rows and
 * its speculative draft batches (src/engine.ts:4684, forwardDraft :8036);
 * more rows go to the tensor-core GEMM, whose weights are rounded to fp16 as
 * the reference's f16 prompt route rounds them (src/gpu/kernels.ts:467).
 * A speculative verify batch raises it to its rows so that its picks use the
 * arithmetic of the decode steps they check. */
#define WG_OPT_EXACT_ROWS 1
int wg_set_option(wg_ctx *ctx, int option, int value);
/* Gpu.texture (src/gpu/gl.ts:263): `bytes` of device memory. */
int wg_alloc(wg_ctx *ctx, size_t bytes, void **dptr);
/* Gpu.delete (src/gpu/gl.ts:448). */
int wg_free(wg_ctx *ctx, void *dptr);
/* Page-locked host memory for fast transfers (the reference's upload
 * staging, src/upload-staging.ts, has no such notion). */
int wg_host_alloc(wg_ctx *ctx, size_t bytes, void **hptr);
int wg_host_free(wg_ctx *ctx, void *hptr);
/* Gpu.write (src/gpu/gl.ts:354): host -> device, enqueued on the stream.
 * `src` may be reused once the call returns only when it is pageable
 * memory; page-locked sources are read asynchronously (wg_sync first). */
int wg_upload(wg_ctx *ctx, void *dst, const void *src, size_t bytes);
/* Gpu.read (src/gpu/gl.ts:658): device -> host, waits for the stream. */
int wg_read(wg_ctx *ctx, void *host, const void *src, size_t bytes);
/* Wait for everything enqueued on the context (a fence wait). Reports a
 * kernel's timeout flag as WG_TIMEOUT. */
int wg_sync(wg_ctx *ctx);

/* ---- 4-bit matrices (src/weights.ts:153-178, src/repack.ts) --------------- */

/* newQuantMatrix(N, K, 4, withZeros) (src/repack.ts:14-35) with the engine's
 * allocateMatrix (src/engine.ts:2381): device storage for an N x K 4-bit
 * matrix, zero points if `with_zeros` (else 8 everywhere, as Q4_0). Every
 * weight starts at 0 (scale 0, code 8). */
int wg_q4_new(wg_ctx *ctx, int N, int K, int with_zeros, wg_q4mat **out);
/* Gpu.delete of the matrix's textures. */
int wg_q4_free(wg_ctx *ctx, wg_q4mat *m);
/* The matrix's shape and device footprint in bytes. */
int wg_q4_info(const wg_q4mat *m, int *N, int *K, size_t *device_bytes);

/* packQ4_0 (src/repack.ts:60-87) + writeMatrix (src/engine.ts:3355):
 * `rows` rows of llama.cpp Q4_0 blocks (18 bytes each: fp16 scale, 16 bytes
 * of nibbles, byte j = weight j low, weight j + 16 high; K / 32 blocks a
 * row) from host memory into rows [row0, row0 + rows) of `m`. `src_rows`
 * (nullable, `rows` entries) gives each destination row's source row, for
 * head permutations (src/repack.ts:5-6). The repack runs on the device;
 * `src` may also be device memory. */
int wg_q4_pack_q4_0(wg_ctx *ctx, wg_q4mat *m, int row0, const uint8_t *src,
                    size_t src_len, int rows, const int32_t *src_rows);

/* packMatMulNBits (src/repack.ts:342-392): `rows` rows of onnxruntime
 * MatMulNBits data (bits 4, block 32): `quant` [rows][K/32][16] with
 * element 2i of a block in byte i's low nibble, `scale_bytes` [rows][K/32]
 * fp16, `zp` [rows][ceil(K/64)] two blocks a byte, low nibble first, or
 * NULL (8). zp requires a matrix made with zero points. */
int wg_q4_pack_nbits(wg_ctx *ctx, wg_q4mat *m, int row0, const uint8_t *quant,
                     size_t quant_len, const uint8_t *scale_bytes,
                     size_t scale_len, const uint8_t *zp, size_t zp_len,
                     int rows, const int32_t *src_rows);

/* writeMatrix (src/engine.ts:3355) of a QuantMatrix already packed on the
 * host (src/weights.ts:5-21): `quants` N*K/8 words in row-group order,
 * `scales` N*K/32 fp16 bits, `zeros` N*K/32 bytes or NULL. */
int wg_q4_write_quantmatrix(wg_ctx *ctx, wg_q4mat *m, const uint32_t *quants,
                            const uint16_t *scales, const uint8_t *zeros);

/* matrixRow (src/repack.ts:865-891): row n as K floats, scale * (q - zero),
 * read back from the device layout into host memory (waits). */
int wg_q4_matrix_row(wg_ctx *ctx, const wg_q4mat *m, int n, float *out);

/* ---- the matmul (src/engine.ts:4677 project, :4969 matmul, :5241
 *      splitPartials; shaders src/gpu/kernels.ts:163-976) ------------------- */

/* y = x . W^T for M rows of activations: x [M][K] (x_dtype), y [M][N]
 * (y_dtype), both device pointers, row-major and contiguous. Weight
 * (n, k) = scale * (q - zero) of its block. Few rows (the reference's
 * split path, rows <= 8; here up to 16) run the decode GEMV; more rows the
 * tensor-core GEMM. fp16 outputs saturate at +-65504 as packH2 does
 * (src/gpu/kernels.ts:32-36). Enqueued on the context's stream. */
int wg_q4_matmul(wg_ctx *ctx, const wg_q4mat *m, const void *x, int x_dtype,
                 int M, void *y, int y_dtype);

/* The same product as wg_q4_matmul, allocating no device memory. It has no
 * counterpart in the reference (WebGL allocates through textures). For
 * callers that cannot let the library allocate: code capturing the call into
 * a CUDA graph (no allocation is allowed during stream capture), engines that
 * budget device memory up front, and decode loops that cannot afford the
 * device synchronisation of cudaMalloc / cudaFree. Its scratch (the fp16
 * copy of an f32 / bf16 x that the GEMM reads) is one fixed
 * 32 MiB array in the library's device memory, held on every GPU that loads
 * the library until the process exits; a call that would need more returns
 * WG_UNSUPPORTED and says how much. The first call on a device looks up the
 * array's device address (kept for the process's life: do not call it again
 * after a cudaDeviceReset of that device); make it before capturing a
 * stream. All calls on a
 * device share the array, so calls whose work overlaps on the GPU (other
 * streams or contexts of the same device) race on it. */
int wg_q4_matmul_static(wg_ctx *ctx, const wg_q4mat *m, const void *x,
                        int x_dtype, int M, void *y, int y_dtype);

/* ---- matmul with its input pass fused in ------------------------------- */

/* Prologue kinds of wg_q4_matmul_fused. */
#define WG_PRO_RMSNORM 1 /* x = rmsnorm(a + b) * weight (addNormed, src/engine.ts:5695) */
#define WG_PRO_SWIGLU 2  /* x = silu(gate) * up (REDUCE_SWIGLU, src/gpu/kernels.ts:1066) */

typedef struct wg_prologue {
  int kind;             /* WG_PRO_* */
  const float *a;       /* RMSNORM: residual [M][K]; SWIGLU: gate | up [M][2K] */
  const float *b;       /* RMSNORM: added to the residual [M][K], or NULL */
  const float *weight;  /* RMSNORM: norm weight [K] */
  float eps;            /* RMSNORM: x / sqrt(mean(x^2) + eps) */
  float *resid_out;     /* RMSNORM: receives a + b [M][K], or NULL; must not
                           alias a or b */
  const float *stats;   /* RMSNORM: NULL, or the sums of squares of a per 16
                           columns, [K/16][M], from wg_q4_matmul_residual: the
                           row statistics come from them (b and resid_out
                           NULL), so the norm fuses into the matmul at any M
                           <= 8 without each CTA reading all of a */
} wg_prologue;

/* y = x . W^T where x (fp16, as the reference rounds matmul inputs) is made
 * from `pro` inside the matmul's own launch for M <= 8 rows (the decode
 * GEMV stages x in shared memory; each CTA computes the row statistics of
 * the norm itself): the engine's norm / SwiGLU pass and the matmul that
 * consumes it become one kernel. More rows, or a norm whose statistics
 * would make every CTA read over 64 KB (M * K * 4 bytes, twice with b), run
 * the prologue as its own kernel into the context's scratch (it may
 * allocate, as wg_q4_matmul).
 * Tensors are device pointers, 16-byte aligned. No reference counterpart as
 * one call: the engine runs the two passes back to back
 * (src/engine.ts:8875-9304). */
int wg_q4_matmul_fused(wg_ctx *ctx, const wg_q4mat *m, const wg_prologue *pro,
                       int M, void *y, int y_dtype);

/* Epilogues of wg_q4_matmul_ex. */
#define WG_EPI_SWIGLU_PAIRS 1 /* REDUCE_SWIGLU (src/gpu/kernels.ts:1066) in the matmul's epilogue */

/* The matmul with an optional prologue (as wg_q4_matmul_fused; x unused
 * then) and epilogue. WG_EPI_SWIGLU_PAIRS: the matrix is a gate|up pair
 * whose rows were packed interleaved by 8 (rows 16t .. 16t+7 = gate rows
 * 8t .. 8t+7, rows 16t+8 .. 16t+15 = the same up rows; packQ4_0's srcRows
 * does this at load time), and y [M][N/2] receives silu(gate) * up, so the
 * gate|up product is never stored. Epilogues run in the decode GEMV
 * (M <= 32, N % 16 == 0). */
int wg_q4_matmul_ex(wg_ctx *ctx, const wg_q4mat *m, const wg_prologue *pro,
                    const void *x, int x_dtype, int M, void *y, int y_dtype,
                    int epilogue);

/* The residual add of a decoder layer in the matmul's epilogue, and the
 * statistics of the RMS norm that follows it: resid fp32 [M][N] += x . W^T
 * (x as wg_q4_matmul_ex: given, or made by `pro`), and stats fp32 [N/16][M]
 * receives, per 16 rows of W and per row m of x, the sum of squares of those
 * 16 new residual values. The next matmul's prologue WG_PRO_RMSNORM with
 * a = resid, stats = stats then normalises without reading every residual
 * value: the engine's addNormed (src/engine.ts:5695) split across the two
 * matmuls instead of a pass of its own. M <= 8, N % 16 == 0, 16-byte aligned
 * tensors; the decode GEMV. */
int wg_q4_matmul_residual(wg_ctx *ctx, const wg_q4mat *m, const wg_prologue *pro, const void *x, int x_dtype,
                          int M, float *resid, float *stats);

/* ---- tracing ------------------------------------------------------------- */

/* Gpu.trace / drawTrace (src/gpu/gl.ts:553-598), per CTA instead of per
 * pass: while `buf` (device memory, `bytes` long) is set, every matmul
 * launch appends one record of WG_TRACE_WORDS u64 per CTA: %globaltimer (ns)
 * at entry, after its weight copies are issued, after the wait on the
 * producer of x, after x is staged, after the last multiply, at exit; then
 * the SM id and (launch index << 32 | CTA index). Records past the end of
 * `buf` are dropped. NULL stops tracing; wg_trace_count() gives the number
 * of records written since wg_trace() was called. */
#define WG_TRACE_WORDS 8
int wg_trace(wg_ctx *ctx, void *buf, size_t bytes);
int wg_trace_count(wg_ctx *ctx, size_t *records);

/* ---- recorded steps ------------------------------------------------------ */

/* The engine submits a decode step as a fixed sequence of passes, each its
 * own Gpu.run (the layer loop, src/engine.ts:9106; one pass per matmul,
 * src/engine.ts:4677). A host that repeats such a sequence can record it
 * once and replay it as one submission: the launches then cost one host
 * call, not one each, and keep their programmatic dependent launch edges.
 * No reference counterpart (WebGL has no recorded command buffers). */
typedef struct wg_graph wg_graph;
/* Starts recording on the context's stream (CUDA stream capture, this
 * thread only): the calls that enqueue work on it until wg_graph_end are
 * recorded, not run. They read and write the device pointers they were
 * given at every replay. Recorded calls must allocate nothing (make each
 * kind of call once before recording, or use wg_q4_matmul_static) and must
 * not wait (wg_read, wg_sync, wg_q4_matrix_row, wg_free): such a call fails
 * and spoils the recording, which wg_graph_end then reports. Not on the
 * legacy default stream. */
int wg_graph_begin(wg_ctx *ctx);
/* Ends the recording: *out replays it. If the recording failed, *out is
 * NULL, nothing was enqueued, and the status says why. */
int wg_graph_end(wg_ctx *ctx, wg_graph **out);
/* Enqueues one replay of `g` on the context's stream (returns without
 * waiting, like every other launch). */
int wg_graph_launch(wg_ctx *ctx, const wg_graph *g);
/* Releases `g` once the context's stream has finished its replays. */
int wg_graph_free(wg_ctx *ctx, wg_graph *g);

/* ---- errors -------------------------------------------------------------- */

/* The name of a status code. */
const char *wg_error_string(int status);
/* The message of the last failed call on `ctx` (empty if none). */
const char *wg_last_error(const wg_ctx *ctx);

#ifdef __cplusplus
}
#endif

#endif /* WEBGLLM_Q4_H */
