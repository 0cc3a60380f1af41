// The C ABI of include/webgllm_q4.h.
//
// Host-side plumbing only: contexts, memory, transfers, argument checks (with
// the reference's error rules), and the dispatch of the Q4 matmul by row
// count, as Engine.project does (src/engine.ts:4677-4688: rows <= 8 take the
// split GEMV, more rows the prompt matmul).
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "capi_internal.cuh"
#include "common.cuh"
#include "q4_kernels.cuh"
#include "q4_layout.cuh"

namespace {

int fail(wg_ctx *ctx, int status, const char *fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    ctx->last_error = buf;
  }
  return status;
}

int cuda_fail(wg_ctx *ctx, cudaError_t e, const char *what) {
  return fail(ctx, wg::status_of(e), "%s: %s", what, cudaGetErrorString(e));
}

#define WG_CUDA(ctx, call)                                 \
  do {                                                     \
    cudaError_t e_ = (call);                               \
    if (e_ != cudaSuccess) return cuda_fail(ctx, e_, #call); \
  } while (0)

int use_device(wg_ctx *ctx) {
  WG_CUDA(ctx, cudaSetDevice(ctx->device));
  return WG_OK;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Grows the context's device staging buffer to `bytes` (stream-ordered: the
// old buffer is released only after the stream has drained).
int ensure_staging(wg_ctx *ctx, size_t bytes) {
  if (bytes <= ctx->staging_bytes) return WG_OK;
  WG_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (ctx->staging) WG_CUDA(ctx, cudaFree(ctx->staging));
  ctx->staging = nullptr;
  ctx->staging_bytes = 0;
  size_t want = align_up(bytes, 1 << 20);
  WG_CUDA(ctx, cudaMalloc(&ctx->staging, want));
  ctx->staging_bytes = want;
  return WG_OK;
}

bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

// Grows the matmul scratch to `bytes` (stream-ordered, as ensure_staging).
// It only grows, so a shape that has run once never allocates again (and
// may then be captured into a CUDA graph).
int ensure_work(wg_ctx *ctx, size_t bytes) {
  if (bytes <= ctx->work_bytes) return WG_OK;
  WG_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  if (ctx->work) WG_CUDA(ctx, cudaFree(ctx->work));
  ctx->work = nullptr;
  ctx->work_bytes = 0;
  size_t want = align_up(bytes, 1 << 20);
  WG_CUDA(ctx, cudaMalloc(&ctx->work, want));
  ctx->work_bytes = want;
  return WG_OK;
}

int check_shape(wg_ctx *ctx, int N, int K) {
  if (N <= 0 || K <= 0)
    return fail(ctx, WG_INVALID_SHAPE, "matrix shape %d x %d must be positive", N, K);
  // src/repack.ts:21-24
  if (N % 4 != 0) return fail(ctx, WG_INVALID_SHAPE, "matrix rows (%d) must be a multiple of 4", N);
  if (K % 32 != 0)
    return fail(ctx, WG_INVALID_SHAPE, "matrix columns (%d) must be a multiple of 32", K);
  return WG_OK;
}

int check_rows(wg_ctx *ctx, const wg_q4mat *m, int row0, int rows) {
  // src/repack.ts:52-53
  if (row0 < 0 || rows < 0 || row0 + rows > m->d.N)
    return fail(ctx, WG_OUT_OF_RANGE, "rows %d..%d are outside the matrix", row0, row0 + rows);
  return WG_OK;
}

// Copies `parts` host buffers into the staging buffer (each 256-byte
// aligned) and returns their device addresses.
struct Part {
  const void *host;
  size_t bytes;
  const uint8_t *dev;
};

int stage(wg_ctx *ctx, std::vector<Part> &parts) {
  size_t total = 0;
  for (auto &p : parts) total += align_up(p.bytes, 256);
  int st = ensure_staging(ctx, total);
  if (st) return st;
  size_t off = 0;
  for (auto &p : parts) {
    p.dev = nullptr;
    if (p.host && p.bytes) {
      // cudaMemcpyDefault: the source may be host memory (a file's bytes) or
      // device memory (bytes produced on the GPU).
      WG_CUDA(ctx, cudaMemcpyAsync(ctx->staging + off, p.host, p.bytes, cudaMemcpyDefault, ctx->stream));
      p.dev = ctx->staging + off;
    }
    off += align_up(p.bytes, 256);
  }
  return WG_OK;
}

int run_repack(wg_ctx *ctx, wg_q4mat *m, int kind, int row0, int rows, const uint8_t *src,
               size_t src_bytes, const uint8_t *scale_src, size_t scale_bytes,
               const uint8_t *zero_src, size_t zero_bytes, const int32_t *src_rows) {
  std::vector<Part> parts = {{src, src_bytes, nullptr},
                             {scale_src, scale_bytes, nullptr},
                             {zero_src, zero_bytes, nullptr},
                             {src_rows, src_rows ? (size_t)rows * 4 : 0, nullptr}};
  int st = stage(ctx, parts);
  if (st) return st;
  wg::RepackArgs a{};
  a.d = m->d;
  a.nib = m->nib;
  a.scl = m->scl;
  a.zro = m->zro;
  a.src = parts[0].dev;
  a.scale_src = parts[1].dev;
  a.zero_src = parts[2].dev;
  a.src_rows = reinterpret_cast<const int32_t *>(parts[3].dev);
  a.row0 = row0;
  a.rows = rows;
  a.kind = kind;
  WG_CUDA(ctx, wg::launch_repack(a, ctx->stream));
  return WG_OK;
}

}  // namespace

extern "C" {

int wg_init(int device, wg_ctx **out) {
  if (!out) return WG_INVALID_ARGUMENT;
  *out = nullptr;
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) return WG_NO_DEVICE;
  if (device < 0 || device >= count) return WG_NO_DEVICE;
  wg_ctx *ctx = new (std::nothrow) wg_ctx;
  if (!ctx) return WG_OUT_OF_MEMORY;
  ctx->device = device;
  int st = WG_OK;
  if ((e = cudaSetDevice(device)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device)) !=
          cudaSuccess ||
      (e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking)) != cudaSuccess ||
      (e = cudaMalloc(&ctx->d_flags, 256)) != cudaSuccess ||
      (e = cudaMemset(ctx->d_flags, 0, 256)) != cudaSuccess ||
      (e = cudaMalloc(&ctx->d_reduce, wg::kReduceBytes)) != cudaSuccess) {
    st = wg::status_of(e);
    if (ctx->d_reduce) cudaFree(ctx->d_reduce);
    if (ctx->d_flags) cudaFree(ctx->d_flags);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return st;
  }
  ctx->d_count = ctx->d_flags + 32;  // its own 128-byte line of the flags block
  ctx->stream = ctx->own_stream;
  const char *pdl = getenv("WG_PDL");
  if (pdl && pdl[0] == '0') ctx->pdl = false;
  const char *wide = getenv("WG_GEMV_WIDE");
  if (wide && (wide[0] == '0' || wide[0] == '1')) ctx->gemv_wide = wide[0] - '0';
  const char *nfb = getenv("WG_NORM_FUSE_BYTES");
  if (nfb && atol(nfb) >= 0) ctx->norm_fuse_bytes = (size_t)atol(nfb);
  const char *trig = getenv("WG_GEMV_TRIGGER");
  if (trig && trig[0] >= '0' && trig[0] <= '2') ctx->trigger_at = trig[0] - '0';
  *out = ctx;
  return WG_OK;
}

int wg_set_option(wg_ctx *ctx, int option, int value) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  switch (option) {
    case WG_OPT_EXACT_ROWS:
      if (value < 0 || value > 256) return fail(ctx, WG_INVALID_ARGUMENT, "exact rows %d (0 .. 256)", value);
      ctx->exact_rows = value;
      return WG_OK;
    default:
      return fail(ctx, WG_INVALID_ARGUMENT, "unknown option %d", option);
  }
}

int wg_destroy(wg_ctx *ctx) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->staging) cudaFree(ctx->staging);
  if (ctx->work) cudaFree(ctx->work);
  if (ctx->d_flags) cudaFree(ctx->d_flags);
  if (ctx->d_reduce) cudaFree(ctx->d_reduce);
  if (ctx->d_trace_next) cudaFree(ctx->d_trace_next);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return WG_OK;
}

int wg_set_stream(wg_ctx *ctx, void *stream) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  ctx->stream = stream ? reinterpret_cast<cudaStream_t>(stream) : ctx->own_stream;
  return WG_OK;
}

int wg_alloc(wg_ctx *ctx, size_t bytes, void **dptr) {
  if (!ctx || !dptr) return fail(ctx, WG_INVALID_ARGUMENT, "wg_alloc: null argument");
  *dptr = nullptr;
  int st = use_device(ctx);
  if (st) return st;
  WG_CUDA(ctx, cudaMalloc(dptr, bytes ? bytes : 1));
  return WG_OK;
}

int wg_free(wg_ctx *ctx, void *dptr) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  if (!dptr) return WG_OK;
  int st = use_device(ctx);
  if (st) return st;
  WG_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  WG_CUDA(ctx, cudaFree(dptr));
  return WG_OK;
}

int wg_host_alloc(wg_ctx *ctx, size_t bytes, void **hptr) {
  if (!ctx || !hptr) return fail(ctx, WG_INVALID_ARGUMENT, "wg_host_alloc: null argument");
  *hptr = nullptr;
  int st = use_device(ctx);
  if (st) return st;
  WG_CUDA(ctx, cudaMallocHost(hptr, bytes ? bytes : 1));
  return WG_OK;
}

int wg_host_free(wg_ctx *ctx, void *hptr) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  if (!hptr) return WG_OK;
  WG_CUDA(ctx, cudaFreeHost(hptr));
  return WG_OK;
}

int wg_upload(wg_ctx *ctx, void *dst, const void *src, size_t bytes) {
  if (!ctx || (!dst && bytes) || (!src && bytes))
    return fail(ctx, WG_INVALID_ARGUMENT, "wg_upload: null argument");
  if (!bytes) return WG_OK;
  int st = use_device(ctx);
  if (st) return st;
  WG_CUDA(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
  return WG_OK;
}

int wg_read(wg_ctx *ctx, void *host, const void *src, size_t bytes) {
  if (!ctx || (!host && bytes) || (!src && bytes))
    return fail(ctx, WG_INVALID_ARGUMENT, "wg_read: null argument");
  int st = use_device(ctx);
  if (st) return st;
  if (bytes) WG_CUDA(ctx, cudaMemcpyAsync(host, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return wg_sync(ctx);
}

int wg_sync(wg_ctx *ctx) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  int st = use_device(ctx);
  if (st) return st;
  WG_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  unsigned flags = 0;
  WG_CUDA(ctx, cudaMemcpy(&flags, ctx->d_flags, sizeof flags, cudaMemcpyDeviceToHost));
  if (flags) {
    WG_CUDA(ctx, cudaMemset(ctx->d_flags, 0, sizeof(unsigned)));
    if (flags & wg::kFlagTimeout)
      return fail(ctx, WG_TIMEOUT, "a device-side wait ran out (flags 0x%x)", flags);
    return fail(ctx, WG_INVALID_ARGUMENT, "a kernel rejected its arguments (flags 0x%x)", flags);
  }
  return WG_OK;
}

int wg_q4_new(wg_ctx *ctx, int N, int K, int with_zeros, wg_q4mat **out) {
  if (!ctx || !out) return fail(ctx, WG_INVALID_ARGUMENT, "wg_q4_new: null argument");
  *out = nullptr;
  int st = check_shape(ctx, N, K);
  if (st) return st;
  st = use_device(ctx);
  if (st) return st;
  wg_q4mat *m = new (std::nothrow) wg_q4mat{};
  if (!m) return fail(ctx, WG_OUT_OF_MEMORY, "host allocation failed");
  m->d = wg::q4_dims(N, K);
  m->device = ctx->device;
  const size_t tiles = (size_t)m->d.NT * m->d.KT;
  const size_t nib = align_up(tiles * wg::kTileNibBytes, 256);
  const size_t scl = align_up(tiles * wg::kTileSclBytes, 256);
  const size_t zro = with_zeros ? align_up(tiles * wg::kTileZroBytes, 256) : 0;
  m->bytes = nib + scl + zro;
  cudaError_t e = cudaMalloc(&m->base, m->bytes);
  if (e != cudaSuccess) {
    delete m;
    return cuda_fail(ctx, e, "wg_q4_new: cudaMalloc");
  }
  m->nib = reinterpret_cast<uint32_t *>(m->base);
  m->scl = reinterpret_cast<uint16_t *>(m->base + nib);
  m->zro = with_zeros ? m->base + nib + scl : nullptr;
  // Every weight 0: code 8 (0x88 bytes), scale 0, zero point 8.
  if ((e = cudaMemsetAsync(m->nib, 0x88, nib, ctx->stream)) != cudaSuccess ||
      (e = cudaMemsetAsync(m->scl, 0, scl, ctx->stream)) != cudaSuccess ||
      (with_zeros && (e = cudaMemsetAsync(m->zro, 8, zro, ctx->stream)) != cudaSuccess)) {
    cudaFree(m->base);
    delete m;
    return cuda_fail(ctx, e, "wg_q4_new: memset");
  }
  *out = m;
  return WG_OK;
}

int wg_q4_free(wg_ctx *ctx, wg_q4mat *m) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  if (!m) return WG_OK;
  int st = use_device(ctx);
  if (st) return st;
  WG_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  WG_CUDA(ctx, cudaFree(m->base));
  delete m;
  return WG_OK;
}

int wg_q4_info(const wg_q4mat *m, int *N, int *K, size_t *device_bytes) {
  if (!m) return WG_INVALID_ARGUMENT;
  if (N) *N = m->d.N;
  if (K) *K = m->d.K;
  if (device_bytes) *device_bytes = m->bytes;
  return WG_OK;
}

int wg_q4_pack_q4_0(wg_ctx *ctx, wg_q4mat *m, int row0, const uint8_t *src, size_t src_len,
                    int rows, const int32_t *src_rows) {
  if (!ctx || !m) return fail(ctx, WG_INVALID_ARGUMENT, "wg_q4_pack_q4_0: null argument");
  int st = check_rows(ctx, m, row0, rows);
  if (st) return st;
  const size_t need = (size_t)rows * (m->d.K / 32) * 18;
  // src/repack.ts:69
  if (src_len < need || (!src && need)) return fail(ctx, WG_DATA_TOO_SHORT, "Q4_0 data is too short");
  if (src_rows)
    for (int i = 0; i < rows; i++)
      if (src_rows[i] < 0 || (size_t)(src_rows[i] + 1) * (m->d.K / 32) * 18 > src_len)
        return fail(ctx, WG_DATA_TOO_SHORT, "Q4_0 data is too short for source row %d", src_rows[i]);
  if (!rows) return WG_OK;
  st = use_device(ctx);
  if (st) return st;
  size_t src_bytes = need;
  if (src_rows) {
    int hi = 0;
    for (int i = 0; i < rows; i++) hi = src_rows[i] > hi ? src_rows[i] : hi;
    src_bytes = (size_t)(hi + 1) * (m->d.K / 32) * 18;
  }
  return run_repack(ctx, m, wg::kSrcGguf, row0, rows, src, src_bytes, nullptr, 0, nullptr, 0,
                    src_rows);
}

int wg_q4_pack_nbits(wg_ctx *ctx, wg_q4mat *m, int row0, const uint8_t *quant, size_t quant_len,
                     const uint8_t *scale_bytes, size_t scale_len, const uint8_t *zp, size_t zp_len,
                     int rows, const int32_t *src_rows) {
  if (!ctx || !m) return fail(ctx, WG_INVALID_ARGUMENT, "wg_q4_pack_nbits: null argument");
  int st = check_rows(ctx, m, row0, rows);
  if (st) return st;
  const size_t blocks = m->d.K / 32, zstride = (blocks + 1) / 2;
  size_t src_n = rows;
  if (src_rows) {
    int hi = -1;
    for (int i = 0; i < rows; i++) {
      if (src_rows[i] < 0) return fail(ctx, WG_INVALID_ARGUMENT, "negative source row");
      hi = src_rows[i] > hi ? src_rows[i] : hi;
    }
    src_n = (size_t)(hi + 1);
  }
  // src/repack.ts:353-363
  if (quant_len < src_n * blocks * 16 || scale_len < src_n * blocks * 2 ||
      (!quant && rows) || (!scale_bytes && rows))
    return fail(ctx, WG_DATA_TOO_SHORT, "MatMulNBits data is too short");
  if (zp && !m->zro)
    return fail(ctx, WG_INVALID_ARGUMENT, "zero points given for a matrix without them");
  if (zp && zp_len < src_n * zstride)
    return fail(ctx, WG_DATA_TOO_SHORT, "MatMulNBits zero points are too short");
  if (!rows) return WG_OK;
  st = use_device(ctx);
  if (st) return st;
  return run_repack(ctx, m, wg::kSrcNbits, row0, rows, quant, src_n * blocks * 16, scale_bytes,
                    src_n * blocks * 2, zp, zp ? src_n * zstride : 0, src_rows);
}

int wg_q4_write_quantmatrix(wg_ctx *ctx, wg_q4mat *m, const uint32_t *quants,
                            const uint16_t *scales, const uint8_t *zeros) {
  if (!ctx || !m || !quants || !scales)
    return fail(ctx, WG_INVALID_ARGUMENT, "wg_q4_write_quantmatrix: null argument");
  if (zeros && !m->zro)
    return fail(ctx, WG_INVALID_ARGUMENT, "zero points given for a matrix without them");
  int st = use_device(ctx);
  if (st) return st;
  const size_t blocks = (size_t)m->d.N * (m->d.K / 32);
  return run_repack(ctx, m, wg::kSrcQmat, 0, m->d.N, reinterpret_cast<const uint8_t *>(quants),
                    blocks * 16, reinterpret_cast<const uint8_t *>(scales), blocks * 2, zeros,
                    zeros ? blocks : 0, nullptr);
}

int wg_q4_matrix_row(wg_ctx *ctx, const wg_q4mat *m, int n, float *out) {
  if (!ctx || !m || !out) return fail(ctx, WG_INVALID_ARGUMENT, "wg_q4_matrix_row: null argument");
  if (n < 0 || n >= m->d.N) return fail(ctx, WG_OUT_OF_RANGE, "row %d is outside the matrix", n);
  int st = use_device(ctx);
  if (st) return st;
  const int nt = n / wg::kTileRows, KT = m->d.KT;
  std::vector<uint8_t> nib((size_t)KT * wg::kTileNibBytes);
  std::vector<uint16_t> scl((size_t)KT * 32);
  std::vector<uint8_t> zro(m->zro ? (size_t)KT * 32 : 0);
  const size_t t0 = (size_t)nt * KT;
  WG_CUDA(ctx, cudaMemcpyAsync(nib.data(), reinterpret_cast<uint8_t *>(m->nib) + t0 * wg::kTileNibBytes,
                               nib.size(), cudaMemcpyDeviceToHost, ctx->stream));
  WG_CUDA(ctx, cudaMemcpyAsync(scl.data(), m->scl + t0 * 32, scl.size() * 2, cudaMemcpyDeviceToHost,
                               ctx->stream));
  if (m->zro)
    WG_CUDA(ctx, cudaMemcpyAsync(zro.data(), m->zro + t0 * 32, zro.size(), cudaMemcpyDeviceToHost,
                                 ctx->stream));
  st = wg_sync(ctx);
  if (st) return st;
  for (int k = 0; k < m->d.K; k++) {
    wg::Q4Place pl = wg::q4_place(m->d, n, k);
    const size_t nb = pl.nib_byte - t0 * wg::kTileNibBytes;
    const size_t si = pl.sz_index - t0 * 32;
    const int code = pl.nib_high ? (nib[nb] >> 4) : (nib[nb] & 15);
    const float d = __half2float(*reinterpret_cast<const __half *>(&scl[si]));
    const float z = m->zro ? (float)zro[si] : 8.0f;
    out[k] = d * ((float)code - z);
  }
  return WG_OK;
}

}  // extern "C"

// Which GEMV serves a launch of up to 8 rows: the wide one (x resident per
// CTA, columns streamed) when the tile-column GEMV would need several waves
// of CTAs or re-stage several rows of x in each of them. WG_GEMV_WIDE=0 / 1
// forces one or the other (measurement).
bool wg::gemv_use_wide(const wg_ctx *ctx, const wg::GemvArgs &a) {
  if (a.M > 32 || (a.pro.kind != wg::kProNone && a.M > wg::kProMaxTokens)) return false;
  if (ctx->gemv_wide >= 0) return ctx->gemv_wide == 1;
  wg::GemvArgs t = a;
  if (!wg::plan_gemv(t, ctx->num_sms)) return true;
  // Measured on B200 (M x N x K): the wide kernel wins from 4 rows on, and
  // for long K (>= 8192: the tile-column kernel's x re-staging) or, at 2-3
  // rows, many columns; one row of a short-K matrix stays on the
  // tile-column kernel, whose smaller CTAs overlap a chain's launches.
  if (a.M >= 4) return true;
  if (a.K >= 8192) return true;
  return a.M >= 2 && a.N >= 16384;
}

namespace {

// The matmul behind wg_q4_matmul and wg_q4_matmul_fused: y = x . W^T, with
// x given (pro == null) or made by a prologue. Arguments are checked.
int run_matmul(wg_ctx *ctx, const wg_q4mat *m, const void *x, int x_dtype, int M, void *y, int y_dtype,
               const wg::Prologue *pro, const wg_comm *push = nullptr, int epi = wg::kEpiNone,
               float *stats = nullptr) {
  int st = use_device(ctx);
  if (st) return st;
  const size_t K = m->d.K;
  if (epi == wg::kEpiSwigluPairs && (M > wg::kGemvMaxTokens || push || m->d.N % 16))
    return fail(ctx, WG_UNSUPPORTED, "the SwiGLU-pairs epilogue takes at most %d rows, N %% 16 == 0 (M %d, N %d)",
                wg::kGemvMaxTokens, M, m->d.N);
  if (epi == wg::kEpiResidual && (M > wg::kProMaxTokens || push || m->d.N % 16 || !stats))
    return fail(ctx, WG_UNSUPPORTED, "the residual epilogue takes at most %d rows, N %% 16 == 0 (M %d, N %d)",
                wg::kProMaxTokens, M, m->d.N);
  if (push && M > wg::kGemvMaxTokens)
    return fail(ctx, WG_UNSUPPORTED, "a pushing matmul takes at most %d rows (got %d)", wg::kGemvMaxTokens, M);
  // Many rows: the tcgen05 GEMM (src/engine.ts:4684: more rows than the
  // split path takes go to the prompt matmul), from ctx->exact_rows + 1 rows
  // (WG_OPT_EXACT_ROWS; measured on B200, the GEMM beats the GEMV from 17
  // rows on); pushes and epilogues stay in the GEMV, which has them (up to
  // 32 rows).
  const bool gemm_rows = push || epi != wg::kEpiNone ? M > wg::kGemvMaxTokens : M > ctx->exact_rows;
  if (gemm_rows && wg::gemm_supported()) {
    wg::GemmArgs g{};
    g.nib = m->nib;
    g.scl = m->scl;
    g.zro = m->zro;
    g.y = y;
    g.M = M;
    g.N = m->d.N;
    g.K = m->d.K;
    g.NT = m->d.NT;
    g.KT = m->d.KT;
    g.y_dtype = y_dtype;
    g.flags = ctx->d_flags;
    g.trace = ctx->trace;
    g.trace_next = ctx->d_trace_next;
    g.trace_cap = ctx->trace_cap;
    g.launch_index = ctx->launch_index++;
    wg::plan_gemm(g, ctx->num_sms);
    const size_t xh_bytes = (x_dtype == WG_F16 && !pro) ? 0 : align_up((size_t)M * K * 2, 256);
    st = ensure_work(ctx, xh_bytes);
    if (st) return st;
    const void *xh = x;
    if (pro) {
      WG_CUDA(ctx, wg::launch_prologue(*pro, M, (int)K, ctx->work, ctx->stream, ctx->pdl));
      xh = ctx->work;
    } else if (x_dtype != WG_F16) {
      WG_CUDA(ctx, wg::launch_to_f16(x, x_dtype, ctx->work, (size_t)M * K, ctx->stream));
      xh = ctx->work;
    }
    WG_CUDA(ctx, wg::launch_gemm(g, xh, ctx->stream, ctx->pdl));
    return WG_OK;
  }
  // A prologue over more rows than one fused GEMV takes runs on its own; so
  // does a norm whose row statistics would cost every CTA more than
  // ctx->norm_fuse_bytes of reads (each CTA of the fused form reads all of a
  // and b for them; 64 KB by default, WG_NORM_FUSE_BYTES for measurement).
  const bool heavy_norm = pro && pro->kind == wg::kProRmsNorm && !pro->stats &&
                          (size_t)M * K * 4 * (pro->b ? 2 : 1) > ctx->norm_fuse_bytes;
  if (pro && pro->stats && M > wg::kProMaxTokens)
    return fail(ctx, WG_UNSUPPORTED, "a norm from stats takes at most %d rows (got %d)", wg::kProMaxTokens, M);
  if (pro && (M > wg::kProMaxTokens || heavy_norm)) {
    st = ensure_work(ctx, (size_t)M * K * 2);
    if (st) return st;
    WG_CUDA(ctx, wg::launch_prologue(*pro, M, (int)K, ctx->work, ctx->stream, ctx->pdl));
    x = ctx->work;
    x_dtype = WG_F16;
    pro = nullptr;
  }
  const size_t xsz = x_dtype == WG_F32 ? 4 : 2, ysz = y_dtype == WG_F32 ? 4 : 2;
  // Rows beyond one GEMV launch go in chunks (only where the GEMM is
  // unavailable).
  for (int m0 = 0; m0 < M; m0 += wg::kGemvMaxTokens) {
    const int mc = M - m0 < wg::kGemvMaxTokens ? M - m0 : wg::kGemvMaxTokens;
    wg::GemvArgs a{};
    a.nib = m->nib;
    a.scl = m->scl;
    a.zro = m->zro;
    a.x = pro ? nullptr : reinterpret_cast<const uint8_t *>(x) + (size_t)m0 * K * xsz;
    a.y = reinterpret_cast<uint8_t *>(y) + (size_t)m0 * m->d.N * ysz;
    a.M = mc;
    a.N = m->d.N;
    a.K = m->d.K;
    a.NT = m->d.NT;
    a.KT = m->d.KT;
    a.x_dtype = pro ? WG_F16 : x_dtype;
    a.y_dtype = y_dtype;
    a.flags = ctx->d_flags;
    a.trace = ctx->trace;
    a.trace_next = ctx->d_trace_next;
    a.trace_cap = ctx->trace_cap;
    a.launch_index = ctx->launch_index++;
    a.trigger_at = ctx->trigger_at;
    if (pro) a.pro = *pro;  // M <= kProMaxTokens: one launch
    if (push) {
      a.push_on = 1;
      a.push = push->dev;
    }
    a.epi = epi;
    a.stats = stats;
    wg::GemvArgs w = a;
    if ((epi == wg::kEpiResidual || wg::gemv_use_wide(ctx, a)) && wg::plan_gemv_wide(w, ctx->num_sms)) {
      WG_CUDA(ctx, wg::launch_gemv_wide(w, ctx->stream, ctx->pdl));
      continue;
    }
    if (epi == wg::kEpiResidual)  // the residual epilogue lives in the wide kernel
      return fail(ctx, WG_UNSUPPORTED, "no wide GEMV plan for the residual epilogue (K = %d)", m->d.K);
    if (!wg::plan_gemv(a, ctx->num_sms))
      return fail(ctx, WG_UNSUPPORTED, "K = %d is beyond the GEMV's largest cluster split", m->d.K);
    WG_CUDA(ctx, wg::launch_gemv(a, ctx->stream, ctx->pdl));
  }
  return WG_OK;
}

// The device form of a caller's prologue, checked: a known kind, its inputs
// present and 16-byte aligned, resid_out aliasing neither input.
int to_prologue(wg_ctx *ctx, const wg_prologue *pro, const char *who, wg::Prologue *p) {
  *p = wg::Prologue{};
  p->kind = pro->kind;
  p->a = pro->a;
  p->b = pro->b;
  p->w = pro->weight;
  p->eps = pro->eps;
  p->out = pro->resid_out;
  p->stats = pro->stats;
  if (p->kind != WG_PRO_RMSNORM && p->kind != WG_PRO_SWIGLU)
    return fail(ctx, WG_INVALID_ARGUMENT, "%s: unknown prologue kind %d", who, p->kind);
  if (!p->a || (p->kind == WG_PRO_RMSNORM && !p->w))
    return fail(ctx, WG_INVALID_ARGUMENT, "%s: null prologue input", who);
  if (!aligned16(p->a) || !aligned16(p->b) || !aligned16(p->w) || !aligned16(p->out))
    return fail(ctx, WG_INVALID_ARGUMENT, "%s: prologue tensors must be 16-byte aligned", who);
  if (p->out && (p->out == p->a || (p->b && p->out == p->b)))
    return fail(ctx, WG_INVALID_ARGUMENT, "%s: resid_out must not alias the residual or the addend", who);
  if (p->stats && (p->kind != WG_PRO_RMSNORM || p->b || p->out || !aligned16(p->stats)))
    return fail(ctx, WG_INVALID_ARGUMENT,
                "%s: stats take a RMSNORM prologue without b and resid_out, 16-byte aligned", who);
  if (p->kind == WG_PRO_SWIGLU) p->b = nullptr, p->w = nullptr, p->out = nullptr, p->stats = nullptr;
  return WG_OK;
}

int check_matmul(wg_ctx *ctx, const wg_q4mat *m, int M, const void *y, int y_dtype) {
  if (M < 0) return fail(ctx, WG_INVALID_ARGUMENT, "negative row count %d", M);
  if (!y && M) return fail(ctx, WG_INVALID_ARGUMENT, "null y");
  if (y_dtype < WG_F32 || y_dtype > WG_BF16) return fail(ctx, WG_INVALID_ARGUMENT, "unknown y dtype %d", y_dtype);
  if (!aligned16(y)) return fail(ctx, WG_INVALID_ARGUMENT, "x and y must be 16-byte aligned");
  if (m->device != ctx->device)
    return fail(ctx, WG_INVALID_ARGUMENT, "matrix lives on device %d, context on %d", m->device, ctx->device);
  return WG_OK;
}

}  // namespace

extern "C" {

int wg_q4_matmul(wg_ctx *ctx, const wg_q4mat *m, const void *x, int x_dtype, int M, void *y,
                 int y_dtype) {
  if (!ctx || !m) return fail(ctx, WG_INVALID_ARGUMENT, "wg_q4_matmul: null argument");
  if (M < 0) return fail(ctx, WG_INVALID_ARGUMENT, "negative row count %d", M);
  if (M == 0) return WG_OK;
  if (!x || !y) return fail(ctx, WG_INVALID_ARGUMENT, "wg_q4_matmul: null x or y");
  if (x_dtype < WG_F32 || x_dtype > WG_BF16 || y_dtype < WG_F32 || y_dtype > WG_BF16)
    return fail(ctx, WG_INVALID_ARGUMENT, "unknown dtype (x %d, y %d)", x_dtype, y_dtype);
  if (!aligned16(x) || !aligned16(y))
    return fail(ctx, WG_INVALID_ARGUMENT, "x and y must be 16-byte aligned");
  int st = check_matmul(ctx, m, M, y, y_dtype);
  if (st) return st;
  return run_matmul(ctx, m, x, x_dtype, M, y, y_dtype, nullptr);
}

int wg_q4_matmul_push(wg_ctx *ctx, const wg_q4mat *m, const wg_prologue *pro, const void *x, int x_dtype, int M,
                      wg_comm *comm) {
  if (!ctx || !m || !comm) return fail(ctx, WG_INVALID_ARGUMENT, "wg_q4_matmul_push: null argument");
  if (M < 0) return fail(ctx, WG_INVALID_ARGUMENT, "negative row count %d", M);
  if (M == 0) return WG_OK;
  if (m->device != ctx->device || comm->device != ctx->device)
    return fail(ctx, WG_INVALID_ARGUMENT, "matrix, exchange and context must share a device");
  if ((size_t)M * m->d.N > (size_t)comm->dev.slot)
    return fail(ctx, WG_UNSUPPORTED, "%d x %d outputs exceed the exchange slot (%lld floats)", M, m->d.N,
                (long long)comm->dev.slot);
  if (pro) {
    wg::Prologue p;
    if (int st = to_prologue(ctx, pro, "wg_q4_matmul_push", &p)) return st;
    return run_matmul(ctx, m, nullptr, WG_F16, M, nullptr, WG_F32, &p, comm);
  }
  if (!x || !aligned16(x)) return fail(ctx, WG_INVALID_ARGUMENT, "x must be a 16-byte aligned device pointer");
  if (x_dtype < WG_F32 || x_dtype > WG_BF16) return fail(ctx, WG_INVALID_ARGUMENT, "unknown x dtype %d", x_dtype);
  return run_matmul(ctx, m, x, x_dtype, M, nullptr, WG_F32, nullptr, comm);
}

int wg_q4_matmul_ex(wg_ctx *ctx, const wg_q4mat *m, const wg_prologue *pro, const void *x, int x_dtype, int M,
                    void *y, int y_dtype, int epilogue) {
  if (!ctx || !m) return fail(ctx, WG_INVALID_ARGUMENT, "wg_q4_matmul_ex: null argument");
  int st = check_matmul(ctx, m, M, y, y_dtype);
  if (st) return st;
  if (M == 0) return WG_OK;
  if (epilogue != 0 && epilogue != WG_EPI_SWIGLU_PAIRS)
    return fail(ctx, WG_INVALID_ARGUMENT, "unknown epilogue %d", epilogue);
  const int epi = epilogue == WG_EPI_SWIGLU_PAIRS ? wg::kEpiSwigluPairs : wg::kEpiNone;
  if (pro) {
    wg::Prologue p;
    if ((st = to_prologue(ctx, pro, "wg_q4_matmul_ex", &p))) return st;
    return run_matmul(ctx, m, nullptr, WG_F16, M, y, y_dtype, &p, nullptr, epi);
  }
  if (!x || !aligned16(x)) return fail(ctx, WG_INVALID_ARGUMENT, "x must be a 16-byte aligned device pointer");
  if (x_dtype < WG_F32 || x_dtype > WG_BF16) return fail(ctx, WG_INVALID_ARGUMENT, "unknown x dtype %d", x_dtype);
  return run_matmul(ctx, m, x, x_dtype, M, y, y_dtype, nullptr, nullptr, epi);
}

int wg_q4_matmul_residual(wg_ctx *ctx, const wg_q4mat *m, const wg_prologue *pro, const void *x, int x_dtype,
                          int M, float *resid, float *stats) {
  if (!ctx || !m) return fail(ctx, WG_INVALID_ARGUMENT, "wg_q4_matmul_residual: null argument");
  int st = check_matmul(ctx, m, M, resid, WG_F32);
  if (st) return st;
  if (M == 0) return WG_OK;
  if (!stats || !aligned16(stats)) return fail(ctx, WG_INVALID_ARGUMENT, "stats must be a 16-byte aligned pointer");
  if (pro) {
    wg::Prologue p;
    if ((st = to_prologue(ctx, pro, "wg_q4_matmul_residual", &p))) return st;
    return run_matmul(ctx, m, nullptr, WG_F16, M, resid, WG_F32, &p, nullptr, wg::kEpiResidual, stats);
  }
  if (!x || !aligned16(x)) return fail(ctx, WG_INVALID_ARGUMENT, "x must be a 16-byte aligned device pointer");
  if (x_dtype < WG_F32 || x_dtype > WG_BF16) return fail(ctx, WG_INVALID_ARGUMENT, "unknown x dtype %d", x_dtype);
  return run_matmul(ctx, m, x, x_dtype, M, resid, WG_F32, nullptr, nullptr, wg::kEpiResidual, stats);
}

int wg_q4_matmul_fused(wg_ctx *ctx, const wg_q4mat *m, const wg_prologue *pro, int M, void *y, int y_dtype) {
  if (!ctx || !m || !pro) return fail(ctx, WG_INVALID_ARGUMENT, "wg_q4_matmul_fused: null argument");
  int st = check_matmul(ctx, m, M, y, y_dtype);
  if (st) return st;
  if (M == 0) return WG_OK;
  wg::Prologue p;
  if ((st = to_prologue(ctx, pro, "wg_q4_matmul_fused", &p))) return st;
  return run_matmul(ctx, m, nullptr, WG_F16, M, y, y_dtype, &p);
}

int wg_trace(wg_ctx *ctx, void *buf, size_t bytes) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  int st = use_device(ctx);
  if (st) return st;
  if (!ctx->d_trace_next) WG_CUDA(ctx, cudaMalloc(&ctx->d_trace_next, sizeof(unsigned long long)));
  WG_CUDA(ctx, cudaMemsetAsync(ctx->d_trace_next, 0, sizeof(unsigned long long), ctx->stream));
  ctx->trace = reinterpret_cast<unsigned long long *>(buf);
  ctx->trace_cap = buf ? bytes / (WG_TRACE_WORDS * sizeof(unsigned long long)) : 0;
  ctx->launch_index = 0;
  return WG_OK;
}

int wg_trace_count(wg_ctx *ctx, size_t *records) {
  if (!ctx || !records) return fail(ctx, WG_INVALID_ARGUMENT, "wg_trace_count: null argument");
  *records = 0;
  if (!ctx->d_trace_next) return WG_OK;
  int st = wg_sync(ctx);
  if (st) return st;
  unsigned long long n = 0;
  WG_CUDA(ctx, cudaMemcpy(&n, ctx->d_trace_next, sizeof n, cudaMemcpyDeviceToHost));
  *records = (size_t)(n < ctx->trace_cap ? n : ctx->trace_cap);
  return WG_OK;
}

// ---- recorded steps (CUDA graphs of the context's stream) -------------------

struct wg_graph {
  cudaGraphExec_t exec = nullptr;
  int device = 0;
};

int wg_graph_begin(wg_ctx *ctx) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  int st = use_device(ctx);
  if (st) return st;
  if (ctx->stream == nullptr || ctx->stream == cudaStreamLegacy)
    return fail(ctx, WG_INVALID_ARGUMENT, "wg_graph_begin: the legacy default stream cannot be recorded");
  WG_CUDA(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  return WG_OK;
}

int wg_graph_end(wg_ctx *ctx, wg_graph **out) {
  if (!ctx || !out) return fail(ctx, WG_INVALID_ARGUMENT, "wg_graph_end: null argument");
  *out = nullptr;
  int st = use_device(ctx);
  if (st) return st;
  cudaGraph_t graph = nullptr;
  cudaError_t e = cudaStreamEndCapture(ctx->stream, &graph);
  if (e != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    (void)cudaGetLastError();  // a spoilt capture is not a context error
    return fail(ctx, WG_CUDA_ERROR, "wg_graph_end: the recording failed (%s): a recorded call allocated or waited",
                cudaGetErrorString(e));
  }
  cudaGraphExec_t exec = nullptr;
  e = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "wg_graph_end: cudaGraphInstantiate");
  wg_graph *g = new (std::nothrow) wg_graph;
  if (!g) {
    cudaGraphExecDestroy(exec);
    return fail(ctx, WG_OUT_OF_MEMORY, "wg_graph_end: host allocation");
  }
  g->exec = exec;
  g->device = ctx->device;
  *out = g;
  return WG_OK;
}

int wg_graph_launch(wg_ctx *ctx, const wg_graph *g) {
  if (!ctx || !g) return fail(ctx, WG_INVALID_ARGUMENT, "wg_graph_launch: null argument");
  if (g->device != ctx->device)
    return fail(ctx, WG_INVALID_ARGUMENT, "wg_graph_launch: recorded on device %d, context on %d", g->device,
                ctx->device);
  int st = use_device(ctx);
  if (st) return st;
  WG_CUDA(ctx, cudaGraphLaunch(g->exec, ctx->stream));
  return WG_OK;
}

int wg_graph_free(wg_ctx *ctx, wg_graph *g) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  if (!g) return WG_OK;
  int st = use_device(ctx);
  if (st) return st;
  WG_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  cudaGraphExecDestroy(g->exec);
  delete g;
  return WG_OK;
}

const char *wg_error_string(int status) {
  switch (status) {
    case WG_OK: return "ok";
    case WG_INVALID_ARGUMENT: return "invalid argument";
    case WG_INVALID_SHAPE: return "invalid shape";
    case WG_OUT_OF_RANGE: return "out of range";
    case WG_DATA_TOO_SHORT: return "data too short";
    case WG_OUT_OF_MEMORY: return "out of memory";
    case WG_CUDA_ERROR: return "CUDA error";
    case WG_TIMEOUT: return "device wait timed out";
    case WG_DEVICE_LOST: return "the GPU context was lost";
    case WG_UNSUPPORTED: return "unsupported";
    case WG_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

const char *wg_last_error(const wg_ctx *ctx) { return ctx ? ctx->last_error.c_str() : ""; }

}  // extern "C"
