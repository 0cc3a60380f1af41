// wg_q4_matmul_static: the Q4 matmul without any device allocation.
//
// wg_q4_matmul keeps its scratch (the fp16 copy of x that the GEMM reads when
// x is f32 / bf16) in a buffer that it grows with cudaMalloc on first use of
// a larger shape. Some callers
// cannot let a library allocate: code recording a CUDA graph (allocation is
// not allowed while a stream is being captured), engines that budget device
// memory up front and must not see it grow behind their back, and decode
// loops where cudaMalloc / cudaFree would stall on an implicit device
// synchronisation. This entry point serves them: its scratch is a fixed
// array in the library's own device memory, present from the moment the
// library is loaded on a GPU.
//
// Limits and sharing:
// - kScratchBytes (32 MiB) is the most scratch one call may use; a call that
//   would need more is rejected with WG_UNSUPPORTED and a message naming
//   both sizes. Every GPU that loads the library holds the array until the
//   process exits.
// - All calls on a device share the one array and it keeps the last call's
//   contents: two calls whose work overlaps on the GPU (different streams, or
//   different contexts of the same device) race on it. Nothing in it needs to
//   start at zero (each call writes the whole fp16 copy it then reads).
// - The first call on a device looks up the array's device address
//   (cudaGetSymbolAddress); make that first call before capturing a stream.
//   The address is kept for the life of the process: after a
//   cudaDeviceReset of that device (which destroys the context the address
//   belongs to) this entry point must not be called again.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "capi_internal.cuh"
#include "q4_kernels.cuh"

namespace {

constexpr size_t kScratchBytes = (size_t)32 << 20;
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void *g_scratch_addr[kMaxDevices];  // device address of g_scratch, per device
std::mutex g_scratch_lock;

int fail_static(wg_ctx *ctx, int status, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  ctx->last_error = buf;
  return status;
}

// The device address of this device's array. In host code `g_scratch` names
// a host-side stand-in, not device memory: only this address may be passed
// to kernels.
int scratch_address(wg_ctx *ctx, unsigned char **out) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices)
    return fail_static(ctx, WG_UNSUPPORTED, "device %d is beyond the static scratch table", ctx->device);
  std::lock_guard<std::mutex> guard(g_scratch_lock);
  if (!g_scratch_addr[ctx->device]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || !p)
      return fail_static(ctx, wg::status_of(e == cudaSuccess ? cudaErrorInvalidSymbol : e),
                         "cudaGetSymbolAddress of the static scratch: %s", cudaGetErrorString(e));
    g_scratch_addr[ctx->device] = p;
  }
  *out = static_cast<unsigned char *>(g_scratch_addr[ctx->device]);
  return WG_OK;
}

size_t round256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

extern "C" int wg_q4_matmul_static(wg_ctx *ctx, const wg_q4mat *m, const void *x, int x_dtype, int M, void *y,
                                   int y_dtype) {
  if (!ctx || !m) return ctx ? fail_static(ctx, WG_INVALID_ARGUMENT, "wg_q4_matmul_static: null argument")
                             : WG_INVALID_ARGUMENT;
  if (M < 0) return fail_static(ctx, WG_INVALID_ARGUMENT, "negative row count %d", M);
  if (M == 0) return WG_OK;
  if (!x || !y) return fail_static(ctx, WG_INVALID_ARGUMENT, "wg_q4_matmul_static: null x or y");
  if (x_dtype < WG_F32 || x_dtype > WG_BF16 || y_dtype < WG_F32 || y_dtype > WG_BF16)
    return fail_static(ctx, WG_INVALID_ARGUMENT, "unknown dtype (x %d, y %d)", x_dtype, y_dtype);
  if (((uintptr_t)x & 15u) || ((uintptr_t)y & 15u))
    return fail_static(ctx, WG_INVALID_ARGUMENT, "x and y must be 16-byte aligned");
  if (m->device != ctx->device)
    return fail_static(ctx, WG_INVALID_ARGUMENT, "matrix lives on device %d, context on %d", m->device,
                       ctx->device);
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return fail_static(ctx, wg::status_of(e), "cudaSetDevice: %s", cudaGetErrorString(e));

  // The same routing as wg_q4_matmul: the GEMM above the context's exact rows.
  if (M > ctx->exact_rows && wg::gemm_supported()) {
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
    wg::plan_gemm(g, ctx->num_sms);
    const size_t xh_bytes = x_dtype == WG_F16 ? 0 : round256((size_t)M * m->d.K * 2);
    if (xh_bytes > kScratchBytes)
      return fail_static(ctx, WG_UNSUPPORTED,
                         "this matmul needs %zu bytes of scratch; the static scratch holds %zu "
                         "(use wg_q4_matmul, which allocates)",
                         xh_bytes, kScratchBytes);
    unsigned char *scratch = nullptr;
    int st = scratch_address(ctx, &scratch);
    if (st) return st;
    const void *xh = x;
    if (x_dtype != WG_F16) {
      e = wg::launch_to_f16(x, x_dtype, scratch, (size_t)M * m->d.K, ctx->stream);
      if (e != cudaSuccess) return fail_static(ctx, wg::status_of(e), "x conversion: %s", cudaGetErrorString(e));
      xh = scratch;
    }
    e = wg::launch_gemm(g, xh, ctx->stream, ctx->pdl);
    if (e != cudaSuccess) return fail_static(ctx, wg::status_of(e), "GEMM launch: %s", cudaGetErrorString(e));
    return WG_OK;
  }

  // Few rows: the GEMV (tile-column or wide kernel, chosen as wg_q4_matmul
  // chooses), which needs no scratch at all.
  const size_t xsz = x_dtype == WG_F32 ? 4 : 2, ysz = y_dtype == WG_F32 ? 4 : 2;
  for (int m0 = 0; m0 < M; m0 += wg::kGemvMaxTokens) {
    const int mc = M - m0 < wg::kGemvMaxTokens ? M - m0 : wg::kGemvMaxTokens;
    wg::GemvArgs a{};
    a.nib = m->nib;
    a.scl = m->scl;
    a.zro = m->zro;
    a.x = reinterpret_cast<const uint8_t *>(x) + (size_t)m0 * m->d.K * xsz;
    a.y = reinterpret_cast<uint8_t *>(y) + (size_t)m0 * m->d.N * ysz;
    a.M = mc;
    a.N = m->d.N;
    a.K = m->d.K;
    a.NT = m->d.NT;
    a.KT = m->d.KT;
    a.x_dtype = x_dtype;
    a.y_dtype = y_dtype;
    a.flags = ctx->d_flags;
    a.trigger_at = ctx->trigger_at;
    wg::GemvArgs w = a;
    if (wg::gemv_use_wide(ctx, a) && wg::plan_gemv_wide(w, ctx->num_sms)) {
      e = wg::launch_gemv_wide(w, ctx->stream, ctx->pdl);
      if (e != cudaSuccess) return fail_static(ctx, wg::status_of(e), "GEMV launch: %s", cudaGetErrorString(e));
      continue;
    }
    if (!wg::plan_gemv(a, ctx->num_sms))
      return fail_static(ctx, WG_UNSUPPORTED, "K = %d is beyond the GEMV's largest cluster split", m->d.K);
    e = wg::launch_gemv(a, ctx->stream, ctx->pdl);
    if (e != cudaSuccess) return fail_static(ctx, wg::status_of(e), "GEMV launch: %s", cudaGetErrorString(e));
  }
  return WG_OK;
}
