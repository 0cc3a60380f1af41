// The C ABI of include/webgllm_decoder.h: argument checks and launches.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/webgllm_decoder.h"
#include "capi_internal.cuh"
#include "decoder_kernels.cuh"

namespace {

int dfail(wg_ctx *ctx, int status, const char *fmt, ...) {
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

int finish(wg_ctx *ctx, cudaError_t e, const char *what) {
  if (e == cudaSuccess) return WG_OK;
  return dfail(ctx, wg::status_of(e), "%s: %s", what, cudaGetErrorString(e));
}

int begin(wg_ctx *ctx) {
  if (!ctx) return WG_INVALID_ARGUMENT;
  cudaError_t e = cudaSetDevice(ctx->device);
  return e == cudaSuccess ? WG_OK : finish(ctx, e, "cudaSetDevice");
}

bool dtype_ok(int d) { return d >= WG_F32 && d <= WG_BF16; }

}  // namespace

#define WG_BEGIN(ctx)          \
  do {                         \
    int st_ = begin(ctx);      \
    if (st_) return st_;       \
  } while (0)

extern "C" {

int wg_embed(wg_ctx *ctx, const int32_t *ids, int rows, const void *table, int V, int D, float *out) {
  WG_BEGIN(ctx);
  if (rows < 0 || V <= 0 || D <= 0) return dfail(ctx, WG_INVALID_SHAPE, "wg_embed: bad shape");
  if (!rows) return WG_OK;
  if (!ids || !table || !out) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_embed: null argument");
  return finish(ctx, wg::launch_embed(ids, rows, table, V, D, out, ctx->stream, ctx->pdl), "wg_embed");
}

int wg_rmsnorm(wg_ctx *ctx, float *x, const float *add, const float *weight, float eps, int rows, int D,
               void *out, int out_dtype) {
  WG_BEGIN(ctx);
  if (rows < 0 || D <= 0) return dfail(ctx, WG_INVALID_SHAPE, "wg_rmsnorm: bad shape");
  if (!rows) return WG_OK;
  if (!x || !weight || !out || !dtype_ok(out_dtype)) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_rmsnorm: argument");
  return finish(ctx, wg::launch_rmsnorm(x, add, weight, eps, rows, D, out, out_dtype, ctx->stream, ctx->pdl), "wg_rmsnorm");
}

static int check_batch(wg_ctx *ctx, const char *what, int rows, int batch) {
  if (batch <= 0 || rows % batch)
    return dfail(ctx, WG_INVALID_SHAPE, "%s: rows (%d) must be a positive multiple of batch (%d)", what, rows, batch);
  return WG_OK;
}

int wg_rope_kv(wg_ctx *ctx, const float *qkv, int rows, int batch, int H, int Hkv, int Dh, const int32_t *pos,
               float theta, const float *q_norm, const float *k_norm, float eps, void *q_out, void *k_cache,
               void *v_cache, int cache_len) {
  WG_BEGIN(ctx);
  if (rows < 0 || H <= 0 || Hkv <= 0 || H % Hkv || Dh <= 0 || Dh % 64 || Dh > 2048 || cache_len <= 0)
    return dfail(ctx, WG_INVALID_SHAPE, "wg_rope_kv: bad shape (H %d, Hkv %d, Dh %d)", H, Hkv, Dh);
  if (!rows) return WG_OK;
  if (int st = check_batch(ctx, "wg_rope_kv", rows, batch)) return st;
  if (!qkv || !pos || !q_out || !k_cache || !v_cache) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_rope_kv: null");
  return finish(ctx,
                wg::launch_rope_kv(qkv, rows, batch, H, Hkv, Dh, pos, theta, q_norm, k_norm, eps, q_out, k_cache,
                                   v_cache, cache_len, ctx->d_flags, ctx->stream, ctx->pdl),
                "wg_rope_kv");
}

// The context's wg_trace buffer for one launch (a launch index of its own).
static wg::TraceSink trace_sink(wg_ctx *ctx) {
  wg::TraceSink t;
  t.buf = ctx->trace;
  t.next = ctx->d_trace_next;
  t.cap = ctx->trace_cap;
  t.launch_index = ctx->launch_index++;
  return t;
}

int wg_attention(wg_ctx *ctx, const void *q, int rows, int batch, int H, int Hkv, int Dh, const void *k_cache,
                 const void *v_cache, int cache_len, const int32_t *pos, void *out) {
  WG_BEGIN(ctx);
  if (rows < 0 || H <= 0 || Hkv <= 0 || H % Hkv || H / Hkv > 16 ||
      !(Dh == 32 || Dh == 64 || Dh == 128 || Dh == 256) || cache_len <= 0)
    return dfail(ctx, WG_INVALID_SHAPE, "wg_attention: bad shape (H %d, Hkv %d, Dh %d, cache_len %d)", H, Hkv, Dh,
                 cache_len);
  if (!rows) return WG_OK;
  if (int st = check_batch(ctx, "wg_attention", rows, batch)) return st;
  if (!q || !k_cache || !v_cache || !pos || !out) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_attention: null");
  return finish(ctx,
                wg::launch_attention(q, rows, batch, H, Hkv, Dh, k_cache, v_cache, cache_len, pos, out, ctx->num_sms,
                                     ctx->stream, ctx->pdl, trace_sink(ctx)),
                "wg_attention");
}

int wg_rope_attention(wg_ctx *ctx, const float *qkv, int batch, int H, int Hkv, int Dh, const int32_t *pos,
                      float theta, const float *q_norm, const float *k_norm, float eps, void *k_cache, void *v_cache,
                      int cache_len, void *out) {
  WG_BEGIN(ctx);
  if (batch < 0 || H <= 0 || Hkv <= 0 || H % Hkv || H / Hkv > 16 || !(Dh == 64 || Dh == 128 || Dh == 256) ||
      cache_len <= 0)
    return dfail(ctx, WG_INVALID_SHAPE, "wg_rope_attention: bad shape (H %d, Hkv %d, Dh %d)", H, Hkv, Dh);
  if (!batch) return WG_OK;
  if (!qkv || !pos || !k_cache || !v_cache || !out) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_rope_attention: null");
  return finish(ctx,
                wg::launch_rope_attention(qkv, batch, H, Hkv, Dh, pos, theta, q_norm, k_norm, eps, k_cache, v_cache,
                                          cache_len, out, ctx->d_flags, ctx->num_sms, ctx->stream, ctx->pdl,
                                          trace_sink(ctx)),
                "wg_rope_attention");
}

int wg_swiglu(wg_ctx *ctx, const float *gate_up, int rows, int I, void *out, int out_dtype) {
  WG_BEGIN(ctx);
  if (rows < 0 || I <= 0) return dfail(ctx, WG_INVALID_SHAPE, "wg_swiglu: bad shape");
  if (!rows) return WG_OK;
  if (!gate_up || !out || !dtype_ok(out_dtype)) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_swiglu: argument");
  return finish(ctx, wg::launch_swiglu(gate_up, rows, I, out, out_dtype, ctx->stream, ctx->pdl), "wg_swiglu");
}

int wg_swiglu_pairs(wg_ctx *ctx, const float *gate_up, int rows, int I, void *out, int out_dtype) {
  WG_BEGIN(ctx);
  if (rows < 0 || I <= 0 || I % 8) return dfail(ctx, WG_INVALID_SHAPE, "wg_swiglu_pairs: bad shape (I %d)", I);
  if (!rows) return WG_OK;
  if (!gate_up || !out || !dtype_ok(out_dtype)) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_swiglu_pairs: argument");
  return finish(ctx, wg::launch_swiglu_pairs(gate_up, rows, I, out, out_dtype, ctx->stream, ctx->pdl),
                "wg_swiglu_pairs");
}

int wg_short_conv(wg_ctx *ctx, const float *bcx, int rows, int batch, int D, int W, const float *weight,
                  void *state, void *out, int out_dtype) {
  WG_BEGIN(ctx);
  if (rows < 0 || D <= 0 || W < 1 || W > 8) return dfail(ctx, WG_INVALID_SHAPE, "wg_short_conv: bad shape");
  if (!rows) return WG_OK;
  if (int st = check_batch(ctx, "wg_short_conv", rows, batch)) return st;
  if (!bcx || !weight || !state || !out || !dtype_ok(out_dtype))
    return dfail(ctx, WG_INVALID_ARGUMENT, "wg_short_conv: argument");
  return finish(ctx,
                wg::launch_short_conv(bcx, rows, batch, D, W, weight, state, out, out_dtype, nullptr, 0, 0,
                                      ctx->stream, ctx->pdl),
                "wg_short_conv");
}

int wg_short_conv_prefixes(wg_ctx *ctx, const float *bcx, int rows, int batch, int D, int W, const float *weight,
                           void *state, void *out, int out_dtype, void *prefixes, int slot0, int slots) {
  WG_BEGIN(ctx);
  if (rows < 0 || D <= 0 || W < 2 || W > 8) return dfail(ctx, WG_INVALID_SHAPE, "wg_short_conv_prefixes: bad shape");
  if (!rows) return WG_OK;
  if (int st = check_batch(ctx, "wg_short_conv_prefixes", rows, batch)) return st;
  if (!bcx || !weight || !state || !out || !prefixes || !dtype_ok(out_dtype))
    return dfail(ctx, WG_INVALID_ARGUMENT, "wg_short_conv_prefixes: argument");
  if (slot0 < 0 || slots < 1 || slot0 + rows / batch > slots)
    return dfail(ctx, WG_INVALID_SHAPE, "wg_short_conv_prefixes: %d rows a sequence from slot %d of %d", rows / batch,
                 slot0, slots);
  return finish(ctx,
                wg::launch_short_conv(bcx, rows, batch, D, W, weight, state, out, out_dtype, prefixes, slot0, slots,
                                      ctx->stream, ctx->pdl),
                "wg_short_conv_prefixes");
}

int wg_conv_restore(wg_ctx *ctx, const void *prefixes, int slots, int batch, int D, int W, const int32_t *pos_before,
                    const int32_t *pos_after, void *state) {
  WG_BEGIN(ctx);
  if (batch < 0 || D <= 0 || W < 2 || W > 8 || slots < 1)
    return dfail(ctx, WG_INVALID_SHAPE, "wg_conv_restore: bad shape");
  if (!batch) return WG_OK;
  if (!prefixes || !pos_before || !pos_after || !state)
    return dfail(ctx, WG_INVALID_ARGUMENT, "wg_conv_restore: argument");
  return finish(ctx,
                wg::launch_conv_restore(prefixes, slots, batch, D, W, pos_before, pos_after, state, ctx->stream,
                                        ctx->pdl),
                "wg_conv_restore");
}

static int check_head(wg_ctx *ctx, int rows, int D, int V) {
  if (rows < 0 || rows > 8 || D <= 0 || D % 8 || V <= 0 || (size_t)rows * D * 4 > 200 * 1024)
    return dfail(ctx, WG_INVALID_SHAPE, "head: rows %d (<= 8), D %d (multiple of 8, rows * D <= 51200)", rows, D);
  return WG_OK;
}

int wg_head(wg_ctx *ctx, const void *x, int rows, int D, const void *W, int V, float *logits, int32_t *argmax) {
  WG_BEGIN(ctx);
  if (int st = check_head(ctx, rows, D, V)) return st;
  if (!rows) return WG_OK;
  if (!x || !W || !logits) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_head: null");
  return finish(ctx,
                wg::launch_head(x, nullptr, nullptr, nullptr, 0.0f, rows, 1, D, W, V, 0, logits, argmax, nullptr,
                                ctx->d_reduce, wg::kReduceBytes, ctx->d_count, ctx->d_flags, ctx->num_sms,
                                ctx->stream, ctx->pdl),
                "wg_head");
}

int wg_head_rmsnorm(wg_ctx *ctx, const float *resid, const float *add, const float *weight, float eps, int rows,
                    int row_stride, int D, const void *W, int V, int vocab_offset, float *logits, int32_t *argmax,
                    int64_t *keys) {
  WG_BEGIN(ctx);
  if (int st = check_head(ctx, rows, D, V)) return st;
  if (row_stride < 1 || vocab_offset < 0)
    return dfail(ctx, WG_INVALID_SHAPE, "wg_head_rmsnorm: row_stride %d, vocab_offset %d", row_stride, vocab_offset);
  if (!rows) return WG_OK;
  if (!resid || !weight || !W || !logits) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_head_rmsnorm: null");
  return finish(ctx,
                wg::launch_head(nullptr, resid, add, weight, eps, rows, row_stride, D, W, V, vocab_offset, logits,
                                argmax, reinterpret_cast<unsigned long long *>(keys), ctx->d_reduce, wg::kReduceBytes,
                                ctx->d_count, ctx->d_flags, ctx->num_sms, ctx->stream, ctx->pdl),
                "wg_head_rmsnorm");
}

int wg_pick_keys(wg_ctx *ctx, const int64_t *keys, int rows, int32_t *ids) {
  WG_BEGIN(ctx);
  if (rows < 0) return dfail(ctx, WG_INVALID_SHAPE, "wg_pick_keys: rows %d", rows);
  if (!rows) return WG_OK;
  if (!keys || !ids) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_pick_keys: null");
  return finish(ctx,
                wg::launch_pick_keys(reinterpret_cast<const unsigned long long *>(keys), rows, ids, ctx->stream,
                                     ctx->pdl),
                "wg_pick_keys");
}

int wg_argmax(wg_ctx *ctx, const float *logits, int rows, int V, int32_t *out) {
  WG_BEGIN(ctx);
  if (rows < 0 || V <= 0) return dfail(ctx, WG_INVALID_SHAPE, "wg_argmax: bad shape");
  if (!rows) return WG_OK;
  if (!logits || !out) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_argmax: null");
  return finish(ctx, wg::launch_argmax(logits, rows, V, out, ctx->stream, ctx->pdl), "wg_argmax");
}

int wg_spec_accept(wg_ctx *ctx, const int32_t *drafts, const int32_t *picks, int batch, int k, int32_t *pos_target,
                   int32_t *pos_draft, int32_t *next_target, int32_t *next_draft, int32_t *out, int out_cap,
                   int32_t *out_len, int32_t *accepted) {
  WG_BEGIN(ctx);
  if (batch < 0 || k < 0 || out_cap < 0) return dfail(ctx, WG_INVALID_SHAPE, "wg_spec_accept: bad shape");
  if (!batch) return WG_OK;
  if ((k && !drafts) || !picks || !pos_target || !pos_draft || !next_target || !next_draft || !out_len || !accepted ||
      (out_cap && !out))
    return dfail(ctx, WG_INVALID_ARGUMENT, "wg_spec_accept: null");
  return finish(ctx,
                wg::launch_spec_accept(drafts, picks, batch, k, pos_target, pos_draft, next_target, next_draft, out,
                                       out_cap, out_len, accepted, ctx->stream, ctx->pdl),
                "wg_spec_accept");
}

int wg_add_i32(wg_ctx *ctx, int32_t *counters, int n, int delta) {
  WG_BEGIN(ctx);
  if (n < 0) return dfail(ctx, WG_INVALID_SHAPE, "wg_add_i32: n %d", n);
  if (!n) return WG_OK;
  if (!counters) return dfail(ctx, WG_INVALID_ARGUMENT, "wg_add_i32: null");
  return finish(ctx, wg::launch_add_i32(counters, n, delta, ctx->stream, ctx->pdl), "wg_add_i32");
}

}  // extern "C"
