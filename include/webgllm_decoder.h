/*
 * webgllm_decoder.h: the decoder-layer kernels around the Q4 matmuls
 * (libwebgllm_b200.so), standing in for the engine's other per-layer passes
 * (src/engine.ts:8875-9304 forwardBatch) on the B200. Paths are inside the
 * webgllm package (packages/webgllm/). Conventions as webgllm_q4.h: status
 * returns, device pointers, work enqueued on the context's stream.
 *
 * Layouts: row-major [rows][features]. The residual stream is fp32; matmul
 * inputs fp16 (WG_F16); caches fp16. Sequences: where a call takes `batch`,
 * its `rows` are `batch` independent sequences of rows / batch consecutive
 * tokens each (a decode step of 8 sequences: rows 8, batch 8; one prompt:
 * rows = its length, batch 1); `pos` is a device int32 [batch] holding each
 * sequence's position of its first row, and caches / states carry a leading
 * [batch] dimension. Positions live on the device, so a decode step can be
 * replayed from a CUDA graph while they advance.
 */
#ifndef WEBGLLM_DECODER_H
#define WEBGLLM_DECODER_H

#include <stddef.h>
#include <stdint.h>

#include "webgllm_q4.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Embedding rows (src/gpu/kernels.ts:1092; engine.ts:8961-9030): out[r] =
 * table[ids[r]] as fp32, table fp16 [V][D]; ids outside [0, V) read row 0. */
int wg_embed(wg_ctx *ctx, const int32_t *ids, int rows, const void *table, int V, int D, float *out);

/* Residual add + RMS norm (addNormed, src/engine.ts:5695; RMS passes
 * src/gpu/kernels.ts:1158-1372): x += add (if add is not NULL; x keeps the
 * sum), out = x / sqrt(mean(x^2) + eps) * weight in out_dtype. */
int wg_rmsnorm(wg_ctx *ctx, float *x, const float *add, const float *weight, float eps, int rows, int D,
               void *out, int out_dtype);

/* qk-norm + RoPE + KV append (headPrep, src/gpu/kernels.ts:2196-2322):
 * qkv fp32 [rows][(H + 2 Hkv) Dh] (q | k | v). Per head, optional RMS norm
 * over Dh with q_norm / k_norm weights (NULL: none), then rotate-half RoPE
 * of the pairs (j, j + Dh/2) by p * theta^(-2j/Dh), p the row's position.
 * q_out fp16 [rows][H][Dh] scaled by 1/sqrt(Dh); k (rotated) and v appended
 * to the fp16 caches [batch][Hkv][cache_len][Dh] at each row's position.
 * Dh % 64 == 0. A position past cache_len is skipped and reported by
 * wg_sync. */
int wg_rope_kv(wg_ctx *ctx, const float *qkv, int rows, int batch, int H, int Hkv, int Dh, const int32_t *pos,
               float theta, const float *q_norm, const float *k_norm, float eps, void *q_out, void *k_cache,
               void *v_cache, int cache_len);

/* Causal GQA attention over the fp16 caches [batch][Hkv][cache_len][Dh]
 * (scores / attend, src/gpu/kernels.ts:2386-2579): a query row at position p
 * of head h attends keys 0..p of its sequence's KV head h / (H / Hkv). q fp16 [rows][H][Dh]
 * (already scaled), out fp16 [rows][H][Dh]. Dh in {32, 64, 128, 256},
 * H / Hkv <= 16. Each (row, KV head) is served by a cluster of up to 8
 * CTAs that split the keys and merge through distributed shared memory. */
int wg_attention(wg_ctx *ctx, const void *q, int rows, int batch, int H, int Hkv, int Dh, const void *k_cache,
                 const void *v_cache, int cache_len, const int32_t *pos, void *out);

/* wg_rope_kv followed by wg_attention for a decode step (one row per
 * sequence: rows = batch), in one launch: each CTA forms its heads' rotated
 * queries itself and the CTA whose key slice holds the new position appends
 * the new key and value to the caches. Same results as the two calls;
 * Dh in {64, 128, 256}. */
int wg_rope_attention(wg_ctx *ctx, const float *qkv, int batch, int H, int Hkv, int Dh, const int32_t *pos,
                      float theta, const float *q_norm, const float *k_norm, float eps, void *k_cache, void *v_cache,
                      int cache_len, void *out);

/* SwiGLU (REDUCE_SWIGLU, src/gpu/kernels.ts:1066-1077): gate_up fp32
 * [rows][2I] (gate | up) -> out[r][i] = silu(gate) * up, in out_dtype. */
int wg_swiglu(wg_ctx *ctx, const float *gate_up, int rows, int I, void *out, int out_dtype);

/* The same for a gate|up matrix packed interleaved by 8 (see
 * WG_EPI_SWIGLU_PAIRS): gate_up [rows][2I] with columns 16t .. 16t+7 = gate
 * features 8t .. 8t+7 and 16t+8 .. 16t+15 = their up values. I % 8 == 0. */
int wg_swiglu_pairs(wg_ctx *ctx, const float *gate_up, int rows, int I, void *out, int out_dtype);

/* LFM2 gated short convolution (shortConv / convState,
 * src/gpu/kernels.ts:1380-1437): bcx fp32 [rows][3D] = B | C | x,
 * y = B * x, out[t] = C[t] * sum_k weight[c][k] * y[t - (W-1-k)] (weight fp32
 * [D][W]); per sequence, y before its rows comes from its state fp16
 * [W-1][D] (oldest first; states [batch][W-1][D]), which is updated to the
 * sequence's last W-1 values of y. W <= 8. */
int wg_short_conv(wg_ctx *ctx, const float *bcx, int rows, int batch, int D, int W, const float *weight,
                  void *state, void *out, int out_dtype);

/* wg_short_conv that also keeps the state after each prefix of a
 * sequence's rows (convPrefixes, src/gpu/kernels.ts:1504 and
 * src/engine.ts:5902, for speculative decoding, which may keep only some of
 * a draft batch's tokens): prefixes fp16 [batch][slots][W-1][D], slot
 * slot0 + p - 1 = the state after the first p rows (p = 1 .. rows/batch;
 * slot0 + rows/batch <= slots). A draft model decoding one row at a time
 * passes slot0 = its step index. W >= 2. */
int wg_short_conv_prefixes(wg_ctx *ctx, const float *bcx, int rows, int batch, int D, int W, const float *weight,
                           void *state, void *out, int out_dtype, void *prefixes, int slot0, int slots);

/* The conv-state rollback of accept (src/engine.ts:8063-8085): per sequence,
 * kept = pos_after[b] - pos_before[b] tokens of the last `slots`-token draft
 * batch were kept; when 1 <= kept < slots, state[b] = prefixes[b][kept-1]
 * (positions on the device, as wg_spec_accept leaves them). */
int wg_conv_restore(wg_ctx *ctx, const void *prefixes, int slots, int batch, int D, int W, const int32_t *pos_before,
                    const int32_t *pos_after, void *state);

/* fp16 output head (head, src/engine.ts:8557): logits fp32 [rows][V] =
 * x fp16 [rows][D] . W^T, W fp16 [V][D]; rows <= 8, D % 8 == 0,
 * rows * D <= 51200. If `argmax` is not NULL it also receives each row's
 * greedy token as wg_argmax would (same launch). Calls that pass `argmax`
 * must not overlap on one context (they share its reduction buffer). */
int wg_head(wg_ctx *ctx, const void *x, int rows, int D, const void *W, int V, float *logits, int32_t *argmax);

/* wg_head on the final norm of the residual stream, in one launch: input
 * row r = rmsnorm(resid + add) * weight of row r * row_stride of resid /
 * add (fp32, [.][D], not written; add may be NULL), rounded to fp16 as
 * wg_rmsnorm would store it (the engine's last addNormed before head,
 * src/engine.ts:9304). For a vocabulary shard W = rows vocab_offset ..
 * vocab_offset + V - 1 of the full head: argmax receives global indices,
 * and `keys` (NULL: not written) each row's packed key, an int64 that
 * orders as (logit, then lower index): the maximum over shards (an
 * all-reduce MAX on int64) is the full head's greedy pick; see
 * wg_pick_keys. */
int wg_head_rmsnorm(wg_ctx *ctx, const float *resid, const float *add, const float *weight, float eps, int rows,
                    int row_stride, int D, const void *W, int V, int vocab_offset, float *logits, int32_t *argmax,
                    int64_t *keys);

/* ids[r] = the token index packed in keys[r] (wg_head_rmsnorm). */
int wg_pick_keys(wg_ctx *ctx, const int64_t *keys, int rows, int32_t *ids);

/* Greedy pick (src/engine.ts:8271 argmax): out[r] = index of the largest
 * logit of row r (the lowest index on ties). */
int wg_argmax(wg_ctx *ctx, const float *logits, int rows, int V, int32_t *out);

/* Greedy speculative decoding: acceptance of a draft's k proposals per
 * sequence (forwardDraft / accept, src/engine.ts:8035,8063: keys and values
 * past the kept rows are never read before they are written again, so the
 * rollback is the position alone for attention layers; conv layers restore
 * their state with wg_conv_restore). drafts [batch][k] = the draft's tokens d_1..d_k;
 * picks [k+1][batch] = the target's greedy picks after each verified row
 * (rows: the last kept token, then d_1..d_k). Keeps the longest prefix with
 * d_{j+1} == picks[j], appends it and the target's pick after it to
 * out [batch][out_cap] at out_len[b] (which advances), adds the number of
 * accepted draft tokens to accepted[b], sets both next tokens to that pick and
 * both positions to just past the kept rows (pos_target had advanced by k + 1
 * in the verify forward). */
int wg_spec_accept(wg_ctx *ctx, const int32_t *drafts, const int32_t *picks, int batch, int k, int32_t *pos_target,
                   int32_t *pos_draft, int32_t *next_target, int32_t *next_draft, int32_t *out, int out_cap,
                   int32_t *out_len, int32_t *accepted);

/* counters[0..n) += delta on the device (advances the positions of a
 * replayed decode step). */
int wg_add_i32(wg_ctx *ctx, int32_t *counters, int n, int delta);

#ifdef __cplusplus
}
#endif

#endif /* WEBGLLM_DECODER_H */
