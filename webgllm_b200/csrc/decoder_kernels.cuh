// Launchers of the decoder-layer kernels (decoder.cu); internal. `pdl`:
// launch with programmatic dependent launch (the kernels wait for their
// predecessor on the device).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace wg {

// Where a traced launch appends its per-CTA records (wg_trace); buf null:
// no tracing.
struct TraceSink {
  unsigned long long *buf = nullptr;
  unsigned long long *next = nullptr;
  unsigned long long cap = 0;
  unsigned launch_index = 0;
};

cudaError_t launch_embed(const int32_t *ids, int rows, const void *table, int V, int D, float *out, cudaStream_t s,
                         bool pdl);
cudaError_t launch_rmsnorm(float *x, const float *add, const float *w, float eps, int rows, int D, void *out,
                           int out_dtype, cudaStream_t s, bool pdl);
// rope / attention / short conv: `rows` = batch sequences x rows / batch
// consecutive tokens each; pos0[batch]; caches / states [batch][...].
cudaError_t launch_rope_kv(const float *qkv, int rows, int batch, int H, int Hkv, int Dh, const int *pos0,
                           float theta, const float *q_norm, const float *k_norm, float eps, void *q_out,
                           void *k_cache, void *v_cache, int cache_len, unsigned *flags, cudaStream_t s, bool pdl);
cudaError_t launch_attention(const void *q, int rows, int batch, int H, int Hkv, int Dh, const void *k_cache,
                             const void *v_cache, int cache_len, const int *pos0, void *out, int num_sms,
                             cudaStream_t s, bool pdl, const TraceSink &tr = TraceSink{});
// Prompts (attention_prefill.cu): flash attention on the tensor cores for
// rows / batch >= kFaPrefillMinRows query rows per sequence and Dh 64 / 128;
// launch_attention routes those shapes to it.
constexpr int kFaPrefillMinRows = 16;
bool flash_prefill_supported(int rps, int Dh);
cudaError_t launch_flash_prefill(const void *q, int rps, int batch, int H, int Hkv, int Dh, const void *k_cache,
                                 const void *v_cache, int cache_len, const int *pos0, void *out, cudaStream_t s,
                                 bool pdl);
// Decode (one row per sequence): rope_kv + attention in one launch.
cudaError_t launch_rope_attention(const float *qkv, int batch, int H, int Hkv, int Dh, const int *pos0, float theta,
                                  const float *q_norm, const float *k_norm, float eps, void *k_cache, void *v_cache,
                                  int cache_len, void *out, unsigned *flags, int num_sms, cudaStream_t s, bool pdl,
                                  const TraceSink &tr = TraceSink{});
cudaError_t launch_swiglu(const float *gu, int rows, int I, void *out, int out_dtype, cudaStream_t s, bool pdl);
cudaError_t launch_swiglu_pairs(const float *gu, int rows, int I, void *out, int out_dtype, cudaStream_t s,
                                bool pdl);
// prefixes (nullable): fp16 [batch][slots][W-1][D], the state after each
// prefix of a sequence's rows into slots slot0 ...
cudaError_t launch_short_conv(const float *bcx, int rows, int batch, int D, int W, const float *w, void *state,
                              void *out, int out_dtype, void *prefixes, int slot0, int slots, cudaStream_t s,
                              bool pdl);
cudaError_t launch_conv_restore(const void *prefixes, int slots, int batch, int D, int W, const int32_t *pos_before,
                                const int32_t *pos_after, void *state, cudaStream_t s, bool pdl);
// x fp16 [rows][D], or with na != null the norm rmsnorm(na + nb) * nw; input
// row r is row r * row_stride of x / na / nb.
cudaError_t launch_head(const void *x, const float *na, const float *nb, const float *nw, float eps, int rows,
                        int row_stride, int D, const void *W, int V, int vocab_offset, float *logits, int32_t *amax,
                        unsigned long long *keys, unsigned long long *part, size_t part_bytes, unsigned *count,
                        unsigned *flags, int num_sms, cudaStream_t s, bool pdl);
cudaError_t launch_pick_keys(const unsigned long long *keys, int rows, int32_t *ids, cudaStream_t s, bool pdl);
cudaError_t launch_argmax(const float *logits, int rows, int V, int32_t *out, cudaStream_t s, bool pdl);
cudaError_t launch_add_i32(int32_t *p, int n, int delta, cudaStream_t s, bool pdl);
cudaError_t launch_spec_accept(const int32_t *drafts, const int32_t *picks, int batch, int k, int32_t *pos_t,
                               int32_t *pos_d, int32_t *next_t, int32_t *next_d, int32_t *out, int out_cap,
                               int32_t *out_len, int32_t *accepted, cudaStream_t s, bool pdl);

}  // namespace wg
