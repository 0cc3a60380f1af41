// Launchers of the decoder-layer kernels (decoder.cu); internal. `pdl`:
// launch with programmatic dependent launch (the kernels wait for their
// predecessor on the device).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace wg {

cudaError_t launch_embed(const int32_t *ids, int rows, const void *table, int V, int D, float *out, cudaStream_t s,
                         bool pdl);
cudaError_t launch_rmsnorm(float *x, const float *add, const float *w, float eps, int rows, int D, void *out,
                           int out_dtype, cudaStream_t s, bool pdl);
cudaError_t launch_rope_kv(const float *qkv, int rows, int H, int Hkv, int Dh, const int *pos0, float theta,
                           const float *q_norm, const float *k_norm, float eps, void *q_out, void *k_cache,
                           void *v_cache, int cache_len, unsigned *flags, cudaStream_t s, bool pdl);
cudaError_t launch_attention(const void *q, int rows, int H, int Hkv, int Dh, const void *k_cache,
                             const void *v_cache, int cache_len, const int *pos0, void *out, cudaStream_t s,
                             bool pdl);
cudaError_t launch_swiglu(const float *gu, int rows, int I, void *out, int out_dtype, cudaStream_t s, bool pdl);
cudaError_t launch_short_conv(const float *bcx, int rows, int D, int W, const float *w, void *state, void *out,
                              int out_dtype, cudaStream_t s, bool pdl);
// x fp16 [rows][D], or with na != null the norm rmsnorm(na + nb) * nw.
cudaError_t launch_head(const void *x, const float *na, const float *nb, const float *nw, float eps, int rows, int D,
                        const void *W, int V, float *logits, int32_t *amax, unsigned long long *part,
                        size_t part_bytes, unsigned *count, int num_sms, cudaStream_t s, bool pdl);
cudaError_t launch_argmax(const float *logits, int rows, int V, int32_t *out, cudaStream_t s, bool pdl);
cudaError_t launch_add_i32(int32_t *p, int delta, cudaStream_t s, bool pdl);

}  // namespace wg
