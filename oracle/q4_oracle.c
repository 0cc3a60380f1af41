/*
 * CPU ORACLE for the Q4 matmul hot path. TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic of webgllm's 4-bit matmul
 * path so that the CUDA library can be checked against it. Nothing in the
 * product links or calls it: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py load it, as the checker or as
 * the timed CPU baseline.
 *
 * Each function names the reference lines it follows (paths inside the
 * webgllm package, packages/webgllm/):
 *
 *   orc_to_half            src/half.ts:7-32        (round to nearest even)
 *   orc_to_half_bench      bench/q4-matmul.js:196-213 (adds 0x1000: ties up)
 *   orc_from_half          src/half.ts:36-53
 *   orc_pack_q4_0          src/repack.ts:60-87     (+ checks repack.ts:21-24,47-54)
 *   orc_pack_matmulnbits   src/repack.ts:342-392
 *   orc_quants_from_raw    src/repack.ts:216-242
 *   orc_matrix_row         src/repack.ts:865-891
 *   orc_q4_ref_f64         bench/gpu-bench-worker.js:41-55 (fp64 reference)
 *   orc_q4_split_emulate   src/gpu/kernels.ts:744-895 (matmulSplitRgba4 block
 *                          math, words form kernels.ts:182-217), split sizing
 *                          src/engine.ts:5316-5327, fp16 partials
 *                          src/engine.ts:343,1483-1489, consumer sum
 *                          kernels.ts:69-79
 *   orc_q4_prefill_emulate src/gpu/kernels.ts:436-597 (dequant to fp16),
 *                          :620-735 (f16 matmul), slicing engine.ts:4957-4967,
 *                          fp16 outputs kernels.ts:32-36 (packH2), consumer
 *                          sum kernels.ts:55-68 (pfq)
 *
 * QuantMatrix layout (src/weights.ts:5-21): quants index in words
 * ((g * blocks + b) * 4 + r) * 4 + w for row group g = n / 4, row r = n % 4;
 * scales/zeros index (g * blocks + b) * 4 + r. Zero pointer NULL means 8.
 *
 * Status codes returned here match include/webgllm_q4.h's WG_* values.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_OK 0
#define ORC_INVALID_ARGUMENT 1
#define ORC_INVALID_SHAPE 2
#define ORC_OUT_OF_RANGE 3
#define ORC_DATA_TOO_SHORT 4

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* src/half.ts:7-32: float to IEEE half bits, round to nearest even. */
uint16_t orc_to_half(float value) {
  uint32_t x = f2u(value);
  uint32_t sign = (x >> 16) & 0x8000u;
  int exp = (int)((x >> 23) & 0xffu);
  uint32_t mant = x & 0x7fffffu;
  if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
  int e = exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    mant |= 0x800000u;
    int shift = 14 - e;
    uint32_t half = 1u << (shift - 1);
    uint32_t rest = mant & ((1u << shift) - 1u);
    uint32_t h = mant >> shift;
    if (rest > half || (rest == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)e << 10) | (mant >> 13);
  uint32_t rest = mant & 0x1fffu;
  if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

/* bench/q4-matmul.js:196-213: the bench's toHalf (mantissa + 0x1000, so
 * ties round up in magnitude; no NaN case). Used for the bench's scales. */
uint16_t orc_to_half_bench(float value) {
  uint32_t x = f2u(value);
  uint32_t sign = (x >> 16) & 0x8000u;
  int exp = (int)((x >> 23) & 0xffu) - 127 + 15;
  uint32_t mant = x & 0x7fffffu;
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    mant = (mant | 0x800000u) >> (1 - exp);
    return (uint16_t)(sign | ((mant + 0x1000u) >> 13));
  }
  if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
  return (uint16_t)(sign | ((uint32_t)exp << 10) | ((mant + 0x1000u) >> 13));
}

/* src/half.ts:36-53 (halfTable / fromHalf). */
float orc_from_half(uint16_t h) {
  float sign = (h & 0x8000u) ? -1.0f : 1.0f;
  int exp = (h >> 10) & 0x1f;
  int mant = h & 0x3ff;
  if (exp == 0) return sign * (float)mant * 5.9604644775390625e-8f; /* 2^-24 */
  if (exp == 31) return mant ? NAN : sign * INFINITY;
  return sign * (1.0f + (float)mant / 1024.0f) * ldexpf(1.0f, exp - 15);
}

/* Round a float through fp16 and back (packH2's clamp to +-65504 first,
 * src/gpu/kernels.ts:32-36). */
static float round_h2(float v) {
  if (v > 65504.0f) v = 65504.0f;
  if (v < -65504.0f) v = -65504.0f;
  return orc_from_half(orc_to_half(v));
}

/* src/repack.ts:21-24 (newQuantMatrix's shape checks). */
int orc_check_shape(int N, int K) {
  if (N <= 0 || K <= 0) return ORC_INVALID_SHAPE;
  if (N % 4 != 0) return ORC_INVALID_SHAPE;
  if (K % 32 != 0) return ORC_INVALID_SHAPE;
  return ORC_OK;
}

/*
 * src/repack.ts:60-87: `rows` rows of llama.cpp Q4_0 blocks (18 bytes: fp16
 * scale, 16 nibble bytes) into the QuantMatrix at row0. src_rows (nullable)
 * names the source row of each destination row.
 */
int orc_pack_q4_0(int N, int K, uint32_t *quants, uint16_t *scales, int row0,
                  const uint8_t *src, size_t src_len, int rows,
                  const int32_t *src_rows) {
  int st = orc_check_shape(N, K);
  if (st) return st;
  if (row0 < 0 || rows < 0 || row0 + rows > N) return ORC_OUT_OF_RANGE;
  size_t blocks = (size_t)K / 32;
  if (src_len < (size_t)rows * blocks * 18) return ORC_DATA_TOO_SHORT;
  for (int i = 0; i < rows; i++) {
    int n = row0 + i;
    size_t p = (size_t)(src_rows ? src_rows[i] : i) * blocks * 18;
    size_t si = (size_t)(n >> 2) * blocks * 4 + (size_t)(n & 3);
    size_t qi = si * 4;
    for (size_t b = 0; b < blocks; b++, p += 18, si += 4, qi += 16) {
      scales[si] = (uint16_t)(src[p] | (src[p + 1] << 8));
      for (int w = 0; w < 4; w++) {
        const uint8_t *s = src + p + 2 + 4 * w;
        quants[qi + w] = (uint32_t)s[0] | ((uint32_t)s[1] << 8) |
                         ((uint32_t)s[2] << 16) | ((uint32_t)s[3] << 24);
      }
    }
  }
  return ORC_OK;
}

/*
 * src/repack.ts:342-392: onnxruntime MatMulNBits rows (element 2i of a
 * block in byte i's low nibble, 2i+1 in its high one; fp16 scale bytes;
 * zero points two blocks a byte, low nibble first) into the QuantMatrix.
 * `zeros` may be NULL only when `zp` is NULL.
 */
int orc_pack_matmulnbits(int N, int K, uint32_t *quants, uint16_t *scales,
                         uint8_t *zeros, int row0, const uint8_t *quant,
                         size_t quant_len, const uint8_t *scale_bytes,
                         size_t scale_len, const uint8_t *zp, size_t zp_len,
                         int rows, const int32_t *src_rows) {
  int st = orc_check_shape(N, K);
  if (st) return st;
  if (row0 < 0 || rows < 0 || row0 + rows > N) return ORC_OUT_OF_RANGE;
  size_t blocks = (size_t)K / 32;
  size_t zp_stride = (blocks + 1) / 2;
  if (quant_len < (size_t)rows * blocks * 16 || scale_len < (size_t)rows * blocks * 2)
    return ORC_DATA_TOO_SHORT;
  if (zp && !zeros) return ORC_INVALID_ARGUMENT;
  if (zp && zp_len < (size_t)rows * zp_stride) return ORC_DATA_TOO_SHORT;
  uint8_t *q = (uint8_t *)quants;
  for (int i = 0; i < rows; i++) {
    int n = row0 + i;
    size_t s = (size_t)(src_rows ? src_rows[i] : i);
    size_t p = s * blocks * 16, sp = s * blocks * 2, zr = s * zp_stride;
    size_t si = (size_t)(n >> 2) * blocks * 4 + (size_t)(n & 3);
    size_t qi = si * 16;
    for (size_t b = 0; b < blocks; b++, p += 16, sp += 2, si += 4, qi += 64) {
      for (int k = 0; k < 8; k++) {
        uint8_t lo = quant[p + k], hi = quant[p + 8 + k];
        q[qi + 2 * k] = (uint8_t)((lo & 0x0f) | ((hi & 0x0f) << 4));
        q[qi + 2 * k + 1] = (uint8_t)((lo >> 4) | (hi & 0xf0));
      }
      scales[si] = (uint16_t)(scale_bytes[sp] | (scale_bytes[sp + 1] << 8));
      if (zp && zeros) zeros[si] = (uint8_t)((zp[zr + (b >> 1)] >> ((b & 1) << 2)) & 15);
    }
  }
  return ORC_OK;
}

/* src/repack.ts:216-242: raw MatMulNBits quants to QuantMatrix words, the
 * word-at-a-time form (4 nibble pairs per step). */
void orc_quants_from_raw(const uint8_t *raw, int N, int K, uint32_t *out) {
  size_t blocks = (size_t)K / 32;
  for (int n = 0; n < N; n++) {
    size_t s = (size_t)n * blocks * 4;
    size_t o = ((size_t)(n >> 2) * blocks * 4 + (size_t)(n & 3)) * 4;
    for (size_t b = 0; b < blocks; b++, s += 4, o += 16) {
      for (int h = 0; h < 2; h++) {
        uint32_t lo, hi;
        memcpy(&lo, raw + 4 * (s + h), 4);
        memcpy(&hi, raw + 4 * (s + 2 + h), 4);
        uint32_t even = (lo & 0x0f0f0f0fu) | ((hi & 0x0f0f0f0fu) << 4);
        uint32_t odd = ((lo >> 4) & 0x0f0f0f0fu) | (hi & 0xf0f0f0f0u);
        uint32_t e0 = even & 0xffffu, o0 = odd & 0xffffu;
        uint32_t e1 = even >> 16, o1 = odd >> 16;
        out[o + 2 * h] = ((e0 | (e0 << 8)) & 0x00ff00ffu) |
                         (((o0 | (o0 << 8)) & 0x00ff00ffu) << 8);
        out[o + 2 * h + 1] = ((e1 | (e1 << 8)) & 0x00ff00ffu) |
                             (((o1 | (o1 << 8)) & 0x00ff00ffu) << 8);
      }
    }
  }
}

/* src/repack.ts:865-891: row n of a 4-bit QuantMatrix as floats,
 * scale * (q - zero), zero 8 when zeros is NULL. */
void orc_matrix_row(int N, int K, const uint32_t *quants, const uint16_t *scales,
                    const uint8_t *zeros, int n, float *out) {
  (void)N;
  size_t blocks = (size_t)K / 32;
  const uint8_t *q = (const uint8_t *)quants;
  for (size_t b = 0; b < blocks; b++) {
    size_t si = (size_t)(n >> 2) * blocks * 4 + (size_t)(n & 3) + 4 * b;
    float scale = orc_from_half(scales[si]);
    float zero = zeros ? (float)zeros[si] : 8.0f;
    for (int j = 0; j < 32; j++) {
      size_t at = (si - 4 * b) * 16 + b * 64 + (size_t)(j < 16 ? j : j - 16);
      int nib = j < 16 ? (q[at] & 15) : (q[at] >> 4);
      out[b * 32 + (size_t)j] = scale * ((float)nib - zero);
    }
  }
}

/*
 * bench/gpu-bench-worker.js:41-55: out[m * N + n] = sum_k W[n][k] * act[m][k]
 * in doubles, straight from GGUF Q4_0 blocks (weight j = d * ((q & 15) - 8),
 * weight j + 16 = d * ((q >> 4) - 8)), in the reference's summation order.
 */
void orc_q4_ref_f64(const uint8_t *blocks, const float *act, int M, int N, int K,
                    double *out, int threads) {
  int kb = K / 32;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
  for (int n = 0; n < N; n++) {
    for (int m = 0; m < M; m++) {
      double sum = 0.0;
      for (int b = 0; b < kb; b++) {
        size_t src = ((size_t)n * kb + b) * 18;
        double d = (double)orc_from_half((uint16_t)(blocks[src] | (blocks[src + 1] << 8)));
        for (int j = 0; j < 16; j++) {
          int q = blocks[src + 2 + j];
          size_t k = (size_t)b * 32 + j;
          sum += d * (double)((q & 15) - 8) * (double)act[(size_t)m * K + k];
          sum += d * (double)((q >> 4) - 8) * (double)act[(size_t)m * K + k + 16];
        }
      }
      out[(size_t)m * N + n] = sum;
    }
  }
}

/* src/engine.ts:5316-5327: K-slices of a split (few-row) matmul. */
void orc_split_slices(int N, int K, int *kb_slice, int *slices) {
  double groups = (double)(N / 4), blocks = (double)(K / 32);
  const double max_split = 16.0, split_fragments = 4096.0; /* engine.ts:295,299 */
  double split = ceil(split_fragments / groups);
  if (max_split < split) split = max_split;
  if (blocks / 4.0 < split) split = blocks / 4.0;
  if (split < 1.0) split = 1.0;
  int kbs = (int)ceil(blocks / split);
  *kb_slice = kbs;
  *slices = (int)ceil(blocks / (double)kbs);
}

/* src/engine.ts:4957-4967 (quadSlices with `most` = quadMaxSplit = 4). */
void orc_quad_slices(int N, int K, int *kb_slice, int *slices) {
  int groups = N / 4, blocks = K / 32;
  double slice_k = 512.0 * (groups > 2048 ? 2.0 : 1.0); /* TUNING.quadSliceK */
  double parts = round((double)K / slice_k);
  if (parts > 4.0) parts = 4.0;
  if (parts < 1.0) parts = 1.0;
  int kbs = (int)ceil((double)blocks / parts);
  *kb_slice = kbs;
  *slices = (int)ceil((double)blocks / (double)kbs);
}

/*
 * The decode (split) matmul as the shader computes it, for a QuantMatrix and
 * M rows of activations: activations rounded to halves (the h2 tensor), per
 * block fp32 sa = sum a and b_r = sum q * a, acc_r += d_r * (b_r - z_r * sa)
 * (kernels.ts:182-217, 744-895), each K-slice's sums stored as a half
 * (RGBA16F partials), the slices added in fp32 by the consumer.
 */
void orc_q4_split_emulate(int N, int K, const uint32_t *quants,
                          const uint16_t *scales, const uint8_t *zeros,
                          const float *act, int M, float *out, int threads) {
  int blocks = K / 32, kb_slice, slices;
  orc_split_slices(N, K, &kb_slice, &slices);
  float *a16 = (float *)malloc(sizeof(float) * (size_t)M * K);
  for (size_t i = 0; i < (size_t)M * K; i++) a16[i] = round_h2(act[i]);
  const uint8_t *q = (const uint8_t *)quants;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
  for (int g = 0; g < N / 4; g++) {
    for (int m = 0; m < M; m++) {
      const float *a = a16 + (size_t)m * K;
      float total[4] = {0, 0, 0, 0};
      for (int s = 0; s < slices; s++) {
        int kb0 = s * kb_slice, kb1 = kb0 + kb_slice < blocks ? kb0 + kb_slice : blocks;
        float acc[4] = {0, 0, 0, 0};
        for (int kb = kb0; kb < kb1; kb++) {
          const float *ab = a + (size_t)kb * 32;
          float sa = 0.0f;
          for (int j = 0; j < 32; j++) sa += ab[j];
          for (int r = 0; r < 4; r++) {
            size_t si = ((size_t)g * blocks + kb) * 4 + r;
            const uint8_t *qb = q + si * 16;
            float b = 0.0f;
            for (int w = 0; w < 4; w++) {
              float lo = 0.0f, hi = 0.0f;
              for (int i = 0; i < 4; i++) {
                uint8_t byte = qb[4 * w + i];
                lo += (float)(byte & 15) * ab[4 * w + i];
                hi += (float)(byte >> 4) * ab[16 + 4 * w + i];
              }
              b += lo + hi;
            }
            float d = orc_from_half(scales[si]);
            float z = zeros ? (float)zeros[si] : 8.0f;
            acc[r] += d * (b - z * sa);
          }
        }
        for (int r = 0; r < 4; r++) total[r] += round_h2(acc[r]);
      }
      for (int r = 0; r < 4; r++) out[(size_t)m * N + 4 * g + r] = total[r];
    }
  }
  free(a16);
}

/*
 * The prompt matmul's f16 route: weights dequantized to halves,
 * (q - z) * d rounded (kernels.ts:436-597), activations as halves, fp32 dot
 * products over each K-slice (kernels.ts:620-735), each slice's result
 * stored as a half (packH2), slices added in fp32 by the consumer (pfq).
 */
void orc_q4_prefill_emulate(int N, int K, const uint32_t *quants,
                            const uint16_t *scales, const uint8_t *zeros,
                            const float *act, int M, float *out, int threads) {
  int kb_slice, slices;
  orc_quad_slices(N, K, &kb_slice, &slices);
  float *a16 = (float *)malloc(sizeof(float) * (size_t)M * K);
  for (size_t i = 0; i < (size_t)M * K; i++) a16[i] = round_h2(act[i]);
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel
#endif
  {
    float *w16 = (float *)malloc(sizeof(float) * (size_t)K);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
    for (int n = 0; n < N; n++) {
      orc_matrix_row(N, K, quants, scales, zeros, n, w16);
      for (int k = 0; k < K; k++) w16[k] = orc_from_half(orc_to_half(w16[k]));
      for (int m = 0; m < M; m++) {
        const float *a = a16 + (size_t)m * K;
        float total = 0.0f;
        for (int s = 0; s < slices; s++) {
          int k0 = s * kb_slice * 32, k1 = (s + 1) * kb_slice * 32;
          if (k1 > K) k1 = K;
          float acc = 0.0f;
          for (int k = k0; k < k1; k++) acc += w16[k] * a[k];
          total += round_h2(acc);
        }
        out[(size_t)m * N + n] = total;
      }
    }
    free(w16);
  }
  free(a16);
}

/*
 * Q4_0 quantisation of float rows, the llama.cpp rule restated from the
 * format: per block of 32, the element of largest magnitude max gives
 * d = max / -8, q = clamp(round(w / d) + 8, 0, 15) (round half away from
 * zero), scale stored as fp16 (round to nearest even). Output: GGUF blocks.
 * Used to make random-init model weights; not a reference function.
 */
void orc_quantize_q4_0(const float *w, int N, int K, uint8_t *blocks_out) {
  int kb = K / 32;
  for (int n = 0; n < N; n++) {
    for (int b = 0; b < kb; b++) {
      const float *x = w + (size_t)n * K + (size_t)b * 32;
      float amax = 0.0f, max = 0.0f;
      for (int j = 0; j < 32; j++) {
        if (fabsf(x[j]) > amax) { amax = fabsf(x[j]); max = x[j]; }
      }
      float d = max / -8.0f;
      float id = d != 0.0f ? 1.0f / d : 0.0f;
      uint8_t *o = blocks_out + ((size_t)n * kb + b) * 18;
      uint16_t h = orc_to_half(d);
      o[0] = (uint8_t)(h & 255);
      o[1] = (uint8_t)(h >> 8);
      for (int j = 0; j < 16; j++) {
        float x0 = x[j] * id, x1 = x[j + 16] * id;
        int q0 = (int)(x0 + 8.5f), q1 = (int)(x1 + 8.5f);
        if (q0 > 15) q0 = 15;
        if (q1 > 15) q1 = 15;
        if (q0 < 0) q0 = 0;
        if (q1 < 0) q1 = 0;
        o[2 + j] = (uint8_t)(q0 | (q1 << 4));
      }
    }
  }
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
