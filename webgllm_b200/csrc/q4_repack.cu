// Subsystem 1 on the device: 4-bit weights from their file layouts into the
// tiled layout of q4_layout.cuh.
//
// The reference repacks on the CPU (packQ4_0, src/repack.ts:60-87;
// packMatMulNBits, src/repack.ts:342-392; the QuantMatrix itself,
// src/weights.ts:5-21) and uploads textures. Here the file bytes are copied
// to the device as they are and one kernel gathers them: each thread owns
// one 32-bit word of a tile (8 codes) and, for lanes 4g, one scale and zero
// entry, so a repack is race-free and rows outside [row0, row0 + rows) keep
// what earlier calls wrote (matrices are filled part by part, as
// load-gguf.ts:245-283 concatenates q|k|v and gate|up).
#include "common.cuh"
#include "q4_layout.cuh"
#include "q4_kernels.cuh"

namespace wg {

namespace {

__device__ __forceinline__ int gguf_code(const uint8_t *src, int blocks, int s, int k) {
  int b = k >> 5, kk = k & 31;
  uint8_t byte = src[((size_t)s * blocks + b) * 18 + 2 + (kk & 15)];
  return kk < 16 ? (byte & 15) : (byte >> 4);
}

__device__ __forceinline__ int nbits_code(const uint8_t *quant, int blocks, int s, int k) {
  int b = k >> 5, kk = k & 31;
  uint8_t byte = quant[((size_t)s * blocks + b) * 16 + (kk >> 1)];
  return (kk & 1) ? (byte >> 4) : (byte & 15);
}

__device__ __forceinline__ int qmat_code(const uint8_t *quants, int blocks, int n, int k) {
  int b = k >> 5, kk = k & 31;
  size_t si = ((size_t)(n >> 2) * blocks + b) * 4 + (n & 3);
  uint8_t byte = quants[si * 16 + (kk & 15)];
  return kk < 16 ? (byte & 15) : (byte >> 4);
}

__global__ void repack_kernel(RepackArgs a) {
  const Q4Dims d = a.d;
  const int blocks = d.K / 32;
  const int nt0 = a.row0 / kTileRows;
  const int nts = (a.row0 + a.rows - 1) / kTileRows - nt0 + 1;
  const size_t total = (size_t)nts * d.KT * 128;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int j = (int)(idx & 3);
    const int lane = (int)((idx >> 2) & 31);
    const size_t tile_rel = idx >> 7;
    const int kt = (int)(tile_rel % d.KT);
    const int nt = nt0 + (int)(tile_rel / d.KT);
    const int g = lane >> 2, t = lane & 3;
    const size_t tile = (size_t)nt * d.KT + kt;
    uint32_t *wp = a.nib + tile * (kTileNibBytes / 4) + lane * 4 + j;
    // Codes of the word's 8 positions (-1: keep the old nibble).
    uint32_t word = 0, keep_mask = 0;
    bool need_old = false;
#pragma unroll
    for (int p = 0; p < 8; p++) {
      int row, kk;
      q4_unplace(lane, j, p, &row, &kk);
      const int n = nt * kTileRows + row;
      const int k = kt * kTileK + kk;
      const int i = n - a.row0;
      int code = -1;
      if (i >= 0 && i < a.rows && k < d.K) {
        const int s = a.src_rows ? a.src_rows[i] : i;
        if (a.kind == kSrcGguf) code = gguf_code(a.src, blocks, s, k);
        else if (a.kind == kSrcNbits) code = nbits_code(a.src, blocks, s, k);
        else code = qmat_code(a.src, blocks, n, k);
      }
      if (code < 0) {
        need_old = true;
        keep_mask |= 0xFu << (4 * p);
      } else {
        word |= (uint32_t)code << (4 * p);
      }
    }
    if (need_old) word |= *wp & keep_mask;
    *wp = word;

    if (t == 0) {
      // Scale / zero entry j of group g: (row g + 8 * (j & 1), block 2kt + (j >> 1)).
      const int hi_row = j & 1, bsel = j >> 1;
      const int n = nt * kTileRows + g + 8 * hi_row;
      const int b = 2 * kt + bsel;
      const int i = n - a.row0;
      if (i >= 0 && i < a.rows && b < blocks) {
        const size_t e = tile * 32 + g * 4 + bsel * 2 + hi_row;
        uint16_t scale;
        int zero = 8;
        if (a.kind == kSrcGguf) {
          const int s = a.src_rows ? a.src_rows[i] : i;
          const uint8_t *p = a.src + ((size_t)s * blocks + b) * 18;
          scale = (uint16_t)(p[0] | (p[1] << 8));
        } else if (a.kind == kSrcNbits) {
          const int s = a.src_rows ? a.src_rows[i] : i;
          const uint8_t *p = a.scale_src + ((size_t)s * blocks + b) * 2;
          scale = (uint16_t)(p[0] | (p[1] << 8));
          if (a.zero_src) {
            const int zstride = (blocks + 1) / 2;
            zero = (a.zero_src[(size_t)s * zstride + (b >> 1)] >> ((b & 1) << 2)) & 15;
          }
        } else {
          const size_t si = ((size_t)(n >> 2) * blocks + b) * 4 + (n & 3);
          scale = ((const uint16_t *)a.scale_src)[si];
          if (a.zero_src) zero = a.zero_src[si];
        }
        a.scl[e] = scale;
        if (a.zro) a.zro[e] = (uint8_t)zero;
      }
    }
  }
}

}  // namespace

cudaError_t launch_repack(const RepackArgs &a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  const int nts = (a.row0 + a.rows - 1) / kTileRows - a.row0 / kTileRows + 1;
  const size_t total = (size_t)nts * a.d.KT * 128;
  const int threads = 256;
  size_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 64) blocks = 148 * 64;
  repack_kernel<<<(unsigned)blocks, threads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace wg
