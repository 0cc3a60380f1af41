// The device layout of a 4-bit matrix (subsystem 1's output, the GEMV's and
// GEMM's input).
//
// The reference keeps a QuantMatrix in row groups of 4 (src/weights.ts:5-21):
// per group and block, 4 rows x 16 bytes, one texel per block row. On the
// B200 the matrix is cut into TILES of 16 rows x 64 K (two 32-weight blocks
// per row): 512 bytes of codes, laid out so that lane L of a warp loads its
// 16 bytes with one vector load and, after an in-register unpack, holds four
// half2 registers per 16-wide K step in the register layout that both
// tensor-core paths want:
//   - tcgen05.st.16x256b (the GEMM writes dequantised weights into tensor
//     memory as the MMA's A operand: thread L -> TMEM lanes L/4 and L/4 + 8,
//     columns 2(L%4) and 2(L%4)+1, a column holding two consecutive K);
//   - mma.m16n8k16's A fragment (the GEMV), with K permuted inside each
//     16-step: fragment k index 2t, 2t+1, 2t+8, 2t+9 <-> K offset 4t .. 4t+3,
//     the same permutation being applied to the activations.
//
//   nib  [NT][KT][32 lanes][4 words]   u32   NT = ceil(N/16), KT = ceil(K/64)
//   scl  [NT][KT][8 g][4]              fp16  (row g, blk 0), (row g+8, blk 0),
//                                            (row g, blk 1), (row g+8, blk 1)
//   zro  [NT][KT][8 g][4]              u8    same order; absent for Q4_0 (8)
//
// A tile's rows are 16*nt + g and 16*nt + g + 8 for g = L / 4. Word j of
// lane L = 4g + t covers K offsets 64*kt + 16*j + 4t + e, e = 0..3, of both
// rows: nibble position p (bits 4p..4p+3) holds
//   p = 0: (row g,   e 0)     p = 4: (row g,   e 1)
//   p = 1: (row g,   e 2)     p = 5: (row g,   e 3)
//   p = 2: (row g+8, e 0)     p = 6: (row g+8, e 1)
//   p = 3: (row g+8, e 2)     p = 7: (row g+8, e 3)
// so that (w & 0x000F000F), (w & 0x00F000F0), ((w >> 8) & 0x000F000F) and
// ((w >> 8) & 0x00F000F0), OR'd into the exponent of 1024.0h, are the half2
// pairs (row g, e 0-1), (row g, e 2-3), (row g+8, e 0-1), (row g+8, e 2-3).
//
// Rows >= N and K >= K are padding: code 8, scale 0 (weight 0).
#pragma once
#include <cstdint>

namespace wg {

constexpr int kTileRows = 16;
constexpr int kTileK = 64;
constexpr int kTileNibBytes = 512;
constexpr int kTileSclBytes = 64;
constexpr int kTileZroBytes = 32;

struct Q4Dims {
  int N, K;    // logical shape (N % 4 == 0, K % 32 == 0)
  int NT, KT;  // tiles
};

__host__ __device__ inline Q4Dims q4_dims(int N, int K) {
  return Q4Dims{N, K, (N + kTileRows - 1) / kTileRows, (K + kTileK - 1) / kTileK};
}

// Where weight (n, k) lives: byte offset of its nibble in `nib`, the nibble
// half (0 low, 1 high), and the index of its scale / zero (in halves / bytes)
// in `scl` / `zro`.
struct Q4Place {
  size_t nib_byte;
  int nib_high;
  size_t sz_index;
};

__host__ __device__ inline Q4Place q4_place(const Q4Dims &d, int n, int k) {
  int nt = n / kTileRows, r = n % kTileRows;
  int g = r & 7, hi_row = r >> 3;
  int kt = k / kTileK, kk = k % kTileK;
  int j = kk >> 4, c = kk & 15;
  int t = c >> 2, e = c & 3;
  int lane = 4 * g + t;
  int p = 2 * hi_row + ((e >> 1) & 1) + 4 * (e & 1);
  size_t tile = (size_t)nt * d.KT + kt;
  Q4Place pl;
  pl.nib_byte = tile * kTileNibBytes + (size_t)lane * 16 + (size_t)j * 4 + (size_t)(p >> 1);
  pl.nib_high = p & 1;
  pl.sz_index = tile * 32 + (size_t)g * 4 + (size_t)(j >> 1) * 2 + (size_t)hi_row;
  return pl;
}

// The inverse for one code of a word: nibble position p of word j of lane
// `lane` in a tile -> (row in tile 0..15, K offset in tile 0..63).
__host__ __device__ inline void q4_unplace(int lane, int j, int p, int *row, int *kk) {
  const int g = lane >> 2, t = lane & 3;
  const int hi_row = (p >> 1) & 1;
  const int e = ((p >> 2) & 1) | ((p & 1) << 1);
  *row = g + 8 * hi_row;
  *kk = 16 * j + 4 * t + e;
}

}  // namespace wg
