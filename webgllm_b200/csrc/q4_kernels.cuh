// Kernel entry points of the Q4 library (internal; the C ABI is capi.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "comm.cuh"
#include "q4_layout.cuh"

namespace wg {

// Source layouts the repack kernel reads.
enum SrcKind : int {
  kSrcGguf = 0,   // llama.cpp Q4_0 blocks (src/repack.ts:60-87)
  kSrcNbits = 1,  // onnxruntime MatMulNBits (src/repack.ts:342-392)
  kSrcQmat = 2,   // the reference's QuantMatrix (src/weights.ts:5-21)
};

struct RepackArgs {
  Q4Dims d;
  uint32_t *nib;
  uint16_t *scl;
  uint8_t *zro;               // null for matrices without zero points
  const uint8_t *src;         // codes (and GGUF scales), on the device
  const uint8_t *scale_src;   // Nbits: fp16 scale bytes; Qmat: u16 scales
  const uint8_t *zero_src;    // Nbits: packed zero points; Qmat: u8 zeros
  const int32_t *src_rows;    // nullable, device
  int row0, rows;
  int kind;
};

cudaError_t launch_repack(const RepackArgs &a, cudaStream_t stream);

// The decode GEMV: y[M][N] = x[M][K] . W^T for M <= 32.
// A transform that produces the matmul's fp16 input from other tensors in
// the same launch (the decoder's norm and SwiGLU passes fused into the
// matmul that consumes them).
enum ProKind { kProNone = 0, kProRmsNorm = 1, kProSwiglu = 2 };
struct Prologue {
  int kind;        // ProKind
  const float *a;  // kProRmsNorm: residual [M][K]; kProSwiglu: gate | up [M][2K]
  const float *b;  // kProRmsNorm: added to the residual [M][K], or null
  const float *w;  // kProRmsNorm: norm weight [K]
  float eps;
  float *out;      // kProRmsNorm: receives residual + b [M][K], or null
  // kProRmsNorm: per-16-column-tile sums of squares of a [K/16][M] (written
  // by a kEpiResidual matmul): the row statistics without reading all of a
  // (b and out are null then)
  const float *stats;
};
// Rows of one fused GEMV launch (the prologue needs the whole row per CTA).
constexpr int kProMaxTokens = 8;
// The prologue alone: x fp16 [M][K] (for matmuls that do not fuse it).
cudaError_t launch_prologue(const Prologue &p, int M, int K, void *x_f16, cudaStream_t stream, bool pdl);

struct GemvArgs {
  const uint32_t *nib;
  const uint16_t *scl;
  const uint8_t *zro;  // nullable
  const void *x;
  void *y;
  int M, N, K, NT, KT;
  int x_dtype, y_dtype;
  int kt_per_cta;  // K tiles per CTA (the cluster splits KT)
  int cluster;     // CTAs per cluster along K
  unsigned *flags; // device error flags (kFlagTimeout)
  // Tracing (wg_trace): records of WG_TRACE_WORDS u64, or null.
  unsigned long long *trace;
  unsigned long long *trace_next;  // device counter of records claimed
  unsigned long long trace_cap;    // records that fit
  unsigned launch_index;
  int trigger_at;  // when dependents may launch: 0 entry, 1 x staged, 2 multiplies done
  Prologue pro;    // kProNone: x as given; else x is made from pro (M <= kProMaxTokens)
  int groups;      // wide GEMV: column groups (grid.y)
  int stages;      // wide GEMV: weight ring stages
  int part_cols;   // wide GEMV with a K split: columns reduced across the cluster at a time
  int push_on;     // outputs go to every rank's exchange buffer (comm.cuh), not y
  CommDev push;
  int epi;         // kEpiNone, or kEpiSwigluPairs: y [M][N/2] = silu(rows 16t..16t+7) * rows 16t+8..16t+15,
                   // or kEpiResidual: y fp32 [M][N] += the product, stats [N/16][M] = per-tile sums of squares
  float *stats;    // kEpiResidual
  int wide_groups; // wide GEMV without a K split: two 8-warp groups take alternate columns
  int wide_norm_rows;  // wide GEMV, norm prologue: stage x row by row (WG_WIDE_NORM_ROWS=1, measurement)
};
enum EpiKind { kEpiNone = 0, kEpiSwigluPairs = 1, kEpiResidual = 2 };

constexpr int kGemvMaxTokens = 32;
cudaError_t launch_gemv(const GemvArgs &a, cudaStream_t stream, bool pdl);
// Plans kt_per_cta / cluster for a shape; false if the shape is too large.
bool plan_gemv(GemvArgs &a, int num_sms);
// The wide GEMV (M <= kProMaxTokens): x resident per CTA, tile columns
// streamed through a ring; plans kt_per_cta / cluster / groups / stages.
bool plan_gemv_wide(GemvArgs &a, int num_sms);
cudaError_t launch_gemv_wide(const GemvArgs &a, cudaStream_t stream, bool pdl);

// The prefill GEMM (tcgen05): y[M][N] = x[M][K] . W^T for M > 32, x fp16.
struct GemmArgs {
  const uint32_t *nib;
  const uint16_t *scl;
  const uint8_t *zro;  // nullable
  void *y;
  int M, N, K, NT, KT;
  int y_dtype;
  int splits, kt_per_split;  // K splits of a tile (one thread-block cluster), K tiles each
  unsigned *flags;
  int fwd_relaxed;  // pair kernel: forward A stages with relaxed arrives (measurement knob)
  // Tracing (wg_trace), as GemvArgs: entry, weight copies issued, x's
  // producer released, first x stage landed, last multiply done, exit.
  unsigned long long *trace;
  unsigned long long *trace_next;
  unsigned long long trace_cap;
  unsigned launch_index;
};

bool gemm_supported();
// Chooses the K split (splits, kt_per_split): the splits of a tile reduce on
// chip across a thread-block cluster, so no workspace is needed (returns 0).
size_t plan_gemm(GemmArgs &a, int num_sms);
// pdl: programmatic dependent launch (weights prefetched before the wait
// for x's producer).
cudaError_t launch_gemm(const GemmArgs &a, const void *x_f16, cudaStream_t stream, bool pdl);
// x (f32 / bf16) -> fp16, saturating like packH2; n a multiple of 8.
cudaError_t launch_to_f16(const void *x, int dtype, void *out, size_t n, cudaStream_t stream);

}  // namespace wg
