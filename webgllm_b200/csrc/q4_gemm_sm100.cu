// The Q4 prefill GEMM on Blackwell tensor cores: y = x . W^T for many rows.
//
// Replaces the reference's prompt matmuls (src/engine.ts:4969-5234:
// matmulQuad, src/gpu/kernels.ts:370-429; the f16 route dequantRgba4 /
// dequantBytes + matmulF16, kernels.ts:436-735), whose weights are first
// dequantised to an fp16 scratch texture (`(q - z) * d` rounded to half,
// kernels.ts:467, :562) and then multiplied with fp32 sums. Here the
// dequantisation is fused: the fp16 weights never leave the SM.
//
// One CTA computes a 128-row (weights) x BM-row (tokens, 64 / 128 / 256)
// tile over a range of K, in stages of 64 K:
//   warp 0     TMA producer: the x tile (tensor map, 128-byte swizzle, the
//              MMA's B operand) and the stage's 8 code tiles, scales and
//              zero points (3-D tensor maps over the tiled planes) into a
//              shared-memory ring;
//   warps 2-9  dequantisers: codes -> fp16 (q - z) * d with the scale rounded
//              in as the reference's f16 route does, written straight into
//              tensor memory with tcgen05.st.16x256b, whose thread layout is
//              the tile layout's (q4_layout.cuh): the MMA's A operand lives in
//              TMEM, so dequantised weights cost no shared-memory bandwidth;
//   warp 1     one thread issues tcgen05.mma (kind::f16, A from TMEM, B from
//              shared memory, fp32 accumulator in TMEM) and commits each
//              stage back to the ring;
//   warps 2-9  epilogue: tcgen05.ld of the accumulator, stored as y. When
//              K is split across CTAs for parallelism (few token rows), the
//              splits of a tile form one thread-block cluster: each stages
//              its fp32 tile in its own shared memory and CTA r sums slice r
//              of the tile over the cluster's CTAs in rank order through
//              distributed shared memory (deterministic, no atomics, no
//              workspace, no second kernel).
// Launched with programmatic dependent launch: barriers, tensor memory and
// the first stages' weight copies are set up before the kernel waits for
// the one that produced x (griddepcontrol.wait), so in a chain of matmuls
// they overlap the previous kernel's tail.
// Every wait is bounded (mbar_wait_bounded) and TMEM is freed on every path.
#include <cuda.h>

#include <cstdlib>

#include "common.cuh"
#include "device_utils.cuh"
#include "q4_kernels.cuh"
#include "tma.cuh"

namespace wg {

namespace {

constexpr int kStages = 4;         // tensor-memory A stages (dequantised weights)
constexpr int kMaxSplits = 8;  // K splits of a tile: one portable thread-block cluster
// Shared-memory stages (x + codes) per tile height: at BM = 64 a split's
// whole K range (8 tiles) is in flight at once within the two-CTAs-an-SM
// budget; larger tiles keep 4 (measured at M = 1024: 5 stages 45.5 us, 4
// stages 42.4 us).
// (BM = 256, one CTA an SM, measured the same or 1-3 % slower with 6 smem
// stages and an 8-stage A ring: the waits are not latency.)
__host__ __device__ constexpr int smem_stages(int BM) { return BM <= 64 ? 8 : 4; }
// K tiles (of 64) a pipeline stage carries: two at BM = 256, so that each
// round of barrier waits (x landed, A dequantised) feeds eight N = 256 MMAs
// instead of four; the rings keep their bytes (half as many stages).
__host__ __device__ constexpr int stage_ktiles(int BM) { return BM == 256 ? 2 : 1; }
constexpr int kBN = 128;          // weight rows per CTA = MMA M
constexpr int kDequantWarps = 8;  // warps 2..9
constexpr int kGemmThreads = (2 + kDequantWarps) * 32;
constexpr int kXStageBytes(int BM) { return BM * 128; }
constexpr int kNibStageBytes = 8 * kTileNibBytes;  // 4096
constexpr int kSclStageBytes = 8 * kTileSclBytes;  // 512
constexpr int kZroStageBytes = 8 * kTileZroBytes;  // 256
// TMEM: the fp32 accumulator at columns [0, BM), the A ring (4 stages x 32
// columns) after it. BM <= 128: 256 columns a CTA, two CTAs an SM; BM = 256:
// all 512 columns, one CTA an SM.
__host__ __device__ constexpr int tmem_a_col(int BM) { return BM <= 128 ? 128 : 256; }
__host__ __device__ constexpr int tmem_cols(int BM) { return BM <= 128 ? 256 : 512; }
// The launch asks for at least this much shared memory so that no more CTAs
// share an SM than its 512 TMEM columns hold (a surplus CTA would wait in
// tcgen05.alloc).
__host__ __device__ constexpr int min_smem(int BM) { return BM <= 128 ? 100 * 1024 : 120 * 1024; }

struct GemmSmem {
  int x, nib, scl, zro, bar, tmem_slot, total;
};

__host__ __device__ inline GemmSmem gemm_smem(int BM) {
  GemmSmem s;
  const int S = smem_stages(BM);  // K tiles of ring (stage_ktiles(BM) a stage)
  s.x = 0;  // 1024-aligned (SW128 atoms)
  s.nib = s.x + S * kXStageBytes(BM);
  s.scl = s.nib + S * kNibStageBytes;
  s.zro = s.scl + S * kSclStageBytes;
  s.bar = s.zro + S * kZroStageBytes;
  // wfull[S] (weights), xfull[S] (x), sempty[S], afull[T], tempty[T], accfull
  s.tmem_slot = s.bar + (3 * S + 2 * kStages + 1) * 8;
  s.total = s.tmem_slot + 16;
  return s;
}


// ---- tcgen05 / TMA wrappers ------------------------------------------------

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st_16x256b_x4(uint32_t taddr, const uint32_t v[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, float v[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// Shared-memory descriptor of a K-major operand tile in the canonical
// 128-byte-swizzled layout (8-row atoms of 128-byte rows, 1024 bytes apart).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) /* LBO (unused) */ |
         ((uint64_t)(1024 >> 4) << 32) /* SBO */ | ((uint64_t)1 << 46) /* version */ |
         ((uint64_t)2 << 61) /* SWIZZLE_128B */;
}

// Instruction descriptor: kind::f16, A and B fp16, K-major, fp32 accumulator,
// M = 128, N = BM.
__host__ __device__ constexpr uint32_t idesc_f16(int BM) {
  return (1u << 4) | ((uint32_t)(BM >> 3) << 17) | ((uint32_t)(kBN >> 4) << 24);
}

__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float4 ld_cluster_f32x4(uint32_t caddr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(caddr)
               : "memory");
  return v;
}

template <int BM, bool ZEROS>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_nib,
                const __grid_constant__ CUtensorMap tm_scl, const __grid_constant__ CUtensorMap tm_zro,
                const GemmArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte-swizzled tiles (the launch adds
  // 1024 bytes of slack).
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const GemmSmem L = gemm_smem(BM);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // weights and x of a stage complete separately: the dequantisers start on
  // prefetched weights while x is still waiting for its producer. A stage
  // carries P K tiles (S stages, T tensor-memory A stages: the rings keep
  // their bytes).
  constexpr int P = stage_ktiles(BM);
  constexpr int S = smem_stages(BM) / P, T = kStages / P;
  constexpr int XS = P * kXStageBytes(BM), NS = P * kNibStageBytes, SS = P * kSclStageBytes, ZS = P * kZroStageBytes;
  uint64_t *wfull = reinterpret_cast<uint64_t *>(smem + L.bar);
  uint64_t *xfull = wfull + S;
  uint64_t *sempty = xfull + S;  // shared-memory stage free (the MMA that read it is done)
  uint64_t *afull = sempty + S;  // tensor-memory A stage written
  uint64_t *tempty = afull + T;  // tensor-memory A stage free
  uint64_t *accfull = tempty + T;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.tmem_slot);
  __shared__ int aborted;
  __shared__ unsigned long long ts[6];  // wg_trace timestamps
  if (a.trace && threadIdx.x == 0) ts[0] = globaltimer();

  const int nt0 = blockIdx.x * (kBN / kTileRows);  // first 16-row tile
  const int m0 = blockIdx.y * BM;
  const int kpc = a.kt_per_split;  // K tiles per split
  const int kt_begin = blockIdx.z * kpc;
  const int kt_end = min(a.KT, kt_begin + kpc);
  // stages of this split (P tiles each; kt_per_split is a multiple of P, so
  // a stage's tiles past kt_end are past K: the copies read zeros there)
  const int nk = (kt_end - kt_begin + P - 1) / P;

  if (threadIdx.x == 0) {
    aborted = 0;
    for (int i = 0; i < S; i++) {
      mbar_init(&wfull[i], 1);
      mbar_init(&xfull[i], 1);
      mbar_init(&sempty[i], 1);
    }
    for (int i = 0; i < T; i++) {
      mbar_init(&afull[i], kDequantWarps);
      mbar_init(&tempty[i], 1);
    }
    mbar_init(accfull, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, tmem_cols(BM));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_d = tmem;               // accumulator columns [0, BM)
  const uint32_t tmem_a = tmem + tmem_a_col(BM);   // A stage s at columns + 32 s

  auto wait = [&](uint64_t *bar, uint32_t parity) {
    if (aborted) return;
    if (!mbar_wait_bounded(bar, parity, a.flags)) aborted = 1;
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t wbytes = NS + SS + (ZEROS ? ZS : 0);
      const uint32_t xbytes = XS;
      auto load_w = [&](int it) {
        const int s = it % S;
        mbar_expect_tx(&wfull[s], wbytes);
#pragma unroll
        for (int p = 0; p < P; p++) {
          const int kt = kt_begin + it * P + p;
          tma_load_3d(smem + L.nib + s * NS + p * kNibStageBytes, &tm_nib, 0, kt, nt0, &wfull[s]);
          tma_load_3d(smem + L.scl + s * SS + p * kSclStageBytes, &tm_scl, 0, kt, nt0, &wfull[s]);
          if (ZEROS) tma_load_3d(smem + L.zro + s * ZS + p * kZroStageBytes, &tm_zro, 0, kt, nt0, &wfull[s]);
        }
      };
      auto load_x = [&](int it) {
        const int s = it % S;
        mbar_expect_tx(&xfull[s], xbytes);
#pragma unroll
        for (int p = 0; p < P; p++)
          tma_load_2d(smem + L.x + s * XS + p * kXStageBytes(BM), &tm_x, (kt_begin + it * P + p) * kTileK, m0,
                      &xfull[s]);
      };
      // The first stages' weights depend on no earlier kernel: copied (and
      // dequantised) before the dependency wait; x, the previous kernel's
      // output, after it.
      const int pre = nk < S ? nk : S;
      for (int it = 0; it < pre; it++) load_w(it);
      if (a.trace) ts[1] = globaltimer();
      pdl_wait();
      if (a.trace) ts[2] = globaltimer();
      for (int it = 0; it < pre; it++) load_x(it);
      for (int it = pre; it < nk; it++) {
        wait(&sempty[it % S], ((it / S) & 1) ^ 1);
        load_w(it);
        load_x(it);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BM);
      for (int it = 0; it < nk; it++) {
        const int s = it % S, t = it % T;
        wait(&xfull[s], (it / S) & 1);
        if (a.trace && it == 0) ts[3] = globaltimer();
        wait(&afull[t], (it / T) & 1);
        tc_fence_after();
#pragma unroll
        for (int p = 0; p < P; p++) {
          const uint64_t bdesc = sw128_desc(smem_u32(smem + L.x + s * XS + p * kXStageBytes(BM)));
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            mma_f16_tmem_a(tmem_d, tmem_a + (t * P + p) * 32 + kk * 8, bdesc + 2 * kk, idesc,
                           (it > 0 || p > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&sempty[s]);  // x and codes of stage s read (the dequantisers finished before afull)
        tc_commit(&tempty[t]);
      }
      tc_commit(accfull);
    }
  } else {
    // Dequantisers: warp w handles tile 2q + sub of each stage (16 rows),
    // q = w % 4 its TMEM lane quarter.
    const int q = warp & 3;
    const int sub = (warp - 2) >> 2;
    const int tile = 2 * q + sub;
    const int g = lane >> 2;
    for (int it = 0; it < nk; it++) {
      const int s = it % S, t = it % T;
      wait(&wfull[s], (it / S) & 1);
      wait(&tempty[t], ((it / T) & 1) ^ 1);  // the MMA that last read A stage t is done
      tc_fence_after();
#pragma unroll
      for (int p = 0; p < P; p++) {
        const uint4 wv = *reinterpret_cast<const uint4 *>(smem + L.nib + s * NS + p * kNibStageBytes +
                                                          tile * kTileNibBytes + lane * 16);
        const uint2 sv = *reinterpret_cast<const uint2 *>(smem + L.scl + s * SS + p * kSclStageBytes +
                                                          tile * kTileSclBytes + g * 8);
        uint32_t zv = 0x08080808u;
        if (ZEROS)
          zv = *reinterpret_cast<const uint32_t *>(smem + L.zro + s * ZS + p * kZroStageBytes +
                                                   tile * kTileZroBytes + g * 4);
        const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t v[16];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int bsel = j >> 1;
          const uint32_t zz = zv >> (16 * bsel);
          const uint32_t z_g = zz & 15u, z_g8 = (zz >> 8) & 15u;
          uint32_t pc[4];
          unpack_codes(w[j], zp_lo(z_g), zp_hi(z_g), zp_lo(z_g8), zp_hi(z_g8), pc);
          const uint32_t sp = bsel ? sv.y : sv.x;  // (d_g, d_g8)
          const uint32_t d_g = (sp & 0xFFFFu) * 0x00010001u;
          const uint32_t d_g8 = (sp >> 16) * 0x00010001u;
          // (q - z) * d rounded to fp16, as the reference's dequant pass.
          v[4 * j + 0] = hmul2_u(pc[0], d_g);
          v[4 * j + 1] = hmul2_u(pc[1], d_g);
          v[4 * j + 2] = hmul2_u(pc[2], d_g8);
          v[4 * j + 3] = hmul2_u(pc[3], d_g8);
        }
        tmem_st_16x256b_x4(tmem_a + ((uint32_t)(32 * q + 16 * sub) << 16) + (t * P + p) * 32, v);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[t]);
    }

    // Epilogue: this warp's 32 TMEM lanes (weight rows 32q..32q+31) and half
    // of the token columns: into y, or (K split over the cluster) into this
    // CTA's staging tile red[token][128 rows] over the idle ring.
    wait(accfull, 0);
    if (a.trace && warp == 2 && lane == 0) ts[4] = globaltimer();
    tc_fence_after();
    pdl_wait();  // y may still be read by an earlier kernel until it completes
    const int n = nt0 * kTileRows + 32 * q + lane;
    const int c_begin = sub * (BM / 2), c_end = c_begin + BM / 2;
    float *red = reinterpret_cast<float *>(smem + L.x);
    for (int c = c_begin; c < c_end; c += 16) {
      float v[16];
      tmem_ld_32x32b_x16(tmem_d + ((uint32_t)(32 * q) << 16) + c, v);
      if (a.splits > 1) {
#pragma unroll
        for (int i = 0; i < 16; i++) red[(c + i) * kBN + 32 * q + lane] = v[i];
      } else if (n < a.N) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int tok = m0 + c + i;
          if (tok < a.M) store_out(a.y, a.y_dtype, (size_t)tok * a.N + n, v[i]);
        }
      }
    }
  }
  pdl_wait();  // every thread that stores y below (the cluster reduction) has waited
  pdl_trigger();

  if (a.splits > 1) {
    // The cluster's CTAs are the K splits of this tile: CTA r sums elements
    // [r E / C, (r+1) E / C) of the E = BM x 128 tile over ranks 0..C-1 (a
    // fixed order) and stores them. Every thread of every CTA passes both
    // cluster barriers on every path (a CTA that skipped one would stall
    // its peers).
    cluster_sync_all();  // every split's tile is staged
    const int C = a.splits;
    uint32_t crank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
    const int E4 = BM * kBN / 4;  // float4 entries: 4 consecutive weight rows of a token
    const int e0 = (int)((long long)E4 * crank / C), e1 = (int)((long long)E4 * (crank + 1) / C);
    uint32_t peer[kMaxSplits];
#pragma unroll
    for (int r = 0; r < kMaxSplits; r++) peer[r] = r < C ? map_rank(smem_u32(smem + L.x), (uint32_t)r) : 0u;
    for (int e = e0 + (int)threadIdx.x; e < e1; e += kGemmThreads) {
      // every rank's partial in flight at once, then summed in rank order
      // (interleaving each load with its add serialised C round trips of
      // distributed shared memory)
      float4 v[kMaxSplits];
#pragma unroll
      for (int r = 0; r < kMaxSplits; r++)
        if (r < C) v[r] = ld_cluster_f32x4(peer[r] + (uint32_t)e * 16u);
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int r = 0; r < kMaxSplits; r++)
        if (r < C) {
          acc.x += v[r].x;
          acc.y += v[r].y;
          acc.z += v[r].z;
          acc.w += v[r].w;
        }
      const int tok = m0 + (4 * e) / kBN, nn = nt0 * kTileRows + (4 * e) % kBN;
      if (tok < a.M && nn < a.N) {  // N % 4 == 0: all four rows or none
        const size_t o = (size_t)tok * a.N + nn;
        store_out(a.y, a.y_dtype, o, acc.x);
        store_out(a.y, a.y_dtype, o + 1, acc.y);
        store_out(a.y, a.y_dtype, o + 2, acc.z);
        store_out(a.y, a.y_dtype, o + 3, acc.w);
      }
    }
    cluster_sync_all();  // no CTA leaves while a peer still reads its tile
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols(BM));
  }
  if (a.trace && threadIdx.x == 0) {
    ts[5] = globaltimer();
    trace_record(a.trace, a.trace_next, a.trace_cap, ts, a.launch_index,
                 (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x);
  }
  // No TMA may still be writing this CTA's shared memory when it exits (only
  // possible after a timed-out wait): wait for the last round of each stage.
  if (threadIdx.x == 0 && aborted) {
    for (int it = nk > S ? nk - S : 0; it < nk; it++) {
      mbar_wait_bounded(&wfull[it % S], (it / S) & 1, a.flags);
      mbar_wait_bounded(&xfull[it % S], (it / S) & 1, a.flags);
    }
  }
}

// ---- the 2-SM GEMM (cta_group::2) -----------------------------------------
//
// A cluster of two CTAs computes a 256-row (weights) x BM2-row (tokens) tile
// with tcgen05.mma.cta_group::2 (MMA M = 256): each CTA dequantises its own
// 128 weight rows into its own tensor memory (the A operand's two halves)
// and loads half of the token tile (the B operand's two halves) into its own
// shared memory; the leader CTA (rank 0) issues the MMAs, which read A and B
// from both SMs and accumulate each CTA's 128 rows of D in that CTA's tensor
// memory. Per SM, the activation tile in shared memory is half of the 1-SM
// kernel's for the same tensor work — the operand whose TMA writes and MMA
// reads bound that kernel.
//
// Rings: shared-memory stages (x half + code tiles), kStages2 deep, and a
// TMEM A ring of kTmemStages2 stages, decoupled so that loads run further
// ahead than the dequantised weights. Barriers: wfull (each CTA: its code
// tiles), xfull (leader: both x halves, two arrive.expect_tx), afull
// (leader: both CTAs' dequantisers), sempty / tempty / accfull (each CTA,
// arrived by the leader's commits multicast to the pair). Loads that signal
// the leader's barrier from the peer use the .cta_group::2 form (no
// multicast). Every wait is bounded; TMEM (256 columns, one CTA per SM) is
// freed on every path.

constexpr int kStages2 = 8;
constexpr int kTmemStages2 = 12;
constexpr int kBM2 = 128;                        // tokens per CTA pair (MMA N)
constexpr int kX2StageBytes = (kBM2 / 2) * 128;  // this CTA's half: 64 tokens x 64 K fp16
constexpr int kTmemCols2 = 512;                  // D [0, 128), A ring [128, 512)
constexpr int kMinSmem2 = 130 * 1024;            // one CTA per SM

struct Gemm2Smem {
  int x, nib, scl, zro, bar, tmem_slot, total;
};

__host__ __device__ inline Gemm2Smem gemm2_smem() {
  Gemm2Smem s;
  s.x = 0;
  s.nib = s.x + kStages2 * kX2StageBytes;
  s.scl = s.nib + kStages2 * kNibStageBytes;
  s.zro = s.scl + kStages2 * kSclStageBytes;
  s.bar = s.zro + kStages2 * kZroStageBytes;
  // wfull[S], xfull[S], sempty[S], afull[T], tempty[T], pfull[T], accfull
  s.tmem_slot = s.bar + (3 * kStages2 + 3 * kTmemStages2 + 1) * 8;
  s.total = s.tmem_slot + 16;
  return s;
}


// arrive on an mbarrier given by its shared::cluster address
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// Relaxed: no memory ordering of its own (the caller orders what it must).
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// Waits (bounded) with cluster-scope acquire: the phase may have been
// completed by the peer CTA's arrivals.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, unsigned *flags) {
  const long long t0 = clock64();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > 2000000000LL) {
      raise_flag(flags, kFlagTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, int c0, int c1,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc2(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Arrives on `bar` (same shared-memory offset) in both CTAs of the pair once
// the leader's MMAs issued so far are complete.
__device__ __forceinline__ void tc_commit_pair(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((unsigned short)3)
      : "memory");
}

__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}


template <bool ZEROS>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_nib,
                 const __grid_constant__ CUtensorMap tm_scl, const __grid_constant__ CUtensorMap tm_zro,
                 const GemmArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const Gemm2Smem L = gemm2_smem();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t *wfull = reinterpret_cast<uint64_t *>(smem + L.bar);
  uint64_t *xfull = wfull + kStages2;
  uint64_t *sempty = xfull + kStages2;
  uint64_t *afull = sempty + kStages2;
  uint64_t *tempty = afull + kTmemStages2;
  uint64_t *pfull = tempty + kTmemStages2;  // peer only: its dequantisers, before forwarding
  uint64_t *accfull = pfull + kTmemStages2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.tmem_slot);
  __shared__ int aborted;

  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int pair = blockIdx.x >> 1;
  const int nt0 = pair * 16 + (int)rank * 8;  // this CTA's eight 16-row tiles
  const int m0 = blockIdx.y * kBM2;            // the pair's tokens; this CTA loads half
  const int kpc = a.kt_per_split;
  const int kt_begin = blockIdx.z * kpc;
  const int kt_end = min(a.KT, kt_begin + kpc);
  const int nk = kt_end - kt_begin;

  if (threadIdx.x == 0) {
    aborted = 0;
    for (int i = 0; i < kStages2; i++) {
      mbar_init(&wfull[i], 1);
      mbar_init(&xfull[i], 1);   // the leader expects both CTAs' x halves
      mbar_init(&sempty[i], 1);
    }
    for (int i = 0; i < kTmemStages2; i++) {
      mbar_init(&afull[i], kDequantWarps + 1);  // the leader's dequant warps + the peer's forward
      mbar_init(&tempty[i], 1);
      mbar_init(&pfull[i], kDequantWarps);
    }
    mbar_init(accfull, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc2(tmem_slot, kTmemCols2);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_d = tmem;
  const uint32_t tmem_a = tmem + 128;

  auto wait = [&](uint64_t *bar, uint32_t parity) {
    if (aborted) return;
    if (!mbar_wait_cluster(bar, parity, a.flags)) aborted = 1;
  };

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t wbytes = kNibStageBytes + kSclStageBytes + (ZEROS ? kZroStageBytes : 0);
      const uint32_t xfull_leader = map_rank(smem_u32(xfull), 0);
      for (int it = 0; it < nk; it++) {
        const int s = it % kStages2;
        const uint32_t ph = (it / kStages2) & 1;
        wait(&sempty[s], ph ^ 1);
        const int kt = kt_begin + it;
        mbar_expect_tx(&wfull[s], wbytes);
        tma_load_3d(smem + L.nib + s * kNibStageBytes, &tm_nib, 0, kt, nt0, &wfull[s]);
        tma_load_3d(smem + L.scl + s * kSclStageBytes, &tm_scl, 0, kt, nt0, &wfull[s]);
        if (ZEROS) tma_load_3d(smem + L.zro + s * kZroStageBytes, &tm_zro, 0, kt, nt0, &wfull[s]);
        const uint32_t xbar = xfull_leader + (uint32_t)(s * 8);
        // the leader expects both halves (the peer's load may complete first:
        // the transaction count dips below zero, the phase cannot complete
        // before the leader's arrive)
        if (rank == 0) mbar_expect_tx(&xfull[s], 2 * kX2StageBytes);
        tma_load_2d_pair(smem + L.x + s * kX2StageBytes, &tm_x, kt * kTileK, m0 + (int)rank * (kBM2 / 2), xbar);
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = (1u << 4) | ((uint32_t)(kBM2 >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
      for (int it = 0; it < nk; it++) {
        const int s = it % kStages2, t = it % kTmemStages2;
        wait(&xfull[s], (it / kStages2) & 1);
        wait(&afull[t], (it / kTmemStages2) & 1);
        tc_fence_after();
        const uint64_t bdesc = sw128_desc(smem_u32(smem + L.x + s * kX2StageBytes));
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
          mma_f16_pair(tmem_d, tmem_a + t * 32 + kk * 8, bdesc + 2 * kk, idesc, (it > 0 || kk > 0) ? 1u : 0u);
        tc_commit_pair(&sempty[s]);
        tc_commit_pair(&tempty[t]);
      }
      tc_commit_pair(accfull);
    } else if (rank == 1 && lane == 0) {
      // Forward each A stage of this CTA to the leader: one cluster-scope
      // release per stage, off the dequantisers' path.
      const uint32_t afull_leader = map_rank(smem_u32(afull), 0);
      for (int it = 0; it < nk; it++) {
        const int t = it % kTmemStages2;
        wait(&pfull[t], (it / kTmemStages2) & 1);
        if (a.fwd_relaxed)
          mbar_arrive_remote_relaxed(afull_leader + (uint32_t)(t * 8));
        else
          mbar_arrive_remote(afull_leader + (uint32_t)(t * 8));
      }
    }
  } else {
    const int q = warp & 3;
    const int sub = (warp - 2) >> 2;
    const int tile = 2 * q + sub;
    const int g = lane >> 2;
    for (int it = 0; it < nk; it++) {
      const int s = it % kStages2, t = it % kTmemStages2;
      wait(&wfull[s], (it / kStages2) & 1);
      wait(&tempty[t], ((it / kTmemStages2) & 1) ^ 1);  // the MMA that last read A stage t is done
      tc_fence_after();
      const uint4 wv = *reinterpret_cast<const uint4 *>(smem + L.nib + s * kNibStageBytes + tile * kTileNibBytes +
                                                        lane * 16);
      const uint2 sv =
          *reinterpret_cast<const uint2 *>(smem + L.scl + s * kSclStageBytes + tile * kTileSclBytes + g * 8);
      uint32_t zv = 0x08080808u;
      if (ZEROS)
        zv = *reinterpret_cast<const uint32_t *>(smem + L.zro + s * kZroStageBytes + tile * kTileZroBytes + g * 4);
      const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t v[16];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int bsel = j >> 1;
        const uint32_t zz = zv >> (16 * bsel);
        const uint32_t z_g = zz & 15u, z_g8 = (zz >> 8) & 15u;
        uint32_t P[4];
        unpack_codes(w[j], zp_lo(z_g), zp_hi(z_g), zp_lo(z_g8), zp_hi(z_g8), P);
        const uint32_t sp = bsel ? sv.y : sv.x;
        const uint32_t d_g = (sp & 0xFFFFu) * 0x00010001u;
        const uint32_t d_g8 = (sp >> 16) * 0x00010001u;
        v[4 * j + 0] = hmul2_u(P[0], d_g);
        v[4 * j + 1] = hmul2_u(P[1], d_g);
        v[4 * j + 2] = hmul2_u(P[2], d_g8);
        v[4 * j + 3] = hmul2_u(P[3], d_g8);
      }
      tmem_st_16x256b_x4(tmem_a + ((uint32_t)(32 * q + 16 * sub) << 16) + t * 32, v);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(rank == 0 ? &afull[t] : &pfull[t]);
    }

    // Epilogue: this CTA's 128 rows of D (its weight rows) x the pair's tokens.
    // (Waited for even after a timeout: TMEM must not be freed under MMAs.)
    mbar_wait_cluster(accfull, 0, a.flags);
    tc_fence_after();
    const int n = nt0 * kTileRows + 32 * q + lane;
    const int c_begin = sub * (kBM2 / 2), c_end = c_begin + kBM2 / 2;
    for (int c = c_begin; c < c_end; c += 16) {
      float v[16];
      tmem_ld_32x32b_x16(tmem_d + ((uint32_t)(32 * q) << 16) + c, v);
      if (n < a.N) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int tok = m0 + c + i;
          if (tok < a.M) {
            store_out(a.y, a.y_dtype, (size_t)tok * a.N + n, v[i]);
          }
        }
      }
    }
  }

  // No TMA may still be writing when the pair exits (only possible after a
  // timed-out wait): each CTA waits for its own code tiles, the leader for
  // both x halves (they complete on its barrier).
  if (threadIdx.x == 0 && aborted) {
    for (int it = nk > kStages2 ? nk - kStages2 : 0; it < nk; it++) {
      mbar_wait_cluster(&wfull[it % kStages2], (it / kStages2) & 1, a.flags);
      if (rank == 0) mbar_wait_cluster(&xfull[it % kStages2], (it / kStages2) & 1, a.flags);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs (which use both SMs) are done; neither CTA exits early
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem, kTmemCols2);
  }
}

// ---- host side -------------------------------------------------------------

bool encode_x(CUtensorMap *m, const void *x, int M, int K, int BM) {
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)BM};
  cuuint32_t elem[2] = {1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(x), dims, strides, box, elem,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A tiled plane (q4_layout.cuh) as a 3-D u32 tensor [NT][KT][words].
bool encode_plane(CUtensorMap *m, const void *base, int words, int KT, int NT) {
  cuuint64_t dims[3] = {(cuuint64_t)words, (cuuint64_t)KT, (cuuint64_t)NT};
  cuuint64_t strides[2] = {(cuuint64_t)words * 4, (cuuint64_t)words * 4 * KT};
  cuuint32_t box[3] = {(cuuint32_t)words, 1, 8};
  cuuint32_t elem[3] = {1, 1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void *>(base), dims, strides, box, elem,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BM, bool ZEROS>
cudaError_t launch_bm(const GemmArgs &a, const void *x, cudaStream_t stream, bool pdl) {
  const GemmSmem L = gemm_smem(BM);
  auto kern = gemm_kernel<BM, ZEROS>;
  static_assert(BM <= tmem_a_col(BM) && tmem_a_col(BM) + kStages * 32 <= tmem_cols(BM), "TMEM columns");
  static_assert(BM * kBN * 4 <= smem_stages(BM) * kXStageBytes(BM), "the split-K staging tile fits the x ring");
  const int smem_bytes = L.total + 1024 > min_smem(BM) ? L.total + 1024 : min_smem(BM);
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  CUtensorMap tx, tn, ts, tz;
  if (!encode_x(&tx, x, a.M, a.K, BM) || !encode_plane(&tn, a.nib, kTileNibBytes / 4, a.KT, a.NT) ||
      !encode_plane(&ts, a.scl, kTileSclBytes / 4, a.KT, a.NT))
    return cudaErrorInvalidValue;
  tz = ts;
  if (ZEROS && !encode_plane(&tz, a.zro, kTileZroBytes / 4, a.KT, a.NT)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.NT + 7) / 8), (unsigned)((a.M + BM - 1) / BM), (unsigned)a.splits);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = (size_t)smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute at[2];
  int n = 0;
  if (a.splits > 1) {  // the K splits of a tile form one cluster
    at[n].id = cudaLaunchAttributeClusterDimension;
    at[n].val.clusterDim.x = 1;
    at[n].val.clusterDim.y = 1;
    at[n].val.clusterDim.z = (unsigned)a.splits;
    n++;
  }
  if (pdl) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, tx, tn, ts, tz, a);
}

template <bool ZEROS>
cudaError_t launch_pair(const GemmArgs &a, const void *x, cudaStream_t stream) {
  const Gemm2Smem L = gemm2_smem();
  auto kern = gemm2_kernel<ZEROS>;
  const int smem_bytes = L.total + 1024 > kMinSmem2 ? L.total + 1024 : kMinSmem2;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  CUtensorMap tx, tn, ts, tz;
  if (!encode_x(&tx, x, a.M, a.K, kBM2 / 2) || !encode_plane(&tn, a.nib, kTileNibBytes / 4, a.KT, a.NT) ||
      !encode_plane(&ts, a.scl, kTileSclBytes / 4, a.KT, a.NT))
    return cudaErrorInvalidValue;
  tz = ts;
  if (ZEROS && !encode_plane(&tz, a.zro, kTileZroBytes / 4, a.KT, a.NT)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * ((a.NT + 15) / 16)), (unsigned)((a.M + kBM2 - 1) / kBM2), (unsigned)a.splits);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = (size_t)smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tx, tn, ts, tz, a);
}

}  // namespace

bool gemm_supported() { return encode_fn() != nullptr; }

// The 2-SM kernel runs only when asked (WG_GEMM_PAIR=1, N % 256 == 0): on
// B200 it measured 300 TFLOP/s (490 with relaxed forwarding) against the
// 1-SM kernel's 900-1000 at M = 4096 — the per-stage hand-offs between the
// two SMs (a cluster-scope release per 64-K stage) serialise the pipeline.
static bool gemm_use_pair(const GemmArgs &a) {
  static int forced = -2;
  if (forced == -2) {
    const char *e = getenv("WG_GEMM_PAIR");
    forced = e ? atoi(e) : 0;
  }
  return forced == 1 && a.N % 256 == 0 && a.M >= 2;
}

// Token rows per CTA; WG_GEMM_BM (64 / 128 / 256) overrides (tuning).
static int gemm_tile_m(int M) {
  static int forced = -1;
  if (forced < 0) {
    const char *e = getenv("WG_GEMM_BM");
    forced = e ? atoi(e) : 0;
    if (forced != 64 && forced != 128 && forced != 256) forced = 0;
  }
  if (forced) return forced;
  // Measured at 4096 x 4096 (8-launch CUDA graph): M = 128: 14.9 us at BM =
  // 128, 17.0 at 256; M = 256: 18.1 / 17.4; M = 1024: 45.0 / 40.5; M = 4096:
  // 161 / 156. A BM = 256 tile issues MMAs of N = 256: the single issuing
  // thread spends ~80-100 cycles an MMA whatever its N, so N = 128 MMAs
  // (75 cycles of tensor work each) leave the tensor pipe waiting on issue.
  return M <= 64 ? 64 : M <= 128 ? 128 : 256;
}

size_t plan_gemm(GemmArgs &a, int num_sms) {
  const bool pair = gemm_use_pair(a);
  const int BM = pair ? kBM2 : gemm_tile_m(a.M);
  // CTAs of one K range (the pair kernel runs one per SM, the 1-SM kernel two)
  const int tiles = pair ? 2 * ((a.NT + 15) / 16) * ((a.M + BM - 1) / BM)
                         : ((a.NT + 7) / 8) * ((a.M + BM - 1) / BM);
  // Split K while the grid stays one wave: two CTAs an SM where a CTA holds
  // 256 TMEM columns (BM <= 128; the shared-memory padding allows two), one
  // where it holds all 512 (BM = 256), keeping >= 4 stages per split.
  // Measured at 4096 x 4096: M = 64, 17 us with 9 splits vs 19 with 4-5;
  // M = 256, 26 us with 4 splits vs 31 with 2. WG_GEMM_SPLITS overrides
  // (tuning).
  const int per_sm = pair || tmem_cols(BM) == 512 ? 1 : 2;
  static int force = -1;
  if (force < 0) {
    const char *e = getenv("WG_GEMM_SPLITS");
    force = e ? atoi(e) : 0;
  }
  // The splits of a tile form one thread-block cluster (at most a portable 8;
  // the 2-SM kernel keeps its workspace and does not split).
  int splits = 1;
  if (!pair)
    while (splits < kMaxSplits && tiles * (splits + 1) <= per_sm * num_sms && a.KT / (splits + 1) >= 4) splits++;
  if (force > 0 && !pair) splits = force < kMaxSplits ? force : kMaxSplits;
  if (splits > a.KT) splits = a.KT;
  a.kt_per_split = (a.KT + splits - 1) / splits;
  // whole stages per split: a stage's tiles past its split would be the
  // next split's
  const int P = pair ? 1 : stage_ktiles(BM);
  a.kt_per_split = (a.kt_per_split + P - 1) / P * P;
  a.splits = (a.KT + a.kt_per_split - 1) / a.kt_per_split;
  return 0;
}

cudaError_t launch_gemm(const GemmArgs &args, const void *x_f16, cudaStream_t stream, bool pdl) {
  if (!encode_fn()) return cudaErrorNotSupported;
  GemmArgs a = args;
  static int relaxed = -1;
  if (relaxed < 0) {
    const char *e = getenv("WG_GEMM_FWD_RELAXED");
    relaxed = e && e[0] == '1' ? 1 : 0;
  }
  a.fwd_relaxed = relaxed;
  if (a.splits < 1 || a.splits > kMaxSplits) return cudaErrorInvalidValue;
  const int BM = gemm_tile_m(a.M);
  const bool z = a.zro != nullptr;
  if (gemm_use_pair(a)) {
    if (a.splits != 1) return cudaErrorInvalidValue;
    return z ? launch_pair<true>(a, x_f16, stream) : launch_pair<false>(a, x_f16, stream);
  }
  if (BM == 64) return z ? launch_bm<64, true>(a, x_f16, stream, pdl) : launch_bm<64, false>(a, x_f16, stream, pdl);
  if (BM == 128)
    return z ? launch_bm<128, true>(a, x_f16, stream, pdl) : launch_bm<128, false>(a, x_f16, stream, pdl);
  return z ? launch_bm<256, true>(a, x_f16, stream, pdl) : launch_bm<256, false>(a, x_f16, stream, pdl);
}

namespace {
__global__ void to_f16_kernel(const void *x, int dtype, uint4 *out, size_t n8) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x)
    out[i] = load_x8_f16(x, dtype, i * 8);
}
}  // namespace

cudaError_t launch_to_f16(const void *x, int dtype, void *out, size_t n, cudaStream_t stream) {
  const size_t n8 = n / 8;
  const size_t blocks = (n8 + 255) / 256 < 4096 ? (n8 + 255) / 256 : 4096;
  to_f16_kernel<<<(unsigned)(blocks ? blocks : 1), 256, 0, stream>>>(x, dtype, reinterpret_cast<uint4 *>(out), n8);
  return cudaGetLastError();
}

}  // namespace wg
