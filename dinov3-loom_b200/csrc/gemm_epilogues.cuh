// gemm_epilogues.cuh - the fused epilogues of the tcgen05 GEMM (gemm.cu).
//
// Interface of an epilogue type E:
//   static constexpr int  kSmem;       bytes of shared memory for staged per-column vectors
//   static constexpr bool kTmaStore;   the output leaves through per-warp TMA bulk stores
//   void init(uint8_t *smem, int tid, int n)
//       all CTA threads, before the first barrier: stage per-column vectors (bias, LayerScale,
//       gamma, beta, RoPE angles) into shared memory, so the per-row work reads them as
//       shared-memory broadcasts instead of global loads
//   struct Pre; Pre prefetch(int n0, const EpiCtx &ctx)
//       called before the wait for the tile's accumulator: loads that do not depend on the
//       MMAs (the residual row) start here and overlap the wait
//   static constexpr bool kTmaInput;   (optional) prefetch() loads the tile's input blocks by TMA
//       into the warp's staging blocks, one mbarrier per block (ctx.in_bar)
//   template <int COLS> void run(uint32_t taddr, int n0, EpiCtx &ctx, Pre &pre)
//       processes COLS accumulator columns starting at TMEM address `taddr` (this warp's lane
//       quarter) that belong to output columns n0..n0+COLS-1 of output row ctx.row. ctx.row may
//       be >= M on the last M tile: TMEM loads still run, because tcgen05.ld is
//       warp-collective, but global accesses are skipped (TMA stores clip such rows). For a
//       narrow unit (ctx.narrow) taddr and n0 are the unit's start and the epilogue takes its
//       column half's part itself (by ctx.half).
//   Optional traits: kNarrowOk (a BN = 128 epilogue that takes narrow 128 x 64 units),
//       kStagingBufs (TMA-store staging blocks per warp, default 2), kStagingInTiles (stages in
//       the mainloop's tile buffers; one tile per CTA), kEarlyInput (the TMA producer loads the
//       input blocks into the stage buffers the last k-blocks free first), kWarpStaging (bytes
//       of a warp's staging region in the tile buffers).
//
// Output path of kTmaStore epilogues: each warp owns 32 rows (its TMEM lane quarter) and emits
// 32 columns at a time: the 32x32 f16 block goes into one of the warp's two 2 KB shared-memory
// buffers in the 64-byte-swizzled layout (row r holds its 16-byte chunk j at chunk
// j ^ ((r >> 1) & 3), so the 32 row writes of a warp hit every bank group evenly), and lane 0
// sends it to global memory with one cp.async.bulk.tensor store. The per-row scattered stores
// of a row-per-thread epilogue (32 rows touched per warp instruction) are replaced by full-line
// TMA writes that run in the background.
#pragma once

#include "kernels.h"
#include "sm100.cuh"

namespace dv3 {

constexpr int kEpilogueWarps = 8;
constexpr int kEpilogueThreads = 32 * kEpilogueWarps;
constexpr int kStageBlockBytes = 32 * 64;  // 32 rows x 32 f16 columns

struct EpiCtx {
  int row;     // output row of this thread
  int M;       // rows of the GEMM
  int half;    // column half of the tile (0: warps 2-5, 1: warps 6-9)
  int r;       // row within the tile == TMEM lane
  int lane;
  int row0;    // first row of this warp's 32 rows
  uint8_t *smem;       // epilogue's staged vectors
  uint8_t *staging;    // this warp's two staging blocks
  int buf;             // staging block to use next
  int nbuf;            // staging blocks per warp (2: double-buffered; 1: Epi::kStagingBufs)
  bool narrow;         // BM x BN/2 unit: run() gets the whole unit and takes its part by `half`
  int split;           // split-K launches: the K slice (partial slab) of this unit
  const CUtensorMap *out_map;
  const CUtensorMap *ln_map;  // EpiResidLN: the LayerNorm output
  uint64_t *in_bar;    // kTmaInput epilogues: this warp's two input-block mbarriers
  uint32_t iter;       // tiles this warp has processed (input-block barrier parity)
  volatile int *abort_flag;
  bool failed;         // a bounded wait expired inside run()
  uint8_t *blocks[3];  // EpiResidLN: this warp's three 4 KB staging blocks
};

struct NoPre {};

__device__ __forceinline__ float u2f(uint32_t v) { return __uint_as_float(v); }

__device__ __forceinline__ void stage_floats(float *dst, const float *src, int n, int tid,
                                             int nthreads) {
  for (int i = tid; i < n; i += nthreads) dst[i] = __ldg(src + i);
}

// 32 consecutive floats from shared memory at an address common to the warp (broadcast).
__device__ __forceinline__ void lds32(const float *s, float (&v)[32]) {
  const float4 *p = reinterpret_cast<const float4 *>(s);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 q = p[j];
    v[4 * j + 0] = q.x;
    v[4 * j + 1] = q.y;
    v[4 * j + 2] = q.z;
    v[4 * j + 3] = q.w;
  }
}

// 32 consecutive floats from global memory at an address common to the warp (one L1 line pair,
// served to all lanes).
__device__ __forceinline__ void ldg32(const float *s, float (&v)[32]) {
  const float4 *p = reinterpret_cast<const float4 *>(s);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 q = __ldg(p + j);
    v[4 * j + 0] = q.x;
    v[4 * j + 1] = q.y;
    v[4 * j + 2] = q.z;
    v[4 * j + 3] = q.w;
  }
}

__device__ __forceinline__ void ldg_half32(const __half *src, uint4 (&q)[4]) {
  const uint4 *p = reinterpret_cast<const uint4 *>(src);
#pragma unroll
  for (int j = 0; j < 4; ++j) q[j] = p[j];
}

__device__ __forceinline__ void unpack_half32(const uint4 (&q)[4], float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t w[4] = {q[j].x, q[j].y, q[j].z, q[j].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_half2(w[e]);
      v[8 * j + 2 * e] = f.x;
      v[8 * j + 2 * e + 1] = f.y;
    }
  }
}

__device__ __forceinline__ uint4 pack8(const float (&v)[32], int j) {
  return make_uint4(pack_half2(v[8 * j + 0], v[8 * j + 1]), pack_half2(v[8 * j + 2], v[8 * j + 3]),
                    pack_half2(v[8 * j + 4], v[8 * j + 5]), pack_half2(v[8 * j + 6], v[8 * j + 7]));
}

__device__ __forceinline__ void store_half32(__half *dst, const float (&v)[32]) {
  uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
  for (int j = 0; j < 4; ++j) d[j] = pack8(v, j);
}

// The bias of 192 columns (`b`, in shared memory) into 32 TMEM lanes x 192 columns from `taddr`,
// every lane the same row: the start value of a full-row accumulator (Epi::kBiasInTmem).
__device__ __forceinline__ void fill_acc_bias192(uint32_t taddr, const float *b) {
#pragma unroll
  for (int j = 0; j < 6; ++j) {
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 v = reinterpret_cast<const float4 *>(b + 32 * j)[i / 4];
      r[i] = __float_as_uint(v.x);
      r[i + 1] = __float_as_uint(v.y);
      r[i + 2] = __float_as_uint(v.z);
      r[i + 3] = __float_as_uint(v.w);
    }
    tmem_st32(taddr + 32 * j, r);
  }
}

// Emit this warp's 32 rows x 32 columns (f16 of v, one row per lane) at output column `col`
// through a staging block and a TMA store.
__device__ __forceinline__ void tma_emit32(EpiCtx &c, const float (&v)[32], int col) {
  uint8_t *blk = c.staging + c.buf * kStageBlockBytes;
  if (c.lane == 0) {  // the store that last used this block has read it
    if (c.nbuf == 2) bulk_wait_read<1>();
    else bulk_wait_read<0>();
  }
  __syncwarp();
  uint8_t *rowp = blk + c.lane * 64;
  const int sw = (c.lane >> 1) & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4 *>(rowp + ((j ^ sw) << 4)) = pack8(v, j);
  fence_proxy_async_smem();
  __syncwarp();
  if (c.lane == 0) {
    tma_store_2d(c.out_map, blk, col, c.row0);
    bulk_commit();
  }
  c.buf = c.nbuf == 2 ? c.buf ^ 1 : 0;
}

// ---------------------------------------------------------------------------------------------
// Patch embedding: x[(p/196)*201 + 5 + p%196][n] = f16(acc + b[n]). The destination rows are
// not contiguous (5 prefix rows per image interleave), so the rows are written directly.
// ---------------------------------------------------------------------------------------------
struct EpiPatch {
  const float *bias;
  __half *x;
  static constexpr int kSmem = kHidden * 4;
  static constexpr bool kTmaStore = false;
  static constexpr bool kNarrowOk = true;  // a narrow 128 x 64 unit: 32 columns per column half
  using Pre = NoPre;
  __device__ Pre prefetch(int, const EpiCtx &) const { return {}; }
  __device__ void init(uint8_t *smem, int tid, int n) const {
    stage_floats(reinterpret_cast<float *>(smem), bias, kHidden, tid, n);
  }
  template <int COLS>
  __device__ void run(uint32_t taddr, int n0, EpiCtx &c, Pre &pre) const {
    const float *sb = reinterpret_cast<const float *>(c.smem);
    const bool ok = c.row < c.M;
    const int token = (c.row / kPatches) * kTokens + kPrefix + c.row % kPatches;
    const int k0 = c.narrow ? 32 * c.half : 0, k1 = c.narrow ? k0 + 32 : COLS;
#pragma unroll 1
    for (int k = k0; k < k1; k += 32) {
      uint32_t r[32];
      tmem_load32(taddr + k, r);
      float v[32];
      lds32(sb + n0 + k, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += u2f(r[i]);
      if (ok) store_half32(x + static_cast<size_t>(token) * kHidden + n0 + k, v);
    }
  }
};

// ---------------------------------------------------------------------------------------------
// QKV projection with 2D-axial RoPE on the q and k columns of patch rows.
// RoPE angles depend only on (position along one axis, frequency index j < 16): channel c of
// patch p uses row position p/14 when c%32 < 16 and column position p%14 otherwise, frequency
// c%16 (src/weights.rs:127-144). init() copies those 14x16 cos/sin values of each axis out of
// the packed [196][64] table (rows padded to 17 floats so the 32 rows of a warp fall in distinct
// banks); the packed entries for channels c and c+32 are equal. Columns >= 1152 (the zero-filled
// tail of the last 256-wide tile) are neither computed nor stored.
// Folded form (kFold): A is x instead of LN(x) and the kernel's extra K=16 step adds the row's
// -mean s + c / rstd (weights.cpp), so the projection before RoPE is rstd acc.
// ---------------------------------------------------------------------------------------------
template <bool kFold>
struct EpiQkvRopeT {
  const float *bias;  // unused when kFold (the bias is in the weight aux)
  const float *cosv;
  const float *sinv;
  const float2 *rowstat = nullptr;  // kFold: each row's (rstd, -mean rstd)
  static constexpr int kPad = 17;
  static constexpr int kTab = 14 * kPad;                   // floats per (axis, function)
  static constexpr int kRopeBytes = ((4 * kTab * 4 + 15) / 16) * 16;
  static constexpr int kSmem = kRopeBytes + (kFold ? 0 : kQkv * 4);  // + bias
  static constexpr bool kTmaStore = true;
  // One staging block per warp: the 16 KB saved let a fourth 48 KB mainloop stage fit beside
  // the RoPE tables and the bias. Measured no faster: the two 16-column halves of that block
  // used in turn (twice the TMA store instructions delayed the producer's loads), and the
  // second head's accumulator loaded from TMEM during the first head's stores.
  static constexpr int kStagingBufs = 1;
  static constexpr bool kAuxK = kFold;  // one more K=16 step: the aux rows (gemm_kernel)
  struct Pre {
    float a;  // kFold: this row's rstd
  };
  __device__ Pre prefetch(int, const EpiCtx &c) const {
    if constexpr (kFold) {
      if (c.row < c.M) return {__ldg(&rowstat[c.row].x)};
    }
    return {1.f};
  }
  __device__ void init(uint8_t *smem, int tid, int n) const {
    float *t = reinterpret_cast<float *>(smem);
    for (int i = tid; i < 4 * 14 * 16; i += n) {
      const int which = i / 224, pos = (i / 16) % 14, j = i % 16;
      // axis 0 (rows): patch pos*14, channel j; axis 1 (columns): patch pos, channel 16+j
      const int src = (which < 2) ? (pos * 14) * 64 + j : pos * 64 + 16 + j;
      t[which * kTab + pos * kPad + j] = __ldg(((which & 1) ? sinv : cosv) + src);
    }
    if constexpr (!kFold) stage_floats(reinterpret_cast<float *>(smem + kRopeBytes), bias, kQkv, tid, n);
  }
  template <int COLS>
  __device__ void run(uint32_t taddr, int n0, EpiCtx &c, Pre &pre) const {
    static_assert(COLS % 64 == 0, "a thread owns whole heads");
    const int t = c.row % kTokens;
    const bool patch_row = t >= kPrefix;
    const int p = patch_row ? t - kPrefix : 0;
    const float *tab = reinterpret_cast<const float *>(c.smem);
    const float *sb = reinterpret_cast<const float *>(c.smem + kRopeBytes);
    const float *cy = tab + (p / 14) * kPad, *sy = tab + kTab + (p / 14) * kPad;
    const float *cx = tab + 2 * kTab + (p % 14) * kPad, *sx = tab + 3 * kTab + (p % 14) * kPad;
    // a narrow unit (128 columns: two heads) gives each column half one head
    const int h0 = c.narrow ? 64 * c.half : 0, h1 = c.narrow ? h0 + 64 : COLS;
#pragma unroll 1
    for (int h = h0; h < h1; h += 64) {
      const int col = n0 + h;  // first column of this 64-wide head
      if (col >= kQkv) break;  // warp-uniform
      float lo[32], hi[32];
      if constexpr (kFold) {  // the accumulator holds (LN(x) W^T + b) / rstd
        uint32_t ra[32], rb[32];
        tmem_load32x2(taddr + h, ra, taddr + h + 32, rb);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          lo[i] = pre.a * u2f(ra[i]);
          hi[i] = pre.a * u2f(rb[i]);
        }
      } else {
        uint32_t ra[32], rb[32];
        tmem_load32x2(taddr + h, ra, taddr + h + 32, rb);
        lds32(sb + col, lo);
        lds32(sb + col + 32, hi);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          lo[i] += u2f(ra[i]);
          hi[i] += u2f(rb[i]);
        }
      }
      if (patch_row && col < 2 * kHidden) {  // q and k columns of patch tokens rotate
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float cs = i < 16 ? cy[i] : cx[i - 16];
          const float sn = i < 16 ? sy[i] : sx[i - 16];
          const float a = lo[i], b = hi[i];
          lo[i] = a * cs - b * sn;
          hi[i] = b * cs + a * sn;
        }
      }
      tma_emit32(c, lo, col);
      tma_emit32(c, hi, col + 32);
    }
  }
};
using EpiQkvRope = EpiQkvRopeT<false>;
using EpiQkvRopeFold = EpiQkvRopeT<true>;

// ---------------------------------------------------------------------------------------------
// Split-K partial product (kernels/matmul_splitk_f16_wmma.loom): the f32 accumulator of this
// unit's K slice, without the bias, into slab ctx.split of partials [splits][rows][384]. Each warp
// emits 32-row x 32-column f32 blocks (128-byte rows, 128-byte swizzle: row r's 16-byte chunk k
// at chunk k ^ (r & 7)) through two 4 KB staging blocks and TMA stores; the map clips rows past
// the GEMM's rows inside each slab.
// ---------------------------------------------------------------------------------------------
struct EpiPartialF32 {
  static constexpr int kSmem = 0;
  static constexpr bool kTmaStore = true;
  static constexpr int kStagingBufs = 4;  // 4 x 2 KB = two 4 KB f32 blocks per warp
  using Pre = NoPre;
  __device__ Pre prefetch(int, const EpiCtx &) const { return {}; }
  __device__ void init(uint8_t *, int, int) const {}
  template <int COLS>
  __device__ void run(uint32_t taddr, int n0, EpiCtx &c, Pre &) const {
    const int sw = c.lane & 7;
#pragma unroll 1
    for (int j = 0; j < COLS; j += 32) {
      uint32_t r[32];
      tmem_load32(taddr + j, r);
      uint8_t *blk = c.staging + c.buf * 4096;
      if (c.lane == 0) bulk_wait_read<1>();  // the store that last used this block has read it
      __syncwarp();
      uint8_t *rowp = blk + c.lane * 128;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        *reinterpret_cast<uint4 *>(rowp + ((k ^ sw) << 4)) =
            make_uint4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (c.lane == 0) {
        tma_store_3d(c.out_map, blk, n0 + j, c.row0, c.split);
        bulk_commit();
      }
      c.buf ^= 1;
    }
  }
};

// ---------------------------------------------------------------------------------------------
// Residual update with LayerScale: x[row][n] = f16(x + lambda[n] (acc + b[n])), in place. The
// warp's residual block (its 32 rows x 64 columns) arrives by TMA in the warp's two staging
// blocks, requested before the accumulator wait (prefetch). Each thread then rewrites its row of
// a block in shared memory and the block leaves by TMA store, so x is read and written in whole
// lines instead of one 16-byte piece per row and warp instruction.
// ---------------------------------------------------------------------------------------------
struct EpiResid {
  const float *bias;
  const float *lambda;
  static constexpr int kSmem = 2 * kHidden * 4;
  static constexpr bool kTmaStore = true;
  static constexpr bool kTmaInput = true;
  // Narrow 128 x 64 units (small batches): each column half of the epilogue warps takes one
  // 32-column block of the unit; the second input barrier gets a plain arrival, so both barriers
  // complete one phase per unit whatever its width.
  static constexpr bool kNarrowOk = true;
  using Pre = NoPre;
  __device__ Pre prefetch(int n0, const EpiCtx &c) const {
    if (c.lane == 0) {
      bulk_wait_read<0>();  // the previous tile's stores have read both blocks
      if (c.narrow) {
        mbar_arrive_expect_tx(&c.in_bar[0], kStageBlockBytes);
        tma_load_2d(c.staging, c.out_map, &c.in_bar[0], n0 + 32 * c.half, c.row0);
        mbar_arrive(&c.in_bar[1]);
      } else {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          mbar_arrive_expect_tx(&c.in_bar[j], kStageBlockBytes);
          tma_load_2d(c.staging + j * kStageBlockBytes, c.out_map, &c.in_bar[j], n0 + 32 * j,
                      c.row0);
        }
      }
    }
    return {};
  }
  __device__ void init(uint8_t *smem, int tid, int n) const {
    float *s = reinterpret_cast<float *>(smem);
    stage_floats(s, bias, kHidden, tid, n);
    stage_floats(s + kHidden, lambda, kHidden, tid, n);
  }
  template <int COLS>
  __device__ void run(uint32_t taddr, int n0, EpiCtx &c, Pre &) const {
    static_assert(COLS == 64, "one 32-column block per staging buffer");
    const float *sb = reinterpret_cast<const float *>(c.smem);
    const float *sl = sb + kHidden;
    const int sw = (c.lane >> 1) & 3;
    // narrow: the unit's accumulator starts at taddr; this column half's block is block 0 of the
    // staging, at TMEM column 32 * half and output column n0 + 32 * half
    const int blocks = c.narrow ? 1 : 2;
    if (c.narrow) {
      taddr += 32 * c.half;
      n0 += 32 * c.half;
    }
#pragma unroll 1
    for (int j = 0; j < blocks; ++j) {
      uint32_t r[32];
      tmem_ld32(taddr + 32 * j, r);
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&c.in_bar[j], c.iter & 1u, c.abort_flag));
      tmem_wait_ld(r);
      if (!ok) {
        c.failed = true;
        return;
      }
      uint8_t *rowp = c.staging + j * kStageBlockBytes + c.lane * 64;
      uint4 q[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) q[k] = *reinterpret_cast<const uint4 *>(rowp + ((k ^ sw) << 4));
      float v[32], b[32], l[32];
      unpack_half32(q, v);
      lds32(sb + n0 + 32 * j, b);
      lds32(sl + n0 + 32 * j, l);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += l[i] * (u2f(r[i]) + b[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) *reinterpret_cast<uint4 *>(rowp + ((k ^ sw) << 4)) = pack8(v, k);
      fence_proxy_async_smem();
      __syncwarp();
      if (c.lane == 0) {
        tma_store_2d(c.out_map, c.staging + j * kStageBlockBytes, n0 + 32 * j, c.row0);
        bulk_commit();
      }
    }
  }
};

// ---------------------------------------------------------------------------------------------
// The same residual update on full 384-wide rows (a 128 x 384 tile per CTA, one tile per CTA).
// Once the tile's accumulator is complete the mainloop's tile buffers are idle: each warp loads
// its residual block (32 rows x 192 columns, six 32-column TMA blocks) into its part of them with
// one mbarrier, rewrites it row by row and stores the six blocks by TMA.
// ---------------------------------------------------------------------------------------------
struct EpiResidWide {
  const float *bias;
  const float *lambda;
  static constexpr int kSmem = 2 * kHidden * 4;
  static constexpr bool kTmaStore = true;
  static constexpr bool kTmaInput = true;
  static constexpr bool kStagingInTiles = true;
  static constexpr int kBlocks = 6;  // 32-column blocks per warp (192 columns)
  static constexpr int kWarpStaging = kBlocks * kStageBlockBytes;
  using Pre = NoPre;
  __device__ Pre prefetch(int, const EpiCtx &) const { return {}; }
  __device__ void init(uint8_t *smem, int tid, int n) const {
    float *s = reinterpret_cast<float *>(smem);
    stage_floats(s, bias, kHidden, tid, n);
    stage_floats(s + kHidden, lambda, kHidden, tid, n);
  }
  template <int COLS>
  __device__ void run(uint32_t taddr, int n0, EpiCtx &c, Pre &) const {
    static_assert(COLS == 32 * kBlocks, "six 32-column blocks per warp");
    if (c.lane == 0) {
      mbar_arrive_expect_tx(&c.in_bar[0], kBlocks * kStageBlockBytes);
#pragma unroll
      for (int j = 0; j < kBlocks; ++j)
        tma_load_2d(c.staging + j * kStageBlockBytes, c.out_map, &c.in_bar[0], n0 + 32 * j, c.row0);
    }
    const float *sb = reinterpret_cast<const float *>(c.smem);
    const float *sl = sb + kHidden;
    const int sw = (c.lane >> 1) & 3;
    if (!__all_sync(0xffffffffu, mbar_wait(&c.in_bar[0], c.iter & 1u, c.abort_flag))) {
      c.failed = true;
      return;
    }
#pragma unroll 1
    for (int j = 0; j < kBlocks; ++j) {
      uint32_t r[32];
      tmem_load32(taddr + 32 * j, r);
      uint8_t *rowp = c.staging + j * kStageBlockBytes + c.lane * 64;
      uint4 q[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) q[k] = *reinterpret_cast<const uint4 *>(rowp + ((k ^ sw) << 4));
      float v[32], b[32], l[32];
      unpack_half32(q, v);
      lds32(sb + n0 + 32 * j, b);
      lds32(sl + n0 + 32 * j, l);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += l[i] * (u2f(r[i]) + b[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) *reinterpret_cast<uint4 *>(rowp + ((k ^ sw) << 4)) = pack8(v, k);
      fence_proxy_async_smem();
      __syncwarp();
      if (c.lane == 0) {
        tma_store_2d(c.out_map, c.staging + j * kStageBlockBytes, n0 + 32 * j, c.row0);
        bulk_commit();
      }
    }
  }
};

// ---------------------------------------------------------------------------------------------
// Gate/up with SwiGLU: the weight rows are packed 64 gate rows, the matching 64 up rows, ...;
// act[row][j] = f16(silu(g + bg) (u + bu)), silu through the hardware tanh (one MUFU op).
// Folded form (kFold): A is x instead of LN(x) and the kernel's extra K=16 step adds the row's
// -mean s + c / rstd (weights.cpp), so g = rstd acc_g and u = rstd acc_u.
// ---------------------------------------------------------------------------------------------
template <bool kFold>
struct EpiSwiGLUT {
  const float *bias;  // packed like the weight rows (unused when kFold: it is in the weight aux)
  const float2 *rowstat = nullptr;  // kFold: each row's (rstd, -mean rstd)
  // The bias is read through L1 (every lane of a warp reads the same 32 floats) rather than staged
  // in shared memory: without it four 48 KB stages fit beside the TMA-store staging (three with).
  static constexpr int kSmem = 0;
  static constexpr bool kTmaStore = true;
  static constexpr bool kAuxK = kFold;  // one more K=16 step: the aux rows (gemm_kernel)
  struct Pre {
    float a;  // kFold: this row's rstd
  };
  __device__ Pre prefetch(int, const EpiCtx &c) const {
    if constexpr (kFold) {
      if (c.row < c.M) return {__ldg(&rowstat[c.row].x)};
    }
    return {1.f};
  }
  __device__ void init(uint8_t *, int, int) const {}
  template <int COLS>
  __device__ void run(uint32_t taddr, int n0, EpiCtx &c, Pre &pre) const {
    static_assert(COLS % 128 == 0, "a thread owns whole 64 gate + 64 up groups");
    const float *sb = bias;
    // a narrow unit is one group: each column half takes 32 of its 64 outputs
    const int g1 = c.narrow ? 128 : COLS;
    const int s0 = c.narrow ? 32 * c.half : 0, s1 = c.narrow ? s0 + 32 : 64;
#pragma unroll 1
    for (int g = 0; g < g1; g += 128) {
#pragma unroll 1
      for (int sub = s0; sub < s1; sub += 32) {
        uint32_t rg[32], ru[32];
        tmem_load32x2(taddr + g + sub, rg, taddr + g + 64 + sub, ru);
        float gv[32];
        if constexpr (kFold) {  // the accumulator holds (LN(x) W^T + b) / rstd
#pragma unroll
          for (int i = 0; i < 32; ++i)
            gv[i] = silu(pre.a * u2f(rg[i])) * (pre.a * u2f(ru[i]));
        } else {
          float uv[32];
          ldg32(sb + n0 + g + sub, gv);
          ldg32(sb + n0 + g + 64 + sub, uv);
#pragma unroll
          for (int i = 0; i < 32; ++i) gv[i] = silu(gv[i] + u2f(rg[i])) * (uv[i] + u2f(ru[i]));
        }
        tma_emit32(c, gv, (n0 + g) / 2 + sub);
      }
    }
  }
};
using EpiSwiGLU = EpiSwiGLUT<false>;
using EpiSwiGLUFold = EpiSwiGLUT<true>;

// ---------------------------------------------------------------------------------------------
// Residual update fused with the following LayerNorm, on full-row tiles (BN = 384, one tile per
// CTA, staged in mainloop buffers that are idle by then):
//   x[row] = f16(x + lambda (acc + b))                        (matmul_resid_f16_wmma.loom)
//   h[row] = f16(LN(x[row]))  or  out[row] = LN(x[row]) f32   (layernorm_rowwave_*.loom)
// Each warp owns 32 rows x 192 columns (its lane quarter, its column half) and a 12 KB staging
// region: three 32-row x 64-column f16 blocks in the 128-byte-swizzled layout of the TMA maps
// (row r at r*128 bytes, its 16-byte chunk k at chunk k ^ (r & 7)). The TMA producer loads the
// x blocks into these regions as soon as the mainloop has finished with the stage buffers that
// hold them (kEarlyInput: the stages of the last-but-two and last-but-one k-blocks), so the load
// overlaps the last MMAs. The updated blocks are written in place and leave by TMA one 64-column
// block at a time; the stored f16 values also go back into TMEM over the accumulator columns
// already consumed (16 packed columns per 32), which is where the LayerNorm reads them, as the
// separate kernel reads x from memory. Statistics: each warp takes the mean and the centred sum
// of squares of its 192 values, and the two warps of a row merge them through shared memory
// (Chan et al.: M2 = M2a + M2b + d^2 n_a n_b / n), eps 1e-5, f32. The normalised blocks reuse
// the staging region once the x stores have read it: three f16 blocks, or (f32 output) two
// rounds of three 32-row x 32-column f32 blocks. With `rowstat` set (GemmOp::ResidStats*, the
// LayerNorm folded into the next GEMM) the epilogue stops after the statistics and leaves
// (rstd, -mean rstd) and the aux row of each row instead of normalising it.
// ---------------------------------------------------------------------------------------------
struct EpiResidLN {
  const float *bias;
  const float *lambda;
  const float *gamma;
  const float *beta;
  bool f32_out;
  // GemmOp::ResidStats*: the LayerNorm is folded into the next GEMM, so instead of normalising
  // the row this epilogue leaves rowstat[row] = (rstd, -mean rstd) and the row's aux row
  // (store_row_aux) in row_aux [rows][16] (gamma and beta unused).
  float2 *rowstat = nullptr;
  __half *row_aux = nullptr;
  static constexpr int kVecs = 4 * kHidden;  // bias, lambda, gamma, beta
  static constexpr int kSmem = kVecs * 4 + 4 * 128 * 4;  // + [mean|M2][2 halves][128 rows]
  static constexpr bool kTmaStore = true;
  static constexpr bool kTmaInput = true;
  static constexpr bool kStagingInTiles = true;
  static constexpr bool kEarlyInput = true;
  static constexpr bool kBiasInTmem = true;  // the accumulator starts at b (gemm_kernel fills it)
  static constexpr int kBlockBytes = 32 * 128;              // 32 rows x 64 f16 columns
  static constexpr int kInBlocks = 3;                       // per warp (192 columns)
  static constexpr int kWarpStaging = kInBlocks * kBlockBytes;
  static constexpr int kSub = 6;                            // 32-column accumulator chunks
  using Pre = NoPre;
  __device__ Pre prefetch(int, const EpiCtx &) const { return {}; }
  __device__ void init(uint8_t *smem, int tid, int n) const {
    float *s = reinterpret_cast<float *>(smem);
    stage_floats(s, bias, kHidden, tid, n);
    stage_floats(s + kHidden, lambda, kHidden, tid, n);
    if (rowstat) return;
    stage_floats(s + 2 * kHidden, gamma, kHidden, tid, n);
    stage_floats(s + 3 * kHidden, beta, kHidden, tid, n);
  }
  // The bias of this warp's 192 columns into its 32 TMEM lanes (every lane the same row).
  __device__ void fill_acc(uint32_t taddr, const uint8_t *smem, int half) const {
    fill_acc_bias192(taddr, reinterpret_cast<const float *>(smem) + half * (kHidden / 2));
  }
  // Eight consecutive floats of a staged vector (a shared-memory broadcast).
  __device__ static void lds8(const float *p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4 *>(p)[0];
    const float4 b = reinterpret_cast<const float4 *>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  template <int COLS>
  __device__ void run(uint32_t taddr, int n0, EpiCtx &c, Pre &) const {
    static_assert(COLS == 32 * kSub, "six 32-column accumulator chunks per warp");
    const float *sv = reinterpret_cast<const float *>(c.smem);
    float *red = const_cast<float *>(sv) + kVecs;  // [0..255] means, [256..511] M2
    const int sw = c.lane & 7;
    // A warp whose accumulator (c.failed on entry) or residual never arrives (the kernel is
    // aborting) skips its work but still meets its partner warp at the barrier below, then
    // reports the failure.
    const bool landed =
        !c.failed && __all_sync(0xffffffffu, mbar_wait(&c.in_bar[0], c.iter & 1u, c.abort_flag));
    // x = f16(x + lambda (acc + b)) in place (the accumulator started at b); back into TMEM as
    // packed f16; out by TMA. Each
    // 32-column chunk's shared-memory loads come before its stores, so they issue together
    // instead of one 16-byte group at a time behind the previous group's store. The mean and the
    // centred sum of squares of this warp's 192 columns build up chunk by chunk from the stored
    // f16 values in registers (two passes within a chunk, chunks merged by Chan's formula).
    float mean = 0.f, m2 = 0.f;
    if (landed) {
      uint32_t ra[32], rb[32];
      tmem_ld32(taddr, ra);
      tmem_wait_ld(ra);
#pragma unroll
      for (int j = 0; j < kSub; ++j) {
        uint32_t(&r)[32] = (j & 1) ? rb : ra;
        uint32_t(&rn)[32] = (j & 1) ? ra : rb;
        if (j + 1 < kSub) tmem_ld32(taddr + 32 * (j + 1), rn);
        uint8_t *rowp = c.blocks[j >> 1] + c.lane * 128;
        uint4 q[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
          q[k] = *reinterpret_cast<const uint4 *>(rowp + ((((j & 1) * 4 + k) ^ sw) << 4));
        uint32_t o[16];
        float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t w[4] = {q[k].x, q[k].y, q[k].z, q[k].w};
          float ll[8];
          lds8(sv + kHidden + n0 + 32 * j + 8 * k, ll);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const float2 t = make_float2(u2f(r[8 * k + 2 * p]), u2f(r[8 * k + 2 * p + 1]));
            const float2 v =
                __ffma2_rn(make_float2(ll[2 * p], ll[2 * p + 1]), t, unpack_half2(w[p]));
            o[4 * k + p] = pack_half2(v.x, v.y);
            s2 = __fadd2_rn(s2, unpack_half2(o[4 * k + p]));
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *reinterpret_cast<uint4 *>(rowp + ((((j & 1) * 4 + k) ^ sw) << 4)) =
              make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
        tmem_st16(taddr + 32 * j, o);
        const float cm = (s2.x + s2.y) * (1.0f / 32);
        const float2 ncm = make_float2(-cm, -cm);
        float2 qa = make_float2(0.f, 0.f), qb = qa;
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float2 d0 = __fadd2_rn(unpack_half2(o[i]), ncm);
          qa = __ffma2_rn(d0, d0, qa);
          const float2 d1 = __fadd2_rn(unpack_half2(o[i + 1]), ncm);
          qb = __ffma2_rn(d1, d1, qb);
        }
        const float cq = (qa.x + qa.y) + (qb.x + qb.y);
        if (j == 0) {
          mean = cm;
          m2 = cq;
        } else {  // j chunks so far (32 j values) merged with 32 more
          const float d = cm - mean;
          mean += d * (1.0f / (j + 1));
          m2 += cq + d * d * (32.0f * j / (j + 1));
        }
        if (j & 1) {  // a 64-column block is complete
          fence_proxy_async_smem();
          __syncwarp();
          if (c.lane == 0) {
            tma_store_2d(c.out_map, c.blocks[j >> 1], n0 + 64 * (j >> 1), c.row0);
            bulk_commit();
          }
        }
        if (j + 1 < kSub) tmem_wait_ld(rn);
      }
      tmem_st_wait();
    }
    // merged with the other half of the row: only the two warps of this lane quarter meet
    red[c.half * 128 + c.r] = mean;
    red[256 + c.half * 128 + c.r] = m2;
    named_barrier(1 + (c.r >> 5), 64);
    if (!landed) {
      c.failed = true;
      return;
    }
    const float m0 = red[c.r], m1 = red[128 + c.r];
    const float d = m1 - m0;
    mean = 0.5f * (m0 + m1);
    m2 = red[256 + c.r] + red[384 + c.r] + d * d * (kHidden / 4);
    const float rstd = rsqrtf(m2 * (1.0f / kHidden) + 1e-5f);
    if (rowstat) {  // folded LayerNorm: the consumer normalises
      if (c.row < c.M) {
        if (c.half == 0) rowstat[c.row] = make_float2(rstd, -mean * rstd);
        else store_row_aux(row_aux + static_cast<size_t>(c.row) * 16, mean, rstd);
      }
      return;
    }
    // h = (x rstd - mean rstd) gamma + beta, staged where the x blocks were. Each output block
    // overwrites a block whose store was committed three groups earlier (an x block, or for f32
    // output the first round of f32 blocks), so waiting until at most two groups are still
    // reading lets it go ahead.
    const float2 nm = make_float2(-mean * rstd, -mean * rstd), rs = make_float2(rstd, rstd);
    uint32_t xa[16], xb[16];
    tmem_ld16(taddr, xa);
    tmem_ld_wait();
    tmem_regs_ready16(xa);
#pragma unroll
    for (int j = 0; j < kSub; ++j) {
      uint32_t(&xr)[16] = (j & 1) ? xb : xa;
      uint32_t(&xn)[16] = (j & 1) ? xa : xb;
      if (j + 1 < kSub) tmem_ld16(taddr + 32 * (j + 1), xn);
      float y[32];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float gg[8], tt[8];
        lds8(sv + 2 * kHidden + n0 + 32 * j + 8 * k, gg);
        lds8(sv + 3 * kHidden + n0 + 32 * j + 8 * k, tt);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float2 z = __ffma2_rn(unpack_half2(xr[4 * k + p]), rs, nm);
          const float2 v = __ffma2_rn(z, make_float2(gg[2 * p], gg[2 * p + 1]),
                                      make_float2(tt[2 * p], tt[2 * p + 1]));
          y[8 * k + 2 * p] = v.x;
          y[8 * k + 2 * p + 1] = v.y;
        }
      }
      if (!f32_out) {
        uint8_t *rowp = c.blocks[j >> 1] + c.lane * 128;
        if (!(j & 1)) {
          if (c.lane == 0) bulk_wait_read<2>();
          __syncwarp();
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *reinterpret_cast<uint4 *>(rowp + ((((j & 1) * 4 + k) ^ sw) << 4)) = pack8(y, k);
        if (j & 1) {
          fence_proxy_async_smem();
          __syncwarp();
          if (c.lane == 0) {
            tma_store_2d(c.ln_map, c.blocks[j >> 1], n0 + 64 * (j >> 1), c.row0);
            bulk_commit();
          }
        }
      } else {
        // f32: 32 columns (128-byte rows, 128-byte swizzle) per block, three blocks at a time
        if (c.lane == 0) bulk_wait_read<2>();
        __syncwarp();
        uint8_t *blk = c.blocks[j % 3];  // three 4 KB f32 blocks at a time
        uint8_t *rowp = blk + c.lane * 128;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<float4 *>(rowp + ((k ^ sw) << 4)) =
              make_float4(y[4 * k], y[4 * k + 1], y[4 * k + 2], y[4 * k + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (c.lane == 0) {
          tma_store_2d(c.ln_map, blk, n0 + 32 * j, c.row0);
          bulk_commit();
        }
      }
      if (j + 1 < kSub) {
        tmem_ld_wait();
        tmem_regs_ready16(xn);
      }
    }
  }
};

}  // namespace dv3
