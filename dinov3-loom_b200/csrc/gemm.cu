// gemm.cu - persistent, warp-specialised tcgen05 GEMM for the projections of the forward, each
// with its epilogue fused (gemm_epilogues.cuh):
//   Patch     x[token(p)] = f16(A W^T + b)                 kernels/matmul_bias_f16_wmma.loom
//                                                          + kernels/embed_scatter_f32.loom
//   QkvRope   qkv = f16(rope(A W^T + b))                   kernels/matmul_qkv_rope_f16_wmma.loom
//   Resid*    x = f16(x + lambda (A W^T + b))              kernels/matmul_resid_f16_wmma.loom
//   ResidLN*  the same on full rows, then LayerNorm        + kernels/layernorm_rowwave_*.loom
//   SwiGLU    act = f16(silu(A Wg^T + bg) (A Wu^T + bu))   kernels/matmul_swiglu_f16_wmma.loom
//   SplitK    partials[s] = A[:, K_s] W[:, K_s]^T (f32)     kernels/matmul_splitk_f16_wmma.loom
//   PatchPixels  Patch with A built from the f32 images    + the patchify of src/lib.rs:265-280
//                in the mainloop (pixel_a_tiles)
// and down_qkv_kernel: ResidLN1536 followed in the same CTA by the next layer's QkvRope on the
// LayerNorm rows it keeps in shared memory (launch_down_qkv).
//
// Layout: A [M][K] f16 activations and W [N][K] f16 weights, both K-major, are streamed by TMA
// in 128-row x 64-column boxes with the 128-byte swizzle into a ring of shared-memory stages.
// One thread issues tcgen05.mma (M=128, N=BN or BN/2, K=16 steps) into an f32 accumulator in
// TMEM; for BN <= 256 TMEM holds two accumulators so the epilogue of tile i overlaps the MMAs of
// tile i+1.
//
// Warp roles (320 threads): warp 0 lane 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer
// (lane 0), warps 2-9 = epilogue. An epilogue warp may read only TMEM lanes 32*(w%4)..+31, so
// two warps share each lane quarter: warps 2-5 take the left half of the tile's columns and
// warps 6-9 the right half. Each epilogue thread owns one output row and walks its half in
// 32-column chunks (tcgen05.ld 32x32b.x32). Two warps per SM sub-partition hide the latency of
// the epilogue arithmetic, which otherwise limits the whole GEMM.
//
// Units of work (TileSched: full tiles in m-major order with the N tile fastest, so the CTAs
// working at one time share A rows through L2, then narrow half-width units) are dealt
// round-robin to a grid of min(units, SMs) persistent CTAs.
#include <type_traits>

#include "gemm_epilogues.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace dv3 {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kGemmThreads = 64 + kEpilogueThreads;  // 320

// BN <= 256: one MMA of N=BN per K step, two TMEM accumulators (epilogue overlaps MMAs).
// BN  > 256 (full 384-wide rows): two MMAs of N=BN/2 per K step into adjacent TMEM columns, the
// weight tile arrives as two TMA boxes of BN/2 rows, and one accumulator fills TMEM.
// Shared memory: [stages x (A 16 KB | B BN*128 B)] [TMA-store staging: 8 warps x 2 x 2 KB]
// [mbarriers, TMEM slot, abort flag] [epilogue vectors]. As many stages as fit (at most 6).
// Whether an epilogue loads input blocks by TMA (EpiResid): Epi::kTmaInput when it exists.
template <class Epi, class = void>
struct TmaInput {
  static constexpr bool value = false;
};
template <class Epi>
struct TmaInput<Epi, decltype(void(Epi::kTmaInput))> {
  static constexpr bool value = Epi::kTmaInput;
};

// Whether an epilogue stages through the mainloop's tile buffers instead of a region of its own
// (EpiResidWide): Epi::kStagingInTiles when it exists. Such an epilogue runs only when every CTA
// has at most one tile, so the buffers are idle once the tile's accumulator is complete.
template <class Epi, class = void>
struct StagingInTiles {
  static constexpr bool value = false;
};
template <class Epi>
struct StagingInTiles<Epi, decltype(void(Epi::kStagingInTiles))> {
  static constexpr bool value = Epi::kStagingInTiles;
};

// Whether the TMA producer loads the epilogue's input blocks into the stage buffers that the last
// k-blocks free first (EpiResidLN), so that the load overlaps the last MMAs: Epi::kEarlyInput.
template <class Epi, class = void>
struct EarlyInput {
  static constexpr bool value = false;
};
template <class Epi>
struct EarlyInput<Epi, decltype(void(Epi::kEarlyInput))> {
  static constexpr bool value = Epi::kEarlyInput;
};

// TMA-store staging blocks per epilogue warp: Epi::kStagingBufs when it exists, else 2.
template <class Epi, class = void>
struct StagingBufs {
  static constexpr int value = 2;
};
template <class Epi>
struct StagingBufs<Epi, decltype(void(Epi::kStagingBufs))> {
  static constexpr int value = Epi::kStagingBufs;
};

// Whether a BN = 128 epilogue takes narrow BM x 64 units (Epi::kNarrowOk; BN = 256 epilogues all
// do).
template <class Epi, class = void>
struct NarrowOk {
  static constexpr bool value = false;
};
template <class Epi>
struct NarrowOk<Epi, decltype(void(Epi::kNarrowOk))> {
  static constexpr bool value = Epi::kNarrowOk;
};

// Whether the epilogue warps write the bias into the (single) accumulator before the first MMA,
// which then accumulates onto it (Epi::kBiasInTmem, one tile per CTA): the epilogue reads
// acc + b from TMEM. The fill runs while the previous kernel finishes (before the dependency
// wait).
template <class Epi, class = void>
struct BiasInTmem {
  static constexpr bool value = false;
};
template <class Epi>
struct BiasInTmem<Epi, decltype(void(Epi::kBiasInTmem))> {
  static constexpr bool value = Epi::kBiasInTmem;
};

// Whether the epilogue warps build the A tiles from f32 NCHW images (Epi::kAFromPixels, the
// fused patchify of the patch embedding) while the producer loads only the weights. One tile per
// CTA: the epilogue warps are idle during its mainloop.
template <class Epi, class = void>
struct AFromPixels {
  static constexpr bool value = false;
};
template <class Epi>
struct AFromPixels<Epi, decltype(void(Epi::kAFromPixels))> {
  static constexpr bool value = Epi::kAFromPixels;
};

// Bytes of one epilogue warp's staging region in the tile buffers: Epi::kWarpStaging when it
// exists.
template <class Epi, class = void>
struct EpiWarpStaging {
  static constexpr int value = 0;
};
template <class Epi>
struct EpiWarpStaging<Epi, decltype(void(Epi::kWarpStaging))> {
  static constexpr int value = Epi::kWarpStaging;
};

template <int BN, class Epi>
struct GemmCfg {
  static constexpr int kSplit = BN > 256 ? 2 : 1;    // MMAs per K step
  static constexpr int kMmaN = BN / kSplit;
  // BN = 256 (and BN = 128 with a kNarrowOk epilogue): a unit of work may be a narrow BM x BN/2
  // tile (TileSched); the weight tile then arrives as BN/2-row boxes, two per K step for a full
  // tile and one for a narrow one.
  static constexpr bool kNarrow = BN == 256 || (BN == 128 && NarrowOk<Epi>::value);
  static constexpr int kBBox = kNarrow ? BN / 2 : kMmaN;  // rows of one weight box
  static constexpr int kAccBufs = 2 * BN <= 512 ? 2 : 1;
  static constexpr int kA = BM * BK * 2;  // 16 KB
  static constexpr int kB = BN * BK * 2;
  static constexpr int kStage = kA + kB;
  static constexpr bool kInTiles = StagingInTiles<Epi>::value;
  static constexpr int kStaging =
      Epi::kTmaStore && !kInTiles ? kEpilogueWarps * StagingBufs<Epi>::value * kStageBlockBytes : 0;
  static constexpr bool kInput = TmaInput<Epi>::value;
  static constexpr bool kEarly = EarlyInput<Epi>::value;
  static constexpr bool kBiasInit = BiasInTmem<Epi>::value;
  static constexpr bool kAPix = AFromPixels<Epi>::value;
  // configurations whose launches have exactly one tile per CTA
  static constexpr bool kOneTile = kInTiles || kBiasInit || kAPix;
  static_assert(!kBiasInit || BN == 384, "bias fill: one full-row tile per CTA");
  static_assert(!kAPix || (kBiasInit && BN == 384), "pixel A tiles: one full-row tile per CTA");
  // full-barrier arrivals per stage: the producer's (with the TMA bytes), and with kAPix one per
  // epilogue warp once its rows of the A tile are written
  static constexpr int kFullArrivals = kAPix ? 1 + kEpilogueWarps : 1;
  static constexpr int kBarBytes = kInput ? 384 : 256;  // + 2 input-block mbarriers per warp
  static constexpr int kFixed = 1024 + kStaging + kBarBytes + ((Epi::kSmem + 127) / 128) * 128;
  static constexpr int kFit = (227 * 1024 - kFixed) / kStage;
  static constexpr int kStages = kFit < 6 ? kFit : 6;
  static constexpr int kTiles = kStages * kStage;
  static constexpr int kStagingOffset = kTiles;
  static constexpr int kBarOffset = kStagingOffset + kStaging;
  static constexpr int kExtraOffset = kBarOffset + kBarBytes;
  static constexpr int kTmemCols = kAccBufs * BN <= 256 ? 256 : 512;
  // kEarly: epilogue warps whose staging region lies in the first freed stage (the rest go to
  // the second); each warp's region is Epi::kWarpStaging bytes.
  static constexpr int kWarpsPerStage = kEarly ? kStage / EpiWarpStaging<Epi>::value : 0;
  static constexpr int kEarlyA = kWarpsPerStage < kEpilogueWarps ? kWarpsPerStage : kEpilogueWarps;
  static_assert(!kEarly || (kStages >= 3 && kEarlyA > 0 &&
                            (kEpilogueWarps - kEarlyA) * EpiWarpStaging<Epi>::value <= kStage),
                "early epilogue input: two freed stages hold every warp's staging region");
  static constexpr int kSmemBytes = 1024 + kExtraOffset + Epi::kSmem;
  static_assert(kMmaN % 16 == 0 && kMmaN <= 256, "tcgen05.mma N for M=128");
  static_assert((2 * kStages + 2 * kAccBufs + (kInput ? 2 * kEpilogueWarps : 0)) * 8 + 12 <=
                    kBarBytes,
                "barrier region");
  static_assert(kStages >= 2 && kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <int BN, class Epi>
__host__ __device__ constexpr int gemm_smem_bytes() {
  return GemmCfg<BN, Epi>::kSmemBytes;
}

// The units of work of one launch, dealt round-robin to the persistent CTAs (unit u to CTA
// u % grid). Units [0, split_from) are full BM x BN tiles in m-major order with the N tile
// fastest (full_n of them per M tile, so the CTAs working at one time share A rows through L2);
// the rest are narrow BM x BN/2 units (GemmCfg::kNarrow configurations): first the two halves of
// each full tile from split_from on, then, when N leaves half a tile over (N = full_n*BN + BN/2),
// the narrow tile of each M tile at column full_n*BN. Narrow units at the end fill a partial last
// wave with half-length work instead of whole tiles that leave most CTAs idle; at small batches
// every tile runs as two narrow units. Split-K launches repeat the full tiles once per K slice.
struct TileSched {
  int m_tiles;
  int full_n;      // full-width tiles per M tile
  int split_from;  // full tiles processed whole
  int num_units;
  int k_splits;    // split-K: the full tiles repeat for each K slice (slice-major); else 1
  const void *l2_next;    // weights of a later kernel to prefetch into L2 (or null)
  size_t l2_next_bytes;
};

template <int BN>
__device__ __forceinline__ void unit_coords(const TileSched &s, int u, int &m0, int &n0,
                                            bool &narrow, int &k_slice) {
  k_slice = 0;
  if (s.k_splits > 1) {  // split-K launches have full tiles only
    const int per = s.m_tiles * s.full_n;
    k_slice = u / per;
    u -= k_slice * per;
  }
  if (u < s.split_from) {
    m0 = (u / s.full_n) * BM;
    n0 = (u % s.full_n) * BN;
    narrow = false;
    return;
  }
  narrow = true;
  const int v = u - s.split_from;
  const int halves = 2 * (s.m_tiles * s.full_n - s.split_from);
  if (v < halves) {
    const int t = s.split_from + v / 2;
    m0 = (t / s.full_n) * BM;
    n0 = (t % s.full_n) * BN + (v & 1) * (BN / 2);
  } else {
    m0 = (v - halves) * BM;
    n0 = s.full_n * BN;
  }
}

// ---------------------------------------------------------------------------------------------
// The patchify of the patch embedding inside its mainloop (Epi::kAFromPixels). A[p][k] is pixel
// (c, dy, dx) = (k / 256, k / 16 % 16, k % 16) of patch p (src/lib.rs:265-280), so the 64
// columns of k-block kb are channel kb / 4, pixel rows 4 (kb % 4) .. + 3 of the patch, 16 pixels
// each. Lane l of epilogue warp ew takes tile row 16 ew + l / 2 and two of those pixel rows
// (l % 2): 32 floats as eight 16-byte loads, rounded to f16 like patchify and written as four
// 16-byte chunks of the 128-byte-swizzled row (chunk j of row r at j ^ (r % 8)). The loads of
// the next two k-blocks are issued before the wait for a free stage, so three k-blocks of pixel
// reads are in flight per thread (the reads are latency-bound: HBM under the whole grid's load). Rows past `rows` are zeros. Any non-finite pixel sets status[1] bit 0,
// the flag patchify sets. Returns false when a stage never frees (the kernel is aborting).
// ---------------------------------------------------------------------------------------------
template <class C>
__device__ bool pixel_a_tiles(const float *images, int rows, int m0, int ew, int lane,
                              uint8_t *tiles, uint64_t *full, uint64_t *empty, int k_blocks,
                              volatile int *abort_flag, uint32_t *status) {
  const int r = 16 * ew + (lane >> 1);
  const int part = lane & 1;
  const int p = m0 + r;
  const bool valid = p < rows;
  const int img = valid ? p / kPatches : 0, pp = valid ? p % kPatches : 0;
  const float *base = images + static_cast<int64_t>(img) * 3 * kImage * kImage +
                      (pp / 14) * 16 * kImage + (pp % 14) * 16 + 2 * part * kImage;
  auto load = [&](int kb, float4 (&v)[8]) {
    const float4 *src =
        reinterpret_cast<const float4 *>(base + (kb >> 2) * kImage * kImage + (kb & 3) * 4 * kImage);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = valid ? __ldg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[4 + i] = valid ? __ldg(src + kImage / 4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  float4 cur[8], nxt[8], nxt2[8];
  load(0, cur);
  if (k_blocks > 1) load(1, nxt);
  int stage = 0;
  uint32_t phase = 0;
  bool bad = false, ok = true;
  for (int kb = 0; kb < k_blocks; ++kb) {
    if (kb + 2 < k_blocks) load(kb + 2, nxt2);
    if (!__all_sync(0xffffffffu, mbar_wait(&empty[stage], phase ^ 1u, abort_flag))) {
      ok = false;
      break;
    }
    uint8_t *row = tiles + stage * C::kStage + r * 128;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 a = cur[2 * j], b = cur[2 * j + 1];
      bad |= !(isfinite(a.x) && isfinite(a.y) && isfinite(a.z) && isfinite(a.w) &&
               isfinite(b.x) && isfinite(b.y) && isfinite(b.z) && isfinite(b.w));
      *reinterpret_cast<uint4 *>(row + (((4 * part + j) ^ (r & 7)) << 4)) =
          make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y),
                     pack_half2(b.z, b.w));
    }
    fence_proxy_async_smem();  // the MMA reads the tile through the async proxy
    __syncwarp();
    if (lane == 0) mbar_arrive(&full[stage]);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      cur[i] = nxt[i];
      nxt[i] = nxt2[i];
    }
    if (++stage == C::kStages) {
      stage = 0;
      phase ^= 1u;
    }
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0 && status) atomicOr(status + 1, 1u);
  return ok;
}

// ---------------------------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------------------------
template <int BN, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                int M, TileSched sched, int k_blocks, Epi epi, uint32_t *status) {
  using C = GemmCfg<BN, Epi>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t *smem = smem_raw + pad;
  uint8_t *tiles = smem;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::kBarOffset);
  uint64_t *empty = full + C::kStages;
  uint64_t *tfull = empty + C::kStages;
  uint64_t *tempty = tfull + C::kAccBufs;
  uint64_t *in_bars = tempty + C::kAccBufs;  // 2 per epilogue warp (kInput only)
  uint32_t *tmem_slot =
      reinterpret_cast<uint32_t *>(in_bars + (C::kInput ? 2 * kEpilogueWarps : 0));
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile int *in_armed = abort_flag + 1;  // kEarly: epilogue warps whose input the producer armed
  uint8_t *extra = smem + C::kExtraOffset;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], C::kFullArrivals);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < C::kAccBufs; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * kEpilogueWarps);
    }
    if (C::kInput)
      for (int i = 0; i < 2 * kEpilogueWarps; ++i) mbar_init(&in_bars[i], 1);
    *abort_flag = 0;
    *in_armed = 0;
    fence_mbar_init();
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
    if (Epi::kTmaStore) tma_prefetch_map(&tmC);
    if (std::is_same<Epi, EpiResidLN>::value) tma_prefetch_map(&tmD);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  epi.init(extra, threadIdx.x, kGemmThreads);  // weights only: may overlap the previous kernel
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if constexpr (C::kBiasInit) {
    // Each epilogue warp writes the bias into its lane quarter and column half of the
    // accumulator; the MMAs of the CTA's one tile accumulate onto it.
    if (warp >= 2) {
      const int q = warp & 3, half = (warp - 2) >> 2;
      epi.fill_acc(*tmem_slot + (static_cast<uint32_t>(q * 32) << 16) +
                       static_cast<uint32_t>(half * (BN / 2)),
                   extra, half);
      tmem_st_wait();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  pdl_wait();  // activations of the previous kernel are complete from here on
  pdl_trigger();
  // an epilogue thread, idle until the first accumulator, starts the next weights toward L2
  if (threadIdx.x == 64 && sched.l2_next) l2_prefetch_share(sched.l2_next, sched.l2_next_bytes);
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = sched.num_units;
  if (C::kOneTile && num_tiles > static_cast<int>(gridDim.x)) {  // the host never launches this
    if (threadIdx.x == 0) report(status, kErrEpilogueWait);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem_base, C::kTmemCols);
    }
    return;
  }

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, last_parity = 0;  // per stage: loads issued, parity of the last phase
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int m0, n0, k_slice;
        bool narrow;
        unit_coords<BN>(sched, tile, m0, n0, narrow, k_slice);
        if constexpr (!C::kNarrow) narrow = false;
        const int b_boxes = narrow ? 1 : BN / C::kBBox;
        const int kb0 = k_slice * k_blocks;  // split-K: this unit's slice of the k-blocks
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            report(status, kErrProducerWait);
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t *a = tiles + stage * C::kStage;
          mbar_arrive_expect_tx(&full[stage], (C::kAPix ? 0 : C::kA) + b_boxes * C::kBBox * BK * 2);
          if constexpr (!C::kAPix) tma_load_2d(a, &tmA, &full[stage], (kb0 + kb) * BK, m0);
          for (int s = 0; s < b_boxes; ++s)
            tma_load_2d(a + C::kA + s * C::kBBox * BK * 2, &tmB, &full[stage], (kb0 + kb) * BK,
                        n0 + s * C::kBBox);
          armed |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if constexpr (C::kEarly) {
          // The epilogue's x blocks go into the stages of the last-but-two and last-but-one
          // k-blocks (one tile per CTA) once their MMAs have completed: epilogue warps 0..kEarlyA-1
          // into the first, the others into the second (the staging pointers of the epilogue).
          for (int part = 0; ok && part < 2; ++part) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
              report(status, kErrProducerWait);
              *abort_flag = 1;
              ok = false;
              break;
            }
            uint8_t *base = tiles + stage * C::kStage;
            const int w0 = part == 0 ? 0 : C::kEarlyA, w1 = part == 0 ? C::kEarlyA : kEpilogueWarps;
            *in_armed = w1;
            for (int ew = w0; ew < w1; ++ew) {
              uint64_t *bar = &in_bars[2 * ew];
              mbar_arrive_expect_tx(bar, Epi::kWarpStaging);
              const int row0 = m0 + 32 * ((ew + 2) & 3);  // the warp's TMEM lane quarter
              const int col0 = n0 + (ew >> 2) * (BN / 2);  // its column half
              for (int b = 0; b < Epi::kInBlocks; ++b)
                tma_load_2d(base + (ew - w0) * Epi::kWarpStaging + b * Epi::kBlockBytes, &tmC, bar,
                            col0 + 64 * b, row0);
            }
            if (++stage == C::kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      // Copies still in flight (only after an abort) land before shared memory is released.
      for (int st = 0; st < C::kStages; ++st)
        if ((armed >> st) & 1u) mbar_drain(&full[st], (last_parity >> st) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_full = idesc_f16_f32(BM, C::kMmaN, false);
      constexpr uint32_t idesc_narrow = idesc_f16_f32(BM, C::kNarrow ? BN / 2 : C::kMmaN, false);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag)) {
          report(status, kErrMmaWait);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        int m0_unused, n0_unused, k_slice_unused;
        bool narrow;
        unit_coords<BN>(sched, tile, m0_unused, n0_unused, narrow, k_slice_unused);
        const uint32_t idesc = C::kNarrow && narrow ? idesc_narrow : idesc_full;
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            report(status, kErrMmaWait);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + stage * C::kStage);
          const uint64_t adesc = sw128_desc(a_addr);
#pragma unroll
          for (int s = 0; s < C::kSplit; ++s) {
            const uint64_t bdesc = sw128_desc(a_addr + C::kA + s * C::kMmaN * BK * 2);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_f16(d + s * C::kMmaN, adesc + 2 * k, bdesc + 2 * k, idesc,
                       C::kBiasInit || (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == C::kAccBufs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else {
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;       // which half of the tile's columns
    constexpr int kCols = BN / 2;
    const int row_in_tile = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    EpiCtx ctx;
    ctx.M = M;
    ctx.half = half;
    ctx.r = row_in_tile;
    ctx.lane = lane;
    ctx.smem = extra;
    if constexpr (C::kEarly) {
      const int ew = warp - 2;  // in the stage of k-block k_blocks-3 or k_blocks-2 (see producer)
      const int st = (k_blocks + (ew < C::kEarlyA ? 0 : 1)) % C::kStages;
      ctx.staging = tiles + st * C::kStage + (ew < C::kEarlyA ? ew : ew - C::kEarlyA) * Epi::kWarpStaging;
    } else if constexpr (C::kInTiles) {
      static_assert(kEpilogueWarps * Epi::kWarpStaging <= C::kTiles, "staging in tile buffers");
      ctx.staging = tiles + (warp - 2) * Epi::kWarpStaging;
    } else
      ctx.staging = smem + C::kStagingOffset + (warp - 2) * StagingBufs<Epi>::value * kStageBlockBytes;
    ctx.buf = 0;
    ctx.nbuf = StagingBufs<Epi>::value;
    ctx.out_map = &tmC;
    ctx.ln_map = &tmD;
    ctx.in_bar = in_bars + 2 * (warp - 2);
    ctx.iter = 0;
    ctx.abort_flag = abort_flag;
    ctx.failed = false;
    for (int b = 0; b < 3; ++b) ctx.blocks[b] = ctx.staging + b * (32 * 128);  // EpiResidLN
    ctx.h_in_smem = false;
    if constexpr (C::kAPix) {
      // the CTA's one tile: this warp writes rows 16 (warp - 2) .. + 15 of each k-block's A tile
      int m0, n0_unused, k_slice_unused;
      bool narrow_unused;
      unit_coords<BN>(sched, blockIdx.x, m0, n0_unused, narrow_unused, k_slice_unused);
      if (!pixel_a_tiles<C>(epi.images, M, m0, warp - 2, lane, tiles, full, empty, k_blocks,
                            abort_flag, status) &&
          lane == 0) {
        report(status, kErrProducerWait);
        *abort_flag = 1;
      }
    }
    int acc = 0;
    uint32_t acc_phase = 0;
    bool in_pending = false;  // input blocks requested for a tile not yet processed
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int m0, n0, k_slice;
      bool narrow;
      unit_coords<BN>(sched, tile, m0, n0, narrow, k_slice);
      if constexpr (!C::kNarrow) narrow = false;
      ctx.split = k_slice;
      // a full tile: this warp's column half; a narrow unit: the epilogue splits it itself
      const uint32_t col_off = narrow ? 0u : static_cast<uint32_t>(half * kCols);
      if (!narrow) n0 += half * kCols;
      ctx.narrow = narrow;
      ctx.row = m0 + row_in_tile;
      ctx.row0 = m0 + q * 32;
      typename Epi::Pre pre = epi.prefetch(n0, ctx);
      in_pending = C::kInput && !C::kInTiles;  // kInTiles epilogues load inside run()
      const bool waited = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      if (!__all_sync(0xffffffffu, waited)) {
        if (lane == 0) {
          report(status, kErrEpilogueWait);
          *abort_flag = 1;
        }
        if constexpr (std::is_same<Epi, EpiResidLN>::value) {
          // no work, but the partner warp of this lane quarter waits at the LayerNorm's barrier
          ctx.failed = true;
          epi.template run<kCols>(tmem_base + lane_base + col_off, n0, ctx, pre);
        }
        break;
      }
      tc_fence_after();
      if (C::kInTiles && !C::kEarly) in_pending = true;  // run() requests its input blocks
      epi.template run<kCols>(tmem_base + lane_base + static_cast<uint32_t>(acc * BN) + col_off,
                              n0, ctx, pre);
      if (ctx.failed) {
        if (lane == 0) {
          report(status, kErrEpilogueWait);
          *abort_flag = 1;
        }
        break;
      }
      in_pending = false;
      ++ctx.iter;
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == C::kAccBufs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (Epi::kTmaStore && lane == 0) bulk_wait<0>();  // stores done before the CTA retires
    // Input blocks requested for a tile that was never processed (after an abort) land before
    // shared memory is released.
    if (C::kInput && lane == 0 && in_pending)
      for (int j = 0; j < (C::kInTiles ? 1 : 2); ++j) mbar_drain(&ctx.in_bar[j], ctx.iter & 1u);
  }

  tc_fence_before();
  __syncthreads();
  // Input blocks the producer requested land before shared memory is released (immediate
  // unless the epilogue unwound without consuming them).
  if (C::kEarly && threadIdx.x == 0)
    for (int ew = 0; ew < *in_armed; ++ew) mbar_drain(&in_bars[2 * ew], 0);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// The down projection of layer i with its LayerScale residual and the LayerNorm that follows it
// (EpiResidLN, one 128-row full-width tile per CTA), then, in the same CTA, layer i+1's QKV GEMM
// with RoPE (EpiQkvRope) on the 128 h rows the LayerNorm has just produced: those rows are the
// QKV's whole A operand, so they stay in shared memory instead of going out and back, and the
// QKV's launch start and its uneven last wave go. Layout after the down projection's mainloop
// (three 64 KB stages s_a, s_b, s_c in ring order after its last k-block): h as six 16 KB
// k-block tiles (128 rows x 64 columns, 128-byte swizzle; tiles 0-3 in s_a, 4-5 in the first
// half of s_b; the residual x arrives in the same slots, updated in place, stored, then
// overwritten by h), and three 32 KB QKV weight stages (s_c, s_c + 32 KB, s_b + 32 KB). TMEM:
// the 384-column accumulator, then two 256-column QKV accumulators once the LayerNorm has read
// its rows back. Units of the QKV phase: columns 0-1023 as four 256-wide tiles and 1024-1151 as
// one narrow tile, as in the QKV GEMM.
// ---------------------------------------------------------------------------------------------
namespace {
constexpr int kDqQTile = BM * BK * 2;             // 16 KB: one h k-block tile
constexpr int kDqWStage = 256 * BK * 2;           // 32 KB: one QKV weight k-block
constexpr int kDqBars = 35;                        // mbarriers of the fused kernel
constexpr int kDqBarBytes = 512;
constexpr int kDqStagingBytes = kEpilogueWarps * kStageBlockBytes;
using DqCfg = GemmCfg<384, EpiResidLN>;
// the QKV output staging holds 64-byte-swizzled blocks: it starts on a 1024-byte boundary so
// the swizzle phase of each block row is the one the TMA store applies
constexpr int kDqStagingOffset =
    (DqCfg::kTiles + kDqBarBytes + EpiResidLN::kSmem + EpiQkvRope::kSmem + 1023) / 1024 * 1024;
constexpr int kDqSmem = 1024 + kDqStagingOffset + kDqStagingBytes;
static_assert(DqCfg::kStages == 3 && DqCfg::kStage == 4 * kDqQTile, "three 64 KB stages");
static_assert(kDqBars * 8 + 12 <= kDqBarBytes, "barrier region");
static_assert(kDqSmem <= 227 * 1024, "shared memory budget");
}  // namespace

__global__ void __launch_bounds__(kGemmThreads, 1)
    down_qkv_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmQ, int M, int k_blocks, EpiResidLN epi1,
                    EpiQkvRope epi2, uint32_t *status) {
  using C = DqCfg;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t *smem = smem_raw + pad;
  uint8_t *tiles = smem;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::kTiles);
  uint64_t *empty = full + 3;
  uint64_t *tfull = empty + 3;  // the down projection's accumulator is complete
  uint64_t *in_bars = tfull + 1;  // 2 per epilogue warp (the first used)
  uint64_t *full2 = in_bars + 2 * kEpilogueWarps;
  uint64_t *empty2 = full2 + 3;
  uint64_t *tfull2 = empty2 + 3;
  uint64_t *tempty2 = tfull2 + 2;
  uint64_t *h_ready = tempty2 + 2;
  uint64_t *mma_drain = h_ready + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile int *in_armed = abort_flag + 1;
  uint8_t *extra1 = smem + C::kTiles + kDqBarBytes;
  uint8_t *extra2 = extra1 + EpiResidLN::kSmem;
  uint8_t *staging2 = smem + kDqStagingOffset;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int m0 = static_cast<int>(blockIdx.x) * BM;
  const int sa = k_blocks % 3, sb = (k_blocks + 1) % 3, sc = (k_blocks + 2) % 3;
  auto stage_ptr = [&](int s) { return tiles + s * C::kStage; };
  auto htile = [&](int kb) {
    return kb < 4 ? stage_ptr(sa) + kb * kDqQTile : stage_ptr(sb) + (kb - 4) * kDqQTile;
  };
  auto wstage = [&](int s) {
    return s == 0 ? stage_ptr(sc) : s == 1 ? stage_ptr(sc) + kDqWStage : stage_ptr(sb) + kDqWStage;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < 3; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&full2[s], 1);
      mbar_init(&empty2[s], 1);
    }
    mbar_init(&tfull[0], 1);
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull2[a], 1);
      mbar_init(&tempty2[a], kEpilogueThreads);
    }
    for (int i = 0; i < 2 * kEpilogueWarps; ++i) mbar_init(&in_bars[i], 1);
    mbar_init(h_ready, kEpilogueWarps);
    mbar_init(mma_drain, 1);
    *abort_flag = 0;
    *in_armed = 0;
    fence_mbar_init();
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
    tma_prefetch_map(&tmX);
    tma_prefetch_map(&tmW);
    tma_prefetch_map(&tmQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  epi1.init(extra1, threadIdx.x, kGemmThreads);  // weights only: may overlap the previous kernel
  epi2.init(extra2, threadIdx.x, kGemmThreads);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp >= 2) {  // the down projection's accumulator starts at its bias
    const int q = warp & 3, half = (warp - 2) >> 2;
    epi1.fill_acc(*tmem_slot + (static_cast<uint32_t>(q * 32) << 16) +
                      static_cast<uint32_t>(half * 192),
                  extra1, half);
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();  // activations of the previous kernel are complete from here on
  pdl_trigger();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, armed = 0, last_parity = 0;
      bool ok = true;
      auto next = [&] {
        if (++stage == 3) {
          stage = 0;
          phase ^= 1u;
        }
      };
      auto take = [&](int st, uint32_t ph) {  // a phase-1 stage is free (its MMAs completed)
        if (mbar_wait(&empty[st], ph ^ 1u, abort_flag)) return true;
        report(status, kErrProducerWait);
        *abort_flag = 1;
        return false;
      };
      for (int kb = 0; ok && kb < k_blocks; ++kb) {
        if (!(ok = take(stage, phase))) break;
        uint8_t *a = stage_ptr(stage);
        mbar_arrive_expect_tx(&full[stage], C::kA + 2 * C::kBBox * BK * 2);
        tma_load_2d(a, &tmA, &full[stage], kb * BK, m0);
        for (int s = 0; s < 2; ++s)
          tma_load_2d(a + C::kA + s * C::kBBox * BK * 2, &tmB, &full[stage], kb * BK, s * C::kBBox);
        armed |= 1u << stage;
        last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
        next();
      }
      // Each epilogue warp's x blocks (its lane quarter's 32 rows, its 192 columns) into its h
      // tile slots: tiles 0-3 once s_a is free (after the last-but-two k-block), 4-5 once s_b is.
      for (int part = 0; ok && part < 2; ++part) {
        if (!(ok = take(stage, phase))) break;
        if (part == 0) {
          *in_armed = kEpilogueWarps;
          for (int ew = 0; ew < kEpilogueWarps; ++ew)
            mbar_arrive_expect_tx(&in_bars[2 * ew], 3 * EpiResidLN::kBlockBytes);
        }
        for (int ew = 0; ew < kEpilogueWarps; ++ew) {
          const int q = (ew + 2) & 3, half = ew >> 2;
          for (int b = 0; b < 3; ++b) {
            const int kb = 3 * half + b;
            if ((kb < 4) == (part == 0))
              tma_load_2d(htile(kb) + q * EpiResidLN::kBlockBytes, &tmX, &in_bars[2 * ew],
                          half * 192 + 64 * b, m0 + 32 * q);
          }
        }
        next();
      }
      // QKV weights: s_c takes two weight stages once the last k-block's MMAs are done.
      if (ok) ok = take(stage, phase);
      int s2 = 0;
      uint32_t ph2 = 0, armed2 = 0, last2 = 0;
      for (int u = 0; ok && u < 5; ++u) {
        const int boxes = u < 4 ? 2 : 1;
        for (int kb = 0; kb < kHidden / BK; ++kb) {
          if (!mbar_wait(&empty2[s2], ph2 ^ 1u, abort_flag)) {
            report(status, kErrProducerWait);
            *abort_flag = 1;
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full2[s2], boxes * 128 * BK * 2);
          for (int bx = 0; bx < boxes; ++bx)
            tma_load_2d(wstage(s2) + bx * 128 * BK * 2, &tmW, &full2[s2], kb * BK,
                        256 * u + 128 * bx);
          armed2 |= 1u << s2;
          last2 = (last2 & ~(1u << s2)) | (ph2 << s2);
          if (++s2 == 3) {
            s2 = 0;
            ph2 ^= 1u;
          }
        }
      }
      // copies still in flight (only after an abort) land before shared memory is released
      for (int st = 0; st < 3; ++st) {
        if ((armed >> st) & 1u) mbar_drain(&full[st], (last_parity >> st) & 1u);
        if ((armed2 >> st) & 1u) mbar_drain(&full2[st], (last2 >> st) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      {  // the down projection: two N=192 MMAs per K step onto the bias in TMEM
        constexpr uint32_t idesc = idesc_f16_f32(BM, 192, false);
        int stage = 0;
        uint32_t phase = 0;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!(ok = mbar_wait(&full[stage], phase, abort_flag))) break;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(stage_ptr(stage));
          const uint64_t adesc = sw128_desc(a_addr);
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const uint64_t bdesc = sw128_desc(a_addr + C::kA + s * 192 * BK * 2);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_f16(tmem_base + s * 192, adesc + 2 * k, bdesc + 2 * k, idesc, 1u);
          }
          umma_commit(&empty[stage]);
          if (++stage == 3) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull[0]);
      }
      // the QKV GEMM, once h is in its tiles and the LayerNorm has read its rows out of TMEM
      if (ok) ok = mbar_wait(h_ready, 0, abort_flag);
      tc_fence_after();
      int s2 = 0;
      uint32_t ph2 = 0;
      for (int u = 0; ok && u < 5; ++u) {
        const int acc = u & 1;
        if (u >= 2 && !(ok = mbar_wait(&tempty2[acc], ((u >> 1) - 1) & 1u, abort_flag))) break;
        tc_fence_after();
        const uint32_t idesc = u < 4 ? idesc_f16_f32(BM, 256, false) : idesc_f16_f32(BM, 128, false);
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * 256);
        for (int kb = 0; kb < kHidden / BK; ++kb) {
          if (!(ok = mbar_wait(&full2[s2], ph2, abort_flag))) break;
          tc_fence_after();
          const uint64_t adesc = sw128_desc(smem_u32(htile(kb)));
          const uint64_t bdesc = sw128_desc(smem_u32(wstage(s2)));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty2[s2]);
          if (++s2 == 3) {
            s2 = 0;
            ph2 ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull2[acc]);
      }
      if (!ok) {
        report(status, kErrMmaWait);
        *abort_flag = 1;
      }
      umma_commit(mma_drain);  // every MMA issued has completed before TMEM is freed
      mbar_drain(mma_drain, 0);
    }
  } else {
    const int ew = warp - 2, q = warp & 3, half = ew >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    EpiCtx ctx;
    ctx.M = M;
    ctx.half = half;
    ctx.r = r;
    ctx.lane = lane;
    ctx.row = m0 + r;
    ctx.row0 = m0 + q * 32;
    ctx.smem = extra1;
    ctx.staging = htile(3 * half) + q * EpiResidLN::kBlockBytes;
    for (int b = 0; b < 3; ++b) ctx.blocks[b] = htile(3 * half + b) + q * EpiResidLN::kBlockBytes;
    ctx.h_in_smem = true;
    ctx.buf = 0;
    ctx.nbuf = 1;
    ctx.narrow = false;
    ctx.split = 0;
    ctx.out_map = &tmX;
    ctx.ln_map = &tmX;  // unused: h stays in shared memory
    ctx.in_bar = in_bars + 2 * ew;
    ctx.iter = 0;
    ctx.abort_flag = abort_flag;
    ctx.failed = false;
    bool ok = __all_sync(0xffffffffu, mbar_wait(&tfull[0], 0, abort_flag));
    {  // a warp without its accumulator still meets its partner at the LayerNorm's barrier
      ctx.failed = !ok;
      tc_fence_after();
      EpiResidLN::Pre pre;
      epi1.template run<192>(tmem_base + lane_base + static_cast<uint32_t>(half * 192), half * 192,
                             ctx, pre);
      ok = !ctx.failed;
    }
    // h written (generic proxy) and read by the MMAs (async proxy); TMEM rows read
    fence_proxy_async_smem();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(h_ready);
    EpiCtx c2 = ctx;
    c2.smem = extra2;
    c2.staging = staging2 + ew * kStageBlockBytes;
    c2.out_map = &tmQ;
    c2.h_in_smem = false;
    EpiQkvRope::Pre pre2;
    for (int u = 0; ok && u < 5; ++u) {
      const int acc = u & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull2[acc], (u >> 1) & 1u, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool narrow = u == 4;
      c2.narrow = narrow;
      const uint32_t col_off = narrow ? 0u : static_cast<uint32_t>(half * 128);
      epi2.template run<128>(tmem_base + lane_base + static_cast<uint32_t>(acc * 256) + col_off,
                             256 * u + (narrow ? 0 : half * 128), c2, pre2);
      tc_fence_before();
      mbar_arrive(&tempty2[acc]);
    }
    if (!ok && lane == 0) {
      report(status, kErrEpilogueWait);
      *abort_flag = 1;
    }
    if (lane == 0) bulk_wait<0>();  // stores done before the CTA retires
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0)  // x blocks requested but never consumed (after an abort) land first
    for (int ew = 0; ew < *in_armed; ++ew) mbar_drain(&in_bars[2 * ew], 0);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

bool make_down_qkv_maps(const void *act, uint32_t rows, const void *down_w, void *x,
                        const void *qkv_w, void *qkv, DownQkvMaps *maps, std::string *err) {
  return encode_map_f16(&maps->a, act, kMlp, rows, BK, BM, err) &&
         encode_map_f16(&maps->b, down_w, kMlp, kHidden, BK, 192, err) &&
         encode_map_f16_swizzled(&maps->x, x, kHidden, rows, 64, 32, 128, err) &&
         encode_map_f16(&maps->w, qkv_w, kHidden, kQkv, BK, 128, err) &&
         encode_map_f16_swizzled(&maps->qkv, qkv, kQkv, rows, 32, 32, 64, err);
}

cudaError_t launch_down_qkv(const DownQkvMaps &maps, uint32_t rows, const GemmArgs &down,
                            const GemmArgs &qkv, uint32_t *status, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint32_t m_tiles = (rows + BM - 1) / BM;
  if (m_tiles > static_cast<uint32_t>(sm_count(dev)) || down.ln_out_f32) return cudaErrorInvalidValue;
  static bool configured[64] = {};
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(down_qkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kDqSmem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  return launch_pdl(down_qkv_kernel, dim3(m_tiles), dim3(kGemmThreads), kDqSmem, stream, maps.a,
                    maps.b, maps.x, maps.w, maps.qkv, static_cast<int>(rows), kMlp / BK,
                    EpiResidLN{down.bias, down.lambda, down.gamma, down.beta, false},
                    EpiQkvRope{qkv.bias, qkv.rope_cos, qkv.rope_sin}, status);
}

// The residual GEMMs run on full 384-wide rows (one tile per CTA, A read once: about 0.56 us per
// 64-deep k-block for three 128-column tiles' worth of MMAs, against 0.31 us per k-block for one
// 128-wide tile; the LayerNorm fused) once the row tiles outnumber half the SMs, as long as they
// all fit one wave. Below that the 128-wide tiles (with narrow units for a partial second wave)
// keep three times as many SMs busy and fit about one and a half waves, which measured faster
// (batch 32: 852 against 897 us per forward; even at 48, faster from 56 on).
bool resid_wide(uint32_t rows) {
  int dev = 0;
  cudaGetDevice(&dev);
  const uint32_t m_tiles = (rows + BM - 1) / BM, sms = static_cast<uint32_t>(sm_count(dev));
  return 2 * m_tiles > sms && m_tiles <= sms;
}

// Partial slabs of the no-alloc split-K entry point (dv3k_down_splitk_noalloc): a file-scope
// device array, so that call needs no workspace from its caller and allocates nothing. Sized for
// the largest splits x rows the plan uses (2 slices of 3015 rows at batch 15; 8 of 603 at 3).
constexpr size_t kSplitkScratchFloats = static_cast<size_t>(6144) * kHidden;
static __device__ __align__(256) float g_splitk_scratch[kSplitkScratchFloats];

float *splitk_scratch(size_t *capacity_floats) {
  static void *addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!addr[dev] && cudaGetSymbolAddress(&addr[dev], g_splitk_scratch) != cudaSuccess) {
    addr[dev] = nullptr;
    return nullptr;
  }
  if (capacity_floats) *capacity_floats = kSplitkScratchFloats;
  return static_cast<float *>(addr[dev]);
}

uint32_t splitk_splits(uint32_t rows) {
  int dev = 0;
  cudaGetDevice(&dev);
  const uint32_t tiles = 3 * ((rows + BM - 1) / BM), sms = static_cast<uint32_t>(sm_count(dev));
  for (uint32_t s : {8u, 6u, 4u, 3u, 2u})
    if (tiles * s <= sms) return s;
  return 1;
}

GemmShape gemm_shape(GemmOp op, uint32_t rows) {
  if ((op == GemmOp::Resid384 || op == GemmOp::Resid1536) && resid_wide(rows)) {
    GemmShape s = gemm_shape(op);
    s.bn = 384;
    return s;
  }
  return gemm_shape(op);
}

GemmShape gemm_shape(GemmOp op) {
  switch (op) {
    case GemmOp::Patch: return {128, kHidden, kPatchK};
    case GemmOp::QkvRope: return {256, kQkv, kHidden};  // 4 full tiles + a narrow one per M tile
    case GemmOp::Resid384: return {128, kHidden, kHidden};
    case GemmOp::Resid1536: return {128, kHidden, kMlp};
    case GemmOp::SwiGLU: return {256, kGateUp, kHidden};
    case GemmOp::ResidLN384: return {384, kHidden, kHidden};
    case GemmOp::ResidLN1536: return {384, kHidden, kMlp};
    case GemmOp::SplitK1536: return {128, kHidden, kMlp};
    case GemmOp::PatchPixels: return {384, kHidden, kPatchK};
  }
  return {0, 0, 0};
}

const char *gemm_name(GemmOp op) {
  switch (op) {
    case GemmOp::Patch: return "gemm_patch_embed";
    case GemmOp::QkvRope: return "gemm_qkv_rope";
    case GemmOp::Resid384: return "gemm_o_resid";
    case GemmOp::Resid1536: return "gemm_down_resid";
    case GemmOp::SwiGLU: return "gemm_gateup_swiglu";
    case GemmOp::ResidLN384: return "gemm_o_resid_layernorm";
    case GemmOp::ResidLN1536: return "gemm_down_resid_layernorm";
    case GemmOp::SplitK1536: return "gemm_down_splitk";
    case GemmOp::PatchPixels: return "gemm_patch_pixels";
  }
  return "?";
}

// Width of the tensor the epilogue stores by TMA (0: it writes rows itself).
static uint32_t tma_store_cols(GemmOp op) {
  switch (op) {
    case GemmOp::QkvRope: return kQkv;
    case GemmOp::SwiGLU: return kMlp;
    case GemmOp::Resid384:
    case GemmOp::Resid1536:
    case GemmOp::ResidLN384:
    case GemmOp::ResidLN1536: return kHidden;
    default: return 0;
  }
}

bool make_gemm_maps(GemmOp op, const void *a, uint32_t rows, const void *w, void *out,
                    GemmMaps *maps, std::string *err, const void *ln_out, bool ln_f32,
                    uint32_t splits) {
  const GemmShape s = gemm_shape(op, rows);
  // weight boxes: one per MMA of the K step (BN = 384: two of 192 rows), or BN/2 rows for the
  // ops that take narrow units (BN = 256, and the 128-wide residual GEMMs): two per full tile,
  // one per narrow unit
  const bool narrow_ops =
      s.bn == 256 ||
      (s.bn == 128 && (op == GemmOp::Resid384 || op == GemmOp::Resid1536 || op == GemmOp::Patch));
  const uint32_t b_rows = s.bn >= 256 || narrow_ops ? s.bn / 2 : s.bn;
  if (!encode_map_f16(&maps->b, w, s.k, s.n, BK, b_rows, err)) return false;
  if (op == GemmOp::PatchPixels)
    maps->a = maps->b;  // no A map: the epilogue warps build the A tiles from the images
  else if (!encode_map_f16(&maps->a, a, s.k, rows, BK, BM, err))
    return false;
  maps->d = maps->a;  // unused unless the epilogue writes a LayerNorm output
  if (op == GemmOp::SplitK1536)  // f32 partial slabs [splits][rows][384], 32x32 blocks
    return encode_map_f32_slabs(&maps->c, out, kHidden, rows, splits, 32, err);
  const uint32_t c_cols = tma_store_cols(op);
  if (c_cols == 0) {
    maps->c = maps->a;  // unused by this epilogue
    return true;
  }
  const bool ln = op == GemmOp::ResidLN384 || op == GemmOp::ResidLN1536;
  // the LayerNorm epilogue moves 64-column blocks (128-byte rows), the others 32-column blocks
  if (!encode_map_f16_swizzled(&maps->c, out, c_cols, rows, ln ? 64 : 32, 32, ln ? 128 : 64, err))
    return false;
  if (ln) {
    if (ln_out == nullptr) {
      if (err) *err = "the fused LayerNorm needs an output tensor";
      return false;
    }
    return ln_f32 ? encode_map_f32(&maps->d, ln_out, kHidden, rows, 32, 32, err)
                  : encode_map_f16_swizzled(&maps->d, ln_out, kHidden, rows, 64, 32, 128, err);
  }
  return true;
}

template <int BN, class Epi>
static cudaError_t configure_one() {
  return cudaFuncSetAttribute(gemm_kernel<BN, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              gemm_smem_bytes<BN, Epi>());
}

// The schedule of a launch (TileSched). BN = 256: N = full_n*256 (+ 128 for QKV's last
// columns, one narrow unit per M tile, last); when the 2L halves of a partial last wave of L
// full tiles (plus QKV's narrow tiles) fit one wave of CTAs, those L tiles run as 2L narrow
// units, so the last wave costs half a tile instead of a whole one.
template <int BN, class Epi>
static TileSched tile_sched(uint32_t rows, int n, int sms, int k_splits = 1) {
  TileSched t;
  t.k_splits = k_splits;
  t.m_tiles = static_cast<int>((rows + BM - 1) / BM);
  const bool narrow_ok = GemmCfg<BN, Epi>::kNarrow && k_splits == 1;
  t.full_n = narrow_ok ? n / BN : (n + BN - 1) / BN;
  const bool native_half = narrow_ok && n % BN != 0;  // n % BN == BN / 2 (QKV)
  const int full = t.m_tiles * t.full_n;
  t.split_from = full;
  if (narrow_ok && full > sms) {  // the halves of a partial last wave, with QKV's native narrow
    const int left = full % sms;  // tiles, in at most one more wave of narrow units
    if (left > 0 && 2 * left + (native_half ? t.m_tiles : 0) <= sms) t.split_from = full - left;
  }
  // Small batches: when even the halves of every tile fit one wave, all of them run as narrow
  // units, so twice as many SMs share the work and each epilogue has half as much.
  if (narrow_ok && 2 * full <= sms) t.split_from = 0;
  t.num_units = t.split_from + 2 * (full - t.split_from) + (native_half ? t.m_tiles : 0);
  if (k_splits > 1) t.num_units = full * k_splits;  // full tiles only, repeated per K slice
  t.l2_next = nullptr;
  t.l2_next_bytes = 0;
  return t;
}

template <int BN, class Epi>
static cudaError_t launch_one(const GemmMaps &maps, uint32_t rows, int n, int k, const Epi &epi,
                              uint32_t *status, cudaStream_t stream, const GemmArgs &args,
                              int k_splits = 1) {
  static bool configured[64] = {};  // per template instance and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = configure_one<BN, Epi>();
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  TileSched sched = tile_sched<BN, Epi>(rows, n, sm_count(dev), k_splits);
  sched.l2_next = args.l2_next;
  sched.l2_next_bytes = args.l2_next_bytes & ~static_cast<size_t>(15);
  const int grid = sched.num_units < sm_count(dev) ? sched.num_units : sm_count(dev);
  return launch_pdl(gemm_kernel<BN, Epi>, dim3(grid), dim3(kGemmThreads),
                    gemm_smem_bytes<BN, Epi>(), stream, maps.a, maps.b, maps.c, maps.d,
                    static_cast<int>(rows), sched, k / BK / k_splits, epi, status);
}

// Set the shared-memory limits of every GEMM instance on the current device (done at load, so
// that graph capture never meets a first-use attribute call).
cudaError_t configure_gemm_kernels() {
  cudaError_t e;
  if ((e = configure_one<128, EpiPatch>()) != cudaSuccess) return e;
  if ((e = configure_one<256, EpiQkvRope>()) != cudaSuccess) return e;
  if ((e = configure_one<128, EpiResid>()) != cudaSuccess) return e;
  if ((e = configure_one<384, EpiResidWide>()) != cudaSuccess) return e;
  if ((e = configure_one<256, EpiSwiGLU>()) != cudaSuccess) return e;
  if ((e = configure_one<384, EpiResidLN>()) != cudaSuccess) return e;
  if ((e = configure_one<128, EpiPartialF32>()) != cudaSuccess) return e;
  if ((e = configure_one<384, EpiPatchPixels>()) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(down_qkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kDqSmem)) != cudaSuccess)
    return e;
  int dev = 0;
  cudaGetDevice(&dev);
  sm_count(dev);
  return cudaSuccess;
}

cudaError_t launch_gemm(GemmOp op, const GemmMaps &maps, uint32_t rows, const GemmArgs &args,
                        uint32_t *status, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  const GemmShape s = gemm_shape(op);
  switch (op) {
    case GemmOp::Patch:
      return launch_one<128>(maps, rows, s.n, s.k, EpiPatch{args.bias, args.out}, status, stream,
                             args);
    case GemmOp::QkvRope:
      return launch_one<256>(maps, rows, s.n, s.k,
                             EpiQkvRope{args.bias, args.rope_cos, args.rope_sin}, status, stream, args);
    case GemmOp::Resid384:
    case GemmOp::Resid1536:
      if (resid_wide(rows))
        return launch_one<384>(maps, rows, s.n, s.k, EpiResidWide{args.bias, args.lambda}, status,
                               stream, args);
      return launch_one<128>(maps, rows, s.n, s.k, EpiResid{args.bias, args.lambda},
                             status, stream, args);
    case GemmOp::SwiGLU:
      return launch_one<256>(maps, rows, s.n, s.k, EpiSwiGLU{args.bias}, status, stream,
                             args);
    case GemmOp::ResidLN384:
    case GemmOp::ResidLN1536:
      return launch_one<384>(maps, rows, s.n, s.k,
                             EpiResidLN{args.bias, args.lambda, args.gamma, args.beta,
                                        args.ln_out_f32 != nullptr},
                             status, stream, args);
    case GemmOp::SplitK1536:
      if (args.splits == 0 || (kMlp / BK) % args.splits != 0) return cudaErrorInvalidValue;
      return launch_one<128>(maps, rows, s.n, s.k, EpiPartialF32{}, status, stream, args,
                             static_cast<int>(args.splits));
    case GemmOp::PatchPixels: {
      // one tile per CTA: at most one wave of 128-row tiles (96 images on 148 SMs)
      int dev = 0;
      cudaGetDevice(&dev);
      if (!args.images || !args.prefix || !args.out || rows % kPatches != 0 ||
          (rows + BM - 1) / BM > static_cast<uint32_t>(sm_count(dev)))
        return cudaErrorInvalidValue;
      return launch_one<384>(maps, rows, s.n, s.k,
                             EpiPatchPixels{args.bias, args.out, args.images, args.prefix},
                             status, stream, args);
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace dv3
