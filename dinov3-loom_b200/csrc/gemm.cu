// gemm.cu - persistent, warp-specialised tcgen05 GEMM for the projections of the forward, each
// with its epilogue fused (gemm_epilogues.cuh):
//   Patch     x[token(p)] = f16(A W^T + b)                 kernels/matmul_bias_f16_wmma.loom
//                                                          + kernels/embed_scatter_f32.loom
//   QkvRope   qkv = f16(rope(A W^T + b))                   kernels/matmul_qkv_rope_f16_wmma.loom
//   Resid*    x = f16(x + lambda (A W^T + b))              kernels/matmul_resid_f16_wmma.loom
//   ResidLN*  the same on full rows, then LayerNorm        + kernels/layernorm_rowwave_*.loom
//   SwiGLU    act = f16(silu(A Wg^T + bg) (A Wu^T + bu))   kernels/matmul_swiglu_f16_wmma.loom
//   SplitK    partials[s] = A[:, K_s] W[:, K_s]^T (f32)     kernels/matmul_splitk_f16_wmma.loom
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
#include <atomic>
#include <mutex>
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

// Whether the GEMM runs one more K=16 step per unit after its k-blocks (Epi::kAuxK, the folded
// LayerNorm): A from the row aux [rows][16] (map tmD) and B from the weight aux [n][16] (map
// tmE), 32-byte rows with the 32-byte swizzle, loaded into the next stage buffer of the ring.
template <class Epi, class = void>
struct AuxK {
  static constexpr bool value = false;
};
template <class Epi>
struct AuxK<Epi, decltype(void(Epi::kAuxK))> {
  static constexpr bool value = Epi::kAuxK;
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
  static constexpr bool kAux = AuxK<Epi>::value;
  static constexpr int kAuxA = BM * 32;  // bytes of the aux A tile (128 rows x 16 f16)
  // configurations whose launches have exactly one tile per CTA
  static constexpr bool kOneTile = kInTiles || kBiasInit;
  static_assert(!kBiasInit || BN == 384, "bias fill: one full-row tile per CTA");
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
  const void *discard;    // a dead intermediate to drop from L2 after the dependency wait
  size_t discard_bytes;
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
// The kernel
// ---------------------------------------------------------------------------------------------
template <int BN, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                const __grid_constant__ CUtensorMap tmE, int M, TileSched sched, int k_blocks,
                Epi epi, uint32_t *status) {
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
  // The scalar launch parameters are read here, in the set-up that overlaps the previous kernel:
  // a first read from the parameter bank misses the constant cache (hundreds of cycles), and
  // the roles would otherwise take those misses after their dependency wait.
  asm volatile("" ::"r"(M), "r"(sched.m_tiles), "r"(sched.full_n), "r"(sched.split_from),
               "r"(sched.num_units), "r"(sched.k_splits), "r"(k_blocks));

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
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
    if (std::is_same<Epi, EpiResidLN>::value || C::kAux) tma_prefetch_map(&tmD);
    if (C::kAux) tma_prefetch_map(&tmE);
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
  // Programmatic dependent launch: only the roles that touch what earlier kernels wrote or read
  // wait for the previous kernel (griddepcontrol.wait): the TMA producer right before its first
  // load, and the epilogue warps before their first input request or store. The MMA issuer reads
  // only shared memory that the producer filled after its wait. Each role's entry code (and the
  // fetch of its instructions) thus overlaps the previous kernel's tail.
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
          if (tile == static_cast<int>(blockIdx.x) && kb == 0) {
            pdl_wait();  // activations of the previous kernel are complete from here on
            pdl_trigger();
          }
          uint8_t *a = tiles + stage * C::kStage;
          mbar_arrive_expect_tx(&full[stage], C::kA + b_boxes * C::kBBox * BK * 2);
          tma_load_2d(a, &tmA, &full[stage], (kb0 + kb) * BK, m0);
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
        if constexpr (C::kAux) {
          // the extra K=16 step: the unit's 128 aux rows (A) and its columns' aux rows (B)
          if (ok && !mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            report(status, kErrProducerWait);
            *abort_flag = 1;
            ok = false;
          }
          if (ok) {
            uint8_t *a = tiles + stage * C::kStage;
            mbar_arrive_expect_tx(&full[stage], C::kAuxA + b_boxes * C::kBBox * 32);
            tma_load_2d(a, &tmD, &full[stage], 0, m0);
            for (int s = 0; s < b_boxes; ++s)
              tma_load_2d(a + C::kA + s * C::kBBox * 32, &tmE, &full[stage], 0,
                          n0 + s * C::kBBox);
            armed |= 1u << stage;
            last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
            if (++stage == C::kStages) {
              stage = 0;
              phase ^= 1u;
            }
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
        if constexpr (C::kAux) {  // the extra K=16 step (see the producer)
          if (ok && !mbar_wait(&full[stage], phase, abort_flag)) {
            report(status, kErrMmaWait);
            *abort_flag = 1;
            ok = false;
          }
          if (ok) {
            tc_fence_after();
            const uint32_t a_addr = smem_u32(tiles + stage * C::kStage);
            umma_f16(d, sw32_desc(a_addr), sw32_desc(a_addr + C::kA), idesc, 1u);
            umma_commit(&empty[stage]);
            if (++stage == C::kStages) {
              stage = 0;
              phase ^= 1u;
            }
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
    pdl_wait();  // before the first input request or store (see above)
    pdl_trigger();
    if (sched.discard)  // idle until the first accumulator
      l2_discard_share(sched.discard, sched.discard_bytes, threadIdx.x - 64, kEpilogueThreads);
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

// With the LayerNorms folded (the full-row residual GEMMs leave only the row statistics, and QKV
// and gate/up apply the LayerNorm), the full-row plan wins as soon as the 128-wide residual
// tiles (three per row tile) need more than one wave: on 148 SMs from 50 row tiles (batch 32),
// where the 128-wide plan steps from 742 to 837 us per forward between batch 31 and 32 and the
// folded plan takes 798 us (906 against 968 us at batch 47; below 32 the 128-wide plan is faster:
// 696 against 741 us at 25, 742 against 772 at 31).
bool resid_full_rows_plan(uint32_t rows) {
  int dev = 0;
  cudaGetDevice(&dev);
  const uint32_t m_tiles = (rows + BM - 1) / BM, sms = static_cast<uint32_t>(sm_count(dev));
  return 3 * m_tiles > sms && m_tiles <= sms;
}

// Partial slabs of the no-alloc split-K entry point (dv3k_down_splitk_noalloc): a file-scope
// device array, so that call needs no workspace from its caller and allocates nothing. Its size
// is fixed when the library is built (6144 partial rows of 384 floats, 9 MiB on every device that
// loads the library); it is not derived from splitk_splits, which may pick more slices on a GPU
// with more SMs. 6144 covers the slices the model's plan takes on a 148-SM B200 (2 slices of 3015
// rows at batch 15, 8 of 603 at batch 3); callers size splits x rows to fit it.
constexpr size_t kSplitkScratchFloats = static_cast<size_t>(6144) * kHidden;
static __device__ __align__(256) float g_splitk_scratch[kSplitkScratchFloats];

// The array's device address is looked up once per device (with that device current) under a
// lock, so concurrent first calls from several host threads are safe. The address belongs to the
// device's primary context: a cudaDeviceReset of that device invalidates it, as it does every
// other device resource of this library.
float *splitk_scratch(size_t *capacity_floats) {
  static std::mutex lock;
  static void *addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> guard(lock);
  if (!addr[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_splitk_scratch) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    addr[dev] = p;
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
    case GemmOp::ResidStats384: return {384, kHidden, kHidden};
    case GemmOp::ResidStats1536: return {384, kHidden, kMlp};
    case GemmOp::QkvRopeFold: return {256, kQkv, kHidden};
    case GemmOp::SwiGLUFold: return {256, kGateUp, kHidden};
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
    case GemmOp::ResidStats384: return "gemm_o_resid_rowstat";
    case GemmOp::ResidStats1536: return "gemm_down_resid_rowstat";
    case GemmOp::QkvRopeFold: return "gemm_qkv_rope_folded";
    case GemmOp::SwiGLUFold: return "gemm_gateup_swiglu_folded";
  }
  return "?";
}

// Width of the tensor the epilogue stores by TMA (0: it writes rows itself).
static uint32_t tma_store_cols(GemmOp op) {
  switch (op) {
    case GemmOp::QkvRope:
    case GemmOp::QkvRopeFold: return kQkv;
    case GemmOp::SwiGLU:
    case GemmOp::SwiGLUFold: return kMlp;
    case GemmOp::Resid384:
    case GemmOp::Resid1536:
    case GemmOp::ResidLN384:
    case GemmOp::ResidLN1536:
    case GemmOp::ResidStats384:
    case GemmOp::ResidStats1536: return kHidden;
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
  if (!encode_map_f16(&maps->a, a, s.k, rows, BK, BM, err)) return false;
  maps->d = maps->a;  // unused unless the epilogue writes a LayerNorm output (or the fold's aux)
  maps->e = maps->a;  // unused unless the fold's aux
  if (op == GemmOp::SplitK1536)  // f32 partial slabs [splits][rows][384], 32x32 blocks
    return encode_map_f32_slabs(&maps->c, out, kHidden, rows, splits, 32, err);
  const uint32_t c_cols = tma_store_cols(op);
  if (c_cols == 0) {
    maps->c = maps->a;  // unused by this epilogue
    return true;
  }
  const bool ln = op == GemmOp::ResidLN384 || op == GemmOp::ResidLN1536;
  const bool full_row = ln || op == GemmOp::ResidStats384 || op == GemmOp::ResidStats1536;
  // the full-row residual epilogue moves 64-column blocks (128-byte rows), the others 32-column
  // blocks
  if (!encode_map_f16_swizzled(&maps->c, out, c_cols, rows, full_row ? 64 : 32, 32,
                               full_row ? 128 : 64, err))
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

bool make_fold_maps(GemmOp op, const void *row_aux, uint32_t rows, const void *w_aux,
                    GemmMaps *maps, std::string *err) {
  if (op != GemmOp::QkvRopeFold && op != GemmOp::SwiGLUFold) {
    if (err) *err = "no folded LayerNorm in this GEMM";
    return false;
  }
  const GemmShape s = gemm_shape(op, rows);
  // 16-column boxes: 128 rows of the unit (A), and the weight boxes' rows (B: BN/2 rows, two per
  // full tile and one per narrow unit, as for the weights)
  return encode_map_f16_swizzled(&maps->d, row_aux, 16, rows, 16, BM, 32, err) &&
         encode_map_f16_swizzled(&maps->e, w_aux, 16, s.n, 16, s.bn / 2, 32, err);
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
  t.discard = nullptr;
  t.discard_bytes = 0;
  return t;
}

template <int BN, class Epi>
static cudaError_t launch_one(const GemmMaps &maps, uint32_t rows, int n, int k, const Epi &epi,
                              uint32_t *status, cudaStream_t stream, const GemmArgs &args,
                              int k_splits = 1) {
  static std::atomic<bool> configured[64] = {};  // per template instance and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev].load(std::memory_order_acquire)) {
    // setting the attribute twice (two threads racing here) is harmless
    cudaError_t e = configure_one<BN, Epi>();
    if (e != cudaSuccess) return e;
    configured[dev].store(true, std::memory_order_release);
  }
  TileSched sched = tile_sched<BN, Epi>(rows, n, sm_count(dev), k_splits);
  sched.l2_next = args.l2_next;
  sched.l2_next_bytes = args.l2_next_bytes & ~static_cast<size_t>(15);
  discard_range(args.discard, args.discard_bytes, &sched.discard, &sched.discard_bytes);
  const int grid = sched.num_units < sm_count(dev) ? sched.num_units : sm_count(dev);
  return launch_pdl(gemm_kernel<BN, Epi>, dim3(grid), dim3(kGemmThreads),
                    gemm_smem_bytes<BN, Epi>(), stream, maps.a, maps.b, maps.c, maps.d, maps.e,
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
  if ((e = configure_one<256, EpiSwiGLUFold>()) != cudaSuccess) return e;
  if ((e = configure_one<256, EpiQkvRopeFold>()) != cudaSuccess) return e;
  if ((e = configure_one<384, EpiResidLN>()) != cudaSuccess) return e;
  if ((e = configure_one<128, EpiPartialF32>()) != cudaSuccess) return e;
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
    case GemmOp::ResidStats384:
    case GemmOp::ResidStats1536:
      if (args.rowstat == nullptr || args.row_aux == nullptr) return cudaErrorInvalidValue;
      return launch_one<384>(maps, rows, s.n, s.k,
                             EpiResidLN{args.bias, args.lambda, nullptr, nullptr, false,
                                        args.rowstat, args.row_aux},
                             status, stream, args);
    case GemmOp::QkvRopeFold:
      if (args.rowstat == nullptr) return cudaErrorInvalidValue;
      return launch_one<256>(maps, rows, s.n, s.k,
                             EpiQkvRopeFold{nullptr, args.rope_cos, args.rope_sin, args.rowstat},
                             status, stream, args);
    case GemmOp::SwiGLUFold:
      if (args.rowstat == nullptr) return cudaErrorInvalidValue;
      return launch_one<256>(maps, rows, s.n, s.k, EpiSwiGLUFold{nullptr, args.rowstat}, status,
                             stream, args);
    case GemmOp::SplitK1536:
      if (args.splits == 0 || (kMlp / BK) % args.splits != 0) return cudaErrorInvalidValue;
      return launch_one<128>(maps, rows, s.n, s.k, EpiPartialF32{}, status, stream, args,
                             static_cast<int>(args.splits));
  }
  return cudaErrorInvalidValue;
}

}  // namespace dv3
