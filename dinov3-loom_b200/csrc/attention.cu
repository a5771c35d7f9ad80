// attention.cu - multi-head attention of the forward on tcgen05 tensor cores: one persistent
// CTA per SM walks (image, head) work items. Replaces kernels/attention_online_f16_wmma_cf16.loom
// (6 heads x 64, 201 tokens, scale 0.125).
//
// A work item covers the 201 queries of one head of one image as two 128-row tiles (tile 1 holds
// tokens 128..200 and rows that are dropped) against all 201 keys. Every key fits one tile, so
// the softmax is exact in one pass over S instead of online.
//
// Global memory is seen through per-image 3D tensor maps [image][201 tokens][columns]: token
// rows past 201 read as zeros and are clipped on store, so no tile reaches into the next image.
//
// Roles (352 threads):
//   warp 8     TMA producer. Per item: Q as two 128-token boxes, K and V as 208-token boxes of
//              this head's columns of the fused QKV rows, 128-byte swizzle, into one of two
//              shared-memory stages, so item i+1 loads while item i computes.
//   warps 9/10 MMA issuers of tile 0 / tile 1 (lane 0); warp 9 also allocates TMEM (512
//              columns). Tile t owns TMEM columns 256t..256t+255:
//                S_t = Q_t K^T   M=128, N=208, K=64 (4 MMAs)         columns   0..207, f32
//                P_t = f16 probabilities written by the softmax       columns   0..103 (2 keys
//                      per column, over the consumed S)
//                O_t = P_t V     A read from TMEM, V the MN-major B   columns 128..191, f32
//                                operand in shared memory, K=208 (13 MMAs)
//              Each issuer walks the items in order: S_t (needs the item's loads and tile t's
//              TMEM released), then PV_t (needs P_t); a stage is released after both tiles' PVs
//              of its item. An MMA holds its issuing thread about 80 cycles whatever its N (PV's
//              13 MMAs of N=64 cost about 1000 cycles, S's 4 of N=208 about 430), so one issuer
//              per tile keeps either tile from waiting behind the other's issue. Tile 1 starts
//              when tile 0's first P is written: from then on one tile's softmax overlaps the
//              other tile's MMAs and output instead of both competing for the exp2 unit.
//   warps 0-3  softmax and output of tile 0, warps 4-7 of tile 1 (warp 7 idles: tile 1 rows
//              96..127 are tokens 224..255). One query row per thread (TMEM lane 32*(w%4)+lane).
//              Pass 1: row max over the 201 valid keys. Pass 2: w = exp(0.125 (s - max)) =
//              2^(s c - max c) with c = 0.125 log2(e) (one FFMA and the hardware exp2), f32 sum of
//              w, P = f16(w) (keys >= 201 zero) stored to TMEM. Once O is in TMEM: O / sum rounded
//              to f16 into a per-warp 32-row staging tile (128-byte swizzle), written out by one
//              TMA store per warp.
// Small batches (two query tiles per item still fit one CTA each, 2 x items <= SMs): the grid
// has two CTAs per item and each computes one query tile (tile_split); the other tile's roles
// idle, so an item costs one tile's chain instead of one and a half.
// The probabilities are rounded to f16 before PV and the normaliser is the f32 sum of the
// unrounded weights, as in the reference kernel (:214-216).
//
// Every wait is bounded; on a timeout the kernel records kErrAttentionWait, raises the CTA's
// abort flag, lets its own copies and MMAs in flight land, frees TMEM and returns.
#include <atomic>

#include "attention_softmax.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace dv3 {

namespace {
using namespace attn;
constexpr int kAttnThreads = 352;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;  // TMEM allocator; issues tile 0's MMAs, warp 10 tile 1's
constexpr int kKvBox = kSKeys;       // K, V token rows loaded per item
constexpr int kQBytes = 128 * 128;   // 128 rows x 64 f16
constexpr int kKvBytes = kKvBox * 128;
// One stage: Q tile 0 | Q tile 1 | K | V, each 1024-byte aligned (8-row swizzle atoms).
constexpr int kStageQ0 = 0;
constexpr int kStageQ1 = kQBytes;
constexpr int kStageK = 2 * kQBytes;
constexpr int kStageV = kStageK + kKvBytes;
constexpr int kStageBytes = kStageV + kKvBytes;
constexpr uint32_t kLoadBytes = 2 * kQBytes + 2 * kKvBytes;
constexpr int kStages = 2;
constexpr int kStagingOff = kStages * kStageBytes;  // 8 warps x 32 rows x 128 B
constexpr int kStagingBytes = kOutBox * 128;
constexpr int kBarOff = kStagingOff + 8 * kStagingBytes;
// 14 mbarriers: load_full[2], load_empty[2], s_full[2], p_full[2], o_full[2], tmem_empty[2],
// drain[2]; then the TMEM slot and the abort flag.
constexpr int kAttnSmem = 1024 + kBarOff + 128;
constexpr int kTmemCols = 512;
static_assert(kStageV % 1024 == 0 && kStageBytes % 1024 == 0 && kStagingOff % 1024 == 0,
              "swizzle atoms");
static_assert(kAttnSmem <= 227 * 1024, "shared memory budget");
}  // namespace

__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmq,
                     const __grid_constant__ CUtensorMap tmkv,
                     const __grid_constant__ CUtensorMap tmo, int n_items, int tile_split,
                     const void *l2_next, size_t l2_next_bytes, const void *discard,
                     size_t discard_bytes, uint32_t *status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t *smem = smem_raw + pad;
  uint64_t *load_full = reinterpret_cast<uint64_t *>(smem + kBarOff);
  uint64_t *load_empty = load_full + 2;
  uint64_t *s_full = load_full + 4;
  uint64_t *p_full = load_full + 6;
  uint64_t *o_full = load_full + 8;
  uint64_t *tmem_empty = load_full + 10;
  uint64_t *drain = load_full + 12;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(load_full + 14);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // Items of this CTA: blockIdx.x, blockIdx.x + gridDim.x, ... With tile_split (small batches,
  // a grid of two CTAs per item) CTA b takes only query tile b & 1 of item b >> 1, and the other
  // tile's roles have nothing to do.
  const int only_tile = tile_split ? static_cast<int>(blockIdx.x & 1u) : -1;
  const int count = tile_split ? (static_cast<int>(blockIdx.x >> 1) < n_items ? 1 : 0)
                    : static_cast<int>(blockIdx.x) < n_items
                        ? (n_items - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                        : 0;
  auto item_of = [&](int k) {
    return tile_split ? static_cast<int>(blockIdx.x >> 1)
                      : static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&load_full[i], 1);
      mbar_init(&load_empty[i], tile_split ? 1 : 2);  // one commit per active tile's issuer
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&tmem_empty[i], 128);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_map(&tmq);
    tma_prefetch_map(&tmkv);
    tma_prefetch_map(&tmo);
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent launch: only the TMA producer reads what the previous kernel wrote,
  // so only it waits for that kernel (before its first load); the other roles start on the data
  // it brings. Their entry code overlaps the previous kernel's tail.
  // the producer warp's idle lane starts a later kernel's weights toward L2
  if (warp == kProducerWarp && lane == 1 && l2_next) l2_prefetch_share(l2_next, l2_next_bytes);
  // its other idle lanes drop a dead intermediate from L2 once the previous kernel is complete
  if (warp == kProducerWarp && lane >= 2 && discard) {
    pdl_wait();
    l2_discard_share(discard, discard_bytes, lane - 2, 30);
  }

  if (warp == kProducerWarp) {
    if (lane == 0) {
      uint32_t armed = 0, last_parity = 0;  // per stage: armed at least once, parity of the last
      for (int k = 0; k < count; ++k) {
        const int s = k & 1;
        const uint32_t ph = (k >> 1) & 1;
        if (!mbar_wait(&load_empty[s], ph ^ 1u, abort_flag)) {
          report(status, kErrAttentionWait);
          *abort_flag = 1;
          break;
        }
        if (k == 0) {
          pdl_wait();  // the QKV rows of the previous kernel are complete from here on
          pdl_trigger();
        }
        const int item = item_of(k);
        const int img = item / kHeads, head = item % kHeads;
        uint8_t *st = smem + s * kStageBytes;
        mbar_arrive_expect_tx(&load_full[s], only_tile < 0 ? kLoadBytes : kLoadBytes - kQBytes);
        if (only_tile != 1) tma_load_3d(st + kStageQ0, &tmq, &load_full[s], head * 64, 0, img);
        if (only_tile != 0) tma_load_3d(st + kStageQ1, &tmq, &load_full[s], head * 64, 128, img);
        tma_load_3d(st + kStageK, &tmkv, &load_full[s], kHidden + head * 64, 0, img);
        tma_load_3d(st + kStageV, &tmkv, &load_full[s], 2 * kHidden + head * 64, 0, img);
        armed |= 1u << s;
        last_parity = (last_parity & ~(1u << s)) | (ph << s);
      }
      // Copies still in flight (only after an abort) land before shared memory is released.
      for (int s = 0; s < kStages; ++s)
        if ((armed >> s) & 1u) mbar_drain(&load_full[s], (last_parity >> s) & 1u);
    }
  } else if (warp == kMmaWarp || warp == kMmaWarp + 1) {
    // One issuer thread per tile, so neither tile's MMAs wait behind the other's issue.
    if (lane == 0 && (only_tile < 0 || warp - kMmaWarp == only_tile)) {
      const int t = warp - kMmaWarp;
      constexpr uint32_t idesc_s = idesc_f16_f32(128, kSKeys, false);
      constexpr uint32_t idesc_o = idesc_f16_f32(128, 64, true);
      const uint32_t d_s = tmem + t * kTileCols, d_o = d_s + kOCol;
      bool ok = true;
      for (int k = 0; ok && k < count; ++k) {
        const uint32_t par = k & 1;
        const uint8_t *st = smem + (k & 1) * kStageBytes;
        // Tile 1 starts once tile 0's first P is written: from then on one tile's softmax
        // overlaps the other tile's MMAs and output instead of both competing for the exp2 unit.
        // A CTA with a single item (small batches) has nothing to overlap and starts both.
        ok = mbar_wait(&load_full[k & 1], (k >> 1) & 1, abort_flag) &&
             mbar_wait(&tmem_empty[t], par ^ 1u, abort_flag) &&
             (t == 0 || k > 0 || count == 1 || mbar_wait(&p_full[0], 0, abort_flag));
        if (!ok) break;
        tc_fence_after();
        const uint64_t qd = sw128_desc(smem_u32(st + (t ? kStageQ1 : kStageQ0)));
        const uint64_t kd = sw128_desc(smem_u32(st + kStageK));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_f16(d_s, qd + 2 * kk, kd + 2 * kk, idesc_s, kk > 0);
        umma_commit(&s_full[t]);
        ok = mbar_wait(&p_full[t], par, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t vb = smem_u32(st + kStageV);
#pragma unroll
        for (int kk = 0; kk < kSKeys / 16; ++kk)
          umma_f16_ts(d_o, d_s + 8 * kk, sw128_desc(vb + kk * 2048), idesc_o, kk > 0);
        umma_commit(&o_full[t]);
        umma_commit(&load_empty[k & 1]);  // this tile is done with the item's stage
      }
      if (!ok) {
        report(status, kErrAttentionWait);
        *abort_flag = 1;
      }
      umma_commit(&drain[t]);  // every MMA this thread issued has completed before TMEM is freed
      mbar_drain(&drain[t], 0);
    }
  } else {
    const int t = warp >> 2, q = warp & 3;
    const int my_count = only_tile < 0 || t == only_tile ? count : 0;
    const int r = q * 32 + lane;
    const uint32_t tl = tmem + (static_cast<uint32_t>(q * 32) << 16) + t * kTileCols;
    const bool active = !(t == 1 && q == 3);  // warp-uniform
    uint8_t *stg = smem + kStagingOff + warp * kStagingBytes;
    uint8_t *stg_row = stg + r % 32 * 128;
    for (int k = 0; k < my_count; ++k) {
      const uint32_t par = k & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[t], par, abort_flag))) {
        if (lane == 0) {
          report(status, kErrAttentionWait);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      float sum = 1.f;
      if (active) sum = softmax_row(tl);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
      if (!__all_sync(0xffffffffu, mbar_wait(&o_full[t], par, abort_flag))) {
        if (lane == 0) {
          report(status, kErrAttentionWait);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      uint32_t o0[32], o1[32];
      if (active) tmem_load32x2(tl + kOCol, o0, tl + kOCol + 32, o1);
      tc_fence_before();
      mbar_arrive(&tmem_empty[t]);
      if (active) {
        const float inv = 1.0f / sum;
        if (lane == 0) bulk_wait_read<0>();  // the previous store has read the staging tile
        __syncwarp();
        stage_output_row(stg_row, lane, o0, o1, inv);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int item = item_of(k);
          tma_store_3d(&tmo, stg, (item % kHeads) * 64, t * 128 + q * 32, item / kHeads);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait<0>();  // output stores complete before the CTA retires
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

bool make_attention_map(const void *qkv, const void *out, uint32_t rows, AttentionMaps *maps,
                        std::string *err) {
  const uint32_t n_images = rows / kTokens;
  return encode_map_f16_images(&maps->q, qkv, kQkv, n_images, 128, err) &&
         encode_map_f16_images(&maps->kv, qkv, kQkv, n_images, kKvBox, err) &&
         encode_map_f16_images(&maps->out, out, kHidden, n_images, kOutBox, err);
}

cudaError_t configure_attention_kernel() {
  return cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kAttnSmem);
}

cudaError_t launch_attention(const AttentionMaps &maps, uint32_t rows, uint32_t *status,
                             cudaStream_t stream, const void *l2_next, size_t l2_next_bytes,
                             const void *discard, size_t discard_bytes) {
  if (rows == 0) return cudaSuccess;
  static std::atomic<bool> configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev].load(std::memory_order_acquire)) {
    // setting the attribute twice (two threads racing here) is harmless
    cudaError_t e = configure_attention_kernel();
    if (e != cudaSuccess) return e;
    configured[dev].store(true, std::memory_order_release);
  }
  const int n_items = static_cast<int>(rows / kTokens) * kHeads;
  // Small batches (every query tile fits its own SM): one CTA per query tile.
  const int tile_split = 2 * n_items <= sm_count(dev) ? 1 : 0;
  const int grid = tile_split ? 2 * n_items : (n_items < sm_count(dev) ? n_items : sm_count(dev));
  const void *dp;
  size_t db;
  discard_range(discard, discard_bytes, &dp, &db);
  return launch_pdl(attention_kernel, dim3(grid), dim3(kAttnThreads), kAttnSmem, stream, maps.q,
                    maps.kv, maps.out, n_items, tile_split, l2_next,
                    l2_next_bytes & ~static_cast<size_t>(15), dp, db, status);
}

}  // namespace dv3
