// qkv_attention.cu - the folded QKV projection with RoPE and the attention after it in one
// kernel: one persistent CTA per SM walks (image, head) work items, and each item's q, k and v
// go from the tensor-memory accumulator through the RoPE epilogue straight into the shared-memory
// operand tiles of the attention MMAs, so the 1152-column qkv rows never reach global memory.
// Replaces, for large batches, the launch pair kernels/matmul_qkv_rope_f16_wmma.loom +
// kernels/attention_online_f16_wmma_cf16.loom (src/lib.rs:183-199 records them back to back);
// arithmetic per value is that of gemm_kernel<256, EpiQkvRopeT<true>> followed by
// attention_kernel.
//
// A work item covers the 201 tokens of one head of one image as two 128-row tiles (tile 1 holds
// tokens 128..200; the rows past 200 read x as zero through the per-image tensor maps).
//
// Per item:
//   QKV     A = x rows of the image (two 128-row boxes per 64-wide k-block), B = the head's 192
//           rows of the folded weights (its q, k and v rows, three 64-row boxes), six k-blocks
//           through a two-stage shared-memory ring, then the folded LayerNorm's K=16 aux step
//           (row aux x weight aux); M=128, N=192 MMAs into TMEM columns 256t..256t+191 of tile t.
//   drain   warps 0-7 (tile t = warp / 4, lane quarter = warp % 4, one token row per thread):
//           value = rstd * acc, RoPE on the q and k columns of patch tokens, f16, written with the
//           128-byte swizzle into Q_t (128 x 64), K and V (208 x 64; rows 201..207 zero, the
//           zero-filled rows of tile 1).
//   attention  as attention_kernel: S_t = Q_t K^T (N = 208) over the consumed accumulator
//           columns, softmax by warps 4t..4t+3 with P in TMEM, O_t = P_t V (A from TMEM), O / sum
//           staged in Q_t's rows (dead once S_t is complete) and written by one TMA store per warp.
// Items run one after another (the accumulator and S share TMEM, K and V have one buffer); the
// producer loads the next item's k-blocks while the current item's attention runs.
//
// Roles (352 threads): warp 8 TMA producer; warp 9 lane 0 issues the QKV MMAs and tile 0's
// attention MMAs (warp 9 allocates 512 TMEM columns), warp 10 lane 0 tile 1's attention MMAs;
// warps 0-7 drain, softmax and output (warp 7 holds tile 1 rows 96..127, tokens 224..255, which
// only take part in the drain).
//
// Every wait is bounded; on a timeout the kernel records kErrAttentionWait, raises the CTA's
// abort flag, lets its own copies and MMAs in flight land, frees TMEM and returns.
#include <atomic>

#include "attention_softmax.cuh"
#include "gemm_epilogues.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace dv3 {

namespace {
using namespace attn;
constexpr int kQaThreads = 352;
constexpr int kQaProducer = 8;
constexpr int kQaMma = 9;           // TMEM allocator, QKV and tile 0 issuer; warp 10: tile 1
constexpr int kQaN = 192;           // q, k, v columns of one head
constexpr int kQaBK = 64;           // k-block depth
constexpr int kQaKBlocks = kHidden / kQaBK;  // 6
constexpr int kQaATile = 128 * 128;          // 128 rows x 64 f16
constexpr int kQaBBox = 64 * 128;            // 64 weight rows x 64 f16
constexpr int kQaStage = 2 * kQaATile + 3 * kQaBBox;  // 56 KB
constexpr int kQaStages = 2;
constexpr uint32_t kQaLoadBytes = kQaStage;
constexpr int kQaAuxA = 128 * 32;   // aux step: 128 rows x 16 f16 per tile
constexpr int kQaAuxB = 64 * 32;    // one 64-row weight aux box
constexpr uint32_t kQaAuxBytes = 2 * kQaAuxA + 3 * kQaAuxB;
constexpr int kQaQ = kQaStages * kQaStage;   // Q_0 | Q_1 | K | V
constexpr int kQaKvBytes = kSKeys * 128;
constexpr int kQaK = kQaQ + 2 * kQaATile;
constexpr int kQaV = kQaK + kQaKvBytes;
constexpr int kQaRope = kQaV + kQaKvBytes;
constexpr int kQaRopeBytes = ((EpiQkvRopeT<true>::kRopeBytes + 127) / 128) * 128;
constexpr int kQaBar = kQaRope + kQaRopeBytes;
// 16 mbarriers: full[2], empty[2], qkv_full, qkv_ready, s_full[2], p_full[2], o_full[2],
// tmem_empty[2], drain[2]; then the TMEM slot and the abort flag.
constexpr int kQaSmem = 1024 + kQaBar + 256;
static_assert(kQaStage % 1024 == 0 && kQaQ % 1024 == 0 && kQaK % 1024 == 0 && kQaV % 1024 == 0,
              "swizzle atoms");
static_assert(kQaSmem <= 227 * 1024, "shared memory budget");
}  // namespace

__global__ void __launch_bounds__(kQaThreads, 1)
    qkv_attention_kernel(const __grid_constant__ CUtensorMap tmx,
                         const __grid_constant__ CUtensorMap tmw,
                         const __grid_constant__ CUtensorMap tmxa,
                         const __grid_constant__ CUtensorMap tmwa,
                         const __grid_constant__ CUtensorMap tmo, int n_items,
                         const float2 *rowstat, const float *rope_cos, const float *rope_sin,
                         const void *l2_next, size_t l2_next_bytes, const void *l2_next2,
                         size_t l2_next2_bytes, const void *discard, size_t discard_bytes,
                         uint32_t *status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t *smem = smem_raw + pad;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kQaBar);
  uint64_t *empty = full + 2;
  uint64_t *qkv_full = full + 4;
  uint64_t *qkv_ready = full + 5;
  uint64_t *s_full = full + 6;
  uint64_t *p_full = full + 8;
  uint64_t *o_full = full + 10;
  uint64_t *tmem_empty = full + 12;
  uint64_t *drain = full + 14;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(full + 16);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int count = static_cast<int>(blockIdx.x) < n_items
                        ? (n_items - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                        : 0;
  auto item_of = [&](int k) { return static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&tmem_empty[i], 128);
      mbar_init(&drain[i], 1);
    }
    mbar_init(qkv_full, 1);
    mbar_init(qkv_ready, 256);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kQaProducer && lane == 0) {
    tma_prefetch_map(&tmx);
    tma_prefetch_map(&tmw);
    tma_prefetch_map(&tmxa);
    tma_prefetch_map(&tmwa);
    tma_prefetch_map(&tmo);
  }
  if (warp == kQaMma) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // the RoPE tables (weights only: may overlap the previous kernel)
  const EpiQkvRopeT<true> rope{nullptr, rope_cos, rope_sin, rowstat};
  rope.init(smem + kQaRope, threadIdx.x, kQaThreads);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent launch: the producer waits for the previous kernel before its first
  // load, the drain warps before their first read of rowstat; the MMA issuers consume only what
  // those two roles bring.
  if (warp == kQaProducer && lane == 1) {
    if (l2_next) l2_prefetch_share(l2_next, l2_next_bytes);
    if (l2_next2) l2_prefetch_share(l2_next2, l2_next2_bytes);
  }
  if (warp == kQaProducer && lane >= 2 && discard) {
    pdl_wait();
    l2_discard_share(discard, discard_bytes, lane - 2, 30);
  }

  if (warp == kQaProducer) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, armed = 0, last_parity = 0;
      bool ok = true;
      bool first = true;
      auto next_stage = [&](uint32_t bytes) -> uint8_t * {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
          report(status, kErrAttentionWait);
          *abort_flag = 1;
          ok = false;
          return nullptr;
        }
        if (first) {  // the previous kernel's x and row aux are complete from here on
          pdl_wait();
          pdl_trigger();
          first = false;
        }
        mbar_arrive_expect_tx(&full[stage], bytes);
        return smem + stage * kQaStage;
      };
      auto advance = [&]() {
        armed |= 1u << stage;
        last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == kQaStages) {
          stage = 0;
          phase ^= 1u;
        }
      };
      for (int k = 0; ok && k < count; ++k) {
        const int item = item_of(k);
        const int img = item / kHeads, head = item % kHeads;
        for (int kb = 0; kb < kQaKBlocks; ++kb) {
          uint8_t *st = next_stage(kQaLoadBytes);
          if (!st) break;
          tma_load_3d(st, &tmx, &full[stage], kb * kQaBK, 0, img);
          tma_load_3d(st + kQaATile, &tmx, &full[stage], kb * kQaBK, 128, img);
          for (int s = 0; s < 3; ++s)
            tma_load_2d(st + 2 * kQaATile + s * kQaBBox, &tmw, &full[stage], kb * kQaBK,
                        s * kHidden + head * 64);
          advance();
        }
        if (!ok) break;
        uint8_t *st = next_stage(kQaAuxBytes);  // the folded LayerNorm's K=16 step
        if (!st) break;
        tma_load_3d(st, &tmxa, &full[stage], 0, 0, img);
        tma_load_3d(st + kQaAuxA, &tmxa, &full[stage], 0, 128, img);
        for (int s = 0; s < 3; ++s)
          tma_load_2d(st + 2 * kQaAuxA + s * kQaAuxB, &tmwa, &full[stage], 0,
                      s * kHidden + head * 64);
        advance();
      }
      // Copies still in flight (only after an abort) land before shared memory is released.
      for (int s = 0; s < kQaStages; ++s)
        if ((armed >> s) & 1u) mbar_drain(&full[s], (last_parity >> s) & 1u);
    }
  } else if (warp == kQaMma || warp == kQaMma + 1) {
    if (lane == 0) {
      const int t = warp - kQaMma;
      constexpr uint32_t idesc_qkv = idesc_f16_f32(128, kQaN, false);
      constexpr uint32_t idesc_s = idesc_f16_f32(128, kSKeys, false);
      constexpr uint32_t idesc_o = idesc_f16_f32(128, 64, true);
      const uint32_t d_s = tmem + t * kTileCols, d_o = d_s + kOCol;
      const uint8_t *qt = smem + kQaQ + t * kQaATile;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int k = 0; ok && k < count; ++k) {
        const uint32_t par = k & 1;
        if (t == 0) {
          // QKV of this item: both tiles' accumulators free (the previous item's O read out)
          ok = mbar_wait(&tmem_empty[0], par ^ 1u, abort_flag) &&
               mbar_wait(&tmem_empty[1], par ^ 1u, abort_flag);
          if (!ok) break;
          tc_fence_after();
          for (int kb = 0; ok && kb <= kQaKBlocks; ++kb) {
            if (!mbar_wait(&full[stage], phase, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + stage * kQaStage);
            if (kb < kQaKBlocks) {
              const uint64_t bdesc = sw128_desc(sa + 2 * kQaATile);
#pragma unroll
              for (int tt = 0; tt < 2; ++tt) {
                const uint64_t adesc = sw128_desc(sa + tt * kQaATile);
#pragma unroll
                for (int kk = 0; kk < kQaBK / 16; ++kk)
                  umma_f16(tmem + tt * kTileCols, adesc + 2 * kk, bdesc + 2 * kk, idesc_qkv,
                           (kb | kk) != 0 ? 1u : 0u);
              }
            } else {  // aux step: -mean s + r c into both accumulators
#pragma unroll
              for (int tt = 0; tt < 2; ++tt)
                umma_f16(tmem + tt * kTileCols, sw32_desc(sa + tt * kQaAuxA),
                         sw32_desc(sa + 2 * kQaAuxA), idesc_qkv, 1u);
            }
            umma_commit(&empty[stage]);
            if (++stage == kQaStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit(qkv_full);
        }
        // S_t once every drain warp has written Q, K and V (and read the accumulators)
        ok = mbar_wait(qkv_ready, par, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint64_t qd = sw128_desc(smem_u32(qt));
        const uint64_t kd = sw128_desc(smem_u32(smem + kQaK));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_f16(d_s, qd + 2 * kk, kd + 2 * kk, idesc_s, kk > 0);
        umma_commit(&s_full[t]);
        ok = mbar_wait(&p_full[t], par, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t vb = smem_u32(smem + kQaV);
#pragma unroll
        for (int kk = 0; kk < kSKeys / 16; ++kk)
          umma_f16_ts(d_o, d_s + 8 * kk, sw128_desc(vb + kk * 2048), idesc_o, kk > 0);
        umma_commit(&o_full[t]);
      }
      if (!ok) {
        report(status, kErrAttentionWait);
        *abort_flag = 1;
      }
      umma_commit(&drain[t]);  // every MMA this thread issued has completed before TMEM is freed
      mbar_drain(&drain[t], 0);
    }
  } else {
    pdl_wait();  // rowstat and the output rows: the previous kernel is complete from here on
    const int t = warp >> 2, q = warp & 3;
    const int r = q * 32 + lane;   // row within the tile == TMEM lane
    const int tok = t * 128 + r;   // token of this thread's row
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t tl = tmem + lane_off + t * kTileCols;
    const bool active = !(t == 1 && q == 3);  // warp-uniform: tile 1 rows 96..127 are padding
    uint8_t *qrow = smem + kQaQ + t * kQaATile + r * 128;
    uint8_t *krow = smem + kQaK + tok * 128;
    uint8_t *vrow = smem + kQaV + tok * 128;
    uint8_t *stg = smem + kQaQ + t * kQaATile + q * (kOutBox * 128);  // output staging in Q_t
    const int sw = r & 7;  // == tok & 7
    const bool in_kv = tok < kSKeys;
    const bool patch = tok >= kPrefix && tok < kTokens;
    const int p = patch ? tok - kPrefix : 0;
    const float *tab = reinterpret_cast<const float *>(smem + kQaRope);
    constexpr int kPad = EpiQkvRopeT<true>::kPad, kTab = EpiQkvRopeT<true>::kTab;
    const float *cy = tab + (p / 14) * kPad, *sy = tab + kTab + (p / 14) * kPad;
    const float *cx = tab + 2 * kTab + (p % 14) * kPad, *sx = tab + 3 * kTab + (p % 14) * kPad;
    for (int k = 0; k < count; ++k) {
      const uint32_t par = k & 1;
      const int item = item_of(k);
      const int img = item / kHeads, head = item % kHeads;
      const float rs = tok < kTokens ? __ldg(&rowstat[img * kTokens + tok].x) : 0.f;
      if (!__all_sync(0xffffffffu, mbar_wait(qkv_full, par, abort_flag))) {
        if (lane == 0) {
          report(status, kErrAttentionWait);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      // The previous item's output store has read this warp's staging rows of Q_t.
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
#pragma unroll 1
      for (int part = 0; part < 3; ++part) {  // q, k, v columns of the head
        uint32_t ra[32], rb[32];
        tmem_load32x2(tl + part * 64, ra, tl + part * 64 + 32, rb);
        float lo[32], hi[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          lo[i] = rs * u2f(ra[i]);
          hi[i] = rs * u2f(rb[i]);
        }
        if (patch && part < 2) {  // q and k of patch tokens rotate (EpiQkvRopeT)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float cs = i < 16 ? cy[i] : cx[i - 16];
            const float sn = i < 16 ? sy[i] : sx[i - 16];
            const float a = lo[i], b = hi[i];
            lo[i] = a * cs - b * sn;
            hi[i] = b * cs + a * sn;
          }
        }
        uint8_t *row = part == 0 ? qrow : part == 1 ? krow : vrow;
        if (part == 0 || in_kv) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            *reinterpret_cast<uint4 *>(row + ((j ^ sw) << 4)) = pack8(lo, j);
            *reinterpret_cast<uint4 *>(row + (((4 + j) ^ sw) << 4)) = pack8(hi, j);
          }
        }
      }
      fence_proxy_async_smem();  // the tensor cores read Q, K and V through the async proxy
      tc_fence_before();
      mbar_arrive(qkv_ready);

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
        stage_output_row(stg + lane * 128, lane, o0, o1, 1.0f / sum);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&tmo, stg, head * 64, t * 128 + q * 32, img);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait<0>();  // output stores complete before the CTA retires
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kQaMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool make_qkv_attention_maps(const void *x, uint32_t rows, const void *wf, const void *row_aux,
                             const void *w_aux, const void *out, QkvAttentionMaps *maps,
                             std::string *err) {
  const uint32_t n_images = rows / kTokens;
  return encode_map_f16_images(&maps->x, x, kHidden, n_images, 128, err) &&
         encode_map_f16(&maps->w, wf, kHidden, kQkv, 64, 64, err) &&
         encode_map_f16_images_box(&maps->x_aux, row_aux, 16, n_images, 16, 128, 32, err) &&
         encode_map_f16_swizzled(&maps->w_aux, w_aux, 16, kQkv, 16, 64, 32, err) &&
         encode_map_f16_images(&maps->out, out, kHidden, n_images, kOutBox, err);
}

cudaError_t launch_qkv_attention(const QkvAttentionMaps &maps, uint32_t rows,
                                 const float2 *rowstat, const float *rope_cos,
                                 const float *rope_sin, uint32_t *status, cudaStream_t stream,
                                 const void *l2_next, size_t l2_next_bytes, const void *l2_next2,
                                 size_t l2_next2_bytes, const void *discard,
                                 size_t discard_bytes) {
  if (rows == 0) return cudaSuccess;
  static std::atomic<bool> configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev].load(std::memory_order_acquire)) {
    // setting the attribute twice (two threads racing here) is harmless
    cudaError_t e = cudaFuncSetAttribute(qkv_attention_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, kQaSmem);
    if (e != cudaSuccess) return e;
    configured[dev].store(true, std::memory_order_release);
  }
  const int n_items = static_cast<int>(rows / kTokens) * kHeads;
  const int grid = n_items < sm_count(dev) ? n_items : sm_count(dev);
  const void *dp;
  size_t db;
  discard_range(discard, discard_bytes, &dp, &db);
  return launch_pdl(qkv_attention_kernel, dim3(grid), dim3(kQaThreads), kQaSmem, stream, maps.x,
                    maps.w, maps.x_aux, maps.w_aux, maps.out, n_items, rowstat, rope_cos,
                    rope_sin, l2_next, l2_next_bytes & ~static_cast<size_t>(15), l2_next2,
                    l2_next2_bytes & ~static_cast<size_t>(15), dp, db, status);
}

}  // namespace dv3
