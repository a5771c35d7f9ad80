// attention.cu - per-(image, head, 128-query tile) attention on tcgen05 tensor cores.
// Replaces kernels/attention_online_f16_wmma_cf16.loom (6 heads x 64, 201 tokens, scale 0.125).
//
// All 201 keys of an image fit one tile, so the softmax is exact in one pass instead of online:
//   1. TMA brings Q (128 rows) and K, V (256 rows: this image's 201 plus following rows, masked)
//      of this head out of the fused QKV rows into 128-byte-swizzled shared memory.
//   2. S = Q K^T: 4 tcgen05.mma (M=128, N=208, K=16) into TMEM columns 0..207, f32.
//   3. 8 warps: the two warps of each TMEM lane quarter split a query row's keys (0..127 and
//      128..207). Pass 1 takes the row max over the 201 valid keys (the halves meet in shared
//      memory); pass 2 forms w = exp(0.125 s - 0.125 max) (one FFMA and the hardware exp2), sums
//      w in f32 and writes P = f16(w)
//      (keys >= 201 zero) into shared memory in the K-major layout the MMA reads: keys 0..191 as
//      three 128-byte-swizzled 64-key blocks over the now dead Q and K tiles, keys 192..207 as a
//      32-byte-swizzled 16-key block.
//   4. O = P V: 13 tcgen05.mma (M=128, N=64, K=16 keys; V is the MN-major B operand) into TMEM
//      columns 0..63 (S is consumed by then). Each thread divides its 32 of the 64 output columns
//      by the row sum, rounds to f16 and stores them to out[token][64h..64h+63].
// The probabilities are rounded to f16 before PV and the normaliser is the f32 sum of the
// unrounded weights, as in the reference kernel (:214-216). Query rows past the image's 201 are
// computed and dropped; rows past the batch read as zeros (TMA out-of-bounds fill).
// Footprint: 256 TMEM columns and ~89 KB of shared memory, so two CTAs share an SM and one CTA's
// loads and MMAs overlap the other's softmax.
#include "kernels.h"
#include "sm100.cuh"

namespace dv3 {

namespace {
constexpr int kAttnThreads = 256;
constexpr int kQ = 0;            // 128 x 64 f16 (16 KB); P keys 0..63 afterwards
constexpr int kK = 16384;        // 256 x 64 f16 (32 KB); P keys 64..191 afterwards
constexpr int kV = 49152;        // 256 x 64 f16 (32 KB)
constexpr int kPTail = 81920;    // 128 x 16 f16, 32-byte swizzle (4 KB): P keys 192..207
constexpr int kRed = 86016;      // [2 halves][128 rows] max, then [2][128] sum (2 KB)
constexpr int kBar = 88064;      // 3 mbarriers, TMEM slot, abort flag
constexpr int kAttnSmem = 1024 + kBar + 64;
constexpr int kValidKeys = kTokens;  // 201
constexpr int kSKeys = 208;          // S columns computed (201 rounded up to 16)
constexpr int kTmemCols = 256;

// K-major 32-byte-swizzled tile descriptor: 32-byte rows (16 f16), 8-row groups 256 bytes apart,
// layout type 6 (32-byte swizzle).
__device__ __forceinline__ uint64_t sw32_desc(uint32_t smem_addr) {
  return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) | (1ull << 16) |
         (static_cast<uint64_t>(256 >> 4) << 32) | (1ull << 46) | (6ull << 61);
}
}  // namespace

__global__ void __launch_bounds__(kAttnThreads, 2)
    attention_kernel(const __grid_constant__ CUtensorMap tm, int rows, __half *out,
                     uint32_t *status) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t *smem = smem_raw + pad;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBar);  // 0 loads, 1 S ready, 2 O ready
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  float *red_max = reinterpret_cast<float *>(smem + kRed);
  float *red_sum = red_max + 256;

  const int qt = blockIdx.x, head = blockIdx.y, img = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int quarter = warp & 3, half = warp >> 2;
  const int tok0 = img * kTokens;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_map(&tm);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // the QKV rows of the previous kernel are complete from here on
  pdl_trigger();

  // Thread 0 drives the pipeline and alone polls the mbarriers (bounded waits); the other warps
  // sleep in __syncthreads, leaving issue slots to the co-resident CTA.
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bars[0], 5 * 16384);
    const int qx = head * 64, kx = kHidden + head * 64, vx = 2 * kHidden + head * 64;
    tma_load_2d(smem + kQ, &tm, &bars[0], qx, tok0 + qt * 128);
    tma_load_2d(smem + kK, &tm, &bars[0], kx, tok0);
    tma_load_2d(smem + kK + 16384, &tm, &bars[0], kx, tok0 + 128);
    tma_load_2d(smem + kV, &tm, &bars[0], vx, tok0);
    tma_load_2d(smem + kV + 16384, &tm, &bars[0], vx, tok0 + 128);
    bool ok = mbar_wait(&bars[0], 0, abort_flag);
    if (ok) {
      tc_fence_after();
      const uint64_t qd = sw128_desc(smem_u32(smem + kQ));
      const uint64_t kd = sw128_desc(smem_u32(smem + kK));
      constexpr uint32_t idesc = idesc_f16_f32(128, kSKeys, false);
#pragma unroll
      for (int k = 0; k < 4; ++k) umma_f16(tmem, qd + 2 * k, kd + 2 * k, idesc, k > 0);
      umma_commit(&bars[1]);
      ok = mbar_wait(&bars[1], 0, abort_flag);
    }
    if (!ok) {
      report(status, kErrAttentionWait);
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();  // S is in TMEM (or the kernel is unwinding)
  tc_fence_after();

  const int r = quarter * 32 + lane;  // query row in the tile == TMEM lane
  const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
  // Key chunks of 32 owned by this half: 0..3 (keys 0..127) or 4..6 (keys 128..223, of which
  // 128..207 exist in S and 128..200 are valid).
  const int c_begin = half ? 4 : 0, c_end = half ? 7 : 4;
  const bool ok = !*abort_flag;
  if (ok) {
    float mx = -INFINITY;
#pragma unroll 1
    for (int c = c_begin; c < c_end; ++c) {
      uint32_t v[32];
      tmem_load32(trow + c * 32, v);
      if (c < 6) {
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, __uint_as_float(v[i]));
      } else {  // keys 192..223: only 192..200 are valid
#pragma unroll
        for (int i = 0; i < kValidKeys - 192; ++i) mx = fmaxf(mx, __uint_as_float(v[i]));
      }
    }
    red_max[half * 128 + r] = mx;
  }
  __syncthreads();
  float sum = 0.f;
  if (ok) {
    // w = exp(0.125 s - 0.125 max) = 2^(s c - max c), c = 0.125 log2(e)
    constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;
    const float mxc = fmaxf(red_max[r], red_max[128 + r]) * kScaleLog2;
#pragma unroll 1
    for (int c = c_begin; c < c_end; ++c) {
      uint32_t v[32];
      tmem_load32(trow + c * 32, v);
      float p[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int key = c * 32 + i;
        p[i] = key < kValidKeys ? ex2_approx(fmaf(__uint_as_float(v[i]), kScaleLog2, -mxc)) : 0.f;
        sum += p[i];
      }
      if (c < 6) {  // keys c*32 .. c*32+31 into 128-byte-swizzled block c/2 (over Q and K)
        uint8_t *blk = smem + (c / 2) * 16384 + (r / 8) * 1024 + (r % 8) * 128;
        const int chunk0 = (c % 2) * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 val = make_uint4(pack_half2(p[8 * j + 0], p[8 * j + 1]),
                                       pack_half2(p[8 * j + 2], p[8 * j + 3]),
                                       pack_half2(p[8 * j + 4], p[8 * j + 5]),
                                       pack_half2(p[8 * j + 6], p[8 * j + 7]));
          *reinterpret_cast<uint4 *>(blk + (((chunk0 + j) ^ (r % 8)) * 16)) = val;
        }
      } else {  // keys 192..207 into the 32-byte-swizzled tail block
        uint8_t *rowp = smem + kPTail + (r / 8) * 256 + (r % 8) * 32;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const uint4 val = make_uint4(pack_half2(p[8 * j + 0], p[8 * j + 1]),
                                       pack_half2(p[8 * j + 2], p[8 * j + 3]),
                                       pack_half2(p[8 * j + 4], p[8 * j + 5]),
                                       pack_half2(p[8 * j + 6], p[8 * j + 7]));
          *reinterpret_cast<uint4 *>(rowp + ((j ^ ((r % 8) >> 2)) * 16)) = val;
        }
      }
    }
    red_sum[half * 128 + r] = sum;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();

  if (threadIdx.x == 0 && !*abort_flag) {
    tc_fence_after();
    const uint32_t pbase = smem_u32(smem);
    const uint32_t vbase = smem_u32(smem + kV);
    constexpr uint32_t idesc = idesc_f16_f32(128, 64, true);
#pragma unroll
    for (int kk = 0; kk < 12; ++kk) {
      const uint64_t pd = sw128_desc(pbase + (kk / 4) * 16384 + (kk % 4) * 32);
      umma_f16(tmem, pd, sw128_desc(vbase + kk * 2048), idesc, kk > 0);
    }
    umma_f16(tmem, sw32_desc(smem_u32(smem + kPTail)), sw128_desc(vbase + 12 * 2048), idesc, 1);
    umma_commit(&bars[2]);
    if (!mbar_wait(&bars[2], 0, abort_flag)) {
      report(status, kErrAttentionWait);
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();  // O is in TMEM (or the kernel is unwinding)
  tc_fence_after();

  if (!*abort_flag) {
    uint32_t o[32];
    tmem_load32(trow + half * 32, o);
    const int q_local = qt * 128 + r;
    const int token = tok0 + q_local;
    if (q_local < kValidKeys && token < rows) {
      const float inv = 1.0f / (red_sum[r] + red_sum[128 + r]);
      uint4 *dst =
          reinterpret_cast<uint4 *>(out + static_cast<size_t>(token) * kHidden + head * 64 + half * 32);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        dst[j] = make_uint4(pack_half2(__uint_as_float(o[8 * j + 0]) * inv, __uint_as_float(o[8 * j + 1]) * inv),
                            pack_half2(__uint_as_float(o[8 * j + 2]) * inv, __uint_as_float(o[8 * j + 3]) * inv),
                            pack_half2(__uint_as_float(o[8 * j + 4]) * inv, __uint_as_float(o[8 * j + 5]) * inv),
                            pack_half2(__uint_as_float(o[8 * j + 6]) * inv, __uint_as_float(o[8 * j + 7]) * inv));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

bool make_attention_map(const void *qkv, uint32_t rows, CUtensorMap *map, std::string *err) {
  return encode_map_f16(map, qkv, kQkv, rows, 64, 128, err);
}

cudaError_t configure_attention_kernel() {
  return cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kAttnSmem);
}

cudaError_t launch_attention(const CUtensorMap &map, uint32_t rows, __half *out, uint32_t *status,
                             cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = configure_attention_kernel();
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const dim3 grid(2, 6, rows / kTokens);
  return launch_pdl(attention_kernel, grid, dim3(kAttnThreads), kAttnSmem, stream, map,
                    static_cast<int>(rows), out, status);
}

}  // namespace dv3
