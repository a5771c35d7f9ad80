// gemm.cu - persistent, warp-specialised tcgen05 GEMM for the five projections of the forward,
// each with its epilogue fused:
//   Patch     x[token(p)] = f16(A W^T + b)                 kernels/matmul_bias_f16_wmma.loom
//                                                          + kernels/embed_scatter_f32.loom
//   QkvRope   qkv = f16(rope(A W^T + b))                   kernels/matmul_qkv_rope_f16_wmma.loom
//   Resid*    x = f16(x + lambda (A W^T + b))              kernels/matmul_resid_f16_wmma.loom
//   SwiGLU    act = f16(silu(A Wg^T + bg) (A Wu^T + bu))   kernels/matmul_swiglu_f16_wmma.loom
//
// Layout: A [M][K] f16 activations and W [N][K] f16 weights, both K-major, are streamed by TMA
// in 128-row x 64-column boxes with the 128-byte swizzle into a ring of shared-memory stages.
// One thread issues tcgen05.mma (M=128, N=BN, K=16 steps) into an f32 accumulator in TMEM;
// TMEM holds two accumulators so the epilogue of tile i overlaps the MMAs of tile i+1.
//
// Warp roles (320 threads): warp 0 lane 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer
// (lane 0), warps 2-9 = epilogue. An epilogue warp may read only TMEM lanes 32*(w%4)..+31, so
// two warps share each lane quarter: warps 2-5 take the left half of the tile's columns and
// warps 6-9 the right half. Each epilogue thread owns one output row and walks its half in
// 32-column chunks (tcgen05.ld 32x32b.x32). Two warps per SM sub-partition hide the latency of
// the epilogue arithmetic, which otherwise limits the whole GEMM.
//
// Tiles are walked m-major with the N tile fastest (tile t -> m = t / n_tiles, n = t % n_tiles)
// by a grid of min(tiles, SMs) persistent CTAs, so the CTAs working at one time share A rows
// through L2.
#include "kernels.h"
#include "sm100.cuh"

namespace dv3 {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpilogueWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpilogueWarps;  // 320

template <int BN>
struct GemmCfg {
  static constexpr int kA = BM * BK * 2;  // 16 KB
  static constexpr int kB = BN * BK * 2;
  static constexpr int kStage = kA + kB;
  static constexpr int kStages = (BN >= 256) ? 4 : 6;
  static constexpr int kTiles = kStages * kStage;
  static constexpr int kTmemCols = (2 * BN <= 256) ? 256 : 512;
  static constexpr int kBarBytes = (2 * kStages + 4) * 8 + 16;
  static constexpr int kExtraOffset = kTiles + ((kBarBytes + 127) / 128) * 128;
};

__device__ __forceinline__ float u2f(uint32_t v) { return __uint_as_float(v); }

__device__ __forceinline__ void store_half32(__half *dst, const float (&v)[32]) {
  uint4 *d = reinterpret_cast<uint4 *>(dst);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    d[j] = make_uint4(pack_half2(v[8 * j + 0], v[8 * j + 1]), pack_half2(v[8 * j + 2], v[8 * j + 3]),
                      pack_half2(v[8 * j + 4], v[8 * j + 5]), pack_half2(v[8 * j + 6], v[8 * j + 7]));
  }
}

// 32 consecutive floats at an address shared by the whole warp (one broadcast per float4).
__device__ __forceinline__ void load_bias32(const float *b, float (&v)[32]) {
  const float4 *p = reinterpret_cast<const float4 *>(b);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 q = __ldg(p + j);
    v[4 * j + 0] = q.x;
    v[4 * j + 1] = q.y;
    v[4 * j + 2] = q.z;
    v[4 * j + 3] = q.w;
  }
}

// ---------------------------------------------------------------------------------------------
// Epilogues. run<COLS>() processes COLS accumulator columns starting at `taddr` (this warp's
// lane quarter) that belong to output columns n0..n0+COLS-1; `row` is this thread's output row
// (it may be >= M on the last M tile: TMEM loads still run, because tcgen05.ld is
// warp-collective, but global accesses are skipped). kSmem bytes of shared memory are set up by
// init() (all threads, before the first barrier) and passed to run().
// ---------------------------------------------------------------------------------------------
struct EpiPatch {
  const float *bias;
  __half *x;
  static constexpr int kSmem = 0;
  __device__ void init(uint8_t *, int, int) const {}
  template <int COLS>
  __device__ void run(uint32_t taddr, int row, int n0, int M, const uint8_t *) const {
    const bool ok = row < M;
    const int token = (row / kPatches) * kTokens + kPrefix + row % kPatches;
#pragma unroll 1
    for (int c = 0; c < COLS; c += 32) {
      uint32_t r[32];
      tmem_load32(taddr + c, r);
      float v[32];
      load_bias32(bias + n0 + c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += u2f(r[i]);
      if (ok) store_half32(x + static_cast<size_t>(token) * kHidden + n0 + c, v);
    }
  }
};

// RoPE angles depend only on (position along one axis, frequency index j < 16): channel c of
// patch p uses row position p/14 when c%32 < 16 and column position p%14 otherwise, frequency
// c%16 (src/weights.rs:127-144). init() copies those 14x16 cos/sin values of each axis out of
// the packed [196][64] table into shared memory (rows padded to 17 floats so that the 32 rows
// of a warp fall in distinct banks); the packed entries for channels c and c+32 are equal.
struct EpiQkvRope {
  const float *bias;
  const float *cosv;
  const float *sinv;
  __half *out;
  static constexpr int kPad = 17;
  static constexpr int kTab = 14 * kPad;                  // floats per (axis, function)
  static constexpr int kSmem = 4 * kTab * sizeof(float);  // cos_y, sin_y, cos_x, sin_x
  __device__ void init(uint8_t *smem, int tid, int nthreads) const {
    float *t = reinterpret_cast<float *>(smem);
    for (int i = tid; i < 4 * 14 * 16; i += nthreads) {
      const int which = i / 224, pos = (i / 16) % 14, j = i % 16;
      // axis 0 (rows): patch pos*14, channel j; axis 1 (columns): patch pos, channel 16+j
      const int src = (which < 2) ? (pos * 14) * 64 + j : pos * 64 + 16 + j;
      t[which * kTab + pos * kPad + j] = __ldg(((which & 1) ? sinv : cosv) + src);
    }
  }
  template <int COLS>
  __device__ void run(uint32_t taddr, int row, int n0, int M, const uint8_t *smem) const {
    static_assert(COLS % 64 == 0, "a thread owns whole heads");
    const bool ok = row < M;
    const int t = row % kTokens;
    const bool patch_row = t >= kPrefix;
    const int p = patch_row ? t - kPrefix : 0;
    const float *tab = reinterpret_cast<const float *>(smem);
    const float *cy = tab + (p / 14) * kPad, *sy = tab + kTab + (p / 14) * kPad;
    const float *cx = tab + 2 * kTab + (p % 14) * kPad, *sx = tab + 3 * kTab + (p % 14) * kPad;
#pragma unroll 1
    for (int h = 0; h < COLS; h += 64) {
      uint32_t ra[32], rb[32];
      tmem_load32x2(taddr + h, ra, taddr + h + 32, rb);
      const int col = n0 + h;  // first column of this 64-wide head
      float lo[32], hi[32];
      load_bias32(bias + col, lo);
      load_bias32(bias + col + 32, hi);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        lo[i] += u2f(ra[i]);
        hi[i] += u2f(rb[i]);
      }
      if (patch_row && col < 2 * kHidden) {  // q and k columns of patch tokens rotate
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float c = i < 16 ? cy[i] : cx[i - 16];
          const float s = i < 16 ? sy[i] : sx[i - 16];
          const float a = lo[i], b = hi[i];
          lo[i] = a * c - b * s;
          hi[i] = b * c + a * s;
        }
      }
      if (ok) {
        __half *dst = out + static_cast<size_t>(row) * kQkv + col;
        store_half32(dst, lo);
        store_half32(dst + 32, hi);
      }
    }
  }
};

struct EpiResid {
  const float *bias;
  const float *lambda;
  __half *x;
  static constexpr int kSmem = 0;
  __device__ void init(uint8_t *, int, int) const {}
  template <int COLS>
  __device__ void run(uint32_t taddr, int row, int n0, int M, const uint8_t *) const {
    const bool ok = row < M;
#pragma unroll 1
    for (int c = 0; c < COLS; c += 32) {
      uint32_t r[32];
      tmem_load32(taddr + c, r);
      if (ok) {
        float b[32], l[32];
        load_bias32(bias + n0 + c, b);
        load_bias32(lambda + n0 + c, l);
        __half *xr = x + static_cast<size_t>(row) * kHidden + n0 + c;
        const uint4 *src = reinterpret_cast<const uint4 *>(xr);
        float v[32];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 q = src[j];
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = unpack_half2(w[e]);
            v[8 * j + 2 * e] = f.x;
            v[8 * j + 2 * e + 1] = f.y;
          }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += l[i] * (u2f(r[i]) + b[i]);
        store_half32(xr, v);
      }
    }
  }
};

struct EpiSwiGLU {
  const float *bias;  // packed like the weight rows
  __half *act;
  static constexpr int kSmem = 0;
  __device__ void init(uint8_t *, int, int) const {}
  template <int COLS>
  __device__ void run(uint32_t taddr, int row, int n0, int M, const uint8_t *) const {
    static_assert(COLS % 128 == 0, "a thread owns whole 64 gate + 64 up groups");
    const bool ok = row < M;
#pragma unroll 1
    for (int g = 0; g < COLS; g += 128) {
#pragma unroll 1
      for (int half = 0; half < 64; half += 32) {
        uint32_t rg[32], ru[32];
        tmem_load32x2(taddr + g + half, rg, taddr + g + 64 + half, ru);
        float gv[32], uv[32];
        load_bias32(bias + n0 + g + half, gv);
        load_bias32(bias + n0 + g + 64 + half, uv);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float a = gv[i] + u2f(rg[i]);
          const float u = uv[i] + u2f(ru[i]);
          gv[i] = __fdividef(a, 1.0f + __expf(-a)) * u;  // silu(a) * u
        }
        if (ok) store_half32(act + static_cast<size_t>(row) * kMlp + (n0 + g) / 2 + half, gv);
      }
    }
  }
};

template <int BN, class Epi>
__host__ __device__ constexpr int gemm_smem_bytes() {
  return 1024 + GemmCfg<BN>::kExtraOffset + Epi::kSmem;
}

// ---------------------------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------------------------
template <int BN, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                int M, int n_tiles_n, int k_blocks, Epi epi, uint32_t *status) {
  using C = GemmCfg<BN>;
  static_assert(gemm_smem_bytes<BN, Epi>() <= 227 * 1024, "shared memory budget");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t *smem = smem_raw + pad;
  uint8_t *tiles = smem;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::kTiles);
  uint64_t *empty = full + C::kStages;
  uint64_t *tfull = empty + C::kStages;
  uint64_t *tempty = tfull + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(tempty + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  uint8_t *extra = smem + C::kExtraOffset;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * kEpilogueWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  epi.init(extra, threadIdx.x, kGemmThreads);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = ((M + BM - 1) / BM) * n_tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int m0 = (tile / n_tiles_n) * BM;
        const int n0 = (tile % n_tiles_n) * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            report(status, kErrProducerWait);
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t *a = tiles + stage * C::kStage;
          mbar_arrive_expect_tx(&full[stage], C::kStage);
          tma_load_2d(a, &tmA, &full[stage], kb * BK, m0);
          tma_load_2d(a + C::kA, &tmB, &full[stage], kb * BK, n0);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(BM, BN, false);
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
          const uint64_t bdesc = sw128_desc(a_addr + C::kA);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
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
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const bool waited = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      if (!__all_sync(0xffffffffu, waited)) {
        if (lane == 0) {
          report(status, kErrEpilogueWait);
          *abort_flag = 1;
        }
        break;
      }
      tc_fence_after();
      const int m0 = (tile / n_tiles_n) * BM;
      const int n0 = (tile % n_tiles_n) * BN + half * kCols;
      epi.template run<kCols>(
          tmem_base + lane_base + static_cast<uint32_t>(acc * BN + half * kCols), m0 + row_in_tile,
          n0, M, extra);
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
GemmShape gemm_shape(GemmOp op) {
  switch (op) {
    case GemmOp::Patch: return {128, kHidden, kPatchK};
    case GemmOp::QkvRope: return {128, kQkv, kHidden};
    case GemmOp::Resid384: return {128, kHidden, kHidden};
    case GemmOp::Resid1536: return {128, kHidden, kMlp};
    case GemmOp::SwiGLU: return {256, kGateUp, kHidden};
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
  }
  return "?";
}

bool make_gemm_maps(GemmOp op, const void *a, uint32_t rows, const void *w, GemmMaps *maps,
                    std::string *err) {
  const GemmShape s = gemm_shape(op);
  return encode_map_f16(&maps->a, a, s.k, rows, BK, BM, err) &&
         encode_map_f16(&maps->b, w, s.k, s.n, BK, s.bn, err);
}

template <int BN, class Epi>
static cudaError_t configure_one() {
  return cudaFuncSetAttribute(gemm_kernel<BN, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              gemm_smem_bytes<BN, Epi>());
}

template <int BN, class Epi>
static cudaError_t launch_one(const GemmMaps &maps, uint32_t rows, int n, int k, const Epi &epi,
                              uint32_t *status, cudaStream_t stream) {
  static bool configured[64] = {};  // per template instance and device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = configure_one<BN, Epi>();
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int n_tiles_n = n / BN;
  const int tiles = static_cast<int>((rows + BM - 1) / BM) * n_tiles_n;
  const int grid = tiles < sm_count(dev) ? tiles : sm_count(dev);
  gemm_kernel<BN, Epi><<<grid, kGemmThreads, gemm_smem_bytes<BN, Epi>(), stream>>>(
      maps.a, maps.b, static_cast<int>(rows), n_tiles_n, k / BK, epi, status);
  return cudaGetLastError();
}

// Set the shared-memory limits of every GEMM instance on the current device (done at load, so
// that graph capture never meets a first-use attribute call).
cudaError_t configure_gemm_kernels() {
  cudaError_t e;
  if ((e = configure_one<128, EpiPatch>()) != cudaSuccess) return e;
  if ((e = configure_one<128, EpiQkvRope>()) != cudaSuccess) return e;
  if ((e = configure_one<128, EpiResid>()) != cudaSuccess) return e;
  if ((e = configure_one<256, EpiSwiGLU>()) != cudaSuccess) return e;
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
      return launch_one<128>(maps, rows, s.n, s.k, EpiPatch{args.bias, args.out}, status, stream);
    case GemmOp::QkvRope:
      return launch_one<128>(maps, rows, s.n, s.k,
                             EpiQkvRope{args.bias, args.rope_cos, args.rope_sin, args.out},
                             status, stream);
    case GemmOp::Resid384:
    case GemmOp::Resid1536:
      return launch_one<128>(maps, rows, s.n, s.k, EpiResid{args.bias, args.lambda, args.out},
                             status, stream);
    case GemmOp::SwiGLU:
      return launch_one<256>(maps, rows, s.n, s.k, EpiSwiGLU{args.bias, args.out}, status, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace dv3
