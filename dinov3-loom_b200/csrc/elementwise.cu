// elementwise.cu - the HBM-bound kernels of the forward.
//
// patchify: normalised NCHW f32 images -> patch rows [p][768] f16 in (c, dy, dx) order (the
//   host loop of src/lib.rs:265-280 moved onto the device), plus the CLS/register prefix rows of
//   the residual stream (the prefix half of kernels/embed_scatter_f32.loom). One thread moves 8
//   pixels: two 16-byte loads of a 32-byte run of one image row, one 16-byte store. It also
//   flags any non-finite pixel (the check of src/lib.rs:95), so the host never scans the input.
//
// layernorm: a warp per two 384-channel rows (kernels/layernorm_rowwave_f16.loom and _f32out).
//   Lane l holds channels 8l..8l+7 (one 16-byte load) and 256+4l..256+4l+3 (one 8-byte load):
//   both loads are contiguous across the warp. Mean and variance are reduced with shuffles in
//   two passes over the registers (the reference's E[x^2]-mean^2 is replaced by the better
//   conditioned centred sum), eps 1e-5, f32 arithmetic.
#include <atomic>

#include "kernels.h"
#include "sm100.cuh"

namespace dv3 {

__global__ void __launch_bounds__(256)
    patchify_kernel(const float *__restrict__ images, int n_images,
                    const float *__restrict__ prefix, __half *__restrict__ patches,
                    __half *__restrict__ x, uint32_t *status, const void *l2_next,
                    size_t l2_next_bytes) {
  pdl_wait();  // the input upload (and the previous forward's readers) are done from here on
  pdl_trigger();
  // the patch GEMM's weights toward L2 (64 KB per block, the first blocks of the grid)
  if (threadIdx.x == 0 && l2_next) l2_prefetch_share(l2_next, l2_next_bytes);
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t n_patch_chunks = static_cast<int64_t>(n_images) * kPatches * 96;
  const int64_t n_prefix_chunks = static_cast<int64_t>(n_images) * kPrefix * 48;
  bool bad = false;
  if (i < n_patch_chunks) {
    const int chunk = static_cast<int>(i % 96);  // 8-element chunk of the 768-wide patch row
    const int64_t prow = i / 96;
    const int img = static_cast<int>(prow / kPatches);
    const int p = static_cast<int>(prow % kPatches);
    const int gy = p / 14, gx = p % 14;
    const int c = chunk / 32, dy = (chunk / 2) % 16, dx0 = (chunk % 2) * 8;
    const float *src = images + (static_cast<int64_t>(img) * 3 + c) * 224 * 224 +
                       (gy * 16 + dy) * 224 + gx * 16 + dx0;
    const float4 a = __ldg(reinterpret_cast<const float4 *>(src));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(src) + 1);
    bad = !(isfinite(a.x) && isfinite(a.y) && isfinite(a.z) && isfinite(a.w) && isfinite(b.x) &&
            isfinite(b.y) && isfinite(b.z) && isfinite(b.w));
    const uint4 v = make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y),
                               pack_half2(b.z, b.w));
    *reinterpret_cast<uint4 *>(patches + prow * kPatchK + chunk * 8) = v;
  } else if (i < n_patch_chunks + n_prefix_chunks) {
    const int64_t j = i - n_patch_chunks;
    const int chunk = static_cast<int>(j % 48);
    const int t = static_cast<int>((j / 48) % kPrefix);
    const int64_t img = j / (48 * kPrefix);
    const float4 *src = reinterpret_cast<const float4 *>(prefix + t * kHidden + chunk * 8);
    const float4 a = __ldg(src), b = __ldg(src + 1);
    const uint4 v = make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y),
                               pack_half2(b.z, b.w));
    *reinterpret_cast<uint4 *>(x + (img * kTokens + t) * kHidden + chunk * 8) = v;
  }
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x % 32) == 0 && status)
    atomicOr(status + 1, 1u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Rows per warp: both rows' loads are issued before either is reduced, so each warp keeps two
// independent memory round trips in flight and the grid (12,864 rows at batch 64) fits in one
// wave of resident warps.
constexpr int kLnRowsPerWarp = 2;
constexpr int kLnRowsPerBlock = 8 * kLnRowsPerWarp;

template <bool kF32Out>
__global__ void __launch_bounds__(256)
    layernorm_kernel(const __half *__restrict__ x, int rows, const float *__restrict__ gamma,
                     const float *__restrict__ beta, void *__restrict__ out) {
  pdl_wait();  // the rows written by the previous kernel are complete from here on
  pdl_trigger();
  const int row0 = (blockIdx.x * 8 + threadIdx.x / 32) * kLnRowsPerWarp;
  const int lane = threadIdx.x % 32;
  if (row0 >= rows) return;  // whole warp leaves together
  const int c0 = lane * 8, c1 = 256 + lane * 4;
  uint4 a[kLnRowsPerWarp];
  uint2 b[kLnRowsPerWarp];
#pragma unroll
  for (int k = 0; k < kLnRowsPerWarp; ++k) {
    const int row = row0 + k < rows ? row0 + k : row0;
    const __half *xr = x + static_cast<int64_t>(row) * kHidden;
    a[k] = __ldg(reinterpret_cast<const uint4 *>(xr) + lane);
    b[k] = __ldg(reinterpret_cast<const uint2 *>(xr + 256) + lane);
  }
  float g[12], bb[12];
  {
    const float4 g0 = __ldg(reinterpret_cast<const float4 *>(gamma + c0));
    const float4 g1 = __ldg(reinterpret_cast<const float4 *>(gamma + c0) + 1);
    const float4 g2 = __ldg(reinterpret_cast<const float4 *>(gamma + c1));
    const float4 b0 = __ldg(reinterpret_cast<const float4 *>(beta + c0));
    const float4 b1 = __ldg(reinterpret_cast<const float4 *>(beta + c0) + 1);
    const float4 b2 = __ldg(reinterpret_cast<const float4 *>(beta + c1));
    const float gg[12] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w, g2.x, g2.y, g2.z, g2.w};
    const float bv[12] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w, b2.x, b2.y, b2.z, b2.w};
#pragma unroll
    for (int e = 0; e < 12; ++e) {
      g[e] = gg[e];
      bb[e] = bv[e];
    }
  }
#pragma unroll
  for (int k = 0; k < kLnRowsPerWarp; ++k) {
    const int row = row0 + k;
    float v[12];
    const uint32_t w[6] = {a[k].x, a[k].y, a[k].z, a[k].w, b[k].x, b[k].y};
#pragma unroll
    for (int e = 0; e < 6; ++e) {
      const float2 f = unpack_half2(w[e]);
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 12; ++e) s += v[e];
    const float mean = warp_sum(s) * (1.0f / kHidden);
    float d = 0.f;
#pragma unroll
    for (int e = 0; e < 12; ++e) {
      v[e] -= mean;
      d += v[e] * v[e];
    }
    const float rstd = rsqrtf(warp_sum(d) * (1.0f / kHidden) + 1e-5f);
    float y[12];
#pragma unroll
    for (int e = 0; e < 12; ++e) y[e] = v[e] * rstd * g[e] + bb[e];
    if (row >= rows) break;
    if constexpr (kF32Out) {
      float *o = static_cast<float *>(out) + static_cast<int64_t>(row) * kHidden;
      reinterpret_cast<float4 *>(o + c0)[0] = make_float4(y[0], y[1], y[2], y[3]);
      reinterpret_cast<float4 *>(o + c0)[1] = make_float4(y[4], y[5], y[6], y[7]);
      reinterpret_cast<float4 *>(o + c1)[0] = make_float4(y[8], y[9], y[10], y[11]);
    } else {
      __half *o = static_cast<__half *>(out) + static_cast<int64_t>(row) * kHidden;
      reinterpret_cast<uint4 *>(o + c0)[0] =
          make_uint4(pack_half2(y[0], y[1]), pack_half2(y[2], y[3]), pack_half2(y[4], y[5]),
                     pack_half2(y[6], y[7]));
      reinterpret_cast<uint2 *>(o + c1)[0] =
          make_uint2(pack_half2(y[8], y[9]), pack_half2(y[10], y[11]));
    }
  }
}

// The statistics of the LayerNorm only (folded LayerNorm, GemmOp::QkvRopeFold): rowstat[r] =
// (rstd, -mean rstd) and the aux row (store_row_aux) of row r, computed as layernorm_kernel
// computes them. One row per warp.
__global__ void __launch_bounds__(256)
    layernorm_rowstat_kernel(const __half *__restrict__ x, int rows, float2 *__restrict__ rowstat,
                             __half *__restrict__ row_aux) {
  pdl_wait();  // the rows written by the previous kernel are complete from here on
  pdl_trigger();
  const int row = blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;  // whole warp leaves together
  const __half *xr = x + static_cast<int64_t>(row) * kHidden;
  const uint4 a = __ldg(reinterpret_cast<const uint4 *>(xr) + lane);
  const uint2 b = __ldg(reinterpret_cast<const uint2 *>(xr + 256) + lane);
  const uint32_t w[6] = {a.x, a.y, a.z, a.w, b.x, b.y};
  float v[12];
#pragma unroll
  for (int e = 0; e < 6; ++e) {
    const float2 f = unpack_half2(w[e]);
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 12; ++e) s += v[e];
  const float mean = warp_sum(s) * (1.0f / kHidden);
  float d = 0.f;
#pragma unroll
  for (int e = 0; e < 12; ++e) {
    const float t = v[e] - mean;
    d += t * t;
  }
  const float rstd = rsqrtf(warp_sum(d) * (1.0f / kHidden) + 1e-5f);
  if (lane == 0) rowstat[row] = make_float2(rstd, -mean * rstd);
  if (lane == 1) store_row_aux(row_aux + static_cast<size_t>(row) * 16, mean, rstd);
}

cudaError_t launch_layernorm_rowstat(const __half *x, uint32_t rows, float2 *rowstat,
                                     __half *row_aux, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  return launch_pdl(layernorm_rowstat_kernel, dim3((rows + 7) / 8), dim3(256), 0, stream, x,
                    static_cast<int>(rows), rowstat, row_aux);
}

cudaError_t launch_patchify(const float *images, uint32_t n_images, const float *prefix,
                            __half *patches, __half *x, uint32_t *status, cudaStream_t stream,
                            const void *l2_next, size_t l2_next_bytes) {
  if (n_images == 0) return cudaSuccess;
  const int64_t total = static_cast<int64_t>(n_images) * (kPatches * 96 + kPrefix * 48);
  const int blocks = static_cast<int>((total + 255) / 256);
  return launch_pdl(patchify_kernel, dim3(blocks), dim3(256), 0, stream, images,
                    static_cast<int>(n_images), prefix, patches, x, status, l2_next,
                    l2_next_bytes & ~static_cast<size_t>(15));
}

cudaError_t launch_layernorm_f16(const __half *x, uint32_t rows, const float *gamma,
                                 const float *beta, __half *out, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  return launch_pdl(layernorm_kernel<false>, dim3((rows + kLnRowsPerBlock - 1) / kLnRowsPerBlock),
                    dim3(256), 0, stream, x,
                    static_cast<int>(rows), gamma, beta, static_cast<void *>(out));
}

cudaError_t launch_layernorm_f32(const __half *x, uint32_t rows, const float *gamma,
                                 const float *beta, float *out, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  return launch_pdl(layernorm_kernel<true>, dim3((rows + kLnRowsPerBlock - 1) / kLnRowsPerBlock),
                    dim3(256), 0, stream, x,
                    static_cast<int>(rows), gamma, beta, static_cast<void *>(out));
}

// Split-K completion (kernels/splitk_reduce_f16.loom): one warp per row, lane columns
// 8*lane..8*lane+7 and 256+4*lane..+3 (coalesced f32 and f16 loads). The slabs are added in order
// s = 0..splits-1 onto zero, then the bias, times lambda, onto the f16 residual, each step rounded
// as the reference does it (no fused multiply-add). kLn: the LayerNorm of the stored f16 row
// follows in registers, as layernorm_kernel computes it (two-pass centred variance, eps 1e-5),
// into h (f16) or out (f32).
template <int kLn>  // 0: reduce only, 1: + LayerNorm to f16 h, 2: + LayerNorm to f32 out
__global__ void __launch_bounds__(256)
    splitk_reduce_kernel(const float *__restrict__ partials, int rows, int splits,
                         const float *__restrict__ bias, const float *__restrict__ lambda,
                         __half *__restrict__ x, const float *__restrict__ gamma,
                         const float *__restrict__ beta, void *__restrict__ out) {
  pdl_wait();  // the partial slabs of the previous kernel are complete from here on
  pdl_trigger();
  const int row = blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;  // whole warp leaves together
  const int c0 = lane * 8, c1 = 256 + lane * 4;
  auto load12 = [&](const float *base, float (&v)[12]) {
    const float4 a0 = __ldg(reinterpret_cast<const float4 *>(base + c0));
    const float4 a1 = __ldg(reinterpret_cast<const float4 *>(base + c0) + 1);
    const float4 a2 = __ldg(reinterpret_cast<const float4 *>(base + c1));
    const float t[12] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w, a2.x, a2.y, a2.z, a2.w};
#pragma unroll
    for (int e = 0; e < 12; ++e) v[e] = t[e];
  };
  float acc[12];
#pragma unroll
  for (int e = 0; e < 12; ++e) acc[e] = 0.f;
  const size_t slab = static_cast<size_t>(rows) * kHidden;
  const float *prow = partials + static_cast<size_t>(row) * kHidden;
  // up to eight slabs' loads in flight at once, then added in slab order
  for (int s0 = 0; s0 < splits; s0 += 8) {
    float p[8][12];
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (s0 + k < splits) load12(prow + (s0 + k) * slab, p[k]);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (s0 + k < splits) {
#pragma unroll
        for (int e = 0; e < 12; ++e) acc[e] = __fadd_rn(acc[e], p[k][e]);
      }
  }
  float b[12], l[12];
  load12(bias, b);
  load12(lambda, l);
  __half *xr = x + static_cast<size_t>(row) * kHidden;
  const uint4 xa = *reinterpret_cast<const uint4 *>(xr + c0);
  const uint2 xb = *reinterpret_cast<const uint2 *>(xr + c1);
  const uint32_t w[6] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y};
  float v[12];
  uint32_t o[6];
#pragma unroll
  for (int e = 0; e < 6; ++e) {
    const float2 prior = unpack_half2(w[e]);
    const float u0 = __fadd_rn(prior.x, __fmul_rn(__fadd_rn(acc[2 * e], b[2 * e]), l[2 * e]));
    const float u1 =
        __fadd_rn(prior.y, __fmul_rn(__fadd_rn(acc[2 * e + 1], b[2 * e + 1]), l[2 * e + 1]));
    o[e] = pack_half2(u0, u1);
    const float2 r = unpack_half2(o[e]);  // the LayerNorm reads the stored f16 values
    v[2 * e] = r.x;
    v[2 * e + 1] = r.y;
  }
  *reinterpret_cast<uint4 *>(xr + c0) = make_uint4(o[0], o[1], o[2], o[3]);
  *reinterpret_cast<uint2 *>(xr + c1) = make_uint2(o[4], o[5]);
  if constexpr (kLn != 0) {
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 12; ++e) s += v[e];
    const float mean = warp_sum(s) * (1.0f / kHidden);
    float d = 0.f;
#pragma unroll
    for (int e = 0; e < 12; ++e) {
      v[e] -= mean;
      d += v[e] * v[e];
    }
    const float rstd = rsqrtf(warp_sum(d) * (1.0f / kHidden) + 1e-5f);
    float g[12], bt[12], y[12];
    load12(gamma, g);
    load12(beta, bt);
#pragma unroll
    for (int e = 0; e < 12; ++e) y[e] = v[e] * rstd * g[e] + bt[e];
    if constexpr (kLn == 2) {
      float *orow = static_cast<float *>(out) + static_cast<size_t>(row) * kHidden;
      reinterpret_cast<float4 *>(orow + c0)[0] = make_float4(y[0], y[1], y[2], y[3]);
      reinterpret_cast<float4 *>(orow + c0)[1] = make_float4(y[4], y[5], y[6], y[7]);
      *reinterpret_cast<float4 *>(orow + c1) = make_float4(y[8], y[9], y[10], y[11]);
    } else {
      __half *hrow = static_cast<__half *>(out) + static_cast<size_t>(row) * kHidden;
      *reinterpret_cast<uint4 *>(hrow + c0) =
          make_uint4(pack_half2(y[0], y[1]), pack_half2(y[2], y[3]), pack_half2(y[4], y[5]),
                     pack_half2(y[6], y[7]));
      *reinterpret_cast<uint2 *>(hrow + c1) = make_uint2(pack_half2(y[8], y[9]), pack_half2(y[10], y[11]));
    }
  }
}

cudaError_t launch_splitk_reduce(const float *partials, uint32_t rows, uint32_t splits,
                                 const float *bias, const float *lambda, __half *x,
                                 const float *gamma, const float *beta, __half *h, float *out_f32,
                                 cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  const dim3 grid((rows + 7) / 8), block(256);
  const int r = static_cast<int>(rows), sp = static_cast<int>(splits);
  if (gamma == nullptr)
    return launch_pdl(splitk_reduce_kernel<0>, grid, block, 0, stream, partials, r, sp, bias,
                      lambda, x, gamma, beta, static_cast<void *>(nullptr));
  if (out_f32 != nullptr)
    return launch_pdl(splitk_reduce_kernel<2>, grid, block, 0, stream, partials, r, sp, bias,
                      lambda, x, gamma, beta, static_cast<void *>(out_f32));
  return launch_pdl(splitk_reduce_kernel<1>, grid, block, 0, stream, partials, r, sp, bias, lambda,
                    x, gamma, beta, static_cast<void *>(h));
}

// patch_mean (src/lib.rs:134-148) on the device: one thread per (image, channel) adds
// row / 196 over the patch rows 5..200 in order, in f32 with correctly rounded division, so the
// result equals the reference's host loop bit for bit. Reads are coalesced across channels.
__global__ void __launch_bounds__(128)
    patch_mean_kernel(const float *__restrict__ out, int n_images, float *__restrict__ dst) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;  // channel
  const int img = blockIdx.y;
  if (c >= kHidden || img >= n_images) return;
  const float *src = out + static_cast<size_t>(img) * kTokens * kHidden + c;
  float acc = 0.f;
#pragma unroll 4
  for (int t = kPrefix; t < kTokens; ++t) acc = __fadd_rn(acc, __fdiv_rn(src[t * kHidden], 196.0f));
  dst[static_cast<size_t>(img) * kHidden + c] = acc;
}

cudaError_t launch_patch_mean(const float *out, uint32_t n_images, float *dst,
                              cudaStream_t stream) {
  if (n_images == 0) return cudaSuccess;
  patch_mean_kernel<<<dim3(kHidden / 128, n_images), 128, 0, stream>>>(
      out, static_cast<int>(n_images), dst);
  return cudaGetLastError();
}

// Self-test of the failure path every kernel uses (no reference counterpart): two mbarriers
// that nothing ever arrives at. Warp 0 waits on the first with a short limit; when it expires it
// records kErrSelfTestWait and raises the CTA's abort flag, as a kernel role does. Warp 1 waits
// on the second with a limit a thousand times longer and must leave on the abort flag, recording
// kErrSelfTestAbort. The kernel then returns normally: no trap, no fault, the context stays
// usable, and the host reads the status word.
__global__ void __launch_bounds__(64) bounded_wait_selftest_kernel(uint64_t short_ns,
                                                                   uint32_t *status) {
  __shared__ uint64_t bars[2];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int *abort = &abort_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    if (warp == 0) {
      if (!mbar_wait(&bars[0], 0, abort, short_ns)) {
        report(status, kErrSelfTestWait);
        *abort = 1;
      }
    } else {
      if (!mbar_wait(&bars[1], 0, abort, short_ns * 1000) && *abort)
        report(status, kErrSelfTestAbort);
    }
  }
  __syncthreads();
}

cudaError_t launch_bounded_wait_selftest(uint64_t short_ns, uint32_t *status,
                                         cudaStream_t stream) {
  bounded_wait_selftest_kernel<<<1, 64, 0, stream>>>(short_ns, status);
  return cudaGetLastError();
}

int sm_count(int device) {
  static std::atomic<int> cache[64] = {};
  if (device < 0 || device >= 64) return 148;
  int n = cache[device].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    cache[device].store(n, std::memory_order_relaxed);
  }
  return n;
}

}  // namespace dv3
