// kernels.h - internal C++ interface of the sm_100a kernels (used by the model engine and by
// the per-kernel C ABI in capi.cpp). All launches are asynchronous on the given stream.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace dv3 {

constexpr int kTokens = 201;
constexpr int kPatches = 196;
constexpr int kPrefix = 5;
constexpr int kHidden = 384;
constexpr int kQkv = 1152;
constexpr int kMlp = 1536;
constexpr int kGateUp = 3072;
constexpr int kPatchK = 768;
constexpr int kImage = 224;  // image side in pixels
constexpr int kImageElements = 3 * kImage * kImage;

// ---- tensor maps (tma.cpp) ----
// 2D f16 tensor [rows][cols] (row-major, `cols` contiguous), box = box_cols x box_rows, 128-byte
// swizzle (box_cols must be 64), out-of-bounds elements read as zero.
bool encode_map_f16(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                    uint32_t box_cols, uint32_t box_rows, std::string *err);
// The same with a 32-, 64- or 128-byte swizzle (box_cols * 2 must equal the swizzle width).
bool encode_map_f16_swizzled(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                             uint32_t box_cols, uint32_t box_rows, uint32_t swizzle_bytes,
                             std::string *err);

// 2D f32 tensor [rows][cols], box = 32 columns (128 bytes) x box_rows, 128-byte swizzle.
bool encode_map_f32(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                    uint32_t box_cols, uint32_t box_rows, std::string *err);

// 3D f16 view [n_images][201 tokens][cols] of token rows, box = 64 columns x box_rows tokens x 1
// image, 128-byte swizzle. Tokens past 201 fall outside the image: loads read zeros, stores
// are clipped.
bool encode_map_f16_images(CUtensorMap *map, const void *base, uint64_t cols, uint64_t n_images,
                           uint32_t box_rows, std::string *err);
// 3D f32 view [slabs][rows][cols] (split-K partials), box = 32 columns x box_rows x 1 slab,
// 128-byte swizzle; stores past `rows` are clipped inside each slab.
bool encode_map_f32_slabs(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                          uint64_t slabs, uint32_t box_rows, std::string *err);

// ---- GEMM operations (gemm.cu) ----
// Resid*: x += lambda (A W^T + b) on 128-column tiles. ResidLN*: the same on full 384-column
// rows, followed in the same kernel by the LayerNorm of the updated row into ln_out (f16) or
// ln_out_f32. SplitK1536: the down projection's K split into `splits` slices, each CTA writing
// the f32 partial product of its slice (no bias) into slab s of partials [splits][rows][384]
// (kernels/matmul_splitk_f16_wmma.loom); splitk_reduce completes it.
// Folded LayerNorm (no counterpart in the reference; the weights in weights.cpp): ResidStats*
// update x like ResidLN* but leave only the statistics of the updated row, rowstat[row] =
// (rstd, -mean rstd) and the f16 aux row (-mean_hi, -mean_lo, -mean_hi, r_hi, r_lo, r_hi,
// 0...) with r = 1 / rstd; QkvRopeFold and SwiGLUFold then read x itself with W' = f16(W gamma),
// run one more K=16 MMA step of the aux row against W_aux = (s_hi, s_hi, s_lo, c_hi, c_hi, c_lo,
// 0...) per output column (s the row sums of W', c = b + W beta), so that the accumulator holds
// x W'^T - mean s + r c, and scale it by rstd in their epilogues before RoPE or SwiGLU.
enum class GemmOp {
  Patch,
  QkvRope,
  Resid384,
  Resid1536,
  SwiGLU,
  ResidLN384,
  ResidLN1536,
  SplitK1536,
  ResidStats384,
  ResidStats1536,
  QkvRopeFold,
  SwiGLUFold
};

struct GemmShape {
  int bn;      // tile width along N
  int n;       // output width of the GEMM
  int k;       // reduction length
};
GemmShape gemm_shape(GemmOp op);
// The shape a launch over `rows` rows uses (the residual GEMMs widen to 384 columns when their M
// tiles fit one wave).
GemmShape gemm_shape(GemmOp op, uint32_t rows);
// Whether the residual GEMMs over `rows` rows run on full 384-wide rows (the ResidLN* ops always
// do; they need every 128-row tile in one wave of CTAs).
bool resid_wide(uint32_t rows);
// Whether the forward plan over `rows` rows runs the residual GEMMs on full rows with the
// LayerNorms fused and folded (the 128-wide residual tiles would need more than one wave, and
// every full-row tile fits one).
bool resid_full_rows_plan(uint32_t rows);

// Tensor maps of one GEMM launch: A = activations [rows][k], B = weights [n][k].
struct GemmMaps {
  CUtensorMap a;
  CUtensorMap b;
  CUtensorMap c;  // the epilogue's output, for epilogues that store through TMA
  CUtensorMap d;  // ResidLN*: the LayerNorm output (f16 h, or the f32 final output);
                  // QkvRopeFold / SwiGLUFold: the row aux [rows][16]
  CUtensorMap e;  // QkvRopeFold / SwiGLUFold: the weight aux [n][16]
};
// `out` is the tensor the epilogue writes (qkv, act or x; unused by Patch, which writes x through
// GemmArgs). ResidLN* also takes the LayerNorm output: `ln_out` f16 [rows][384], or f32 when
// `ln_f32`.
// SplitK1536: `out` is the f32 partials [splits][rows][384].
bool make_gemm_maps(GemmOp op, const void *a, uint32_t rows, const void *w, void *out,
                    GemmMaps *maps, std::string *err, const void *ln_out = nullptr,
                    bool ln_f32 = false, uint32_t splits = 1);
// QkvRopeFold / SwiGLUFold: the maps of the extra K step, the row aux [rows][16] and the weight
// aux [n][16] (f16, 16-column boxes with the 32-byte swizzle), after make_gemm_maps.
bool make_fold_maps(GemmOp op, const void *row_aux, uint32_t rows, const void *w_aux,
                    GemmMaps *maps, std::string *err);

struct GemmArgs {
  const float *bias = nullptr;
  const float *lambda = nullptr;    // Resid*
  const float *rope_cos = nullptr;  // QkvRope
  const float *rope_sin = nullptr;
  __half *out = nullptr;  // Patch: x; QkvRope: qkv; Resid*: x (in place); SwiGLU: act
  const float *gamma = nullptr;  // ResidLN*: LayerNorm weight and bias
  const float *beta = nullptr;
  __half *ln_out = nullptr;      // ResidLN*: f16 LayerNorm output, or
  float *ln_out_f32 = nullptr;   //           f32 LayerNorm output when non-null
  float *partials = nullptr;     // SplitK1536: [splits][rows][384] f32
  uint32_t splits = 1;           // SplitK1536: K slices (a divisor of 24, the 64-wide k-blocks)
  // Folded LayerNorm: ResidStats* write, and QkvRopeFold / SwiGLUFold read, rowstat (rstd,
  // -mean rstd) and the row aux [rows][16] f16 of each row (`bias` unused by the folded GEMMs,
  // whose bias is in the weight aux of their maps).
  float2 *rowstat = nullptr;
  __half *row_aux = nullptr;
  // Weights of a later kernel (16-byte aligned; no kernel writes them) that this launch starts
  // toward L2, so that kernel's first tiles do not wait for DRAM.
  const void *l2_next = nullptr;
  size_t l2_next_bytes = 0;
  // An intermediate that earlier kernels wrote and read and that nothing reads any more (and this
  // launch does not write): its whole 128-byte lines are dropped from L2 without a write-back
  // after this launch's dependency wait (see discard_range).
  const void *discard = nullptr;
  size_t discard_bytes = 0;
};

// The whole 128-byte lines inside [p, p + bytes), as the (pointer, bytes) pair that the kernels'
// L2 discard takes (null when none).
inline void discard_range(const void *p, size_t bytes, const void **out, size_t *out_bytes) {
  *out = nullptr;
  *out_bytes = 0;
  if (!p) return;
  const uintptr_t a = reinterpret_cast<uintptr_t>(p), lo = (a + 127) & ~uintptr_t{127},
                  hi = (a + bytes) & ~uintptr_t{127};
  if (hi <= lo) return;
  *out = reinterpret_cast<const void *>(lo);
  *out_bytes = hi - lo;
}

// The K split of the down projection over `rows` rows in the model's plan: the most slices (at
// most 8, a divisor of 24, so each CTA walks at least three 64-wide k-blocks) whose
// 128x128 partial tiles still fit one wave of CTAs; 1 means no split (the unsplit residual
// GEMM runs instead).
uint32_t splitk_splits(uint32_t rows);
// The device address (current device) of the file-scope partial-slab array of the no-alloc
// split-K entry point, and its size in floats; null if the address cannot be had.
float *splitk_scratch(size_t *capacity_floats);

cudaError_t launch_gemm(GemmOp op, const GemmMaps &maps, uint32_t rows, const GemmArgs &args,
                        uint32_t *status, cudaStream_t stream);
const char *gemm_name(GemmOp op);

// ---- attention (attention.cu) ----
// Per-image tensor maps: q (128-token boxes) and kv (208-token boxes) over the fused QKV rows,
// out (32-token boxes) over the attention output.
struct AttentionMaps {
  CUtensorMap q;
  CUtensorMap kv;
  CUtensorMap out;
};
bool make_attention_map(const void *qkv, const void *out, uint32_t rows, AttentionMaps *maps,
                        std::string *err);
// l2_next/l2_next_bytes: weights of a later kernel to prefetch into L2; discard/discard_bytes: a
// dead intermediate to drop from L2 (see GemmArgs).
cudaError_t launch_attention(const AttentionMaps &maps, uint32_t rows, uint32_t *status,
                             cudaStream_t stream, const void *l2_next = nullptr,
                             size_t l2_next_bytes = 0, const void *discard = nullptr,
                             size_t discard_bytes = 0);

// ---- bandwidth kernels (elementwise.cu) ----
// l2_next/l2_next_bytes: weights of a later kernel to prefetch into L2 (see GemmArgs).
cudaError_t launch_patchify(const float *images, uint32_t n_images, const float *prefix,
                            __half *patches, __half *x, uint32_t *status, cudaStream_t stream,
                            const void *l2_next = nullptr, size_t l2_next_bytes = 0);
cudaError_t launch_layernorm_f16(const __half *x, uint32_t rows, const float *gamma,
                                 const float *beta, __half *out, cudaStream_t stream);
cudaError_t launch_layernorm_f32(const __half *x, uint32_t rows, const float *gamma,
                                 const float *beta, float *out, cudaStream_t stream);
// The statistics of the LayerNorm only: rowstat[r] = (rstd, -mean rstd) and the aux row of row
// r of x (GemmOp::ResidStats*; the folded LayerNorm of the QKV GEMM after the patch embedding).
cudaError_t launch_layernorm_rowstat(const __half *x, uint32_t rows, float2 *rowstat,
                                     __half *row_aux, cudaStream_t stream);

// Split-K completion (kernels/splitk_reduce_f16.loom): x[r][n] = f16(x + lambda[n] (sum over
// s = 0..splits-1 in that order of partials[s][r][n] + b[n])), one warp per row. With gamma and
// beta it also writes the LayerNorm of the updated f16 row, like the separate LayerNorm kernel
// that follows the reduce in the reference's plan, into h (f16) or, when out_f32 is non-null,
// out_f32.
cudaError_t launch_splitk_reduce(const float *partials, uint32_t rows, uint32_t splits,
                                 const float *bias, const float *lambda, __half *x,
                                 const float *gamma, const float *beta, __half *h, float *out_f32,
                                 cudaStream_t stream);

// Mean of each image's 196 patch rows of the f32 output (the reference's f32 order), n x 384.
cudaError_t launch_patch_mean(const float *out, uint32_t n_images, float *dst,
                              cudaStream_t stream);

// Packed gate/up row order: 64 gate rows, the matching 64 up rows, then the next 64 of each.
inline uint32_t gateup_source_row(uint32_t packed) {
  const uint32_t block = packed / 128, within = packed % 128;
  return within < 64 ? block * 64 + within : kMlp + block * 64 + (within - 64);
}

// Failure-path self-test: an mbarrier wait that expires after `short_ns` and a second role that
// unwinds on the abort flag; reports through status[0] (bits 4 and 5).
cudaError_t launch_bounded_wait_selftest(uint64_t short_ns, uint32_t *status, cudaStream_t stream);

int sm_count(int device);

// Launch `kernel` with programmatic stream serialization (see pdl_wait in sm100.cuh), so its
// launch and set-up overlap the tail of the previous kernel on the stream; inside stream capture
// the edge becomes a programmatic dependency of the graph.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args &&...args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

}  // namespace dv3
