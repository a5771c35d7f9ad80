/*
 * dinov3_kernels.h - C ABI of the individual sm_100a kernels of the DINOv3 ViT-S+/16 forward.
 *
 * One entry point per kernel specialisation of the reference (kernels/*.loom of
 * zacharydenton/dinov3-loom, listed in specifications(), src/lib.rs:281-300). These are what the
 * reference's engine dispatches per launch (src/engine.rs:87-129: a kernel index, one scalar
 * `m_size`/`token_count`, a grid and buffer bindings); here each takes plain device pointers,
 * the row count and a stream. The model API (dinov3.h) records the same kernels into one CUDA
 * graph per batch size.
 *
 * Common rules:
 *   - All pointers are device pointers on the current device, 16-byte aligned.
 *   - f16 tensors are IEEE binary16 (uint16_t storage), f32 tensors float.
 *   - `rows` is the number of token rows (201 per image) or patch rows (196 per image).
 *     rows == 0 launches nothing and returns 0.
 *   - `status` is an optional device array of two uint32_t words (NULL allowed). Word 0
 *     collects device-side failure bits (a bounded wait that expired; the kernel then exits
 *     without finishing). Word 1 is set nonzero by dv3k_patchify when an input value is not
 *     finite. The caller clears and reads them.
 *   - `stream` is a cudaStream_t (NULL: the legacy default stream). Launches are asynchronous.
 *   - Return value: 0, DV3_INVALID_ARGUMENT (shape/alignment) or DV3_DEVICE (launch failed),
 *     with the message in dv3_last_error().
 *
 * Weight layouts (the load-time packing contract, src/weights.rs:62-144):
 *   patch_w  [384][768] f16, columns in (c, dy, dx) order (the conv weight flattened);
 *   patch_b  [384] f32;  prefix [5][384] f32 = CLS token then the 4 register tokens;
 *   qkv_w    [1152][384] f16 = q rows, k rows, v rows;  qkv_b [1152] f32 with the k part 0;
 *   o_w      [384][384] f16;  down_w [384][1536] f16;  o_b, down_b, ls1, ls2 [384] f32;
 *   gateup_w [3072][384] f16 and gateup_b [3072] f32 in the interleaved order of
 *            dv3k_gateup_source_row() (64 gate rows, then the matching 64 up rows, ...);
 *   rope_cos, rope_sin [196][64] f32 (per patch: row freqs 0..15, column freqs 0..15, row,
 *            column; angle 2*pi*(2*(pos+0.5)/14-1)/100^(j/16));
 *   LayerNorm gamma/beta [384] f32.
 */
#ifndef DINOV3_KERNELS_H
#define DINOV3_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Device-side patchify and prefix placement. Replaces the host loop patchify (src/lib.rs:
 * 265-280) and the prefix half of kernels/embed_scatter_f32.loom:
 *   patches[i*196 + gy*14 + gx][(c*16 + dy)*16 + dx] = f16(images[i][c][gy*16+dy][gx*16+dx])
 *   x[i*201 + t][:] = f16(prefix[t][:])  for t < 5
 * Sets status[1] when any input value is not finite (the check of src/lib.rs:95). */
int dv3k_patchify(const float *images, uint32_t n_images, const float *prefix, uint16_t *patches,
                  uint16_t *x, uint32_t *status, void *stream);

/* Patch embedding GEMM and scatter. Replaces kernels/matmul_bias_f16_wmma.loom (k=768, n=384)
 * and the patch half of kernels/embed_scatter_f32.loom:
 *   x[(p/196)*201 + 5 + p%196][n] = f16(sum_k patches[p][k] * w[n][k] + bias[n]),
 * with f32 accumulation, for p < n_patches. */
int dv3k_patch_embed(const uint16_t *patches, uint32_t n_patches, const uint16_t *w,
                     const float *bias, uint16_t *x, uint32_t *status, void *stream);

/* LayerNorm over 384 channels, eps 1e-5, f16 -> f16. Replaces
 * kernels/layernorm_rowwave_f16.loom. */
int dv3k_layernorm_f16(const uint16_t *x, uint32_t rows, const float *gamma, const float *beta,
                       uint16_t *out, void *stream);

/* The final LayerNorm, f16 -> f32. Replaces kernels/layernorm_rowwave_f32out.loom. */
int dv3k_layernorm_f32out(const uint16_t *x, uint32_t rows, const float *gamma,
                          const float *beta, float *out, void *stream);

/* QKV projection with 2D-axial RoPE. Replaces kernels/matmul_qkv_rope_f16_wmma.loom (k=384,
 * n=1152, head_dim 64, prefix 5, tokens_per_image 201, rope_channels 768):
 *   y = h @ w^T + bias (f32);  for columns < 768 of patch rows (t = row % 201 >= 5, p = t-5),
 *   within each 64-wide head: c < 32: y_c cos[p][c] - y_{c+32} sin[p][c];
 *                             c >= 32: y_c cos[p][c] + y_{c-32} sin[p][c];
 *   qkv[row][:] = f16(y). */
int dv3k_qkv_rope(const uint16_t *h, uint32_t rows, const uint16_t *w, const float *bias,
                  const float *rope_cos, const float *rope_sin, uint16_t *qkv, uint32_t *status,
                  void *stream);

/* Multi-head attention per image (6 heads x 64, 201 tokens, scale 0.125) reading q, k, v from
 * the fused QKV rows (stride 1152) and writing head h to columns 64h..64h+63 of out [rows][384].
 * Replaces kernels/attention_online_f16_wmma_cf16.loom. Probabilities are rounded to f16 before
 * the PV product; the normaliser is the f32 sum of the unrounded weights. rows must be a
 * multiple of 201. */
int dv3k_attention(const uint16_t *qkv, uint32_t rows, uint16_t *out, uint32_t *status,
                   void *stream);

/* Projection with LayerScale and residual: x[row][n] = f16(x + lambda[n] * (a @ w^T + bias)[n])
 * for n < 384, in place. k is 384 (attention output projection) or 1536 (MLP down projection).
 * Replaces kernels/matmul_resid_f16_wmma.loom (both specialisations). */
int dv3k_matmul_resid(const uint16_t *a, uint32_t rows, uint32_t k, const uint16_t *w,
                      const float *bias, const float *lambda, uint16_t *x, uint32_t *status,
                      void *stream);

/* Projection with LayerScale and residual followed by the LayerNorm of the updated rows, in one
 * kernel on full 384-column row tiles. Replaces kernels/matmul_resid_f16_wmma.loom followed by
 * kernels/layernorm_rowwave_f16.loom (or kernels/layernorm_rowwave_f32out.loom for the final
 * norm), which the reference launches separately (src/lib.rs:200-211,227-253):
 *   x[row] = f16(x + lambda * (a @ w^T + bias));
 *   h[row] = f16(LN(x[row]) * gamma + beta), or, when h is NULL, out_f32[row] = the same in f32.
 * The LayerNorm reads the f16-rounded x, eps 1e-5. k is 384 or 1536. */
int dv3k_matmul_resid_layernorm(const uint16_t *a, uint32_t rows, uint32_t k, const uint16_t *w,
                                const float *bias, const float *lambda, uint16_t *x,
                                const float *gamma, const float *beta, uint16_t *h,
                                float *out_f32, uint32_t *status, void *stream);

/* Folded LayerNorm (no counterpart in the reference, which normalises each row into h and
 * then multiplies): for a GEMM that consumes h = LN(x) gamma + beta with f16 weights W and bias
 * b, h W^T + b = rstd (x W'^T - mean s + r c) with W' = f16(W gamma), s[n] = sum_k W'[n][k],
 * c = b + W beta and r = 1 / rstd. The correction -mean s + r c is a rank-2 product that the
 * tensor cores add as one more K=16 step: the kernel that updates x leaves, per row, rowstat =
 * (rstd, -mean rstd) (f32 [rows][2]) and the row aux (f16 [rows][16]: -mean_hi, -mean_lo,
 * -mean_hi, r_hi, r_lo, r_hi, then zeros, each *_lo the f16 of what the f16 *_hi leaves over),
 * and the consumer reads x itself with w_aux (f16 [n][16] per output column: s_hi, s_hi, s_lo,
 * c_hi, c_hi, c_lo, then zeros) and scales its accumulator by rstd. The model folds the
 * LayerNorms before the QKV and gate/up projections this way whenever the residual GEMMs run on
 * full rows; the final LayerNorm is not folded. The model's loader derives wf and w_aux from the
 * checkpoint.
 *
 * dv3k_matmul_resid_rowstat: dv3k_matmul_resid_layernorm without the normalised output: x is
 * updated the same way, and rowstat and row_aux get the LayerNorm statistics of the f16-rounded
 * row (eps 1e-5). k is 384 or 1536. */
int dv3k_matmul_resid_rowstat(const uint16_t *a, uint32_t rows, uint32_t k, const uint16_t *w,
                              const float *bias, const float *lambda, uint16_t *x, float *rowstat,
                              uint16_t *row_aux, uint32_t *status, void *stream);

/* rowstat and row_aux of each row of x [rows][384] f16 (eps 1e-5), the statistics
 * dv3k_layernorm_f16 computes (the folded LayerNorm of the first QKV projection). */
int dv3k_layernorm_rowstat(const uint16_t *x, uint32_t rows, float *rowstat, uint16_t *row_aux,
                           void *stream);

/* dv3k_qkv_rope on x instead of h = LN(x): qkv = rope(rstd (x wf^T - mean s + r c)), wf =
 * f16(qkv_w gamma1) [1152][384], w_aux [1152][16] and rowstat, row_aux as above. */
int dv3k_qkv_rope_folded(const uint16_t *x, uint32_t rows, const uint16_t *wf,
                         const uint16_t *w_aux, const float *rowstat, const uint16_t *row_aux,
                         const float *rope_cos, const float *rope_sin, uint16_t *qkv,
                         uint32_t *status, void *stream);

/* dv3k_matmul_swiglu on x instead of h = LN(x): g and u = rstd (x wf^T - mean s + r c), act =
 * f16(silu(g) u), with gateup_wf = f16(gateup_w gamma2) and w_aux [3072][16] in the packed row
 * order. */
int dv3k_matmul_swiglu_folded(const uint16_t *x, uint32_t rows, const uint16_t *gateup_wf,
                              const uint16_t *w_aux, const float *rowstat,
                              const uint16_t *row_aux, uint16_t *act, uint32_t *status,
                              void *stream);

/* Down projection split over K (kernels/matmul_splitk_f16_wmma.loom, launched at batch 1 by
 * src/lib.rs:218-224 with the specialisation of :297): for each slice s < splits of the 1536-long
 * reduction, partials[s][row][n] = sum over k in slice s of a[row][k] * w[n][k], f32, no bias.
 * a: [rows][1536] f16, w: [384][1536] f16, partials: [splits][rows][384] f32. splits divides 24
 * (the 64-wide k-blocks): 1, 2, 3, 4, 6, 8, 12 or 24 (the reference fixes 4). */
int dv3k_matmul_splitk(const uint16_t *a, uint32_t rows, const uint16_t *w, uint32_t splits,
                       float *partials, uint32_t *status, void *stream);

/* Split-K completion (kernels/splitk_reduce_f16.loom, src/lib.rs:225-226, :298): in place,
 * x[row][n] = f16(x + lambda[n] * ((partials[0][row][n] + ... + partials[splits-1][row][n]) +
 * bias[n])), the slabs summed in order onto zero, each step rounded as written. */
int dv3k_splitk_reduce(const float *partials, uint32_t rows, uint32_t splits, const float *bias,
                       const float *lambda, uint16_t *x, void *stream);

/* dv3k_splitk_reduce followed in the same kernel by the LayerNorm that the reference launches
 * after it (kernels/layernorm_rowwave_f16.loom, or _f32out for the final norm): h[row] =
 * f16(LN(x[row]) * gamma + beta), or, when h is NULL, out_f32[row] = the same in f32. The
 * LayerNorm reads the f16-rounded x, eps 1e-5. */
int dv3k_splitk_reduce_layernorm(const float *partials, uint32_t rows, uint32_t splits,
                                 const float *bias, const float *lambda, uint16_t *x,
                                 const float *gamma, const float *beta, uint16_t *h,
                                 float *out_f32, void *stream);

/* dv3k_matmul_splitk followed by dv3k_splitk_reduce (x[row][n] = f16(x + lambda[n] * (sum of
 * the slices + bias[n])), in place) without a workspace argument, for callers that may not
 * allocate device memory themselves (an allocator-free embedding, a caller inside a region
 * where cudaMalloc would synchronise or is forbidden). No counterpart in the reference.
 *   - The partial slabs live in a file-scope device array of the library whose size is fixed
 *     when the library is built: 6144 partial rows of 384 floats (9 MiB, held on every device
 *     that loads the library until the process exits). It is not derived from any SM count;
 *     the caller sizes splits x rows <= 6144, and larger requests return DV3_INVALID_ARGUMENT.
 *   - The call allocates nothing (no cudaMalloc, cudaFree or allocating library routine). The
 *     first call on a device looks up the array's device address once (cudaGetSymbolAddress,
 *     with that device current); make that first call before any stream capture.
 *   - Two launches on `stream`. Every call shares the one array and overwrites the slabs it
 *     uses (no clearing is needed: each slab is fully written before it is read), so calls
 *     that overlap on the GPU race: calls on different streams of one device must be ordered by
 *     the caller. Calls in sequence on one stream are ordered by the stream. */
int dv3k_down_splitk_noalloc(const uint16_t *a, uint32_t rows, const uint16_t *w, uint32_t splits,
                             const float *bias, const float *lambda, uint16_t *x, uint32_t *status,
                             void *stream);

/* Gate/up projection with SwiGLU: act[row][j] = f16(silu(g) * u), g = h@Wg^T+bg, u = h@Wu^T+bu,
 * j < 1536, from the interleaved gateup_w / gateup_b. Replaces
 * kernels/matmul_swiglu_f16_wmma.loom (k=384, n=1536). */
int dv3k_matmul_swiglu(const uint16_t *h, uint32_t rows, const uint16_t *gateup_w,
                       const float *gateup_b, uint16_t *act, uint32_t *status, void *stream);

/* Row of the reference's concatenated gate||up matrix ([3072][384], src/weights.rs:103-108)
 * that packed row `packed_row` (< 3072) of gateup_w holds. Host function. */
uint32_t dv3k_gateup_source_row(uint32_t packed_row);

/* Self-test of the kernels' failure path (no reference counterpart): one CTA whose first role
 * waits on an mbarrier that nothing arrives at, with a limit of `wait_ns` nanoseconds, then
 * records bit 4 in status[0] and raises the CTA's abort flag; a second role waiting (with a
 * thousand-fold limit) on another such barrier leaves on that flag and records bit 5. The kernel
 * returns normally, so the context stays usable; every kernel above unwinds the same way. */
int dv3k_bounded_wait_selftest(uint64_t wait_ns, uint32_t *status, void *stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif /* DINOV3_KERNELS_H */
