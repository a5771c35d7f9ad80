// capi.cpp - the exported C ABI (include/dinov3.h, include/dinov3_kernels.h). Every entry point
// converts C++ exceptions into a status code and a thread-local message.
#include <cstring>
#include <new>
#include <string>

#include "dinov3.h"
#include "dinov3_kernels.h"
#include "kernels.h"
#include "model.h"
#include "weights.h"

struct dv3_model {
  dv3::Model impl;
  dv3_model(const std::string &path, dv3_options o) : impl(path, o) {}
};

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string &message) {
  g_last_error = message;
  return code;
}

template <class F>
int guarded(F &&f) {
  try {
    f();
    return DV3_OK;
  } catch (const dv3::Error &e) {
    return fail(e.code, e.what());
  } catch (const std::bad_alloc &) {
    return fail(DV3_DEVICE, "out of host memory");
  } catch (const std::exception &e) {
    return fail(DV3_DEVICE, e.what());
  }
}

int check_model(dv3_model *m) {
  if (!m) return fail(DV3_INVALID_ARGUMENT, "null model");
  return DV3_OK;
}

}  // namespace

namespace dv3 {
bool hub_weights(bool offline, std::string *path, std::string *err);
}

extern "C" {

dv3_options dv3_default_options(void) {
  dv3_options o;
  o.device = 0;
  o.max_batch = 32;
  return o;
}

int dv3_load(const char *path, dv3_options options, dv3_model **out) {
  if (!out) return fail(DV3_INVALID_ARGUMENT, "null output handle");
  *out = nullptr;
  return guarded([&] {
    if (options.max_batch < 1 || options.max_batch > DV3_MAX_BATCH_LIMIT)
      throw dv3::Error(DV3_INVALID_ARGUMENT, "max_batch must be 1..=64");
    if (!path) throw dv3::Error(DV3_INVALID_ARGUMENT, "null path");
    *out = new dv3_model(path, options);
  });
}

int dv3_from_pretrained(dv3_options options, dv3_model **out) {
  if (!out) return fail(DV3_INVALID_ARGUMENT, "null output handle");
  *out = nullptr;
  if (options.max_batch < 1 || options.max_batch > DV3_MAX_BATCH_LIMIT)
    return fail(DV3_INVALID_ARGUMENT, "max_batch must be 1..=64");
  std::string path, err;
  if (!dv3::hub_weights(false, &path, &err)) return fail(DV3_WEIGHTS, err);
  return dv3_load(path.c_str(), options, out);
}

int dv3_forward(dv3_model *m, const float *pixels, size_t n, float *out, size_t out_n) {
  if (int rc = check_model(m)) return rc;
  return guarded([&] { m->impl.forward(pixels, n, out, out_n); });
}

int dv3_cls(dv3_model *m, const float *pixels, size_t n, float *out, size_t out_n) {
  if (int rc = check_model(m)) return rc;
  return guarded([&] { m->impl.forward(pixels, n, out, out_n, dv3::Model::Readout::Cls); });
}

int dv3_patch_mean(dv3_model *m, const float *pixels, size_t n, float *out, size_t out_n) {
  if (int rc = check_model(m)) return rc;
  return guarded([&] { m->impl.forward(pixels, n, out, out_n, dv3::Model::Readout::PatchMean); });
}

int dv3_benchmark(dv3_model *m, const float *pixels, size_t n, size_t samples, dv3_timings *out) {
  if (int rc = check_model(m)) return rc;
  if (!out) return fail(DV3_INVALID_ARGUMENT, "null timings");
  return guarded([&] { *out = m->impl.benchmark(pixels, n, samples); });
}

void dv3_free(dv3_model *m) { delete m; }

const char *dv3_last_error(void) { return g_last_error.c_str(); }

float *dv3_input_buffer(dv3_model *m) { return m ? m->impl.input_buffer() : nullptr; }
float *dv3_output_buffer(dv3_model *m) { return m ? m->impl.output_buffer() : nullptr; }
void *dv3_stream(dv3_model *m) { return m ? static_cast<void *>(m->impl.stream()) : nullptr; }

int dv3_run(dv3_model *m, size_t batch) {
  if (int rc = check_model(m)) return rc;
  return guarded([&] { m->impl.run(batch); });
}

int dv3_synchronize(dv3_model *m) {
  if (int rc = check_model(m)) return rc;
  return guarded([&] { m->impl.synchronize(); });
}

int dv3_submit(dv3_model *m, const float *pixels, size_t n, float *out, size_t out_n,
               uint64_t *ticket) {
  if (int rc = check_model(m)) return rc;
  if (!ticket) return fail(DV3_INVALID_ARGUMENT, "null ticket");
  return guarded([&] { *ticket = m->impl.submit(pixels, n, out, out_n); });
}

int dv3_wait(dv3_model *m, uint64_t ticket) {
  if (!m) return fail(DV3_INVALID_ARGUMENT, "null model");
  // a poisoned model still reports each ticket's own status, then DV3_POISONED afterwards
  return guarded([&] { m->impl.wait(ticket); });
}

int dv3_forward_device(dv3_model *m, const float *pixels, size_t n, float *out, size_t out_n) {
  if (int rc = check_model(m)) return rc;
  return guarded([&] { m->impl.forward_device(pixels, n, out, out_n); });
}

int dv3_launches_per_forward(dv3_model *m, size_t batch, size_t *out) {
  if (int rc = check_model(m)) return rc;
  if (!out) return fail(DV3_INVALID_ARGUMENT, "null output");
  return guarded([&] { *out = m->impl.launches_per_forward(batch); });
}

int dv3_profile_launches(dv3_model *m, size_t batch, size_t iterations, double *ms,
                         const char **names, size_t capacity, size_t *count) {
  if (int rc = check_model(m)) return rc;
  return guarded([&] {
    auto r = m->impl.profile_launches(batch, iterations);
    for (size_t i = 0; i < r.size() && i < capacity; ++i) {
      if (ms) ms[i] = r[i].second;
      if (names) names[i] = r[i].first;
    }
    if (count) *count = r.size();
  });
}

int dv3_profile_forward(dv3_model *m, size_t batch, size_t replays, size_t flush_bytes,
                        double *ms, const char **names, size_t capacity, size_t *count) {
  if (int rc = check_model(m)) return rc;
  return guarded([&] {
    auto r = m->impl.profile_forward(batch, replays, flush_bytes);
    for (size_t i = 0; i < r.size() && i < capacity; ++i) {
      if (ms) ms[i] = r[i].second;
      if (names) names[i] = r[i].first;
    }
    if (count) *count = r.size();
  });
}

int dv3_debug_inject_fault(dv3_model *m, uint32_t bits) {
  if (int rc = check_model(m)) return rc;
  return guarded([&] { m->impl.inject_fault(bits); });
}

int dv3_hub_weights(int offline, char *path, size_t capacity) {
  if (!path || capacity == 0) return fail(DV3_INVALID_ARGUMENT, "null path buffer");
  std::string p, err;
  if (!dv3::hub_weights(offline != 0, &p, &err)) return fail(DV3_WEIGHTS, err);
  if (p.size() + 1 > capacity)
    return fail(DV3_INVALID_ARGUMENT, "path buffer too small: " + std::to_string(p.size() + 1) +
                                          " bytes needed");
  std::memcpy(path, p.c_str(), p.size() + 1);
  return DV3_OK;
}

int dv3_pack_f16(const char *name, const float *values, size_t n, uint16_t *out, size_t *bad) {
  if ((n && (!values || !out)) || !name) return fail(DV3_INVALID_ARGUMENT, "null argument");
  std::string msg;
  const size_t at = dv3::pack_f16(name, values, n, out, &msg);
  if (bad) *bad = at;
  if (at != SIZE_MAX) return fail(DV3_WEIGHTS, msg);
  return DV3_OK;
}

// ------------------------------------------------------------------------------------------
// Per-kernel entry points
// ------------------------------------------------------------------------------------------

}  // extern "C"

namespace {

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return DV3_OK;
  cudaGetLastError();
  return fail(DV3_DEVICE, std::string(what) + ": " + cudaGetErrorString(e));
}

template <class... P>
bool all_aligned(P... p) {
  return (aligned16(p) && ...);
}

int bad_args(const char *what) { return fail(DV3_INVALID_ARGUMENT, what); }

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int gemm_entry(dv3::GemmOp op, const void *a, uint32_t rows, const void *w,
               const dv3::GemmArgs &args, uint32_t *status, void *stream,
               const void *w_aux = nullptr) {
  if (rows == 0) return DV3_OK;
  dv3::GemmMaps maps;
  std::string err;
  const bool ln = op == dv3::GemmOp::ResidLN384 || op == dv3::GemmOp::ResidLN1536;
  const void *ln_out = args.ln_out_f32 ? static_cast<const void *>(args.ln_out_f32)
                                       : static_cast<const void *>(args.ln_out);
  if (!dv3::make_gemm_maps(op, a, rows, w, args.out, &maps, &err, ln ? ln_out : nullptr,
                           args.ln_out_f32 != nullptr))
    return bad_args(err.c_str());
  if (w_aux && !dv3::make_fold_maps(op, args.row_aux, rows, w_aux, &maps, &err))
    return bad_args(err.c_str());
  return launch_status(dv3::launch_gemm(op, maps, rows, args, status, static_cast<cudaStream_t>(stream)),
                       dv3::gemm_name(op));
}

}  // namespace

extern "C" {

int dv3k_bounded_wait_selftest(uint64_t wait_ns, uint32_t *status, void *stream) {
  if (!status) return bad_args("null status");
  if (wait_ns == 0 || wait_ns > 1000000000ull) return bad_args("wait_ns must be 1..1e9");
  return launch_status(dv3::launch_bounded_wait_selftest(wait_ns, status,
                                                         static_cast<cudaStream_t>(stream)),
                       "bounded wait self-test");
}

int dv3k_patchify(const float *images, uint32_t n_images, const float *prefix, uint16_t *patches,
                  uint16_t *x, uint32_t *status, void *stream) {
  if (n_images == 0) return DV3_OK;
  if (!all_aligned(images, prefix, patches, x)) return bad_args("pointers must be 16-byte aligned");
  return launch_status(dv3::launch_patchify(images, n_images, prefix, reinterpret_cast<__half *>(patches),
                                            reinterpret_cast<__half *>(x), status,
                                            static_cast<cudaStream_t>(stream)),
                       "patchify");
}

int dv3k_patch_embed(const uint16_t *patches, uint32_t n_patches, const uint16_t *w,
                     const float *bias, uint16_t *x, uint32_t *status, void *stream) {
  if (!all_aligned(patches, w, bias, x)) return bad_args("pointers must be 16-byte aligned");
  if (n_patches % dv3::kPatches != 0) return bad_args("n_patches must be a multiple of 196");
  dv3::GemmArgs g;
  g.bias = bias;
  g.out = reinterpret_cast<__half *>(x);
  return gemm_entry(dv3::GemmOp::Patch, patches, n_patches, w, g, status, stream);
}

int dv3k_layernorm_f16(const uint16_t *x, uint32_t rows, const float *gamma, const float *beta,
                       uint16_t *out, void *stream) {
  if (!all_aligned(x, gamma, beta, out)) return bad_args("pointers must be 16-byte aligned");
  return launch_status(dv3::launch_layernorm_f16(reinterpret_cast<const __half *>(x), rows, gamma, beta,
                                                 reinterpret_cast<__half *>(out),
                                                 static_cast<cudaStream_t>(stream)),
                       "layernorm_f16");
}

int dv3k_layernorm_f32out(const uint16_t *x, uint32_t rows, const float *gamma, const float *beta,
                          float *out, void *stream) {
  if (!all_aligned(x, gamma, beta, out)) return bad_args("pointers must be 16-byte aligned");
  return launch_status(dv3::launch_layernorm_f32(reinterpret_cast<const __half *>(x), rows, gamma, beta,
                                                 out, static_cast<cudaStream_t>(stream)),
                       "layernorm_f32out");
}

int dv3k_qkv_rope(const uint16_t *h, uint32_t rows, const uint16_t *w, const float *bias,
                  const float *rope_cos, const float *rope_sin, uint16_t *qkv, uint32_t *status,
                  void *stream) {
  if (!all_aligned(h, w, bias, rope_cos, rope_sin, qkv)) return bad_args("pointers must be 16-byte aligned");
  dv3::GemmArgs g;
  g.bias = bias;
  g.rope_cos = rope_cos;
  g.rope_sin = rope_sin;
  g.out = reinterpret_cast<__half *>(qkv);
  return gemm_entry(dv3::GemmOp::QkvRope, h, rows, w, g, status, stream);
}

int dv3k_attention(const uint16_t *qkv, uint32_t rows, uint16_t *out, uint32_t *status, void *stream) {
  if (rows == 0) return DV3_OK;
  if (!all_aligned(qkv, out)) return bad_args("pointers must be 16-byte aligned");
  if (rows % dv3::kTokens != 0) return bad_args("rows must be a multiple of 201");
  dv3::AttentionMaps map;
  std::string err;
  if (!dv3::make_attention_map(qkv, out, rows, &map, &err)) return bad_args(err.c_str());
  return launch_status(dv3::launch_attention(map, rows, status, static_cast<cudaStream_t>(stream)),
                       "attention");
}

int dv3k_matmul_splitk(const uint16_t *a, uint32_t rows, const uint16_t *w, uint32_t splits,
                       float *partials, uint32_t *status, void *stream) {
  if (!all_aligned(a, w, partials)) return bad_args("pointers must be 16-byte aligned");
  if (splits == 0 || (dv3::kMlp / 64) % splits != 0)
    return bad_args("splits must divide 24 (the 64-wide k-blocks of 1536)");
  if (rows == 0) return DV3_OK;
  dv3::GemmMaps maps;
  std::string err;
  if (!dv3::make_gemm_maps(dv3::GemmOp::SplitK1536, a, rows, w, partials, &maps, &err, nullptr,
                           false, splits))
    return bad_args(err.c_str());
  dv3::GemmArgs g;
  g.partials = partials;
  g.splits = splits;
  return launch_status(dv3::launch_gemm(dv3::GemmOp::SplitK1536, maps, rows, g, status,
                                        static_cast<cudaStream_t>(stream)),
                       dv3::gemm_name(dv3::GemmOp::SplitK1536));
}

int dv3k_splitk_reduce(const float *partials, uint32_t rows, uint32_t splits, const float *bias,
                       const float *lambda, uint16_t *x, void *stream) {
  if (!all_aligned(partials, bias, lambda, x)) return bad_args("pointers must be 16-byte aligned");
  if (splits == 0 || splits > 24) return bad_args("splits must be 1..24");
  return launch_status(dv3::launch_splitk_reduce(partials, rows, splits, bias, lambda,
                                                 reinterpret_cast<__half *>(x), nullptr, nullptr,
                                                 nullptr, nullptr, static_cast<cudaStream_t>(stream)),
                       "splitk_reduce");
}

int dv3k_splitk_reduce_layernorm(const float *partials, uint32_t rows, uint32_t splits,
                                 const float *bias, const float *lambda, uint16_t *x,
                                 const float *gamma, const float *beta, uint16_t *h,
                                 float *out_f32, void *stream) {
  if (!all_aligned(partials, bias, lambda, x, gamma, beta, h, out_f32))
    return bad_args("pointers must be 16-byte aligned");
  if (splits == 0 || splits > 24) return bad_args("splits must be 1..24");
  if ((h == nullptr) == (out_f32 == nullptr)) return bad_args("exactly one of h and out_f32");
  return launch_status(dv3::launch_splitk_reduce(partials, rows, splits, bias, lambda,
                                                 reinterpret_cast<__half *>(x), gamma, beta,
                                                 reinterpret_cast<__half *>(h), out_f32,
                                                 static_cast<cudaStream_t>(stream)),
                       "splitk_reduce_layernorm");
}

int dv3k_down_splitk_noalloc(const uint16_t *a, uint32_t rows, const uint16_t *w, uint32_t splits,
                             const float *bias, const float *lambda, uint16_t *x, uint32_t *status,
                             void *stream) {
  if (!all_aligned(a, w, bias, lambda, x)) return bad_args("pointers must be 16-byte aligned");
  if (splits == 0 || (dv3::kMlp / 64) % splits != 0)
    return bad_args("splits must divide 24 (the 64-wide k-blocks of 1536)");
  if (rows == 0) return DV3_OK;
  size_t capacity = 0;
  float *partials = dv3::splitk_scratch(&capacity);
  if (!partials) return fail(DV3_DEVICE, "split-K scratch: no device address");
  if (static_cast<size_t>(splits) * rows * dv3::kHidden > capacity)
    return bad_args("splits x rows exceeds the 6144 partial rows of the no-alloc scratch");
  dv3::GemmMaps maps;
  std::string err;
  if (!dv3::make_gemm_maps(dv3::GemmOp::SplitK1536, a, rows, w, partials, &maps, &err, nullptr,
                           false, splits))
    return bad_args(err.c_str());
  dv3::GemmArgs g;
  g.partials = partials;
  g.splits = splits;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rc = launch_status(dv3::launch_gemm(dv3::GemmOp::SplitK1536, maps, rows, g, status, s),
                               dv3::gemm_name(dv3::GemmOp::SplitK1536));
  if (rc != DV3_OK) return rc;
  return launch_status(dv3::launch_splitk_reduce(partials, rows, splits, bias, lambda,
                                                 reinterpret_cast<__half *>(x), nullptr, nullptr,
                                                 nullptr, nullptr, s),
                       "splitk_reduce");
}

int dv3k_matmul_resid(const uint16_t *a, uint32_t rows, uint32_t k, const uint16_t *w,
                      const float *bias, const float *lambda, uint16_t *x, uint32_t *status,
                      void *stream) {
  if (!all_aligned(a, w, bias, lambda, x)) return bad_args("pointers must be 16-byte aligned");
  if (k != 384 && k != 1536) return bad_args("k must be 384 or 1536");
  dv3::GemmArgs g;
  g.bias = bias;
  g.lambda = lambda;
  g.out = reinterpret_cast<__half *>(x);
  return gemm_entry(k == 384 ? dv3::GemmOp::Resid384 : dv3::GemmOp::Resid1536, a, rows, w, g, status,
                    stream);
}

int dv3k_matmul_resid_layernorm(const uint16_t *a, uint32_t rows, uint32_t k, const uint16_t *w,
                                const float *bias, const float *lambda, uint16_t *x,
                                const float *gamma, const float *beta, uint16_t *h,
                                float *out_f32, uint32_t *status, void *stream) {
  if (!all_aligned(a, w, bias, lambda, x, gamma, beta, h, out_f32))
    return bad_args("pointers must be 16-byte aligned");
  if (k != 384 && k != 1536) return bad_args("k must be 384 or 1536");
  if ((h == nullptr) == (out_f32 == nullptr)) return bad_args("exactly one of h and out_f32");
  if (rows > 128u * static_cast<uint32_t>(dv3::sm_count(current_device())))
    return bad_args("rows must fit one 128-row tile per SM");
  dv3::GemmArgs g;
  g.bias = bias;
  g.lambda = lambda;
  g.out = reinterpret_cast<__half *>(x);
  g.gamma = gamma;
  g.beta = beta;
  g.ln_out = reinterpret_cast<__half *>(h);
  g.ln_out_f32 = out_f32;
  return gemm_entry(k == 384 ? dv3::GemmOp::ResidLN384 : dv3::GemmOp::ResidLN1536, a, rows, w, g,
                    status, stream);
}

int dv3k_matmul_swiglu(const uint16_t *h, uint32_t rows, const uint16_t *gateup_w,
                       const float *gateup_b, uint16_t *act, uint32_t *status, void *stream) {
  if (!all_aligned(h, gateup_w, gateup_b, act)) return bad_args("pointers must be 16-byte aligned");
  dv3::GemmArgs g;
  g.bias = gateup_b;
  g.out = reinterpret_cast<__half *>(act);
  return gemm_entry(dv3::GemmOp::SwiGLU, h, rows, gateup_w, g, status, stream);
}

int dv3k_matmul_resid_rowstat(const uint16_t *a, uint32_t rows, uint32_t k, const uint16_t *w,
                              const float *bias, const float *lambda, uint16_t *x, float *rowstat,
                              uint16_t *row_aux, uint32_t *status, void *stream) {
  if (!all_aligned(a, w, bias, lambda, x, rowstat, row_aux))
    return bad_args("pointers must be 16-byte aligned");
  if (k != 384 && k != 1536) return bad_args("k must be 384 or 1536");
  if (rowstat == nullptr || row_aux == nullptr) return bad_args("rowstat and row_aux are required");
  if (rows > 128u * static_cast<uint32_t>(dv3::sm_count(current_device())))
    return bad_args("rows must fit one 128-row tile per SM");
  dv3::GemmArgs g;
  g.bias = bias;
  g.lambda = lambda;
  g.out = reinterpret_cast<__half *>(x);
  g.rowstat = reinterpret_cast<float2 *>(rowstat);
  g.row_aux = reinterpret_cast<__half *>(row_aux);
  return gemm_entry(k == 384 ? dv3::GemmOp::ResidStats384 : dv3::GemmOp::ResidStats1536, a, rows,
                    w, g, status, stream);
}

int dv3k_layernorm_rowstat(const uint16_t *x, uint32_t rows, float *rowstat, uint16_t *row_aux,
                           void *stream) {
  if (!all_aligned(x, rowstat, row_aux)) return bad_args("pointers must be 16-byte aligned");
  if (rowstat == nullptr || row_aux == nullptr) return bad_args("rowstat and row_aux are required");
  return launch_status(dv3::launch_layernorm_rowstat(reinterpret_cast<const __half *>(x), rows,
                                                     reinterpret_cast<float2 *>(rowstat),
                                                     reinterpret_cast<__half *>(row_aux),
                                                     static_cast<cudaStream_t>(stream)),
                       "layernorm_rowstat");
}

int dv3k_qkv_rope_folded(const uint16_t *x, uint32_t rows, const uint16_t *wf,
                         const uint16_t *w_aux, const float *rowstat, const uint16_t *row_aux,
                         const float *rope_cos, const float *rope_sin, uint16_t *qkv,
                         uint32_t *status, void *stream) {
  if (!all_aligned(x, wf, w_aux, rowstat, row_aux, rope_cos, rope_sin, qkv))
    return bad_args("pointers must be 16-byte aligned");
  if (w_aux == nullptr || rowstat == nullptr || row_aux == nullptr)
    return bad_args("w_aux, rowstat and row_aux are required");
  dv3::GemmArgs g;
  g.rowstat = reinterpret_cast<float2 *>(const_cast<float *>(rowstat));
  g.row_aux = reinterpret_cast<__half *>(const_cast<uint16_t *>(row_aux));
  g.rope_cos = rope_cos;
  g.rope_sin = rope_sin;
  g.out = reinterpret_cast<__half *>(qkv);
  return gemm_entry(dv3::GemmOp::QkvRopeFold, x, rows, wf, g, status, stream, w_aux);
}

int dv3k_matmul_swiglu_folded(const uint16_t *x, uint32_t rows, const uint16_t *gateup_wf,
                              const uint16_t *w_aux, const float *rowstat,
                              const uint16_t *row_aux, uint16_t *act, uint32_t *status,
                              void *stream) {
  if (!all_aligned(x, gateup_wf, w_aux, rowstat, row_aux, act))
    return bad_args("pointers must be 16-byte aligned");
  if (w_aux == nullptr || rowstat == nullptr || row_aux == nullptr)
    return bad_args("w_aux, rowstat and row_aux are required");
  dv3::GemmArgs g;
  g.rowstat = reinterpret_cast<float2 *>(const_cast<float *>(rowstat));
  g.row_aux = reinterpret_cast<__half *>(const_cast<uint16_t *>(row_aux));
  g.out = reinterpret_cast<__half *>(act);
  return gemm_entry(dv3::GemmOp::SwiGLUFold, x, rows, gateup_wf, g, status, stream, w_aux);
}

uint32_t dv3k_gateup_source_row(uint32_t packed_row) { return dv3::gateup_source_row(packed_row); }

}  // extern "C"
