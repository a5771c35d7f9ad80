// model.h - the resident model: mirrors DINOv3 (src/lib.rs) and Engine (src/engine.rs).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <functional>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "dinov3.h"
#include "kernels.h"

namespace dv3 {

// An error with the C ABI status it maps to.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

struct LayerWeights {
  const __half *qkv_w, *gateup_w, *o_w, *down_w;
  const float *qkv_b, *gateup_b, *o_b, *down_b;
  const float *norm1_w, *norm1_b, *norm2_w, *norm2_b, *ls1, *ls2;
  // The QKV and gate/up projections with the LayerNorm before them folded in (weights.cpp):
  // W' = f16(W gamma) and the weight aux rows of the extra K=16 step.
  const __half *qkv_wf, *gateup_wf, *qkv_aux, *gateup_aux;
};

struct DeviceWeights {
  const __half *patch_w;
  const float *patch_b, *prefix, *norm_w, *norm_b, *rope_cos, *rope_sin;
  LayerWeights layer[12];
};

// One step of the launch plan (src/engine.rs:21-27): a named closure that enqueues one kernel
// (or, for the status clear, one memset) on a stream.
struct Launch {
  const char *name;
  bool kernel;
  std::function<cudaError_t(cudaStream_t)> enqueue;
};

struct Plan {
  std::vector<Launch> launches;
  cudaGraphExec_t exec = nullptr;
  size_t kernels = 0;
};


class Model {
 public:
  Model(const std::string &path, dv3_options options);
  ~Model();
  Model(const Model &) = delete;
  Model &operator=(const Model &) = delete;

  // What a forward returns to the host: every token (b x 201 x 384), the CLS token of each image
  // (b x 384; only those rows are read back), or the mean of the patch tokens (b x 384, reduced
  // on the device, only the means read back).
  enum class Readout { Full, Cls, PatchMean };
  void forward(const float *pixels, size_t n_floats, float *out, size_t out_floats,
               Readout readout = Readout::Full);
  void forward_device(const float *pixels, size_t n_floats, float *out, size_t out_floats);
  void run(size_t batch);
  void synchronize();
  // Serving path (no reference counterpart): enqueue upload, forward and download of one batch
  // of 1..=max_batch images without waiting, into one of two buffer slots, so that the upload
  // of one submission overlaps the forward of the previous one and the download of the one
  // before. `wait` blocks until that submission's output is in `out` and reports its errors.
  uint64_t submit(const float *pixels, size_t n_floats, float *out, size_t out_floats);
  void wait(uint64_t ticket);
  dv3_timings benchmark(const float *pixels, size_t n_floats, size_t samples);
  size_t launches_per_forward(size_t batch);
  std::vector<std::pair<const char *, double>> profile_launches(size_t batch, size_t iterations);
  // Per-launch device time inside whole forwards (see model.cpp).
  std::vector<std::pair<const char *, double>> profile_forward(size_t batch, size_t replays,
                                                               size_t flush_bytes);
  // Test hook (no reference counterpart): the next forward enqueued on this model (any path)
  // writes `bits` into the device failure word after its kernels, as a kernel whose bounded wait
  // expired would, so the host sees a device failure without one.
  void inject_fault(uint32_t bits);

  float *input_buffer() const { return image_; }
  float *output_buffer() const { return out_; }
  cudaStream_t stream() const { return stream_; }
  size_t max_batch() const { return max_batch_; }

 private:
  void check_usable() const;
  void cuda(cudaError_t e, const char *what);  // poisons and throws on failure
  Plan &prepare(size_t batch, int slot = 0);    // build + capture once per batch size and slot
  void drain();                                  // finish every outstanding submission
  bool fuse_layernorm(size_t batch) const;      // plan variant for this batch size
  int fold_layernorm(size_t batch) const;       // LayerNorms folded into QKV (1), gate/up (2)
  uint32_t down_splits(uint32_t rows) const;    // split-K slices of the down projection
  void check_status();                          // read the device status words (synchronous)
  void activate() const;
  void release();  // free every device resource (idempotent)

  int device_;
  size_t max_batch_;
  bool failed_ = false;
  cudaStream_t stream_ = nullptr;      // the forward (compute) stream
  cudaStream_t h2d_stream_ = nullptr;  // serving uploads
  cudaStream_t d2h_stream_ = nullptr;  // serving downloads
  void *weight_blob_ = nullptr;
  void *act_blob_ = nullptr;
  DeviceWeights w_{};
  __half *x_ = nullptr, *h_ = nullptr, *qkv_ = nullptr, *attn_ = nullptr, *act_ = nullptr,
         *patches_ = nullptr;
  float *image_ = nullptr, *out_ = nullptr, *pmean_ = nullptr;
  float *partials_ = nullptr;  // split-K partial slabs of the down projection
  float2 *rowstat_ = nullptr;  // per token row (rstd, -mean rstd) of the folded LayerNorm
  __half *row_aux_ = nullptr;  // per token row: its aux row of the folded LayerNorm [201B][16]
  float *image_slot_[2] = {}, *out_slot_[2] = {};  // slot 0 aliases image_ / out_
  // Per slot: upload done, forward done (input consumed, output ready), download done.
  cudaEvent_t ev_in_[2] = {}, ev_done_[2] = {}, ev_out_[2] = {};
  uint32_t *slot_status_host_ = nullptr;  // pinned [2][2]: each submission's status words
  uint64_t next_ticket_ = 0;
  bool submitted_[2] = {};     // the slot holds a submission nobody has waited for yet
  uint64_t slot_ticket_[2] = {};
  std::map<uint64_t, std::pair<uint32_t, uint32_t>> finished_;  // completed, not yet waited
  void retire(int slot);       // complete the slot's submission and keep its status words
  uint32_t *status_ = nullptr;       // device: [0] failure bits, [1] non-finite input
  uint32_t *status_host_ = nullptr;  // pinned mirror
  bool status_pending_ = false;      // work enqueued since the last status check
  uint32_t *inject_host_ = nullptr;  // pinned: the failure bits inject_fault asked for
  bool inject_pending_ = false;
  void apply_injection();            // enqueue the injected failure bits (if any) on stream_
  std::map<std::pair<size_t, int>, Plan> plans_;
};

}  // namespace dv3
