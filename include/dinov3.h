/*
 * dinov3.h - C ABI of the B200 (sm_100a) DINOv3 ViT-S+/16 forward.
 *
 * This is the drop-in boundary for the reference crate's public model API (src/lib.rs of
 * zacharydenton/dinov3-loom, crate `dinov3-hrx`). Each entry point below names the Rust item it
 * replaces. Conventions follow the reference:
 *   - A model owns its device, stream, packed weights, resident activations (sized for
 *     `max_batch` images), one CUDA graph per batch size it has seen, and its error state.
 *   - The caller owns every host buffer it passes; the library never keeps a pointer to one.
 *   - One caller per model at a time (the reference takes `&mut self`); separate models are
 *     independent and may run concurrently, one per device or several on one device.
 *   - Errors: every function returning int returns 0 on success or a nonzero DV3_* status.
 *     dv3_last_error() then gives the message of the calling thread's last failure. The texts
 *     carry the reference's messages ("max_batch must be 1..=64", "input must contain complete
 *     3x224x224 images", "input must be finite", "tensor patch_w[0] cannot be represented as
 *     finite float16: ...", "session is unusable after a GPU failure").
 *   - After a CUDA error or a device-side timeout the model is poisoned: every later call
 *     returns DV3_POISONED (src/engine.rs:36,93,168-171,198-200,210-212,265-267).
 *
 * Shapes: an image is 3x224x224 normalised float32 NCHW (DV3_IMAGE_ELEMENTS floats); the output
 * of one image is 201 tokens x 384 float32 (CLS, 4 registers, 196 patches).
 */
#ifndef DINOV3_H
#define DINOV3_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define DV3_IMAGE_ELEMENTS (3 * 224 * 224) /* src/lib.rs:11 */
#define DV3_TOKENS 201                     /* src/lib.rs:12 */
#define DV3_HIDDEN 384                     /* src/lib.rs:13 */
#define DV3_MAX_BATCH_LIMIT 64

enum {
  DV3_OK = 0,
  DV3_INVALID_ARGUMENT = 1, /* options, shapes, non-finite or incomplete input */
  DV3_WEIGHTS = 2,          /* unreadable, malformed or unrepresentable weights */
  DV3_DEVICE = 3,           /* no usable sm_100 device, or a CUDA call failed */
  DV3_POISONED = 4,         /* an earlier GPU failure made this model unusable */
};

typedef struct dv3_model dv3_model;

/* Options (src/lib.rs:15-27). Defaults: device 0, max_batch 32. */
typedef struct {
  int32_t device;
  size_t max_batch; /* resident capacity, 1..=64; larger inputs are processed in chunks */
} dv3_options;

/* Distribution / ForwardTimings (src/engine.rs:272-284): host-clock milliseconds. */
typedef struct {
  double median_ms;
  double p95_ms;
} dv3_distribution;

typedef struct {
  size_t samples;
  dv3_distribution graph;  /* one CUDA graph launch per sample */
  dv3_distribution direct; /* the same launch list issued kernel by kernel */
} dv3_timings;

dv3_options dv3_default_options(void);

/* DINOv3::load (src/lib.rs:49-88). Checks the options first (before touching the file), then
 * reads and packs the weights (before touching the GPU), then opens the device (which must be
 * sm_100), uploads, allocates and builds the kernels' state. */
int dv3_load(const char *safetensors_path, dv3_options options, dv3_model **out);

/* DINOv3::from_pretrained (src/lib.rs:40-46): checks max_batch, resolves the pinned weights with
 * dv3_hub_weights(0, ...) (a cache miss is DV3_WEIGHTS; nothing is downloaded), then dv3_load. */
int dv3_from_pretrained(dv3_options options, dv3_model **out);

/* DINOv3::forward (src/lib.rs:90-114). `pixels` holds n_floats = k*DV3_IMAGE_ELEMENTS floats
 * (k >= 0); `out` must have room for k*201*384 floats (out_floats). Synchronous. Inputs larger
 * than max_batch are processed in chunks of max_batch. Non-finite input is an error; it is
 * detected on the device while each chunk is read. On any error `out` is unspecified: the
 * chunks before the failing one, and the failing chunk itself, may already have been written
 * (the reference returns a fresh vector instead, src/lib.rs:90-114). Host buffers may be
 * pageable; pinned buffers transfer faster. */
int dv3_forward(dv3_model *m, const float *pixels, size_t n_floats, float *out, size_t out_floats);

/* DINOv3::cls (src/lib.rs:126-132): the CLS token of each image, k*384 floats. Only those
 * rows are copied back from the device. */
int dv3_cls(dv3_model *m, const float *pixels, size_t n_floats, float *out, size_t out_floats);

/* DINOv3::patch_mean (src/lib.rs:134-148): mean of the 196 patch tokens, k*384 floats,
 * reduced on the device in the reference's f32 order (row / 196 added for rows 5..200), so it
 * equals the reference's host loop over the full output bit for bit; only the means are copied
 * back. */
int dv3_patch_mean(dv3_model *m, const float *pixels, size_t n_floats, float *out,
                   size_t out_floats);

/* DINOv3::benchmark (src/lib.rs:116-124, src/engine.rs:130-190): stages one non-empty batch of
 * at most max_batch images, then alternates graph replay and direct dispatch for 10 warm-up
 * plus `samples` (>= 10) rounds, each synchronised and timed with the host clock. */
int dv3_benchmark(dv3_model *m, const float *pixels, size_t n_floats, size_t samples,
                  dv3_timings *out);

/* Drop the model and every device resource it owns. NULL is allowed. */
void dv3_free(dv3_model *m);

/* Message of the calling thread's last failure ("" if none). Valid until the next call on
 * this thread. */
const char *dv3_last_error(void);

/* ---- Device-resident path (no reference counterpart: the reference always copies through
 * host memory). For callers whose images are already in device memory of the model's device,
 * and for measurement. ---- */

/* The model's resident input buffer: max_batch*DV3_IMAGE_ELEMENTS floats of device memory on
 * the model's device. Images staged there are consumed by dv3_run. */
float *dv3_input_buffer(dv3_model *m);

/* The model's resident output buffer: max_batch*201*384 floats of device memory. */
float *dv3_output_buffer(dv3_model *m);

/* The model's CUDA stream (a cudaStream_t), on which all of its work is ordered. */
void *dv3_stream(dv3_model *m);

/* Enqueue one forward of the first `batch` images of the input buffer (1 <= batch <=
 * max_batch) into the output buffer, as one CUDA graph launch on the model's stream. Does not
 * wait. Non-finite input and device faults are reported by the next dv3_synchronize. */
int dv3_run(dv3_model *m, size_t batch);

/* Wait for the model's stream and report any error raised by work enqueued since the last
 * check (DV3_INVALID_ARGUMENT for non-finite input; DV3_POISONED for a device fault). */
int dv3_synchronize(dv3_model *m);

/* Serving path (no reference counterpart; the reference's forward is synchronous). Enqueue the
 * upload of k = n_floats/DV3_IMAGE_ELEMENTS images (1 <= k <= max_batch) from `pixels`, one
 * forward and the download of its k*201*384 floats into `out`, and return at once with a ticket.
 * Submissions alternate between two device buffer slots on three streams, so the upload of one
 * overlaps the forward of the previous and the download of the one before; a third outstanding
 * submission first completes the oldest (keeping its status for its own dv3_wait). The caller
 * keeps `pixels` and `out` valid and unchanged until dv3_wait(ticket) returns; pinned host memory
 * lets the copies overlap (pageable memory is staged synchronously by the CUDA driver).
 * Synchronous calls on the model (dv3_forward, dv3_run, ...) first complete every submission. */
int dv3_submit(dv3_model *m, const float *pixels, size_t n_floats, float *out, size_t out_floats,
               uint64_t *ticket);

/* Wait for one submission: 0 when its output is in `out`; DV3_INVALID_ARGUMENT for non-finite
 * input (`out` unspecified) or an unknown / already waited ticket; DV3_POISONED after a device
 * fault in that submission (the model is then unusable). */
int dv3_wait(dv3_model *m, uint64_t ticket);

/* dv3_forward on device pointers (same device as the model): copies each chunk into the input
 * buffer, runs it and copies its output out, all on the model's stream, then synchronises. */
int dv3_forward_device(dv3_model *m, const float *device_pixels, size_t n_floats,
                       float *device_out, size_t out_floats);

/* Number of kernel launches in one forward of `batch` images (the graph's kernel nodes). */
int dv3_launches_per_forward(dv3_model *m, size_t batch, size_t *out);

/* Per-kernel device time of the launches of one forward of `batch` staged images: each launch
 * of the plan is captured `iterations` times back to back into a CUDA graph, replayed once to
 * warm up and once between two events on the model's stream; its time is the interval divided
 * by `iterations`. Writes up to `capacity` entries (launch order) of average milliseconds and a
 * static kernel name, and the count to *count. Leaves the model's activations undefined (the
 * next forward recomputes them). */
int dv3_profile_launches(dv3_model *m, size_t batch, size_t iterations, double *ms,
                         const char **names, size_t capacity, size_t *count);

/* Per-launch device time of the launches of whole forwards of `batch` staged images, in the
 * plan's order, cache state and overlap: for every j the first j launches are captured into a
 * CUDA graph (programmatic dependencies between kernels, as in the forward's graph) and replayed
 * `replays` times between two CUDA events on the model's stream, each replay after a write of
 * `flush_bytes` bytes to a scratch buffer the call allocates (outside the events; evicts L2 when
 * larger than it; 0: no flush). With T(j) the mean time of the first j launches, launch j takes
 * T(j) - T(j-1), so the times add up to one forward. Writes up to `capacity` entries (launch
 * order) of milliseconds and static kernel names, and the count to *count. */
int dv3_profile_forward(dv3_model *m, size_t batch, size_t replays, size_t flush_bytes,
                        double *ms, const char **names, size_t capacity, size_t *count);

/* Test hook (no reference counterpart): the next forward enqueued on `m` (dv3_forward, dv3_cls,
 * dv3_patch_mean, dv3_run, dv3_submit, dv3_forward_device) writes the nonzero `bits` into the
 * model's device failure word after its kernels, where a kernel whose bounded wait expired
 * records its bit, so that forward reports DV3_POISONED and the model stays poisoned
 * (src/engine.rs:93,168-171), without faulting the GPU. Returns DV3_POISONED on a model that is
 * already poisoned. */
int dv3_debug_inject_fault(dv3_model *m, uint32_t bits);

/* ---- Pinned weights in the Hugging Face cache (src/hub.rs), usable without a GPU. ---- */

/* Path of facebook/dinov3-vits16plus-pretrain-lvd1689m at revision
 * c93d816fc9e567563bc068f01475bec89cc634a6, model.safetensors, in the shared Hugging Face cache
 * (HF_HUB_CACHE, else HF_HOME/hub, else XDG_CACHE_HOME/huggingface/hub, else
 * ~/.cache/huggingface/hub; .../models--facebook--dinov3-vits16plus-pretrain-lvd1689m/
 * snapshots/<revision>/model.safetensors), written NUL-terminated into `path`. Offline when
 * `offline` is nonzero or HF_HUB_OFFLINE is set to anything but "" or "0". A file that is not
 * cached gives DV3_WEIGHTS with the reference's message "<org>/<name> at <revision>:
 * model.safetensors is not cached and model downloads are disabled" (offline), or, since this
 * library has no network client, a "cannot download ..." message otherwise. */
int dv3_hub_weights(int offline, char *path, size_t capacity);

/* ---- Weight packing (src/weights.rs:6-17), usable without a GPU. ---- */

/* Round each float to IEEE binary16 (round to nearest, ties to even), failing on the first
 * value whose result is not finite: returns DV3_WEIGHTS with *bad_index set and the message
 * "tensor <name>[<index>] cannot be represented as finite float16: <value>". */
int dv3_pack_f16(const char *name, const float *values, size_t n, uint16_t *out,
                 size_t *bad_index);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif /* DINOV3_H */
