// weights.h - safetensors reading and the load-time packing contract (src/weights.rs).
#pragma once

#include <stdint.h>

#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace dv3 {

// Error raised while reading or packing weights; what() is the user-facing message.
struct WeightsError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// IEEE binary16 conversions with round-to-nearest-even (the narrowing of half 2.7.1's
// f16::from_f32, src/weights.rs:9).
uint16_t f32_to_f16(float v);
float f16_to_f32(uint16_t h);
float bf16_to_f32(uint16_t h);

// pack_f16 (src/weights.rs:6-17): fails on the first value that does not narrow to a finite
// f16, with "tensor <name>[<index>] cannot be represented as finite float16: <value>".
// Returns the index of that value, or SIZE_MAX when every value packed.
size_t pack_f16(const std::string &name, const float *values, size_t n, uint16_t *out,
                std::string *message);

// Shortest decimal that reads back as the same float (how Rust displays an f32).
std::string format_f32(float v);

// One packed tensor: f16 payload for matrices, f32 for vectors.
struct Packed {
  bool half = false;
  std::vector<uint16_t> h;
  std::vector<float> f;
  size_t bytes() const { return half ? h.size() * 2 : f.size() * 4; }
  const void *data() const { return half ? static_cast<const void *>(h.data()) : f.data(); }
};

// Read `path` (safetensors; F32, F16 or BF16 tensors with Hugging Face names) and produce the
// packed tensors keyed by the reference's short names (patch_w, patch_b, prefix, l{i}_qkv_w,
// l{i}_qkv_b, l{i}_gateup_w, l{i}_gateup_b, l{i}_o_w, ..., norm_w, norm_b, rope_cos, rope_sin),
// validating in the reference's order so that the first error is the same one.
// gateup_w / gateup_b are then re-ordered into the kernel's interleaved layout.
std::map<std::string, Packed> load_weights(const std::string &path);

}  // namespace dv3
