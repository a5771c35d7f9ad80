// attention_softmax.cuh - the per-row softmax and output staging of the attention kernel
// (attention.cu), on S and O held in tensor memory.
//
// One query row per thread (its TMEM lane). Pass 1: row max over the 201 valid keys. Pass 2:
// w = exp(0.125 (s - max)) = 2^(s c - max c) with c = 0.125 log2(e) (one FFMA and the hardware
// exp2), f32 sum of w, P = f16(w) (keys >= 201 zero) stored to TMEM over the consumed S. The
// probabilities are rounded to f16 before PV and the normaliser is the f32 sum of the unrounded
// weights, as in kernels/attention_online_f16_wmma_cf16.loom:214-216.
#pragma once

#include "kernels.h"
#include "sm100.cuh"

namespace dv3 {
namespace attn {

constexpr int kHeads = 6;
constexpr int kValidKeys = kTokens;  // 201
constexpr int kSKeys = 208;          // S columns computed (201 rounded up to 16)
constexpr int kOutBox = 32;          // token rows per output store (one warp's rows)
constexpr int kTileCols = 256;       // TMEM columns per query tile
constexpr int kOCol = 128;           // O_t within the tile's columns
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// w = 2^(s c - mc) for one pair of keys, summed into `sum`, returned as packed f16.
__device__ __forceinline__ uint32_t exp_pair(uint32_t s0, uint32_t s1, float mc, float &sum,
                                             bool v0 = true, bool v1 = true) {
  const float p0 = v0 ? ex2_approx(fmaf(__uint_as_float(s0), kScaleLog2, -mc)) : 0.f;
  const float p1 = v1 ? ex2_approx(fmaf(__uint_as_float(s1), kScaleLog2, -mc)) : 0.f;
  sum += p0 + p1;
  return pack_half2(p0, p1);
}

// Softmax of one query row whose S sits in TMEM columns tl..tl+207 (this thread's lane): stores
// P over columns tl..tl+103 and returns the f32 sum of the weights. Both passes walk S in
// 32-column chunks and load chunk c+1 while computing on chunk c. Each P store lands on S
// columns that this thread has already read.
__device__ __forceinline__ float softmax_row(uint32_t tl) {
  uint32_t x[32], y[32];
  float m0 = -INFINITY, m1 = -INFINITY;
  auto max_chunk = [&](uint32_t (&v)[32], int n) {
#pragma unroll
    for (int i = 0; i + 1 < n; i += 4) {
      m0 = max3(m0, __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
      if (i + 3 < n) m1 = max3(m1, __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
      else if (i + 2 < n) m1 = fmaxf(m1, __uint_as_float(v[i + 2]));
    }
    if (n % 2) m0 = fmaxf(m0, __uint_as_float(v[n - 1]));
  };
  // Pass 1: chunks 0..5 (32 keys each) and keys 192..200 of chunk 6.
  tmem_load32(tl, x);
#pragma unroll
  for (int c = 0; c < 6; c += 2) {
    tmem_ld32(tl + (c + 1) * 32, y);
    max_chunk(x, 32);
    tmem_wait_ld(y);
    tmem_ld32(tl + (c + 2) * 32, x);  // c + 2 == 6: columns 192..223 (only 192..200 are used)
    max_chunk(y, 32);
    tmem_wait_ld(x);
  }
  max_chunk(x, kValidKeys - 192);
  const float mc = fmaxf(m0, m1) * kScaleLog2;

  // Pass 2: keys 32c .. 32c+31 -> P columns 16c .. 16c+15.
  float sum = 0.f;
  auto exp_chunk = [&](uint32_t (&v)[32], int c) {
    uint32_t p[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) p[j] = exp_pair(v[2 * j], v[2 * j + 1], mc, sum);
    tmem_st16(tl + c * 16, p);
  };
  tmem_load32(tl, x);
#pragma unroll
  for (int c = 0; c < 6; c += 2) {
    tmem_ld32(tl + (c + 1) * 32, y);
    exp_chunk(x, c);
    tmem_wait_ld(y);
    if (c + 2 < 6) {
      tmem_ld32(tl + (c + 2) * 32, x);
      exp_chunk(y, c + 1);
      tmem_wait_ld(x);
    } else {
      exp_chunk(y, c + 1);
    }
  }
  uint32_t e[16];
  tmem_ld16(tl + 192, e);  // keys 192..207 -> P columns 96..103
  tmem_ld_wait();
  tmem_regs_ready16(e);
  uint32_t pe[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    pe[j] = exp_pair(e[2 * j], e[2 * j + 1], mc, sum, 192 + 2 * j < kValidKeys,
                     192 + 2 * j + 1 < kValidKeys);
  tmem_st8(tl + 96, pe);
  return sum;
}

__device__ __forceinline__ uint32_t scaled_pair(uint32_t a, uint32_t b, float inv) {
  return pack_half2(__uint_as_float(a) * inv, __uint_as_float(b) * inv);
}

// This warp's 32 rows of O (TMEM columns tl+kOCol..+63, one row per lane) divided by the row's
// softmax sum, rounded to f16, into a 32-row staging block of 128-byte rows with the 128-byte
// swizzle (row r's 16-byte chunk j at chunk j ^ (r & 7)), the layout of a 64-column TMA box.
__device__ __forceinline__ void stage_output_row(uint8_t *stg_row, int lane, const uint32_t (&o0)[32],
                                                 const uint32_t (&o1)[32], float inv) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    *reinterpret_cast<uint4 *>(stg_row + ((j ^ (lane & 7)) * 16)) =
        make_uint4(scaled_pair(o0[8 * j], o0[8 * j + 1], inv),
                   scaled_pair(o0[8 * j + 2], o0[8 * j + 3], inv),
                   scaled_pair(o0[8 * j + 4], o0[8 * j + 5], inv),
                   scaled_pair(o0[8 * j + 6], o0[8 * j + 7], inv));
    *reinterpret_cast<uint4 *>(stg_row + (((4 + j) ^ (lane & 7)) * 16)) =
        make_uint4(scaled_pair(o1[8 * j], o1[8 * j + 1], inv),
                   scaled_pair(o1[8 * j + 2], o1[8 * j + 3], inv),
                   scaled_pair(o1[8 * j + 4], o1[8 * j + 5], inv),
                   scaled_pair(o1[8 * j + 6], o1[8 * j + 7], inv));
  }
}

}  // namespace attn
}  // namespace dv3
