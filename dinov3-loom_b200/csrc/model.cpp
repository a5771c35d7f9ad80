// model.cpp - the resident model: load (src/lib.rs:49-88), the launch plan (src/lib.rs:149-263),
// one CUDA graph per batch size (src/engine.rs:87-129), forward with chunking
// (src/lib.rs:90-114), and the graph-vs-direct benchmark (src/engine.rs:130-190).
//
// Device memory: one allocation holds every packed weight (f16 matrices, f32 vectors, 256-byte
// aligned), one holds the activations sized for max_batch images:
//   image   f32 [B][3][224][224]   the staged input
//   patches f16 [196B][768]        patchified input (A operand of the patch GEMM)
//   x       f16 [201B][384]        residual stream
//   h       f16 [201B][384]        LayerNorm output
//   qkv     f16 [201B][1152]       q | k | v (RoPE applied)
//   attn    f16 [201B][384]        attention output
//   act     f16 [201B][1536]       SwiGLU output
//   out     f32 [201B][384]        final LayerNorm output
//   status  u32 [2]                device failure bits, non-finite input flag (sticky until read)
//   pmean   f32 [B][384]           patch-token means (patch_mean readout)
//   rowstat f32 [201B][2]          (rstd, -mean rstd) of each token row, and
//   row_aux f16 [201B][16]         its aux row: the LayerNorm that the QKV and gate/up GEMMs
//                                  apply themselves (folded plan)
//   image1, out1                   the second serving slot's input and output (slot 0 uses
//                                  image and out)
// The QKV buffer needs no headroom rows: attention reads through TMA, whose out-of-bounds rows
// are zero.
#include "model.h"

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>

#include "weights.h"

namespace dv3 {

cudaError_t configure_gemm_kernels();
cudaError_t configure_attention_kernel();

namespace {
size_t align256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }
}  // namespace

void Model::activate() const { cudaSetDevice(device_); }

void Model::cuda(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return;
  failed_ = true;
  cudaGetLastError();  // clear a non-sticky error so later host calls report afresh
  throw Error(DV3_DEVICE, std::string(what) + ": " + cudaGetErrorString(e));
}

void Model::check_usable() const {
  if (failed_) throw Error(DV3_POISONED, "session is unusable after a GPU failure");
}

Model::Model(const std::string &path, dv3_options options)
    : device_(options.device), max_batch_(options.max_batch) {
  // Options first, before any file access (tests/model.rs:5-27).
  if (options.max_batch < 1 || options.max_batch > DV3_MAX_BATCH_LIMIT)
    throw Error(DV3_INVALID_ARGUMENT, "max_batch must be 1..=64");
  // Weights next, before any GPU initialisation (tests/model.rs:29-59).
  std::map<std::string, Packed> packed;
  try {
    packed = load_weights(path);
  } catch (const WeightsError &e) {
    throw Error(DV3_WEIGHTS, e.what());
  }
  // Engine::new (src/engine.rs:40-46): the kernels are built for sm_100a only.
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    throw Error(DV3_DEVICE, "no CUDA device is available");
  }
  if (device_ < 0 || device_ >= count)
    throw Error(DV3_DEVICE, "CUDA device " + std::to_string(device_) + " does not exist");
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device_) != cudaSuccess)
    throw Error(DV3_DEVICE, "cannot query CUDA device " + std::to_string(device_));
  if (prop.major != 10 || prop.minor != 0)
    throw Error(DV3_DEVICE, "these kernels are built for sm_100 (B200), found sm_" +
                                std::to_string(prop.major) + std::to_string(prop.minor));
  activate();
  try {
    cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "create stream");
    cuda(cudaStreamCreateWithFlags(&h2d_stream_, cudaStreamNonBlocking), "create stream");
    cuda(cudaStreamCreateWithFlags(&d2h_stream_, cudaStreamNonBlocking), "create stream");
    for (int i = 0; i < 2; ++i) {
      cuda(cudaEventCreateWithFlags(&ev_in_[i], cudaEventDisableTiming), "create event");
      cuda(cudaEventCreateWithFlags(&ev_done_[i], cudaEventDisableTiming), "create event");
      cuda(cudaEventCreateWithFlags(&ev_out_[i], cudaEventDisableTiming), "create event");
    }
    cuda(configure_gemm_kernels(), "configure GEMM kernels");
    cuda(configure_attention_kernel(), "configure attention kernel");

    // Weights: one blob, every tensor 256-byte aligned.
    std::map<std::string, size_t> offset;
    size_t total = 0;
    for (auto &kv : packed) {
      offset[kv.first] = total;
      total += align256(kv.second.bytes());
    }
    std::vector<uint8_t> host(total, 0);
    for (auto &kv : packed) std::memcpy(host.data() + offset[kv.first], kv.second.data(), kv.second.bytes());
    cuda(cudaMalloc(&weight_blob_, total), "allocate weights");
    cuda(cudaMemcpy(weight_blob_, host.data(), total, cudaMemcpyHostToDevice), "upload weights");
    auto hp = [&](const std::string &n) {
      return reinterpret_cast<const __half *>(static_cast<uint8_t *>(weight_blob_) + offset.at(n));
    };
    auto fp = [&](const std::string &n) {
      return reinterpret_cast<const float *>(static_cast<uint8_t *>(weight_blob_) + offset.at(n));
    };
    w_.patch_w = hp("patch_w");
    w_.patch_b = fp("patch_b");
    w_.prefix = fp("prefix");
    w_.norm_w = fp("norm_w");
    w_.norm_b = fp("norm_b");
    w_.rope_cos = fp("rope_cos");
    w_.rope_sin = fp("rope_sin");
    for (int i = 0; i < 12; ++i) {
      const std::string s = "l" + std::to_string(i) + "_";
      LayerWeights &l = w_.layer[i];
      l.qkv_w = hp(s + "qkv_w");
      l.gateup_w = hp(s + "gateup_w");
      l.o_w = hp(s + "o_w");
      l.down_w = hp(s + "down_w");
      l.qkv_b = fp(s + "qkv_b");
      l.gateup_b = fp(s + "gateup_b");
      l.o_b = fp(s + "o_b");
      l.down_b = fp(s + "down_b");
      l.norm1_w = fp(s + "norm1_w");
      l.norm1_b = fp(s + "norm1_b");
      l.norm2_w = fp(s + "norm2_w");
      l.norm2_b = fp(s + "norm2_b");
      l.ls1 = fp(s + "ls1");
      l.ls2 = fp(s + "ls2");
      l.qkv_wf = hp(s + "qkv_wf");
      l.gateup_wf = hp(s + "gateup_wf");
      l.qkv_aux = hp(s + "qkv_aux");
      l.gateup_aux = hp(s + "gateup_aux");
    }

    // Activations for max_batch images.
    const size_t B = max_batch_, R = kTokens * B, P = kPatches * B;
    // split-K partial slabs of the down projection: the largest splits x rows of any batch size
    size_t partial_floats = 0;
    for (size_t b = 1; b <= B; ++b) {
      const uint32_t r = static_cast<uint32_t>(kTokens * b);
      partial_floats = std::max(partial_floats, static_cast<size_t>(splitk_splits(r)) * r * kHidden);
    }
    const size_t sizes[15] = {B * kImageElements * 4, P * kPatchK * 2, R * kHidden * 2,
                              R * kHidden * 2,        R * kQkv * 2,    R * kHidden * 2,
                              R * kMlp * 2,           R * kHidden * 4, 256,
                              B * kHidden * 4,        B * kImageElements * 4, R * kHidden * 4,
                              partial_floats * 4,     R * 8,           R * 32};
    size_t at[15], act_total = 0;
    for (int i = 0; i < 15; ++i) {
      at[i] = act_total;
      act_total += align256(sizes[i]);
    }
    cuda(cudaMalloc(&act_blob_, act_total), "allocate activations");
    uint8_t *a = static_cast<uint8_t *>(act_blob_);
    image_ = reinterpret_cast<float *>(a + at[0]);
    partials_ = reinterpret_cast<float *>(a + at[12]);
    rowstat_ = reinterpret_cast<float2 *>(a + at[13]);
    row_aux_ = reinterpret_cast<__half *>(a + at[14]);
    patches_ = reinterpret_cast<__half *>(a + at[1]);
    x_ = reinterpret_cast<__half *>(a + at[2]);
    h_ = reinterpret_cast<__half *>(a + at[3]);
    qkv_ = reinterpret_cast<__half *>(a + at[4]);
    attn_ = reinterpret_cast<__half *>(a + at[5]);
    act_ = reinterpret_cast<__half *>(a + at[6]);
    out_ = reinterpret_cast<float *>(a + at[7]);
    status_ = reinterpret_cast<uint32_t *>(a + at[8]);
    pmean_ = reinterpret_cast<float *>(a + at[9]);
    image_slot_[0] = image_;
    out_slot_[0] = out_;
    image_slot_[1] = reinterpret_cast<float *>(a + at[10]);
    out_slot_[1] = reinterpret_cast<float *>(a + at[11]);
    cuda(cudaMallocHost(reinterpret_cast<void **>(&slot_status_host_), 4 * sizeof(uint32_t)),
         "allocate pinned status");
    for (int i = 0; i < 4; ++i) slot_status_host_[i] = 0;
    cuda(cudaMemset(status_, 0, 256), "clear status");
    cuda(cudaMallocHost(reinterpret_cast<void **>(&status_host_), 4 * sizeof(uint32_t)),
         "allocate pinned status");
    status_host_[0] = status_host_[1] = status_host_[2] = 0;
    inject_host_ = status_host_ + 2;
  } catch (...) {
    release();
    throw;
  }
}

Model::~Model() { release(); }

void Model::release() {
  cudaSetDevice(device_);
  for (auto &kv : plans_)
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
  plans_.clear();
  if (stream_) cudaStreamSynchronize(stream_);
  if (h2d_stream_) cudaStreamSynchronize(h2d_stream_);
  if (d2h_stream_) cudaStreamSynchronize(d2h_stream_);
  for (int i = 0; i < 2; ++i) {
    if (ev_in_[i]) cudaEventDestroy(ev_in_[i]);
    if (ev_done_[i]) cudaEventDestroy(ev_done_[i]);
    if (ev_out_[i]) cudaEventDestroy(ev_out_[i]);
    ev_in_[i] = ev_done_[i] = ev_out_[i] = nullptr;
  }
  if (h2d_stream_) cudaStreamDestroy(h2d_stream_);
  if (d2h_stream_) cudaStreamDestroy(d2h_stream_);
  h2d_stream_ = d2h_stream_ = nullptr;
  if (slot_status_host_) cudaFreeHost(slot_status_host_);
  slot_status_host_ = nullptr;
  if (status_host_) cudaFreeHost(status_host_);
  inject_host_ = nullptr;
  if (act_blob_) cudaFree(act_blob_);
  if (weight_blob_) cudaFree(weight_blob_);
  if (stream_) cudaStreamDestroy(stream_);
  status_host_ = nullptr;
  act_blob_ = weight_blob_ = nullptr;
  stream_ = nullptr;
  cudaGetLastError();
}

// The launch plan of one batch size (src/lib.rs:149-263): patchify, the patch GEMM (with the
// embed scatter), LN1 of layer 0,
// then per layer QKV+RoPE, attention, o-proj+LS1+residual+LN2, gate/up+SwiGLU, and
// down-proj+LS2+residual+(LN1 of the next layer | final LN). The reference launches each
// LayerNorm separately (87 launches at b > 1); here each one after layer 0's first rides in the
// epilogue of the GEMM that produces its input row (3 + 12*5 = 63 launches), whenever the
// residual GEMMs run on full rows (batch 32 and up; see resid_full_rows_plan); small batches keep 128-wide
// residual tiles and separate LayerNorm launches (3 + 12*7 = 87). With the full-row residual
// GEMMs, the LayerNorms before QKV and gate/up are further folded into those GEMMs
// (fold_layernorm): the residual GEMM (and, for layer 0, layernorm_rowstat) leaves only each
// row's statistics and QKV / gate/up read x.
// DV3_FUSE_LAYERNORM=0 in the environment restores the separate LayerNorm launches (the
// reference's plan) for comparison; =1 forces fusion.
// K slices of the down projection at this batch size (1: unsplit). DV3_SPLITK=0 in the
// environment turns the split off for comparison.
uint32_t Model::down_splits(uint32_t rows) const {
  if (const char *v = std::getenv("DV3_SPLITK"))
    if (v[0] == '0') return 1;
  return splitk_splits(rows);
}

// The full-row plan starts where the 128-wide residual tiles need a second wave when the
// LayerNorms are folded (batch 32 on 148 SMs, resid_full_rows_plan), and only where the row
// tiles outnumber half the SMs when they are not (batch 48, resid_wide): the normalise-and-store
// phase makes the unfolded full-row GEMMs slower than 128-wide tiles in one and a half waves.
bool Model::fuse_layernorm(size_t b) const {
  if (const char *v = std::getenv("DV3_FUSE_LAYERNORM")) return v[0] == '1';
  const uint32_t rows = static_cast<uint32_t>(kTokens * b);
  const char *f = std::getenv("DV3_FOLD_LAYERNORM");
  const bool unfolded = f != nullptr && ((f[0] - '0') & 3) == 0;
  return unfolded ? resid_wide(rows) : resid_full_rows_plan(rows);
}

// With the LayerNorms fused into the full-row residual GEMMs, each of them except the final one
// is folded one step further into the GEMM that consumes it: the residual GEMM leaves only
// (rstd, -mean rstd) per row instead of normalising the row, and the QKV and gate/up GEMMs read
// x with the folded weights (weights.cpp). Returns which LayerNorms are folded: bit 0 LN1
// (into QKV), bit 1 LN2 (into gate/up). DV3_FOLD_LAYERNORM in the environment picks them for
// comparison (0: none, keeping the normalised h; 1: LN1; 2: LN2; 3: both).
int Model::fold_layernorm(size_t b) const {
  if (!fuse_layernorm(b)) return 0;
  if (const char *v = std::getenv("DV3_FOLD_LAYERNORM")) return (v[0] - '0') & 3;
  return 3;
}

// Bytes of each projection's f16 weights. Each launch of the plan starts the weights of a GEMM
// one or two launches later toward L2 (GemmArgs::l2_next), so that kernel's first tiles do not
// wait for DRAM: the weights are read once per forward, after activations have cycled the L2.
constexpr size_t kQkvWBytes = size_t{kQkv} * kHidden * 2;
constexpr size_t kOWBytes = size_t{kHidden} * kHidden * 2;
constexpr size_t kGateUpWBytes = size_t{kGateUp} * kHidden * 2;
constexpr size_t kDownWBytes = size_t{kHidden} * kMlp * 2;

Plan &Model::prepare(size_t b, int slot) {
  auto it = plans_.find({b, slot});
  if (it != plans_.end()) return it->second;
  const uint32_t r = static_cast<uint32_t>(kTokens * b), p = static_cast<uint32_t>(kPatches * b);
  std::string err;
  auto need = [&](bool ok) {
    if (!ok) {
      failed_ = true;
      throw Error(DV3_DEVICE, "tensor map: " + err);
    }
  };
  Plan plan;
  auto add = [&](const char *name, std::function<cudaError_t(cudaStream_t)> f) {
    plan.launches.push_back({name, true, std::move(f)});
    ++plan.kernels;
  };
  uint32_t *st = status_;
  const DeviceWeights w = w_;
  float *image = image_slot_[slot], *out = out_slot_[slot];
  __half *x = x_, *h = h_, *qkv = qkv_, *attn = attn_, *act = act_, *patches = patches_;
  float2 *rowstat = rowstat_;
  __half *row_aux = row_aux_;
  const int fold_mask = fold_layernorm(b);
  const bool fold = fold_mask & 1, fold2 = (fold_mask & 2) != 0;  // LN1 into QKV, LN2 into gate/up

  GemmMaps patch_maps;
  need(make_gemm_maps(GemmOp::Patch, patches, p, w.patch_w, x, &patch_maps, &err));
  AttentionMaps attn_map;
  need(make_attention_map(qkv, attn, r, &attn_map, &err));

  add("patchify", [=](cudaStream_t s) {
    return launch_patchify(image, static_cast<uint32_t>(b), w.prefix, patches, x, st, s,
                           w.patch_w, size_t{kHidden} * kPatchK * 2);
  });
  add(gemm_name(GemmOp::Patch), [=](cudaStream_t s) {
    GemmArgs g;
    g.l2_next = fold ? w.layer[0].qkv_wf : w.layer[0].qkv_w;
    g.l2_next_bytes = kQkvWBytes;
    g.bias = w.patch_b;
    g.out = x;
    return launch_gemm(GemmOp::Patch, patch_maps, p, g, st, s);
  });
  if (fold)
    add("layernorm_rowstat", [=](cudaStream_t s) {
      return launch_layernorm_rowstat(x, r, rowstat, row_aux, s);
    });
  else
    add("layernorm_f16", [=](cudaStream_t s) {
      return launch_layernorm_f16(x, r, w.layer[0].norm1_w, w.layer[0].norm1_b, h, s);
    });
  const bool fuse = fuse_layernorm(b);
  const GemmOp o_op = fuse ? GemmOp::ResidLN384 : GemmOp::Resid384;
  const GemmOp down_op = fuse ? GemmOp::ResidLN1536 : GemmOp::Resid1536;
  // Small batches: the down projection splits K (its 6 to 39 128x128 tiles alone would leave most
  // SMs idle for 24 k-blocks) and the reduce kernel also does the LayerNorm after it (the
  // reference splits K at batch 1, src/lib.rs:218-226).
  const uint32_t splits = fuse ? 1u : down_splits(r);
  float *partials = partials_;
  // Each intermediate is dropped from L2 (GemmArgs::discard) by the launch after the one that
  // last reads it, once that reader is complete: its lines neither cost a DRAM write-back when
  // they are evicted nor hold L2 space until the next layer rewrites them. The dropping launch
  // never touches the buffer itself.
  const size_t patches_bytes = size_t{p} * kPatchK * 2, h_bytes = size_t{r} * kHidden * 2,
               qkv_bytes = size_t{r} * kQkv * 2, attn_bytes = h_bytes,
               act_bytes = size_t{r} * kMlp * 2;
  for (int i = 0; i < 12; ++i) {
    const LayerWeights &l = w.layer[i];
    GemmMaps qkv_maps, o_maps, gu_maps, down_maps;
    // folded: QKV and gate/up read x, the residual GEMMs leave row statistics
    const GemmOp qkv_op = fold ? GemmOp::QkvRopeFold : GemmOp::QkvRope;
    const GemmOp gu_op = fold2 ? GemmOp::SwiGLUFold : GemmOp::SwiGLU;
    const GemmOp o_op_l = fold2 ? GemmOp::ResidStats384 : o_op;
    const GemmOp down_op_l = fold && i < 11 ? GemmOp::ResidStats1536 : down_op;
    need(make_gemm_maps(qkv_op, fold ? x : h, r, fold ? l.qkv_wf : l.qkv_w, qkv, &qkv_maps, &err));
    if (fold) need(make_fold_maps(qkv_op, row_aux, r, l.qkv_aux, &qkv_maps, &err));
    need(make_gemm_maps(o_op_l, attn, r, l.o_w, x, &o_maps, &err, h));
    need(make_gemm_maps(gu_op, fold2 ? x : h, r, fold2 ? l.gateup_wf : l.gateup_w, act, &gu_maps,
                        &err));
    if (fold2) need(make_fold_maps(gu_op, row_aux, r, l.gateup_aux, &gu_maps, &err));
    if (splits > 1)
      need(make_gemm_maps(GemmOp::SplitK1536, act, r, l.down_w, partials, &down_maps, &err,
                          nullptr, false, splits));
    else
      need(make_gemm_maps(down_op_l, act, r, l.down_w, x, &down_maps, &err,
                          i == 11 ? static_cast<const void *>(out) : static_cast<const void *>(h),
                          i == 11));
    add(gemm_name(qkv_op), [=](cudaStream_t s) {
      GemmArgs g;
      g.bias = l.qkv_b;
      g.rowstat = rowstat;
      g.rope_cos = w.rope_cos;
      g.rope_sin = w.rope_sin;
      g.out = qkv;
      g.l2_next = l.o_w;
      g.l2_next_bytes = kOWBytes;
      // the patch GEMM's input (layer 0), or the previous layer's down-projection input
      g.discard = i == 0 ? static_cast<const void *>(patches) : static_cast<const void *>(act);
      g.discard_bytes = i == 0 ? patches_bytes : act_bytes;
      return launch_gemm(qkv_op, qkv_maps, r, g, st, s);
    });
    add("attention", [=](cudaStream_t s) {  // h: the QKV GEMM's input (x, still live, if folded)
      return launch_attention(attn_map, r, st, s, fold2 ? l.gateup_wf : l.gateup_w, kGateUpWBytes,
                              fold ? nullptr : h, fold ? 0 : h_bytes);
    });
    // o-proj + LayerScale 1 + residual, and LN2 of this layer (fused or separate): x -> x, h
    add(gemm_name(o_op_l), [=](cudaStream_t s) {
      GemmArgs g;
      g.bias = l.o_b;
      g.lambda = l.ls1;
      g.out = x;
      g.gamma = l.norm2_w;
      g.beta = l.norm2_b;
      g.ln_out = h;
      g.rowstat = rowstat;
      g.row_aux = row_aux;
      g.l2_next = l.down_w;
      g.l2_next_bytes = kDownWBytes;
      g.discard = qkv;  // the attention's input
      g.discard_bytes = qkv_bytes;
      return launch_gemm(o_op_l, o_maps, r, g, st, s);
    });
    if (!fuse)
      add("layernorm_f16", [=](cudaStream_t s) {
        return launch_layernorm_f16(x, r, l.norm2_w, l.norm2_b, h, s);
      });
    add(gemm_name(gu_op), [=](cudaStream_t s) {
      GemmArgs g;
      g.bias = l.gateup_b;
      g.rowstat = rowstat;
      g.out = act;
      g.discard = attn;  // the o-projection's input
      g.discard_bytes = attn_bytes;
      if (i < 11) {
        g.l2_next = fold ? w.layer[i + 1].qkv_wf : w.layer[i + 1].qkv_w;
        g.l2_next_bytes = kQkvWBytes;
      }
      return launch_gemm(gu_op, gu_maps, r, g, st, s);
    });
    // down-proj + LayerScale 2 + residual, fused with LN1 of the next layer (f16 h) or, after
    // the last layer, with the final LayerNorm (f32 output)
    const bool last = i == 11;
    const float *ng = last ? w.norm_w : w.layer[i + 1].norm1_w;
    const float *nb = last ? w.norm_b : w.layer[i + 1].norm1_b;
    if (splits > 1) {
      add(gemm_name(GemmOp::SplitK1536), [=](cudaStream_t s) {
        GemmArgs g;
        g.partials = partials;
        g.splits = splits;
        return launch_gemm(GemmOp::SplitK1536, down_maps, r, g, st, s);
      });
      add("splitk_reduce_layernorm", [=](cudaStream_t s) {
        return launch_splitk_reduce(partials, r, splits, l.down_b, l.ls2, x, ng, nb,
                                    last ? nullptr : h, last ? out : nullptr, s);
      });
      continue;
    }
    add(gemm_name(down_op_l), [=](cudaStream_t s) {
      GemmArgs g;
      g.bias = l.down_b;
      g.lambda = l.ls2;
      g.out = x;
      g.gamma = ng;
      g.beta = nb;
      g.ln_out = last ? nullptr : h;
      g.ln_out_f32 = last ? out : nullptr;
      g.rowstat = rowstat;
      g.row_aux = row_aux;
      return launch_gemm(down_op_l, down_maps, r, g, st, s);
    });
    if (!fuse) {
      if (last)
        add("layernorm_f32out", [=](cudaStream_t s) {
          return launch_layernorm_f32(x, r, ng, nb, out, s);
        });
      else
        add("layernorm_f16", [=](cudaStream_t s) {
          return launch_layernorm_f16(x, r, ng, nb, h, s);
        });
    }
  }

  // Record the plan as one CUDA graph (the HRX execution graph of src/engine.rs:87-129).
  cudaGraph_t graph = nullptr;
  cuda(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "begin capture");
  for (auto &l : plan.launches) {
    cudaError_t e = l.enqueue(stream_);
    if (e != cudaSuccess) {
      cudaStreamEndCapture(stream_, &graph);
      if (graph) cudaGraphDestroy(graph);
      cuda(e, l.name);
    }
  }
  cuda(cudaStreamEndCapture(stream_, &graph), "end capture");
  cudaError_t e = cudaGraphInstantiate(&plan.exec, graph, 0);
  cudaGraphDestroy(graph);
  cuda(e, "instantiate graph");
  return plans_.emplace(std::make_pair(b, slot), std::move(plan)).first->second;
}

void Model::check_status() {
  cuda(cudaMemcpyAsync(status_host_, status_, 2 * sizeof(uint32_t), cudaMemcpyDeviceToHost, stream_),
       "read status");
  cuda(cudaStreamSynchronize(stream_), "synchronize");
  status_pending_ = false;
  const uint32_t fault = status_host_[0], nonfinite = status_host_[1];
  if (fault || nonfinite) {
    cuda(cudaMemsetAsync(status_, 0, 2 * sizeof(uint32_t), stream_), "clear status");
    status_host_[0] = status_host_[1] = 0;
  }
  if (fault) {
    failed_ = true;
    char buf[96];
    std::snprintf(buf, sizeof buf, "a kernel wait expired (device status 0x%x)", fault);
    throw Error(DV3_POISONED, std::string(buf) + "; session is unusable after a GPU failure");
  }
  if (nonfinite) throw Error(DV3_INVALID_ARGUMENT, "input must be finite");
}

void Model::forward(const float *pixels, size_t n_floats, float *out, size_t out_floats,
                    Readout readout) {
  drain();
  if (n_floats % kImageElements != 0)
    throw Error(DV3_INVALID_ARGUMENT, "input must contain complete 3×224×224 images");
  const size_t batch = n_floats / kImageElements;
  const size_t tokens = static_cast<size_t>(kTokens) * kHidden;  // floats per image on the device
  const size_t per = readout == Readout::Full ? tokens : kHidden;  // floats per image returned
  if (out_floats < batch * per)
    throw Error(DV3_INVALID_ARGUMENT, "output must hold " + std::to_string(batch * per) + " floats");
  if (batch && (!pixels || !out)) throw Error(DV3_INVALID_ARGUMENT, "null buffer");
  activate();
  for (size_t i = 0; i < batch; i += max_batch_) {
    check_usable();
    const size_t b = std::min(max_batch_, batch - i);
    Plan &plan = prepare(b);
    cuda(cudaMemcpyAsync(image_, pixels + i * kImageElements, b * kImageElements * sizeof(float),
                         cudaMemcpyHostToDevice, stream_),
         "upload input");
    cuda(cudaGraphLaunch(plan.exec, stream_), "launch graph");
    apply_injection();
    if (readout == Readout::Full) {
      cuda(cudaMemcpyAsync(out + i * per, out_, b * per * sizeof(float), cudaMemcpyDeviceToHost,
                           stream_),
           "read output");
    } else if (readout == Readout::Cls) {  // row 0 of each image: one strided copy
      cuda(cudaMemcpy2DAsync(out + i * per, kHidden * sizeof(float), out_, tokens * sizeof(float),
                             kHidden * sizeof(float), b, cudaMemcpyDeviceToHost, stream_),
           "read CLS rows");
    } else {
      cuda(launch_patch_mean(out_, static_cast<uint32_t>(b), pmean_, stream_), "patch mean");
      cuda(cudaMemcpyAsync(out + i * per, pmean_, b * per * sizeof(float), cudaMemcpyDeviceToHost,
                           stream_),
           "read patch means");
    }
    status_pending_ = true;
    check_status();
  }
}

void Model::forward_device(const float *pixels, size_t n_floats, float *out, size_t out_floats) {
  drain();
  if (n_floats % kImageElements != 0)
    throw Error(DV3_INVALID_ARGUMENT, "input must contain complete 3×224×224 images");
  const size_t batch = n_floats / kImageElements;
  const size_t per = static_cast<size_t>(kTokens) * kHidden;
  if (out_floats < batch * per)
    throw Error(DV3_INVALID_ARGUMENT, "output must hold " + std::to_string(batch * per) + " floats");
  if (batch && (!pixels || !out)) throw Error(DV3_INVALID_ARGUMENT, "null buffer");
  activate();
  for (size_t i = 0; i < batch; i += max_batch_) {
    check_usable();
    const size_t b = std::min(max_batch_, batch - i);
    Plan &plan = prepare(b);
    cuda(cudaMemcpyAsync(image_, pixels + i * kImageElements, b * kImageElements * sizeof(float),
                         cudaMemcpyDeviceToDevice, stream_),
         "copy input");
    cuda(cudaGraphLaunch(plan.exec, stream_), "launch graph");
    apply_injection();
    cuda(cudaMemcpyAsync(out + i * per, out_, b * per * sizeof(float), cudaMemcpyDeviceToDevice, stream_),
         "copy output");
    status_pending_ = true;
  }
  if (batch) check_status();
}

// ---- serving path ----
// Per submission: upload on h2d_stream_ (after the slot's previous forward consumed its input),
// forward on stream_ (after the upload and after the slot's previous download read its output),
// with the status words cleared before and copied to the slot's pinned words after, and the
// download on d2h_stream_. Two slots, so consecutive submissions overlap; a third submission
// first completes the one occupying its slot (its status is kept for its own wait).
uint64_t Model::submit(const float *pixels, size_t n_floats, float *out, size_t out_floats) {
  check_usable();
  if (n_floats == 0 || n_floats % kImageElements != 0)
    throw Error(DV3_INVALID_ARGUMENT, "input must contain complete 3×224×224 images");
  const size_t b = n_floats / kImageElements;
  if (b > max_batch_) throw Error(DV3_INVALID_ARGUMENT, "a submission holds at most max_batch images");
  const size_t per = static_cast<size_t>(kTokens) * kHidden;
  if (out_floats < b * per)
    throw Error(DV3_INVALID_ARGUMENT, "output must hold " + std::to_string(b * per) + " floats");
  if (!pixels || !out) throw Error(DV3_INVALID_ARGUMENT, "null buffer");
  activate();
  const uint64_t ticket = next_ticket_;
  const int slot = static_cast<int>(ticket & 1);
  if (submitted_[slot]) retire(slot);
  Plan &plan = prepare(b, slot);
  ++next_ticket_;
  cuda(cudaStreamWaitEvent(h2d_stream_, ev_done_[slot], 0), "order upload");
  cuda(cudaMemcpyAsync(image_slot_[slot], pixels, b * kImageElements * sizeof(float),
                       cudaMemcpyHostToDevice, h2d_stream_),
       "upload input");
  cuda(cudaEventRecord(ev_in_[slot], h2d_stream_), "record upload");
  cuda(cudaStreamWaitEvent(stream_, ev_in_[slot], 0), "order forward");
  cuda(cudaStreamWaitEvent(stream_, ev_out_[slot], 0), "order forward");
  cuda(cudaMemsetAsync(status_, 0, 2 * sizeof(uint32_t), stream_), "clear status");
  cuda(cudaGraphLaunch(plan.exec, stream_), "launch graph");
  apply_injection();
  cuda(cudaMemcpyAsync(slot_status_host_ + 2 * slot, status_, 2 * sizeof(uint32_t),
                       cudaMemcpyDeviceToHost, stream_),
       "read status");
  cuda(cudaEventRecord(ev_done_[slot], stream_), "record forward");
  cuda(cudaStreamWaitEvent(d2h_stream_, ev_done_[slot], 0), "order download");
  cuda(cudaMemcpyAsync(out, out_slot_[slot], b * per * sizeof(float), cudaMemcpyDeviceToHost,
                       d2h_stream_),
       "read output");
  cuda(cudaEventRecord(ev_out_[slot], d2h_stream_), "record download");
  submitted_[slot] = true;
  slot_ticket_[slot] = ticket;
  return ticket;
}

void Model::retire(int slot) {
  cuda(cudaEventSynchronize(ev_out_[slot]), "finish submission");
  const uint32_t fault = slot_status_host_[2 * slot], nonfinite = slot_status_host_[2 * slot + 1];
  finished_[slot_ticket_[slot]] = {fault, nonfinite};
  submitted_[slot] = false;
  if (fault) failed_ = true;  // the session is poisoned whether or not that ticket is waited
}

void Model::wait(uint64_t ticket) {
  if (ticket >= next_ticket_) throw Error(DV3_INVALID_ARGUMENT, "unknown ticket");
  const int slot = static_cast<int>(ticket & 1);
  auto it = finished_.find(ticket);
  if (it == finished_.end()) {
    if (!submitted_[slot] || slot_ticket_[slot] != ticket)
      throw Error(DV3_INVALID_ARGUMENT, "ticket already waited");
    activate();
    retire(slot);
    it = finished_.find(ticket);
  }
  const auto [fault, nonfinite] = it->second;
  finished_.erase(it);
  if (fault) {
    char buf[96];
    std::snprintf(buf, sizeof buf, "a kernel wait expired (device status 0x%x)", fault);
    throw Error(DV3_POISONED, std::string(buf) + "; session is unusable after a GPU failure");
  }
  if (nonfinite) throw Error(DV3_INVALID_ARGUMENT, "input must be finite");
}

void Model::drain() {
  for (int slot = 0; slot < 2; ++slot)
    if (submitted_[slot]) retire(slot);
}

void Model::run(size_t batch) {
  drain();
  check_usable();
  if (batch < 1 || batch > max_batch_)
    throw Error(DV3_INVALID_ARGUMENT, "batch must be 1..=max_batch");
  activate();
  Plan &plan = prepare(batch);
  cuda(cudaGraphLaunch(plan.exec, stream_), "launch graph");
  apply_injection();
  status_pending_ = true;
}

void Model::inject_fault(uint32_t bits) {
  check_usable();
  if (bits == 0) throw Error(DV3_INVALID_ARGUMENT, "inject at least one failure bit");
  *inject_host_ = bits;
  inject_pending_ = true;
}

// The injected bits land in the failure word on the compute stream after the forward's kernels
// and before its status is read, exactly where a kernel's expired wait would have put them.
void Model::apply_injection() {
  if (!inject_pending_) return;
  inject_pending_ = false;
  cuda(cudaMemcpyAsync(status_, inject_host_, sizeof(uint32_t), cudaMemcpyHostToDevice, stream_),
       "inject failure bits");
}

void Model::synchronize() {
  check_usable();
  activate();
  check_status();
}

size_t Model::launches_per_forward(size_t batch) {
  check_usable();
  if (batch < 1 || batch > max_batch_)
    throw Error(DV3_INVALID_ARGUMENT, "batch must be 1..=max_batch");
  activate();
  return prepare(batch).kernels;
}

dv3_timings Model::benchmark(const float *pixels, size_t n_floats, size_t samples) {
  drain();
  if (n_floats == 0 || n_floats > max_batch_ * kImageElements)
    throw Error(DV3_INVALID_ARGUMENT, "benchmark requires one nonempty batch");
  std::vector<float> first(n_floats / kImageElements * kTokens * kHidden);
  forward(pixels, n_floats, first.data(), first.size());
  if (samples < 10) throw Error(DV3_INVALID_ARGUMENT, "use at least ten timing samples");
  check_usable();
  const size_t b = n_floats / kImageElements;
  Plan &plan = prepare(b);
  std::vector<double> times[2];
  for (size_t i = 0; i < samples + 10; ++i) {
    const int order[2] = {static_cast<int>(i % 2), static_cast<int>(1 - i % 2)};
    for (int mode : order) {
      const auto t0 = std::chrono::steady_clock::now();
      if (mode == 0) {
        cuda(cudaGraphLaunch(plan.exec, stream_), "launch graph");
      } else {
        for (auto &l : plan.launches) cuda(l.enqueue(stream_), l.name);
      }
      cuda(cudaStreamSynchronize(stream_), "synchronize");
      const auto t1 = std::chrono::steady_clock::now();
      if (i >= 10) times[mode].push_back(std::chrono::duration<double, std::milli>(t1 - t0).count());
    }
  }
  check_status();
  auto summarize = [](std::vector<double> t) {
    std::sort(t.begin(), t.end());
    dv3_distribution d;
    d.median_ms = t[t.size() / 2];
    d.p95_ms = t[(t.size() * 95 + 99) / 100 - 1];
    return d;
  };
  dv3_timings out;
  out.samples = samples;
  out.graph = summarize(times[0]);
  out.direct = summarize(times[1]);
  return out;
}

// Per-launch device time without host enqueue gaps: for each launch of the plan, a graph of
// `iterations` back-to-back copies of that launch is captured and replayed between two events
// on the model's stream (after one warm-up replay); the launch's time is the interval divided by
// the copies. Consecutive copies overlap their start-up as the production graph does. The
// residual GEMMs update x in place, so x holds garbage afterwards; the next forward rebuilds it.
std::vector<std::pair<const char *, double>> Model::profile_launches(size_t batch,
                                                                     size_t iterations) {
  drain();
  check_usable();
  if (batch < 1 || batch > max_batch_)
    throw Error(DV3_INVALID_ARGUMENT, "batch must be 1..=max_batch");
  if (iterations < 1) throw Error(DV3_INVALID_ARGUMENT, "iterations must be >= 1");
  activate();
  Plan &plan = prepare(batch);
  const size_t n = plan.launches.size();
  cudaEvent_t ev[2] = {nullptr, nullptr};
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  auto release_graph = [&] {
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    exec = nullptr;
    graph = nullptr;
  };
  std::vector<std::pair<const char *, double>> result;
  try {
    for (auto &e : ev) cuda(cudaEventCreate(&e), "create event");
    for (size_t j = 0; j < n; ++j) {
      cuda(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "begin capture");
      cudaError_t e = cudaSuccess;
      for (size_t it = 0; it < iterations && e == cudaSuccess; ++it) e = plan.launches[j].enqueue(stream_);
      cudaError_t e2 = cudaStreamEndCapture(stream_, &graph);
      cuda(e != cudaSuccess ? e : e2, "capture profiling graph");
      cuda(cudaGraphInstantiate(&exec, graph, 0), "instantiate profiling graph");
      cuda(cudaGraphLaunch(exec, stream_), "launch profiling graph");  // warm-up
      cuda(cudaEventRecord(ev[0], stream_), "record event");
      cuda(cudaGraphLaunch(exec, stream_), "launch profiling graph");
      cuda(cudaEventRecord(ev[1], stream_), "record event");
      cuda(cudaEventSynchronize(ev[1]), "synchronize");
      float ms = 0;
      cuda(cudaEventElapsedTime(&ms, ev[0], ev[1]), "elapsed time");
      result.emplace_back(plan.launches[j].name, ms / static_cast<double>(iterations));
      release_graph();
    }
  } catch (...) {
    release_graph();
    for (auto &e : ev)
      if (e) cudaEventDestroy(e);
    throw;
  }
  for (auto &e : ev) cudaEventDestroy(e);
  check_status();
  return result;
}

// Per-launch device time inside whole forwards, in the production plan's order, cache state and
// overlap: for every j the first j launches of the plan are captured into a CUDA graph (kernel
// nodes joined by programmatic dependencies, as in the production graph), and each prefix graph
// is replayed `replays` times between two CUDA events on the model's stream, each replay after
// a write of `flush_bytes` bytes to a scratch buffer outside the events (evicting L2 when larger
// than it, as between timed steps). T(j) is the mean replay time of the first j launches, and
// launch j's time is T(j) - T(j-1): what that launch adds to the forward, including the part of
// its set-up that overlaps the previous kernel's tail. The times add up to a whole forward. The
// scratch buffer and the graphs are made for the call and released after it.
std::vector<std::pair<const char *, double>> Model::profile_forward(size_t batch, size_t replays,
                                                                    size_t flush_bytes) {
  drain();
  check_usable();
  if (batch < 1 || batch > max_batch_)
    throw Error(DV3_INVALID_ARGUMENT, "batch must be 1..=max_batch");
  if (replays < 1) throw Error(DV3_INVALID_ARGUMENT, "replays must be >= 1");
  activate();
  Plan &plan = prepare(batch);
  const size_t n = plan.launches.size();
  cudaEvent_t ev[2] = {nullptr, nullptr};
  void *flush = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  auto release_graph = [&] {
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    exec = nullptr;
    graph = nullptr;
  };
  auto release_all = [&] {
    release_graph();
    for (auto &e : ev)
      if (e) cudaEventDestroy(e);
    if (flush) cudaFree(flush);
    flush = nullptr;
  };
  std::vector<double> prefix(n + 1, 0.0);  // T(j), ms
  try {
    for (auto &e : ev) cuda(cudaEventCreate(&e), "create event");
    if (flush_bytes) cuda(cudaMalloc(&flush, flush_bytes), "allocate flush buffer");
    for (size_t j = 1; j <= n; ++j) {
      cuda(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "begin capture");
      cudaError_t e = cudaSuccess;
      for (size_t k = 0; k < j && e == cudaSuccess; ++k) e = plan.launches[k].enqueue(stream_);
      const cudaError_t e2 = cudaStreamEndCapture(stream_, &graph);
      cuda(e != cudaSuccess ? e : e2, "capture profiling graph");
      cuda(cudaGraphInstantiate(&exec, graph, 0), "instantiate profiling graph");
      cuda(cudaGraphLaunch(exec, stream_), "launch profiling graph");  // warm-up
      double sum = 0.0;
      for (size_t r = 0; r < replays; ++r) {
        if (flush) cuda(cudaMemsetAsync(flush, static_cast<int>(r & 0xff), flush_bytes, stream_),
                        "flush L2");
        cuda(cudaEventRecord(ev[0], stream_), "record event");
        cuda(cudaGraphLaunch(exec, stream_), "launch profiling graph");
        cuda(cudaEventRecord(ev[1], stream_), "record event");
        cuda(cudaEventSynchronize(ev[1]), "synchronize");
        float ms = 0;
        cuda(cudaEventElapsedTime(&ms, ev[0], ev[1]), "elapsed time");
        sum += ms;
      }
      prefix[j] = sum / static_cast<double>(replays);
      release_graph();
    }
  } catch (...) {
    release_all();
    throw;
  }
  release_all();
  check_status();
  std::vector<std::pair<const char *, double>> result;
  for (size_t j = 0; j < n; ++j) result.emplace_back(plan.launches[j].name, prefix[j + 1] - prefix[j]);
  return result;
}

}  // namespace dv3
