// weights.cpp - safetensors reading and packing, following src/weights.rs:19-146.
//
// safetensors 0.6.2 format (Cargo.lock:2092-2094): an 8-byte little-endian header length, a
// JSON object {name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}},
// then the raw little-endian tensor bytes (offsets relative to the end of the header).
#include "weights.h"

#include <charconv>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>

#include "kernels.h"

namespace dv3 {

// ---------------------------------------------------------------------------------------------
// f16 / bf16
// ---------------------------------------------------------------------------------------------
uint16_t f32_to_f16(float v) {
  uint32_t x;
  std::memcpy(&x, &v, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return static_cast<uint16_t>(sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u));
  if (ax >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);  // >= 65520 rounds to inf
  if (ax < 0x38800000u) {  // below 2^-14: an f16 subnormal, step 2^-24
    float a;
    std::memcpy(&a, &ax, 4);
    const uint32_t m = static_cast<uint32_t>(std::nearbyint(a * 16777216.0f));  // ties to even
    return static_cast<uint16_t>(sign | m);
  }
  const uint32_t e = ((ax >> 23) - 127u + 15u);
  const uint32_t mant = ax & 0x7FFFFFu;
  uint32_t h = (e << 10) | (mant >> 13);
  const uint32_t rem = mant & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;  // carry may roll into the exponent
  return static_cast<uint16_t>(sign | h);
}

float f16_to_f32(uint16_t h) {
  const uint32_t sign = (static_cast<uint32_t>(h) & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  const uint32_t m = h & 0x3FFu;
  uint32_t x;
  if (e == 0x1F) {
    x = sign | 0x7F800000u | (m << 13);
  } else if (e == 0) {
    const float f = static_cast<float>(m) * (1.0f / 16777216.0f);  // m * 2^-24, exact
    std::memcpy(&x, &f, 4);
    x |= sign;
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

float bf16_to_f32(uint16_t h) {
  const uint32_t x = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

std::string format_f32(float v) {
  char buf[64];
  auto r = std::to_chars(buf, buf + sizeof buf, v, std::chars_format::fixed);
  if (r.ec != std::errc()) return "?";
  return std::string(buf, r.ptr);
}

size_t pack_f16(const std::string &name, const float *values, size_t n, uint16_t *out,
                std::string *message) {
  for (size_t i = 0; i < n; ++i) {
    const uint16_t h = f32_to_f16(values[i]);
    if ((h & 0x7C00u) == 0x7C00u) {
      if (message)
        *message = "tensor " + name + "[" + std::to_string(i) +
                   "] cannot be represented as finite float16: " + format_f32(values[i]);
      return i;
    }
    out[i] = h;
  }
  return SIZE_MAX;
}

// ---------------------------------------------------------------------------------------------
// A minimal JSON reader for the safetensors header
// ---------------------------------------------------------------------------------------------
namespace {

struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json *get(const std::string &k) const {
    for (auto &kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct Parser {
  const char *p, *end;
  [[noreturn]] void fail() { throw WeightsError("malformed safetensors header"); }
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  char peek() {
    ws();
    if (p >= end) fail();
    return *p;
  }
  void expect(char c) {
    if (peek() != c) fail();
    ++p;
  }
  std::string string() {
    expect('"');
    std::string s;
    while (true) {
      if (p >= end) fail();
      char c = *p++;
      if (c == '"') break;
      if (c == '\\') {
        if (p >= end) fail();
        char e = *p++;
        switch (e) {
          case '"': s += '"'; break;
          case '\\': s += '\\'; break;
          case '/': s += '/'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'n': s += '\n'; break;
          case 'r': s += '\r'; break;
          case 't': s += '\t'; break;
          case 'u': {
            if (end - p < 4) fail();
            unsigned code = 0;
            for (int i = 0; i < 4; ++i) {
              char h = *p++;
              code <<= 4;
              if (h >= '0' && h <= '9') code |= h - '0';
              else if (h >= 'a' && h <= 'f') code |= h - 'a' + 10;
              else if (h >= 'A' && h <= 'F') code |= h - 'A' + 10;
              else fail();
            }
            if (code < 0x80) {
              s += static_cast<char>(code);
            } else if (code < 0x800) {
              s += static_cast<char>(0xC0 | (code >> 6));
              s += static_cast<char>(0x80 | (code & 0x3F));
            } else {
              s += static_cast<char>(0xE0 | (code >> 12));
              s += static_cast<char>(0x80 | ((code >> 6) & 0x3F));
              s += static_cast<char>(0x80 | (code & 0x3F));
            }
            break;
          }
          default: fail();
        }
      } else {
        s += c;
      }
    }
    return s;
  }
  Json value(int depth = 0) {
    if (depth > 16) fail();
    Json j;
    char c = peek();
    if (c == '{') {
      ++p;
      j.kind = Json::Object;
      if (peek() == '}') {
        ++p;
        return j;
      }
      while (true) {
        std::string k = string();
        expect(':');
        j.obj.emplace_back(std::move(k), value(depth + 1));
        char d = peek();
        ++p;
        if (d == '}') break;
        if (d != ',') fail();
      }
    } else if (c == '[') {
      ++p;
      j.kind = Json::Array;
      if (peek() == ']') {
        ++p;
        return j;
      }
      while (true) {
        j.arr.push_back(value(depth + 1));
        char d = peek();
        ++p;
        if (d == ']') break;
        if (d != ',') fail();
      }
    } else if (c == '"') {
      j.kind = Json::String;
      j.str = string();
    } else if (c == 't' || c == 'f' || c == 'n') {
      const char *w = c == 't' ? "true" : c == 'f' ? "false" : "null";
      size_t n = std::strlen(w);
      if (static_cast<size_t>(end - p) < n || std::strncmp(p, w, n) != 0) fail();
      p += n;
      j.kind = c == 'n' ? Json::Null : Json::Bool;
    } else {
      const char *s = p;
      while (p < end && (std::strchr("+-.eE", *p) || (*p >= '0' && *p <= '9'))) ++p;
      if (p == s) fail();
      j.kind = Json::Number;
      j.num = std::strtod(std::string(s, p).c_str(), nullptr);
    }
    return j;
  }
};

struct TensorView {
  std::string dtype;
  std::vector<size_t> shape;
  const uint8_t *data = nullptr;
  size_t bytes = 0;
};

class SafeTensors {
 public:
  explicit SafeTensors(const std::string &path) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) throw WeightsError("read " + path + ": No such file or directory");
    const std::streamsize size = f.tellg();
    f.seekg(0);
    buf_.resize(static_cast<size_t>(size));
    if (size > 0 && !f.read(reinterpret_cast<char *>(buf_.data()), size))
      throw WeightsError("read " + path + ": I/O error");
    if (buf_.size() < 8) throw WeightsError("HeaderTooSmall");
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | buf_[i];
    if (n > buf_.size() - 8) throw WeightsError("InvalidHeaderLength");
    Parser ps{reinterpret_cast<const char *>(buf_.data() + 8),
              reinterpret_cast<const char *>(buf_.data() + 8 + n)};
    Json root = ps.value();
    if (root.kind != Json::Object) throw WeightsError("malformed safetensors header");
    const uint8_t *base = buf_.data() + 8 + n;
    const size_t avail = buf_.size() - 8 - n;
    for (auto &kv : root.obj) {
      if (kv.first == "__metadata__") continue;
      const Json &t = kv.second;
      const Json *dt = t.get("dtype"), *sh = t.get("shape"), *off = t.get("data_offsets");
      if (!dt || !sh || !off || dt->kind != Json::String || sh->kind != Json::Array ||
          off->kind != Json::Array || off->arr.size() != 2)
        throw WeightsError("malformed safetensors header");
      TensorView v;
      v.dtype = dt->str;
      size_t count = 1;
      for (auto &d : sh->arr) {
        if (d.kind != Json::Number || d.num < 0) throw WeightsError("malformed safetensors header");
        v.shape.push_back(static_cast<size_t>(d.num));
        count *= static_cast<size_t>(d.num);
      }
      const size_t b0 = static_cast<size_t>(off->arr[0].num), b1 = static_cast<size_t>(off->arr[1].num);
      if (b1 < b0 || b1 > avail) throw WeightsError("InvalidOffset: " + kv.first);
      size_t esize = v.dtype == "F32" ? 4 : (v.dtype == "F16" || v.dtype == "BF16") ? 2 : 0;
      if (esize && count * esize != b1 - b0) throw WeightsError("TensorInvalidInfo: " + kv.first);
      v.data = base + b0;
      v.bytes = b1 - b0;
      tensors_.emplace(kv.first, std::move(v));
    }
  }
  const TensorView *find(const std::string &name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
  }

 private:
  std::vector<uint8_t> buf_;
  std::map<std::string, TensorView> tensors_;
};

std::string shape_str(const std::vector<size_t> &s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

}  // namespace

std::map<std::string, Packed> load_weights(const std::string &path) {
  SafeTensors st(path);
  // get (src/weights.rs:22-51): existence, exact shape, dtype conversion, finiteness.
  auto get = [&](const std::string &name, const std::vector<size_t> &shape) {
    const TensorView *t = st.find(name);
    if (!t) throw WeightsError("missing tensor " + name);
    if (t->shape != shape)
      throw WeightsError(name + ": expected " + shape_str(shape) + ", found " + shape_str(t->shape));
    std::vector<float> v;
    if (t->dtype == "F32") {
      v.resize(t->bytes / 4);
      std::memcpy(v.data(), t->data, t->bytes);
    } else if (t->dtype == "F16" || t->dtype == "BF16") {
      v.resize(t->bytes / 2);
      const bool bf = t->dtype == "BF16";
      for (size_t i = 0; i < v.size(); ++i) {
        uint16_t h;
        std::memcpy(&h, t->data + 2 * i, 2);
        v[i] = bf ? bf16_to_f32(h) : f16_to_f32(h);
      }
    } else {
      throw WeightsError("unsupported dtype " + t->dtype + " for " + name);
    }
    for (float x : v)
      if (!std::isfinite(x)) throw WeightsError("non-finite tensor " + name);
    return v;
  };
  std::map<std::string, Packed> out;
  auto emit = [&](const std::string &name, const std::vector<float> &values, bool half) {
    Packed p;
    p.half = half;
    if (half) {
      p.h.resize(values.size());
      std::string msg;
      if (pack_f16(name, values.data(), values.size(), p.h.data(), &msg) != SIZE_MAX)
        throw WeightsError(msg);
    } else {
      p.f = values;
    }
    out[name] = std::move(p);
  };
  const size_t H = kHidden;
  emit("patch_w", get("embeddings.patch_embeddings.weight", {H, 3, 16, 16}), true);
  emit("patch_b", get("embeddings.patch_embeddings.bias", {H}), false);
  {
    auto prefix = get("embeddings.cls_token", {1, 1, H});
    auto regs = get("embeddings.register_tokens", {1, 4, H});
    prefix.insert(prefix.end(), regs.begin(), regs.end());
    emit("prefix", prefix, false);
  }
  for (int i = 0; i < 12; ++i) {
    const std::string p = "layer." + std::to_string(i) + ".";
    const std::string s = "l" + std::to_string(i) + "_";
    const char *vecs[6][2] = {{"norm1_w", "norm1.weight"}, {"norm1_b", "norm1.bias"},
                              {"norm2_w", "norm2.weight"}, {"norm2_b", "norm2.bias"},
                              {"ls1", "layer_scale1.lambda1"}, {"ls2", "layer_scale2.lambda1"}};
    for (auto &v : vecs) emit(s + v[0], get(p + v[1], {H}), false);
    std::vector<float> qw, qb;
    for (const char *q : {"q", "k", "v"}) {
      auto w = get(p + "attention." + q + "_proj.weight", {H, H});
      qw.insert(qw.end(), w.begin(), w.end());
      if (std::string(q) == "k") {
        qb.insert(qb.end(), H, 0.0f);  // no key bias (src/weights.rs:97-101)
      } else {
        auto b = get(p + "attention." + q + "_proj.bias", {H});
        qb.insert(qb.end(), b.begin(), b.end());
      }
    }
    emit(s + "qkv_w", qw, true);
    emit(s + "qkv_b", qb, false);
    auto gw = get(p + "mlp.gate_proj.weight", {static_cast<size_t>(kMlp), H});
    auto uw = get(p + "mlp.up_proj.weight", {static_cast<size_t>(kMlp), H});
    gw.insert(gw.end(), uw.begin(), uw.end());
    auto gb = get(p + "mlp.gate_proj.bias", {static_cast<size_t>(kMlp)});
    auto ub = get(p + "mlp.up_proj.bias", {static_cast<size_t>(kMlp)});
    gb.insert(gb.end(), ub.begin(), ub.end());
    emit(s + "gateup_w", gw, true);
    emit(s + "gateup_b", gb, false);
    emit(s + "o_w", get(p + "attention.o_proj.weight", {H, H}), true);
    emit(s + "o_b", get(p + "attention.o_proj.bias", {H}), false);
    emit(s + "down_w", get(p + "mlp.down_proj.weight", {H, static_cast<size_t>(kMlp)}), true);
    emit(s + "down_b", get(p + "mlp.down_proj.bias", {H}), false);
  }
  emit("norm_w", get("norm.weight", {H}), false);
  emit("norm_b", get("norm.bias", {H}), false);
  {  // RoPE tables in f64, stored f32 (src/weights.rs:127-144)
    std::vector<float> c, sn;
    for (int y = 0; y < 14; ++y)
      for (int x = 0; x < 14; ++x)
        for (int rep = 0; rep < 2; ++rep)
          for (int pos : {y, x})
            for (int j = 0; j < 16; ++j) {
              const double coord = 2.0 * (pos + 0.5) / 14.0 - 1.0;
              const double a = 2.0 * M_PI * coord / std::pow(100.0, j / 16.0);
              c.push_back(static_cast<float>(std::cos(a)));
              sn.push_back(static_cast<float>(std::sin(a)));
            }
    emit("rope_cos", c, false);
    emit("rope_sin", sn, false);
  }
  // Re-tile gate||up into the kernel's interleaved order (64 gate rows, then the matching 64
  // up rows), so one 256-wide N tile of the gate/up GEMM holds matching gate and up columns.
  for (int i = 0; i < 12; ++i) {
    const std::string s = "l" + std::to_string(i) + "_";
    Packed &w = out[s + "gateup_w"];
    Packed &b = out[s + "gateup_b"];
    std::vector<uint16_t> wp(w.h.size());
    std::vector<float> bp(b.f.size());
    for (uint32_t r = 0; r < static_cast<uint32_t>(kGateUp); ++r) {
      const uint32_t src = gateup_source_row(r);
      std::memcpy(&wp[static_cast<size_t>(r) * H], &w.h[static_cast<size_t>(src) * H], H * 2);
      bp[r] = b.f[src];
    }
    w.h = std::move(wp);
    b.f = std::move(bp);
  }
  // LayerNorm folded into the GEMM that consumes it (no counterpart in the reference). With
  // h = (x - mu) rstd gamma + beta and W the packed f16 weights,
  //   h W^T + b = rstd (x W'^T - mu s + c / rstd),  W' = f16(W gamma),  s[n] = sum_k W'[n][k],
  //   c[n] = b[n] + sum_k W[n][k] beta[k],
  // so the kernel that updates x leaves only the row's statistics and the QKV and gate/up GEMMs
  // read x itself. The correction -mu s + c / rstd is a rank-2 product that the tensor cores add
  // as one more K=16 step: the row side holds (-mu_hi, -mu_lo, -mu_hi, r_hi, r_lo, r_hi, 0...)
  // with r = 1 / rstd, and W_aux[n] = (s_hi, s_hi, s_lo, c_hi, c_hi, c_lo, 0...), each value
  // split into an f16 and the f16 of its remainder, so the products sum to -mu s + r c up to
  // 2^-22 of their size. s sums the rounded W', so rstd (x W'^T - mu s) = rstd ((x - mu) W'^T)
  // up to the f32 accumulation. Emitted after every reference tensor, so the reference's first
  // error is still the one reported.
  auto fold = [&](const std::string &s, const std::string &mat, const std::string &norm) {
    const Packed &w = out.at(s + mat + "_w");
    const Packed &b = out.at(s + mat + "_b");
    const std::vector<float> &g = out.at(s + norm + "_w").f, &be = out.at(s + norm + "_b").f;
    const size_t n = b.f.size();
    std::vector<float> wf(w.h.size());
    std::vector<double> cv(n);
    for (size_t r = 0; r < n; ++r) {
      double c = b.f[r];
      for (size_t k = 0; k < H; ++k) {
        const float v = f16_to_f32(w.h[r * H + k]);
        wf[r * H + k] = v * g[k];
        c += static_cast<double>(v) * be[k];
      }
      cv[r] = c;
    }
    emit(s + mat + "_wf", wf, true);
    const std::vector<uint16_t> &packed = out.at(s + mat + "_wf").h;
    auto hi = [](double v) { return f16_to_f32(f32_to_f16(static_cast<float>(v))); };
    std::vector<float> aux(16 * n, 0.0f);
    for (size_t r = 0; r < n; ++r) {
      double sum = 0.0;
      for (size_t k = 0; k < H; ++k) sum += f16_to_f32(packed[r * H + k]);
      const float sh = hi(sum), ch = hi(cv[r]);
      float *a = &aux[16 * r];
      a[0] = sh;
      a[1] = sh;
      a[2] = static_cast<float>(sum - sh);
      a[3] = ch;
      a[4] = ch;
      a[5] = static_cast<float>(cv[r] - ch);
    }
    emit(s + mat + "_aux", aux, true);
  };
  for (int i = 0; i < 12; ++i) {
    const std::string s = "l" + std::to_string(i) + "_";
    fold(s, "qkv", "norm1");
    fold(s, "gateup", "norm2");
  }
  return out;
}

}  // namespace dv3
