// Config parsing / validation / catalogue and the host quantizers
// (crates/omg-wgpu/src/model.rs).
#include "model.h"

#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "capi_util.h"
#include "json.h"

namespace omg {

uint16_t f32_to_f16(float v) {
  const __half h = __float2half_rn(v);
  uint16_t b;
  std::memcpy(&b, &h, 2);
  return b;
}

float f16_to_f32(uint16_t b) {
  __half h;
  std::memcpy(&h, &b, 2);
  return __half2float(h);
}

Config Config::from_json(const std::string& text) {
  const Json root = Json::parse(text);
  // HF multimodal configs nest the text model (model.rs:68-73).
  const Json& v = root.has("text_config") ? root["text_config"] : root;
  Config c;
  const std::string* mt = v["model_type"].as_str();
  const std::string model_type = mt ? *mt : "gemma3_text";
  c.arch = (model_type == "gemma4_text" || model_type == "gemma4") ? Arch::Gemma4 : Arch::Gemma3;
  auto n = [&](const char* k) -> int {
    uint64_t x;
    if (!v[k].as_u64(&x)) fail("config.json: missing %s", k);
    return static_cast<int>(x);
  };
  c.layers = n("num_hidden_layers");
  const int layers = c.layers;
  if (v["layer_types"].kind == Json::Array) {
    for (const Json& t : v["layer_types"].arr) {
      const std::string* s = t.as_str();
      c.sliding.push_back(s && *s == "sliding_attention");
    }
  } else {
    // Older configs: every k-th layer is global (model.rs:85-91).
    uint64_t k = 6;
    v["_sliding_window_pattern"].as_u64(&k);
    for (int i = 0; i < layers; ++i) c.sliding.push_back((i + 1) % static_cast<int>(k) != 0);
  }
  if (static_cast<int>(c.sliding.size()) != layers)
    fail("config.json: layer_types has %zu entries for %d layers", c.sliding.size(), layers);
  const Json& rope = v["rope_parameters"];
  auto theta = [&](const char* kind, double fallback) -> float {
    double x;
    if (rope[kind]["rope_theta"].as_f64(&x)) return static_cast<float>(x);
    return static_cast<float>(fallback);
  };
  double fb_global = 1e6, fb_local = 1e4;
  v["rope_theta"].as_f64(&fb_global);
  v["rope_local_base_freq"].as_f64(&fb_local);
  c.theta_global = theta("full_attention", fb_global);
  c.theta_local = theta("sliding_attention", fb_local);
  const int hd_local = n("head_dim");
  uint64_t hg;
  const int hd_global = v["global_head_dim"].as_u64(&hg) ? static_cast<int>(hg) : hd_local;
  for (int i = 0; i < layers; ++i) c.head_dim.push_back(c.sliding[i] ? hd_local : hd_global);
  auto rot = [&](const char* kind) -> double {
    double x;
    return rope[kind]["partial_rotary_factor"].as_f64(&x) ? x : 1.0;
  };
  const double rot_local = rot("sliding_attention"), rot_global = rot("full_attention");
  for (int i = 0; i < layers; ++i)
    c.rope_dims.push_back(static_cast<int>(static_cast<double>(c.head_dim[i]) *
                                           (c.sliding[i] ? rot_local : rot_global)));
  uint64_t shared = 0;
  v["num_kv_shared_layers"].as_u64(&shared);
  if (static_cast<int>(shared) >= layers)
    fail("num_kv_shared_layers %d >= %d layers", static_cast<int>(shared), layers);
  const int first_shared = layers - static_cast<int>(shared);
  for (int i = 0; i < layers; ++i) {
    int src = i;
    if (i >= first_shared) {
      // The last own-K/V layer of the same attention type (model.rs:126-140).
      for (int j = first_shared - 1; j >= 0; --j)
        if (c.sliding[j] == c.sliding[i]) {
          src = j;
          break;
        }
    }
    c.kv_source.push_back(src);
  }
  for (int i = 0; i < layers; ++i)
    if (c.kv_source[i] >= first_shared && c.kv_source[i] != i)
      fail("layer %d has no earlier K/V layer of its type to share", i);
  const Json& is = v["intermediate_size"];
  if (is.kind == Json::Array) {
    for (const Json& x : is.arr) {
      uint64_t f = 0;
      x.as_u64(&f);
      c.ff.push_back(static_cast<int>(f));
    }
  } else if (is.kind == Json::Number) {
    uint64_t base = 0;
    is.as_u64(&base);
    const bool dbl = v["use_double_wide_mlp"].kind == Json::Bool && v["use_double_wide_mlp"].b;
    for (int i = 0; i < layers; ++i)
      c.ff.push_back(static_cast<int>(dbl && i >= first_shared ? base * 2 : base));
  } else {
    fail("config.json: missing intermediate_size");
  }
  if (static_cast<int>(c.ff.size()) != layers)
    fail("config.json: intermediate_size has %zu entries for %d layers", c.ff.size(), layers);
  if (c.arch == Arch::Gemma3) {
    double qps = hd_local;
    v["query_pre_attn_scalar"].as_f64(&qps);
    c.query_scale = std::pow(static_cast<float>(qps), -0.5f);
    c.norm_offset = 1.f;
    c.v_norm = false;
  } else {
    c.query_scale = 1.f;
    c.norm_offset = 0.f;
    c.v_norm = true;
  }
  double off;
  if (v["omg_norm_offset"].as_f64(&off)) c.norm_offset = static_cast<float>(off);
  c.vocab = n("vocab_size");
  c.d = n("hidden_size");
  c.heads = n("num_attention_heads");
  c.kv_heads = n("num_key_value_heads");
  double eps = 1e-6;
  v["rms_norm_eps"].as_f64(&eps);
  c.eps = static_cast<float>(eps);
  uint64_t w = 512;
  v["sliding_window"].as_u64(&w);
  c.window = static_cast<int>(w);
  uint64_t pl = 0;
  v["hidden_size_per_layer_input"].as_u64(&pl);
  c.per_layer_dim = static_cast<int>(pl);
  double sc = 0;
  v["final_logit_softcapping"].as_f64(&sc);
  c.softcap = static_cast<float>(sc);
  uint64_t bos = 2;
  v["bos_token_id"].as_u64(&bos);
  c.bos = static_cast<uint32_t>(bos);
  return c;
}

void Config::validate() const {
  if (kv_heads == 0 || heads % kv_heads != 0)
    fail("num_key_value_heads %d must divide num_attention_heads %d", kv_heads, heads);
  const int hpg = heads / kv_heads;
  if (!(hpg == 1 || hpg == 2 || hpg == 4 || hpg == 8 || hpg == 16))
    fail("query heads per KV head must divide 16 (got %d / %d)", heads, kv_heads);
  for (int i = 0; i < layers; ++i) {
    const int hd = head_dim[i];
    if (hd != 256 && hd != 512) fail("layer %d: head_dim must be 256 or 512 (got %d)", i, hd);
    if (rope_dims[i] > hd || rope_dims[i] % 2 != 0)
      fail("layer %d: rope_dims %d for head_dim %d", i, rope_dims[i], hd);
    if (kv_source[i] != i && head_dim[kv_source[i]] != hd)
      fail("layer %d: shares K/V with layer %d of a different head_dim", i, kv_source[i]);
  }
  if (d % 32 != 0 || std::any_of(ff.begin(), ff.end(), [](int f) { return f % 32 != 0; }))
    fail("hidden_size and intermediate_size must be multiples of 32");
  if (per_layer_dim % 32 != 0) fail("hidden_size_per_layer_input must be a multiple of 32");
  if (d > 8192) fail("hidden_size %d exceeds the 8192 the row kernels hold", d);
}

int Config::max_head_dim() const {
  return head_dim.empty() ? 256 : *std::max_element(head_dim.begin(), head_dim.end());
}

int Config::max_ff() const { return ff.empty() ? 0 : *std::max_element(ff.begin(), ff.end()); }

std::vector<Config::TensorSpec> Config::tensors() const {
  std::vector<TensorSpec> v;
  v.push_back({"embed", {vocab, d}});
  v.push_back({"final_norm", {d}});
  if (per_layer_dim > 0) {
    v.push_back({"pl_model_proj", {static_cast<int64_t>(per_layer_dim) * layers, d}});
    v.push_back({"pl_proj_norm", {per_layer_dim}});
  }
  for (int l = 0; l < layers; ++l) {
    const int hd = head_dim[l], f = ff[l];
    auto n = [&](const char* s) { return "blk." + std::to_string(l) + "." + s; };
    v.push_back({n("attn_norm"), {d}});
    v.push_back({n("qkv"), {qkv_width(l), d}});
    v.push_back({n("q_norm"), {hd}});
    if (has_kv(l)) v.push_back({n("k_norm"), {hd}});
    v.push_back({n("o"), {d, static_cast<int64_t>(heads) * hd}});
    v.push_back({n("post_attn_norm"), {d}});
    v.push_back({n("ffn_norm"), {d}});
    v.push_back({n("gate"), {f, d}});
    v.push_back({n("up"), {f, d}});
    v.push_back({n("down"), {d, f}});
    v.push_back({n("post_ffn_norm"), {d}});
    if (per_layer_dim > 0) {
      v.push_back({n("pl_gate"), {per_layer_dim, d}});
      v.push_back({n("pl_proj"), {d, per_layer_dim}});
      v.push_back({n("pl_norm"), {d}});
      v.push_back({n("out_scale"), {1}});
    }
  }
  return v;
}

size_t payload_bytes(int dtype, size_t n) {
  return dtype == 0 ? n * 2 : (dtype == 1 ? n : n / 2);
}

static void put_f16(uint8_t* p, float v) {
  const uint16_t h = f32_to_f16(v);
  p[0] = static_cast<uint8_t>(h & 0xff);
  p[1] = static_cast<uint8_t>(h >> 8);
}

static float get_f16(const uint8_t* p) {
  return f16_to_f32(static_cast<uint16_t>(p[0] | (static_cast<uint16_t>(p[1]) << 8)));
}

void quantize_q8(const float* v, size_t n, uint8_t* codes, uint8_t* scales) {
  for (size_t b = 0; b < n / 32; ++b) {
    const float* blk = v + 32 * b;
    float amax = 0.f;
    for (int j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(blk[j]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_f16(scales + 2 * b, d);
    for (int j = 0; j < 32; ++j) {
      // Rust f32::round rounds half away from zero, as std::round does.
      float q = std::round(blk[j] * id);
      q = std::min(127.0f, std::max(-127.0f, q));
      codes[32 * b + j] = static_cast<uint8_t>(static_cast<int8_t>(q));
    }
  }
}

static int trunc_clamp15(float x) {
  // Rust `as i32` saturates and maps NaN to 0; then clamp(0, 15).
  int q = 0;
  if (x == x) q = x >= 2147483647.0f ? 2147483647 : (x <= -2147483648.0f ? INT32_MIN : static_cast<int>(x));
  return std::min(15, std::max(0, q));
}

void quantize_q4(const float* v, size_t n, uint8_t* codes, uint8_t* scales) {
  for (size_t b = 0; b < n / 32; ++b) {
    const float* blk = v + 32 * b;
    float max = 0.f, amax = 0.f;
    for (int j = 0; j < 32; ++j)
      if (std::fabs(blk[j]) > amax) {
        amax = std::fabs(blk[j]);
        max = blk[j];
      }
    const float d = max / -8.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    put_f16(scales + 2 * b, d);
    for (int j = 0; j < 16; ++j) {
      // Two roundings (multiply, then add), as Rust evaluates a * b + c.
      volatile float plo = blk[j] * id;
      volatile float phi = blk[j + 16] * id;
      const int lo = trunc_clamp15(plo + 8.5f);
      const int hi = trunc_clamp15(phi + 8.5f);
      codes[16 * b + j] = static_cast<uint8_t>(lo | (hi << 4));
    }
  }
}

void dequantize(int dtype, const uint8_t* codes, const uint8_t* scales, size_t n, float* out) {
  for (size_t i = 0; i < n; ++i) {
    if (dtype == 0) {
      out[i] = get_f16(codes + 2 * i);
    } else if (dtype == 1) {
      out[i] = static_cast<float>(static_cast<int8_t>(codes[i])) * get_f16(scales + 2 * (i / 32));
    } else {
      const size_t b = i / 32, j = i % 32;
      const uint8_t byte = codes[b * 16 + j % 16];
      const uint8_t q = j < 16 ? (byte & 0xf) : (byte >> 4);
      out[i] = (static_cast<float>(q) - 8.0f) * get_f16(scales + 2 * b);
    }
  }
}

}  // namespace omg
