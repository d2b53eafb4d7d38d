// The Laya / ModernBERT encoder engine (see laya.h), following
// crates/omg-wgpu/src/laya.rs: config parsing and the tensor catalogue
// (:88-328), the builder (:612-1084), the pass (:1138-1432) and the host
// scorer / act head (:1442-1543).
#include "laya.h"

#include <cuda_profiler_api.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>

#include "capi_util.h"
#include "json.h"

namespace omg {

// ---- config --------------------------------------------------------------------

LayaConfig LayaConfig::from_json(const std::string& text) {
  const Json root = Json::parse(text);
  const Json& enc = root;
  const Json& agent = root["laya_agent"];
  const Json& tokens = root["laya_tokens"];
  if (agent.kind != Json::Object) fail("config.json: missing laya_agent");
  if (tokens.kind != Json::Object) fail("config.json: missing laya_tokens");
  const std::string* mt = enc["model_type"].as_str();
  if (!mt || *mt != "modernbert")
    fail("encoder model_type \"%s\" is not modernbert", mt ? mt->c_str() : "null");
  if (const std::string* a = enc["hidden_activation"].as_str())
    if (*a != "gelu") fail("encoder hidden_activation %s is not gelu", a->c_str());
  auto n = [&](const char* k) -> int {
    uint64_t x;
    if (!enc[k].as_u64(&x)) fail("encoder/config.json: missing %s", k);
    return static_cast<int>(x);
  };
  LayaConfig c;
  c.layers = n("num_hidden_layers");
  uint64_t every = 3;
  enc["global_attn_every_n_layers"].as_u64(&every);
  if (enc["layer_types"].kind == Json::Array) {
    for (const Json& t : enc["layer_types"].arr) {
      const std::string* s = t.as_str();
      c.sliding.push_back(s && *s == "sliding_attention");
    }
  } else {
    for (int i = 0; i < c.layers; ++i)
      c.sliding.push_back(every == 0 || i % static_cast<int>(every) != 0);
  }
  if (static_cast<int>(c.sliding.size()) != c.layers)
    fail("layer_types has %zu entries for %d layers", c.sliding.size(), c.layers);
  const Json& rope = enc["rope_parameters"];
  auto theta = [&](const char* kind, const char* key, double fallback) -> float {
    double x;
    if (rope[kind]["rope_theta"].as_f64(&x)) return static_cast<float>(x);
    if (enc[key].as_f64(&x)) return static_cast<float>(x);
    return static_cast<float>(fallback);
  };
  // The special tokens: surface form from laya_tokens, id from the
  // caller-resolved map (the reference's tokenizer lookup).
  const Json& ids = root["laya_special_ids"];
  auto tok = [&](const char* name, std::string* text_out) -> uint32_t {
    const Json& v = tokens[name];
    const std::string* text = v.as_str();
    if (!text) text = v["content"].as_str();
    if (!text) fail("tokenizer_config.json: missing %s", name);
    uint64_t id;
    if (!ids[*text].as_u64(&id)) fail("tokenizer has no %s", text->c_str());
    if (text_out) *text_out = *text;
    return static_cast<uint32_t>(id);
  };
  c.mask = tok("mask_token", &c.mask_text);
  if (agent["temperature"].kind == Json::Array) {
    const auto& t = agent["temperature"].arr;
    if (t.size() != 3) fail("rl_agent_config.json: temperature has %zu entries", t.size());
    for (int i = 0; i < 3; ++i) {
      double x = 1.0;
      t[i].as_f64(&x);
      c.temperature[i] = static_cast<float>(x);
    }
  }
  if (agent["temperature_by_options"].kind == Json::Object)
    for (const auto& kv : agent["temperature_by_options"].obj) {
      double x = 1.0;
      kv.second.as_f64(&x);
      c.temperature_by_options[kv.first] = static_cast<float>(x);
    }
  for (float t : c.temperature)
    if (!std::isfinite(t) || t <= 0.f) fail("calibration temperatures must be finite and positive");
  for (const auto& kv : c.temperature_by_options)
    if (!std::isfinite(kv.second) || kv.second <= 0.f)
      fail("calibration temperatures must be finite and positive");
  uint64_t u;
  c.max_len = agent["max_len"].as_u64(&u) ? static_cast<int>(u) : 512;
  c.head_max_len = agent["head_max_len"].as_u64(&u) ? static_cast<int>(u) : 192;
  if (!(4 < c.head_max_len && c.head_max_len < c.max_len))
    fail("expected 4 < head_max_len %d < max_len %d", c.head_max_len, c.max_len);
  c.d = n("hidden_size");
  c.heads = n("num_attention_heads");
  c.vocab = n("vocab_size");
  c.ff = n("intermediate_size");
  c.window = enc["local_attention"].as_u64(&u) ? static_cast<int>(u) / 2 : 64;
  c.theta_global = theta("full_attention", "global_rope_theta", 160000.0);
  c.theta_local = theta("sliding_attention", "local_rope_theta", 10000.0);
  double eps;
  if (enc["norm_eps"].as_f64(&eps) || enc["layer_norm_eps"].as_f64(&eps))
    c.eps = static_cast<float>(eps);
  else
    c.eps = 1e-5f;
  c.head_layers = agent["head_layers"].as_u64(&u) ? static_cast<int>(u) : 2;
  c.type_emb = agent["type_emb"].kind == Json::Bool ? agent["type_emb"].b : true;
  c.act_hidden = 256;
  if (agent["act_head"].kind == Json::Bool && !agent["act_head"].b)
    c.act_out = 0;
  else
    c.act_out = agent["act_costs"].kind == Json::Object
                    ? static_cast<int>(agent["act_costs"].obj.size()) + 1
                    : 0;
  c.cls = tok("cls_token", nullptr);
  c.sep = tok("sep_token", nullptr);
  c.pad = tok("pad_token", nullptr);
  c.validate();
  return c;
}

void LayaConfig::validate() const {
  if (heads <= 0 || d % heads != 0) fail("hidden_size %d / heads %d", d, heads);
  const int hd = head_dim();
  // attention_bi: every invocation owns HD / KB output dims as vec4s, KB = 8
  // (engine.rs:66-69).
  const int kb = 8;
  if (hd % (4 * kb) != 0 || hd < 32) fail("head_dim %d must be a multiple of %d", hd, 4 * kb);
  if (d % 32 != 0 || ff % 32 != 0) fail("hidden_size and intermediate_size must be multiples of 32");
  if (d > 2048) fail("hidden_size %d > 2048", d);
  // This engine's kernels: tensor-core attention over 64-dim heads, one
  // warp per LayerNorm row in float4s.
  if (hd != kLayaHd) fail("head_dim %d: this engine runs 64-dim attention heads", hd);
  if (d % 128 != 0) fail("hidden_size %d must be a multiple of 128 on this engine", d);
  if (vocab <= 0 || layers <= 0) fail("vocab_size and num_hidden_layers must be positive");
  if (ff % 64 != 0) fail("intermediate_size %d must be a multiple of 64 on this engine", ff);
}

float LayaConfig::temperature_for(int qtype, size_t k) const {
  const char* size = k <= 2 ? "2" : k <= 5 ? "3-5" : k <= 10 ? "6-10" : "11+";
  static const char* kTypes[3] = {"choice", "score", "noul"};
  auto it = temperature_by_options.find(std::string(kTypes[qtype]) + ":" + size);
  return it != temperature_by_options.end() ? it->second : temperature[qtype];
}

std::vector<Config::TensorSpec> LayaConfig::tensors() const {
  std::vector<Config::TensorSpec> v;
  auto add = [&](std::string name, std::vector<int64_t> shape) {
    v.push_back(Config::TensorSpec{std::move(name), std::move(shape)});
  };
  add("embed", {vocab, d});
  add("embed_norm", {d});
  add("final_norm", {d});
  if (type_emb) add("type_emb", {3, d});
  for (int l = 0; l < layers; ++l) {
    const std::string p = "enc." + std::to_string(l) + ".";
    if (l > 0) add(p + "attn_norm", {d});
    add(p + "qkv", {3 * d, d});
    add(p + "o", {d, d});
    add(p + "mlp_norm", {d});
    add(p + "wi_val", {ff, d});
    add(p + "wi_gate", {ff, d});
    add(p + "wo", {d, ff});
  }
  for (int h = 0; h < head_layers; ++h) {
    const std::string p = "head." + std::to_string(h) + ".";
    add(p + "norm1_w", {d});
    add(p + "norm1_b", {d});
    add(p + "in_proj", {3 * d, d});
    add(p + "in_proj_b", {3 * d});
    add(p + "out_proj", {d, d});
    add(p + "out_proj_b", {d});
    add(p + "norm2_w", {d});
    add(p + "norm2_b", {d});
    add(p + "l1", {4 * d, d});
    add(p + "l1_b", {4 * d});
    add(p + "l2", {d, 4 * d});
    add(p + "l2_b", {d});
  }
  add("scorer.norm_w", {d});
  add("scorer.norm_b", {d});
  add("scorer.l1", {d, d});
  add("scorer.l1_b", {d});
  add("scorer.l2", {1, d});
  add("scorer.l2_b", {1});
  if (act_out > 0) {
    add("act.l1", {act_hidden, d + 4});
    add("act.l1_b", {act_hidden});
    add("act.l2", {act_out, act_hidden});
    add("act.l2_b", {act_out});
  }
  return v;
}

bool laya_is_host_tensor(const std::string& name) {
  return name.rfind("scorer.", 0) == 0 || name.rfind("act.", 0) == 0;
}

// ---- builder -------------------------------------------------------------------

static std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

LayaBuilder::LayaBuilder(LayaConfig cfg, int device) : cfg_(std::move(cfg)), device_(device) {
  cfg_.validate();
  int n = 0;
  CUDA_TRY(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) fail("CUDA device %d not present (%d visible)", device, n);
  CUDA_TRY(cudaSetDevice(device_));
  int major = 0, minor = 0;
  CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device_));
  CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device_));
  if (major != 10 || minor != 0)
    fail("device %d is sm_%d%d; this library is built for sm_100a (B200)", device, major, minor);
  CUDA_TRY(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  for (const auto& s : cfg_.tensors()) expected_[s.name] = s.shape;
}

LayaBuilder::~LayaBuilder() {
  if (stream_) cudaStreamDestroy(stream_);
}

std::vector<std::string> LayaBuilder::missing() const {
  std::vector<std::string> v;
  for (const auto& kv : expected_)
    if (!pushed_.count(kv.first)) v.push_back(kv.first);
  std::sort(v.begin(), v.end());
  return v;
}

static bool ends_with(const std::string& s, const char* suf) {
  const size_t n = std::strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

void LayaBuilder::push(const std::string& name, const HostTensor& t) {
  CUDA_TRY(cudaSetDevice(device_));
  auto it = expected_.find(name);
  if (it == expected_.end()) fail("unexpected tensor %s", name.c_str());
  if (t.shape != it->second)
    fail("%s: shape %s, expected %s", name.c_str(), shape_str(t.shape).c_str(),
         shape_str(it->second).c_str());
  const size_t n = t.numel();
  if (t.dtype < 0 || t.dtype > 2) fail("%s: unsupported dtype %d", name.c_str(), t.dtype);
  if (t.data.size() != payload_bytes(t.dtype, n))
    fail("%s: %zu payload bytes, expected %zu", name.c_str(), t.data.size(),
         payload_bytes(t.dtype, n));
  const size_t want_scales = t.dtype == 0 ? 0 : n / 32 * 2;
  if (t.scales.size() != want_scales)
    fail("%s: %zu scale bytes, expected %zu", name.c_str(), t.scales.size(), want_scales);
  std::vector<float> f(n);
  if (laya_is_host_tensor(name)) {
    // laya.rs:677-680: the scorer and act head stay on the host in f32.
    if (t.dtype != 0 && n % 32 != 0)
      fail("%s: a quantized tensor needs a multiple of 32 elements", name.c_str());
    dequantize(t.dtype, t.data.data(), t.scales.data(), n, f.data());
    host_[name] = std::move(f);
    pushed_[name] = true;
    return;
  }
  if (t.shape.size() == 1 && t.dtype != 0) fail("%s: 1-D tensors must be f16", name.c_str());
  if (t.shape.size() == 2 && t.shape[1] % 32 != 0)
    fail("%s: inner dimension %lld is not a multiple of 32", name.c_str(),
         static_cast<long long>(t.shape[1]));
  if (t.shape.size() == 1 || name == "type_emb") {
    // Vectors (and the 3-row type embedding) as f32 copies of their values.
    dequantize(t.dtype, t.data.data(), t.scales.data(), n, f.data());
    DevBuffer b;
    b.alloc(n * 4, false);
    CUDA_TRY(cudaMemcpy(b.p, f.data(), n * 4, cudaMemcpyHostToDevice));
    vec_[name] = std::move(b);
    pushed_[name] = true;
    return;
  }
  if (name == "embed") {
    embed_dtype_ = t.dtype;
    embed_codes_.alloc(t.data.size(), false);
    CUDA_TRY(cudaMemcpy(embed_codes_.p, t.data.data(), t.data.size(), cudaMemcpyHostToDevice));
    embed_scales_.alloc(std::max<size_t>(t.scales.size(), 16), true);
    if (!t.scales.empty())
      CUDA_TRY(cudaMemcpy(embed_scales_.p, t.scales.data(), t.scales.size(),
                          cudaMemcpyHostToDevice));
    pushed_[name] = true;
    return;
  }
  // A linear: dequantized once into f16 rows (the values matmul.wgsl rounds
  // its weight operand to on every use).
  const int rows = static_cast<int>(t.shape[0]), k = static_cast<int>(t.shape[1]);
  DevBuffer codes, scales;
  codes.alloc(t.data.size(), false);
  CUDA_TRY(cudaMemcpy(codes.p, t.data.data(), t.data.size(), cudaMemcpyHostToDevice));
  if (!t.scales.empty()) {
    scales.alloc(t.scales.size(), false);
    CUDA_TRY(cudaMemcpy(scales.p, t.scales.data(), t.scales.size(), cudaMemcpyHostToDevice));
  }
  std::string key = name;
  int remap = 0;
  size_t out_rows = static_cast<size_t>(rows);
  if (ends_with(name, ".wi_val") || ends_with(name, ".wi_gate")) {
    // GeGLU layout of gemm.cu: [val 128 | gate 128] row blocks, so one MMA
    // tile holds gelu's input and its gate for the same 128 columns.
    key = name.substr(0, name.rfind('.')) + ".wi";
    remap = ends_with(name, ".wi_val") ? 1 : 2;
    out_rows = static_cast<size_t>((rows + 127) / 128) * 256;
  }
  auto lit = lin_.find(key);
  if (lit == lin_.end()) {
    DevBuffer b;
    b.alloc(out_rows * k * 2, remap != 0);
    lit = lin_.emplace(key, std::move(b)).first;
  }
  launch_dequant_f16(t.dtype, codes.p, scales.p, rows, k, remap, lit->second.as<__half>(), stream_);
  CUDA_TRY(cudaGetLastError());
  CUDA_TRY(cudaStreamSynchronize(stream_));
  pushed_[name] = true;
}

std::unique_ptr<LayaEngine> LayaBuilder::finish(size_t capacity, size_t max_rows) {
  const auto miss = missing();
  if (!miss.empty()) {
    std::string e;
    for (size_t i = 0; i < std::min<size_t>(4, miss.size()); ++i) e += (i ? ", " : "") + miss[i];
    fail("%zu tensors missing, e.g. %s", miss.size(), e.c_str());
  }
  if (capacity == 0) fail("capacity must be positive");
  return std::unique_ptr<LayaEngine>(new LayaEngine(std::move(*this), capacity, max_rows));
}

// ---- engine --------------------------------------------------------------------

LayaEngine::LayaEngine(LayaBuilder&& b, size_t capacity_, size_t max_rows_)
    : config(b.cfg_), capacity(capacity_), max_rows(max_rows_), device_(b.device_) {
  CUDA_TRY(cudaSetDevice(device_));
  CUDA_TRY(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device_));
  stream_ = b.stream_;
  b.stream_ = nullptr;
  lin_ = std::move(b.lin_);
  vec_ = std::move(b.vec_);
  // The decision head's f32 weights (laya.rs:677-680 keeps them on the host
  // in f32; here they run on the device in f32).
  for (auto& kv : b.host_) {
    DevBuffer& buf = headw_[kv.first];
    buf.alloc(kv.second.size() * 4, false);
    CUDA_TRY(cudaMemcpy(buf.p, kv.second.data(), kv.second.size() * 4, cudaMemcpyHostToDevice));
  }
  l2_bias_ = b.host_.at("scorer.l2_b").at(0);
  b.host_.clear();
  embed_dtype_ = b.embed_dtype_;
  embed_codes_ = std::move(b.embed_codes_);
  embed_scales_ = std::move(b.embed_scales_);
  gemm_setup_device();
  laya_setup_device();

  const LayaConfig& c = config;
  const int d = c.d, ff = c.ff, L = c.layers;
  // Rows rounded up to whole 128-row tiles.
  cap_rows_ = (capacity + kLayaTile - 1) / kLayaTile * kLayaTile;
  const size_t R = cap_rows_;
  act_stride_ = std::max(ff, c.head_layers > 0 ? 4 * d : 0);

  // Workspace. Zero-initialised, so rows a kernel reads past the pass's
  // tokens (tile tails) are finite.
  ids_.alloc(R * 4);
  pos_.alloc(R * 4);
  qtype_.alloc(R * 4);
  span_.alloc(R * sizeof(int2));
  row_map_.alloc(std::max<size_t>(max_rows, 1) * 4);
  x_.alloc(R * d * 4);
  h16_.alloc(R * d * 2);
  qkv16_.alloc(R * 3 * d * 2);
  attn16_.alloc(R * d * 2);
  act16_.alloc(R * act_stride_ * 2);
  rows_.alloc(std::max<size_t>(max_rows, 1) * d * 4);
  // Head indices: max_rows int4 sequence entries, then max_rows marker rows;
  // head outputs: max_rows logits, then max_rows act probabilities.
  head_idx_.alloc(std::max<size_t>(max_rows, 1) * (sizeof(int4) + 4));
  h_head_idx_.alloc(std::max<size_t>(max_rows, 1) * (sizeof(int4) + 4));
  head_out_.alloc(std::max<size_t>(max_rows, 1) * 2 * 4);
  status_.alloc(16);
  h_ids_.alloc(R * 4);
  h_pos_.alloc(R * 4);
  h_qtype_.alloc(R * 4);
  h_span_.alloc(R * sizeof(int2));
  h_row_map_.alloc(std::max<size_t>(max_rows, 1) * 4);
  h_out_.alloc(std::max<size_t>(max_rows, 1) * d * 4);
  h_status_.alloc(16);
  for (auto& e : events_) CUDA_TRY(cudaEventCreate(&e));

  // RoPE tables for the two thetas over every position a sequence may have.
  const int hd = c.head_dim();
  rope_local_.alloc(static_cast<size_t>(c.max_len) * (hd / 2) * sizeof(float2), false);
  rope_global_.alloc(static_cast<size_t>(c.max_len) * (hd / 2) * sizeof(float2), false);
  launch_laya_rope_table(c.theta_local, hd, c.max_len, rope_local_.as<float2>(), stream_);
  launch_laya_rope_table(c.theta_global, hd, c.max_len, rope_global_.as<float2>(), stream_);
  CUDA_TRY(cudaGetLastError());

  char err[256];
  if (!laya_attention_map(&tqkv_, qkv16_.p, static_cast<int>(R), d, err, sizeof err))
    fail("%s", err);
  auto W = [&](const std::string& n) -> const void* {
    auto it = lin_.find(n);
    if (it == lin_.end()) fail("missing tensor %s", n.c_str());
    return it->second.p;
  };
  auto V = [&](const std::string& n) -> const float* {
    auto it = vec_.find(n);
    if (it == vec_.end()) fail("missing tensor %s", n.c_str());
    return it->second.as<float>();
  };
  auto plan = [&](GemmPlan* p, const void* a, int lda, const std::string& w, int w_rows, int n_out,
                  int k, int epi) {
    if (!gemm_plan(p, a, static_cast<int>(R), lda, W(w), w_rows, n_out, k, epi,
                   n_out % 256 == 0 || epi == kEpiGeGluErf ? 256 : 128, 1, err, sizeof err))
      fail("%s: %s", w.c_str(), err);
    // Batches of many rows take the CTA-pair kernel (same results).
    if (p->s.bn == 256 &&
        !gemm_plan_pair(p, W(w), w_rows, false, err, sizeof err))
      fail("%s: %s", w.c_str(), err);
  };
  embed_norm_ = V("embed_norm");
  final_norm_ = V("final_norm");
  type_emb_ = c.type_emb ? V("type_emb") : nullptr;
  enc_.resize(L);
  for (int l = 0; l < L; ++l) {
    EncLayer& e = enc_[l];
    const std::string p = "enc." + std::to_string(l) + ".";
    e.sliding = c.sliding[l];
    e.attn_norm = l > 0 ? V(p + "attn_norm") : nullptr;
    e.mlp_norm = V(p + "mlp_norm");
    plan(&e.qkv, h16_.p, d, p + "qkv", 3 * d, 3 * d, d, kEpiRopeF16);
    plan(&e.o, attn16_.p, d, p + "o", d, d, d, kEpiResidF32);
    plan(&e.wi, h16_.p, d, p + "wi", (ff + 127) / 128 * 256, ff, d, kEpiGeGluErf);
    plan(&e.wo, act16_.p, act_stride_, p + "wo", d, d, ff, kEpiResidF32);
  }
  head_.resize(c.head_layers);
  for (int h = 0; h < c.head_layers; ++h) {
    HeadLayer& e = head_[h];
    const std::string p = "head." + std::to_string(h) + ".";
    e.n1w = V(p + "norm1_w");
    e.n1b = V(p + "norm1_b");
    e.in_b = V(p + "in_proj_b");
    e.out_b = V(p + "out_proj_b");
    e.n2w = V(p + "norm2_w");
    e.n2b = V(p + "norm2_b");
    e.l1_b = V(p + "l1_b");
    e.l2_b = V(p + "l2_b");
    plan(&e.in, h16_.p, d, p + "in_proj", 3 * d, 3 * d, d, kEpiBiasF16);
    plan(&e.out, attn16_.p, d, p + "out_proj", d, d, d, kEpiResidF32);
    plan(&e.l1, h16_.p, d, p + "l1", 4 * d, 4 * d, d, kEpiBiasReluF16);
    plan(&e.l2, act16_.p, act_stride_, p + "l2", d, d, 4 * d, kEpiResidF32);
  }
  CUDA_TRY(cudaStreamSynchronize(stream_));
}

LayaEngine::~LayaEngine() {
  if (stream_) {
    cudaSetDevice(device_);
    cudaStreamSynchronize(stream_);
  }
  for (auto e : events_)
    if (e) cudaEventDestroy(e);
  for (auto e : prof_events_) cudaEventDestroy(e);
  if (stream_) cudaStreamDestroy(stream_);
}

// laya.rs:1142-1199: validation, packing and the read-back plan.
LayaEngine::Packing LayaEngine::pack(const LayaSequence* seqs, size_t n) const {
  const LayaConfig& c = config;
  size_t total = 0;
  for (size_t i = 0; i < n; ++i) total += seqs[i].n_ids;
  if (total == 0) fail("empty request");
  if (total > capacity) fail("%zu tokens exceed the engine capacity %zu", total, capacity);
  Packing p;
  p.t = total;
  p.ids.reserve(total);
  p.pos.reserve(total);
  p.qtype.reserve(total);
  p.span.reserve(total);
  for (size_t si = 0; si < n; ++si) {
    const LayaSequence& s = seqs[si];
    if (s.n_ids == 0) fail("sequence %zu is empty", si);
    if (s.n_ids > static_cast<size_t>(c.max_len))
      fail("sequence %zu: %zu tokens > max_len %d", si, s.n_ids, c.max_len);
    if (s.qtype < 0 || s.qtype >= 3) fail("sequence %zu: question type %d", si, s.qtype);
    const int start = static_cast<int>(p.ids.size());
    const int end = start + static_cast<int>(s.n_ids);
    for (size_t i = 0; i < s.n_ids; ++i) {
      const uint32_t t = s.ids[i];
      if (static_cast<int64_t>(t) >= c.vocab)
        fail("token id %u outside the vocabulary of %d", t, c.vocab);
      p.ids.push_back(static_cast<int32_t>(t));
      p.pos.push_back(static_cast<int32_t>(i));
      p.qtype.push_back(s.qtype);
      p.span.push_back(make_int2(start, end));
    }
    p.head_seq.push_back(make_int4(static_cast<int>(p.row_map.size()),
                                   static_cast<int>(p.marker_row.size()),
                                   static_cast<int>(s.n_markers), 0));
    p.row_map.push_back(start);
    for (size_t j = 0; j < s.n_markers; ++j) {
      const size_t m = s.markers[j];
      if (m >= s.n_ids) fail("sequence %zu: marker %zu past its %zu tokens", si, m, s.n_ids);
      p.marker_row.push_back(static_cast<int32_t>(p.row_map.size()));
      p.row_map.push_back(start + static_cast<int32_t>(m));
    }
  }
  if (p.row_map.size() > max_rows)
    fail("%zu rows requested, engine reads back at most %zu", p.row_map.size(), max_rows);
  const int t = static_cast<int>(total);
  laya_attention_items(p.span.data(), t, c.window, &p.items[0]);
  laya_attention_items(p.span.data(), t, 0, &p.items[1]);
  return p;
}

void LayaEngine::upload(const Packing& p) {
  const size_t t = p.t;
  std::memcpy(h_ids_.p, p.ids.data(), t * 4);
  std::memcpy(h_pos_.p, p.pos.data(), t * 4);
  std::memcpy(h_qtype_.p, p.qtype.data(), t * 4);
  std::memcpy(h_span_.p, p.span.data(), t * sizeof(int2));
  std::memcpy(h_row_map_.p, p.row_map.data(), p.row_map.size() * 4);
  CUDA_TRY(cudaMemcpyAsync(ids_.p, h_ids_.p, t * 4, cudaMemcpyHostToDevice, stream_));
  CUDA_TRY(cudaMemcpyAsync(pos_.p, h_pos_.p, t * 4, cudaMemcpyHostToDevice, stream_));
  CUDA_TRY(cudaMemcpyAsync(qtype_.p, h_qtype_.p, t * 4, cudaMemcpyHostToDevice, stream_));
  CUDA_TRY(cudaMemcpyAsync(span_.p, h_span_.p, t * sizeof(int2), cudaMemcpyHostToDevice, stream_));
  CUDA_TRY(cudaMemcpyAsync(row_map_.p, h_row_map_.p, p.row_map.size() * 4,
                           cudaMemcpyHostToDevice, stream_));
  {
    // Sequences and markers number at most the rows read back (<= max_rows).
    const size_t cap = std::max<size_t>(max_rows, 1);
    auto* hs = h_head_idx_.as<int4>();
    std::memcpy(hs, p.head_seq.data(), p.head_seq.size() * sizeof(int4));
    std::memcpy(reinterpret_cast<int32_t*>(hs + cap), p.marker_row.data(),
                p.marker_row.size() * 4);
    CUDA_TRY(cudaMemcpyAsync(head_idx_.p, h_head_idx_.p, cap * (sizeof(int4) + 4),
                             cudaMemcpyHostToDevice, stream_));
  }
  // Attention items of both windows in one staged block; the buffers grow
  // to the largest pass seen.
  const size_t ni = p.items[0].size() + p.items[1].size();
  if (ni > items_cap_) {
    CUDA_TRY(cudaStreamSynchronize(stream_));
    const size_t cap = std::max<size_t>(ni * 2, 256);
    h_items_.alloc(cap * sizeof(LayaAttnItem));
    items_.alloc(cap * sizeof(LayaAttnItem), false);
    items_cap_ = cap;
  }
  auto* hi = h_items_.as<LayaAttnItem>();
  std::memcpy(hi, p.items[0].data(), p.items[0].size() * sizeof(LayaAttnItem));
  std::memcpy(hi + p.items[0].size(), p.items[1].data(), p.items[1].size() * sizeof(LayaAttnItem));
  CUDA_TRY(cudaMemcpyAsync(items_.p, h_items_.p, ni * sizeof(LayaAttnItem),
                           cudaMemcpyHostToDevice, stream_));
}

void LayaEngine::prof_mark(const char* name) {
  if (prof_used_ == prof_events_.size()) {
    cudaEvent_t e;
    CUDA_TRY(cudaEventCreate(&e));
    prof_events_.push_back(e);
    prof_names_.push_back(nullptr);
  }
  CUDA_TRY(cudaEventRecord(prof_events_[prof_used_], stream_));
  prof_names_[prof_used_] = name;
  ++prof_used_;
}

// laya.rs:1263-1345, one launch per step: the residual adds ride in the
// projections' epilogues and each LayerNorm is one row sweep.
int LayaEngine::launch_forward(const Packing& p, bool head) {
  const LayaConfig& c = config;
  const int t = static_cast<int>(p.t), d = c.d;
  uint32_t* status = status_.as<uint32_t>();
  CUDA_TRY(cudaMemsetAsync(status_.p, 0, 4, stream_));
  int launches = 0;
  auto k = [&](const char* name) {
    ++launches;
    if (profiling_) prof_mark(name);
  };
  float* x = x_.as<float>();
  __half* h16 = h16_.as<__half>();
  const int* pos = pos_.as<int>();
  const auto* items = items_.as<LayaAttnItem>();
  auto attention = [&](int w) {
    LayaAttnArgs a{};
    a.items = items + (w == 0 ? 0 : p.items[0].size());
    a.n_items = static_cast<int>(p.items[w].size());
    a.span = span_.as<int2>();
    a.out = attn16_.as<__half>();
    a.status = status;
    a.heads = c.heads;
    a.d = d;
    a.window = w == 0 ? c.window : 0;
    a.single_tile = 1;
    for (const LayaAttnItem& it : p.items[w])
      if (it.nk > kLayaTile) a.single_tile = 0;
    a.num_sms = num_sms_;
    k("attention");
    launch_laya_attention(tqkv_, a, stream_);
  };
  auto ln = [&](const float* w1, const float* b1, int in_place, const float* te, const float* w2,
                const float* b2) {
    LayaLnArgs a{};
    a.x = x;
    a.t = t;
    a.d = d;
    a.eps = c.eps;
    a.w1 = w1;
    a.b1 = b1;
    a.in_place = in_place;
    a.type_emb = te;
    a.qtype = qtype_.as<int>();
    a.w2 = w2;
    a.b2 = b2;
    a.h16 = h16;
    k("layernorm");
    launch_laya_ln(a, stream_);
  };
  GemmEpi resid{};

  k("embed_ln");
  launch_laya_embed_ln(embed_dtype_, ids_.as<int>(), t, embed_codes_.p, embed_scales_.p, d,
                       embed_norm_, c.eps, x, h16, stream_);
  for (int l = 0; l < c.layers; ++l) {
    const EncLayer& e = enc_[l];
    GemmEpi rope{};
    rope.rope = e.sliding ? rope_local_.as<float2>() : rope_global_.as<float2>();
    rope.rope_stride = c.max_len;
    rope.pos = pos;
    rope.q_scale = 1.0f / std::sqrt(static_cast<float>(c.head_dim()));
    rope.q_cols = d;
    k("gemm_qkv");
    gemm_run_epi(e.qkv, t, qkv16_.p, 3 * d, rope, status, stream_);
    attention(e.sliding ? 0 : 1);
    k("gemm_o");
    gemm_run_epi(e.o, t, x, d, resid, status, stream_);
    ln(e.mlp_norm, nullptr, 0, nullptr, nullptr, nullptr);
    k("gemm_wi");
    gemm_run(e.wi, t, act16_.p, act_stride_, 0, status, stream_);
    k("gemm_wo");
    gemm_run_epi(e.wo, t, x, d, resid, status, stream_);
    if (l + 1 < c.layers) {
      ln(enc_[l + 1].attn_norm, nullptr, 0, nullptr, nullptr, nullptr);
    } else {
      // x = final_norm(x) + type_emb[qtype], then the head's first norm1.
      const bool head = !head_.empty();
      ln(final_norm_, nullptr, 1, type_emb_, head ? head_[0].n1w : nullptr,
         head ? head_[0].n1b : nullptr);
    }
  }
  for (size_t hl = 0; hl < head_.size(); ++hl) {
    const HeadLayer& e = head_[hl];
    const bool last = hl + 1 == head_.size();
    GemmEpi bias_in{};
    bias_in.bias = e.in_b;
    k("gemm_in");
    gemm_run_epi(e.in, t, qkv16_.p, 3 * d, bias_in, status, stream_);
    // No RoPE and no query scale on the head's attention (laya.rs:1322-1327).
    attention(1);
    GemmEpi out{};
    out.bias = e.out_b;
    k("gemm_out");
    gemm_run_epi(e.out, t, x, d, out, status, stream_);
    ln(e.n2w, e.n2b, 0, nullptr, nullptr, nullptr);
    GemmEpi l1{};
    l1.bias = e.l1_b;
    k("gemm_l1");
    gemm_run_epi(e.l1, t, act16_.p, act_stride_, l1, status, stream_);
    GemmEpi l2{};
    l2.bias = e.l2_b;
    l2.bias_first = last ? 1 : 0;  // bias_act.wgsl: x = (a + b) + x on the last layer
    k("gemm_l2");
    gemm_run_epi(e.l2, t, x, d, l2, status, stream_);
    if (!last) ln(head_[hl + 1].n1w, head_[hl + 1].n1b, 0, nullptr, nullptr, nullptr);
  }
  k("gather");
  launch_laya_gather(x, d, row_map_.as<int>(), static_cast<int>(p.row_map.size()), rows_.as<float>(),
                     stream_);
  if (head) {
    // laya.rs:1442-1486 on the device: scorer logits of every marker, then
    // the act head of every sequence.
    const size_t cap = std::max<size_t>(max_rows, 1);
    const int4* hseq = head_idx_.as<int4>();
    const int* mrow = reinterpret_cast<const int*>(hseq + cap);
    float* logits = head_out_.as<float>();
    auto H = [&](const char* n) { return headw_.at(n).as<float>(); };
    LayaScoreArgs sa{};
    sa.rows = rows_.as<float>();
    sa.marker_row = mrow;
    sa.k = static_cast<int>(p.marker_row.size());
    sa.d = d;
    sa.norm_w = H("scorer.norm_w");
    sa.norm_b = H("scorer.norm_b");
    sa.l1 = H("scorer.l1");
    sa.l1_b = H("scorer.l1_b");
    sa.l2 = H("scorer.l2");
    sa.l2_b = l2_bias_;
    sa.eps = c.eps;
    sa.logits = logits;
    k("head_score");
    launch_laya_score(sa, stream_);
    if (c.act_out > 0) {
      LayaActArgs aa{};
      aa.rows = rows_.as<float>();
      aa.seq = hseq;
      aa.n = static_cast<int>(p.head_seq.size());
      aa.d = d;
      aa.hidden = c.act_hidden;
      aa.outs = c.act_out;
      aa.l1 = H("act.l1");
      aa.l1_b = H("act.l1_b");
      aa.l2 = H("act.l2");
      aa.l2_b = H("act.l2_b");
      aa.logits = logits;
      aa.act = logits + cap;
      k("head_act");
      launch_laya_act(aa, stream_);
    }
  }
  if (profiling_) prof_mark(nullptr);
  CUDA_TRY(cudaGetLastError());
  return launches;
}

void LayaEngine::check_status() {
  const uint32_t st = *h_status_.as<uint32_t>();
  if (st != 0) fail("a kernel gave up waiting (device status %u); the pass was abandoned", st);
}

void LayaEngine::hidden(const LayaSequence* seqs, size_t n, float* out, size_t out_floats) {
  std::lock_guard<std::mutex> g(mu_);
  CUDA_TRY(cudaSetDevice(device_));
  Packing p = pack(seqs, n);
  const size_t nrows = p.row_map.size(), d = config.d;
  if (out_floats < nrows * d)
    fail("output buffer holds %zu floats, the request returns %zu", out_floats, nrows * d);
  upload(p);
  launch_forward(p);
  CUDA_TRY(cudaMemcpyAsync(h_out_.p, rows_.p, nrows * d * 4, cudaMemcpyDeviceToHost, stream_));
  CUDA_TRY(cudaMemcpyAsync(h_status_.p, status_.p, 4, cudaMemcpyDeviceToHost, stream_));
  CUDA_TRY(cudaStreamSynchronize(stream_));
  check_status();
  std::memcpy(out, h_out_.p, nrows * d * 4);
}

// laya.rs:1489-1493's softmax for the calibrated probabilities.
static std::vector<float> host_softmax(const std::vector<float>& z) {
  float m = -INFINITY;
  for (float v : z) m = std::max(m, v);
  std::vector<float> e(z.size());
  float s = 0.f;
  for (size_t i = 0; i < z.size(); ++i) {
    e[i] = std::exp(z[i] - m);
    s += e[i];
  }
  for (float& v : e) v /= s;
  return e;
}

// laya.rs:1435-1486: the pass, then the decision head on the device (the
// reference reads the rows back and scores them on the host); only the
// logits and act probabilities come back.
std::vector<LayaOutput> LayaEngine::evaluate(const LayaSequence* seqs, size_t n) {
  std::lock_guard<std::mutex> g(mu_);
  CUDA_TRY(cudaSetDevice(device_));
  Packing p = pack(seqs, n);
  upload(p);
  launch_forward(p, true);
  const size_t cap = std::max<size_t>(max_rows, 1), k = p.marker_row.size();
  float* h = h_out_.as<float>();
  if (k) CUDA_TRY(cudaMemcpyAsync(h, head_out_.p, k * 4, cudaMemcpyDeviceToHost, stream_));
  if (config.act_out > 0)
    CUDA_TRY(cudaMemcpyAsync(h + cap, head_out_.as<float>() + cap, n * 4, cudaMemcpyDeviceToHost,
                             stream_));
  CUDA_TRY(cudaMemcpyAsync(h_status_.p, status_.p, 4, cudaMemcpyDeviceToHost, stream_));
  CUDA_TRY(cudaStreamSynchronize(stream_));
  check_status();
  std::vector<LayaOutput> out(n);
  for (size_t i = 0; i < n; ++i) {
    const int4 q = p.head_seq[i];
    out[i].logits.assign(h + q.y, h + q.y + q.z);
    if (config.act_out > 0) {
      out[i].has_act = true;
      out[i].act_probability = h[cap + i];
    }
  }
  return out;
}

std::vector<double> LayaEngine::probabilities(int qtype, const float* logits, size_t k) const {
  if (qtype < 0 || qtype >= 3) fail("question type %d", qtype);
  const float t = std::max(config.temperature_for(qtype, k), 1e-3f);
  std::vector<float> z(k);
  for (size_t i = 0; i < k; ++i) z[i] = logits[i] / t;
  const std::vector<float> p = host_softmax(z);
  return std::vector<double>(p.begin(), p.end());
}

void LayaEngine::warmup() {
  const uint32_t ids[3] = {config.cls, config.mask, config.sep};
  const size_t markers[1] = {1};
  LayaSequence s{ids, 3, markers, 1, 2};
  evaluate(&s, 1);
}

float LayaEngine::time_forward(const LayaSequence* seqs, size_t n, int iters, int* launches) {
  std::lock_guard<std::mutex> g(mu_);
  CUDA_TRY(cudaSetDevice(device_));
  Packing p = pack(seqs, n);
  upload(p);
  CUDA_TRY(cudaStreamSynchronize(stream_));
  int nl = 0;
  CUDA_TRY(cudaEventRecord(events_[6], stream_));
  for (int i = 0; i < iters; ++i) nl = launch_forward(p, true);
  CUDA_TRY(cudaEventRecord(events_[7], stream_));
  CUDA_TRY(cudaMemcpyAsync(h_status_.p, status_.p, 4, cudaMemcpyDeviceToHost, stream_));
  CUDA_TRY(cudaStreamSynchronize(stream_));
  check_status();
  float ms = 0;
  CUDA_TRY(cudaEventElapsedTime(&ms, events_[6], events_[7]));
  if (launches) *launches = nl;
  return ms;
}

std::string LayaEngine::profile_forward(const LayaSequence* seqs, size_t n, int iters) {
  std::lock_guard<std::mutex> g(mu_);
  CUDA_TRY(cudaSetDevice(device_));
  Packing p = pack(seqs, n);
  upload(p);
  profiling_ = true;
  prof_used_ = 0;
  // The profiled passes are the range an external profiler run with
  // --profile-from-start off captures.
  CUDA_TRY(cudaProfilerStart());
  for (int i = 0; i < iters; ++i) launch_forward(p, true);
  CUDA_TRY(cudaProfilerStop());
  profiling_ = false;
  CUDA_TRY(cudaMemcpyAsync(h_status_.p, status_.p, 4, cudaMemcpyDeviceToHost, stream_));
  CUDA_TRY(cudaStreamSynchronize(stream_));
  check_status();
  std::vector<std::pair<std::string, std::pair<int, double>>> acc;
  for (size_t i = 0; i + 1 < prof_used_; ++i) {
    if (!prof_names_[i]) continue;
    float ms = 0;
    CUDA_TRY(cudaEventElapsedTime(&ms, prof_events_[i], prof_events_[i + 1]));
    auto it = std::find_if(acc.begin(), acc.end(),
                           [&](const auto& e) { return e.first == prof_names_[i]; });
    if (it == acc.end()) {
      acc.push_back({prof_names_[i], {0, 0.0}});
      it = acc.end() - 1;
    }
    it->second.first += 1;
    it->second.second += ms;
  }
  std::string s = "{";
  for (size_t i = 0; i < acc.size(); ++i) {
    char buf[160];
    snprintf(buf, sizeof buf, "%s\"%s\": [%d, %.6f]", i ? ", " : "", acc[i].first.c_str(),
             acc[i].second.first, acc[i].second.second);
    s += buf;
  }
  return s + "}";
}

void LayaEngine::record_event(int slot) {
  if (slot < 0 || slot >= 6) fail("event slot %d out of range", slot);
  CUDA_TRY(cudaSetDevice(device_));
  CUDA_TRY(cudaEventRecord(events_[slot], stream_));
}

float LayaEngine::elapsed_ms(int a, int b) {
  if (a < 0 || a >= 6 || b < 0 || b >= 6) fail("event slot out of range");
  CUDA_TRY(cudaEventSynchronize(events_[b]));
  float ms = 0;
  CUDA_TRY(cudaEventElapsedTime(&ms, events_[a], events_[b]));
  return ms;
}

}  // namespace omg
