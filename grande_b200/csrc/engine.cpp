// The decoder engine (see engine.h). Reference: crates/omg-wgpu/src/engine.rs.
#include "engine.h"
#include "packed.cuh"

#include <sys/stat.h>

#include <cuda_profiler_api.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>

#include "attention.cuh"
#include "capi_util.h"

namespace omg {

// The attention's P enters P.V as f16 only (the reference rounds Q, K and V
// to f16; P's own f16 rounding adds ~2^-12 relative error, below the f16
// rounding of the attention output that follows). Set to feed P's rounding
// residue too, for ~22-bit P: the branch rows of a pass then move by up to
// 3.4e-4 relative when the same branches sit at other cache rows, past the
// reference's 1e-4 layout tolerance (f16 P: 7e-6).
constexpr bool kAttnPLo = false;

// ---- buffers ----------------------------------------------------------------

void DevBuffer::alloc(size_t n, bool zero) {
  release();
  bytes = n ? n : 16;
  CUDA_TRY(cudaMalloc(&p, bytes));
  if (zero) {
    // cudaMemset runs on the legacy default stream, which does not order
    // with the engines' non-blocking streams: wait for it here, or a pass
    // launched right after could race with the zero fill.
    CUDA_TRY(cudaMemset(p, 0, bytes));
    CUDA_TRY(cudaStreamSynchronize(nullptr));
  }
}

void DevBuffer::release() {
  if (p) cudaFree(p);
  p = nullptr;
  bytes = 0;
}

void PinnedBuffer::alloc(size_t n) {
  if (p) cudaFreeHost(p);
  bytes = n ? n : 16;
  CUDA_TRY(cudaMallocHost(&p, bytes));
}

PinnedBuffer::~PinnedBuffer() {
  if (p) cudaFreeHost(p);
}

float HostTensor::get(size_t i) const {
  if (dtype == 0) return f16_to_f32(static_cast<uint16_t>(data[2 * i] | (data[2 * i + 1] << 8)));
  // Decode the 32-element block holding element i (model.rs:508-525).
  float blk[32];
  const size_t b = i / 32;
  dequantize(dtype, data.data() + (dtype == 1 ? b * 32 : b * 16), scales.data() + 2 * b, 32, blk);
  return blk[i % 32];
}

// ---- page-locked host blocks --------------------------------------------------

namespace {

// Page-locked blocks for saved states, reused across saves: pinning fresh
// memory costs more than copying 50 MB over the host link, so freed blocks
// (sizes rounded up to 1 MiB) go back to a pool that keeps up to 1 GiB idle.
// The pool is never destroyed (blocks may be freed after the CUDA runtime
// has begun to shut down at exit).
class HostBlocks {
 public:
  static HostBlocks& get() {
    static HostBlocks* pool = new HostBlocks();
    return *pool;
  }
  std::shared_ptr<uint8_t> take(size_t n) {
    const size_t size = (std::max<size_t>(n, 1) + kStep - 1) / kStep * kStep;
    uint8_t* p = nullptr;
    size_t got = size;
    {
      std::lock_guard<std::mutex> g(mu_);
      // The smallest idle block that holds `size` without wasting half of it.
      auto best = free_.end();
      for (auto it = free_.begin(); it != free_.end(); ++it)
        if (it->second >= size && it->second <= 2 * size &&
            (best == free_.end() || it->second < best->second))
          best = it;
      if (best != free_.end()) {
        p = best->first;
        got = best->second;
        idle_ -= got;
        free_.erase(best);
      }
    }
    bool pinned = true;
    if (!p && cudaHostAlloc(reinterpret_cast<void**>(&p), size, cudaHostAllocPortable) !=
                  cudaSuccess) {
      // Out of page-locked memory: pageable memory still works (slower copies).
      (void)cudaGetLastError();
      p = static_cast<uint8_t*>(std::malloc(size));
      pinned = false;
      if (!p) fail("out of host memory for a %zu-byte state", size);
    }
    return std::shared_ptr<uint8_t>(p, [this, got, pinned](uint8_t* q) { give(q, got, pinned); });
  }

 private:
  static constexpr size_t kStep = size_t(1) << 20;
  static constexpr size_t kKeepIdle = size_t(1) << 30;
  void give(uint8_t* p, size_t size, bool pinned) {
    if (!pinned) {
      std::free(p);
      return;
    }
    {
      std::lock_guard<std::mutex> g(mu_);
      if (idle_ + size <= kKeepIdle) {
        free_.emplace_back(p, size);
        idle_ += size;
        return;
      }
    }
    cudaFreeHost(p);
  }
  std::mutex mu_;
  std::vector<std::pair<uint8_t*, size_t>> free_;
  size_t idle_ = 0;
};

void put_u32(uint8_t* out, uint32_t v) {
  for (int i = 0; i < 4; ++i) out[i] = static_cast<uint8_t>(v >> (8 * i));
}

}  // namespace

// ---- SavedState (engine.rs:503-580) ----------------------------------------

size_t SavedState::byte_len() const {
  size_t n = prefix.size() * 4;
  for (const auto& l : layers) n += l.len;
  return n;
}

size_t SavedState::file_len(const std::string& model_id) const {
  return 6 + 4 + model_id.size() + body_len;
}

SavedState SavedState::make(const uint32_t* prefix, size_t n,
                            const std::vector<std::array<size_t, 3>>& layers) {
  SavedState s;
  s.prefix.assign(prefix, prefix + n);
  size_t len = 4 + 4 * n + 4;
  for (const auto& l : layers) len += 12 + l[2];
  s.body = HostBlocks::get().take(len);
  s.body_len = len;
  uint8_t* b = s.body.get();
  put_u32(b, static_cast<uint32_t>(n));
  for (size_t i = 0; i < n; ++i) put_u32(b + 4 + 4 * i, prefix[i]);
  size_t at = 4 + 4 * n;
  put_u32(b + at, static_cast<uint32_t>(layers.size()));
  at += 4;
  for (const auto& l : layers) {
    put_u32(b + at, static_cast<uint32_t>(l[0]));
    put_u32(b + at + 4, static_cast<uint32_t>(l[1]));
    put_u32(b + at + 8, static_cast<uint32_t>(l[2]));
    Layer ly;
    ly.layer = static_cast<int>(l[0]);
    ly.row0 = static_cast<int>(l[1]);
    ly.off = at + 12;
    ly.len = l[2];
    s.layers.push_back(ly);
    at += 12 + l[2];
  }
  return s;
}

void SavedState::write_bytes(const std::string& model_id, uint8_t* out) const {
  std::memcpy(out, "GRWS1\0", 6);
  put_u32(out + 6, static_cast<uint32_t>(model_id.size()));
  std::memcpy(out + 10, model_id.data(), model_id.size());
  if (body_len) std::memcpy(out + 10 + model_id.size(), body.get(), body_len);
}

std::vector<uint8_t> SavedState::to_bytes(const std::string& model_id) const {
  std::vector<uint8_t> out(file_len(model_id));
  write_bytes(model_id, out.data());
  return out;
}

SavedState SavedState::from_bytes(const uint8_t* b, size_t n, const std::string& model_id) {
  size_t at = 0;
  auto take = [&](size_t k) -> const uint8_t* {
    if (at + k > n || at + k < at) fail("state file truncated");
    const uint8_t* p = b + at;
    at += k;
    return p;
  };
  auto u32 = [&]() -> size_t {
    const uint8_t* p = take(4);
    return static_cast<size_t>(p[0]) | (static_cast<size_t>(p[1]) << 8) |
           (static_cast<size_t>(p[2]) << 16) | (static_cast<size_t>(p[3]) << 24);
  };
  const uint8_t* magic = take(6);
  if (std::memcmp(magic, "GRWS1\0", 6) != 0) fail("not a omg wgpu state file");
  const size_t idn = u32();
  const uint8_t* id = take(idn);
  if (idn != model_id.size() || std::memcmp(id, model_id.data(), idn) != 0)
    fail("state file is for a different model");
  const size_t body0 = at;
  const size_t np = u32();
  const uint8_t* pp = take(np * 4);
  std::vector<uint32_t> prefix(np);
  for (size_t i = 0; i < np; ++i)
    prefix[i] = static_cast<uint32_t>(pp[4 * i]) | (static_cast<uint32_t>(pp[4 * i + 1]) << 8) |
                (static_cast<uint32_t>(pp[4 * i + 2]) << 16) |
                (static_cast<uint32_t>(pp[4 * i + 3]) << 24);
  const size_t nl = u32();
  std::vector<std::array<size_t, 3>> specs;
  for (size_t i = 0; i < nl; ++i) {
    const size_t layer = u32(), row0 = u32(), len = u32();
    take(len);
    specs.push_back({layer, row0, len});
  }
  SavedState s = make(prefix.data(), np, specs);
  // The body as read: the same bytes make() laid out, rows included.
  std::memcpy(s.body.get(), b + body0, s.body_len);
  return s;
}

std::optional<SavedState> StateCache::get(const std::vector<uint32_t>& prefix) {
  for (size_t i = 0; i < entries.size(); ++i) {
    if (entries[i].prefix == prefix) {
      SavedState s = std::move(entries[i]);
      entries.erase(entries.begin() + static_cast<long>(i));
      entries.push_back(s);
      return s;
    }
  }
  return std::nullopt;
}

void StateCache::put(SavedState s) {
  const size_t len = s.byte_len();
  if (len > budget) return;
  for (size_t i = 0; i < entries.size(); ++i)
    if (entries[i].prefix == s.prefix) {
      used -= entries[i].byte_len();
      entries.erase(entries.begin() + static_cast<long>(i));
      break;
    }
  while (used + len > budget && !entries.empty()) {
    used -= entries.front().byte_len();
    entries.erase(entries.begin());
  }
  used += len;
  entries.push_back(std::move(s));
}

uint64_t state_key(const std::string& model_id, const uint32_t* prefix, size_t n) {
  uint64_t h = 0xcbf29ce484222325ull;
  auto eat = [&](uint8_t b) {
    h ^= b;
    h *= 0x00000100000001b3ull;
  };
  for (char c : model_id) eat(static_cast<uint8_t>(c));
  eat(0);
  for (size_t i = 0; i < n; ++i)
    for (int k = 0; k < 4; ++k) eat(static_cast<uint8_t>(prefix[i] >> (8 * k)));
  return h;
}

// ---- builder (engine.rs:845-952) --------------------------------------------

static std::string shape_str(const std::vector<int64_t>& s) {
  std::string o = "[";
  for (size_t i = 0; i < s.size(); ++i) o += (i ? ", " : "") + std::to_string(s[i]);
  return o + "]";
}

EngineBuilder::EngineBuilder(Config cfg, int device) : cfg_(std::move(cfg)), device_(device) {
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

EngineBuilder::~EngineBuilder() {
  if (stream_) cudaStreamDestroy(stream_);
}

std::vector<std::string> EngineBuilder::missing() const {
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

void EngineBuilder::push(const std::string& name, const HostTensor& t) {
  CUDA_TRY(cudaSetDevice(device_));
  auto it = expected_.find(name);
  if (it == expected_.end()) fail("unexpected tensor %s", name.c_str());
  if (t.shape != it->second)
    fail("%s: shape %s, expected %s", name.c_str(), shape_str(t.shape).c_str(),
         shape_str(it->second).c_str());
  const size_t n = t.numel();
  if (t.dtype < 0 || t.dtype > 2) fail("%s: unsupported dtype %d", name.c_str(), t.dtype);
  // QTensor::from_raw's payload checks (model.rs:484-505).
  if (t.data.size() != payload_bytes(t.dtype, n))
    fail("%s: %zu payload bytes, expected %zu", name.c_str(), t.data.size(),
         payload_bytes(t.dtype, n));
  const size_t want_scales = t.dtype == 0 ? 0 : n / 32 * 2;
  if (t.scales.size() != want_scales)
    fail("%s: %zu scale bytes, expected %zu", name.c_str(), t.scales.size(), want_scales);
  if (ends_with(name, "out_scale")) {
    scalars_[name] = t.get(0);
    pushed_[name] = true;
    return;
  }
  if (t.shape.size() == 1 && t.dtype != 0) fail("%s: 1-D tensors must be f16", name.c_str());
  if (t.shape.size() == 2 && t.shape[1] % 32 != 0)
    fail("%s: inner dimension %lld is not a multiple of 32", name.c_str(),
         static_cast<long long>(t.shape[1]));
  if (t.shape.size() == 1) {
    std::vector<float> f(n);
    dequantize(0, t.data.data(), nullptr, n, f.data());
    DevBuffer b;
    b.alloc(n * 4, false);
    CUDA_TRY(cudaMemcpy(b.p, f.data(), n * 4, cudaMemcpyHostToDevice));
    norms_[name] = std::move(b);
    pushed_[name] = true;
    return;
  }
  if (name == "embed") {
    embed_.dtype = t.dtype;
    embed_.codes.alloc(t.data.size(), false);
    CUDA_TRY(cudaMemcpy(embed_.codes.p, t.data.data(), t.data.size(), cudaMemcpyHostToDevice));
    embed_.scales.alloc(std::max<size_t>(t.scales.size(), 16), true);
    if (!t.scales.empty())
      CUDA_TRY(cudaMemcpy(embed_.scales.p, t.scales.data(), t.scales.size(),
                          cudaMemcpyHostToDevice));
    pushed_[name] = true;
    return;
  }
  // A linear. Q4_0 / Q8_0: kept packed in the GEMMs' chunk layout, decoded
  // per tile in shared memory (weight.wgsl decodes per use, too); f16: kept
  // as f16 rows.
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
  if (ends_with(name, ".gate") || ends_with(name, ".up")) {
    key = name.substr(0, name.rfind('.')) + ".gate_up";
    remap = ends_with(name, ".gate") ? 1 : 2;
    out_rows = static_cast<size_t>((rows + 127) / 128) * 256;
  }
  auto pit = pk_.find(key);
  if (t.dtype != 0 && (packed_ || pit != pk_.end()) && !lin_.count(key) &&
      (pit == pk_.end() || pit->second.dtype == t.dtype)) {
    if (pit == pk_.end()) {
      PackedLinear w;
      w.dtype = t.dtype;
      w.rows = static_cast<int>(out_rows);
      w.k = k;
      w.chunks.alloc(packed_bytes(t.dtype, w.rows, k), true);
      pit = pk_.emplace(key, std::move(w)).first;
    }
    launch_pack_weight(t.dtype, codes.p, scales.p, rows, k, remap, pit->second.rows,
                       pit->second.chunks.as<uint8_t>(), stream_);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaStreamSynchronize(stream_));
    pushed_[name] = true;
    return;
  }
  if (pit != pk_.end()) {
    // Gate and up of different dtypes: the pair is kept as f16 rows.
    DevBuffer b;
    b.alloc(out_rows * k * 2, true);
    launch_unpack_weight(pit->second.dtype, pit->second.chunks.as<uint8_t>(), pit->second.rows, k,
                         b.as<__half>(), stream_);
    CUDA_TRY(cudaGetLastError());
    lin_.emplace(key, std::move(b));
    pk_.erase(pit);
  }
  // f16 rows: bit-exact QTensor::get rounded to f16, what weight.wgsl's
  // dq*_pair decoders produce per use.
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

void EngineBuilder::set_per_layer_table(HostTensor t) {
  const std::vector<int64_t> want = {cfg_.vocab,
                                     static_cast<int64_t>(cfg_.per_layer_dim) * cfg_.layers};
  if (t.shape != want)
    fail("per-layer table: shape %s, expected %s", shape_str(t.shape).c_str(),
         shape_str(want).c_str());
  per_layer_table_ = std::move(t);
}

std::unique_ptr<Engine> EngineBuilder::finish(size_t capacity, size_t max_rows) {
  const auto miss = missing();
  if (!miss.empty()) {
    std::string e;
    for (size_t i = 0; i < std::min<size_t>(4, miss.size()); ++i) e += (i ? ", " : "") + miss[i];
    fail("%zu tensors missing, e.g. %s", miss.size(), e.c_str());
  }
  if (capacity == 0) fail("capacity must be positive");
  return std::unique_ptr<Engine>(new Engine(std::move(*this), capacity, max_rows));
}

// ---- engine ------------------------------------------------------------------

Engine::Engine(EngineBuilder&& b, size_t capacity_, size_t max_rows_)
    : config(b.cfg_), capacity(capacity_), max_rows(max_rows_), device_(b.device_) {
  CUDA_TRY(cudaSetDevice(device_));
  CUDA_TRY(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device_));
  stream_ = b.stream_;
  b.stream_ = nullptr;
  lin_ = std::move(b.lin_);
  pk_ = std::move(b.pk_);
  norms_ = std::move(b.norms_);
  embed_.dtype = b.embed_.dtype;
  embed_.codes = std::move(b.embed_.codes);
  embed_.scales = std::move(b.embed_.scales);
  per_layer_table_ = std::move(b.per_layer_table_);
  gemm_setup_device();
  attention_setup_device();
  logits_setup_device(config.d);

  const Config& c = config;
  const int d = c.d, L = c.layers, P = c.per_layer_dim;
  for (int l = 0; l < L; ++l) {
    max_qkv_ = std::max(max_qkv_, c.qkv_width(l));
    max_ff_ = std::max(max_ff_, c.ff[l]);
  }
  max_attn_ = c.heads * c.max_head_dim();
  // Cache rows rounded up to whole 64-key tiles: the attention kernel may
  // stage a tile that ends past the last used row.
  cap_rows_ = (capacity + 63) / 64 * 64;
  const size_t C = capacity;
  const size_t Cpad = cap_rows_;
  const int S = 4;  // split-K slabs the f32 GEMM outputs may use

  // Workspace. Zero-initialised, so rows a kernel reads but no pass has
  // written (padding, stale tile tails) are finite.
  ids_.alloc(Cpad * 4);
  meta_.alloc(Cpad * sizeof(TokMeta));
  row_map_.alloc(Cpad * 4);
  x_.alloc(Cpad * d * 4);
  h16_.alloc(Cpad * d * 2);
  qkv_.alloc(S * Cpad * max_qkv_ * 4);
  q16_.alloc(Cpad * max_attn_ * 2);
  attn16_.alloc(Cpad * max_attn_ * 2);
  a32_.alloc(S * Cpad * d * 4);
  act16_.alloc(Cpad * std::max(max_ff_, P) * 2);
  rows_.alloc(std::max<size_t>(max_rows, 1) * d * 4);
  logits_.alloc(std::max<size_t>(max_rows, 1) * c.vocab * 4);
  status_.alloc(16);
  if (P > 0) {
    x16_.alloc(Cpad * d * 2);
    pl_rows16_.alloc(Cpad * P * L * 2);
    pli_.alloc(Cpad * P * L * 4);
    plp_.alloc(Cpad * std::max(P * L, d) * 4);
  }
  kv_.resize(L);
  for (int l = 0; l < L; ++l)
    if (c.has_kv(l)) kv_[l].alloc(Cpad * 2 * c.kv_heads * c.head_dim[l] * 2);
  mlp_ready_.alloc((Cpad + 127) / 128 * S * sizeof(int));
  {
    char err[256];
    // q16 holds a layer's rows as [t][heads * head_dim]: one map per width.
    for (int hi = 0; hi < 2; ++hi)
      if (!attention_map_q(&attn_tq_[hi], q16_.p, static_cast<int>(Cpad), c.heads, c.kv_heads,
                           256 << hi, err, sizeof err))
        fail("%s", err);
    attn_tkv_.resize(L);
    for (int l = 0; l < L; ++l)
      if (c.has_kv(l) &&
          !attention_map_kv(&attn_tkv_[l], kv_[l].p, static_cast<int>(Cpad), c.kv_heads,
                            c.head_dim[l], err, sizeof err))
        fail("layer %d: %s", l, err);
  }
  h_ids_.alloc(Cpad * 4);
  h_meta_.alloc(Cpad * sizeof(TokMeta));
  h_row_map_.alloc(Cpad * 4);
  h_out_.alloc(std::max<size_t>(max_rows, 1) * std::max(c.vocab, d) * 4);
  h_status_.alloc(16);
  for (auto& e : events_) CUDA_TRY(cudaEventCreate(&e));

  auto norm = [&](const std::string& n) -> const float* { return norms_.at(n).as<float>(); };
  auto lin = [&](const std::string& n) { return weight(n); };
  final_norm_ = norm("final_norm");
  char err[512];
  auto plan = [&](GemmPlan* p, const void* a, int lda, const WeightRef& w, int w_rows, int n_out,
                  int k, int epi, const char* what, int l, int force_splits = 0) {
    int bn = 256, splits = 1;
    if (epi == kEpiF32) gemm_pick(n_out, k, num_sms_, &bn, &splits);
    if (force_splits > 0) {
      bn = 256;
      splits = force_splits;
    }
    if (w.pk != kF16) {
      // Packed Q4_0 / Q8_0 weights: decoded per tile in shared memory.
      if (!gemm_plan_packed(p, a, static_cast<int>(C), lda, w.p, w.pk, w_rows, n_out, k, epi, bn,
                            std::min(splits, S), err, sizeof err))
        fail("layer %d %s: %s", l, what, err);
      if (p->s.bn == 256 && !gemm_plan_pair(p, nullptr, w_rows, false, err, sizeof err))
        fail("layer %d %s: %s", l, what, err);
      return;
    }
    if (!gemm_plan(p, a, static_cast<int>(C), lda, w.p, w_rows, n_out, k, epi, bn,
                   std::min(splits, S), err, sizeof err))
      fail("layer %d %s: %s", l, what, err);
    // Passes of many rows (a long state's prefill) take the CTA-pair kernel.
    if (p->s.bn == 256 &&
        !gemm_plan_pair(p, w.p, w_rows, false, err, sizeof err))
      fail("layer %d %s: %s", l, what, err);
  };
  layers_.resize(L);
  for (int l = 0; l < L; ++l) {
    Layer& ly = layers_[l];
    auto n = [&](const char* s) { return "blk." + std::to_string(l) + "." + s; };
    ly.hd = c.head_dim[l];
    ly.ff = c.ff[l];
    ly.qkv_w = c.qkv_width(l);
    ly.sliding = c.sliding[l];
    ly.has_kv = c.has_kv(l);
    ly.kv_src = c.kv_source[l];
    ly.attn_norm = norm(n("attn_norm"));
    ly.q_norm = norm(n("q_norm"));
    ly.k_norm = ly.has_kv ? norm(n("k_norm")) : nullptr;
    ly.post_attn_norm = norm(n("post_attn_norm"));
    ly.ffn_norm = norm(n("ffn_norm"));
    ly.post_ffn_norm = norm(n("post_ffn_norm"));
    ly.next_norm = l + 1 == L ? final_norm_ : norm("blk." + std::to_string(l + 1) + ".attn_norm");
    auto sc = b.scalars_.find(n("out_scale"));
    ly.out_scale = sc == b.scalars_.end() ? 1.f : sc->second;
    const WeightRef w_qkv = lin(n("qkv")), w_o = lin(n("o")), w_gu = lin(n("gate_up")),
                    w_down = lin(n("down"));
    const int attn_w = c.heads * ly.hd;
    // 256-dim heads: q/k norm, RoPE and the K/V-cache write ride in the
    // projection's epilogue (one 256-column tile per head).
    plan(&ly.qkv, h16_.p, d, w_qkv, ly.qkv_w, ly.qkv_w, d,
         ly.hd == 256 ? kEpiQkPrep : kEpiF32, "qkv", l);
    plan(&ly.o, attn16_.p, attn_w, w_o, d, d, attn_w, kEpiF32, "o", l);
    plan(&ly.gate_up, h16_.p, d, w_gu, (ly.ff + 127) / 128 * 256, ly.ff, d, kEpiGeGluTanh,
         "gate_up", l);
    // The down projection joins gate_up's launch, split so that each split
    // reads whole gate_up column tiles: into units as long as a gate_up tile
    // where that divides (E2B, E4B), else into the most splits (up to S)
    // that do, for the shortest up -> down chain (a split count that
    // depends on the layer's shape only).
    const int kb_up = (d + 63) / 64, kb_dn = (ly.ff + 63) / 64;
    const int up_tiles = (ly.ff + 127) / 128;
    int fuse_splits = kb_dn % kb_up == 0 ? kb_dn / kb_up : 0;
    for (int sp = S; fuse_splits == 0 && sp >= 1; --sp)
      if (kb_dn % sp == 0 && (kb_dn / sp) % 2 == 0 && up_tiles == sp * (kb_dn / sp / 2))
        fuse_splits = sp;
    if (fuse_splits >= 1 && fuse_splits <= S) {
      plan(&ly.down, act16_.p, ly.ff, w_down, d, d, ly.ff, kEpiF32, "down", l, fuse_splits);
      ly.fused_mlp = gemm_mlp_ok(ly.gate_up, ly.down);
    }
    if (!ly.fused_mlp)
      plan(&ly.down, act16_.p, ly.ff, w_down, d, d, ly.ff, kEpiF32, "down", l);
    if (P > 0) {
      ly.pl_norm = norm(n("pl_norm"));
      plan(&ly.pl_gate, x16_.p, d, lin(n("pl_gate")), P, P, d, kEpiF32, "pl_gate", l);
      plan(&ly.pl_proj, act16_.p, P, lin(n("pl_proj")), d, d, P, kEpiF32, "pl_proj", l);
    }
  }
  if (P > 0) plan(&pl_model_proj_, x16_.p, d, lin("pl_model_proj"), P * L, P * L, d, kEpiF32,
                  "pl_model_proj", -1);
  // RoPE rotations of every cache position for the two thetas (the fused
  // QKV epilogue's table).
  for (int w = 0; w < 2; ++w) {
    rope_tab_[w].alloc(cap_rows_ * 128 * sizeof(float2), false);
    launch_rope_table(w == 0 ? c.theta_local : c.theta_global, 128, static_cast<int>(cap_rows_),
                      rope_tab_[w].as<float2>(), stream_);
  }
  CUDA_TRY(cudaGetLastError());
  CUDA_TRY(cudaStreamSynchronize(stream_));
}

Engine::~Engine() {
  cudaSetDevice(device_);
  if (stream_) cudaStreamSynchronize(stream_);
  for (auto& g : graphs_) cudaGraphExecDestroy(g.exec);
  for (auto e : prof_events_) cudaEventDestroy(e);
  for (auto& e : events_)
    if (e) cudaEventDestroy(e);
  if (stream_) cudaStreamDestroy(stream_);
}

std::optional<PrefixSource> Engine::prefix_source() const {
  std::lock_guard<std::mutex> g(mu_);
  return last_source_;
}

bool Engine::is_resident(const uint32_t* prefix, size_t n) const {
  std::lock_guard<std::mutex> g(mu_);
  return n > 0 && resident_ && resident_->size() == n &&
         std::equal(resident_->begin(), resident_->end(), prefix);
}

void Engine::evict_resident() {
  std::lock_guard<std::mutex> g(mu_);
  resident_.reset();
}

void Engine::set_state_cache(size_t bytes, const std::string& dir, const std::string& model_id) {
  std::lock_guard<std::mutex> g(mu_);
  states_ = StateCache{};
  states_.budget = bytes;
  state_dir_ = dir;
  model_id_ = model_id;
}

std::vector<uint8_t> Engine::gather_per_layer(const uint32_t* ids, size_t n) const {
  if (!per_layer_table_) fail("this model needs per-layer embedding rows; none loaded");
  const HostTensor& t = *per_layer_table_;
  const size_t width = static_cast<size_t>(t.shape[1]);
  std::vector<uint8_t> out(n * width * 2);
  std::vector<float> row(width);
  for (size_t i = 0; i < n; ++i) {
    const size_t r = ids[i];
    if (t.dtype == 0) {
      std::memcpy(out.data() + i * width * 2, t.data.data() + r * width * 2, width * 2);
      continue;
    }
    const size_t bpr = width / 32;
    dequantize(t.dtype, t.data.data() + r * bpr * (t.dtype == 1 ? 32 : 16),
               t.scales.data() + r * bpr * 2, width, row.data());
    for (size_t j = 0; j < width; ++j) {
      const uint16_t h = f32_to_f16(row[j]);
      out[i * width * 2 + 2 * j] = static_cast<uint8_t>(h & 0xff);
      out[i * width * 2 + 2 * j + 1] = static_cast<uint8_t>(h >> 8);
    }
  }
  return out;
}

Engine::WeightRef Engine::weight(const std::string& name) const {
  auto pit = pk_.find(name);
  if (pit != pk_.end()) return {pit->second.dtype, pit->second.chunks.p};
  auto it = lin_.find(name);
  if (it == lin_.end()) fail("no device weight %s", name.c_str());
  return {kF16, it->second.p};
}

std::vector<uint16_t> Engine::weight_f16(const std::string& name) const {
  CUDA_TRY(cudaSetDevice(device_));
  std::vector<int64_t> shape;
  for (const auto& t : config.tensors())
    if (t.name == name) shape = t.shape;
  if (shape.size() != 2 || name == "embed")
    fail("weight_f16: %s is not a projection weight", name.c_str());
  const size_t rows = static_cast<size_t>(shape[0]), k = static_cast<size_t>(shape[1]);
  std::vector<uint16_t> out(rows * k);
  const bool gate = ends_with(name, ".gate"), up = ends_with(name, ".up");
  const std::string key = gate || up ? name.substr(0, name.rfind('.')) + ".gate_up" : name;
  const size_t stored_rows = gate || up ? (rows + 127) / 128 * 256 : rows;
  std::vector<uint16_t> all(stored_rows * k);
  auto pit = pk_.find(key);
  if (pit != pk_.end()) {
    // Packed: decoded by the GEMMs' tile decoder (unpack_block).
    DevBuffer tmp;
    tmp.alloc(all.size() * 2, false);
    launch_unpack_weight(pit->second.dtype, pit->second.chunks.as<uint8_t>(),
                         static_cast<int>(stored_rows), static_cast<int>(k), tmp.as<__half>(),
                         stream_);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaStreamSynchronize(stream_));
    CUDA_TRY(cudaMemcpy(all.data(), tmp.p, all.size() * 2, cudaMemcpyDeviceToHost));
  } else {
    auto it = lin_.find(key);
    if (it == lin_.end()) fail("weight_f16: no device weight %s", key.c_str());
    CUDA_TRY(cudaMemcpy(all.data(), it->second.p, all.size() * 2, cudaMemcpyDeviceToHost));
  }
  if (!gate && !up) return all;
  // Gate and up rows interleave in 256-row blocks [128 gate | 128 up].
  for (size_t r = 0; r < rows; ++r) {
    const size_t src = (r / 128) * 256 + (up ? 128 : 0) + r % 128;
    std::memcpy(out.data() + r * k, all.data() + src * k, k * 2);
  }
  return out;
}

// engine.rs:1467-1477
std::pair<size_t, std::optional<PrefixSource>> Engine::admit(const GroupIn* groups, size_t n) {
  for (size_t i = 0; i < n; ++i)
    if (is_resident(groups[i].prefix, groups[i].n_prefix))
      return {i, PrefixSource::Resident};
  for (size_t i = 0; i < n; ++i) {
    auto src = restore_from_cache(groups[i].prefix, groups[i].n_prefix);
    if (src) return {i, src};
  }
  return {0, std::nullopt};
}

// engine.rs:1492-1583: layout order (first, then the rest), per-token
// metadata, wanted rows, and the request checks with the reference's
// messages.
Engine::Packing Engine::pack(const GroupIn* groups, size_t n, size_t first,
                             bool resident_first) const {
  Packing p;
  size_t total = 0;
  for (size_t i = 0; i < n; ++i) total += groups[i].tokens();
  if (total > capacity) fail("%zu tokens exceed the engine capacity %zu", total, capacity);
  if (total == 0) fail("empty request");
  const size_t p0 = groups[first].n_prefix;
  p.base = resident_first ? p0 : 0;
  p.t = total - p.base;
  p.ids.reserve(p.t);
  p.meta.reserve(p.t);
  // Flat output offsets: groups in call order, branches, want slots.
  std::vector<size_t> group_off(n + 1, 0);
  for (size_t i = 0; i < n; ++i) group_off[i + 1] = group_off[i] + groups[i].rows();
  std::vector<size_t> order;
  order.push_back(first);
  for (size_t i = 0; i < n; ++i)
    if (i != first) order.push_back(i);
  struct Want {
    size_t out_row, ws_row;
  };
  std::vector<Want> wanted;
  for (size_t k = 0; k < order.size(); ++k) {
    const size_t gi = order[k];
    const GroupIn& g = groups[gi];
    if (g.n_branches >= (1u << 12))
      fail("%zu branches in one group; the engine addresses at most %u", g.n_branches,
           (1u << 12) - 1);
    const int seq_hi = static_cast<int>(k) << 12;
    const size_t row_lo = k == 0 ? 0 : p.base + p.ids.size();
    if (!(k == 0 && p.base > 0)) {
      p.decoded.emplace_back(gi, p.base + p.ids.size());
      for (size_t i = 0; i < g.n_prefix; ++i) {
        const size_t row = p.base + p.ids.size();
        p.meta.push_back({static_cast<int>(i), seq_hi, static_cast<int>(row_lo),
                          static_cast<int>(row + 1)});
        p.ids.push_back(static_cast<int32_t>(g.prefix[i]));
      }
    }
    size_t out_row = group_off[gi];
    for (size_t bi = 0; bi < g.n_branches; ++bi) {
      const BranchIn& br = g.branches[bi];
      const size_t start = p.ids.size();
      for (size_t j = 0; j < br.n_tokens; ++j) {
        const size_t row = p.base + p.ids.size();
        p.meta.push_back({static_cast<int>(g.n_prefix + j), seq_hi | static_cast<int>(bi + 1),
                          static_cast<int>(row_lo), static_cast<int>(row + 1)});
        p.ids.push_back(br.tokens[j]);
      }
      for (size_t s = 0; s < br.n_want; ++s) {
        if (br.want[s] >= br.n_tokens)
          fail("branch %zu: wanted position %zu past its %zu tokens", bi, br.want[s],
               br.n_tokens);
        wanted.push_back({out_row++, start + br.want[s]});
      }
    }
  }
  if (wanted.size() > max_rows)
    fail("%zu rows requested, engine reads back at most %zu", wanted.size(), max_rows);
  for (int32_t id : p.ids)
    if (id < 0 || id >= config.vocab)
      fail("token id %u outside the vocabulary of %d", static_cast<uint32_t>(id), config.vocab);
  // Several wanted slots may name the same token; the device writes each
  // token's row once (to its first slot) and the host copies duplicates.
  p.row_map.assign(p.t, -1);
  p.out_index.resize(wanted.size());
  p.nwanted = 0;
  std::vector<int32_t> dev_row_of_ws(p.t, -1);
  for (size_t w = 0; w < wanted.size(); ++w) {
    const size_t ws = wanted[w].ws_row;
    if (dev_row_of_ws[ws] < 0) {
      dev_row_of_ws[ws] = static_cast<int32_t>(p.nwanted++);
      p.row_map[ws] = dev_row_of_ws[ws];
    }
    // out_index[device row order] is filled below
  }
  {
    const int t = static_cast<int>(p.t), base = static_cast<int>(p.base);
    const int hpg = config.heads / config.kv_heads;
    attention_intervals(p.meta.data(), t, base, &p.attn_vis);
    p.attn_slots = 0;
    for (int w = 0; w < 2; ++w)
      p.attn_slots = std::max(
          p.attn_slots, attention_flash_runs(p.meta.data(), p.attn_vis.data(), t, hpg,
                                             w == 0 ? config.window : 0, &p.attn_runs[w],
                                             &p.attn_tiles[w], &p.attn_items[w], &p.attn_merges[w]));
    size_t off = 0;
    auto put = [&](int i, size_t bytes) {
      p.attn_off[i] = off;
      off += (bytes + 255) / 256 * 256;
    };
    put(0, p.attn_vis.size() * sizeof(int4));
    for (int w = 0; w < 2; ++w) {
      put(attn_sched_part(w, 0), p.attn_runs[w].size() * sizeof(AttnFlashRun));
      put(attn_sched_part(w, 1), p.attn_tiles[w].size() * sizeof(int));
      put(attn_sched_part(w, 2), p.attn_items[w].size() * sizeof(AttnFlashItem));
      put(attn_sched_part(w, 3), p.attn_merges[w].size() * sizeof(AttnFlashMerge));
    }
    p.attn_bytes = off;
  }
  // out_index[w] = device row of wanted slot w, paired with its flat out row.
  p.out_index.clear();
  for (const auto& w : wanted) {
    p.out_index.push_back(static_cast<size_t>(dev_row_of_ws[w.ws_row]));
    p.out_index.push_back(w.out_row);
  }
  return p;
}

void Engine::upload(const Packing& p, const uint8_t* per_layer_rows, size_t rows_bytes) {
  std::memcpy(h_ids_.p, p.ids.data(), p.t * 4);
  std::memcpy(h_meta_.p, p.meta.data(), p.t * sizeof(TokMeta));
  std::memcpy(h_row_map_.p, p.row_map.data(), p.t * 4);
  CUDA_TRY(cudaMemcpyAsync(ids_.p, h_ids_.p, p.t * 4, cudaMemcpyHostToDevice, stream_));
  CUDA_TRY(cudaMemcpyAsync(meta_.as<TokMeta>() + p.base, h_meta_.p, p.t * sizeof(TokMeta),
                           cudaMemcpyHostToDevice, stream_));
  CUDA_TRY(cudaMemcpyAsync(row_map_.p, h_row_map_.p, p.t * 4, cudaMemcpyHostToDevice, stream_));
  // Tensor-core attention schedule: one staged block, grown to the largest
  // pass seen.
  if (h_attn_sched_.bytes < p.attn_bytes || attn_sched_.bytes < p.attn_bytes) {
    CUDA_TRY(cudaStreamSynchronize(stream_));
    const size_t cap = std::max<size_t>(p.attn_bytes * 2, 1 << 16);
    h_attn_sched_.alloc(cap);
    attn_sched_.alloc(cap, false);
  }
  {
    uint8_t* h = h_attn_sched_.as<uint8_t>();
    std::memcpy(h + p.attn_off[0], p.attn_vis.data(), p.attn_vis.size() * sizeof(int4));
    for (int w = 0; w < 2; ++w) {
      std::memcpy(h + p.attn_off[attn_sched_part(w, 0)], p.attn_runs[w].data(),
                  p.attn_runs[w].size() * sizeof(AttnFlashRun));
      std::memcpy(h + p.attn_off[attn_sched_part(w, 1)], p.attn_tiles[w].data(),
                  p.attn_tiles[w].size() * sizeof(int));
      std::memcpy(h + p.attn_off[attn_sched_part(w, 2)], p.attn_items[w].data(),
                  p.attn_items[w].size() * sizeof(AttnFlashItem));
      std::memcpy(h + p.attn_off[attn_sched_part(w, 3)], p.attn_merges[w].data(),
                  p.attn_merges[w].size() * sizeof(AttnFlashMerge));
    }
    CUDA_TRY(cudaMemcpyAsync(attn_sched_.p, h, p.attn_bytes, cudaMemcpyHostToDevice, stream_));
  }
  // Partials of the chunk-split attention, grown to the largest pass seen
  // (a new buffer is a new graph key, so no cached graph keeps the old one).
  {
    const size_t rows = static_cast<size_t>(p.attn_slots) * config.kv_heads * kAttnTileRows;
    if (attn_part_ml_.bytes < rows * sizeof(float2)) {
      CUDA_TRY(cudaStreamSynchronize(stream_));
      const size_t cap = std::max<size_t>(rows * 2, 8 * kAttnTileRows);
      int hd_max = 256;
      for (int hd : config.head_dim) hd_max = std::max(hd_max, hd);
      attn_part_o_.alloc(cap * hd_max * sizeof(float), false);
      attn_part_ml_.alloc(cap * sizeof(float2), false);
    }
  }
  const int P = config.per_layer_dim;
  if (P > 0) {
    if (!per_layer_rows) fail("per-layer embedding rows required");
    const size_t row_bytes = static_cast<size_t>(P) * config.layers * 2;
    const size_t total = p.base + p.t;
    const uint8_t* src = per_layer_rows;
    if (rows_bytes == total * row_bytes)
      src = per_layer_rows + p.base * row_bytes;
    else if (rows_bytes != p.t * row_bytes)
      fail("per-layer rows: %zu bytes, expected %zu (or %zu with the prefix)", rows_bytes,
           p.t * row_bytes, total * row_bytes);
    CUDA_TRY(cudaMemcpyAsync(pl_rows16_.p, src, p.t * row_bytes, cudaMemcpyHostToDevice, stream_));
  }
}

// The whole network for one pass, launched on the engine's stream
// (engine.rs:1610-1759 records the same plan). Returns the number of kernel
// launches.
int Engine::launch_forward(const Packing& p, Want want) {
  const Config& c = config;
  const int t = static_cast<int>(p.t);
  const int d = c.d, L = c.layers, P = c.per_layer_dim;
  const size_t slab_a = cap_rows_ * d;
  const size_t slab_qkv = cap_rows_ * max_qkv_;
  uint32_t* status = status_.as<uint32_t>();
  int launches = 0;
  // `k(name)` names the launch that follows (profiling) and counts it.
  auto k = [&](const char* name) {
    ++launches;
    if (profiling_) prof_mark(name);
  };
  CUDA_TRY(cudaMemsetAsync(status, 0, 4, stream_));
  // Fused FFN launches count finished up tiles per row tile, cumulatively over
  // the pass (each launch waits for its own running total).
  CUDA_TRY(cudaMemsetAsync(mlp_ready_.p, 0, mlp_ready_.bytes, stream_));
  int mlp_target = 0;

  k("embed_norm");
  launch_embed_norm(embed_.dtype, ids_.as<int>(), t, embed_.codes.p, embed_.scales.p, d,
                    std::sqrt(static_cast<float>(d)), layers_[0].attn_norm, c.eps, c.norm_offset,
                    x_.as<float>(), P > 0 ? x16_.as<__half>() : nullptr, h16_.as<__half>(), d,
                    stream_);
  if (P > 0) {
    k("gemm_pl_model_proj");
    gemm_run(pl_model_proj_, t, plp_.p, P * L, 0, status, stream_);
    k("pl_combine");
    launch_pl_combine(plp_.as<float>(), t, P, L, norms_.at("pl_proj_norm").as<float>(),
                      pl_rows16_.as<__half>(), c.eps, c.norm_offset,
                      1.0f / std::sqrt(static_cast<float>(d)), std::sqrt(static_cast<float>(P)),
                      1.0f / std::sqrt(2.0f), pli_.as<float>(), stream_);
  }
  for (int li = 0; li < L; ++li) {
    const Layer& ly = layers_[li];
    const bool last = li + 1 == L;
    if (ly.qkv.s.epi == kEpiQkPrep) {
      // QKV projection with q/k norm + RoPE, K/V into the cache, in one launch.
      GemmEpi e{};
      QkEpi& q = e.qk;
      q.q16 = q16_.as<__half>();
      q.kv = ly.has_kv ? kv_[li].as<__half>() : nullptr;
      q.meta = meta_.as<TokMeta>();
      q.qn = ly.q_norm;
      q.kn = ly.k_norm;
      q.rope = rope_tab_[ly.sliding ? 0 : 1].as<float2>();
      q.rope_stride = static_cast<int>(cap_rows_);
      q.base = static_cast<int>(p.base);
      q.heads = c.heads;
      q.kv_heads = c.kv_heads;
      q.rope_dims = c.rope_dims[li];
      q.v_norm = c.v_norm;
      q.has_kv = ly.has_kv;
      q.q_scale = c.query_scale;
      q.eps = c.eps;
      q.offset = c.norm_offset;
      k("gemm_qkv");
      gemm_run_epi(ly.qkv, t, nullptr, 0, e, status, stream_);
    } else {
      // Other head sizes: the projection's f32 output, then qk_prep.
      k("gemm_qkv");
      gemm_run(ly.qkv, t, qkv_.p, ly.qkv_w, slab_qkv, status, stream_);
      // q/k norm + RoPE, K/V into the cache.
      QkArgs qa{};
      qa.qkv = qkv_.as<float>();
      qa.q_stride = ly.qkv_w;
      qa.splits = ly.qkv.s.splits;
      qa.split_stride = slab_qkv;
      qa.t = t;
      qa.heads = c.heads;
      qa.kv_heads = c.kv_heads;
      qa.hd = ly.hd;
      qa.has_kv = ly.has_kv;
      qa.v_norm = c.v_norm;
      qa.rope_dims = c.rope_dims[li];
      qa.theta = ly.sliding ? c.theta_local : c.theta_global;
      qa.q_scale = c.query_scale;
      qa.eps = c.eps;
      qa.offset = c.norm_offset;
      qa.qn = ly.q_norm;
      qa.kn = ly.k_norm;
      qa.meta = meta_.as<TokMeta>();
      qa.base = static_cast<int>(p.base);
      qa.q16 = q16_.as<__half>();
      qa.kv = ly.has_kv ? kv_[li].as<__half>() : nullptr;
      k("qk_prep");
      launch_qk_prep(qa, stream_);
    }
    // Block-causal attention over the cache (head_dim 256 or 512).
    {
      const int w = ly.sliding ? 0 : 1;
      const uint8_t* sched = attn_sched_.as<uint8_t>();
      AttnFlashArgs ta{};
      ta.vis = reinterpret_cast<const int4*>(sched + p.attn_off[0]);
      ta.meta = meta_.as<TokMeta>();
      ta.runs = reinterpret_cast<const AttnFlashRun*>(sched + p.attn_off[attn_sched_part(w, 0)]);
      ta.tiles = reinterpret_cast<const int*>(sched + p.attn_off[attn_sched_part(w, 1)]);
      ta.n_runs = static_cast<int>(p.attn_runs[w].size());
      ta.items = reinterpret_cast<const AttnFlashItem*>(sched + p.attn_off[attn_sched_part(w, 2)]);
      ta.n_items = static_cast<int>(p.attn_items[w].size());
      ta.merges = reinterpret_cast<const AttnFlashMerge*>(sched + p.attn_off[attn_sched_part(w, 3)]);
      ta.n_merges = static_cast<int>(p.attn_merges[w].size());
      ta.part_o = attn_part_o_.as<float>();
      ta.part_ml = attn_part_ml_.as<float2>();
      ta.out = attn16_.as<__half>();
      ta.status = status;
      ta.t = t;
      ta.base = static_cast<int>(p.base);
      ta.heads = c.heads;
      ta.kv_heads = c.kv_heads;
      ta.hpg = c.heads / c.kv_heads;
      ta.window = ly.sliding ? c.window : 0;
      ta.hd = ly.hd;
      k("attention");
      launch_attention_flash(attn_tq_[ly.hd == 512 ? 1 : 0], attn_tkv_[ly.kv_src], ta, kAttnPLo,
                             stream_);
      if (ta.n_merges > 0) {
        k("attention_merge");
        launch_attention_merge(ta, stream_);
      }
    }
    // Output projection, then x += norm(a); h = ffn_norm(x).
    k("gemm_o");
    gemm_run(ly.o, t, a32_.p, d, slab_a, status, stream_);
    k("residual_norm");
    launch_residual_norm(a32_.as<float>(), ly.o.s.splits, slab_a, d, t, d, ly.post_attn_norm,
                         c.eps, c.norm_offset, 1.0f, x_.as<float>(), nullptr, ly.ffn_norm,
                         h16_.as<__half>(), d, nullptr, nullptr, stream_);
    // GeGLU and down projection.
    // The fused FFN launch (on CTA pairs for passes of kPairMlpMinTiles row
    // tiles or more).
    if (ly.fused_mlp) {
      k("gemm_mlp");
      mlp_target += 4 * ly.gate_up.s.n_tiles / ly.down.s.splits;
      // arm_wait_timeout: one band more than the up tiles deliver, a short limit.
      const long long stall = stall_clocks_;
      stall_clocks_ = 0;
      gemm_run_mlp(ly.gate_up, ly.down, t, act16_.p, ly.ff, a32_.p, d, slab_a,
                   mlp_ready_.as<int>(), mlp_target + (stall ? 1 : 0), status, stream_, -1,
                   stall);
    } else {
      k("gemm_gate_up");
      gemm_run(ly.gate_up, t, act16_.p, ly.ff, 0, status, stream_);
      k("gemm_down");
      gemm_run(ly.down, t, a32_.p, d, slab_a, status, stream_);
    }
    const int* rmap = last ? row_map_.as<int>() : nullptr;
    float* rows = last ? rows_.as<float>() : nullptr;
    __half* hnext = last ? nullptr : h16_.as<__half>();
    if (P == 0) {
      k("residual_norm");
      launch_residual_norm(a32_.as<float>(), ly.down.s.splits, slab_a, d, t, d, ly.post_ffn_norm,
                           c.eps, c.norm_offset, ly.out_scale, x_.as<float>(), nullptr,
                           ly.next_norm, hnext, d, rmap, rows, stream_);
    } else {
      // Per-layer input chain (engine.rs:1733-1749).
      k("residual_norm");
      launch_residual_norm(a32_.as<float>(), ly.down.s.splits, slab_a, d, t, d, ly.post_ffn_norm,
                           c.eps, c.norm_offset, 1.0f, x_.as<float>(), x16_.as<__half>(),
                           nullptr, nullptr, d, nullptr, nullptr, stream_);
      k("gemm_pl_gate");
      gemm_run(ly.pl_gate, t, plp_.p, P, 0, status, stream_);
      k("pl_gate");
      launch_pl_gate(plp_.as<float>(), pli_.as<float>(), t, P, L, li, act16_.as<__half>(),
                     stream_);
      k("gemm_pl_proj");
      gemm_run(ly.pl_proj, t, a32_.p, d, slab_a, status, stream_);
      k("residual_norm");
      launch_residual_norm(a32_.as<float>(), ly.pl_proj.s.splits, slab_a, d, t, d, ly.pl_norm,
                           c.eps, c.norm_offset, ly.out_scale, x_.as<float>(), nullptr,
                           ly.next_norm, hnext, d, rmap, rows, stream_);
    }
  }
  if (want == Want::Logits) {
    k("logits");
    launch_logits(embed_.dtype, rows_.as<float>(), static_cast<int>(p.nwanted), embed_.codes.p,
                  embed_.scales.p, c.vocab, d, c.softcap, logits_.as<float>(), num_sms_, status,
                  stream_);
  }
  if (profiling_) prof_mark(nullptr);
  CUDA_TRY(cudaGetLastError());
  return launches;
}

bool Engine::GraphKey::operator==(const GraphKey& o) const {
  return t == o.t && base == o.base && nwanted == o.nwanted &&
         sched_bytes == o.sched_bytes && want == o.want && sched == o.sched &&
         std::equal(attn_off, attn_off + kAttnSchedParts, o.attn_off) && runs[0] == o.runs[0] &&
         runs[1] == o.runs[1] && tiles[0] == o.tiles[0] && tiles[1] == o.tiles[1] &&
         items[0] == o.items[0] && items[1] == o.items[1] && merges[0] == o.merges[0] &&
         merges[1] == o.merges[1] && part == o.part;
}

Engine::GraphKey Engine::graph_key(const Packing& p, Want want) const {
  GraphKey k;
  k.t = p.t;
  k.base = p.base;
  k.nwanted = p.nwanted;
  k.sched_bytes = p.attn_bytes;
  std::copy(p.attn_off, p.attn_off + kAttnSchedParts, k.attn_off);
  for (int w = 0; w < 2; ++w) {
    k.runs[w] = p.attn_runs[w].size();
    k.tiles[w] = p.attn_tiles[w].size();
    k.items[w] = p.attn_items[w].size();
    k.merges[w] = p.attn_merges[w].size();
  }
  k.part = attn_part_o_.p;
  k.want = static_cast<int>(want);
  k.sched = attn_sched_.p;
  return k;
}

int Engine::run_forward(const Packing& p, Want want) {
  const GraphKey key = graph_key(p, want);
  ++graph_clock_;
  for (auto& g : graphs_)
    if (g.key == key) {
      g.used = graph_clock_;
      CUDA_TRY(cudaGraphLaunch(g.exec, stream_));
      return g.launches;
    }
  cudaGraph_t graph = nullptr;
  CUDA_TRY(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
  int launches = 0;
  try {
    launches = launch_forward(p, want);
  } catch (...) {
    cudaStreamEndCapture(stream_, &graph);
    if (graph) cudaGraphDestroy(graph);
    throw;
  }
  CUDA_TRY(cudaStreamEndCapture(stream_, &graph));
  CachedGraph g;
  g.key = key;
  g.launches = launches;
  g.used = graph_clock_;
  const cudaError_t e = cudaGraphInstantiate(&g.exec, graph, 0);
  cudaGraphDestroy(graph);
  CUDA_TRY(e);
  if (graphs_.size() >= kMaxGraphs) {
    auto lru = std::min_element(graphs_.begin(), graphs_.end(),
                                [](const CachedGraph& a, const CachedGraph& b) { return a.used < b.used; });
    cudaGraphExecDestroy(lru->exec);
    graphs_.erase(lru);
  }
  graphs_.push_back(g);
  CUDA_TRY(cudaGraphLaunch(g.exec, stream_));
  return launches;
}

void Engine::prof_mark(const char* name) {
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

std::string Engine::profile_forward(const GroupIn* groups, size_t n, Want want, bool resident,
                                    int iters) {
  CUDA_TRY(cudaSetDevice(device_));
  if (resident && !is_resident(groups[0].prefix, groups[0].n_prefix))
    fail("profile_forward: the first group's prefix is not resident");
  Packing p = pack(groups, n, 0, resident);
  std::vector<uint8_t> rows;
  if (config.per_layer_dim > 0)
    rows = gather_per_layer(reinterpret_cast<const uint32_t*>(p.ids.data()), p.ids.size());
  upload(p, rows.empty() ? nullptr : rows.data(), rows.size());
  profiling_ = true;
  prof_used_ = 0;
  // The profiled passes are the range an external profiler run with
  // --profile-from-start off captures.
  CUDA_TRY(cudaProfilerStart());
  for (int i = 0; i < iters; ++i) launch_forward(p, want);
  CUDA_TRY(cudaProfilerStop());
  profiling_ = false;
  CUDA_TRY(cudaMemcpyAsync(h_status_.p, status_.p, 4, cudaMemcpyDeviceToHost, stream_));
  CUDA_TRY(cudaStreamSynchronize(stream_));
  check_status();
  // name -> (launches, total ms), in first-seen order.
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
  std::string js = "{";
  for (size_t i = 0; i < acc.size(); ++i) {
    char buf[160];
    snprintf(buf, sizeof buf, "%s\"%s\": [%d, %.6f]", i ? ", " : "", acc[i].first.c_str(),
             acc[i].second.first, acc[i].second.second);
    js += buf;
  }
  js += "}";
  if (!resident) {
    std::lock_guard<std::mutex> g(mu_);
    resident_ = std::vector<uint32_t>(groups[0].prefix, groups[0].prefix + groups[0].n_prefix);
  }
  return js;
}

void Engine::arm_wait_timeout(long long clocks) {
  if (clocks <= 0) fail("arm_wait_timeout: the limit must be positive");
  bool fused = false;
  for (const auto& ly : layers_) fused = fused || ly.fused_mlp;
  if (!fused) fail("arm_wait_timeout: this engine has no fused FFN launch");
  stall_clocks_ = clocks;
}

void Engine::check_status() {
  const uint32_t st = *h_status_.as<uint32_t>();
  if (st != 0)
    fail("a kernel gave up waiting (device status %u); the pass was abandoned", st);
}

void Engine::run(const GroupIn* groups, size_t n, size_t first,
                 std::optional<PrefixSource> source, Want want, const uint8_t* per_layer_rows,
                 size_t rows_bytes, float* out, size_t out_floats, int32_t* sources) {
  CUDA_TRY(cudaSetDevice(device_));
  Packing p = pack(groups, n, first, source.has_value());
  const size_t width = want == Want::Hidden ? config.d : config.vocab;
  size_t total_rows = 0;
  for (size_t i = 0; i < n; ++i) total_rows += groups[i].rows();
  if (out_floats < total_rows * width)
    fail("output buffer holds %zu floats, the request returns %zu", out_floats,
         total_rows * width);
  upload(p, per_layer_rows, rows_bytes);
  if (stall_clocks_)
    launch_forward(p, want);  // a test pass that must fail: never captured
  else
    run_forward(p, want);
  const float* src = want == Want::Logits ? logits_.as<float>() : rows_.as<float>();
  // A page-locked output buffer (omg_host_alloc) takes the rows straight from
  // the device, one copy per run of consecutive rows; any other buffer gets
  // them through the engine's own page-locked staging buffer.
  cudaPointerAttributes attr{};
  const bool pinned = out && cudaPointerGetAttributes(&attr, out) == cudaSuccess &&
                      attr.type == cudaMemoryTypeHost;
  if (!pinned) (void)cudaGetLastError();
  if (pinned) {
    for (size_t i = 0; i + 1 < p.out_index.size();) {
      const size_t s0 = p.out_index[i], d0 = p.out_index[i + 1];
      size_t run = 1;
      while (i + 2 * run + 1 < p.out_index.size() && p.out_index[i + 2 * run] == s0 + run &&
             p.out_index[i + 2 * run + 1] == d0 + run)
        ++run;
      CUDA_TRY(cudaMemcpyAsync(out + d0 * width, src + s0 * width, run * width * 4,
                               cudaMemcpyDeviceToHost, stream_));
      i += 2 * run;
    }
  } else if (p.nwanted) {
    CUDA_TRY(cudaMemcpyAsync(h_out_.p, src, p.nwanted * width * 4, cudaMemcpyDeviceToHost,
                             stream_));
  }
  CUDA_TRY(cudaMemcpyAsync(h_status_.p, status_.p, 4, cudaMemcpyDeviceToHost, stream_));
  CUDA_TRY(cudaStreamSynchronize(stream_));
  check_status();
  if (!pinned) {
    const float* h = h_out_.as<float>();
    for (size_t i = 0; i + 1 < p.out_index.size(); i += 2)
      std::memcpy(out + p.out_index[i + 1] * width, h + p.out_index[i] * width, width * 4);
  }
  {
    std::lock_guard<std::mutex> g(mu_);
    resident_ = std::vector<uint32_t>(groups[first].prefix,
                                      groups[first].prefix + groups[first].n_prefix);
  }
  for (const auto& dec : p.decoded)
    remember(groups[dec.first].prefix, groups[dec.first].n_prefix, dec.second);
  if (sources) {
    for (size_t i = 0; i < n; ++i) sources[i] = static_cast<int32_t>(PrefixSource::Decoded);
    sources[first] = static_cast<int32_t>(source.value_or(PrefixSource::Decoded));
  }
  std::lock_guard<std::mutex> g(mu_);
  last_source_ = source.value_or(PrefixSource::Decoded);
}

void Engine::evaluate_groups(const GroupIn* groups, size_t n, Want want, float* out,
                             size_t out_floats, int32_t* sources) {
  if (n == 0) fail("empty request");
  auto [first, source] = admit(groups, n);
  std::vector<uint8_t> rows;
  if (config.per_layer_dim > 0) {
    std::vector<uint32_t> ids;
    std::vector<size_t> order{first};
    for (size_t i = 0; i < n; ++i)
      if (i != first) order.push_back(i);
    for (size_t gi : order) {
      const GroupIn& g = groups[gi];
      if (!(gi == first && source)) ids.insert(ids.end(), g.prefix, g.prefix + g.n_prefix);
      for (size_t b = 0; b < g.n_branches; ++b)
        for (size_t j = 0; j < g.branches[b].n_tokens; ++j)
          ids.push_back(static_cast<uint32_t>(g.branches[b].tokens[j]));
    }
    for (uint32_t id : ids)
      if (id >= static_cast<uint32_t>(config.vocab))
        fail("token id %u outside the vocabulary of %d", id, config.vocab);
    rows = gather_per_layer(ids.data(), ids.size());
  }
  run(groups, n, first, source, want, rows.empty() ? nullptr : rows.data(), rows.size(), out,
      out_floats, sources);
}

void Engine::evaluate_rows(const GroupIn& g, Want want, const uint8_t* per_layer_rows,
                           size_t rows_bytes, float* out, size_t out_floats) {
  auto [first, source] = admit(&g, 1);
  run(&g, 1, first, source, want, per_layer_rows, rows_bytes, out, out_floats, nullptr);
}

// engine.rs:1341-1352: a two-token request so the first real one does not
// pay for first-touch costs.
void Engine::warmup() {
  const int32_t tok = 0;
  const size_t want0 = 0;
  BranchIn b{&tok, 1, &want0, 1};
  const uint32_t bos = config.bos;
  GroupIn g{&bos, 1, &b, 1};
  std::vector<float> out(config.vocab);
  std::vector<uint8_t> rows;
  if (config.per_layer_dim > 0)
    rows.assign(2 * static_cast<size_t>(config.per_layer_dim) * config.layers * 2, 0);
  evaluate_rows(g, Want::Logits, rows.empty() ? nullptr : rows.data(), rows.size(), out.data(),
                out.size());
}

std::pair<size_t, size_t> Engine::state_rows(int l, size_t p) const {
  if (config.sliding[l] && config.window > 0)
    return {p > static_cast<size_t>(config.window) ? p - config.window : 0, p};
  return {0, p};
}

SavedState Engine::save_state(const uint32_t* prefix, size_t n) {
  return save_state_at(prefix, n, 0);
}

SavedState Engine::save_state_at(const uint32_t* prefix, size_t n, size_t row0) {
  CUDA_TRY(cudaSetDevice(device_));
  std::vector<std::array<size_t, 3>> specs;
  for (int l = 0; l < config.layers; ++l) {
    if (!config.has_kv(l)) continue;
    auto [r0, r1] = state_rows(l, n);
    const size_t row_bytes = static_cast<size_t>(2) * config.kv_heads * config.head_dim[l] * 2;
    specs.push_back({static_cast<size_t>(l), r0, (r1 - r0) * row_bytes});
  }
  // One device-to-host copy per layer, straight into the page-locked file body.
  SavedState s = SavedState::make(prefix, n, specs);
  for (const auto& ly : s.layers) {
    const size_t row_bytes =
        static_cast<size_t>(2) * config.kv_heads * config.head_dim[ly.layer] * 2;
    if (ly.len)
      CUDA_TRY(cudaMemcpyAsync(s.data(ly), kv_[ly.layer].as<uint8_t>() + (row0 + ly.row0) * row_bytes,
                               ly.len, cudaMemcpyDeviceToHost, stream_));
  }
  CUDA_TRY(cudaStreamSynchronize(stream_));
  return s;
}

void Engine::restore_state(const SavedState& s) {
  CUDA_TRY(cudaSetDevice(device_));
  const size_t p = s.prefix.size();
  if (p > capacity) fail("state of %zu tokens exceeds the engine capacity %zu", p, capacity);
  for (const auto& ly : s.layers) {
    if (ly.layer < 0 || ly.layer >= config.layers || !config.has_kv(ly.layer))
      fail("state has K/V for layer %d, which owns none", ly.layer);
    const size_t row = static_cast<size_t>(2) * config.kv_heads * config.head_dim[ly.layer];
    auto [r0, r1] = state_rows(ly.layer, p);
    if (static_cast<size_t>(ly.row0) != r0 || ly.len != (r1 - r0) * row * 2)
      fail("state layer %d: %zu bytes at row %d, expected %zu at %zu", ly.layer, ly.len,
           ly.row0, (r1 - r0) * row * 2, r0);
  }
  for (const auto& ly : s.layers) {
    const size_t row_bytes = static_cast<size_t>(2) * config.kv_heads * config.head_dim[ly.layer] * 2;
    if (ly.len)
      CUDA_TRY(cudaMemcpyAsync(kv_[ly.layer].as<uint8_t>() + ly.row0 * row_bytes, s.data(ly),
                               ly.len, cudaMemcpyHostToDevice, stream_));
  }
  std::vector<TokMeta> meta(p);
  for (size_t i = 0; i < p; ++i)
    meta[i] = {static_cast<int>(i), 0, 0, static_cast<int>(i + 1)};
  if (p)
    CUDA_TRY(cudaMemcpyAsync(meta_.p, meta.data(), p * sizeof(TokMeta), cudaMemcpyHostToDevice,
                             stream_));
  CUDA_TRY(cudaStreamSynchronize(stream_));
  std::lock_guard<std::mutex> g(mu_);
  resident_ = s.prefix;
}

size_t Engine::state_image_bytes(size_t n) const {
  size_t total = 0;
  for (int l = 0; l < config.layers; ++l) {
    if (!config.has_kv(l)) continue;
    auto [r0, r1] = state_rows(l, n);
    total += (r1 - r0) * static_cast<size_t>(2) * config.kv_heads * config.head_dim[l] * 2;
  }
  return total;
}

namespace {
// `p` must be device memory of GPU `device` (a collective writes or reads it there).
void check_device_ptr(const void* p, int device, const char* what) {
  cudaPointerAttributes a{};
  if (!p || cudaPointerGetAttributes(&a, p) != cudaSuccess ||
      (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) || a.device != device) {
    cudaGetLastError();
    fail("%s is not device memory of GPU %d", what, device);
  }
}
}  // namespace

void Engine::export_state_device(const uint32_t* prefix, size_t n, void* dst, size_t cap) {
  CUDA_TRY(cudaSetDevice(device_));
  if (!is_resident(prefix, n)) fail("export_state_device: the prefix is not resident");
  const size_t need = state_image_bytes(n);
  if (cap < need) fail("export_state_device: buffer holds %zu bytes, need %zu", cap, need);
  check_device_ptr(dst, device_, "export_state_device: dst");
  size_t off = 0;
  for (int l = 0; l < config.layers; ++l) {
    if (!config.has_kv(l)) continue;
    auto [r0, r1] = state_rows(l, n);
    const size_t row_bytes = static_cast<size_t>(2) * config.kv_heads * config.head_dim[l] * 2;
    const size_t bytes = (r1 - r0) * row_bytes;
    if (bytes)
      CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(dst) + off, kv_[l].as<uint8_t>() + r0 * row_bytes,
                               bytes, cudaMemcpyDeviceToDevice, stream_));
    off += bytes;
  }
  CUDA_TRY(cudaStreamSynchronize(stream_));
}

void Engine::import_state_device(const uint32_t* prefix, size_t n, const void* src,
                                 size_t nbytes) {
  CUDA_TRY(cudaSetDevice(device_));
  if (n > capacity) fail("state of %zu tokens exceeds the engine capacity %zu", n, capacity);
  const size_t need = state_image_bytes(n);
  if (nbytes != need)
    fail("import_state_device: %zu bytes for a %zu-token state, expected %zu", nbytes, n, need);
  check_device_ptr(src, device_, "import_state_device: src");
  size_t off = 0;
  for (int l = 0; l < config.layers; ++l) {
    if (!config.has_kv(l)) continue;
    auto [r0, r1] = state_rows(l, n);
    const size_t row_bytes = static_cast<size_t>(2) * config.kv_heads * config.head_dim[l] * 2;
    const size_t bytes = (r1 - r0) * row_bytes;
    if (bytes)
      CUDA_TRY(cudaMemcpyAsync(kv_[l].as<uint8_t>() + r0 * row_bytes,
                               static_cast<const uint8_t*>(src) + off, bytes,
                               cudaMemcpyDeviceToDevice, stream_));
    off += bytes;
  }
  std::vector<TokMeta> meta(n);
  for (size_t i = 0; i < n; ++i) meta[i] = {static_cast<int>(i), 0, 0, static_cast<int>(i + 1)};
  if (n)
    CUDA_TRY(cudaMemcpyAsync(meta_.p, meta.data(), n * sizeof(TokMeta), cudaMemcpyHostToDevice,
                             stream_));
  CUDA_TRY(cudaStreamSynchronize(stream_));
  std::lock_guard<std::mutex> g(mu_);
  resident_ = std::vector<uint32_t>(prefix, prefix + n);
}

std::string Engine::state_path(const uint32_t* prefix, size_t n) const {
  if (state_dir_.empty()) return "";
  char name[32];
  snprintf(name, sizeof name, "%016llx.state",
           static_cast<unsigned long long>(state_key(model_id_, prefix, n)));
  return state_dir_ + "/" + name;
}

// engine.rs:2096-2120: RAM first, then the state directory (promoted).
std::optional<PrefixSource> Engine::restore_from_cache(const uint32_t* prefix, size_t n) {
  bool on;
  {
    std::lock_guard<std::mutex> g(mu_);
    on = states_.budget > 0 || !state_dir_.empty();
  }
  if (n == 0 || !on) return std::nullopt;
  std::optional<SavedState> ram;
  {
    std::lock_guard<std::mutex> g(mu_);
    ram = states_.get(std::vector<uint32_t>(prefix, prefix + n));
  }
  if (ram) {
    try {
      restore_state(*ram);
      return PrefixSource::Ram;
    } catch (const Error&) {
      return std::nullopt;
    }
  }
  const std::string path = state_path(prefix, n);
  if (path.empty()) return std::nullopt;
  std::ifstream f(path, std::ios::binary);
  if (!f) return std::nullopt;
  std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  try {
    SavedState s = SavedState::from_bytes(bytes.data(), bytes.size(), model_id_);
    if (s.prefix.size() != n || !std::equal(s.prefix.begin(), s.prefix.end(), prefix))
      return std::nullopt;
    restore_state(s);
    std::lock_guard<std::mutex> g(mu_);
    states_.put(std::move(s));
    return PrefixSource::Disk;
  } catch (const Error&) {
    return std::nullopt;
  }
}

void Engine::remember(const uint32_t* prefix, size_t n, size_t row0) {
  bool on;
  {
    std::lock_guard<std::mutex> g(mu_);
    on = states_.budget > 0 || !state_dir_.empty();
  }
  if (n == 0 || !on) return;
  SavedState s = save_state_at(prefix, n, row0);
  const std::string path = state_path(prefix, n);
  if (!path.empty()) {
    mkdir(state_dir_.c_str(), 0755);
    std::ofstream f(path, std::ios::binary);
    uint8_t head[10];
    std::memcpy(head, "GRWS1\0", 6);
    put_u32(head + 6, static_cast<uint32_t>(model_id_.size()));
    f.write(reinterpret_cast<const char*>(head), 10);
    f.write(model_id_.data(), static_cast<std::streamsize>(model_id_.size()));
    f.write(reinterpret_cast<const char*>(s.body.get()), static_cast<std::streamsize>(s.body_len));
    if (!f) fail("writing %s", path.c_str());
  }
  std::lock_guard<std::mutex> g(mu_);
  states_.put(std::move(s));
}

float Engine::time_forward(const GroupIn* groups, size_t n, Want want, bool resident, int iters,
                           int* launches) {
  CUDA_TRY(cudaSetDevice(device_));
  if (resident && !is_resident(groups[0].prefix, groups[0].n_prefix))
    fail("time_forward: the first group's prefix is not resident");
  Packing p = pack(groups, n, 0, resident);
  std::vector<uint8_t> rows;
  if (config.per_layer_dim > 0) rows = gather_per_layer(reinterpret_cast<const uint32_t*>(p.ids.data()), p.ids.size());
  upload(p, rows.empty() ? nullptr : rows.data(), rows.size());
  CUDA_TRY(cudaStreamSynchronize(stream_));
  int nl = 0;
  CUDA_TRY(cudaEventRecord(events_[6], stream_));
  for (int i = 0; i < iters; ++i) nl = run_forward(p, want);
  CUDA_TRY(cudaEventRecord(events_[7], stream_));
  CUDA_TRY(cudaMemcpyAsync(h_status_.p, status_.p, 4, cudaMemcpyDeviceToHost, stream_));
  CUDA_TRY(cudaStreamSynchronize(stream_));
  check_status();
  float ms = 0;
  CUDA_TRY(cudaEventElapsedTime(&ms, events_[6], events_[7]));
  if (launches) *launches = nl;
  if (!resident) {
    // The timed passes decoded groups[0]'s prefix into rows 0..P.
    std::lock_guard<std::mutex> g(mu_);
    resident_ = std::vector<uint32_t>(groups[0].prefix, groups[0].prefix + groups[0].n_prefix);
  }
  return ms;
}

void Engine::record_event(int slot) {
  if (slot < 0 || slot >= 6) fail("event slot %d out of range", slot);
  CUDA_TRY(cudaSetDevice(device_));
  CUDA_TRY(cudaEventRecord(events_[slot], stream_));
}

float Engine::elapsed_ms(int a, int b) {
  if (a < 0 || a >= 6 || b < 0 || b >= 6) fail("event slot out of range");
  CUDA_TRY(cudaEventSynchronize(events_[b]));
  float ms = 0;
  CUDA_TRY(cudaEventElapsedTime(&ms, events_[a], events_[b]));
  return ms;
}

}  // namespace omg
