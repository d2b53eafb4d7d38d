// extern "C" entry points of the engine (declared in include/omg_b200.h).
#include <cmath>
#include <cstring>
#include <string>

#include "capi_tensor.h"
#include "capi_util.h"
#include "engine.h"
#include "omg_b200.h"

using namespace omg;

struct omg_builder {
  std::unique_ptr<EngineBuilder> b;
};
struct omg_engine {
  std::unique_ptr<Engine> e;
};
struct omg_state {
  SavedState s;
};

namespace {

std::vector<GroupIn> to_groups(const omg_group* g, size_t n) {
  if (n && !g) fail("groups is null");
  std::vector<GroupIn> out(n);
  for (size_t i = 0; i < n; ++i) {
    out[i].prefix = g[i].prefix;
    out[i].n_prefix = g[i].n_prefix;
    out[i].branches = reinterpret_cast<const BranchIn*>(g[i].branches);
    out[i].n_branches = g[i].n_branches;
  }
  return out;
}

Want want_of(int w) {
  if (w == OMG_WANT_LOGITS) return Want::Logits;
  if (w == OMG_WANT_HIDDEN) return Want::Hidden;
  fail("want must be OMG_WANT_LOGITS or OMG_WANT_HIDDEN (got %d)", w);
}

Engine& eng(omg_engine* e) {
  if (!e || !e->e) fail("engine is null");
  return *e->e;
}

}  // namespace

static_assert(sizeof(omg_branch) == sizeof(BranchIn), "omg_branch layout");

extern "C" {

int omg_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

int omg_host_alloc(int device, size_t bytes, void** out) {
  return guarded([&] {
    if (!out) fail("null argument");
    *out = nullptr;
    CUDA_TRY(cudaSetDevice(device));
    void* p = nullptr;
    const cudaError_t e = cudaHostAlloc(&p, bytes ? bytes : 1, cudaHostAllocPortable);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      fail("cudaHostAlloc of %zu bytes: %s", bytes, cudaGetErrorString(e));
    }
    *out = p;
    return 0;
  });
}

void omg_host_free(void* p) {
  if (p) (void)cudaFreeHost(p);
}

int omg_config_check(const char* config_json, char* summary, size_t cap) {
  return guarded([&] {
    if (!config_json) fail("config is null");
    Config c = Config::from_json(config_json);
    c.validate();
    char buf[256];
    snprintf(buf, sizeof buf, "layers=%d d=%d heads=%d kv_heads=%d vocab=%d", c.layers, c.d,
             c.heads, c.kv_heads, c.vocab);
    return copy_out(buf, summary, cap, nullptr);
  });
}

int omg_config_tensors(const char* config_json, char* buf, size_t cap, size_t* needed) {
  return guarded([&] {
    if (!config_json) fail("config is null");
    Config c = Config::from_json(config_json);
    std::string s;
    for (const auto& t : c.tensors()) {
      s += t.name;
      for (size_t i = 0; i < t.shape.size(); ++i)
        s += (i ? "," : " ") + std::to_string(t.shape[i]);
      s += "\n";
    }
    return copy_out(s, buf, cap, needed);
  });
}

int omg_builder_new(const char* config_json, int device, omg_builder** out) {
  return guarded([&] {
    if (!config_json || !out) fail("null argument");
    auto b = std::make_unique<omg_builder>();
    b->b = std::make_unique<EngineBuilder>(Config::from_json(config_json), device);
    *out = b.release();
    return 0;
  });
}

int omg_builder_push(omg_builder* b, const char* name, int dtype, const int64_t* shape, int ndim,
                     const void* data, size_t nbytes, const void* scales, size_t nscales) {
  return guarded([&] {
    if (!b || !b->b) fail("builder is null");
    if (!name) fail("name is null");
    b->b->push(name, make_tensor(dtype, shape, ndim, data, nbytes, scales, nscales));
    return 0;
  });
}

int omg_builder_set_per_layer_table(omg_builder* b, int dtype, const int64_t* shape, int ndim,
                                    const void* data, size_t nbytes, const void* scales,
                                    size_t nscales) {
  return guarded([&] {
    if (!b || !b->b) fail("builder is null");
    b->b->set_per_layer_table(make_tensor(dtype, shape, ndim, data, nbytes, scales, nscales));
    return 0;
  });
}

int omg_builder_set_weight_layout(omg_builder* b, int layout) {
  return guarded([&] {
    if (!b || !b->b) fail("builder is null");
    if (layout != OMG_WEIGHTS_PACKED && layout != OMG_WEIGHTS_F16)
      fail("weight layout must be OMG_WEIGHTS_PACKED or OMG_WEIGHTS_F16 (got %d)", layout);
    b->b->set_packed(layout == OMG_WEIGHTS_PACKED);
    return 0;
  });
}

int omg_builder_missing(omg_builder* b, char* buf, size_t cap, size_t* needed) {
  return guarded([&] {
    if (!b || !b->b) fail("builder is null");
    std::string s;
    for (const auto& n : b->b->missing()) s += n + "\n";
    return copy_out(s, buf, cap, needed);
  });
}

int omg_builder_finish(omg_builder* b, size_t capacity, size_t max_rows, omg_engine** out) {
  int rc = guarded([&] {
    if (!b || !b->b) fail("builder is null");
    if (!out) fail("out is null");
    auto e = std::make_unique<omg_engine>();
    e->e = b->b->finish(capacity, max_rows);
    *out = e.release();
    return 0;
  });
  delete b;
  return rc;
}

void omg_builder_free(omg_builder* b) { delete b; }

int omg_engine_evaluate_groups(omg_engine* e, const omg_group* groups, size_t n_groups, int want,
                               float* out, size_t out_floats, int32_t* prefix_sources) {
  return guarded([&] {
    auto gs = to_groups(groups, n_groups);
    if (!out && out_floats) fail("out is null");
    eng(e).evaluate_groups(gs.data(), gs.size(), want_of(want), out, out_floats, prefix_sources);
    return 0;
  });
}

int omg_engine_evaluate(omg_engine* e, const uint32_t* prefix, size_t n_prefix,
                        const omg_branch* branches, size_t n_branches, int want, float* out,
                        size_t out_floats) {
  omg_group g{prefix, n_prefix, branches, n_branches};
  return omg_engine_evaluate_groups(e, &g, 1, want, out, out_floats, nullptr);
}

int omg_engine_evaluate_rows(omg_engine* e, const uint32_t* prefix, size_t n_prefix,
                             const omg_branch* branches, size_t n_branches, int want,
                             const void* per_layer_rows, size_t rows_bytes, float* out,
                             size_t out_floats) {
  return guarded([&] {
    omg_group g{prefix, n_prefix, branches, n_branches};
    auto gs = to_groups(&g, 1);
    eng(e).evaluate_rows(gs[0], want_of(want), static_cast<const uint8_t*>(per_layer_rows),
                         rows_bytes, out, out_floats);
    return 0;
  });
}

int omg_engine_warmup(omg_engine* e) {
  return guarded([&] {
    eng(e).warmup();
    return 0;
  });
}

int omg_engine_prefix_source(omg_engine* e) {
  if (!e || !e->e) return OMG_SOURCE_NONE;
  auto s = e->e->prefix_source();
  return s ? static_cast<int>(*s) : OMG_SOURCE_NONE;
}

int omg_engine_is_resident(omg_engine* e, const uint32_t* prefix, size_t n) {
  if (!e || !e->e || (!prefix && n)) return 0;
  return e->e->is_resident(prefix, n) ? 1 : 0;
}

void omg_engine_evict_resident(omg_engine* e) {
  if (e && e->e) e->e->evict_resident();
}

int omg_engine_set_state_cache(omg_engine* e, size_t bytes, const char* dir,
                               const char* model_id) {
  return guarded([&] {
    eng(e).set_state_cache(bytes, dir ? dir : "", model_id ? model_id : "wgpu");
    return 0;
  });
}

int omg_engine_save_state(omg_engine* e, const uint32_t* prefix, size_t n, omg_state** out) {
  return guarded([&] {
    if (!out) fail("out is null");
    auto s = std::make_unique<omg_state>();
    s->s = eng(e).save_state(prefix, n);
    *out = s.release();
    return 0;
  });
}

int omg_engine_restore_state(omg_engine* e, const omg_state* s) {
  return guarded([&] {
    if (!s) fail("state is null");
    eng(e).restore_state(s->s);
    return 0;
  });
}

size_t omg_engine_state_image_bytes(omg_engine* e, size_t n) {
  if (!e || !e->e) return 0;
  return e->e->state_image_bytes(n);
}

int omg_engine_export_state_device(omg_engine* e, const uint32_t* prefix, size_t n, void* dst,
                                   size_t cap) {
  return guarded([&] {
    eng(e).export_state_device(prefix, n, dst, cap);
    return 0;
  });
}

int omg_engine_import_state_device(omg_engine* e, const uint32_t* prefix, size_t n,
                                   const void* src, size_t nbytes) {
  return guarded([&] {
    if (n && !prefix) fail("prefix is null");
    eng(e).import_state_device(prefix, n, src, nbytes);
    return 0;
  });
}

int omg_engine_gather_per_layer(omg_engine* e, const uint32_t* ids, size_t n, uint8_t* out,
                                size_t cap) {
  return guarded([&] {
    auto rows = eng(e).gather_per_layer(ids, n);
    if (cap < rows.size()) fail("gather_per_layer: buffer holds %zu bytes, need %zu", cap, rows.size());
    std::memcpy(out, rows.data(), rows.size());
    return 0;
  });
}

int omg_engine_weight_f16(omg_engine* e, const char* name, uint16_t* out, size_t n) {
  return guarded([&] {
    if (!name) fail("weight name is null");
    auto w = eng(e).weight_f16(name);
    if (n != w.size()) fail("weight_f16: %s has %zu values, the buffer %zu", name, w.size(), n);
    std::memcpy(out, w.data(), w.size() * 2);
    return 0;
  });
}

int omg_engine_arm_wait_timeout(omg_engine* e, long long clocks) {
  return guarded([&] {
    eng(e).arm_wait_timeout(clocks);
    return 0;
  });
}

int omg_engine_get_info(omg_engine* e, omg_engine_info* info) {
  return guarded([&] {
    Engine& x = eng(e);
    if (!info) fail("info is null");
    info->d = x.config.d;
    info->vocab = x.config.vocab;
    info->layers = x.config.layers;
    info->embed_dtype = x.embed_dtype();
    info->per_layer_dim = x.config.per_layer_dim;
    info->device = x.device();
    info->capacity = x.capacity;
    info->max_rows = x.max_rows;
    info->bos = x.config.bos;
    return 0;
  });
}

int omg_engine_time_forward(omg_engine* e, const omg_group* groups, size_t n_groups, int want,
                            int resident, int iters, float* ms, int* launches) {
  return guarded([&] {
    auto gs = to_groups(groups, n_groups);
    if (gs.empty()) fail("empty request");
    const float t = eng(e).time_forward(gs.data(), gs.size(), want_of(want), resident != 0,
                                        iters, launches);
    if (ms) *ms = t;
    return 0;
  });
}

int omg_engine_profile_forward(omg_engine* e, const omg_group* groups, size_t n_groups, int want,
                               int resident, int iters, char* json, size_t cap, size_t* needed) {
  return guarded([&] {
    auto gs = to_groups(groups, n_groups);
    if (gs.empty()) fail("empty request");
    const std::string js =
        eng(e).profile_forward(gs.data(), gs.size(), want_of(want), resident != 0, iters);
    return copy_out(js, json, cap, needed);
  });
}

int omg_engine_record_event(omg_engine* e, int slot) {
  return guarded([&] {
    eng(e).record_event(slot);
    return 0;
  });
}

int omg_engine_elapsed_ms(omg_engine* e, int a, int b, float* ms) {
  return guarded([&] {
    const float t = eng(e).elapsed_ms(a, b);
    if (ms) *ms = t;
    return 0;
  });
}

void omg_engine_destroy(omg_engine* e) { delete e; }

size_t omg_state_byte_len(const omg_state* s) { return s ? s->s.byte_len() : 0; }

int omg_state_to_bytes(const omg_state* s, const char* model_id, uint8_t* buf, size_t cap,
                       size_t* needed) {
  return guarded([&] {
    if (!s) fail("state is null");
    const std::string id = model_id ? model_id : "";
    const size_t len = s->s.file_len(id);
    if (needed) *needed = len;
    if (buf) {
      if (cap < len) fail("buffer holds %zu bytes, the state needs %zu", cap, len);
      s->s.write_bytes(id, buf);
    }
    return 0;
  });
}

int omg_state_from_bytes(const uint8_t* bytes, size_t n, const char* model_id, omg_state** out) {
  return guarded([&] {
    if (!out || (!bytes && n)) fail("null argument");
    auto s = std::make_unique<omg_state>();
    s->s = SavedState::from_bytes(bytes, n, model_id ? model_id : "");
    *out = s.release();
    return 0;
  });
}

int omg_state_prefix(const omg_state* s, uint32_t* buf, size_t cap, size_t* n) {
  return guarded([&] {
    if (!s) fail("state is null");
    if (n) *n = s->s.prefix.size();
    if (buf) std::memcpy(buf, s->s.prefix.data(), std::min(cap, s->s.prefix.size()) * 4);
    return 0;
  });
}

void omg_state_free(omg_state* s) { delete s; }

uint64_t omg_state_key(const char* model_id, const uint32_t* prefix, size_t n) {
  return state_key(model_id ? model_id : "", prefix, n);
}

int omg_quantize(int dtype, const float* v, size_t n, uint8_t* codes, uint8_t* scales) {
  return guarded([&] {
    if (dtype != OMG_DTYPE_F16 && n % 32) fail("%zu values is not a multiple of 32", n);
    if (dtype == OMG_DTYPE_Q8)
      quantize_q8(v, n, codes, scales);
    else if (dtype == OMG_DTYPE_Q4)
      quantize_q4(v, n, codes, scales);
    else if (dtype == OMG_DTYPE_F16) {
      for (size_t i = 0; i < n; ++i) {
        const uint16_t h = f32_to_f16(v[i]);
        codes[2 * i] = static_cast<uint8_t>(h & 0xff);
        codes[2 * i + 1] = static_cast<uint8_t>(h >> 8);
      }
    } else
      fail("unsupported dtype %d", dtype);
    return 0;
  });
}

int omg_dequantize(int dtype, const uint8_t* codes, const uint8_t* scales, size_t n, float* out) {
  return guarded([&] {
    if (dtype < 0 || dtype > 2) fail("unsupported dtype %d", dtype);
    if (dtype != 0 && n % 32) fail("%zu values is not a multiple of 32", n);
    dequantize(dtype, codes, scales, n, out);
    return 0;
  });
}

// Seeded N(mean, std) values for synthetic checkpoints: xorshift64 (the
// generator of crates/omg-wgpu/tests/reference.rs:17-26) seeded with
// FNV-1a(name) ^ seed, feeding Box-Muller on 53-bit uniforms.
int omg_synth_normal(uint64_t seed, const char* name, float mean, float stddev, float* out,
                     size_t n) {
  return guarded([&] {
    uint64_t s = 0xcbf29ce484222325ull;
    for (const char* p = name ? name : ""; *p; ++p) {
      s ^= static_cast<uint8_t>(*p);
      s *= 0x00000100000001b3ull;
    }
    s ^= seed;
    if (s == 0) s = 0x9e3779b97f4a7c15ull;
    auto next = [&]() {
      s ^= s << 13;
      s ^= s >> 7;
      s ^= s << 17;
      return (static_cast<double>(s >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    };
    const double two_pi = 6.283185307179586;
    for (size_t i = 0; i < n; i += 2) {
      const double u1 = next(), u2 = next();
      const double r = std::sqrt(-2.0 * std::log(u1));
      out[i] = static_cast<float>(mean + stddev * r * std::cos(two_pi * u2));
      if (i + 1 < n) out[i + 1] = static_cast<float>(mean + stddev * r * std::sin(two_pi * u2));
    }
    return 0;
  });
}

}  // extern "C"
