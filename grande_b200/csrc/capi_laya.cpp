// extern "C" entry points of the Laya encoder engine (declared in
// include/omg_b200.h).
#include <cmath>
#include <cstring>
#include <limits>
#include <string>

#include "capi_tensor.h"
#include "capi_util.h"
#include "laya.h"
#include "omg_b200.h"

using namespace omg;

struct omg_laya_builder {
  std::unique_ptr<LayaBuilder> b;
};
struct omg_laya_engine {
  std::unique_ptr<LayaEngine> e;
};

namespace {

const LayaSequence* to_seqs(const omg_laya_sequence* s, size_t n) {
  if (n && !s) fail("sequences is null");
  static_assert(sizeof(omg_laya_sequence) == sizeof(LayaSequence), "layout");
  for (size_t i = 0; i < n; ++i) {
    if (s[i].n_ids && !s[i].ids) fail("sequence %zu: ids is null", i);
    if (s[i].n_markers && !s[i].markers) fail("sequence %zu: markers is null", i);
  }
  return reinterpret_cast<const LayaSequence*>(s);
}

}  // namespace

extern "C" {

int omg_laya_config_check(const char* config_json, char* summary, size_t cap) {
  return guarded([&] {
    if (!config_json) fail("config is null");
    LayaConfig c = LayaConfig::from_json(config_json);
    char buf[256];
    snprintf(buf, sizeof buf, "layers=%d d=%d heads=%d ff=%d vocab=%d head_layers=%d act_out=%d",
             c.layers, c.d, c.heads, c.ff, c.vocab, c.head_layers, c.act_out);
    return copy_out(buf, summary, cap, nullptr);
  });
}

int omg_laya_config_tensors(const char* config_json, char* buf, size_t cap, size_t* needed) {
  return guarded([&] {
    if (!config_json) fail("config is null");
    LayaConfig c = LayaConfig::from_json(config_json);
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

int omg_laya_builder_new(const char* config_json, int device, omg_laya_builder** out) {
  return guarded([&] {
    if (!config_json || !out) fail("null argument");
    auto b = std::make_unique<omg_laya_builder>();
    b->b = std::make_unique<LayaBuilder>(LayaConfig::from_json(config_json), device);
    *out = b.release();
    return 0;
  });
}

int omg_laya_builder_push(omg_laya_builder* b, const char* name, int dtype, const int64_t* shape,
                          int ndim, const void* data, size_t nbytes, const void* scales,
                          size_t scales_nbytes) {
  return guarded([&] {
    if (!b || !b->b || !name || (ndim && !shape)) fail("null argument");
    b->b->push(name, make_tensor(dtype, shape, ndim, data, nbytes, scales, scales_nbytes));
    return 0;
  });
}

int omg_laya_builder_missing(omg_laya_builder* b, char* buf, size_t cap, size_t* needed) {
  return guarded([&] {
    if (!b || !b->b) fail("null builder");
    std::string s;
    for (const auto& n : b->b->missing()) s += n + "\n";
    return copy_out(s, buf, cap, needed);
  });
}

int omg_laya_builder_finish(omg_laya_builder* b, size_t capacity, size_t max_rows,
                            omg_laya_engine** out) {
  std::unique_ptr<omg_laya_builder> owned(b);
  return guarded([&] {
    if (!owned || !owned->b || !out) fail("null argument");
    auto e = std::make_unique<omg_laya_engine>();
    e->e = owned->b->finish(capacity, max_rows);
    *out = e.release();
    return 0;
  });
}

void omg_laya_builder_free(omg_laya_builder* b) { delete b; }

int omg_laya_warmup(omg_laya_engine* e) {
  return guarded([&] {
    if (!e || !e->e) fail("null engine");
    e->e->warmup();
    return 0;
  });
}

int omg_laya_hidden(omg_laya_engine* e, const omg_laya_sequence* seqs, size_t n, float* out_rows,
                    size_t out_floats) {
  return guarded([&] {
    if (!e || !e->e) fail("null engine");
    if (out_floats && !out_rows) fail("output is null");
    e->e->hidden(to_seqs(seqs, n), n, out_rows, out_floats);
    return 0;
  });
}

int omg_laya_evaluate(omg_laya_engine* e, const omg_laya_sequence* seqs, size_t n,
                      float* out_logits, size_t logits_cap, float* out_act) {
  return guarded([&] {
    if (!e || !e->e) fail("null engine");
    const LayaSequence* s = to_seqs(seqs, n);
    size_t k = 0;
    for (size_t i = 0; i < n; ++i) k += s[i].n_markers;
    if (logits_cap < k) fail("logits buffer holds %zu floats, the request returns %zu", logits_cap, k);
    if (k && !out_logits) fail("logits output is null");
    const std::vector<LayaOutput> outs = e->e->evaluate(s, n);
    size_t o = 0;
    for (size_t i = 0; i < n; ++i) {
      std::memcpy(out_logits + o, outs[i].logits.data(), outs[i].logits.size() * 4);
      o += outs[i].logits.size();
      if (out_act)
        out_act[i] = outs[i].has_act ? outs[i].act_probability
                                     : std::numeric_limits<float>::quiet_NaN();
    }
    return 0;
  });
}

int omg_laya_probabilities(omg_laya_engine* e, int qtype, const float* logits, size_t k,
                           double* out) {
  return guarded([&] {
    if (!e || !e->e) fail("null engine");
    if (k && (!logits || !out)) fail("null argument");
    const std::vector<double> p = e->e->probabilities(qtype, logits, k);
    std::memcpy(out, p.data(), k * sizeof(double));
    return 0;
  });
}

int omg_laya_time_forward(omg_laya_engine* e, const omg_laya_sequence* seqs, size_t n, int iters,
                          float* ms, int* launches) {
  return guarded([&] {
    if (!e || !e->e || !ms) fail("null argument");
    if (iters < 1) fail("iters must be positive");
    *ms = e->e->time_forward(to_seqs(seqs, n), n, iters, launches);
    return 0;
  });
}

int omg_laya_profile_forward(omg_laya_engine* e, const omg_laya_sequence* seqs, size_t n,
                             int iters, char* buf, size_t cap, size_t* needed) {
  return guarded([&] {
    if (!e || !e->e) fail("null engine");
    if (iters < 1) fail("iters must be positive");
    return copy_out(e->e->profile_forward(to_seqs(seqs, n), n, iters), buf, cap, needed);
  });
}

int omg_laya_record_event(omg_laya_engine* e, int slot) {
  return guarded([&] {
    if (!e || !e->e) fail("null engine");
    e->e->record_event(slot);
    return 0;
  });
}

int omg_laya_elapsed_ms(omg_laya_engine* e, int a, int b, float* ms) {
  return guarded([&] {
    if (!e || !e->e || !ms) fail("null argument");
    *ms = e->e->elapsed_ms(a, b);
    return 0;
  });
}

void omg_laya_destroy(omg_laya_engine* e) { delete e; }

}  // extern "C"
