// The Laya / ModernBERT encoder engine: crates/omg-wgpu/src/laya.rs
// re-designed for one B200.
//
// Every question is one sequence; a request's sequences are packed into one
// token stream and evaluated in one pass, isolated by the attention's
// same-sequence rule (plus the local window on ModernBERT's local layers).
// The encoder and the decision-head layers run on the GPU; the scorer and
// the act head (a few hundred KFLOP per sequence) run on the host in f32, as
// in the reference (laya.rs:1442-1493).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "engine.h"
#include "gemm.cuh"
#include "laya_kernels.cuh"
#include "model.h"

namespace omg {

// laya.rs:46-83 LayaConfig.
struct LayaConfig {
  int vocab = 0, d = 0, layers = 0, heads = 0, ff = 0;
  std::vector<bool> sliding;  // per encoder layer: local attention
  int window = 64;            // inclusive local distance: local_attention / 2
  float theta_global = 160000.f, theta_local = 10000.f, eps = 1e-5f;
  int head_layers = 2;
  bool type_emb = true;
  int act_hidden = 256, act_out = 0;
  int max_len = 512, head_max_len = 192;
  float temperature[3] = {1.f, 1.f, 1.f};
  std::map<std::string, float> temperature_by_options;
  uint32_t cls = 0, sep = 0, mask = 0, pad = 0;
  std::string mask_text;

  // laya.rs:88-209 + 312-323 (config_from_export): an exported directory's
  // config.json — the encoder config with the agent config under
  // `laya_agent` and the special tokens' surface forms under `laya_tokens`.
  // The reference resolves a surface form with the tokenizer; here the
  // caller passes that map as `laya_special_ids` ({"[MASK]": id, ...}).
  static LayaConfig from_json(const std::string& text);
  int head_dim() const { return heads > 0 ? d / heads : 0; }
  // laya.rs:212-230 plus what this engine's kernels need.
  void validate() const;
  // laya.rs:234-249.
  float temperature_for(int qtype, size_t k) const;
  // laya.rs:252-309: every tensor, in catalogue order.
  std::vector<Config::TensorSpec> tensors() const;
};

// laya.rs:326-328: tensors evaluated on the host.
bool laya_is_host_tensor(const std::string& name);

// laya.rs:469-476 Sequence (borrowed).
struct LayaSequence {
  const uint32_t* ids;
  size_t n_ids;
  const size_t* markers;  // token index of each option's [MASK]
  size_t n_markers;
  int qtype;              // 0 choice, 1 score, 2 noul
};

// laya.rs:482-485 Output.
struct LayaOutput {
  std::vector<float> logits;
  bool has_act = false;
  float act_probability = 0.f;
};

class LayaEngine;

// laya.rs:612-1084 LayaBuilder: receives the weights one tensor at a time.
class LayaBuilder {
 public:
  LayaBuilder(LayaConfig cfg, int device);
  ~LayaBuilder();
  const LayaConfig& config() const { return cfg_; }
  std::vector<std::string> missing() const;
  void push(const std::string& name, const HostTensor& t);
  std::unique_ptr<LayaEngine> finish(size_t capacity, size_t max_rows);

 private:
  friend class LayaEngine;
  LayaConfig cfg_;
  int device_;
  cudaStream_t stream_ = nullptr;
  std::map<std::string, std::vector<int64_t>> expected_;
  std::map<std::string, bool> pushed_;
  std::map<std::string, DevBuffer> lin_;  // f16 [N, K]; Wi as "enc.l.wi" ([val 128 | gate 128] blocks)
  std::map<std::string, DevBuffer> vec_;  // f32 vectors (norms, biases) and type_emb [3, d]
  std::map<std::string, std::vector<float>> host_;
  int embed_dtype_ = 0;
  DevBuffer embed_codes_, embed_scales_;
};

class LayaEngine {
 public:
  ~LayaEngine();
  const LayaConfig config;
  const size_t capacity;
  const size_t max_rows;

  // laya.rs:1138-1432: per sequence, the [CLS] row then each marker's row
  // (d floats each), written in sequence order into `out`.
  void hidden(const LayaSequence* seqs, size_t n, float* out, size_t out_floats);
  // laya.rs:1435-1438: the scorer's logits per option and the act head's
  // probability per sequence.
  std::vector<LayaOutput> evaluate(const LayaSequence* seqs, size_t n);
  // laya.rs:1489-1493: softmax of logits / temperature_for(qtype, k).
  std::vector<double> probabilities(int qtype, const float* logits, size_t k) const;
  // laya.rs:1126-1134.
  void warmup();

  // Device-resident timing: pack and upload once, then `iters` decision
  // passes (encoder, gather and head) between two CUDA events on the
  // engine's stream; total milliseconds.
  float time_forward(const LayaSequence* seqs, size_t n, int iters, int* launches);
  // Per-kernel device time of `iters` passes: JSON {"kernel": [launches, ms]}.
  std::string profile_forward(const LayaSequence* seqs, size_t n, int iters);
  void record_event(int slot);
  float elapsed_ms(int a, int b);
  cudaStream_t stream() const { return stream_; }
  int device() const { return device_; }

 private:
  friend class LayaBuilder;
  LayaEngine(LayaBuilder&& b, size_t capacity, size_t max_rows);

  struct Packing {
    std::vector<int32_t> ids, pos, qtype;
    std::vector<int2> span;
    std::vector<int32_t> row_map;
    std::vector<LayaAttnItem> items[2];  // [0] local window, [1] global
    // Decision head: per sequence (its [CLS] row in the gathered rows, its
    // first logit, its marker count, 0); the gathered row of each marker.
    std::vector<int4> head_seq;
    std::vector<int32_t> marker_row;
    size_t t = 0;
  };
  struct EncLayer {
    GemmPlan qkv, o, wi, wo;
    const float *attn_norm = nullptr, *mlp_norm = nullptr;
    bool sliding = false;
  };
  struct HeadLayer {
    GemmPlan in, out, l1, l2;
    const float *n1w, *n1b, *in_b, *out_b, *n2w, *n2b, *l1_b, *l2_b;
  };

  Packing pack(const LayaSequence* seqs, size_t n) const;
  void upload(const Packing& p);
  // The encoder pass and the row gather; with `head`, also the decision
  // head (scorer logits and act probabilities) on the device.
  int launch_forward(const Packing& p, bool head = false);
  void check_status();
  void prof_mark(const char* name);

  int device_;
  int num_sms_ = 148;
  cudaStream_t stream_ = nullptr;
  std::map<std::string, DevBuffer> lin_, vec_;
  std::map<std::string, DevBuffer> headw_;  // scorer.* / act.* as f32
  float l2_bias_ = 0.f;                      // scorer.l2_b
  int embed_dtype_ = 0;
  DevBuffer embed_codes_, embed_scales_;
  std::vector<EncLayer> enc_;
  std::vector<HeadLayer> head_;
  const float *embed_norm_ = nullptr, *final_norm_ = nullptr, *type_emb_ = nullptr;
  size_t cap_rows_ = 0;
  int act_stride_ = 0;

  // Workspace.
  DevBuffer ids_, pos_, qtype_, span_, row_map_, items_, x_, h16_, qkv16_, attn16_, act16_,
      rows_, rope_local_, rope_global_, status_, head_idx_, head_out_;
  PinnedBuffer h_ids_, h_pos_, h_qtype_, h_span_, h_row_map_, h_items_, h_out_, h_status_,
      h_head_idx_;
  size_t items_cap_ = 0;
  CUtensorMap tqkv_;

  bool profiling_ = false;
  std::vector<cudaEvent_t> prof_events_;
  std::vector<const char*> prof_names_;
  size_t prof_used_ = 0;
  cudaEvent_t events_[8] = {};
  mutable std::mutex mu_;
};

}  // namespace omg
