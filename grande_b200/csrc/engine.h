// The decoder engine: crates/omg-wgpu/src/engine.rs re-designed for one B200.
//
// Weights and a token-capacity-sized workspace live in HBM for the life of
// the engine. A request (one or more groups of prefix + branches) is packed
// into one block-causal pass exactly as engine.rs:1492-1571 packs it, the
// whole network is launched on the engine's stream, and only the wanted rows
// come back. The prefix of the first group stays resident (its K/V rows are
// kept), and decoded prefixes can be kept in a RAM / file state cache.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <array>
#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <vector>

#include "attention.cuh"
#include "gemm.cuh"
#include "kernels.cuh"
#include "model.h"

namespace omg {

enum class PrefixSource : int { Resident = 0, Ram = 1, Disk = 2, Decoded = 3 };
enum class Want : int { Logits = 0, Hidden = 1 };

// A tensor as pushed (model.rs:376-384 QTensor).
struct HostTensor {
  int dtype = 0;
  std::vector<int64_t> shape;
  std::vector<uint8_t> data, scales;
  size_t numel() const {
    size_t n = 1;
    for (auto s : shape) n *= static_cast<size_t>(s);
    return n;
  }
  float get(size_t i) const;
};

// omg_core::BranchTokens (backend.rs:26-30) and engine.rs Group (:29-32).
struct BranchIn {
  const int32_t* tokens;
  size_t n_tokens;
  const size_t* want;
  size_t n_want;
};
struct GroupIn {
  const uint32_t* prefix;
  size_t n_prefix;
  const BranchIn* branches;
  size_t n_branches;
  size_t tokens() const {
    size_t n = n_prefix;
    for (size_t b = 0; b < n_branches; ++b) n += branches[b].n_tokens;
    return n;
  }
  size_t rows() const {
    size_t n = 0;
    for (size_t b = 0; b < n_branches; ++b) n += branches[b].n_want;
    return n;
  }
};

// engine.rs:503-580: a prefix's K/V rows as f16 per layer that owns K/V;
// sliding layers keep only the last `window` rows. The rows live in one
// page-locked host block laid out as the GRWS1 file from the prefix count
// on (prefix, layer count, per layer its header and rows), so the device
// copies land straight in the file's bytes and a save or restore moves at
// the host link's speed.
struct SavedState {
  std::vector<uint32_t> prefix;
  struct Layer {
    int layer = 0;
    int row0 = 0;
    size_t off = 0;  // f16 LE rows of [kv_heads * hd K | kv_heads * hd V] at body + off
    size_t len = 0;
  };
  std::vector<Layer> layers;
  std::shared_ptr<uint8_t> body;
  size_t body_len = 0;

  const uint8_t* data(const Layer& l) const { return body.get() + l.off; }
  uint8_t* data(const Layer& l) { return body.get() + l.off; }
  size_t byte_len() const;
  size_t file_len(const std::string& model_id) const;
  // The GRWS1 file (engine.rs:510-579) into `out` (file_len bytes).
  void write_bytes(const std::string& model_id, uint8_t* out) const;
  std::vector<uint8_t> to_bytes(const std::string& model_id) const;
  static SavedState from_bytes(const uint8_t* b, size_t n, const std::string& model_id);
  // A state for `prefix` with layers (layer, row0, bytes); rows unset.
  static SavedState make(const uint32_t* prefix, size_t n,
                         const std::vector<std::array<size_t, 3>>& layers);
};

// engine.rs:584-620: LRU of saved states keyed by the exact prefix, most
// recently used last.
struct StateCache {
  size_t budget = 0, used = 0;
  std::vector<SavedState> entries;
  std::optional<SavedState> get(const std::vector<uint32_t>& prefix);
  void put(SavedState s);
};

// engine.rs:625-641: FNV-1a of (model id, 0, prefix LE bytes).
uint64_t state_key(const std::string& model_id, const uint32_t* prefix, size_t n);

struct DevBuffer {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuffer() = default;
  DevBuffer(const DevBuffer&) = delete;
  DevBuffer& operator=(const DevBuffer&) = delete;
  DevBuffer(DevBuffer&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
  DevBuffer& operator=(DevBuffer&& o) noexcept {
    if (this != &o) {
      release();
      p = o.p; bytes = o.bytes;
      o.p = nullptr; o.bytes = 0;
    }
    return *this;
  }
  ~DevBuffer() { release(); }
  void alloc(size_t n, bool zero = true);
  void release();
  template <class T> T* as() const { return static_cast<T*>(p); }
};

struct PinnedBuffer {
  void* p = nullptr;
  size_t bytes = 0;
  PinnedBuffer() = default;
  PinnedBuffer(const PinnedBuffer&) = delete;
  PinnedBuffer& operator=(const PinnedBuffer&) = delete;
  ~PinnedBuffer();
  void alloc(size_t n);
  template <class T> T* as() const { return static_cast<T*>(p); }
};

class Engine;

// engine.rs:805-1334 EngineBuilder: receives the weights one tensor at a
// time (dequantizing each linear straight into its f16 device layout) and
// allocates the workspace in finish().
class EngineBuilder {
 public:
  EngineBuilder(Config cfg, int device);
  ~EngineBuilder();
  const Config& config() const { return cfg_; }
  std::vector<std::string> missing() const;
  void push(const std::string& name, const HostTensor& t);
  void set_per_layer_table(HostTensor t);
  // Q4_0 / Q8_0 linears pushed from now on: packed chunks decoded per tile
  // (true) or f16 rows decoded once here (false, the default: faster).
  void set_packed(bool on) { packed_ = on; }
  std::unique_ptr<Engine> finish(size_t capacity, size_t max_rows);

 private:
  friend class Engine;
  struct Packed {
    int dtype = 0;
    DevBuffer codes, scales;
  };
  // A Q4_0 / Q8_0 linear kept packed in the GEMMs' chunk layout (packed.cuh).
  struct PackedLinear {
    int dtype = 0;
    int rows = 0;  // rows as stored (gate_up: interleaved, padded to 256-row blocks)
    int k = 0;
    DevBuffer chunks;
  };
  Config cfg_;
  int device_;
  cudaStream_t stream_ = nullptr;
  std::map<std::string, std::vector<int64_t>> expected_;
  std::map<std::string, bool> pushed_;
  std::map<std::string, DevBuffer> lin_;    // f16 linears (gate+up interleaved as "blk.N.gate_up")
  std::map<std::string, PackedLinear> pk_;  // Q4_0 / Q8_0 linears, packed
  bool packed_ = false;
  std::map<std::string, DevBuffer> norms_;  // f32 norm weights
  std::map<std::string, float> scalars_;
  Packed embed_;
  std::optional<HostTensor> per_layer_table_;
};

class Engine {
 public:
  ~Engine();
  const Config config;
  const size_t capacity;
  const size_t max_rows;

  // engine.rs:1404-1444. `out` gets the wanted rows in (group, branch, want)
  // order, `width` floats each (vocab for logits, d for hidden);
  // `sources[g]` the PrefixSource of each group (-1 none).
  void evaluate_groups(const GroupIn* groups, size_t n, Want want, float* out, size_t out_floats,
                       int32_t* sources);
  // engine.rs:1449-1463: caller-gathered per-layer rows (f16 LE).
  void evaluate_rows(const GroupIn& g, Want want, const uint8_t* per_layer_rows,
                     size_t rows_bytes, float* out, size_t out_floats);
  void warmup();
  std::optional<PrefixSource> prefix_source() const;
  bool is_resident(const uint32_t* prefix, size_t n) const;
  void evict_resident();
  void set_state_cache(size_t bytes, const std::string& dir, const std::string& model_id);
  SavedState save_state(const uint32_t* prefix, size_t n);
  void restore_state(const SavedState& s);
  // A state's K/V rows as one device buffer on this engine's GPU (the layer
  // payloads of save_state, f16, concatenated in layer order), so that a
  // collective can move a prefill from one GPU to others without a host copy.
  size_t state_image_bytes(size_t n) const;
  void export_state_device(const uint32_t* prefix, size_t n, void* dst, size_t cap);
  void import_state_device(const uint32_t* prefix, size_t n, const void* src, size_t nbytes);
  int embed_dtype() const { return embed_.dtype; }
  cudaStream_t stream() const { return stream_; }
  int device() const { return device_; }

  // Device-resident timing: pack `groups` once (no state cache), upload it,
  // then launch the forward `iters` times on the stream between two CUDA
  // events; returns the total milliseconds. With `resident`, the first
  // group's prefix must be resident and only the branches run (config 3).
  // Kernel launches per pass go to *launches.
  float time_forward(const GroupIn* groups, size_t n, Want want, bool resident, int iters,
                     int* launches);
  // Per-kernel device time of `iters` passes (CUDA events between launches on
  // the stream, the role of the reference's OMG_WGPU_PROFILE timestamps,
  // engine.rs:643-726): JSON {"kernel": [launches, total_ms], ...}.
  std::string profile_forward(const GroupIn* groups, size_t n, Want want, bool resident,
                              int iters);
  // Test hook for the bounded device waits: the next pass's first fused FFN
  // launch waits for an activation band that never completes and gives up
  // after `clocks` SM clocks, so the pass fails with the wait-timeout error
  // (the pass runs outside the graph cache; the hook disarms itself).
  void arm_wait_timeout(long long clocks);
  // Events on the engine's stream for end-to-end timing around API calls.
  void record_event(int slot);
  float elapsed_ms(int a, int b);
  // The f16 values the projection GEMMs multiply for the linear `name` (a
  // catalogue name; blk.N.gate and blk.N.up read their rows of the
  // interleaved gate/up weight), row-major [rows, k]: the device copy read
  // back, for bit-exact checks of the device dequantization.
  std::vector<uint16_t> weight_f16(const std::string& name) const;
  // Gather per-layer table rows for ids (engine.rs:1370-1381), f16 LE.
  std::vector<uint8_t> gather_per_layer(const uint32_t* ids, size_t n) const;

 private:
  friend class EngineBuilder;
  Engine(EngineBuilder&& b, size_t capacity, size_t max_rows);

  // A linear's device weight: f16 rows (pk kF16) or packed chunks.
  struct WeightRef {
    int pk = 0;
    const void* p = nullptr;
  };
  WeightRef weight(const std::string& name) const;
  struct Layer {
    GemmPlan qkv, o, gate_up, down, pl_gate, pl_proj;
    const float *attn_norm, *q_norm, *k_norm, *post_attn_norm, *ffn_norm, *post_ffn_norm;
    const float *pl_norm = nullptr;
    const float* next_norm;  // the norm that reads the stream after this layer
    float out_scale = 1.f;
    bool fused_mlp = false;  // gate_up and down as one launch (gemm_run_mlp)
    int hd, ff, qkv_w;
    bool sliding, has_kv;
    int kv_src;
  };

  struct Packing {
    std::vector<int32_t> ids;
    std::vector<TokMeta> meta;
    std::vector<int32_t> row_map;
    // (group, branch, slot) -> flat output row
    std::vector<size_t> out_index;
    std::vector<std::pair<size_t, size_t>> decoded;  // (group, cache row of its prefix)
    // Tensor-core attention schedule (head_dim 256): per-token visible rows,
    // then items and multi-item runs for sliding [0] and global [1] layers,
    // staged as one block: vis | items[0] | runs[0] | items[1] | runs[1].
    std::vector<int4> attn_vis;
    std::vector<AttnFlashRun> attn_runs[2];
    std::vector<int> attn_tiles[2];
    std::vector<AttnFlashItem> attn_items[2];
    std::vector<AttnFlashMerge> attn_merges[2];
    int attn_slots = 0;  // partial slots of the chunk split (the larger window's)
    // Offsets in the staged schedule block: vis, then per window
    // runs, tiles, items, merges.
    size_t attn_off[kAttnSchedParts] = {}, attn_bytes = 0;
    size_t t = 0, base = 0, nwanted = 0;
  };

  // The launch sequence of a pass is fixed by these values (kernel shapes and
  // the schedule's offsets); everything else it reads lives at fixed device
  // addresses and is uploaded before each pass.
  struct GraphKey {
    size_t t = 0, base = 0, nwanted = 0, sched_bytes = 0;
    size_t attn_off[kAttnSchedParts] = {};
    size_t items[2] = {}, merges[2] = {};
    const void* part = nullptr;
    size_t runs[2] = {}, tiles[2] = {};
    int want = 0;
    const void* sched = nullptr;
    bool operator==(const GraphKey& o) const;
  };
  struct CachedGraph {
    GraphKey key;
    cudaGraphExec_t exec = nullptr;
    int launches = 0;
    uint64_t used = 0;
  };
  GraphKey graph_key(const Packing& p, Want want) const;
  // launch_forward through a cached CUDA graph of this packing's shape
  // (captured on first use; a few shapes are kept, least recently used
  // dropped).
  int run_forward(const Packing& p, Want want);
  std::vector<CachedGraph> graphs_;
  uint64_t graph_clock_ = 0;
  static constexpr size_t kMaxGraphs = 8;

  std::pair<size_t, std::optional<PrefixSource>> admit(const GroupIn* groups, size_t n);
  Packing pack(const GroupIn* groups, size_t n, size_t first, bool resident_first) const;
  void upload(const Packing& p, const uint8_t* per_layer_rows, size_t rows_bytes);
  int launch_forward(const Packing& p, Want want);
  void run(const GroupIn* groups, size_t n, size_t first, std::optional<PrefixSource> source,
           Want want, const uint8_t* per_layer_rows, size_t rows_bytes, float* out,
           size_t out_floats, int32_t* sources);
  void check_status();
  void prof_mark(const char* name);
  bool profiling_ = false;
  long long stall_clocks_ = 0;  // arm_wait_timeout
  std::vector<cudaEvent_t> prof_events_;
  std::vector<const char*> prof_names_;
  size_t prof_used_ = 0;
  std::pair<size_t, size_t> state_rows(int l, size_t p) const;
  SavedState save_state_at(const uint32_t* prefix, size_t n, size_t row0);
  std::optional<PrefixSource> restore_from_cache(const uint32_t* prefix, size_t n);
  void remember(const uint32_t* prefix, size_t n, size_t row0);
  std::string state_path(const uint32_t* prefix, size_t n) const;

  int device_;
  int num_sms_ = 148;
  cudaStream_t stream_ = nullptr;
  std::map<std::string, DevBuffer> lin_, norms_;
  std::map<std::string, EngineBuilder::PackedLinear> pk_;
  EngineBuilder::Packed embed_;
  std::optional<HostTensor> per_layer_table_;
  std::vector<Layer> layers_;
  const float* final_norm_ = nullptr;
  int gemm_splits_max_ = 2;
  int max_qkv_ = 0, max_attn_ = 0, max_ff_ = 0;

  // Workspace.
  DevBuffer attn_sched_, mlp_ready_;
  // Chunk-split attention partials: O [slots x kv_heads][128][256] f32 and
  // (max, sum) [slots x kv_heads][128], grown to the largest pass seen.
  DevBuffer attn_part_o_, attn_part_ml_;
  PinnedBuffer h_attn_sched_;
  CUtensorMap attn_tq_[2];             // q16 as head_dim 256 / 512 rows
  std::vector<CUtensorMap> attn_tkv_;  // per layer owning K/V
  DevBuffer ids_, meta_, row_map_, x_, x16_, h16_, qkv_, q16_, attn16_, a32_, act16_, rows_,
      logits_, status_, pl_rows16_, pli_, plp_;
  std::vector<DevBuffer> kv_;  // per layer that owns K/V: [cap_rows, 2 * kv_heads * hd] f16
  size_t cap_rows_ = 0;
  PinnedBuffer h_ids_, h_meta_, h_row_map_, h_out_, h_status_;
  DevBuffer rope_tab_[2];  // [cap_rows][128] (cos, sin): local theta, global theta
  GemmPlan pl_model_proj_;
  DevBuffer w_pl_model_proj_;

  mutable std::mutex mu_;
  std::optional<std::vector<uint32_t>> resident_;
  std::optional<PrefixSource> last_source_;
  StateCache states_;
  std::string state_dir_;
  std::string model_id_ = "wgpu";
  cudaEvent_t events_[8] = {};
};

}  // namespace omg
