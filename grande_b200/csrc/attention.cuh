// Block-causal grouped-query attention over the K/V cache
// (crates/omg-wgpu/src/shaders/attention.wgsl:1-35): a query at (pos, seq)
// sees a key of its own request group that is in the prefix or in its own
// branch, at or before its position, and within the window on sliding
// layers. Q, K and V are f16, scores and the online softmax f32.
#pragma once
#include <cuda_fp16.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <vector>

#include "kernels.cuh"

namespace omg {

// attention.wgsl:70-76 (groups: engine.rs SEQ_GROUP_SHIFT = 12): a query at
// (qp, qs) sees a key at (kp, ks) of its own request group that is a prefix
// key or in its own branch, at or before its position, within the window.
__host__ __device__ inline bool attn_visible(int qp, int qs, int kp, int ks, int window) {
  const bool same_group = ((ks ^ qs) >> 12) == 0;
  return same_group && ((ks & 0xfff) == 0 || ks == qs) && kp <= qp &&
         (window == 0 || static_cast<unsigned>(qp - kp) < static_cast<unsigned>(window));
}

// ---- tensor-core (tcgen05) kernel, head_dim 256 and 512 ---------------------
//
// A run is up to 128 / (heads per KV head) consecutive query tokens of one
// request group: 128 query rows (the tokens x the query heads sharing one KV
// head). One CTA per (run, KV head; head_dim 512: and 256-dim half of V)
// visits, with an online softmax, every
// 64-key tile that any of its rows sees; tiles sit on a grid anchored at the
// group's first cache row, so a token meets its keys in the same tiles
// whatever else shares the pass.

constexpr int kAttnTileRows = 128;  // query rows per run
constexpr int kAttnTileKeys = 64;   // keys per tile

struct AttnFlashRun {
  int tok0, ntok;       // workspace tokens of the run
  int tile0, ntiles;    // its key tiles: tiles[tile0 .. tile0 + ntiles)
};

// A run's key tiles are split into chunks of kAttnChunkTiles grid tiles,
// counted from the group's first cache row (so a token's chunks do not
// depend on what shares its run). One CTA per (item, KV head): a run whose
// tiles fall in one chunk writes its output directly (slot -1); a run that
// spans several writes, per chunk, the unnormalised O (f32) and the row's
// (reference max, sum) to a partial slot, and a merge combines the chunks in
// order. The chain of dependent key tiles per CTA is at most a chunk.
constexpr int kAttnChunkTiles = 3;

// Parts of a pass's staged attention schedule: the visibility intervals,
// then per window (sliding, global) runs, tiles, items and merges.
constexpr int kAttnSchedParts = 9;
constexpr int attn_sched_part(int window_kind, int what) { return 1 + 4 * window_kind + what; }

struct AttnFlashItem {
  int run;      // index into the runs
  int t0, nt;   // tiles[run.tile0 + t0 .. + nt)
  int slot;     // partial slot (x kv_heads + KV head), or -1: final output
};

struct AttnFlashMerge {
  int run;
  int slot0;    // its chunk c sits in slot slot0 + c
  int nchunks;
};

struct AttnFlashArgs {
  const int4* vis;       // per workspace token: visible cache rows [x, y) U [z, w), no window
  const TokMeta* meta;   // cache-row order
  const AttnFlashRun* runs;
  const int* tiles;      // first cache row of each key tile
  int n_runs;
  const AttnFlashItem* items;
  int n_items;
  const AttnFlashMerge* merges;
  int n_merges;
  float* part_o;         // [slot x kv_heads][128 rows][hd] unnormalised O
  float2* part_ml;       // [slot x kv_heads][128 rows] (reference max, row sum)
  __half* out;           // [t, heads * hd] f16
  uint32_t* status;      // device status word (bounded waits)
  int t, base, heads, kv_heads, hpg, window;
  int hd = 256;          // head_dim: 256 or 512
};

// Per workspace token (metadata `meta_ws` = cache rows base..base+t) the
// cache rows it may see before any window: its group's prefix rows up to
// itself (prefix tokens) or all of them (branch tokens), and its own branch's
// rows up to itself. Derived from the packing's metadata alone.
void attention_intervals(const TokMeta* meta_ws, int t, int base, std::vector<int4>* vis);

// Check attention_intervals against attn_visible for every (query, key)
// pair; `meta_all` covers cache rows 0..base+t. Returns false on the first
// disagreement (a packing the interval form does not describe).
bool attention_check_intervals(const TokMeta* meta_all, int t, int base, const int4* vis,
                               int window);

// Runs of a pass, their key tiles, and the CTA items / merges of the chunk
// split for one window (0 = global). Returns the partial slots used.
int attention_flash_runs(const TokMeta* meta_ws, const int4* vis, int t, int hpg, int window,
                         std::vector<AttnFlashRun>* runs, std::vector<int>* tiles,
                         std::vector<AttnFlashItem>* items, std::vector<AttnFlashMerge>* merges);

// Tensor maps of the tensor-core kernel: q16 [t_cap][heads * hd] f16 and one
// layer's K/V cache [rows_cap][2 * kv_heads * hd] f16 (64-key boxes); hd 256
// or 512.
bool attention_map_q(CUtensorMap* m, const void* q16, int t_cap, int heads, int kv_heads, int hd,
                     char* err, size_t errlen);
bool attention_map_kv(CUtensorMap* m, const void* kv, int rows_cap, int kv_heads, int hd,
                      char* err, size_t errlen);

// `p_lo`: also feed what f16 rounding dropped from P (a second P.V product),
// so P carries ~22 bits instead of f16's 11.
void launch_attention_flash(const CUtensorMap& tq, const CUtensorMap& tkv,
                            const AttnFlashArgs& a, bool p_lo, cudaStream_t s);

// Combine the chunk partials of the split runs (after launch_attention_flash,
// when a.n_merges > 0): per row, out = sum_c w_c O_c / sum_c w_c l_c with
// w_c = exp(m_c - max_c m_c), chunks in order.
void launch_attention_merge(const AttnFlashArgs& a, cudaStream_t s);

// Dynamic shared memory the attention kernels need (set once per device).
// Shared-memory limits of the attention kernels on the current device.
void attention_setup_device();

}  // namespace omg
