// Block-causal grouped-query attention over the K/V cache
// (crates/omg-wgpu/src/shaders/attention.wgsl:1-35): a query at (pos, seq)
// sees a key of its own request group that is in the prefix or in its own
// branch, at or before its position, and within the window on sliding
// layers. Q, K and V are f16, scores and the online softmax f32.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <vector>

#include "kernels.cuh"

namespace omg {

struct AttnArgs {
  const __half* q;      // [t, heads * hd]: workspace rows 0..t = cache rows base..base+t
  const __half* kv;     // [rows, 2 * kv_heads * hd]: K heads then V heads per cache row
  const TokMeta* meta;  // cache-row order
  __half* out;          // [t, heads * hd]
  const int2* ctas;     // per CTA: first workspace token, token count (attention_schedule)
  int n_ctas;
  // Key-range splits (head_dim 256): partials [nsplit][t][heads][256] f32 and
  // (max, sum) [nsplit][t][heads], merged by a second kernel when nsplit > 1.
  int nsplit;
  float* part_o;
  float2* part_ml;
  int t, base, heads, kv_heads, hd, window;
};

// Split the t tokens of a pass (their metadata, workspace order) into CTA
// runs of at most 64 / (heads per KV head) tokens that never cross a request
// group (groups differ in row_lo).
void attention_schedule(const TokMeta* meta, int t, int hpg, std::vector<int2>* out);

// Most key-range splits per query tile (sizes the partial buffers).
constexpr int kAttnMaxSplits = 16;

// Splits for a pass (`meta` the workspace tokens' metadata, `ctas` from
// attention_schedule): enough that every query tile's visible key tiles come
// in chunks of >= 4 tiles, at most kAttnMaxSplits. 1 = no split.
int attention_splits(const TokMeta* meta, int t, int base, int hpg,
                     const std::vector<int2>& ctas, int hd);

// Dynamic shared memory the attention kernels need (set once per device).
void attention_setup_device();

void launch_attention(const AttnArgs& a, cudaStream_t s);

}  // namespace omg
