// Kernels of the Laya / ModernBERT encoder pass (crates/omg-wgpu/src/laya.rs)
// other than its GEMMs: the embedding + embedding norm, the LayerNorms of
// the residual stream, the bidirectional attention on the tensor cores, and
// the read-back gather. The projections are gemm.cu's tcgen05 GEMM with the
// encoder epilogues (fused RoPE, bias, bias + ReLU, in-place residual add).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

namespace omg {

// rope_bi.wgsl:28-31 for every position < n_pos and pair i < hd / 2:
// angle = pos * theta^(-2i / hd), tab[i * n_pos + pos] = (cos, sin).
void launch_laya_rope_table(float theta, int hd, int n_pos, float2* tab, cudaStream_t s);

// embed.wgsl (scale 1) then layernorm.wgsl (no bias) with `w`:
// x[t] = LN(dequant(embed[ids[t]])), h16[t] = f16(x[t]). d % 128 == 0.
void launch_laya_embed_ln(int dtype, const int* ids, int t, const void* codes, const void* scales,
                          int d, const float* w, float eps, float* x, __half* h16,
                          cudaStream_t s);

// layernorm.wgsl over the residual stream x [t, d] (the residual add itself
// rides in the previous GEMM's epilogue):
//  * in_place == 0: h16 = f16(LN(x; w1, b1));
//  * in_place == 1: x = LN(x; w1, b1) (+ type_emb[qtype[t]] when type_emb),
//    then, when w2 is set, h16 = f16(LN(x; w2, b2)).
// b1 / b2 may be null (no bias). d % 128 == 0, d <= 2048.
struct LayaLnArgs {
  float* x;
  int t, d;
  float eps;
  const float *w1, *b1;
  int in_place;
  const float* type_emb;  // [3, d] f32, or null
  const int* qtype;
  const float *w2, *b2;
  __half* h16;
};
void launch_laya_ln(const LayaLnArgs& a, cudaStream_t s);

// rows[r] = x[row_map[r]] for r < n (the wanted rows, f32).
void launch_laya_gather(const float* x, int d, const int* row_map, int n, float* rows,
                        cudaStream_t s);

// ---- bidirectional attention (attention_bi.wgsl) on tcgen05 ---------------
//
// A work item is up to 128 consecutive token rows of one sequence (the whole
// sequence, or a 128-row chunk of a long one) of one head against the key
// rows they can see, visited in 128-key tiles anchored at the sequence's
// first row, with an online softmax. Because nothing in an item depends on
// the other sequences of the pass, a sequence's rows are the same bits
// whatever it is packed with.
// A query row r sees key row j iff both lie in the same sequence
// [lo_r, hi_r) and, on local layers, |r - j| <= window (positions count up
// from each sequence's first row, so the row distance is the position
// distance). Q, K, V are f16 (the rounding attention_bi.wgsl applies when it
// stages them); scores and the softmax are f32; the probabilities enter the
// P.V product as f16.
constexpr int kLayaHd = 64;
constexpr int kLayaTile = 128;

struct LayaAttnItem {
  int q0, nq;  // query rows [q0, q0 + nq)
  int k0, nk;  // key rows [k0, k0 + nk), visited 128 at a time
};

struct LayaAttnArgs {
  const LayaAttnItem* items;
  const int2* span;  // per token row: its sequence's rows [lo, hi)
  __half* out;       // [t][heads * 64] f16
  uint32_t* status;
  int n_items, heads, d, window;
  int single_tile;   // every item's keys fit one 128-key tile (nk <= 128)
  int num_sms;       // persistent grid bound
};

// Items of a pass from the per-row spans (host).
void laya_attention_items(const int2* span, int t, int window, std::vector<LayaAttnItem>* items);

// Tensor map over the fused f16 projection rows [rows_cap][3 d]
// (q heads | k heads | v heads), box 64 x 128.
bool laya_attention_map(CUtensorMap* m, const void* qkv16, int rows_cap, int d, char* err,
                        size_t errlen);

void launch_laya_attention(const CUtensorMap& tqkv, const LayaAttnArgs& a, cudaStream_t s);

// Shared-memory limits of the encoder kernels (once per device).
void laya_setup_device();

// ---- the decision head on the device (laya.rs:1442-1486) --------------------
//
// The scorer of every [MASK] row and the act head of every sequence, in f32
// on the CUDA cores, over the gathered rows (per sequence its [CLS] row
// then its marker rows). Same operations as the reference's host code; sums
// run in another order (warp trees instead of index order), so results
// agree with it to f32 reassociation.
//
// Scorer, per marker row x: z = LN(x; norm_w, norm_b) (biased variance,
// 1 / sqrt(var + eps)), y = GELU_erf(l1 z + l1_b), logit = l2 . y + l2_b.
struct LayaScoreArgs {
  const float* rows;        // [*, d]
  const int* marker_row;    // [k] row of each marker in `rows`
  int k, d;
  const float *norm_w, *norm_b, *l1, *l1_b, *l2;
  float l2_b, eps;
  float* logits;            // [k]
};
void launch_laya_score(const LayaScoreArgs& a, cudaStream_t s);

// Act head, per sequence: the softmax of its marker logits padded to at
// least two slots with -1e4 gives top1, top1 - top2 and the normalised
// entropy; u = [cls row, top1, top1 - top2, entropy, slots / 255],
// a = GELU_erf(l1 u + l1_b), p = softmax(l2 a + l2_b), act = p[0].
// hidden <= 256 (the act head's width, laya.rs:1474-1486).
struct LayaActArgs {
  const float* rows;
  const int4* seq;          // [n] (cls row, first logit, marker count, 0)
  int n, d, hidden, outs;
  const float *l1, *l1_b, *l2, *l2_b;
  const float* logits;
  float* act;               // [n]
};
void launch_laya_act(const LayaActArgs& a, cudaStream_t s);

}  // namespace omg
