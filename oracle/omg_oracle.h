/*
 * omg_oracle — TEST INFRASTRUCTURE ONLY.
 *
 * A CPU restatement, in plain C, of the reference's own CPU algorithms for the
 * omg-wgpu forward pass (github.com/bokuweb/omg, crates/omg-wgpu). It is the
 * checker the parity tests compare the CUDA engine against. Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it; the
 * product (grande_b200) never links, imports or calls it.
 *
 * Each function cites the reference file:line it restates. Pinning: the
 * quantizers are checked byte-for-byte against gguf-py 0.19's Q8_0 / Q4_0
 * quantizers as repacked by the reference's tools/export_wgpu_gguf.py, the
 * visibility rule against the reference's python/omg_train/model.py
 * branch_mask, and the decoder forward against transformers 5.5's Gemma 3
 * text model driven the way python/omg_train/model.py:67-80 drives it
 * (fixtures in tests/golden/, made by tests/golden/make_golden.py).
 */
#ifndef OMG_ORACLE_H
#define OMG_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE half <-> float, round to nearest even (the `half` crate's rules). */
uint16_t oracle_f32_to_f16(float v);
float oracle_f16_to_f32(uint16_t h);

/* Element-wise batch versions of the two conversions above. */
void oracle_f32_to_f16_n(const float* in, size_t n, uint16_t* out);
void oracle_f16_to_f32_n(const uint16_t* in, size_t n, float* out);

/* tests/reference.rs:17-26: xorshift64, uniform in [-1, 1). Fills n values
 * times `scale`, advancing *state. */
void oracle_rng_values(uint64_t* state, float* out, size_t n, float scale);
/* The synthetic models' normal draws (FNV-1a(name) ^ seed, xorshift64,
 * Box-Muller in double). */
void oracle_synth_normal(uint64_t seed, const char* name, float mean, float stddev, float* out,
                         size_t n);

/* model.rs:409-427 (Q8_0) and model.rs:431-466 (Q4_0). n is a multiple of 32;
 * codes get n (Q8) or n/2 (Q4) bytes, scales n/32 little-endian f16. */
int oracle_quantize_q8(const float* v, size_t n, uint8_t* codes, uint8_t* scales);
int oracle_quantize_q4(const float* v, size_t n, uint8_t* codes, uint8_t* scales);

/* model.rs:508-525 QTensor::get for every element. dtype 0 f16 (codes are
 * little-endian f16), 1 Q8, 2 Q4. */
int oracle_dequant(int dtype, const uint8_t* codes, const uint8_t* scales, size_t n, float* out);

/* Model description (model.rs:28-63). Per-layer arrays have `layers`
 * entries. */
typedef struct {
  int vocab, d, layers, heads, kv_heads;
  const int* head_dim;
  const int* ff;
  const int* sliding;
  const int* kv_source;
  const int* rope_dims;
  float eps;
  int window;
  float theta_global, theta_local, query_scale, norm_offset;
  int v_norm;
  int per_layer_dim;
  float softcap;
} oracle_config;

/* Rounding modes of oracle_forward. */
enum {
  ORACLE_EXACT = 0,   /* tests/reference.rs as written: all f32 */
  ORACLE_KERNEL = 1   /* the kernels' rounding points: linear inputs and weights
                         to f16 (matmul.wgsl:1-9), Q/K/V to f16 in attention
                         (attention.wgsl:80-92,110-117) */
};

/* tests/reference.rs:175-349, the plain forward over a packed sequence,
 * with the shader's visibility rule for grouped sequence ids
 * (attention.wgsl:70-76; engine.rs:21-24 SEQ_GROUP_SHIFT = 12).
 *
 * `tensors` holds dequantized f32 values of every catalogued tensor in the
 * order of Config::tensors (model.rs:277-314), followed by the per-layer
 * token table when per_layer_dim > 0. Writes the final-norm hidden state of
 * every token: hidden[t * d]. threads <= 0 uses all cores. */
int oracle_forward(const oracle_config* cfg, const float* const* tensors, size_t n_tensors,
                   const uint32_t* ids, const int32_t* pos, const int32_t* seq, size_t t,
                   int mode, int threads, float* hidden);
/* The same, and per_layer [layers][t][d] (or NULL) gets, after each layer
 * l, the final norm of the residual stream: the hidden rows of the model cut
 * after layer l. */
int oracle_forward_layers(const oracle_config* cfg, const float* const* tensors,
                          size_t n_tensors, const uint32_t* ids, const int32_t* pos,
                          const int32_t* seq, size_t t, int mode, int threads, float* hidden,
                          float* per_layer);

/* The block-causal visibility rule (attention.wgsl:70-76): 1 if a query at
 * (qp, qs) sees a key at (kp, ks) on a layer with this window (0 = global). */
int oracle_visible(int32_t qp, int32_t qs, int32_t kp, int32_t ks, int window);

/* tests/reference.rs:581-590 + engine.rs:1901-1906: logits of one hidden row
 * against the (dequantized) embedding, then softcap if > 0. */
void oracle_logits(const float* hidden, const float* embed, int vocab, int d, float softcap,
                   float* out);

/* crates/omg-core/src/math.rs:5-17: softmax of z / temperature and
 * log-sum-exp, both in f64. */
void oracle_softmax(const float* z, size_t n, float temperature, double* out);
double oracle_log_sum_exp(const float* z, size_t n);

/* ---- Laya / ModernBERT encoder (crates/omg-wgpu/src/laya.rs) ------------- */

/* LayaConfig (laya.rs:46-83), the fields the forward reads. */
typedef struct {
  int vocab, d, layers, heads, ff;
  const int* sliding; /* per encoder layer: 1 = local attention */
  int window;         /* inclusive |query pos - key pos| on local layers */
  float theta_global, theta_local, eps;
  int head_layers;
  int type_emb;
} oracle_laya_config;

/* LayaEngine::hidden's GPU plan (laya.rs:1263-1345) over a packed batch of
 * sequences: embed -> embed_norm -> per layer [Wqkv, RoPE (q * hd^-0.5),
 * bidirectional attention, Wo, x += o & mlp_norm, GeGLU(erf), Wo_mlp,
 * x += wo & next norm] -> x = final_norm(x) + type_emb[qtype] -> decision-head
 * layers. `tensors` are dequantized f32 in LayaConfig::tensors order
 * (laya.rs:265-313; trailing host tensors are ignored). pos = index within
 * the sequence, seq = sequence index. Writes the residual stream x of every
 * token (the rows the scorer reads): x_out[t * d]. Mode ORACLE_KERNEL rounds
 * linear inputs and weights to f16 and Q/K/V to f16 in attention
 * (matmul.wgsl, attention_bi.wgsl:80-90). */
int oracle_laya_hidden(const oracle_laya_config* cfg, const float* const* tensors,
                       size_t n_tensors, const uint32_t* ids, const int32_t* pos,
                       const int32_t* seq, const uint32_t* qtype, size_t t, int mode,
                       int threads, float* x_out);

/* LayaEngine::score (laya.rs:1442-1493): rows = [CLS] row then k marker
 * rows (d each). w = scorer.norm_w, scorer.norm_b, scorer.l1, scorer.l1_b,
 * scorer.l2, scorer.l2_b, act.l1, act.l1_b, act.l2, act.l2_b. Writes k
 * logits and, when act_out > 0, the act probability. */
int oracle_laya_score(const float* rows, int k, int d, float eps, const float* const* w,
                      int act_hidden, int act_out, float* logits, float* act_prob);

#ifdef __cplusplus
}
#endif

#endif /* OMG_ORACLE_H */
