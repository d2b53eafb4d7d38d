// Row kernels of the decoder pass: everything but the GEMMs and attention.
// All are HBM-bound row sweeps (one CTA per token row) fused so each row of
// the residual stream is read and written once per step.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace omg {

// Weight storage (model.rs:338-371 Dtype): F16 = 0, Q8 = 1, Q4 = 2.
enum Dtype : int { kF16 = 0, kQ8 = 1, kQ4 = 2 };

// Per-token metadata in cache-row order (engine.rs:1519-1571): position,
// sequence id, first key row of its group, own row + 1.
struct TokMeta {
  int pos, seq, row_lo, row_hi;
};

// Dequantize a [rows, k] weight (QTensor::get, model.rs:508-525) into f16
// rows of `out` (row stride k). Row r lands at out row `remap(r)`:
// remap 0 = identity; 1 / 2 = the gate / up half of the interleaved GeGLU
// layout (256-row blocks: 128 gate rows, then the 128 up rows of the same
// output columns).
// The lm_head's in-shared-memory decoder over a whole table of n values:
// hi = f16(w), lo = w - hi (f16), row-major (test entry point).
void launch_table_hilo(int dtype, const void* codes, const void* scales, size_t n, __half* hi,
                       __half* lo, cudaStream_t s);
void launch_dequant_f16(int dtype, const void* codes, const void* scales, int rows, int k,
                        int remap, __half* out, cudaStream_t s);

// x[t] = dequant(embed[ids[t]]) * scale (embed.wgsl), then
// h16[t] = f16(x[t] * rsqrt(mean x^2 + eps) * (offset + w)) (rmsnorm.wgsl
// with residual = 0): the embedding and layer 0's input norm in one sweep.
// x16 (optional) gets f16(x) for the per-layer-input projection.
void launch_embed_norm(int dtype, const int* ids, int t, const void* codes, const void* scales,
                       int d, float scale, const float* w, float eps, float offset, float* x,
                       __half* x16, __half* h16, int ldh, cudaStream_t s);

// The residual-stream norm of rmsnorm.wgsl with residual = 1 and `second`:
// a = sum of `splits` slabs of the projection output (fixed order), then
// x = (x + a * rsqrt(mean a^2 + eps) * (offset + w1)) * out_scale and, when
// w2 is set, y = x * rsqrt(mean x^2 + eps) * (offset + w2) goes to h16 (f16)
// and, for rows with row_map[t] >= 0, to rows_out[row_map[t]] (f32).
// x16 (optional) gets f16(x) after the update (the per-layer gate reads it).
void launch_residual_norm(const float* a, int splits, size_t split_stride, int lda, int t, int d,
                          const float* w1, float eps, float offset, float out_scale, float* x,
                          __half* x16, const float* w2, __half* h16, int ldh,
                          const int* row_map, float* rows_out, cudaStream_t s);

// pl_combine.wgsl: per (token, layer) slice of P:
// out = (RMSNorm(proj * proj_scale; w) + emb * emb_scale) * out_scale,
// emb the gathered per-layer token rows (f16), all [t][layers * P].
void launch_pl_combine(const float* proj, int t, int P, int layers, const float* w,
                       const __half* emb, float eps, float offset, float proj_scale,
                       float emb_scale, float out_scale, float* out, cudaStream_t s);

// pl_gate.wgsl: out16[t, j] = f16(gelu_tanh(g[t, j]) * pli[t, layer * P + j]).
void launch_pl_gate(const float* g, const float* pli, int t, int P, int layers, int layer,
                    __half* out16, cudaStream_t s);

// qk_prep.wgsl: per token on the fused projection row [q heads | k heads |
// v heads]: RMSNorm each q and k head (q_norm / k_norm weights), RoPE the
// first rope_dims dims, q times q_scale into q16 [t, heads * hd]; k and the
// (optionally RMS-normalized) v heads into the K/V cache at row base + t as
// f16 [row][kv_heads * hd K | kv_heads * hd V].
struct QkArgs {
  const float* qkv;
  int q_stride;
  int splits;
  size_t split_stride;
  int t, heads, kv_heads, hd, has_kv, v_norm, rope_dims;
  float theta, q_scale, eps, offset;
  const float* qn;
  const float* kn;
  const TokMeta* meta;
  int base;
  __half* q16;
  __half* kv;
};
void launch_qk_prep(const QkArgs& a, cudaStream_t s);

// tab[dd * n_pos + pos] = (cos, sin) of qk_prep's RoPE angle
// pos * theta^(-dd / half) for pos < n_pos: the table the fused QKV GEMM
// epilogue (gemm.cuh kEpiQkPrep) reads.
void launch_rope_table(float theta, int half, int n_pos, float2* tab, cudaStream_t s);

// logits.wgsl + the host softcap (engine.rs:1901-1906): out[r, v] =
// sum_k rows[r, k] * dequant(embed[v, k]) in f32, then cap * tanh(z / cap).
// Shared-memory limit of the logits kernel for row width d (once per device
// and width, before the first launch).
void logits_setup_device(int d);

// logits.wgsl: out[r, v] = rows[r] . W[v] (+ softcap). With d % 64 == 0 on
// the tensor cores (logits_tc_kernel: the packed table dequantized into
// shared memory, f16 hi + lo splits), otherwise on the CUDA cores. `status`
// takes the tensor-core kernel's bounded-wait errors.
void launch_logits(int dtype, const float* rows, int nrows, const void* codes, const void* scales,
                   int vocab, int d, float softcap, float* out, int num_sms, uint32_t* status,
                   cudaStream_t s);

// Copy K/V cache rows for a state save / restore: contiguous f16 rows.
// (Plain cudaMemcpyAsync; kept here for symmetry with the kernels.)

}  // namespace omg
