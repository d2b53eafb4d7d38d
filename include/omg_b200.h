/*
 * omg_b200: C ABI of the B200 engine for the omg decision forward pass.
 *
 * This is the boundary a host-language shim binds: the reference's Rust
 * `omg_wgpu` crate would wrap it in an `extern "C"` block and keep its own
 * API (EngineBuilder / Engine / SavedState / WgpuBackend) on top. Every
 * entry point takes plain pointers and sizes, returns
 * 0 on success and -1 on error, and leaves a message for omg_last_error()
 * (thread-local, valid until the next call on the same thread). Outputs are
 * caller-allocated; nothing is written to them on error. Calls on one engine
 * must not overlap (the reference's Engine is driven from one thread too);
 * engines on different devices may be driven from different threads.
 *
 * Each declaration names the reference interface it replaces, as
 * `path:line` within github.com/bokuweb/omg.
 */
#ifndef OMG_B200_H
#define OMG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Weight storage types, numbered as model::Dtype::code
 * (crates/omg-wgpu/src/model.rs:357-363). Quantized tensors are 32-element
 * blocks with the codes in one buffer and the f16 block scales in another
 * (model.rs:330-337). */
enum { OMG_DTYPE_F16 = 0, OMG_DTYPE_Q8 = 1, OMG_DTYPE_Q4 = 2 };

/* omg_core::Want (crates/omg-core/src/backend.rs:15-20). */
enum { OMG_WANT_LOGITS = 0, OMG_WANT_HIDDEN = 1 };

/* omg_core::PrefixSource (crates/omg-core/src/backend.rs:95-104); NONE when
 * no pass has run yet. */
enum {
  OMG_SOURCE_NONE = -1,
  OMG_SOURCE_RESIDENT = 0,
  OMG_SOURCE_RAM = 1,
  OMG_SOURCE_DISK = 2,
  OMG_SOURCE_DECODED = 3
};

/* GEMM epilogues exposed to the kernel tests. */
enum { OMG_EPI_F32 = 0, OMG_EPI_GEGLU_TANH = 1, OMG_EPI_GEGLU_ERF = 2, OMG_EPI_F16 = 3 };

typedef struct omg_builder omg_builder;
typedef struct omg_engine omg_engine;
typedef struct omg_state omg_state;

/* omg_core::BranchTokens (crates/omg-core/src/backend.rs:26-30): one
 * question branch, its token ids and the branch-relative positions whose
 * rows are wanted, ascending. */
typedef struct {
  const int32_t* tokens;
  size_t n_tokens;
  const size_t* want;
  size_t n_want;
} omg_branch;

/* omg_wgpu::Group (crates/omg-wgpu/src/engine.rs:26-38): a prefix and the
 * branches that continue from it. */
typedef struct {
  const uint32_t* prefix;
  size_t n_prefix;
  const omg_branch* branches;
  size_t n_branches;
} omg_group;

typedef struct {
  int d;             /* Config::d (n_embd, backend.rs:130) */
  int vocab;         /* Config::vocab (n_vocab, backend.rs:132) */
  int layers;
  int embed_dtype;   /* Engine::embed_dtype (engine.rs:2163-2166) */
  int per_layer_dim; /* Config::per_layer_dim */
  int device;
  size_t capacity;   /* Engine::capacity (engine.rs:454) */
  size_t max_rows;   /* Engine::max_rows (engine.rs:456) */
  uint32_t bos;      /* Config::bos (backend.rs:128) */
} omg_engine_info;

/* The message of the last failed call on this thread ("" if none). */
const char* omg_last_error(void);

/* Library version string. */
const char* omg_version(void);

/* Number of visible CUDA devices (0 when none). */
int omg_device_count(void);

/* Page-locked host memory for output buffers (no reference counterpart: a
 * B200-side addition), allocated with `device` current so that no other
 * device gets a context. The evaluate calls detect such a buffer and copy
 * the rows into it straight from the device, skipping the staging copy that
 * a pageable buffer needs. omg_host_free releases it (NULL is a no-op). */
int omg_host_alloc(int device, size_t bytes, void** out);
void omg_host_free(void* p);

/* ---- model configuration -------------------------------------------------- */

/* Config::from_json + Config::validate (model.rs:66-254). Writes a one-line
 * summary into `summary` (may be NULL). */
int omg_config_check(const char* config_json, char* summary, size_t cap);

/* Config::tensors (model.rs:277-314): "name d0,d1\n" per catalogued tensor,
 * in catalogue order. *needed gets the buffer size required. */
int omg_config_tensors(const char* config_json, char* buf, size_t cap, size_t* needed);

/* ---- EngineBuilder (crates/omg-wgpu/src/engine.rs:805-1334) -------------- */

/* EngineBuilder::new (engine.rs:845-869) on CUDA device `device`. */
int omg_builder_new(const char* config_json, int device, omg_builder** out);

/* EngineBuilder::push (engine.rs:888-933) of a QTensor (model.rs:376-384):
 * payload bytes and, for Q8/Q4, the f16 block scales. */
int omg_builder_push(omg_builder* b, const char* name, int dtype, const int64_t* shape, int ndim,
                     const void* data, size_t nbytes, const void* scales, size_t scales_nbytes);

/* How Q4_0 / Q8_0 linears pushed after this call are kept on the device
 * (the reference keeps them packed and decodes per use, weight.wgsl:29-54):
 * OMG_WEIGHTS_PACKED keeps the packed blocks (18 / 34 bytes per 32 weights)
 * and decodes them per tile in shared memory inside the tensor-core GEMMs;
 * OMG_WEIGHTS_F16 (the default) decodes each once at push into f16 rows
 * (3.6x / 1.9x the memory, no per-tile decode, faster). Both give the same
 * results bit for bit. */
#define OMG_WEIGHTS_PACKED 0
#define OMG_WEIGHTS_F16 1
int omg_builder_set_weight_layout(omg_builder* b, int layout);

/* EngineBuilder::set_per_layer_table (engine.rs:938-949). */
int omg_builder_set_per_layer_table(omg_builder* b, int dtype, const int64_t* shape, int ndim,
                                    const void* data, size_t nbytes, const void* scales,
                                    size_t scales_nbytes);

/* EngineBuilder::missing (engine.rs:874-885): newline-separated names. */
int omg_builder_missing(omg_builder* b, char* buf, size_t cap, size_t* needed);

/* EngineBuilder::finish (engine.rs:952-1334). Consumes the builder (it is
 * freed whether or not this succeeds). */
int omg_builder_finish(omg_builder* b, size_t capacity, size_t max_rows, omg_engine** out);

/* Free a builder that was not finished. */
void omg_builder_free(omg_builder* b);

/* ---- Engine (crates/omg-wgpu/src/engine.rs:449-2171) --------------------- */

/* Engine::evaluate_groups (engine.rs:1404-1444): every group in one pass.
 * `out` receives the wanted rows in (group, branch, want) order, each row
 * `vocab` floats (OMG_WANT_LOGITS, softcapped as engine.rs:1901-1906) or `d`
 * floats (OMG_WANT_HIDDEN, the final-norm hidden state). prefix_sources
 * (may be NULL) gets one OMG_SOURCE_* per group. */
int omg_engine_evaluate_groups(omg_engine* e, const omg_group* groups, size_t n_groups, int want,
                               float* out, size_t out_floats, int32_t* prefix_sources);

/* Engine::evaluate (engine.rs:1386-1398): one group. */
int omg_engine_evaluate(omg_engine* e, const uint32_t* prefix, size_t n_prefix,
                        const omg_branch* branches, size_t n_branches, int want, float* out,
                        size_t out_floats);

/* Engine::evaluate_rows (engine.rs:1449-1463): per-layer embedding rows
 * supplied by the caller (f16 LE, [tokens][layers x P], with or without the
 * prefix rows). */
int omg_engine_evaluate_rows(omg_engine* e, const uint32_t* prefix, size_t n_prefix,
                             const omg_branch* branches, size_t n_branches, int want,
                             const void* per_layer_rows, size_t rows_bytes, float* out,
                             size_t out_floats);

/* Engine::warmup (engine.rs:1341-1352). */
int omg_engine_warmup(omg_engine* e);

/* Engine::prefix_source (engine.rs:2153-2156): OMG_SOURCE_* of the last pass. */
int omg_engine_prefix_source(omg_engine* e);

/* Engine::is_resident (engine.rs:2146-2150): 1 or 0. */
int omg_engine_is_resident(omg_engine* e, const uint32_t* prefix, size_t n);

/* Engine::evict_resident (engine.rs:2158-2161). */
void omg_engine_evict_resident(omg_engine* e);

/* Engine::set_state_cache (engine.rs:1945-1955): RAM LRU of `bytes` and,
 * when `dir` is non-empty, one GRWS1 file per state in it. */
int omg_engine_set_state_cache(omg_engine* e, size_t bytes, const char* dir,
                               const char* model_id);

/* Engine::save_state (engine.rs:1977-1981): the resident prefix's K/V rows as
 * f16. Free the state with omg_state_free. */
int omg_engine_save_state(omg_engine* e, const uint32_t* prefix, size_t n, omg_state** out);

/* Engine::restore_state (engine.rs:2051-2092): the prefix becomes resident. */
int omg_engine_restore_state(omg_engine* e, const omg_state* s);

/* A state moved between GPUs without a host copy (extends Engine::save_state /
 * restore_state, engine.rs:1977-2092, which the reference runs on one device):
 * the image is save_state's layer payloads (f16 K/V rows, sliding layers
 * window-only) concatenated in layer order, in device memory of the engine's
 * GPU, so one NCCL broadcast can hand a prefill to the GPUs that run the rest
 * of its branches. state_image_bytes: the image size of an n-token state.
 * export: the prefix must be resident; the copy is complete on return.
 * import: the prefix becomes resident, as after restore_state; the caller
 * makes sure whatever wrote `src` (a collective on another stream) is done. */
size_t omg_engine_state_image_bytes(omg_engine* e, size_t n);
int omg_engine_export_state_device(omg_engine* e, const uint32_t* prefix, size_t n, void* dst,
                                   size_t cap);
int omg_engine_import_state_device(omg_engine* e, const uint32_t* prefix, size_t n,
                                   const void* src, size_t nbytes);

/* Engine::gather_per_layer (engine.rs:1370-1381) with the engine's table:
 * f16 LE rows for `ids`, n * layers * P * 2 bytes. */
int omg_engine_gather_per_layer(omg_engine* e, const uint32_t* ids, size_t n, uint8_t* out,
                                size_t cap);

/* Config / capacity of the engine (the pub fields of engine.rs:449-457). */
int omg_engine_get_info(omg_engine* e, omg_engine_info* info);

/* Timing hook for benchmarks (no reference counterpart; the reference's
 * OMG_WGPU_PROFILE timestamps, engine.rs:643-726, serve the same purpose):
 * upload the request once, then launch the full forward `iters` times on the
 * engine's stream between two CUDA events. `resident` = 1 runs only the
 * branches over the resident first prefix. *ms gets the total time,
 * *launches the kernel launches of one pass. */
int omg_engine_time_forward(omg_engine* e, const omg_group* groups, size_t n_groups, int want,
                            int resident, int iters, float* ms, int* launches);

/* Per-kernel device time of `iters` full passes of the request (the role of
 * the reference's OMG_WGPU_PROFILE per-dispatch timestamps,
 * engine.rs:643-726 and :1778-1795): CUDA events between launches on the
 * engine's stream. Writes JSON {"kernel": [launches, total_ms], ...}. */
int omg_engine_profile_forward(omg_engine* e, const omg_group* groups, size_t n_groups, int want,
                               int resident, int iters, char* json, size_t cap, size_t* needed);

/* CUDA events on the engine's stream (slots 0..5) for end-to-end timing of
 * API calls: record, then the elapsed milliseconds between two slots. */
int omg_engine_record_event(omg_engine* e, int slot);
int omg_engine_elapsed_ms(omg_engine* e, int a, int b, float* ms);

/* Drop the engine and everything it holds on the device. */
void omg_engine_destroy(omg_engine* e);

/* ---- SavedState (crates/omg-wgpu/src/engine.rs:503-580) ------------------ */

/* SavedState::byte_len (engine.rs:510-512). */
size_t omg_state_byte_len(const omg_state* s);

/* SavedState::to_bytes (engine.rs:516-534): the GRWS1 file image. With
 * buf == NULL only *needed is set. */
int omg_state_to_bytes(const omg_state* s, const char* model_id, uint8_t* buf, size_t cap,
                       size_t* needed);

/* SavedState::from_bytes (engine.rs:536-579). */
int omg_state_from_bytes(const uint8_t* bytes, size_t n, const char* model_id, omg_state** out);

/* The state's prefix tokens (*n gets the count). */
int omg_state_prefix(const omg_state* s, uint32_t* buf, size_t cap, size_t* n);

void omg_state_free(omg_state* s);

/* state_key (engine.rs:625-641): FNV-1a of (model id, prefix), the on-disk
 * state file name. */
uint64_t omg_state_key(const char* model_id, const uint32_t* prefix, size_t n);

/* ---- tensors (crates/omg-wgpu/src/model.rs:395-525) ---------------------- */

/* QTensor::from_f32 / quantize_q8 / quantize_q4 (model.rs:395-466): codes
 * get 2n (f16), n (Q8) or n/2 (Q4) bytes, scales n/16 bytes (Q8 / Q4 only,
 * n a multiple of 32; f16 takes any n and no scales). */
int omg_quantize(int dtype, const float* values, size_t n, uint8_t* codes, uint8_t* scales);

/* QTensor::get over every element (model.rs:508-525). */
int omg_dequantize(int dtype, const uint8_t* codes, const uint8_t* scales, size_t n, float* out);

/* Seeded N(mean, std) values for synthetic checkpoints (no reference
 * counterpart: the reference's tests draw uniform values,
 * crates/omg-wgpu/tests/reference.rs:17-38; this uses the same xorshift64
 * seeded with FNV-1a(name) ^ seed, through Box-Muller). */
int omg_synth_normal(uint64_t seed, const char* name, float mean, float stddev, float* out,
                     size_t n);

/* ---- kernel-level entry points (parity tests) ------------------------------
 * Host buffers in and out; each call allocates its own device memory.
 */

/* Y = X * W^T on the tcgen05 GEMM: X [m, k] f16 (row stride lda), W [w_rows, k]
 * f16. epi OMG_EPI_F32 writes f32 [m, ldo] (split-K slabs summed on the host),
 * OMG_EPI_F16 writes f16 [m, ldo], the GeGLU epilogues expect W rows
 * interleaved in 256-row blocks [128 gate | 128 up] and write f16
 * act = gelu(g) * u for n_out columns. bn = 0 picks the engine's tiling;
 * bn = 512 runs the CTA-pair kernel (256 x 256 tiles over two SMs).
 * Replaces crates/omg-wgpu/src/shaders/matmul.wgsl:1-9 and
 * matmul_gated.wgsl:1-7 (the tests of crates/omg-wgpu/tests/matmul.rs:201-290). */
int omg_debug_gemm(int device, const uint16_t* x_f16, int m, int k, int lda, const uint16_t* w_f16,
                   int w_rows, int n_out, int epi, int bn, int splits, void* out, int ldo);

/* The fused FFN launch (matmul_gated.wgsl then matmul.wgsl for mm_gate_up /
 * mm_down, engine.rs:1253-1273): act = gelu_tanh(X Wg^T) * (X Wu^T) f16
 * [m, ff], Y = act Wd^T f32 [m, d]. X [m, d] f16; W_up [2 ff, d] f16 with gate
 * and up rows interleaved in 256-row blocks [128 gate | 128 up]; W_down
 * [d, ff] f16. pair = 1 runs it on CTA pairs (tcgen05 cta_group::2), 0 on
 * one-CTA tiles. Needs d % 128 == 0 and ff % d == 0. */
int omg_debug_mlp(int device, const uint16_t* x, int m, int d, const uint16_t* w_up, int ff,
                  const uint16_t* w_down, int pair, uint16_t* act_out, float* y_out);

/* Block-causal GQA attention (replaces crates/omg-wgpu/src/shaders/attention.wgsl:1-35):
 * q [t, heads * hd] f16 for cache rows base..base+t, kv [base + t, 2 * kv_heads * hd]
 * f16 (K heads then V heads per row), meta 4 ints per cache row (position,
 * sequence id, first key row of its group, own row + 1; engine.rs:1519-1571),
 * window 0 = global, hd 256 or 512 (the tcgen05 kernel either way). p_lo:
 * also feed P's f16 rounding residue into P.V. Writes out [t, heads * hd]
 * f16. */
int omg_debug_attention(int device, const uint16_t* q, const uint16_t* kv, const int32_t* meta,
                        int t, int base, int heads, int kv_heads, int hd, int window, int p_lo,
                        uint16_t* out);
/* The same launch (and merge) timed: `iters` runs after one untimed run,
 * *ms the average per run (CUDA events). */
int omg_debug_attention_time(int device, const uint16_t* q, const uint16_t* kv,
                             const int32_t* meta, int t, int base, int heads, int kv_heads, int hd,
                             int window, int p_lo, int iters, float* ms);

/* omg_debug_gemm and omg_debug_mlp over weights kept packed as Q4_0 / Q8_0
 * (wdtype 2 / 1; codes and f16 scales as omg_builder_push takes them, W rows
 * as the f16 entry points take them): the kernels decode each K step's
 * blocks into the f16 tile in shared memory, as weight.wgsl:29-54 decodes
 * per use, so the results equal the f16 entry points' on f16(QTensor::get)
 * bit for bit. bn = 512 (and pair = 1) run the CTA-pair kernels, each CTA
 * decoding its half of the weight tile. */
int omg_debug_gemm_q(int device, const uint16_t* x_f16, int m, int k, int lda, int wdtype,
                     const uint8_t* w_codes, const uint8_t* w_scales, int w_rows, int n_out,
                     int epi, int bn, int splits, void* out, int ldo);
int omg_debug_mlp_q(int device, const uint16_t* x, int m, int d, int wdtype,
                    const uint8_t* up_codes, const uint8_t* up_scales, int ff,
                    const uint8_t* down_codes, const uint8_t* down_scales, int pair,
                    uint16_t* act_out, float* y_out);

/* Bit-exact checks of the device dequantization (model.rs:508-525
 * QTensor::get; weight.wgsl:29-54 decodes the same blocks per use). mode 0:
 * the load-time decoder the engine runs on each pushed linear, hi [rows, k]
 * = f16(QTensor::get); mode 1: the lm_head's in-shared-memory decoder
 * (logits.wgsl:21-55 reads the table in f32), hi = f16(w) and lo = w - hi in
 * f16, so hi + lo == w exactly. codes / scales as omg_builder_push takes them. */
int omg_debug_dequant(int device, int dtype, const uint8_t* codes, const uint8_t* scales,
                      int rows, int k, int mode, uint16_t* hi, uint16_t* lo);

/* The f16 values an engine's projection GEMMs multiply for linear `name`
 * (blk.N.qkv, .o, .gate, .up, .down, ...), [rows, k] row-major, read back
 * from the device: the weight EngineBuilder::push received
 * (crates/omg-wgpu/src/engine.rs:845-952), as the GEMM sees it. */
int omg_engine_weight_f16(omg_engine* e, const char* name, uint16_t* out, size_t n);

/* Test hook for the bounded device waits (no counterpart in the reference,
 * whose GPU path has no waits of its own): the engine's next pass arms its
 * first fused FFN launch to wait for an activation band that never
 * completes, so that wait gives up after `clocks` SM clocks; the pass then
 * fails with "a kernel gave up waiting" and the engine keeps working. */
int omg_engine_arm_wait_timeout(omg_engine* e, long long clocks);

/* Kernel timing for tile sweeps (no reference counterpart; the reference
 * times dispatches with timestamp queries, crates/omg-wgpu/src/engine.rs:643-726):
 * `iters` launches of the GEMM on device-resident operands of the given shape
 * (bn = 0 picks the engine's tiling), CUDA events around them; *ms gets the
 * average per launch. */
int omg_debug_gemm_time(int device, int m, int n, int k, int epi, int bn, int splits, int iters,
                        float* ms);
/* The same over packed Q4_0 / Q8_0 weights (wdtype 2 / 1), and the fused FFN
 * launch of an [m, d] x ff layer (wdtype 0: f16 weights; pair 1: CTA pairs):
 * average ms per launch. */
int omg_debug_gemm_time_q(int device, int m, int n, int k, int epi, int bn, int splits,
                          int wdtype, int iters, float* ms);
int omg_debug_mlp_time(int device, int m, int d, int ff, int wdtype, int pair, int iters,
                       float* ms);

/* ---- Laya / ModernBERT encoder (crates/omg-wgpu/src/laya.rs) ---------------
 * The encoder behind omg_core::Decider (crates/omg-core/src/engine.rs:70-93,
 * via LayaBackend, crates/omg-wgpu/src/laya/backend.rs:139). */

typedef struct omg_laya_builder omg_laya_builder;
typedef struct omg_laya_engine omg_laya_engine;

/* laya::Sequence (laya.rs:469-476): one question's token ids, the token
 * index of each option's [MASK] in option order, and its question type
 * (0 choice, 1 score, 2 noul). */
typedef struct {
  const uint32_t* ids;
  size_t n_ids;
  const size_t* markers;
  size_t n_markers;
  int qtype;
} omg_laya_sequence;

/* config_from_export + LayaConfig::from_json / validate (laya.rs:88-230,
 * 312-323): the exported config.json (encoder config, `laya_agent`,
 * `laya_tokens`). The reference resolves the special tokens' surface forms
 * with its tokenizer; the caller passes that map as `laya_special_ids`
 * ({"[CLS]": id, ...}) in the same object. One-line summary into `summary`. */
int omg_laya_config_check(const char* config_json, char* summary, size_t cap);

/* LayaConfig::tensors (laya.rs:252-309): "name d0,d1\n" per tensor. */
int omg_laya_config_tensors(const char* config_json, char* buf, size_t cap, size_t* needed);

/* LayaBuilder::new (laya.rs:623-645) on CUDA device `device`. */
int omg_laya_builder_new(const char* config_json, int device, omg_laya_builder** out);

/* LayaBuilder::push (laya.rs:662-708). */
int omg_laya_builder_push(omg_laya_builder* b, const char* name, int dtype, const int64_t* shape,
                          int ndim, const void* data, size_t nbytes, const void* scales,
                          size_t scales_nbytes);

/* LayaBuilder::missing (laya.rs:651-660): newline-separated names. */
int omg_laya_builder_missing(omg_laya_builder* b, char* buf, size_t cap, size_t* needed);

/* LayaBuilder::finish (laya.rs:711-1084): `capacity` packed tokens,
 * `max_rows` read-back rows (one per sequence plus one per marker).
 * Consumes the builder. */
int omg_laya_builder_finish(omg_laya_builder* b, size_t capacity, size_t max_rows,
                            omg_laya_engine** out);

void omg_laya_builder_free(omg_laya_builder* b);

/* LayaEngine::warmup (laya.rs:1126-1134). */
int omg_laya_warmup(omg_laya_engine* e);

/* LayaEngine::hidden (laya.rs:1138-1432): per sequence the [CLS] row then
 * each marker's row, d floats each, in sequence order. */
int omg_laya_hidden(omg_laya_engine* e, const omg_laya_sequence* seqs, size_t n, float* out_rows,
                    size_t out_floats);

/* LayaEngine::evaluate (laya.rs:1435-1438) = hidden + the scorer and act
 * head (laya.rs:1442-1486; f32, run on the device here, so only the logits
 * and act probabilities cross PCIe): out_logits gets each sequence's option
 * logits back to back (sum of n_markers floats), out_act (n floats, may be
 * NULL) the act probability, NaN without an act head. */
int omg_laya_evaluate(omg_laya_engine* e, const omg_laya_sequence* seqs, size_t n,
                      float* out_logits, size_t logits_cap, float* out_act);

/* LayaEngine::probabilities (laya.rs:1489-1493). */
int omg_laya_probabilities(omg_laya_engine* e, int qtype, const float* logits, size_t k,
                           double* out);

/* Device-resident timing and per-kernel profile (no reference counterpart
 * beyond OMG_WGPU_PROFILE, engine.rs:643-726): as omg_engine_time_forward /
 * omg_engine_profile_forward. */
int omg_laya_time_forward(omg_laya_engine* e, const omg_laya_sequence* seqs, size_t n, int iters,
                          float* ms, int* launches);
int omg_laya_profile_forward(omg_laya_engine* e, const omg_laya_sequence* seqs, size_t n,
                             int iters, char* buf, size_t cap, size_t* needed);
int omg_laya_record_event(omg_laya_engine* e, int slot);
int omg_laya_elapsed_ms(omg_laya_engine* e, int a, int b, float* ms);

void omg_laya_destroy(omg_laya_engine* e);

/* ---- allocation-free entry point -------------------------------------------
 * No counterpart in the reference. For callers that own every device buffer
 * and cannot let a library allocate (their own memory pool, or code where an
 * allocation would synchronise the device): Y = X * W^T with split-K on the
 * tcgen05 GEMM, all pointers device memory of the caller — X [m, k] f16
 * (row stride lda), W [n, k] f16, out [m, ldo] f32 — `stream` a cudaStream_t
 * or NULL. The partial slabs and the status word live in a file-scope
 * __device__ array of 32 MiB (held on every GPU that loads the library), so
 * splits * m * round_up(n, 4) * 4 bytes must fit in 32 MiB - 256; larger
 * problems are rejected with an error. Calls that overlap on the GPU share
 * that array and race. The first call on a device looks the array up and
 * sets kernel attributes. Every call synchronises `stream` and checks the
 * status word before it returns, so it must never be called while a stream
 * capture is in progress. lda >= k and ldo >= n are required. The caller's
 * current device is left as it was. */
int omg_gemm_splitk_noalloc(int device, const void* x_f16, int m, int k, int lda,
                            const void* w_f16, int n, int splits, float* out, int ldo,
                            void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OMG_B200_H */
