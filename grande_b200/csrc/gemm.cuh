// Dense f16 GEMM on the 5th-generation tensor cores: Y = X * W^T with X
// [M, K] and W [N, K] both row-major f16 (K-major for the MMA), f32
// accumulation in tensor memory. This is the linear layer of the decoder and
// the encoder (reference: crates/omg-wgpu/src/shaders/matmul.wgsl:1-9 and
// matmul_gated.wgsl:1-7 — X rounded to f16, the dequantized weight rounded to
// f16, f32 accumulate; here the weight is dequantized once at load into the
// exact f16 values the reference produces per use).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "kernels.cuh"

namespace omg {

// What the epilogue does with the f32 accumulator tile.
enum GemmEpilogue : int {
  kEpiF32 = 0,        // store f32 rows (split-K partial `blockIdx.z` into its own slab)
  kEpiGeGluTanh = 1,  // W rows interleaved [gate 128 | up 128]: store f16 gelu_tanh(g) * u
  kEpiGeGluErf = 2,   // same with the exact (erf) GELU
  kEpiF16 = 3,        // store f16 rows
  // Encoder epilogues (GemmEpi carries their operands):
  kEpiRopeF16 = 4,      // fused [q | k | v] projection: rotate q and k heads at the row's
                        // position (rope_bi.wgsl), q times q_scale, store f16
  kEpiBiasF16 = 5,      // store f16(acc + bias)
  kEpiBiasReluF16 = 6,  // store f16(max(acc + bias, 0))
  kEpiResidF32 = 7,     // residual update in place: x = (x + acc) + bias, or
                        // (acc + bias) + x with bias_first
  // Decoder epilogue (GemmEpi::qk):
  kEpiQkPrep = 8,       // fused [q heads | k heads | v heads] projection with 256-dim heads,
                        // one 256-column tile per head: qk_prep.wgsl on the accumulator
};

// Operands of kEpiQkPrep: per row, RMSNorm each q / k head with its norm
// weights, RoPE the first rope_dims dims, q times q_scale into q16; k and the
// (optionally RMS-normalised) v heads into the K/V cache at row base + row.
struct QkEpi {
  __half* q16 = nullptr;        // [rows][heads * 256]
  __half* kv = nullptr;         // [cache rows][2 * kv_heads * 256], null without own K/V
  const TokMeta* meta = nullptr;  // cache-row order
  const float* qn = nullptr;
  const float* kn = nullptr;
  const float2* rope = nullptr;   // [128][rope_stride positions] (cos, sin)
  int rope_stride = 0;
  int base = 0, heads = 0, kv_heads = 0, rope_dims = 256, v_norm = 0, has_kv = 0;
  float q_scale = 1.f, eps = 1e-6f, offset = 0.f;
};

// Operands of the encoder epilogues.
struct GemmEpi {
  const float* bias = nullptr;   // per output column, f32
  const float2* rope = nullptr;  // [hd / 2][rope_stride positions] (cos, sin)
  int rope_stride = 0;
  const int* pos = nullptr;      // per row: its position (the rope table column)
  float q_scale = 1.f;
  int q_cols = 0;                // columns [0, q_cols) are q heads, [q_cols, 2 q_cols) k heads
  int bias_first = 0;
  QkEpi qk;
};

struct GemmShape {
  int n_out;     // valid output columns (N, or the GeGLU width)
  int k;         // reduction length (multiple of 8)
  int bn;        // MMA N tile: 128 or 256 (always 256 for GeGLU)
  int splits;    // split-K factor (f32 epilogue only)
  int epi;       // GemmEpilogue
  int n_tiles;   // grid.x
  int pair;      // CTA-pair kernel (tcgen05 cta_group::2): 0 never, 1 for passes of
                 // >= kPairMinTiles row tiles, 2 always
};

// Tensor maps and launch shape of one (activation buffer, weight) pair,
// built once when the engine wires its layers.
struct GemmPlan {
  CUtensorMap a;  // activations [rows_cap, K] f16, box 64 x 128
  CUtensorMap b;  // weights [N_rows, K] f16, box 64 x bn (f16 weights)
  CUtensorMap b_half;  // the same, box 64 x 128 (each CTA of a pair loads half a tile)
  GemmShape s;
  int rows_cap;
  int num_sms;  // persistent grid size (CTAs = min(tiles, SMs))
  int pk;       // kF16: TMA-loaded f16 weights; kQ4 / kQ8: packed chunks (packed.cuh)
  const uint8_t* wpack;  // the packed weight (pk != kF16)
};

// Build the plan. `a_rows_cap` bounds the activation rows the tensor map
// covers (the workspace capacity); `w_rows` is the weight's row count as
// stored (for GeGLU: 2 x padded width).
bool gemm_plan(GemmPlan* p, const void* a, int a_rows_cap, int lda, const void* w, int w_rows,
               int n_out, int k, int epi, int bn, int splits, char* err, size_t errlen);

// The same over a weight kept packed as Q4_0 / Q8_0 chunks (packed.cuh;
// `dtype` kQ4 or kQ8, `w_rows` the weight's rows, padded to whole chunks in
// memory): the kernels fetch each K step's chunks with a bulk copy and
// decode them into the f16 tile in shared memory, so the product is the one
// the f16 weight gives, bit for bit. Epilogues kEpiF32, kEpiF16, the GeGLUs
// and kEpiQkPrep; one-CTA and CTA-pair kernels (gemm_plan_pair).
bool gemm_plan_packed(GemmPlan* p, const void* a, int a_rows_cap, int lda, const void* wpack,
                      int dtype, int w_rows, int n_out, int k, int epi, int bn, int splits,
                      char* err, size_t errlen);

// Switch a BN-256 plan to the CTA-pair kernel: two CTAs on one TPC share a
// 256 x 256 tile, each staging its own 128 rows of A and 128 of the 256
// weight rows, so each SM moves 2/3 of the operand bytes per FLOP and keeps
// six K steps in flight. Same results as the one-CTA kernel, bit for bit
// (same K order per output element).
bool gemm_plan_pair(GemmPlan* p, const void* w, int w_rows, bool always, char* err,
                    size_t errlen);

// Row tiles from which a pass takes the CTA-pair kernel: with fewer, pairing
// 128-row tiles wastes too much of the last pair (7 tiles run as 8).
constexpr int kPairMinTiles = 16;
// The fused FFN launch takes CTA pairs from 16 row tiles too. (At an E2B
// pass's 7 tiles, run as 4 pairs, the deeper pipeline only pays for the
// empty half: 2.48 vs 2.40-2.44 ms per pass on one-CTA tiles.)
constexpr int kPairMlpMinTiles = 16;

// Packed weights take CTA pairs from as many row tiles as f16 weights do
// (each SM of a pair decodes only its half of the weight tile, but at the
// decoder's ~4 instructions per weight the pair kernels measured slower
// than one-CTA tiles on the E2B FFN: 214 vs 148 us).
constexpr int kPairMinTilesPacked = kPairMinTiles;

// Whether a launch of this plan over `m` rows takes the CTA-pair kernel.
bool use_pair(const GemmPlan& p, int m);

// Launch over `m` rows. f32 epilogue: `out` is [splits][m_stride][ldo] f32
// (slab z at out + z * split_stride). f16 epilogues: [m][ldo] f16.
void gemm_run(const GemmPlan& p, int m, void* out, int ldo, size_t split_stride,
              uint32_t* status, cudaStream_t stream);

// The same for the epilogues that take GemmEpi operands (kEpiRopeF16 ..
// kEpiQkPrep; no split-K). kEpiRopeF16 needs 64-dim heads (one 64-column pair of 32-column
// halves per head).
void gemm_run_epi(const GemmPlan& p, int m, void* out, int ldo, const GemmEpi& epi,
                  uint32_t* status, cudaStream_t stream);

// Gate+up (GeGLU epilogue into `act`) and down (f32 split slabs) of one FFN
// as one persistent launch whose down units start as soon as the up tiles
// of their columns are stored. Needs both plans at BN 256 and each down
// split reading whole up column tiles (gemm_mlp_ok). `ready` holds
// one counter per (128-row tile, down split), zeroed at the start of a pass;
// `ready_target` is the running sum over the pass's fused launches of
// 4 x (up column tiles / down splits). A down unit waits at most
// `wait_limit` SM clocks (0: about a second) for its band, then records
// kDevWaitTimeout in `status` and its CTA stops.
bool gemm_mlp_ok(const GemmPlan& up, const GemmPlan& down);
void gemm_run_mlp(const GemmPlan& up, const GemmPlan& down, int m, void* act, int ld_act,
                  void* slabs, int ld_slab, size_t split_stride, int* ready, int ready_target,
                  uint32_t* status, cudaStream_t stream, int force_pair = -1,
                  long long wait_limit = 0);

// Encode a TMA tensor map over f16 data with the 128-byte swizzle: `rank`
// dimensions innermost first, byte strides of dimensions 1..rank-1, box
// extents per dimension (the innermost box must be 64 elements = 128 bytes).
bool make_tmap_f16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides, const uint32_t* box, char* err, size_t errlen);

// Set the kernels' shared-memory limits on the current device (once per
// device, before the first launch).
void gemm_setup_device();

// Pick (bn, splits) for an f32-output GEMM of this shape on this GPU. Depends
// only on (N, K), never on M, so a row's result is the same in every pass.
void gemm_pick(int n, int k, int num_sms, int* bn, int* splits);

}  // namespace omg
