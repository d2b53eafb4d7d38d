// tcgen05 GEMM: TMA-fed, single-thread-issued UMMA with the accumulator in
// tensor memory, warp-specialised (1 TMA warp, 1 MMA warp, 4 epilogue warps).
//
// Tile: 128 rows x BN (128 or 256) x 64 K per stage, 128-byte swizzled K-major
// operands in shared memory, a 4- or 6-stage mbarrier ring. One output tile
// per CTA; split-K slabs along grid.z for the narrow f32 projections so the
// grid covers the 148 SMs.
#include "gemm.cuh"
#include "launch.cuh"
#include "packed.cuh"
#include "ptx.cuh"
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstring>

namespace omg {

bool make_tmap_f16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides, const uint32_t* box, char* err, size_t errlen);

namespace {

constexpr int BM = 128;
constexpr int BK = 64;

struct GemmArgs {
  int m;             // valid rows
  int n_out;         // valid output columns
  int kb_total;      // 64-wide K blocks
  int kb_per_split;  // K blocks per split-K slab
  int m_tiles, n_tiles, splits;
  int n_fast;        // tile order: 0 = M tile fastest, 1 = N tile fastest
  void* out;
  int ldo;           // output row stride in elements
  size_t split_stride;
  uint32_t* status;
  GemmEpi epi;
  const uint8_t* wpack;  // packed weight chunks (packed kernels only)
};

// Tile t of a launch: split-major, then (m fastest) or (n fastest).
// M-fastest suits the decoder's projections (a few M tiles against a large
// weight: the CTAs running at once share weight tiles in L2); N-fastest the
// encoder's (32k rows against a weight of a few MB: each block of A rows is
// read from HBM once, by CTAs running side by side).
struct TileId {
  int m, n, split;
};
__device__ __forceinline__ TileId decode_tile(const GemmArgs& g, int t) {
  const int mn = g.m_tiles * g.n_tiles;
  const int r = t % mn;
  TileId x;
  x.split = t / mn;
  x.m = g.n_fast ? r / g.n_tiles : r % g.m_tiles;
  x.n = g.n_fast ? r % g.n_tiles : r / g.m_tiles;
  return x;
}

// PK: where the weight tile comes from. kF16: a TMA load of row-major f16
// weights. kQ4 / kQ8: packed chunks (packed.cuh) fetched by a bulk copy into
// a raw ring and decoded into the swizzled f16 tile by four converter warps.
template <int BN, int PK = kF16>
struct Cfg {
  static constexpr bool PACKED = PK != kF16;
  static constexpr int STAGES = PACKED ? (BN == 256 ? 3 : 4) : (BN == 256 ? 4 : 6);
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int CHUNK = PK == kQ4 ? PackChunk<kQ4>::BYTES
                                         : (PK == kQ8 ? PackChunk<kQ8>::BYTES : 0);
  static constexpr int RAW_BYTES = (BN / 128) * CHUNK;
  static constexpr int RAW_STAGES = !PACKED ? 0 : (PK == kQ8 && BN == 256 ? 3 : 6);
  static constexpr int RING = STAGES * STAGE_BYTES + RAW_STAGES * RAW_BYTES;
  // Ring + alignment slack + barriers, 2 KB the epilogue may stage its
  // per-column constants in (the q / k norm weights of kEpiQkPrep), and a
  // 4 KB row-staging slot per epilogue warp.
  static constexpr int SMEM = RING + 1024 + 256 + 2048 + 4 * 4096;
  // Two accumulators: the epilogue drains one while the MMAs fill the other.
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  // Warps: 0 TMA (A, and B when f16), 1 MMA, 2-5 epilogue; packed: 6 bulk
  // copies of the raw chunks, 7-10 converters.
  static constexpr int THREADS = PACKED ? 352 : 192;
  static_assert(SMEM <= 232448, "shared memory");
  static_assert(2 * STAGES + 4 + 2 * RAW_STAGES <= 30, "barrier area");
};

// Shared-memory carve-up: A ring, B ring, raw ring, then barriers, epilogue
// constants and row-staging slots (one-CTA and CTA-pair configs alike).
template <class C>
struct Smem {
  uint8_t *sa, *sb, *raw;
  uint64_t *full, *empty, *tfull, *tempty, *raw_full, *raw_empty;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
  float* epi_consts;
  uint8_t* slots;
  __device__ explicit Smem(uint8_t* smem) {
    sa = smem;
    sb = smem + C::STAGES * C::A_BYTES;
    raw = sb + C::STAGES * C::B_BYTES;
    uint8_t* bars = smem + C::RING;
    full = reinterpret_cast<uint64_t*>(bars);
    empty = full + C::STAGES;
    tfull = empty + C::STAGES;  // [2] accumulator ready
    tempty = tfull + 2;         // [2] accumulator drained
    raw_full = tempty + 2;
    raw_empty = raw_full + C::RAW_STAGES;
    tmem_slot = reinterpret_cast<uint32_t*>(raw_empty + C::RAW_STAGES);
    abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    epi_consts = reinterpret_cast<float*>(bars + 256);
    slots = bars + 256 + 2048;
  }
};

// The packed-weight side of a one-CTA kernel's pipeline, shared by its raw
// producer warp and its converter warps. K step `it` of the CTA (counted over
// all its tiles) uses ring slot it % STAGES and raw slot it % RAW_STAGES.
template <int BN, int PK>
struct PackedPipe {
  using C = Cfg<BN, PK>;
  using S = Smem<C>;
  // Producer (one thread): the BN / 128 chunks of weight rows
  // [n_tile * BN, n_tile * BN + BN) at K step kb into raw slot it.
  __device__ static bool load(const S& sm, const uint8_t* wpack, int kb_total,
                              int n_tile, int kb, int it, uint32_t* status) {
    const int r = it % C::RAW_STAGES;
    if (!mbar_wait(&sm.raw_empty[r], ((it / C::RAW_STAGES) & 1) ^ 1, sm.abort_flag, status))
      return false;
    mbar_arrive_expect_tx(&sm.raw_full[r], C::RAW_BYTES);
#pragma unroll
    for (int c = 0; c < BN / 128; ++c)
      bulk_load(sm.raw + r * C::RAW_BYTES + c * C::CHUNK,
                wpack + (static_cast<size_t>(n_tile * (BN / 128) + c) * kb_total + kb) * C::CHUNK,
                C::CHUNK, &sm.raw_full[r]);
    return true;
  }
  // Producer, after its last load: see the copies land before the CTA exits
  // (they have unless the CTA gave up).
  __device__ static void drain(const S& sm, int issued) {
    for (int j = issued - C::RAW_STAGES > 0 ? issued - C::RAW_STAGES : 0; j < issued; ++j)
      if (!mbar_drain(&sm.raw_full[j % C::RAW_STAGES], (j / C::RAW_STAGES) & 1, 1ll << 24)) break;
  }
  // Converter warps (t = 0..127 over the four): K step `it` from its raw slot
  // into ring slot it % STAGES (free once the MMAs of step it - STAGES are
  // done), then arrive on full[s] and hand the raw slot back.
  __device__ static bool convert(const S& sm, int it, int t, uint32_t* status) {
    const int r = it % C::RAW_STAGES, s = it % C::STAGES;
    const uint32_t pr = (it / C::RAW_STAGES) & 1, pe = ((it / C::STAGES) & 1) ^ 1;
    int ok = 1;
    if ((t & 31) == 0)
      ok = mbar_wait(&sm.raw_full[r], pr, sm.abort_flag, status) &&
           mbar_wait(&sm.empty[s], pe, sm.abort_flag, status);
    if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
    // Both phases are complete (neither barrier can move on before this warp
    // arrives): every lane observes them, acquiring the raw slot's bytes.
    mbar_try_wait(&sm.raw_full[r], pr);
    mbar_try_wait(&sm.empty[s], pe);
    const uint8_t* raw = sm.raw + r * C::RAW_BYTES;
    uint8_t* tile = sm.sb + s * C::B_BYTES;
#pragma unroll
    for (int c = 0; c < BN / 128; ++c) unpack_row_to_tile<PK>(raw + c * C::CHUNK, t, tile, c * 128 + t);
    // The tile's stores to the async proxy (the MMA reads it), then one
    // arrival per warp on each barrier.
    fence_proxy_async();
    __syncwarp();
    if ((t & 31) == 0) {
      mbar_arrive(&sm.full[s]);
      mbar_arrive(&sm.raw_empty[r]);
    }
    return true;
  }
};

__device__ __forceinline__ float gelu_tanh(float x) {
  // Gemma's tanh GELU with the argument clamped to +-15
  // (matmul_gated.wgsl:126-134), in its logistic form:
  // 0.5 x (1 + tanh z) = x / (1 + e^(-2 z)), with the fast hardware
  // exponential and division (relative error ~1e-6, far below the f16
  // rounding of the stored activation; WGSL's tanh is not correctly rounded
  // either). 1-1.5 us less per E2B / E4B FFN launch than tanhf.
  float z = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  z = fminf(fmaxf(z, -15.0f), 15.0f);
  return __fdividef(x, 1.0f + __expf(-2.0f * z));
}

__device__ __forceinline__ float erf_as(float x) {
  // Abramowitz & Stegun 7.1.26, the erf the reference's ModernBERT GeGLU
  // uses (matmul_gated.wgsl:114-124). The formula's own error is 1.5e-7 and
  // WGSL's `/` and `exp` are not correctly rounded either, so the reciprocal
  // and the exponential use the fast hardware forms (a few ulp): this
  // epilogue runs once per output element of the encoder's largest GEMM and
  // its instruction count, not the tensor pipe, set that GEMM's pace.
  const float s = x < 0.f ? -1.f : (x > 0.f ? 1.f : 0.f);
  const float a = fabsf(x);
  const float t = __fdividef(1.0f, fmaf(0.3275911f, a, 1.0f));
  const float p =
      fmaf(fmaf(fmaf(fmaf(1.061405429f, t, -1.453152027f), t, 1.421413741f), t, -0.284496736f),
           t, 0.254829592f);
  const float y = 1.0f - p * t * __expf(-a * a);
  return s * y;
}

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erf_as(x * 0.7071067811865476f));
}

__device__ __forceinline__ void store_f16x32(__half* o, const float (&v)[32], int col0, int n_out) {
  if (col0 + 32 <= n_out) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 pk;
      __half2 h0 = __floats2half2_rn(v[j], v[j + 1]);
      __half2 h1 = __floats2half2_rn(v[j + 2], v[j + 3]);
      __half2 h2 = __floats2half2_rn(v[j + 4], v[j + 5]);
      __half2 h3 = __floats2half2_rn(v[j + 6], v[j + 7]);
      pk.x = *reinterpret_cast<uint32_t*>(&h0);
      pk.y = *reinterpret_cast<uint32_t*>(&h1);
      pk.z = *reinterpret_cast<uint32_t*>(&h2);
      pk.w = *reinterpret_cast<uint32_t*>(&h3);
      *reinterpret_cast<uint4*>(o + j) = pk;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < n_out) o[j] = __float2half_rn(v[j]);
  }
}

__device__ __forceinline__ uint4 pack_f16x8(const float* v) {
  const __half2 h0 = __floats2half2_rn(v[0], v[1]);
  const __half2 h1 = __floats2half2_rn(v[2], v[3]);
  const __half2 h2 = __floats2half2_rn(v[4], v[5]);
  const __half2 h3 = __floats2half2_rn(v[6], v[7]);
  return make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                    *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
}

__device__ __forceinline__ uint4 pack_f32x4(const float* v) {
  return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                    __float_as_uint(v[3]));
}

// Row staging for coalesced epilogue stores. Lane i of an epilogue warp owns
// row i of the warp's 32 rows and 128 bytes of it (eight 16-byte pieces);
// piece p of row r sits at r * 128 + (p ^ (r & 7)) * 16 of the warp's 4 KB
// slot, so neither the writes (a row per lane) nor the reads (a row per 8
// lanes) conflict on banks.
__device__ __forceinline__ void stage_pieces(uint8_t* slot, int lane, int first, const uint4* pc,
                                             int n) {
#pragma unroll
  for (int i = 0; i < n; ++i)
    *reinterpret_cast<uint4*>(slot + lane * 128 + (((first + i) ^ (lane & 7)) << 4)) = pc[i];
}

// Store the staged 32 x 128 bytes: row r to base + r * stride, rows
// >= nrows skipped; four full 128-byte row segments per instruction.
__device__ __forceinline__ void flush_rows(uint8_t* slot, int lane, uint8_t* base, size_t stride,
                                           int nrows) {
  __syncwarp();
  const int p = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (lane >> 3);
    const uint4 v = *reinterpret_cast<const uint4*>(slot + r * 128 + ((p ^ (r & 7)) << 4));
    if (r < nrows) *reinterpret_cast<uint4*>(base + r * stride + p * 16) = v;
  }
  __syncwarp();
}

// The same with two destinations: pieces 0-3 of row r (64 bytes) to
// base_lo + r * stride, pieces 4-7 to base_hi + r * stride.
__device__ __forceinline__ void flush_rows_split(uint8_t* slot, int lane, uint8_t* base_lo,
                                                 uint8_t* base_hi, size_t stride, int nrows) {
  __syncwarp();
  const int p = lane & 7;
  uint8_t* base = p < 4 ? base_lo + p * 16 : base_hi + (p - 4) * 16;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = 4 * i + (lane >> 3);
    const uint4 v = *reinterpret_cast<const uint4*>(slot + r * 128 + ((p ^ (r & 7)) << 4));
    if (r < nrows) *reinterpret_cast<uint4*>(base + r * stride) = v;
  }
  __syncwarp();
}

// Epilogue of one accumulator tile: epilogue warp q (lanes = TMEM lanes
// 32 q .. 32 q + 31, one output row each) drains its rows from `tbase` and
// stores them through its staging slot.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& g, int m_tile, int n_tile, int split,
                                              uint32_t tbase, int q, int lane, uint8_t* slot,
                                              const float* epi_consts) {
  const int row = m_tile * BM + q * 32 + lane;
  const int row0 = m_tile * BM + q * 32;   // this warp's first row
  const int nrows = min(32, g.m - row0);   // its rows below m (may be <= 0)
  if constexpr (EPI == kEpiF32) {
    float* wbase = static_cast<float*>(g.out) + split * g.split_stride +
                   static_cast<size_t>(row0 > 0 ? row0 : 0) * g.ldo;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      tmem_ld32(tbase + c * 32, v);
      const int col0 = n_tile * BN + c * 32;
      if (nrows <= 0 || col0 >= g.n_out) continue;
      if (col0 + 32 <= g.n_out) {
        uint4 pc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pc[i] = pack_f32x4(v + 4 * i);
        stage_pieces(slot, lane, 0, pc, 8);
        flush_rows(slot, lane, reinterpret_cast<uint8_t*>(wbase + col0),
                   static_cast<size_t>(g.ldo) * 4, nrows);
      } else if (lane < nrows) {
        float* o = wbase + static_cast<size_t>(lane) * g.ldo + col0;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < g.n_out) o[j] = v[j];
      }
    }
  } else if constexpr (EPI == kEpiF16) {
    __half* wbase =
        static_cast<__half*>(g.out) + static_cast<size_t>(row0 > 0 ? row0 : 0) * g.ldo;
#pragma unroll 1
    for (int c = 0; c < BN / 32; c += 2) {
      float lo[32], hi[32];
      tmem_ld32(tbase + c * 32, lo);
      tmem_ld32(tbase + (c + 1) * 32, hi);
      const int col0 = n_tile * BN + c * 32;
      if (nrows <= 0 || col0 >= g.n_out) continue;
      if (col0 + 64 <= g.n_out) {
        uint4 pc[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pc[i] = pack_f16x8(lo + 8 * i);
          pc[4 + i] = pack_f16x8(hi + 8 * i);
        }
        stage_pieces(slot, lane, 0, pc, 8);
        flush_rows(slot, lane, reinterpret_cast<uint8_t*>(wbase + col0),
                   static_cast<size_t>(g.ldo) * 2, nrows);
      } else if (lane < nrows) {
        __half* o = wbase + static_cast<size_t>(lane) * g.ldo;
        store_f16x32(o + col0, lo, col0, g.n_out);
        if (col0 + 32 < g.n_out) store_f16x32(o + col0 + 32, hi, col0 + 32, g.n_out);
      }
    }
  } else if constexpr (EPI == kEpiRopeF16) {
    // 64-dim heads: columns c and c + 32 of a head form a rotation pair.
    __half* wbase =
        static_cast<__half*>(g.out) + static_cast<size_t>(row0 > 0 ? row0 : 0) * g.ldo;
    // Table [pair][position]: the rows of a tile are mostly consecutive
    // positions, so a warp's reads of one pair are contiguous.
    const int p = row < g.m ? g.epi.pos[row] : 0;
    const float2* rt = g.epi.rope + p;
    const size_t rs = static_cast<size_t>(g.epi.rope_stride);
    // Every head of the row rotates by the same 32 (cos, sin) pairs: read
    // them once per tile, all in flight together, before the first chunk.
    float2 cs[32];
    if (n_tile * BN < 2 * g.epi.q_cols) {
#pragma unroll
      for (int j = 0; j < 32; ++j) cs[j] = rt[j * rs];
    }
#pragma unroll 1
    for (int c = 0; c < BN / 32; c += 2) {
      float lo[32], hi[32];
      tmem_ld32(tbase + c * 32, lo);
      tmem_ld32(tbase + (c + 1) * 32, hi);
      const int col0 = n_tile * BN + c * 32;
      if (nrows <= 0 || col0 >= g.n_out) continue;
      if (col0 < 2 * g.epi.q_cols) {
        const float sc = col0 < g.epi.q_cols ? g.epi.q_scale : 1.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float a = lo[j], b = hi[j];
          lo[j] = (a * cs[j].x - b * cs[j].y) * sc;
          hi[j] = (b * cs[j].x + a * cs[j].y) * sc;
        }
      }
      if (col0 + 64 <= g.n_out) {
        uint4 pc[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pc[i] = pack_f16x8(lo + 8 * i);
          pc[4 + i] = pack_f16x8(hi + 8 * i);
        }
        stage_pieces(slot, lane, 0, pc, 8);
        flush_rows(slot, lane, reinterpret_cast<uint8_t*>(wbase + col0),
                   static_cast<size_t>(g.ldo) * 2, nrows);
      } else if (lane < nrows) {
        __half* o = wbase + static_cast<size_t>(lane) * g.ldo;
        store_f16x32(o + col0, lo, col0, g.n_out);
        if (col0 + 32 < g.n_out) store_f16x32(o + col0 + 32, hi, col0 + 32, g.n_out);
      }
    }
  } else if constexpr (EPI == kEpiBiasF16 || EPI == kEpiBiasReluF16) {
    __half* wbase =
        static_cast<__half*>(g.out) + static_cast<size_t>(row0 > 0 ? row0 : 0) * g.ldo;
#pragma unroll 1
    for (int c = 0; c < BN / 32; c += 2) {
      const int col0 = n_tile * BN + c * 32;
      // The chunk pair's 64 bias values, the same for every row: 16-byte
      // broadcast loads issued before the accumulator is read.
      float bv[64];
      if (col0 + 64 <= g.n_out && (reinterpret_cast<uintptr_t>(g.epi.bias) & 15) == 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float4 b4 = __ldg(reinterpret_cast<const float4*>(g.epi.bias + col0) + j);
          bv[4 * j] = b4.x;
          bv[4 * j + 1] = b4.y;
          bv[4 * j + 2] = b4.z;
          bv[4 * j + 3] = b4.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) bv[j] = col0 + j < g.n_out ? g.epi.bias[col0 + j] : 0.f;
      }
      float v[2][32];
      tmem_ld32(tbase + c * 32, v[0]);
      tmem_ld32(tbase + (c + 1) * 32, v[1]);
      if (nrows <= 0 || col0 >= g.n_out) continue;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[h][j] += bv[32 * h + j];
          if constexpr (EPI == kEpiBiasReluF16) v[h][j] = fmaxf(v[h][j], 0.f);
        }
      }
      if (col0 + 64 <= g.n_out) {
        uint4 pc[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pc[i] = pack_f16x8(v[0] + 8 * i);
          pc[4 + i] = pack_f16x8(v[1] + 8 * i);
        }
        stage_pieces(slot, lane, 0, pc, 8);
        flush_rows(slot, lane, reinterpret_cast<uint8_t*>(wbase + col0),
                   static_cast<size_t>(g.ldo) * 2, nrows);
      } else if (lane < nrows) {
        __half* o = wbase + static_cast<size_t>(lane) * g.ldo;
        store_f16x32(o + col0, v[0], col0, g.n_out);
        if (col0 + 32 < g.n_out) store_f16x32(o + col0 + 32, v[1], col0 + 32, g.n_out);
      }
    }
  } else if constexpr (EPI == kEpiResidF32) {
    // Each output element belongs to one tile (no split-K), so the
    // read-modify-write of the residual row is race-free. The accumulator
    // chunk is staged by row; then each lane updates 16 bytes of four
    // rows per step (a row segment per 8 lanes). Its bias values are read
    // before any row is touched, so no bias load waits behind a store to
    // the (possibly aliasing) residual row.
    float* __restrict__ wbase =
        static_cast<float*>(g.out) + static_cast<size_t>(row0 > 0 ? row0 : 0) * g.ldo;
    const float* __restrict__ bias = g.epi.bias;
    const bool bias_first = g.epi.bias_first != 0;
    const int pc4 = lane & 7;  // this lane's 4 columns of a chunk: 4 pc4 .. 4 pc4 + 3
    if (nrows == 32 && (n_tile + 1) * BN <= g.n_out) {
      // Whole 32-row x BN block: the residual values of chunk c + 1 are
      // loaded before chunk c is stored, so each chunk's loads are in flight
      // together and overlap the previous chunk's math and stores (the
      // caller has asked L2 for these rows a tile ahead).
      float* __restrict__ xrow = wbase + static_cast<size_t>(lane >> 3) * g.ldo + n_tile * BN + 4 * pc4;
      const size_t step = static_cast<size_t>(4) * g.ldo;  // rows r and r + 4
      auto load = [&](float4 (&x)[8], int c) {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = *reinterpret_cast<const float4*>(xrow + i * step + c * 32);
      };
      auto update = [&](float4 (&x)[8], int c) {
        const int col = n_tile * BN + c * 32 + 4 * pc4;
        float bl[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) bl[e] = bias ? __ldg(bias + col + e) : 0.f;
        float v[32];
        tmem_ld32(tbase + c * 32, v);
        uint4 pc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pc[i] = pack_f32x4(v + 4 * i);
        stage_pieces(slot, lane, 0, pc, 8);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = 4 * i + (lane >> 3);
          const float4 a = *reinterpret_cast<const float4*>(slot + r * 128 + ((pc4 ^ (r & 7)) << 4));
          const float av[4] = {a.x, a.y, a.z, a.w};
          float* xe = reinterpret_cast<float*>(&x[i]);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            xe[e] = bias_first ? (av[e] + bl[e]) + xe[e] : (xe[e] + av[e]) + bl[e];
          *reinterpret_cast<float4*>(xrow + i * step + c * 32) = x[i];
        }
        __syncwarp();
      };
      float4 xa[8], xb[8];
      load(xa, 0);
#pragma unroll 1
      for (int c = 0; c < BN / 32; c += 2) {
        load(xb, c + 1);
        update(xa, c);
        if (c + 2 < BN / 32) load(xa, c + 2);
        update(xb, c + 1);
      }
      return;
    }
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      const int col0 = n_tile * BN + c * 32;
      float bl[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = col0 + 4 * pc4 + e;
        bl[e] = (bias && col < g.n_out) ? __ldg(bias + col) : 0.f;
      }
      tmem_ld32(tbase + c * 32, v);
      if (nrows <= 0 || col0 >= g.n_out) continue;
      if (col0 + 32 <= g.n_out) {
        uint4 pc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pc[i] = pack_f32x4(v + 4 * i);
        stage_pieces(slot, lane, 0, pc, 8);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = 4 * i + (lane >> 3);
          if (r >= nrows) continue;
          const float4 a = *reinterpret_cast<const float4*>(slot + r * 128 + ((pc4 ^ (r & 7)) << 4));
          float* __restrict__ o = wbase + static_cast<size_t>(r) * g.ldo + col0 + 4 * pc4;
          float4 x = *reinterpret_cast<const float4*>(o);
          const float av[4] = {a.x, a.y, a.z, a.w};
          float* xe = reinterpret_cast<float*>(&x);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            xe[e] = bias_first ? (av[e] + bl[e]) + xe[e] : (xe[e] + av[e]) + bl[e];
          *reinterpret_cast<float4*>(o) = x;
        }
        __syncwarp();
      } else if (lane < nrows) {
        float* __restrict__ o = wbase + static_cast<size_t>(lane) * g.ldo + col0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (col0 + j >= g.n_out) continue;
          const float b = bias ? __ldg(bias + col0 + j) : 0.f;
          o[j] = bias_first ? (v[j] + b) + o[j] : (o[j] + v[j]) + b;
        }
      }
    }
  } else if constexpr (EPI == kEpiQkPrep) {
    // qk_prep.wgsl on the accumulator: this tile is head n_tile of the
    // row, all 256 of its dims in this thread's TMEM lane. Loads are
    // batched ahead of the math (one thread per row has little else to
    // hide their latency with): the norm weights come from shared memory,
    // each 32-pair chunk's RoPE entries are read before they are used.
    static_assert(BN == 256, "one 256-column tile per head");
    const QkEpi& q = g.epi.qk;
    const int h = n_tile;
    const bool is_q = h < q.heads;
    const bool is_v = h >= q.heads + q.kv_heads;
    const bool ok_row = row < g.m;
    const int crow = q.base + (ok_row ? row : 0);
    // Table [pair][position]: consecutive rows read consecutive entries.
    // Each chunk's 32 entries are requested a step ahead of their use
    // (chunk 0's before the sum of squares), so their latency overlaps
    // other work.
    const float2* rt = q.rope + (ok_row ? q.meta[crow].pos : 0);
    const size_t rs = static_cast<size_t>(q.rope_stride);
    const int half_rot = q.rope_dims / 2;
    float2 cs[32];
    if (!is_v && 0 < half_rot) {
#pragma unroll
      for (int j = 0; j < 32; ++j) cs[j] = rt[static_cast<size_t>(j) * rs];
    }
    float ssp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
    for (int c = 0; c < 8; ++c) {
      float v[32];
      tmem_ld32(tbase + c * 32, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) ssp[j & 7] = fmaf(v[j], v[j], ssp[j & 7]);
    }
    const float ss = ((ssp[0] + ssp[1]) + (ssp[2] + ssp[3])) + ((ssp[4] + ssp[5]) + (ssp[6] + ssp[7]));
    const float inv = (is_v && !q.v_norm) ? 1.0f : rsqrtf(ss / 256.0f + q.eps);
    // This warp's first output row (rows are contiguous in both targets).
    const int wrow = row0 > 0 ? row0 : 0;
    uint8_t* wbase;
    size_t wstride;
    if (is_q) {
      wbase = reinterpret_cast<uint8_t*>(q.q16 + static_cast<size_t>(wrow) * q.heads * 256 + h * 256);
      wstride = static_cast<size_t>(q.heads) * 256 * 2;
    } else {
      wbase = reinterpret_cast<uint8_t*>(
          q.kv + static_cast<size_t>(q.base + wrow) * 2 * q.kv_heads * 256 + (h - q.heads) * 256);
      wstride = static_cast<size_t>(2 * q.kv_heads) * 256 * 2;
    }
    const float* wn = epi_consts + (is_q ? 0 : 256);
    const float scale = is_q ? q.q_scale : 1.0f;
    // Dims d and d + 128 rotate together: chunk c of each half per step,
    // both staged by row and stored as two 64-byte row segments.
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float a[32], b[32];
      const bool rot = !is_v && c * 32 < half_rot;
      tmem_ld32(tbase + c * 32, a);
      tmem_ld32(tbase + (c + 4) * 32, b);
      if (is_v) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          a[j] *= inv;
          b[j] *= inv;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int dd = c * 32 + j;
          float y1 = a[j] * inv * (q.offset + wn[dd]);
          float y2 = b[j] * inv * (q.offset + wn[dd + 128]);
          if (rot && dd < half_rot) {
            const float r1 = y1 * cs[j].x - y2 * cs[j].y;
            const float r2 = y2 * cs[j].x + y1 * cs[j].y;
            y1 = r1;
            y2 = r2;
          }
          a[j] = y1 * scale;
          b[j] = y2 * scale;
        }
      }
      uint4 pc[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        pc[i] = pack_f16x8(a + 8 * i);
        pc[4 + i] = pack_f16x8(b + 8 * i);
      }
      if (c + 1 < 4 && !is_v && (c + 1) * 32 < half_rot) {
#pragma unroll
        for (int j = 0; j < 32; ++j) cs[j] = rt[static_cast<size_t>((c + 1) * 32 + j) * rs];
      }
      if (nrows > 0) {
        stage_pieces(slot, lane, 0, pc, 8);
        flush_rows_split(slot, lane, wbase + c * 64, wbase + 256 + c * 64, wstride, nrows);
      }
    }
  } else {
    // GeGLU: accumulator columns 0..127 hold the gate products, 128..255
    // the up products of the same 128 output columns.
    static_assert(BN == 256, "GeGLU tiles pair 128 gate rows with 128 up rows");
    __half* wbase =
        static_cast<__half*>(g.out) + static_cast<size_t>(row0 > 0 ? row0 : 0) * g.ldo;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float gv[32], uv[32];
      tmem_ld32(tbase + c * 32, gv);
      tmem_ld32(tbase + 128 + c * 32, uv);
      const int col0 = n_tile * 128 + (c & ~1) * 32;  // first column of this chunk pair
#pragma unroll
      for (int j = 0; j < 32; ++j)
        gv[j] = ((EPI == kEpiGeGluTanh) ? gelu_tanh(gv[j]) : gelu_erf(gv[j])) * uv[j];
      if (nrows <= 0 || col0 >= g.n_out) continue;
      if (col0 + 64 <= g.n_out) {
        uint4 pc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) pc[i] = pack_f16x8(gv + 8 * i);
        stage_pieces(slot, lane, (c & 1) * 4, pc, 4);
        if (c & 1)
          flush_rows(slot, lane, reinterpret_cast<uint8_t*>(wbase + col0),
                     static_cast<size_t>(g.ldo) * 2, nrows);
      } else if (lane < nrows) {
        const int cc = col0 + (c & 1) * 32;
        if (cc < g.n_out) store_f16x32(wbase + static_cast<size_t>(lane) * g.ldo + cc, gv, cc, g.n_out);
      }
    }
  }
}

// L2 prefetch of the residual rows tile `tile` of a kEpiResidF32 GEMM
// updates: lane i of epilogue warp q asks for its own row's BN columns.
template <int BN>
__device__ __forceinline__ void residual_prefetch(const GemmArgs& g, int tile, int q, int lane) {
  if (tile >= g.m_tiles * g.n_tiles * g.splits) return;
  const TileId id = decode_tile(g, tile);
  const int row = id.m * BM + q * 32 + lane;
  const int col0 = id.n * BN;
  if (row >= g.m) return;
  const float* p = static_cast<const float*>(g.out) + static_cast<size_t>(row) * g.ldo + col0;
  const int n = min(BN, g.n_out - col0);
#pragma unroll 1
  for (int c = 0; c < n; c += 32) prefetch_l2(p + c);
}

// Persistent: CTA b handles tiles b, b + gridDim.x, ... in decode_tile's
// order.
template <int BN, int EPI, int PK>
__global__ void __launch_bounds__(Cfg<BN, PK>::THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                GemmArgs g) {
  using C = Cfg<BN, PK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const Smem<C> sm(smem);
  uint8_t* sa = sm.sa;
  uint8_t* sb = sm.sb;
  uint64_t* full = sm.full;
  uint64_t* empty = sm.empty;
  uint64_t* tfull = sm.tfull;
  uint64_t* tempty = sm.tempty;
  uint32_t* tmem_slot = sm.tmem_slot;
  volatile int* abort_flag = sm.abort_flag;
  float* epi_consts = sm.epi_consts;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total = g.m_tiles * g.n_tiles * g.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      // Packed: the TMA bytes of A plus one arrival per converter warp.
      mbar_init(&full[s], C::PACKED ? 5 : 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    for (int r = 0; r < C::RAW_STAGES; ++r) {
      mbar_init(&sm.raw_full[r], 1);
      mbar_init(&sm.raw_empty[r], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tma);
    if constexpr (!C::PACKED) prefetch_tmap(&tmb);
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Operands and residual rows come from earlier kernels (programmatic
  // dependent launch: the prologue above may overlap their tail); the packed
  // weights never change during a pass, so their copies start at once. The
  // grid is persistent (one wave), so the next kernel may begin launching now.
  if (!(C::PACKED && warp == 6) && warp != 0) griddep_wait();
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      // f16 weights never change during a pass: the first tile's first ring
      // of weight tiles is requested before the wait for the previous
      // kernel, which produces only the activations.
      int pre = 0;
      if constexpr (!C::PACKED) {
        if (static_cast<int>(blockIdx.x) < total) {
          const TileId id = decode_tile(g, blockIdx.x);
          const int kb0 = id.split * g.kb_per_split;
          const int kb1 = min(g.kb_total, kb0 + g.kb_per_split);
          pre = min(C::STAGES, kb1 - kb0);
          for (int j = 0; j < pre; ++j) {
            mbar_expect_tx(&full[j], C::B_BYTES);
            tma_load_2d(sb + j * C::B_BYTES, &tmb, &full[j], (kb0 + j) * BK, id.n * BN);
          }
        }
      }
      griddep_wait();
      int it = 0;
      for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x) {
        const TileId id = decode_tile(g, tile);
        const int m_tile = id.m, n_tile = id.n, split = id.split;
        const int kb0 = split * g.kb_per_split;
        const int kb1 = min(g.kb_total, kb0 + g.kb_per_split);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, g.status)) {
            ok = false;
            break;
          }
          if constexpr (C::PACKED) {
            mbar_arrive_expect_tx(&full[s], C::A_BYTES);
            tma_load_2d(sa + s * C::A_BYTES, &tma, &full[s], kb * BK, m_tile * BM);
          } else if (it < pre) {
            mbar_arrive_expect_tx(&full[s], C::A_BYTES);
            tma_load_2d(sa + s * C::A_BYTES, &tma, &full[s], kb * BK, m_tile * BM);
          } else {
            mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
            tma_load_2d(sa + s * C::A_BYTES, &tma, &full[s], kb * BK, m_tile * BM);
            tma_load_2d(sb + s * C::B_BYTES, &tmb, &full[s], kb * BK, n_tile * BN);
          }
        }
        if (!ok) break;
      }
    } else {
      griddep_wait();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(BM, BN);
      int it = 0, local = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++local) {
        const int split = tile / (g.m_tiles * g.n_tiles);
        const int kb0 = split * g.kb_per_split;
        const int kb1 = min(g.kb_total, kb0 + g.kb_per_split);
        const int b = local & 1;
        if (!mbar_wait(&tempty[b], ((local >> 1) & 1) ^ 1, abort_flag, g.status)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag, g.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sw128_desc(sa + s * C::A_BYTES);
          const uint64_t db = sw128_desc(sb + s * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d, da + 2 * k, db + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
    }
  } else if (warp < 6) {
    // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +32, one row per thread.
    const int q = warp & 3;
    if constexpr (EPI == kEpiQkPrep) {
      // The q and k norm weights, staged while the first tile's mainloop runs.
      for (int i = threadIdx.x - 64; i < 512; i += 128) {
        const float* src = i < 256 ? g.epi.qk.qn : g.epi.qk.kn;
        epi_consts[i] = src ? src[i & 255] : 0.f;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
    }
    int local = 0;
    if constexpr (EPI == kEpiResidF32) residual_prefetch<BN>(g, blockIdx.x, q, lane);
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++local) {
      const TileId id = decode_tile(g, tile);
      const int m_tile = id.m, n_tile = id.n, split = id.split;
      const int b = local & 1;
      // The residual rows the next tile updates, requested a tile ahead.
      if constexpr (EPI == kEpiResidF32) residual_prefetch<BN>(g, tile + gridDim.x, q, lane);
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&tfull[b], (local >> 1) & 1, abort_flag, g.status) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      uint8_t* slot = sm.slots + q * 4096;
      const uint32_t tbase =
          tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * BN);
      epilogue_tile<BN, EPI>(g, m_tile, n_tile, split, tbase, q, lane, slot, epi_consts);
      // This warp is done with accumulator b.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  } else if constexpr (C::PACKED) {
    if (warp == 6) {
      // Bulk copies of the packed weight chunks, up to RAW_STAGES K steps ahead.
      if (lane == 0) {
        int it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < total && ok && !*abort_flag; tile += gridDim.x) {
          const TileId id = decode_tile(g, tile);
          const int kb0 = id.split * g.kb_per_split;
          const int kb1 = min(g.kb_total, kb0 + g.kb_per_split);
          for (int kb = kb0; kb < kb1 && ok; ++kb, ++it)
            ok = PackedPipe<BN, PK>::load(sm, g.wpack, g.kb_total, id.n, kb, it, g.status);
        }
        PackedPipe<BN, PK>::drain(sm, it);
      }
    } else {
      // Converters: chunk row t of each K step into the swizzled f16 tile.
      const int t = threadIdx.x - 224;
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const TileId id = decode_tile(g, tile);
        const int kb0 = id.split * g.kb_per_split;
        const int kb1 = min(g.kb_total, kb0 + g.kb_per_split);
        for (int kb = kb0; kb < kb1 && ok; ++kb, ++it)
          ok = PackedPipe<BN, PK>::convert(sm, it, t, g.status);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---- CTA-pair GEMM (tcgen05 cta_group::2) ---------------------------------
//
// A cluster of two CTAs on one TPC computes 256-row x 256-column tiles: CTA
// rank r stages its own 128 rows of A (M tile 2 p + r of pair tile p) and
// its half of the 256 weight rows (rows 128 r .. 128 r + 127 of the tile),
// 32 KB per 64-wide K step instead of 48, so six steps are in flight per SM
// instead of four. The leader's MMA thread issues M = 256, N = 256 MMAs that
// read both CTAs' halves; each CTA's TMEM receives its own 128 rows, which
// its epilogue warps drain with the same epilogue as the one-CTA kernel.
//
// Barriers (same offsets in both CTAs): full[s] on the leader counts both
// CTAs' TMA bytes (the leader posts the expectation; each CTA's loads
// complete on the leader's barrier); empty[s] and tfull[b] are signalled in
// both CTAs by the leader's commits; tempty[b] on the leader counts the
// epilogue warps of both CTAs (the peer's arrive remotely).
template <int PK = kF16>
struct Cfg2 {
  static constexpr bool PACKED = PK != kF16;
  static constexpr int STAGES = PACKED ? 5 : 6;
  static constexpr int A_BYTES = BM * BK * 2;       // 128 rows of A
  static constexpr int B_BYTES = 128 * BK * 2;      // this CTA's 128 weight rows
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int CHUNK = PK == kQ4 ? PackChunk<kQ4>::BYTES
                                         : (PK == kQ8 ? PackChunk<kQ8>::BYTES : 0);
  static constexpr int RAW_BYTES = CHUNK;           // this CTA's 128 weight rows, packed
  static constexpr int RAW_STAGES = !PACKED ? 0 : (PK == kQ4 ? 6 : 4);
  static constexpr int RING = STAGES * STAGE_BYTES + RAW_STAGES * RAW_BYTES;
  static constexpr int SMEM = RING + 1024 + 256 + 2048 + 4 * 4096;
  static constexpr uint32_t TMEM_COLS = 512;        // two 256-column accumulators
  static constexpr int THREADS = PACKED ? 352 : 192;
  static_assert(SMEM <= 232448, "shared memory");
  static_assert(2 * STAGES + 4 + 2 * RAW_STAGES <= 30, "barrier area");
};

// The packed-weight side of the CTA-pair kernels: each CTA fetches and
// decodes its own 128 weight rows of the tile (chunk 2 n + rank) into its
// half of the B operand; both CTAs' converter warps arrive on the leader's
// full barrier (releasing their stores at cluster scope), which the
// leader's MMA thread waits on with cluster-scope acquire.
template <int PK>
struct PackedPipe2 {
  using C = Cfg2<PK>;
  using S = Smem<C>;
  __device__ static bool load(const S& sm, const uint8_t* wpack, int kb_total, int chunk_row,
                              int kb, int it, uint32_t* status) {
    const int r = it % C::RAW_STAGES;
    if (!mbar_wait(&sm.raw_empty[r], ((it / C::RAW_STAGES) & 1) ^ 1, sm.abort_flag, status))
      return false;
    mbar_arrive_expect_tx(&sm.raw_full[r], C::RAW_BYTES);
    bulk_load(sm.raw + r * C::RAW_BYTES,
              wpack + (static_cast<size_t>(chunk_row) * kb_total + kb) * C::CHUNK, C::CHUNK,
              &sm.raw_full[r]);
    return true;
  }
  __device__ static void drain(const S& sm, int issued) {
    for (int j = issued - C::RAW_STAGES > 0 ? issued - C::RAW_STAGES : 0; j < issued; ++j)
      if (!mbar_drain(&sm.raw_full[j % C::RAW_STAGES], (j / C::RAW_STAGES) & 1, 1ll << 24)) break;
  }
  __device__ static bool convert(const S& sm, int it, int t, uint32_t* status) {
    const int r = it % C::RAW_STAGES, s = it % C::STAGES;
    const uint32_t pr = (it / C::RAW_STAGES) & 1, pe = ((it / C::STAGES) & 1) ^ 1;
    int ok = 1;
    if ((t & 31) == 0)
      ok = mbar_wait(&sm.raw_full[r], pr, sm.abort_flag, status) &&
           mbar_wait(&sm.empty[s], pe, sm.abort_flag, status);
    if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
    mbar_try_wait(&sm.raw_full[r], pr);
    mbar_try_wait(&sm.empty[s], pe);
    unpack_row_to_tile<PK>(sm.raw + r * C::RAW_BYTES, t, sm.sb + s * C::B_BYTES, t);
    fence_proxy_async();
    __syncwarp();
    if ((t & 31) == 0) {
      mbar_arrive_release_cluster(cluster_addr(&sm.full[s], 0));
      mbar_arrive(&sm.raw_empty[r]);
    }
    return true;
  }
};

// Pair tile t: split-major, then (M pair fastest) or (N fastest).
__device__ __forceinline__ TileId decode_pair_tile(const GemmArgs& g, int m_pairs, int t) {
  const int mn = m_pairs * g.n_tiles;
  const int r = t % mn;
  TileId x;
  x.split = t / mn;
  x.m = g.n_fast ? r / g.n_tiles : r % m_pairs;
  x.n = g.n_fast ? r % g.n_tiles : r / m_pairs;
  return x;
}

template <int EPI, int PK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg2<PK>::THREADS, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmb,
                 GemmArgs g) {
  constexpr int BN = 256;
  using C = Cfg2<PK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const Smem<C> sm(smem);
  uint8_t* sa = sm.sa;
  uint8_t* sb = sm.sb;
  uint64_t* full = sm.full;
  uint64_t* empty = sm.empty;
  uint64_t* tfull = sm.tfull;    // [2] accumulator ready (both CTAs)
  uint64_t* tempty = sm.tempty;  // [2] accumulator drained (leader: 8 warps)
  uint32_t* tmem_slot = sm.tmem_slot;
  volatile int* abort_flag = sm.abort_flag;
  float* epi_consts = sm.epi_consts;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = static_cast<int>(cluster_index());
  const int npairs = static_cast<int>(cluster_count());
  const int m_pairs = (g.m_tiles + 1) / 2;
  const int total = m_pairs * g.n_tiles * g.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      // Packed: the leader's also counts both CTAs' converter warps.
      mbar_init(&full[s], C::PACKED ? 9 : 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    for (int r = 0; r < C::RAW_STAGES; ++r) {
      mbar_init(&sm.raw_full[r], 1);
      mbar_init(&sm.raw_empty[r], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tma);
    if constexpr (!C::PACKED) prefetch_tmap(&tmb);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (!(C::PACKED && warp == 6)) griddep_wait();
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int tile = pair; tile < total && !*abort_flag; tile += npairs) {
        const TileId id = decode_pair_tile(g, m_pairs, tile);
        const int m_tile = 2 * id.m + static_cast<int>(rank);
        const int kb0 = id.split * g.kb_per_split;
        const int kb1 = min(g.kb_total, kb0 + g.kb_per_split);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, g.status)) {
            ok = false;
            break;
          }
          const uint32_t bar = cluster_addr(&full[s], 0);
          if constexpr (C::PACKED) {
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * C::A_BYTES);
            tma_load_2d_pair(sa + s * C::A_BYTES, &tma, bar, kb * BK, m_tile * BM);
          } else {
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * C::STAGE_BYTES);
            tma_load_2d_pair(sa + s * C::A_BYTES, &tma, bar, kb * BK, m_tile * BM);
            tma_load_2d_pair(sb + s * C::B_BYTES, &tmb, bar, kb * BK,
                             id.n * BN + 128 * static_cast<int>(rank));
          }
        }
        if (!ok) break;
      }
      // The leader's last commits to this CTA's empty barriers are
      // asynchronous: see them land before the CTA can exit.
      for (int j = max(0, it - C::STAGES); j < it && !*abort_flag; ++j)
        if (!mbar_wait(&empty[j % C::STAGES], (j / C::STAGES) & 1, abort_flag, g.status)) break;
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(2 * BM, BN);
      int it = 0, local = 0;
      for (int tile = pair; tile < total; tile += npairs, ++local) {
        const TileId id = decode_pair_tile(g, m_pairs, tile);
        const int kb0 = id.split * g.kb_per_split;
        const int kb1 = min(g.kb_total, kb0 + g.kb_per_split);
        const int b = local & 1;
        if (!mbar_wait(&tempty[b], ((local >> 1) & 1) ^ 1, abort_flag, g.status)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait_cluster(&full[s], ph, abort_flag, g.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sw128_desc(sa + s * C::A_BYTES);
          const uint64_t db = sw128_desc(sb + s * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_pair(d, da + 2 * k, db + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit_pair(&empty[s]);
        }
        if (!ok) break;
        umma_commit_pair(&tfull[b]);
      }
    }
  } else if (warp < 6) {
    const int q = warp & 3;
    if constexpr (EPI == kEpiQkPrep) {
      for (int i = threadIdx.x - 64; i < 512; i += 128) {
        const float* src = i < 256 ? g.epi.qk.qn : g.epi.qk.kn;
        epi_consts[i] = src ? src[i & 255] : 0.f;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
    }
    auto prefetch = [&](int tile) {
      // The residual rows of this CTA's half of pair tile `tile`, into L2.
      if constexpr (EPI == kEpiResidF32) {
        if (tile >= total) return;
        const TileId id = decode_pair_tile(g, m_pairs, tile);
        const int row = (2 * id.m + static_cast<int>(rank)) * BM + q * 32 + lane;
        if (row >= g.m) return;
        const float* p = static_cast<const float*>(g.out) + static_cast<size_t>(row) * g.ldo + id.n * BN;
        const int n = min(BN, g.n_out - id.n * BN);
#pragma unroll 1
        for (int c = 0; c < n; c += 32) prefetch_l2(p + c);
      }
    };
    prefetch(pair);
    int local = 0;
    for (int tile = pair; tile < total; tile += npairs, ++local) {
      const TileId id = decode_pair_tile(g, m_pairs, tile);
      const int b = local & 1;
      prefetch(tile + npairs);
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&tfull[b], (local >> 1) & 1, abort_flag, g.status) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      uint8_t* slot = sm.slots + q * 4096;
      const uint32_t tbase =
          tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * BN);
      epilogue_tile<BN, EPI>(g, 2 * id.m + static_cast<int>(rank), id.n, id.split, tbase, q, lane,
                             slot, epi_consts);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(&tempty[b], 0));
    }
  } else if constexpr (C::PACKED) {
    if (warp == 6) {
      // This CTA's 128 weight rows of each tile, packed, RAW_STAGES K steps ahead.
      if (lane == 0) {
        int it = 0;
        bool ok = true;
        for (int tile = pair; tile < total && ok && !*abort_flag; tile += npairs) {
          const TileId id = decode_pair_tile(g, m_pairs, tile);
          const int kb0 = id.split * g.kb_per_split;
          const int kb1 = min(g.kb_total, kb0 + g.kb_per_split);
          for (int kb = kb0; kb < kb1 && ok; ++kb, ++it)
            ok = PackedPipe2<PK>::load(sm, g.wpack, g.kb_total, 2 * id.n + static_cast<int>(rank),
                                       kb, it, g.status);
        }
        PackedPipe2<PK>::drain(sm, it);
      }
    } else {
      const int t = threadIdx.x - 224;
      int it = 0;
      bool ok = true;
      for (int tile = pair; tile < total && ok; tile += npairs) {
        const TileId id = decode_pair_tile(g, m_pairs, tile);
        const int kb0 = id.split * g.kb_per_split;
        const int kb1 = min(g.kb_total, kb0 + g.kb_per_split);
        for (int kb = kb0; kb < kb1 && ok; ++kb, ++it)
          ok = PackedPipe2<PK>::convert(sm, it, t, g.status);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  // Neither CTA leaves (or frees TMEM) while the other may still read its
  // shared memory or signal its barriers.
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Orders this thread's generic-proxy global accesses with async-proxy (TMA)
// accesses to global memory.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Gate+up and down projections of one FFN in one persistent launch. Units:
// the up tiles in the standalone order (m = t % m_tiles, n = t / m_tiles, so
// the CTAs running at once share weight tiles in L2), then the down units
// split-major (split, then m fastest, then n). CTA b takes units b,
// b + gridDim.x, ... Both problems' units run the same number of K blocks
// (down's split count is chosen so), so the rounds stay even and the down
// units fill what would be the up projection's last, partial round. Down
// split s of M tile m reads the activation columns that up column tiles
// [s * band, (s + 1) * band) of m store: every epilogue warp of such an up
// tile counts itself in ready[m * splits + s] once its rows are stored
// (cumulative over a pass: this launch's count is reached at ready_target),
// and the down unit's producer waits for that count before its first load.
// Up tiles finish band by band in unit order, so a down unit rarely waits.
// Each unit's result is the one the two separate launches compute.
struct MlpArgs {
  GemmArgs up, down;
  int* ready;
  int ready_target;
  int band;  // up column tiles per down split
  long long wait_limit;  // SM clocks a down unit waits for its band before giving up
};

template <int EPI_UP, int PK>
__global__ void __launch_bounds__(Cfg<256, PK>::THREADS, 1)
    gemm_mlp_kernel(const __grid_constant__ CUtensorMap ta_up,
                    const __grid_constant__ CUtensorMap tb_up,
                    const __grid_constant__ CUtensorMap ta_dn,
                    const __grid_constant__ CUtensorMap tb_dn, MlpArgs g) {
  constexpr int BN = 256;
  using C = Cfg<BN, PK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const Smem<C> sm(smem);
  uint8_t* sa = sm.sa;
  uint8_t* sb = sm.sb;
  uint64_t* full = sm.full;
  uint64_t* empty = sm.empty;
  uint64_t* tfull = sm.tfull;
  uint64_t* tempty = sm.tempty;
  uint32_t* tmem_slot = sm.tmem_slot;
  volatile int* abort_flag = sm.abort_flag;
  float* epi_consts = sm.epi_consts;
  uint32_t* status = g.up.status;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int up_units = g.up.m_tiles * g.up.n_tiles;
  const int dn_per_split = g.down.m_tiles * g.down.n_tiles;
  const int total = up_units + dn_per_split * g.down.splits;
  struct Unit {
    bool up;
    int m, n, split, kb0, kb1;
  };
  auto decode = [&](int u) {
    Unit x;
    if (u < up_units) {
      x.up = true;
      x.m = u % g.up.m_tiles;
      x.n = u / g.up.m_tiles;
      x.split = 0;
      x.kb0 = 0;
      x.kb1 = g.up.kb_total;
    } else {
      const int v = u - up_units;
      const int r = v % dn_per_split;
      x.up = false;
      x.split = v / dn_per_split;
      x.m = r % g.down.m_tiles;
      x.n = r / g.down.m_tiles;
      x.kb0 = x.split * g.down.kb_per_split;
      x.kb1 = min(g.down.kb_total, x.kb0 + g.down.kb_per_split);
    }
    return x;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], C::PACKED ? 5 : 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    for (int r = 0; r < C::RAW_STAGES; ++r) {
      mbar_init(&sm.raw_full[r], 1);
      mbar_init(&sm.raw_empty[r], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&ta_up);
    prefetch_tmap(&ta_dn);
    if constexpr (!C::PACKED) {
      prefetch_tmap(&tb_up);
      prefetch_tmap(&tb_dn);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (!(C::PACKED && warp == 6) && warp != 0) griddep_wait();
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      // The first unit's first ring of weight tiles before the wait for the
      // previous kernel (f16 weights never change during a pass).
      int pre = 0;
      if constexpr (!C::PACKED) {
        if (static_cast<int>(blockIdx.x) < total) {
          const Unit x = decode(blockIdx.x);
          pre = min(C::STAGES, x.kb1 - x.kb0);
          for (int j = 0; j < pre; ++j) {
            mbar_expect_tx(&full[j], C::B_BYTES);
            tma_load_2d(sb + j * C::B_BYTES, x.up ? &tb_up : &tb_dn, &full[j], (x.kb0 + j) * BK,
                        x.n * BN);
          }
        }
      }
      griddep_wait();
      int it = 0;
      for (int u = blockIdx.x; u < total && !*abort_flag; u += gridDim.x) {
        const Unit x = decode(u);
        if (!x.up) {
          // This unit's activation columns of its rows: every up tile of the
          // band stored.
          const int* rp = g.ready + x.m * g.down.splits + x.split;
          const long long t0 = clock64();
          bool ok = true;
          while (ld_acquire_gpu(rp) < g.ready_target) {
            if (*abort_flag) {
              ok = false;
              break;
            }
            if (clock64() - t0 > g.wait_limit) {
              *abort_flag = 1;
              atomicCAS(status, 0u, static_cast<uint32_t>(kDevWaitTimeout));
              ok = false;
              break;
            }
            __nanosleep(64);
          }
          if (!ok) break;
          fence_proxy_async_global();
        }
        const CUtensorMap* ta = x.up ? &ta_up : &ta_dn;
        const CUtensorMap* tb = x.up ? &tb_up : &tb_dn;
        bool ok = true;
        for (int kb = x.kb0; kb < x.kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, status)) {
            ok = false;
            break;
          }
          if constexpr (C::PACKED) {
            mbar_arrive_expect_tx(&full[s], C::A_BYTES);
            tma_load_2d(sa + s * C::A_BYTES, ta, &full[s], kb * BK, x.m * BM);
          } else if (it < pre) {
            mbar_arrive_expect_tx(&full[s], C::A_BYTES);
            tma_load_2d(sa + s * C::A_BYTES, ta, &full[s], kb * BK, x.m * BM);
          } else {
            mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
            tma_load_2d(sa + s * C::A_BYTES, ta, &full[s], kb * BK, x.m * BM);
            tma_load_2d(sb + s * C::B_BYTES, tb, &full[s], kb * BK, x.n * BN);
          }
        }
        if (!ok) break;
      }
    } else {
      griddep_wait();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(BM, BN);
      int it = 0, local = 0;
      for (int u = blockIdx.x; u < total; u += gridDim.x, ++local) {
        const Unit x = decode(u);
        const int b = local & 1;
        if (!mbar_wait(&tempty[b], ((local >> 1) & 1) ^ 1, abort_flag, status)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * BN);
        bool ok = true;
        for (int kb = x.kb0; kb < x.kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sw128_desc(sa + s * C::A_BYTES);
          const uint64_t db = sw128_desc(sb + s * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d, da + 2 * k, db + 2 * k, idesc, (kb > x.kb0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
    }
  } else if (warp < 6) {
    const int q = warp & 3;
    int local = 0;
    for (int u = blockIdx.x; u < total; u += gridDim.x, ++local) {
      const Unit x = decode(u);
      const int b = local & 1;
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&tfull[b], (local >> 1) & 1, abort_flag, status) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      uint8_t* slot = sm.slots + q * 4096;
      const uint32_t tbase =
          tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * BN);
      if (x.up) {
        epilogue_tile<BN, EPI_UP>(g.up, x.m, x.n, 0, tbase, q, lane, slot, epi_consts);
        // Publish this warp's rows to the down units' loads (another proxy,
        // other SMs), then count the warp in.
        fence_proxy_async_global();
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(g.ready + x.m * g.down.splits + x.n / g.band, 1);
      } else {
        epilogue_tile<BN, kEpiF32>(g.down, x.m, x.n, x.split, tbase, q, lane, slot, epi_consts);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  } else if constexpr (C::PACKED) {
    if (warp == 6) {
      // The weight chunks of every unit (they do not wait for the
      // activations: a down unit's weights arrive while its band finishes).
      if (lane == 0) {
        int it = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < total && ok && !*abort_flag; u += gridDim.x) {
          const Unit x = decode(u);
          const GemmArgs& ga = x.up ? g.up : g.down;
          for (int kb = x.kb0; kb < x.kb1 && ok; ++kb, ++it)
            ok = PackedPipe<BN, PK>::load(sm, ga.wpack, ga.kb_total, x.n, kb, it, status);
        }
        PackedPipe<BN, PK>::drain(sm, it);
      }
    } else {
      const int t = threadIdx.x - 224;
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const Unit x = decode(u);
        for (int kb = x.kb0; kb < x.kb1 && ok; ++kb, ++it)
          ok = PackedPipe<BN, PK>::convert(sm, it, t, status);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// The fused FFN launch on CTA pairs: the units of gemm_mlp_kernel with
// 256-row pair tiles (CTA rank r of pair tile p holds M tile 2 p + r), the
// pipeline and barriers of gemm2_kernel. A down unit's producer waits for
// its own M tile's activation band (a CTA whose half lies past the last M
// tile has no rows and waits for nothing); the leader's full barrier then
// holds the MMA until both halves are loaded.
template <int EPI_UP, int PK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg2<PK>::THREADS, 1)
    gemm_mlp2_kernel(const __grid_constant__ CUtensorMap ta_up,
                     const __grid_constant__ CUtensorMap tb_up,
                     const __grid_constant__ CUtensorMap ta_dn,
                     const __grid_constant__ CUtensorMap tb_dn, MlpArgs g) {
  constexpr int BN = 256;
  using C = Cfg2<PK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const Smem<C> sm(smem);
  uint8_t* sa = sm.sa;
  uint8_t* sb = sm.sb;
  uint64_t* full = sm.full;
  uint64_t* empty = sm.empty;
  uint64_t* tfull = sm.tfull;
  uint64_t* tempty = sm.tempty;
  uint32_t* tmem_slot = sm.tmem_slot;
  volatile int* abort_flag = sm.abort_flag;
  float* epi_consts = sm.epi_consts;
  uint32_t* status = g.up.status;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = static_cast<int>(cluster_index());
  const int npairs = static_cast<int>(cluster_count());
  const int m_tiles = g.up.m_tiles;
  const int m_pairs = (m_tiles + 1) / 2;
  const int up_units = m_pairs * g.up.n_tiles;
  const int dn_per_split = m_pairs * g.down.n_tiles;
  const int total = up_units + dn_per_split * g.down.splits;
  struct Unit {
    bool up;
    int m, n, split, kb0, kb1;  // m: this CTA's M tile
  };
  auto decode = [&](int u) {
    Unit x;
    if (u < up_units) {
      x.up = true;
      x.m = 2 * (u % m_pairs) + static_cast<int>(rank);
      x.n = u / m_pairs;
      x.split = 0;
      x.kb0 = 0;
      x.kb1 = g.up.kb_total;
    } else {
      const int v = u - up_units;
      const int r = v % dn_per_split;
      x.up = false;
      x.split = v / dn_per_split;
      x.m = 2 * (r % m_pairs) + static_cast<int>(rank);
      x.n = r / m_pairs;
      x.kb0 = x.split * g.down.kb_per_split;
      x.kb1 = min(g.down.kb_total, x.kb0 + g.down.kb_per_split);
    }
    return x;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], C::PACKED ? 9 : 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    for (int r = 0; r < C::RAW_STAGES; ++r) {
      mbar_init(&sm.raw_full[r], 1);
      mbar_init(&sm.raw_empty[r], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&ta_up);
    prefetch_tmap(&ta_dn);
    if constexpr (!C::PACKED) {
      prefetch_tmap(&tb_up);
      prefetch_tmap(&tb_dn);
    }
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (!(C::PACKED && warp == 6)) griddep_wait();
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int u = pair; u < total && !*abort_flag; u += npairs) {
        const Unit x = decode(u);
        if (!x.up && x.m < m_tiles) {
          const int* rp = g.ready + x.m * g.down.splits + x.split;
          const long long t0 = clock64();
          bool ok = true;
          while (ld_acquire_gpu(rp) < g.ready_target) {
            if (*abort_flag) {
              ok = false;
              break;
            }
            if (clock64() - t0 > g.wait_limit) {
              *abort_flag = 1;
              atomicCAS(status, 0u, static_cast<uint32_t>(kDevWaitTimeout));
              ok = false;
              break;
            }
            __nanosleep(64);
          }
          if (!ok) break;
          fence_proxy_async_global();
        }
        const CUtensorMap* ta = x.up ? &ta_up : &ta_dn;
        const CUtensorMap* tb = x.up ? &tb_up : &tb_dn;
        bool ok = true;
        for (int kb = x.kb0; kb < x.kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, status)) {
            ok = false;
            break;
          }
          const uint32_t bar = cluster_addr(&full[s], 0);
          if constexpr (C::PACKED) {
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * C::A_BYTES);
            tma_load_2d_pair(sa + s * C::A_BYTES, ta, bar, kb * BK, x.m * BM);
          } else {
            if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * C::STAGE_BYTES);
            tma_load_2d_pair(sa + s * C::A_BYTES, ta, bar, kb * BK, x.m * BM);
            tma_load_2d_pair(sb + s * C::B_BYTES, tb, bar, kb * BK,
                             x.n * BN + 128 * static_cast<int>(rank));
          }
        }
        if (!ok) break;
      }
      for (int j = max(0, it - C::STAGES); j < it && !*abort_flag; ++j)
        if (!mbar_wait(&empty[j % C::STAGES], (j / C::STAGES) & 1, abort_flag, status)) break;
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(2 * BM, BN);
      int it = 0, local = 0;
      for (int u = pair; u < total; u += npairs, ++local) {
        const Unit x = decode(u);
        const int b = local & 1;
        if (!mbar_wait(&tempty[b], ((local >> 1) & 1) ^ 1, abort_flag, status)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * BN);
        bool ok = true;
        for (int kb = x.kb0; kb < x.kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1;
          if (!mbar_wait_cluster(&full[s], ph, abort_flag, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sw128_desc(sa + s * C::A_BYTES);
          const uint64_t db = sw128_desc(sb + s * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_pair(d, da + 2 * k, db + 2 * k, idesc, (kb > x.kb0 || k > 0) ? 1u : 0u);
          umma_commit_pair(&empty[s]);
        }
        if (!ok) break;
        umma_commit_pair(&tfull[b]);
      }
    }
  } else if (warp < 6) {
    const int q = warp & 3;
    int local = 0;
    for (int u = pair; u < total; u += npairs, ++local) {
      const Unit x = decode(u);
      const int b = local & 1;
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&tfull[b], (local >> 1) & 1, abort_flag, status) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      uint8_t* slot = sm.slots + q * 4096;
      const uint32_t tbase =
          tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * BN);
      if (x.up) {
        epilogue_tile<BN, EPI_UP>(g.up, x.m, x.n, 0, tbase, q, lane, slot, epi_consts);
        if (x.m < m_tiles) {
          fence_proxy_async_global();
          __threadfence();
          __syncwarp();
          if (lane == 0) atomicAdd(g.ready + x.m * g.down.splits + x.n / g.band, 1);
        }
      } else {
        epilogue_tile<BN, kEpiF32>(g.down, x.m, x.n, x.split, tbase, q, lane, slot, epi_consts);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(&tempty[b], 0));
    }
  } else if constexpr (C::PACKED) {
    if (warp == 6) {
      if (lane == 0) {
        int it = 0;
        bool ok = true;
        for (int u = pair; u < total && ok && !*abort_flag; u += npairs) {
          const Unit x = decode(u);
          const GemmArgs& ga = x.up ? g.up : g.down;
          for (int kb = x.kb0; kb < x.kb1 && ok; ++kb, ++it)
            ok = PackedPipe2<PK>::load(sm, ga.wpack, ga.kb_total, 2 * x.n + static_cast<int>(rank),
                                       kb, it, status);
        }
        PackedPipe2<PK>::drain(sm, it);
      }
    } else {
      const int t = threadIdx.x - 224;
      int it = 0;
      bool ok = true;
      for (int u = pair; u < total && ok; u += npairs) {
        const Unit x = decode(u);
        for (int kb = x.kb0; kb < x.kb1 && ok; ++kb, ++it)
          ok = PackedPipe2<PK>::convert(sm, it, t, status);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool make_tmap_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer,
                  uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, char* err,
                  size_t errlen) {
  const uint64_t dims[2] = {inner, outer};
  const uint64_t strides[1] = {row_bytes};
  const uint32_t box[2] = {box_inner, box_outer};
  return make_tmap_f16(m, base, 2, dims, strides, box, err, errlen);
}

// N-fastest tile order when the A rows outweigh the weight rows four to one.
int n_fast_order(int m, int n) { return static_cast<int64_t>(m) > 4 * static_cast<int64_t>(n) ? 1 : 0; }

// The epilogues that have packed-weight kernels.
constexpr bool packed_epi(int epi) {
  return epi == kEpiF32 || epi == kEpiF16 || epi == kEpiGeGluTanh || epi == kEpiGeGluErf ||
         epi == kEpiQkPrep;
}

template <int BN, int EPI>
void set_smem_attr() {
  cudaFuncSetAttribute(gemm_kernel<BN, EPI, kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       Cfg<BN>::SMEM);
  if constexpr (packed_epi(EPI)) {
    cudaFuncSetAttribute(gemm_kernel<BN, EPI, kQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Cfg<BN, kQ4>::SMEM);
    cudaFuncSetAttribute(gemm_kernel<BN, EPI, kQ8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Cfg<BN, kQ8>::SMEM);
  }
}

template <int EPI>
void set_smem_attr_pair() {
  cudaFuncSetAttribute(gemm2_kernel<EPI, kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       Cfg2<>::SMEM);
  if constexpr (packed_epi(EPI)) {
    cudaFuncSetAttribute(gemm2_kernel<EPI, kQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Cfg2<kQ4>::SMEM);
    cudaFuncSetAttribute(gemm2_kernel<EPI, kQ8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Cfg2<kQ8>::SMEM);
  }
}

template <int EPI, int PK>
void launch_pair_pk(const GemmPlan& p, const GemmArgs& a, int grid, cudaStream_t stream) {
  using C = Cfg2<PK>;
  launch_pdl(gemm2_kernel<EPI, PK>, dim3(grid), dim3(C::THREADS), C::SMEM, stream, p.a, p.b_half,
             a);
}

template <int EPI>
void launch_pair(const GemmPlan& p, const GemmArgs& a0, cudaStream_t stream) {
  GemmArgs a = a0;
  a.wpack = p.wpack;
  const int pairs = ((a.m_tiles + 1) / 2) * a.n_tiles * a.splits;
  const int max_pairs = p.num_sms / 2;
  const int grid = 2 * (pairs < max_pairs ? pairs : max_pairs);
  if constexpr (packed_epi(EPI)) {
    if (p.pk == kQ4) return launch_pair_pk<EPI, kQ4>(p, a, grid, stream);
    if (p.pk == kQ8) return launch_pair_pk<EPI, kQ8>(p, a, grid, stream);
  }
  launch_pair_pk<EPI, kF16>(p, a, grid, stream);
}

template <int BN, int EPI, int PK>
void launch_pk(const GemmPlan& p, const GemmArgs& a, int grid, cudaStream_t stream) {
  using C = Cfg<BN, PK>;
  launch_pdl(gemm_kernel<BN, EPI, PK>, dim3(grid), dim3(C::THREADS), C::SMEM, stream, p.a, p.b, a);
}

template <int BN, int EPI>
void launch(const GemmPlan& p, const GemmArgs& a0, cudaStream_t stream) {
  GemmArgs a = a0;
  a.wpack = p.wpack;
  const int total = a.m_tiles * a.n_tiles * a.splits;
  const int grid = total < p.num_sms ? total : p.num_sms;
  if constexpr (packed_epi(EPI)) {
    if (p.pk == kQ4) return launch_pk<BN, EPI, kQ4>(p, a, grid, stream);
    if (p.pk == kQ8) return launch_pk<BN, EPI, kQ8>(p, a, grid, stream);
  }
  launch_pk<BN, EPI, kF16>(p, a, grid, stream);
}

}  // namespace

bool make_tmap_f16(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides, const uint32_t* box, char* err, size_t errlen) {
  auto fn = encode_fn();
  if (!fn) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled is not available from the driver");
    return false;
  }
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides[i];
  }
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, static_cast<cuuint32_t>(rank),
                  const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(err, errlen, "cuTensorMapEncodeTiled failed (%d) for a rank-%d map, dims [%llu x %llu]",
             static_cast<int>(r), rank, static_cast<unsigned long long>(dims[0]),
             static_cast<unsigned long long>(dims[rank - 1]));
    return false;
  }
  return true;
}

void gemm_setup_device() {
  cudaFuncSetAttribute(gemm_mlp_kernel<kEpiGeGluTanh, kF16>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<256>::SMEM);
  cudaFuncSetAttribute(gemm_mlp_kernel<kEpiGeGluErf, kF16>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<256>::SMEM);
  cudaFuncSetAttribute(gemm_mlp_kernel<kEpiGeGluTanh, kQ4>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<256, kQ4>::SMEM);
  cudaFuncSetAttribute(gemm_mlp_kernel<kEpiGeGluTanh, kQ8>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<256, kQ8>::SMEM);
  cudaFuncSetAttribute(gemm_mlp_kernel<kEpiGeGluErf, kQ4>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<256, kQ4>::SMEM);
  cudaFuncSetAttribute(gemm_mlp_kernel<kEpiGeGluErf, kQ8>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<256, kQ8>::SMEM);
  set_smem_attr<128, kEpiF32>();
  set_smem_attr<256, kEpiF32>();
  set_smem_attr<128, kEpiF16>();
  set_smem_attr<256, kEpiF16>();
  set_smem_attr<256, kEpiGeGluTanh>();
  set_smem_attr<256, kEpiGeGluErf>();
  set_smem_attr<128, kEpiRopeF16>();
  set_smem_attr<256, kEpiRopeF16>();
  set_smem_attr<128, kEpiBiasF16>();
  set_smem_attr<256, kEpiBiasF16>();
  set_smem_attr<128, kEpiBiasReluF16>();
  set_smem_attr<256, kEpiBiasReluF16>();
  set_smem_attr<128, kEpiResidF32>();
  set_smem_attr<256, kEpiResidF32>();
  set_smem_attr<256, kEpiQkPrep>();
  cudaFuncSetAttribute(gemm_mlp2_kernel<kEpiGeGluTanh, kF16>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg2<>::SMEM);
  cudaFuncSetAttribute(gemm_mlp2_kernel<kEpiGeGluErf, kF16>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg2<>::SMEM);
  cudaFuncSetAttribute(gemm_mlp2_kernel<kEpiGeGluTanh, kQ4>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg2<kQ4>::SMEM);
  cudaFuncSetAttribute(gemm_mlp2_kernel<kEpiGeGluTanh, kQ8>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg2<kQ8>::SMEM);
  cudaFuncSetAttribute(gemm_mlp2_kernel<kEpiGeGluErf, kQ4>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg2<kQ4>::SMEM);
  cudaFuncSetAttribute(gemm_mlp2_kernel<kEpiGeGluErf, kQ8>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg2<kQ8>::SMEM);
  set_smem_attr_pair<kEpiF32>();
  set_smem_attr_pair<kEpiF16>();
  set_smem_attr_pair<kEpiGeGluTanh>();
  set_smem_attr_pair<kEpiGeGluErf>();
  set_smem_attr_pair<kEpiRopeF16>();
  set_smem_attr_pair<kEpiResidF32>();
  set_smem_attr_pair<kEpiBiasF16>();
  set_smem_attr_pair<kEpiBiasReluF16>();
  set_smem_attr_pair<kEpiQkPrep>();
}

bool gemm_plan_pair(GemmPlan* p, const void* w, int w_rows, bool always, char* err,
                    size_t errlen) {
  if (p->s.bn != 256) {
    snprintf(err, errlen, "gemm: the CTA-pair kernel needs BN 256 (got %d)", p->s.bn);
    return false;
  }
  switch (p->s.epi) {
    case kEpiF32: case kEpiF16: case kEpiGeGluTanh: case kEpiGeGluErf: case kEpiRopeF16:
    case kEpiBiasF16: case kEpiBiasReluF16: case kEpiResidF32: case kEpiQkPrep:
      break;
    default:
      snprintf(err, errlen, "gemm: no CTA-pair kernel for epilogue %d", p->s.epi);
      return false;
  }
  // Packed weights: each CTA bulk-copies its own chunks instead.
  if (p->pk == kF16 &&
      !make_tmap_2d(&p->b_half, w, p->s.k, w_rows, static_cast<uint64_t>(p->s.k) * 2, BK, 128, err,
                    errlen))
    return false;
  p->s.pair = always ? 2 : 1;
  return true;
}

// Whether a launch over `m` rows takes the CTA-pair kernel.
bool use_pair(const GemmPlan& p, int m) {
  const int min_tiles = p.pk == kF16 ? kPairMinTiles : kPairMinTilesPacked;
  return p.s.pair == 2 || (p.s.pair == 1 && (m + BM - 1) / BM >= min_tiles);
}

void gemm_pick(int n, int k, int num_sms, int* bn, int* splits) {
  // BN 256 moves half the operand bytes per FLOP of BN 128 and measured
  // faster at every projection shape (1.46 vs 1.02 PFLOP/s at 8192^3). Split
  // K into s slabs (the consumer adds them in a fixed order) when that cuts
  // the rounds of tiles per SM: cost ~ ceil(tiles * s / SMs) / s, for a
  // nominal 7 row tiles (a ~900-token pass). The choice depends on (N, K)
  // only, so a row's result never depends on how many rows share its pass.
  const int kb = (k + BK - 1) / BK;
  *bn = n <= 128 ? 128 : 256;
  const int tiles = 7 * ((n + *bn - 1) / *bn);
  const int sms = num_sms > 0 ? num_sms : 148;
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= 2; ++s) {
    if (kb < 16 * s) break;  // keep >= 16 K blocks per slab
    const int rounds = (tiles * s + sms - 1) / sms;
    const double cost = static_cast<double>(rounds) / s + (s > 1 ? 0.05 : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  *splits = best;
}

bool gemm_plan_packed(GemmPlan* p, const void* a, int a_rows_cap, int lda, const void* wpack,
                      int dtype, int w_rows, int n_out, int k, int epi, int bn, int splits,
                      char* err, size_t errlen) {
  if (dtype != kQ4 && dtype != kQ8) {
    snprintf(err, errlen, "gemm: packed weights are Q4_0 or Q8_0 (dtype %d)", dtype);
    return false;
  }
  if (!packed_epi(epi)) {
    snprintf(err, errlen, "gemm: no packed-weight kernel for epilogue %d", epi);
    return false;
  }
  if (k % 32 != 0) {
    snprintf(err, errlen, "gemm: packed weights need K %% 32 == 0 (K %d)", k);
    return false;
  }
  if (!gemm_plan(p, a, a_rows_cap, lda, nullptr, w_rows, n_out, k, epi, bn, splits, err, errlen))
    return false;
  p->pk = dtype;
  p->wpack = static_cast<const uint8_t*>(wpack);
  return true;
}

bool gemm_plan(GemmPlan* p, const void* a, int a_rows_cap, int lda, const void* w, int w_rows,
               int n_out, int k, int epi, int bn, int splits, char* err, size_t errlen) {
  memset(p, 0, sizeof(*p));
  p->pk = kF16;
  if (k % 8 != 0 || lda % 8 != 0) {
    snprintf(err, errlen, "gemm: K %d and lda %d must be multiples of 8", k, lda);
    return false;
  }
  if (epi == kEpiGeGluTanh || epi == kEpiGeGluErf || epi == kEpiQkPrep) {
    bn = 256;
    splits = 1;
  }
  if (epi != kEpiF32) splits = 1;
  if (bn != 128 && bn != 256) {
    snprintf(err, errlen, "gemm: BN %d", bn);
    return false;
  }
  const int kb = (k + BK - 1) / BK;
  if (splits < 1 || splits > kb) splits = 1;
  // Every slab must own at least one K block.
  while (splits > 1 && (splits - 1) * ((kb + splits - 1) / splits) >= kb) --splits;
  p->rows_cap = a_rows_cap;
  int dev = 0;
  cudaGetDevice(&dev);
  p->num_sms = 148;
  cudaDeviceGetAttribute(&p->num_sms, cudaDevAttrMultiProcessorCount, dev);
  p->s.n_out = n_out;
  p->s.k = k;
  p->s.bn = bn;
  p->s.splits = splits;
  p->s.epi = epi;
  if (epi == kEpiGeGluTanh || epi == kEpiGeGluErf)
    p->s.n_tiles = (n_out + 127) / 128;
  else
    p->s.n_tiles = (n_out + bn - 1) / bn;
  if (!make_tmap_2d(&p->a, a, k, a_rows_cap, static_cast<uint64_t>(lda) * 2, BK, BM, err, errlen))
    return false;
  // A packed plan (w null) reads its weight through bulk copies instead.
  if (w && !make_tmap_2d(&p->b, w, k, w_rows, static_cast<uint64_t>(k) * 2, BK, bn, err, errlen))
    return false;
  return true;
}

void gemm_run(const GemmPlan& p, int m, void* out, int ldo, size_t split_stride, uint32_t* status,
              cudaStream_t stream) {
  if (m <= 0) return;
  GemmArgs a;
  a.m = m;
  a.n_out = p.s.n_out;
  a.kb_total = (p.s.k + BK - 1) / BK;
  a.kb_per_split = (a.kb_total + p.s.splits - 1) / p.s.splits;
  a.out = out;
  a.ldo = ldo;
  a.split_stride = split_stride;
  a.status = status;
  a.m_tiles = (m + BM - 1) / BM;
  a.n_tiles = p.s.n_tiles;
  a.splits = p.s.splits;
  a.n_fast = n_fast_order(m, p.s.n_tiles * p.s.bn);
  if (use_pair(p, m)) {
    switch (p.s.epi) {
      case kEpiF32: launch_pair<kEpiF32>(p, a, stream); break;
      case kEpiF16: launch_pair<kEpiF16>(p, a, stream); break;
      case kEpiGeGluTanh: launch_pair<kEpiGeGluTanh>(p, a, stream); break;
      case kEpiGeGluErf: launch_pair<kEpiGeGluErf>(p, a, stream); break;
      default: break;
    }
    return;
  }
  switch (p.s.epi) {
    case kEpiF32:
      if (p.s.bn == 256)
        launch<256, kEpiF32>(p, a, stream);
      else
        launch<128, kEpiF32>(p, a, stream);
      break;
    case kEpiF16:
      if (p.s.bn == 256)
        launch<256, kEpiF16>(p, a, stream);
      else
        launch<128, kEpiF16>(p, a, stream);
      break;
    case kEpiGeGluTanh:
      launch<256, kEpiGeGluTanh>(p, a, stream);
      break;
    case kEpiGeGluErf:
      launch<256, kEpiGeGluErf>(p, a, stream);
      break;
    default:
      break;
  }
}

void gemm_run_epi(const GemmPlan& p, int m, void* out, int ldo, const GemmEpi& epi,
                  uint32_t* status, cudaStream_t stream) {
  if (m <= 0) return;
  GemmArgs a;
  a.m = m;
  a.n_out = p.s.n_out;
  a.kb_total = (p.s.k + BK - 1) / BK;
  a.kb_per_split = a.kb_total;
  a.out = out;
  a.ldo = ldo;
  a.split_stride = 0;
  a.status = status;
  a.m_tiles = (m + BM - 1) / BM;
  a.n_tiles = p.s.n_tiles;
  a.splits = 1;
  a.n_fast = n_fast_order(m, p.s.n_tiles * p.s.bn);
  a.epi = epi;
  const bool wide = p.s.bn == 256;
  if (use_pair(p, m)) {
    switch (p.s.epi) {
      case kEpiRopeF16: launch_pair<kEpiRopeF16>(p, a, stream); break;
      case kEpiBiasF16: launch_pair<kEpiBiasF16>(p, a, stream); break;
      case kEpiBiasReluF16: launch_pair<kEpiBiasReluF16>(p, a, stream); break;
      case kEpiResidF32: launch_pair<kEpiResidF32>(p, a, stream); break;
      case kEpiQkPrep: launch_pair<kEpiQkPrep>(p, a, stream); break;
      default: break;
    }
    return;
  }
  switch (p.s.epi) {
    case kEpiRopeF16:
      wide ? launch<256, kEpiRopeF16>(p, a, stream) : launch<128, kEpiRopeF16>(p, a, stream);
      break;
    case kEpiBiasF16:
      wide ? launch<256, kEpiBiasF16>(p, a, stream) : launch<128, kEpiBiasF16>(p, a, stream);
      break;
    case kEpiBiasReluF16:
      wide ? launch<256, kEpiBiasReluF16>(p, a, stream)
           : launch<128, kEpiBiasReluF16>(p, a, stream);
      break;
    case kEpiResidF32:
      wide ? launch<256, kEpiResidF32>(p, a, stream) : launch<128, kEpiResidF32>(p, a, stream);
      break;
    case kEpiQkPrep:
      launch<256, kEpiQkPrep>(p, a, stream);
      break;
    default:
      gemm_run(p, m, out, ldo, 0, status, stream);
      break;
  }
}


bool gemm_mlp_ok(const GemmPlan& up, const GemmPlan& down) {
  const int kb_up = (up.s.k + BK - 1) / BK;
  const int kb_dn = (down.s.k + BK - 1) / BK;
  // Down split s must read exactly the columns of up column tiles
  // [s * band, (s + 1) * band) (an up tile stores 128 activation columns).
  // Up and down units may differ in length (kb_up vs kb_split K blocks).
  const int kb_split = (kb_dn + down.s.splits - 1) / down.s.splits;
  return up.pk == down.pk && (up.s.epi == kEpiGeGluTanh || up.s.epi == kEpiGeGluErf) &&
         up.s.bn == 256 && kb_up >= 1 &&
         down.s.epi == kEpiF32 && down.s.bn == 256 &&
         kb_dn == kb_split * down.s.splits && kb_split % 2 == 0 &&
         up.s.n_tiles == down.s.splits * (kb_split / 2) && up.s.n_out == down.s.k;
}

void gemm_run_mlp(const GemmPlan& up, const GemmPlan& down, int m, void* act, int ld_act,
                  void* slabs, int ld_slab, size_t split_stride, int* ready, int ready_target,
                  uint32_t* status, cudaStream_t stream, int force_pair, long long wait_limit) {
  if (m <= 0) return;
  // force_pair: -1 by row tiles, 0 one-CTA tiles, 1 CTA pairs (kernel tests).
  const int min_tiles = up.pk == kF16 ? kPairMlpMinTiles : kPairMinTilesPacked;
  const bool pair = up.s.pair && down.s.pair &&
                    (force_pair >= 0 ? force_pair == 1 : (m + BM - 1) / BM >= min_tiles);
  MlpArgs a{};
  auto fill = [&](GemmArgs& x, const GemmPlan& p, void* out, int ldo, size_t stride) {
    x.m = m;
    x.n_out = p.s.n_out;
    x.kb_total = (p.s.k + BK - 1) / BK;
    x.kb_per_split = (x.kb_total + p.s.splits - 1) / p.s.splits;
    x.out = out;
    x.ldo = ldo;
    x.split_stride = stride;
    x.status = status;
    x.m_tiles = (m + BM - 1) / BM;
    x.n_tiles = p.s.n_tiles;
    x.splits = p.s.splits;
  };
  fill(a.up, up, act, ld_act, 0);
  fill(a.down, down, slabs, ld_slab, split_stride);
  a.up.splits = 1;
  a.ready = ready;
  a.ready_target = ready_target;
  a.wait_limit = wait_limit > 0 ? wait_limit : kWaitLimitClocks;
  a.band = a.down.kb_per_split / 2;
  a.up.wpack = up.wpack;
  a.down.wpack = down.wpack;
  const bool tanh_ = up.s.epi == kEpiGeGluTanh;
  if (pair) {
    const int m_pairs = (a.up.m_tiles + 1) / 2;
    const int units = m_pairs * (a.up.n_tiles + a.down.n_tiles * a.down.splits);
    const int max_pairs = up.num_sms / 2;
    const int grid = 2 * (units < max_pairs ? units : max_pairs);
    auto go = [&](auto kernel, int threads, int smem) {
      launch_pdl(kernel, dim3(grid), dim3(threads), smem, stream, up.a, up.b_half, down.a,
                 down.b_half, a);
    };
    if (up.pk == kQ4)
      tanh_ ? go(gemm_mlp2_kernel<kEpiGeGluTanh, kQ4>, Cfg2<kQ4>::THREADS, Cfg2<kQ4>::SMEM)
            : go(gemm_mlp2_kernel<kEpiGeGluErf, kQ4>, Cfg2<kQ4>::THREADS, Cfg2<kQ4>::SMEM);
    else if (up.pk == kQ8)
      tanh_ ? go(gemm_mlp2_kernel<kEpiGeGluTanh, kQ8>, Cfg2<kQ8>::THREADS, Cfg2<kQ8>::SMEM)
            : go(gemm_mlp2_kernel<kEpiGeGluErf, kQ8>, Cfg2<kQ8>::THREADS, Cfg2<kQ8>::SMEM);
    else
      tanh_ ? go(gemm_mlp2_kernel<kEpiGeGluTanh, kF16>, 192, Cfg2<>::SMEM)
            : go(gemm_mlp2_kernel<kEpiGeGluErf, kF16>, 192, Cfg2<>::SMEM);
    return;
  }
  const int total = a.up.m_tiles * a.up.n_tiles + a.down.m_tiles * a.down.n_tiles * a.down.splits;
  const int grid = total < up.num_sms ? total : up.num_sms;
  auto go = [&](auto kernel, int threads, int smem) {
    launch_pdl(kernel, dim3(grid), dim3(threads), smem, stream, up.a, up.b, down.a, down.b, a);
  };
  if (up.pk == kQ4)
    tanh_ ? go(gemm_mlp_kernel<kEpiGeGluTanh, kQ4>, Cfg<256, kQ4>::THREADS, Cfg<256, kQ4>::SMEM)
          : go(gemm_mlp_kernel<kEpiGeGluErf, kQ4>, Cfg<256, kQ4>::THREADS, Cfg<256, kQ4>::SMEM);
  else if (up.pk == kQ8)
    tanh_ ? go(gemm_mlp_kernel<kEpiGeGluTanh, kQ8>, Cfg<256, kQ8>::THREADS, Cfg<256, kQ8>::SMEM)
          : go(gemm_mlp_kernel<kEpiGeGluErf, kQ8>, Cfg<256, kQ8>::THREADS, Cfg<256, kQ8>::SMEM);
  else
    tanh_ ? go(gemm_mlp_kernel<kEpiGeGluTanh, kF16>, 192, Cfg<256>::SMEM)
          : go(gemm_mlp_kernel<kEpiGeGluErf, kF16>, 192, Cfg<256>::SMEM);
}

}  // namespace omg
