// Block-causal GQA flash attention (see attention.cuh).
//
// One CTA = 64 query rows of one KV head: 64/hpg tokens x the hpg query heads
// that share the head, so every K/V tile staged in shared memory serves all
// of them. Keys stream in tiles aligned to absolute cache rows (64 keys at
// head_dim 256, 32 at 512); a tile is skipped when no row of the CTA can see
// any of its keys, and only cache rows [min row_lo, max own row] are
// visited, so a pass holding many branches costs each its own length
// (attention.wgsl:134-199 does the same with its krange / run test).
//
// Warps: 4 row groups x (head_dim / 128) column groups. A warp computes the
// partial scores of its 16 rows over its 128 dims with mma.sync
// (m16n8k16, f16 in, f32 accumulate); the partials meet in shared memory,
// every warp of a row group then runs the same online softmax on the full
// scores and accumulates P.V for its 128 output dims.
#include <climits>

#include "attention.cuh"
#include "ptx.cuh"

namespace omg {

namespace {

constexpr int QROWS = 64;
constexpr float kLog2e = 1.4426950408889634f;

template <int HD>
struct AttnCfg {
  static constexpr int KT = HD == 256 ? 64 : 32;
  static constexpr int NC = HD / 128;
  static constexpr int THREADS = 4 * NC * 32;
  static constexpr int ROWB = HD * 2;
  static constexpr int Q_BYTES = QROWS * ROWB;
  static constexpr int K_BYTES = KT * ROWB;
  static constexpr int SP_STRIDE = KT + 8;
  static constexpr int SP_BYTES = NC * QROWS * SP_STRIDE * 4;
  static constexpr int META_BYTES = (2 * QROWS + 2 * KT + 4) * 4;
  static constexpr int SMEM = Q_BYTES + 2 * K_BYTES + SP_BYTES + META_BYTES;
};

__device__ __forceinline__ uint32_t swz(int row, int chunk, int row_bytes) {
  return static_cast<uint32_t>(row * row_bytes + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float x, float y) {
  __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}

// (x, y) as an f16 pair `hi` plus the f16 pair `lo` of what hi missed.
__device__ __forceinline__ void split_half2(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 hf = __half22float2(h);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = pack_half2(x - hf.x, y - hf.y);
}

// attention.wgsl:70-76 (groups: engine.rs SEQ_GROUP_SHIFT = 12).
__device__ __forceinline__ bool visible(int qp, int qs, int kp, int ks, int window) {
  const bool same_group = ((ks ^ qs) >> 12) == 0;
  return same_group && ((ks & 0xfff) == 0 || ks == qs) && kp <= qp &&
         (window == 0 || static_cast<unsigned>(qp - kp) < static_cast<unsigned>(window));
}

template <int HD>
__global__ void __launch_bounds__(AttnCfg<HD>::THREADS, 1) attention_kernel(AttnArgs g) {
  using C = AttnCfg<HD>;
  constexpr int KT = C::KT;
  constexpr int NT = KT / 8;     // key n-tiles
  constexpr int CH = HD / 8;     // 16-byte chunks per row
  constexpr int ROWB = C::ROWB;
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* qs = sm;
  uint8_t* ks = qs + C::Q_BYTES;
  uint8_t* vs = ks + C::K_BYTES;
  float* sp = reinterpret_cast<float*>(vs + C::K_BYTES);
  int* qpos = reinterpret_cast<int*>(sp + C::NC * QROWS * C::SP_STRIDE);
  int* qseq = qpos + QROWS;
  int* kpos = qseq + QROWS;
  int* kseq = kpos + KT;
  int* range = kseq + KT;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rg = warp & 3, cg = warp >> 2;
  const int hpg = g.heads / g.kv_heads;
  const int kvh = blockIdx.y;
  // This CTA's tokens: one run of one request group (attention_schedule).
  const int2 cta = g.ctas[blockIdx.x];
  const int tok0 = cta.x, tend = cta.x + cta.y;
  const int qt = cta.y;
  const int nkeys = g.base + g.t;
  const size_t row_stride = static_cast<size_t>(2) * g.kv_heads * HD;
  const uint32_t qs_a = smem_u32(qs), ks_a = smem_u32(ks), vs_a = smem_u32(vs);

  for (int i = tid; i < QROWS * CH; i += C::THREADS) {
    const int r = i / CH, c = i % CH;
    const int tok = tok0 + r / hpg, head = kvh * hpg + r % hpg;
    const bool ok = tok < tend;
    const __half* src =
        ok ? g.q + static_cast<size_t>(tok) * g.heads * HD + head * HD + c * 8 : g.q;
    cp_async16(qs_a + swz(r, c, ROWB), src, ok);
  }
  cp_async_commit();
  if (tid < QROWS) {
    const int tok = tok0 + tid / hpg;
    if (tok < tend) {
      const TokMeta m = g.meta[g.base + tok];
      qpos[tid] = m.pos;
      qseq[tid] = m.seq;
    } else {
      qpos[tid] = -1;
      qseq[tid] = -2;
    }
  }
  if (tid == 0) {
    int lo = INT_MAX, hi = 0;
    for (int i = 0; i < qt; ++i) {
      const int tok = tok0 + i;
      {
        const TokMeta m = g.meta[g.base + tok];
        lo = min(lo, m.row_lo);
        hi = max(hi, m.row_hi);
      }
    }
    range[0] = lo == INT_MAX ? 0 : lo;
    range[1] = min(hi, nkeys);
  }
  __syncthreads();
  const int klo = range[0], khi = range[1];

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const int r_a = 16 * rg + (lane >> 2);
  const int r_b = r_a + 8;

  // Key tiles start at the group's first cache row, so a group's keys fall
  // into the same tile slots wherever the group sits in the cache and its
  // rows come out bit-identical in any packing.
  for (int j0 = klo; j0 < khi; j0 += KT) {
    __syncthreads();
    if (tid < KT) {
      const int j = j0 + tid;
      if (j < nkeys) {
        const TokMeta m = g.meta[j];
        kpos[tid] = m.pos;
        kseq[tid] = m.seq;
      } else {
        kpos[tid] = INT_MAX;
        kseq[tid] = -3;
      }
    }
    __syncthreads();
    bool any = false;
    for (int i = tid; i < qt * KT; i += C::THREADS) {
      const int qi = (i / KT) * hpg;
      const int kk = i % KT;
      any |= visible(qpos[qi], qseq[qi], kpos[kk], kseq[kk], g.window);
    }
    if (!__syncthreads_or(any)) continue;

    for (int i = tid; i < KT * CH; i += C::THREADS) {
      const int r = i / CH, c = i % CH;
      const int j = j0 + r;
      const bool ok = j < nkeys;
      const __half* base = g.kv + static_cast<size_t>(ok ? j : 0) * row_stride + c * 8;
      cp_async16(ks_a + swz(r, c, ROWB), base + kvh * HD, ok);
      cp_async16(vs_a + swz(r, c, ROWB), base + (g.kv_heads + kvh) * HD, ok);
    }
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();

    // Partial scores over this warp's 128 dims.
    float s[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int chunk0 = cg * 16 + kk * 2;
      uint32_t a[4];
      ldsm_x4(qs_a + swz(16 * rg + (lane & 15), chunk0 + (lane >> 4), ROWB), a);
#pragma unroll
      for (int nt = 0; nt < NT; nt += 2) {
        uint32_t b[4];
        ldsm_x4(ks_a + swz(nt * 8 + (lane & 7) + ((lane >> 4) << 3), chunk0 + ((lane >> 3) & 1),
                           ROWB),
                b);
        mma16816(s[nt], a, b[0], b[1]);
        mma16816(s[nt + 1], a, b[2], b[3]);
      }
    }
    if constexpr (C::NC > 1) {
      float* spw = sp + cg * QROWS * C::SP_STRIDE;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int col = nt * 8 + 2 * (lane & 3);
        *reinterpret_cast<float2*>(spw + r_a * C::SP_STRIDE + col) = make_float2(s[nt][0], s[nt][1]);
        *reinterpret_cast<float2*>(spw + r_b * C::SP_STRIDE + col) = make_float2(s[nt][2], s[nt][3]);
      }
      __syncthreads();
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int col = nt * 8 + 2 * (lane & 3);
        float2 x = *reinterpret_cast<const float2*>(sp + r_a * C::SP_STRIDE + col);
        float2 y = *reinterpret_cast<const float2*>(sp + r_b * C::SP_STRIDE + col);
#pragma unroll
        for (int c2 = 1; c2 < C::NC; ++c2) {
          const float2 x2 =
              *reinterpret_cast<const float2*>(sp + (c2 * QROWS + r_a) * C::SP_STRIDE + col);
          const float2 y2 =
              *reinterpret_cast<const float2*>(sp + (c2 * QROWS + r_b) * C::SP_STRIDE + col);
          x.x += x2.x;
          x.y += x2.y;
          y.x += y2.x;
          y.y += y2.y;
        }
        s[nt][0] = x.x;
        s[nt][1] = x.y;
        s[nt][2] = y.x;
        s[nt][3] = y.y;
      }
    }
    // Mask and online softmax for rows r_a (s[][0..1]) and r_b (s[][2..3]).
    const int qpa = qpos[r_a], qsa = qseq[r_a], qpb = qpos[r_b], qsb = qseq[r_b];
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = nt * 8 + 2 * (lane & 3) + e;
        const int kp = kpos[col], kq = kseq[col];
        if (!visible(qpa, qsa, kp, kq, g.window)) s[nt][e] = -INFINITY;
        if (!visible(qpb, qsb, kp, kq, g.window)) s[nt][2 + e] = -INFINITY;
        mx_a = fmaxf(mx_a, s[nt][e]);
        mx_b = fmaxf(mx_b, s[nt][2 + e]);
      }
    }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float mn_a = fmaxf(m_run[0], mx_a), mn_b = fmaxf(m_run[1], mx_b);
    const float sc_a = mn_a == -INFINITY ? 1.f : exp2f((m_run[0] - mn_a) * kLog2e);
    const float sc_b = mn_b == -INFINITY ? 1.f : exp2f((m_run[1] - mn_b) * kLog2e);
    float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float pa = s[nt][e] == -INFINITY ? 0.f : exp2f((s[nt][e] - mn_a) * kLog2e);
        const float pb = s[nt][2 + e] == -INFINITY ? 0.f : exp2f((s[nt][2 + e] - mn_b) * kLog2e);
        s[nt][e] = pa;
        s[nt][2 + e] = pb;
        sum_a += pa;
        sum_b += pb;
      }
    }
    sum_a += __shfl_xor_sync(0xffffffffu, sum_a, 1);
    sum_a += __shfl_xor_sync(0xffffffffu, sum_a, 2);
    sum_b += __shfl_xor_sync(0xffffffffu, sum_b, 1);
    sum_b += __shfl_xor_sync(0xffffffffu, sum_b, 2);
    l_run[0] = l_run[0] * sc_a + sum_a;
    l_run[1] = l_run[1] * sc_b + sum_b;
    m_run[0] = mn_a;
    m_run[1] = mn_b;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= sc_a;
      o[i][1] *= sc_a;
      o[i][2] *= sc_b;
      o[i][3] *= sc_b;
    }
    // P.V on this warp's 128 output dims. The reference keeps P in f32
    // (attention.wgsl:230-268); here P = hi + lo with both halves f16, two
    // MMAs, so P carries ~22 bits and a row's result does not depend on where
    // the tile boundaries fall (the running max at which P was formed).
#pragma unroll
    for (int kk = 0; kk < KT / 16; ++kk) {
      uint32_t a[4], alo[4];
      split_half2(s[2 * kk][0], s[2 * kk][1], a[0], alo[0]);
      split_half2(s[2 * kk][2], s[2 * kk][3], a[1], alo[1]);
      split_half2(s[2 * kk + 1][0], s[2 * kk + 1][1], a[2], alo[2]);
      split_half2(s[2 * kk + 1][2], s[2 * kk + 1][3], a[3], alo[3]);
#pragma unroll
      for (int nt = 0; nt < 16; nt += 2) {
        uint32_t b[4];
        ldsm_x4_t(vs_a + swz(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3),
                             cg * 16 + nt + (lane >> 4), ROWB),
                  b);
        mma16816(o[nt], a, b[0], b[1]);
        mma16816(o[nt + 1], a, b[2], b[3]);
        mma16816(o[nt], alo, b[0], b[1]);
        mma16816(o[nt + 1], alo, b[2], b[3]);
      }
    }
  }

  const int rows[2] = {r_a, r_b};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = rows[h];
    const int tok = tok0 + r / hpg;
    if (tok >= tend) continue;
    const int head = kvh * hpg + r % hpg;
    const float inv = 1.0f / l_run[h];
    __half* orow = g.out + static_cast<size_t>(tok) * g.heads * HD + head * HD + cg * 128;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int col = nt * 8 + 2 * (lane & 3);
      *reinterpret_cast<uint32_t*>(orow + col) =
          pack_half2(o[nt][2 * h] * inv, o[nt][2 * h + 1] * inv);
    }
  }
}

// ---- head_dim 256 ------------------------------------------------------------
//
// Each of the 4 warps owns 16 query rows and all 256 output dims, so scores
// never leave the warp. Keys stream in 32-key tiles, double-buffered with
// cp.async; the CTA first lists the tiles any of its rows can see, and a warp
// skips the 16-key halves none of its own rows can see.

constexpr int K2_KT = 32;
constexpr int K2_ROWS = 64;
constexpr int K2_MAXT = 1024;
constexpr int K2_ROWB = 512;
constexpr int K2_Q_BYTES = K2_ROWS * K2_ROWB;
constexpr int K2_KV_BYTES = K2_KT * K2_ROWB;
constexpr int K2_STAGE = 2 * K2_KV_BYTES;
constexpr int K2_SMEM = K2_Q_BYTES + 2 * K2_STAGE + (4 * K2_KT + 2 * K2_ROWS + K2_MAXT + 8) * 4;

template <bool PLO>
__global__ void __launch_bounds__(128, 2) attention256_kernel(AttnArgs g) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* qs = sm;
  uint8_t* kvs = sm + K2_Q_BYTES;  // [2 stages][K tile | V tile]
  int* kpos = reinterpret_cast<int*>(kvs + 2 * K2_STAGE);  // [2][KT]
  int* kseq = kpos + 2 * K2_KT;                            // [2][KT]
  int* qpos = kseq + 2 * K2_KT;                            // [ROWS]
  int* qseq = qpos + K2_ROWS;                              // [ROWS]
  int* tiles = qseq + K2_ROWS;                             // [MAXT]
  int* misc = tiles + K2_MAXT;                             // ntiles

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hpg = g.heads / g.kv_heads;
  const int kvh = blockIdx.y;
  const int2 cta = g.ctas[blockIdx.x];
  const int tok0 = cta.x, cnt = cta.y;
  const int nkeys = g.base + g.t;
  const size_t row_stride = static_cast<size_t>(2) * g.kv_heads * 256;
  const uint32_t qs_a = smem_u32(qs), kv_a = smem_u32(kvs);

  for (int i = tid; i < K2_ROWS * 32; i += 128) {
    const int r = i >> 5, c = i & 31;
    const int ti = r / hpg;
    const bool ok = ti < cnt;
    const __half* src =
        ok ? g.q + static_cast<size_t>(tok0 + ti) * g.heads * 256 + (kvh * hpg + r % hpg) * 256 +
                 c * 8
           : g.q;
    cp_async16(qs_a + swz(r, c, K2_ROWB), src, ok);
  }
  cp_async_commit();
  if (tid < K2_ROWS) {
    const int ti = tid / hpg;
    if (ti < cnt) {
      const TokMeta m = g.meta[g.base + tok0 + ti];
      qpos[tid] = m.pos;
      qseq[tid] = m.seq;
    } else {
      qpos[tid] = -1;
      qseq[tid] = -2;
    }
  }
  const int klo = g.meta[g.base + tok0].row_lo;
  const int khi = min(g.meta[g.base + tok0 + cnt - 1].row_hi, nkeys);
  __syncthreads();

  float o[32][4];
#pragma unroll
  for (int i = 0; i < 32; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const int r_a = 16 * warp + (lane >> 2), r_b = r_a + 8;
  const int qpa = qpos[r_a], qsa = qseq[r_a], qpb = qpos[r_b], qsb = qseq[r_b];

  // Key-range split: this CTA (blockIdx.z) takes chunk `split` of the visible
  // tiles, chunk_tiles of them; the chunking depends only on this query
  // tile's own key range, so rows are bit-identical in any packing.
  const int split = blockIdx.z;
  const int range_tiles = (khi - klo + K2_KT - 1) / K2_KT;
  const int chunk_tiles = g.nsplit > 1 ? max(4, (range_tiles + 15) / 16) : 1 << 30;
  int seen = 0;  // visible tiles before the current list chunk
  for (int c0 = klo; c0 < khi; c0 += K2_MAXT * K2_KT) {
    const int c1 = min(khi, c0 + K2_MAXT * K2_KT);
    const int nt_all = (c1 - c0 + K2_KT - 1) / K2_KT;
    // Which tiles does any row of this CTA see? Warp w tests tiles w, w+4, ...
    for (int ti = warp; ti < nt_all; ti += 4) {
      const int j = c0 + ti * K2_KT + lane;
      bool vis = false;
      if (j < c1) {
        const TokMeta km = g.meta[j];
        for (int r = 0; r < cnt * hpg && !vis; r += hpg)
          vis = visible(qpos[r], qseq[r], km.pos, km.seq, g.window);
      }
      const unsigned any = __ballot_sync(0xffffffffu, vis);
      if (lane == 0) tiles[ti] = any ? 1 : 0;
    }
    __syncthreads();
    if (tid == 0) {
      int n = 0;
      for (int ti = 0; ti < nt_all; ++ti)
        if (tiles[ti]) tiles[n++] = c0 + ti * K2_KT;
      misc[0] = n;
    }
    __syncthreads();
    const int nvis = misc[0];
    // This split's share of the visible tiles (global visible index range
    // [split * chunk_tiles, (split + 1) * chunk_tiles)).
    const long long lo_g = static_cast<long long>(split) * chunk_tiles;
    const long long hi_g = lo_g + chunk_tiles;
    const int first = static_cast<int>(max(0LL, min(static_cast<long long>(nvis), lo_g - seen)));
    const int last = static_cast<int>(max(0LL, min(static_cast<long long>(nvis), hi_g - seen)));
    seen += nvis;
    const int ntiles = last - first;
    int* tl = tiles + first;

    auto load = [&](int i, int st) {
      const int j0 = tl[i];
      const uint32_t kbase = kv_a + st * K2_STAGE;
      for (int e = tid; e < K2_KT * 32; e += 128) {
        const int r = e >> 5, c = e & 31;
        const int j = j0 + r;
        const bool ok = j < nkeys;
        const __half* src = g.kv + static_cast<size_t>(ok ? j : 0) * row_stride + c * 8;
        cp_async16(kbase + swz(r, c, K2_ROWB), src + kvh * 256, ok);
        cp_async16(kbase + K2_KV_BYTES + swz(r, c, K2_ROWB), src + (g.kv_heads + kvh) * 256, ok);
      }
      if (tid < K2_KT) {
        const int j = j0 + tid;
        if (j < nkeys) {
          const TokMeta m = g.meta[j];
          kpos[st * K2_KT + tid] = m.pos;
          kseq[st * K2_KT + tid] = m.seq;
        } else {
          kpos[st * K2_KT + tid] = INT_MAX;
          kseq[st * K2_KT + tid] = -3;
        }
      }
    };

    if (ntiles > 0) {
      load(0, 0);
      cp_async_commit();
    }
    for (int i = 0; i < ntiles; ++i) {
      const int st = i & 1;
      if (i + 1 < ntiles) {
        load(i + 1, st ^ 1);
        cp_async_commit();
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      } else {
        cp_async_wait_all();
      }
      __syncthreads();
      const int* kp = kpos + st * K2_KT;
      const int* kq = kseq + st * K2_KT;
      const uint32_t ks_a = kv_a + st * K2_STAGE, vs_a = ks_a + K2_KV_BYTES;
      // Which 16-key halves does this warp see at all, and does every one of
      // its rows see every key of the tile? Lane l tests key l against the
      // warp's 16 rows.
      bool v_any = false, v_all = true;
      {
        const int kpp = kp[lane], kqq = kq[lane];
        for (int r = 16 * warp; r < 16 * warp + 16; ++r) {
          const bool vr = visible(qpos[r], qseq[r], kpp, kqq, g.window);
          v_any |= vr;
          v_all &= vr;
        }
      }
      const unsigned vm = __ballot_sync(0xffffffffu, v_any);
      const bool vis0 = (vm & 0xffffu) != 0, vis1 = (vm >> 16) != 0;
      const bool all_vis = __all_sync(0xffffffffu, v_all);

      // Scores: two accumulators per key n-tile (dims 0..127 and 128..255),
      // eight independent MMA chains, added at the end.
      float s[4][4], s2[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        s[a][0] = s[a][1] = s[a][2] = s[a][3] = 0.f;
        s2[a][0] = s2[a][1] = s2[a][2] = s2[a][3] = 0.f;
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a[4], a2[4];
        ldsm_x4(qs_a + swz(16 * warp + (lane & 15), 2 * kk + (lane >> 4), K2_ROWB), a);
        ldsm_x4(qs_a + swz(16 * warp + (lane & 15), 16 + 2 * kk + (lane >> 4), K2_ROWB), a2);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          if (np == 0 ? !vis0 : !vis1) continue;
          uint32_t b[4], b2[4];
          const int krow = np * 16 + (lane & 7) + ((lane >> 4) << 3);
          ldsm_x4(ks_a + swz(krow, 2 * kk + ((lane >> 3) & 1), K2_ROWB), b);
          ldsm_x4(ks_a + swz(krow, 16 + 2 * kk + ((lane >> 3) & 1), K2_ROWB), b2);
          mma16816(s[2 * np], a, b[0], b[1]);
          mma16816(s[2 * np + 1], a, b[2], b[3]);
          mma16816(s2[2 * np], a2, b2[0], b2[1]);
          mma16816(s2[2 * np + 1], a2, b2[2], b2[3]);
        }
      }
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        s[a][0] += s2[a][0];
        s[a][1] += s2[a][1];
        s[a][2] += s2[a][2];
        s[a][3] += s2[a][3];
      }
      float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (!all_vis) {
            const int col = nt * 8 + 2 * (lane & 3) + e;
            const int kpp = kp[col], kqq = kq[col];
            if (!visible(qpa, qsa, kpp, kqq, g.window)) s[nt][e] = -INFINITY;
            if (!visible(qpb, qsb, kpp, kqq, g.window)) s[nt][2 + e] = -INFINITY;
          }
          mx_a = fmaxf(mx_a, s[nt][e]);
          mx_b = fmaxf(mx_b, s[nt][2 + e]);
        }
      }
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
      const float mn_a = fmaxf(m_run[0], mx_a), mn_b = fmaxf(m_run[1], mx_b);
      const float sc_a = mn_a == -INFINITY ? 1.f : exp2f((m_run[0] - mn_a) * kLog2e);
      const float sc_b = mn_b == -INFINITY ? 1.f : exp2f((m_run[1] - mn_b) * kLog2e);
      float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pa = s[nt][e] == -INFINITY ? 0.f : exp2f((s[nt][e] - mn_a) * kLog2e);
          const float pb =
              s[nt][2 + e] == -INFINITY ? 0.f : exp2f((s[nt][2 + e] - mn_b) * kLog2e);
          s[nt][e] = pa;
          s[nt][2 + e] = pb;
          sum_a += pa;
          sum_b += pb;
        }
      }
      sum_a += __shfl_xor_sync(0xffffffffu, sum_a, 1);
      sum_a += __shfl_xor_sync(0xffffffffu, sum_a, 2);
      sum_b += __shfl_xor_sync(0xffffffffu, sum_b, 1);
      sum_b += __shfl_xor_sync(0xffffffffu, sum_b, 2);
      l_run[0] = l_run[0] * sc_a + sum_a;
      l_run[1] = l_run[1] * sc_b + sum_b;
      m_run[0] = mn_a;
      m_run[1] = mn_b;
      // Rescale only when some row's running max moved (x * 1 == x).
      if (!__all_sync(0xffffffffu, sc_a == 1.f && sc_b == 1.f)) {
#pragma unroll
        for (int i2 = 0; i2 < 32; ++i2) {
          o[i2][0] *= sc_a;
          o[i2][1] *= sc_a;
          o[i2][2] *= sc_b;
          o[i2][3] *= sc_b;
        }
      }
#pragma unroll
      for (int kc = 0; kc < 2; ++kc) {
        if (kc == 0 ? !vis0 : !vis1) continue;
        uint32_t a[4], alo[4];
        split_half2(s[2 * kc][0], s[2 * kc][1], a[0], alo[0]);
        split_half2(s[2 * kc][2], s[2 * kc][3], a[1], alo[1]);
        split_half2(s[2 * kc + 1][0], s[2 * kc + 1][1], a[2], alo[2]);
        split_half2(s[2 * kc + 1][2], s[2 * kc + 1][3], a[3], alo[3]);
#pragma unroll
        for (int nt = 0; nt < 32; nt += 2) {
          uint32_t b[4];
          ldsm_x4_t(vs_a + swz(kc * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), nt + (lane >> 4),
                               K2_ROWB),
                    b);
          mma16816(o[nt], a, b[0], b[1]);
          mma16816(o[nt + 1], a, b[2], b[3]);
          if constexpr (PLO) {
            mma16816(o[nt], alo, b[0], b[1]);
            mma16816(o[nt + 1], alo, b[2], b[3]);
          }
        }
      }
      __syncthreads();
    }
    __syncthreads();
  }

  const int rows[2] = {r_a, r_b};
  if (g.nsplit > 1) {
    // Unnormalised partial output, running max and sum of this split.
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = rows[h];
      const int ti = r / hpg;
      if (ti >= cnt) continue;
      const size_t prow =
          (static_cast<size_t>(split) * g.t + tok0 + ti) * g.heads + (kvh * hpg + r % hpg);
      if ((lane & 3) == 0) g.part_ml[prow] = make_float2(m_run[h], l_run[h]);
      if (!(l_run[h] > 0.f)) continue;  // nothing seen: the merge skips this split
      float* orow = g.part_o + prow * 256;
#pragma unroll
      for (int nt = 0; nt < 32; ++nt) {
        const int col = nt * 8 + 2 * (lane & 3);
        *reinterpret_cast<float2*>(orow + col) = make_float2(o[nt][2 * h], o[nt][2 * h + 1]);
      }
    }
    return;
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = rows[h];
    const int ti = r / hpg;
    if (ti >= cnt) continue;
    const float inv = 1.0f / l_run[h];
    __half* orow = g.out + static_cast<size_t>(tok0 + ti) * g.heads * 256 + (kvh * hpg + r % hpg) * 256;
#pragma unroll
    for (int nt = 0; nt < 32; ++nt) {
      const int col = nt * 8 + 2 * (lane & 3);
      *reinterpret_cast<uint32_t*>(orow + col) =
          pack_half2(o[nt][2 * h] * inv, o[nt][2 * h + 1] * inv);
    }
  }
}

// out[row] = sum_s exp(m_s - M) o_s / sum_s exp(m_s - M) l_s over the splits
// in order; splits that saw no key of the row (l = 0) are skipped.
__global__ void __launch_bounds__(64) attention_combine(const float* __restrict__ part_o,
                                                        const float2* __restrict__ part_ml,
                                                        int nsplit, int rows, __half* __restrict__ out) {
  const int row = blockIdx.x;
  if (row >= rows) return;
  float mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s) {
    const float2 ml = part_ml[static_cast<size_t>(s) * rows + row];
    if (ml.y > 0.f) mx = fmaxf(mx, ml.x);
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float den = 0.f;
  const int d = threadIdx.x * 4;
  for (int s = 0; s < nsplit; ++s) {
    const size_t pr = static_cast<size_t>(s) * rows + row;
    const float2 ml = part_ml[pr];
    if (!(ml.y > 0.f)) continue;
    const float w = exp2f((ml.x - mx) * kLog2e);
    const float4 v = *reinterpret_cast<const float4*>(part_o + pr * 256 + d);
    acc.x += w * v.x;
    acc.y += w * v.y;
    acc.z += w * v.z;
    acc.w += w * v.w;
    den += w * ml.y;
  }
  const float inv = 1.0f / den;
  __half* o = out + static_cast<size_t>(row) * 256 + d;
  *reinterpret_cast<__half2*>(o) = __floats2half2_rn(acc.x * inv, acc.y * inv);
  *reinterpret_cast<__half2*>(o + 2) = __floats2half2_rn(acc.z * inv, acc.w * inv);
}

}  // namespace

int attention_splits(const TokMeta* meta, int t, int base, int hpg,
                     const std::vector<int2>& ctas, int hd) {
  if (hd != 256) return 1;
  (void)hpg;
  int best = 1;
  for (const int2& c : ctas) {
    const int klo = meta[c.x].row_lo;
    const int khi = std::min(meta[c.x + c.y - 1].row_hi, base + t);
    const int range = (khi - klo + K2_KT - 1) / K2_KT;
    const int chunk = std::max(4, (range + 15) / 16);
    best = std::max(best, (range + chunk - 1) / chunk);
  }
  return std::min(best, kAttnMaxSplits);
}

void attention_setup_device() {
  cudaFuncSetAttribute(attention256_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       K2_SMEM);
  cudaFuncSetAttribute(attention256_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       K2_SMEM);
  cudaFuncSetAttribute(attention_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       AttnCfg<256>::SMEM);
  cudaFuncSetAttribute(attention_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       AttnCfg<512>::SMEM);
}

void attention_schedule(const TokMeta* meta, int t, int hpg, std::vector<int2>* out) {
  out->clear();
  const int qt = QROWS / hpg;
  for (int i = 0; i < t;) {
    int n = 1;
    while (i + n < t && n < qt && meta[i + n].row_lo == meta[i].row_lo) ++n;
    out->push_back(make_int2(i, n));
    i += n;
  }
}

void launch_attention(const AttnArgs& a, cudaStream_t s) {
  if (a.t <= 0 || a.n_ctas <= 0) return;
  dim3 grid(a.n_ctas, a.kv_heads);
  if (a.hd == 512)
    attention_kernel<512><<<grid, AttnCfg<512>::THREADS, AttnCfg<512>::SMEM, s>>>(a);
  else {
    dim3 g2(a.n_ctas, a.kv_heads, a.nsplit);
    attention256_kernel<true><<<g2, 128, K2_SMEM, s>>>(a);
    if (a.nsplit > 1)
      attention_combine<<<a.t * a.heads, 64, 0, s>>>(a.part_o, a.part_ml, a.nsplit,
                                                      a.t * a.heads, a.out);
  }
}

}  // namespace omg
