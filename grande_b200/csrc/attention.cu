// Block-causal GQA flash attention on mma.sync (see attention.cuh): the
// head_dim-512 layers of Gemma-4-style models (head_dim 256 runs on the
// tensor-core kernel in attention_tc.cu).
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
      any |= attn_visible(qpos[qi], qseq[qi], kpos[kk], kseq[kk], g.window);
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
        if (!attn_visible(qpa, qsa, kp, kq, g.window)) s[nt][e] = -INFINITY;
        if (!attn_visible(qpb, qsb, kp, kq, g.window)) s[nt][2 + e] = -INFINITY;
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

}  // namespace

void attention_setup_device() {
  attention_flash_setup_device();
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
  else
    attention_kernel<256><<<grid, AttnCfg<256>::THREADS, AttnCfg<256>::SMEM, s>>>(a);
}

}  // namespace omg
