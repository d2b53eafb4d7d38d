// Row kernels and the tensor-core bidirectional attention of the Laya /
// ModernBERT encoder (see laya_kernels.cuh). Reference shaders:
// crates/omg-wgpu/src/shaders/{embed,layernorm,rope_bi,attention_bi}.wgsl.
#include <algorithm>
#include <cstdio>

#include "gemm.cuh"
#include "laya_kernels.cuh"
#include "launch.cuh"
#include "ptx.cuh"
#include "quant.cuh"

namespace omg {

namespace {

// ---- RoPE table ---------------------------------------------------------------

__global__ void rope_table_kernel(float theta, int hd, int n_pos, float2* tab) {
  const int half = hd / 2;
  const int n = n_pos * half;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int k = i / n_pos, p = i % n_pos;
    // rope_bi.wgsl:28: angle = pos * pow(theta, -f32(2 d) / f32(HD)).
    const float angle = static_cast<float>(p) * powf(theta, -static_cast<float>(2 * k) /
                                                                static_cast<float>(hd));
    tab[i] = make_float2(cosf(angle), sinf(angle));
  }
}

// ---- LayerNorm helpers ---------------------------------------------------------

constexpr int kLnMaxVec = 16;  // float4 per lane: d <= 2048

// Mean, then the variance around it (layernorm.wgsl:51-61), of a row held as
// float4s by one warp (lane l owns float4 l + 32 k, k < nv).
template <int N>
__device__ __forceinline__ void ln_stats(const float4 (&v)[N], int nv, int d, float eps,
                                         float* mean, float* inv) {
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < N; ++k)
    if (k < nv) s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
  const float m = warp_sum(s) / static_cast<float>(d);
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < N; ++k)
    if (k < nv) {
      const float a = v[k].x - m, b = v[k].y - m, c = v[k].z - m, e = v[k].w - m;
      q += (a * a + b * b) + (c * c + e * e);
    }
  *mean = m;
  *inv = rsqrtf(warp_sum(q) / static_cast<float>(d) + eps);
}

__device__ __forceinline__ float4 ln_apply(float4 v, float mean, float inv, float4 w, float4 b) {
  return make_float4((v.x - mean) * inv * w.x + b.x, (v.y - mean) * inv * w.y + b.y,
                     (v.z - mean) * inv * w.z + b.z, (v.w - mean) * inv * w.w + b.w);
}

__device__ __forceinline__ void store_h4(__half* p, float4 v) {
  const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
  uint2 pk;
  pk.x = *reinterpret_cast<const uint32_t*>(&a);
  pk.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = pk;
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// One warp per row, 8 rows per CTA; NV = d / 128 float4s per lane, so the
// registers a row takes (and with them how many rows an SM keeps in
// flight) follow the row width.
template <int NV>
__global__ void __launch_bounds__(256) laya_ln_kernel(LayaLnArgs a) {
  griddep_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= a.t) return;
  constexpr int nv = NV;
  float* xr = a.x + static_cast<size_t>(row) * a.d;
  float4 v[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) v[k] = ld4(xr + (lane + 32 * k) * 4);
  float mean, inv;
  ln_stats(v, nv, a.d, a.eps, &mean, &inv);
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  __half* hr = a.h16 ? a.h16 + static_cast<size_t>(row) * a.d : nullptr;
  if (!a.in_place) {
#pragma unroll
    for (int k = 0; k < NV; ++k)
      if (k < nv) {
        const int c = (lane + 32 * k) * 4;
        store_h4(hr + c, ln_apply(v[k], mean, inv, ld4(a.w1 + c), a.b1 ? ld4(a.b1 + c) : zero));
      }
    return;
  }
  const float* te = a.type_emb ? a.type_emb + static_cast<size_t>(a.qtype[row]) * a.d : nullptr;
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (k < nv) {
      const int c = (lane + 32 * k) * 4;
      float4 y = ln_apply(v[k], mean, inv, ld4(a.w1 + c), a.b1 ? ld4(a.b1 + c) : zero);
      if (te) {
        // embed.wgsl with residual = 1: the type row is added after the norm.
        const float4 e = ld4(te + c);
        y.x += e.x;
        y.y += e.y;
        y.z += e.z;
        y.w += e.w;
      }
      v[k] = y;
      *reinterpret_cast<float4*>(xr + c) = y;
    }
  if (!a.w2) return;
  ln_stats(v, nv, a.d, a.eps, &mean, &inv);
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (k < nv) {
      const int c = (lane + 32 * k) * 4;
      store_h4(hr + c, ln_apply(v[k], mean, inv, ld4(a.w2 + c), a.b2 ? ld4(a.b2 + c) : zero));
    }
}

// embed.wgsl (scale 1) + layernorm.wgsl: one warp per row; lane l dequantizes
// 32-element blocks l, l + 32, ... into x, then normalises the row.
template <int DT>
__global__ void __launch_bounds__(256)
    laya_embed_ln_kernel(const int* __restrict__ ids, int t, const uint8_t* __restrict__ codes,
                         const uint8_t* __restrict__ scales, int d, const float* __restrict__ w,
                         float eps, float* __restrict__ x, __half* __restrict__ h16) {
  griddep_wait();
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= t) return;
  const size_t id = static_cast<size_t>(ids[row]);
  const int nb = d / 32;
  float* xr = x + static_cast<size_t>(row) * d;
  for (int b = lane; b < nb; b += 32) {
    float e[32];
    load_block_f32<DT>(codes, scales, id * nb + b, e);
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4*>(xr + b * 32 + j) = make_float4(e[j], e[j + 1], e[j + 2], e[j + 3]);
  }
  __syncwarp();
  const int nv = d / 128;
  float4 v[kLnMaxVec];
#pragma unroll
  for (int k = 0; k < kLnMaxVec; ++k)
    if (k < nv) v[k] = ld4(xr + (lane + 32 * k) * 4);
  float mean, inv;
  ln_stats(v, nv, d, eps, &mean, &inv);
  __half* hr = h16 + static_cast<size_t>(row) * d;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int k = 0; k < kLnMaxVec; ++k)
    if (k < nv) {
      const int c = (lane + 32 * k) * 4;
      const float4 y = ln_apply(v[k], mean, inv, ld4(w + c), zero);
      *reinterpret_cast<float4*>(xr + c) = y;
      store_h4(hr + c, y);
    }
}

__global__ void laya_gather_kernel(const float* __restrict__ x, int d, const int* __restrict__ map,
                                   int n, float* __restrict__ rows) {
  griddep_wait();
  const int r = blockIdx.x;
  if (r >= n) return;
  const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(map[r]) * d);
  float4* dst = reinterpret_cast<float4*>(rows + static_cast<size_t>(r) * d);
  for (int i = threadIdx.x; i < d / 4; i += blockDim.x) dst[i] = src[i];
}

// ---- bidirectional attention on the tensor cores ------------------------------
//
// One CTA = one item x one head:
//   warp 0     TMA: Q [128 rows][64 dims] once, then per 128-key tile K and V
//   warp 1     MMA: S = Q K^T (M 128, N 128, K 64) into TMEM columns 0..127;
//              after the softmax, O_j = P V (M 128, N 64, K 128) into columns
//              128..191
//   warps 2-5  one query row per thread (its TMEM lane): masked max over the
//              tile, exp, row sum, P (f16) into shared memory; then fold O_j
//              into the running output in registers; finally out = o / l.
// Two CTAs fit on an SM (83 KB of shared memory and 256 TMEM columns each),
// so one CTA's loads overlap the other's math.

constexpr int LA_CHUNK = kLayaTile * 128;  // [128 rows][128 bytes] f16
constexpr int LA_SMEM = 1024 + 5 * LA_CHUNK + 256;
constexpr uint32_t LA_TMEM_COLS = 256;
constexpr uint32_t LA_TMEM_O = 128;
constexpr float kLog2e = 1.4426950408889634f;

enum { LB_Q = 0, LB_K, LB_V, LB_S, LB_P, LB_O, LB_KFREE, LB_VFREE, LB_N };

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint32_t* status, int lane) {
  int ok = 0;
  if (lane == 0) ok = mbar_wait(bar, parity, abort_flag, status) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__global__ void __launch_bounds__(192, 2)
    laya_attention_kernel(const __grid_constant__ CUtensorMap tqkv, LayaAttnArgs g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* qs = sm;
  uint8_t* ks = qs + LA_CHUNK;
  uint8_t* vs = ks + LA_CHUNK;
  uint8_t* ps = vs + LA_CHUNK;  // 2 chunks: keys 0..63, 64..127
  uint64_t* bars = reinterpret_cast<uint64_t*>(ps + 2 * LA_CHUNK);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + LB_N);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const LayaAttnItem it = g.items[blockIdx.x];
  const int head = blockIdx.y;
  const int ntiles = (it.nk + kLayaTile - 1) / kLayaTile;

  if (threadIdx.x == 0) {
    for (int i = 0; i < LB_N; ++i) mbar_init(&bars[i], i == LB_P ? 4 : 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tqkv);
  }
  if (warp == 1) tmem_alloc(tmem_slot, LA_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars[LB_Q], LA_CHUNK);
      tma_load_2d(qs, &tqkv, &bars[LB_Q], head * kLayaHd, it.q0);
      for (int j = 0; j < ntiles; ++j) {
        const int kt = it.k0 + j * kLayaTile;
        if (j > 0 && !mbar_wait(&bars[LB_KFREE], (j - 1) & 1, abort_flag, g.status)) break;
        mbar_arrive_expect_tx(&bars[LB_K], LA_CHUNK);
        tma_load_2d(ks, &tqkv, &bars[LB_K], g.d + head * kLayaHd, kt);
        if (j > 0 && !mbar_wait(&bars[LB_VFREE], (j - 1) & 1, abort_flag, g.status)) break;
        mbar_arrive_expect_tx(&bars[LB_V], LA_CHUNK);
        tma_load_2d(vs, &tqkv, &bars[LB_V], 2 * g.d + head * kLayaHd, kt);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(128, kLayaTile);
      constexpr uint32_t idesc_o = idesc_f16_f32_bmn(128, kLayaHd);
      bool ok = mbar_wait(&bars[LB_Q], 0, abort_flag, g.status);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (!mbar_wait(&bars[LB_K], j & 1, abort_flag, g.status)) break;
        tc_fence_after();
        const uint64_t da = sw128_desc(qs), db = sw128_desc(ks);
#pragma unroll
        for (int k = 0; k < kLayaHd / 16; ++k) umma_f16(tmem, da + 2 * k, db + 2 * k, idesc_s, k);
        umma_commit(&bars[LB_S]);
        umma_commit(&bars[LB_KFREE]);
        if (!mbar_wait(&bars[LB_P], j & 1, abort_flag, g.status) ||
            !mbar_wait(&bars[LB_V], j & 1, abort_flag, g.status))
          break;
        tc_fence_after();
        // K = 128 keys in 8 steps of 16; P chunk kk / 4 holds keys 64 (kk / 4) ..
#pragma unroll
        for (int kk = 0; kk < kLayaTile / 16; ++kk) {
          const uint64_t pa = sw128_desc(ps + (kk >> 2) * LA_CHUNK) + 2 * (kk & 3);
          const uint64_t vb = sw128_mn_desc(vs + kk * 2048, LA_CHUNK);
          umma_f16(tmem + LA_TMEM_O, pa, vb, idesc_o, kk ? 1u : 0u);
        }
        umma_commit(&bars[LB_O]);
        umma_commit(&bars[LB_VFREE]);
      }
    }
  } else {
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;
    const bool valid = r < it.nq;
    const int tok = it.q0 + r;
    int vlo = 0, vhi = 0;
    if (valid) {
      const int2 sp = g.span[tok];
      vlo = sp.x;
      vhi = sp.y;
      if (g.window > 0) {
        vlo = max(vlo, tok - g.window);
        vhi = min(vhi, tok + g.window + 1);
      }
    }
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * q4) << 16);
    float o[kLayaHd];
#pragma unroll
    for (int i = 0; i < kLayaHd; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int kt = it.k0 + j * kLayaTile;
      int c0 = min(max(vlo - kt, 0), kLayaTile), c1 = min(max(vhi - kt, 0), kLayaTile);
      if (c1 < c0) c1 = c0;
      if (!warp_wait(&bars[LB_S], j & 1, abort_flag, g.status, lane)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // Pass 1: the tile's masked row max. A 32-key chunk is wholly visible,
      // wholly hidden or (at the window and sequence edges) split; eight
      // independent partial maxima keep the warp issuing.
      float mt = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < kLayaTile / 32; ++c) {
        float s[32];
        tmem_ld32(trow + c * 32, s);
        const int k0 = c * 32;
        if (c1 <= k0 || c0 >= k0 + 32) continue;
        if (c0 > k0 || c1 < k0 + 32) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (k0 + e < c0 || k0 + e >= c1) s[e] = -INFINITY;
        }
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = s[e];
#pragma unroll
        for (int e = 8; e < 32; ++e) mx[e & 7] = fmaxf(mx[e & 7], s[e]);
        mt = fmaxf(mt, fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))));
      }
      const float m_new = fmaxf(m, mt);
      const float alpha = m_new == -INFINITY ? 1.f : exp2f((m - m_new) * kLog2e);
      const float mb = m_new == -INFINITY ? 0.f : m_new * kLog2e;
      // Fold the previous tile's P.V into the running output: the MMA that
      // made it is done, so its P buffer is free again.
      if (j > 0) {
        if (!warp_wait(&bars[LB_O], (j - 1) & 1, abort_flag, g.status, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kLayaHd / 32; ++c) {
          float ov[32];
          tmem_ld32(trow + LA_TMEM_O + c * 32, ov);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[c * 32 + e] = fmaf(o[c * 32 + e], alpha_prev, ov[e]);
        }
      }
      // Pass 2: P = exp(s - m_new) on visible keys, 0 elsewhere, as f16 in
      // the 128-byte-swizzled K-major layout the MMA reads.
      float ps8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int c = 0; c < kLayaTile / 32; ++c) {
        float s[32];
        tmem_ld32(trow + c * 32, s);
        const int k0 = c * 32;
        if (c1 <= k0 || c0 >= k0 + 32 || m_new == -INFINITY) {
#pragma unroll
          for (int e = 0; e < 32; ++e) s[e] = 0.f;
        } else {
          const bool split = c0 > k0 || c1 < k0 + 32;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float p = exp2f(fmaf(s[e], kLog2e, -mb));
            if (split && (k0 + e < c0 || k0 + e >= c1)) p = 0.f;
            s[e] = p;
            ps8[e & 7] += p;
          }
        }
#pragma unroll
        for (int pc = 0; pc < 4; ++pc) {
          uint32_t w4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __half2 h = __floats2half2_rn(s[pc * 8 + 2 * e], s[pc * 8 + 2 * e + 1]);
            w4[e] = *reinterpret_cast<const uint32_t*>(&h);
          }
          const int key0 = c * 32 + pc * 8;
          const int kc = key0 >> 6, pw = (key0 & 63) >> 3;
          *reinterpret_cast<uint4*>(ps + kc * LA_CHUNK + r * 128 + ((pw ^ (r & 7)) << 4)) =
              make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
      const float sum = ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
      l = l * alpha + sum;
      m = m_new;
      alpha_prev = alpha;
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[LB_P]);
    }
    if (ok && warp_wait(&bars[LB_O], (ntiles - 1) & 1, abort_flag, g.status, lane)) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < kLayaHd / 32; ++c) {
        float ov[32];
        tmem_ld32(trow + LA_TMEM_O + c * 32, ov);
#pragma unroll
        for (int e = 0; e < 32; ++e) o[c * 32 + e] = fmaf(o[c * 32 + e], alpha_prev, ov[e]);
      }
      if (valid) {
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        __half* orow = g.out + static_cast<size_t>(tok) * g.d + head * kLayaHd;
#pragma unroll
        for (int e = 0; e < kLayaHd; e += 8) {
          uint32_t w4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const __half2 h = __floats2half2_rn(o[e + 2 * q] * inv, o[e + 2 * q + 1] * inv);
            w4[q] = *reinterpret_cast<const uint32_t*>(&h);
          }
          *reinterpret_cast<uint4*>(orow + e) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
    }
  }
  griddep_launch();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, LA_TMEM_COLS);
  }
}

// The same attention for passes whose items each see one 128-key tile (every
// sequence <= 128 tokens, as in a batch of questions): a persistent CTA per
// SM walks (item, head) units; two groups of four softmax warps take
// alternate units, each group with its own MMA thread and two buffer slots
// (Q, K, V in shared memory; 128 TMEM columns), so one group's softmax runs
// while the other's loads, MMAs and output proceed.
//
//   warp 0        TMA: Q, K, V of unit i into slot (i & 1, (i >> 1) & 1)
//   warps 1, 2    MMA for group 0 / 1: S = Q K^T into the slot's TMEM
//                 columns; after the softmax, O = P V into the first 64 of
//                 them (S is dead by then)
//   warps 3-6,    softmax group 0 / 1, one query row per thread: masked max,
//   7-10          exp, row sum, P (f16) over the slot's Q and K (dead after
//                 S); then out = O / l, staged in the same bytes and stored a
//                 row segment per lane
//
// Each row's arithmetic is the one-tile case of laya_attention_kernel step
// for step (same MMAs, same partial sums in the same order), so a row gets
// the same bits from either kernel.
constexpr int LP_THREADS = 352;
constexpr int LP_SMEM = 1024 + 4 * 3 * LA_CHUNK + 256;
constexpr uint32_t LP_TMEM_COLS = 512;  // slot (g, s): columns 128 (2 g + s) .. + 128

enum { LP_FULL = 0, LP_SFULL = 4, LP_PFULL = 8, LP_OFULL = 12, LP_TFREE = 16, LP_N = 20 };

__global__ void __launch_bounds__(LP_THREADS, 1)
    laya_attention_tile_kernel(const __grid_constant__ CUtensorMap tqkv, LayaAttnArgs g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  auto chunk = [&](int slot, int c) { return sm + (slot * 3 + c) * LA_CHUNK; };  // Q, K, V
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + 4 * 3 * LA_CHUNK);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + LP_N);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = g.n_items * g.heads;

  if (threadIdx.x == 0) {
    for (int i = 0; i < LP_N; ++i)
      mbar_init(&bars[i], (i >= LP_PFULL && i < LP_PFULL + 4) || i >= LP_TFREE ? 4 : 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tqkv);
  }
  if (warp == 1) tmem_alloc(tmem_slot, LP_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch();

  // Unit i of this CTA: group i & 1, its (i >> 1)-th unit, slot 2 (i & 1) +
  // ((i >> 1) & 1), that slot's (i >> 2)-th use.
  if (warp == 0) {
    if (lane == 0) {
      int i = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x, ++i) {
        const int slot = 2 * (i & 1) + ((i >> 1) & 1), use = i >> 2;
        if (use > 0 && !mbar_wait(&bars[LP_TFREE + slot], (use - 1) & 1, abort_flag, g.status))
          break;
        const LayaAttnItem it = g.items[u / g.heads];
        const int head = u % g.heads;
        uint64_t* full = &bars[LP_FULL + slot];
        mbar_arrive_expect_tx(full, 3 * LA_CHUNK);
        tma_load_2d(chunk(slot, 0), &tqkv, full, head * kLayaHd, it.q0);
        tma_load_2d(chunk(slot, 1), &tqkv, full, g.d + head * kLayaHd, it.k0);
        tma_load_2d(chunk(slot, 2), &tqkv, full, 2 * g.d + head * kLayaHd, it.k0);
      }
    }
  } else if (warp == 1 || warp == 2) {
    if (lane == 0) {
      const int grp = warp - 1;
      constexpr uint32_t idesc_s = idesc_f16_f32(128, kLayaTile);
      constexpr uint32_t idesc_o = idesc_f16_f32_bmn(128, kLayaHd);
      int i = grp;
      for (int u = blockIdx.x + grp * gridDim.x; u < units; u += 2 * gridDim.x, i += 2) {
        const int slot = 2 * grp + ((i >> 1) & 1);
        const uint32_t par = (i >> 2) & 1;
        const uint32_t d = tmem + 128u * slot;
        if (!mbar_wait(&bars[LP_FULL + slot], par, abort_flag, g.status)) break;
        tc_fence_after();
        const uint64_t da = sw128_desc(chunk(slot, 0)), db = sw128_desc(chunk(slot, 1));
#pragma unroll
        for (int k = 0; k < kLayaHd / 16; ++k) umma_f16(d, da + 2 * k, db + 2 * k, idesc_s, k);
        umma_commit(&bars[LP_SFULL + slot]);
        if (!mbar_wait(&bars[LP_PFULL + slot], par, abort_flag, g.status)) break;
        tc_fence_after();
        uint8_t* ps = chunk(slot, 0);  // P over Q and K
#pragma unroll
        for (int kk = 0; kk < kLayaTile / 16; ++kk) {
          const uint64_t pa = sw128_desc(ps + (kk >> 2) * LA_CHUNK) + 2 * (kk & 3);
          const uint64_t vb = sw128_mn_desc(chunk(slot, 2) + kk * 2048, LA_CHUNK);
          umma_f16(d, pa, vb, idesc_o, kk ? 1u : 0u);
        }
        umma_commit(&bars[LP_OFULL + slot]);
      }
    }
  } else {
    const int grp = (warp - 3) >> 2;
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;
    int i = grp;
    for (int u = blockIdx.x + grp * gridDim.x; u < units; u += 2 * gridDim.x, i += 2) {
      const int slot = 2 * grp + ((i >> 1) & 1);
      const uint32_t par = (i >> 2) & 1;
      const LayaAttnItem it = g.items[u / g.heads];
      const int head = u % g.heads;
      const bool valid = r < it.nq;
      const int tok = it.q0 + r;
      int vlo = 0, vhi = 0;
      if (valid) {
        const int2 sp = g.span[tok];
        vlo = sp.x;
        vhi = sp.y;
        if (g.window > 0) {
          vlo = max(vlo, tok - g.window);
          vhi = min(vhi, tok + g.window + 1);
        }
      }
      int c0 = min(max(vlo - it.k0, 0), kLayaTile), c1 = min(max(vhi - it.k0, 0), kLayaTile);
      if (c1 < c0) c1 = c0;
      if (!warp_wait(&bars[LP_SFULL + slot], par, abort_flag, g.status, lane)) break;
      tc_fence_after();
      const uint32_t trow = tmem + (static_cast<uint32_t>(32 * q4) << 16) + 128u * slot;
      // Pass 1: the masked row max.
      float mt = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < kLayaTile / 32; ++c) {
        float s[32];
        tmem_ld32(trow + c * 32, s);
        const int k0 = c * 32;
        if (c1 <= k0 || c0 >= k0 + 32) continue;
        if (c0 > k0 || c1 < k0 + 32) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (k0 + e < c0 || k0 + e >= c1) s[e] = -INFINITY;
        }
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = s[e];
#pragma unroll
        for (int e = 8; e < 32; ++e) mx[e & 7] = fmaxf(mx[e & 7], s[e]);
        mt = fmaxf(mt, fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))));
      }
      const float m_new = mt;
      const float alpha = m_new == -INFINITY ? 1.f : 0.f;  // exp2((-inf - m_new) log2e)
      const float mb = m_new == -INFINITY ? 0.f : m_new * kLog2e;
      // Pass 2: P = exp(s - m) on visible keys, 0 elsewhere, f16, K-major
      // with the 128-byte swizzle, over the slot's Q and K.
      uint8_t* ps = chunk(slot, 0);
      float ps8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int c = 0; c < kLayaTile / 32; ++c) {
        float s[32];
        tmem_ld32(trow + c * 32, s);
        const int k0 = c * 32;
        if (c1 <= k0 || c0 >= k0 + 32 || m_new == -INFINITY) {
#pragma unroll
          for (int e = 0; e < 32; ++e) s[e] = 0.f;
        } else {
          const bool split = c0 > k0 || c1 < k0 + 32;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float p = exp2f(fmaf(s[e], kLog2e, -mb));
            if (split && (k0 + e < c0 || k0 + e >= c1)) p = 0.f;
            s[e] = p;
            ps8[e & 7] += p;
          }
        }
#pragma unroll
        for (int pc = 0; pc < 4; ++pc) {
          uint32_t w4[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __half2 h = __floats2half2_rn(s[pc * 8 + 2 * e], s[pc * 8 + 2 * e + 1]);
            w4[e] = *reinterpret_cast<const uint32_t*>(&h);
          }
          const int key0 = c * 32 + pc * 8;
          const int kc = key0 >> 6, pw = (key0 & 63) >> 3;
          *reinterpret_cast<uint4*>(ps + kc * LA_CHUNK + r * 128 + ((pw ^ (r & 7)) << 4)) =
              make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
      const float sum = ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
      const float l = 0.f * alpha + sum;
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[LP_PFULL + slot]);
      if (!warp_wait(&bars[LP_OFULL + slot], par, abort_flag, g.status, lane)) break;
      tc_fence_after();
      // out = O / l as f16, staged over P (the P.V that read it is done): row
      // r at r * 128 bytes, piece p at p ^ (r & 7); each warp then stores
      // its 32 rows, four 128-byte row segments per instruction.
      const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
      for (int c = 0; c < kLayaHd / 32; ++c) {
        float ov[32];
        tmem_ld32(trow + c * 32, ov);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t w4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            // fmaf(0, alpha, O): the one-tile running output, exactly as the
            // general kernel folds its only tile in.
            const float o0 = fmaf(0.f, alpha, ov[8 * e + 2 * q]);
            const float o1 = fmaf(0.f, alpha, ov[8 * e + 2 * q + 1]);
            const __half2 h = __floats2half2_rn(o0 * inv, o1 * inv);
            w4[q] = *reinterpret_cast<const uint32_t*>(&h);
          }
          const int piece = 4 * c + e;
          *reinterpret_cast<uint4*>(ps + r * 128 + ((piece ^ (r & 7)) << 4)) =
              make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
      __syncwarp();
      {
        const int p = lane & 7;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int row = 32 * q4 + 4 * k + (lane >> 3);
          const uint4 v = *reinterpret_cast<const uint4*>(ps + row * 128 + ((p ^ (row & 7)) << 4));
          if (row < it.nq)
            *reinterpret_cast<uint4*>(g.out + static_cast<size_t>(it.q0 + row) * g.d +
                                      head * kLayaHd + 8 * p) = v;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[LP_TFREE + slot]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, LP_TMEM_COLS);
  }
}

}  // namespace

void launch_laya_rope_table(float theta, int hd, int n_pos, float2* tab, cudaStream_t s) {
  const int n = n_pos * (hd / 2);
  rope_table_kernel<<<std::max(1, std::min(1024, (n + 255) / 256)), 256, 0, s>>>(theta, hd, n_pos,
                                                                                  tab);
}

void launch_laya_embed_ln(int dtype, const int* ids, int t, const void* codes, const void* scales,
                          int d, const float* w, float eps, float* x, __half* h16,
                          cudaStream_t s) {
  if (t <= 0) return;
  const auto* c = static_cast<const uint8_t*>(codes);
  const auto* sc = static_cast<const uint8_t*>(scales);
  const unsigned grid = static_cast<unsigned>((t + 7) / 8);
  if (dtype == kQ4)
    launch_pdl(laya_embed_ln_kernel<kQ4>, dim3(grid), dim3(256), 0, s, ids, t, c, sc, d, w, eps, x, h16);
  else if (dtype == kQ8)
    launch_pdl(laya_embed_ln_kernel<kQ8>, dim3(grid), dim3(256), 0, s, ids, t, c, sc, d, w, eps, x, h16);
  else
    launch_pdl(laya_embed_ln_kernel<kF16>, dim3(grid), dim3(256), 0, s, ids, t, c, sc, d, w, eps, x, h16);
}

void launch_laya_ln(const LayaLnArgs& a, cudaStream_t s) {
  if (a.t <= 0) return;
  const dim3 grid(static_cast<unsigned>((a.t + 7) / 8));
  switch (a.d / 128) {
#define OMG_LN_CASE(n) \
  case n:              \
    launch_pdl(laya_ln_kernel<n>, grid, dim3(256), 0, s, a); \
    break;
    OMG_LN_CASE(1) OMG_LN_CASE(2) OMG_LN_CASE(3) OMG_LN_CASE(4) OMG_LN_CASE(5) OMG_LN_CASE(6)
    OMG_LN_CASE(7) OMG_LN_CASE(8) OMG_LN_CASE(9) OMG_LN_CASE(10) OMG_LN_CASE(11)
    OMG_LN_CASE(12) OMG_LN_CASE(13) OMG_LN_CASE(14) OMG_LN_CASE(15) OMG_LN_CASE(16)
#undef OMG_LN_CASE
    default:
      break;
  }
}

void launch_laya_gather(const float* x, int d, const int* row_map, int n, float* rows,
                        cudaStream_t s) {
  if (n <= 0) return;
  launch_pdl(laya_gather_kernel, dim3(n), dim3(128), 0, s, x, d, row_map, n, rows);
}

void laya_attention_items(const int2* span, int t, int window, std::vector<LayaAttnItem>* items) {
  items->clear();
  int i = 0;
  while (i < t) {
    // Each sequence gets its own items, with query and key tiles anchored at
    // its first row: a row meets its keys at the same tile columns whatever
    // else shares the pass, so its result does not depend on the packing.
    const int lo = span[i].x, hi = span[i].y;
    for (int q0 = lo; q0 < hi; q0 += kLayaTile) {
      const int nq = std::min(kLayaTile, hi - q0);
      int k0 = lo, k1 = hi;
      if (window > 0) {
        // Keep the key grid anchored at lo: start at the tile holding the
        // first key the chunk sees.
        const int first = std::max(lo, q0 - window);
        k0 = lo + (first - lo) / kLayaTile * kLayaTile;
        k1 = std::min(hi, q0 + nq + window);
      }
      items->push_back(LayaAttnItem{q0, nq, k0, k1 - k0});
    }
    i = hi;
  }
}

bool laya_attention_map(CUtensorMap* m, const void* qkv16, int rows_cap, int d, char* err,
                        size_t errlen) {
  const uint64_t dims[2] = {static_cast<uint64_t>(3 * d), static_cast<uint64_t>(rows_cap)};
  const uint64_t strides[1] = {static_cast<uint64_t>(3 * d) * 2};
  const uint32_t box[2] = {64, static_cast<uint32_t>(kLayaTile)};
  return make_tmap_f16(m, qkv16, 2, dims, strides, box, err, errlen);
}

void launch_laya_attention(const CUtensorMap& tqkv, const LayaAttnArgs& a, cudaStream_t s) {
  if (a.n_items <= 0) return;
  if (a.single_tile) {
    const int units = a.n_items * a.heads;
    const int sms = a.num_sms > 0 ? a.num_sms : 148;
    launch_pdl(laya_attention_tile_kernel, dim3(units < sms ? units : sms), dim3(LP_THREADS),
               LP_SMEM, s, tqkv, a);
    return;
  }
  dim3 grid(a.n_items, a.heads);
  launch_pdl(laya_attention_kernel, grid, dim3(192), LA_SMEM, s, tqkv, a);
}

void laya_setup_device() {
  cudaFuncSetAttribute(laya_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, LA_SMEM);
  cudaFuncSetAttribute(laya_attention_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       LP_SMEM);
}


// ---- the decision head on the device -------------------------------------------

namespace {

constexpr int kHeadThreads = 256;  // eight warps
constexpr int kHeadWarps = kHeadThreads / 32;

// erf by Abramowitz & Stegun 7.1.26 (|error| < 1.5e-7), the form laya.rs
// uses for the host head.
__device__ __forceinline__ float head_erf(float x) {
  const float sgn = x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
  const float a = fabsf(x);
  const float t = 1.0f / (1.0f + 0.3275911f * a);
  const float poly =
      ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t +
       0.254829592f) *
      t;
  return sgn * (1.0f - poly * expf(-a * a));
}

__device__ __forceinline__ float head_gelu(float x) {
  return 0.5f * x * (1.0f + head_erf(x * 0.70710678118654752f));
}

__device__ __forceinline__ float warp_sum_all(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float dot4(float4 a, float4 b) {
  return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
}

// The rows r = warp, warp + 8, ... < rows of W ([rows][n4] float4s) against
// the MR inputs whose float4 slots lane + 32 j (j < NV) this lane holds in
// `in` (zero past n4). The next row's slots are loaded while the current
// row is summed, so each warp keeps NV loads in flight. consume(r, y) gets
// the MR full sums (every lane holds them).
template <int NV, int MR, class F>
__device__ __forceinline__ void head_rows(const float4* __restrict__ W, int n4, int rows,
                                          const float4 (&in)[MR][NV], F&& consume) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 wn[NV];
  auto load = [&](int r) {
    const float4* wr = W + static_cast<size_t>(r) * n4;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      wn[j] = i < n4 ? __ldg(wr + i) : zero;
    }
  };
  if (warp < rows) load(warp);
  for (int r = warp; r < rows; r += kHeadWarps) {
    float4 w[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) w[j] = wn[j];
    if (r + kHeadWarps < rows) load(r + kHeadWarps);
    float y[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      y[m] = 0.f;
#pragma unroll
      for (int j = 0; j < NV; ++j) y[m] += dot4(w[j], in[m][j]);
      y[m] = warp_sum_all(y[m]);
    }
    consume(r, y);
  }
}

// Scorer: MR marker rows per CTA; NV = d / 128 float4 slots per lane.
template <int NV, int MR>
__global__ void __launch_bounds__(kHeadThreads) laya_score_kernel(LayaScoreArgs a) {
  griddep_wait();
  __shared__ float part[kHeadWarps][MR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * MR;
  const int d = a.d, n4 = d / 4;
  // Every warp normalises the MR rows itself (each warp reduces the same
  // values the same way, so all hold the same results) and keeps its lane's
  // slots in registers.
  float4 z[MR][NV];
  const float4* nw = reinterpret_cast<const float4*>(a.norm_w);
  const float4* nb = reinterpret_cast<const float4*>(a.norm_b);
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    const bool live = m0 + m < a.k;
    const float4* x = reinterpret_cast<const float4*>(
        a.rows + static_cast<size_t>(live ? a.marker_row[m0 + m] : 0) * d);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      z[m][j] = x[lane + 32 * j];
      s += (z[m][j].x + z[m][j].y) + (z[m][j].z + z[m][j].w);
    }
    const float mean = warp_sum_all(s) / static_cast<float>(d);
    float v = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float4 c = make_float4(z[m][j].x - mean, z[m][j].y - mean, z[m][j].z - mean,
                                   z[m][j].w - mean);
      v += dot4(c, c);
    }
    const float inv = 1.0f / sqrtf(warp_sum_all(v) / static_cast<float>(d) + a.eps);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float4 w = __ldg(nw + lane + 32 * j), b = __ldg(nb + lane + 32 * j);
      const float4 q = z[m][j];
      z[m][j] = live ? make_float4((q.x - mean) * inv * w.x + b.x, (q.y - mean) * inv * w.y + b.y,
                                   (q.z - mean) * inv * w.z + b.z, (q.w - mean) * inv * w.w + b.w)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  float acc[MR];
#pragma unroll
  for (int m = 0; m < MR; ++m) acc[m] = 0.f;
  head_rows<NV, MR>(reinterpret_cast<const float4*>(a.l1), n4, d, z,
                    [&](int r, const float (&y)[MR]) {
                      const float b = __ldg(a.l1_b + r), w2 = __ldg(a.l2 + r);
#pragma unroll
                      for (int m = 0; m < MR; ++m) acc[m] += head_gelu(y[m] + b) * w2;
                    });
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < MR; ++m) part[warp][m] = acc[m];
  }
  __syncthreads();
  if (threadIdx.x < MR && m0 + static_cast<int>(threadIdx.x) < a.k) {
    float s = 0.f;
    for (int w = 0; w < kHeadWarps; ++w) s += part[w][threadIdx.x];
    a.logits[m0 + threadIdx.x] = s + a.l2_b;
  }
}

// Act head: MR sequences per CTA; the input u = [cls row (d), 4 features]
// is NV = d / 128 full slots per lane plus one more slot that only lane 0
// fills (the features).
template <int NV, int MR>
__global__ void __launch_bounds__(kHeadThreads) laya_act_kernel(LayaActArgs a) {
  griddep_wait();
  __shared__ float hid[MR][256];
  __shared__ float4 feat[MR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s0 = blockIdx.x * MR;
  const int d = a.d, n4 = d / 4 + 1;
  // The confidence features of sequence m (laya.rs:1463-1475), by thread m.
  if (threadIdx.x < MR) {
    const int m = threadIdx.x;
    float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s0 + m < a.n) {
      const int4 q = a.seq[s0 + m];
      const float* lg = a.logits + q.y;
      const int k = q.z, kk = k > 2 ? k : 2;
      float mx = -INFINITY;
      for (int j = 0; j < kk; ++j) mx = fmaxf(mx, j < k ? lg[j] : -1e4f);
      float sum = 0.f;
      for (int j = 0; j < kk; ++j) sum += expf((j < k ? lg[j] : -1e4f) - mx);
      float ent = 0.f, top1 = -INFINITY, top2 = -INFINITY;
      for (int j = 0; j < kk; ++j) {
        const float p = expf((j < k ? lg[j] : -1e4f) - mx) / sum;
        ent += p * logf(fmaxf(p, 1e-9f));
        if (p > top1) {
          top2 = top1;
          top1 = p;
        } else if (p > top2) {
          top2 = p;
        }
      }
      f = make_float4(top1, top1 - top2, -ent / logf(static_cast<float>(kk)),
                      static_cast<float>(kk) / 255.0f);
    }
    feat[m] = f;
  }
  __syncthreads();
  float4 u[MR][NV + 1];
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    const bool live = s0 + m < a.n;
    const float4* x = reinterpret_cast<const float4*>(
        a.rows + static_cast<size_t>(live ? a.seq[s0 + m].x : 0) * d);
#pragma unroll
    for (int j = 0; j < NV; ++j)
      u[m][j] = live ? x[lane + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
    u[m][NV] = lane == 0 ? feat[m] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  head_rows<NV + 1, MR>(reinterpret_cast<const float4*>(a.l1), n4, a.hidden, u,
                        [&](int r, const float (&y)[MR]) {
                          if (lane == 0) {
                            const float b = __ldg(a.l1_b + r);
#pragma unroll
                            for (int m = 0; m < MR; ++m) hid[m][r] = head_gelu(y[m] + b);
                          }
                        });
  __syncthreads();
  // Output layer and softmax: warp m for sequence m, in two passes over the
  // outputs (max, then the exponentials), each logit recomputed identically,
  // so any number of outputs needs no storage.
  for (int m = warp; m < MR; m += kHeadWarps) {
    if (s0 + m >= a.n) break;
    auto out_logit = [&](int o) {
      const float* w = a.l2 + static_cast<size_t>(o) * a.hidden;
      float s = 0.f;
      for (int i = lane; i < a.hidden; i += 32) s += w[i] * hid[m][i];
      return warp_sum_all(s) + a.l2_b[o];
    };
    float mx = -INFINITY;
    for (int o = 0; o < a.outs; ++o) mx = fmaxf(mx, out_logit(o));
    float sum = 0.f, e0 = 0.f;
    for (int o = 0; o < a.outs; ++o) {
      const float e = expf(out_logit(o) - mx);
      if (o == 0) e0 = e;
      sum += e;
    }
    if (lane == 0) a.act[s0 + m] = e0 / sum;
  }
}

}  // namespace

// Marker rows (sequences) per CTA by the registers a lane's slots take:
// MR x NV float4s stay within 24. NV = hidden_size / 128 (1..16).
#define OMG_HEAD_NV(X)                                                                    \
  X(1, 8) X(2, 8) X(3, 8) X(4, 4) X(5, 4) X(6, 4) X(7, 2) X(8, 2) X(9, 2) X(10, 2) X(11, 2) \
  X(12, 2) X(13, 1) X(14, 1) X(15, 1) X(16, 1)

void launch_laya_score(const LayaScoreArgs& a, cudaStream_t s) {
  if (a.k <= 0) return;
  const int nv = a.d / 128;
#define OMG_SCORE(NV, MR)                                                                     \
  if (nv == NV) {                                                                             \
    launch_pdl(laya_score_kernel<NV, MR>, dim3((a.k + MR - 1) / MR), dim3(kHeadThreads), 0, s, \
               a);                                                                            \
    return;                                                                                   \
  }
  OMG_HEAD_NV(OMG_SCORE)
#undef OMG_SCORE
}

void launch_laya_act(const LayaActArgs& a, cudaStream_t s) {
  if (a.n <= 0) return;
  const int nv = a.d / 128;
#define OMG_ACT(NV, MR)                                                                     \
  if (nv == NV) {                                                                           \
    launch_pdl(laya_act_kernel<NV, MR>, dim3((a.n + MR - 1) / MR), dim3(kHeadThreads), 0, s, \
               a);                                                                          \
    return;                                                                                 \
  }
  OMG_HEAD_NV(OMG_ACT)
#undef OMG_ACT
}
#undef OMG_HEAD_NV


}  // namespace omg
