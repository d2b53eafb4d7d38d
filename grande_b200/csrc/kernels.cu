// Row kernels of the decoder pass (see kernels.cuh). Reference shaders:
// crates/omg-wgpu/src/shaders/{weight,embed,rmsnorm,qk_prep,logits}.wgsl.
#include <algorithm>

#include "kernels.cuh"
#include "packed.cuh"
#include "launch.cuh"
#include "ptx.cuh"
#include "quant.cuh"

namespace omg {

namespace {

// ---- weight dequantization --------------------------------------------------

__device__ __forceinline__ int remap_row(int r, int mode) {
  if (mode == 1) return (r / 128) * 256 + (r % 128);
  if (mode == 2) return (r / 128) * 256 + 128 + (r % 128);
  return r;
}

__global__ void dequant_f16_kernel(int dtype, const uint8_t* __restrict__ codes,
                                   const uint8_t* __restrict__ scales, int rows, int k, int remap,
                                   __half* __restrict__ out) {
  const size_t nblk = static_cast<size_t>(rows) * (k / 32);
  for (size_t b = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; b < nblk;
       b += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(b / (k / 32));
    const int c = static_cast<int>(b % (k / 32)) * 32;
    __half* o = out + static_cast<size_t>(remap_row(r, remap)) * k + c;
    __align__(16) __half v[32];
    if (dtype == kF16) {
      const uint4* src = reinterpret_cast<const uint4*>(codes + b * 64);
#pragma unroll
      for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(v)[i] = src[i];
    } else {
      const uint16_t sb = static_cast<uint16_t>(scales[2 * b]) |
                          (static_cast<uint16_t>(scales[2 * b + 1]) << 8);
      const float d = half_bits_to_float(sb);
      if (dtype == kQ8) {
        __align__(16) int8_t q[32];
        reinterpret_cast<uint4*>(q)[0] = reinterpret_cast<const uint4*>(codes + b * 32)[0];
        reinterpret_cast<uint4*>(q)[1] = reinterpret_cast<const uint4*>(codes + b * 32)[1];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __float2half_rn(static_cast<float>(q[j]) * d);
      } else {
        __align__(16) uint8_t q[16];
        reinterpret_cast<uint4*>(q)[0] = reinterpret_cast<const uint4*>(codes + b * 16)[0];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          v[j] = __float2half_rn((static_cast<float>(q[j] & 0xf) - 8.0f) * d);
          v[j + 16] = __float2half_rn((static_cast<float>(q[j] >> 4) - 8.0f) * d);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(o)[i] = reinterpret_cast<uint4*>(v)[i];
  }
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) s += red[i];
  return s;
}

// The same for a block of blockDim.x threads (a multiple of 32, <= 1024).
__device__ __forceinline__ float block_sum_dyn(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) s += red[i];
  return s;
}

// ---- embedding + first norm ------------------------------------------------

template <int DT>
__global__ void __launch_bounds__(128) embed_norm_kernel(const int* __restrict__ ids, int t,
                                                         const uint8_t* __restrict__ codes,
                                                         const uint8_t* __restrict__ scales,
                                                         int d, float scale,
                                                         const float* __restrict__ w, float eps,
                                                         float offset, float* __restrict__ x,
                                                         __half* __restrict__ x16,
                                                         __half* __restrict__ h16, int ldh) {
  griddep_wait();
  // Let the next kernel start its prologue; its CTAs wait for this grid.
  griddep_launch();
  __shared__ float red[4];
  const int row = blockIdx.x;
  if (row >= t) return;
  const size_t id = static_cast<size_t>(ids[row]);
  float* xr = x + static_cast<size_t>(row) * d;
  const int nb = d / 32;
  float ss = 0.f;
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    float v[32];
    load_block_f32<DT>(codes, scales, id * nb + b, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      v[j] = v[j] * scale;
      ss += v[j] * v[j];
    }
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4*>(xr + b * 32 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    if (x16) {
      __half* xh = x16 + static_cast<size_t>(row) * d + b * 32;
#pragma unroll
      for (int j = 0; j < 32; j += 2)
        *reinterpret_cast<__half2*>(xh + j) = __floats2half2_rn(v[j], v[j + 1]);
    }
  }
  const float inv = rsqrtf(block_sum<128>(ss, red) / static_cast<float>(d) + eps);
  __half* hr = h16 + static_cast<size_t>(row) * ldh;
  for (int i = threadIdx.x * 4; i < d; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float4 ww = *reinterpret_cast<const float4*>(w + i);
    __half2 a = __floats2half2_rn(v.x * inv * (offset + ww.x), v.y * inv * (offset + ww.y));
    __half2 b = __floats2half2_rn(v.z * inv * (offset + ww.z), v.w * inv * (offset + ww.w));
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&a);
    pk.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(hr + i) = pk;
  }
}

// ---- residual-stream norms -------------------------------------------------

// One CTA per row, NV float4 per thread and as many threads as the row needs
// (d / (4 NV), rounded up to whole warps): no idle lanes holding registers
// (a 2560-wide row took 256 threads x 4 float4 before, 40% of them idle).
constexpr int kNormMaxThreads = 512;

template <int NV>
__global__ void __launch_bounds__(kNormMaxThreads) residual_norm_kernel(
    const float* __restrict__ a, int splits, size_t split_stride, int lda, int t, int d,
    const float* __restrict__ w1, float eps, float offset, float out_scale, float* __restrict__ x,
    __half* __restrict__ x16, const float* __restrict__ w2, __half* __restrict__ h16, int ldh,
    const int* __restrict__ row_map, float* __restrict__ rows_out) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nthr = static_cast<int>(blockDim.x);
  float4 y[NV], xo[NV], wa[NV], wb[NV];
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  // The norms' weights are never written by a pass: load them while the
  // previous kernel drains.
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = (threadIdx.x + j * nthr) * 4;
    wa[j] = wb[j] = zero;
    if (i < d) {
      wa[j] = __ldg(reinterpret_cast<const float4*>(w1 + i));
      if (w2) wb[j] = __ldg(reinterpret_cast<const float4*>(w2 + i));
    }
  }
  griddep_wait();
  // Let the next kernel start its prologue; its CTAs wait for this grid.
  griddep_launch();
  if (row >= t) return;
  const float* ar = a + static_cast<size_t>(row) * lda;
  float* xr = x + static_cast<size_t>(row) * d;
  // Every load of the row up front (the slabs and the residual row): only
  // the two reductions order the work after them.
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = (threadIdx.x + j * nthr) * 4;
    y[j] = xo[j] = zero;
    if (i < d) {
      y[j] = *reinterpret_cast<const float4*>(ar + i);
      xo[j] = *reinterpret_cast<const float4*>(xr + i);
    }
  }
  for (int z = 1; z < splits; ++z) {
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = (threadIdx.x + j * nthr) * 4;
      if (i < d) {
        const float4 u = *reinterpret_cast<const float4*>(ar + z * split_stride + i);
        y[j].x += u.x;
        y[j].y += u.y;
        y[j].z += u.z;
        y[j].w += u.w;
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j)
    ss += y[j].x * y[j].x + y[j].y * y[j].y + y[j].z * y[j].z + y[j].w * y[j].w;
  const float inv1 = rsqrtf(block_sum_dyn(ss, red) / static_cast<float>(d) + eps);
  float ss2 = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = (threadIdx.x + j * nthr) * 4;
    if (i < d) {
      const float4 ww = wa[j];
      float4 v = y[j];
      v.x = (v.x * inv1 * (offset + ww.x) + xo[j].x) * out_scale;
      v.y = (v.y * inv1 * (offset + ww.y) + xo[j].y) * out_scale;
      v.z = (v.z * inv1 * (offset + ww.z) + xo[j].z) * out_scale;
      v.w = (v.w * inv1 * (offset + ww.w) + xo[j].w) * out_scale;
      *reinterpret_cast<float4*>(xr + i) = v;
      if (x16) {
        __half2 p = __floats2half2_rn(v.x, v.y);
        __half2 q = __floats2half2_rn(v.z, v.w);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&p);
        pk.y = *reinterpret_cast<uint32_t*>(&q);
        *reinterpret_cast<uint2*>(x16 + static_cast<size_t>(row) * d + i) = pk;
      }
      y[j] = v;
      ss2 += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
  }
  if (w2 == nullptr) return;
  const float inv2 = rsqrtf(block_sum_dyn(ss2, red) / static_cast<float>(d) + eps);
  const int out_row = row_map ? row_map[row] : -1;
  __half* hr = h16 ? h16 + static_cast<size_t>(row) * ldh : nullptr;
  float* orow = out_row >= 0 ? rows_out + static_cast<size_t>(out_row) * d : nullptr;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = (threadIdx.x + j * nthr) * 4;
    if (i < d) {
      const float4 ww = wb[j];
      float4 v = y[j];
      v.x = v.x * inv2 * (offset + ww.x);
      v.y = v.y * inv2 * (offset + ww.y);
      v.z = v.z * inv2 * (offset + ww.z);
      v.w = v.w * inv2 * (offset + ww.w);
      if (hr) {
        __half2 p = __floats2half2_rn(v.x, v.y);
        __half2 q = __floats2half2_rn(v.z, v.w);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&p);
        pk.y = *reinterpret_cast<uint32_t*>(&q);
        *reinterpret_cast<uint2*>(hr + i) = pk;
      }
      if (orow) *reinterpret_cast<float4*>(orow + i) = v;
    }
  }
}

// ---- q / k norm, RoPE, K/V cache write (qk_prep.wgsl) ----------------------

template <int HD>
__global__ void __launch_bounds__(128) qk_prep_kernel(QkArgs g) {
  griddep_wait();
  // Let the next kernel start its prologue; its CTAs wait for this grid.
  griddep_launch();
  constexpr int E = HD / 64;  // elements per lane in each half of the head
  constexpr int HALF = HD / 2;
  const int tok = blockIdx.x;
  if (tok >= g.t) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int crow = g.base + tok;
  const float pos = static_cast<float>(g.meta[crow].pos);
  // The token's RoPE rotation, shared by all its q and k heads:
  // angle = pos * theta^(-dd / (HD/2)) (qk_prep.wgsl:52-64).
  __shared__ float rope_c[HALF], rope_s[HALF];
  for (int dd = threadIdx.x; dd < g.rope_dims / 2; dd += blockDim.x) {
    const float ang = pos * powf(g.theta, -static_cast<float>(dd) / static_cast<float>(HALF));
    sincosf(ang, &rope_s[dd], &rope_c[dd]);
  }
  __syncthreads();
  const float* row = g.qkv + static_cast<size_t>(tok) * g.q_stride;
  const int n_heads = g.heads + (g.has_kv ? 2 * g.kv_heads : 0);
  __half* kvrow = g.kv ? g.kv + static_cast<size_t>(crow) * 2 * g.kv_heads * HD : nullptr;
  for (int h = warp; h < n_heads; h += 4) {
    float a[E], b[E];
    const int off = h * HD + lane * E;
#pragma unroll
    for (int e = 0; e < E; e += 4) {
      float4 u = *reinterpret_cast<const float4*>(row + off + e);
      float4 v = *reinterpret_cast<const float4*>(row + off + HALF + e);
      for (int z = 1; z < g.splits; ++z) {
        const float4 u2 = *reinterpret_cast<const float4*>(row + z * g.split_stride + off + e);
        const float4 v2 =
            *reinterpret_cast<const float4*>(row + z * g.split_stride + off + HALF + e);
        u.x += u2.x; u.y += u2.y; u.z += u2.z; u.w += u2.w;
        v.x += v2.x; v.y += v2.y; v.z += v2.z; v.w += v2.w;
      }
      a[e] = u.x; a[e + 1] = u.y; a[e + 2] = u.z; a[e + 3] = u.w;
      b[e] = v.x; b[e + 1] = v.y; b[e + 2] = v.z; b[e + 3] = v.w;
    }
    const bool is_q = h < g.heads;
    const bool is_v = h >= g.heads + g.kv_heads;
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss += a[e] * a[e] + b[e] * b[e];
    ss = warp_sum(ss);
    if (is_v) {
      const float inv = g.v_norm ? rsqrtf(ss / static_cast<float>(HD) + g.eps) : 1.0f;
      __half* o = kvrow + (g.kv_heads + (h - g.heads - g.kv_heads)) * HD + lane * E;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        o[e] = __float2half_rn(a[e] * inv);
        o[HALF + e] = __float2half_rn(b[e] * inv);
      }
      continue;
    }
    const float inv = rsqrtf(ss / static_cast<float>(HD) + g.eps);
    const float* wn = is_q ? g.qn : g.kn;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int dd = lane * E + e;
      float y1 = a[e] * inv * (g.offset + wn[dd]);
      float y2 = b[e] * inv * (g.offset + wn[dd + HALF]);
      if (dd < g.rope_dims / 2) {
        const float cs = rope_c[dd], sn = rope_s[dd];
        const float r1 = y1 * cs - y2 * sn;
        const float r2 = y2 * cs + y1 * sn;
        y1 = r1;
        y2 = r2;
      }
      a[e] = y1;
      b[e] = y2;
    }
    if (is_q) {
      __half* o = g.q16 + static_cast<size_t>(tok) * g.heads * HD + h * HD + lane * E;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        o[e] = __float2half_rn(a[e] * g.q_scale);
        o[HALF + e] = __float2half_rn(b[e] * g.q_scale);
      }
    } else {
      __half* o = kvrow + (h - g.heads) * HD + lane * E;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        o[e] = __float2half_rn(a[e]);
        o[HALF + e] = __float2half_rn(b[e]);
      }
    }
  }
}

// ---- Gemma 4 per-layer inputs (pl_combine.wgsl, pl_gate.wgsl) -------------

__global__ void __launch_bounds__(128) pl_combine_kernel(const float* __restrict__ proj, int t,
                                                         int P, int layers,
                                                         const float* __restrict__ w,
                                                         const __half* __restrict__ emb,
                                                         float eps, float offset,
                                                         float proj_scale, float emb_scale,
                                                         float out_scale, float* __restrict__ out) {
  griddep_wait();
  __shared__ float red[4];
  const int layer = blockIdx.x, tok = blockIdx.y;
  if (layer >= layers || tok >= t) return;
  const size_t base = (static_cast<size_t>(tok) * layers + layer) * P;
  float ss = 0.f;
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const float v = proj[base + i] * proj_scale;
    ss += v * v;
  }
  const float inv = rsqrtf(block_sum<128>(ss, red) / static_cast<float>(P) + eps);
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const float n = proj[base + i] * proj_scale * inv * (offset + w[i]);
    const float e = __half2float(emb[base + i]);
    out[base + i] = (n + e * emb_scale) * out_scale;
  }
}

__global__ void pl_gate_kernel(const float* __restrict__ g, const float* __restrict__ pli, int t,
                               int P, int layers, int layer, __half* __restrict__ out16) {
  griddep_wait();
  const size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (i >= static_cast<size_t>(t) * P) return;
  const size_t tok = i / P, c = i % P;
  const float x = g[i];
  float z = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  z = fminf(fmaxf(z, -15.0f), 15.0f);
  const float gl = 0.5f * x * (1.0f + tanhf(z));
  out16[i] = __float2half_rn(gl * pli[(tok * layers + layer) * P + c]);
}

// ---- logits at readout rows (logits.wgsl) ----------------------------------

// One 32-element block of a table row as stored (model.rs:338-371): its codes
// and its scale.
template <int DT>
struct RawBlock {
  uint4 c[DT == kF16 ? 4 : (DT == kQ8 ? 2 : 1)];
  float scale;
  uint32_t scale2;  // the f16 scale in both halves of a half2
};

template <int DT>
__device__ __forceinline__ void load_raw_block(const uint8_t* __restrict__ codes,
                                               const uint8_t* __restrict__ scales, size_t gb,
                                               bool ok, RawBlock<DT>& r) {
  constexpr int NC = DT == kF16 ? 4 : (DT == kQ8 ? 2 : 1);
  if (!ok) {
#pragma unroll
    for (int i = 0; i < NC; ++i) r.c[i] = make_uint4(0u, 0u, 0u, 0u);
    r.scale = 0.f;
    r.scale2 = 0u;
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(codes + gb * (NC * 16));
#pragma unroll
  for (int i = 0; i < NC; ++i) r.c[i] = src[i];
  if constexpr (DT == kF16) {
    r.scale = 1.f;
    r.scale2 = 0x3C003C00u;
  } else {
    const uint16_t sb = *reinterpret_cast<const uint16_t*>(scales + 2 * gb);
    r.scale = half_bits_to_float(sb);
    r.scale2 = static_cast<uint32_t>(sb) * 0x00010001u;
  }
}

// Elements 4 j .. 4 j + 3 of a block as f32 (QTensor::get, model.rs:508-525):
// Q4 blocks hold elements 0..15 in the low nibbles of their 16 bytes and
// 16..31 in the high nibbles.
template <int DT, int J>
__device__ __forceinline__ float4 raw_chunk(const RawBlock<DT>& r) {
  if constexpr (DT == kF16) {
    const uint4 q = r.c[J / 2];
    const uint32_t lo = (J & 1) ? q.z : q.x, hi = (J & 1) ? q.w : q.y;
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
    return make_float4(a.x, a.y, b.x, b.y);
  } else if constexpr (DT == kQ8) {
    // Code c as (c + 128) in the mantissa of 2^23, less 2^23 + 128: c exactly,
    // with integer and add instructions instead of the conversion unit.
    const uint4 q = r.c[J / 4];
    const uint32_t w = ((J & 3) == 0 ? q.x : (J & 3) == 1 ? q.y : (J & 3) == 2 ? q.z : q.w) ^
                       0x80808080u;
    return make_float4((__uint_as_float(0x4B000000u | (w & 0xff)) - 8388736.0f) * r.scale,
                       (__uint_as_float(0x4B000000u | ((w >> 8) & 0xff)) - 8388736.0f) * r.scale,
                       (__uint_as_float(0x4B000000u | ((w >> 16) & 0xff)) - 8388736.0f) * r.scale,
                       (__uint_as_float(0x4B000000u | (w >> 24)) - 8388736.0f) * r.scale);
  } else {
    // Nibble q in the mantissa of 2^23, less 2^23 + 8: q - 8 exactly.
    const uint4 q = r.c[0];
    const uint32_t w = (J & 3) == 0 ? q.x : (J & 3) == 1 ? q.y : (J & 3) == 2 ? q.z : q.w;
    constexpr int sh = J < 4 ? 0 : 4;
    return make_float4(
        (__uint_as_float(0x4B000000u | ((w >> sh) & 0xf)) - 8388616.0f) * r.scale,
        (__uint_as_float(0x4B000000u | ((w >> (8 + sh)) & 0xf)) - 8388616.0f) * r.scale,
        (__uint_as_float(0x4B000000u | ((w >> (16 + sh)) & 0xf)) - 8388616.0f) * r.scale,
        (__uint_as_float(0x4B000000u | ((w >> (24 + sh)) & 0xf)) - 8388616.0f) * r.scale);
  }
}

constexpr int kLogitsRows = 12;   // readout rows per pass over the table

template <int DT>
constexpr int logits_group() {
  return DT == kF16 ? 2 : 4;  // vocab rows a warp takes at once
}

// logits.wgsl in f32: out[r, v] = sum_k rows[r, k] * W[v, k] (+ the host
// softcap). A warp takes logits_group vocab rows at a time against up to
// kLogitsRows readout rows staged in shared memory. Lane l owns blocks
// l, l + 32, ... of each vocab row: its codes are one coalesced 16-byte
// piece per 16 bytes of block, and the next block's codes are requested while
// the current one is multiplied, so loads stay in flight. The readout rows'
// 16-byte chunk j of block b sits at chunk j ^ (b & 7) of the block, so the
// lanes' reads of one chunk are conflict-free. d % 32 == 0.
template <int DT>
__global__ void __launch_bounds__(256, 1) logits_kernel(const float* __restrict__ rows, int nrows,
                                                     const uint8_t* __restrict__ codes,
                                                     const uint8_t* __restrict__ scales,
                                                     int vocab, int d, float softcap,
                                                     float* __restrict__ out) {
  constexpr int G = logits_group<DT>();
  griddep_wait();
  extern __shared__ float4 xs4[];  // [kLogitsRows][d / 4], chunks swizzled per block
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = d / 32;
  const int nbl = (nb + 31) / 32;  // blocks per lane
  const int ngroups = (vocab + G - 1) / G;
  const int gstride = gridDim.x * (blockDim.x >> 5);
  const int d4 = d / 4;
  for (int r0 = 0; r0 < nrows; r0 += kLogitsRows) {
    const int nr = min(kLogitsRows, nrows - r0);
    __syncthreads();
    {
      const float4* src = reinterpret_cast<const float4*>(rows + static_cast<size_t>(r0) * d);
      const int n4 = nr * d4;
#pragma unroll 8
      for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const int r = i / d4, c = i - r * d4;  // chunk c of row r: block c / 8, chunk c % 8
        xs4[r * d4 + (c & ~7) + ((c ^ (c >> 3)) & 7)] = src[i];
      }
    }
    __syncthreads();
    int g = blockIdx.x * (blockDim.x >> 5) + warp;
    RawBlock<DT> cur[G], nxt[G];
    auto load = [&](RawBlock<DT>(&dst)[G], int gg, int i) {
      const int b = lane + 32 * i;
#pragma unroll
      for (int u = 0; u < G; ++u) {
        const int v = gg * G + u;
        load_raw_block<DT>(codes, scales, static_cast<size_t>(v) * nb + b, b < nb && v < vocab,
                           dst[u]);
      }
    };
    if (g < ngroups) load(cur, g, 0);
    for (; g < ngroups; g += gstride) {
      float acc[G][kLogitsRows];
#pragma unroll
      for (int u = 0; u < G; ++u)
#pragma unroll
        for (int r = 0; r < kLogitsRows; ++r) acc[u][r] = 0.f;
      for (int i = 0; i < nbl; ++i) {
        // The next (group, block) of this warp, fetched ahead.
        const int ng = i + 1 < nbl ? g : g + gstride;
        const int ni = i + 1 < nbl ? i + 1 : 0;
        if (ng < ngroups) load(nxt, ng, ni);
        const int b = lane + 32 * i;
        const float4* xb = xs4 + (b < nb ? b : 0) * 8;
        const int sw = b & 7;
#define OMG_LOGITS_CHUNK(J)                                                          \
  {                                                                                  \
    float4 x[kLogitsRows];                                                           \
    _Pragma("unroll") for (int r = 0; r < kLogitsRows; ++r) x[r] =                   \
        xb[(r < nr ? r : 0) * d4 + ((J) ^ sw)];                                      \
    float4 w[G];                                                                     \
    _Pragma("unroll") for (int u = 0; u < G; ++u) w[u] = raw_chunk<DT, J>(cur[u]);   \
    /* Component-major: consecutive FMAs update different accumulators. */           \
    _Pragma("unroll") for (int r = 0; r < kLogitsRows; ++r)                          \
        _Pragma("unroll") for (int u = 0; u < G; ++u) acc[u][r] =                    \
            fmaf(w[u].x, x[r].x, acc[u][r]);                                         \
    _Pragma("unroll") for (int r = 0; r < kLogitsRows; ++r)                          \
        _Pragma("unroll") for (int u = 0; u < G; ++u) acc[u][r] =                    \
            fmaf(w[u].y, x[r].y, acc[u][r]);                                         \
    _Pragma("unroll") for (int r = 0; r < kLogitsRows; ++r)                          \
        _Pragma("unroll") for (int u = 0; u < G; ++u) acc[u][r] =                    \
            fmaf(w[u].z, x[r].z, acc[u][r]);                                         \
    _Pragma("unroll") for (int r = 0; r < kLogitsRows; ++r)                          \
        _Pragma("unroll") for (int u = 0; u < G; ++u) acc[u][r] =                    \
            fmaf(w[u].w, x[r].w, acc[u][r]);                                         \
  }
        OMG_LOGITS_CHUNK(0)
        OMG_LOGITS_CHUNK(1)
        OMG_LOGITS_CHUNK(2)
        OMG_LOGITS_CHUNK(3)
        OMG_LOGITS_CHUNK(4)
        OMG_LOGITS_CHUNK(5)
        OMG_LOGITS_CHUNK(6)
        OMG_LOGITS_CHUNK(7)
#undef OMG_LOGITS_CHUNK
#pragma unroll
        for (int u = 0; u < G; ++u) cur[u] = nxt[u];
      }
#pragma unroll
      for (int u = 0; u < G; ++u)
#pragma unroll
        for (int r = 0; r < kLogitsRows; ++r) {
          if (r < nr) {
            float z = warp_sum(acc[u][r]);
            const int v = g * G + u;
            if (lane == 0 && v < vocab) {
              if (softcap > 0.f) z = softcap * tanhf(z / softcap);
              out[static_cast<size_t>(r0 + r) * vocab + v] = z;
            }
          }
        }
    }
  }
}

// ---- lm_head on the tensor cores ---------------------------------------------
//
// logits.wgsl in f32 on tcgen05: a CTA takes 128-row tiles of the packed
// embedding table (M = 128 vocab rows) against up to 32 readout rows (N = 32)
// over K = d in 64-wide steps. Eight warps dequantize the table's Q4_0 / Q8_0
// / f16 blocks straight from HBM into 128-byte-swizzled f16 tiles in shared
// memory (each thread half a row: one 32-element block), the MMA thread
// multiplies. W = (q - 8) d has at most 15 significant bits and each readout
// value 24, so both are split into f16 hi + lo and three products
// W_hi X_hi + W_hi X_lo + W_lo X_hi (exact f16 x f16 products, f32
// accumulation) keep the f32 dot product of logits.wgsl: the dropped
// W_lo X_lo term is ~2^-22 of each product.
//
//   warp 0      MMA (lane 0)
//   warp 1      TMEM allocation
//   warps 2-9   dequant: row 32 (w & 3) + lane of the tile, block 2 kb + half
//               of K step kb; then, for the previous tile, the epilogue:
//               the thread owning a TMEM lane (vocab row) writes its logits
//               for every readout row, softcapped (engine.rs:1901-1906)
constexpr int LT_STAGES = 3;
constexpr int LT_N = 32;                          // readout rows per pass
constexpr int LT_W_BYTES = 128 * 128;             // 128 rows x 64 f16
constexpr int LT_X_BYTES = LT_N * 128;            // 32 rows x 64 f16
constexpr int LT_STAGE = 2 * LT_W_BYTES + 2 * LT_X_BYTES;  // W hi, W lo, X hi, X lo
constexpr int LT_SMEM = 1024 + LT_STAGES * LT_STAGE + 256;
constexpr int LT_THREADS = 320;

__device__ __forceinline__ void split_store8(uint8_t* hi_row, uint8_t* lo_row, int piece, int r,
                                             const float* v) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __half2 a = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
    const float2 af = __half22float2(a);
    const __half2 b = __floats2half2_rn(v[2 * e] - af.x, v[2 * e + 1] - af.y);
    h[e] = *reinterpret_cast<const uint32_t*>(&a);
    l[e] = *reinterpret_cast<const uint32_t*>(&b);
  }
  const int off = ((piece ^ (r & 7)) << 4);
  *reinterpret_cast<uint4*>(hi_row + off) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(lo_row + off) = make_uint4(l[0], l[1], l[2], l[3]);
}

// Elements 8 PC .. 8 PC + 7 of a table block as f16 hi + lo (W = hi + lo;
// hi = f16(W)), computed in half2: a code pair is permuted into the two
// 16-bit lanes as 1024 + q (the f16 0x6400 | q), one subtraction gives the
// signed code exactly, hi = f16(code x d) is the f16 product, and
// lo = code x d - hi (an f16 fma: the residual's <= 4 significant bits are
// exact unless it falls below the f16 normal range).
template <int DT, int PC>
__device__ __forceinline__ void raw_piece_f16(const RawBlock<DT>& r, uint4& hi, uint4& lo) {
  if constexpr (DT == kF16) {
    // Each 16-byte chunk of an f16 block holds 8 values: piece PC is chunk PC.
    hi = r.c[PC];
    lo = make_uint4(0u, 0u, 0u, 0u);
  } else {
    const __half2 d2 = bits_half2(r.scale2);  // the block's f16 scale
    uint32_t w0, w1;
    __half2 bias;
    uint32_t key;
    if constexpr (DT == kQ8) {
      const uint4 q = r.c[PC / 2];
      w0 = (PC & 1) ? q.z : q.x;
      w1 = (PC & 1) ? q.w : q.y;
      bias = bits_half2(0x64806480u);  // 1152 = 1024 + 128: codes stored as c + 128
      key = 0x64806480u;                 // (c ^ 0x80) | 0x6400 per lane
    } else {
      const uint4 q = r.c[0];
      // Low nibbles of bytes 0..15 are elements 0..15, high nibbles 16..31.
      w0 = (PC & 1) ? q.z : q.x;
      w1 = (PC & 1) ? q.w : q.y;
      if (PC >= 2) {
        w0 >>= 4;
        w1 >>= 4;
      }
      bias = bits_half2(0x64086408u);  // 1032 = 1024 + 8: w = (q - 8) d
      key = 0x64006400u;
    }
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t w = e < 2 ? w0 : w1;
      uint32_t x = __byte_perm(w, 0u, (e & 1) ? 0x4342u : 0x4140u);  // bytes -> 16-bit lanes
      x = DT == kQ8 ? (x ^ key) : ((x & 0x000F000Fu) | key);
      const __half2 c = __hsub2(*reinterpret_cast<const __half2*>(&x), bias);
      const __half2 hv = __hmul2(c, d2);
      const __half2 lv = __hfma2(c, d2, __hneg2(hv));
      h[e] = *reinterpret_cast<const uint32_t*>(&hv);
      l[e] = *reinterpret_cast<const uint32_t*>(&lv);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

template <int DT>
__global__ void __launch_bounds__(LT_THREADS, 1)
    logits_tc_kernel(const float* __restrict__ rows, int nrows, const uint8_t* __restrict__ codes,
                     const uint8_t* __restrict__ scales, int vocab, int d, float softcap,
                     float* __restrict__ out, uint32_t* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  auto stage = [&](int s) { return sm + s * LT_STAGE; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + LT_STAGES * LT_STAGE);
  uint64_t* full = bars;                    // [stages] 8 dequant warps
  uint64_t* empty = full + LT_STAGES;       // [stages] MMA commit
  uint64_t* tfull = empty + LT_STAGES;      // [2] MMA commit
  uint64_t* tempty = tfull + 2;             // [2] 8 epilogue warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = d / 32, ksteps = d / 64;
  const int tiles = (vocab + 127) / 128;
  const int rgroups = (nrows + LT_N - 1) / LT_N;
  const int units = tiles * rgroups;  // (vocab tile, group of 32 readout rows)
  if (threadIdx.x == 0) {
    for (int i = 0; i < LT_STAGES; ++i) {
      mbar_init(&full[i], 8);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(128, LT_N);
      int it = 0, local = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x, ++local) {
        const int b = local & 1;
        if (!mbar_wait(&tempty[b], ((local >> 1) & 1) ^ 1, abort_flag, status)) break;
        tc_fence_after();
        const uint32_t acc = tmem + 32u * b;
        bool ok = true;
        for (int kb = 0; kb < ksteps; ++kb, ++it) {
          const int s = it % LT_STAGES;
          if (!mbar_wait(&full[s], (it / LT_STAGES) & 1, abort_flag, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* st = stage(s);
          const uint64_t wh = sw128_desc(st), wl = sw128_desc(st + LT_W_BYTES);
          const uint64_t xh = sw128_desc(st + 2 * LT_W_BYTES);
          const uint64_t xl = sw128_desc(st + 2 * LT_W_BYTES + LT_X_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            umma_f16(acc, wh + 2 * k, xh + 2 * k, idesc, (kb | k) ? 1u : 0u);
            umma_f16(acc, wh + 2 * k, xl + 2 * k, idesc, 1u);
            umma_f16(acc, wl + 2 * k, xh + 2 * k, idesc, 1u);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
      }
    }
  } else if (warp >= 2) {
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = 32 * q + lane;  // this thread's tile row (and TMEM lane)
    const int t256 = threadIdx.x - 64;
    auto epilogue = [&](int u, int local) -> bool {
      const int b = local & 1;
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&tfull[b], (local >> 1) & 1, abort_flag, status) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) return false;
      tc_fence_after();
      // Both halves read the row's 32 columns; each writes 16 readout rows.
      float z[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + 32u * b, z);
      const int v = (u / rgroups) * 128 + r;
      const int r0 = (u % rgroups) * LT_N;
      if (v < vocab) {
        // Registers are indexed at compile time: one loop per half.
        auto put = [&](int j, float x) {
          const int rr = r0 + 16 * half + j;
          if (rr < nrows) {
            if (softcap > 0.f) x = softcap * tanhf(x / softcap);
            out[static_cast<size_t>(rr) * vocab + v] = x;
          }
        };
        if (half == 0) {
#pragma unroll
          for (int j = 0; j < 16; ++j) put(j, z[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) put(j, z[16 + j]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
      return true;
    };
    // The steps of this CTA's units in order: step i is K step i % ksteps of
    // local unit i / ksteps. Each thread keeps the packed block and readout
    // values of the next four steps in flight in registers (a ring indexed
    // at compile time), so a step's conversion never waits on HBM.
    const int n_local = units > static_cast<int>(blockIdx.x)
                            ? (units - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                            : 0;
    const int steps = n_local * ksteps;
    const int xr = t256 >> 3, xp = t256 & 7;
    RawBlock<DT> rb[4];
    float4 xa[4], xb[4];
    // The fetch position (step fi: K step f_kb of local unit f_lu) advances
    // one step per call, in step order, so the unit's table row and readout
    // row are recomputed once per unit instead of dividing per step.
    int fi = 0, f_lu = 0, f_kb = 0;
    int f_v = 0, f_rr = 0;
    auto unit_rows = [&]() {
      const int u = static_cast<int>(blockIdx.x) + f_lu * static_cast<int>(gridDim.x);
      f_v = (u / rgroups) * 128 + r;
      f_rr = (u % rgroups) * LT_N + xr;
    };
    unit_rows();
    auto fetch = [&](RawBlock<DT>& dst, float4& a, float4& b) {
      const bool live = fi < steps;
      load_raw_block<DT>(codes, scales, static_cast<size_t>(f_v) * nb + 2 * f_kb + half,
                         live && f_v < vocab, dst);
      if (live && f_rr < nrows) {
        const float4* src =
            reinterpret_cast<const float4*>(rows + static_cast<size_t>(f_rr) * d + f_kb * 64 + 8 * xp);
        a = __ldg(src);
        b = __ldg(src + 1);
      } else {
        a = b = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      ++fi;
      if (++f_kb == ksteps) {
        f_kb = 0;
        ++f_lu;
        unit_rows();
      }
    };
#pragma unroll
    for (int j = 0; j < 4; ++j) fetch(rb[j], xa[j], xb[j]);
    int prev = -1;
    bool ok = true;
    int s = 0, sph = 0;     // ring slot of step i and its wrap count
    int kb_i = 0, lu_i = 0; // K step and local unit of step i
    for (int i0 = 0; i0 < steps && ok; i0 += 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = i0 + j;
        if (i >= steps || !ok) break;
        if (i >= LT_STAGES) {
          int w = 0;
          if (lane == 0) w = mbar_wait(&empty[s], (sph & 1) ^ 1, abort_flag, status) ? 1 : 0;
          if (!__shfl_sync(0xffffffffu, w, 0)) {
            ok = false;
            break;
          }
        }
        uint8_t* st = stage(s);
        // W: this thread's 32-element block of its row as f16 hi / lo, in
        // pieces of 8 values.
#define OMG_LT_PIECE(PC)                                                             \
  {                                                                                  \
    uint4 hv, lv;                                                                    \
    raw_piece_f16<DT, PC>(rb[j], hv, lv);                                            \
    const int off = r * 128 + (((4 * half + (PC)) ^ (r & 7)) << 4);                 \
    *reinterpret_cast<uint4*>(st + off) = hv;                                        \
    *reinterpret_cast<uint4*>(st + LT_W_BYTES + off) = lv;                           \
  }
        OMG_LT_PIECE(0)
        OMG_LT_PIECE(1)
        OMG_LT_PIECE(2)
        OMG_LT_PIECE(3)
#undef OMG_LT_PIECE
        // X: 32 readout rows x 64 values of this K step, 8 per thread.
        {
          const float x8[8] = {xa[j].x, xa[j].y, xa[j].z, xa[j].w,
                               xb[j].x, xb[j].y, xb[j].z, xb[j].w};
          split_store8(st + 2 * LT_W_BYTES + xr * 128, st + 2 * LT_W_BYTES + LT_X_BYTES + xr * 128,
                       xp, xr, x8);
        }
        // Every thread's stores to the async proxy, then one arrival per warp.
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
        fetch(rb[j], xa[j], xb[j]);
        if (++s == LT_STAGES) {
          s = 0;
          ++sph;
        }
        if (++kb_i == ksteps) {
          kb_i = 0;
          // The previous unit's logits (its MMAs ran while this one was staged).
          if (prev >= 0 && !epilogue(prev, lu_i - 1)) {
            ok = false;
            break;
          }
          prev = static_cast<int>(blockIdx.x) + lu_i * static_cast<int>(gridDim.x);
          ++lu_i;
        }
      }
    }
    if (ok && prev >= 0) epilogue(prev, n_local - 1);
  }
  griddep_launch();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// The lm_head's block decoder (raw_piece_f16) over a whole table, row-major
// hi and lo f16 outputs: the values logits_tc_kernel stages in shared memory.
template <int DT>
__global__ void table_hilo_kernel(const uint8_t* __restrict__ codes,
                                  const uint8_t* __restrict__ scales, size_t nblk,
                                  __half* __restrict__ hi, __half* __restrict__ lo) {
  for (size_t b = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; b < nblk;
       b += static_cast<size_t>(gridDim.x) * blockDim.x) {
    RawBlock<DT> rb;
    load_raw_block<DT>(codes, scales, b, true, rb);
    uint4 h[4], l[4];
    raw_piece_f16<DT, 0>(rb, h[0], l[0]);
    raw_piece_f16<DT, 1>(rb, h[1], l[1]);
    raw_piece_f16<DT, 2>(rb, h[2], l[2]);
    raw_piece_f16<DT, 3>(rb, h[3], l[3]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      reinterpret_cast<uint4*>(hi + b * 32)[i] = h[i];
      reinterpret_cast<uint4*>(lo + b * 32)[i] = l[i];
    }
  }
}

// One thread per (row, 32-element block) of the pushed weight: its codes
// and scale into the chunk layout of packed.cuh.
template <int DT>
__global__ void pack_weight_kernel(const uint8_t* __restrict__ codes,
                                   const uint8_t* __restrict__ scales, int rows, int k, int remap,
                                   uint8_t* __restrict__ out) {
  using P = PackChunk<DT>;
  const int kb32 = k / 32, ksteps = (k + 63) / 64;
  const size_t nblk = static_cast<size_t>(rows) * kb32;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nblk;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / kb32), blk = static_cast<int>(i % kb32);
    const int dr = remap_row(r, remap);
    uint8_t* chunk = out + (static_cast<size_t>(dr / 128) * ksteps + blk / 2) * P::BYTES;
    const int b = blk & 1, cr = dr % 128;
    const uint4* src = reinterpret_cast<const uint4*>(codes + i * P::CODE_BYTES);
    uint4* dst = reinterpret_cast<uint4*>(chunk + (b * 128 + cr) * P::CODE_BYTES);
    dst[0] = src[0];
    if constexpr (DT == kQ8) dst[1] = src[1];
    *reinterpret_cast<uint16_t*>(chunk + P::CODES + (b * 128 + cr) * 2) =
        static_cast<uint16_t>(scales[2 * i]) | (static_cast<uint16_t>(scales[2 * i + 1]) << 8);
  }
}

// One thread per (row, 32-element block): the GEMM's tile decoder, written
// row-major.
template <int DT>
__global__ void unpack_weight_kernel(const uint8_t* __restrict__ packed, int rows, int k,
                                     __half* __restrict__ out) {
  using P = PackChunk<DT>;
  const int kb32 = k / 32, ksteps = (k + 63) / 64;
  const size_t nblk = static_cast<size_t>(rows) * kb32;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nblk;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / kb32), blk = static_cast<int>(i % kb32);
    const uint8_t* chunk = packed + (static_cast<size_t>(r / 128) * ksteps + blk / 2) * P::BYTES;
    uint4 pc[4];
    unpack_block<DT>(chunk, r % 128, blk & 1, pc);
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(r) * k + blk * 32);
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = pc[j];
  }
}

}  // namespace

void launch_pack_weight(int dtype, const void* codes, const void* scales, int rows, int k,
                        int remap, int out_rows, uint8_t* out, cudaStream_t s) {
  (void)out_rows;
  const size_t nblk = static_cast<size_t>(rows) * (k / 32);
  const int grid = static_cast<int>(std::min<size_t>((nblk + 255) / 256, 148 * 16));
  const auto* c = static_cast<const uint8_t*>(codes);
  const auto* sc = static_cast<const uint8_t*>(scales);
  if (dtype == kQ4)
    pack_weight_kernel<kQ4><<<grid, 256, 0, s>>>(c, sc, rows, k, remap, out);
  else
    pack_weight_kernel<kQ8><<<grid, 256, 0, s>>>(c, sc, rows, k, remap, out);
}

void launch_unpack_weight(int dtype, const uint8_t* packed, int rows, int k, __half* out,
                          cudaStream_t s) {
  const size_t nblk = static_cast<size_t>(rows) * (k / 32);
  const int grid = static_cast<int>(std::min<size_t>((nblk + 255) / 256, 148 * 16));
  if (dtype == kQ4)
    unpack_weight_kernel<kQ4><<<grid, 256, 0, s>>>(packed, rows, k, out);
  else
    unpack_weight_kernel<kQ8><<<grid, 256, 0, s>>>(packed, rows, k, out);
}

void launch_table_hilo(int dtype, const void* codes, const void* scales, size_t n, __half* hi,
                       __half* lo, cudaStream_t s) {
  const size_t nblk = n / 32;
  const int grid = static_cast<int>(std::min<size_t>((nblk + 255) / 256, 148 * 16));
  const auto* c = static_cast<const uint8_t*>(codes);
  const auto* sc = static_cast<const uint8_t*>(scales);
  if (dtype == kQ4)
    table_hilo_kernel<kQ4><<<grid, 256, 0, s>>>(c, sc, nblk, hi, lo);
  else if (dtype == kQ8)
    table_hilo_kernel<kQ8><<<grid, 256, 0, s>>>(c, sc, nblk, hi, lo);
  else
    table_hilo_kernel<kF16><<<grid, 256, 0, s>>>(c, sc, nblk, hi, lo);
}

void launch_dequant_f16(int dtype, const void* codes, const void* scales, int rows, int k,
                        int remap, __half* out, cudaStream_t s) {
  const size_t nblk = static_cast<size_t>(rows) * (k / 32);
  const int threads = 256;
  const int grid = static_cast<int>(std::min<size_t>((nblk + threads - 1) / threads, 148 * 16));
  dequant_f16_kernel<<<grid, threads, 0, s>>>(dtype, static_cast<const uint8_t*>(codes),
                                              static_cast<const uint8_t*>(scales), rows, k, remap,
                                              out);
}

void launch_embed_norm(int dtype, const int* ids, int t, const void* codes, const void* scales,
                       int d, float scale, const float* w, float eps, float offset, float* x,
                       __half* x16, __half* h16, int ldh, cudaStream_t s) {
  const auto* c = static_cast<const uint8_t*>(codes);
  const auto* sc = static_cast<const uint8_t*>(scales);
  if (dtype == kQ4)
    launch_pdl(embed_norm_kernel<kQ4>, dim3(t), dim3(128), 0, s, ids, t, c, sc, d, scale, w, eps, offset,
               x, x16, h16, ldh);
  else if (dtype == kQ8)
    launch_pdl(embed_norm_kernel<kQ8>, dim3(t), dim3(128), 0, s, ids, t, c, sc, d, scale, w, eps, offset,
               x, x16, h16, ldh);
  else
    launch_pdl(embed_norm_kernel<kF16>, dim3(t), dim3(128), 0, s, ids, t, c, sc, d, scale, w, eps, offset,
               x, x16, h16, ldh);
}

void launch_residual_norm(const float* a, int splits, size_t split_stride, int lda, int t, int d,
                          const float* w1, float eps, float offset, float out_scale, float* x,
                          __half* x16, const float* w2, __half* h16, int ldh,
                          const int* row_map, float* rows_out, cudaStream_t s) {
  if (t <= 0) return;
  // Config::validate caps d at 8192.
  const int nv = d <= 1024 ? 1 : d <= 4096 ? 2 : 4;
  const int threads = ((d + 4 * nv - 1) / (4 * nv) + 31) / 32 * 32;
#define OMG_NORM(NV)                                                                        \
  launch_pdl(residual_norm_kernel<NV>, dim3(t), dim3(threads), 0, s, a, splits,              \
             split_stride, lda, t, d, w1, eps, offset, out_scale, x, x16, w2, h16, ldh, row_map, \
             rows_out)
  if (nv == 1)
    OMG_NORM(1);
  else if (nv == 2)
    OMG_NORM(2);
  else
    OMG_NORM(4);
#undef OMG_NORM
}

void launch_pl_combine(const float* proj, int t, int P, int layers, const float* w,
                       const __half* emb, float eps, float offset, float proj_scale,
                       float emb_scale, float out_scale, float* out, cudaStream_t s) {
  dim3 grid(layers, t);
  launch_pdl(pl_combine_kernel, grid, dim3(128), 0, s, proj, t, P, layers, w, emb, eps, offset,
             proj_scale, emb_scale, out_scale, out);
}

void launch_pl_gate(const float* g, const float* pli, int t, int P, int layers, int layer,
                    __half* out16, cudaStream_t s) {
  const size_t n = static_cast<size_t>(t) * P;
  launch_pdl(pl_gate_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, s, g, pli,
             t, P, layers, layer, out16);
}

namespace {

// The RoPE rotation of qk_prep.wgsl:52-64 for every position < n_pos and
// pair dd < half: angle = pos * theta^(-dd / half), the same float
// operations qk_prep_kernel performs per token.
__global__ void rope_table_kernel(float theta, int half, int n_pos, float2* tab) {
  const int n = n_pos * half;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int dd = i / n_pos, p = i % n_pos;
    const float ang =
        static_cast<float>(p) * powf(theta, -static_cast<float>(dd) / static_cast<float>(half));
    float sn, cs;
    sincosf(ang, &sn, &cs);
    tab[i] = make_float2(cs, sn);
  }
}

}  // namespace

void launch_rope_table(float theta, int half, int n_pos, float2* tab, cudaStream_t s) {
  const int n = n_pos * half;
  rope_table_kernel<<<std::max(1, std::min(2048, (n + 255) / 256)), 256, 0, s>>>(theta, half,
                                                                                   n_pos, tab);
}

void launch_qk_prep(const QkArgs& a, cudaStream_t s) {
  if (a.hd == 512)
    launch_pdl(qk_prep_kernel<512>, dim3(a.t), dim3(128), 0, s, a);
  else
    launch_pdl(qk_prep_kernel<256>, dim3(a.t), dim3(128), 0, s, a);
}

void logits_setup_device(int d) {
  cudaFuncSetAttribute(logits_tc_kernel<kQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize, LT_SMEM);
  cudaFuncSetAttribute(logits_tc_kernel<kQ8>, cudaFuncAttributeMaxDynamicSharedMemorySize, LT_SMEM);
  cudaFuncSetAttribute(logits_tc_kernel<kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, LT_SMEM);
  const int smem = kLogitsRows * d * 4;
  cudaFuncSetAttribute(logits_kernel<kQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(logits_kernel<kQ8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(logits_kernel<kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

void launch_logits(int dtype, const float* rows, int nrows, const void* codes, const void* scales,
                   int vocab, int d, float softcap, float* out, int num_sms, uint32_t* status,
                   cudaStream_t s) {
  if (nrows <= 0) return;
  const size_t smem = static_cast<size_t>(kLogitsRows) * d * 4;
  const auto* c = static_cast<const uint8_t*>(codes);
  const auto* sc = static_cast<const uint8_t*>(scales);
  if (d % 64 == 0) {
    const int units = ((vocab + 127) / 128) * ((nrows + LT_N - 1) / LT_N);
    const int sms = num_sms > 0 ? num_sms : 148;
    const dim3 grid(units < sms ? units : sms);
    if (dtype == kQ4)
      launch_pdl(logits_tc_kernel<kQ4>, grid, dim3(LT_THREADS), LT_SMEM, s, rows, nrows, c, sc, vocab,
                 d, softcap, out, status);
    else if (dtype == kQ8)
      launch_pdl(logits_tc_kernel<kQ8>, grid, dim3(LT_THREADS), LT_SMEM, s, rows, nrows, c, sc, vocab,
                 d, softcap, out, status);
    else
      launch_pdl(logits_tc_kernel<kF16>, grid, dim3(LT_THREADS), LT_SMEM, s, rows, nrows, c, sc,
                 vocab, d, softcap, out, status);
    return;
  }
  // Persistent sweep of the table: one CTA per SM, staging the readout rows
  // once; 8 warps per CTA, a group of vocab rows per warp at a time.
  const int groups = (vocab + 1) / 2;  // an upper bound for every table type
  const int grid = std::max(1, std::min((groups + 7) / 8, num_sms > 0 ? num_sms : 148));
  if (dtype == kQ4) {
    launch_pdl(logits_kernel<kQ4>, dim3(grid), dim3(256), smem, s, rows, nrows, c, sc, vocab, d, softcap,
               out);
  } else if (dtype == kQ8) {
    launch_pdl(logits_kernel<kQ8>, dim3(grid), dim3(256), smem, s, rows, nrows, c, sc, vocab, d, softcap,
               out);
  } else {
    launch_pdl(logits_kernel<kF16>, dim3(grid), dim3(256), smem, s, rows, nrows, c, sc, vocab, d, softcap,
               out);
  }
}

}  // namespace omg
