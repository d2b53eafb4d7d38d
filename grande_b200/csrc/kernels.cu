// Row kernels of the decoder pass (see kernels.cuh). Reference shaders:
// crates/omg-wgpu/src/shaders/{weight,embed,rmsnorm,qk_prep,logits}.wgsl.
#include "kernels.cuh"
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

constexpr int kNormThreads = 256;  // NV float4 per thread: d <= 1024 NV

template <int NV>
__global__ void __launch_bounds__(kNormThreads) residual_norm_kernel(
    const float* __restrict__ a, int splits, size_t split_stride, int lda, int t, int d,
    const float* __restrict__ w1, float eps, float offset, float out_scale, float* __restrict__ x,
    __half* __restrict__ x16, const float* __restrict__ w2, __half* __restrict__ h16, int ldh,
    const int* __restrict__ row_map, float* __restrict__ rows_out) {
  griddep_wait();
  // Let the next kernel start its prologue; its CTAs wait for this grid.
  griddep_launch();
  __shared__ float red[kNormThreads / 32];
  const int row = blockIdx.x;
  if (row >= t) return;
  const float* ar = a + static_cast<size_t>(row) * lda;
  float* xr = x + static_cast<size_t>(row) * d;
  // Every load of the row up front (the slabs, the residual row and both
  // norms' weights): only the two reductions order the work after them.
  float4 y[NV], xo[NV], wa[NV], wb[NV];
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = (threadIdx.x + j * kNormThreads) * 4;
    y[j] = xo[j] = wa[j] = wb[j] = zero;
    if (i < d) {
      y[j] = *reinterpret_cast<const float4*>(ar + i);
      xo[j] = *reinterpret_cast<const float4*>(xr + i);
      wa[j] = *reinterpret_cast<const float4*>(w1 + i);
      if (w2) wb[j] = *reinterpret_cast<const float4*>(w2 + i);
    }
  }
  for (int z = 1; z < splits; ++z) {
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = (threadIdx.x + j * kNormThreads) * 4;
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
  const float inv1 = rsqrtf(block_sum<kNormThreads>(ss, red) / static_cast<float>(d) + eps);
  float ss2 = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = (threadIdx.x + j * kNormThreads) * 4;
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
  const float inv2 = rsqrtf(block_sum<kNormThreads>(ss2, red) / static_cast<float>(d) + eps);
  const int out_row = row_map ? row_map[row] : -1;
  __half* hr = h16 ? h16 + static_cast<size_t>(row) * ldh : nullptr;
  float* orow = out_row >= 0 ? rows_out + static_cast<size_t>(out_row) * d : nullptr;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = (threadIdx.x + j * kNormThreads) * 4;
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

// Element k (k % 4 == 0) and the three after it of vocab row v as f32
// (QTensor::get): Q4 blocks hold elements 0..15 in the low nibbles of their
// 16 bytes and 16..31 in the high nibbles.
template <int DT>
__device__ __forceinline__ float4 load4_f32(const uint8_t* __restrict__ codes,
                                            const uint8_t* __restrict__ scales, size_t v, int nb,
                                            int k) {
  const size_t gb = v * nb + (k >> 5);
  const int e = k & 31;
  if constexpr (DT == kF16) {
    const uint2 q = *reinterpret_cast<const uint2*>(codes + (gb * 32 + e) * 2);
    const __half2 a = *reinterpret_cast<const __half2*>(&q.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&q.y);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
  } else {
    const uint16_t sb =
        static_cast<uint16_t>(scales[2 * gb]) | (static_cast<uint16_t>(scales[2 * gb + 1]) << 8);
    const float dq = half_bits_to_float(sb);
    if constexpr (DT == kQ8) {
      const uint32_t q = *reinterpret_cast<const uint32_t*>(codes + gb * 32 + e);
      return make_float4(static_cast<float>(static_cast<int8_t>(q & 0xff)) * dq,
                         static_cast<float>(static_cast<int8_t>((q >> 8) & 0xff)) * dq,
                         static_cast<float>(static_cast<int8_t>((q >> 16) & 0xff)) * dq,
                         static_cast<float>(static_cast<int8_t>(q >> 24)) * dq);
    } else {
      const uint32_t q = *reinterpret_cast<const uint32_t*>(codes + gb * 16 + (e & 15));
      const int sh = e < 16 ? 0 : 4;
      return make_float4((static_cast<float>((q >> sh) & 0xf) - 8.0f) * dq,
                         (static_cast<float>((q >> (8 + sh)) & 0xf) - 8.0f) * dq,
                         (static_cast<float>((q >> (16 + sh)) & 0xf) - 8.0f) * dq,
                         (static_cast<float>((q >> (24 + sh)) & 0xf) - 8.0f) * dq);
    }
  }
}

constexpr int kLogitsVocab = 4;   // vocab rows per warp at once
constexpr int kLogitsRows = 12;   // readout rows per pass over the table

// logits.wgsl in f32: out[r, v] = sum_k rows[r, k] * W[v, k] (+ the host
// softcap). A warp takes kLogitsVocab vocab rows against up to kLogitsRows
// readout rows staged in shared memory; lane l owns elements 4 l + 128 i,
// so each readout float4 it reads from shared memory serves kLogitsVocab
// rows of the table and a warp's reads are conflict-free. d % 32 == 0.
template <int DT>
__global__ void __launch_bounds__(256) logits_kernel(const float* __restrict__ rows, int nrows,
                                                     const uint8_t* __restrict__ codes,
                                                     const uint8_t* __restrict__ scales,
                                                     int vocab, int d, float softcap,
                                                     float* __restrict__ out) {
  griddep_wait();
  extern __shared__ float xs[];  // [kLogitsRows][d]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int nb = d / 32;
  const int steps = (d + 127) / 128;
  for (int r0 = 0; r0 < nrows; r0 += kLogitsRows) {
    const int nr = min(kLogitsRows, nrows - r0);
    __syncthreads();
    for (int i = threadIdx.x; i < nr * d; i += blockDim.x)
      xs[i] = rows[static_cast<size_t>(r0) * d + i];
    __syncthreads();
    for (int v0 = (blockIdx.x * nwarps + warp) * kLogitsVocab; v0 < vocab;
         v0 += gridDim.x * nwarps * kLogitsVocab) {
      float acc[kLogitsVocab][kLogitsRows];
#pragma unroll
      for (int u = 0; u < kLogitsVocab; ++u)
#pragma unroll
        for (int r = 0; r < kLogitsRows; ++r) acc[u][r] = 0.f;
#pragma unroll 2
      for (int i = 0; i < steps; ++i) {
        const int k = 4 * lane + 128 * i;
        if (k >= d) continue;  // d % 32 == 0: the lane's four elements are all in or all out
        float4 w[kLogitsVocab];
#pragma unroll
        for (int u = 0; u < kLogitsVocab; ++u)
          w[u] = v0 + u < vocab ? load4_f32<DT>(codes, scales, static_cast<size_t>(v0 + u), nb, k)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < kLogitsRows; ++r) {
          if (r < nr) {
            const float4 x = *reinterpret_cast<const float4*>(xs + r * d + k);
#pragma unroll
            for (int u = 0; u < kLogitsVocab; ++u)
              acc[u][r] += w[u].x * x.x + w[u].y * x.y + w[u].z * x.z + w[u].w * x.w;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kLogitsVocab; ++u)
#pragma unroll
        for (int r = 0; r < kLogitsRows; ++r) {
          if (r < nr) {
            float z = warp_sum(acc[u][r]);
            if (lane == 0 && v0 + u < vocab) {
              if (softcap > 0.f) z = softcap * tanhf(z / softcap);
              out[static_cast<size_t>(r0 + r) * vocab + v0 + u] = z;
            }
          }
        }
    }
  }
}

}  // namespace

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
#define OMG_NORM(NV)                                                                        \
  launch_pdl(residual_norm_kernel<NV>, dim3(t), dim3(kNormThreads), 0, s, a, splits,         \
             split_stride, lda, t, d, w1, eps, offset, out_scale, x, x16, w2, h16, ldh, row_map, \
             rows_out)
  if (d <= 1024)
    OMG_NORM(1);
  else if (d <= 2048)
    OMG_NORM(2);
  else if (d <= 4096)
    OMG_NORM(4);
  else
    OMG_NORM(8);
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
  const int smem = kLogitsRows * d * 4;
  cudaFuncSetAttribute(logits_kernel<kQ4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(logits_kernel<kQ8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(logits_kernel<kF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

void launch_logits(int dtype, const float* rows, int nrows, const void* codes, const void* scales,
                   int vocab, int d, float softcap, float* out, int num_sms, cudaStream_t s) {
  if (nrows <= 0) return;
  const size_t smem = static_cast<size_t>(kLogitsRows) * d * 4;
  const auto* c = static_cast<const uint8_t*>(codes);
  const auto* sc = static_cast<const uint8_t*>(scales);
  // One sweep of the table: 4 vocab rows per warp, 8 warps per CTA.
  (void)num_sms;
  const int grid = (vocab + 31) / 32;
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
