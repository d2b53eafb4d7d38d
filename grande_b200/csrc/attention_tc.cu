// Block-causal GQA attention on the 5th-generation tensor cores, head_dim 256
// (see attention.cuh). Replaces crates/omg-wgpu/src/shaders/attention.wgsl
// for the decoder's head_dim-256 layers.
//
// One CTA = one work item: 128 query rows (a run's tokens x the query heads of
// one KV head) against one 128-key tile.
//
//   warp 0  TMA: Q (4 x [128 rows][64 dims]), K and V tiles of the cache
//   warp 1  MMA: S = Q K^T (M 128, N 128, K 256) into TMEM; after the softmax,
//           O = P V (M 128, N 256, K 128 keys, V read MN-major as stored)
//   warps 2-5  one query row per thread (its TMEM lane): mask, max, exp, sum,
//           P to shared memory, then O out of TMEM to global memory
//
// Numerics follow attention.wgsl: Q, K, V f16; scores, max, exp and the row
// sum f32. The probabilities enter the tensor-core product as an f16 pair
// hi + lo (two MMAs), so P carries ~22 bits rather than f16's 11.
#include <algorithm>
#include <climits>
#include <cstdio>

#include "attention.cuh"
#include "gemm.cuh"
#include "ptx.cuh"

namespace omg {

namespace {

constexpr int TA_HD = 256;
constexpr int TA_CHUNK = 16384;                        // [128 rows][128 bytes]
constexpr int TA_Q_BYTES = 4 * TA_CHUNK;               // 128 rows x 256 dims
constexpr int TA_KV_BYTES = 4 * TA_CHUNK;              // 128 keys x 256 dims
constexpr int TA_SMEM = 1024 + TA_Q_BYTES + 2 * TA_KV_BYTES + 256;
constexpr uint32_t TA_TMEM_COLS = 256;                 // O [128 x 256]; S overlays cols 0..127
constexpr float kLog2e = 1.4426950408889634f;

enum { BAR_Q = 0, BAR_K, BAR_V, BAR_S, BAR_P, BAR_O, NBARS };

__device__ __forceinline__ uint32_t pack_h2(float x, float y) {
  __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Wait on a barrier with one lane of the warp and share the outcome, so the
// warp stays converged for the .sync.aligned tcgen05 loads that follow.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint32_t* status, int lane) {
  int ok = 0;
  if (lane == 0) ok = mbar_wait(bar, parity, abort_flag, status) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <bool PLO>
__global__ void __launch_bounds__(192, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkv,
                        AttnTcArgs g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* qs = sm;                    // Q, then P hi (chunks 0-1) and P lo (chunks 2-3)
  uint8_t* ks = sm + TA_Q_BYTES;
  uint8_t* vs = ks + TA_KV_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(vs + TA_KV_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const AttnItem it = g.items[blockIdx.x];
  const int kvh = blockIdx.y;
  const int tok_per_tile = kAttnTileRows / g.hpg;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NBARS; ++i) mbar_init(&bars[i], i == BAR_P ? 4 : 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&tkv);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TA_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t qbytes = 4u * 64u * 2u * static_cast<uint32_t>(g.hpg * tok_per_tile);
      mbar_arrive_expect_tx(&bars[BAR_Q], qbytes);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tma_load_4d(qs + c * TA_CHUNK, &tq, &bars[BAR_Q], c * 64, 0, kvh, it.tok0);
      mbar_arrive_expect_tx(&bars[BAR_K], TA_KV_BYTES);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tma_load_2d(ks + c * TA_CHUNK, &tkv, &bars[BAR_K], kvh * TA_HD + c * 64, it.key0);
      mbar_arrive_expect_tx(&bars[BAR_V], TA_KV_BYTES);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tma_load_2d(vs + c * TA_CHUNK, &tkv, &bars[BAR_V], (g.kv_heads + kvh) * TA_HD + c * 64,
                    it.key0);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(&bars[BAR_Q], 0, abort_flag, g.status) &&
                mbar_wait(&bars[BAR_K], 0, abort_flag, g.status);
      if (ok) {
        tc_fence_after();
        constexpr uint32_t idesc_s = idesc_f16_f32(128, 128);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint64_t da = sw128_desc(qs + c * TA_CHUNK);
          const uint64_t db = sw128_desc(ks + c * TA_CHUNK);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem, da + 2 * k, db + 2 * k, idesc_s, (c | k) ? 1u : 0u);
        }
        umma_commit(&bars[BAR_S]);
        ok = mbar_wait(&bars[BAR_P], 0, abort_flag, g.status) &&
             mbar_wait(&bars[BAR_V], 0, abort_flag, g.status);
      }
      if (ok) {
        tc_fence_after();
        constexpr uint32_t idesc_o = idesc_f16_f32_bmn(128, 256);
        // K = 128 keys in 8 steps of 16; P chunk kk / 4 holds keys 64 (kk / 4) ..
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t da = sw128_desc(qs + (kk >> 2) * TA_CHUNK) + 2 * (kk & 3);
          const uint64_t db = sw128_mn_desc(vs + kk * 2048, TA_CHUNK);
          umma_f16(tmem, da, db, idesc_o, kk ? 1u : 0u);
        }
        if constexpr (PLO) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t da = sw128_desc(qs + 2 * TA_CHUNK + (kk >> 2) * TA_CHUNK) + 2 * (kk & 3);
            const uint64_t db = sw128_mn_desc(vs + kk * 2048, TA_CHUNK);
            umma_f16(tmem, da, db, idesc_o, 1u);
          }
        }
        umma_commit(&bars[BAR_O]);
      }
    }
  } else {
    // One query row per thread: TMEM lane r.
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;
    const int tl = r / g.hpg;
    const bool valid = tl < it.ntok && tl < tok_per_tile;
    const int tok = it.tok0 + tl;
    // Visible key columns of this tile: [ca0, ca1) U [cb0, cb1).
    int ca0 = 0, ca1 = 0, cb0 = 0, cb1 = 0;
    if (valid) {
      const int4 v = g.vis[tok];
      const int qp = g.meta[g.base + tok].pos;
      int a0 = v.x, b0 = v.z;
      if (g.window > 0) {
        a0 = max(a0, v.x + qp - g.window + 1);
        b0 = max(b0, v.w - g.window);
      }
      ca0 = min(max(a0 - it.key0, 0), kAttnTileKeys);
      ca1 = min(max(v.y - it.key0, 0), kAttnTileKeys);
      cb0 = min(max(b0 - it.key0, 0), kAttnTileKeys);
      cb1 = min(max(v.w - it.key0, 0), kAttnTileKeys);
      if (ca1 < ca0) ca1 = ca0;
      if (cb1 < cb0) cb1 = cb0;
    }
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * q4) << 16);
    float row_max = -INFINITY, row_sum = 0.f;
    bool ok = warp_wait(&bars[BAR_S], 0, abort_flag, g.status, lane);
    if (ok) {
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tmem_ld32_nowait(trow + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
      tmem_ld_wait();
      const bool all_vis = (ca0 == 0 && ca1 == kAttnTileKeys) || (cb0 == 0 && cb1 == kAttnTileKeys);
      const bool none_vis = ca0 == ca1 && cb0 == cb1;
      if (none_vis) {
#pragma unroll
        for (int j = 0; j < 128; ++j) s[j] = 0.f;
      } else {
        if (!all_vis) {
#pragma unroll
          for (int j = 0; j < 128; ++j) {
            const bool vj = (j >= ca0 && j < ca1) || (j >= cb0 && j < cb1);
            if (!vj) s[j] = -INFINITY;
          }
        }
#pragma unroll
        for (int j = 0; j < 128; ++j) row_max = fmaxf(row_max, s[j]);
        const float mb = row_max * kLog2e;
#pragma unroll
        for (int j = 0; j < 128; ++j) {
          const float p = exp2f(fmaf(s[j], kLog2e, -mb));
          s[j] = p;
          row_sum += p;
        }
      }
      // P (hi, then lo = what hi missed) into the Q buffer, K-major with the
      // 128-byte swizzle: key chunk kc = keys 64 kc.., 16-byte piece pw.
#pragma unroll
      for (int pc = 0; pc < 16; ++pc) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = s[pc * 8 + 2 * e], y = s[pc * 8 + 2 * e + 1];
          const __half2 h = __floats2half2_rn(x, y);
          const float2 hf = __half22float2(h);
          hi[e] = *reinterpret_cast<const uint32_t*>(&h);
          lo[e] = pack_h2(x - hf.x, y - hf.y);
        }
        const int kc = pc >> 3, pw = pc & 7;
        const uint32_t off = kc * TA_CHUNK + r * 128 + ((pw ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(qs + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        if constexpr (PLO)
          *reinterpret_cast<uint4*>(qs + 2 * TA_CHUNK + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[BAR_P]);
      ok = warp_wait(&bars[BAR_O], 0, abort_flag, g.status, lane);
    }
    if (ok) {
      tc_fence_after();
      const bool direct = it.slot < 0;
      const int head = kvh * g.hpg + (r % g.hpg);
      __half* orow = g.out + (static_cast<size_t>(tok) * g.heads + head) * TA_HD;
      const size_t prow = (static_cast<size_t>(it.slot < 0 ? 0 : it.slot) * g.kv_heads + kvh) *
                              kAttnTileRows + r;
      float* porow = g.part_o + prow * TA_HD;
      if (valid && !direct) g.part_ml[prow] = make_float2(row_max, row_sum);
      const float inv = row_sum > 0.f ? 1.0f / row_sum : 0.f;
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t raw[32];
        tmem_ld32_nowait(trow + c * 32, raw);
        tmem_ld_wait();
        if (!valid) continue;
        if (direct) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 pk;
            pk.x = pack_h2(__uint_as_float(raw[j]) * inv, __uint_as_float(raw[j + 1]) * inv);
            pk.y = pack_h2(__uint_as_float(raw[j + 2]) * inv, __uint_as_float(raw[j + 3]) * inv);
            pk.z = pack_h2(__uint_as_float(raw[j + 4]) * inv, __uint_as_float(raw[j + 5]) * inv);
            pk.w = pack_h2(__uint_as_float(raw[j + 6]) * inv, __uint_as_float(raw[j + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + j) = pk;
          }
        } else if (row_sum > 0.f) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<uint4*>(porow + c * 32 + j) =
                make_uint4(raw[j], raw[j + 1], raw[j + 2], raw[j + 3]);
        }
      }
    }
  }
  griddep_launch();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TA_TMEM_COLS);
  }
}

// out[row] = sum_s w_s o_s / sum_s w_s l_s, w_s = exp(m_s - max m), over the
// run's partials in tile order; partials that saw none of the row's keys
// (l = 0) are skipped. 64 threads per query row, 4 dims each.
__global__ void __launch_bounds__(256) attention_tc_combine(AttnTcArgs g) {
  griddep_wait();
  const AttnRun rn = g.runs[blockIdx.x];
  const int kvh = blockIdx.y;
  const int nrows = rn.ntok * g.hpg;
  const int d = (threadIdx.x & 63) * 4;
  for (int r = blockIdx.z * 4 + (threadIdx.x >> 6); r < nrows; r += gridDim.z * 4) {
    float mx = -INFINITY;
    for (int s = 0; s < rn.nslots; ++s) {
      const float2 ml =
          g.part_ml[(static_cast<size_t>(rn.slot0 + s) * g.kv_heads + kvh) * kAttnTileRows + r];
      if (ml.y > 0.f) mx = fmaxf(mx, ml.x);
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float den = 0.f;
    for (int s = 0; s < rn.nslots; ++s) {
      const size_t pr = (static_cast<size_t>(rn.slot0 + s) * g.kv_heads + kvh) * kAttnTileRows + r;
      const float2 ml = g.part_ml[pr];
      if (!(ml.y > 0.f)) continue;
      const float w = exp2f((ml.x - mx) * kLog2e);
      const float4 v = *reinterpret_cast<const float4*>(g.part_o + pr * TA_HD + d);
      acc.x = fmaf(w, v.x, acc.x);
      acc.y = fmaf(w, v.y, acc.y);
      acc.z = fmaf(w, v.z, acc.z);
      acc.w = fmaf(w, v.w, acc.w);
      den = fmaf(w, ml.y, den);
    }
    const float inv = den > 0.f ? 1.0f / den : 0.f;
    const int tok = rn.tok0 + r / g.hpg;
    const int head = kvh * g.hpg + (r % g.hpg);
    __half* o = g.out + (static_cast<size_t>(tok) * g.heads + head) * TA_HD + d;
    uint2 pk;
    pk.x = pack_h2(acc.x * inv, acc.y * inv);
    pk.y = pack_h2(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(o) = pk;
  }
  griddep_launch();
}

}  // namespace

void attention_intervals(const TokMeta* m, int t, int base, std::vector<int4>* vis) {
  vis->resize(static_cast<size_t>(t));
  for (int i = 0; i < t; ++i) {
    const int row = base + i;
    if ((m[i].seq & 0xfff) == 0) {
      (*vis)[i] = make_int4(m[i].row_lo, row + 1, row + 1, row + 1);
      continue;
    }
    // The branch's first token: scan back while the sequence id holds (a
    // branch's tokens are contiguous and all in this pass). Its position
    // is the group's prefix length.
    int j = i;
    while (j > 0 && m[j - 1].seq == m[i].seq) --j;
    const int prefix_len = m[j].pos;
    (*vis)[i] = make_int4(m[i].row_lo, m[i].row_lo + prefix_len, base + j, row + 1);
  }
}

bool attention_check_intervals(const TokMeta* meta_all, int t, int base, const int4* vis,
                               int window) {
  for (int i = 0; i < t; ++i) {
    const TokMeta q = meta_all[base + i];
    const int4 v = vis[i];
    int a0 = v.x, b0 = v.z;
    if (window > 0) {
      a0 = std::max(a0, v.x + q.pos - window + 1);
      b0 = std::max(b0, v.w - window);
    }
    for (int k = 0; k < base + t; ++k) {
      const TokMeta kk = meta_all[k];
      const bool want = attn_visible(q.pos, q.seq, kk.pos, kk.seq, window);
      const bool got = (k >= a0 && k < v.y) || (k >= b0 && k < v.w);
      if (want != got) return false;
    }
  }
  return true;
}

int attention_items(const TokMeta* m, const int4* vis, int t, int base, int hpg, int window,
                    std::vector<AttnItem>* items, std::vector<AttnRun>* runs) {
  items->clear();
  runs->clear();
  const int tok_per_tile = kAttnTileRows / hpg;
  int slots = 0;
  for (int i = 0; i < t;) {
    int n = 1;
    while (i + n < t && n < tok_per_tile && m[i + n].row_lo == m[i].row_lo) ++n;
    const int row_lo = m[i].row_lo;
    // Tiles on the grid anchored at row_lo that any token of the run sees.
    int lo = INT_MAX, hi = INT_MIN;
    std::vector<int2> ivs;
    ivs.reserve(2 * n);
    for (int k = 0; k < n; ++k) {
      const int4 v = vis[i + k];
      int a0 = v.x, b0 = v.z;
      if (window > 0) {
        a0 = std::max(a0, v.x + m[i + k].pos - window + 1);
        b0 = std::max(b0, v.w - window);
      }
      if (a0 < v.y) ivs.push_back(make_int2(a0, v.y));
      if (b0 < v.w) ivs.push_back(make_int2(b0, v.w));
    }
    for (const int2& iv : ivs) {
      lo = std::min(lo, iv.x);
      hi = std::max(hi, iv.y);
    }
    const size_t first = items->size();
    if (lo < hi) {
      for (int j = (lo - row_lo) / kAttnTileKeys; row_lo + j * kAttnTileKeys < hi; ++j) {
        const int k0 = row_lo + j * kAttnTileKeys, k1 = k0 + kAttnTileKeys;
        bool any = false;
        for (const int2& iv : ivs) any |= iv.x < k1 && iv.y > k0;
        if (any) items->push_back(AttnItem{i, n, k0, -1});
      }
    }
    const int cnt = static_cast<int>(items->size() - first);
    if (cnt > 1) {
      runs->push_back(AttnRun{i, n, slots, cnt});
      for (int k = 0; k < cnt; ++k) (*items)[first + k].slot = slots++;
    }
    i += n;
  }
  (void)base;
  return slots;
}

bool attention_tc_map_q(CUtensorMap* mp, const void* q16, int t_cap, int heads, int kv_heads,
                        char* err, size_t errlen) {
  const int hpg = heads / kv_heads;
  if (hpg < 1 || hpg > kAttnTileRows || heads % kv_heads != 0) {
    snprintf(err, errlen, "attention: %d query heads over %d KV heads", heads, kv_heads);
    return false;
  }
  const uint64_t dims[4] = {static_cast<uint64_t>(TA_HD), static_cast<uint64_t>(hpg),
                            static_cast<uint64_t>(kv_heads), static_cast<uint64_t>(t_cap)};
  const uint64_t strides[3] = {TA_HD * 2ull, static_cast<uint64_t>(hpg) * TA_HD * 2,
                               static_cast<uint64_t>(heads) * TA_HD * 2};
  const uint32_t box[4] = {64, static_cast<uint32_t>(hpg), 1,
                           static_cast<uint32_t>(kAttnTileRows / hpg)};
  return make_tmap_f16(mp, q16, 4, dims, strides, box, err, errlen);
}

bool attention_tc_map_kv(CUtensorMap* mp, const void* kv, int rows_cap, int kv_heads, char* err,
                         size_t errlen) {
  const uint64_t dims[2] = {static_cast<uint64_t>(2 * kv_heads * TA_HD),
                            static_cast<uint64_t>(rows_cap)};
  const uint64_t strides[1] = {static_cast<uint64_t>(2 * kv_heads * TA_HD) * 2};
  const uint32_t box[2] = {64, static_cast<uint32_t>(kAttnTileKeys)};
  return make_tmap_f16(mp, kv, 2, dims, strides, box, err, errlen);
}

void attention_tc_setup_device() {
  cudaFuncSetAttribute(attention_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       TA_SMEM);
  cudaFuncSetAttribute(attention_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       TA_SMEM);
}

int launch_attention_tc(const CUtensorMap& tq, const CUtensorMap& tkv, const AttnTcArgs& a,
                        cudaStream_t s) {
  if (a.n_items <= 0) return 0;
  dim3 grid(a.n_items, a.kv_heads);
  attention_tc_kernel<true><<<grid, 192, TA_SMEM, s>>>(tq, tkv, a);
  if (a.n_runs <= 0) return 1;
  dim3 g2(a.n_runs, a.kv_heads, 8);
  attention_tc_combine<<<g2, 256, 0, s>>>(a);
  return 2;
}

}  // namespace omg
