// Block-causal GQA attention on the 5th-generation tensor cores, head_dim
// 256 and 512 (see attention.cuh). Replaces
// crates/omg-wgpu/src/shaders/attention.wgsl for the decoder's layers.
//
// One CTA = one run (up to 128 query rows: a run's tokens x the query heads of
// one KV head) against every 64-key tile any of its rows sees, with an online
// softmax; the output accumulates in tensor memory.
//
//   warp 0     TMA: Q (4 x [128 rows][64 dims]) once; K and V tiles
//              (4 x [64 keys][64 dims] each) into two alternating buffers
//   warp 1     MMA: S_j = Q K_j^T (M 128, N 64, K 256) into one of two TMEM
//              score buffers, issued one tile ahead; O += P_j V_j (M 128,
//              N 256, K 64 keys, V read MN-major as stored)
//   warps 2-5  one query row per thread (its TMEM lane): mask, tile max,
//              exp, row sum, P as f16 into shared memory; rescale O in TMEM
//              when the row's reference max moves; finally out = O / l.
//
// Numerics follow attention.wgsl: Q, K, V f16; scores, max, exp and the row
// sum f32. A row keeps a reference max m and only moves it (rescaling O and
// l) when a tile's max exceeds it by more than kTau, so P = exp(s - m) stays
// below e^kTau (well inside f16) and most tiles need no rescale; the ratio
// O / l is the same softmax. Keys no row of the tile sees contribute exact
// zeros, so a row's result depends only on its own visible keys and the
// key grid anchored at its group's first row: a group's rows are the same
// bits wherever it sits in the pass, and whether its prefix is resident.
//
// head_dim 512 (Gemma 4's global layers): a 128 x 512 f32 O would fill all
// 512 TMEM columns, so two CTAs (grid.z) share a run, each accumulating the
// O of one 256-dim half of V; both compute the whole S = Q K^T (K = 512)
// and so the same softmax, bit for bit. Q (8 x [128 rows][64 dims], 128 KB)
// stays resident; K streams through a ring of four [64 keys][64 dims]
// chunks, the S MMAs of a tile consuming them as they land; the V half is
// one buffer of 4 chunks.
#include <algorithm>
#include <climits>
#include <cstdio>

#include "attention.cuh"
#include "gemm.cuh"
#include "launch.cuh"
#include "ptx.cuh"

namespace omg {

namespace {

constexpr int FA_HD = 256;                              // dims of O per CTA
constexpr int FA_KEYS = kAttnTileKeys;                  // 64 keys per tile
constexpr int FA_QCH = 128 * 128;                       // [128 rows][128 bytes]
constexpr int FA_KVCH = FA_KEYS * 128;                  // [64 keys][128 bytes]
constexpr int FA_Q_BYTES = 4 * FA_QCH;                  // 128 rows x 256 dims
constexpr int FA_KV_BYTES = 4 * FA_KVCH;                // 64 keys x 256 dims
constexpr int FA_P_BYTES = 128 * FA_KEYS * 2;           // [128 rows][64 keys] f16
constexpr uint32_t FA_TMEM_COLS = 512;
constexpr uint32_t FA_TMEM_O = 256;                     // O [128 x 256]; S buffers at 0, 64
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kTau = 8.0f;                            // reference-max slack (natural log)

// P slots: two with f16 P, so the softmax of tile j + 1 writes its P while
// P_j V_j still runs; one (hi, then lo) with PLO.
template <bool PLO>
constexpr int fa_p_slots() {
  return PLO ? 1 : 2;
}
template <bool PLO>
constexpr int fa_p_slot_bytes() {
  return (PLO ? 2 : 1) * FA_P_BYTES;
}
// head_dim 512: the K ring's chunks.
constexpr int FA_KRING = 4;
// Q, then K/V: head_dim 256 two K and two V tiles; 512 the K ring and one V
// half.
template <int HD>
constexpr int fa_q_bytes() {
  return (HD / 64) * FA_QCH;
}
template <int HD>
constexpr int fa_kv_area() {
  return HD == 256 ? 4 * FA_KV_BYTES : FA_KRING * FA_KVCH + FA_KV_BYTES;
}
template <int HD, bool PLO>
constexpr int fa_smem() {
  return 1024 + fa_q_bytes<HD>() + fa_kv_area<HD>() + fa_p_slots<PLO>() * fa_p_slot_bytes<PLO>() +
         256;
}
static_assert(fa_smem<256, false>() <= 227 * 1024 && fa_smem<256, true>() <= 227 * 1024 &&
                  fa_smem<512, false>() <= 227 * 1024 && fa_smem<512, true>() <= 227 * 1024,
              "attention shared memory above the per-CTA limit");

// B_P*: P of the slot written (4 softmax warps arrive); B_O*: the P.V of the
// tiles of that parity done. head_dim 512: B_R* / B_E* the K ring's chunks
// landed / consumed, B_V0 / B_VF0 the one V buffer.
enum {
  B_Q = 0, B_K0, B_K1, B_V0, B_V1, B_S0, B_S1, B_P0, B_P1, B_O0, B_O1, B_KF0, B_KF1, B_VF0,
  B_VF1, B_R0, B_R1, B_R2, B_R3, B_E0, B_E1, B_E2, B_E3, B_N
};
static_assert(B_R0 + FA_KRING == B_E0 && B_E0 + FA_KRING == B_N, "K ring barriers");

// Bits [a, b) of a 64-bit set, 0 <= a <= b <= 64.
__device__ __forceinline__ uint64_t key_bits(int a, int b) {
  const uint64_t below_b = b >= 64 ? ~0ull : (1ull << b) - 1;
  const uint64_t below_a = a >= 64 ? ~0ull : (1ull << a) - 1;
  return below_b & ~below_a;
}

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32; relative error
// about 2^-22; -inf gives +0 without a special-value path).
__device__ __forceinline__ float fa_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint32_t* status, int lane) {
  int ok = 0;
  if (lane == 0) ok = mbar_wait(bar, parity, abort_flag, status) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <int HD, bool PLO>
__global__ void __launch_bounds__(192, 1)
    attention_flash_kernel(const __grid_constant__ CUtensorMap tq,
                           const __grid_constant__ CUtensorMap tkv, AttnFlashArgs g) {
  static_assert(HD == 256 || HD == 512, "head_dim 256 or 512");
  constexpr int QB = fa_q_bytes<HD>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* qs = sm;
  auto ks = [&](int b) { return qs + QB + b * FA_KV_BYTES; };  // K buffer b (head_dim 256)
  // V buffer b (head_dim 512: the one buffer after the K ring).
  auto vs = [&](int b) {
    return HD == 256 ? qs + QB + (2 + b) * FA_KV_BYTES : qs + QB + FA_KRING * FA_KVCH;
  };
  auto kr = [&](int c) { return qs + QB + c * FA_KVCH; };  // K ring chunk c (head_dim 512)
  uint8_t* ps = qs + QB + fa_kv_area<HD>();  // P hi, then (PLO) P lo
  constexpr int NPS = fa_p_slots<PLO>(), PSB = fa_p_slot_bytes<PLO>();
  uint64_t* bars = reinterpret_cast<uint64_t*>(ps + NPS * PSB);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_N);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const AttnFlashItem item = g.items[blockIdx.x];
  const AttnFlashRun run = g.runs[item.run];
  const int kvh = blockIdx.y;
  const int vhalf = HD == 512 ? static_cast<int>(blockIdx.z) : 0;  // this CTA's 256 dims of V
  const int tok_per_tile = kAttnTileRows / g.hpg;
  const int* tiles = g.tiles + run.tile0 + item.t0;
  const int nt = item.nt;

  if (threadIdx.x == 0) {
    for (int i = 0; i < B_N; ++i) mbar_init(&bars[i], (i == B_P0 || i == B_P1) ? 4 : 1);
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&tkv);
  }
  if (warp == 1) tmem_alloc(tmem_slot, FA_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch();  // one CTA per (item, KV head)

  if (warp == 0) {
    if (lane == 0) {
      constexpr int QC = HD / 64;
      const uint32_t qbytes = QC * 64u * 2u * static_cast<uint32_t>(g.hpg * tok_per_tile);
      mbar_arrive_expect_tx(&bars[B_Q], qbytes);
#pragma unroll
      for (int c = 0; c < QC; ++c)
        tma_load_4d(qs + c * FA_QCH, &tq, &bars[B_Q], c * 64, 0, kvh, run.tok0);
      if constexpr (HD == 512) {
        // K of each tile in 8 ring chunks; then its V half, once P_{j-1} V_{j-1}
        // freed the buffer.
        int it = 0;
        bool ok = true;
        for (int j = 0; j < nt && ok; ++j) {
          for (int c = 0; c < 8 && ok; ++c, ++it) {
            const int s = it % FA_KRING, n = it / FA_KRING;
            if (n > 0 && !mbar_wait(&bars[B_E0 + s], (n - 1) & 1, abort_flag, g.status)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars[B_R0 + s], FA_KVCH);
            tma_load_2d(kr(s), &tkv, &bars[B_R0 + s], kvh * HD + c * 64, tiles[j]);
          }
          if (!ok) break;
          if (j > 0 && !mbar_wait(&bars[B_VF0], (j - 1) & 1, abort_flag, g.status)) break;
          mbar_arrive_expect_tx(&bars[B_V0], FA_KV_BYTES);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            tma_load_2d(vs(0) + c * FA_KVCH, &tkv, &bars[B_V0],
                        (g.kv_heads + kvh) * HD + vhalf * 256 + c * 64, tiles[j]);
        }
      }
      for (int j = 0; HD == 256 && j < nt; ++j) {
        const int b = j & 1, u = j >> 1;
        if (u > 0 && !mbar_wait(&bars[B_KF0 + b], (u - 1) & 1, abort_flag, g.status)) break;
        mbar_arrive_expect_tx(&bars[B_K0 + b], FA_KV_BYTES);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tma_load_2d(ks(b) + c * FA_KVCH, &tkv, &bars[B_K0 + b], kvh * FA_HD + c * 64, tiles[j]);
        if (u > 0 && !mbar_wait(&bars[B_VF0 + b], (u - 1) & 1, abort_flag, g.status)) break;
        mbar_arrive_expect_tx(&bars[B_V0 + b], FA_KV_BYTES);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tma_load_2d(vs(b) + c * FA_KVCH, &tkv, &bars[B_V0 + b],
                      (g.kv_heads + kvh) * FA_HD + c * 64, tiles[j]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(128, FA_KEYS);
      constexpr uint32_t idesc_o = idesc_f16_f32_bmn(128, FA_HD);
      int kit = 0;  // K ring chunks consumed (head_dim 512)
      // S_j = Q K_j^T into score buffer j & 1.
      auto issue_s = [&](int j) -> bool {
        const int b = j & 1;
        if constexpr (HD == 512) {
          for (int c = 0; c < 8; ++c, ++kit) {
            const int s = kit % FA_KRING;
            if (!mbar_wait(&bars[B_R0 + s], (kit / FA_KRING) & 1, abort_flag, g.status))
              return false;
            tc_fence_after();
            const uint64_t da = sw128_desc(qs + c * FA_QCH);
            const uint64_t db = sw128_desc(kr(s));
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16(tmem + b * FA_KEYS, da + 2 * k, db + 2 * k, idesc_s, (c | k) ? 1u : 0u);
            umma_commit(&bars[B_E0 + s]);
          }
          umma_commit(&bars[B_S0 + b]);
          return true;
        }
        if (!mbar_wait(&bars[B_K0 + b], (j >> 1) & 1, abort_flag, g.status)) return false;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint64_t da = sw128_desc(qs + c * FA_QCH);
          const uint64_t db = sw128_desc(ks(b) + c * FA_KVCH);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem + b * FA_KEYS, da + 2 * k, db + 2 * k, idesc_s, (c | k) ? 1u : 0u);
        }
        umma_commit(&bars[B_S0 + b]);
        umma_commit(&bars[B_KF0 + b]);
        return true;
      };
      bool ok = mbar_wait(&bars[B_Q], 0, abort_flag, g.status) && issue_s(0);
      for (int j = 0; ok && j < nt; ++j) {
        const int b = j & 1;
        // S_{j+1} one tile ahead, so the softmax of tile j + 1 overlaps
        // P_j V_j. Its score buffer held S_{j-1}, which the softmax warps
        // finished with before P_{j-1} (waited for last iteration).
        if (j + 1 < nt && !issue_s(j + 1)) break;
        // P_j sits in slot j & 1 (the only slot with PLO).
        const int slot = NPS == 2 ? b : 0;
        const uint32_t p_par = NPS == 2 ? (j >> 1) & 1 : j & 1;
        // V_j: buffer j & 1 (head_dim 256), the one buffer (512).
        const int vb_i = HD == 256 ? b : 0;
        const uint32_t v_par = HD == 256 ? (j >> 1) & 1 : j & 1;
        if (!mbar_wait(&bars[B_P0 + slot], p_par, abort_flag, g.status) ||
            !mbar_wait(&bars[B_V0 + vb_i], v_par, abort_flag, g.status))
          break;
        tc_fence_after();
        const uint8_t* pj = ps + slot * PSB;
#pragma unroll
        for (int kk = 0; kk < FA_KEYS / 16; ++kk) {
          const uint64_t pa = sw128_desc(pj) + 2 * kk;
          const uint64_t vb = sw128_mn_desc(vs(vb_i) + kk * 2048, FA_KVCH);
          umma_f16(tmem + FA_TMEM_O, pa, vb, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        if constexpr (PLO) {
#pragma unroll
          for (int kk = 0; kk < FA_KEYS / 16; ++kk) {
            const uint64_t pa = sw128_desc(pj + FA_P_BYTES) + 2 * kk;
            const uint64_t vb = sw128_mn_desc(vs(vb_i) + kk * 2048, FA_KVCH);
            umma_f16(tmem + FA_TMEM_O, pa, vb, idesc_o, 1u);
          }
        }
        umma_commit(&bars[B_O0 + b]);
        umma_commit(&bars[B_VF0 + vb_i]);
      }
    }
  } else {
    // One query row per thread: TMEM lane r.
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;
    const int tl = r / g.hpg;
    const bool valid = tl < run.ntok && tl < tok_per_tile;
    const int tok = run.tok0 + tl;
    // This row's visible cache rows: [a0, a1) U [b0, b1).
    int a0 = 0, a1 = 0, b0 = 0, b1 = 0;
    if (valid) {
      const int4 v = g.vis[tok];
      const int qp = g.meta[g.base + tok].pos;
      a0 = v.x;
      a1 = v.y;
      b0 = v.z;
      b1 = v.w;
      if (g.window > 0) {
        a0 = max(a0, v.x + qp - g.window + 1);
        b0 = max(b0, v.w - g.window);
      }
    }
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * q4) << 16);
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const int key0 = tiles[j];
      int ca0 = min(max(a0 - key0, 0), FA_KEYS), ca1 = min(max(a1 - key0, 0), FA_KEYS);
      int cb0 = min(max(b0 - key0, 0), FA_KEYS), cb1 = min(max(b1 - key0, 0), FA_KEYS);
      if (ca1 < ca0) ca1 = ca0;
      if (cb1 < cb0) cb1 = cb0;
      if (!warp_wait(&bars[B_S0 + (j & 1)], (j >> 1) & 1, abort_flag, g.status, lane)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[FA_KEYS];
      {
        uint32_t raw0[32], raw1[32];
        tmem_ld32_nowait(trow + (j & 1) * FA_KEYS, raw0);
        tmem_ld32_nowait(trow + (j & 1) * FA_KEYS + 32, raw1);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          s[c] = __uint_as_float(raw0[c]);
          s[32 + c] = __uint_as_float(raw1[c]);
        }
      }
      // Mask with the row's visible keys as a 64-bit set: one branch-free
      // path for rows that see all, some or none of the tile (per-row
      // branches made the warp run every path). Eight independent partial
      // maxima and sums keep the one warp per sub-partition issuing.
      {
        const uint64_t vis = key_bits(ca0, ca1) | key_bits(cb0, cb1);
        const uint32_t vlo = static_cast<uint32_t>(vis), vhi = static_cast<uint32_t>(vis >> 32);
#pragma unroll
        for (int c = 0; c < FA_KEYS; ++c) {
          const uint32_t w = c < 32 ? vlo : vhi;
          s[c] = ((w >> (c & 31)) & 1u) ? s[c] : -INFINITY;
        }
      }
      float mt;
      {
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = s[e];
#pragma unroll
        for (int c = 8; c < FA_KEYS; ++c) mx[c & 7] = fmaxf(mx[c & 7], s[c]);
        mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                   fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      }
      float alpha = 1.f;
      bool rescale = false;
      if (mt > m_ref + kTau) {
        // O holds earlier tiles only when the old reference was finite.
        rescale = m_ref != -INFINITY;
        alpha = rescale ? fa_exp2((m_ref - mt) * kLog2e) : 0.f;
        m_ref = mt;
      }
      float sum = 0.f;
      if (m_ref == -INFINITY) {
#pragma unroll
        for (int c = 0; c < FA_KEYS; ++c) s[c] = 0.f;
      } else {
        // exp2(-inf) = 0 for the masked keys.
        const float mb = m_ref * kLog2e;
        float psum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < FA_KEYS; ++c) {
          s[c] = fa_exp2(fmaf(s[c], kLog2e, -mb));
          psum[c & 7] += s[c];
        }
        sum = ((psum[0] + psum[1]) + (psum[2] + psum[3])) +
              ((psum[4] + psum[5]) + (psum[6] + psum[7]));
      }
      l = l * alpha + sum;
      // Rescaling O needs P_{j-1} V_{j-1} done; with one P slot, so does
      // writing P_j. (That barrier's next phase needs P_{j+1}: no parity
      // alias.)
      const bool any_rescale = __any_sync(0xffffffffu, rescale);
      if (j > 0 && (any_rescale || NPS == 1)) {
        if (!warp_wait(&bars[B_O0 + ((j - 1) & 1)], ((j - 1) >> 1) & 1, abort_flag, g.status,
                       lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // With two slots, slot j & 1 is free once P_{j-2} V_{j-2} is done.
      if (NPS == 2 && j >= 2) {
        if (!warp_wait(&bars[B_O0 + (j & 1)], ((j - 2) >> 1) & 1, abort_flag, g.status, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (any_rescale) {
        const float f = rescale ? alpha : 1.0f;
#pragma unroll 1
        for (int c = 0; c < FA_HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32_nowait(trow + FA_TMEM_O + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          tmem_st32(trow + FA_TMEM_O + c * 32, o);
        }
        tmem_st_wait();
      }
      // P (and, with PLO, what f16 missed of it) K-major with the 128-byte
      // swizzle: 16-byte piece pw holds keys 8 pw .. 8 pw + 7.
      const int slot = NPS == 2 ? (j & 1) : 0;
      uint8_t* pj = ps + slot * PSB;
#pragma unroll
      for (int pw = 0; pw < FA_KEYS / 8; ++pw) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = s[pw * 8 + 2 * e], y = s[pw * 8 + 2 * e + 1];
          const __half2 h = __floats2half2_rn(x, y);
          hi[e] = *reinterpret_cast<const uint32_t*>(&h);
          if constexpr (PLO) {
            const float2 hf = __half22float2(h);
            const __half2 d = __floats2half2_rn(x - hf.x, y - hf.y);
            lo[e] = *reinterpret_cast<const uint32_t*>(&d);
          }
        }
        const uint32_t off = r * 128 + ((pw ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(pj + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        if constexpr (PLO)
          *reinterpret_cast<uint4*>(pj + FA_P_BYTES + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_P0 + slot]);
    }
    const bool done =
        ok && warp_wait(&bars[B_O0 + ((nt - 1) & 1)], ((nt - 1) >> 1) & 1, abort_flag, g.status, lane);
    if (done && item.slot >= 0) {
      tc_fence_after();
      // One chunk of a split run: this row's reference max and sum, and its
      // unnormalised O (f32) in two 128-column halves, each staged in the Q
      // buffer like the f16 output below (512 bytes per row) and stored a
      // row per warp instruction.
      const size_t ps = static_cast<size_t>(item.slot) * g.kv_heads + kvh;
      if (vhalf == 0) g.part_ml[ps * kAttnTileRows + r] = make_float2(m_ref, l);
      float* po = g.part_o + ps * kAttnTileRows * HD + vhalf * FA_HD;
      uint8_t* stage = qs;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tmem_ld32(trow + FA_TMEM_O + (4 * half + c) * 32, o);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int piece = 8 * c + e;
            *reinterpret_cast<uint4*>(stage + r * 512 + ((piece ^ (r & 7)) << 4)) =
                make_uint4(__float_as_uint(o[4 * e]), __float_as_uint(o[4 * e + 1]),
                           __float_as_uint(o[4 * e + 2]), __float_as_uint(o[4 * e + 3]));
          }
        }
        __syncwarp();
        for (int i = 0; i < 32; ++i) {
          const int row = 32 * q4 + i;
          const uint4 v =
              *reinterpret_cast<const uint4*>(stage + row * 512 + ((lane ^ (row & 7)) << 4));
          *reinterpret_cast<uint4*>(po + static_cast<size_t>(row) * HD + 128 * half + 4 * lane) = v;
        }
        __syncwarp();
      }
    } else if (done) {
      tc_fence_after();
      // out = O / l as f16, staged in the Q buffer (every S MMA is done):
      // row r at r * 512 bytes, its 16-byte piece p at slot p ^ (r & 7), so
      // neither the writes (a row per lane) nor the reads (a row per warp)
      // conflict. Then each warp stores its 32 rows, 512 contiguous bytes
      // per instruction.
      uint8_t* stage = qs;
      const float inv = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < FA_HD / 32; ++c) {
        float o[32];
        tmem_ld32(trow + FA_TMEM_O + c * 32, o);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t w4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const __half2 h =
                __floats2half2_rn(o[8 * e + 2 * q] * inv, o[8 * e + 2 * q + 1] * inv);
            w4[q] = *reinterpret_cast<const uint32_t*>(&h);
          }
          const int piece = 4 * c + e;
          *reinterpret_cast<uint4*>(stage + r * 512 + ((piece ^ (r & 7)) << 4)) =
              make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
      __syncwarp();
      // Row 32 q4 + i is head hh of run token rt (counted along, no division
      // per row).
      int rt = (32 * q4) / g.hpg, hh = (32 * q4) % g.hpg;
      for (int i = 0; i < 32; ++i) {
        if (rt >= run.ntok || rt >= tok_per_tile) break;  // later rows are past the run too
        const int row = 32 * q4 + i;
        const uint4 v = *reinterpret_cast<const uint4*>(stage + row * 512 + ((lane ^ (row & 7)) << 4));
        __half* orow = g.out +
                       (static_cast<size_t>(run.tok0 + rt) * g.heads + kvh * g.hpg + hh) * HD +
                       vhalf * FA_HD;
        *reinterpret_cast<uint4*>(orow + lane * 8) = v;
        if (++hh == g.hpg) {
          hh = 0;
          ++rt;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, FA_TMEM_COLS);
  }
}

// A warp per query row of a split run (8 rows per CTA; grid.x = merges x 16
// row groups, grid.y = KV heads), lane l holding dims 8 l .. 8 l + 7. Lane c
// reads chunk c's (max, sum); the chunk with the largest reference max
// weighs exactly 1 and a chunk the row sees nothing of contributes exact
// zeros, so a row whose keys all sit in one chunk gets the bits the unsplit
// path writes, whatever else shares its run. Chunks are added in order, four
// at a time with all their loads issued first.
constexpr int kMergeRows = 8;

template <int HD>
__global__ void __launch_bounds__(32 * kMergeRows) attention_merge_kernel(AttnFlashArgs g) {
  griddep_wait();
  constexpr int groups = kAttnTileRows / kMergeRows;
  const AttnFlashMerge mg = g.merges[blockIdx.x / groups];
  const AttnFlashRun run = g.runs[mg.run];
  const int kvh = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int r = (blockIdx.x % groups) * kMergeRows + (threadIdx.x >> 5);
  const int tok_per_tile = kAttnTileRows / g.hpg;
  if (r < min(run.ntok, tok_per_tile) * g.hpg) {
    const size_t kvs = static_cast<size_t>(g.kv_heads);
    auto slot_row = [&](int c) {
      return ((static_cast<size_t>(mg.slot0 + c)) * kvs + kvh) * kAttnTileRows + r;
    };
    // The row's overall reference max (chunks beyond 32 folded per lane).
    float mmax = -INFINITY;
    for (int c = lane; c < mg.nchunks; c += 32) mmax = fmaxf(mmax, g.part_ml[slot_row(c)].x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, o));
    // head_dim 512: the two 256-dim halves one after the other (the same
    // chunk weights and sum).
#pragma unroll 1
    for (int dh = 0; dh < HD / FA_HD; ++dh) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float lsum = 0.f;
    for (int c0 = 0; c0 < mg.nchunks; c0 += 4) {
      float4 a[4], b[4];
      float2 ml[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (c0 + k < mg.nchunks) {
          const size_t sr = slot_row(c0 + k);
          ml[k] = g.part_ml[sr];
          const float4* src =
              reinterpret_cast<const float4*>(g.part_o + sr * HD + dh * FA_HD + 8 * lane);
          a[k] = src[0];
          b[k] = src[1];
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (c0 + k >= mg.nchunks) break;
        // exp2(-inf) = +0 for a chunk the row sees nothing of.
        const float w = ml[k].x == mmax ? 1.0f : fa_exp2((ml[k].x - mmax) * kLog2e);
        acc[0] = fmaf(w, a[k].x, acc[0]);
        acc[1] = fmaf(w, a[k].y, acc[1]);
        acc[2] = fmaf(w, a[k].z, acc[2]);
        acc[3] = fmaf(w, a[k].w, acc[3]);
        acc[4] = fmaf(w, b[k].x, acc[4]);
        acc[5] = fmaf(w, b[k].y, acc[5]);
        acc[6] = fmaf(w, b[k].z, acc[6]);
        acc[7] = fmaf(w, b[k].w, acc[7]);
        lsum = fmaf(w, ml[k].y, lsum);
      }
    }
    const float inv = lsum > 0.f ? 1.0f / lsum : 0.f;
    const int tl = r / g.hpg, hh = r - tl * g.hpg;
    __half* orow = g.out +
                   (static_cast<size_t>(run.tok0 + tl) * g.heads + kvh * g.hpg + hh) * HD +
                   dh * FA_HD + 8 * lane;
    uint32_t w4[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __half2 h = __floats2half2_rn(acc[2 * q] * inv, acc[2 * q + 1] * inv);
      w4[q] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(orow) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
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

int attention_flash_runs(const TokMeta* m, const int4* vis, int t, int hpg, int window,
                         std::vector<AttnFlashRun>* runs, std::vector<int>* tiles,
                         std::vector<AttnFlashItem>* items, std::vector<AttnFlashMerge>* merges) {
  runs->clear();
  tiles->clear();
  items->clear();
  merges->clear();
  int slots = 0;
  const int tok_per_tile = kAttnTileRows / hpg;
  std::vector<int2> ivs;
  for (int i = 0; i < t;) {
    int n = 1;
    while (i + n < t && n < tok_per_tile && m[i + n].row_lo == m[i].row_lo) ++n;
    const int row_lo = m[i].row_lo;
    ivs.clear();
    int lo = INT_MAX, hi = INT_MIN;
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
    const int first = static_cast<int>(tiles->size());
    if (lo < hi) {
      // 64-key tiles on the grid anchored at the group's first row; tiles no
      // row of the run sees are skipped.
      for (int j = (lo - row_lo) / kAttnTileKeys; row_lo + j * kAttnTileKeys < hi; ++j) {
        const int k0 = row_lo + j * kAttnTileKeys, k1 = k0 + kAttnTileKeys;
        bool any = false;
        for (const int2& iv : ivs) any |= iv.x < k1 && iv.y > k0;
        if (any) tiles->push_back(k0);
      }
    }
    const int nt = static_cast<int>(tiles->size()) - first;
    const int ri = static_cast<int>(runs->size());
    runs->push_back(AttnFlashRun{i, n, first, nt});
    // Chunks: grid tile index (from row_lo) / kAttnChunkTiles.
    auto chunk_of = [&](int j) { return ((*tiles)[first + j] - row_lo) / kAttnTileKeys / kAttnChunkTiles; };
    int nchunks = 0;
    for (int j = 0; j < nt; ++j)
      if (j == 0 || chunk_of(j) != chunk_of(j - 1)) ++nchunks;
    if (nchunks <= 1) {
      items->push_back(AttnFlashItem{ri, 0, nt, -1});
    } else {
      merges->push_back(AttnFlashMerge{ri, slots, nchunks});
      int c = 0;
      for (int j = 0; j < nt;) {
        int e = j + 1;
        while (e < nt && chunk_of(e) == chunk_of(j)) ++e;
        items->push_back(AttnFlashItem{ri, j, e - j, slots + c});
        ++c;
        j = e;
      }
      slots += nchunks;
    }
    i += n;
  }
  return slots;
}

bool attention_map_q(CUtensorMap* mp, const void* q16, int t_cap, int heads, int kv_heads, int hd,
                     char* err, size_t errlen) {
  const int hpg = heads / kv_heads;
  if (hpg < 1 || hpg > kAttnTileRows || heads % kv_heads != 0) {
    snprintf(err, errlen, "attention: %d query heads over %d KV heads", heads, kv_heads);
    return false;
  }
  if (hd != 256 && hd != 512) {
    snprintf(err, errlen, "attention: head_dim %d (256 or 512)", hd);
    return false;
  }
  const uint64_t dims[4] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(hpg),
                            static_cast<uint64_t>(kv_heads), static_cast<uint64_t>(t_cap)};
  const uint64_t strides[3] = {hd * 2ull, static_cast<uint64_t>(hpg) * hd * 2,
                               static_cast<uint64_t>(heads) * hd * 2};
  const uint32_t box[4] = {64, static_cast<uint32_t>(hpg), 1,
                           static_cast<uint32_t>(kAttnTileRows / hpg)};
  return make_tmap_f16(mp, q16, 4, dims, strides, box, err, errlen);
}

bool attention_map_kv(CUtensorMap* mp, const void* kv, int rows_cap, int kv_heads, int hd,
                      char* err, size_t errlen) {
  if (hd != 256 && hd != 512) {
    snprintf(err, errlen, "attention: head_dim %d (256 or 512)", hd);
    return false;
  }
  const uint64_t dims[2] = {static_cast<uint64_t>(2 * kv_heads * hd),
                            static_cast<uint64_t>(rows_cap)};
  const uint64_t strides[1] = {static_cast<uint64_t>(2 * kv_heads * hd) * 2};
  const uint32_t box[2] = {64, static_cast<uint32_t>(FA_KEYS)};
  return make_tmap_f16(mp, kv, 2, dims, strides, box, err, errlen);
}

void attention_setup_device() {
  cudaFuncSetAttribute(attention_flash_kernel<256, true>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, fa_smem<256, true>());
  cudaFuncSetAttribute(attention_flash_kernel<256, false>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, fa_smem<256, false>());
  cudaFuncSetAttribute(attention_flash_kernel<512, true>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, fa_smem<512, true>());
  cudaFuncSetAttribute(attention_flash_kernel<512, false>,
                       cudaFuncAttributeMaxDynamicSharedMemorySize, fa_smem<512, false>());
}

void launch_attention_flash(const CUtensorMap& tq, const CUtensorMap& tkv,
                            const AttnFlashArgs& a, bool p_lo, cudaStream_t s) {
  if (a.n_items <= 0) return;
  if (a.hd == 512) {
    dim3 grid(a.n_items, a.kv_heads, 2);  // z: the V half
    if (p_lo)
      launch_pdl(attention_flash_kernel<512, true>, grid, dim3(192), fa_smem<512, true>(), s, tq,
                 tkv, a);
    else
      launch_pdl(attention_flash_kernel<512, false>, grid, dim3(192), fa_smem<512, false>(), s, tq,
                 tkv, a);
    return;
  }
  dim3 grid(a.n_items, a.kv_heads);
  if (p_lo)
    launch_pdl(attention_flash_kernel<256, true>, grid, dim3(192), fa_smem<256, true>(), s, tq, tkv,
               a);
  else
    launch_pdl(attention_flash_kernel<256, false>, grid, dim3(192), fa_smem<256, false>(), s, tq,
               tkv, a);
}

void launch_attention_merge(const AttnFlashArgs& a, cudaStream_t s) {
  if (a.n_merges <= 0) return;
  const dim3 grid(a.n_merges * (kAttnTileRows / kMergeRows), a.kv_heads);
  if (a.hd == 512)
    launch_pdl(attention_merge_kernel<512>, grid, dim3(32 * kMergeRows), 0, s, a);
  else
    launch_pdl(attention_merge_kernel<256>, grid, dim3(32 * kMergeRows), 0, s, a);
}

}  // namespace omg
