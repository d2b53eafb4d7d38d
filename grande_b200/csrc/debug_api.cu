// Kernel-level entry points for the parity tests: each takes host buffers,
// runs one kernel on `device` and copies the result back. They allocate their
// own device memory per call; the engine never uses them.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <algorithm>
#include <cstring>
#include <vector>

#include "capi_util.h"
#include "attention.cuh"
#include "gemm.cuh"
#include "packed.cuh"
#include "omg_b200.h"

using namespace omg;

namespace {

struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  bool alloc(size_t n) { return cudaMalloc(&p, n ? n : 16) == cudaSuccess; }
};

}  // namespace

extern "C" int omg_debug_gemm(int device, const uint16_t* x_f16, int m, int k, int lda,
                              const uint16_t* w_f16, int w_rows, int n_out, int epi, int bn,
                              int splits, void* out, int ldo) {
  return guarded([&]() -> int {
    CUDA_TRY(cudaSetDevice(device));
    gemm_setup_device();
    if (bn == 0) {
      int sms = 148;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
      gemm_pick(n_out, k, sms, &bn, &splits);
    }
    DevBuf dx, dw, dout, dstat;
    const size_t xb = static_cast<size_t>(m) * lda * 2;
    const size_t wb = static_cast<size_t>(w_rows) * k * 2;
    const bool f32 = epi == kEpiF32;
    if (!dx.alloc(xb) || !dw.alloc(wb) || !dstat.alloc(4)) return set_error("cudaMalloc failed");
    CUDA_TRY(cudaMemcpy(dx.p, x_f16, xb, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(dw.p, w_f16, wb, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemset(dstat.p, 0, 4));
    GemmPlan plan;
    char err[256];
    // bn 512 asks for the CTA-pair kernel (256 x 256 tiles over two SMs).
    const bool pair = bn == 512;
    if (!gemm_plan(&plan, dx.p, m, lda, dw.p, w_rows, n_out, k, epi, pair ? 256 : bn, splits, err,
                   sizeof err))
      return set_error(err);
    if (pair && !gemm_plan_pair(&plan, dw.p, w_rows, true, err, sizeof err)) return set_error(err);
    const int sp = f32 ? plan.s.splits : 1;
    const size_t slab = static_cast<size_t>(m) * ldo;
    const size_t ob = slab * sp * (f32 ? 4 : 2);
    if (!dout.alloc(ob)) return set_error("cudaMalloc failed");
    CUDA_TRY(cudaMemset(dout.p, 0, ob));
    gemm_run(plan, m, dout.p, ldo, slab, static_cast<uint32_t*>(dstat.p), 0);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaDeviceSynchronize());
    uint32_t st = 0;
    CUDA_TRY(cudaMemcpy(&st, dstat.p, 4, cudaMemcpyDeviceToHost));
    if (st) return set_error("gemm kernel reported device status %u", st);
    if (f32 && sp > 1) {
      std::vector<float> h(slab * sp);
      CUDA_TRY(cudaMemcpy(h.data(), dout.p, ob, cudaMemcpyDeviceToHost));
      float* o = static_cast<float*>(out);
      for (size_t i = 0; i < slab; ++i) {
        float s = h[i];
        for (int z = 1; z < sp; ++z) s += h[z * slab + i];
        o[i] = s;
      }
    } else {
      CUDA_TRY(cudaMemcpy(out, dout.p, ob, cudaMemcpyDeviceToHost));
    }
    return 0;
  });
}

// The fused FFN launch on host buffers: act = gelu_tanh(X Wg^T) * (X Wu^T)
// (f16 [m, ff]) and Y = act Wd^T (f32 [m, d], the split-K slabs summed in
// order on the host). X [m, d] f16; W_up [2 ff, d] f16 with gate and up rows
// interleaved in 256-row blocks [128 gate | 128 up]; W_down [d, ff] f16.
// pair: 0 one-CTA tiles, 1 CTA pairs. Needs d % 128 == 0 and ff % d == 0
// (the down split's K blocks equal the up projection's).
extern "C" int omg_debug_mlp(int device, const uint16_t* x, int m, int d, const uint16_t* w_up,
                             int ff, const uint16_t* w_down, int pair, uint16_t* act_out,
                             float* y_out) {
  return guarded([&]() -> int {
    CUDA_TRY(cudaSetDevice(device));
    gemm_setup_device();
    if (m <= 0 || d <= 0 || ff <= 0 || d % 128 != 0 || ff % d != 0)
      return set_error("debug_mlp: needs d %% 128 == 0 and ff %% d == 0 (d %d, ff %d)", d, ff);
    const int splits = ff / d;
    DevBuf dx, dwu, dwd, dact, dslab, dready, dstat;
    const size_t xb = static_cast<size_t>(m) * d * 2, wub = static_cast<size_t>(2) * ff * d * 2;
    const size_t wdb = static_cast<size_t>(d) * ff * 2, actb = static_cast<size_t>(m) * ff * 2;
    const size_t slab = static_cast<size_t>(m) * d;
    const int m_tiles = (m + 127) / 128;
    if (!dx.alloc(xb) || !dwu.alloc(wub) || !dwd.alloc(wdb) || !dact.alloc(actb) ||
        !dslab.alloc(slab * splits * 4) || !dready.alloc(static_cast<size_t>(m_tiles) * splits * 4) ||
        !dstat.alloc(4))
      return set_error("cudaMalloc failed");
    CUDA_TRY(cudaMemcpy(dx.p, x, xb, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(dwu.p, w_up, wub, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(dwd.p, w_down, wdb, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemset(dready.p, 0, static_cast<size_t>(m_tiles) * splits * 4));
    CUDA_TRY(cudaMemset(dstat.p, 0, 4));
    GemmPlan up, down;
    char err[256];
    if (!gemm_plan(&up, dx.p, m, d, dwu.p, 2 * ff, ff, d, kEpiGeGluTanh, 256, 1, err, sizeof err) ||
        !gemm_plan(&down, dact.p, m, ff, dwd.p, d, d, ff, kEpiF32, 256, splits, err, sizeof err) ||
        !gemm_plan_pair(&up, dwu.p, 2 * ff, false, err, sizeof err) ||
        !gemm_plan_pair(&down, dwd.p, d, false, err, sizeof err))
      return set_error(err);
    if (!gemm_mlp_ok(up, down)) return set_error("debug_mlp: shapes not fusable");
    gemm_run_mlp(up, down, m, dact.p, ff, dslab.p, d, slab, static_cast<int*>(dready.p),
                 4 * up.s.n_tiles / down.s.splits, static_cast<uint32_t*>(dstat.p), 0, pair ? 1 : 0);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaDeviceSynchronize());
    uint32_t st = 0;
    CUDA_TRY(cudaMemcpy(&st, dstat.p, 4, cudaMemcpyDeviceToHost));
    if (st) return set_error("mlp kernel reported device status %u", st);
    CUDA_TRY(cudaMemcpy(act_out, dact.p, actb, cudaMemcpyDeviceToHost));
    std::vector<float> h(slab * splits);
    CUDA_TRY(cudaMemcpy(h.data(), dslab.p, h.size() * 4, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < slab; ++i) {
      float v = h[i];
      for (int z = 1; z < splits; ++z) v += h[z * slab + i];
      y_out[i] = v;
    }
    return 0;
  });
}

// Block-causal attention on host buffers: q [t, heads * hd] f16 (cache rows
// base..base+t), kv [rows, 2 * kv_heads * hd] f16, meta 4 ints per cache row
// (pos, seq, row_lo, row_hi), out [t, heads * hd] f16.
// iters > 0: time that many launches (and merges) with CUDA events after
// one untimed run; *ms gets the average.
static int debug_attention(int device, const uint16_t* q, const uint16_t* kv, const int32_t* meta,
                           int t, int base, int heads, int kv_heads, int hd, int window, int p_lo,
                           uint16_t* out, int iters, float* ms) {
  return guarded([&]() -> int {
    CUDA_TRY(cudaSetDevice(device));
    omg::attention_setup_device();
    const int rows = base + t;
    const int rows_pad = (rows + 63) / 64 * 64;
    DevBuf dq, dkv, dm, dout;
    const size_t qb = static_cast<size_t>(t) * heads * hd * 2;
    const size_t kvb = static_cast<size_t>(rows_pad) * 2 * kv_heads * hd * 2;
    if (!dq.alloc(qb) || !dkv.alloc(kvb) || !dm.alloc(static_cast<size_t>(rows_pad) * 16) ||
        !dout.alloc(qb))
      return set_error("cudaMalloc failed");
    CUDA_TRY(cudaMemset(dkv.p, 0, kvb));
    CUDA_TRY(cudaMemcpy(dq.p, q, qb, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(dkv.p, kv, static_cast<size_t>(rows) * 2 * kv_heads * hd * 2,
                        cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(dm.p, meta, static_cast<size_t>(rows) * 16, cudaMemcpyHostToDevice));
    const omg::TokMeta* hm = reinterpret_cast<const omg::TokMeta*>(meta);
    if (hd != 256 && hd != 512) return set_error("attention: head_dim %d (256 or 512)", hd);
    {
      // Tensor-core path: the engine's schedule, with the interval form of
      // the visibility rule checked against the rule itself on every pair.
      std::vector<int4> vis;
      omg::attention_intervals(hm + base, t, base, &vis);
      if (!omg::attention_check_intervals(hm, t, base, vis.data(), window))
        return set_error("attention: the packing's visibility is not two intervals per token");
      std::vector<omg::AttnFlashRun> runs;
      std::vector<int> tiles;
      std::vector<omg::AttnFlashItem> items;
      std::vector<omg::AttnFlashMerge> merges;
      const int slots = omg::attention_flash_runs(hm + base, vis.data(), t, heads / kv_heads, window,
                                                  &runs, &tiles, &items, &merges);
      DevBuf dv, dr, dti, dst, dit, dmg, dpo, dpml;
      const size_t prow = static_cast<size_t>(std::max(slots, 1)) * kv_heads * omg::kAttnTileRows;
      if (!dv.alloc(vis.size() * sizeof(int4)) ||
          !dr.alloc(runs.size() * sizeof(omg::AttnFlashRun)) ||
          !dti.alloc(std::max<size_t>(tiles.size(), 1) * sizeof(int)) || !dst.alloc(4) ||
          !dit.alloc(items.size() * sizeof(omg::AttnFlashItem)) ||
          !dmg.alloc(std::max<size_t>(merges.size(), 1) * sizeof(omg::AttnFlashMerge)) ||
          !dpo.alloc(prow * hd * sizeof(float)) || !dpml.alloc(prow * sizeof(float2)))
        return set_error("cudaMalloc failed");
      CUDA_TRY(cudaMemcpy(dit.p, items.data(), items.size() * sizeof(omg::AttnFlashItem),
                          cudaMemcpyHostToDevice));
      if (!merges.empty())
        CUDA_TRY(cudaMemcpy(dmg.p, merges.data(), merges.size() * sizeof(omg::AttnFlashMerge),
                            cudaMemcpyHostToDevice));
      CUDA_TRY(cudaMemcpy(dv.p, vis.data(), vis.size() * sizeof(int4), cudaMemcpyHostToDevice));
      CUDA_TRY(cudaMemcpy(dr.p, runs.data(), runs.size() * sizeof(omg::AttnFlashRun),
                          cudaMemcpyHostToDevice));
      CUDA_TRY(cudaMemcpy(dti.p, tiles.data(), tiles.size() * sizeof(int), cudaMemcpyHostToDevice));
      CUDA_TRY(cudaMemset(dst.p, 0, 4));
      CUtensorMap tq, tkv;
      char err[256];
      if (!omg::attention_map_q(&tq, dq.p, t, heads, kv_heads, hd, err, sizeof err) ||
          !omg::attention_map_kv(&tkv, dkv.p, rows_pad, kv_heads, hd, err, sizeof err))
        return set_error("%s", err);
      omg::AttnFlashArgs a{};
      a.vis = static_cast<const int4*>(dv.p);
      a.meta = static_cast<const omg::TokMeta*>(dm.p);
      a.runs = static_cast<const omg::AttnFlashRun*>(dr.p);
      a.tiles = static_cast<const int*>(dti.p);
      a.n_runs = static_cast<int>(runs.size());
      a.items = static_cast<const omg::AttnFlashItem*>(dit.p);
      a.n_items = static_cast<int>(items.size());
      a.merges = static_cast<const omg::AttnFlashMerge*>(dmg.p);
      a.n_merges = static_cast<int>(merges.size());
      a.part_o = static_cast<float*>(dpo.p);
      a.part_ml = static_cast<float2*>(dpml.p);
      a.out = static_cast<__half*>(dout.p);
      a.status = static_cast<uint32_t*>(dst.p);
      a.t = t;
      a.base = base;
      a.heads = heads;
      a.kv_heads = kv_heads;
      a.hpg = heads / kv_heads;
      a.window = window;
      a.hd = hd;
      auto once = [&]() {
        omg::launch_attention_flash(tq, tkv, a, p_lo != 0, 0);
        if (a.n_merges > 0) omg::launch_attention_merge(a, 0);
      };
      once();
      CUDA_TRY(cudaGetLastError());
      CUDA_TRY(cudaDeviceSynchronize());
      if (iters > 0) {
        cudaEvent_t e0, e1;
        CUDA_TRY(cudaEventCreate(&e0));
        CUDA_TRY(cudaEventCreate(&e1));
        CUDA_TRY(cudaEventRecord(e0, 0));
        for (int i = 0; i < iters; ++i) once();
        CUDA_TRY(cudaEventRecord(e1, 0));
        CUDA_TRY(cudaEventSynchronize(e1));
        float tms = 0.f;
        CUDA_TRY(cudaEventElapsedTime(&tms, e0, e1));
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        *ms = tms / iters;
      }
      uint32_t st = 0;
      CUDA_TRY(cudaMemcpy(&st, dst.p, 4, cudaMemcpyDeviceToHost));
      if (st) return set_error("attention kernel reported device status %u", st);
      if (out) CUDA_TRY(cudaMemcpy(out, dout.p, qb, cudaMemcpyDeviceToHost));
      return 0;
    }
  });
}

extern "C" int omg_debug_attention(int device, const uint16_t* q, const uint16_t* kv,
                                   const int32_t* meta, int t, int base, int heads, int kv_heads,
                                   int hd, int window, int p_lo, uint16_t* out) {
  return debug_attention(device, q, kv, meta, t, base, heads, kv_heads, hd, window, p_lo, out, 0,
                         nullptr);
}

extern "C" int omg_debug_attention_time(int device, const uint16_t* q, const uint16_t* kv,
                                        const int32_t* meta, int t, int base, int heads,
                                        int kv_heads, int hd, int window, int p_lo, int iters,
                                        float* ms) {
  if (iters <= 0 || !ms) return set_error("omg_debug_attention_time: iters > 0 and ms needed");
  return debug_attention(device, q, kv, meta, t, base, heads, kv_heads, hd, window, p_lo, nullptr,
                         iters, ms);
}

// Time `iters` launches of the GEMM on device-resident random operands
// (m x k activations, n x k weights, f16) with CUDA events; *ms gets the
// average per launch (bn 512: the CTA-pair kernel). For the kernel sweeps
// behind profiles/.
extern "C" int omg_debug_gemm_time(int device, int m, int n, int k, int epi, int bn, int splits,
                                   int iters, float* ms) {
  return guarded([&]() -> int {
    CUDA_TRY(cudaSetDevice(device));
    gemm_setup_device();
    if (bn == 0) {
      int sms = 148;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
      gemm_pick(n, k, sms, &bn, &splits);
    }
    const bool gated = epi == kEpiGeGluTanh || epi == kEpiGeGluErf;
    const int w_rows = gated ? (n + 127) / 128 * 256 : n;
    DevBuf dx, dw, dout, dstat;
    if (!dx.alloc(static_cast<size_t>(m) * k * 2) || !dw.alloc(static_cast<size_t>(w_rows) * k * 2) ||
        !dout.alloc(static_cast<size_t>(m) * n * 4 * std::max(splits, 1)) || !dstat.alloc(4))
      return set_error("cudaMalloc failed");
    CUDA_TRY(cudaMemset(dx.p, 0x3c, static_cast<size_t>(m) * k * 2));   // 1.0-ish halves
    CUDA_TRY(cudaMemset(dw.p, 0x20, static_cast<size_t>(w_rows) * k * 2));
    CUDA_TRY(cudaMemset(dstat.p, 0, 4));
    GemmPlan plan;
    char err[256];
    const bool pair = bn == 512;  // the CTA-pair kernel
    if (!gemm_plan(&plan, dx.p, m, k, dw.p, w_rows, n, k, epi, pair ? 256 : bn, splits, err,
                   sizeof err))
      return set_error(err);
    if (pair && !gemm_plan_pair(&plan, dw.p, w_rows, true, err, sizeof err)) return set_error(err);
    cudaEvent_t a, b;
    CUDA_TRY(cudaEventCreate(&a));
    CUDA_TRY(cudaEventCreate(&b));
    for (int i = 0; i < 3; ++i)
      gemm_run(plan, m, dout.p, n, static_cast<size_t>(m) * n, static_cast<uint32_t*>(dstat.p), 0);
    CUDA_TRY(cudaEventRecord(a, 0));
    for (int i = 0; i < iters; ++i)
      gemm_run(plan, m, dout.p, n, static_cast<size_t>(m) * n, static_cast<uint32_t*>(dstat.p), 0);
    CUDA_TRY(cudaEventRecord(b, 0));
    CUDA_TRY(cudaEventSynchronize(b));
    float t = 0;
    CUDA_TRY(cudaEventElapsedTime(&t, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    uint32_t st = 0;
    CUDA_TRY(cudaMemcpy(&st, dstat.p, 4, cudaMemcpyDeviceToHost));
    if (st) return set_error("gemm kernel reported device status %u", st);
    *ms = t / iters;
    return 0;
  });
}

extern "C" int omg_debug_dequant(int device, int dtype, const uint8_t* codes,
                                 const uint8_t* scales, int rows, int k, int mode, uint16_t* hi,
                                 uint16_t* lo) {
  return guarded([&]() -> int {
    if (rows <= 0 || k <= 0 || k % 32) fail("omg_debug_dequant: %d x %d is not whole blocks", rows, k);
    if (dtype < 0 || dtype > 2) fail("omg_debug_dequant: dtype %d", dtype);
    if (mode != 0 && mode != 1) fail("omg_debug_dequant: mode %d", mode);
    if (mode == 1 && !lo) fail("omg_debug_dequant: mode 1 writes lo too");
    CUDA_TRY(cudaSetDevice(device));
    const size_t n = static_cast<size_t>(rows) * k;
    const size_t cb = dtype == 0 ? n * 2 : (dtype == 1 ? n : n / 2);
    const size_t sb = dtype == 0 ? 0 : n / 32 * 2;
    DevBuf dc, ds, dh, dl;
    if (!dc.alloc(cb) || !ds.alloc(sb) || !dh.alloc(n * 2) || !dl.alloc(n * 2))
      return set_error("cudaMalloc failed");
    CUDA_TRY(cudaMemcpy(dc.p, codes, cb, cudaMemcpyHostToDevice));
    if (sb) CUDA_TRY(cudaMemcpy(ds.p, scales, sb, cudaMemcpyHostToDevice));
    if (mode == 0)
      launch_dequant_f16(dtype, dc.p, ds.p, rows, k, 0, static_cast<__half*>(dh.p), 0);
    else
      launch_table_hilo(dtype, dc.p, ds.p, n, static_cast<__half*>(dh.p),
                        static_cast<__half*>(dl.p), 0);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaMemcpy(hi, dh.p, n * 2, cudaMemcpyDeviceToHost));
    if (mode == 1) CUDA_TRY(cudaMemcpy(lo, dl.p, n * 2, cudaMemcpyDeviceToHost));
    return 0;
  });
}

namespace {

// A QTensor-layout weight [rows, k] (codes, f16 scales) packed on the device.
bool upload_packed(int dtype, const uint8_t* codes, const uint8_t* scales, int rows, int k,
                   DevBuf* out) {
  const size_t n = static_cast<size_t>(rows) * k;
  const size_t cb = dtype == kQ8 ? n : n / 2, sb = n / 32 * 2;
  DevBuf dc, ds;
  if (!dc.alloc(cb) || !ds.alloc(sb) || !out->alloc(packed_bytes(dtype, rows, k))) return false;
  if (cudaMemcpy(dc.p, codes, cb, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(ds.p, scales, sb, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(out->p, 0, packed_bytes(dtype, rows, k)) != cudaSuccess)
    return false;
  launch_pack_weight(dtype, dc.p, ds.p, rows, k, 0, rows, static_cast<uint8_t*>(out->p), 0);
  return cudaDeviceSynchronize() == cudaSuccess;
}

}  // namespace

extern "C" int omg_debug_gemm_q(int device, const uint16_t* x_f16, int m, int k, int lda,
                                int wdtype, const uint8_t* w_codes, const uint8_t* w_scales,
                                int w_rows, int n_out, int epi, int bn, int splits, void* out,
                                int ldo) {
  return guarded([&]() -> int {
    if (wdtype != kQ4 && wdtype != kQ8) fail("omg_debug_gemm_q: dtype %d is not Q4_0 / Q8_0", wdtype);
    if (k % 32) fail("omg_debug_gemm_q: K %d is not whole blocks", k);
    CUDA_TRY(cudaSetDevice(device));
    gemm_setup_device();
    if (bn == 0) {
      int sms = 148;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
      gemm_pick(n_out, k, sms, &bn, &splits);
    }
    DevBuf dx, dw, dout, dstat;
    const size_t xb = static_cast<size_t>(m) * lda * 2;
    const bool f32 = epi == kEpiF32;
    if (!dx.alloc(xb) || !dstat.alloc(4)) return set_error("cudaMalloc failed");
    if (!upload_packed(wdtype, w_codes, w_scales, w_rows, k, &dw))
      return set_error("packing the weight failed");
    CUDA_TRY(cudaMemcpy(dx.p, x_f16, xb, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemset(dstat.p, 0, 4));
    GemmPlan plan;
    char err[256];
    // bn 512 asks for the CTA-pair kernel (256 x 256 tiles over two SMs).
    const bool pair = bn == 512;
    if (!gemm_plan_packed(&plan, dx.p, m, lda, dw.p, wdtype, w_rows, n_out, k, epi,
                          pair ? 256 : bn, splits, err, sizeof err))
      return set_error(err);
    if (pair && !gemm_plan_pair(&plan, nullptr, w_rows, true, err, sizeof err)) return set_error(err);
    const int sp = f32 ? plan.s.splits : 1;
    const size_t slab = static_cast<size_t>(m) * ldo;
    const size_t ob = slab * sp * (f32 ? 4 : 2);
    if (!dout.alloc(ob)) return set_error("cudaMalloc failed");
    CUDA_TRY(cudaMemset(dout.p, 0, ob));
    gemm_run(plan, m, dout.p, ldo, slab, static_cast<uint32_t*>(dstat.p), 0);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaDeviceSynchronize());
    uint32_t st = 0;
    CUDA_TRY(cudaMemcpy(&st, dstat.p, 4, cudaMemcpyDeviceToHost));
    if (st) return set_error("gemm kernel reported device status %u", st);
    if (f32 && sp > 1) {
      std::vector<float> h(slab * sp);
      CUDA_TRY(cudaMemcpy(h.data(), dout.p, ob, cudaMemcpyDeviceToHost));
      float* o = static_cast<float*>(out);
      for (size_t i = 0; i < slab; ++i) {
        float s = h[i];
        for (int z = 1; z < sp; ++z) s += h[z * slab + i];
        o[i] = s;
      }
    } else {
      CUDA_TRY(cudaMemcpy(out, dout.p, ob, cudaMemcpyDeviceToHost));
    }
    return 0;
  });
}

extern "C" int omg_debug_mlp_q(int device, const uint16_t* x, int m, int d, int wdtype,
                               const uint8_t* up_codes, const uint8_t* up_scales, int ff,
                               const uint8_t* down_codes, const uint8_t* down_scales, int pair,
                               uint16_t* act_out, float* y_out) {
  return guarded([&]() -> int {
    if (wdtype != kQ4 && wdtype != kQ8) fail("omg_debug_mlp_q: dtype %d is not Q4_0 / Q8_0", wdtype);
    CUDA_TRY(cudaSetDevice(device));
    gemm_setup_device();
    if (m <= 0 || d <= 0 || ff <= 0 || d % 128 != 0 || ff % d != 0)
      return set_error("debug_mlp_q: needs d %% 128 == 0 and ff %% d == 0 (d %d, ff %d)", d, ff);
    const int splits = ff / d;
    DevBuf dx, dwu, dwd, dact, dslab, dready, dstat;
    const size_t xb = static_cast<size_t>(m) * d * 2, actb = static_cast<size_t>(m) * ff * 2;
    const size_t slab = static_cast<size_t>(m) * d;
    const int m_tiles = (m + 127) / 128;
    if (!dx.alloc(xb) || !dact.alloc(actb) || !dslab.alloc(slab * splits * 4) ||
        !dready.alloc(static_cast<size_t>(m_tiles) * splits * 4) || !dstat.alloc(4))
      return set_error("cudaMalloc failed");
    if (!upload_packed(wdtype, up_codes, up_scales, 2 * ff, d, &dwu) ||
        !upload_packed(wdtype, down_codes, down_scales, d, ff, &dwd))
      return set_error("packing the weights failed");
    CUDA_TRY(cudaMemcpy(dx.p, x, xb, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemset(dready.p, 0, static_cast<size_t>(m_tiles) * splits * 4));
    CUDA_TRY(cudaMemset(dstat.p, 0, 4));
    GemmPlan up, down;
    char err[256];
    if (!gemm_plan_packed(&up, dx.p, m, d, dwu.p, wdtype, 2 * ff, ff, d, kEpiGeGluTanh, 256, 1, err,
                          sizeof err) ||
        !gemm_plan_packed(&down, dact.p, m, ff, dwd.p, wdtype, d, d, ff, kEpiF32, 256, splits, err,
                          sizeof err) ||
        !gemm_plan_pair(&up, nullptr, 2 * ff, false, err, sizeof err) ||
        !gemm_plan_pair(&down, nullptr, d, false, err, sizeof err))
      return set_error(err);
    if (!gemm_mlp_ok(up, down)) return set_error("debug_mlp_q: shapes not fusable");
    gemm_run_mlp(up, down, m, dact.p, ff, dslab.p, d, slab, static_cast<int*>(dready.p),
                 4 * up.s.n_tiles / down.s.splits, static_cast<uint32_t*>(dstat.p), 0,
                 pair ? 1 : 0);
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaDeviceSynchronize());
    uint32_t st = 0;
    CUDA_TRY(cudaMemcpy(&st, dstat.p, 4, cudaMemcpyDeviceToHost));
    if (st) return set_error("mlp kernel reported device status %u", st);
    CUDA_TRY(cudaMemcpy(act_out, dact.p, actb, cudaMemcpyDeviceToHost));
    std::vector<float> h(slab * splits);
    CUDA_TRY(cudaMemcpy(h.data(), dslab.p, h.size() * 4, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < slab; ++i) {
      float v = h[i];
      for (int z = 1; z < splits; ++z) v += h[z * slab + i];
      y_out[i] = v;
    }
    return 0;
  });
}

extern "C" int omg_debug_gemm_time_q(int device, int m, int n, int k, int epi, int bn, int splits,
                                     int wdtype, int iters, float* ms) {
  return guarded([&]() -> int {
    if (wdtype != kQ4 && wdtype != kQ8) fail("omg_debug_gemm_time_q: dtype %d", wdtype);
    CUDA_TRY(cudaSetDevice(device));
    gemm_setup_device();
    if (bn == 0) {
      int sms = 148;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
      gemm_pick(n, k, sms, &bn, &splits);
    }
    const bool gated = epi == kEpiGeGluTanh || epi == kEpiGeGluErf;
    const int w_rows = gated ? (n + 127) / 128 * 256 : n;
    const size_t wb = packed_bytes(wdtype, w_rows, k);
    DevBuf dx, dw, dout, dstat;
    if (!dx.alloc(static_cast<size_t>(m) * k * 2) || !dw.alloc(wb) ||
        !dout.alloc(static_cast<size_t>(m) * n * 4 * std::max(splits, 1)) || !dstat.alloc(4))
      return set_error("cudaMalloc failed");
    CUDA_TRY(cudaMemset(dx.p, 0x3c, static_cast<size_t>(m) * k * 2));
    CUDA_TRY(cudaMemset(dw.p, 0x21, wb));
    CUDA_TRY(cudaMemset(dstat.p, 0, 4));
    GemmPlan plan;
    char err[256];
    const bool pair = bn == 512;
    if (!gemm_plan_packed(&plan, dx.p, m, k, dw.p, wdtype, w_rows, n, k, epi, pair ? 256 : bn,
                          splits, err, sizeof err))
      return set_error(err);
    if (pair && !gemm_plan_pair(&plan, nullptr, w_rows, true, err, sizeof err)) return set_error(err);
    cudaEvent_t a, b;
    CUDA_TRY(cudaEventCreate(&a));
    CUDA_TRY(cudaEventCreate(&b));
    for (int i = 0; i < 3; ++i)
      gemm_run(plan, m, dout.p, n, static_cast<size_t>(m) * n, static_cast<uint32_t*>(dstat.p), 0);
    CUDA_TRY(cudaEventRecord(a, 0));
    for (int i = 0; i < iters; ++i)
      gemm_run(plan, m, dout.p, n, static_cast<size_t>(m) * n, static_cast<uint32_t*>(dstat.p), 0);
    CUDA_TRY(cudaEventRecord(b, 0));
    CUDA_TRY(cudaEventSynchronize(b));
    float t = 0;
    CUDA_TRY(cudaEventElapsedTime(&t, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    uint32_t st = 0;
    CUDA_TRY(cudaMemcpy(&st, dstat.p, 4, cudaMemcpyDeviceToHost));
    if (st) return set_error("gemm kernel reported device status %u", st);
    *ms = t / iters;
    return 0;
  });
}

extern "C" int omg_debug_mlp_time(int device, int m, int d, int ff, int wdtype, int pair, int iters,
                                  float* ms) {
  return guarded([&]() -> int {
    CUDA_TRY(cudaSetDevice(device));
    gemm_setup_device();
    if (m <= 0 || d % 128 != 0 || ff % d != 0) fail("omg_debug_mlp_time: shapes");
    const int splits = ff / d;
    const bool pk = wdtype == kQ4 || wdtype == kQ8;
    const size_t wub = pk ? packed_bytes(wdtype, 2 * ff, d) : static_cast<size_t>(2) * ff * d * 2;
    const size_t wdb = pk ? packed_bytes(wdtype, d, ff) : static_cast<size_t>(d) * ff * 2;
    const size_t slab = static_cast<size_t>(m) * d;
    const int m_tiles = (m + 127) / 128;
    DevBuf dx, dwu, dwd, dact, dslab, dready, dstat;
    if (!dx.alloc(slab * 2) || !dwu.alloc(wub) || !dwd.alloc(wdb) ||
        !dact.alloc(static_cast<size_t>(m) * ff * 2) || !dslab.alloc(slab * splits * 4) ||
        !dready.alloc(static_cast<size_t>(m_tiles) * splits * 4) || !dstat.alloc(4))
      return set_error("cudaMalloc failed");
    CUDA_TRY(cudaMemset(dx.p, 0x3c, slab * 2));
    CUDA_TRY(cudaMemset(dwu.p, pk ? 0x21 : 0x20, wub));
    CUDA_TRY(cudaMemset(dwd.p, pk ? 0x21 : 0x20, wdb));
    CUDA_TRY(cudaMemset(dstat.p, 0, 4));
    GemmPlan up, down;
    char err[256];
    bool ok = pk ? gemm_plan_packed(&up, dx.p, m, d, dwu.p, wdtype, 2 * ff, ff, d, kEpiGeGluTanh,
                                    256, 1, err, sizeof err) &&
                       gemm_plan_packed(&down, dact.p, m, ff, dwd.p, wdtype, d, d, ff, kEpiF32,
                                        256, splits, err, sizeof err)
                 : gemm_plan(&up, dx.p, m, d, dwu.p, 2 * ff, ff, d, kEpiGeGluTanh, 256, 1, err,
                             sizeof err) &&
                       gemm_plan(&down, dact.p, m, ff, dwd.p, d, d, ff, kEpiF32, 256, splits, err,
                                 sizeof err);
    ok = ok && gemm_plan_pair(&up, pk ? nullptr : dwu.p, 2 * ff, false, err, sizeof err) &&
         gemm_plan_pair(&down, pk ? nullptr : dwd.p, d, false, err, sizeof err);
    if (!ok) return set_error(err);
    if (!gemm_mlp_ok(up, down)) return set_error("omg_debug_mlp_time: shapes not fusable");
    const int target_step = 4 * up.s.n_tiles / down.s.splits;
    cudaEvent_t a, b;
    CUDA_TRY(cudaEventCreate(&a));
    CUDA_TRY(cudaEventCreate(&b));
    auto once = [&]() {
      cudaMemsetAsync(dready.p, 0, static_cast<size_t>(m_tiles) * splits * 4, 0);
      gemm_run_mlp(up, down, m, dact.p, ff, dslab.p, d, slab, static_cast<int*>(dready.p),
                   target_step, static_cast<uint32_t*>(dstat.p), 0, pair ? 1 : 0);
    };
    for (int i = 0; i < 3; ++i) once();
    CUDA_TRY(cudaEventRecord(a, 0));
    for (int i = 0; i < iters; ++i) once();
    CUDA_TRY(cudaEventRecord(b, 0));
    CUDA_TRY(cudaEventSynchronize(b));
    float t = 0;
    CUDA_TRY(cudaEventElapsedTime(&t, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    uint32_t st = 0;
    CUDA_TRY(cudaMemcpy(&st, dstat.p, 4, cudaMemcpyDeviceToHost));
    if (st) return set_error("mlp kernel reported device status %u", st);
    *ms = t / iters;
    return 0;
  });
}
