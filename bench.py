#!/usr/bin/env python
"""Benchmark of the omg decision forward pass on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config e2b-q4|e2b-q4-resident|gemma3-270m-q8|e4b-q4|mmbert-q8]

Metric: questions/s on the E2B-shaped Q4_0 decoder, one
request = a 500-token state + 12 question branches of 24 tokens evaluated in
one block-causal pass with logits read at the 12 answer rows; p50 request
latency alongside. A step is one such request on each GPU (weak scaling: N
ranks, one engine per GPU, weights replicated, independent requests, no
collective on the data path). Rank 0 prints one JSON line.

* ``value``: device-resident passes (request uploaded once), timed with CUDA
  events on the engine's stream, max over ranks.
* ``e2e``: the same requests through the C ABI (``omg_engine_evaluate``)
  with host buffers: ids/metadata uploaded and logits read back every step,
  a fresh state each step (the resident prefix is evicted), CUDA events on
  the engine's stream around the K calls.
* ``roofline``: the largest kernel -- the fused FFN launch (gate+up with the
  GeGLU epilogue, then down) on the decoder, the erf-GeGLU Wi GEMM on the
  encoder -- from per-launch CUDA events, against MEASURED_PEAKS.json's burst
  tensor peak (the kernels are timed one launch at a time inside a pass of a
  few ms), with ``traffic`` from the committed ncu summary under profiles/.
* ``pass_roofline``: the whole pass's algorithmic FLOPs and bytes
  (``pass_work``) against the measured ms per pass; ``kernels``: the same per
  kernel class (projections and attention against the tensor peak, the
  lm_head and the residual norms against HBM).
* ``kv_broadcast`` (resident config, N > 1): one state's K/V handed from
  rank 0 to every rank with one NCCL broadcast (grande_b200/split.py).
* ``cpu_baseline`` / ``--impl reference``: the reference's CPU forward
  (tests/reference.rs), restated in oracle/, on all host cores: whole
  requests (every layer) on the same synthetic model, which oracle/ builds
  itself (the product library is not loaded on that arm).

``--config mmbert-q8`` measures BASELINE.json's encoder configuration instead
(not the headline metric): 256 sequences of 128 tokens through the Laya /
mmBERT-shaped encoder and its decision head, the [CLS] and [MASK] rows read
back, questions/s = sequences/s.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "questions/s/GPU E2B-shape Q4_0 (500-tok state, 12 branches); p50 latency"
UNIT = "questions/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def args_():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", default="e2b-q4")
    ap.add_argument("--profile-iters", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--weights", choices=["packed", "f16"], default="f16",
                    help="Q4_0/Q8_0 linears kept packed (decoded per tile) or as f16 rows")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (small cases for ncu captures only)")
    return ap.parse_args()


def metric_of(shape, resident: bool) -> str:
    """BASELINE.json's headline metric for its E2B configuration; the same
    measure, named for the shape, for the others."""
    if shape.name == "e2b-q4":
        return METRIC
    what = (f"resident {shape.state}-tok state, {shape.branches} branches" if resident else
            f"{shape.state}-tok state, {shape.branches} branches")
    return f"questions/s/GPU {shape.name} ({what}); p50 latency"


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# ---- distributed plumbing ---------------------------------------------------------

class Dist:
    def __init__(self, n: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", device_id=torch.device(f"cuda:{self.local}"),
                                    timeout=datetime.timedelta(seconds=300))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{self.local}")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---- clocks -------------------------------------------------------------------------

class Clocks:
    """nvidia-smi samples (200 ms) of this rank's GPU during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def gpu_index(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v for v in vis.split(",") if v.strip()]
        if local < len(ids) and ids[local].strip().isdigit():
            return int(ids[local])
    return local


# ---- CPU side: the reference's CPU forward (oracle/) -------------------------------

def oracle_model(shape, seed: int = 0):
    """The synthetic model of `shape` as the oracle takes it: the same draws,
    codes and scales as the GPU arm's model, generated, quantized and
    dequantized by oracle/ alone (the product library is not loaded)."""
    from oracle import oracle as O
    sliding = [t == "sliding_attention" for t in shape.config()["layer_types"]]
    L = shape.layers
    ocfg = O.OracleConfig(vocab=shape.vocab, d=shape.d, layers=L, heads=shape.heads,
                          kv_heads=shape.kv_heads, head_dim=[256] * L, ff=[shape.ff] * L,
                          sliding=sliding, kv_source=list(range(L)), rope_dims=[256] * L,
                          window=512, query_scale=256 ** -0.5 if shape.gemma3_numerics else 1.0,
                          norm_offset=0.0, v_norm=not shape.gemma3_numerics,
                          softcap=0.0 if shape.gemma3_numerics else 30.0)
    return ocfg, O.synth_tensors(ocfg.tensors(), seed, int(shape.dtype))


def oracle_request(ocfg, tensors, req, threads: int) -> float:
    """One request through the oracle (the reference's CPU forward,
    tests/reference.rs:175-349, with the lm_head and softcap at the answer
    rows, reference.rs:581-590): seconds of wall clock."""
    from oracle import oracle as O
    ids, pos, seq = O.pack(req.prefix, [(b.tokens, b.want) for b in req.branches])
    rows, at = [], len(req.prefix)
    for b in req.branches:
        rows += [at + w for w in b.want]
        at += len(b.tokens)
    t0 = time.perf_counter()
    hid = O.forward(ocfg, tensors, ids, pos, seq, O.ORACLE_EXACT, threads)
    for r in rows:
        O.logits(hid[r], tensors[0], ocfg.vocab, ocfg.d, ocfg.softcap)
    return time.perf_counter() - t0


def cpu_sample(shape, seed: int = 0) -> dict:
    """The GPU arm's CPU baseline: one whole request of `shape` (every layer,
    the lm_head at its answer rows) through the oracle on all host cores."""
    from grande_b200 import synth
    threads = os.cpu_count() or 1
    ocfg, tensors = oracle_model(shape, seed)
    s = oracle_request(ocfg, tensors, synth.request(shape, seed=1000), threads)
    return {"per_request_s": s, "threads": threads, "sampled_s": s}


# ---- algorithmic work of one pass ------------------------------------------------

def visible_pairs(prefix: int, branches: list, resident: bool, window: int) -> int:
    """(query, key) pairs one pass's attention visits on a layer: the prefix
    rows causally (when the prefix is decoded in this pass), each branch's
    rows over the prefix and the branch's own earlier rows, keys within
    `window` positions (0 = no window) -- the visibility rule of
    attention.wgsl:70-76."""
    import numpy as np
    w = window or (1 << 30)
    n = 0
    if not resident:
        i = np.arange(prefix)
        n += int(np.minimum(i + 1, w).sum())
    for bl in branches:
        j = np.arange(bl)
        qp = prefix + j
        lo = np.maximum(qp - w + 1, 0)
        n += int(np.maximum(prefix - lo, 0).sum() + np.minimum(j + 1, w).sum())
    return n


def pass_work(shape, req, resident: bool) -> dict:
    """FLOPs and bytes one pass needs at the least, per kernel class: 2
    FLOP per multiply-add of every linear over the pass's rows, 4 * head_dim
    per visible (query, key) pair and head for attention (QK^T and P.V),
    2 * rows * vocab * d for the lm_head; bytes = the packed weights read once
    (Q4_0 18 B / Q8_0 34 B per 32 weights), the packed embedding table once
    (the lm_head), and each layer's f16 K/V rows read once."""
    bpw = 18 / 32 if shape.dtype.name == "Q4" else 34 / 32
    d, ff, L, hd = shape.d, shape.ff, shape.layers, 256
    qkv_w = (shape.heads + 2 * shape.kv_heads) * hd
    t = (0 if resident else len(req.prefix)) + sum(len(b.tokens) for b in req.branches)
    rows = sum(len(b.want) for b in req.branches)
    blens = [len(b.tokens) for b in req.branches]
    P = len(req.prefix)
    kinds = ["sliding_attention" if (l + 1) % shape.global_every else "full_attention"
             for l in range(L)]
    pairs = {w: visible_pairs(P, blens, resident, w) for w in (0, 512)}
    attn = sum(4 * hd * shape.heads * pairs[512 if k == "sliding_attention" else 0]
               for k in kinds)
    kv_rows = sum(min(P, 512) + sum(blens) if k == "sliding_attention" else P + sum(blens)
                  for k in kinds)
    f = {"gemm_qkv": 2.0 * t * d * qkv_w * L,
         "gemm_o": 2.0 * t * shape.heads * hd * d * L,
         "gemm_mlp": 2.0 * t * d * 3 * ff * L,
         "attention": float(attn),
         "logits": 2.0 * rows * shape.vocab * d}
    w_bytes = (d * qkv_w + shape.heads * hd * d + 3 * ff * d) * L * bpw
    b = {"weights": w_bytes, "embed_table": shape.vocab * d * bpw,
         "kv": kv_rows * 2 * shape.kv_heads * hd * 2.0}
    return {"tokens": t, "rows": rows, "flop": f, "bytes": b,
            "flop_total": sum(f.values()), "bytes_total": sum(b.values()),
            "visible_pairs": pairs}


def workload_config(shape, resident: bool, n: int) -> dict:
    """The `config` of both arms' JSON lines for a decoder shape."""
    return {
        "workload": f"{shape.name}: {'resident ' if resident else ''}{shape.state}-token "
                    f"state + {shape.branches} branches x {shape.branch_len} tokens, one "
                    f"block-causal pass, logits at {shape.branches} answer rows; "
                    f"{shape.questions} questions per request, 1 request per GPU per step",
        "model": f"{shape.name} shape, random init ({shape.layers} layers, d {shape.d}, "
                 f"{shape.heads}q/{shape.kv_heads}kv heads x 256, ff {shape.ff}, "
                 f"vocab {shape.vocab}, {shape.dtype.name}_0)",
        "tokens_per_pass": (0 if resident else shape.state) + shape.branches * shape.branch_len,
        "parallelism": f"replicas x{n} (independent requests)",
        "l2": "inputs larger than L2: the f16 weights (3.6 GB at E2B) stream from HBM every "
              "pass",
    }


# ---- the B200 arm -----------------------------------------------------------------------

def run_b200(a, dist: Dist):
    from grande_b200 import synth
    from grande_b200.engine import Want
    shape = synth.CONFIGS[a.config]
    if a.layers:
        import dataclasses
        shape = dataclasses.replace(shape, layers=a.layers)
    resident = a.config.endswith("resident")
    cap = shape.tokens() + 64
    t_build = time.perf_counter()
    eng = synth.build_engine(shape, cap, shape.branches, device=dist.local, seed=0,
                             packed=a.weights == "packed")
    t_build = time.perf_counter() - t_build
    req = synth.request(shape, seed=1000 + dist.rank)
    if resident:
        # Make the 2,000-token state resident, then time branch-only passes.
        eng.evaluate(req.prefix, req.branches[:1], Want.LOGITS)
    q_per_step = shape.questions

    # Device-resident passes.
    eng.time_forward([req], Want.LOGITS, max(a.warmup, 3), resident=resident)
    dist.barrier()
    clocks = Clocks(gpu_index(dist.local))
    clocks.start()
    time.sleep(0.25)
    ms, launches = eng.time_forward([req], Want.LOGITS, a.steps, resident=resident)
    ms_max = dist.max(ms)
    dist.barrier()

    # End to end through the C ABI with host buffers.
    reqs = [synth.request(shape, seed=2000 + dist.rank * 100003 + i) for i in range(8)]
    if resident:
        for r in reqs:
            r.prefix = req.prefix
    width = shape.vocab
    for i in range(max(a.warmup, 3)):
        if not resident:
            eng.evict_resident()
        eng.evaluate(reqs[i % len(reqs)].prefix, reqs[i % len(reqs)].branches, Want.LOGITS)
    dist.barrier()
    lat = []
    eng.record_event(0)
    for i in range(a.steps):
        r = reqs[i % len(reqs)]
        if not resident:
            eng.evict_resident()
        t0 = time.perf_counter()
        eng.evaluate(r.prefix, r.branches, Want.LOGITS)
        lat.append((time.perf_counter() - t0) * 1e3)
    eng.record_event(1)
    e2e_ms = eng.elapsed_ms(0, 1)
    e2e_max = dist.max(e2e_ms)
    dist.barrier()
    clk = clocks.stop()

    kv_state = None
    if resident:
        # the resident state's f16 K/V (sliding layers
        # window-only) to host memory and back, wall clock per call (the call
        # returns after the copies complete), median of 5.
        saves, restores, nbytes = [], [], 0
        for _ in range(5):
            t0 = time.perf_counter()
            st = eng.save_state(req.prefix)
            saves.append((time.perf_counter() - t0) * 1e3)
            nbytes = st.byte_len()
            t0 = time.perf_counter()
            eng.restore_state(st)
            restores.append((time.perf_counter() - t0) * 1e3)
        sm, rm = statistics.median(saves), statistics.median(restores)
        kv_state = {"tokens": len(req.prefix), "bytes": nbytes, "save_ms": round(sm, 3),
                    "restore_ms": round(rm, 3), "save_gbs": round(nbytes / sm / 1e6, 2),
                    "restore_gbs": round(nbytes / rm / 1e6, 2)}
    prof = eng.profile_forward([req], Want.LOGITS, a.profile_iters, resident=resident)
    kv_bcast = bench_kv_broadcast(eng, synth.request(shape, seed=1000).prefix, dist) \
        if resident and dist.world > 1 else None
    work = pass_work(shape, req, resident)
    t_pass = work["tokens"]
    pk, pk_kind = peaks()
    # Kernels timed one launch at a time inside a pass of a few ms (well under
    # a second of load): the burst tensor peak is their ceiling.
    peak_tc = pk.get("bf16_tflops")
    peak_hbm = pk.get("hbm_gbs")
    n_pass = a.profile_iters
    kernels = {}
    for name, (launches_k, ms_k) in prof.items():
        e = {"launches_per_pass": launches_k // n_pass, "ms_per_pass": round(ms_k / n_pass, 4)}
        kernels[name] = e
    # The FLOP-bound kernels against the tensor peak, the lm_head against HBM.
    for name, key in (("gemm_qkv", "gemm_qkv"), ("gemm_o", "gemm_o"), ("gemm_mlp", "gemm_mlp")):
        if name in kernels:
            ms_k = kernels[name]["ms_per_pass"]
            ach = work["flop"][key] / (ms_k * 1e-3) / 1e12
            kernels[name].update(flop_per_pass=work["flop"][key], achieved_tflops=round(ach, 1),
                                 frac=round(ach / peak_tc, 4), bound="tensor")
    if "attention" in kernels:
        ms_k = kernels["attention"]["ms_per_pass"] + kernels.get(
            "attention_merge", {}).get("ms_per_pass", 0.0)
        ach = work["flop"]["attention"] / (ms_k * 1e-3) / 1e12
        kernels["attention"].update(flop_per_pass=work["flop"]["attention"],
                                    achieved_tflops_with_merge=round(ach, 1),
                                    frac=round(ach / peak_tc, 4), bound="tensor")
    if "logits" in kernels:
        ms_k = kernels["logits"]["ms_per_pass"]
        lb = work["bytes"]["embed_table"] + work["rows"] * shape.d * 4 + \
            work["rows"] * shape.vocab * 4
        ach = lb / (ms_k * 1e-3) / 1e9
        kernels["logits"].update(bytes_per_pass=lb, achieved_gbs=round(ach, 1),
                                 frac=round(ach / peak_hbm, 4), bound="hbm")
    if "residual_norm" in kernels:
        ms_k = kernels["residual_norm"]["ms_per_pass"]
        # Per launch: the f32 slabs (2 for the o and down projections), the
        # residual stream read and written, the next norm's f16 rows.
        rb = kernels["residual_norm"]["launches_per_pass"] * t_pass * shape.d * (2 * 4 + 8 + 2)
        ach = rb / (ms_k * 1e-3) / 1e9
        kernels["residual_norm"].update(bytes_per_pass=rb, achieved_gbs=round(ach, 1),
                                        frac=round(ach / peak_hbm, 4), bound="hbm")
    # The dominant kernel: the FFN (gate+up with the fused GeGLU, and down) as
    # one launch where the engine fuses them, else the gate+up GEMM alone.
    if "gemm_mlp" in prof:
        top_kernel = "gemm_mlp (tcgen05: gate+up with fused GeGLU, then down, one launch)"
        top_launches, top_ms = prof["gemm_mlp"]
        top_flops = 2.0 * t_pass * shape.d * 3 * shape.ff
        traffic = read_traffic("gemm_mlp", a.config)
    else:
        top_kernel = "gemm_gate_up (tcgen05, fused GeGLU)"
        top_launches, top_ms = prof["gemm_gate_up"]
        top_flops = 2.0 * t_pass * shape.d * 2 * shape.ff
        traffic = read_traffic("gemm_gate_up", a.config)
    top_avg = top_ms / top_launches
    achieved = top_flops / (top_avg * 1e-3) / 1e12
    n = dist.world
    value = n * q_per_step * a.steps / (ms_max * 1e-3)
    e2e_value = n * q_per_step * a.steps / (e2e_max * 1e-3)
    ms_step = ms_max / a.steps
    rl_tc = work["flop_total"] / (peak_tc * 1e12) * 1e3
    rl_hbm = work["bytes_total"] / (peak_hbm * 1e9) * 1e3
    bytes_in = t_pass * (4 + 16 + 4) + 8 * (t_pass // 4 + 1)
    out = {
        "metric": metric_of(shape, resident), "value": round(value, 2), "unit": UNIT, "n_gpus": n,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: seeded N(0,0.02) weights quantized to "
                f"{shape.dtype.name}_0, uniform token ids",
        "config": {**workload_config(shape, resident, n), "weights": a.weights},
        "p50_latency_ms": round(statistics.median(lat), 3) if lat else None,
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                "h2d_bytes_per_step": bytes_in, "d2h_bytes_per_step": shape.branches * width * 4,
                "ms_per_step": round(e2e_max / a.steps, 4)},
        "gpu_launches": launches * a.steps,
        "roofline": {"kernel": top_kernel, "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": peak_tc, "unit": "TFLOP/s",
                     "frac": round(achieved / peak_tc, 4), "peak_kind": f"{pk_kind} burst",
                     "traffic": traffic, "avg_launch_ms": round(top_avg, 5),
                     "flop_per_launch": top_flops},
        "pass_roofline": {
            "flop": work["flop_total"], "bytes": work["bytes_total"],
            "roofline_ms": round(max(rl_tc, rl_hbm), 4),
            "bound": "tensor" if rl_tc >= rl_hbm else "hbm",
            "tensor_ms": round(rl_tc, 4), "hbm_ms": round(rl_hbm, 4),
            "measured_ms": round(ms_step, 4), "frac": round(max(rl_tc, rl_hbm) / ms_step, 4),
            "hbm_frac": round(rl_hbm / ms_step, 4),
            "peaks": {"tflops": peak_tc, "gbs": peak_hbm, "kind": f"{pk_kind} burst"},
            "what": ("the whole pass: roofline time max(FLOP / tensor peak, bytes / HBM peak) "
                     "over the measured ms per pass; hbm_frac = bytes / HBM peak over it"),
        },
        "kernels": kernels,
        "kernels_note": "ms_per_pass from CUDA events between launches (serialised: the "
                        "events break the programmatic-dependent-launch overlap, so they sum "
                        "above ms_per_step); frac against the burst peaks",
        "clocks": clk,
        "build_s": round(t_build, 1),
    }
    if kv_state:
        out["kv_state"] = kv_state
    if kv_bcast:
        out["kv_broadcast"] = kv_bcast
    if dist.world == 1 and not a.no_cpu_baseline:
        cb = cpu_sample(shape)
        out["cpu_baseline"] = {
            "value": round(q_per_step / cb["per_request_s"], 4), "unit": UNIT,
            "cores": cb["threads"], "kind": "port",
            "sample": f"one whole {shape.name} request ({shape.layers} layers, the "
                      f"{shape.branches}-row lm_head) through oracle/ (the reference's CPU "
                      f"forward, tests/reference.rs:175-349, restated in C with OpenMP), "
                      f"{cb['sampled_s']:.1f} s"
                      + ("; the oracle keeps no K/V between calls, so the resident prefix is "
                         "recomputed" if resident else ""),
        }
    if dist.rank == 0:
        print(json.dumps(out), flush=True)
    eng.close()


def laya_oracle_model(shape, seed: int = 0):
    """The synthetic encoder of `shape` as the oracle takes it (the GPU arm's
    model, generated by oracle/ alone)."""
    from oracle import oracle as O
    ocfg = O.OracleLayaConfig(vocab=shape.vocab, d=shape.d, layers=shape.layers,
                              heads=shape.heads, ff=shape.ff, sliding=[0] * shape.layers,
                              window=64, head_layers=shape.head_layers,
                              act_out=shape.act_costs + 1)
    return ocfg, O.synth_tensors(ocfg.tensors(), seed, int(shape.dtype), laya=True)


def laya_oracle_batch(ocfg, tensors, seqs, threads: int) -> float:
    """`seqs` sequences through oracle/ (the GPU plan of laya.rs:1263-1345
    restated, every encoder and head layer): seconds of wall clock."""
    from oracle import oracle as O
    ids, pos, seq, qt = O.laya_pack([(r.ids, r.qtype) for r in seqs])
    t0 = time.perf_counter()
    O.laya_hidden(ocfg, tensors, ids, pos, seq, qt, O.ORACLE_EXACT, threads)
    return time.perf_counter() - t0


def laya_cpu_sample(shape, seqs: int, seed: int = 0) -> dict:
    """`seqs` of the batch's sequences at full depth through the oracle on all
    host cores; the sequences are independent, so sequences/s over the sample
    is the batch's rate."""
    from grande_b200 import synth
    threads = os.cpu_count() or 1
    ocfg, tensors = laya_oracle_model(shape, seed)
    s = laya_oracle_batch(ocfg, tensors, synth.laya_request(shape, 1000)[:seqs], threads)
    return {"seqs_per_s": seqs / s, "threads": threads, "sampled_s": s}


def laya_workload_config(shape, n: int) -> dict:
    return {
        "workload": f"{shape.name}: {shape.seqs} sequences x {shape.seq_len} tokens, full "
                    f"bidirectional attention, [CLS] + {shape.markers} [MASK] row(s) per "
                    f"sequence read back; 1 question per sequence",
        "model": f"{shape.name} shape, random init ({shape.layers} layers, d {shape.d}, "
                 f"{shape.heads} heads x 64, GeGLU ff {shape.ff}, vocab {shape.vocab}, "
                 f"{shape.head_layers} decision-head layers)",
        "tokens_per_pass": shape.tokens(), "parallelism": f"replicas x{n} (independent batches)",
        "l2": "activations larger than L2 (32768 x 768 f32 residual stream per pass)",
    }


def run_laya(a, dist: Dist):
    """the encoder over a batch of sequences."""
    from grande_b200 import synth
    shape = synth.LAYA_CONFIGS[a.config]
    if a.layers:
        import dataclasses
        shape = dataclasses.replace(shape, layers=a.layers)
    t_build = time.perf_counter()
    eng = synth.build_laya_engine(shape, shape.tokens(), shape.rows(), device=dist.local, seed=0)
    t_build = time.perf_counter() - t_build
    req = synth.laya_request(shape, seed=1000 + dist.rank)
    eng.time_forward(req, max(a.warmup, 3))
    dist.barrier()
    clocks = Clocks(gpu_index(dist.local))
    clocks.start()
    time.sleep(0.25)
    ms, launches = eng.time_forward(req, a.steps)
    ms_max = dist.max(ms)
    dist.barrier()
    reqs = [synth.laya_request(shape, seed=2000 + dist.rank * 100003 + i) for i in range(4)]
    for i in range(max(a.warmup, 3)):
        eng.evaluate(reqs[i % len(reqs)])
    dist.barrier()
    lat = []
    eng.record_event(0)
    for i in range(a.steps):
        t0 = time.perf_counter()
        eng.evaluate(reqs[i % len(reqs)])
        lat.append((time.perf_counter() - t0) * 1e3)
    eng.record_event(1)
    e2e_ms = eng.elapsed_ms(0, 1)
    e2e_max = dist.max(e2e_ms)
    dist.barrier()
    clk = clocks.stop()
    prof = eng.profile_forward(req, a.profile_iters)
    t = shape.tokens()
    wi_launches, wi_ms = prof["gemm_wi"]
    wi_avg = wi_ms / wi_launches
    flops_wi = 2.0 * t * shape.d * 2 * shape.ff
    pk, pk_kind = peaks()
    peak = pk.get("bf16_tflops")
    achieved = flops_wi / (wi_avg * 1e-3) / 1e12
    n = dist.world
    value = n * shape.seqs * a.steps / (ms_max * 1e-3)
    e2e_value = n * shape.seqs * a.steps / (e2e_max * 1e-3)
    out = {
        "metric": "questions/s/GPU mmBERT-shape Q8_0 encoder (256 seqs x 128 tokens)",
        "value": round(value, 2), "unit": UNIT, "n_gpus": n, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms_max / a.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: seeded N(0,0.02) weights quantized to Q8_0, uniform token ids",
        "config": laya_workload_config(shape, n),
        "p50_latency_ms": round(statistics.median(lat), 3) if lat else None,
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                "h2d_bytes_per_step": t * 4 * 4 + 8 * shape.markers * shape.seqs,
                "d2h_bytes_per_step": (shape.seqs * shape.markers + shape.seqs) * 4,
                "ms_per_step": round(e2e_max / a.steps, 4)},
        "gpu_launches": launches * a.steps,
        "roofline": {"kernel": "gemm_wi (tcgen05, fused erf GeGLU)", "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_kind": f"{pk_kind} burst",
                     "traffic": read_traffic("gemm_wi", a.config), "avg_launch_ms": round(wi_avg, 5),
                     "flop_per_launch": flops_wi},
        "kernels_ms_per_pass": {k: round(v[1] / a.profile_iters, 4) for k, v in prof.items()},
        "kernels_note": "CUDA events between launches (serialised: they sum above ms_per_step)",
        "clocks": clk,
        "build_s": round(t_build, 1),
    }
    if dist.world == 1 and not a.no_cpu_baseline:
        cb = laya_cpu_sample(shape, 32)
        out["cpu_baseline"] = {
            "value": round(cb["seqs_per_s"], 4), "unit": UNIT,
            "cores": cb["threads"], "kind": "port",
            "sample": f"32 of the batch's {shape.seqs} sequences through oracle/ "
                      f"(laya.rs:1263-1345 restated in C with OpenMP), all {shape.layers} "
                      f"encoder and {shape.head_layers} head layers; {cb['sampled_s']:.1f} s",
        }
    if dist.rank == 0:
        print(json.dumps(out), flush=True)
    eng.close()


def bench_kv_broadcast(eng, prefix, dist: Dist, iters: int = 10):
    """One state's K/V handed from rank 0 to every rank (grande_b200/split.py:
    export on rank 0, one NCCL broadcast, import on the others), the step that
    lets one state's branches run on several GPUs. CUDA events on torch's
    stream (where the broadcast runs; export and import complete before they
    return), max over ranks, median of `iters`."""
    import torch
    import torch.distributed as tdist
    from grande_b200.engine import Want
    from grande_b200.split import share_prefix
    if dist.rank == 0 and not eng.is_resident(prefix):
        eng.evaluate(prefix, [], Want.LOGITS)
    nbytes = eng.state_image_bytes(len(prefix))
    dev = torch.device("cuda", dist.local)
    buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    shares, bcasts = [], []
    for i in range(iters + 2):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        torch.cuda.synchronize(dev)
        dist.barrier()
        ev[0].record(stream)
        share_prefix(eng, prefix, src=0)
        ev[1].record(stream)
        ev[2].record(stream)
        tdist.broadcast(buf, src=0)
        ev[3].record(stream)
        torch.cuda.synchronize(dev)
        if i >= 2:
            shares.append(dist.max(ev[0].elapsed_time(ev[1])))
            bcasts.append(dist.max(ev[2].elapsed_time(ev[3])))
    share_ms, bcast_ms = statistics.median(shares), statistics.median(bcasts)
    return {"tokens": len(prefix), "bytes": nbytes, "ranks": dist.world,
            "share_ms": round(share_ms, 4), "broadcast_ms": round(bcast_ms, 4),
            "broadcast_gbs": round(nbytes / bcast_ms / 1e6, 1),
            "what": "export on rank 0 + NCCL broadcast + import on the others (share_ms); "
                    "the broadcast alone (broadcast_ms); CUDA events, max over ranks"}


def read_traffic(kernel: str, config: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary."""
    p = ROOT / "profiles" / f"{kernel}_{config}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            return float(line.split(":")[1])
    return None


# ---- the reference arm ------------------------------------------------------------------

def run_reference(a, dist: Dist):
    """The reference's CPU implementation of the path (its CPU forward,
    tests/reference.rs:175-349, restated in oracle/; the reference's own
    llama.cpp CPU backend cannot be built here), on this host's cores, on the
    GPU arm's workload: every step one whole request (all layers, the lm_head
    at the answer rows) on the same synthetic model, built by oracle/ alone."""
    if dist.rank != 0:
        return
    from grande_b200 import synth
    if a.config in synth.LAYA_CONFIGS:
        return run_reference_laya(a)
    shape = synth.CONFIGS[a.config]
    resident = a.config.endswith("resident")
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    ocfg, tensors = oracle_model(shape)
    setup_s = time.perf_counter() - t0
    req = synth.request(shape, seed=1000)
    per = []
    for i in range(a.warmup + a.steps):
        s = oracle_request(ocfg, tensors, req, threads)
        if i >= a.warmup:
            per.append(s)
    total = sum(per)
    value = shape.questions * len(per) / total
    sample = (f"per step: one whole {shape.name} request ({shape.layers} layers + the "
              f"{shape.branches}-row lm_head) through oracle/ (tests/reference.rs:175-349 "
              f"restated in C, OpenMP over {threads} threads)"
              + ("; the oracle keeps no K/V between calls, so the resident prefix is "
                 "recomputed every step" if resident else ""))
    out = {
        "impl": "reference", "metric": metric_of(shape, resident),
        "value": round(value, 4), "unit": UNIT,
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(total / len(per) * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,0.02) weights quantized to "
                f"{shape.dtype.name}_0, uniform token ids",
        "config": workload_config(shape, resident, a.gpus),
        "p50_latency_ms": round(statistics.median(per) * 1e3, 2),
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "setup_s": round(setup_s, 1),
    }
    print(json.dumps(out), flush=True)


def run_reference_laya(a):
    from grande_b200 import synth
    shape = synth.LAYA_CONFIGS[a.config]
    threads = os.cpu_count() or 1
    sample_seqs = 32
    t0 = time.perf_counter()
    ocfg, tensors = laya_oracle_model(shape)
    setup_s = time.perf_counter() - t0
    seqs = synth.laya_request(shape, 1000)[:sample_seqs]
    per = []
    for i in range(a.warmup + a.steps):
        s = laya_oracle_batch(ocfg, tensors, seqs, threads)
        if i >= a.warmup:
            per.append(s)
    total = sum(per)
    value = sample_seqs * len(per) / total
    out = {
        "impl": "reference",
        "metric": "questions/s/GPU mmBERT-shape Q8_0 encoder (256 seqs x 128 tokens)",
        "value": round(value, 4), "unit": UNIT, "n_gpus": a.gpus, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(total / len(per) * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,0.02) weights quantized to Q8_0, uniform token ids",
        "config": laya_workload_config(shape, a.gpus),
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"per step: {sample_seqs} of the batch's {shape.seqs} "
                                   f"sequences (independent, so sequences/s is the batch's "
                                   f"rate) through oracle/, all {shape.layers} encoder and "
                                   f"{shape.head_layers} head layers"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "setup_s": round(setup_s, 1),
    }
    print(json.dumps(out), flush=True)


def main():
    a = args_()
    dist = Dist(a.gpus)
    try:
        from grande_b200 import synth
        if a.impl == "reference":
            run_reference(a, dist)
        elif a.config in synth.LAYA_CONFIGS:
            run_laya(a, dist)
        else:
            run_b200(a, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
