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
  encoder -- from per-launch CUDA events, against MEASURED_PEAKS.json, with
  ``traffic`` from the committed ncu summary under profiles/.
* ``kv_broadcast`` (resident config, N > 1): one state's K/V handed from
  rank 0 to every rank with one NCCL broadcast (grande_b200/split.py).
* ``cpu_baseline`` / ``--impl reference``: the reference's CPU forward
  (tests/reference.rs), restated in oracle/, on the host cores.

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
    ap.add_argument("--cpu-sample-layers", type=int, default=2)
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

def cpu_sample(shape, layers: int, seed: int = 0) -> dict:
    """One request of `shape` through the oracle with `layers` of the model's
    layers (same shapes, same synthetic weights), timed on the host cores;
    extrapolated linearly to the full depth (every layer has the same cost
    at this length up to the window) plus the 12-row lm_head."""
    import dataclasses

    from grande_b200 import synth
    from oracle import oracle as O
    small = dataclasses.replace(shape, layers=layers)
    cfgd = small.config()
    sliding = [t == "sliding_attention" for t in cfgd["layer_types"]]
    qs = 256 ** -0.5 if shape.gemma3_numerics else 1.0
    ocfg = O.OracleConfig(vocab=shape.vocab, d=shape.d, layers=layers, heads=shape.heads,
                          kv_heads=shape.kv_heads, head_dim=[256] * layers, ff=[shape.ff] * layers,
                          sliding=sliding, kv_source=list(range(layers)), rope_dims=[256] * layers,
                          window=512, query_scale=qs, norm_offset=0.0,
                          v_norm=not shape.gemma3_numerics,
                          softcap=0.0 if shape.gemma3_numerics else 30.0)
    tensors = []
    for name, dims in ocfg.tensors():
        qt = synth.tensor(seed, name, dims, shape.dtype)
        tensors.append(O.dequantize(int(qt.dtype), qt.data, qt.scales, qt.numel()))
    g = synth.request(shape, seed)
    ids, pos, seq = O.pack(g.prefix, [(b.tokens, b.want) for b in g.branches])
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    hid = O.forward(ocfg, tensors, ids, pos, seq, O.ORACLE_EXACT, threads)
    t_layers = time.perf_counter() - t0
    rows = [len(g.prefix) + sum(len(x.tokens) for x in g.branches[:i]) + g.branches[i].want[0]
            for i in range(len(g.branches))]
    emb = tensors[0]
    t1 = time.perf_counter()
    for r in rows:
        O.logits(hid[r], emb, shape.vocab, shape.d, ocfg.softcap)
    t_logits = time.perf_counter() - t1
    per_request = t_layers * shape.layers / layers + t_logits
    return {"per_request_s": per_request, "threads": threads, "sampled_s": t_layers + t_logits}


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
    eng = synth.build_engine(shape, cap, shape.branches, device=dist.local, seed=0)
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
    t_pass = len(req.prefix) * (0 if resident else 1) + sum(len(b.tokens) for b in req.branches)
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
    pk, pk_kind = peaks()
    peak = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
    achieved = top_flops / (top_avg * 1e-3) / 1e12
    n = dist.world
    value = n * q_per_step * a.steps / (ms_max * 1e-3)
    e2e_value = n * q_per_step * a.steps / (e2e_max * 1e-3)
    bytes_in = t_pass * (4 + 16 + 4) + 8 * (t_pass // 4 + 1)
    out = {
        "metric": metric_of(shape, resident), "value": round(value, 2), "unit": UNIT, "n_gpus": n,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_max / a.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: seeded N(0,0.02) weights quantized to "
                f"{shape.dtype.name}_0, uniform token ids",
        "config": {
            "workload": f"{shape.name}: {'resident ' if resident else ''}{shape.state}-token "
                        f"state + {shape.branches} branches x {shape.branch_len} tokens, one "
                        f"block-causal pass, logits at {shape.branches} answer rows; "
                        f"{q_per_step} questions per request, 1 request per GPU per step",
            "model": f"{shape.name} shape, random init ({shape.layers} layers, d {shape.d}, "
                     f"{shape.heads}q/{shape.kv_heads}kv heads x 256, ff {shape.ff}, "
                     f"vocab {shape.vocab})",
            "tokens_per_pass": t_pass, "parallelism": f"replicas x{n} (independent requests)",
            "l2": "inputs larger than L2: 3.6 GB of f16 weights stream from HBM every pass",
        },
        "p50_latency_ms": round(statistics.median(lat), 3) if lat else None,
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                "h2d_bytes_per_step": bytes_in, "d2h_bytes_per_step": shape.branches * width * 4,
                "ms_per_step": round(e2e_max / a.steps, 4)},
        "gpu_launches": launches * a.steps,
        "roofline": {"kernel": top_kernel, "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_kind": f"{pk_kind} sustained",
                     "traffic": traffic, "avg_launch_ms": round(top_avg, 5),
                     "flop_per_launch": top_flops},
        "kernels_ms_per_pass": {k: round(v[1] / a.profile_iters, 4) for k, v in prof.items()},
        "clocks": clk,
        "build_s": round(t_build, 1),
    }
    if kv_state:
        out["kv_state"] = kv_state
    if kv_bcast:
        out["kv_broadcast"] = kv_bcast
    if dist.world == 1 and not a.no_cpu_baseline:
        cb = cpu_sample(shape, a.cpu_sample_layers)
        out["cpu_baseline"] = {
            "value": round(q_per_step / cb["per_request_s"], 4), "unit": UNIT,
            "cores": cb["threads"], "kind": "port",
            "sample": f"one {shape.name} request through oracle/ (the reference's CPU forward, "
                      f"tests/reference.rs:141-349, restated in C with OpenMP) with "
                      f"{a.cpu_sample_layers} of {shape.layers} layers, extrapolated per layer, "
                      f"+ the {shape.branches}-row lm_head; {cb['sampled_s']:.1f} s sampled",
        }
    if dist.rank == 0:
        print(json.dumps(out), flush=True)
    eng.close()


def laya_cpu_sample(shape, seqs: int, seed: int = 0) -> dict:
    """`seqs` sequences of the encoder shape through oracle/ (the restated
    GPU plan of laya.rs:1263-1345) with one encoder layer, then one encoder
    layer + one head layer; per-layer times extrapolated to the full depth
    and to the whole batch."""
    import dataclasses

    from grande_b200 import synth
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    reqs = synth.laya_request(shape, seed)[:seqs]
    ids, pos, seq, qt = O.laya_pack([(r.ids, r.qtype) for r in reqs])
    times = []
    for head in (0, 1):
        ocfg = O.OracleLayaConfig(vocab=shape.vocab, d=shape.d, layers=1, heads=shape.heads,
                                  ff=shape.ff, sliding=[0], window=64, head_layers=head,
                                  act_out=shape.act_costs + 1)
        tensors = []
        for name, dims in ocfg.tensors():
            qt_ = synth.laya_tensor(seed, name, dims, shape.dtype)
            tensors.append(O.dequantize(int(qt_.dtype), qt_.data, qt_.scales, qt_.numel()))
        t0 = time.perf_counter()
        O.laya_hidden(ocfg, tensors, ids, pos, seq, qt, O.ORACLE_EXACT, threads)
        times.append(time.perf_counter() - t0)
    t_enc, t_head = times[0], max(times[1] - times[0], 0.0)
    per_batch = (t_enc * shape.layers + t_head * shape.head_layers) * shape.seqs / seqs
    return {"per_batch_s": per_batch, "threads": threads, "sampled_s": sum(times)}


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
    peak = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
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
        "config": {
            "workload": f"{shape.name}: {shape.seqs} sequences x {shape.seq_len} tokens, full "
                        f"bidirectional attention, [CLS] + {shape.markers} [MASK] row(s) per "
                        f"sequence read back; 1 question per sequence",
            "model": f"{shape.name} shape, random init ({shape.layers} layers, d {shape.d}, "
                     f"{shape.heads} heads x 64, GeGLU ff {shape.ff}, vocab {shape.vocab}, "
                     f"{shape.head_layers} decision-head layers)",
            "tokens_per_pass": t, "parallelism": f"replicas x{n} (independent batches)",
            "l2": "activations larger than L2 (32768 x 768 f32 residual stream per pass)",
        },
        "p50_latency_ms": round(statistics.median(lat), 3) if lat else None,
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                "h2d_bytes_per_step": t * 4 * 4 + 8 * shape.markers * shape.seqs,
                "d2h_bytes_per_step": (shape.seqs * shape.markers + shape.seqs) * 4,
                "ms_per_step": round(e2e_max / a.steps, 4)},
        "gpu_launches": launches * a.steps,
        "roofline": {"kernel": "gemm_wi (tcgen05, fused erf GeGLU)", "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_kind": f"{pk_kind} sustained",
                     "traffic": read_traffic("gemm_wi", a.config), "avg_launch_ms": round(wi_avg, 5),
                     "flop_per_launch": flops_wi},
        "kernels_ms_per_pass": {k: round(v[1] / a.profile_iters, 4) for k, v in prof.items()},
        "clocks": clk,
        "build_s": round(t_build, 1),
    }
    if dist.world == 1 and not a.no_cpu_baseline:
        cb = laya_cpu_sample(shape, 8)
        out["cpu_baseline"] = {
            "value": round(shape.seqs / cb["per_batch_s"], 4), "unit": UNIT,
            "cores": cb["threads"], "kind": "port",
            "sample": f"8 of {shape.seqs} sequences through oracle/ (laya.rs:1263-1345 restated "
                      f"in C with OpenMP), one encoder layer and one head layer, extrapolated "
                      f"to {shape.layers} + {shape.head_layers} layers and the whole batch; "
                      f"{cb['sampled_s']:.1f} s sampled",
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
    restated in oracle/), on this host's cores, on the same workload."""
    if dist.rank != 0:
        return
    from grande_b200 import synth
    if a.config in synth.LAYA_CONFIGS:
        return run_reference_laya(a)
    shape = synth.CONFIGS[a.config]
    # Each step is a bounded sample (a.cpu_sample_layers layers of one request,
    # extrapolated to the full depth) so K steps end within minutes.
    per = []
    threads = os.cpu_count() or 1
    for i in range(a.warmup + a.steps):
        cb = cpu_sample(shape, a.cpu_sample_layers, seed=i)
        if i >= a.warmup:
            per.append(cb["per_request_s"])
    total = sum(per)
    value = shape.questions * len(per) / total
    out = {
        "impl": "reference", "metric": metric_of(shape, a.config.endswith("resident")),
        "value": round(value, 4), "unit": UNIT,
        "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(total / len(per) * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{shape.name}: {shape.state}-token state + {shape.branches} "
                               f"branches x {shape.branch_len} tokens, logits at "
                               f"{shape.branches} rows"},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"per step: {a.cpu_sample_layers} of {shape.layers} layers "
                                   "of one request through oracle/ (tests/reference.rs:141-349 "
                                   "restated in C, OpenMP), extrapolated per layer, + lm_head"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def run_reference_laya(a):
    from grande_b200 import synth
    shape = synth.LAYA_CONFIGS[a.config]
    per = []
    threads = os.cpu_count() or 1
    for i in range(a.warmup + a.steps):
        cb = laya_cpu_sample(shape, 8, seed=i)
        if i >= a.warmup:
            per.append(cb["per_batch_s"])
    total = sum(per)
    value = shape.seqs * len(per) / total
    out = {
        "impl": "reference",
        "metric": "questions/s/GPU mmBERT-shape Q8_0 encoder (256 seqs x 128 tokens)",
        "value": round(value, 4), "unit": UNIT, "n_gpus": a.gpus, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(total / len(per) * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"{shape.name}: {shape.seqs} sequences x {shape.seq_len} tokens"},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": "per step: 8 sequences, one encoder + one head layer through "
                                   "oracle/, extrapolated to the full depth and batch"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
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
