"""TEST INFRASTRUCTURE ONLY: ctypes wrapper of the C oracle (omg_oracle.c).

The oracle restates the reference's CPU algorithms for the omg-wgpu forward
pass; the parity tests compare the CUDA engine against it. Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline leg may use this module.
The model catalogue below restates crates/omg-wgpu/src/model.rs:277-314 on
its own, independently of the product's copy.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libomg_oracle.so"
_lib = None

ORACLE_EXACT = 0
ORACLE_KERNEL = 1

F16, Q8, Q4 = 0, 1, 2


class _Cfg(C.Structure):
    _fields_ = [
        ("vocab", C.c_int), ("d", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
        ("kv_heads", C.c_int),
        ("head_dim", C.POINTER(C.c_int)), ("ff", C.POINTER(C.c_int)),
        ("sliding", C.POINTER(C.c_int)), ("kv_source", C.POINTER(C.c_int)),
        ("rope_dims", C.POINTER(C.c_int)),
        ("eps", C.c_float), ("window", C.c_int), ("theta_global", C.c_float),
        ("theta_local", C.c_float), ("query_scale", C.c_float), ("norm_offset", C.c_float),
        ("v_norm", C.c_int), ("per_layer_dim", C.c_int), ("softcap", C.c_float),
    ]


class _LayaCfg(C.Structure):
    _fields_ = [
        ("vocab", C.c_int), ("d", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
        ("ff", C.c_int), ("sliding", C.POINTER(C.c_int)), ("window", C.c_int),
        ("theta_global", C.c_float), ("theta_local", C.c_float), ("eps", C.c_float),
        ("head_layers", C.c_int), ("type_emb", C.c_int),
    ]


def build() -> Path:
    """Compile the oracle with its Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = C.CDLL(str(LIB_PATH))
        fp = C.POINTER(C.c_float)
        u8 = C.POINTER(C.c_uint8)
        _lib.oracle_f32_to_f16_n.argtypes = [fp, C.c_size_t, C.POINTER(C.c_uint16)]
        _lib.oracle_f16_to_f32_n.argtypes = [C.POINTER(C.c_uint16), C.c_size_t, fp]
        _lib.oracle_rng_values.argtypes = [C.POINTER(C.c_uint64), fp, C.c_size_t, C.c_float]
        _lib.oracle_synth_normal.argtypes = [C.c_uint64, C.c_char_p, C.c_float, C.c_float, fp,
                                             C.c_size_t]
        _lib.oracle_quantize_q8.argtypes = [fp, C.c_size_t, u8, u8]
        _lib.oracle_quantize_q4.argtypes = [fp, C.c_size_t, u8, u8]
        _lib.oracle_dequant.argtypes = [C.c_int, u8, u8, C.c_size_t, fp]
        _lib.oracle_forward.argtypes = [
            C.POINTER(_Cfg), C.POINTER(fp), C.c_size_t, C.POINTER(C.c_uint32),
            C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.c_size_t, C.c_int, C.c_int, fp]
        _lib.oracle_forward_layers.argtypes = _lib.oracle_forward.argtypes + [fp]
        _lib.oracle_visible.argtypes = [C.c_int32] * 4 + [C.c_int]
        _lib.oracle_logits.argtypes = [fp, fp, C.c_int, C.c_int, C.c_float, fp]
        _lib.oracle_softmax.argtypes = [fp, C.c_size_t, C.c_float, C.POINTER(C.c_double)]
        _lib.oracle_log_sum_exp.argtypes = [fp, C.c_size_t]
        _lib.oracle_log_sum_exp.restype = C.c_double
        _lib.oracle_laya_hidden.argtypes = [
            C.POINTER(_LayaCfg), C.POINTER(fp), C.c_size_t, C.POINTER(C.c_uint32),
            C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.POINTER(C.c_uint32), C.c_size_t,
            C.c_int, C.c_int, fp]
        _lib.oracle_laya_score.argtypes = [fp, C.c_int, C.c_int, C.c_float, C.POINTER(fp),
                                           C.c_int, C.c_int, fp, fp]
    return _lib


def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t))


# ---- numerics ---------------------------------------------------------------

def f32_to_f16_bits(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_f16_n(_p(x, C.c_float), x.size, _p(out, C.c_uint16))
    return out


def f16_bits_to_f32(h) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().oracle_f16_to_f32_n(_p(h, C.c_uint16), h.size, _p(out, C.c_float))
    return out


class Rng:
    """tests/reference.rs:17-38: xorshift64 in [-1, 1)."""

    def __init__(self, seed: int):
        self.state = C.c_uint64(seed)

    def values(self, n: int, scale: float) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        lib().oracle_rng_values(C.byref(self.state), _p(out, C.c_float), n, scale)
        return out

    def next(self) -> float:
        return float(self.values(1, 1.0)[0])


def quantize(dtype: int, values) -> tuple[bytes, bytes]:
    """QTensor::{from_f32, quantize_q8, quantize_q4} (model.rs:395-466):
    (payload bytes, scale bytes)."""
    v = np.ascontiguousarray(values, dtype=np.float32).ravel()
    if dtype == F16:
        return f32_to_f16_bits(v).tobytes(), b""
    n = v.size
    codes = np.empty(n if dtype == Q8 else n // 2, dtype=np.uint8)
    scales = np.empty(n // 32 * 2, dtype=np.uint8)
    fn = lib().oracle_quantize_q8 if dtype == Q8 else lib().oracle_quantize_q4
    if fn(_p(v, C.c_float), n, _p(codes, C.c_uint8), _p(scales, C.c_uint8)) != 0:
        raise ValueError(f"{n} values is not a multiple of 32")
    return codes.tobytes(), scales.tobytes()


def dequantize(dtype: int, data: bytes, scales: bytes, n: int) -> np.ndarray:
    """QTensor::get over every element (model.rs:508-525)."""
    d = np.frombuffer(data, dtype=np.uint8).copy()
    s = np.frombuffer(scales, dtype=np.uint8).copy() if scales else np.zeros(2, np.uint8)
    out = np.empty(n, dtype=np.float32)
    if lib().oracle_dequant(dtype, _p(d, C.c_uint8), _p(s, C.c_uint8), n, _p(out, C.c_float)):
        raise ValueError("bad dtype")
    return out


# ---- synthetic models (the benchmark's random checkpoints) -----------------------

def synth_normal(seed: int, name: str, n: int, mean: float, std: float) -> np.ndarray:
    """The synthetic models' draws: FNV-1a(name) ^ seed into xorshift64, Box-Muller."""
    out = np.empty(n, dtype=np.float32)
    lib().oracle_synth_normal(seed, name.encode(), mean, std, _p(out, C.c_float), n)
    return out


def synth_tensor(seed: int, name: str, shape, dtype: int, laya: bool = False,
                 qk_scale: float = 1.0) -> np.ndarray:
    """One tensor of a synthetic model, quantized and dequantized by the
    reference's rules (model.rs:395-525), as f32. Decoder: 2-D linears and
    tables ~N(0, 0.02) in `dtype`, 1-D norm weights 1 + N(0, 0.02) in f16.
    Encoder (`laya`): the same, except biases (names ending in `_b`) are
    N(0, 0.02), and the type embedding and the host head (scorer.*, act.*)
    stay f16. `qk_scale` multiplies the decoder's q / k head norm weights
    (the conditioned variant of the model)."""
    n = int(np.prod(shape))
    last = name.rsplit(".", 1)[-1]
    if len(shape) == 1:
        mean = 0.0 if (laya and last.endswith("_b")) else 1.0
        v, dt = synth_normal(seed, name, n, mean, 0.02), F16
        if qk_scale != 1.0 and (name.endswith(".q_norm") or name.endswith(".k_norm")):
            v = v * np.float32(qk_scale)
    else:
        v, dt = synth_normal(seed, name, n, 0.0, 0.02), dtype
        if laya and (name.startswith("scorer.") or name.startswith("act.") or name == "type_emb"):
            dt = F16
    data, scales = quantize(dt, v)
    return dequantize(dt, data, scales, n)


def synth_tensors(specs, seed: int, dtype: int, laya: bool = False, threads: int = 0,
                  qk_scale: float = 1.0) -> list:
    """Every tensor of `specs` [(name, shape)] as f32, generated in a thread
    pool (the C calls release the GIL)."""
    import os
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=threads or os.cpu_count() or 1) as ex:
        futs = [ex.submit(synth_tensor, seed, name, shape, dtype, laya, qk_scale)
                for name, shape in specs]
        return [f.result() for f in futs]


# ---- model description --------------------------------------------------------

@dataclass
class OracleConfig:
    """model.rs:28-63, the fields the forward uses."""
    vocab: int
    d: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: list
    ff: list
    sliding: list
    kv_source: list
    rope_dims: list
    eps: float = 1e-6
    window: int = 512
    theta_global: float = 1e6
    theta_local: float = 1e4
    query_scale: float = 1.0
    norm_offset: float = 0.0
    v_norm: bool = False
    per_layer_dim: int = 0
    softcap: float = 0.0
    bos: int = 2
    _keep: list = field(default_factory=list, repr=False)

    def has_kv(self, l: int) -> bool:
        return self.kv_source[l] == l

    def qkv_width(self, l: int) -> int:
        hd = self.head_dim[l]
        return (self.heads + 2 * self.kv_heads) * hd if self.has_kv(l) else self.heads * hd

    def tensors(self) -> list[tuple[str, list[int]]]:
        """model.rs:277-314."""
        d = self.d
        v = [("embed", [self.vocab, d]), ("final_norm", [d])]
        if self.per_layer_dim > 0:
            p = self.per_layer_dim
            v += [("pl_model_proj", [p * self.layers, d]), ("pl_proj_norm", [p])]
        for l in range(self.layers):
            hd, ff = self.head_dim[l], self.ff[l]
            n = lambda s: f"blk.{l}.{s}"  # noqa: E731
            v.append((n("attn_norm"), [d]))
            v.append((n("qkv"), [self.qkv_width(l), d]))
            v.append((n("q_norm"), [hd]))
            if self.has_kv(l):
                v.append((n("k_norm"), [hd]))
            v += [(n("o"), [d, self.heads * hd]), (n("post_attn_norm"), [d]),
                  (n("ffn_norm"), [d]), (n("gate"), [ff, d]), (n("up"), [ff, d]),
                  (n("down"), [d, ff]), (n("post_ffn_norm"), [d])]
            if self.per_layer_dim > 0:
                p = self.per_layer_dim
                v += [(n("pl_gate"), [p, d]), (n("pl_proj"), [d, p]), (n("pl_norm"), [d]),
                      (n("out_scale"), [1])]
        return v

    def _c(self) -> _Cfg:
        arr = lambda xs: (C.c_int * len(xs))(*[int(x) for x in xs])  # noqa: E731
        keep = [arr(self.head_dim), arr(self.ff), arr([int(s) for s in self.sliding]),
                arr(self.kv_source), arr(self.rope_dims)]
        self._keep = keep
        return _Cfg(self.vocab, self.d, self.layers, self.heads, self.kv_heads, *keep,
                    self.eps, self.window, self.theta_global, self.theta_local,
                    self.query_scale, self.norm_offset, int(self.v_norm), self.per_layer_dim,
                    self.softcap)


def forward(cfg: OracleConfig, tensors: list, ids, pos, seq, mode: int = ORACLE_EXACT,
            threads: int = 0, per_layer: bool = False):
    """tests/reference.rs:175-349: final-norm hidden rows [t, d]. `tensors` are
    dequantized f32 arrays in catalogue order (+ the per-layer table). With
    `per_layer`, also [layers, t, d]: after each layer l, the hidden rows the
    model cut after layer l returns (the final norm of its stream)."""
    arrs = [np.ascontiguousarray(t, dtype=np.float32).ravel() for t in tensors]
    ptrs = (C.POINTER(C.c_float) * len(arrs))(*[_p(a, C.c_float) for a in arrs])
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    seq = np.ascontiguousarray(seq, dtype=np.int32)
    t = ids.size
    out = np.empty((t, cfg.d), dtype=np.float32)
    layers = np.empty((cfg.layers, t, cfg.d), dtype=np.float32) if per_layer else None
    c = cfg._c()
    rc = lib().oracle_forward_layers(C.byref(c), ptrs, len(arrs), _p(ids, C.c_uint32),
                                     _p(pos, C.c_int32), _p(seq, C.c_int32), t, mode, threads,
                                     _p(out, C.c_float),
                                     _p(layers, C.c_float) if per_layer else None)
    if rc != 0:
        raise ValueError(f"oracle_forward failed ({rc})")
    return (out, layers) if per_layer else out


def visible(qp, qs, kp, ks, window) -> bool:
    return bool(lib().oracle_visible(qp, qs, kp, ks, window))


def logits(hidden_row, embed, vocab, d, softcap=0.0) -> np.ndarray:
    h = np.ascontiguousarray(hidden_row, dtype=np.float32)
    e = np.ascontiguousarray(embed, dtype=np.float32)
    out = np.empty(vocab, dtype=np.float32)
    lib().oracle_logits(_p(h, C.c_float), _p(e, C.c_float), vocab, d, softcap,
                        _p(out, C.c_float))
    return out


def softmax(z, temperature=1.0) -> np.ndarray:
    z = np.ascontiguousarray(z, dtype=np.float32)
    out = np.empty(z.size, dtype=np.float64)
    lib().oracle_softmax(_p(z, C.c_float), z.size, temperature, _p(out, C.c_double))
    return out


def log_sum_exp(z) -> float:
    z = np.ascontiguousarray(z, dtype=np.float32)
    return float(lib().oracle_log_sum_exp(_p(z, C.c_float), z.size))


def pack(prefix, branches):
    """tests/reference.rs:368-378: ids and (pos, seq) of prefix + branches."""
    ids = list(prefix)
    pos = list(range(len(prefix)))
    seq = [0] * len(prefix)
    for bi, (toks, _want) in enumerate(branches):
        for j, t in enumerate(toks):
            ids.append(t)
            pos.append(len(prefix) + j)
            seq.append(bi + 1)
    return np.array(ids, np.uint32), np.array(pos, np.int32), np.array(seq, np.int32)


def pack_groups(groups):
    """engine.rs:1512-1571 for groups laid out in order, all decoded: ids,
    pos, seq with group k's sequence ids under k << 12."""
    ids, pos, seq = [], [], []
    for k, (prefix, branches) in enumerate(groups):
        hi = k << 12
        for i, t in enumerate(prefix):
            ids.append(t)
            pos.append(i)
            seq.append(hi)
        for bi, (toks, _want) in enumerate(branches):
            for j, t in enumerate(toks):
                ids.append(t)
                pos.append(len(prefix) + j)
                seq.append(hi | (bi + 1))
    return np.array(ids, np.uint32), np.array(pos, np.int32), np.array(seq, np.int32)


# ---- Laya / ModernBERT encoder (crates/omg-wgpu/src/laya.rs) ------------------

@dataclass
class OracleLayaConfig:
    """LayaConfig (laya.rs:46-83), the fields the forward and scorer read."""
    vocab: int
    d: int
    layers: int
    heads: int
    ff: int
    sliding: list
    window: int = 64
    theta_global: float = 160000.0
    theta_local: float = 10000.0
    eps: float = 1e-5
    head_layers: int = 2
    type_emb: bool = True
    act_hidden: int = 256
    act_out: int = 0
    _keep: list = field(default_factory=list, repr=False)

    def tensors(self) -> list[tuple[str, list[int]]]:
        """LayaConfig::tensors (laya.rs:265-313)."""
        d, ff = self.d, self.ff
        v = [("embed", [self.vocab, d]), ("embed_norm", [d]), ("final_norm", [d])]
        if self.type_emb:
            v.append(("type_emb", [3, d]))
        for l in range(self.layers):
            n = lambda s: f"enc.{l}.{s}"  # noqa: E731
            if l > 0:
                v.append((n("attn_norm"), [d]))
            v += [(n("qkv"), [3 * d, d]), (n("o"), [d, d]), (n("mlp_norm"), [d]),
                  (n("wi_val"), [ff, d]), (n("wi_gate"), [ff, d]), (n("wo"), [d, ff])]
        for h in range(self.head_layers):
            n = lambda s: f"head.{h}.{s}"  # noqa: E731
            v += [(n("norm1_w"), [d]), (n("norm1_b"), [d]), (n("in_proj"), [3 * d, d]),
                  (n("in_proj_b"), [3 * d]), (n("out_proj"), [d, d]), (n("out_proj_b"), [d]),
                  (n("norm2_w"), [d]), (n("norm2_b"), [d]), (n("l1"), [4 * d, d]),
                  (n("l1_b"), [4 * d]), (n("l2"), [d, 4 * d]), (n("l2_b"), [d])]
        v += [("scorer.norm_w", [d]), ("scorer.norm_b", [d]), ("scorer.l1", [d, d]),
              ("scorer.l1_b", [d]), ("scorer.l2", [1, d]), ("scorer.l2_b", [1])]
        if self.act_out > 0:
            v += [("act.l1", [self.act_hidden, d + 4]), ("act.l1_b", [self.act_hidden]),
                  ("act.l2", [self.act_out, self.act_hidden]), ("act.l2_b", [self.act_out])]
        return v

    def _c(self) -> _LayaCfg:
        sl = (C.c_int * len(self.sliding))(*[int(s) for s in self.sliding])
        self._keep = [sl]
        return _LayaCfg(self.vocab, self.d, self.layers, self.heads, self.ff, sl, self.window,
                        self.theta_global, self.theta_local, self.eps, self.head_layers,
                        int(self.type_emb))


def laya_pack(seqs):
    """laya.rs:1161-1189: ids, positions (index in the sequence), sequence
    index and question type per token of the sequences [(ids, qtype), ...]."""
    ids, pos, seq, qt = [], [], [], []
    for si, (toks, qtype) in enumerate(seqs):
        for i, t in enumerate(toks):
            ids.append(t)
            pos.append(i)
            seq.append(si)
            qt.append(qtype)
    return (np.array(ids, np.uint32), np.array(pos, np.int32), np.array(seq, np.int32),
            np.array(qt, np.uint32))


def laya_hidden(cfg: OracleLayaConfig, tensors: list, ids, pos, seq, qtype,
                mode: int = ORACLE_EXACT, threads: int = 0) -> np.ndarray:
    """The residual stream x [t, d] after the decision-head layers (the rows
    LayaEngine::hidden reads back). `tensors` in LayaConfig::tensors order."""
    arrs = [np.ascontiguousarray(t, dtype=np.float32).ravel() for t in tensors]
    ptrs = (C.POINTER(C.c_float) * len(arrs))(*[_p(a, C.c_float) for a in arrs])
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    seq = np.ascontiguousarray(seq, dtype=np.int32)
    qtype = np.ascontiguousarray(qtype, dtype=np.uint32)
    t = ids.size
    out = np.empty((t, cfg.d), dtype=np.float32)
    c = cfg._c()
    rc = lib().oracle_laya_hidden(C.byref(c), ptrs, len(arrs), _p(ids, C.c_uint32),
                                  _p(pos, C.c_int32), _p(seq, C.c_int32),
                                  _p(qtype, C.c_uint32), t, mode, threads, _p(out, C.c_float))
    if rc != 0:
        raise ValueError(f"oracle_laya_hidden failed ({rc})")
    return out


def laya_score(cfg: OracleLayaConfig, host: dict, rows) -> tuple[np.ndarray, float | None]:
    """LayaEngine::score (laya.rs:1442-1493) on [CLS] + marker rows."""
    rows = np.ascontiguousarray(rows, dtype=np.float32)
    k = rows.shape[0] - 1
    names = ["scorer.norm_w", "scorer.norm_b", "scorer.l1", "scorer.l1_b", "scorer.l2",
             "scorer.l2_b", "act.l1", "act.l1_b", "act.l2", "act.l2_b"]
    arrs = [np.ascontiguousarray(host.get(n, np.zeros(1, np.float32)), dtype=np.float32).ravel()
            for n in names]
    ptrs = (C.POINTER(C.c_float) * len(arrs))(*[_p(a, C.c_float) for a in arrs])
    logits = np.empty(k, np.float32)
    act = np.zeros(1, np.float32)
    rc = lib().oracle_laya_score(_p(rows, C.c_float), k, cfg.d, cfg.eps, ptrs, cfg.act_hidden,
                                 cfg.act_out, _p(logits, C.c_float), _p(act, C.c_float))
    if rc != 0:
        raise ValueError("oracle_laya_score failed")
    return logits, (float(act[0]) if cfg.act_out > 0 else None)
