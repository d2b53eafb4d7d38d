"""Python mirror of the reference's Laya encoder API
(crates/omg-wgpu/src/laya.rs): ``LayaBuilder``, ``LayaEngine``, ``Sequence``
and ``Output``, over the C ABI (include/omg_b200.h, ``omg_laya_*``).

The config is the exported directory's ``config.json`` (the ModernBERT
encoder config with ``laya_agent`` and ``laya_tokens``, laya.rs:312-323) plus
``laya_special_ids``: the special tokens' ids, which the reference looks up
with its tokenizer (the caller owns tokenization here, as it owns the prompt
layout of laya/prompt.rs).

There is no CPU fallback: without the native library every call raises.
"""
from __future__ import annotations

import ctypes as C
from itertools import chain
import json
from dataclasses import dataclass, field
from typing import Optional, Sequence as Seq

import numpy as np

from . import _lib
from ._lib import OmgError, check, lib
from .engine import QTensor, _buf, _shape

QTYPES = ("choice", "score", "noul")  # laya.rs:43


@dataclass
class Sequence:
    """laya.rs:469-476: one question's ids, its options' [MASK] indices,
    its question type (0 choice, 1 score, 2 noul)."""
    ids: list
    markers: list
    qtype: int = 0


@dataclass
class Output:
    """laya.rs:482-485: scorer logits per option (before temperature) and
    the act head's probability (None without an act head)."""
    logits: np.ndarray
    act_probability: Optional[float] = None


class _Seqs:
    """Keeps the ctypes arrays of a request alive for one call."""

    def __init__(self, seqs: Seq[Sequence]):
        n = len(seqs)
        self.arr = (_lib.LayaSeqC * max(1, n))()
        # One array for every sequence's ids and one for every marker; each
        # sequence points at its slice (one conversion per field, not per
        # sequence).
        lens = [len(s.ids) for s in seqs]
        nmk = [len(s.markers) for s in seqs]
        ids = np.fromiter(chain.from_iterable(s.ids for s in seqs), dtype=np.int64,
                          count=sum(lens)).astype(np.uint32)
        mk = np.fromiter(chain.from_iterable(s.markers for s in seqs), dtype=np.int64,
                         count=sum(nmk)).astype(np.uint64)
        self.keep = [ids, mk]
        ib, mb = ids.ctypes.data, mk.ctypes.data
        io = mo = 0
        for i, s in enumerate(seqs):
            a = self.arr[i]
            a.ids = ib + 4 * io
            a.n_ids = lens[i]
            a.markers = mb + 8 * mo
            a.n_markers = nmk[i]
            a.qtype = int(s.qtype)
            io += lens[i]
            mo += nmk[i]
        self.n = len(seqs)


def _text(fn, *args) -> str:
    need = C.c_size_t(0)
    check(fn(*args, None, 0, C.byref(need)))
    buf = C.create_string_buffer(need.value)
    check(fn(*args, buf, need.value, C.byref(need)))
    return buf.value.decode()


def config_tensors(config_json: str) -> list:
    """LayaConfig::tensors (laya.rs:252-309): [(name, shape)]."""
    out = []
    for line in _text(lib().omg_laya_config_tensors, config_json.encode()).split("\n"):
        if line:
            name, dims = line.split(" ")
            out.append((name, [int(x) for x in dims.split(",")]))
    return out


def config_check(config_json: str) -> str:
    """LayaConfig::from_json + validate (laya.rs:88-230)."""
    buf = C.create_string_buffer(256)
    check(lib().omg_laya_config_check(config_json.encode(), buf, 256))
    return buf.value.decode()


def is_host_tensor(name: str) -> bool:
    """laya.rs:326-328."""
    return name.startswith("scorer.") or name.startswith("act.")


class LayaEngine:
    """laya.rs:1086-1494 on one B200."""

    def __init__(self, handle, config: dict, capacity: int, max_rows: int):
        self._h = handle
        self.config = config
        self.capacity = capacity
        self.max_rows = max_rows
        self.d = int(config["hidden_size"])

    def close(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            lib().omg_laya_destroy(h)

    def __del__(self):
        self.close()

    @staticmethod
    def new(weights: "dict[str, QTensor]", config_json, capacity: int, max_rows: int,
            device: int = 0) -> "LayaEngine":
        """LayaEngine::new (laya.rs:1115-1122): upload a whole checkpoint."""
        b = LayaBuilder(config_json, device)
        for name, _ in config_tensors(b.config_json):
            if name not in weights:
                raise OmgError(f"missing tensor {name}")
            b.push(name, weights[name])
        return b.finish(capacity, max_rows)

    def warmup(self):
        check(lib().omg_laya_warmup(self._h))

    def hidden(self, seqs: Seq[Sequence]) -> list:
        """laya.rs:1138-1432: per sequence [CLS] row then each marker's row."""
        req = _Seqs(seqs)
        nrows = sum(1 + len(s.markers) for s in seqs)
        out = np.empty((max(nrows, 1), self.d), dtype=np.float32)
        check(lib().omg_laya_hidden(self._h, req.arr, req.n, _lib.ptr(out, C.c_float), out.size))
        res, r = [], 0
        for s in seqs:
            res.append(out[r:r + 1 + len(s.markers)])  # views into this call's array
            r += 1 + len(s.markers)
        return res

    def evaluate(self, seqs: Seq[Sequence]) -> list:
        """laya.rs:1435-1438."""
        req = _Seqs(seqs)
        k = sum(len(s.markers) for s in seqs)
        logits = np.empty(max(k, 1), dtype=np.float32)
        act = np.empty(max(len(seqs), 1), dtype=np.float32)
        check(lib().omg_laya_evaluate(self._h, req.arr, req.n, _lib.ptr(logits, C.c_float), k,
                                      _lib.ptr(act, C.c_float)))
        res, o = [], 0
        for i, s in enumerate(seqs):
            a = float(act[i])
            res.append(Output(logits[o:o + len(s.markers)], None if np.isnan(a) else a))
            o += len(s.markers)
        return res

    def probabilities(self, qtype: int, logits) -> np.ndarray:
        """laya.rs:1489-1493."""
        z = np.ascontiguousarray(logits, dtype=np.float32)
        out = np.empty(z.size, dtype=np.float64)
        check(lib().omg_laya_probabilities(self._h, int(qtype), _lib.ptr(z, C.c_float), z.size,
                                           out.ctypes.data_as(C.POINTER(C.c_double))))
        return out

    def time_forward(self, seqs: Seq[Sequence], iters: int) -> tuple[float, int]:
        req = _Seqs(seqs)
        ms, n = C.c_float(0), C.c_int(0)
        check(lib().omg_laya_time_forward(self._h, req.arr, req.n, iters, C.byref(ms),
                                          C.byref(n)))
        return ms.value, n.value

    def profile_forward(self, seqs: Seq[Sequence], iters: int) -> dict:
        """Per-kernel device time: {name: (launches, total_ms)} (one run of
        the passes, so one call with a buffer large enough for the report)."""
        req = _Seqs(seqs)
        need = C.c_size_t(0)
        buf = C.create_string_buffer(16384)
        check(lib().omg_laya_profile_forward(self._h, req.arr, req.n, iters, buf, 16384,
                                             C.byref(need)))
        if need.value > 16384:
            raise OmgError(f"profile report needs {need.value} bytes")
        return {k: tuple(v) for k, v in json.loads(buf.value.decode()).items()}

    def record_event(self, slot: int):
        check(lib().omg_laya_record_event(self._h, slot))

    def elapsed_ms(self, a: int, b: int) -> float:
        ms = C.c_float(0)
        check(lib().omg_laya_elapsed_ms(self._h, a, b, C.byref(ms)))
        return ms.value


class LayaBuilder:
    """laya.rs:612-1084."""

    def __init__(self, config_json, device: int = 0):
        if isinstance(config_json, dict):
            config_json = json.dumps(config_json)
        self.config_json = config_json
        self.config = json.loads(config_json)
        h = C.c_void_p()
        check(lib().omg_laya_builder_new(config_json.encode(), device, C.byref(h)))
        self._h = h

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            lib().omg_laya_builder_free(h)

    def push(self, name: str, t: QTensor):
        check(lib().omg_laya_builder_push(self._h, name.encode(), int(t.dtype), _shape(t.shape),
                                          len(t.shape), _buf(t.data), len(t.data),
                                          _buf(t.scales), len(t.scales)))

    def missing(self) -> list:
        return [s for s in _text(lib().omg_laya_builder_missing, self._h).split("\n") if s]

    def finish(self, capacity: int, max_rows: int) -> LayaEngine:
        h = C.c_void_p()
        b, self._h = self._h, None
        check(lib().omg_laya_builder_finish(b, capacity, max_rows, C.byref(h)))
        return LayaEngine(h, self.config, capacity, max_rows)


def synthetic_config(vocab: int, d: int, layers: int, heads: int, ff: int, *,
                     local_attention: int = 128, head_layers: int = 2, act_costs: int = 0,
                     every: int = 3, layer_types: Optional[list] = None,
                     temperature=(1.0, 1.0, 1.0), max_len: int = 512) -> dict:
    """An exported-directory config.json (laya.rs:312-323) for a model of
    this shape, special tokens at ids 1..4 ([CLS], [SEP], [MASK], [PAD])."""
    enc = {"model_type": "modernbert", "hidden_activation": "gelu", "vocab_size": vocab,
           "hidden_size": d, "num_hidden_layers": layers, "num_attention_heads": heads,
           "intermediate_size": ff, "global_attn_every_n_layers": every,
           "local_attention": local_attention, "global_rope_theta": 160000.0,
           "local_rope_theta": 10000.0, "norm_eps": 1e-5}
    if layer_types is not None:
        enc["layer_types"] = layer_types
    agent = {"head_layers": head_layers, "type_emb": True, "temperature": list(temperature),
             "max_len": max_len, "head_max_len": min(192, max_len - 1)}
    if act_costs:
        agent["act_costs"] = {f"a{i}": 1.0 for i in range(act_costs)}
    else:
        agent["act_head"] = False
    enc["laya_agent"] = agent
    enc["laya_tokens"] = {"cls_token": "[CLS]", "sep_token": "[SEP]",
                          "mask_token": {"content": "[MASK]"}, "pad_token": "[PAD]"}
    enc["laya_special_ids"] = {"[CLS]": 1, "[SEP]": 2, "[MASK]": 3, "[PAD]": 4}
    return enc
