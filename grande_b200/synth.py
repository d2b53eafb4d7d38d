"""Synthetic checkpoints and requests of the BASELINE configurations.

No real checkpoint ships with this repo (and the box has no network), so the
benchmark and the large-shape parity tests run on random models of the
reference's shapes: linear weights ~N(0, 0.02) and norm weights
1 + N(0, 0.02) (``norm_offset`` 0), quantized with the reference's Q8_0 /
Q4_0 rules; token ids uniform in [0, vocab). Every draw is seeded by
FNV-1a(tensor name) ^ seed (``omg_synth_normal``).
"""
from __future__ import annotations

import ctypes as C
import json
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np

from . import _lib
from .engine import BranchTokens, Dtype, EngineBuilder, Group, QTensor


@dataclass
class Shape:
    """One BASELINE.json configuration."""
    name: str
    layers: int
    d: int
    heads: int
    kv_heads: int
    ff: int
    global_every: int   # layer l is global iff (l + 1) % global_every == 0
    vocab: int
    dtype: Dtype
    gemma3_numerics: bool
    state: int          # prefix tokens
    branches: int
    branch_len: int
    questions: int      # questions per request (branches / option orders)

    def config(self) -> dict:
        types = ["full_attention" if (l + 1) % self.global_every == 0 else "sliding_attention"
                 for l in range(self.layers)]
        c = {
            "model_type": "gemma3_text" if self.gemma3_numerics else "gemma4_text",
            "vocab_size": self.vocab, "hidden_size": self.d, "num_hidden_layers": self.layers,
            "num_attention_heads": self.heads, "num_key_value_heads": self.kv_heads,
            "head_dim": 256, "intermediate_size": self.ff, "layer_types": types,
            "sliding_window": 512, "rms_norm_eps": 1e-6,
            "rope_parameters": {"full_attention": {"rope_theta": 1e6},
                                "sliding_attention": {"rope_theta": 1e4}},
            # Norm weights are drawn around 1 and applied as w.
            "omg_norm_offset": 0.0,
        }
        if self.gemma3_numerics:
            c["query_pre_attn_scalar"] = 256
        else:
            c["final_logit_softcapping"] = 30.0
        return c

    def config_json(self) -> str:
        return json.dumps(self.config())

    def tokens(self) -> int:
        return self.state + self.branches * self.branch_len


# BASELINE.json configs[0..3] (the decoder shapes).
CONFIGS = {
    "gemma3-270m-q8": Shape("gemma3-270m-q8", 18, 640, 4, 1, 2048, 6, 25000, Dtype.Q8, True,
                            90, 5, 12, 5),
    "e2b-q4": Shape("e2b-q4", 30, 2048, 8, 2, 8192, 5, 25000, Dtype.Q4, False, 500, 12, 24, 12),
    "e2b-q4-resident": Shape("e2b-q4-resident", 30, 2048, 8, 2, 8192, 5, 25000, Dtype.Q4, False,
                             2000, 12, 24, 12),
    "e4b-q4": Shape("e4b-q4", 35, 2560, 8, 2, 10240, 5, 25000, Dtype.Q4, False, 2000, 20, 32, 5),
}


def normal(seed: int, name: str, n: int, mean: float, std: float) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    _lib.check(_lib.lib().omg_synth_normal(seed, name.encode(), mean, std,
                                           _lib.ptr(out, C.c_float), n))
    return out


def tensor(seed: int, name: str, shape, dtype: Dtype) -> QTensor:
    n = int(np.prod(shape))
    if len(shape) == 1:
        return QTensor.from_f32(shape, normal(seed, name, n, 1.0, 0.02))
    v = normal(seed, name, n, 0.0, 0.02)
    return QTensor._encode(dtype, shape, v)


def build_engine(shape: Shape, capacity: int, max_rows: int, device: int = 0, seed: int = 0,
                 threads: int = 8):
    """Generate, quantize and push every tensor (generation in a thread pool;
    ctypes releases the GIL), then finish the engine."""
    b = EngineBuilder(shape.config_json(), device)
    specs = _lib_specs(shape.config_json())
    with ThreadPoolExecutor(max_workers=threads) as ex:
        futs = [(name, ex.submit(tensor, seed, name, dims, shape.dtype)) for name, dims in specs]
        for name, f in futs:
            b.push(name, f.result())
    return b.finish(capacity, max_rows)


def _lib_specs(config_json: str):
    from .engine import config_tensors
    return config_tensors(config_json)


def request(shape: Shape, seed: int = 0, state: int | None = None) -> Group:
    """A request of this shape: uniform token ids, the readout at each
    branch's last position."""
    rng = np.random.default_rng(seed)
    p = shape.state if state is None else state
    prefix = rng.integers(0, shape.vocab, p).tolist()
    branches = [BranchTokens(rng.integers(0, shape.vocab, shape.branch_len).tolist(),
                             [shape.branch_len - 1]) for _ in range(shape.branches)]
    return Group(prefix, branches)
