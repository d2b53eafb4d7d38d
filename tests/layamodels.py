"""Seeded Laya / ModernBERT test models: an oracle config, the exported
config.json the engine parses, the engine's QTensors and the oracle's
dequantized f32 tensors (LayaConfig::tensors order, laya.rs:252-309).
Test infrastructure."""
from __future__ import annotations

import json
import math

import numpy as np

from oracle import oracle as O


def laya_weights(cfg: O.OracleLayaConfig, seed: int) -> list[np.ndarray]:
    """Seeded f16-representable weights in catalogue order, from the xorshift
    of tests/reference.rs:17-26: norm weights 1 + U(-0.1, 0.1), biases
    U(-0.1, 0.1), the embedding U(-1, 1), the type embedding U(-0.2, 0.2),
    linears U(-s, s) with s = 1.2 / sqrt(fan_in)."""
    r = O.Rng(seed)
    out = []
    for name, shape in cfg.tensors():
        n = int(np.prod(shape))
        last = name.rsplit(".", 1)[-1]
        if name in ("embed", "type_emb"):
            v = r.values(n, 1.0 if name == "embed" else 0.2)
        elif len(shape) == 1 and last.endswith("_b"):
            v = r.values(n, 0.1)
        elif len(shape) == 1:
            v = r.values(n, 0.1) + 1.0
        else:
            v = r.values(n, 1.2 / math.sqrt(shape[1]))
        out.append(O.f16_bits_to_f32(O.f32_to_f16_bits(v)).reshape(shape))
    return out


def config_json(cfg: O.OracleLayaConfig, temperature=(1.0, 1.0, 1.0), by_options=None,
                max_len: int = 512) -> dict:
    """The exported config.json (laya.rs:312-323) for `cfg`, with the
    special-token ids the caller resolves ([CLS] 1, [SEP] 2, [MASK] 3,
    [PAD] 4)."""
    enc = {"model_type": "modernbert", "hidden_activation": "gelu", "vocab_size": cfg.vocab,
           "hidden_size": cfg.d, "num_hidden_layers": cfg.layers,
           "num_attention_heads": cfg.heads, "intermediate_size": cfg.ff,
           "layer_types": ["sliding_attention" if s else "full_attention" for s in cfg.sliding],
           "local_attention": 2 * cfg.window, "global_rope_theta": cfg.theta_global,
           "local_rope_theta": cfg.theta_local, "norm_eps": cfg.eps}
    agent = {"head_layers": cfg.head_layers, "type_emb": bool(cfg.type_emb),
             "temperature": list(temperature), "max_len": max_len,
             "head_max_len": min(192, max_len - 1)}
    if by_options:
        agent["temperature_by_options"] = by_options
    if cfg.act_out > 0:
        agent["act_costs"] = {f"a{i}": 1.0 for i in range(cfg.act_out - 1)}
    else:
        agent["act_head"] = False
    enc["laya_agent"] = agent
    enc["laya_tokens"] = {"cls_token": "[CLS]", "sep_token": {"content": "[SEP]"},
                          "mask_token": "[MASK]", "pad_token": "[PAD]"}
    enc["laya_special_ids"] = {"[CLS]": 1, "[SEP]": 2, "[MASK]": 3, "[PAD]": 4}
    return enc


def small(layers=3, window=4, head_layers=2, act_out=3, d=128, heads=2, ff=192, vocab=96):
    """A tiny model with 64-dim heads: global layer 0, local layers after
    (ModernBERT's every-third pattern)."""
    return O.OracleLayaConfig(vocab=vocab, d=d, layers=layers, heads=heads, ff=ff,
                              sliding=[int(l % 3 != 0) for l in range(layers)], window=window,
                              head_layers=head_layers, act_hidden=256, act_out=act_out)


class LayaModel:
    """A seeded checkpoint: engine QTensors and oracle f32 tensors."""

    def __init__(self, cfg: O.OracleLayaConfig, seed: int, linear: int, embed: int, **js):
        from grande_b200.engine import Dtype, QTensor

        self.cfg = cfg
        self.config = config_json(cfg, **js)
        self.qtensors = {}
        self.f32 = []
        self.host = {}
        for (name, shape), v in zip(cfg.tensors(), laya_weights(cfg, seed)):
            n = int(np.prod(shape))
            host = name.startswith("scorer.") or name.startswith("act.")
            if name == "embed":
                dt = embed
            elif len(shape) == 2 and not host and name != "type_emb":
                dt = linear
            else:
                dt = O.F16
            data, scales = O.quantize(dt, v)
            self.qtensors[name] = QTensor(Dtype(dt), list(shape), data, scales)
            f = O.dequantize(dt, data, scales, n).reshape(shape)
            self.f32.append(f)
            if host:
                self.host[name] = f

    def engine(self, capacity=2048, max_rows=256, device=0):
        from grande_b200.laya import LayaEngine

        return LayaEngine.new(self.qtensors, json.dumps(self.config), capacity, max_rows, device)

    def hidden(self, seqs, mode=O.ORACLE_KERNEL) -> np.ndarray:
        ids, pos, seq, qt = O.laya_pack([(s.ids, s.qtype) for s in seqs])
        return O.laya_hidden(self.cfg, self.f32, ids, pos, seq, qt, mode)

    def rows(self, seqs, x: np.ndarray) -> list:
        """[CLS] + marker rows of each sequence out of the oracle's x."""
        out, start = [], 0
        for s in seqs:
            idx = [start] + [start + m for m in s.markers]
            out.append(x[idx])
            start += len(s.ids)
        return out
