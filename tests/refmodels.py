"""The reference's test models (crates/omg-wgpu/tests/reference.rs:40-139) as
HF-style config.json text for the engine plus an oracle config, and the
seeded weight generator `weights()` (:108-139) built on the oracle's
xorshift and quantizers. Test infrastructure."""
from __future__ import annotations

import json

import numpy as np

from grande_b200.engine import Dtype, QTensor
from oracle import oracle as O


def gemma3():
    """reference.rs:40-65."""
    cfg = O.OracleConfig(vocab=40, d=64, layers=3, heads=2, kv_heads=1, head_dim=[256] * 3,
                         ff=[96] * 3, sliding=[True, False, True], kv_source=[0, 1, 2],
                         rope_dims=[256] * 3, eps=1e-6, window=6, theta_global=1e6,
                         theta_local=1e4, query_scale=256 ** -0.5, norm_offset=1.0,
                         v_norm=False, per_layer_dim=0, softcap=0.0)
    js = {"model_type": "gemma3_text", "vocab_size": 40, "hidden_size": 64,
          "num_hidden_layers": 3, "num_attention_heads": 2, "num_key_value_heads": 1,
          "head_dim": 256, "intermediate_size": 96, "sliding_window": 6,
          "layer_types": ["sliding_attention", "full_attention", "sliding_attention"],
          "rope_parameters": {"full_attention": {"rope_theta": 1e6},
                              "sliding_attention": {"rope_theta": 1e4}},
          "query_pre_attn_scalar": 256, "rms_norm_eps": 1e-6}
    return cfg, json.dumps(js)


def gemma4(heads=4, kv_heads=1):
    """reference.rs:69-94 (and :98-104 with 8 / 2 heads)."""
    cfg = O.OracleConfig(vocab=64, d=64, layers=4, heads=heads, kv_heads=kv_heads,
                         head_dim=[256, 512, 256, 512], ff=[96, 96, 192, 192],
                         sliding=[True, False, True, False], kv_source=[0, 1, 0, 1],
                         rope_dims=[256, 128, 256, 128], eps=1e-6, window=5, theta_global=1e6,
                         theta_local=1e4, query_scale=1.0, norm_offset=0.0, v_norm=True,
                         per_layer_dim=32, softcap=30.0)
    js = {"model_type": "gemma4_text", "vocab_size": 64, "hidden_size": 64,
          "num_hidden_layers": 4, "num_attention_heads": heads, "num_key_value_heads": kv_heads,
          "head_dim": 256, "global_head_dim": 512, "intermediate_size": 96,
          "use_double_wide_mlp": True, "num_kv_shared_layers": 2, "sliding_window": 5,
          "layer_types": ["sliding_attention", "full_attention"] * 2,
          "rope_parameters": {"full_attention": {"rope_theta": 1e6, "partial_rotary_factor": 0.25},
                              "sliding_attention": {"rope_theta": 1e4}},
          "hidden_size_per_layer_input": 32, "final_logit_softcapping": 30.0,
          "rms_norm_eps": 1e-6}
    return cfg, json.dumps(js)


def gemma4_gqa():
    return gemma4(heads=8, kv_heads=2)


class RefModel:
    """weights() of reference.rs:108-139: the engine's QTensors, the oracle's
    dequantized tensors (catalogue order), and the per-layer table."""

    def __init__(self, cfg: O.OracleConfig, config_json: str, seed: int, linear: int, embed: int):
        self.cfg = cfg
        self.config_json = config_json
        r = O.Rng(seed | 1)
        self.qtensors: dict[str, QTensor] = {}
        self.f32: list[np.ndarray] = []
        base = np.float32(1.0 if cfg.norm_offset == 0.0 else 0.0)
        for name, shape in cfg.tensors():
            n = int(np.prod(shape))
            if name == "embed":
                dt, v = embed, r.values(n, 1.0)
            elif name.endswith("out_scale"):
                dt, v = O.F16, np.array([np.float32(0.6) + np.float32(0.2) * np.float32(r.next())],
                                        np.float32)
            elif len(shape) == 1:
                dt, v = O.F16, (r.values(n, 0.5) + base).astype(np.float32)
            else:
                scale = 0.15 if shape[1] == cfg.d else 0.08
                dt, v = linear, r.values(n, scale)
            self._add(name, shape, dt, v)
        self.per_layer_table = None
        if cfg.per_layer_dim > 0:
            shape = [cfg.vocab, cfg.per_layer_dim * cfg.layers]
            v = r.values(int(np.prod(shape)), 1.0)
            data, scales = O.quantize(linear, v)
            self.per_layer_table = QTensor(Dtype(linear), shape, data, scales)
            self.f32.append(O.dequantize(linear, data, scales, v.size))

    def _add(self, name, shape, dt, v):
        data, scales = O.quantize(dt, v)
        self.qtensors[name] = QTensor(Dtype(dt), list(shape), data, scales)
        self.f32.append(O.dequantize(dt, data, scales, v.size))

    def tensor_f32(self, name: str) -> np.ndarray:
        names = [n for n, _ in self.cfg.tensors()]
        return self.f32[names.index(name)]

    def engine(self, capacity=64, max_rows=16, device=0):
        from grande_b200.engine import Engine
        return Engine.new(self.qtensors, self.config_json, capacity, max_rows, device,
                          self.per_layer_table)

    def hidden(self, ids, pos, seq, mode=O.ORACLE_EXACT):
        return O.forward(self.cfg, self.f32, ids, pos, seq, mode)
