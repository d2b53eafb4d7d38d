"""Generate the golden fixtures that pin the Laya encoder oracle.

    python tests/golden/make_golden_laya.py

The reference runs its Laya / ModernBERT encoder only on the GPU
(crates/omg-wgpu/src/laya.rs) and ships no CPU code or test for it. Its
checkpoints are a ModernBERT encoder (`encoder.*` weights, laya.rs:340-414)
plus a decision head made of PyTorch `nn.TransformerEncoderLayer`s
(`head.layers.{h}.self_attn.in_proj_weight`, `norm1`, `linear1`, ...). This
script runs the same seeded tiny model through transformers 5.5's
`ModernBertModel` (one sequence per call, explicit positions, no padding) and
through `torch.nn.TransformerEncoderLayer(norm_first=True, activation="relu")`
for the head, and stores the resulting residual stream of every token:

* laya_small.npz — x after the decision head (the rows laya.rs:1399-1409
  reads back) and x after the encoder + type embedding.

Two behaviours of the reference are carried over on purpose:

* the head's attention has no 1/sqrt(head_dim) query scale (laya.rs:1322-1327
  passes the in_proj output straight to attention_bi): torch scales, so the
  query rows of in_proj (weight and bias) are multiplied by sqrt(head_dim)
  before torch sees them, which cancels its scale;
* the type embedding is added after the final norm (laya.rs:1302-1311).

The weights are regenerated from tests/layamodels.py's `laya_weights`
(xorshift of tests/reference.rs:17-26, through oracle.Rng), so only the
outputs are stored.
"""
from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402  (config and catalogue only)

sys.path.insert(0, str(HERE.parent))
from layamodels import laya_weights  # noqa: E402  (the seeded weight generator)

SMALL = dict(vocab=61, d=64, layers=4, heads=2, ff=48, local_attention=8, eps=1e-5,
             head_layers=2, act_out=3, act_hidden=16, seed=11)
SEQS = [([1, 5, 9, 2, 40, 33, 7, 8, 12, 3, 3, 19, 60], 0),
        ([4, 17, 23, 1, 2], 2),
        ([9, 9, 30, 31, 32, 33, 34, 35, 36, 0, 50, 51, 52, 53, 54, 55, 56, 57, 58, 59], 1)]


def small_config(s=SMALL) -> O.OracleLayaConfig:
    # ModernBERT's default pattern: global attention every 3rd layer from 0.
    sliding = [int(l % 3 != 0) for l in range(s["layers"])]
    return O.OracleLayaConfig(vocab=s["vocab"], d=s["d"], layers=s["layers"], heads=s["heads"],
                              ff=s["ff"], sliding=sliding, window=s["local_attention"] // 2,
                              eps=s["eps"], head_layers=s["head_layers"],
                              act_hidden=s["act_hidden"], act_out=s["act_out"])


def _torch_reference(cfg: O.OracleLayaConfig, w: dict, seqs, theta_g=160000.0, theta_l=10000.0):
    import torch
    from transformers import ModernBertConfig, ModernBertModel

    d, L = cfg.d, cfg.layers
    hc = ModernBertConfig(
        vocab_size=cfg.vocab, hidden_size=d, intermediate_size=cfg.ff, num_hidden_layers=L,
        num_attention_heads=cfg.heads, hidden_activation="gelu", norm_eps=cfg.eps,
        norm_bias=False, attention_bias=False, mlp_bias=False,
        local_attention=2 * cfg.window, pad_token_id=0, bos_token_id=1, eos_token_id=2,
        cls_token_id=1, sep_token_id=2,
        layer_types=["sliding_attention" if s else "full_attention" for s in cfg.sliding],
        rope_parameters={"full_attention": {"rope_type": "default", "rope_theta": theta_g},
                         "sliding_attention": {"rope_type": "default", "rope_theta": theta_l}})
    hc._attn_implementation = "eager"
    m = ModernBertModel(hc).eval().float()
    sd = {"embeddings.tok_embeddings.weight": w["embed"],
          "embeddings.norm.weight": w["embed_norm"], "final_norm.weight": w["final_norm"]}
    for l in range(L):
        p = f"layers.{l}."
        if l > 0:
            sd[p + "attn_norm.weight"] = w[f"enc.{l}.attn_norm"]
        sd[p + "attn.Wqkv.weight"] = w[f"enc.{l}.qkv"]
        sd[p + "attn.Wo.weight"] = w[f"enc.{l}.o"]
        sd[p + "mlp_norm.weight"] = w[f"enc.{l}.mlp_norm"]
        sd[p + "mlp.Wi.weight"] = np.concatenate([w[f"enc.{l}.wi_val"], w[f"enc.{l}.wi_gate"]])
        sd[p + "mlp.Wo.weight"] = w[f"enc.{l}.wo"]
    missing, unexpected = m.load_state_dict({k: torch.tensor(v) for k, v in sd.items()},
                                            strict=False)
    assert not unexpected, unexpected
    assert all("rotary" in k or "inv_freq" in k for k in missing), missing

    hd = d // cfg.heads
    heads = []
    for h in range(cfg.head_layers):
        layer = torch.nn.TransformerEncoderLayer(d, cfg.heads, dim_feedforward=4 * d, dropout=0.0,
                                                 activation="relu", layer_norm_eps=cfg.eps,
                                                 batch_first=True, norm_first=True).eval()
        inw = w[f"head.{h}.in_proj"].copy()
        inb = w[f"head.{h}.in_proj_b"].copy()
        inw[:d] *= math.sqrt(hd)  # cancel torch's query scale (the reference has none)
        inb[:d] *= math.sqrt(hd)
        hsd = {"self_attn.in_proj_weight": inw, "self_attn.in_proj_bias": inb,
               "self_attn.out_proj.weight": w[f"head.{h}.out_proj"],
               "self_attn.out_proj.bias": w[f"head.{h}.out_proj_b"],
               "linear1.weight": w[f"head.{h}.l1"], "linear1.bias": w[f"head.{h}.l1_b"],
               "linear2.weight": w[f"head.{h}.l2"], "linear2.bias": w[f"head.{h}.l2_b"],
               "norm1.weight": w[f"head.{h}.norm1_w"], "norm1.bias": w[f"head.{h}.norm1_b"],
               "norm2.weight": w[f"head.{h}.norm2_w"], "norm2.bias": w[f"head.{h}.norm2_b"]}
        layer.load_state_dict({k: torch.tensor(v) for k, v in hsd.items()})
        heads.append(layer)

    enc_rows, head_rows = [], []
    with torch.no_grad():
        for ids, qtype in seqs:
            ii = torch.tensor([ids], dtype=torch.long)
            pos = torch.arange(len(ids))[None]
            x = m(input_ids=ii, position_ids=pos).last_hidden_state[0]
            x = x + torch.tensor(w["type_emb"][qtype])
            enc_rows.append(x.numpy().copy())
            y = x[None]
            for layer in heads:
                y = layer(y)
            head_rows.append(y[0].numpy().copy())
    return np.concatenate(enc_rows), np.concatenate(head_rows)


def main():
    cfg = small_config()
    ws = laya_weights(cfg, SMALL["seed"])
    w = {n: v for (n, _), v in zip(cfg.tensors(), ws)}
    enc, head = _torch_reference(cfg, w, SEQS)
    np.savez_compressed(HERE / "laya_small.npz", config=json.dumps(SMALL),
                        seqs=json.dumps(SEQS), x_encoder=enc.astype(np.float32),
                        x_head=head.astype(np.float32))
    print("laya_small.npz:", enc.shape, head.shape)


if __name__ == "__main__":
    main()
