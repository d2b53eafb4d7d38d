"""Generate the golden fixtures that pin the oracle to the reference.

Run in a container that has the reference checkout (read-only) mounted:

    python tests/golden/make_golden.py --reference /path/to/bokuweb-grande

It imports the reference's own Python code and writes small .npz fixtures
next to this script; the tests read only the fixtures (the GPU box has no
reference checkout):

* quant_q8.npz / quant_q4.npz — Q8_0 / Q4_0 codes and scales of seeded
  values as the reference's exporter (tools/export_wgpu_gguf.py, `Writer.quant`)
  lays out the GGUF blocks that gguf-py 0.19 (`gguf.quants.quantize`, the
  llama.cpp reference quantizer the engine's `QTensor::quantize_*`
  restates, crates/omg-wgpu/src/model.rs:409-466) produces.
* branch_mask.npz — the reference's block-causal mask
  (python/omg_train/model.py:16-32, `branch_mask`) for several packings.
* gemma3_*.npz — a seeded tiny Gemma 3 model run through transformers 5.5's
  Gemma3TextModel with the reference's branch_mask and explicit position ids,
  as python/omg_train/model.py:67-80 (`DecisionModel.hidden`) drives it:
  the final-norm hidden state of every token.
"""
from __future__ import annotations

import argparse
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402  (the xorshift generator only)


def quant_fixtures(ref: Path):
    sys.path.insert(0, str(ref / "tools"))
    import export_wgpu_gguf as ex  # the reference exporter
    from gguf.constants import GGMLQuantizationType as T
    from gguf.quants import quantize

    rng = np.random.default_rng(0)
    cases = []
    cases.append(O.Rng(5).values(256, 0.3))  # tests/reference.rs:600-610 input
    cases.append((rng.standard_normal(32 * 64) * 0.02).astype(np.float32))
    cases.append(O.Rng(7 | 1).values(32 * 40, 0.15))
    edge = np.zeros(32 * 6, np.float32)
    edge[32:64] = 0.5 * np.sign(rng.standard_normal(32))  # ties in |max|
    edge[64:96] = np.linspace(-1, 1, 32)
    edge[96:128] = -np.arange(32, dtype=np.float32) / 31.0 * 7.25
    edge[128:160] = (np.arange(32) - 16) / 16.0 * 3.0  # codes at rounding midpoints
    edge[160:192] = rng.standard_normal(32).astype(np.float32) * 1e3
    cases.append(edge)
    values = np.concatenate(cases).astype(np.float32)
    for kind, name, bb in ((T.Q8_0, "q8", 34), (T.Q4_0, "q4", 18)):
        blocks = quantize(values.reshape(-1, 32), kind).reshape(-1, bb)
        with tempfile.TemporaryDirectory() as td:
            w = ex.Writer(Path(td) / "t.bin")
            w.quant("t", kind, blocks, [values.size // 32, 32])
            entry = w.close()["tensors"][0]
            raw = (Path(td) / "t.bin").read_bytes()
        codes = np.frombuffer(raw[entry["offset"]:entry["offset"] + entry["nbytes"]], np.uint8)
        scales = np.frombuffer(
            raw[entry["scales_offset"]:entry["scales_offset"] + entry["scales_nbytes"]], np.uint8)
        np.savez_compressed(HERE / f"quant_{name}.npz", values=values, codes=codes,
                            scales=scales, dtype=entry["dtype"])
        print(f"quant_{name}.npz: {values.size} values")


def mask_fixtures(ref: Path):
    sys.path.insert(0, str(ref / "python"))
    import torch
    from omg_train.model import branch_mask

    layouts = {
        "single": [0] * 7 + [1] * 5,
        "two": [0] * 10 + [1] * 5 + [2] * 8,
        "three": [0] * 4 + [1] * 3 + [2] * 4 + [3] * 2,
        "noprefix": [1] * 3 + [2] * 4,
    }
    out = {}
    for name, seg in layouts.items():
        for window in (None, 3, 6):
            m = branch_mask([seg], torch.device("cpu"), window)[0, 0]
            out[f"{name}_w{window or 0}"] = (m == 0).numpy()
        out[f"{name}_seg"] = np.array(seg, np.int32)
    np.savez_compressed(HERE / "branch_mask.npz", **out)
    print(f"branch_mask.npz: {len(layouts)} layouts")


def gemma3_fixture(ref: Path, name: str, window: int, prefix, branches, seed: int):
    sys.path.insert(0, str(ref / "python"))
    import torch
    from omg_train.model import branch_mask
    from transformers import Gemma3TextConfig, Gemma3TextModel

    layers, d, heads, kvh, hd, ff, vocab = 3, 64, 2, 1, 256, 96, 40
    types = ["sliding_attention", "full_attention", "sliding_attention"]
    hf = Gemma3TextConfig(
        vocab_size=vocab, hidden_size=d, intermediate_size=ff, num_hidden_layers=layers,
        num_attention_heads=heads, num_key_value_heads=kvh, head_dim=hd,
        query_pre_attn_scalar=256, sliding_window=window, layer_types=types,
        rms_norm_eps=1e-6, hidden_activation="gelu_pytorch_tanh",
        rope_parameters={"sliding_attention": {"rope_type": "default", "rope_theta": 1e4},
                         "full_attention": {"rope_type": "default", "rope_theta": 1e6}},
        attn_implementation="eager")
    model = Gemma3TextModel(hf).float().eval()
    # Seeded weights rounded to f16 (the checkpoint dtype the engine loads),
    # generated like tests/reference.rs:108-139 (norms around 0: Gemma 3
    # applies 1 + w).
    r = O.Rng(seed | 1)
    f16 = lambda a: O.f16_bits_to_f32(O.f32_to_f16_bits(a))  # noqa: E731
    tensors = {}
    assigned = set()
    sd = dict(model.named_parameters())

    def put(key, name, shape, scale, base=0.0):
        v = f16(r.values(int(np.prod(shape)), scale) + base).reshape(shape)
        sd[key].data.copy_(torch.from_numpy(v))
        assigned.add(key)
        tensors[name] = v

    put("embed_tokens.weight", "embed", [vocab, d], 1.0)
    put("norm.weight", "final_norm", [d], 0.5)
    for l in range(layers):
        p = f"layers.{l}."
        put(p + "input_layernorm.weight", f"blk.{l}.attn_norm", [d], 0.5)
        q = f16(r.values(heads * hd * d, 0.15)).reshape(heads * hd, d)
        k = f16(r.values(kvh * hd * d, 0.15)).reshape(kvh * hd, d)
        v = f16(r.values(kvh * hd * d, 0.15)).reshape(kvh * hd, d)
        for key, val in (("q_proj", q), ("k_proj", k), ("v_proj", v)):
            sd[p + f"self_attn.{key}.weight"].data.copy_(torch.from_numpy(val))
            assigned.add(p + f"self_attn.{key}.weight")
        tensors[f"blk.{l}.qkv"] = np.concatenate([q, k, v])
        put(p + "self_attn.q_norm.weight", f"blk.{l}.q_norm", [hd], 0.5)
        put(p + "self_attn.k_norm.weight", f"blk.{l}.k_norm", [hd], 0.5)
        put(p + "self_attn.o_proj.weight", f"blk.{l}.o", [d, heads * hd], 0.08)
        put(p + "post_attention_layernorm.weight", f"blk.{l}.post_attn_norm", [d], 0.5)
        put(p + "pre_feedforward_layernorm.weight", f"blk.{l}.ffn_norm", [d], 0.5)
        put(p + "mlp.gate_proj.weight", f"blk.{l}.gate", [ff, d], 0.15)
        put(p + "mlp.up_proj.weight", f"blk.{l}.up", [ff, d], 0.15)
        put(p + "mlp.down_proj.weight", f"blk.{l}.down", [d, ff], 0.08)
        put(p + "post_feedforward_layernorm.weight", f"blk.{l}.post_ffn_norm", [d], 0.5)
    assert assigned == set(sd), sorted(set(sd) - assigned)

    ids, pos, seg = [], [], []
    for i, t in enumerate(prefix):
        ids.append(t), pos.append(i), seg.append(0)
    for bi, toks in enumerate(branches):
        for j, t in enumerate(toks):
            ids.append(t), pos.append(len(prefix) + j), seg.append(bi + 1)
    dev = torch.device("cpu")
    mask = {"full_attention": branch_mask([seg], dev),
            "sliding_attention": branch_mask([seg], dev, window)}
    with torch.no_grad():
        hid = model(input_ids=torch.tensor([ids]), position_ids=torch.tensor([pos]),
                    attention_mask=mask).last_hidden_state[0].numpy()
    config = {
        "model_type": "gemma3_text", "vocab_size": vocab, "hidden_size": d,
        "num_hidden_layers": layers, "num_attention_heads": heads, "num_key_value_heads": kvh,
        "head_dim": hd, "intermediate_size": ff, "layer_types": types,
        "sliding_window": window, "rms_norm_eps": 1e-6, "query_pre_attn_scalar": 256,
        "rope_parameters": hf.rope_parameters,
    }
    np.savez_compressed(
        HERE / f"gemma3_{name}.npz", config=json.dumps(config),
        names=np.array(list(tensors)), ids=np.array(ids, np.uint32),
        pos=np.array(pos, np.int32), seg=np.array(seg, np.int32), hidden=hid.astype(np.float32),
        **{f"t:{k}": O.f32_to_f16_bits(v) for k, v in tensors.items()})
    print(f"gemma3_{name}.npz: {len(ids)} tokens")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference checkout (read-only)")
    a = ap.parse_args()
    ref = Path(a.reference)
    quant_fixtures(ref)
    mask_fixtures(ref)
    # One branch: token index == position, so the reference mask's
    # index-based window equals the engine's position-based one.
    gemma3_fixture(ref, "sliding", 6, [2, 5, 9, 14, 20, 31, 7, 8, 3, 22], [[11, 12, 13, 14, 15, 16]], 7)
    # Several branches with a window wider than the pass: branch isolation.
    gemma3_fixture(ref, "branches", 512, [2, 5, 9, 14, 20, 31, 7, 8, 3, 22],
                   [[11, 12, 13, 14, 15], [30, 31, 32, 33, 34, 35, 36, 37], [4, 6]], 11)


if __name__ == "__main__":
    main()
