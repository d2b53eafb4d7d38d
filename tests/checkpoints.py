"""Writers for the two on-disk model formats the loader reads, for tests:
a safetensors file (the published format: an 8-byte little-endian header
length, a JSON header of name -> dtype / shape / data_offsets, the payload)
and an exported directory laid out as tools/export_wgpu_gguf.py:46-96 writes
it (per tensor the f16 block scales, then the codes, each run padded to 4
bytes; one file for the embedding tables, one per layer, the per-layer
token table in its own file). Test infrastructure."""
from __future__ import annotations

import json
import re
from pathlib import Path

import numpy as np


def f32_to_bf16_bits(v: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even truncation of f32 to bf16 (no NaNs here)."""
    u = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def write_safetensors(path: Path, tensors: dict):
    """``tensors``: name -> (dtype, shape, raw little-endian bytes)."""
    header, blobs, off = {}, [], 0
    for name, (dtype, shape, raw) in tensors.items():
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    Path(path).write_bytes(len(h).to_bytes(8, "little") + h + b"".join(blobs))


def hf_name(name: str) -> list:
    """The HF names of one catalogue tensor of a Gemma 3 model (qkv is three)."""
    if name == "embed":
        return ["embed_tokens.weight"]
    if name == "final_norm":
        return ["norm.weight"]
    m = re.fullmatch(r"blk\.(\d+)\.(\w+)", name)
    i, t = m.group(1), m.group(2)
    sub = {"attn_norm": "input_layernorm", "q_norm": "self_attn.q_norm",
           "k_norm": "self_attn.k_norm", "o": "self_attn.o_proj",
           "post_attn_norm": "post_attention_layernorm", "ffn_norm": "pre_feedforward_layernorm",
           "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj",
           "post_ffn_norm": "post_feedforward_layernorm"}
    if t == "qkv":
        return [f"layers.{i}.self_attn.{p}_proj.weight" for p in "qkv"]
    return [f"layers.{i}.{sub[t]}.weight"]


class Exporter:
    """One tensor file of an exported directory and its manifest entries."""

    def __init__(self, path: Path):
        self.path = Path(path)
        self.buf = bytearray()
        self.entries = []

    def _put(self, b: bytes):
        off = len(self.buf)
        self.buf += b
        self.buf += b"\0" * (-len(self.buf) % 4)
        return off, len(b)

    def add(self, name: str, t) -> dict:
        dtype = {0: "f16", 1: "q8", 2: "q4"}[int(t.dtype)]
        e = {"name": name, "dtype": dtype, "shape": list(t.shape)}
        if t.scales:
            e["scales_offset"], e["scales_nbytes"] = self._put(t.scales)
        e["offset"], e["nbytes"] = self._put(t.data)
        self.entries.append(e)
        return e

    def close(self) -> dict:
        self.path.write_bytes(bytes(self.buf))
        return {"path": self.path.name, "tensors": self.entries}


def write_export(dir: Path, config_json: str, tensors: dict, per_layer_table=None) -> dict:
    """An exported directory of ``tensors`` (catalogue name -> QTensor);
    returns the manifest it wrote."""
    dir = Path(dir)
    dir.mkdir(parents=True, exist_ok=True)
    (dir / "config.json").write_text(config_json)
    files = {}
    for name, t in tensors.items():
        m = re.match(r"blk\.(\d+)\.", name)
        fname = f"blk.{m.group(1)}.bin" if m else "embed.bin"
        files.setdefault(fname, Exporter(dir / fname)).add(name, t)
    manifest = {"files": [f.close() for f in files.values()]}
    if per_layer_table is not None:
        ex = Exporter(dir / "per_layer_table.bin")
        e = ex.add("per_layer_table", per_layer_table)
        ex.close()
        e["path"] = "per_layer_table.bin"
        manifest["per_layer_table"] = e
    (dir / "manifest.json").write_text(json.dumps(manifest, indent=1))
    return manifest
