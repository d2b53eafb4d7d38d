"""Model directories on disk, as the reference's native backend loads them
(crates/omg-wgpu/src/backend.rs:25-63, ``WgpuBackend::load``):

* an exported directory (tools/export_wgpu_gguf.py:1-80): ``config.json``,
  ``manifest.json`` and the tensor files it names. Each entry is an encoded
  ``QTensor``: a byte range of codes plus, for Q8_0/Q4_0, a separate byte
  range of f16 block scales (``Manifest``, model.rs:742-795). The per-layer
  token table of Gemma 4 is its own entry with its own file;
* a Hugging Face Gemma 3 checkpoint: ``config.json`` + ``model.safetensors``
  with F32/F16/BF16 tensors, converted to f16 and renamed to the engine's
  catalogue, q/k/v stacked into one ``qkv`` (``Weights::load``,
  model.rs:556-617; ``SafeTensors``, model.rs:655-740).

Error messages are the reference's. The tokenizer files of a directory are
not read here: tokenization stays with the caller (omg-core).
"""
from __future__ import annotations

import json
import mmap
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import numpy as np

from ._lib import OmgError
from .engine import Dtype, Engine, EngineBuilder, QTensor, config_tensors


def _read(dir: Path, name: str) -> bytes:
    """backend.rs:29-32: a file of the directory, with its path on failure."""
    p = dir / name
    try:
        return p.read_bytes()
    except OSError as e:
        raise OmgError(f"reading {p}: {e}") from e


def _map(dir: Path, name: str) -> memoryview:
    """A read-only view of a (large) tensor file without reading it all into
    memory first; slices of it become the tensors' own bytes."""
    p = dir / name
    try:
        with open(p, "rb") as f:
            if os.fstat(f.fileno()).st_size == 0:
                return memoryview(b"")
            return memoryview(mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ))
    except OSError as e:
        raise OmgError(f"reading {p}: {e}") from e


def text_config(config: dict) -> dict:
    """Config::from_json (model.rs:66-71): HF multimodal configs nest the
    text model under ``text_config``."""
    return config["text_config"] if "text_config" in config else config


def is_gemma4(config: dict) -> bool:
    """model.rs:72-75: ``model_type`` gemma4_text / gemma4, else Gemma 3."""
    return text_config(config).get("model_type", "gemma3_text") in ("gemma4_text", "gemma4")


# --- safetensors ---------------------------------------------------------


class SafeTensors:
    """model.rs:655-726: the minimal safetensors reader. ``tensor`` returns
    the shape and the values as f16 bits: F16 as stored, F32 and BF16
    rounded to nearest even (``f16::from_f32``)."""

    def __init__(self, header: dict, data: memoryview):
        self.header = header
        self.data = data

    @staticmethod
    def parse(raw) -> "SafeTensors":
        raw = memoryview(raw)
        if len(raw) < 8:
            raise OmgError("safetensors: too short")
        n = int.from_bytes(raw[:8], "little")
        if 8 + n > len(raw):
            raise OmgError("safetensors: header out of range")
        try:
            header = json.loads(bytes(raw[8:8 + n]))
        except ValueError as e:
            raise OmgError(f"safetensors header: {e}") from e
        if not isinstance(header, dict):
            raise OmgError("safetensors header: not an object")
        return SafeTensors(header, raw[8 + n:])

    def tensor(self, name: str) -> tuple[list, np.ndarray]:
        t = self.header.get(name)
        if t is None:
            raise OmgError(f"safetensors: missing {name}")
        shape = t.get("shape") if isinstance(t, dict) else None
        if not isinstance(shape, list):
            raise OmgError(f"{name}: shape")
        shape = [int(v) if isinstance(v, int) and v >= 0 else 0 for v in shape]
        off = t.get("data_offsets")
        if not isinstance(off, list) or len(off) < 2:
            raise OmgError(f"{name}: data_offsets")
        a, b = (int(v) if isinstance(v, int) and v >= 0 else 0 for v in off[:2])
        if a > b or b > len(self.data):
            raise OmgError(f"{name}: offsets out of range")
        raw = self.data[a:b]
        dtype = t.get("dtype", "")
        with np.errstate(over="ignore"):  # out-of-range values become infinities
            bits = self._f16_bits(name, dtype, raw)
        if bits.size != int(np.prod(shape)):
            raise OmgError(f"{name}: {bits.size} values for shape {shape}")
        return shape, bits

    @staticmethod
    def _f16_bits(name: str, dtype: str, raw: memoryview) -> np.ndarray:
        if dtype == "F32":
            v = np.frombuffer(raw, dtype="<f4", count=len(raw) // 4)
            bits = v.astype(np.float16).view(np.uint16)
        elif dtype == "F16":
            bits = np.frombuffer(raw, dtype="<u2", count=len(raw) // 2).copy()
        elif dtype == "BF16":
            hi = np.frombuffer(raw, dtype="<u2", count=len(raw) // 2).astype(np.uint32) << 16
            bits = hi.view(np.float32).astype(np.float16).view(np.uint16)
        else:
            raise OmgError(f"{name}: unsupported dtype {dtype}")
        return bits


def _f16(shape, bits: np.ndarray) -> QTensor:
    """QTensor::from_f16 (model.rs:390-401)."""
    return QTensor(Dtype.F16, list(shape), np.ascontiguousarray(bits, dtype="<u2").tobytes(), b"")


def _concat_rows(parts) -> tuple[list, np.ndarray]:
    """model.rs:728-740: stack 2-D tensors along rows."""
    cols = parts[0][0][1]
    for shape, _ in parts:
        if len(shape) != 2 or shape[1] != cols:
            raise OmgError(f"cannot stack rows of shapes {[p[0] for p in parts]}")
    return [sum(s[0] for s, _ in parts), cols], np.concatenate([b for _, b in parts])


def check_weights(config_json: str, tensors: dict, per_layer_table: Optional[QTensor]):
    """Weights::check (model.rs:619-645): every catalogued tensor present
    with the right shape, and the per-layer table when the model has one."""
    for name, shape in config_tensors(config_json):
        t = tensors.get(name)
        if t is None:
            raise OmgError(f"missing tensor {name}")
        if list(t.shape) != list(shape):
            raise OmgError(f"{name}: shape {list(t.shape)}, expected {list(shape)}")
    cfg = text_config(json.loads(config_json))
    pld = int(cfg.get("hidden_size_per_layer_input") or 0)
    if pld > 0:
        if per_layer_table is None:
            raise OmgError("missing per-layer token table")
        want = [int(cfg["vocab_size"]), pld * int(cfg["num_hidden_layers"])]
        if list(per_layer_table.shape) != want:
            raise OmgError(f"per-layer table: shape {list(per_layer_table.shape)}, expected {want}")


def gemma3_weights(config_json, safetensors) -> dict:
    """Weights::load (model.rs:556-617): a Gemma 3 HF checkpoint as the
    engine's catalogue of f16 tensors."""
    if isinstance(config_json, (bytes, bytearray)):
        config_json = config_json.decode()
    try:
        config = json.loads(config_json)
    except ValueError as e:
        raise OmgError(f"config.json: {e}") from e
    # Config::from_json + validate: a bad config fails before the tensors
    # are read.
    config_tensors(config_json)
    if is_gemma4(config):
        raise OmgError("safetensors loading is for Gemma 3 checkpoints; "
                       "export Gemma 4 with tools/export_wgpu_gguf.py")
    cfg = text_config(config)
    vocab, d = int(cfg["vocab_size"]), int(cfg["hidden_size"])
    layers = int(cfg["num_hidden_layers"])
    st = SafeTensors.parse(safetensors)
    # Checkpoints may or may not carry the `model.` prefix.
    prefix = "model." if "model.embed_tokens.weight" in st.header else ""

    def get(name):
        return st.tensor(prefix + name)

    out = {}
    embed = get("embed_tokens.weight")
    if embed[0] != [vocab, d]:
        raise OmgError(f"embed_tokens is {embed[0]}, config says [{vocab}, {d}]")
    out["embed"] = _f16(*embed)
    out["final_norm"] = _f16(*get("norm.weight"))
    for i in range(layers):
        def l(n):
            return get(f"layers.{i}.{n}")
        blk = f"blk.{i}."
        out[blk + "attn_norm"] = _f16(*l("input_layernorm.weight"))
        out[blk + "qkv"] = _f16(*_concat_rows([l("self_attn.q_proj.weight"),
                                               l("self_attn.k_proj.weight"),
                                               l("self_attn.v_proj.weight")]))
        out[blk + "q_norm"] = _f16(*l("self_attn.q_norm.weight"))
        out[blk + "k_norm"] = _f16(*l("self_attn.k_norm.weight"))
        out[blk + "o"] = _f16(*l("self_attn.o_proj.weight"))
        out[blk + "post_attn_norm"] = _f16(*l("post_attention_layernorm.weight"))
        out[blk + "ffn_norm"] = _f16(*l("pre_feedforward_layernorm.weight"))
        out[blk + "gate"] = _f16(*l("mlp.gate_proj.weight"))
        out[blk + "up"] = _f16(*l("mlp.up_proj.weight"))
        out[blk + "down"] = _f16(*l("mlp.down_proj.weight"))
        out[blk + "post_ffn_norm"] = _f16(*l("post_feedforward_layernorm.weight"))
    check_weights(config_json, out, None)
    return out


# --- exported directory ----------------------------------------------------


@dataclass
class ManifestEntry:
    """model.rs:758-774: one encoded tensor of a file."""
    name: str
    dtype: str
    shape: list
    offset: int
    nbytes: int
    scales_offset: int = 0
    scales_nbytes: int = 0
    path: Optional[str] = None

    @staticmethod
    def from_json(v) -> "ManifestEntry":
        if not isinstance(v, dict):
            raise OmgError("manifest.json: tensor entry is not an object")
        try:
            return ManifestEntry(
                name=str(v["name"]), dtype=str(v["dtype"]), shape=[int(x) for x in v["shape"]],
                offset=int(v["offset"]), nbytes=int(v["nbytes"]),
                scales_offset=int(v.get("scales_offset", 0)),
                scales_nbytes=int(v.get("scales_nbytes", 0)),
                path=v.get("path"))
        except KeyError as e:
            raise OmgError(f"manifest.json: missing field `{e.args[0]}`") from e
        except (TypeError, ValueError) as e:
            raise OmgError(f"manifest.json: {e}") from e

    def tensor(self, file) -> QTensor:
        """ManifestEntry::tensor (model.rs:776-795): decode this entry out of
        its file's bytes."""
        def piece(off, n):
            if off < 0 or n < 0 or off + n > len(file):
                raise OmgError(f"{self.name}: byte range {off}..{off + n} outside the file")
            return bytes(file[off:off + n])
        return QTensor.from_raw(Dtype.parse(self.dtype), self.shape,
                                piece(self.offset, self.nbytes),
                                piece(self.scales_offset, self.scales_nbytes))


@dataclass
class ManifestFile:
    """model.rs:752-756."""
    path: str
    tensors: list


@dataclass
class Manifest:
    """model.rs:742-750: tensors grouped into files, plus the optional
    per-layer token table (its own file)."""
    files: list
    per_layer_table: Optional[ManifestEntry] = None

    @staticmethod
    def parse(raw) -> "Manifest":
        try:
            v = json.loads(raw)
        except ValueError as e:
            raise OmgError(f"manifest.json: {e}") from e
        if not isinstance(v, dict) or not isinstance(v.get("files"), list):
            raise OmgError("manifest.json: missing field `files`")
        files = []
        for f in v["files"]:
            if not isinstance(f, dict) or "path" not in f or not isinstance(f.get("tensors"), list):
                raise OmgError("manifest.json: a file needs `path` and `tensors`")
            files.append(ManifestFile(str(f["path"]),
                                      [ManifestEntry.from_json(t) for t in f["tensors"]]))
        plt = v.get("per_layer_table")
        return Manifest(files, ManifestEntry.from_json(plt) if plt is not None else None)


def load_engine(dir, capacity: int, max_rows: int, device: int = 0,
                warmup: bool = True) -> Engine:
    """WgpuBackend::load (backend.rs:25-63) without the tokenizer: build the
    engine from an exported directory (``manifest.json`` present) or from a
    Gemma 3 ``model.safetensors``, then warm it up. An exported directory is
    streamed file by file into the builder, so host memory holds one tensor
    file at a time."""
    dir = Path(dir)
    config_json = _read(dir, "config.json").decode()
    if (dir / "manifest.json").is_file():
        manifest = Manifest.parse(_read(dir, "manifest.json"))
        b = EngineBuilder(config_json, device)
        for f in manifest.files:
            data = _map(dir, f.path)
            try:
                for entry in f.tensors:
                    t = entry.tensor(data)
                    try:
                        b.push(entry.name, t)
                    except OmgError as e:
                        raise OmgError(f"{f.path}: {entry.name}: {e}") from e
            finally:
                _release(data)
        if manifest.per_layer_table is not None:
            entry = manifest.per_layer_table
            if not entry.path:
                raise OmgError("manifest: per_layer_table has no path")
            data = _map(dir, entry.path)
            try:
                b.set_per_layer_table(entry.tensor(data))
            finally:
                _release(data)
        engine = b.finish(capacity, max_rows)
    else:
        data = _map(dir, "model.safetensors")
        try:
            weights = gemma3_weights(config_json, data)
        finally:
            _release(data)
        engine = Engine.new(weights, config_json, capacity, max_rows, device)
    if warmup:
        # The state cache is off until set_state_cache, so warmup's
        # two-token prefix is never saved.
        engine.warmup()
    return engine


def _release(view: memoryview):
    obj = view.obj
    view.release()
    if isinstance(obj, mmap.mmap):
        try:
            obj.close()
        except BufferError:
            # Views of it are still alive (an exception's frames); the map
            # closes when they are collected.
            pass


def model_id(dir) -> str:
    """backend.rs:80-96: the state cache's model id, the directory's name and
    the byte size of its ``*.bin`` tensor files."""
    dir = Path(dir)
    size = 0
    try:
        for e in os.scandir(dir):
            if e.name.endswith(".bin") and len(e.name) > 4:
                try:
                    size += e.stat(follow_symlinks=False).st_size
                except OSError:
                    pass
    except OSError:
        size = 0
    return f"{dir.name or 'wgpu'}:{size}"
