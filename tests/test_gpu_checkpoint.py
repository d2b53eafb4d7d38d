"""Engines loaded from model directories (WgpuBackend::load,
crates/omg-wgpu/src/backend.rs:25-63) against engines built from the same
tensors in memory: a Gemma 3 HF safetensors checkpoint (the golden fixture
of tests/golden/make_golden.py, also checked against transformers' hidden
rows) and an exported Gemma 4 directory with Q4_0/Q8_0 tensors and the
per-layer token table (tools/export_wgpu_gguf.py layout)."""
import json

import numpy as np
import pytest

from checkpoints import write_export, write_safetensors
from grande_b200 import checkpoint as ck
from grande_b200._lib import OmgError
from grande_b200.engine import B200Backend, BranchTokens, Dtype, Engine, QTensor, Want
from oracle import oracle as O
from refmodels import RefModel, gemma4
from test_checkpoint import GOLDEN, hf_tensors

pytestmark = pytest.mark.gpu


def test_gemma3_safetensors_directory(tmp_path, device):
    g = np.load(GOLDEN / "gemma3_branches.npz")
    cfg = str(g["config"])
    bits = {k[2:]: g[k] for k in g.files if k.startswith("t:")}
    (tmp_path / "config.json").write_text(cfg)
    write_safetensors(tmp_path / "model.safetensors", hf_tensors(cfg, bits))
    backend = B200Backend.load(tmp_path, 64, 16, device)
    loaded = backend.engine
    direct = Engine.new({n: QTensor(Dtype.F16, list(b.shape), b.tobytes(), b"")
                         for n, b in bits.items()}, cfg, 64, 16, device)
    seg, ids = g["seg"], g["ids"]
    prefix = [int(i) for i, s in zip(ids, seg) if s == 0]
    branches, idx = [], []
    for b in sorted(set(int(s) for s in seg if s > 0)):
        toks = [int(i) for i, s in zip(ids, seg) if s == b]
        branches.append(BranchTokens(toks, list(range(len(toks)))))
        idx += [k for k, s in enumerate(seg) if s == b]
    got = loaded.evaluate(prefix, branches, Want.HIDDEN)
    exp = direct.evaluate(prefix, branches, Want.HIDDEN)
    for a, b in zip(got, exp):
        assert np.array_equal(a.rows, b.rows)
    rows = np.concatenate([o.rows for o in got])
    ref = g["hidden"][idx]
    scale = np.maximum(np.abs(ref).max(axis=1, keepdims=True), 1.0)
    assert (np.abs(rows - ref) / scale).max() < 2e-2
    la = loaded.evaluate(prefix, branches, Want.LOGITS)
    lb = direct.evaluate(prefix, branches, Want.LOGITS)
    for a, b in zip(la, lb):
        assert np.array_equal(a.rows, b.rows)
    loaded.close()
    direct.close()


def test_exported_gemma4_directory(tmp_path, device):
    m = RefModel(*gemma4(), 17, O.Q4, O.Q8)
    d = tmp_path / "gemma4-tiny-wgpu"
    write_export(d, m.config_json, m.qtensors, m.per_layer_table)
    loaded = ck.load_engine(d, 64, 16, device)
    direct = m.engine(64, 16, device)
    prefix = [2, 7, 11, 19, 23, 31, 40, 41]
    branches = [BranchTokens([5, 6, 9], [0, 2]), BranchTokens([50, 51], [1])]
    for want in (Want.HIDDEN, Want.LOGITS):
        for a, b in zip(loaded.evaluate(prefix, branches, want),
                        direct.evaluate(prefix, branches, want)):
            assert np.array_equal(a.rows, b.rows)
    # The state cache's model id is the directory's name and tensor bytes.
    size = sum(p.stat().st_size for p in d.glob("*.bin"))
    assert ck.model_id(d) == f"gemma4-tiny-wgpu:{size}"
    B200Backend(loaded).set_state_cache(d, 1 << 20, None)
    state = loaded.save_state(prefix)
    blob = state.to_bytes(ck.model_id(d))
    with pytest.raises(OmgError, match="state file is for a different model"):
        type(state).from_bytes(blob, "another-model:1")
    loaded.evict_resident()
    loaded.restore_state(type(state).from_bytes(blob, ck.model_id(d)))
    for a, b in zip(loaded.evaluate(prefix, branches, Want.LOGITS),
                    direct.evaluate(prefix, branches, Want.LOGITS)):
        assert np.array_equal(a.rows, b.rows)
    loaded.close()
    direct.close()


def test_exported_directory_errors(tmp_path, device):
    m = RefModel(*gemma4(), 5, O.Q8, O.Q8)
    manifest = write_export(tmp_path, m.config_json, m.qtensors, m.per_layer_table)
    # The per-layer table entry must name its file.
    broken = json.loads(json.dumps(manifest))
    del broken["per_layer_table"]["path"]
    (tmp_path / "manifest.json").write_text(json.dumps(broken))
    with pytest.raises(OmgError, match="^manifest: per_layer_table has no path$"):
        ck.load_engine(tmp_path, 64, 16, device)
    # A tensor the builder rejects is reported with its file and name.
    broken = json.loads(json.dumps(manifest))
    f = next(f for f in broken["files"] if f["path"] == "blk.0.bin")
    e = next(e for e in f["tensors"] if e["name"] == "blk.0.o")
    e["shape"] = [e["shape"][1], e["shape"][0]]
    (tmp_path / "manifest.json").write_text(json.dumps(broken))
    with pytest.raises(OmgError, match=r"^blk\.0\.bin: blk\.0\.o: "):
        ck.load_engine(tmp_path, 64, 16, device)
    # A missing tensor file.
    (tmp_path / "manifest.json").write_text(json.dumps(manifest))
    (tmp_path / "blk.2.bin").unlink()
    with pytest.raises(OmgError, match=r"^reading .*blk\.2\.bin"):
        ck.load_engine(tmp_path, 64, 16, device)
