"""CPU tests of the Laya encoder path: the oracle pinned to HF ModernBERT +
torch's TransformerEncoderLayer (tests/golden/laya_small.npz, made by
tests/golden/make_golden_laya.py), and the engine's config parsing and
tensor catalogue against crates/omg-wgpu/src/laya.rs:88-309 (no GPU call)."""
import copy
import json
import sys
from pathlib import Path

import numpy as np
import pytest

from grande_b200 import laya as LY
from grande_b200._lib import OmgError
from oracle import oracle as O

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))

import make_golden_laya as G  # noqa: E402
from layamodels import config_json, laya_weights, small  # noqa: E402


def _fixture():
    z = np.load(HERE / "golden" / "laya_small.npz")
    return z, G.small_config(json.loads(str(z["config"]))), [tuple(s) for s in json.loads(str(z["seqs"]))]


def test_oracle_matches_modernbert_and_torch_head():
    z, cfg, seqs = _fixture()
    ws = laya_weights(cfg, G.SMALL["seed"])
    ids, pos, seq, qt = O.laya_pack(seqs)
    x = O.laya_hidden(cfg, ws, ids, pos, seq, qt, O.ORACLE_EXACT)
    exp = z["x_head"]
    assert np.abs(x - exp).max() <= 1e-4 * max(1.0, np.abs(exp).max())


def test_oracle_encoder_matches_modernbert():
    z, cfg, seqs = _fixture()
    enc_only = copy.copy(cfg)
    enc_only.head_layers = 0
    ws = [w for (n, _), w in zip(cfg.tensors(), laya_weights(cfg, G.SMALL["seed"]))
          if not n.startswith("head.")]
    ids, pos, seq, qt = O.laya_pack(seqs)
    x = O.laya_hidden(enc_only, ws, ids, pos, seq, qt, O.ORACLE_EXACT)
    exp = z["x_encoder"]
    assert np.abs(x - exp).max() <= 1e-4 * max(1.0, np.abs(exp).max())


def test_oracle_kernel_rounding_stays_close():
    """The f16 rounding points move x by far less than the 2e-2 the GPU
    tests allow."""
    z, cfg, seqs = _fixture()
    ws = laya_weights(cfg, G.SMALL["seed"])
    ids, pos, seq, qt = O.laya_pack(seqs)
    a = O.laya_hidden(cfg, ws, ids, pos, seq, qt, O.ORACLE_EXACT)
    b = O.laya_hidden(cfg, ws, ids, pos, seq, qt, O.ORACLE_KERNEL)
    assert np.abs(a - b).max() / np.abs(a).max() < 5e-3


def test_oracle_sequences_are_isolated():
    """A sequence's rows do not depend on what else is packed with it."""
    z, cfg, seqs = _fixture()
    ws = laya_weights(cfg, G.SMALL["seed"])
    ids, pos, seq, qt = O.laya_pack(seqs)
    both = O.laya_hidden(cfg, ws, ids, pos, seq, qt)
    ids1, pos1, seq1, qt1 = O.laya_pack(seqs[1:2])
    alone = O.laya_hidden(cfg, ws, ids1, pos1, seq1, qt1)
    n0 = len(seqs[0][0])
    assert np.abs(both[n0:n0 + len(seqs[1][0])] - alone).max() < 1e-5


def test_catalogue_matches_reference_order():
    for cfg in (small(), small(layers=4, head_layers=0, act_out=0), small(layers=1, head_layers=1)):
        js = json.dumps(config_json(cfg))
        assert LY.config_tensors(js) == [(n, list(s)) for n, s in cfg.tensors()]


def test_config_summary_and_defaults():
    cfg = small(layers=4, window=64)
    js = config_json(cfg)
    assert LY.config_check(json.dumps(js)) == (
        "layers=4 d=128 heads=2 ff=192 vocab=96 head_layers=2 act_out=3")
    # ModernBERT's default pattern when layer_types is absent: global every 3rd.
    js2 = copy.deepcopy(js)
    del js2["layer_types"]
    js2["global_attn_every_n_layers"] = 3
    assert LY.config_check(json.dumps(js2)) == LY.config_check(json.dumps(js))


@pytest.mark.parametrize("mutate,message", [
    (lambda j: j.update(model_type="bert"), 'encoder model_type "bert" is not modernbert'),
    (lambda j: j.update(hidden_activation="relu"), "encoder hidden_activation relu is not gelu"),
    (lambda j: j.pop("hidden_size"), "encoder/config.json: missing hidden_size"),
    (lambda j: j.update(layer_types=["full_attention"]), "layer_types has 1 entries for 3 layers"),
    (lambda j: j["laya_agent"].update(temperature=[1.0, 2.0]),
     "rl_agent_config.json: temperature has 2 entries"),
    (lambda j: j["laya_agent"].update(temperature=[1.0, 0.0, 1.0]),
     "calibration temperatures must be finite and positive"),
    (lambda j: j["laya_agent"].update(head_max_len=600),
     "expected 4 < head_max_len 600 < max_len 512"),
    (lambda j: j.update(num_attention_heads=3), "hidden_size 128 / heads 3"),
    (lambda j: j["laya_tokens"].pop("mask_token"), "tokenizer_config.json: missing mask_token"),
    (lambda j: j["laya_special_ids"].pop("[SEP]"), "tokenizer has no [SEP]"),
    (lambda j: j.pop("laya_agent"), "config.json: missing laya_agent"),
    (lambda j: j.update(hidden_size=4096, num_attention_heads=64), "hidden_size 4096 > 2048"),
    (lambda j: j.update(num_attention_heads=4), "head_dim 32: this engine runs 64-dim attention heads"),
])
def test_config_errors_match_reference(mutate, message):
    js = config_json(small())
    mutate(js)
    with pytest.raises(OmgError) as e:
        LY.config_check(json.dumps(js))
    assert message in str(e.value)


def test_attention_pattern_and_window():
    """ModernBERT's local_attention is the full window width; the engine
    keeps half of it as the inclusive distance (laya.rs:185)."""
    js = config_json(small(window=64))
    assert js["local_attention"] == 128
    js["local_attention"] = 9
    LY.config_check(json.dumps(js))  # odd widths round down like the reference
