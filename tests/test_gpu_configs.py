"""The BASELINE.json configurations other than the headline pass, at their
production widths, against the reference's CPU forward (oracle/):

* configs[0], the Gemma-3-270M shape with Q8_0 weights, all 18 layers (its
  query scale 256^-0.5 keeps attention logits of unit spread, so the
  benchmark's own model is checked at full depth): hidden rows within 2e-2
  (tests/reference.rs:380-407), logits within 2e-2 max-abs with the same
  argmax;
* configs[2], a 2,000-token resident state at E2B widths with 12 branches of
  24 tokens (2 layers, one sliding and one global, the conditioned q / k
  norms of test_gpu_depth): the cold pass against the reference, the
  resident pass and a pass after a save / restore of the state equal to it
  bit for bit (reference.rs:509,520);
* Gemma 4's real layer layout at E2B and E4B widths (a 256-dim sliding
  layer, a 512-dim global layer with partial RoPE) on their requests;
* configs[3], E4B widths (d 2560, GeGLU 10240) with a 2,000-token state and
  20 branches of 32 tokens (2,640 rows, the CTA-pair kernels), 2 layers;
* configs[4], mmBERT widths at the full 22 encoder layers + 2 decision-head
  layers, 16 sequences of 128 tokens."""
import dataclasses

import numpy as np
import pytest

from grande_b200 import synth
from grande_b200.engine import PrefixSource, Want
from grande_b200.laya import Sequence
from oracle import oracle as O

from layamodels import LayaModel
from test_gpu_depth import oracle_cfg, rel

pytestmark = pytest.mark.gpu


def answer_rows(req):
    rows, at = [], len(req.prefix)
    for b in req.branches:
        rows.append(at + b.want[0])
        at += len(b.tokens)
    return rows


def oracle_model(shape, qk_scale=1.0):
    ocfg = oracle_cfg(shape)
    if shape.gemma3_numerics:
        ocfg.query_scale = 256 ** -0.5
        ocfg.v_norm = False
        ocfg.softcap = 0.0
    return ocfg, O.synth_tensors(ocfg.tensors(), 0, int(shape.dtype), qk_scale=qk_scale)


def check_pass(shape, qk_scale, device, logits=True):
    req = synth.request(shape, seed=3)
    eng = synth.build_engine(shape, shape.tokens() + 64, shape.branches, device=device,
                             qk_scale=qk_scale)
    hid = np.stack([o.rows[0] for o in eng.evaluate(req.prefix, req.branches, Want.HIDDEN)])
    got_logits = None
    if logits:
        eng.evict_resident()
        got_logits = np.stack([o.rows[0] for o in
                               eng.evaluate(req.prefix, req.branches, Want.LOGITS)])
    ocfg, tensors = oracle_model(shape, qk_scale)
    ids, pos, seq = O.pack(req.prefix, [(b.tokens, b.want) for b in req.branches])
    rows = answer_rows(req)
    kern = O.forward(ocfg, tensors, ids, pos, seq, O.ORACLE_KERNEL)[rows]
    exact = O.forward(ocfg, tensors, ids, pos, seq, O.ORACLE_EXACT)[rows]
    modes = max(rel(k, e) for k, e in zip(kern, exact))
    drift = max(rel(g, k) for g, k in zip(hid, kern))
    assert drift < 1.5 * max(modes, 1e-3), (drift, modes)
    assert max(rel(g, e) for g, e in zip(hid, exact)) < 2e-2
    if logits:
        for i, got in enumerate(got_logits):
            exp = O.logits(exact[i], tensors[0], ocfg.vocab, ocfg.d, ocfg.softcap)
            err = float(np.abs(got - exp).max())
            assert err < 2e-2, f"branch {i}: logits max-abs diff {err}"
            top2 = np.sort(exp)[-2:]
            if top2[1] - top2[0] > 2 * err:
                assert int(np.argmax(got)) == int(np.argmax(exp)), f"branch {i}: argmax"
    return eng, req


def test_gemma3_270m_q8_full_depth(device):
    eng, _ = check_pass(synth.CONFIGS["gemma3-270m-q8"], 1.0, device)
    eng.close()


def test_e2b_resident_state_two_layers(device):
    shape = dataclasses.replace(synth.CONFIGS["e2b-q4-resident"], layers=2, global_every=2)
    eng, req = check_pass(shape, 0.25, device, logits=False)
    # A cold pass, then the prefix is resident: a branches-only pass.
    eng.evict_resident()
    cold = eng.evaluate(req.prefix, req.branches, Want.HIDDEN)
    assert eng.prefix_source() == PrefixSource.DECODED
    warm = eng.evaluate(req.prefix, req.branches, Want.HIDDEN)
    assert eng.prefix_source() == PrefixSource.RESIDENT
    for a, b in zip(cold, warm):
        assert np.array_equal(a.rows, b.rows)
    # The state (sliding layer window-only) through host memory and back.
    st = eng.save_state(req.prefix)
    eng.evict_resident()
    eng.restore_state(st)
    again = eng.evaluate(req.prefix, req.branches, Want.HIDDEN)
    assert eng.prefix_source() == PrefixSource.RESIDENT
    for a, b in zip(cold, again):
        assert np.array_equal(a.rows, b.rows)
    eng.close()


@pytest.mark.parametrize("base", ["e2b-q4", "e4b-q4"])
def test_gemma4_global_head_dim_512(device, base):
    """Gemma 4's real layer layout (model.rs:110-148) at E2B and E4B widths:
    a sliding layer with 256-dim heads, then a global layer with 512-dim
    heads rotated over a quarter of their dims, on the config's request (E2B:
    500-token state, 12 branches of 24; E4B: 2,000-token state, 20 branches
    of 32, chunk-split runs and their merges): the tcgen05 head_dim-512
    attention and the 512-dim q / k / v norms and partial RoPE against the
    reference."""
    shape = dataclasses.replace(synth.CONFIGS[base], layers=2, global_every=2,
                                global_head_dim=512, global_rotary=0.25)
    eng, req = check_pass(shape, 0.25, device)
    eng.evict_resident()
    cold = eng.evaluate(req.prefix, req.branches, Want.HIDDEN)
    warm = eng.evaluate(req.prefix, req.branches, Want.HIDDEN)
    assert eng.prefix_source() == PrefixSource.RESIDENT
    for a, b in zip(cold, warm):
        assert np.array_equal(a.rows, b.rows)
    eng.close()


def test_e4b_widths_two_layers(device):
    shape = dataclasses.replace(synth.CONFIGS["e4b-q4"], layers=2, global_every=2)
    eng, _ = check_pass(shape, 0.25, device)
    eng.close()


def test_mmbert_widths_full_depth(device):
    cfg = O.OracleLayaConfig(vocab=512, d=768, layers=22, heads=12, ff=1152,
                             sliding=[0] * 22, window=64, head_layers=2, act_hidden=256,
                             act_out=3)
    m = LayaModel(cfg, 23, O.Q8, O.Q8)
    rng = np.random.default_rng(2)
    seqs = [Sequence([1] + list(rng.integers(5, 512, 126)) + [2], [int(rng.integers(1, 127))],
                     i % 3) for i in range(16)]
    eng = m.engine(capacity=16 * 128, max_rows=64, device=device)
    got = eng.hidden(seqs)
    kern = m.rows(seqs, m.hidden(seqs, O.ORACLE_KERNEL))
    exact = m.rows(seqs, m.hidden(seqs, O.ORACLE_EXACT))
    modes = max(rel(k, e) for k, e in zip(kern, exact))
    drift = max(rel(g, k) for g, k in zip(got, kern))
    assert drift < 1.5 * max(modes, 1e-3), (drift, modes)
    assert max(rel(g, e) for g, e in zip(got, exact)) < 2e-2
    eng.close()
