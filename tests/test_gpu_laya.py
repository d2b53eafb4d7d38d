"""The Laya encoder engine (crates/omg-wgpu/src/laya.rs) on the GPU against
the oracle on the same seeded checkpoints: read-back rows within the
reference's 2e-2 relative tolerance (tests/reference.rs:380-407 uses it for
hidden rows), scorer logits and calibrated probabilities, isolation of
packed sequences, long sequences over several key tiles with the local
window, and the request errors with the reference's messages."""
import json
import sys
from pathlib import Path

import numpy as np
import pytest

from grande_b200._lib import OmgError
from grande_b200.laya import Sequence
from oracle import oracle as O

sys.path.insert(0, str(Path(__file__).resolve().parent))
from layamodels import LayaModel, small  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = 2e-2


def seqs_mixed(vocab=96):
    """Short sequences of different lengths, each with a few option markers."""
    rng = np.random.default_rng(3)
    out = []
    for n, qt in ((13, 0), (5, 2), (40, 1), (1, 0), (22, 2), (9, 1)):
        ids = [1] + list(rng.integers(5, vocab, n - 1)) if n > 1 else [1]
        markers = sorted(set(int(m) for m in rng.integers(0, n, min(3, n))))
        out.append(Sequence(ids, markers, qt))
    return out


def seqs_long(vocab=96):
    """Sequences longer than a 128-row tile, with many marker rows."""
    rng = np.random.default_rng(5)
    out = []
    for n, qt in ((300, 0), (7, 1), (150, 2), (129, 0), (64, 1)):
        ids = [1] + list(rng.integers(5, vocab, n - 1))
        markers = list(range(0, n, 7)) + [n - 1]
        out.append(Sequence(ids, sorted(set(markers)), qt))
    return out


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1.0))


def check_rows(m: LayaModel, seqs, tol=TOL, capacity=2048, max_rows=256):
    eng = m.engine(capacity=capacity, max_rows=max_rows)
    got = eng.hidden(seqs)
    exp = m.rows(seqs, m.hidden(seqs))
    worst = max(rel(g, e) for g, e in zip(got, exp))
    assert worst < tol, f"relative diff {worst}"
    eng.close()
    return worst


@pytest.mark.parametrize("linear,embed", [(O.Q8, O.Q8), (O.F16, O.F16), (O.Q4, O.Q8)])
def test_hidden_matches_oracle(linear, embed):
    check_rows(LayaModel(small(), 7, linear, embed), seqs_mixed())


def test_hidden_long_sequences_local_window():
    """Several 128-key tiles per item, window 64 on the local layers."""
    check_rows(LayaModel(small(layers=3, window=64), 9, O.Q8, O.Q8), seqs_long(), capacity=1024)


def test_hidden_long_sequences_small_window():
    check_rows(LayaModel(small(layers=3, window=5), 13, O.Q8, O.F16), seqs_long(), capacity=1024)


def test_mmbert_shape_two_layers():
    """mmBERT-base widths (d 768, 12 heads of 64, GeGLU 1152) on 2 layers +
    the decision head, 8 sequences of 128 tokens with a [MASK] row each."""
    cfg = small(layers=2, window=64, d=768, heads=12, ff=1152, vocab=512)
    m = LayaModel(cfg, 21, O.Q8, O.Q8)
    rng = np.random.default_rng(1)
    seqs = [Sequence([1] + list(rng.integers(5, 512, 127)), [int(rng.integers(1, 128))], i % 3)
            for i in range(8)]
    check_rows(m, seqs, capacity=1024, max_rows=64)


def test_large_batch_n_fastest_tiles():
    """48 sequences of 128 tokens (6,144 rows): every projection has more
    than four times as many rows as weight rows, so the GEMMs walk their
    tiles N-fastest and the in-place residual epilogue takes its whole-block
    path, as at the mmBERT bench size."""
    m = LayaModel(small(layers=2, window=64), 31, O.Q8, O.Q8)
    rng = np.random.default_rng(11)
    seqs = [Sequence([1] + list(rng.integers(5, 96, 127)), [int(rng.integers(1, 128))], i % 3)
            for i in range(48)]
    check_rows(m, seqs, capacity=48 * 128, max_rows=128)


@pytest.mark.parametrize("long", [False, True])
def test_sequences_are_isolated(long):
    """A sequence's rows do not depend on what is packed beside it: the same
    bits alone or in a batch (the reference allows 1e-4 for its layout
    invariance, reference.rs:720-735; this engine is exact)."""
    m = LayaModel(small(window=64 if long else 4), 17, O.Q8, O.Q8)
    eng = m.engine()
    seqs = seqs_long() if long else seqs_mixed()
    both = eng.hidden(seqs)
    for i in (0, 2, 4):
        alone = eng.hidden([seqs[i]])[0]
        assert np.array_equal(alone, both[i])
        shuffled = eng.hidden([seqs[(i + 1) % len(seqs)], seqs[i]])[1]
        assert np.array_equal(shuffled, both[i])
    eng.close()


def test_evaluate_scores_and_probabilities():
    """evaluate() = hidden + the scorer / act head (laya.rs:1442-1486, run
    on the device here); probabilities() with the calibration temperature
    (laya.rs:1489-1493)."""
    by = {"choice:3-5": 0.7, "noul:2": 1.9}
    m = LayaModel(small(), 23, O.Q8, O.Q8, temperature=(1.3, 0.8, 1.1), by_options=by)
    eng = m.engine()
    seqs = seqs_mixed()
    outs = eng.evaluate(seqs)
    rows = eng.hidden(seqs)
    exp_rows = m.rows(seqs, m.hidden(seqs))
    for s, o, r, er in zip(seqs, outs, rows, exp_rows):
        # The head agrees with the reference's host head on the engine's own
        # rows to f32 reassociation (the device sums in warp trees, the host
        # in index order) ...
        lg, act = O.laya_score(m.cfg, m.host, r)
        np.testing.assert_allclose(o.logits, lg, rtol=1e-4, atol=1e-5)
        assert o.act_probability is not None and abs(o.act_probability - act) < 1e-5
        # ... and close to the oracle end to end.
        lg2, act2 = O.laya_score(m.cfg, m.host, er)
        assert np.abs(o.logits - lg2).max() < TOL
        t = {0: 1.3, 1: 0.8, 2: 1.1}[s.qtype]
        k = len(s.markers)
        size = "2" if k <= 2 else "3-5" if k <= 5 else "6-10"
        t = by.get(f"{['choice', 'score', 'noul'][s.qtype]}:{size}", t)
        p = eng.probabilities(s.qtype, o.logits)
        z = np.asarray(lg2, np.float32) / np.float32(t)
        pe = np.exp(z - z.max())
        pe /= pe.sum()
        assert np.abs(p - pe).max() < 1e-3
        assert abs(p.sum() - 1.0) < 1e-6
    eng.close()


def test_device_head_many_sequences_and_markers():
    """The device head over more sequences and markers than one CTA takes
    (eight of each), one-marker sequences (the act head sees two slots, one
    padded) and sequences of up to 20 markers, against the reference's host
    head on the engine's own rows."""
    m = LayaModel(small(), 37, O.Q8, O.Q8)
    eng = m.engine(capacity=2048, max_rows=512)
    rng = np.random.default_rng(11)
    seqs = seqs_long()
    for i in range(19):
        n = int(rng.integers(2, 60))
        ids = [1] + list(rng.integers(5, 96, n - 1))
        k = 1 if i % 5 == 4 else int(rng.integers(1, min(n, 20) + 1))
        markers = sorted(set(int(x) for x in rng.choice(np.arange(n), k, replace=False)))
        seqs.append(Sequence(ids, markers, i % 3))
    outs = eng.evaluate(seqs)
    rows = eng.hidden(seqs)
    assert sum(len(s.markers) for s in seqs) > 16 and len(seqs) > 16
    for s, o, r in zip(seqs, outs, rows):
        lg, act = O.laya_score(m.cfg, m.host, r)
        assert len(o.logits) == len(s.markers)
        np.testing.assert_allclose(o.logits, lg, rtol=1e-4, atol=1e-5)
        assert abs(o.act_probability - act) < 1e-5
    eng.close()


def test_no_act_head_and_no_head_layers():
    m = LayaModel(small(head_layers=0, act_out=0), 29, O.Q8, O.Q8)
    eng = m.engine()
    seqs = seqs_mixed()
    got = eng.hidden(seqs)
    exp = m.rows(seqs, m.hidden(seqs))
    assert max(rel(g, e) for g, e in zip(got, exp)) < TOL
    assert all(o.act_probability is None for o in eng.evaluate(seqs))
    eng.close()


def test_warmup_and_repeat_are_deterministic():
    m = LayaModel(small(), 31, O.Q8, O.Q8)
    eng = m.engine()
    eng.warmup()
    seqs = seqs_mixed()
    a = eng.hidden(seqs)
    b = eng.hidden(seqs)
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
    eng.close()


@pytest.mark.parametrize("seqs,message", [
    ([], "empty request"),
    ([Sequence([], [], 0)], "empty request"),
    ([Sequence([1, 2], [], 0), Sequence([], [], 0)], "sequence 1 is empty"),
    ([Sequence([1, 500], [0], 0)], "token id 500 outside the vocabulary of 96"),
    ([Sequence([1, 2, 3], [3], 0)], "sequence 0: marker 3 past its 3 tokens"),
    ([Sequence([1, 2, 3], [0], 3)], "sequence 0: question type 3"),
    ([Sequence([1] * 600, [0], 0)], "sequence 0: 600 tokens > max_len 512"),
    ([Sequence([1] * 100, [0], 0)] * 25, "2500 tokens exceed the engine capacity 2048"),
    ([Sequence([1, 2, 3], [0, 1, 2], 0)] * 70, "280 rows requested, engine reads back at most 256"),
])
def test_request_errors(seqs, message):
    """laya.rs:1145-1205's errors, message for message."""
    m = LayaModel(small(layers=1, head_layers=1), 37, O.Q8, O.Q8)
    eng = m.engine()
    with pytest.raises(OmgError) as e:
        eng.hidden(seqs)
    assert message in str(e.value)
    # The engine still works after a rejected request.
    eng.hidden(seqs_mixed()[:2])
    eng.close()
