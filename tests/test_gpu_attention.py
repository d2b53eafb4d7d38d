"""The block-causal attention kernel against an f64 reference of the same op
(Q, K, V rounded to f16 as attention.wgsl:80-92,110-117 rounds them; the
visibility rule of attention.wgsl:70-76), on packed prefix + branch layouts
with groups, GQA and sliding windows; plus the layout invariance the
reference's group test relies on (tests/reference.rs:716-735)."""
import ctypes as C

import numpy as np
import pytest

from grande_b200 import _lib as L
from oracle import oracle as O

pytestmark = pytest.mark.gpu



def run_attention(device, q, kv, meta, t, base, heads, kvh, hd, window, p_lo=False):
    out = np.zeros((t, heads * hd), np.float16)
    L.check(L.lib().omg_debug_attention(device, L.ptr(q.view(np.uint16), C.c_uint16),
                                        L.ptr(kv.view(np.uint16), C.c_uint16),
                                        L.ptr(meta, C.c_int32), t, base, heads, kvh, hd, window,
                                        int(p_lo), L.ptr(out.view(np.uint16), C.c_uint16)))
    return out.astype(np.float32)


def reference(q, kv, meta, t, base, heads, kvh, hd, window):
    hpg = heads // kvh
    out = np.zeros((t, heads * hd), np.float64)
    K = kv[:, :kvh * hd].astype(np.float64)
    V = kv[:, kvh * hd:].astype(np.float64)
    for i in range(t):
        qp, qs = meta[base + i, 0], meta[base + i, 1]
        vis = np.array([O.visible(int(qp), int(qs), int(meta[j, 0]), int(meta[j, 1]), window)
                        for j in range(base + t)])
        for h in range(heads):
            g = h // hpg
            qh = q[i, h * hd:(h + 1) * hd].astype(np.float64)
            s = K[:base + t, g * hd:(g + 1) * hd] @ qh
            s = np.where(vis, s, -np.inf)
            p = np.exp(s - s.max())
            p /= p.sum()
            out[i, h * hd:(h + 1) * hd] = p @ V[:base + t, g * hd:(g + 1) * hd]
    return out


def layout(groups, lead=0):
    """(pos, seq, row_lo, row_hi) per cache row for groups of (prefix_len,
    [branch_len...]), packed as engine.rs:1512-1571 packs them, after `lead`
    rows of a separate group."""
    meta = []
    if lead:
        for i in range(lead):
            meta.append((i, 0, 0, i + 1))
    for k, (p, branches) in enumerate(groups):
        k += 1 if lead else 0
        lo = len(meta)
        for i in range(p):
            meta.append((i, k << 12, lo, len(meta) + 1))
        for b, n in enumerate(branches):
            for j in range(n):
                meta.append((p + j, (k << 12) | (b + 1), lo, len(meta) + 1))
    return np.array(meta, np.int32)


def make_inputs(rng, rows, heads, kvh, hd, scale):
    q = (rng.standard_normal((rows, heads * hd)) * scale).astype(np.float16)
    kv = (rng.standard_normal((rows, 2 * kvh * hd)) * scale).astype(np.float16)
    kv[:, kvh * hd:] = rng.standard_normal((rows, kvh * hd)).astype(np.float16)
    return q, kv


@pytest.mark.parametrize("heads,kvh,hd", [(2, 1, 256), (8, 2, 256), (4, 1, 512), (8, 2, 512),
                                          (16, 1, 256)])
@pytest.mark.parametrize("window", [0, 5, 40])
def test_attention_matches_reference(device, heads, kvh, hd, window):
    rng = np.random.default_rng(heads * 1000 + hd + window)
    meta = layout([(37, [5, 9, 1, 12]), (3, [6]), (70, [24, 24])])
    rows = len(meta)
    q, kv = make_inputs(rng, rows, heads, kvh, hd, 1.0 / np.sqrt(np.sqrt(hd)))
    got = run_attention(device, q, kv, meta, rows, 0, heads, kvh, hd, window)
    exp = reference(q, kv, meta, rows, 0, heads, kvh, hd, window)
    # f16 output rounding bounds the error: 2^-11 relative per element.
    assert np.abs(got - exp).max() < 2e-3 * max(np.abs(exp).max(), 1.0)


def test_attention_resident_base(device):
    """Queries are the cache rows base..base+t (a resident prefix)."""
    rng = np.random.default_rng(5)
    heads, kvh, hd = 8, 2, 256
    meta = layout([(150, [24, 24, 24])])
    rows = len(meta)
    q, kv = make_inputs(rng, rows, heads, kvh, hd, 0.5)
    base = 150
    got = run_attention(device, q[base:], kv, meta, rows - base, base, heads, kvh, hd, 64)
    exp = reference(q[base:], kv, meta, rows - base, base, heads, kvh, hd, 64)
    assert np.abs(got - exp).max() < 2e-3 * max(np.abs(exp).max(), 1.0)


@pytest.mark.parametrize("hd", [256, 512])
@pytest.mark.parametrize("window", [0, 6])
def test_attention_layout_invariance(device, hd, window):
    """The same group behind 1, 7, 16 or 64 rows of another group gives
    bit-identical rows: CTAs never cross groups and key tiles start at the
    group's first row (large scores, as Gemma 4's unscaled q.k)."""
    rng = np.random.default_rng(hd + window)
    heads, kvh = 4, 1
    grp = [(9, [5, 8, 3])]
    base_meta = layout(grp)
    n = len(base_meta)
    q, kv = make_inputs(rng, n, heads, kvh, hd, 1.0)  # |q.k| ~ hd: peaked softmax
    ref = run_attention(device, q, kv, base_meta, n, 0, heads, kvh, hd, window)
    for lead in (1, 7, 16, 64):
        meta = layout(grp, lead)
        pad_q = np.concatenate([np.zeros((lead, heads * hd), np.float16), q])
        pad_kv = np.concatenate([np.zeros((lead, 2 * kvh * hd), np.float16), kv])
        got = run_attention(device, pad_q, pad_kv, meta, lead + n, 0, heads, kvh, hd, window)[lead:]
        assert np.array_equal(got, ref), (lead, float(np.abs(got - ref).max()))


@pytest.mark.parametrize("window", [0, 512, 100])
@pytest.mark.parametrize("p_lo", [False, True])
def test_attention_e2b_packing(device, window, p_lo):
    """A 500-token state with 12 branches of 24 (the E2B request) at GQA 8/2:
    runs span many 64-key tiles, with and without P's f16 residue."""
    rng = np.random.default_rng(window + 11)
    heads, kvh, hd = 8, 2, 256
    meta = layout([(500, [24] * 12)])
    rows = len(meta)
    q, kv = make_inputs(rng, rows, heads, kvh, hd, 1.0 / np.sqrt(np.sqrt(hd)))
    got = run_attention(device, q, kv, meta, rows, 0, heads, kvh, hd, window, p_lo)
    exp = reference(q, kv, meta, rows, 0, heads, kvh, hd, window)
    assert np.abs(got - exp).max() < 2e-3 * max(np.abs(exp).max(), 1.0)


def test_attention_peaked_scores_rescale(device):
    """Scores growing along the keys (each tile's max above the last by more
    than the reference-max slack) force the output rescale on every tile."""
    rng = np.random.default_rng(9)
    heads, kvh, hd = 4, 1, 256
    meta = layout([(400, [30, 7])])
    rows = len(meta)
    q, kv = make_inputs(rng, rows, heads, kvh, hd, 0.2)
    # Positive queries against K rows that grow with the row index: a 64-key
    # tile's scores exceed the previous tile's by ~9, more than the slack.
    kv[:, :hd] = np.repeat(np.linspace(0.0, 3.0, rows)[:, None], hd, 1).astype(np.float16)
    q[:] = (np.abs(q.astype(np.float32)) * 0.5).astype(np.float16)
    got = run_attention(device, q, kv, meta, rows, 0, heads, kvh, hd, 0)
    exp = reference(q, kv, meta, rows, 0, heads, kvh, hd, 0)
    assert np.abs(got - exp).max() < 2e-3 * max(np.abs(exp).max(), 1.0)


@pytest.mark.parametrize("hd", [256, 512])
@pytest.mark.parametrize("window", [0, 60])
def test_attention_resident_equals_cold(device, hd, window):
    """Branch rows computed with the prefix resident (queries = branch rows
    only) equal, bit for bit, the same rows of a cold pass over prefix and
    branches (tests/reference.rs:432-480 asserts this on the engine)."""
    rng = np.random.default_rng(hd + window + 3)
    heads, kvh = 8, 2
    prefix = 300
    meta = layout([(prefix, [24, 17, 40])])
    rows = len(meta)
    q, kv = make_inputs(rng, rows, heads, kvh, hd, 1.0)
    cold = run_attention(device, q, kv, meta, rows, 0, heads, kvh, hd, window)
    warm = run_attention(device, q[prefix:], kv, meta, rows - prefix, prefix, heads, kvh, hd,
                         window)
    assert np.array_equal(cold[prefix:], warm), float(np.abs(cold[prefix:] - warm).max())


def test_attention_layout_invariance_long(device):
    """A group spanning several key tiles behind other rows of another group:
    its rows are bit-identical wherever it sits."""
    rng = np.random.default_rng(77)
    heads, kvh, hd = 8, 2, 256
    grp = [(260, [31, 12])]
    base_meta = layout(grp)
    n = len(base_meta)
    q, kv = make_inputs(rng, n, heads, kvh, hd, 1.0)
    ref = run_attention(device, q, kv, base_meta, n, 0, heads, kvh, hd, 0)
    for lead in (3, 130):
        meta = layout(grp, lead)
        pad_q = np.concatenate([np.ones((lead, heads * hd), np.float16), q])
        pad_kv = np.concatenate([np.ones((lead, 2 * kvh * hd), np.float16), kv])
        got = run_attention(device, pad_q, pad_kv, meta, lead + n, 0, heads, kvh, hd, 0)[lead:]
        assert np.array_equal(got, ref), (lead, float(np.abs(got - ref).max()))
