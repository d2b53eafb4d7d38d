"""The engine against the oracle on the reference's own test scenarios
(crates/omg-wgpu/tests/reference.rs): same tiny seeded models, same packed
requests, same tolerances, same exact-equality invariants."""
import numpy as np
import pytest

from grande_b200.engine import BranchTokens, Dtype, Group, PrefixSource, SavedState, Want
from oracle import oracle as O

from refmodels import RefModel, gemma3, gemma4, gemma4_gqa

pytestmark = pytest.mark.gpu

F16, Q8, Q4 = O.F16, O.Q8, O.Q4


def model(kind, seed, linear, embed):
    cfg, js = {"g3": gemma3, "g4": gemma4, "gqa": gemma4_gqa}[kind]()
    return RefModel(cfg, js, seed, linear, embed)


def check_hidden(m: RefModel, tol: float):
    """reference.rs:380-407."""
    eng = m.engine()
    prefix = [2, 5, 9, 14, 20, 31, 7, 8, 3, 22]
    branches = [BranchTokens([11, 12, 13, 14, 15], [1, 4]),
                BranchTokens([30, 31, 32, 33, 34, 35, 36, 37], [0, 7])]
    out = eng.evaluate(prefix, branches, Want.HIDDEN)
    ids, pos, seq = O.pack(prefix, [(b.tokens, b.want) for b in branches])
    hidden = m.hidden(ids, pos, seq)
    idx = len(prefix)
    for b, o in zip(branches, out):
        for slot, w in enumerate(b.want):
            got, exp = o.rows[slot], hidden[idx + w]
            scale = max(np.abs(exp).max(), 1.0)
            d = np.abs(got - exp).max() / scale
            assert d < tol, f"row {slot}: relative diff {d}"
        idx += len(b.tokens)
    eng.close()


def test_gemma3_matches_cpu_reference():
    check_hidden(model("g3", 7, F16, F16), 2e-2)


def test_gemma4_q8_matches_cpu_reference():
    check_hidden(model("g4", 7, Q8, Q8), 2e-2)


def test_gemma4_q4_matches_cpu_reference():
    check_hidden(model("g4", 9, Q4, Q8), 2e-2)


def test_gemma4_f16_matches_cpu_reference():
    check_hidden(model("g4", 5, F16, F16), 2e-2)


def test_gemma4_gqa_q4_matches_cpu_reference():
    check_hidden(model("gqa", 11, Q4, Q8), 2e-2)


def rows_equal(a, b):
    return len(a) == len(b) and all(np.array_equal(x.rows, y.rows) for x, y in zip(a, b))


def test_long_prefix_matches_cpu_reference():
    """A 2,100-token prefix: the pass has more than 16 row tiles, so its
    projections run on the CTA-pair (cta_group::2) GEMM and its FFN as two
    pair launches; rows vs the CPU reference at the reference's 2e-2
    (reference.rs:380-407), and a branch alone equals the branch beside a
    resident prefix bit for bit."""
    for kind, lin, emb in (("g3", F16, F16), ("gqa", Q4, Q8)):
        m = model(kind, 37, lin, emb)
        eng = m.engine(capacity=2304, max_rows=16)
        rng = np.random.default_rng(5)
        prefix = [int(x) for x in rng.integers(1, m.cfg.vocab, 2100)]
        branches = [BranchTokens([int(x) for x in rng.integers(1, m.cfg.vocab, 9)], [0, 8]),
                    BranchTokens([int(x) for x in rng.integers(1, m.cfg.vocab, 5)], [4])]
        out = eng.evaluate(prefix, branches, Want.HIDDEN)
        ids, pos, seq = O.pack(prefix, [(b.tokens, b.want) for b in branches])
        hidden = m.hidden(ids, pos, seq)
        idx = len(prefix)
        for b, o in zip(branches, out):
            for slot, w in enumerate(b.want):
                exp = hidden[idx + w]
                d = np.abs(o.rows[slot] - exp).max() / max(np.abs(exp).max(), 1.0)
                assert d < 2e-2, f"{kind}: relative diff {d}"
            idx += len(b.tokens)
        again = eng.evaluate(prefix, branches, Want.HIDDEN)
        assert eng.prefix_source() == PrefixSource.RESIDENT
        assert rows_equal(out, again)
        eng.close()


def test_resident_prefix_matches_full_pass():
    """reference.rs:432-480."""
    for m in (model("g3", 13, F16, F16), model("g4", 13, Q4, Q8), model("gqa", 13, Q4, Q8)):
        eng = m.engine()
        prefix = [2, 5, 9, 14, 20, 31, 7]
        branches = [BranchTokens([11, 12, 13, 14, 15], [1, 4]), BranchTokens([30, 31, 32], [0, 2])]
        other = [BranchTokens([33, 34, 35, 36, 37, 38], [5])]
        full = eng.evaluate(prefix, branches, Want.HIDDEN)
        assert eng.prefix_source() == PrefixSource.DECODED
        cont = eng.evaluate(prefix, other, Want.HIDDEN)
        assert eng.prefix_source() == PrefixSource.RESIDENT
        eng.evict_resident()
        cold = eng.evaluate(prefix, other, Want.HIDDEN)
        assert eng.prefix_source() == PrefixSource.DECODED
        assert np.array_equal(cont[0].rows, cold[0].rows)
        again = eng.evaluate(prefix, branches, Want.HIDDEN)
        assert eng.prefix_source() == PrefixSource.RESIDENT
        assert rows_equal(full, again)
        prefix2 = [2, 3, 4]
        p2 = eng.evaluate(prefix2, branches, Want.LOGITS)
        assert eng.prefix_source() == PrefixSource.DECODED
        p2r = eng.evaluate(prefix2, branches, Want.LOGITS)
        assert eng.prefix_source() == PrefixSource.RESIDENT
        assert rows_equal(p2, p2r)
        eng.close()


def test_state_cache_restores_exactly(tmp_path):
    """reference.rs:484-522."""
    for m in (model("g3", 17, F16, F16), model("g4", 17, Q4, Q8), model("gqa", 17, Q4, Q8)):
        eng = m.engine()
        eng.set_state_cache(64 << 20, None, "test")
        a = [2, 5, 9, 14, 20, 31, 7, 8, 3, 22, 4, 6]
        b = [2, 3, 4]
        branches = [BranchTokens([11, 12, 13, 14, 15], [0, 2, 4])]
        full_a = eng.evaluate(a, branches, Want.HIDDEN)
        assert eng.prefix_source() == PrefixSource.DECODED
        saved = eng.save_state(a)
        eng.evaluate(b, branches, Want.HIDDEN)
        assert eng.prefix_source() == PrefixSource.DECODED
        ram_a = eng.evaluate(a, branches, Want.HIDDEN)
        assert eng.prefix_source() == PrefixSource.RAM
        assert np.array_equal(full_a[0].rows, ram_a[0].rows)
        data = saved.to_bytes("test")
        back = SavedState.from_bytes(data, "test")
        with pytest.raises(Exception):
            SavedState.from_bytes(data, "other")
        eng.evaluate(b, branches, Want.HIDDEN)
        eng.evict_resident()
        eng.restore_state(back)
        assert eng.is_resident(a)
        file_a = eng.evaluate(a, branches, Want.HIDDEN)
        assert eng.prefix_source() == PrefixSource.RESIDENT
        assert np.array_equal(full_a[0].rows, file_a[0].rows)
        eng.close()


def test_state_cache_directory(tmp_path):
    """Disk tier of the state cache (engine.rs:2096-2150): a fresh engine
    with an empty RAM budget finds the state file and restores it."""
    m = model("g4", 17, Q4, Q8)
    eng = m.engine()
    eng.set_state_cache(0, str(tmp_path), "test")
    a = [2, 5, 9, 14, 20, 31, 7, 8, 3, 22, 4, 6]
    branches = [BranchTokens([11, 12, 13], [2])]
    full = eng.evaluate(a, branches, Want.HIDDEN)
    assert len(list(tmp_path.glob("*.state"))) == 1
    eng.evict_resident()
    disk = eng.evaluate(a, branches, Want.HIDDEN)
    assert eng.prefix_source() == PrefixSource.DISK
    assert np.array_equal(full[0].rows, disk[0].rows)
    eng.close()


def test_branches_do_not_see_each_other():
    """reference.rs:533-562."""
    for m in (model("g3", 11, F16, F16), model("g4", 11, Q8, Q8), model("gqa", 11, Q4, Q8)):
        eng = m.engine()
        prefix = [2, 4, 6, 8]
        a = BranchTokens([10, 11, 12], [2])
        b1 = BranchTokens([20, 21, 22, 23], [3])
        b2 = BranchTokens([30, 31], [1])
        with_b1 = eng.evaluate(prefix, [a, b1], Want.HIDDEN)
        with_b2 = eng.evaluate(prefix, [a, b2], Want.HIDDEN)
        alone = eng.evaluate(prefix, [a], Want.HIDDEN)
        assert np.array_equal(with_b1[0].rows[0], with_b2[0].rows[0])
        assert np.array_equal(with_b1[0].rows[0], alone[0].rows[0])
        eng.close()


def test_logits_are_hidden_times_embedding():
    """reference.rs:564-598."""
    for m, softcap in ((model("g3", 3, F16, F16), 0.0), (model("g4", 3, Q8, Q8), 30.0)):
        eng = m.engine()
        prefix = [2, 1, 3]
        branches = [BranchTokens([4, 5], [1])]
        hidden = eng.evaluate(prefix, branches, Want.HIDDEN)
        logits = eng.evaluate(prefix, branches, Want.LOGITS)
        h = hidden[0].rows[0]
        emb = m.tensor_f32("embed")
        exp = O.logits(h, emb, m.cfg.vocab, m.cfg.d, softcap)
        scale = max(np.abs(exp).max(), 1.0)
        assert np.abs(logits[0].rows[0] - exp).max() / scale < 1e-3
        eng.close()


def assert_close(a, b, what):
    """reference.rs:716-735."""
    assert len(a) == len(b), what
    worst, scale = 0.0, 0.0
    for x, y in zip(a, b):
        worst = max(worst, float(np.abs(x - y).max()))
        scale = max(scale, float(np.abs(x).max()))
    assert worst <= 1e-4 * max(scale, 1.0), f"{what}: max |d| {worst:e} at scale {scale:e}"


def test_groups_match_separate_passes():
    """reference.rs:616-714."""
    for m in (model("g3", 19, F16, F16), model("g4", 19, Q4, Q8), model("gqa", 19, Q4, Q8)):
        eng = m.engine()
        eng.set_state_cache(64 << 20, None, "test")
        prefixes = [[2, 5, 9, 14, 20, 31, 7, 8, 3], [2, 3, 4], [2, 22, 4, 6, 9, 9, 14, 1, 30, 31, 5]]
        branches = [
            [BranchTokens([11, 12, 13, 14, 15], [1, 4]), BranchTokens([30, 31, 32], [0, 2])],
            [BranchTokens([33, 34, 35, 36, 37, 38], [5])],
            [BranchTokens([7, 8], [1]), BranchTokens([11, 12, 13, 14, 15, 16, 17], [3, 6]),
             BranchTokens([1, 2, 3], [2])],
        ]
        groups = [Group(p, b) for p, b in zip(prefixes, branches)]
        for want in (Want.HIDDEN, Want.LOGITS):
            alone = []
            for g in groups:
                eng.evict_resident()
                alone.append(eng.evaluate(g.prefix, g.branches, want))
            eng.evict_resident()
            together = eng.evaluate_groups(groups, want)
            for i, (a, t) in enumerate(zip(alone, together)):
                assert len(t.branches) == len(a)
                for x, y in zip(a, t.branches):
                    assert_close(x.rows, y.rows, f"group {i} in the batch")
            assert together[0].prefix_source == PrefixSource.RAM
            assert together[1].prefix_source == PrefixSource.DECODED
            assert together[2].prefix_source == PrefixSource.DECODED
            assert eng.is_resident(prefixes[0])
            eng.evaluate(prefixes[1], branches[1], want)
            again = eng.evaluate_groups(groups, want)
            assert again[1].prefix_source == PrefixSource.RESIDENT
            for i, (a, t) in enumerate(zip(alone, again)):
                for x, y in zip(a, t.branches):
                    assert_close(x.rows, y.rows, f"group {i} with group 1 resident")
            eng.evaluate(prefixes[1], branches[1], want)
            from_cache = eng.evaluate(prefixes[2], branches[2], want)
            assert eng.prefix_source() == PrefixSource.RAM
            for x, y in zip(alone[2], from_cache):
                assert_close(x.rows, y.rows, "group 2 from the state cache")
        eng.close()


def test_request_errors_carry_reference_messages():
    """engine.rs:1503-1583 error texts, no partial outputs."""
    m = model("g3", 7, F16, F16)
    eng = m.engine(capacity=16, max_rows=2)
    with pytest.raises(Exception, match="exceed the engine capacity 16"):
        eng.evaluate(list(range(2, 20)), [BranchTokens([1], [0])], Want.HIDDEN)
    with pytest.raises(Exception, match="rows requested, engine reads back at most 2"):
        eng.evaluate([2, 3], [BranchTokens([1, 2, 3], [0, 1, 2])], Want.HIDDEN)
    with pytest.raises(Exception, match="outside the vocabulary of 40"):
        eng.evaluate([2, 3], [BranchTokens([41], [0])], Want.HIDDEN)
    with pytest.raises(Exception, match="wanted position 3 past its 2 tokens"):
        eng.evaluate([2, 3], [BranchTokens([4, 5], [3])], Want.HIDDEN)
    # The engine still works afterwards.
    out = eng.evaluate([2, 3], [BranchTokens([4, 5], [1])], Want.HIDDEN)
    assert np.isfinite(out[0].rows).all()
    eng.close()


@pytest.mark.parametrize("name", ["sliding", "branches"])
def test_engine_matches_transformers_gemma3(name):
    """The engine directly against the golden fixtures of make_golden.py
    (transformers Gemma 3 driven as python/omg_train/model.py drives it)."""
    import json
    from pathlib import Path
    from grande_b200.engine import Engine, QTensor
    g = np.load(Path(__file__).parent / "golden" / f"gemma3_{name}.npz")
    cfg_json = str(g["config"])
    tensors = {}
    for key in g.files:
        if key.startswith("t:"):
            bits = g[key]
            tensors[key[2:]] = QTensor(Dtype.F16, list(bits.shape), bits.tobytes(), b"")
    eng = Engine.new(tensors, cfg_json, 64, 16)
    seg, ids = g["seg"], g["ids"]
    prefix = [int(i) for i, s in zip(ids, seg) if s == 0]
    branches, idx = [], []
    for b in sorted(set(int(s) for s in seg if s > 0)):
        toks = [int(i) for i, s in zip(ids, seg) if s == b]
        branches.append(BranchTokens(toks, list(range(len(toks)))))
        idx += [k for k, s in enumerate(seg) if s == b]
    out = eng.evaluate(prefix, branches, Want.HIDDEN)
    got = np.concatenate([o.rows for o in out])
    exp = g["hidden"][idx]
    scale = np.maximum(np.abs(exp).max(axis=1, keepdims=True), 1.0)
    assert (np.abs(got - exp) / scale).max() < 2e-2
    eng.close()
