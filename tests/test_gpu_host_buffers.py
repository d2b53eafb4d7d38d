"""Output buffers: the engine copies rows straight from the device into a
page-locked buffer (omg_host_alloc) and through its staging buffer into any
other. Both give the same rows in the same slots, for one group and for a
multi-group request whose rows leave the device in another order than the
caller's (evaluate_groups, engine.rs:1404-1444), and an array handed out
keeps its rows while later calls run."""
import types

import numpy as np
import pytest

from grande_b200 import _lib
from grande_b200.engine import BranchTokens, Group, Want
from oracle import oracle as O
from refmodels import RefModel, gemma4

pytestmark = pytest.mark.gpu


def requests():
    one = [Group([2, 7, 11, 19, 23], [BranchTokens([5, 6, 9], [0, 2]),
                                      BranchTokens([50, 51], [1])])]
    many = [Group([3, 4, 5, 6], [BranchTokens([7, 8], [1]), BranchTokens([9], [0])]),
            Group([2, 7, 11, 19, 23], [BranchTokens([5, 6, 9], [2, 0, 1])]),
            Group([12, 13], [BranchTokens([14, 15, 16], [0, 2])])]
    return one, many


def test_pinned_and_pageable_outputs_agree(device):
    m = RefModel(*gemma4(), 29, O.Q4, O.Q8)
    eng = m.engine(64, 16, device)
    one, many = requests()
    pinned_pool = eng._pool
    for want in (Want.HIDDEN, Want.LOGITS):
        for groups in (one, many):
            eng.evict_resident()
            eng._pool = pinned_pool
            a = eng.evaluate_groups(groups, want)
            base = a[0].branches[0].rows.base
            while getattr(base, "base", None) is not None:
                base = base.base
            assert type(base).__name__ == "_HostBlock"
            eng.evict_resident()
            eng._pool = types.SimpleNamespace(
                array=lambda shape: np.empty(shape, dtype=np.float32))
            b = eng.evaluate_groups(groups, want)
            for ga, gb in zip(a, b):
                for ba, bb in zip(ga.branches, gb.branches):
                    assert np.array_equal(ba.rows, bb.rows)
    eng._pool = pinned_pool
    eng.close()


def test_output_arrays_outlive_later_calls(device):
    m = RefModel(*gemma4(), 31, O.Q8, O.Q8)
    eng = m.engine(64, 16, device)
    one, many = requests()
    first = eng.evaluate_groups(one, Want.LOGITS)
    kept = [b.rows.copy() for b in first[0].branches]
    for _ in range(6):
        eng.evict_resident()
        eng.evaluate_groups(many, Want.LOGITS)
    for b, k in zip(first[0].branches, kept):
        assert np.array_equal(b.rows, k)
    eng.close()


def test_host_alloc_entry_points(device):
    lib = _lib.lib()
    p = _lib.C.c_void_p()
    assert lib.omg_host_alloc(device, 1 << 20, _lib.C.byref(p)) == 0 and p.value
    lib.omg_host_free(p)
    lib.omg_host_free(None)
    assert lib.omg_host_alloc(device, 1, None) == -1
    assert "null argument" in lib.omg_last_error().decode()
