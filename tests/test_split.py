"""Host logic of one state's branches split across ranks (grande_b200/split.py),
on the CPU: the branch shares, and the prefill -> broadcast -> import ->
share -> all-gather sequence run as world-size 2 and 3 `gloo` process groups
over a stand-in engine whose state image lives in host memory. The stand-in
refuses to evaluate branches over a prefix that is not resident, and derives
every output row from the K/V image it holds, so a rank that skipped the
import or received the wrong bytes gives different rows."""
import ctypes
import os
import socket
import zlib

import numpy as np
import pytest

from grande_b200.split import branch_shares


def test_branch_shares_cover_every_branch_once():
    for n in range(0, 30):
        for world in range(1, 9):
            shares = branch_shares(n, world)
            assert len(shares) == world
            assert shares[0][0] == 0 and shares[-1][1] == n
            for (lo, hi), (lo2, _) in zip(shares, shares[1:]):
                assert hi == lo2
            sizes = [hi - lo for lo, hi in shares]
            assert max(sizes) - min(sizes) <= 1
            assert sizes == sorted(sizes, reverse=True)


def test_branch_shares_rejects_bad_sizes():
    with pytest.raises(ValueError):
        branch_shares(3, 0)
    with pytest.raises(ValueError):
        branch_shares(-1, 2)


class HostEngine:
    """The parts of grande_b200.engine.Engine that split.py calls, with the
    state image in host memory (8 bytes per prefix token)."""

    def __init__(self):
        self.resident = None
        self.kv = b""
        self.passes = []

    @staticmethod
    def _image(prefix):
        return b"".join(zlib.crc32(bytes([i % 251, t % 251])).to_bytes(4, "little") * 2
                        for i, t in enumerate(prefix))

    def state_image_bytes(self, n):
        return 8 * n

    def is_resident(self, prefix):
        return self.resident == list(prefix)

    def evaluate(self, prefix, branches, want):
        from grande_b200.engine import BranchOutput
        if not branches:
            self.resident, self.kv = list(prefix), self._image(prefix)
            self.passes.append(("prefill", len(prefix)))
            return []
        if not self.is_resident(prefix):
            raise AssertionError("branches evaluated over a prefix that is not resident")
        self.passes.append(("branches", len(branches)))
        seed = zlib.crc32(self.kv)
        out = []
        for b in branches:
            rows = [np.full(4, float(zlib.crc32(bytes(b.tokens[:w + 1]), seed) % 1000), np.float32)
                    for w in b.want]
            out.append(BranchOutput(np.stack(rows)))
        return out

    def export_state_device(self, prefix, dst, cap):
        assert self.is_resident(prefix) and cap >= len(self.kv)
        ctypes.memmove(dst, self.kv, len(self.kv))

    def import_state_device(self, prefix, src, nbytes):
        self.kv = ctypes.string_at(src, nbytes)
        self.resident = list(prefix)


def _request():
    from grande_b200.engine import BranchTokens
    prefix = [7, 3, 250, 9, 11, 40, 2, 2, 8]
    branches = [BranchTokens([i + 1, 2 * i + 3, 5], [0, 2]) for i in range(7)]
    return prefix, branches


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from grande_b200.engine import Want
    from grande_b200.split import evaluate_split
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        eng = HostEngine()
        prefix, branches = _request()
        out = evaluate_split(eng, prefix, branches, Want.LOGITS, src=world - 1, device="cpu")
        q.put((rank, [o.rows for o in out], eng.passes))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_split_matches_one_engine(world):
    import torch.multiprocessing as mp
    from grande_b200.engine import Want
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, rows, passes = q.get(timeout=120)
        results[rank] = (rows, passes)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    prefix, branches = _request()
    one = HostEngine()
    one.evaluate(prefix, [], Want.LOGITS)
    expect = [o.rows for o in one.evaluate(prefix, branches, Want.LOGITS)]
    shares = branch_shares(len(branches), world)
    for rank, (rows, passes) in results.items():
        assert len(rows) == len(expect)
        for a, b in zip(rows, expect):
            assert np.array_equal(a, b)
        # Only the source rank prefills; every rank runs just its own share.
        lo, hi = shares[rank]
        expect_passes = ([("prefill", len(prefix))] if rank == world - 1 else [])
        expect_passes += [("branches", hi - lo)] if hi > lo else []
        assert passes == expect_passes
