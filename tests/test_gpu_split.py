"""A state's K/V moved between engines as a device image (the path that lets
one state's branches run on several GPUs, grande_b200/split.py), through the
C ABI: the image is save_state's payload byte for byte, an engine that
imports it evaluates branches exactly as the engine that prefilled it, and
the request errors are clear. The last test runs evaluate_split over NCCL on
two GPUs when the box has them."""
import os
import socket
import struct

import numpy as np
import pytest

from grande_b200.engine import BranchTokens, OmgError, PrefixSource, Want
from oracle import oracle as O

from refmodels import RefModel, gemma3, gemma4, gemma4_gqa

pytestmark = pytest.mark.gpu

F16, Q8, Q4 = O.F16, O.Q8, O.Q4

PREFIX = [2, 5, 9, 14, 20, 31, 7, 8, 3, 22, 1]
BRANCHES = [BranchTokens([11, 12, 13, 14, 15], [1, 4]), BranchTokens([30, 31, 32], [0, 2]),
            BranchTokens([33, 34, 35, 36, 37, 38], [5]), BranchTokens([4, 6], [0, 1])]


def models():
    return [RefModel(*gemma3(), 23, F16, F16), RefModel(*gemma4(), 23, Q4, Q8),
            RefModel(*gemma4_gqa(), 23, Q4, Q8)]


def payload(state_bytes: bytes) -> bytes:
    """The layer payloads of a GRWS1 image, concatenated (engine.rs:516-534)."""
    at = 6
    (n,) = struct.unpack_from("<I", state_bytes, at)
    at += 4 + n
    (n,) = struct.unpack_from("<I", state_bytes, at)
    at += 4 + 4 * n
    (layers,) = struct.unpack_from("<I", state_bytes, at)
    at += 4
    out = b""
    for _ in range(layers):
        _, _, n = struct.unpack_from("<III", state_bytes, at)
        at += 12
        out += state_bytes[at:at + n]
        at += n
    return out


def test_state_image_moves_a_prefill_between_engines(device):
    import torch
    for m in models():
        a, b = m.engine(device=device), m.engine(device=device)
        assert a.evaluate(PREFIX, [], Want.HIDDEN) == []
        assert a.is_resident(PREFIX)
        n = a.state_image_bytes(len(PREFIX))
        st = a.save_state(PREFIX)
        assert n == st.byte_len() - 4 * len(PREFIX)
        img = torch.empty(n, dtype=torch.uint8, device=f"cuda:{device}")
        a.export_state_device(PREFIX, img.data_ptr(), n)
        assert img.cpu().numpy().tobytes() == payload(st.to_bytes("m"))
        b.import_state_device(PREFIX, img.data_ptr(), n)
        assert b.is_resident(PREFIX)
        got = b.evaluate(PREFIX, BRANCHES, Want.HIDDEN)
        assert b.prefix_source() == PrefixSource.RESIDENT
        want = a.evaluate(PREFIX, BRANCHES, Want.HIDDEN)
        assert a.prefix_source() == PrefixSource.RESIDENT
        for x, y in zip(got, want):
            assert np.array_equal(x.rows, y.rows)
        # ...and a cold pass of the whole request gives the same rows.
        a.evict_resident()
        cold = a.evaluate(PREFIX, BRANCHES, Want.LOGITS)
        again = b.evaluate(PREFIX, BRANCHES, Want.LOGITS)
        for x, y in zip(cold, again):
            assert np.array_equal(x.rows, y.rows)
        a.close()
        b.close()


def test_state_image_errors(device):
    import torch
    m = RefModel(*gemma3(), 29, F16, F16)
    a = m.engine(device=device)
    n = a.state_image_bytes(len(PREFIX))
    img = torch.empty(n, dtype=torch.uint8, device=f"cuda:{device}")
    with pytest.raises(OmgError, match="not resident"):
        a.export_state_device(PREFIX, img.data_ptr(), n)
    a.evaluate(PREFIX, [], Want.HIDDEN)
    with pytest.raises(OmgError, match="buffer holds"):
        a.export_state_device(PREFIX, img.data_ptr(), n - 1)
    host = np.zeros(n, np.uint8)
    with pytest.raises(OmgError, match="not device memory"):
        a.export_state_device(PREFIX, host.ctypes.data, n)
    with pytest.raises(OmgError, match="expected"):
        a.import_state_device(PREFIX, img.data_ptr(), n - 2)
    with pytest.raises(OmgError, match="not device memory"):
        a.import_state_device(PREFIX, host.ctypes.data, n)
    with pytest.raises(OmgError, match="exceeds the engine capacity"):
        a.import_state_device(list(range(1, 66)), img.data_ptr(), a.state_image_bytes(65))
    # A failed call leaves the resident prefix as it was.
    assert a.is_resident(PREFIX)
    a.close()


def _split_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from grande_b200.split import evaluate_split
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        out = []
        for m in models():
            eng = m.engine(device=rank)
            rows = evaluate_split(eng, PREFIX, BRANCHES, Want.HIDDEN)
            out.append([r.rows for r in rows])
            eng.close()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_split_across_two_gpus(device):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_split_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for mi, m in enumerate(models()):
        eng = m.engine(device=device)
        one = eng.evaluate(PREFIX, BRANCHES, Want.HIDDEN)
        eng.close()
        for rank in range(2):
            rows = got[rank][mi]
            assert len(rows) == len(one)
            for x, y in zip(rows, one):
                # The branches sit at other cache rows than in the one-GPU
                # pass; the reference's layout tolerance (reference.rs:716-735).
                scale = max(float(np.abs(y.rows).max()), 1.0)
                assert float(np.abs(x - y.rows).max()) <= 1e-4 * scale
