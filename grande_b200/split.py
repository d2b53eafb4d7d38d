"""One state's branches evaluated on several GPUs.

The reference evaluates a state and all of its branches on one device
(``Engine::evaluate``, crates/omg-wgpu/src/engine.rs:1386-1398): the prefix's
K/V rows are computed once and every branch attends to them
(``attention.wgsl:70-76``). When one state carries more branches than one GPU
should run (or its latency matters more than throughput), the branches can be
split across the ranks of a process group, one engine per GPU with the
weights replicated:

1. rank ``src`` prefills the prefix alone; it becomes resident there;
2. its K/V rows (the f16 payload of ``save_state``, sliding layers
   window-only, engine.rs:1966-1981) are packed into one device buffer and
   sent to every rank with one NCCL broadcast over NVLink -- the only
   collective on the forward path;
3. every other rank imports the image, which makes the prefix resident there
   exactly as ``restore_state`` would (engine.rs:2051-2092);
4. each rank evaluates its contiguous share of the branches against the
   resident prefix (branches only, no prefix rows);
5. the rows are all-gathered, so every rank returns all branches' outputs in
   branch order.

A branch attends only to the prefix and to itself, so its rows do not depend
on which other branches share its pass: the split result equals the
single-GPU one row for row.
"""
from __future__ import annotations

from typing import Optional, Sequence

import numpy as np

from .engine import BranchOutput, Want


def branch_shares(n_branches: int, world: int) -> list[tuple[int, int]]:
    """Contiguous [lo, hi) branch ranges per rank; the first
    ``n_branches % world`` ranks take one branch more. Ranks past the branch
    count get empty ranges."""
    if world <= 0:
        raise ValueError(f"world size must be positive (got {world})")
    if n_branches < 0:
        raise ValueError(f"branch count must be non-negative (got {n_branches})")
    base, extra = divmod(n_branches, world)
    out, lo = [], 0
    for r in range(world):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def share_prefix(engine, prefix: Sequence[int], *, src: int = 0, group=None, device=None,
                 want: Want = Want.LOGITS) -> int:
    """Make ``prefix`` resident on every rank of ``group``: rank ``src``
    prefills it (unless it is resident there already) and broadcasts the K/V
    image. Returns the image's size in bytes."""
    import torch
    import torch.distributed as dist

    rank = dist.get_rank(group)
    nbytes = engine.state_image_bytes(len(prefix))
    dev = torch.device("cuda", engine.device) if device is None else torch.device(device)
    buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    if rank == src:
        if not engine.is_resident(prefix):
            engine.evaluate(prefix, [], want)
        if dev.type == "cuda":
            # The buffer comes from torch's caching allocator, which orders it
            # only against torch's stream; the export writes it on the
            # engine's own stream.
            torch.cuda.current_stream(dev).synchronize()
        engine.export_state_device(prefix, buf.data_ptr(), nbytes)
    dist.broadcast(buf, src=dist.get_global_rank(group, src) if group is not None else src,
                   group=group)
    if rank != src:
        if dev.type == "cuda":
            # The broadcast ran on torch's stream; the import reads the buffer
            # on the engine's own stream.
            torch.cuda.current_stream(dev).synchronize()
        engine.import_state_device(prefix, buf.data_ptr(), nbytes)
    return nbytes


def evaluate_split(engine, prefix: Sequence[int], branches: Sequence, want: Want, *,
                   src: int = 0, group=None, device=None) -> list[BranchOutput]:
    """``Engine::evaluate`` of one state with its branches shared out over
    the ranks of ``group`` (module docstring). Every rank passes the same
    prefix and branches and gets every branch's output, in branch order."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    share_prefix(engine, prefix, src=src, group=group, device=device, want=want)
    lo, hi = branch_shares(len(branches), world)[rank]
    mine = engine.evaluate(prefix, list(branches[lo:hi]), want) if hi > lo else []
    parts: list[Optional[list[np.ndarray]]] = [None] * world
    dist.all_gather_object(parts, [np.asarray(o.rows) for o in mine], group=group)
    return [BranchOutput(rows) for part in parts for rows in part]
