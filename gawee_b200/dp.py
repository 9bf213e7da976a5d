"""Data parallelism for batched inference: batch sharding with replicated weights.

Every rank runs the same graph on a contiguous slice of the batch (for
ResNet-18 at batch 256 on W GPUs: 256/W images per rank; for the decoder:
64/W sequences).  No op of these graphs mixes batch rows, so the only
communication is gathering each rank's output rows to rank 0.  On GPUs that
gather is one NCCL send/recv group issued by libgawee_cuda
(`gawee_dp_gather_output`); the rendezvous (sharing the NCCL id) goes through
`torch.distributed`, which is plumbing only.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import numpy as np


def shard_range(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) rows of `total` for `rank`; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def shard_args(args: Sequence[np.ndarray], batched: Sequence[bool], world: int, rank: int) -> List[np.ndarray]:
    """Slice the batched arguments (leading dim) for `rank`; weights are replicated."""
    out = []
    for a, b in zip(args, batched):
        if b:
            s, e = shard_range(a.shape[0], world, rank)
            out.append(np.ascontiguousarray(a[s:e]))
        else:
            out.append(a)
    return out


def assemble(parts: Sequence[np.ndarray]) -> np.ndarray:
    """Rank-ordered concatenation of per-rank output rows (what rank 0 receives)."""
    return np.concatenate(list(parts), axis=0)


def share_nccl_id(uid: bytes, rank: int, group=None) -> bytes:
    """Broadcast rank 0's NCCL unique id to every rank over torch.distributed."""
    import torch
    import torch.distributed as dist

    t = torch.zeros(128, dtype=torch.uint8)
    if rank == 0:
        t[:] = torch.frombuffer(bytearray(uid), dtype=torch.uint8)
    if dist.get_backend(group) == "nccl":
        t = t.cuda()
    dist.broadcast(t, src=0, group=group)
    return bytes(t.cpu().numpy().tobytes())


def gather_offsets(rows: Sequence[int]) -> List[int]:
    """Row offset of each rank's block in the gathered output (rank order);
    what libgawee_cuda computes from the sizes exchanged at gawee_dp_init."""
    out, acc = [], 0
    for r in rows:
        if r < 0:
            raise ValueError("negative row count")
        out.append(acc)
        acc += r
    return out


def gather_rows_host(local: np.ndarray, rank: int, world: int, group=None):
    """Host-side gather of row blocks to rank 0 (gloo), in rank order; the
    blocks may differ in length (shards of an uneven batch).  Returns the
    assembled array on rank 0 and None elsewhere.  Used where no GPU exists.
    Like gawee_dp_init / gawee_dp_gather_output, the ranks first exchange
    their row counts, then rank 0 places each block at its offset."""
    import torch
    import torch.distributed as dist

    local = np.ascontiguousarray(local)
    counts = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(counts, torch.tensor([local.shape[0]], dtype=torch.int64), group=group)
    rows = [int(c.item()) for c in counts]
    width = max(rows)
    padded = np.zeros((width,) + local.shape[1:], local.dtype)
    padded[:local.shape[0]] = local
    t = torch.from_numpy(padded)
    parts = [torch.empty_like(t) for _ in range(world)] if rank == 0 else None
    dist.gather(t, gather_list=parts, dst=0, group=group)
    if rank != 0:
        return None
    out = np.empty((sum(rows),) + local.shape[1:], local.dtype)
    for r, off in enumerate(gather_offsets(rows)):
        out[off:off + rows[r]] = parts[r].numpy()[:rows[r]]
    return out
