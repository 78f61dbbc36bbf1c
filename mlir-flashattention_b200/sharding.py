"""Slice sharding across ranks and the validation gather.

Every (batch, head) slice of the attention op is an independent problem, so N
processes (one per GPU) each own a contiguous block of slices and run with no
collective on the data path.  The collectives here run outside timed
regions: :func:`gather_rows` brings sampled outputs to rank 0 for checking
and :func:`rank_values` gathers each rank's timed duration (NCCL over NVLink
for CUDA tensors, gloo for CPU tensors).

For grouped-query attention a rank owns whole groups (all q-heads that share
a kv head), so it needs only its own K/V heads.
"""
from __future__ import annotations

from . import shard_slices  # noqa: F401  (re-exported)


def shard_groups(B: int, Hkv: int, world: int, rank: int):
    """Flat (batch, kv-head) group range [a, b) owned by ``rank``."""
    return shard_slices(B * Hkv, world, rank)


def gather_rows(t, world: int, rank: int, dst: int = 0):
    """Gather tensors of possibly different first-dimension sizes to ``dst``.

    Returns the list of per-rank tensors on ``dst`` and None elsewhere.  Every
    rank must call it (it pads to the largest shard, then trims).
    """
    import torch  # noqa: PLC0415
    import torch.distributed as dist  # noqa: PLC0415

    n = torch.tensor([t.shape[0]], dtype=torch.int64, device=t.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n)
    sizes = [int(s.item()) for s in sizes]
    m = max(sizes)
    pad = torch.zeros((m,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    pad[: t.shape[0]] = t
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad)
    if rank != dst:
        return None
    return [b[:s] for b, s in zip(bufs, sizes)]


def rank_values(x: float, world: int, device=None):
    """Every rank's value of ``x`` (a float), in rank order, on every rank.

    Every rank must call it; with one rank no collective is made."""
    if world == 1:
        return [float(x)]
    import torch  # noqa: PLC0415
    import torch.distributed as dist  # noqa: PLC0415

    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    return [float(v.item()) for v in parts]
