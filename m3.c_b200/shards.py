"""Multi-GPU plumbing for the sharded configurations: one process per GPU,
torch.distributed for the host side, NCCL (or gloo on CPU) for the one real
exchange, the global abs-max of a signal sharded along time.

Each rank owns a slab of the logical signal (weak scaling: the slab size is
fixed per rank, so N ranks process an N-times longer signal).  Element-wise
and row operators need nothing from other ranks.  The abs-max of the whole
signal is the maximum of the per-slab abs-max bit patterns: |x| bit patterns
of non-NaN F32 values order like the values, so an integer MAX all-reduce of
one 32-bit word per rank is exact and independent of reduction order.
"""

from __future__ import annotations

SEQUENCE_STRIDE = 64


def shard_sequence(base_sequence: int, rank: int) -> int:
    """PCG32 stream selector of `rank`'s slab: each rank draws its slab from
    its own stream of the reference RNG (the stream id is the reference's
    `sequence` argument, src/m3_rng.c:22-31), so the slabs are independent
    draws of the configuration's distribution."""
    if base_sequence < 0 or base_sequence >= SEQUENCE_STRIDE or rank < 0:
        raise ValueError("sequence must be in [0, 64) and rank non-negative")
    return base_sequence + SEQUENCE_STRIDE * rank


def global_abs_max_bits(local_bits, group=None):
    """All-reduce (MAX) of one rank's abs-max bit pattern, in place.

    `local_bits` is a one-element int32 tensor on the rank's device (CUDA for
    NCCL, CPU for gloo) holding the raw bits of the slab's F32 abs-max, which
    lie in [0, 0x7f800000] and so compare correctly as signed integers."""
    import torch.distributed as dist

    if local_bits.numel() != 1:
        raise ValueError("one abs-max word per rank")
    dist.all_reduce(local_bits, op=dist.ReduceOp.MAX, group=group)
    return local_bits


def max_over_ranks(milliseconds: float, device, group=None) -> float:
    """The slowest rank's time: every multi-GPU figure is the whole job's
    work divided by this."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([milliseconds], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
