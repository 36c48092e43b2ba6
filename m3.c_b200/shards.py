"""Host plumbing of the sharding layer for torchrun jobs (one process per GPU).

The partition, the per-rank arenas and the per-run NCCL all-reduce live in
the C library (m3_cuda_shard_session_create).  What a Python job adds is the
exchange of the communicator id, which the library leaves to the caller
(rank 0 creates it, everyone needs the same bytes), and the slowest-rank
timing of the benchmark.
"""

from __future__ import annotations


def shared_shard_id(m3, device=None, group=None):
    """One communicator id for all ranks of the default process group: rank 0
    creates it with m3_cuda_shard_id_create and broadcasts its 128 bytes
    (a CUDA tensor on `device` for NCCL, a CPU tensor for gloo)."""
    import torch
    import torch.distributed as dist

    data = torch.zeros(128, dtype=torch.uint8, device=device)
    if dist.get_rank(group) == 0:
        created = m3.shard_id()
        data.copy_(torch.tensor(list(created.bytes), dtype=torch.uint8))
    dist.broadcast(data, src=0, group=group)
    out = m3.ShardId()
    for i, b in enumerate(data.cpu().tolist()):
        out.bytes[i] = b
    return out


def max_over_ranks(milliseconds: float, device, group=None) -> float:
    """The slowest rank's time: every multi-GPU figure is the whole job's
    work divided by this."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([milliseconds], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
