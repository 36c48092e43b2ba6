"""Host logic of the sharding layer, run as gloo ranks on the CPU.

* Every rank plans its slabs with the library's host-only partition
  (m3_cuda_shard_plan, no GPU); gathered over the ranks, the slabs of each
  split value tile its split axis exactly, in rank order, and replicated
  values (a snake alpha split along time, a norm scale, scalar constants)
  stay whole.
* The exchange the library runs after each C5 run, a MAX all-reduce of each
  slab's abs-max bit pattern, gives the whole signal's abs-max: each rank
  computes its slab's snake and abs-max with the CPU oracle on the slab the
  partition assigns it.
* The communicator id reaches every rank unchanged (shards.shared_shard_id)
  and the slowest-rank timing helper takes the maximum.
"""

from __future__ import annotations

import importlib.util
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _load(name: str, path: str):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


def _modules():
    m3 = _load("m3cuda", os.path.join(ROOT, "m3.c_b200", "m3cuda.py"))
    oracle = _load("m3_oracle_py", os.path.join(ROOT, "oracle", "oracle.py"))
    shards = _load("m3_shards", os.path.join(ROOT, "m3.c_b200", "shards.py"))
    return m3, oracle, shards


SIGNAL = (2, 8, 1028)   # [batch, channels, time], time split (1028 = 4 * 257)


def _snake_graph(m3, alpha):
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, SIGNAL)
    a = g.constant(m3.F32, alpha)
    z = g.inferred("SNAKE1D", [x, a], m3.TEMPORARY, m3.F32)
    g.node("SNAKE1D", [x, a], [z])
    m = g.inferred("ABS_MAX", [z], m3.OUTPUT, m3.F32)
    g.node("ABS_MAX", [z], [m])
    y = g.inferred("CLAMP_UNIT", [z], m3.OUTPUT, m3.F32)
    g.node("CLAMP_UNIT", [z], [y])
    return g, (x, a, m, y)


def _rank_main(rank: int, world: int, port: int) -> None:
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m3, oracle, shards = _modules()
        m3.load()
        oracle.restatement()
        signal = m3.fill_normal(4, 0, 0.0, 0.5, int(np.prod(SIGNAL))).reshape(SIGNAL)
        alpha = m3.fill_uniform(4, 1, 0.2, 2.0, SIGNAL[1]).reshape(1, SIGNAL[1], 1)
        g, (x, a, m, y) = _snake_graph(m3, alpha)

        slab, axis = m3.shard_plan(g, rank, world, 2, x)
        assert axis == 2 and slab.split and slab.axis == 2
        assert m3.shard_plan(g, rank, world, 2, a)[0].split is False
        assert m3.shard_plan(g, rank, world, 2, m)[0].split is False
        ys = m3.shard_plan(g, rank, world, 2, y)[0]
        assert (ys.begin, ys.extent) == (slab.begin, slab.extent)
        # the slabs tile the time axis in rank order, in whole 4-blocks
        mine = torch.tensor([slab.begin, slab.extent], dtype=torch.int64)
        every = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(every, mine)
        begin = 0
        for part in every:
            assert int(part[0]) == begin and int(part[1]) % 4 == 0
            begin += int(part[1])
        assert begin == SIGNAL[2]

        # the per-run exchange: MAX of each slab's abs-max bits
        part = np.ascontiguousarray(signal[:, :, slab.begin:slab.begin + slab.extent])
        z = np.empty_like(part)
        assert oracle.run("snake1d", part, alpha, z) == 0
        local = np.zeros(1, np.float32)
        assert oracle.run("abs_max", z, local) == 0
        word = torch.tensor([int(local.view(np.uint32)[0])], dtype=torch.int64)
        dist.all_reduce(word, op=dist.ReduceOp.MAX)
        whole = np.empty_like(signal)
        assert oracle.run("snake1d", signal, alpha, whole) == 0
        expected = np.zeros(1, np.float32)
        assert oracle.run("abs_max", whole, expected) == 0
        assert int(word.item()) == int(expected.view(np.uint32)[0])

        # rows of a softmax graph split along rows, never along the row axis
        gs = m3.Graph()
        xs = gs.value(m3.INPUT, m3.F32, (37, 64))
        ps = gs.inferred("SOFTMAX", [xs], m3.OUTPUT, m3.F32)
        gs.node("SOFTMAX", [xs], [ps])
        rows, axis = m3.shard_plan(gs, rank, world, m3.ShardOptions.AXIS_AUTO, xs)
        assert axis == 0 and rows.local.shape[1] == 64
        counts = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(counts, torch.tensor([rows.extent], dtype=torch.int64))
        assert sum(int(c) for c in counts) == 37
        with pytest.raises(m3.M3Failure) as failure:
            m3.shard_plan(gs, rank, world, 1, xs)
        assert failure.value.status == m3.UNSUPPORTED

        # the communicator id and the slowest-rank time
        ident = shards.shared_shard_id(m3)
        digest = torch.tensor(list(ident.bytes), dtype=torch.int64)
        first = digest.clone()
        dist.broadcast(first, src=0)
        assert torch.equal(first, digest)
        slowest = shards.max_over_ranks(1.5 + rank, torch.device("cpu"))
        assert slowest == 1.5 + world - 1
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_shard_partition_and_exchange(world):
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(world, _free_port()), nprocs=world, join=True,
                       start_method="spawn")


def test_shard_plan_rules():
    m3, _, _ = _modules()
    m3.load()
    alpha = np.ones((1, SIGNAL[1], 1), np.float32)
    g, (x, a, m, y) = _snake_graph(m3, alpha)
    # the automatic axis is the outermost one every value allows
    slab, axis = m3.shard_plan(g, 1, 2, m3.ShardOptions.AXIS_AUTO, x)
    assert axis == 0 and (slab.begin, slab.extent) == (1, 1)
    # the channel axis splits alpha along with the signal
    alpha_slab = m3.shard_plan(g, 1, 2, 1, a)[0]
    assert alpha_slab.split and (alpha_slab.begin, alpha_slab.extent) == (4, 4)
    # more shards than the axis holds, a bad rank, an axis outside the rank
    for rank, count, axis in ((0, 3, 0), (2, 2, 2), (0, 2, 3)):
        with pytest.raises(m3.M3Failure):
            m3.shard_plan(g, rank, count, axis, x)
    # an ABS_MAX result may not feed another node of a sharded graph
    h = m3.Graph()
    hx = h.value(m3.INPUT, m3.F32, (8, 16))
    hm = h.inferred("ABS_MAX", [hx], m3.TEMPORARY, m3.F32)
    h.node("ABS_MAX", [hx], [hm])
    hy = h.inferred("MUL", [hx, hm], m3.OUTPUT, m3.F32)
    h.node("MUL", [hx, hm], [hy])
    with pytest.raises(m3.M3Failure):
        m3.shard_plan(h, 0, 2, 0, hx)
