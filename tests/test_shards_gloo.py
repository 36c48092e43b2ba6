"""Host logic of the multi-GPU path, run as two gloo ranks on the CPU.

The sharded vocoder configuration keeps one slab of a signal per rank and
needs one exchange: the global abs-max, an integer MAX all-reduce of each
slab's abs-max bit pattern (m3.c_b200/shards.py).  Here each rank computes
its slab's snake output and abs-max with the CPU oracle, the ranks exchange
through the same function the benchmark calls, and the result must equal the
oracle's abs-max of the whole (concatenated) signal.  The slowest-rank timing
helper is checked the same way.
"""

from __future__ import annotations

import importlib.util
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORLD = 2
SHAPE = (2, 8, 1024)  # [batch, channels, time] slab per rank


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


def _slab(m3, shards, rank: int):
    n = int(np.prod(SHAPE))
    x = m3.fill_normal(4, shards.shard_sequence(0, rank), 0.0, 0.5, n).reshape(SHAPE)
    alpha = m3.fill_uniform(4, 1, 0.2, 2.0, SHAPE[1]).reshape(1, SHAPE[1], 1)
    return x, alpha


def _snake_abs_max(oracle, x, alpha) -> np.ndarray:
    z = np.empty_like(x)
    assert oracle.run("snake1d", x, alpha, z) == 0
    m = np.zeros(1, np.float32)
    assert oracle.run("abs_max", z, m) == 0
    return m


def _rank_main(rank: int, port: int) -> None:
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        m3, oracle, shards = _modules()
        m3.load()
        oracle.restatement()
        x, alpha = _slab(m3, shards, rank)
        local = _snake_abs_max(oracle, x, alpha)
        word = torch.tensor([int(local.view(np.int32)[0])], dtype=torch.int32)
        shards.global_abs_max_bits(word)

        # the whole signal: every rank's slab along the time axis
        whole = np.concatenate([_slab(m3, shards, r)[0] for r in range(WORLD)], axis=2)
        expected = _snake_abs_max(oracle, whole, alpha)
        assert int(word.item()) == int(expected.view(np.int32)[0])
        if rank == 0:
            other = _slab(m3, shards, 1)[0]
            assert not np.array_equal(x, other), "slabs must be distinct draws"

        slowest = shards.max_over_ranks(1.5 + rank, torch.device("cpu"))
        assert slowest == 1.5 + WORLD - 1
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_abs_max_matches_whole_signal():
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(_free_port(),), nprocs=WORLD, join=True,
                       start_method="spawn")


def test_shard_sequence_rules():
    _, _, shards = _modules()
    assert shards.shard_sequence(3, 0) == 3
    assert shards.shard_sequence(3, 2) == 3 + 2 * shards.SEQUENCE_STRIDE
    with pytest.raises(ValueError):
        shards.shard_sequence(64, 0)
