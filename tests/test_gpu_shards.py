"""The sharding layer on the GPU.

On one GPU (no communicator): every rank's shard session of a graph runs in
turn on device 0, each fed its slab out of the global input through
m3_cuda_shard_write_input and drained into its place of a global output
buffer through m3_cuda_shard_read_output.  The assembled outputs must equal
the unsharded session's bit for bit; a global abs-max, which without a
communicator each rank reduces over its own slab, must combine (MAX of the
bit patterns) to the unsharded result.

On two GPUs (skipped with fewer): two processes join one NCCL communicator
through the library; the global abs-max arrives on both ranks after one
run, and a NaN in rank 1's slab fails the run on BOTH ranks while their
committed outputs stay as they were.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _snake_graph(m3, shape, alpha):
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, shape)
    a = g.constant(m3.F32, alpha)
    z = g.inferred("SNAKE1D", [x, a], m3.TEMPORARY, m3.F32)
    g.node("SNAKE1D", [x, a], [z])
    m = g.inferred("ABS_MAX", [z], m3.OUTPUT, m3.F32)
    g.node("ABS_MAX", [z], [m])
    y = g.inferred("CLAMP_UNIT", [z], m3.OUTPUT, m3.F32)
    g.node("CLAMP_UNIT", [z], [y])
    return g, x, m, y


def _softmax_graph(m3, shape):
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, shape)
    p = g.inferred("SOFTMAX", [x], m3.OUTPUT, m3.F32)
    g.node("SOFTMAX", [x], [p])
    v = g.inferred("TOP_K", [x], m3.OUTPUT, m3.F32, 0, k=1)
    i = g.inferred("TOP_K", [x], m3.OUTPUT, m3.I32, 1, k=1)
    g.node("TOP_K", [x], [v, i], k=1)
    return g, x, (p, v, i)


@pytest.mark.parametrize("count", [2, 3])
def test_time_shards_assemble_to_the_whole(m3, gpu, count):
    shape = (2, 16, 4100)
    x_host = m3.fill_normal(4, 0, 0.0, 0.5, int(np.prod(shape))).reshape(shape)
    x_host[1, 3, 17] = 40.0        # one large value, in one slab only
    alpha = m3.fill_uniform(4, 1, 0.2, 2.0, shape[1]).reshape(1, shape[1], 1)
    g, x, m, y = _snake_graph(m3, shape, alpha)
    whole = m3.Session(g)
    whole.write(x, x_host)
    whole.run()
    want_y = whole.read(y)
    want_m = whole.read(m)
    whole.close()
    got_y = np.full(shape, np.nan, np.float32)
    maxima = []
    for rank in range(count):
        s = m3.Session(g, shard=m3.ShardOptions(rank, count, 2, None))
        slab = s.shard_slab(x)
        assert slab.split and slab.axis == 2
        s.shard_write(x, x_host.ctypes.data, x_host.nbytes)
        s.run()
        s.shard_read(y, got_y.ctypes.data, got_y.nbytes)
        maxima.append(int(s.read(m).view(np.uint32)[0]))
        s.close()
    assert np.array_equal(got_y.view(np.uint32), want_y.view(np.uint32))
    assert max(maxima) == int(want_m.view(np.uint32)[0])


@pytest.mark.parametrize("count", [2, 4])
def test_row_shards_assemble_to_the_whole(m3, gpu, count):
    import torch

    shape = (1030, 1024)
    x_host = m3.fill_normal(1, 0, 0.0, 3.0, int(np.prod(shape))).reshape(shape)
    x_host[m3.fill_uniform(1, 1, 0.0, 1.0, x_host.size).reshape(shape) < 0.01] = 20.0
    g, x, outs = _softmax_graph(m3, shape)
    whole = m3.Session(g)
    whole.write(x, x_host)
    whole.run()
    want = [whole.read(v) for v in outs]
    whole.close()
    device_x = torch.from_numpy(x_host).cuda()
    torch.cuda.synchronize()
    got = [np.zeros_like(w) for w in want]
    for rank in range(count):
        s = m3.Session(g, shard=m3.ShardOptions(rank, count, m3.ShardOptions.AXIS_AUTO, None))
        assert s.shard_slab(x).axis == 0
        s.shard_write(x, device_x.data_ptr(), x_host.nbytes, device=True)
        s.run()
        for v, buf in zip(outs, got):
            s.shard_read(v, buf.ctypes.data, buf.nbytes)
        s.close()
    for w, gt in zip(want, got):
        assert np.array_equal(w.view(np.uint8), gt.view(np.uint8))


def test_shard_of_one_is_the_whole_session(m3, gpu):
    shape = (64, 256)
    x_host = m3.fill_normal(1, 0, 0.0, 1.0, int(np.prod(shape))).reshape(shape)
    g, x, outs = _softmax_graph(m3, shape)
    s = m3.Session(g, shard=m3.ShardOptions(0, 1, m3.ShardOptions.AXIS_AUTO, None))
    s.write(x, x_host)
    s.run()
    t = m3.Session(g)
    t.write(x, x_host)
    t.run()
    for v in outs:
        assert np.array_equal(s.read(v).view(np.uint8), t.read(v).view(np.uint8))
    s.close()
    t.close()


# ------------------------------------------------------------ two GPUs

def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _nccl_rank(rank: int, port: int, shape, queue) -> None:
    import importlib.util
    import sys

    import torch
    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

    def load(name, path):
        spec = importlib.util.spec_from_file_location(name, path)
        module = importlib.util.module_from_spec(spec)
        sys.modules[name] = module
        spec.loader.exec_module(module)
        return module

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        m3 = load("m3cuda", os.path.join(root, "m3.c_b200", "m3cuda.py"))
        shards = load("m3_shards", os.path.join(root, "m3.c_b200", "shards.py"))
        m3.load()
        ident = shards.shared_shard_id(m3)
        x_host = m3.fill_normal(4, 0, 0.0, 0.5, int(np.prod(shape))).reshape(shape)
        alpha = m3.fill_uniform(4, 1, 0.2, 2.0, shape[1]).reshape(1, shape[1], 1)
        g, x, m, y = _snake_graph(m3, shape, alpha)
        s = m3.Session(g, device=rank,
                       shard=m3.ShardOptions(rank, 2, 2, ident, timeout_seconds=60.0))
        s.shard_write(x, x_host.ctypes.data, x_host.nbytes)
        s.run()
        first_m = s.read(m).copy()
        first_y = s.read(y).copy()
        # a NaN in rank 1's slab: both ranks fail, nothing is committed
        bad = x_host.copy()
        slab = s.shard_slab(x)
        if rank == 1:
            bad[0, 0, slab.begin + 3] = np.nan
        s.shard_write(x, bad.ctypes.data, bad.nbytes)
        status, message = s.run_status()
        queue.put((rank, int(first_m.view(np.uint32)[0]), status, message,
                   bool(np.array_equal(s.read(y).view(np.uint32), first_y.view(np.uint32))),
                   bool(np.array_equal(s.read(m).view(np.uint32), first_m.view(np.uint32)))))
        s.close()
    finally:
        dist.destroy_process_group()


def test_two_gpu_abs_max_all_reduce_and_shared_failure(m3, gpu):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    shape = (2, 8, 8192)
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    mp.start_processes(_nccl_rank, args=(_free_port(), shape, queue), nprocs=2, join=True,
                       start_method="spawn")
    results = sorted(queue.get(timeout=10) for _ in range(2))
    # the unsharded abs-max on one GPU
    x_host = m3.fill_normal(4, 0, 0.0, 0.5, int(np.prod(shape))).reshape(shape)
    alpha = m3.fill_uniform(4, 1, 0.2, 2.0, shape[1]).reshape(1, shape[1], 1)
    g, x, m, y = _snake_graph(m3, shape, alpha)
    whole = m3.Session(g)
    whole.write(x, x_host)
    whole.run()
    want = int(whole.read(m).view(np.uint32)[0])
    whole.close()
    for rank, got, status, message, y_kept, m_kept in results:
        assert got == want, f"rank {rank} abs-max"
        assert status == m3.OUT_OF_RANGE and "NaN" in message, f"rank {rank}: {message}"
        assert y_kept and m_kept
