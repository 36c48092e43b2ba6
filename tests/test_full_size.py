"""The benchmark configurations (BASELINE.json configs C1-C5) at their full
sizes, through the same graphs bench.py times, checked by properties that do
not depend on size and by comparisons on sampled rows/positions:

* C1, C4: every element, bit-exact against F32 numpy statements (each
  statement is one IEEE operation, as in the reference);
* C2: every row's max and argmax bit-exact; sampled rows' probabilities
  against the oracle within 1e-6 relative; every row sums to 1;
* C3: the residual sum bit-exact everywhere; sampled rows of RMSNorm
  (bit-exact) and gated SiLU (1 ulp) against the reference CPU provider;
* C5: the abs-max bit-exact against the oracle's abs-max of the oracle's
  snake over the WHOLE input (row slices on all host threads); sampled
  positions against the oracle's snake and clamp (0x1p-19);
* one element-wise launch over more than 2^32 elements (64-bit indexing).
"""

from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    if "m3_bench" not in sys.modules:
        spec = importlib.util.spec_from_file_location("m3_bench", os.path.join(ROOT, "bench.py"))
        module = importlib.util.module_from_spec(spec)
        sys.modules["m3_bench"] = module
        spec.loader.exec_module(module)
    return sys.modules["m3_bench"]


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype.itemsize == 4 else np.uint16)


def _rng(m3):
    return _bench().ProductRng(m3)


def _session(m3, name):
    cfg = _bench().CONFIGS[name]
    g = m3.Graph()
    handles, outputs = cfg.build(m3, g, _rng(m3))
    return cfg, m3.Session(g), handles, outputs


def test_c1_full_size_bit_exact(m3, oracle, gpu):
    cfg, s, h, o = _session(m3, "c1")
    x = cfg.inputs_host(_rng(m3))["x"]
    s.write(h["x"], x)
    s.run()
    c = m3.fill_uniform(0, 1, 0.5, 2.0, cfg.width)
    b = m3.fill_normal(0, 2, 0.0, 1.0, cfg.width)
    assert np.array_equal(_bits(s.read(o[0])), _bits((x * c) + b))


def test_c2_full_size(m3, oracle, gpu):
    cfg, s, h, o = _session(m3, "c2")
    x = cfg.inputs_host(_rng(m3))["x"]
    s.write(h["x"], x)
    s.run()
    probs, values, indices = (s.read(v) for v in o)
    assert np.array_equal(indices[:, 0], np.argmax(x, axis=1).astype(np.int32))
    assert np.array_equal(_bits(values[:, 0]), _bits(x.max(axis=1)))
    sums = probs.astype(np.float64).sum(axis=1)
    assert np.abs(sums - 1.0).max() < 1e-4
    rows = np.random.default_rng(0).choice(x.shape[0], 256, replace=False)
    for r in rows:
        want = np.zeros(x.shape[1], np.float32)
        assert oracle.run("softmax", x[r:r + 1].copy(), want.reshape(1, -1)) == 0
        got = probs[r].astype(np.float64)
        diff = np.abs(got - want)
        assert bool(np.all((diff <= 1e-6 * np.maximum(np.abs(got), np.abs(want))) | (got == want)))


def test_c3_full_size(m3, ref, oracle, gpu):
    cfg, s, h, o = _session(m3, "c3")
    data = cfg.inputs_host(_rng(m3))
    for name, vid in h.items():
        s.write(vid, data[name])
    s.run()
    total, normed, act = (s.read(v) for v in o)
    f16 = lambda bits: bits.view(np.float16).astype(np.float32)
    expect = (f16(data["h"]) + f16(data["r"])).astype(np.float16).view(np.uint16)
    assert np.array_equal(total, expect)
    # sampled rows through the reference CPU provider (rows are independent)
    rows = np.sort(np.random.default_rng(1).choice(cfg.rows, 48, replace=False))
    g = m3.Graph(lib=ref)
    sub = type(cfg)()
    sub.rows = len(rows)
    handles, outputs = sub.build(m3, g, _rng(m3))
    rs = m3.Session(g, allow_metal=False, allow_neural_engine=False, cuda=False)
    for name, vid in handles.items():
        rs.write(vid, np.ascontiguousarray(data[name][rows]))
    rs.run()
    ref_total, ref_normed, ref_act = (rs.read(v) for v in outputs)
    assert np.array_equal(total[rows], ref_total)
    assert np.array_equal(normed[rows], ref_normed)
    signed = lambda b: np.where(b & 0x8000, -(b & 0x7FFF), b & 0x7FFF).astype(np.int64)
    assert np.abs(signed(act[rows].astype(np.int64)) - signed(ref_act.astype(np.int64))).max() <= 1


def test_c4_full_size_thirty_steps_bit_exact(m3, oracle, gpu):
    cfg, s, h, o = _session(m3, "c4")
    data = cfg.inputs_host(_rng(m3))
    for name, vid in h.items():
        s.write(vid, data[name])
    s.run_steps(30, *cfg.carry)
    s.synchronize()
    x, vc, vu = data["x"].copy(), data["vc"], data["vu"]
    dt = np.float32(1.0) / np.float32(30.0)
    for _ in range(30):
        a = vu * np.float32(-1.0)
        a = vc + a
        a = a * np.float32(4.0)
        v = vu + a
        x = x + v * dt
    assert np.array_equal(_bits(s.read(o[0])), _bits(x))
    assert np.array_equal(s.read(o[1]), oracle.to_bf16(x))


def test_c5_full_size(m3, oracle, gpu):
    import torch

    bench = _bench()
    cfg = bench.CONFIGS["c5"]
    device = torch.device("cuda", 0)
    g = m3.Graph()
    handles, outputs = cfg.build(m3, g, _rng(m3))
    s = m3.Session(g, device=0, stream=torch.cuda.current_stream(device).cuda_stream)
    x = cfg.inputs_device(m3, torch, device)["x"]
    torch.cuda.synchronize(device)  # the session's stream does not wait on torch's
    s.write_device(handles["x"], x.data_ptr(), x.numel() * 4)
    s.run()
    m = float(s.read(outputs[0])[0])
    y = torch.empty_like(x)
    s.read_device(outputs[1], y.data_ptr(), y.numel() * 4)
    ymax = float(y.abs().max().item())
    assert m >= ymax and (ymax == m if m <= 1.0 else ymax == 1.0)
    assert float(y.min().item()) >= -1.0 and float(y.max().item()) <= 1.0
    # sampled positions against the oracle's snake (same alpha as the graph)
    alpha = m3.fill_uniform(4, 1, 0.2, 2.0, cfg.channels)
    flat = x.view(-1)
    pos = torch.randint(0, flat.numel(), (1 << 20,), device=device,
                        generator=torch.Generator(device=device).manual_seed(5))
    xs = flat[pos].cpu().numpy()
    ys = y.view(-1)[pos].cpu().numpy()
    channel = ((pos // cfg.length) % cfg.channels).cpu().numpy()
    z = np.empty_like(xs)
    for ch in np.unique(channel):
        sel = channel == ch
        xc = xs[sel].reshape(1, 1, -1).copy()
        zc = np.empty_like(xc)
        assert oracle.run("snake1d", xc, np.array([[[alpha[ch]]]], np.float32), zc) == 0
        z[sel] = zc.reshape(-1)
    want = np.clip(z, -1.0, 1.0)
    diff = np.abs(ys.astype(np.float64) - want)
    assert bool(np.all((diff <= 2.0 ** -19) | (diff <= 2.0 ** -19 * np.abs(want))))
    assert np.abs(z).max() <= m * (1 + 2.0 ** -19)
    s.close()
    # the abs-max bits against the oracle over the whole signal: snake of
    # each (batch, channel) row, then its abs-max, rows spread over threads
    host = x.cpu().numpy().reshape(-1, cfg.length)
    del x, y, flat
    torch.cuda.empty_cache()
    assert _oracle_abs_max_bits(oracle, host, alpha, cfg.channels) == \
        np.float32(m).view(np.uint32)


def _oracle_abs_max_bits(oracle, rows, alpha, channels):
    """max over rows of the oracle's abs-max of snake1d(row, alpha[channel])
    as F32 bits, rows processed by all host threads (ctypes releases the
    GIL)."""
    import threading

    threads = max(1, os.cpu_count() or 1)
    best = [0] * threads

    def work(t):
        z = np.empty((1, 1, rows.shape[1]), np.float32)
        out = np.zeros(1, np.float32)
        for r in range(t, rows.shape[0], threads):
            a = np.array([[[alpha[r % channels]]]], np.float32)
            assert oracle.run("snake1d", rows[r].reshape(1, 1, -1), a, z) == 0
            assert oracle.run("abs_max", z, out) == 0
            best[t] = max(best[t], int(out.view(np.uint32)[0]))

    workers = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
    for w in workers:
        w.start()
    for w in workers:
        w.join()
    return np.uint32(max(best))


def test_element_wise_beyond_two_to_the_32_elements(m3, gpu):
    """(x * 1.5) + (-0.25) over 2^32 + 12 elements: the 64-bit index path,
    checked at the first elements, across the 2^32 boundary, at the tail and
    at random positions against torch's IEEE F32 operations."""
    import torch

    n = (1 << 32) + 12
    device = torch.device("cuda", 0)
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (n,))
    c = g.constant(m3.F32, np.array([1.5], np.float32))
    d = g.constant(m3.F32, np.array([-0.25], np.float32))
    t = g.inferred("MUL", [x, c], m3.TEMPORARY, m3.F32)
    g.node("MUL", [x, c], [t])
    y = g.inferred("ADD", [t, d], m3.OUTPUT, m3.F32)
    g.node("ADD", [t, d], [y])
    s = m3.Session(g, device=0, stream=torch.cuda.current_stream(device).cuda_stream)
    data = torch.empty(n, dtype=torch.float32, device=device).uniform_(-4.0, 4.0)
    torch.cuda.synchronize(device)  # the session's stream does not wait on torch's
    s.write_device(x, data.data_ptr(), n * 4)
    s.run()
    out = torch.empty(n, dtype=torch.float32, device=device)
    s.read_device(y, out.data_ptr(), n * 4)
    s.close()
    picks = torch.cat([torch.arange(0, 16), torch.arange((1 << 32) - 8, n),
                       torch.randint(0, n, (100000,),
                                     generator=torch.Generator().manual_seed(3))]).to(device)
    want = (data[picks] * 1.5) + (-0.25)
    assert torch.equal(out[picks].view(torch.int32), want.view(torch.int32))
