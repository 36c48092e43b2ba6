"""ROW_SUM (extension operator) on the GPU against the oracle's restatement:
the left-to-right F32 sum of each row, the order of the reference's softmax
sum (src/m3_op_execute_basic.c:150-158), so the results must be bit-exact.

Covered: the compiled-width F32 pipeline (ROW_SUM alone, and with TOP_K) at
the C2 shape [32768, 1024], the general tile kernel (F16/BF16 inputs, other
widths, fused with SOFTMAX and TOP_K in one row pass), the one-warp-per-row
kernel (ragged widths), empty rows, NaN propagation and the failure
semantics of a fused launch, and the backend plug-in command."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _sums(oracle, x, dtype=None):
    out = np.zeros(x.shape[:-1] + (1,), np.float32)
    assert oracle.run("row_sum", (x, dtype), out) == 0
    return out


def _graph(m3, shape, dtype, kinds):
    g = m3.Graph()
    x = g.value(m3.INPUT, dtype, shape)
    outs = []
    for kind in kinds:
        if kind == "ROW_SUM":
            r = g.inferred("ROW_SUM", [x], m3.OUTPUT, m3.F32)
            g.node("ROW_SUM", [x], [r])
            outs.append(r)
        elif kind == "SOFTMAX":
            p = g.inferred("SOFTMAX", [x], m3.OUTPUT, m3.F32 if dtype == m3.F32 else dtype)
            g.node("SOFTMAX", [x], [p])
            outs.append(p)
        else:
            tv = g.inferred("TOP_K", [x], m3.OUTPUT, m3.F32, 0, k=1)
            ti = g.inferred("TOP_K", [x], m3.OUTPUT, m3.I32, 1, k=1)
            g.node("TOP_K", [x], [tv, ti], k=1)
            outs += [tv, ti]
    return g, x, outs


def test_row_sum_c2_shape_bit_exact(m3, oracle, gpu):
    rows, width = 32768, 1024
    x = m3.fill_normal(1, 0, 0.0, 3.0, rows * width).reshape(rows, width)
    x[m3.fill_uniform(1, 1, 0.0, 1.0, rows * width).reshape(rows, width) < 0.01] = 20.0
    want = _sums(oracle, x)
    for kinds in (["ROW_SUM"], ["TOP_K", "ROW_SUM"]):
        g, v, outs = _graph(m3, x.shape, m3.F32, kinds)
        s = m3.Session(g)
        _, text = s.plan_report()
        assert text.startswith("row[") and "ROW_SUM" in text
        s.write(v, x)
        s.run()
        got = s.read(outs[-1])
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        if "TOP_K" in kinds:
            assert np.array_equal(s.read(outs[1])[:, 0], np.argmax(x, axis=1).astype(np.int32))
        s.close()


@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
@pytest.mark.parametrize("width", [1024, 512, 2048, 96])
def test_row_sum_fused_with_softmax_and_top_k(m3, ref, oracle, gpu, dtype, width):
    dt = getattr(m3, dtype)
    rows = 301
    raw = m3.fill_normal(7, width, 0.0, 2.0, rows * width).reshape(rows, width)
    x = raw if dtype == "F32" else (oracle.to_f16(raw) if dtype == "F16" else oracle.to_bf16(raw))
    g, v, outs = _graph(m3, x.shape, dt, ["SOFTMAX", "TOP_K", "ROW_SUM"])
    s = m3.Session(g)
    _, text = s.plan_report()
    assert "row[SOFTMAX+TOP_K+ROW_SUM]" in text
    s.write(v, x)
    s.run()
    sums = s.read(outs[-1])
    assert np.array_equal(sums.view(np.uint32), _sums(oracle, x, dt).view(np.uint32))
    # the softmax and top-k of the same pass still match the reference
    rg = m3.Graph(lib=ref)
    rx = rg.value(m3.INPUT, dt, x.shape)
    rp = rg.inferred("SOFTMAX", [rx], m3.OUTPUT, m3.F32 if dt == m3.F32 else dt)
    rg.node("SOFTMAX", [rx], [rp])
    rtv = rg.inferred("TOP_K", [rx], m3.OUTPUT, m3.F32, 0, k=1)
    rti = rg.inferred("TOP_K", [rx], m3.OUTPUT, m3.I32, 1, k=1)
    rg.node("TOP_K", [rx], [rtv, rti], k=1)
    rs = m3.Session(rg, allow_metal=False, allow_neural_engine=False, cuda=False)
    rs.write(rx, x)
    rs.run()
    assert np.array_equal(s.read(outs[2]), rs.read(rti))
    assert np.array_equal(s.read(outs[1]).view(np.uint32), rs.read(rtv).view(np.uint32))
    p, want_p = s.read(outs[0]), rs.read(rp)
    if dt == m3.F32:
        rel = np.abs(p.astype(np.float64) - want_p) / np.maximum(np.abs(want_p), 1e-30)
        assert rel.max() <= 1e-6
    else:
        assert np.abs(p.astype(np.int64) - want_p.astype(np.int64)).max() <= 1
    s.close()
    rs.close()


@pytest.mark.parametrize("shape", [(3, 5, 7), (1, 1), (17, 1001), (4, 0), (0, 8)])
def test_row_sum_ragged_and_empty(m3, oracle, gpu, shape):
    n = int(np.prod(shape))
    x = m3.fill_normal(3, 1, 0.0, 1.0, max(n, 1))[:n].reshape(shape)
    g, v, outs = _graph(m3, shape, m3.F32, ["ROW_SUM"])
    s = m3.Session(g)
    s.write(v, x)
    s.run()
    got = s.read(outs[0])
    want = _sums(oracle, x) if n else np.zeros(shape[:-1] + (1,), np.float32)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    s.close()


@pytest.mark.parametrize("order", ["row_sum_first", "softmax_first"])
def test_row_sum_nan_and_failure_order(m3, gpu, order):
    """A NaN propagates into the row's sum (no data check); in one row pass
    with SOFTMAX the softmax fails, and the row sums are committed exactly
    when ROW_SUM comes before SOFTMAX in node order (the reference would have
    executed it before the failing command)."""
    kinds = ["ROW_SUM", "SOFTMAX"] if order == "row_sum_first" else ["SOFTMAX", "ROW_SUM"]
    g, v, outs = _graph(m3, (6, 1024), m3.F32, kinds)
    s = m3.Session(g)
    good = np.ones((6, 1024), np.float32)
    s.write(v, good)
    s.run()
    r = outs[kinds.index("ROW_SUM")]
    assert np.all(s.read(r) == 1024.0)
    bad = good * 2.0
    bad[4, 9] = np.nan
    s.write(v, bad)
    status, message = s.run_status()
    assert status == m3.OUT_OF_RANGE and message == "softmax input contains NaN"
    sums = s.read(r)
    if order == "row_sum_first":
        assert np.isnan(sums[4, 0]) and np.all(np.delete(sums, 4) == 2048.0)
    else:
        assert np.all(sums == 1024.0)
    s.close()


def test_row_sum_backend_command(m3, oracle, gpu):
    """ROW_SUM through the reference-facing plug-in (m3_cuda_backend_execute)
    on a strided view: every other row of a [40, 256] tensor."""
    import torch

    lib = m3.load()
    full = torch.from_numpy(m3.fill_normal(5, 2, 0.0, 1.0, 40 * 256).reshape(40, 256)).cuda()
    out = torch.zeros((20, 1), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    storage_of = m3.STORAGE_DATA(lambda storage: storage)
    options = m3.BackendOptions(0, storage_of, False)
    ctx = ctypes.c_void_p()
    err = m3.M3Error()
    m3.check(lib.m3_cuda_backend_context_create(ctypes.byref(options), ctypes.byref(ctx),
                                                ctypes.byref(err)), err)
    src = m3.TensorView()
    src.metadata.dtype = m3.F32
    src.metadata.rank = 2
    src.metadata.shape[0], src.metadata.shape[1] = 20, 256
    src.metadata.element_count = 20 * 256
    src.metadata.byte_count = 20 * 256 * 4
    src.byte_offset = 0
    src.byte_strides[0], src.byte_strides[1] = 2 * 256 * 4, 4
    src.storage = full.data_ptr()
    dst = m3.TensorView()
    dst.metadata.dtype = m3.F32
    dst.metadata.rank = 2
    dst.metadata.shape[0], dst.metadata.shape[1] = 20, 1
    dst.metadata.element_count = 20
    dst.metadata.byte_count = 80
    dst.byte_strides[0], dst.byte_strides[1] = 4, 4
    dst.storage = out.data_ptr()
    cmd = m3.Command()
    cmd.kind = m3.OPS["ROW_SUM"]
    cmd.descriptor.copy.input = ctypes.pointer(src)
    cmd.descriptor.copy.output = ctypes.pointer(dst)
    m3.check(lib.m3_cuda_backend_execute(ctx, ctypes.byref(cmd), 1, None, ctypes.byref(err)), err)
    lib.m3_cuda_backend_destroy_context(ctx)
    want = _sums(oracle, np.ascontiguousarray(full.cpu().numpy()[::2]))
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
