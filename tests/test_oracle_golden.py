"""Pin the CPU oracle (oracle/m3_oracle.c) before trusting it.

1. Known-answer values from the reference's own tests, each cited by the
   reference test file:line it comes from.
2. Bit-exact agreement with the reference CPU provider compiled from its
   sources (oracle/_ref/libm3ref.so) on seeded random inputs, driven through
   the reference's command-level API.
3. The F16/BF16 codecs over large structured samples of the F32 bit space.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

INF = np.float32(np.inf)


def f32(bits: int) -> np.float32:
    return np.array([bits], dtype=np.uint32).view(np.float32)[0]


def bits_of(values) -> np.ndarray:
    return np.asarray(values, dtype=np.float32).view(np.uint32)


def binop(oracle, multiply: bool, left, right):
    left = np.asarray(left, dtype=np.float32)
    right = np.asarray(right, dtype=np.float32)
    out = np.zeros(np.broadcast(left, right).shape, dtype=np.float32)
    status = oracle._call("m3o_binary", int(multiply),
                          ctypes.byref(oracle.view(left)),
                          ctypes.byref(oracle.view(right)),
                          ctypes.byref(oracle.view(out)))
    assert status == 0
    return out


# ------------------------------------------------------------ 1. KATs


def test_f16_bf16_i32_conversions(oracle):
    # tests/test_op_basic.c:16-23 (values) and :71-88 (expectations)
    source = np.array([1.00048828125, 1.00146484375, np.inf, -np.inf, np.nan,
                       2.0 ** -24, 2.0 ** -25], dtype=np.float32)
    half = oracle.to_f16(source)
    assert half[0] == 0x3C00 and half[1] == 0x3C02          # RN-even halfway
    assert half[2] == 0x7C00 and half[3] == 0xFC00
    assert (half[4] & 0x7C00) == 0x7C00 and (half[4] & 0x03FF) != 0
    assert half[5] == 0x0001 and half[6] == 0x0000          # subnormal RN-even
    back = oracle.widen(half, oracle.F16)                   # :90-101
    assert back[0] == 1.0 and back[1] == 1.001953125
    assert np.isinf(back[2]) and back[2] > 0 and np.isinf(back[3]) and back[3] < 0
    assert np.isnan(back[4]) and back[5] == 2.0 ** -24 and back[6] == 0.0
    # tests/test_op_basic.c:25-27, :117-123
    brain = oracle.to_bf16(np.array([1.00390625, 1.01171875, np.inf, np.nan],
                                    dtype=np.float32))
    assert brain[0] == 0x3F80 and brain[1] == 0x3F82 and brain[2] == 0x7F80
    assert (brain[3] & 0x7F80) == 0x7F80 and (brain[3] & 0x007F) != 0
    # tests/test_op_basic.c:30, :136-139: truncation toward zero
    ints = np.zeros(2, dtype=np.int32)
    assert oracle.run("cast", np.array([2.9, -2.9], np.float32), ints) == 0
    assert list(ints) == [2, -2]
    # tests/test_op_basic.c:31-33, :149-152: invalid casts fail atomically
    sentinel = np.full(4, 77, dtype=np.int32)
    bad = np.array([np.nan, np.inf, -np.inf, 2147483648.0], dtype=np.float32)
    assert oracle.run("cast", bad, sentinel) == 2
    assert list(sentinel) == [77, 77, 77, 77]


def test_broadcast_add_mul(oracle):
    # tests/test_op_basic.c:165-171, :214-222: strided left [2,3] + [3]
    backing = np.array([1, 4, 2, 5, 3, 6], dtype=np.float32)
    left = np.lib.stride_tricks.as_strided(backing, shape=(2, 3),
                                           strides=(4, 8))
    out = binop(oracle, False, left, np.array([10, 20, 30], np.float32))
    assert list(out.ravel()) == [11, 22, 33, 14, 25, 36]
    # :228-237: scalar [1] broadcast
    scaled = binop(oracle, True, out, np.array([2.0], np.float32))
    assert scaled.ravel()[0] == 22 and scaled.ravel()[5] == 72


def test_softmax_special_rows(oracle):
    # tests/test_op_sampling.c:14, :48-52
    out = np.zeros(2, np.float32)
    assert oracle.run("softmax", np.array([1000, 1001], np.float32), out) == 0
    assert abs(out[0] - 0.268941432) <= 1e-6 and abs(out[1] - 0.731058598) <= 1e-6
    # :15, :55-66: all -inf row -> zeros
    out = np.full(2, 9, np.float32)
    assert oracle.run("softmax", np.array([-np.inf, -np.inf], np.float32), out) == 0
    assert list(out) == [0, 0]
    # :16, :67-82: only +inf entries share the mass
    out = np.zeros(3, np.float32)
    assert oracle.run("softmax", np.array([np.inf, 1, np.inf], np.float32), out) == 0
    assert list(out) == [0.5, 0.0, 0.5]
    # :19-20, :83-96: NaN fails and leaves the output unchanged
    out = np.full(2, -7, np.float32)
    assert oracle.run("softmax", np.array([0, np.nan], np.float32), out) == 2
    assert list(out) == [-7, -7]


def test_top_k_order_and_nan(oracle):
    # tests/test_op_sampling.c:104, :148-169: descending, ties -> lower index
    logits = np.array([[3, 5, 5, 1]], np.float32)
    values = np.full((1, 3), -9, np.float32)
    indices = np.full((1, 3), -9, np.int32)
    assert oracle.run("top_k", logits, values, indices, k=3) == 0
    assert list(values.ravel()) == [5, 5, 3] and list(indices.ravel()) == [1, 2, 0]
    # :108, :170-180: NaN logits fail
    values[:] = -9
    nan_logits = np.array([[3, np.nan, 5, 1]], np.float32)
    assert oracle.run("top_k", nan_logits, values, indices, k=3) == 2
    assert list(values.ravel()) == [-9, -9, -9]


def test_norms_and_gated_silu(oracle):
    # tests/test_op_dense.c:31-32, :157-165 (in place, eps 3.5)
    x = np.array([[3, 4]], np.float32)
    out = np.zeros_like(x)
    assert oracle.run("rms_norm", x, np.array([1, 2], np.float32), out,
                      eps=3.5) == 0
    assert abs(out[0, 0] - 0.75) <= 1e-6 and abs(out[0, 1] - 2.0) <= 1e-6
    # :35-37, :183-193 (eps 1/3, with bias)
    out = np.zeros((1, 3), np.float32)
    assert oracle.run("layer_norm", np.array([[1, 2, 3]], np.float32),
                      np.array([1, 2, 1], np.float32),
                      np.array([0, 1, -1], np.float32), out,
                      eps=np.float32(1.0 / 3.0)) == 0
    assert np.allclose(out.ravel(), [-1, 1, 0], atol=1e-6)
    # :39-40, :216-219
    out = np.zeros(2, np.float32)
    assert oracle.run("gated_silu", np.array([0, 1], np.float32),
                      np.array([2, 2], np.float32), out) == 0
    assert out[0] == 0.0 and abs(out[1] - 1.46211720) <= 1e-6


def test_bf16_precision_contracts(oracle):
    # tests/test_transformer_precision.c:176-218: BF16 RMSNorm rounds the
    # normalised value before scaling -> 0x3d88 / 0x3f88
    x = np.array([[0x3D00, 0x3F00]], np.uint16)
    scale = np.array([0x3F40, 0x3F40], np.uint16)
    out = np.zeros((1, 2), np.uint16)
    assert oracle.run("rms_norm", (x, oracle.BF16), (scale, oracle.BF16),
                      (out, oracle.BF16), eps=1e-6) == 0
    assert list(out.ravel()) == [0x3D88, 0x3F88]
    # :181-183, :236-242 F32 control
    out32 = np.zeros((1, 2), np.float32)
    assert oracle.run("rms_norm", np.array([[0.03125, 0.5]], np.float32),
                      np.array([0.75, 0.75], np.float32), out32, eps=1e-6) == 0
    assert abs(out32[0, 0] - 0.0661619008) <= 1e-7
    assert abs(out32[0, 1] - 1.05859041) <= 1e-7
    # :246-288: BF16 gated SiLU rounds the activation first -> 0x3e6e
    out = np.zeros(1, np.uint16)
    assert oracle.run("gated_silu", (np.array([0x3F00], np.uint16), oracle.BF16),
                      (np.array([0x3F40], np.uint16), oracle.BF16),
                      (out, oracle.BF16)) == 0
    assert out[0] == 0x3E6E
    # :250-252, :305-308 F32 control
    out32 = np.zeros(1, np.float32)
    assert oracle.run("gated_silu", np.array([0.5], np.float32),
                      np.array([0.75], np.float32), out32) == 0
    assert abs(out32[0] - 0.233422250) <= 1e-7


def test_snake_and_tanh_bits(oracle):
    # tests/test_vocoder_activations.c:65-71, :128-137: seven rounded
    # statements; alpha = -eps gives a +0 denominator and +inf
    x = np.array([f32(0x3E1D90CD), 1.0], np.float32).reshape(1, 2, 1)
    alpha = np.array([f32(0x3E0B9EEF), f32(0xB089705F)], np.float32).reshape(1, 2, 1)
    out = np.zeros_like(x)
    assert oracle.run("snake1d", x, alpha, out) == 0
    assert list(bits_of(out).ravel()) == [0x3E20DEF4, 0x7F800000]
    # :174-216: tanh special values
    values = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf,
                       f32(0x7FC12345), 0.5], np.float32)
    out = np.zeros_like(values)
    assert oracle.run("tanh", values, out) == 0
    b = bits_of(out)
    assert list(b[:6]) == [0x00000000, 0x80000000, 0x3F42F7D6, 0xBF42F7D6,
                           0x3F800000, 0xBF800000]
    assert np.isnan(out[6]) and b[7] == 0x3EEC9A9F


def test_flow_cfg_and_euler_bits(oracle):
    # tests/test_flow_model.c:300-311 with the fixture's guidance 1.7
    # (tests/flow_runtime_test.c:198): v = v_u + g * (v_c + (-1 * v_u))
    v_c = np.array([5432.875, 1.0], np.float32)
    v_u = np.array([-12345.625, -1.0], np.float32)
    a = binop(oracle, True, v_u, np.array([-1.0], np.float32))
    a = binop(oracle, False, v_c, a)
    a = binop(oracle, True, a, np.array([1.7], np.float32))
    v = binop(oracle, False, v_u, a)
    assert bits_of(v)[0] == 0x468BABA7
    # :313-329: x' = x + v * delta(0, 30)
    delta = oracle.restatement().m3o_flow_timestep_delta(0, 30)
    t = binop(oracle, True, np.array([-0.1259765625, 0], np.float32),
              np.array([delta], np.float32))
    x = binop(oracle, False, np.array([123456.75, 0], np.float32), t)
    assert bits_of(x)[0] == 0x47F1205F


def test_clamp_bits(oracle):
    # tests/test_waveform_assembly.c:96-140
    source = np.array([0x40000000, 0xC0000000, 0x3F800000, 0xBF800000,
                       0x00000000, 0x80000000, 0x00000001, 0x80000001,
                       0x7FC12345, 0xFFC54321, 0x7F800000, 0xFF800000,
                       0x7FA12345, 0xFFA54321], dtype=np.uint32)
    expected = [0x3F800000, 0xBF800000, 0x3F800000, 0xBF800000,
                0x00000000, 0x80000000, 0x00000001, 0x80000001,
                0x7FC12345, 0xFFC54321, 0x3F800000, 0xBF800000,
                0x7FA12345, 0xFFA54321]
    out = np.zeros(14, np.uint32)
    assert oracle.run("clamp_unit", (source, oracle.F32), (out, oracle.F32)) == 0
    assert list(out) == expected


def test_abs_max_extension(oracle):
    out = np.full(1, 7, np.float32)
    data = np.array([-3.5, 2.0, -0.0, 1e-40], np.float32)
    assert oracle.run("abs_max", data, out) == 0 and out[0] == 3.5
    assert oracle.run("abs_max", np.array([], np.float32), out) == 0 and out[0] == 0
    out[:] = 7
    assert oracle.run("abs_max", np.array([1, np.nan], np.float32), out) == 2
    assert out[0] == 7


def test_row_sum_extension(oracle):
    """Row sums accumulate left to right in F32: a row whose tree sum
    differs from its sequential sum shows the order."""
    x = np.array([[1.0, 2.0 ** -24, 2.0 ** -24, 2.0 ** -24, 2.0 ** -24]], np.float32)
    out = np.zeros((1, 1), np.float32)
    assert oracle.run("row_sum", x, out) == 0
    assert out[0, 0] == np.float32(1.0)          # each 2^-24 rounds away
    rng = np.random.default_rng(5)
    x = rng.standard_normal((7, 33)).astype(np.float32)
    want = np.zeros(7, np.float32)
    for j in range(33):
        want = (want + x[:, j]).astype(np.float32)
    out = np.zeros((7, 1), np.float32)
    assert oracle.run("row_sum", x, out) == 0
    assert np.array_equal(out[:, 0].view(np.uint32), want.view(np.uint32))
    h = oracle.to_f16(x)
    assert oracle.run("row_sum", (h, oracle.F16), out) == 0
    widened = oracle.widen(h, oracle.F16)
    want = np.zeros(7, np.float32)
    for j in range(33):
        want = (want + widened[:, j]).astype(np.float32)
    assert np.array_equal(out[:, 0].view(np.uint32), want.view(np.uint32))


# ----------------------------------- 2. against the compiled reference


def _reference_session(m3, ref, build):
    """Run a graph built by `build(graph) -> (inputs, outputs)` on the
    reference CPU provider."""
    graph = m3.Graph(lib=ref)
    inputs, outputs = build(graph)
    session = m3.Session(graph, allow_metal=False, allow_neural_engine=False,
                         allow_cpu=True, cuda=False)
    for vid, data in inputs:
        session.write(vid, data)
    session.run()
    return [session.read(vid) for vid in outputs]


@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_matches_reference_library(m3, ref, oracle, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((64, 96)) * 3).astype(np.float32)
    x[rng.random(x.shape) < 0.02] = 20.0
    c = rng.uniform(0.5, 2, 96).astype(np.float32)
    b = rng.standard_normal((1, 96)).astype(np.float32)
    scale = rng.normal(1, 0.05, 96).astype(np.float32)

    def build(g):
        vx = g.value(m3.INPUT, m3.F32, (64, 96))
        vc = g.constant(m3.F32, c)
        vb = g.constant(m3.F32, b)
        t = g.inferred("MUL", [vx, vc], m3.TEMPORARY, m3.F32)
        g.node("MUL", [vx, vc], [t])
        y = g.inferred("ADD", [t, vb], m3.OUTPUT, m3.F32)
        g.node("ADD", [t, vb], [y])
        p = g.inferred("SOFTMAX", [vx], m3.OUTPUT, m3.F32)
        g.node("SOFTMAX", [vx], [p])
        tv = g.inferred("TOP_K", [vx], m3.OUTPUT, m3.F32, 0, k=3)
        ti = g.inferred("TOP_K", [vx], m3.OUTPUT, m3.I32, 1, k=3)
        g.node("TOP_K", [vx], [tv, ti], k=3)
        vs = g.constant(m3.F32, scale)
        n = g.inferred("RMS_NORM", [vx, vs], m3.OUTPUT, m3.F32, epsilon=1e-6)
        g.node("RMS_NORM", [vx, vs], [n], epsilon=1e-6)
        ln = g.inferred("LAYER_NORM", [vx, vs], m3.OUTPUT, m3.F32, epsilon=1e-5)
        g.node("LAYER_NORM", [vx, vs, m3.VALUE_NONE], [ln], epsilon=1e-5)
        gs = g.inferred("GATED_SILU", [vx, vx], m3.OUTPUT, m3.F32)
        g.node("GATED_SILU", [vx, vx], [gs])
        th = g.inferred("TANH", [vx], m3.OUTPUT, m3.F32)
        g.node("TANH", [vx], [th])
        return [(vx, x)], [y, p, tv, ti, n, ln, gs, th]

    y, p, tv, ti, n, ln, gs, th = _reference_session(m3, ref, build)
    t = binop(oracle, True, x, c)
    assert np.array_equal(bits_of(binop(oracle, False, t, b)), bits_of(y))
    mp = np.zeros_like(x)
    assert oracle.run("softmax", x, mp) == 0
    assert np.array_equal(bits_of(mp), bits_of(p))
    mv = np.zeros((64, 3), np.float32)
    mi = np.zeros((64, 3), np.int32)
    assert oracle.run("top_k", x, mv, mi, k=3) == 0
    assert np.array_equal(bits_of(mv), bits_of(tv)) and np.array_equal(mi, ti)
    mn = np.zeros_like(x)
    assert oracle.run("rms_norm", x, scale, mn, eps=1e-6) == 0
    assert np.array_equal(bits_of(mn), bits_of(n))
    ml = np.zeros_like(x)
    assert oracle.run("layer_norm", x, scale, None, ml, eps=1e-5) == 0
    assert np.array_equal(bits_of(ml), bits_of(ln))
    mg = np.zeros_like(x)
    assert oracle.run("gated_silu", x, x, mg) == 0
    assert np.array_equal(bits_of(mg), bits_of(gs))
    mt = np.zeros_like(x)
    assert oracle.run("tanh", x, mt) == 0
    assert np.array_equal(bits_of(mt), bits_of(th))


def test_oracle_f16_graph_matches_reference(m3, ref, oracle):
    rng = np.random.default_rng(7)
    h = oracle.to_f16(rng.standard_normal((16, 40)).astype(np.float32))
    r = oracle.to_f16(rng.standard_normal((16, 40)).astype(np.float32))
    w = oracle.to_f16(rng.normal(1, 0.05, 40).astype(np.float32))

    def build(g):
        vh = g.value(m3.INPUT, m3.F16, (16, 40))
        vr = g.value(m3.INPUT, m3.F16, (16, 40))
        vw = g.constant(m3.F16, w)
        s = g.inferred("ADD", [vh, vr], m3.OUTPUT, m3.F16)
        g.node("ADD", [vh, vr], [s])
        n = g.inferred("RMS_NORM", [s, vw], m3.OUTPUT, m3.F16, epsilon=1e-6)
        g.node("RMS_NORM", [s, vw], [n], epsilon=1e-6)
        y = g.inferred("GATED_SILU", [vh, vr], m3.OUTPUT, m3.F16)
        g.node("GATED_SILU", [vh, vr], [y])
        xb = g.inferred("CAST", [s], m3.OUTPUT, m3.BF16)
        g.node("CAST", [s], [xb])
        return [(vh, h), (vr, r)], [s, n, y, xb]

    s, n, y, xb = _reference_session(m3, ref, build)
    ms = np.zeros_like(h)
    assert oracle._call("m3o_binary", 0, ctypes.byref(oracle.view(h, oracle.F16)),
                        ctypes.byref(oracle.view(r, oracle.F16)),
                        ctypes.byref(oracle.view(ms, oracle.F16))) == 0
    assert np.array_equal(ms, s)
    mn = np.zeros_like(h)
    assert oracle.run("rms_norm", (ms, oracle.F16), (w, oracle.F16),
                      (mn, oracle.F16), eps=1e-6) == 0
    assert np.array_equal(mn, n)
    my = np.zeros_like(h)
    assert oracle.run("gated_silu", (h, oracle.F16), (r, oracle.F16),
                      (my, oracle.F16)) == 0
    assert np.array_equal(my, y)
    mb = np.zeros_like(h)
    assert oracle.run("cast", (ms, oracle.F16), (mb, oracle.BF16)) == 0
    assert np.array_equal(mb, xb)


# ----------------------------------------------------------- 3. codecs


def _special_bit_sample(count: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    random_bits = rng.integers(0, 2 ** 32, count, dtype=np.uint64).astype(np.uint32)
    # every exponent with the low mantissa bits swept around rounding points
    exps = np.arange(256, dtype=np.uint32) << 23
    lows = np.array([0, 1, 0xFFF, 0x1000, 0x1001, 0x1FFF, 0x2000, 0x7FFF,
                     0x8000, 0x8001, 0xFFFF, 0x10000, 0x7FFFFF, 0x400000,
                     0x200000, 0x3FF000], dtype=np.uint32)
    grid = (exps[:, None] | lows[None, :]).ravel()
    sweep = np.concatenate([grid, grid | 0x80000000])
    return np.concatenate([random_bits, sweep])


def test_codecs_match_reference_cast(m3, ref, oracle):
    sample = _special_bit_sample(1 << 18, 3)
    source = sample.view(np.float32)

    for dtype, encode in ((m3.F16, oracle.to_f16), (m3.BF16, oracle.to_bf16)):
        def build(g, dtype=dtype):
            vx = g.value(m3.INPUT, m3.F32, (source.size,))
            y = g.inferred("CAST", [vx], m3.OUTPUT, dtype)
            g.node("CAST", [vx], [y])
            back = g.inferred("CAST", [y], m3.OUTPUT, m3.F32)
            g.node("CAST", [y], [back])
            return [(vx, source)], [y, back]

        encoded, decoded = _reference_session(m3, ref, build)
        mine = encode(source)
        assert np.array_equal(mine, encoded)
        assert np.array_equal(bits_of(oracle.widen(mine, dtype)), bits_of(decoded))
