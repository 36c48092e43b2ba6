"""GPU parity: libm3cuda.so against the reference CPU provider.

Every case builds one graph twice through the same m3.h API -- once on the
CUDA library, once on the reference's own CPU provider compiled from its
sources (oracle/_ref) -- feeds both the same seeded inputs, and compares:

* bit-exact: ADD/MUL/CAST/COPY (incl. broadcast), residual sums, RMSNorm,
  LayerNorm (the kernels sum in the reference's order), top-k values and
  indices, clamp, abs-max;
* softmax probabilities: within 1e-6 relative (F32 reduction bar);
  the only source of difference is expf (CUDA vs glibc);
* gated SiLU in F16/BF16: within 1 ulp of the output dtype (expf);
* snake1d and tanh: within 0x1p-19 absolute-or-relative (sinf/tanhf),
  the reference's own device tolerance (tests/test_metal_vocoder_activations.c:14).

Where the reference has no operator (abs-max, clamp), the oracle
restatement (oracle/m3_oracle.c) is the checker.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_SIN = 2.0 ** -19


def bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype.itemsize == 4 else np.uint16)


def ordered(b: np.ndarray, width: int) -> np.ndarray:
    """Map float bit patterns to integers whose order is the float order."""
    b = b.astype(np.int64)
    sign = 1 << (width - 1)
    return np.where(b & sign, -(b & (sign - 1)), b)


def ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    width = 8 * a.dtype.itemsize
    return np.abs(ordered(bits(a), width) - ordered(bits(b), width))


def close_abs_or_rel(a, b, tol) -> bool:
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    same_special = (np.isnan(a) & np.isnan(b)) | (a == b)
    diff = np.abs(a - b)
    ok = same_special | (diff <= tol) | (diff <= tol * np.maximum(np.abs(a), np.abs(b)))
    return bool(ok.all())


def run_both(m3, ref, build, inputs, fuse=True):
    """Run `build` on both libraries; returns (cuda_outputs, reference_outputs)."""
    results = []
    for lib, cuda in ((m3.load(), True), (ref, False)):
        g = m3.Graph(lib=lib)
        handles, outputs = build(g)
        if cuda:
            s = m3.Session(g, fuse=fuse)
        else:
            s = m3.Session(g, allow_metal=False, allow_neural_engine=False, cuda=False)
        for name, vid in handles.items():
            s.write(vid, inputs[name])
        s.run()
        results.append([s.read(v) for v in outputs])
        if cuda:
            assert all(s.provider(i) == m3.PROVIDER_CUDA for i in range(len(g.values) and 1))
        s.close()
    return results


# ------------------------------------------------------------ codecs


def test_hardware_codecs_match_reference_encoders_exhaustively(m3, gpu):
    import ctypes

    mismatches = ctypes.c_uint64(12345)
    err = m3.M3Error()
    m3.check(m3.load().m3_cuda_codec_self_test(0, ctypes.byref(mismatches),
                                               ctypes.byref(err)), err)
    assert mismatches.value == 0


def test_markstein_division_matches_ieee_on_softmax_domain(m3, gpu):
    import ctypes

    mismatches = ctypes.c_uint64(12345)
    err = m3.M3Error()
    m3.check(m3.load().m3_cuda_division_self_test(0, 1 << 32, ctypes.byref(mismatches),
                                                  ctypes.byref(err)), err)
    assert mismatches.value == 0


def test_moderate_exponential_error_bound(m3, gpu):
    """The exponential of the 16-bit gated SiLU path: every F32 argument in
    [-87, 87] within 4 ulps (4 * 2^-23 = 4.8e-7 relative) of the correctly
    rounded e^d, and exactly 1 at 0.  A 16-bit result's half ulp is 2^-12
    (F16) or 2^-9 (BF16) relative, so such an error moves the rounded
    result only when the exact value lies within 4.8e-7 of a rounding
    boundary, and then by one ulp."""
    import ctypes

    worst = ctypes.c_uint32(99)
    violations = ctypes.c_uint64(99)
    err = m3.M3Error()
    m3.check(m3.load().m3_cuda_exp_self_test(0, ctypes.byref(worst), ctypes.byref(violations),
                                             ctypes.byref(err)), err)
    print("exp_moderate: max ulp", worst.value)
    assert violations.value == 0
    assert worst.value <= 4


def test_sin_squared_error_bound(m3, gpu):
    """The snake activation's sin^2 for |alpha x| <= 8192, every F32 argument
    of that range: absolute error below 2^-22 (so the output x + sin^2/alpha
    moves by under 5 * 2^-22 < 0x1p-19 for alpha >= 0.2) and within 4 ulps
    where sin^2 >= 2^-10."""
    import ctypes

    abs_error = ctypes.c_float(99.0)
    worst = ctypes.c_uint32(99)
    err = m3.M3Error()
    m3.check(m3.load().m3_cuda_sin_squared_self_test(0, ctypes.byref(abs_error), ctypes.byref(worst),
                                                     ctypes.byref(err)), err)
    print("sin_squared: max abs error", abs_error.value, "max ulp", worst.value)
    assert abs_error.value < 2.0 ** -22
    assert worst.value <= 4


def test_sin_squared_packed_matches_scalar(m3, gpu):
    """The snake's packed (F32x2) sin^2 gives the scalar evaluation's bits on
    every F32 argument in [-8192, 8192], in either lane."""
    import ctypes

    mismatches = ctypes.c_uint64(99)
    err = m3.M3Error()
    m3.check(m3.load().m3_cuda_sin_squared_packed_self_test(0, ctypes.byref(mismatches),
                                                            ctypes.byref(err)), err)
    assert mismatches.value == 0


# ------------------------------------------------------------ element-wise


@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
@pytest.mark.parametrize("fuse", [True, False])
def test_binary_broadcast_chain(m3, ref, oracle, gpu, dtype, fuse):
    dt = getattr(m3, dtype)
    rng = np.random.default_rng(11)
    shape = (37, 130)          # ragged: not a multiple of the vector width

    def encode(x):
        return {"F32": x, "F16": oracle.to_f16(x), "BF16": oracle.to_bf16(x)}[dtype]

    inputs = {"x": encode(rng.standard_normal(shape).astype(np.float32)),
              "r": encode(rng.standard_normal((1, 130)).astype(np.float32)),
              "c": encode(rng.standard_normal((37, 1)).astype(np.float32))}
    scalar = encode(np.array([0.37], np.float32))

    def build(g):
        x = g.value(m3.INPUT, dt, shape)
        r = g.value(m3.INPUT, dt, (1, 130))
        c = g.value(m3.INPUT, dt, (37, 1))
        k = g.constant(dt, scalar)
        a = g.inferred("MUL", [x, r], m3.TEMPORARY, dt)
        g.node("MUL", [x, r], [a])
        b = g.inferred("ADD", [a, c], m3.TEMPORARY, dt)
        g.node("ADD", [a, c], [b])
        d = g.inferred("MUL", [b, k], m3.OUTPUT, dt)
        g.node("MUL", [b, k], [d])
        e = g.inferred("ADD", [c, d], m3.OUTPUT, m3.F32)
        g.node("ADD", [c, d], [e])
        return {"x": x, "r": r, "c": c}, [d, e]

    mine, theirs = run_both(m3, ref, build, inputs, fuse)
    for a, b in zip(mine, theirs):
        assert np.array_equal(bits(a), bits(b))


@pytest.mark.parametrize("pair", [("F32", "F16"), ("F32", "BF16"), ("F16", "F32"),
                                  ("BF16", "F16"), ("F16", "BF16"), ("I32", "F32"),
                                  ("F32", "I32"), ("F16", "I32"), ("F16", "F16")])
def test_cast_and_copy(m3, ref, oracle, gpu, pair):
    src, dst = (getattr(m3, p) for p in pair)
    rng = np.random.default_rng(5)
    raw = (rng.standard_normal(1003) * 1000).astype(np.float32)
    raw[:6] = [0.0, -0.0, 1e-8, -65520.0, 70000.0, 2.0 ** -25]
    if src == m3.F32:
        x = raw
    elif src == m3.I32:
        x = raw.astype(np.int32)
    elif src == m3.F16:
        x = oracle.to_f16(raw)
        x[6:10] = [0x7C00, 0x7E01, 0x7D00, 0x8001]   # inf, qNaN, sNaN payload, -subnormal
        if dst == m3.I32:
            # finite F16 values only, so the cast is valid on both sides
            x = oracle.to_f16(np.clip(raw, -60000.0, 60000.0))
    else:
        x = oracle.to_bf16(raw)

    def build(g):
        v = g.value(m3.INPUT, src, (1003,))
        y = g.inferred("CAST", [v], m3.OUTPUT, dst)
        g.node("CAST", [v], [y])
        z = g.inferred("COPY", [v], m3.OUTPUT, src)
        g.node("COPY", [v], [z])
        return {"x": v}, [y, z]

    mine, theirs = run_both(m3, ref, build, {"x": x})
    for a, b in zip(mine, theirs):
        assert np.array_equal(bits(a) if a.dtype != np.int32 else a,
                              bits(b) if b.dtype != np.int32 else b)


def test_cast_to_i32_failure_is_atomic(m3, gpu):
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (4,))
    y = g.inferred("CAST", [x], m3.OUTPUT, m3.I32)
    g.node("CAST", [x], [y])
    s = m3.Session(g)
    s.write(x, np.array([2.9, -2.9, 7.5, -0.5], np.float32))
    s.run()
    assert list(s.read(y)) == [2, -2, 7, 0]
    # tests/test_op_basic.c:141-158: any invalid value fails the whole cast
    s.write(x, np.array([np.nan, 1.0, np.inf, 2147483648.0], np.float32))
    status, message = s.run_status()
    assert status == m3.OUT_OF_RANGE and "I32" in message
    assert list(s.read(y)) == [2, -2, 7, 0]
    s.write(x, np.array([1.5, 2.5, 3.5, 4.5], np.float32))
    s.run()
    assert list(s.read(y)) == [1, 2, 3, 4]


def test_fused_failure_keeps_earlier_commands(m3, gpu):
    """ADD then a range-checked CAST fuse into one launch.  When the cast
    fails, the reference has already stored the ADD (it ran first), so the
    ADD output must be complete while the cast output is unchanged."""
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (300_000,))
    c = g.constant(m3.F32, np.array([0.5], np.float32))
    y = g.inferred("ADD", [x, c], m3.OUTPUT, m3.F32)
    g.node("ADD", [x, c], [y])
    z = g.inferred("CAST", [y], m3.OUTPUT, m3.I32)
    g.node("CAST", [y], [z])
    s = m3.Session(g)
    _, text = s.plan_report()
    assert text.startswith("ew[ADD,CAST]")
    data = np.arange(300_000, dtype=np.float32)
    s.write(x, data)
    s.run()
    before_z = s.read(z).copy()
    data2 = data * 2
    data2[-1] = 3e9                       # out of the I32 range after the add
    s.write(x, data2)
    status, _ = s.run_status()
    assert status == m3.OUT_OF_RANGE
    assert np.array_equal(s.read(y), data2 + np.float32(0.5))
    assert np.array_equal(s.read(z), before_z)


@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
def test_gated_silu(m3, ref, oracle, gpu, dtype):
    dt = getattr(m3, dtype)
    rng = np.random.default_rng(3)
    g32 = (rng.standard_normal((64, 257)) * 4).astype(np.float32)
    u32 = rng.standard_normal((64, 257)).astype(np.float32)
    enc = {"F32": lambda v: v, "F16": oracle.to_f16, "BF16": oracle.to_bf16}[dtype]

    def build(g):
        a = g.value(m3.INPUT, dt, (64, 257))
        b = g.value(m3.INPUT, dt, (64, 257))
        y = g.inferred("GATED_SILU", [a, b], m3.OUTPUT, dt)
        g.node("GATED_SILU", [a, b], [y])
        return {"g": a, "u": b}, [y]

    (mine,), (theirs,) = run_both(m3, ref, build, {"g": enc(g32), "u": enc(u32)})
    if dtype == "F32":
        assert close_abs_or_rel(mine, theirs, 2.0 ** -20)
    else:
        assert ulp_distance(mine, theirs).max() <= 1


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
def test_gated_silu_16_bit_across_gate_range(m3, ref, oracle, gpu, dtype):
    """16-bit gated SiLU over a million elements whose gates cover every
    binade the 16-bit type has, both sides of the |g| = 80 switch between the
    approximate and the IEEE evaluation, infinities, zeros and subnormals:
    within 1 ulp of the reference everywhere."""
    dt = getattr(m3, dtype)
    enc = {"F16": oracle.to_f16, "BF16": oracle.to_bf16}[dtype]
    rng = np.random.default_rng(17)
    shape = (4096, 257)
    top = 15 if dtype == "F16" else 100
    mags = np.exp2(rng.uniform(-24 if dtype == "F16" else -120, top, shape))
    g32 = (mags * rng.choice([-1.0, 1.0], shape)).astype(np.float32)
    g32[0, :16] = [0.0, -0.0, 79.9, -79.9, 80.0, -80.0, 80.5, -80.5, 90.0, -90.0,
                   np.inf, -np.inf, 1e-7, -1e-7, 6e-8, 3.0]
    u32 = (rng.standard_normal(shape) * 2).astype(np.float32)

    def build(g):
        a = g.value(m3.INPUT, dt, shape)
        b = g.value(m3.INPUT, dt, shape)
        y = g.inferred("GATED_SILU", [a, b], m3.OUTPUT, dt)
        g.node("GATED_SILU", [a, b], [y])
        return {"g": a, "u": b}, [y]

    (mine,), (theirs,) = run_both(m3, ref, build, {"g": enc(g32), "u": enc(u32)})
    # -inf / inf makes a NaN from non-NaN operands, whose bits are the
    # platform's default NaN (x86 and ARM differ; the GPU has its own): both
    # sides must be NaN there, and within 1 ulp everywhere else
    exponent = 0x7C00 if dtype == "F16" else 0x7F80
    nan = lambda b: ((b & 0x7FFF) > exponent)
    both_nan = nan(mine) & nan(theirs)
    assert np.array_equal(nan(mine), nan(theirs))
    assert ulp_distance(mine[~both_nan], theirs[~both_nan]).max() <= 1


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
@pytest.mark.parametrize("shape", [(33, 257), (3,), (1, 5)])
def test_gated_silu_16_bit_ragged(m3, ref, oracle, gpu, dtype, shape):
    """Element counts that are not a multiple of four: the dedicated 16-bit
    loop's full blocks and its element-wise tail."""
    dt = getattr(m3, dtype)
    enc = {"F16": oracle.to_f16, "BF16": oracle.to_bf16}[dtype]
    rng = np.random.default_rng(sum(shape))
    g32 = (rng.standard_normal(shape) * 6).astype(np.float32)
    u32 = rng.standard_normal(shape).astype(np.float32)

    def build(g):
        a = g.value(m3.INPUT, dt, shape)
        b = g.value(m3.INPUT, dt, shape)
        y = g.inferred("GATED_SILU", [a, b], m3.OUTPUT, dt)
        g.node("GATED_SILU", [a, b], [y])
        return {"g": a, "u": b}, [y]

    (mine,), (theirs,) = run_both(m3, ref, build, {"g": enc(g32), "u": enc(u32)})
    assert ulp_distance(mine, theirs).max() <= 1


def test_snake_tanh_clamp_absmax(m3, ref, oracle, gpu):
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((2, 24, 1000)) * 0.5).astype(np.float32)
    x[0, 0, :8] = [0.0, -0.0, 40.0, -40.0, 1e-30, 3.0, -3.0, 1e4]
    alpha = rng.uniform(0.2, 2.0, (1, 24, 1)).astype(np.float32)

    def build(g):
        vx = g.value(m3.INPUT, m3.F32, x.shape)
        va = g.value(m3.INPUT, m3.F32, alpha.shape)
        z = g.inferred("SNAKE1D", [vx, va], m3.OUTPUT, m3.F32)
        g.node("SNAKE1D", [vx, va], [z])
        t = g.inferred("TANH", [z], m3.OUTPUT, m3.F32)
        g.node("TANH", [z], [t])
        return {"x": vx, "a": va}, [z, t]

    (z, t), (rz, rt) = run_both(m3, ref, build, {"x": x, "a": alpha})
    assert close_abs_or_rel(z, rz, TOL_SIN)
    assert close_abs_or_rel(t, rt, TOL_SIN)

    # extensions: abs-max over the snake output and the clamp (oracle)
    g = m3.Graph()
    vx = g.value(m3.INPUT, m3.F32, x.shape)
    va = g.constant(m3.F32, alpha)
    vz = g.inferred("SNAKE1D", [vx, va], m3.OUTPUT, m3.F32)
    g.node("SNAKE1D", [vx, va], [vz])
    vm = g.inferred("ABS_MAX", [vz], m3.OUTPUT, m3.F32)
    g.node("ABS_MAX", [vz], [vm])
    vy = g.inferred("CLAMP_UNIT", [vz], m3.OUTPUT, m3.F32)
    g.node("CLAMP_UNIT", [vz], [vy])
    s = m3.Session(g)
    s.write(vx, x)
    s.run()
    z2, m, y = s.read(vz), s.read(vm), s.read(vy)
    assert np.array_equal(bits(z2), bits(z))
    om = np.zeros(1, np.float32)
    assert oracle.run("abs_max", z2, om) == 0
    assert bits(m)[0] == bits(om)[0]
    oy = np.zeros_like(z2)
    assert oracle.run("clamp_unit", z2, oy) == 0
    assert np.array_equal(bits(y), bits(oy))


def test_clamp_special_bits(m3, gpu):
    source = np.array([0x40000000, 0xC0000000, 0x3F800000, 0xBF800000,
                       0x00000000, 0x80000000, 0x00000001, 0x80000001,
                       0x7FC12345, 0xFFC54321, 0x7F800000, 0xFF800000,
                       0x7FA12345, 0xFFA54321], dtype=np.uint32)
    expected = [0x3F800000, 0xBF800000, 0x3F800000, 0xBF800000, 0, 0x80000000,
                1, 0x80000001, 0x7FC12345, 0xFFC54321, 0x3F800000, 0xBF800000,
                0x7FA12345, 0xFFA54321]
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (14,))
    y = g.inferred("CLAMP_UNIT", [x], m3.OUTPUT, m3.F32)
    g.node("CLAMP_UNIT", [x], [y])
    s = m3.Session(g)
    s.write(x, source.view(np.float32))
    s.run()
    assert list(bits(s.read(y))) == expected


def test_abs_max_nan_and_empty(m3, gpu):
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (1000,))
    m = g.inferred("ABS_MAX", [x], m3.OUTPUT, m3.F32)
    g.node("ABS_MAX", [x], [m])
    s = m3.Session(g)
    data = np.linspace(-3, 2, 1000).astype(np.float32)
    s.write(x, data)
    s.run()
    assert s.read(m)[0] == 3.0
    data[500] = np.nan
    s.write(x, data)
    status, _ = s.run_status()
    assert status == m3.OUT_OF_RANGE and s.read(m)[0] == 3.0
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (0,))
    m = g.inferred("ABS_MAX", [x], m3.OUTPUT, m3.F32)
    g.node("ABS_MAX", [x], [m])
    s = m3.Session(g)
    s.run()
    assert s.read(m)[0] == 0.0


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
@pytest.mark.parametrize("count", [1, 7, 4099, 1 << 20])
def test_abs_max_16_bit_against_oracle(m3, oracle, gpu, dtype, count):
    """ABS_MAX of F16/BF16 tensors through a session
    against the oracle's abs-max over the same bits: signed zeros,
    subnormals, infinities and the largest finite values included."""
    dt = getattr(m3, dtype)
    enc = oracle.to_f16 if dtype == "F16" else oracle.to_bf16
    x = enc(m3.fill_normal(9, count % 13, 0.0, 2.0, count))
    specials = np.array([0x8000, 0x0001, 0x8003, 0x7BFF if dtype == "F16" else 0x7F7F],
                        np.uint16)
    x[: min(count, len(specials))] = specials[: min(count, len(specials))]
    if count > 4:
        x[count // 2] = 0xFC00 if dtype == "F16" else 0xFF80      # -inf
    g = m3.Graph()
    v = g.value(m3.INPUT, dt, (count,))
    m = g.inferred("ABS_MAX", [v], m3.OUTPUT, m3.F32)
    g.node("ABS_MAX", [v], [m])
    s = m3.Session(g)
    s.write(v, x)
    s.run()
    want = np.zeros(1, np.float32)
    assert oracle.run("abs_max", (x, dt), want) == 0
    assert bits(s.read(m))[0] == bits(want)[0]
    s.close()


def test_async_device_read_follows_pending_runs(m3, gpu):
    """read_device_async copies the output of the runs enqueued before it
    (ABS_MAX writes a shadow buffer that only becomes current when its run
    is committed), with no host wait in between."""
    import torch

    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (1000,))
    m = g.inferred("ABS_MAX", [x], m3.OUTPUT, m3.F32)
    g.node("ABS_MAX", [x], [m])
    s = m3.Session(g)
    data = np.linspace(-3, 2, 1000).astype(np.float32)
    out = torch.zeros(2, dtype=torch.float32, device="cuda")
    for k, scale in enumerate((1.0, 2.0)):
        s.write(x, data * np.float32(scale))
        s.run_async()
        s.read_device_async(m, out.data_ptr() + 4 * k, 4)
    s.synchronize()
    assert out.cpu().tolist() == [3.0, 6.0]


def test_pipelined_host_submissions_match_synchronous_runs(m3, gpu):
    """Five submissions with host buffers in flight at once (uploads of one
    overlapping downloads of the previous) give each batch exactly the
    outputs of a synchronous write/run/read; a NaN batch fails the
    synchronise."""
    import torch

    rows, width = 64, 300

    def build(g):
        x = g.value(m3.INPUT, m3.F32, (rows, width))
        b = g.value(m3.INPUT, m3.F32, (1, width))
        t = g.inferred("ADD", [x, b], m3.TEMPORARY, m3.F32)
        g.node("ADD", [x, b], [t])
        p = g.inferred("SOFTMAX", [t], m3.OUTPUT, m3.F32)
        g.node("SOFTMAX", [t], [p])
        v = g.inferred("TOP_K", [t], m3.OUTPUT, m3.F32, k=1)
        i = g.inferred("TOP_K", [t], m3.OUTPUT, m3.I32, output_index=1, k=1)
        g.node("TOP_K", [t], [v, i], k=1)
        return x, b, p, v, i

    rng = np.random.default_rng(21)
    batches = [((rng.standard_normal((rows, width)) * 3).astype(np.float32),
                rng.standard_normal((1, width)).astype(np.float32)) for _ in range(5)]
    g = m3.Graph()
    x, b, p, v, i = build(g)
    s = m3.Session(g)
    expected = []
    for xs, bs in batches:
        s.write(x, xs)
        s.write(b, bs)
        s.run()
        expected.append([s.read(p).copy(), s.read(v).copy(), s.read(i).copy()])

    def pinned(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
        return t

    ins = [(pinned(xs), pinned(bs)) for xs, bs in batches]
    outs = [[torch.empty(e.shape, dtype=torch.from_numpy(e).dtype).pin_memory() for e in exp]
            for exp in expected]
    for (tx, tb), (tp, tv, ti) in zip(ins, outs):
        s.submit_host({x: tx.data_ptr(), b: tb.data_ptr()},
                      {p: tp.data_ptr(), v: tv.data_ptr(), i: ti.data_ptr()})
    s.synchronize()
    for got, exp in zip(outs, expected):
        for t, e in zip(got, exp):
            assert np.array_equal(bits(t.numpy()), bits(e))

    poisoned = ins[2][0].clone().pin_memory()
    poisoned[3, 7] = float("nan")
    s.submit_host({x: ins[1][0].data_ptr(), b: ins[1][1].data_ptr()},
                  {p: outs[0][0].data_ptr(), v: outs[0][1].data_ptr(), i: outs[0][2].data_ptr()})
    s.submit_host({x: poisoned.data_ptr(), b: ins[2][1].data_ptr()},
                  {p: outs[1][0].data_ptr(), v: outs[1][1].data_ptr(), i: outs[1][2].data_ptr()})
    with pytest.raises(m3.M3Failure) as failure:
        s.synchronize()
    assert failure.value.status == m3.OUT_OF_RANGE
    # the batch before the failure was delivered in full
    for t, e in zip(outs[0], expected[1]):
        assert np.array_equal(bits(t.numpy()), bits(e))


# ----------------------------------------------------------- row kernels


@pytest.mark.parametrize("width", [1, 7, 128, 1000, 1024, 3000])
@pytest.mark.parametrize("k", [1, 3])
def test_softmax_top_k(m3, ref, gpu, width, k):
    k = min(k, width)
    rng = np.random.default_rng(width)
    x = (rng.standard_normal((33, width)) * 3).astype(np.float32)
    x[rng.random(x.shape) < 0.01] = 20.0
    x[0, :] = -np.inf                       # all -inf row
    if width > 2:
        x[1, 0] = x[1, 2] = np.inf          # +inf entries split the mass
        x[2, :] = 5.0                       # ties -> lowest indices
        x[3, 0], x[3, 1] = -0.0, 0.0        # signed zeros compare equal

    def build(g):
        v = g.value(m3.INPUT, m3.F32, x.shape)
        p = g.inferred("SOFTMAX", [v], m3.OUTPUT, m3.F32)
        g.node("SOFTMAX", [v], [p])
        tv = g.inferred("TOP_K", [v], m3.OUTPUT, m3.F32, 0, k=k)
        ti = g.inferred("TOP_K", [v], m3.OUTPUT, m3.I32, 1, k=k)
        g.node("TOP_K", [v], [tv, ti], k=k)
        return {"x": v}, [p, tv, ti]

    (p, tv, ti), (rp, rtv, rti) = run_both(m3, ref, build, {"x": x})
    assert np.array_equal(bits(tv), bits(rtv)) and np.array_equal(ti, rti)
    rel = np.abs(p.astype(np.float64) - rp) / np.maximum(np.abs(rp), 1e-30)
    assert rel.max() <= 1e-6, rel.max()
    assert np.array_equal(p[0], rp[0]) and np.array_equal(p[1], rp[1])


@pytest.mark.parametrize("width", [512, 1024])
@pytest.mark.parametrize("mode", ["both", "softmax", "top_k"])
def test_softmax_compiled_widths_many_tiles(m3, ref, gpu, width, mode):
    """The compiled-width F32 kernel runs a ring of tile stages per CTA:
    enough rows for several tiles per CTA, a ragged last tile, special rows
    (all -inf, +inf entries, ties, exponentials below 2^-100) spread over
    the tensor, and each of the three output combinations."""
    rows = 8 * 2500 + 5
    rng = np.random.default_rng(width + len(mode))
    x = (rng.standard_normal((rows, width)) * 3).astype(np.float32)
    for r in rng.choice(rows, 40, replace=False):
        kind = r % 4
        if kind == 0:
            x[r, :] = -np.inf
        elif kind == 1:
            x[r, rng.choice(width, 3, replace=False)] = np.inf
        elif kind == 2:
            x[r, :] = 5.0
        else:
            x[r, rng.choice(width, 5, replace=False)] = 90.0   # the rest underflow past 2^-100
    x[-1, :] = -np.inf

    def build(g):
        v = g.value(m3.INPUT, m3.F32, x.shape)
        outs = []
        if mode != "top_k":
            p = g.inferred("SOFTMAX", [v], m3.OUTPUT, m3.F32)
            g.node("SOFTMAX", [v], [p])
            outs.append(p)
        if mode != "softmax":
            tv = g.inferred("TOP_K", [v], m3.OUTPUT, m3.F32, 0, k=1)
            ti = g.inferred("TOP_K", [v], m3.OUTPUT, m3.I32, 1, k=1)
            g.node("TOP_K", [v], [tv, ti], k=1)
            outs += [tv, ti]
        return {"x": v}, outs

    got, want = run_both(m3, ref, build, {"x": x})
    if mode != "top_k":
        p, rp = got.pop(0), want.pop(0)
        rel = np.abs(p.astype(np.float64) - rp) / np.maximum(np.abs(rp), 1e-30)
        assert rel.max() <= 1e-6, rel.max()
    if mode != "softmax":
        assert np.array_equal(bits(got[0]), bits(want[0])) and np.array_equal(got[1], want[1])


def test_softmax_compiled_width_nan_deep_in_tensor(m3, gpu):
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (20000, 1024))
    p = g.inferred("SOFTMAX", [x], m3.OUTPUT, m3.F32)
    g.node("SOFTMAX", [x], [p])
    s = m3.Session(g)
    good = np.random.default_rng(4).standard_normal((20000, 1024)).astype(np.float32)
    s.write(x, good)
    s.run()
    before = s.read(p).copy()
    bad = good.copy()
    bad[17771, 1000] = np.nan
    s.write(x, bad)
    status, message = s.run_status()
    assert status == m3.OUT_OF_RANGE and message == "softmax input contains NaN"
    assert np.array_equal(s.read(p), before)


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
def test_softmax_low_precision(m3, ref, oracle, gpu, dtype):
    dt = getattr(m3, dtype)
    enc = oracle.to_f16 if dtype == "F16" else oracle.to_bf16
    rng = np.random.default_rng(9)
    x = enc((rng.standard_normal((40, 512)) * 3).astype(np.float32))

    def build(g):
        v = g.value(m3.INPUT, dt, x.shape)
        p = g.inferred("SOFTMAX", [v], m3.OUTPUT, dt)
        g.node("SOFTMAX", [v], [p])
        return {"x": v}, [p]

    (p,), (rp,) = run_both(m3, ref, build, {"x": x})
    assert ulp_distance(p, rp).max() <= 1


def test_softmax_nan_leaves_outputs_untouched(m3, gpu):
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (4, 64))
    p = g.inferred("SOFTMAX", [x], m3.OUTPUT, m3.F32)
    g.node("SOFTMAX", [x], [p])
    tv = g.inferred("TOP_K", [x], m3.OUTPUT, m3.F32, 0, k=2)
    ti = g.inferred("TOP_K", [x], m3.OUTPUT, m3.I32, 1, k=2)
    g.node("TOP_K", [x], [tv, ti], k=2)
    s = m3.Session(g)
    good = np.arange(256, dtype=np.float32).reshape(4, 64) / 64
    s.write(x, good)
    s.run()
    before = [s.read(v).copy() for v in (p, tv, ti)]
    bad = good.copy()
    bad[3, 17] = np.nan
    s.write(x, bad)
    status, message = s.run_status()
    # tests/test_op_sampling.c:83-96
    assert status == m3.OUT_OF_RANGE and message == "softmax input contains NaN"
    after = [s.read(v) for v in (p, tv, ti)]
    for a, b in zip(before, after):
        assert np.array_equal(a, b)
    # the session stays usable and commits again
    s.write(x, good * 2.0)           # a different (not shift-equivalent) input
    s.run()
    assert not np.array_equal(s.read(p), before[0])


@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
@pytest.mark.parametrize("rows,width", [(70, 1024), (33, 64), (5, 4096)])
@pytest.mark.parametrize("residual", ["none", "temporary"])
def test_rms_norm_row_groups_bit_exact(m3, ref, oracle, gpu, dtype, rows, width, residual):
    """RMSNorm without a residual (the lane-per-row kernel reads the input
    twice) and with a residual sum that is not an output (the row-tile
    kernel), over ragged row counts: bit-exact against the reference."""
    dt = getattr(m3, dtype)
    enc = {"F32": lambda v: v, "F16": oracle.to_f16, "BF16": oracle.to_bf16}[dtype]
    rng = np.random.default_rng(rows * width)
    h = enc(rng.standard_normal((rows, width)).astype(np.float32))
    r = enc(rng.standard_normal((rows, width)).astype(np.float32))
    w = enc(rng.normal(1, 0.05, width).astype(np.float32))

    def build(g):
        vh = g.value(m3.INPUT, dt, h.shape)
        vw = g.constant(dt, w)
        handles = {"h": vh}
        x = vh
        if residual == "temporary":
            vr = g.value(m3.INPUT, dt, r.shape)
            handles["r"] = vr
            x = g.inferred("ADD", [vh, vr], m3.TEMPORARY, dt)
            g.node("ADD", [vh, vr], [x])
        n = g.inferred("RMS_NORM", [x, vw], m3.OUTPUT, dt, epsilon=1e-6)
        g.node("RMS_NORM", [x, vw], [n], epsilon=1e-6)
        return handles, [n]

    inputs = {"h": h, "r": r}
    (mine,), (theirs,) = run_both(m3, ref, build, inputs)
    assert np.array_equal(bits(mine), bits(theirs))


@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
@pytest.mark.parametrize("width", [5, 64, 2048, 3000])
def test_residual_rms_norm_bit_exact(m3, ref, oracle, gpu, dtype, width):
    dt = getattr(m3, dtype)
    enc = {"F32": lambda v: v, "F16": oracle.to_f16, "BF16": oracle.to_bf16}[dtype]
    rng = np.random.default_rng(width)
    h = enc(rng.standard_normal((48, width)).astype(np.float32))
    r = enc(rng.standard_normal((48, width)).astype(np.float32))
    w = enc(rng.normal(1, 0.05, width).astype(np.float32))

    def build(g):
        vh = g.value(m3.INPUT, dt, h.shape)
        vr = g.value(m3.INPUT, dt, r.shape)
        vw = g.constant(dt, w)
        s = g.inferred("ADD", [vh, vr], m3.OUTPUT, dt)
        g.node("ADD", [vh, vr], [s])
        n = g.inferred("RMS_NORM", [s, vw], m3.OUTPUT, dt, epsilon=1e-6)
        g.node("RMS_NORM", [s, vw], [n], epsilon=1e-6)
        return {"h": vh, "r": vr}, [s, n]

    mine, theirs = run_both(m3, ref, build, {"h": h, "r": r})
    for a, b in zip(mine, theirs):
        assert np.array_equal(bits(a), bits(b))


@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
@pytest.mark.parametrize("rows", [1, 23, 25, 97, 148 * 24 + 7])
@pytest.mark.parametrize("residual", ["none", "temporary", "output"])
def test_rms_norm_4k_rows_bit_exact(m3, ref, oracle, gpu, dtype, rows, residual):
    """RMSNorm over the benchmark's 4 KiB rows (2048 16-bit or 1024 F32
    elements) with the residual sum absent, a temporary, or a graph output,
    over row counts from one row to many tiles per CTA: bit-exact against the
    reference, rows holding an infinity or a NaN included."""
    dt = getattr(m3, dtype)
    width = 1024 if dtype == "F32" else 2048
    enc = {"F32": lambda v: v, "F16": oracle.to_f16, "BF16": oracle.to_bf16}[dtype]
    rng = np.random.default_rng(rows + width)
    h = rng.standard_normal((rows, width)).astype(np.float32)
    r = rng.standard_normal((rows, width)).astype(np.float32)
    if rows > 2:
        h[1, 7] = np.inf          # an infinite row and a NaN row stay row-local
        h[2, 9] = np.nan
        h[rows - 1] *= 300.0      # large squares
    h, r = enc(h), enc(r)
    w = enc(rng.normal(1, 0.05, width).astype(np.float32))

    def build(g):
        vh = g.value(m3.INPUT, dt, h.shape)
        vw = g.constant(dt, w)
        handles = {"h": vh}
        outputs = []
        x = vh
        if residual != "none":
            vr = g.value(m3.INPUT, dt, r.shape)
            handles["r"] = vr
            kind = m3.OUTPUT if residual == "output" else m3.TEMPORARY
            x = g.inferred("ADD", [vh, vr], kind, dt)
            g.node("ADD", [vh, vr], [x])
            if residual == "output":
                outputs.append(x)
        n = g.inferred("RMS_NORM", [x, vw], m3.OUTPUT, dt, epsilon=1e-6)
        g.node("RMS_NORM", [x, vw], [n], epsilon=1e-6)
        return handles, outputs + [n]

    def nan_mask(b):
        if b.dtype.itemsize == 4:
            return np.isnan(b.view(np.float32))
        exponent, mantissa = (0x7c00, 0x03ff) if dtype == "F16" else (0x7f80, 0x007f)
        return ((b & exponent) == exponent) & ((b & mantissa) != 0)

    mine, theirs = run_both(m3, ref, build, {"h": h, "r": r})
    for a, b in zip(mine, theirs):
        ba, bb = bits(a), bits(b)
        na, nb = nan_mask(ba), nan_mask(bb)
        # NaNs made by arithmetic carry each platform's default NaN: compare
        # NaN-ness there and bits everywhere else
        assert np.array_equal(na, nb)
        assert np.array_equal(ba[~na], bb[~nb])
    if rows > 2:
        assert nan_mask(bits(mine[-1]))[2].all()   # the NaN row of the norm


@pytest.mark.parametrize("dtype", ["F32", "F16"])
@pytest.mark.parametrize("bias", [True, False])
def test_layer_norm_bit_exact(m3, ref, oracle, gpu, dtype, bias):
    dt = getattr(m3, dtype)
    enc = {"F32": lambda v: v, "F16": oracle.to_f16}[dtype]
    rng = np.random.default_rng(21)
    x = enc((rng.standard_normal((40, 771)) * 2 + 0.5).astype(np.float32))
    w = enc(rng.normal(1, 0.1, 771).astype(np.float32))
    b = enc(rng.normal(0, 0.1, 771).astype(np.float32))

    def build(g):
        vx = g.value(m3.INPUT, dt, x.shape)
        vw = g.constant(dt, w)
        vb = g.constant(dt, b) if bias else m3.VALUE_NONE
        n = g.inferred("LAYER_NORM", [vx, vw], m3.OUTPUT, m3.F32, epsilon=1e-5)
        g.node("LAYER_NORM", [vx, vw, vb], [n], epsilon=1e-5)
        return {"x": vx}, [n]

    (n,), (rn,) = run_both(m3, ref, build, {"x": x})
    assert np.array_equal(bits(n), bits(rn))


# -------------------------------------------------------- session runtime


def test_liveness_graph_and_plan_info(m3, gpu):
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (4,))
    c = np.array([0.5, -1, 2, 3], np.float32)
    vc = g.constant(m3.F32, c)
    a = g.inferred("ADD", [x, vc], m3.TEMPORARY, m3.F32)
    g.node("ADD", [x, vc], [a])
    t = g.inferred("TANH", [a], m3.TEMPORARY, m3.F32)
    g.node("TANH", [a], [t])
    m = g.inferred("MUL", [t, vc], m3.TEMPORARY, m3.F32)
    g.node("MUL", [t, vc], [m])
    y = g.inferred("ADD", [m, x], m3.OUTPUT, m3.F32)
    g.node("ADD", [m, x], [y])
    s = m3.Session(g)
    g.close()                                   # the session outlives its graph
    info = s.plan_info()
    assert (info.value_count, info.node_count, info.storage_slot_count,
            info.allocated_bytes) == (6, 4, 5, 80)
    assert all(s.provider(i) == m3.PROVIDER_CUDA for i in range(4))
    data = np.array([1.0, 2.0, -3.0, 0.25], np.float32)
    s.write(x, data)
    s.run()
    out = s.read(y)
    expect = np.tanh(data + c) * c + data        # tests/test_graph_runtime.c:140-146
    assert np.allclose(out, expect, rtol=1e-6)
    # role and size checks (tests/test_graph_runtime.c:148-160)
    with pytest.raises(m3.M3Failure) as failure:
        s.write(y, data)
    assert failure.value.status == m3.INVALID_ARGUMENT
    with pytest.raises(m3.M3Failure) as failure:
        s.write(x, data[:3])
    assert failure.value.status == m3.INVALID_ARGUMENT


@pytest.mark.parametrize("mode", ["async", "async_no_graphs", "steps"])
def test_async_runs_and_swap_carry_state(m3, ref, gpu, mode):
    """Thirty Euler steps carried on the device equal thirty synchronous
    runs with host round trips: run_async + swap (each run one graph launch,
    or plain launches), and run_steps (the thirty runs as one graph launch).
    The sequence runs twice so the second pass replays cached graphs."""
    rng = np.random.default_rng(3)
    shape = (2, 8, 96)
    x0, vc, vu = (rng.standard_normal(shape).astype(np.float32) for _ in range(3))

    def build(g):
        x = g.value(m3.INPUT, m3.F32, shape)
        c = g.value(m3.INPUT, m3.F32, shape)
        u = g.value(m3.INPUT, m3.F32, shape)
        k1 = g.constant(m3.F32, np.array([-1], np.float32))
        kg = g.constant(m3.F32, np.array([4], np.float32))
        kd = g.constant(m3.F32, np.array([1.0 / 30.0], np.float32))
        a = g.inferred("MUL", [u, k1], m3.TEMPORARY, m3.F32)
        g.node("MUL", [u, k1], [a])
        a2 = g.inferred("ADD", [c, a], m3.TEMPORARY, m3.F32)
        g.node("ADD", [c, a], [a2])
        a3 = g.inferred("MUL", [a2, kg], m3.TEMPORARY, m3.F32)
        g.node("MUL", [a2, kg], [a3])
        v = g.inferred("ADD", [u, a3], m3.TEMPORARY, m3.F32)
        g.node("ADD", [u, a3], [v])
        t = g.inferred("MUL", [v, kd], m3.TEMPORARY, m3.F32)
        g.node("MUL", [v, kd], [t])
        xn = g.inferred("ADD", [x, t], m3.OUTPUT, m3.F32)
        g.node("ADD", [x, t], [xn])
        xb = g.inferred("CAST", [xn], m3.OUTPUT, m3.BF16)
        g.node("CAST", [xn], [xb])
        return x, c, u, xn, xb

    rg = m3.Graph(lib=ref)
    rx, rc, ru, rxn, rxb = build(rg)
    rs = m3.Session(rg, allow_metal=False, allow_neural_engine=False, cuda=False)
    rs.write(rc, vc)
    rs.write(ru, vu)
    state = x0
    for _ in range(30):
        rs.write(rx, state)
        rs.run()
        state = rs.read(rxn).copy()
    ref_bf16 = rs.read(rxb)

    g = m3.Graph()
    x, c, u, xn, xb = build(g)
    s = m3.Session(g, cuda_graphs=mode != "async_no_graphs")
    s.write(c, vc)
    s.write(u, vu)
    for _ in range(2):
        s.write(x, x0)
        if mode == "steps":
            s.run_steps(30, x, xn)
        else:
            for step in range(30):
                s.run_async()
                if step != 29:
                    s.swap(x, xn)
        s.synchronize()
        assert np.array_equal(bits(s.read(xn)), bits(state))
        assert np.array_equal(s.read(xb), ref_bf16)


# ------------------------------------------------- backend plug-in path


def test_backend_plugin_strided_commands(m3, oracle, gpu):
    """The vtable functions run reference-layout commands on strided views."""
    import ctypes

    lib = m3.load()
    storages = {}

    @m3.STORAGE_DATA
    def storage_data(storage):
        return storages[storage]

    options = m3.BackendOptions(0, storage_data, False)
    context = ctypes.c_void_p()
    err = m3.M3Error()
    m3.check(lib.m3_cuda_backend_context_create(ctypes.byref(options),
                                                ctypes.byref(context),
                                                ctypes.byref(err)), err)

    def allocate(nbytes):
        handle, data = ctypes.c_void_p(), ctypes.c_void_p()
        m3.check(lib.m3_cuda_backend_allocate(context, nbytes, 64,
                                              ctypes.byref(handle),
                                              ctypes.byref(data),
                                              ctypes.byref(err)), err)
        key = len(storages) + 1
        storages[key] = data.value
        return key, data.value

    def view(key, dtype, shape, strides, offset=0):
        v = m3.TensorView()
        v.metadata.dtype = dtype
        v.metadata.rank = len(shape)
        count = int(np.prod(shape))
        for i, (n, st) in enumerate(zip(shape, strides)):
            v.metadata.shape[i] = n
            v.byte_strides[i] = st
        v.metadata.element_count = count
        v.metadata.byte_count = count * m3.ITEMSIZE[dtype]
        v.byte_offset = offset
        v.storage = key
        return v

    # transposed [2,3] view of a [3,2] buffer + row vector [3] -> contiguous
    backing = np.array([1, 4, 2, 5, 3, 6], np.float32)
    k_in, p_in = allocate(backing.nbytes)
    lib.m3_cuda_backend_write(context, p_in, 0, backing.ctypes.data, backing.nbytes,
                              ctypes.byref(err))
    vec = np.array([10, 20, 30], np.float32)
    k_vec, p_vec = allocate(vec.nbytes)
    lib.m3_cuda_backend_write(context, p_vec, 0, vec.ctypes.data, vec.nbytes,
                              ctypes.byref(err))
    k_out, p_out = allocate(24)
    left = view(k_in, m3.F32, (2, 3), (4, 8))
    right = view(k_vec, m3.F32, (3,), (4,))
    out = view(k_out, m3.F32, (2, 3), (12, 4))
    cmd = (m3.Command * 2)()
    cmd[0].kind = m3.OPS["ADD"]
    cmd[0].descriptor.add.left = ctypes.pointer(left)
    cmd[0].descriptor.add.right = ctypes.pointer(right)
    cmd[0].descriptor.add.output = ctypes.pointer(out)
    cmd[1].kind = m3.OPS["SOFTMAX"]
    cmd[1].descriptor.softmax.input = ctypes.pointer(left)
    k_p, p_p = allocate(24)
    probs = view(k_p, m3.F32, (2, 3), (12, 4))
    cmd[1].descriptor.softmax.output = ctypes.pointer(probs)
    m3.check(lib.m3_cuda_backend_execute(context, cmd, 2, None, ctypes.byref(err)), err)
    host = np.zeros(6, np.float32)
    lib.m3_cuda_backend_read(context, p_out, 0, host.ctypes.data, 24, ctypes.byref(err))
    assert list(host) == [11, 22, 33, 14, 25, 36]     # tests/test_op_basic.c:214-222
    lib.m3_cuda_backend_read(context, p_p, 0, host.ctypes.data, 24, ctypes.byref(err))
    dense = np.lib.stride_tricks.as_strided(backing, (2, 3), (4, 8)).copy()
    expect = np.zeros_like(dense)
    assert oracle.run("softmax", dense, expect) == 0
    assert np.abs(host.reshape(2, 3) - expect).max() <= 1e-6
    # NaN: the failing command writes nothing and later commands do not run
    sentinel = np.full(6, -7, np.float32)
    lib.m3_cuda_backend_write(context, p_p, 0, sentinel.ctypes.data, 24, ctypes.byref(err))
    poisoned = backing.copy()
    poisoned[2] = np.nan
    lib.m3_cuda_backend_write(context, p_in, 0, poisoned.ctypes.data, 24, ctypes.byref(err))
    status = lib.m3_cuda_backend_execute(context, cmd, 2, None, ctypes.byref(err))
    assert status == m3.OUT_OF_RANGE
    lib.m3_cuda_backend_read(context, p_p, 0, host.ctypes.data, 24, ctypes.byref(err))
    assert list(host) == list(sentinel)
    for key in list(storages):
        lib.m3_cuda_backend_free_storage(context, storages[key], storages[key])
    lib.m3_cuda_backend_destroy_context(context)


class _Backend:
    """The plug-in context with host-side storage bookkeeping, as the
    reference's backend layer would hold it."""

    def __init__(self, m3):
        import ctypes

        self.m3, self.ctypes = m3, ctypes
        self.lib = m3.load()
        self.storages = {}
        self.err = m3.M3Error()

        @m3.STORAGE_DATA
        def storage_data(storage):
            return self.storages[storage]

        self._keep = storage_data
        options = m3.BackendOptions(0, storage_data, False)
        self.context = ctypes.c_void_p()
        m3.check(self.lib.m3_cuda_backend_context_create(
            ctypes.byref(options), ctypes.byref(self.context), ctypes.byref(self.err)), self.err)

    def tensor(self, array):
        ctypes = self.ctypes
        handle, data = ctypes.c_void_p(), ctypes.c_void_p()
        self.m3.check(self.lib.m3_cuda_backend_allocate(
            self.context, array.nbytes, 64, ctypes.byref(handle), ctypes.byref(data),
            ctypes.byref(self.err)), self.err)
        key = len(self.storages) + 1
        self.storages[key] = data.value
        self.m3.check(self.lib.m3_cuda_backend_write(
            self.context, data.value, 0, array.ctypes.data, array.nbytes,
            ctypes.byref(self.err)), self.err)
        return key

    def view(self, key, shape, offset=0, dtype=None):
        m3 = self.m3
        v = m3.TensorView()
        v.metadata.dtype = m3.F32 if dtype is None else dtype
        v.metadata.rank = len(shape)
        stride = 4
        for i in reversed(range(len(shape))):
            v.metadata.shape[i] = shape[i]
            v.byte_strides[i] = stride
            stride *= shape[i]
        count = int(np.prod(shape))
        v.metadata.element_count = count
        v.metadata.byte_count = count * 4
        v.byte_offset = offset
        v.storage = key
        return v

    def read(self, key, count):
        host = np.zeros(count, np.float32)
        self.m3.check(self.lib.m3_cuda_backend_read(
            self.context, self.storages[key], 0, host.ctypes.data, host.nbytes,
            self.ctypes.byref(self.err)), self.err)
        return host

    def execute(self, commands):
        cmd = (self.m3.Command * len(commands))()
        keep = []
        for i, (kind, a, b, out) in enumerate(commands):
            cmd[i].kind = self.m3.OPS[kind]
            keep += [a, b, out]
            cmd[i].descriptor.add.left = self.ctypes.pointer(a)
            cmd[i].descriptor.add.right = self.ctypes.pointer(b)
            cmd[i].descriptor.add.output = self.ctypes.pointer(out)
        return self.lib.m3_cuda_backend_execute(self.context, cmd, len(commands), None,
                                                self.ctypes.byref(self.err))

    def close(self):
        for key in list(self.storages):
            self.lib.m3_cuda_backend_free_storage(self.context, self.storages[key],
                                                  self.storages[key])
        self.lib.m3_cuda_backend_destroy_context(self.context)


def test_flow_overlap_blend_through_backend_commands(m3, gpu):
    """The flow solver's overlap blend as the reference issues it
    (src/m3_flow_solver_math.c:137-205): MUL(noise_prompt, scalar) ->
    arithmetic; MUL(previous_latent, scalar) -> the latent's first `overlap`
    time steps (a view into the latent); ADD(arithmetic, that view) -> the
    same view (exact alias).  Bit-exact with F32 statements; the rest of the
    latent is untouched."""
    rng = np.random.default_rng(31)
    length, overlap, channels = 40, 12, 24
    latent = rng.standard_normal((1, length, channels)).astype(np.float32)
    prompt = rng.standard_normal((1, overlap, channels)).astype(np.float32)
    previous = rng.standard_normal((1, overlap, channels)).astype(np.float32)
    c_noise, c_prev = np.float32(0.3125), np.float32(0.6875)
    be = _Backend(m3)
    try:
        k_lat = be.tensor(latent)
        k_pr = be.tensor(prompt)
        k_pv = be.tensor(previous)
        k_s1 = be.tensor(np.array([c_noise], np.float32))
        k_s2 = be.tensor(np.array([c_prev], np.float32))
        k_ar = be.tensor(np.zeros((1, overlap, channels), np.float32))
        head = be.view(k_lat, (1, overlap, channels))
        status = be.execute([
            ("MUL", be.view(k_pr, (1, overlap, channels)), be.view(k_s1, (1,)),
             be.view(k_ar, (1, overlap, channels))),
            ("MUL", be.view(k_pv, (1, overlap, channels)), be.view(k_s2, (1,)), head),
            ("ADD", be.view(k_ar, (1, overlap, channels)), head, head),
        ])
        assert status == m3.OK
        got = be.read(k_lat, latent.size).reshape(latent.shape)
        expect = latent.copy()
        expect[:, :overlap] = prompt * c_noise + previous * c_prev
        assert np.array_equal(bits(got), bits(expect))
    finally:
        be.close()


# ------------------------------------------------------ categorical sampling


def _categorical_inputs(dtype_name, oracle, rows=37, vocab=1000, seed=41):
    rng = np.random.default_rng(seed)
    probs = rng.random((rows, vocab)).astype(np.float32)
    probs[rng.random((rows, vocab)) < 0.3] = 0.0
    probs[4] = 0.0
    probs[4, 17] = 0.25                      # one positive entry
    probs[6, -1] = 0.0                       # last positive is not the last
    # at most 0.99, so rounding to a 16-bit dtype cannot reach 1.0
    uniforms = np.minimum(rng.random(rows), 0.99).astype(np.float32)
    uniforms[0] = 0.0
    uniforms[1] = (np.nextafter(np.float32(1.0), np.float32(0.0)) if dtype_name == "F32"
                   else np.float32(0.99609375))  # largest below one in the dtype
    enc = {"F32": lambda v: v, "F16": oracle.to_f16, "BF16": oracle.to_bf16}[dtype_name]
    return enc(probs), enc(uniforms)


def _categorical_graph(m3, g, dt, rows, vocab):
    p = g.value(m3.INPUT, dt, (rows, vocab))
    u = g.value(m3.INPUT, dt, (rows,))
    i = g.inferred("CATEGORICAL", [p, u], m3.OUTPUT, m3.I32)
    g.node("CATEGORICAL", [p, u], [i])
    return {"p": p, "u": u}, [i]


@pytest.mark.parametrize("vocab", [1000, 1024])
@pytest.mark.parametrize("dtype", ["F32", "F16", "BF16"])
def test_categorical_matches_reference(m3, ref, oracle, gpu, dtype, vocab):
    """Categorical sampling (src/m3_op_execute_sampling.c:90-137): the same
    index as the reference CPU provider for every row, including a zero
    uniform, the largest uniform below one and rows with few positives.
    Rows of whole 128-byte chunks (vocab 1024) take the warp-group kernel,
    others the thread-per-row kernel."""
    probs, uniforms = _categorical_inputs(dtype, oracle, vocab=vocab)
    dt = getattr(m3, dtype)
    (mine,), (theirs,) = run_both(
        m3, ref, lambda g: _categorical_graph(m3, g, dt, *probs.shape),
        {"p": probs, "u": uniforms})
    assert np.array_equal(mine, theirs)


@pytest.mark.parametrize("dtype,rows,vocab", [("F32", 20000, 1024), ("F16", 3000, 2048),
                                              ("BF16", 45, 4096), ("F32", 70, 2048),
                                              ("F32", 50, 1001), ("F32", 9, 3000)])
def test_categorical_shapes_match_reference(m3, ref, oracle, gpu, dtype, rows, vocab):
    """Warp groups of 32 rows over 128-byte chunks (rows of 2 to 8 KiB, a
    ragged last group), and widths that are not whole chunks or exceed
    8 KiB (read straight from global memory): the reference's index for
    every row."""
    probs, uniforms = _categorical_inputs(dtype, oracle, rows=rows, vocab=vocab, seed=rows + vocab)
    dt = getattr(m3, dtype)
    (mine,), (theirs,) = run_both(
        m3, ref, lambda g: _categorical_graph(m3, g, dt, *probs.shape),
        {"p": probs, "u": uniforms})
    assert np.array_equal(mine, theirs)


@pytest.mark.parametrize("vocab", [1000, 1024])
def test_categorical_checks_match_reference(m3, ref, oracle, gpu, vocab):
    """Each failing check fails the run with the reference's message, picks
    the failure of the earliest row, and leaves the output untouched."""
    probs, uniforms = _categorical_inputs("F32", oracle, vocab=vocab)
    rows, vocab = probs.shape
    g = m3.Graph()
    handles, (out,) = _categorical_graph(m3, g, m3.F32, rows, vocab)
    s = m3.Session(g)
    s.write(handles["p"], probs)
    s.write(handles["u"], uniforms)
    s.run()
    good = s.read(out).copy()
    rg = m3.Graph(lib=ref)
    rhandles, _ = _categorical_graph(m3, rg, m3.F32, rows, vocab)
    rs = m3.Session(rg, allow_metal=False, allow_neural_engine=False, cuda=False)

    def poison(kind):
        p, u = probs.copy(), uniforms.copy()
        if kind == "uniform":
            u[9] = 1.0
        elif kind == "probability":
            p[5, 7] = -1.0
        elif kind == "nan":
            p[8, 3] = np.nan
        elif kind == "sum":
            p[2] = 0.0
        elif kind == "order":          # a probability failure in an earlier
            p[3, 1] = np.inf           # row than a uniform failure
            u[11] = -0.5
        return p, u

    for kind in ("uniform", "probability", "nan", "sum", "order"):
        p, u = poison(kind)
        for session, hs in ((s, handles), (rs, rhandles)):
            session.write(hs["p"], p)
            session.write(hs["u"], u)
        status, message = s.run_status()
        ref_status, ref_message = rs.run_status()
        assert status == ref_status == m3.OUT_OF_RANGE, kind
        assert message == ref_message, kind
        assert np.array_equal(s.read(out), good), kind


def test_categorical_through_backend_commands(m3, oracle, gpu):
    """The plug-in path: checks first, then the draws; a failing command
    writes nothing."""
    probs, uniforms = _categorical_inputs("F32", oracle, rows=9, vocab=64, seed=5)
    g = m3.Graph(lib=m3.load())
    handles, (out,) = _categorical_graph(m3, g, m3.F32, *probs.shape)
    s = m3.Session(g)
    s.write(handles["p"], probs)
    s.write(handles["u"], uniforms)
    s.run()
    expected = s.read(out).copy()
    be = _Backend(m3)
    try:
        k_p = be.tensor(probs)
        k_u = be.tensor(uniforms)
        k_o = be.tensor(np.full(9, -3, np.int32).view(np.float32))
        cmd = (m3.Command * 1)()
        pv = be.view(k_p, probs.shape)
        uv = be.view(k_u, (9,))
        ov = be.view(k_o, (9,), dtype=m3.I32)
        cmd[0].kind = m3.OPS["CATEGORICAL"]
        cmd[0].descriptor.categorical.probabilities = be.ctypes.pointer(pv)
        cmd[0].descriptor.categorical.uniforms = be.ctypes.pointer(uv)
        cmd[0].descriptor.categorical.output = be.ctypes.pointer(ov)
        status = be.lib.m3_cuda_backend_execute(be.context, cmd, 1, None, be.ctypes.byref(be.err))
        assert status == m3.OK
        assert np.array_equal(be.read(k_o, 9).view(np.int32), expected)
        bad = uniforms.copy()
        bad[4] = 2.0
        be.lib.m3_cuda_backend_write(be.context, be.storages[k_u], 0, bad.ctypes.data, bad.nbytes,
                                     be.ctypes.byref(be.err))
        sentinel = np.full(9, -3, np.int32)
        be.lib.m3_cuda_backend_write(be.context, be.storages[k_o], 0, sentinel.ctypes.data, 36,
                                     be.ctypes.byref(be.err))
        status = be.lib.m3_cuda_backend_execute(be.context, cmd, 1, None, be.ctypes.byref(be.err))
        assert status == m3.OUT_OF_RANGE
        assert be.err.message.decode() == "categorical uniform is outside [0,1)"
        assert np.array_equal(be.read(k_o, 9).view(np.int32), sentinel)
    finally:
        be.close()


def test_wave_interleave_through_backend_copy(m3, gpu):
    """The WAVE writer's sample layout (src/m3_wav.c:232-276): IEEE float32
    stereo, frame by frame the left sample's bits then the right's.  From the
    assembled planar [1, 2, N] signal that is one COPY whose input view walks
    frames with a 4-byte stride and channels with a 4N-byte stride, into a
    contiguous [N, 2] tensor: bit for bit, NaN payloads included."""
    rng = np.random.default_rng(67)
    n = 1001                                   # not a multiple of the vector width
    planar = rng.uniform(-1.0, 1.0, (1, 2, n)).astype(np.float32)
    planar[0, 0, 3] = np.float32(-0.0)
    planar[0, 1, 4] = np.uint32(0x7FC0BEEF).view(np.float32)
    planar[0, 0, 5] = np.float32(1e-42)
    planar[0, 1, 6] = np.float32(np.inf)
    be = _Backend(m3)
    try:
        k_planar = be.tensor(planar)
        k_wave = be.tensor(np.zeros((n, 2), np.float32))
        src = be.view(k_planar, (n, 2))
        src.byte_strides[0] = 4                # next frame
        src.byte_strides[1] = 4 * n            # next channel plane
        dst = be.view(k_wave, (n, 2))
        cmd = (m3.Command * 1)()
        cmd[0].kind = m3.OPS["COPY"]
        cmd[0].descriptor.copy.input = be.ctypes.pointer(src)
        cmd[0].descriptor.copy.output = be.ctypes.pointer(dst)
        status = be.lib.m3_cuda_backend_execute(be.context, cmd, 1, None, be.ctypes.byref(be.err))
        assert status == m3.OK
        got = be.read(k_wave, 2 * n).view(np.uint32)
        want = np.stack([planar[0, 0], planar[0, 1]], axis=1).reshape(-1).view(np.uint32)
        assert np.array_equal(got, want)
    finally:
        be.close()


def test_waveform_assembly_through_backend_commands(m3, gpu):
    """Waveform assembly's per-channel crop-and-clamp copy
    (src/m3_waveform.c:360-450) as CLAMP_UNIT commands on views: two decoded
    chunks of a stereo signal, each cropped and written at its place in the
    planar output.  Values beyond +-1 become +-1; NaN payloads, signed zeros
    and subnormals are copied bit for bit."""
    rng = np.random.default_rng(61)
    chunks = [(rng.standard_normal((2, 100)) * 1.5).astype(np.float32) for _ in range(2)]
    chunks[0][0, 12] = np.float32(-0.0)
    chunks[0][1, 20] = np.uint32(0x7FC01234).view(np.float32)
    chunks[1][0, 30] = np.float32(1e-42)
    crops = [(10, 60), (5, 70)]          # (crop start, copy count) per chunk
    total = sum(count for _, count in crops)
    be = _Backend(m3)
    try:
        keys = [be.tensor(c) for c in chunks]
        k_out = be.tensor(np.zeros((1, 2, total), np.float32))
        commands = []
        written = 0
        for key, (start, count) in zip(keys, crops):
            for ch in range(2):
                src = be.view(key, (count,), offset=(ch * 100 + start) * 4)
                dst = be.view(k_out, (count,), offset=(ch * total + written) * 4)
                commands.append(("CLAMP_UNIT", src, dst))
            written += count
        cmd = (m3.Command * len(commands))()
        for k, (kind, src, dst) in enumerate(commands):
            cmd[k].kind = m3.OPS[kind]
            cmd[k].descriptor.copy.input = be.ctypes.pointer(src)
            cmd[k].descriptor.copy.output = be.ctypes.pointer(dst)
        status = be.lib.m3_cuda_backend_execute(be.context, cmd, len(commands), None,
                                                be.ctypes.byref(be.err))
        assert status == m3.OK
        got = be.read(k_out, 2 * total).reshape(2, total)
        want = np.concatenate([c[:, s:s + n] for c, (s, n) in zip(chunks, crops)], axis=1)
        w = want.view(np.uint32).copy()
        mag = w & 0x7FFFFFFF
        beyond = (mag > 0x3F800000) & (mag <= 0x7F800000)
        w[beyond] = (w[beyond] & 0x80000000) | 0x3F800000
        assert np.array_equal(got.view(np.uint32), w)
    finally:
        be.close()
