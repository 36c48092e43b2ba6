"""Host-side logic of libm3cuda.so, without a GPU.

* The library loads on a machine without a device and exports every function
  include/m3_cuda.h declares.
* The session compiler (m3_cuda_graph_plan: topology, liveness slots,
  validation, placement, fusion) agrees with the reference's session compiler
  on plan info and on every rejection the reference's tests exercise.
* The fusion pass produces the launch groups the benchmark configurations
  rely on.
* The host RNG reproduces the reference's m3_rng streams bit for bit.
"""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions() -> list[str]:
    text = open(os.path.join(ROOT, "include", "m3_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(m3_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(m3):
    lib = m3.load()
    names = declared_functions()
    assert len(names) > 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert missing == []


def test_library_loads_without_device(m3):
    # on a GPU-less host this is 0 and no call faults
    assert m3.load().m3_cuda_device_count() >= 0
    assert m3.load().m3_version().decode().startswith("0.1")


def build_liveness_graph(m3, lib):
    # tests/test_graph_runtime.c:29-85 (the reference's liveness fixture):
    # out = tanh(in + c) * c + in
    g = m3.Graph(lib=lib)
    x = g.value(m3.INPUT, m3.F32, (4,))
    c = g.constant(m3.F32, np.array([0.5, -1, 2, 3], np.float32))
    a = g.inferred("ADD", [x, c], m3.TEMPORARY, m3.F32)
    g.node("ADD", [x, c], [a])
    t = g.inferred("TANH", [a], m3.TEMPORARY, m3.F32)
    g.node("TANH", [a], [t])
    m = g.inferred("MUL", [t, c], m3.TEMPORARY, m3.F32)
    g.node("MUL", [t, c], [m])
    y = g.inferred("ADD", [m, x], m3.OUTPUT, m3.F32)
    g.node("ADD", [m, x], [y])
    return g, x, y


def test_liveness_plan_matches_reference(m3, ref):
    g, _, _ = build_liveness_graph(m3, m3.load())
    info, report, text = m3.graph_plan(g)
    # tests/test_graph_runtime.c:118-124
    assert (info.value_count, info.node_count, info.storage_slot_count,
            info.allocated_bytes) == (6, 4, 5, 80)
    rg, _, _ = build_liveness_graph(m3, ref)
    session = m3.Session(rg, allow_metal=False, allow_neural_engine=False,
                         cuda=False)
    theirs = session.plan_info()
    assert (theirs.value_count, theirs.node_count, theirs.storage_slot_count,
            theirs.allocated_bytes) == (6, 4, 5, 80)
    # the whole chain fuses into one launch; temporaries stay in registers
    assert report.launch_count == 1 and report.fused_node_count == 4
    assert text == "ew[ADD,TANH,MUL,ADD] stores=1"


def _status(m3, fn):
    try:
        fn()
    except m3.M3Failure as failure:
        return failure.status
    return m3.OK


@pytest.mark.parametrize("which", ["cuda", "reference"])
def test_malformed_graphs_rejected_like_reference(m3, ref, which):
    lib = m3.load() if which == "cuda" else ref
    # tests/test_graph_runtime.c:162-248
    g = m3.Graph(lib=lib)
    x = g.value(m3.INPUT, m3.F32, (2,))
    t = g.value(m3.TEMPORARY, m3.F32, (2,))
    o = g.value(m3.OUTPUT, m3.F32, (2,))
    g.node("ADD", [t, x], [o])
    create = (lambda: m3.graph_plan(g)) if which == "cuda" else (
        lambda: m3.Session(g, cuda=False))
    assert _status(m3, create) == m3.INVALID_ARGUMENT      # read before produce
    assert _status(m3, lambda: g.inferred("ADD", [m3.VALUE_NONE, x],
                                          m3.TEMPORARY, m3.F32)) == m3.OUT_OF_RANGE
    assert _status(m3, lambda: g.inferred(999, [x], m3.TEMPORARY,
                                          m3.F32)) == m3.UNSUPPORTED
    g2 = m3.Graph(lib=lib)
    c = g2.value(m3.CONSTANT, m3.F32, (2,))                 # never set
    o2 = g2.value(m3.OUTPUT, m3.F32, (2,))
    g2.node("COPY", [c], [o2])
    create2 = (lambda: m3.graph_plan(g2)) if which == "cuda" else (
        lambda: m3.Session(g2, cuda=False))
    assert _status(m3, create2) == m3.INVALID_ARGUMENT
    # a second producer of one value
    g3 = m3.Graph(lib=lib)
    a = g3.value(m3.INPUT, m3.F32, (2,))
    b = g3.value(m3.OUTPUT, m3.F32, (2,))
    g3.node("COPY", [a], [b])
    g3.node("COPY", [a], [b])
    create3 = (lambda: m3.graph_plan(g3)) if which == "cuda" else (
        lambda: m3.Session(g3, cuda=False))
    assert _status(m3, create3) == m3.INVALID_ARGUMENT
    # writing an input
    g4 = m3.Graph(lib=lib)
    a = g4.value(m3.INPUT, m3.F32, (2,))
    b = g4.value(m3.INPUT, m3.F32, (2,))
    g4.node("COPY", [a], [b])
    create4 = (lambda: m3.graph_plan(g4)) if which == "cuda" else (
        lambda: m3.Session(g4, cuda=False))
    assert _status(m3, create4) == m3.INVALID_ARGUMENT


def test_validation_rejections(m3):
    # norm epsilon must be finite and > 0 (src/m3_op_validate_nn.c:141-145)
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (2, 3))
    s = g.constant(m3.F32, np.ones(3, np.float32))
    y = g.value(m3.OUTPUT, m3.F32, (2, 3))
    g.node("RMS_NORM", [x, s], [y], epsilon=0.0)
    assert _status(m3, lambda: m3.graph_plan(g)) == m3.INVALID_ARGUMENT
    # broadcast disagreement
    g = m3.Graph()
    a = g.value(m3.INPUT, m3.F32, (2, 3))
    b = g.value(m3.INPUT, m3.F32, (4,))
    y = g.value(m3.OUTPUT, m3.F32, (2, 3))
    g.node("ADD", [a, b], [y])
    assert _status(m3, lambda: m3.graph_plan(g)) == m3.INVALID_ARGUMENT
    # an operator outside the provider (no CPU fallback in this library)
    g = m3.Graph()
    a = g.value(m3.INPUT, m3.F32, (2, 3))
    b = g.value(m3.INPUT, m3.F32, (3, 4))
    y = g.value(m3.OUTPUT, m3.F32, (2, 4))
    g.node("MATMUL", [a, b], [y])
    assert _status(m3, lambda: m3.graph_plan(g)) == m3.UNSUPPORTED
    # top-k outputs must be F32 / I32
    g = m3.Graph()
    a = g.value(m3.INPUT, m3.F32, (2, 8))
    v = g.value(m3.OUTPUT, m3.F16, (2, 1))
    i = g.value(m3.OUTPUT, m3.I32, (2, 1))
    g.node("TOP_K", [a], [v, i], k=1)
    assert _status(m3, lambda: m3.graph_plan(g)) == m3.INVALID_ARGUMENT


# ------------------------------------------------- benchmark-shape plans


def config_graphs(m3, lib=None):
    """The five benchmark graphs at reduced sizes (plans are size-free)."""
    graphs = {}
    g = m3.Graph(lib=lib)
    x = g.value(m3.INPUT, m3.F32, (8, 64))
    c = g.constant(m3.F32, np.ones(64, np.float32))
    b = g.constant(m3.F32, np.zeros((1, 64), np.float32))
    t = g.inferred("MUL", [x, c], m3.TEMPORARY, m3.F32)
    g.node("MUL", [x, c], [t])
    y = g.inferred("ADD", [t, b], m3.OUTPUT, m3.F32)
    g.node("ADD", [t, b], [y])
    graphs["c1"] = g
    g = m3.Graph(lib=lib)
    x = g.value(m3.INPUT, m3.F32, (8, 64))
    p = g.inferred("SOFTMAX", [x], m3.OUTPUT, m3.F32)
    g.node("SOFTMAX", [x], [p])
    v = g.inferred("TOP_K", [x], m3.OUTPUT, m3.F32, 0, k=1)
    i = g.inferred("TOP_K", [x], m3.OUTPUT, m3.I32, 1, k=1)
    g.node("TOP_K", [x], [v, i], k=1)
    graphs["c2"] = g
    g = m3.Graph(lib=lib)
    h = g.value(m3.INPUT, m3.F16, (8, 64))
    r = g.value(m3.INPUT, m3.F16, (8, 64))
    w = g.constant(m3.F16, np.full(64, 0x3C00, np.uint16))
    gate = g.value(m3.INPUT, m3.F16, (8, 96))
    up = g.value(m3.INPUT, m3.F16, (8, 96))
    s = g.inferred("ADD", [h, r], m3.OUTPUT, m3.F16)
    g.node("ADD", [h, r], [s])
    n = g.inferred("RMS_NORM", [s, w], m3.OUTPUT, m3.F16, epsilon=1e-6)
    g.node("RMS_NORM", [s, w], [n], epsilon=1e-6)
    yv = g.inferred("GATED_SILU", [gate, up], m3.OUTPUT, m3.F16)
    g.node("GATED_SILU", [gate, up], [yv])
    graphs["c3"] = g
    g = m3.Graph(lib=lib)
    x = g.value(m3.INPUT, m3.F32, (2, 4, 8))
    vc = g.value(m3.INPUT, m3.F32, (2, 4, 8))
    vu = g.value(m3.INPUT, m3.F32, (2, 4, 8))
    k1 = g.constant(m3.F32, np.array([-1], np.float32))
    kg = g.constant(m3.F32, np.array([4], np.float32))
    kd = g.constant(m3.F32, np.array([1 / 30], np.float32))
    a = g.inferred("MUL", [vu, k1], m3.TEMPORARY, m3.F32)
    g.node("MUL", [vu, k1], [a])
    a2 = g.inferred("ADD", [vc, a], m3.TEMPORARY, m3.F32)
    g.node("ADD", [vc, a], [a2])
    a3 = g.inferred("MUL", [a2, kg], m3.TEMPORARY, m3.F32)
    g.node("MUL", [a2, kg], [a3])
    v = g.inferred("ADD", [vu, a3], m3.TEMPORARY, m3.F32)
    g.node("ADD", [vu, a3], [v])
    t = g.inferred("MUL", [v, kd], m3.TEMPORARY, m3.F32)
    g.node("MUL", [v, kd], [t])
    xn = g.inferred("ADD", [x, t], m3.OUTPUT, m3.F32)
    g.node("ADD", [x, t], [xn])
    xb = g.inferred("CAST", [xn], m3.OUTPUT, m3.BF16)
    g.node("CAST", [xn], [xb])
    graphs["c4"] = g
    g = m3.Graph(lib=lib)
    x = g.value(m3.INPUT, m3.F32, (2, 4, 16))
    al = g.constant(m3.F32, np.ones((1, 4, 1), np.float32))
    z = g.inferred("SNAKE1D", [x, al], m3.TEMPORARY, m3.F32)
    g.node("SNAKE1D", [x, al], [z])
    m = g.inferred("ABS_MAX", [z], m3.OUTPUT, m3.F32)
    g.node("ABS_MAX", [z], [m])
    y = g.inferred("CLAMP_UNIT", [z], m3.OUTPUT, m3.F32)
    g.node("CLAMP_UNIT", [z], [y])
    graphs["c5"] = g
    return graphs


def test_benchmark_graphs_fuse(m3):
    expected = {
        "c1": (1, "ew[MUL,ADD] stores=1"),
        "c2": (1, "row[SOFTMAX+TOP_K]"),
        "c3": (2, "row[ADD+RMS_NORM]; ew[GATED_SILU] stores=1"),
        "c4": (1, "ew[MUL,ADD,MUL,ADD,MUL,ADD,CAST] stores=2"),
        "c5": (1, "ew[SNAKE1D,ABS_MAX,CLAMP_UNIT] stores=2"),
    }
    for name, g in config_graphs(m3).items():
        _, report, text = m3.graph_plan(g)
        assert (report.launch_count, text) == expected[name], name
        # unfused plans: one launch per node
        _, plain, _ = m3.graph_plan(g, fuse=False)
        assert plain.launch_count >= report.launch_count


def test_data_checked_outputs_get_shadow_buffers(m3):
    graphs = config_graphs(m3)
    _, report, _ = m3.graph_plan(graphs["c2"])
    # probabilities [8,64] F32 + values [8,1] + indices [8,1], 256-B aligned
    assert report.shadow_bytes == 2048 + 256 + 256
    _, report, _ = m3.graph_plan(graphs["c1"])
    assert report.shadow_bytes == 0
    _, report, _ = m3.graph_plan(graphs["c5"])
    # abs-max (checked) and the clamp after it share the commit
    assert report.shadow_bytes == 256 + 512


def test_host_rng_matches_reference(m3, ref):
    ref.m3_rng_seed.argtypes = [ctypes.c_void_p, ctypes.c_uint64,
                                ctypes.c_uint64, ctypes.c_void_p]
    ref.m3_rng_normal_f32_fill.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_size_t, ctypes.c_void_p]
    ref.m3_rng_uniform_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p]
    state = ctypes.create_string_buffer(64)
    for seed, sequence in ((0, 0), (3, 2), (12345, 7)):
        ref.m3_rng_seed(state, seed, sequence, None)
        theirs = np.empty(1001, np.float32)
        ref.m3_rng_normal_f32_fill(state, theirs.ctypes.data, theirs.size, None)
        mine = m3.fill_normal(seed, sequence, 0.0, 1.0, 1001)
        assert np.array_equal(mine.view(np.uint32), theirs.view(np.uint32))
        ref.m3_rng_seed(state, seed, sequence, None)
        value = ctypes.c_float()
        uniform = []
        for _ in range(257):
            ref.m3_rng_uniform_f32(state, ctypes.byref(value), None)
            uniform.append(value.value)
        mine = m3.fill_uniform(seed, sequence, 0.0, 1.0, 257)
        assert np.array_equal(mine, np.array(uniform, np.float32))


def test_categorical_plans_as_checked_row_launch(m3):
    """CATEGORICAL (src/m3_op_execute_sampling.c:90-137) is a row launch whose
    I32 output is committed only by a clean run (a shadow buffer); shapes
    and dtypes follow the reference's rules."""
    g = m3.Graph()
    p = g.value(m3.INPUT, m3.F32, (4, 100))
    u = g.value(m3.INPUT, m3.F32, (4,))
    i = g.inferred("CATEGORICAL", [p, u], m3.OUTPUT, m3.I32)
    g.node("CATEGORICAL", [p, u], [i])
    info, report, text = m3.graph_plan(g)
    assert text == "row[CATEGORICAL]"
    assert report.launch_count == 1 and report.shadow_bytes == 256
    bad = m3.Graph()
    p = bad.value(m3.INPUT, m3.F32, (4, 100))
    u = bad.value(m3.INPUT, m3.F32, (5,))
    o = bad.value(m3.OUTPUT, m3.I32, (5,))
    bad.node("CATEGORICAL", [p, u], [o])
    with pytest.raises(m3.M3Failure) as failure:
        m3.graph_plan(bad)
    assert failure.value.message == "categorical dtype or shape is invalid"


def test_row_sum_plans_and_fuses_as_a_row_pass_sibling(m3):
    """ROW_SUM (extension) alone is a row launch; beside SOFTMAX and TOP_K of
    the same input the three share one row pass, and in that launch every
    output is committed per command (shadow buffers); shape and dtype rules."""
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F16, (6, 40))
    r = g.inferred("ROW_SUM", [x], m3.OUTPUT, m3.F32)
    g.node("ROW_SUM", [x], [r])
    assert g.values[r][:2] == (m3.F32, (6, 1))
    info, report, text = m3.graph_plan(g)
    assert text == "row[ROW_SUM]" and report.launch_count == 1 and report.shadow_bytes == 0
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (6, 40))
    p = g.inferred("SOFTMAX", [x], m3.OUTPUT, m3.F32)
    g.node("SOFTMAX", [x], [p])
    tv = g.inferred("TOP_K", [x], m3.OUTPUT, m3.F32, 0, k=1)
    ti = g.inferred("TOP_K", [x], m3.OUTPUT, m3.I32, 1, k=1)
    g.node("TOP_K", [x], [tv, ti], k=1)
    r = g.inferred("ROW_SUM", [x], m3.OUTPUT, m3.F32)
    g.node("ROW_SUM", [x], [r])
    info, report, text = m3.graph_plan(g)
    assert text == "row[SOFTMAX+TOP_K+ROW_SUM]"
    assert report.launch_count == 1 and report.fused_node_count == 3
    assert m3.graph_plan(g, fuse=False)[1].launch_count == 3
    for shape, dtype in (((6, 2), m3.F32), ((6, 1), m3.F16), ((1, 6), m3.F32)):
        bad = m3.Graph()
        x = bad.value(m3.INPUT, m3.F32, (6, 40))
        o = bad.value(m3.OUTPUT, dtype, shape)
        bad.node("ROW_SUM", [x], [o])
        with pytest.raises(m3.M3Failure) as failure:
            m3.graph_plan(bad)
        assert "row-sum" in failure.value.message


def test_out_of_scope_inference_is_unsupported(m3):
    """Shape inference covers the provider's operators; the reference's
    other kinds are rejected at once."""
    g = m3.Graph()
    a = g.value(m3.INPUT, m3.F32, (2, 3))
    b = g.value(m3.INPUT, m3.F32, (3, 4))
    with pytest.raises(m3.M3Failure) as failure:
        g.inferred("MATMUL", [a, b], m3.OUTPUT, m3.F32)
    assert failure.value.status == m3.UNSUPPORTED


def test_reference_rng_words_restated(oracle, ref):
    """The oracle's PCG32 word stream, which the benchmark's reference arm
    scales into uniforms, is the reference's m3_rng_u32 stream."""
    ref.m3_rng_seed.argtypes = [ctypes.c_void_p, ctypes.c_uint64,
                                ctypes.c_uint64, ctypes.c_void_p]
    ref.m3_rng_u32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    state = ctypes.create_string_buffer(64)
    for seed, sequence in ((1, 1), (4, 1), (99, 5)):
        ref.m3_rng_seed(state, seed, sequence, None)
        word = ctypes.c_uint32()
        theirs = []
        for _ in range(513):
            ref.m3_rng_u32(state, ctypes.byref(word), None)
            theirs.append(word.value)
        assert np.array_equal(oracle.pcg32_words(seed, sequence, 513),
                              np.array(theirs, np.uint32))
