"""Golden cases: small graphs of every reference operator on the path (and
categorical sampling), with
seeded inputs (test infrastructure).

Each case is (builder, inputs, checks): `builder(m3, g)` adds the graph to
`g` and returns ({input name: value id}, [output value ids]); `inputs(m3,
oracle)` returns the input arrays; `checks` gives, per output, the parity
bar the GPU path must meet against the reference's output:

  "bits"   bit-exact (integer/index work, F32 add/mul/cast, ordered sums)
  "ulp1"   within one unit in the last place of the output dtype
  "rel6"   within 1e-6 relative (F32 reductions through expf)
  "sin"    within 0x1p-19 absolute-or-relative (sinf/tanhf)
  "rel20"  within 2^-20 relative (F32 gated SiLU through expf)

make_golden.py runs the cases through the reference's CPU provider
(oracle/_ref/libm3ref.so, compiled from the reference sources) and stores
inputs and outputs in golden.npz.
"""

from __future__ import annotations

import numpy as np


def _enc(oracle, dtype_name, values):
    return {"F32": lambda v: v.astype(np.float32), "F16": oracle.to_f16,
            "BF16": oracle.to_bf16}[dtype_name](values)


def broadcast_mul_add(dt):
    """C1 pattern: y = (x * c) + b with a [W] and a [1, W] broadcast."""
    shape, w = (16, 96), 96

    def build(m3, g):
        d = getattr(m3, dt)
        x = g.value(m3.INPUT, d, shape)
        c = g.value(m3.INPUT, d, (w,))
        b = g.value(m3.INPUT, d, (1, w))
        t = g.inferred("MUL", [x, c], m3.TEMPORARY, d)
        g.node("MUL", [x, c], [t])
        y = g.inferred("ADD", [t, b], m3.OUTPUT, d)
        g.node("ADD", [t, b], [y])
        return {"x": x, "c": c, "b": b}, [y]

    def inputs(m3, oracle):
        r = np.random.default_rng(100)
        return {"x": _enc(oracle, dt, r.uniform(-1, 1, shape)),
                "c": _enc(oracle, dt, r.uniform(0.5, 2, (w,))),
                "b": _enc(oracle, dt, r.standard_normal((1, w)))}
    return build, inputs, ["bits"]


def softmax_top1(dt):
    """C2 pattern with special rows: all -inf, +inf ties, +20 spikes."""
    rows, w = 12, 200

    def build(m3, g):
        d = getattr(m3, dt)
        x = g.value(m3.INPUT, d, (rows, w))
        p = g.inferred("SOFTMAX", [x], m3.OUTPUT, d)
        g.node("SOFTMAX", [x], [p])
        v = g.inferred("TOP_K", [x], m3.OUTPUT, m3.F32, k=1)
        i = g.inferred("TOP_K", [x], m3.OUTPUT, m3.I32, output_index=1, k=1)
        g.node("TOP_K", [x], [v, i], k=1)
        return {"x": x}, [p, v, i]

    def inputs(m3, oracle):
        r = np.random.default_rng(101)
        x = (r.standard_normal((rows, w)) * 3).astype(np.float32)
        x[r.random((rows, w)) < 0.01] = 20.0
        x[2] = -np.inf
        x[3, 5] = np.inf
        x[3, 77] = np.inf
        x[4, 9] = -0.0
        x[5] = 7.0
        return {"x": _enc(oracle, dt, x)}
    return build, inputs, ["rel6" if dt == "F32" else "ulp1", "bits", "bits"]


def residual_rms_norm(dt):
    """C3 pattern: s = h + r (an output), n = RMSNorm(s, w)."""
    rows, w = 8, 256

    def build(m3, g):
        d = getattr(m3, dt)
        h = g.value(m3.INPUT, d, (rows, w))
        rr = g.value(m3.INPUT, d, (rows, w))
        sc = g.value(m3.INPUT, d, (w,))
        s = g.inferred("ADD", [h, rr], m3.OUTPUT, d)
        g.node("ADD", [h, rr], [s])
        n = g.inferred("RMS_NORM", [s, sc], m3.OUTPUT, d, epsilon=1e-6)
        g.node("RMS_NORM", [s, sc], [n], epsilon=1e-6)
        return {"h": h, "r": rr, "w": sc}, [s, n]

    def inputs(m3, oracle):
        r = np.random.default_rng(102)
        return {"h": _enc(oracle, dt, r.standard_normal((rows, w))),
                "r": _enc(oracle, dt, r.standard_normal((rows, w))),
                "w": _enc(oracle, dt, 1 + 0.05 * r.standard_normal(w))}
    return build, inputs, ["bits", "bits"]


def layer_norm(dt):
    rows, w = 6, 160

    def build(m3, g):
        d = getattr(m3, dt)
        x = g.value(m3.INPUT, d, (rows, w))
        sc = g.value(m3.INPUT, d, (w,))
        bi = g.value(m3.INPUT, d, (w,))
        y = g.inferred("LAYER_NORM", [x, sc, bi], m3.OUTPUT, d, epsilon=1e-5)
        g.node("LAYER_NORM", [x, sc, bi], [y], epsilon=1e-5)
        return {"x": x, "w": sc, "b": bi}, [y]

    def inputs(m3, oracle):
        r = np.random.default_rng(103)
        return {"x": _enc(oracle, dt, 2 + r.standard_normal((rows, w))),
                "w": _enc(oracle, dt, r.uniform(0.5, 1.5, w)),
                "b": _enc(oracle, dt, r.standard_normal(w))}
    return build, inputs, ["bits"]


def gated_silu(dt):
    shape = (8, 300)

    def build(m3, g):
        d = getattr(m3, dt)
        a = g.value(m3.INPUT, d, shape)
        b = g.value(m3.INPUT, d, shape)
        y = g.inferred("GATED_SILU", [a, b], m3.OUTPUT, d)
        g.node("GATED_SILU", [a, b], [y])
        return {"gate": a, "up": b}, [y]

    def inputs(m3, oracle):
        r = np.random.default_rng(104)
        return {"gate": _enc(oracle, dt, 4 * r.standard_normal(shape)),
                "up": _enc(oracle, dt, r.standard_normal(shape))}
    return build, inputs, ["rel20" if dt == "F32" else "ulp1"]


def cfg_euler_bf16():
    """C4 pattern, one Euler step: x' = x + dt * (vu + 4 (vc - vu)), BF16 cast."""
    shape = (2, 4, 64)

    def build(m3, g):
        x = g.value(m3.INPUT, m3.F32, shape)
        vc = g.value(m3.INPUT, m3.F32, shape)
        vu = g.value(m3.INPUT, m3.F32, shape)
        k1 = g.constant(m3.F32, np.array([-1.0], np.float32))
        kg = g.constant(m3.F32, np.array([4.0], np.float32))
        kd = g.constant(m3.F32, np.array([np.float32(1.0) / np.float32(30.0)], np.float32))
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
        return {"x": x, "vc": vc, "vu": vu}, [xn, xb]

    def inputs(m3, oracle):
        r = np.random.default_rng(105)
        return {k: r.standard_normal(shape).astype(np.float32) for k in ("x", "vc", "vu")}
    return build, inputs, ["bits", "bits"]


def snake_tanh():
    """C5 activation: z = snake(x, alpha) per channel, then tanh(z)."""
    shape = (2, 16, 64)

    def build(m3, g):
        x = g.value(m3.INPUT, m3.F32, shape)
        al = g.value(m3.INPUT, m3.F32, (1, 16, 1))
        z = g.inferred("SNAKE1D", [x, al], m3.OUTPUT, m3.F32)
        g.node("SNAKE1D", [x, al], [z])
        y = g.inferred("TANH", [z], m3.OUTPUT, m3.F32)
        g.node("TANH", [z], [y])
        return {"x": x, "alpha": al}, [z, y]

    def inputs(m3, oracle):
        r = np.random.default_rng(106)
        return {"x": (0.5 * r.standard_normal(shape)).astype(np.float32),
                "alpha": r.uniform(0.2, 2, (1, 16, 1)).astype(np.float32)}
    return build, inputs, ["sin", "sin"]


def casts():
    """F32 -> F16 / BF16 / I32 and back, with halfway, subnormal and
    overflow values."""
    n = 64

    def build(m3, g):
        x = g.value(m3.INPUT, m3.F32, (n,))
        outs = []
        for d in (m3.F16, m3.BF16, m3.I32):
            y = g.inferred("CAST", [x], m3.OUTPUT, d)
            g.node("CAST", [x], [y])
            outs.append(y)
        back = g.inferred("CAST", [outs[0]], m3.OUTPUT, m3.F32)
        g.node("CAST", [outs[0]], [back])
        return {"x": x}, outs + [back]

    def inputs(m3, oracle):
        r = np.random.default_rng(107)
        x = (r.standard_normal(n) * 1000).astype(np.float32)
        x[:8] = np.array([1 + 2 ** -11, 1 + 3 * 2 ** -11, 2 ** -25, 2 ** -24 * 1.5,
                          65504, 65520, -0.0, 1e-30], np.float32)
        return {"x": x}
    return build, inputs, ["bits", "bits", "bits", "bits"]


def categorical(dt):
    """Categorical sampling: rows with zeros, a single positive entry, a zero
    uniform and the largest uniform below one."""
    rows, vocab = 12, 257

    def build(m3, g):
        d = getattr(m3, dt)
        p = g.value(m3.INPUT, d, (rows, vocab))
        u = g.value(m3.INPUT, d, (rows,))
        i = g.inferred("CATEGORICAL", [p, u], m3.OUTPUT, m3.I32)
        g.node("CATEGORICAL", [p, u], [i])
        return {"p": p, "u": u}, [i]

    def inputs(m3, oracle):
        r = np.random.default_rng(108)
        p = r.random((rows, vocab)).astype(np.float32)
        p[r.random((rows, vocab)) < 0.4] = 0.0
        p[3] = 0.0
        p[3, 100] = 0.5
        u = r.random(rows).astype(np.float32)
        u[0] = 0.0
        u[1] = np.nextafter(np.float32(1.0), np.float32(0.0)) if dt == "F32" else np.float32(0.99609375)
        return {"p": _enc(oracle, dt, p), "u": _enc(oracle, dt, u)}
    return build, inputs, ["bits"]


CASES = {
    "broadcast_mul_add_f32": broadcast_mul_add("F32"),
    "broadcast_mul_add_f16": broadcast_mul_add("F16"),
    "broadcast_mul_add_bf16": broadcast_mul_add("BF16"),
    "softmax_top1_f32": softmax_top1("F32"),
    "softmax_top1_f16": softmax_top1("F16"),
    "residual_rms_norm_f16": residual_rms_norm("F16"),
    "residual_rms_norm_bf16": residual_rms_norm("BF16"),
    "residual_rms_norm_f32": residual_rms_norm("F32"),
    "layer_norm_f32": layer_norm("F32"),
    "layer_norm_f16": layer_norm("F16"),
    "gated_silu_f16": gated_silu("F16"),
    "gated_silu_bf16": gated_silu("BF16"),
    "gated_silu_f32": gated_silu("F32"),
    "cfg_euler_bf16": cfg_euler_bf16(),
    "snake_tanh": snake_tanh(),
    "casts": casts(),
    "categorical_f32": categorical("F32"),
    "categorical_f16": categorical("F16"),
}
