"""Benchmark of the CUDA provider on BASELINE.json's configurations.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5]
    python bench.py --impl reference ...      # the reference CPU provider

Headline workload (`--config`, default c5): BASELINE.json's largest
configuration, the vocoder activation on stereo F32 [2,512,1572864] (snake,
global abs-max, clamp), 12.9 GB per run.  Every other configuration (c1-c4)
is measured the same way in the same run and reported under `per_config`,
each with its own value, roofline, CPU baseline and end-to-end figure.  At
N=1, `per_config` also holds C1 and C2 through the reference-facing backend
plug-in (`c1_plugin`, `c2_plugin`: m3_cuda_backend_execute on the command
lists the reference's scheduler issues).

One step = one session run over one batch (C4: its 30 carried Euler runs).
With N ranks (torchrun, one process per GPU) every configuration's FIXED
tensor is split N ways by the library's sharding layer
(m3_cuda_shard_session_create): rows for C1-C3, the time axis for C4 and C5,
one arena per GPU, constants replicated; C5's global abs-max is one NCCL
all-reduce issued by the library on the session's stream.  Scaling is
"strong": `value` = the whole tensor's algorithmic bytes / the slowest
rank's step time.

Metric: achieved HBM GB/s = algorithmic bytes (each input read once, each
graph output written once) / device time, inputs resident in HBM, L2 evicted
between timed steps.  `e2e` is the same metric through the public C API with
pinned host buffers: every step uploads its inputs and downloads its outputs
inside the timed region.

The reference arm (--impl reference) runs the reference's own CPU provider
(oracle/_ref/libm3ref.so, compiled from the reference sources) on all host
threads over bounded samples of the same workloads.  Its inputs come from the
reference's RNG (m3_rng_normal_f32_fill) and the restated PCG32 word stream of
oracle/; the product library is never loaded in that process.
"""

from __future__ import annotations

import argparse
import ctypes
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))


def _module(name: str, path: str):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


def m3mod():
    """The ctypes binding (m3.c_b200/m3cuda.py).  Importing it loads nothing;
    only `load()` maps libm3cuda.so."""
    return _module("m3cuda", os.path.join(ROOT, "m3.c_b200", "m3cuda.py"))


def oraclemod():
    return _module("m3_oracle_py", os.path.join(ROOT, "oracle", "oracle.py"))


def shardsmod():
    return _module("m3_shards", os.path.join(ROOT, "m3.c_b200", "shards.py"))


METRIC = ("achieved HBM GB/s (fraction of B200 peak) per op; "
          "elems/s at 1/2/4/8 GPUs vs CPU")
L2_NOTE = "256 MiB buffer written, then another 256 MiB read, between timed steps"
REFERENCE_C5_NOTE = ("; SNAKE1D by the reference's CPU provider, then the abs-max and the "
                     "waveform clamp loop (no reference operators) by the oracle's C "
                     "restatements on the host")

F32, F16, BF16 = 0, 1, 2


# ----------------------------------------------------------------- RNGs

class ProductRng:
    """Seeded inputs from libm3cuda.so's restatement of the reference RNG."""

    def __init__(self, m3):
        self.m3 = m3

    def uniform(self, seed, sequence, low, high, count):
        return self.m3.fill_uniform(seed, sequence, low, high, count)

    def normal(self, seed, sequence, mean, deviation, count):
        return self.m3.fill_normal(seed, sequence, mean, deviation, count)


class _RefRng(ctypes.Structure):
    # src/m3_rng.h:10-15
    _fields_ = [("state", ctypes.c_uint64), ("increment", ctypes.c_uint64),
                ("spare_normal", ctypes.c_float), ("has_spare_normal", ctypes.c_bool)]


class ReferenceRng:
    """Seeded inputs from the reference itself: m3_rng_seed and
    m3_rng_normal_f32_fill of libm3ref.so (src/m3_rng.c:22-110) for normals,
    the restated PCG32 word stream (oracle/, pinned against m3_rng_u32) for
    uniforms.  mean + deviation * z and low + (high - low) * u are separate
    F32 statements, as in the product's fills."""

    def __init__(self, reference_lib, oracle):
        self.lib = reference_lib
        self.oracle = oracle

    def uniform(self, seed, sequence, low, high, count):
        return self.oracle.uniform(seed, sequence, low, high, count)

    def normal(self, seed, sequence, mean, deviation, count):
        rng = _RefRng()
        err = (ctypes.c_char * 264)()
        out = np.empty(count, dtype=np.float32)
        if self.lib.m3_rng_seed(ctypes.byref(rng), ctypes.c_uint64(seed),
                                ctypes.c_uint64(sequence), err) != 0:
            raise RuntimeError("m3_rng_seed failed")
        if self.lib.m3_rng_normal_f32_fill(ctypes.byref(rng), out.ctypes.data_as(ctypes.c_void_p),
                                           ctypes.c_size_t(count), err) != 0:
            raise RuntimeError("m3_rng_normal_f32_fill failed")
        scaled = (np.float32(deviation) * out).astype(np.float32)
        return (np.float32(mean) + scaled).astype(np.float32)


# ---------------------------------------------------------------- configs

class Config:
    """One benchmark graph: builder, seeded inputs, algorithmic bytes.

    `scale` shrinks the configuration along its shard axis (rows, or time
    for C4/C5): CPU samples and profiling cases use it; reported GPU
    numbers use 1.0."""

    name = ""
    workload = ""
    dtype = "f32"
    runs_per_step = 1
    shard_axis = 0
    shard_axis_name = "rows"

    def build(self, m3, g, rng, scale: float = 1.0):  # -> ({name: vid}, [vid])
        raise NotImplementedError

    def inputs_host(self, rng, scale: float = 1.0):  # -> {name: ndarray}
        raise NotImplementedError

    def algorithmic_bytes(self, scale: float = 1.0) -> int:
        raise NotImplementedError

    def elements(self, scale: float = 1.0) -> int:
        raise NotImplementedError


def _rows(full, scale):
    return max(1, int(round(full * scale)))


def _length(full, scale):
    return max(4, int(full * scale) // 4 * 4)


class C1(Config):
    name = "c1"
    workload = "y = (x * c) + b F32 [1024,4096], c [4096] / b [1,4096] constants, seed 0"
    rows, width = 1024, 4096

    def shape(self, scale=1.0):
        return (_rows(self.rows, scale), self.width)

    def build(self, m3, g, rng, scale=1.0):
        c = rng.uniform(0, 1, 0.5, 2.0, self.width)
        b = rng.normal(0, 2, 0.0, 1.0, self.width).reshape(1, self.width)
        x = g.value(m3.INPUT, m3.F32, self.shape(scale))
        vc = g.constant(m3.F32, c)
        vb = g.constant(m3.F32, b)
        t = g.inferred("MUL", [x, vc], m3.TEMPORARY, m3.F32)
        g.node("MUL", [x, vc], [t])
        y = g.inferred("ADD", [t, vb], m3.OUTPUT, m3.F32)
        g.node("ADD", [t, vb], [y])
        return {"x": x}, [y]

    def inputs_host(self, rng, scale=1.0):
        shape = self.shape(scale)
        return {"x": rng.uniform(0, 0, -1.0, 1.0, shape[0] * shape[1]).reshape(shape)}

    def inputs_device(self, m3, torch, device, scale=1.0):
        shape = self.shape(scale)
        x = torch.empty(shape[0] * shape[1], dtype=torch.float32, device=device)
        fill(m3, "uniform", 0, 0, -1.0, 1.0, x, torch.cuda.current_stream(device).cuda_stream)
        return {"x": x.view(shape)}

    def algorithmic_bytes(self, scale=1.0):
        rows = self.shape(scale)[0]
        return rows * self.width * 8 + 2 * self.width * 4

    def elements(self, scale=1.0):
        return self.shape(scale)[0] * self.width


class C2(Config):
    name = "c2"
    workload = ("softmax + row max/argmax (TOP_K k=1) F32 [32768,1024], "
                "N(0,3^2) logits with 1% = +20, seed 1")
    rows, width = 32768, 1024

    def shape(self, scale=1.0):
        return (_rows(self.rows, scale), self.width)

    def build(self, m3, g, rng, scale=1.0):
        x = g.value(m3.INPUT, m3.F32, self.shape(scale))
        p = g.inferred("SOFTMAX", [x], m3.OUTPUT, m3.F32)
        g.node("SOFTMAX", [x], [p])
        v = g.inferred("TOP_K", [x], m3.OUTPUT, m3.F32, 0, k=1)
        i = g.inferred("TOP_K", [x], m3.OUTPUT, m3.I32, 1, k=1)
        g.node("TOP_K", [x], [v, i], k=1)
        return {"x": x}, [p, v, i]

    def inputs_host(self, rng, scale=1.0):
        shape = self.shape(scale)
        n = shape[0] * shape[1]
        x = rng.normal(1, 0, 0.0, 3.0, n)
        x[rng.uniform(1, 1, 0.0, 1.0, n) < 0.01] = 20.0
        return {"x": x.reshape(shape)}

    def inputs_device(self, m3, torch, device, scale=1.0):
        shape = self.shape(scale)
        n = shape[0] * shape[1]
        x = torch.empty(n, dtype=torch.float32, device=device)
        u = torch.empty(n, dtype=torch.float32, device=device)
        stream = torch.cuda.current_stream(device).cuda_stream
        fill(m3, "normal", 1, 0, 0.0, 3.0, x, stream)
        fill(m3, "uniform", 1, 1, 0.0, 1.0, u, stream)
        x[u < 0.01] = 20.0
        return {"x": x.view(shape)}

    def algorithmic_bytes(self, scale=1.0):
        rows, width = self.shape(scale)
        return rows * width * 4 * 2 + rows * 4 * 2

    def elements(self, scale=1.0):
        rows, width = self.shape(scale)
        return rows * width


class C3(Config):
    name = "c3"
    dtype = "f16"
    workload = ("F16 residual add + RMSNorm [8192,2048] (eps 1e-6, w N(1,0.05)) "
                "and SiLU(gate)*up [8192,5632], seed 2")
    rows, width, ffn = 8192, 2048, 5632

    def _sizes(self, scale):
        rows = _rows(self.rows, scale)
        return {"h": (rows, self.width, 0), "r": (rows, self.width, 1),
                "gate": (rows, self.ffn, 3), "up": (rows, self.ffn, 4)}

    def build(self, m3, g, rng, scale=1.0):
        rows = _rows(self.rows, scale)
        w = f16_bits(rng.normal(2, 2, 1.0, 0.05, self.width))
        h = g.value(m3.INPUT, m3.F16, (rows, self.width))
        r = g.value(m3.INPUT, m3.F16, (rows, self.width))
        vw = g.constant(m3.F16, w)
        gate = g.value(m3.INPUT, m3.F16, (rows, self.ffn))
        up = g.value(m3.INPUT, m3.F16, (rows, self.ffn))
        s = g.inferred("ADD", [h, r], m3.OUTPUT, m3.F16)
        g.node("ADD", [h, r], [s])
        n = g.inferred("RMS_NORM", [s, vw], m3.OUTPUT, m3.F16, epsilon=1e-6)
        g.node("RMS_NORM", [s, vw], [n], epsilon=1e-6)
        y = g.inferred("GATED_SILU", [gate, up], m3.OUTPUT, m3.F16)
        g.node("GATED_SILU", [gate, up], [y])
        return {"h": h, "r": r, "gate": gate, "up": up}, [s, n, y]

    def inputs_host(self, rng, scale=1.0):
        out = {}
        for name, (rows, cols, seq) in self._sizes(scale).items():
            out[name] = f16_bits(rng.normal(2, seq, 0.0, 1.0, rows * cols)).reshape(rows, cols)
        return out

    def inputs_device(self, m3, torch, device, scale=1.0):
        out = {}
        stream = torch.cuda.current_stream(device).cuda_stream
        for name, (rows, cols, seq) in self._sizes(scale).items():
            tmp = torch.empty(rows * cols, dtype=torch.float32, device=device)
            fill(m3, "normal", 2, seq, 0.0, 1.0, tmp, stream)
            out[name] = device_cast_f16(m3, tmp, device).view(rows, cols)
            del tmp
        return out

    def algorithmic_bytes(self, scale=1.0):
        rows = _rows(self.rows, scale)
        return rows * self.width * 2 * 4 + self.width * 2 + rows * self.ffn * 2 * 3

    def elements(self, scale=1.0):
        return _rows(self.rows, scale) * (self.width + self.ffn)


class C4(Config):
    name = "c4"
    workload = ("flow-matching CFG + Euler step, F32 [2,64,8192], g = 4, dt = 1/30, "
                "then BF16 cast; 30 steps carried on device; seed 3")
    batch, channels, length = 2, 64, 8192
    runs_per_step = 30
    shard_axis = 2
    shard_axis_name = "time"

    def shape(self, scale=1.0):
        return (self.batch, self.channels, _length(self.length, scale))

    def build(self, m3, g, rng, scale=1.0):
        shape = self.shape(scale)
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
        self.carry = (x, xn)
        return {"x": x, "vc": vc, "vu": vu}, [xn, xb]

    def inputs_host(self, rng, scale=1.0):
        shape = self.shape(scale)
        n = int(np.prod(shape))
        return {name: rng.normal(3, seq, 0.0, 1.0, n).reshape(shape)
                for seq, name in enumerate(("x", "vc", "vu"))}

    def inputs_device(self, m3, torch, device, scale=1.0):
        shape = self.shape(scale)
        n = int(np.prod(shape))
        stream = torch.cuda.current_stream(device).cuda_stream
        out = {}
        for seq, name in enumerate(("x", "vc", "vu")):
            t = torch.empty(n, dtype=torch.float32, device=device)
            fill(m3, "normal", 3, seq, 0.0, 1.0, t, stream)
            out[name] = t.view(shape)
        return out

    def algorithmic_bytes(self, scale=1.0):
        n = int(np.prod(self.shape(scale)))
        return 30 * (n * 4 * 3 + n * 4 + n * 2)

    def elements(self, scale=1.0):
        return 30 * int(np.prod(self.shape(scale)))


class C5(Config):
    name = "c5"
    workload = ("snake x + sin^2(a x)/a on stereo F32 [2,512,1572864], a U[0.2,2], "
                "x N(0,0.5); global abs-max and clamp to [-1,1]; seed 4")
    batch, channels, length = 2, 512, 1572864
    shard_axis = 2
    shard_axis_name = "time"

    def shape(self, scale=1.0):
        return (self.batch, self.channels, _length(self.length, scale))

    def build(self, m3, g, rng, scale=1.0):
        alpha = rng.uniform(4, 1, 0.2, 2.0, self.channels).reshape(1, self.channels, 1)
        x = g.value(m3.INPUT, m3.F32, self.shape(scale))
        va = g.constant(m3.F32, alpha)
        z = g.inferred("SNAKE1D", [x, va], m3.TEMPORARY, m3.F32)
        g.node("SNAKE1D", [x, va], [z])
        m = g.inferred("ABS_MAX", [z], m3.OUTPUT, m3.F32)
        g.node("ABS_MAX", [z], [m])
        y = g.inferred("CLAMP_UNIT", [z], m3.OUTPUT, m3.F32)
        g.node("CLAMP_UNIT", [z], [y])
        return {"x": x}, [m, y]

    def inputs_host(self, rng, scale=1.0):
        shape = self.shape(scale)
        return {"x": rng.normal(4, 0, 0.0, 0.5, int(np.prod(shape))).reshape(shape)}

    def reference_build(self, m3, g, rng, scale=1.0):
        """The reference has SNAKE1D but no abs-max or clamp operator (its
        waveform assembly clamps in a host loop, src/m3_waveform.c:360-380):
        its graph stops at z, and the CPU leg finishes each run with the
        oracle's restatements of the abs-max and of that clamp loop."""
        alpha = rng.uniform(4, 1, 0.2, 2.0, self.channels).reshape(1, self.channels, 1)
        x = g.value(m3.INPUT, m3.F32, self.shape(scale))
        va = g.constant(m3.F32, alpha)
        z = g.inferred("SNAKE1D", [x, va], m3.OUTPUT, m3.F32)
        g.node("SNAKE1D", [x, va], [z])
        return {"x": x}, [z]

    def reference_finish(self, oracle):
        """Host work after each reference run: abs-max and clamp of z."""
        def finish(session, outputs, buffers):
            z = session.read(outputs[0], out=buffers.setdefault(
                "z", np.empty(session.values[outputs[0]][1], np.float32)))
            y = buffers.setdefault("y", np.empty_like(z))
            m = buffers.setdefault("m", np.zeros(1, np.float32))
            assert oracle.run("abs_max", z, m) == 0
            assert oracle.run("clamp_unit", z, y) == 0
        return finish

    def inputs_device(self, m3, torch, device, scale=1.0):
        shape = self.shape(scale)
        x = torch.empty(int(np.prod(shape)), dtype=torch.float32, device=device)
        fill(m3, "normal", 4, 0, 0.0, 0.5, x, torch.cuda.current_stream(device).cuda_stream)
        return {"x": x.view(shape)}

    def algorithmic_bytes(self, scale=1.0):
        n = int(np.prod(self.shape(scale)))
        return n * 8 + self.channels * 4 + 4

    def elements(self, scale=1.0):
        return int(np.prod(self.shape(scale)))


CONFIGS = {c.name: c for c in (C1(), C2(), C3(), C4(), C5())}


def config_dict(cfg, world: int) -> dict:
    """The `config` object of both arms' JSON lines (identical by design)."""
    return {"workload": cfg.workload, "name": cfg.name, "scale": 1.0,
            "shards": world, "shard_axis": cfg.shard_axis_name,
            "split": "one fixed tensor split across the ranks (strong scaling)",
            "l2": L2_NOTE,
            "parallelism": ("one GPU" if world == 1 else
                            f"{world}-way {cfg.shard_axis_name} shards" +
                            (", NCCL all-reduce(max) of the abs-max" if cfg.name == "c5" else
                             ", no data-path collective"))}


# ------------------------------------------------------------- helpers

def f16_bits(values: np.ndarray) -> np.ndarray:
    """F32 -> F16 bits with the reference's RN-even encoder (exact integer
    restatement; vectorised in numpy for input preparation)."""
    b = np.ascontiguousarray(values, np.float32).view(np.uint32).astype(np.uint64)
    sign = ((b >> 16) & 0x8000).astype(np.uint64)
    exp = ((b >> 23) & 0xFF).astype(np.int64)
    frac = (b & 0x7FFFFF).astype(np.uint64)
    e = exp - 127
    out = np.zeros(b.shape, np.uint64)
    normal = (e >= -14) & (e <= 15)
    half = ((np.clip(e + 15, 0, 31).astype(np.uint64)) << 10) | (frac >> 13)
    rest = frac & 0x1FFF
    up = (rest > 0x1000) | ((rest == 0x1000) & ((half & 1) == 1))
    half = half + up.astype(np.uint64)
    half = np.where(half >= 0x7C00, 0x7C00, half)
    out = np.where(normal, half, out)
    sub = (e >= -25) & (e < -14)
    shift = np.clip(-e - 1, 1, 63).astype(np.uint64)
    sig = 0x800000 | frac
    kept = sig >> shift
    remainder = sig & ((np.uint64(1) << shift) - 1)
    halfway = np.uint64(1) << (shift - 1)
    kept = kept + ((remainder > halfway) | ((remainder == halfway) & ((kept & 1) == 1))).astype(np.uint64)
    out = np.where(sub, kept, out)
    out = np.where(e > 15, 0x7C00, out)
    nan = (exp == 0xFF) & (frac != 0)
    payload = frac >> 13
    out = np.where(nan, 0x7E00 | payload | (payload == 0).astype(np.uint64), out)
    out = np.where((exp == 0xFF) & (frac == 0), 0x7C00, out)
    return (out | sign).astype(np.uint16)


def fill(m3, kind, seed, sequence, a, b, tensor, stream):
    """Device fill from the restated reference RNG (the configuration's own
    streams: every rank generates the same global tensor)."""
    lib = m3.load()
    err = m3.M3Error()
    fn = lib.m3_cuda_fill_normal_device if kind == "normal" else lib.m3_cuda_fill_uniform_device
    m3.check(fn(seed, sequence, a, b, ctypes.c_void_p(tensor.data_ptr()), tensor.numel(),
                ctypes.c_void_p(stream), ctypes.byref(err)), err)


def device_cast_f16(m3, tensor, device):
    """F32 -> F16 on the device with the library's CAST (reference codec)."""
    import torch
    n = tensor.numel()
    g = m3.Graph()
    x = g.value(m3.INPUT, m3.F32, (n,))
    y = g.inferred("CAST", [x], m3.OUTPUT, m3.F16)
    g.node("CAST", [x], [y])
    s = m3.Session(g, device=device.index,
                   stream=torch.cuda.current_stream(device).cuda_stream)
    s.write_device(x, tensor.data_ptr(), n * 4)
    s.run()
    out = torch.empty(n, dtype=torch.int16, device=device)
    s.read_device(y, out.data_ptr(), n * 2)
    s.close()
    return out


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        data = json.load(open(path))
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic(config_name: str):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu
    summary (profiles/ncu_traffic.json): cold-cache figures of one captured
    launch, scaled to a full launch where the capture ran a scaled case."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(path):
        return None
    data = json.load(open(path))
    entry = data.get(config_name)
    return None if entry is None else entry.get("dram_bytes_per_launch")


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.index = device_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[4:8]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------- reference timing

class ReferenceRunner:
    """One reference CPU-only session over a slice of a configuration, and
    the host work the reference does after each run (C5's abs-max/clamp)."""

    def __init__(self, m3, lib, rng, config, scale, oracle):
        g = m3.Graph(lib=lib)
        build = getattr(config, "reference_build", config.build)
        handles, self.outputs = build(m3, g, rng, scale)
        self.session = m3.Session(g, allow_metal=False, allow_neural_engine=False, cuda=False)
        data = config.inputs_host(rng, scale)
        for name, vid in handles.items():
            self.session.write(vid, data[name])
        finish = getattr(config, "reference_finish", None)
        self.finish = finish(oracle) if finish is not None else None
        self.buffers = {}

    def run(self):
        self.session.run()
        if self.finish is not None:
            self.finish(self.session, self.outputs, self.buffers)

    def close(self):
        self.session.close()


def reference_sessions(m3, lib, rng, config, scale, threads):
    """`threads` reference CPU-only sessions, each over its own 1/threads
    slice of the scaled workload along the configuration's shard axis (the
    data of every slice is the configuration's seeded stream)."""
    oracle = oraclemod()
    return [ReferenceRunner(m3, lib, rng, config, scale / threads, oracle)
            for _ in range(threads)]


def time_reference(sessions, runs):
    """Seconds for every session to make `runs` runs, one thread per session
    (ctypes releases the GIL during each run)."""
    def work(s):
        for _ in range(runs):
            s.run()

    workers = [threading.Thread(target=work, args=(s,)) for s in sessions]
    start = time.perf_counter()
    for w in workers:
        w.start()
    for w in workers:
        w.join()
    return time.perf_counter() - start


def reference_scale(m3, lib, rng, config, threads, seconds):
    """Sample scale whose one step takes about `seconds` on `threads`
    threads (from a 1/64 probe on one thread)."""
    probe = 1.0 / 64
    sessions = reference_sessions(m3, lib, rng, config, probe, 1)
    time_reference(sessions, 1)
    t = time_reference(sessions, config.runs_per_step)
    for s in sessions:
        s.close()
    scale = probe * seconds * threads / max(t, 1e-6)
    return float(min(1.0, max(probe, scale)))


def cpu_baseline(m3, oracle, config, budget_seconds):
    """Single-core reference CPU provider on a bounded sample (rank 0, N=1)."""
    if not oracle.reference_available():
        return None
    lib = m3.bind(oracle.reference(), cuda=False)
    rng = ReferenceRng(lib, oracle)
    scale = reference_scale(m3, lib, rng, config, 1, budget_seconds / 3)
    sessions = reference_sessions(m3, lib, rng, config, scale, 1)
    time_reference(sessions, 1)
    times = [time_reference(sessions, config.runs_per_step) for _ in range(3)]
    for s in sessions:
        s.close()
    sec = statistics.median(times)
    return {"value": config.algorithmic_bytes(scale) / sec / 1e9, "unit": "GB/s",
            "cores": 1, "kind": "reference",
            "sample": f"{config.name} at {scale:.4g} of full size along its "
                      f"{config.shard_axis_name} axis (median of 3 steps, {sec:.2f} s each), "
                      "reference CPU-only m3_session_run, 1 thread" +
                      (REFERENCE_C5_NOTE if config.name == "c5" else ""),
            "elems_per_s": config.elements(scale) / sec}


def run_reference_arm(args, headline):
    """The reference's CPU provider, all host threads, bounded samples of
    every configuration: one JSON line (rank 0 only)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    m3 = m3mod()
    oracle = oraclemod()
    if not oracle.reference_available():
        print(json.dumps({"impl": "reference",
                          "unavailable": "reference CPU library oracle/_ref/libm3ref.so not built"}))
        return 0
    lib = m3.bind(oracle.reference(), cuda=False)
    rng = ReferenceRng(lib, oracle)
    threads = max(1, os.cpu_count() or 1)
    world = args.gpus

    def measure(config, seconds):
        scale = reference_scale(m3, lib, rng, config, threads, seconds)
        sessions = reference_sessions(m3, lib, rng, config, scale, threads)
        for _ in range(args.warmup):
            time_reference(sessions, config.runs_per_step)
        times = [time_reference(sessions, config.runs_per_step) for _ in range(args.steps)]
        for s in sessions:
            s.close()
        sec = statistics.mean(times)
        value = config.algorithmic_bytes(scale) / sec / 1e9
        sample = (f"{config.name} at {scale:.4g} of full size along its {config.shard_axis_name} "
                  f"axis per step, split into {threads} slices run by {threads} threads, each its "
                  "own reference CPU-only session (libm3ref.so; inputs from the reference RNG)" +
                  (REFERENCE_C5_NOTE if config.name == "c5" else ""))
        return value, sec, scale, sample

    value, sec, scale, sample = measure(headline, args.ref_seconds)
    per_config = {}
    if not args.no_per_config:
        for name, config in CONFIGS.items():
            if name == headline.name:
                continue
            v, s, sc, smp = measure(config, args.ref_seconds / 3)
            per_config[name] = {"workload": config.workload, "value": v, "unit": "GB/s",
                                "ms_per_step": s * 1e3, "sample_scale": sc,
                                "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads,
                                                 "kind": "reference", "sample": smp},
                                "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": headline.dtype, "data": "synthetic (seeded PCG32, reference RNG)",
            "impl": "reference", "config": config_dict(headline, world),
            "sample_scale": scale, "threads": threads,
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads,
                             "kind": "reference", "sample": sample},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "elems_per_s": headline.elements(scale) / sec,
            "per_config": per_config}
    print(json.dumps(line))
    return 0


# ------------------------------------------------------------- CUDA arm

class L2Flush:
    """Evicts every cached line between timed steps: a 256 MiB buffer (twice
    the 126 MB L2) is written, then a second one is read, so the L2 holds
    clean lines of unrelated data and the timed step neither hits in L2 nor
    pays for writing back the flush's dirty lines."""

    def __init__(self, torch, device):
        n = 256 * 1024 * 1024 // 4
        self.write = torch.empty(n, dtype=torch.float32, device=device)
        self.read = torch.zeros(n, dtype=torch.float32, device=device)
        self.sink = torch.empty((), dtype=torch.float32, device=device)

    def __call__(self):
        self.write.zero_()
        self.sink.copy_(self.read.max())


class Env:
    """This process's place in the job (torchrun variables) and its device."""

    def __init__(self, torch):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.device = torch.device("cuda", self.local)


def make_session(m3, env, g, stream, config):
    """A plain session at N=1; at N>1 this rank's shard of the fixed graph
    (the library partitions it along the configuration's shard axis and
    all-reduces global reductions and data-check verdicts over NCCL, on a
    communicator of its own: a fresh id per session)."""
    if env.world == 1:
        return m3.Session(g, device=env.local, stream=stream.cuda_stream)
    ident = shardsmod().shared_shard_id(m3, env.device)
    return m3.Session(g, device=env.local, stream=stream.cuda_stream,
                      shard=m3.ShardOptions(env.rank, env.world, config.shard_axis, ident))


def write_inputs(session, env, handles, data):
    """Each input's device data into the session: the whole tensor at N=1,
    this rank's slab of the global tensor (a strided device copy) at N>1."""
    for name, vid in handles.items():
        t = data[name]
        nbytes = t.numel() * t.element_size()
        if env.world == 1:
            session.write_device(vid, t.data_ptr(), nbytes)
        else:
            session.shard_write(vid, t.data_ptr(), nbytes, device=True)


def measure_cuda(m3, torch, dist, env, config, args, stream, flush, with_baseline):
    """One configuration at its full size on this rank: device-timed steps,
    the roofline of its dominant kernel, end to end through the C API and
    (rank 0, N=1) the single-core reference CPU baseline."""
    rng = ProductRng(m3)
    g = m3.Graph()
    handles, outputs = config.build(m3, g, rng, args.scale)
    session = make_session(m3, env, g, stream, config)
    report, plan_text = session.plan_report()
    data = config.inputs_device(m3, torch, env.device, args.scale)
    torch.cuda.synchronize(env.device)
    write_inputs(session, env, handles, data)
    host_in = {}
    if not args.no_e2e:
        # pinned host copies of this rank's inputs for the end-to-end leg
        for name, vid in handles.items():
            t = data[name]
            if env.world > 1:
                slab = session.shard_slab(vid)
                if slab.split:
                    t = t.narrow(slab.axis, slab.begin, slab.extent)
            pinned = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            pinned.copy_(t)
            host_in[vid] = pinned
    del data
    session.synchronize()
    torch.cuda.empty_cache()

    def one_step():
        if config.name == "c4":
            session.run_steps(config.runs_per_step, *config.carry)
        else:
            for _ in range(config.runs_per_step):
                session.run_async()

    for _ in range(args.warmup):
        one_step()
    session.synchronize()
    torch.cuda.synchronize(env.device)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(env.local)
    if env.world > 1:
        dist.barrier()
    torch.cuda.synchronize(env.device)
    sampler.start()
    time.sleep(0.3)
    align = torch.zeros(1, device=env.device) if env.world > 1 else None
    for k in range(args.steps):
        flush()
        if align is not None:
            # the flush takes a different time on each GPU: the ranks start
            # each step together, so a rank's time holds no wait for another
            # rank's flush inside the run's collective
            dist.all_reduce(align)
        starts[k].record(stream)
        one_step()
        ends[k].record(stream)
    session.synchronize()
    torch.cuda.synchronize(env.device)
    if env.world > 1:
        dist.barrier()
    clocks = sampler.stop()
    per_step = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(per_step)
    if env.world > 1:
        total_ms = shardsmod().max_over_ranks(total_ms, env.device)
    ms_per_step = total_ms / args.steps
    bytes_step = config.algorithmic_bytes(args.scale)
    value = bytes_step / (ms_per_step / 1e3) / 1e9

    # the dominant kernel: one launch per run for c1/c2/c4/c5 (C5 at N>1 adds
    # the all-reduce's launches); c3's gated-SiLU launch timed on its own graph
    peak, peak_kind = measured_peaks()
    kernel_ms = ms_per_step / config.runs_per_step
    kernel_bytes = bytes_step / config.runs_per_step / env.world
    kernel_name = plan_text
    if config.name == "c3":
        kernel_ms, kernel_bytes, kernel_name = time_c3_gsilu(m3, torch, env, stream, flush,
                                                            args.steps, args.scale)
    achieved = kernel_bytes / (kernel_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": ncu_traffic(config.name) if args.scale == 1.0 and env.world == 1 else None,
                "peak_source": (f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                                else "fallback 6650 GB/s"),
                "kernel": kernel_name, "algorithmic_bytes_per_launch": kernel_bytes,
                "launch_ms": kernel_ms}
    e2e = None
    if not args.no_e2e:
        e2e = measure_e2e(m3, torch, dist, env, stream, config, session, host_in, outputs,
                          flush, args)
    del host_in
    baseline = None
    if with_baseline:
        baseline = cpu_baseline(m3, oraclemod(), config, args.cpu_seconds)
    session.close()
    torch.cuda.empty_cache()
    return {"workload": config.workload, "value": value, "unit": "GB/s",
            "ms_per_step": ms_per_step, "dtype": config.dtype, "plan": plan_text,
            "roofline": roofline, "cpu_baseline": baseline, "e2e": e2e, "clocks": clocks,
            "gpu_launches": report.launch_count * config.runs_per_step * args.steps,
            "elems_per_s": config.elements(args.scale) / (ms_per_step / 1e3)}


def measure_plugin(m3, torch, env, stream, flush, args):
    """C1 and C2 as the reference's scheduler hands them to the backend
    plug-in (m3_cuda_backend_execute, the vtable call of
    src/m3_backend.c:113-154): C1's MUL into a temporary then ADD, C2's
    SOFTMAX then TOP_K, over device storages.  The context runs on the bench
    stream (m3_cuda_backend_set_stream), so CUDA events time each call; a
    call returns after its stream is idle, as the vtable requires.  `value`
    uses the session path's algorithmic bytes, so the two compare directly;
    the plug-in also writes C1's temporary (no liveness reaches a backend) and
    scans C2's input for NaN before its row pass."""
    lib = m3.load()
    tensors = {}
    # storages are the tensors' device addresses, resolved by a C accessor
    # (as the reference's m3_storage_data is C): no Python in the call
    storage_data = ctypes.cast(lib.m3_cuda_storage_is_address, m3.STORAGE_DATA)

    err = m3.M3Error()
    context = ctypes.c_void_p()
    options = m3.BackendOptions(env.local, storage_data, False)
    m3.check(lib.m3_cuda_backend_context_create(ctypes.byref(options), ctypes.byref(context),
                                                ctypes.byref(err)), err)
    m3.check(lib.m3_cuda_backend_set_stream(context, stream.cuda_stream, ctypes.byref(err)), err)
    views = []

    def view(key, shape, dtype=m3.F32):
        v = m3.TensorView()
        v.metadata.dtype = dtype
        v.metadata.rank = len(shape)
        step = 4
        for axis in reversed(range(len(shape))):
            v.metadata.shape[axis] = shape[axis]
            v.byte_strides[axis] = step
            step *= shape[axis]
        v.metadata.element_count = int(np.prod(shape))
        v.metadata.byte_count = v.metadata.element_count * 4
        v.storage = tensors[key].data_ptr()
        views.append(v)
        return ctypes.pointer(v)

    results = {}
    try:
        for name in ("c1", "c2"):
            config = CONFIGS[name]
            rows, width = config.shape(args.scale)
            x = config.inputs_device(m3, torch, env.device, args.scale)["x"]
            cmd = (m3.Command * 2)()
            if name == "c1":
                rng = ProductRng(m3)
                c = torch.from_numpy(rng.uniform(0, 1, 0.5, 2.0, width)).to(env.device)
                b = torch.from_numpy(rng.normal(0, 2, 0.0, 1.0, width)).to(env.device)
                tensors.clear()
                tensors.update({1: x, 2: c, 3: b, 4: torch.empty_like(x), 5: torch.empty_like(x)})
                cmd[0].kind, cmd[1].kind = m3.OPS["MUL"], m3.OPS["ADD"]
                cmd[0].descriptor.mul.left = view(1, (rows, width))
                cmd[0].descriptor.mul.right = view(2, (width,))
                cmd[0].descriptor.mul.output = view(4, (rows, width))
                cmd[1].descriptor.add.left = view(4, (rows, width))
                cmd[1].descriptor.add.right = view(3, (1, width))
                cmd[1].descriptor.add.output = view(5, (rows, width))
            else:
                tensors.clear()
                tensors.update({1: x, 2: torch.empty_like(x),
                                3: torch.empty(rows, dtype=torch.float32, device=env.device),
                                4: torch.empty(rows, dtype=torch.int32, device=env.device)})
                cmd[0].kind, cmd[1].kind = m3.OPS["SOFTMAX"], m3.OPS["TOP_K"]
                cmd[0].descriptor.softmax.input = view(1, (rows, width))
                cmd[0].descriptor.softmax.output = view(2, (rows, width))
                cmd[1].descriptor.top_k.logits = view(1, (rows, width))
                cmd[1].descriptor.top_k.values = view(3, (rows, 1))
                cmd[1].descriptor.top_k.indices = view(4, (rows, 1), m3.I32)
                cmd[1].descriptor.top_k.k = 1
            torch.cuda.synchronize(env.device)

            def call():
                m3.check(lib.m3_cuda_backend_execute(context, cmd, 2, None, ctypes.byref(err)), err)

            for _ in range(args.warmup):
                flush()
                call()
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            for i in range(args.steps):
                flush()
                starts[i].record(stream)
                call()
                ends[i].record(stream)
            torch.cuda.synchronize(env.device)
            ms = sum(a.elapsed_time(e) for a, e in zip(starts, ends)) / args.steps
            launches = int(lib.m3_cuda_backend_launch_count(context))
            results[name + "_plugin"] = {
                "workload": config.workload + " through m3_cuda_backend_execute",
                "value": config.algorithmic_bytes(args.scale) / (ms / 1e3) / 1e9,
                "unit": "GB/s", "ms_per_step": ms, "dtype": config.dtype,
                "launches_per_call": launches, "gpu_launches": launches * args.steps,
                "timing": "CUDA events on the bench stream around each call; L2 evicted between calls",
                "bytes": "the session path's algorithmic bytes"}
    finally:
        lib.m3_cuda_backend_destroy_context(context)
        tensors.clear()
    return results


def time_c3_gsilu(m3, torch, env, stream, flush, steps, scale):
    """C3's dominant kernel (the gated-SiLU launch, this rank's rows), timed
    alone."""
    c = CONFIGS["c3"]
    rows = _rows(c.rows, scale) // env.world
    g = m3.Graph()
    gate = g.value(m3.INPUT, m3.F16, (rows, c.ffn))
    up = g.value(m3.INPUT, m3.F16, (rows, c.ffn))
    y = g.inferred("GATED_SILU", [gate, up], m3.OUTPUT, m3.F16)
    g.node("GATED_SILU", [gate, up], [y])
    s = m3.Session(g, device=env.local, stream=stream.cuda_stream)
    _, text = s.plan_report()
    for _ in range(3):
        s.run_async()
    s.synchronize()
    times = []
    for _ in range(steps):
        flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        s.run_async()
        b.record(stream)
        times.append((a, b))
    s.synchronize()
    torch.cuda.synchronize(env.device)
    ms = statistics.mean(a.elapsed_time(b) for a, b in times)
    s.close()
    return ms, rows * c.ffn * 2 * 3, text


def measure_e2e(m3, torch, dist, env, stream, config, session, host_in, outputs, flush, args):
    """The same metric through the public C API with pinned host buffers of
    this rank's data, every step's host-to-device input copies and
    device-to-host output copies inside the timed region: single-run
    configurations submit each step with m3_cuda_session_submit_host_async
    (steps pipelined, timed from the first submission to the synchronise
    after the last); C4 writes, runs its 30 carried steps and reads back per
    step."""
    host_out = {}
    for vid in outputs:
        host_out[vid] = torch.empty(session.value_bytes(vid), dtype=torch.uint8, pin_memory=True)
    err = m3.M3Error()
    lib = m3.load()

    def call(fn, *a):
        m3.check(fn(session.handle, *a, ctypes.byref(err)), err)

    def one():
        for vid, buf in host_in.items():
            call(lib.m3_session_write_input, vid, ctypes.c_void_p(buf.data_ptr()), buf.nbytes)
        x_in, x_out = config.carry
        call(lib.m3_cuda_session_run_steps_async, config.runs_per_step, x_in, x_out)
        call(lib.m3_cuda_session_synchronize)
        for vid, buf in host_out.items():
            call(lib.m3_session_read_output, vid, ctypes.c_void_p(buf.data_ptr()), buf.nbytes)

    pipelined = config.runs_per_step == 1
    ins = {vid: buf.data_ptr() for vid, buf in host_in.items()}
    outs = {vid: buf.data_ptr() for vid, buf in host_out.items()}

    def submit():
        session.submit_host(ins, outs)

    for _ in range(2):
        submit() if pipelined else one()
    session.synchronize()
    torch.cuda.synchronize(env.device)
    if env.world > 1:
        dist.barrier()
    if pipelined:
        count = max(4, min(args.steps, 8) if config.name == "c5" else args.steps)
        flush()
        torch.cuda.synchronize(env.device)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(count):
            submit()
        session.synchronize()
        b.record(stream)
        torch.cuda.synchronize(env.device)
        ms = a.elapsed_time(b) / count
    else:
        times = []
        for _ in range(max(3, args.steps // 2)):
            flush()
            torch.cuda.synchronize(env.device)
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            one()
            b.record(stream)
            torch.cuda.synchronize(env.device)
            times.append(a.elapsed_time(b))
        ms = statistics.mean(times)
    if env.world > 1:
        ms = shardsmod().max_over_ranks(ms, env.device)
    h2d = sum(b.nbytes for b in host_in.values())
    d2h = sum(b.nbytes for b in host_out.values())
    mode = ("m3_cuda_session_submit_host_async per step, steps pipelined (one step's upload "
            "overlaps the previous step's download)" if pipelined else
            "m3_session_write_input, m3_cuda_session_run_steps_async + synchronize, "
            "m3_session_read_output per step")
    del host_out
    return {"value": config.algorithmic_bytes(args.scale) / (ms / 1e3) / 1e9, "unit": "GB/s",
            "ms_per_step": ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "per_rank": env.world > 1, "mode": mode}


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--config", default="c5", choices=sorted(CONFIGS),
                        help="headline configuration (the others go to per_config)")
    parser.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    parser.add_argument("--cpu-seconds", type=float, default=9.0,
                        help="CPU work budget of each cpu_baseline sample")
    parser.add_argument("--ref-seconds", type=float, default=1.0,
                        help="reference arm: seconds per step of the headline sample")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-per-config", action="store_true")
    parser.add_argument("--scale", type=float, default=1.0,
                        help="fraction of each configuration along its shard axis "
                             "(profiling only; reported numbers use 1.0)")
    args = parser.parse_args()
    headline = CONFIGS[args.config]
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args, headline)

    import torch
    import torch.distributed as dist

    env = Env(torch)
    if env.world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=env.device)
    m3 = m3mod()
    m3.load()
    stream = torch.cuda.Stream(env.device)
    torch.cuda.set_stream(stream)
    flush = L2Flush(torch, env.device)
    baseline_here = env.rank == 0 and env.world == 1 and not args.no_cpu_baseline

    result = measure_cuda(m3, torch, dist, env, headline, args, stream, flush, baseline_here)
    per_config = {}
    if not args.no_per_config:
        for name, config in CONFIGS.items():
            if name != headline.name:
                per_config[name] = measure_cuda(m3, torch, dist, env, config, args, stream, flush,
                                                baseline_here)
        if env.world == 1:
            per_config.update(measure_plugin(m3, torch, env, stream, flush, args))
    launches = result["gpu_launches"] + sum(r["gpu_launches"] for r in per_config.values())
    config = config_dict(headline, env.world)
    if args.scale != 1.0:
        config["scale"] = args.scale
    line = {"metric": METRIC, "value": result["value"], "unit": "GB/s", "n_gpus": env.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": result["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": headline.dtype,
            "data": "synthetic: seeded PCG32 streams of the reference RNG, generated on device",
            "config": config, "plan": result["plan"],
            "roofline": result["roofline"], "cpu_baseline": result["cpu_baseline"],
            "e2e": result["e2e"], "clocks": result["clocks"],
            "gpu_launches": launches, "gpu_launches_headline": result["gpu_launches"],
            "elems_per_s": result["elems_per_s"], "per_config": per_config}
    if env.world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if env.rank == 0:
        print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
