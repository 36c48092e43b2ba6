"""Python access to the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Only the tests, `__graft_entry__.smoke()` and the benchmark's CPU-baseline
leg import this module; the product library never does.

* `restatement()` loads _build/libm3oracle.so, this repository's C
  restatement of the reference algorithms (m3_oracle.c).
* `reference()` loads _ref/libm3ref.so, the reference's own CPU provider
  compiled from its sources (see Makefile).  It exports the reference's m3.h
  graph/session API and its command-level backend API.

Both are built by `make -C oracle` (the reference library only where the
reference tree is present; it travels prebuilt).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
RESTATEMENT_PATH = os.path.join(HERE, "_build", "libm3oracle.so")
REFERENCE_PATH = os.path.join(HERE, "_ref", "libm3ref.so")

F32, F16, BF16, I32 = 0, 1, 2, 3
_DTYPE_OF = {np.dtype(np.float32): F32, np.dtype(np.int32): I32}


class View(ctypes.Structure):
    """m3o_view of m3_oracle.h."""

    _fields_ = [("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("shape", ctypes.c_uint64 * 8),
                ("byte_strides", ctypes.c_uint64 * 8),
                ("byte_offset", ctypes.c_uint64), ("base", ctypes.c_void_p)]


def view(array: np.ndarray, dtype: int | None = None) -> View:
    """A view of a numpy array (any non-negative strides).  16-bit float data
    is carried as uint16 arrays, so pass dtype=F16 or BF16 for those."""
    if dtype is None:
        dtype = _DTYPE_OF[array.dtype]
    v = View()
    v.dtype = dtype
    v.rank = array.ndim
    for axis in range(array.ndim):
        v.shape[axis] = array.shape[axis]
        assert array.strides[axis] >= 0
        v.byte_strides[axis] = array.strides[axis]
    v.byte_offset = 0
    v.base = array.ctypes.data
    return v


_restatement = None
_reference = None


def build() -> None:
    """Compile the checkers: the restatement always, the reference library
    when M3_REFERENCE names the reference tree (a library built earlier is
    kept and used otherwise)."""
    targets = ["oracle"]
    reference = os.environ.get("M3_REFERENCE", "")
    if reference and os.path.isdir(reference):
        targets.append("ref")
    subprocess.run(["make", "-C", HERE, *targets], check=True,
                   stdout=subprocess.DEVNULL)


def restatement() -> ctypes.CDLL:
    global _restatement
    if _restatement is None:
        lib = ctypes.CDLL(RESTATEMENT_PATH)
        vp = ctypes.POINTER(View)
        for name, args in {
            "m3o_copy": [vp, vp], "m3o_cast": [vp, vp],
            "m3o_binary": [ctypes.c_int, vp, vp, vp],
            "m3o_gated_silu": [vp, vp, vp], "m3o_snake1d": [vp, vp, vp],
            "m3o_tanh": [vp, vp], "m3o_softmax": [vp, vp],
            "m3o_top_k": [vp, vp, vp, ctypes.c_uint64],
            "m3o_rms_norm": [vp, vp, vp, ctypes.c_float],
            "m3o_layer_norm": [vp, vp, vp, vp, ctypes.c_float],
            "m3o_abs_max": [vp, vp], "m3o_clamp_unit": [vp, vp],
            "m3o_row_sum": [vp, vp],
        }.items():
            getattr(lib, name).argtypes = args
            getattr(lib, name).restype = ctypes.c_int
        lib.m3o_f32_to_f16.argtypes = [ctypes.c_float]
        lib.m3o_f32_to_f16.restype = ctypes.c_uint16
        lib.m3o_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.m3o_f16_to_f32.restype = ctypes.c_float
        lib.m3o_f32_to_bf16.argtypes = [ctypes.c_float]
        lib.m3o_f32_to_bf16.restype = ctypes.c_uint16
        lib.m3o_bf16_to_f32.argtypes = [ctypes.c_uint16]
        lib.m3o_bf16_to_f32.restype = ctypes.c_float
        lib.m3o_flow_timestep_delta.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        lib.m3o_flow_timestep_delta.restype = ctypes.c_float
        lib.m3o_flow_timestep.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        lib.m3o_flow_timestep.restype = ctypes.c_float
        lib.m3o_pcg32_fill.argtypes = [ctypes.c_uint64, ctypes.c_uint64,
                                       ctypes.c_void_p, ctypes.c_size_t]
        lib.m3o_pcg32_fill.restype = None
        _restatement = lib
    return _restatement


def reference() -> ctypes.CDLL:
    """The reference CPU provider (raw CDLL; bind its m3.h signatures with
    the product binding's `bind(lib, cuda=False)`)."""
    global _reference
    if _reference is None:
        if not os.path.exists(REFERENCE_PATH):
            raise FileNotFoundError(f"{REFERENCE_PATH} has not been built")
        _reference = ctypes.CDLL(REFERENCE_PATH, mode=ctypes.RTLD_LOCAL)
    return _reference


def reference_available() -> bool:
    return os.path.exists(REFERENCE_PATH)


# ------------------------------------------------------------ conveniences

def _call(name: str, *args) -> int:
    return getattr(restatement(), name)(*args)


def to_f16(values: np.ndarray) -> np.ndarray:
    """F32 -> F16 bits with the reference's encoder (vectorised through C)."""
    flat = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(flat.shape, dtype=np.uint16)
    status = _call("m3o_cast", ctypes.byref(view(flat)),
                   ctypes.byref(view(out, F16)))
    assert status == 0
    return out


def to_bf16(values: np.ndarray) -> np.ndarray:
    flat = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(flat.shape, dtype=np.uint16)
    status = _call("m3o_cast", ctypes.byref(view(flat)),
                   ctypes.byref(view(out, BF16)))
    assert status == 0
    return out


def widen(bits: np.ndarray, dtype: int) -> np.ndarray:
    """F16/BF16 bits -> F32 with the reference's decoder."""
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(bits.shape, dtype=np.float32)
    status = _call("m3o_cast", ctypes.byref(view(bits, dtype)),
                   ctypes.byref(view(out)))
    assert status == 0
    return out


def pcg32_words(seed: int, sequence: int, count: int) -> np.ndarray:
    """`count` words of the reference's PCG32 stream (src/m3_rng.c:9-39)."""
    out = np.empty(count, dtype=np.uint32)
    restatement().m3o_pcg32_fill(seed, sequence, out.ctypes.data, count)
    return out


def uniform(seed: int, sequence: int, low: float, high: float,
            count: int) -> np.ndarray:
    """Uniforms on [low, high) from the reference stream: 24 bits scaled by
    2^-24 (src/m3_rng.c:53-66), then low + (high - low) * u in F32 (the
    benchmark's scaling, one rounding per statement)."""
    u = (pcg32_words(seed, sequence, count) >> np.uint32(8)).astype(np.float32)
    u *= np.float32(2.0 ** -24)
    span = np.float32(high) - np.float32(low)
    return (np.float32(low) + span * u).astype(np.float32)


def run(name: str, *arrays_and_dtypes, **scalars) -> int:
    """Call m3o_<name> on (array, dtype) pairs (dtype None = infer)."""
    views = []
    for item in arrays_and_dtypes:
        if item is None:
            views.append(None)
            continue
        array, dtype = item if isinstance(item, tuple) else (item, None)
        views.append(ctypes.byref(view(array, dtype)))
    extra = list(scalars.values())
    return _call("m3o_" + name, *views, *extra)
