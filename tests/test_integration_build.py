"""The reference-side integration, without a GPU.

integration/cuda_provider.patch applies to the reference's sources and the
patched reference (integration/_ref/libm3ref_cuda.so) builds and links
against libm3cuda.so.  On a host without a device the patched scheduler
behaves as the reference does when Metal is absent: the CUDA backend
reports M3_STATUS_UNSUPPORTED, backend creation falls through to the host
backend, and the graph runs on the CPU provider with the reference's own
results.  (On a GPU host the same session places on the CUDA provider:
tests/test_gpu_integration.py.)
"""

from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBRARY = os.path.join(ROOT, "integration", "_ref", "libm3ref_cuda.so")


def test_patch_touches_only_the_scheduler_files():
    text = open(os.path.join(ROOT, "integration", "cuda_provider.patch")).read()
    files = sorted({line.split()[1] for line in text.splitlines() if line.startswith("--- ")})
    assert files == ["a/src/m3_backend.c", "a/src/m3_backend.h",
                     "a/src/m3_backend_internal.h", "a/src/m3_provider.c"]


def test_patched_reference_falls_back_without_a_device(m3, ref):
    if not os.path.exists(LIBRARY):
        pytest.skip("integration/_ref has not been built (set M3_REFERENCE and build)")
    lib = m3.bind(ctypes.CDLL(LIBRARY, mode=ctypes.RTLD_LOCAL), cuda=False)
    devices = m3.load().m3_cuda_device_count()
    x = np.linspace(-2, 2, 64, dtype=np.float32).reshape(4, 16)
    results = []
    for library in (lib, ref):
        g = m3.Graph(lib=library)
        v = g.value(m3.INPUT, m3.F32, (4, 16))
        c = g.constant(m3.F32, np.full(16, 1.5, np.float32))
        t = g.inferred("MUL", [v, c], m3.TEMPORARY, m3.F32)
        g.node("MUL", [v, c], [t])
        p = g.inferred("SOFTMAX", [t], m3.OUTPUT, m3.F32)
        g.node("SOFTMAX", [t], [p])
        s = m3.Session(g, allow_metal=True, allow_neural_engine=False, allow_cpu=True,
                       cuda=False)
        expected = m3.PROVIDER_CUDA if (devices > 0 and library is lib) else m3.PROVIDER_CPU
        assert s.provider(0) == expected and s.provider(1) == expected
        s.write(v, x)
        s.run()
        results.append(s.read(p))
        s.close()
    if devices == 0:
        assert np.array_equal(results[0], results[1])
