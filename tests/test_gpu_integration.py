"""The CUDA provider inside the reference's own scheduler.

integration/_ref/libm3ref_cuda.so is the reference's graph/session library,
backend layer and provider scheduler compiled from its own sources with
integration/cuda_provider.patch applied and integration/m3_backend_cuda.c
added (the registration a maintainer would commit), linked against
libm3cuda.so.  Here the reference's code decides everything: backend creation
(m3_backend_create_preferred), placement (m3_provider_select_regular),
execution (m3_provider_execute_regular -> m3_backend_execute ->
m3_cuda_backend_execute) and storage I/O (m3_storage_write/read).

* C1 and C2 run through the reference's m3_session_create / m3_session_run
  with every node placed on the CUDA provider, in both storage modes
  (managed memory, and device memory with the vtable I/O hooks), against
  the reference's CPU-only session on the same inputs: C1 bit-exact, C2's
  max/argmax bit-exact and its probabilities within 1e-6 relative.
* The reference's flow-solver arithmetic (m3_flow_guided_velocity,
  m3_flow_euler_step, m3_flow_blend_overlap) issues its commands on offset
  views through m3_command_executor_execute; on the CUDA backend (managed
  storage: the solver fills its scalar operands on the host) the results
  equal the host backend's bit for bit.
"""

from __future__ import annotations

import ctypes
import importlib.util
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBRARY = os.path.join(ROOT, "integration", "_ref", "libm3ref_cuda.so")


def _bench():
    if "m3_bench" not in sys.modules:
        spec = importlib.util.spec_from_file_location("m3_bench", os.path.join(ROOT, "bench.py"))
        module = importlib.util.module_from_spec(spec)
        sys.modules["m3_bench"] = module
        spec.loader.exec_module(module)
    return sys.modules["m3_bench"]


@pytest.fixture(scope="module")
def refcuda(m3):
    assert os.path.exists(LIBRARY), "integration/_ref/libm3ref_cuda.so has not been built"
    lib = m3.bind(ctypes.CDLL(LIBRARY, mode=ctypes.RTLD_LOCAL), cuda=False)
    lib.m3_backend_cuda_configure.argtypes = [ctypes.c_int, ctypes.c_bool]
    lib.m3_backend_cuda_configure.restype = None
    fp = ctypes.POINTER(ctypes.c_float)
    lib.m3h_flow_solver_math.argtypes = [
        ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_float, ctypes.c_float,
        ctypes.c_uint64, ctypes.c_float, fp, fp, fp, fp, fp, fp,
        ctypes.POINTER(ctypes.c_int), ctypes.POINTER(m3.M3Error)]
    lib.m3h_flow_solver_math.restype = ctypes.c_int
    yield lib
    lib.m3_backend_cuda_configure(0, True)


def _run(m3, lib, cfg, data, cuda_placement):
    rng = _bench().ProductRng(m3)
    g = m3.Graph(lib=lib)
    handles, outputs = cfg.build(m3, g, rng)
    s = m3.Session(g, allow_metal=cuda_placement, allow_neural_engine=False,
                   allow_cpu=not cuda_placement, cuda=False)
    providers = {s.provider(n) for n in range(2)}   # both graphs have two nodes
    for name, vid in handles.items():
        s.write(vid, data[name])
    s.run()
    out = [s.read(v).copy() for v in outputs]
    s.close()
    return out, providers


@pytest.mark.parametrize("managed", [True, False])
def test_reference_session_runs_on_the_cuda_provider(m3, ref, refcuda, gpu, managed):
    refcuda.m3_backend_cuda_configure(0, managed)
    bench = _bench()
    rng = bench.ProductRng(m3)
    for name in ("c1", "c2"):
        cfg = bench.CONFIGS[name]
        data = cfg.inputs_host(rng)
        got, providers = _run(m3, refcuda, cfg, data, True)
        want, cpu = _run(m3, ref, cfg, data, False)
        assert providers == {m3.PROVIDER_CUDA} and cpu == {m3.PROVIDER_CPU}
        if name == "c1":
            assert np.array_equal(got[0].view(np.uint32), want[0].view(np.uint32))
        else:
            p, v, i = got
            rp, rv, ri = want
            assert np.array_equal(i, ri) and np.array_equal(v.view(np.uint32), rv.view(np.uint32))
            rel = np.abs(p.astype(np.float64) - rp) / np.maximum(np.abs(rp), 1e-30)
            assert rel.max() <= 1e-6, rel.max()


def test_reference_flow_solver_through_the_command_executor(m3, refcuda, gpu):
    refcuda.m3_backend_cuda_configure(0, True)
    length, channels, overlap = 320, 64, 48
    velocity = m3.fill_normal(3, 1, 0.0, 1.0, 2 * length * channels)
    latent = m3.fill_normal(3, 0, 0.0, 1.0, length * channels)
    noise = m3.fill_normal(3, 5, 0.0, 1.0, overlap * channels)
    previous = m3.fill_normal(3, 6, 0.0, 1.0, overlap * channels)
    delta = np.float32(1.0) / np.float32(30.0)
    fp = ctypes.POINTER(ctypes.c_float)
    results = []
    for cuda in (1, 0):
        guided = np.zeros(length * channels, np.float32)
        after = np.zeros(length * channels, np.float32)
        provider = ctypes.c_int(-1)
        err = m3.M3Error()
        status = refcuda.m3h_flow_solver_math(
            cuda, length, channels, 4.0, float(delta), overlap, 0.6,
            velocity.ctypes.data_as(fp), latent.ctypes.data_as(fp), noise.ctypes.data_as(fp),
            previous.ctypes.data_as(fp), guided.ctypes.data_as(fp), after.ctypes.data_as(fp),
            ctypes.byref(provider), ctypes.byref(err))
        m3.check(status, err)
        results.append((guided, after, provider.value))
    (g_cuda, l_cuda, p_cuda), (g_host, l_host, p_host) = results
    assert p_cuda == m3.PROVIDER_CUDA and p_host == m3.PROVIDER_CPU
    assert np.array_equal(g_cuda.view(np.uint32), g_host.view(np.uint32))
    assert np.array_equal(l_cuda.view(np.uint32), l_host.view(np.uint32))
    # the Euler step moved the latent and the blend rewrote its first rows
    assert not np.array_equal(l_cuda, latent)
