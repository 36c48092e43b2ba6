"""Golden fixtures (tests/golden/golden.npz): outputs of the reference's own
CPU provider for every operator on the path, committed so that the GPU
parity check needs no reference sources on the GPU host.

* CPU: the fixtures' inputs are still what cases.py generates, and, where
  the compiled reference is available, it still produces the stored outputs
  (the fixtures are not stale).
* GPU: the CUDA path meets each output's parity bar against the stored
  reference outputs (bars listed in tests/golden/cases.py).
"""

from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


def _cases():
    name = "golden_cases"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, os.path.join(GOLDEN, "cases.py"))
        module = importlib.util.module_from_spec(spec)
        sys.modules[name] = module
        spec.loader.exec_module(module)
    return sys.modules[name].CASES


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "golden.npz"))


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype.itemsize == 4 else np.uint16)


def _ordered(b, width):
    b = b.astype(np.int64)
    sign = 1 << (width - 1)
    return np.where(b & sign, -(b & (sign - 1)), b)


def _meets(check, mine, want):
    if check == "bits":
        return np.array_equal(_bits(mine), _bits(want))
    if check == "ulp1":
        width = 8 * mine.dtype.itemsize
        return int(np.abs(_ordered(_bits(mine), width) - _ordered(_bits(want), width)).max(initial=0)) <= 1
    tol = {"rel6": 1e-6, "sin": 2.0 ** -19, "rel20": 2.0 ** -20}[check]
    a = mine.astype(np.float64)
    b = want.astype(np.float64)
    diff = np.abs(a - b)
    same = (np.isnan(a) & np.isnan(b)) | (a == b)
    if check == "sin":
        ok = same | (diff <= tol) | (diff <= tol * np.maximum(np.abs(a), np.abs(b)))
    else:
        ok = same | (diff <= tol * np.maximum(np.abs(a), np.abs(b)))
    return bool(ok.all())


@pytest.mark.parametrize("name", sorted(_cases()))
def test_fixture_inputs_match_cases(m3, oracle, golden, name):
    build, inputs, checks = _cases()[name]
    for key, value in inputs(m3, oracle).items():
        assert np.array_equal(golden[f"{name}/in/{key}"], value)


@pytest.mark.parametrize("name", sorted(_cases()))
def test_reference_reproduces_fixture(m3, ref, golden, name):
    build, inputs, checks = _cases()[name]
    g = m3.Graph(lib=ref)
    handles, outputs = build(m3, g)
    s = m3.Session(g, allow_metal=False, allow_neural_engine=False, cuda=False)
    for key, vid in handles.items():
        s.write(vid, golden[f"{name}/in/{key}"])
    s.run()
    for k, vid in enumerate(outputs):
        assert np.array_equal(_bits(s.read(vid)), _bits(golden[f"{name}/out/{k}"]))


@pytest.mark.gpu
@pytest.mark.parametrize("fuse", [True, False])
@pytest.mark.parametrize("name", sorted(_cases()))
def test_cuda_matches_reference_fixture(m3, gpu, golden, name, fuse):
    build, inputs, checks = _cases()[name]
    g = m3.Graph()
    handles, outputs = build(m3, g)
    s = m3.Session(g, fuse=fuse)
    for key, vid in handles.items():
        s.write(vid, golden[f"{name}/in/{key}"])
    s.run()
    for k, (vid, check) in enumerate(zip(outputs, checks)):
        mine = s.read(vid)
        want = golden[f"{name}/out/{k}"]
        assert mine.dtype == want.dtype and mine.shape == want.shape
        assert _meets(check, mine, want), f"{name} output {k} ({check})"
