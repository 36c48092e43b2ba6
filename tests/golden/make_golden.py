"""Regenerates tests/golden/golden.npz: every case of cases.py run through
the reference's own CPU provider (oracle/_ref/libm3ref.so, built by
`make -C oracle` from the reference sources).  Test infrastructure; run here,
where the reference sources are available:

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    sys.modules[name] = module
    spec.loader.exec_module(module)
    return module


def main() -> None:
    m3 = _load("m3cuda", os.path.join(ROOT, "m3.c_b200", "m3cuda.py"))
    oracle = _load("m3_oracle_py", os.path.join(ROOT, "oracle", "oracle.py"))
    cases = _load("golden_cases", os.path.join(HERE, "cases.py"))
    oracle.build()
    ref = m3.bind(oracle.reference(), cuda=False)
    arrays = {}
    for name, (build, inputs, checks) in cases.CASES.items():
        data = inputs(m3, oracle)
        g = m3.Graph(lib=ref)
        handles, outputs = build(m3, g)
        s = m3.Session(g, allow_metal=False, allow_neural_engine=False, cuda=False)
        for key, vid in handles.items():
            s.write(vid, data[key])
            arrays[f"{name}/in/{key}"] = np.ascontiguousarray(data[key])
        s.run()
        for k, vid in enumerate(outputs):
            arrays[f"{name}/out/{k}"] = s.read(vid).copy()
        s.close()
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    print(f"{len(cases.CASES)} cases, {len(arrays)} arrays")


if __name__ == "__main__":
    main()
