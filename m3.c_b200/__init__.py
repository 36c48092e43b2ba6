"""B200 CUDA provider for m3.c's tensor hot path.

The product is libm3cuda.so (C ABI in include/m3_cuda.h); `m3cuda` is its
ctypes binding.  The directory name contains a dot, so load the package by
path, e.g.

    spec = importlib.util.spec_from_file_location(
        "m3c_b200", "m3.c_b200/__init__.py",
        submodule_search_locations=["m3.c_b200"])
"""

from . import m3cuda  # noqa: F401
