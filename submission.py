"""Drop-in submission module: ``custom_kernel(data)`` and ``solve(data)``.

The harness of the reference imports a module named ``submission`` and calls
``custom_kernel`` (submission.py:788, :889-891 of the reference). This file keeps
that name and signature and forwards to the B200-native package in
``nvfp4-group-gemm_b200/`` (a directory name that is not a Python identifier, so
it is registered here under the import name ``nvfp4_group_gemm_b200``).
"""
from __future__ import annotations

import importlib.util
import os
import sys

PACKAGE_NAME = "nvfp4_group_gemm_b200"
PACKAGE_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "nvfp4-group-gemm_b200")


def load_package():
    """Import the package from its directory (once) and return the module."""
    mod = sys.modules.get(PACKAGE_NAME)
    if mod is not None:
        return mod
    spec = importlib.util.spec_from_file_location(
        PACKAGE_NAME, os.path.join(PACKAGE_DIR, "__init__.py"),
        submodule_search_locations=[PACKAGE_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[PACKAGE_NAME] = mod
    try:
        spec.loader.exec_module(mod)
    except BaseException:
        sys.modules.pop(PACKAGE_NAME, None)
        raise
    return mod


_pkg = load_package()
input_t = _pkg.input_t
output_t = _pkg.output_t


def custom_kernel(data: input_t) -> output_t:
    return _pkg.custom_kernel(data)


def solve(data: input_t) -> output_t:
    return _pkg.custom_kernel(data)
