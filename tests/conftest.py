"""pytest configuration: the ``gpu`` marker, the package loader and shared fixtures.

The product package lives in the directory ``verace-v1_b200/`` (not an importable
identifier), so it is registered here under the module name ``verace_v1_b200``.
"""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _load_package():
    if "verace_v1_b200" in sys.modules:
        return sys.modules["verace_v1_b200"]
    pkg_dir = os.path.join(ROOT, "verace-v1_b200")
    spec = importlib.util.spec_from_file_location(
        "verace_v1_b200", os.path.join(pkg_dir, "__init__.py"),
        submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["verace_v1_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


_load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


GOLDEN = os.path.join(ROOT, "tests", "golden")


def load_golden(name):
    """Return {case: {key: array}} for tests/golden/<name>_golden.npz."""
    z = np.load(os.path.join(GOLDEN, f"{name}_golden.npz"))
    out = {}
    for key in z.files:
        case, rest = key.split("/", 1)
        d = out.setdefault(case, {"p": {}})
        if rest.startswith("p/"):
            d["p"][rest[2:]] = z[key]
        else:
            d[rest] = z[key]
    return out
