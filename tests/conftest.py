"""Shared test setup: loads the ``clj-xla_b200`` package as ``cljxla_b200``
(the directory name is not a Python identifier) and registers markers."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _load_pkg():
    if "cljxla_b200" in sys.modules:
        return sys.modules["cljxla_b200"]
    pkg_dir = os.path.join(ROOT, "clj-xla_b200")
    spec = importlib.util.spec_from_file_location(
        "cljxla_b200", os.path.join(pkg_dir, "__init__.py"), submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["cljxla_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


_load_pkg()

# compiled fused kernels are cached on disk; the tests keep that cache inside the
# repository's build folder instead of the user's home
os.environ.setdefault("CLJXLA_B200_CACHE_DIR", os.path.join(ROOT, "_build", "jit_cache"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device and the built library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
