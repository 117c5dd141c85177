"""Shared test setup: the `gpu` marker, the package loader and small helpers.

`-m "not gpu"` runs on a CPU-only machine (oracle vs golden vectors, host logic, library exports).
`-m gpu` runs the parity tests proper on a B200, through the C ABI of libd1kernels.
"""
import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "fast-d1-omni_b200"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def load_package():
    name = "fast_d1_omni_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; parity tests through the C ABI")


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def gpu_lib(pkg):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return pkg.lib()
