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


REF_LIB = ROOT / "oracle" / "_ref" / "libd1ref.so"


@pytest.fixture(scope="session")
def ref_lib(pkg, gpu_lib):
    """The reference's own kernels (cuda/kernels.cu + cuda/gemm.cu built unchanged by oracle/Makefile)."""
    import ctypes
    if not REF_LIB.exists():
        pytest.skip("oracle/_ref/libd1ref.so not built (make -C oracle)")
    lib = ctypes.CDLL(str(REF_LIB))
    pkg.abi.bind(lib, (pkg.abi.KERNELS,))
    return lib


def half_ulp_close(a, b, rel=2.0 ** -10, abs_tol=1e-6):
    """|a - b| <= rel*|b| + abs_tol elementwise (one fp16 rounding step)."""
    import numpy as np
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.abs(a - b) <= rel * np.abs(b) + abs_tol


load_package()  # make `fast_d1_omni_b200` importable for module-level imports in the tests
