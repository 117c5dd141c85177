"""fast-d1-omni_b200 — the d1rs forward pass (LFM2.5 hybrid trunk, decision head, SigLIP2 vision tower,
FastConformer audio encoder) as sm_100a (B200) kernels behind the reference's C ABI (src/cuda.rs:102-175).

The product is libd1kernels.{so,a} built from csrc/ by build.py. This Python package only loads it and drives it
(synthetic weights, batches, replicas across GPUs); there is no Python or CPU compute path: if the library is
missing, `lib()` raises.

The directory name contains dashes, so the package is imported under the name `fast_d1_omni_b200` via
`load_package()` in the repository's entry points.
"""
import ctypes
from pathlib import Path

from . import abi

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libd1kernels.so"
INCLUDE = HERE.parent / "include"

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded libd1kernels.so with prototypes attached. Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python fast-d1-omni_b200/build.py` "
                               "(the CUDA extension is required; there is no fallback path)")
        _lib = ctypes.CDLL(str(LIB_PATH))
        abi.bind(_lib)
    return _lib


def check(status: int, what: str = "") -> None:
    """Raise on a nonzero status from the library (the reference panics on nonzero, src/cuda.rs:182-186)."""
    if status != 0:
        err = lib().d1h_last_error()
        raise RuntimeError(f"d1 call failed ({status}) {what}: {err.decode() if err else ''}")
