"""Generates the golden vectors in this folder from the REFERENCE's own CUDA kernels.

The reference (cnmoro/fast-d1-omni) ships no numeric golden vectors or known-answer tests for its kernels. This
script runs the reference's cuda/kernels.cu + cuda/gemm.cu, rebuilt unchanged into oracle/_ref/libd1ref.so by
oracle/Makefile, on small seeded inputs on a B200, and stores inputs and outputs as .npz fixtures:

  kernels.npz  every d1_* kernel of the hot path (norms, short conv, QK-norm+RoPE, flash attention with GQA /
               bias / prefix keys / marker queries, SwiGLU, bias+act, scorer, gathers, unshuffle, audio pieces)
  gemm.npz     d1_lt_gemm (cuBLASLt) on small config-1 shapes, fp16 and fp32-residual outputs
  engine.npz   logits of a small text model (4 layers, attention at layer 2, vocab 4096, 2-layer head; weights from
               weights.text_weights(seed=0, ...)) run through the host runner with the reference's kernels

tests/test_golden.py checks the oracle against these on the CPU (-m "not gpu") and libd1kernels against them on
the GPU. Run on a GPU machine from the repository root:  python tests/golden/make_golden.py [--out DIR]
(default DIR: this folder).
"""
import ctypes as C
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))
OUT = Path(__file__).resolve().parent

from conftest import REF_LIB, load_package  # noqa: E402

import torch  # noqa: E402

from golden_cases import engine_case, gemm_cases, kernel_cases  # noqa: E402


def main():
    global OUT
    if "--out" in sys.argv:
        OUT = Path(sys.argv[sys.argv.index("--out") + 1])
        OUT.mkdir(parents=True, exist_ok=True)
    pkg = load_package()
    lib = C.CDLL(str(REF_LIB))
    pkg.abi.bind(lib, (pkg.abi.KERNELS,))
    torch.cuda.set_device(0)

    out = {}
    for name, case in kernel_cases().items():
        res = case.run(lib)
        for k, v in case.inputs.items():
            out[f"{name}/in/{k}"] = v
        for k, v in res.items():
            out[f"{name}/out/{k}"] = v
    np.savez_compressed(OUT / "kernels.npz", **out)

    ctx = lib.d1_lt_init(32 << 20)
    out = {}
    for name, case in gemm_cases().items():
        res = case.run(lib, ctx)
        for k, v in case.inputs.items():
            out[f"{name}/in/{k}"] = v
        for k, v in res.items():
            out[f"{name}/out/{k}"] = v
    np.savez_compressed(OUT / "gemm.npz", **out)

    logits, meta = engine_case(pkg, str(REF_LIB))
    np.savez_compressed(OUT / "engine.npz", logits=logits, **meta)
    for f in ("kernels.npz", "gemm.npz", "engine.npz"):
        print(f, (OUT / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
