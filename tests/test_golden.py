"""Golden vectors produced by the REFERENCE's own CUDA kernels (tests/golden/make_golden.py):
  -m "not gpu": the oracle (oracle/d1_oracle.py) reproduces them on the CPU — this pins the oracle;
  -m gpu:       libd1kernels reproduces them through its C ABI on the same inputs.

Tolerances by output kind: f16 — within one fp16 rounding step (2^-10 relative, the reference and the restatement
round the same fp32 value and may land on either side of a tie after a different reduction order); f32 — 1e-5;
attn — 4e-3 absolute (fp16 P, online vs global softmax); exact — bitwise. The engine logits: per question
(option logits), centred |dlogit| mean <= 0.01 and max <= 0.06 with no top-answer flip (tools/logit_err.py).
"""
from pathlib import Path

import numpy as np
import pytest

import golden_cases as G
from oracle import d1_oracle as O

GOLD = Path(__file__).resolve().parent / "golden"


def load(name):
    p = GOLD / name
    if not p.exists():
        pytest.skip(f"{p} not generated (python tests/golden/make_golden.py on a GPU machine)")
    z = np.load(p)
    cases = {}
    for k in z.files:
        case, kind, field = k.split("/")
        cases.setdefault(case, {"in": {}, "out": {}})[kind][field] = z[k]
    return cases


def close(got, want, tol):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    if tol == "exact":
        return np.array_equal(got, want)
    if tol == "f16":
        return bool((np.abs(got - want) <= 2.0 ** -10 * np.abs(want) + 1e-4).all())
    if tol == "f32":
        return bool(np.allclose(got, want, rtol=1e-5, atol=1e-5))
    if tol == "attn":
        return bool(np.abs(got - want).max() <= 4e-3)
    raise ValueError(tol)


def kernel_case_names():
    return sorted(G.kernel_cases().keys())


@pytest.mark.parametrize("name", kernel_case_names())
def test_oracle_matches_reference_kernels(name):
    gold = load("kernels.npz")[name]
    case = G.kernel_cases()[name]
    case.inputs = gold["in"]
    want = case.oracle()
    for k, ref in gold["out"].items():
        assert close(want[k], ref, case.tol), (name, k)


@pytest.mark.parametrize("name", ["f16_out", "f32_residual"])
def test_oracle_matches_reference_gemm(name):
    gold = load("gemm.npz")[name]
    case = G.gemm_cases()[name]
    case.inputs = gold["in"]
    want = case.oracle()
    tol = "f16" if case.tol == "f16" else "f32"
    # the reference GEMM's fp32 accumulation order differs from numpy's: allow fp32 noise around the rounding
    got = want["y"]
    ref = gold["out"]["y"]
    if tol == "f16":
        assert (np.abs(got - ref) <= 2.0 ** -10 * np.abs(ref) + 2e-3).all()
    else:
        assert np.allclose(got, ref, rtol=1e-5, atol=1e-4)


def test_oracle_matches_reference_engine():
    from fast_d1_omni_b200.weights import text_weights
    p = GOLD / "engine.npz"
    if not p.exists():
        pytest.skip("engine.npz not generated")
    z = np.load(p)
    w = text_weights(**G.ENGINE)
    b = G.engine_batch()
    sizes = list(z["sizes"])
    for prec in ("f16", "f32"):
        got = O.launch_text(w, b, prec)
        errs = O.centred_logit_err(z["logits"], got, sizes)
        assert errs.mean() <= 0.01 and errs.max() <= 0.06, (prec, errs)
        assert O.top_flips(z["logits"], got, sizes) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("name", kernel_case_names())
def test_kernels_match_reference_golden(gpu_lib, name):
    gold = load("kernels.npz")[name]
    case = G.kernel_cases()[name]
    case.inputs = gold["in"]
    got = case._run(gpu_lib, gold["in"])
    for k, ref in gold["out"].items():
        assert close(got[k], ref, case.tol), (name, k)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["f16_out", "f32_residual"])
def test_gemm_matches_reference_golden(gpu_lib, name):
    gold = load("gemm.npz")[name]
    case = G.gemm_cases()[name]
    ctx = gpu_lib.d1_lt_init(0)
    try:
        got = case._run(gpu_lib, gold["in"], ctx)["y"]
    finally:
        gpu_lib.d1_lt_destroy(ctx)
    ref = gold["out"]["y"]
    if case.tol == "f16":
        assert (np.abs(got.astype(np.float64) - ref) <= 2.0 ** -10 * np.abs(ref) + 2e-3).all()
    else:
        assert np.allclose(got, ref, rtol=1e-5, atol=1e-4)


@pytest.mark.gpu
def test_engine_matches_reference_golden(pkg, gpu_lib):
    p = GOLD / "engine.npz"
    if not p.exists():
        pytest.skip("engine.npz not generated")
    z = np.load(p)
    for fused in (False, True):
        from fast_d1_omni_b200.model import TextModel
        from fast_d1_omni_b200.weights import text_weights
        m = TextModel(text_weights(**G.ENGINE), fused=fused, cap_tokens=512)
        try:
            got = m(G.engine_batch())
        finally:
            m.close()
        errs = O.centred_logit_err(z["logits"], got, list(z["sizes"]))
        assert errs.mean() <= 0.01 and errs.max() <= 0.06, errs
        assert O.top_flips(z["logits"], got, list(z["sizes"])) == 0
