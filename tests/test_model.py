"""End-to-end parity of the text forward (trunk + decision head) through the runner and the C ABI.

random-init weights seed 0 N(0, 0.02), norms 1, 16 layers (attention at {2,5,8,10,12,14}),
8 packed sequences x 256 uniform token ids. The north-star bar, per question (3 option logits): mean |dlogit|
<= 0.01, max <= 0.06, zero top-answer flips, |dlogit| defined as tools/logit_err.py does (centred logits), against
  - the fp32 restatement (oracle, prec="f32": the stand-in for the fp32 PyTorch reference),
  - the reference's own F16 engine (its kernels and cuBLASLt GEMMs, oracle/_ref/libd1ref.so) run through the same
    host runner.
"""
import numpy as np
import pytest

from oracle import d1_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def weights(pkg):
    from fast_d1_omni_b200.weights import text_weights
    return text_weights(0)


@pytest.fixture(scope="module")
def model(pkg, gpu_lib, weights):
    from fast_d1_omni_b200.model import TextModel
    m = TextModel(weights, cap_tokens=8192)
    yield m
    m.close()


@pytest.fixture(scope="module")
def batch0():
    from fast_d1_omni_b200.weights import text_batch
    return text_batch(1, 8, 256)


@pytest.fixture(scope="module")
def oracle_f32(weights, batch0):
    return O.launch_text(weights, batch0, "f32")


def assert_bar(ref, got, n_q, mean_tol=0.01, max_tol=0.06):
    errs = O.centred_logit_err(ref, got, [3] * n_q)
    assert errs.mean() <= mean_tol and errs.max() <= max_tol, (errs.mean(), errs.max())
    assert O.top_flips(ref, got, [3] * n_q) == 0
    return errs


def test_config0_vs_fp32_oracle(model, batch0, oracle_f32):
    got = model(batch0)
    assert got.shape == oracle_f32.shape and np.isfinite(got).all()
    assert_bar(oracle_f32, got, len(batch0))


def test_config0_vs_reference_engine(pkg, gpu_lib, ref_lib, weights, model, batch0, oracle_f32):
    from conftest import REF_LIB
    from fast_d1_omni_b200.model import TextModel
    ref = TextModel(weights, kernel_lib=str(REF_LIB), fused=False, cap_tokens=4096)
    try:
        ref_logits = ref(batch0)
    finally:
        ref.close()
    assert_bar(oracle_f32, ref_logits, len(batch0))   # the reference engine meets the bar itself
    assert_bar(ref_logits, model(batch0), len(batch0))


def test_fused_equals_unfused(weights, model, batch0, gpu_lib):
    from fast_d1_omni_b200.model import TextModel
    un = TextModel(weights, fused=False, cap_tokens=4096)
    try:
        a = un(batch0)
    finally:
        un.close()
    assert_bar(a, model(batch0), len(batch0), 0.005, 0.03)


def test_batching_invariance(model, batch0):
    """A burst packed differently must answer like the sequential runs (tests/e2e.py:163-180)."""
    whole = model(batch0)
    parts = np.concatenate([model(batch0[i:i + 1]) for i in range(len(batch0))])
    rev = model(batch0[::-1])
    rev = np.concatenate([rev[3 * i:3 * i + 3] for i in reversed(range(len(batch0)))])
    assert_bar(whole, parts, len(batch0), 0.005, 0.03)
    assert_bar(whole, rev, len(batch0), 0.005, 0.03)


def test_ragged_lengths_vs_oracle(weights, model):
    from fast_d1_omni_b200.weights import text_batch
    b = text_batch(5, 0, lengths=[1, 2, 63, 64, 65, 300, 17])
    for s in b:  # 1-token and 2-token rows carry fewer markers
        s["markers"] = s["markers"][:len(s["ids"])]
    got = model(b)
    ref = O.launch_text(weights, b, "f32")
    sizes = [len(s["markers"]) for s in b]
    errs = O.centred_logit_err(ref, got, sizes)
    assert errs.mean() <= 0.01 and errs.max() <= 0.06


def test_media_prefix(pkg, weights, model):
    """Media prefix pass + text over the cached prefix (src/model.rs:402-459, 511-528) against the oracle."""
    from fast_d1_omni_b200.weights import text_batch
    rng = np.random.default_rng(21)
    plen = 200
    emb = (rng.standard_normal((plen, 1024)) * 0.02).astype(np.float32)
    pc = model.prefix_alloc(plen)
    model.launch_prefix([(torch.from_numpy(emb).cuda(), pc)])
    b = text_batch(22, 2, 50)
    b[0]["prefix"] = pc
    got = model(b)
    cache = O.launch_prefix(weights, [emb], "f32")[0]
    ob = [dict(b[0], prefix=cache), dict(b[1])]
    ref = O.launch_text(weights, ob, "f32")
    model.prefix_free(pc)
    torch.cuda.synchronize()
    assert_bar(ref, got, 2)
