"""Vision encoder (SigLIP2 tower + 2x2 pixel-unshuffle projector, src/vision.rs:305-385) through the runner and
the C ABI, against the fp32 oracle and against the reference's own kernels (oracle/_ref/libd1ref.so: its kernels
and cuBLASLt GEMMs) run through the same host runner.

random-init weights seed 3, 16 images with sides uniform in 224-768 px rounded to multiples of
32, pixels uniform in [0, 1] fed directly as patches, all crops packed into one varlen batch (14,632 patches).
Tolerance: relative RMS error of the fp32 output embeddings, <= 1e-2 against the fp32 oracle (the engines keep
fp16 activations through 12 layers, as the reference does) and <= 1e-2 between this engine and the reference's.
"""
import numpy as np
import pytest

from oracle import d1_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def rel_rms(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.sqrt(((got - ref) ** 2).mean()) / np.sqrt((ref ** 2).mean()))


@pytest.fixture(scope="module")
def vw(pkg):
    from fast_d1_omni_b200.weights import vision_weights
    return vision_weights(3)


@pytest.fixture(scope="module")
def vmodel(pkg, gpu_lib, vw):
    from fast_d1_omni_b200.model import VisionModel
    m = VisionModel(vw, max_patches=16384)
    yield m
    m.close()


def small_crops():
    rng = np.random.default_rng(30)
    return [(ph, pw, rng.uniform(0, 1, (ph * pw, 768)).astype(np.float16)) for ph, pw in [(4, 6), (2, 2), (8, 10)]]


def test_small_vs_oracle(vmodel, vw):
    crops = small_crops()
    got = vmodel.encode(crops).cpu().numpy()
    ref = O.vision_encode(vw, crops, "f32")
    assert got.shape == ref.shape == (6 + 1 + 20, 1024)
    assert np.isfinite(got).all()
    assert rel_rms(got, ref) <= 1e-2


def test_small_vs_reference_engine(pkg, ref_lib, vmodel, vw):
    from conftest import REF_LIB
    from fast_d1_omni_b200.model import VisionModel
    crops = small_crops()
    ref_m = VisionModel(vw, kernel_lib=str(REF_LIB), fused=False, max_patches=4096)
    try:
        ref = ref_m.encode(crops).cpu().numpy()
    finally:
        ref_m.close()
    assert rel_rms(vmodel.encode(crops).cpu().numpy(), ref) <= 1e-2
    assert rel_rms(ref, O.vision_encode(vw, crops, "f32")) <= 1e-2


def test_unfused_equals_fused(pkg, vmodel, vw):
    from fast_d1_omni_b200.model import VisionModel
    crops = small_crops()
    un = VisionModel(vw, fused=False, max_patches=4096)
    try:
        a = un.encode(crops).cpu().numpy()
    finally:
        un.close()
    assert rel_rms(vmodel.encode(crops).cpu().numpy(), a) <= 5e-3


def test_config3(pkg, ref_lib, vmodel, vw):
    from conftest import REF_LIB
    from fast_d1_omni_b200.model import VisionModel
    from fast_d1_omni_b200.weights import vision_crops
    crops = vision_crops(3)
    assert sum(ph * pw for ph, pw, _ in crops) == 14632
    got = vmodel.encode(crops).cpu().numpy()
    ref_m = VisionModel(vw, kernel_lib=str(REF_LIB), fused=False, max_patches=16384)
    try:
        ref = ref_m.encode(crops).cpu().numpy()
    finally:
        ref_m.close()
    assert np.isfinite(got).all()
    assert rel_rms(got, ref) <= 1e-2
    # the fp32 oracle on the first 4 crops (a packed batch gives each crop the same result as alone)
    want = O.vision_encode(vw, crops[:4], "f32")
    assert rel_rms(got[:want.shape[0]], want) <= 1e-2


@pytest.mark.parametrize("ph,pw", [(14, 22), (2, 2), (48, 48), (16, 16), (4, 40)])
def test_vision_pos_kernel_bit_exact(gpu_lib, vw, ph, pw):
    """d1_vision_pos (the GPU form of src/vision.rs:263-302) against the oracle's restatement: same fp32 order."""
    import ctypes as C
    taps_y, taps_x = O.aa_weights(16, ph), O.aa_weights(16, pw)
    taps = max(len(w) for _, w in taps_y + taps_x)
    spans = np.array([[s, len(w)] for s, w in taps_y + taps_x], np.int32)
    wts = np.zeros((ph + pw, taps), np.float32)
    for r, (_, w) in enumerate(taps_y + taps_x):
        wts[r, :len(w)] = w
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    grid, pb, sp, wt = d(np.asarray(vw["pos"], np.float32)), d(vw["patch_b"]), d(spans), d(wts)
    out = torch.full((ph * pw, 768), float("nan"), device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    assert gpu_lib.d1_vision_pos(P(grid), P(pb), P(sp), P(wt), taps, ph, pw, 768, P(out),
                                 C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    assert np.array_equal(out.cpu().numpy(), O.vision_pos(vw["pos"], vw["patch_b"], ph, pw))
