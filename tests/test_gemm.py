"""tcgen05 GEMM parity through the C ABI (d1_lt_gemm, d1_gemm_swiglu, d1_gemm_bias_act) against an fp32
reference GEMM of the same fp16 inputs ("each GEMM is checked against an fp32 host GEMM").

Tolerances: fp16 outputs within 1 fp16 ulp of the fp32 result plus accumulation-order noise
(|err| <= 2^-10 |ref| + 2e-3 * rms(ref)); fp32 outputs within 1e-4 * max|ref| (fp32 accumulation in a
different order than the reference GEMM).
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

CONFIG1_NK = [(3072, 1024), (2048, 1024), (1024, 1024), (9216, 1024), (1024, 4608)]


def _p(t):
    return C.c_void_p(t.data_ptr())


def ref_gemm(x, w):
    return x.double() @ w.double().T


def check_f16(y, ref):
    ref = ref.float()
    err = (y.float() - ref).abs()
    tol = ref.abs() * 2.0 ** -10 + 2e-3 * ref.pow(2).mean().sqrt()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{bad} elements off, max err {err.max().item():.3e}"


@pytest.fixture(scope="module")
def ctx(gpu_lib):
    c = gpu_lib.d1_lt_init(32 << 20)
    assert c, "d1_lt_init failed"
    yield c
    assert gpu_lib.d1_lt_error(c) == 0
    gpu_lib.d1_lt_destroy(c)


def run_gemm(lib, ctx, x, w, y, alpha=1.0, beta=0.0):
    M, K = x.shape
    N = w.shape[0]
    y_f32 = int(y.dtype == torch.float32)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    r = lib.d1_lt_gemm(ctx, M, N, K, _p(x), x.stride(0), _p(w), w.stride(0), 0, _p(y), y.stride(0), y_f32, 0,
                       alpha, beta, st)
    assert r == 0
    torch.cuda.synchronize()
    assert lib.d1_lt_error(ctx) == 0


CONFIG1_M = [256, 1024, 4096, 8192, 16384]
# tile configurations a plan can name (csrc/gemm.cu Cfg): 1-SM 128/256/64-column tiles, CTA pair 256x256 / 256x128
CFGS = {0: "1sm_128", 1: "1sm_256", 2: "pair_256", 3: "pair_128", 4: "1sm_64"}


@pytest.mark.gpu
@pytest.mark.parametrize("N,K", CONFIG1_NK)
@pytest.mark.parametrize("M", CONFIG1_M)
def test_config1_f16_out(gpu_lib, ctx, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    y = torch.empty(M, N, device="cuda", dtype=torch.float16)
    run_gemm(gpu_lib, ctx, x, w, y)
    check_f16(y, ref_gemm(x, w))


def _forced_ctx(lib, tmp_path, M, N, K, ldy, y_f32, cfg, split):
    """A fresh context whose only plan runs (N, K) at M's bucket with tile configuration `cfg` and split-K `split`
    (written in d1_lt_save's format and read back by d1_lt_load)."""
    c = lib.d1_lt_init(0)
    assert c
    path = tmp_path / f"plan_{cfg}_{split}_{y_f32}.txt"
    path.write_text(f"d1b200-gemm-plans v1 {lib.d1_build_id().decode()}\n"
                    f"{N} {K} {K} {K} {ldy} 0 {y_f32} 0 {lib.d1_lt_bucket(M)} {cfg} {split} 1.0\n")
    assert lib.d1_lt_load(c, str(path).encode()) == 1
    return c


@pytest.mark.gpu
@pytest.mark.parametrize("N,K", CONFIG1_NK)
@pytest.mark.parametrize("M", CONFIG1_M)
def test_config1_every_plan(gpu_lib, tmp_path, M, N, K):
    """BASELINE config 1 under every tile configuration the tuner can pick (the tuned plan of a shape depends on
    the timing of the GPU it runs on): the fp16 store form, and for the residual projections (N = 1024) the trunk's
    fp32 reduce-add form Y += X.W^T with split-K 1, 2 and 4."""
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    ref = ref_gemm(x, w)
    y0 = torch.randn(M, N, device="cuda", generator=g) if N == 1024 else None
    for cfg in CFGS:
        c = _forced_ctx(gpu_lib, tmp_path, M, N, K, N, 0, cfg, 1)
        try:
            y = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float16)
            run_gemm(gpu_lib, c, x, w, y)
            assert gpu_lib.d1_lt_error(c) == 0
            check_f16(y, ref)
        finally:
            gpu_lib.d1_lt_destroy(c)
        if y0 is None:
            continue
        for split in (1, 2, 4):
            c = _forced_ctx(gpu_lib, tmp_path, M, N, K, N, 1, cfg, split)
            try:
                y = y0.clone()
                run_gemm(gpu_lib, c, x, w, y, 1.0, 1.0)
                assert gpu_lib.d1_lt_error(c) == 0
                want = ref + y0.double()
                err = (y.double() - want).abs().max().item()
                assert err <= 1e-4 * want.abs().max().item(), (CFGS[cfg], split, err)
            finally:
                gpu_lib.d1_lt_destroy(c)


@pytest.mark.gpu
@pytest.mark.parametrize("N,K", [(1024, 1024), (1024, 4608)])
@pytest.mark.parametrize("M", [1, 3, 127, 129, 512, 1000, 4096, 16384])
def test_residual_f32(gpu_lib, ctx, M, N, K):
    """The trunk's residual projections: Y32 = X.W^T + Y32 (beta = 1, src/model.rs:373,390,396)."""
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    y0 = torch.randn(M, N, device="cuda", generator=g)
    y = y0.clone()
    run_gemm(gpu_lib, ctx, x, w, y, 1.0, 1.0)
    ref = ref_gemm(x, w) + y0.double()
    err = (y.double() - ref).abs().max().item()
    assert err <= 1e-4 * ref.abs().max().item(), err


@pytest.mark.gpu
def test_alpha_beta_general(gpu_lib, ctx):
    """alpha/beta as the audio half-step FFN uses them (alpha 0.5, beta 1, src/audio.rs:553) and fp16 beta."""
    g = torch.Generator(device="cuda").manual_seed(3)
    M, N, K = 300, 512, 2048
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    y0 = torch.randn(M, N, device="cuda", generator=g)
    y = y0.clone()
    run_gemm(gpu_lib, ctx, x, w, y, 0.5, 1.0)
    ref = 0.5 * ref_gemm(x, w) + y0.double()
    assert (y.double() - ref).abs().max().item() <= 1e-4 * ref.abs().max().item()
    yh0 = torch.randn(M, N, device="cuda", generator=g).half()
    yh = yh0.clone()
    run_gemm(gpu_lib, ctx, x, w, yh, 1.0, 0.5)
    check_f16(yh, ref_gemm(x, w) + 0.5 * yh0.double())


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(77, 200, 136), (130, 1000, 1000), (5, 40, 72), (777, 1000, 1000), (600, 96, 4608)])
def test_ragged_shapes(gpu_lib, ctx, M, N, K):
    """N and K that are not tile multiples (TMA zero fill on loads, masked epilogue stores)."""
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    y = torch.full((M, N), 7.0, device="cuda", dtype=torch.float16)
    run_gemm(gpu_lib, ctx, x, w, y)
    check_f16(y, ref_gemm(x, w))


@pytest.mark.gpu
def test_strided_views(gpu_lib, ctx):
    """Column-offset views into a wider buffer, as the runner passes big.add(D) etc. (src/model.rs:383)."""
    g = torch.Generator(device="cuda").manual_seed(5)
    M, N, K = 512, 1024, 1024
    xb = torch.randn(M, 3 * K, device="cuda", generator=g).half()
    x = xb[:, K:2 * K]
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    yb = torch.zeros(M, 2 * N, device="cuda", dtype=torch.float16)
    y = yb[:, N:]
    run_gemm(gpu_lib, ctx, x, w, y)
    check_f16(y, ref_gemm(x, w))
    assert yb[:, :N].abs().max().item() == 0


@pytest.mark.gpu
def test_wkn_layout(gpu_lib, ctx):
    """W given as [K, N] (w_kn = 1, cuda/gemm.cu:63-71)."""
    g = torch.Generator(device="cuda").manual_seed(6)
    M, N, K = 100, 64, 96
    x = torch.randn(M, K, device="cuda", generator=g).half()
    wkn = (torch.randn(K, N, device="cuda", generator=g) * 0.05).half()
    y = torch.empty(M, N, device="cuda", dtype=torch.float32)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert gpu_lib.d1_lt_gemm(ctx, M, N, K, _p(x), K, _p(wkn), N, 1, _p(y), N, 1, 0, 1.0, 0.0, st) == 0
    torch.cuda.synchronize()
    ref = x.double() @ wkn.double()
    assert (y.double() - ref).abs().max().item() <= 1e-4 * ref.abs().max().item()


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 200, 256, 1024, 4096, 8192, 16384])
def test_swiglu_fused(gpu_lib, ctx, M):
    """d1_gemm_swiglu == d1_lt_gemm(N = 2F) + d1_swiglu (src/model.rs:394-395)."""
    g = torch.Generator(device="cuda").manual_seed(7)
    F, K = 4608, 1024
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(2 * F, K, device="cuda", generator=g) * 0.02).half()
    out = torch.empty(M, F, device="cuda", dtype=torch.float16)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert gpu_lib.d1_gemm_swiglu(ctx, M, F, K, _p(x), K, _p(w), K, _p(out), F, st) == 0
    # unfused path of the same library
    gu = torch.empty(M, 2 * F, device="cuda", dtype=torch.float16)
    run_gemm(gpu_lib, ctx, x, w, gu)
    out2 = torch.empty(M, F, device="cuda", dtype=torch.float16)
    assert gpu_lib.d1_swiglu(_p(gu), _p(out2), M, F, st) == 0
    torch.cuda.synchronize()
    assert gpu_lib.d1_lt_error(ctx) == 0
    ref = ref_gemm(x, w)
    gg, uu = ref[:, :F], ref[:, F:]
    sig = torch.sigmoid(gg)
    exact = gg * sig * uu
    # g and u are rounded to fp16 before the gate (as the reference stores them): allow one fp16 ulp on each,
    # propagated through silu(g) * u, plus the final rounding of the product.
    slack = 2.0 ** -10 * ((sig * (1 + gg * (1 - sig)) * gg * uu).abs() + (gg * sig * uu).abs())
    err = (out.double() - exact).abs()
    # plus fp32 accumulation noise over K (~1e-6 absolute near zero)
    assert (err <= 2 * slack + 2.0 ** -10 * exact.abs() + 2e-5).all(), err.max().item()
    # fused vs unfused: identical up to the rounding of g and u (1 fp16 ulp on either side)
    d = (out.float() - out2.float()).abs()
    assert (d <= out2.float().abs() * 2.0 ** -9 + 1e-3).all()


@pytest.mark.gpu
@pytest.mark.parametrize("act", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("M", [333, 1000])
def test_bias_act_fused(gpu_lib, ctx, act, M):
    """d1_gemm_bias_act == d1_lt_gemm(fp16) + d1_bias_act_h (src/model.rs:568-569); M 333 runs the single-SM
    kernel, M 1000 the CTA-pair kernel."""
    g = torch.Generator(device="cuda").manual_seed(8 + act)
    N, K = 2048, 1024
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    b = torch.randn(N, device="cuda", generator=g) * 0.1
    y = torch.empty(M, N, device="cuda", dtype=torch.float16)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert gpu_lib.d1_gemm_bias_act(ctx, M, N, K, _p(x), K, _p(w), K, _p(b), act, _p(y), N, st) == 0
    y2 = torch.empty(M, N, device="cuda", dtype=torch.float16)
    run_gemm(gpu_lib, ctx, x, w, y2)
    assert gpu_lib.d1_bias_act_h(_p(y2), _p(b), M, N, act, st) == 0
    torch.cuda.synchronize()
    d = (y.float() - y2.float()).abs()
    assert (d <= y2.float().abs() * 2.0 ** -9 + 2e-3).all(), d.max().item()


@pytest.mark.gpu
def test_tune_save_load(gpu_lib, ctx, tmp_path):
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    us = gpu_lib.d1_lt_tune(ctx, 1000, 1024, 1024, 1024, 1024, 0, 1024, 1, 0, 1, st)
    assert us > 0
    assert gpu_lib.d1_lt_bucket(1000) == 1024
    path = str(tmp_path / "plans.txt").encode()
    assert gpu_lib.d1_lt_save(ctx, path) == 0
    c2 = gpu_lib.d1_lt_init(0)
    assert gpu_lib.d1_lt_load(c2, path) >= 1
    gpu_lib.d1_lt_destroy(c2)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [300, 8192])
def test_qk_norm_rope_fused(pkg, gpu_lib, ctx, M):
    """d1_gemm_qk_norm_rope == d1_lt_gemm(fp16) + d1_qk_norm_rope (src/model.rs:376-381) on ragged sequences with
    position offsets (text after a media prefix); M 300 runs the small-tile kernel, M 8192 the 256-column one. The
    epilogue repeats the kernel's arithmetic on the same fp16-rounded GEMM output, so the two agree to within one
    fp16 rounding (different instruction scheduling may contract one multiply-add differently); both against the
    oracle's fp32 QK-norm + RoPE of that output."""
    from oracle import d1_oracle as O
    rng = np.random.default_rng(20 + M)
    H, KVH, K = 16, 8, 1024
    N = (H + 2 * KVH) * 64
    lens = [M // 3, M // 3 + 5, M - 2 * (M // 3) - 5]
    pos_off = [0, 77, 4000]
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float16)).cuda()
    w = torch.from_numpy((rng.standard_normal((N, K)) * 0.03).astype(np.float16)).cuda()
    qn = torch.from_numpy(rng.uniform(0.5, 1.5, 64).astype(np.float32)).cuda()
    kn = torch.from_numpy(rng.uniform(0.5, 1.5, 64).astype(np.float32)).cuda()
    rope_np = O.rope_table(1e6)
    rope = torch.from_numpy(np.ascontiguousarray(rope_np, np.float32)).cuda()
    arr = (pkg.abi.SeqInfo * len(lens))()
    s = 0
    for i, n in enumerate(lens):
        arr[i].start, arr[i].len, arr[i].pos_off = s, n, pos_off[i]
        s += n
    seqs = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).cuda()
    tok = torch.from_numpy(np.concatenate([np.full(n, i, np.int32) for i, n in enumerate(lens)])).cuda()
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    y = torch.empty(M, N, device="cuda", dtype=torch.float16)
    assert gpu_lib.d1_gemm_qk_norm_rope(ctx, M, K, _p(x), K, _p(w), K, _p(y), N, H, KVH, _p(qn), _p(kn), _p(rope),
                                        _p(tok), _p(seqs), 1e-5, st) == 0
    y2 = torch.empty(M, N, device="cuda", dtype=torch.float16)
    run_gemm(gpu_lib, ctx, x, w, y2)
    raw = y2.float().cpu().numpy()
    assert gpu_lib.d1_qk_norm_rope(_p(y2), N, H, KVH, _p(qn), _p(kn), _p(rope), _p(tok), _p(seqs), 0, M, 1e-5,
                                   st) == 0
    torch.cuda.synchronize()
    assert gpu_lib.d1_lt_error(ctx) == 0
    a, b = y.float().cpu().numpy(), y2.float().cpu().numpy()
    assert np.abs(a - b).max() <= 2.0 ** -10 * np.abs(b).max() + 1e-6 or \
        (np.abs(a - b) <= np.abs(b) * 2.0 ** -10 + 1e-4).all()
    assert np.array_equal(a[:, (H + KVH) * 64:], raw[:, (H + KVH) * 64:])  # value heads: the GEMM output
    pos = np.concatenate([np.arange(n) + po for n, po in zip(lens, pos_off)])
    want = O.qk_norm_rope(raw, H, KVH, qn.cpu().numpy(), kn.cpu().numpy(), rope_np, pos, 1e-5)
    assert (np.abs(a - want) <= np.abs(want) * 2.0 ** -10 + 2e-4).all()
