"""Parity of the HBM-bound kernels through the C ABI: each against the oracle (oracle/d1_oracle.py) and against
the reference's own kernel (oracle/_ref/libd1ref.so) on the same seeded inputs.

Bit-exact where this library keeps the reference's arithmetic per element (swiglu, bias+act, short conv,
unshuffle, gathers, the audio kernels); within one fp16 rounding step where a reduction runs in a different
order (the norms, QK-norm, the scorer's dot product)."""
import ctypes as C

import numpy as np
import pytest

from conftest import half_ulp_close
from oracle import d1_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def P(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def ST():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


_KEEP = []  # device copies stay alive until the test ends (a freed temporary's block is reused at once)


@pytest.fixture(autouse=True)
def _release_inputs():
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


def cu(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    t = t.cuda()
    _KEEP.append(t)
    return t


def np_(t):
    torch.cuda.synchronize()
    return t.float().cpu().numpy()


def libs(gpu_lib, ref_lib):
    return [("d1", gpu_lib), ("ref", ref_lib)]


@pytest.mark.parametrize("D", [512, 768, 1024])
@pytest.mark.parametrize("rows", [1, 7, 300])
def test_rmsnorm(gpu_lib, ref_lib, D, rows):
    rng = np.random.default_rng(D + rows)
    x = rng.standard_normal((rows, D)).astype(np.float32) * 3
    w = rng.standard_normal(D).astype(np.float32)
    ref = O.rmsnorm(x, w, 1e-5)
    outs = {}
    for name, lib in libs(gpu_lib, ref_lib):
        y = torch.empty(rows, D, dtype=torch.float16, device="cuda")
        assert lib.d1_rmsnorm(P(cu(x)), P(cu(w)), P(y), rows, D, 1e-5, ST()) == 0
        outs[name] = np_(y)
        assert half_ulp_close(outs[name], ref, 2.0 ** -10, 1e-4).all(), name
    assert half_ulp_close(outs["d1"], outs["ref"], 2.0 ** -10, 1e-4).all()


@pytest.mark.parametrize("D", [512, 768, 1024])
@pytest.mark.parametrize("pend", [False, True])
def test_layernorm(gpu_lib, ref_lib, D, pend):
    rng = np.random.default_rng(D)
    rows = 130
    x = rng.standard_normal((rows, D)).astype(np.float32) + 0.5
    pb = rng.standard_normal(D).astype(np.float32) if pend else None
    w = rng.standard_normal(D).astype(np.float32)
    b = rng.standard_normal(D).astype(np.float32)
    x_new, ref = O.layernorm(x, w, b, 1e-5, pb, 0.5)
    for name, lib in libs(gpu_lib, ref_lib):
        xd = cu(x)
        y = torch.empty(rows, D, dtype=torch.float16, device="cuda")
        yf = torch.empty(rows, D, dtype=torch.float32, device="cuda")
        assert lib.d1_layernorm(P(xd), P(cu(pb)) if pend else None, 0.5, P(cu(w)), P(cu(b)), P(y), P(yf), rows, D,
                                1e-5, ST()) == 0
        assert np.allclose(np_(xd), x_new, atol=1e-6), name
        assert half_ulp_close(np_(y), ref, 2.0 ** -10, 1e-4).all(), name
        assert np.allclose(np_(yf), ref, rtol=1e-5, atol=1e-5), name
        # fp32 output in place (yf aliases x), as the conformer's norm_out does (src/audio.rs:575)
        xd = cu(x)
        assert lib.d1_layernorm(P(xd), P(cu(pb)) if pend else None, 0.5, P(cu(w)), P(cu(b)), None, P(xd), rows, D,
                                1e-5, ST()) == 0
        assert np.allclose(np_(xd), ref, rtol=1e-5, atol=1e-5), name


def _seqinfo(pkg, spans, qtypes=None, pos_off=None, ext_bx=None, save_bx=None, save_k=None, save_v=None):
    arr = (pkg.abi.SeqInfo * len(spans))()
    for i, (s, n) in enumerate(spans):
        arr[i].start, arr[i].len = s, n
        arr[i].qtype = qtypes[i] if qtypes else 0
        arr[i].pos_off = pos_off[i] if pos_off else 0
        if ext_bx and ext_bx[i] is not None:
            arr[i].ext_bx = ext_bx[i]
        if save_bx and save_bx[i] is not None:
            arr[i].save_bx = save_bx[i]
        if save_k and save_k[i] is not None:
            arr[i].save_k, arr[i].save_v = save_k[i], save_v[i]
    t = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).cuda()
    tok = np.concatenate([np.full(n, i, np.int32) for i, (s, n) in enumerate(spans)])
    return t, cu(tok)


def test_head_init(pkg, gpu_lib, ref_lib):
    rng = np.random.default_rng(3)
    spans = [(0, 5), (5, 1), (6, 90)]
    T = 96
    h = rng.standard_normal((T, 1024)).astype(np.float32)
    w = rng.standard_normal(1024).astype(np.float32)
    te = rng.standard_normal((4, 1024)).astype(np.float32)
    qt = [2, 0, 3]
    seqs, tok = _seqinfo(pkg, spans, qtypes=qt)
    ref = O.head_init(h, w, te, np.repeat(qt, [n for _, n in spans]), 1e-5)
    for name, lib in libs(gpu_lib, ref_lib):
        hd = cu(h)
        assert lib.d1_head_init(P(hd), P(cu(w)), P(cu(te)), P(tok), P(seqs), P(hd), T, 1e-5, ST()) == 0
        assert np.allclose(np_(hd), ref, rtol=2e-6, atol=2e-6), name


def test_embed_gather_unshuffle(gpu_lib, ref_lib):
    rng = np.random.default_rng(4)
    table = rng.standard_normal((500, 1024)).astype(np.float16)
    ids = rng.integers(0, 500, 77).astype(np.int32)
    src = rng.standard_normal((40, 3072)).astype(np.float16)
    idx = np.array([3, 0, 39, 39, 7], np.int32)
    ph, pw, Cc = 6, 8, 768
    x = rng.standard_normal((ph * pw, Cc)).astype(np.float16)
    for name, lib in libs(gpu_lib, ref_lib):
        h = torch.empty(77, 1024, device="cuda")
        assert lib.d1_embed(P(cu(table)), P(cu(ids)), P(h), 77, 1024, ST()) == 0
        assert np.array_equal(np_(h), table.astype(np.float32)[ids]), name
        dst = torch.empty(5, 3072, dtype=torch.float16, device="cuda")
        assert lib.d1_gather_rows(P(cu(src)), P(dst), P(cu(idx)), 5, 3072 * 2, ST()) == 0
        assert np.array_equal(np_(dst), src.astype(np.float32)[idx]), name
        out = torch.empty(ph * pw // 4, 4 * Cc, dtype=torch.float16, device="cuda")
        assert lib.d1_unshuffle(P(cu(x)), P(out), ph, pw, Cc, ST()) == 0
        assert np.array_equal(np_(out), O.unshuffle(x, ph, pw, Cc).astype(np.float32)), name


@pytest.mark.parametrize("F", [4608, 12])
def test_swiglu(gpu_lib, ref_lib, F):
    rng = np.random.default_rng(F)
    rows = 65
    gu = (rng.standard_normal((rows, 2 * F)) * 2).astype(np.float16)
    ref = O.swiglu(gu.astype(np.float32), F)
    outs = {}
    for name, lib in libs(gpu_lib, ref_lib):
        out = torch.empty(rows, F, dtype=torch.float16, device="cuda")
        assert lib.d1_swiglu(P(cu(gu)), P(out), rows, F, ST()) == 0
        outs[name] = np_(out)
        assert half_ulp_close(outs[name], ref, 2.0 ** -10, 1e-6).all(), name
    assert np.array_equal(outs["d1"], outs["ref"])


@pytest.mark.parametrize("act", [0, 1, 2, 3, 4])
def test_bias_act(gpu_lib, ref_lib, act):
    rng = np.random.default_rng(act)
    rows, N = 33, 2048
    x = (rng.standard_normal((rows, N)) * 2).astype(np.float16)
    b = rng.standard_normal(N).astype(np.float32)
    xf = rng.standard_normal((rows, N)).astype(np.float32)
    ref = O.bias_act(x.astype(np.float32), b, act)
    outs = {}
    for name, lib in libs(gpu_lib, ref_lib):
        xd = cu(x)
        assert lib.d1_bias_act_h(P(xd), P(cu(b)), rows, N, act, ST()) == 0
        outs[name] = np_(xd)
        assert half_ulp_close(outs[name], ref, 2.0 ** -10, 1e-5).all(), name
        xfd = cu(xf)
        assert lib.d1_bias_act_f(P(xfd), P(cu(b)), rows, N, act, ST()) == 0
        assert np.allclose(np_(xfd), O.bias_act(xf, b, act), rtol=1e-6, atol=1e-6), name
    assert np.array_equal(outs["d1"], outs["ref"])


def test_fill_rows_and_cast(gpu_lib, ref_lib):
    rng = np.random.default_rng(5)
    rows, N = 19, 512
    b = rng.standard_normal(N).astype(np.float32)
    add = rng.standard_normal((rows, N)).astype(np.float32)
    for name, lib in libs(gpu_lib, ref_lib):
        out = torch.empty(rows, N, device="cuda")
        assert lib.d1_fill_rows(P(out), P(cu(b)), P(cu(add)), rows, N, ST()) == 0
        assert np.array_equal(np_(out), b + add), name
        y = torch.empty(rows * N, dtype=torch.float16, device="cuda")
        assert lib.d1_f32_to_f16(P(cu(add)), P(y), rows * N, ST()) == 0
        assert np.array_equal(np_(y), add.reshape(-1).astype(np.float16).astype(np.float32)), name


@pytest.mark.parametrize("ext", [False, True])
def test_shortconv(pkg, gpu_lib, ref_lib, ext):
    """Ragged packed sequences (1, 2, 17, 16, 33, 64 rows: boundaries inside and at the edges of the 16-row
    runs), the prefix's left state (ext_bx) and the saved last state (save_bx), conv_idx 3 of 10."""
    rng = np.random.default_rng(6)
    Dm = 1024
    lens = [1, 2, 17, 16, 33, 64]
    spans, s = [], 0
    for n in lens:
        spans.append((s, n))
        s += n
    T = s
    bcu = (rng.standard_normal((T, 3 * Dm)) * 1.5).astype(np.float16)
    convw = (rng.standard_normal((Dm, 3)) * 0.5).astype(np.float32)
    conv_idx, n_conv = 3, 10
    ext_np = [(rng.standard_normal((n_conv, Dm)) * 0.5).astype(np.float16) if ext else None for _ in lens]
    ref, saved = O.shortconv(bcu.astype(np.float32), convw, spans, conv_idx,
                             [e[conv_idx].astype(np.float32) if e is not None else None for e in ext_np])
    outs = {}
    for name, lib in libs(gpu_lib, ref_lib):
        ext_d = [cu(e) if e is not None else None for e in ext_np]
        save_d = [torch.zeros(n_conv, Dm, dtype=torch.float16, device="cuda") for _ in lens]
        seqs, tok = _seqinfo(pkg, spans, ext_bx=[e.data_ptr() if e is not None else None for e in ext_d],
                             save_bx=[t.data_ptr() for t in save_d])
        out = torch.empty(T, Dm, dtype=torch.float16, device="cuda")
        assert lib.d1_shortconv(P(cu(bcu)), P(cu(convw)), P(tok), P(seqs), P(out), T, Dm, conv_idx, ST()) == 0
        outs[name] = np_(out)
        assert half_ulp_close(outs[name], ref, 2.0 ** -10, 1e-5).all(), name
        for i in range(len(lens)):
            assert np.array_equal(np_(save_d[i])[conv_idx], saved[i]), (name, i)
    assert np.array_equal(outs["d1"], outs["ref"])


@pytest.mark.parametrize("save", [False, True])
def test_qk_norm_rope(pkg, gpu_lib, ref_lib, save):
    rng = np.random.default_rng(7)
    spans = [(0, 3), (3, 40), (43, 1)]
    pos_off = [0, 100, 16000]
    T, ld, H, KVH = 44, 2048, 16, 8
    qkv = rng.standard_normal((T, ld)).astype(np.float16)
    qn = rng.standard_normal(64).astype(np.float32)
    kn = rng.standard_normal(64).astype(np.float32)
    rope = O.rope_table(1e6)
    pos = np.concatenate([np.arange(n) + po for (s, n), po in zip(spans, pos_off)])
    ref = O.qk_norm_rope(qkv.astype(np.float32), H, KVH, qn, kn, rope, pos, 1e-5)
    attn_idx, n_attn = 2, 6
    outs = {}
    for name, lib in libs(gpu_lib, ref_lib):
        sk = [torch.zeros(n_attn, n, 512, dtype=torch.float16, device="cuda") for _, n in spans] if save else None
        sv = [torch.zeros(n_attn, n, 512, dtype=torch.float16, device="cuda") for _, n in spans] if save else None
        seqs, tok = _seqinfo(pkg, spans, pos_off=pos_off,
                             save_k=[t.data_ptr() for t in sk] if save else None,
                             save_v=[t.data_ptr() for t in sv] if save else None)
        d = cu(qkv)
        assert lib.d1_qk_norm_rope(P(d), ld, H, KVH, P(cu(qn)), P(cu(kn)), P(cu(rope)), P(tok), P(seqs), attn_idx, T,
                                   1e-5, ST()) == 0
        outs[name] = np_(d)
        assert half_ulp_close(outs[name], ref, 2.0 ** -10, 2e-4).all(), name
        if save:
            for i, (s, n) in enumerate(spans):
                assert np.array_equal(np_(sk[i])[attn_idx], outs[name][s:s + n, 1024:1536]), name
                assert np.array_equal(np_(sv[i])[attn_idx], qkv[s:s + n, 1536:].astype(np.float32)), name
    assert half_ulp_close(outs["d1"], outs["ref"], 2.0 ** -10, 2e-4).all()


def test_scorer_out(gpu_lib, ref_lib):
    rng = np.random.default_rng(8)
    rows, Dm = 37, 1024
    x = rng.standard_normal((rows, Dm)).astype(np.float16)
    b1 = rng.standard_normal(Dm).astype(np.float32)
    w2 = (rng.standard_normal(Dm) * 0.05).astype(np.float16)
    ref = O.scorer_out(x.astype(np.float32), b1, w2.astype(np.float32), 0.25)
    for name, lib in libs(gpu_lib, ref_lib):
        out = torch.empty(rows, device="cuda")
        assert lib.d1_scorer_out(P(cu(x)), P(cu(b1)), P(cu(w2)), 0.25, P(out), rows, Dm, ST()) == 0
        assert np.allclose(np_(out), ref, rtol=1e-5, atol=1e-5), name


def test_audio_kernels(gpu_lib, ref_lib):
    """FastConformer pieces (cuda/kernels.cu:529-637) on a 3 s clip's shapes, against the reference's kernels."""
    rng = np.random.default_rng(9)
    Tin, Fm = 301, 128
    l1 = (Tin - 1) // 2 + 1
    mel = rng.standard_normal((Tin, Fm)).astype(np.float32)
    w0 = rng.standard_normal((256, 9)).astype(np.float32) * 0.3
    b0 = rng.standard_normal(256).astype(np.float32) * 0.1
    w2 = rng.standard_normal((256, 9)).astype(np.float32) * 0.3
    T, Dm = 38, 512
    qkv = rng.standard_normal((T, 3 * Dm)).astype(np.float16)
    vecs = [rng.standard_normal(Dm).astype(np.float32) * 0.1 for _ in range(5)]
    ac = rng.standard_normal((8, T, T)).astype(np.float32)
    bd = rng.standard_normal((8, T, 2 * T - 1)).astype(np.float32)
    a2 = rng.standard_normal((T, 2 * Dm)).astype(np.float16)
    b1 = rng.standard_normal(2 * Dm).astype(np.float32) * 0.1
    dw = rng.standard_normal((Dm, 9)).astype(np.float32) * 0.3
    res = {}
    for name, lib in libs(gpu_lib, ref_lib):
        r = {}
        s1 = torch.empty(l1, 64, 256, device="cuda")
        assert lib.d1_sub_conv0(P(cu(mel)), Tin, Fm, P(cu(w0)), P(cu(b0)), P(s1), l1, 64, ST()) == 0
        r["conv0"] = np_(s1)
        l2 = (l1 - 1) // 2 + 1
        s2 = torch.empty(l2, 32, 256, device="cuda")
        assert lib.d1_sub_dwconv(P(s1), l1, 64, P(cu(w2)), P(cu(b0)), P(s2), l2, 32, ST()) == 0
        r["dw"] = np_(s2)
        outs = [torch.empty(T, Dm, dtype=torch.float16, device="cuda") for _ in range(4)]
        assert lib.d1_relpos_prep(P(cu(qkv)), *[P(cu(v)) for v in vecs], *[P(o) for o in outs], T, Dm, ST()) == 0
        r["prep"] = [np_(o) for o in outs]
        p = torch.empty(8, T, T, dtype=torch.float16, device="cuda")
        assert lib.d1_relpos_softmax(P(cu(ac)), P(cu(bd)), P(p), T, 8, 0.125, ST()) == 0
        r["softmax"] = np_(p)
        o = torch.empty(T, Dm, dtype=torch.float16, device="cuda")
        assert lib.d1_conformer_dw(P(cu(a2)), P(cu(b1)), P(cu(dw)), P(cu(vecs[0])), P(cu(vecs[1])), P(cu(vecs[2])),
                                   P(o), T, Dm, 9, ST()) == 0
        r["cdw"] = np_(o)
        res[name] = r
    d, f = res["d1"], res["ref"]
    # the reference's per-element arithmetic (bias, then fused multiply-adds over the taps in order): bit-identical
    assert np.array_equal(d["conv0"], f["conv0"])
    assert np.array_equal(d["dw"], f["dw"])
    assert all(np.array_equal(x, y) for x, y in zip(d["prep"], f["prep"]))
    assert half_ulp_close(d["softmax"], f["softmax"], 2.0 ** -10, 1e-6).all()
    assert np.array_equal(d["cdw"], f["cdw"])
    # softmax rows against numpy
    i = np.arange(T)[:, None]
    j = np.arange(T)[None, :]
    s = (ac + bd[:, i, j + T - 1 - i]) * 0.125
    s = np.exp(s - s.max(-1, keepdims=True))
    assert np.allclose(d["softmax"], s / s.sum(-1, keepdims=True), atol=2e-3)


@pytest.mark.parametrize("tin", [1, 2, 5, 301, 3000])
def test_subsampling_fused(gpu_lib, ref_lib, tin):
    """d1_sub_conv01 (conv0 + the first depthwise conv, the conv0 rows in shared memory) equals d1_sub_conv0 +
    d1_sub_dwconv bit for bit, and both equal the reference's two kernels; ragged lengths down to one frame and
    a 30 s clip; the second depthwise conv (16 bins) against the reference's too."""
    rng = np.random.default_rng(tin)
    Fm = 128
    l1 = (tin - 1) // 2 + 1
    l2 = (l1 - 1) // 2 + 1
    l3 = (l2 - 1) // 2 + 1
    mel = rng.standard_normal((tin + 3, Fm)).astype(np.float32)  # rows past tin_valid must be ignored
    w0, w2, w5 = [rng.standard_normal((256, 9)).astype(np.float32) * 0.3 for _ in range(3)]
    b0, b2, b5 = [rng.standard_normal(256).astype(np.float32) * 0.1 for _ in range(3)]
    s2s = {}
    for name, lib in libs(gpu_lib, ref_lib):
        s1 = torch.empty(l1, 64, 256, device="cuda")
        s2 = torch.empty(l2, 32, 256, device="cuda")
        s3 = torch.empty(l3, 16, 256, device="cuda")
        assert lib.d1_sub_conv0(P(cu(mel)), tin, Fm, P(cu(w0)), P(cu(b0)), P(s1), l1, 64, ST()) == 0
        assert lib.d1_sub_dwconv(P(s1), l1, 64, P(cu(w2)), P(cu(b2)), P(s2), l2, 32, ST()) == 0
        assert lib.d1_sub_dwconv(P(s2), l2, 32, P(cu(w5)), P(cu(b5)), P(s3), l3, 16, ST()) == 0
        s2s[name] = (np_(s2), np_(s3))
    assert np.array_equal(s2s["d1"][0], s2s["ref"][0]) and np.array_equal(s2s["d1"][1], s2s["ref"][1])
    fused = torch.full((l2, 32, 256), float("nan"), device="cuda")
    assert gpu_lib.d1_sub_conv01(P(cu(mel)), tin, Fm, P(cu(w0)), P(cu(b0)), P(cu(w2)), P(cu(b2)), P(fused), l1, l2,
                                 ST()) == 0
    assert np.array_equal(np_(fused), s2s["ref"][0])
    assert gpu_lib.d1_sub_conv01(P(cu(mel)), tin, 129, P(cu(w0)), P(cu(b0)), P(cu(w2)), P(cu(b2)), P(fused), l1, l2,
                                 ST()) == -1  # more bins than the fused kernel stages


@pytest.mark.parametrize("lens", [[38], [1, 9, 4, 200], [375, 375, 17]])
def test_conformer_dw_clips(gpu_lib, ref_lib, lens):
    """The packed form (every clip in one launch, zero padding at each clip's edges) equals the reference's kernel
    run once per clip, bit for bit."""
    rng = np.random.default_rng(sum(lens))
    Dm, R = 512, sum(lens)
    a = rng.standard_normal((R, 2 * Dm)).astype(np.float16)
    b1 = rng.standard_normal(2 * Dm).astype(np.float32) * 0.1
    dw = rng.standard_normal((Dm, 9)).astype(np.float32) * 0.3
    dwb, s, sh = [rng.standard_normal(Dm).astype(np.float32) * 0.2 for _ in range(3)]
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    ad = cu(a)
    got = torch.full((R, Dm), float("nan"), dtype=torch.float16, device="cuda")
    assert gpu_lib.d1_conformer_dw_clips(P(ad), P(cu(b1)), P(cu(dw)), P(cu(dwb)), P(cu(s)), P(cu(sh)), P(got),
                                         P(cu(offs)), len(lens), R, Dm, 9, ST()) == 0
    want = torch.empty(R, Dm, dtype=torch.float16, device="cuda")
    for c in range(len(lens)):
        o, t = int(offs[c]), lens[c]
        assert ref_lib.d1_conformer_dw(C.c_void_p(ad.data_ptr() + o * 2 * Dm * 2), P(cu(b1)), P(cu(dw)), P(cu(dwb)),
                                       P(cu(s)), P(cu(sh)), C.c_void_p(want.data_ptr() + o * Dm * 2), t, Dm, 9,
                                       ST()) == 0
    assert np.array_equal(np_(got), np_(want))


@pytest.mark.parametrize("T", [38, 200, 400, 600])
def test_relpos_softmax_lengths(gpu_lib, ref_lib, T):
    """Every register-window width of the warp-per-row softmax (rows up to 128, 256, 512 columns, and longer)."""
    rng = np.random.default_rng(T)
    H = 8
    ac = rng.standard_normal((H, T, T)).astype(np.float32)
    bd = rng.standard_normal((H, T, 2 * T - 1)).astype(np.float32)
    out = {}
    for name, lib in libs(gpu_lib, ref_lib):
        p = torch.empty(H, T, T, dtype=torch.float16, device="cuda")
        assert lib.d1_relpos_softmax(P(cu(ac)), P(cu(bd)), P(p), T, H, 0.125, ST()) == 0
        out[name] = np_(p)
    assert half_ulp_close(out["d1"], out["ref"], 2.0 ** -10, 1e-6).all()


@pytest.mark.parametrize("Dm", [512, 100])
def test_relpos_prep_widths(gpu_lib, ref_lib, Dm):
    """16-byte vectors (Dm a multiple of 8) and the one-column form, bit-exact against the reference."""
    rng = np.random.default_rng(Dm)
    T = 77
    qkv = rng.standard_normal((T, 3 * Dm)).astype(np.float16)
    vecs = [rng.standard_normal(Dm).astype(np.float32) * 0.1 for _ in range(5)]
    res = {}
    for name, lib in libs(gpu_lib, ref_lib):
        outs = [torch.empty(T, Dm, dtype=torch.float16, device="cuda") for _ in range(4)]
        assert lib.d1_relpos_prep(P(cu(qkv)), *[P(cu(v)) for v in vecs], *[P(o) for o in outs], T, Dm, ST()) == 0
        res[name] = [np_(o) for o in outs]
    assert all(np.array_equal(x, y) for x, y in zip(res["d1"], res["ref"]))


def test_layernorm_rows_unshuffle(gpu_lib, ref_lib):
    """d1_layernorm_rows with the unshuffle permutation as output rows equals d1_layernorm then d1_unshuffle per
    crop (the vision tower's post-LayerNorm and projector input), pending bias included."""
    rng = np.random.default_rng(12)
    crops = [(4, 6), (2, 2), (8, 10)]
    D = 768
    rows = sum(h * w for h, w in crops)
    x = rng.standard_normal((rows, D)).astype(np.float32) * 2
    pend = rng.standard_normal(D).astype(np.float32) * 0.1
    wn = rng.standard_normal(D).astype(np.float32)
    bn = rng.standard_normal(D).astype(np.float32) * 0.1
    yr, src, dst = [], 0, 0
    for ph, pw in crops:
        for y in range(ph):
            for xx in range(pw):
                yr.append(4 * (dst + (y // 2) * (pw // 2) + xx // 2) + 2 * (y % 2) + xx % 2)
        dst += ph * pw // 4
    got = torch.full((rows // 4, 4 * D), float("nan"), dtype=torch.float16, device="cuda")
    xd = cu(x)
    assert gpu_lib.d1_layernorm_rows(P(xd), P(cu(pend)), 1.0, P(cu(wn)), P(cu(bn)), P(got), P(cu(np.array(yr, np.int32))),
                                     rows, D, 1e-6, ST()) == 0
    x_after = np_(xd)
    xr = cu(x)
    xn = torch.empty(rows, D, dtype=torch.float16, device="cuda")
    assert ref_lib.d1_layernorm(P(xr), P(cu(pend)), 1.0, P(cu(wn)), P(cu(bn)), P(xn), None, rows, D, 1e-6, ST()) == 0
    want = torch.empty(rows // 4, 4 * D, dtype=torch.float16, device="cuda")
    src = dst = 0
    for ph, pw in crops:
        assert ref_lib.d1_unshuffle(C.c_void_p(xn.data_ptr() + src * D * 2), C.c_void_p(want.data_ptr() + dst * 4 * D * 2),
                                    ph, pw, D, ST()) == 0
        src += ph * pw
        dst += ph * pw // 4
    assert np.array_equal(x_after, np_(xr))  # the pending bias folded into x as d1_layernorm does
    assert half_ulp_close(np_(got), np_(want), 2.0 ** -10, 1e-6).all()
