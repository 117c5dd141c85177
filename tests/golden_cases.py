"""Golden-vector cases shared by tests/golden/make_golden.py (which runs them on the reference's own kernels) and
tests/test_golden.py (which checks the oracle on the CPU and libd1kernels on the GPU against the stored outputs).

Each case holds seeded numpy inputs, `run(lib, ...)` calling the d1_* C ABI of any library (the reference's or
this one), and `oracle()` computing the same outputs with oracle/d1_oracle.py. Sizes are small (fixtures stay a
few MB) but cover the edge cases: ragged packed sequences (1, 2, 63, 64, 65 rows), prefix state and keys,
marker-row queries, all activation codes, and both GQA and MHA attention.
"""
import ctypes as C

import numpy as np

from oracle import d1_oracle as O


class Case:
    def __init__(self, inputs, run, oracle, tol):
        self.inputs, self._run, self._oracle, self.tol = inputs, run, oracle, tol

    def run(self, lib, *a):
        return self._run(lib, self.inputs, *a)

    def oracle(self):
        return self._oracle(self.inputs)


# ---------------------------------------------------------------------------------------------- GPU helpers
def _torch():
    import torch
    return torch


class _Dev:
    """Keeps device copies alive for the duration of one case run."""

    def __init__(self):
        self.keep = []

    def __call__(self, a):
        torch = _torch()
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        self.keep.append(t)
        return t

    def empty(self, shape, dtype):
        torch = _torch()
        t = torch.empty(shape, dtype=dtype, device="cuda")
        self.keep.append(t)
        return t

    def zeros(self, shape, dtype):
        torch = _torch()
        t = torch.zeros(shape, dtype=dtype, device="cuda")
        self.keep.append(t)
        return t


def P(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def ST():
    torch = _torch()
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def host(t):
    torch = _torch()
    torch.cuda.synchronize()
    return t.cpu().numpy()


def seqinfo_bytes(abi, spans, qtypes=None, pos_off=None, ext_bx=None, save_bx=None, save_k=None, save_v=None):
    arr = (abi.SeqInfo * len(spans))()
    for i, (s, n) in enumerate(spans):
        arr[i].start, arr[i].len = s, n
        arr[i].qtype = qtypes[i] if qtypes is not None else 0
        arr[i].pos_off = pos_off[i] if pos_off is not None else 0
        if ext_bx is not None and ext_bx[i] is not None:
            arr[i].ext_bx = ext_bx[i]
        if save_bx is not None and save_bx[i] is not None:
            arr[i].save_bx = save_bx[i]
        if save_k is not None and save_k[i] is not None:
            arr[i].save_k, arr[i].save_v = save_k[i], save_v[i]
    return np.frombuffer(bytes(arr), np.uint8).copy()


def attnseq_bytes(abi, seqs, ext=None):
    arr = (abi.AttnSeq * len(seqs))()
    for i, (qs, ql, ks, kl) in enumerate(seqs):
        arr[i].q_start, arr[i].q_len, arr[i].kv_start, arr[i].kv_len = qs, ql, ks, kl
        if ext is not None and ext[i] is not None:
            arr[i].ext_len = ext[i][0]
            arr[i].ext_k, arr[i].ext_v = ext[i][1], ext[i][2]
    return np.frombuffer(bytes(arr), np.uint8).copy()


def work_items(seqs):
    w = []
    for i, (qs, ql, ks, kl) in enumerate(seqs):
        w += [i, 0] if ql == 0 else sum([[i, q] for q in range(0, ql, 64)], [])
    return np.asarray(w, np.int32)


def spans_of(lens):
    out, s = [], 0
    for n in lens:
        out.append((s, n))
        s += n
    return out


# ---------------------------------------------------------------------------------------------- kernel cases
def kernel_cases():
    from fast_d1_omni_b200 import abi
    rng = np.random.default_rng(1234)
    cases = {}

    # rmsnorm, D = 1024 and 768
    for D in (1024, 768):
        x = (rng.standard_normal((9, D)) * 2).astype(np.float32)
        w = rng.standard_normal(D).astype(np.float32)

        def run(lib, i, D=D):
            d = _Dev()
            y = d.empty((i["x"].shape[0], D), _torch().float16)
            assert lib.d1_rmsnorm(P(d(i["x"])), P(d(i["w"])), P(y), i["x"].shape[0], D, 1e-5, ST()) == 0
            return {"y": host(y)}

        cases[f"rmsnorm{D}"] = Case({"x": x, "w": w}, run,
                                    lambda i: {"y": O.r16(O.rmsnorm(i["x"], i["w"], 1e-5))}, "f16")

    # layernorm with a pending bias, fp16 + fp32 outputs, D = 1024
    x = rng.standard_normal((7, 1024)).astype(np.float32)
    pb, w, b = (rng.standard_normal(1024).astype(np.float32) for _ in range(3))

    def run_ln(lib, i):
        d = _Dev()
        xd = d(i["x"])
        y = d.empty((7, 1024), _torch().float16)
        yf = d.empty((7, 1024), _torch().float32)
        assert lib.d1_layernorm(P(xd), P(d(i["pb"])), 0.5, P(d(i["w"])), P(d(i["b"])), P(y), P(yf), 7, 1024, 1e-5,
                                ST()) == 0
        return {"x": host(xd), "y": host(y), "yf": host(yf)}

    def or_ln(i):
        xn, y = O.layernorm(i["x"], i["w"], i["b"], 1e-5, i["pb"], 0.5)
        return {"x": xn, "y": O.r16(y), "yf": y}

    cases["layernorm"] = Case({"x": x, "pb": pb, "w": w, "b": b}, run_ln, or_ln, "f16")

    # head_init
    spans = [(0, 3), (3, 1), (4, 6)]
    h = rng.standard_normal((10, 1024)).astype(np.float32)
    te = rng.standard_normal((4, 1024)).astype(np.float32)
    hw = rng.standard_normal(1024).astype(np.float32)
    qt = np.asarray([1, 3, 0], np.int32)

    def run_hi(lib, i):
        d = _Dev()
        sp = spans_of([3, 1, 6])
        seqs = d(seqinfo_bytes(abi, sp, qtypes=list(i["qt"])))
        tok = d(np.repeat(np.arange(3, dtype=np.int32), [3, 1, 6]))
        out = d.empty((10, 1024), _torch().float32)
        assert lib.d1_head_init(P(d(i["h"])), P(d(i["w"])), P(d(i["te"])), P(tok), P(seqs), P(out), 10, 1e-5,
                                ST()) == 0
        return {"out": host(out)}

    cases["head_init"] = Case({"h": h, "w": hw, "te": te, "qt": qt}, run_hi,
                              lambda i: {"out": O.head_init(i["h"], i["w"], i["te"], np.repeat(i["qt"], [3, 1, 6]),
                                                            1e-5)}, "f32")

    # swiglu and bias+act (all activation codes)
    gu = (rng.standard_normal((5, 2 * 64)) * 2).astype(np.float16)

    def run_sw(lib, i):
        d = _Dev()
        out = d.empty((5, 64), _torch().float16)
        assert lib.d1_swiglu(P(d(i["gu"])), P(out), 5, 64, ST()) == 0
        return {"out": host(out)}

    cases["swiglu"] = Case({"gu": gu}, run_sw, lambda i: {"out": O.r16(O.swiglu(i["gu"].astype(np.float32), 64))},
                           "f16")
    xa = (rng.standard_normal((4, 64)) * 2).astype(np.float16)
    ba = rng.standard_normal(64).astype(np.float32)
    for act in range(5):
        def run_ba(lib, i, act=act):
            d = _Dev()
            xd = d(i["x"])
            assert lib.d1_bias_act_h(P(xd), P(d(i["b"])), 4, 64, act, ST()) == 0
            return {"y": host(xd)}

        cases[f"bias_act{act}"] = Case({"x": xa, "b": ba}, run_ba,
                                       lambda i, act=act: {"y": O.r16(O.bias_act(i["x"].astype(np.float32), i["b"],
                                                                                 act))}, "f16")

    # short conv: ragged sequences, prefix state on the second sequence, saved last states
    lens = [1, 2, 17, 9]
    sp = spans_of(lens)
    T, Dm = sum(lens), 1024
    bcu = (rng.standard_normal((T, 3 * Dm)) * 1.5).astype(np.float16)
    cw = (rng.standard_normal((Dm, 3)) * 0.5).astype(np.float32)
    ext = (rng.standard_normal((3, Dm)) * 0.5).astype(np.float16)  # [n_conv=3][D], conv_idx 1

    def run_sc(lib, i, sp=sp, lens=lens, T=T, Dm=Dm):
        d = _Dev()
        torch = _torch()
        ext_d = d(i["ext"])
        saves = [d.zeros((3, Dm), torch.float16) for _ in lens]
        seqs = d(seqinfo_bytes(abi, sp, ext_bx=[None, ext_d.data_ptr(), None, None],
                               save_bx=[t.data_ptr() for t in saves]))
        tok = d(np.repeat(np.arange(len(lens), dtype=np.int32), lens))
        out = d.empty((T, Dm), torch.float16)
        assert lib.d1_shortconv(P(d(i["bcu"])), P(d(i["cw"])), P(tok), P(seqs), P(out), T, Dm, 1, ST()) == 0
        return {"out": host(out), "saved": np.stack([host(t)[1] for t in saves])}

    def or_sc(i, sp=sp):
        out, saved = O.shortconv(i["bcu"].astype(np.float32), i["cw"], sp, 1,
                                 [None, i["ext"][1].astype(np.float32), None, None])
        return {"out": O.r16(out), "saved": np.stack(saved)}

    cases["shortconv"] = Case({"bcu": bcu, "cw": cw, "ext": ext}, run_sc, or_sc, "f16")

    # QK RMSNorm + RoPE with K/V save, positions after a prefix
    lens = [3, 12]
    sp = spans_of(lens)
    T, ld = 15, 2048
    qkv = rng.standard_normal((T, ld)).astype(np.float16)
    qn = rng.standard_normal(64).astype(np.float32)
    kn = rng.standard_normal(64).astype(np.float32)
    pos_off = [0, 37]

    def run_qk(lib, i, sp=sp, lens=lens, T=T, ld=ld, pos_off=pos_off):
        d = _Dev()
        torch = _torch()
        sk = [d.zeros((2, n, 512), torch.float16) for n in lens]
        sv = [d.zeros((2, n, 512), torch.float16) for n in lens]
        seqs = d(seqinfo_bytes(abi, sp, pos_off=pos_off, save_k=[t.data_ptr() for t in sk],
                               save_v=[t.data_ptr() for t in sv]))
        tok = d(np.repeat(np.arange(2, dtype=np.int32), lens))
        q = d(i["qkv"])
        rope = d(O.rope_table(1e6))
        assert lib.d1_qk_norm_rope(P(q), ld, 16, 8, P(d(i["qn"])), P(d(i["kn"])), P(rope), P(tok), P(seqs), 1, T,
                                   1e-5, ST()) == 0
        return {"qkv": host(q), "save_k": np.concatenate([host(t)[1] for t in sk]),
                "save_v": np.concatenate([host(t)[1] for t in sv])}

    def or_qk(i, lens=lens, pos_off=pos_off):
        pos = np.concatenate([np.arange(n) + po for n, po in zip(lens, pos_off)])
        out = O.qk_norm_rope(i["qkv"].astype(np.float32), 16, 8, i["qn"], i["kn"], O.rope_table(1e6), pos, 1e-5)
        return {"qkv": out, "save_k": out[:, 1024:1536], "save_v": i["qkv"][:, 1536:].astype(np.float32)}

    cases["qk_norm_rope"] = Case({"qkv": qkv, "qn": qn, "kn": kn}, run_qk, or_qk, "f16")

    # flash attention: GQA trunk form with prefix keys (ragged 1/63/65 rows), MHA+bias head form, marker queries
    lens = [1, 63, 65]
    sp = spans_of(lens)
    T = sum(lens)
    qkv = rng.standard_normal((T, 2048)).astype(np.float16)
    ek = rng.standard_normal((70, 512)).astype(np.float16)
    ev = rng.standard_normal((70, 512)).astype(np.float16)

    def run_fa(lib, i, sp=sp, T=T):
        d = _Dev()
        q = d(i["qkv"])
        ekd, evd = d(i["ek"]), d(i["ev"])
        seqs = [(s, n, s, n) for s, n in sp]
        meta = d(attnseq_bytes(abi, seqs, [None, (70, ekd.data_ptr(), evd.data_ptr()), None]))
        w = work_items(seqs)
        o = d.zeros((T, 1024), _torch().float16)
        assert lib.d1_flash_attn(P(q), 2048, P(q[:, 1024:]), P(q[:, 1536:]), 2048, 512, None, None, None, P(o), 1024,
                                 P(meta), P(d(w)), len(w) // 2, 16, 2, 0.125, ST()) == 0
        return {"o": host(o)}

    def or_fa(i, sp=sp):
        q = i["qkv"].astype(np.float32)
        ext = [None, (i["ek"].astype(np.float32), i["ev"].astype(np.float32)), None]
        return {"o": O.r16(O.attention(q[:, :1024], q[:, 1024:1536], q[:, 1536:], [(s, n, s, n) for s, n in sp], 16, 2,
                                       0.125, ext=ext))}

    cases["flash_gqa_prefix"] = Case({"qkv": qkv, "ek": ek, "ev": ev}, run_fa, or_fa, "attn")

    lens2, marks = [40, 90], [[0, 39], [5, 50, 89]]
    sp2 = spans_of(lens2)
    T2 = sum(lens2)
    qkv3 = rng.standard_normal((T2, 3072)).astype(np.float16)
    bias = (rng.standard_normal(3072) * 0.5).astype(np.float32)
    rows = np.asarray([s + m for (s, n), mk in zip(sp2, marks) for m in mk], np.int64)

    def run_fb(lib, i, sp2=sp2, T2=T2, rows=rows, marks=marks):
        d = _Dev()
        q = d(i["qkv"])
        bd = d(i["bias"])
        seqs = [(s, n, s, n) for s, n in sp2]
        meta = d(attnseq_bytes(abi, seqs))
        w = work_items(seqs)
        o = d.zeros((T2, 1024), _torch().float16)
        assert lib.d1_flash_attn(P(q), 3072, P(q[:, 1024:]), P(q[:, 2048:]), 3072, 0, P(bd[:1024]), P(bd[1024:2048]),
                                 P(bd[2048:]), P(o), 1024, P(meta), P(d(w)), len(w) // 2, 16, 1, 0.125, ST()) == 0
        mq = d(np.ascontiguousarray(i["qkv"][rows]))
        ms, mseqs = 0, []
        for (s, n), mk in zip(sp2, marks):
            mseqs.append((ms, len(mk), s, n))
            ms += len(mk)
        mmeta = d(attnseq_bytes(abi, mseqs))
        mw = work_items(mseqs)
        mo = d.zeros((len(rows), 1024), _torch().float16)
        assert lib.d1_flash_attn(P(mq), 3072, P(q[:, 1024:]), P(q[:, 2048:]), 3072, 0, P(bd[:1024]), P(bd[1024:2048]),
                                 P(bd[2048:]), P(mo), 1024, P(mmeta), P(d(mw)), len(mw) // 2, 16, 1, 0.125, ST()) == 0
        return {"o": host(o), "mo": host(mo)}

    def or_fb(i, sp2=sp2, rows=rows, marks=marks):
        q = i["qkv"].astype(np.float32)
        b = i["bias"]
        o = O.attention(q[:, :1024], q[:, 1024:2048], q[:, 2048:], [(s, n, s, n) for s, n in sp2], 16, 1, 0.125,
                        b[:1024], b[1024:2048], b[2048:])
        ms, mseqs = 0, []
        for (s, n), mk in zip(sp2, marks):
            mseqs.append((ms, len(mk), s, n))
            ms += len(mk)
        mo = O.attention(q[rows, :1024], q[:, 1024:2048], q[:, 2048:], mseqs, 16, 1, 0.125, b[:1024], b[1024:2048],
                         b[2048:])
        return {"o": O.r16(o), "mo": O.r16(mo)}

    cases["flash_mha_bias_markers"] = Case({"qkv": qkv3, "bias": bias}, run_fb, or_fb, "attn")

    # scorer, gathers, unshuffle
    xs = rng.standard_normal((6, 1024)).astype(np.float16)
    b1 = rng.standard_normal(1024).astype(np.float32)
    w2 = (rng.standard_normal(1024) * 0.05).astype(np.float16)

    def run_so(lib, i):
        d = _Dev()
        out = d.empty((6,), _torch().float32)
        assert lib.d1_scorer_out(P(d(i["x"])), P(d(i["b1"])), P(d(i["w2"])), 0.3, P(out), 6, 1024, ST()) == 0
        return {"logits": host(out)}

    cases["scorer_out"] = Case({"x": xs, "b1": b1, "w2": w2}, run_so,
                               lambda i: {"logits": O.scorer_out(i["x"].astype(np.float32), i["b1"],
                                                                 i["w2"].astype(np.float32), 0.3)}, "f32")
    xu = rng.standard_normal((4 * 6, 768)).astype(np.float16)

    def run_un(lib, i):
        d = _Dev()
        out = d.empty((6, 3072), _torch().float16)
        assert lib.d1_unshuffle(P(d(i["x"])), P(out), 4, 6, 768, ST()) == 0
        return {"out": host(out)}

    cases["unshuffle"] = Case({"x": xu}, run_un, lambda i: {"out": O.unshuffle(i["x"], 4, 6, 768)}, "exact")
    return cases


# ---------------------------------------------------------------------------------------------- GEMM cases
def gemm_cases():
    rng = np.random.default_rng(99)
    cases = {}
    for name, (M, N, K, f32) in {"f16_out": (70, 384, 256, False), "f32_residual": (130, 256, 512, True)}.items():
        x = rng.standard_normal((M, K)).astype(np.float16)
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
        y0 = rng.standard_normal((M, N)).astype(np.float32)

        def run(lib, i, ctx, M=M, N=N, K=K, f32=f32):
            d = _Dev()
            torch = _torch()
            y = d(i["y0"]) if f32 else d.empty((M, N), torch.float16)
            r = lib.d1_lt_gemm(ctx, M, N, K, P(d(i["x"])), K, P(d(i["w"])), K, 0, P(y), N, int(f32), 0, 1.0,
                               1.0 if f32 else 0.0, ST())
            if r == -2:  # the reference needs a plan: tune the shape first (src/engine.rs:528-616)
                assert lib.d1_lt_tune(ctx, M, N, K, K, K, 0, N, int(f32), 0, 0, ST()) > 0
                r = lib.d1_lt_gemm(ctx, M, N, K, P(d(i["x"])), K, P(d(i["w"])), K, 0, P(y), N, int(f32), 0, 1.0,
                                   1.0 if f32 else 0.0, ST())
            assert r == 0
            return {"y": host(y)}

        def orc(i, f32=f32):
            y = O.gemm(i["x"], i["w"], i["y0"] if f32 else None, 1.0, 1.0 if f32 else 0.0)
            return {"y": y if f32 else O.r16(y)}

        cases[name] = Case({"x": x, "w": w, "y0": y0}, run, orc, "f32" if f32 else "f16")
    return cases


# ---------------------------------------------------------------------------------------------- engine case
ENGINE = dict(seed=0, n_layers=4, attn_layers=(2,), vocab=4096, n_head=2, head_ffn=512)


def engine_batch():
    from fast_d1_omni_b200.weights import text_batch
    b = text_batch(7, 0, lengths=[70, 1, 130, 64], vocab=4096)
    b[1]["markers"] = b[1]["markers"][:1]
    return b


def engine_case(pkg, kernel_lib):
    """Logits of the small model through the host runner with `kernel_lib`'s kernels."""
    from fast_d1_omni_b200.model import TextModel
    from fast_d1_omni_b200.weights import text_weights
    w = text_weights(**ENGINE)
    b = engine_batch()
    m = TextModel(w, kernel_lib=kernel_lib, fused=False, cap_tokens=512)
    try:
        logits = m(b)
    finally:
        m.close()
    sizes = np.asarray([len(s["markers"]) for s in b], np.int32)
    return logits, {"sizes": sizes}
