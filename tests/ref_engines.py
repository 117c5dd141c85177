"""The reference's F16 engine pieces that have no host runner here, restated for the GPU tests: the audio encoder
of src/audio.rs:505-594 driven call for call through the reference's own kernels and its cuBLASLt GEMM
(oracle/_ref/libd1ref.so). Test infrastructure only."""
import ctypes as C

import numpy as np
import torch

from oracle import d1_oracle as O


def P(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def ST():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


class RefAudioEngine:
    """src/audio.rs:505-594 for one clip, with the reference's kernels and d1_lt_gemm (libd1ref.so); the Rust
    side's direct cuBLAS calls (Blas::sgemm, Blas::gemm_batched) are torch matmuls with fp32 accumulation."""

    def __init__(self, lib, w):
        self.lib = lib
        self.lt = lib.d1_lt_init(32 << 20)
        assert self.lt
        self.w = w
        f16 = {"ff1_up", "ff1_down", "qkv", "pos", "out", "pw1", "pw2", "ff2_up", "ff2_down", "ad1", "ad2",
               "res_down", "res_up"}
        d = lambda k, a: dev(np.asarray(a, np.float16 if k in f16 else np.float32))  # noqa: E731
        self.g = {k: d(k, v) for k, v in w.items() if k not in ("layers", "eps")}
        self.layers = [{k: d(k, v) for k, v in l.items()} for l in w["layers"]]
        self.eps = float(w["eps"])

    def gemm(self, m, n, k, x, ldx, wt, ldw, y, ldy, y32, alpha, beta):
        L = self.lib
        args = (self.lt, m, n, k, P(x), ldx, P(wt), ldw, 0, P(y), ldy, int(y32), 0, alpha, beta, ST())
        e = L.d1_lt_gemm(*args)
        if e == -2:
            assert L.d1_lt_tune(self.lt, m, n, k, ldx, ldw, 0, ldy, int(y32), 0, 0, ST()) > 0
            e = L.d1_lt_gemm(*args)
        assert e == 0

    def encode(self, mel, valid):
        L, g, eps = self.lib, self.g, self.eps
        l1 = (valid - 1) // 2 + 1
        l2 = (l1 - 1) // 2 + 1
        t = (l2 - 1) // 2 + 1
        m = dev(np.asarray(mel[:valid], np.float32))
        s1 = torch.empty(l1 * 64 * 256, device="cuda")
        s2 = torch.empty(l2 * 32 * 256, device="cuda")
        s3 = torch.empty(l2 * 32 * 256, device="cuda")
        assert L.d1_sub_conv0(P(m), valid, 128, P(g["c0_w"]), P(g["c0_b"]), P(s1), l1, 64, ST()) == 0
        assert L.d1_sub_dwconv(P(s1), l1, 64, P(g["c2_w"]), P(g["c2_b"]), P(s2), l2, 32, ST()) == 0
        s3v = s3.view(l2 * 32, 256)
        assert L.d1_fill_rows(P(s3), P(g["c3_b"]), None, l2 * 32, 256, ST()) == 0
        s3v += s2.view(l2 * 32, 256) @ g["c3_w"].T
        assert L.d1_bias_act_f(P(s3), None, l2 * 32, 256, 1, ST()) == 0
        assert L.d1_sub_dwconv(P(s3), l2, 32, P(g["c5_w"]), P(g["c5_b"]), P(s2), t, 16, ST()) == 0
        s1v = s1[:t * 16 * 256].view(t * 16, 256)
        assert L.d1_fill_rows(P(s1), P(g["c6_b"]), None, t * 16, 256, ST()) == 0
        s1v += s2[:t * 16 * 256].view(t * 16, 256) @ g["c6_w"].T
        assert L.d1_bias_act_f(P(s1), None, t * 16, 256, 1, ST()) == 0
        x = torch.empty(t, 512, device="cuda")
        assert L.d1_fill_rows(P(x), P(g["pre_out_b"]), None, t, 512, ST()) == 0
        x += s1[:t * 4096].view(t, 4096) @ g["pre_out"].T
        pe = dev(O.relpos_pe(t).astype(np.float16))
        xn = torch.empty(t, 1024, dtype=torch.float16, device="cuda")
        big = torch.empty(t, 2048, dtype=torch.float16, device="cuda")
        qu, qv, kk, vv, o = [torch.empty(t, 512, dtype=torch.float16, device="cuda") for _ in range(5)]
        pp = torch.empty(2 * t - 1, 512, dtype=torch.float16, device="cuda")
        probs = torch.empty(8, t, t, dtype=torch.float16, device="cuda")

        def ln(xx, pb, ps, wn, bn, y, yf, d=512):
            assert L.d1_layernorm(P(xx), P(pb), ps, P(wn), P(bn), P(y), P(yf), t, d, eps, ST()) == 0

        for l in self.layers:
            ln(x, None, 1.0, l["ff1_n_w"], l["ff1_n_b"], xn, None)
            self.gemm(t, 2048, 512, xn, 512, l["ff1_up"], 512, big, 2048, False, 1.0, 0.0)
            assert L.d1_bias_act_h(P(big), P(l["ff1_up_b"]), t, 2048, 4, ST()) == 0
            self.gemm(t, 512, 2048, big, 2048, l["ff1_down"], 2048, x, 512, True, 0.5, 1.0)
            ln(x, l["ff1_down_b"], 0.5, l["att_n_w"], l["att_n_b"], xn, None)
            self.gemm(t, 1536, 512, xn, 512, l["qkv"], 512, big, 1536, False, 1.0, 0.0)
            assert L.d1_relpos_prep(P(big), *[P(l[n]) for n in ("bq", "bk", "bv", "pu", "pv")],
                                    P(qu), P(qv), P(kk), P(vv), t, 512, ST()) == 0
            self.gemm(2 * t - 1, 512, 512, pe, 512, l["pos"], 512, pp, 512, False, 1.0, 0.0)
            heads = lambda a, n: a.float().view(n, 8, 64).transpose(0, 1)  # noqa: E731
            ac = (heads(qu, t) @ heads(kk, t).transpose(1, 2)).contiguous()
            bd = (heads(qv, t) @ heads(pp, 2 * t - 1).transpose(1, 2)).contiguous()
            assert L.d1_relpos_softmax(P(ac), P(bd), P(probs), t, 8, 0.125, ST()) == 0
            o.copy_((probs.float() @ heads(vv, t)).transpose(0, 1).reshape(t, 512).half())
            self.gemm(t, 512, 512, o, 512, l["out"], 512, x, 512, True, 1.0, 1.0)
            ln(x, l["out_b"], 1.0, l["conv_n_w"], l["conv_n_b"], xn, None)
            self.gemm(t, 1024, 512, xn, 512, l["pw1"], 512, big, 1024, False, 1.0, 0.0)
            assert L.d1_conformer_dw(P(big), P(l["pw1_b"]), P(l["dw"]), P(l["dw_b"]), P(l["bn_s"]), P(l["bn_b"]),
                                     P(o), t, 512, 9, ST()) == 0
            self.gemm(t, 512, 512, o, 512, l["pw2"], 512, x, 512, True, 1.0, 1.0)
            ln(x, l["pw2_b"], 1.0, l["ff2_n_w"], l["ff2_n_b"], xn, None)
            self.gemm(t, 2048, 512, xn, 512, l["ff2_up"], 512, big, 2048, False, 1.0, 0.0)
            assert L.d1_bias_act_h(P(big), P(l["ff2_up_b"]), t, 2048, 4, ST()) == 0
            self.gemm(t, 512, 2048, big, 2048, l["ff2_down"], 2048, x, 512, True, 0.5, 1.0)
            ln(x, l["ff2_down_b"], 0.5, l["out_n_w"], l["out_n_b"], None, x)
        ln(x, None, 1.0, g["ad_n_w"], g["ad_n_b"], xn, None)
        self.gemm(t, 1024, 512, xn, 512, g["ad1"], 512, big, 1024, False, 1.0, 0.0)
        assert L.d1_bias_act_h(P(big), P(g["ad1_b"]), t, 1024, 2, ST()) == 0
        out = torch.empty(t, 1024, device="cuda")
        assert L.d1_fill_rows(P(out), P(g["ad2_b"]), None, t, 1024, ST()) == 0
        self.gemm(t, 1024, 1024, big, 1024, g["ad2"], 1024, out, 1024, True, 1.0, 1.0)
        ln(out, None, 1.0, g["res_n_w"], g["res_n_b"], xn, None, 1024)
        self.gemm(t, 512, 1024, xn, 1024, g["res_down"], 1024, big, 512, False, 1.0, 0.0)
        assert L.d1_bias_act_h(P(big), P(g["res_down_b"]), t, 512, 2, ST()) == 0
        self.gemm(t, 1024, 512, big, 512, g["res_up"], 512, out, 1024, True, 1.0, 1.0)
        assert L.d1_bias_act_f(P(out), P(g["res_up_b"]), t, 1024, 0, ST()) == 0
        torch.cuda.synchronize()
        return out.cpu().numpy()
