"""CPU oracle for the d1rs forward pass — TEST INFRASTRUCTURE, not product code.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs may import this module; the
product path (libd1kernels + its runner) never calls it.

A numpy restatement of the reference's arithmetic for the hot path, function by function, each citing the
reference file:line it follows (paths within cnmoro/fast-d1-omni). Two precisions:
  * prec="f16": activations are rounded to fp16 exactly where the reference's F16 engine stores fp16
    (GEMM outputs, normed inputs, attention outputs ...), math in fp32 — the model of the F16 engine;
  * prec="f32": everything in fp32 with the same (fp16-valued) weights — the stand-in for the fp32 PyTorch
    reference of tools/ref_model.py, whose remote modeling code and weights are not available here.
Sequences are packed without padding: `spans` is a list of (start, len) row ranges.

Pinning: the reference ships no numeric golden vectors (its only KATs are host-side: SHA-256, JSON, sniffing).
tests/golden/*.npz are outputs of the reference's own CUDA kernels (cuda/kernels.cu, built unchanged into
oracle/_ref by oracle/Makefile) run on a B200 by tests/golden/make_golden.py; tests/test_oracle_golden.py checks
this module against them.
"""
from __future__ import annotations

import math

import numpy as np

D = 1024          # src/model.rs:12
HEADS = 16        # :13
KV_HEADS = 8      # :14
HD = 64           # :15
KV_DIM = KV_HEADS * HD
MAX_POS = 16384 + 64  # :17


def r16(x, prec="f16"):
    """Round to fp16 and back when modelling the F16 engine."""
    if prec != "f16":
        return np.asarray(x, dtype=np.float32)
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


# ------------------------------------------------------------------------------------------------ activations
# cuda/kernels.cu:40-54: 0 none, 1 ReLU, 2 GELU (erf), 3 GELU (tanh), 4 SiLU.

def _erf(x):
    try:
        from scipy.special import erf
        return erf(x).astype(np.float32)
    except Exception:  # pragma: no cover
        return np.vectorize(math.erf)(x).astype(np.float32)


def gelu_erf(x):
    x = np.asarray(x, np.float32)
    return (0.5 * x * (1.0 + _erf(x * np.float32(0.70710678118654752)))).astype(np.float32)


def gelu_tanh(x):
    x = np.asarray(x, np.float32)
    k0, k1 = np.float32(0.7978845608028654), np.float32(0.044715)
    return (0.5 * x * (1.0 + np.tanh(k0 * (x + k1 * x * x * x)))).astype(np.float32)


def silu(x):
    x = np.asarray(x, np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def apply_act(x, act):
    if act == 1:
        return np.maximum(x, 0).astype(np.float32)
    if act == 2:
        return gelu_erf(x)
    if act == 3:
        return gelu_tanh(x)
    if act == 4:
        return silu(x)
    return np.asarray(x, np.float32)


# ------------------------------------------------------------------------------------------------ kernels

def rmsnorm(x, w, eps):
    """cuda/kernels.cu:59-79: y = x * rsqrt(sum(x^2)/D + eps) * w (fp32 math)."""
    x = np.asarray(x, np.float32)
    r = 1.0 / np.sqrt((x * x).sum(-1, keepdims=True, dtype=np.float32) / x.shape[-1] + np.float32(eps))
    return (x * r.astype(np.float32) * w).astype(np.float32)


def layernorm(x, w, b, eps, pend=None, pend_scale=1.0):
    """cuda/kernels.cu:82-117: x += s*pend (returned as the new x), then LayerNorm(x)*w + b."""
    x = np.asarray(x, np.float32)
    if pend is not None:
        x = (x + np.float32(pend_scale) * pend).astype(np.float32)
    mean = x.mean(-1, keepdims=True, dtype=np.float32)
    d = x - mean
    r = 1.0 / np.sqrt((d * d).sum(-1, keepdims=True, dtype=np.float32) / x.shape[-1] + np.float32(eps))
    return x, (d * r.astype(np.float32) * w + b).astype(np.float32)


def head_init(h, w, type_emb, row_qtype, eps):
    """cuda/kernels.cu:120-142: RMSNorm(h)*w + type_emb[qtype of the row's sequence]."""
    return (rmsnorm(h, w, eps) + type_emb[row_qtype]).astype(np.float32)


def embed(table, ids):
    """cuda/kernels.cu:146-156."""
    return np.asarray(table, np.float32)[np.asarray(ids)]


def swiglu(gu, F):
    """cuda/kernels.cu:159-168: silu(gu[:, :F]) * gu[:, F:]."""
    gu = np.asarray(gu, np.float32)
    return silu(gu[:, :F]) * gu[:, F:2 * F]


def bias_act(x, bias, act):
    """cuda/kernels.cu:171-194."""
    x = np.asarray(x, np.float32)
    if bias is not None:
        x = x + bias
    return apply_act(x, act)


def gemm(x, w, y=None, alpha=1.0, beta=0.0):
    """cuda/gemm.cu:8 semantics: Y = alpha * X . W^T + beta * Y (fp32 accumulation)."""
    out = np.float32(alpha) * (np.asarray(x, np.float32) @ np.asarray(w, np.float32).T)
    if y is not None and beta != 0.0:
        out = out + np.float32(beta) * y
    return out.astype(np.float32)


def shortconv(bcu, convw, spans, conv_idx=0, ext_bx=None, prec="f16"):
    """cuda/kernels.cu:224-259: bcu [T,3D] = [b|c|u]; bx = b*u; out[t] = c[t]*(w0*bx[t-1] + w1*bx[t] + w2*bx[t+1]),
    zero outside each sequence (centred 3-tap). ext_bx[i] (optional, [D] fp16 values) is sequence i's left state.
    Returns (out, saved) where saved[i] is half(bx of the sequence's last row) (the save_bx store)."""
    bcu = np.asarray(bcu, np.float32)
    Dm = bcu.shape[1] // 3
    b, c, u = bcu[:, :Dm], bcu[:, Dm:2 * Dm], bcu[:, 2 * Dm:]
    bx = (b * u).astype(np.float32)
    w = np.asarray(convw, np.float32).reshape(Dm, 3)
    out = np.zeros_like(c)
    saved = []
    for i, (s, n) in enumerate(spans):
        seg = bx[s:s + n]
        left = np.zeros_like(seg)
        left[1:] = seg[:-1]
        if ext_bx is not None and ext_bx[i] is not None:
            left[0] = ext_bx[i]
        right = np.zeros_like(seg)
        right[:-1] = seg[1:]
        y = w[:, 0] * left + w[:, 1] * seg + w[:, 2] * right
        out[s:s + n] = c[s:s + n] * y
        saved.append(r16(seg[-1], prec))
    return out.astype(np.float32), saved


def rope_table(theta=1e6):
    """src/model.rs:121-136: [MAX_POS][32] (cos, sin), fp32 inverse frequency and fp32 angle, cos/sin in f64."""
    e = (2.0 * np.arange(32, dtype=np.float32) / np.float32(HD)).astype(np.float32)
    inv = (np.float32(1.0) / np.power(np.float32(theta), e, dtype=np.float32)).astype(np.float32)
    pos = np.arange(MAX_POS, dtype=np.float32)[:, None]
    ang = (pos * inv[None, :]).astype(np.float32).astype(np.float64)
    t = np.empty((MAX_POS, 32, 2), np.float32)
    t[..., 0] = np.cos(ang)
    t[..., 1] = np.sin(ang)
    return t


def qk_norm_rope(qkv, H, KVH, qn, kn, rope, pos, eps, prec="f16"):
    """cuda/kernels.cu:263-303: per-head RMSNorm (dim 64, per-dim weights) of the q and k heads, then RoPE
    rotate-half on pairs (l, l+32) at position pos[row]. Returns the updated qkv (v untouched)."""
    qkv = np.array(qkv, np.float32, copy=True)
    T = qkv.shape[0]
    cs = rope[np.asarray(pos)]  # [T, 32, 2]
    cos, sin = cs[:, None, :, 0], cs[:, None, :, 1]
    for lo, nh, wt in ((0, H, qn), (H * 64, KVH, kn)):
        x = qkv[:, lo:lo + nh * 64].reshape(T, nh, 64)
        r = 1.0 / np.sqrt((x * x).sum(-1, keepdims=True, dtype=np.float32) / 64.0 + np.float32(eps))
        x = x * r.astype(np.float32) * wt
        a, b = x[..., :32], x[..., 32:]
        oa = a * cos - b * sin
        ob = b * cos + a * sin
        qkv[:, lo:lo + nh * 64] = r16(np.concatenate([oa, ob], -1), prec).reshape(T, nh * 64)
    return qkv


def attention(Q, K, V, seqs, heads, group, scale, bq=None, bk=None, bv=None, ext=None, prec="f16"):
    """cuda/kernels.cu:351-500: bidirectional softmax(scale * q . k^T) . v within each sequence, kv head
    g = h // group, keys = [ext prefix | local]; optional fp32 biases added on load (rounded to fp16 as the
    kernel's load8 does). seqs: list of (q_start, q_len, kv_start, kv_len); ext: per seq (k, v) [ext_len, 512]
    or None. Q/K/V are [rows, heads*64] (K/V [rows, kv_heads*64]). Returns O [Q rows, heads*64]."""
    Q = np.asarray(Q, np.float32)
    K = np.asarray(K, np.float32)
    V = np.asarray(V, np.float32)
    if bq is not None:
        Q = r16(Q + bq, prec)
    if bk is not None:
        K = r16(K + bk, prec)
    if bv is not None:
        V = r16(V + bv, prec)
    O = np.zeros((Q.shape[0], heads * 64), np.float32)
    for i, (qs, ql, ks, kl) in enumerate(seqs):
        if ql == 0:
            continue
        k_all, v_all = K[ks:ks + kl], V[ks:ks + kl]
        if ext is not None and ext[i] is not None:
            k_all = np.concatenate([np.asarray(ext[i][0], np.float32), k_all])
            v_all = np.concatenate([np.asarray(ext[i][1], np.float32), v_all])
        q = Q[qs:qs + ql].reshape(ql, heads, 64).transpose(1, 0, 2)  # [h, q, 64]
        kvh = k_all.shape[1] // 64
        k = k_all.reshape(-1, kvh, 64).transpose(1, 0, 2)
        v = v_all.reshape(-1, kvh, 64).transpose(1, 0, 2)
        g = np.arange(heads) // group
        s = np.einsum("hqd,hkd->hqk", q, k[g], dtype=np.float32) * np.float32(scale)
        s = s - s.max(-1, keepdims=True)
        pexp = np.exp(s).astype(np.float32)
        l = pexp.sum(-1, keepdims=True, dtype=np.float32)
        pr = r16(pexp, prec)  # the kernel feeds fp16 P to the PV product and divides by the fp32 row sum
        o = np.einsum("hqk,hkd->hqd", pr, v[g], dtype=np.float32) / l
        O[qs:qs + ql] = o.transpose(1, 0, 2).reshape(ql, heads * 64)
    return O


def scorer_out(x, b1, w2, b2):
    """cuda/kernels.cu:504-513: sum_i gelu_erf(x + b1) * w2 + b2."""
    return (gelu_erf(np.asarray(x, np.float32) + b1) @ np.asarray(w2, np.float32) + np.float32(b2)).astype(np.float32)


def unshuffle(x, ph, pw, C):
    """cuda/kernels.cu:517-525: [ph*pw, C] -> [(ph/2)*(pw/2), 4C], quadrant order (0,0),(0,1),(1,0),(1,1)."""
    x = np.asarray(x).reshape(ph // 2, 2, pw // 2, 2, C)
    return x.transpose(0, 2, 1, 3, 4).reshape((ph // 2) * (pw // 2), 4 * C)


# ------------------------------------------------------------------------------------------------ text model

def work_spans(seqs):
    return [(s, n) for s, n in seqs]


def trunk(w, h, spans, pos, prec="f16", fused_swiglu=True, prefix=None, prefix_pass=False):
    """src/model.rs:355-399. h: fp32 [T, D] residual (modified copy returned). spans: [(start, len)].
    prefix: per sequence None or dict(k=[n_attn][len][512], v=..., bx=[n_conv][D]) of a cached media prefix.
    prefix_pass: stop after the last layer's mixer and return the saved per-sequence K/V/bx (src/model.rs:370-372).
    fused_swiglu: model the fused GEMM epilogue (g and u rounded to fp16, the product rounded once), which is
    also exactly what the reference's GEMM + k_swiglu compute."""
    h = np.array(h, np.float32, copy=True)
    T = h.shape[0]
    eps = w["eps"]
    rope = w["rope"]
    n_attn = sum(1 for l in w["layers"] if l["is_attn"])
    n_conv = len(w["layers"]) - n_attn
    saves = {"k": [[None] * n_attn for _ in spans], "v": [[None] * n_attn for _ in spans],
             "bx": [[None] * n_conv for _ in spans]}
    ai = ci = 0
    nl = len(w["layers"])
    for li, l in enumerate(w["layers"]):
        last = li + 1 == nl
        xn = r16(rmsnorm(h, l["op_norm"], eps), prec)
        if not l["is_attn"]:
            big = r16(gemm(xn, l["in_proj"]), prec)
            ext = [p["bx"][ci] if p is not None else None for p in prefix] if prefix is not None else None
            act, saved = shortconv(big, l["convw"], spans, ci, ext, prec)
            act = r16(act, prec)
            if prefix_pass:
                for i in range(len(spans)):
                    saves["bx"][i][ci] = saved[i]
            if prefix_pass and last:
                return h, saves
            h = gemm(act, l["out_proj"], h, 1.0, 1.0)
            ci += 1
        else:
            big = r16(gemm(xn, l["qkv"]), prec)
            big = qk_norm_rope(big, HEADS, KV_HEADS, l["qn"], l["kn"], rope, pos, eps, prec)
            q, k, v = big[:, :D], big[:, D:D + KV_DIM], big[:, D + KV_DIM:]
            if prefix_pass:
                for i, (s, n) in enumerate(spans):
                    saves["k"][i][ai] = k[s:s + n].copy()
                    saves["v"][i][ai] = v[s:s + n].copy()
            ext = None
            if prefix is not None:
                ext = [(p["k"][ai], p["v"][ai]) if p is not None else None for p in prefix]
            seqs = [(s, n, s, n) for s, n in spans]
            act = r16(attention(q, k, v, seqs, HEADS, HEADS // KV_HEADS, 0.125, ext=ext, prec=prec), prec)
            if prefix_pass and last:
                return h, saves
            h = gemm(act, l["out"], h, 1.0, 1.0)
            ai += 1
        xn = r16(rmsnorm(h, l["ffn_norm"], eps), prec)
        F = l["ffn"]
        gu = r16(gemm(xn, l["gate_up"]), prec)
        act = r16(swiglu(gu, F), prec)
        h = gemm(act, l["down"], h, 1.0, 1.0)
    return h, saves


def launch_text(w, batch, prec="f16"):
    """src/model.rs:470-599 for a list of sequences dict(ids, markers, qtype[, prefix]) -> logits per marker
    (sequence order, then marker order)."""
    spans, ids, pos, row_qtype, mrows, mspans = [], [], [], [], [], []
    prefix = []
    start = 0
    for s in batch:
        n = len(s["ids"])
        spans.append((start, n))
        ids.extend(s["ids"])
        off = s["prefix"]["len"] if s.get("prefix") is not None else 0
        pos.extend(range(off, off + n))
        row_qtype.extend([s["qtype"]] * n)
        mspans.append((len(mrows), len(s["markers"])))
        mrows.extend(start + m for m in s["markers"])
        prefix.append(s.get("prefix"))
        start += n
    T = start
    h = embed(w["embed"], ids)
    h, _ = trunk(w, h, spans, np.asarray(pos), prec, prefix=prefix if any(p is not None for p in prefix) else None)
    h = head_init(h, w["final_norm"], w["type_emb"], np.asarray(row_qtype), w["eps"])
    pend = None
    nh = len(w["head"])
    mrows = np.asarray(mrows, dtype=np.int64)
    logits = np.zeros(len(mrows), np.float32)
    for li, l in enumerate(w["head"]):
        h, xn = layernorm(h, l["n1_w"], l["n1_b"], 1e-5, pend)
        xn = r16(xn, prec)
        big = r16(gemm(xn, l["qkv"]), prec)
        qb = l["qkv_b"]
        if li + 1 < nh:
            seqs = [(s, n, s, n) for s, n in spans]
            act = r16(attention(big[:, :D], big[:, D:2 * D], big[:, 2 * D:], seqs, HEADS, 1, 0.125,
                                qb[:D], qb[D:2 * D], qb[2 * D:], prec=prec), prec)
            h = gemm(act, l["out"], h, 1.0, 1.0)
            h, xn = layernorm(h, l["n2_w"], l["n2_b"], 1e-5, l["out_b"])
            xn = r16(xn, prec)
            up = r16(bias_act(r16(gemm(xn, l["up"]), prec), l["up_b"], 1), prec)
            h = gemm(up, l["down"], h, 1.0, 1.0)
            pend = l["down_b"]
        else:
            if len(mrows) == 0:
                break
            mq = big[mrows]
            mh = h[mrows]
            seqs = [(ms, mn, s, n) for (ms, mn), (s, n) in zip(mspans, spans)]
            mo = r16(attention(mq[:, :D], big[:, D:2 * D], big[:, 2 * D:], seqs, HEADS, 1, 0.125,
                               qb[:D], qb[D:2 * D], qb[2 * D:], prec=prec), prec)
            mh = gemm(mo, l["out"], mh, 1.0, 1.0)
            mh, mx = layernorm(mh, l["n2_w"], l["n2_b"], 1e-5, l["out_b"])
            mx = r16(mx, prec)
            mbig = r16(bias_act(r16(gemm(mx, l["up"]), prec), l["up_b"], 1), prec)
            mh = gemm(mbig, l["down"], mh, 1.0, 1.0)
            mh, mx = layernorm(mh, w["cls_norm_w"], w["cls_norm_b"], 1e-5, l["down_b"])
            mx = r16(mx, prec)
            mo = r16(gemm(mx, w["cls_w"]), prec)
            logits = scorer_out(mo, w["cls_b"], w["out_w"], w["out_b"])
    return logits


def launch_prefix(w, embs, prec="f16"):
    """src/model.rs:402-459: run media embeddings [len, D] (fp32) through the trunk, saving per attention layer
    K/V and the last conv state. Returns one cache dict(len, k, v, bx) per item."""
    spans, start, pos = [], 0, []
    for e in embs:
        spans.append((start, e.shape[0]))
        pos.extend(range(e.shape[0]))
        start += e.shape[0]
    h = np.concatenate([np.asarray(e, np.float32) for e in embs])
    _, saves = trunk(w, h, spans, np.asarray(pos), prec, prefix_pass=True)
    return [{"len": n, "k": saves["k"][i], "v": saves["v"][i], "bx": saves["bx"][i]}
            for i, (s, n) in enumerate(spans)]


# ------------------------------------------------------------------------------------------------ vision

def aa_weights(inp, out):
    """src/vision.rs:173-196: separable antialiased bilinear weights (first input index, normalised weights)."""
    scale = inp / out
    support = scale if scale >= 1.0 else 1.0
    invscale = 1.0 / scale if scale >= 1.0 else 1.0
    res = []
    for i in range(out):
        center = scale * (i + 0.5)
        xmin = max(int(center - support + 0.5), 0)
        xmax = min(int(center + support + 0.5), inp)
        w = [max(0.0, 1.0 - abs((j - center + 0.5) * invscale)) for j in range(xmin, xmax)]
        t = sum(w)
        res.append((xmin, np.asarray([v / t if t else v for v in w], np.float32)))
    return res


def vision_pos(pos, patch_b, ph, pw):
    """src/vision.rs:263-302: the 16x16 position grid resized to (ph, pw) (horizontal then vertical pass) plus the
    patch bias; fp32 [ph*pw, 768]."""
    pos = np.asarray(pos, np.float32).reshape(16, 16, -1)
    tmp = np.zeros((16, pw, pos.shape[-1]), np.float32)
    for x, (s0, ws) in enumerate(aa_weights(16, pw)):
        for j, wt in enumerate(ws):
            tmp[:, x] += wt * pos[:, s0 + j]
    out = np.zeros((ph, pw, pos.shape[-1]), np.float32)
    for y, (s0, ws) in enumerate(aa_weights(16, ph)):
        for j, wt in enumerate(ws):
            out[y] += wt * tmp[s0 + j]
    return (out + patch_b).reshape(ph * pw, -1)


def vision_encode(w, crops, prec="f16"):
    """src/vision.rs:305-385. crops: [(ph, pw, patches fp16 [ph*pw, 768])] -> fp32 [sum ph*pw/4, 1024]."""
    VD = 768
    eps = float(w["eps"])
    h = np.concatenate([vision_pos(w["pos"], w["patch_b"], ph, pw) for ph, pw, _ in crops])
    pix = np.concatenate([np.asarray(c[2], np.float32) for c in crops])
    h = gemm(pix, w["patch_w"], h, 1.0, 1.0)
    spans, s = [], 0
    for ph, pw, _ in crops:
        spans.append((s, ph * pw, s, ph * pw))
        s += ph * pw
    pend = None
    for l in w["layers"]:
        h, xn = layernorm(h, l["ln1_w"], l["ln1_b"], eps, pend)
        xn = r16(xn, prec)
        big = r16(gemm(xn, l["qkv"]), prec)
        b = l["qkv_b"]
        act = r16(attention(big[:, :VD], big[:, VD:2 * VD], big[:, 2 * VD:], spans, 12, 1, 0.125,
                            b[:VD], b[VD:2 * VD], b[2 * VD:], prec=prec), prec)
        h = gemm(act, l["out"], h, 1.0, 1.0)
        h, xn = layernorm(h, l["ln2_w"], l["ln2_b"], eps, l["out_b"])
        xn = r16(xn, prec)
        big = r16(bias_act(r16(gemm(xn, l["fc1"]), prec), l["fc1_b"], 3), prec)
        h = gemm(big, l["fc2"], h, 1.0, 1.0)
        pend = l["fc2_b"]
    h, xn = layernorm(h, w["post_w"], w["post_b"], eps, pend)
    xn = r16(xn, prec)
    parts, s = [], 0
    for ph, pw, _ in crops:
        parts.append(unshuffle(xn[s:s + ph * pw], ph, pw, VD))
        s += ph * pw
    big = np.concatenate(parts)
    act = r16(bias_act(r16(gemm(big, w["proj1"]), prec), w["proj1_b"], 2), prec)
    return gemm(act, w["proj2"], np.broadcast_to(w["proj2_b"], (act.shape[0], 1024)), 1.0, 1.0)


# ------------------------------------------------------------------------------------------------ audio

AD = 512          # src/audio.rs:16
AHEADS = 8        # :17
SUB_C = 256       # :18
N_MELS = 128      # :15
A_MAX_T = 384     # :401


def sub_conv0(mel, valid, w, b, Tout, Fout):
    """cuda/kernels.cu:529-545: 3x3 stride-2 conv (pad 1) from 1 to 256 channels over the valid mel rows, ReLU;
    mel [>= valid, F] -> [Tout, Fout, 256] fp32."""
    mel = np.asarray(mel, np.float32)
    F = mel.shape[1]
    xp = np.zeros((2 * Tout + 2, max(F, 2 * Fout) + 2), np.float32)
    xp[1:1 + min(valid, 2 * Tout + 1), 1:1 + F] = mel[:min(valid, 2 * Tout + 1)]
    patches = np.stack([xp[dt:dt + 2 * Tout:2, df:df + 2 * Fout:2] for dt in range(3) for df in range(3)], -1)
    return np.maximum(patches @ np.asarray(w, np.float32).T + b, 0).astype(np.float32)


def sub_dwconv(x, tin_valid, w, b, Tout, Fout):
    """cuda/kernels.cu:548-564: depthwise 3x3 stride-2 conv (pad 1) on [Tin, Fin, 256] -> [Tout, Fout, 256]."""
    x = np.asarray(x, np.float32)
    Fin = x.shape[1]
    xp = np.zeros((2 * Tout + 2, max(Fin, 2 * Fout) + 2, x.shape[2]), np.float32)
    n = min(tin_valid, 2 * Tout + 1)
    xp[1:1 + n, 1:1 + Fin] = x[:n]
    out = np.broadcast_to(np.asarray(b, np.float32), (Tout, Fout, x.shape[2])).copy()
    for dt in range(3):
        for df in range(3):
            out += w[:, dt * 3 + df] * xp[dt:dt + 2 * Tout:2, df:df + 2 * Fout:2]
    return out


def relpos_prep(qkv, bq, bk, bv, pu, pv, prec="f16"):
    """cuda/kernels.cu:567-580: qu = q+bq+u, qv = q+bq+v, k+bk, v+bv (fp16 outputs in the F16 engine)."""
    qkv = np.asarray(qkv, np.float32)
    q = qkv[:, :AD] + bq
    return (r16(q + pu, prec), r16(q + pv, prec), r16(qkv[:, AD:2 * AD] + bk, prec), r16(qkv[:, 2 * AD:] + bv, prec))


def relpos_pe(t):
    """src/audio.rs:546-558: sinusoid rows for relative positions t-1 .. -(t-1), [2t-1, 512] (fp16 values):
    row n, columns (2i, 2i+1) = sin, cos of (t-1-n) * exp(2i * -(ln 10000 / 512)) (fp32 angle, f64 sin/cos)."""
    c = np.float32(-(math.log(10000.0) / AD))
    div = np.exp(np.arange(0, AD, 2, dtype=np.float32) * c).astype(np.float32)
    p = (t - 1 - np.arange(2 * t - 1)).astype(np.float32)
    a = (p[:, None] * div[None, :]).astype(np.float32).astype(np.float64)
    pe = np.empty((2 * t - 1, AD), np.float32)
    pe[:, 0::2] = np.sin(a).astype(np.float32)
    pe[:, 1::2] = np.cos(a).astype(np.float32)
    return pe.astype(np.float16).astype(np.float32)


def relpos_attention(qu, qv, k, v, pp, scale=0.125, prec="f16"):
    """src/audio.rs:567-571 with cuda/kernels.cu:583-616: per head, ac = qu.k^T and bd = qv.pp^T (fp32), score
    (i, j) = (ac[i, j] + bd[i, j + T-1-i]) * scale, row softmax, probs fp16, O = probs.V (fp16 out)."""
    T = qu.shape[0]
    i = np.arange(T)[:, None]
    j = np.arange(T)[None, :]
    out = np.empty((T, AD), np.float32)
    for h in range(AHEADS):
        c = slice(h * 64, h * 64 + 64)
        ac = np.asarray(qu[:, c], np.float32) @ np.asarray(k[:, c], np.float32).T
        bd = np.asarray(qv[:, c], np.float32) @ np.asarray(pp[:, c], np.float32).T
        s = (ac + bd[i, j + T - 1 - i]) * np.float32(scale)
        e = np.exp(s - s.max(-1, keepdims=True))
        p = r16(e / e.sum(-1, keepdims=True), prec)
        out[:, c] = p @ np.asarray(v[:, c], np.float32)
    return r16(out, prec)


def conformer_dw(a, b1, dw, dwb, bn_s, bn_b, ksize=9, prec="f16"):
    """cuda/kernels.cu:620-637: GLU of the pw1 output (+bias), depthwise conv (zero pad, 'same'), bias, batch-norm
    affine, SiLU; a [T, 2C] -> [T, C]."""
    a = np.asarray(a, np.float32)
    C = a.shape[1] // 2
    T = a.shape[0]
    x = a[:, :C] + b1[:C]
    g = a[:, C:] + b1[C:]
    glu = (x / (np.float32(1) + np.exp(-g))).astype(np.float32)
    pad = (ksize - 1) // 2
    gp = np.zeros((T + 2 * pad, C), np.float32)
    gp[pad:pad + T] = glu
    acc = np.broadcast_to(np.asarray(dwb, np.float32), (T, C)).copy()
    for kk in range(ksize):
        acc += dw[:, kk] * gp[kk:kk + T]
    return r16(silu(acc * bn_s + bn_b), prec)


def audio_encode(w, mel, valid, prec="f16"):
    """src/audio.rs:505-594: one clip's normalised log-mel rows (the first `valid` of mel [frames, 128]) ->
    fp32 prefix embeddings [T, 1024], T = ceil(valid / 8)."""
    eps = float(w["eps"])
    l1 = (valid - 1) // 2 + 1
    l2 = (l1 - 1) // 2 + 1
    t = (l2 - 1) // 2 + 1
    s1 = sub_conv0(mel, valid, w["c0_w"], w["c0_b"], l1, 64)
    s2 = sub_dwconv(s1, l1, w["c2_w"], w["c2_b"], l2, 32)
    s3 = np.maximum(s2.reshape(-1, SUB_C) @ w["c3_w"].T + w["c3_b"], 0).astype(np.float32).reshape(l2, 32, SUB_C)
    s2 = sub_dwconv(s3, l2, w["c5_w"], w["c5_b"], t, 16)
    s1 = np.maximum(s2.reshape(-1, SUB_C) @ w["c6_w"].T + w["c6_b"], 0).astype(np.float32)
    x = (s1.reshape(t, 16 * SUB_C) @ w["pre_out"].T + w["pre_out_b"]).astype(np.float32)
    pe = relpos_pe(t)
    pend, pscale = None, 1.0
    for l in w["layers"]:
        x, xn = layernorm(x, l["ff1_n_w"], l["ff1_n_b"], eps, pend, pscale)
        big = r16(bias_act(r16(gemm(r16(xn, prec), l["ff1_up"]), prec), l["ff1_up_b"], 4), prec)
        x = gemm(big, l["ff1_down"], x, 0.5, 1.0)
        x, xn = layernorm(x, l["att_n_w"], l["att_n_b"], eps, l["ff1_down_b"], 0.5)
        big = r16(gemm(r16(xn, prec), l["qkv"]), prec)
        qu, qv, kk, vv = relpos_prep(big, l["bq"], l["bk"], l["bv"], l["pu"], l["pv"], prec)
        pp = r16(gemm(pe, l["pos"]), prec)
        o = relpos_attention(qu, qv, kk, vv, pp, 0.125, prec)
        x = gemm(o, l["out"], x, 1.0, 1.0)
        x, xn = layernorm(x, l["conv_n_w"], l["conv_n_b"], eps, l["out_b"])
        big = r16(gemm(r16(xn, prec), l["pw1"]), prec)
        o = conformer_dw(big, l["pw1_b"], l["dw"], l["dw_b"], l["bn_s"], l["bn_b"], 9, prec)
        x = gemm(o, l["pw2"], x, 1.0, 1.0)
        x, xn = layernorm(x, l["ff2_n_w"], l["ff2_n_b"], eps, l["pw2_b"])
        big = r16(bias_act(r16(gemm(r16(xn, prec), l["ff2_up"]), prec), l["ff2_up_b"], 4), prec)
        x = gemm(big, l["ff2_down"], x, 0.5, 1.0)
        _, x = layernorm(x, l["out_n_w"], l["out_n_b"], eps, l["ff2_down_b"], 0.5)  # norm_out replaces x
        pend, pscale = None, 1.0
    _, xn = layernorm(x, w["ad_n_w"], w["ad_n_b"], eps)
    big = r16(bias_act(r16(gemm(r16(xn, prec), w["ad1"]), prec), w["ad1_b"], 2), prec)
    out = gemm(big, w["ad2"], np.broadcast_to(w["ad2_b"], (t, 1024)), 1.0, 1.0)
    _, xn = layernorm(out, w["res_n_w"], w["res_n_b"], eps)
    big = r16(bias_act(r16(gemm(r16(xn, prec), w["res_down"]), prec), w["res_down_b"], 2), prec)
    out = gemm(big, w["res_up"], out, 1.0, 1.0)
    return bias_act(out, w["res_up_b"], 0)


def slaney_filterbank(n_fft=512, sr=16000, n_mels=N_MELS):
    """src/audio.rs:151-176: Slaney-scale triangular filters with area normalisation, [n_mels, n_fft/2+1] fp32."""
    f_sp, min_log_hz, logstep = 200.0 / 3.0, 1000.0, math.log(6.4) / 27.0
    min_log_mel = min_log_hz / f_sp

    def hz_to_mel(f):
        return min_log_mel + math.log(f / min_log_hz) / logstep if f >= min_log_hz else f / f_sp

    def mel_to_hz(m):
        return min_log_hz * math.exp(logstep * (m - min_log_mel)) if m >= min_log_mel else f_sp * m

    nb = n_fft // 2 + 1
    m0, m1 = hz_to_mel(0.0), hz_to_mel(sr / 2.0)
    mel_f = np.array([mel_to_hz(m0 + (m1 - m0) * i / (n_mels + 1)) for i in range(n_mels + 2)])
    freqs = np.arange(nb) * sr / n_fft
    w = np.zeros((n_mels, nb), np.float32)
    for i in range(n_mels):
        lower = -(mel_f[i] - freqs) / (mel_f[i + 1] - mel_f[i])
        upper = (mel_f[i + 2] - freqs) / (mel_f[i + 2] - mel_f[i + 1])
        enorm = np.float32(2.0 / (mel_f[i + 2] - mel_f[i]))
        w[i] = np.maximum(np.minimum(lower, upper), 0.0).astype(np.float32) * enorm
    return w


def resample_taps(src_rate, dst_rate):
    """src/audio.rs:113-140: the polyphase Kaiser-windowed sinc filter of resample(): (up, down, half, table) with
    table fp32 [up, 2*half + 1]; entry [p][j] = tap((j - half) - p/up), evaluated in f64 in the reference's order
    (cutoff * sinc * I0(beta * sqrt(1 - r^2)) / I0(beta), beta 8.6, I0 by its 49-term series) and rounded to fp32.
    The reference builds this table when up <= 4096 and evaluates the same tap() per sample otherwise (same
    values)."""
    g = math.gcd(src_rate, dst_rate)
    up, down = dst_rate // g, src_rate // g
    cutoff = min(up / down, 1.0) * 0.97
    half = int(math.ceil(32.0 / cutoff))

    def i0(x):
        s = t = 1.0
        for k in range(1, 50):
            y = x / (2.0 * k)
            t *= y * y
            s += t
        return s

    beta = 8.6
    i0b = i0(beta)
    taps = 2 * half + 1

    def tap(t):
        r = t / half
        if abs(r) >= 1.0:
            return 0.0
        sinc = 1.0 if t == 0.0 else math.sin(math.pi * t * cutoff) / (math.pi * t * cutoff)
        return cutoff * sinc * i0(beta * math.sqrt(1.0 - r * r)) / i0b

    table = np.empty((up, taps), np.float32)
    for ph in range(up):
        frac = ph / up
        for j in range(taps):
            table[ph, j] = np.float32(tap(float(j - half) - frac))
    return up, down, half, table


def resample(x, src_rate, dst_rate=16000):
    """src/audio.rs:108-148: output n reads input position n * down / up (phase (n * down) % up); the sum runs over
    the 2*half + 1 taps in order, skipping inputs outside the clip, as fp32 products added to an fp32 accumulator
    (no fused multiply-add, as the reference's Rust compiles it)."""
    x = np.asarray(x, np.float32)
    if src_rate == dst_rate or x.shape[0] == 0:
        return x.copy()
    up, down, half, table = resample_taps(src_rate, dst_rate)
    n_out = x.shape[0] * up // down
    pos = np.arange(n_out, dtype=np.int64) * down
    base, ph = pos // up, pos % up
    acc = np.zeros(n_out, np.float32)
    for j in range(2 * half + 1):
        idx = base - half + j
        ok = (idx >= 0) & (idx < x.shape[0])
        prod = (table[ph[ok], j] * x[idx[ok]]).astype(np.float32)
        acc[ok] = (acc[ok] + prod).astype(np.float32)
    return acc


def log_mel(samples):
    """src/audio.rs:238-299: pre-emphasis 0.97, centred 512-point frames (hop 160, 400-sample periodic-free Hann
    window centred in the frame), power spectrum, Slaney mel, ln(x + 2^-24), per-channel normalisation over the
    valid frames (unbiased std + 1e-5). Returns (fp32 [frames, 128], valid)."""
    x = np.asarray(samples, np.float32)[:30 * 16000]
    if x.shape[0] < 8000:
        x = np.concatenate([x, np.zeros(8000 - x.shape[0], np.float32)])
    n = x.shape[0]
    valid, frames = n // 160, 1 + n // 160
    y = np.empty(n, np.float32)
    y[0] = x[0]
    y[1:] = x[1:] - np.float32(0.97) * x[:-1]
    win = np.zeros(512)
    win[56:456] = 0.5 - 0.5 * np.cos(2.0 * math.pi * np.arange(400) / 399.0)
    yp = np.concatenate([np.zeros(256), y.astype(np.float64), np.zeros(512)])
    idx = np.arange(frames)[:, None] * 160 + np.arange(512)[None, :]
    spec = np.fft.rfft(yp[idx] * win, axis=1)
    pw = (spec.real ** 2 + spec.imag ** 2).astype(np.float32)
    out = np.log((pw @ slaney_filterbank().T).astype(np.float32) + np.float32(2.0 ** -24)).astype(np.float32)
    v = out[:valid].astype(np.float64)
    mean = v.mean(0)
    std = np.sqrt(((v - mean) ** 2).sum(0) / (valid - 1.0))
    std = np.where(np.isnan(std), 0.0, std)
    res = np.zeros_like(out)
    res[:valid] = ((v - mean) / (std + 1e-5)).astype(np.float32)
    return res, valid


# ------------------------------------------------------------------------------------------------ metrics

def centred_logit_err(ref_logits, logits, group_sizes):
    """tools/logit_err.py:6-14: per question (a group of option logits), max over options of the difference of
    centred log-probs; log-softmax is the logits minus a constant, so centring the logits is equivalent."""
    errs, o = [], 0
    for n in group_sizes:
        a = np.asarray(ref_logits[o:o + n], np.float64)
        b = np.asarray(logits[o:o + n], np.float64)
        errs.append(float(np.max(np.abs((a - a.mean()) - (b - b.mean())))) if n else 0.0)
        o += n
    return np.asarray(errs)


def top_flips(ref_logits, logits, group_sizes):
    """tools/compare.py:10-15: questions whose top answer differs."""
    flips, o = 0, 0
    for n in group_sizes:
        if n and int(np.argmax(ref_logits[o:o + n])) != int(np.argmax(logits[o:o + n])):
            flips += 1
        o += n
    return flips
