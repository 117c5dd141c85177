"""Seeded synthetic weights and batches of the shapes the reference loads (numpy only, no GPU).

There is no network and no GGUF file here, so every benchmark and parity check runs on random-init weights of the
d1-omni-600M architecture (the reference's BASELINE configs): weights N(0, 0.02) rounded to fp16 (the F16 GGUF
stores fp16, src/model.rs:106-118), norm weights set to 1, biases N(0, 0.02).

The text trunk follows src/model.rs:139-231 (hidden 1024, 16 layers, attention at {2,5,8,10,12,14}, SwiGLU 4608,
vocab 65536). The decision head's sizes come from GGUF metadata in the reference (src/model.rs:145,193) and are not
given by the configs; this build fixes 2 head layers with a ReLU FFN of width 2048 and 4 question types.
"""
from __future__ import annotations

import numpy as np

D = 1024
KV_DIM = 512
ATTN_LAYERS = (2, 5, 8, 10, 12, 14)


class _Gen:
    """Each tensor draws from its own stream seeded by (seed, tensor index), so tensors can be generated in
    parallel threads and still come out the same on every machine."""

    def __init__(self, seed: int):
        self.seed = seed
        self.n = 0
        self.jobs = []

    def _rng(self):
        self.n += 1
        return np.random.default_rng([self.seed, self.n])

    def mat(self, *shape, std=0.02):
        rng = self._rng()
        out = np.empty(shape, np.float32)
        self.jobs.append((rng, out, std, True))
        return out

    def vec(self, n, std=0.02):
        rng = self._rng()
        out = np.empty(n, np.float32)
        self.jobs.append((rng, out, std, False))
        return out

    def run(self):
        from concurrent.futures import ThreadPoolExecutor

        def fill(job):
            rng, out, std, round16 = job
            v = rng.standard_normal(out.shape, dtype=np.float32)
            v *= np.float32(std)
            if round16:  # fp16-representable values, as the F16 GGUF stores them
                try:
                    import torch
                    v = torch.from_numpy(v).half().float().numpy()
                except Exception:  # pragma: no cover
                    v = v.astype(np.float16).astype(np.float32)
            out[...] = v

        with ThreadPoolExecutor(8) as ex:
            list(ex.map(fill, self.jobs))
        self.jobs.clear()


def _rope(theta):
    # same table as src/model.rs:121-136 (the runner builds its own on the device)
    e = (2.0 * np.arange(32, dtype=np.float32) / np.float32(64)).astype(np.float32)
    inv = (np.float32(1.0) / np.power(np.float32(theta), e, dtype=np.float32)).astype(np.float32)
    pos = np.arange(16384 + 64, dtype=np.float32)[:, None]
    ang = (pos * inv[None, :]).astype(np.float32).astype(np.float64)
    t = np.empty((16384 + 64, 32, 2), np.float32)
    t[..., 0] = np.cos(ang)
    t[..., 1] = np.sin(ang)
    return t


def text_weights(seed=0, n_layers=16, attn_layers=ATTN_LAYERS, ffn=4608, vocab=65536, n_head=2, head_ffn=2048,
                 n_types=4, eps=1e-5, rope_theta=1e6):
    """Weights in the layout the runner and the oracle take (matrices as fp16-valued float32 arrays)."""
    g = _Gen(seed)
    w = {"eps": np.float32(eps), "rope_theta": np.float32(rope_theta), "vocab": vocab}
    w["embed"] = g.mat(vocab, D)
    layers = []
    for i in range(n_layers):
        l = {"is_attn": i in attn_layers, "ffn": ffn,
             "op_norm": np.ones(D, np.float32), "ffn_norm": np.ones(D, np.float32)}
        if l["is_attn"]:
            l["qkv"] = g.mat(D + 2 * KV_DIM, D)   # [q; k; v] rows (src/model.rs:160)
            l["out"] = g.mat(D, D)
            l["qn"] = np.ones(64, np.float32)
            l["kn"] = np.ones(64, np.float32)
        else:
            l["in_proj"] = g.mat(3 * D, D)
            l["out_proj"] = g.mat(D, D)
            l["convw"] = g.vec(D * 3).reshape(D, 3)
        l["gate_up"] = g.mat(2 * ffn, D)           # [gate; up] rows (src/model.rs:184)
        l["down"] = g.mat(D, ffn)
        layers.append(l)
    w["layers"] = layers
    w["final_norm"] = np.ones(D, np.float32)
    w["type_emb"] = g.vec(n_types * D).reshape(n_types, D)
    head = []
    for _ in range(n_head):
        head.append({
            "n1_w": np.ones(D, np.float32), "n1_b": g.vec(D),
            "qkv": g.mat(3 * D, D), "qkv_b": g.vec(3 * D),
            "out": g.mat(D, D), "out_b": g.vec(D),
            "n2_w": np.ones(D, np.float32), "n2_b": g.vec(D),
            "up": g.mat(head_ffn, D), "up_b": g.vec(head_ffn),
            "down": g.mat(D, head_ffn), "down_b": g.vec(D), "ffn": head_ffn})
    w["head"] = head
    w["cls_norm_w"] = np.ones(D, np.float32)
    w["cls_norm_b"] = g.vec(D)
    w["cls_w"] = g.mat(D, D)
    w["cls_b"] = g.vec(D)
    w["out_w"] = g.mat(D, std=0.02)
    out_b = g.vec(1)
    g.run()
    w["out_b"] = np.float32(out_b[0])
    w["rope"] = _rope(rope_theta)
    return w


def text_batch(seed, n_seqs, seq_len=None, lengths=None, vocab=65536, n_markers=3, n_types=4):
    """A packed batch of question sequences: uniform token ids, n_markers distinct marker rows per sequence
    (option rows), a random question type. lengths overrides seq_len per sequence."""
    rng = np.random.default_rng(seed)
    if lengths is None:
        lengths = [seq_len] * n_seqs
    batch = []
    for n in lengths:
        ids = rng.integers(0, vocab, size=n, dtype=np.int32)
        k = min(n_markers, n)
        markers = np.sort(rng.choice(n, size=k, replace=False)).astype(np.int32)
        batch.append({"ids": ids, "markers": markers, "qtype": int(rng.integers(0, n_types))})
    return batch


def lognormal_lengths(seed, total, median=384, sigma=1.0, lo=32, hi=16384):
    """Per-sequence lengths drawn log-normal (median, sigma), clipped to [lo, hi], until they fill `total`
    tokens; the last one is cut to fit (sigma is not given there and is fixed to 1.0)."""
    rng = np.random.default_rng(seed)
    out, used = [], 0
    while used < total:
        n = int(np.clip(round(median * np.exp(sigma * rng.standard_normal())), lo, hi))
        n = min(n, total - used)
        out.append(n)
        used += n
    return out


def loguniform_lengths(seed, total, lo=128, hi=2048):
    """Text rows of 128-2048 tokens, log-uniform, packed up to `total` tokens."""
    rng = np.random.default_rng(seed)
    out, used = [], 0
    while True:
        n = int(round(np.exp(rng.uniform(np.log(lo), np.log(hi)))))
        if used + n > total:
            if total - used >= lo:
                out.append(total - used)
            break
        out.append(n)
        used += n
    return out


# ---------------------------------------------------------------------------------------------------- vision
VD, VFF, VHID, VOUT = 768, 3072, 2048, 1024


def vision_weights(seed=3, n_layers=12, eps=1e-6):
    """SigLIP2 tower + projector weights in the layout of src/vision.rs:198-260 (patch weight already in
    (y, x, c) input order, fused QKV rows [q; k; v]); BASELINE config 3 uses seed 3."""
    g = _Gen(seed)
    w = {"eps": np.float32(eps), "patch_w": g.mat(VD, VD), "patch_b": g.vec(VD), "pos": g.vec(256 * VD).reshape(256, VD)}
    layers = []
    for _ in range(n_layers):
        layers.append({"ln1_w": np.ones(VD, np.float32), "ln1_b": g.vec(VD), "qkv": g.mat(3 * VD, VD),
                       "qkv_b": g.vec(3 * VD), "out": g.mat(VD, VD), "out_b": g.vec(VD),
                       "ln2_w": np.ones(VD, np.float32), "ln2_b": g.vec(VD), "fc1": g.mat(VFF, VD), "fc1_b": g.vec(VFF),
                       "fc2": g.mat(VD, VFF), "fc2_b": g.vec(VD)})
    w["layers"] = layers
    w["post_w"] = np.ones(VD, np.float32)
    w["post_b"] = g.vec(VD)
    w["proj1"] = g.mat(VHID, 4 * VD)
    w["proj1_b"] = g.vec(VHID)
    w["proj2"] = g.mat(VOUT, VHID)
    w["proj2_b"] = g.vec(VOUT)
    g.run()
    return w


def vision_crops(seed=3, n_images=16, lo=224, hi=768):
    """images with sides uniform in [lo, hi] rounded to multiples of 32, pixels uniform in
    [0, 1] fed directly as 16x16x3 patch rows in (y, x, c) order (the layout() tiling is bypassed).
    Returns [(ph, pw, fp16 patches [ph*pw, 768])]."""
    rng = np.random.default_rng(seed)
    crops = []
    for _ in range(n_images):
        hh, ww = (int(round(rng.uniform(lo, hi) / 32.0)) * 32 for _ in range(2))
        ph, pw = hh // 16, ww // 16
        crops.append((ph, pw, rng.uniform(0.0, 1.0, size=(ph * pw, VD)).astype(np.float16)))
    return crops


# ------------------------------------------------------------------------------------------------ audio

AD = 512        # src/audio.rs:16 (DM)
AHEADS = 8      # :17
SUB_C = 256     # :18
AOUT = 1024     # :19
N_MELS = 128    # :15
A_MAX_T = 384   # :401


def audio_weights(seed=4, n_layers=17, eps=1e-5):
    """FastConformer encoder + adapter weights in the layout src/audio.rs:302-455 builds on the device: fused QKV
    rows [q; k; v], pos_bias_u/v flattened [8*64], the pre-encode output weight with its columns already in the
    (f, c) order the subsampled activations use, subsampling convs fp32 [256][9] / [256][256]. Subsampling
    weights use std 1/sqrt(fan_in) so the fp32 front keeps unit scale; the rest follow the text weights' recipe
    (matrices N(0, 0.02) as fp16 values, norm weights 1, batch-norm scale 1 + N(0, 0.02))."""
    g = _Gen(seed)
    w = {"eps": np.float32(eps)}
    w["c0_w"], w["c0_b"] = g.vec(SUB_C * 9, 1 / 3).reshape(SUB_C, 9), g.vec(SUB_C)
    w["c2_w"], w["c2_b"] = g.vec(SUB_C * 9, 1 / 3).reshape(SUB_C, 9), g.vec(SUB_C)
    w["c3_w"], w["c3_b"] = g.vec(SUB_C * SUB_C, 1 / 16).reshape(SUB_C, SUB_C), g.vec(SUB_C)
    w["c5_w"], w["c5_b"] = g.vec(SUB_C * 9, 1 / 3).reshape(SUB_C, 9), g.vec(SUB_C)
    w["c6_w"], w["c6_b"] = g.vec(SUB_C * SUB_C, 1 / 16).reshape(SUB_C, SUB_C), g.vec(SUB_C)
    w["pre_out"], w["pre_out_b"] = g.vec(AD * 16 * SUB_C, 1 / 64).reshape(AD, 16 * SUB_C), g.vec(AD)
    one = lambda n: np.ones(n, np.float32)  # noqa: E731
    layers = []
    for _ in range(n_layers):
        layers.append({
            "ff1_n_w": one(AD), "ff1_n_b": g.vec(AD), "ff1_up": g.mat(4 * AD, AD), "ff1_up_b": g.vec(4 * AD),
            "ff1_down": g.mat(AD, 4 * AD), "ff1_down_b": g.vec(AD),
            "att_n_w": one(AD), "att_n_b": g.vec(AD), "qkv": g.mat(3 * AD, AD),
            "bq": g.vec(AD), "bk": g.vec(AD), "bv": g.vec(AD), "pu": g.vec(AD), "pv": g.vec(AD),
            "pos": g.mat(AD, AD), "out": g.mat(AD, AD), "out_b": g.vec(AD),
            "conv_n_w": one(AD), "conv_n_b": g.vec(AD), "pw1": g.mat(2 * AD, AD), "pw1_b": g.vec(2 * AD),
            "dw": g.vec(AD * 9, 1 / 3).reshape(AD, 9), "dw_b": g.vec(AD), "bn_s": g.vec(AD), "bn_b": g.vec(AD),
            "pw2": g.mat(AD, AD), "pw2_b": g.vec(AD),
            "ff2_n_w": one(AD), "ff2_n_b": g.vec(AD), "ff2_up": g.mat(4 * AD, AD), "ff2_up_b": g.vec(4 * AD),
            "ff2_down": g.mat(AD, 4 * AD), "ff2_down_b": g.vec(AD),
            "out_n_w": one(AD), "out_n_b": g.vec(AD)})
    w["layers"] = layers
    w["ad_n_w"], w["ad_n_b"] = one(AD), g.vec(AD)
    w["ad1"], w["ad1_b"] = g.mat(AOUT, AD), g.vec(AOUT)
    w["ad2"], w["ad2_b"] = g.mat(AOUT, AOUT), g.vec(AOUT)
    w["res_n_w"], w["res_n_b"] = one(AOUT), g.vec(AOUT)
    w["res_down"], w["res_down_b"] = g.mat(AD, AOUT), g.vec(AD)
    w["res_up"], w["res_up_b"] = g.mat(AOUT, AD), g.vec(AOUT)
    g.run()
    for l in layers:
        l["bn_s"] += np.float32(1.0)
    return w


def audio_clip_frames(n_samples: int) -> int:
    """Valid mel frames of a clip (src/audio.rs:241-249: capped at 30 s, padded to 0.5 s, hop 160)."""
    n = min(max(n_samples, 8000), 30 * 16000)
    return n // 160


def audio_out_len(valid: int) -> int:
    """Encoder output rows for `valid` mel frames: three stride-2 stages (src/audio.rs:506-509)."""
    l1 = (valid - 1) // 2 + 1
    l2 = (l1 - 1) // 2 + 1
    return (l2 - 1) // 2 + 1


def audio_clips(seed=4, n_clips=4, lo_s=1.0, hi_s=30.0):
    """BASELINE config 4's audio: clips of 1-30 s of N(0, 0.1) waveform at 16 kHz (float32 samples)."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n_clips):
        n = int(round(rng.uniform(lo_s, hi_s) * 16000))
        out.append((rng.standard_normal(n, dtype=np.float32) * np.float32(0.1)).astype(np.float32))
    return out


def mixed_requests(seed=4, n_requests=64, vocab=65536, n_types=4, questions=3, options=4):
    """a mixed request stream for the continuous-batching engine (engine.py request dicts).
    70% text (each question 128-2048 tokens, log-uniform), 20% text+image (one image with config-3 sides, uniform
    in 224-768 px rounded to 32, pixels U[0, 1] as 16x16x3 patch rows; questions 128-896 tokens, the reference's
    image_text_length), 10% text+audio (1-30 s of N(0, 0.1) waveform at 16 kHz, features computed by the engine;
    questions 128-2048 tokens). Every request carries `questions` questions with `options` answer markers each,
    at distinct sorted positions; question types uniform in [0, n_types)."""
    rng = np.random.default_rng(seed)
    reqs = []
    for _ in range(n_requests):
        u = rng.uniform()
        kind = "text" if u < 0.7 else "images" if u < 0.9 else "audio"
        hi = 896 if kind == "images" else 2048
        rows = []
        for _ in range(questions):
            n = int(round(np.exp(rng.uniform(np.log(128), np.log(hi)))))
            ids = rng.integers(0, vocab, size=n, dtype=np.int32)
            markers = np.sort(rng.choice(n, size=options, replace=False)).astype(np.int32)
            rows.append({"ids": ids, "markers": markers, "qtype": int(rng.integers(0, n_types))})
        media = None
        if kind == "images":
            hh, ww = (int(round(rng.uniform(224, 768) / 32.0)) * 32 for _ in range(2))
            ph, pw = hh // 16, ww // 16
            media = {"kind": "images", "crops": [(ph, pw, rng.uniform(0.0, 1.0, size=(ph * pw, VD)).astype(np.float16))]}
        elif kind == "audio":
            n = int(round(rng.uniform(1.0, 30.0) * 16000))
            media = {"kind": "audio", "pcm": (rng.standard_normal(n, dtype=np.float32) * np.float32(0.1))}
        reqs.append({"rows": rows, "media": media})
    return reqs
