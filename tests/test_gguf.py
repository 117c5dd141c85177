"""GGUF loading (fast_d1_omni_b200.gguf) against files written by a test-side GGUF writer.

The writer below emits GGUF v2/v3 containers as the format defines them (header, typed metadata, tensor infos with
ggml dims, aligned tensor data) with the tensor names the reference's loaders read (src/model.rs:139-231,
src/vision.rs:198-260, src/audio.rs:403-455). CPU tests: every metadata type, every tensor type the reference
decodes (F32, F16, BF16, Q8_0; src/gguf.rs:186-214) against the reference's conversion formulas restated in numpy,
the error cases, and each model mapping back to the dict it was written from. GPU tests: models loaded from GGUF against
the same models built from the dicts. The two are not bit-identical: split-K tiles add into fp32 residuals in
arrival order, and the encoders tune their GEMM plans per instance by timing, so the text logits agree within 2e-3
(the engine tests' run-to-run bound) and the encoder outputs to a relative RMS of 5e-3 — a wrong mapping (a
transposed patch or pre-encode weight, swapped q/k/v) is off by O(1).
"""
import struct

import numpy as np
import pytest

from fast_d1_omni_b200 import gguf as G
from fast_d1_omni_b200 import weights as W

# --------------------------------------------------------------------------------------------- the writer
_FMT = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


def _enc_str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _enc_value(t, v):
    if t in _FMT:
        return struct.pack(_FMT[t], v)
    if t == 8:
        return _enc_str(v)
    et, items = v  # arrays: (element type, list)
    out = struct.pack("<IQ", et, len(items))
    for it in items:
        out += _enc_value(et, it)
    return out


def q8_0_encode(x):
    """Q8_0 blocks (fp16 scale d = max|x|/127, int8 round(x/d)) of a flat array whose length is a multiple of 32."""
    x = np.asarray(x, np.float32).reshape(-1, 32)
    d = (np.abs(x).max(axis=1) / 127.0).astype(np.float16)
    df = d.astype(np.float32)
    q = np.where(df[:, None] > 0, np.rint(x / np.where(df > 0, df, 1)[:, None]), 0).clip(-127, 127).astype(np.int8)
    blk = np.empty((x.shape[0], 34), np.uint8)
    blk[:, :2] = d.view(np.uint8).reshape(-1, 2)
    blk[:, 2:] = q.view(np.uint8)
    return blk.tobytes()


def encode_tensor(a, ty):
    a = np.asarray(a)
    if ty == G.GGML_F32:
        return np.ascontiguousarray(a, np.float32).tobytes()
    if ty == G.GGML_F16:
        return np.ascontiguousarray(a, np.float16).tobytes()
    if ty == G.GGML_BF16:  # round to nearest even on the upper 16 bits
        u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16).tobytes()
    if ty == G.GGML_Q8_0:
        return q8_0_encode(a)
    raise ValueError(ty)


class Writer:
    def __init__(self, version=3, alignment=None):
        self.version = version
        self.alignment = alignment
        self.meta = []
        self.tensors = []
        if alignment is not None:
            self.kv("general.alignment", 4, alignment)

    def kv(self, key, t, v):
        self.meta.append((key, t, v))
        return self

    def tensor(self, name, a, ty=G.GGML_F16, shape=None):
        a = np.asarray(a)
        shape = list(a.shape if shape is None else shape)
        self.tensors.append((name, shape, ty, encode_tensor(a, ty)))
        return self

    def write(self, path):
        align = self.alignment or 32
        head = b"GGUF" + struct.pack("<IQQ", self.version, len(self.tensors), len(self.meta))
        for k, t, v in self.meta:
            head += _enc_str(k) + struct.pack("<I", t) + _enc_value(t, v)
        off, infos, blobs = 0, b"", []
        for name, shape, ty, data in self.tensors:
            infos += _enc_str(name) + struct.pack("<I", len(shape))
            infos += b"".join(struct.pack("<Q", d) for d in reversed(shape))  # ggml order: contiguous dim first
            infos += struct.pack("<IQ", ty, off)
            pad = (-len(data)) % align
            blobs.append(data + b"\0" * pad)
            off += len(data) + pad
        head += infos
        head += b"\0" * ((-len(head)) % align)
        with open(path, "wb") as f:
            f.write(head)
            for b in blobs:
                f.write(b)
        return path


# -------------------------------------------------------------------------- writers for the three models
def write_text(path, w, ty=G.GGML_F16):
    wr = Writer().kv("general.architecture", 8, "lfm2").kv("lfm2.block_count", 4, len(w["layers"]) + len(w["head"]))
    wr.kv("lfm2.decision.block_count", 4, len(w["head"]))
    wr.kv("lfm2.attention.layer_norm_rms_epsilon", 6, float(w["eps"])).kv("lfm2.rope.freq_base", 6, float(w["rope_theta"]))
    f32 = G.GGML_F32
    for i, l in enumerate(w["layers"]):
        t = f"blk.{i}."
        wr.tensor(t + "attn_norm.weight", l["op_norm"], f32).tensor(t + "ffn_norm.weight", l["ffn_norm"], f32)
        ffn = l["ffn"]
        wr.tensor(t + "ffn_gate.weight", l["gate_up"][:ffn], ty).tensor(t + "ffn_up.weight", l["gate_up"][ffn:], ty)
        wr.tensor(t + "ffn_down.weight", l["down"], ty)
        if l["is_attn"]:
            q, k, v = np.split(l["qkv"], [W.D, W.D + W.KV_DIM])
            wr.tensor(t + "attn_q.weight", q, ty).tensor(t + "attn_k.weight", k, ty).tensor(t + "attn_v.weight", v, ty)
            wr.tensor(t + "attn_output.weight", l["out"], ty)
            wr.tensor(t + "attn_q_norm.weight", l["qn"], f32).tensor(t + "attn_k_norm.weight", l["kn"], f32)
        else:
            wr.tensor(t + "shortconv.in_proj.weight", l["in_proj"], ty)
            wr.tensor(t + "shortconv.out_proj.weight", l["out_proj"], ty)
            wr.tensor(t + "shortconv.conv.weight", l["convw"], f32)
    for j, l in enumerate(w["head"]):
        t = f"blk.{len(w['layers']) + j}."
        for k, n in (("n1", "attn_norm"), ("n2", "ffn_norm")):
            wr.tensor(t + n + ".weight", l[k + "_w"], f32).tensor(t + n + ".bias", l[k + "_b"], f32)
        for k, n in (("qkv", "attn_qkv"), ("out", "attn_output"), ("up", "ffn_up"), ("down", "ffn_down")):
            wr.tensor(t + n + ".weight", l[k], ty).tensor(t + n + ".bias", l[k + "_b"], f32)
    wr.tensor("token_embd.weight", w["embed"], ty).tensor("token_embd_norm.weight", w["final_norm"], f32)
    wr.tensor("token_types.weight", w["type_emb"], f32)
    wr.tensor("cls.norm.weight", w["cls_norm_w"], f32).tensor("cls.norm.bias", w["cls_norm_b"], f32)
    wr.tensor("cls.weight", w["cls_w"], ty).tensor("cls.bias", w["cls_b"], f32)
    wr.tensor("cls.output.weight", np.asarray(w["out_w"]).reshape(1, -1), ty)
    wr.tensor("cls.output.bias", np.array([w["out_b"]], np.float32), f32)
    return wr.write(path)


def write_vision(wr, w, ty=G.GGML_F16):
    f32 = G.GGML_F32
    wr.kv("clip.vision.block_count", 4, len(w["layers"])).kv("clip.vision.attention.layer_norm_epsilon", 6, float(w["eps"]))
    pw = np.asarray(w["patch_w"]).reshape(768, 16, 16, 3).transpose(0, 3, 1, 2)  # (y, x, c) -> (c, y, x)
    wr.tensor("v.patch_embd.weight", np.ascontiguousarray(pw), f32).tensor("v.patch_embd.bias", w["patch_b"], f32)
    wr.tensor("v.position_embd.weight", w["pos"], f32)
    for i, l in enumerate(w["layers"]):
        t = f"v.blk.{i}."
        qkv, qkv_b = np.split(l["qkv"], 3), np.split(l["qkv_b"], 3)
        for n, m, b in zip(("attn_q", "attn_k", "attn_v"), qkv, qkv_b):
            wr.tensor(t + n + ".weight", m, ty).tensor(t + n + ".bias", b, f32)
        for k, n in (("out", "attn_out"), ("fc1", "ffn_up"), ("fc2", "ffn_down")):
            wr.tensor(t + n + ".weight", l[k], ty).tensor(t + n + ".bias", l[k + "_b"], f32)
        for k, n in (("ln1", "ln1"), ("ln2", "ln2")):
            wr.tensor(t + n + ".weight", l[k + "_w"], f32).tensor(t + n + ".bias", l[k + "_b"], f32)
    wr.tensor("v.post_ln.weight", w["post_w"], f32).tensor("v.post_ln.bias", w["post_b"], f32)
    wr.tensor("mm.1.weight", w["proj1"], ty).tensor("mm.1.bias", w["proj1_b"], f32)
    wr.tensor("mm.2.weight", w["proj2"], ty).tensor("mm.2.bias", w["proj2_b"], f32)
    return wr


_AUDIO_LAYER = (  # (dict key, GGUF suffix, is a matrix)
    ("ff1_n_w", "ffn_norm.weight", 0), ("ff1_n_b", "ffn_norm.bias", 0), ("ff1_up", "ffn_up.weight", 1),
    ("ff1_up_b", "ffn_up.bias", 0), ("ff1_down", "ffn_down.weight", 1), ("ff1_down_b", "ffn_down.bias", 0),
    ("att_n_w", "ln1.weight", 0), ("att_n_b", "ln1.bias", 0), ("bq", "attn_q.bias", 0), ("bk", "attn_k.bias", 0),
    ("bv", "attn_v.bias", 0), ("pu", "pos_bias_u", 0), ("pv", "pos_bias_v", 0), ("pos", "linear_pos.weight", 1),
    ("out", "attn_out.weight", 1), ("out_b", "attn_out.bias", 0), ("conv_n_w", "norm_conv.weight", 0),
    ("conv_n_b", "norm_conv.bias", 0), ("pw1", "conv_pw1.weight", 1), ("pw1_b", "conv_pw1.bias", 0),
    ("dw", "conv_dw.weight", 0), ("dw_b", "conv_dw.bias", 0), ("bn_s", "conv_norm.weight", 0),
    ("bn_b", "conv_norm.bias", 0), ("pw2", "conv_pw2.weight", 1), ("pw2_b", "conv_pw2.bias", 0),
    ("ff2_n_w", "ffn_norm_1.weight", 0), ("ff2_n_b", "ffn_norm_1.bias", 0), ("ff2_up", "ffn_up_1.weight", 1),
    ("ff2_up_b", "ffn_up_1.bias", 0), ("ff2_down", "ffn_down_1.weight", 1), ("ff2_down_b", "ffn_down_1.bias", 0),
    ("out_n_w", "ln2.weight", 0), ("out_n_b", "ln2.bias", 0))
_AUDIO_TOP = (("c0", "a.conv1d.0", (256, 1, 3, 3)), ("c2", "a.conv1d.2", (256, 1, 3, 3)),
              ("c3", "a.conv1d.3", (256, 256, 1, 1)), ("c5", "a.conv1d.5", (256, 1, 3, 3)),
              ("c6", "a.conv1d.6", (256, 256, 1, 1)))
_AUDIO_ADAPTER = (("ad_n", 0, 0), ("ad1", 1, 1), ("ad2", 3, 1), ("res_n", 4, 0), ("res_down", 5, 1), ("res_up", 6, 1))


def write_audio(wr, w, ty=G.GGML_F16):
    f32 = G.GGML_F32
    wr.kv("clip.audio.block_count", 4, len(w["layers"])).kv("clip.audio.attention.layer_norm_epsilon", 6, float(w["eps"]))
    for k, n, shape in _AUDIO_TOP:
        wr.tensor(n + ".weight", np.asarray(w[k + "_w"]).reshape(shape), f32).tensor(n + ".bias", w[k + "_b"], f32)
    pre = np.asarray(w["pre_out"]).reshape(512, 16, 256).transpose(0, 2, 1).reshape(512, 4096)  # (f, c) -> (c, f)
    wr.tensor("a.pre_encode.out.weight", np.ascontiguousarray(pre), f32)
    wr.tensor("a.pre_encode.out.bias", w["pre_out_b"], f32)
    for i, l in enumerate(w["layers"]):
        t = f"a.blk.{i}."
        q, k, v = np.split(l["qkv"], 3)
        wr.tensor(t + "attn_q.weight", q, ty).tensor(t + "attn_k.weight", k, ty).tensor(t + "attn_v.weight", v, ty)
        for key, n, mat in _AUDIO_LAYER:
            a = np.asarray(l[key])
            if key in ("pu", "pv"):
                a = a.reshape(8, 64)
            if key == "dw":
                a = a.reshape(512, 1, 9)
            wr.tensor(t + n, a, ty if mat else f32)
    for k, idx, mat in _AUDIO_ADAPTER:
        wa, wb = (k + "_w", k + "_b") if not mat else (k, k + "_b")
        wr.tensor(f"mm.a.mlp.{idx}.weight", w[wa], ty if mat else f32).tensor(f"mm.a.mlp.{idx}.bias", w[wb], f32)
    return wr


def assert_same_dict(got, want, path=""):
    assert set(got) >= set(want) - {"rope"}, (path, set(want) - set(got))
    for k, v in want.items():
        if k == "rope":
            continue
        g = got[k]
        if isinstance(v, dict):
            assert_same_dict(g, v, f"{path}.{k}")
        elif isinstance(v, list):
            assert len(g) == len(v), (path, k)
            for i, (a, b) in enumerate(zip(g, v)):
                assert_same_dict(a, b, f"{path}.{k}[{i}]")
        else:
            a, b = np.asarray(g), np.asarray(v)
            assert a.shape == b.shape or a.size == b.size == 1, (path, k, a.shape, b.shape)
            assert np.array_equal(a.astype(np.float32), b.astype(np.float32)), (path, k)


# ------------------------------------------------------------------------------------------- CPU tests
def restated_f32_to_f16(x):
    """The reference's f32 -> f16 bit conversion (round to nearest even, flush below half the smallest subnormal;
    src/cuda.rs:532-564), vectorised."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.int64)
    sign = (u >> 16) & 0x8000
    exp = (u >> 23) & 0xFF
    mant = u & 0x7FFFFF
    e = exp - 127 + 15
    r = (e << 10) | (mant >> 13)
    rest = mant & 0x1FFF
    r = np.where((rest > 0x1000) | ((rest == 0x1000) & (r & 1 == 1)), r + 1, r)
    m = mant | 0x800000
    shift = np.clip(14 - e, 1, 31)
    half = 1 << (shift - 1)
    sr = m >> shift
    srest = m & ((1 << shift) - 1)
    sr = np.where((srest > half) | ((srest == half) & (sr & 1 == 1)), sr + 1, sr)
    out = np.where(e >= 0x1F, 0x7C00, np.where(e <= 0, np.where(e < -10, 0, sr), r))
    out = np.where(exp == 0xFF, 0x7C00 | np.where(mant != 0, 0x200, 0), out)
    return (sign | out).astype(np.uint16)


def test_f16_conversion_matches_reference_rounding():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(200000).astype(np.float32) * 10.0 ** rng.integers(-9, 5, 200000),
                        np.float32([0.0, -0.0, 65504, 65519.99, 65520, 1e9, -1e9, np.inf, -np.inf, 2 ** -24, 2 ** -25,
                                    1.5 * 2 ** -25, 3 * 2 ** -26, 2 ** -14, 2 ** -14 - 2 ** -25])]).astype(np.float32)
    got = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, restated_f32_to_f16(x))


@pytest.mark.parametrize("version,alignment", [(3, None), (2, 64), (3, 256)])
def test_metadata_types_round_trip(tmp_path, version, alignment):
    wr = Writer(version, alignment)
    vals = {"u8": (0, 250), "i8": (1, -100), "u16": (2, 60000), "i16": (3, -30000), "u32": (4, 4000000000),
            "i32": (5, -2000000000), "f32": (6, 0.5), "bool": (7, True), "str": (8, "lfm2 ünïcode"),
            "u64": (10, 2 ** 63 + 5), "i64": (11, -(2 ** 40)), "f64": (12, 1e-300)}
    for k, (t, v) in vals.items():
        wr.kv(k, t, v)
    wr.kv("arr.str", 9, (8, ["a", "", "bc"])).kv("arr.i32", 9, (5, [1, -2, 3]))
    wr.kv("arr.nested", 9, (9, [(4, [1, 2]), (4, [])])).kv("arr.empty", 9, (12, []))
    x = np.arange(6, dtype=np.float32).reshape(2, 3) - 2.5
    wr.tensor("t.a", x, G.GGML_F32).tensor("t.b", np.float32([7.0]), G.GGML_F16)
    g = G.Gguf(wr.write(str(tmp_path / "m.gguf")))
    for k, (t, v) in vals.items():
        assert g.meta[k] == v, k
    assert g.meta["arr.str"] == ["a", "", "bc"] and g.meta["arr.i32"] == [1, -2, 3]
    assert g.meta["arr.nested"] == [[1, 2], []] and g.meta["arr.empty"] == []
    assert g.data_start % (alignment or 32) == 0
    assert g.dims("t.a") == [2, 3] and np.array_equal(g.f32("t.a"), x)
    assert g.f32("t.b").tolist() == [7.0]


def test_tensor_types_decode_as_reference(tmp_path):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((64, 96)) * 0.05).astype(np.float32)
    x[0, :5] = [0.0, -0.0, 1e-8, 70000.0, -3.0]
    wr = Writer()
    for name, ty in (("f32", G.GGML_F32), ("f16", G.GGML_F16), ("bf16", G.GGML_BF16), ("q8", G.GGML_Q8_0)):
        wr.tensor(name, x, ty)
    g = G.Gguf(wr.write(str(tmp_path / "t.gguf")))
    assert all(g.dims(n) == [64, 96] for n in ("f32", "f16", "bf16", "q8"))
    assert np.array_equal(g.f32("f32"), x)
    # F16 decode: exact widening; f16() passes F16 bits through untouched
    h = restated_f32_to_f16(x)
    assert np.array_equal(g.f32("f16"), h.view(np.float16).astype(np.float32))
    assert np.array_equal(g.f16("f16").view(np.uint16), h)
    # F32 -> f16() rounds like the reference
    assert np.array_equal(g.f16("f32").view(np.uint16), h)
    # BF16: the 16 stored bits are the upper half of an f32
    bits = np.frombuffer(encode_tensor(x, G.GGML_BF16), np.uint16)
    assert np.array_equal(g.f32("bf16").reshape(-1).view(np.uint32), bits.astype(np.uint32) << 16)
    # Q8_0: (int8 q as f32) * f16 scale, block by block in storage order
    raw = np.frombuffer(q8_0_encode(x), np.uint8).reshape(-1, 34)
    d = raw[:, :2].copy().view(np.float16).astype(np.float32)
    q = raw[:, 2:].copy().view(np.int8).astype(np.float32)
    want = np.float32(q * d).reshape(64, 96)
    assert np.array_equal(g.f32("q8"), want)
    assert np.abs(want - x).max() <= np.abs(x).max() / 127
    assert np.array_equal(g.f16("q8").view(np.uint16), restated_f32_to_f16(want))


def test_errors(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGML" + b"\0" * 64)
    with pytest.raises(ValueError, match="not a GGUF file"):
        G.Gguf(str(p))
    p.write_bytes(b"GGUF" + struct.pack("<IQQ", 1, 0, 0))
    with pytest.raises(ValueError, match="v1 unsupported"):
        G.Gguf(str(p))
    p.write_bytes(b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + _enc_str("k") + struct.pack("<I", 13) + b"\0" * 8)
    with pytest.raises(ValueError, match="bad GGUF value type 13"):
        G.Gguf(str(p))
    p.write_bytes(b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + _enc_str("k"))
    with pytest.raises(ValueError, match="truncated"):
        G.Gguf(str(p))
    wr = Writer().tensor("x", np.zeros((4, 32), np.float32), G.GGML_F32)
    wr.tensors.append(("q4", [32], 2, b"\0" * 32))  # Q4_0: not decoded by the reference
    g = G.Gguf(wr.write(str(tmp_path / "e.gguf")))
    with pytest.raises(KeyError, match="missing tensor nope"):
        g.f32("nope")
    with pytest.raises(ValueError, match="unsupported ggml type 2"):
        g.f32("q4")
    p2 = tmp_path / "short.gguf"  # the data of "x" (512 bytes, then "q4"'s 32) cut 64 bytes short
    p2.write_bytes((tmp_path / "e.gguf").read_bytes()[:-64])
    with pytest.raises(ValueError, match="past the end"):
        G.Gguf(str(p2)).f32("x")
    t = Writer().kv("general.architecture", 8, "llama").write(str(tmp_path / "arch.gguf"))
    with pytest.raises(ValueError, match="want lfm2"):
        G.load_text(t)
    t = Writer().kv("general.architecture", 8, "lfm2").write(str(tmp_path / "nb.gguf"))
    with pytest.raises(ValueError, match="missing lfm2.block_count"):
        G.load_text(t)


def small_text():
    return W.text_weights(7, n_layers=5, attn_layers=(1, 3), ffn=256, vocab=320, n_head=2, head_ffn=128)


def test_text_mapping_round_trip(tmp_path):
    w = small_text()
    got = G.load_text(write_text(str(tmp_path / "text.gguf"), w))
    assert_same_dict(got, w)
    assert np.array_equal(got["rope"], w["rope"])
    assert [l["is_attn"] for l in got["layers"]] == [l["is_attn"] for l in w["layers"]]
    assert got["vocab"] == 320 and [l["ffn"] for l in got["head"]] == [128, 128]


def test_text_mapping_quantised(tmp_path):
    """Q8_0 matrices decode to (q * d) and reach the runner layout as the fp16 rounding of that."""
    w = small_text()
    got = G.load_text(write_text(str(tmp_path / "q.gguf"), w, G.GGML_Q8_0))
    m = np.asarray(w["layers"][0]["down"], np.float32)
    raw = np.frombuffer(q8_0_encode(m), np.uint8).reshape(-1, 34)
    want = (raw[:, 2:].copy().view(np.int8).astype(np.float32) *
            raw[:, :2].copy().view(np.float16).astype(np.float32)).reshape(m.shape)
    assert np.array_equal(got["layers"][0]["down"], want.astype(np.float16))
    assert np.array_equal(got["final_norm"], w["final_norm"])


def test_vision_and_audio_mapping_round_trip(tmp_path):
    vw = W.vision_weights(3, n_layers=2)
    aw = W.audio_weights(4, n_layers=2)
    wr = write_audio(write_vision(Writer(), vw), aw)  # one mmproj file holds both towers
    g = G.Gguf(wr.write(str(tmp_path / "mmproj.gguf")))
    assert_same_dict(G.load_vision(g), vw)
    assert_same_dict(G.load_audio(g), aw)


# ------------------------------------------------------------------------------------------- GPU tests
@pytest.mark.gpu
def test_text_model_from_gguf_identical(tmp_path, gpu_lib):
    import torch  # noqa: F401
    from fast_d1_omni_b200.model import TextModel
    w = W.text_weights(0)
    batch = W.text_batch(5, 6, lengths=[37, 512, 200, 1000, 64, 129])
    a = TextModel(w, cap_tokens=4096)
    try:
        want = a(batch)
    finally:
        a.close()
    b = TextModel(G.load_text(write_text(str(tmp_path / "text.gguf"), w)), cap_tokens=4096)
    try:
        got = b(batch)
    finally:
        b.close()
    assert got.shape == want.shape and np.abs(got - want).max() <= 2e-3


@pytest.mark.gpu
def test_media_models_from_gguf_identical(tmp_path, gpu_lib):
    import torch  # noqa: F401
    from fast_d1_omni_b200.model import AudioModel, VisionModel
    vw, aw = W.vision_weights(3), W.audio_weights(4)
    g = G.Gguf(write_audio(write_vision(Writer(), vw), aw).write(str(tmp_path / "mmproj.gguf")))
    crops = W.vision_crops(3, n_images=2)
    clips = W.audio_clips(4, n_clips=2, hi_s=8.0)
    outs = []
    for vws, aws in ((vw, aw), (G.load_vision(g), G.load_audio(g))):
        v = VisionModel(vws, max_patches=16384)
        a = AudioModel(aws, max_rows=512)
        try:
            outs.append((v.encode(crops).cpu().numpy(), a.encode_pcm(clips).cpu().numpy()))
        finally:
            v.close()
            a.close()
    for want, got in zip(outs[0], outs[1]):
        assert got.shape == want.shape
        assert np.sqrt(((got - want) ** 2).mean() / (want ** 2).mean()) <= 5e-3
