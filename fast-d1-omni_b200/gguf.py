"""GGUF loading into this package's weight layouts (the dicts TextModel, VisionModel and AudioModel take).

The reader follows the GGUF v2/v3 container as src/gguf.rs:1-220 reads it: little-endian header ("GGUF", version,
tensor count, metadata count), typed metadata values (types 0-12, arrays included), tensor infos (name, ggml dims
with the contiguous dimension first, type, offset), tensor data from the next `general.alignment` boundary (default
32). Tensor types F32 (0), F16 (1), BF16 (30) and Q8_0 (8) are converted as the reference converts them; data is
read through a memory map, so loading does not copy the file.

The model mappings restate the reference's loaders:
  * text (LFM2 trunk + decision head), src/model.rs:139-231: fused [q; k; v] attention rows, fused [gate; up] FFN
    rows, the last `lfm2.decision.block_count` blocks as decision-head layers;
  * vision tower + projector (mmproj), src/vision.rs:198-260: the patch embedding permuted from [768][3][16][16]
    (c, y, x) to (y, x, c) input order, fused q/k/v rows and biases;
  * audio encoder + adapter (mmproj), src/audio.rs:403-455: fused q/k/v rows, the pre-encode output weight's
    columns permuted from (c, f) to (f, c).
"""
from __future__ import annotations

import struct

import numpy as np

from .weights import _rope

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


class Gguf:
    def __init__(self, path: str):
        self.path = path
        self.buf = np.memmap(path, dtype=np.uint8, mode="r")
        self.pos = 0
        if bytes(self.buf[:4]) != b"GGUF":
            raise ValueError(f"{path}: not a GGUF file")
        self.pos = 4
        version = self._u32()
        if version < 2:
            raise ValueError(f"{path}: GGUF v{version} unsupported")
        n_tensors, n_kv = self._u64(), self._u64()
        self.meta: dict = {}
        for _ in range(n_kv):
            key = self._str()
            self.meta[key] = self._value(self._u32())
        self.tensors: dict = {}
        for _ in range(n_tensors):
            name = self._str()
            nd = self._u32()
            dims = [self._u64() for _ in range(nd)]
            ty = self._u32()
            off = self._u64()
            self.tensors[name] = (dims, ty, off)
        align = int(self.meta.get("general.alignment", 32))
        self.data_start = (self.pos + align - 1) // align * align

    # ------------------------------------------------------------------------------------------------ parsing
    def _take(self, n):
        b = bytes(self.buf[self.pos:self.pos + n])
        if len(b) != n:
            raise ValueError(f"{self.path}: truncated")
        self.pos += n
        return b

    def _u32(self):
        return struct.unpack("<I", self._take(4))[0]

    def _u64(self):
        return struct.unpack("<Q", self._take(8))[0]

    def _str(self):
        return self._take(self._u64()).decode("utf-8", errors="replace")

    def _value(self, t):
        if t in _SCALAR:
            fmt = _SCALAR[t]
            v = struct.unpack(fmt, self._take(struct.calcsize(fmt)))[0]
            return bool(v) if t == 7 else v
        if t == 8:
            return self._str()
        if t == 9:
            et, n = self._u32(), self._u64()
            return [self._value(et) for _ in range(n)]
        raise ValueError(f"{self.path}: bad GGUF value type {t}")

    # ------------------------------------------------------------------------------------------------ tensors
    def has(self, name):
        return name in self.tensors

    def dims(self, name):
        """PyTorch-order shape (ggml dims reversed)."""
        return [int(d) for d in reversed(self._info(name)[0])]

    def _info(self, name):
        if name not in self.tensors:
            raise KeyError(f"{self.path}: missing tensor {name}")
        return self.tensors[name]

    def _raw(self, name):
        dims, ty, off = self._info(name)
        n = int(np.prod(dims)) if dims else 1
        nbytes = {GGML_F32: n * 4, GGML_F16: n * 2, GGML_BF16: n * 2}.get(ty)
        if ty == GGML_Q8_0:
            nbytes = n // 32 * 34
        if nbytes is None:
            raise ValueError(f"{name}: unsupported ggml type {ty}")
        start = self.data_start + off
        if start + nbytes > len(self.buf):
            raise ValueError(f"{self.path}: tensor {name} runs past the end of the file (truncated)")
        return ty, n, self.buf[start:start + nbytes]

    def f32(self, name):
        """The tensor as fp32 in PyTorch order (src/gguf.rs:185-205)."""
        ty, n, raw = self._raw(name)
        if ty == GGML_F32:
            out = raw.view(np.float32)
        elif ty == GGML_F16:
            out = raw.view(np.float16).astype(np.float32)
        elif ty == GGML_BF16:
            out = (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:  # Q8_0: blocks of an fp16 scale and 32 int8 values
            blk = raw.reshape(-1, 34)
            d = blk[:, :2].copy().view(np.float16).astype(np.float32)
            q = blk[:, 2:].view(np.int8).astype(np.float32)
            out = (q * d).reshape(-1)
        return np.asarray(out, np.float32).reshape(self.dims(name))

    def f16(self, name):
        """The tensor as fp16 (F16 passed through, other types converted; src/gguf.rs:207-214)."""
        ty, n, raw = self._raw(name)
        if ty == GGML_F16:
            return np.asarray(raw.view(np.float16)).reshape(self.dims(name))
        with np.errstate(over="ignore"):  # out-of-range values become inf, as the reference's conversion gives
            return self.f32(name).astype(np.float16)


def _cat16(g, names):
    return np.concatenate([g.f16(n) for n in names], axis=0)


def load_text(path_or_gguf) -> dict:
    """The text model (src/model.rs:139-231) as a weights dict for model.TextModel."""
    g = path_or_gguf if isinstance(path_or_gguf, Gguf) else Gguf(path_or_gguf)
    arch = g.meta.get("general.architecture", "")
    if arch != "lfm2":
        raise ValueError(f"unexpected architecture {arch!r} (want lfm2)")
    if "lfm2.block_count" not in g.meta:
        raise ValueError("missing lfm2.block_count")
    n_layers = int(g.meta["lfm2.block_count"])
    n_head = int(g.meta.get("lfm2.decision.block_count", 2))
    n_trunk = n_layers - n_head
    eps = float(g.meta.get("lfm2.attention.layer_norm_rms_epsilon", 1e-5))
    theta = float(g.meta.get("lfm2.rope.freq_base", 1e6))
    vocab, hidden = g.dims("token_embd.weight")
    if hidden != 1024:
        raise ValueError(f"hidden size {hidden} unsupported (want 1024)")
    layers = []
    for i in range(n_trunk):
        t = lambda s: f"blk.{i}.{s}"  # noqa: E731
        lay = {"op_norm": g.f32(t("attn_norm.weight")).reshape(-1), "ffn_norm": g.f32(t("ffn_norm.weight")).reshape(-1),
               "gate_up": _cat16(g, [t("ffn_gate.weight"), t("ffn_up.weight")]), "down": g.f16(t("ffn_down.weight")),
               "ffn": g.dims(t("ffn_gate.weight"))[0]}
        if g.has(t("attn_q.weight")):
            lay.update(is_attn=True, qkv=_cat16(g, [t("attn_q.weight"), t("attn_k.weight"), t("attn_v.weight")]),
                       out=g.f16(t("attn_output.weight")), qn=g.f32(t("attn_q_norm.weight")).reshape(-1),
                       kn=g.f32(t("attn_k_norm.weight")).reshape(-1))
        else:
            lay.update(is_attn=False, in_proj=g.f16(t("shortconv.in_proj.weight")),
                       out_proj=g.f16(t("shortconv.out_proj.weight")),
                       convw=g.f32(t("shortconv.conv.weight")).reshape(hidden, 3))
        layers.append(lay)
    head = []
    for i in range(n_trunk, n_layers):
        t = lambda s: f"blk.{i}.{s}"  # noqa: E731
        v = lambda s: g.f32(t(s)).reshape(-1)  # noqa: E731
        head.append({"n1_w": v("attn_norm.weight"), "n1_b": v("attn_norm.bias"), "qkv": g.f16(t("attn_qkv.weight")),
                     "qkv_b": v("attn_qkv.bias"), "out": g.f16(t("attn_output.weight")), "out_b": v("attn_output.bias"),
                     "n2_w": v("ffn_norm.weight"), "n2_b": v("ffn_norm.bias"), "up": g.f16(t("ffn_up.weight")),
                     "up_b": v("ffn_up.bias"), "down": g.f16(t("ffn_down.weight")), "down_b": v("ffn_down.bias"),
                     "ffn": g.dims(t("ffn_up.weight"))[0]})
    return {"layers": layers, "head": head, "vocab": vocab, "embed": g.f16("token_embd.weight"),
            "final_norm": g.f32("token_embd_norm.weight").reshape(-1), "type_emb": g.f32("token_types.weight"),
            "cls_norm_w": g.f32("cls.norm.weight").reshape(-1), "cls_norm_b": g.f32("cls.norm.bias").reshape(-1),
            "cls_w": g.f16("cls.weight"), "cls_b": g.f32("cls.bias").reshape(-1),
            "out_w": g.f16("cls.output.weight").reshape(-1), "out_b": np.float32(g.f32("cls.output.bias").reshape(-1)[0]),
            "eps": np.float32(eps), "rope_theta": np.float32(theta), "rope": _rope(theta)}


def load_vision(path_or_gguf) -> dict:
    """The SigLIP2 tower + projector of an mmproj file (src/vision.rs:198-260) as a dict for model.VisionModel."""
    g = path_or_gguf if isinstance(path_or_gguf, Gguf) else Gguf(path_or_gguf)
    n = int(g.meta.get("clip.vision.block_count", 12))
    eps = float(g.meta.get("clip.vision.attention.layer_norm_epsilon", 1e-6))
    pw = g.f32("v.patch_embd.weight").reshape(768, 3, 16, 16)  # (out, c, y, x)
    patch_w = np.ascontiguousarray(pw.transpose(0, 2, 3, 1).reshape(768, 768)).astype(np.float16)
    v = lambda s: g.f32(s).reshape(-1)  # noqa: E731
    layers = []
    for i in range(n):
        t = lambda s: f"v.blk.{i}.{s}"  # noqa: E731
        layers.append({"ln1_w": v(t("ln1.weight")), "ln1_b": v(t("ln1.bias")),
                       "qkv": _cat16(g, [t("attn_q.weight"), t("attn_k.weight"), t("attn_v.weight")]),
                       "qkv_b": np.concatenate([v(t("attn_q.bias")), v(t("attn_k.bias")), v(t("attn_v.bias"))]),
                       "out": g.f16(t("attn_out.weight")), "out_b": v(t("attn_out.bias")),
                       "ln2_w": v(t("ln2.weight")), "ln2_b": v(t("ln2.bias")),
                       "fc1": g.f16(t("ffn_up.weight")), "fc1_b": v(t("ffn_up.bias")),
                       "fc2": g.f16(t("ffn_down.weight")), "fc2_b": v(t("ffn_down.bias"))})
    return {"eps": np.float32(eps), "patch_w": patch_w, "patch_b": v("v.patch_embd.bias"),
            "pos": v("v.position_embd.weight").reshape(256, 768), "layers": layers,
            "post_w": v("v.post_ln.weight"), "post_b": v("v.post_ln.bias"),
            "proj1": g.f16("mm.1.weight"), "proj1_b": v("mm.1.bias"), "proj2": g.f16("mm.2.weight"),
            "proj2_b": v("mm.2.bias")}


def load_audio(path_or_gguf) -> dict:
    """The FastConformer encoder + adapter of an mmproj file (src/audio.rs:403-455) as a dict for model.AudioModel."""
    g = path_or_gguf if isinstance(path_or_gguf, Gguf) else Gguf(path_or_gguf)
    n = int(g.meta.get("clip.audio.block_count", 17))
    eps = float(g.meta.get("clip.audio.attention.layer_norm_epsilon", 1e-5))
    v = lambda s: g.f32(s).reshape(-1)  # noqa: E731
    layers = []
    for i in range(n):
        t = lambda s: f"a.blk.{i}.{s}"  # noqa: E731
        layers.append({
            "ff1_n_w": v(t("ffn_norm.weight")), "ff1_n_b": v(t("ffn_norm.bias")),
            "ff1_up": g.f16(t("ffn_up.weight")), "ff1_up_b": v(t("ffn_up.bias")),
            "ff1_down": g.f16(t("ffn_down.weight")), "ff1_down_b": v(t("ffn_down.bias")),
            "att_n_w": v(t("ln1.weight")), "att_n_b": v(t("ln1.bias")),
            "qkv": _cat16(g, [t("attn_q.weight"), t("attn_k.weight"), t("attn_v.weight")]),
            "bq": v(t("attn_q.bias")), "bk": v(t("attn_k.bias")), "bv": v(t("attn_v.bias")),
            "pu": v(t("pos_bias_u")), "pv": v(t("pos_bias_v")), "pos": g.f16(t("linear_pos.weight")),
            "out": g.f16(t("attn_out.weight")), "out_b": v(t("attn_out.bias")),
            "conv_n_w": v(t("norm_conv.weight")), "conv_n_b": v(t("norm_conv.bias")),
            "pw1": g.f16(t("conv_pw1.weight")), "pw1_b": v(t("conv_pw1.bias")),
            "dw": v(t("conv_dw.weight")).reshape(512, -1), "dw_b": v(t("conv_dw.bias")),
            "bn_s": v(t("conv_norm.weight")), "bn_b": v(t("conv_norm.bias")),
            "pw2": g.f16(t("conv_pw2.weight")), "pw2_b": v(t("conv_pw2.bias")),
            "ff2_n_w": v(t("ffn_norm_1.weight")), "ff2_n_b": v(t("ffn_norm_1.bias")),
            "ff2_up": g.f16(t("ffn_up_1.weight")), "ff2_up_b": v(t("ffn_up_1.bias")),
            "ff2_down": g.f16(t("ffn_down_1.weight")), "ff2_down_b": v(t("ffn_down_1.bias")),
            "out_n_w": v(t("ln2.weight")), "out_n_b": v(t("ln2.bias"))})
    pre = v("a.pre_encode.out.weight").reshape(512, 256, 16)  # [out][c][f] -> [out][f][c]
    return {"eps": np.float32(eps),
            "c0_w": v("a.conv1d.0.weight").reshape(256, 9), "c0_b": v("a.conv1d.0.bias"),
            "c2_w": v("a.conv1d.2.weight").reshape(256, 9), "c2_b": v("a.conv1d.2.bias"),
            "c3_w": v("a.conv1d.3.weight").reshape(256, 256), "c3_b": v("a.conv1d.3.bias"),
            "c5_w": v("a.conv1d.5.weight").reshape(256, 9), "c5_b": v("a.conv1d.5.bias"),
            "c6_w": v("a.conv1d.6.weight").reshape(256, 256), "c6_b": v("a.conv1d.6.bias"),
            "pre_out": np.ascontiguousarray(pre.transpose(0, 2, 1).reshape(512, 4096)),
            "pre_out_b": v("a.pre_encode.out.bias"), "layers": layers,
            "ad_n_w": v("mm.a.mlp.0.weight"), "ad_n_b": v("mm.a.mlp.0.bias"),
            "ad1": g.f16("mm.a.mlp.1.weight"), "ad1_b": v("mm.a.mlp.1.bias"),
            "ad2": g.f16("mm.a.mlp.3.weight"), "ad2_b": v("mm.a.mlp.3.bias"),
            "res_n_w": v("mm.a.mlp.4.weight"), "res_n_b": v("mm.a.mlp.4.bias"),
            "res_down": g.f16("mm.a.mlp.5.weight"), "res_down_b": v("mm.a.mlp.5.bias"),
            "res_up": g.f16("mm.a.mlp.6.weight"), "res_up_b": v("mm.a.mlp.6.bias")}
