"""The text model on one GPU: uploads weights, owns a d1h runner (include/d1h.h) and its workspace, and runs
packed batches (src/model.rs Runner::launch_text / launch_prefix / finish).

torch is used only for device memory and streams; every kernel is libd1kernels'.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import abi, check, lib


def _ptr(t: torch.Tensor):
    return C.c_void_p(t.data_ptr())


class TextModel:
    """Device copy of `weights.text_weights(...)` plus a runner.

    kernel_lib: None runs this library's kernels; a path runs another library with the d1kernels.h ABI through the
    same host runner (the tests use it for the reference's own kernels). fused: use the fused GEMM epilogues.
    """

    def __init__(self, w: dict, device: int = 0, kernel_lib: str | None = None, fused: bool = True,
                 cap_tokens: int = 8192):
        self.device = torch.device("cuda", device)
        self.L = lib()
        self._keep = []

        def h16(a):
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float16)).to(self.device)
            self._keep.append(t)
            return _ptr(t)

        def f32(a):
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(self.device)
            self._keep.append(t)
            return _ptr(t)

        with torch.cuda.device(self.device):
            layers = (abi.TrunkLayer * len(w["layers"]))()
            for i, l in enumerate(w["layers"]):
                x = layers[i]
                x.is_attn = int(l["is_attn"])
                x.ffn = l["ffn"]
                x.op_norm = f32(l["op_norm"])
                x.ffn_norm = f32(l["ffn_norm"])
                x.gate_up = h16(l["gate_up"])
                x.down = h16(l["down"])
                if l["is_attn"]:
                    x.qkv, x.out, x.qn, x.kn = h16(l["qkv"]), h16(l["out"]), f32(l["qn"]), f32(l["kn"])
                else:
                    x.in_proj, x.out_proj, x.convw = h16(l["in_proj"]), h16(l["out_proj"]), f32(l["convw"])
            head = (abi.HeadLayer * max(1, len(w["head"])))()
            for i, l in enumerate(w["head"]):
                x = head[i]
                x.n1_w, x.n1_b, x.qkv, x.qkv_b = f32(l["n1_w"]), f32(l["n1_b"]), h16(l["qkv"]), f32(l["qkv_b"])
                x.out, x.out_b, x.n2_w, x.n2_b = h16(l["out"]), f32(l["out_b"]), f32(l["n2_w"]), f32(l["n2_b"])
                x.up, x.up_b, x.down, x.down_b = h16(l["up"]), f32(l["up_b"]), h16(l["down"]), f32(l["down_b"])
                x.ffn = l["ffn"]
            tw = abi.TextWeights()
            tw.n_layers = len(w["layers"])
            tw.layers = layers
            tw.n_head = len(w["head"])
            tw.head = head
            tw.vocab = w["vocab"]
            tw.embed = h16(w["embed"])
            tw.final_norm = f32(w["final_norm"])
            tw.type_emb = f32(w["type_emb"])
            tw.cls_norm_w, tw.cls_norm_b = f32(w["cls_norm_w"]), f32(w["cls_norm_b"])
            tw.cls_w, tw.cls_b, tw.out_w = h16(w["cls_w"]), f32(w["cls_b"]), h16(w["out_w"])
            tw.out_b = float(w["out_b"])
            tw.eps = float(w["eps"])
            tw.rope_theta = float(w["rope_theta"])
            torch.cuda.synchronize(self.device)
            self.m = self.L.d1h_model_create(C.byref(tw), kernel_lib.encode() if kernel_lib else None, int(fused))
            if not self.m:
                raise RuntimeError(f"d1h_model_create failed: {self.L.d1h_last_error().decode()}")
            self.ws = self.L.d1h_workspace_create(self.m, cap_tokens)
            if not self.ws:
                raise RuntimeError(f"d1h_workspace_create failed: {self.L.d1h_last_error().decode()}")
        self.cap_tokens = cap_tokens
        self._pending = {}

    # ---------------------------------------------------------------------------------------------------- runs
    def _stream(self, stream):
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        return C.c_void_p(s.cuda_stream)

    def launch(self, batch, slot: int = 0, stream=None) -> None:
        """Enqueue a batch (list of dict(ids, markers, qtype[, prefix])) on `stream` (default: current)."""
        seqs = (abi.TextSeq * len(batch))()
        keep = []
        for i, s in enumerate(batch):
            ids = np.ascontiguousarray(s["ids"], dtype=np.int32)
            mk = np.ascontiguousarray(s["markers"], dtype=np.int32)
            keep += [ids, mk]
            seqs[i].ids = ids.ctypes.data_as(C.POINTER(C.c_int))
            seqs[i].n_ids = len(ids)
            seqs[i].markers = mk.ctypes.data_as(C.POINTER(C.c_int))
            seqs[i].n_markers = len(mk)
            seqs[i].qtype = int(s["qtype"])
            pc = s.get("prefix")
            seqs[i].prefix = C.pointer(pc) if pc is not None else None
        with torch.cuda.device(self.device):
            check(self.L.d1h_launch_text(self.m, self.ws, slot, seqs, len(batch), self._stream(stream)), "launch_text")
        self._pending[slot] = sum(len(s["markers"]) for s in batch)

    def finish(self, slot: int = 0) -> np.ndarray:
        n = self._pending.pop(slot)
        out = np.zeros(max(n, 1), np.float32)
        r = self.L.d1h_finish(self.m, self.ws, slot, out.ctypes.data_as(C.POINTER(C.c_float)), len(out))
        if r < 0:
            raise RuntimeError(f"d1h_finish failed: {self.L.d1h_last_error().decode()}")
        return out[:n]

    def __call__(self, batch, stream=None) -> np.ndarray:
        self.launch(batch, 0, stream)
        return self.finish(0)

    # ---------------------------------------------------------------------------------------------------- prefixes
    def prefix_alloc(self, n: int, stream=None) -> abi.PrefixCache:
        pc = abi.PrefixCache()
        with torch.cuda.device(self.device):
            check(self.L.d1h_prefix_alloc(self.m, n, C.byref(pc), self._stream(stream)), "prefix_alloc")
        return pc

    def prefix_free(self, pc: abi.PrefixCache, stream=None) -> None:
        with torch.cuda.device(self.device):
            self.L.d1h_prefix_free(C.byref(pc), self._stream(stream))

    def launch_prefix(self, items, slot: int = 0, stream=None) -> None:
        """items: list of (emb fp32 [len, 1024] CUDA tensor, PrefixCache)."""
        arr = (abi.PrefixSeq * len(items))()
        for i, (emb, pc) in enumerate(items):
            assert emb.is_cuda and emb.dtype == torch.float32 and emb.is_contiguous()
            arr[i].emb = _ptr(emb)
            arr[i].cache = C.pointer(pc)
        with torch.cuda.device(self.device):
            check(self.L.d1h_launch_prefix(self.m, self.ws, slot, arr, len(items), self._stream(stream)), "prefix")

    def tune(self, max_tokens: int | None = None, stream=None) -> int:
        with torch.cuda.device(self.device):
            n = self.L.d1h_tune(self.m, self.ws, max_tokens or self.cap_tokens, self._stream(stream))
        if n < 0:
            raise RuntimeError(f"d1h_tune failed: {self.L.d1h_last_error().decode()}")
        return n

    def set_tune_effort(self, effort: int) -> None:
        """Effort of the GEMM plans tuned on the first use of a shape and M bucket (d1h_set_tune_effort)."""
        if self.L.d1h_set_tune_effort(self.m, int(effort)) != 0:
            raise ValueError(f"tune effort {effort} outside 0..2")

    def save_plans(self, path: str) -> None:
        """Writes the tuned GEMM plans (d1_lt_save on the model's GEMM context)."""
        if self.L.d1_lt_save(self.L.d1h_gemm_ctx(self.m), path.encode()) != 0:
            raise RuntimeError(f"d1_lt_save failed for {path}")

    def load_plans(self, path: str) -> int:
        """Reads GEMM plans written by save_plans for this build; returns how many were loaded."""
        n = self.L.d1_lt_load(self.L.d1h_gemm_ctx(self.m), path.encode())
        if n < 0:
            raise RuntimeError(f"d1_lt_load failed for {path} ({n}: missing file or another build)")
        return n

    @property
    def launches(self) -> int:
        return int(self.L.d1h_launch_count(self.m))

    def close(self) -> None:
        if getattr(self, "ws", None):
            self.L.d1h_workspace_destroy(self.ws)
            self.ws = None
        if getattr(self, "m", None):
            self.L.d1h_model_destroy(self.m)
            self.m = None
        self._keep.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class VisionModel:
    """Device copy of `weights.vision_weights(...)` plus the vision runner (include/d1h.h d1h_vision_*)."""

    def __init__(self, w: dict, device: int = 0, kernel_lib: str | None = None, fused: bool = True,
                 max_patches: int = 16384):
        self.device = torch.device("cuda", device)
        self.L = lib()
        self._keep = []

        def h16(a):
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float16)).to(self.device)
            self._keep.append(t)
            return _ptr(t)

        def f32(a):
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(self.device)
            self._keep.append(t)
            return _ptr(t)

        def host32(a):
            arr = np.ascontiguousarray(a, dtype=np.float32)
            self._keep.append(arr)
            return C.c_void_p(arr.ctypes.data)

        with torch.cuda.device(self.device):
            layers = (abi.VisionLayer * len(w["layers"]))()
            for i, l in enumerate(w["layers"]):
                x = layers[i]
                x.ln1_w, x.ln1_b, x.qkv, x.qkv_b = f32(l["ln1_w"]), f32(l["ln1_b"]), h16(l["qkv"]), f32(l["qkv_b"])
                x.out, x.out_b, x.ln2_w, x.ln2_b = h16(l["out"]), f32(l["out_b"]), f32(l["ln2_w"]), f32(l["ln2_b"])
                x.fc1, x.fc1_b, x.fc2, x.fc2_b = h16(l["fc1"]), f32(l["fc1_b"]), h16(l["fc2"]), f32(l["fc2_b"])
            vw = abi.VisionWeights()
            vw.n_layers = len(w["layers"])
            vw.layers = layers
            vw.patch_w = h16(w["patch_w"])
            vw.patch_b = host32(w["patch_b"])
            vw.pos = host32(w["pos"])
            vw.post_w, vw.post_b = f32(w["post_w"]), f32(w["post_b"])
            vw.proj1, vw.proj1_b = h16(w["proj1"]), f32(w["proj1_b"])
            vw.proj2, vw.proj2_b = h16(w["proj2"]), f32(w["proj2_b"])
            vw.eps = float(w["eps"])
            torch.cuda.synchronize(self.device)
            self.v = self.L.d1h_vision_create(C.byref(vw), kernel_lib.encode() if kernel_lib else None, int(fused),
                                              max_patches)
            if not self.v:
                raise RuntimeError(f"d1h_vision_create failed: {self.L.d1h_last_error().decode()}")

    def encode(self, crops, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """crops: [(ph, pw, fp16 [ph*pw, 768] host patches)] -> fp32 [sum ph*pw/4, 1024] on the device."""
        n = len(crops)
        ph = (C.c_int * n)(*[c[0] for c in crops])
        pw = (C.c_int * n)(*[c[1] for c in crops])
        pix = np.ascontiguousarray(np.concatenate([c[2] for c in crops]), dtype=np.float16)
        rows = sum(c[0] * c[1] // 4 for c in crops)
        if out is None:
            out = torch.empty(rows, 1024, device=self.device, dtype=torch.float32)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            check(self.L.d1h_vision_encode(self.v, n, ph, pw, C.c_void_p(pix.ctypes.data), _ptr(out),
                                           C.c_void_p(s.cuda_stream)), "vision_encode")
        return out

    def close(self) -> None:
        if getattr(self, "v", None):
            self.L.d1h_vision_destroy(self.v)
            self.v = None
        self._keep.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_AUDIO_F16 = {"ff1_up", "ff1_down", "qkv", "pos", "out", "pw1", "pw2", "ff2_up", "ff2_down", "ad1", "ad2", "res_down",
              "res_up"}


class AudioModel:
    """Device copy of `weights.audio_weights(...)` plus the audio runner (include/d1h.h d1h_audio_*)."""

    def __init__(self, w: dict, device: int = 0, fused: bool = True, max_rows: int = 1536):
        self.device = torch.device("cuda", device)
        self.L = lib()
        self._keep = []

        def dev(name, a):
            dt = np.float16 if name in _AUDIO_F16 else np.float32
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=dt)).to(self.device)
            self._keep.append(t)
            return _ptr(t)

        with torch.cuda.device(self.device):
            layers = (abi.AudioLayer * len(w["layers"]))()
            for i, l in enumerate(w["layers"]):
                for name, _ in abi.AudioLayer._fields_:
                    setattr(layers[i], name, dev(name, l[name]))
            aw = abi.AudioWeights()
            for name, _ in abi.AudioWeights._fields_:
                if name not in ("n_layers", "layers", "eps"):
                    setattr(aw, name, dev(name, w[name]))
            aw.n_layers = len(w["layers"])
            aw.layers = layers
            aw.eps = float(w["eps"])
            torch.cuda.synchronize(self.device)
            self.a = self.L.d1h_audio_create(C.byref(aw), int(fused), max_rows)
            if not self.a:
                raise RuntimeError(f"d1h_audio_create failed: {self.L.d1h_last_error().decode()}")
        self.max_rows = max_rows

    @staticmethod
    def out_len(valid: int) -> int:
        l1 = (valid - 1) // 2 + 1
        l2 = (l1 - 1) // 2 + 1
        return (l2 - 1) // 2 + 1

    def encode(self, clips, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """clips: [(mel fp32 [>= valid, 128], valid)] -> fp32 [sum ceil(valid/8), 1024] on the device."""
        n = len(clips)
        valid = (C.c_int * n)(*[int(v) for _, v in clips])
        mel = np.ascontiguousarray(np.concatenate([np.asarray(m, np.float32)[:v] for m, v in clips]), np.float32)
        rows = sum(self.out_len(v) for _, v in clips)
        if out is None:
            out = torch.empty(rows, 1024, device=self.device, dtype=torch.float32)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            r = self.L.d1h_audio_encode(self.a, n, valid, C.c_void_p(mel.ctypes.data), _ptr(out),
                                        C.c_void_p(s.cuda_stream))
        if r < 0:
            raise RuntimeError(f"d1h_audio_encode failed: {self.L.d1h_last_error().decode()}")
        assert r == rows
        return out

    def encode_pcm(self, waves, out: torch.Tensor | None = None, stream=None, rates=None) -> torch.Tensor:
        """waves: [fp32 samples] (16 kHz, or rates[i] Hz: resampled to 16 kHz on the GPU first) -> fp32 [sum T, 1024]
        on the device; log-mel features computed on the GPU (each clip cut to 30 s and padded to 0.5 s first)."""
        from .engine import pcm_len_16k
        n = len(waves)
        rates = [int(r or 16000) for r in rates] if rates is not None else [16000] * n
        ns = (C.c_int * n)(*[len(w) for w in waves])
        rt = (C.c_int * n)(*rates)
        pcm = np.ascontiguousarray(np.concatenate([np.asarray(w, np.float32) for w in waves]), np.float32)
        valid = [max(min(pcm_len_16k(len(w), r), 30 * 16000), 8000) // 160 for w, r in zip(waves, rates)]
        rows = sum(self.out_len(v) for v in valid)
        if out is None:
            out = torch.empty(rows, 1024, device=self.device, dtype=torch.float32)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        vo = (C.c_int * n)()
        with torch.cuda.device(self.device):
            r = self.L.d1h_audio_encode_pcm_rates(self.a, n, ns, rt, C.c_void_p(pcm.ctypes.data), _ptr(out), vo,
                                                  C.c_void_p(s.cuda_stream))
        if r < 0:
            raise RuntimeError(f"d1h_audio_encode_pcm failed: {self.L.d1h_last_error().decode()}")
        assert r == rows and list(vo) == valid
        return out

    def close(self) -> None:
        if getattr(self, "a", None):
            self.L.d1h_audio_destroy(self.a)
            self.a = None
        self._keep.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
