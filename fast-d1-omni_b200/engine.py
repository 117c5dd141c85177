"""Continuous-batching engine (include/d1h.h d1e_*, a restatement of src/engine.rs) and the multi-GPU dispatcher.

A request is a dict: {"rows": [{"ids": int32[n], "markers": int32[k], "qtype": int}, ...], "media": None |
{"kind": "images", "crops": [(ph, pw, fp16 [ph*pw, 768] patches)]} | {"kind": "audio", "mel": fp32 [>=valid, 128],
"valid": int} or {"kind": "audio", "pcm": fp32 16 kHz samples}}. Its result is (logits fp32 [sum of markers], error str) — one logit per option marker, rows in order.

The 600M model fits every GPU and requests are independent, so multi-GPU serving is one replica per device:
  * in one process, `Dispatcher` runs one Engine per device on its own host thread and hands each request, whole,
    to the engine with the fewest queued tokens (prefix caches stay on the device that encoded them);
  * under torchrun (one process per GPU), `assign` gives every rank the same deterministic least-loaded split of
    the request list and `gather_results` collects the results on rank 0 — a host-side gather, no collective on
    the data path.
"""
from __future__ import annotations

import ctypes as C
import math
import threading
import time

import numpy as np

from . import abi, lib

MEDIA_NONE, MEDIA_IMAGES, MEDIA_AUDIO = 0, 1, 2


def audio_rows(valid: int) -> int:
    """Encoder rows of `valid` mel frames (three stride-2 stages, src/engine.rs:36-42)."""
    for _ in range(3):
        valid = (valid - 1) // 2 + 1
    return valid


def pcm_len_16k(n: int, rate: int) -> int:
    """16 kHz samples of a waveform of n samples at `rate` Hz: the WAV decoder keeps at most 30 s + 1 s
    (src/audio.rs:59), resample() writes n * up / down samples (up / down = 16000 / rate reduced, :108-113)."""
    if rate == 16000:
        return n
    g = math.gcd(rate, 16000)
    return min(n, 31 * rate) * (16000 // g) // (rate // g)


def prefix_len(req) -> int:
    m = req.get("media")
    if not m:
        return 0
    if m["kind"] == "images":
        return sum(ph * pw // 4 for ph, pw, _ in m["crops"])
    if m.get("pcm") is not None:  # src/audio.rs:241-247: cut to 30 s, padded to 0.5 s, hop 160
        return audio_rows(max(min(pcm_len_16k(len(m["pcm"]), int(m.get("rate") or 16000)), 30 * 16000), 8000) // 160)
    return audio_rows(int(m["valid"]))


def request_tokens(req) -> int:
    """Trunk positions a request costs: its question tokens plus its media prefix (the dispatcher's measure)."""
    return sum(len(r["ids"]) for r in req["rows"]) + prefix_len(req)


class Engine:
    """One device's engine over a TextModel and optional VisionModel / AudioModel (model.py)."""

    def __init__(self, text, vision=None, audio=None, max_batch_tokens: int = 8192, cap_tokens: int | None = None,
                 media_cache_mb: int = 1536, stream=None):
        import torch
        self.L = lib()
        self.device = text.device
        self.text, self.vision, self.audio = text, vision, audio
        self.stream = stream if stream is not None else torch.cuda.Stream(self.device)
        cfg = abi.EngineConfig()
        cfg.max_batch_tokens = max_batch_tokens
        cfg.cap_tokens = cap_tokens or max(max_batch_tokens, 8192)
        cfg.media_cache_bytes = media_cache_mb << 20
        with torch.cuda.device(self.device):
            self.e = self.L.d1e_create(text.m, vision.v if vision else None, audio.a if audio else None,
                                       C.byref(cfg), C.c_void_p(self.stream.cuda_stream))
        if not self.e:
            raise RuntimeError(f"d1e_create failed: {self.L.d1e_last_error().decode()}")
        self.lock = threading.Lock()
        self.results: dict[int, tuple[np.ndarray, str]] = {}

    # ------------------------------------------------------------------------------------------------ requests
    def submit(self, req) -> int:
        rows = req["rows"]
        arr = (abi.Row * max(1, len(rows)))()
        keep = []
        for i, r in enumerate(rows):
            ids = np.ascontiguousarray(r["ids"], dtype=np.int32)
            mk = np.ascontiguousarray(r["markers"], dtype=np.int32)
            keep += [ids, mk]
            arr[i].ids = ids.ctypes.data_as(C.POINTER(C.c_int))
            arr[i].n_ids = len(ids)
            arr[i].markers = mk.ctypes.data_as(C.POINTER(C.c_int))
            arr[i].n_markers = len(mk)
            arr[i].qtype = int(r.get("qtype", 0))
        job = abi.Job()
        job.rows = arr
        job.n_rows = len(rows)
        m = req.get("media")
        if m and m["kind"] == "images":
            crops = m["crops"]
            ph = np.array([c[0] for c in crops], np.int32)
            pw = np.array([c[1] for c in crops], np.int32)
            pix = np.ascontiguousarray(np.concatenate([np.asarray(c[2], np.float16) for c in crops]))
            keep += [ph, pw, pix]
            job.media.kind = MEDIA_IMAGES
            job.media.n_crops = len(crops)
            job.media.ph = ph.ctypes.data_as(C.POINTER(C.c_int))
            job.media.pw = pw.ctypes.data_as(C.POINTER(C.c_int))
            job.media.patches = C.c_void_p(pix.ctypes.data)
        elif m and m["kind"] == "audio" and m.get("pcm") is not None:
            pcm = np.ascontiguousarray(m["pcm"], np.float32)
            keep.append(pcm)
            job.media.kind = MEDIA_AUDIO
            job.media.pcm = pcm.ctypes.data_as(C.POINTER(C.c_float))
            job.media.n_samples = len(pcm)
            job.media.sample_rate = int(m.get("rate") or 16000)
        elif m and m["kind"] == "audio":
            v = int(m["valid"])
            mel = np.ascontiguousarray(np.asarray(m["mel"], np.float32)[:v])
            keep.append(mel)
            job.media.kind = MEDIA_AUDIO
            job.media.mel = mel.ctypes.data_as(C.POINTER(C.c_float))
            job.media.valid = v
        with self.lock:
            jid = self.L.d1e_submit(self.e, C.byref(job))  # copies everything it needs
        if jid < 0:
            raise RuntimeError(f"d1e_submit failed: {self.L.d1e_last_error().decode()}")
        return int(jid)

    def step(self) -> int:
        """One engine iteration; collects finished requests into self.results. Returns how many finished."""
        import torch
        with self.lock, torch.cuda.device(self.device):
            n = self.L.d1e_step(self.e)
            if n < 0:
                raise RuntimeError(f"d1e_step failed: {self.L.d1e_last_error().decode()}")
            self._take()
        return n

    def _take(self):
        err = C.create_string_buffer(512)
        jid = C.c_longlong()
        while True:
            n = self.L.d1e_next_logits(self.e)
            if n < 0:
                return
            buf = np.zeros(max(n, 1), np.float32)
            got = self.L.d1e_take(self.e, C.byref(jid), buf.ctypes.data_as(C.POINTER(C.c_float)), len(buf), err, 512)
            if got < 0:
                raise RuntimeError(f"d1e_take failed: {self.L.d1e_last_error().decode()}")
            self.results[int(jid.value)] = (buf[:got], err.value.decode())

    @property
    def pending(self) -> int:
        with self.lock:
            return int(self.L.d1e_pending(self.e))

    @property
    def queued_tokens(self) -> int:
        with self.lock:
            return int(self.L.d1e_queued_tokens(self.e))

    def drain(self) -> None:
        while self.pending:
            self.step()

    def run(self, requests):
        """Submit all requests, run to completion; results in request order."""
        ids = [self.submit(r) for r in requests]
        self.drain()
        return [self.results.pop(i) for i in ids]

    def stats(self) -> dict:
        s = abi.EngineStats()
        self.L.d1e_stats(self.e, C.byref(s))
        return {k: int(getattr(s, k)) for k, _ in abi.EngineStats._fields_}

    def close(self) -> None:
        if getattr(self, "e", None):
            import torch
            with torch.cuda.device(self.device):
                self.L.d1e_destroy(self.e)
            self.e = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Dispatcher:
    """One Engine per device, each stepped by its own host thread; whole requests go to the engine with the fewest
    queued tokens at submission (src/engine.rs runs one engine thread per process; this is its multi-GPU form)."""

    def __init__(self, engines):
        self.engines = list(engines)
        self.assigned: list[int] = []

    def run(self, requests):
        stop = threading.Event()
        errors = []

        def worker(e):
            try:
                while not (stop.is_set() and e.pending == 0):
                    if e.pending:
                        e.step()
                    else:
                        time.sleep(2e-4)
            except Exception as ex:  # surfaced after the join
                errors.append(ex)
                stop.set()

        threads = [threading.Thread(target=worker, args=(e,), daemon=True) for e in self.engines]
        for t in threads:
            t.start()
        placed = []
        try:
            for r in requests:
                d = min(range(len(self.engines)), key=lambda i: (self.engines[i].queued_tokens, i))
                placed.append((d, self.engines[d].submit(r)))
        finally:
            stop.set()
            for t in threads:
                t.join()
        if errors:
            raise errors[0]
        self.assigned = [d for d, _ in placed]
        return [self.engines[d].results.pop(i) for d, i in placed]


# Media work in trunk-position equivalents, for the static split: a least-squares fit of the per-rank device times of
# the config-4 stream on B200 at 1, 2, 4 and 8 GPUs against each rank's trunk positions, image patches and audio
# frames gave 0.7245 us per trunk position, 0.80 us per 16x16 image patch (vision tower and projector) and 1.05 us
# per 10 ms audio frame (front end, subsampling, FastConformer and adapter at a few hundred rows per clip); residual
# 1.5 ms of ~84 ms per pass. (A first fit, on a split that balanced positions only and an older build, gave 1.8 and
# 1.18.)
PATCH_COST = 1.10
FRAME_COST = 1.45


def request_cost(req) -> float:
    """A request's device work in trunk-position equivalents: its trunk positions (questions and media prefix) plus
    the encoder work of its media."""
    cost = float(request_tokens(req))
    m = req.get("media")
    if m and m["kind"] == "images":
        cost += PATCH_COST * sum(ph * pw for ph, pw, _ in m["crops"])
    elif m and m["kind"] == "audio":
        if m.get("pcm") is not None:
            frames = max(min(pcm_len_16k(len(m["pcm"]), int(m.get("rate") or 16000)), 30 * 16000), 8000) // 160
        else:
            frames = int(m["valid"])
        cost += FRAME_COST * frames
    return cost


def assign(requests, world: int):
    """Deterministic least-loaded split for one-process-per-GPU serving: request i goes to the rank with the least
    work so far (request_cost; ties to the lowest rank), in arrival order. Every rank computes the same list."""
    load = [0.0] * world
    out = []
    for r in requests:
        d = min(range(world), key=lambda i: (load[i], i))
        out.append(d)
        load[d] += request_cost(r)
    return out


def gather_results(local: dict, world: int, rank: int, n_requests: int):
    """Host-side gather of {request index: result} from every rank to rank 0 (torch.distributed object gather over
    the process group's backend). Returns the list in request order on rank 0, None elsewhere."""
    import torch.distributed as dist
    if world == 1:
        return [local[i] for i in range(n_requests)]
    parts = [None] * world if rank == 0 else None
    dist.gather_object(local, parts, dst=0)
    if rank != 0:
        return None
    merged = {}
    for p in parts:
        merged.update(p)
    return [merged[i] for i in range(n_requests)]
