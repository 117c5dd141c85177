"""Benchmark of the d1rs text prefill forward on B200 (one JSON line on rank 0).

Metric: prefill tokens/s per B200 at 8192-token batches, plus the GEMM share of the tensor-core
peak. One step = one Runner::launch_text (src/model.rs:470-599) of an 8192-token batch: the config-0 architecture
(hidden 1024, 16 layers, attention at {2,5,8,10,12,14}, SwiGLU 4608, 2-layer decision head), random-init weights
(seed 0; no checkpoint is available offline), 32 packed sequences x 256 uniform token ids, 3 option markers each.

  value   tokens/s over all ranks, device-timed (CUDA events on the launch stream) over K back-to-back steps; the
          weights and activations (>700 MB) exceed the 126 MB L2, so no flush is needed between steps.
  e2e     the same steps through the public API with host buffers: host token ids -> d1h_launch_text (metadata
          built on the host, one pinned H2D copy) -> d1h_finish (logits D2H + sync), wall clock.
  roofline the dominant kernel (the fused SwiGLU projection GEMM, 302.0 MFLOP/token, 52.5% of the trunk FLOPs)
          timed alone with CUDA events: algorithmic FLOPs per launch / average launch time, against the measured
          cuBLAS bf16 peak (MEASURED_PEAKS.json, burst figure: the kernel is timed alone).
  cpu_baseline the oracle port (numpy fp32, oracle/d1_oracle.py) on a bounded sample of the same workload.

--impl reference: the reference's CPU implementation of the path. The reference has none (its forward is CUDA
only; its fp32 PyTorch path needs remote code and weights that are not available offline), so this arm times the
oracle port (fp32 numpy restatement of the reference's arithmetic) on all host threads, on bounded samples. When a
GPU and oracle/_ref/libd1ref.so (the reference's cuda/*.cu built unchanged) are present, the line also carries
`reference_gpu_engine`: the reference's own F16 engine (its kernels + cuBLASLt, plans tuned at the effort its engine
uses) timed on the same batches, in a child process that runs the cuBLASLt the reference was compiled against.

--gemm-sweep: BASELINE config 1, every projection GEMM shape, one JSON line per shape, with the reference's
cuBLASLt GEMM (d1_lt_tune at effort 1, then d1_lt_gemm of oracle/_ref/libd1ref.so) timed beside each form.
--attn-config2: BASELINE config 2 (packed varlen GQA attention, log-normal lengths) at 2048 / 8192 / 16384 tokens:
the tcgen05 kernel, this library's mma.sync kernel and the reference's k_flash_attn, one JSON line per size.
--workload mixed: BASELINE config 4 — the mixed text / image / audio request stream through the continuous-batching
engine, one replica per GPU (torchrun for N > 1).

Multi-GPU (torchrun, one process per GPU): every rank runs its own replica on its own batches (the model is
replicated and requests are sharded; no collective on the data path); value = all ranks' tokens / max time.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SEQ_LEN = 256
N_SEQS = 32
TOKENS = SEQ_LEN * N_SEQS
GEMM_FLOP_PER_TOKEN = 574_619_648          # trunk projection GEMMs (2 x 287,309,824 linear params)
SWIGLU_FLOP_PER_TOKEN = 2 * 9216 * 1024    # w1|w3, fused SwiGLU epilogue
# ncu dram__bytes_read.sum + dram__bytes_write.sum of one d1_gemm_swiglu launch at M=8192 (the capture of
# profiles/gemm_swiglu_pair_m8192.md, taken 2026-12-01 on one B200). It is below the launch's 111 MB of
# algorithmic bytes (A 16.8 MB + W 18.9 MB read, 75.5 MB written) because most of the output is still dirty in the
# 126 MB L2 when the kernel ends: ncu counts DRAM writes of the launch only.
SWIGLU_NCU_DRAM_BYTES_M8192 = 69.6e6
REF_SWEEP_EFFORT = 0   # the reference's d1_lt_tune effort in --gemm-sweep (effort 1 crashes on B200)
SUSTAINED_STEPS = 440  # second timed region: >= 2 s of back-to-back steps (clocks settle at the power cap)


def load_package():
    import importlib.util
    name = "fast_d1_omni_b200"
    if name in sys.modules:
        return sys.modules[name]
    d = ROOT / "fast-d1-omni_b200"
    spec = importlib.util.spec_from_file_location(name, d / "__init__.py", submodule_search_locations=[str(d)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """SM clock and throttle-reason sampling during the timed region (read-only). NVML from a background thread every
    10 ms, so even a ~0.1 s region gets ~10 samples; nvidia-smi at 200 ms when NVML is unavailable. The GPU is found
    by the UUID torch reports for the CUDA device (CUDA_VISIBLE_DEVICES-safe)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits (nvml.h): sw power cap 0x4, hw slowdown 0x8, sw thermal 0x20, hw thermal 0x40
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.thread = None
        self.samples = []  # (sm MHz, reason bits)
        self.max_mhz = None
        self.lines = []

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def __enter__(self):
        import threading
        try:
            import pynvml
            h = self._nvml_handle()
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.stop = threading.Event()

            def run():
                while not self.stop.is_set():
                    try:
                        self.samples.append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                                             int(reasons(h))))
                    except Exception:
                        return
                    self.stop.wait(0.01)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], self.max_mhz, set()
        for mhz, bits in self.samples:
            sm.append(mhz)
            reasons.update(n for n, b in self.BITS.items() if bits & b)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvml" if self.samples else "nvidia-smi"}


def use_all_cores() -> int:
    """Lets the oracle port use every host thread this process may run on, whatever OMP_NUM_THREADS the launcher
    set (torchrun sets 1): the BLAS pools through threadpoolctl, torch's intra-op pool through set_num_threads.
    Returns the thread count."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        import numpy  # noqa: F401  (load the BLAS before limiting it)
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n)
    except Exception:
        pass
    if "torch" in sys.modules:
        sys.modules["torch"].set_num_threads(n)
    return n


def cpu_sample(n_seqs: int, seed: int = 3):
    """Time the oracle port (fp32 numpy) on a bounded sample: n_seqs x 256-token sequences of the workload."""
    use_all_cores()
    from oracle import d1_oracle as O
    pkg = load_package()
    from fast_d1_omni_b200.weights import text_batch, text_weights
    w = text_weights(0)
    b = text_batch(seed, n_seqs, SEQ_LEN)
    O.launch_text(w, b[:1], "f32")  # warm the BLAS pool
    t0 = time.perf_counter()
    O.launch_text(w, b, "f32")
    dt = time.perf_counter() - t0
    return n_seqs * SEQ_LEN / dt, dt


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        return max(i.get("num_threads", 1) for i in threadpool_info()) or os.cpu_count()
    except Exception:
        return os.cpu_count()


def run_reference(args, rank, world):
    """--impl reference: the oracle port on the host cores, rank 0 only."""
    if rank != 0:
        return
    use_all_cores()
    from oracle import d1_oracle as O
    load_package()
    from fast_d1_omni_b200.weights import text_batch, text_weights
    w = text_weights(0)
    n_sample = 2  # 512 tokens per step: a bounded sample of the 8192-token batch
    for i in range(args.warmup):
        O.launch_text(w, text_batch(100 + i, n_sample, SEQ_LEN), "f32")
    t0 = time.perf_counter()
    for i in range(args.steps):
        O.launch_text(w, text_batch(200 + i, n_sample, SEQ_LEN), "f32")
    dt = time.perf_counter() - t0
    v = n_sample * SEQ_LEN * args.steps / dt
    cores = cpu_threads()
    line = {"impl": "reference", "metric": "prefill tokens/s per B200 at 8192-token batches", "value": v,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random weights and token ids)",
            "config": {"workload": f"text trunk+head forward, {TOKENS}-token batches of {N_SEQS}x{SEQ_LEN}",
                       "sample_per_step": f"{n_sample}x{SEQ_LEN} tokens"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"{n_sample} sequences x {SEQ_LEN} tokens per step, oracle/d1_oracle.py fp32"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    gpu = reference_gpu_engine_child(args.steps, args.warmup)
    if gpu is not None:
        line["reference_gpu_engine"] = gpu
    print(json.dumps(line), flush=True)


REF_LIB = ROOT / "oracle" / "_ref" / "libd1ref.so"


def preload_reference_cublaslt():
    """Loads the CUDA toolkit's cuBLASLt / cuBLAS (the libraries oracle/_ref/libd1ref.so was compiled and linked
    against) into the process before torch, whose wheels bundle an older cuBLASLt under the same soname
    (libcublasLt.so.12): without this, libd1ref.so binds to whichever copy torch loaded first. Returns the loaded
    cuBLASLt version, or None when the toolkit copy is not found (torch's is then used)."""
    import ctypes as C
    cuda_home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH") or "/usr/local/cuda"
    lt = Path(cuda_home) / "lib64" / "libcublasLt.so.12"
    if "torch" in sys.modules or not lt.exists():
        return None
    h = C.CDLL(str(lt), mode=C.RTLD_GLOBAL)
    blas = lt.with_name("libcublas.so.12")
    if blas.exists():
        C.CDLL(str(blas), mode=C.RTLD_GLOBAL)
    h.cublasLtGetVersion.restype = C.c_size_t
    return int(h.cublasLtGetVersion())


def reference_gpu_engine_child(steps, warmup):
    """Runs reference_gpu_engine in a child process at the reference engine's tuning effort (1, src/engine.rs:593);
    if that child does not finish cleanly, once more at effort 0, and says why. None when there is no reference
    library or no GPU."""
    if not REF_LIB.exists():
        return None
    out = {}
    for effort in (1, 0):
        cmd = [sys.executable, str(Path(__file__).resolve()), "--ref-engine-child", str(effort),
               "--steps", str(steps), "--warmup", str(warmup)]
        try:
            r = subprocess.run(cmd, capture_output=True, text=True, timeout=420 if effort else 300)
        except subprocess.TimeoutExpired:
            out[f"effort{effort}_failure"] = "timed out"
            continue
        sys.stderr.write(r.stderr[-2000:])
        lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
        if r.returncode == 0 and lines:
            res = json.loads(lines[-1])
            if res.get("unavailable"):
                return None
            res.update(out)
            return res
        out[f"effort{effort}_failure"] = (f"exit {r.returncode}" if r.returncode >= 0 else
                                          f"killed by signal {-r.returncode}")
    return out or None


def reference_gpu_engine(steps, warmup, effort):
    """The reference's own F16 CUDA engine on this GPU: cuda/kernels.cu + cuda/gemm.cu (cuBLASLt autotuner) built
    unchanged into oracle/_ref/libd1ref.so, driven by the same host runner (src/model.rs restated), on the same
    8192-token batches as this library's arm. Its GEMM plans come from d1_lt_tune at `effort` on the first use of
    each shape during the warm-up steps (the buckets these batches touch; the reference's engine tunes every bucket
    at startup with effort 1). Device time over `steps` back-to-back launch_text steps (CUDA events)."""
    lt_version = preload_reference_cublaslt()
    import torch
    if not torch.cuda.is_available():
        return {"unavailable": "no GPU"}
    load_package()
    from fast_d1_omni_b200.model import TextModel
    from fast_d1_omni_b200.weights import text_batch, text_weights
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    print(f"reference GPU engine: loading (cuBLASLt {lt_version})", file=sys.stderr, flush=True)
    model = TextModel(text_weights(0), device=0, kernel_lib=str(REF_LIB), fused=False, cap_tokens=TOKENS)
    model.set_tune_effort(effort)
    try:
        print(f"reference GPU engine: warm-up (effort-{effort} plans on first use)", file=sys.stderr, flush=True)
        batches = [text_batch(i, N_SEQS, SEQ_LEN) for i in range(4)]
        stream = torch.cuda.Stream(dev)
        t_tune = time.perf_counter()
        with torch.cuda.stream(stream):
            for i in range(warmup):
                model.launch(batches[i % 4], i % 2, stream)
            torch.cuda.synchronize(dev)
            t_tune = time.perf_counter() - t_tune
            model._pending.clear()
            print("reference GPU engine: timing", file=sys.stderr, flush=True)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i in range(steps):
                model.launch(batches[i % 4], i % 2, stream)
            e1.record(stream)
            torch.cuda.synchronize(dev)
            model._pending.clear()
        ms = e0.elapsed_time(e1)
        return {"value": TOKENS * steps / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms / steps,
                "device": torch.cuda.get_device_name(dev),
                "gemm_plans": f"d1_lt_tune effort {effort} on first use of each shape and bucket",
                "warmup_with_tuning_s": round(t_tune, 1), "cublaslt_version": lt_version,
                "source": "oracle/_ref/libd1ref.so: the reference's cuda/kernels.cu + cuda/gemm.cu (cuBLASLt) built "
                          "unchanged, driven through this repository's C++ restatement of src/model.rs (the "
                          "reference's Rust host needs cargo, which this image lacks)"}
    finally:
        model.close()


ONLY_GEMM = {"in_proj": (3072, 1024, 0), "qkv": (2048, 1024, 0), "out_proj": (1024, 1024, 1), "w2": (1024, 4608, 1)}


def only_gemm(pkg, dev, stream, name, reps=20, warm=3):
    """One trunk projection at M=8192 in its trunk form (fp16 store for in_proj / qkv, the fp32 residual reduce-add
    for out_proj / w2) under the plan d1_lt_tune picks: the small case for an ncu capture of that GEMM."""
    import ctypes as C
    import torch
    lib = pkg.lib()
    ctx = lib.d1_lt_init(0)
    N, K, res = ONLY_GEMM[name]
    M = TOKENS
    st = C.c_void_p(stream.cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    g = torch.Generator(device=dev).manual_seed(9)
    x = torch.randn(M, K, device=dev, generator=g).half()
    wt = (torch.randn(N, K, device=dev, generator=g) * 0.02).half()
    y = torch.zeros(M, N, device=dev) if res else torch.empty(M, N, device=dev, dtype=torch.float16)
    lib.d1_lt_tune(ctx, M, N, K, K, K, 0, N, res, 0, 1, st)
    fn = lambda: lib.d1_lt_gemm(ctx, M, N, K, P(x), K, P(wt), K, 0, P(y), N, res, 0, 1.0, float(res), st)  # noqa: E731
    for _ in range(warm):
        assert fn() == 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    err = lib.d1_lt_error(ctx)
    lib.d1_lt_destroy(ctx)
    if err:
        raise RuntimeError(f"GEMM kernel reported error {err}")
    us = e0.elapsed_time(e1) / reps * 1e3
    _, tflops, _ = peaks()
    tf = 2.0 * M * N * K / (us * 1e-6) / 1e12
    return {"gemm": name, "M": M, "N": N, "K": K, "form": "residual f32" if res else "store f16", "us": round(us, 2),
            "tflops": round(tf, 1), "frac_of_peak": round(tf / tflops, 3)}


def swiglu_gemm_ms(pkg, dev, stream, reps=20):
    """Average CUDA-event time of one d1_gemm_swiglu launch at M=8192 (the trunk's w1|w3 projection)."""
    import ctypes as C
    import torch
    lib = pkg.lib()
    ctx = lib.d1_lt_init(0)
    M, F, K = TOKENS, 4608, 1024
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(M, K, device=dev, generator=g).half()
    wt = (torch.randn(2 * F, K, device=dev, generator=g) * 0.02).half()
    out = torch.empty(M, F, device=dev, dtype=torch.float16)
    st = C.c_void_p(stream.cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())
    for _ in range(3):
        lib.d1_gemm_swiglu(ctx, M, F, K, P(x), K, P(wt), K, P(out), F, st)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    for _ in range(reps):
        lib.d1_gemm_swiglu(ctx, M, F, K, P(x), K, P(wt), K, P(out), F, st)
    g1.record(stream)
    torch.cuda.synchronize(dev)
    err = lib.d1_lt_error(ctx)
    lib.d1_lt_destroy(ctx)
    if err:
        raise RuntimeError(f"GEMM kernel reported error {err}")
    return g0.elapsed_time(g1) / reps


SWEEP_M = (256, 1024, 4096, 8192, 16384)
SWEEP_NK = ((3072, 1024, "conv in_proj"), (2048, 1024, "fused QKV"), (1024, 1024, "out_proj"),
            (9216, 1024, "w1|w3"), (1024, 4608, "w2"))


def gemm_sweep(pkg, dev, stream, reps=20):
    """C = A.W^T for every M x (N, K), fp16 in, fp32 accumulate, after d1_lt_tune (effort 1).
    Per shape: the plain fp16-store GEMM and the trunk's own form of that projection (residual add into the fp32
    stream for out_proj / w2, the fused SwiGLU for w1|w3). Beside each form, the reference's own path for it
    (oracle/_ref/libd1ref.so, the reference's cuda/gemm.cu + cuda/kernels.cu built unchanged): d1_lt_tune at
    effort 0 (the cuBLASLt heuristic candidates, each timed; the reference engine's effort-1 search ends the process
    with SIGSEGV on B200), then d1_lt_gemm; for w1|w3 its GEMM into [g|u] plus its k_swiglu. One JSON line per shape;
    CUDA-event averages over `reps` launches of inputs larger than L2 at M >= 8192 (the smaller shapes are
    L2-resident by nature)."""
    import ctypes as C
    import torch
    lib = pkg.lib()
    ctx = lib.d1_lt_init(0)
    ref = None
    if REF_LIB.exists():
        ref = C.CDLL(str(REF_LIB))
        pkg.abi.bind(ref, (pkg.abi.KERNELS,))
        rctx = ref.d1_lt_init(32 << 20)
    st = C.c_void_p(stream.cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    _, tflops, kind = peaks()
    g = torch.Generator(device=dev).manual_seed(1)
    out = []

    def timed(fn):
        for _ in range(3):
            assert fn() == 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps * 1e3

    for (N, K, name) in SWEEP_NK:
        wt = (torch.randn(N, K, device=dev, generator=g) * 0.02).half()
        for M in SWEEP_M:
            x = torch.randn(M, K, device=dev, generator=g).half()
            y16 = torch.empty(M, N, device=dev, dtype=torch.float16)
            forms = {"store_f16": lambda lb, c: lb.d1_lt_gemm(c, M, N, K, P(x), K, P(wt), K, 0, P(y16), N, 0, 0, 1.0,
                                                               0.0, st)}
            tunes = [(0,)]
            if N == 1024:
                y32 = torch.zeros(M, N, device=dev)
                forms["trunk_residual_f32"] = lambda lb, c: lb.d1_lt_gemm(c, M, N, K, P(x), K, P(wt), K, 0, P(y32),
                                                                           N, 1, 0, 1.0, 1.0, st)
                tunes.append((1,))
            if N == 9216:
                act = torch.empty(M, N // 2, device=dev, dtype=torch.float16)

                def swiglu(lb, c):
                    if lb is lib:
                        return lb.d1_gemm_swiglu(c, M, N // 2, K, P(x), K, P(wt), K, P(act), N // 2, st)
                    e = lb.d1_lt_gemm(c, M, N, K, P(x), K, P(wt), K, 0, P(y16), N, 0, 0, 1.0, 0.0, st)
                    return e or lb.d1_swiglu(P(y16), P(act), M, N // 2, st)
                forms["trunk_swiglu"] = swiglu
            for (y_f32,) in tunes:
                lib.d1_lt_tune(ctx, M, N, K, K, K, 0, N, y_f32, 0, 1, st)
                if ref is not None:
                    assert ref.d1_lt_tune(rctx, M, N, K, K, K, 0, N, y_f32, 0, REF_SWEEP_EFFORT, st) > 0
            if ref is not None:
                ref.d1_lt_free_scratch(rctx)
            rec = {"sweep": "config1", "shape": name, "M": M, "N": N, "K": K}
            for fname, fn in forms.items():
                us = timed(lambda: fn(lib, ctx))
                tf = 2.0 * M * N * K / (us * 1e-6) / 1e12
                rec[fname] = {"us": round(us, 2), "tflops": round(tf, 1), "frac_of_peak": round(tf / tflops, 3)}
                if ref is not None:
                    rus = timed(lambda: fn(ref, rctx))
                    rtf = 2.0 * M * N * K / (rus * 1e-6) / 1e12
                    rec[fname]["reference"] = {"us": round(rus, 2), "tflops": round(rtf, 1),
                                               "frac_of_peak": round(rtf / tflops, 3)}
                    rec[fname]["speedup_vs_reference"] = round(rus / us, 3)
            rec["peak"] = f"{tflops} TFLOP/s ({kind}, bf16 cuBLAS burst)"
            if ref is not None:
                rec["reference_plans"] = (f"d1_lt_tune effort {REF_SWEEP_EFFORT}: the cuBLASLt heuristic candidates, "
                                          "each timed (its effort-1 search ends the process with SIGSEGV on B200)")
            out.append(rec)
            print(json.dumps(rec), flush=True)
    err = lib.d1_lt_error(ctx)
    lib.d1_lt_destroy(ctx)
    if err:
        raise RuntimeError(f"GEMM kernel reported error {err}")
    return out


def hbm_kernels(pkg, dev, reps=40, warm=5):
    """The trunk's HBM-bound kernels at the metric's shape (8192 rows, D = 1024), each launched alone: RMSNorm (fp32
    [T, D] -> fp16, 6,144 B/token), LayerNorm (same bytes), the double-gated short conv (fp16 [T, 3D] -> fp16 [T, D],
    8,192 B/token). Inputs rotate over enough buffer sets to exceed the 126 MB L2, so every launch reads from DRAM.
    CUDA-event average per launch; achieved GB/s = algorithmic bytes / time, against the measured HBM copy peak."""
    import ctypes as C
    import torch
    lib = pkg.lib()
    hbm, _, kind = peaks()
    T, D = TOKENS, 1024
    st = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    g = torch.Generator(device=dev).manual_seed(5)
    arr = (pkg.abi.SeqInfo * N_SEQS)()
    for i in range(N_SEQS):
        arr[i].start, arr[i].len = i * SEQ_LEN, SEQ_LEN
    seqs = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(dev)
    tok = torch.arange(T, device=dev, dtype=torch.int32) // SEQ_LEN
    w = torch.ones(D, device=dev)
    b = torch.zeros(D, device=dev)
    convw = torch.randn(D, 3, device=dev, generator=g) * 0.3
    sets = 4  # 4 x (32 + 16) MB for the norms, 4 x (48 + 16) MB for the conv: each above L2
    hs = [torch.randn(T, D, device=dev, generator=g) for _ in range(sets)]
    ys = [torch.empty(T, D, device=dev, dtype=torch.float16) for _ in range(sets)]
    bcus = [torch.randn(T, 3 * D, device=dev, generator=g).half() for _ in range(sets)]
    cases = {
        "k_rmsnorm": (6144, lambda i: lib.d1_rmsnorm(P(hs[i]), P(w), P(ys[i]), T, D, 1e-5, st)),
        "k_layernorm": (6144, lambda i: lib.d1_layernorm(P(hs[i]), None, 1.0, P(w), P(b), P(ys[i]), None, T, D, 1e-5,
                                                         st)),
        "k_shortconv": (8192, lambda i: lib.d1_shortconv(P(bcus[i]), P(convw), P(tok), P(seqs), P(ys[i]), T, D, 0, st)),
    }
    out = {}
    for name, (bpt, fn) in cases.items():
        for i in range(warm):
            assert fn(i % sets) == 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            fn(i % sets)
        e1.record()
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) / reps * 1e3
        gbs = bpt * T / (us * 1e-6) / 1e9
        out[name] = {"us": round(us, 2), "bytes_per_launch": bpt * T, "gbs": round(gbs, 1),
                     "frac_of_hbm": round(gbs / hbm, 3)}
    rec = {"sweep": "hbm_kernels", "rows": T, "D": D, "kernels": out, "peak": f"{hbm} GB/s ({kind} HBM copy)"}
    print(json.dumps(rec), flush=True)


def attn_config2(pkg, dev, reps=20, warm=3):
    """packed varlen bidirectional GQA attention (16 query heads, 8 KV heads, head dim 64,
    Q/K/V N(0,1) fp16, seed 2), lengths log-normal (median 384, sigma 1) clipped to 32..16384, at 2048, 8192 and
    16384 packed tokens. Times this library's tcgen05 kernel (d1_flash_attn_tc, 256-row work items longest sequence
    first, as the runners build them), its reference
    ABI entry d1_flash_attn with 64-row items as the reference builds them ("abi": the list split onto the tcgen05
    kernel), the same entry with that list shuffled ("mma_sync": no whole block left, so every item runs on the
    mma.sync kernel) and the reference's own k_flash_attn (d1_flash_attn of oracle/_ref/libd1ref.so) on the same
    inputs; FLOPs = sum over sequences of 4 L^2 64 x 16."""
    import ctypes as C
    import torch
    from fast_d1_omni_b200.weights import lognormal_lengths
    lib = pkg.lib()
    ref = None
    if REF_LIB.exists():
        ref = C.CDLL(str(REF_LIB))
        pkg.abi.bind(ref, (pkg.abi.KERNELS,))
    _, tflops, kind = peaks()
    st = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    for total in (2048, 8192, 16384):
        lens = lognormal_lengths(2, total)
        arr = (pkg.abi.AttnSeq * len(lens))()
        s = 0
        for i, n in enumerate(lens):
            arr[i].q_start, arr[i].q_len, arr[i].kv_start, arr[i].kv_len = s, n, s, n
            s += n
        meta = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(dev)

        def work(step, order):
            w = [(i, q) for i in order for q in range(0, lens[i], step)]
            return torch.tensor(np.asarray(w, np.int32).reshape(-1), device=dev), len(w)
        w64, n64 = work(64, range(len(lens)))  # the reference's list: every 64-row tile, in sequence order
        # the runners' list: one item per 256-row block, longest sequence first (runner.cpp work_items)
        w256, n256 = work(256, sorted(range(len(lens)), key=lambda i: -lens[i]))
        wsh = w64.view(-1, 2)[torch.randperm(n64, generator=torch.Generator().manual_seed(5)).to(dev)].reshape(-1)
        g = torch.Generator(device=dev).manual_seed(2)
        qkv = torch.randn(total, 2048, device=dev, generator=g).half()
        out = torch.empty(total, 1024, device=dev, dtype=torch.float16)
        Q, K, V = qkv, qkv[:, 1024:], qkv[:, 1536:]
        runs = {"tcgen05": lambda: lib.d1_flash_attn_tc(P(Q), 2048, P(K), P(V), 2048, 512, P(out), 1024, P(meta),
                                                        P(w256), n256, 16, 2, 0.125, total, total, st),
                "abi": lambda: lib.d1_flash_attn(P(Q), 2048, P(K), P(V), 2048, 512, None, None, None, P(out), 1024,
                                                 P(meta), P(w64), n64, 16, 2, 0.125, st),
                "mma_sync": lambda: lib.d1_flash_attn(P(Q), 2048, P(K), P(V), 2048, 512, None, None, None, P(out),
                                                      1024, P(meta), P(wsh), n64, 16, 2, 0.125, st)}
        if ref is not None:
            runs["reference"] = lambda: ref.d1_flash_attn(P(Q), 2048, P(K), P(V), 2048, 512, None, None, None,
                                                          P(out), 1024, P(meta), P(w64), n64, 16, 2, 0.125, st)
        flops = sum(4.0 * n * n * 64 * 16 for n in lens)
        rec = {"sweep": "config2", "tokens": total, "sequences": len(lens), "gflop": round(flops / 1e9, 2)}
        for name, fn in runs.items():
            for _ in range(warm):
                assert fn() == 0
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            torch.cuda.synchronize(dev)
            us = e0.elapsed_time(e1) / reps * 1e3
            tf = flops / (us * 1e-6) / 1e12
            rec[name] = {"us": round(us, 2), "tflops": round(tf, 1), "frac_of_peak": round(tf / tflops, 3)}
        if lib.d1_flash_attn_error():
            raise RuntimeError("attention kernel reported a wait that gave up")
        if "reference" in rec:
            rec["tcgen05_speedup_vs_reference"] = round(rec["reference"]["us"] / rec["tcgen05"]["us"], 3)
            rec["abi_speedup_vs_reference"] = round(rec["reference"]["us"] / rec["abi"]["us"], 3)
        rec["peak"] = f"{tflops} TFLOP/s ({kind}, bf16 cuBLAS burst)"
        print(json.dumps(rec), flush=True)


MIXED_PER_GPU = 48  # config-4 requests per GPU (weak scaling): ~90K trunk tokens, ~11 batches of 8192


def run_mixed(args, rank, world, local, dev):
    """the mixed request stream (70% text, 20% text+image, 10% text+audio; 3 questions each)
    through the continuous-batching engine (csrc/engine.cpp) at max-batch-tokens 8192, one replica per GPU; every
    rank takes its deterministic least-loaded share of the stream (engine.assign) and runs it on its own engine.
    A step is one pass over the rank's share; value = trunk tokens (questions + media prefixes) of all ranks over
    all passes / the slowest rank's device time."""
    import torch
    import torch.distributed as dist
    pkg = load_package()
    from fast_d1_omni_b200.engine import Engine, assign, request_tokens
    from fast_d1_omni_b200.model import AudioModel, TextModel, VisionModel
    from fast_d1_omni_b200.weights import audio_weights, mixed_requests, text_weights, vision_weights
    text = TextModel(text_weights(0), device=local, cap_tokens=TOKENS)
    # GEMM plans: loaded from --plans when a previous run of this build saved them there, else tuned (and saved)
    n_tuned = 0
    if args.plans and Path(args.plans).exists():
        try:
            n_tuned = text.load_plans(args.plans)
        except RuntimeError:
            n_tuned = 0
    if n_tuned == 0:
        n_tuned = text.tune(TOKENS)
        if args.plans and rank == 0:
            text.save_plans(args.plans)
    vision = VisionModel(vision_weights(3), device=local, max_patches=16384)
    audio = AudioModel(audio_weights(4), device=local, max_rows=1536)
    eng = Engine(text, vision, audio, max_batch_tokens=TOKENS)
    reqs = mixed_requests(4, MIXED_PER_GPU * world)
    mine = [r for r, d in zip(reqs, assign(reqs, world)) if d == rank]
    # warm-up covers every request kind (first-use setup of each path stays out of the timed passes), including
    # a 30 s clip and a large image
    warm = mixed_requests(99, 8)
    rng = np.random.default_rng(98)
    warm[0]["media"] = {"kind": "audio", "pcm": rng.standard_normal(30 * 16000, dtype=np.float32) * np.float32(0.1)}
    warm[1]["media"] = {"kind": "images", "crops": [(48, 48, rng.uniform(0, 1, (48 * 48, 768)).astype(np.float16))]}
    passes = max(1, args.steps // 4)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(1, args.warmup // 3)):
        eng.run(warm)
    torch.cuda.synchronize(dev)
    s0 = eng.stats()
    l0 = text.launches
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        torch.cuda.cudart().cudaProfilerStart()  # a profiler started with --profile-from-start off sees only this
        t0 = time.perf_counter()
        e0.record(eng.stream)
        for _ in range(passes):
            res = eng.run(mine)
        e1.record(eng.stream)
        torch.cuda.synchronize(dev)
        wall = time.perf_counter() - t0
        torch.cuda.cudart().cudaProfilerStop()
    s1 = eng.stats()
    dev_s = e0.elapsed_time(e1) / 1e3
    tokens = (s1["tokens"] - s0["tokens"]) + (s1["media_tokens"] - s0["media_tokens"])
    assert tokens == passes * sum(request_tokens(r) for r in mine) and all(e == "" for _, e in res)
    t = torch.tensor([dev_s, wall, float(tokens), float(len(mine) * passes)], dtype=torch.float64, device=dev)
    per_rank = [t.clone()]
    if world > 1:
        per_rank = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(per_rank, t)
        mx = t[:2].clone()
        sm = t[2:].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        t = torch.cat([mx, sm])
    if rank == 0:
        dev_max, wall_max, tok_all, nreq = (float(x) for x in t)
        line = {"metric": "mixed continuous-batching trunk tokens/s (BASELINE config 4)", "value": tok_all / dev_max,
                "unit": "tokens/s", "n_gpus": world, "warmup": args.warmup,
                "steps": passes, "ms_per_step": dev_max * 1e3 / passes, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None,
                "dtype": "f16", "data": "synthetic (seeded random weights, token ids, images and waveforms)",
                "config": {"workload": f"config 4: {MIXED_PER_GPU} requests per GPU (70% text 128-2048 tokens per "
                                       "question, 20% text+image of config-3 sides, 10% text+audio 1-30 s through the "
                                       "GPU log-mel front end), 3 questions x 4 options, max-batch-tokens 8192",
                           "parallelism": f"replicas x{world}, deterministic least-loaded request split",
                           "gemm_plans": f"tuned at startup ({n_tuned} plans)"},
                "requests": int(nreq), "requests_per_s": nreq / dev_max,
                "e2e": {"value": tok_all / wall_max, "unit": "tokens/s", "note": "wall clock, host request buffers"},
                "engine": {k: s1[k] - s0[k] for k in s1}, "gpu_launches_text_runner": text.launches - l0,
                "per_rank": [{"rank": i, "device_s": round(float(r[0]), 4), "wall_s": round(float(r[1]), 4),
                              "tokens": int(r[2]), "requests": int(r[3])} for i, r in enumerate(per_rank)],
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    eng.close()
    audio.close()
    vision.close()
    text.close()


def attention_launches(pkg, dev, seq_len, reps=20, warm=3):
    """The runners' attention (d1_flash_attn_tc: trunk shapes, 16 heads, GQA 2, head dim 64) on 8192 / seq_len packed
    sequences of seq_len tokens; average CUDA-event time per launch. The small case for an ncu capture."""
    import ctypes as C
    import torch
    lib = pkg.lib()
    n = TOKENS // seq_len
    arr = (pkg.abi.AttnSeq * n)()
    work = []
    for i in range(n):
        arr[i].q_start, arr[i].q_len, arr[i].kv_start, arr[i].kv_len = i * seq_len, seq_len, i * seq_len, seq_len
        work += [(i, q) for q in range(0, seq_len, 256)]  # one item per 256-row block, as the runners pass it
    meta = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(dev)
    wk = torch.tensor(np.asarray(work, np.int32).reshape(-1), device=dev)
    g = torch.Generator(device=dev).manual_seed(2)
    qkv = torch.randn(TOKENS, 2048, device=dev, generator=g).half()
    out = torch.empty(TOKENS, 1024, device=dev, dtype=torch.float16)
    st = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    f = lambda: lib.d1_flash_attn_tc(P(qkv), 2048, P(qkv[:, 1024:]), P(qkv[:, 1536:]), 2048, 512, P(out), 1024,  # noqa: E731
                                     P(meta), P(wk), len(work), 16, 2, 0.125, TOKENS, TOKENS, st)
    for _ in range(warm):
        assert f() == 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        f()
    e1.record()
    torch.cuda.synchronize(dev)
    if lib.d1_flash_attn_error():
        raise RuntimeError("attention kernel reported a wait that gave up")
    us = e0.elapsed_time(e1) / reps * 1e3
    flops = n * 4.0 * seq_len * seq_len * 64 * 16
    return us, flops / (us * 1e-6) / 1e12


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="d1", choices=["d1", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="text", choices=["text", "mixed"],
                    help="text: the metric's 8192-token text batches; mixed: BASELINE config 4 through the engine")
    ap.add_argument("--gemm-sweep", action="store_true",
                    help="BASELINE config 1: time every GEMM shape (one JSON line each) instead of the forward")
    ap.add_argument("--only-attention", type=int, default=0, metavar="L",
                    help="run only the runners' attention kernel on 8192/L sequences of L tokens (an ncu case)")
    ap.add_argument("--only-roofline", action="store_true",
                    help="run only the dominant GEMM (fused SwiGLU, M=8192) launches: the small case for ncu")
    ap.add_argument("--only-gemm", default="", choices=[""] + list(ONLY_GEMM),
                    help="run only one trunk projection GEMM at M=8192 in its trunk form (an ncu case)")
    ap.add_argument("--hbm-kernels", action="store_true",
                    help="time RMSNorm, LayerNorm and the short conv alone at 8192 x 1024 (an ncu case as well)")
    ap.add_argument("--attn-config2", action="store_true",
                    help="BASELINE config 2: attention at 2048/8192/16384 packed tokens, this library and the reference")
    ap.add_argument("--ref-engine-child", type=int, default=-1, metavar="EFFORT", help=argparse.SUPPRESS)
    ap.add_argument("--plans", default="", metavar="PATH",
                    help="--workload mixed: GEMM plan file to load (or to write after tuning when it is missing)")
    ap.add_argument("--sustained-steps", type=int, default=SUSTAINED_STEPS,
                    help="steps of the second (>= 2 s) timed region; 0 skips it")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.ref_engine_child >= 0:  # the reference engine in its own process (see reference_gpu_engine_child)
        res = reference_gpu_engine(args.steps, args.warmup, args.ref_engine_child)
        print(json.dumps(res), flush=True)
        return
    if args.gemm_sweep:  # the reference's cuBLASLt beside this library's GEMMs: load its cuBLASLt before torch
        preload_reference_cublaslt()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    pkg = load_package()
    if args.workload == "mixed":
        run_mixed(args, rank, world, local, dev)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.gemm_sweep:
        if rank == 0:
            gemm_sweep(pkg, dev, torch.cuda.Stream(dev))
        return
    if args.only_gemm:
        if rank == 0:
            print(json.dumps(only_gemm(pkg, dev, torch.cuda.Stream(dev), args.only_gemm, reps=args.steps,
                                       warm=args.warmup)), flush=True)
        return
    if args.hbm_kernels:
        if rank == 0:
            hbm_kernels(pkg, dev, reps=max(args.steps, 10), warm=args.warmup)
        return
    if args.attn_config2:
        if rank == 0:
            attn_config2(pkg, dev, reps=args.steps, warm=args.warmup)
        return
    if args.only_attention:
        us, tf = attention_launches(pkg, dev, args.only_attention, reps=args.steps, warm=args.warmup)
        if rank == 0:
            print(json.dumps({"kernel": "k_flash_attn_tc", "seq_len": args.only_attention, "us": us, "tflops": tf}),
                  flush=True)
        return
    if args.only_roofline:
        ms = swiglu_gemm_ms(pkg, dev, torch.cuda.Stream(dev))
        if rank == 0:
            print(json.dumps({"kernel": "fused SwiGLU GEMM", "M": TOKENS, "gemm_ms": ms}), flush=True)
        return
    from fast_d1_omni_b200.model import TextModel
    from fast_d1_omni_b200.weights import text_batch, text_weights
    import ctypes as C

    w = text_weights(0)
    model = TextModel(w, device=local, cap_tokens=TOKENS)
    # GEMM plan tuning at startup, as the reference's engine does (src/engine.rs:528-616): every trunk/head shape,
    # every M bucket up to the batch budget; d1_lt_tune times this library's tile configurations and split-K.
    n_tuned = model.tune(TOKENS)
    batches = [text_batch(1000 * rank + i, N_SEQS, SEQ_LEN) for i in range(4)]
    stream = torch.cuda.Stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    # ---------------------------------------------------------------- device-timed steps (value)
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            model.launch(batches[i % 4], i % 2, stream)
        for s in (0, 1):
            model.finish(s) if s in model._pending else None
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        l0 = model.launches
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local) as clk:
            torch.cuda.cudart().cudaProfilerStart()  # a profiler started with --profile-from-start off sees only this
            e0.record(stream)
            for i in range(args.steps):
                model.launch(batches[i % 4], i % 2, stream)
            e1.record(stream)
            torch.cuda.synchronize(dev)
            torch.cuda.cudart().cudaProfilerStop()
        for s in (0, 1):
            model._pending.pop(s, None)
        launches = model.launches - l0
        dev_ms = e0.elapsed_time(e1)
        barrier()

        # ---------------------------------------------------------------- roofline: the fused SwiGLU GEMM alone
        gemm_ms = swiglu_gemm_ms(pkg, dev, stream)
        barrier()

        # ---------------------------------------------------------------- end to end through the API (e2e)
        torch.cuda.synchronize(dev)
        barrier()
        t0 = time.perf_counter()
        for i in range(args.steps):
            model.launch(batches[i % 4], i % 2, stream)
            if i >= 1:
                model.finish((i - 1) % 2)
        model.finish((args.steps - 1) % 2)
        torch.cuda.synchronize(dev)
        e2e_s = time.perf_counter() - t0
        h2d = int(model.L.d1h_h2d_bytes(model.ws, 0))
        d2h = int(model.L.d1h_d2h_bytes(model.ws, 0))
        barrier()

        # ---------------------------------------------------------------- sustained: >= 2 s of steps (value_sustained)
        sus_ms, sus_clk = 0.0, None
        if args.sustained_steps > 0:
            torch.cuda.synchronize(dev)
            barrier()
            torch.cuda.synchronize(dev)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with Clocks(local) as sus_clk:
                s0.record(stream)
                for i in range(args.sustained_steps):
                    model.launch(batches[i % 4], i % 2, stream)
                s1.record(stream)
                torch.cuda.synchronize(dev)
            for s in (0, 1):
                model._pending.pop(s, None)
            sus_ms = s0.elapsed_time(s1)
            barrier()

    # ---------------------------------------------------------------- aggregate over ranks
    t = torch.tensor([dev_ms, e2e_s, sus_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_ms_max, e2e_max, sus_ms_max = float(t[0]), float(t[1]), float(t[2])
    total_tokens = TOKENS * args.steps * world
    value = total_tokens / (dev_ms_max / 1e3)
    e2e_value = total_tokens / e2e_max

    if rank == 0:
        hbm, tflops, kind = peaks()
        achieved = SWIGLU_FLOP_PER_TOKEN * TOKENS / (gemm_ms / 1e3) / 1e12
        line = {
            "metric": "prefill tokens/s per B200 at 8192-token batches", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dev_ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded random weights and token ids)",
            "config": {"workload": f"text trunk+head forward (config-0 architecture), {TOKENS}-token batches of "
                                   f"{N_SEQS}x{SEQ_LEN} tokens, 3 markers per sequence",
                       "global_batch_tokens": TOKENS * world, "parallelism": f"replicas x{world}",
                       "l2": "inputs larger than L2 (weights + activations > 700 MB)",
                       "gemm_plans": f"tuned at startup ({n_tuned} shape x bucket plans)"},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gemm_tflops_trunk_equiv": GEMM_FLOP_PER_TOKEN * value / world / 1e12,
            "roofline": {"bound": "tensor", "kernel": "k_gemm_tc2<256,6,EPI_SWIGLU> (w1|w3 + SwiGLU, CTA pair), M=8192",
                         "achieved": achieved, "peak": tflops, "unit": "TFLOP/s", "frac": achieved / tflops,
                         "peak_kind": f"{kind} (bf16 cuBLAS burst)", "traffic": SWIGLU_NCU_DRAM_BYTES_M8192,
                         "traffic_note": "ncu DRAM read+write of one launch at this shape (2026-12-01 capture); below "
                                         "the 111 MB algorithmic bytes because the output is still dirty in L2 when "
                                         "the kernel ends",
                         "gemm_ms": gemm_ms},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        if sus_ms_max > 0:
            sus_tokens = TOKENS * args.sustained_steps * world
            line["value_sustained"] = {"value": sus_tokens / (sus_ms_max / 1e3), "unit": "tokens/s",
                                       "steps": args.sustained_steps, "seconds": sus_ms_max / 1e3,
                                       "ms_per_step": sus_ms_max / args.sustained_steps,
                                       "clocks": sus_clk.summary() if sus_clk else None,
                                       "note": "the same steps back to back for >= 2 s, after the burst region; "
                                               "clocks settle at the 1 kW power cap"}
        if not args.no_cpu_baseline:
            v, dt = cpu_sample(2)
            line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
                                    "sample": f"2 sequences x {SEQ_LEN} tokens of the workload, oracle fp32 "
                                              f"({dt:.1f} s)"}
        print(json.dumps(line), flush=True)

    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
