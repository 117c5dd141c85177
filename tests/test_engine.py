"""The continuous-batching engine (src/engine.rs:149-525 restated in csrc/engine.cpp), the dispatcher, and the GPU
log-mel front end (src/audio.rs:238-299), through the C ABI.

* Text requests through the engine (several batches under a small token budget, two batches in flight) give the
  logits the runner gives for the same questions in one batch.
* Media requests end to end — image crops through the vision tower, a waveform through the GPU log-mel front end
  and the audio encoder, each prefix through the trunk once, the questions over the cached prefix — against the
  fp32 oracle chain (vision_encode / log_mel + audio_encode -> launch_prefix -> launch_text), with the north-star
  bar: per question centred |dlogit| mean <= 0.01, max <= 0.06, no top-answer flips.
* The dispatcher over two engines gives the single engine's results and spreads the requests.
* d1_log_mel against the oracle's restatement (numpy f64 FFT): within 1e-4 absolute on normalised features.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import d1_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tw(pkg):
    from fast_d1_omni_b200.weights import text_weights
    return text_weights(0)


@pytest.fixture(scope="module")
def tmodel(pkg, gpu_lib, tw):
    from fast_d1_omni_b200.model import TextModel
    m = TextModel(tw, cap_tokens=8192)
    yield m
    m.close()


@pytest.fixture(scope="module")
def vw(pkg):
    from fast_d1_omni_b200.weights import vision_weights
    return vision_weights(3)


@pytest.fixture(scope="module")
def aw(pkg):
    from fast_d1_omni_b200.weights import audio_weights
    return audio_weights(4)


@pytest.fixture(scope="module")
def vmodel(pkg, gpu_lib, vw):
    from fast_d1_omni_b200.model import VisionModel
    m = VisionModel(vw, max_patches=16384)
    yield m
    m.close()


@pytest.fixture(scope="module")
def amodel(pkg, gpu_lib, aw):
    from fast_d1_omni_b200.model import AudioModel
    m = AudioModel(aw, max_rows=1536)
    yield m
    m.close()


def text_requests(seed, n, lo=40, hi=700, questions=3, options=4):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        rows = []
        for _ in range(questions):
            L = int(rng.integers(lo, hi))
            rows.append({"ids": rng.integers(0, 65536, L, dtype=np.int32),
                         "markers": np.sort(rng.choice(L, options, replace=False)).astype(np.int32),
                         "qtype": int(rng.integers(0, 4))})
        out.append({"rows": rows, "media": None})
    return out


def assert_bar(ref, got, sizes, mean_tol=0.01, max_tol=0.06):
    err = O.centred_logit_err(ref, got, sizes)
    assert err.mean() <= mean_tol and err.max() <= max_tol, (err.mean(), err.max())
    assert O.top_flips(ref, got, sizes) == 0


def test_engine_text_equals_runner(tmodel):
    from fast_d1_omni_b200.engine import Engine
    reqs = text_requests(40, 12)
    eng = Engine(tmodel, max_batch_tokens=2048)
    try:
        res = eng.run(reqs)
        st = eng.stats()
    finally:
        eng.close()
    assert st["batches"] >= 6 and st["rows"] == 36 and st["tokens"] == sum(len(r["ids"]) for q in reqs for r in q["rows"])
    for req, (logits, err) in zip(reqs, res):
        assert err == ""
        ref = tmodel([dict(r) for r in req["rows"]])
        assert logits.shape == ref.shape
        assert np.abs(logits - ref).max() <= 2e-3
        assert O.top_flips(ref, logits, [len(r["markers"]) for r in req["rows"]]) == 0


def test_engine_media_vs_oracle(tmodel, vmodel, amodel, tw, vw, aw):
    from fast_d1_omni_b200.engine import Engine
    rng = np.random.default_rng(41)
    img = [(16, 20, rng.uniform(0, 1, (320, 768)).astype(np.float16))]
    wave = (rng.standard_normal(24000, dtype=np.float32) * np.float32(0.1))
    base = text_requests(42, 3, lo=30, hi=200)
    reqs = [dict(base[0], media={"kind": "images", "crops": img}),
            dict(base[1], media={"kind": "audio", "pcm": wave}),
            base[2]]
    eng = Engine(tmodel, vmodel, amodel, max_batch_tokens=8192)
    try:
        res = eng.run(reqs)
        st = eng.stats()
    finally:
        eng.close()
    assert st["media_jobs"] == 2 and st["media_tokens"] == 80 + 19
    mel, valid = O.log_mel(wave)
    embs = [O.vision_encode(vw, img, "f32"), O.audio_encode(aw, mel, valid, "f32"), None]
    for req, emb, (logits, err) in zip(reqs, embs, res):
        assert err == ""
        rows = [dict(r) for r in req["rows"]]
        if emb is not None:
            cache = O.launch_prefix(tw, [emb], "f32")[0]
            rows = [dict(r, prefix=cache) for r in rows]
        ref = O.launch_text(tw, rows, "f32")
        assert_bar(ref, logits, [len(r["markers"]) for r in req["rows"]])


def test_dispatcher_two_engines(tmodel):
    """Two engines of one device sharing one model (and its GEMM context), stepped by two host threads."""
    from fast_d1_omni_b200.engine import Dispatcher, Engine
    reqs = text_requests(43, 10)
    single = Engine(tmodel, max_batch_tokens=4096)
    try:
        want = single.run(reqs)
    finally:
        single.close()
    engines = [Engine(tmodel, max_batch_tokens=4096) for _ in range(2)]
    try:
        d = Dispatcher(engines)
        got = d.run(reqs)
    finally:
        for e in engines:
            e.close()
    assert set(d.assigned) == {0, 1}
    for (a, ea), (b, eb) in zip(got, want):
        assert ea == eb == "" and np.abs(a - b).max() <= 2e-3


def test_engine_rejects_oversized_question(tmodel):
    from fast_d1_omni_b200.engine import Engine
    eng = Engine(tmodel, max_batch_tokens=1024, cap_tokens=1024)
    try:
        big = text_requests(44, 1, lo=1500, hi=1600)[0]
        ok = text_requests(45, 1)[0]
        res = eng.run([big, ok])
    finally:
        eng.close()
    assert "exceeds" in res[0][1] and res[1][1] == ""


@pytest.mark.parametrize("seconds", [0.3, 3.7, 31.0])
def test_log_mel_vs_oracle(gpu_lib, seconds):
    rng = np.random.default_rng(int(seconds * 10))
    wave = rng.standard_normal(int(seconds * 16000), dtype=np.float32) * np.float32(0.1)
    want, valid = O.log_mel(wave)
    x = wave[:30 * 16000]
    if len(x) < 8000:
        x = np.concatenate([x, np.zeros(8000 - len(x), np.float32)])
    xd = torch.from_numpy(x).cuda()
    mel = torch.full((1 + len(x) // 160, 128), float("nan"), device="cuda")
    assert gpu_lib.d1_log_mel(C.c_void_p(xd.data_ptr()), len(x), C.c_void_p(mel.data_ptr()),
                              C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    got = mel.cpu().numpy()
    assert got.shape == want.shape and valid == len(x) // 160
    assert np.abs(got - want).max() <= 1e-4
    assert (got[valid:] == 0).all()


def test_audio_pcm_equals_mel(amodel):
    rng = np.random.default_rng(46)
    waves = [rng.standard_normal(n, dtype=np.float32) * np.float32(0.1) for n in (5000, 50000, 170000)]
    a = amodel.encode_pcm(waves).cpu().numpy()
    b = amodel.encode([O.log_mel(w) for w in waves]).cpu().numpy()
    assert np.sqrt(((a - b) ** 2).mean() / (b ** 2).mean()) <= 1e-3


@pytest.mark.parametrize("rate,seconds", [(8000, 1.3), (22050, 2.0), (44100, 1.7), (48000, 3.1), (11025, 0.9),
                                          (16000, 0.5)])
def test_resample_vs_oracle(gpu_lib, rate, seconds):
    """d1_resample (the WAV front end's conversion to 16 kHz, src/audio.rs:108-148) bit for bit against the oracle's
    restatement: the same fp32 filter table and the same fp32 accumulation order."""
    rng = np.random.default_rng(rate)
    x = (rng.standard_normal(int(rate * seconds)) * 0.1).astype(np.float32)
    want = O.resample(x, rate, 16000)
    n_out = gpu_lib.d1_resample_len(len(x), rate, 16000)
    assert n_out == len(want)
    xd = torch.from_numpy(x).cuda()
    y = torch.full((n_out,), float("nan"), device="cuda")
    assert gpu_lib.d1_resample(C.c_void_p(xd.data_ptr()), len(x), rate, 16000, C.c_void_p(y.data_ptr()),
                               C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    assert np.array_equal(y.cpu().numpy(), want)


def test_resample_rejects_bad_rates(gpu_lib):
    assert gpu_lib.d1_resample_len(100, 0, 16000) == -1
    assert gpu_lib.d1_resample(None, 100, 44100, 0, None, None) == -1
    assert gpu_lib.d1_resample_len(0, 44100, 16000) == 0


def test_audio_pcm_rates_equals_resampled(amodel):
    """Clips at 44.1, 22.05 and 8 kHz through d1h_audio_encode_pcm_rates (resampled on the device) equal the same
    clips resampled by the oracle and encoded as 16 kHz waveforms. The resampler is bit-exact, so the features are
    the same; the encoder's split-K GEMMs sum partial tiles in arrival order, so two calls agree to the run-to-run
    bound of test_audio_pcm_equals_mel (relative RMS 1e-3), not bit for bit."""
    rng = np.random.default_rng(47)
    rates = [44100, 22050, 8000, 16000]
    waves = [(rng.standard_normal(int(r * s)) * 0.1).astype(np.float32) for r, s in zip(rates, (2.3, 1.1, 4.0, 0.7))]
    got = amodel.encode_pcm(waves, rates=rates).cpu().numpy()
    want = amodel.encode_pcm([O.resample(w, r) for w, r in zip(waves, rates)]).cpu().numpy()
    assert got.shape == want.shape
    assert np.sqrt(((got - want) ** 2).mean() / (want ** 2).mean()) <= 1e-3


def test_engine_resampled_audio_vs_oracle(tmodel, amodel, tw, aw):
    """A request whose waveform is at 44.1 kHz: the engine resamples it on the device, computes the log-mel
    features, encodes it and runs the prefix; against the oracle chain resample -> log_mel -> audio_encode ->
    launch_prefix -> launch_text."""
    from fast_d1_omni_b200.engine import Engine, prefix_len
    rng = np.random.default_rng(48)
    wave = (rng.standard_normal(int(44100 * 1.6)) * np.float32(0.1)).astype(np.float32)
    req = dict(text_requests(49, 1, lo=30, hi=150)[0], media={"kind": "audio", "pcm": wave, "rate": 44100})
    eng = Engine(tmodel, None, amodel, max_batch_tokens=8192)
    try:
        (logits, err), = eng.run([req])
        st = eng.stats()
    finally:
        eng.close()
    assert err == ""
    mel, valid = O.log_mel(O.resample(wave, 44100))
    emb = O.audio_encode(aw, mel, valid, "f32")
    assert st["media_tokens"] == emb.shape[0] == prefix_len(req)
    cache = O.launch_prefix(tw, [emb], "f32")[0]
    rows = [dict(r, prefix=cache) for r in req["rows"]]
    ref = O.launch_text(tw, rows, "f32")
    assert_bar(ref, logits, [len(r["markers"]) for r in req["rows"]])
