"""Audio encoder (FastConformer + adapter, src/audio.rs:505-594) and its two new kernels through the C ABI.

* d1_sgemm (fp32 GEMM + bias/act) against a float64 host GEMM; deterministic across calls.
* d1_relpos_attn against the reference's path for the same op: fp32 ac / bd from the same fp16 operands, the
  reference's own d1_relpos_softmax (oracle/_ref/libd1ref.so), P.V — and against the oracle.
* The encoder (AudioModel, several clips packed into one call) against the fp32 oracle and against the
  reference's F16 engine: src/audio.rs:505-594 restated call for call below with the reference's kernels and its
  cuBLASLt GEMM (d1_lt_gemm of libd1ref.so); Blas::sgemm / Blas::gemm_batched, which the reference calls in
  cuBLAS directly from Rust, are torch matmuls (cuBLAS) with fp32 accumulation.

Inputs: BASELINE config 4's audio — clips of 1-30 s of N(0, 0.1) waveform at 16 kHz through the log-mel front end
(the oracle's restatement of src/audio.rs:238-299), random-init encoder weights seed 4.
Tolerances: relative RMS of the fp32 output embeddings <= 1e-2 against the fp32 oracle and <= 5e-3 against the
reference engine; fp32 GEMMs within 1e-5 relative to the row scale; attention within 4e-3 absolute.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import REF_LIB
from oracle import d1_oracle as O
from ref_engines import RefAudioEngine

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def P(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def ST():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


def rel_rms(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.sqrt(((got - ref) ** 2).mean()) / np.sqrt((ref ** 2).mean()))


# ------------------------------------------------------------------------------------------------ d1_sgemm

@pytest.mark.parametrize("M,N,K,beta,bias,act", [
    (24000, 256, 256, 0.0, True, 1),     # subsampling pointwise conv of a 30 s clip (128 x 128 tiles)
    (1500, 256, 256, 1.0, False, 0),     # 64 x 64 tiles, beta = 1 (the reference's fill_rows + sgemm form)
    (375, 512, 4096, 0.0, True, 0),      # pre-encode projection: split-K across a CTA cluster
    (13, 512, 4096, 0.0, True, 0),
    (100, 70, 37, 0.5, True, 4),         # ragged, unaligned K: scalar loads
])
def test_sgemm(gpu_lib, M, N, K, beta, bias, act):
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K)).astype(np.float32)
    y0 = rng.standard_normal((M, N), dtype=np.float32)
    b = rng.standard_normal(N, dtype=np.float32) * np.float32(0.1)
    ref = x.astype(np.float64) @ w.astype(np.float64).T + beta * y0
    if bias:
        ref = ref + b
    ref = O.apply_act(ref.astype(np.float32), act)
    outs = []
    for _ in range(2):
        y = dev(y0)
        assert gpu_lib.d1_sgemm(M, N, K, P(dev(x)), K, P(dev(w)), K, P(y), N, beta, P(dev(b)) if bias else None, act,
                                ST()) == 0
        outs.append(y.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])  # deterministic (split-K sums in a fixed order)
    scale = np.abs(ref).max(axis=1, keepdims=True) + 1e-3
    assert (np.abs(outs[0] - ref) <= 1e-5 * scale + 1e-6).all()


def test_sgemm_rejects_bad_arguments(gpu_lib):
    x = torch.zeros(4, 4, device="cuda")
    assert gpu_lib.d1_sgemm(4, 4, 4, P(x), 3, P(x), 4, P(x), 4, 0.0, None, 0, ST()) == -1  # ldx < K
    assert gpu_lib.d1_sgemm(0, 4, 4, P(x), 4, P(x), 4, P(x), 4, 0.0, None, 0, ST()) == 0    # empty: no-op


# ------------------------------------------------------------------------------------------------ d1_relpos_attn

def _relpos_inputs(lengths, seed=7):
    rng = np.random.default_rng(seed)
    R = sum(lengths)
    mk = lambda *s: (rng.standard_normal(s, dtype=np.float32)).astype(np.float16)  # noqa: E731
    return mk(R, 512), mk(R, 512), mk(R, 512), mk(R, 512)


@pytest.mark.parametrize("lengths", [[38], [1, 64, 65, 130], [375, 13, 200]])
def test_relpos_attn_vs_reference_pieces(gpu_lib, ref_lib, lengths):
    """Per clip the reference computes ac = qu.k^T, bd = qv.pp^T (fp32, cuBLAS), d1_relpos_softmax, P.V."""
    qu, qv, k, v = _relpos_inputs(lengths)
    rng = np.random.default_rng(11)
    max_len = max(lengths)
    # per-layer table layout: row center + j - i, center = 383 (the runner's), 767 rows
    table = (rng.standard_normal((767, 512), dtype=np.float32) * np.float32(0.5)).astype(np.float16)
    offs = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    o = torch.zeros(offs[-1], 512, dtype=torch.float16, device="cuda")
    ins = [dev(a) for a in (qu, qv, k, v)]
    assert gpu_lib.d1_relpos_attn(*[P(t) for t in ins], 512, P(dev(table)), 512, 767, 383, P(o), 512, P(dev(offs)),
                                  len(lengths), max_len, 8, 0.125, ST()) == 0
    got = o.cpu().numpy().astype(np.float32)
    assert gpu_lib.d1_relpos_attn_error() == 0
    for c, T in enumerate(lengths):
        s = slice(offs[c], offs[c + 1])
        pp = table[383 - (T - 1):383 + T]  # the reference's per-clip pp rows: relative positions T-1 .. -(T-1)
        tq = [torch.from_numpy(a[s]).cuda().float().view(T, 8, 64).transpose(0, 1) for a in (qu, qv, k, v)]
        tp = torch.from_numpy(pp).cuda().float().view(2 * T - 1, 8, 64).transpose(0, 1)
        ac = (tq[0] @ tq[2].transpose(1, 2)).contiguous()
        bd = (tq[1] @ tp.transpose(1, 2)).contiguous()
        probs = torch.empty(8, T, T, dtype=torch.float16, device="cuda")
        assert ref_lib.d1_relpos_softmax(P(ac), P(bd), P(probs), T, 8, 0.125, ST()) == 0
        ref = (probs.float() @ tq[3]).transpose(0, 1).reshape(T, 512).half().cpu().numpy().astype(np.float32)
        assert np.abs(got[s] - ref).max() <= 4e-3, (T, np.abs(got[s] - ref).max())
        want = O.relpos_attention(qu[s], qv[s], k[s], v[s], pp.astype(np.float32))
        assert np.abs(got[s] - want).max() <= 4e-3
    # the reference's own layout (pp of the clip alone, center T-1) gives the same result
    T = lengths[0]
    o2 = torch.zeros(T, 512, dtype=torch.float16, device="cuda")
    pp = dev(table[383 - (T - 1):383 + T])
    assert gpu_lib.d1_relpos_attn(*[P(t) for t in ins], 512, P(pp), 512, 2 * T - 1, T - 1, P(o2), 512,
                                  P(dev(np.array([0, T], np.int32))), 1, T, 8, 0.125, ST()) == 0
    assert np.array_equal(o2.cpu().numpy(), o[:T].cpu().numpy())


def test_relpos_attn_rejects_long_clips(gpu_lib):
    x = torch.zeros(8, 512, dtype=torch.float16, device="cuda")
    offs = dev(np.array([0, 8], np.int32))
    assert gpu_lib.d1_relpos_attn(P(x), P(x), P(x), P(x), 512, P(x), 512, 8, 4, P(x), 512, P(offs), 1, 385, 8,
                                  0.125, ST()) == -1


# ------------------------------------------------------------------------------------------------ encoder

@pytest.fixture(scope="module")
def aw(pkg):
    from fast_d1_omni_b200.weights import audio_weights
    return audio_weights(4)


@pytest.fixture(scope="module")
def clips(pkg):
    """Config-4 audio: 4 clips (28.3, 10.3, 10.8, 5.7 s) plus a 0.4 s clip (padded to 0.5 s by the front end)."""
    from fast_d1_omni_b200.weights import audio_clips
    waves = audio_clips(4) + [np.random.default_rng(5).standard_normal(6400).astype(np.float32) * np.float32(0.1)]
    return [O.log_mel(w) for w in waves]


@pytest.fixture(scope="module")
def amodel(pkg, gpu_lib, aw):
    from fast_d1_omni_b200.model import AudioModel
    m = AudioModel(aw, max_rows=1536)
    yield m
    m.close()


def test_encoder_vs_oracle(amodel, aw, clips):
    got = amodel.encode(clips).cpu().numpy()
    assert got.shape == (sum(amodel.out_len(v) for _, v in clips), 1024)
    assert np.isfinite(got).all()
    o = 0
    for mel, valid in clips:
        t = amodel.out_len(valid)
        if valid <= 1100:  # the fp32 oracle on the shorter clips (the long one is covered by the engine check)
            want = O.audio_encode(aw, mel, valid, "f32")
            assert rel_rms(got[o:o + t], want) <= 1e-2, (valid, rel_rms(got[o:o + t], want))
        o += t


def test_encoder_vs_reference_engine(pkg, ref_lib, amodel, aw, clips):
    m = torch.backends.cuda.matmul
    old = (m.allow_tf32, m.allow_fp16_reduced_precision_reduction)
    m.allow_tf32, m.allow_fp16_reduced_precision_reduction = False, False
    try:
        eng = RefAudioEngine(ref_lib, aw)
        got = amodel.encode(clips).cpu().numpy()
        o = 0
        for mel, valid in clips:
            t = amodel.out_len(valid)
            ref = eng.encode(mel, valid)
            assert rel_rms(got[o:o + t], ref) <= 5e-3, (valid, rel_rms(got[o:o + t], ref))
            o += t
    finally:
        m.allow_tf32, m.allow_fp16_reduced_precision_reduction = old


def test_encoder_batching_and_unfused(pkg, amodel, aw, clips):
    """Packed clips equal clips encoded one by one; the reference's unfused call sequence gives the same result."""
    from fast_d1_omni_b200.model import AudioModel
    packed = amodel.encode(clips).cpu().numpy()
    o = 0
    for c in clips:
        alone = amodel.encode([c]).cpu().numpy()
        assert rel_rms(alone, packed[o:o + alone.shape[0]]) <= 1e-3
        o += alone.shape[0]
    un = AudioModel(aw, fused=False, max_rows=1536)
    try:
        assert rel_rms(un.encode(clips).cpu().numpy(), packed) <= 2e-3
    finally:
        un.close()


def test_encoder_rejects_bad_clips(amodel):
    mel = np.zeros((3001, 128), np.float32)
    with pytest.raises(RuntimeError):
        amodel.encode([(mel, 3001)])
    with pytest.raises(RuntimeError):
        amodel.encode([(mel, 3000)] * 5)  # 5 x 375 rows > max_rows 1536
