"""Host side of the GPU resampler (no GPU): the output length the engine and the runner plan with, and properties of
the oracle's restatement of the reference's resampler (src/audio.rs:108-148) that its own tests would check.

* `engine.pcm_len_16k` (the Python dispatcher's prefix length) equals the library's `d1_resample_len` after the WAV
  decoder's 30 s + 1 s cap, for the common rates and for rates with no small common divisor with 16 kHz.
* The filter table: `2*half + 1` taps per phase, symmetric between phase p and the mirrored taps of phase up - p,
  and each phase's taps summing to ~1 (the Kaiser-windowed sinc at cutoff < 1 passes DC).
* The resampled signal: a constant stays constant away from the clip edges; a low-frequency sine keeps its
  amplitude; 16 kHz input passes through unchanged.
"""
import math

import numpy as np
import pytest

from oracle import d1_oracle as O


@pytest.mark.parametrize("rate", [8000, 11025, 22050, 24000, 32000, 44100, 48000, 44101, 96000, 16000])
@pytest.mark.parametrize("n", [0, 1, 999, 48000, 31 * 48000 + 17])
def test_pcm_len_matches_library(pkg, rate, n):
    from fast_d1_omni_b200.engine import pcm_len_16k
    lib = pkg.lib()
    kept = n if rate == 16000 else min(n, 31 * rate)
    assert pcm_len_16k(n, rate) == lib.d1_resample_len(kept, rate, 16000)
    g = math.gcd(rate, 16000)
    assert lib.d1_resample_len(kept, rate, 16000) == kept * (16000 // g) // (rate // g)


@pytest.mark.parametrize("rate", [8000, 22050, 44100, 48000])
def test_filter_table(rate):
    up, down, half, table = O.resample_taps(rate, 16000)
    g = math.gcd(rate, 16000)
    assert (up, down) == (16000 // g, rate // g)
    cutoff = min(up / down, 1.0) * 0.97
    assert half == math.ceil(32.0 / cutoff) and table.shape == (up, 2 * half + 1)
    sums = table.astype(np.float64).sum(1)
    assert np.all(np.abs(sums - 1.0) < 2e-3), sums
    # tap j of phase p sits at j - half - p/up, tap 2*half + 1 - j of phase up - p at the negated offset
    for p in range(1, min(up, 8)):
        np.testing.assert_allclose(table[p, 1:], table[up - p, :0:-1], rtol=0, atol=1e-7)


@pytest.mark.parametrize("rate", [8000, 44100, 48000])
def test_resampled_signals(rate):
    n = rate // 2
    ones = np.ones(n, np.float32)
    y = O.resample(ones, rate)
    inner = y[200:-200]
    assert len(y) == n * 16000 // rate and np.abs(inner - 1.0).max() < 2e-3
    t = np.arange(n) / rate
    x = np.sin(2 * np.pi * 440.0 * t).astype(np.float32)
    ys = O.resample(x, rate)[200:-200]
    ts = (np.arange(len(O.resample(x, rate))) / 16000.0)[200:-200]
    np.testing.assert_allclose(ys, np.sin(2 * np.pi * 440.0 * ts), atol=5e-3)
    assert np.array_equal(O.resample(x, 16000), x)
