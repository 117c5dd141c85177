"""BASELINE config 4 at its real scale: the mixed request stream through the continuous-batching engine, every
request's answer logits against the reference's own F16 engine on the same requests.

The stream is `weights.mixed_requests(4, 48)`: 48 requests (70% text, 20% text+image of config-3 sides, 10%
text+audio of 1-30 s waveforms), 3 questions of 128-2048 tokens each, 4 answer markers per question,
max-batch-tokens 8192 (src/engine.rs:399-485 packs them; media prefixes go through the trunk once and the
questions read the cached prefix).

The reference side runs each request alone, in the order src/engine.rs would:
  - images: the reference's kernels + cuBLASLt through the vision runner (VisionModel over libd1ref.so), then the
    prefix pass and the questions through the text runner over libd1ref.so;
  - audio: the host log-mel front end (the oracle's restatement of src/audio.rs:238-299, which the reference runs
    on the CPU), the encoder call for call through libd1ref.so (tests/ref_engines.py), then prefix + questions;
  - text: the questions through the text runner over libd1ref.so.
The bar is the north star's, per question: centred |dlogit| mean <= 0.01, max <= 0.06, zero top-answer flips.
"""
import numpy as np
import pytest

from conftest import REF_LIB
from oracle import d1_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def stream(pkg):
    from fast_d1_omni_b200.weights import mixed_requests
    return mixed_requests(4, 48)


@pytest.fixture(scope="module")
def ours(pkg, gpu_lib, stream):
    """This library's engine over the whole stream (all three runners on this library's kernels)."""
    from fast_d1_omni_b200.engine import Engine
    from fast_d1_omni_b200.model import AudioModel, TextModel, VisionModel
    from fast_d1_omni_b200.weights import audio_weights, text_weights, vision_weights
    text = TextModel(text_weights(0), cap_tokens=8192)
    vision = VisionModel(vision_weights(3), max_patches=16384)
    audio = AudioModel(audio_weights(4), max_rows=1536)
    eng = Engine(text, vision, audio, max_batch_tokens=8192)
    try:
        res = eng.run(stream)
        st = eng.stats()
    finally:
        eng.close()
        audio.close()
        vision.close()
        text.close()
    return res, st


@pytest.fixture(scope="module")
def reference(pkg, ref_lib, stream):
    """The reference's F16 engine (its kernels and cuBLASLt GEMMs), one request at a time."""
    from fast_d1_omni_b200.model import TextModel, VisionModel
    from fast_d1_omni_b200.weights import audio_weights, text_weights, vision_weights
    from ref_engines import RefAudioEngine
    m = torch.backends.cuda.matmul
    old = (m.allow_tf32, m.allow_fp16_reduced_precision_reduction)
    m.allow_tf32, m.allow_fp16_reduced_precision_reduction = False, False
    text = TextModel(text_weights(0), kernel_lib=str(REF_LIB), fused=False, cap_tokens=8192)
    vision = VisionModel(vision_weights(3), kernel_lib=str(REF_LIB), fused=False, max_patches=16384)
    audio = RefAudioEngine(ref_lib, audio_weights(4))
    out = []
    try:
        for req in stream:
            rows = [dict(r) for r in req["rows"]]
            media = req["media"]
            pc = None
            if media is not None:
                if media["kind"] == "images":
                    emb = vision.encode(media["crops"])
                else:
                    pcm = media["pcm"][:30 * 16000]
                    mel, valid = O.log_mel(pcm)
                    emb = torch.from_numpy(np.ascontiguousarray(audio.encode(mel, valid))).cuda()
                pc = text.prefix_alloc(emb.shape[0])
                text.launch_prefix([(emb, pc)])
                rows = [dict(r, prefix=pc) for r in rows]
            out.append(text(rows))
            if pc is not None:
                text.prefix_free(pc)
        torch.cuda.synchronize()
    finally:
        text.close()
        vision.close()
        m.allow_tf32, m.allow_fp16_reduced_precision_reduction = old
    return out


def test_stream_shape(stream, ours):
    res, st = ours
    kinds = [r["media"]["kind"] if r["media"] else "text" for r in stream]
    assert len(stream) == 48 and {"text", "images", "audio"} <= set(kinds)
    assert all(err == "" for _, err in res)
    assert st["rows"] == 3 * len(stream)
    assert st["media_jobs"] == sum(k != "text" for k in kinds)
    assert st["batches"] >= 11  # ~90K question tokens under the 8192-token budget


def test_stream_vs_reference_engine(stream, ours, reference):
    res, _ = ours
    all_errs = []
    flips = 0
    for req, (got, err), want in zip(stream, res, reference):
        sizes = [len(r["markers"]) for r in req["rows"]]
        assert err == "" and got.shape == want.shape == (sum(sizes),)
        e = O.centred_logit_err(want, got, sizes)
        all_errs.append(e)
        flips += O.top_flips(want, got, sizes)
    errs = np.concatenate(all_errs)
    assert len(errs) == 3 * len(stream)
    assert errs.mean() <= 0.01 and errs.max() <= 0.06, (errs.mean(), errs.max())
    assert flips == 0
