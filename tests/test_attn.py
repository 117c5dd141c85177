"""Flash attention parity through the C ABI (d1_flash_attn) against the oracle and the reference's own kernel.

packed varlen bidirectional attention, 16 query heads, 8 KV heads, head dim 64, Q/K/V N(0,1)
fp16 (seed 2), lengths log-normal (median 384, sigma 1.0) clipped to [32, 16384]. Plus the decision-head forms
(MHA with q/k/v bias, marker-row queries) and the media-prefix form (external keys before the local ones).
Tolerance: |O - O_ref| <= 4e-3 (fp16 output of a convex combination of N(0,1) values; fp16 P as the reference)."""
import ctypes as C

import numpy as np
import pytest

from oracle import d1_oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def P(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def attn_meta(pkg, seqs, ext=None, step=64):
    """seqs: [(q_start, q_len, kv_start, kv_len)]; ext: per seq None or (k tensor, v tensor) [ext_len, ext_ld];
    step: rows per work item (64: every tile, as the reference builds the list; 256: the tcgen05 kernel's blocks)."""
    arr = (pkg.abi.AttnSeq * len(seqs))()
    for i, (qs, ql, ks, kl) in enumerate(seqs):
        arr[i].q_start, arr[i].q_len, arr[i].kv_start, arr[i].kv_len = qs, ql, ks, kl
        if ext is not None and ext[i] is not None:
            arr[i].ext_len = ext[i][0].shape[0]
            arr[i].ext_k, arr[i].ext_v = ext[i][0].data_ptr(), ext[i][1].data_ptr()
    meta = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).cuda()
    work = []
    for i, (qs, ql, ks, kl) in enumerate(seqs):
        work += [(i, q) for q in range(0, ql, step)]
    w = torch.tensor(np.asarray(work, np.int32).reshape(-1), device="cuda")
    return meta, w, len(work)


def run(lib, pkg, Q, ldq, K, V, ldkv, seqs, heads, group, bias=None, ext=None, ext_ld=0, q_rows=None, tc=False,
        step=64):
    meta, work, n_work = attn_meta(pkg, seqs, ext, step)
    rows = q_rows if q_rows is not None else Q.shape[0]
    O_ = torch.zeros(rows, heads * 64, dtype=torch.float16, device="cuda")
    bq, bk, bv = bias if bias is not None else (None, None, None)
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if tc:  # the tcgen05 form (extension), bias-free only
        assert bias is None
        r = lib.d1_flash_attn_tc(P(Q), ldq, P(K), P(V), ldkv, ext_ld, P(O_), heads * 64, P(meta), P(work), n_work,
                                 heads, group, 0.125, Q.shape[0], K.shape[0], st)
    else:
        r = lib.d1_flash_attn(P(Q), ldq, P(K), P(V), ldkv, ext_ld, P(bq), P(bk), P(bv), P(O_), heads * 64, P(meta),
                              P(work), n_work, heads, group, 0.125, st)
    assert r == 0
    torch.cuda.synchronize()
    if hasattr(lib, "d1_flash_attn_error"):
        assert lib.d1_flash_attn_error() == 0
    return O_.float().cpu().numpy()


def lognormal(total, seed=2):
    from fast_d1_omni_b200.weights import lognormal_lengths
    return lognormal_lengths(seed, total)


@pytest.mark.parametrize("total", [2048, 8192, 16384])
def test_config2_gqa(pkg, gpu_lib, ref_lib, total):
    lens = lognormal(total)
    g = torch.Generator(device="cuda").manual_seed(2)
    qkv = torch.randn(total, 2048, device="cuda", generator=g).half()
    spans, s = [], 0
    for n in lens:
        spans.append((s, n, s, n))
        s += n
    Q, K, V = qkv, qkv[:, 1024:], qkv[:, 1536:]
    got = run(gpu_lib, pkg, Q, 2048, K, V, 2048, spans, 16, 2)
    got_tc = run(gpu_lib, pkg, Q, 2048, K, V, 2048, spans, 16, 2, tc=True)
    ref_k = run(ref_lib, pkg, Q, 2048, K, V, 2048, spans, 16, 2)
    q = qkv.float().cpu().numpy()
    want = O.attention(q[:, :1024], q[:, 1024:1536], q[:, 1536:], spans, 16, 2, 0.125)
    assert np.abs(got - want).max() <= 4e-3
    assert np.abs(got_tc - want).max() <= 4e-3
    assert np.abs(ref_k - want).max() <= 4e-3
    assert np.abs(got - ref_k).max() <= 4e-3


@pytest.mark.parametrize("lens", [[1], [63, 64, 65], [1, 2, 3, 130, 7]])
def test_edge_lengths_mha_bias(pkg, gpu_lib, ref_lib, lens):
    """Decision-head / SigLIP2 form: MHA (group 1) with fp32 q/k/v biases added on load, ld = 3D."""
    rng = np.random.default_rng(len(lens))
    T = sum(lens)
    qkv = rng.standard_normal((T, 3072)).astype(np.float16)
    b = (rng.standard_normal(3072) * 0.5).astype(np.float32)
    spans, s = [], 0
    for n in lens:
        spans.append((s, n, s, n))
        s += n
    d = torch.from_numpy(qkv).cuda()
    bd = torch.from_numpy(b).cuda()
    bias = (bd[:1024], bd[1024:2048], bd[2048:])
    got = run(gpu_lib, pkg, d, 3072, d[:, 1024:], d[:, 2048:], 3072, spans, 16, 1, bias)
    ref_k = run(ref_lib, pkg, d, 3072, d[:, 1024:], d[:, 2048:], 3072, spans, 16, 1, bias)
    q = qkv.astype(np.float32)
    want = O.attention(q[:, :1024], q[:, 1024:2048], q[:, 2048:], spans, 16, 1, 0.125, b[:1024], b[1024:2048], b[2048:])
    assert np.abs(got - want).max() <= 4e-3
    assert np.abs(got - ref_k).max() <= 4e-3


@pytest.mark.parametrize("step", [64, 256])
@pytest.mark.parametrize("group", [1, 2])
@pytest.mark.parametrize("lens", [[1], [63, 64, 65], [127, 128, 129, 255, 256, 257], [300, 1, 513, 2]])
def test_tc_edge_lengths(pkg, gpu_lib, lens, group, step):
    """d1_flash_attn_tc on ragged lengths around its 128-row tiles and 256-row units (units whose second tile is
    empty, single-tile units, partial key tiles), MHA and GQA, with the reference's 64-row work list and the
    256-row one, against the oracle and the mma.sync kernel."""
    rng = np.random.default_rng(sum(lens) + group)
    T = sum(lens)
    ld = 1024 + 2 * 1024 // group
    qkv = rng.standard_normal((T, ld)).astype(np.float16)
    spans, s = [], 0
    for n in lens:
        spans.append((s, n, s, n))
        s += n
    d = torch.from_numpy(qkv).cuda()
    kvw = 1024 // group
    K, V = d[:, 1024:], d[:, 1024 + kvw:]
    got_tc = run(gpu_lib, pkg, d, ld, K, V, ld, spans, 16, group, tc=True, step=step)
    got = run(gpu_lib, pkg, d, ld, K, V, ld, spans, 16, group)
    q = qkv.astype(np.float32)
    want = O.attention(q[:, :1024], q[:, 1024:1024 + kvw], q[:, 1024 + kvw:], spans, 16, group, 0.125)
    assert np.abs(got_tc - want).max() <= 4e-3
    assert np.abs(got_tc - got).max() <= 4e-3


def test_tc_marker_queries(pkg, gpu_lib):
    """d1_flash_attn_tc with fewer query rows than keys (gathered marker rows, the last head layer's form)."""
    rng = np.random.default_rng(12)
    lens, marks = [700, 40, 300], [list(range(0, 700, 3)), [0, 39], [1, 2, 150, 299]]
    T = sum(lens)
    qkv = rng.standard_normal((T, 3072)).astype(np.float16)
    rows, seqs, s, ms = [], [], 0, 0
    for n, mk in zip(lens, marks):
        rows += [s + m for m in mk]
        seqs.append((ms, len(mk), s, n))
        s += n
        ms += len(mk)
    mq = qkv[rows]
    d = torch.from_numpy(qkv).cuda()
    dq = torch.from_numpy(np.ascontiguousarray(mq)).cuda()
    got = run(gpu_lib, pkg, dq, 3072, d[:, 1024:], d[:, 2048:], 3072, seqs, 16, 1, tc=True)
    q = qkv.astype(np.float32)
    want = O.attention(mq.astype(np.float32)[:, :1024], q[:, 1024:2048], q[:, 2048:], seqs, 16, 1, 0.125)
    assert np.abs(got - want).max() <= 4e-3


def test_marker_queries(pkg, gpu_lib, ref_lib):
    """Last head layer: queries are gathered marker rows (q_start indexes the gathered buffer), keys cover every
    row of the sequence (src/model.rs:534-539)."""
    rng = np.random.default_rng(11)
    lens, marks = [100, 40, 300], [[3, 50, 99], [0, 39], [1, 2, 150, 299]]
    T = sum(lens)
    qkv = rng.standard_normal((T, 3072)).astype(np.float16)
    rows, seqs, s, ms = [], [], 0, 0
    for n, mk in zip(lens, marks):
        rows += [s + m for m in mk]
        seqs.append((ms, len(mk), s, n))
        s += n
        ms += len(mk)
    mq = qkv[rows]
    d = torch.from_numpy(qkv).cuda()
    dq = torch.from_numpy(np.ascontiguousarray(mq)).cuda()
    got = run(gpu_lib, pkg, dq, 3072, d[:, 1024:], d[:, 2048:], 3072, seqs, 16, 1)
    ref_k = run(ref_lib, pkg, dq, 3072, d[:, 1024:], d[:, 2048:], 3072, seqs, 16, 1)
    q = qkv.astype(np.float32)
    want = O.attention(mq.astype(np.float32)[:, :1024], q[:, 1024:2048], q[:, 2048:], seqs, 16, 1, 0.125)
    assert np.abs(got - want).max() <= 4e-3
    assert np.abs(got - ref_k).max() <= 4e-3


@pytest.mark.parametrize("lens", [[70, 5], [300, 200]])
def test_prefix_keys(pkg, gpu_lib, ref_lib, lens):
    """Text after a media prefix: the prefix's cached K/V ([ext_len][512]) come before the local keys. The longer
    case gives the tcgen05 kernel every kind of key tile: prefix only, prefix + local, whole local tiles (TMA) and a
    partial last tile."""
    rng = np.random.default_rng(12 + lens[0])
    ext_lens = [129, 64]
    T = sum(lens)
    qkv = rng.standard_normal((T, 2048)).astype(np.float16)
    ext_np = [(rng.standard_normal((e, 512)).astype(np.float16), rng.standard_normal((e, 512)).astype(np.float16))
              for e in ext_lens]
    ext = [(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()) for k, v in ext_np]
    spans, s = [], 0
    for n in lens:
        spans.append((s, n, s, n))
        s += n
    d = torch.from_numpy(qkv).cuda()
    got = run(gpu_lib, pkg, d, 2048, d[:, 1024:], d[:, 1536:], 2048, spans, 16, 2, ext=ext, ext_ld=512)
    got_tc = run(gpu_lib, pkg, d, 2048, d[:, 1024:], d[:, 1536:], 2048, spans, 16, 2, ext=ext, ext_ld=512, tc=True)
    ref_k = run(ref_lib, pkg, d, 2048, d[:, 1024:], d[:, 1536:], 2048, spans, 16, 2, ext=ext, ext_ld=512)
    q = qkv.astype(np.float32)
    want = O.attention(q[:, :1024], q[:, 1024:1536], q[:, 1536:], spans, 16, 2, 0.125,
                       ext=[(k.astype(np.float32), v.astype(np.float32)) for k, v in ext_np])
    assert np.abs(got - want).max() <= 4e-3
    assert np.abs(got_tc - want).max() <= 4e-3
    assert np.abs(got - ref_k).max() <= 4e-3


@pytest.mark.parametrize("case", ["shuffled", "holes", "mixed"])
def test_abi_any_work_list(pkg, gpu_lib, case):
    """d1_flash_attn takes any list of (seq, first row) items, each covering 64 query rows (cuda/kernels.cu:351-500):
    the bias-free call runs the tcgen05 kernel on the 256-row blocks listed whole and in order, and the mma.sync
    kernel on every other item. Rows named by the list match the oracle; rows it does not name are left as they
    were."""
    rng = np.random.default_rng({"shuffled": 21, "holes": 22, "mixed": 23}[case])
    lens = [300, 513, 70, 256]
    T = sum(lens)
    qkv = rng.standard_normal((T, 2048)).astype(np.float16)
    spans, s = [], 0
    for n in lens:
        spans.append((s, n, s, n))
        s += n
    canon = [(i, q) for i, n in enumerate(lens) for q in range(0, n, 64)]
    if case == "shuffled":
        work = [canon[i] for i in rng.permutation(len(canon))]
    elif case == "holes":
        work = [it for k, it in enumerate(canon) if k % 3 != 1]
    else:  # whole blocks, a block missing a tile, duplicates, out-of-order items, rows not on a 64-row boundary
        work = [(0, 0), (0, 64), (0, 128), (0, 192), (0, 256), (1, 0), (1, 64), (1, 192), (1, 256), (1, 320),
                (1, 384), (1, 448), (1, 512), (1, 256), (2, 30), (3, 192), (3, 128), (3, 64), (3, 0), (3, 0), (3, 64),
                (3, 128), (3, 192)]
    arr = (pkg.abi.AttnSeq * len(spans))()
    for i, (qs, ql, ks, kl) in enumerate(spans):
        arr[i].q_start, arr[i].q_len, arr[i].kv_start, arr[i].kv_len = qs, ql, ks, kl
    meta = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).cuda()
    wk = torch.tensor(np.asarray(work, np.int32).reshape(-1), device="cuda")
    d = torch.from_numpy(qkv).cuda()
    out = torch.full((T, 1024), 7.0, dtype=torch.float16, device="cuda")
    st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert gpu_lib.d1_flash_attn(P(d), 2048, P(d[:, 1024:]), P(d[:, 1536:]), 2048, 0, None, None, None, P(out), 1024,
                                 P(meta), P(wk), len(work), 16, 2, 0.125, st) == 0
    torch.cuda.synchronize()
    assert gpu_lib.d1_flash_attn_error() == 0
    got = out.float().cpu().numpy()
    covered = np.zeros(T, bool)
    for i, q0 in work:
        qs, ql = spans[i][0], spans[i][1]
        covered[qs + q0: qs + min(q0 + 64, ql)] = True
    q = qkv.astype(np.float32)
    want = O.attention(q[:, :1024], q[:, 1024:1536], q[:, 1536:], spans, 16, 2, 0.125)
    assert np.abs(got[covered] - want[covered]).max() <= 4e-3
    assert np.all(got[~covered] == 7.0)
