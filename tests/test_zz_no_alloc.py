"""The allocation-free GEMM entry point (d1_gemm_noalloc: its scratch is a static device buffer). This file is
collected last, so the test also runs after every other test has used the device."""
import ctypes as C

import numpy as np
import pytest

from conftest import half_ulp_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def P(t):
    return C.c_void_p(t.data_ptr())


def ST():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _case(rng, M, N, K):
    x = rng.standard_normal((M, K)).astype(np.float16)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    return x, w, x.astype(np.float64) @ w.astype(np.float64).T


def test_noalloc_gemm_two_calls(gpu_lib):
    rng = np.random.default_rng(77)
    cases = [(96, 1024, 2048, 8), (333, 1000, 1024, 4)]  # head-sized rows; ragged M and N
    outs = []
    for i, (M, N, K, split) in enumerate(cases):
        x, w, ref = _case(rng, M, N, K)
        xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        assert gpu_lib.d1_gemm_noalloc(M, N, K, P(xd), K, P(wd), K, P(y), N, split, ST()) == 0
        torch.cuda.synchronize()
        assert gpu_lib.d1_gemm_noalloc_error() == 0  # every bounded wait of the GEMM completed
        if i > 0:  # the second call in a row leaves the device's free memory untouched
            assert torch.cuda.mem_get_info()[0] == free0
        got = y.cpu().numpy().astype(np.float64)
        assert np.isfinite(got).all()
        # one fp16 rounding of the fp32 sum, plus fp32 accumulation noise near zero
        assert half_ulp_close(got, ref, 2.0 ** -10, 2e-4).all()
        outs.append(got)
    # the first shape again: the buffer was cleared, the result is the same GEMM
    M, N, K, split = cases[0]
    rng = np.random.default_rng(77)
    x, w, ref = _case(rng, M, N, K)
    y = torch.empty((M, N), dtype=torch.float16, device="cuda")
    assert gpu_lib.d1_gemm_noalloc(M, N, K, P(torch.from_numpy(x).cuda()), K, P(torch.from_numpy(w).cuda()), K, P(y),
                                   N, split, ST()) == 0
    assert gpu_lib.d1_gemm_noalloc_error() == 0
    assert half_ulp_close(y.cpu().numpy().astype(np.float64), outs[0], 2.0 ** -10, 2e-4).all()


def test_noalloc_gemm_rejects_oversize(gpu_lib):
    x = torch.zeros(1025, 1024, dtype=torch.float16, device="cuda")
    y = torch.zeros(1025, 1024, dtype=torch.float16, device="cuda")
    assert gpu_lib.d1_gemm_noalloc(1025, 1024, 1024, P(x), 1024, P(x), 1024, P(y), 1024, 2, ST()) == -1  # M*N > 2^20
    assert gpu_lib.d1_gemm_noalloc(8, 1022, 1024, P(x), 1024, P(x), 1024, P(y), 1024, 2, ST()) == -1     # N % 4
    assert gpu_lib.d1_gemm_noalloc(8, 1024, 1024, None, 1024, P(x), 1024, P(y), 1024, 2, ST()) == -1      # null X
    assert gpu_lib.d1_gemm_noalloc(8, 1024, 1024, P(x), 1024, None, 1024, P(y), 1024, 2, ST()) == -1      # null W
    assert gpu_lib.d1_gemm_noalloc_error() == 0
