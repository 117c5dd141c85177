"""Multi-GPU host logic on the CPU: the deterministic least-loaded request split every rank computes, and the
host-side result gather to rank 0, with world_size-2 gloo process groups (no GPU, no collective on a data path)."""
import multiprocessing as mp
import os
import socket

import numpy as np

from conftest import load_package


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_assign_is_balanced_and_whole():
    load_package()
    from fast_d1_omni_b200.engine import assign, request_cost, request_tokens
    from fast_d1_omni_b200.weights import mixed_requests
    reqs = mixed_requests(4, 40)
    for world in (1, 2, 3, 8):
        a = assign(reqs, world)
        assert len(a) == len(reqs) and set(a) <= set(range(world))
        assert a == assign(reqs, world)  # every rank computes the same split
        loads = [sum(request_cost(r) for r, d in zip(reqs, a) if d == i) for i in range(world)]
        biggest = max(request_cost(r) for r in reqs)
        assert max(loads) - min(loads) <= biggest  # greedy least-loaded: within one request of balance


def test_request_cost_weights_media():
    """Media requests cost their encoder work on top of their trunk positions; text requests cost their tokens."""
    load_package()
    from fast_d1_omni_b200.engine import FRAME_COST, PATCH_COST, request_cost, request_tokens
    from fast_d1_omni_b200.weights import mixed_requests
    for r in mixed_requests(4, 40):
        m = r["media"]
        extra = request_cost(r) - request_tokens(r)
        if m is None:
            assert extra == 0
        elif m["kind"] == "images":
            assert np.isclose(extra, PATCH_COST * sum(ph * pw for ph, pw, _ in m["crops"]))
        else:
            assert np.isclose(extra, FRAME_COST * (max(min(len(m["pcm"]), 480000), 8000) // 160))


def _fake_result(req):
    """Stand-in for an engine result: one value per option marker, derived from the request's tokens."""
    return (np.concatenate([np.full(len(r["markers"]), float(r["ids"].sum() % 9973), np.float32) for r in req["rows"]]),
            "")


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        load_package()
        from fast_d1_omni_b200.engine import assign, gather_results
        from fast_d1_omni_b200.weights import mixed_requests
        reqs = mixed_requests(5, 16)
        mine = [i for i, d in enumerate(assign(reqs, world)) if d == rank]
        local = {i: _fake_result(reqs[i]) for i in mine}
        res = gather_results(local, world, rank, len(reqs))
        if rank == 0:
            want = [_fake_result(r) for r in reqs]
            q.put(all(np.array_equal(a[0], b[0]) for a, b in zip(res, want)) and len(res) == len(reqs))
        else:
            q.put(res is None)
    finally:
        dist.destroy_process_group()


def test_gather_world2_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert [q.get(timeout=5) for _ in range(2)] == [True, True]
