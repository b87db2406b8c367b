"""Expert-parallel dispatch / combine host logic on CPU ranks (gloo, world size 2).

The expert math here is the CPU restatement (oracle/moe.py) row by row, so the
checks are about routing rows to their owners and back: the 2-rank output must
equal the 1-rank output bit for bit and match the unsharded moe_layer combine
(src/deepseeker/mlx_forward.py:388-419).  A peer that leaves between steps
must turn the next exchange into an error on the other rank, not a hang.
"""
from __future__ import annotations

import multiprocessing as mp
import socket

import pytest
import torch

from tests import ep_worker


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def spawn(world: int, mode: str, timeout: float = 120.0) -> dict:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=ep_worker.rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, v = q.get(timeout=timeout)
            res[r] = v
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return res


def test_dispatch_plan_blocks():
    from deepseeker.ep import ExpertParallelMoE

    ep = ExpertParallelMoE(8, 3, lambda *a: None, fixed_capacity=True)
    ep.world, ep.local_experts = 2, 4
    ids = torch.tensor([[0, 5, 3], [7, -1, 1]])
    dest, index, valid = ep.dispatch_plan(ids)
    assert dest.tolist() == [0, 1, 0, 1, 0, 0]
    assert valid.tolist() == [True, True, True, True, False, True]
    assert index[valid].tolist() == [0, 0, 1, 1, 2]


def test_single_rank_matches_unsharded_combine():
    from oracle import moe as omoe

    ep, x, ids, w = ep_worker.cpu_ep(1, 0)
    out = ep(x, ids, w)
    w1, w3, w2, sh, *_ = ep_worker.cpu_problem()
    ref = omoe.moe_combine(x, ids.long(), w, lambda e: (w1[e], w3[e], w2[e]), shared=sh, limit=ep_worker.LIMIT)
    assert out.dtype == torch.bfloat16
    diff = (out.float() - ref.float()).abs().max()
    assert float(diff) <= 2 ** -7 * float(ref.float().abs().max()), float(diff)


def test_two_ranks_equal_one_rank_bitwise():
    ep1, x, ids, w = ep_worker.cpu_ep(1, 0)
    single = ep1(x, ids, w)
    res = spawn(2, "cpu")
    for r in (0, 1):
        assert isinstance(res[r], torch.Tensor), res[r]
        assert torch.equal(res[r], single), f"rank {r} differs"


def test_two_ranks_fixed_capacity_equal_one_rank_bitwise():
    """The fixed-capacity exchange (no host read, graph-capturable) gives the
    same bits as the counted one."""
    ep1, x, ids, w = ep_worker.cpu_ep(1, 0)
    single = ep1(x, ids, w)
    ep1f = ep_worker.cpu_ep(1, 0, fixed_capacity=True)[0]
    assert torch.equal(ep1f(x, ids, w), single)
    res = spawn(2, "cpu_fixed")
    for r in (0, 1):
        assert isinstance(res[r], torch.Tensor), res[r]
        assert torch.equal(res[r], single), f"rank {r} differs"


def test_peer_that_left_fails_the_exchange_not_hangs():
    res = spawn(2, "cpu_dead_peer", timeout=90.0)
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith(("error", "exception")), res[0]


def test_decode_scheme_two_ranks_match_one_rank():
    """All-gather / local partial / reduce-scatter scheme (ExpertParallelDecode)."""
    ep1, x, ids, w = ep_worker.cpu_ep_decode(1, 0)
    single = ep1(x, ids, w)
    res = spawn(2, "cpu_decode")
    for r in (0, 1):
        assert isinstance(res[r], torch.Tensor), res[r]
        # f32 partial sums are added in another order; the bf16 results agree to the last place or two
        diff = (res[r].float() - single.float()).abs().max()
        assert float(diff) <= 2 ** -7 * float(single.float().abs().max()), float(diff)
    from oracle import moe as omoe
    w1, w3, w2, sh, *_ = ep_worker.cpu_problem()
    ref = omoe.moe_combine(x, ids.long(), w, lambda e: (w1[e], w3[e], w2[e]), shared=sh, limit=ep_worker.LIMIT)
    assert float((single.float() - ref.float()).abs().max()) <= 2 ** -7 * float(ref.float().abs().max())
