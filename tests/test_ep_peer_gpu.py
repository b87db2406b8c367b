"""Expert-parallel decode over NVLink peer memory (ds_ep_*), B200 ranks.

* one GPU, one rank: the exchange kernels degenerate to copies into the
  rank's own region; the output must equal ds_moe_decode's bit for bit, and
  a CUDA-graph replay must equal the eager call;
* one GPU, bounded waits: rank 0 of a two-rank group runs alone, its
  dispatch waits on a flag nothing raises, gives up after the timeout and
  reports it; the context stays usable;
* two GPUs (skipped with fewer): each rank holds half of the experts and
  half of the shared expert's intermediate features (or, when those do not
  split, the whole shared expert for its own rows); outputs within 1e-3
  rel-L2 of the one-rank decode, graph replays likewise.
"""
from __future__ import annotations

import multiprocessing as mp
import socket

import pytest
import torch

from tests import ep_worker

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def test_peer_single_rank_equals_decode(cuda):
    from deepseeker import ep, moe

    layer, x, ids, w, E, K = ep_worker.gpu_problem(0, 1)
    comm = ep.PeerComm(4, layer.hidden, K)
    pl = ep.PeerDecodeLayer(comm, layer, E, K, rows=4)
    x4, i4, w4 = x[:4].contiguous(), ids[:4].contiguous(), w[:4].contiguous()
    out = pl(x4, i4, w4)
    ref = moe.moe_decode(x4, layer, i4, w4)
    torch.cuda.synchronize()
    assert comm.status() == 0
    assert out.dtype == torch.bfloat16
    assert torch.equal(out, ref), rel_l2(out, ref)
    # fewer rows than the communicator holds
    out1 = pl.__class__(comm, layer, E, K, rows=1)(x4[:1].contiguous(), i4[:1].contiguous(), w4[:1].contiguous())
    ref1 = moe.moe_decode(x4[:1].contiguous(), layer, i4[:1].contiguous(), w4[:1].contiguous())
    # one row: ds_moe_decode takes the single-token kernel, the exchange path
    # the tcgen05 kernels, so the two agree within the decode tolerance
    assert rel_l2(out1, ref1) < 1e-3
    comm.close()


def test_peer_single_rank_q3_equals_decode(cuda):
    """q3 banks take the CUDA-core decode kernels inside the exchange."""
    from deepseeker import ep, moe

    layer, x, ids, w, E, K = ep_worker.gpu_problem(0, 1, fmt="q3")
    comm = ep.PeerComm(4, layer.hidden, K)
    x4, i4, w4 = x[:4].contiguous(), ids[:4].contiguous(), w[:4].contiguous()
    out = ep.PeerDecodeLayer(comm, layer, E, K, rows=4)(x4, i4, w4)
    ref = moe.moe_decode(x4, layer, i4, w4)
    torch.cuda.synchronize()
    assert comm.status() == 0
    assert torch.equal(out, ref), rel_l2(out, ref)
    comm.close()


def test_peer_graph_replays_match_eager(cuda):
    from deepseeker import ep, moe

    layer, x, ids, w, E, K = ep_worker.gpu_problem(0, 1)
    comm = ep.PeerComm(2, layer.hidden, K)
    pl = ep.PeerDecodeLayer(comm, layer, E, K, rows=2)
    gr = ep.PeerDecodeGraph(pl)
    g = torch.Generator(device=x.device).manual_seed(3)
    for step in range(3):
        xs = torch.randn(2, layer.hidden, generator=g, device=x.device).to(torch.bfloat16)
        lg = torch.randn(2, E, generator=g, device=x.device)
        gr.x.copy_(xs)
        gr.logits.copy_(lg)
        out_g = gr.replay().clone()
        wr, ir = moe.route_softmax_topk(lg, K)
        ref = moe.moe_decode(xs, layer, ir, wr)
        torch.cuda.synchronize()
        assert torch.equal(out_g, ref), (step, rel_l2(out_g, ref))
    assert comm.status() == 0
    del gr
    # host in / host out through one graph launch
    gh = ep.PeerDecodeGraph(pl, host_io=True)
    xs = torch.randn(2, layer.hidden).to(torch.bfloat16)
    lg = torch.randn(2, E)
    gh.x_host.copy_(xs)
    gh.logits_host.copy_(lg)
    got = gh.replay_host().clone()
    wr, ir = moe.route_softmax_topk(lg.to(x.device), K)
    ref = moe.moe_decode(xs.to(x.device), layer, ir, wr).cpu()
    assert torch.equal(got, ref), rel_l2(got, ref)
    assert comm.status() == 0
    del gh
    comm.close()


def test_peer_wait_times_out_and_reports(cuda):
    from deepseeker import ep, moe

    layer, x, ids, w, E, K = ep_worker.gpu_problem(0, 1)
    half = ep_worker.gpu_problem(0, 2)[0]         # rank 0's shard of a two-rank split
    c0, c1 = ep.PeerComm.local_group([0, 0], 1, layer.hidden, K, timeout_ms=300)
    pl = ep.PeerDecodeLayer(c0, half, E, K, rows=1)
    x1, i1, w1 = x[:1].contiguous(), ids[:1].contiguous(), w[:1].contiguous()
    pl(x1, i1, w1)                                 # rank 1 never runs: rank 0 waits ~300 ms, gives up
    torch.cuda.synchronize()
    assert c0.status() & 2
    pl(x1, i1, w1)                                 # aborted communicator: returns at once
    torch.cuda.synchronize()
    assert c0.status() & 2
    assert c1.status() == 0
    # the context is still usable
    ref = moe.moe_decode(x1, layer, i1, w1)
    torch.cuda.synchronize()
    assert torch.isfinite(ref.float()).all()
    c0.close()
    c1.close()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_two_ranks(cuda):
    from deepseeker import moe

    layer, x, ids, w, E, K = ep_worker.gpu_problem(0, 1)
    layer.prepare_tc()
    x4, i4, w4 = x[:4].contiguous(), ids[:4].contiguous(), w[:4].contiguous()
    single = moe.moe_decode(x4, layer, i4, w4).cpu()
    layer2 = ep_worker.gpu_problem(0, 1, shared_inter=256)[0].prepare_tc()
    single2 = moe.moe_decode(x4, layer2, i4, w4).cpu()
    layer3 = ep_worker.gpu_problem(0, 1, fmt="q3")[0]
    single3 = moe.moe_decode(x4, layer3, i4, w4).cpu()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=ep_worker.rank_main, args=(r, 2, port, "gpu_peer", q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r, v = q.get(timeout=300)
            res[r] = v
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in (0, 1):
        assert isinstance(res[r], tuple), res[r]
        eager, out_g, logits, status, eager2, eager3 = res[r]
        assert rel_l2(eager3, single3) <= 1e-3, rel_l2(eager3, single3)      # q3 banks
        assert status == 0
        assert rel_l2(eager, single) <= 1e-3, rel_l2(eager, single)            # shared expert split 2 ways
        assert rel_l2(eager2, single2) <= 1e-3, rel_l2(eager2, single2)        # shared expert per own rows
        wr, ir = moe.route_softmax_topk(logits.to(x.device), K)
        ref_g = moe.moe_decode(x4, layer, ir, wr).cpu()
        assert rel_l2(out_g, ref_g) <= 1e-3, rel_l2(out_g, ref_g)
    # both ranks hold the same tokens: identical partial sums in the same order
    assert torch.equal(res[0][0], res[1][0])
