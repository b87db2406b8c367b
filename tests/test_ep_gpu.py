"""Expert-parallel MoE on B200 ranks.

* one GPU: the EP path (exchange degenerates to a copy) against the fused
  decode layer ds_moe_decode, which is checked against the CPU oracle;
* two GPUs (skipped with fewer): NCCL ranks, each holding half of the experts;
  output must equal the one-rank output bit for bit.
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


def test_ep_single_rank_matches_decode(cuda):
    from deepseeker import ep, moe

    layer, x, ids, w, E, K = ep_worker.gpu_problem(0, 1)
    out = ep.gpu_layer(layer, E, K)(x, ids, w)
    ref = moe.moe_decode(x, layer, ids, w)
    assert out.dtype == torch.bfloat16
    assert rel_l2(out, ref) <= 1e-3


@pytest.mark.parametrize("fmt", ["fp4", "q3"])
def test_ep_single_rank_batch_above_8_vs_oracle(fmt, cuda):
    """b = 16 and 64 rows (config 5's batches): routed experts on the grouped
    kernels (FP4 or q3 banks), the shared expert as bf16 GEMMs over the whole
    batch; against the CPU oracle (dequant + moe_combine)."""
    import numpy as np

    from deepseeker import ep, metal_fp4, synthetic
    from oracle import moe as omoe
    from oracle import q3 as oq3

    H, I, E, K, Is = 512, 256, 16, 4, 384
    layer = synthetic.make_layer(fmt, H, I, E, seed=3, shared_inter=Is, std=0.05, device=cuda)
    lay = ep.gpu_layer(layer, E, K)

    def ew(e):
        out = []
        for b in (layer.w1, layer.w3, layer.w2):
            if b.fmt == 0:
                out.append(metal_fp4.dequant(b.data[e], b.scales[e]).view(b.rows, b.cols).cpu())
            else:
                out.append(torch.from_numpy(oq3.dequant(b.data[e].cpu().numpy().view(np.uint32),
                                                        b.scales[e].cpu().numpy(), b.biases[e].cpu().numpy())))
        return tuple(out)
    shared = (layer.shared_w1.cpu(), layer.shared_w3.cpu(), layer.shared_w2.cpu())
    for b in (16, 64):
        g = torch.Generator().manual_seed(b)
        x = torch.randn(b, H, generator=g).to(torch.bfloat16)
        w, ids = omoe.route_softmax_topk(torch.randn(b, E, generator=g), K)
        ids = ids.to(torch.int32)
        out = lay(x.to(cuda), ids.to(cuda), w.float().to(cuda))
        ref = omoe.moe_combine(x, ids.long(), w.float(), ew, shared=shared, limit=10.0)
        assert out.dtype == torch.bfloat16
        assert rel_l2(out, ref) <= 1e-3, (b, rel_l2(out, ref))


def test_ep_decode_scheme_single_rank_matches_decode(cuda):
    from deepseeker import ep, moe

    layer, x, ids, w, E, K = ep_worker.gpu_problem(0, 1)
    out = ep.gpu_decode_layer(layer, E, K)(x[:4], ids[:4], w[:4])
    ref = moe.moe_decode(x[:4], layer, ids[:4], w[:4])
    assert out.dtype == torch.bfloat16
    assert rel_l2(out, ref) <= 1e-3


def spawn_gpu(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=ep_worker.rank_main, args=(r, 2, port, mode, q)) for r in range(2)]
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
    return res


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_decode_scheme_two_ranks(cuda):
    from deepseeker import ep

    layer, x, ids, w, E, K = ep_worker.gpu_problem(0, 1)
    single = ep.gpu_decode_layer(layer, E, K)(x[:4], ids[:4], w[:4]).cpu()
    del layer
    torch.cuda.synchronize()
    res = spawn_gpu("gpu_decode")
    for r in (0, 1):
        assert isinstance(res[r], torch.Tensor), res[r]
        assert rel_l2(res[r], single) <= 1e-3


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_ranks_bitwise_equal_one_rank(cuda):
    from deepseeker import ep

    layer, x, ids, w, E, K = ep_worker.gpu_problem(0, 1)
    single = ep.gpu_layer(layer, E, K)(x, ids, w).cpu()
    del layer
    torch.cuda.synchronize()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=ep_worker.rank_main, args=(r, 2, port, "gpu", q)) for r in range(2)]
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
        assert isinstance(res[r], torch.Tensor), res[r]
        assert torch.equal(res[r], single), f"rank {r}: rel {rel_l2(res[r], single)}"
