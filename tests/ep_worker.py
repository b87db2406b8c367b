"""Rank body for the expert-parallel tests (spawned processes; gloo on CPU or
NCCL on GPUs).  Imported by tests/test_ep_host.py and tests/test_ep_gpu.py."""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT / "deepseeker-v4.1_b200"), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

H, I, E, K, B, LIMIT = 64, 32, 8, 3, 5, 10.0


def cpu_problem(seed: int = 0):
    """Dense f32 experts + shared expert + tokens and routing (with dropped slots)."""
    g = torch.Generator().manual_seed(seed)
    w1 = torch.randn(E, I, H, generator=g) * 0.2
    w3 = torch.randn(E, I, H, generator=g) * 0.2
    w2 = torch.randn(E, H, I, generator=g) * 0.2
    sh = (torch.randn(16, H, generator=g) * 0.2, torch.randn(16, H, generator=g) * 0.2,
          torch.randn(H, 16, generator=g) * 0.2)
    x = torch.randn(B, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(B, E, generator=g)
    w, ids = torch.softmax(logits, -1).topk(K, dim=-1)
    ids = ids.to(torch.int32)
    ids[1, 2] = -1        # a dropped slot
    ids[3, :] = torch.tensor([0, 1, 2], dtype=torch.int32)   # all on rank 0 when G = 2
    return w1, w3, w2, sh, x, ids, (w / w.sum(-1, keepdim=True)).float()


def cpu_ep(world: int, rank: int, seed: int = 0, fixed_capacity: bool = False):
    """ExpertParallelMoE with row-by-row f32 experts (batch-independent results)."""
    from deepseeker.ep import ExpertParallelMoE
    from oracle import moe as omoe

    w1, w3, w2, sh, x, ids, w = cpu_problem(seed)
    El = E // world

    def local_ffn(xr, expert, gate):
        out = torch.zeros(xr.shape[0], H)
        for r in range(xr.shape[0]):
            e = int(expert[r])
            if e < 0:
                continue
            ge = rank * El + e
            h = omoe.swiglu_hidden(xr[r:r + 1].float(), w1[ge], w3[ge], LIMIT) * gate[r]
            out[r] = (h @ w2[ge].T)[0]
        return out

    def shared_fn(xx):
        return omoe.shared_expert(xx.float(), *sh, limit=LIMIT).to(xx.dtype).float()

    return ExpertParallelMoE(E, K, local_ffn, shared_fn, fixed_capacity=fixed_capacity), x, ids, w


def cpu_ep_decode(world: int, rank: int, seed: int = 0):
    """ExpertParallelDecode with the oracle's f32 expert math (row by row)."""
    from deepseeker.ep import ExpertParallelDecode
    from oracle import moe as omoe

    w1, w3, w2, sh, x, ids, w = cpu_problem(seed)
    El = E // world

    def local_partial(xg, il, gg):
        out = torch.zeros(xg.shape[0], H)
        for r in range(xg.shape[0]):
            for c in range(il.shape[1]):
                e = int(il[r, c])
                if e < 0:
                    continue
                ge = rank * El + e
                h = omoe.swiglu_hidden(xg[r:r + 1].float(), w1[ge], w3[ge], LIMIT) * gg[r, c]
                out[r] += (h @ w2[ge].T)[0]
        return out

    def shared_fn(xx):
        return omoe.shared_expert(xx.float(), *sh, limit=LIMIT).to(xx.dtype).float()

    return ExpertParallelDecode(E, K, local_partial, shared_fn), x, ids, w


def rank_main(rank: int, world: int, port: int, mode: str, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        if mode.startswith("cpu"):
            dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
            if mode == "cpu_dead_peer" and rank == 1:
                q.put((rank, "left"))           # leaves between steps: never joins the exchange
                dist.destroy_process_group()
                return
            ep, x, ids, w = (cpu_ep_decode(world, rank) if mode == "cpu_decode" else
                             cpu_ep(world, rank, fixed_capacity=(mode == "cpu_fixed")))
            try:
                out = ep(x, ids, w)
            except RuntimeError as e:
                q.put((rank, f"error: {type(e).__name__}: {str(e)[:300]}"))
                return
            q.put((rank, out))
        elif mode == "gpu_peer":
            run_gpu_peer_rank(rank, world, q)
        else:
            run_gpu_rank(rank, world, q, decode=(mode == "gpu_decode"))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, f"exception: {e!r}"))


def gpu_problem(rank: int, world: int, shared_inter: int = 512, fmt: str = "fp4"):
    from deepseeker import synthetic
    from oracle import moe as omoe

    dev = torch.device("cuda", rank)
    Hg, Ig, Eg, Kg, Bg = 1024, 1024, 16, 4, 6
    El = Eg // world
    layer = synthetic.make_layer(fmt, Hg, Ig, El, seed=5, shared_inter=shared_inter, device=dev,
                                 expert_offset=rank * El)
    g = torch.Generator().manual_seed(77)
    x = torch.randn(Bg, Hg, generator=g).to(torch.bfloat16).to(dev)
    w, ids = omoe.route_softmax_topk(torch.randn(Bg, Eg, generator=g), Kg)
    return layer, x, ids.to(torch.int32).to(dev), w.float().to(dev), Eg, Kg


def run_gpu_rank(rank: int, world: int, q, decode: bool = False) -> None:
    from deepseeker import ep

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    layer, x, ids, w, Eg, Kg = gpu_problem(rank, world)
    if decode:
        out = ep.gpu_decode_layer(layer, Eg, Kg)(x[:4], ids[:4], w[:4])
    else:
        out = ep.gpu_layer(layer, Eg, Kg)(x, ids, w)
    torch.cuda.synchronize()
    q.put((rank, out.cpu()))


def run_gpu_peer_rank(rank: int, world: int, q) -> None:
    """PeerComm decode of the first 4 tokens on every rank: eager call, then
    the same step replayed from a CUDA graph (routing from the oracle's logits
    inside the graph); returns both outputs."""
    from deepseeker import ep

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    layer, x, ids, w, Eg, Kg = gpu_problem(rank, world)
    comm = ep.PeerComm(4, layer.hidden, Kg, timeout_ms=10000)
    pl = ep.PeerDecodeLayer(comm, layer, Eg, Kg, rows=4)
    eager = pl(x[:4].contiguous(), ids[:4].contiguous(), w[:4].contiguous())
    g = torch.Generator().manual_seed(78)
    logits = torch.randn(4, Eg, generator=g).to(x.device)
    gr = ep.PeerDecodeGraph(pl)
    gr.x.copy_(x[:4])
    gr.logits.copy_(logits)
    out_g = gr.replay().clone()
    torch.cuda.synchronize()
    # shared inter 256 does not split over 2 ranks: each rank evaluates the
    # whole shared expert for its own rows
    layer2 = gpu_problem(rank, world, shared_inter=256)[0]
    pl2 = ep.PeerDecodeLayer(comm, layer2, Eg, Kg, rows=4)
    eager2 = pl2(x[:4].contiguous(), ids[:4].contiguous(), w[:4].contiguous())
    # q3 layer through the same communicator
    layer3 = gpu_problem(rank, world, fmt="q3")[0]
    pl3 = ep.PeerDecodeLayer(comm, layer3, Eg, Kg, rows=4)
    eager3 = pl3(x[:4].contiguous(), ids[:4].contiguous(), w[:4].contiguous())
    torch.cuda.synchronize()
    status = comm.status()
    del gr
    comm.close()
    q.put((rank, (eager.cpu(), out_g.cpu(), logits.cpu(), status, eager2.cpu(), eager3.cpu())))
