#!/usr/bin/env python3
"""Benchmark of the B200 routed-expert MoE hot path (BASELINE.json metric).

Default workload (N=1): BASELINE config 2 -- one MoE layer, decode B=1:
hidden 4096, 256 routed experts (inter 2048, FP4 e2m1 + ue8m0/32), top-8
softmax-renormalised gates from router logits ~ N(0,1), one bf16 shared
expert (inter 2048), bf16 activations, all experts resident.

One step = router (softmax top-8 over the step's logits) + the fused decode
layer for one token, one routed-decode call (on the tcgen05 kernels the
first kernel routes).  Steps rotate over L distinct resident layer instances
(8 x 3.47 GB) with fresh logits each step, so every step streams its 157 MB
cold from HBM (the working set per step exceeds the 126 MB L2 and the next
step touches different memory).

Printed JSON line (rank 0): value = tokens/s over the device-timed region
(inputs resident); e2e = tokens/s through the public API with the step's x and
logits copied from pinned host memory and the output copied back each step;
roofline = algorithmic bytes of the decode launch pair / its CUDA-event
duration vs MEASURED_PEAKS.json hbm_gbs; cpu_baseline = the reference CPU
path (oracle port) on this host's cores for a bounded sample.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2|c3|c4]

--config c4 measures BASELINE config 4 instead: one batched grouped FFN over
2048 tokens (256 FP4 experts, top-8 Zipf(1.1) routing) per step; value is
TFLOP/s of algorithmic FFN FLOPs, roofline is HBM GB/s of the weights
streamed, and a second "tensor" object gives the MMA-side fraction.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent


def init_nccl(dev, seconds: int):
    """torch.distributed over NCCL for this rank's device, communicator built
    eagerly; NCCL's start-up banner is written to stdout by the library, so
    fd 1 points at stderr meanwhile (stdout carries the one JSON line)."""
    import datetime

    import torch.distributed as dist

    sys.stdout.flush()
    saved = os.dup(1)
    try:
        os.dup2(2, 1)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=seconds), device_id=dev)
        dist.barrier()
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)
    return dist
sys.path.insert(0, str(ROOT / "deepseeker-v4.1_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/s + achieved HBM GB/s (B=1) and grouped-GEMM TFLOPS at 1/2/4/8 B200"
H, I, E, K_TOP, IS = 4096, 2048, 256, 8, 2048


def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def ncu_traffic(kernel_key: str):
    p = ROOT / "profiles" / "ncu_traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(kernel_key)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"ds_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        rows = []
        if self.path.exists():
            for line in self.path.read_text().splitlines():
                f = [c.strip() for c in line.split(",")]
                if len(f) >= 10:
                    rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None
        loaded = [r for r in rows if (num(r[4]) or 0) >= 50] or rows
        sm = [num(r[1]) for r in loaded if num(r[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i in range(4) if r[6 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(rows[0][2]),
                "reasons": reasons, "samples": len(loaded)}


# ------------------------------------------------------------------ reference CPU path

def reference_step_factory(seed: int, fmt: str = "fp4"):
    """The reference's CPU path for one decode token of config 2, restated in
    oracle/ (numpy dequant_fp4_rowmajor + torch f32 matmuls + sorted combine +
    shared expert), on random FP4 bytes of the real shapes (timing only)."""
    import numpy as np
    import torch
    from concurrent.futures import ThreadPoolExecutor

    from oracle import fp4 as ofp4
    from oracle import moe as omoe

    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(seed)
    pool = 16  # distinct random experts; routing ids map onto them

    def mat(n, k):
        return (rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8),
                rng.integers(118, 128, size=(n, k // 32), dtype=np.uint8))
    experts = [(mat(I, H), mat(I, H), mat(H, I)) for _ in range(pool)]
    shared = tuple((torch.randn(*s, generator=torch.Generator().manual_seed(seed + i)) * 0.02).to(torch.bfloat16)
                   for i, s in enumerate(((IS, H), (IS, H), (H, IS))))
    ex = ThreadPoolExecutor(max_workers=os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)

    def step():
        x = torch.randn(1, H, generator=g).to(torch.bfloat16)
        logits = torch.randn(1, E, generator=g)
        w, ids = omoe.route_softmax_topk(logits, K_TOP)
        chosen = sorted({int(e) for e in ids.flatten()})
        jobs = {(e, r): ex.submit(ofp4.dequant_matrix, *experts[e % pool][r]) for e in chosen for r in range(3)}
        dense = {e: tuple(torch.from_numpy(jobs[(e, r)].result()) for r in range(3)) for e in chosen}
        return omoe.moe_combine(x, ids, w, lambda e: dense[e], shared=shared, limit=10.0)
    return step, ex


C4_TOKENS = 2048


def workload(config: str, tokens: int = 1) -> str:
    """config.workload of a bench line; the reference arm prints the same text."""
    if config == "c4":
        return (f"BASELINE config 4: batched grouped expert FFN, {tokens} tokens, hidden 4096, "
                "256 FP4 experts inter 2048, top-8 Zipf(1.1), bf16 out")
    fmt = "FP4" if config == "c2" else "q3"
    return (f"BASELINE config {'2' if config == 'c2' else '3'}: one MoE layer decode B={tokens}, hidden 4096, "
            f"256 {fmt} experts inter 2048 top-8 softmax, bf16 shared expert")


def grouped_flops(pairs: int) -> float:
    """Algorithmic FLOPs of the routed SwiGLU FFN over `pairs` (token, expert) pairs."""
    return 2.0 * pairs * 3 * H * I


def time_reference_grouped(budget_s: float) -> tuple[float, int, str]:
    """TFLOP/s of the reference CPU path on config 4 (numpy FP4 dequant +
    torch f32 expert matmuls, the restatement in oracle/), measured on a
    sample of experts and extrapolated to the 256-expert batch: per-expert
    dequant time x experts touched + per-pair matmul time x pairs."""
    import numpy as np
    import torch

    from deepseeker import synthetic
    from oracle import fp4 as ofp4
    from oracle import moe as omoe

    torch.set_num_threads(os.cpu_count() or 1)
    rng = np.random.default_rng(4)
    ids, w = synthetic.zipf_routing(C4_TOKENS, E, K_TOP, seed=4, device="cpu")
    x = torch.randn(C4_TOKENS, H, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).float()
    counts = torch.bincount(ids.flatten().long(), minlength=E)
    touched = int((counts > 0).sum())
    order = torch.argsort(counts, descending=True).tolist()
    t_deq = t_mm = 0.0
    n_exp = n_pairs = 0
    t_start = time.perf_counter()
    for e in order[::max(1, E // 16)]:   # a spread of heavy and light experts
        mats = [(rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8),
                 rng.integers(118, 128, size=(n, k // 32), dtype=np.uint8)) for n, k in ((I, H), (I, H), (H, I))]
        t0 = time.perf_counter()
        w1, w3, w2 = (torch.from_numpy(ofp4.dequant_matrix(*m)) for m in mats)
        t1 = time.perf_counter()
        rows, slots = torch.nonzero(ids == e, as_tuple=True)
        h = omoe.swiglu_hidden(x[rows], w1, w3, 10.0) * w[rows, slots][:, None]
        _ = h @ w2.T
        t2 = time.perf_counter()
        t_deq += t1 - t0
        t_mm += t2 - t1
        n_exp += 1
        n_pairs += int(rows.numel())
        if time.perf_counter() - t_start > budget_s:
            break
    total = touched * (t_deq / n_exp) + C4_TOKENS * K_TOP * (t_mm / max(n_pairs, 1))
    value = grouped_flops(C4_TOKENS * K_TOP) / total / 1e12
    return value, os.cpu_count() or 1, (f"{n_exp} of {touched} touched experts of config 4 ({n_pairs} pairs) timed, "
                                       f"extrapolated to 16384 pairs; f32 CPU")


def time_reference(steps: int, warmup: int, budget_s: float | None = None) -> tuple[float, int, str]:
    """tokens/s of the reference CPU path; returns (value, cores, sample description)."""
    step, ex = reference_step_factory(seed=1234)
    for _ in range(max(0, warmup)):
        step()
    n = 0
    t0 = time.perf_counter()
    while n < steps:
        step()
        n += 1
        if budget_s is not None and time.perf_counter() - t0 > budget_s and n >= 1:
            break
    dt = time.perf_counter() - t0
    ex.shutdown(wait=False)
    cores = os.cpu_count() or 1
    return n / dt, cores, f"{n} decode tokens of config 2 (8 FP4 experts dequantised + shared bf16 expert), f32 CPU"


# ------------------------------------------------------------------ our arm

def run_ours(args) -> dict:
    if args.config == "c4":
        return run_grouped(args)
    if args.config == "c5":
        return run_stack(args)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        return run_ep(args)
    return run_decode(args)


def run_ep(args) -> dict:
    """N > 1: config 2's layer expert-parallel over the N ranks (rank g owns
    experts [g*E/N, (g+1)*E/N) of every rotated layer, shared expert
    replicated); every rank decodes its own --batch tokens per step (weak
    scaling).  Ranks x tokens <= 8 (FP4): ds_ep_decode, token rows and partial
    sums exchanged over NVLink peer memory by the library's kernels, one CUDA
    graph per layer; otherwise NCCL all_to_all_single dispatch + combine."""
    import datetime

    import torch
    import torch.distributed as dist

    from deepseeker import ep, moe, synthetic

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    init_nccl(dev, 120)
    fmt = "q3" if args.config == "c3" else "fp4"
    El = E // world
    L = args.layers
    b = args.batch
    layers = [synthetic.make_layer(fmt, H, I, El, seed=1000 + l, shared_inter=IS, std=0.02, device=dev,
                                   expert_offset=rank * El) for l in range(L)]
    # decode-sized batches: token rows exchanged over NVLink peer memory by the
    # library's own kernels (no collective call; one CUDA graph per layer);
    # larger batches: NCCL all-to-all dispatch + combine
    small = fmt == "fp4" and world * b <= 8
    comm = None
    graphs = None
    if small:
        comm = ep.PeerComm(b, H, K_TOP, timeout_ms=30000)
        eps = [ep.PeerDecodeLayer(comm, layer, E, K_TOP, rows=b) for layer in layers]
        if os.environ.get("DEEPSEEKER_BENCH_NO_GRAPH") != "1":
            stage_x = torch.zeros(L, b, H, dtype=torch.bfloat16, device=dev)
            stage_l = torch.zeros(L, b, E, dtype=torch.float32, device=dev)
            graphs = [ep.PeerDecodeGraph(pl, x=stage_x[l], logits=stage_l[l], host_io=True)
                      for l, pl in enumerate(eps)]
    else:
        eps = [ep.gpu_layer(layer, E, K_TOP) for layer in layers]
    # graph mode: the L layers back to back in one CUDA graph (no collective
    # inside: the exchange is the library's own kernels)
    chain = moe.GraphChain(graphs, x=stage_x, logits=stage_l) \
        if graphs is not None and os.environ.get("DEEPSEEKER_BENCH_NO_CHAIN") != "1" else None
    total_steps = args.warmup + args.steps
    n_in = (total_steps + 64 + L - 1) // L * L
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    logits = torch.randn(n_in, b, E, generator=g, device=dev)
    xs = torch.randn(n_in, b, H, generator=g, device=dev).to(torch.bfloat16)
    stream = torch.cuda.current_stream(dev)

    def step(i, ev=None):
        i %= n_in
        if graphs is not None:
            gr = graphs[i % L]
            gr.x.copy_(xs[i])
            gr.logits.copy_(logits[i])
            if ev is not None:
                ev[0].record(stream)
            out = gr.replay()
        else:
            w, ids = moe.route_softmax_topk(logits[i], K_TOP)
            if ev is not None:
                ev[0].record(stream)
            out = eps[i % L](xs[i], ids, w)
        if ev is not None:
            ev[1].record(stream)
        return out

    def run_steps(i0, n, timed=None):
        """Steps i0 .. i0+n-1 (every rank the same); `timed` collects (start, end, layers)."""
        i = i0
        while i < i0 + n:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) \
                if timed is not None else None
            j = i % n_in
            if chain is not None and j % L == 0 and i + L <= i0 + n:
                chain.x.copy_(xs[j:j + L])
                chain.logits.copy_(logits[j:j + L])
                if ev is not None:
                    ev[0].record(stream)
                chain.replay()
                if ev is not None:
                    ev[1].record(stream)
                    timed.append((ev[0], ev[1], L))
                i += L
            else:
                step(i, ev)
                if ev is not None:
                    timed.append((ev[0], ev[1], 1))
                i += 1

    def agreed_steps(ms_per_step: float, target_ms: float) -> int:
        """A step count (multiple of L) worth ~target_ms, the same on every rank."""
        n = int(target_ms / max(ms_per_step, 1e-3)) // L * L
        t = torch.tensor([min(max(n, L), 40000)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return int(t.item())

    with ClockSampler(local) as clk:
        w_steps = max(args.warmup, 3)
        w_steps = (w_steps + L - 1) // L * L
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        run_steps(0, w_steps)
        c1.record(stream)
        torch.cuda.synchronize(dev)
        if not args.quick:
            # more warm-up, ~1 s, so that clocks settle and get sampled
            extra = agreed_steps(c0.elapsed_time(c1) / w_steps, 1000.0)
            run_steps(w_steps, extra)
            w_steps += extra
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)
        timed = []
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")
        start.record(stream)
        run_steps(w_steps, args.steps, timed)
        end.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)
        ms = start.elapsed_time(end)
        layer_ms = sum(a.elapsed_time(c) for a, c, _ in timed) / sum(n for _, _, n in timed)
        if not args.quick:
            # keep the GPUs busy a little longer so the sampler sees the load
            run_steps(0, agreed_steps(ms / args.steps, 500.0))
            torch.cuda.synchronize(dev)
    clocks = clk.summary()

    # e2e: the step's x and logits from pinned host memory, output back to the host
    e2e_steps = 0 if args.quick else min(args.steps, 50)
    pin_x = xs[:max(e2e_steps, 1)].cpu().pin_memory()
    pin_l = logits[:max(e2e_steps, 1)].cpu().pin_memory()
    pin_o = torch.empty(b, H, dtype=torch.bfloat16).pin_memory()
    dx = torch.empty(b, H, dtype=torch.bfloat16, device=dev)
    dl = torch.empty(b, E, dtype=torch.float32, device=dev)
    # numpy views of the pinned buffers (bf16 as int16): a step's input lands
    # in the graph's staging buffers by a plain memory copy
    np_x, np_l, np_o = pin_x.view(torch.int16).numpy(), pin_l.numpy(), pin_o.view(torch.int16).numpy()
    np_io = [(g_.x_host.view(torch.int16).numpy(), g_.logits_host.numpy(), g_.out_host.view(torch.int16).numpy())
             for g_ in graphs] if graphs is not None else None

    def e2e_step(s_):
        if graphs is not None:
            # host in -> one graph launch (staging, router, exchange, decode) -> host out
            gr = graphs[s_ % L]
            xv, lv, ov = np_io[s_ % L]
            np.copyto(xv, np_x[s_])
            np.copyto(lv, np_l[s_])
            gr.replay_host()
            np.copyto(np_o, ov)
            return
        else:
            dx.copy_(pin_x[s_], non_blocking=True)
            dl.copy_(pin_l[s_], non_blocking=True)
            w, ids = moe.route_softmax_topk(dl, K_TOP)
            out = eps[s_ % L](dx, ids, w)
        pin_o.copy_(out, non_blocking=True)
        stream.synchronize()
    for s_ in range(min(3, e2e_steps)):
        e2e_step(s_)
    dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s_ in range(e2e_steps):
        e2e_step(s_)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max(e0.elapsed_time(e1), 1e-9)

    per_expert = sum(bk.nbytes() // El for bk in (layers[0].w1, layers[0].w3, layers[0].w2))
    # bytes one rank streams per step: the distinct experts of this rank that
    # the step's routing of ALL ranks touches (counted from the timed steps'
    # routing, gathered after the timing) + the shared expert for its tokens
    timed_ids = torch.stack([moe.route_softmax_topk(logits[(w_steps + s_) % n_in], K_TOP)[1]
                             for s_ in range(args.steps)])                    # [steps, b, k]
    all_ids = torch.empty((world,) + tuple(timed_ids.shape), dtype=timed_ids.dtype, device=dev)
    dist.all_gather_into_tensor(all_ids, timed_ids.contiguous())
    all_ids = all_ids.permute(1, 0, 2, 3).reshape(args.steps, -1).cpu()
    mine = [len({int(e) for e in row.tolist() if rank * El <= e < (rank + 1) * El}) for row in all_ids]
    distinct = statistics.mean(mine) if mine else float(b * K_TOP)
    # shared expert: split over the ranks when its inter divides into world slices of 256
    shared_b = 3 * IS * H * 2 // world if (small and IS % (256 * world) == 0) else 3 * IS * H * 2 * ((b + 7) // 8)
    step_bytes = distinct * per_expert + shared_b + 2 * b * H * 2
    ms_t = torch.tensor([ms, e2e_ms, layer_ms], device=dev)
    dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, layer_ms = (float(v) for v in ms_t.cpu())
    result = None
    if rank == 0:
        pk, kind = peaks()
        gbs = step_bytes / (layer_ms * 1e-3) / 1e9
        result = {
            "metric": METRIC,
            "value": round(world * b * args.steps / (ms * 1e-3), 2),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": f"{fmt} weights, bf16 activations, f32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights quantised on device; router logits N(0,1))",
            "config": {"workload": f"BASELINE config {'2' if fmt == 'fp4' else '3'} layer, expert-parallel over "
                                   f"{world} GPUs ({El} experts each; shared expert split over the ranks by "
                                   f"intermediate slices), {b} decode "
                                   "token(s) per GPU per step",
                       "format": fmt, "tokens_per_step_per_gpu": b, "layers_rotated": L,
                       "l2": f"rotating {L} resident layer shards per GPU",
                       "parallelism": (f"ep{world} (token rows and partial sums exchanged over NVLink peer "
                                       "memory by the library's kernels; the rotated layers back to back in one CUDA graph)"
                                       if small else f"ep{world} (NCCL all_to_all_single dispatch + combine)"),
                       "distinct_local_experts_per_step": round(distinct, 3)},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / pk["hbm_gbs"], 4), "traffic": None,
                         "kernel": "ep layer step (dispatch + local experts + combine), per GPU",
                         "bytes_per_launch": int(step_bytes), "peak_kind": kind},
            "e2e": {"value": round(world * b * max(e2e_steps, 1) / (e2e_ms * 1e-3), 2) if e2e_steps else None,
                    "unit": "tokens/s", "h2d_bytes_per_step": b * (H * 2 + E * 4), "d2h_bytes_per_step": b * H * 2},
            "gpu_launches": args.steps * ((1 + 1 + 5 + 1) if small else (1 + 5 + 2 * ((b + 7) // 8))),
            "clocks": clocks,
        }
    del chain, graphs, eps
    torch.cuda.synchronize(dev)
    dist.barrier()
    if comm is not None:
        if comm.status() != 0:
            raise RuntimeError(f"rank {rank}: peer exchange reported error {comm.status()}")
        comm.close()
    dist.barrier()
    dist.destroy_process_group()
    return result


def run_stack(args) -> dict:
    """a decode step through a 40-layer stack (layers 0-19
    FP4, 20-39 q3, each a config-2 layer), --batch tokens per GPU per step,
    each layer's output feeding the next.  N = 1: all 256 experts of every
    layer on the GPU (131 GB resident), the whole step one CUDA graph (batch
    <= 8: the decode kernels; above: the grouped kernels for the routed
    experts and bf16 GEMMs for the shared expert).
    N > 1: rank g holds experts [g E/N, (g+1) E/N) of every layer; with
    N * batch <= 8 the layers exchange through ds_ep_decode (NVLink peer
    memory, one CUDA graph per step), otherwise through NCCL all-to-all."""
    import datetime

    import torch

    from deepseeker import ep, grouped, moe, synthetic

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import torch.distributed as dist
        init_nccl(dev, 300)
    NL = args.stack_layers
    b = args.batch
    El = E // world
    fmts = ["fp4" if l < NL // 2 else "q3" for l in range(NL)]
    layers = []
    for l in range(NL):
        layer = synthetic.make_layer(fmts[l], H, I, El, seed=1000 * l + 1, shared_inter=IS, std=0.02, device=dev,
                                     expert_offset=rank * El)
        layers.append(layer.prepare_tc())
    torch.cuda.synchronize(dev)
    peer = world > 1 and world * b <= 8
    if world > 1 and not peer:
        eps = [ep.gpu_layer(layer, E, K_TOP) for layer in layers]
    n_in = 64                                     # distinct step inputs, cycled
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    x_pool = torch.randn(n_in, b, H, generator=g, device=dev).to(torch.bfloat16)
    l_pool = torch.randn(n_in, NL, b, E, generator=g, device=dev)
    stage_x = torch.zeros(b, H, dtype=torch.bfloat16, device=dev)
    stage_l = torch.zeros(NL, b, E, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    graph = None
    comm = None
    if world == 1 and b > 8:
        # one graph: for every layer, routing + the grouped FFN over the
        # routed experts (each used expert's weights once per step) + the
        # shared expert as bf16 GEMMs, ping-pong activation buffers
        ffns = [grouped.GroupedFFN(layer, K_TOP) for layer in layers]
        bufs = [torch.zeros(b, H, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        wbuf = torch.empty(b, K_TOP, dtype=torch.float32, device=dev)
        ibuf = torch.empty(b, K_TOP, dtype=torch.int32, device=dev)
        rout = torch.empty(b, H, dtype=torch.float32, device=dev)

        def body():
            cur = stage_x
            for l, layer in enumerate(layers):
                nxt = bufs[l % 2]
                moe.route_softmax_topk(stage_l[l], K_TOP, out=(wbuf, ibuf))
                ffns[l](cur, ibuf, wbuf, out=rout, route_before_down=True)
                rout.add_(ep.shared_dense(layer.shared_w1, layer.shared_w3, layer.shared_w2, cur))
                nxt.copy_(rout)
                cur = nxt
            return cur
        out_buf = body()                          # eager once: workspaces, attributes
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with moe.graph_capture(graph):
            out_buf = body()
    elif world == 1:
        # one graph: for every layer, routing + the decode kernels over
        # chunks of 8 tokens (up to 8 tokens: one routed-decode call, whose
        # tcgen05 prep kernel routes), ping-pong activation buffers
        bufs = [torch.zeros(b, H, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        wbuf = torch.empty(b, K_TOP, dtype=torch.float32, device=dev)
        ibuf = torch.empty(b, K_TOP, dtype=torch.int32, device=dev)
        ws_bytes = max(max(layer.decode_workspace_bytes(min(8, b), K_TOP) for layer in layers[::NL // 2]), 1 << 20)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)

        def body():
            cur = stage_x
            for l, layer in enumerate(layers):
                nxt = bufs[l % 2]
                if b <= 8:
                    moe.moe_decode_routed(cur, layer, stage_l[l], K_TOP, out=nxt, route_out=(wbuf, ibuf),
                                          workspace=ws)
                    cur = nxt
                    continue
                moe.route_softmax_topk(stage_l[l], K_TOP, out=(wbuf, ibuf))
                for r0 in range(0, b, 8):
                    r1 = min(b, r0 + 8)
                    moe.moe_decode(cur[r0:r1], layer, ibuf[r0:r1], wbuf[r0:r1], out=nxt[r0:r1], workspace=ws)
                cur = nxt
            return cur
        out_buf = body()                          # eager once: attributes, caches
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with moe.graph_capture(graph):
            out_buf = body()
    elif peer:
        comm = ep.PeerComm(b, H, K_TOP, timeout_ms=30000)
        pgs = []
        for l, layer in enumerate(layers):
            pl = ep.PeerDecodeLayer(comm, layer, E, K_TOP, rows=b)
            pgs.append(ep.PeerDecodeGraph(pl, x=stage_x if l == 0 else pgs[-1].out, logits=stage_l[l]))
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with moe.graph_capture(graph):
            for pg in pgs:
                pg._step()
        out_buf = pgs[-1].out

    def step(i):
        j = i % n_in
        stage_x.copy_(x_pool[j])
        stage_l.copy_(l_pool[j])
        if graph is not None:
            graph.replay()
            return out_buf
        cur = stage_x
        for l in range(NL):
            w, ids = moe.route_softmax_topk(stage_l[l], K_TOP)
            cur = eps[l](cur, ids, w)
        return cur

    def agreed(n: int) -> int:
        if dist is None:
            return n
        t = torch.tensor([n], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return int(t.item())

    with ClockSampler(local) as clk:
        for i in range(max(args.warmup, 3)):
            step(i)
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")
        start.record(stream)
        for s_ in range(args.steps):
            step(args.warmup + s_)
        end.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ms = start.elapsed_time(end)
        if not args.quick:
            extra = agreed(int(500.0 / max(ms / args.steps, 1e-3)))
            for i in range(min(extra, 2000)):
                step(i)
            torch.cuda.synchronize(dev)
    clocks = clk.summary()

    # e2e: the step's x and logits from pinned host memory, output back
    e2e_steps = 0 if args.quick else min(args.steps, 20)
    pin_x = x_pool[:max(e2e_steps, 1)].cpu().pin_memory()
    pin_l = l_pool[:max(e2e_steps, 1)].cpu().pin_memory()
    pin_o = torch.empty(b, H, dtype=torch.bfloat16).pin_memory()

    def e2e_step(s_):
        stage_x.copy_(pin_x[s_], non_blocking=True)
        stage_l.copy_(pin_l[s_], non_blocking=True)
        if graph is not None:
            graph.replay()
            o = out_buf
        else:
            cur = stage_x
            for l in range(NL):
                w, ids = moe.route_softmax_topk(stage_l[l], K_TOP)
                cur = eps[l](cur, ids, w)
            o = cur
        pin_o.copy_(o, non_blocking=True)
        stream.synchronize()
    for s_ in range(min(2, e2e_steps)):
        e2e_step(s_)
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s_ in range(e2e_steps):
        e2e_step(s_)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max(e0.elapsed_time(e1), 1e-9)

    # bytes one GPU streams per step: per layer, its distinct local experts of
    # the step's routing (all ranks' tokens) + the shared expert (split over
    # the ranks on the peer path) + activations
    per_exp = {f: sum(bk.nbytes() // El for bk in (layers[i].w1, layers[i].w3, layers[i].w2))
               for f, i in (("fp4", 0), ("q3", NL - 1))}
    steps_idx = [(args.warmup + s_) % n_in for s_ in range(args.steps)]
    ids_all = torch.stack([torch.stack([moe.route_softmax_topk(l_pool[j][l], K_TOP)[1] for l in range(NL)])
                           for j in steps_idx])                               # [steps, NL, b, k]
    if dist is not None:
        gathered = torch.empty((world,) + tuple(ids_all.shape), dtype=ids_all.dtype, device=dev)
        dist.all_gather_into_tensor(gathered, ids_all.contiguous())
        ids_all = gathered.permute(1, 2, 0, 3, 4).reshape(args.steps, NL, -1)
    ids_all = ids_all.reshape(args.steps, NL, -1).cpu()
    # the shared expert streams once per step (decode kernels up to 8 rows, one
    # set of GEMMs above), split over the ranks on the peer path
    shared_b = 3 * IS * H * 2 // world if (peer and IS % (256 * world) == 0) else 3 * IS * H * 2
    tot = 0.0
    for st_ in range(args.steps):
        for l in range(NL):
            mine = {int(e) for e in ids_all[st_, l].tolist() if rank * El <= e < (rank + 1) * El}
            tot += len(mine) * per_exp[fmts[l]] + shared_b + 2 * b * H * 2
    step_bytes = tot / args.steps
    ms_t = torch.tensor([ms, e2e_ms], device=dev)
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = (float(v) for v in ms_t.cpu())
    result = None
    if rank == 0:
        pk, kind = peaks()
        gbs = step_bytes / (ms / args.steps * 1e-3) / 1e9
        result = {
            "metric": METRIC,
            "value": round(world * b * args.steps / (ms * 1e-3), 2),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp4-e2m1 (layers 0-19) and q3-affine (20-39) weights, bf16 activations, f32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights quantised on device, seed 1000*layer+1; router logits "
                    "N(0,1) per layer and step)",
            "config": {"workload": f"BASELINE config 5: {NL}-layer MoE stack decode, {b} token(s) per GPU per step, "
                                   "hidden 4096, 256 experts inter 2048 top-8 softmax, bf16 shared expert per layer",
                       "layers": NL, "tokens_per_step_per_gpu": b,
                       "resident_gb_per_gpu": round(sum(sum(bk.nbytes() for bk in (ly.w1, ly.w3, ly.w2)) +
                                                        3 * IS * H * 2 for ly in layers) / 1e9, 1),
                       "l2": "each step streams every layer's experts once (the stack is far above L2)",
                       "parallelism": ((f"single GPU, the step in one CUDA graph ("
                                        + ("grouped routed FFN + bf16 GEMM shared expert" if b > 8 else
                                           "decode kernels") + ")") if world == 1 else
                                       f"ep{world} over NVLink peer memory (ds_ep_decode), the step in one CUDA graph"
                                       if peer else f"ep{world} over NCCL all_to_all_single")},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / pk["hbm_gbs"], 4), "traffic": None,
                         "kernel": "whole stack step per GPU (40 layers: router + decode kernels)",
                         "bytes_per_launch": int(step_bytes), "peak_kind": kind},
            "e2e": {"value": round(world * b * max(e2e_steps, 1) / (e2e_ms * 1e-3), 2) if e2e_steps else None,
                    "unit": "tokens/s", "h2d_bytes_per_step": b * (H * 2 + NL * E * 4),
                    "d2h_bytes_per_step": b * H * 2},
            # ours per layer: router + prep/gemm/h/gemm/combine (FP4, tcgen05;
            # on one GPU the prep kernel routes: no router launch) or
            # gate_up/down/combine (q3), + 2 exchange kernels (peer); above 8
            # tokens on one GPU: router + align/xquant/gemm/gemm/combine
            "gpu_launches": args.steps * sum(
                (5 if (f == "fp4" and not peer) else
                 1 + (5 if f == "fp4" else 3) + (2 if peer else 0)) if b <= 8 else 1 + 5
                for f in fmts) if (world == 1 or peer) else None,
            "clocks": clocks,
        }
    graph = None
    torch.cuda.synchronize(dev)
    if comm is not None:
        if dist is not None:
            dist.barrier()
        comm.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_grouped(args) -> dict:
    """one batched grouped FFN over 2048 tokens, FP4 experts."""
    import torch

    from deepseeker import grouped, synthetic

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        init_nccl(dev, 120)
    T = args.tokens or C4_TOKENS
    fp4act = bool(getattr(args, "fp4_activations", False))
    layer = synthetic.make_layer("fp4", H, I, E, seed=1000 * (rank + 1), shared_inter=None, std=0.02, device=dev)
    ffn = grouped.GroupedFFN(layer, K_TOP, activations="fp4" if fp4act else "exact")
    R = 4  # distinct routings / inputs rotated
    routes = [synthetic.zipf_routing(T, E, K_TOP, s=1.1, seed=100 * rank + r, device=dev) for r in range(R)]
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)
    xs = [torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16) for _ in range(R)]
    outs = [torch.empty(T, H, dtype=torch.bfloat16, device=dev) for _ in range(R)]
    stream = torch.cuda.current_stream(dev)

    def step(i, ev=None):
        ids, w = routes[i % R]
        if ev is not None:
            ev[0].record(stream)
        ffn(xs[i % R], ids, w, out=outs[i % R], route_before_down=True)
        if ev is not None:
            ev[1].record(stream)

    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        i = 0
        while i < args.warmup or time.perf_counter() - t0 < (0.0 if args.quick else 1.0):
            step(i)
            i += 1
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)
        pairs_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    for _ in range(args.steps)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")
        start.record(stream)
        for s_ in range(args.steps):
            step(s_, pairs_ev[s_])
        end.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ms = start.elapsed_time(end)
        step_ms = statistics.mean(a.elapsed_time(b) for a, b in pairs_ev)
        t1 = time.perf_counter()
        j = 0
        while time.perf_counter() - t1 < (0.0 if args.quick else 0.6):
            step(j)
            j += 1
        torch.cuda.synchronize(dev)
    clocks = clk.summary()

    # e2e: x and routing from pinned host memory, output back to host, every step synchronised
    e2e_steps = 0 if args.quick else min(args.steps, 20)
    pin_x = [x.cpu().pin_memory() for x in xs]
    pin_i = [r[0].cpu().pin_memory() for r in routes]
    pin_w = [r[1].cpu().pin_memory() for r in routes]
    pin_o = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    dx = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    di = torch.empty(T, K_TOP, dtype=torch.int32, device=dev)
    dw = torch.empty(T, K_TOP, dtype=torch.float32, device=dev)
    do = torch.empty(T, H, dtype=torch.bfloat16, device=dev)

    def e2e_step(s_):
        dx.copy_(pin_x[s_ % R], non_blocking=True)
        di.copy_(pin_i[s_ % R], non_blocking=True)
        dw.copy_(pin_w[s_ % R], non_blocking=True)
        ffn(dx, di, dw, out=do, route_before_down=True)
        pin_o.copy_(do, non_blocking=True)
        stream.synchronize()
    for s_ in range(min(3, e2e_steps)):
        e2e_step(s_)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s_ in range(e2e_steps):
        e2e_step(s_)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max(e0.elapsed_time(e1), 1e-9)

    per_expert = sum(b.nbytes() // E for b in (layer.w1, layer.w3, layer.w2))
    touched = statistics.mean(int(torch.unique(r[0]).numel()) for r in routes)
    step_bytes = touched * per_expert + 2 * T * H * 2
    flops = grouped_flops(T * K_TOP)
    ms_t = torch.tensor([ms, e2e_ms, step_ms], device=dev)
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, step_ms = (float(v) for v in ms_t.cpu())
    result = None
    if rank == 0:
        pk, kind = peaks()
        tflops = world * flops * args.steps / (ms * 1e-3) / 1e12
        per_step_ms = ms / args.steps          # the value's timed region
        gbs = step_bytes / (per_step_ms * 1e-3) / 1e9
        result = {
            "metric": METRIC,
            "value": round(tflops, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": ("fp4-e2m1 weights x fp4-e2m1 activations (x and h rounded to FP4, per-32 scales), "
                      "f32 accumulate" if fp4act else
                      "fp4-e2m1 weights x e4m3 activation pieces (bf16-exact x, ~14-bit h), f32 accumulate"),
            "data": "synthetic (seeded N(0,0.02) weights quantised on device; Zipf(1.1) top-8 routing)",
            "config": {"workload": workload("c4", T) + (" (FP4 throughput mode: activations rounded to FP4)"
                                                         if fp4act else ""),
                       "tokens_per_step": T, "pairs_per_step": T * K_TOP, "experts_touched": touched,
                       "l2": f"each step streams {step_bytes / 1e9:.2f} GB of expert weights (> 126 MB L2)",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "tokens_per_s": round(world * T * args.steps / (ms * 1e-3), 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / pk["hbm_gbs"], 4), "traffic": ncu_traffic("grouped_fp4_c4") if T == C4_TOKENS else None,
                         "timing": "the value's timed region: K steps / total device time",
                         "launch_frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
                         "kernel": ("ds_grouped_ffn_fp4: align + fp4x_quant + fp4_gemm<gate/up> + fp4_gemm<down> + combine"
                                    if fp4act else
                                    "ds_grouped_ffn: align + xquant + gemm<gate/up> + gemm<down> + combine"),
                         "bytes_per_launch": int(step_bytes), "peak_kind": kind},
            "tensor": ({"achieved_tflops": round(flops / (per_step_ms * 1e-3) / 1e12, 1),
                        "peak_tflops": 9000.0, "peak_kind": "nominal dense FP4 (kind::mxf4) rate; no measured FP4 peak",
                        "frac": round(flops / (per_step_ms * 1e-3) / 1e12 / 9000.0, 4),
                        "note": "one MMA per weight byte; parity against an FP4-rounding emulation, not the exact layer"}
                       if fp4act else
                       {"achieved_tflops": round(flops / (per_step_ms * 1e-3) / 1e12, 1),
                        "peak_tflops": 4500.0, "peak_kind": "nominal dense mxf8f6f4 rate",
                        "frac": round(flops / (per_step_ms * 1e-3) / 1e12 / 4500.0, 4),
                        "note": "activation pieces make the MMA do 2x (gate/up) and 3x (down) the algorithmic FLOPs"}),
            "e2e": {"value": round(world * flops * max(e2e_steps, 1) / (e2e_ms * 1e-3) / 1e12, 2) if e2e_steps else None,
                    "unit": "TFLOP/s", "h2d_bytes_per_step": T * H * 2 + T * K_TOP * 8,
                    "d2h_bytes_per_step": T * H * 2},
            "gpu_launches": 5 * args.steps,
            "clocks": clocks,
        }
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_decode(args) -> dict:
    import torch

    from deepseeker import moe, synthetic

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        init_nccl(dev, 120)

    fmt = "q3" if args.config == "c3" else "fp4"
    tokens = args.batch
    if not 1 <= tokens <= 8:
        raise SystemExit("--batch must be 1..8 for the decode configs")
    L = args.layers
    layers = [synthetic.make_layer(fmt, H, I, E, seed=1000 * (rank + 1) + l, shared_inter=IS, std=0.02,
                                   device=dev) for l in range(L)]
    use_t5 = fmt == "fp4"
    if use_t5:
        for layer in layers:
            layer.prepare_tc()   # scale atoms: ds_moe_decode then runs its tcgen05 kernels
    total_steps = args.warmup + args.steps
    n_in = (total_steps + 64 + L - 1) // L * L          # input slots, a whole number of layer rotations
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    logits = torch.randn(n_in, tokens, E, generator=g, device=dev)
    xs = torch.randn(n_in, tokens, H, generator=g, device=dev).to(torch.bfloat16)
    outs = torch.empty(L, tokens, H, dtype=torch.bfloat16, device=dev)
    ws = moe._workspace(dev, moe.decode_workspace_bytes(layers[0], tokens, K_TOP))
    stream = torch.cuda.current_stream(dev)

    # routing (device) + decode for step i on layer i % L.  Graph mode: the L
    # layers' steps are captured back to back into one CUDA graph
    # (moe.GraphChain over one moe.DecodeGraph per layer), so L consecutive
    # steps are one launch whose inputs are staged by two copies; steps that
    # do not fill a whole rotation replay their layer's own graph.
    use_graph = os.environ.get("DEEPSEEKER_BENCH_NO_GRAPH") != "1"
    stage_x = torch.zeros(L, tokens, H, dtype=torch.bfloat16, device=dev)
    stage_l = torch.zeros(L, tokens, E, dtype=torch.float32, device=dev)
    graphs = [moe.DecodeGraph(layer, tokens, K_TOP, dev, x=stage_x[l], logits=stage_l[l], host_io=True)
              for l, layer in enumerate(layers)] if use_graph else None
    chain = moe.GraphChain(graphs, x=stage_x, logits=stage_l) \
        if use_graph and os.environ.get("DEEPSEEKER_BENCH_NO_CHAIN") != "1" else None

    def step(i, ev=None):
        i %= n_in
        if use_graph:
            gr = graphs[i % L]
            gr.x.copy_(xs[i])
            gr.logits.copy_(logits[i])
            if ev is not None:
                ev[0].record(stream)
            gr.replay()
        else:
            w, ids = moe.route_softmax_topk(logits[i], K_TOP)
            if ev is not None:
                ev[0].record(stream)
            moe.moe_decode(xs[i], layers[i % L], ids, w, out=outs[i % L], workspace=ws)
        if ev is not None:
            ev[1].record(stream)

    def run_steps(i0, n, timed=None):
        """Steps i0 .. i0+n-1; `timed` collects (start, end, layers) events."""
        i = i0
        while i < i0 + n:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) \
                if timed is not None else None
            j = i % n_in
            if chain is not None and j % L == 0 and i + L <= i0 + n:
                chain.x.copy_(xs[j:j + L])
                chain.logits.copy_(logits[j:j + L])
                if ev is not None:
                    ev[0].record(stream)
                chain.replay()
                if ev is not None:
                    ev[1].record(stream)
                    timed.append((ev[0], ev[1], L))
                i += L
            else:
                step(i, ev)
                if ev is not None:
                    timed.append((ev[0], ev[1], 1))
                i += 1

    min_warm_s = 0.0 if args.quick else 1.0
    with ClockSampler(local) as clk:
        # warm-up: at least W steps and at least ~1 s so clocks settle and get sampled
        t0 = time.perf_counter()
        i = 0
        while i < args.warmup or time.perf_counter() - t0 < min_warm_s:
            run_steps(i, L)
            i += L
            if i % 256 < L:
                torch.cuda.synchronize(dev)
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)
        # ---- timed region: K steps, inputs resident (NVTX range "timed" for profilers)
        timed = []
        i_start = (args.warmup + L - 1) // L * L
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed")
        start.record(stream)
        run_steps(i_start, args.steps, timed)
        end.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ms = start.elapsed_time(end)
        decode_ms = [a.elapsed_time(b) / n for a, b, n in timed for _ in range(n)]
        # keep the GPU busy a little longer so the sampler sees the load
        t1 = time.perf_counter()
        j = 0
        while time.perf_counter() - t1 < (0.0 if args.quick else 0.6):
            run_steps(j, L)
            j += L
            if j % 256 < L:
                torch.cuda.synchronize(dev)
        torch.cuda.synchronize(dev)
    clocks = clk.summary()

    # ---- e2e: public API with host buffers, every step synchronised
    e2e_steps = 0 if args.quick else args.steps
    pin_x = torch.empty(args.steps, tokens, H, dtype=torch.bfloat16).pin_memory()
    pin_l = torch.empty(args.steps, tokens, E, dtype=torch.float32).pin_memory()
    pin_o = torch.empty(args.steps, tokens, H, dtype=torch.bfloat16).pin_memory()
    pin_x.copy_(xs[:args.steps].cpu())
    pin_l.copy_(logits[:args.steps].cpu())
    dx = torch.empty(tokens, H, dtype=torch.bfloat16, device=dev)
    dl = torch.empty(tokens, E, dtype=torch.float32, device=dev)
    do = torch.empty(tokens, H, dtype=torch.bfloat16, device=dev)

    # numpy views of the pinned buffers (bf16 as int16): a step's input lands
    # in the graph's staging buffers by a plain memory copy
    np_x, np_l, np_o = pin_x.view(torch.int16).numpy(), pin_l.numpy(), pin_o.view(torch.int16).numpy()
    np_io = [(g_.x_host.view(torch.int16).numpy(), g_.logits_host.numpy(), g_.out_host.view(torch.int16).numpy())
             for g_ in graphs] if use_graph else None

    def e2e_step(s):
        if use_graph:
            # host in -> one graph launch (staging kernel, routed decode, staging
            # kernel) -> host out
            gr = graphs[s % L]
            xv, lv, ov = np_io[s % L]
            np.copyto(xv, np_x[s])
            np.copyto(lv, np_l[s])
            gr.replay_host()
            np.copyto(np_o[s], ov)
            return
        else:
            dx.copy_(pin_x[s], non_blocking=True)
            dl.copy_(pin_l[s], non_blocking=True)
            w, ids = moe.route_softmax_topk(dl, K_TOP)
            moe.moe_decode(dx, layers[s % L], ids, w, out=do, workspace=ws)
            pin_o[s].copy_(do, non_blocking=True)
        stream.synchronize()
    for s in range(min(args.warmup, e2e_steps)):
        e2e_step(s)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(e2e_steps):
        e2e_step(s)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max(e0.elapsed_time(e1), 1e-9)

    # per-step algorithmic bytes: distinct experts x expert bytes + shared + x/out/route traffic
    per_expert = sum(b.nbytes() // E for b in (layers[0].w1, layers[0].w3, layers[0].w2))
    shared_b = 3 * IS * H * 2
    # distinct experts of each timed step's routing (8 for B = 1)
    timed_idx = [(i_start + s_) % n_in for s_ in range(args.steps)]
    ids_t = torch.stack([moe.route_softmax_topk(logits[j], K_TOP)[1] for j in timed_idx]).cpu()
    distinct = statistics.mean(len(set(r.flatten().tolist())) for r in ids_t)
    step_bytes = int(round(distinct * per_expert)) + shared_b + tokens * H * 2 * 2

    ms_t = torch.tensor([ms, e2e_ms, statistics.mean(decode_ms)], device=dev)
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, dec_ms = (float(v) for v in ms_t.cpu())
    result = None
    if rank == 0:
        pk, kind = peaks()
        # roofline on the same timed region as `value` (ms over the K steps);
        # the mean per-launch CUDA-event time inside the graph chain is kept
        # apart as launch_achieved / launch_frac
        achieved = step_bytes / (ms / args.steps * 1e-3) / 1e9
        launch_achieved = step_bytes / (dec_ms * 1e-3) / 1e9
        traffic = ncu_traffic(f"decode_{fmt}_{args.config}") if tokens == 1 else None
        result = {
            "metric": METRIC,
            "value": round(world * tokens * args.steps / (ms * 1e-3), 2),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp4-e2m1 weights, bf16 activations, f32 accumulate" if fmt == "fp4"
                     else "q3-affine weights, bf16 activations, f32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights quantised on device; router logits N(0,1))",
            "config": {"workload": workload(args.config, tokens),
                       "format": fmt, "tokens_per_step": tokens, "layers_rotated": L,
                       "distinct_experts_per_step": round(distinct, 3),
                       "l2": f"rotating {L} resident layers (>{L * 3.4:.0f} GB), each step streams its "
                             f"{step_bytes / 1e6:.1f} MB cold",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "gbs_per_gpu": round(achieved, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                         "timing": "the value's timed region: K steps / total device time",
                         "launch_achieved": round(launch_achieved, 1),
                         "launch_frac": round(launch_achieved / pk["hbm_gbs"], 4),
                         "traffic": traffic,
                         "kernel": ("ds_moe_decode_route: t5_prep (routing, slot list, x pieces) + t5_gemm(gate/up)"
                                    " + t5_h + t5_gemm(down) + t5_combine" if fmt == "fp4" else
                                    "route_topk + ds_moe_decode: q3_gate_up + q3_down + q3_combine"),
                         "bytes_per_launch": step_bytes, "peak_kind": kind},
            "e2e": {"value": round(world * tokens * e2e_steps / (e2e_ms * 1e-3), 2) if e2e_steps else None,
                    "unit": "tokens/s",
                    "h2d_bytes_per_step": tokens * (H * 2 + E * 4), "d2h_bytes_per_step": tokens * H * 2},
            # the layer's decode kernels per step (FP4: the prep kernel routes;
            # q3: the router launch first)
            "gpu_launches": (5 if fmt == "fp4" else 1 + 3) * args.steps,
            "clocks": clocks,
        }
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return result


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["c2", "c3", "c4", "c5"], default="c2")
    ap.add_argument("--stack-layers", type=int, default=40, help="config 5: layers in the stack (half FP4, half q3)")
    ap.add_argument("--layers", type=int, default=8, help="distinct resident layers rotated (L2-cold)")
    ap.add_argument("--batch", type=int, default=1, help="decode tokens per GPU per step (N > 1)")
    ap.add_argument("--tokens", type=int, default=0, help="config 4: tokens per step (default 2048)")
    ap.add_argument("--fp4-activations", action="store_true",
                    help="config 4: the FP4 throughput mode (activations rounded to FP4)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-nested", action="store_true",
                    help="config 2 only: skip the nested config 3 / config 4 measurements")
    ap.add_argument("--quick", action="store_true",
                    help="profiling runs: no time-based warm-up, no e2e / CPU-baseline legs")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        if args.config == "c4":
            value, cores, sample = time_reference_grouped(budget_s=20.0)
            line = {"metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s", "n_gpus": args.gpus,
                    "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": round(grouped_flops(C4_TOKENS * K_TOP) / (value * 1e12) * 1e3, 1),
                    "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "impl": "reference",
                    "dtype": "f32 (reference CPU path)", "data": "synthetic",
                    "config": {"workload": workload("c4", C4_TOKENS), "path": "reference CPU path"},
                    "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                                     "sample": sample},
                    "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                            "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
            return 0
        # bounded per-step sample: one decode token of config 2 through the reference CPU path
        value, cores, sample = time_reference(args.steps, args.warmup)
        line = {"metric": METRIC, "value": round(value, 4), "unit": "tokens/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 / value, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "impl": "reference",
                "dtype": "f32 (reference CPU path)", "data": "synthetic",
                "config": {"workload": workload("c2", 1), "path": "reference CPU path"},
                "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": cores, "kind": "port",
                                 "sample": sample},
                "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    result = run_ours(args)
    nested = (args.config == "c2" and not args.quick and not args.no_nested
              and int(os.environ.get("WORLD_SIZE", "1")) == 1)
    if rank == 0 and result is not None and nested:
        # configs 3 and 4 measured in the same process, each under its own
        # clock sampler, with the same timing rules as the headline
        import copy
        import gc

        import torch
        for key, cfg, steps, tokens, fp4act in (("c3", "c3", min(args.steps, 100), 0, False),
                                                ("c4", "c4", min(args.steps, 20), 0, False),
                                                ("c4_fp4", "c4", min(args.steps, 10), 16384, True)):
            gc.collect()
            torch.cuda.empty_cache()
            sub = copy.copy(args)
            sub.config, sub.steps, sub.batch, sub.tokens, sub.fp4_activations = cfg, steps, 1, tokens, fp4act
            r = run_ours(sub)
            result[key] = {k: r[k] for k in ("value", "unit", "ms_per_step", "steps", "warmup", "dtype", "config",
                                             "roofline", "tensor", "e2e", "gpu_launches", "clocks") if k in r}
    if rank == 0 and result is not None:
        if not (args.no_cpu_baseline or args.quick) and int(os.environ.get("WORLD_SIZE", "1")) == 1:
            if args.config == "c4":
                value, cores, sample = time_reference_grouped(budget_s=20.0)
                result["cpu_baseline"] = {"value": round(value, 6), "unit": "TFLOP/s", "cores": cores,
                                          "kind": "port", "sample": sample}
            elif args.config == "c5":
                # one layer of the reference CPU path, timed; a stack step is
                # args.stack_layers such layers in sequence
                value, cores, sample = time_reference(steps=1000, warmup=1, budget_s=15.0)
                result["cpu_baseline"] = {"value": round(value / args.stack_layers, 5), "unit": "tokens/s",
                                          "cores": cores, "kind": "port",
                                          "sample": sample + f"; divided by the {args.stack_layers} layers of a "
                                                             "stack step"}
            else:
                value, cores, sample = time_reference(steps=1000, warmup=1, budget_s=15.0)
                result["cpu_baseline"] = {"value": round(value, 4), "unit": "tokens/s", "cores": cores,
                                          "kind": "port", "sample": sample}
        print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
