"""Seeded synthetic expert banks for the BASELINE configs (no checkpoint is available).

Weights ~ N(0, std) are drawn on the device with a seeded torch generator per
(layer, role, expert) and quantised on the device by the library's builder
quantisers (``ds_fp4_quantize``: e2m1 + ue8m0 per 32; ``ds_q3_quantize``: 3-bit
affine per 64), so a full 256-expert layer is built in well under a second.
"""
from __future__ import annotations

import torch

from . import _abi
from ._dev import ptr, stream_handle
from .moe import ExpertBank, MoEWeights
from .requant import quantize_q3

_CHUNK_ELEMS = 1 << 26  # quantise at most 64M elements (256 MB f32) at a time


def _normal(shape, std: float, seed: int, device) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std


def quantize_fp4(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Device f32 [rows, cols] -> (packed u8 [rows, cols/2], ue8m0 scales u8 [rows, cols/32])."""
    w = w.contiguous()
    rows, cols = w.shape
    packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((rows, cols // 32), dtype=torch.uint8, device=w.device)
    _abi.call("ds_fp4_quantize", ptr(w), rows, cols, ptr(packed), ptr(scales), stream_handle(w.device))
    return packed, scales


def make_bank(fmt: str, n_experts: int, rows: int, cols: int, seed: int, std: float = 0.02,
              device: torch.device | str = "cuda", expert_offset: int = 0) -> ExpertBank:
    """Stacked [E, rows, cols] bank; local expert e is global expert
    `expert_offset + e` and uses seed `seed * 100003 + expert_offset + e`, so an
    expert-parallel shard holds exactly the experts of the unsharded bank."""
    device = torch.device(device)
    per = max(1, _CHUNK_ELEMS // (rows * cols))
    if fmt == "fp4":
        data = torch.empty((n_experts, rows, cols // 2), dtype=torch.uint8, device=device)
        scales = torch.empty((n_experts, rows, cols // 32), dtype=torch.uint8, device=device)
        for e0 in range(0, n_experts, per):
            e1 = min(n_experts, e0 + per)
            w = torch.cat([_normal((rows, cols), std, seed * 100003 + expert_offset + e, device) for e in range(e0, e1)])
            p, s = quantize_fp4(w)
            data[e0:e1] = p.view(e1 - e0, rows, cols // 2)
            scales[e0:e1] = s.view(e1 - e0, rows, cols // 32)
        return ExpertBank.fp4(data, scales)
    if fmt == "q3":
        data = torch.empty((n_experts, rows, cols * 3 // 32), dtype=torch.int32, device=device)
        scales = torch.empty((n_experts, rows, cols // 64), dtype=torch.float16, device=device)
        biases = torch.empty_like(scales)
        for e0 in range(0, n_experts, per):
            e1 = min(n_experts, e0 + per)
            w = torch.cat([_normal((rows, cols), std, seed * 100003 + expert_offset + e, device) for e in range(e0, e1)])
            q, s, b = quantize_q3(w)
            data[e0:e1] = q.view(e1 - e0, rows, -1)
            scales[e0:e1] = s.view(e1 - e0, rows, -1)
            biases[e0:e1] = b.view(e1 - e0, rows, -1)
        return ExpertBank.q3(data, scales, biases)
    raise ValueError(f"unknown format {fmt!r}")


def make_layer(fmt: str, hidden: int, inter: int, n_experts: int, seed: int, shared_inter: int | None = None,
               std: float = 0.02, device: torch.device | str = "cuda", limit: float | None = 10.0,
               expert_offset: int = 0) -> MoEWeights:
    """One MoE layer: w1/w3 [E, I, H], w2 [E, H, I] in `fmt`, shared expert bf16 (None to omit).

    expert_offset: the layer holds global experts [offset, offset + E) (an expert-parallel shard)."""
    w1 = make_bank(fmt, n_experts, inter, hidden, seed * 10 + 1, std, device, expert_offset)
    w3 = make_bank(fmt, n_experts, inter, hidden, seed * 10 + 3, std, device, expert_offset)
    w2 = make_bank(fmt, n_experts, hidden, inter, seed * 10 + 2, std, device, expert_offset)
    sw = [None, None, None]
    if shared_inter:
        sw = [_normal(shape, std, seed * 10 + 7 + i, device).to(torch.bfloat16)
              for i, shape in enumerate(((shared_inter, hidden), (shared_inter, hidden), (hidden, shared_inter)))]
    return MoEWeights(w1, w3, w2, *sw, swiglu_limit=limit if limit is not None else 0.0)


def zipf_routing(tokens: int, n_experts: int, top_k: int, s: float = 1.1, seed: int = 0,
                 device: torch.device | str = "cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """Top-k routing with Zipf(s) expert popularity.

    Expert rank r (1-based) has popularity r^-s; ranks map to ids through a
    seeded permutation.  Every token draws k distinct experts without
    replacement by Gumbel-top-k on log popularity; gates are a softmax of
    N(0, 1) logits over the k picks.  Returns ids [T, k] int32, gates [T, k] f32.
    """
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    rank_to_id = torch.randperm(n_experts, generator=g)
    logp = -s * torch.log(torch.arange(1, n_experts + 1, dtype=torch.float64))
    u = torch.rand(tokens, n_experts, generator=g, dtype=torch.float64).clamp_min(1e-300)
    gumbel = -torch.log(-torch.log(u))
    ranks = torch.topk(logp[None, :] + gumbel, top_k, dim=1).indices
    ids = rank_to_id[ranks].to(torch.int32)
    w = torch.softmax(torch.randn(tokens, top_k, generator=g), dim=1).float()
    return ids.to(device), w.to(device)
