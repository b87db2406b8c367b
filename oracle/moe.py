"""MoE routing / SwiGLU expert FFN / combine / alignment CPU oracle (torch fp32, numpy)
-- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates:
  * ``sqrtsoftplus_scores``, ``route_topk``        src/deepseeker/mlx_forward.py:62-81
  * BASELINE config 2 router: softmax over all experts, top-k, gates
    renormalised to sum 1 (builder restatement of the config text)
  * routed expert FFN + sorted scatter-add combine + shared add
                                                   mlx_forward.py:388-419 (moe_layer loop),
                                                   mlx_forward.py:84-103 (qmm: x f32 @ dequant(W).T)
  * shared expert                                  src/deepseeker/mlx_runner.py:765-783
  * ``plan_groups``, ``grouped_swiglu``, ``naive_swiglu``   src/deepseeker/grouped.py:19-81
  * ``align_block_size``                           src/deepseeker/moe_align.py:21-46
"""
from __future__ import annotations

import numpy as np
import torch


# ---------------------------------------------------------------- routing

def sqrtsoftplus_scores(x: torch.Tensor, gate_w: torch.Tensor) -> torch.Tensor:
    """sqrt(softplus(x @ W.T)) in f32 (mlx_forward.py:62-65; logaddexp(s, 0) == softplus)."""
    s = x.float() @ gate_w.float().T
    return torch.sqrt(torch.logaddexp(s, torch.zeros_like(s)))


def route_topk(scores: torch.Tensor, bias: torch.Tensor, top_k: int,
               route_scale: float = 1.5) -> tuple[torch.Tensor, torch.Tensor]:
    """mlx_forward.py:68-81: indices = last top_k of an ascending argsort of
    scores + bias; weights = scores[indices] / (sum + 1e-20) * route_scale."""
    biased = scores + bias.float()
    order = torch.argsort(biased, dim=-1, stable=True)
    idx = order[:, -top_k:]
    w = torch.gather(scores, 1, idx)
    w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return w * route_scale, idx


def route_softmax_topk(logits: torch.Tensor, top_k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Softmax over all experts, top-k (ties -> lower id), gates renormalised to 1.

    Returns (weights [S, k] f32, ids [S, k] int64), slots in descending gate order.
    """
    p = torch.softmax(logits.float(), dim=-1)
    # stable descending order: sort ascending on (-p) with stable ties -> lower id first
    order = torch.argsort(-p, dim=-1, stable=True)
    idx = order[:, :top_k]
    w = torch.gather(p, 1, idx)
    return w / w.sum(-1, keepdim=True), idx


# ---------------------------------------------------------------- expert FFN

def swiglu_hidden(xf: torch.Tensor, w1: torch.Tensor, w3: torch.Tensor,
                  limit: float | None) -> torch.Tensor:
    """h = silu(min(x W1^T, L)) * clip(x W3^T, -L, L) in f32 (mlx_forward.py:399-403)."""
    g = xf @ w1.T
    u = xf @ w3.T
    if limit is not None:
        g = torch.clamp(g, max=limit)
        u = torch.clamp(u, -limit, limit)
    return (g / (1.0 + torch.exp(-g))) * u


def expert_ffn(x: torch.Tensor, w1: torch.Tensor, w3: torch.Tensor, w2: torch.Tensor,
               limit: float | None = 10.0) -> torch.Tensor:
    """Single routed expert: down(silu(gate x) * up x), f32."""
    return swiglu_hidden(x.float(), w1.float(), w3.float(), limit) @ w2.float().T


def shared_expert(x: torch.Tensor, w1: torch.Tensor, w3: torch.Tensor, w2: torch.Tensor,
                  limit: float = 10.0) -> torch.Tensor:
    """mlx_runner.py:776-781: f32 SwiGLU with clamps, result cast to x.dtype."""
    h = swiglu_hidden(x.float(), w1.float(), w3.float(), limit)
    return (h @ w2.float().T).to(x.dtype)


def moe_combine(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor,
                expert_weights, shared=None, limit: float | None = 10.0) -> torch.Tensor:
    """Routed experts + sorted scatter-add + shared add (mlx_forward.py:388-419).

    ``expert_weights(e) -> (w1 [I,H], w3 [I,H], w2 [H,I])`` dense f32 (already
    dequantised); ``shared`` is None or dense (w1, w3, w2).  The route weight is
    applied to h before the down projection (mlx_forward.py:404-405).  Experts
    are visited in ascending id order; a token uses its first slot for an
    expert (mlx_forward.py:394-396).  Returns ``out.to(x.dtype)``.
    """
    idx = topk_ids.cpu().numpy().astype(np.int64)
    wts = topk_w.float().cpu()
    out = torch.zeros(x.shape, dtype=torch.float32)
    for expert in np.unique(idx):
        if expert < 0:
            continue
        mask = idx == expert
        rows = np.where(mask.any(axis=1))[0]
        cols = [int(np.where(mask[r])[0][0]) for r in rows]
        w1, w3, w2 = expert_weights(int(expert))
        xr = x[torch.as_tensor(rows)].float()
        h = swiglu_hidden(xr, w1.float(), w3.float(), limit)
        rw = wts[torch.as_tensor(rows), torch.as_tensor(cols)].reshape(-1, 1)
        out[torch.as_tensor(rows)] += (h * rw) @ w2.float().T
    if shared is not None:
        out = out + shared_expert(x, *shared, limit=10.0 if limit is None else limit).float()
    return out.to(x.dtype)


# ---------------------------------------------------------------- grouped (grouped.py)

def plan_groups(topk_ids, n_experts: int) -> dict[int, list[tuple[int, int]]]:
    """grouped.py:19-31: expert -> [(row, pos)] in ascending row order."""
    groups: dict[int, list[tuple[int, int]]] = {}
    for row, experts in enumerate(topk_ids):
        for pos, expert in enumerate(experts):
            expert = int(expert)
            if not 0 <= expert < n_experts:
                raise ValueError(f"expert {expert} out of range [0, {n_experts})")
            groups.setdefault(expert, []).append((row, pos))
    return groups


def grouped_swiglu(x: torch.Tensor, weights, groups, router_weights=None) -> torch.Tensor:
    """grouped.py:34-56: dense weights (gate [H,I], up [H,I], down [I,H]), no clamp,
    router weight applied AFTER the down projection, scatter-add per expert."""
    out = torch.zeros(x.shape, dtype=torch.float32)
    xf = x.float()
    for expert, occ in groups.items():
        gate, up, down = (t.float() for t in weights[expert])
        rows = torch.as_tensor([r for r, _ in occ])
        xr = xf[rows]
        g = xr @ gate
        y = (g * torch.sigmoid(g) * (xr @ up)) @ down
        if router_weights is not None:
            w = torch.tensor([router_weights[r][p] for r, p in occ], dtype=torch.float32)
            y = y * w.reshape(-1, 1)
        out.index_add_(0, rows, y)
    return out.to(x.dtype)


def naive_swiglu(x: torch.Tensor, weights, topk_ids, router_weights=None) -> torch.Tensor:
    """grouped.py:59-81: per-(token, expert) GEMV, accumulated in top-k order."""
    out = torch.zeros(x.shape, dtype=torch.float32)
    xf = x.float()
    for row, experts in enumerate(topk_ids):
        acc = torch.zeros(x.shape[1])
        for i, expert in enumerate(experts):
            gate, up, down = (t.float() for t in weights[int(expert)])
            xr = xf[row:row + 1]
            g = xr @ gate
            y = ((g * torch.sigmoid(g) * (xr @ up)) @ down).reshape(-1)
            if router_weights is not None:
                y = y * router_weights[row][i]
            acc = acc + y
        out[row] += acc
    return out.to(x.dtype)


# ---------------------------------------------------------------- align (moe_align.py)

def align_block_size(topk_ids: np.ndarray, block_size: int, num_experts: int):
    """moe_align.py:21-46: stable sort of flat ids by expert, each run padded to a
    multiple of block_size with sentinel M*K; expert id per block; padded length."""
    topk_ids = np.asarray(topk_ids)
    if topk_ids.ndim != 2:
        raise ValueError(f"topk_ids must be 2-D, got shape {topk_ids.shape}")
    if block_size < 1 or num_experts < 1:
        raise ValueError("block_size and num_experts must be >= 1")
    flat = topk_ids.reshape(-1)
    if flat.size and (flat.min() < 0 or flat.max() >= num_experts):
        raise ValueError("expert ids out of range")
    sentinel = flat.size
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=num_experts) if flat.size else np.zeros(num_experts, np.int64)
    sorted_ids: list[np.ndarray] = []
    expert_ids: list[int] = []
    start = 0
    for expert in range(num_experts):
        c = int(counts[expert])
        run = order[start:start + c]
        start += c
        pad = (-c) % block_size
        sorted_ids.append(np.concatenate([run, np.full(pad, sentinel)]).astype(np.int64))
        expert_ids.extend([expert] * ((c + pad) // block_size))
    s = np.concatenate(sorted_ids) if sorted_ids else np.zeros(0, np.int64)
    return s.astype(np.int64), np.asarray(expert_ids, dtype=np.int64), int(s.size)
