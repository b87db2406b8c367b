"""Expert-wise token grouping and grouped SwiGLU execution on the GPU.

Drop-in for ``deepseeker.grouped`` (src/deepseeker/grouped.py):
  * ``plan_groups(topk_ids, n_experts)`` -- the planner, same dict and the
    same ValueError (grouped.py:19-31);
  * ``grouped_swiglu(x, weights, groups, router_weights=None)`` and
    ``naive_swiglu(x, weights, topk_ids, router_weights=None)`` with dense
    per-expert weights ``weights[e] = (gate [H, I], up [H, I], down [I, H])``
    (grouped.py:34-81), executed by ``ds_dense_swiglu`` in f32 with the
    reference's addition order;
plus the resident-bank path the batched workloads use (the batched expert
loop of ``moe_layer`` / ``gather_pinned_contributions``, mlx_forward.py:159-210):
  * ``GroupedFFN(layer)`` / ``grouped_ffn(x, layer, topk_ids, topk_w)`` --
    pairs sorted by expert on the device and pushed through tcgen05
    block-scaled MMAs (``ds_grouped_ffn``): FP4 banks as e2m1 operands
    (grouped.cu), q3 banks dequantised in shared memory to exact e4m3 codes
    with the per-64 scale and bias applied per group (grouped_q3.cu).
"""
from __future__ import annotations

import ctypes

import torch

from . import _abi
from ._dev import ptr, require_cuda, stream_handle
from .moe import MoEWeights


def plan_groups(topk_ids: list[list[int]], n_experts: int) -> dict[int, list[tuple[int, int]]]:
    """Map expert -> [(row, topk position)] (stable: ascending row order).

    Duplicate (row, expert) pairs are kept: the executor evaluates each
    occurrence, matching the naive loop exactly.
    """
    groups: dict[int, list[tuple[int, int]]] = {}
    for row, experts in enumerate(topk_ids):
        for pos, expert in enumerate(experts):
            expert = int(expert)
            if not 0 <= expert < n_experts:
                raise ValueError(f"expert {expert} out of range [0, {n_experts})")
            groups.setdefault(expert, []).append((row, pos))
    return groups


def _stack_dense(weights: dict, device) -> tuple[dict[int, int], torch.Tensor, torch.Tensor, torch.Tensor]:
    keys = sorted(int(e) for e in weights)
    index = {e: i for i, e in enumerate(keys)}
    g = torch.stack([torch.as_tensor(weights[e][0]).float() for e in keys]).to(device).contiguous()
    u = torch.stack([torch.as_tensor(weights[e][1]).float() for e in keys]).to(device).contiguous()
    d = torch.stack([torch.as_tensor(weights[e][2]).float() for e in keys]).to(device).contiguous()
    return index, g, u, d


def _dense_pairs(x: torch.Tensor, weights: dict, pairs: list[tuple[int, int, float | None]],
                 limit: float | None) -> torch.Tensor:
    """pairs: (row, expert, weight or None) in the order they are to be added per row."""
    if not isinstance(x, torch.Tensor):
        x = torch.as_tensor(x)
    dev = x.device if x.is_cuda else torch.device("cuda")
    T, H = x.shape
    out = torch.zeros(T, H, dtype=torch.float32, device=dev)
    if T == 0:
        return out.to(x.dtype)
    index, g, u, d = _stack_dense(weights, dev) if pairs else ({}, None, None, None)
    I = g.shape[2] if g is not None else 1
    # CSR by row, stable (the per-row order of `pairs` is the addition order)
    order = sorted(range(len(pairs)), key=lambda i: pairs[i][0])
    rows = [pairs[i][0] for i in order]
    exps = [index[pairs[i][1]] for i in order]
    has_w = any(p[2] is not None for p in pairs)
    wts = [float(pairs[i][2]) if pairs[i][2] is not None else 1.0 for i in order]
    row_ptr = [0] * (T + 1)
    for r in rows:
        row_ptr[r + 1] += 1
    for t in range(T):
        row_ptr[t + 1] += row_ptr[t]
    xf = x.to(dev).float().contiguous()
    pr = torch.tensor(rows or [0], dtype=torch.int32, device=dev)
    pe = torch.tensor(exps or [0], dtype=torch.int32, device=dev)
    pw = torch.tensor(wts or [0.0], dtype=torch.float32, device=dev) if has_w else None
    rp = torch.tensor(row_ptr, dtype=torch.int32, device=dev)
    ws_n = ctypes.c_size_t(0)
    _abi.call("ds_dense_swiglu_workspace_size", len(pairs), H, ctypes.byref(ws_n))
    ws = torch.empty(max(ws_n.value, 4), dtype=torch.uint8, device=dev)
    _abi.call("ds_dense_swiglu", ptr(xf), T, H, I, max(len(index), 1), ptr(g), ptr(u), ptr(d), len(pairs),
              ptr(pr), ptr(pe), ptr(pw), ptr(rp), float(limit or 0.0), ptr(out), ptr(ws), ws.numel(),
              stream_handle(dev))
    return out.to(x.dtype)


def grouped_swiglu(x: torch.Tensor, weights: dict, groups: dict[int, list[tuple[int, int]]],
                   router_weights: list[list[float]] | None = None) -> torch.Tensor:
    """Batched SwiGLU per expert + weighted scatter-add. Returns [T, H] (x.dtype).

    Contributions reach each row in the order of ``groups`` (grouped.py:43-55).
    """
    pairs = []
    for expert, occurrences in groups.items():
        for row, pos in occurrences:
            pairs.append((row, expert, router_weights[row][pos] if router_weights is not None else None))
    return _dense_pairs(x, weights, pairs, None)


def naive_swiglu(x: torch.Tensor, weights: dict, topk_ids: list[list[int]],
                 router_weights: list[list[float]] | None = None) -> torch.Tensor:
    """Per-(token, expert) path, accumulated in top-k order (grouped.py:59-81)."""
    pairs = []
    for row, experts in enumerate(topk_ids):
        for i, expert in enumerate(experts):
            pairs.append((row, int(expert), router_weights[row][i] if router_weights is not None else None))
    return _dense_pairs(x, weights, pairs, None)


class GroupedFFN:
    """Expert layer prepared for the batched grouped path: FP4 banks hold
    their re-laid-out scales (same bytes as the bank scales), q3 banks are
    read as stored; plus a workspace."""

    def __init__(self, layer: MoEWeights, top_k: int, activations: str = "exact"):
        """activations="exact": x and h enter the MMAs exactly (the parity
        mode); "fp4": FP4 banks only, x and h rounded to FP4 with per-32
        scales (the throughput mode, ds_grouped_ffn_fp4; its result carries
        that rounding)."""
        if layer.w1.fmt not in (_abi.DS_FMT_FP4, _abi.DS_FMT_Q3):
            raise NotImplementedError("grouped_ffn needs FP4 or q3 expert banks")
        if activations not in ("exact", "fp4"):
            raise ValueError('activations must be "exact" or "fp4"')
        if activations == "fp4":
            if layer.w1.fmt != _abi.DS_FMT_FP4:
                raise NotImplementedError("the FP4 activation mode needs FP4 banks")
            layer.prepare_tc()                     # the mode reads the tensor-core scale atoms
        self.activations = activations
        self.layer = layer
        self.top_k = top_k
        self._desc = self._routed_desc(top_k)
        a, b = ctypes.c_size_t(0), ctypes.c_size_t(0)
        if activations == "exact":                 # the FP4 activation mode reads the scale atoms instead
            _abi.call("ds_grouped_scales_size", ctypes.byref(self._desc), ctypes.byref(a), ctypes.byref(b))
        dev = layer.w1.data.device
        self.w13_sf = torch.empty(a.value, dtype=torch.uint8, device=dev)
        self.w2_sf = torch.empty(b.value, dtype=torch.uint8, device=dev)
        if activations == "exact":
            _abi.call("ds_grouped_prepare_scales", ctypes.byref(self._desc), ptr(self.w13_sf), ptr(self.w2_sf),
                      stream_handle(dev))
        self._ws: torch.Tensor | None = None

    def _routed_desc(self, top_k: int, route_before_down: bool | None = None) -> _abi.DsMoeDesc:
        d = self.layer.desc(top_k)
        d.shared_w1 = d.shared_w3 = d.shared_w2 = None
        d.shared_inter = 0
        if route_before_down is not None:
            d.route_before_down = 1 if route_before_down else 0
        return d

    def workspace_bytes(self, tokens: int) -> int:
        n = ctypes.c_size_t(0)
        fn = "ds_grouped_ffn_fp4_workspace_size" if self.activations == "fp4" else "ds_grouped_ffn_workspace_size"
        _abi.call(fn, ctypes.byref(self._desc), tokens, ctypes.byref(n))
        return n.value

    def __call__(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor,
                 out: torch.Tensor | None = None, route_before_down: bool | None = None,
                 out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        x = require_cuda(x, "x", torch.bfloat16)
        T, H = x.shape
        if H != self.layer.hidden:
            raise ValueError(f"x must be [T, {self.layer.hidden}]")
        topk_ids = require_cuda(topk_ids, "topk_ids", torch.int32)
        topk_w = require_cuda(topk_w, "topk_w", torch.float32)
        if topk_ids.shape != (T, self.top_k) or topk_w.shape != (T, self.top_k):
            raise ValueError(f"topk_ids / topk_w must be [T, {self.top_k}]")
        d = self._routed_desc(self.top_k, route_before_down)
        need = self.workspace_bytes(T)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        if out is None:
            out = torch.empty(T, H, dtype=out_dtype, device=x.device)
        if out.dtype not in (torch.bfloat16, torch.float32) or out.shape != (T, H) or not out.is_contiguous():
            raise ValueError("out must be a contiguous [T, H] bf16 or f32 tensor")
        odt = _abi.DS_F32 if out.dtype == torch.float32 else _abi.DS_BF16
        if self.activations == "fp4":
            _abi.call("ds_grouped_ffn_fp4", ctypes.byref(d), ptr(x), _abi.DS_BF16, T, ptr(topk_ids), ptr(topk_w),
                      ptr(out), odt, ptr(self._ws), self._ws.numel(), stream_handle(x.device))
            return out
        _abi.call("ds_grouped_ffn", ctypes.byref(d), ptr(self.w13_sf), ptr(self.w2_sf), ptr(x), _abi.DS_BF16, T,
                  ptr(topk_ids), ptr(topk_w), ptr(out), odt, ptr(self._ws), self._ws.numel(),
                  stream_handle(x.device))
        return out


def grouped_ffn(x: torch.Tensor, layer: MoEWeights, topk_ids: torch.Tensor, topk_w: torch.Tensor,
                route_before_down: bool | None = None) -> torch.Tensor:
    """One-shot form of GroupedFFN (prepares the scales on every call)."""
    return GroupedFFN(layer, topk_ids.shape[1])(x, topk_ids, topk_w, route_before_down=route_before_down)
