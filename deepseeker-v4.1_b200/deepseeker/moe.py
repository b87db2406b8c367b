"""Routed-expert MoE layer on B200 -- the MoE subset of the reference's ``deepseeker.mlx_forward``.

Reference: src/deepseeker/mlx_forward.py:62-419 (router, qmm, gate/up
stacking, banked gather, union cap, moe_layer) and
src/deepseeker/mlx_runner.py:765-783 (shared expert).  ``moe_layer`` keeps the
reference's signature (``expert_fn`` / ``shared_fn`` callables, trace and
prefetch hooks, union cap); experts are best held resident in HBM as stacked
banks (``ExpertBank``: [E, N, ...] in the checkpoint's FP4 layout, or the
build's 3-bit layout; ``MoEWeights.resident()`` / ``shared_expert()``), which
lets the whole routed loop run as one fused decode call.  The reference's
SSD read pipeline (``pipeline=True`` with its submit / finalize hooks) is
accepted and gives the same result as the plain path.

Semantics kept from the reference:
  * router: sqrt(softplus(x Wg^T)), top-k of scores + bias, gates = scores /
    (sum + 1e-20) * route_scale (mlx_forward.py:62-81); BASELINE's softmax
    top-k router is also available;
  * per distinct expert, ascending id: g = min(x W1^T, L), u = clip(x W3^T, ±L),
    h = silu(g) * u, h *= gate BEFORE the down projection, out += h W2^T, in
    f32 with the weights dequantised exactly (mlx_forward.py:388-405);
  * shared expert: bf16 weights, same clamps, output rounded to x.dtype before
    being added (mlx_runner.py:776-781, mlx_forward.py:309-310, 409-410);
  * result cast to x.dtype (bf16).
"""
from __future__ import annotations

import contextlib
import ctypes
import gc
from dataclasses import dataclass, field

import torch

from . import _abi
from ._dev import ptr, require_cuda, stream_handle

MAX_DECODE_TOKENS = 8


# ------------------------------------------------------------------ routing

def sqrtsoftplus_scores(x: torch.Tensor, gate_w: torch.Tensor) -> torch.Tensor:
    """Router scores sqrt(softplus(x @ Wg^T)) in f32 (mlx_forward.py:62-65)."""
    s = x.float() @ gate_w.float().T
    return torch.sqrt(torch.nn.functional.softplus(s))


def _route(inp: torch.Tensor, bias: torch.Tensor | None, top_k: int, kind: int,
           route_scale: float, out: tuple[torch.Tensor, torch.Tensor] | None = None
           ) -> tuple[torch.Tensor, torch.Tensor]:
    inp = require_cuda(inp, "router input", torch.float32)
    if inp.dim() != 2:
        raise ValueError("router input must be [rows, n_experts]")
    rows, n_exp = inp.shape
    if bias is not None:
        bias = require_cuda(bias.float(), "bias")
    if out is not None:
        w, ids = out
        if (w.shape != (rows, top_k) or ids.shape != (rows, top_k) or w.dtype != torch.float32
                or ids.dtype != torch.int32 or not (w.is_contiguous() and ids.is_contiguous())):
            raise ValueError("out must be (weights f32 [rows, k], ids int32 [rows, k]), contiguous")
    else:
        ids = torch.empty((rows, top_k), dtype=torch.int32, device=inp.device)
        w = torch.empty((rows, top_k), dtype=torch.float32, device=inp.device)
    _abi.call("ds_route_topk", ptr(inp), ptr(bias), rows, n_exp, top_k, kind, ctypes.c_float(route_scale),
              ptr(ids), ptr(w), stream_handle(inp.device))
    return w, ids


def route_topk(scores: torch.Tensor, bias: torch.Tensor, top_k: int,
               route_scale: float = 1.5) -> tuple[torch.Tensor, torch.Tensor]:
    """(weights [n, k] f32, indices [n, k] int32): top-k of scores + bias, gates from raw scores.

    Slots come in descending biased-score order (the reference returns the same
    pairs in ascending order; pairs are equal as sets)."""
    return _route(scores, bias, top_k, _abi.DS_ROUTE_SCORES, route_scale)


def route_sqrtsoftplus(logits: torch.Tensor, bias: torch.Tensor | None, top_k: int,
                       route_scale: float = 1.5) -> tuple[torch.Tensor, torch.Tensor]:
    """sqrt(softplus) + route_topk fused in one kernel, from router logits x Wg^T."""
    return _route(logits, bias, top_k, _abi.DS_ROUTE_SQRTSOFTPLUS, route_scale)


def route_softmax_topk(logits: torch.Tensor, top_k: int,
                       out: tuple[torch.Tensor, torch.Tensor] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Softmax over experts, top-k (ties -> lower id), gates renormalised to 1.

    out: optional preallocated (weights, ids) to write into."""
    return _route(logits, None, top_k, _abi.DS_ROUTE_SOFTMAX, 1.0, out)


# ------------------------------------------------------------------ banks

@dataclass
class ExpertBank:
    """Resident stacked expert matrices [E, N, K] in a compressed format.

    FP4 : data [E, N, K/2] u8 (checkpoint layout), scales [E, N, K/32] u8 (ue8m0)
    Q3  : data [E, N, K*3/32] int32 (u32 words), scales/biases [E, N, K/64] f16
    """
    fmt: int
    data: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor | None = None
    scales_tc: torch.Tensor | None = None   # FP4: tensor-core scale atoms (prepare_atoms)

    @property
    def n_experts(self) -> int:
        return self.data.shape[0]

    @property
    def rows(self) -> int:
        return self.data.shape[1]

    @property
    def cols(self) -> int:
        if self.fmt == _abi.DS_FMT_FP4:
            return self.data.shape[2] * 2
        return self.scales.shape[2] * 64

    @classmethod
    def fp4(cls, packed: torch.Tensor, scales: torch.Tensor) -> "ExpertBank":
        packed = require_cuda(packed, "packed", torch.uint8)
        scales = require_cuda(scales, "scales", torch.uint8)
        if packed.dim() != 3 or scales.shape != (*packed.shape[:2], packed.shape[2] // 16):
            raise ValueError(f"FP4 bank shapes {tuple(packed.shape)} / {tuple(scales.shape)} disagree")
        return cls(_abi.DS_FMT_FP4, packed, scales)

    @classmethod
    def q3(cls, words: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor) -> "ExpertBank":
        words = require_cuda(words, "words", (torch.int32, torch.uint32))
        scales = require_cuda(scales, "scales", torch.float16)
        biases = require_cuda(biases, "biases", torch.float16)
        if scales.shape != biases.shape or words.shape != (*scales.shape[:2], scales.shape[2] * 6):
            raise ValueError("q3 bank shapes disagree")
        return cls(_abi.DS_FMT_Q3, words, scales, biases)

    def c_struct(self) -> _abi.DsExpertBank:
        return _abi.DsExpertBank(self.fmt, self.n_experts, self.rows, self.cols, self.data.data_ptr(),
                                 self.scales.data_ptr(), 0 if self.biases is None else self.biases.data_ptr(),
                                 0 if self.scales_tc is None else self.scales_tc.data_ptr())

    def prepare_atoms(self) -> "ExpertBank":
        """FP4: build the tensor-core scale atoms once (same byte count as the scales)."""
        if self.fmt != _abi.DS_FMT_FP4:
            raise NotImplementedError("scale atoms exist for FP4 banks only")
        if self.scales_tc is None:
            atoms = torch.empty_like(self.scales)
            _abi.call("ds_fp4_scale_atoms", ptr(self.scales), self.n_experts, self.rows, self.cols, ptr(atoms),
                      stream_handle(self.scales.device))
            self.scales_tc = atoms
        return self

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.data, self.scales, self.biases) if t is not None)


@dataclass
class MoEWeights:
    """One MoE layer's resident weights: routed banks + optional bf16 shared expert."""
    w1: ExpertBank
    w3: ExpertBank
    w2: ExpertBank
    shared_w1: torch.Tensor | None = None    # [Is, H] bf16
    shared_w3: torch.Tensor | None = None    # [Is, H] bf16
    shared_w2: torch.Tensor | None = None    # [H, Is] bf16
    swiglu_limit: float = 10.0
    route_before_down: bool = True
    _descs: dict = field(default_factory=dict, repr=False)
    _ws_bytes: dict = field(default_factory=dict, repr=False)

    @property
    def hidden(self) -> int:
        return self.w1.cols

    def prepare_tc(self) -> "MoEWeights":
        """FP4 layers: prepare the scale atoms the tcgen05 decode kernels read
        (q3 layers need no preparation: a no-op)."""
        if self.w1.fmt != _abi.DS_FMT_FP4:
            return self
        for b in (self.w1, self.w3, self.w2):
            b.prepare_atoms()
        self._descs.clear()
        self._ws_bytes.clear()
        return self

    def cached_desc(self, top_k: int) -> _abi.DsMoeDesc:
        """desc(top_k), built once per top_k (the banks are immutable once resident)."""
        d = self._descs.get(top_k)
        if d is None:
            d = self._descs[top_k] = self.desc(top_k)
        return d

    def decode_workspace_bytes(self, tokens: int, top_k: int) -> int:
        key = (tokens, top_k)
        n = self._ws_bytes.get(key)
        if n is None:
            c = ctypes.c_size_t(0)
            _abi.call("ds_moe_decode_workspace_size", ctypes.byref(self.cached_desc(top_k)), tokens, ctypes.byref(c))
            n = self._ws_bytes[key] = c.value
        return n

    @property
    def inter(self) -> int:
        return self.w1.rows

    @property
    def n_experts(self) -> int:
        return self.w1.n_experts

    def desc(self, top_k: int) -> _abi.DsMoeDesc:
        sh = self.shared_w1 is not None
        for t, name in ((self.shared_w1, "shared_w1"), (self.shared_w3, "shared_w3"), (self.shared_w2, "shared_w2")):
            if sh and (t is None or t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous()):
                raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor")
        d = _abi.DsMoeDesc()
        d.hidden, d.inter, d.n_experts, d.top_k = self.hidden, self.inter, self.n_experts, top_k
        d.w1, d.w3, d.w2 = self.w1.c_struct(), self.w3.c_struct(), self.w2.c_struct()
        d.shared_w1 = self.shared_w1.data_ptr() if sh else 0
        d.shared_w3 = self.shared_w3.data_ptr() if sh else 0
        d.shared_w2 = self.shared_w2.data_ptr() if sh else 0
        d.shared_inter = self.shared_w1.shape[0] if sh else 0
        d.swiglu_limit = float(self.swiglu_limit) if self.swiglu_limit is not None else 0.0
        d.route_before_down = 1 if self.route_before_down else 0
        return d

    def resident(self) -> "ResidentExperts":
        """The routed banks in the role of moe_layer's ``expert_fn``."""
        return ResidentExperts(self)

    def shared_expert(self) -> "SharedExpert | None":
        """The bf16 shared expert in the role of moe_layer's ``shared_fn`` (None without one)."""
        if self.shared_w1 is None:
            return None
        return SharedExpert(self.shared_w1, self.shared_w3, self.shared_w2)

    def streamed_bytes(self, n_distinct: int) -> int:
        """Algorithmic HBM bytes of one decode step touching `n_distinct` experts."""
        per_expert = sum(b.nbytes() // b.n_experts for b in (self.w1, self.w3, self.w2))
        shared = sum(t.numel() * 2 for t in (self.shared_w1, self.shared_w3, self.shared_w2) if t is not None)
        return n_distinct * per_expert + shared


_WS: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), 0)
    ws = _WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = ws
    return ws


def decode_workspace_bytes(weights: MoEWeights, tokens: int, top_k: int) -> int:
    return weights.decode_workspace_bytes(tokens, top_k)


def _decode_call(x: torch.Tensor, weights: MoEWeights, k: int, out: torch.Tensor | None,
                 workspace: torch.Tensor | None, out_f32: bool):
    """Checks and arguments shared by moe_decode and moe_decode_routed."""
    x = require_cuda(x, "x", (torch.bfloat16, torch.float32))
    if x.dim() != 2 or x.shape[1] != weights.hidden:
        raise ValueError(f"x must be [T, {weights.hidden}]")
    T = x.shape[0]
    if not 1 <= T <= MAX_DECODE_TOKENS:
        raise ValueError(f"moe_decode handles 1..{MAX_DECODE_TOKENS} tokens, got {T}")
    d = weights.cached_desc(k)
    if (bool(d.route_before_down) != bool(weights.route_before_down)
            or d.swiglu_limit != ctypes.c_float(weights.swiglu_limit or 0.0).value):
        weights._descs.clear()
        d = weights.cached_desc(k)
    need = weights.decode_workspace_bytes(T, k)
    ws = workspace if workspace is not None else _workspace(x.device, need)
    if out_f32 and x.dtype != torch.float32:
        d = _abi.DsMoeDesc.from_buffer_copy(d)
        d.out_f32 = 1
    odt = torch.float32 if (out_f32 or x.dtype == torch.float32) else x.dtype
    if out is None:
        out = torch.empty(x.shape, dtype=odt, device=x.device)
    elif out.dtype != odt or out.shape != x.shape or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous {tuple(x.shape)} {odt} tensor")
    xdt = _abi.DS_F32 if x.dtype == torch.float32 else _abi.DS_BF16
    return x, T, d, ws, out, xdt


def moe_decode(x: torch.Tensor, weights: MoEWeights, topk_ids: torch.Tensor, topk_w: torch.Tensor,
               out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
               out_f32: bool = False) -> torch.Tensor:
    """Fused routed-expert MoE for up to 8 tokens: x [T, H] bf16 (or f32) -> [T, H] of x's dtype.

    topk_ids [T, k] int32 (-1 = dropped slot), topk_w [T, k] f32.  out_f32
    (bf16 x, FP4 banks with prepared scale atoms): f32 output without the final
    rounding, for partial sums that are added across ranks.
    """
    topk_ids = require_cuda(topk_ids, "topk_ids", torch.int32)
    topk_w = require_cuda(topk_w, "topk_w", torch.float32)
    k = topk_ids.shape[1]
    x, T, d, ws, out, xdt = _decode_call(x, weights, k, out, workspace, out_f32)
    if topk_ids.shape != (T, k) or topk_w.shape != (T, k):
        raise ValueError("topk_ids / topk_w must be [T, k]")
    _abi.call("ds_moe_decode", ctypes.byref(d), ptr(x), xdt, T, ptr(topk_ids), ptr(topk_w), ptr(out), ptr(ws),
              ws.numel() * ws.element_size(), stream_handle(x.device))
    return out


ROUTE_KINDS = {"softmax": _abi.DS_ROUTE_SOFTMAX, "sqrtsoftplus": _abi.DS_ROUTE_SQRTSOFTPLUS,
               "scores": _abi.DS_ROUTE_SCORES}


def moe_decode_routed(x: torch.Tensor, weights: MoEWeights, logits: torch.Tensor, top_k: int,
                      kind: str = "softmax", bias: torch.Tensor | None = None, route_scale: float = 1.0,
                      out: torch.Tensor | None = None,
                      route_out: tuple[torch.Tensor, torch.Tensor] | None = None,
                      workspace: torch.Tensor | None = None, out_f32: bool = False
                      ) -> tuple[torch.Tensor, tuple[torch.Tensor, torch.Tensor]]:
    """Router + fused decode in one C call (``ds_moe_decode_route``).

    logits [T, E] f32 -> (out [T, H], (weights [T, k] f32, ids [T, k] int32)):
    the same results as ``route_*`` followed by ``moe_decode``, bit for bit
    (route_topk / the softmax router, mlx_forward.py:62-81).  On the tcgen05
    kernels the routing is computed inside the decode's first kernel, one
    launch fewer per layer.  kind: "softmax" (route_scale unused),
    "sqrtsoftplus" (scores + bias, the reference's route_topk) or "scores".
    ``out`` may be a pinned host tensor: the layer then writes its output
    rows straight into it through its device mapping (read it after the
    stream has been waited for).
    """
    if kind not in ROUTE_KINDS:
        raise ValueError(f"kind must be one of {sorted(ROUTE_KINDS)}")
    logits = require_cuda(logits, "logits", torch.float32)
    out_addr = None
    if out is not None and not out.is_cuda:
        out_addr = host_device_pointer(out)          # ValueError unless pinned and mapped
    x, T, d, ws, out, xdt = _decode_call(x, weights, top_k, out, workspace, out_f32)
    if out_addr is None:
        out_addr = out.data_ptr()
    if logits.shape != (T, weights.n_experts) or not logits.is_contiguous():
        raise ValueError(f"logits must be a contiguous [T, {weights.n_experts}] f32 tensor")
    if bias is not None:
        bias = require_cuda(bias.float().contiguous(), "bias")
        if bias.shape != (weights.n_experts,):
            raise ValueError(f"bias must be [{weights.n_experts}]")
    if route_out is not None:
        w, ids = route_out
        if (w.shape != (T, top_k) or ids.shape != (T, top_k) or w.dtype != torch.float32
                or ids.dtype != torch.int32 or not (w.is_contiguous() and ids.is_contiguous())):
            raise ValueError("route_out must be (weights f32 [T, k], ids int32 [T, k]), contiguous")
    else:
        w = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
        ids = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    _abi.call("ds_moe_decode_route", ctypes.byref(d), ptr(x), xdt, T, ptr(logits), ptr(bias), ROUTE_KINDS[kind],
              ctypes.c_float(route_scale), ptr(ids), ptr(w), ctypes.c_void_p(out_addr), ptr(ws),
              ws.numel() * ws.element_size(), stream_handle(x.device))
    return out, (w, ids)


# ------------------------------------------------------------------ qmm (mlx_forward.py:84-156)

def _matrix_bank(w: tuple) -> ExpertBank:
    """One compressed matrix as a one-expert bank view: (packed, scales) FP4
    (packed u8 [N, K/2] or the u32 view [N, K/8] of pack_fp4_mxfp4, scales u8
    [N, K/32]) or (words, scales, biases) Q3 (words u32/int32 [N, K*3/32],
    f16 [N, K/64] scales and biases)."""
    if not isinstance(w, (tuple, list)) or len(w) not in (2, 3):
        raise ValueError("qmm operands must be (packed, scales) mxfp4 or (words, scales, biases) q3")
    if len(w) == 2:
        packed, scales = w
        packed = require_cuda(packed, "packed", (torch.uint8, torch.int32, torch.uint32))
        if packed.dtype != torch.uint8:
            packed = packed.view(torch.uint8)
        scales = require_cuda(scales, "scales", torch.uint8)
        if packed.dim() != 2 or scales.dim() != 2:
            raise ValueError("mxfp4 operands must be 2-D [N, K/2] (or u32 [N, K/8]) and [N, K/32]")
        return ExpertBank.fp4(packed.unsqueeze(0), scales.unsqueeze(0))
    words, scales, biases = w
    if words.dim() != 2 or scales.dim() != 2:
        raise ValueError("q3 operands must be 2-D [N, K*3/32], [N, K/64], [N, K/64]")
    return ExpertBank.q3(words.unsqueeze(0), scales.unsqueeze(0), biases.unsqueeze(0))


def qmm(x: torch.Tensor, w: tuple) -> torch.Tensor:
    """x @ W.T with W held compressed: arity 2 = mxfp4 (packed, ue8m0 scales),
    arity 3 = q3 affine (words, f16 scales, f16 biases), group 64
    (mlx_forward.py:84-103).  x [..., K] f32 (or bf16) -> [..., N] f32; the
    weights are dequantised in registers, never materialised."""
    bank = _matrix_bank(w)
    x = require_cuda(x, "x", (torch.float32, torch.bfloat16))
    K = bank.cols
    if x.shape[-1] != K:
        raise ValueError(f"x has {x.shape[-1]} features, the matrix {K}")
    x2 = x.reshape(-1, K)
    out = torch.empty((x2.shape[0], bank.rows), dtype=torch.float32, device=x.device)
    if x2.shape[0]:
        wb = bank.c_struct()
        xdt = _abi.DS_F32 if x2.dtype == torch.float32 else _abi.DS_BF16
        with torch.cuda.device(x.device):
            _abi.call("ds_qmm", ctypes.byref(wb), ptr(x2), xdt, x2.shape[0], ptr(out), stream_handle(x.device))
    return out.reshape(*x.shape[:-1], bank.rows)


def stack_gate_up_expert(weights: dict) -> dict:
    """w1 / w3 operands concatenated along the output rows into one "w13"
    (mlx_forward.py:106-120); a dict that already holds w13 is returned as is."""
    if "w13" in weights:
        return weights
    w1, w3 = weights["w1"], weights["w3"]
    if len(w1) != len(w3) or len(w1) not in (2, 3):
        raise ValueError("w1/w3 operand arity must be 2 (mxfp4) or 3 (q3)")
    for a, b in zip(w1, w3):
        if a.shape[1:] != b.shape[1:] or a.shape[0] != b.shape[0]:
            raise ValueError("gate/up packed shapes must agree")
    return {"w13": tuple(torch.cat((a, b), dim=0) for a, b in zip(w1, w3)), "w2": weights["w2"]}


def split_gate_up_expert(weights: dict) -> dict:
    """w1 / w3 views of a stacked "w13" without copying (mlx_forward.py:123-140)."""
    if "w13" not in weights:
        return weights
    parts = weights["w13"]
    halves: dict[str, list] = {"w1": [], "w3": []}
    for part in parts:
        if part.shape[0] % 2:
            raise ValueError("stacked gate/up operand rows must divide evenly")
        n = part.shape[0] // 2
        halves["w1"].append(part[:n])
        halves["w3"].append(part[n:])
    return {"w1": tuple(halves["w1"]), "w3": tuple(halves["w3"]), "w2": weights["w2"]}


def gate_up_qmm(x: torch.Tensor, weights, *, stack_single_row: bool = False
                ) -> tuple[torch.Tensor, torch.Tensor, tuple]:
    """(gate, up, w2 operands) for rows x; with stack_single_row and one row,
    gate and up come from one qmm over the stacked w13 (mlx_forward.py:143-156)."""
    if isinstance(weights, dict):
        expert = weights
    else:
        w1, w3, w2 = weights
        expert = {"w1": w1, "w3": w3, "w2": w2}
    single = stack_single_row and x.shape[0] == 1
    if "w13" not in expert and single:
        expert = stack_gate_up_expert(expert)
    if "w13" in expert and single:
        gate, up = torch.chunk(qmm(x, expert["w13"]), 2, dim=-1)
    else:
        sep = split_gate_up_expert(expert)
        gate, up = qmm(x, sep["w1"]), qmm(x, sep["w3"])
    return gate, up, expert["w2"]


def gather_pinned_contributions(x: torch.Tensor, indices, weights, banks: dict[str, tuple],
                                slots: dict[int, int], limit: float = 10.0) -> dict[int, tuple]:
    """Per-expert weighted outputs of the (expert, row, column) pairs whose
    expert sits in a resident bank (mlx_forward.py:159-210): banks[role] holds
    stacked operands [E_b, N, ...], slots maps expert -> bank index.  Pairs in
    (expert, row) order; every matching column counts (duplicates included);
    the route weight multiplies h before the down projection.  Returns
    {expert: (rows int32 numpy, contributions [n, H] f32)}."""
    import numpy as np

    idx = np.asarray(indices)
    wts = np.asarray(weights, dtype=np.float32)
    out = {}
    for expert in sorted(slots):
        rr, cc = np.nonzero(idx == int(expert))
        if rr.size == 0:
            continue
        order = np.lexsort((cc, rr))
        rr, cc = rr[order], cc[order]
        b = slots[expert]
        ops = {role: tuple(part[b] for part in banks[role]) for role in ("w1", "w3", "w2")}
        xr = x[torch.as_tensor(rr, device=x.device)].float()
        g = torch.clamp(qmm(xr, ops["w1"]), max=limit)
        u = torch.clamp(qmm(xr, ops["w3"]), -limit, limit)
        h = g / (1.0 + torch.exp(-g)) * u
        rw = torch.as_tensor(wts[rr, cc], device=x.device).reshape(-1, 1)
        out[int(expert)] = (rr.astype(np.int32), qmm(h * rw, ops["w2"]))
    return out


def cap_union(idx, w, n_experts: int, budget: int, *, scores=None, strict: bool = False):
    """Cap the batch's expert union at ``budget`` experts (mlx_forward.py:213-254):
    keep the experts with the largest summed gate weight (or summed raw score
    when ``scores`` is given), drop the others' slots (index -1, weight 0),
    renormalise each row to its original weight sum; unless ``strict``, a row
    that would lose every slot keeps its heaviest one.  Returns (indices
    int64, weights f32, share of the total weight kept before renormalising)."""
    import numpy as np

    idx = np.asarray(idx)
    w = np.asarray(w, dtype=np.float32)
    if np.unique(idx).size <= budget:
        return idx, w, 1.0
    mass = np.zeros(n_experts, dtype=np.float32)
    if scores is not None:
        np.add.at(mass, idx.ravel(), np.asarray(scores)[np.arange(idx.shape[0])[:, None], idx].ravel())
    else:
        np.add.at(mass, idx.ravel(), w.ravel())
    keep = np.zeros(n_experts, dtype=bool)
    keep[np.argpartition(mass, -budget)[-budget:]] = True
    kept = keep[idx]
    lost = ~kept.any(axis=1)
    if lost.any() and not strict:
        kept[np.nonzero(lost)[0], w[lost].argmax(axis=1)] = True
    kept_w = np.where(kept, w, 0.0)
    total, kept_total = float(w.sum()), float(kept_w.sum())
    rescale = w.sum(axis=1, keepdims=True) / (kept_w.sum(axis=1, keepdims=True) + 1e-20)
    return (np.where(kept, idx, -1).astype(np.int64), (kept_w * rescale).astype(np.float32),
            kept_total / total if total > 0 else 1.0)


# ------------------------------------------------------------------ moe_layer (mlx_forward.py:257-419)

class ResidentExperts:
    """A layer's routed experts held resident as banks (``MoEWeights``), in the
    role of the reference's ``expert_fn``: calling it with an expert id gives
    that expert's (w1, w3, w2) operand tuples (views into the banks), and
    ``moe_layer`` runs the whole routed loop as one fused kernel when it gets
    one of these."""

    def __init__(self, weights: "MoEWeights"):
        self.weights = weights

    def __call__(self, expert: int) -> tuple:
        e = int(expert)
        out = []
        for b in (self.weights.w1, self.weights.w3, self.weights.w2):
            out.append((b.data[e], b.scales[e]) if b.biases is None else (b.data[e], b.scales[e], b.biases[e]))
        return tuple(out)


class SharedExpert:
    """A resident bf16 shared expert in the role of the reference's
    ``shared_fn`` (mlx_runner.py:765-783): f32 SwiGLU with g <= 10 and u in
    [-10, 10], output cast to x.dtype.  ``moe_layer`` folds it into the fused
    decode kernel when the routed experts are resident too."""

    def __init__(self, w1: torch.Tensor, w3: torch.Tensor, w2: torch.Tensor, limit: float = 10.0):
        self.w1, self.w3, self.w2, self.limit = w1, w3, w2, limit

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        g = torch.clamp(xf @ self.w1.float().T, max=self.limit)
        u = torch.clamp(xf @ self.w3.float().T, -self.limit, self.limit)
        return ((g / (1.0 + torch.exp(-g)) * u) @ self.w2.float().T).to(x.dtype)


def _routed_only(weights: "MoEWeights", shared: SharedExpert | None, limit: float) -> "MoEWeights":
    sw = (shared.w1, shared.w3, shared.w2) if shared is not None else (None, None, None)
    return MoEWeights(weights.w1, weights.w3, weights.w2, *sw, limit, True)


def moe_layer(x: torch.Tensor, gate_w: torch.Tensor, gate_b: torch.Tensor | None, expert_fn, shared_fn,
              top_k: int = 6, limit: float = 10.0, trace_hook=None, layer_id: int = 0, prefetch_fn=None,
              union_budget: int = 0, route_stats: dict | None = None, union_strict: bool = False,
              pipeline: bool = False, async_submit_fn=None, async_finalize_fn=None, pinned_gather_fn=None,
              stack_gateup: bool = False, route_scale: float = 1.5) -> torch.Tensor:
    """Route (exact), routed experts, shared expert add (mlx_forward.py:257-419).

    Same arguments and semantics as the reference:
      * router: s = sqrt(softplus(x Wg^T)), top-k of s + gate_b, gates =
        s / (sum + 1e-20) * 1.5; ``trace_hook(layer_id, indices, weights)``
        gets the routing (slots in ascending biased-score order);
      * ``union_budget > 0`` with several rows caps the expert union
        (``cap_union``), accumulating the kept share in ``route_stats``;
      * ``expert_fn(e) -> (w1, w3, w2)`` operand tuples; per distinct expert,
        ascending: g = min(x W1^T, limit), u = clip(x W3^T, +-limit),
        h = silu(g) * u * gate (first slot of the row), out[rows] += h W2^T;
      * ``shared_fn(x)`` (None = no shared expert) is added in f32 after the
        routed sum; the result is cast to x.dtype.  x enters the experts as
        f32 (bf16 x exactly; f32 x is not rounded).
    With ``expert_fn`` a ``ResidentExperts`` (or ``MoEWeights``) and no
    ``pinned_gather_fn``, the routed loop and a ``SharedExpert`` run in the
    fused decode kernels (ds_moe_decode) instead of one qmm per expert.
    ``prefetch_fn(layer_id, experts)`` is called before the experts run.
    ``pipeline=True`` with ``async_submit_fn(layer, e) -> future of (operands
    dict, nbytes, was_hit, read_s, pack_s)`` and ``async_finalize_fn(layer,
    experts, saved)`` takes every expert's operands from its future and calls
    the finalize hook before the sorted scatter-add, as the reference's read
    pipeline does; the result equals the plain path.
    """
    import numpy as np

    H = x.shape[-1]
    x2 = require_cuda(x.reshape(-1, H), "x", (torch.bfloat16, torch.float32))
    T = x2.shape[0]
    gate_w = require_cuda(gate_w, "gate_w")
    scores = sqrtsoftplus_scores(x2, gate_w).contiguous()
    bias = gate_b if gate_b is not None else torch.zeros(gate_w.shape[0], device=x2.device)
    w_d, idx_d = route_topk(scores, bias, top_k, route_scale)
    w_d, idx_d = w_d.flip(-1).contiguous(), idx_d.flip(-1).contiguous()   # ascending, as the reference
    idx_np = idx_d.cpu().numpy().astype(np.int64)
    w_np = w_d.cpu().numpy().astype(np.float32)
    if union_budget > 0 and T > 1:
        idx_np, w_np, coverage = cap_union(idx_np, w_np, scores.shape[1], union_budget,
                                           scores=scores.cpu().numpy(), strict=union_strict)
        if route_stats is not None:
            route_stats["coverage"] += coverage * T
            route_stats["calls"] += T
        idx_d = torch.as_tensor(idx_np, dtype=torch.int32, device=x2.device)
        w_d = torch.as_tensor(w_np, device=x2.device)
    unique = np.unique(idx_np)
    unique = unique[unique >= 0]
    if prefetch_fn is not None:
        prefetch_fn(layer_id, [int(e) for e in unique])

    resident = expert_fn.weights if isinstance(expert_fn, ResidentExperts) else (
        expert_fn if isinstance(expert_fn, MoEWeights) else None)
    piped = pipeline and async_submit_fn is not None and async_finalize_fn is not None
    if resident is not None and pinned_gather_fn is None and not piped:
        fuse_shared = isinstance(shared_fn, SharedExpert) and shared_fn.limit == limit
        layer = _routed_only(resident, shared_fn if fuse_shared else None, limit)
        ids32 = idx_d.to(torch.int32).contiguous()
        # a shared expert computed apart is added to the unrounded routed sum
        f32_sum = shared_fn is not None and not fuse_shared and x2.dtype != torch.float32
        if f32_sum and resident.w1.fmt == _abi.DS_FMT_FP4:
            resident.prepare_tc()          # the f32-output decode kernels read the scale atoms
        out = torch.empty(x2.shape, dtype=torch.float32 if f32_sum else x2.dtype, device=x2.device)
        try:
            for r0 in range(0, T, MAX_DECODE_TOKENS):
                r1 = min(T, r0 + MAX_DECODE_TOKENS)
                moe_decode(x2[r0:r1], layer, ids32[r0:r1], w_d[r0:r1].contiguous(), out=out[r0:r1],
                           out_f32=f32_sum)
        except NotImplementedError:
            out = None                     # no unrounded-output kernel for this geometry: per-expert path
        if out is not None:
            if trace_hook is not None:
                trace_hook(layer_id, idx_np.tolist(), w_np.tolist())
            if shared_fn is not None and not fuse_shared:
                out = (out.float() + shared_fn(x2).float()).to(x2.dtype)
            return out.reshape(x.shape)

    if resident is not None:
        expert_fn = ResidentExperts(resident)
    shared_out = shared_fn(x2).float() if shared_fn is not None else None
    out = torch.zeros((T, H), dtype=torch.float32, device=x2.device)

    def contrib(e: int, ops):
        """rows routed to e (first slot each), and their weighted expert outputs."""
        mask = idx_np == e
        rows = np.nonzero(mask.any(axis=1))[0]
        cols = mask[rows].argmax(axis=1)
        rows_d = torch.as_tensor(rows, dtype=torch.int64, device=x2.device)
        g, u, w2 = gate_up_qmm(x2[rows_d].float(), ops, stack_single_row=stack_gateup)
        g = torch.clamp(g, max=limit)
        u = torch.clamp(u, -limit, limit)
        h = g / (1.0 + torch.exp(-g)) * u
        rw = torch.as_tensor(w_np[rows, cols], device=x2.device).reshape(-1, 1)
        return rows_d, qmm(h * rw, w2)

    if piped and pinned_gather_fn is None:
        # the reference's read pipeline: every expert's operands come from a
        # future, the caller's finalize hook runs before the sorted scatter-add
        futs = {int(e): async_submit_fn(layer_id, int(e)) for e in unique}
        saved = {}
        try:
            for e, fut in futs.items():
                ops, nbytes, was_hit, read_s, pack_s = fut.result()
                rows_d, c = contrib(e, ops)
                saved[e] = (rows_d.cpu().numpy(), c, ops, nbytes, was_hit, read_s, pack_s)
        except Exception:
            for fut in futs.values():
                if not fut.done():
                    fut.cancel()
            raise
        async_finalize_fn(layer_id, [int(e) for e in unique], saved)
        for e in unique:
            rows, c = saved[int(e)][:2]
            out.index_add_(0, torch.as_tensor(rows, dtype=torch.int64, device=x2.device), c)
    else:
        pinned = pinned_gather_fn(layer_id, x2, idx_np, w_np) if pinned_gather_fn is not None else {}
        for expert in unique:
            e = int(expert)
            if e in pinned:
                rows, c = pinned[e]
                out.index_add_(0, torch.as_tensor(rows, dtype=torch.int64, device=x2.device), c.float())
                continue
            rows_d, c = contrib(e, expert_fn(e))
            out.index_add_(0, rows_d, c)
    if trace_hook is not None:
        trace_hook(layer_id, idx_np.tolist(), w_np.tolist())
    if shared_out is not None:
        out = out + shared_out
    return out.to(x2.dtype).reshape(x.shape)


def _static_input(t: torch.Tensor | None, shape, dtype, device, name: str) -> torch.Tensor:
    if t is None:
        return torch.zeros(shape, dtype=dtype, device=device)
    if tuple(t.shape) != tuple(shape) or t.dtype != dtype or not t.is_contiguous() or t.device != device:
        raise ValueError(f"{name} must be a contiguous {tuple(shape)} {dtype} tensor on {device}")
    return t


_WAIT_EVENTS: dict = {}


@contextlib.contextmanager
def graph_capture(graph: torch.cuda.CUDAGraph):
    """``torch.cuda.graph(graph)`` with unreachable Python objects collected
    first and the cycle collector paused during the capture: a collection
    inside the capture could finalize an unreachable object that owns a CUDA
    graph or event, and those calls invalidate a capture."""
    gc.collect()
    was_enabled = gc.isenabled()
    gc.disable()
    try:
        with torch.cuda.graph(graph):
            yield
    finally:
        if was_enabled:
            gc.enable()


def wait_stream(device) -> None:
    """Wait for the current stream by polling an event (a decode step is tens
    of microseconds: a blocking synchronisation adds its own wake-up time).
    One event per device is reused."""
    device = torch.device(device)
    key = device.index if device.index is not None else torch.cuda.current_device()
    ev = _WAIT_EVENTS.get(key)
    if ev is None:
        ev = _WAIT_EVENTS[key] = torch.cuda.Event()
    ev.record(torch.cuda.current_stream(device))
    while not ev.query():
        pass


def host_device_pointer(t: torch.Tensor) -> int:
    """Device address of a pinned host tensor's storage (``ds_host_device_pointer``)."""
    if t.is_cuda or not t.is_pinned():
        raise ValueError("host_device_pointer needs a pinned host tensor")
    d = ctypes.c_void_p(0)
    _abi.call("ds_host_device_pointer", ctypes.c_void_p(t.data_ptr()), ctypes.byref(d))
    return int(d.value)


def copy_ranges(ranges: list[tuple[int, int, int]], device) -> None:
    """``ds_copy_ranges`` on the device's current stream: (dst, src, bytes)
    device addresses (pinned host memory through ``host_device_pointer``),
    up to four ranges in one launch.  A host-fed decode step stages its
    inputs and output with it instead of copy-engine transfers, whose
    per-copy latency dominates moves of a few kilobytes."""
    n = len(ranges)
    dst = (ctypes.c_void_p * n)(*[r[0] for r in ranges])
    src = (ctypes.c_void_p * n)(*[r[1] for r in ranges])
    nb = (ctypes.c_size_t * n)(*[r[2] for r in ranges])
    _abi.call("ds_copy_ranges", n, dst, src, nb, stream_handle(torch.device(device)))


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


class DecodeGraph:
    """Softmax top-k routing + ``moe_decode`` for one resident layer and a fixed
    token count, captured once into a CUDA graph over static device buffers.

    A decode loop writes the step's activations into ``x`` and router logits
    into ``logits`` (device copies, or host copies from pinned memory), calls
    ``replay()`` and reads ``out``: one graph launch per layer instead of the
    router + decode launches and their host-side argument handling.
    """

    def __init__(self, weights: MoEWeights, tokens: int, top_k: int, device: torch.device | str | None = None,
                 x: torch.Tensor | None = None, logits: torch.Tensor | None = None, host_io: bool = False):
        """``x`` [tokens, H] bf16 / ``logits`` [tokens, E] f32: input buffers to
        read (e.g. rows of a ``GraphChain`` staging tensor); allocated here if None.

        ``host_io``: pinned host buffers ``x_host``, ``logits_host`` and
        ``out_host``, copied in and out inside the graph: ``replay_host()`` is
        then one launch per token step, host data in, host data out."""
        device = torch.device(device) if device is not None else weights.w1.data.device
        self.weights, self.tokens, self.top_k = weights, tokens, top_k
        H, E = weights.hidden, weights.n_experts
        self.x = _static_input(x, (tokens, H), torch.bfloat16, device, "x")
        self.logits = _static_input(logits, (tokens, E), torch.float32, device, "logits")
        self.host_io = host_io
        if host_io:
            self.x_host = torch.zeros(tokens, H, dtype=torch.bfloat16).pin_memory()
            self.logits_host = torch.zeros(tokens, E, dtype=torch.float32).pin_memory()
            self.out_host = torch.zeros(tokens, H, dtype=torch.bfloat16).pin_memory()
        self.w = torch.empty(tokens, top_k, dtype=torch.float32, device=device)
        self.ids = torch.empty(tokens, top_k, dtype=torch.int32, device=device)
        self.out = torch.empty(tokens, H, dtype=torch.bfloat16, device=device)
        self.workspace = torch.zeros(weights.decode_workspace_bytes(tokens, top_k), dtype=torch.uint8, device=device)
        self._step()                      # first call outside the capture: module load, attributes, caches
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with graph_capture(self.graph):
            self._step()
        if host_io:
            # inputs staged by one small kernel (copy_ranges), not by
            # copy-engine transfers (they are a few KB); the layer writes its
            # output rows straight into out_host through its device mapping
            stage_in = [(self.x.data_ptr(), host_device_pointer(self.x_host), _nbytes(self.x)),
                        (self.logits.data_ptr(), host_device_pointer(self.logits_host), _nbytes(self.logits))]
            self.graph_host = torch.cuda.CUDAGraph()
            with graph_capture(self.graph_host):
                copy_ranges(stage_in, device)
                moe_decode_routed(self.x, self.weights, self.logits, self.top_k, out=self.out_host,
                                  route_out=(self.w, self.ids), workspace=self.workspace)

    def _step(self) -> None:
        moe_decode_routed(self.x, self.weights, self.logits, self.top_k, out=self.out, route_out=(self.w, self.ids),
                          workspace=self.workspace)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out

    def replay_host(self) -> torch.Tensor:
        """x_host / logits_host -> out_host in one graph launch (host_io=True);
        synchronises the stream and returns ``out_host``."""
        if not self.host_io:
            raise ValueError("DecodeGraph was built without host_io")
        self.graph_host.replay()
        wait_stream(self.x.device)
        return self.out_host


class GraphChain:
    """Several captured layers (``DecodeGraph`` or ``ep.PeerDecodeGraph``:
    objects with static ``x``, ``logits``, ``out`` buffers and ``_step()``)
    captured back to back into ONE CUDA graph: a decode step through many
    layers is one graph launch, the way a serving loop runs its layer stack.

    ``x [n, T, H]`` and ``logits [n, T, E]`` hold layer i's inputs at [i].
    Pass the stacked tensors whose rows the layers were built on (their
    ``x=`` / ``logits=`` arguments) and the graph reads them in place;
    without them the chain allocates its own and copies row i into layer i's
    buffers inside the graph.  ``replay()`` runs all n layers (layer i's
    output in ``layers[i].out``)."""

    def __init__(self, layers, x: torch.Tensor | None = None, logits: torch.Tensor | None = None):
        if not layers:
            raise ValueError("GraphChain needs at least one layer")
        self.layers = list(layers)
        n = len(self.layers)
        x0, l0 = self.layers[0].x, self.layers[0].logits
        in_place = x is not None and logits is not None
        if in_place:
            for i, layer in enumerate(self.layers):
                if layer.x.data_ptr() != x[i].data_ptr() or layer.logits.data_ptr() != logits[i].data_ptr():
                    raise ValueError(f"layer {i} does not read rows {i} of the given x / logits")
            self.x, self.logits = x, logits
        else:
            self.x = torch.zeros((n,) + tuple(x0.shape), dtype=x0.dtype, device=x0.device)
            self.logits = torch.zeros((n,) + tuple(l0.shape), dtype=l0.dtype, device=l0.device)
        torch.cuda.synchronize(x0.device)
        self.graph = torch.cuda.CUDAGraph()
        with graph_capture(self.graph):
            for i, layer in enumerate(self.layers):
                if not in_place:
                    layer.x.copy_(self.x[i])
                    layer.logits.copy_(self.logits[i])
                layer._step()

    def replay(self) -> None:
        self.graph.replay()
