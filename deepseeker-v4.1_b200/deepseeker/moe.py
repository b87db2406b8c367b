"""Routed-expert MoE layer on B200 -- the MoE subset of the reference's ``deepseeker.mlx_forward``.

Reference: src/deepseeker/mlx_forward.py:62-419 (router, qmm, moe_layer) and
src/deepseeker/mlx_runner.py:765-783 (shared expert).  Experts are held
resident in HBM as stacked banks (``ExpertBank``: [E, N, ...] in the
checkpoint's FP4 layout, or the build's 3-bit layout) instead of being
streamed from SSD through a cache, so ``expert_fn`` / prefetch / pipeline /
union-cap arguments of the reference have no counterpart here.

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

import ctypes
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
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = ws
    return ws


def decode_workspace_bytes(weights: MoEWeights, tokens: int, top_k: int) -> int:
    return weights.decode_workspace_bytes(tokens, top_k)


def moe_decode(x: torch.Tensor, weights: MoEWeights, topk_ids: torch.Tensor, topk_w: torch.Tensor,
               out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
               out_f32: bool = False) -> torch.Tensor:
    """Fused routed-expert MoE for up to 8 tokens: x [T, H] bf16 (or f32) -> [T, H] of x's dtype.

    topk_ids [T, k] int32 (-1 = dropped slot), topk_w [T, k] f32.  out_f32
    (bf16 x, FP4 banks with prepared scale atoms): f32 output without the final
    rounding, for partial sums that are added across ranks.
    """
    x = require_cuda(x, "x", (torch.bfloat16, torch.float32))
    if x.dim() != 2 or x.shape[1] != weights.hidden:
        raise ValueError(f"x must be [T, {weights.hidden}]")
    T = x.shape[0]
    if not 1 <= T <= MAX_DECODE_TOKENS:
        raise ValueError(f"moe_decode handles 1..{MAX_DECODE_TOKENS} tokens, got {T}")
    topk_ids = require_cuda(topk_ids, "topk_ids", torch.int32)
    topk_w = require_cuda(topk_w, "topk_w", torch.float32)
    k = topk_ids.shape[1]
    if topk_ids.shape != (T, k) or topk_w.shape != (T, k):
        raise ValueError("topk_ids / topk_w must be [T, k]")
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
    _abi.call("ds_moe_decode", ctypes.byref(d), ptr(x), xdt, T, ptr(topk_ids), ptr(topk_w), ptr(out), ptr(ws),
              ws.numel() * ws.element_size(), stream_handle(x.device))
    return out


def moe_layer(x: torch.Tensor, gate_w: torch.Tensor, gate_b: torch.Tensor | None, weights: MoEWeights,
              top_k: int = 6, limit: float = 10.0, trace_hook=None, layer_id: int = 0,
              route_scale: float = 1.5, **unsupported) -> torch.Tensor:
    """MoE layer: sqrt-softplus router (exact), routed experts, shared expert add.

    Mirrors ``moe_layer`` (mlx_forward.py:257-419) with resident banks in place
    of ``expert_fn``; ``trace_hook(layer, indices, weights)`` receives the
    routing like the reference.  Token counts above the fused decode limit are
    processed in groups of 8 rows (the grouped tensor-core path serves large
    batches through ``grouped``).
    """
    bad = {k for k, v in unsupported.items() if v not in (None, False, 0)}
    if bad:
        raise NotImplementedError(f"moe_layer: SSD-paging options {sorted(bad)} have no counterpart "
                                  "(experts are resident in HBM)")
    if limit != weights.swiglu_limit:
        weights = MoEWeights(weights.w1, weights.w3, weights.w2, weights.shared_w1, weights.shared_w3,
                             weights.shared_w2, limit, weights.route_before_down)
    x2 = x.reshape(-1, x.shape[-1])
    logits = (x2.float() @ gate_w.float().T).contiguous()
    w, idx = route_sqrtsoftplus(logits, gate_b, top_k, route_scale)
    if trace_hook is not None:
        trace_hook(layer_id, idx.cpu().tolist(), w.cpu().tolist())
    xb = x2.to(torch.bfloat16).contiguous()
    out = torch.empty_like(xb)
    for r0 in range(0, xb.shape[0], MAX_DECODE_TOKENS):
        r1 = min(xb.shape[0], r0 + MAX_DECODE_TOKENS)
        moe_decode(xb[r0:r1], weights, idx[r0:r1].contiguous(), w[r0:r1].contiguous(), out=out[r0:r1])
    return out.reshape(x.shape).to(x.dtype)


def _static_input(t: torch.Tensor | None, shape, dtype, device, name: str) -> torch.Tensor:
    if t is None:
        return torch.zeros(shape, dtype=dtype, device=device)
    if tuple(t.shape) != tuple(shape) or t.dtype != dtype or not t.is_contiguous() or t.device != device:
        raise ValueError(f"{name} must be a contiguous {tuple(shape)} {dtype} tensor on {device}")
    return t


def wait_stream(device) -> None:
    """Wait for the current stream by polling an event (a decode step is tens
    of microseconds: a blocking synchronisation adds its own wake-up time)."""
    ev = torch.cuda.Event()
    ev.record(torch.cuda.current_stream(device))
    while not ev.query():
        pass


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
        self.workspace = torch.empty(weights.decode_workspace_bytes(tokens, top_k), dtype=torch.uint8, device=device)
        self._step()                      # first call outside the capture: module load, attributes, caches
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        if host_io:
            self.graph_host = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph_host):
                self.x.copy_(self.x_host, non_blocking=True)
                self.logits.copy_(self.logits_host, non_blocking=True)
                self._step()
                self.out_host.copy_(self.out, non_blocking=True)

    def _step(self) -> None:
        route_softmax_topk(self.logits, self.top_k, out=(self.w, self.ids))
        moe_decode(self.x, self.weights, self.ids, self.w, out=self.out, workspace=self.workspace)

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
        with torch.cuda.graph(self.graph):
            for i, layer in enumerate(self.layers):
                if not in_place:
                    layer.x.copy_(self.x[i])
                    layer.logits.copy_(self.logits[i])
                layer._step()

    def replay(self) -> None:
        self.graph.replay()
