"""Expert-parallel MoE layer: routed experts sharded over the ranks of a
process group (NCCL over NVLink on B200 ranks; the CPU tests drive the same
host logic over gloo).  Two exchange schemes:

* ``ExpertParallelMoE`` -- token rows dispatched to the owners of their
  experts and combined back with all-to-all (any batch size; below);
* ``ExpertParallelDecode`` -- for decode-sized batches (ranks x tokens <= 8):
  the tokens are all-gathered, every rank runs the fused decode layer over
  all of them restricted to its own experts (f32 partial outputs), the
  partials are reduce-scattered back to their home ranks, which add the
  shared expert.  Every rank streams only the weights of its own experts
  that the batch uses, i.e. about one decode layer's worth per rank.

Rank g owns global experts [g * E_l, (g + 1) * E_l), E_l = E / G; the shared
expert is replicated.  One layer step for the b tokens a rank holds (its
"home" tokens):

  1. dispatch: every (token, slot) pair with expert e goes to rank e // E_l,
     as 32-bit words: the activation row followed by (local expert id, route
     weight).  Two forms: counted -- the ranks first exchange how many rows
     each sends to each (one all_to_all of G counts, read on the host), then
     send exactly those rows with one uneven all_to_all_single; fixed
     capacity -- a block of b * k rows to every peer (unused rows carry
     expert -1), nothing read on the host, so the host queues the next
     layers while the GPU works (and a step could be captured in a CUDA
     graph), at up to G times the exchanged bytes.  ``fixed_capacity=None``
     (default) picks fixed capacity while G * b * k <= 1024 rows.
  2. experts: the owner runs its local experts over the received rows -- route
     weight applied before the down projection, SwiGLU clamp -- producing f32
     rows (GPU: ds_grouped_ffn with top_k = 1, rows of expert -1 skipped).
  3. combine: rows return with a second all_to_all_single; the home rank adds
     each token's k contributions in slot order, then the shared expert (its
     output rounded to the activation dtype first, as the reference does) and
     casts to the activation dtype.

A row's result does not depend on which other rows share its launch, so the
G-rank output equals the 1-rank output bit for bit.  The layer contract is
moe_layer's (src/deepseeker/mlx_forward.py:388-419, shared add
src/deepseeker/mlx_runner.py:776-781); the reference itself runs on one device.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

# the fixed-capacity exchange is used up to this many rows (G * b * k) when not chosen explicitly
FIXED_CAPACITY_ROWS = 1024

# local_ffn(x_rows [R, H] (activation dtype), expert [R] int32 (-1 = none), gate [R] f32) -> f32 [R, H]
LocalFFN = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]
# shared_fn(x [b, H]) -> f32 [b, H], already rounded to the activation dtype
SharedFn = Callable[[torch.Tensor], torch.Tensor]


class ExpertParallelMoE:
    def __init__(self, n_experts: int, top_k: int, local_ffn: LocalFFN, shared_fn: SharedFn | None = None,
                 group: dist.ProcessGroup | None = None, fixed_capacity: bool | None = None):
        self.fixed_capacity = fixed_capacity
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not shard over {self.world} ranks")
        self.n_experts = n_experts
        self.local_experts = n_experts // self.world
        self.first_expert = self.rank * self.local_experts
        self.top_k = top_k
        self.local_ffn = local_ffn
        self.shared_fn = shared_fn

    # -- packing: [rows, H] activations + (expert int32, gate f32) as int32 words
    @staticmethod
    def _pack(x: torch.Tensor, expert: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
        words = x.contiguous().view(torch.uint8).view(x.shape[0], -1).view(torch.int32)
        meta = torch.stack([expert.to(torch.int32), gate.to(torch.float32).view(torch.int32)], dim=1)
        return torch.cat([words, meta], dim=1)

    @staticmethod
    def _unpack(buf: torch.Tensor, dtype: torch.dtype, H: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        n = buf.shape[1] - 2
        x = buf[:, :n].contiguous().view(torch.uint8).view(buf.shape[0], -1).view(dtype)
        expert = buf[:, n].contiguous()
        gate = buf[:, n + 1].contiguous().view(torch.float32)
        return x[:, :H], expert, gate

    def _all_to_all(self, out: torch.Tensor, inp: torch.Tensor, out_splits=None, in_splits=None) -> None:
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits,
                                   group=self.group)

    def dispatch_plan(self, ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(dest rank, slot index inside the block for that rank, valid) per pair, [b*k] each."""
        flat = ids.reshape(-1).to(torch.int64)
        valid = flat >= 0
        dest = torch.where(valid, flat // self.local_experts, torch.zeros_like(flat))
        onehot = torch.zeros(flat.shape[0], self.world, dtype=torch.int64, device=ids.device)
        onehot.scatter_(1, dest[:, None], valid[:, None].to(torch.int64))   # no host-side bounds check
        index = (torch.cumsum(onehot, dim=0) - 1).gather(1, dest[:, None]).view(-1)
        return dest, index, valid

    def forward(self, x: torch.Tensor, ids: torch.Tensor, gates: torch.Tensor) -> torch.Tensor:
        """x [b, H], ids [b, k] global expert ids (-1 = dropped slot), gates [b, k] -> [b, H] of x.dtype."""
        if (x.shape[1] * x.element_size()) % 4:
            raise ValueError("rows must be a whole number of 32-bit words")
        fixed = self.fixed_capacity
        if fixed is None:
            fixed = self.world * ids.numel() <= FIXED_CAPACITY_ROWS
        return self._forward_fixed(x, ids, gates) if fixed else self._forward_counted(x, ids, gates)

    @staticmethod
    def _combine(back: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
        """Each token's k contributions (rows of `back`, src [b, k]) summed in slot order."""
        acc = back[src[:, 0]]
        for s_ in range(1, src.shape[1]):
            acc = acc + back[src[:, s_]]
        return acc

    def _forward_counted(self, x: torch.Tensor, ids: torch.Tensor, gates: torch.Tensor) -> torch.Tensor:
        """Exact-size exchange: counts first, then only the routed rows."""
        b, H = x.shape
        k = ids.shape[1]
        G = self.world
        flat = ids.reshape(-1).to(torch.int64)
        valid = flat >= 0
        dest = torch.where(valid, flat // self.local_experts, torch.full_like(flat, G))   # G: dropped
        order = torch.sort(dest, stable=True).indices          # pairs grouped by owner, pair order kept
        counts = torch.bincount(dest, minlength=G + 1)[:G]
        recv_counts = torch.empty_like(counts)
        self._all_to_all(recv_counts, counts)
        host = torch.cat([counts, recv_counts]).cpu().tolist()   # the one host read of the step
        send_c, recv_c = host[:G], host[G:]
        n_send, n_recv = sum(send_c), sum(recv_c)
        sel = order[:n_send]
        token = sel // k
        rows = self._pack(x[token], flat[sel] - dest[sel] * self.local_experts, gates.reshape(-1)[sel])
        words = rows.shape[1]
        recv = torch.empty(n_recv, words, dtype=torch.int32, device=x.device)
        self._all_to_all(recv, rows, recv_c, send_c)
        if n_recv:
            rx, rexp, rgate = self._unpack(recv, x.dtype, H)
            y = self.local_ffn(rx, rexp, rgate)
            if y.dtype != torch.float32 or y.shape != (n_recv, H):
                raise ValueError("local_ffn must return f32 [rows, H]")
        else:
            y = torch.empty(0, H, dtype=torch.float32, device=x.device)
        back = torch.empty(n_send + 1, H, dtype=torch.float32, device=x.device)
        back[n_send].zero_()
        self._all_to_all(back[:n_send], y.contiguous(), send_c, recv_c)
        # pair -> its row in send order (dropped pairs -> the zero row), then
        # each token's k contributions in slot order
        src = torch.full((b * k,), n_send, dtype=torch.int64, device=x.device)
        src[sel] = torch.arange(n_send, device=x.device)
        acc = self._combine(back, src.view(b, k))
        if self.shared_fn is not None:
            acc = acc + self.shared_fn(x)
        return acc.to(x.dtype)

    def _forward_fixed(self, x: torch.Tensor, ids: torch.Tensor, gates: torch.Tensor) -> torch.Tensor:
        b, H = x.shape
        k = ids.shape[1]
        cap = b * k
        G = self.world
        dest, index, valid = self.dispatch_plan(ids)
        flat = ids.reshape(-1).to(torch.int64)
        token = torch.arange(cap, device=x.device) // k
        # 1. dispatch (no host read: every pair is written, dropped ones to a
        # spare row past the blocks)
        words = H * x.element_size() // 4
        send = torch.zeros(G * cap + 1, words + 2, dtype=torch.int32, device=x.device)
        send[:, words] = -1  # expert -1: unused row
        slot = torch.where(valid, dest * cap + index, torch.full_like(dest, G * cap))
        send[slot] = self._pack(x[token], torch.where(valid, flat - dest * self.local_experts, -1),
                                gates.reshape(-1))
        send = send[:G * cap]
        recv = torch.empty_like(send)
        self._all_to_all(recv, send)
        # 2. local experts
        rx, rexp, rgate = self._unpack(recv, x.dtype, H)
        y = self.local_ffn(rx, rexp, rgate)
        if y.dtype != torch.float32 or y.shape != (G * cap, H):
            raise ValueError("local_ffn must return f32 [rows, H]")
        back = torch.empty(G * cap + 1, H, dtype=torch.float32, device=x.device)
        back[G * cap].zero_()
        self._all_to_all(back[:G * cap], y.contiguous())
        # 3. combine in slot order (+ shared), cast
        acc = self._combine(back, slot.view(b, k))
        if self.shared_fn is not None:
            acc = acc + self.shared_fn(x)
        return acc.to(x.dtype)

    __call__ = forward


# ---------------------------------------------------------------- GPU defaults

def gpu_local_ffn(local_layer) -> LocalFFN:
    """Owner-side expert FFN on the B200 kernels: FP4 and q3 shards both run
    ds_grouped_ffn (top_k = 1, f32 rows), so every local expert's weights
    stream once per call whatever the number of rows routed to it."""
    from . import grouped

    ffn = grouped.GroupedFFN(local_layer, 1)

    def run(xr, expert, gate):
        return ffn(xr.to(torch.bfloat16).contiguous(), expert.view(-1, 1).contiguous(),
                   gate.view(-1, 1).contiguous(), route_before_down=True, out_dtype=torch.float32)
    return run


def shared_dense(w1: torch.Tensor, w3: torch.Tensor, w2: torch.Tensor, x: torch.Tensor,
                 limit: float = 10.0) -> torch.Tensor:
    """Shared expert for a batch of rows as plain bf16 GEMMs (cuBLAS, f32
    output): g = min(x W1^T, L), u = clip(x W3^T, +-L), h = silu(g) u in f32,
    then h W2^T with h split into bf16 hi + lo (16 significant bits), so the
    weights stream once for the whole batch.  Returns f32 [b, H], rounded to
    x's dtype first as the reference does (mlx_runner.py:776-781)."""
    xb = x.to(torch.bfloat16)
    g = torch.mm(xb, w1.t(), out_dtype=torch.float32).clamp_(max=limit)
    u = torch.mm(xb, w3.t(), out_dtype=torch.float32).clamp_(-limit, limit)
    h = g / (1.0 + torch.exp(-g)) * u
    hi = h.to(torch.bfloat16)
    lo = (h - hi.float()).to(torch.bfloat16)
    y = torch.mm(hi, w2.t(), out_dtype=torch.float32) + torch.mm(lo, w2.t(), out_dtype=torch.float32)
    return y.to(x.dtype).float()


def gpu_shared_fn(local_layer) -> SharedFn | None:
    """Shared expert: up to 8 rows on the fused decode kernels (no routed
    slot); more rows as one set of bf16 GEMMs (``shared_dense``), so the
    shared weights stream once per call, not once per 8 rows.  f32 math,
    output rounded to the activation dtype before it is added."""
    from . import moe

    if local_layer.shared_w1 is None:
        return None
    w1, w3, w2 = local_layer.shared_w1, local_layer.shared_w3, local_layer.shared_w2

    def run(x):
        b, H = x.shape
        if b > moe.MAX_DECODE_TOKENS:
            return shared_dense(w1, w3, w2, x)
        ids = torch.full((b, 1), -1, dtype=torch.int32, device=x.device)
        w = torch.zeros(b, 1, dtype=torch.float32, device=x.device)
        return moe.moe_decode(x.float().contiguous(), local_layer, ids, w).to(x.dtype).float()
    return run


def gpu_layer(local_layer, n_experts: int, top_k: int, group=None) -> ExpertParallelMoE:
    """ExpertParallelMoE over this rank's shard `local_layer` (global experts
    [rank * E_l, (rank + 1) * E_l) as built with synthetic.make_layer(expert_offset=...))."""
    return ExpertParallelMoE(n_experts, top_k, gpu_local_ffn(local_layer), gpu_shared_fn(local_layer), group)


# ---------------------------------------------------------------- decode-sized batches

# local_partial(x_all [G*b, H], ids_local [G*b, k] (-1 = not this rank's), gates [G*b, k]) -> f32 [G*b, H]
LocalPartial = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


class ExpertParallelDecode:
    def __init__(self, n_experts: int, top_k: int, local_partial: LocalPartial, shared_fn: SharedFn | None = None,
                 group: dist.ProcessGroup | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not shard over {self.world} ranks")
        self.n_experts, self.top_k = n_experts, top_k
        self.local_experts = n_experts // self.world
        self.first_expert = self.rank * self.local_experts
        self.local_partial, self.shared_fn = local_partial, shared_fn
        self._nccl = dist.is_initialized() and dist.get_backend(group) == "nccl"

    def _gather(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t
        out = torch.empty((self.world * t.shape[0], *t.shape[1:]), dtype=t.dtype, device=t.device)
        if self._nccl:
            dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        else:
            dist.all_gather(list(out.chunk(self.world)), t.contiguous(), group=self.group)
        return out

    def _reduce_scatter(self, t: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return t
        b = t.shape[0] // self.world
        if self._nccl:
            out = torch.empty((b, *t.shape[1:]), dtype=t.dtype, device=t.device)
            dist.reduce_scatter_tensor(out, t.contiguous(), group=self.group)
            return out
        t = t.contiguous().clone()
        dist.all_reduce(t, group=self.group)
        return t[self.rank * b:(self.rank + 1) * b].contiguous()

    def forward(self, x: torch.Tensor, ids: torch.Tensor, gates: torch.Tensor) -> torch.Tensor:
        """x [b, H] (same b on every rank), ids [b, k] global ids (-1 = dropped), gates [b, k] -> [b, H] of x.dtype."""
        b, H = x.shape
        k = ids.shape[1]
        # one gather of 32-bit words per token: activations, ids, gates
        words = (H * x.element_size()) // 4
        row = torch.cat([x.contiguous().view(torch.uint8).view(b, -1).view(torch.int32), ids.to(torch.int32),
                         gates.to(torch.float32).view(torch.int32)], dim=1)
        rg = self._gather(row)
        xg = rg[:, :words].contiguous().view(torch.uint8).view(rg.shape[0], -1).view(x.dtype)
        ig = rg[:, words:words + k].contiguous()
        gg = rg[:, words + k:].contiguous().view(torch.float32)
        mine = (ig >= self.first_expert) & (ig < self.first_expert + self.local_experts)
        il = torch.where(mine, ig - self.first_expert, torch.full_like(ig, -1))
        part = self.local_partial(xg, il, gg)
        if part.dtype != torch.float32 or part.shape != xg.shape:
            raise ValueError("local_partial must return f32 [rows, H]")
        acc = self._reduce_scatter(part)
        if self.shared_fn is not None:
            acc = acc + self.shared_fn(x)
        return acc.to(x.dtype)

    __call__ = forward


def gpu_decode_layer(local_layer, n_experts: int, top_k: int, group=None,
                     shared_rank: int | None = None) -> ExpertParallelDecode:
    """ExpertParallelDecode on the decode kernels: routed partials in f32 from
    this rank's FP4 shard (scale atoms prepared).

    ``shared_rank=None``: every rank evaluates the shared expert for its own
    tokens after the reduce-scatter (gpu_shared_fn).  ``shared_rank=r``: rank
    r evaluates it for every gathered token inside its routed decode call (its
    output is rounded to bf16 before it joins the f32 partial, the reference's
    order) and the reduce-scatter adds it to each token exactly once; the
    other ranks skip it."""
    from . import moe

    local_layer.prepare_tc()
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    shared_fn = None
    if shared_rank is None:
        shared_fn = gpu_shared_fn(local_layer)
    if (shared_rank is not None and rank == shared_rank) or local_layer.shared_w1 is None:
        layer = local_layer
    else:
        layer = moe.MoEWeights(local_layer.w1, local_layer.w3, local_layer.w2, swiglu_limit=local_layer.swiglu_limit,
                               route_before_down=local_layer.route_before_down)

    def local_partial(xg, il, gg):
        out = torch.empty(xg.shape, dtype=torch.float32, device=xg.device)
        for r0 in range(0, xg.shape[0], moe.MAX_DECODE_TOKENS):
            r1 = min(xg.shape[0], r0 + moe.MAX_DECODE_TOKENS)
            moe.moe_decode(xg[r0:r1], layer, il[r0:r1], gg[r0:r1], out=out[r0:r1], out_f32=True)
        return out
    return ExpertParallelDecode(n_experts, top_k, local_partial, shared_fn, group)


# ---------------------------------------------------------------- decode over peer memory (native exchange)

class PeerComm:
    """ds_ep_* communicator: one device region per rank, mapped into every
    rank through CUDA IPC; the library's own kernels move the token rows and
    partial outputs over NVLink, so a decode step contains no collective call
    and captures into a CUDA graph (``PeerDecodeGraph``).

    Setup uses the process group once (handle exchange, barrier).  Device
    waits give up after ``timeout_ms``; ``status()`` then reports bit 2 and
    later exchanges of this communicator return at once."""

    def __init__(self, max_rows: int, hidden: int, top_k: int, group=None, timeout_ms: int = 5000,
                 _local: tuple[int, int] | None = None):
        import ctypes

        from . import _abi

        self.group = group
        if _local is not None:
            self.world, self.rank = _local
        else:
            self.world = dist.get_world_size(group) if dist.is_initialized() else 1
            self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.max_rows, self.hidden, self.top_k = max_rows, hidden, top_k
        self.device = torch.device("cuda", torch.cuda.current_device())
        h = ctypes.c_void_p()
        _abi.call("ds_ep_create", self.world, self.rank, max_rows, hidden, top_k, timeout_ms, ctypes.byref(h))
        self._h = h
        if _local is not None:
            return                       # connected by local_group
        try:
            buf = ctypes.create_string_buffer(64)
            _abi.call("ds_ep_ipc_handle", h, buf)
            handles = [bytes(buf.raw)]
            if self.world > 1:
                handles = [None] * self.world
                dist.all_gather_object(handles, bytes(buf.raw), group=group)
            joined = ctypes.create_string_buffer(b"".join(handles), 64 * self.world)
            _abi.call("ds_ep_connect", h, joined)
            if self.world > 1:
                dist.barrier(group)      # nobody writes into a peer before it has connected
        except Exception:
            self.close()
            raise

    @classmethod
    def local_group(cls, devices: list, max_rows: int, hidden: int, top_k: int,
                    timeout_ms: int = 5000) -> list["PeerComm"]:
        """Communicators of all ranks in THIS process, rank i on devices[i]
        (ds_ep_connect_peers).  Ranks that share a device must never wait on
        each other; that form only serves tests of the bounded waits."""
        import ctypes

        from . import _abi

        n = len(devices)
        comms = []
        for i, d in enumerate(devices):
            with torch.cuda.device(torch.device(d)):
                comms.append(cls(max_rows, hidden, top_k, timeout_ms=timeout_ms, _local=(n, i)))
        arr = (ctypes.c_void_p * n)(*[c.handle.value for c in comms])
        for c in comms:
            with torch.cuda.device(c.device):
                _abi.call("ds_ep_connect_peers", c.handle, arr)
        return comms

    @property
    def handle(self):
        if self._h is None:
            raise ValueError("communicator is closed")
        return self._h

    def status(self) -> int:
        import ctypes

        from . import _abi

        v = ctypes.c_int32(0)
        _abi.call("ds_ep_status", self.handle, ctypes.byref(v))
        return v.value

    def close(self) -> None:
        from . import _abi

        if getattr(self, "_h", None) is not None:
            torch.cuda.synchronize(self.device)
            h, self._h = self._h, None
            _abi.call("ds_ep_destroy", h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PeerDecodeLayer:
    """One layer of expert-parallel decode on ``PeerComm``: this rank's FP4
    (scale atoms prepared here) or q3 shard ``local_layer`` (global experts
    [rank * E_l, (rank + 1) * E_l)), ``rows`` tokens per rank and step.

    ``layer(x [rows, H] bf16, ids [rows, k] int32 global, gates [rows, k] f32)``
    -> [rows, H] bf16: all ranks' routed experts plus the shared expert, the
    layer contract of moe_layer (src/deepseeker/mlx_forward.py:388-419).
    Every rank calls its layers in the same order."""

    def __init__(self, comm: PeerComm, local_layer, n_experts: int, top_k: int, rows: int):
        import ctypes

        from . import _abi

        if n_experts % comm.world:
            raise ValueError(f"{n_experts} experts do not shard over {comm.world} ranks")
        if local_layer.n_experts != n_experts // comm.world:
            raise ValueError("local_layer must hold n_experts / world experts")
        if not 1 <= rows <= comm.max_rows or top_k != comm.top_k or local_layer.hidden != comm.hidden:
            raise ValueError("rows / top_k / hidden do not match the communicator")
        local_layer.prepare_tc()
        self.comm, self.layer, self.rows, self.top_k = comm, local_layer, rows, top_k
        self.first_expert = comm.rank * local_layer.n_experts
        self.desc = local_layer.cached_desc(top_k)
        c = ctypes.c_size_t(0)
        _abi.call("ds_ep_decode_workspace_size", comm.handle, ctypes.byref(self.desc), rows, ctypes.byref(c))
        self.workspace = torch.zeros(c.value, dtype=torch.uint8, device=comm.device)

    def __call__(self, x: torch.Tensor, ids: torch.Tensor, gates: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        import ctypes

        from . import _abi
        from ._dev import ptr, stream_handle

        b, k = self.rows, self.top_k
        H = self.comm.hidden
        if x.shape != (b, H) or x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise ValueError(f"x must be a contiguous [{b}, {H}] bf16 tensor")
        if ids.shape != (b, k) or ids.dtype != torch.int32 or not ids.is_contiguous():
            raise ValueError(f"ids must be a contiguous [{b}, {k}] int32 tensor")
        if gates.shape != (b, k) or gates.dtype != torch.float32 or not gates.is_contiguous():
            raise ValueError(f"gates must be a contiguous [{b}, {k}] f32 tensor")
        if out is None:
            out = torch.empty(b, H, dtype=torch.bfloat16, device=x.device)
        _abi.call("ds_ep_decode", self.comm.handle, ctypes.byref(self.desc), self.first_expert, ptr(x), b, ptr(ids),
                  ptr(gates), ptr(out), ptr(self.workspace), self.workspace.numel(), stream_handle(x.device))
        return out


class PeerDecodeGraph:
    """Softmax top-k routing + ``PeerDecodeLayer`` captured into one CUDA graph
    over static buffers (``x``, ``logits`` in; ``out`` out).  The exchange is
    the library's own kernels, so the graph holds no collective call; every
    rank must replay its graphs in the same order."""

    def __init__(self, layer: PeerDecodeLayer, x: torch.Tensor | None = None, logits: torch.Tensor | None = None,
                 host_io: bool = False):
        from . import moe

        self.layer = layer
        b, k, H = layer.rows, layer.top_k, layer.comm.hidden
        E = layer.layer.n_experts * layer.comm.world
        dev = layer.comm.device
        self.x = moe._static_input(x, (b, H), torch.bfloat16, dev, "x")
        self.logits = moe._static_input(logits, (b, E), torch.float32, dev, "logits")
        self.host_io = host_io
        if host_io:
            self.x_host = torch.zeros(b, H, dtype=torch.bfloat16).pin_memory()
            self.logits_host = torch.zeros(b, E, dtype=torch.float32).pin_memory()
            self.out_host = torch.zeros(b, H, dtype=torch.bfloat16).pin_memory()
        self.w = torch.empty(b, k, dtype=torch.float32, device=dev)
        self.ids = torch.empty(b, k, dtype=torch.int32, device=dev)
        self.out = torch.empty(b, H, dtype=torch.bfloat16, device=dev)
        self._step()                      # eager once on every rank (the exchange pairs up)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with moe.graph_capture(self.graph):
            self._step()
        if host_io:
            # staging by one small kernel each way (moe.copy_ranges), not by
            # copy-engine transfers: the inputs and output are a few KB
            stage_in = [(self.x.data_ptr(), moe.host_device_pointer(self.x_host), moe._nbytes(self.x)),
                        (self.logits.data_ptr(), moe.host_device_pointer(self.logits_host), moe._nbytes(self.logits))]
            stage_out = [(moe.host_device_pointer(self.out_host), self.out.data_ptr(), moe._nbytes(self.out))]
            self.graph_host = torch.cuda.CUDAGraph()
            with moe.graph_capture(self.graph_host):
                moe.copy_ranges(stage_in, dev)
                self._step()
                moe.copy_ranges(stage_out, dev)

    def _step(self) -> None:
        from . import moe

        moe.route_softmax_topk(self.logits, self.layer.top_k, out=(self.w, self.ids))
        self.layer(self.x, self.ids, self.w, out=self.out)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out

    def replay_host(self) -> torch.Tensor:
        """x_host / logits_host -> out_host in one graph launch (host_io=True),
        waited for; returns ``out_host``."""
        from . import moe

        if not self.host_io:
            raise ValueError("PeerDecodeGraph was built without host_io")
        self.graph_host.replay()
        moe.wait_stream(self.x.device)
        return self.out_host
