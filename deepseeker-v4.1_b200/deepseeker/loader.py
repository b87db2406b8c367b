"""Checkpoint -> resident expert banks: the on-disk side of the decode path.

Reference: the tensor manifest convention of scripts/build_model_manifest.py
(tests/test_manifest.py:30-63: every tensor entry carries its shard and a
``file_range`` = 8 + header_len + the safetensors ``data_offsets``), the q3
payload entries written by scripts/requant_experts_3bit.py:193-225 (weight
dtype ``U32_Q3_AFFINE`` [rows, words], ``F16`` scale and bias [rows, groups],
file_range = payload offsets), and ``ExpertLoader`` /
``load_expert_banks`` (src/deepseeker/mlx_weights.py:221-356, 576-649):
tensors are found by name (``layers.{L}.ffn.experts.{e}.{w1,w2,w3}.{weight,
scale[,bias]}``), one expert's weight / scale / bias ranges are merged into
contiguous runs (one read each), and a layer's experts are stacked into one
bank per projection.

Here a bank lands in device memory as an ``ExpertBank`` (FP4: packed codes
[E, N, K/2] + ue8m0 scales [E, N, K/32], the tensor-core scale atoms built on
the device; q3: u32 words + f16 scales / biases): every expert is read
straight into one pinned host staging buffer per tensor, then one
host->device copy per tensor.  The shared expert
(``layers.{L}.ffn.shared_experts.{w1,w2,w3}``) is made resident as bf16; an
FP8 (e4m3 with 32x32 ue8m0 block scales) shared expert is dequantised on the
device (``ds_fp8_block_dequant``), the reference's resident-dequantised
shared expert (mlx_runner.py:765-783).
"""
from __future__ import annotations

import json
import os
import struct
import threading
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

from . import _abi
from ._dev import ptr, stream_handle
from .moe import ExpertBank, MoEWeights

ROLES = ("w1", "w2", "w3")

# bytes per element of the safetensors / manifest dtypes this path reads
_DTYPE_BYTES = {"I8": 1, "U8": 1, "F8_E8M0": 1, "F8_E4M3": 1, "F16": 2, "BF16": 2, "F32": 4, "U32_Q3_AFFINE": 4}


# ------------------------------------------------------------------ safetensors / manifest

def parse_safetensors_header(path: Path | str) -> tuple[int, dict]:
    """(header_len, {name: {dtype, shape, data_offsets}}) of one safetensors file
    (8-byte little-endian header length, JSON header; ``__metadata__`` skipped)."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file (short header length)")
        (n,) = struct.unpack("<Q", raw)
        body = f.read(n)
    if len(body) != n:
        raise ValueError(f"{path}: truncated safetensors header")
    header = json.loads(body)
    header.pop("__metadata__", None)
    return n, header


def manifest_from_shards(model_root: Path | str, shards: list[str]) -> dict:
    """Tensor manifest ``{"tensors": [{name, shard, dtype, shape, bytes,
    data_range, file_range}]}`` of safetensors shards under ``model_root``."""
    tensors = []
    for shard in shards:
        n, header = parse_safetensors_header(Path(model_root) / shard)
        for name, e in header.items():
            a, b = e["data_offsets"]
            tensors.append({"name": name, "shard": shard, "dtype": e["dtype"], "shape": list(e["shape"]),
                            "bytes": b - a, "data_range": [a, b], "file_range": [8 + n + a, 8 + n + b]})
    return {"tensors": tensors}


_FD_CACHE: dict[tuple[str, str], int] = {}
_FD_LOCK = threading.Lock()


def _fd(model_root: Path, shard: str) -> int:
    key = (str(model_root), shard)
    fd = _FD_CACHE.get(key)
    if fd is None:
        with _FD_LOCK:
            fd = _FD_CACHE.get(key)
            if fd is None:
                fd = os.open(Path(model_root) / shard, os.O_RDONLY)
                _FD_CACHE[key] = fd
    return fd


def read_bytes(model_root: Path | str, shard: str, start: int, end: int) -> bytes:
    """Bytes [start, end) of a shard (positional read; raises on a short read)."""
    data = os.pread(_fd(Path(model_root), shard), end - start, start)
    if len(data) != end - start:
        raise RuntimeError(f"short read {shard}@{start}")
    return data


def read_into(model_root: Path | str, shard: str, start: int, target) -> int:
    """Read a shard range straight into a writable C-contiguous buffer."""
    view = memoryview(target)
    if view.readonly or not view.c_contiguous:
        raise ValueError("read target must be writable and C-contiguous")
    view = view.cast("B")
    fd = _fd(Path(model_root), shard)
    done = 0
    while done < view.nbytes:
        n = os.preadv(fd, [view[done:]], start + done)
        if n <= 0:
            raise RuntimeError(f"short read {shard}@{start + done}")
        done += n
    return done


# ------------------------------------------------------------------ loader

class ExpertLoader:
    """Manifest-addressed expert tensors -> resident device banks."""

    def __init__(self, model_root: Path | str, manifest: dict, io_threads: int = 16) -> None:
        self._root = Path(model_root)
        self._by_name = {t["name"]: t for t in manifest.get("tensors", [])}
        self._pool = ThreadPoolExecutor(max_workers=io_threads, thread_name_prefix="expert-io")
        self._run_cache: dict[tuple[str, int, int], list[dict]] = {}
        self.bytes_read = 0

    def close(self) -> None:
        self._pool.shutdown(wait=True)

    @staticmethod
    def expert_name(layer: int, expert: int, prefix: str, role: str) -> str:
        if prefix == "layers":
            return f"layers.{layer}.ffn.experts.{expert}.{role}"
        return f"mtp.{layer}.ffn.experts.{expert}.{role}"

    def entry(self, name: str) -> dict:
        e = self._by_name.get(name)
        if e is None:
            raise KeyError(f"tensor {name!r} is not in the manifest")
        return e

    def expert_runs(self, prefix: str, layer: int, expert: int) -> list[dict]:
        """Contiguous on-disk byte runs covering one expert's tensors: entries
        sorted by (shard, offset), adjacent ranges merged (the checkpoint keeps
        an expert's weights back to back and its scales back to back)."""
        key = (prefix, layer, expert)
        runs = self._run_cache.get(key)
        if runs is not None:
            return runs
        ents = []
        for role in ROLES:
            base = self.expert_name(layer, expert, prefix, role)
            ents.append((role, "weight", self.entry(f"{base}.weight")))
            ents.append((role, "scale", self.entry(f"{base}.scale")))
            bias = self._by_name.get(f"{base}.bias")
            if bias is not None:
                ents.append((role, "bias", bias))
        ents.sort(key=lambda t: (t[2]["shard"], t[2]["file_range"][0]))
        runs = []
        for role, kind, e in ents:
            start, end = e["file_range"]
            if runs and runs[-1]["shard"] == e["shard"] and runs[-1]["end"] == start:
                runs[-1]["end"] = end
                runs[-1]["parts"].append((role, kind, start - runs[-1]["start"], e))
            else:
                runs.append({"shard": e["shard"], "start": start, "end": end, "parts": [(role, kind, 0, e)]})
        self._run_cache[key] = runs
        return runs

    def _layout(self, layer: int, expert: int, prefix: str) -> dict:
        """Per role and part: (dtype, shape, bytes); checks the format's shape rules."""
        out = {}
        for role in ROLES:
            base = self.expert_name(layer, expert, prefix, role)
            w, s = self.entry(f"{base}.weight"), self.entry(f"{base}.scale")
            b = self._by_name.get(f"{base}.bias")
            parts = {"weight": w, "scale": s} if b is None else {"weight": w, "scale": s, "bias": b}
            for kind, e in parts.items():
                n = int(np.prod(e["shape"])) * _DTYPE_BYTES.get(e["dtype"], 0)
                if n != e["bytes"] or e["file_range"][1] - e["file_range"][0] != e["bytes"]:
                    raise ValueError(f"{base}.{kind}: {e['dtype']} {e['shape']} does not match {e['bytes']} bytes")
            rows = w["shape"][0]
            if b is None:   # FP4: [rows, K/2] codes, [rows, K/32] ue8m0
                if w["dtype"] not in ("I8", "U8") or s["dtype"] not in ("F8_E8M0", "U8"):
                    raise ValueError(f"{base}: FP4 expects I8/U8 codes and F8_E8M0 scales")
                if s["shape"] != [rows, w["shape"][1] // 16] or w["shape"][1] % 16:
                    raise ValueError(f"{base}: FP4 scale shape {s['shape']} for codes {w['shape']}")
            else:           # q3: [rows, K*3/32] u32 words, [rows, K/64] f16 scale and bias
                if w["dtype"] != "U32_Q3_AFFINE" or s["dtype"] != "F16" or b["dtype"] != "F16":
                    raise ValueError(f"{base}: q3 expects U32_Q3_AFFINE words and F16 scale / bias")
                if s["shape"] != b["shape"] or s["shape"][0] != rows or w["shape"][1] != s["shape"][1] * 6:
                    raise ValueError(f"{base}: q3 shapes {w['shape']} / {s['shape']} / {b['shape']} disagree")
            out[role] = {k: (e["dtype"], tuple(e["shape"]), e["bytes"]) for k, e in parts.items()}
        return out

    def read_banks_host(self, layer: int, experts: list[int], prefix: str = "layers") -> dict:
        """One layer's experts read into pinned host staging: {role: {part:
        tensor [E, ...]}} (uint8 codes / scales for FP4; int32 words and f16
        scales / biases for q3), experts stacked in the given order."""
        if not experts:
            raise ValueError("no experts to load")
        layout = self._layout(layer, experts[0], prefix)
        for e in experts[1:]:
            if self._layout(layer, e, prefix) != layout:
                raise ValueError(f"layer {layer}: expert {e} has a different tensor layout than expert {experts[0]}")
        tdt = {"I8": torch.uint8, "U8": torch.uint8, "F8_E8M0": torch.uint8, "U32_Q3_AFFINE": torch.int32,
               "F16": torch.float16}
        pin = torch.cuda.is_available()
        staging = {role: {kind: torch.empty((len(experts), *shape), dtype=tdt[dt], pin_memory=pin)
                          for kind, (dt, shape, _n) in parts.items()}
                   for role, parts in layout.items()}

        def _read(i_e):
            i, e = i_e
            n = 0
            for run in self.expert_runs(prefix, layer, e):
                blob = read_bytes(self._root, run["shard"], run["start"], run["end"])
                n += len(blob)
                for role, kind, off, ent in run["parts"]:
                    dst = staging[role][kind][i].view(torch.uint8).reshape(-1).numpy()
                    dst[:] = np.frombuffer(blob, dtype=np.uint8, count=ent["bytes"], offset=off)
            return n

        self.bytes_read += sum(self._pool.map(_read, list(enumerate(experts))))
        return staging

    def load_expert_banks(self, specs: list[tuple[int, int, str]], device: torch.device | str | None = None
                          ) -> dict[int, dict]:
        """Experts given as (layer, expert, prefix) -> {layer: {"banks": {role:
        ExpertBank}, "slots": {expert: slot}}}, one resident bank per projection
        and layer (slots in the order the experts were given).

        The result is keyed by layer index alone (as the reference's
        load_expert_banks, mlx_weights.py:576-649), so one call takes one
        prefix: specs that mix "layers" and "mtp" raise ValueError instead of
        letting equal layer indices overwrite each other."""
        if not specs:
            return {}
        prefixes = {prefix for _, _, prefix in specs}
        if len(prefixes) > 1:
            raise ValueError(f"load_expert_banks: one prefix per call, got {sorted(prefixes)}")
        device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        grouped: dict[tuple[int, str], list[int]] = {}
        for layer, expert, prefix in specs:
            grouped.setdefault((int(layer), prefix), []).append(int(expert))
        out: dict[int, dict] = {}
        for (layer, prefix), experts in sorted(grouped.items()):
            host = self.read_banks_host(layer, experts, prefix)
            banks = {}
            for role, parts in host.items():
                dev = {k: t.to(device, non_blocking=True) for k, t in parts.items()}
                if "bias" in dev:
                    banks[role] = ExpertBank.q3(dev["weight"], dev["scale"], dev["bias"])
                else:
                    banks[role] = ExpertBank.fp4(dev["weight"], dev["scale"]).prepare_atoms()
            torch.cuda.current_stream(device).synchronize()   # staging buffers are reused by the caller's next load
            out[layer] = {"banks": banks, "slots": {e: i for i, e in enumerate(experts)}}
        return out

    def load_shared(self, layer: int, device: torch.device | str | None = None, prefix: str = "layers"
                    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """The shared expert of a layer as resident bf16 (w1, w3, w2); FP8 e4m3
        weights with [R/32, C/32] ue8m0 scales are dequantised on the device."""
        device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        res = {}
        for role in ROLES:
            base = f"{prefix}.{layer}.ffn.shared_experts.{role}"
            w = self.entry(f"{base}.weight")
            data = read_bytes(self._root, w["shard"], *w["file_range"])
            rows, cols = w["shape"]
            if w["dtype"] == "F8_E4M3":
                s = self.entry(f"{base}.scale")
                if rows % 32 or cols % 32 or s["shape"] != [rows // 32, cols // 32]:
                    raise ValueError(f"{base}: FP8 shape {w['shape']} with scales {s['shape']}")
                sdata = read_bytes(self._root, s["shard"], *s["file_range"])
                p = torch.frombuffer(bytearray(data), dtype=torch.uint8).to(device)
                sc = torch.frombuffer(bytearray(sdata), dtype=torch.uint8).to(device)
                f32 = torch.empty((rows, cols), dtype=torch.float32, device=device)
                _abi.call("ds_fp8_block_dequant", ptr(p), rows, cols, ptr(sc), ptr(f32), stream_handle(device))
                res[role] = f32.to(torch.bfloat16)
            elif w["dtype"] in ("BF16", "F16", "F32"):
                dt = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}[w["dtype"]]
                t = torch.frombuffer(bytearray(data), dtype=dt).reshape(rows, cols)
                res[role] = t.to(device).to(torch.bfloat16)
            else:
                raise ValueError(f"{base}: shared-expert dtype {w['dtype']} is not supported")
            self.bytes_read += len(data)
        return res["w1"], res["w3"], res["w2"]

    def layer_experts(self, layer: int, prefix: str = "layers") -> list[int]:
        """Expert ids of a layer that the manifest names, ascending."""
        head = f"{prefix}.{layer}.ffn.experts."
        return sorted({int(n[len(head):].split(".", 1)[0]) for n in self._by_name if n.startswith(head)})

    def load_layer(self, layer: int, experts: list[int] | None = None, shared: bool = True,
                   device: torch.device | str | None = None, prefix: str = "layers") -> MoEWeights:
        """One decode layer resident on the device: routed banks of ``experts``
        (default: every expert of the layer in the manifest, ascending) and,
        when present, the shared expert; FP4 banks come with their scale atoms."""
        if experts is None:
            experts = self.layer_experts(layer, prefix)
        banks = self.load_expert_banks([(layer, e, prefix) for e in experts], device)[layer]["banks"]
        sw = (None, None, None)
        if shared and f"{prefix}.{layer}.ffn.shared_experts.w1.weight" in self._by_name:
            sw = self.load_shared(layer, device, prefix)
        return MoEWeights(banks["w1"], banks["w3"], banks["w2"], *sw)
