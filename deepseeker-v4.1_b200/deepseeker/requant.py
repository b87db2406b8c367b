"""q3 payload conversion API -- drop-in for the reference's
``scripts/requant_experts_3bit.py``: ``parse_layers``, ``parse_experts``,
``convert_tensor`` (reference lines 52-83) and the payload writer with its
manifest rewrite (``requant_experts``, reference lines 86-259).

``convert_tensor`` quantises on the device with the builder's 3-bit affine
rule (group 64: per-group min/max, scale = (max-min)/7 and bias = min rounded
to f16, q = clamp(rint((w - bias)/scale), 0, 7)), dequantises the result on
the device and reports the same relative-RMS quality figure as the reference
(rms(err) / max|roundtrip|, float64).  The resulting words use this build's
documented 3-bit layout (the reference's MLX packing is MLX-internal).

``requant_experts`` converts FP4 experts named in a tensor manifest into a
q3 payload file and rewrites the manifest the way the reference script does:
per expert the three weights, then the three scales, then the three biases
are appended to the payload; the weight and scale entries are rewritten in
place (``U32_Q3_AFFINE`` [rows, words], ``F16`` [rows, groups], shard = the
payload, file_range = payload offsets) and the bias entries are added;
experts already converted are skipped, so an interrupted run resumes.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Callable

import numpy as np
import torch

from . import _abi
from ._dev import ptr, stream_handle, to_device
from .mlx_weights import Q3_GROUP_SIZE, dequant_q3

FP4_EXPERT_BYTES = 18800640  # reference geometry: 3 x (2304 x 5120) FP4 + scales per expert


def parse_layers(arg: str) -> list[int]:
    """"20-23" -> [20..23]; "2,5,7" -> [2,5,7]; mixed lists allowed."""
    layers: list[int] = []
    for item in arg.split(","):
        lo, sep, hi = item.partition("-")
        if sep:
            layers.extend(range(int(lo), int(hi) + 1))
        else:
            layers.append(int(item))
    return layers


def parse_experts(arg: str | None, total: int = 384) -> list[int]:
    """None / "" -> every expert id; otherwise the same syntax as parse_layers."""
    return list(range(total)) if not arg else parse_layers(arg)


def quantize_q3(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Device f32 [rows, cols] -> (words int32-view [rows, cols*3/32], scales f16, biases f16)."""
    if w.dtype != torch.float32 or not w.is_cuda or w.dim() != 2:
        raise ValueError("quantize_q3 expects a 2-D float32 CUDA tensor")
    w = w.contiguous()
    rows, cols = w.shape
    if cols % Q3_GROUP_SIZE:
        raise ValueError(f"cols {cols} not a multiple of {Q3_GROUP_SIZE}")
    words = torch.empty((rows, cols * 3 // 32), dtype=torch.int32, device=w.device)
    scales = torch.empty((rows, cols // 64), dtype=torch.float16, device=w.device)
    biases = torch.empty_like(scales)
    _abi.call("ds_q3_quantize", ptr(w), rows, cols, ptr(words), ptr(scales), ptr(biases),
              stream_handle(w.device))
    return words, scales, biases


def convert_tensor(vals: np.ndarray, rows: int, cols: int, bits: int) -> tuple[bytes, bytes, bytes, float]:
    """f32 values -> (u32 word bytes, f16 scale bytes, f16 bias bytes, relative RMS error)."""
    if bits != 3:
        raise NotImplementedError("only 3-bit affine quantisation is implemented")
    w = to_device(np.asarray(vals, dtype=np.float32).reshape(rows, cols))
    words, scales, biases = quantize_q3(w)
    rt = dequant_q3(words, scales, biases)
    rt_scale = max(float(rt.abs().max()), 1e-9)
    err = w.double() - rt.double()
    rms = float(torch.sqrt(torch.mean(err * err))) / rt_scale
    return (words.cpu().numpy().view("<u4").tobytes(), scales.cpu().numpy().astype("<f2").tobytes(),
            biases.cpu().numpy().astype("<f2").tobytes(), rms)


ROLES = ("w1", "w2", "w3")


def _convert_fp4_device(wdata: bytes, sdata: bytes, rows: int, cols: int) -> tuple[bytes, bytes, bytes, float]:
    """FP4 codes + ue8m0 scales of one matrix -> q3 bytes and quality, all on the device."""
    from .metal_fp4 import dequant
    packed = to_device(np.frombuffer(wdata, dtype=np.uint8).copy())
    scales = to_device(np.frombuffer(sdata, dtype=np.uint8).copy())
    w = dequant(packed, scales).reshape(rows, cols)
    words, sc, bi = quantize_q3(w)
    rt = dequant_q3(words, sc, bi)
    rt_scale = max(float(rt.abs().max()), 1e-9)
    err = w.double() - rt.double()
    rms = float(torch.sqrt(torch.mean(err * err))) / rt_scale
    return (words.cpu().numpy().view("<u4").tobytes(), sc.cpu().numpy().astype("<f2").tobytes(),
            bi.cpu().numpy().astype("<f2").tobytes(), rms)


def requant_experts(manifest: dict, source_root: Path | str, payload_path: Path | str, layers: list[int],
                    experts: list[int], *, quality_log: Path | str | None = None,
                    out_manifest: Path | str | None = None, flush_every: int = 128,
                    convert: Callable[[bytes, bytes, int, int], tuple[bytes, bytes, bytes, float]] | None = None
                    ) -> dict:
    """Convert the FP4 experts (layers x experts) of ``manifest`` to q3.

    Appends to ``payload_path`` (created if missing), rewrites ``manifest``
    in place and returns it; writes it to ``out_manifest`` every
    ``flush_every`` experts and at the end, and one ``{"tensor", "rms_rel"}``
    JSON line per converted matrix to ``quality_log``.  ``convert`` maps
    (codes, scales, rows, cols) to (word, scale, bias bytes, rel-RMS); the
    default runs on the device.
    """
    from .loader import read_bytes
    convert = convert or _convert_fp4_device
    by_name = {t["name"]: t for t in manifest["tensors"]}
    payload_path = Path(payload_path)
    payload_name = payload_path.name
    if not payload_path.exists():
        payload_path.touch()
    pending = []
    for layer in layers:
        for expert in experts:
            base = f"layers.{layer}.ffn.experts.{expert}"
            if all(by_name[f"{base}.{r}.weight"].get("dtype") == "U32_Q3_AFFINE" for r in ROLES):
                continue
            pending.append((layer, expert))
    qlog = open(quality_log, "a") if quality_log else None   # noqa: SIM115
    done = written = 0

    def summary() -> dict:
        return {"payload": payload_name, "group_size": Q3_GROUP_SIZE, "bits": 3,
                "layer_range": [min(layers), max(layers)] if layers else [],
                "experts_converted": done, "original_mxfp4_expert_bytes": done * FP4_EXPERT_BYTES,
                "q3_expert_bytes": written // max(done, 1), "payload_bytes_written": written}

    def flush() -> None:
        manifest["q3_requant"] = summary()
        if out_manifest:
            Path(out_manifest).write_text(json.dumps(manifest, separators=(",", ":")))

    try:
        with open(payload_path, "r+b") as payload:
            payload.seek(0, 2)
            for layer, expert in pending:
                base = f"layers.{layer}.ffn.experts.{expert}"
                blocks, dims = {}, {}
                for role in ROLES:
                    w, sc = by_name[f"{base}.{role}.weight"], by_name[f"{base}.{role}.scale"]
                    rows, cols = w["shape"][0], w["shape"][1] * 2
                    words, sraw, braw, rms = convert(read_bytes(source_root, w["shard"], *w["file_range"]),
                                                     read_bytes(source_root, sc["shard"], *sc["file_range"]),
                                                     rows, cols)
                    blocks[f"{role}.weight"], blocks[f"{role}.scale"], blocks[f"{role}.bias"] = words, sraw, braw
                    dims[role] = (rows, cols)
                    if qlog:
                        qlog.write(json.dumps({"tensor": f"{base}.{role}", "rms_rel": round(rms, 8)}) + "\n")
                        qlog.flush()
                new = {}
                for part in ("weight", "scale", "bias"):
                    for role in ROLES:
                        blob = blocks[f"{role}.{part}"]
                        start = payload.tell()
                        payload.write(blob)
                        rows, cols = dims[role]
                        if part == "weight":
                            shape, elements, dtype = [rows, cols * 3 // 32], len(blob) // 4, "U32_Q3_AFFINE"
                        else:
                            shape, elements, dtype = [rows, cols // Q3_GROUP_SIZE], len(blob) // 2, "F16"
                        new[(role, part)] = {
                            "name": f"{base}.{role}.{part}", "shape": shape, "dtype": dtype, "elements": elements,
                            "bytes": len(blob), "shard": payload_name, "data_range": [start, start + len(blob)],
                            "file_range": [start, start + len(blob)], "subsystem": "routed-expert", "layer": layer,
                            "expert": expert, "routed": True, "detail": f"{role}-{part}"}
                payload.flush()
                for role in ROLES:
                    for part in ("weight", "scale", "bias"):
                        ent = new[(role, part)]
                        if part == "bias" and ent["name"] not in by_name:
                            manifest["tensors"].append(ent)
                            by_name[ent["name"]] = ent
                        else:
                            by_name[ent["name"]].update(ent)
                done += 1
                written += sum(len(b) for b in blocks.values())
                if done % flush_every == 0:
                    flush()
    finally:
        if qlog:
            qlog.close()
    flush()
    return manifest
