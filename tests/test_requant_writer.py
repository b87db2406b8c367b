"""q3 payload writer (deepseeker.requant.requant_experts) on synthetic FP4 checkpoints.

The reference script (scripts/requant_experts_3bit.py:150-259) appends, per
expert, the three weights, the three scales and the three biases to the
payload, rewrites the weight / scale manifest entries in place, adds the bias
entries, and skips experts that are already converted.  The CPU tests drive
the writer with the oracle's converter (oracle.fp4 dequant + oracle.q3
quantiser) and read the result back through deepseeker.loader; the GPU test
checks that the device converter writes the same bytes and that the loaded q3
layer runs through the decode kernel.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from deepseeker import loader, requant
from oracle import fp4 as ofp4
from oracle import q3 as oq3
from tests.test_loader import LAYER, E, make_fp4_checkpoint


def oracle_convert(wdata: bytes, sdata: bytes, rows: int, cols: int):
    vals = ofp4.dequant_matrix(np.frombuffer(wdata, dtype=np.uint8).reshape(rows, cols // 2),
                               np.frombuffer(sdata, dtype=np.uint8).reshape(rows, cols // 32))
    words, sc, bi = oq3.quantize(vals)
    rt = oq3.dequant(words, sc, bi)
    rms = float(np.sqrt(np.mean((vals.astype(np.float64) - rt) ** 2))) / max(float(np.abs(rt).max()), 1e-9)
    return words.astype("<u4").tobytes(), sc.astype("<f2").tobytes(), bi.astype("<f2").tobytes(), rms


def fp4_manifest(tmp_path):
    root, src = make_fp4_checkpoint(tmp_path)
    return root, src, loader.manifest_from_shards(root, ["a.safetensors", "b.safetensors"])


def test_writer_layout_and_manifest(tmp_path):
    root, src, man = fp4_manifest(tmp_path)
    n_before = len(man["tensors"])
    qlog = tmp_path / "q.jsonl"
    out = tmp_path / "model-manifest-q3.json"
    requant.requant_experts(man, root, root / "routed-q3.payload", [LAYER], [1, 2], quality_log=qlog,
                            out_manifest=out, convert=oracle_convert)
    by = {t["name"]: t for t in man["tensors"]}
    assert len(man["tensors"]) == n_before + 2 * 3          # bias entries added
    base = f"layers.{LAYER}.ffn.experts.1"
    w1 = by[f"{base}.w1.weight"]
    assert w1["dtype"] == "U32_Q3_AFFINE" and w1["shard"] == "routed-q3.payload" and w1["shape"] == [128, 24]
    assert by[f"{base}.w2.scale"]["dtype"] == "F16" and by[f"{base}.w2.scale"]["shape"] == [256, 2]
    # payload order per expert: weights w1 w2 w3, scales, biases; expert 1 then 2
    offs = [by[f"layers.{LAYER}.ffn.experts.{e}.{r}.{p}"]["file_range"]
            for e in (1, 2) for p in ("weight", "scale", "bias") for r in ("w1", "w2", "w3")]
    assert offs[0][0] == 0 and all(a[1] == b[0] for a, b in zip(offs, offs[1:]))
    assert (root / "routed-q3.payload").stat().st_size == offs[-1][1]
    # unconverted experts keep their FP4 entries
    assert by[f"layers.{LAYER}.ffn.experts.0.w1.weight"]["dtype"] == "I8"
    assert man["q3_requant"]["experts_converted"] == 2
    assert json.loads(out.read_text())["q3_requant"]["payload_bytes_written"] == offs[-1][1]
    lines = [json.loads(x) for x in qlog.read_text().splitlines()]
    assert len(lines) == 6 and all(0.0 < x["rms_rel"] < 0.5 for x in lines)
    # read back through the loader: the words / scales / biases the converter made
    ld = loader.ExpertLoader(root, man)
    host = ld.read_banks_host(LAYER, [2])
    ld.close()
    for r in ("w1", "w2", "w3"):
        w = src[f"layers.{LAYER}.ffn.experts.2.{r}.weight"]
        s = src[f"layers.{LAYER}.ffn.experts.2.{r}.scale"]
        words, sc, bi, _ = oracle_convert(w.tobytes(), s.tobytes(), w.shape[0], w.shape[1] * 2)
        assert host[r]["weight"].numpy().tobytes() == words
        assert host[r]["scale"].numpy().tobytes() == sc and host[r]["bias"].numpy().tobytes() == bi


def test_writer_resumes(tmp_path):
    root, _, man = fp4_manifest(tmp_path)
    pay = root / "routed-q3.payload"
    requant.requant_experts(man, root, pay, [LAYER], [0, 1], convert=oracle_convert)
    size = pay.stat().st_size
    requant.requant_experts(man, root, pay, [LAYER], [0, 1], convert=oracle_convert)   # nothing to do
    assert pay.stat().st_size == size and man["q3_requant"]["experts_converted"] == 0
    requant.requant_experts(man, root, pay, [LAYER], list(range(E)), convert=oracle_convert)
    assert pay.stat().st_size == 2 * size
    by = {t["name"]: t for t in man["tensors"]}
    assert by[f"layers.{LAYER}.ffn.experts.3.w3.bias"]["file_range"][1] == 2 * size
    assert sum(1 for t in man["tensors"] if t["name"].endswith(".bias")) == 3 * E


@pytest.mark.gpu
def test_device_writer_matches_oracle_and_decodes(tmp_path, cuda):
    import torch

    from deepseeker import moe
    from tests.test_decode_gpu import TOL, oracle_out, rel_l2, routing
    root, _, man = fp4_manifest(tmp_path)
    man_cpu = json.loads(json.dumps(man))
    requant.requant_experts(man, root, root / "dev.payload", [LAYER], list(range(E)))
    requant.requant_experts(man_cpu, root, root / "cpu.payload", [LAYER], list(range(E)), convert=oracle_convert)
    assert (root / "dev.payload").read_bytes() == (root / "cpu.payload").read_bytes()
    ld = loader.ExpertLoader(root, man)
    layer = ld.load_layer(LAYER)
    ld.close()
    assert layer.w1.fmt == 1
    ids, wts = routing(2, E, 2, seed=11)
    x = torch.randn(2, 256, generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x, ids, wts, layer, 10.0)
    assert rel_l2(out, ref) < TOL, rel_l2(out, ref)
