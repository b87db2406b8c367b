"""Checkpoint loader (deepseeker.loader) against synthetic checkpoints.

The checkpoints follow the reference's on-disk conventions: safetensors
shards addressed by a manifest whose ``file_range`` is 8 + header_len + the
tensor's data offsets (tests/test_manifest.py:55-59 of the reference), an
expert's three weights stored back to back and its three scales back to back
(mlx_weights.py:275-279), and the q3 payload entries of
scripts/requant_experts_3bit.py:193-225 (``U32_Q3_AFFINE`` words + ``F16``
scale and bias, file_range = payload offsets).  CPU tests cover the manifest,
the run merging, the host staging and the error contracts; GPU tests load a
layer onto the device and run the decode kernel against the oracle.
"""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest
import torch

from deepseeker import loader
from oracle import fp4 as ofp4
from oracle import q3 as oq3

H, I, Is, E, LAYER = 256, 128, 64, 4, 3


def write_safetensors(path, tensors: dict[str, tuple[str, list[int], np.ndarray]]) -> None:
    """name -> (dtype, shape, raw array); data laid out in dict order."""
    header, blobs, off = {}, [], 0
    for name, (dt, shape, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    raw = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)) + raw + b"".join(blobs))


def fp4_expert(rng, rows, cols):
    codes = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    scales = rng.integers(118, 126, size=(rows, cols // 32), dtype=np.uint8)
    return codes, scales


def fp8_matrix(rng, rows, cols):
    b = rng.integers(0, 0x7E, size=(rows, cols), dtype=np.uint8)     # finite magnitudes
    b |= (rng.integers(0, 2, size=(rows, cols), dtype=np.uint8) << 7)
    s = rng.integers(118, 124, size=(rows // 32, cols // 32), dtype=np.uint8)
    return b, s


def make_fp4_checkpoint(tmp_path, seed=0):
    """Two shards: experts of LAYER in shard a (every expert's three weights
    back to back, then every expert's three scales), the FP8 shared expert in
    shard b.  Returns (root, src) with the
    source arrays by tensor name."""
    rng = np.random.default_rng(seed)
    src, ta, tb = {}, {}, {}
    dims = {"w1": (I, H), "w3": (I, H), "w2": (H, I)}
    parts = [{r: fp4_expert(rng, *dims[r]) for r in ("w1", "w2", "w3")} for _ in range(E)]
    for kind, idx, dt in (("weight", 0, "I8"), ("scale", 1, "F8_E8M0")):
        for e in range(E):
            for r in ("w1", "w2", "w3"):
                name = f"layers.{LAYER}.ffn.experts.{e}.{r}.{kind}"
                ta[name] = (dt, list(parts[e][r][idx].shape), parts[e][r][idx])
                src[name] = parts[e][r][idx]
    sdims = {"w1": (Is, H), "w3": (Is, H), "w2": (H, Is)}
    for r in ("w1", "w2", "w3"):
        w, s = fp8_matrix(rng, *sdims[r])
        tb[f"layers.{LAYER}.ffn.shared_experts.{r}.weight"] = ("F8_E4M3", list(w.shape), w)
        tb[f"layers.{LAYER}.ffn.shared_experts.{r}.scale"] = ("F8_E8M0", list(s.shape), s)
        src[f"shared.{r}.weight"], src[f"shared.{r}.scale"] = w, s
    write_safetensors(tmp_path / "a.safetensors", ta)
    write_safetensors(tmp_path / "b.safetensors", tb)
    return tmp_path, src


def make_q3_checkpoint(tmp_path, seed=1):
    """A raw q3 payload file and its manifest entries (requant layout: per
    expert the three weights, then the three scales, then the three biases)."""
    rng = np.random.default_rng(seed)
    src, tensors, blob = {}, [], bytearray()
    dims = {"w1": (I, H), "w3": (I, H), "w2": (H, I)}
    for e in range(E):
        q = {}
        for r in ("w1", "w2", "w3"):
            rows, cols = dims[r]
            w = rng.normal(0, 0.02, size=(rows, cols)).astype(np.float32)
            q[r] = oq3.quantize(w)   # (u32 words, f16 scales, f16 biases)
        for part, idx, dt in (("weight", 0, "U32_Q3_AFFINE"), ("scale", 1, "F16"), ("bias", 2, "F16")):
            for r in ("w1", "w2", "w3"):
                a = np.ascontiguousarray(q[r][idx])
                b = a.tobytes()
                name = f"layers.{LAYER}.ffn.experts.{e}.{r}.{part}"
                tensors.append({"name": name, "shape": list(a.shape), "dtype": dt, "bytes": len(b),
                                "shard": "routed-q3.payload", "file_range": [len(blob), len(blob) + len(b)]})
                src[name] = a
                blob += b
    (tmp_path / "routed-q3.payload").write_bytes(bytes(blob))
    return tmp_path, {"tensors": tensors}, src


# ------------------------------------------------------------------ CPU: manifest, runs, staging

def test_manifest_file_range_convention(tmp_path):
    root, src = make_fp4_checkpoint(tmp_path)
    n, header = loader.parse_safetensors_header(root / "a.safetensors")
    man = loader.manifest_from_shards(root, ["a.safetensors", "b.safetensors"])
    ent = {t["name"]: t for t in man["tensors"]}
    name = f"layers.{LAYER}.ffn.experts.1.w2.scale"
    a, b = header[name]["data_offsets"]
    assert ent[name]["file_range"] == [8 + n + a, 8 + n + b]
    assert ent[name]["bytes"] == b - a and ent[name]["shard"] == "a.safetensors"
    got = loader.read_bytes(root, "a.safetensors", *ent[name]["file_range"])
    assert got == src[name].tobytes()


def test_expert_runs_merge_contiguous_ranges(tmp_path):
    root, _ = make_fp4_checkpoint(tmp_path)
    man = loader.manifest_from_shards(root, ["a.safetensors", "b.safetensors"])
    ld = loader.ExpertLoader(root, man)
    runs = ld.expert_runs("layers", LAYER, 2)
    assert len(runs) == 2   # the weight run and the scale run
    assert [(r, k) for r, k, _, _ in runs[0]["parts"]] == [("w1", "weight"), ("w2", "weight"), ("w3", "weight")]
    assert [(r, k) for r, k, _, _ in runs[1]["parts"]] == [("w1", "scale"), ("w2", "scale"), ("w3", "scale")]
    assert runs[0]["end"] - runs[0]["start"] == sum(e["bytes"] for _, _, _, e in runs[0]["parts"])
    ld.close()


def test_read_banks_host_fp4(tmp_path):
    root, src = make_fp4_checkpoint(tmp_path)
    man = loader.manifest_from_shards(root, ["a.safetensors", "b.safetensors"])
    ld = loader.ExpertLoader(root, man)
    order = [2, 0, 3]
    host = ld.read_banks_host(LAYER, order)
    for r in ("w1", "w2", "w3"):
        for kind in ("weight", "scale"):
            want = np.stack([src[f"layers.{LAYER}.ffn.experts.{e}.{r}.{kind}"] for e in order])
            assert np.array_equal(host[r][kind].numpy(), want), (r, kind)
    assert ld.bytes_read == sum(src[f"layers.{LAYER}.ffn.experts.{e}.{r}.{k}"].nbytes
                                for e in order for r in ("w1", "w2", "w3") for k in ("weight", "scale"))
    ld.close()


def test_read_banks_host_q3_payload(tmp_path):
    root, man, src = make_q3_checkpoint(tmp_path)
    ld = loader.ExpertLoader(root, man)
    assert len(ld.expert_runs("layers", LAYER, 1)) == 1   # one expert = one contiguous run
    host = ld.read_banks_host(LAYER, [1, 3])
    for r in ("w1", "w2", "w3"):
        assert host[r]["weight"].dtype == torch.int32 and host[r]["scale"].dtype == torch.float16
        for kind in ("weight", "scale", "bias"):
            want = np.stack([src[f"layers.{LAYER}.ffn.experts.{e}.{r}.{kind}"] for e in (1, 3)])
            got = host[r][kind].numpy()
            assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (r, kind)
    ld.close()


def test_layer_experts_and_runs_cache(tmp_path):
    root, _ = make_fp4_checkpoint(tmp_path)
    man = loader.manifest_from_shards(root, ["a.safetensors", "b.safetensors"])
    ld = loader.ExpertLoader(root, man)
    assert ld.layer_experts(LAYER) == list(range(E))
    assert ld.layer_experts(LAYER + 1) == []
    assert ld.expert_runs("layers", LAYER, 1) is ld.expert_runs("layers", LAYER, 1)
    ld.close()


def test_layout_errors(tmp_path):
    root, _ = make_fp4_checkpoint(tmp_path)
    man = loader.manifest_from_shards(root, ["a.safetensors", "b.safetensors"])
    bad = json.loads(json.dumps(man))
    for t in bad["tensors"]:
        if t["name"] == f"layers.{LAYER}.ffn.experts.1.w1.scale":
            t["shape"] = [t["shape"][0] // 2, t["shape"][1] * 2]   # same bytes, wrong geometry
    ld = loader.ExpertLoader(root, bad)
    with pytest.raises(ValueError):
        ld.read_banks_host(LAYER, [0, 1])
    with pytest.raises(KeyError):
        ld.read_banks_host(LAYER, [7])
    # one prefix per call: the result is keyed by layer index alone
    with pytest.raises(ValueError, match="one prefix per call"):
        ld.load_expert_banks([(LAYER, 0, "layers"), (LAYER, 1, "mtp")])
    ld.close()


def test_read_into_buffer(tmp_path):
    root, src = make_fp4_checkpoint(tmp_path)
    man = loader.manifest_from_shards(root, ["a.safetensors", "b.safetensors"])
    ent = {t["name"]: t for t in man["tensors"]}[f"layers.{LAYER}.ffn.experts.3.w1.weight"]
    buf = np.zeros(ent["bytes"], dtype=np.uint8)
    assert loader.read_into(root, ent["shard"], ent["file_range"][0], buf) == ent["bytes"]
    assert buf.tobytes() == src[f"layers.{LAYER}.ffn.experts.3.w1.weight"].tobytes()
    with pytest.raises(ValueError):
        loader.read_into(root, ent["shard"], ent["file_range"][0], bytes(4))   # read-only target
    with pytest.raises(RuntimeError):
        loader.read_bytes(root, ent["shard"], (root / ent["shard"]).stat().st_size - 2,
                          (root / ent["shard"]).stat().st_size + 2)   # past the end: short read


def test_not_safetensors(tmp_path):
    p = tmp_path / "x.safetensors"
    p.write_bytes(b"\x01\x02")
    with pytest.raises(ValueError):
        loader.parse_safetensors_header(p)


# ------------------------------------------------------------------ GPU: resident layer through the decode kernel

@pytest.mark.gpu
def test_load_layer_fp4_fp8_shared_decode(tmp_path, cuda):
    from deepseeker import moe
    from tests.test_decode_gpu import TOL, oracle_out, rel_l2, routing
    root, src = make_fp4_checkpoint(tmp_path)
    man = loader.manifest_from_shards(root, ["a.safetensors", "b.safetensors"])
    ld = loader.ExpertLoader(root, man)
    layer = ld.load_layer(LAYER)
    ld.close()
    assert layer.n_experts == E and layer.hidden == H and layer.inter == I
    assert layer.w1.scales_tc is not None
    for r, t in (("w1", layer.shared_w1), ("w3", layer.shared_w3), ("w2", layer.shared_w2)):
        want = torch.from_numpy(ofp4.dequant_fp8_block(src[f"shared.{r}.weight"], src[f"shared.{r}.scale"]))
        assert torch.equal(t.cpu(), want.float().to(torch.bfloat16)), r
    ids, wts = routing(2, E, 2, seed=3)
    x = torch.randn(2, H, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x, ids, wts, layer, 10.0)
    assert rel_l2(out, ref) < TOL, rel_l2(out, ref)


@pytest.mark.gpu
def test_load_layer_q3_decode(tmp_path, cuda):
    from deepseeker import moe
    from tests.test_decode_gpu import TOL, oracle_out, rel_l2, routing
    root, man, src = make_q3_checkpoint(tmp_path)
    ld = loader.ExpertLoader(root, man)
    layer = ld.load_layer(LAYER)
    ld.close()
    assert layer.shared_w1 is None and layer.w1.fmt == 1
    ids, wts = routing(1, E, 2, seed=5)
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x, ids, wts, layer, 10.0)
    assert rel_l2(out, ref) < TOL, rel_l2(out, ref)
