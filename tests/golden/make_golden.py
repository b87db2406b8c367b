"""Generate the golden vectors that pin the CPU oracle to the reference.

Run once in a container that has the reference checkout (path given by
``--reference``, default the sibling checkout used during development):

    python tests/golden/make_golden.py --reference <path-to-reference-root>

It imports the reference's OWN numpy / torch CPU functions with a stub ``mlx``
module (the reference imports MLX at module top level but only uses it inside
functions that are not called here), runs them on the seeded inputs that the
reference's tests and benches use, and writes:

  * ``ref_vectors.npz``  -- small arrays (inputs and reference outputs);
  * ``ref_hashes.json``  -- SHA-256 digests of large reference outputs whose
                            inputs are regenerated from their seeds.

Nothing at test time reads the reference checkout; the tests read only these
two files.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _stub_mlx() -> None:
    mlx = types.ModuleType("mlx")
    core = types.ModuleType("mlx.core")

    class _Array:  # only used in annotations / isinstance checks
        pass

    core.array = _Array
    mlx.core = core
    sys.modules.setdefault("mlx", mlx)
    sys.modules.setdefault("mlx.core", core)


def _load(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def exhaustive_inputs() -> tuple[np.ndarray, np.ndarray]:
    """Every packed byte value under every ue8m0 scale byte.

    For scale byte b (0..255): 256 packed bytes 0..255 = 512 elements = 16
    blocks, all with scale byte b.  65536 packed bytes, 4096 scale bytes.
    """
    packed = np.tile(np.arange(256, dtype=np.uint8), 256)
    scales = np.repeat(np.arange(256, dtype=np.uint8), 16)
    return packed, scales


def bench_fp4_inputs() -> tuple[np.ndarray, np.ndarray]:
    """scripts/bench_fp4.py:49-51: 5120 x 2304 matrix, default_rng(9)."""
    hidden, inter = 5120, 2304
    rng = np.random.default_rng(9)
    packed = rng.integers(0, 256, size=(hidden * inter) // 2, dtype=np.uint8)
    scales = np.exp2(rng.integers(-2, 3, size=(hidden * inter) // 32).astype(np.float32))
    return packed, scales


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True,
                    help="root of the reference checkout (contains src/deepseeker)")
    args = ap.parse_args()
    src = args.reference / "src" / "deepseeker"
    _stub_mlx()
    sys.path.insert(0, str(args.reference / "src"))
    mf = _load("deepseeker.metal_fp4", src / "metal_fp4.py")
    mw = _load("deepseeker.mlx_weights", src / "mlx_weights.py")
    ma = _load("deepseeker.moe_align", src / "moe_align.py")
    gr = _load("deepseeker.grouped", src / "grouped.py")

    vec: dict[str, np.ndarray] = {}
    hashes: dict[str, str] = {}

    # tests/test_metal_fp4.py:44-53 (seed 3, 512 bytes, f32 scales 2^[-3,3))
    rng = np.random.default_rng(3)
    packed = rng.integers(0, 256, size=512, dtype=np.uint8)
    scales = np.exp2(rng.integers(-3, 3, size=32).astype(np.float32))
    vec["fp4_seed3_packed"] = packed
    vec["fp4_seed3_scales"] = scales
    vec["fp4_seed3_out"] = mf.reference_dequant(packed, scales)
    vec["fp4_seed3_torch"] = mf.torch_reference(packed, scales).numpy()

    # tests/test_mlx_weights.py:77-88 (seed 2, raw u8 scales 120..134)
    rng = np.random.default_rng(2)
    packed = rng.integers(0, 256, size=512, dtype=np.uint8)
    raw = rng.integers(120, 135, size=32, dtype=np.uint8)
    vec["fp4_seed2_packed"] = packed
    vec["fp4_seed2_raw_scales"] = raw
    vec["fp4_seed2_out"] = mw.dequant_fp4_rowmajor(packed, raw)

    # tests/test_q3.py:132-141 (byte 0x13, scale byte 128 -> [2.0, 1.0])
    vec["fp4_nibble_out"] = mw.dequant_fp4_rowmajor(np.array([0x13], np.uint8),
                                                    np.array([128], np.uint8))

    # tail block: 3 bytes = 6 elements, one partial scale block
    vec["fp4_tail_out"] = mw.dequant_fp4_rowmajor(np.array([0x21, 0x9F, 0x78], np.uint8),
                                                  np.array([130], np.uint8))

    # every ue8m0 byte through both reference decoders
    vec["u8m0_all"] = mw.decode_u8m0(np.arange(256, dtype=np.uint8))
    vec["u8m0_all_metal"] = mf.decode_scales_u8m0(bytes(range(256)))
    vec["fp4_table"] = mf.FP4_TABLE.copy()
    vec["e4m3_table"] = mw.E4M3_TABLE.copy()

    # exhaustive: every byte x every scale byte
    packed, sc = exhaustive_inputs()
    out = mw.dequant_fp4_rowmajor(packed, sc)
    vec["fp4_exhaustive_out"] = out
    out2 = mf.reference_dequant(packed, mw.decode_u8m0(sc))
    assert np.array_equal(out.view(np.uint32), out2.view(np.uint32))

    # scripts/bench_fp4.py:49-58 (5120 x 2304, seed 9): hash only
    packed, scales = bench_fp4_inputs()
    hashes["bench_fp4_seed9_inputs"] = sha(packed) + ":" + sha(scales)
    hashes["bench_fp4_seed9_out"] = sha(mf.reference_dequant(packed, scales))

    # tests/test_mlx_weights.py:64-75 (fp8 32x32 block, seed 1)
    rng = np.random.default_rng(1)
    p8 = rng.integers(0, 256, size=(32, 64), dtype=np.uint8)
    s8 = rng.integers(120, 135, size=(1, 2), dtype=np.uint8)
    vec["fp8_seed1_packed"] = p8
    vec["fp8_seed1_scales"] = s8
    vec["fp8_seed1_out"] = mw.dequant_fp8_block(p8, s8)

    # tests/test_audit.py:37-60 (align docstring example + random 256x6 / E=384 / block 16)
    topk = np.array([[1, 2, 3], [0, 1, 3], [0, 2, 3], [0, 1, 2]])
    s_ids, e_ids, n_pad = ma.align_block_size(topk, 4, 4)
    vec["align_doc_sorted"], vec["align_doc_experts"] = s_ids, e_ids
    vec["align_doc_npad"] = np.array([n_pad])
    rng = np.random.default_rng(0)
    topk = rng.integers(0, 384, size=(256, 6))
    s_ids, e_ids, n_pad = ma.align_block_size(topk, 16, 384)
    vec["align_rand_topk"] = topk
    vec["align_rand_sorted"], vec["align_rand_experts"] = s_ids, e_ids
    vec["align_rand_npad"] = np.array([n_pad])

    # tests/test_grouped.py:29-39 plan_groups golden
    groups = gr.plan_groups([[2, 0], [1, 2], [0, 0]], 3)
    hashes["plan_groups_golden"] = json.dumps({str(k): v for k, v in groups.items()})

    np.savez_compressed(HERE / "ref_vectors.npz", **vec)
    (HERE / "ref_hashes.json").write_text(json.dumps(hashes, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(vec)} arrays, {len(hashes)} hashes")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
