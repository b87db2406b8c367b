"""CPU oracle for the routed-expert MoE hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy / torch fp32 on the CPU, the reference's
algorithms for the path this repository accelerates (FP4 e2m1 and 3-bit affine
expert weights, their dequantisation, the SwiGLU expert FFN, the routed MoE
combine, routing and the sort-and-pad alignment).  Every function cites the
reference file:line (paths relative to the reference project root) it follows.

Rules:
  * only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
    leg (``cpu_baseline`` and ``--impl reference``) may import this package, and
    only as the checker / the timed reference CPU path;
  * the product (``deepseeker``) never imports it: the product path is the
    CUDA library and fails loudly when that library is missing.

Pinning: ``tests/golden/make_golden.py`` imports the reference's own numpy /
torch CPU functions (``metal_fp4.reference_dequant``, ``torch_reference``,
``decode_scales_u8m0``; ``mlx_weights.decode_u8m0``, ``dequant_fp4_rowmajor``,
``E4M3_TABLE``, ``dequant_fp8_block``, ``unpack_int3_affine``;
``moe_align.align_block_size``; ``grouped.plan_groups``) with a stub ``mlx``
module and writes golden vectors under ``tests/golden/``; ``tests/test_oracle.py``
checks this oracle against them.  The 3-bit bit layout and the quantisers are
builder-defined (MLX, which owns the reference's 3-bit packing, is not
available): that part of the oracle is "parity unpinned" at the bit level and
pinned only through the reference's shape contracts.
"""
