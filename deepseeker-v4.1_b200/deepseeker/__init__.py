"""deepseeker (B200 build): drop-in operators for DeepSeeker-V4.1's routed-expert hot path.

Modules mirror the reference package's hot-path surface:
  metal_fp4    FP4 e2m1 dequant (`metal_dequant`, device-resident `dequant`)
  mlx_weights  weight-format helpers (u8m0 / e4m3 / FP8 block / FP4 row-major / q3)
  requant      q3 payload conversion API of scripts/requant_experts_3bit.py
  variant_q3   DEEPSEEKER_VARIANT selection
  moe          routing, resident expert banks, fused decode MoE layer, `moe_layer`
  grouped      `plan_groups` and the grouped expert FFN
  moe_align    device sort-and-pad alignment
  ep           expert-parallel dispatch / combine over torch.distributed
  loader       checkpoint manifest / shards -> resident expert banks

All compute runs in libdeepseeker_b200.so (CUDA, sm_100a), loaded lazily on the
first operator call; there is no CPU fallback.
"""
__all__ = ["metal_fp4", "mlx_weights", "requant", "variant_q3", "moe", "grouped", "moe_align", "ep", "loader"]
