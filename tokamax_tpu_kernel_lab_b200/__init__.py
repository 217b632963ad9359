"""B200 (sm_100a) LatentMoE expert path: router, dispatch, grouped GEMMs with
fused SiTU-GLU, combine, expert parallelism -- behind the reference's
operator API (tokamax `ragged_dot`, fused gate/up, `latent_moe_forward`)."""

from ._native import LIB_PATH, NativeLibraryMissing, load as load_native
from .latent_moe import (LatentMoEConfig, LatentMoEWeights, PreparedWeights, full_layer_config,
                         init_prepared_mxfp4, init_weights, kimi_k3_config, latent_moe_forward,
                         latent_moe_forward_ragged_dot, prepare_weights, random_mxfp4,
                         reduced_cpu_config, toy_config)
from .ops import (Dispatch, MXFP4Weights, check_device_status, combine_rmsnorm, combine_shard_contribution,
                  dispatch, filter_and_pad_to_shard_jittable, fp8_ragged_dot, RaggedDotOp,
                  fused_gateup_situ, gather_rows, gemm,
                  mxfp4_fused_gateup_situ, mxfp4_ragged_dot, parse_fused_activation, prefuse_gateup_weights, ragged_dot, router_gate,
                  router_logits, router_topk, situ_and_mul)

__all__ = [
    "LIB_PATH", "NativeLibraryMissing", "load_native", "LatentMoEConfig", "LatentMoEWeights",
    "PreparedWeights", "full_layer_config", "init_weights", "kimi_k3_config",
    "latent_moe_forward", "latent_moe_forward_ragged_dot", "prepare_weights",
    "reduced_cpu_config", "toy_config", "Dispatch", "check_device_status", "combine_rmsnorm",
    "combine_shard_contribution", "dispatch", "filter_and_pad_to_shard_jittable",
    "fused_gateup_situ", "fp8_ragged_dot", "RaggedDotOp", "gather_rows", "gemm", "parse_fused_activation",
    "prefuse_gateup_weights", "ragged_dot", "router_gate", "router_logits", "router_topk",
    "situ_and_mul", "MXFP4Weights", "mxfp4_ragged_dot", "mxfp4_fused_gateup_situ",
    "init_prepared_mxfp4", "random_mxfp4",
]
