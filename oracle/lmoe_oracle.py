"""CPU oracle for the LatentMoE expert path -- TEST INFRASTRUCTURE ONLY.

This module is a numpy restatement of the reference's JAX algorithm for the
LatentMoE expert path. It exists so that the CUDA path can be checked against
it. Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg
(and `bench.py --impl reference`) may import it, and only as the checker or as
the timed CPU baseline -- never as the thing measured or shipped. The product
package never imports it.

Pinning: `tests/test_oracle_golden.py` checks this restatement against the six
golden bundles the reference generated from the official PyTorch block
(`06_kimi_k3_golden_validation/golden_bundle_*`, re-packed under
`tests/golden/` by `tests/golden/make_golden.py`), stage by stage, with the
reference's own canonicalisation and tolerances
(`06_kimi_k3_golden_validation/test_jax_reference_against_pytorch_golden.py:94-97,278-289`).

Every function cites the reference file:line it restates.  Paths are relative
to the reference project root:
  KR  = 05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py
  KRD = 05_ragged_dot_on_tpu/kimi_k3_latent_moe_ragged_dot.py
  MXD = 05_ragged_dot_on_tpu/mxfp4_dequant.py
  GUS = 05_ragged_dot_on_tpu/own_gateup_situ_pallas_kernel.py

dtype model: arrays are numpy float32 throughout.  A "bf16" compute dtype is
emulated by rounding to bfloat16 (round-to-nearest-even, via ml_dtypes) at
exactly the points where JAX would materialise a bf16 array; matmuls
accumulate in float32 (what XLA:CPU and PyTorch-CPU do for bf16 dots).
"""

from __future__ import annotations

import dataclasses
import math

import numpy as np

try:
  import ml_dtypes

  _BF16 = ml_dtypes.bfloat16
except ImportError:  # pragma: no cover - ml_dtypes ships with the image
  _BF16 = None

_MOSAIC_TILE_SIZE = 128  # KR:149


# ----------------------------------------------------------------------------
# dtype helpers
# ----------------------------------------------------------------------------


def bf16_round(x: np.ndarray) -> np.ndarray:
  """float32 -> bfloat16 (round to nearest even) -> float32."""
  x = np.asarray(x, dtype=np.float32)
  if _BF16 is not None:
    return x.astype(_BF16).astype(np.float32)
  b = x.view(np.uint32).astype(np.uint64)
  b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
  return b.astype(np.uint32).view(np.float32)


def to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
  """Materialise `x` in the compute dtype ("fp32" or "bf16"), held as float32."""
  if dtype == "bf16":
    return bf16_round(x)
  if dtype == "fp32":
    return np.asarray(x, dtype=np.float32)
  raise ValueError(f"unknown dtype {dtype!r}")


def matmul(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
  """`a @ b` in the compute dtype: float32 accumulate, result rounded to dtype."""
  out = np.matmul(a.astype(np.float32), b.astype(np.float32))
  return to_dtype(out, dtype)


def _sigmoid(x: np.ndarray) -> np.ndarray:
  x = x.astype(np.float32)
  return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


# ----------------------------------------------------------------------------
# config / weights  (KR:156-283)
# ----------------------------------------------------------------------------


@dataclasses.dataclass(frozen=True)
class LatentMoEConfig:
  """Restates `LatentMoEConfig` (KR:156-171)."""

  hidden_size: int
  latent_size: int
  intermediate_size: int
  num_experts: int
  top_k: int
  num_shared_experts: int
  moe_renormalize: bool = True
  routed_scaling_factor: float = 1.0
  rms_norm_eps: float = 1e-5
  activation_situ_beta: float = 4.0
  activation_situ_linear_beta: float = 25.0


def toy_config() -> LatentMoEConfig:
  """KR:174-188."""
  return LatentMoEConfig(64, 32, 48, 8, 2, 1)


def mosaic_golden_config() -> LatentMoEConfig:
  """Dimensions of the `golden_bundle_mosaic_*` bundles (their config.json)."""
  return LatentMoEConfig(256, 128, 128, 8, 2, 1)


@dataclasses.dataclass
class Weights:
  """Restates `LatentMoEWeights` (KR:217-252): (in, out) layout throughout."""

  router_weight: np.ndarray  # (d, E)
  e_score_correction_bias: np.ndarray  # (E,)
  down_proj: np.ndarray  # (d, L)
  up_proj: np.ndarray  # (L, d)
  expert_gate: np.ndarray  # (E, L, I)
  expert_up: np.ndarray  # (E, L, I)
  expert_down: np.ndarray  # (E, I, L)
  norm_scale: np.ndarray  # (L,)
  shared_gate: np.ndarray  # (d, I*ns)
  shared_up: np.ndarray  # (d, I*ns)
  shared_down: np.ndarray  # (I*ns, d)


def init_weights_np(cfg: LatentMoEConfig, seed: int, dtype: str = "fp32",
                    bias_std: float = 0.0) -> Weights:
  """Seeded N(0, 0.02^2) weights (the distribution of KR:255-283, numpy PCG64
  instead of jax.random).  `bias_std` > 0 draws the per-expert router bias from
  N(0, bias_std^2) (the skewed-load configs)."""
  rng = np.random.default_rng(seed)
  s = 0.02
  si = cfg.intermediate_size * cfg.num_shared_experts

  def normal(shape):
    return to_dtype(rng.standard_normal(shape, dtype=np.float32) * np.float32(s), dtype)

  w = Weights(
      router_weight=normal((cfg.hidden_size, cfg.num_experts)),
      e_score_correction_bias=np.zeros((cfg.num_experts,), np.float32),
      down_proj=normal((cfg.hidden_size, cfg.latent_size)),
      up_proj=normal((cfg.latent_size, cfg.hidden_size)),
      expert_gate=normal((cfg.num_experts, cfg.latent_size, cfg.intermediate_size)),
      expert_up=normal((cfg.num_experts, cfg.latent_size, cfg.intermediate_size)),
      expert_down=normal((cfg.num_experts, cfg.intermediate_size, cfg.latent_size)),
      norm_scale=np.ones((cfg.latent_size,), np.float32),
      shared_gate=normal((cfg.hidden_size, si)),
      shared_up=normal((cfg.hidden_size, si)),
      shared_down=normal((si, cfg.hidden_size)),
  )
  if bias_std > 0:
    w.e_score_correction_bias = to_dtype(
        rng.standard_normal(cfg.num_experts, dtype=np.float32) * np.float32(bias_std), dtype)
  return w


# ----------------------------------------------------------------------------
# primitives
# ----------------------------------------------------------------------------


def rms_norm(x: np.ndarray, scale: np.ndarray, eps: float, dtype: str) -> np.ndarray:
  """KR:286-293: float32 statistics, cast back to dtype, then * scale in dtype."""
  x32 = x.astype(np.float32)
  var = np.mean(np.square(x32), axis=-1, keepdims=True, dtype=np.float32)
  normalized = x32 * (np.float32(1.0) / np.sqrt(var + np.float32(eps)))
  return to_dtype(to_dtype(normalized, dtype) * scale.astype(np.float32), dtype)


def situ_and_mul(gate: np.ndarray, up: np.ndarray, beta: float, linear_beta: float,
                 dtype: str) -> np.ndarray:
  """KR:296-310: beta*tanh(g/beta)*sigmoid(g) * lb*tanh(u/lb), float32, cast back.

  `gate`/`up` are already in the compute dtype (the bf16-round-then-upcast
  convention of GUS:116-125); the fused path with an fp32 accumulator passes
  unrounded values."""
  g = gate.astype(np.float32)
  u = up.astype(np.float32)
  b = np.float32(beta)
  lb = np.float32(linear_beta)
  situ_gate = b * np.tanh(g / b) * _sigmoid(g)
  bounded_up = lb * np.tanh(u / lb)
  return to_dtype(situ_gate * bounded_up, dtype)


def situ_glu_mlp(x, w_gate, w_up, w_down, beta, linear_beta, dtype):
  """KR:313-327."""
  return matmul(
      situ_and_mul(matmul(x, w_gate, dtype), matmul(x, w_up, dtype), beta, linear_beta, dtype),
      w_down, dtype)


def top_k_desc(scores: np.ndarray, k: int) -> np.ndarray:
  """`jax.lax.top_k` (used at KR:351): descending, ties -> lower index."""
  order = np.argsort(-scores.astype(np.float32), axis=-1, kind="stable")
  return order[:, :k].astype(np.int32)


def router_gate(hidden_states: np.ndarray, router_weight: np.ndarray, bias: np.ndarray,
                top_k: int, renormalize: bool = True, routed_scaling_factor: float = 1.0,
                activation: str = "sigmoid"):
  """Router of `latent_moe_forward` (KR:347-356); weights stay float32.

  `activation="softmax"` is the official gate's other branch (the golden
  generator's `moe_router_activation_func`), exposed for BASELINE.json's
  wording; only "sigmoid" is pinned by reference data.
  Returns (logits, scores, scores_for_choice, topk_idx, topk_weight)."""
  logits = np.matmul(hidden_states.astype(np.float32), router_weight.astype(np.float32))
  return router_from_logits(logits, bias, top_k, renormalize, routed_scaling_factor, activation)


def router_from_logits(logits, bias, top_k, renormalize=True, routed_scaling_factor=1.0,
                       activation="sigmoid"):
  """KR:348-356 given the float32 logits."""
  logits = logits.astype(np.float32)
  if activation == "sigmoid":
    scores = _sigmoid(logits)
  elif activation == "softmax":
    m = logits.max(axis=-1, keepdims=True)
    e = np.exp(logits - m)
    scores = (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
  else:
    raise ValueError(activation)
  scores_for_choice = scores + bias.astype(np.float32)[None, :]
  topk_idx = top_k_desc(scores_for_choice, top_k)
  topk_weight = np.take_along_axis(scores, topk_idx, axis=-1).astype(np.float32)
  if top_k > 1 and renormalize:
    denom = np.sum(topk_weight, axis=-1, keepdims=True, dtype=np.float32) + np.float32(1e-20)
    topk_weight = (topk_weight / denom).astype(np.float32)
  topk_weight = (topk_weight * np.float32(routed_scaling_factor)).astype(np.float32)
  return logits, scores, scores_for_choice, topk_idx, topk_weight


def dispatch_full(topk_idx: np.ndarray, num_experts: int):
  """KR:370-378: stable argsort of flat ids, token of slot, bincount.

  Returns (order, sorted_token_idx, group_sizes)."""
  t, k = topk_idx.shape
  flat = topk_idx.reshape(-1)
  order = np.argsort(flat, kind="stable").astype(np.int32)
  token_of_slot = np.arange(t * k, dtype=np.int32) // k
  sorted_token_idx = token_of_slot[order]
  group_sizes = np.bincount(flat, minlength=num_experts)[:num_experts].astype(np.int32)
  return order, sorted_token_idx, group_sizes


def ragged_dot(lhs: np.ndarray, rhs: np.ndarray, group_sizes: np.ndarray, dtype: str = "bf16",
               rhs_layout: str = "gkn") -> np.ndarray:
  """Semantics of `tokamax.ragged_dot(lhs, rhs, group_sizes)` as the reference
  uses it (KRD:358-369), pinned by the per-expert loop it replaces (KR:383-406):
  rows [off_g, off_g + gs[g]) of the output are lhs rows @ rhs[g]; rows at or
  past sum(group_sizes) are zero.  `rhs_layout="gnk"` takes rhs as (G, N, K)."""
  m = lhs.shape[0]
  n = rhs.shape[2] if rhs_layout == "gkn" else rhs.shape[1]
  out = np.zeros((m, n), np.float32)
  start = 0
  for g, size in enumerate(np.asarray(group_sizes).tolist()):
    size = int(size)
    if size > 0:
      w = rhs[g] if rhs_layout == "gkn" else rhs[g].T
      out[start:start + size] = np.matmul(lhs[start:start + size].astype(np.float32),
                                          w.astype(np.float32))
    start += size
  return to_dtype(out, dtype)


def fused_gateup_situ(lhs, w_gateup, group_sizes, intermediate, beta, linear_beta, dtype="bf16",
                      round_gate_up=True, rhs_layout="gkn", out_dtype=None):
  """One grouped matmul against `[gate | up]` concatenated along N (KRD:610-641),
  SiTU-GLU on the result (KRD:644-723).  `round_gate_up=True` rounds gate/up to
  the compute dtype before the activation (KR:296-310 / GUS:116-125);
  False applies it to the float32 accumulator (tokamax `fuse_act`).
  The result is rounded to `out_dtype` (default: the compute dtype)."""
  acc = ragged_dot(lhs, w_gateup, group_sizes, dtype="fp32", rhs_layout=rhs_layout)
  gate, up = acc[:, :intermediate], acc[:, intermediate:2 * intermediate]
  if round_gate_up:
    gate, up = to_dtype(gate, dtype), to_dtype(up, dtype)
  out = situ_and_mul(gate, up, beta, linear_beta, out_dtype or dtype)
  total = int(np.sum(group_sizes))
  out[total:] = 0
  return out


def combine_full(outs: np.ndarray, order: np.ndarray, topk_weight: np.ndarray, dtype: str):
  """KR:413-416: scatter back to (token, slot) order, float32 weighted sum over
  the top_k slots, cast to the compute dtype."""
  t, k = topk_weight.shape
  unsorted = np.zeros_like(outs)
  unsorted[order] = outs
  unsorted = unsorted.reshape(t, k, -1).astype(np.float32)
  routed = np.zeros((t, unsorted.shape[-1]), np.float32)
  for s in range(k):  # slot order
    routed += unsorted[:, s, :] * topk_weight[:, s:s + 1].astype(np.float32)
  return to_dtype(routed, dtype), unsorted


def latent_moe_forward(hidden_states: np.ndarray, w: Weights, cfg: LatentMoEConfig,
                       dtype: str = "fp32", router_activation: str = "sigmoid",
                       return_intermediates: bool = False, quantize_activations=False):
  """Restates `latent_moe_forward` (KR:330-435) with the 18 staged
  intermediates of the golden bundles (06_.../generate_pytorch_golden.py).
  quantize_activations=True (or "mxfp8") models the block-scaled fast path:
  the expert FFN's two activation operands (the dispatched latent rows and
  the SiTU output) are rounded to MXFP8 (quantize_mxfp8) before their
  matmuls; "mxfp4" rounds them to MXFP4 (quantize_mxfp4_act) instead."""
  inter = {}
  h = to_dtype(hidden_states, dtype)
  logits, scores, sfc, topk_idx, topk_weight = router_gate(
      h, w.router_weight, w.e_score_correction_bias, cfg.top_k, cfg.moe_renormalize,
      cfg.routed_scaling_factor, router_activation)
  inter.update(router_logits=logits, router_scores_before_bias=scores,
               router_scores_for_choice=sfc, topk_indices=topk_idx, topk_weights=topk_weight)
  x = matmul(h, w.down_proj, dtype)
  inter["latent_projection"] = x
  order, sorted_token_idx, group_sizes = dispatch_full(topk_idx, cfg.num_experts)
  inter["sorted_token_indices"] = order
  inter["group_sizes"] = group_sizes
  sorted_tokens = x[sorted_token_idx]
  if quantize_activations == "mxfp4":
    mx = lambda a: dequantize_mxfp8(*quantize_mxfp4_act(a))  # values * 2^(byte - 127)
  elif quantize_activations:
    mx = lambda a: dequantize_mxfp8(*quantize_mxfp8(a))
  else:
    mx = lambda a: a
  gate = ragged_dot(mx(sorted_tokens), w.expert_gate, group_sizes, dtype)
  up = ragged_dot(mx(sorted_tokens), w.expert_up, group_sizes, dtype)
  situ = situ_and_mul(gate, up, cfg.activation_situ_beta, cfg.activation_situ_linear_beta, dtype)
  down = ragged_dot(mx(situ), w.expert_down, group_sizes, dtype)
  inter.update(expert_gate_output=gate, expert_up_output=up, situ_output=situ,
               expert_down_output=down)
  routed, unsorted = combine_full(down, order, topk_weight, dtype)
  inter["routed_output_before_combine"] = unsorted.reshape(-1, unsorted.shape[-1])
  inter["routed_output_after_combine"] = routed
  normed = rms_norm(routed, w.norm_scale, cfg.rms_norm_eps, dtype)
  inter["normalized_output"] = normed
  upo = matmul(normed, w.up_proj, dtype)
  inter["up_projection_output"] = upo
  shared = situ_glu_mlp(h, w.shared_gate, w.shared_up, w.shared_down,
                        cfg.activation_situ_beta, cfg.activation_situ_linear_beta, dtype)
  inter["shared_expert_output"] = shared
  final = to_dtype(upo + shared, dtype)
  inter["final_output"] = final
  return (final, inter) if return_intermediates else final


# ----------------------------------------------------------------------------
# expert-parallel shard form  (KR:658-877, KR:1113-1141)
# ----------------------------------------------------------------------------


def round_up_to_tile(value: int, tile_size: int = _MOSAIC_TILE_SIZE) -> int:
  """KR:152-153."""
  return -(-value // tile_size) * tile_size


def shard_m_padded(num_tokens: int, top_k: int, num_experts: int, local_num_experts: int,
                   capacity_factor: float, tile_size: int) -> int:
  """KR:825-826 (math.ceil of the same Python float expression)."""
  expected_total = num_tokens * top_k * local_num_experts / num_experts
  return round_up_to_tile(math.ceil(expected_total * capacity_factor), tile_size)


def filter_and_pad_to_shard_jittable(topk_idx, topk_weight, x, num_experts, top_k,
                                     local_expert_start, local_num_experts,
                                     capacity_factor=2.0, tile_size=_MOSAIC_TILE_SIZE,
                                     weight_dtype="fp32"):
  """KR:754-877: sentinel-key stable sort, static m_padded prefix, trailing
  padding bucket.  Returns (sorted_tokens, group_sizes, valid_mask,
  per_expert_counts, padded_token_idx, padded_combine_weight)."""
  t = topk_idx.shape[0]
  total = t * top_k
  flat = topk_idx.reshape(-1).astype(np.int64)
  token_of_slot = np.arange(total, dtype=np.int64) // top_k
  flat_w = topk_weight.reshape(-1).astype(np.float32)
  local_end = local_expert_start + local_num_experts
  in_shard = (flat >= local_expert_start) & (flat < local_end)
  sort_key = np.where(in_shard, flat - local_expert_start, local_num_experts)
  m_padded = shard_m_padded(t, top_k, num_experts, local_num_experts, capacity_factor, tile_size)
  pad_amount = max(0, m_padded - total)
  if pad_amount > 0:
    sort_key = np.concatenate([sort_key, np.full(pad_amount, local_num_experts, np.int64)])
    token_of_slot = np.concatenate([token_of_slot, np.zeros(pad_amount, np.int64)])
    flat_w = np.concatenate([flat_w, np.zeros(pad_amount, np.float32)])
  order = np.argsort(sort_key, kind="stable")[:m_padded]
  sorted_key = sort_key[order]
  valid = sorted_key < local_num_experts
  tok_all = token_of_slot[order]
  padded_token_idx = np.where(valid, tok_all, -1).astype(np.int32)
  padded_w = np.where(valid, flat_w[order], np.float32(0)).astype(np.float32)
  padded_w = to_dtype(padded_w, weight_dtype)
  counts = np.bincount(sorted_key[valid], minlength=local_num_experts)[:local_num_experts]
  counts = counts.astype(np.int32)
  pad_size = m_padded - int(counts.sum())
  group_sizes = np.concatenate([counts, np.array([pad_size], np.int32)])
  sorted_tokens = np.where(valid[:, None], x[tok_all], np.float32(0)).astype(np.float32)
  return sorted_tokens, group_sizes, valid, counts, padded_token_idx, padded_w


def filter_and_pad_to_shard(topk_idx, topk_weight, x, num_experts, top_k, local_expert_start,
                            local_num_experts, capacity_factor=2.0,
                            tile_size=_MOSAIC_TILE_SIZE, weight_dtype="fp32"):
  """KR:658-751 (eager filter-then-sort form).  Bit-identical outputs to the
  jittable form (the reference proves this at KR:880-939); restated
  separately so tests can check the equivalence here too."""
  t = topk_idx.shape[0]
  flat = topk_idx.reshape(-1).astype(np.int64)
  token_of_slot = np.arange(t * top_k, dtype=np.int64) // top_k
  flat_w = topk_weight.reshape(-1).astype(np.float32)
  local_end = local_expert_start + local_num_experts
  in_shard = (flat >= local_expert_start) & (flat < local_end)
  kept_ids = flat[in_shard] - local_expert_start
  kept_tok = token_of_slot[in_shard]
  kept_w = flat_w[in_shard]
  order = np.argsort(kept_ids, kind="stable")
  s_ids, s_tok, s_w = kept_ids[order], kept_tok[order], kept_w[order]
  m_padded = shard_m_padded(t, top_k, num_experts, local_num_experts, capacity_factor, tile_size)
  keep = min(len(s_ids), m_padded)
  counts = np.bincount(s_ids[:keep], minlength=local_num_experts)[:local_num_experts]
  counts = counts.astype(np.int32)
  pad = m_padded - keep
  group_sizes = np.concatenate([counts, np.array([pad], np.int32)])
  sorted_tokens = np.concatenate([x[s_tok[:keep]].astype(np.float32),
                                  np.zeros((pad, x.shape[-1]), np.float32)])
  valid = np.concatenate([np.ones(keep, bool), np.zeros(pad, bool)])
  padded_token_idx = np.concatenate([s_tok[:keep], -np.ones(pad, np.int64)]).astype(np.int32)
  padded_w = to_dtype(np.concatenate([s_w[:keep], np.zeros(pad, np.float32)]), weight_dtype)
  return sorted_tokens, group_sizes, valid, counts, padded_token_idx, padded_w


def combine_shard_contribution(routed_out, shard_out, padded_token_idx, padded_combine_weight,
                               dtype: str):
  """KR:1113-1141: routed_out.at[idx].add((shard_out * w).astype(dtype)).

  Duplicate indices accumulate in row order, one rounding per add (the
  sequential scatter-add of XLA:CPU); index -1 addresses the last token with
  a zero contribution."""
  out = routed_out.astype(np.float32).copy()
  weighted = to_dtype(shard_out.astype(np.float32) *
                      padded_combine_weight.astype(np.float32)[:, None], dtype)
  for p, t in enumerate(np.asarray(padded_token_idx).tolist()):
    out[t] = to_dtype(out[t] + weighted[p], dtype)
  return out


def local_shard_expert_ffn(sorted_tokens, expert_gate, expert_up, expert_down, group_sizes,
                           beta, linear_beta, dtype):
  """KR:1486-1528 (naive per-group loop, trailing padding bucket included)."""
  gate = ragged_dot(sorted_tokens, expert_gate, group_sizes, dtype)
  up = ragged_dot(sorted_tokens, expert_up, group_sizes, dtype)
  situ = situ_and_mul(gate, up, beta, linear_beta, dtype)
  total = int(np.sum(group_sizes))
  situ[total:] = 0
  return ragged_dot(situ, expert_down, group_sizes, dtype)


# ----------------------------------------------------------------------------
# MXFP4  (MXD:26-67, MXO:65-91)
# ----------------------------------------------------------------------------

FP4_E2M1_TABLE = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)  # MXD:26


def dequantize_mxfp4(weight_packed: np.ndarray, weight_scale: np.ndarray) -> np.ndarray:
  """MXD:29-67: (N, K/2) u8 e2m1 codes (low nibble = even K) and (N, K/gs) u8
  E8M0 scales -> (N, K) float32.  Nibble 8 decodes to -0.0 (sign applied as a
  sign bit, MXO:65-75); the scale is 2^(s-127) with the exponent taken through
  bfloat16 (MXD:54-64), which is exact for every integer exponent in range."""
  n, half = weight_packed.shape
  k = half * 2
  groups = weight_scale.shape[1]
  gs = k // groups
  p = weight_packed.astype(np.uint8)
  codes = np.stack([p & 0x0F, (p >> 4) & 0x0F], axis=-1).reshape(n, k)
  mag = FP4_E2M1_TABLE[codes & 0x07]
  sign_bits = ((codes & 0x08).astype(np.uint32) << 28)
  values = (mag.view(np.uint32) | sign_bits).view(np.float32)
  exp = bf16_round((weight_scale.astype(np.int32) - 127).astype(np.float32))
  scale = np.power(np.float32(2.0), exp).astype(np.float32)
  return (values * np.repeat(scale, gs, axis=1)).astype(np.float32)


class LazyMXFP4Experts:
  """Expert weights held as MXFP4 (E, N, K/2) codes + (E, N, K/32) scales in
  the checkpoint's (out, in) layout, presented to `ragged_dot` /
  `latent_moe_forward` as the (E, K, N) float32 array of their dequantised
  transposes (rows [row0, row1) of N), dequantised per expert on first use and
  cached.  This is the reference's dequant-then-matmul path
  (05_ragged_dot_on_tpu/prepare_real_checkpoint_layer.py:181-216 dequantises the
  checkpoint, then the forward runs on the dense weights)."""

  def __init__(self, packed, scale, row0=0, row1=None):
    self.packed, self.scale = packed, scale
    self.row0 = row0
    self.row1 = packed.shape[1] if row1 is None else row1
    self._cache = {}

  @property
  def shape(self):
    return (self.packed.shape[0], self.packed.shape[2] * 2, self.row1 - self.row0)

  def __len__(self):
    return self.packed.shape[0]

  def __getitem__(self, e):
    e = int(e)
    w = self._cache.get(e)
    if w is None:
      w = np.ascontiguousarray(dequantize_mxfp4(self.packed[e, self.row0:self.row1],
                                                self.scale[e, self.row0:self.row1]).T)
      self._cache[e] = w
    return w


def mxfp4_ragged_dot(lhs, weight_packed, weight_scale, group_sizes, dtype="bf16"):
  """Dequant-then-matmul reference for the MXFP4 grouped matmul: weights
  (G, N, K/2) + (G, N, K/32) in the checkpoint's (out, in) layout."""
  m = lhs.shape[0]
  n = weight_packed.shape[1]
  out = np.zeros((m, n), np.float32)
  start = 0
  for g, size in enumerate(np.asarray(group_sizes).tolist()):
    size = int(size)
    if size > 0:
      w = dequantize_mxfp4(weight_packed[g], weight_scale[g])  # (N, K)
      out[start:start + size] = np.matmul(lhs[start:start + size].astype(np.float32), w.T)
    start += size
  return to_dtype(out, dtype)


# ----------------------------------------------------------------------------
# fp8 (e4m3) block-quantised weights  (KRD:2714-2953)
# ----------------------------------------------------------------------------

FP8_E4M3_MAX = 448.0  # jnp.finfo(float8_e4m3fn).max


def e4m3_round(x: np.ndarray) -> np.ndarray:
  """float32 -> float8_e4m3fn (round to nearest even, as jnp's astype) -> float32."""
  return np.asarray(x, np.float32).astype(ml_dtypes.float8_e4m3fn).astype(np.float32)


def quantize_fp8_blockwise(rhs: np.ndarray, block_size: int):
  """The reference's weight quantisation for the rhs_scale API (KRD:2883-2898;
  block_size = K gives the whole-row form of KRD:2775-2786): per (group,
  K block, column) scale = absmax / 448 in f32, codes = e4m3(clip(w / scale)).
  rhs (G, K, N) -> (codes as float32 values (G, K, N), scale (G, K/block, N))."""
  rhs = np.asarray(rhs, np.float32)
  g, k, n = rhs.shape
  nb = k // block_size
  blocks = rhs.reshape(g, nb, block_size, n)
  scale = (np.abs(blocks).max(axis=2) / np.float32(FP8_E4M3_MAX)).astype(np.float32)
  with np.errstate(divide="ignore", invalid="ignore"):
    q = np.clip(blocks / scale[:, :, None, :], -FP8_E4M3_MAX, FP8_E4M3_MAX)
  q = e4m3_round(np.nan_to_num(q, nan=0.0))
  return q.reshape(g, k, n), scale


def dequantize_fp8_blockwise(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
  """bf16(f32(q) * scale) per K block: the dequantised weight the reference
  compares the quantised op against (KRD:2815, 2923-2924)."""
  g, k, n = q.shape
  nb = scale.shape[1]
  w = q.reshape(g, nb, k // nb, n).astype(np.float32) * scale.reshape(g, nb, 1, n)
  return bf16_round(w.reshape(g, k, n))


def fp8_ragged_dot(lhs, q, scale, group_sizes, dtype="bf16"):
  """ragged_dot(lhs, dequantize_fp8_blockwise(q, scale)) (KRD:2816-2821, 2925-2931)."""
  return ragged_dot(lhs, dequantize_fp8_blockwise(q, scale), group_sizes, dtype=dtype)


# ----------------------------------------------------------------------------
# MXFP8 activations x MXFP4 weights: the block-scaled fast path
# ----------------------------------------------------------------------------
# The reference's operator has a hook for quantising the activations inside
# the grouped matmul (`maybe_quantize_lhs`, KRD:257-263, 2749-2757) but never
# exercises it; its MXFP4 weights are always dequantised first (MXD:29-67).
# The fast path quantises each activation row to MXFP8 (OCP microscaling:
# one E8M0 power-of-two scale per 32 consecutive K values, e4m3 elements)
# and multiplies it with the MXFP4 weights on the block-scaled tensor core.
# Scale rule: the smallest power of two 2^e with amax <= 448 * 2^e (so no
# element saturates), elements rounded to nearest even in e4m3.


def mxfp8_scale_exponent(amax: np.ndarray) -> np.ndarray:
  """Per-block exponent e (int32) with amax <= 448 * 2^e, the smallest such:
  with amax = f * 2^E (f in [1, 2)), e = E - 8, or E - 7 when f > 1.75.
  amax == 0 gives -127 (E8M0 byte 0).  Clamped to [-127, 127]."""
  a = np.asarray(amax, np.float32)
  bits = a.view(np.uint32)
  E = ((bits >> 23) & 0xFF).astype(np.int32) - 127
  mant = (bits & 0x7FFFFF).astype(np.int64)
  e = E - 8 + (mant > 0x600000).astype(np.int32)
  e = np.where(a == 0, -127, e)
  return np.clip(e, -127, 127).astype(np.int32)


def quantize_mxfp8(x: np.ndarray, block: int = 32):
  """(rows, K) float32 -> (e4m3 values as float32 (rows, K), E8M0 bytes
  (rows, K / block) uint8); x ~= values * 2^(byte - 127) blockwise."""
  x = np.asarray(x, np.float32)
  r, k = x.shape
  xb = x.reshape(r, k // block, block)
  e = mxfp8_scale_exponent(np.abs(xb).max(axis=2))
  q = e4m3_round(xb * np.ldexp(np.float32(1.0), -e)[:, :, None].astype(np.float32))
  return q.reshape(r, k), (e + 127).astype(np.uint8)


def dequantize_mxfp8(q: np.ndarray, sf: np.ndarray, block: int = 32) -> np.ndarray:
  r, k = q.shape
  scale = np.ldexp(np.float32(1.0), sf.astype(np.int32) - 127).astype(np.float32)
  return (q.reshape(r, k // block, block) * scale[:, :, None]).reshape(r, k).astype(np.float32)


# MXFP4 activations (kind::mxf4): the same blocks and scale rule with e2m1
# elements -- the smallest 2^e with amax <= 6 * 2^e (e2m1's largest finite is
# 6 = 1.5 * 2^2), values rounded to nearest even on the e2m1 grid; a row of K
# values is stored as K/2 bytes, the even K index in the low nibble (the
# packing of the MXFP4 weights, MXD:29-40).

FP4_E2M1_MAX = 6.0


def mxfp4_act_scale_exponent(amax: np.ndarray) -> np.ndarray:
  """Per-block exponent e (int32) with amax <= 6 * 2^e, the smallest such:
  with amax = f * 2^E (f in [1, 2)), e = E - 2, or E - 1 when f > 1.5.
  amax == 0 gives -127 (E8M0 byte 0).  Clamped to [-127, 127]."""
  a = np.asarray(amax, np.float32)
  bits = a.view(np.uint32)
  E = ((bits >> 23) & 0xFF).astype(np.int32) - 127
  mant = (bits & 0x7FFFFF).astype(np.int64)
  e = E - 2 + (mant > 0x400000).astype(np.int32)
  e = np.where(a == 0, -127, e)
  return np.clip(e, -127, 127).astype(np.int32)


def e2m1_round(x: np.ndarray) -> np.ndarray:
  """float32 -> e2m1 (round to nearest even; the sign of a value rounded to
  zero is kept) -> float32."""
  return np.asarray(x, np.float32).astype(ml_dtypes.float4_e2m1fn).astype(np.float32)


def quantize_mxfp4_act(x: np.ndarray, block: int = 32):
  """(rows, K) float32 -> (e2m1 values as float32 (rows, K), E8M0 bytes
  (rows, K / block) uint8); x ~= values * 2^(byte - 127) blockwise."""
  x = np.asarray(x, np.float32)
  r, k = x.shape
  xb = x.reshape(r, k // block, block)
  e = mxfp4_act_scale_exponent(np.abs(xb).max(axis=2))
  q = e2m1_round(xb * np.ldexp(np.float32(1.0), -e)[:, :, None].astype(np.float32))
  return q.reshape(r, k), (e + 127).astype(np.uint8)


def pack_e2m1(values: np.ndarray) -> np.ndarray:
  """(rows, K) e2m1 values (float32) -> (rows, K/2) bytes: code = sign bit 3
  | grid index (FP4_E2M1_TABLE), the even K index in the low nibble."""
  codes = np.asarray(values, np.float32).astype(ml_dtypes.float4_e2m1fn).view(np.uint8) & 0x0F
  return (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)


# The exact form on the same tensor core: each row split into two e4m3 planes
# under the MXFP8 block scale 2^e -- hi = e4m3(x / 2^e), lo = e4m3(x / 2^e -
# hi), both rounded to nearest even.  A bf16 value has 8 significant bits;
# hi takes the top 4 (rounded), and the remainder is a multiple of the value's
# bf16 spacing no larger than half hi's spacing, so it has at most 4
# significant bits: e4m3 holds it exactly whenever it is not below e4m3's
# subnormal step 2^-9, i.e. for |x| >= 2^(e-2).  hi + lo is then x itself, and
# the GEMM on both planes is the exact product.


def split_e4m3(x: np.ndarray, block: int = 32):
  """(rows, K) float32 -> (hi values (rows, K), lo values (rows, K), E8M0
  bytes (rows, K / block)) with x ~= (hi + lo) * 2^(byte - 127) blockwise."""
  x = np.asarray(x, np.float32)
  r, k = x.shape
  xb = x.reshape(r, k // block, block)
  e = mxfp8_scale_exponent(np.abs(xb).max(axis=2))
  v = (xb * np.ldexp(np.float32(1.0), -e)[:, :, None].astype(np.float32)).astype(np.float32)
  hi = e4m3_round(v)
  lo = e4m3_round((v - hi).astype(np.float32))
  return hi.reshape(r, k), lo.reshape(r, k), (e + 127).astype(np.uint8)


def dequantize_split(hi: np.ndarray, lo: np.ndarray, sf: np.ndarray, block: int = 32):
  """(hi + lo) * 2^(byte - 127) per block, in float32 (exact: hi + lo has at
  most 8 significant bits)."""
  return dequantize_mxfp8((hi + lo).astype(np.float32), sf, block)


def mxfp8_mxfp4_ragged_dot(lhs_q, lhs_sf, weight_packed, weight_scale, group_sizes):
  """f32 result of the block-scaled grouped matmul: the dequantised MXFP8
  rows times the dequantised MXFP4 weights (every product is exact in f32;
  only the summation order can differ).  weight (G, N, K/2) codes + (G, N,
  K/32) scales in the checkpoint's (out, in) layout."""
  lhs = dequantize_mxfp8(lhs_q, lhs_sf)
  return ragged_dot(lhs, LazyMXFP4Experts(weight_packed, weight_scale), group_sizes, dtype="fp32")


def mxfp4_mxfp4_ragged_dot(lhs_q, lhs_sf, weight_packed, weight_scale, group_sizes):
  """The same for MXFP4 activation rows (e2m1 values as float32, E8M0 bytes):
  every product is again exact in f32."""
  return mxfp8_mxfp4_ragged_dot(lhs_q, lhs_sf, weight_packed, weight_scale, group_sizes)


# ----------------------------------------------------------------------------
# comparison metrics  (05_ragged_dot_on_tpu/hw_session_common.py:193-225)
# ----------------------------------------------------------------------------


def error_report(ref: np.ndarray, got: np.ndarray, rel_floor: float = 1e-3) -> dict:
  """max_abs, rmse, relative_max_diff = max_abs / std(ref), element-wise
  relative error with a floor, non-finite count, number of differing elements."""
  ref = np.asarray(ref, np.float64)
  got = np.asarray(got, np.float64)
  diff = np.abs(ref - got)
  std = float(ref.std()) if ref.size else 0.0
  max_abs = float(diff.max()) if diff.size else 0.0
  return {
      "max_abs": max_abs,
      "rmse": float(np.sqrt(np.mean(diff ** 2))) if diff.size else 0.0,
      "relative_max_diff": max_abs / std if std > 0 else float("inf") if max_abs else 0.0,
      "max_rel": float((diff / np.maximum(np.abs(ref), rel_floor)).max()) if diff.size else 0.0,
      "nonfinite": int((~np.isfinite(got)).sum()),
      "n_diff": int((diff > 0).sum()),
  }


def canonical_slot_order(dispatch_order: np.ndarray, group_sizes: np.ndarray, top_k: int):
  """06_.../test_jax_reference_against_pytorch_golden.py:278-289: re-sort
  per-dispatch-slot arrays by (expert_id, token_id)."""
  token_ids = np.asarray(dispatch_order) // top_k
  expert_of_slot = np.repeat(np.arange(len(group_sizes)), np.asarray(group_sizes))
  return np.lexsort((token_ids, expert_of_slot)), token_ids
