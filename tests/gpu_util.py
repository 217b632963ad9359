"""Helpers shared by the GPU parity tests (import only from tests)."""

import numpy as np
import torch

from oracle import lmoe_oracle as O

# Tolerance for bf16 outputs against the f32 reference:
#   max_abs                     <= 2e-2
#   max_abs / max|reference|    <= 1e-2   (normwise relative error)
#   max_abs / std(reference)    <= 2e-2   for plain matmul outputs (the reference's
#       own `relative_max_diff` bar, mxfp4_online_dequant_matmul_pallas.py:254-268;
#       rounding a bf16 output alone costs ~0.015 on this metric, so 1e-2 on it
#       would reject an exact kernel).  Not applied to heavy-tailed outputs
#       (SiTU activations, the layer output), whose std is far below their peak.
BF16_MAX_ABS = 2e-2
BF16_REL = 1e-2
GEMM_REL_STD = 2e-2


def to_dev(a: np.ndarray, dtype=torch.bfloat16) -> torch.Tensor:
  return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda").to(dtype)


def to_np(t: torch.Tensor) -> np.ndarray:
  return t.detach().float().cpu().numpy()


def assert_bf16_close(ref: np.ndarray, got: np.ndarray, what: str = "",
                      max_abs: float = BF16_MAX_ABS, rel: float = BF16_REL,
                      rel_std: float | None = None) -> dict:
  rep = O.error_report(ref, got)
  peak = float(np.abs(np.asarray(ref, np.float64)).max()) if np.size(ref) else 0.0
  rep["normwise_rel"] = rep["max_abs"] / peak if peak > 0 else 0.0
  assert rep["nonfinite"] == 0, f"{what}: non-finite outputs {rep}"
  assert rep["max_abs"] <= max_abs, f"{what}: {rep}"
  assert rep["normwise_rel"] <= rel, f"{what}: {rep}"
  if rel_std is not None:
    assert rep["relative_max_diff"] <= rel_std, f"{what}: {rep}"
  return rep


def assert_bf16_allclose(ref: np.ndarray, got: np.ndarray, what: str = "",
                         atol: float = BF16_MAX_ABS, rtol: float = BF16_REL) -> dict:
  """Element-wise |got - ref| <= atol + rtol * |ref| (numpy allclose) and
  max_abs / max|ref| <= rtol.  For outputs that reach magnitudes of several
  units (the full configuration-5 layer), where one bf16 spacing (1/32 in
  [4, 8)) alone exceeds a flat 2e-2 bound."""
  rep = O.error_report(ref, got)
  r = np.asarray(ref, np.float64)
  peak = float(np.abs(r).max()) if np.size(ref) else 0.0
  rep["normwise_rel"] = rep["max_abs"] / peak if peak > 0 else 0.0
  excess = np.abs(np.asarray(got, np.float64) - r) - (atol + rtol * np.abs(r))
  rep["allclose_violations"] = int((excess > 0).sum())
  assert rep["nonfinite"] == 0, f"{what}: non-finite outputs {rep}"
  assert rep["allclose_violations"] == 0, f"{what}: {rep}"
  assert rep["normwise_rel"] <= rtol, f"{what}: {rep}"
  return rep


def assert_gemm_close(ref: np.ndarray, got: np.ndarray, what: str = "") -> dict:
  """bf16 tolerance plus the std-based bar for plain matmul outputs."""
  return assert_bf16_close(ref, got, what, rel_std=GEMM_REL_STD)


# End-to-end routing parity: a token's top-k set may differ from the oracle's
# only where the oracle's k-th and (k+1)-th selection scores are this close
# (the router logits are f32 sums in a different order on the GPU).
NEAR_TIE = 1e-5


def routing_agreement(got_idx: np.ndarray, sfc: np.ndarray, ref_idx: np.ndarray,
                      max_mismatch: int | None = None) -> np.ndarray:
  """Boolean mask of the tokens whose selected expert set equals the
  oracle's.  Every other token must be a near-tie (gap < NEAR_TIE), and at
  most `max_mismatch` of them may differ (default: 1% of the tokens, at
  least 2)."""
  k = ref_idx.shape[1]
  same = np.all(np.sort(got_idx, -1) == np.sort(ref_idx, -1), axis=1)
  if not same.all():
    srt = -np.sort(-np.asarray(sfc, np.float32), axis=1)
    gap = srt[:, k - 1] - srt[:, k] if k < srt.shape[1] else np.full(len(same), np.inf)
    bad = (~same) & (gap >= NEAR_TIE)
    assert not bad.any(), f"{int(bad.sum())} tokens differ beyond near-ties: gaps {gap[bad][:5]}"
  limit = max(2, len(same) // 100) if max_mismatch is None else max_mismatch
  assert int((~same).sum()) <= limit, f"{int((~same).sum())} near-tie mismatches"
  return same


def zipf_group_sizes(rng: np.random.Generator, m: int, g: int, s: float = 1.1,
                     n_zero: int = 8) -> np.ndarray:
  """Zipf(s) multinomial over a seeded permutation of the groups, with n_zero
  groups forced empty and their mass renormalised (benchmark configuration 2)."""
  p = (np.arange(g) + 1.0) ** (-s)
  p = p[rng.permutation(g)]
  zero = rng.choice(g, size=min(n_zero, g - 1), replace=False)
  p[zero] = 0
  p /= p.sum()
  return rng.multinomial(m, p).astype(np.int32)


DISTRIBUTIONS = ("uniform", "mild_skew", "heavy_skew", "empty_groups", "single_dominant")


def distribution_sizes(name: str, m: int, g: int, rng: np.random.Generator) -> np.ndarray:
  """Group-size distributions of 05_ragged_dot_on_tpu/benchmark_harness.py:118-153."""
  if name == "uniform":
    p = np.full(g, 1.0 / g)
  elif name == "mild_skew":
    p = np.ones(g); p[0] = 2.0; p /= p.sum()
  elif name == "heavy_skew":
    p = np.ones(g); p[0] = float(g); p /= p.sum()
  elif name == "empty_groups":
    half = max(g // 2, 1)
    p = np.array([1.0] * half + [0.0] * (g - half)); p /= p.sum()
  elif name == "single_dominant":
    p = np.zeros(g); p[0] = 1.0
  else:
    raise ValueError(name)
  return rng.multinomial(m, p).astype(np.int32)
