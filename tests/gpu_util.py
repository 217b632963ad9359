"""Helpers shared by the GPU parity tests (import only from tests)."""

import numpy as np
import torch

from oracle import lmoe_oracle as O

# bf16 outputs within max-abs 2e-2 and relative 1e-2 of
# the f32 reference; relative = max_abs / std(reference) (the reference's
# relative_max_diff, 05_ragged_dot_on_tpu/hw_session_common.py:193-225).
BF16_MAX_ABS = 2e-2
BF16_REL = 1e-2


def to_dev(a: np.ndarray, dtype=torch.bfloat16) -> torch.Tensor:
  return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda").to(dtype)


def to_np(t: torch.Tensor) -> np.ndarray:
  return t.detach().float().cpu().numpy()


def assert_bf16_close(ref: np.ndarray, got: np.ndarray, what: str = "",
                      max_abs: float = BF16_MAX_ABS, rel: float = BF16_REL) -> dict:
  rep = O.error_report(ref, got)
  assert rep["nonfinite"] == 0, f"{what}: non-finite outputs {rep}"
  assert rep["max_abs"] <= max_abs, f"{what}: {rep}"
  assert rep["relative_max_diff"] <= rel, f"{what}: {rep}"
  return rep


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
