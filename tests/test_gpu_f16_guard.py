"""The f16-operand path's range guard.

On the f16-operand path the MXFP4 kernels read the latent rows as f16 that
carry bf16-rounded values.  That is exact for magnitudes up to 65504; a larger
value would silently become inf, and a row whose values are all tiny would
lose precision in the f16 subnormals.  The kernels that write f16 operands
(the dense GEMM's f16 output, the converting row gather) record
LMOE_F16_RANGE in the device status word in both cases, and the layer
forward has a bf16-operand mode (`mxfp4_operand="bf16"`) that carries such
rows exactly.  The default mode (`"auto"` = `"split"`, the block-scaled
kernels on two e4m3 planes under a per-32-value power-of-two scale) has no
such range: it matches the bf16 mode on the same inputs and records nothing.  Reference: the latent x is held in the compute dtype, bf16
(05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:365)."""

import numpy as np
import pytest
import torch

from oracle import lmoe_oracle as O
from tests.gpu_util import assert_bf16_close, routing_agreement, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm():
  import tokamax_tpu_kernel_lab_b200 as lm
  lm.load_native()
  return lm


def _status(lm):
  from tokamax_tpu_kernel_lab_b200 import ops
  torch.cuda.synchronize()
  return int(ops.device_status().item())


def _clear(lm):
  from tokamax_tpu_kernel_lab_b200 import ops
  torch.cuda.synchronize()
  ops.device_status().zero_()


def test_f16_output_above_65504_is_flagged(lm):
  from tokamax_tpu_kernel_lab_b200 import _native
  _clear(lm)
  a = torch.zeros(256, 128, dtype=torch.bfloat16, device="cuda")
  w = torch.zeros(256, 128, dtype=torch.bfloat16, device="cuda")
  a[:, 0] = 1.0
  w[:, 0] = 0.5
  out = lm.gemm(a, w, out_dtype=torch.float16)
  assert _status(lm) == 0 and bool((out == 0.5).all())
  a[7, 0] = 256.0
  w[3, 0] = 273.0  # 69888: a bf16 value above f16's largest finite
  out = lm.gemm(a, w, out_dtype=torch.float16)
  assert _status(lm) == _native.LMOE_F16_RANGE
  assert torch.isinf(out[7, 3])
  _clear(lm)
  with pytest.raises(_native.LmoeError):
    lm.gemm(a, w, out_dtype=torch.float16)
    lm.check_device_status()
  _clear(lm)


def test_f16_output_of_a_tiny_row_is_flagged(lm):
  from tokamax_tpu_kernel_lab_b200 import _native
  _clear(lm)
  rng = np.random.default_rng(1)
  a = to_dev(rng.standard_normal((128, 256)).astype(np.float32))
  w = to_dev(rng.standard_normal((128, 256)).astype(np.float32) * 0.02)
  lm.gemm(a, w, out_dtype=torch.float16)
  assert _status(lm) == 0  # ordinary rows: values near zero occur, runs of them do not
  a[5] = a[5] * 1e-6       # one token whose whole latent row is ~1e-6
  lm.gemm(a, w, out_dtype=torch.float16)
  assert _status(lm) == _native.LMOE_F16_RANGE
  _clear(lm)


def test_converting_gather_flags_out_of_range_rows(lm):
  from tokamax_tpu_kernel_lab_b200 import _native
  _clear(lm)
  gen = torch.Generator(device="cuda").manual_seed(7)
  x = torch.randn(64, 512, generator=gen, device="cuda").to(torch.bfloat16)
  idx = torch.arange(64, dtype=torch.int32, device="cuda").flip(0)
  out = lm.gather_rows(x, idx, to_f16=True)
  assert _status(lm) == 0
  # round-to-nearest-even bf16 -> f16 (exact except below 2^-17, where the
  # f16 subnormal spacing 2^-24 rounds)
  assert torch.equal(out, x.flip(0).to(torch.float16))
  x[10, 100] = 7e4
  lm.gather_rows(x, idx, to_f16=True)
  assert _status(lm) == _native.LMOE_F16_RANGE
  _clear(lm)
  x[10, 100] = 1.0
  x[20] = x[20] * 1e-7
  lm.gather_rows(x, idx, to_f16=True)
  assert _status(lm) == _native.LMOE_F16_RANGE
  _clear(lm)


def _mx_layer(lm):
  cfg = lm.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  pw = lm.init_prepared_mxfp4(cfg, seed=12, bias_std=0.5)
  return cfg, pw


def _oracle_weights(pw, cfg):
  npf = lambda t: t.float().cpu().numpy()
  I = cfg.intermediate_size
  si = I * cfg.num_shared_experts
  gu_p, gu_s = pw.expert_gu_mx.packed.cpu().numpy(), pw.expert_gu_mx.scale.cpu().numpy()
  dn_p, dn_s = pw.expert_down_mx.packed.cpu().numpy(), pw.expert_down_mx.scale.cpu().numpy()
  return O.Weights(
      router_weight=npf(pw.router).T, e_score_correction_bias=npf(pw.bias),
      down_proj=npf(pw.down).T, up_proj=npf(pw.up).T,
      expert_gate=O.LazyMXFP4Experts(gu_p, gu_s, 0, I),
      expert_up=O.LazyMXFP4Experts(gu_p, gu_s, I, 2 * I),
      expert_down=O.LazyMXFP4Experts(dn_p, dn_s),
      norm_scale=npf(pw.norm_scale),
      shared_gate=npf(pw.shared_gu)[:si].T, shared_up=npf(pw.shared_gu)[si:].T,
      shared_down=npf(pw.shared_down).T)


def _oracle_forward(cfg, pw, h):
  ocfg = O.LatentMoEConfig(cfg.hidden_size, cfg.latent_size, cfg.intermediate_size,
                           cfg.num_experts, cfg.top_k, cfg.num_shared_experts)
  return O.latent_moe_forward(to_np(h), _oracle_weights(pw, cfg), ocfg, dtype="bf16",
                              return_intermediates=True)


def _assert_default_mode_matches(lm, h, pw, cfg, exact):
  """The default (split) forward on the same inputs records nothing and
  matches the bf16-operand forward `exact` at the bf16 tolerance, on the
  scale of each token's own output."""
  _clear(lm)
  got = to_np(lm.latent_moe_forward(h, pw, cfg))
  assert _status(lm) == 0
  scale = np.abs(exact).max(axis=1, keepdims=True)
  assert_bf16_close(exact / scale, got / scale, "default (split) mode, per-token scale")


def test_layer_with_huge_latent_values_flags_and_bf16_mode_is_exact(lm):
  """Token 0's hidden state is scaled so its latent row reaches ~1e5: the
  default (f16) path records LMOE_F16_RANGE; mxfp4_operand="bf16" runs the
  same forward on bf16 operands and matches the oracle, token 0 included."""
  from tokamax_tpu_kernel_lab_b200 import _native
  cfg, pw = _mx_layer(lm)
  assert lm.latent_moe.mxfp4_f16_path(pw)
  gen = torch.Generator(device="cuda").manual_seed(12)
  h = torch.randn(256, cfg.hidden_size, generator=gen, device="cuda")
  h[0] *= 40000.0
  h = h.to(torch.bfloat16)
  _clear(lm)
  lm.latent_moe_forward(h, pw, cfg, mxfp4_operand="f16")
  assert _status(lm) == _native.LMOE_F16_RANGE
  _clear(lm)
  final, inter = lm.latent_moe_forward(h, pw, cfg, mxfp4_operand="bf16",
                                       return_intermediates=True)
  assert _status(lm) == 0
  assert inter["latent_projection"].dtype == torch.bfloat16
  assert float(inter["latent_projection"][0].float().abs().max()) > 65504
  ref, rinter = _oracle_forward(cfg, pw, h)
  same = routing_agreement(inter["topk_indices"].cpu().numpy(),
                           rinter["router_scores_for_choice"], rinter["topk_indices"])
  assert same[0]
  got = to_np(final)
  # token 0's output is ~100 in magnitude (bf16 spacing 0.5 there): it is
  # compared on its own scale, the other tokens at the standard bar
  s0 = float(np.abs(ref[0]).max())
  assert_bf16_close(ref[0] / s0, got[0] / s0, "the huge token, on its own scale")
  rest = same.copy()
  rest[0] = False
  assert_bf16_close(ref[rest], got[rest], "bf16-operand layer, other tokens")
  _assert_default_mode_matches(lm, h, pw, cfg, got)


def test_layer_with_tiny_rows_flags_and_bf16_mode_is_exact(lm):
  """Hidden states scaled by 3e-3: the latent rows (~2e-3) still fit f16, but
  the SiTU activations (~gate * up / 2, ~4e-7) would sit deep in the f16
  subnormals, where they keep only a few bits.  The gate/up kernel flags the
  runs as LMOE_F16_RANGE; mxfp4_operand="bf16" matches the oracle."""
  from tokamax_tpu_kernel_lab_b200 import _native
  cfg, pw = _mx_layer(lm)
  gen = torch.Generator(device="cuda").manual_seed(13)
  h = (torch.randn(256, cfg.hidden_size, generator=gen, device="cuda") * 3e-3).to(torch.bfloat16)
  _clear(lm)
  lm.latent_moe_forward(h, pw, cfg, mxfp4_operand="f16")
  assert _status(lm) == _native.LMOE_F16_RANGE
  _clear(lm)
  final, inter = lm.latent_moe_forward(h, pw, cfg, mxfp4_operand="bf16",
                                       return_intermediates=True)
  assert _status(lm) == 0
  ref, rinter = _oracle_forward(cfg, pw, h)
  same = routing_agreement(inter["topk_indices"].cpu().numpy(),
                           rinter["router_scores_for_choice"], rinter["topk_indices"])
  s0 = float(np.abs(ref).max())  # outputs ~1e-4: compared on their own scale
  assert_bf16_close(ref[same] / s0, to_np(final)[same] / s0, "bf16-operand layer, tiny rows")
  _assert_default_mode_matches(lm, h, pw, cfg, to_np(final))


def test_layer_with_small_latent_values_matches_oracle(lm):
  """Ordinary N(0, 1) hidden states: some latent values and activations fall
  below 2^-14 (f16 subnormals, exact down to 2^-17, within 2^-25 below) but
  no whole run does, so the f16 path raises nothing and matches the bf16
  oracle at the standard tolerance."""
  cfg, pw = _mx_layer(lm)
  gen = torch.Generator(device="cuda").manual_seed(14)
  h = torch.randn(256, cfg.hidden_size, generator=gen, device="cuda").to(torch.bfloat16)
  _clear(lm)
  final, inter = lm.latent_moe_forward(h, pw, cfg, return_intermediates=True,
                                       mxfp4_operand="f16")
  assert _status(lm) == 0
  x, act = inter["latent_projection"], inter["situ_output"]
  assert x.dtype == torch.float16 and act.dtype == torch.float16
  sub = lambda t: int(((t.float().abs() < 6.1e-5) & (t != 0)).sum())
  assert sub(x) + sub(act) > 0
  ref, rinter = _oracle_forward(cfg, pw, h)
  same = routing_agreement(inter["topk_indices"].cpu().numpy(),
                           rinter["router_scores_for_choice"], rinter["topk_indices"])
  assert_bf16_close(ref[same], to_np(final)[same], "f16 layer with subnormal values")
