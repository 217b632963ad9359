"""Parity at the benchmarked sizes.

- Configuration 5 (the bench line): the full LatentMoE layer over 16384 tokens,
  896 MXFP4 experts, router bias N(0, 0.5^2), run as one batch on the GPU; a
  seeded sample of tokens is re-run through the CPU oracle on those tokens
  alone (the dropless forward is per-token independent) and compared.
- Configuration 3: the bf16 fused gate/up + SiTU-GLU grouped GEMM and the down
  grouped GEMM over 65536 routed rows and 896 experts, compared with the
  oracle on sampled rows of sampled non-empty experts.

Routing parity follows the end-to-end rule: a token's top-k set may differ
from the oracle's only where the oracle's k-th and (k+1)-th selection scores
are within 1e-5 (the logits are f32 sums in a different order); those
tokens are counted and left out of the output comparison, every other token
must match within the bf16 tolerance.
Reference: 05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:330-435."""

import numpy as np
import pytest
import torch

from oracle import lmoe_oracle as O
from tests.gpu_util import assert_bf16_allclose, assert_bf16_close, routing_agreement, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm():
  import tokamax_tpu_kernel_lab_b200 as lm
  lm.load_native()
  return lm


class _DeviceMXFP4Experts:
  """Oracle view of device-resident MXFP4 experts: (E, K, N) float32 of the
  dequantised transposes of rows [row0, row1), each expert copied to the host
  and dequantised on first use (only the experts the sample touches)."""

  def __init__(self, w, row0=0, row1=None):
    self.packed, self.scale = w.packed, w.scale
    self.row0 = row0
    self.row1 = w.packed.shape[1] if row1 is None else row1
    self._cache = {}

  @property
  def shape(self):
    return (self.packed.shape[0], self.packed.shape[2] * 2, self.row1 - self.row0)

  def __len__(self):
    return self.packed.shape[0]

  def __getitem__(self, e):
    e = int(e)
    if e not in self._cache:
      p = self.packed[e, self.row0:self.row1].cpu().numpy()
      s = self.scale[e, self.row0:self.row1].cpu().numpy()
      self._cache[e] = np.ascontiguousarray(O.dequantize_mxfp4(p, s).T)
    return self._cache[e]


def test_config5_full_layer_sampled_tokens_match_oracle(lm):
  cfg = lm.full_layer_config()
  pw = lm.init_prepared_mxfp4(cfg, seed=4, bias_std=0.5)
  gen = torch.Generator(device="cuda").manual_seed(4 * 7919)
  T = 16384
  h = torch.randn(T, cfg.hidden_size, generator=gen, device="cuda").to(torch.bfloat16)
  final, inter = lm.latent_moe_forward(h, pw, cfg, return_intermediates=True)
  torch.cuda.synchronize()
  lm.check_device_status()
  # the benchmarked skew: most rows land on a few dozen experts
  gs = inter["group_sizes"].cpu().numpy()
  assert gs.sum() == T * cfg.top_k and (gs == 0).sum() > cfg.num_experts // 2
  rng = np.random.default_rng(5)
  sample = np.sort(rng.choice(T, size=24, replace=False))
  npf = lambda t: t.float().cpu().numpy()
  I = cfg.intermediate_size
  si = I * cfg.num_shared_experts
  w = O.Weights(
      router_weight=npf(pw.router).T, e_score_correction_bias=npf(pw.bias),
      down_proj=npf(pw.down).T, up_proj=npf(pw.up).T,
      expert_gate=_DeviceMXFP4Experts(pw.expert_gu_mx, 0, I),
      expert_up=_DeviceMXFP4Experts(pw.expert_gu_mx, I, 2 * I),
      expert_down=_DeviceMXFP4Experts(pw.expert_down_mx),
      norm_scale=npf(pw.norm_scale),
      shared_gate=npf(pw.shared_gu)[:si].T, shared_up=npf(pw.shared_gu)[si:].T,
      shared_down=npf(pw.shared_down).T)
  ocfg = O.LatentMoEConfig(cfg.hidden_size, cfg.latent_size, I, cfg.num_experts, cfg.top_k,
                           cfg.num_shared_experts)
  hs = npf(h[torch.from_numpy(sample).cuda()])
  ref, rinter = O.latent_moe_forward(hs, w, ocfg, dtype="bf16", return_intermediates=True)
  got_idx = inter["topk_indices"].cpu().numpy()[sample]
  same = routing_agreement(got_idx, rinter["router_scores_for_choice"], rinter["topk_indices"])
  sel = lambda name: to_np(inter[name])[sample][same]
  # every stage: per element |d| <= 2e-2 + 1e-2 |ref| (the RMS-normalised
  # values and the dense branches reach 4-8, where one bf16 spacing is 1/32)
  # and 1e-2 normwise
  for name in ("routed_output_after_combine", "normalized_output"):
    assert_bf16_allclose(rinter[name][same], sel(name), f"config 5 {name}")
  upo, shr = rinter["up_projection_output"][same], rinter["shared_expert_output"][same]
  assert_bf16_allclose(upo, sel("up_projection_output"), "config 5 up-projection")
  assert_bf16_allclose(shr, sel("shared_expert_output"), "config 5 shared expert")
  # the output is bf16(upo + shared): where the two cancel, their own one-ulp
  # differences remain, so the per-element bound scales with |upo| + |shared|
  got = to_np(final)[sample][same]
  ref_f = ref[same]
  bound = 2e-2 + 1e-2 * (np.abs(upo) + np.abs(shr))
  assert np.all(np.abs(got - ref_f) <= bound), float((np.abs(got - ref_f) - bound).max())
  assert float(np.abs(got - ref_f).max() / np.abs(ref_f).max()) <= 1e-2


def test_config3_bf16_fused_gateup_and_down_full_size(lm):
  """65536 routed rows (4096 tokens x top-16) over 896 experts, latent 2048,
  intermediate 1024: the routed rows go through the fused gate/up + SiTU-GLU
  grouped GEMM and the down grouped GEMM exactly as the layer runs them."""
  E, L, I, T, k = 896, 2048, 1024, 4096, 16
  gen = torch.Generator(device="cuda").manual_seed(2)
  x = torch.randn(T, L, generator=gen, device="cuda").to(torch.bfloat16)
  wr = (torch.randn(E, L, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
  bias = torch.randn(E, generator=gen, device="cuda") * 0.5
  idx, wts = lm.router_gate(x, wr, bias, k)
  d = lm.dispatch(idx, wts, E)
  rows = lm.gather_rows(x, d.token_idx)
  w_gu = torch.empty(E, 2 * I, L, dtype=torch.bfloat16, device="cuda")
  w_dn = torch.empty(E, L, I, dtype=torch.bfloat16, device="cuda")
  for e0 in range(0, E, 64):  # chunked to keep the f32 temporaries small
    w_gu[e0:e0 + 64] = (torch.randn(64, 2 * I, L, generator=gen, device="cuda") * 0.02).to(
        torch.bfloat16)
    w_dn[e0:e0 + 64] = (torch.randn(64, L, I, generator=gen, device="cuda") * 0.02).to(
        torch.bfloat16)
  act = lm.fused_gateup_situ(rows, w_gu, d.group_sizes, beta=4.0, linear_beta=25.0,
                             round_gate_up=True, rhs_layout="gnk")
  down = lm.ragged_dot(act, w_dn, d.group_sizes, rhs_layout="gnk")
  torch.cuda.synchronize()
  lm.check_device_status()
  gs = d.group_sizes.cpu().numpy()
  assert gs.sum() == T * k
  off = np.concatenate([[0], np.cumsum(gs)])
  rng = np.random.default_rng(3)
  nonempty = np.nonzero(gs)[0]
  groups = rng.choice(nonempty, size=min(24, len(nonempty)), replace=False)
  sel = []
  for g in groups:
    n = int(gs[g])
    picks = {0, n - 1} | set(rng.integers(0, n, size=2).tolist())
    sel += [int(off[g]) + p for p in sorted(picks)]
  sel = np.array(sel)
  ref_act = np.empty((len(sel), I), np.float32)
  ref_down = np.empty((len(sel), L), np.float32)
  rows_np = to_np(rows[torch.from_numpy(sel).cuda()])
  act_np = to_np(act[torch.from_numpy(sel).cuda()])
  i = 0
  for g in groups:
    n = int(np.sum((sel >= off[g]) & (sel < off[g + 1])))
    gu = to_np(w_gu[g]).T[None]   # (1, L, 2I)
    dn = to_np(w_dn[g]).T[None]   # (1, I, L)
    one = np.array([n], np.int32)
    ref_act[i:i + n] = O.fused_gateup_situ(rows_np[i:i + n], gu, one, I, 4.0, 25.0, dtype="bf16",
                                           round_gate_up=True)
    # the down GEMM is checked on the kernel's own activations (its input)
    ref_down[i:i + n] = O.ragged_dot(act_np[i:i + n], dn, one, dtype="fp32")
    i += n
  assert_bf16_close(ref_act, act_np, "config 3 gate/up + SiTU")
  s = float(np.abs(ref_down).max())
  assert_bf16_close(ref_down / s, to_np(down[torch.from_numpy(sel).cuda()]) / s,
                    "config 3 down", rel_std=2e-2)
  # rows past sum(group_sizes): none here (dropless, every row routed)
  assert down.shape[0] == T * k
