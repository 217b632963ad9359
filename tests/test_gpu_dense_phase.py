"""The per-phase dense kernels (persistent split-K, one launch per phase) for
small token counts, against the oracle's arithmetic:

- input phase (kimi_k3_latent_moe_reference.py:347-365, 428-433): router
  logits f32, the latent rows bf16, the shared expert's SiTU-GLU activation
  with bf16-rounded gate/up (own_gateup_situ_pallas_kernel.py:116-125);
- output phase (kimi_k3_latent_moe_reference.py:419-435): the up-projection
  plus the shared expert's down projection, summed in f32 and rounded once;
- the layer forward that uses them: against the oracle forward, against the
  same forward with the phases off, bit-identical across calls, across batch
  sizes (the split count does not depend on the token count) and under
  CUDA-graph replay.

Tolerances: f32 logits within 1e-5 of the largest |logit| (f32 sums of the
same bf16 products in another order); bf16 outputs at the bf16 tolerance of
tests/gpu_util.py."""

import numpy as np
import pytest
import torch

from oracle import lmoe_oracle as O
from tests.gpu_util import assert_bf16_close, assert_gemm_close, routing_agreement, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm():
  import tokamax_tpu_kernel_lab_b200 as lm
  lm.load_native()
  return lm


def _ops():
  from tokamax_tpu_kernel_lab_b200 import ops
  return ops


def _bf16(rng, *shape, scale=1.0):
  return O.bf16_round(rng.standard_normal(shape, dtype=np.float32) * np.float32(scale))


@pytest.mark.parametrize("t,d,e,latent,si", [(128, 1024, 256, 512, 512), (77, 2048, 96, 256, 192),
                                             (256, 512, 64, 128, 64), (1, 1024, 128, 256, 128)])
def test_input_phase_matches_oracle(lm, t, d, e, latent, si):
  ops = _ops()
  rng = np.random.default_rng(t + d)
  h = _bf16(rng, t, d)
  wr, wd = _bf16(rng, e, d, scale=0.02), _bf16(rng, latent, d, scale=0.02)
  wgu = _bf16(rng, 2 * si, d, scale=0.02)
  logits, x, act = ops.dense_input_phase(to_dev(h), to_dev(wr), to_dev(wd), to_dev(wgu),
                                         beta=4.0, linear_beta=25.0, round_gate_up=True)
  torch.cuda.synchronize()
  lm.check_device_status()
  ref_logits = h @ wr.T
  err = float(np.abs(to_np(logits) - ref_logits).max() / np.abs(ref_logits).max())
  assert err <= 1e-5, f"logits normwise {err:.2e}"
  assert_gemm_close(h @ wd.T, to_np(x), "latent rows")
  g, u = O.bf16_round(h @ wgu[:si].T), O.bf16_round(h @ wgu[si:].T)
  ref_act = O.situ_and_mul(g, u, 4.0, 25.0, "fp32")
  assert_bf16_close(ref_act, to_np(act), "shared SiTU-GLU activation")


@pytest.mark.parametrize("t,latent,si,d", [(128, 512, 512, 1024), (200, 256, 128, 384),
                                           (3, 128, 64, 7168)])
def test_output_phase_matches_oracle(lm, t, latent, si, d):
  ops = _ops()
  rng = np.random.default_rng(t + latent)
  a0, a1 = _bf16(rng, t, latent), _bf16(rng, t, si)
  wu, wsd = _bf16(rng, d, latent, scale=0.02), _bf16(rng, d, si, scale=0.02)
  out = ops.dense_output_phase(to_dev(a0), to_dev(wu), to_dev(a1), to_dev(wsd))
  torch.cuda.synchronize()
  lm.check_device_status()
  assert_gemm_close(a0 @ wu.T + a1 @ wsd.T, to_np(out), "output phase")


def test_phases_reject_unsupported_shapes(lm):
  ops = _ops()
  h = torch.zeros(8, 100, dtype=torch.bfloat16, device="cuda")  # d % 64 != 0
  w = torch.zeros(64, 100, dtype=torch.bfloat16, device="cuda")
  with pytest.raises(NotImplementedError):
    ops.dense_input_phase(h, w, w, w)


def _layer(lm, seed):
  cfg = lm.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  return cfg, lm.init_prepared_mxfp4(cfg, seed=seed, bias_std=0.5)


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
      expert_down=O.LazyMXFP4Experts(dn_p, dn_s), norm_scale=npf(pw.norm_scale),
      shared_gate=npf(pw.shared_gu)[:si].T, shared_up=npf(pw.shared_gu)[si:].T,
      shared_down=npf(pw.shared_down).T)


def _routing(ops, pw, cfg, h, phases):
  """The layer's top-k under each router form: the logits of the input
  phase + router_topk, or the fused router."""
  if phases:
    logits, _, _ = ops.dense_input_phase(h, pw.router, pw.down, pw.shared_gu)
    return ops.router_topk(logits, pw.bias, cfg.top_k, renormalize=cfg.moe_renormalize,
                           routed_scaling_factor=cfg.routed_scaling_factor)[0]
  return ops.router_gate(h, pw.router, pw.bias, cfg.top_k, renormalize=cfg.moe_renormalize,
                         routed_scaling_factor=cfg.routed_scaling_factor)[0]


@pytest.mark.parametrize("t", [96, 200])
def test_layer_with_phases_matches_oracle_and_unfused(lm, t):
  ops = _ops()
  cfg, pw = _layer(lm, 31)
  gen = torch.Generator(device="cuda").manual_seed(31 + t)
  h = torch.randn(t, cfg.hidden_size, generator=gen, device="cuda").to(torch.bfloat16)
  assert lm.latent_moe._use_dense_phases(None, pw, cfg, t, h, torch.bfloat16, False)
  got = lm.latent_moe_forward(h, pw, cfg)
  unfused = lm.latent_moe_forward(h, pw, cfg, dense_phases=False)
  idx_p, idx_u = _routing(ops, pw, cfg, h, True), _routing(ops, pw, cfg, h, False)
  torch.cuda.synchronize()
  lm.check_device_status()
  ocfg = O.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  ref, rinter = O.latent_moe_forward(to_np(h), _oracle_weights(pw, cfg), ocfg, dtype="bf16",
                                     return_intermediates=True)
  sfc, ridx = rinter["router_scores_for_choice"], rinter["topk_indices"]
  same = routing_agreement(idx_p.cpu().numpy(), sfc, ridx)
  same_u = routing_agreement(idx_u.cpu().numpy(), sfc, ridx)
  assert_bf16_close(ref[same], to_np(got)[same], "layer with dense phases vs oracle")
  both = same & same_u
  assert_bf16_close(to_np(unfused)[both], to_np(got)[both], "dense phases vs unfused forward")


def test_layer_with_phases_is_deterministic_batch_invariant_and_replays(lm):
  cfg, pw = _layer(lm, 33)
  gen = torch.Generator(device="cuda").manual_seed(33)
  h = torch.randn(200, cfg.hidden_size, generator=gen, device="cuda").to(torch.bfloat16)
  a = lm.latent_moe_forward(h, pw, cfg)
  b = lm.latent_moe_forward(h, pw, cfg)
  part = lm.latent_moe_forward(h[:70].contiguous(), pw, cfg)
  torch.cuda.synchronize()
  assert torch.equal(a, b)
  assert torch.equal(a[:70], part)
  static_h = h.clone()
  s = torch.cuda.Stream()
  s.wait_stream(torch.cuda.current_stream())
  with torch.cuda.stream(s):
    lm.latent_moe_forward(static_h, pw, cfg)
  torch.cuda.current_stream().wait_stream(s)
  graph = torch.cuda.CUDAGraph()
  with torch.cuda.graph(graph):
    out = lm.latent_moe_forward(static_h, pw, cfg)
  graph.replay()
  graph.replay()
  torch.cuda.synchronize()
  lm.check_device_status()
  assert torch.equal(out, a)


def test_config5_small_batch_with_phases(lm):
  """Configuration 5's shapes (d 7168, 896 experts, latent 2048, shared
  intermediate 2048) at 128 tokens: the default forward takes the phase
  kernels and agrees with the forward without them on every token whose
  routing agrees."""
  ops = _ops()
  cfg = lm.full_layer_config()
  pw = lm.init_prepared_mxfp4(cfg, seed=4, bias_std=0.5)
  gen = torch.Generator(device="cuda").manual_seed(4 * 7919 + 128)
  h = torch.randn(128, cfg.hidden_size, generator=gen, device="cuda").to(torch.bfloat16)
  assert lm.latent_moe._use_dense_phases(None, pw, cfg, 128, h, torch.bfloat16, False)
  got = lm.latent_moe_forward(h, pw, cfg)
  unfused = lm.latent_moe_forward(h, pw, cfg, dense_phases=False)
  idx_p, idx_u = _routing(ops, pw, cfg, h, True), _routing(ops, pw, cfg, h, False)
  torch.cuda.synchronize()
  lm.check_device_status()
  # selection scores from the two-step router's logits: a token may route
  # differently under the two logit summation orders only at a near-tie
  logits = to_np(ops.router_logits(h, pw.router))
  sfc = 1.0 / (1.0 + np.exp(-logits)) + to_np(pw.bias)[None, :]
  both = routing_agreement(idx_p.cpu().numpy(), sfc, idx_u.cpu().numpy())
  g, u = to_np(got)[both], to_np(unfused)[both]
  err = float(np.abs(g - u).max() / np.abs(u).max())
  assert err <= 1e-2, f"normwise {err:.2e}"
  assert np.all(np.abs(g - u) <= 2e-2 + 1e-2 * np.abs(u))


def test_bf16_expert_layer_with_phases_matches_oracle(lm):
  """bf16 routed experts (not MXFP4) with the dense phase kernels: the layer
  against the oracle forward on the same weights, routing compared up to
  near-ties."""
  cfg = lm.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  w = lm.init_weights(cfg, seed=35, bias_std=0.5)
  pw = lm.prepare_weights(w)
  gen = torch.Generator(device="cuda").manual_seed(35)
  h = torch.randn(96, cfg.hidden_size, generator=gen, device="cuda").to(torch.bfloat16)
  assert lm.latent_moe._use_dense_phases(None, pw, cfg, 96, h, torch.bfloat16, False)
  got = lm.latent_moe_forward(h, pw, cfg)
  idx = _routing(_ops(), pw, cfg, h, True)
  torch.cuda.synchronize()
  lm.check_device_status()
  npw = {k: (to_np(v) if isinstance(v, torch.Tensor) else v) for k, v in vars(w).items()}
  ow = O.Weights(**{k: npw[k] for k in O.Weights.__dataclass_fields__})
  ocfg = O.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  ref, rinter = O.latent_moe_forward(to_np(h), ow, ocfg, dtype="bf16", return_intermediates=True)
  same = routing_agreement(idx.cpu().numpy(), rinter["router_scores_for_choice"],
                           rinter["topk_indices"])
  assert_bf16_close(ref[same], to_np(got)[same], "bf16-expert layer with dense phases")
