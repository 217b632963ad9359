"""GPU parity of the fused router gate (lmoe_router_fused_bf16): the logits
GEMM with the top-k selection in its epilogue must return the same bits as
the two-step path (f32 logits GEMM, then lmoe_router_topk) on the same
inputs -- indices and weights -- and agree with the oracle's gate
(kimi_k3_latent_moe_reference.py:347-356) up to near-ties."""

import numpy as np
import pytest
import torch

from oracle import lmoe_oracle as O
from tests.gpu_util import routing_agreement, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm():
  import tokamax_tpu_kernel_lab_b200 as lm
  lm.load_native()
  return lm


def _inputs(seed, t, d, e, bias_std=0.5, bias=True):
  g = torch.Generator(device="cuda").manual_seed(seed)
  h = torch.randn(t, d, generator=g, device="cuda").to(torch.bfloat16)
  w = (torch.randn(e, d, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
  b = torch.randn(e, generator=g, device="cuda") * bias_std if bias else None
  return h, w, b


def _two_step(lm, h, w, b, k, **kw):
  """f32 logits from the dense GEMM (its output width must be a multiple of
  8: zero router rows pad it and are sliced off), then router_topk."""
  e = w.shape[0]
  pad = -e % 8
  wp = torch.cat([w, w.new_zeros(pad, w.shape[1])]) if pad else w
  logits = lm.ops.router_logits(h, wp)[:, :e].contiguous()
  return lm.ops.router_topk(logits, b, k, **kw)


def _assert_same_bits(got, ref):
  gi, gw = got
  ri, rw = ref
  assert torch.equal(gi, ri), f"indices differ in {int((gi != ri).any(1).sum())} tokens"
  assert torch.equal(gw.view(torch.int32), rw.view(torch.int32)), "weights differ"


# (tokens, hidden, experts, top_k): one chunk (E <= 256), the 4 x 224 split of
# 896 experts, the widest 4 x 256 split, two chunks with a ragged second one
# (257 -> 144 + 113), a chunk narrower than the 16-entry candidate list
# (E = 10, k = 10), a partial token block and a single token
SHAPES = [(1000, 512, 64, 8), (777, 1024, 896, 16), (129, 2048, 1024, 16), (300, 512, 257, 4),
          (300, 256, 10, 10), (1, 512, 384, 6), (4100, 7168, 896, 16)]


@pytest.mark.parametrize("t,d,e,k", SHAPES)
def test_fused_router_equals_two_step_bits(lm, t, d, e, k):
  h, w, b = _inputs(t + e, t, d, e)
  _assert_same_bits(lm.ops.router_gate_fused(h, w, b, k), _two_step(lm, h, w, b, k))
  lm.ops.check_device_status()


@pytest.mark.parametrize("renormalize,rsf,bias", [(False, 1.0, True), (True, 2.5, False),
                                                  (False, 0.75, False)])
def test_fused_router_options(lm, renormalize, rsf, bias):
  h, w, b = _inputs(11, 513, 768, 896, bias=bias)
  kw = dict(renormalize=renormalize, routed_scaling_factor=rsf)
  _assert_same_bits(lm.ops.router_gate_fused(h, w, b, 16, **kw), _two_step(lm, h, w, b, 16, **kw))


def test_fused_router_ties_go_to_the_lower_expert(lm):
  """Zero hidden rows give every expert the same key (sigmoid(0) + 0): the
  selection is experts 0..k-1 in id order.  Duplicated router rows with equal
  bias tie across chunks (expert 5 and 700, 3 and 451): the lower id first."""
  t, d, e, k = 256, 512, 896, 16
  h, w, _ = _inputs(3, t, d, e)
  h[:64] = 0
  w[700] = w[5]
  w[451] = w[3]
  b = torch.zeros(e, device="cuda")
  got = lm.ops.router_gate_fused(h, w, b, k)
  _assert_same_bits(got, _two_step(lm, h, w, b, k))
  idx = got[0].cpu().numpy()
  assert np.array_equal(idx[:64], np.tile(np.arange(k, dtype=np.int32), (64, 1)))
  pos = {int(x): i for i, x in enumerate(idx[100])}
  for lo, hi in ((5, 700), (3, 451)):
    if lo in pos and hi in pos:
      assert pos[lo] < pos[hi]


def test_fused_router_matches_oracle(lm):
  t, d, e, k = 600, 1024, 896, 16
  h, w, b = _inputs(5, t, d, e)
  idx, wts = lm.ops.router_gate_fused(h, w, b, k)
  logits, _, sfc, ref_idx, ref_w = O.router_gate(to_np(h), to_np(w).T, to_np(b), k)
  same = routing_agreement(idx.cpu().numpy(), sfc, ref_idx)
  got_w = wts.cpu().numpy()
  assert np.allclose(got_w[same], ref_w[same], rtol=2e-5, atol=1e-6)


def test_fused_router_full_configuration(lm):
  """Configuration 5's gate: 16384 tokens x d 7168 over 896 experts, top-16,
  bias N(0, 0.5^2); the same bits as the two-step path."""
  h, w, b = _inputs(7, 16384, 7168, 896)
  _assert_same_bits(lm.ops.router_gate_fused(h, w, b, 16), _two_step(lm, h, w, b, 16))
  lm.ops.check_device_status()


def test_fused_router_errors(lm):
  h, w, b = _inputs(1, 64, 256, 64)
  ws = torch.empty(16, dtype=torch.uint8, device="cuda")
  idx = torch.empty(64, 8, dtype=torch.int32, device="cuda")
  wt = torch.empty(64, 8, dtype=torch.float32, device="cuda")
  nat = lm._native
  rc = nat.load().lmoe_router_fused_bf16(h.data_ptr(), w.data_ptr(), b.data_ptr(), 64, 256, 64, 8,
                                         1, 1.0, idx.data_ptr(), wt.data_ptr(), ws.data_ptr(),
                                         ws.numel(), None, None)
  assert rc == nat.LMOE_SCRATCH_TOO_SMALL
  with pytest.raises(ValueError):
    lm.ops.router_gate_fused(h, w, b, 17)  # top_k above 16
  assert not lm.ops.router_fused_supported(h, w, 8, "softmax")
  assert not lm.ops.router_fused_supported(h.float(), w, 8)


def test_forward_fused_route_same_output(lm):
  """latent_moe_forward routes through the fused gate unless the
  intermediates are requested (they include the logits); both give the same
  output bits."""
  from tokamax_tpu_kernel_lab_b200.latent_moe import (LatentMoEConfig, init_weights,
                                                      latent_moe_forward, prepare_weights)
  cfg = LatentMoEConfig(1024, 512, 256, 128, 8, 1)
  pw = prepare_weights(init_weights(cfg, seed=3, bias_std=0.5))
  x = (torch.randn(300, 1024, device="cuda")).to(torch.bfloat16)
  # (dense_phases=False: the forward with intermediates runs the dense
  # projections unfused, and this compares the router forms alone)
  fused = latent_moe_forward(x, pw, cfg, dense_phases=False)
  plain, inter = latent_moe_forward(x, pw, cfg, return_intermediates=True)
  assert torch.equal(fused, plain)
  lm.ops.check_device_status()
