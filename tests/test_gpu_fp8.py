"""Quantised-weight grouped matmul (e4m3 weights + per-block f32 scales), the
rhs_scale form of the reference's ragged_dot op
(05_ragged_dot_on_tpu/kimi_k3_latent_moe_ragged_dot.py:2714-2953): the kernel
expands the e4m3 tile to the dequantised bf16 weight bit for bit, and the
matmul matches ragged_dot on that weight."""

import numpy as np
import pytest
import torch

from oracle import lmoe_oracle as O
from tests.gpu_util import assert_gemm_close, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm():
  import tokamax_tpu_kernel_lab_b200 as lm
  lm.load_native()
  return lm


def _quantised(rng, g, k, n, block):
  w = (rng.standard_normal((g, k, n)) * 0.02).astype(np.float32)
  q, scale = O.quantize_fp8_blockwise(O.bf16_round(w), block)
  return q, scale


def _dev_fp8(q, scale):
  qd = torch.from_numpy(q).cuda().to(torch.float8_e4m3fn)
  sd = torch.from_numpy(scale[:, :, None, :].copy()).cuda()  # (G, nb, 1, N) as the reference
  return qd, sd


@pytest.mark.parametrize("block", [32, 256])
def test_fp8_expansion_is_bit_exact(lm, block):
  """lhs = identity rows -> every output row is one dequantised weight row."""
  rng = np.random.default_rng(block)
  g, k, n = 2, 256, 512
  q, scale = _quantised(rng, g, k, n, block)
  lhs = np.concatenate([np.eye(k, dtype=np.float32)] * g)
  gs = np.full(g, k, np.int32)
  qd, sd = _dev_fp8(q, scale)
  out = lm.fp8_ragged_dot(to_dev(lhs), qd, torch.from_numpy(gs).cuda(), sd,
                          preferred_element_type=torch.float32)
  torch.cuda.synchronize()
  lm.check_device_status()
  ref = O.dequantize_fp8_blockwise(q, scale).reshape(g * k, n)
  assert np.array_equal(to_np(out), ref)


@pytest.mark.parametrize("m,k,n,g,block", [(512, 256, 512, 4, 32), (1000, 2048, 1024, 8, 32),
                                           (640, 512, 256, 3, 512)])
def test_fp8_ragged_dot_matches_dequantised(lm, m, k, n, g, block):
  rng = np.random.default_rng(m + k + n)
  q, scale = _quantised(rng, g, k, n, block)
  gs = rng.multinomial(m, np.full(g, 1.0 / g)).astype(np.int32)
  gs[1] = 0  # an empty group
  gs[0] += m - gs.sum()
  lhs = O.bf16_round(rng.standard_normal((m, k)).astype(np.float32) * 0.02)
  qd, sd = _dev_fp8(q, scale)
  out = lm.fp8_ragged_dot(to_dev(lhs), qd, torch.from_numpy(gs).cuda(), sd)
  torch.cuda.synchronize()
  lm.check_device_status()
  ref = O.fp8_ragged_dot(lhs, q, scale, gs, dtype="fp32")
  got = to_np(out)
  # the reference's own bar for this check (KRD:2833-2835): max |diff| < 0.05
  assert float(np.abs(got - ref).max()) < 0.05
  assert_gemm_close(ref, got, f"fp8 {m}x{k}x{n} block {block}")


def test_fp8_op_instance_call_matches_function(lm):
  """RaggedDotOp()(lhs, rhs, group_sizes=..., rhs_scale=...) is the same call."""
  rng = np.random.default_rng(7)
  g, k, n, m = 2, 256, 256, 200
  q, scale = _quantised(rng, g, k, n, k)  # whole-row scale, the simplest form
  gs = np.array([150, 50], np.int32)
  lhs = to_dev(O.bf16_round(rng.standard_normal((m, k)).astype(np.float32) * 0.02))
  qd, sd = _dev_fp8(q, scale)
  gsd = torch.from_numpy(gs).cuda()
  a = lm.RaggedDotOp()(lhs, qd, group_sizes=gsd, rhs_scale=sd, maybe_quantize_lhs=False)
  b = lm.fp8_ragged_dot(lhs, qd, gsd, sd)
  torch.cuda.synchronize()
  assert torch.equal(a, b)
  with pytest.raises(NotImplementedError):
    lm.RaggedDotOp()(lhs, qd, group_sizes=gsd, rhs_scale=sd, maybe_quantize_lhs=True)
