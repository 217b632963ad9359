"""GPU parity of the MXFP4 grouped matmul (weights packed in HBM, expanded to
bf16 per tile in shared memory, tensor-core MMA) against the dequant-then-matmul
oracle (05_ragged_dot_on_tpu/mxfp4_dequant.py:29-67), and of the MXFP4 layer."""

import numpy as np
import pytest
import torch

from oracle import lmoe_oracle as O
from tests.gpu_util import (assert_bf16_close, assert_gemm_close, routing_agreement, to_dev,
                            to_np)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm():
  import tokamax_tpu_kernel_lab_b200 as lm
  lm.load_native()
  return lm


def _mx(rng, g, n, k, lo=121, hi=129):
  packed = rng.integers(0, 256, (g, n, k // 2), dtype=np.uint8)
  scale = rng.integers(lo, hi + 1, (g, n, k // 32), dtype=np.uint8)
  return packed, scale


def _dev_mx(lm, packed, scale):
  return lm.MXFP4Weights(torch.from_numpy(packed).cuda(), torch.from_numpy(scale).cuda())


def test_in_kernel_dequant_is_bit_exact(lm):
  """lhs = identity rows, f32 output: out[k, n] = dequant(W)[n, k] exactly
  (e2m1 x 2^e is exact in bf16 and one product per output is nonzero).
  Scale bytes span 1..200 (0 decodes to 2^-127, checked separately)."""
  rng = np.random.default_rng(0)
  k, n = 256, 384
  packed, scale = _mx(rng, 1, n, k, lo=1, hi=200)
  scale[0, 0, 0] = 0
  lhs = np.eye(k, dtype=np.float32)
  out = lm.mxfp4_ragged_dot(to_dev(lhs), _dev_mx(lm, packed, scale),
                            torch.tensor([k], dtype=torch.int32, device="cuda"),
                            preferred_element_type=torch.float32)
  ref = O.dequantize_mxfp4(packed[0], scale[0]).T
  assert np.array_equal(to_np(out), ref)


def test_f16_operand_dequant_is_bit_exact(lm):
  """The f16-operand kernel (hardware e2m1 -> f16 expansion, f16 x f16 UMMA)
  reproduces dequant(W) exactly for every scale byte in its range [104, 140]."""
  rng = np.random.default_rng(10)
  k, n = 256, 256
  packed, scale = _mx(rng, 1, n, k, lo=104, hi=140)
  scale[0, 0, :2] = (104, 140)
  lhs = torch.eye(k, dtype=torch.float16, device="cuda")
  w = _dev_mx(lm, packed, scale)
  assert w.f16_operand_ok
  out = lm.mxfp4_ragged_dot(lhs, w, torch.tensor([k], dtype=torch.int32, device="cuda"),
                            preferred_element_type=torch.float32)
  ref = O.dequantize_mxfp4(packed[0], scale[0]).T
  assert np.array_equal(to_np(out), ref)


def test_f16_operand_rejects_out_of_range_scales(lm):
  rng = np.random.default_rng(11)
  packed, scale = _mx(rng, 1, 128, 64, lo=141, hi=150)
  w = _dev_mx(lm, packed, scale)
  assert not w.f16_operand_ok
  with pytest.raises(NotImplementedError):
    lm.mxfp4_ragged_dot(torch.zeros(4, 64, dtype=torch.float16, device="cuda"), w,
                        torch.tensor([4], dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("lhs_dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,k,n,g", [(700, 256, 256, 3), (2048, 1024, 512, 16), (1, 64, 128, 2)])
def test_mxfp4_ragged_dot(lm, m, k, n, g, lhs_dtype):
  rng = np.random.default_rng(m + k + n)
  packed, scale = _mx(rng, g, n, k)
  gs = rng.multinomial(m, np.full(g, 1.0 / g)).astype(np.int32)
  lhs = O.bf16_round(rng.standard_normal((m, k), dtype=np.float32))
  ref = O.mxfp4_ragged_dot(lhs, packed, scale, gs, dtype="fp32")
  out = lm.mxfp4_ragged_dot(to_dev(lhs).to(lhs_dtype), _dev_mx(lm, packed, scale),
                            torch.from_numpy(gs).cuda())
  torch.cuda.synchronize()
  lm.check_device_status()
  scale_ref = float(np.abs(ref).max()) or 1.0
  # compare on a unit scale (outputs here are O(100)): the MXFP4 bar is 1e-2 relative
  assert_gemm_close(ref / scale_ref, to_np(out) / scale_ref, f"mxfp4 {m}x{k}x{n}")


def test_mxfp4_config4_full_size(lm):
  """Benchmark configuration 4: weights (128, K=4096, N=2048) with e2m1 codes
  uniform over all 16 and scale exponents uniform in [-6, 2]; x (16384, 4096)
  bf16 N(0,1); uniform-random group sizes summing to 16384."""
  rng = np.random.default_rng(3)
  g, k, n, m = 128, 4096, 2048, 16384
  packed, scale = _mx(rng, g, n, k, lo=121, hi=129)
  gs = rng.multinomial(m, np.full(g, 1.0 / g)).astype(np.int32)
  lhs = O.bf16_round(rng.standard_normal((m, k), dtype=np.float32))
  ref = O.mxfp4_ragged_dot(lhs, packed, scale, gs, dtype="fp32")
  out = lm.mxfp4_ragged_dot(to_dev(lhs), _dev_mx(lm, packed, scale), torch.from_numpy(gs).cuda())
  s = float(np.abs(ref).max())
  rep = assert_gemm_close(ref / s, to_np(out) / s, "config 4")
  assert rep["normwise_rel"] <= 1e-2


@pytest.mark.parametrize("f16", [False, True])
@pytest.mark.parametrize("round_gate_up", [True, False])
def test_mxfp4_fused_gateup_situ(lm, round_gate_up, f16):
  rng = np.random.default_rng(9)
  m, k, inter, g = 1200, 512, 256, 5
  packed, scale = _mx(rng, g, 2 * inter, k, lo=120, hi=121)  # weights rms ~0.02
  gs = rng.multinomial(m - 17, np.full(g, 1.0 / g)).astype(np.int32)
  lhs = O.bf16_round(rng.standard_normal((m, k), dtype=np.float32))
  lazy = O.LazyMXFP4Experts(packed, scale)
  ref = O.fused_gateup_situ(lhs, lazy, gs, inter, 4.0, 25.0, dtype="bf16",
                            round_gate_up=round_gate_up, out_dtype="fp32")
  dt = torch.float16 if f16 else torch.bfloat16
  out = lm.mxfp4_fused_gateup_situ(to_dev(lhs).to(dt), _dev_mx(lm, packed, scale),
                                   torch.from_numpy(gs).cuda(), round_gate_up=round_gate_up,
                                   out_dtype=dt)
  assert out.dtype == dt
  got = to_np(out)
  # the f16 output carries the bf16-rounded activation exactly
  assert np.array_equal(O.bf16_round(got), got)
  assert np.all(got[gs.sum():] == 0)
  assert_bf16_close(ref, got, f"mxfp4 situ round={round_gate_up}")


def test_mxfp4_layer_matches_oracle(lm):
  """A LatentMoE layer with MXFP4 routed experts (the configuration-5 format,
  scaled down) against the dequant-then-forward oracle."""
  cfg = lm.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  pw = lm.init_prepared_mxfp4(cfg, seed=5, bias_std=0.5)
  gen = torch.Generator(device="cuda").manual_seed(5)
  h = torch.randn(384, 1024, generator=gen, device="cuda").to(torch.bfloat16)
  final, inter = lm.latent_moe_forward(h, pw, cfg, return_intermediates=True)
  torch.cuda.synchronize()
  lm.check_device_status()
  I = cfg.intermediate_size
  si = I * cfg.num_shared_experts
  npf = lambda t: t.float().cpu().numpy()
  gu_p, gu_s = pw.expert_gu_mx.packed.cpu().numpy(), pw.expert_gu_mx.scale.cpu().numpy()
  dn_p, dn_s = pw.expert_down_mx.packed.cpu().numpy(), pw.expert_down_mx.scale.cpu().numpy()
  w = O.Weights(
      router_weight=npf(pw.router).T, e_score_correction_bias=npf(pw.bias),
      down_proj=npf(pw.down).T, up_proj=npf(pw.up).T,
      expert_gate=O.LazyMXFP4Experts(gu_p, gu_s, 0, I),
      expert_up=O.LazyMXFP4Experts(gu_p, gu_s, I, 2 * I),
      expert_down=O.LazyMXFP4Experts(dn_p, dn_s),
      norm_scale=npf(pw.norm_scale),
      shared_gate=npf(pw.shared_gu)[:si].T, shared_up=npf(pw.shared_gu)[si:].T,
      shared_down=npf(pw.shared_down).T)
  ocfg = O.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  ref, rinter = O.latent_moe_forward(npf(h), w, ocfg, dtype="bf16", return_intermediates=True)
  same = routing_agreement(inter["topk_indices"].cpu().numpy(),
                           rinter["router_scores_for_choice"], rinter["topk_indices"])
  assert_bf16_close(ref[same], to_np(final)[same], "mxfp4 layer")


@pytest.mark.parametrize("f16", [False, True])
def test_mxfp4_gateup_with_row_gather(lm, f16):
  rng = np.random.default_rng(14)
  t, k, inter, g, m = 200, 512, 256, 3, 900
  packed, scale = _mx(rng, g, 2 * inter, k, lo=120, hi=121)
  x = O.bf16_round(rng.standard_normal((t, k), dtype=np.float32))
  idx = rng.integers(-1, t, m).astype(np.int32)
  gs = rng.multinomial(m - 5, np.full(g, 1.0 / g)).astype(np.int32)
  rows = np.where(idx[:, None] >= 0, x[np.maximum(idx, 0)], 0).astype(np.float32)
  dt = torch.float16 if f16 else torch.bfloat16
  w = _dev_mx(lm, packed, scale)
  out = lm.mxfp4_fused_gateup_situ(to_dev(x).to(dt), w, torch.from_numpy(gs).cuda(),
                                   out_dtype=dt, row_index=torch.from_numpy(idx).cuda())
  direct = lm.mxfp4_fused_gateup_situ(to_dev(rows).to(dt), w, torch.from_numpy(gs).cuda(),
                                      out_dtype=dt)
  assert torch.equal(out, direct)
  ref = O.fused_gateup_situ(rows, O.LazyMXFP4Experts(packed, scale), gs, inter, 4.0, 25.0,
                            dtype="bf16", out_dtype="fp32")
  assert_bf16_close(ref, to_np(out), f"mxfp4 gather f16={f16}")


def test_checkpoint_layer_runs_identically(lm, tmp_path):
  """A layer exported in the checkpoint's key layout (safetensors) and loaded
  back gives the same forward bits as the in-memory weights."""
  from safetensors.torch import save_file
  from tokamax_tpu_kernel_lab_b200 import checkpoint as ck
  cfg = lm.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  pw = lm.init_prepared_mxfp4(cfg, seed=8, bias_std=0.5)
  path = tmp_path / "layer7.safetensors"
  save_file(ck.layer_state_dict(pw, 7, cfg), str(path))
  loaded = ck.load_latent_moe_layer(path, 7, cfg, device="cuda")
  gen = torch.Generator(device="cuda").manual_seed(8)
  h = torch.randn(256, 1024, generator=gen, device="cuda").to(torch.bfloat16)
  a = lm.latent_moe_forward(h, pw, cfg)
  b = lm.latent_moe_forward(h, loaded, cfg)
  torch.cuda.synchronize()
  lm.check_device_status()
  assert torch.equal(a, b)


def test_mxfp4_ragged_dot_scatter_matches_gathered_output(lm):
  """Output rows stored at per-row addresses (here a permutation of a local
  buffer) equal the ordinary MXFP4 ragged_dot rows moved by that permutation."""
  rng = np.random.default_rng(21)
  g, n, k, m = 5, 512, 1024, 1500
  packed, scale = _mx(rng, g, n, k)
  gs = rng.multinomial(m - 100, np.full(g, 1.0 / g)).astype(np.int32)  # 100 tail rows unused
  w = _dev_mx(lm, packed, scale)
  lhs = to_dev(O.bf16_round(rng.standard_normal((m, k)).astype(np.float32))).to(torch.float16)
  gsd = torch.from_numpy(gs).cuda()
  ref = lm.mxfp4_ragged_dot(lhs, w, gsd)
  perm = torch.from_numpy(rng.permutation(m)).cuda()
  out = torch.full((m, n), 7.0, dtype=torch.bfloat16, device="cuda")
  row_dest = (out.data_ptr() + perm.to(torch.int64) * n * 2).contiguous()
  from tokamax_tpu_kernel_lab_b200 import ops
  ops.mxfp4_ragged_dot_scatter(lhs, w, gsd, row_dest)
  torch.cuda.synchronize()
  lm.check_device_status()
  used = int(gs.sum())
  assert torch.equal(out[perm[:used]], ref[:used])
  untouched = torch.ones(m, dtype=torch.bool, device="cuda")
  untouched[perm[:used]] = False
  assert bool((out[untouched] == 7.0).all())


def test_mxfp4_kernels_repeat_bit_exactly_at_full_size(lm):
  """Configuration-5 shapes (262144 routed rows over 896 experts, skewed
  group sizes, f16 operands): repeated gate/up + SiTU and down calls give
  identical bits, with every output element written.  Many thousands of
  tiles per call cycle each CTA's packed-code, expanded-weight and token rings
  through many laps, so a slot reused before its reader finished shows up
  here as a few changed rows."""
  from tokamax_tpu_kernel_lab_b200.latent_moe import random_mxfp4
  rng = np.random.default_rng(31)
  g, latent, inter, m = 896, 2048, 1024, 262144
  gs = rng.multinomial(m, rng.dirichlet(np.full(g, 0.5))).astype(np.int32)
  gsd = torch.from_numpy(gs).cuda()
  gu = random_mxfp4(g, 2 * inter, latent, seed=31)
  dn = random_mxfp4(g, latent, inter, seed=32)
  assert gu.f16_operand_ok and dn.f16_operand_ok
  gen = torch.Generator(device="cuda").manual_seed(31)
  rows = torch.randn(m, latent, generator=gen, device="cuda").to(torch.bfloat16).to(torch.float16)
  kw = dict(round_gate_up=True, out_dtype=torch.float16)
  act0 = lm.mxfp4_fused_gateup_situ(rows, gu, gsd, **kw)
  down0 = lm.mxfp4_ragged_dot(act0, dn, gsd)
  for _ in range(4):
    act = torch.full_like(act0, float("nan"))
    lm.mxfp4_fused_gateup_situ(rows, gu, gsd, out=act, **kw)
    down = torch.full_like(down0, float("nan"))
    lm.mxfp4_ragged_dot(act0, dn, gsd, out=down)
    torch.cuda.synchronize()
    lm.check_device_status()
    assert torch.equal(act.view(torch.int16), act0.view(torch.int16))
    assert torch.equal(down.view(torch.int16), down0.view(torch.int16))
  assert not bool(torch.isnan(act0).any()) and not bool(torch.isnan(down0).any())
