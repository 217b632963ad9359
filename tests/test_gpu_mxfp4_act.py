"""The MXFP4-activation form of the block-scaled path (e2m1 activations x
MXFP4 weights on tcgen05.mma kind::mxf4.block_scale) against the oracle's
restatement of its arithmetic: activations quantised per 32 K values to e2m1
with an E8M0 scale (oracle.quantize_mxfp4_act: the smallest 2^e with
amax <= 6 * 2^e, round to nearest even), times the dequantised MXFP4 weights
(05_ragged_dot_on_tpu/mxfp4_dequant.py:29-67).

- The quantise kernels are exact: the e2m1 codes (two per byte, the even K
  index in the low nibble) and the scale bytes equal the oracle's, each row at
  its padded position; codes are compared with the sign of a zero folded
  (+0 and -0 multiply to the same products).
- The GEMM's products are exact in f32, so its f32 output matches the oracle
  to f32 summation-order rounding (normwise 1e-5), bf16/SiTU outputs to the
  bf16 tolerance.
- Its error against the EXACT computation (bf16 activations) is the e2m1
  rounding, ~10% normwise: measured and bounded here, and the reason this
  form is opt-in."""

import numpy as np
import pytest
import torch

from oracle import lmoe_oracle as O
from tests.gpu_util import assert_bf16_close, to_dev, to_np
from tests.test_gpu_mxfp8 import _layer_oracle_weights, _mx, padded_rows_of, sf_bytes_at

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm():
  import tokamax_tpu_kernel_lab_b200 as lm
  lm.load_native()
  return lm


def _ops():
  from tokamax_tpu_kernel_lab_b200 import ops
  return ops


def fold_zero_sign(packed: np.ndarray) -> np.ndarray:
  """Bytes of e2m1 pairs with each nibble 8 (-0) replaced by 0 (+0)."""
  lo, hi = packed & 0x0F, packed >> 4
  lo = np.where(lo == 8, 0, lo)
  hi = np.where(hi == 8, 0, hi)
  return (lo | (hi << 4)).astype(np.uint8)


@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float16])
def test_quantize_rows_exact_with_gather_and_padding(lm, x_dtype):
  ops = _ops()
  rng = np.random.default_rng(50)
  t, k = 300, 512
  x = rng.standard_normal((t, k)).astype(np.float32)
  x *= (10.0 ** rng.uniform(-3, 3, size=(t, 1))).astype(np.float32)  # rows of every scale
  x[7] = 0.0
  x[9, :] = 1e-3
  x[9, 100] = 300.0      # one block dominated by a single value
  x[11, :32] = 6.0       # exactly at e2m1's top: scale 2^0
  x[12, :32] = np.tile(np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25], np.float32), 4)
  x[12, 32:64] = 7.0     # f > 1.5: the next power of two, no saturation
  xd = to_dev(x).to(x_dtype)
  xr = xd.float().cpu().numpy()
  gs = np.array([5, 0, 130, 1, 40, 90], np.int32)
  m = int(gs.sum())
  idx = rng.integers(-1, t, m).astype(np.int32)
  idx[:14] = np.arange(14)
  a = ops.quantize_mxfp4_rows(xd, torch.from_numpy(gs).cuda(), torch.from_numpy(idx).cuda())
  torch.cuda.synchronize()
  lm.check_device_status()
  assert isinstance(a, ops.MXFP4Rows)
  assert a.q.shape == (ops.mxfp8_padded_rows(m, len(gs)), k // 2)
  rows = np.where(idx[:, None] >= 0, xr[np.maximum(idx, 0)], 0).astype(np.float32)
  qv, sf = O.quantize_mxfp4_act(rows)
  prow = padded_rows_of(gs)
  got = a.q.cpu().numpy()[prow]
  assert np.array_equal(fold_zero_sign(got), fold_zero_sign(O.pack_e2m1(qv)))
  assert np.array_equal(sf_bytes_at(a.sf.cpu().numpy(), prow, k, a.q.shape[0]), sf)
  # the tie row: 0.25 -> 0, 0.75 -> 1, 1.25 -> 1, 1.75 -> 2, 2.5 -> 2, 3.5 -> 4, 5 -> 4
  assert np.array_equal(qv[12, :8], np.array([0, 1, 1, 2, 2, 4, 4, -0.0], np.float32))


@pytest.mark.parametrize("t,k,e,dim,f16", [(300, 8, 64, 256, False), (1000, 16, 896, 2048, True),
                                           (7, 3, 4, 128, False)])
def test_quantize_scatter_equals_row_order(lm, t, k, e, dim, f16):
  """The token-order quantising gather writes the same codes and scale bytes
  as the row-order kernel on every row of the groups."""
  ops = _ops()
  g = torch.Generator(device="cuda").manual_seed(t + k + 1)
  x = torch.randn(t, dim, generator=g, device="cuda").to(torch.float16 if f16 else torch.bfloat16)
  idx = torch.stack([torch.randperm(e, generator=g, device="cuda")[:k] for _ in range(t)]).int()
  d = ops.dispatch(idx, torch.ones(t, k, device="cuda"), e, want_order=False)
  a = ops.quantize_mxfp4_rows(x, d.group_sizes, d.token_idx)
  b = ops.quantize_mxfp4_scatter(x, d.group_sizes, d.slot_pos, k)
  torch.cuda.synchronize()
  lm.check_device_status()
  gs = d.group_sizes.cpu().numpy()
  prow = padded_rows_of(gs)
  m_pad = a.q.shape[0]
  assert b.q.shape == a.q.shape == (m_pad, dim // 2)
  assert np.array_equal(b.q.cpu().numpy()[prow], a.q.cpu().numpy()[prow])
  assert np.array_equal(sf_bytes_at(b.sf.cpu().numpy(), prow, dim, m_pad),
                        sf_bytes_at(a.sf.cpu().numpy(), prow, dim, m_pad))


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("g,n,k,gs", [(3, 256, 512, [100, 0, 300]),
                                      (5, 128, 1024, [1, 129, 0, 17, 256]),
                                      (2, 384, 256, [64, 200]),
                                      (2, 128, 4096, [192, 191])])
def test_mxf4_gemm_matches_oracle(lm, g, n, k, gs, out_dtype):
  ops = _ops()
  rng = np.random.default_rng(g * n + k + 1)
  packed, scale = _mx(rng, g, n, k)
  gs = np.array(gs, np.int32)
  m = int(gs.sum())
  x = O.bf16_round(rng.standard_normal((m, k), dtype=np.float32))
  a = ops.quantize_mxfp4_rows(to_dev(x), torch.from_numpy(gs).cuda())
  w = ops.prepare_mxfp4_blockscaled(lm.MXFP4Weights(torch.from_numpy(packed).cuda(),
                                                     torch.from_numpy(scale).cuda()))
  out = ops.mxfp4_mxfp4_ragged_dot(a, w, out_dtype=out_dtype)
  torch.cuda.synchronize()
  lm.check_device_status()
  qv, sf = O.quantize_mxfp4_act(x)
  ref = O.mxfp4_mxfp4_ragged_dot(qv, sf, packed, scale, gs)
  got = to_np(out)[padded_rows_of(gs)]
  s = float(np.abs(ref).max())
  if out_dtype == torch.float32:
    err = float(np.abs(got - ref).max()) / s
    assert err <= 1e-5, f"normwise {err}"
  else:
    assert_bf16_close(ref / s, got / s, f"mxf4 {g}x{n}x{k}")


def test_mxf4_gateup_situ_matches_oracle(lm):
  ops = _ops()
  rng = np.random.default_rng(54)
  g, inter, k = 4, 256, 512
  gs = np.array([200, 0, 37, 300], np.int32)
  m = int(gs.sum())
  packed, scale = _mx(rng, g, 2 * inter, k, lo=120, hi=121)  # weights rms ~0.02
  x = O.bf16_round(rng.standard_normal((m, k), dtype=np.float32))
  a = ops.quantize_mxfp4_rows(to_dev(x), torch.from_numpy(gs).cuda())
  w = ops.prepare_mxfp4_blockscaled(lm.MXFP4Weights(torch.from_numpy(packed).cuda(),
                                                     torch.from_numpy(scale).cuda()), gateup=True)
  out = ops.mxfp4_mxfp4_gateup_situ(a, w)
  torch.cuda.synchronize()
  lm.check_device_status()
  qv, sf = O.quantize_mxfp4_act(x)
  ref = O.fused_gateup_situ(O.dequantize_mxfp8(qv, sf), O.LazyMXFP4Experts(packed, scale), gs,
                            inter, 4.0, 25.0, dtype="bf16", round_gate_up=True, out_dtype="fp32")
  got = to_np(out)[padded_rows_of(gs)]
  assert_bf16_close(ref[:m], got, "mxf4 gate/up + SiTU")


def test_mxf4_error_against_the_exact_product(lm):
  """What this form costs: the e2m1 activation rounding against the exact
  product (bf16 activations x dequantised MXFP4), configuration-4 style data
  (N(0,1) rows, K = 4096).  e2m1 keeps one mantissa bit: ~10% normwise."""
  ops = _ops()
  rng = np.random.default_rng(55)
  g, n, k = 2, 256, 4096
  gs = np.array([300, 212], np.int32)
  packed, scale = _mx(rng, g, n, k, lo=121, hi=129)
  x = O.bf16_round(rng.standard_normal((int(gs.sum()), k), dtype=np.float32))
  a = ops.quantize_mxfp4_rows(to_dev(x), torch.from_numpy(gs).cuda())
  w = ops.prepare_mxfp4_blockscaled(lm.MXFP4Weights(torch.from_numpy(packed).cuda(),
                                                     torch.from_numpy(scale).cuda()))
  out = ops.mxfp4_mxfp4_ragged_dot(a, w, out_dtype=torch.float32)
  exact = O.mxfp4_ragged_dot(x, packed, scale, gs, dtype="fp32")
  got = to_np(out)[padded_rows_of(gs)]
  normwise = float(np.abs(got - exact).max() / np.abs(exact).max())
  rms = float(np.sqrt(np.mean((got - exact) ** 2)) / np.sqrt(np.mean(exact ** 2)))
  print(f"mxf4 vs exact: normwise {normwise:.4f}, rms {rms:.4f}")
  assert 1e-2 < normwise < 0.3 and rms < 0.2


def test_layer_mxfp4_mode_stages_and_error(lm):
  """latent_moe_forward(..., mxfp4_operand="mxfp4"): gate/up + SiTU and the
  down GEMM against the oracle given the GPU's own stage inputs, the whole
  forward against the oracle forward with the same activation rounding and
  against the exact forward, and a CUDA graph of it replaying to the same bits."""
  from tests.gpu_util import routing_agreement
  cfg = lm.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  pw = lm.init_prepared_mxfp4(cfg, seed=56, bias_std=0.5)
  gen = torch.Generator(device="cuda").manual_seed(56)
  h = torch.randn(384, 1024, generator=gen, device="cuda").to(torch.bfloat16)
  final, inter = lm.latent_moe_forward(h, pw, cfg, mxfp4_operand="mxfp4",
                                       return_intermediates=True)
  exact = lm.latent_moe_forward(h, pw, cfg)
  torch.cuda.synchronize()
  lm.check_device_status()
  I = cfg.intermediate_size
  gs = inter["group_sizes"].cpu().numpy()
  prow = padded_rows_of(gs)
  gu_p, gu_s = pw.expert_gu_mx.packed.cpu().numpy(), pw.expert_gu_mx.scale.cpu().numpy()
  dn_p, dn_s = pw.expert_down_mx.packed.cpu().numpy(), pw.expert_down_mx.scale.cpu().numpy()
  x = to_np(inter["latent_projection"])[inter["token_idx"].cpu().numpy()]
  qv, sf = O.quantize_mxfp4_act(x)
  act_ref = O.fused_gateup_situ(O.dequantize_mxfp8(qv, sf), O.LazyMXFP4Experts(gu_p, gu_s), gs,
                                I, 4.0, 25.0, dtype="bf16", round_gate_up=True, out_dtype="fp32")
  act = to_np(inter["situ_output"])[prow]
  assert_bf16_close(act_ref, act, "mxfp4 layer: gate/up + SiTU")
  aq, asf = O.quantize_mxfp4_act(act)
  down_ref = O.mxfp4_mxfp4_ragged_dot(aq, asf, dn_p, dn_s, gs)
  down = to_np(inter["expert_down_output"])[prow]
  s = float(np.abs(down_ref).max())
  assert_bf16_close(down_ref / s, down / s, "mxfp4 layer: down GEMM")
  w = _layer_oracle_weights(lm, pw, cfg)
  ocfg = O.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  ref, rinter = O.latent_moe_forward(to_np(h), w, ocfg, dtype="bf16", return_intermediates=True,
                                     quantize_activations="mxfp4")
  same = routing_agreement(inter["topk_indices"].cpu().numpy(),
                           rinter["router_scores_for_choice"], rinter["topk_indices"])
  got = to_np(final)
  vs_oracle = float(np.abs(got[same] - ref[same]).max() / np.abs(ref[same]).max())
  e = to_np(exact)
  vs_exact = float(np.abs(got - e).max() / np.abs(e).max())
  print(f"mxfp4 layer: normwise vs its oracle {vs_oracle:.4f}, vs the exact forward {vs_exact:.4f}")
  assert vs_oracle < 1e-1 and vs_exact < 0.3
  static_h = h.clone()
  st = torch.cuda.Stream()
  st.wait_stream(torch.cuda.current_stream())
  with torch.cuda.stream(st):
    lm.latent_moe_forward(static_h, pw, cfg, mxfp4_operand="mxfp4", dense_phases=False)
  torch.cuda.current_stream().wait_stream(st)
  graph = torch.cuda.CUDAGraph()
  with torch.cuda.graph(graph):
    # the forward with intermediates runs the dense projections unfused
    out = lm.latent_moe_forward(static_h, pw, cfg, mxfp4_operand="mxfp4", dense_phases=False)
  graph.replay()
  torch.cuda.synchronize()
  assert torch.equal(out, final)
