"""The exact MXFP4 matmul on the block-scaled tensor core: bf16/f16 rows split
into two e4m3 planes under one E8M0 scale per 32 K values (hi = e4m3(x/2^e),
lo = e4m3(x/2^e - hi); oracle.split_e4m3), both multiplied by the MXFP4
weights (05_ragged_dot_on_tpu/mxfp4_dequant.py:29-67) into one f32
accumulator (tcgen05.mma kind::mxf8f6f4.block_scale, twice per K step).

- The split kernels are bit-exact: both planes' e4m3 bytes and the scale bytes
  equal the oracle's, each row at its padded position.
- hi + lo is the bf16 value itself for |x| >= 2^(e-2) (every element of these
  N(0,1) rows but the smallest ~0.2%, and those within 2^(e-10)), so the GEMM
  matches the EXACT dequant-then-matmul product to f32 summation rounding
  (normwise 1e-5), not just its own oracle.
- mxfp4_ragged_dot_blockscaled writes the ragged_dot layout (unpadded rows,
  zero tail) and agrees with the exact weights-major kernel."""

import ml_dtypes
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


def e4m3_values(q: np.ndarray) -> np.ndarray:
  return q.view(ml_dtypes.float8_e4m3fn).astype(np.float32)


@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float16])
def test_split_rows_bit_exact(lm, x_dtype):
  ops = _ops()
  rng = np.random.default_rng(60)
  t, k = 300, 512
  x = rng.standard_normal((t, k)).astype(np.float32)
  x *= (10.0 ** rng.uniform(-3, 3, size=(t, 1))).astype(np.float32)
  x[7] = 0.0
  x[9, :] = 1e-3
  x[9, 100] = 300.0      # tiny elements beside one large one: lo goes subnormal
  x[11, :32] = 448.0
  xd = to_dev(x).to(x_dtype)
  xr = xd.float().cpu().numpy()
  gs = np.array([5, 0, 130, 1, 40, 90], np.int32)
  m = int(gs.sum())
  idx = rng.integers(-1, t, m).astype(np.int32)
  idx[:12] = np.arange(12)
  a = ops.quantize_split_rows(xd, torch.from_numpy(gs).cuda(), torch.from_numpy(idx).cuda())
  torch.cuda.synchronize()
  lm.check_device_status()
  m_pad = ops.mxfp8_padded_rows(m, len(gs))
  assert isinstance(a, ops.SplitRows) and a.q.shape == (2, m_pad, k)
  rows = np.where(idx[:, None] >= 0, xr[np.maximum(idx, 0)], 0).astype(np.float32)
  hi, lo, sf = O.split_e4m3(rows)
  prow = padded_rows_of(gs)
  q = a.q.cpu().numpy()
  assert np.array_equal(e4m3_values(q[0][prow]), hi)
  assert np.array_equal(e4m3_values(q[1][prow]), lo)
  assert np.array_equal(sf_bytes_at(a.sf.cpu().numpy(), prow, k, m_pad), sf)
  # hi + lo is the row itself wherever |x| >= 2^(e-2)
  d = O.dequantize_split(hi, lo, sf)
  e = np.repeat(sf.astype(np.int32) - 127, 32, axis=1)
  big = np.abs(rows) >= np.ldexp(1.0, e - 2)
  assert np.array_equal(d[big], rows[big])
  assert np.all(np.abs(d - rows)[~big] <= np.ldexp(1.0, e - 10)[~big])


@pytest.mark.parametrize("t,k,e,dim", [(300, 8, 64, 256), (1000, 16, 896, 2048)])
def test_split_scatter_equals_row_order(lm, t, k, e, dim):
  ops = _ops()
  g = torch.Generator(device="cuda").manual_seed(t + k + 2)
  x = torch.randn(t, dim, generator=g, device="cuda").to(torch.bfloat16)
  idx = torch.stack([torch.randperm(e, generator=g, device="cuda")[:k] for _ in range(t)]).int()
  d = ops.dispatch(idx, torch.ones(t, k, device="cuda"), e, want_order=False)
  a = ops.quantize_split_rows(x, d.group_sizes, d.token_idx)
  b = ops.quantize_split_scatter(x, d.group_sizes, d.slot_pos, k)
  torch.cuda.synchronize()
  lm.check_device_status()
  prow = padded_rows_of(d.group_sizes.cpu().numpy())
  m_pad = a.q.shape[1]
  assert b.q.shape == a.q.shape
  for p in range(2):
    assert np.array_equal(b.q[p].cpu().numpy()[prow], a.q[p].cpu().numpy()[prow])
  assert np.array_equal(sf_bytes_at(b.sf.cpu().numpy(), prow, dim, m_pad),
                        sf_bytes_at(a.sf.cpu().numpy(), prow, dim, m_pad))


@pytest.mark.parametrize("g,n,k,gs", [(3, 256, 512, [100, 0, 300]),
                                      (5, 128, 1024, [1, 129, 0, 17, 256]),
                                      (2, 384, 256, [64, 200]),
                                      (2, 128, 4096, [192, 191])])
def test_split_gemm_is_the_exact_product(lm, g, n, k, gs):
  """Padded output, f32: within f32 summation rounding of the exact
  dequant-then-matmul product (the reference's mxfp4 ragged_dot)."""
  ops = _ops()
  rng = np.random.default_rng(g * n + k + 2)
  packed, scale = _mx(rng, g, n, k)
  gs = np.array(gs, np.int32)
  m = int(gs.sum())
  x = O.bf16_round(rng.standard_normal((m, k), dtype=np.float32))
  a = ops.quantize_split_rows(to_dev(x), torch.from_numpy(gs).cuda())
  w = ops.prepare_mxfp4_blockscaled(lm.MXFP4Weights(torch.from_numpy(packed).cuda(),
                                                     torch.from_numpy(scale).cuda()))
  out = ops.mxfp8_mxfp4_ragged_dot(a, w, out_dtype=torch.float32)
  torch.cuda.synchronize()
  lm.check_device_status()
  exact = O.mxfp4_ragged_dot(x, packed, scale, gs, dtype="fp32")
  got = to_np(out)[padded_rows_of(gs)]
  err = float(np.abs(got - exact).max()) / float(np.abs(exact).max())
  assert err <= 1e-5, f"normwise {err}"


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_ragged_dot_blockscaled_layout_and_exactness(lm, out_dtype):
  """The ragged_dot layout: rows in group order, rows past sum(group_sizes)
  zero; results within f32 rounding of the exact product (f32 out) or
  within the bf16 tolerance (bf16 out), and next to the weights-major exact
  kernel."""
  ops = _ops()
  rng = np.random.default_rng(61)
  g, n, k = 6, 384, 1024
  gs = np.array([40, 0, 300, 129, 1, 200], np.int32)
  m = int(gs.sum()) + 37   # a tail of rows past the groups
  packed, scale = _mx(rng, g, n, k)
  x = O.bf16_round(rng.standard_normal((m, k), dtype=np.float32))
  wm = lm.MXFP4Weights(torch.from_numpy(packed).cuda(), torch.from_numpy(scale).cuda())
  w = ops.prepare_mxfp4_blockscaled(wm)
  gsd = torch.from_numpy(gs).cuda()
  out = torch.full((m, n), 7.0, dtype=out_dtype, device="cuda")  # the tail must be zeroed
  ops.mxfp4_ragged_dot_blockscaled(to_dev(x), w, gsd, out=out)
  torch.cuda.synchronize()
  lm.check_device_status()
  exact = O.mxfp4_ragged_dot(x, packed, scale, gs, dtype="fp32")
  got = to_np(out)
  s = float(np.abs(exact).max())
  assert np.all(got[int(gs.sum()):] == 0)
  if out_dtype == torch.float32:
    assert float(np.abs(got - exact).max()) / s <= 1e-5
  else:
    assert_bf16_close(exact / s, got / s, "split ragged_dot (bf16)")
    ref_kernel = to_np(ops.mxfp4_ragged_dot(to_dev(x), wm, gsd))
    assert float(np.abs(got - ref_kernel).max()) / s <= 1e-2


def test_split_gateup_situ_matches_exact(lm):
  ops = _ops()
  rng = np.random.default_rng(62)
  g, inter, k = 4, 256, 512
  gs = np.array([200, 0, 37, 300], np.int32)
  m = int(gs.sum())
  packed, scale = _mx(rng, g, 2 * inter, k, lo=120, hi=121)
  x = O.bf16_round(rng.standard_normal((m, k), dtype=np.float32))
  a = ops.quantize_split_rows(to_dev(x), torch.from_numpy(gs).cuda())
  w = ops.prepare_mxfp4_blockscaled(lm.MXFP4Weights(torch.from_numpy(packed).cuda(),
                                                     torch.from_numpy(scale).cuda()), gateup=True)
  out = ops.mxfp8_mxfp4_gateup_situ(a, w)
  torch.cuda.synchronize()
  lm.check_device_status()
  ref = O.fused_gateup_situ(x, O.LazyMXFP4Experts(packed, scale), gs, inter, 4.0, 25.0,
                            dtype="bf16", round_gate_up=True, out_dtype="fp32")
  got = to_np(out)[padded_rows_of(gs)]
  assert_bf16_close(ref[:m], got, "split gate/up + SiTU")


def test_layer_split_mode_matches_the_exact_forward(lm):
  """latent_moe_forward(..., mxfp4_operand="split") against the exact
  forward (same routing, bf16 output): within the bf16 tolerance; and a CUDA
  graph of it replays to the same bits."""
  cfg = lm.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  pw = lm.init_prepared_mxfp4(cfg, seed=63, bias_std=0.5)
  gen = torch.Generator(device="cuda").manual_seed(63)
  h = torch.randn(384, 1024, generator=gen, device="cuda").to(torch.bfloat16)
  final, inter = lm.latent_moe_forward(h, pw, cfg, mxfp4_operand="split",
                                       return_intermediates=True)
  exact, einter = lm.latent_moe_forward(h, pw, cfg, mxfp4_operand="bf16",
                                        return_intermediates=True)
  torch.cuda.synchronize()
  lm.check_device_status()
  assert torch.equal(inter["topk_indices"], einter["topk_indices"])
  e, got = to_np(exact), to_np(final)
  vs_exact = float(np.abs(got - e).max() / np.abs(e).max())
  print(f"split layer: normwise vs the exact forward {vs_exact:.2e}")
  assert_bf16_close(e, got, "split layer vs exact")
  # against the oracle forward on the same weights
  w = _layer_oracle_weights(lm, pw, cfg)
  ocfg = O.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  from tests.gpu_util import routing_agreement
  ref, rinter = O.latent_moe_forward(to_np(h), w, ocfg, dtype="bf16", return_intermediates=True)
  same = routing_agreement(inter["topk_indices"].cpu().numpy(),
                           rinter["router_scores_for_choice"], rinter["topk_indices"])
  assert float(np.abs(got[same] - ref[same]).max() / np.abs(ref[same]).max()) < 1e-2
  static_h = h.clone()
  st = torch.cuda.Stream()
  st.wait_stream(torch.cuda.current_stream())
  with torch.cuda.stream(st):
    lm.latent_moe_forward(static_h, pw, cfg, mxfp4_operand="split", dense_phases=False)
  torch.cuda.current_stream().wait_stream(st)
  graph = torch.cuda.CUDAGraph()
  with torch.cuda.graph(graph):
    # the forward with intermediates runs the dense projections unfused
    out = lm.latent_moe_forward(static_h, pw, cfg, mxfp4_operand="split", dense_phases=False)
  graph.replay()
  torch.cuda.synchronize()
  assert torch.equal(out, final)


@pytest.mark.parametrize("kind,fmt", [("e4m3x2", "e4m3x2"), ("e4m3", "e4m3"), ("e2m1", "e2m1"),
                                      ("e4m3x2", "e4m3")])
def test_quantising_gateup_epilogue_equals_quantising_the_activations(lm, kind, fmt):
  """The gate/up kernel that writes its SiTU activations straight into the
  down GEMM's block-scaled rows (the 32-feature block's maximum met across
  two epilogue warps) gives the same bytes as the bf16 activations quantised
  by the row kernel."""
  ops = _ops()
  rng = np.random.default_rng(64)
  g, inter, k = 4, 256, 512
  gs = np.array([200, 0, 37, 300], np.int32)
  packed, scale = _mx(rng, g, 2 * inter, k, lo=120, hi=121)
  x = to_dev(O.bf16_round(rng.standard_normal((int(gs.sum()), k), dtype=np.float32)))
  gsd = torch.from_numpy(gs).cuda()
  quant = {"e4m3": ops.quantize_mxfp8_rows, "e2m1": ops.quantize_mxfp4_rows,
           "e4m3x2": ops.quantize_split_rows}
  a = quant[kind](x, gsd)
  w = ops.prepare_mxfp4_blockscaled(lm.MXFP4Weights(torch.from_numpy(packed).cuda(),
                                                     torch.from_numpy(scale).cuda()), gateup=True)
  act = ops.mxfp8_mxfp4_gateup_situ(a, w)
  want = quant[fmt](act, gsd, padded_input=True)
  got = ops.blockscaled_gateup_situ_quantized(a, w, fmt)
  torch.cuda.synchronize()
  lm.check_device_status()
  prow = padded_rows_of(gs)
  m_pad = a.q.shape[-2]
  assert got.q.shape == want.q.shape
  gq, wq = got.q.cpu().numpy(), want.q.cpu().numpy()
  if fmt == "e4m3x2":
    for p in range(2):
      assert np.array_equal(gq[p][prow], wq[p][prow])
  else:
    assert np.array_equal(gq[prow], wq[prow])
  assert np.array_equal(sf_bytes_at(got.sf.cpu().numpy(), prow, inter, m_pad),
                        sf_bytes_at(want.sf.cpu().numpy(), prow, inter, m_pad))


def test_split_scatter_writes_the_padded_positions(lm):
  """lmoe_bf16split_quantize_scatter_positions: the same split rows as the
  plain token-order gather, and the slot positions of lmoe_mxfp8_pad_positions,
  bit for bit (a dropless dispatch of 700 tokens, top-8 over 96 experts)."""
  from tokamax_tpu_kernel_lab_b200 import ops
  rng = np.random.default_rng(71)
  t, k, e, dim = 700, 8, 96, 512
  ids = np.stack([rng.choice(e, size=k, replace=False) for _ in range(t)]).astype(np.int32)
  w = rng.random((t, k), dtype=np.float32)
  d = ops.dispatch(torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), e)
  x = torch.randn(t, dim, device="cuda").to(torch.bfloat16)
  rows, pos = ops.quantize_split_scatter_with_positions(x, d.group_sizes, d.slot_pos, k)
  ref = ops.quantize_split_scatter(x, d.group_sizes, d.slot_pos, k)
  ref_pos = ops.mxfp8_pad_positions(d.slot_pos, d.group_sizes)
  torch.cuda.synchronize()
  lm.check_device_status()
  assert torch.equal(pos, ref_pos)
  live = to_np(ref_pos) >= 0
  used = np.unique(to_np(ref_pos)[live].astype(np.int64))
  assert torch.equal(rows.q[:, used], ref.q[:, used])
  # the scale bytes of the written rows (atoms (K/128, M_pad/128, 512 B): byte
  # (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4 of atom (kb // 4, r // 128))
  m_pad = rows.q.shape[-2]
  kb = np.arange(dim // 32)
  atom = (kb[None, :] // 4) * (m_pad // 128) + used[:, None] // 128
  byte = (used[:, None] % 32) * 16 + ((used[:, None] % 128) // 32) * 4 + kb[None, :] % 4
  idx = atom * 512 + byte
  a, b = rows.sf.reshape(-1).cpu().numpy(), ref.sf.reshape(-1).cpu().numpy()
  assert np.array_equal(a[idx], b[idx])
