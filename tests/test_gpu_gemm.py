"""GPU parity: tensor-core grouped GEMM (ragged_dot), fused gate/up SiTU-GLU,
dense GEMM with residual add, f32 CUDA-core path -- all through the C ABI,
checked against the CPU oracle."""

import zlib

import numpy as np
import pytest
import torch

from oracle import lmoe_oracle as O
from tests.gpu_util import (DISTRIBUTIONS, assert_bf16_close, assert_gemm_close,
                            distribution_sizes, to_dev, to_np, zipf_group_sizes)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm():
  import tokamax_tpu_kernel_lab_b200 as lm
  lm.load_native()
  return lm


def _rand(rng, *shape, scale=1.0):
  return (rng.standard_normal(shape, dtype=np.float32) * np.float32(scale))


def _ragged_case(lm, rng, m, k, n, gs, layout, extra_rows=0):
  g = len(gs)
  lhs = O.bf16_round(_rand(rng, m + extra_rows, k, scale=1 / np.sqrt(k)))
  rhs = O.bf16_round(_rand(rng, g, k, n, scale=1 / np.sqrt(k)))
  ref = O.ragged_dot(lhs, rhs, gs, dtype="fp32")
  rhs_dev = rhs if layout == "gkn" else np.ascontiguousarray(rhs.transpose(0, 2, 1))
  out = lm.ragged_dot(to_dev(lhs), to_dev(rhs_dev), torch.from_numpy(gs).cuda(),
                      rhs_layout=layout)
  torch.cuda.synchronize()
  lm.check_device_status()
  return ref, to_np(out)


@pytest.mark.parametrize("layout", ["gkn", "gnk"])
@pytest.mark.parametrize("dist", DISTRIBUTIONS)
def test_ragged_dot_distributions(lm, layout, dist):
  """benchmark_harness.py:156-205 distributions, small shape (m 512, k 256, n 384, g 4)."""
  rng = np.random.default_rng(zlib.crc32(f"{layout}/{dist}".encode()))
  gs = distribution_sizes(dist, 512, 4, rng)
  ref, got = _ragged_case(lm, rng, 512, 256, 384, gs, layout)
  assert_gemm_close(ref, got, f"{layout}/{dist}")


@pytest.mark.parametrize("layout", ["gkn", "gnk"])
@pytest.mark.parametrize("m,k,n,g", [(1, 64, 128, 1), (300, 200, 136, 7), (2048, 512, 512, 8),
                                     (1000, 1024, 1024, 16)])
def test_ragged_dot_shapes(lm, layout, m, k, n, g):
  """Ragged boundaries mid-tile, K and N tails, single row."""
  rng = np.random.default_rng(m * 7 + k)
  gs = rng.multinomial(m, np.full(g, 1.0 / g)).astype(np.int32)
  ref, got = _ragged_case(lm, rng, m, k, n, gs, layout)
  assert_gemm_close(ref, got, f"{layout} {m}x{k}x{n} g{g}")


def test_ragged_dot_rows_past_sum_are_zero(lm):
  rng = np.random.default_rng(3)
  gs = np.array([100, 0, 37], np.int32)
  ref, got = _ragged_case(lm, rng, 137, 128, 256, gs, "gkn", extra_rows=91)
  assert np.all(got[137:] == 0)
  assert_gemm_close(ref, got)


def test_ragged_dot_f32_output(lm):
  rng = np.random.default_rng(4)
  gs = np.array([70, 130, 56], np.int32)
  lhs = O.bf16_round(_rand(rng, 256, 256))
  rhs = O.bf16_round(_rand(rng, 3, 256, 128))
  ref = O.ragged_dot(lhs, rhs, gs, dtype="fp32")
  out = lm.ragged_dot(to_dev(lhs), to_dev(rhs), torch.from_numpy(gs).cuda(),
                      preferred_element_type=torch.float32)
  # bf16 products are exact in f32; only the accumulation order differs
  assert np.abs(to_np(out) - ref).max() <= 1e-4 * np.abs(ref).max()


def test_ragged_dot_config2_full_size(lm):
  """Benchmark configuration 2: lhs (8192, 2048), rhs (128, 2048, 1536) bf16,
  Zipf(1.1) group sizes with empty groups; values N(0,1)/sqrt(K)."""
  rng = np.random.default_rng(1)
  m, k, n, g = 8192, 2048, 1536, 128
  gs = zipf_group_sizes(rng, m, g)
  assert (gs == 0).any()
  ref, got = _ragged_case(lm, rng, m, k, n, gs, "gkn")
  assert_gemm_close(ref, got, "config 2")


def test_ragged_dot_f32_kernel(lm):
  rng = np.random.default_rng(5)
  gs = np.array([5, 0, 60, 35], np.int32)
  lhs = _rand(rng, 110, 96)
  rhs = _rand(rng, 4, 96, 72)
  for layout in ("gkn", "gnk"):
    r = rhs if layout == "gkn" else np.ascontiguousarray(rhs.transpose(0, 2, 1))
    out = lm.ragged_dot(torch.from_numpy(lhs).cuda(), torch.from_numpy(r).cuda(),
                        torch.from_numpy(gs).cuda(), rhs_layout=layout)
    ref = O.ragged_dot(lhs, rhs, gs, dtype="fp32")
    assert np.allclose(to_np(out), ref, atol=1e-5, rtol=1e-5)
    assert np.all(to_np(out)[100:] == 0)


@pytest.mark.parametrize("layout", ["gkn", "gnk"])
@pytest.mark.parametrize("round_gate_up", [True, False])
def test_fused_gateup_situ(lm, layout, round_gate_up):
  rng = np.random.default_rng(6)
  m, k, inter, g = 1500, 512, 384, 6
  gs = rng.multinomial(m - 20, np.full(g, 1.0 / g)).astype(np.int32)
  lhs = O.bf16_round(_rand(rng, m, k))
  wg = O.bf16_round(_rand(rng, g, k, inter, scale=0.02))
  wu = O.bf16_round(_rand(rng, g, k, inter, scale=0.02))
  fused = np.concatenate([wg, wu], axis=-1)
  # compute dtype bf16 (gate/up rounded when round_gate_up), f32 result
  ref = O.fused_gateup_situ(lhs, fused, gs, inter, 4.0, 25.0, dtype="bf16",
                            round_gate_up=round_gate_up, out_dtype="fp32")
  w_dev = fused if layout == "gkn" else np.ascontiguousarray(fused.transpose(0, 2, 1))
  out = lm.fused_gateup_situ(to_dev(lhs), to_dev(w_dev), torch.from_numpy(gs).cuda(),
                             round_gate_up=round_gate_up, rhs_layout=layout)
  got = to_np(out)
  assert np.all(got[gs.sum():] == 0)
  assert_bf16_close(ref, got, f"situ {layout} round={round_gate_up}")


def test_fused_gateup_matches_unfused_kernels(lm):
  """Fused vs unfused: ragged_dot(gate), ragged_dot(up), situ_and_mul; with the
  bf16-round convention the two are bit-identical."""
  rng = np.random.default_rng(7)
  m, k, inter, g = 640, 256, 256, 5
  gs = rng.multinomial(m, np.full(g, 1.0 / g)).astype(np.int32)
  lhs = to_dev(_rand(rng, m, k))
  wg = to_dev(_rand(rng, g, k, inter, scale=0.05))
  wu = to_dev(_rand(rng, g, k, inter, scale=0.05))
  gsd = torch.from_numpy(gs).cuda()
  gate = lm.ragged_dot(lhs, wg, gsd)
  up = lm.ragged_dot(lhs, wu, gsd)
  unfused = lm.situ_and_mul(gate, up)
  fused = lm.fused_gateup_situ(lhs, lm.prefuse_gateup_weights(wg, wu), gsd)
  assert torch.equal(unfused, fused)


def test_dense_gemm_residual_add(lm):
  rng = np.random.default_rng(8)
  a = O.bf16_round(_rand(rng, 333, 512))
  w = O.bf16_round(_rand(rng, 512, 264, scale=0.02))
  add = O.bf16_round(_rand(rng, 333, 264, scale=0.25))
  ref = a @ w + add
  out = lm.gemm(to_dev(a), to_dev(np.ascontiguousarray(w.T)), addend=to_dev(add))
  assert_bf16_close(ref, to_np(out), "gemm+add")


def test_device_status_reports_oversized_groups(lm):
  """group sizes summing past M are rejected on the device (no out-of-bounds
  access): the status word records LMOE_DEVICE_BOUNDS."""
  lhs = torch.zeros(64, 64, dtype=torch.bfloat16, device="cuda")
  rhs = torch.zeros(2, 64, 64, dtype=torch.bfloat16, device="cuda")
  gs = torch.tensor([60, 60], dtype=torch.int32, device="cuda")
  lm.ragged_dot(lhs, rhs, gs)
  with pytest.raises(RuntimeError, match="status 4"):
    lm.check_device_status()
  lm.check_device_status()  # reset by the previous check


def test_unsupported_shapes_raise(lm):
  lhs = torch.zeros(16, 20, dtype=torch.bfloat16, device="cuda")
  rhs = torch.zeros(1, 20, 16, dtype=torch.bfloat16, device="cuda")
  with pytest.raises(NotImplementedError):
    lm.ragged_dot(lhs, rhs, torch.tensor([16], dtype=torch.int32, device="cuda"))
  with pytest.raises(NotImplementedError):
    lm.ragged_dot(lhs, rhs, torch.tensor([16], dtype=torch.int32, device="cuda"),
                  implementation="mosaic_tpu_v2")


@pytest.mark.parametrize("layout", ["gkn", "gnk"])
def test_fused_gateup_with_row_gather(lm, layout):
  """The dispatch gather fused into the operand load (TMA tile::gather4):
  logical row r = x[row_index[r]], index -1 = a zero row."""
  rng = np.random.default_rng(13)
  t, k, inter, g, m = 300, 256, 256, 4, 1000
  x = O.bf16_round(_rand(rng, t, k))
  idx = rng.integers(-1, t, m).astype(np.int32)
  gs = rng.multinomial(m - 9, np.full(g, 1.0 / g)).astype(np.int32)
  fused = O.bf16_round(_rand(rng, g, k, 2 * inter, scale=0.02))
  rows = np.where(idx[:, None] >= 0, x[np.maximum(idx, 0)], 0).astype(np.float32)
  ref = O.fused_gateup_situ(rows, fused, gs, inter, 4.0, 25.0, dtype="bf16", out_dtype="fp32")
  w_dev = fused if layout == "gkn" else np.ascontiguousarray(fused.transpose(0, 2, 1))
  out = lm.fused_gateup_situ(to_dev(x), to_dev(w_dev), torch.from_numpy(gs).cuda(),
                             rhs_layout=layout, row_index=torch.from_numpy(idx).cuda())
  direct = lm.fused_gateup_situ(to_dev(rows), to_dev(w_dev), torch.from_numpy(gs).cuda(),
                                rhs_layout=layout)
  assert torch.equal(out, direct)  # same rows, same bits
  assert_bf16_close(ref, to_np(out), f"gather {layout}")


def test_token_major_kernels_repeat_bit_exactly(lm):
  """Large grouped calls of the token-major kernel -- bf16 ragged_dot, fused
  gate/up with the in-kernel row gather, its MXFP4 form (more groups than the
  weights-major kernel's schedule holds) and the fp8 form -- give identical
  bits on every call, with every output element written (NaN-prefilled)."""
  from tokamax_tpu_kernel_lab_b200.latent_moe import random_mxfp4
  rng = np.random.default_rng(41)
  gen = torch.Generator(device="cuda").manual_seed(41)
  m, k, inter, g = 65536, 2048, 1024, 128

  def groups(rows, n, alpha):
    return torch.from_numpy(rng.multinomial(rows, rng.dirichlet(np.full(n, alpha)))
                            .astype(np.int32)).cuda()

  def repeats(shape, dtype, run, reps=3):
    first = None
    for _ in range(reps):
      o = torch.full(shape, float("nan"), dtype=dtype, device="cuda")
      run(o)
      torch.cuda.synchronize()
      lm.check_device_status()
      assert not bool(torch.isnan(o).any())
      if first is None:
        first = o
      else:
        assert torch.equal(o.view(torch.int16), first.view(torch.int16))

  x = torch.randn(m, k, generator=gen, device="cuda").to(torch.bfloat16)
  gs = groups(m, g, 0.5)
  w_gu = (torch.randn(g, 2 * inter, k, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
  row_index = torch.randint(-1, m, (m,), generator=gen, device="cuda").to(torch.int32)
  repeats((m, inter), torch.bfloat16,
          lambda o: lm.fused_gateup_situ(x, w_gu, gs, rhs_layout="gnk", out=o,
                                         row_index=row_index))
  w_dn = (torch.randn(g, k, inter, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
  act = torch.randn(m, inter, generator=gen, device="cuda").to(torch.bfloat16)
  repeats((m, k), torch.bfloat16, lambda o: lm.ragged_dot(act, w_dn, gs, rhs_layout="gnk", out=o))
  del w_gu, w_dn
  g_many = 2000
  gs_many = groups(m, g_many, 2.0)
  gu_mx = random_mxfp4(g_many, 2 * inter, k, seed=41)
  repeats((m, inter), torch.float16,
          lambda o: lm.mxfp4_fused_gateup_situ(x.to(torch.float16), gu_mx, gs_many, out=o,
                                               out_dtype=torch.float16))
  del gu_mx
  q = (torch.randn(32, k, k, generator=gen, device="cuda") * 4).to(torch.float8_e4m3fn)
  scale = torch.rand(32, k // 128, k, generator=gen, device="cuda") * 0.01
  gs_fp8 = groups(m // 2, 32, 0.5)
  repeats((m // 2, k), torch.bfloat16,
          lambda o: lm.fp8_ragged_dot(x[:m // 2], q, gs_fp8, scale, out=o))


@pytest.mark.parametrize("kind", ["bf16", "f32", "f16", "add", "situ"])
def test_narrow_tiles_equal_wide_tiles(lm, kind):
  """A dense GEMM with few token rows takes 128-wide weight tiles (more CTAs,
  a deeper ring); one with many rows, 256-wide tiles.  Rows present in both
  must come out bit-identical (each output element sums its K products in
  the same order either way), for every epilogue the layer's dense
  projections use; the narrow result also matches the oracle."""
  from tokamax_tpu_kernel_lab_b200 import ops
  g = torch.Generator(device="cuda").manual_seed(12)
  m_small, m_big, k, n = 200, 5120, 1024, 2048
  a = (torch.randn(m_big, k, generator=g, device="cuda") / k ** 0.5).to(torch.bfloat16)
  if kind == "situ":
    w = (torch.randn(2 * n, k, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    run = lambda x: ops.fused_gateup_situ(x, w, None, rhs_layout="gnk")
  else:
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    add = torch.randn(m_big, n, generator=g, device="cuda").to(torch.bfloat16)
    dt = {"bf16": torch.bfloat16, "f32": torch.float32, "f16": torch.float16,
          "add": torch.bfloat16}[kind]
    run = lambda x: ops.gemm(x, w, out_dtype=dt,
                             addend=add[:x.shape[0]].contiguous() if kind == "add" else None)
  wide = run(a)      # 40 token blocks x 8 (or 16) tiles: 256-wide tiles
  narrow = run(a[:m_small].contiguous())  # 2 token blocks: 128-wide tiles
  torch.cuda.synchronize()
  lm.check_device_status()
  assert torch.equal(narrow.view(torch.uint8), wide[:m_small].contiguous().view(torch.uint8))
  if kind == "bf16":
    ref = to_np(a[:m_small]) @ to_np(w).T
    assert_gemm_close(ref, to_np(narrow), "narrow-tile gemm")
