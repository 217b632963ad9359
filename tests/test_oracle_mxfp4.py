"""CPU checks of the oracle's MXFP4 decode (MXD:29-67, MXO:65-91).

compressed-tensors (the library MXD:70-112 checks against) is not installed,
so the decode is pinned by the E2M1 table, the sign-bit rule for nibble 8
(-0.0, MXO:65-75), the low-nibble-first packing order (MXD:14-20) and the
exact power-of-two scale for every byte the format allows.
"""

import numpy as np

from oracle import lmoe_oracle as O


def test_e2m1_table_and_negative_zero():
  packed = np.array([[0x10, 0x32, 0x54, 0x76, 0x98, 0xBA, 0xDC, 0xFE]], np.uint8)
  scale = np.array([[127, 127]], np.uint8)[:, :1].repeat(1, 1)
  out = O.dequantize_mxfp4(packed, np.array([[127]], np.uint8))
  assert out.shape == (1, 16)
  expect = [0, .5, 1, 1.5, 2, 3, 4, 6, -0.0, -.5, -1, -1.5, -2, -3, -4, -6]
  assert out[0].tolist() == expect
  assert np.signbit(out[0, 8]) and not np.signbit(out[0, 0])
  del scale


def test_low_nibble_is_even_k():
  packed = np.array([[0x2F]], np.uint8)  # low nibble 0xF (-6), high 0x2 (1.0)
  out = O.dequantize_mxfp4(np.repeat(packed, 16, axis=1), np.array([[127]], np.uint8))
  assert out[0, 0] == -6.0 and out[0, 1] == 1.0


def test_scale_is_exact_power_of_two():
  codes = np.full((1, 16), 0x22, np.uint8)  # every element 1.0
  for s in range(1, 255):
    out = O.dequantize_mxfp4(codes, np.array([[s]], np.uint8))
    assert np.all(out == np.float32(2.0) ** (s - 127)), s


def test_group_size_32_blocks():
  rng = np.random.default_rng(0)
  packed = rng.integers(0, 256, (4, 64), dtype=np.uint8)
  scale = rng.integers(120, 130, (4, 4), dtype=np.uint8)
  out = O.dequantize_mxfp4(packed, scale)
  base = O.dequantize_mxfp4(packed, np.full_like(scale, 127))
  for b in range(4):
    f = (2.0 ** (scale[:, b].astype(np.float64) - 127))[:, None]
    assert np.array_equal(out[:, b * 32:(b + 1) * 32], (base[:, b * 32:(b + 1) * 32] * f).astype(np.float32))


def test_mxfp4_ragged_dot_matches_dense_loop():
  rng = np.random.default_rng(1)
  g, n, k = 3, 16, 64
  packed = rng.integers(0, 256, (g, n, k // 2), dtype=np.uint8)
  scale = rng.integers(121, 130, (g, n, k // 32), dtype=np.uint8)
  gs = np.array([5, 0, 7], np.int32)
  lhs = rng.standard_normal((14, k)).astype(np.float32)
  out = O.mxfp4_ragged_dot(lhs, packed, scale, gs, dtype="fp32")
  w0 = O.dequantize_mxfp4(packed[0], scale[0])
  w2 = O.dequantize_mxfp4(packed[2], scale[2])
  assert np.allclose(out[:5], lhs[:5] @ w0.T, atol=1e-5)
  assert np.allclose(out[5:12], lhs[5:12] @ w2.T, atol=1e-5)
  assert np.all(out[12:] == 0)


def test_fp8_blockwise_quantisation_round_trip():
  """The restated rhs_scale quantisation (KRD:2883-2898): codes are e4m3
  values within +-448, every block's absmax maps to 448, and the dequantised
  weight is within e4m3's relative step (2^-3 of the block absmax) of the
  input."""
  rng = np.random.default_rng(11)
  w = (rng.standard_normal((3, 256, 96)) * 0.02).astype(np.float32)
  for block in (32, 256):
    q, scale = O.quantize_fp8_blockwise(w, block)
    assert q.shape == w.shape and scale.shape == (3, 256 // block, 96)
    assert np.array_equal(O.e4m3_round(q), q)
    assert float(np.abs(q).max()) == 448.0
    d = O.dequantize_fp8_blockwise(q, scale)
    blocks = np.abs(w.reshape(3, 256 // block, block, 96)).max(axis=2)
    bound = np.repeat(blocks, block, axis=1).reshape(w.shape) * (2.0 ** -3) + 1e-8
    assert np.all(np.abs(d - w) <= bound)


def test_fp8_ragged_dot_is_ragged_dot_on_the_dequantised_weight():
  rng = np.random.default_rng(12)
  w = (rng.standard_normal((2, 64, 32)) * 0.02).astype(np.float32)
  q, scale = O.quantize_fp8_blockwise(w, 32)
  lhs = O.bf16_round(rng.standard_normal((10, 64)).astype(np.float32))
  gs = np.array([7, 3], np.int32)
  ref = O.ragged_dot(lhs, O.dequantize_fp8_blockwise(q, scale), gs, dtype="fp32")
  assert np.array_equal(O.fp8_ragged_dot(lhs, q, scale, gs, dtype="fp32"), ref)


def test_mxfp4_activation_scale_rule_and_rounding():
  """MXFP4 activation rows: per 32 values the scale is the smallest power of
  two 2^e with amax <= 6 * 2^e (no element saturates), the values are the
  nearest-even e2m1 grid points of x / 2^e, and an all-zero block gets byte 0."""
  rng = np.random.default_rng(13)
  x = (rng.standard_normal((64, 256)) * 10.0 ** rng.uniform(-4, 4, (64, 1))).astype(np.float32)
  x[0] = 0.0
  x[1, :32] = 6.0
  x[2, :32] = 6.0000005   # just above: the next scale
  q, sf = O.quantize_mxfp4_act(x)
  e = sf.astype(np.int32) - 127
  amax = np.abs(x.reshape(64, 8, 32)).max(axis=2)
  nz = amax > 0
  assert np.all(amax[nz] <= 6.0 * np.ldexp(1.0, e[nz]))
  assert np.all(amax[nz] > 6.0 * np.ldexp(1.0, e[nz] - 1))  # the smallest such
  assert np.all(sf[0] == 0) and sf[1, 0] == 127 and sf[2, 0] == 128
  grid = np.concatenate([-O.FP4_E2M1_TABLE, O.FP4_E2M1_TABLE])
  assert np.all(np.isin(q, grid))
  scaled = x.reshape(64, 8, 32) / np.ldexp(1.0, e)[:, :, None]
  err = np.abs(q.reshape(64, 8, 32) - scaled)
  # nearest grid point: within half the local grid spacing (0.25 below 2, 0.5 below 4, 1 above)
  half = np.where(np.abs(scaled) < 2, 0.25, np.where(np.abs(scaled) < 4, 0.5, 1.0))
  assert np.all(err <= half + 1e-6)


def test_mxfp4_activation_ties_and_packing():
  """Ties go to the even grid point; two values per byte, the even K index in
  the low nibble, sign in bit 3 (the packing of the MXFP4 weights, so
  dequantize_mxfp4 reads the activation rows back)."""
  ties = np.array([[0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.75] * 4], np.float32)
  q, sf = O.quantize_mxfp4_act(ties)
  assert sf[0, 0] == 127
  assert np.array_equal(q[0, :8], np.array([0, 1, 1, 2, 2, 4, 4, -1], np.float32))
  packed = O.pack_e2m1(q)
  assert packed.shape == (1, 16)
  assert packed[0, 0] == (0x0 | (0x2 << 4)) and packed[0, 3] == (0x6 | (0xA << 4))
  back = O.dequantize_mxfp4(packed, sf)
  assert np.array_equal(back, O.dequantize_mxfp8(q, sf))


def test_mxfp4_activation_error_is_the_e2m1_step():
  """N(0,1) rows lose ~10% normwise to e2m1 (one mantissa bit), against ~3%
  for e4m3: the size of the opt-in error."""
  rng = np.random.default_rng(14)
  x = rng.standard_normal((256, 1024)).astype(np.float32)
  e4 = O.dequantize_mxfp8(*O.quantize_mxfp4_act(x))
  e8 = O.dequantize_mxfp8(*O.quantize_mxfp8(x))
  r4 = float(np.linalg.norm(e4 - x) / np.linalg.norm(x))
  r8 = float(np.linalg.norm(e8 - x) / np.linalg.norm(x))
  assert 0.08 < r4 < 0.16 and 0.015 < r8 < 0.04


def test_split_e4m3_holds_the_bf16_value():
  """Two e4m3 planes under the MXFP8 block scale 2^e (hi, and lo = the
  rounding remainder) hold every bf16 value with |x| >= 2^(e-2) exactly and
  the rest to within 2^(e-10): the exact product on the block-scaled MMA."""
  rng = np.random.default_rng(15)
  x = O.bf16_round((rng.standard_normal((128, 512)) *
                    10.0 ** rng.uniform(-6, 6, (128, 1))).astype(np.float32))
  x[0, :32] = 448.0
  x[1, :31] = 1e-30
  x[1, 31] = 1.0
  hi, lo, sf = O.split_e4m3(x)
  assert np.array_equal(O.e4m3_round(hi), hi) and np.array_equal(O.e4m3_round(lo), lo)
  np.testing.assert_array_equal(sf, O.quantize_mxfp8(x)[1])
  e = np.repeat(sf.astype(np.int32) - 127, 32, axis=1)
  d = O.dequantize_split(hi, lo, sf)
  big = np.abs(x) >= np.ldexp(1.0, e - 2)
  assert big.mean() > 0.99
  assert np.array_equal(d[big], x[big])
  assert np.all(np.abs(d - x)[~big] <= np.ldexp(1.0, e - 10)[~big])
