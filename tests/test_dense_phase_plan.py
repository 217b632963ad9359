"""Host-side planning of the dense phase kernels (no GPU needed): when the
layer takes them, and the split plan the workspace size reveals -- the same
split count at every token count (so each token's result does not depend on
how many tokens share the call), one partial tile per (split, token block,
column tile)."""

import pytest

from tokamax_tpu_kernel_lab_b200 import _native, ops

TILE = 128 * 128 * 4  # one f32 partial tile


def _in_ws(t, d=7168, e=896, latent=2048, si=2048):
  return int(_native.load().lmoe_dense_input_workspace_size(t, d, e, latent, si))


def _out_ws(t, latent=2048, si=2048, d=7168):
  return int(_native.load().lmoe_dense_output_workspace_size(t, latent, si, d))


def test_layer_takes_the_phases_up_to_two_waves_of_tiles():
  # configuration 5: 7 + 16 + 32 = 55 input-phase tiles per 128-token block
  pay = lambda t: ops.dense_phases_pay_off(t, 896, 2048, 2048, sms=148)
  assert pay(1) and pay(128) and pay(512)
  assert pay(640) and not pay(641) and not pay(1024) and not pay(16384)
  assert not pay(0)


@pytest.mark.parametrize("t", [1, 100, 128, 129, 256, 512])
def test_split_count_does_not_depend_on_tokens(t):
  n_tiles = 7 + 16 + 32
  m_tiles = -(-t // 128)
  counters = (m_tiles * n_tiles * 4 + 255) // 256 * 256
  partials = _in_ws(t) - counters
  assert partials % (m_tiles * n_tiles * TILE) == 0
  splits = partials // (m_tiles * n_tiles * TILE)
  assert splits == (_in_ws(128) - 256) // (n_tiles * TILE)
  assert 1 <= splits <= 32
  out_tiles = 7168 // 128
  out_counters = (m_tiles * out_tiles * 4 + 255) // 256 * 256
  out_splits = (_out_ws(t) - out_counters) // (m_tiles * out_tiles * TILE)
  assert out_splits >= 2  # one split per K segment at least (normed x W_up, shared x W_sd)


def test_unsupported_shapes_report_zero():
  assert _in_ws(128, d=100) == 0           # K not a multiple of 64
  assert _in_ws(128, e=6) == 0             # logits rows not 16-byte multiples
  assert _out_ws(128, latent=100) == 0
  assert _in_ws(-1) == 0
