"""Host-side selection logic of the layer (no GPU needed): which MXFP4
expert path each `mxfp4_operand` runs, and the expert sharding of the
expert-parallel path."""

import pytest
import torch

from tokamax_tpu_kernel_lab_b200 import ops
from tokamax_tpu_kernel_lab_b200.expert_parallel import shard_experts
from tokamax_tpu_kernel_lab_b200.latent_moe import (PreparedWeights, mxfp4_f16_path,
                                                     resolve_mxfp4_operand)


def _pw(e=8, scale_byte=120):
  z = lambda *s: torch.zeros(*s, dtype=torch.bfloat16)
  gu = ops.MXFP4Weights(torch.arange(e * 32 * 32, dtype=torch.int32).to(torch.uint8).view(e, 32, 32),
                        torch.full((e, 32, 2), scale_byte, dtype=torch.uint8))
  dn = ops.MXFP4Weights(torch.zeros(e, 64, 8, dtype=torch.uint8),
                        torch.full((e, 64, 1), scale_byte, dtype=torch.uint8))
  return PreparedWeights(dtype=torch.bfloat16, router=z(e, 128), bias=torch.zeros(e),
                         down=z(64, 128), up=z(128, 64), expert_gu=None, expert_gate=None,
                         expert_up=None, expert_down=None, norm_scale=z(64), shared_gu=z(32, 128),
                         shared_gate=None, shared_up=None, shared_down=z(128, 16),
                         expert_gu_mx=gu, expert_down_mx=dn)


def test_auto_is_the_exact_block_scaled_path():
  pw = _pw()
  assert resolve_mxfp4_operand(pw, "auto") == "split"
  for mode in ("split", "f16", "bf16", "mxfp8", "mxfp4"):
    assert resolve_mxfp4_operand(pw, mode) == mode
  with pytest.raises(ValueError):
    resolve_mxfp4_operand(pw, "fp8")
  # bf16 experts: "auto" stays "auto" (no MXFP4 kernels involved)
  bf = _pw()
  bf.expert_gu_mx = bf.expert_down_mx = None
  assert resolve_mxfp4_operand(bf, "auto") == "auto"


def test_f16_operands_only_in_f16_mode_and_exact_scale_range():
  assert mxfp4_f16_path(_pw(), "f16")
  assert not mxfp4_f16_path(_pw(), "split")
  assert not mxfp4_f16_path(_pw(), "bf16")
  assert not mxfp4_f16_path(_pw(scale_byte=150), "f16")  # 2^23: outside f16's exact range
  assert not mxfp4_f16_path(_pw(scale_byte=100), "f16")


def test_shard_experts_slices_and_drops_the_full_block_scaled_repack():
  pw = _pw(e=8)
  pw.expert_gu_bs = object()  # stands for the full set's repack
  pw.expert_down_bs = object()
  sh = shard_experts(pw, 1, 4)
  assert sh.expert_gu_bs is None and sh.expert_down_bs is None
  assert torch.equal(sh.expert_gu_mx.packed, pw.expert_gu_mx.packed[2:4])
  assert torch.equal(sh.expert_down_mx.scale, pw.expert_down_mx.scale[2:4])
  assert pw.expert_gu_bs is not None  # the full set keeps its own
