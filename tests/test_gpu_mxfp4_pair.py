"""GPU parity of the CTA-pair MXFP4 kernel (csrc/mxfp4_pair.cu: one
`tcgen05.mma.cta_group::2` over two SMs, each SM expanding its 128 weight rows
and staging half of the tokens).  The kernel is selected per process by
LMOE_MXFP4_PAIR=1, so the checks run in a child process with that variable
set and compare against the single-CTA kernel's bits in this process."""

import os
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent("""
    import sys, zlib, numpy as np, torch
    sys.path.insert(0, {root!r})
    import tokamax_tpu_kernel_lab_b200 as lm
    from tokamax_tpu_kernel_lab_b200.latent_moe import random_mxfp4
    rng = np.random.default_rng(51)
    out = []
    for (g, inter, latent, m, f16) in [(7, 384, 512, 3000, True), (33, 1024, 2048, 40000, True),
                                       (5, 256, 1024, 1500, False)]:
        gs = torch.from_numpy(rng.multinomial(m - 37, rng.dirichlet(np.full(g, 0.7)))
                              .astype(np.int32)).cuda()
        gu = random_mxfp4(g, 2 * inter, latent, seed=g)
        dn = random_mxfp4(g, latent, inter, seed=g + 1)
        gen = torch.Generator(device="cuda").manual_seed(g)
        x = torch.randn(m, latent, generator=gen, device="cuda").to(torch.bfloat16)
        if f16:
            x = x.to(torch.float16)
        dt = torch.float16 if f16 else torch.bfloat16
        act = lm.mxfp4_fused_gateup_situ(x, gu, gs, out_dtype=dt)
        down = lm.mxfp4_ragged_dot(act, dn, gs)
        down32 = lm.mxfp4_ragged_dot(act, dn, gs, preferred_element_type=torch.float32)
        torch.cuda.synchronize()
        lm.check_device_status()
        for t in (act, down, down32):
            out.append(zlib.crc32(t.contiguous().view(torch.uint8).cpu().numpy().tobytes()))
    print(" ".join(map(str, out)))
""").format(root=ROOT)


def _run(pair: bool) -> list[int]:
  env = dict(os.environ)
  env["LMOE_MXFP4_PAIR"] = "1" if pair else "0"
  res = subprocess.run([sys.executable, "-c", CHILD], env=env, capture_output=True, text=True,
                       timeout=600)
  assert res.returncode == 0, res.stderr[-2000:]
  return [int(v) for v in res.stdout.split()]


def test_pair_kernel_matches_single_cta_kernel_bit_for_bit():
  """gate/up + SiTU (f16 and bf16 operands), bf16 and f32 down outputs, ragged
  groups with a tail of unused rows: the pair kernel's bits equal the
  single-CTA kernel's, whose parity against the oracle the other MXFP4 tests
  pin."""
  assert torch.cuda.is_available()
  single = _run(pair=False)
  pair = _run(pair=True)
  assert len(single) == 9
  assert pair == single
