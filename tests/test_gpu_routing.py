"""GPU parity of the routing kernels through the C ABI: router top-k (indices
bit-exact given the oracle's logits), dispatch (order / group sizes /
slot positions bit-exact; shard form bit-exact incl. overflow, sentinel
padding, padding bucket), row gather (bit-exact), weighted combine + RMSNorm
and the scatter-add shard combine (within tolerance)."""

import numpy as np
import pytest
import torch

from oracle import lmoe_oracle as O
from tests.gpu_util import assert_bf16_close, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm():
  import tokamax_tpu_kernel_lab_b200 as lm
  lm.load_native()
  return lm


def _logits(rng, t, e, bias_std=0.5):
  logits = rng.standard_normal((t, e), dtype=np.float32) * np.float32(2.0)
  bias = rng.standard_normal(e, dtype=np.float32) * np.float32(bias_std)
  return logits, bias


@pytest.mark.parametrize("t,e,k", [(64, 8, 2), (256, 64, 8), (1000, 896, 16), (37, 1024, 32),
                                   (5, 33, 1)])
def test_router_topk_bit_exact_given_logits(lm, t, e, k):
  rng = np.random.default_rng(t + e + k)
  logits, bias = _logits(rng, t, e)
  _, scores, sfc, ref_idx, ref_w = O.router_from_logits(logits, bias, k)
  idx, w = lm.router_topk(torch.from_numpy(logits).cuda(), torch.from_numpy(bias).cuda(), k)
  got_idx = idx.cpu().numpy()
  # indices bit-exact except where the oracle's k-th / (k+1)-th selection
  # scores are within 1e-6 (a 1-ulp sigmoid difference can flip a near-tie)
  mismatch = np.any(got_idx != ref_idx, axis=1)
  if mismatch.any():
    srt = -np.sort(-sfc, axis=1)
    gap = srt[:, k - 1] - srt[:, min(k, e - 1)] if k < e else np.full(t, np.inf)
    assert np.all(gap[mismatch] < 1e-6), f"{mismatch.sum()} rows differ beyond near-ties"
  assert mismatch.sum() <= max(1, t // 1000)
  ok = ~mismatch
  assert np.allclose(w.cpu().numpy()[ok], ref_w[ok], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("k", [16, 32])
def test_router_topk_one_lane_holds_every_winner(lm, k):
  """All winners among experts e = 3 (mod 32): the kernel's lane 3 (which
  holds those experts) wins every round and rescans its entries after every
  second win; the selection and its slot order still equal the oracle's."""
  rng = np.random.default_rng(k)
  t, e = 300, 1024
  logits = rng.standard_normal((t, e), dtype=np.float32) * np.float32(0.5)
  bias = np.zeros(e, np.float32)
  bias[3::32] = np.float32(4.0) + rng.random(e // 32, dtype=np.float32)
  _, _, sfc, ref_idx, ref_w = O.router_from_logits(logits, bias, k)
  idx, w = lm.router_topk(torch.from_numpy(logits).cuda(), torch.from_numpy(bias).cuda(), k)
  got = idx.cpu().numpy()
  assert np.all(got % 32 == 3)
  mismatch = np.any(got != ref_idx, axis=1)
  if mismatch.any():
    srt = -np.sort(-sfc, axis=1)
    gap = srt[:, k - 1] - srt[:, k]
    assert np.all(gap[mismatch] < 1e-6), f"{mismatch.sum()} rows differ beyond near-ties"
  assert mismatch.sum() <= 1
  ok = ~mismatch
  assert np.allclose(w.cpu().numpy()[ok], ref_w[ok], rtol=1e-6, atol=1e-7)


def test_router_ties_go_to_lower_index(lm):
  logits = np.zeros((3, 16), np.float32)
  logits[0, [3, 7, 9]] = 1.0
  logits[1, :] = 0.25
  logits[2, [15, 0]] = 2.0
  idx, _ = lm.router_topk(torch.from_numpy(logits).cuda(), None, 3)
  assert idx.cpu().tolist() == [[3, 7, 9], [0, 1, 2], [0, 15, 1]]


def test_router_softmax_branch(lm):
  rng = np.random.default_rng(11)
  logits, bias = _logits(rng, 200, 64)
  _, _, _, ref_idx, ref_w = O.router_from_logits(logits, bias, 6, activation="softmax")
  idx, w = lm.router_topk(torch.from_numpy(logits).cuda(), torch.from_numpy(bias).cuda(), 6,
                          activation="softmax")
  assert (idx.cpu().numpy() == ref_idx).mean() > 0.99
  same = np.all(idx.cpu().numpy() == ref_idx, axis=1)
  assert np.allclose(w.cpu().numpy()[same], ref_w[same], rtol=1e-5, atol=1e-6)


def test_router_gate_end_to_end_bf16(lm):
  """Logits on the tensor cores (bf16 operands, f32 accumulate) then top-k:
  index mismatches vs the f32 oracle only on near-ties."""
  rng = np.random.default_rng(12)
  t, d, e, k = 512, 1024, 256, 8
  h = O.bf16_round(rng.standard_normal((t, d), dtype=np.float32))
  wr = O.bf16_round(rng.standard_normal((d, e), dtype=np.float32) * np.float32(0.02))
  bias = rng.standard_normal(e, dtype=np.float32) * np.float32(0.5)
  _, _, sfc, ref_idx, _ = O.router_gate(h, wr, bias, k)
  idx, _ = lm.router_gate(to_dev(h), to_dev(np.ascontiguousarray(wr.T)),
                          torch.from_numpy(bias).cuda(), k)
  mismatch = np.any(idx.cpu().numpy() != ref_idx, axis=1)
  srt = -np.sort(-sfc, axis=1)
  gap = srt[:, k - 1] - srt[:, k]
  assert np.all(gap[mismatch] < 1e-5)


@pytest.mark.parametrize("t,k,e", [(20, 2, 8), (4096, 16, 896), (3000, 8, 64), (1, 16, 896),
                                   (700, 4, 2048)])
def test_dispatch_full_bit_exact(lm, t, k, e):
  rng = np.random.default_rng(t * k + e)
  scores = rng.random((t, e)).astype(np.float32) + rng.standard_normal(e).astype(np.float32)
  topk = O.top_k_desc(scores, k)
  w = rng.random((t, k)).astype(np.float32)
  order, sorted_tok, gs = O.dispatch_full(topk, e)
  d = lm.dispatch(torch.from_numpy(topk).cuda(), torch.from_numpy(w).cuda(), e)
  assert np.array_equal(d.order.cpu().numpy(), order)
  assert np.array_equal(d.group_sizes.cpu().numpy(), gs)
  assert np.array_equal(d.token_idx.cpu().numpy(), sorted_tok)
  slot_pos = d.slot_pos.cpu().numpy()
  assert np.array_equal(order[slot_pos], np.arange(t * k))
  assert np.array_equal(d.weight.cpu().numpy(), w.reshape(-1)[order])


@pytest.mark.parametrize("case", [
    # name, T, E, k, start, n_local, capacity_factor, tile
    ("standard", 64, 32, 2, 5, 8, 2.0, 128),
    ("overflow", 64, 32, 2, 5, 8, 0.05, 128),
    ("decode_scale", 1, 32, 2, 5, 8, 2.0, 128),
    ("kimi_shard", 256, 896, 16, 137, 64, 2.0, 128),
    ("ep8_shard", 2048, 896, 16, 784, 112, 2.0, 128),
    ("empty_shard", 5, 8, 2, 4, 2, 4.0, 1),
    ("tight", 4096, 896, 16, 0, 112, 1.0, 128),
])
def test_dispatch_shard_bit_exact(lm, case):
  """filter_and_pad_to_shard_jittable (kimi_k3_latent_moe_reference.py:754-877)."""
  name, t, e, k, start, n_local, cf, tile = case
  rng = np.random.default_rng(len(name) * 1000 + t)
  if name == "empty_shard":
    topk = np.array([[0, 1], [1, 2], [6, 7], [7, 0], [2, 3]], np.int32)
  else:
    scores = rng.random((t, e)).astype(np.float32) + np.float32(0.5) * rng.standard_normal(e).astype(np.float32)
    topk = O.top_k_desc(scores, k)
  w = rng.random((t, k)).astype(np.float32)
  x = O.bf16_round(rng.standard_normal((t, 64), dtype=np.float32))
  ref = O.filter_and_pad_to_shard_jittable(topk, w, x, e, k, start, n_local, cf, tile)
  got = lm.filter_and_pad_to_shard_jittable(torch.from_numpy(topk).cuda(),
                                            torch.from_numpy(w).cuda(), to_dev(x), e, k, start,
                                            n_local, cf, tile)
  names = ("sorted_tokens", "group_sizes", "valid_mask", "per_expert_counts", "padded_token_idx",
           "padded_combine_weight")
  for nm, r, g in zip(names, ref, got):
    g = g.float().cpu().numpy() if g.dtype == torch.bfloat16 else g.cpu().numpy()
    assert np.array_equal(np.asarray(r), g.astype(np.asarray(r).dtype)), nm


def test_gather_rows_bit_exact(lm):
  rng = np.random.default_rng(21)
  x = to_dev(rng.standard_normal((300, 2048), dtype=np.float32))
  idx = rng.integers(-1, 300, 5000).astype(np.int32)
  out = lm.gather_rows(x, torch.from_numpy(idx).cuda())
  xn = x.cpu()
  ref = torch.where(torch.from_numpy(idx)[:, None] >= 0, xn[np.maximum(idx, 0)], 0)
  assert torch.equal(out.cpu(), ref)


@pytest.mark.parametrize("t,k,e,dim,to_f16", [(300, 8, 64, 2048, False), (1000, 16, 896, 2048, True),
                                              (5, 3, 4, 8, False), (2, 1, 2, 4104, True)])
def test_scatter_rows_equals_gather(lm, t, k, e, dim, to_f16):
  """The token-order gather (each row read once, stored k times) writes the
  rows of the sorted-order gather bit for bit for a dropless dispatch,
  including rows longer than one 4 KB pass and the bf16 -> f16 conversion."""
  g = torch.Generator(device="cuda").manual_seed(t * k)
  x = torch.randn(t, dim, generator=g, device="cuda").to(torch.bfloat16)
  idx = torch.stack([torch.randperm(e, generator=g, device="cuda")[:k] for _ in range(t)]).int()
  d = lm.dispatch(idx, None, e, want_order=False)
  ref = lm.gather_rows(x, d.token_idx, to_f16=to_f16)
  got = lm.ops.scatter_rows(x, d.slot_pos, k, to_f16=to_f16)
  torch.cuda.synchronize()
  lm.check_device_status()
  assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


def test_scatter_rows_bounds(lm):
  """A slot position past the output is skipped and reported."""
  x = torch.ones(4, 64, dtype=torch.bfloat16, device="cuda")
  pos = torch.tensor([0, 1, 2, 3, 4, 5, 6, 100], dtype=torch.int32, device="cuda")
  out = torch.zeros(8, 64, dtype=torch.bfloat16, device="cuda")
  lm.ops.scatter_rows(x, pos, 2, out=out)
  torch.cuda.synchronize()
  with pytest.raises(lm._native.LmoeError):
    lm.check_device_status()
  assert torch.equal(out[:7], torch.ones(7, 64, dtype=torch.bfloat16, device="cuda"))
  assert torch.equal(out[7], torch.zeros(64, dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_combine_rmsnorm(lm, dtype):
  rng = np.random.default_rng(31)
  t, k, e, L = 333, 8, 64, 256
  topk = O.top_k_desc(rng.random((t, e)).astype(np.float32), k)
  w = rng.random((t, k)).astype(np.float32)
  w /= w.sum(1, keepdims=True)
  order, _, _ = O.dispatch_full(topk, e)
  outs = O.to_dtype(rng.standard_normal((t * k, L), dtype=np.float32), dtype)
  scale = O.to_dtype(1 + 0.1 * rng.standard_normal(L, dtype=np.float32), dtype)
  routed_ref, _ = O.combine_full(outs, order, w, dtype)
  normed_ref = O.rms_norm(routed_ref, scale, 1e-5, dtype)
  tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
  d = lm.dispatch(torch.from_numpy(topk).cuda(), torch.from_numpy(w).cuda(), e)
  routed, normed = lm.combine_rmsnorm(to_dev(outs, tdt), d.slot_pos, torch.from_numpy(w).cuda(),
                                      to_dev(scale, tdt), 1e-5, want_routed=True)
  if dtype == "bf16":
    # slot-order f32 accumulation as in the oracle: routed is bit-exact
    assert np.array_equal(to_np(routed), routed_ref)
    assert_bf16_close(normed_ref, to_np(normed), "normed")
  else:
    assert np.allclose(to_np(routed), routed_ref, atol=1e-6)
    assert np.allclose(to_np(normed), normed_ref, atol=1e-5, rtol=1e-5)


def test_combine_shard_scatter_add(lm):
  """_combine_shard_contribution (kimi_k3_latent_moe_reference.py:1113-1141),
  including padding rows with non-zero content and weight 0, idx -1."""
  rng = np.random.default_rng(41)
  t, L, rows = 50, 128, 300
  idx = rng.integers(-1, t, rows).astype(np.int32)
  w = rng.random(rows).astype(np.float32)
  w[idx < 0] = 0
  shard = O.bf16_round(rng.standard_normal((rows, L), dtype=np.float32) * np.float32(0.2))
  routed = O.bf16_round(rng.standard_normal((t, L), dtype=np.float32) * np.float32(0.2))
  ref = O.combine_shard_contribution(routed, shard, idx, w, "bf16")
  got = lm.combine_shard_contribution(to_dev(routed), to_dev(shard), torch.from_numpy(idx).cuda(),
                                      torch.from_numpy(w).cuda())
  # bf16 accumulation order of duplicate tokens differs from the sequential
  # scatter: compare within a few bf16 ulps of the running sum
  assert_bf16_close(ref, to_np(got), "scatter-add", rel=2e-2)
