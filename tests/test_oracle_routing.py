"""CPU checks of the oracle's routing / dispatch / combine restatement.

Restates the reference's own CPU-only checks:
- dispatch round trip (KR:438-471)
- the ten edge cases of 05_ragged_dot_on_tpu/test_sharded_routing_local.py
  (empty shard, extreme skew, capacity overflow, padding non-contamination,
  top_k=16, shard boundary, first/last shard, batch/seq invariance, dtype,
  sharded sum == unsharded)
- jittable dispatch == eager dispatch (KR:880-939), incl. overflow and
  decode-scale cases
- sharded forward == unsharded forward (KR:1531-1674)
Seeds are fixed integers (the reference's `hash(name)` seeds are not
reproducible across processes).
"""

import numpy as np
import pytest

from oracle import lmoe_oracle as O


def _cfg(top_k=4, num_experts=32):
  return O.LatentMoEConfig(64, 32, 48, num_experts, top_k, 1)


def test_dispatch_roundtrip():
  rng = np.random.default_rng(0)
  cfg = O.toy_config()
  x = rng.standard_normal((20, cfg.latent_size)).astype(np.float32)
  scores = rng.random((20, cfg.num_experts)).astype(np.float32)
  topk = O.top_k_desc(scores, cfg.top_k)
  order, sorted_tok, gs = O.dispatch_full(topk, cfg.num_experts)
  outs = x[sorted_tok]
  unsorted = np.zeros_like(outs)
  unsorted[order] = outs
  assert np.array_equal(unsorted.reshape(20, cfg.top_k, -1),
                        np.broadcast_to(x[:, None, :], (20, cfg.top_k, cfg.latent_size)))
  assert gs.sum() == 20 * cfg.top_k


def test_top_k_ties_go_to_lower_index():
  scores = np.array([[0.5, 0.7, 0.7, 0.1, 0.7]], np.float32)
  assert O.top_k_desc(scores, 3).tolist() == [[1, 2, 4]]


def test_dispatch_is_stable():
  topk = np.array([[3, 1], [1, 3], [3, 0]], np.int32)
  order, sorted_tok, gs = O.dispatch_full(topk, 4)
  assert order.tolist() == [5, 1, 2, 0, 3, 4]
  assert gs.tolist() == [1, 2, 0, 3]


def _shard(topk, w, x, cfg, start, n_local, cf, tile=1, jittable=True):
  fn = O.filter_and_pad_to_shard_jittable if jittable else O.filter_and_pad_to_shard
  return fn(topk, w, x, cfg.num_experts, cfg.top_k, start, n_local, cf, tile)


def test_empty_shard():
  """test_sharded_routing_local.py:62-94."""
  cfg = _cfg(top_k=2, num_experts=8)
  topk = np.array([[0, 1], [1, 2], [6, 7], [7, 0], [2, 3]], np.int32)
  w = np.full((5, 2), 0.5, np.float32)
  x = np.random.default_rng(0).standard_normal((5, cfg.latent_size)).astype(np.float32)
  for jit in (True, False):
    st, gs, valid, counts, idx, pw = _shard(topk, w, x, cfg, 4, 2, 4.0, jittable=jit)
    assert counts.sum() == 0 and valid.sum() == 0
    assert np.all(st == 0) and np.all(pw == 0) and np.all(idx == -1)


def test_extreme_skew():
  """test_sharded_routing_local.py:97-125."""
  cfg = _cfg(top_k=1, num_experts=16)
  topk = np.full((50, 1), 5, np.int32)
  w = np.full((50, 1), 0.7, np.float32)
  x = np.random.default_rng(1).standard_normal((50, cfg.latent_size)).astype(np.float32)
  st, gs, valid, counts, idx, pw = _shard(topk, w, x, cfg, 3, 5, 4.0)
  assert counts.tolist() == [0, 0, 50, 0, 0] and valid.sum() == 50


def test_capacity_overflow_drops_tail():
  """test_sharded_routing_local.py:128-167."""
  cfg = _cfg(top_k=1, num_experts=8)
  rng = np.random.default_rng(2)
  topk = rng.integers(0, 4, (20, 1)).astype(np.int32)
  w = np.full((20, 1), 0.3, np.float32)
  x = rng.standard_normal((20, cfg.latent_size)).astype(np.float32)
  for jit in (True, False):
    st, gs, valid, counts, idx, pw = _shard(topk, w, x, cfg, 0, 4, 0.1, jittable=jit)
    m_padded = int(gs.sum())
    keep = int(valid.sum())
    assert keep < 20 and keep == m_padded
    ref = [tok for tok, _ in sorted(enumerate(topk.reshape(-1).tolist()),
                                    key=lambda p: p[1])[:m_padded]]
    assert idx[:keep].tolist() == ref


def test_padding_does_not_contaminate():
  """test_sharded_routing_local.py:170-194."""
  shard_out = np.random.default_rng(3).standard_normal((6, 8)).astype(np.float32)
  idx = np.array([0, 1, 2, 3, -1, -1], np.int32)
  w = np.array([0.5, 0.5, 0.5, 0.5, 0.0, 0.0], np.float32)
  routed = O.combine_shard_contribution(np.zeros((4, 8), np.float32), shard_out, idx, w, "fp32")
  assert np.abs(routed - shard_out[:4] * 0.5).max() < 1e-6


@pytest.mark.parametrize("jit", [True, False])
def test_top_k_16_and_boundaries(jit):
  """test_sharded_routing_local.py:197-305: top_k=16, ids exactly at the shard
  start/end, first and last shard of a tiling."""
  cfg = _cfg(top_k=16, num_experts=64)
  rng = np.random.default_rng(4)
  t = 24
  scores = rng.random((t, 64)).astype(np.float32)
  topk = O.top_k_desc(scores, 16)
  topk[0, 0], topk[1, 0] = 16, 31  # shard [16, 32) boundaries
  w = rng.random((t, 16)).astype(np.float32)
  x = rng.standard_normal((t, cfg.latent_size)).astype(np.float32)
  total = 0
  for start in range(0, 64, 16):
    st, gs, valid, counts, idx, pw = _shard(topk, w, x, cfg, start, 16, 8.0, jittable=jit)
    in_shard = (topk >= start) & (topk < start + 16)
    assert counts.sum() == in_shard.sum()
    for e in range(16):
      assert counts[e] == (topk == start + e).sum()
    total += int(valid.sum())
  assert total == t * 16


def test_batch_seq_invariance():
  """test_sharded_routing_local.py:308-339: only the flattened token axis matters."""
  cfg = O.toy_config()
  w = O.init_weights_np(cfg, 5)
  rng = np.random.default_rng(5)
  h = rng.standard_normal((2, 16, cfg.hidden_size)).astype(np.float32)
  a = O.latent_moe_forward(h.reshape(32, -1), w, cfg)
  b = np.concatenate([O.latent_moe_forward(h[i], w, cfg) for i in range(2)])
  assert np.abs(a - b).max() < 1e-6


def test_bf16_stays_bf16_with_empty_groups():
  """test_sharded_routing_local.py:342-392: every bf16 stage is bf16-valued,
  including when experts receive zero tokens."""
  cfg = O.LatentMoEConfig(64, 32, 48, 64, 2, 1)
  w = O.init_weights_np(cfg, 6, dtype="bf16")
  h = np.random.default_rng(6).standard_normal((4, 64)).astype(np.float32)
  final, inter = O.latent_moe_forward(h, w, cfg, dtype="bf16", return_intermediates=True)
  assert (inter["group_sizes"] == 0).any()
  for key in ("latent_projection", "expert_down_output", "routed_output_after_combine",
              "normalized_output", "final_output"):
    assert np.array_equal(O.bf16_round(inter[key]), inter[key]), key


@pytest.mark.parametrize("case", [("standard", 64, 32, 5, 8, 2.0), ("overflow", 64, 32, 5, 8, 0.05),
                                  ("decode_scale", 1, 32, 5, 8, 2.0)])
def test_jittable_matches_eager(case):
  """KR:880-939."""
  name, t, e, start, n_local, cf = case
  cfg = O.LatentMoEConfig(64, 32, 48, e, 2, 1)
  rng = np.random.default_rng(len(name))
  scores = rng.random((t, e)).astype(np.float32)
  topk = O.top_k_desc(scores, 2)
  w = rng.random((t, 2)).astype(np.float32)
  x = rng.standard_normal((t, 32)).astype(np.float32)
  a = _shard(topk, w, x, cfg, start, n_local, cf, tile=128, jittable=True)
  b = _shard(topk, w, x, cfg, start, n_local, cf, tile=128, jittable=False)
  for u, v in zip(a, b):
    assert np.array_equal(u, v)


@pytest.mark.parametrize("seed,t,e,n_local,k", [(0, 96, 32, 8, 4), (1, 40, 16, 4, 2),
                                                (2, 64, 64, 16, 8), (3, 33, 24, 6, 3)])
def test_sharded_sum_matches_unsharded(seed, t, e, n_local, k):
  """KR:1531-1674 and test_sharded_routing_local.py:395-412 (fp32)."""
  cfg = O.LatentMoEConfig(64, 32, 48, e, k, 1)
  w = O.init_weights_np(cfg, seed)
  h = np.random.default_rng(100 + seed).standard_normal((t, 64)).astype(np.float32)
  ref = O.latent_moe_forward(h, w, cfg)
  _, _, _, topk, tw = O.router_gate(h, w.router_weight, w.e_score_correction_bias, k)
  x = O.matmul(h, w.down_proj, "fp32")
  routed = np.zeros((t, cfg.latent_size), np.float32)
  for start in range(0, e, n_local):
    st, gs, valid, counts, idx, pw = O.filter_and_pad_to_shard_jittable(
        topk, tw, x, e, k, start, n_local, 4.0, 1)
    pad = lambda a: np.concatenate([a[start:start + n_local], np.zeros_like(a[:1])])
    out = O.local_shard_expert_ffn(st, pad(w.expert_gate), pad(w.expert_up), pad(w.expert_down),
                                   gs, 4.0, 25.0, "fp32")
    routed = O.combine_shard_contribution(routed, out, idx, pw, "fp32")
  normed = O.rms_norm(routed, w.norm_scale, cfg.rms_norm_eps, "fp32")
  final = O.matmul(normed, w.up_proj, "fp32") + O.situ_glu_mlp(
      h, w.shared_gate, w.shared_up, w.shared_down, 4.0, 25.0, "fp32")
  assert np.abs(final - ref).max() < 1e-4
