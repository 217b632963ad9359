"""Expert-parallel orchestration on CPU `gloo` ranks (world size 2 and 4).

`ep_forward` (counts all-to-all, uneven payload all-to-all, expert-major
reordering, reverse all-to-all, slot-order combine) runs unchanged; the
oracle stands in for the GPU kernels through the `Backend` interface.  The
gathered multi-rank output must equal the single-process oracle forward of
all tokens -- bit for bit, since every row meets the same expert weights and
the combine runs in slot order.  Also: a rank that raises before the
exchange makes its peers fail fast (short process-group timeout) instead of
hanging."""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import lmoe_oracle as O


def _free_port() -> int:
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    return s.getsockname()[1]


class OracleBackend:
  """The Backend interface of expert_parallel.py on the CPU oracle."""

  def __init__(self, w: O.Weights, cfg: O.LatentMoEConfig, dtype: str, rank: int, world: int):
    self.w, self.cfg, self.dtype = w, cfg, dtype
    n = cfg.num_experts // world
    self.e0, self.e1 = rank * n, (rank + 1) * n

  def route(self, h):
    c = self.cfg
    _, _, _, idx, wt = O.router_gate(h.numpy(), self.w.router_weight,
                                     self.w.e_score_correction_bias, c.top_k)
    return torch.from_numpy(idx), torch.from_numpy(wt)

  def down(self, h):
    return torch.from_numpy(O.matmul(h.numpy(), self.w.down_proj, self.dtype))

  def dispatch(self, idx, w):
    order, sorted_tok, gs = O.dispatch_full(idx.numpy(), self.cfg.num_experts)
    slot_pos = np.empty_like(order)
    slot_pos[order] = np.arange(order.size, dtype=np.int32)
    return torch.from_numpy(sorted_tok), torch.from_numpy(slot_pos), torch.from_numpy(gs)

  def gather(self, x, index):
    idx = index.numpy().astype(np.int64)
    out = np.zeros((idx.size, x.shape[1]), np.float32)
    ok = idx >= 0
    out[ok] = x.numpy()[idx[ok]]
    return torch.from_numpy(out)

  def gather_send(self, x, index):
    return self.gather(x, index)

  def reorder(self, recv_counts, world, n_local, rows):
    cnt = recv_counts.numpy().reshape(world, n_local)
    src_off = np.concatenate([[0], np.cumsum(cnt.reshape(-1))])[:-1].reshape(world, n_local)
    em = np.empty(rows, np.int32)
    p = 0
    for e in range(n_local):
      for s in range(world):
        c = cnt[s, e]
        em[p:p + c] = src_off[s, e] + np.arange(c)
        p += c
    sm = np.empty(rows, np.int32)
    sm[em] = np.arange(rows, dtype=np.int32)
    return torch.from_numpy(em), torch.from_numpy(sm), torch.from_numpy(cnt.sum(0).astype(np.int32))

  def experts_indexed(self, src, index, gs_local):
    return self.experts(self.gather(src, index), gs_local)

  def experts(self, xe, gs_local):
    c, w = self.cfg, self.w
    sl = slice(self.e0, self.e1)
    out = O.local_shard_expert_ffn(xe.numpy(), w.expert_gate[sl], w.expert_up[sl],
                                   w.expert_down[sl], gs_local.numpy(), c.activation_situ_beta,
                                   c.activation_situ_linear_beta, self.dtype)
    return torch.from_numpy(out)

  def combine(self, back, slot_pos, w):
    t, k = w.shape
    rows = back.numpy()[slot_pos.numpy()].reshape(t, k, -1)
    routed = np.zeros((t, rows.shape[-1]), np.float32)
    for s in range(k):
      routed += rows[:, s, :] * w.numpy()[:, s:s + 1]
    routed = O.to_dtype(routed, self.dtype)
    return torch.from_numpy(O.rms_norm(routed, self.w.norm_scale, self.cfg.rms_norm_eps,
                                       self.dtype))

  def tail(self, normed, h):
    c, w = self.cfg, self.w
    upo = O.matmul(normed.numpy(), w.up_proj, self.dtype)
    shared = O.situ_glu_mlp(h.numpy(), w.shared_gate, w.shared_up, w.shared_down,
                            c.activation_situ_beta, c.activation_situ_linear_beta, self.dtype)
    return torch.from_numpy(O.to_dtype(upo + shared, self.dtype))


def _problem(dtype):
  cfg = O.LatentMoEConfig(64, 32, 48, 16, 4, 1)
  w = O.init_weights_np(cfg, 11, dtype=dtype, bias_std=0.5)
  h = O.to_dtype(np.random.default_rng(11).standard_normal((48, 64), dtype=np.float32), dtype)
  return cfg, w, h


def _worker(rank, world, port, dtype, results):
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world,
                          timeout=datetime.timedelta(seconds=30))
  from tokamax_tpu_kernel_lab_b200.expert_parallel import EPStats, ep_forward
  cfg, w, h = _problem(dtype)
  t = h.shape[0] // world
  backend = OracleBackend(w, cfg, dtype, rank, world)
  stats = EPStats([], [])
  out = ep_forward(torch.from_numpy(h[rank * t:(rank + 1) * t]), backend, cfg, stats=stats)
  results[rank] = (out.numpy(), stats.send_rows, stats.recv_rows)
  dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_ep_forward_matches_single_process(world, dtype):
  mgr = mp.get_context("spawn").Manager()
  results = mgr.dict()
  mp.spawn(_worker, args=(world, _free_port(), dtype, results), nprocs=world, join=True)
  cfg, w, h = _problem(dtype)
  ref = O.latent_moe_forward(h, w, cfg, dtype=dtype)
  got = np.concatenate([results[r][0] for r in range(world)])
  assert np.array_equal(got, ref)
  # every (token, slot) row crosses exactly once each way
  sent = sum(sum(results[r][1]) for r in range(world))
  recv = sum(sum(results[r][2]) for r in range(world))
  assert sent == recv == h.shape[0] * cfg.top_k


def _failing_worker(rank, world, port, results):
  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  dist.init_process_group("gloo", rank=rank, world_size=world,
                          timeout=datetime.timedelta(seconds=5))
  from tokamax_tpu_kernel_lab_b200.expert_parallel import ep_forward
  cfg, w, h = _problem("fp32")
  t = h.shape[0] // world
  backend = OracleBackend(w, cfg, "fp32", rank, world)
  if rank == 1:
    results[rank] = "raised"
    raise SystemExit(0)  # this rank leaves before the exchange
  try:
    ep_forward(torch.from_numpy(h[rank * t:(rank + 1) * t]), backend, cfg)
    results[rank] = "completed"
  except Exception as e:  # the collective must end with an error, not hang
    results[rank] = f"error: {type(e).__name__}"


def test_peer_failure_ends_collective_with_error():
  mgr = mp.get_context("spawn").Manager()
  results = mgr.dict()
  ctx = mp.get_context("spawn")
  port = _free_port()
  procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, results)) for r in range(2)]
  for p in procs:
    p.start()
  for p in procs:
    p.join(timeout=60)
  for p in procs:
    if p.is_alive():
      p.kill()
      pytest.fail("a rank hung after its peer left")
  assert results[1] == "raised"
  assert results[0].startswith("error")
