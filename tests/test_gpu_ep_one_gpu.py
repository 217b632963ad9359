"""The NVLink peer-memory exchange (csrc/ep_peer.cu) checked on ONE GPU.

1. Emulated ranks.  W ranks' exchange buffers all live on this GPU and every
   rank's calls run in one stream, rank after rank.  The exchange kernels
   only wait for signals that other ranks would raise; here each buffer's
   signal words are set to the forward's epoch beforehand, and the calls are
   ordered so that every row a rank reads is already in place when it reads
   it (all counts exchanges, then all row puts, then all expert GEMMs, then
   all returns, then all combines).  No kernel ever waits for a later one.
   The per-rank outputs must equal the single-GPU forward of all tokens bit
   for bit -- the same bar as the multi-GPU test -- over two forwards through
   the same buffers (epoch reuse), with the separate return copy and with the
   fused return (the MXFP4 down GEMM storing rows into the source buffers).
2. Bounded waits.  A rank whose peer never signals: the counts exchange, the
   row put and the return put each give up after the configured limit, record
   LMOE_WAIT_TIMEOUT, leave empty offset tables (so nothing downstream
   writes), and the context stays usable.

Reference: the sharded forward is summed over simulated shards in
05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:1531-1674."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lm():
  import tokamax_tpu_kernel_lab_b200 as lm
  lm.load_native()
  return lm


class EmulatedRank:
  """One rank's exchange geometry over buffers that all live on this GPU."""

  def __init__(self, lm, cfg, rank, world, t_local, bufs):
    from tokamax_tpu_kernel_lab_b200 import _native
    self.native = _native
    self.rank, self.world = rank, world
    self.E = cfg.num_experts
    self.n_local = self.E // world
    self.row_bytes = cfg.latent_size * 2
    self.back_cap = t_local * cfg.top_k
    self.recv_cap = self.back_cap * world
    self.bufs = bufs
    self.peers_dev = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    lib = _native.load()
    geo = (world, self.E, self.recv_cap, self.back_cap, self.row_bytes)
    self.recv_off = int(lib.lmoe_ep_region_offset(*geo, 0))
    self.back_off = int(lib.lmoe_ep_region_offset(*geo, 1))
    self.counts_off = int(lib.lmoe_ep_region_offset(*geo, 2))
    # offset tables follow the counts matrix, 256-byte aligned
    self.tables_off = (self.counts_off + world * self.E * 4 + 255) // 256 * 256
    self.local_gs = torch.zeros(self.n_local, dtype=torch.int32, device="cuda")
    self.row_dest = torch.zeros(self.recv_cap, dtype=torch.int64, device="cuda")

  def geo(self):
    return (self.peers_dev.data_ptr(), self.rank, self.world, self.E, self.recv_cap,
            self.back_cap, self.row_bytes)

  def counts(self, buf):
    return buf[self.counts_off:self.counts_off + self.world * self.E * 4].view(torch.int32).view(
        self.world, self.E)

  def tables(self):
    own = self.bufs[self.rank]
    return own[self.tables_off:self.tables_off + (4 * self.E + 2) * 4].view(torch.int32)

  def recv(self, dtype):
    own = self.bufs[self.rank]
    return own[self.recv_off:self.recv_off + self.recv_cap * self.row_bytes].view(dtype).view(
        self.recv_cap, -1)

  def back(self, rows, dtype):
    own = self.bufs[self.rank]
    return own[self.back_off:self.back_off + rows * self.row_bytes].view(dtype).view(rows, -1)


def buffer_bytes(lm, cfg, world, t_local):
  from tokamax_tpu_kernel_lab_b200 import _native
  back = t_local * cfg.top_k
  return int(_native.load().lmoe_ep_buffer_bytes(world, cfg.num_experts, back * world, back,
                                                 cfg.latent_size * 2))


def preset_signals(ranks, group_sizes, epoch):
  """What the other ranks would have published by the time each rank waits:
  every source's per-expert counts in every buffer's counts matrix, and every
  source's counts / rows / returns signal set to `epoch` (the signal words
  are the first 3 * world u32 of each buffer)."""
  world = len(ranks)
  for b in ranks[0].bufs:
    cnt = ranks[0].counts(b)
    for s in range(world):
      cnt[s].copy_(group_sizes[s])
    b[:12 * world].view(torch.int32).fill_(epoch)


def emulated_forward(lm, ranks, backends, hs, cfg, epoch, fused_return):
  from tokamax_tpu_kernel_lab_b200 import ops
  world = len(ranks)
  status = ops._ptr(ops.device_status())
  stream = ops._stream()
  st = []
  for r in range(world):
    be = backends[r]
    idx, w = be.route(hs[r])
    x = be.down(hs[r])
    token_idx, slot_pos, gs = be.dispatch(idx, w)
    st.append((idx, w, x, token_idx, slot_pos, gs))
  preset_signals(ranks, [s[5] for s in st], epoch)
  for r in range(world):
    ranks[r].native.call("lmoe_ep_exchange_counts", *ranks[r].geo(), st[r][5].data_ptr(),
                         ranks[r].local_gs.data_ptr(), status, stream)
  for r in range(world):
    x, token_idx = st[r][2], st[r][3]
    ranks[r].native.call("lmoe_ep_dispatch_put", *ranks[r].geo(), x.data_ptr(), x.shape[0],
                         token_idx.data_ptr(), token_idx.shape[0], status, stream)
  dt = st[0][2].dtype
  if fused_return:
    for r in range(world):
      rk = ranks[r]
      rk.native.call("lmoe_ep_return_destinations", *rk.geo(), rk.row_dest.data_ptr(),
                     rk.recv_cap, status, stream)
      backends[r].experts_received_scatter(rk.recv(dt), rk.local_gs, rk.row_dest)
    for r in range(world):
      ranks[r].native.call("lmoe_ep_return_signal", *ranks[r].geo(), status, stream)
  else:
    ys = [backends[r].experts_received(ranks[r].recv(dt), ranks[r].local_gs)
          for r in range(world)]
    for r in range(world):
      ranks[r].native.call("lmoe_ep_return_put", *ranks[r].geo(), ys[r].data_ptr(),
                           ys[r].shape[0], status, stream)
  outs = []
  for r in range(world):
    idx, w, x, token_idx, slot_pos, gs = st[r]
    back = ranks[r].back(token_idx.shape[0], torch.bfloat16)
    normed = backends[r].combine(back, slot_pos, w)
    outs.append(backends[r].tail(normed, hs[r]))
  return torch.cat(outs)


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("fused_return,mode", [(False, "f16"), (True, "f16"), (False, "split")])
def test_peer_exchange_emulated_ranks_bit_exact(lm, world, fused_return, mode):
  """Both expert forms: the weights-major f16-operand kernels (with and
  without the fused return) and the block-scaled kernels on split rows, each
  bit-exact against the one-GPU forward in the same mode (its dense
  projections as separate GEMMs, as the expert-parallel path runs them)."""
  from tokamax_tpu_kernel_lab_b200.expert_parallel import GpuBackend, shard_experts
  cfg = lm.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  pw = lm.init_prepared_mxfp4(cfg, seed=23, bias_std=0.5)
  gen = torch.Generator(device="cuda").manual_seed(23)
  t = 512
  t_local = t // world
  nbytes = buffer_bytes(lm, cfg, world, t_local)
  bufs = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(world)]
  ranks = [EmulatedRank(lm, cfg, r, world, t_local, bufs) for r in range(world)]
  backends = [GpuBackend(shard_experts(pw, r, world), cfg, mxfp4_operand=mode)
              for r in range(world)]
  for epoch in (1, 2):
    h = torch.randn(t, cfg.hidden_size, generator=gen, device="cuda").to(torch.bfloat16)
    ref = lm.latent_moe_forward(h, pw, cfg, mxfp4_operand=mode, dense_phases=False)
    hs = [h[r * t_local:(r + 1) * t_local].contiguous() for r in range(world)]
    out = emulated_forward(lm, ranks, backends, hs, cfg, epoch, fused_return)
    torch.cuda.synchronize()
    lm.check_device_status()
    assert torch.equal(out, ref), f"epoch {epoch}: {(out != ref).sum().item()} elements differ"
    # every buffer's epoch word advanced once per forward
    for b in bufs:
      done = b[((3 * world * 4 + 255) // 256) * 256:][:12].view(torch.int32)
      assert int(done[2]) == epoch


def test_peer_waits_time_out_and_leave_empty_tables(lm):
  """World 2 on one GPU, rank 0 only: 'rank 1' (a second local buffer) never
  signals, so each wait runs out after the configured 20 ms."""
  from tokamax_tpu_kernel_lab_b200 import _native, ops
  cfg = lm.LatentMoEConfig(1024, 512, 256, 64, 8, 2)
  world, t_local = 2, 64
  nbytes = buffer_bytes(lm, cfg, world, t_local)
  bufs = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(world)]
  rk = EmulatedRank(lm, cfg, 0, world, t_local, bufs)
  lib = _native.load()
  default = int(lib.lmoe_peer_wait_timeout_ns())
  status_t = ops.device_status()
  status_t.zero_()
  status, stream = status_t.data_ptr(), ops._stream()
  gs = torch.full((cfg.num_experts,), 8, dtype=torch.int32, device="cuda")  # 512 rows
  token_idx = torch.arange(t_local * cfg.top_k, dtype=torch.int32, device="cuda") % t_local
  x = torch.randn(t_local, cfg.latent_size, device="cuda").to(torch.bfloat16)
  y = torch.randn(t_local * cfg.top_k, cfg.latent_size, device="cuda").to(torch.bfloat16)
  rk.local_gs.fill_(-1)
  rk.tables().fill_(12345)  # stale tables: the timed-out exchange must empty them
  recv_before = rk.recv(torch.bfloat16).clone()
  try:
    assert _native.call("lmoe_set_peer_wait_timeout_ns", 20_000_000) == 0
    assert int(lib.lmoe_peer_wait_timeout_ns()) == 20_000_000
    _native.call("lmoe_ep_exchange_counts", *rk.geo(), gs.data_ptr(), rk.local_gs.data_ptr(),
                 status, stream)
    torch.cuda.synchronize()
    assert int(status_t.item()) == _native.LMOE_WAIT_TIMEOUT
    assert int(rk.local_gs.abs().sum()) == 0
    tables = rk.tables()
    E = cfg.num_experts
    assert int(tables[E + E]) == 0          # cum[E]: nothing to send
    assert int(tables[2 * E + 1 + E]) == 0  # exp_off[El * W]: nothing received
    # the puts then move nothing, and their own waits run out the same way
    status_t.zero_()
    _native.call("lmoe_ep_dispatch_put", *rk.geo(), x.data_ptr(), x.shape[0],
                 token_idx.data_ptr(), token_idx.shape[0], status, stream)
    torch.cuda.synchronize()
    assert int(status_t.item()) == _native.LMOE_WAIT_TIMEOUT
    assert torch.equal(rk.recv(torch.bfloat16), recv_before)
    status_t.zero_()
    _native.call("lmoe_ep_return_put", *rk.geo(), y.data_ptr(), y.shape[0], status, stream)
    torch.cuda.synchronize()
    assert int(status_t.item()) == _native.LMOE_WAIT_TIMEOUT
    assert bool((rk.back(y.shape[0], torch.bfloat16) == 0).all())
  finally:
    _native.call("lmoe_set_peer_wait_timeout_ns", 0)
    status_t.zero_()
  assert int(lib.lmoe_peer_wait_timeout_ns()) == default
  # the context is still usable
  a = torch.randn(256, 256, device="cuda").to(torch.bfloat16)
  w = torch.randn(256, 256, device="cuda").to(torch.bfloat16)
  out = lm.gemm(a, w)
  torch.cuda.synchronize()
  ref = (a.float() @ w.float().T)
  assert float((out.float() - ref).abs().max()) < 0.1 * float(ref.abs().max())
