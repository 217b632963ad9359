"""Expert-parallel LatentMoE forward over N GPUs (one process per GPU, NCCL).

The reference only simulates expert shards, summing per-shard contributions
in one process (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:1531-1674,
kimi_k3_latent_moe_ragged_dot.py:1035-1137).  Here the shards are real ranks:

  rank r holds experts [r*E/n, (r+1)*E/n) and T/n tokens; dense weights
  (router, down/up projections, shared expert) are replicated.
  1 route + down-project local tokens; dispatch = stable sort of the
    (token, slot) entries by global expert id, which also groups them by
    destination rank (experts are contiguous per rank)
  2 counts all-to-all: per-(destination, local expert) row counts, int32
  3 payload all-to-all of latent rows (L bf16 each: the dispatch happens after
    the down-projection, so rows are latent-width)
  4 receive side: reorder (source, expert) blocks to expert-major, grouped
    gate/up + SiTU-GLU, grouped down GEMM, reorder back
  5 reverse all-to-all of the outputs
  6 combine in f32, slot order, + RMSNorm, up-projection, shared expert

Every row meets the same weights and the same K-reduction as on one GPU and
the combine order is the slot order, so the n-rank output equals the 1-rank
output bit for bit (dropless dispatch).

`ep_forward` runs the exchange on NCCL (all_to_all_single, one host read of
the counts per forward); `ep_forward_peer` runs it as device kernels that
store rows straight into the peer GPUs' buffers over NVLink (CUDA IPC
mappings), with the counts exchanged in peer memory too: no host
synchronisation inside the forward, and rows land expert-major in the
receiver's buffer, so the expert GEMMs read them in place.

The orchestration is written against a small kernel interface
(`Backend`) so the exchange logic can be exercised on CPU `gloo` ranks with
the oracle standing in for the kernels; production uses `GpuBackend`.
"""

from __future__ import annotations

import ctypes
import dataclasses

import numpy as np
import torch
import torch.distributed as dist

from . import _native, ops
from .latent_moe import (LatentMoEConfig, PreparedWeights, _dense, blockscaled_experts,
                         mxfp4_f16_path)


class GpuBackend:
  """The sm_100a kernels.  mxfp4_operand (MXFP4 experts): "f16" runs the
  routed experts on the weights-major kernels with f16 operands (bf16 when
  the weight scales do not allow f16), "split" on the block-scaled tensor
  core with the rows split into two e4m3 planes -- the same results as
  latent_moe_forward with that mode.  The fused return
  (ep_forward_peer(..., fused_return=True)) runs the weights-major kernels."""

  def __init__(self, pw: PreparedWeights, cfg: LatentMoEConfig, mxfp4_operand: str = "f16"):
    if mxfp4_operand not in ("f16", "split"):
      raise ValueError(f"mxfp4_operand={mxfp4_operand!r}: 'f16' or 'split'")
    self.pw, self.cfg = pw, cfg
    self.split = mxfp4_operand == "split" and pw.expert_gu_mx is not None
    if self.split:
      blockscaled_experts(pw)  # the one-time repack, outside any graph capture

  def route(self, h):
    c = self.cfg
    return ops.router_gate(h, self.pw.router, self.pw.bias, c.top_k,
                           renormalize=c.moe_renormalize,
                           routed_scaling_factor=c.routed_scaling_factor)

  def down(self, h):
    # f16 latent rows when the MXFP4 f16-operand kernels consume them
    f16 = not self.split and mxfp4_f16_path(self.pw)
    return _dense(h, self.pw.down, out_dtype=torch.float16 if f16 else None)

  def _split_experts(self, rows_in, gs_local, out_rows: int, zero_tail: bool):
    """Expert FFN on the block-scaled tensor core of rows already in expert
    order: the split quantisation into the padded layout, gate/up + SiTU-GLU
    writing the down GEMM's split rows, the down GEMM writing the unpadded
    (ragged_dot) layout."""
    c = self.cfg
    gu, dn = blockscaled_experts(self.pw)
    rows = ops.quantize_split_rows(rows_in, gs_local)
    act_q = ops.blockscaled_gateup_situ_quantized(rows, gu, "e4m3x2", beta=c.activation_situ_beta,
                                                  linear_beta=c.activation_situ_linear_beta,
                                                  round_gate_up=True)
    return ops.mxfp8_mxfp4_ragged_dot(act_q, dn, unpadded_rows=out_rows, zero_tail=zero_tail)

  def dispatch(self, idx, w):
    d = ops.dispatch(idx, w, self.cfg.num_experts, want_order=False)
    return d.token_idx, d.slot_pos, d.group_sizes

  def gather(self, x, index):
    return ops.gather_rows(x, index)

  def gather_send(self, x, index):
    """Rows to send, in destination-rank-major expert order."""
    return ops.gather_rows(x, index)

  def reorder(self, recv_counts, world, n_local, rows):
    dev = recv_counts.device
    em = torch.empty(max(rows, 1), dtype=torch.int32, device=dev)
    sm = torch.empty(max(rows, 1), dtype=torch.int32, device=dev)
    gs = torch.empty(n_local, dtype=torch.int32, device=dev)
    from . import _native
    _native.call("lmoe_ep_reorder", recv_counts.data_ptr(), world, n_local, rows, em.data_ptr(),
                 sm.data_ptr(), gs.data_ptr(), ops._stream())
    return em[:rows], sm[:rows], gs

  def experts_indexed(self, src, index, gs_local):
    """Expert FFN of rows src[index[p]] in expert-major order."""
    c, pw = self.cfg, self.pw
    b, lb = c.activation_situ_beta, c.activation_situ_linear_beta
    xe = ops.gather_rows(src, index)
    if self.split:
      return self._split_experts(xe, gs_local, xe.shape[0], True)
    if pw.expert_gu_mx is not None:
      act = ops.mxfp4_fused_gateup_situ(xe, pw.expert_gu_mx, gs_local, beta=b, linear_beta=lb,
                                        out_dtype=xe.dtype)
      return ops.mxfp4_ragged_dot(act, pw.expert_down_mx, gs_local)
    act = ops.fused_gateup_situ(xe, pw.expert_gu, gs_local, beta=b, linear_beta=lb,
                                rhs_layout="gnk")
    return ops.ragged_dot(act, pw.expert_down, gs_local, rhs_layout="gnk")

  def experts_received(self, recv, gs_local):
    """Expert FFN of rows already in expert-major order (the peer exchange's
    receive buffer, sized by capacity: rows past sum(gs_local) are neither
    read nor written)."""
    c, pw = self.cfg, self.pw
    b, lb = c.activation_situ_beta, c.activation_situ_linear_beta
    if self.split:
      return self._split_experts(recv, gs_local, recv.shape[0], False)
    if pw.expert_gu_mx is not None:
      act = ops.mxfp4_fused_gateup_situ(recv, pw.expert_gu_mx, gs_local, beta=b, linear_beta=lb,
                                        out_dtype=recv.dtype, zero_tail=False)
      return ops.mxfp4_ragged_dot(act, pw.expert_down_mx, gs_local, zero_tail=False)
    act = ops.fused_gateup_situ(recv, pw.expert_gu, gs_local, beta=b, linear_beta=lb,
                                rhs_layout="gnk", zero_tail=False)
    return ops.ragged_dot(act, pw.expert_down, gs_local, rhs_layout="gnk", zero_tail=False)

  def experts_received_scatter(self, recv, gs_local, row_dest):
    """experts_received with the down projection storing each result row at
    row_dest[q] -- the exchange buffer of the rank row q came from -- instead
    of returning it (MXFP4 experts only)."""
    c, pw = self.cfg, self.pw
    act = ops.mxfp4_fused_gateup_situ(recv, pw.expert_gu_mx, gs_local,
                                      beta=c.activation_situ_beta,
                                      linear_beta=c.activation_situ_linear_beta,
                                      out_dtype=recv.dtype, zero_tail=False)
    ops.mxfp4_ragged_dot_scatter(act, pw.expert_down_mx, gs_local, row_dest)

  def combine(self, back, slot_pos, w):
    return ops.combine_rmsnorm(back, slot_pos, w, self.pw.norm_scale, self.cfg.rms_norm_eps)

  def tail(self, normed, h):
    c, pw = self.cfg, self.pw
    upo = _dense(normed, pw.up)
    shared = ops.fused_gateup_situ(h, pw.shared_gu, None, beta=c.activation_situ_beta,
                                   linear_beta=c.activation_situ_linear_beta, rhs_layout="gnk")
    return _dense(shared, pw.shared_down, addend=upo)

  def shared_expert_buffers(self, h):
    """(activation, output) buffers of shared_expert for tokens h."""
    si = self.pw.shared_gu.shape[0] // 2
    return (torch.empty(h.shape[0], si, dtype=torch.bfloat16, device=h.device),
            torch.empty(h.shape[0], self.pw.shared_down.shape[0], dtype=torch.bfloat16,
                        device=h.device))

  def shared_expert(self, h, out=None):
    """The shared-expert MLP alone (it depends only on h): bf16(situ-glu(h) @ W_sd),
    into `out` = shared_expert_buffers(h) when given."""
    c, pw = self.cfg, self.pw
    act, res = out if out is not None else (None, None)
    shared = ops.fused_gateup_situ(h, pw.shared_gu, None, beta=c.activation_situ_beta,
                                   linear_beta=c.activation_situ_linear_beta, rhs_layout="gnk",
                                   out=act)
    return ops.gemm(shared, pw.shared_down, rhs_layout="nk", out=res)

  def tail_with_shared(self, normed, shared_out):
    """bf16(bf16(normed @ W_up) + shared_out): the same bits as tail() (the
    output sum of KR:435 is one bf16 add of two bf16 terms)."""
    return _dense(normed, self.pw.up, addend=shared_out)


@dataclasses.dataclass
class EPStats:
  send_rows: list
  recv_rows: list


def ep_forward(h: torch.Tensor, backend, cfg: LatentMoEConfig, group=None,
               stats: EPStats | None = None) -> torch.Tensor:
  """Expert-parallel forward of this rank's tokens `h` (T_local, d)."""
  world = dist.get_world_size(group)
  E = cfg.num_experts
  if E % world:
    raise ValueError(f"num_experts {E} is not divisible by world size {world}")
  n_local = E // world
  L = cfg.latent_size
  idx, w = backend.route(h)
  x = backend.down(h)
  token_idx, slot_pos, group_sizes = backend.dispatch(idx, w)
  send = backend.gather_send(x, token_idx)  # destination-rank-major, expert-sorted
  recv_counts = torch.empty_like(group_sizes)
  dist.all_to_all_single(recv_counts, group_sizes, group=group)
  counts = torch.cat([group_sizes, recv_counts]).cpu().numpy().astype(np.int64)
  send_rows = counts[:E].reshape(world, n_local).sum(1).tolist()
  recv_rows = counts[E:].reshape(world, n_local).sum(1).tolist()
  if stats is not None:
    stats.send_rows, stats.recv_rows = send_rows, recv_rows
  n_recv = int(sum(recv_rows))
  recv = torch.empty(n_recv, L, dtype=send.dtype, device=send.device)
  dist.all_to_all_single(recv, send, output_split_sizes=recv_rows, input_split_sizes=send_rows,
                         group=group)
  em_src, sm_src, gs_local = backend.reorder(recv_counts.view(world, n_local), world, n_local,
                                             n_recv)
  ye = backend.experts_indexed(recv, em_src, gs_local)
  back_send = backend.gather(ye, sm_src)
  back = torch.empty(send.shape[0], L, dtype=ye.dtype, device=ye.device)
  dist.all_to_all_single(back, back_send, output_split_sizes=send_rows,
                         input_split_sizes=recv_rows, group=group)
  normed = backend.combine(back, slot_pos, w)
  return backend.tail(normed, h)


class _RawDevice:
  """A device byte range as a torch tensor (zero-copy, not owned)."""

  def __init__(self, ptr: int, rows: int, row_bytes: int):
    self.__cuda_array_interface__ = {"shape": (rows, row_bytes), "typestr": "|u1",
                                     "data": (ptr, False), "version": 3, "strides": None}


class PeerExchange:
  """Buffers and peer mappings of the peer-memory expert exchange.

  Every rank allocates one buffer (flags, counts, offset tables, a receive
  region of `world * tokens_per_rank * top_k` rows -- the worst case, every
  routed row of every rank landing here -- and a return region of
  `tokens_per_rank * top_k` rows), sends its CUDA IPC handle to every peer
  and maps theirs.  Collective: every rank of `group` constructs it, and
  every rank calls close()."""

  def __init__(self, cfg: LatentMoEConfig, tokens_per_rank: int, group=None):
    self.group = group
    self.world = dist.get_world_size(group)
    self.rank = dist.get_rank(group)
    if cfg.num_experts % self.world:
      raise ValueError(f"num_experts {cfg.num_experts} is not divisible by world {self.world}")
    self.E = cfg.num_experts
    self.n_local = self.E // self.world
    self.row_bytes = cfg.latent_size * 2
    self.back_cap = tokens_per_rank * cfg.top_k
    self.recv_cap = self.back_cap * self.world
    lib = _native.load()
    geo = (self.world, self.E, self.recv_cap, self.back_cap, self.row_bytes)
    self.nbytes = int(lib.lmoe_ep_buffer_bytes(*geo))
    if self.nbytes <= 0:
      raise ValueError("invalid exchange geometry")
    own = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * 64)()
    _native.call("lmoe_ep_buffer_alloc", self.nbytes, ctypes.byref(own), handle)
    self._own = own.value
    handles = [None] * self.world
    dist.all_gather_object(handles, bytes(handle), group=group)
    ptrs, self._opened = [], []
    for r, hb in enumerate(handles):
      if r == self.rank:
        ptrs.append(self._own)
        continue
      peer = ctypes.c_void_p()
      _native.call("lmoe_ep_buffer_open", (ctypes.c_uint8 * 64).from_buffer_copy(hb),
                   ctypes.byref(peer))
      ptrs.append(peer.value)
      self._opened.append(peer.value)
    self.peers_dev = torch.tensor(ptrs, dtype=torch.int64, device="cuda")
    self.local_gs = torch.zeros(self.n_local, dtype=torch.int32, device="cuda")
    # per received row: where its result goes (the fused return)
    self.row_dest = torch.zeros(self.recv_cap, dtype=torch.int64, device="cuda")
    self._recv = torch.as_tensor(
        _RawDevice(self._own + int(lib.lmoe_ep_region_offset(*geo, 0)), self.recv_cap,
                   self.row_bytes), device="cuda")
    self._back = torch.as_tensor(
        _RawDevice(self._own + int(lib.lmoe_ep_region_offset(*geo, 1)), self.back_cap,
                   self.row_bytes), device="cuda")
    dist.barrier(group)  # every buffer is zeroed and mapped before the first signal

  def _geo(self):
    return (self.peers_dev.data_ptr(), self.rank, self.world, self.E, self.recv_cap,
            self.back_cap, self.row_bytes)

  def recv_rows(self, dtype: torch.dtype) -> torch.Tensor:
    return self._recv.view(dtype)

  def back_rows(self, rows: int, dtype: torch.dtype) -> torch.Tensor:
    return self._back[:rows].view(dtype)

  def exchange(self, x: torch.Tensor, token_idx: torch.Tensor, group_sizes: torch.Tensor,
               experts, after_counts=None, experts_scatter=None, mark=None) -> torch.Tensor:
    """Send row x[token_idx[p]] of every dispatched row p to the owner of its
    expert, run `experts(recv, local_group_sizes)` on the rows this rank
    received, send each result back; returns the returned rows in this rank's
    dispatch order (token_idx.shape[0] rows).  `after_counts()` (optional) is
    called once the counts exchange is enqueued, before the row puts -- the
    place to fork work that should overlap the NVLink transfers.  With
    `experts_scatter(recv, local_group_sizes, row_dest)` the experts store each
    result row straight into its source's return region (row_dest[q] is its
    address there), so the return overlaps the down projection instead of
    following it as a copy.  No host
    synchronisation: the exchange epoch lives in the device buffer, so a
    forward that calls this can be captured as a CUDA graph.  `mark(name)`
    (optional) is called on the host after each phase is enqueued ("counts",
    "dispatch put", "experts", "return"), e.g. to record timing events.

    Device-side errors (a bounded wait that ran out, a row past the buffer)
    are recorded in this rank's device status word only; the other ranks see
    empty or stale rows, not an error.  Call ops.check_device_status() on every
    rank at step boundaries (bench.py does after each timed region)."""
    if x.shape[1] * x.element_size() != self.row_bytes:
      raise ValueError("row width does not match the exchange buffer")
    rows = token_idx.shape[0]
    if rows > self.back_cap or group_sizes.shape[0] != self.E:
      raise ValueError("dispatch does not fit the exchange buffer")
    status = ops._ptr(ops.device_status(x.device))
    stream = ops._stream()
    geo = self._geo()
    mark = mark or (lambda name: None)
    _native.call("lmoe_ep_exchange_counts", *geo, group_sizes.data_ptr(),
                 self.local_gs.data_ptr(), status, stream)
    mark("counts")
    if after_counts is not None:
      after_counts()
    _native.call("lmoe_ep_dispatch_put", *geo, x.data_ptr(), x.shape[0],
                 token_idx.data_ptr(), rows, status, stream)
    mark("dispatch put")
    if experts_scatter is not None:
      _native.call("lmoe_ep_return_destinations", *geo, self.row_dest.data_ptr(), self.recv_cap,
                   status, stream)
      experts_scatter(self.recv_rows(x.dtype), self.local_gs, self.row_dest)
      mark("experts")
      _native.call("lmoe_ep_return_signal", *geo, status, stream)
      mark("return")
      return self.back_rows(rows, torch.bfloat16)
    y = experts(self.recv_rows(x.dtype), self.local_gs)
    mark("experts")
    if y.shape[1] * y.element_size() != self.row_bytes or not y.is_contiguous():
      raise ValueError("expert output rows do not match the exchange buffer")
    _native.call("lmoe_ep_return_put", *geo, y.data_ptr(), y.shape[0], status,
                 stream)
    mark("return")
    return self.back_rows(rows, y.dtype)

  def close(self):
    """Collective: unmap the peers' buffers and free this rank's, once every
    rank has finished with the exchange."""
    if self._own is None:
      return
    torch.cuda.synchronize()
    dist.barrier(self.group)
    for p in self._opened:
      _native.call("lmoe_ep_buffer_close", p)
    self._opened = []
    self._recv = self._back = None
    _native.call("lmoe_ep_buffer_free", self._own)
    self._own = None


def ep_forward_peer(h: torch.Tensor, backend, cfg: LatentMoEConfig,
                    xchg: PeerExchange, fused_return: bool = False, mark=None) -> torch.Tensor:
  """Expert-parallel forward of this rank's tokens `h` (T_local, d) with the
  exchange over NVLink peer memory (no host synchronisation).  The shared
  expert depends only on h, so it runs on a side stream forked after the
  counts exchange, filling the SMs while the row puts wait on NVLink; its
  buffers are allocated on the main stream before the fork, and the streams
  join before the output sum.

  fused_return=True (MXFP4 experts): the down-projection GEMM stores each
  result row straight into its source rank's return region over NVLink
  (lmoe_mxfp4_ragged_dot_scatter) instead of a separate return copy.  Same
  bits; slower on B200 at configuration 5 (n = 2: 4.69 vs 3.83 ms per step),
  because the epilogue's scattered peer stores hold up the GEMM's
  accumulator hand-off longer than the separate copy takes.

  `mark(name)` (optional) is called on the host after each phase of the main
  stream is enqueued (route, down-projection, dispatch, the exchange's
  phases, combine, tail), e.g. to record CUDA events for a phase timeline.
  Device-side errors land in this rank's status word only: check it on every
  rank at step boundaries (ops.check_device_status)."""
  mark = mark or (lambda name: None)
  main = torch.cuda.current_stream(h.device)
  side = ops.side_stream(h.device)
  idx, w = backend.route(h)
  mark("route")
  x = backend.down(h)
  mark("down-projection")
  token_idx, slot_pos, group_sizes = backend.dispatch(idx, w)
  mark("dispatch sort")
  bufs = backend.shared_expert_buffers(h)

  def fork_shared():
    side.wait_stream(main)
    with torch.cuda.stream(side):
      backend.shared_expert(h, out=bufs)

  fused = fused_return and backend.pw.expert_gu_mx is not None
  back = xchg.exchange(x, token_idx, group_sizes, backend.experts_received,
                       after_counts=fork_shared,
                       experts_scatter=backend.experts_received_scatter if fused else None,
                       mark=mark)
  normed = backend.combine(back, slot_pos, w)
  mark("combine")
  main.wait_stream(side)
  out = backend.tail_with_shared(normed, bufs[1])
  mark("tail")
  return out


def shard_experts(pw_full: PreparedWeights, rank: int, world: int) -> PreparedWeights:
  """This rank's contiguous expert range of a fully materialised weight set."""
  e = (pw_full.expert_gu_mx.packed.shape[0] if pw_full.expert_gu_mx is not None
       else pw_full.expert_gu.shape[0])
  n = e // world
  sl = slice(rank * n, (rank + 1) * n)
  # the block-scaled repack (if the full set has one) covers every expert:
  # the shard builds its own on first use
  out = dataclasses.replace(pw_full, expert_gu_bs=None, expert_down_bs=None)
  if pw_full.expert_gu_mx is not None:
    out.expert_gu_mx = ops.MXFP4Weights(pw_full.expert_gu_mx.packed[sl].contiguous(),
                                        pw_full.expert_gu_mx.scale[sl].contiguous())
    out.expert_down_mx = ops.MXFP4Weights(pw_full.expert_down_mx.packed[sl].contiguous(),
                                          pw_full.expert_down_mx.scale[sl].contiguous())
  else:
    out.expert_gu = pw_full.expert_gu[sl].contiguous()
    out.expert_down = pw_full.expert_down[sl].contiguous()
  return out
