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

The orchestration is written against a small kernel interface
(`Backend`) so the exchange logic can be exercised on CPU `gloo` ranks with
the oracle standing in for the kernels; production uses `GpuBackend`.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import torch
import torch.distributed as dist

from . import ops
from .latent_moe import LatentMoEConfig, PreparedWeights, _dense, mxfp4_f16_path


class GpuBackend:
  """The sm_100a kernels."""

  def __init__(self, pw: PreparedWeights, cfg: LatentMoEConfig):
    self.pw, self.cfg = pw, cfg

  def route(self, h):
    c = self.cfg
    logits = ops.router_logits(h, self.pw.router)
    return ops.router_topk(logits, self.pw.bias, c.top_k, renormalize=c.moe_renormalize,
                           routed_scaling_factor=c.routed_scaling_factor)

  def down(self, h):
    # f16 latent rows when the MXFP4 f16-operand kernels consume them
    return _dense(h, self.pw.down, out_dtype=torch.float16 if mxfp4_f16_path(self.pw) else None)

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
    if pw.expert_gu_mx is not None:
      act = ops.mxfp4_fused_gateup_situ(xe, pw.expert_gu_mx, gs_local, beta=b, linear_beta=lb,
                                        out_dtype=xe.dtype)
      return ops.mxfp4_ragged_dot(act, pw.expert_down_mx, gs_local)
    act = ops.fused_gateup_situ(xe, pw.expert_gu, gs_local, beta=b, linear_beta=lb,
                                rhs_layout="gnk")
    return ops.ragged_dot(act, pw.expert_down, gs_local, rhs_layout="gnk")

  def combine(self, back, slot_pos, w):
    return ops.combine_rmsnorm(back, slot_pos, w, self.pw.norm_scale, self.cfg.rms_norm_eps)

  def tail(self, normed, h):
    c, pw = self.cfg, self.pw
    upo = _dense(normed, pw.up)
    shared = ops.fused_gateup_situ(h, pw.shared_gu, None, beta=c.activation_situ_beta,
                                   linear_beta=c.activation_situ_linear_beta, rhs_layout="gnk")
    return _dense(shared, pw.shared_down, addend=upo)


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


def shard_experts(pw_full: PreparedWeights, rank: int, world: int) -> PreparedWeights:
  """This rank's contiguous expert range of a fully materialised weight set."""
  e = (pw_full.expert_gu_mx.packed.shape[0] if pw_full.expert_gu_mx is not None
       else pw_full.expert_gu.shape[0])
  n = e // world
  sl = slice(rank * n, (rank + 1) * n)
  out = dataclasses.replace(pw_full)
  if pw_full.expert_gu_mx is not None:
    out.expert_gu_mx = ops.MXFP4Weights(pw_full.expert_gu_mx.packed[sl].contiguous(),
                                        pw_full.expert_gu_mx.scale[sl].contiguous())
    out.expert_down_mx = ops.MXFP4Weights(pw_full.expert_down_mx.packed[sl].contiguous(),
                                          pw_full.expert_down_mx.scale[sl].contiguous())
  else:
    out.expert_gu = pw_full.expert_gu[sl].contiguous()
    out.expert_down = pw_full.expert_down[sl].contiguous()
  return out
