"""Expert parallelism on real GPUs, with the exchange over NCCL all-to-all
and over NVLink peer memory (device-side puts): the concatenated per-rank
outputs must equal the single-GPU forward of all tokens bit for bit.  The
peer form runs several forwards through one exchange buffer (epoch reuse).
Needs at least 2 GPUs; skipped otherwise."""

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    return s.getsockname()[1]


def _cfg(lm):
  return lm.LatentMoEConfig(1024, 512, 256, 64, 8, 2)


def _worker(rank, world, port, results, mode="nccl"):
  import torch.distributed as dist

  import tokamax_tpu_kernel_lab_b200 as lm
  from tokamax_tpu_kernel_lab_b200.expert_parallel import (EPStats, GpuBackend, PeerExchange,
                                                           ep_forward, ep_forward_peer)

  os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
  torch.cuda.set_device(rank)
  dev = torch.device("cuda", rank)
  dist.init_process_group("nccl", rank=rank, world_size=world,
                          timeout=datetime.timedelta(seconds=60), device_id=dev)
  try:
    cfg = _cfg(lm)
    n_local = cfg.num_experts // world
    pw = lm.init_prepared_mxfp4(cfg, seed=21, device=dev, bias_std=0.5,
                                expert_start=rank * n_local, num_local_experts=n_local)
    gen = torch.Generator(device=dev).manual_seed(21)
    h = torch.randn(512, cfg.hidden_size, generator=gen, device=dev).to(torch.bfloat16)
    t = h.shape[0] // world
    if mode == "peer":
      hs = [h] + [torch.randn(512, cfg.hidden_size, generator=gen, device=dev).to(torch.bfloat16)
                  for _ in range(2)]
      backend = GpuBackend(pw, cfg)
      xchg = PeerExchange(cfg, t)
      try:
        outs = [ep_forward_peer(x[rank * t:(rank + 1) * t].contiguous(), backend, cfg, xchg)
                for x in hs]
        # the same exchange captured as a CUDA graph, replayed on new inputs
        static_h = hs[0][rank * t:(rank + 1) * t].clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
          ep_forward_peer(static_h, backend, cfg, xchg, fused_return=True)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):  # the fused-return form, captured
          g_out = ep_forward_peer(static_h, backend, cfg, xchg, fused_return=True)
        replays = []
        for x in hs[:2]:
          static_h.copy_(x[rank * t:(rank + 1) * t])
          graph.replay()
          replays.append(g_out.clone())
        torch.cuda.synchronize()
        lm.check_device_status()
        del graph
        # the routed experts on the block-scaled tensor core (split rows)
        split = GpuBackend(pw, cfg, mxfp4_operand="split")
        outs_split = [ep_forward_peer(x[rank * t:(rank + 1) * t].contiguous(), split, cfg, xchg)
                      for x in hs[:2]]
        torch.cuda.synchronize()
        lm.check_device_status()
      finally:
        xchg.close()
      results[rank] = ([o.cpu() for o in outs] + [o.cpu() for o in replays] +
                       [o.cpu() for o in outs_split])
      if rank == 0:
        full = lm.init_prepared_mxfp4(cfg, seed=21, device=dev, bias_std=0.5)
        results["ref"] = [lm.latent_moe_forward(x, full, cfg, mxfp4_operand="f16").cpu()
                          for x in hs]
        results["ref_split"] = [lm.latent_moe_forward(x, full, cfg, mxfp4_operand="split",
                                                      dense_phases=False).cpu() for x in hs[:2]]
      dist.barrier()
      return
    stats = EPStats([], [])
    out = ep_forward(h[rank * t:(rank + 1) * t].contiguous(), GpuBackend(pw, cfg), cfg,
                     stats=stats)
    torch.cuda.synchronize()
    lm.check_device_status()
    results[rank] = (out.cpu(), stats.send_rows, stats.recv_rows)
    if rank == 0:
      full = lm.init_prepared_mxfp4(cfg, seed=21, device=dev, bias_std=0.5)
      results["ref"] = lm.latent_moe_forward(h, full, cfg, mxfp4_operand="f16").cpu()
    dist.barrier()
  finally:
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_forward_bit_exact_vs_single_gpu(world):
  if torch.cuda.device_count() < world:
    pytest.skip(f"needs {world} GPUs")
  import torch.multiprocessing as mp
  mgr = mp.get_context("spawn").Manager()
  results = mgr.dict()
  mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
  got = torch.cat([results[r][0] for r in range(world)])
  assert torch.equal(got, results["ref"])
  assert sum(sum(results[r][1]) for r in range(world)) == 512 * 8


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_forward_peer_bit_exact_vs_single_gpu(world):
  if torch.cuda.device_count() < world:
    pytest.skip(f"needs {world} GPUs")
  import torch.multiprocessing as mp
  mgr = mp.get_context("spawn").Manager()
  results = mgr.dict()
  mp.spawn(_worker, args=(world, _free_port(), results, "peer"), nprocs=world, join=True)
  # eager x3, graph replays x2 (fused return), then the split-row experts x2
  refs = list(results["ref"]) + list(results["ref"])[:2] + list(results["ref_split"])
  for i, ref in enumerate(refs):
    got = torch.cat([results[r][i] for r in range(world)])
    assert torch.equal(got, ref), f"forward {i}"
