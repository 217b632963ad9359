"""LatentMoE layer throughput on B200 (benchmark configuration 5).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl b200|reference]

Workload: one forward of the full LatentMoE layer -- d_model 7168, latent 2048,
896 MXFP4 routed experts (intermediate 1024, top-16), 2 shared experts, bf16
activations, router bias N(0, 0.5^2) for skewed load -- over T tokens
(default 16384, global).  N > 1 runs expert parallelism under torchrun: rank r
holds experts [r*E/N, (r+1)*E/N) and T/N tokens; dispatch and return are
device-side stores into the peers' buffers over NVLink (`--exchange nccl`: NCCL
all-to-alls instead) (strong scaling: the global token count is fixed).
Synthetic data: seeded N(0,1) hidden states, N(0, 0.02^2) dense weights,
MXFP4 expert codes uniform over the 16 e2m1 values with E8M0 scales
2^U{-8..-6} (rms ~0.02).  The working set (3 GB of expert weights, 0.2 GB of
dense weights) is far above the 126 MB L2, so no flush is needed between steps.

One JSON line (rank 0): `value` = tokens/s of the whole job with inputs
resident in HBM, device-timed with CUDA events (max over ranks); `e2e` = the
same through the public API with every step's input copied from pinned host
memory and its output copied back inside the timed region (the copies of
neighbouring steps overlap the forward, on their own streams); `roofline` for the dominant
kernel (the MXFP4 fused gate/up grouped GEMM); `cpu_baseline` = the CPU
restatement of the reference forward on a token sample; `clocks` sampled
with nvidia-smi during the timed region.

`--impl reference` times the reference's algorithm on the host CPU instead
(the reference is JAX/TPU code; JAX is not installed, so its numpy
restatement runs, with all host threads), same metric and config.
"""

from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "LatentMoE layer tokens/s"
UNIT = "tokens/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# dram bytes (read + write) per launch of the dominant kernel: the ncu capture
# summarised in profiles/mxfp4_swap_gemm_t8192.md measured 746.5 MB read +
# 246.5 MB written at 8192 tokens (131072 routed rows); scaled by the routed
# rows to the 16384-token launch (the weight bytes, about a fifth of it, do
# not grow with the rows, so this overstates by at most ~12%)
DOMINANT_TRAFFIC_BYTES = int((746.5e6 + 246.5e6) * 2)


def parse_args():
  p = argparse.ArgumentParser()
  p.add_argument("--gpus", type=int, default=1)
  p.add_argument("--steps", type=int, default=10)
  p.add_argument("--warmup", type=int, default=3)
  p.add_argument("--tokens", type=int, default=16384)
  p.add_argument("--impl", default="b200", choices=["b200", "reference"])
  p.add_argument("--seed", type=int, default=4)
  p.add_argument("--cpu-sample-tokens", type=int, default=16)
  p.add_argument("--no-cpu-baseline", action="store_true")
  p.add_argument("--no-graph", action="store_true",
                 help="time eager launches instead of a captured CUDA graph")
  p.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                 help="expert-parallel exchange (N>1): NVLink peer-memory puts or NCCL all-to-all")
  return p.parse_args()


def config_dict(args, world):
  return {
      "workload": "full LatentMoE layer (benchmark configuration 5)",
      "num_tokens": args.tokens,
      "tokens_per_gpu": args.tokens // world,
      "d_model": 7168, "latent_dim": 2048, "num_experts": 896, "expert_intermediate": 1024,
      "top_k": 16, "num_shared_experts": 2, "expert_format": "mxfp4 (e2m1 + E8M0/32)",
      "activations": "bf16", "router_bias_std": 0.5,
      "parallelism": f"ep{world}" if world > 1 else "single GPU",
      "exchange": ("nvlink peer-memory puts" if args.exchange == "peer" else
                   "nccl all_to_all_single") if world > 1 else None,
      "l2": "working set (3.2 GB weights) > 126 MB L2; no flush between steps",
      "launch": ("cuda graph replay" if (world == 1 or args.exchange == "peer") and not args.no_graph
                 else "eager"),
  }


def load_peaks():
  path = ROOT / "MEASURED_PEAKS.json"
  if path.exists():
    d = json.loads(path.read_text())
    return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
  return dict(FALLBACK_PEAKS), "fallback"


# --------------------------------------------------------------------------- CPU side


def cpu_weights(seed: int, cfg, touched):
  """Host (numpy) weights of the configuration-5 layer for the CPU runs:
  dense N(0, 0.02^2) rounded to bf16; MXFP4 experts drawn per expert id on
  demand (only the experts the sampled tokens touch are materialised)."""
  from oracle import lmoe_oracle as O
  import numpy as np

  rng = np.random.default_rng(seed)
  d, L, I, E = cfg.hidden_size, cfg.latent_size, cfg.intermediate_size, cfg.num_experts
  si = I * cfg.num_shared_experts
  nrm = lambda *s: O.bf16_round(rng.standard_normal(s, dtype=np.float32) * np.float32(0.02))
  router, down, up = nrm(d, E), nrm(d, L), nrm(L, d)
  bias = rng.standard_normal(E, dtype=np.float32) * np.float32(0.5)
  sg, su, sd = nrm(d, si), nrm(d, si), nrm(si, d)

  class Experts:
    def __init__(self, rows0, rows1, n, k, tag):
      self.rows0, self.rows1, self.n, self.k, self.tag = rows0, rows1, n, k, tag
      self.cache = {}

    @property
    def shape(self):
      return (E, self.k, self.rows1 - self.rows0)

    def __getitem__(self, e):
      e = int(e)
      if e not in self.cache:
        r = np.random.default_rng(seed * 100003 + 2 * e + self.tag)
        packed = r.integers(0, 256, (self.n, self.k // 2), dtype=np.uint8)
        scale = r.integers(119, 122, (self.n, self.k // 32), dtype=np.uint8)
        self.cache[e] = np.ascontiguousarray(
            O.dequantize_mxfp4(packed[self.rows0:self.rows1], scale[self.rows0:self.rows1]).T)
      return self.cache[e]

  w = O.Weights(router_weight=router, e_score_correction_bias=bias, down_proj=down, up_proj=up,
                expert_gate=Experts(0, I, 2 * I, L, 1), expert_up=Experts(I, 2 * I, 2 * I, L, 1),
                expert_down=Experts(0, L, L, I, 2), norm_scale=np.ones(L, np.float32),
                shared_gate=sg, shared_up=su, shared_down=sd)
  del touched
  return w


def cpu_forward_timer(seed: int, sample_tokens: int):
  """Returns (callable running one oracle forward of the sample, description)."""
  from oracle import lmoe_oracle as O
  import numpy as np

  cfg = O.LatentMoEConfig(7168, 2048, 1024, 896, 16, 2)
  w = cpu_weights(seed, cfg, None)
  h = O.bf16_round(np.random.default_rng(seed + 1).standard_normal((sample_tokens, 7168),
                                                                   dtype=np.float32))

  def run():
    return O.latent_moe_forward(h, w, cfg, dtype="bf16")

  run()  # materialise (dequantise) the touched experts outside the timing
  return run, (f"{sample_tokens} tokens of configuration 5 through the numpy restatement of "
               "latent_moe_forward (bf16 emulated, MXFP4 experts dequantised once before "
               "timing, as the reference dequantises its checkpoint)")


def cpu_baseline(seed: int, sample_tokens: int, reps: int = 3) -> dict:
  run, desc = cpu_forward_timer(seed, sample_tokens)
  times = []
  for _ in range(reps):
    t0 = time.perf_counter()
    run()
    times.append(time.perf_counter() - t0)
  t = statistics.median(times)
  return {"value": sample_tokens / t, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
          "sample": desc + f"; median of {reps}"}


def run_reference(args, world, rank):
  if rank != 0:
    return
  run, desc = cpu_forward_timer(args.seed, args.cpu_sample_tokens)
  for _ in range(args.warmup):
    run()
  t0 = time.perf_counter()
  for _ in range(args.steps):
    run()
  dt = time.perf_counter() - t0
  value = args.cpu_sample_tokens * args.steps / dt
  line = {
      "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
      "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
      "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
      "data": "synthetic", "config": config_dict(args, world),
      "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                       "sample": desc + " (JAX is not installed: the reference's own JAX path "
                                        "cannot run; its numpy restatement runs instead)"},
      "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
  }
  print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU side


class ClockSampler:
  """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

  FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
            "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
            "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

  def __init__(self, device_index: int):
    self.device_index = device_index
    self.proc = None
    self.path = None

  def __enter__(self):
    fd, self.path = tempfile.mkstemp(suffix=".csv")
    os.close(fd)
    try:
      self.proc = subprocess.Popen(
          ["nvidia-smi", "-i", str(self.device_index), f"--query-gpu={self.FIELDS}",
           "--format=csv,noheader,nounits", "-lms", "200"],
          stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
    except OSError:
      self.proc = None
    time.sleep(0.3)
    return self

  def __exit__(self, *exc):
    if self.proc is not None:
      self.proc.terminate()
      try:
        self.proc.wait(timeout=5)
      except subprocess.TimeoutExpired:
        self.proc.kill()

  def summary(self):
    if self.path is None or not os.path.exists(self.path):
      return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
    rows = [r.split(",") for r in open(self.path).read().strip().splitlines() if r.strip()]
    os.unlink(self.path)
    sm, smax, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for r in rows:
      try:
        sm.append(float(r[1]))
        smax = float(r[2])
        for nm, v in zip(names, r[5:9]):
          if v.strip().lower() == "active":
            reasons.add(nm)
      except (ValueError, IndexError):
        continue
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
            "reasons": sorted(reasons), "samples": len(sm)}


def main():
  args = parse_args()
  world = int(os.environ.get("WORLD_SIZE", "1"))
  rank = int(os.environ.get("RANK", "0"))
  local_rank = int(os.environ.get("LOCAL_RANK", "0"))
  if args.impl == "reference":
    run_reference(args, world, rank)
    return

  import torch
  import torch.distributed as dist

  import tokamax_tpu_kernel_lab_b200 as lm
  from tokamax_tpu_kernel_lab_b200 import _native, ops
  from tokamax_tpu_kernel_lab_b200.expert_parallel import (GpuBackend, PeerExchange, ep_forward,
                                                           ep_forward_peer)

  torch.cuda.set_device(local_rank)
  dev = torch.device("cuda", local_rank)
  if world > 1:
    import datetime
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
  lm.load_native()
  cfg = lm.full_layer_config()
  E = cfg.num_experts
  n_local = E // world
  t_local = args.tokens // world
  pw = lm.init_prepared_mxfp4(cfg, seed=args.seed, device=dev, bias_std=0.5,
                              expert_start=rank * n_local, num_local_experts=n_local)
  gen = torch.Generator(device=dev).manual_seed(args.seed * 7919 + rank)
  h = torch.randn(t_local, cfg.hidden_size, generator=gen, device=dev).to(torch.bfloat16)
  backend = GpuBackend(pw, cfg)
  xchg = PeerExchange(cfg, t_local) if world > 1 and args.exchange == "peer" else None

  def forward(x):
    if xchg is not None:
      return ep_forward_peer(x, backend, cfg, xchg)
    if world > 1:
      return ep_forward(x, backend, cfg)
    return lm.latent_moe_forward(x, pw, cfg)

  def barrier():
    if world > 1:
      dist.barrier()

  def max_over_ranks(v: float) -> float:
    if world == 1:
      return v
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())

  stream = torch.cuda.current_stream()
  for _ in range(args.warmup):
    forward(h)
  torch.cuda.synchronize()
  ops.check_device_status()

  # The forward is captured once as a CUDA graph and replayed, so the timed
  # steps do not depend on host launch speed (every kernel still runs every
  # step).  The peer-memory exchange is capturable (its epoch lives on the
  # device); the NCCL form reads its counts on the host and runs eagerly.
  graph = None
  launches_per_step = None
  if (world == 1 or xchg is not None) and not args.no_graph:
    graph = torch.cuda.CUDAGraph()
    launches_cap = _native.launch_count
    with torch.cuda.graph(graph):
      out_graph = forward(h)
    launches_per_step = _native.launch_count - launches_cap
    graph.replay()
    torch.cuda.synchronize()
    ops.check_device_status()

  def step():
    if graph is not None:
      graph.replay()
      return out_graph
    return forward(h)

  # ---------------------------------------------------------------- device-timed steps
  barrier()
  torch.cuda.synchronize()
  launches0 = _native.launch_count
  ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  with ClockSampler(local_rank) as clk:
    ev0.record(stream)
    for _ in range(args.steps):
      out = step()
    ev1.record(stream)
    torch.cuda.synchronize()
  barrier()
  ops.check_device_status()
  launches = (launches_per_step if graph is not None else
              (_native.launch_count - launches0) // max(args.steps, 1))
  ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
  value = args.tokens / (ms / 1e3)
  clocks = clk.summary()

  # ---------------------------------------------------------------- end to end (host buffers)
  # Every step copies its tokens from pinned host memory, runs the forward
  # through the public call (eager) and reads its output back.  The copies run
  # on their own streams and overlap the neighbouring steps' compute, as a
  # serving loop would stream batches: step i's upload on the H2D engine,
  # step i-1's forward, step i-2's download on the D2H engine.  Two device
  # input buffers; a buffer is refilled only after the forward that read it.
  h_host = h.cpu().pin_memory()
  out_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()
  h_dev = [torch.empty_like(h), torch.empty_like(h)]
  up_stream, down_stream = torch.cuda.Stream(), torch.cuda.Stream()
  barrier()
  torch.cuda.synchronize()
  ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  ev2.record(up_stream)
  used = [None, None]  # forward-done event of the last step that read each buffer
  for i in range(args.steps):
    buf = h_dev[i % 2]
    with torch.cuda.stream(up_stream):
      if used[i % 2] is not None:
        up_stream.wait_event(used[i % 2])
      buf.copy_(h_host, non_blocking=True)
      uploaded = torch.cuda.Event()
      uploaded.record(up_stream)
    stream.wait_event(uploaded)
    y = forward(buf)
    computed = torch.cuda.Event()
    computed.record(stream)
    used[i % 2] = computed
    with torch.cuda.stream(down_stream):
      down_stream.wait_event(computed)
      out_host.copy_(y, non_blocking=True)
      y.record_stream(down_stream)
  ev3.record(down_stream)
  torch.cuda.synchronize()
  barrier()
  ms_e2e = max_over_ranks(ev2.elapsed_time(ev3) / args.steps)
  e2e = {"value": args.tokens / (ms_e2e / 1e3), "unit": UNIT,
         "h2d_bytes_per_step": h_host.numel() * h_host.element_size() * world,
         "d2h_bytes_per_step": out_host.numel() * out_host.element_size() * world,
         "ms_per_step": ms_e2e,
         "pipelining": "upload, forward and download of neighbouring steps overlap"}

  # ---------------------------------------------------------------- dominant kernel
  # the MXFP4 fused gate/up grouped GEMM on this rank's routed rows (already
  # gathered into expert order, as the forward feeds it), timed alone
  rows = t_local * cfg.top_k
  if world == 1:
    _, inter = lm.latent_moe_forward(h, pw, cfg, return_intermediates=True)
    gs = inter["group_sizes"]
    xs = ops.gather_rows(inter["latent_projection"], inter["token_idx"])
  else:
    # stand-in for the expert-major rows this rank receives: the local share of
    # the routed rows spread evenly over the local experts
    gs = torch.full((n_local,), rows // n_local, dtype=torch.int32, device=dev)
    gs[0] += rows - int(gs.sum().item())
    xs = torch.randn(rows, cfg.latent_size, generator=gen, device=dev).to(
        torch.float16 if lm.latent_moe.mxfp4_f16_path(pw) else torch.bfloat16)
  act = torch.empty(rows, cfg.intermediate_size, dtype=xs.dtype, device=dev)
  for _ in range(2):
    ops.mxfp4_fused_gateup_situ(xs, pw.expert_gu_mx, gs, out=act)
  torch.cuda.synchronize()
  starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
  ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
  for i in range(args.steps):
    starts[i].record(stream)
    ops.mxfp4_fused_gateup_situ(xs, pw.expert_gu_mx, gs, out=act)
    ends[i].record(stream)
  torch.cuda.synchronize()
  k_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
  flops = 2.0 * rows * cfg.latent_size * 2 * cfg.intermediate_size
  peaks, peak_src = load_peaks()
  achieved = flops / (k_ms / 1e3) / 1e12
  roofline = {"kernel": "mxfp4 fused gate/up + SiTU-GLU grouped GEMM (tcgen05)",
              "bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
              "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
              "peak_source": f"{peak_src} dense bf16 burst (the kernel is timed alone)",
              "traffic": DOMINANT_TRAFFIC_BYTES, "ms_per_launch": k_ms,
              "flops_per_launch": flops,
              "weight_bytes_per_launch": int(pw.expert_gu_mx.packed.numel() +
                                             pw.expert_gu_mx.scale.numel())}

  # ---------------------------------------------------------------- CPU baseline
  cpu = None
  if rank == 0 and world == 1 and not args.no_cpu_baseline:
    cpu = cpu_baseline(args.seed, args.cpu_sample_tokens)

  if world > 1:
    torch.cuda.synchronize()
    ops.check_device_status()
    if xchg is not None:
      xchg.close()
    dist.barrier()
    dist.destroy_process_group()
  if rank != 0:
    return
  line = {
      "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
      "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
      "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
      "config": config_dict(args, world), "e2e": e2e, "gpu_launches": launches,
      "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks,
      "tflops": (2.0 * args.tokens * layer_macs(cfg)) / (ms / 1e3) / 1e12,
  }
  print(json.dumps(line), flush=True)


def layer_macs(cfg) -> float:
  """Multiply-accumulates per token of the layer (router, down, routed experts,
  up, shared expert)."""
  d, L, I, E, k = (cfg.hidden_size, cfg.latent_size, cfg.intermediate_size, cfg.num_experts,
                   cfg.top_k)
  si = I * cfg.num_shared_experts
  return d * E + d * L + k * (L * 2 * I + I * L) + L * d + d * 2 * si + si * d


if __name__ == "__main__":
  main()
