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
kernel (the MXFP4 fused gate/up + SiTU-GLU grouped GEMM: on one GPU the default
forward's block-scaled kernel on split activation rows, under expert parallelism
the weights-major kernel the exchange runs); `cpu_baseline` = the CPU
restatement of the reference forward on a token sample; `clocks` sampled
with nvidia-smi during the timed region.

`--impl reference` times the reference's algorithm on the host CPU instead
(the reference is JAX/TPU code; JAX is not installed, so its numpy
restatement runs, with all host threads), same metric and config.

On one GPU the line also carries `configs`: the standalone kernels of the
other benchmark configurations (2: bf16 ragged_dot; 3: bf16 fused gate/up +
SiTU-GLU and down grouped GEMMs over 65536 routed rows; 4: the MXFP4 grouped
matmul) with their time, TFLOP/s and fraction of the roofline that binds
them, and configuration 5 at 128, 1024 and 4096 tokens (`--no-extras` skips
them).  `--phases` instead prints one line of per-phase device times of
eager forwards (CUDA events between the phases, every rank, max over steps
of the median), the phase table of the expert-parallel exchange.
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
# dram bytes (read + write) per launch of the dominant kernel, from one ncu
# capture at this configuration (16384 tokens, 262144 routed rows; metrics
# dram__bytes_read.sum / dram__bytes_write.sum, the first gate/up launch of the
# default forward: the block-scaled gate/up + SiTU kernel on split rows):
# 1319.6 MB read + 520.5 MB written
DOMINANT_TRAFFIC_BYTES = int(1319579904 + 520499456)


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
  p.add_argument("--no-extras", action="store_true",
                 help="skip the standalone-kernel and token-sweep measurements (N=1)")
  p.add_argument("--phases", action="store_true",
                 help="print per-phase device times of eager forwards instead of the bench line")
  p.add_argument("--config2", action="store_true",
                 help="time only benchmark configuration 2 (bf16 ragged_dot) and print its line")
  p.add_argument("--config4", action="store_true",
                 help="time only benchmark configuration 4 (MXFP4 ragged_dot: exact and "
                      "block-scaled paths) and print its line")
  p.add_argument("--routing", action="store_true",
                 help="time only the routing-phase kernels (router, dispatch, gather, combine) "
                      "at configuration-5 shapes with --tokens tokens and print their line")
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


def cpu_forward_timer(seed: int, sample_tokens: int, w=None):
  """Returns (callable running one oracle forward of the sample, description,
  the host weights -- pass them back in to reuse their dequantised experts)."""
  from oracle import lmoe_oracle as O
  import numpy as np

  cfg = O.LatentMoEConfig(7168, 2048, 1024, 896, 16, 2)
  w = cpu_weights(seed, cfg, None) if w is None else w
  h = O.bf16_round(np.random.default_rng(seed + 1).standard_normal((sample_tokens, 7168),
                                                                   dtype=np.float32))

  def run():
    return O.latent_moe_forward(h, w, cfg, dtype="bf16")

  run()  # materialise (dequantise) the touched experts outside the timing
  return run, (f"{sample_tokens} tokens of configuration 5 through the numpy restatement of "
               "latent_moe_forward (bf16 emulated, MXFP4 experts dequantised once before "
               "timing, as the reference dequantises its checkpoint)"), w


def _median_s(run, reps: int) -> float:
  times = []
  for _ in range(reps):
    t0 = time.perf_counter()
    run()
    times.append(time.perf_counter() - t0)
  return statistics.median(times)


def cpu_threads() -> dict:
  """The host threads the CPU runs could use: cores, affinity, thread env,
  and the BLAS pools numpy actually runs (threadpoolctl)."""
  info = {"cpu_count": os.cpu_count(),
          "affinity_cores": len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity")
          else None,
          "env": {k: os.environ.get(k) for k in ("OMP_NUM_THREADS", "MKL_NUM_THREADS",
                                                 "OPENBLAS_NUM_THREADS")}}
  try:
    from threadpoolctl import threadpool_info
    info["blas"] = [{"api": d.get("internal_api"), "threads": d.get("num_threads")}
                    for d in threadpool_info()]
  except Exception:  # pragma: no cover - threadpoolctl missing
    info["blas"] = None
  return info


def cpu_coverage(seed: int, reps: int, w5) -> dict:
  """The numpy restatement on the other benchmark configurations, each a
  bounded sample, median of `reps` runs after one warm-up."""
  from oracle import lmoe_oracle as O
  import numpy as np

  out = {}
  # configuration 1: the reduced fp32 layer, all 128 tokens
  c1 = O.LatentMoEConfig(512, 256, 512, 64, 8, 1)
  w1 = O.init_weights_np(c1, 0, dtype="fp32")
  h1 = np.random.default_rng(0).standard_normal((128, 512), dtype=np.float32)
  run1 = lambda: O.latent_moe_forward(h1, w1, c1, dtype="fp32")
  run1()
  t = _median_s(run1, reps)
  out["config1"] = {"tokens_per_s": 128 / t, "ms": t * 1e3, "sample": "all 128 tokens, fp32"}
  # configuration 2: ragged_dot 8192 x 2048 @ (128, 2048, 1536), Zipf(1.1) groups
  rng = np.random.default_rng(1)
  m, k, n, g = 8192, 2048, 1536, 128
  gs = zipf_group_sizes(rng, m, g)
  lhs = O.bf16_round(rng.standard_normal((m, k), dtype=np.float32) / np.float32(np.sqrt(k)))
  rhs = O.bf16_round(rng.standard_normal((g, k, n), dtype=np.float32) / np.float32(np.sqrt(k)))
  run2 = lambda: O.ragged_dot(lhs, rhs, gs, dtype="bf16")
  run2()
  t = _median_s(run2, reps)
  out["config2"] = {"tflops": 2.0 * m * k * n / t / 1e12, "ms": t * 1e3,
                    "sample": "the full configuration (f32 matmuls of bf16 values)"}
  del lhs, rhs
  # configuration 4: MXFP4 dequant-then-matmul, 8 of the 128 experts with
  # their rows (uniform group sizes over 16384 rows), dequantised once
  k4, n4, g4 = 4096, 2048, 8
  gs4 = rng.multinomial(16384, np.full(128, 1 / 128))[:g4].astype(np.int32)
  packed = rng.integers(0, 256, (g4, n4, k4 // 2), dtype=np.uint8)
  scale = rng.integers(121, 130, (g4, n4, k4 // 32), dtype=np.uint8)
  lazy = O.LazyMXFP4Experts(packed, scale)
  x4 = O.bf16_round(rng.standard_normal((int(gs4.sum()), k4), dtype=np.float32))
  run4 = lambda: O.ragged_dot(x4, lazy, gs4, dtype="bf16")
  run4()
  t = _median_s(run4, reps)
  rows4 = int(gs4.sum())
  out["config4"] = {"tflops": 2.0 * rows4 * k4 * n4 / t / 1e12, "ms": t * 1e3,
                    "sample": f"{g4} of 128 experts, their {rows4} rows (weights dequantised "
                              "once before timing)"}
  # configuration 5 at 128 and 1024 tokens (n = 1 semantics)
  for t5 in (128, 1024):
    run5, _, _ = cpu_forward_timer(seed, t5, w5)
    t = _median_s(run5, reps)
    out[f"config5_t{t5}"] = {"tokens_per_s": t5 / t, "ms": t * 1e3,
                             "sample": f"{t5} tokens, n = 1 semantics"}
  return out


def zipf_group_sizes(rng, m: int, g: int, s: float = 1.1, n_zero: int = 8):
  """Zipf(s) multinomial over a seeded permutation of the groups with n_zero
  groups forced empty (benchmark configuration 2)."""
  import numpy as np
  p = (np.arange(g) + 1.0) ** (-s)
  p = p[rng.permutation(g)]
  p[rng.choice(g, size=min(n_zero, g - 1), replace=False)] = 0
  p /= p.sum()
  return rng.multinomial(m, p).astype(np.int32)


def cpu_baseline(seed: int, sample_tokens: int, reps: int = 5, coverage: bool = True) -> dict:
  run, desc, w = cpu_forward_timer(seed, sample_tokens)
  t = _median_s(run, reps)
  res = {"value": sample_tokens / t, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
         "sample": desc + f"; median of {reps} after one warm-up", "threads": cpu_threads()}
  if coverage:
    res["coverage"] = cpu_coverage(seed, reps, w)
  return res


def run_reference(args, world, rank):
  if rank != 0:
    return
  run, desc, _ = cpu_forward_timer(args.seed, args.cpu_sample_tokens)
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
                                        "cannot run; its numpy restatement runs instead)",
                       "threads": cpu_threads()},
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


def time_launches(fn, iters: int, warmup: int = 2) -> float:
  """Mean device time (ms) of fn() over `iters` back-to-back launches: CUDA
  events on the current stream before the first and after the last, no host
  synchronisation in between (so the host's launch work overlaps the device's
  execution of the previous launch instead of adding idle gaps)."""
  import torch
  stream = torch.cuda.current_stream()
  for _ in range(warmup):
    fn()
  torch.cuda.synchronize()
  a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  a.record(stream)
  for _ in range(iters):
    fn()
  b.record(stream)
  torch.cuda.synchronize()
  return a.elapsed_time(b) / iters


def roofline_entry(ms: float, flops: float, bytes_: float, peaks: dict, peak_src: str) -> dict:
  """Achieved TFLOP/s and GB/s of the algorithmic work, and the fraction of
  the binding roofline (the larger of the tensor-time and HBM-time floors)."""
  t_tc = flops / (peaks["bf16_tflops"] * 1e12)
  t_hbm = bytes_ / (peaks["hbm_gbs"] * 1e9)
  bound = "tensor" if t_tc >= t_hbm else "hbm"
  return {"ms": ms, "tflops": flops / (ms / 1e3) / 1e12, "gbs": bytes_ / (ms / 1e3) / 1e9,
          "bound": bound, "frac": max(t_tc, t_hbm) / (ms / 1e3),
          "flops": flops, "bytes": bytes_,
          "peak": f"{peak_src}: {peaks['bf16_tflops']} TFLOP/s bf16, {peaks['hbm_gbs']} GB/s"}


def gpu_routing_kernels(args, lm, ops, dev, peaks, peak_src, tokens: int) -> dict:
  """The routing-phase kernels of configuration 5 at `tokens` tokens, each
  timed alone (back-to-back launches): the fused router gate beside the
  two-step path it replaces, the dispatch sort, the row gather in token order
  (each latent row read once and stored top_k times, as the layer runs it)
  beside the sorted-order gather, the MXFP8 quantising gather in both orders
  and the weighted combine + RMSNorm.  The gathers write k times what they
  read; their bytes are the rows written (+ the rows read once), against the
  measured copy bandwidth (a torch fill and copy of the same size are timed
  beside them for reference)."""
  import torch

  iters = max(3, min(args.steps, 20))
  cfg = lm.full_layer_config()
  T, d, L, E, K = tokens, cfg.hidden_size, cfg.latent_size, cfg.num_experts, cfg.top_k
  gen = torch.Generator(device=dev).manual_seed(args.seed)
  h = torch.randn(T, d, generator=gen, device=dev).to(torch.bfloat16)
  wr = (torch.randn(E, d, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
  bias = torch.randn(E, generator=gen, device=dev) * 0.5
  x = torch.randn(T, L, generator=gen, device=dev).to(torch.bfloat16)
  rows = T * K
  out = {"tokens": T}
  ws = torch.empty(ops.router_fused_workspace_size(T, E, K), dtype=torch.uint8, device=dev)
  idx, w = ops.router_gate_fused(h, wr, bias, K, workspace=ws)
  ms = time_launches(lambda: ops.router_gate_fused(h, wr, bias, K, workspace=ws), iters)
  out["router_fused"] = roofline_entry(ms, 2.0 * T * d * E, T * d * 2 + E * d * 2 + T * K * 8,
                                       peaks, peak_src)
  logits = ops.router_logits(h, wr)
  ms_l = time_launches(lambda: ops.router_logits(h, wr), iters)
  ms_k = time_launches(lambda: ops.router_topk(logits, bias, K), iters)
  out["router_two_step"] = {"logits_ms": ms_l, "topk_ms": ms_k, "ms": ms_l + ms_k}
  del logits
  d_ = ops.dispatch(idx, w, E, want_order=False)
  out["dispatch"] = {"ms": time_launches(lambda: ops.dispatch(idx, w, E, want_order=False), iters),
                     "nonempty_experts": int((d_.group_sizes > 0).sum())}
  gb = rows * L * 2
  buf = torch.empty(rows, L, dtype=torch.float16, device=dev)
  ms_fill = time_launches(lambda: buf.fill_(1.0), iters)
  src = torch.empty_like(buf)
  ms_copy = time_launches(lambda: buf.copy_(src), iters)
  del src
  out["torch_reference_kernels"] = {"fill_gbs": gb / (ms_fill / 1e3) / 1e9,
                                    "copy_gbs": 2 * gb / (ms_copy / 1e3) / 1e9,
                                    "how": f"torch fill_ / copy_ of {gb / 1e9:.2f} GB"}
  moved = gb + T * L * 2  # rows written + each source row read once
  ms = time_launches(lambda: ops.scatter_rows(x, d_.slot_pos, K, out=buf, to_f16=True), iters)
  out["gather_rows_f16_token_order"] = {"ms": ms, "gbs": moved / (ms / 1e3) / 1e9,
                                        "frac_of_copy_peak": moved / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]}
  ms = time_launches(lambda: ops.gather_rows(x, d_.token_idx, out=buf, to_f16=True), iters)
  out["gather_rows_f16_sorted_order"] = {"ms": ms, "gbs": moved / (ms / 1e3) / 1e9,
                                         "frac_of_copy_peak": moved / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]}
  mx = ops.quantize_mxfp8_scatter(x, d_.group_sizes, d_.slot_pos, K)
  qb = rows * L + rows * L // 32 + T * L * 2
  ms = time_launches(lambda: ops.quantize_mxfp8_scatter(x, d_.group_sizes, d_.slot_pos, K, out=mx),
                     iters)
  out["gather_quantize_mxfp8_token_order"] = {"ms": ms, "gbs": qb / (ms / 1e3) / 1e9,
                                              "frac_of_copy_peak": qb / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]}
  ms = time_launches(lambda: ops.quantize_mxfp8_rows(x, d_.group_sizes, d_.token_idx, out=mx),
                     iters)
  out["gather_quantize_mxfp8_sorted_order"] = {"ms": ms, "gbs": qb / (ms / 1e3) / 1e9}
  del mx
  eo = buf.view(torch.bfloat16)
  ns = torch.ones(L, device=dev).to(torch.bfloat16)
  ms = time_launches(lambda: ops.combine_rmsnorm(eo, d_.slot_pos, w, ns, cfg.rms_norm_eps), iters)
  cb = gb + T * L * 2
  out["combine_rmsnorm"] = {"ms": ms, "gbs": cb / (ms / 1e3) / 1e9,
                            "frac_of_copy_peak": (cb / (ms / 1e3) / 1e9) / peaks["hbm_gbs"]}
  ops.check_device_status(dev)
  return out


def gpu_config2(args, ops, dev, peaks, peak_src, iters: int) -> dict:
  """Benchmark configuration 2 alone: ragged_dot, lhs (8192, 2048), rhs
  (128, 2048, 1536) in the reference's (G, K, N) layout, Zipf(1.1) group
  sizes with empty groups."""
  import numpy as np
  import torch

  gen = torch.Generator(device=dev).manual_seed(args.seed)
  m, k, n, g = 8192, 2048, 1536, 128
  gs = zipf_group_sizes(np.random.default_rng(1), m, g)
  lhs = (torch.randn(m, k, generator=gen, device=dev) / k ** 0.5).to(torch.bfloat16)
  rhs = (torch.randn(g, k, n, generator=gen, device=dev) / k ** 0.5).to(torch.bfloat16)
  gsd = torch.from_numpy(gs).to(dev)
  res = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
  ms = time_launches(lambda: ops.ragged_dot(lhs, rhs, gsd, out=res), iters)
  nz = int((gs > 0).sum())
  entry = roofline_entry(ms, 2.0 * m * k * n, m * k * 2 + nz * k * n * 2 + m * n * 2, peaks,
                         peak_src)
  entry["nonempty_groups"] = nz
  return entry


def gpu_config4(args, lm, ops, dev, peaks, peak_src, iters: int, exact: bool = True,
                blockscaled: bool = True) -> dict:
  """Benchmark configuration 4 alone: MXFP4 experts (128 x N 2048 x K 4096;
  codes uniform over all 16, scale exponents uniform in [-6, 2]), x (16384,
  4096) N(0, 1), uniform-random group sizes.  The exact path runs with bf16
  and with f16 operands; the block-scaled path (x quantised to MXFP8,
  kind::mxf8f6f4) is timed as the GEMM alone and with the quantisation, its
  peak twice the measured bf16 burst."""
  import numpy as np
  import torch

  g4, k4, n4, m4 = 128, 4096, 2048, 16384
  gen = torch.Generator(device=dev).manual_seed(args.seed + 4)
  w4 = lm.random_mxfp4(g4, n4, k4, seed=3, device=dev, scale_exp=(-6, 2))
  x4 = torch.randn(m4, k4, generator=gen, device=dev).to(torch.bfloat16)
  gs4 = torch.from_numpy(np.random.default_rng(3).multinomial(m4, np.full(g4, 1 / g4)).astype(
      np.int32)).to(dev)
  o4 = torch.empty(m4, n4, dtype=torch.bfloat16, device=dev)
  flops = 2.0 * m4 * k4 * n4
  w_bytes = g4 * n4 * (k4 // 2 + k4 // 32)
  out = {}
  if exact:
    byt = m4 * k4 * 2 + w_bytes + m4 * n4 * 2
    ms = time_launches(lambda: ops.mxfp4_ragged_dot(x4, w4, gs4, out=o4), iters)
    out["config4_mxfp4_bf16_operands"] = roofline_entry(ms, flops, byt, peaks, peak_src)
    x4h = x4.to(torch.float16)
    ms = time_launches(lambda: ops.mxfp4_ragged_dot(x4h, w4, gs4, out=o4), iters)
    out["config4_mxfp4_f16_operands"] = roofline_entry(ms, flops, byt, peaks, peak_src)
    del x4h
    # the same exact matmul on the block-scaled tensor core: the rows split
    # into two e4m3 planes (the split timed with the GEMM), two MMAs per K
    # step at the MXFP8 rate, so its peak is the bf16 one
    wb = ops.prepare_mxfp4_blockscaled(w4)
    rows = ops.quantize_split_rows(x4, gs4)
    ms = time_launches(lambda: ops.mxfp4_ragged_dot_blockscaled(x4, wb, gs4, out=o4, rows=rows),
                       iters)
    out["config4_exact_split_blockscaled"] = roofline_entry(ms, flops, byt, peaks, peak_src)
    del wb, rows
  if blockscaled:
    fp8_peak = dict(peaks, bf16_tflops=2 * peaks["bf16_tflops"])
    src = f"{peak_src} (fp8 = 2 x bf16 burst)"
    wb = ops.prepare_mxfp4_blockscaled(w4)
    a4 = ops.quantize_mxfp8_rows(x4, gs4)
    # these GEMMs write the padded row layout: every group starts at a
    # multiple of 128 rows, so their output has the padded row count
    o4 = torch.empty(a4.q.shape[-2], n4, dtype=torch.bfloat16, device=dev)
    ops.mxfp8_mxfp4_ragged_dot(a4, wb, out=o4)
    ms = time_launches(lambda: ops.mxfp8_mxfp4_ragged_dot(a4, wb, out=o4), iters)
    out["config4_blockscaled_gemm"] = roofline_entry(
        ms, flops, m4 * k4 * (1 + 1 / 32) + w_bytes + m4 * n4 * 2, fp8_peak, src)
    ms = time_launches(lambda: (ops.quantize_mxfp8_rows(x4, gs4, out=a4),
                                ops.mxfp8_mxfp4_ragged_dot(a4, wb, out=o4)), iters)
    out["config4_blockscaled_with_quantize"] = roofline_entry(
        ms, flops, m4 * k4 * 2 + w_bytes + m4 * n4 * 2, fp8_peak, src)
    # MXFP4 activations (kind::mxf4): its MMA runs at four times the bf16 rate
    fp4_peak = dict(peaks, bf16_tflops=4 * peaks["bf16_tflops"])
    src4 = f"{peak_src} (fp4 = 4 x bf16 burst)"
    a4f = ops.quantize_mxfp4_rows(x4, gs4)
    ops.mxfp4_mxfp4_ragged_dot(a4f, wb, out=o4)
    ms = time_launches(lambda: ops.mxfp4_mxfp4_ragged_dot(a4f, wb, out=o4), iters)
    out["config4_mxf4_gemm"] = roofline_entry(
        ms, flops, m4 * k4 * (0.5 + 1 / 32) + w_bytes + m4 * n4 * 2, fp4_peak, src4)
    ms = time_launches(lambda: (ops.quantize_mxfp4_rows(x4, gs4, out=a4f),
                                ops.mxfp4_mxfp4_ragged_dot(a4f, wb, out=o4)), iters)
    out["config4_mxf4_with_quantize"] = roofline_entry(
        ms, flops, m4 * k4 * 2 + w_bytes + m4 * n4 * 2, fp4_peak, src4)
    del wb, a4, a4f
  del w4, x4, o4
  torch.cuda.synchronize()
  torch.cuda.empty_cache()
  return out


def gpu_config_extras(args, lm, ops, dev, peaks, peak_src) -> dict:
  """Standalone kernels of benchmark configurations 2, 3 and 4 at full size."""
  import numpy as np
  import torch

  iters = max(3, min(args.steps, 10))
  out = {}
  gen = torch.Generator(device=dev).manual_seed(args.seed)

  out["config2_ragged_dot_bf16"] = gpu_config2(args, ops, dev, peaks, peak_src, iters)

  # configuration 3: 4096 tokens x top-16 over 896 experts (router bias
  # N(0, 0.5^2)), latent 2048, intermediate 1024, bf16 weights
  E, L, I, T, K = 896, 2048, 1024, 4096, 16
  x = torch.randn(T, L, generator=gen, device=dev).to(torch.bfloat16)
  wr = (torch.randn(E, L, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
  bias = torch.randn(E, generator=gen, device=dev) * 0.5
  idx, wts = ops.router_gate(x, wr, bias, K)
  d = ops.dispatch(idx, wts, E)
  rows = ops.gather_rows(x, d.token_idx)
  w_gu = torch.empty(E, 2 * I, L, dtype=torch.bfloat16, device=dev)
  w_dn = torch.empty(E, L, I, dtype=torch.bfloat16, device=dev)
  for e0 in range(0, E, 64):
    w_gu[e0:e0 + 64] = (torch.randn(64, 2 * I, L, generator=gen, device=dev) * 0.02).to(
        torch.bfloat16)
    w_dn[e0:e0 + 64] = (torch.randn(64, L, I, generator=gen, device=dev) * 0.02).to(
        torch.bfloat16)
  M = T * K
  act = torch.empty(M, I, dtype=torch.bfloat16, device=dev)
  dn = torch.empty(M, L, dtype=torch.bfloat16, device=dev)
  ms_gu = time_launches(lambda: ops.fused_gateup_situ(rows, w_gu, d.group_sizes, rhs_layout="gnk",
                                                      out=act), iters)
  ms_dn = time_launches(lambda: ops.ragged_dot(act, w_dn, d.group_sizes, rhs_layout="gnk",
                                               out=dn), iters)
  nz = int((d.group_sizes > 0).sum())
  out["config3_gateup_situ_bf16"] = roofline_entry(
      ms_gu, 2.0 * M * L * 2 * I, M * L * 2 + nz * 2 * I * L * 2 + M * I * 2, peaks, peak_src)
  out["config3_down_bf16"] = roofline_entry(
      ms_dn, 2.0 * M * I * L, M * I * 2 + nz * L * I * 2 + M * L * 2, peaks, peak_src)
  out["config3_gateup_situ_bf16"]["nonempty_groups"] = nz
  del x, w_gu, w_dn, act, dn, rows

  out.update(gpu_config4(args, lm, ops, dev, peaks, peak_src, iters, blockscaled=False))
  torch.cuda.synchronize()
  torch.cuda.empty_cache()
  return out


def gpu_mxfp8_extras(args, lm, ops, pw, cfg, h, dev, peaks, peak_src) -> dict:
  """The opt-in block-scaled path (MXFP8 activations x MXFP4 weights on
  kind::mxf8f6f4): the configuration-5 layer forward with
  mxfp4_operand="mxfp8" (and with "mxfp4": MXFP4 activations on kind::mxf4),
  its two routed GEMMs and the quantising gather standalone, and
  configuration 4 on it.  Its MMA runs at twice the bf16 rate, so its
  roofline peak here is twice the measured bf16 burst."""
  import torch

  iters = max(3, min(args.steps, 10))
  fp8_peak = dict(peaks, bf16_tflops=2 * peaks["bf16_tflops"])
  src = f"{peak_src} (fp8 = 2 x bf16 burst)"
  out = {}
  for _ in range(2):
    lm.latent_moe_forward(h, pw, cfg, mxfp4_operand="mxfp8")
  torch.cuda.synchronize()
  graph = torch.cuda.CUDAGraph()
  with torch.cuda.graph(graph):
    lm.latent_moe_forward(h, pw, cfg, mxfp4_operand="mxfp8")
  ms = time_launches(graph.replay, max(5, args.steps))
  out["layer"] = {"ms": ms, "tokens_per_s": h.shape[0] / (ms / 1e3)}
  del graph
  # the same layer with MXFP4 activations (kind::mxf4), and exact on the
  # weights-major kernels (codes expanded to f16 tiles, kind::f16)
  for mode, key in (("mxfp4", "layer_mxfp4_activations"), ("f16", "layer_exact_weights_major")):
    for _ in range(2):
      lm.latent_moe_forward(h, pw, cfg, mxfp4_operand=mode)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
      lm.latent_moe_forward(h, pw, cfg, mxfp4_operand=mode)
    ms = time_launches(graph.replay, max(5, args.steps))
    out[key] = {"ms": ms, "tokens_per_s": h.shape[0] / (ms / 1e3)}
    del graph
  _, inter = lm.latent_moe_forward(h, pw, cfg, return_intermediates=True, mxfp4_operand="mxfp8")
  gs, tix = inter["group_sizes"], inter["token_idx"]
  x = inter["latent_projection"]
  gu, dn = lm.latent_moe.blockscaled_experts(pw)
  rows = ops.quantize_mxfp8_rows(x, gs, tix)
  act = ops.mxfp8_mxfp4_gateup_situ(rows, gu)
  act_q = ops.quantize_mxfp8_rows(act, gs, padded_input=True)
  down = ops.mxfp8_mxfp4_ragged_dot(act_q, dn)
  M = tix.shape[0]
  L, I = cfg.latent_size, cfg.intermediate_size
  nz = int((gs > 0).sum())
  ms_q = time_launches(lambda: ops.quantize_mxfp8_rows(x, gs, tix, out=rows), iters)
  ms_gu = time_launches(lambda: ops.mxfp8_mxfp4_gateup_situ(rows, gu, out=act), iters)
  ms_dn = time_launches(lambda: ops.mxfp8_mxfp4_ragged_dot(act_q, dn, out=down), iters)
  out["gather_quantize"] = {"ms": ms_q, "gbs": (M * L * 2 + M * L * (1 + 1 / 32)) / (ms_q / 1e3) / 1e9}
  out["gateup_situ"] = roofline_entry(ms_gu, 2.0 * M * L * 2 * I,
                                      M * L * (1 + 1 / 32) + nz * 2 * I * L * 0.53 + M * I * 2,
                                      fp8_peak, src)
  out["down"] = roofline_entry(ms_dn, 2.0 * M * I * L,
                               M * I * (1 + 1 / 32) + nz * L * I * 0.53 + M * L * 2, fp8_peak, src)
  c4 = gpu_config4(args, lm, ops, dev, peaks, peak_src, iters, exact=False)
  out["config4"] = c4["config4_blockscaled_with_quantize"]
  out["config4_gemm"] = c4["config4_blockscaled_gemm"]
  out["config4_mxf4_gemm"] = c4["config4_mxf4_gemm"]
  out["config4_mxf4_with_quantize"] = c4["config4_mxf4_with_quantize"]
  torch.cuda.synchronize()
  torch.cuda.empty_cache()
  return out


def gpu_token_sweep(args, lm, pw, cfg, dev, tokens=(128, 1024, 4096)) -> dict:
  """Configuration 5 at smaller token counts (one GPU, CUDA-graph replay):
  the default forward (the exact product on the block-scaled tensor core,
  and at token counts whose dense projections would not fill the SMs, the
  split-K phase kernels for them), the weights-major f16-operand kernels
  (mxfp4_operand="f16") as `f16_ms`, and, where the default takes the phase
  kernels, the same forward without them as `no_dense_phases_ms`."""
  import torch
  out = {}
  for t in tokens:
    gen = torch.Generator(device=dev).manual_seed(args.seed * 7919 + t)
    h = torch.randn(t, cfg.hidden_size, generator=gen, device=dev).to(torch.bfloat16)
    variants = {"auto": {}, "f16": {"mxfp4_operand": "f16"}}
    if lm.latent_moe._use_dense_phases(None, pw, cfg, t, h, torch.bfloat16, False):
      variants["no_dense_phases"] = {"dense_phases": False}
    res = {}
    for name, kw in variants.items():
      for _ in range(2):
        lm.latent_moe_forward(h, pw, cfg, **kw)
      torch.cuda.synchronize()
      graph = torch.cuda.CUDAGraph()
      with torch.cuda.graph(graph):
        lm.latent_moe_forward(h, pw, cfg, **kw)
      res[name] = time_launches(graph.replay, max(5, args.steps))
      del graph
    out[f"T{t}"] = {"ms": res["auto"], "tokens_per_s": t / (res["auto"] / 1e3),
                    "f16_ms": res["f16"]}
    if "no_dense_phases" in res:
      out[f"T{t}"]["no_dense_phases_ms"] = res["no_dense_phases"]
  return out


def run_phases(args, lm, ops, forward_marked, world, rank, dev, stats=None):
  """Per-phase device times of eager forwards: CUDA events recorded on the
  main stream after each phase is enqueued; per rank the median over steps."""
  import torch
  import torch.distributed as dist
  stream = torch.cuda.current_stream()
  for _ in range(args.warmup):
    forward_marked(None)
  torch.cuda.synchronize()
  per_step = []
  for _ in range(args.steps):
    names, evs = [], []
    e0 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)

    def mark(name):
      e = torch.cuda.Event(enable_timing=True)
      e.record(torch.cuda.current_stream())
      names.append(name)
      evs.append(e)

    forward_marked(mark)
    torch.cuda.synchronize()
    prev, d = e0, {}
    for nm, e in zip(names, evs):
      d[nm] = d.get(nm, 0.0) + prev.elapsed_time(e)
      prev = e
    d["total"] = e0.elapsed_time(evs[-1])
    per_step.append(d)
  ops.check_device_status()
  med = {k: statistics.median(s[k] for s in per_step) for k in per_step[0]}
  if stats is not None:
    med.update(stats())
  table = [None] * world
  if world > 1:
    dist.all_gather_object(table, med)
  else:
    table = [med]
  return table


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
  if args.config2:
    if rank == 0:
      peaks, peak_src = load_peaks()
      res = gpu_config2(args, ops, dev, peaks, peak_src, max(3, min(args.steps, 20)))
      print(json.dumps({"config2_ragged_dot_bf16": res,
                        "launch": "alone, back-to-back launches between CUDA events"}), flush=True)
    if world > 1:
      dist.barrier()
      dist.destroy_process_group()
    return

  if args.config4:
    if rank == 0:
      peaks, peak_src = load_peaks()
      res = gpu_config4(args, lm, ops, dev, peaks, peak_src, max(3, min(args.steps, 20)))
      print(json.dumps({"config4": res,
                        "launch": "alone, back-to-back launches between CUDA events"}), flush=True)
    if world > 1:
      dist.barrier()
      dist.destroy_process_group()
    return

  if args.routing:
    if rank == 0:
      peaks, peak_src = load_peaks()
      res = gpu_routing_kernels(args, lm, ops, dev, peaks, peak_src, args.tokens)
      print(json.dumps({"routing_kernels": res, "config": config_dict(args, 1),
                        "launch": "each kernel alone, back-to-back launches between CUDA events"}),
            flush=True)
    if world > 1:
      dist.barrier()
      dist.destroy_process_group()
    return

  pw = lm.init_prepared_mxfp4(cfg, seed=args.seed, device=dev, bias_std=0.5,
                              expert_start=rank * n_local, num_local_experts=n_local)
  gen = torch.Generator(device=dev).manual_seed(args.seed * 7919 + rank)
  h = torch.randn(t_local, cfg.hidden_size, generator=gen, device=dev).to(torch.bfloat16)
  # Several GPUs: the routed experts on the weights-major f16-operand kernels.
  # The receive region holds the rows unpadded in bf16/f16, so the split path
  # needs a separate quantising pass there (the one-GPU forward folds it into
  # the gather); measured at n = 2 the experts phase took 2.00 / 2.24 ms per
  # rank with it against 1.94 / 2.21 ms on the weights-major kernels.
  backend = GpuBackend(pw, cfg, mxfp4_operand="f16")
  xchg = PeerExchange(cfg, t_local) if world > 1 and args.exchange == "peer" else None

  def forward(x, mark=None):
    if xchg is not None:
      return ep_forward_peer(x, backend, cfg, xchg, mark=mark)
    if world > 1:
      return ep_forward(x, backend, cfg)
    return lm.latent_moe_forward(x, pw, cfg, mark=mark)

  if args.phases:
    stats = (lambda: {"rows_received": int(xchg.local_gs.sum().item())}) if xchg else None
    table = run_phases(args, lm, ops, lambda mark: forward(h, mark), world, rank, dev, stats)
    if xchg is not None:
      xchg.close()
    if world > 1:
      dist.barrier()
      dist.destroy_process_group()
    if rank == 0:
      print(json.dumps({"phases_ms": table, "n_gpus": world, "steps": args.steps,
                        "warmup": args.warmup, "config": config_dict(args, world),
                        "launch": "eager, CUDA events between phases on the main stream; "
                                  "median over steps per rank"}), flush=True)
    return

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
  # The routed gate/up + SiTU-GLU grouped GEMM on this rank's routed rows, fed
  # as the forward feeds it, timed alone.  One GPU: the default forward's
  # kernel -- the block-scaled MMA (kind::mxf8f6f4) on the e2m1 weight codes
  # and the latent rows split into two e4m3 planes (hi + remainder), two MMAs
  # per 32-wide K slice, i.e. the exact product at the FP8 instruction rate
  # twice over = the bf16 rate; it writes the down GEMM's split rows.
  # Several GPUs: the expert-parallel path's weights-major kernel (codes
  # expanded to f16 tiles in shared memory, kind::f16) on a stand-in for the
  # rows this rank's experts receive.
  rows = t_local * cfg.top_k
  if world == 1:
    _, inter = lm.latent_moe_forward(h, pw, cfg, return_intermediates=True)
    gs = inter["group_sizes"]
    gu_bs, _ = lm.latent_moe.blockscaled_experts(pw)
    xs = ops.quantize_split_scatter(inter["latent_projection"], gs, inter["slot_pos"],
                                    cfg.top_k)
    act = ops.blockscaled_gateup_situ_quantized(xs, gu_bs, "e4m3x2")
    gateup = lambda: ops.blockscaled_gateup_situ_quantized(xs, gu_bs, "e4m3x2", out=act)
    dom_kernel = ("mxfp4 fused gate/up + SiTU-GLU grouped GEMM, block-scaled tcgen05 "
                  "kind::mxf8f6f4 on split (hi + lo e4m3) activation rows: the exact product")
    # the capture holds for the configuration it was taken at
    traffic = DOMINANT_TRAFFIC_BYTES if args.tokens == 16384 else None
    del inter
  else:
    # stand-in for the expert-major rows this rank receives: the local share of
    # the routed rows spread evenly over the local experts
    gs = torch.full((n_local,), rows // n_local, dtype=torch.int32, device=dev)
    gs[0] += rows - int(gs.sum().item())
    xs = torch.randn(rows, cfg.latent_size, generator=gen, device=dev).to(
        torch.float16 if lm.latent_moe.mxfp4_f16_path(pw) else torch.bfloat16)
    act = torch.empty(rows, cfg.intermediate_size, dtype=xs.dtype, device=dev)
    gateup = lambda: ops.mxfp4_fused_gateup_situ(xs, pw.expert_gu_mx, gs, out=act)
    dom_kernel = ("mxfp4 fused gate/up + SiTU-GLU grouped GEMM, weights-major (tcgen05 "
                  "kind::f16), this rank's experts")
    traffic = None  # the one-GPU capture does not cover this rank's row count
  flops = 2.0 * rows * cfg.latent_size * 2 * cfg.intermediate_size
  peaks, peak_src = load_peaks()
  # (1) alone on an idle GPU, at its boost clock: the condition of the burst
  # peak (a short run from idle)
  torch.cuda.synchronize()
  time.sleep(2.0)
  with ClockSampler(local_rank) as dclk:
    k_ms = time_launches(gateup, max(args.steps, 10))
  # (2) right after about three seconds of back-to-back layer forwards: the power-
  # capped clock the kernel runs at inside a long serving loop, against the
  # sustained peak (cuBLAS measured the same way)
  for _ in range(max(1, int(3000.0 / ms))):  # ms is the max over ranks: the same count everywhere
    step()
  torch.cuda.synchronize()
  with ClockSampler(local_rank) as hclk:
    k_ms_hot = time_launches(gateup, max(args.steps, 10), warmup=0)
  achieved = flops / (k_ms / 1e3) / 1e12
  achieved_hot = flops / (k_ms_hot / 1e3) / 1e12
  roofline = {"kernel": dom_kernel,
              "bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
              "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
              "peak_source": f"{peak_src} dense bf16 burst (the kernel is timed alone, from idle)",
              "traffic": traffic, "ms_per_launch": k_ms,
              "flops_per_launch": flops, "clocks": dclk.summary(),
              "weight_bytes_per_launch": int(pw.expert_gu_mx.packed.numel() +
                                             pw.expert_gu_mx.scale.numel()),
              "sustained": {"ms_per_launch": k_ms_hot, "achieved": achieved_hot,
                            "peak": peaks["bf16_tflops_sustained"],
                            "frac": achieved_hot / peaks["bf16_tflops_sustained"],
                            "clocks": hclk.summary(),
                            "how": "timed right after 3 s of back-to-back layer forwards"}}

  # ---------------------------------------------------------------- other configurations
  configs = sweep = mx8 = routing = None
  if world == 1 and not args.no_extras:
    del xs, act, gs
    configs = gpu_config_extras(args, lm, ops, dev, peaks, peak_src)
    sweep = gpu_token_sweep(args, lm, pw, cfg, dev)
    mx8 = gpu_mxfp8_extras(args, lm, ops, pw, cfg, h, dev, peaks, peak_src)
    routing = gpu_routing_kernels(args, lm, ops, dev, peaks, peak_src, args.tokens)

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
  if configs is not None:
    line["configs"] = configs
    line["token_sweep"] = sweep
    line["mxfp8_fast_path"] = mx8
    line["routing_kernels"] = routing
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
