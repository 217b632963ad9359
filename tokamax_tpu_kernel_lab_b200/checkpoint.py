"""One LatentMoE layer of the Kimi K3 checkpoint -> the kernel layouts.

The checkpoint stores, under `model.layers.{i}.block_sparse_moe.` for MoE
layers i >= 1 (layer 0 is dense), the field mapping of
06_kimi_k3_golden_validation/prepare_real_checkpoint_layer.py:101-178 and
README.md:303-318:

  gate.weight                          (E, d)   bf16 router, (out, in)
  gate.e_score_correction_bias         (E,)     selection bias
  routed_expert_down_proj.weight       (L, d)   nn.Linear(d, L)
  routed_expert_up_proj.weight         (d, L)   nn.Linear(L, d)
  routed_expert_norm.weight            (L,)     RMSNorm scale
  shared_experts.{gate,up}_proj.weight (Is, d); shared_experts.down_proj.weight (d, Is)
  experts.{e}.w{1,3}.weight_packed     (I, L/2) u8 MXFP4 codes (gate, up), low nibble = even k
  experts.{e}.w{1,3}.weight_scale      (I, L/32) u8 E8M0
  experts.{e}.w2.weight_packed/scale   (L, I/2), (L, I/32)  (down)

Every nn.Linear (out, in) matrix is already the K-major layout the kernels
read, so loading is stacking: w1 over w3 per expert gives the fused
[gate | up] MXFP4 operand (E, 2I, L/2), w2 gives (E, L, I/2).  Expert
parallelism loads only the rank's contiguous expert range.  Files are read
with safetensors (lazily, key by key); a sharded checkpoint is a list of
files or its `model.safetensors.index.json`.
"""

from __future__ import annotations

import dataclasses
import json
import pathlib
from typing import Iterable, Mapping

import torch

from . import ops
from .latent_moe import LatentMoEConfig, PreparedWeights

FIRST_MOE_LAYER = 1  # prepare_real_checkpoint_layer.py:90 (layer 0 is a dense MLP)


@dataclasses.dataclass(frozen=True)
class LayerKeys:
  """Key names of one MoE layer (prepare_real_checkpoint_layer.py:101-178)."""

  layer_idx: int

  @property
  def prefix(self) -> str:
    return f"model.layers.{self.layer_idx}.block_sparse_moe"

  def dense(self) -> dict[str, str]:
    p = self.prefix
    return {
        "router": f"{p}.gate.weight",
        "bias": f"{p}.gate.e_score_correction_bias",
        "down": f"{p}.routed_expert_down_proj.weight",
        "up": f"{p}.routed_expert_up_proj.weight",
        "norm": f"{p}.routed_expert_norm.weight",
        "shared_gate": f"{p}.shared_experts.gate_proj.weight",
        "shared_up": f"{p}.shared_experts.up_proj.weight",
        "shared_down": f"{p}.shared_experts.down_proj.weight",
    }

  def expert(self, e: int, w: str) -> tuple[str, str]:
    """(packed, scale) keys of expert e's w1 (gate), w3 (up) or w2 (down)."""
    base = f"{self.prefix}.experts.{e}.{w}"
    return f"{base}.weight_packed", f"{base}.weight_scale"


class TensorSource:
  """Key -> tensor over one or more safetensors files (or an in-memory
  mapping), opened lazily."""

  def __init__(self, source: str | pathlib.Path | Iterable | Mapping[str, torch.Tensor]):
    self._mem = None
    self._where: dict[str, pathlib.Path] = {}
    self._handles = {}
    if isinstance(source, Mapping):
      self._mem = source
      return
    paths = [source] if isinstance(source, (str, pathlib.Path)) else list(source)
    from safetensors import safe_open
    for p in map(pathlib.Path, paths):
      if p.name.endswith(".index.json"):
        weight_map = json.loads(p.read_text())["weight_map"]
        for key, fname in weight_map.items():
          self._where[key] = p.parent / fname
        continue
      with safe_open(str(p), framework="pt") as f:
        for key in f.keys():
          self._where[key] = p

  def __contains__(self, key: str) -> bool:
    return key in (self._mem if self._mem is not None else self._where)

  def get(self, key: str) -> torch.Tensor:
    if self._mem is not None:
      if key not in self._mem:
        raise KeyError(f"checkpoint has no tensor {key!r}")
      return self._mem[key]
    if key not in self._where:
      raise KeyError(f"checkpoint has no tensor {key!r}")
    path = self._where[key]
    if path not in self._handles:
      from safetensors import safe_open
      self._handles[path] = safe_open(str(path), framework="pt")
    return self._handles[path].get_tensor(key)


def _check(name: str, t: torch.Tensor, shape: tuple, dtype: torch.dtype | None = None):
  if tuple(t.shape) != tuple(shape):
    raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")
  if dtype is not None and t.dtype != dtype:
    raise ValueError(f"{name}: dtype {t.dtype}, expected {dtype}")


def load_latent_moe_layer(source, layer_idx: int, config: LatentMoEConfig, *,
                          device: str | torch.device = "cuda",
                          dtype: torch.dtype = torch.bfloat16, expert_start: int = 0,
                          num_local_experts: int | None = None) -> PreparedWeights:
  """PreparedWeights of MoE layer `layer_idx` with MXFP4 routed experts
  [expert_start, expert_start + num_local_experts) (all experts by default).
  Dense tensors are cast to `dtype`; the router bias stays float32."""
  if layer_idx < FIRST_MOE_LAYER:
    raise ValueError(f"layer {layer_idx} is a dense MLP layer; MoE layers start at {FIRST_MOE_LAYER}")
  c = config
  d, L, I, E = c.hidden_size, c.latent_size, c.intermediate_size, c.num_experts
  si = I * c.num_shared_experts
  n_loc = E - expert_start if num_local_experts is None else num_local_experts
  if expert_start < 0 or n_loc <= 0 or expert_start + n_loc > E:
    raise ValueError(f"expert range [{expert_start}, {expert_start + n_loc}) outside [0, {E})")
  if L % 32 or I % 32:
    raise ValueError("MXFP4 needs latent and intermediate sizes divisible by 32")
  src = source if isinstance(source, TensorSource) else TensorSource(source)
  keys = LayerKeys(layer_idx)
  dk = keys.dense()
  get = lambda name: src.get(dk[name])
  shapes = {"router": (E, d), "bias": (E,), "down": (L, d), "up": (d, L), "norm": (L,),
            "shared_gate": (si, d), "shared_up": (si, d), "shared_down": (d, si)}
  dense = {}
  for name, shape in shapes.items():
    t = get(name)
    _check(dk[name], t, shape)
    dense[name] = t
  dev = torch.device(device)
  cv = lambda t: t.to(device=dev, dtype=dtype).contiguous()
  bf16 = dtype == torch.bfloat16

  def expert_pair(e: int, w: str, n: int, k: int):
    pk, sk = keys.expert(e, w)
    packed, scale = src.get(pk), src.get(sk)
    _check(pk, packed, (n, k // 2), torch.uint8)
    _check(sk, scale, (n, k // 32), torch.uint8)
    return packed, scale

  gu_p, gu_s, dn_p, dn_s = [], [], [], []
  for e in range(expert_start, expert_start + n_loc):
    p1, s1 = expert_pair(e, "w1", I, L)
    p3, s3 = expert_pair(e, "w3", I, L)
    p2, s2 = expert_pair(e, "w2", L, I)
    gu_p.append(torch.cat([p1, p3]))
    gu_s.append(torch.cat([s1, s3]))
    dn_p.append(p2)
    dn_s.append(s2)
  stack = lambda ts: torch.stack(ts).to(dev).contiguous()
  shared_gu = torch.cat([dense["shared_gate"], dense["shared_up"]])
  return PreparedWeights(
      dtype=dtype,
      router=cv(dense["router"]),
      bias=dense["bias"].to(device=dev, dtype=torch.float32).contiguous(),
      down=cv(dense["down"]),
      up=cv(dense["up"]),
      expert_gu=None, expert_gate=None, expert_up=None, expert_down=None,
      norm_scale=cv(dense["norm"]),
      shared_gu=cv(shared_gu) if bf16 else None,
      shared_gate=None if bf16 else cv(dense["shared_gate"]),
      shared_up=None if bf16 else cv(dense["shared_up"]),
      shared_down=cv(dense["shared_down"]),
      expert_gu_mx=ops.MXFP4Weights(stack(gu_p), stack(gu_s)),
      expert_down_mx=ops.MXFP4Weights(stack(dn_p), stack(dn_s)),
  )


def layer_state_dict(pw: PreparedWeights, layer_idx: int, config: LatentMoEConfig,
                     expert_start: int = 0) -> dict[str, torch.Tensor]:
  """The inverse: a prepared MXFP4 layer as checkpoint-named CPU tensors
  (for exporting synthetic layers and for round-trip tests)."""
  if pw.expert_gu_mx is None:
    raise ValueError("layer_state_dict writes MXFP4 routed experts only")
  c = config
  I = c.intermediate_size
  si = I * c.num_shared_experts
  keys = LayerKeys(layer_idx)
  dk = keys.dense()
  cpu = lambda t: t.detach().to("cpu").contiguous()
  shared_gu = pw.shared_gu if pw.shared_gu is not None else torch.cat([pw.shared_gate, pw.shared_up])
  out = {
      dk["router"]: cpu(pw.router), dk["bias"]: cpu(pw.bias), dk["down"]: cpu(pw.down),
      dk["up"]: cpu(pw.up), dk["norm"]: cpu(pw.norm_scale),
      dk["shared_gate"]: cpu(shared_gu[:si]), dk["shared_up"]: cpu(shared_gu[si:]),
      dk["shared_down"]: cpu(pw.shared_down),
  }
  gp, gs = cpu(pw.expert_gu_mx.packed), cpu(pw.expert_gu_mx.scale)
  dp, ds = cpu(pw.expert_down_mx.packed), cpu(pw.expert_down_mx.scale)
  for j in range(gp.shape[0]):
    e = expert_start + j
    for w, (p, s) in (("w1", (gp[j, :I], gs[j, :I])), ("w3", (gp[j, I:], gs[j, I:])),
                      ("w2", (dp[j], ds[j]))):
      pk, sk = keys.expert(e, w)
      out[pk], out[sk] = p.contiguous(), s.contiguous()
  return out
