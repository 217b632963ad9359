"""Checkpoint ingestion (CPU): the reference's key layout for one MoE layer
(06_kimi_k3_golden_validation/prepare_real_checkpoint_layer.py:101-178)
through safetensors files into the kernel layouts, and back."""

import json

import pytest
import torch
from safetensors.torch import save_file

from tokamax_tpu_kernel_lab_b200 import checkpoint as ck
from tokamax_tpu_kernel_lab_b200.latent_moe import LatentMoEConfig

CFG = LatentMoEConfig(96, 64, 32, 6, 2, 2)  # d, L, I, E, k, n_shared


def _layer(layer_idx=3, seed=0):
  g = torch.Generator().manual_seed(seed)
  c = CFG
  d, L, I, E = c.hidden_size, c.latent_size, c.intermediate_size, c.num_experts
  si = I * c.num_shared_experts
  keys = ck.LayerKeys(layer_idx)
  dk = keys.dense()
  bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)
  sd = {dk["router"]: bf(E, d), dk["bias"]: torch.randn(E, generator=g),
        dk["down"]: bf(L, d), dk["up"]: bf(d, L), dk["norm"]: bf(L),
        dk["shared_gate"]: bf(si, d), dk["shared_up"]: bf(si, d), dk["shared_down"]: bf(d, si)}
  u8 = lambda *s: torch.randint(0, 256, s, generator=g, dtype=torch.uint8)
  for e in range(E):
    for w, (n, k) in (("w1", (I, L)), ("w3", (I, L)), ("w2", (L, I))):
      pk, sk = keys.expert(e, w)
      sd[pk], sd[sk] = u8(n, k // 2), torch.randint(118, 122, (n, k // 32), generator=g,
                                                     dtype=torch.uint8)
  return sd


def test_round_trip_through_safetensors(tmp_path):
  sd = _layer()
  path = tmp_path / "layer.safetensors"
  save_file(sd, str(path))
  pw = ck.load_latent_moe_layer(path, 3, CFG, device="cpu")
  keys = ck.LayerKeys(3)
  I = CFG.intermediate_size
  assert torch.equal(pw.router, sd[keys.dense()["router"]])
  assert pw.bias.dtype == torch.float32
  assert pw.expert_gu_mx.packed.shape == (6, 2 * I, CFG.latent_size // 2)
  for e in (0, 5):
    assert torch.equal(pw.expert_gu_mx.packed[e, :I], sd[keys.expert(e, "w1")[0]])
    assert torch.equal(pw.expert_gu_mx.packed[e, I:], sd[keys.expert(e, "w3")[0]])
    assert torch.equal(pw.expert_gu_mx.scale[e, I:], sd[keys.expert(e, "w3")[1]])
    assert torch.equal(pw.expert_down_mx.packed[e], sd[keys.expert(e, "w2")[0]])
  back = ck.layer_state_dict(pw, 3, CFG)
  assert sorted(back) == sorted(sd)
  for k, v in sd.items():
    assert torch.equal(back[k], v), k


def test_expert_parallel_slice_and_sharded_index(tmp_path):
  sd = _layer(layer_idx=1, seed=1)
  names = sorted(sd)
  a, b = dict((k, sd[k]) for k in names[::2]), dict((k, sd[k]) for k in names[1::2])
  save_file(a, str(tmp_path / "part-1.safetensors"))
  save_file(b, str(tmp_path / "part-2.safetensors"))
  index = {"weight_map": {**{k: "part-1.safetensors" for k in a},
                          **{k: "part-2.safetensors" for k in b}}}
  (tmp_path / "model.safetensors.index.json").write_text(json.dumps(index))
  pw = ck.load_latent_moe_layer(tmp_path / "model.safetensors.index.json", 1, CFG,
                                device="cpu", expert_start=2, num_local_experts=3)
  keys = ck.LayerKeys(1)
  assert pw.expert_gu_mx.packed.shape[0] == 3
  assert torch.equal(pw.expert_down_mx.scale[0], sd[keys.expert(2, "w2")[1]])
  assert torch.equal(pw.expert_gu_mx.packed[2, :CFG.intermediate_size], sd[keys.expert(4, "w1")[0]])


def test_errors_name_the_problem(tmp_path):
  sd = _layer()
  with pytest.raises(ValueError, match="dense MLP layer"):
    ck.load_latent_moe_layer(sd, 0, CFG, device="cpu")
  missing = dict(sd)
  del missing[ck.LayerKeys(3).expert(4, "w3")[1]]
  with pytest.raises(KeyError, match="experts.4.w3.weight_scale"):
    ck.load_latent_moe_layer(missing, 3, CFG, device="cpu")
  bad = dict(sd)
  bad[ck.LayerKeys(3).dense()["up"]] = torch.zeros(5, 5, dtype=torch.bfloat16)
  with pytest.raises(ValueError, match="routed_expert_up_proj"):
    ck.load_latent_moe_layer(bad, 3, CFG, device="cpu")
  with pytest.raises(ValueError, match="expert range"):
    ck.load_latent_moe_layer(sd, 3, CFG, device="cpu", expert_start=5, num_local_experts=2)
