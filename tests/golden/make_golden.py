"""Re-pack the reference's six golden bundles into compact test fixtures.

The reference generated these bundles from the official PyTorch LatentMoE
block (06_kimi_k3_golden_validation/generate_pytorch_golden.py:135-356) and
checks its JAX oracle against them stage by stage
(06_kimi_k3_golden_validation/test_jax_reference_against_pytorch_golden.py).
This script reads each bundle's inputs.npz / weights.npz / golden_outputs.npz /
config.json / metadata.json and writes one `<bundle>.npz` next to itself with:

  hidden_states            (T, d) float32 (leading batch dim dropped)
  w.<field>                every `LatentMoEWeights` field in the (in, out)
                           layout of KR:217-252 (torch nn.Linear weights are
                           transposed and per-expert weights stacked, exactly
                           the mapping of the reference test's
                           `_pt_weights_to_jax`, lines 139-170)
  out.<stage>              the 18 golden intermediates (float32 / int64)
  config_json, meta_json   the bundle's own config.json / metadata.json

Weights and inputs of the bf16 bundles are bfloat16 values stored upcast;
they are written as raw bfloat16 bit patterns (uint16, key suffix `.bf16`)
to halve the fixture size.  The loader in tests/golden/__init__.py undoes it.

Run from the repository root, in a container where the reference is mounted:
    python tests/golden/make_golden.py /path/to/reference
"""

import json
import pathlib
import sys

import numpy as np

BUNDLES = (
    "golden_bundle_small",
    "golden_bundle_small_bf16",
    "golden_bundle_mosaic_fp32",
    "golden_bundle_mosaic_bf16",
    "golden_bundle_mosaic_fp32_n64",
    "golden_bundle_mosaic_bf16_n64",
)


def _bf16_bits(a: np.ndarray) -> np.ndarray:
  a = np.ascontiguousarray(a, np.float32)
  bits = a.view(np.uint32)
  if np.any(bits & 0xFFFF):
    raise ValueError("array is not bfloat16-representable")
  return (bits >> 16).astype(np.uint16)


def repack(bundle_dir: pathlib.Path, out_path: pathlib.Path) -> None:
  inputs = np.load(bundle_dir / "inputs.npz")
  w = np.load(bundle_dir / "weights.npz")
  outs = np.load(bundle_dir / "golden_outputs.npz")
  config = json.loads((bundle_dir / "config.json").read_text())
  meta = json.loads((bundle_dir / "metadata.json").read_text())
  is_bf16 = meta["dtype"].endswith("bfloat16")
  e = config["num_experts"]
  fields = {
      "router_weight": w["gate.weight"].T,
      "e_score_correction_bias": w["gate.e_score_correction_bias"],
      "down_proj": w["routed_expert_down_proj.weight"].T,
      "up_proj": w["routed_expert_up_proj.weight"].T,
      "expert_gate": np.stack([w[f"experts.{i}.w1.weight"].T for i in range(e)]),
      "expert_up": np.stack([w[f"experts.{i}.w3.weight"].T for i in range(e)]),
      "expert_down": np.stack([w[f"experts.{i}.w2.weight"].T for i in range(e)]),
      "norm_scale": w["routed_expert_norm.weight"],
      "shared_gate": w["shared_experts.gate_proj.weight"].T,
      "shared_up": w["shared_experts.up_proj.weight"].T,
      "shared_down": w["shared_experts.down_proj.weight"].T,
  }
  payload = {}
  hs = inputs["hidden_states"][0]
  if is_bf16:
    payload["hidden_states.bf16"] = _bf16_bits(hs)
  else:
    payload["hidden_states"] = hs.astype(np.float32)
  for name, arr in fields.items():
    if is_bf16:
      payload[f"w.{name}.bf16"] = _bf16_bits(arr)
    else:
      payload[f"w.{name}"] = np.ascontiguousarray(arr, np.float32)
  for name in outs.files:
    payload[f"out.{name}"] = outs[name]
  payload["config_json"] = np.frombuffer(json.dumps(config).encode(), np.uint8)
  payload["meta_json"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
  np.savez_compressed(out_path, **payload)


def main(reference_root: str) -> None:
  root = pathlib.Path(reference_root) / "06_kimi_k3_golden_validation"
  here = pathlib.Path(__file__).resolve().parent
  for b in BUNDLES:
    out = here / f"{b.replace('golden_bundle_', '')}.npz"
    repack(root / b, out)
    print(f"wrote {out} ({out.stat().st_size} bytes)")


if __name__ == "__main__":
  if len(sys.argv) != 2:
    sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
  main(sys.argv[1])
