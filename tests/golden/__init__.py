"""Loader for the golden fixtures written by make_golden.py."""

import json
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
NAMES = ("small", "small_bf16", "mosaic_fp32", "mosaic_bf16", "mosaic_fp32_n64", "mosaic_bf16_n64")


def _from_bits(bits: np.ndarray) -> np.ndarray:
  return (bits.astype(np.uint32) << 16).view(np.float32)


def load(name: str) -> dict:
  """Returns {"hidden_states", "weights": {field: arr}, "outputs": {stage: arr},
  "config": dict, "meta": dict, "dtype": "fp32"|"bf16"} as float32 arrays."""
  z = np.load(HERE / f"{name}.npz")
  weights, outputs = {}, {}
  hidden = None
  for key in z.files:
    if key in ("config_json", "meta_json"):
      continue
    arr = z[key]
    base = key[:-5] if key.endswith(".bf16") else key
    if key.endswith(".bf16"):
      arr = _from_bits(arr)
    if base == "hidden_states":
      hidden = arr
    elif base.startswith("w."):
      weights[base[2:]] = arr
    elif base.startswith("out."):
      outputs[base[4:]] = arr
  meta = json.loads(bytes(z["meta_json"]).decode())
  return {
      "hidden_states": hidden,
      "weights": weights,
      "outputs": outputs,
      "config": json.loads(bytes(z["config_json"]).decode()),
      "meta": meta,
      "dtype": "bf16" if meta["dtype"].endswith("bfloat16") else "fp32",
  }
