"""Build the sm_100a shared library `liblmoe_b200.so` in-tree with nvcc.

    python -m tokamax_tpu_kernel_lab_b200.build [--force]

Every translation unit under csrc/ is compiled for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a`), the CUDA runtime is linked
statically, and the result lands next to this file so it travels with the
source tree.  Nothing is installed into site-packages.
"""

from __future__ import annotations

import concurrent.futures
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
LIB = HERE / "liblmoe_b200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
  for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
    if cand and os.path.exists(cand):
      return cand
  raise RuntimeError("nvcc not found")


def sources() -> list[pathlib.Path]:
  return sorted(CSRC.glob("*.cu"))


def _headers() -> list[pathlib.Path]:
  return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
  if not LIB.exists():
    return False
  t = LIB.stat().st_mtime
  return all(p.stat().st_mtime <= t for p in sources() + _headers() + [pathlib.Path(__file__)])


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
  if not force and up_to_date():
    return LIB
  nvcc = _nvcc()
  BUILD.mkdir(exist_ok=True)
  includes = ["-I", str(CSRC), "-I", str(INCLUDE)]

  def compile_one(src: pathlib.Path) -> pathlib.Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc, *NVCC_FLAGS, *includes, "-c", str(src), "-o", str(obj)]
    if verbose:
      print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
      raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj

  with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
    objs = list(ex.map(compile_one, sources()))
  tmp = LIB.with_suffix(".so.tmp")
  cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-cudart", "static",
         "-o", str(tmp), *map(str, objs)]
  res = subprocess.run(cmd, capture_output=True, text=True)
  if res.returncode != 0:
    raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
  os.replace(tmp, LIB)
  return LIB


if __name__ == "__main__":
  out = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
  print(out)
