"""ctypes binding of the in-tree C ABI (`include/lmoe.h`, `liblmoe_b200.so`).

There is no fallback: if the shared library is missing or fails to load, every
operator raises `NativeLibraryMissing`.  Build it with
`python -m tokamax_tpu_kernel_lab_b200.build`.
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

LIB_PATH = pathlib.Path(__file__).resolve().with_name("liblmoe_b200.so")

LMOE_OK = 0
LMOE_BAD_SHAPE = 1
LMOE_UNSUPPORTED = 2
LMOE_LAUNCH_FAILED = 3
LMOE_DEVICE_BOUNDS = 4
LMOE_WAIT_TIMEOUT = 5
LMOE_SCRATCH_TOO_SMALL = 6
LMOE_F16_RANGE = 7

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/lmoe.h one to one
SIGNATURES = {
    "lmoe_version": (_i32, []),
    "lmoe_ragged_dot_bf16": (_i32, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _p,
                                    _p]),
    "lmoe_ragged_dot_f32": (_i32, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _p, _p]),
    "lmoe_gemm_f32": (_i32, [_p, _p, _p, _p, _i64, _i64, _i64, _i32, _p, _p]),
    "lmoe_gemm_bf16": (_i32, [_p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _p, _p]),
    "lmoe_gateup_situ_bf16": (_i32, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _f32, _f32,
                                     _i32, _p, _i64, _i32, _p, _p]),
    "lmoe_mxfp4_ragged_dot": (_i32, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _i32, _i32,
                                     _p, _p]),
    "lmoe_mxfp4_gateup_situ": (_i32, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _f32, _f32,
                                      _i32, _i32, _i32, _p, _i64, _i32, _p, _p]),
    "lmoe_mxfp4_ragged_dot_scatter": (_i32, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _p,
                                             _p]),
    "lmoe_ep_return_destinations": (_i32, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _p,
                                           _p]),
    "lmoe_ep_return_signal": (_i32, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p]),
    "lmoe_fp8_ragged_dot": (_i32, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _i32,
                                   _p, _p]),
    "lmoe_situ_and_mul": (_i32, [_p, _p, _i64, _p, _i64, _i64, _f32, _f32, _i32, _p]),
    "lmoe_router_topk": (_i32, [_p, _p, _i64, _i64, _i64, _i32, _i32, _f32, _p, _p, _p]),
    "lmoe_dispatch_workspace_size": (_sz, [_i64, _i64]),
    "lmoe_router_fused_workspace_size": (_sz, [_i64, _i64, _i64]),
    "lmoe_router_fused_bf16": (_i32, [_p, _p, _p, _i64, _i64, _i64, _i64, _i32, _f32, _p, _p, _p,
                                      _sz, _p, _p]),
    "lmoe_dispatch": (_i32, [_p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _p, _p, _p, _p, _p, _p,
                             _p, _p, _sz, _p]),
    "lmoe_gather_rows": (_i32, [_p, _i64, _p, _p, _i64, _i64, _i32, _p, _p]),
    "lmoe_scatter_rows": (_i32, [_p, _p, _i64, _i64, _p, _i64, _i64, _i32, _p, _p]),
    "lmoe_combine_rmsnorm": (_i32, [_p, _p, _p, _p, _i64, _i64, _i64, _f32, _i32, _p, _p, _p]),
    "lmoe_combine_scatter_add": (_i32, [_p, _p, _p, _p, _i64, _i64, _i64, _i32, _p]),
    "lmoe_ep_reorder": (_i32, [_p, _i64, _i64, _i64, _p, _p, _p, _p]),
    "lmoe_mxfp8_padded_rows": (_i64, [_i64, _i64]),
    "lmoe_mxfp4_repack_blockscaled": (_i32, [_p, _p, _i64, _i64, _i64, _i32, _p, _p, _p]),
    "lmoe_mxfp8_quantize_rows": (_i32, [_p, _i64, _i32, _p, _p, _i64, _i64, _i64, _p, _p, _i64,
                                        _p, _p]),
    "lmoe_mxfp8_quantize_scatter": (_i32, [_p, _i32, _p, _i64, _i64, _i64, _p, _i64, _p, _p,
                                           _i64, _p, _p]),
    "lmoe_mxfp8_pad_positions": (_i32, [_p, _i64, _p, _i64, _p, _p]),
    "lmoe_mxfp8_mxfp4_grouped_gemm": (_i32, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32,
                                             _f32, _f32, _i32, _i32, _p, _p]),
    "lmoe_mxfp4_quantize_rows": (_i32, [_p, _i64, _i32, _p, _p, _i64, _i64, _i64, _p, _p, _i64,
                                        _p, _p]),
    "lmoe_mxfp4_quantize_scatter": (_i32, [_p, _i32, _p, _i64, _i64, _i64, _p, _i64, _p, _p,
                                           _i64, _p, _p]),
    "lmoe_mxfp4_mxfp4_grouped_gemm": (_i32, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32,
                                             _f32, _f32, _i32, _i32, _p, _p]),
    "lmoe_bf16split_quantize_rows": (_i32, [_p, _i64, _i32, _p, _p, _i64, _i64, _i64, _p, _p,
                                            _i64, _p, _p]),
    "lmoe_bf16split_quantize_scatter": (_i32, [_p, _i32, _p, _i64, _i64, _i64, _p, _i64, _p, _p,
                                               _i64, _p, _p]),
    "lmoe_bf16split_quantize_scatter_positions": (_i32, [_p, _i32, _p, _i64, _i64, _i64, _p, _i64,
                                                         _p, _p, _i64, _p, _p, _p]),
    "lmoe_bf16split_mxfp4_grouped_gemm": (_i32, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                                 _i32, _f32, _f32, _i32, _i32, _i64, _p, _p]),
    "lmoe_blockscaled_gateup_situ_quantized": (_i32, [_p, _p, _i32, _p, _p, _p, _i64, _i64, _i64,
                                                      _i64, _f32, _f32, _i32, _i32, _p, _p, _p,
                                                      _p]),
    "lmoe_dispatch_static_scratch": (_i32, [_p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _p, _p,
                                            _p, _p, _p, _p, _p, _p]),
    "lmoe_ep_buffer_bytes": (_i64, [_i64, _i64, _i64, _i64, _i64]),
    "lmoe_set_peer_wait_timeout_ns": (_i32, [ctypes.c_uint64]),
    "lmoe_peer_wait_timeout_ns": (ctypes.c_uint64, []),
    "lmoe_ep_region_offset": (_i64, [_i64, _i64, _i64, _i64, _i64, _i32]),
    "lmoe_ep_buffer_alloc": (_i32, [_i64, _p, _p]),
    "lmoe_ep_buffer_open": (_i32, [_p, _p]),
    "lmoe_ep_buffer_close": (_i32, [_p]),
    "lmoe_ep_buffer_free": (_i32, [_p]),
    "lmoe_ep_exchange_counts": (_i32, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p]),
    "lmoe_ep_dispatch_put": (_i32, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _p, _i64, _p,
                                    _p]),
    "lmoe_ep_return_put": (_i32, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "lmoe_dense_input_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "lmoe_dense_input_phase": (_i32, [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                      _f32, _f32, _i32, _p, _sz, _p, _p]),
    "lmoe_dense_output_workspace_size": (_sz, [_i64, _i64, _i64, _i64]),
    "lmoe_dense_output_phase": (_i32, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _sz, _p,
                                       _p]),
}

# kernels launched by one call of each entry point (for the bench's launch count)
KERNELS_PER_CALL = {"lmoe_dispatch": 3, "lmoe_ep_dispatch_put": 2, "lmoe_ep_return_put": 2,
                    "lmoe_ep_buffer_alloc": 0, "lmoe_ep_buffer_open": 0,
                    "lmoe_ep_buffer_close": 0, "lmoe_ep_buffer_free": 0,
                    "lmoe_set_peer_wait_timeout_ns": 0,
                    "lmoe_mxfp4_repack_blockscaled": 2, "lmoe_router_fused_bf16": 2}
launch_count = 0


class NativeLibraryMissing(RuntimeError):
  pass


class LmoeError(RuntimeError):
  def __init__(self, name: str, code: int):
    super().__init__(f"{name} failed with status {code}")
    self.code = code


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
  """Load liblmoe_b200.so (once) and attach the C signatures."""
  global _lib
  with _lock:
    if _lib is not None:
      return _lib
    if not LIB_PATH.exists():
      raise NativeLibraryMissing(
          f"{LIB_PATH} not found; build it with `python -m tokamax_tpu_kernel_lab_b200.build`")
    try:
      lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as e:  # pragma: no cover
      raise NativeLibraryMissing(f"cannot load {LIB_PATH}: {e}") from e
    for name, (res, args) in SIGNATURES.items():
      fn = getattr(lib, name)
      fn.restype = res
      fn.argtypes = args
    _lib = lib
    return lib


def call(name: str, *args, kernels: int | None = None) -> int:
  """Invoke an entry point; raise on a non-OK host status.  `kernels` (the
  launch count of this call, when it depends on the arguments) overrides
  KERNELS_PER_CALL.

  LMOE_UNSUPPORTED maps to NotImplementedError (the reference's error class for
  shapes an implementation does not support), LMOE_BAD_SHAPE to ValueError."""
  global launch_count
  rc = getattr(load(), name)(*args)
  if rc == LMOE_OK:
    launch_count += KERNELS_PER_CALL.get(name, 1) if kernels is None else kernels
    return rc
  if rc == LMOE_UNSUPPORTED:
    raise NotImplementedError(f"{name}: unsupported shape or alignment (status {rc})")
  if rc == LMOE_BAD_SHAPE:
    raise ValueError(f"{name}: invalid shape (status {rc})")
  raise LmoeError(name, rc)
