"""CPU checks of the C-ABI library: it loads, and it exports exactly the entry
points include/lmoe.h declares (no compute calls -- there is no GPU here)."""

import ctypes
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "lmoe.h"


def declared_symbols() -> list[str]:
  text = HEADER.read_text()
  return sorted(set(re.findall(r"LMOE_API\s+\w+\s+(lmoe_\w+)\s*\(", text)))


def test_header_declares_entry_points():
  syms = declared_symbols()
  assert "lmoe_ragged_dot_bf16" in syms and "lmoe_dispatch" in syms
  assert len(syms) >= 12


def test_library_loads_and_exports_every_declared_symbol():
  from tokamax_tpu_kernel_lab_b200 import _native
  if not _native.LIB_PATH.exists():
    pytest.fail(f"{_native.LIB_PATH} is not built")
  lib = ctypes.CDLL(str(_native.LIB_PATH))
  for name in declared_symbols():
    assert hasattr(lib, name), f"{name} declared in lmoe.h but not exported"


def test_ctypes_signatures_cover_the_header():
  from tokamax_tpu_kernel_lab_b200 import _native
  assert sorted(_native.SIGNATURES) == declared_symbols()


def test_version_call_needs_no_gpu():
  from tokamax_tpu_kernel_lab_b200 import _native
  assert _native.load().lmoe_version() >= 100


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
  from tokamax_tpu_kernel_lab_b200 import _native
  monkeypatch.setattr(_native, "LIB_PATH", tmp_path / "absent.so")
  monkeypatch.setattr(_native, "_lib", None)
  with pytest.raises(_native.NativeLibraryMissing):
    _native.load()


def test_peer_wait_limit_is_a_runtime_setting():
  """The limit of the exchange's waits on other ranks is set per process
  (no GPU work: the value is read when an exchange call is enqueued)."""
  from tokamax_tpu_kernel_lab_b200 import _native
  lib = _native.load()
  default = int(lib.lmoe_peer_wait_timeout_ns())
  assert default == 2_000_000_000
  try:
    assert lib.lmoe_set_peer_wait_timeout_ns(5_000_000) == _native.LMOE_OK
    assert int(lib.lmoe_peer_wait_timeout_ns()) == 5_000_000
    assert lib.lmoe_set_peer_wait_timeout_ns(10) == _native.LMOE_BAD_SHAPE  # below 1 us
    assert lib.lmoe_set_peer_wait_timeout_ns(61 * 10**9) == _native.LMOE_BAD_SHAPE
    assert int(lib.lmoe_peer_wait_timeout_ns()) == 5_000_000
  finally:
    assert lib.lmoe_set_peer_wait_timeout_ns(0) == _native.LMOE_OK
  assert int(lib.lmoe_peer_wait_timeout_ns()) == default


def test_mxf4_gemm_checks_k_before_any_launch():
  """The MXFP4-activation grouped GEMM needs k a multiple of 256 (one 256-K
  stage of 128-byte rows); the host check answers before touching a device."""
  from tokamax_tpu_kernel_lab_b200 import _native
  lib = _native.load()
  rc = lib.lmoe_mxfp4_mxfp4_grouped_gemm(None, None, None, None, None, None, 128, 384, 128, 1, 0,
                                         0.0, 0.0, 0, 0, None, None)
  assert rc == _native.LMOE_BAD_SHAPE
  rc = lib.lmoe_mxfp4_quantize_rows(None, 0, 0, None, None, 1, 4, 200, None, None, 128, None, None)
  assert rc == _native.LMOE_BAD_SHAPE


def test_split_gemm_checks_m_out_before_any_launch():
  """|m_out| must fit 31 bits (m_out < 0 asks for the unpadded layout without
  zeroing the rows past sum(group_sizes))."""
  from tokamax_tpu_kernel_lab_b200 import _native
  lib = _native.load()
  for m_out in (1 << 31, -(1 << 31)):
    rc = lib.lmoe_bf16split_mxfp4_grouped_gemm(None, None, None, None, None, None, 128, 256, 128,
                                               1, 0, 0.0, 0.0, 0, 0, m_out, None, None)
    assert rc == _native.LMOE_BAD_SHAPE
