"""GPU test of lmoe_dispatch_static_scratch, the dispatch entry point that
allocates nothing (its scratch is a fixed array inside the library), for
callers that cannot allocate device memory where they dispatch.

Called through the C ABI and compared with lmoe_dispatch (caller-provided
workspace) on two calls in a row with different inputs -- the second call
runs on scratch the first one left behind.  Outputs are integers, so the
comparison is exact.  This file is collected last on purpose."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
  from tokamax_tpu_kernel_lab_b200 import _native
  return _native.load()


def _outputs(t, k, m_out, n_local, pad_bucket):
  dev = "cuda"
  i32 = lambda n: torch.full((n,), -7, dtype=torch.int32, device=dev)
  return {
      "order": i32(m_out), "token_idx": i32(m_out),
      "weight": torch.full((m_out,), -7.0, dtype=torch.float32, device=dev),
      "slot_pos": i32(t * k), "group_sizes": i32(n_local + (1 if pad_bucket else 0)),
      "per_expert_counts": i32(n_local),
      "valid": torch.full((m_out,), 7, dtype=torch.uint8, device=dev),
  }


def _args(o):
  p = lambda x: ctypes.c_void_p(x.data_ptr())
  return [p(o["order"]), p(o["token_idx"]), p(o["weight"]), p(o["slot_pos"]),
          p(o["group_sizes"]), p(o["per_expert_counts"]), p(o["valid"])]


def _run_pair(lib, topk, w, n_local, start, m_out, pad_bucket):
  t, k = topk.shape
  stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
  ref = _outputs(t, k, m_out, n_local, pad_bucket)
  ws_bytes = lib.lmoe_dispatch_workspace_size(max(t * k, m_out), n_local)
  ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
  rc = lib.lmoe_dispatch(ctypes.c_void_p(topk.data_ptr()), ctypes.c_void_p(w.data_ptr()), t, k,
                         start, n_local, m_out, pad_bucket, *_args(ref),
                         ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream)
  assert rc == 0
  got = _outputs(t, k, m_out, n_local, pad_bucket)
  rc = lib.lmoe_dispatch_static_scratch(ctypes.c_void_p(topk.data_ptr()),
                                        ctypes.c_void_p(w.data_ptr()), t, k, start, n_local,
                                        m_out, pad_bucket, *_args(got), stream)
  assert rc == 0
  torch.cuda.synchronize()
  for name in ref:
    assert torch.equal(ref[name], got[name]), name


def _routing(seed, t, k, e):
  rng = np.random.default_rng(seed)
  scores = rng.random((t, e)).astype(np.float32) + rng.standard_normal(e).astype(np.float32)
  topk = np.argsort(-scores, axis=1, kind="stable")[:, :k].astype(np.int32)
  w = rng.random((t, k)).astype(np.float32)
  return torch.from_numpy(topk).cuda(), torch.from_numpy(w).cuda()


def test_static_scratch_matches_workspace_dispatch_twice(lib):
  # call 1: full dropless dispatch of a 16384-token top-16 batch over 896 experts
  topk, w = _routing(1, 16384, 16, 896)
  _run_pair(lib, topk, w, 896, 0, 16384 * 16, 0)
  # call 2: a smaller, capacity-padded shard dispatch over the scratch call 1 left behind
  topk, w = _routing(2, 3000, 8, 256)
  _run_pair(lib, topk, w, 64, 128, 6144, 1)


def test_static_scratch_rejects_oversized_requests(lib):
  topk = torch.zeros(16385, 16, dtype=torch.int32, device="cuda")
  o = _outputs(16385, 16, 16385 * 16, 896, 0)
  stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
  rc = lib.lmoe_dispatch_static_scratch(ctypes.c_void_p(topk.data_ptr()), None, 16385, 16, 0, 896,
                                        16385 * 16, 0, *_args(o), stream)
  assert rc == 6  # LMOE_SCRATCH_TOO_SMALL, nothing launched
  torch.cuda.synchronize()
  assert int(o["token_idx"][0]) == -7
