"""Operator API of the LatentMoE expert path on B200 -- the drop-in for the
reference's JAX-facing operators.  Tensors are torch CUDA tensors (torch is
used only for device memory and the current stream); every computation runs
in the sm_100a kernels of `liblmoe_b200.so` through the C ABI.

Reference interfaces mirrored (paths relative to the reference project):
  ragged_dot                  tokamax.ragged_dot(lhs, rhs, group_sizes, implementation=...)
                              as called at 05_ragged_dot_on_tpu/kimi_k3_latent_moe_ragged_dot.py:358-369
  prefuse_gateup_weights      kimi_k3_latent_moe_ragged_dot.py:610-641
  fused_gateup_situ           PallasMosaicTpuV2RaggedDot()(..., fuse_gateup_activation="situ:b:lb")
                              kimi_k3_latent_moe_ragged_dot.py:644-723
  situ_and_mul                kimi_k3_latent_moe_reference.py:296-310
  router_gate                 kimi_k3_latent_moe_reference.py:347-356 / 601-631
  filter_and_pad_to_shard_jittable   kimi_k3_latent_moe_reference.py:754-877
  combine_shard_contribution  kimi_k3_latent_moe_reference.py:1113-1141
  fp8_ragged_dot / RaggedDotOp  PallasMosaicTpuV2RaggedDot()(..., rhs_scale=...)
                              kimi_k3_latent_moe_ragged_dot.py:2714-2953
"""

from __future__ import annotations

import dataclasses
import math

import torch

from . import _native

_SUPPORTED_IMPLEMENTATIONS = (None, "sm100", "b200")
_status_buffers: dict[int, torch.Tensor] = {}


def _stream() -> int:
  return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
  return None if t is None else t.data_ptr()


def _need_cuda(*ts: torch.Tensor) -> None:
  for t in ts:
    if t is not None and not t.is_cuda:
      raise ValueError("all operands must be CUDA tensors (there is no CPU path)")


def device_status(device: torch.device | int | None = None) -> torch.Tensor:
  """The per-device int32 word kernels record device-side errors into."""
  idx = torch.cuda.current_device() if device is None else torch.device("cuda", device).index \
      if isinstance(device, int) else (device.index if device.index is not None
                                       else torch.cuda.current_device())
  buf = _status_buffers.get(idx)
  if buf is None:
    buf = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
    _status_buffers[idx] = buf
  return buf


def check_device_status(device=None, reset: bool = True) -> None:
  """Synchronise and raise if a kernel recorded a device-side error."""
  buf = device_status(device)
  code = int(buf.item())
  if code != 0:
    if reset:
      buf.zero_()
    raise _native.LmoeError("device status", code)


_side_streams: dict[tuple[int, int], torch.cuda.Stream] = {}


def side_stream(device: torch.device | None = None, which: int = 0) -> torch.cuda.Stream:
  """Extra streams per device (`which` = 0, 1, ...), for work that runs beside
  the main path."""
  idx = (device.index if device is not None and device.index is not None
         else torch.cuda.current_device())
  if (idx, which) not in _side_streams:
    _side_streams[(idx, which)] = torch.cuda.Stream(device=idx)
  return _side_streams[(idx, which)]


def _check_impl(implementation):
  if implementation not in _SUPPORTED_IMPLEMENTATIONS:
    raise NotImplementedError(
        f"implementation={implementation!r}: this build has one implementation, the sm_100a kernels")


# ----------------------------------------------------------------------------- GEMMs


def _out(out: torch.Tensor | None, shape: tuple, dtype: torch.dtype, device) -> torch.Tensor:
  """The output tensor of an op: `out` when the caller passes one, else a new
  tensor.  The kernels write a dense row-major block of exactly `shape`, so
  a given `out` must be contiguous, have that shape and sit on the inputs'
  device (its dtype selects the output format where an op offers several);
  anything else raises ValueError before a kernel could write past it."""
  if out is None:
    return torch.empty(shape, dtype=dtype, device=device)
  shape = tuple(int(d) for d in shape)
  if tuple(out.shape) != shape or not out.is_contiguous() or out.device != torch.device(device):
    raise ValueError(f"out: expected a contiguous {shape} tensor on {device}, got "
                     f"{tuple(out.shape)} (contiguous={out.is_contiguous()}) on {out.device}")
  return out


def ragged_dot(lhs: torch.Tensor, rhs: torch.Tensor, group_sizes: torch.Tensor, *,
               implementation: str | None = None, precision=None,
               preferred_element_type: torch.dtype | None = None, rhs_layout: str = "gkn",
               out: torch.Tensor | None = None, zero_tail: bool = True) -> torch.Tensor:
  """out[r] = lhs[r] @ rhs[g] for the rows r of group g; rows past
  sum(group_sizes) are zero (zero_tail=False leaves them unwritten, for a
  buffer sized by capacity).  lhs (M, K); rhs (G, K, N) ("gkn", the
  reference's layout) or (G, N, K) ("gnk"); group_sizes (G,) int32 on the
  device.

  bf16 operands run on the tensor cores (f32 accumulate, bf16 or f32 out);
  f32 operands run the f32 CUDA-core kernel."""
  _check_impl(implementation)
  del precision
  _need_cuda(lhs, rhs, group_sizes)
  if lhs.dim() != 2 or rhs.dim() != 3:
    raise ValueError("lhs must be (M, K) and rhs (G, K, N) / (G, N, K)")
  layout = {"gkn": 0, "gnk": 1}[rhs_layout]
  m, k = lhs.shape
  g = rhs.shape[0]
  n = rhs.shape[2] if layout == 0 else rhs.shape[1]
  kk = rhs.shape[1] if layout == 0 else rhs.shape[2]
  if kk != k or group_sizes.shape != (g,):
    raise ValueError(f"shape mismatch lhs {tuple(lhs.shape)} rhs {tuple(rhs.shape)} "
                     f"group_sizes {tuple(group_sizes.shape)}")
  gs = group_sizes if group_sizes.dtype == torch.int32 else group_sizes.to(torch.int32)
  lhs, rhs, gs = lhs.contiguous(), rhs.contiguous(), gs.contiguous()
  status = device_status(lhs.device)
  if lhs.dtype == torch.float32:
    if rhs.dtype != torch.float32:
      raise ValueError("f32 lhs needs f32 rhs")
    res = _out(out, (m, n), torch.float32, lhs.device)
    _native.call("lmoe_ragged_dot_f32", _ptr(lhs), _ptr(rhs), _ptr(gs), _ptr(res), m, k, n, g,
                 layout, _ptr(status), _stream())
    return res
  if lhs.dtype != torch.bfloat16 or rhs.dtype != torch.bfloat16:
    raise NotImplementedError(f"dtypes {lhs.dtype}/{rhs.dtype}: bf16 or f32 operands only")
  out_dtype = preferred_element_type or torch.bfloat16
  if out_dtype not in (torch.bfloat16, torch.float32):
    raise NotImplementedError(f"preferred_element_type={out_dtype}")
  res = _out(out, (m, n), out_dtype, lhs.device)
  _native.call("lmoe_ragged_dot_bf16", _ptr(lhs), _ptr(rhs), _ptr(gs), _ptr(res), m, k, n, g,
               layout, int(out_dtype == torch.float32), int(zero_tail), _ptr(status),
               _stream())
  return res


def gemm(lhs: torch.Tensor, rhs: torch.Tensor, *, addend: torch.Tensor | None = None,
         rhs_layout: str = "nk", out_dtype: torch.dtype = torch.bfloat16,
         out: torch.Tensor | None = None) -> torch.Tensor:
  """Dense bf16 GEMM (one group of the tensor-core kernel):
  out = bf16(bf16(lhs @ W) + addend) with W given as (N, K) ("nk") or (K, N) ("kn").
  out_dtype float32 keeps the f32 accumulator; float16 stores the bf16-rounded
  result as f16."""
  _need_cuda(lhs, rhs, addend)
  layout = {"kn": 0, "nk": 1}[rhs_layout]
  m, k = lhs.shape
  n = rhs.shape[1] if layout == 0 else rhs.shape[0]
  res = _out(out, (m, n), out_dtype, lhs.device)
  code = {torch.bfloat16: 0, torch.float32: 1, torch.float16: 2}[res.dtype]
  _native.call("lmoe_gemm_bf16", _ptr(lhs), _ptr(rhs), _ptr(addend), _ptr(res), m, k, n, layout,
               code, _ptr(device_status(lhs.device)), _stream())
  return res


def prefuse_gateup_weights(expert_gate: torch.Tensor, expert_up: torch.Tensor,
                           layout: str = "gkn") -> torch.Tensor:
  """[gate | up] concatenated along N, plain, not interleaved
  (kimi_k3_latent_moe_ragged_dot.py:610-641).  Done once per weight set.
  Inputs are (G, K, I); "gnk" returns the (G, 2I, K) K-major form the
  kernels read fastest."""
  fused = torch.cat([expert_gate, expert_up], dim=-1)
  if layout == "gnk":
    fused = fused.transpose(-1, -2).contiguous()
  return fused


def fused_gateup_situ(lhs: torch.Tensor, w_gateup: torch.Tensor, group_sizes: torch.Tensor | None,
                      *, beta: float = 4.0, linear_beta: float = 25.0, round_gate_up: bool = True,
                      rhs_layout: str = "gkn", out: torch.Tensor | None = None,
                      row_index: torch.Tensor | None = None,
                      zero_tail: bool = True) -> torch.Tensor:
  """SiTU-GLU(lhs @ gate_g, lhs @ up_g) from ONE grouped matmul against the
  fused [gate | up] weight.  `group_sizes=None` means one dense group
  (the shared expert).  With `row_index` (int32, one entry per logical row)
  the dispatch gather happens inside the kernel's operand load: logical row r
  is lhs[row_index[r]] (-1 = zeros).  Returns (M, I) bf16."""
  _need_cuda(lhs, w_gateup, group_sizes, row_index)
  layout = {"gkn": 0, "gnk": 1}[rhs_layout]
  w = w_gateup if w_gateup.dim() == 3 else w_gateup.unsqueeze(0)
  src_rows, k = lhs.shape
  m = src_rows if row_index is None else row_index.shape[0]
  two_i = w.shape[2] if layout == 0 else w.shape[1]
  inter = two_i // 2
  g = w.shape[0]
  if group_sizes is not None and group_sizes.shape != (g,):
    raise ValueError("group_sizes must have one entry per weight group")
  gs = None if group_sizes is None else group_sizes.to(torch.int32).contiguous()
  ri = None if row_index is None else row_index.to(torch.int32).contiguous()
  res = _out(out, (m, inter), torch.bfloat16, lhs.device)
  _native.call("lmoe_gateup_situ_bf16", _ptr(lhs.contiguous()), _ptr(w.contiguous()), _ptr(gs),
               _ptr(res), m, k, inter, g, layout, float(beta), float(linear_beta),
               int(round_gate_up), _ptr(ri), src_rows, int(zero_tail),
               _ptr(device_status(lhs.device)), _stream())
  return res


@dataclasses.dataclass
class MXFP4Weights:
  """MXFP4 expert weights in the checkpoint's (out, in) layout:
  `packed` (G, N, K/2) uint8 e2m1 codes, low nibble = even k;
  `scale` (G, N, K/32) uint8 E8M0 exponents (2^(s-127)).
  (05_ragged_dot_on_tpu/mxfp4_dequant.py:14-20, README.md:303-318)."""

  packed: torch.Tensor
  scale: torch.Tensor
  _f16_ok: bool | None = None

  @property
  def shape(self):
    g, n, kh = self.packed.shape
    return g, n, kh * 2

  @property
  def f16_operand_ok(self) -> bool:
    """True when every scale byte lies in [104, 140], so the f16-operand
    kernel (hardware e2m1 -> f16 expansion) represents every weight exactly.
    Checked once per weight set (weights are static) and cached."""
    if self._f16_ok is None:
      lo, hi = torch.aminmax(self.scale)
      self._f16_ok = bool(int(lo) >= 104 and int(hi) <= 140)
    return self._f16_ok


def mxfp4_ragged_dot(lhs: torch.Tensor, w: MXFP4Weights, group_sizes: torch.Tensor, *,
                     preferred_element_type: torch.dtype | None = None,
                     out: torch.Tensor | None = None, zero_tail: bool = True) -> torch.Tensor:
  """lhs (M, K) @ dequant(w[g])^T per group -> (M, N); the weights stay
  packed in HBM and are expanded tile by tile in shared memory.  lhs is bf16,
  or f16 carrying bf16 values (the f16-operand kernel; needs
  w.f16_operand_ok)."""
  _need_cuda(lhs, w.packed, w.scale, group_sizes)
  g, n, k = w.shape
  m = lhs.shape[0]
  if lhs.shape[1] != k or w.scale.shape != (g, n, k // 32):
    raise ValueError("MXFP4 shape mismatch")
  lhs_f16 = lhs.dtype == torch.float16
  if lhs_f16 and not w.f16_operand_ok:
    raise NotImplementedError("f16 lhs needs MXFP4 scale bytes in [104, 140]")
  out_dtype = preferred_element_type or torch.bfloat16
  res = _out(out, (m, n), out_dtype, lhs.device)
  _native.call("lmoe_mxfp4_ragged_dot", _ptr(lhs.contiguous()), _ptr(w.packed), _ptr(w.scale),
               _ptr(group_sizes.to(torch.int32).contiguous()), _ptr(res), m, k, n, g,
               int(lhs_f16), int(out_dtype == torch.float32), int(zero_tail),
               _ptr(device_status(lhs.device)), _stream())
  return res


def mxfp4_ragged_dot_scatter(lhs: torch.Tensor, w: MXFP4Weights, group_sizes: torch.Tensor,
                             row_dest: torch.Tensor) -> None:
  """mxfp4_ragged_dot with each bf16 output row r stored at the byte address
  row_dest[r] (int64 device tensor; 16-byte aligned addresses, a peer GPU's
  mapped buffer included).  Rows past sum(group_sizes) are not written."""
  _need_cuda(lhs, w.packed, w.scale, group_sizes, row_dest)
  g, n, k = w.shape
  m = lhs.shape[0]
  if lhs.shape[1] != k or row_dest.shape[0] < m or row_dest.dtype != torch.int64:
    raise ValueError("shape mismatch")
  lhs_f16 = lhs.dtype == torch.float16
  if lhs_f16 and not w.f16_operand_ok:
    raise NotImplementedError("f16 lhs needs MXFP4 scale bytes in [104, 140]")
  _native.call("lmoe_mxfp4_ragged_dot_scatter", _ptr(lhs.contiguous()), _ptr(w.packed),
               _ptr(w.scale), _ptr(group_sizes.to(torch.int32).contiguous()), _ptr(row_dest), m, k,
               n, g, int(lhs_f16), _ptr(device_status(lhs.device)), _stream())


def mxfp4_fused_gateup_situ(lhs: torch.Tensor, w_gateup: MXFP4Weights,
                            group_sizes: torch.Tensor | None, *, beta: float = 4.0,
                            linear_beta: float = 25.0, round_gate_up: bool = True,
                            out_dtype: torch.dtype = torch.bfloat16,
                            out: torch.Tensor | None = None,
                            row_index: torch.Tensor | None = None,
                            zero_tail: bool = True) -> torch.Tensor:
  """SiTU-GLU of one grouped matmul against MXFP4 [gate rows | up rows].
  lhs bf16, or f16 carrying bf16 values; out_dtype=torch.float16 stores the
  bf16-rounded activation as f16 (the lhs of an f16 down-projection).
  `row_index` fuses the dispatch gather into the operand load (see
  fused_gateup_situ)."""
  _need_cuda(lhs, w_gateup.packed, w_gateup.scale, group_sizes, row_index)
  g, two_i, k = w_gateup.shape
  inter = two_i // 2
  src_rows = lhs.shape[0]
  m = src_rows if row_index is None else row_index.shape[0]
  lhs_f16 = lhs.dtype == torch.float16
  if lhs_f16 and not w_gateup.f16_operand_ok:
    raise NotImplementedError("f16 lhs needs MXFP4 scale bytes in [104, 140]")
  gs = None if group_sizes is None else group_sizes.to(torch.int32).contiguous()
  ri = None if row_index is None else row_index.to(torch.int32).contiguous()
  res = _out(out, (m, inter), out_dtype, lhs.device)
  _native.call("lmoe_mxfp4_gateup_situ", _ptr(lhs.contiguous()), _ptr(w_gateup.packed),
               _ptr(w_gateup.scale), _ptr(gs), _ptr(res), m, k, inter, g, float(beta),
               float(linear_beta), int(round_gate_up), int(lhs_f16),
               int(res.dtype == torch.float16), _ptr(ri), src_rows, int(zero_tail),
               _ptr(device_status(lhs.device)), _stream())
  return res


def fp8_ragged_dot(lhs: torch.Tensor, rhs: torch.Tensor, group_sizes: torch.Tensor,
                   rhs_scale: torch.Tensor, *, preferred_element_type: torch.dtype | None = None,
                   out: torch.Tensor | None = None, zero_tail: bool = True) -> torch.Tensor:
  """lhs (M, K) bf16 @ bf16(f32(rhs[g]) * rhs_scale[g]) per group, with rhs
  (G, K, N) float8_e4m3fn and rhs_scale (G, K / block, 1, N) (or (G, K / block,
  N)) float32 -- the quantised-weight form of PallasMosaicTpuV2RaggedDot
  (kimi_k3_latent_moe_ragged_dot.py:2804-2811).  The e4m3 tiles are expanded
  to the dequantised bf16 weight inside the kernel."""
  _need_cuda(lhs, rhs, group_sizes, rhs_scale)
  if lhs.dtype != torch.bfloat16:
    raise NotImplementedError(f"lhs dtype {lhs.dtype}: bf16 only")
  if rhs.dtype not in (torch.float8_e4m3fn, torch.uint8):
    raise NotImplementedError(f"rhs dtype {rhs.dtype}: float8_e4m3fn only")
  g, k, n = rhs.shape
  m = lhs.shape[0]
  if lhs.shape[1] != k or group_sizes.shape != (g,):
    raise ValueError("shape mismatch")
  scale = rhs_scale.reshape(g, -1, n) if rhs_scale.dim() == 4 else rhs_scale
  if scale.dim() != 3 or scale.shape[0] != g or scale.shape[2] != n or k % scale.shape[1]:
    raise ValueError(f"rhs_scale shape {tuple(rhs_scale.shape)} does not match rhs {tuple(rhs.shape)}")
  if scale.dtype != torch.float32:
    raise NotImplementedError("rhs_scale must be float32")
  block = k // scale.shape[1]
  out_dtype = preferred_element_type or torch.bfloat16
  res = _out(out, (m, n), out_dtype, lhs.device)
  _native.call("lmoe_fp8_ragged_dot", _ptr(lhs.contiguous()), _ptr(rhs.contiguous()),
               _ptr(scale.contiguous()), _ptr(group_sizes.to(torch.int32).contiguous()),
               _ptr(res), m, k, n, g, block, int(res.dtype == torch.float32), int(zero_tail),
               _ptr(device_status(lhs.device)), _stream())
  return res


class RaggedDotOp:
  """Instance-call form of the grouped matmul, mirroring
  `PallasMosaicTpuV2RaggedDot()(lhs, rhs, *, group_sizes, rhs_scale=None,
  fuse_gateup_activation=None, maybe_quantize_lhs=False)`
  (kimi_k3_latent_moe_ragged_dot.py:257-263, 713-723, 2804-2811): the keyword
  arguments the public ragged_dot does not take."""

  def __call__(self, lhs: torch.Tensor, rhs: torch.Tensor, *, group_sizes: torch.Tensor,
               rhs_scale: torch.Tensor | None = None, fuse_gateup_activation: str | None = None,
               maybe_quantize_lhs: bool = False, preferred_element_type=None) -> torch.Tensor:
    if maybe_quantize_lhs:
      raise NotImplementedError("maybe_quantize_lhs=True: activations stay bf16 on this path")
    if rhs_scale is not None:
      if fuse_gateup_activation is not None:
        raise NotImplementedError("fused activation with quantised weights")
      return fp8_ragged_dot(lhs, rhs, group_sizes, rhs_scale,
                            preferred_element_type=preferred_element_type)
    if fuse_gateup_activation is not None:
      beta, linear_beta = parse_fused_activation(fuse_gateup_activation)
      return fused_gateup_situ(lhs, rhs, group_sizes, beta=beta, linear_beta=linear_beta,
                               round_gate_up=False)
    return ragged_dot(lhs, rhs, group_sizes, preferred_element_type=preferred_element_type)


def parse_fused_activation(spec: str) -> tuple[float, float]:
  """"situ:<beta>:<linear_beta>" (kimi_k3_latent_moe_ragged_dot.py:718)."""
  parts = spec.split(":")
  if len(parts) != 3 or parts[0] != "situ":
    raise NotImplementedError(f"fused activation {spec!r}")
  return float(parts[1]), float(parts[2])


def situ_and_mul(gate: torch.Tensor, up: torch.Tensor, beta: float = 4.0,
                 linear_beta: float = 25.0) -> torch.Tensor:
  """Elementwise SiTU-GLU in f32, cast back to the input dtype."""
  _need_cuda(gate, up)
  if gate.shape != up.shape or gate.dtype != up.dtype:
    raise ValueError("gate/up mismatch")
  g2, u2 = gate.reshape(-1, gate.shape[-1]).contiguous(), up.reshape(-1, up.shape[-1]).contiguous()
  out = torch.empty_like(g2)
  _native.call("lmoe_situ_and_mul", _ptr(g2), _ptr(u2), g2.shape[1], _ptr(out), g2.shape[0],
               g2.shape[1], float(beta), float(linear_beta), int(gate.dtype == torch.bfloat16),
               _stream())
  return out.reshape(gate.shape)


# ----------------------------------------------------------------------------- routing


def router_topk(logits: torch.Tensor, bias: torch.Tensor | None, top_k: int, *,
                renormalize: bool = True, routed_scaling_factor: float = 1.0,
                activation: str = "sigmoid") -> tuple[torch.Tensor, torch.Tensor]:
  """Gate math of kimi_k3_latent_moe_reference.py:348-356 from f32 logits:
  returns (topk_idx int32 (T, k), topk_weight f32 (T, k))."""
  _need_cuda(logits, bias)
  logits = logits.float().contiguous()
  t, e = logits.shape
  b = None if bias is None else bias.float().contiguous()
  idx = torch.empty(t, top_k, dtype=torch.int32, device=logits.device)
  w = torch.empty(t, top_k, dtype=torch.float32, device=logits.device)
  act = {"sigmoid": 0, "softmax": 1}[activation]
  _native.call("lmoe_router_topk", _ptr(logits), _ptr(b), t, e, top_k, act, int(renormalize),
               float(routed_scaling_factor), _ptr(idx), _ptr(w), _stream())
  return idx, w


def router_logits(hidden_states: torch.Tensor, router_weight_nk: torch.Tensor) -> torch.Tensor:
  """f32 logits = h @ W_router.  bf16 h and W: tensor cores, exact bf16
  products, f32 accumulation.  f32 h and W: the f32 CUDA-core kernel.
  `router_weight_nk` is (E, d)."""
  if hidden_states.dtype == torch.float32:
    gs = torch.tensor([hidden_states.shape[0]], dtype=torch.int32, device=hidden_states.device)
    return ragged_dot(hidden_states, router_weight_nk.unsqueeze(0), gs, rhs_layout="gnk")
  return gemm(hidden_states, router_weight_nk, rhs_layout="nk", out_dtype=torch.float32)


def router_fused_supported(hidden_states: torch.Tensor, router_weight_nk: torch.Tensor,
                           top_k: int, activation: str = "sigmoid") -> bool:
  """True when router_gate can run the fused kernel: sigmoid activation, bf16
  hidden states and router weight, E <= 1024, top_k <= 16, d % 8 == 0."""
  e, d = router_weight_nk.shape
  return (activation == "sigmoid" and hidden_states.dtype == torch.bfloat16
          and router_weight_nk.dtype == torch.bfloat16 and 0 < top_k <= 16 and top_k <= e <= 1024
          and d % 8 == 0 and hidden_states.shape[-1] == d)


def router_fused_workspace_size(num_tokens: int, num_experts: int, top_k: int) -> int:
  return int(_native.load().lmoe_router_fused_workspace_size(num_tokens, num_experts, top_k))


def router_gate_fused(hidden_states: torch.Tensor, router_weight_nk: torch.Tensor,
                      bias: torch.Tensor | None, top_k: int, *, renormalize: bool = True,
                      routed_scaling_factor: float = 1.0,
                      workspace: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
  """The gate of kimi_k3_latent_moe_reference.py:347-356 straight from bf16
  hidden states (sigmoid): the logits GEMM runs on the tensor cores with the
  top-k selection in its epilogue, so the f32 logits are never stored.
  Returns the same bits as router_topk(router_logits(h, W), ...)."""
  _need_cuda(hidden_states, router_weight_nk, bias)
  h = hidden_states.contiguous()
  w = router_weight_nk.contiguous()
  t, d = h.shape
  e = w.shape[0]
  b = None if bias is None else bias.float().contiguous()
  idx = torch.empty(t, top_k, dtype=torch.int32, device=h.device)
  tw = torch.empty(t, top_k, dtype=torch.float32, device=h.device)
  ws_bytes = router_fused_workspace_size(t, e, top_k)
  if workspace is None or workspace.numel() < ws_bytes:
    workspace = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=h.device)
  _native.call("lmoe_router_fused_bf16", _ptr(h), _ptr(w), _ptr(b), t, d, e, top_k,
               int(renormalize), float(routed_scaling_factor), _ptr(idx), _ptr(tw),
               _ptr(workspace), workspace.numel(), _ptr(device_status(h.device)), _stream())
  return idx, tw


def dense_phases_pay_off(num_tokens: int, num_experts: int, latent_size: int,
                         shared_intermediate: int, device=None, sms: int | None = None) -> bool:
  """True when the layer's dense projections should run as the split-K phase
  kernels: their output tiles (128 tokens x 128 columns) would fill the SMs
  at most twice over, so the separate GEMMs (and the fused router, whose
  CTAs each run a K loop over d) would leave SMs idle or run few waves of
  long serial K loops.  Measured at configuration 5 (graph replay): 128
  tokens 0.253 vs 0.284 ms, 512 tokens 0.390 vs 0.396 ms, and at 1024 tokens
  (above the rule) 0.569 vs 0.542 ms."""
  if sms is None:
    sms = torch.cuda.get_device_properties(device).multi_processor_count
  m_tiles = -(-num_tokens // 128)
  n_tiles = -(-num_experts // 128) + -(-latent_size // 128) + -(-shared_intermediate // 64)
  return 0 < m_tiles * n_tiles <= 2 * sms


def dense_input_phase(hidden_states: torch.Tensor, router_weight_nk: torch.Tensor,
                      down_weight_nk: torch.Tensor, shared_gu_nk: torch.Tensor, *,
                      beta: float = 4.0, linear_beta: float = 25.0, round_gate_up: bool = True,
                      workspace: torch.Tensor | None = None):
  """The layer's input phase in one persistent split-K kernel
  (kimi_k3_latent_moe_reference.py:347-365, 428-433): router logits
  h @ Wr^T (f32), the latent rows bf16(h @ Wd^T) and the shared expert's
  SiTU-GLU activation from the fused [gate | up] weight (2 Is, d).  Weights
  are (N, K) with K contiguous.  Returns (logits, latent, shared_act)."""
  _need_cuda(hidden_states, router_weight_nk, down_weight_nk, shared_gu_nk)
  h = hidden_states.contiguous()
  if h.dtype != torch.bfloat16:
    raise NotImplementedError("the dense phase kernels take bf16 hidden states")
  t, d = h.shape
  e, latent, si = router_weight_nk.shape[0], down_weight_nk.shape[0], shared_gu_nk.shape[0] // 2
  for w in (router_weight_nk, down_weight_nk, shared_gu_nk):
    if w.dim() != 2 or w.shape[1] != d or w.dtype != torch.bfloat16:
      raise ValueError("weights must be bf16 (N, d) matrices")
  logits = torch.empty(t, e, dtype=torch.float32, device=h.device)
  x = torch.empty(t, latent, dtype=torch.bfloat16, device=h.device)
  act = torch.empty(t, si, dtype=torch.bfloat16, device=h.device)
  ws = int(_native.load().lmoe_dense_input_workspace_size(t, d, e, latent, si))
  if ws == 0:
    raise NotImplementedError(f"dense input phase: unsupported shape t={t} d={d} e={e} "
                              f"latent={latent} shared={si}")
  if workspace is None or workspace.numel() < ws:
    workspace = torch.empty(ws, dtype=torch.uint8, device=h.device)
  _native.call("lmoe_dense_input_phase", _ptr(h), _ptr(router_weight_nk.contiguous()),
               _ptr(down_weight_nk.contiguous()), _ptr(shared_gu_nk.contiguous()), _ptr(logits),
               _ptr(x), _ptr(act), t, d, e, latent, si, float(beta), float(linear_beta),
               int(round_gate_up), _ptr(workspace), workspace.numel(),
               _ptr(device_status(h.device)), _stream())
  return logits, x, act


def dense_output_phase(normed: torch.Tensor, up_weight_nk: torch.Tensor, shared_act: torch.Tensor,
                       shared_down_nk: torch.Tensor, *, workspace: torch.Tensor | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
  """The layer's output phase in one persistent split-K kernel
  (kimi_k3_latent_moe_reference.py:419-435): bf16(normed @ Wup^T +
  shared_act @ Wsd^T), the up-projection, the shared expert's down
  projection and the output sum, the f32 sum rounded once."""
  _need_cuda(normed, up_weight_nk, shared_act, shared_down_nk)
  a0, a1 = normed.contiguous(), shared_act.contiguous()
  t, latent = a0.shape
  si = a1.shape[1]
  d = up_weight_nk.shape[0]
  if (a1.shape[0] != t or up_weight_nk.shape != (d, latent) or
      tuple(shared_down_nk.shape) != (d, si)):
    raise ValueError("shape mismatch in the dense output phase")
  res = _out(out, (t, d), torch.bfloat16, a0.device)
  ws = int(_native.load().lmoe_dense_output_workspace_size(t, latent, si, d))
  if ws == 0:
    raise NotImplementedError(f"dense output phase: unsupported shape t={t} latent={latent} "
                              f"shared={si} d={d}")
  if workspace is None or workspace.numel() < ws:
    workspace = torch.empty(ws, dtype=torch.uint8, device=a0.device)
  _native.call("lmoe_dense_output_phase", _ptr(a0), _ptr(up_weight_nk.contiguous()), _ptr(a1),
               _ptr(shared_down_nk.contiguous()), _ptr(res), t, latent, si, d, _ptr(workspace),
               workspace.numel(), _ptr(device_status(a0.device)), _stream())
  return res


def router_gate(hidden_states, router_weight_nk, bias, top_k, *, renormalize=True,
                routed_scaling_factor=1.0, activation="sigmoid", fused: bool | None = None):
  """(topk_idx, topk_weight f32) on the original hidden states.  fused=None
  takes the fused logits+selection kernel whenever router_fused_supported
  allows it (the results are the same bits either way)."""
  if fused is None:
    fused = router_fused_supported(hidden_states, router_weight_nk, top_k, activation)
  if fused:
    return router_gate_fused(hidden_states, router_weight_nk, bias, top_k,
                             renormalize=renormalize, routed_scaling_factor=routed_scaling_factor)
  logits = router_logits(hidden_states, router_weight_nk)
  return router_topk(logits, bias, top_k, renormalize=renormalize,
                     routed_scaling_factor=routed_scaling_factor, activation=activation)


@dataclasses.dataclass
class Dispatch:
  """Device outputs of the dispatch kernels."""

  order: torch.Tensor | None       # (m_out,) flat (token*k+slot) entry at each sorted position
  token_idx: torch.Tensor          # (m_out,) source token, -1 for padding
  weight: torch.Tensor | None      # (m_out,) f32 combine weight, 0 for padding
  slot_pos: torch.Tensor | None    # (T*k,) sorted position of each entry, -1 if not kept
  group_sizes: torch.Tensor        # (E_local [+1],) int32
  per_expert_counts: torch.Tensor | None
  valid: torch.Tensor | None       # (m_out,) bool


def dispatch_workspace_size(num_entries: int, num_local_experts: int) -> int:
  return int(_native.load().lmoe_dispatch_workspace_size(num_entries, num_local_experts))


def dispatch(topk_idx: torch.Tensor, topk_weight: torch.Tensor | None, num_local_experts: int, *,
             expert_start: int = 0, m_out: int | None = None, pad_bucket: bool = False,
             want_order: bool = True, want_slot_pos: bool = True, want_valid: bool = False,
             workspace: torch.Tensor | None = None) -> Dispatch:
  """Stable counting sort of the (token, slot) entries by local expert id
  (argsort + bincount of kimi_k3_latent_moe_reference.py:370-378; with
  expert_start / m_out / pad_bucket the shard form of 754-877)."""
  _need_cuda(topk_idx, topk_weight)
  t, k = topk_idx.shape
  s = t * k
  m_out = s if m_out is None else int(m_out)
  dev = topk_idx.device
  ids = topk_idx.to(torch.int32).contiguous()
  w = None if topk_weight is None else topk_weight.float().contiguous()
  n_ext = max(s, m_out)
  ws_bytes = dispatch_workspace_size(n_ext, num_local_experts)
  if workspace is None or workspace.numel() < ws_bytes:
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
  i32 = lambda n: torch.empty(n, dtype=torch.int32, device=dev)
  res = Dispatch(
      order=i32(m_out) if want_order else None,
      token_idx=i32(m_out),
      weight=torch.empty(m_out, dtype=torch.float32, device=dev) if w is not None else None,
      slot_pos=i32(s) if want_slot_pos else None,
      group_sizes=i32(num_local_experts + (1 if pad_bucket else 0)),
      per_expert_counts=i32(num_local_experts) if pad_bucket else None,
      valid=torch.empty(m_out, dtype=torch.uint8, device=dev) if want_valid else None,
  )
  _native.call("lmoe_dispatch", _ptr(ids), _ptr(w), t, k, expert_start, num_local_experts, m_out,
               int(pad_bucket), _ptr(res.order), _ptr(res.token_idx), _ptr(res.weight),
               _ptr(res.slot_pos), _ptr(res.group_sizes), _ptr(res.per_expert_counts),
               _ptr(res.valid), _ptr(workspace), workspace.numel(), _stream(),
               kernels=0 if n_ext == 0 else (1 if n_ext <= 2048 else 3))  # fused: one chunk
  if res.valid is not None:
    res.valid = res.valid.view(torch.bool)
  return res


def gather_rows(x: torch.Tensor, token_idx: torch.Tensor, out: torch.Tensor | None = None,
                to_f16: bool = False):
  """out[p] = x[token_idx[p]] (zero where token_idx < 0); to_f16 converts bf16
  rows to f16 on the way (exact in f16's normal range; a magnitude above 65504
  becomes inf and records LMOE_F16_RANGE in the device status word)."""
  _need_cuda(x, token_idx)
  x = x.contiguous()
  rows = token_idx.shape[0]
  if to_f16 and x.dtype != torch.bfloat16:
    raise ValueError("to_f16 converts bf16 rows")
  dt = torch.float16 if to_f16 else x.dtype
  res = _out(out, (rows, x.shape[1]), dt, x.device)
  _native.call("lmoe_gather_rows", _ptr(x), x.shape[0], _ptr(token_idx.to(torch.int32)),
               _ptr(res), rows, x.shape[1] * x.element_size(), int(to_f16),
               _ptr(device_status(x.device)), _stream())
  return res


def scatter_rows(x: torch.Tensor, slot_pos: torch.Tensor, top_k: int, out_rows: int | None = None,
                 out: torch.Tensor | None = None, to_f16: bool = False):
  """The dropless gather in token order: out[slot_pos[t*k + s]] = x[t].  Each
  source row is read (and converted, to_f16 as in gather_rows) once; for a
  dropless dispatch the result equals gather_rows(x, token_idx) bit for bit.
  Rows no slot points at are left as they were (uninitialised when `out` is
  allocated here)."""
  _need_cuda(x, slot_pos)
  x = x.contiguous()
  t = x.shape[0]
  rows = t * top_k if out_rows is None else int(out_rows)
  if to_f16 and x.dtype != torch.bfloat16:
    raise ValueError("to_f16 converts bf16 rows")
  dt = torch.float16 if to_f16 else x.dtype
  res = _out(out, (rows, x.shape[1]), dt, x.device)
  _native.call("lmoe_scatter_rows", _ptr(x), _ptr(slot_pos.to(torch.int32).contiguous()), t, top_k,
               _ptr(res), res.shape[0], x.shape[1] * x.element_size(), int(to_f16),
               _ptr(device_status(x.device)), _stream())
  return res


def shard_m_padded(num_tokens, top_k, num_experts, local_num_experts, capacity_factor, tile_size):
  """kimi_k3_latent_moe_reference.py:825-826."""
  expected_total = num_tokens * top_k * local_num_experts / num_experts
  v = math.ceil(expected_total * capacity_factor)
  return -(-v // tile_size) * tile_size


def filter_and_pad_to_shard_jittable(topk_idx, topk_weight, x, num_experts, top_k,
                                     local_expert_start, local_num_experts,
                                     capacity_factor=2.0, tile_size=128):
  """Static-shape shard dispatch (kimi_k3_latent_moe_reference.py:754-877).
  Returns (sorted_tokens, group_sizes, valid_mask, per_expert_counts,
  padded_token_idx, padded_combine_weight)."""
  t = topk_idx.shape[0]
  m_padded = shard_m_padded(t, top_k, num_experts, local_num_experts, capacity_factor, tile_size)
  d = dispatch(topk_idx, topk_weight, local_num_experts, expert_start=local_expert_start,
               m_out=m_padded, pad_bucket=True, want_order=False, want_slot_pos=False,
               want_valid=True)
  sorted_tokens = gather_rows(x, d.token_idx)
  return sorted_tokens, d.group_sizes, d.valid, d.per_expert_counts, d.token_idx, d.weight


def combine_rmsnorm(expert_out: torch.Tensor, slot_pos: torch.Tensor, topk_weight: torch.Tensor,
                    norm_scale: torch.Tensor, eps: float, *, want_routed: bool = False):
  """routed = dtype(sum_s out[slot_pos] * w) (f32, slot order) and its RMSNorm.
  Returns normed, or (routed, normed) with want_routed."""
  _need_cuda(expert_out, slot_pos, topk_weight, norm_scale)
  t, k = topk_weight.shape
  L = expert_out.shape[1]
  bf16 = expert_out.dtype == torch.bfloat16
  normed = torch.empty(t, L, dtype=expert_out.dtype, device=expert_out.device)
  routed = torch.empty_like(normed) if want_routed else None
  _native.call("lmoe_combine_rmsnorm", _ptr(expert_out.contiguous()), _ptr(slot_pos),
               _ptr(topk_weight.float().contiguous()), _ptr(norm_scale.to(expert_out.dtype)),
               t, k, L, float(eps), int(bf16), _ptr(routed), _ptr(normed), _stream())
  return (routed, normed) if want_routed else normed


def combine_shard_contribution(routed_out: torch.Tensor, shard_out: torch.Tensor,
                               padded_token_idx: torch.Tensor,
                               padded_combine_weight: torch.Tensor) -> torch.Tensor:
  """routed_out.at[idx].add((shard_out * w).astype(routed_out.dtype)) as a
  scatter-add kernel (in place on a copy of routed_out, which is returned)."""
  _need_cuda(routed_out, shard_out, padded_token_idx, padded_combine_weight)
  out = routed_out.clone()
  rows, L = shard_out.shape
  _native.call("lmoe_combine_scatter_add", _ptr(shard_out.to(out.dtype).contiguous()),
               _ptr(padded_token_idx.to(torch.int32).contiguous()),
               _ptr(padded_combine_weight.float().contiguous()), _ptr(out), rows, L,
               out.shape[0], int(out.dtype == torch.bfloat16), _stream())
  return out


# ----------------------------------------------------------------------------- MXFP8 x MXFP4
# The block-scaled fast path (opt-in): activations rounded to MXFP8 (e4m3, one
# E8M0 scale per 32 K values), MXFP4 weights fed to the block-scaled tensor
# core as they are.  Rows live in a padded layout where every group starts at
# a multiple of 128; scales live in 512-byte atoms of 128 rows x 4 K blocks.


@dataclasses.dataclass
class MXFP4BlockScaled:
  """MXFP4 weights prepared for the block-scaled MMA: codes (G, N, K/2)
  (gate/up rows interleaved when `gateup`), scale atoms (G, N/128, K/128, 512)."""

  packed: torch.Tensor
  sf: torch.Tensor
  gateup: bool

  @property
  def shape(self):
    g, n, kh = self.packed.shape
    return g, n, kh * 2


def prepare_mxfp4_blockscaled(w: MXFP4Weights, gateup: bool = False) -> MXFP4BlockScaled:
  """One-time repack of MXFP4 weights (G, N, K/2) codes + (G, N, K/32) scales;
  `gateup` marks a fused [gate | up] weight (N = 2I) whose rows are then
  interleaved so each (gate, up) pair meets in adjacent accumulator lanes."""
  _need_cuda(w.packed, w.scale)
  g, n, k = w.shape
  sf = torch.empty(g, n // 128, k // 128, 512, dtype=torch.uint8, device=w.packed.device)
  packed = torch.empty_like(w.packed) if gateup else w.packed
  _native.call("lmoe_mxfp4_repack_blockscaled", _ptr(w.packed.contiguous()),
               _ptr(w.scale.contiguous()), g, n, k, int(gateup), _ptr(packed) if gateup else None,
               _ptr(sf), _stream())
  return MXFP4BlockScaled(packed, sf, gateup)


@dataclasses.dataclass
class MXFP8Rows:
  """Activation rows quantised to MXFP8 in the padded layout: q (M_pad, K)
  e4m3 bytes, sf (K/128, M_pad/128, 512) scale atoms, group_sizes (G,) the
  true row counts (group g's rows start at the sum of the earlier groups'
  counts rounded up to 128)."""

  q: torch.Tensor
  sf: torch.Tensor
  group_sizes: torch.Tensor


@dataclasses.dataclass
class MXFP4Rows:
  """Activation rows quantised to MXFP4 in the same padded layout: q (M_pad,
  K/2) bytes of e2m1 pairs (the even K index in the low nibble), sf and
  group_sizes as in MXFP8Rows."""

  q: torch.Tensor
  sf: torch.Tensor
  group_sizes: torch.Tensor


@dataclasses.dataclass
class SplitRows:
  """bf16/f16 activation rows split into two e4m3 planes under one E8M0 scale
  per 32 K values, in the padded layout: q (2, M_pad, K) (plane 0 hi =
  e4m3(x / 2^e), plane 1 lo = e4m3(x / 2^e - hi)), sf and group_sizes as in
  MXFP8Rows.  hi + lo carries the rows' bf16 values (see quantize_split_rows)."""

  q: torch.Tensor
  sf: torch.Tensor
  group_sizes: torch.Tensor


_MX_FORMATS = {  # element format -> (rows class, K values per byte, quantising C entry points)
    "e4m3": (MXFP8Rows, 1, "lmoe_mxfp8_quantize_rows", "lmoe_mxfp8_quantize_scatter"),
    "e2m1": (MXFP4Rows, 2, "lmoe_mxfp4_quantize_rows", "lmoe_mxfp4_quantize_scatter"),
    "e4m3x2": (SplitRows, 1, "lmoe_bf16split_quantize_rows", "lmoe_bf16split_quantize_scatter"),
}


def mxfp8_padded_rows(num_rows: int, num_groups: int) -> int:
  return int(_native.load().lmoe_mxfp8_padded_rows(num_rows, num_groups))


def _mx_rows(fmt: str, m_pad: int, k: int, group_sizes: torch.Tensor, device):
  cls, k_per_byte, _, _ = _MX_FORMATS[fmt]
  planes = (2,) if cls is SplitRows else ()
  return cls(torch.empty(*planes, m_pad, k // k_per_byte, dtype=torch.uint8, device=device),
             torch.empty(k // 128, m_pad // 128, 512, dtype=torch.uint8, device=device),
             group_sizes)


def _check_mx_rows(out, fmt: str, m_pad: int, k: int):
  """A caller's block-scaled row buffer must be the one _mx_rows(fmt, m_pad,
  k, ...) would allocate (codes and scale atoms of exactly those shapes), so
  no kernel writes past it."""
  cls, k_per_byte, _, _ = _MX_FORMATS[fmt]
  planes = (2,) if cls is SplitRows else ()
  want_q, want_sf = (*planes, m_pad, k // k_per_byte), (k // 128, m_pad // 128, 512)
  if (type(out) is not cls or tuple(out.q.shape) != want_q or tuple(out.sf.shape) != want_sf or
      not out.q.is_contiguous() or not out.sf.is_contiguous()):
    raise ValueError(f"out: expected {cls.__name__} with codes {want_q} and scale atoms {want_sf}, "
                     f"got {type(out).__name__} {tuple(out.q.shape)} / {tuple(out.sf.shape)}")


def _quantize_rows(fmt, x, group_sizes, token_idx, padded_input, out):
  _need_cuda(x, group_sizes, token_idx)
  rows = token_idx.shape[0] if token_idx is not None else x.shape[0]
  k = x.shape[1]
  g = group_sizes.shape[0]
  m_pad = x.shape[0] if padded_input else mxfp8_padded_rows(rows, g)
  if out is None:
    out = _mx_rows(fmt, m_pad, k, group_sizes, x.device)
  else:
    _check_mx_rows(out, fmt, m_pad, k)
  gs = group_sizes.to(torch.int32).contiguous()
  out.group_sizes = gs
  ti = None if token_idx is None else token_idx.to(torch.int32).contiguous()
  _native.call(_MX_FORMATS[fmt][2], _ptr(x.contiguous()), x.shape[0],
               int(x.dtype == torch.float16), _ptr(ti), None if padded_input else _ptr(gs), g,
               rows, k, _ptr(out.q), _ptr(out.sf), out.q.shape[-2], _ptr(device_status(x.device)),
               _stream())
  return out


def _quantize_scatter(fmt, x, group_sizes, slot_pos, top_k, out):
  _need_cuda(x, group_sizes, slot_pos)
  t, k = x.shape
  g = group_sizes.shape[0]
  if out is None:
    out = _mx_rows(fmt, mxfp8_padded_rows(t * top_k, g), k, group_sizes, x.device)
  else:
    _check_mx_rows(out, fmt, mxfp8_padded_rows(t * top_k, g), k)
  gs = group_sizes.to(torch.int32).contiguous()
  out.group_sizes = gs
  _native.call(_MX_FORMATS[fmt][3], _ptr(x.contiguous()), int(x.dtype == torch.float16),
               _ptr(slot_pos.to(torch.int32).contiguous()), t, top_k, k, _ptr(gs), g, _ptr(out.q),
               _ptr(out.sf), out.q.shape[-2], _ptr(device_status(x.device)), _stream())
  return out


def quantize_mxfp8_rows(x: torch.Tensor, group_sizes: torch.Tensor,
                        token_idx: torch.Tensor | None = None, *, padded_input: bool = False,
                        out: MXFP8Rows | None = None) -> MXFP8Rows:
  """Rows x[token_idx[p]] (or x[p]) quantised to MXFP8 and placed in the
  padded layout of `group_sizes` (the gather, the quantisation and the
  padding in one kernel).  With padded_input=True, x is already in that
  layout (the padded output of an earlier block-scaled GEMM) and every row
  keeps its position.  x bf16 or f16 (K a multiple of 128)."""
  return _quantize_rows("e4m3", x, group_sizes, token_idx, padded_input, out)


def quantize_mxfp8_scatter(x: torch.Tensor, group_sizes: torch.Tensor, slot_pos: torch.Tensor,
                           top_k: int, *, out: MXFP8Rows | None = None) -> MXFP8Rows:
  """quantize_mxfp8_rows(x, group_sizes, token_idx) of a dropless dispatch,
  in token order: each token's row is quantised once and stored at the padded
  positions of its top_k sorted positions (the same bits; padding rows are
  left untouched)."""
  return _quantize_scatter("e4m3", x, group_sizes, slot_pos, top_k, out)


def quantize_mxfp4_rows(x: torch.Tensor, group_sizes: torch.Tensor,
                        token_idx: torch.Tensor | None = None, *, padded_input: bool = False,
                        out: MXFP4Rows | None = None) -> MXFP4Rows:
  """quantize_mxfp8_rows with e2m1 elements (MXFP4: scale 2^e, the smallest
  with amax <= 6 * 2^e per 32 K values; values rounded to nearest even)."""
  return _quantize_rows("e2m1", x, group_sizes, token_idx, padded_input, out)


def quantize_mxfp4_scatter(x: torch.Tensor, group_sizes: torch.Tensor, slot_pos: torch.Tensor,
                           top_k: int, *, out: MXFP4Rows | None = None) -> MXFP4Rows:
  """quantize_mxfp8_scatter with e2m1 elements (the rows quantize_mxfp4_rows
  writes for the dispatch's token_idx, bit for bit)."""
  return _quantize_scatter("e2m1", x, group_sizes, slot_pos, top_k, out)


def quantize_split_rows(x: torch.Tensor, group_sizes: torch.Tensor,
                        token_idx: torch.Tensor | None = None, *, padded_input: bool = False,
                        out: SplitRows | None = None) -> SplitRows:
  """quantize_mxfp8_rows into two e4m3 planes: hi = e4m3(x / 2^e) and lo =
  e4m3(x / 2^e - hi) under the MXFP8 block scale.  Every bf16 value with
  |x| >= 2^(e-2) is held exactly by hi + lo (smaller ones to within 2^(e-10)),
  so a block-scaled GEMM on both planes is the exact product."""
  return _quantize_rows("e4m3x2", x, group_sizes, token_idx, padded_input, out)


def quantize_split_scatter(x: torch.Tensor, group_sizes: torch.Tensor, slot_pos: torch.Tensor,
                           top_k: int, *, out: SplitRows | None = None) -> SplitRows:
  """quantize_mxfp8_scatter into the two planes of quantize_split_rows."""
  return _quantize_scatter("e4m3x2", x, group_sizes, slot_pos, top_k, out)


def quantize_split_scatter_with_positions(x: torch.Tensor, group_sizes: torch.Tensor,
                                          slot_pos: torch.Tensor, top_k: int
                                          ) -> tuple[SplitRows, torch.Tensor]:
  """quantize_split_scatter that also returns the slot positions moved to
  the padded rows (mxfp8_pad_positions(slot_pos, group_sizes)), written by
  the same kernel."""
  _need_cuda(x, group_sizes, slot_pos)
  t, k = x.shape
  g = group_sizes.shape[0]
  out = _mx_rows("e4m3x2", mxfp8_padded_rows(t * top_k, g), k, group_sizes, x.device)
  gs = group_sizes.to(torch.int32).contiguous()
  out.group_sizes = gs
  pos = torch.empty(t * top_k, dtype=torch.int32, device=x.device)
  _native.call("lmoe_bf16split_quantize_scatter_positions", _ptr(x.contiguous()),
               int(x.dtype == torch.float16), _ptr(slot_pos.to(torch.int32).contiguous()), t,
               top_k, k, _ptr(gs), g, _ptr(out.q), _ptr(out.sf), out.q.shape[-2], _ptr(pos),
               _ptr(device_status(x.device)), _stream())
  return out, pos


def mxfp8_pad_positions(positions: torch.Tensor, group_sizes: torch.Tensor) -> torch.Tensor:
  """Sorted-order row positions -> their rows in the padded layout."""
  _need_cuda(positions, group_sizes)
  pos = positions.to(torch.int32).contiguous()
  out = torch.empty_like(pos)
  _native.call("lmoe_mxfp8_pad_positions", _ptr(pos), pos.numel(),
               _ptr(group_sizes.to(torch.int32).contiguous()), group_sizes.shape[0], _ptr(out),
               _stream())
  return out


def _mx_gemm(a, w, res, m_pad, k, n, g, epi, beta, linear_beta, round_gate_up, code, m_out=0):
  common = (_ptr(a.q), _ptr(a.sf), _ptr(w.packed), _ptr(w.sf), _ptr(a.group_sizes), _ptr(res),
            m_pad, k, n, g, epi, float(beta), float(linear_beta), int(round_gate_up), code)
  tail = (_ptr(device_status(a.q.device)), _stream())
  if isinstance(a, SplitRows):
    _native.call("lmoe_bf16split_mxfp4_grouped_gemm", *common, m_out, *tail)
  elif m_out:
    raise ValueError("unpadded output rows need split rows")
  elif isinstance(a, MXFP8Rows):
    _native.call("lmoe_mxfp8_mxfp4_grouped_gemm", *common, *tail)
  elif isinstance(a, MXFP4Rows):
    _native.call("lmoe_mxfp4_mxfp4_grouped_gemm", *common, *tail)
  else:
    raise TypeError(f"block-scaled rows expected, got {type(a).__name__}")


def mxfp8_mxfp4_ragged_dot(a: MXFP8Rows | MXFP4Rows | SplitRows, w: MXFP4BlockScaled,
                           out_dtype: torch.dtype = torch.bfloat16,
                           out: torch.Tensor | None = None, unpadded_rows: int | None = None,
                           zero_tail: bool = True) -> torch.Tensor:
  """Padded block-scaled rows @ dequant(w[g])^T per group -> (M_pad, N); rows
  past each group's count are not written.  MXFP8 rows run kind::mxf8f6f4,
  MXFP4 rows (K a multiple of 256) kind::mxf4, split rows kind::mxf8f6f4 on
  both planes (the exact product).  With `unpadded_rows` (split rows only)
  the output is (unpadded_rows, N) in the ragged_dot layout: row r of group g
  at the sum of the earlier groups' sizes + r, and the rows past
  sum(group_sizes) zeroed, or left unwritten with zero_tail=False (an output
  sized by capacity)."""
  g, n, k = w.shape
  if w.gateup:
    raise ValueError("gate/up-interleaved weights go through mxfp8_mxfp4_gateup_situ")
  m_pad = a.q.shape[-2]
  if unpadded_rows is None:
    res = _out(out, (m_pad, n), out_dtype, a.q.device)
    code = {torch.bfloat16: 0, torch.float32: 1, torch.float16: 2}[res.dtype]
    _mx_gemm(a, w, res, m_pad, k, n, g, 0, 0.0, 0.0, 0, code)
    return res
  if not isinstance(a, SplitRows):
    raise ValueError("unpadded output rows need split rows")
  rows = int(unpadded_rows)
  res = _out(out, (rows, n), out_dtype, a.q.device)
  code = {torch.bfloat16: 0, torch.float32: 1, torch.float16: 2}[res.dtype]
  if rows > 0:
    _mx_gemm(a, w, res, m_pad, k, n, g, 0, 0.0, 0.0, 0, code, m_out=rows if zero_tail else -rows)
  return res


def mxfp8_mxfp4_gateup_situ(a: MXFP8Rows | MXFP4Rows | SplitRows, w: MXFP4BlockScaled, *,
                            beta: float = 4.0, linear_beta: float = 25.0,
                            round_gate_up: bool = True, out_dtype: torch.dtype = torch.bfloat16,
                            out: torch.Tensor | None = None) -> torch.Tensor:
  """SiTU-GLU of the block-scaled grouped matmul against gate/up-interleaved
  MXFP4 weights -> (M_pad, I) (padded rows); MXFP8, MXFP4 or split rows."""
  g, two_i, k = w.shape
  if not w.gateup:
    raise ValueError("prepare the fused weight with prepare_mxfp4_blockscaled(..., gateup=True)")
  m_pad = a.q.shape[-2]
  res = _out(out, (m_pad, two_i // 2), out_dtype, a.q.device)
  code = {torch.bfloat16: 0, torch.float16: 2}[res.dtype]
  _mx_gemm(a, w, res, m_pad, k, two_i // 2, g, 3, beta, linear_beta, round_gate_up, code)
  return res


def mxfp4_ragged_dot_blockscaled(lhs: torch.Tensor, w: MXFP4BlockScaled,
                                 group_sizes: torch.Tensor,
                                 out_dtype: torch.dtype = torch.bfloat16,
                                 out: torch.Tensor | None = None,
                                 rows: SplitRows | None = None) -> torch.Tensor:
  """mxfp4_ragged_dot (the exact MXFP4 grouped matmul, ragged_dot layout:
  lhs (M, K) bf16/f16 in group order, out (M, N), rows past sum(group_sizes)
  zero) on the block-scaled tensor core: the rows split into two e4m3 planes
  (quantize_split_rows), both multiplied into one accumulator, the output
  written at the unpadded rows.  Within ~1e-6 normwise of the exact kernel.
  `rows` (optional) is reused as the split buffer."""
  g, n, k = w.shape
  if w.gateup:
    raise ValueError("gate/up-interleaved weights go through mxfp8_mxfp4_gateup_situ")
  m = lhs.shape[0]
  a = quantize_split_rows(lhs, group_sizes, out=rows)
  res = _out(out, (m, n), out_dtype, lhs.device)
  code = {torch.bfloat16: 0, torch.float32: 1, torch.float16: 2}[res.dtype]
  if m > 0:
    _mx_gemm(a, w, res, a.q.shape[-2], k, n, g, 0, 0.0, 0.0, 0, code, m_out=m)
  return res


_ROWS_KIND = {MXFP8Rows: 0, MXFP4Rows: 1, SplitRows: 2}
_FMT_CODE = {"e4m3": 0, "e2m1": 1, "e4m3x2": 2}


def blockscaled_gateup_situ_quantized(a: MXFP8Rows | MXFP4Rows | SplitRows, w: MXFP4BlockScaled,
                                      fmt: str, *, beta: float = 4.0, linear_beta: float = 25.0,
                                      round_gate_up: bool = True, out=None):
  """mxfp8_mxfp4_gateup_situ with the SiTU activations written straight into
  block-scaled rows of format `fmt` ("e4m3", "e2m1" or "e4m3x2") for the down
  GEMM: the same bytes as quantising the bf16 output (padded_input=True), with
  no bf16 activation tensor in between."""
  g, two_i, k = w.shape
  if not w.gateup:
    raise ValueError("prepare the fused weight with prepare_mxfp4_blockscaled(..., gateup=True)")
  m_pad = a.q.shape[-2]
  if out is None:
    res = _mx_rows(fmt, m_pad, two_i // 2, a.group_sizes, a.q.device)
  else:
    _check_mx_rows(out, fmt, m_pad, two_i // 2)
    res = out
  res.group_sizes = a.group_sizes
  _native.call("lmoe_blockscaled_gateup_situ_quantized", _ptr(a.q), _ptr(a.sf),
               _ROWS_KIND[type(a)], _ptr(w.packed), _ptr(w.sf), _ptr(a.group_sizes), m_pad, k,
               two_i // 2, g, float(beta), float(linear_beta), int(round_gate_up), _FMT_CODE[fmt],
               _ptr(res.q), _ptr(res.sf), _ptr(device_status(a.q.device)), _stream())
  return res


# the same functions under the names of the MXFP4-activation form
mxfp4_mxfp4_ragged_dot = mxfp8_mxfp4_ragged_dot
mxfp4_mxfp4_gateup_situ = mxfp8_mxfp4_gateup_situ
