"""LatentMoE layer forward on B200: the model-level drop-in for
`latent_moe_forward` (05_ragged_dot_on_tpu/kimi_k3_latent_moe_reference.py:330-435)
and `latent_moe_forward_ragged_dot` (kimi_k3_latent_moe_ragged_dot.py:317-391).

Weights arrive in the reference's (in, out) layout (`LatentMoEWeights`,
kimi_k3_latent_moe_reference.py:217-252) and are re-laid out ONCE by
`prepare_weights` into the K-major forms the kernels stream (the analogue of
the reference's one-time `prefuse_gateup_weights`, kimi_k3_latent_moe_ragged_dot.py:610-641):

  router      (E, d)          bf16/f32    logits = h @ W^T in f32
  down        (L, d)          x = h @ W_down
  expert_gu   (E, 2I, L)      [gate | up] rows, one fused grouped GEMM + SiTU-GLU
  expert_down (E, L, I)
  up          (d, L)
  shared_gu   (2*Is, d)       [gate | up] of the shared expert (one dense group)
  shared_down (d, Is)

bf16 forward, in stream order (no host synchronisation):
  1 logits      tensor-core GEMM with the top-k selection in its epilogue
                (exact bf16 products, f32 sums; sigmoid, bias for selection
                only; the f32 logits stay in tensor memory)
  2 top-k       merge of the per-chunk candidates (router_topk on stored
                logits when the intermediates are requested)
  3 x           tensor-core GEMM (down-projection)
  4-6 dispatch  stable counting sort by expert      (order, slot_pos, group_sizes)
  7 gather      sorted rows of x
  8 gate/up     grouped GEMM + fused SiTU-GLU epilogue
  9 down        grouped GEMM
  10 combine    f32 weighted sum in slot order + RMSNorm
  11 up-proj    GEMM;  12 shared gate/up GEMM + SiTU;  13 shared down GEMM + residual add
The f32 forward runs the same steps on the f32 CUDA-core kernels.
"""

from __future__ import annotations

import dataclasses

import torch

from . import ops


@dataclasses.dataclass(frozen=True)
class LatentMoEConfig:
  """kimi_k3_latent_moe_reference.py:156-171."""

  hidden_size: int
  latent_size: int
  intermediate_size: int
  num_experts: int
  top_k: int
  num_shared_experts: int
  moe_renormalize: bool = True
  routed_scaling_factor: float = 1.0
  rms_norm_eps: float = 1e-5
  activation_situ_beta: float = 4.0
  activation_situ_linear_beta: float = 25.0


def toy_config() -> LatentMoEConfig:
  """kimi_k3_latent_moe_reference.py:174-188."""
  return LatentMoEConfig(64, 32, 48, 8, 2, 1)


def kimi_k3_config() -> LatentMoEConfig:
  """kimi_k3_latent_moe_reference.py:191-208."""
  return LatentMoEConfig(7168, 3584, 3072, 896, 16, 2)


def reduced_cpu_config() -> LatentMoEConfig:
  """Configuration 1 of the benchmark plan: d 512 -> L 256, 64 experts, I 512, top-8."""
  return LatentMoEConfig(512, 256, 512, 64, 8, 1)


def full_layer_config() -> LatentMoEConfig:
  """Configuration 5: d 7168, L 2048, 896 experts, I 1024, top-16, 2 shared."""
  return LatentMoEConfig(7168, 2048, 1024, 896, 16, 2)


@dataclasses.dataclass
class LatentMoEWeights:
  """kimi_k3_latent_moe_reference.py:217-252, (in, out) layout, torch tensors."""

  router_weight: torch.Tensor  # (d, E)
  e_score_correction_bias: torch.Tensor  # (E,)
  down_proj: torch.Tensor  # (d, L)
  up_proj: torch.Tensor  # (L, d)
  expert_gate: torch.Tensor  # (E, L, I)
  expert_up: torch.Tensor  # (E, L, I)
  expert_down: torch.Tensor  # (E, I, L)
  norm_scale: torch.Tensor  # (L,)
  shared_gate: torch.Tensor  # (d, I*ns)
  shared_up: torch.Tensor  # (d, I*ns)
  shared_down: torch.Tensor  # (I*ns, d)


def init_weights(config: LatentMoEConfig, seed: int = 0, dtype: torch.dtype = torch.bfloat16,
                 device: str | torch.device = "cuda", bias_std: float = 0.0,
                 experts: bool = True) -> LatentMoEWeights:
  """N(0, 0.02^2) weights (the distribution of kimi_k3_latent_moe_reference.py:255-283),
  drawn on the device from a seeded generator; optional N(0, bias_std^2)
  router bias for the skewed-load configurations.  experts=False leaves the
  routed-expert tensors out (None), for MXFP4 experts supplied separately."""
  gen = torch.Generator(device=device)
  gen.manual_seed(seed)
  c = config
  si = c.intermediate_size * c.num_shared_experts

  def normal(*shape):
    return (torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * 0.02).to(dtype)

  bias = torch.zeros(c.num_experts, device=device, dtype=torch.float32)
  if bias_std > 0:
    bias = torch.randn(c.num_experts, generator=gen, device=device) * bias_std
  ex = (lambda *s: normal(*s)) if experts else (lambda *s: None)
  return LatentMoEWeights(
      router_weight=normal(c.hidden_size, c.num_experts),
      e_score_correction_bias=bias.to(dtype),
      down_proj=normal(c.hidden_size, c.latent_size),
      up_proj=normal(c.latent_size, c.hidden_size),
      expert_gate=ex(c.num_experts, c.latent_size, c.intermediate_size),
      expert_up=ex(c.num_experts, c.latent_size, c.intermediate_size),
      expert_down=ex(c.num_experts, c.intermediate_size, c.latent_size),
      norm_scale=torch.ones(c.latent_size, device=device, dtype=dtype),
      shared_gate=normal(c.hidden_size, si),
      shared_up=normal(c.hidden_size, si),
      shared_down=normal(si, c.hidden_size),
  )


@dataclasses.dataclass
class PreparedWeights:
  """Kernel layouts (see the module docstring).  Routed experts are either
  bf16/f32 tensors or MXFP4 (`expert_gu_mx`, `expert_down_mx`)."""

  dtype: torch.dtype
  router: torch.Tensor
  bias: torch.Tensor  # f32
  down: torch.Tensor
  up: torch.Tensor
  expert_gu: torch.Tensor | None
  expert_gate: torch.Tensor | None  # f32 path keeps gate and up apart (G, I, L)
  expert_up: torch.Tensor | None
  expert_down: torch.Tensor | None
  norm_scale: torch.Tensor
  shared_gu: torch.Tensor | None
  shared_gate: torch.Tensor | None
  shared_up: torch.Tensor | None
  shared_down: torch.Tensor
  expert_gu_mx: ops.MXFP4Weights | None = None     # (E, 2I, L/2) codes: [w1 gate | w3 up]
  expert_down_mx: ops.MXFP4Weights | None = None   # (E, L, I/2) codes: w2
  # the same experts prepared for the block-scaled MMA (built on the first
  # forward that uses it -- the default "split" mode among them -- then kept)
  expert_gu_bs: ops.MXFP4BlockScaled | None = None
  expert_down_bs: ops.MXFP4BlockScaled | None = None


def random_mxfp4(num_experts: int, n: int, k: int, seed: int, device="cuda",
                 scale_exp=(-8, -6)) -> ops.MXFP4Weights:
  """Seeded synthetic MXFP4 weights: e2m1 codes uniform over all 16 values and
  E8M0 scales with unbiased exponent uniform in [scale_exp[0], scale_exp[1]]
  ((-8, -6) gives weights of rms ~0.02, the N(0, 0.02^2) scale of the dense
  weights; (-6, 2) is benchmark configuration 4)."""
  gen = torch.Generator(device=device)
  gen.manual_seed(seed)
  packed = torch.randint(0, 256, (num_experts, n, k // 2), generator=gen, device=device,
                         dtype=torch.int32).to(torch.uint8)
  scale = torch.randint(127 + scale_exp[0], 127 + scale_exp[1] + 1, (num_experts, n, k // 32),
                        generator=gen, device=device, dtype=torch.int32).to(torch.uint8)
  return ops.MXFP4Weights(packed, scale)


def init_prepared_mxfp4(config: LatentMoEConfig, seed: int = 0, device="cuda",
                        bias_std: float = 0.5, expert_start: int = 0,
                        num_local_experts: int | None = None) -> PreparedWeights:
  """bf16 dense weights (N(0, 0.02^2)) plus MXFP4 routed experts, directly in
  the kernel layouts.  With expert_start / num_local_experts only that
  contiguous expert range is materialised (expert parallelism); the experts
  are drawn per global index so every rank sees the same global weights."""
  c = config
  e_loc = c.num_experts if num_local_experts is None else num_local_experts
  dense = init_weights(dataclasses.replace(c, num_experts=c.num_experts), seed=seed,
                       dtype=torch.bfloat16, device=device, bias_std=bias_std, experts=False)
  pw = prepare_weights(dense, torch.bfloat16)
  gus, downs = [], []
  for e in range(expert_start, expert_start + e_loc):
    gus.append(random_mxfp4(1, 2 * c.intermediate_size, c.latent_size, seed * 100003 + 2 * e + 1,
                            device))
    downs.append(random_mxfp4(1, c.latent_size, c.intermediate_size, seed * 100003 + 2 * e + 2,
                              device))
  pw.expert_gu_mx = ops.MXFP4Weights(torch.cat([w.packed for w in gus]),
                                     torch.cat([w.scale for w in gus]))
  pw.expert_down_mx = ops.MXFP4Weights(torch.cat([w.packed for w in downs]),
                                       torch.cat([w.scale for w in downs]))
  return pw


def _t(w: torch.Tensor) -> torch.Tensor:
  return w.transpose(-1, -2).contiguous()


def prepare_weights(w: LatentMoEWeights, dtype: torch.dtype | None = None) -> PreparedWeights:
  """One-time re-layout of (in, out) weights into the K-major kernel layouts."""
  dtype = dtype or w.down_proj.dtype
  cv = lambda a: a.to(dtype)
  bf16 = dtype == torch.bfloat16
  has_ex = w.expert_gate is not None
  return PreparedWeights(
      dtype=dtype,
      router=_t(cv(w.router_weight)),
      bias=w.e_score_correction_bias.float().contiguous(),
      down=_t(cv(w.down_proj)),
      up=_t(cv(w.up_proj)),
      expert_gu=_t(torch.cat([cv(w.expert_gate), cv(w.expert_up)], dim=-1))
      if bf16 and has_ex else None,
      expert_gate=None if bf16 or not has_ex else _t(cv(w.expert_gate)),
      expert_up=None if bf16 or not has_ex else _t(cv(w.expert_up)),
      expert_down=_t(cv(w.expert_down)) if has_ex else None,
      norm_scale=cv(w.norm_scale).contiguous(),
      shared_gu=_t(torch.cat([cv(w.shared_gate), cv(w.shared_up)], dim=-1)) if bf16 else None,
      shared_gate=None if bf16 else _t(cv(w.shared_gate)),
      shared_up=None if bf16 else _t(cv(w.shared_up)),
      shared_down=_t(cv(w.shared_down)),
  )


def latent_moe_forward(hidden_states: torch.Tensor, weights, config: LatentMoEConfig, *,
                       router_activation: str = "sigmoid",
                       return_intermediates: bool = False, mxfp4_operand: str = "auto",
                       dense_phases: bool | None = None, mark=None):
  """The 8-step LatentMoE forward (kimi_k3_latent_moe_reference.py:330-435).
  `weights` is a LatentMoEWeights (prepared on the fly) or PreparedWeights.

  mxfp4_operand (MXFP4 experts only): "auto" (the default) is "split": the
  exact product on the block-scaled tensor core -- each latent or SiTU
  activation row becomes two e4m3 planes under one E8M0 scale per 32 values
  (hi and the rounding remainder lo, which together hold its bf16 value for
  every |x| >= 2^-2 of the block scale, and within 2^-10 of it below), both
  multiplied into one f32 accumulator by kind::mxf8f6f4 MMAs that read the
  e2m1 weight codes as stored (~1e-6 normwise from the dequant-then-matmul
  product).  "f16" runs the weights-major kernels, which expand the codes
  into f16 tiles in shared memory, when every weight scale allows it (see
  mxfp4_f16_path; otherwise their bf16 form): the latent rows then travel as
  f16 carrying their bf16-rounded values, exact up to 65504 in magnitude (a
  larger value would become inf, so the kernel that writes the f16 rows
  records LMOE_F16_RANGE in the device status word, which
  check_device_status raises).  "bf16" runs the weights-major kernels on
  bf16 operands without that range limit.  "mxfp8" is the opt-in fast path:
  the latent rows and the SiTU activations are rounded to MXFP8 (e4m3, one
  E8M0 scale per 32 values) and run one kind::mxf8f6f4 MMA per K slice; the
  activation rounding adds ~3% normwise error against the exact forward.
  "mxfp4" rounds them to MXFP4 instead (e2m1, one E8M0 scale per 32 values)
  and runs kind::mxf4, at twice the MMA rate and a larger error (~10%
  normwise).

  dense_phases (bf16 dense weights with a shared expert): the dense
  projections run as two persistent split-K kernels, one per phase -- the
  router logits, the down-projection and the shared expert's gate/up in one
  launch over the hidden states (then the top-k from the logits), the
  up-projection, the shared expert's down projection and the output sum in
  another (the sum of the two branches rounded once to bf16 instead of each
  branch first: within about one bf16 spacing of the output).  None (the
  default) takes them when their output tiles would not fill the SMs (a few
  hundred tokens or fewer on one GPU); False never; True whenever the shapes
  allow.  Not with return_intermediates.

  `mark(name)` (optional) is called on the host after each phase of the main
  stream is enqueued, e.g. to record CUDA events for a phase timeline."""
  mark = mark or (lambda name: None)
  pw = weights if isinstance(weights, PreparedWeights) else prepare_weights(weights)
  h = hidden_states.to(pw.dtype).contiguous()
  c = config
  t = h.shape[0]
  inter = {}
  beta, lbeta = c.activation_situ_beta, c.activation_situ_linear_beta
  # The shared expert depends only on h: on the bf16 path it runs on a side
  # stream beside the routing, dispatch and gather kernels (which leave most of
  # the tensor cores idle) and joins before the output sum, computed as
  # bf16(bf16(normed @ W_up) + shared) -- the same bits as the other order.
  # The down-projection depends only on h too.  When it is small (its 128 x
  # 128 tiles would fill at most half the SMs: a few hundred tokens) it runs on
  # a second side stream beside the router and the dispatch sort, which then
  # use few SMs as well, and joins before the gather.  With more tokens each
  # of these GEMMs fills the GPU and running them at the same time only slows
  # both (measured: 16384 tokens 5.66 -> 6.12 ms), so they stay in order.
  mxfp4_operand = resolve_mxfp4_operand(pw, mxfp4_operand)
  x_dtype = torch.float16 if mxfp4_f16_path(pw, mxfp4_operand) else torch.bfloat16
  phases = _use_dense_phases(dense_phases, pw, c, t, h, x_dtype, return_intermediates)
  overlap = pw.dtype == torch.bfloat16 and not return_intermediates and not phases
  down_tiles = -(-t // 128) * -(-pw.down.shape[0] // 128)
  overlap_x = overlap and 2 * down_tiles <= torch.cuda.get_device_properties(
      h.device).multi_processor_count
  if overlap:
    main = torch.cuda.current_stream(h.device)
    side = ops.side_stream(h.device)
    shared_act = torch.empty(t, pw.shared_gu.shape[0] // 2, dtype=h.dtype, device=h.device)
    shared_out = torch.empty(t, pw.shared_down.shape[0], dtype=h.dtype, device=h.device)
    side.wait_stream(main)
  if overlap_x:
    side_x = ops.side_stream(h.device, 1)
    x = torch.empty(t, pw.down.shape[0], dtype=x_dtype, device=h.device)
    side_x.wait_stream(main)
    with torch.cuda.stream(side_x):
      ops.gemm(h, pw.down, rhs_layout="nk", out=x)
  if overlap:
    with torch.cuda.stream(side):
      ops.fused_gateup_situ(h, pw.shared_gu, None, beta=beta, linear_beta=lbeta,
                            round_gate_up=True, rhs_layout="gnk", out=shared_act)
      ops.gemm(shared_act, pw.shared_down, rhs_layout="nk", out=shared_out)
  if phases:
    logits, x, shared_act = ops.dense_input_phase(h, pw.router, pw.down, pw.shared_gu, beta=beta,
                                                  linear_beta=lbeta, round_gate_up=True)
    topk_idx, topk_w = ops.router_topk(logits, pw.bias, c.top_k, renormalize=c.moe_renormalize,
                                       routed_scaling_factor=c.routed_scaling_factor,
                                       activation=router_activation)
  elif return_intermediates or not ops.router_fused_supported(h, pw.router, c.top_k,
                                                               router_activation):
    logits = ops.router_logits(h, pw.router)
    topk_idx, topk_w = ops.router_topk(logits, pw.bias, c.top_k, renormalize=c.moe_renormalize,
                                       routed_scaling_factor=c.routed_scaling_factor,
                                       activation=router_activation)
  else:
    # logits GEMM with the selection in its epilogue: the same bits, no f32
    # logits in memory
    topk_idx, topk_w = ops.router_gate_fused(h, pw.router, pw.bias, c.top_k,
                                             renormalize=c.moe_renormalize,
                                             routed_scaling_factor=c.routed_scaling_factor)
  mark("route")
  if not overlap_x and not phases:
    x = _dense(h, pw.down, out_dtype=None if x_dtype == torch.bfloat16 else x_dtype)
    mark("down-projection")
  d = ops.dispatch(topk_idx, topk_w, c.num_experts, want_order=return_intermediates)
  mark("dispatch sort")
  if overlap_x:
    main.wait_stream(side_x)
    mark("down-projection")
  slot_pos = d.slot_pos
  if pw.expert_gu_mx is not None and mxfp4_operand in ("mxfp8", "mxfp4", "split"):
    fmt = {"mxfp8": "e4m3", "mxfp4": "e2m1", "split": "e4m3x2"}[mxfp4_operand]
    act, down, slot_pos = mxfp8_expert_ffn(x, d.token_idx, d.group_sizes, d.slot_pos, pw, c,
                                           mark, fmt=fmt, keep_activation=return_intermediates)
  elif pw.expert_gu_mx is not None:
    act, down = mxfp4_expert_ffn(x, d.token_idx, d.group_sizes, pw, c, mark, d.slot_pos)
  elif pw.dtype == torch.bfloat16:
    sorted_tokens = ops.scatter_rows(x, d.slot_pos, c.top_k)
    act = ops.fused_gateup_situ(sorted_tokens, pw.expert_gu, d.group_sizes, beta=beta,
                                linear_beta=lbeta, round_gate_up=True, rhs_layout="gnk")
    down = ops.ragged_dot(act, pw.expert_down, d.group_sizes, rhs_layout="gnk")
  else:
    sorted_tokens = ops.scatter_rows(x, d.slot_pos, c.top_k)
    gate = ops.ragged_dot(sorted_tokens, pw.expert_gate, d.group_sizes, rhs_layout="gnk")
    up = ops.ragged_dot(sorted_tokens, pw.expert_up, d.group_sizes, rhs_layout="gnk")
    act = ops.situ_and_mul(gate, up, beta, lbeta)
    down = ops.ragged_dot(act, pw.expert_down, d.group_sizes, rhs_layout="gnk")
  if pw.expert_gu_mx is None:
    mark("experts")
  routed, normed = ops.combine_rmsnorm(down, slot_pos, topk_w, pw.norm_scale, c.rms_norm_eps,
                                       want_routed=True)
  mark("combine")
  if phases:
    out = ops.dense_output_phase(normed, pw.up, shared_act, pw.shared_down)
    mark("tail")
    return out
  if overlap:
    main.wait_stream(side)
    out = _dense(normed, pw.up, addend=shared_out)
    mark("tail")
    return out
  upo = _dense(normed, pw.up)
  if pw.dtype == torch.bfloat16:
    shared_act = ops.fused_gateup_situ(h, pw.shared_gu, None, beta=beta, linear_beta=lbeta,
                                       round_gate_up=True, rhs_layout="gnk")
  else:
    shared_act = ops.situ_and_mul(_dense(h, pw.shared_gate), _dense(h, pw.shared_up), beta, lbeta)
  final = _dense(shared_act, pw.shared_down, addend=upo)
  if return_intermediates:
    # the shared expert's own output (the golden bundles' stage of that name)
    shared = _dense(shared_act, pw.shared_down)
    inter.update(router_logits=logits, topk_indices=topk_idx, topk_weights=topk_w,
                 latent_projection=x, sorted_token_indices=d.order, group_sizes=d.group_sizes,
                 situ_output=act, expert_down_output=down, routed_output_after_combine=routed,
                 normalized_output=normed, up_projection_output=upo,
                 shared_expert_output=shared, final_output=final,
                 slot_pos=d.slot_pos, token_idx=d.token_idx)
    return final, inter
  return final


def _use_dense_phases(dense_phases, pw: "PreparedWeights", c: LatentMoEConfig, t: int, h,
                      x_dtype, return_intermediates: bool) -> bool:
  """Whether latent_moe_forward runs the dense projections as the split-K
  phase kernels (see its `dense_phases` argument)."""
  if dense_phases is False or return_intermediates or t == 0:
    return False
  si = pw.shared_gu.shape[0] // 2 if pw.shared_gu is not None else 0
  supported = (pw.dtype == torch.bfloat16 and x_dtype == torch.bfloat16 and si > 0 and
               pw.shared_down is not None and
               ops._native.load().lmoe_dense_input_workspace_size(
                   t, c.hidden_size, c.num_experts, pw.down.shape[0], si) > 0 and
               ops._native.load().lmoe_dense_output_workspace_size(
                   t, pw.down.shape[0], si, pw.up.shape[0]) > 0)
  if not supported:
    return False
  return dense_phases is True or ops.dense_phases_pay_off(t, c.num_experts, pw.down.shape[0], si,
                                                          h.device)


MXFP4_OPERANDS = ("auto", "split", "f16", "bf16", "mxfp8", "mxfp4")


def resolve_mxfp4_operand(pw: PreparedWeights, mxfp4_operand: str = "auto") -> str:
  """The MXFP4 expert mode a forward runs: "auto" is "split" (the exact
  product on the block-scaled tensor core) when the experts are MXFP4."""
  if mxfp4_operand not in MXFP4_OPERANDS:
    raise ValueError(f"mxfp4_operand={mxfp4_operand!r}: one of {', '.join(MXFP4_OPERANDS)}")
  if mxfp4_operand == "auto" and pw.expert_gu_mx is not None:
    return "split"
  return mxfp4_operand


def mxfp4_f16_path(pw: PreparedWeights, mxfp4_operand: str = "f16") -> bool:
  """True when the MXFP4 experts run the weights-major f16-operand kernels:
  mxfp4_operand is "f16" and every scale byte lies in their exact range.
  The latent activations then travel as f16 (the same bf16-rounded values)."""
  if mxfp4_operand not in MXFP4_OPERANDS:
    raise ValueError(f"mxfp4_operand={mxfp4_operand!r}: one of {', '.join(MXFP4_OPERANDS)}")
  return (mxfp4_operand == "f16" and pw.expert_gu_mx is not None and
          pw.expert_gu_mx.f16_operand_ok and pw.expert_down_mx.f16_operand_ok)


def mxfp4_expert_ffn(x, token_idx, group_sizes, pw: PreparedWeights, c: LatentMoEConfig,
                     mark=None, slot_pos=None):
  """Routed-expert FFN on MXFP4 weights: row gather into expert-sorted order,
  fused gate/up + SiTU-GLU, down GEMM.  x is f16 on the f16-operand path (see
  mxfp4_f16_path), bf16 otherwise.  With slot_pos (a dropless dispatch's) the
  gather runs in token order (each row read once, stored top_k times).  (The
  gather can also run inside the gate/up kernel's operand load, `row_index=`;
  at these sizes the one-row TMA gathers feed the tensor cores ~2.5x slower
  than a separate gather kernel plus contiguous tile loads, so the forward
  gathers first.)  Returns (activation, down output bf16)."""
  mark = mark or (lambda name: None)
  rows = (ops.gather_rows(x, token_idx) if slot_pos is None else
          ops.scatter_rows(x, slot_pos, c.top_k, out_rows=token_idx.shape[0]))
  mark("gather")
  act = ops.mxfp4_fused_gateup_situ(rows, pw.expert_gu_mx, group_sizes,
                                    beta=c.activation_situ_beta,
                                    linear_beta=c.activation_situ_linear_beta, round_gate_up=True,
                                    out_dtype=x.dtype)
  mark("expert gate/up")
  down = ops.mxfp4_ragged_dot(act, pw.expert_down_mx, group_sizes)
  mark("expert down")
  return act, down


def blockscaled_experts(pw: PreparedWeights):
  """The MXFP4 experts prepared for the block-scaled MMA (one repack, kept)."""
  if pw.expert_gu_bs is None:
    pw.expert_gu_bs = ops.prepare_mxfp4_blockscaled(pw.expert_gu_mx, gateup=True)
    pw.expert_down_bs = ops.prepare_mxfp4_blockscaled(pw.expert_down_mx)
  return pw.expert_gu_bs, pw.expert_down_bs


def mxfp8_expert_ffn(x, token_idx, group_sizes, slot_pos, pw: PreparedWeights,
                     c: LatentMoEConfig, mark=None, fmt: str = "e4m3",
                     keep_activation: bool = True):
  """Routed-expert FFN on the block-scaled tensor core: the gather quantises
  the latent rows to MXFP8 (fmt "e4m3"), MXFP4 ("e2m1") or two e4m3 planes
  ("e4m3x2", the exact split) into the padded layout (every expert's rows
  start at a multiple of 128; in token order, each row quantised once and
  stored top_k times), gate/up + SiTU-GLU, the
  activations quantised again (inside the gate/up kernel's epilogue unless
  keep_activation asks for the bf16 activations), the down GEMM; the slot
  positions are moved to the padded rows for the combine.  Returns
  (activation or None, down output, padded slot positions)."""
  mark = mark or (lambda name: None)
  gu, dn = blockscaled_experts(pw)
  quantize_scatter, quantize_rows = {
      "e4m3": (ops.quantize_mxfp8_scatter, ops.quantize_mxfp8_rows),
      "e2m1": (ops.quantize_mxfp4_scatter, ops.quantize_mxfp4_rows),
      "e4m3x2": (ops.quantize_split_scatter, ops.quantize_split_rows)}[fmt]
  padded_pos = None
  if fmt == "e4m3x2":
    # the gather also writes the slot positions moved to the padded rows
    rows, padded_pos = ops.quantize_split_scatter_with_positions(x, group_sizes, slot_pos, c.top_k)
  else:
    rows = quantize_scatter(x, group_sizes, slot_pos, c.top_k)
  mark("gather")
  if keep_activation:
    act = ops.mxfp8_mxfp4_gateup_situ(rows, gu, beta=c.activation_situ_beta,
                                      linear_beta=c.activation_situ_linear_beta,
                                      round_gate_up=True)
    act_q = quantize_rows(act, group_sizes, padded_input=True)
  else:
    # the gate/up kernel writes the down GEMM's quantised rows directly
    act = None
    act_q = ops.blockscaled_gateup_situ_quantized(
        rows, gu, fmt, beta=c.activation_situ_beta, linear_beta=c.activation_situ_linear_beta,
        round_gate_up=True)
  mark("expert gate/up")
  down = ops.mxfp8_mxfp4_ragged_dot(act_q, dn)
  mark("expert down")
  if padded_pos is None:
    padded_pos = ops.mxfp8_pad_positions(slot_pos, group_sizes)
  return act, down, padded_pos


def _dense(a: torch.Tensor, w_nk: torch.Tensor, addend: torch.Tensor | None = None,
           out_dtype: torch.dtype | None = None):
  """a @ W^T for W given (N, K); bf16 on the tensor cores (out_dtype float16:
  the bf16-rounded result stored as f16), f32 on the CUDA cores."""
  if a.dtype == torch.float32:
    from . import _native
    m, k = a.shape
    n = w_nk.shape[0]
    out = torch.empty(m, n, dtype=torch.float32, device=a.device)
    _native.call("lmoe_gemm_f32", a.contiguous().data_ptr(), w_nk.data_ptr(),
                 None if addend is None else addend.contiguous().data_ptr(), out.data_ptr(), m, k,
                 n, 1, ops.device_status(a.device).data_ptr(), ops._stream())
    return out
  return ops.gemm(a, w_nk, addend=addend, rhs_layout="nk", out_dtype=out_dtype or torch.bfloat16)


def latent_moe_forward_ragged_dot(hidden_states, weights, config, implementation=None):
  """kimi_k3_latent_moe_ragged_dot.py:317-391: same forward, routed FFN as
  ragged_dot calls (here always the sm_100a kernels)."""
  ops._check_impl(implementation)
  return latent_moe_forward(hidden_states, weights, config)
