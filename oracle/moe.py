"""Oracle for the MoE expert math -- TEST INFRASTRUCTURE ONLY.

Torch-CPU restatement of the reference's MLX layer math with its BF16
rounding points, for the three families the reference runs:

  generic  runtime/layer_runner.py run_moe_mlp (:347-394), _swiglu (:185-190):
           BF16 router logits, fp32 softmax, top-k, optional renormalisation,
           BF16 route weights, contributions accumulated in first-appearance
           order of the experts over (position, slot).
  qwen35   runtime/qwen35.py _route_experts (:584-593) and _moe (:596-638):
           as generic but always renormalised, scores cast to BF16, experts
           accumulated in ascending id order, then a gated shared expert:
           routed + bf16(sigmoid(bf16(h @ Wsg.T)) * shared(h)).  Its RMSNorm is
           zero-centred (x * rsqrt(..) * (1 + w), qwen35.py:133-150).
  glm      runtime/glm.py _route_experts (:364-392) and _glm_mlp_residual
           (:429-486): fp32 router logits (h and W cast to fp32), sigmoid
           scores, top-k by score + e_score_correction_bias, weights = the
           unbiased scores, renormalised with +1e-20 when norm_topk, times
           routed_scaling_factor, kept in fp32; contributions bf16(y * w_fp32)
           in ascending expert order, then + shared expert.

quant.matmul is x @ W.T with a BF16 result (runtime/quant.py:431-444);
mx.fast.rms_norm rounds x * rsqrt(mean(x^2) + eps) * w once.  Top-k order:
descending key, ties to the lower expert id (MLX's argpartition leaves the
order unspecified; only the generic accumulation order depends on it).

Pinned against Hugging Face transformers' sparse-MoE blocks run in BF16
(OLMoE, Qwen3.5-MoE, GLM-MoE-DSA), the ground truth the reference's own MoE
oracle tests use (tests/test_f33_router_oracle.py:30-40): with
`hf_rounding=True` (HF's rounding points: SiLU fused into one BF16 rounding,
fp32 route weights, experts in ascending id order) this restatement
reproduces those blocks bit for bit, which pins the routing, grouping, the
matmul conventions and the shared-expert wiring; the reference's own
rounding points (the default) then differ from HF only by BF16 rounding.
"""

from __future__ import annotations

import torch

bf16 = torch.bfloat16
FAMILIES = ("generic", "qwen35", "glm")


def _mm(a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """BF16 x @ W.T with fp32 accumulation and a BF16 result."""
    return (a.float() @ w.float().T).to(bf16)


def rms_norm(x: torch.Tensor, w: torch.Tensor | None, eps: float, plus_one: bool = False) -> torch.Tensor:
    if w is None:
        return x
    xf = x.float()
    wf = w.float() + 1.0 if plus_one else w.float()
    return (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + eps) * wf).to(bf16)


def route(h: torch.Tensor, wr: torch.Tensor, k: int, norm_topk: bool, family: str = "generic",
          bias: torch.Tensor | None = None, routed_scale: float = 1.0):
    """(expert ids (T, k), route weights (T, k) fp32) for one family.  For the
    generic family `bias` (fp32, E) is added to the BF16 logits: synthetic
    workloads use it to skew expert popularity; for glm it is the score
    correction bias that only affects the choice."""
    if family == "glm":
        s = torch.sigmoid(h.float() @ wr.float().T)
        key = s + bias.float() if bias is not None else s
        order = torch.argsort(-key, dim=-1, stable=True)[:, :k]
        pw = torch.gather(s, -1, order)
        if norm_topk:
            pw = pw / (pw.sum(-1, keepdim=True) + 1e-20)
        return order, pw * routed_scale
    logits = _mm(h, wr).float()
    if bias is not None:
        logits = logits + bias.float()
    probs = torch.softmax(logits, dim=-1)
    order = torch.argsort(-probs, dim=-1, stable=True)[:, :k]
    pw = torch.gather(probs, -1, order)
    if norm_topk or family == "qwen35":
        pw = pw / pw.sum(-1, keepdim=True)
    return order, pw


def swiglu(h: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor, wd: torch.Tensor,
           fused_silu: bool = False) -> torch.Tensor:
    """_swiglu (layer_runner.py:185-190): sigmoid(g) * g * u with a BF16
    rounding after each op; `fused_silu` rounds silu(g) once (HF's act_fn)."""
    g = _mm(h, wg)
    u = _mm(h, wu)
    if fused_silu:
        a = (torch.nn.functional.silu(g.float()).to(bf16).float() * u.float()).to(bf16)
    else:
        s = torch.sigmoid(g.float()).to(bf16)
        a = ((s.float() * g.float()).to(bf16).float() * u.float()).to(bf16)
    return _mm(a, wd)


def moe_layer(x: torch.Tensor, wr: torch.Tensor, norm_w: torch.Tensor | None, experts, k: int,
              norm_topk: bool = True, eps: float = 1e-6, residual: bool = True, *, family: str = "generic",
              shared=None, shared_gate_w: torch.Tensor | None = None, bias: torch.Tensor | None = None,
              routed_scale: float = 1.0, hf_rounding: bool = False) -> torch.Tensor:
    """x: (T, H) BF16; experts[e] = (Wg, Wu, Wd) BF16; shared = (Wg, Wu, Wd) of
    the shared expert (qwen35 / glm) or None; shared_gate_w: (H,) BF16 (qwen35).
    Returns x + moe(x) (or moe(x)).  `hf_rounding`: HF transformers' rounding
    points instead of the reference's (see the module docstring)."""
    if family not in FAMILIES:
        raise ValueError(family)
    h = rms_norm(x, norm_w, eps, plus_one=family == "qwen35")
    idx, pw = route(h, wr, k, norm_topk, family, bias, routed_scale)
    groups: dict[int, list[tuple[int, float]]] = {}
    for pos in range(x.shape[0]):
        for j in range(k):
            groups.setdefault(int(idx[pos, j]), []).append((pos, float(pw[pos, j])))
    order = list(groups) if family == "generic" and not hf_rounding else sorted(groups)
    out = torch.zeros_like(h)
    for e in order:
        positions = [p for p, _ in groups[e]]
        w = torch.tensor([wt for _, wt in groups[e]], dtype=torch.float32)
        if family != "glm" and not hf_rounding:
            w = w.to(bf16).float()
        y = swiglu(h[positions], *experts[e], fused_silu=hf_rounding)
        contrib = (y.float() * w[:, None]).to(bf16)
        out[positions] = (out[positions].float() + contrib.float()).to(bf16)
    if shared is not None:
        sh = swiglu(h, *shared, fused_silu=hf_rounding)
        if family == "qwen35":
            gate = torch.sigmoid(_mm(h, shared_gate_w[None, :]).float()).to(bf16)  # (T, 1)
            sh = (gate.float() * sh.float()).to(bf16)
        out = (out.float() + sh.float()).to(bf16)
    return (x.float() + out.float()).to(bf16) if residual else out


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))
