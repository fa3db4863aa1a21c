"""Oracle for the MoE expert math -- TEST INFRASTRUCTURE ONLY.

Torch-CPU restatement of the reference's MLX layer math with its BF16
rounding points: runtime/layer_runner.py run_moe_mlp (:347-394) and _swiglu
(:185-190), quant.matmul (runtime/quant.py:431-444: x @ W.T, BF16 result),
mx.fast.rms_norm (one rounding of x * rsqrt(mean(x^2) + eps) * w).
Top-k order: descending probability, ties to the lower expert id (MLX's
argpartition leaves the order unspecified; only the accumulation order
depends on it).
"""

from __future__ import annotations

import torch

bf16 = torch.bfloat16


def _mm(a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """BF16 x @ W.T with fp32 accumulation and a BF16 result."""
    return (a.float() @ w.float().T).to(bf16)


def rms_norm(x: torch.Tensor, w: torch.Tensor | None, eps: float) -> torch.Tensor:
    if w is None:
        return x
    xf = x.float()
    return (xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + eps) * w.float()).to(bf16)


def route(h: torch.Tensor, wr: torch.Tensor, k: int, norm_topk: bool):
    logits = _mm(h, wr).float()
    probs = torch.softmax(logits, dim=-1)
    order = torch.argsort(-probs, dim=-1, stable=True)[:, :k]
    pw = torch.gather(probs, -1, order)
    if norm_topk:
        pw = pw / pw.sum(-1, keepdim=True)
    return order, pw


def swiglu(h: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor, wd: torch.Tensor) -> torch.Tensor:
    g = _mm(h, wg)
    u = _mm(h, wu)
    s = torch.sigmoid(g.float()).to(bf16)
    a = ((s.float() * g.float()).to(bf16).float() * u.float()).to(bf16)
    return _mm(a, wd)


def moe_layer(x: torch.Tensor, wr: torch.Tensor, norm_w: torch.Tensor | None, experts, k: int,
              norm_topk: bool = True, eps: float = 1e-6, residual: bool = True) -> torch.Tensor:
    """x: (T, H) BF16; experts[e] = (Wg, Wu, Wd) BF16.  Returns x + moe(x) (or moe(x))."""
    h = rms_norm(x, norm_w, eps)
    idx, pw = route(h, wr, k, norm_topk)
    groups: dict[int, list[tuple[int, float]]] = {}
    for pos in range(x.shape[0]):
        for j in range(k):
            groups.setdefault(int(idx[pos, j]), []).append((pos, float(pw[pos, j])))
    out = torch.zeros_like(h)
    for e, plist in groups.items():
        positions = [p for p, _ in plist]
        w = torch.tensor([wt for _, wt in plist], dtype=torch.float32).to(bf16)
        y = swiglu(h[positions], *experts[e])
        contrib = (y.float() * w.float()[:, None]).to(bf16)
        out[positions] = (out[positions].float() + contrib.float()).to(bf16)
    return (x.float() + out.float()).to(bf16) if residual else out


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))
