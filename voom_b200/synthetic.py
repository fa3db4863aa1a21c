"""Seeded synthetic inputs with the shapes and value distributions of the
workloads the reference path is measured on (no checkpoints or datasets are
available offline).  All generators use numpy's default_rng(seed) and round
fp32 to BF16 with round-to-nearest-even.
"""

from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> BF16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return rounded.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def bf16_normal(shape, std: float, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return f32_to_bf16_bits(rng.standard_normal(size=shape, dtype=np.float32) * np.float32(std))


def outlier_matrix(rows: int = 4096, cols: int = 4096, std: float = 0.02, seed: int = 0,
                   outlier_frac: float = 0.001, scale: float = 50.0) -> np.ndarray:
    """Config 1: BF16 N(0, std) with `outlier_frac` of the columns scaled x`scale`."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(size=(rows, cols), dtype=np.float32) * np.float32(std)
    n_out = max(1, int(round(cols * outlier_frac)))
    cols_sel = rng.choice(cols, size=n_out, replace=False)
    x[:, cols_sel] *= np.float32(scale)
    return f32_to_bf16_bits(x)


# Config 2: SmolLM2-135M tensor shapes (30 layers, hidden 576, intermediate
# 1536, 9 query heads / 3 KV heads x head_dim 64, vocab 49152), HF names.
SMOLLM2_135M = dict(layers=30, hidden=576, intermediate=1536, heads=9, kv_heads=3, head_dim=64,
                    vocab=49152)


def smollm2_tensors(cfg: dict | None = None) -> list[tuple[str, tuple[int, ...]]]:
    c = dict(SMOLLM2_135M if cfg is None else cfg)
    h, i, hd = c["hidden"], c["intermediate"], c["head_dim"]
    q, kv = c["heads"] * hd, c["kv_heads"] * hd
    out: list[tuple[str, tuple[int, ...]]] = [("model.embed_tokens.weight", (c["vocab"], h))]
    for layer in range(c["layers"]):
        p = f"model.layers.{layer}."
        out += [
            (p + "input_layernorm.weight", (h,)),
            (p + "self_attn.q_proj.weight", (q, h)),
            (p + "self_attn.k_proj.weight", (kv, h)),
            (p + "self_attn.v_proj.weight", (kv, h)),
            (p + "self_attn.o_proj.weight", (h, q)),
            (p + "post_attention_layernorm.weight", (h,)),
            (p + "mlp.gate_proj.weight", (i, h)),
            (p + "mlp.up_proj.weight", (i, h)),
            (p + "mlp.down_proj.weight", (h, i)),
        ]
    out.append(("model.norm.weight", (h,)))
    return out


def kv_pages(n_pages: int, heads: int = 8, positions: int = 16, head_dim: int = 128,
             seed: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Config 5: K and V pages (n, 1, H, P, D) BF16, N(0, 1) x per-head U(0.5, 4)."""
    rng = np.random.default_rng(seed)
    shape = (n_pages, 1, heads, positions, head_dim)
    out = []
    for _ in range(2):
        x = rng.standard_normal(size=shape, dtype=np.float32)
        scale = rng.uniform(0.5, 4.0, size=(n_pages, 1, heads, 1, 1)).astype(np.float32)
        out.append(f32_to_bf16_bits(x * scale))
    return out[0], out[1]
