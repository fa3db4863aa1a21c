"""WarmTier (runtime/warm_tier.py:22-103 of the reference): admission rules,
budget, frames checked against libzstd through the oracle on CPU; `take` /
`take_many` (batched GPU decode) and the weight-cache miss path on the GPU."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import vpack as ov
from oracle import zstd as oz
from voom_b200.runtime.warm_tier import WarmTier


def _bf16_page(seed: int, rows: int = 64, cols: int = 256) -> dict:
    g = torch.Generator().manual_seed(seed)
    return {"w": (torch.randn((rows, cols), generator=g) * 0.02).to(torch.bfloat16),
            "b": (torch.randn((cols,), generator=g) * 0.02).to(torch.bfloat16)}


def _raw(t: torch.Tensor) -> bytes:
    return t.contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()


def test_admit_frames_are_libzstd_level1_of_raw_bytes():
    tier = WarmTier(1 << 30, threads=2)
    page = _bf16_page(1)
    tier.admit("p", page)
    assert tier.admits == 1 and "p" in tier
    comp = tier._held["p"].frames
    assert [(n, k, s) for n, k, s, _ in comp] == [("w", "bf16", (64, 256)), ("b", "bf16", (256,))]
    for (name, _, _, frame) in comp:
        raw = _raw(page[name])
        assert frame == ov.zstd_compress(raw, 1)
        assert oz.libzstd_decompress(frame, len(raw)) == raw
    assert tier.resident_bytes == sum(len(c) for *_, c in comp)


def test_incompressible_and_unsupported_pages_are_rejected():
    tier = WarmTier(1 << 30)
    rnd = torch.from_numpy(np.random.default_rng(0).integers(0, 256, 1 << 16, dtype=np.uint8))
    tier.admit("u8", {"q": rnd})  # ~1.0x: below MIN_RATIO
    tier.admit("i32", {"x": torch.zeros(16, dtype=torch.int32)})
    tier.admit("obj", {"x": object()})
    assert tier.rejects == 3 and tier.admits == 0 and tier.resident_bytes == 0
    tier.admit("f32", {"x": torch.zeros(4096, dtype=torch.float32)})
    tier.admit("u8z", {"x": torch.zeros(4096, dtype=torch.uint8)})
    assert tier.admits == 2


def test_budget_drops_oldest_admissions_and_duplicates_are_ignored():
    one = WarmTier(1 << 30)
    one.admit("x", _bf16_page(0))
    size = one.resident_bytes
    tier = WarmTier(int(size * 2.5))
    for i in range(4):
        tier.admit(f"p{i}", _bf16_page(i))
    tier.admit("p3", _bf16_page(99))  # already held: ignored
    assert tier.keys() == ["p2", "p3"]
    assert tier.admits == 4 and tier.resident_bytes <= tier.max_bytes
    assert "warm tier: 0 hits, 4 admits, 0 rejects" in tier.summary()


@pytest.mark.gpu
def test_take_round_trip_bit_exact_and_batched():
    dev = torch.device("cuda:0")
    tier = WarmTier(1 << 30, device=dev)
    pages = {f"p{i}": {k: v.to(dev) for k, v in _bf16_page(i, rows=128 + i, cols=512).items()} for i in range(3)}
    pages["f"] = {"x": (torch.arange(3000) % 17).float().to(dev),
                  "m": torch.zeros((7, 33), dtype=torch.uint8, device=dev)}
    for k, p in pages.items():
        tier.admit(k, p)
    assert tier.admits == 4
    got = tier.take("p1")
    assert set(got) == {"w", "b"}
    for n, t in got.items():
        assert t.is_cuda and t.dtype == torch.bfloat16 and t.shape == pages["p1"][n].shape
        assert torch.equal(t.view(torch.int16), pages["p1"][n].view(torch.int16))
    assert tier.take("p1") is None
    many = tier.take_many(["p0", "missing", "p2", "f"])
    assert many["missing"] is None
    for k in ("p0", "p2", "f"):
        for n, t in many[k].items():
            ref = pages[k][n]
            assert t.dtype == ref.dtype and t.shape == ref.shape
            assert torch.equal(t.view(torch.uint8), ref.view(torch.uint8))
    assert tier.hits == 4 and tier.resident_bytes == 0
