"""Seeded zstd frames for parity tests, produced the way the reference
produces them (libzstd via compression.zstd: one-shot compress at a level, or
a streaming compressor for tensors above 256 MiB)."""

from __future__ import annotations

import numpy as np

from voom_b200 import synthetic
from voom_b200.formats import zstd_host as zh


def cases(scale: int = 1) -> list[tuple[str, bytes, bytes]]:
    rng = np.random.default_rng(1234)
    hi = synthetic.bf16_normal((scale << 20,), 0.02, 1).view(np.uint8)[1::2].tobytes()
    out = [("hi_plane_l1", zh.compress(hi, 1), hi)]
    for lvl in (-5, 3, 9, 19):
        out.append((f"hi_300k_l{lvl}", zh.compress(hi[:300000], lvl), hi[:300000]))
    out.append(("empty", zh.compress(b"", 1), b""))
    out.append(("three_bytes", zh.compress(b"abc", 1), b"abc"))
    txt = b"the quick brown fox jumps over the lazy dog " * 5000
    out.append(("text_l1", zh.compress(txt, 1), txt))
    out.append(("text_l19", zh.compress(txt, 19), txt))
    rnd = rng.integers(0, 256, 200000, dtype=np.uint8).tobytes()
    out.append(("random_raw_blocks", zh.compress(rnd, 1), rnd))
    zer = bytes(300000)
    out.append(("zeros_rle", zh.compress(zer, 1), zer))
    c = zh.ZstdCompressor(1)
    s = c.compress(hi[: len(hi) // 3]) + c.compress(hi[len(hi) // 3:]) + c.flush()
    out.append(("streamed_no_fcs", s, hi))
    c = zh.ZstdCompressor(3, checksum=True)
    out.append(("streamed_checksum", c.compress(txt) + c.flush(), txt))
    out.append(("concat_frames", zh.compress(b"hello", 1) + zh.compress(b"world" * 100, 1),
                b"hello" + b"world" * 100))
    k, _ = synthetic.kv_pages(2)
    kv = k[0].tobytes()
    out.append(("kv_page_l1", zh.compress(kv, 1), kv))
    runs = b"".join(bytes([i % 7]) * (i % 50 + 1) for i in range(20000))
    out.append(("short_runs", zh.compress(runs, 1), runs))
    return out
