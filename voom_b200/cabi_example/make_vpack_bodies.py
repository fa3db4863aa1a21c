"""Writes the vpack bodies of a SmolLM2-135M-shaped checkpoint (BASELINE config
2: BF16 N(0, 0.02), hi plane zstd level 1 + raw lo plane per tensor, access
order) for the C-ABI example driver (kv_decode.cpp): DIR/src.bin (the bodies
back to back), DIR/jobs.bin (one interleaved voom_zstd_job per body, outputs
back to back) and DIR/raw.bin (the expected output).

    python -m voom_b200.cabi_example.make_vpack_bodies DIR [LAYERS]
"""

from __future__ import annotations

import sys
import zlib
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

from voom_b200 import synthetic
from voom_b200.formats import packed, packed2


def main(out_dir: str, layers: int = 30) -> None:
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    specs = synthetic.smollm2_tensors(dict(synthetic.SMOLLM2_135M, layers=layers))

    def make(spec):
        name, shape = spec
        bits = synthetic.bf16_normal(shape, 0.02, zlib.crc32(name.encode()))
        head, body = packed.body_for("BF16", bits.view(np.uint8))
        return name, head, body, bits

    with ThreadPoolExecutor(16) as pool:
        items = {n: (h, b, r) for n, h, b, r in pool.map(make, specs)}
    jobs, bodies, raws = [], [], []
    pos = dst = 0
    for name in packed2.access_order(list(items)):
        head, body, bits = items[name]
        job, n = packed.body_job(head, pos, len(body), dst)
        jobs.append(job)
        bodies.append(body)
        raws.append(bits.reshape(-1).view(np.uint8))
        pos += len(body)
        dst += n
    np.frombuffer(b"".join(bodies), np.uint8).tofile(out / "src.bin")
    np.concatenate(jobs).tofile(out / "jobs.bin")
    np.concatenate(raws).tofile(out / "raw.bin")
    print(f"{len(jobs)} bodies, {pos} archive bytes, {dst} decoded bytes -> {out}")


if __name__ == "__main__":
    main(sys.argv[1], int(sys.argv[2]) if len(sys.argv) > 2 else 30)
