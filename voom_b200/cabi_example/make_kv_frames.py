"""Writes config-5 KV pages as zstd frames for the C-ABI example driver
(kv_decode.cpp): DIR/src.bin (the frames back to back), DIR/jobs.bin
(voom_zstd_job records, K frames then V frames, 32 KiB each) and DIR/raw.bin
(the expected output).

    python -m voom_b200.cabi_example.make_kv_frames DIR [PAGES]
"""

from __future__ import annotations

import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

from voom_b200 import synthetic
from voom_b200.formats import zstd_gpu, zstd_host


def main(out_dir: str, pages: int = 4096) -> None:
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    k, v = synthetic.kv_pages(pages, seed=11)
    planes = [k[i] for i in range(pages)] + [v[i] for i in range(pages)]
    with ThreadPoolExecutor(16) as pool:
        frames = list(pool.map(lambda a: zstd_host.compress(a.tobytes(), 1), planes))
    jobs = np.zeros(len(frames), dtype=zstd_gpu.JOB_DTYPE)
    pos = 0
    for i, f in enumerate(frames):
        jobs[i] = (pos, len(f), i * planes[0].nbytes, planes[0].nbytes, 0, 0, 0)
        pos += len(f)
    np.frombuffer(b"".join(frames), np.uint8).tofile(out / "src.bin")
    jobs.tofile(out / "jobs.bin")
    np.concatenate([p.reshape(-1) for p in planes]).tofile(out / "raw.bin")
    print(f"{len(frames)} frames, {pos} compressed bytes -> {out}")


if __name__ == "__main__":
    main(sys.argv[1], int(sys.argv[2]) if len(sys.argv) > 2 else 4096)
