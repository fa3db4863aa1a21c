"""GPU parity for bf16_rans: the CUDA decoder (through the C ABI) against the
reference's golden frames, the reference's corruption outcomes, and the CPU
oracle at config-1 size.  Bit-exact is the only bar."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from oracle import rans as orans
from tests.conftest import golden_bytes
from tests.golden.make_golden import apply_mutation

pytestmark = pytest.mark.gpu


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


@pytest.fixture(scope="module")
def R(built_lib):
    from voom_b200.formats import bf16_rans

    return bf16_rans


def test_golden_frames_decode_bit_exact(R, rans_cases):
    for case in rans_cases:
        out = R.decode(golden_bytes(case["frame"]))
        assert sha(out) == case["decoded_sha256"], case["name"]


def test_corrupted_frames_raise_like_reference(R, rans_mutations):
    frames = {}
    mismatches = []
    for m in rans_mutations:
        base = frames.setdefault(m["base"], golden_bytes(f"rans_{m['base']}.bin"))
        bad = apply_mutation(base, m["mutation"])
        try:
            got = "ok:" + sha(R.decode(bad))
        except ValueError as exc:
            got = "error:" + str(exc)
        if got != m["outcome"]:
            mismatches.append((m["base"], m["mutation"], m["outcome"], got))
    assert not mismatches, mismatches[:5]


def test_reference_unit_cases_on_gpu(R):
    # tests/test_bf16_rans.py:19-54, decoded by the GPU
    rng = np.random.default_rng(9)
    for size in (0, 1, 2, 3, 257, 8193):
        raw = rng.integers(0, 256, size=size, dtype=np.uint8).tobytes()
        frame, stats = R.encode(raw, tile_bytes=257)
        assert R.decode(frame) == raw
        assert stats.tiles == (size + 256) // 257
    raw = b"".join(bytes((i & 0xFF, 0x3F)) for i in range(32768))
    frame, stats = R.encode(raw, tile_bytes=16384)
    assert R.decode(frame) == raw and stats.compressed_tiles == stats.tiles and stats.ratio > 1.2
    frame, _ = R.encode(bytes(range(256)) * 20, tile_bytes=1024)
    with pytest.raises(ValueError):
        R.decode(frame[:-3])
    raw = b"".join(bytes((i & 0xFF, 0x3F)) for i in range(8192))
    frame, _ = R.encode(raw, tile_bytes=len(raw))
    bad = bytearray(frame)
    bad[R._FRAME.size + R._TILE.size + R._PLANE.size + R._FREQUENCIES.size] ^= 0x40
    with pytest.raises(ValueError, match="checksum"):
        R.decode(bytes(bad))


@pytest.mark.parametrize("tile_bytes", [1 << 20, 1 << 16])
def test_config1_full_size_round_trip(R, tile_bytes):
    from voom_b200 import synthetic

    raw = synthetic.outlier_matrix(4096, 4096, seed=0).tobytes()
    frame, stats = R.encode(raw, tile_bytes=tile_bytes)
    assert stats.tiles == (len(raw) + tile_bytes - 1) // tile_bytes
    out = R.decode_device(frame)
    assert out.numel() == len(raw)
    got = out.cpu().numpy()
    assert np.array_equal(got, np.frombuffer(raw, np.uint8))
    # the oracle agrees on the same frame
    if tile_bytes == (1 << 20):
        assert orans.crc32(raw) == orans.crc32(got.tobytes())


@pytest.mark.parametrize("every", [64, 256, 1024])
def test_indexed_page_decode_matches(R, every):
    from voom_b200 import synthetic

    raw = synthetic.bf16_normal((1536, 2048), 0.02, seed=3).tobytes()  # 6 MiB
    frame, _ = R.encode(raw, tile_bytes=1 << 18)
    page = R.RansPage(frame, every=every)
    for _ in range(2):
        out = page.decode()
        assert np.array_equal(out.cpu().numpy(), np.frombuffer(raw, np.uint8))


def test_indexed_page_detects_corruption(R):
    from voom_b200 import synthetic

    raw = synthetic.bf16_normal((512, 512), 0.02, seed=4).tobytes()
    frame, _ = R.encode(raw, tile_bytes=1 << 16)
    page = R.RansPage(frame, every=64)
    # flip one renormalisation byte deep inside tile 1's low plane, after indexing
    t1 = page.plan.tiles[1]
    pos = int(t1["low_freq"]) + 512 + 4 + 3000
    page.src[pos] ^= 0x21
    with pytest.raises(ValueError):
        page.decode()


def test_odd_and_unaligned_tiles(R):
    rng = np.random.default_rng(21)
    for tile in (255, 1001, 4097, 65537):
        raw = rng.normal(0, 0.02, size=20000).astype(np.float32)
        raw = (raw.view(np.uint32) >> 16).astype(np.uint16).tobytes()[: 39999]
        frame, _ = R.encode(raw, tile_bytes=tile)
        assert R.decode(frame) == raw, tile
        assert orans.decode(frame) == raw


def test_stream_argument_and_no_host_sync(R):
    from voom_b200 import synthetic

    raw = synthetic.bf16_normal((256, 1024), 0.02, seed=5).tobytes()
    frame, _ = R.encode(raw, tile_bytes=1 << 16)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = R.decode_device(frame, stream=s)
    s.synchronize()
    assert out.cpu().numpy().tobytes() == raw
