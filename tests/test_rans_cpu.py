"""CPU tests for the bf16_rans path: the oracle pinned against the reference's
golden frames and corruption outcomes, the library's pack-side encoder, and
the host-side frame walk (plan + resolve) of the C ABI."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from tests.conftest import golden_bytes
from oracle import rans as orans
from tests.golden.make_golden import apply_mutation, make_input


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def test_oracle_encode_matches_reference_frames(rans_cases):
    for case in rans_cases:
        raw = make_input(case)
        assert sha(raw) == case["input_sha256"], case["name"]
        frame, stats = orans.encode(raw, tile_bytes=case["tile_bytes"])
        assert frame == golden_bytes(case["frame"]), case["name"]
        assert stats["tiles"] == case["tiles"] and stats["compressed_tiles"] == case["compressed_tiles"]


def test_oracle_decode_matches_reference(rans_cases):
    for case in rans_cases:
        out = orans.decode(golden_bytes(case["frame"]))
        assert sha(out) == case["decoded_sha256"], case["name"]


def test_oracle_corruption_outcomes_match_reference(rans_mutations):
    frames = {}
    for m in rans_mutations:
        base = frames.setdefault(m["base"], golden_bytes(f"rans_{m['base']}.bin"))
        bad = apply_mutation(base, m["mutation"])
        try:
            got = "ok:" + sha(orans.decode(bad))
        except ValueError as exc:
            got = "error:" + str(exc)
        assert got == m["outcome"], (m["base"], m["mutation"])


def test_reference_unit_cases_on_oracle():
    # tests/test_bf16_rans.py:19-54 restated against the oracle
    rng = np.random.default_rng(5)
    for size in (0, 1, 2, 3, 257, 8193):
        raw = rng.integers(0, 256, size=size, dtype=np.uint8).tobytes()
        frame, stats = orans.encode(raw, tile_bytes=257)
        assert orans.decode(frame) == raw
        assert stats["tiles"] == (size + 256) // 257
    frame, _ = orans.encode(bytes(range(256)) * 20, tile_bytes=1024)
    with pytest.raises(ValueError):
        orans.decode(frame[:-3])
    raw = b"".join(bytes((i & 0xFF, 0x3F)) for i in range(8192))
    frame, stats = orans.encode(raw, tile_bytes=len(raw))
    assert stats["compressed_tiles"] == 1
    bad = bytearray(frame)
    bad[16 + 13 + 4 + 512] ^= 0x40
    with pytest.raises(ValueError, match="checksum"):
        orans.decode(bytes(bad))


def test_library_encoder_is_byte_identical(built_lib, rans_cases):
    from voom_b200.formats import bf16_rans

    for case in rans_cases:
        raw = make_input(case)
        for threads in (1, 3):
            frame, stats = bf16_rans.encode(raw, tile_bytes=case["tile_bytes"], threads=threads)
            assert frame == golden_bytes(case["frame"]), (case["name"], threads)
            assert stats.tiles == case["tiles"]
            assert stats.compressed_tiles == case["compressed_tiles"]


def test_library_encoder_c1_shape_matches_oracle(built_lib):
    # a quarter of config 1 (1024 x 4096 with outlier columns), 1 MiB tiles
    from voom_b200 import synthetic
    from voom_b200.formats import bf16_rans

    raw = synthetic.outlier_matrix(1024, 4096, seed=0).tobytes()
    frame, stats = bf16_rans.encode(raw, tile_bytes=1 << 20)
    ref, _ = orans.encode(raw, tile_bytes=1 << 20)
    assert frame == ref
    assert stats.ratio > 1.3


def test_host_plan_structural_errors_match_reference(built_lib, rans_mutations):
    """With no decode-time error reported, resolve() must give the reference's
    first error whenever that error is structural (header / bounds / totals)."""
    from voom_b200.formats import bf16_rans

    structural = {"truncated rANS frame", "not a vOOM rANS frame", "truncated rANS tile header",
                  "truncated rANS tile payload", "raw rANS tile size mismatch",
                  "truncated rANS plane header", "truncated rANS plane payload",
                  "invalid rANS frequency total", "compressed rANS tile has trailing bytes",
                  "rANS frame length mismatch"}
    frames = {}
    checked = 0
    for m in rans_mutations:
        msg = m["outcome"][6:] if m["outcome"].startswith("error:") else None
        if msg is None or not (msg in structural or msg.startswith("unknown rANS tile mode")):
            continue
        base = frames.setdefault(m["base"], golden_bytes(f"rans_{m['base']}.bin"))
        bad = apply_mutation(base, m["mutation"])
        p = bf16_rans.plan(bad)
        code = bf16_rans.resolve(p, np.zeros(p.info.n_tiles, np.uint32))
        assert code != 0, m
        from voom_b200._lib import RANS_MESSAGES

        assert RANS_MESSAGES[code].format(mode=p.info.bad_mode) == msg, m
        checked += 1
    assert checked > 50


def test_host_plan_of_valid_frames(built_lib, rans_cases):
    from voom_b200.formats import bf16_rans

    for case in rans_cases:
        p = bf16_rans.plan(golden_bytes(case["frame"]))
        assert p.info.struct_error == 0
        assert p.info.n_tiles == case["tiles"]
        assert p.out_bytes == case["raw_bytes"] == p.raw_size
        modes = p.tiles["mode"]
        assert int((modes == 1).sum()) == case["compressed_tiles"]
