"""The GPU zstd encoder's format logic on the CPU: tests/native/zenc_host.cpp
compiles the kernel's own planning code (voom_b200/csrc/zstd_enc.cuh) for the
host, and every frame it makes must decompress with libzstd 1.5.5 (the
library behind the reference's compression.zstd) and with the oracle's
RFC 8878 decoder to exactly the input: KV pages like config 5's, weight
planes, incompressible and single-valued data, very skewed histograms (code
lengths past 11 bits before limiting), tiny and multi-block inputs."""

from __future__ import annotations

import ctypes
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import zstd as oz

HERE = Path(__file__).resolve().parent
BLOCK = 32768


@pytest.fixture(scope="module")
def enc(tmp_path_factory):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    out = tmp_path_factory.mktemp("zenc") / "libzenc_host.so"
    subprocess.run([cxx, "-O2", "-std=c++17", "-shared", "-fPIC", str(HERE / "native" / "zenc_host.cpp"), "-o",
                    str(out)], check=True)
    lib = ctypes.CDLL(str(out))
    lib.zenc_slot_bytes.restype = ctypes.c_uint32
    lib.zenc_encode_block.restype = ctypes.c_uint32
    lib.zenc_encode_block.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32,
                                      ctypes.c_uint32, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]
    return lib


def compress(lib, data: bytes) -> bytes:
    a = np.frombuffer(data, np.uint8) if data else np.zeros(0, np.uint8)
    slot = np.zeros(lib.zenc_slot_bytes(), np.uint8)
    parts = []
    n = len(data)
    starts = list(range(0, n, BLOCK)) or [0]
    for k, b0 in enumerate(starts):
        blk = np.ascontiguousarray(a[b0:b0 + BLOCK])
        st = ctypes.c_uint32(0)
        ln = lib.zenc_encode_block(blk.ctypes.data if blk.size else None, blk.size, n, int(k == 0),
                                   int(k == len(starts) - 1), slot.ctypes.data, ctypes.byref(st))
        parts.append(slot[st.value:st.value + ln].tobytes())
    return b"".join(parts)


def bf16(x: np.ndarray) -> bytes:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16).tobytes()


def cases():
    rng = np.random.default_rng(5)
    kv = rng.standard_normal((8, 16, 128)).astype(np.float32) * rng.uniform(0.5, 4, (8, 1, 1)).astype(np.float32)
    yield "kv_page", bf16(kv)
    yield "weights_0.02", bf16(rng.standard_normal(20000).astype(np.float32) * 0.02)
    yield "uniform_bytes", rng.integers(0, 256, 40000, dtype=np.uint8).tobytes()
    yield "zeros", bytes(50000)
    yield "two_symbols", rng.choice(np.array([7, 200], np.uint8), 30000).tobytes()
    # geometric histogram: optimal codes far longer than 11 bits before the limit
    p = 0.5 ** np.arange(1, 40)
    sym = np.minimum(rng.geometric(0.5, 32768) - 1, 255).astype(np.uint8)
    yield "geometric", sym.tobytes()
    yield "skewed_full_alphabet", np.concatenate([np.arange(256, dtype=np.uint8),
                                                  np.full(32000, 9, np.uint8)]).tobytes()
    for n in (1, 63, 64, 65, 100, 1000, 1023, 1024, 16383, 16384, 32767):
        yield f"text_{n}", (rng.integers(97, 110, n, dtype=np.uint8)).tobytes()
    yield "multi_block_100k", bf16(rng.standard_normal(50000).astype(np.float32))
    yield "multi_block_200k_mixed", bf16(rng.standard_normal(60000).astype(np.float32)) + bytes(70000) + \
        rng.integers(0, 256, 10000, dtype=np.uint8).tobytes()
    yield "empty", b""
    yield "few_symbols_small", bytes([1, 2, 3] * 30)
    yield "all_256_once_each", bytes(range(256))


@pytest.mark.parametrize("name,data", list(cases()), ids=[c[0] for c in cases()])
def test_frames_decode_with_libzstd_and_oracle(enc, name, data):
    fr = compress(enc, data)
    assert oz.libzstd_decompress(fr, max(len(data), 1)) == data
    assert oz.decompress(fr) == data
    if name in ("kv_page", "weights_0.02"):
        assert len(data) / len(fr) > 1.1, (name, len(data) / len(fr))  # Huffman literals do compress these
    if name in ("uniform_bytes",):
        assert len(fr) <= len(data) + 16  # raw blocks: no growth beyond the headers
    if name == "zeros":
        assert len(fr) < 40


def test_kv_pages_ratio_against_libzstd_level1(enc):
    """Config-5-like pages: the Huffman-literal frames stay within reach of
    libzstd level 1 (reported for the record; the two are different valid
    encodings of the same bytes)."""
    from oracle import vpack as ov

    rng = np.random.default_rng(9)
    ours = ref = raw = 0
    for _ in range(16):
        kv = rng.standard_normal((8, 16, 128)).astype(np.float32) * rng.uniform(0.5, 4, (8, 1, 1)).astype(np.float32)
        b = bf16(kv)
        raw += len(b)
        ours += len(compress(enc, b))
        ref += len(ov.zstd_compress(b, 1))
    assert raw / ours > 1.1 and ours < 1.1 * ref, (raw / ours, raw / ref)
