"""GPU zstd encoder (voom_zstd_encode, the KV spill codec) through the C ABI:
its frames equal the host build of the same encoder byte for byte
(tests/native/zenc_host.cpp), decompress with libzstd 1.5.5 and with the GPU
decoder to exactly the input, and config-5 pages spilled on the GPU reload
bit-exact through the reference's load path (unpickle + zstd.decompress,
restated in the oracle) and through the GPU reload."""

from __future__ import annotations

import ctypes
import pickle
import shutil
import subprocess

import numpy as np
import pytest
import torch

from oracle import vpack as ov
from oracle import zstd as oz
from tests.test_zstd_enc_cpu import HERE, cases
from tests.test_zstd_enc_cpu import compress as host_compress

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def host_enc(tmp_path_factory):
    cxx = shutil.which("g++") or shutil.which("c++")
    out = tmp_path_factory.mktemp("zenc") / "libzenc_host.so"
    subprocess.run([cxx, "-O2", "-std=c++17", "-shared", "-fPIC", str(HERE / "native" / "zenc_host.cpp"), "-o",
                    str(out)], check=True)
    lib = ctypes.CDLL(str(out))
    lib.zenc_slot_bytes.restype = ctypes.c_uint32
    lib.zenc_encode_block.restype = ctypes.c_uint32
    lib.zenc_encode_block.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32,
                                      ctypes.c_uint32, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]
    return lib


def test_gpu_frames_equal_host_build_and_decode(built_lib, host_enc):
    from voom_b200 import _device
    from voom_b200.formats import zstd_gpu

    items = list(cases())
    datas = [d for _, d in items]
    offs, pos = [], 0
    for d in datas:
        offs.append(pos)
        pos += (len(d) + 15) // 16 * 16
    buf = np.zeros(max(pos, 16), np.uint8)
    for o, d in zip(offs, datas):
        buf[o:o + len(d)] = np.frombuffer(d, np.uint8)
    dev = torch.device("cuda", 0)
    d_src = _device.upload(buf, dev)
    frames = zstd_gpu.compress_many(d_src, offs, [len(d) for d in datas])
    for (name, d), fr in zip(items, frames):
        assert fr == host_compress(host_enc, d), name
        assert oz.libzstd_decompress(fr, max(len(d), 1)) == d, name
    # the GPU decoder reads them back (non-empty frames)
    keep = [(fr, len(d), d) for fr, d in zip(frames, datas) if d]
    out, spans = zstd_gpu.decompress_many([f for f, _, _ in keep], [n for _, n, _ in keep], device=dev)
    got = out.cpu().numpy()
    for (_, _, d), (o, n) in zip(keep, spans):
        assert got[o:o + n].tobytes() == d


def test_kv_pages_spilled_on_gpu_reload_exactly(built_lib):
    """Config-5 pages (16 x 8 x 128 BF16, N(0, 1) x per-head U(0.5, 4)): the
    .kvz pickles made on the GPU load back through the reference's path
    (kv_paged.py:98-113, restated: unpickle + libzstd) and through the GPU
    reload, and compress like libzstd level 1."""
    from voom_b200.runtime import kv_paged

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    n = 2048
    x = torch.randn((n, 2, 1, 8, 16, 128), generator=g, device=dev)
    s = torch.rand((n, 2, 1, 8, 1, 1), generator=g, device=dev) * 3.5 + 0.5
    kv = (x * s).to(torch.bfloat16)
    blobs = kv_paged.spill_pages_gpu(kv[:, 0], kv[:, 1])
    assert len(blobs) == n
    bits = kv.view(torch.int16).cpu().numpy().view(np.uint16)
    for i in range(0, n, 97):  # the reference's load path
        k, v = ov.kv_load(blobs[i])
        assert np.array_equal(k, bits[i, 0]) and np.array_equal(v, bits[i, 1])
        assert pickle.loads(blobs[i])["shape"] == (1, 8, 16, 128)
    K, V = kv_paged.reload_blobs(blobs, dev)  # the GPU reload of all of them
    assert torch.equal(K.view(torch.int16), kv[:, 0].view(torch.int16))
    assert torch.equal(V.view(torch.int16), kv[:, 1].view(torch.int16))
    ours = sum(len(pickle.loads(b)["k"]) + len(pickle.loads(b)["v"]) for b in blobs[:64])
    ref = sum(len(ov.zstd_compress(bits[i, j].tobytes(), 1)) for i in range(64) for j in range(2))
    assert ours < 1.02 * ref, (ours, ref)


def test_paged_cache_spills_compressed_pages_on_gpu(built_lib, tmp_path):
    """PagedKVCache(compress_spill=True) writes .kvz files made by the GPU
    encoder; the reference's loader reads them, and update() reloads them."""
    from voom_b200.runtime import kv_paged

    dev = torch.device("cuda", 0)
    torch.manual_seed(1)
    cache = kv_paged.PagedKVCache(2, max_bytes=4 * 2 * 2 * 8 * 16 * 128 * 2, spill_dir=tmp_path, page_positions=16,
                                  resident_pages=1, compress_spill=True)
    ks, vs = [[] for _ in range(2)], [[] for _ in range(2)]
    for step in range(10):
        for layer in range(2):
            k = torch.randn((1, 8, 16, 128), device=dev).to(torch.bfloat16)
            v = torch.randn((1, 8, 16, 128), device=dev).to(torch.bfloat16)
            ks[layer].append(k)
            vs[layer].append(v)
            K, V = cache.update(layer, k, v)
            assert torch.equal(K, torch.cat(ks[layer], 2)) and torch.equal(V, torch.cat(vs[layer], 2))
    files = sorted(tmp_path.glob("*.kvz"))
    assert files and cache.stats.spills >= len(files)
    for f in files[:3]:
        k, v = ov.kv_load(f.read_bytes())
        assert k.shape == (1, 8, 16, 128)
    cache.release()
    assert not list(tmp_path.glob("*.kvz"))
