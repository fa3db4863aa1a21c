"""kv_paged spill/reload codec: the reference's unit test
(tests/test_kv_spill_compress.py:22-61) restated on the GPU cache, plus
parity of the .kvz bytes and the batched GPU reload with the oracle codec
(runtime/kv_paged.py:77-113 restated)."""

from __future__ import annotations

import pickle

import numpy as np
import pytest
import torch

from oracle import vpack as ov


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def test_spill_bytes_match_reference_codec():
    """The .kvz bytes written by the spill equal the reference format built by the oracle."""
    from voom_b200.runtime.kv_paged import spill_pages_compressed
    from voom_b200 import synthetic

    k, v = synthetic.kv_pages(3, seed=9)
    ours = spill_pages_compressed(k, v, threads=2)
    for i in range(3):
        assert ours[i] == ov.kv_spill(k[i], v[i])
        kk, vv = ov.kv_load(ours[i])
        assert np.array_equal(kk, k[i]) and np.array_equal(vv, v[i])


@pytest.mark.gpu
def test_compressed_page_round_trips_byte_identical(tmp_path):
    from voom_b200.runtime.kv_paged import PagedKVCache

    kv = PagedKVCache(num_layers=2, max_bytes=1, spill_dir=tmp_path, page_positions=4, resident_pages=0,
                      compress_spill=True)
    g = torch.Generator().manual_seed(0)
    ref_k, ref_v = [], []
    for layer in range(2):
        k = torch.randn((1, 2, 4, 8), generator=g).to(torch.bfloat16).cuda()
        v = torch.randn((1, 2, 4, 8), generator=g).to(torch.bfloat16).cuda()
        ref_k.append(k)
        ref_v.append(v)
        kv.update(layer, k, v)
    for layer in range(2):
        k2 = torch.randn((1, 2, 1, 8), generator=g).to(torch.bfloat16).cuda()
        v2 = torch.randn((1, 2, 1, 8), generator=g).to(torch.bfloat16).cuda()
        K, V = kv.update(layer, k2, v2)
        assert torch.equal(K[:, :, :4], ref_k[layer]) and torch.equal(K[:, :, 4:], k2)
        assert torch.equal(V[:, :, :4], ref_v[layer]) and torch.equal(V[:, :, 4:], v2)
    assert kv.stats.spills > 0
    page = kv._pages[0][0]
    assert not page.resident
    lk, lv = page.load()
    assert lk.dtype == torch.bfloat16 and torch.equal(lk, ref_k[0]) and torch.equal(lv, ref_v[0])
    paths = [p.path for pages in kv._pages for p in pages if p.path is not None]
    assert paths and all(p.exists() for p in paths)
    # the file is the reference format: pickle {"shape", "k", "v"} of zstd frames
    blob = pickle.loads(paths[0].read_bytes())
    assert set(blob) == {"shape", "k", "v"} and tuple(blob["shape"]) == (1, 2, 4, 8)
    kk, vv = ov.kv_load(paths[0].read_bytes())
    assert np.array_equal(kk, bits(ref_k[0])) and np.array_equal(vv, bits(ref_v[0]))
    kv.release()
    assert kv.offset == 0 and kv.nbytes() == 0
    assert not any(p.exists() for p in paths)


@pytest.mark.gpu
def test_uncompressed_spill_round_trip(tmp_path):
    from voom_b200.runtime.kv_paged import PagedKVCache

    kv = PagedKVCache(num_layers=1, max_bytes=1, spill_dir=tmp_path, page_positions=4, resident_pages=0)
    g = torch.Generator().manual_seed(3)
    k = torch.randn((1, 2, 9, 8), generator=g).to(torch.bfloat16).cuda()
    v = torch.randn((1, 2, 9, 8), generator=g).to(torch.bfloat16).cuda()
    K, V = kv.update(0, k, v)
    assert kv.stats.spills == 2
    assert torch.equal(K, k) and torch.equal(V, v)


@pytest.mark.gpu
def test_batched_reload_config5_pages():
    """Config 5 pages (16 x 8 x 128, N(0,1) x U(0.5,4) per head) spilled with the
    reference codec and reloaded by one batched GPU decode, bit-exact."""
    from voom_b200 import synthetic
    from voom_b200.runtime.kv_paged import reload_blobs, spill_pages_compressed

    k, v = synthetic.kv_pages(512, seed=5)
    blobs = spill_pages_compressed(k, v)
    K, V = reload_blobs(blobs)
    assert np.array_equal(bits(K), k) and np.array_equal(bits(V), v)
    raw = k.nbytes + v.nbytes
    assert raw / sum(len(b) for b in blobs) > 1.1
