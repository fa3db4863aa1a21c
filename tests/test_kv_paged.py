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


def _walk(blobs):
    """voom_kvz_gather over `blobs` (native copy + pickle walk, no GPU)."""
    from voom_b200._lib import check, load
    from voom_b200.runtime import kv_paged as kp

    n = len(blobs)
    lens = np.fromiter(map(len, blobs), np.uint64, n)
    offs = np.zeros(n, np.uint64)
    np.cumsum(lens[:-1], out=offs[1:])
    arena = np.zeros(int(lens.sum()) + 16, np.uint8)
    pages = np.zeros(n, kp.KVZ_PAGE_DTYPE)
    addrs = kp._addresses(list(blobs))
    check(load().voom_kvz_gather(addrs.ctypes.data, lens.ctypes.data, offs.ctypes.data, n, arena.ctypes.data,
                                 pages.ctypes.data, 4), "voom_kvz_gather")
    return arena, pages


def test_kvz_walker_matches_pickle_loads():
    """The native .kvz walker finds the same shape and frames as pickle.loads
    for every protocol the reference's pickler may use (3-5), any key order,
    memo gets of a shared bytes object, negative and 64-bit dims; pages it does
    not read (protocol 2, a list shape, a missing key, a foreign value) are
    flagged for the Python unpickler instead of guessed."""
    rng = np.random.default_rng(17)
    blobs, dicts = [], []
    for i in range(600):
        proto = int(rng.choice([2, 3, 4, 5]))
        shape = tuple(int(rng.choice([1, 8, 16, 128, 300, 70000, -1, 2 ** 40])) for _ in range(rng.integers(0, 6)))
        k = rng.integers(0, 256, int(rng.choice([0, 3, 255, 256, 70000])), dtype=np.uint8).tobytes()
        v = rng.integers(0, 256, int(rng.choice([0, 1, 300])), dtype=np.uint8).tobytes()
        d = {"shape": shape, "k": k, "v": v}
        if i % 5 == 0:
            d = {"v": v, "k": k, "shape": shape}
        if i % 7 == 0:
            d = {"shape": shape, "k": k, "v": k}  # one object twice: a memo get
        if i % 11 == 0:
            d = {"shape": list(shape), "k": k, "v": v}
        if i % 13 == 0:
            d = {"shape": shape, "k": k}
        if i % 17 == 0:
            d = {"shape": shape, "k": k, "v": v, "extra": [1]}
        blobs.append(pickle.dumps(d, protocol=proto))
        dicts.append((proto, d))
    arena, pages = _walk(blobs)
    parsed = 0
    for (proto, d), pg in zip(dicts, pages):
        readable = (proto >= 3 and isinstance(d.get("shape"), tuple) and "k" in d and "v" in d
                    and "extra" not in d)
        if not readable:
            assert pg["status"] == 1, d.keys()
            continue
        assert pg["status"] == 0
        parsed += 1
        assert tuple(int(x) for x in pg["shape"][:pg["ndim"]]) == d["shape"]
        assert arena[pg["k_off"]:pg["k_off"] + pg["k_len"]].tobytes() == d["k"]
        assert arena[pg["v_off"]:pg["v_off"] + pg["v_len"]].tobytes() == d["v"]
    assert parsed > 300


def test_kvz_walker_reads_reference_spill_bytes():
    """Pages spilled in the reference format (oracle codec) parse natively."""
    from voom_b200 import synthetic

    k, v = synthetic.kv_pages(4, seed=2)
    blobs = [ov.kv_spill(k[i], v[i]) for i in range(4)]
    arena, pages = _walk(blobs)
    for i, pg in enumerate(pages):
        d = pickle.loads(blobs[i])
        assert pg["status"] == 0 and tuple(pg["shape"][:pg["ndim"]]) == tuple(d["shape"])
        assert arena[pg["k_off"]:pg["k_off"] + pg["k_len"]].tobytes() == d["k"]
        assert arena[pg["v_off"]:pg["v_off"] + pg["v_len"]].tobytes() == d["v"]


@pytest.mark.gpu
def test_reload_takes_unparsed_pages_through_pickle():
    """Pages pickled with protocol 2 (not read natively) reload through the
    Python unpickler in the same batch, bit-exact."""
    from voom_b200 import synthetic
    from voom_b200.formats import zstd_host
    from voom_b200.runtime.kv_paged import reload_blobs

    k, v = synthetic.kv_pages(40, seed=8)
    blobs = []
    for i in range(40):
        d = {"shape": tuple(k[i].shape), "k": zstd_host.compress(k[i].tobytes(), 1),
             "v": zstd_host.compress(v[i].tobytes(), 1)}
        blobs.append(pickle.dumps(d, protocol=2 if i % 3 == 0 else 5))
    K, V = reload_blobs(blobs)
    assert np.array_equal(bits(K), k) and np.array_equal(bits(V), v)


@pytest.mark.gpu
def test_load_pages_mixed_shapes(tmp_path):
    """load_pages reloads compressed pages of different shapes in one batch."""
    from voom_b200.runtime.kv_paged import _Page, load_pages

    g = torch.Generator().manual_seed(4)
    pages, refs = [], []
    for i, shape in enumerate([(1, 2, 4, 8), (1, 3, 5, 7), (1, 8, 16, 128), (1, 1, 1, 1)]):
        k = torch.randn(shape, generator=g).to(torch.bfloat16).cuda()
        v = torch.randn(shape, generator=g).to(torch.bfloat16).cuda()
        p = _Page(k, v)
        p.spill(tmp_path / f"p{i}.safetensors", compress=True)
        pages.append(p)
        refs.append((k, v))
    got = load_pages(pages)
    for (k, v), (gk, gv) in zip(refs, got):
        assert gk.shape == k.shape and torch.equal(gk, k) and torch.equal(gv, v)


@pytest.mark.gpu
def test_reload_corrupt_frame_raises():
    """A truncated frame inside one page fails the whole reload with ZstdError."""
    from voom_b200 import synthetic
    from voom_b200.formats.zstd_gpu import ZstdError
    from voom_b200.runtime.kv_paged import reload_blobs, spill_pages_compressed

    k, v = synthetic.kv_pages(6, seed=1)
    blobs = spill_pages_compressed(k, v)
    d = pickle.loads(blobs[3])
    d["k"] = d["k"][:-40]
    blobs[3] = pickle.dumps(d)
    with pytest.raises(ZstdError):
        reload_blobs(blobs)
