"""PagedKVCache: KV cache with fixed-size pages that spill to disk under a byte
budget and page back in for every attention call (GPU codec).

Same behaviour and files as vOOM's runtime/kv_paged.py (:116-240): closed
pages of `page_positions` positions, the newest `resident_pages` closed pages
of each layer kept resident, oldest pages spilled first (round-robin over
layers) once `nbytes()` exceeds `max_bytes`, and every spilled page of a layer
reloaded transiently at each `update()`.  Spill files:
  compress_spill=False: safetensors with tensors "k" and "v";
  compress_spill=True : `.kvz` = pickle of {"shape", "k": zstd(raw K, 1),
                        "v": zstd(raw V, 1)} (kv_paged.py:77-91),
byte-identical to the reference's.  K/V are CUDA BF16 tensors (1, H, P, D).
Reload decodes the zstd frames of all spilled pages of the layer in ONE
batched GPU decode (kv_paged.py:98-113 did one CPU zstd.decompress per
tensor).  Spill compresses on a host thread pool with libzstd level 1, the
reference's own codec call.

Reference interface replaced: runtime/kv_paged.py:35-240.
"""

from __future__ import annotations

import itertools
import json
import pickle
import struct
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from .. import _device
from .._lib import check, load
from ..formats import zstd_host
from ..formats.zstd_gpu import JOB_DTYPE, ZstdBatch, ZstdError, ZstdPlan, describe


@dataclass
class KVStats:
    spills: int = 0
    reloads: int = 0
    spill_s: float = 0.0
    reload_s: float = 0.0
    spill_bytes_raw: int = 0
    spill_bytes_compressed: int = 0

    def summary(self) -> str:
        base = (f"kv: {self.spills} pages spilled ({self.spill_s:.2f}s), "
                f"{self.reloads} page reloads ({self.reload_s:.2f}s)")
        if self.spill_bytes_compressed:
            ratio = self.spill_bytes_raw / self.spill_bytes_compressed
            base += (f", compress {ratio:.2f}x ({self.spill_bytes_raw / 1e6:.1f}"
                     f"->{self.spill_bytes_compressed / 1e6:.1f}MB)")
        return base


def _bf16_to_raw(t: torch.Tensor) -> bytes:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().tobytes()


def _write_safetensors_raw(path: Path, tensors: dict[str, tuple[tuple, np.ndarray]]) -> None:
    """safetensors file of BF16 tensors given as (shape, int16 bit array)."""
    header, blobs, off = {}, [], 0
    for name, (shape, bits) in tensors.items():
        raw = np.ascontiguousarray(bits).tobytes()
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hj = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)) + hj)
        for b in blobs:
            f.write(b)


def _write_safetensors(path: Path, tensors: dict[str, torch.Tensor]) -> None:
    _write_safetensors_raw(path, {n: (tuple(t.shape), t.detach().contiguous().view(torch.int16).cpu().numpy())
                                  for n, t in tensors.items()})


def _read_safetensors(path: Path, device) -> dict[str, torch.Tensor]:
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        a, b = meta["data_offsets"]
        arr = np.frombuffer(data[a:b], np.int16).reshape(meta["shape"])
        out[name] = torch.from_numpy(arr.copy()).to(device).view(torch.bfloat16)
    return out


class _Page:
    __slots__ = ("k", "v", "path", "nbytes", "_compressed", "shape", "device")

    def __init__(self, k: torch.Tensor, v: torch.Tensor):
        self.k, self.v = k, v
        self.path: Path | None = None
        self.nbytes = k.numel() * k.element_size() + v.numel() * v.element_size()
        self._compressed = False
        self.shape = tuple(k.shape)
        self.device = k.device

    @property
    def resident(self) -> bool:
        return self.k is not None

    def spill(self, path: Path, compress: bool = False) -> int | None:
        """Writes this page out (spill_batch of one page); returns the
        compressed byte count if compress=True, else None."""
        return spill_batch([self], [path], compress, None)

    def load(self) -> tuple[torch.Tensor, torch.Tensor]:
        if self.resident:
            return self.k, self.v
        return load_pages([self])[0]


KVZ_PAGE_DTYPE = np.dtype([("k_off", "<u8"), ("k_len", "<u8"), ("v_off", "<u8"), ("v_len", "<u8"),
                           ("shape", "<i8", (8,)), ("ndim", "<u4"), ("status", "<u4")])
assert KVZ_PAGE_DTYPE.itemsize == 104

_arenas: dict = {}
_arenas_lock = threading.Lock()


def _addresses(blobs: list) -> np.ndarray:
    """Host addresses of the blobs' bytes, read through the buffer protocol
    (the blobs stay referenced by the caller while the addresses are used)."""
    from .. import _hostbuf

    out = np.empty(len(blobs), np.uint64)
    _hostbuf.addresses(blobs, out)
    return out


def _arena(device: torch.device) -> _device.PinnedArena:
    with _arenas_lock:
        a = _arenas.get(device.index)
        if a is None:
            a = _arenas[device.index] = _device.PinnedArena()
        return a


def _reload(blobs: list, dev: torch.device, same_shape: bool):
    """Gather the .kvz pages into the device's pinned arena, walk their
    pickles (pages the native walker does not read are unpickled here), plan
    every K and V frame, upload once and decode in one batch.  Returns the
    output buffer, each page's shape (a list), and arrays of each page's K
    offset, K-to-V distance and bytes per plane."""
    n = len(blobs)
    blobs = list(blobs)
    lens = np.fromiter(map(len, blobs), np.uint64, n)
    offs = np.zeros(n, np.uint64)
    if n > 1:
        np.cumsum(lens[:-1], out=offs[1:])
    total = int(lens.sum())
    addrs = _addresses(blobs)
    pages = np.zeros(n, KVZ_PAGE_DTYPE)
    arena = _arena(dev)
    with arena.lock:
        buf = arena.get(total + _device.PAD)
        host = buf.numpy()
        check(load().voom_kvz_gather(addrs.ctypes.data, lens.ctypes.data, offs.ctypes.data, n, buf.data_ptr(),
                                     pages.ctypes.data, 0), "voom_kvz_gather")
        bad = np.nonzero(pages["status"])[0]
        if bad.size:
            extra = []
            for i in bad:
                d = pickle.loads(blobs[i])
                shape = tuple(int(x) for x in d["shape"])
                extra.append((int(i), shape, bytes(d["k"]), bytes(d["v"])))
            need = total + sum(len(k) + len(v) for _, _, k, v in extra) + _device.PAD
            if need > buf.numel():
                old = host[:total].copy()
                buf = arena.get(need)
                host = buf.numpy()
                host[:total] = old
            pos = total
            for i, shape, k, v in extra:
                pg = pages[i]
                pg["ndim"] = len(shape)
                pg["shape"][:len(shape)] = shape
                for key, fr in (("k", k), ("v", v)):
                    host[pos:pos + len(fr)] = np.frombuffer(fr, np.uint8)
                    pg[key + "_off"], pg[key + "_len"] = pos, len(fr)
                    pos += len(fr)
            total = pos
        ndim = pages["ndim"].astype(np.int64)
        shp = pages["shape"]
        dims = np.where(np.arange(8)[None, :] < ndim[:, None], shp, 1)
        nbytes = dims.prod(axis=1) * 2
        if (shp < 0).any() or (ndim > 8).any():
            raise ValueError("negative dimensions in a .kvz page shape")
        shapes = [tuple(int(x) for x in shp[i, :ndim[i]]) for i in range(n)] if not same_shape else None
        if same_shape:
            if n and (ndim != ndim[0]).any() or n and (shp != shp[0]).any():
                raise ValueError("reload_blobs needs pages of one shape")
            shapes = [tuple(int(x) for x in shp[0, :ndim[0]])] * n if n else []
        span = (nbytes + 255) // 256 * 256
        dst = np.zeros(n, np.int64)
        if n > 1:
            np.cumsum(2 * span[:-1], out=dst[1:])
        jobs = np.zeros(2 * n, dtype=JOB_DTYPE)
        jobs["src"][0::2], jobs["src_len"][0::2] = pages["k_off"], pages["k_len"]
        jobs["src"][1::2], jobs["src_len"][1::2] = pages["v_off"], pages["v_len"]
        jobs["dst"][0::2], jobs["dst"][1::2] = dst, dst + span
        jobs["dst_len"][0::2] = jobs["dst_len"][1::2] = nbytes
        out_bytes = int(dst[-1] + 2 * span[-1]) if n else 0
        with torch.cuda.device(dev):
            d_src = _device.upload(buf[:total], dev)  # one async DMA from pinned memory
            plan = ZstdPlan(host[:total], jobs)       # host plan overlaps the DMA
            out = torch.empty(max(out_bytes, 1), dtype=torch.uint8, device=dev)
            batch = ZstdBatch(plan, dev)
            batch.run(d_src, out)
            st = batch.job_status()                    # waits for the decode (and the DMA)
    if st.any():
        raise ZstdError(describe(int(st[np.nonzero(st)[0][0]])))
    return out, shapes, dst, span, nbytes


def load_pages(pages: list[_Page]) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Reload spilled pages: every zstd frame of every compressed page in one
    batched GPU decode; uncompressed pages through safetensors."""
    out: list = [None] * len(pages)
    comp = [(i, p) for i, p in enumerate(pages) if not p.resident and p._compressed]
    for i, p in enumerate(pages):
        if p.resident:
            out[i] = (p.k, p.v)
        elif not p._compressed:
            d = _read_safetensors(p.path, p.device)
            out[i] = (d["k"], d["v"])
    if not comp:
        return out
    dev = comp[0][1].device
    blobs = []
    for _, p in comp:
        with open(p.path, "rb") as f:
            blobs.append(f.read())
    buf, shapes, dst, span, nbytes = _reload(blobs, dev, same_shape=False)
    for k, (i, _p) in enumerate(comp):
        kd, n = int(dst[k]), int(nbytes[k])
        vd = kd + int(span[k])
        out[i] = (buf[kd:kd + n].view(torch.bfloat16).reshape(shapes[k]),
                  buf[vd:vd + n].view(torch.bfloat16).reshape(shapes[k]))
    return out


class PagedKVCache:
    """Drop-in replacement for KVCache: update()/offset/nbytes()/release()."""

    def __init__(self, num_layers: int, max_bytes: int, spill_dir: str | Path, page_positions: int = 256,
                 resident_pages: int = 1, compress_spill: bool = False, spill_threads: int = 8):
        self.num_layers = num_layers
        self.max_bytes = max_bytes
        self.page_positions = page_positions
        self.resident_pages = resident_pages
        self.compress_spill = compress_spill
        self.spill_dir = Path(spill_dir)
        self.spill_dir.mkdir(parents=True, exist_ok=True)
        self._pages: list[list[_Page]] = []
        self._tail_k: list[torch.Tensor | None] = []
        self._tail_v: list[torch.Tensor | None] = []
        self._reset()
        self.stats = KVStats()
        self._pool = ThreadPoolExecutor(max_workers=max(1, spill_threads))

    def update(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        if self._tail_k[layer] is None:
            self._tail_k[layer], self._tail_v[layer] = k, v
        else:
            self._tail_k[layer] = torch.cat([self._tail_k[layer], k], dim=2)
            self._tail_v[layer] = torch.cat([self._tail_v[layer], v], dim=2)
        while self._tail_k[layer].shape[2] >= self.page_positions:
            pk = self._tail_k[layer][:, :, : self.page_positions, :].contiguous()
            pv = self._tail_v[layer][:, :, : self.page_positions, :].contiguous()
            self._pages[layer].append(_Page(pk, pv))
            self._tail_k[layer] = self._tail_k[layer][:, :, self.page_positions:, :].contiguous()
            self._tail_v[layer] = self._tail_v[layer][:, :, self.page_positions:, :].contiguous()
        if layer == self.num_layers - 1:
            self._offset += k.shape[2]
            self._enforce_budget()
        pages = self._pages[layer]
        spilled = [p for p in pages if not p.resident]
        if spilled:
            t0 = time.perf_counter()
            loaded = load_pages(spilled)
            self.stats.reloads += len(spilled)
            self.stats.reload_s += time.perf_counter() - t0
            it = iter(loaded)
            parts = [(p.k, p.v) if p.resident else next(it) for p in pages]
        else:
            parts = [(p.k, p.v) for p in pages]
        parts_k = [a for a, _ in parts]
        parts_v = [b for _, b in parts]
        if self._tail_k[layer].shape[2] > 0 or not parts_k:
            parts_k.append(self._tail_k[layer])
            parts_v.append(self._tail_v[layer])
        if len(parts_k) == 1:
            return parts_k[0], parts_v[0]
        return torch.cat(parts_k, dim=2), torch.cat(parts_v, dim=2)

    @property
    def offset(self) -> int:
        return self._offset

    def nbytes(self) -> int:
        total = 0
        for layer in range(self.num_layers):
            total += sum(p.nbytes for p in self._pages[layer] if p.resident)
            if self._tail_k[layer] is not None:
                total += self._tail_k[layer].numel() * 2 + self._tail_v[layer].numel() * 2
        return total

    def release(self) -> None:
        """Drops every page and tail and deletes the spill files this cache
        wrote -- and only those (runtime/kv_paged.py:196-212)."""
        files = {pg.path for pg in itertools.chain.from_iterable(self._pages) if pg.path is not None}
        self._reset()
        for f in files:
            f.unlink(missing_ok=True)

    def _reset(self) -> None:
        self._pages = [[] for _ in range(self.num_layers)]
        self._tail_k = [None] * self.num_layers
        self._tail_v = [None] * self.num_layers
        self._offset = 0

    def _spill_victims(self) -> list[tuple[int, int]]:
        """(page index, layer) of the pages that must leave HBM for nbytes() to
        fit max_bytes.  Candidates are the resident closed pages outside each
        layer's newest `resident_pages`, taken oldest page index first and in
        layer order within an index (the reference's round-robin,
        runtime/kv_paged.py:216-240); the victims are the shortest prefix whose
        bytes cover the excess, the pages the reference spills one by one."""
        excess = self.nbytes() - self.max_bytes
        if excess <= 0:
            return []
        cands = sorted((i, layer) for layer, pages in enumerate(self._pages)
                       for i in range(len(pages) - self.resident_pages) if pages[i].resident)
        victims = []
        for i, layer in cands:
            if excess <= 0:
                break
            victims.append((i, layer))
            excess -= self._pages[layer][i].nbytes
        return victims

    def _enforce_budget(self) -> None:
        victims = self._spill_victims()
        if not victims:
            return
        t0 = time.perf_counter()
        pages = [self._pages[layer][i] for i, layer in victims]
        paths = [self.spill_dir / f"kv_l{layer}_p{i}.safetensors" for i, layer in victims]
        comp = spill_batch(pages, paths, self.compress_spill, self._pool)
        self.stats.spills += len(pages)
        self.stats.spill_s += time.perf_counter() - t0
        if comp is not None:
            self.stats.spill_bytes_raw += sum(pg.nbytes for pg in pages)
            self.stats.spill_bytes_compressed += comp


def spill_batch(pages: list[_Page], paths: list[Path], compress: bool,
                pool: ThreadPoolExecutor | None) -> int | None:
    """Spills resident pages together and drops their device tensors.
    Compressed spills write the reference's `.kvz` (a pickle of {"shape", "k":
    zstd frame of raw K, "v": zstd frame of raw V}, kv_paged.py:77-91) with
    every frame made by the GPU encoder in one launch (frames the reference's
    zstd.decompress reads back exactly) and return the compressed byte total;
    uncompressed spills copy K and V to the host in one copy and write
    safetensors with tensors "k" and "v", returning None.  Files are written
    on `pool` (or the calling thread)."""
    if not pages:
        return 0 if compress else None
    if compress and pages[0].k.is_cuda and all(pg.shape == pages[0].shape for pg in pages):
        # every K and V frame compressed in one GPU launch; only frames cross to the host
        blobs = spill_pages_gpu(torch.stack([pg.k for pg in pages]), torch.stack([pg.v for pg in pages]))

        def write_kvz(j: int) -> int:
            with open(paths[j].with_suffix(".kvz"), "wb") as f:
                f.write(blobs[j])
            d = pickle.loads(blobs[j])
            return len(d["k"]) + len(d["v"])

        sizes = list((pool.map if pool is not None else map)(write_kvz, range(len(pages))))
        for pg, path in zip(pages, paths):
            pg.path = path.with_suffix(".kvz")
            pg._compressed = True
            pg.k = pg.v = None
        return sum(sizes)
    flat = torch.cat([t.detach().reshape(-1) for pg in pages for t in (pg.k, pg.v)])
    host = flat.view(torch.int16).cpu().numpy()
    pos, slices = 0, []
    for pg in pages:
        n = pg.k.numel()
        slices.append((host[pos:pos + n], host[pos + n:pos + 2 * n]))
        pos += 2 * n

    def write(j: int) -> int:
        pg, (k, v) = pages[j], slices[j]
        if compress:
            kc, vc = zstd_host.compress(k.tobytes(), 1), zstd_host.compress(v.tobytes(), 1)
            with open(paths[j].with_suffix(".kvz"), "wb") as f:
                pickle.dump({"shape": pg.shape, "k": kc, "v": vc}, f)
            return len(kc) + len(vc)
        _write_safetensors_raw(paths[j], {"k": (pg.shape, k), "v": (pg.shape, v)})
        return 0

    sizes = list((pool.map if pool is not None else map)(write, range(len(pages))))
    for pg, path in zip(pages, paths):
        pg.path = path.with_suffix(".kvz") if compress else path
        pg._compressed = compress
        pg.k = pg.v = None
    return sum(sizes) if compress else None


def spill_pages_gpu(k: torch.Tensor, v: torch.Tensor, *, stream: torch.cuda.Stream | None = None,
                    pinned: torch.Tensor | None = None) -> list[bytes]:
    """The `.kvz` bytes of many pages at once, compressed on the GPU: k and v
    are (n, *shape) BF16 device tensors (a page's K is k[i]).  Every K and V
    becomes one zstd frame in one launch of the GPU encoder
    (zstd_gpu.compress_many: Huffman-coded literals, valid frames the
    reference's zstd.decompress reads back exactly), the frames cross to the
    host in one copy, and each page is pickled as {"shape", "k", "v"}
    (runtime/kv_paged.py:79-91)."""
    from ..formats import zstd_gpu

    n = int(k.shape[0])
    if n == 0:
        return []
    shape = tuple(int(x) for x in k.shape[1:])
    per = int(np.prod(shape)) * 2
    flat = torch.stack([k.reshape(n, -1), v.reshape(n, -1)], dim=1).contiguous().view(torch.uint8).reshape(-1)
    offs = np.arange(2 * n, dtype=np.int64) * per
    frames = zstd_gpu.compress_many(flat, offs, np.full(2 * n, per, np.int64), stream=stream, pinned=pinned)
    return [pickle.dumps({"shape": shape, "k": frames[2 * i], "v": frames[2 * i + 1]}) for i in range(n)]


def spill_pages_compressed(pages_k: np.ndarray, pages_v: np.ndarray, threads: int = 8) -> list[bytes]:
    """Spill many pages at once (host thread pool): the .kvz bytes of each page
    (n, 1, H, P, D) uint16 BF16 bits -> list of pickles."""

    def one(i):
        shape = tuple(int(x) for x in pages_k[i].shape)
        return pickle.dumps({"shape": shape, "k": zstd_host.compress(pages_k[i].tobytes(), 1),
                             "v": zstd_host.compress(pages_v[i].tobytes(), 1)})

    with ThreadPoolExecutor(max_workers=max(1, threads)) as pool:
        return list(pool.map(one, range(len(pages_k))))


def reload_blobs(blobs: list[bytes], device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """Decode many .kvz pages (all of one shape) in one batched GPU decode ->
    (K, V) stacked on a leading page axis (views of one device buffer)."""
    dev = _device.require_cuda(device)
    if not blobs:
        raise ValueError("reload_blobs needs at least one page")
    buf, shapes, _, _, nbytes = _reload(blobs, dev, same_shape=True)
    shape, n = shapes[0], int(nbytes[0])
    span = (n + 255) // 256 * 256
    if span == n:
        kv = buf[:2 * n * len(blobs)].view(torch.bfloat16).reshape(len(blobs), 2, *shape)
        return kv[:, 0], kv[:, 1]
    rows = buf[:2 * span * len(blobs)].view(len(blobs), 2, span)[:, :, :n]
    kv = rows.contiguous().view(torch.bfloat16).reshape(len(blobs), 2, *shape)
    return kv[:, 0], kv[:, 1]
