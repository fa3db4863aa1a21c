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

import ctypes
import json
import pickle
import platform
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


def _write_safetensors(path: Path, tensors: dict[str, torch.Tensor]) -> None:
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        raw = _bf16_to_raw(t)
        header[name] = {"dtype": "BF16", "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hj = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)) + hj)
        for b in blobs:
            f.write(b)


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
        """Returns the compressed byte count if compress=True, else None."""
        if compress:
            k_c = zstd_host.compress(_bf16_to_raw(self.k), 1)
            v_c = zstd_host.compress(_bf16_to_raw(self.v), 1)
            path = path.with_suffix(".kvz")
            with open(path, "wb") as f:
                pickle.dump({"shape": self.shape, "k": k_c, "v": v_c}, f)
            self._compressed = True
            self.path = path
            self.k = self.v = None
            return len(k_c) + len(v_c)
        _write_safetensors(path, {"k": self.k, "v": self.v})
        self._compressed = False
        self.path = path
        self.k = self.v = None
        return None

    def load(self) -> tuple[torch.Tensor, torch.Tensor]:
        if self.resident:
            return self.k, self.v
        return load_pages([self])[0]


KVZ_PAGE_DTYPE = np.dtype([("k_off", "<u8"), ("k_len", "<u8"), ("v_off", "<u8"), ("v_len", "<u8"),
                           ("shape", "<i8", (8,)), ("ndim", "<u4"), ("status", "<u4")])
assert KVZ_PAGE_DTYPE.itemsize == 104

# CPython keeps a bytes object's data inline after a fixed header; the data
# address is id(obj) + this offset (checked once against ctypes below).
_BYTES_DATA = bytes.__basicsize__ - 1
_arenas: dict = {}
_arenas_lock = threading.Lock()


def _inline_bytes_ok() -> bool:
    if platform.python_implementation() != "CPython":
        return False
    probe = bytes(range(97, 123)) * 3
    return ctypes.string_at(id(probe) + _BYTES_DATA, len(probe)) == probe


_INLINE_BYTES = _inline_bytes_ok()


def _addresses(blobs: list) -> np.ndarray:
    """Host addresses of the blobs' bytes (the objects stay alive in `blobs`)."""
    if _INLINE_BYTES and all(type(b) is bytes for b in blobs):
        return np.fromiter(map(id, blobs), np.uint64, len(blobs)) + np.uint64(_BYTES_DATA)
    keep = [b if type(b) is bytes else bytes(b) for b in blobs]
    blobs[:] = keep
    return np.array([ctypes.cast(ctypes.c_char_p(b), ctypes.c_void_p).value for b in keep], np.uint64)


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
    output buffer, each page's (shape, K offset, V offset, bytes)."""
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
    return out, [(shapes[i], int(dst[i]), int(dst[i] + span[i]), int(nbytes[i])) for i in range(n)]


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
    buf, spans = _reload(blobs, dev, same_shape=False)
    for (i, _p), (shape, kd, vd, n) in zip(comp, spans):
        out[i] = (buf[kd:kd + n].view(torch.bfloat16).reshape(shape),
                  buf[vd:vd + n].view(torch.bfloat16).reshape(shape))
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
        self._pages: list[list[_Page]] = [[] for _ in range(num_layers)]
        self._tail_k: list[torch.Tensor | None] = [None] * num_layers
        self._tail_v: list[torch.Tensor | None] = [None] * num_layers
        self._offset = 0
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
        paths = {page.path for pages in self._pages for page in pages if page.path is not None}
        self._pages = [[] for _ in range(self.num_layers)]
        self._tail_k = [None] * self.num_layers
        self._tail_v = [None] * self.num_layers
        self._offset = 0
        for path in paths:
            try:
                path.unlink()
            except FileNotFoundError:
                pass

    def _enforce_budget(self):
        if self.nbytes() <= self.max_bytes:
            return
        for page_idx in range(max(len(p) for p in self._pages)):
            for layer in range(self.num_layers):
                pages = self._pages[layer]
                if page_idx >= len(pages) - self.resident_pages:
                    continue
                page = pages[page_idx]
                if not page.resident:
                    continue
                raw_bytes = page.nbytes
                t0 = time.perf_counter()
                comp = page.spill(self.spill_dir / f"kv_l{layer}_p{page_idx}.safetensors",
                                  compress=self.compress_spill)
                self.stats.spills += 1
                self.stats.spill_s += time.perf_counter() - t0
                if comp is not None:
                    self.stats.spill_bytes_raw += raw_bytes
                    self.stats.spill_bytes_compressed += comp
                if self.nbytes() <= self.max_bytes:
                    return


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
    buf, spans = _reload(blobs, dev, same_shape=True)
    shape, _, _, n = spans[0]
    span = (n + 255) // 256 * 256
    if span == n:
        kv = buf[:2 * n * len(blobs)].view(torch.bfloat16).reshape(len(blobs), 2, *shape)
        return kv[:, 0], kv[:, 1]
    rows = buf[:2 * span * len(blobs)].view(len(blobs), 2, span)[:, :, :n]
    kv = rows.contiguous().view(torch.bfloat16).reshape(len(blobs), 2, *shape)
    return kv[:, 0], kv[:, 1]
