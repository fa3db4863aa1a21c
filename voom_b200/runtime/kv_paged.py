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

import json
import pickle
import struct
import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from .. import _device
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
    blobs, jobs, shapes = [], [], []
    src = dst = 0
    for _, p in comp:
        with open(p.path, "rb") as f:
            d = pickle.load(f)
        shape = tuple(d["shape"])
        n = int(np.prod(shape)) * 2
        for key in ("k", "v"):
            b = d[key]
            blobs.append(b)
            jobs.append((src, len(b), dst, n, 0, 0, 0))
            src += len(b)
            dst += (n + 255) // 256 * 256
        shapes.append((shape, n))
    host = np.frombuffer(b"".join(blobs), np.uint8)
    jarr = np.array(jobs, dtype=JOB_DTYPE)
    plan = ZstdPlan(host, jarr)
    with torch.cuda.device(dev):
        d_src = _device.upload(host, dev)
        buf = torch.empty(max(dst, 1), dtype=torch.uint8, device=dev)
        batch = ZstdBatch(plan, dev)
        batch.run(d_src, buf)
        st = batch.job_status()
    if st.any():
        raise ZstdError(describe(int(st[np.nonzero(st)[0][0]])))
    for q, (i, _p) in enumerate(comp):
        shape, n = shapes[q]
        kd, vd = int(jarr[2 * q]["dst"]), int(jarr[2 * q + 1]["dst"])
        k = buf[kd:kd + n].view(torch.bfloat16).reshape(shape)
        v = buf[vd:vd + n].view(torch.bfloat16).reshape(shape)
        out[i] = (k, v)
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
    """Decode many .kvz pages in one batched GPU decode -> (K, V) stacked on
    a leading page axis."""
    dev = _device.require_cuda(device)
    frames, jobs, shape = [], [], None
    src = dst = 0
    for blob in blobs:
        d = pickle.loads(blob)
        shape = tuple(d["shape"])
        n = int(np.prod(shape)) * 2
        for key in ("k", "v"):
            frames.append(d[key])
            jobs.append((src, len(d[key]), dst, n, 0, 0, 0))
            src += len(d[key])
            dst += n
    host = np.frombuffer(b"".join(frames), np.uint8)
    plan = ZstdPlan(host, np.array(jobs, dtype=JOB_DTYPE))
    with torch.cuda.device(dev):
        d_src = _device.upload(host, dev)
        buf = torch.empty(max(dst, 1), dtype=torch.uint8, device=dev)
        batch = ZstdBatch(plan, dev)
        batch.run(d_src, buf)
        st = batch.job_status()
    if st.any():
        raise ZstdError(describe(int(st[np.nonzero(st)[0][0]])))
    kv = buf.view(torch.bfloat16).reshape(len(blobs), 2, *shape)
    return kv[:, 0], kv[:, 1]
