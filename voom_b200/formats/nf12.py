"""BF16 NF12 exact sidecar: 12-bit block codec, GPU decode and the fused
decode + small-M linear (libvoom_b200, sm_100a).

Same format as vOOM's formats/bf16_nf12_sidecar.py: per 256-value block a
16-byte header, 384 bytes of 12-bit codes (bits 0-10 of the BF16 value, its
sign in bit 11) and 3-byte patches for values whose high exponent nibble is
not the tensor's modal one; a layer stream is every selected tensor's
headers (patch offsets rebased past the header and code streams), then the
codes, then the patches, wrapped in a one-tensor safetensors file.

Host side (numpy): `pack_tensor` (the reference's encoder, byte-identical
output) and `build_layer` (one layer stream and its manifest entry).  Device
side: `decode_layer` / `decode_names` (one launch per contiguous block span)
and `NF12Tensor.matmul`, which for <= 8 activation rows of an eligible
tensor never materialises the weights: `voom_nf12_linear` decodes and
accumulates in one pass over the stream.

Reference interface replaced: formats/bf16_nf12_sidecar.py:72-206,
318-420 (pack_tensor, layer build), runtime/bf16_nf12_sidecar.py:126-248
(decode_layer, decode_names), runtime/bf16_nf12_linear.py:19-244
(direct_linear_eligible, NF12Tensor).
"""

from __future__ import annotations

import ctypes
import json
import math
import struct
from pathlib import Path

import numpy as np
import torch

from .. import _device
from .._lib import VoomError, check, load

BLOCK_VALUES = 256
CODE_BYTES_PER_BLOCK = BLOCK_VALUES * 12 // 8
PATCH_BYTES = 3
BLOCK_HEADER_BYTES = 16
HEADER_DTYPE = np.dtype([("patch_offset", "<u4"), ("output", "<u4"), ("valid", "<u2"), ("count", "<u2"),
                         ("mode", "u1"), ("flags", "u1"), ("reserved", "<u2")])
assert HEADER_DTYPE.itemsize == BLOCK_HEADER_BYTES


class LinearTask(ctypes.Structure):
    """voom_nf12_linear_task: one projection of a batched fused linear."""
    _fields_ = [("d_x", ctypes.c_void_p), ("d_out", ctypes.c_void_p), ("K", ctypes.c_uint32),
                ("N", ctypes.c_uint32), ("first_block", ctypes.c_uint32), ("pad", ctypes.c_uint32)]


class NF12Error(ValueError):
    """Malformed NF12 stream (a header points outside the stream or output)."""


def _codes12(values: np.ndarray, blocks: int) -> np.ndarray:
    """12-bit codes, two per 3 bytes, little-endian (bf16_nf12_sidecar.py:72-94)."""
    v = np.zeros(blocks * BLOCK_VALUES, dtype=np.uint32)
    v[: values.size] = values
    code = (v & 0x07FF) | ((v >> 4) & 0x0800)
    word = code[0::2] | (code[1::2] << 12)  # 24 bits per pair
    out = np.empty((word.size, 3), dtype=np.uint8)
    out[:, 0] = word
    out[:, 1] = word >> 8
    out[:, 2] = word >> 16
    return out.reshape(-1)


def pack_tensor(raw: bytes, *, output_offset: int = 0, patch_base: int = 0) -> tuple[bytes, bytes, bytes, dict]:
    """(headers, codes, patches, report) of one BF16 tensor, or empty streams
    and selected=False when it would not shrink (bf16_nf12_sidecar.py:97-206)."""
    if len(raw) % 2:
        raise ValueError("BF16 tensor byte count must be even")
    values = np.frombuffer(raw, dtype="<u2")
    if not values.size:
        raise ValueError("cannot encode an empty BF16 tensor")
    nib = (values >> 11) & 0x0F
    mode = int(np.bincount(nib, minlength=16).argmax())
    exc = np.flatnonzero(nib != mode)
    blocks = math.ceil(values.size / BLOCK_VALUES)
    charged = blocks * (BLOCK_HEADER_BYTES + CODE_BYTES_PER_BLOCK) + PATCH_BYTES * int(exc.size)
    if charged >= len(raw):
        return b"", b"", b"", {"selected": False, "raw_bytes": len(raw), "encoded_bytes": len(raw), "ratio": 1.0,
                               "mode": mode, "exception_count": int(exc.size), "block_count": blocks}
    counts = np.bincount(exc // BLOCK_VALUES, minlength=blocks).astype(np.uint64)
    starts = int(patch_base) + np.concatenate([np.zeros(1, np.uint64), np.cumsum(counts)[:-1]]) * PATCH_BYTES
    outs = int(output_offset) + np.arange(blocks, dtype=np.uint64) * BLOCK_VALUES
    if starts.max(initial=0) > 0xFFFFFFFF or outs.max(initial=0) > 0xFFFFFFFF:
        raise OverflowError("NF12 layer offsets exceed uint32 format")
    hdr = np.zeros(blocks, dtype=HEADER_DTYPE)
    hdr["patch_offset"] = starts
    hdr["output"] = outs
    hdr["valid"] = BLOCK_VALUES
    if values.size % BLOCK_VALUES:
        hdr["valid"][-1] = values.size % BLOCK_VALUES
    hdr["count"] = counts
    hdr["mode"] = mode
    pat = np.empty((exc.size, PATCH_BYTES), dtype=np.uint8)
    if exc.size:
        exact = values[exc]
        pat[:, 0] = exc % BLOCK_VALUES
        pat[:, 1] = exact & 0xFF
        pat[:, 2] = exact >> 8
    return hdr.tobytes(), _codes12(values, blocks).tobytes(), pat.tobytes(), {
        "selected": True, "raw_bytes": len(raw), "encoded_bytes": charged, "ratio": len(raw) / charged,
        "mode": mode, "exception_count": int(exc.size), "block_count": blocks, "value_count": int(values.size)}


def build_layer(tensors: list[tuple[str, np.ndarray, tuple]]) -> tuple[bytes, dict]:
    """One layer stream + manifest entry from (name, BF16 bits, shape) in the
    given order; tensors that would not shrink are left out, as the
    reference's builder does (bf16_nf12_sidecar.py:318-420)."""
    heads, codes, pats, specs = [], [], [], []
    n_out = n_blocks = n_patch = 0
    raw_total = sel_raw = 0
    for name, bits, shape in tensors:
        raw = np.ascontiguousarray(bits, dtype="<u2").tobytes()
        raw_total += len(raw)
        h, c, p, rep = pack_tensor(raw, output_offset=n_out, patch_base=n_patch)
        if not rep["selected"]:
            continue
        heads.append(np.frombuffer(h, dtype=HEADER_DTYPE).copy())
        codes.append(c)
        pats.append(p)
        specs.append({"physical_name": name, "name": name.removeprefix("language_model."),
                      "shape": [int(s) for s in shape], "output_offset": n_out, "value_count": rep["value_count"],
                      "block_start": n_blocks, "block_count": rep["block_count"], "raw_bytes": rep["raw_bytes"],
                      "encoded_bytes": rep["encoded_bytes"], "ratio": rep["ratio"], "mode": rep["mode"],
                      "exception_count": rep["exception_count"]})
        n_out += rep["value_count"]
        n_blocks += rep["block_count"]
        n_patch += len(p)
        sel_raw += len(raw)
    if not specs:
        raise ValueError("no BF16 tensor shrank")
    hdr = np.concatenate(heads)
    code_bytes = b"".join(codes)
    hdr["patch_offset"] += hdr.nbytes + len(code_bytes)
    payload = hdr.tobytes() + code_bytes + b"".join(pats)
    entry = {"file_bytes": len(payload), "block_values": BLOCK_VALUES, "block_header_bytes": BLOCK_HEADER_BYTES,
             "code_bytes_per_block": CODE_BYTES_PER_BLOCK, "patch_bytes": PATCH_BYTES, "block_count": n_blocks,
             "header_bytes": hdr.nbytes, "code_bytes": len(code_bytes), "patch_stream_bytes": n_patch,
             "output_value_count": n_out, "selected_raw_bytes": sel_raw, "all_bf16_raw_bytes": raw_total,
             "encoded_bytes": len(payload), "ratio_selected_raw_over_encoded": sel_raw / len(payload),
             "saved_bytes": sel_raw - len(payload), "tensors": specs}
    return payload, entry


def safetensors_file(payload: bytes) -> bytes:
    """The layer file: a safetensors header holding one U8 tensor "encoded"."""
    header = json.dumps({"encoded": {"dtype": "U8", "shape": [len(payload)], "data_offsets": [0, len(payload)]}},
                        separators=(",", ":"), sort_keys=True).encode()
    header += b" " * ((-len(header)) % 8)
    return struct.pack("<Q", len(header)) + header + payload


def read_layer_file(path: str | Path) -> bytes:
    """Payload of a layer file (the "encoded" tensor of its safetensors)."""
    data = Path(path).read_bytes()
    n = struct.unpack_from("<Q", data)[0]
    meta = json.loads(data[8:8 + n])["encoded"]
    a, b = meta["data_offsets"]
    return data[8 + n + a:8 + n + b]


def _device_stream(encoded, entry: dict, device) -> torch.Tensor:
    """The layer stream as a 16-byte aligned CUDA uint8 tensor."""
    expected = int(entry["file_bytes"])
    if isinstance(encoded, torch.Tensor) and encoded.is_cuda:
        if encoded.dtype != torch.uint8:
            raise ValueError("BF16 NF12 encoded tensor must be uint8")
        if encoded.numel() < expected:
            raise ValueError(f"BF16 NF12 encoded bytes {encoded.numel()} != {expected}")
        if encoded.data_ptr() % 16:
            encoded = encoded.clone()
        return encoded
    host = _device.as_u8(encoded)
    if host.size != expected:
        raise ValueError(f"BF16 NF12 encoded bytes {host.size} != {expected}")
    return _device.upload(host, _device.require_cuda(device))


def _decode_span(enc: torch.Tensor, entry: dict, first_block: int, block_count: int, output_base: int,
                 output_value_count: int) -> torch.Tensor:
    if block_count <= 0 or output_value_count <= 0:
        raise ValueError("BF16 NF12 decode span must be non-empty")
    total = int(entry["block_count"])
    hb = int(entry["header_bytes"])
    if hb != total * BLOCK_HEADER_BYTES:
        raise ValueError("BF16 NF12 header/block count mismatch")
    if first_block < 0 or first_block + block_count > total:
        raise ValueError("BF16 NF12 decode span exceeds layer blocks")
    dev = enc.device
    out = torch.empty(output_value_count, dtype=torch.int16, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    check(load().voom_nf12_decode(enc.data_ptr(), int(entry["file_bytes"]), hb, first_block, block_count,
                                  output_base, out.data_ptr(), output_value_count, status.data_ptr(),
                                  _device.stream_ptr(dev)), "voom_nf12_decode")
    if int(status.item()):
        raise NF12Error("BF16 NF12 block header points outside the stream or output")
    return out.view(torch.bfloat16)


def decode_layer(encoded, entry: dict, *, device=None) -> dict[str, torch.Tensor]:
    """Every tensor of a layer in one launch (runtime/bf16_nf12_sidecar.py:126-149)."""
    enc = _device_stream(encoded, entry, device)
    dec = _decode_span(enc, entry, 0, int(entry["block_count"]), 0, int(entry["output_value_count"]))
    return {t["name"]: dec[int(t["output_offset"]):int(t["output_offset"]) + int(t["value_count"])]
            .reshape(tuple(int(v) for v in t["shape"])) for t in entry["tensors"]}


def decode_names(encoded, entry: dict, requested_names, *, device=None) -> dict[str, torch.Tensor]:
    """Only the requested tensors, one launch per physically contiguous run
    (runtime/bf16_nf12_sidecar.py:152-248)."""
    enc = _device_stream(encoded, entry, device)
    specs = {t["name"]: t for t in entry["tensors"]}
    names = list(dict.fromkeys(requested_names))
    tensors = []
    for name in names:
        if name not in specs:
            raise KeyError(f"{name}: tensor is not encoded in NF12 layer")
        tensors.append(specs[name])
    runs: list[list[dict]] = []
    for t in sorted(tensors, key=lambda t: int(t["block_start"])):
        if runs:
            prev = runs[-1][-1]
            if (int(t["block_start"]) == int(prev["block_start"]) + int(prev["block_count"])
                    and int(t["output_offset"]) == int(prev["output_offset"]) + int(prev["value_count"])):
                runs[-1].append(t)
                continue
        runs.append([t])
    got = {}
    for run in runs:
        base = int(run[0]["output_offset"])
        dec = _decode_span(enc, entry, int(run[0]["block_start"]), sum(int(t["block_count"]) for t in run), base,
                           sum(int(t["value_count"]) for t in run))
        for t in run:
            o = int(t["output_offset"]) - base
            got[t["name"]] = dec[o:o + int(t["value_count"])].reshape(tuple(int(v) for v in t["shape"]))
    return {n: got[n] for n in names}


def direct_linear_eligible(spec: dict) -> bool:
    """Shapes the fused small-M kernel takes (runtime/bf16_nf12_linear.py:19-27)."""
    shape = tuple(int(v) for v in spec["shape"])
    return len(shape) == 2 and shape[0] % 8 == 0 and shape[1] % 512 == 0 and int(spec["raw_bytes"]) >= 1_000_000


def linear(x: torch.Tensor, enc: torch.Tensor, entry: dict, spec: dict, *,
           status: torch.Tensor | None = None) -> torch.Tensor:
    """x (M <= 8 rows of K, BF16, CUDA) @ W.T with W decoded on the fly:
    (M, N) BF16, fp32 accumulation.  Without `status` the call reads its own
    status back (one synchronisation) and raises on a damaged operand; with
    it, failures accumulate into that int32 device flag for the caller to
    check later (the kernel never reads outside the stream either way)."""
    n_size, k_size = (int(v) for v in spec["shape"])
    m = x.shape[0]
    if x.dtype != torch.bfloat16 or x.shape[1] != k_size or not 1 <= m <= 8:
        raise ValueError("nf12 linear takes 1..8 BF16 rows of K")
    x = x.contiguous()
    if x.data_ptr() % 16:
        x = x.clone()
    lib = load()
    dev = enc.device
    need = int(lib.voom_nf12_linear_scratch_bytes(m, k_size, n_size))
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    out = torch.empty((m, n_size), dtype=torch.bfloat16, device=dev)
    own = status is None
    if own:
        status = torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib.voom_nf12_linear(x.data_ptr(), m, k_size, n_size, enc.data_ptr(), int(entry["file_bytes"]),
                               int(entry["header_bytes"]), int(spec["block_start"]), scratch.data_ptr(), need,
                               out.data_ptr(), status.data_ptr(), _device.stream_ptr(dev)), "voom_nf12_linear")
    if own and int(status.item()):
        raise NF12Error("BF16 NF12 linear operand has a partial block or patches outside the stream")
    return out


def linear_batch(items: list[tuple[torch.Tensor, dict]], enc: torch.Tensor, entry: dict, *,
                 status: torch.Tensor | None = None) -> list[torch.Tensor]:
    """Several fused linears of one layer stream in one launch: items are
    (x, spec) with the same number of rows M <= 8 (up to 16 items); returns
    each x @ W.T as voom_nf12_linear would."""
    if not items or len(items) > 16:
        raise ValueError("nf12 linear_batch takes 1..16 projections")
    m = items[0][0].shape[0]
    dev = enc.device
    keep, outs = [], []
    arr = (LinearTask * len(items))()
    for i, (x, spec) in enumerate(items):
        n_size, k_size = (int(v) for v in spec["shape"])
        if x.dtype != torch.bfloat16 or x.shape != (m, k_size) or not 1 <= m <= 8:
            raise ValueError("nf12 linear_batch takes M x K BF16 rows, the same M for every item")
        x = x.contiguous()
        if x.data_ptr() % 16:
            x = x.clone()
        out = torch.empty((m, n_size), dtype=torch.bfloat16, device=dev)
        keep.append(x)
        outs.append(out)
        arr[i] = LinearTask(x.data_ptr(), out.data_ptr(), k_size, n_size, int(spec["block_start"]), 0)
    lib = load()
    need = int(lib.voom_nf12_linear_batch_scratch_bytes(ctypes.byref(arr), len(items), m))
    scratch = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    own = status is None
    if own:
        status = torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib.voom_nf12_linear_batch(ctypes.byref(arr), len(items), m, enc.data_ptr(), int(entry["file_bytes"]),
                                     int(entry["header_bytes"]), scratch.data_ptr(), need, status.data_ptr(),
                                     _device.stream_ptr(dev)), "voom_nf12_linear_batch")
    if own and int(status.item()):
        raise NF12Error("BF16 NF12 linear operand has a partial block or patches outside the stream")
    return outs


def check_headers(encoded_host: np.ndarray, entry: dict, spec: dict) -> None:
    """Host check of one tensor's block headers: every block full (a linear
    operand), output offsets in order, patches inside the stream."""
    hb = int(entry["header_bytes"])
    hdr = np.frombuffer(encoded_host[:hb], dtype=HEADER_DTYPE)
    b0, nb = int(spec["block_start"]), int(spec["block_count"])
    h = hdr[b0:b0 + nb]
    if h.size != nb:
        raise NF12Error("BF16 NF12 tensor blocks exceed the layer headers")
    end = h["patch_offset"].astype(np.uint64) + h["count"].astype(np.uint64) * PATCH_BYTES
    want_out = int(spec["output_offset"]) + np.arange(nb, dtype=np.uint64) * BLOCK_VALUES
    if (h["valid"] > BLOCK_VALUES).any() or (end > int(entry["file_bytes"])).any() \
            or not np.array_equal(h["output"].astype(np.uint64), want_out):
        raise NF12Error("BF16 NF12 block header points outside the stream or output")


class NF12Tensor:
    """A BF16 weight kept as its NF12 blocks in device memory
    (runtime/bf16_nf12_linear.py:163-244)."""

    def __init__(self, encoded, entry: dict, spec: dict, *, device=None):
        self.entry = entry
        self.spec = spec
        self.encoded = _device_stream(encoded, entry, device)
        hb = int(entry["header_bytes"])
        host = (encoded[:hb].cpu().numpy() if isinstance(encoded, torch.Tensor) else _device.as_u8(encoded)[:hb])
        check_headers(np.concatenate([host, np.zeros(0, np.uint8)]), entry, spec)
        # damaged blocks found by the fused kernel accumulate here (see check())
        self.status = torch.zeros(1, dtype=torch.int32, device=self.encoded.device)

    def check(self) -> None:
        """Raise if any fused product so far met a damaged block."""
        if int(self.status.item()):
            raise NF12Error("BF16 NF12 linear operand has a partial block or patches outside the stream")

    @property
    def nbytes(self) -> int:
        return int(self.spec["encoded_bytes"])

    @property
    def shape(self) -> tuple[int, ...]:
        return tuple(int(v) for v in self.spec["shape"])

    @property
    def dtype(self):
        return torch.bfloat16

    def materialize(self) -> torch.Tensor:
        return decode_names(self.encoded, self.entry, [self.spec["name"]])[self.spec["name"]]

    def reshape(self, *shape) -> torch.Tensor:
        return self.materialize().reshape(*shape)

    def matmul(self, x: torch.Tensor) -> torch.Tensor:
        lead = tuple(int(v) for v in x.shape[:-1])
        positions = int(np.prod(lead, dtype=np.int64)) if lead else 1
        n_size, k_size = self.shape
        if positions <= 8 and x.shape[-1] == k_size and direct_linear_eligible(self.spec) \
                and x.dtype == torch.bfloat16:
            return linear(x.reshape(positions, k_size), self.encoded, self.entry, self.spec,
                          status=self.status).reshape(*lead, n_size)
        dense = decode_layer(self.encoded, self.entry)[self.spec["name"]]
        return x @ dense.T


__all__ = ["BLOCK_VALUES", "CODE_BYTES_PER_BLOCK", "PATCH_BYTES", "BLOCK_HEADER_BYTES", "NF12Error", "NF12Tensor",
           "pack_tensor", "build_layer", "safetensors_file", "read_layer_file", "decode_layer", "decode_names",
           "direct_linear_eligible", "linear", "linear_batch", "check_headers", "LinearTask", "VoomError"]
