"""Oracle for the BF16 NF12 exact sidecar -- TEST INFRASTRUCTURE ONLY.

Restates, with numpy:
  * the block codec (formats/bf16_nf12_sidecar.py:72-94 `_pack_codes12`,
    :97-206 `pack_tensor`, :209-244 `unpack_tensor`): per 256-value block a
    16-byte header (patch offset u32, output offset u32, valid u16, exception
    count u16, modal high exponent nibble u8, flags u8, reserved u16), 384
    bytes of 12-bit codes (bits 0-10 of the BF16 value, bit 11 = its sign),
    and 3-byte patches (local index u8, exact bits u16) for values whose high
    exponent nibble is not the tensor's modal one;
  * the layer stream the sidecar builder writes (:318-420): headers of every
    selected tensor with patch offsets rebased past the header and code
    streams, then all codes, then all patches;
  * the runtime decode of a block span (runtime/bf16_nf12_sidecar.py:21-98):
    a value whose local index has several patches takes the first;
  * the fused small-M linear (runtime/bf16_nf12_linear.py:19-27 eligibility,
    :30-120 kernel): out[p, n] = sum_k x[p, k] * w[n, k] in fp32, cast to the
    activation dtype.
"""

from __future__ import annotations

import math
import struct

import numpy as np

BLOCK_VALUES = 256
CODE_BYTES_PER_BLOCK = BLOCK_VALUES * 12 // 8
PATCH_BYTES = 3
BLOCK_HEADER = struct.Struct("<IIHHBBH")
BLOCK_HEADER_BYTES = BLOCK_HEADER.size


def pack_codes12(values: np.ndarray, blocks: int) -> bytes:
    padded = np.zeros(blocks * BLOCK_VALUES, dtype=np.uint16)
    padded[: values.size] = values
    codes = (padded & 0x07FF) | ((padded >> 4) & 0x0800)
    pairs = codes.reshape(-1, 2).astype(np.uint32)
    packed = np.empty((pairs.shape[0], 3), dtype=np.uint8)
    packed[:, 0] = pairs[:, 0] & 0xFF
    packed[:, 1] = ((pairs[:, 0] >> 8) & 0x0F) | ((pairs[:, 1] & 0x0F) << 4)
    packed[:, 2] = pairs[:, 1] >> 4
    return packed.tobytes()


def pack_tensor(raw: bytes, *, output_offset: int = 0, patch_base: int = 0):
    """(headers, codes, patches, report) as formats/bf16_nf12_sidecar.py:97-206."""
    if len(raw) % 2:
        raise ValueError("BF16 tensor byte count must be even")
    values = np.frombuffer(raw, dtype="<u2")
    if not values.size:
        raise ValueError("cannot encode an empty BF16 tensor")
    high = ((values >> 11) & 0x0F).astype(np.uint8)
    mode = int(np.bincount(high, minlength=16).argmax())
    exc = np.flatnonzero(high != mode)
    blocks = math.ceil(values.size / BLOCK_VALUES)
    charged = blocks * (BLOCK_HEADER_BYTES + CODE_BYTES_PER_BLOCK) + PATCH_BYTES * exc.size
    if charged >= len(raw):
        return b"", b"", b"", {"selected": False, "raw_bytes": len(raw), "encoded_bytes": len(raw), "ratio": 1.0,
                               "mode": mode, "exception_count": int(exc.size), "block_count": blocks}
    counts = np.bincount(exc // BLOCK_VALUES, minlength=blocks)
    starts = patch_base + np.concatenate([[0], np.cumsum(counts[:-1]) * PATCH_BYTES]).astype(np.int64)
    headers = bytearray(blocks * BLOCK_HEADER_BYTES)
    for b in range(blocks):
        valid = min(BLOCK_VALUES, values.size - b * BLOCK_VALUES)
        BLOCK_HEADER.pack_into(headers, b * BLOCK_HEADER_BYTES, int(starts[b]),
                               int(output_offset + b * BLOCK_VALUES), valid, int(counts[b]), mode, 0, 0)
    patches = np.empty((exc.size, PATCH_BYTES), dtype=np.uint8)
    if exc.size:
        exact = values[exc]
        patches[:, 0] = exc % BLOCK_VALUES
        patches[:, 1] = exact & 0xFF
        patches[:, 2] = exact >> 8
    return bytes(headers), pack_codes12(values, blocks), patches.tobytes(), {
        "selected": True, "raw_bytes": len(raw), "encoded_bytes": charged, "ratio": len(raw) / charged,
        "mode": mode, "exception_count": int(exc.size), "block_count": blocks, "value_count": int(values.size)}


def unpack_codes12(codes: bytes) -> np.ndarray:
    p = np.frombuffer(codes, dtype=np.uint8).reshape(-1, 3).astype(np.uint16)
    out = np.empty(p.shape[0] * 2, dtype=np.uint16)
    out[0::2] = p[:, 0] | ((p[:, 1] & 0x0F) << 8)
    out[1::2] = (p[:, 1] >> 4) | (p[:, 2] << 4)
    return out


def decode_span(encoded: bytes, header_bytes: int, first_block: int, block_count: int, output_base: int,
                output_value_count: int) -> np.ndarray:
    """Values of blocks [first_block, first_block + block_count) of a layer
    stream, placed at header output offset - output_base (uint16 bits)."""
    enc = memoryview(encoded)
    out = np.zeros(output_value_count, dtype=np.uint16)
    for blk in range(first_block, first_block + block_count):
        poff, outoff, valid, count, mode, _flags, _res = BLOCK_HEADER.unpack_from(enc, blk * BLOCK_HEADER_BYTES)
        mode &= 15
        c0 = header_bytes + blk * CODE_BYTES_PER_BLOCK
        codes = unpack_codes12(bytes(enc[c0:c0 + CODE_BYTES_PER_BLOCK]))[:valid]
        vals = (codes & 0x07FF) | ((codes & 0x0800) << 4) | np.uint16(mode << 11)
        done = set()
        for p in range(count):
            at = poff + p * PATCH_BYTES
            local = enc[at]
            if local < valid and local not in done:
                done.add(local)
                vals[local] = enc[at + 1] | (enc[at + 2] << 8)
        o = outoff - output_base
        out[o:o + valid] = vals
    return out


def build_layer(tensors: list[tuple[str, np.ndarray, tuple]]) -> tuple[bytes, dict]:
    """Layer stream + manifest entry for (name, uint16 bits, shape) tensors in
    the given order (formats/bf16_nf12_sidecar.py:318-420, without files)."""
    headers, codes, patches, specs = [], [], [], []
    out_count = block_count = patch_bytes = 0
    for name, bits, shape in tensors:
        raw = np.ascontiguousarray(bits, dtype="<u2").tobytes()
        h, c, p, rep = pack_tensor(raw, output_offset=out_count, patch_base=patch_bytes)
        if not rep["selected"]:
            continue
        headers.append(h)
        codes.append(c)
        patches.append(p)
        specs.append({"name": name, "shape": [int(s) for s in shape], "output_offset": out_count,
                      "value_count": rep["value_count"], "block_start": block_count,
                      "block_count": rep["block_count"], "raw_bytes": rep["raw_bytes"],
                      "encoded_bytes": rep["encoded_bytes"], "mode": rep["mode"],
                      "exception_count": rep["exception_count"]})
        out_count += rep["value_count"]
        block_count += rep["block_count"]
        patch_bytes += len(p)
    hb = b"".join(headers)
    cb = b"".join(codes)
    base = len(hb) + len(cb)
    adj = bytearray(hb)
    for off in range(0, len(adj), BLOCK_HEADER_BYTES):
        f = list(BLOCK_HEADER.unpack_from(adj, off))
        f[0] += base
        BLOCK_HEADER.pack_into(adj, off, *f)
    payload = bytes(adj) + cb + b"".join(patches)
    entry = {"file_bytes": len(payload), "block_count": block_count, "header_bytes": len(hb),
             "code_bytes": len(cb), "patch_stream_bytes": patch_bytes, "output_value_count": out_count,
             "tensors": specs}
    return payload, entry


def direct_linear_eligible(spec: dict) -> bool:
    shape = tuple(int(v) for v in spec["shape"])
    return len(shape) == 2 and shape[0] % 8 == 0 and shape[1] % 512 == 0 and int(spec["raw_bytes"]) >= 1_000_000


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)
