"""vpack: lossless byte-plane compressed weight store (GPU decode).

Same on-disk layout as vOOM's formats/packed.py: one `.vt` file per tensor,
an 8-byte little-endian header length, a JSON head, then the body.  For
BF16/F16 the body is `hi_z` (zstd of the odd bytes) followed by `lo` (the even
bytes, raw); tensors above STREAM_THRESHOLD use the streamed variant (lo raw
first, then one zstd stream of the hi plane to EOF); other dtypes are stored
raw.  `pack_model` writes that layout (host zstd, or the GPU encoder for a
fast repack: `bodies_gpu`);
`read_tensor_bytes` and `to_torch` decode on the GPU.

Reference interface replaced: formats/packed.py:63-81 (streamed pack),
:125-358 (pack_model), :361-379 (read_tensor_bytes), :385-397 (to_mx).
"""

from __future__ import annotations

import json
import re
import struct
import time
from pathlib import Path

import numpy as np
import torch

from . import zstd_host
from .zstd_gpu import INTERLEAVE, JOB_DTYPE, ZstdBatch, ZstdError, ZstdPlan, describe

PLANE_DTYPES = {"BF16", "F16"}
STREAM_THRESHOLD = 256 * 1024 * 1024
CHUNK = 64 * 1024 * 1024

_FUSED_BF16_EXPERT_RE = re.compile(r"^(.*\.mlp\.experts)\.(gate_up_proj|down_proj)$")

TORCH_DTYPES = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32, "I64": torch.int64,
                "U8": torch.uint8, "I32": torch.int32, "I8": torch.int8, "U32": torch.uint32}


def body_for(dtype: str, raw, level: int = 1) -> tuple[dict, bytes]:
    """(head, body) of one tensor in ordinary vpack form."""
    a = np.frombuffer(raw, np.uint8) if not isinstance(raw, np.ndarray) else raw.reshape(-1).view(np.uint8)
    if dtype in PLANE_DTYPES:
        hi_z = zstd_host.compress(a[1::2], level)
        lo = a[0::2].tobytes()
        return {"hi_z": len(hi_z), "lo": len(lo)}, hi_z + lo
    return {"raw": a.size}, a.tobytes()


def bodies_gpu(items, device=None) -> list[tuple[dict, bytes]]:
    """(head, body) of many tensors in ordinary vpack form, with every hi plane
    compressed on the GPU: a fast repack path (the reference packs with host
    zstd level 1, formats/packed.py:125-358).  The frames come from
    voom_zstd_encode (Huffman-literal blocks, Raw or RLE where smaller): valid
    zstd frames that the reference's decode_body reads back exactly, not
    libzstd's bytes.  `items`: (dtype, data) pairs, data a CUDA tensor or host
    bytes / uint8 array; plane dtypes are split into byte planes on the device
    (hi = odd bytes, lo = even bytes), other dtypes are stored raw.  All hi
    planes are encoded in one batch and every host transfer is one copy."""
    from .. import _device
    from . import zstd_gpu

    dev = _device.require_cuda(device)
    flat, host_idx = [], []
    for i, (_, data) in enumerate(items):
        if isinstance(data, torch.Tensor):
            flat.append(data.reshape(-1).view(torch.uint8).to(dev))
        else:
            flat.append(None)
            host_idx.append(i)
    if host_idx:  # host data: one pinned staging buffer, one upload
        arrs = [np.frombuffer(items[i][1], np.uint8) if not isinstance(items[i][1], np.ndarray)
                else items[i][1].reshape(-1).view(np.uint8) for i in host_idx]
        pinned = _device.pinned_empty(max(1, sum(a.size for a in arrs)))
        pn = pinned.numpy()
        pos, spans = 0, []
        for a in arrs:
            pn[pos:pos + a.size] = a
            spans.append((pos, a.size))
            pos += a.size
        up = pinned[:pos].to(dev, non_blocking=True) if pos else torch.empty(0, dtype=torch.uint8, device=dev)
        for i, (o, n) in zip(host_idx, spans):
            flat[i] = up[o:o + n]
    plane = [items[i][0] in PLANE_DTYPES for i in range(len(items))]
    # the encoder's source: hi planes at 16-byte aligned offsets
    hi_offs, hi_lens, hpos = [], [], 0
    for i, u8 in enumerate(flat):
        if plane[i]:
            hi_offs.append(hpos)
            hi_lens.append(int(u8.numel()) // 2)
            hpos += (hi_lens[-1] + 15) // 16 * 16
    hi_buf = torch.empty(max(hpos, 16), dtype=torch.uint8, device=dev)
    k = 0
    for i, u8 in enumerate(flat):
        if plane[i]:
            hi_buf[hi_offs[k]:hi_offs[k] + hi_lens[k]].copy_(u8[1::2])
            k += 1
    plan = zstd_gpu.EncodePlan(hi_offs, hi_lens, dev)
    plan.run(hi_buf)
    sz = plan.block_sizes()  # waits for the encode
    flen = [int(v) for v in np.add.reduceat(sz[:, 1], plan.first)] if plan.n_blocks else []
    # the bodies assembled on the device (frame, then lo plane; or raw bytes), one copy to the host
    sizes, k = [], 0
    for i, u8 in enumerate(flat):
        n = int(u8.numel())
        sizes.append(flen[k] + n - n // 2 if plane[i] else n)
        k += plane[i]
    starts = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    total = int(starts[-1])
    bodies = torch.empty(max(total, 1), dtype=torch.uint8, device=dev)
    frame_dst = [int(starts[i]) for i in range(len(items)) if plane[i]]
    if plan.n_blocks:
        zstd_gpu.pack_blocks(plan, sz, frame_dst, bodies)
    k = 0
    for i, u8 in enumerate(flat):
        n, o = int(u8.numel()), int(starts[i])
        if plane[i]:
            bodies[o + flen[k]:o + flen[k] + n - n // 2].copy_(u8[0::2])
            k += 1
        else:
            bodies[o:o + n].copy_(u8)
    arena = _bodies_arena(dev)
    with arena.lock:  # one reused pinned buffer: pinning ~180 MB per call cost more than the copy
        host = arena.get(max(total, 1))[:max(total, 1)]
        host.copy_(bodies)
        mv = memoryview(host.numpy())
        out, k = [], 0
        for i, u8 in enumerate(flat):
            n, o = int(u8.numel()), int(starts[i])
            if plane[i]:
                out.append(({"hi_z": flen[k], "lo": n - n // 2}, bytes(mv[o:o + sizes[i]])))
                k += 1
            else:
                out.append(({"raw": n}, bytes(mv[o:o + n])))
    return out


_arenas: dict = {}


def _bodies_arena(dev: torch.device):
    """The device's pinned buffer for bodies coming back to the host."""
    from .. import _device

    a = _arenas.get(dev.index)
    if a is None:
        a = _arenas.setdefault(dev.index, _device.PinnedArena())
    return a


def streamed_body(raw, level: int = 1, chunk: int = CHUNK) -> tuple[dict, bytes]:
    """Streamed variant (formats/packed.py:63-81): lo raw, then the hi zstd stream."""
    a = np.frombuffer(raw, np.uint8) if not isinstance(raw, np.ndarray) else raw.reshape(-1).view(np.uint8)
    comp = zstd_host.ZstdCompressor(level=level)
    parts = []
    for s in range(0, a.size, chunk):
        parts.append(comp.compress(a[s:s + chunk][1::2]))
    parts.append(comp.flush())
    return {"lo": a.size // 2, "streamed": True}, a[0::2].tobytes() + b"".join(parts)


def write_vt(path: Path, head: dict, body: bytes) -> int:
    hj = json.dumps(head).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)) + hj + body)
    return len(hj) + 8 + len(body)


def _iter_safetensors(path: Path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        base = 8 + n
        for name, meta in header.items():
            if name == "__metadata__":
                continue
            a, b = meta["data_offsets"]
            f.seek(base + a)
            yield name, meta, f.read(b - a)


def pack_model(model_dir: str | Path, out_dir: str | Path | None = None, level: int = 1,
               encoder: str = "host", batch_bytes: int = 512 << 20) -> Path:
    """Pack every *.safetensors tensor of model_dir into a vpack directory
    (formats/packed.py:125-358 layout, including the per-expert split of fused
    BF16 MoE tensors and the streamed variant above STREAM_THRESHOLD).
    encoder="gpu" encodes the ordinary bodies' hi planes on the GPU (bodies_gpu,
    batches of about `batch_bytes`); streamed bodies use host zstd either way."""
    if encoder not in ("host", "gpu"):
        raise ValueError(f"encoder must be 'host' or 'gpu', got {encoder!r}")
    model_dir = Path(model_dir)
    out = Path(out_dir) if out_dir else model_dir / "weights.vpack"
    out.mkdir(parents=True, exist_ok=True)
    manifest: dict[str, str] = {}
    t0 = time.perf_counter()
    total_in = total_out = 0
    pending: list = []  # ordinary bodies waiting for a GPU batch: (name, fname, dtype, shape, raw)

    def emit(name, fname, dtype, shape, raw):
        nonlocal total_out
        if encoder == "gpu":
            pending.append((name, fname, dtype, shape, raw))
            if sum(len(p[4]) for p in pending) >= batch_bytes:
                flush()
            return
        head, body = body_for(dtype, raw, level)
        total_out += write_vt(out / fname, {"dtype": dtype, "shape": shape, **head}, body)
        manifest[name] = fname

    def flush():
        nonlocal total_out
        if not pending:
            return
        for (name, fname, dtype, shape, _), (head, body) in zip(pending, bodies_gpu([(p[2], p[4]) for p in pending])):
            total_out += write_vt(out / fname, {"dtype": dtype, "shape": shape, **head}, body)
            manifest[name] = fname
        pending.clear()

    for shard in sorted(model_dir.glob("*.safetensors")):
        for name, meta, raw in _iter_safetensors(shard):
            fused = _FUSED_BF16_EXPERT_RE.match(name)
            if fused and len(meta["shape"]) == 3 and meta["shape"][0] > 1 and meta["dtype"] in PLANE_DTYPES:
                n_e = meta["shape"][0]
                row = len(raw) // n_e
                for e in range(n_e):
                    raw_e = raw[e * row:(e + 1) * row]
                    if fused.group(2) == "gate_up_proj":
                        half, inter = row // 2, meta["shape"][1] // 2
                        parts = (("gate_proj.weight", [inter, meta["shape"][2]], raw_e[:half]),
                                 ("up_proj.weight", [inter, meta["shape"][2]], raw_e[half:]))
                    else:
                        parts = (("down_proj.weight", list(meta["shape"][1:]), raw_e),)
                    for proj, shape, sub in parts:
                        sub_name = f"{fused.group(1)}.{e}.{proj}"
                        emit(sub_name, sub_name.replace("/", "__") + ".vt", meta["dtype"], shape, sub)
                total_in += len(raw)
                continue
            fname = name.replace("/", "__") + ".vt"
            if meta["dtype"] in PLANE_DTYPES and len(raw) > STREAM_THRESHOLD:
                head, body = streamed_body(raw, level)
                total_out += write_vt(out / fname, {"dtype": meta["dtype"], "shape": meta["shape"], **head}, body)
                manifest[name] = fname
            else:
                emit(name, fname, meta["dtype"], meta["shape"], raw)
            total_in += len(raw)
    flush()
    (out / "manifest.json").write_text(json.dumps(manifest))
    dt = time.perf_counter() - t0
    print(f"packed {total_in / 1e9:.3f}GB -> {total_out / 1e9:.3f}GB "
          f"({total_in / max(total_out, 1):.3f}x) in {dt:.1f}s")
    return out


def _job_row(head: dict, body_off: int, body_len: int, dst: int) -> tuple[tuple | None, int]:
    """body_job's record as a plain tuple (JOB_DTYPE field order)."""
    if "raw" in head:
        return None, int(head["raw"])
    lo = int(head["lo"])
    if head.get("streamed"):
        return (body_off + lo, body_len - lo, dst, lo, body_off, INTERLEAVE, 0), 2 * lo
    hz = int(head["hi_z"])
    return (body_off, hz, dst, lo, body_off + hz, INTERLEAVE, 0), 2 * lo


def body_job(head: dict, body_off: int, body_len: int, dst: int) -> tuple[np.ndarray | None, int]:
    """GPU job for one vpack body held at body_off in a source buffer:
    returns (job record or None for raw bodies, decoded byte count)."""
    row, n = _job_row(head, body_off, body_len, dst)
    return (None if row is None else np.array([row], dtype=JOB_DTYPE)), n


GROUP_BYTES = 64 << 20  # compressed bytes per pipelined group (at most MAX_GROUPS groups)
MAX_GROUPS = 4
_streams: dict = {}
_planners = None  # host threads that build the groups' plans side by side


def _plan_pool():
    global _planners
    if _planners is None:
        import concurrent.futures as cf

        _planners = cf.ThreadPoolExecutor(max_workers=MAX_GROUPS * 2, thread_name_prefix="voom-plan")
    return _planners


def _side_streams(dev: torch.device, n: int) -> list[torch.cuda.Stream]:
    """n cached streams of the device (a copy stream and the group streams)."""
    have = _streams.setdefault(dev.index, [])
    while len(have) < n:
        have.append(torch.cuda.Stream(dev))
    return have[:n]


def body_groups(offsets: list[int], lengths: list[int], groups: int | None = None) -> list[list[int]]:
    """Consecutive bodies cut into groups of about equal compressed bytes, for
    a decode that overlaps the upload of one group with the decode of the one
    before.  `groups` None: one group per GROUP_BYTES, at most MAX_GROUPS.
    One group when the bodies do not lie in ascending, non-overlapping order
    (the groups' byte ranges must not overlap)."""
    n = len(offsets)
    total = sum(lengths)
    g = groups if groups is not None else min(MAX_GROUPS, total // GROUP_BYTES)
    g = max(1, min(int(g), n))
    ordered = all(offsets[i] + lengths[i] <= offsets[i + 1] for i in range(n - 1))
    if g == 1 or not ordered:
        return [list(range(n))]
    out, cur, acc = [], [], 0
    for i, ln in enumerate(lengths):
        cur.append(i)
        acc += ln
        # close the group once it holds its share, or when the bodies left
        # are just enough for one per group still to open
        after, left = g - len(out) - 1, n - i - 1
        if after > 0 and left >= after and (acc >= total * (len(out) + 1) / g or left == after):
            out.append(cur)
            cur = []
    if cur:
        out.append(cur)
    return out


def decode_bodies(heads: list[dict], host_buf: np.ndarray, offsets: list[int], lengths: list[int], *,
                  device=None, src_dev: torch.Tensor | None = None, align: int = 256,
                  stream: torch.cuda.Stream | None = None,
                  groups: int | None = None) -> tuple[torch.Tensor, list[tuple[int, int]]]:
    """Decode many vpack bodies that sit in one host buffer (numpy, bytes or a
    CPU tensor; a pinned tensor is copied in asynchronous DMAs) and optionally
    already in `src_dev`, with batched GPU decodes.  Returns the device output
    buffer and each body's (offset, length) in it.

    The upload is enqueued before any host work, so the job records and the
    plan are built while it runs.  From a pinned host tensor the bodies go up
    in groups (`body_groups`; `groups` overrides the automatic count) on a
    copy stream, and each group's decode starts when its bytes have landed, so
    the upload of one group overlaps the decode of the groups before it."""
    from .. import _device

    dev = _device.require_cuda(device)
    upload_src = host_buf
    host_buf = _device.as_u8(host_buf)
    pinned = isinstance(upload_src, torch.Tensor) and upload_src.device.type == "cpu" and upload_src.is_pinned()
    parts = None
    if src_dev is None and pinned and any("raw" not in h for h in heads):
        parts = body_groups(list(offsets), list(lengths), groups)
    with torch.cuda.device(dev):
        comp = stream if stream is not None else torch.cuda.current_stream(dev)
        events = None
        if parts is not None and len(parts) > 1:
            src_dev, events = _upload_groups(dev, upload_src.reshape(-1).view(torch.uint8), offsets, lengths,
                                             parts, comp)
        elif src_dev is None:
            src_dev = _device.upload(upload_src, dev, stream=stream)
        rows, spans, raw_copies, job_of = [], [], [], {}
        dst = 0
        for i, (head, off, ln) in enumerate(zip(heads, offsets, lengths)):
            row, n = _job_row(head, off, ln, dst)
            if row is None:
                if ln < n:
                    raise EOFError("vpack raw body shorter than its head")
                raw_copies.append((off, dst, n))
            else:
                if "streamed" not in head and int(head["hi_z"]) + int(head["lo"]) > ln:
                    raise EOFError("vpack body shorter than its head")
                job_of[i] = len(rows)
                rows.append(row)
            spans.append((dst, n))
            dst += (n + align - 1) // align * align
        jobs = np.array(rows, dtype=JOB_DTYPE) if rows else np.zeros(0, dtype=JOB_DTYPE)
        if events is not None:
            out = _decode_grouped(dev, src_dev, events, host_buf, parts, jobs, job_of, raw_copies, dst, comp)
            return out, spans
        out = torch.empty(max(dst, 1), dtype=torch.uint8, device=dev)
        for off, d, n in raw_copies:
            out[d:d + n].copy_(src_dev[off:off + n])
        if rows:
            plan = ZstdPlan(host_buf, jobs)
            batch = ZstdBatch(plan, dev)
            batch.run(src_dev, out, stream)
            st = batch.job_status()
            if st.any():
                bad = int(np.nonzero(st)[0][0])
                raise ZstdError(describe(int(st[bad])))
    return out, spans


def _upload_groups(dev, pinned: torch.Tensor, offsets, lengths, parts, comp) -> tuple[torch.Tensor, list]:
    """The source buffer on the device, each group's byte range copied on the
    copy stream (in group order) with an event after it."""
    from .. import _device

    cs = _side_streams(dev, 1)[0]
    n_src = int(pinned.numel())
    with torch.cuda.stream(comp):
        src_dev = torch.empty(n_src + _device.PAD, dtype=torch.uint8, device=dev)
        src_dev[n_src:].zero_()
    cs.wait_stream(comp)  # the buffer exists before the copies write it
    events = []
    for part in parts:
        lo = offsets[part[0]]
        hi = offsets[part[-1]] + lengths[part[-1]]
        with torch.cuda.stream(cs):
            src_dev[lo:hi].copy_(pinned[lo:hi], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(cs)
        events.append(ev)
    src_dev.record_stream(cs)
    return src_dev, events


def _decode_grouped(dev, src_dev: torch.Tensor, events: list, host_buf: np.ndarray, parts, jobs: np.ndarray,
                    job_of: dict, raw_copies, dst: int, comp) -> torch.Tensor:
    """decode_bodies over body groups: group g's decode runs on a stream of its
    own once its copy has landed, so the decodes of the groups overlap one
    another as well as the later copies.  Every kernel read of a body stays
    inside the source buffer; bytes past a body's end (the next group's,
    possibly still in flight) never reach its output, as with any neighbouring
    body.  One status read at the end raises the first failing body's fault."""
    gs = _side_streams(dev, 1 + len(parts))[1:]
    with torch.cuda.stream(comp):
        out = torch.empty(max(dst, 1), dtype=torch.uint8, device=dev)
    # the plans are built side by side, one host thread each (the native
    # planner runs without the GIL and starts no threads of its own for
    # threads=1); each group's decode is enqueued as soon as its plan is ready
    futs = []
    for part in parts:
        idx = [job_of[i] for i in part if i in job_of]
        futs.append(_plan_pool().submit(ZstdPlan, host_buf, jobs[idx], 1) if idx else None)
    batches = []
    for fut, ev, g in zip(futs, events, gs):
        if fut is None:
            continue
        plan = fut.result()
        g.wait_stream(comp)
        g.wait_event(ev)
        with torch.cuda.stream(g):
            batch = ZstdBatch(plan, dev, stream=g)
            batch.run(src_dev, out, g)
        batches.append((batch, g))
    for b, g in batches:
        comp.wait_stream(g)
        for t in (src_dev, out, b.scratch, b.status, b.d_plan):
            t.record_stream(g)
    with torch.cuda.stream(comp):
        comp.wait_event(events[-1])
        for off, d, n in raw_copies:
            out[d:d + n].copy_(src_dev[off:off + n])
        st = torch.cat([b.status[:b.plan.jobs.size] for b, _ in batches]).cpu().numpy().view(np.uint32)
    st = st | np.concatenate([b.plan.plan_status[:b.plan.jobs.size] for b, _ in batches])
    if st.any():
        bad = int(np.nonzero(st)[0][0])
        raise ZstdError(describe(int(st[bad])))
    return out


def read_tensor_bytes(vpack_dir: str | Path, fname: str, *, device=None) -> tuple[dict, torch.Tensor]:
    """Read + decode one `.vt` tensor to its original raw bytes on the GPU."""
    with open(Path(vpack_dir) / fname, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        head = json.loads(f.read(n))
        body = f.read()
    buf = np.frombuffer(body, np.uint8)
    out, spans = decode_bodies([head], buf, [0], [len(body)], device=device)
    d, ln = spans[0]
    return head, out[d:d + ln]


def to_torch(head: dict, raw: torch.Tensor) -> torch.Tensor:
    """Decoded bytes -> typed tensor of head['shape'] (formats/packed.py:385-397)."""
    dt = TORCH_DTYPES[head["dtype"]]
    return raw.view(dt).reshape(head["shape"])


to_mx = to_torch  # the reference's name for the same step
