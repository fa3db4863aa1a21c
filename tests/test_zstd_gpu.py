"""GPU parity for the zstd decoder (through the C ABI): bit-exact against
libzstd / the oracle on frames produced like the reference produces them."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import zstd as oz
from tests.zstd_cases import cases

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def Z(built_lib):
    from voom_b200.formats import zstd_gpu

    return zstd_gpu


@pytest.fixture(scope="module")
def frames():
    return cases()


def test_single_frames_bit_exact(Z, frames):
    bad = []
    for name, fr, raw in frames:
        got = Z.decompress(fr, size=len(raw))
        if got != raw:
            bad.append(name)
    assert not bad, bad


def test_batch_with_interleave_bit_exact(Z, frames):
    # every case as one job of one batch; half of them interleaved with a lo plane
    rng = np.random.default_rng(3)
    src = bytearray()
    jobs = np.zeros(len(frames), dtype=Z.JOB_DTYPE)
    expect = []
    dst = 0
    for i, (name, fr, raw) in enumerate(frames):
        inter = i % 2 == 0
        lo = rng.integers(0, 256, len(raw), dtype=np.uint8).tobytes() if inter else b""
        off = len(src)
        src += fr
        lo_off = len(src)
        src += lo
        jobs[i] = (off, len(fr), dst, len(raw), lo_off, Z.INTERLEAVE if inter else 0, 0)
        if inter:
            e = np.empty(2 * len(raw), np.uint8)
            e[0::2] = np.frombuffer(lo, np.uint8)
            e[1::2] = np.frombuffer(raw, np.uint8)
            expect.append((dst, e.tobytes()))
            dst += 2 * len(raw)
        else:
            expect.append((dst, raw))
            dst += len(raw)
        dst = (dst + 15) // 16 * 16
    host = np.frombuffer(bytes(src), np.uint8)
    plan = Z.ZstdPlan(host, jobs)
    dev = torch.device("cuda", 0)
    from voom_b200 import _device

    d_src = _device.upload(host, dev)
    out = torch.zeros(max(dst, 1), dtype=torch.uint8, device=dev)
    batch = Z.ZstdBatch(plan, dev)
    for _ in range(2):  # the batch is reusable
        batch.run(d_src, out)
        st = batch.job_status()
        assert not st.any(), [(frames[i][0], Z.describe(int(s))) for i, s in enumerate(st) if s]
        got = out.cpu().numpy()
        for (name, _, _), (d, e) in zip(frames, expect):
            assert got[d:d + len(e)].tobytes() == e, name


def test_corrupted_frames_fail_closed(Z, frames):
    """Damaged frames: the GPU decoder takes the oracle's decision (both check
    that every entropy stream is consumed exactly, RFC 8878 4.1/4.2), never
    accepts a frame libzstd rejects, and when it accepts, its bytes equal
    libzstd's.  libzstd itself accepts some damaged frames and returns wrong
    bytes; in the reference the per-body SHA-256 of vpack2 catches those."""
    name, fr, raw = frames[0]
    rng = np.random.default_rng(11)
    rejected = 0
    for _ in range(40):
        b = bytearray(fr)
        b[int(rng.integers(0, len(b)))] ^= int(rng.integers(1, 256))
        b = bytes(b)
        try:
            ref = oz.libzstd_decompress(b, len(raw) + 64)
        except oz.ZstdError:
            ref = None
        try:
            orc = oz.decompress(b, capacity=len(raw) + 64)
        except oz.ZstdError:
            orc = None
        try:
            got = Z.decompress(b, size=len(raw))
        except Z.ZstdError:
            got = None
        assert (got is None) == (orc is None)
        if got is not None:
            assert got == orc
            assert ref is not None and got == ref
        else:
            rejected += 1
    assert rejected > 10


def test_large_hi_plane_multi_block(Z):
    from voom_b200 import synthetic
    from voom_b200.formats import zstd_host as zh

    hi = synthetic.bf16_normal((8 << 20,), 0.02, 5).view(np.uint8)[1::2].tobytes()  # 8 MiB, 64 blocks
    fr = zh.compress(hi, 1)
    assert Z.decompress(fr) == hi


def test_direct_and_segmented_batch_bit_exact(Z):
    """One batch of literal-only KV frames (decoded straight to the output,
    one lane per Huffman stream) and 1.25 GiB of matched jobs (two Z-space
    segments), bit-exact."""
    from voom_b200 import _device, synthetic
    from voom_b200.formats import zstd_host as zh

    k, v = synthetic.kv_pages(64, seed=6)
    pages = [k[i].tobytes() for i in range(64)] + [v[i].tobytes() for i in range(64)]
    lit_frames = [zh.compress(p, 1) for p in pages]
    rep = (np.arange(1 << 22, dtype=np.uint32) % 1021).astype(np.uint8)
    rep[::4093] ^= 0x5A
    seq_frame = zh.compress(rep.tobytes(), 1)
    n_rep = 320  # 1.25 GiB of matched output
    src = b"".join(lit_frames) + seq_frame
    jobs = np.zeros(len(pages) + n_rep, dtype=Z.JOB_DTYPE)
    off = dst = 0
    for i, f in enumerate(lit_frames):
        jobs[i] = (off, len(f), dst, 32768, 0, 0, 0)
        off += len(f)
        dst += 32768
    for i in range(n_rep):
        jobs[len(pages) + i] = (off, len(seq_frame), dst, rep.size, 0, 0, 0)
        dst += rep.size
    plan = Z.ZstdPlan(np.frombuffer(src, np.uint8), jobs)
    assert plan.info.n_segments == 2 and plan.info.n_direct_jobs == len(pages)
    dev = torch.device("cuda", 0)
    d_src = _device.upload(np.frombuffer(src, np.uint8), dev)
    out = torch.empty(dst, dtype=torch.uint8, device=dev)
    batch = Z.ZstdBatch(plan, dev)
    batch.run(d_src, out)
    assert not batch.job_status().any()
    lit_out = out[:len(pages) * 32768].cpu().numpy()
    assert lit_out.tobytes() == b"".join(pages)
    reps = out[len(pages) * 32768:].view(n_rep, rep.size)
    assert torch.equal(reps, torch.from_numpy(rep).to(dev).expand(n_rep, -1))


def test_direct_literals_unaligned_outputs_and_damage(Z):
    """Direct jobs at odd output offsets (byte head / tail around the 32-bit
    stores), single-stream literals, and a truncated literal stream that must
    be reported, never accepted."""
    from voom_b200 import _device, synthetic
    from voom_b200.formats import zstd_host as zh

    rng = np.random.default_rng(12)
    k, _ = synthetic.kv_pages(6, seed=2)
    raws = [k[i].tobytes()[:n] for i, n in enumerate([32768, 32767, 1500, 200, 9001, 32766])]
    frames = [zh.compress(r, 1) for r in raws]
    src = b"".join(frames)
    jobs = np.zeros(len(raws), dtype=Z.JOB_DTYPE)
    off, dst = 0, 3
    for i, (f, r) in enumerate(zip(frames, raws)):
        jobs[i] = (off, len(f), dst, len(r), 0, 0, 0)
        off += len(f)
        dst += len(r) + int(rng.integers(1, 7))
    plan = Z.ZstdPlan(np.frombuffer(src, np.uint8), jobs)
    assert plan.info.n_direct_jobs == len(raws)
    dev = torch.device("cuda", 0)
    out = torch.zeros(dst + 16, dtype=torch.uint8, device=dev)
    batch = Z.ZstdBatch(plan, dev)
    batch.run(_device.upload(np.frombuffer(src, np.uint8), dev), out)
    assert not batch.job_status().any()
    got = out.cpu().numpy()
    for j, r in zip(jobs, raws):
        assert got[int(j["dst"]):int(j["dst"]) + len(r)].tobytes() == r
    # a frame whose last literal stream lost bytes: rejected like the oracle
    f = bytearray(frames[0])
    bad = bytes(f[:-30]) + bytes(30)
    assert oz_reject(bad, len(raws[0]))
    with pytest.raises(Z.ZstdError):
        Z.decompress(bad, size=len(raws[0]))


def oz_reject(frame: bytes, n: int) -> bool:
    try:
        oz.decompress(frame, capacity=n + 64)
    except oz.ZstdError:
        return True
    return False


def test_direct_literals_short_codes(Z):
    """Literal-only frames whose Huffman codes are shorter than 11 bits (small,
    skewed alphabets) next to 11-bit ones (KV bytes), decoded in one batch."""
    from voom_b200 import _device, synthetic
    from voom_b200.formats import zstd_host as zh

    rng = np.random.default_rng(21)
    raws = []
    for alpha, n in ((3, 5000), (12, 20000), (40, 30000), (90, 7777), (200, 32768)):
        p = rng.dirichlet(np.ones(alpha) * 0.7)
        raws.append(rng.choice(alpha, size=n, p=p).astype(np.uint8).tobytes())
    k, _ = synthetic.kv_pages(2, seed=9)
    raws += [k[0].tobytes(), k[1].tobytes()[:20001]]
    frames = [zh.compress(r, 1) for r in raws]
    jobs = np.zeros(len(raws), dtype=Z.JOB_DTYPE)
    off = dst = 0
    for i, (f, r) in enumerate(zip(frames, raws)):
        jobs[i] = (off, len(f), dst, len(r), 0, 0, 0)
        off += len(f)
        dst += len(r)
    src = b"".join(frames)
    plan = Z.ZstdPlan(np.frombuffer(src, np.uint8), jobs)
    assert plan.info.n_direct_jobs >= 3
    dev = torch.device("cuda", 0)
    out = torch.empty(dst, dtype=torch.uint8, device=dev)
    batch = Z.ZstdBatch(plan, dev)
    batch.run(_device.upload(np.frombuffer(src, np.uint8), dev), out)
    assert not batch.job_status().any()
    assert out.cpu().numpy().tobytes() == b"".join(raws)


def _text(n: int, seed: int) -> bytes:
    """Bytes with many short matches (level 1 emits sequences for them)."""
    rng = np.random.default_rng(seed)
    words = [bytes(rng.integers(97, 123, rng.integers(2, 9), dtype=np.uint8)) for _ in range(200)]
    out = bytearray()
    while len(out) < n:
        out += words[int(rng.integers(0, len(words)))] + b" "
    return bytes(out[:n])


@pytest.mark.parametrize("first_len", [70_000, 300_000])
def test_frame_longer_than_its_job_leaves_the_next_job_intact(Z, first_len):
    """A frame without a content size whose decoded bytes exceed its job's
    dst_len must be rejected without writing past that job's share of the
    decode scratch: the next job of the same batch stays bit-exact."""
    from voom_b200 import _device
    from voom_b200.formats import zstd_host

    long_raw = _text(first_len, 1)
    c = zstd_host.ZstdCompressor(level=1)
    long_fr = c.compress(long_raw) + c.flush()  # streamed: no frame content size
    assert Z.frame_content_size(long_fr) is None
    ok_raw = _text(90_000, 2)
    ok_fr = zstd_host.compress(ok_raw, 1)
    short = first_len // 3  # the caller's (wrong) output size for the first job
    src = long_fr + ok_fr
    jobs = np.zeros(2, dtype=Z.JOB_DTYPE)
    d1 = (short + 255) // 256 * 256
    jobs[0] = (0, len(long_fr), 0, short, 0, 0, 0)
    jobs[1] = (len(long_fr), len(ok_fr), d1, len(ok_raw), 0, 0, 0)
    host = np.frombuffer(src, np.uint8)
    plan = Z.ZstdPlan(host, jobs)
    dev = torch.device("cuda", 0)
    d_src = _device.upload(host, dev)
    out = torch.full((d1 + len(ok_raw) + 4096,), 0xA5, dtype=torch.uint8, device=dev)
    batch = Z.ZstdBatch(plan, dev)
    for _ in range(2):
        batch.run(d_src, out)
        st = batch.job_status()
        assert st[0] & Z.ST_SIZE, Z.describe(int(st[0]))
        assert st[1] == 0, Z.describe(int(st[1]))
        got = out.cpu().numpy()
        assert got[d1:d1 + len(ok_raw)].tobytes() == ok_raw
        assert (got[d1 + len(ok_raw):] == 0xA5).all()  # nothing written past the last job


def test_long_chains_take_the_worklist_overflow_path(built_lib):
    """8 MiB copied from two bytes back: after the output pass almost every
    byte is still a link (its chain is far longer than 16 hops), many more
    than worklist 0 holds, so the resolve passes rescan the tiles (pointer
    jumping with path compression) and the patch pass rewrites them.  The
    output is exact and the job's status clean."""
    from voom_b200.formats import zstd_gpu
    from voom_b200.formats import zstd_host as zh

    for data in (b"ab" * (4 << 20), b"xyz" * (3 << 20)):
        fr = zh.compress(data, 1)
        got = zstd_gpu.decompress_device(fr, len(data)).cpu().numpy().tobytes()
        assert got == data
