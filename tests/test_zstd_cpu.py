"""CPU tests for the zstd path: the oracle (RFC 8878 restatement) pinned
against libzstd, and the GPU decoder's host planner."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import zstd as oz
from tests.zstd_cases import cases


@pytest.fixture(scope="module")
def frames():
    return cases()


def test_oracle_matches_libzstd(frames):
    for name, fr, raw in frames:
        assert oz.decompress(fr, capacity=len(raw) + 64) == raw, name
        assert oz.libzstd_decompress(fr, len(raw) + 64) == raw, name


def test_oracle_rejects_corruption_libzstd_rejects(frames):
    name, fr, raw = frames[0]
    rng = np.random.default_rng(7)
    both_reject = 0
    for _ in range(40):
        b = bytearray(fr)
        b[int(rng.integers(0, len(b)))] ^= int(rng.integers(1, 256))
        try:
            ref = oz.libzstd_decompress(bytes(b), len(raw) + 64)
        except oz.ZstdError:
            ref = None
        try:
            got = oz.decompress(bytes(b), capacity=len(raw) + 64)
        except oz.ZstdError:
            got = None
        if ref is None:
            both_reject += got is None
        # when libzstd accepts a damaged frame the oracle must produce the same bytes
        if ref is not None and got is not None:
            assert ref == got
    assert both_reject > 10


def test_xxh64_known_answers():
    # published XXH64 test values (seed 0)
    assert oz.xxh64(b"") == 0xEF46DB3751D8E999
    assert oz.xxh64(b"a") == 0xD24EC4F1A98C6E5B
    assert oz.xxh64(b"abc") == 0x44BC2CF5AD770999


def test_planner_walks_frames(built_lib, frames):
    from voom_b200.formats import zstd_gpu as Z

    src = b"".join(fr for _, fr, _ in frames)
    jobs = np.zeros(len(frames), dtype=Z.JOB_DTYPE)
    off = dst = 0
    for i, (_, fr, raw) in enumerate(frames):
        jobs[i] = (off, len(fr), dst, len(raw), 0, 0, 0)
        off += len(fr)
        dst += len(raw)
    plan = Z.ZstdPlan(np.frombuffer(src, np.uint8), jobs)
    assert plan.info.n_bad_jobs == 0
    assert plan.info.n_jobs == len(frames)
    assert plan.info.n_frames == len(frames) + 1  # one job holds two frames
    assert plan.info.scratch_bytes > 4 * sum(len(r) for _, _, r in frames)
    assert not plan.plan_status[: len(frames)].any()


def test_planner_flags_structural_damage(built_lib, frames):
    from voom_b200.formats import zstd_gpu as Z

    _, fr, raw = frames[0]
    bad = bytearray(fr)
    bad[0] ^= 0xFF  # magic
    jobs = np.zeros(2, dtype=Z.JOB_DTYPE)
    jobs[0] = (0, len(fr), 0, len(raw), 0, 0, 0)
    jobs[1] = (len(fr), len(fr), 0, len(raw), 0, 0, 0)
    plan = Z.ZstdPlan(np.frombuffer(bytes(fr) + bytes(bad), np.uint8), jobs)
    assert plan.plan_status[0] == 0 and plan.plan_status[1] == Z.ST_FORMAT


def test_frame_content_size(frames):
    from voom_b200.formats import zstd_gpu as Z

    for name, fr, raw in frames:
        fcs = Z.frame_content_size(fr)
        if name.startswith("streamed"):
            assert fcs is None
        else:
            assert fcs == len(raw), name


def test_planner_direct_jobs_and_segments(built_lib):
    """Jobs without sequences (and not interleaved) are planned direct, with
    no link-word scratch; jobs with matches are cut into segments of at most
    1 GiB of decoded bytes; one job above 2 GiB - 1 MiB is refused."""
    from voom_b200 import synthetic
    from voom_b200.formats import zstd_gpu as Z
    from voom_b200.formats import zstd_host as zh

    k, _ = synthetic.kv_pages(8, seed=3)
    lit_frames = [zh.compress(k[i].tobytes(), 1) for i in range(8)]
    rep = (np.arange(1 << 20, dtype=np.uint32) % 977).astype(np.uint8).tobytes()
    seq_frame = zh.compress(rep, 1)
    src = b"".join(lit_frames) + seq_frame
    n_rep = 2600  # 2600 MiB of matched output -> 3 segments
    jobs = np.zeros(8 + n_rep + 2, dtype=Z.JOB_DTYPE)
    off = 0
    for i, f in enumerate(lit_frames):
        jobs[i] = (off, len(f), i * 32768, 32768, 0, 0, 0)
        off += len(f)
    for i in range(n_rep):
        jobs[8 + i] = (off, len(seq_frame), (8 + i) << 20, 1 << 20, 0, 0, 0)
    jobs[8 + n_rep] = (0, len(lit_frames[0]), 0, 32768, 0, Z.INTERLEAVE, 0)  # interleaved: not direct
    jobs[9 + n_rep] = (off, len(seq_frame), 0, 3 << 30, 0, 0, 0)  # claims 3 GiB with matches
    plan = Z.ZstdPlan(np.frombuffer(src, np.uint8), jobs)
    info = plan.info
    assert info.n_direct_jobs == 8
    assert info.n_segments == 3
    assert plan.plan_status[9 + n_rep] == Z.ST_TOO_LARGE
    assert not plan.plan_status[:9 + n_rep].any()
    assert "too large" in Z.describe(Z.ST_TOO_LARGE)
    # the link words of the largest segment (1 GiB) bound the scratch
    assert 4 << 30 <= info.scratch_bytes < (4 << 30) + (1 << 30)

    only_direct = Z.ZstdPlan(np.frombuffer(src, np.uint8), jobs[:8])
    assert only_direct.info.n_direct_jobs == 8 and only_direct.info.scratch_bytes < (2 << 20)  # worklists only


def test_planner_direct_decision_edges(built_lib):
    """Direct (straight-to-output) planning only when every block size is
    known and adds up: raw blocks and multi-frame jobs qualify; a job length
    one byte off the frames' content, an interleaved job, or a block with
    sequences does not (those take the general path, which reports the
    mismatch)."""
    from voom_b200.formats import zstd_gpu as Z
    from voom_b200.formats import zstd_host as zh

    rng = np.random.default_rng(0)
    rand = rng.integers(0, 256, 200000, dtype=np.uint8).tobytes()
    cases = {"raw": (zh.compress(rand, 1), len(rand), True),
             "two_frames": (zh.compress(rand[:5000], 1) + zh.compress(rand[5000:9000], 1), 9000, True),
             "sequences": (zh.compress(bytes(150000), 1), 150000, False)}
    for name, (frame, n, direct) in cases.items():
        for extra, flags, want in ((0, 0, direct), (1, 0, False), (0, Z.INTERLEAVE, False)):
            job = np.zeros(1, Z.JOB_DTYPE)
            job[0] = (0, len(frame), 0, n + extra, len(frame) if flags else 0, flags, 0)
            plan = Z.ZstdPlan(np.frombuffer(frame + bytes(n + extra), np.uint8), job)
            assert plan.info.n_direct_jobs == int(want), (name, extra, flags)
            assert plan.plan_status[0] == 0


def test_planner_orders_blocks_for_the_sequence_walk(built_lib):
    """The plan image's walk order (the block list ordered by sequence count,
    most first, that zstd_block_decode pairs its walkers from) is a
    permutation of the block list, sorted, over frames of many blocks."""
    from voom_b200.formats import zstd_gpu as Z

    rng = np.random.default_rng(9)
    # small alphabets: many short matches, their count varying with the alphabet
    datas = [rng.integers(0, a, 300_000, dtype=np.uint8).tobytes() for a in (4, 12, 40)]
    datas.append(bytes(range(256)) * 700)  # very repetitive: few, long sequences
    from oracle import vpack as ov

    frames = [ov.zstd_compress(d, 1) for d in datas]
    jobs = np.zeros(len(frames), dtype=Z.JOB_DTYPE)
    off = dst = 0
    for i, (fr, d) in enumerate(zip(frames, datas)):
        jobs[i] = (off, len(fr), dst, len(d), 0, 0, 0)
        off += len(fr)
        dst += len(d)
    plan = Z.ZstdPlan(np.frombuffer(b"".join(frames), np.uint8), jobs)
    img = plan.image
    hdr = img[:128]
    n_blocks = int(hdr[8:12].view(np.uint32)[0])
    off_blocks = int(hdr[40:48].view(np.uint64)[0])
    n_blist = int(hdr[88:92].view(np.uint32)[0])
    off_blist, off_k1 = (int(x) for x in hdr[96:112].view(np.uint64))
    assert n_blist >= 4  # the blocks of jobs with sequences (direct jobs are not listed)
    blist = img[off_blist:off_blist + 4 * n_blist].view(np.uint32)
    k1 = img[off_k1:off_k1 + 4 * n_blist].view(np.uint32)
    rec = img[off_blocks:off_blocks + 112 * n_blocks].reshape(n_blocks, 112)
    btype = rec[:, 40:44].copy().view(np.uint32).reshape(-1)
    nseq = np.where(btype == 2, rec[:, 88:92].copy().view(np.uint32).reshape(-1), 0)
    assert sorted(k1.tolist()) == sorted(blist.tolist())  # one segment here
    walk = nseq[k1]
    assert (np.diff(walk.astype(np.int64)) <= 0).all() and walk[0] > walk[-1]
