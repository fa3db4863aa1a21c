"""CPU tests for vpack / vpack2: the pack side reproduces the reference's
archive byte for byte, the oracle decode matches the reference's decoded
bytes, and the reader's integrity gates (tests/test_vpack2_integrity.py of
the reference) hold."""

from __future__ import annotations

import hashlib
import json
import shutil
from pathlib import Path

import numpy as np
import pytest

from oracle import vpack as ov
from tests.conftest import GOLDEN
from tests.golden.make_golden import TINY, write_safetensors
from voom_b200 import synthetic


def sha(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


@pytest.fixture(scope="module")
def golden():
    archive = (GOLDEN / "vpack2_tiny.bin").read_bytes()
    index = json.loads((GOLDEN / "vpack2_tiny.index.json").read_text())
    dec = json.loads((GOLDEN / "vpack2_tiny.decoded.json").read_text())
    return archive, index, dec


def source_tensors():
    t = []
    for i, (name, shape) in enumerate(synthetic.smollm2_tensors(TINY)):
        t.append((name, "BF16", list(shape), synthetic.bf16_normal(shape, 0.02, 500 + i).tobytes()))
    t.append(("model.layers.1.mlp.experts.gate_up_proj", "BF16", [4, 32, 64],
              synthetic.bf16_normal((4, 32, 64), 0.02, 99).tobytes()))
    t.append(("model.layers.1.mlp.router.scale", "F32", [8], np.arange(8, dtype=np.float32).tobytes()))
    return t


def test_source_regenerates(golden):
    _, _, dec = golden
    for name, _, _, raw in source_tensors():
        assert sha(raw) == dec["source_sha256"][name]


def test_pack_side_reproduces_reference_archive(tmp_path, golden):
    from voom_b200.formats import packed, packed2

    archive, index, _ = golden
    write_safetensors(tmp_path / "model.safetensors", source_tensors())
    packed.pack_model(tmp_path, level=1)
    packed2.build_from_vpack(tmp_path)
    assert (tmp_path / "weights.vpack2").read_bytes() == archive
    ours = json.loads((tmp_path / "weights.vpack2.index.json").read_text())
    assert ours == index


def test_oracle_decodes_reference_archive(golden):
    archive, index, dec = golden
    for name, e in index.items():
        raw = ov.decode_body(e["head"], archive[e["off"]:e["off"] + e["len"]])
        assert sha(raw.tobytes()) == dec["decoded_sha256"][name], name


def _fixture_dir(tmp_path: Path, body: bytes = b"exact-bf16-body", hashed: bool = True) -> Path:
    (tmp_path / "weights.vpack2").write_bytes(body)
    entry = {"off": 0, "len": len(body), "head": {"raw": len(body), "dtype": "U8", "shape": [len(body)]}}
    if hashed:
        entry["sha"] = hashlib.sha256(body).hexdigest()[:32]
    (tmp_path / "weights.vpack2.index.json").write_text(json.dumps({"w": entry}))
    return tmp_path


def test_integrity_valid_hash(tmp_path):
    from voom_b200.formats.packed2 import Vpack2Reader

    r = Vpack2Reader(_fixture_dir(tmp_path))
    assert r._checked_body("w", r.index["w"], b"exact-bf16-body") == b"exact-bf16-body"


def test_integrity_missing_hash_fails_closed(tmp_path):
    from voom_b200.formats.packed2 import Vpack2Reader

    with pytest.raises(ValueError, match="hash"):
        Vpack2Reader(_fixture_dir(tmp_path, hashed=False), require_hashes=True)


def test_integrity_corrupt_body_rejected(tmp_path):
    from voom_b200.formats.packed2 import Vpack2Reader

    r = Vpack2Reader(_fixture_dir(tmp_path))
    with pytest.raises(IOError, match="hash mismatch"):
        r._checked_body("w", r.index["w"], b"corrupt")


def test_integrity_archive_mutation_rejected(tmp_path):
    from voom_b200.formats.packed2 import Vpack2Reader

    d = _fixture_dir(tmp_path)
    r = Vpack2Reader(d)
    with (d / "weights.vpack2").open("ab") as f:
        f.write(b"!")
    with pytest.raises(IOError, match="changed"):
        r._assert_archive_immutable()


def test_index_validation_rejects_gaps(tmp_path, golden):
    from voom_b200.formats.packed2 import Vpack2Reader

    archive, index, _ = golden
    (tmp_path / "weights.vpack2").write_bytes(archive)
    bad = dict(index)
    first = min(bad, key=lambda n: bad[n]["off"])
    bad[first] = dict(bad[first], off=bad[first]["off"] + 1)
    (tmp_path / "weights.vpack2.index.json").write_text(json.dumps(bad))
    with pytest.raises(ValueError, match="gap/overlap"):
        Vpack2Reader(tmp_path)


def test_access_order_matches_reference_layout(golden):
    from voom_b200.formats.packed2 import access_order

    _, index, _ = golden
    by_off = [n for n, _ in sorted(index.items(), key=lambda kv: kv[1]["off"])]
    assert access_order(list(index)) == by_off


def test_run_coalescing_matches_the_sequential_rule():
    """Vpack2Reader.fetch's vectorised run split against a direct restatement
    of formats/packed2.py:361-372 (extend the run while the next body starts
    within RUN_GAP of the furthest end so far)."""
    import random

    from voom_b200.formats.packed2 import _coalesce

    def runs(ext, gap):
        out, i = [], 0
        while i < len(ext):
            start, end, j = ext[i][0], ext[i][0] + ext[i][1], i + 1
            while j < len(ext) and ext[j][0] - end <= gap:
                end = max(end, ext[j][0] + ext[j][1])
                j += 1
            out.append((start, end, j - i))
            i = j
        return out

    rnd = random.Random(7)
    for _ in range(2000):
        ext = sorted((rnd.randint(0, 100), rnd.randint(0, 30)) for _ in range(rnd.randint(1, 12)))
        gap = rnd.randint(0, 20)
        run, covered = _coalesce(np.array([a for a, _ in ext]), np.array([b for _, b in ext]), gap)
        want = runs(ext, gap)
        assert int(run[-1]) + 1 == len(want)
        assert covered == sum(e - s for s, e, _ in want)
        assert [int((run == k).sum()) for k in range(len(want))] == [c for *_, c in want]


def test_verify_generation_extents_and_hashes(tmp_path):
    """The audit without decoding (CPU): a clean archive, then a damaged body
    and a truncated file, with the reference's report messages."""
    import json
    import shutil

    from tests.conftest import GOLDEN
    from voom_b200.formats.packed2 import verify_generation

    shutil.copy(GOLDEN / "vpack2_tiny.bin", tmp_path / "weights.vpack2")
    shutil.copy(GOLDEN / "vpack2_tiny.index.json", tmp_path / "weights.vpack2.index.json")
    index = json.loads((tmp_path / "weights.vpack2.index.json").read_text())
    rep = verify_generation(tmp_path, decode=False)
    assert rep["errors"] == [] and rep["tensors"] == len(index) == rep["hashed"]
    name = sorted(index, key=lambda n: index[n]["off"])[3]
    blob = bytearray((tmp_path / "weights.vpack2").read_bytes())
    blob[index[name]["off"] + 1] ^= 0xFF
    (tmp_path / "weights.vpack2").write_bytes(bytes(blob))
    rep = verify_generation(tmp_path, decode=False)
    assert rep["errors"] == [f"hash mismatch at {name}"]
    last = max(index, key=lambda n: index[n]["off"])
    (tmp_path / "weights.vpack2").write_bytes(bytes(blob[:-5]))
    rep = verify_generation(tmp_path, decode=False)
    end = index[last]["off"] + index[last]["len"]
    assert rep["errors"] == [f"archive size {end - 5} != indexed extent end {end}",
                             f"hash mismatch at {name}", f"short read at {last}"]


def test_body_groups_for_the_pipelined_upload():
    """Groups of consecutive bodies with about equal compressed bytes, every
    group non-empty; one group for small batches (under GROUP_BYTES per group)
    and for bodies out of order or overlapping."""
    from voom_b200.formats import packed

    lens = [5, 1, 1, 1, 8, 2, 2, 9, 3, 1]
    offs = np.cumsum([0] + lens[:-1]).tolist()
    for g in range(1, len(lens) + 1):
        parts = packed.body_groups(offs, lens, g)
        assert len(parts) == g
        assert [i for p in parts for i in p] == list(range(len(lens)))
        assert all(parts)
    # about equal bytes: no group of the 3-way cut holds more than half
    assert max(sum(lens[i] for i in p) for p in packed.body_groups(offs, lens, 3)) <= 17
    assert packed.body_groups(offs, lens, 99) == [[i] for i in range(len(lens))]
    assert packed.body_groups(offs, lens) == [list(range(len(lens)))]  # 33 bytes: one group
    big = [packed.GROUP_BYTES] * 10
    assert len(packed.body_groups(np.cumsum([0] + big[:-1]).tolist(), big)) == packed.MAX_GROUPS
    assert packed.body_groups([10, 0], [10, 10], 2) == [[0, 1]]  # out of order
    assert packed.body_groups([0, 5], [10, 10], 2) == [[0, 1]]  # overlapping

