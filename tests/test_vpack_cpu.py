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
