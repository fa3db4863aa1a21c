"""GPU parity for vpack / vpack2 decode (batched zstd + lo/hi interleave on the
device) against the reference's archive and its decoded bytes."""

from __future__ import annotations

import hashlib
import json
import shutil

import numpy as np
import pytest
import torch

from oracle import vpack as ov
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu


def sha(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


@pytest.fixture()
def archive_dir(tmp_path, built_lib):
    shutil.copy(GOLDEN / "vpack2_tiny.bin", tmp_path / "weights.vpack2")
    shutil.copy(GOLDEN / "vpack2_tiny.index.json", tmp_path / "weights.vpack2.index.json")
    return tmp_path


@pytest.fixture(scope="module")
def decoded():
    return json.loads((GOLDEN / "vpack2_tiny.decoded.json").read_text())["decoded_sha256"]


def test_reader_fetch_matches_reference(archive_dir, decoded):
    from voom_b200.formats.packed import TORCH_DTYPES
    from voom_b200.formats.packed2 import Vpack2Reader

    r = Vpack2Reader(archive_dir, require_hashes=True)
    names = list(r.index)
    tensors, secs, nbytes = r.fetch(names)
    assert set(tensors) == set(names)
    assert nbytes == (archive_dir / "weights.vpack2").stat().st_size
    for n in names:
        t = tensors[n]
        head = r.index[n]["head"]
        assert t.is_cuda and t.dtype == TORCH_DTYPES[head["dtype"]] and list(t.shape) == head["shape"]
        assert sha(t.contiguous().view(torch.uint8).cpu().numpy().tobytes()) == decoded[n], n


def test_reader_fetch_subset_and_runs(archive_dir, decoded):
    from voom_b200.formats.packed2 import Vpack2Reader

    r = Vpack2Reader(archive_dir)
    names = [n for n in r.index if ".experts." in n][::3] + ["model.embed_tokens.weight"]
    tensors, _, _ = r.fetch(names, parallel=2)
    for n in names:
        assert sha(tensors[n].view(torch.uint8).cpu().numpy().tobytes()) == decoded[n]


def test_decode_body_each(archive_dir, decoded):
    from voom_b200.formats.packed2 import decode_body

    archive = (archive_dir / "weights.vpack2").read_bytes()
    index = json.loads((archive_dir / "weights.vpack2.index.json").read_text())
    for n, e in index.items():
        got = decode_body(e["head"], archive[e["off"]:e["off"] + e["len"]])
        assert sha(got.cpu().numpy().tobytes()) == decoded[n]


def test_streamed_variant(built_lib):
    from voom_b200 import synthetic
    from voom_b200.formats import packed
    from voom_b200.formats.packed2 import decode_body

    raw = synthetic.bf16_normal((3, 700_001), 0.02, 8).view(np.uint8)  # odd element count, 3 zstd calls
    head, body = packed.streamed_body(raw, level=1, chunk=1 << 20)
    assert head["streamed"] and head["lo"] == raw.size // 2
    got = decode_body(head, body).cpu().numpy()
    assert np.array_equal(got, raw.reshape(-1))
    assert np.array_equal(ov.decode_body(head, body), raw.reshape(-1))


def test_corrupt_body_hash_mismatch_refused(archive_dir):
    """The hashes run alongside the GPU decode; a mismatch is still the error
    raised (before any tensor is returned), also when the damaged body no
    longer decodes."""
    from voom_b200.formats.packed2 import Vpack2Reader

    data = bytearray((archive_dir / "weights.vpack2").read_bytes())
    data[100] ^= 1
    (archive_dir / "weights.vpack2").write_bytes(bytes(data))
    r = Vpack2Reader(archive_dir)
    with pytest.raises(IOError, match="hash mismatch"):
        r.fetch(list(r.index))
    assert r.tensors_read == 0


def test_reader_reuses_pinned_buffer(archive_dir, decoded):
    from voom_b200.formats.packed2 import Vpack2Reader

    r = Vpack2Reader(archive_dir, require_hashes=True)
    names = sorted(r.index)
    a, _, _ = r.fetch(names)
    buf = r._host
    assert buf is not None and buf.is_pinned()
    b, _, _ = r.fetch(names[: len(names) // 2], parallel=3)
    assert r._host is buf
    for n in b:
        assert torch.equal(a[n], b[n])


def test_smollm2_scaled_archive(built_lib):
    from voom_b200 import synthetic
    from voom_b200.formats import packed

    cfg = dict(synthetic.SMOLLM2_135M, layers=2)
    heads, bodies, raws = [], [], []
    for i, (name, shape) in enumerate(synthetic.smollm2_tensors(cfg)):
        bits = synthetic.bf16_normal(shape, 0.02, 40 + i)
        h, b = packed.body_for("BF16", bits.view(np.uint8))
        heads.append({"dtype": "BF16", "shape": list(shape), **h})
        bodies.append(b)
        raws.append(bits.view(np.uint8).reshape(-1))
    offs = np.cumsum([0] + [len(b) for b in bodies[:-1]]).tolist()
    buf = np.frombuffer(b"".join(bodies), np.uint8)
    out, spans = packed.decode_bodies(heads, buf, offs, [len(b) for b in bodies])
    got = out.cpu().numpy()
    for (d, n), r in zip(spans, raws):
        assert np.array_equal(got[d:d + n], r)


def test_packed_weight_store_fetch(archive_dir, decoded):
    """WeightStore leg over the reference's archive: canonical -> stored name
    translation at the archive boundary, duplicates fetched once, every page
    decoded on the device in one batched call (the reference's WeightCache
    calls exactly this fetch, runtime/weight_cache.py:116-122)."""
    from voom_b200.runtime.weight_store import PackedWeightStore

    index = json.loads((archive_dir / "weights.vpack2.index.json").read_text())
    stored = sorted(index)
    real = {f"model.{n}": n for n in stored}
    store = PackedWeightStore(archive_dir, real_name=real, require_hashes=True)
    logical = [f"model.{n}" for n in stored]
    tensors, secs, nbytes = store.fetch(logical + logical[:3])
    assert sorted(tensors) == sorted(logical) and secs >= 0
    for name in logical:
        t = tensors[name]
        assert t.is_cuda
        assert sha(t.contiguous().view(torch.uint8).cpu().numpy().tobytes()) == decoded[real[name]], name
    assert nbytes == store.archive_bytes > 0

def test_verify_generation_decodes_every_body(archive_dir):
    """The full audit: every body hashed and decoded in one batched GPU decode;
    a body whose stream is damaged but whose digest was rewritten to match is
    named by the per-body attribution pass."""
    from voom_b200.formats.packed2 import verify_generation

    index = json.loads((archive_dir / "weights.vpack2.index.json").read_text())
    rep = verify_generation(archive_dir)
    assert rep["errors"] == [] and rep["decoded"] == rep["tensors"] == len(index)
    name = next(n for n in sorted(index, key=lambda n: index[n]["off"])
                if "raw" not in index[n]["head"] and index[n]["len"] > 4096)
    e = index[name]
    blob = bytearray((archive_dir / "weights.vpack2").read_bytes())
    blob[e["off"] + 1] ^= 0xFF  # the zstd magic number of the hi plane
    e["sha"] = sha(blob[e["off"]:e["off"] + e["len"]])[:32]
    (archive_dir / "weights.vpack2").write_bytes(bytes(blob))
    (archive_dir / "weights.vpack2.index.json").write_text(json.dumps(index))
    rep = verify_generation(archive_dir)
    assert len(rep["errors"]) == 1 and rep["errors"][0].startswith(f"decode failure at {name}: ")
    assert rep["decoded"] == len(index) - 1
