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


def test_grouped_upload_decode_matches_single_dma(built_lib):
    """From a pinned buffer the bodies go up in groups on a copy stream, each
    group's decode waiting for its own bytes only: the output equals the
    single-DMA decode byte for byte (raw-stored bodies included), and a damaged
    body in the last group raises the same error."""
    from voom_b200 import synthetic
    from voom_b200.formats import packed
    from voom_b200.formats.zstd_gpu import ZstdError

    cfg = dict(synthetic.SMOLLM2_135M, layers=2)
    heads, bodies, raws = [], [], []
    for i, (name, shape) in enumerate(synthetic.smollm2_tensors(cfg)):
        bits = synthetic.bf16_normal(shape, 0.02, 70 + i)
        h, b = packed.body_for("BF16", bits.view(np.uint8))
        heads.append({"dtype": "BF16", "shape": list(shape), **h})
        bodies.append(b)
        raws.append(bits.view(np.uint8).reshape(-1))
        if i == 3:  # a raw-stored (F32) body between the BF16 ones
            f = np.random.default_rng(5).standard_normal(4099).astype(np.float32)
            h, b = packed.body_for("F32", f.view(np.uint8))
            heads.append({"dtype": "F32", "shape": [4099], **h})
            bodies.append(b)
            raws.append(f.view(np.uint8))
    offs = np.cumsum([0] + [len(b) for b in bodies[:-1]]).tolist()
    lens = [len(b) for b in bodies]
    pinned = torch.empty(sum(lens), dtype=torch.uint8, pin_memory=True)
    pinned.numpy()[:] = np.frombuffer(b"".join(bodies), np.uint8)
    ref, spans = packed.decode_bodies(heads, pinned, offs, lens, groups=1)
    for g in (2, 3, 5):
        assert len(packed.body_groups(offs, lens, g)) == g
        out, spans_g = packed.decode_bodies(heads, pinned, offs, lens, groups=g)
        assert spans_g == spans
        for d, n in spans:  # the alignment gaps between bodies are not written
            assert torch.equal(out[d:d + n], ref[d:d + n])
    got = ref.cpu().numpy()
    for (d, n), r in zip(spans, raws):
        assert np.array_equal(got[d:d + n], r)
    last = len(bodies) - 1
    pinned[offs[last]:offs[last] + 4] ^= 0xFF  # the last body's hi-plane frame magic
    with pytest.raises(ZstdError) as one:
        packed.decode_bodies(heads, pinned, offs, lens, groups=1)
    with pytest.raises(ZstdError) as grouped:
        packed.decode_bodies(heads, pinned, offs, lens, groups=3)
    assert str(grouped.value) == str(one.value)


def test_copy_from_host_reads_mapped_pinned_memory(built_lib):
    """voom_copy_from_host: a pinned buffer (aligned and odd offsets and
    lengths) lands byte for byte; pageable memory is refused with
    VOOM_E_INVALID_ARG and nothing is launched."""
    from voom_b200 import _device
    from voom_b200._lib import load

    lib = load()
    rng = np.random.default_rng(11)
    host = torch.empty(300_007, dtype=torch.uint8, pin_memory=True)
    host.numpy()[:] = rng.integers(0, 256, host.numel(), dtype=np.uint8)
    dev = torch.device("cuda", 0)
    s = _device.stream_ptr(dev)
    for off, n in ((0, 300_000), (3, 70_001), (16, 16), (5, 1)):
        out = torch.zeros(n + 32, dtype=torch.uint8, device=dev)
        assert lib.voom_copy_from_host(out.data_ptr() + 7 * (off & 1), host.data_ptr() + off, n, s) == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()[7 * (off & 1):7 * (off & 1) + n]
        assert np.array_equal(got, host.numpy()[off:off + n])
    pageable = np.zeros(4096, np.uint8)
    out = torch.zeros(4096, dtype=torch.uint8, device=dev)
    assert lib.voom_copy_from_host(out.data_ptr(), pageable.ctypes.data, 4096, s) != 0
    assert lib.voom_copy_from_host(out.data_ptr(), host.data_ptr(), 0, s) == 0


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


def test_gpu_repack_bodies_decode_through_reference_path(built_lib):
    """bodies_gpu (hi planes encoded on the GPU): every body decodes through
    the reference's decode_body (restated: libzstd + numpy interleave) and
    through the GPU decoder to the original bytes, for device and host inputs,
    odd and tiny sizes and a raw dtype; BF16 weight bodies stay within 3 % of
    host zstd level 1."""
    from voom_b200 import synthetic
    from voom_b200.formats import packed

    dev = torch.device("cuda", 0)
    specs = [((256, 192), 1), ((1, 2), 2), ((3, 5), 3), ((4096, 576), 4), ((7,), 5)]
    raws = [synthetic.bf16_normal(shape, 0.02, seed).view(np.uint8).reshape(-1) for shape, seed in specs]
    raws.append(np.arange(37, dtype=np.float32).view(np.uint8))
    dtypes = ["BF16"] * len(specs) + ["F32"]
    items = [(dt, torch.from_numpy(r.copy()).to(dev) if i % 2 == 0 else r.tobytes())
             for i, (dt, r) in enumerate(zip(dtypes, raws))]
    bodies = packed.bodies_gpu(items)
    heads = [h for h, _ in bodies]
    for (head, body), raw, dt in zip(bodies, raws, dtypes):
        assert np.array_equal(ov.decode_body(head, body), raw), head
        if dt == "BF16":
            assert head["lo"] == raw.size // 2 and len(body) == head["hi_z"] + head["lo"]
    blob = b"".join(b for _, b in bodies)
    offs = np.cumsum([0] + [len(b) for _, b in bodies[:-1]]).tolist()
    out, spans = packed.decode_bodies(heads, np.frombuffer(blob, np.uint8), offs, [len(b) for _, b in bodies],
                                      device=dev)
    got = out.cpu().numpy()
    for (o, n), raw in zip(spans, raws):
        assert np.array_equal(got[o:o + n], raw)
    big = raws[3]
    ours = len(bodies[3][1])
    ref = len(packed.body_for("BF16", big, 1)[1])
    assert ours <= 1.03 * ref, (ours, ref)


def test_pack_model_gpu_encoder_round_trip(built_lib, tmp_path):
    """pack_model(encoder='gpu') writes the reference layout (fused expert
    split, raw dtypes) whose every tensor the reference's decode path and the
    GPU reader give back exactly."""
    from tests.golden.make_golden import write_safetensors
    from tests.test_vpack_cpu import source_tensors
    from voom_b200.formats import packed

    src = tmp_path / "model"
    src.mkdir()
    tensors = source_tensors()
    write_safetensors(src / "model.safetensors", tensors)
    out = packed.pack_model(src, tmp_path / "gpu.vpack", encoder="gpu", batch_bytes=64 << 10)
    host = packed.pack_model(src, tmp_path / "host.vpack")
    man = json.loads((out / "manifest.json").read_text())
    assert man == json.loads((host / "manifest.json").read_text())
    by_name = {n: raw for n, _, _, raw in tensors}
    for name, fname in man.items():
        data = (out / fname).read_bytes()
        n = int.from_bytes(data[:8], "little")
        head = json.loads(data[8:8 + n])
        raw = ov.decode_body(head, np.frombuffer(data[8 + n:], np.uint8))
        _, t = packed.read_tensor_bytes(out, fname)
        assert np.array_equal(t.cpu().numpy(), raw)
        if name in by_name:
            assert raw.tobytes() == by_name[name]
