"""BF16 NF12 exact sidecar.  CPU: the product encoder and layer builder
against the reference's own outputs (tests/golden/nf12_*, made by
make_nf12_golden.py from the reference codec and sidecar builder) and the
oracle against the same fixtures.  GPU: voom_nf12_decode bit-exact against
the inputs and the oracle (incl. duplicate patches and damaged headers), and
the fused decode + small-M linear against an fp32 matmul of the oracle-decoded
weights (rel-L2 <= 1e-2, the tolerance stated for the floating-point path)."""

from __future__ import annotations

import hashlib
import importlib.util
import json
import struct
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import nf12 as onf
from voom_b200.formats import nf12

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = json.loads((GOLDEN / "nf12_cases.json").read_text())


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def _golden_script():
    spec = importlib.util.spec_from_file_location("make_nf12_golden", GOLDEN / "make_nf12_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _case(name: str) -> tuple[bytes, bytes, dict]:
    raw = (GOLDEN / f"nf12_{name}.bin").read_bytes()
    enc = (GOLDEN / f"nf12_{name}.enc").read_bytes()
    rec = CASES[name]
    assert sha(raw) == rec["input_sha256"]
    return raw, enc, rec


@pytest.mark.parametrize("name", sorted(CASES))
def test_encoder_matches_reference_output(name):
    raw, enc, rec = _case(name)
    for impl in (nf12.pack_tensor, onf.pack_tensor):
        h, c, p, rep = impl(raw)
        assert (sha(h), sha(c), sha(p)) == (rec["headers_sha256"], rec["codes_sha256"], rec["patches_sha256"])
        assert h + c + p == enc
        for k, v in rec["report"].items():
            assert rep[k] == pytest.approx(v) if isinstance(v, float) else rep[k] == v, (impl, k)


@pytest.mark.parametrize("name", [n for n in sorted(CASES) if CASES[n]["report"]["selected"]])
def test_oracle_decode_matches_reference_unpack(name):
    raw, enc, rec = _case(name)
    hb, cb = rec["header_bytes"], rec["code_bytes"]
    blocks = hb // nf12.BLOCK_HEADER_BYTES
    # the standalone streams carry patch offsets relative to the patch stream
    hdr = np.frombuffer(enc[:hb], dtype=nf12.HEADER_DTYPE).copy()
    hdr["patch_offset"] += hb + cb
    stream = hdr.tobytes() + enc[hb:]
    got = onf.decode_span(stream, hb, 0, blocks, 0, rec["values"])
    assert sha(got.tobytes()) == rec["unpack_sha256"] == rec["input_sha256"]


def _layer_inputs():
    g = _golden_script()
    a = g.bf16_normal(64 * 512, 0.02, 11)
    b = g.bf16_normal(2000, 0.1, 12)
    b[[3, 1999]] = np.array([0x4400, 0x0001], dtype=np.uint16)
    return [("model.layers.0.mlp.down_proj.weight", a, (64, 512)),
            ("model.layers.0.post_attention_layernorm.weight", b, (2000,))]


def test_layer_builder_matches_reference_sidecar():
    ref_payload = (GOLDEN / "nf12_layer.bin").read_bytes()
    ref_entry = json.loads((GOLDEN / "nf12_layer.json").read_text())
    tensors = _layer_inputs()
    for name, bits, _ in tensors:
        assert sha(bits.astype("<u2").tobytes()) == ref_entry["inputs"][name]
    payload, entry = nf12.build_layer(tensors)
    assert payload == ref_payload
    opayload, oentry = onf.build_layer(tensors)
    assert opayload == ref_payload
    for k in ("file_bytes", "block_count", "header_bytes", "code_bytes", "patch_stream_bytes", "output_value_count",
              "selected_raw_bytes", "all_bf16_raw_bytes", "saved_bytes"):
        assert entry[k] == ref_entry[k], k
    keys = ("physical_name", "name", "shape", "output_offset", "value_count", "block_start", "block_count",
            "raw_bytes", "encoded_bytes", "mode", "exception_count")
    assert [{k: t[k] for k in keys} for t in entry["tensors"]] == [{k: t[k] for k in keys} for t in ref_entry["tensors"]]
    dec = onf.decode_span(payload, entry["header_bytes"], 0, entry["block_count"], 0, entry["output_value_count"])
    assert np.array_equal(dec, np.concatenate([b for _, b, _ in tensors]))


def test_layer_file_round_trip(tmp_path):
    payload, _ = nf12.build_layer(_layer_inputs())
    p = tmp_path / "layer-000.safetensors"
    p.write_bytes(nf12.safetensors_file(payload))
    assert nf12.read_layer_file(p) == payload
    n = struct.unpack_from("<Q", p.read_bytes())[0]
    assert n % 8 == 0


def test_direct_linear_eligibility():
    ok = {"shape": [1024, 2048], "raw_bytes": 1024 * 2048 * 2}
    assert nf12.direct_linear_eligible(ok) and onf.direct_linear_eligible(ok)
    for bad in ({"shape": [1020, 2048], "raw_bytes": 4 << 20}, {"shape": [1024, 2000], "raw_bytes": 4 << 20},
                {"shape": [8, 512], "raw_bytes": 8192}, {"shape": [4096], "raw_bytes": 8192}):
        assert not nf12.direct_linear_eligible(bad) and not onf.direct_linear_eligible(bad)


def test_empty_and_odd_inputs_rejected():
    with pytest.raises(ValueError, match="empty"):
        nf12.pack_tensor(b"")
    with pytest.raises(ValueError, match="even"):
        nf12.pack_tensor(b"abc")


def _weights(n: int, k: int, seed: int, outliers: int = 50) -> np.ndarray:
    g = _golden_script()
    w = g.bf16_normal(n * k, 0.02, seed)
    idx = np.random.default_rng(seed + 1).choice(w.size, outliers, replace=False)
    w[idx] = g.bf16_normal(outliers, 8.0, seed + 2)
    return w.reshape(n, k)


@pytest.mark.gpu
def test_gpu_decode_layer_and_names_bit_exact():
    payload = (GOLDEN / "nf12_layer.bin").read_bytes()
    entry = json.loads((GOLDEN / "nf12_layer.json").read_text())
    tensors = _layer_inputs()
    dev = torch.device("cuda:0")
    out = nf12.decode_layer(payload, entry, device=dev)
    for name, bits, shape in tensors:
        t = out[name]
        assert t.is_cuda and t.dtype == torch.bfloat16 and tuple(t.shape) == shape
        assert np.array_equal(t.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1), bits)
    enc = torch.from_numpy(np.frombuffer(payload, np.uint8).copy()).to(dev)
    part = nf12.decode_names(enc, entry, ["model.layers.0.post_attention_layernorm.weight"])
    assert np.array_equal(part["model.layers.0.post_attention_layernorm.weight"].view(torch.int16).cpu().numpy()
                          .view(np.uint16), tensors[1][1])
    with pytest.raises(KeyError):
        nf12.decode_names(enc, entry, ["nope"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", [n for n in sorted(CASES) if CASES[n]["report"]["selected"]])
def test_gpu_decode_golden_cases(name):
    raw, _, rec = _case(name)
    bits = np.frombuffer(raw, np.uint16)
    payload, entry = nf12.build_layer([("t", bits, (bits.size,))])
    got = nf12.decode_layer(payload, entry, device="cuda:0")["t"]
    assert sha(got.view(torch.int16).cpu().numpy().tobytes()) == rec["input_sha256"]


@pytest.mark.gpu
def test_gpu_decode_duplicate_patches_first_wins_and_damaged_header():
    bits = _weights(64, 512, 31, outliers=40).reshape(-1)
    payload, entry = nf12.build_layer([("w", bits, (64, 512))])
    hb, cb = entry["header_bytes"], entry["code_bytes"]
    hdr = np.frombuffer(payload[:hb], dtype=nf12.HEADER_DTYPE).copy()
    blk = int(np.flatnonzero(hdr["count"] >= 2)[0])
    p0 = int(hdr["patch_offset"][blk])
    pat = bytearray(payload[hb + cb:])
    rel = p0 - hb - cb
    pat[rel + 3] = pat[rel]  # second patch now names the first one's index
    dup = payload[:hb + cb] + bytes(pat)
    want = onf.decode_span(dup, hb, 0, entry["block_count"], 0, entry["output_value_count"])
    got = nf12.decode_layer(dup, entry, device="cuda:0")["w"]
    assert np.array_equal(got.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1), want)
    bad = hdr.copy()
    bad["patch_offset"][blk] = len(payload) + 1000
    broken = bad.tobytes() + payload[hb:]
    with pytest.raises(nf12.NF12Error):
        nf12.decode_layer(broken, entry, device="cuda:0")


def _rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(1, 1024, 2048), (2, 1024, 2048), (3, 512, 1024), (5, 256, 4096),
                                   (8, 2048, 1536), (8, 64, 4096)])
def test_gpu_fused_linear_matches_fp32_matmul(m, n, k):
    dev = torch.device("cuda:0")
    w = _weights(n, k, 100 + m)
    payload, entry = nf12.build_layer([("w", w.reshape(-1), (n, k))])
    spec = entry["tensors"][0]
    assert nf12.direct_linear_eligible(spec) or n * k * 2 < 1_000_000
    x = torch.randn((m, k), generator=torch.Generator().manual_seed(m)).to(torch.bfloat16)
    wdec = onf.decode_span(payload, entry["header_bytes"], 0, entry["block_count"], 0, entry["output_value_count"])
    assert np.array_equal(wdec, w.reshape(-1))
    ref = x.float() @ torch.from_numpy(onf.bf16_bits_to_f32(wdec).reshape(n, k)).T  # fp32 reference
    enc = torch.from_numpy(np.frombuffer(payload, np.uint8).copy()).to(dev)
    got = nf12.linear(x.to(dev), enc, entry, spec)
    assert got.dtype == torch.bfloat16 and tuple(got.shape) == (m, n)
    assert _rel_l2(got.cpu(), ref) <= 1e-2
    # deterministic: the K split reduces in a fixed order
    again = nf12.linear(x.to(dev), enc, entry, spec)
    assert torch.equal(got, again)


@pytest.mark.gpu
def test_gpu_nf12_tensor_matmul_paths():
    dev = torch.device("cuda:0")
    n, k = 1024, 1024
    w = _weights(n, k, 7)
    payload, entry = nf12.build_layer([("w", w.reshape(-1), (n, k))])
    t = nf12.NF12Tensor(payload, entry, entry["tensors"][0], device=dev)
    assert t.shape == (n, k) and t.nbytes < n * k * 2
    dense = t.materialize()
    assert np.array_equal(dense.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1), w.reshape(-1))
    for lead in ((1,), (2, 3), (12,)):  # 1 and 6 rows fused, 12 rows through the decoded weight
        x = torch.randn(*lead, k, generator=torch.Generator().manual_seed(len(lead))).to(torch.bfloat16).to(dev)
        got = t.matmul(x)
        ref = x.float() @ dense.float().T
        assert tuple(got.shape) == (*lead, n)
        assert _rel_l2(got, ref) <= 1e-2


@pytest.mark.gpu
def test_gpu_batched_linear_equals_single_calls():
    """One launch over a layer's projections (different K and N) gives the
    same bits as one call per projection."""
    dev = torch.device("cuda:0")
    shapes = [("q", 512, 1024), ("k", 128, 1024), ("gate", 1536, 1024), ("down", 1024, 1536)]
    tensors = [(n, _weights(r, c, 200 + i).reshape(-1), (r, c)) for i, (n, r, c) in enumerate(shapes)]
    payload, entry = nf12.build_layer(tensors)
    enc = torch.from_numpy(np.frombuffer(payload, np.uint8).copy()).to(dev)
    for m in (1, 4, 8):
        g = torch.Generator().manual_seed(m)
        xs = {1024: torch.randn((m, 1024), generator=g).to(torch.bfloat16).to(dev),
              1536: torch.randn((m, 1536), generator=g).to(torch.bfloat16).to(dev)}
        items = [(xs[sp["shape"][1]], sp) for sp in entry["tensors"]]
        got = nf12.linear_batch(items, enc, entry)
        for (x, sp), o in zip(items, got):
            assert torch.equal(o, nf12.linear(x, enc, entry, sp))
            w = torch.from_numpy(onf.bf16_bits_to_f32(dict((n, b) for n, b, _ in tensors)[sp["name"]])
                                 .reshape(sp["shape"]))
            assert _rel_l2(o.cpu(), x.float().cpu() @ w.T) <= 1e-2
