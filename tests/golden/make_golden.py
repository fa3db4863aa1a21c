"""Generates the golden fixtures under tests/golden/ by running the REFERENCE
implementation (vOOM's own Python modules, imported from a checkout of the
reference) on seeded inputs.  Run it only where the reference is available:

    VOOM_REFERENCE=/path/to/vOOM python tests/golden/make_golden.py

Outputs (committed): rans_cases.json + rans_*.bin frames produced by the
reference formats/bf16_rans.py encode(), with the SHA-256 of every input and
of the reference decode() output, and rans_mutations.json: the reference
decode() outcome (bytes hash or ValueError message) for corrupted frames.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from voom_b200 import synthetic  # noqa: E402


def _reference_path() -> Path:
    """The reference checkout named by $VOOM_REFERENCE."""
    env = os.environ.get("VOOM_REFERENCE")
    if not env:
        raise SystemExit("set VOOM_REFERENCE to a checkout of the reference (KyleBoyer/vOOM)")
    p = Path(env)
    if not (p / "formats" / "bf16_rans.py").exists():
        raise SystemExit(f"reference checkout not found at {p}")
    return p


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


# ---------------------------------------------------------------- inputs
def rans_inputs() -> list[dict]:
    """Each case regenerates deterministically from (kind, params)."""
    cases = []
    for size in (0, 1, 2, 3, 257, 8193):
        cases.append(dict(name=f"random_{size}", kind="random", size=size, seed=100 + size, tile_bytes=257))
    cases.append(dict(name="structured_planes", kind="structured", pairs=32768, tile_bytes=16384))
    cases.append(dict(name="range_x20", kind="range20", tile_bytes=1024))
    cases.append(dict(name="structured_single_tile", kind="structured", pairs=8192, tile_bytes=16384))
    cases.append(dict(name="bf16_normal_256x256", kind="bf16_normal", shape=[256, 256], std=0.02, seed=7,
                      tile_bytes=16384))
    cases.append(dict(name="bf16_outlier_256x512", kind="outlier", rows=256, cols=512, seed=11,
                      tile_bytes=32768))
    cases.append(dict(name="zeros_100000", kind="zeros", size=100000, tile_bytes=32768))
    cases.append(dict(name="bf16_odd_tiles", kind="bf16_normal", shape=[5000], std=0.02, seed=13,
                      tile_bytes=1001))
    return cases


def make_input(case: dict) -> bytes:
    k = case["kind"]
    if k == "random":
        rng = np.random.default_rng(case["seed"])
        return rng.integers(0, 256, size=case["size"], dtype=np.uint8).tobytes()
    if k == "structured":
        return b"".join(bytes((i & 0xFF, 0x3F)) for i in range(case["pairs"]))
    if k == "range20":
        return bytes(range(256)) * 20
    if k == "bf16_normal":
        return synthetic.bf16_normal(tuple(case["shape"]), case["std"], case["seed"]).tobytes()
    if k == "outlier":
        return synthetic.outlier_matrix(case["rows"], case["cols"], seed=case["seed"]).tobytes()
    if k == "zeros":
        return bytes(case["size"])
    raise ValueError(k)


def mutations(frame: bytes, seed: int, count: int) -> list[dict]:
    """Header-biased corruptions: single-byte xor, truncation, appended bytes."""
    rng = np.random.default_rng(seed)
    out = []
    n = len(frame)
    for i in range(count):
        r = rng.random()
        if r < 0.55:
            # bias towards the first 1.2 KB (frame/tile/plane headers and tables)
            pos = int(rng.integers(0, min(n, 1200))) if rng.random() < 0.7 else int(rng.integers(0, n))
            out.append(dict(op="xor", pos=pos, val=int(rng.integers(1, 256))))
        elif r < 0.85:
            out.append(dict(op="truncate", pos=int(rng.integers(0, n))))
        else:
            out.append(dict(op="append", val=int(rng.integers(0, 256)), count=int(rng.integers(1, 5))))
    return out


def apply_mutation(frame: bytes, m: dict) -> bytes:
    if m["op"] == "xor":
        b = bytearray(frame)
        b[m["pos"]] ^= m["val"]
        return bytes(b)
    if m["op"] == "truncate":
        return frame[: m["pos"]]
    if m["op"] == "append":
        return frame + bytes([m["val"]]) * m["count"]
    raise ValueError(m["op"])


TINY = dict(layers=2, hidden=64, intermediate=128, heads=4, kv_heads=2, head_dim=16, vocab=256)


def write_safetensors(path: Path, tensors: list[tuple[str, str, list[int], bytes]]) -> None:
    header, off = {}, 0
    for name, dtype, shape, raw in tensors:
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + len(raw)]}
        off += len(raw)
    hj = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(len(hj).to_bytes(8, "little") + hj)
        for _, _, _, raw in tensors:
            f.write(raw)


def vpack_fixture(ref: Path) -> None:
    """A tiny SmolLM2-shaped checkpoint (plus one fused BF16 expert tensor and
    one F32 tensor) packed by the reference's pack_model + build_from_vpack."""
    import shutil
    import tempfile

    sys.path.insert(0, str(HERE / "_shim"))
    from formats import packed, packed2  # the reference modules, unmodified

    tensors = []
    for i, (name, shape) in enumerate(synthetic.smollm2_tensors(TINY)):
        tensors.append((name, "BF16", list(shape), synthetic.bf16_normal(shape, 0.02, 500 + i).tobytes()))
    tensors.append(("model.layers.1.mlp.experts.gate_up_proj", "BF16", [4, 32, 64],
                    synthetic.bf16_normal((4, 32, 64), 0.02, 99).tobytes()))
    tensors.append(("model.layers.1.mlp.router.scale", "F32", [8],
                    np.arange(8, dtype=np.float32).tobytes()))
    tmp = Path(tempfile.mkdtemp())
    try:
        write_safetensors(tmp / "model.safetensors", tensors)
        packed.pack_model(tmp, level=1)
        packed2.build_from_vpack(tmp)
        archive = (tmp / "weights.vpack2").read_bytes()
        index = json.loads((tmp / "weights.vpack2.index.json").read_text())
        decoded = {}
        for name, e in index.items():
            raw = packed2.decode_body(e["head"], archive[e["off"]:e["off"] + e["len"]])
            decoded[name] = sha(raw.tobytes() if isinstance(raw, np.ndarray) else bytes(raw))
        (HERE / "vpack2_tiny.bin").write_bytes(archive)
        (HERE / "vpack2_tiny.index.json").write_text(json.dumps(index, indent=0))
        (HERE / "vpack2_tiny.decoded.json").write_text(json.dumps(
            {"decoded_sha256": decoded, "source": [(n, d, s) for n, d, s, _ in tensors],
             "source_sha256": {n: sha(r) for n, _, _, r in tensors}}, indent=0))
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    print(f"vpack2 fixture: {len(index)} bodies, {len(archive)} bytes")


def main() -> None:
    ref = _reference_path()
    sys.path.insert(0, str(ref))
    from formats import bf16_rans as R  # the reference module, unmodified

    vpack_fixture(ref)

    manifest = []
    frames = {}
    for case in rans_inputs():
        raw = make_input(case)
        frame, stats = R.encode(raw, tile_bytes=case["tile_bytes"])
        decoded = R.decode(frame)
        assert decoded == raw
        fname = f"rans_{case['name']}.bin"
        (HERE / fname).write_bytes(frame)
        frames[case["name"]] = frame
        manifest.append(dict(case, frame=fname, input_sha256=sha(raw), frame_sha256=sha(frame),
                             decoded_sha256=sha(decoded), raw_bytes=stats.raw_bytes,
                             encoded_bytes=stats.encoded_bytes, tiles=stats.tiles,
                             compressed_tiles=stats.compressed_tiles))
    (HERE / "rans_cases.json").write_text(json.dumps(manifest, indent=1))

    muts = []
    # targeted: unknown tile mode, raw-size mismatch (stored tile), a compressed
    # tile whose payload length covers one extra byte, and plane-header damage
    targeted = [
        ("structured_single_tile", dict(op="xor", pos=16, val=2)),
        ("structured_single_tile", dict(op="xor", pos=16, val=0x80)),
        ("random_8193", dict(op="xor", pos=17, val=1)),
        ("random_257", dict(op="xor", pos=21, val=4)),
        ("structured_single_tile", dict(op="xor", pos=21, val=1)),
        ("structured_single_tile", dict(op="xor", pos=29, val=0xFF)),
        ("structured_single_tile", dict(op="xor", pos=31, val=0x10)),
        ("bf16_normal_256x256", dict(op="xor", pos=16 + 13 + 4 + 2 * 0x3C, val=1)),
    ]
    for base, m in targeted:
        bad = apply_mutation(frames[base], m)
        try:
            outcome = "ok:" + sha(R.decode(bad))
        except ValueError as exc:
            outcome = "error:" + str(exc)
        muts.append(dict(base=base, mutation=m, outcome=outcome))
    for base, seed, count in (("structured_single_tile", 1, 160), ("bf16_normal_256x256", 2, 160),
                              ("random_8193", 3, 60), ("zeros_100000", 4, 60)):
        for m in mutations(frames[base], seed, count):
            bad = apply_mutation(frames[base], m)
            try:
                outcome = "ok:" + sha(R.decode(bad))
            except ValueError as exc:
                outcome = "error:" + str(exc)
            muts.append(dict(base=base, mutation=m, outcome=outcome))
    (HERE / "rans_mutations.json").write_text(json.dumps(muts, indent=0))
    kinds = {}
    for m in muts:
        kinds[m["outcome"].split(":")[0] + ":" + (m["outcome"][6:] if m["outcome"].startswith("error") else "")] = 1
    print(f"{len(manifest)} rANS cases, {len(muts)} mutations; outcomes: {sorted(kinds)}")


if __name__ == "__main__":
    main()
