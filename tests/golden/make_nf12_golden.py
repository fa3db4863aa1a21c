"""Generates the NF12 golden fixtures under tests/golden/ by running the
REFERENCE codec and sidecar builder (vOOM's formats/bf16_nf12_sidecar.py,
imported from a checkout of the reference) on seeded inputs:

    VOOM_REFERENCE=/path/to/vOOM python tests/golden/make_nf12_golden.py

Outputs (committed): nf12_cases.json (per case: input SHA-256, the
reference's report, SHA-256 of its headers / codes / patches and of its
unpack_tensor output) with nf12_<case>.bin (the input bits) and
nf12_<case>.enc (headers + codes + patches as the reference returned them),
and nf12_layer.bin / nf12_layer.json: the payload and manifest entry of one
layer built by the reference's build_nf12_sidecar.
"""

from __future__ import annotations

import hashlib
import json
import os
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _reference():
    p = os.environ.get("VOOM_REFERENCE")
    if not p or not (Path(p) / "formats" / "bf16_nf12_sidecar.py").exists():
        raise SystemExit("set VOOM_REFERENCE to a checkout of the reference")
    sys.path.insert(0, p)
    import formats.bf16_nf12_sidecar as ref
    return ref


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def bf16_normal(n: int, std: float, seed: int) -> np.ndarray:
    x = np.random.default_rng(seed).standard_normal(n).astype(np.float32) * std
    return ((x.view(np.uint32) + 0x7FFF + ((x.view(np.uint32) >> 16) & 1)) >> 16).astype(np.uint16)


def cases() -> dict[str, np.ndarray]:
    rng = np.random.default_rng(140)
    mixed = rng.integers(0, 1 << 11, size=700, dtype=np.uint16) | np.uint16(7 << 11)
    mixed[[0, 255, 256, 699]] = np.array([0x0000, 0x2F80, 0x8001, 0xFFFF], dtype=np.uint16)
    w = bf16_normal(128 * 1024, 0.02, 7)
    outl = np.random.default_rng(8).choice(w.size, 300, replace=False)
    w[outl] = bf16_normal(300, 4.0, 9)  # values whose high exponent nibble is not modal
    tiny = bf16_normal(40 * 256 + 17, 0.05, 10)
    rng2 = np.random.default_rng(141)
    expand = (np.arange(16, dtype=np.uint16).repeat(64) << 11) | rng2.integers(0, 1 << 11, 1024, dtype=np.uint16)
    return {"mixed_700": mixed, "weights_128x1024": w, "tail_10257": tiny, "expands_1024": expand}


def write_safetensors(path: Path, tensors: dict[str, tuple[np.ndarray, tuple]]) -> None:
    header, body = {}, bytearray()
    for name, (bits, shape) in tensors.items():
        raw = np.ascontiguousarray(bits, dtype="<u2").tobytes()
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [len(body), len(body) + len(raw)]}
        body.extend(raw)
    h = json.dumps(header, separators=(",", ":"), sort_keys=True).encode()
    h += b" " * ((-len(h)) % 8)
    path.write_bytes(struct.pack("<Q", len(h)) + h + body)


def main() -> None:
    ref = _reference()
    out = {}
    for name, bits in cases().items():
        raw = bits.astype("<u2").tobytes()
        h, c, p, rep = ref.pack_tensor(raw)
        rec = {"values": int(bits.size), "input_sha256": sha(raw), "report": rep,
               "headers_sha256": sha(h), "codes_sha256": sha(c), "patches_sha256": sha(p),
               "header_bytes": len(h), "code_bytes": len(c), "patch_bytes": len(p)}
        if rep["selected"]:
            rec["unpack_sha256"] = sha(ref.unpack_tensor(h, c, p, value_count=bits.size))
        (HERE / f"nf12_{name}.bin").write_bytes(raw)
        (HERE / f"nf12_{name}.enc").write_bytes(h + c + p)
        out[name] = rec
    (HERE / "nf12_cases.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")

    # one layer through the reference's sidecar builder
    with tempfile.TemporaryDirectory() as tmp:
        model = Path(tmp) / "model"
        side = Path(tmp) / "side"
        model.mkdir()
        a = bf16_normal(64 * 512, 0.02, 11)
        b = bf16_normal(2000, 0.1, 12)
        b[[3, 1999]] = np.array([0x4400, 0x0001], dtype=np.uint16)
        write_safetensors(model / "model.safetensors", {
            "model.layers.0.mlp.down_proj.weight": (a, (64, 512)),
            "model.layers.0.post_attention_layernorm.weight": (b, (2000,)),
        })
        (model / "config.json").write_text(json.dumps({
            "model_type": "llama", "hidden_size": 512, "num_hidden_layers": 1, "num_attention_heads": 1,
            "num_key_value_heads": 1, "vocab_size": 32, "rms_norm_eps": 1e-6,
            "max_position_embeddings": 128, "torch_dtype": "bfloat16"}))
        rep = ref.build_nf12_sidecar(model, side, layers=[0], enforce_external=False, min_free_after_bytes=0)
        gen = side / rep["generation"]
        manifest = json.loads((gen / "manifest.json").read_text())
        entry = manifest["layers"]["0"]
        data = (gen / entry["file"]).read_bytes()
        payload = data[len(data) - entry["file_bytes"]:]
        entry = {k: v for k, v in entry.items() if k not in ("file_sha256",)}
        entry["inputs"] = {"model.layers.0.mlp.down_proj.weight": sha(a.astype("<u2").tobytes()),
                           "model.layers.0.post_attention_layernorm.weight": sha(b.astype("<u2").tobytes())}
        (HERE / "nf12_layer.bin").write_bytes(payload)
        (HERE / "nf12_layer.json").write_text(json.dumps(entry, indent=1, sort_keys=True) + "\n")
    print("wrote", sorted(out), "and one layer")


if __name__ == "__main__":
    main()
