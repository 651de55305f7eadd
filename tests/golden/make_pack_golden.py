"""Golden output of the reference's own packer for the packer parity test.

    python tests/golden/make_pack_golden.py      (needs the reference tree)

Builds a small seeded synthetic BERT checkpoint directory (config.json,
CHECKPOINT.json, 1_Pooling/config.json, vocab.txt, model.safetensors) and
packs it with the reference's packer, tools/pack/pack_npue.py main(), as
`--dtype f32 --max-seq 128` (its host-layout container).  The reference packer
reads an ONNX export; there is none for a synthetic checkpoint, so its two
ONNX-reading calls are replaced for the run: `load` returns the checkpoint's
tensors (the same arrays written to model.safetensors) and `model_digest`
returns the SHA-256 of model.safetensors.  Everything after that -- QKV
fusion, transposes, the Q-scale fold, the position slice, names, roles,
config keys and the container writer -- is the reference's own code.

The fixture pack_tiny_bert.json records the container's config and, per
tensor, dtype, role, shape and the SHA-256 of its bytes.
tests/test_pack.py packs the same checkpoint with nebw.pack and compares.
"""

from __future__ import annotations

import hashlib
import os
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "npu-embeddings-xdna1_b200"))

GEOMETRY = dict(layers=2, hidden=128, heads=4, ffn=512, vocab=1000, type_vocab=2, max_pos=512)
MAX_SEQ = 128
SEED = 20261202


def write_safetensors(path, tensors: dict):
    """The safetensors format, written directly: an 8-byte little-endian
    header length, a JSON header {name: {dtype, shape, data_offsets}}, then
    the raw little-endian bytes in header order."""
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        b = np.ascontiguousarray(a, "<f4").tobytes()
        header[name] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hj += b" " * ((-len(hj)) % 8)
    with open(path, "wb") as f:
        f.write(len(hj).to_bytes(8, "little"))
        f.write(hj)
        for b in blobs:
            f.write(b)


def synthetic_checkpoint(d: Path) -> dict:
    """A seeded BertModel-style checkpoint directory at d; returns its tensors."""
    g = GEOMETRY
    rng = np.random.default_rng(SEED)
    H, F = g["hidden"], g["ffn"]

    def n(*s):
        return (rng.standard_normal(s) * 0.02).astype(np.float32)

    src = {"embeddings.word_embeddings.weight": n(g["vocab"], H),
           "embeddings.position_embeddings.weight": n(g["max_pos"], H),
           "embeddings.token_type_embeddings.weight": n(g["type_vocab"], H),
           "embeddings.LayerNorm.weight": (1 + n(H)).astype(np.float32),
           "embeddings.LayerNorm.bias": n(H)}
    for i in range(g["layers"]):
        p = f"encoder.layer.{i}."
        for q in ("query", "key", "value"):
            src[p + f"attention.self.{q}.weight"] = n(H, H)
            src[p + f"attention.self.{q}.bias"] = n(H)
        src[p + "attention.output.dense.weight"] = n(H, H)
        src[p + "attention.output.dense.bias"] = n(H)
        src[p + "attention.output.LayerNorm.weight"] = (1 + n(H)).astype(np.float32)
        src[p + "attention.output.LayerNorm.bias"] = n(H)
        src[p + "intermediate.dense.weight"] = n(F, H)
        src[p + "intermediate.dense.bias"] = n(F)
        src[p + "output.dense.weight"] = n(H, F)
        src[p + "output.dense.bias"] = n(H)
        src[p + "output.LayerNorm.weight"] = (1 + n(H)).astype(np.float32)
        src[p + "output.LayerNorm.bias"] = n(H)
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps({
        "model_type": "bert", "num_hidden_layers": g["layers"], "num_attention_heads": g["heads"],
        "hidden_size": H, "intermediate_size": F, "layer_norm_eps": 1e-12,
        "vocab_size": g["vocab"], "type_vocab_size": g["type_vocab"],
        "max_position_embeddings": g["max_pos"], "hidden_act": "gelu"}))
    (d / "CHECKPOINT.json").write_text(json.dumps({"repo_id": "synthetic/tiny-bert"}))
    (d / "1_Pooling").mkdir(exist_ok=True)
    (d / "1_Pooling" / "config.json").write_text(json.dumps(
        {"pooling_mode_cls_token": True, "pooling_mode_mean_tokens": False}))
    (d / "vocab.txt").write_text("\n".join(["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"] +
                                           [f"tok{i}" for i in range(g["vocab"] - 5)]) + "\n")
    write_safetensors(d / "model.safetensors", src)
    return src


def describe(path) -> dict:
    """Config and per-tensor {dtype, role, shape, sha256} of a container."""
    from nebw.npue import ContainerReader
    with ContainerReader(path) as r:
        tensors = {}
        for name, e in r.entries.items():
            tensors[name] = {"dtype": e["dtype"], "role": e["role"], "shape": e["logical_shape"],
                             "sha256": hashlib.sha256(r.tensor(name).tobytes()).hexdigest()}
        return {"config": r.config, "tensors": tensors, "order": list(r.entries)}


# the reference tree: $NEBW_REFERENCE, else a checkout beside this repository
REFERENCE = Path(os.environ.get("NEBW_REFERENCE", str(REPO.parent / "reference")))


def reference_pack(workdir, dtype: str, extra=()) -> Path:
    """Pack synthetic_checkpoint() into workdir with the reference's own
    packer (tools/pack/pack_npue.py main()) at --dtype `dtype`.  Its ONNX
    reads -- the packer's `load` and, for int8, the calibration oracle's
    (reference/encoder.py, reference/onnx_io.py) -- are replaced by the
    checkpoint's own tensors, and `model_digest` by the SHA-256 of
    model.safetensors.  Returns the container's path."""
    for sub in ("tools/pack", "tools/lib", "reference"):
        if str(REFERENCE / sub) not in sys.path:
            sys.path.insert(0, str(REFERENCE / sub))
    import pack_npue as P  # the reference's packer
    d = Path(workdir) / "tiny-bert"
    src = synthetic_checkpoint(d)
    digest = hashlib.sha256((d / "model.safetensors").read_bytes()).hexdigest()
    fake = lambda path, **kw: (src, {})  # noqa: E731
    P.load = fake
    P.model_digest = lambda path: digest
    if dtype == "i8":
        import encoder
        import onnx_io
        onnx_io.load = fake
        encoder.load = fake
    out = Path(workdir) / f"ref_{dtype}.npue"
    argv = sys.argv
    sys.argv = ["pack_npue.py", "--model-dir", str(d), "--out", str(out), "--dtype", dtype,
                "--max-seq", str(MAX_SEQ), *extra]
    try:
        P.main()
    finally:
        sys.argv = argv
    return out


def main():
    with tempfile.TemporaryDirectory() as td:
        out = reference_pack(td, "f32")
        desc = describe(out)
    desc["provenance"] = ("reference tools/pack/pack_npue.py main(), --dtype f32 --max-seq "
                          f"{MAX_SEQ}, on synthetic_checkpoint(seed {SEED}); its ONNX reads "
                          "(load, model_digest) replaced by the checkpoint's own tensors and "
                          "the SHA-256 of model.safetensors")
    (HERE / "pack_tiny_bert.json").write_text(json.dumps(desc, indent=1, sort_keys=True) + "\n")
    print(f"pack_tiny_bert.json: {len(desc['tensors'])} tensors")


if __name__ == "__main__":
    main()
