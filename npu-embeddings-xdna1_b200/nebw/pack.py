"""The weight packer: a Hugging Face BERT checkpoint -> a `.npue` container.

    python -m nebw.pack CHECKPOINT_DIR --out model.npue [--layout tma_bf16|host]
                        [--max-seq 256] [--no-fold-scale]

Replaces the BERT branch of the reference's packer (tools/pack/pack_npue.py:
2620-2835), whose array layout is AIE block panels; this one writes either

  host       GEMM operands row-major F32 [K, N] (`gemm_b_host`), exactly the
             reference packer's `--dtype f32` container (and readable by the
             reference's own host path), or
  tma_bf16   GEMM operands bf16 (round-to-nearest-even) row-major [N, K] --
             K-major, the layout the B200 library's GEMM reads with 128-byte
             swizzled TMA boxes of 64 K-elements, so loading is one upload per
             operand with no re-tiling on the device.

The transformation is the reference packer's (pack_npue.py:2703-2790): Q, K
and V fused along N, every nn.Linear weight transposed from [out, in] to
[K = in, N = out], 1/sqrt(head_dim) folded into the Q columns and the Q bias
(unless --no-fold-scale), the position table sliced to max_seq_len, biases
and LayerNorm parameters F32, config keys and tensor names as that packer
writes them, plus the tokenizer vocabulary when vocab.txt is present.

Input: a checkpoint directory holding config.json, 1_Pooling/config.json (the
pooling mode, read as pack_npue.py:131-154 reads it), optionally
CHECKPOINT.json (repo_id) and vocab.txt, and the weights as model.safetensors
(or pytorch_model.safetensors).  The reference packer reads an ONNX export of
the same checkpoint instead; its `--dtype f32` output loads into this library
unchanged.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import sys
from pathlib import Path

import numpy as np

from .npue import ContainerWriter, tma_b_layout

SAFETENSORS_DTYPES = {"F32": np.dtype("<f4"), "F16": np.dtype("<f2"), "BF16": np.dtype("<u2"),
                      "F64": np.dtype("<f8")}


def read_safetensors(path) -> dict:
    """{name: float32 array} from a .safetensors file (8-byte header length,
    JSON header of {name: {dtype, shape, data_offsets}}, raw little-endian
    data).  BF16 and F16 are widened exactly."""
    raw = Path(path).read_bytes()
    n = int.from_bytes(raw[:8], "little")
    header = json.loads(raw[8:8 + n].decode("utf-8"))
    base = 8 + n
    out = {}
    for name, e in header.items():
        if name == "__metadata__":
            continue
        dt = e["dtype"]
        if dt not in SAFETENSORS_DTYPES:
            raise ValueError(f"{path}: tensor {name} has dtype {dt}; F32, F16, BF16 or F64 expected")
        b0, b1 = e["data_offsets"]
        a = np.frombuffer(raw, dtype=SAFETENSORS_DTYPES[dt], count=(b1 - b0) //
                          SAFETENSORS_DTYPES[dt].itemsize, offset=base + b0)
        if dt == "BF16":
            a = (a.astype(np.uint32) << 16).view(np.float32)
        out[name] = np.asarray(a, np.float32).reshape(e["shape"])
    return out


def strip_prefix(src: dict) -> dict:
    """BertModel checkpoints name tensors embeddings.* / encoder.*; a
    BertFor* or sentence-transformers export may prefix them with `bert.` or
    `0.auto_model.`.  Take them off."""
    for p in ("0.auto_model.", "bert.", "model."):
        if any(k.startswith(p + "embeddings.") for k in src):
            return {k[len(p):]: v for k, v in src.items() if k.startswith(p)}
    return src


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round-to-nearest-even (the reference's
    app::to_bf16, runtime/include/common/host_kernels.hpp:157-161)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def read_pooling(model_dir: Path) -> str:
    p = model_dir / "1_Pooling" / "config.json"
    if not p.exists():
        raise SystemExit(f"{p} not found -- cannot determine the pooling mode")
    c = json.loads(p.read_text(encoding="utf-8"))
    modes = [k for k, v in c.items() if k.startswith("pooling_mode_") and v is True]
    if modes == ["pooling_mode_cls_token"]:
        return "cls"
    if modes == ["pooling_mode_mean_tokens"]:
        return "mean"
    raise SystemExit(f"{p}: cls and mean pooling are implemented; the checkpoint asks for "
                     f"{modes or 'nothing'}")


def find_weights(model_dir: Path) -> Path:
    for name in ("model.safetensors", "pytorch_model.safetensors"):
        if (model_dir / name).exists():
            return model_dir / name
    raise SystemExit(f"no model.safetensors in {model_dir}")


def pack_bert(model_dir, out, layout: str = "tma_bf16", max_seq: int | None = None,
              fold_scale: bool = True, src: dict | None = None, source_sha256: str | None = None):
    """Pack a BERT checkpoint directory (or an already-loaded state dict
    `src` with the checkpoint's own tensor names) into `out`."""
    if layout not in ("tma_bf16", "host"):
        raise SystemExit(f"layout {layout!r}: tma_bf16 or host")
    model_dir = Path(model_dir)
    cfg = json.loads((model_dir / "config.json").read_text(encoding="utf-8"))
    if cfg.get("model_type", "bert") != "bert":
        raise SystemExit(f"model_type {cfg.get('model_type')!r}: this packer handles BERT "
                         "encoders (arch bert_abs_gelu_postln)")
    if src is None:
        wpath = find_weights(model_dir)
        src = read_safetensors(wpath)
        source_sha256 = hashlib.sha256(wpath.read_bytes()).hexdigest()
    src = strip_prefix(src)
    L = cfg["num_hidden_layers"]
    heads = cfg["num_attention_heads"]
    hidden = cfg["hidden_size"]
    head_dim = hidden // heads
    scale = 1.0 / math.sqrt(head_dim)
    max_seq = 256 if max_seq is None else int(max_seq)
    repo_id = "unknown"
    if (model_dir / "CHECKPOINT.json").exists():
        repo_id = json.loads((model_dir / "CHECKPOINT.json").read_text(encoding="utf-8"))["repo_id"]
    host = layout == "host"
    config = {
        "arch": "bert_abs_gelu_postln",
        "source_repo": repo_id,
        "source_sha256": source_sha256 or "unknown",
        "num_layers": L, "num_heads": heads, "hidden": hidden, "head_dim": head_dim,
        "intermediate": cfg["intermediate_size"],
        "layer_norm_eps": cfg["layer_norm_eps"],
        "vocab_size": cfg["vocab_size"],
        "max_seq_len": max_seq,
        "pooling": read_pooling(model_dir), "l2_normalize": True,
        "activation": "gelu_erf_exact",
        "gemm_layout": "host" if host else "tma_bf16",
        "a_dtype": "f32" if host else "bf16",
        "fusions": {
            "qkv_fused": True,
            "transposed_to_kn": True,
            "qk_scale_folded_into_q": fold_scale,
            "gemm_operands_bf16": not host,
            "biases_and_layernorm_fp32": True,
            "position_embeddings_presliced_to": max_seq,
        },
        "not_implemented": ["pooler.dense (unused by sentence-transformers)"],
    }
    if not host:
        config["tma"] = {"operand_order": "NK", "k_box": 64, "swizzle_bytes": 128}
    w = ContainerWriter(config)

    def gemm(name, kn):
        kn = np.ascontiguousarray(kn, np.float32)
        K, N = kn.shape
        if host:
            w.add(name, kn.reshape(-1), "F32", "gemm_b_host", [K, N])
        else:
            w.add(name, to_bf16_bits(kn.T).reshape(-1), "BF16", "gemm_b_tma", [N, K],
                  layout=tma_b_layout())

    w.add("embeddings.word", src["embeddings.word_embeddings.weight"], "F32", "embedding",
          [cfg["vocab_size"], hidden])
    w.add("embeddings.position", src["embeddings.position_embeddings.weight"][:max_seq], "F32",
          "embedding", [max_seq, hidden])
    w.add("embeddings.token_type", src["embeddings.token_type_embeddings.weight"], "F32",
          "embedding", [cfg["type_vocab_size"], hidden])
    w.add("embeddings.ln.weight", src["embeddings.LayerNorm.weight"], "F32", "layernorm",
          [hidden])
    vocab = model_dir / "vocab.txt"
    if vocab.exists():
        vb = np.frombuffer(vocab.read_bytes(), dtype=np.uint8)
        w.add("tokenizer.vocab", vb, "U8", "tokenizer", [int(vb.size)])
    w.add("embeddings.ln.bias", src["embeddings.LayerNorm.bias"], "F32", "layernorm", [hidden])
    for i in range(L):
        p = f"encoder.layer.{i}."
        sa = p + "attention.self."
        qkv = np.concatenate([src[sa + n + ".weight"] for n in ("query", "key", "value")], axis=0)
        qkv_b = np.concatenate([src[sa + n + ".bias"] for n in ("query", "key", "value")], axis=0)
        qkv = np.ascontiguousarray(qkv.T)
        if fold_scale:
            qkv = qkv.copy()
            qkv[:, :hidden] *= scale
            qkv_b = qkv_b.copy()
            qkv_b[:hidden] *= scale
        gemm(f"layer.{i}.qkv", qkv)
        w.add(f"layer.{i}.qkv.bias", qkv_b, "F32", "bias", [3 * hidden])
        ao = p + "attention.output."
        gemm(f"layer.{i}.attn_out", src[ao + "dense.weight"].T)
        w.add(f"layer.{i}.attn_out.bias", src[ao + "dense.bias"], "F32", "bias", [hidden])
        w.add(f"layer.{i}.ln1.weight", src[ao + "LayerNorm.weight"], "F32", "layernorm", [hidden])
        w.add(f"layer.{i}.ln1.bias", src[ao + "LayerNorm.bias"], "F32", "layernorm", [hidden])
        gemm(f"layer.{i}.ffn_up", src[p + "intermediate.dense.weight"].T)
        w.add(f"layer.{i}.ffn_up.bias", src[p + "intermediate.dense.bias"], "F32", "bias",
              [cfg["intermediate_size"]])
        gemm(f"layer.{i}.ffn_down", src[p + "output.dense.weight"].T)
        w.add(f"layer.{i}.ffn_down.bias", src[p + "output.dense.bias"], "F32", "bias", [hidden])
        w.add(f"layer.{i}.ln2.weight", src[p + "output.LayerNorm.weight"], "F32", "layernorm",
              [hidden])
        w.add(f"layer.{i}.ln2.bias", src[p + "output.LayerNorm.bias"], "F32", "layernorm",
              [hidden])
    return w.write(out)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("model_dir")
    ap.add_argument("--out", required=True)
    ap.add_argument("--layout", default="tma_bf16", choices=["tma_bf16", "host"])
    ap.add_argument("--max-seq", type=int, default=None)
    ap.add_argument("--no-fold-scale", action="store_true")
    a = ap.parse_args(argv)
    n = pack_bert(a.model_dir, a.out, a.layout, a.max_seq, not a.no_fold_scale)
    print(f"{a.out}: {n} bytes, layout {a.layout}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
