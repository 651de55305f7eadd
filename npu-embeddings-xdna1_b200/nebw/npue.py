"""The `.npue` weight container, written and read without the reference tree.

The container is the reference's model file (tools/lib/npue.py:1-35, :261,
:790-872; C++ reader runtime/src/model.cpp:214-380).  This module is an
independent implementation of the same on-disk format, because the format is
the interface: a container written here must be readable by the reference's
own `npue::File`, and the B200 library stages its weights from one.

  [0:64]                  header "<4sIII QQQQ 16s": magic b"NPUE", version 1,
                          arch, flags, json_offset, json_length, data_offset,
                          data_length, 16 reserved bytes
  [json_offset:+len]      UTF-8 JSON {"config": {...}, "tensors": [entry...]}
  [data_offset:+len]      tensor bytes, each tensor 4096-byte aligned;
                          data_offset itself 4096-aligned

An entry is {name, role, dtype, logical_shape, padded_shape, offset, nbytes}
with `offset` relative to data_offset.  tests/test_npue_format.py checks that
this writer produces byte-identical files to the reference writer.
"""

from __future__ import annotations

import hashlib
import json
import mmap
import struct
from pathlib import Path

import numpy as np

MAGIC = b"NPUE"
VERSION = 1
HEADER = struct.Struct("<4sIII QQQQ 16s")
ALIGN = 4096
ARCH_BERT = 0
ARCH_NOMIC = 2   # nomic_bert_rope_swiglu
ARCH_GTE = 3     # gte_new_rope_geglu
FLAG_PRETILED = 1

DTYPES = {
    "F32": np.dtype("<f4"),
    "I32": np.dtype("<i4"),
    "I64": np.dtype("<i8"),
    "U16": np.dtype("<u2"),
    "BF16": np.dtype("<u2"),
    "I8": np.dtype("<i1"),
    "U8": np.dtype("<u1"),
}


def tma_b_layout() -> dict:
    """The byte layout of a tma_bf16 container's GEMM operands: dense
    row-major [N, K] bf16, each output column's K weights contiguous -- the
    B operand the library's tcgen05 GEMM tiles with TMA as it loads (the
    swizzle is applied by the load, not stored).  Built here only, so that the
    packer and the tests describe it with one dict."""
    return {"kind": "dense", "order": "n,k", "dtype": "BF16"}


def layout_hash(layout: dict) -> str:
    """sha256 of the descriptor's canonical JSON (sorted keys, no spaces),
    the scheme of the reference's `layout_hash` (tools/lib/npue.py:777-785):
    the loader compares one string and refuses a mismatch rather than read
    bytes laid out for another kernel."""
    canonical = json.dumps(layout, sort_keys=True, separators=(",", ":"))
    return hashlib.sha256(canonical.encode("utf-8")).hexdigest()


def untile_block_panel(flat, K: int, N: int, layout: dict) -> np.ndarray:
    """A `block_panel` GEMM operand (the reference's pre-tiled array layout)
    back to row-major [K, N].  The flat panel runs over the axes (kb, nb, ri,
    ci, si, ti), ti fastest, of sizes (K/tile_k, N/tile_n, tile_k/mac_s,
    tile_n/mac_t, mac_s, mac_t), with k = kb*tile_k + ri*mac_s + si and
    n = nb*tile_n + ci*mac_t + ti (runtime/include/common/host_b.hpp:22-30).
    Only order "k,n,kt,nt" with inner "s,t" is defined there."""
    _check_panel(K, N, layout)
    tk, tn, s, t = (int(layout[k]) for k in ("tile_k", "tile_n", "mac_s", "mac_t"))
    x = np.asarray(flat).reshape(K // tk, N // tn, tk // s, tn // t, s, t)
    return np.ascontiguousarray(x.transpose(0, 2, 4, 1, 3, 5).reshape(K, N))


def tile_block_panel(kn, layout: dict) -> np.ndarray:
    """Row-major [K, N] to the flat `block_panel` order (untile_block_panel's
    inverse)."""
    K, N = kn.shape
    _check_panel(K, N, layout)
    tk, tn, s, t = (int(layout[k]) for k in ("tile_k", "tile_n", "mac_s", "mac_t"))
    x = np.asarray(kn).reshape(K // tk, tk // s, s, N // tn, tn // t, t)
    return np.ascontiguousarray(x.transpose(0, 3, 1, 4, 2, 5).reshape(-1))


def block_panel_layout(tile_k: int, tile_n: int, mac_s: int, mac_t: int, dtype: str) -> dict:
    """The descriptor of a block-panel operand, with the reference's keys."""
    return {"kind": "block_panel", "tile_k": tile_k, "tile_n": tile_n, "order": "k,n,kt,nt",
            "inner": "s,t", "mac_s": mac_s, "mac_t": mac_t, "dtype": dtype}


def _check_panel(K: int, N: int, layout: dict):
    if layout.get("kind") != "block_panel" or layout.get("order") != "k,n,kt,nt" or \
            layout.get("inner") != "s,t":
        raise ValueError(f"layout {layout!r}: only block_panel k,n,kt,nt / s,t is defined")
    tk, tn, s, t = (int(layout[k]) for k in ("tile_k", "tile_n", "mac_s", "mac_t"))
    if K % tk or N % tn or tk % s or tn % t:
        raise ValueError(f"[{K}, {N}] does not tile into ({tk}, {tn}) with mac ({s}, {t})")


def _pad(n: int) -> int:
    return (-n) % ALIGN


class ContainerWriter:
    """Collects tensors, then writes header + directory + aligned data."""

    def __init__(self, config: dict, arch: int = ARCH_BERT, flags: int = FLAG_PRETILED):
        self.config = dict(config)
        self.arch = arch
        self.flags = flags
        self._entries: list[dict] = []
        self._arrays: list[np.ndarray] = []
        self._cursor = 0

    def add(self, name: str, array, dtype: str, role: str, shape, layout: dict | None = None) -> dict:
        arr = np.ascontiguousarray(array, dtype=DTYPES[dtype])
        nbytes = arr.nbytes
        entry = {
            "name": name,
            "role": role,
            "dtype": dtype,
            "logical_shape": [int(s) for s in shape],
            "padded_shape": [int(s) for s in shape],
            "offset": self._cursor,
            "nbytes": nbytes,
        }
        if layout is not None:  # a laid-out operand carries its descriptor and hash
            entry["layout"] = dict(layout)
            entry["layout_hash"] = layout_hash(layout)
        self._entries.append(entry)
        self._arrays.append(arr)
        self._cursor += nbytes + _pad(nbytes)
        return entry

    def write(self, path) -> int:
        directory = json.dumps({"config": self.config, "tensors": self._entries},
                               separators=(",", ":")).encode("utf-8")
        json_offset = HEADER.size
        data_offset = json_offset + len(directory)
        data_offset += _pad(data_offset)
        head = HEADER.pack(MAGIC, VERSION, self.arch, self.flags, json_offset,
                           len(directory), data_offset, self._cursor, b"\0" * 16)
        with open(path, "wb") as f:
            f.write(head)
            f.write(directory)
            f.write(b"\0" * (data_offset - json_offset - len(directory)))
            for arr in self._arrays:
                # tofile streams without building a second copy of big tensors
                arr.tofile(f)
                f.write(b"\0" * _pad(arr.nbytes))
        return data_offset + self._cursor


class ContainerReader:
    """mmap reader; `tensor(name)` returns a read-only numpy view."""

    def __init__(self, path):
        self.path = str(path)
        self._file = open(self.path, "rb")
        self._map = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
        (magic, version, self.arch, self.flags, jo, jl, self.data_offset,
         self.data_length, _) = HEADER.unpack_from(self._map, 0)
        if magic != MAGIC:
            raise ValueError(f"{path}: not a .npue container (magic {magic!r})")
        if version != VERSION:
            raise ValueError(f"{path}: container version {version}, expected {VERSION}")
        if self.data_offset % ALIGN:
            raise ValueError(f"{path}: data_offset is not {ALIGN}-aligned")
        d = json.loads(bytes(self._map[jo:jo + jl]).decode("utf-8"))
        self.config = d["config"]
        self.entries = {e["name"]: e for e in d["tensors"]}

    def tensor(self, name: str) -> np.ndarray:
        e = self.entries[name]
        start = self.data_offset + e["offset"]
        a = np.frombuffer(self._map, dtype=DTYPES[e["dtype"]],
                          count=e["nbytes"] // DTYPES[e["dtype"]].itemsize, offset=start)
        return a.reshape(e["logical_shape"])

    def close(self):
        self._map.close()
        self._file.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False


def _bf16_bits(x) -> np.ndarray:
    """fp32 -> bf16 bits, round to nearest even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def quantise_int8_columns(kn, asmooth):
    """Weight side of the int8 datapath, as this writer produces it: W' =
    diag(asmooth) W, per-column wscale = max_k |W'| / 127 (1 for a zero
    column), q = round-half-even(W' / wscale) clamped to +-127.  Returns
    (q int8 [K, N], wscale f32 [N])."""
    wp = np.asarray(kn, np.float32) * np.asarray(asmooth, np.float32)[:, None]
    mx = np.abs(wp).max(axis=0)
    ws = np.where(mx > 0, mx / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(wp / ws[None, :]), -127, 127).astype(np.int8)
    return q, ws


def _add_gemm_operand(w, name, kn, pretiled: bool, i8: bool, tile, mac, srng):
    """One GEMM operand [K, N]: F32 row-major (host layout), or a block panel
    of bf16, or of int8 with its .wscale and a seeded .asmooth."""
    kn = np.asarray(kn, np.float32)
    K, N = kn.shape
    if not pretiled:
        w.add(name, kn, "F32", "gemm_b_host", [K, N])
        return
    layout = block_panel_layout(int(tile[0]), int(tile[1]), int(mac[0]), int(mac[1]),
                                "I8" if i8 else "BF16")
    if not i8:
        w.add(name, tile_block_panel(_bf16_bits(kn), layout), "BF16", "gemm_b", [K, N],
              layout=layout)
        return
    asm = srng.lognormal(0.0, 0.5, K).astype(np.float32)
    q, ws = quantise_int8_columns(kn, asm)
    w.add(name, tile_block_panel(q, layout), "I8", "gemm_b", [K, N], layout=layout)
    w.add(name + ".wscale", ws, "F32", "quant_scale", [N])
    w.add(name + ".asmooth", asm, "F32", "quant_smooth", [K])


def write_bert_container(path, model, max_seq_len: int, source_repo: str = "synthetic/random-init",
                         config_overrides: dict | None = None, gemm_layout: str = "host",
                         a_dtype: str = "bf16", tile=(64, 32), mac=(8, 8), smooth_seed: int = 0,
                         vocab: bytes | None = None):
    """Write a BERT (arch 0) container in the host layout the reference's CPU
    path reads: GEMM operands F32 row-major [K, N] (`gemm_b_host`), biases and
    LayerNorm F32, embeddings F32.  Tensor names and config keys follow the
    reference packer's BERT branch (tools/pack/pack_npue.py:2640-2790); the
    config keys are the ones set_model_shape() requires
    (runtime/include/common/app_state.hpp:380-631).

    gemm_layout "pretiled_bf16" writes the reference's pre-tiled form instead:
    each GEMM operand a `block_panel` of `tile` = (tile_k, tile_n) tiles in
    `mac` = (mac_s, mac_t) sub-tiles with its layout descriptor and
    layout_hash, as bf16 (a_dtype "bf16") or as int8 (a_dtype "i8") with its
    per-column `.wscale` and the activation's SmoothQuant divisor `.asmooth`
    (seeded positive factors, not calibrated: any factors describe the same
    model, W' = diag(asmooth) W against A / asmooth).

    vocab: the WordPiece vocabulary file's bytes, stored as the packer stores
    it (`tokenizer.vocab`, U8), for the runtime's tokenizer."""
    if gemm_layout not in ("host", "pretiled_bf16") or a_dtype not in ("bf16", "i8"):
        raise ValueError(f"gemm_layout {gemm_layout!r} / a_dtype {a_dtype!r}")
    pretiled = gemm_layout == "pretiled_bf16"
    i8 = pretiled and a_dtype == "i8"
    srng = np.random.default_rng(smooth_seed)
    H, F, L = model.hidden, model.ffn, model.layers
    gated = getattr(model, "gated", "")
    FW = 2 * F if gated else F
    arch_name = {"": "bert_abs_gelu_postln", "swiglu": "nomic_bert_rope_swiglu",
                 "geglu": "gte_new_rope_geglu"}[gated]
    config = {
        "arch": arch_name,
        "source_repo": source_repo,
        "source_sha256": model.fingerprint(),
        "num_layers": L, "num_heads": model.heads, "hidden": H,
        "head_dim": model.head_dim, "intermediate": F,
        "layer_norm_eps": 1e-12,
        "vocab_size": model.vocab,
        "max_seq_len": int(max_seq_len),
        "pooling": "cls" if model.cls_pool else "mean",
        "l2_normalize": True,
        "activation": "gelu_erf_exact",
        "gemm_layout": gemm_layout,
        "a_dtype": a_dtype if pretiled else "f32",
        "fusions": {
            "qkv_fused": True,
            "transposed_to_kn": True,
            "qk_scale_folded_into_q": True,
            "gemm_operands_bf16": pretiled and not i8,
            "biases_and_layernorm_fp32": True,
            "position_embeddings_presliced_to": int(max_seq_len),
        },
    }
    if pretiled:
        config.update(tile_k=int(tile[0]), tile_n=int(tile[1]), mac_s=int(mac[0]),
                      mac_t=int(mac[1]))
    header_arch = ARCH_BERT
    if gated:
        # the keys set_model_shape reads for the gated / rotary families
        # (app_state.hpp:440-560): a zero position placeholder, the fused
        # FFN-up halves' order, the gate's activation, the rotary frequencies
        config["position_embedding_type"] = "rope"
        config["gated_ffn"] = True
        if gated == "swiglu":
            header_arch = ARCH_NOMIC
            config["swiglu_halves"] = "fc11_up|fc12_gate"
            config["activation"] = "silu"
            config["rope_theta"] = float(model.rope_theta)
        else:
            header_arch = ARCH_GTE
            config["glu_halves"] = "up_first|gate_second (gate half gets the activation)"
            config["activation"] = "gelu"
            config["rope_inv_freq"] = json.dumps([float(np.float32(v)) for v in model.rope_inv_freq])
    # config_overrides: keys to replace (None: drop), for malformed-container tests
    for k, v in (config_overrides or {}).items():
        if v is None:
            config.pop(k, None)
        else:
            config[k] = v
    w = ContainerWriter(config, arch=header_arch)

    def gemm(name, kn):
        _add_gemm_operand(w, name, kn, pretiled, i8, tile, mac, srng)

    w.add("embeddings.word", model.word, "F32", "embedding", [model.vocab, H])
    w.add("embeddings.position", model.pos[:max_seq_len], "F32", "embedding", [max_seq_len, H])
    w.add("embeddings.token_type", model.typ, "F32", "embedding", [model.typ.shape[0], H])
    w.add("embeddings.ln.weight", model.emb_ln_g, "F32", "layernorm", [H])
    w.add("embeddings.ln.bias", model.emb_ln_b, "F32", "layernorm", [H])
    if vocab is not None:
        vb = np.frombuffer(vocab, dtype=np.uint8)
        w.add("tokenizer.vocab", vb, "U8", "tokenizer", [int(vb.size)])
    for i in range(L):
        p = f"layer.{i}."
        gemm(p + "qkv", model.w_qkv[i])
        w.add(p + "qkv.bias", model.b_qkv[i], "F32", "bias", [3 * H])
        gemm(p + "attn_out", model.w_ao[i])
        w.add(p + "attn_out.bias", model.b_ao[i], "F32", "bias", [H])
        w.add(p + "ln1.weight", model.ln1_g[i], "F32", "layernorm", [H])
        w.add(p + "ln1.bias", model.ln1_b[i], "F32", "layernorm", [H])
        gemm(p + "ffn_up", model.w_up[i])
        w.add(p + "ffn_up.bias", model.b_up[i], "F32", "bias", [FW])
        gemm(p + "ffn_down", model.w_dn[i])
        w.add(p + "ffn_down.bias", model.b_dn[i], "F32", "bias", [H])
        w.add(p + "ln2.weight", model.ln2_g[i], "F32", "layernorm", [H])
        w.add(p + "ln2.bias", model.ln2_b[i], "F32", "layernorm", [H])
    return w.write(path)


def write_vit_container(path, model, source_repo: str = "synthetic/random-init",
                        gemm_layout: str = "host", a_dtype: str = "bf16", tile=(64, 64),
                        mac=(8, 8), smooth_seed: int = 0):
    """Write a ViT (arch vit_patch16_prenorm_gelu) container in the host
    layout: GEMM operands F32 row-major [K, N], everything else F32.  Config
    keys are the ones read_geometry() requires (runtime/include/vit/
    geometry.hpp), tensor names the ones VitEncoder::stage_all() reads
    (runtime/src/vit/encoder.cpp:125-189).  gemm_layout "pretiled_bf16"
    writes the encoder's GEMM operands (patch embedding and the four per
    layer) as block panels instead, as write_bert_container does; the
    classifier head stays F32."""
    if gemm_layout not in ("host", "pretiled_bf16") or a_dtype not in ("bf16", "i8"):
        raise ValueError(f"gemm_layout {gemm_layout!r} / a_dtype {a_dtype!r}")
    pretiled = gemm_layout == "pretiled_bf16"
    i8 = pretiled and a_dtype == "i8"
    srng = np.random.default_rng(smooth_seed)
    a = model.arch
    H, F, L = a.hidden, a.ffn, model.layers
    pd = a.channels * a.patch_size ** 2
    config = {
        "arch": "vit_patch16_prenorm_gelu",
        "source_repo": source_repo,
        "source_sha256": model.fingerprint(),
        "num_layers": L, "num_heads": a.heads, "hidden": H, "head_dim": a.head_dim,
        "intermediate": F, "num_labels": a.num_labels,
        "image_size": a.image_size, "crop_size": a.image_size, "patch_size": a.patch_size,
        "num_channels": a.channels, "patch_dim": pd, "n_patches": a.n_patches,
        "max_seq_len": a.n_pos, "resample": 3, "image_resize": "square",
        "image_mean": [0.5] * a.channels, "image_std": [0.5] * a.channels,
        "layer_norm_eps": a.ln_eps, "attention_scale": 1.0 / float(np.sqrt(a.head_dim)),
        "qkv_scale_folded": True,
        "gemm_layout": gemm_layout,
        # the ViT packer spells the operand type in capitals
        # (tools/pack/packers/vit.py:113, 554, 637), and its encoder compares so
        "a_dtype": ("I8" if i8 else "BF16") if pretiled else "f32",
    }
    if pretiled:
        config.update(tile_k=int(tile[0]), tile_n=int(tile[1]), mac_s=int(mac[0]),
                      mac_t=int(mac[1]))
    w = ContainerWriter(config)
    shapes = {"frontend.patch_embed": [pd, H], "frontend.patch_embed.bias": [H],
              "frontend.cls_token": [H], "frontend.position_embeddings": [a.n_pos, H],
              "layernorm.weight": [H], "layernorm.bias": [H]}
    for name, arr in model.tensors():
        if name in shapes:
            shape = shapes[name]
        else:
            kind = name.split(".", 2)[2]
            shape = {"qkv": [H, 3 * H], "qkv.bias": [3 * H], "attn_out": [H, H],
                     "attn_out.bias": [H], "ffn_up": [H, F], "ffn_up.bias": [F],
                     "ffn_down": [F, H], "ffn_down.bias": [H]}.get(kind, [H])
        if len(shape) == 2 and name != "frontend.position_embeddings":
            _add_gemm_operand(w, name, np.asarray(arr, np.float32).reshape(shape), pretiled, i8,
                              tile, mac, srng)
            continue
        role = "embedding" if name.startswith("frontend.") else \
            ("layernorm" if ".ln" in name or name.startswith("layernorm") else "bias")
        w.add(name, arr, "F32", role, shape)
    w.add("classifier.weight", model.head_w, "F32", "gemm_b_host", [H, a.num_labels])
    w.add("classifier.bias", model.head_b, "F32", "bias", [a.num_labels])
    return w.write(path)
