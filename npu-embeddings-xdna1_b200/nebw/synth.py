"""Seeded synthetic models and token batches of the benchmark configurations.

No checkpoint or dataset is available offline, so every model here is a
random-init instance of the named architecture and every batch is synthetic
with the stated shape and length distribution:

  weights   word/position/type embeddings and every GEMM weight N(0, 0.02);
            linear biases N(0, 0.02) (so the bias epilogue is exercised);
            LayerNorm gamma = 1, beta = 0; fp32 masters.
  layout    GEMM operands in the container's [K, N] layout with Q|K|V fused
            along N and 1/sqrt(head_dim) folded into the Q columns and the Q
            bias, as the reference packer does (pack_npue.py:2742-2750).
  tokens    ids uniform in [1000, 30521]; [CLS]=101 at 0, [SEP]=102 at len-1,
            pad id 0 after; attention mask 1 on [0, len) and 0 after;
            token_type all 0.
  lengths   per configuration (see CONFIGS); the log-normal of the
            bge-large configuration uses median 96 and sigma 0.8, clipped to
            [8, 512] and rounded.

Seeds: weights 20261201 + config index, tokens 20261301 + config index,
unless a caller passes its own.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np

CLS_ID, SEP_ID, PAD_ID = 101, 102, 0
ID_LO, ID_HI = 1000, 30521
VOCAB = 30522
TYPE_VOCAB = 2
LOGNORMAL_SIGMA = 0.8


@dataclass(frozen=True)
class Arch:
    name: str
    layers: int
    hidden: int
    heads: int
    ffn: int
    max_pos: int = 512
    # the gated / rotary families (container arch nomic_bert_rope_swiglu,
    # gte_new_rope_geglu): "" (BERT), "swiglu" or "geglu"; rotary positions
    # from rope_theta, or from an explicit frequency set
    gated: str = ""
    rope: bool = False
    rope_theta: float = 0.0
    rope_inv_freq: tuple = ()

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


@dataclass(frozen=True)
class Config:
    key: str
    arch: Arch
    batch: int
    seq: int
    lengths: str          # "uniform:lo:hi" | "full" | "lognormal:median:sigma"
    cls_pool: bool
    index: int


MINILM = Arch("all-MiniLM-L6-v2", 6, 384, 12, 1536)
BGE_SMALL = Arch("bge-small-en-v1.5", 12, 384, 12, 1536)
BGE_BASE = Arch("bge-base-en-v1.5", 12, 768, 12, 3072)
BGE_LARGE = Arch("bge-large-en-v1.5", 24, 1024, 16, 4096)
# nomic-embed-text-v1.5's shape: post-LN, no biases, SwiGLU, RoPE theta 1000
NOMIC_BASE = Arch("nomic-embed-text-v1.5", 12, 768, 12, 3072, gated="swiglu", rope=True,
                  rope_theta=1000.0)
# gte-base-en-v1.5's shape: GeGLU (exact erf), real biases, RoPE with the
# scaled frequency set inv_freq_i = 160000^(-i/32) / 8^(1/32) as data
GTE_BASE = Arch("gte-base-en-v1.5", 12, 768, 12, 3072, gated="geglu", rope=True,
                rope_inv_freq=tuple(float(160000.0 ** (-i / 32) / 8.0 ** (1 / 32))
                                    for i in range(32)))

CONFIGS = {
    "minilm": Config("minilm", MINILM, 32, 128, "uniform:8:128", False, 0),
    "bge-small": Config("bge-small", BGE_SMALL, 256, 512, "uniform:16:512", True, 1),
    "bge-base": Config("bge-base", BGE_BASE, 512, 512, "full", True, 2),
    "bge-large": Config("bge-large", BGE_LARGE, 1024, 512,
                        f"lognormal:96:{LOGNORMAL_SIGMA}", True, 3),
    # the gated / rotary families on bge-large's length distribution (mean
    # pooling, as both models are used)
    "nomic-base": Config("nomic-base", NOMIC_BASE, 1024, 512,
                         f"lognormal:96:{LOGNORMAL_SIGMA}", False, 6),
    "gte-base": Config("gte-base", GTE_BASE, 1024, 512,
                       f"lognormal:96:{LOGNORMAL_SIGMA}", False, 7),
}


@dataclass
class BertWeights:
    layers: int
    hidden: int
    heads: int
    ffn: int
    vocab: int
    cls_pool: bool
    word: np.ndarray
    pos: np.ndarray
    typ: np.ndarray
    emb_ln_g: np.ndarray
    emb_ln_b: np.ndarray
    w_qkv: list = field(default_factory=list)
    b_qkv: list = field(default_factory=list)
    w_ao: list = field(default_factory=list)
    b_ao: list = field(default_factory=list)
    ln1_g: list = field(default_factory=list)
    ln1_b: list = field(default_factory=list)
    w_up: list = field(default_factory=list)
    b_up: list = field(default_factory=list)
    w_dn: list = field(default_factory=list)
    b_dn: list = field(default_factory=list)
    ln2_g: list = field(default_factory=list)
    ln2_b: list = field(default_factory=list)
    gelu_erf: bool = False
    seed: int = 0
    gated: str = ""
    rope: bool = False
    rope_theta: float = 0.0
    rope_inv_freq: tuple = ()

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def up_width(self) -> int:
        """Columns of ffn_up: 2F ([up | gate]) for the gated families."""
        return 2 * self.ffn if self.gated else self.ffn

    def fingerprint(self) -> str:
        h = hashlib.sha256()
        h.update(f"{self.layers},{self.hidden},{self.heads},{self.ffn},{self.vocab},{self.seed}".encode())
        h.update(self.word[:4].tobytes())
        h.update(self.w_qkv[0][:4].tobytes())
        return h.hexdigest()

    def tensors(self):
        """(name, array) in the container's naming (pack_npue.py:2684-2790)."""
        yield "embeddings.word", self.word
        yield "embeddings.position", self.pos
        yield "embeddings.token_type", self.typ
        yield "embeddings.ln.weight", self.emb_ln_g
        yield "embeddings.ln.bias", self.emb_ln_b
        for i in range(self.layers):
            p = f"layer.{i}."
            yield p + "qkv", self.w_qkv[i]
            yield p + "qkv.bias", self.b_qkv[i]
            yield p + "attn_out", self.w_ao[i]
            yield p + "attn_out.bias", self.b_ao[i]
            yield p + "ln1.weight", self.ln1_g[i]
            yield p + "ln1.bias", self.ln1_b[i]
            yield p + "ffn_up", self.w_up[i]
            yield p + "ffn_up.bias", self.b_up[i]
            yield p + "ffn_down", self.w_dn[i]
            yield p + "ffn_down.bias", self.b_dn[i]
            yield p + "ln2.weight", self.ln2_g[i]
            yield p + "ln2.bias", self.ln2_b[i]


def make_weights(arch: Arch, seed: int, cls_pool: bool, layers: int | None = None,
                 vocab: int = VOCAB, gelu_erf: bool = False) -> BertWeights:
    """Random-init weights of `arch` (optionally truncated to `layers`)."""
    rng = np.random.default_rng(seed)
    H, F = arch.hidden, arch.ffn
    L = arch.layers if layers is None else layers
    scale = np.float32(1.0 / np.sqrt(arch.head_dim))

    def normal(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)

    # nomic has no biases (zero placeholders in its container); the rotary
    # families carry a zero position table (the reference packer's
    # placeholder, which its embedding adds)
    no_bias = arch.gated == "swiglu"

    def bias(n):
        return np.zeros(n, np.float32) if no_bias else normal(n)

    m = BertWeights(
        layers=L, hidden=H, heads=arch.heads, ffn=F, vocab=vocab, cls_pool=cls_pool,
        word=normal(vocab, H),
        pos=np.zeros((arch.max_pos, H), np.float32) if arch.rope else normal(arch.max_pos, H),
        typ=normal(TYPE_VOCAB, H),
        emb_ln_g=np.ones(H, np.float32), emb_ln_b=np.zeros(H, np.float32),
        gelu_erf=gelu_erf, seed=seed, gated=arch.gated, rope=arch.rope,
        rope_theta=arch.rope_theta, rope_inv_freq=arch.rope_inv_freq)
    FW = 2 * F if arch.gated else F
    for _ in range(L):
        wqkv = normal(H, 3 * H)
        bqkv = bias(3 * H)
        wqkv[:, :H] *= scale          # the packer's Q-scale fold (exact before RoPE: linear)
        bqkv[:H] *= scale
        m.w_qkv.append(wqkv)
        m.b_qkv.append(bqkv)
        m.w_ao.append(normal(H, H))
        m.b_ao.append(bias(H))
        m.ln1_g.append(np.ones(H, np.float32))
        m.ln1_b.append(np.zeros(H, np.float32))
        m.w_up.append(normal(H, FW))
        m.b_up.append(bias(FW))
        m.w_dn.append(normal(F, H))
        m.b_dn.append(bias(H))
        m.ln2_g.append(np.ones(H, np.float32))
        m.ln2_b.append(np.zeros(H, np.float32))
    return m


def sample_lengths(spec: str, batch: int, seq: int, rng: np.random.Generator) -> np.ndarray:
    kind, *args = spec.split(":")
    if kind == "uniform":
        lo, hi = int(args[0]), int(args[1])
        lens = rng.integers(lo, hi + 1, size=batch)
    elif kind == "full":
        lens = np.full(batch, seq)
    elif kind == "lognormal":
        median, sigma = float(args[0]), float(args[1])
        lens = np.rint(rng.lognormal(np.log(median), sigma, size=batch))
        lens = np.clip(lens, 8, seq)
    else:
        raise ValueError(f"unknown length distribution {spec!r}")
    return np.minimum(lens.astype(np.int32), seq)


def make_tokens(batch: int, seq: int, lengths: np.ndarray, seed: int):
    """ids [batch, seq] int32, mask [batch, seq] int32 for given lengths."""
    rng = np.random.default_rng(seed)
    ids = rng.integers(ID_LO, ID_HI + 1, size=(batch, seq)).astype(np.int32)
    pos = np.arange(seq)[None, :]
    lens = np.asarray(lengths, np.int32)[:, None]
    mask = (pos < lens).astype(np.int32)
    ids[np.arange(batch), lens[:, 0] - 1] = SEP_ID
    ids[:, 0] = CLS_ID  # a length-1 row is [CLS] alone
    ids[mask == 0] = PAD_ID
    return ids, mask


def config_batch(cfg: Config, seed: int | None = None):
    """(ids, mask, lens) of a configuration's full synthetic batch."""
    seed = 20261301 + cfg.index if seed is None else seed
    rng = np.random.default_rng(seed)
    lens = sample_lengths(cfg.lengths, cfg.batch, cfg.seq, rng)
    ids, mask = make_tokens(cfg.batch, cfg.seq, lens, seed + 1)
    return ids, mask, lens


def config_weights(cfg: Config, layers: int | None = None, seed: int | None = None) -> BertWeights:
    seed = 20261201 + cfg.index if seed is None else seed
    return make_weights(cfg.arch, seed, cfg.cls_pool, layers=layers)


def mask_to_lengths(mask: np.ndarray) -> np.ndarray:
    """Per-row lengths of a prefix attention mask; refuses any other mask.

    The device path packs each sequence's real tokens contiguously, which is
    only the reference's arithmetic when the mask is a prefix of ones (what
    every reference tokenizer emits: wordpiece.cpp:354-378).  A mask with a
    hole would be answered for a different input, so it is refused."""
    mask = np.asarray(mask)
    lens = mask.sum(axis=1).astype(np.int32)
    pos = np.arange(mask.shape[1])[None, :]
    if not np.array_equal(mask != 0, pos < lens[:, None]):
        raise ValueError("attention mask is not a prefix of ones in every row; "
                         "the packed device path cannot represent it")
    return lens


# ---------------------------------------------------------------------------
# ViT (arch vit_patch16_prenorm_gelu): benchmark configuration 5
# ---------------------------------------------------------------------------
#
#   weights   patch embedding, CLS token, position table and every GEMM
#             weight N(0, 0.02); biases N(0, 0.02); LayerNorm gamma = 1,
#             beta = 0; 1/sqrt(head_dim) folded into the Q columns and Q bias
#             (the container's qkv_scale_folded); a random 1000-label head so
#             the container is complete (the head is not on the hot path).
#   images    [n, 3, S, S] fp32 uniform in [-1, 1] (normalised pixels), fed
#             to the reference's im2col order (runtime/src/vit/image.cpp:
#             732-755).


@dataclass(frozen=True)
class VitArch:
    name: str
    layers: int
    hidden: int
    heads: int
    ffn: int
    image_size: int = 224
    patch_size: int = 16
    channels: int = 3
    num_labels: int = 1000
    ln_eps: float = 1e-12

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def n_patches(self) -> int:
        return (self.image_size // self.patch_size) ** 2

    @property
    def n_pos(self) -> int:
        return self.n_patches + 1


@dataclass(frozen=True)
class VitConfig:
    key: str
    arch: VitArch
    batch: int
    index: int


VIT_BASE = VitArch("vit-base-patch16-224", 12, 768, 12, 3072)
VIT_CONFIGS = {"vit-base": VitConfig("vit-base", VIT_BASE, 2048, 4)}


@dataclass
class VitWeights:
    arch: VitArch
    layers: int
    patch_w: np.ndarray          # [C*P*P, H]
    patch_b: np.ndarray
    cls: np.ndarray              # [H]
    pos: np.ndarray              # [n_pos, H]
    lnf_g: np.ndarray
    lnf_b: np.ndarray
    head_w: np.ndarray           # [H, num_labels]
    head_b: np.ndarray
    w_qkv: list = field(default_factory=list)
    b_qkv: list = field(default_factory=list)
    w_ao: list = field(default_factory=list)
    b_ao: list = field(default_factory=list)
    ln1_g: list = field(default_factory=list)
    ln1_b: list = field(default_factory=list)
    w_up: list = field(default_factory=list)
    b_up: list = field(default_factory=list)
    w_dn: list = field(default_factory=list)
    b_dn: list = field(default_factory=list)
    ln2_g: list = field(default_factory=list)
    ln2_b: list = field(default_factory=list)
    seed: int = 0

    hidden = property(lambda self: self.arch.hidden)
    heads = property(lambda self: self.arch.heads)
    head_dim = property(lambda self: self.arch.head_dim)
    ffn = property(lambda self: self.arch.ffn)

    def fingerprint(self) -> str:
        h = hashlib.sha256()
        a = self.arch
        h.update(f"vit,{self.layers},{a.hidden},{a.heads},{a.ffn},{a.image_size},{self.seed}".encode())
        h.update(self.patch_w[:4].tobytes())
        h.update(self.w_qkv[0][:4].tobytes())
        return h.hexdigest()

    def tensors(self):
        """(name, array) in the ViT container's naming (runtime/src/vit/
        encoder.cpp:125-139, :176-207)."""
        yield "frontend.patch_embed", self.patch_w
        yield "frontend.patch_embed.bias", self.patch_b
        yield "frontend.cls_token", self.cls
        yield "frontend.position_embeddings", self.pos
        for i in range(self.layers):
            p = f"layer.{i}."
            yield p + "qkv", self.w_qkv[i]
            yield p + "qkv.bias", self.b_qkv[i]
            yield p + "attn_out", self.w_ao[i]
            yield p + "attn_out.bias", self.b_ao[i]
            yield p + "ffn_up", self.w_up[i]
            yield p + "ffn_up.bias", self.b_up[i]
            yield p + "ffn_down", self.w_dn[i]
            yield p + "ffn_down.bias", self.b_dn[i]
            yield p + "ln1.weight", self.ln1_g[i]
            yield p + "ln1.bias", self.ln1_b[i]
            yield p + "ln2.weight", self.ln2_g[i]
            yield p + "ln2.bias", self.ln2_b[i]
        yield "layernorm.weight", self.lnf_g
        yield "layernorm.bias", self.lnf_b


def make_vit_weights(arch: VitArch, seed: int, layers: int | None = None) -> VitWeights:
    """Random-init weights of a ViT architecture (optionally truncated)."""
    rng = np.random.default_rng(seed)
    H, F = arch.hidden, arch.ffn
    pd = arch.channels * arch.patch_size ** 2
    if pd != H:
        raise ValueError(f"patch_dim {pd} != hidden {H}: the patch embedding rides the "
                         "attention-out GEMM shape in this architecture")
    L = arch.layers if layers is None else layers
    scale = np.float32(1.0 / np.sqrt(arch.head_dim))

    def normal(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)

    m = VitWeights(arch=arch, layers=L, patch_w=normal(pd, H), patch_b=normal(H), cls=normal(H),
                   pos=normal(arch.n_pos, H), lnf_g=np.ones(H, np.float32),
                   lnf_b=np.zeros(H, np.float32), head_w=normal(H, arch.num_labels),
                   head_b=normal(arch.num_labels), seed=seed)
    for _ in range(L):
        wqkv = normal(H, 3 * H)
        bqkv = normal(3 * H)
        wqkv[:, :H] *= scale          # qkv_scale_folded
        bqkv[:H] *= scale
        m.w_qkv.append(wqkv)
        m.b_qkv.append(bqkv)
        m.w_ao.append(normal(H, H))
        m.b_ao.append(normal(H))
        m.ln1_g.append(np.ones(H, np.float32))
        m.ln1_b.append(np.zeros(H, np.float32))
        m.w_up.append(normal(H, F))
        m.b_up.append(normal(F))
        m.w_dn.append(normal(F, H))
        m.b_dn.append(normal(H))
        m.ln2_g.append(np.ones(H, np.float32))
        m.ln2_b.append(np.zeros(H, np.float32))
    return m


def make_images(n: int, arch: VitArch, seed: int) -> np.ndarray:
    """[n, C, S, S] fp32 uniform in [-1, 1]."""
    rng = np.random.default_rng(seed)
    shape = (n, arch.channels, arch.image_size, arch.image_size)
    return rng.uniform(-1.0, 1.0, size=shape).astype(np.float32)


def vit_config_weights(cfg: VitConfig, layers: int | None = None,
                       seed: int | None = None) -> VitWeights:
    return make_vit_weights(cfg.arch, 20261201 + cfg.index if seed is None else seed, layers)


def vit_config_images(cfg: VitConfig, n: int | None = None, seed: int | None = None) -> np.ndarray:
    return make_images(cfg.batch if n is None else n, cfg.arch,
                       20261301 + cfg.index if seed is None else seed)
