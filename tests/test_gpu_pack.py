"""Containers from the packer (nebw.pack) on a B200: the tma_bf16 layout
(bf16 [N, K] operands uploaded as they are) gives bit-identical embeddings
to the host layout (F32 [K, N] operands re-tiled on the device), and both
match the CPU oracle within the north star's gate."""

import sys
from types import SimpleNamespace

import numpy as np
import pytest

from conftest import REPO, parity

pytestmark = pytest.mark.gpu
sys.path.insert(0, str(REPO / "tests" / "golden"))


def _weights_from_container(path):
    from nebw.npue import ContainerReader
    with ContainerReader(path) as r:
        c = r.config
        L = int(c["num_layers"])
        t = {k: np.array(r.tensor(k), np.float32) for k in r.entries if k != "tokenizer.vocab"}
    per = lambda leaf: [t[f"layer.{i}.{leaf}"] for i in range(L)]  # noqa: E731
    return SimpleNamespace(
        layers=L, hidden=int(c["hidden"]), heads=int(c["num_heads"]), head_dim=int(c["head_dim"]),
        ffn=int(c["intermediate"]), cls_pool=c["pooling"] == "cls", gelu_erf=False,
        word=t["embeddings.word"], pos=t["embeddings.position"], typ=t["embeddings.token_type"],
        emb_ln_g=t["embeddings.ln.weight"], emb_ln_b=t["embeddings.ln.bias"],
        w_qkv=per("qkv"), b_qkv=per("qkv.bias"), w_ao=per("attn_out"), b_ao=per("attn_out.bias"),
        ln1_g=per("ln1.weight"), ln1_b=per("ln1.bias"), w_up=per("ffn_up"),
        b_up=per("ffn_up.bias"), w_dn=per("ffn_down"), b_dn=per("ffn_down.bias"),
        ln2_g=per("ln2.weight"), ln2_b=per("ln2.bias"))


def test_packed_layouts_identical_and_match_oracle(device, port_oracle, tmp_path):
    import nebw
    from make_pack_golden import MAX_SEQ, synthetic_checkpoint
    from nebw import synth
    from nebw.pack import pack_bert
    d = tmp_path / "tiny-bert"
    synthetic_checkpoint(d)
    pack_bert(d, tmp_path / "host.npue", layout="host", max_seq=MAX_SEQ)
    pack_bert(d, tmp_path / "tma.npue", layout="tma_bf16", max_seq=MAX_SEQ)
    lens = np.array([MAX_SEQ, 1, 37, 64, 65, 100, 8, 127], np.int32)
    ids, mask = synth.make_tokens(len(lens), MAX_SEQ, lens, seed=3)
    ids = np.where(ids >= 1000, ids % 995 + 5, ids).astype(np.int32)  # a 1000-id vocabulary
    a = nebw.Model.from_npue(device, tmp_path / "host.npue")
    b = nebw.Model.from_npue(device, tmp_path / "tma.npue")
    ea, eb = a.encode(ids, lens), b.encode(ids, lens)
    a.close()
    b.close()
    np.testing.assert_array_equal(ea, eb)
    want = port_oracle.encode(_weights_from_container(tmp_path / "host.npue"), ids, mask)
    cos, err = parity(ea, want)
    assert np.isfinite(ea).all() and cos >= 0.9999 and err <= 2e-3, (cos, err)
