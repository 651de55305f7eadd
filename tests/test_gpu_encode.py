"""Whole-encoder parity on a B200: the CUDA path, called through the C ABI,
against the CPU oracle on the same seeded weights and tokens.

Gate (the north star's): per row cosine >= 0.9999 and max-abs <= 2e-3 after
L2 normalisation; NaN or Inf fails explicitly.
"""

import numpy as np
import pytest

from conftest import parity

pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAX_ABS = 2e-3


def check(got, want, what):
    assert np.isfinite(got).all(), f"{what}: non-finite embedding"
    cos, err = parity(got, want)
    assert cos >= COS_MIN and err <= MAX_ABS, f"{what}: min cos {cos:.7f}, max abs {err:.3e}"
    return cos, err


@pytest.fixture(scope="module")
def minilm():
    from nebw import synth
    cfg = synth.CONFIGS["minilm"]
    return cfg, synth.config_weights(cfg)


def test_minilm_full_batch_vs_oracle(device, port_oracle, minilm):
    """BASELINE config 1 in full: 32 x 128, 6 layers, mean pooling."""
    import nebw
    from nebw import synth
    cfg, w = minilm
    ids, mask, lens = synth.config_batch(cfg)
    m = nebw.Model.from_weights(device, w, max_seq_len=cfg.seq)
    got = m.encode(ids, lens)
    want = port_oracle.encode(w, ids, mask)
    check(got, want, "minilm")
    m.close()


def test_ragged_edges_vs_oracle(device, port_oracle, minilm):
    """Lengths at the edges: 1 (CLS only), 2, the 64-key tile edges, seq."""
    import nebw
    from nebw import synth
    cfg, w = minilm
    lens = np.array([1, 2, 8, 63, 64, 65, 127, 128], np.int32)
    ids, mask = synth.make_tokens(len(lens), cfg.seq, lens, seed=77)
    m = nebw.Model.from_weights(device, w, max_seq_len=cfg.seq)
    got = m.encode(ids, lens)
    want = port_oracle.encode(w, ids, mask)
    check(got, want, "ragged")
    m.close()


def test_cls_pooling_and_erf_variant(device, port_oracle):
    """CLS pooling (bge configs) and the exact-erf GELU variant."""
    import nebw
    from nebw import synth
    w = synth.make_weights(synth.BGE_SMALL, seed=5, cls_pool=True, layers=3, gelu_erf=True)
    lens = np.array([16, 100, 256, 33], np.int32)
    ids, mask = synth.make_tokens(len(lens), 256, lens, seed=6)
    m = nebw.Model.from_weights(device, w, max_seq_len=256)
    got = m.encode(ids, lens)
    want = port_oracle.encode(w, ids, mask)
    check(got, want, "cls+erf")
    m.close()


def test_bge_base_geometry_vs_oracle(device, port_oracle):
    """hidden 768 / head_dim 64 geometry, 2 layers, full-length rows."""
    import nebw
    from nebw import synth
    w = synth.make_weights(synth.BGE_BASE, seed=9, cls_pool=True, layers=2)
    lens = np.array([512, 300, 8], np.int32)
    ids, mask = synth.make_tokens(len(lens), 512, lens, seed=10)
    m = nebw.Model.from_weights(device, w, max_seq_len=512)
    got = m.encode(ids, lens)
    want = port_oracle.encode(w, ids, mask)
    check(got, want, "bge-base-2L")
    m.close()


@pytest.mark.parametrize("arch", ["BGE_BASE", "BGE_SMALL"])
@pytest.mark.parametrize("kind", [0, 1])
def test_attention_kind_encoder_vs_oracle(device, port_oracle, kind, arch):
    """The whole pass with each attention kernel (0 mma.sync, 1 tcgen05, the
    default) at head_dim 64 (bge-base) and 32 (bge-small) across key-block
    and query-tile boundaries: lengths on, just under and just over multiples
    of 64 (the tcgen05 kernel's key block) and 128 (its query tile), partial
    16-key groups, 1 and 512."""
    import nebw
    from nebw import synth
    w = synth.make_weights(getattr(synth, arch), seed=19, cls_pool=True, layers=2)
    lens = np.array([512, 300, 8, 129, 128, 1, 256, 257, 63, 64, 65, 200, 17], np.int32)
    ids, mask = synth.make_tokens(len(lens), 512, lens, seed=20)
    device.set_attention_kernel(kind)
    try:
        m = nebw.Model.from_weights(device, w, max_seq_len=512)
        got = m.encode(ids, lens)
        m.close()
    finally:
        device.set_attention_kernel(device.ATTN_TCGEN05)
    want = port_oracle.encode(w, ids, mask)
    check(got, want, f"attention kind {kind}, {arch}")


def test_npue_container_roundtrip(device, port_oracle, minilm, tmp_path):
    """The same model staged from a .npue container (the reference's file
    format) encodes identically to the in-memory staging."""
    import nebw
    from nebw import synth
    from nebw.npue import write_bert_container
    cfg, w = minilm
    path = tmp_path / "m.npue"
    write_bert_container(path, w, max_seq_len=cfg.seq)
    ids, mask, lens = synth.config_batch(cfg)
    a = nebw.Model.from_weights(device, w, max_seq_len=cfg.seq)
    b = nebw.Model.from_npue(device, path)
    np.testing.assert_array_equal(a.encode(ids, lens), b.encode(ids, lens))
    a.close()
    b.close()


def test_deterministic_and_batch_independent(device, minilm):
    """Rows are computed independently: a row's embedding is bit-identical
    whether it is encoded in the full batch, alone, or in a shuffled batch,
    and repeated runs are bit-identical."""
    import nebw
    from nebw import synth
    cfg, w = minilm
    ids, mask, lens = synth.config_batch(cfg)
    m = nebw.Model.from_weights(device, w, max_seq_len=cfg.seq)
    full = m.encode(ids, lens)
    np.testing.assert_array_equal(full, m.encode(ids, lens))
    perm = np.random.default_rng(0).permutation(len(lens))
    np.testing.assert_array_equal(full[perm], m.encode(ids[perm], lens[perm]))
    for r in (0, 5, 31):
        np.testing.assert_array_equal(full[r:r + 1], m.encode(ids[r:r + 1], lens[r:r + 1]))
    m.close()


def test_encode_refusals(device):
    """Shapes outside what the model was staged for fail by name."""
    import nebw
    from nebw import synth
    w = synth.make_weights(synth.MINILM, seed=3, cls_pool=False, layers=1)
    m = nebw.Model.from_weights(device, w, max_seq_len=64)
    ids, _ = synth.make_tokens(2, 128, np.array([10, 20]), seed=4)
    with pytest.raises(nebw.NebwError, match="seq"):
        m.encode(ids, np.array([10, 20], np.int32))            # S = 128 > max_seq_len 64
    with pytest.raises(nebw.NebwError, match="empty"):
        m.encode(ids[:0, :64], np.zeros(0, np.int32))          # no rows
    ok = m.encode(ids[:, :64], np.array([10, 20], np.int32))   # the same rows, S = 64
    m.close()
    assert np.isfinite(ok).all()


GATED = ["nomic-base", "gte-base"]


@pytest.mark.parametrize("key", GATED)
def test_gated_rope_vs_oracle(device, port_oracle, key, tmp_path):
    """The rotary / gated families (nomic_bert_rope_swiglu: RoPE from theta,
    SwiGLU, no biases; gte_new_rope_geglu: RoPE frequencies as data, erf
    GeGLU, biases) against the oracle -- staged from weights and loaded from
    a container the reference reads -- with lengths across the 64-key and
    128-query attention boundaries, so that every rotary position 0..511
    of the table is used."""
    import nebw
    from nebw import synth
    from nebw.npue import write_bert_container
    cfg = synth.CONFIGS[key]
    w = synth.config_weights(cfg, layers=2)
    lens = np.array([512, 1, 63, 64, 65, 129, 200, 17], np.int32)
    ids, mask = synth.make_tokens(len(lens), 512, lens, seed=43)
    want = port_oracle.encode(w, ids, mask)
    m = nebw.Model.from_weights(device, w, max_seq_len=512)
    check(m.encode(ids, lens), want, f"{key} from weights")
    m.close()
    path = tmp_path / f"{key}.npue"
    write_bert_container(path, w, max_seq_len=512)
    m = nebw.Model.from_npue(device, path)
    assert m.cfg.gated_ffn == 1 and m.cfg.rope == 1
    check(m.encode(ids, lens), want, f"{key} from container")
    m.close()


@pytest.mark.parametrize("name,key", [("nomic_c6", "nomic-base"), ("gte_c7", "gte-base")])
def test_gated_full_depth_matches_reference_golden(device, name, key):
    """Full 12-layer models at seq 512 against the rows the reference's own
    host path produced (tests/golden/)."""
    from pathlib import Path
    import nebw
    from nebw import synth
    g = np.load(Path(__file__).parent / "golden" / f"{name}.npz")
    w = synth.config_weights(synth.CONFIGS[key])
    m = nebw.Model.from_weights(device, w, max_seq_len=512)
    check(m.encode(g["ids"], g["lens"]), g["embeddings"], f"{key} golden")
    m.close()


@pytest.mark.parametrize("override,needle", [
    ({"swiglu_halves": "fc12_gate|fc11_up"}, "swiglu_halves"),
    ({"position_embedding_type": "absolute"}, "position_embedding_type"),
    ({"gated_ffn": False}, "gated_ffn"),
    ({"activation": "relu"}, "activation"),
    ({"rope_theta": 0.0}, "rope_theta"),
])
def test_gated_container_refusals(device, override, needle, tmp_path):
    """A rotary / gated container that is malformed in one key is refused
    with that key named, as the reference's set_model_shape refuses it."""
    import nebw
    from nebw import synth
    from nebw.npue import write_bert_container
    w = synth.config_weights(synth.CONFIGS["nomic-base"], layers=1)
    path = tmp_path / "bad.npue"
    write_bert_container(path, w, max_seq_len=64, config_overrides=override)
    with pytest.raises(nebw.NebwError, match=needle):
        nebw.Model.from_npue(device, path)


def test_gte_container_refuses_missing_freq_or_activation(device, tmp_path):
    import nebw
    from nebw import synth
    from nebw.npue import write_bert_container
    w = synth.config_weights(synth.CONFIGS["gte-base"], layers=1)
    for override, needle in (({"rope_inv_freq": None}, "rope_inv_freq"),
                             ({"activation": None}, "activation"),
                             ({"rope_inv_freq": "[1.0, 0.5]"}, "rope_inv_freq")):
        path = tmp_path / "bad_gte.npue"
        write_bert_container(path, w, max_seq_len=64, config_overrides=override)
        with pytest.raises(nebw.NebwError, match=needle):
            nebw.Model.from_npue(device, path)


_GATED_SINGLE_CTA_CHILD = r"""
import sys
import numpy as np
import nebw
from nebw import synth

key, out = sys.argv[1], sys.argv[2]
w = synth.config_weights(synth.CONFIGS[key], layers=2)
lens = np.array([512, 1, 63, 64, 65, 129, 200, 17], np.int32)
ids, mask = synth.make_tokens(len(lens), 512, lens, seed=43)
dev = nebw.Device(0)
m = nebw.Model.from_weights(dev, w, max_seq_len=512)
np.save(out, m.encode(ids, lens))
m.close()
dev.close()
"""


@pytest.mark.parametrize("key", GATED)
def test_gated_single_cta_path_vs_oracle(port_oracle, key, tmp_path):
    """Without CTA pairs (forced with NEBW_GEMM_CTAS=1 in a child process)
    the gated FFN runs unfused: FFN-up writes [up | gate] and a separate pass
    forms up * act(gate).  That path against the oracle."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    from nebw import synth
    repo = Path(__file__).resolve().parent.parent
    env = dict(os.environ, NEBW_GEMM_CTAS="1",
               PYTHONPATH=os.pathsep.join([str(repo / "npu-embeddings-xdna1_b200"), str(repo)]))
    out = tmp_path / "single.npy"
    subprocess.run([sys.executable, "-c", _GATED_SINGLE_CTA_CHILD, key, str(out)], env=env,
                   check=True, timeout=600)
    w = synth.config_weights(synth.CONFIGS[key], layers=2)
    lens = np.array([512, 1, 63, 64, 65, 129, 200, 17], np.int32)
    ids, mask = synth.make_tokens(len(lens), 512, lens, seed=43)
    check(np.load(out), port_oracle.encode(w, ids, mask), f"{key} single-CTA path")


def test_graph_replay_matches_direct_launches(device):
    """nebw_model_set_graphs: a (B, S) shape's pass is captured once as a CUDA
    graph and replayed by nebw_encode.  Bit for bit the direct launches'
    results: for new rows of a shape already captured (the packed row count
    and the attention work list are computed on the device, so one graph
    serves every length pattern), across shapes, after the workspace grows
    (the graphs are dropped and captured again), and with the mma.sync
    attention kernel (the kernel choice is part of a graph's key)."""
    import nebw
    from nebw import synth
    cfg = synth.CONFIGS["bge-small"]
    w = synth.config_weights(cfg, layers=2)
    ids, _mask, lens = synth.config_batch(cfg)
    rng = np.random.default_rng(0)
    cases = []
    for B, S in [(4, 128), (4, 128), (7, 512), (64, 512), (4, 128), (7, 512), (1, 64)]:
        sel = rng.choice(len(lens), B, replace=False)
        cases.append((np.ascontiguousarray(ids[sel, :S]),
                      np.minimum(lens[sel], S).astype(np.int32)))
    m = nebw.Model.from_weights(device, w, max_seq_len=cfg.seq)
    try:
        want = [m.encode(i, l) for i, l in cases]
    finally:
        m.close()
    m = nebw.Model.from_weights(device, w, max_seq_len=cfg.seq)  # a fresh, unsized workspace
    try:
        m.set_graphs(True)
        for k, (i, l) in enumerate(cases):
            np.testing.assert_array_equal(m.encode(i, l), want[k], err_msg=f"case {k}")
            np.testing.assert_array_equal(m.encode(i, l), want[k], err_msg=f"case {k} again")
        device.set_attention_kernel(device.ATTN_MMA)
        m.set_graphs(False)
        direct = m.encode(*cases[2])
        m.set_graphs(True)
        np.testing.assert_array_equal(m.encode(*cases[2]), direct)
    finally:
        device.set_attention_kernel(device.ATTN_TCGEN05)
        m.close()


def test_graph_replay_device_path(device):
    """The device-buffer entry point with graphs on: a graph per (shape,
    buffers), replayed for new ids and lengths written into the same buffers
    -- bit for bit the direct launches' rows -- on whichever stream the call
    names, torch's legacy default stream (where no capture is allowed: the
    library captures on a stream of its own) and a side stream alike."""
    import torch

    import nebw
    from nebw import synth
    cfg = synth.CONFIGS["bge-small"]
    w = synth.config_weights(cfg, layers=2)
    ids, _mask, lens = synth.config_batch(cfg)
    B, S = 16, 512
    m = nebw.Model.from_weights(device, w, max_seq_len=S)
    try:
        ids_d = torch.empty((B, S), dtype=torch.int32, device="cuda")
        lens_d = torch.empty(B, dtype=torch.int32, device="cuda")
        out = torch.empty((B, m.hidden), device="cuda")
        batches = [(ids[k * B:(k + 1) * B], lens[k * B:(k + 1) * B].astype(np.int32))
                   for k in range(3)]
        want = [m.encode(i, l) for i, l in batches]
        m.set_graphs(True)
        side = torch.cuda.Stream()
        for st in (torch.cuda.current_stream(), side, torch.cuda.current_stream()):
            for k, (i, l) in enumerate(batches):
                with torch.cuda.stream(st):
                    ids_d.copy_(torch.from_numpy(np.ascontiguousarray(i)))
                    lens_d.copy_(torch.from_numpy(l))
                    m.encode_into(ids_d, lens_d, out, B, S, stream=st)
                st.synchronize()
                device.sync()
                np.testing.assert_array_equal(out.cpu().numpy(), want[k])
    finally:
        m.close()


def test_graph_cache_eviction_and_invalidation(device):
    """More shapes than the graph cache keeps (16): the oldest are dropped
    and captured again when they recur, every result still the direct
    launches' bit for bit; and setting a tensor drops the graphs, so that a
    replay never runs on the weights it was captured with after they change."""
    import nebw
    from nebw import synth
    cfg = synth.CONFIGS["minilm"]
    w = synth.config_weights(cfg, layers=1)
    ids, _mask, lens = synth.config_batch(cfg)
    shapes = [(b, 128) for b in range(1, 19)] + [(1, 128), (2, 128)]
    m = nebw.Model.from_weights(device, w, max_seq_len=cfg.seq)
    try:
        want = [m.encode(ids[:b, :S], lens[:b]) for b, S in shapes]
        m.set_graphs(True)
        for k, (b, S) in enumerate(shapes):
            np.testing.assert_array_equal(m.encode(ids[:b, :S], lens[:b]), want[k],
                                          err_msg=f"shape {b} x {S}")
        g = w.ln1_g[0] * 1.5
        m.set_tensor("layer.0.ln1.weight", g)
        m.set_graphs(False)
        direct = m.encode(ids[:4], lens[:4])
        m.set_graphs(True)
        got = m.encode(ids[:4], lens[:4])
        np.testing.assert_array_equal(got, direct)
        assert not np.array_equal(got, want[3])  # the new weights took effect
    finally:
        m.close()
