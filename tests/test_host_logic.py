"""Host-side logic (CPU, no GPU): synthetic inputs, mask handling, the shard
plan, and the multi-rank gather -- the last with real gloo ranks."""

import os
import socket

import numpy as np
import pytest

from nebw import shard, synth


def test_token_layout():
    lens = np.array([1, 2, 8, 128], np.int32)
    ids, mask = synth.make_tokens(4, 128, lens, seed=0)
    assert (ids[:, 0] == synth.CLS_ID).all()
    for b, L in enumerate(lens):
        assert ids[b, L - 1] == (synth.SEP_ID if L > 1 else synth.CLS_ID)
        assert (ids[b, L:] == synth.PAD_ID).all()
        assert (mask[b, :L] == 1).all() and (mask[b, L:] == 0).all()
        inner = ids[b, 1:L - 1]
        assert ((inner >= synth.ID_LO) & (inner <= synth.ID_HI)).all()


@pytest.mark.parametrize("key", sorted(synth.CONFIGS))
def test_length_distributions(key):
    cfg = synth.CONFIGS[key]
    ids, mask, lens = synth.config_batch(cfg)
    assert ids.shape == (cfg.batch, cfg.seq) and lens.shape == (cfg.batch,)
    np.testing.assert_array_equal(mask.sum(1), lens)
    kind = cfg.lengths.split(":")[0]
    if kind == "uniform":
        lo, hi = map(int, cfg.lengths.split(":")[1:])
        assert lens.min() >= lo and lens.max() <= hi
    elif kind == "full":
        assert (lens == cfg.seq).all()
    else:
        assert lens.min() >= 8 and lens.max() <= cfg.seq
        assert 70 <= np.median(lens) <= 125  # log-normal with median 96


def test_mask_to_lengths_refuses_holes():
    m = np.array([[1, 1, 1, 0], [1, 0, 0, 0]], np.int32)
    np.testing.assert_array_equal(synth.mask_to_lengths(m), [3, 1])
    with pytest.raises(ValueError, match="prefix"):
        synth.mask_to_lengths(np.array([[1, 0, 1, 0]], np.int32))


@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_plan_shards_partitions_and_balances(n):
    _, _, lens = synth.config_batch(synth.CONFIGS["bge-large"])
    parts = shard.plan_shards(lens, n)
    allidx = np.sort(np.concatenate(parts))
    np.testing.assert_array_equal(allidx, np.arange(len(lens)))
    assert all((np.diff(p) > 0).all() for p in parts)
    cost = shard.shard_cost(lens)
    loads = np.array([cost[p].sum() for p in parts])
    assert loads.max() / loads.mean() < 1.01  # greedy LPT on 1024 items balances tightly
    again = shard.plan_shards(lens, n)  # deterministic: every rank computes the same plan
    assert all(np.array_equal(a, b) for a, b in zip(parts, again))


def test_unpermute_restores_request_order():
    lens = np.array([5, 300, 7, 512, 64, 9, 100], np.int32)
    parts = shard.plan_shards(lens, 3)
    max_b = max(len(p) for p in parts)
    H = 4
    rows = np.arange(len(lens) * H, dtype=np.float32).reshape(len(lens), H)
    gathered = np.full((3 * max_b, H), np.nan, np.float32)
    for r, p in enumerate(parts):
        gathered[r * max_b:r * max_b + len(p)] = rows[p]
    np.testing.assert_array_equal(shard.unpermute(gathered, parts, max_b), rows)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, outdir):
    """One gloo rank: encode its shard with the CPU oracle, gather to rank 0."""
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "npu-embeddings-xdna1_b200"))
    sys.path.insert(0, str(repo))
    import torch
    import torch.distributed as dist

    from nebw import shard as sh
    from nebw import synth as sy
    from oracle.oracle import PortOracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w = sy.make_weights(sy.MINILM, seed=4, cls_pool=True, layers=1, vocab=2000)
    lens = np.array([3, 40, 17, 64, 9, 33, 1, 50, 8], np.int32)
    ids, mask = sy.make_tokens(len(lens), 64, lens, seed=5)
    ids = np.minimum(ids, 1999)
    parts = sh.plan_shards(lens, world)
    mine = parts[rank]
    max_b = max(len(p) for p in parts)
    emb = PortOracle().encode(w, ids[mine], mask[mine], threads=1)
    local = torch.zeros((max_b, w.hidden), dtype=torch.float32)
    local[:len(mine)] = torch.from_numpy(emb)
    buf = torch.zeros((world * max_b, w.hidden), dtype=torch.float32) if rank == 0 else None
    sh.gather_to_root(local, buf, world, rank, dist)
    if rank == 0:
        full = sh.unpermute(buf.numpy(), parts, max_b)
        np.save(os.path.join(outdir, "gathered.npy"), full)
        np.save(os.path.join(outdir, "single.npy"),
                PortOracle().encode(w, ids, mask, threads=1))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_rank_gather_matches_single_process(tmp_path):
    """Sharded encode + gather + restore on 2 gloo ranks is bit-identical to
    one process encoding the whole batch (rows are independent)."""
    import torch.multiprocessing as mp
    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    np.testing.assert_array_equal(np.load(tmp_path / "gathered.npy"),
                                  np.load(tmp_path / "single.npy"))
