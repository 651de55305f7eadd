"""Host-side logic (CPU, no GPU): synthetic inputs, mask handling, the
library's shard plan and gather order (nebw_shard_plan / nebw_shard_order
through the C ABI), and the multi-rank gather -- the last with real gloo
ranks."""

import os
import socket

import numpy as np
import pytest

from nebw import synth


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


def _greedy_plan(lens, n):
    """Independent restatement of the plan the library documents: sequences
    in decreasing cost l + l^2/2048 (stable), each to the least-loaded rank
    (lowest on ties)."""
    lens = np.asarray(lens, np.float64)
    cost = lens + lens ** 2 / 2048.0
    load = np.zeros(n)
    owner = np.empty(len(lens), np.int64)
    for i in np.argsort(-cost, kind="stable"):
        r = int(np.argmin(load))
        owner[i] = r
        load[r] += cost[i]
    return owner, cost


@pytest.mark.parametrize("n", [1, 2, 3, 4, 8])
def test_shard_plan_partitions_and_balances(n):
    """nebw_shard_plan (C ABI, host only) against the restatement above, on
    the bge-large batch: the same owners, every sequence once, balanced."""
    import nebw
    _, _, lens = synth.config_batch(synth.CONFIGS["bge-large"])
    owner, counts = nebw.shard_plan(lens, n)
    want, cost = _greedy_plan(lens, n)
    np.testing.assert_array_equal(owner, want)
    np.testing.assert_array_equal(counts, np.bincount(want, minlength=n))
    loads = np.array([cost[owner == r].sum() for r in range(n)])
    assert loads.max() / loads.mean() < 1.01  # greedy LPT on 1024 items balances tightly
    again, _ = nebw.shard_plan(lens, n)  # deterministic: every rank computes the same plan
    np.testing.assert_array_equal(owner, again)


def test_shard_order_restores_request_order():
    """nebw_shard_order: row k of the rank-major gather is request
    order[k]; scattering by it restores request order, bit for bit."""
    import nebw
    lens = np.array([5, 300, 7, 512, 64, 9, 100], np.int32)
    owner, counts = nebw.shard_plan(lens, 3)
    order = nebw.shard_order(owner, 3)
    H = 4
    rows = np.arange(len(lens) * H, dtype=np.float32).reshape(len(lens), H)
    gathered = np.concatenate([rows[owner == r] for r in range(3)])  # rank-major, ascending
    out = np.full_like(rows, np.nan)
    out[order] = gathered
    np.testing.assert_array_equal(out, rows)
    np.testing.assert_array_equal(np.sort(order), np.arange(len(lens)))


def test_shard_plan_refusals():
    import nebw
    with pytest.raises(nebw.NebwError, match="ranks refused"):
        nebw.shard_plan(np.array([3, 4], np.int32), 0)
    with pytest.raises(nebw.NebwError, match="outside"):
        nebw.shard_order(np.array([0, 2], np.int32), 2)


def test_comm_unique_id_needs_no_gpu():
    """A communicator id is made on the host (NCCL's bootstrap), 128 bytes,
    fresh each time."""
    import nebw
    a, b = nebw.comm_unique_id(), nebw.comm_unique_id()
    assert len(a) == len(b) == nebw.COMM_ID_BYTES and a != b


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, outdir):
    """One gloo rank: the library's plan picks its shard, the CPU oracle
    encodes it, gloo gathers the padded blocks to rank 0, which compacts them
    by the plan's counts and scatters them by the library's order."""
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path.insert(0, str(repo / "npu-embeddings-xdna1_b200"))
    sys.path.insert(0, str(repo))
    import torch
    import torch.distributed as dist

    import nebw
    from nebw import synth as sy
    from oracle.oracle import PortOracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w = sy.make_weights(sy.MINILM, seed=4, cls_pool=True, layers=1, vocab=2000)
    lens = np.array([3, 40, 17, 64, 9, 33, 1, 50, 8], np.int32)
    ids, mask = sy.make_tokens(len(lens), 64, lens, seed=5)
    ids = np.minimum(ids, 1999)
    owner, counts = nebw.shard_plan(lens, world)
    mine = np.nonzero(owner == rank)[0]
    max_b = int(counts.max())
    emb = PortOracle().encode(w, ids[mine], mask[mine], threads=1)
    local = torch.zeros((max_b, w.hidden), dtype=torch.float32)
    local[:len(mine)] = torch.from_numpy(emb)
    blocks = [torch.zeros_like(local) for _ in range(world)] if rank == 0 else None
    dist.gather(local, blocks, dst=0)
    if rank == 0:
        gathered = np.concatenate([blocks[r][:counts[r]].numpy() for r in range(world)])
        full = np.empty_like(gathered)
        full[nebw.shard_order(owner, world)] = gathered
        np.save(os.path.join(outdir, "gathered.npy"), full)
        np.save(os.path.join(outdir, "single.npy"),
                PortOracle().encode(w, ids, mask, threads=1))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_rank_gather_matches_single_process(tmp_path):
    """Sharded encode + gather + restore on 2 gloo ranks, with the library's
    plan and order, is bit-identical to one process encoding the whole batch
    (rows are independent)."""
    import torch.multiprocessing as mp
    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    np.testing.assert_array_equal(np.load(tmp_path / "gathered.npy"),
                                  np.load(tmp_path / "single.npy"))
