"""The sharded pass and the NCCL gather in the library (nebw_comm_*,
nebw_encode_sharded / _shard_gather / _multi), on B200s, through the C ABI.

Rows are independent encoder passes, so the sharded result must equal the
single-GPU pass bit for bit, whatever the plan puts where.  On one GPU the
communicator has one rank (the gather is a local copy plus the request-order
scatter); with two or more GPUs visible the same checks run over NCCL.

The timeout test makes a rank wait for a peer that never joins: the wait is
on the host (NCCL's bootstrap), no kernel is in flight, and the library
aborts the communicator when its timeout expires.
"""

import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from conftest import PKG, REPO

pytestmark = pytest.mark.gpu


def _batch(n=24, S=128, seed=61):
    from nebw import synth
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, S + 1, n).astype(np.int32)
    lens[0], lens[-1] = S, 1
    ids, _ = synth.make_tokens(n, S, lens, seed=seed)
    return ids, lens


def _weights():
    from nebw import synth
    return synth.make_weights(synth.BGE_BASE, seed=11, cls_pool=True, layers=2)


def _gpus():
    import torch
    return torch.cuda.device_count()


def test_one_rank_sharded_equals_single_pass(device):
    import nebw
    w = _weights()
    ids, lens = _batch()
    m = nebw.Model.from_weights(device, w, max_seq_len=ids.shape[1])
    want = m.encode(ids, lens)
    c = nebw.Comm.init_rank(device, 1, 0, nebw.comm_unique_id(), timeout_s=30.0)
    try:
        for _ in range(2):  # the second call reuses the staging and gather buffers
            got = c.encode_sharded(m, ids, lens)
            np.testing.assert_array_equal(got, want)
    finally:
        c.close()
        m.close()


def test_one_rank_device_path_and_order(device):
    """nebw_encode_shard_gather with the shard on the device: rank order
    (no order) and request order through nebw_shard_order."""
    import torch

    import nebw
    w = _weights()
    ids, lens = _batch(n=17, S=64, seed=62)
    m = nebw.Model.from_weights(device, w, max_seq_len=64)
    want = m.encode(ids, lens)
    owner, counts = nebw.shard_plan(lens, 1)
    order = torch.from_numpy(nebw.shard_order(owner, 1)).cuda()
    c = nebw.Comm.init_rank(device, 1, 0, nebw.comm_unique_id(), timeout_s=30.0)
    try:
        ids_d = torch.from_numpy(ids).cuda()
        lens_d = torch.from_numpy(lens).cuda()
        out = torch.full((len(lens), w.hidden), float("nan"), device="cuda")
        s = torch.cuda.current_stream()
        c.encode_shard_gather(m, ids_d, lens_d, len(lens), 64, counts, order, out, stream=s)
        c.sync(stream=s)
        np.testing.assert_array_equal(out.cpu().numpy(), want)
    finally:
        c.close()
        m.close()


def test_encode_multi_over_every_visible_gpu(device):
    """One process, one host thread per GPU (nebw_comm_init_all +
    nebw_encode_multi); on a 1-GPU box this is the single-rank form."""
    import nebw
    n = min(_gpus(), 8)
    w = _weights()
    ids, lens = _batch(n=40, S=128, seed=63)
    ref = nebw.Model.from_weights(device, w, max_seq_len=128)
    want = ref.encode(ids, lens)
    ref.close()
    devs = [device] + [nebw.Device(i) for i in range(1, n)]
    models = [nebw.Model.from_weights(d, w, max_seq_len=128) for d in devs]
    comms = nebw.Comm.init_all(devs, timeout_s=60.0)
    try:
        for _ in range(2):
            got = nebw.encode_multi(models, comms, ids, lens)
            np.testing.assert_array_equal(got, want)
    finally:
        for c in comms:
            c.close()
        for m in models:
            m.close()
        for d in devs[1:]:
            d.close()


def test_encode_multi_int8_datapath(device, tmp_path):
    """The sharded pass runs the model's datapath: an int8 container on the
    int8 datapath (its FFN-down on the CTA-pair int8 GEMM at bge-base's FFN
    of 3072) gives the single-GPU int8 pass's rows bit for bit, over every
    visible GPU (one rank on a 1-GPU box)."""
    import nebw
    from nebw.npue import write_bert_container
    n = min(_gpus(), 8)
    w = _weights()
    ids, lens = _batch(n=40, S=128, seed=65)
    path = tmp_path / "i8.npue"
    write_bert_container(path, w, max_seq_len=128, gemm_layout="pretiled_bf16", a_dtype="i8",
                         tile=(64, 64), mac=(8, 8), smooth_seed=3)
    ref = nebw.Model.from_npue(device, path)
    ref.set_datapath("i8")
    want = ref.encode(ids, lens)
    ref.close()
    devs = [device] + [nebw.Device(i) for i in range(1, n)]
    models = [nebw.Model.from_npue(d, path) for d in devs]
    for m in models:
        m.set_datapath("i8")
    comms = nebw.Comm.init_all(devs, timeout_s=60.0)
    try:
        got = nebw.encode_multi(models, comms, ids, lens)
        np.testing.assert_array_equal(got, want)
    finally:
        for c in comms:
            c.close()
        for m in models:
            m.close()
        for d in devs[1:]:
            d.close()


_RANK = textwrap.dedent("""
    import os, sys
    import numpy as np
    sys.path.insert(0, {pkg!r}); sys.path.insert(0, {repo!r}); sys.path.insert(0, {tests!r})
    import torch
    import nebw
    from test_gpu_multi import _batch, _weights
    rank, world, d = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3]
    uid_path = os.path.join(d, "uid")
    if rank == 0:
        with open(uid_path + ".tmp", "wb") as f:
            f.write(nebw.comm_unique_id())
        os.replace(uid_path + ".tmp", uid_path)
    import time
    t0 = time.time()
    while not os.path.exists(uid_path):
        if time.time() - t0 > 60:
            raise SystemExit("no communicator id")
        time.sleep(0.05)
    uid = open(uid_path, "rb").read()
    dev = nebw.Device(rank)
    w = _weights()
    ids, lens = _batch(n=33, S=128, seed=64)
    m = nebw.Model.from_weights(dev, w, max_seq_len=128)
    c = nebw.Comm.init_rank(dev, world, rank, uid, timeout_s=60.0)
    got = c.encode_sharded(m, ids, lens)
    if rank == 0:
        np.save(os.path.join(d, "sharded.npy"), got)
        np.save(os.path.join(d, "single.npy"), m.encode(ids, lens))
    c.close()
    m.close()
    dev.close()
""")


@pytest.mark.skipif("_gpus() < 2", reason="needs two GPUs")
def test_two_processes_sharded_equals_single_gpu(tmp_path):
    """Two processes, one GPU each (nebw_comm_init_rank with the id passed
    through a file): rank 0's gathered rows equal its own single-GPU pass bit
    for bit."""
    script = tmp_path / "rank.py"
    script.write_text(_RANK.format(pkg=str(PKG), repo=str(REPO), tests=str(REPO / "tests")))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, str(script), str(r), "2", str(tmp_path)], env=env)
             for r in range(2)]
    rcs = [p.wait(timeout=300) for p in procs]
    assert rcs == [0, 0]
    np.testing.assert_array_equal(np.load(tmp_path / "sharded.npy"),
                                  np.load(tmp_path / "single.npy"))


_LONELY = textwrap.dedent("""
    import sys
    sys.path.insert(0, {pkg!r})
    import torch
    import nebw
    dev = nebw.Device(0)
    try:
        nebw.Comm.init_rank(dev, 2, 0, nebw.comm_unique_id(), timeout_s=3.0)
    except nebw.NebwError as e:
        print("code", e.code, str(e))
        sys.exit(0 if e.code == 7 else 3)
    sys.exit(4)
""")


def test_rank_whose_peer_never_joins_times_out(tmp_path):
    """Rank 0 of 2 with no rank 1: the bounded wait on initialisation ends
    with NEBW_ECOMM after the 3 s timeout and the communicator is aborted
    (host-side wait; no kernel in flight)."""
    script = tmp_path / "lonely.py"
    script.write_text(_LONELY.format(pkg=str(PKG)))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, str(script)], capture_output=True, text=True, timeout=120,
                       env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "timeout" in r.stdout and "aborted" in r.stdout
