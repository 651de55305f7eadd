"""The no-allocation encoder entry point, nebw_encode_device_static.

It exists for callers that cannot allocate device memory when a request
arrives (a serving process that claims its whole GPU-memory budget at
start-up, or a program sharing the GPU under a fixed partition): it runs the
same kernels as nebw_encode_device with every intermediate in one static
64 MiB device array instead of the model's cudaMalloc'd workspace, so its
output is compared with the allocating entry point's bit for bit.  Every
sequence is computed independently of its batch neighbours, so a permuted
batch gives the permuted rows, also bit for bit.

This file is collected last on purpose, and it must pass both alone in a
fresh process and after every other test.  Device buffers here come from
torch; the entry point is called through the C ABI with ctypes.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _call(fn, *args):
    import nebw
    rc = fn(*args)
    if rc != 0:
        raise nebw.NebwError(rc, nebw.lib().nebw_last_error().decode())


def test_static_entry_matches_allocating_entry_twice(device):
    import torch

    import nebw
    from nebw import synth

    cfg = synth.CONFIGS["minilm"]
    w = synth.config_weights(cfg, layers=3)
    ids, _mask, lens = synth.config_batch(cfg)
    B, S = ids.shape
    model = nebw.Model.from_weights(device, w, max_seq_len=S)
    lib = nebw.lib()
    stream = C.c_void_p(nebw._stream(torch.cuda.current_stream()))
    ids_d = torch.from_numpy(ids).cuda()
    lens_d = torch.from_numpy(lens).cuda()
    want = torch.empty((B, w.hidden), dtype=torch.float32, device="cuda")
    _call(lib.nebw_encode_device, model.h, ids_d.data_ptr(), lens_d.data_ptr(), B, S,
          want.data_ptr(), stream)
    device.sync()
    want_h = want.cpu().numpy()
    # two calls in a row: the second sees the first call's leftovers in the
    # shared static array, and a different batch order
    for order in (np.arange(B), np.random.default_rng(1).permutation(B)):
        ids_o = torch.from_numpy(np.ascontiguousarray(ids[order])).cuda()
        lens_o = torch.from_numpy(np.ascontiguousarray(lens[order])).cuda()
        got = torch.full((B, w.hidden), float("nan"), dtype=torch.float32, device="cuda")
        _call(lib.nebw_encode_device_static, model.h, ids_o.data_ptr(), lens_o.data_ptr(), B, S,
              got.data_ptr(), stream)
        device.sync()
        got_h = got.cpu().numpy()
        assert np.isfinite(got_h).all()
        np.testing.assert_array_equal(got_h, want_h[order])
    model.close()


def test_static_entry_refuses_oversized_batch(device):
    import torch

    import nebw
    from nebw import synth

    w = synth.make_weights(synth.BGE_LARGE, seed=3, cls_pool=True, layers=1)
    model = nebw.Model.from_weights(device, w, max_seq_len=512)
    B, S = 8, 512  # 4096 padded rows of bge-large width: more than 64 MiB of scratch
    ids_d = torch.full((B, S), 1000, dtype=torch.int32, device="cuda")
    lens_d = torch.full((B,), S, dtype=torch.int32, device="cuda")
    out = torch.empty((B, w.hidden), dtype=torch.float32, device="cuda")
    with pytest.raises(nebw.NebwError, match="static scratch"):
        _call(nebw.lib().nebw_encode_device_static, model.h, ids_d.data_ptr(), lens_d.data_ptr(),
              B, S, out.data_ptr(), None)
    model.close()


@pytest.mark.parametrize("key", ["nomic-base", "gte-base"])
def test_static_entry_rotary_models(device, key):
    """The rotary / gated families through the static entry point: their
    rotary tables are built when the model is created (or its frequency set
    is given), and the per-row positions the QKV GEMM's epilogue rotates by
    are carved from the static array, so the pass allocates nothing and runs
    the allocating entry point's kernels; two calls in a row, bit for bit."""
    import torch

    import nebw
    from nebw import synth

    w = synth.config_weights(synth.CONFIGS[key], layers=2)
    lens = np.array([64, 1, 33, 63, 17, 40], np.int32)
    S = 64
    ids, _mask = synth.make_tokens(len(lens), S, lens, seed=47)
    B = len(lens)
    model = nebw.Model.from_weights(device, w, max_seq_len=S)
    try:
        lib = nebw.lib()
        stream = C.c_void_p(nebw._stream(torch.cuda.current_stream()))
        ids_d = torch.from_numpy(ids).cuda()
        lens_d = torch.from_numpy(lens).cuda()
        want = torch.empty((B, w.hidden), dtype=torch.float32, device="cuda")
        _call(lib.nebw_encode_device, model.h, ids_d.data_ptr(), lens_d.data_ptr(), B, S,
              want.data_ptr(), stream)
        device.sync()
        want_h = want.cpu().numpy()
        assert np.isfinite(want_h).all()
        # the scratch holds the earlier tests' leftovers (another layout): the
        # rows past the packed ones must not reach the output
        for _ in range(2):
            got = torch.full((B, w.hidden), float("nan"), dtype=torch.float32, device="cuda")
            _call(lib.nebw_encode_device_static, model.h, ids_d.data_ptr(), lens_d.data_ptr(),
                  B, S, got.data_ptr(), stream)
            device.sync()
            got_h = got.cpu().numpy()
            assert np.isfinite(got_h).all()
            np.testing.assert_array_equal(got_h, want_h)
    finally:
        model.close()
