"""ViT encoder parity on a B200: the CUDA path,
called through the C ABI, against the CPU oracle (the C restatement pinned
bit-exact to the reference's vit/encoder.cpp host path) and against the
golden fixture the reference itself produced.

Gate (the north star's): per row cosine >= 0.9999 and max-abs <= 2e-3 after
L2 normalisation of the CLS rows; NaN or Inf fails explicitly.  Row
independence (a row's result does not depend on the other images of its
batch) is checked bit for bit.
"""

import numpy as np
import pytest

from conftest import REPO, parity

pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAX_ABS = 2e-3


def l2n(x):
    x = np.asarray(x, np.float64)
    return x / np.linalg.norm(x, axis=1, keepdims=True)


def check(got, want, what):
    assert np.isfinite(got).all(), f"{what}: non-finite output"
    cos, err = parity(l2n(got), l2n(want))
    assert cos >= COS_MIN and err <= MAX_ABS, f"{what}: min cos {cos:.7f}, max abs {err:.3e}"
    return cos, err


@pytest.fixture(scope="module")
def small_vit():
    from nebw import synth
    arch = synth.VitArch("vit-test", 2, 768, 12, 3072, image_size=32)
    return arch, synth.make_vit_weights(arch, 7)


@pytest.mark.parametrize("kind", [0, 1])
def test_small_vit_vs_oracle(device, port_oracle, small_vit, kind):
    """Two layers, 32 px images (4 patches + CLS), both attention kernels."""
    import nebw
    from nebw import synth
    arch, w = small_vit
    imgs = synth.make_images(6, arch, 8)
    device.set_attention_kernel(kind)
    try:
        m = nebw.VitModel.from_weights(device, w)
        got = m.encode(imgs)
        m.close()
    finally:
        device.set_attention_kernel(device.ATTN_TCGEN05)
    check(got, port_oracle.vit_encode(w, imgs), f"small ViT, attention kind {kind}")


def test_vit_base_matches_reference_golden(device):
    """vit-base-patch16-224 at full depth: 12 layers, 197 positions, against
    the reference's own output (tests/golden/vit_base_c5.npz)."""
    import hashlib

    import nebw
    from nebw import synth
    g = dict(np.load(REPO / "tests" / "golden" / "vit_base_c5.npz"))
    cfg = synth.VIT_CONFIGS[str(g["config"])]
    imgs = synth.vit_config_images(cfg, n=int(g["n_images"]))
    assert hashlib.sha256(imgs.tobytes()).hexdigest() == str(g["image_sha256"])
    m = nebw.VitModel.from_weights(device, synth.vit_config_weights(cfg))
    got = m.encode(imgs)
    m.close()
    check(got, g["embeddings"], "vit-base golden")


def test_vit_rows_independent_and_deterministic(device, small_vit):
    """An image's CLS row is the same bits whatever else is in its batch."""
    import nebw
    from nebw import synth
    arch, w = small_vit
    imgs = synth.make_images(9, arch, 21)
    m = nebw.VitModel.from_weights(device, w)
    full = m.encode(imgs)
    part = m.encode(imgs[3:5])
    again = m.encode(imgs)
    m.close()
    np.testing.assert_array_equal(full[3:5], part)
    np.testing.assert_array_equal(full, again)


def test_vit_host_path_chunks_match_device_path(device, small_vit):
    """nebw_vit_encode splits a batch of >= 512 images into chunks whose
    host->device copies overlap the pass over the previous chunk: the CLS
    rows are the same bits as one device pass over the whole batch (600
    images -> chunks of 256, 256, 88)."""
    import torch
    import nebw
    from nebw import synth
    arch, w = small_vit
    imgs = synth.make_images(600, arch, 33)
    m = nebw.VitModel.from_weights(device, w)
    host = m.encode(imgs)
    d_img = torch.from_numpy(imgs).cuda()
    d_out = torch.empty((600, m.hidden), dtype=torch.float32, device="cuda")
    m.encode_into(d_img, d_out, 600)
    device.sync()
    dev_rows = d_out.cpu().numpy()
    again = m.encode(imgs)
    m.close()
    assert np.isfinite(host).all()
    np.testing.assert_array_equal(host, dev_rows)
    np.testing.assert_array_equal(host, again)


def test_vit_npue_roundtrip(device, small_vit, tmp_path):
    """A host-layout ViT container loads into the same model as its weights."""
    import nebw
    from nebw import synth
    from nebw.npue import write_vit_container
    arch, w = small_vit
    path = tmp_path / "vit.npue"
    write_vit_container(path, w)
    imgs = synth.make_images(3, arch, 5)
    a = nebw.VitModel.from_weights(device, w)
    b = nebw.VitModel.from_npue(device, path)
    np.testing.assert_array_equal(a.encode(imgs), b.encode(imgs))
    assert b.launch_count() == a.launch_count() > 0
    a.close()
    b.close()


def test_vit_refuses_bad_geometry(device):
    import nebw
    cfg = nebw.VitConfig(num_layers=1, hidden=768, num_heads=12, head_dim=64, intermediate=3072,
                         image_size=30, patch_size=16, num_channels=3, layer_norm_eps=1e-12)
    import ctypes as C
    h = C.c_void_p()
    rc = nebw.lib().nebw_vit_create(device.h, C.byref(cfg), C.byref(h))
    assert rc != 0 and b"patch" in nebw.lib().nebw_last_error()


@pytest.mark.parametrize("name", ["vit_pretiled_bf16_c5", "vit_pretiled_i8_c5"])
def test_vit_pretiled_containers_match_reference_golden(device, tmp_path, name):
    """vit-base with pre-tiled encoder operands (the reference packer's
    default form: bf16 block panels, or int8 with .wscale / .asmooth),
    regenerated byte for byte, loaded by nebw_vit_load_npue and encoded on
    the B200, against the reference's ViT host path on the same container."""
    import hashlib
    import sys

    import nebw
    from nebw import synth
    sys.path.insert(0, str(REPO / "tests" / "golden"))
    import make_golden
    g = dict(np.load(REPO / "tests" / "golden" / f"{name}.npz"))
    key, a_dtype = make_golden.VIT_PRETILED[name]
    path = tmp_path / "v.npue"
    assert make_golden.write_vit_pretiled(path, key, a_dtype) == str(g["container_sha256"])
    images = synth.vit_config_images(synth.VIT_CONFIGS[key], n=int(g["n_images"]))
    assert hashlib.sha256(images.tobytes()).hexdigest() == str(g["image_sha256"])
    m = nebw.VitModel.from_npue(device, path)
    try:
        got = m.encode(images)
    finally:
        m.close()
    check(got, g["embeddings"], name)
