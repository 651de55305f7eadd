"""The CUDA path against the committed golden fixtures (made by the
reference's own host-CPU path, tests/golden/make_golden.py), on a B200,
through the C ABI.  One fixture per benchmark configuration, full-depth
models at the configurations' own sequence lengths.

Gate: per row cosine >= 0.9999 and max-abs <= 2e-3 after L2 normalisation.
"""

import numpy as np
import pytest

from conftest import REPO, parity

pytestmark = pytest.mark.gpu

GOLDEN = REPO / "tests" / "golden"


@pytest.mark.parametrize("name", ["minilm_c1", "bge_small_c2", "bge_base_c3", "bge_large_c4"])
def test_gpu_matches_reference_golden(device, name):
    import nebw
    from nebw import synth
    g = dict(np.load(GOLDEN / f"{name}.npz"))
    cfg = synth.CONFIGS[str(g["config"])]
    w = synth.config_weights(cfg)
    m = nebw.Model.from_weights(device, w, max_seq_len=cfg.seq)
    got = m.encode(g["ids"], g["lens"])
    m.close()
    assert np.isfinite(got).all()
    cos, err = parity(got, g["embeddings"])
    assert cos >= 0.9999 and err <= 2e-3, f"{name}: min cos {cos:.7f}, max abs {err:.3e}"


def test_full_bge_large_batch_holds_the_golden_rows(device):
    """BASELINE configuration 4 at its full size (1024 x 512, log-normal
    lengths): the rows the reference computed for the golden fixture come out
    of the full-batch pass within the gate, every row is finite and unit
    length, and a sub-batch of the same rows gives the same bits."""
    import nebw
    from nebw import synth
    g = dict(np.load(GOLDEN / "bge_large_c4.npz"))
    cfg = synth.CONFIGS["bge-large"]
    ids, mask, lens = synth.config_batch(cfg)
    m = nebw.Model.from_weights(device, synth.config_weights(cfg), max_seq_len=cfg.seq)
    full = m.encode(ids, lens)
    rows = g["rows"]
    part = m.encode(ids[rows], lens[rows])
    m.close()
    assert np.isfinite(full).all()
    np.testing.assert_allclose(np.linalg.norm(full, axis=1), 1.0, rtol=1e-5)
    np.testing.assert_array_equal(full[rows], part)
    cos, err = parity(full[rows], g["embeddings"])
    assert cos >= 0.9999 and err <= 2e-3, f"min cos {cos:.7f}, max abs {err:.3e}"
