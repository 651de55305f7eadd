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
