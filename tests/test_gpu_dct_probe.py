"""Device DCT sensitivity probe (ntcb_dct_probe) against the reference's own host probe (Decoder::dct_fit_all ->
dct_probe_codes, main.cpp:1002-1030, 1663-1669, run through the reference CPU library) on the same model and
decode buffer: codes equal wherever the gain is not on a code boundary (the reference notes that a CPU and a
--cuda run may differ there), one and two level-0 channels."""
import numpy as np
import pytest

from neural_block_textures_b200 import Trainer
from neural_block_textures_b200.model import LevelSpec, ModelSpec
from oracle.oracle import RefSession, refcpu_available

from .helpers import target_for

pytestmark = pytest.mark.gpu

FLOOR = 14.0 / 64.0


@pytest.mark.parametrize("C", [1, 2])
def test_dct_probe_matches_reference(C, cuda_device):
    if not refcpu_available():
        pytest.skip("reference CPU library not built")
    spec = ModelSpec(64, 64, [LevelSpec(64, 64, C, True), LevelSpec(16, 16, 2)], dct_q=(50,) * C, max_pairs=16,
                     max_batch=256, seed=23 + C)
    tgt = target_for(spec)
    z, p = spec.init_params()
    with Trainer() as tr:
        ok, why = tr.init(spec.model_desc(), z, p, tgt)
        assert ok, why
        codes, gains = tr.dct_probe()
    ref = RefSession(spec, tgt)
    ref.set_model(z, p)
    rc = ref.dct_probe_codes(spec.dct_q)
    assert codes.shape == rc.shape == ((64 // 8) * (64 // 8) * C,)
    assert np.unique(rc).size > 1, "a probe whose codes are all equal tests nothing"
    # code k covers log2(g / floor) / 0.6 in [k - 1/2, k + 1/2)
    t = np.log2(np.maximum(gains.astype(np.float64), FLOOR) / FLOOR) / 0.6
    near = np.abs(np.abs(t - np.floor(t)) - 0.5) < 1e-3
    assert near.mean() < 0.05
    assert np.array_equal(codes[~near], rc[~near])
    assert np.all(np.abs(codes.astype(int) - rc.astype(int)) <= 1)
