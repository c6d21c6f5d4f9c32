"""The tensor-core ES kernels (tcgen05, 3xTF32: population and latent pass) against the oracle's loss_subset and against the
bit-exact packed-FP32 kernel, on every fixed shape (nin 5 / 6 / 8, 3 and 12 outputs), including minibatch
sizes that leave a ragged last 128-row tile and the sigma = 0 case where both signs must agree exactly.

Bars: per-candidate fitness within 1e-5 relative of the oracle (the build's fitness tolerance) and within
2e-6 relative of the exact kernel; the ES loss differences dl = L+ - L- within 1e-3 rms(dl) of the
exact kernel's (the reference's --cuda-check bar for dl, main.cpp:3008-3030)."""
import dataclasses

import numpy as np
import pytest

from neural_block_textures_b200 import Trainer
from oracle.oracle import Oracle

from .helpers import rel_err, spec_named, target_for

pytestmark = pytest.mark.gpu

FIT_RTOL = 1e-5
TC_VS_EXACT = 2e-6
SIGMA = 0.02


def _trainer(spec, tgt):
    z, p = spec.init_params()
    tr = Trainer()
    ok, why = tr.init(spec.model_desc(), z, p, tgt)
    assert ok, why
    return tr, z, p


def _fitness(tr, tensor, it, N, M, sigma=SIGMA):
    tr.set_pop_kernel(tensor)
    assert tr.pop_kernel() == ("tensor" if tensor else "ffma")
    tr.mlp_step(it, sigma, 0.0, N, M)
    lp, lm = tr.debug_last_fitness()
    return lp.copy(), lm.copy(), tr.debug_last_batch().copy()


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg5"])
@pytest.mark.parametrize("M", [1024, 300])
def test_tensor_fitness_matches_oracle_and_exact(name, M, cuda_device):
    spec = dataclasses.replace(spec_named(name), max_pairs=64)
    tgt = target_for(spec)
    tr, z, p = _trainer(spec, tgt)
    N, it = 48, 7
    lp_t, lm_t, b_t = _fitness(tr, True, it, N, M)
    lp_e, lm_e, b_e = _fitness(tr, False, it, N, M)
    assert np.array_equal(b_t, b_e)
    # against the exact kernel
    assert rel_err(lp_t, lp_e) < TC_VS_EXACT and rel_err(lm_t, lm_e) < TC_VS_EXACT
    dl_t, dl_e = lp_t - lm_t, lp_e - lm_e
    assert np.abs(dl_t - dl_e).max() < 1e-3 * np.sqrt(np.mean(dl_e ** 2))
    # against the oracle (the reference's CPU loss_subset on the same batch and noise)
    orc = Oracle(spec, tgt)
    olp, olm = orc.es_fitness(p, z, spec.seed, it, SIGMA, 0, N, b_t)
    assert rel_err(lp_t, olp) < FIT_RTOL and rel_err(lm_t, olm) < FIT_RTOL
    tr.close()


def test_tensor_sigma_zero_signs_agree(cuda_device):
    spec = spec_named("cfg2")
    tr, z, p = _trainer(spec, target_for(spec))
    lp, lm, _ = _fitness(tr, True, 3, 16, 512, sigma=0.0)
    assert np.array_equal(lp, lm)
    assert np.all(lp == lp[0])
    tr.close()


def test_tensor_training_steps_track_exact(cuda_device):
    """Ten ES steps with lr > 0 on each kernel: the weights stay within a small fraction of the Adam step."""
    spec = dataclasses.replace(spec_named("cfg2"), max_pairs=64)
    tgt = target_for(spec)
    res = {}
    for tensor in (True, False):
        tr, z, p = _trainer(spec, tgt)
        tr.set_pop_kernel(tensor)
        for it in range(1, 11):
            tr.mlp_step(it, SIGMA, 0.005, 64, 1024)
        res[tensor] = tr.download_model()[1]
        tr.close()
    # Adam moves each weight by ~lr per step; near-zero gradient components may take the other sign
    d = np.abs(res[True] - res[False])
    assert np.median(d) < 1e-4 * 0.005
    assert np.mean(d > 0.5 * 0.005) < 0.02


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg5"])
def test_tensor_latent_gradient_tracks_exact(name, cuda_device):
    """One latent ES pass (lr 0) per kernel on fresh trainers (same noise step): the tensor-core gradient within
    1e-4 rms of the exact kernel's (the reference's --cuda-check bar against the CPU is 1e-3 rms)."""
    spec = spec_named(name)
    tgt = target_for(spec)
    g = {}
    for tensor in (True, False):
        tr, z, p = _trainer(spec, tgt)
        tr.set_pop_kernel(tensor)
        tr.lat_step(1, 0.05, 0.0, 4)
        g[tensor] = tr.debug_last_zgrad().astype(np.float64)
        tr.close()
    rms = np.sqrt(np.mean(g[False] ** 2))
    assert rms > 0
    assert np.abs(g[True] - g[False]).max() < 1e-4 * rms


@pytest.mark.parametrize("tensor", [True, False])
def test_population_beyond_65535_candidates(tensor, cuda_device):
    """40000 pairs = 80000 candidates (the reference's (16, 2N) grid would overflow gridDim.y at 65536): the
    last pairs' fitness against the oracle on the same batch and noise."""
    N, M, it = 40000, 128, 3
    spec = dataclasses.replace(spec_named("cfg2"), max_pairs=N, max_batch=M)
    tgt = target_for(spec)
    tr, z, p = _trainer(spec, tgt)
    lp, lm, bidx = _fitness(tr, tensor, it, N, M)
    tr.close()
    assert lp.shape == (N,) and np.all(lp > 0) and np.all(lm > 0)
    orc = Oracle(spec, tgt)
    tail = 8
    olp, olm = orc.es_fitness(p, z, spec.seed, it, SIGMA, N - tail, tail, bidx)
    assert rel_err(lp[-tail:], olp) < FIT_RTOL and rel_err(lm[-tail:], olm) < FIT_RTOL


@pytest.mark.parametrize("tensor", [True, False])
@pytest.mark.parametrize("N,M", [(1, 1), (1, 129), (3, 7)])
def test_tiny_populations_and_batches(tensor, N, M, cuda_device):
    """One pair / one row and other sizes below a tile: both kernels against the oracle."""
    spec = dataclasses.replace(spec_named("cfg2"), max_pairs=8)
    tgt = target_for(spec)
    tr, z, p = _trainer(spec, tgt)
    lp, lm, bidx = _fitness(tr, tensor, 5, N, M)
    tr.close()
    assert lp.shape == (N,)
    olp, olm = Oracle(spec, tgt).es_fitness(p, z, spec.seed, 5, SIGMA, 0, N, bidx)
    assert rel_err(lp, olp) < FIT_RTOL and rel_err(lm, olm) < FIT_RTOL


@pytest.mark.parametrize("tensor", [True, False])
def test_single_latent_pair(tensor, cuda_device):
    """K = 1: the latent gradient of one antithetic pair, tensor-core and exact passes against each other."""
    spec = spec_named("cfg5")
    tgt = target_for(spec)
    g = {}
    for t in (tensor, False):
        tr, z, p = _trainer(spec, tgt)
        tr.set_pop_kernel(t)
        tr.lat_step(1, 0.05, 0.0, 1)
        g[t] = tr.debug_last_zgrad().astype(np.float64)
        tr.close()
    rms = np.sqrt(np.mean(g[False] ** 2))
    assert rms > 0 and np.abs(g[tensor] - g[False]).max() < 1e-4 * rms
