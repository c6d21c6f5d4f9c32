"""Parity at the benchmark configurations' own shapes and sizes, through the C ABI.

* --dct-shadow-pull (k_shadow_pull + re-snap, cuda/ntc_cuda.cu:978-988; host form main.cpp:4142-4146) on a live
  DCT-coded level 0, against the reference's own host code (oracle/_ref, ref_dct_shadow_pull) on the same state:
  shadow latent, snapped plane, symbols and scale codes bit for bit, with the rate term off and with config 4's
  default --dct-lambda recipe (0.5 at q 50, truncation on, lambda-lo 0.25).
* Per-candidate fitness at config 2's and config 5's full sizes (512^2 and 2048^2 images, M = 4096, 4096 and 16384
  pairs) on the default tensor-core kernel and on the exact kernel, against the oracle's loss_subset restatement
  (main.cpp:1739-1750, 1836-1861) on a sample of the pairs spread over the population: within 1e-5 relative.
"""
import numpy as np
import pytest

from neural_block_textures_b200 import Trainer, abi, model
from oracle.oracle import Oracle, RefSession, refcpu_available

from .helpers import target_for

pytestmark = pytest.mark.gpu

FIT_RTOL = 1e-5


def _desc(fields: dict) -> abi.DctDesc:
    d = abi.DctDesc()
    for k, v in fields.items():
        if k == "lam_t16":
            for i in range(16):
                d.lam_t16[i] = float(v[i])
        else:
            setattr(d, k, v)
    return d


@pytest.mark.parametrize("lam", [0.0, 0.5])
def test_shadow_pull_matches_reference(lam, cuda_device):
    if not refcpu_available():
        pytest.skip("reference CPU library not built")
    from neural_block_textures_b200.model import LevelSpec, ModelSpec
    spec = ModelSpec(128, 128, [LevelSpec(128, 128, 1, True), LevelSpec(32, 32, 2)], dct_q=(50,), max_pairs=16, max_batch=256, seed=41)
    tgt = target_for(spec)
    z, p = spec.init_params()
    ref = RefSession(spec, tgt)
    ref.set_model(z, p)
    ref.dct_probe_codes(spec.dct_q, lam=lam, rate_es=lam > 0, rate_trunc=lam > 0, lambda_lo=0.25 if lam > 0 else 0.0)
    sym, code, step = ref.dct_full_state()
    zr0, _ = ref.get_model()
    nbc = code.size
    n0 = spec.levels[0].size
    with Trainer() as tr:
        ok, why = tr.init(spec.model_desc(), zr0, p, tgt)
        assert ok, why
        tr.set_dct(_desc(ref.dct_desc_fields()), code, sym, step)
        assert np.array_equal(tr.download_zq()[:n0].view(np.uint32), ref.zdec()[:n0].view(np.uint32)), "plane after set_dct"
        for k, f in enumerate((0.01, 0.01, 0.3, 1.0)):
            tr.shadow_pull(0, n0, f)
            ref.dct_shadow_pull(f)
            zd, _ = tr.download_model()
            zr, _ = ref.get_model()
            assert np.array_equal(zd.view(np.uint32), zr.view(np.uint32)), f"pull {k}: shadow latent"
            assert np.array_equal(tr.download_zq()[:n0].view(np.uint32), ref.zdec()[:n0].view(np.uint32)), f"pull {k}: snapped plane"
            dsym, dcode = tr.download_dct(nbc)
            rsym, rcode, _ = ref.dct_full_state()
            assert np.array_equal(dsym, rsym) and np.array_equal(dcode, rcode), f"pull {k}: symbols / codes"
    ref.close()


def test_dct_level_at_config4_size(cuda_device):
    """Config 4's DCT-coded level 0 at its own size (1024 x 1024, q 50, the default --dct-lambda recipe: 0.5 with
    truncation and the ES rate term, lambda-lo 0.25): the reference fits the scale codes and snaps on the host, the
    device rebuilds the plane from the reference's symbols, runs latent ES steps with the rate term and the snap after
    each, and one shadow pull; then pulls both sides once more from the same state and compares shadow, plane, symbols
    and codes bit for bit."""
    if not refcpu_available():
        pytest.skip("reference CPU library not built")
    from neural_block_textures_b200 import dct
    cfg = model.config(4)
    spec = cfg.spec
    tgt = cfg.target()
    z, p = spec.init_params()
    ref = RefSession(spec, tgt)
    ref.set_model(z, p)
    lam = dct.lambda_recipe(list(spec.dct_q))
    ref.dct_probe_codes(spec.dct_q, lam=lam, rate_es=True, rate_trunc=True, lambda_lo=0.25)
    sym, code, step = ref.dct_full_state()
    zr0, _ = ref.get_model()
    n0 = spec.levels[0].size
    with Trainer() as tr:
        ok, why = tr.init(spec.model_desc(), zr0, p, tgt)
        assert ok, why
        d = _desc(ref.dct_desc_fields())
        tr.set_dct(d, code, sym, step)
        assert np.array_equal(tr.download_zq()[:n0].view(np.uint32), ref.zdec()[:n0].view(np.uint32)), "plane after set_dct"
        for it in range(1, 4):                    # latent ES with the rate term, snap after each step, shadow pull
            tr.lat_step(it, cfg.lat_sigma, cfg.lat_lr, cfg.lat_pairs)
            tr.shadow_pull(0, n0, 0.01)
        rate = tr.download_dct_rate(code.size)
        assert rate["evals"] > 0 and np.all(rate["bits"] >= 0)
        zd, pd = tr.download_model()
        dsym, dcode = tr.download_dct(code.size)
        # the same pull from the device's state on both sides
        ref.set_model(zd, pd)
        ref.dct_set_symbols(dsym, dcode)
        ref.dct_shadow_pull(0.0)                  # re-snap the host copy from the device's shadow
        tr.shadow_pull(0, n0, 0.0)
        assert np.array_equal(tr.download_zq()[:n0].view(np.uint32), ref.zdec()[:n0].view(np.uint32)), "re-snapped plane"
        tr.shadow_pull(0, n0, 0.01)
        ref.dct_shadow_pull(0.01)
        zd2, _ = tr.download_model()
        zr2, _ = ref.get_model()
        assert np.array_equal(zd2.view(np.uint32), zr2.view(np.uint32)), "shadow after the pull"
        assert np.array_equal(tr.download_zq()[:n0].view(np.uint32), ref.zdec()[:n0].view(np.uint32)), "plane after the pull"
        dsym, dcode = tr.download_dct(code.size)
        rsym, rcode, _ = ref.dct_full_state()
        assert np.array_equal(dsym, rsym) and np.array_equal(dcode, rcode), "symbols / codes after the pull"
    ref.close()


def _sample_pairs(N: int, n: int) -> list[int]:
    return sorted(set(int(x) for x in np.linspace(0, N - 1, n)))


@pytest.mark.parametrize("cfg_no", [2, 5])
@pytest.mark.parametrize("kernel", ["tensor", "ffma"])
def test_fitness_at_full_size(cfg_no, kernel, cuda_device):
    cfg = model.config(cfg_no)
    spec = cfg.spec
    tgt = cfg.target()
    z, p = spec.init_params()
    orc = Oracle(spec, tgt)
    N, M, it = cfg.pairs, cfg.batch, 3
    with Trainer() as tr:
        ok, why = tr.init(spec.model_desc(), z, p, tgt)
        assert ok, why
        tr.set_pop_kernel(kernel == "tensor")
        tr.mlp_step(it, cfg.mlp_sigma, 0.0, N, M)
        bidx = tr.debug_last_batch()
        lp, lm = tr.debug_last_fitness()
    assert np.array_equal(bidx, orc.draw_batch(spec.seed, it, M))
    assert lp.size == N and np.all(np.isfinite(lp)) and np.all(np.isfinite(lm))
    for i in _sample_pairs(N, 24):
        olp, olm = orc.es_fitness(p, z, spec.seed, it, cfg.mlp_sigma, i, 1, bidx)
        assert abs(lp[i] - olp[0]) <= FIT_RTOL * olp[0], (i, lp[i], olp[0])
        assert abs(lm[i] - olm[0]) <= FIT_RTOL * olm[0], (i, lm[i], olm[0])
