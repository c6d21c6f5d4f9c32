"""ntcb_print_stats (the progress print's statistics on the device) against the oracle (oracle/print_stats.py)
and the reference's own host functions (bitrate_stats / mse_of / latent_stats through oracle/ref_shim.cpp), on
the trainer's own model after a few training steps.

Bars: the quantized copy zq exact; the integer 8-bit squared-error sums exact (recovered from the per-texture
figures); bitrate figures within 1e-12 relative; mse figures within 1e-15; latent moments within 1e-6; the
--qat off-grid count exact."""
import numpy as np
import pytest

from neural_block_textures_b200 import Trainer, abi, qat_grid_table
from oracle import print_stats as ps
from oracle.oracle import RefSession, refcpu_available

from .helpers import spec_named, target_for
from .test_print_stats import BITRATE_RTOL, MSE_RTOL, _moved_model, _qes_spec

pytestmark = pytest.mark.gpu


def _trained(spec, tgt, steps=2):
    z, p = _moved_model(spec)
    tr = Trainer()
    ok, why = tr.init(spec.model_desc(), z, p, tgt)
    assert ok, why
    for it in range(1, steps + 1):
        tr.mlp_step(it, 0.02, 0.005, 16, 512)
        tr.lat_step(it, 0.05, 0.01, 2)
    return tr


def _check_mse(spec, tgt, tr, st, zq, ew, eh):
    npe = (ew or spec.W) * (eh or spec.H)
    for img, mse, tex in ((tr.decode_full(), st.mse, st.mse_tex), (tr.decode_full(zq), st.mse_q, st.mse_q_tex)):
        ow, otex, osse = ps.mse_of(spec, tgt, img, ew, eh)
        dtex = np.array(tex[: spec.T])
        assert np.array_equal(np.rint(dtex * 3.0 * npe), osse)
        assert abs(mse - ow) <= MSE_RTOL * ow and np.allclose(dtex, otex, rtol=MSE_RTOL, atol=0)


def _check_bitrate(st, want: dict):
    for k, v in want.items():
        assert abs(getattr(st, k) - v) <= BITRATE_RTOL * max(abs(v), 1e-300), (k, getattr(st, k), v)


@pytest.mark.parametrize("name,qbits,extent", [("cfg2", 8, (0, 0)), ("cfg3", 8, (-3, -5)), ("cfg5", 6, (0, 0)),
                                               ("generic", 8, (-1, 0)), ("cfg1", 12, (0, 0))])
def test_print_stats_vs_oracle_and_reference(name, qbits, extent, cuda_device):
    spec = spec_named(name)
    tgt = target_for(spec)
    tr = _trained(spec, tgt)
    ew = spec.W + extent[0] if extent[0] else 0
    eh = spec.H + extent[1] if extent[1] else 0
    st, zq = tr.print_stats([qbits] * len(spec.levels), ew, eh, want_zq=True)
    z, p = tr.download_model()
    zdec = tr.download_zq()
    assert st.level0_dct == 0
    # oracle
    want, ozq = ps.bitrate_stats(spec, z, zdec, spec.P, [qbits] * len(spec.levels))
    _check_bitrate(st, want)
    assert np.array_equal(zq, ozq)
    _check_mse(spec, tgt, tr, st, zq, ew, eh)
    for l, (L, off) in enumerate(zip(spec.levels, spec.offsets)):
        o = ps.latent_stats(z[off: off + L.size])
        d = (st.lat_mean[l], st.lat_sd[l], st.lat_max[l])
        assert np.allclose(d, o, rtol=1e-6, atol=1e-7), (l, d, o)
    assert st.qat_off_grid == (ps.qat_off_grid(spec, z, qat_grid_table()) if spec.qat_bits else 0)
    # the reference's own host functions on the same model
    if refcpu_available():
        ref = RefSession(spec, tgt)
        ref.set_model(z, p)
        rs, rzq = ref.bitrate_stats(qbits)
        _check_bitrate(st, rs)
        assert np.array_equal(zq, rzq)
        rw, _ = ref.mse_of(tr.decode_full(), ew, eh)
        assert abs(st.mse - rw) <= MSE_RTOL * rw
        for l in range(len(spec.levels)):
            assert np.allclose((st.lat_mean[l], st.lat_sd[l], st.lat_max[l]), ref.latent_stats(l), rtol=1e-6, atol=1e-7)
        ref.close()
    tr.close()


def test_print_stats_qes_live_level(cuda_device):
    """A live --qes level (tables fitted by the reference on the same latent): grid indices from the table, the
    snapped values as the quantized copy, its depth instead of the post-hoc one."""
    if not refcpu_available():
        pytest.skip("oracle/_ref not built")
    spec = _qes_spec()
    tgt = target_for(spec)
    z, p = _moved_model(spec)
    ref = RefSession(spec, tgt)
    ref.set_model(z, p)
    ref.qes_fit_level(1, 6)
    lo, hi, rng, grid = ref.qes_tables(1, 3, 6)
    tr = Trainer()
    ok, why = tr.init(spec.model_desc(), z, p, tgt)
    assert ok, why
    q = abi.QesDesc()
    q.bits[1] = 6
    q.live, q.frozen = 1, 1
    for c in range(3):
        q.lo[1][c], q.hi[1][c], q.range[1][c] = float(lo[c]), float(hi[c]), float(rng[c])
        q.grid_off[1][c] = c * 64
    tr.set_qes(q, np.ascontiguousarray(grid, np.float32))
    st, zq = tr.print_stats([7, 7], 0, 0, want_zq=True)
    assert np.array_equal(tr.download_zq(), ref.zdec())
    rs, rzq = ref.bitrate_stats(7)
    _check_bitrate(st, rs)
    assert np.array_equal(zq, rzq)
    _check_mse(spec, tgt, tr, st, zq, 0, 0)
    ref.close()
    tr.close()


def test_print_stats_rejects_bad_depth(cuda_device):
    spec = spec_named("cfg1")
    tgt = target_for(spec)
    z, p = spec.init_params()
    tr = Trainer()
    ok, why = tr.init(spec.model_desc(), z, p, tgt)
    assert ok, why
    with pytest.raises(ValueError):
        tr.print_stats([17])
    with pytest.raises(ValueError):
        tr.print_stats([0])
    tr.close()


@pytest.mark.parametrize("C", [1, 2])
def test_print_stats_dct_bit_simulator(C, cuda_device):
    """A live DCT-coded level 0: the device's token statistics and entropy sums against the reference's own bit
    simulator (dct_analyze, main.cpp:1080, g_ctx_stats off as in the progress print) on the same symbols and codes:
    raw bits and header exact, order-0 and context bits within 1e-9 (the same code lengths summed per symbol
    instead of per token); the progress figures against the reference's bitrate_stats on that state."""
    if not refcpu_available():
        pytest.skip("reference CPU library not built")
    from neural_block_textures_b200.model import LevelSpec, ModelSpec
    spec = ModelSpec(64, 64, [LevelSpec(64, 64, C, True), LevelSpec(16, 16, 2)], dct_q=(50,) * C, max_pairs=16,
                     max_batch=256, seed=23 + C)
    tgt = target_for(spec)
    z, p = spec.init_params()
    ref = RefSession(spec, tgt)
    ref.set_model(z, p)
    ref.dct_probe_codes(spec.dct_q)          # the reference fits the scale codes, goes live and snaps
    sym, code, step = ref.dct_full_state()
    assert np.count_nonzero(sym) > 0
    nbc = code.size
    d = abi.DctDesc()
    d.live, d.C, d.BW, d.BH, d.N, d.dc_step = 1, C, spec.W // 8, spec.H // 8, 8, 4
    with Trainer() as tr:
        ok, why = tr.init(spec.model_desc(), z, p, tgt)
        assert ok, why
        tr.set_dct(d, code, sym, step)
        st, _ = tr.print_stats([8] * len(spec.levels))
        dsym, dcode = tr.download_dct(nbc)
    assert st.level0_dct == 1
    ref.dct_set_symbols(dsym, dcode)
    raw, h0, ctx, hdr = ref.dct_analyze()
    assert st.dct_bits_raw == raw and st.dct_bits_header == hdr == 96.0 * C
    assert abs(st.dct_bits_h0 - h0) <= 1e-9 * h0 and abs(st.dct_bits_ctx - ctx) <= 1e-9 * ctx
    want, _ = ref.bitrate_stats(8)
    for k in ("bpp_q8", "bpp_q8_ent", "bpp_q8_ctx", "bpp_ctx_level0", "bpp_est", "bits_header"):
        assert abs(getattr(st, k) - want[k]) <= 1e-9 * max(abs(want[k]), 1e-300), (k, getattr(st, k), want[k])
