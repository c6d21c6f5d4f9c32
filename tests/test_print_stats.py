"""The progress-print statistics oracle (oracle/print_stats.py) pinned against the reference's own bitrate_stats,
mse_of, latent_stats and qat_index (main.cpp, compiled behind oracle/ref_shim.cpp), on the CPU.

Bars: quantized copy zq and the integer 8-bit squared-error sums exact; bitrate figures within 1e-12 relative and
the mse figures within 1e-15 (the reference is built with -ffast-math, which may reorder its double sums and divide
by reciprocals); latent moments within 1e-6."""
import ctypes as C

import numpy as np
import pytest

from neural_block_textures_b200 import qat_grid_table
from neural_block_textures_b200.model import LevelSpec, ModelSpec
from oracle import print_stats as ps
from oracle.oracle import Oracle, RefSession, refcpu_available

from .helpers import spec_named, target_for

pytestmark = pytest.mark.skipif(not refcpu_available(), reason="oracle/_ref not built (needs the reference tree)")

BITRATE_RTOL = 1e-12
MSE_RTOL = 1e-15


def _moved_model(spec, seed=3):
    """init_params with every continuous level spread out (and a few exact min / max ties)."""
    z, p = spec.init_params()
    rng = np.random.default_rng(seed)
    for l, (L, off) in enumerate(zip(spec.levels, spec.offsets)):
        if l == 0 and spec.qat_bits:
            continue
        z[off: off + L.size] = (rng.standard_normal(L.size) * (0.3 + 0.2 * l)).astype(np.float32)
        z[off + 5] = z[off: off + L.size].max()
    return z, p


def _close(a: dict, b: dict):
    for k in a:
        assert abs(a[k] - b[k]) <= BITRATE_RTOL * max(abs(b[k]), 1e-300), (k, a[k], b[k])


def _qes_spec():
    return ModelSpec(48, 40, [LevelSpec(24, 20, 2), LevelSpec(12, 10, 3)], qes_bits=(0, 6, 0), max_pairs=8,
                     max_batch=256, seed=21)


@pytest.mark.parametrize("name,qbits", [("cfg2", 8), ("cfg2", 5), ("cfg3", 8), ("generic", 7), ("cfg5", 8), ("cfg1", 12)])
def test_bitrate_stats_oracle_vs_reference(name, qbits):
    spec = spec_named(name)
    z, p = _moved_model(spec)
    ref = RefSession(spec, target_for(spec))
    ref.set_model(z, p)
    rs, rzq = ref.bitrate_stats(qbits)
    os_, ozq = ps.bitrate_stats(spec, z, z, spec.P, [qbits] * len(spec.levels))
    _close(os_, rs)
    assert np.array_equal(ozq, rzq)
    ref.close()


def test_bitrate_stats_qes_live_level():
    spec = _qes_spec()
    tgt = target_for(spec)
    z, p = _moved_model(spec)
    ref = RefSession(spec, tgt)
    ref.set_model(z, p)
    ref.qes_fit_level(1, 6)
    zdec = ref.zdec()
    lo, hi, rng, _ = ref.qes_tables(1, 3, 6)
    rs, rzq = ref.bitrate_stats(7)
    os_, ozq = ps.bitrate_stats(spec, z, zdec, spec.P, [7, 7], qes={1: (6, lo, rng)})
    _close(os_, rs)
    assert np.array_equal(ozq, rzq)
    ref.close()


@pytest.mark.parametrize("name", ["cfg2", "cfg3"])
@pytest.mark.parametrize("extent", [(0, 0), (-3, -5)])
def test_mse_of_oracle_vs_reference(name, extent):
    spec = spec_named(name)
    tgt = target_for(spec)
    z, p = _moved_model(spec)
    img = Oracle(spec, tgt).decode_full(p, z)
    # values on 8-bit rounding edges, and outside [0, 1]
    img[::7] = (np.arange(img[::7].size) % 256 + 0.5).astype(np.float32) / np.float32(255.0)
    img[::11] = np.float32(1.25)
    img[::13] = np.float32(-0.5)
    ew = spec.W + extent[0] if extent[0] else 0
    eh = spec.H + extent[1] if extent[1] else 0
    ref = RefSession(spec, tgt)
    rw, rtex = ref.mse_of(img, ew, eh)
    ow, otex, osse = ps.mse_of(spec, tgt, img, ew, eh)
    npe = (ew or spec.W) * (eh or spec.H)
    # the integer squared-error sums are exact; the reference's -ffast-math build may divide by a reciprocal,
    # so the derived doubles agree to a few ulp
    assert np.array_equal(np.rint(rtex * 3.0 * npe), osse)
    assert abs(ow - rw) <= MSE_RTOL * rw and np.allclose(otex, rtex, rtol=MSE_RTOL, atol=0)
    ref.close()


@pytest.mark.parametrize("name", ["cfg2", "generic"])
def test_latent_stats_oracle_vs_reference(name):
    spec = spec_named(name)
    z, p = _moved_model(spec)
    ref = RefSession(spec, target_for(spec))
    ref.set_model(z, p)
    for l, (L, off) in enumerate(zip(spec.levels, spec.offsets)):
        r = ref.latent_stats(l)
        o = ps.latent_stats(z[off: off + L.size])
        assert np.allclose(o, r, rtol=1e-6, atol=0), (l, o, r)
    ref.close()


def test_qat_off_grid_oracle_vs_reference_index():
    spec = spec_named("cfg3")
    z, _ = _moved_model(spec)
    L = spec.levels[0]
    z[3 * L.C] = np.float32(0.123)                      # off the 2-bit grid
    z[10 * L.C + 1] = np.nextafter(np.float32(1.0), np.float32(0.0))
    z[11 * L.C] = np.float32(-1.0)                       # on the grid
    grid = qat_grid_table()
    lib = RefSession(spec, target_for(spec)).lib
    want = 0
    k = C.c_int()
    for i in range(L.size):
        b = spec.qat_bits[i % L.C]
        lib.ref_qat_levels_index(C.c_float(z[i]), b, C.byref(k))
        want += int(grid[b, k.value] != z[i])
    assert want == 2
    assert ps.qat_off_grid(spec, z, grid) == want


def test_quantizer_functions_vs_reference():
    """q8 / qes / qat indices of the oracle against the reference's compiled quantizers on edge values."""
    spec = spec_named("cfg2")
    lib = RefSession(spec, target_for(spec)).lib
    rng = np.random.default_rng(9)
    lo, r, levels = np.float32(-0.7), np.float32(1.3), 255
    v = np.concatenate([rng.uniform(-1, 0.7, 4000).astype(np.float32),
                        lo + (np.arange(256, dtype=np.float32) + np.float32(0.5)) / np.float32(levels) * r])
    got = ps.qes_index(v, lo, r, levels)
    want = [lib.ref_qes_index(C.c_float(x), C.c_float(lo), C.c_float(r), levels) for x in v]
    assert np.array_equal(got, want)
    k = C.c_int()
    for b in (1, 2, 3, 8):
        vv = np.concatenate([rng.uniform(-1.2, 1.2, 500), (np.arange(1 << b) + 0.5) / ((1 << b) - 1) * 2 - 1]).astype(np.float32)
        want = []
        for x in vv:
            lib.ref_qat_levels_index(C.c_float(x), b, C.byref(k))
            want.append(k.value)
        assert np.array_equal(ps.qat_index(vv, b), want), b


@pytest.mark.parametrize("C", [1, 2])
def test_dct_bit_simulator_oracle_vs_reference(C):
    """The oracle's restatement of the DCT bit simulator against the reference's own dct_analyze (through the
    reference CPU library) on a live DCT level fitted by the reference: raw and header bits exact, the entropy
    totals to 1e-12 (code lengths summed per symbol instead of per token)."""
    from neural_block_textures_b200 import dct
    spec = ModelSpec(64, 64, [LevelSpec(64, 64, C, True), LevelSpec(16, 16, 2)], dct_q=(50,) * C, max_pairs=16,
                     max_batch=256, seed=23 + C)
    tgt = target_for(spec)
    z, p = spec.init_params()
    ref = RefSession(spec, tgt)
    ref.set_model(z, p)
    ref.dct_probe_codes(spec.dct_q)
    sym, code, _ = ref.dct_full_state()
    assert np.count_nonzero(sym) > 0
    raw, h0, ctx, hdr = ps.dct_bits(sym, code, C, spec.W // 8, spec.H // 8, 4, dct.zigzag_table())
    rraw, rh0, rctx, rhdr = ref.dct_analyze()
    assert raw == rraw and hdr == rhdr
    assert abs(h0 - rh0) <= 1e-12 * rh0 and abs(ctx - rctx) <= 1e-12 * rctx
