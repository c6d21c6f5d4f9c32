"""CUDA path (libntc_b200 through its C ABI) against the oracle on identical seeded inputs.

Thresholds: the reference's own --cuda-check bars (main.cpp:2988-3147) — decode < 1e-5 absolute, ES loss
differences < 1e-3 rms(dl), FD < 1e-2 rms, latent gradient < 1e-3 rms(grad), selector search near-tie rule
and 1e-6 relative loss — plus the build's per-candidate fitness bar of 1e-5 relative; minibatch indices
and u32 noise bit-exact.
"""
import numpy as np
import pytest

from neural_block_textures_b200 import Trainer, qat_grid_table
from oracle.oracle import Oracle

from .helpers import ALL_SPECS, active_mask, rel_err, spec_named, target_for

pytestmark = pytest.mark.gpu

FIT_RTOL = 1e-5      # per-candidate fitness L+- relative to the oracle's loss_subset
SIGMA, LAT_SIGMA = 0.02, 0.05


def make(name, cuda_device, **over):
    import dataclasses
    spec = dataclasses.replace(spec_named(name), **over) if over else spec_named(name)
    tgt = target_for(spec)
    z, p = spec.init_params()
    tr = Trainer()
    ok, why = tr.init(spec.model_desc(), z, p, tgt)
    assert ok, why
    return spec, tgt, z, p, tr, Oracle(spec, tgt)


@pytest.mark.parametrize("name", ALL_SPECS)
def test_decode_full(name, cuda_device):
    spec, tgt, z, p, tr, orc = make(name, cuda_device)
    img = tr.decode_full()
    ref = orc.decode_full(p, z)
    assert np.abs(img - ref).max() < 1e-5
    # a host-supplied latent goes through the scratch copy, not the model latent
    z2 = (z * np.float32(0.5)).astype(np.float32)
    assert np.abs(tr.decode_full(z2) - orc.decode_full(p, z2)).max() < 1e-5
    z3, p3 = tr.download_model()
    assert np.array_equal(z3, z) and np.array_equal(p3, p)
    # into caller arrays (pinned host memory, reused every step in bench.py's end-to-end leg)
    import torch
    zo = torch.full((spec.nz,), -1.0, dtype=torch.float32, pin_memory=True).numpy()
    po = torch.full((spec.P,), -1.0, dtype=torch.float32, pin_memory=True).numpy()
    z4, p4 = tr.download_model(zo, po)
    assert z4 is zo and p4 is po and np.array_equal(zo, z) and np.array_equal(po, p)
    with pytest.raises(ValueError):
        tr.download_model(np.zeros(spec.nz, np.float64), po)


@pytest.mark.parametrize("name", ALL_SPECS)
def test_mlp_es_fitness(name, cuda_device):
    spec, tgt, z, p, tr, orc = make(name, cuda_device)
    N, M, it = 24, 512, 7
    tr.mlp_step(it, SIGMA, 0.0, N, M)
    bidx = tr.debug_last_batch()
    assert np.array_equal(bidx, orc.draw_batch(spec.seed, it, M)), "minibatch indices are bit-exact"
    lp, lm = tr.debug_last_fitness()
    olp, olm = orc.es_fitness(p, z, spec.seed, it, SIGMA, 0, N, bidx)
    assert rel_err(lp, olp) < FIT_RTOL and rel_err(lm, olm) < FIT_RTOL
    dl = tr.debug_last_dl()
    odl = olp - olm
    assert np.abs(dl - odl).max() < 1e-3 * np.sqrt(np.mean(odl ** 2))
    bl, ds = tr.mlp_stats()
    assert abs(bl - np.mean(0.5 * (olp + olm))) < 1e-5 * abs(bl)
    z2, p2 = tr.download_model()
    assert np.array_equal(p2, p), "lr 0 leaves the weights unchanged"


@pytest.mark.parametrize("leak", [1.5, -0.25])
def test_leak_outside_unit_interval(leak, cuda_device):
    """A benchmark shape with a slope outside [0, 1] (where max(x, leak x) is not the reference's select) runs
    the runtime-shaped kernels: decode and ES fitness against the oracle."""
    spec, tgt, z, p, tr, orc = make("cfg2", cuda_device, leak=leak)
    assert np.abs(tr.decode_full() - orc.decode_full(p, z)).max() < 1e-5
    N, M, it = 8, 256, 4
    tr.mlp_step(it, SIGMA, 0.0, N, M)
    bidx = tr.debug_last_batch()
    lp, lm = tr.debug_last_fitness()
    olp, olm = orc.es_fitness(p, z, spec.seed, it, SIGMA, 0, N, bidx)
    assert rel_err(lp, olp) < FIT_RTOL and rel_err(lm, olm) < FIT_RTOL
    tr.close()


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "generic"])
def test_mlp_es_step_updates(name, cuda_device):
    """One ES step with lr > 0: gradient (segmented pair sums) and Adam against the oracle's serial ones."""
    spec, tgt, z, p, tr, orc = make(name, cuda_device, max_pairs=320)
    # Adam's first step is lr * g / (|g| + eps): a gradient component within float noise of zero flips the whole
    # step, so this comparison with the reference's update runs on the bit-exact population kernel (the
    # tensor-core kernel's update is checked against it in test_gpu_tensor_pop.py).
    tr.set_pop_kernel(False)
    N, M, it, lr = 300, 256, 3, 0.005
    tr.mlp_step(it, SIGMA, lr, N, M)
    bidx = tr.debug_last_batch()
    olp, olm = orc.es_fitness(p, z, spec.seed, it, SIGMA, 0, N, bidx)
    g = orc.es_grad(spec.seed, it, SIGMA, olp - olm)
    th, _, _ = orc.adam(p, g, np.zeros_like(p), np.zeros_like(p), lr, 1)
    _, p2 = tr.download_model()
    # Adam's first step moves every weight by ~lr * sign(g); the gradient agrees to float rounding
    assert np.abs(p2 - th).max() < 1e-3 * lr + 1e-7


@pytest.mark.parametrize("kernel", ["tensor", "exact"])
@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "generic3"])
def test_mlp_fd(name, kernel, cuda_device):
    """FD step (the stats pair and the 2P candidates in one launch) on either kernel family."""
    spec, tgt, z, p, tr, orc = make(name, cuda_device)
    tr.set_pop_kernel(kernel == "tensor")
    M, it, h = 256, 5, 1e-3
    tr.mlp_step_fd(it, h, 0.0, M)
    bidx = tr.debug_last_batch()
    dl = tr.debug_last_dl()
    assert dl.shape == (spec.P,)
    js = np.unique(np.array([(q * 7919) % spec.P for q in range(24)] + [0, spec.P - 1]))
    odl, ohh = orc.fd_dl(p, z, bidx, h, js)
    rms = np.sqrt(np.mean(dl ** 2))
    # the reference's FD bar (main.cpp:3034): dl ~ 1e-5 of L, so ulp-level output differences (CUDA's expf
    # against the C library's) reach ~1e-3 of rms(dl)
    assert np.abs(dl[js] - odl).max() < 1e-2 * rms
    l0, fdrms = tr.mlp_stats()
    # the unperturbed loss: the exact kernels to rounding, the 3xTF32 tensor kernel within the fitness bar (1e-5)
    assert abs(l0 - orc.loss_subset(p, z, bidx)) < (1e-5 if tr.pop_kernel() == "tensor" else 1e-6) * l0
    assert abs(fdrms - rms) < 1e-12 + 1e-9 * rms


@pytest.mark.parametrize("name", ALL_SPECS)
def test_latent_grad(name, cuda_device):
    spec, tgt, z, p, tr, orc = make(name, cuda_device)
    mask = active_mask(spec)
    if mask == 0:
        pytest.skip("no ES-trained level")
    for K in (4, 3):
        step = 0 if K == 4 else 1
        tr.lat_step(1, LAT_SIGMA, 0.0, K)
        g = tr.debug_last_zgrad()
        og = orc.lat_grad(p, z, spec.seed, step, K, LAT_SIGMA, mask)
        rms = np.sqrt(np.mean(og.astype(np.float64) ** 2))
        assert rms > 0
        assert np.abs(g - og).max() < 1e-3 * rms, f"K={K}"
        if not (mask & 1):
            assert np.all(g[: spec.levels[0].size] == 0.0)


@pytest.mark.parametrize("name", ["cfg2", "cfg3", "cfg5", "generic"])
def test_qat_search(name, cuda_device):
    """The reference's own acceptance rule (main.cpp:3108-3147): differing texels are near-ties both ways."""
    spec, tgt, z, p, tr, orc = make(name, cuda_device)
    tr.qat_search()
    zg, _ = tr.download_model()
    zc = orc.qat_search(p, z, spec.qat_bits, qat_grid_table())
    n0 = spec.levels[0].size
    assert np.array_equal(zg[n0:], z[n0:]), "only level 0 is searched"
    grid = qat_grid_table()
    for c, b in enumerate(spec.qat_bits):
        assert np.isin(zg[:n0].reshape(-1, spec.levels[0].C)[:, c], grid[b, : 1 << b]).all(), "level 0 stays on its grid"
    diff = int(np.sum(zg[:n0] != zc[:n0]))
    ig = orc.decode_full(p, zg)
    ic = orc.decode_full(p, zc)
    cw = np.tile(np.repeat(np.asarray(spec.wts, np.float64), 3), spec.W * spec.H)
    mg = float(np.sum(cw * (ig - tgt).astype(np.float64) ** 2))
    mc = float(np.sum(cw * (ic - tgt).astype(np.float64) ** 2))
    assert abs(mg - mc) <= 1e-6 * mc + 1e-12, f"{diff} values differ and the loss moved"
    assert diff <= max(16, n0 // 200)


def test_noise_device_vs_oracle(cuda_device):
    import ctypes as C
    from neural_block_textures_b200 import load_library
    from oracle.oracle import noise_gauss_block, noise_u32
    lib = load_library()
    n = 4096
    for (seed, stream, step, pair, i0) in [(1, 2, 7, 3, 0), (12345678901, 1, 0, 0, 1 << 33), (2, 3, 99, 0, 17)]:
        g = np.zeros(n, np.float32); u = np.zeros(n, np.uint32)
        lib.ntcb_noise_fill(seed, stream, step, pair, i0, n, g.ctypes.data_as(C.POINTER(C.c_float)),
                            u.ctypes.data_as(C.POINTER(C.c_uint32)))
        ou = np.array([noise_u32(seed, stream, step, pair, i0 + i) for i in range(256)], np.uint32)
        assert np.array_equal(u[:256], ou), "u32 draws are bit-exact host vs device"
        og = noise_gauss_block(seed, stream, step, pair, i0, n)
        ulps = np.abs(g.view(np.int32).astype(np.int64) - og.view(np.int32).astype(np.int64))
        assert ulps.max() <= 4, "gaussians agree with the C library to a few ulps"


def test_noise_device_vs_reference_device(cuda_device):
    """Bit-exact against the reference's own ntc_noise.h compiled for the device by the same nvcc."""
    import ctypes as C
    from pathlib import Path
    from neural_block_textures_b200 import load_library
    so = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libref_noise.so"
    if not so.exists():
        pytest.skip("oracle/_ref/libref_noise.so not built (needs the reference tree at build time)")
    ref = C.CDLL(str(so))
    ref.ref_device_noise.restype = C.c_int
    ref.ref_device_noise.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64, C.c_size_t,
                                     C.POINTER(C.c_float), C.POINTER(C.c_uint32)]
    lib = load_library()
    n = 1 << 16
    for (seed, stream, step, pair, i0) in [(1, 2, 7, 3, 0), (5, 1, 1234, 9, 1 << 20)]:
        g = np.zeros(n, np.float32); u = np.zeros(n, np.uint32)
        rg = np.zeros(n, np.float32); ru = np.zeros(n, np.uint32)
        lib.ntcb_noise_fill(seed, stream, step, pair, i0, n, g.ctypes.data_as(C.POINTER(C.c_float)), u.ctypes.data_as(C.POINTER(C.c_uint32)))
        assert ref.ref_device_noise(seed, stream, step, pair, i0, n, rg.ctypes.data_as(C.POINTER(C.c_float)),
                                    ru.ctypes.data_as(C.POINTER(C.c_uint32))) == 0
        assert np.array_equal(u, ru)
        assert np.array_equal(g.view(np.uint32), rg.view(np.uint32)), "device gaussians bit-identical to the reference's"
