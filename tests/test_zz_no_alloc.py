"""ntcb_es_fitness_noalloc: the ES fitness evaluation for callers that cannot allocate device memory where
they run (a host engine with a fixed device-memory budget, a plugin that may only use memory it is handed).
It keeps its scratch in one static device array instead of trainer buffers; this checks, through the C ABI,
that two calls in a row give the per-pair fitness of the trainer's own evaluation (ntcb_shard_mlp_eval on
the same minibatch) and of the oracle (the reference's loss_subset restated in C) within the fitness tolerance
of the other GPU tests, with sigma = 0 too, and that bad requests come back as 0 with a reason instead of ending
the process. Collected last on purpose (the file name)."""
import ctypes as C

import numpy as np
import pytest

from neural_block_textures_b200 import Trainer, load_library
from oracle.oracle import Oracle

from .helpers import spec_named, target_for

pytestmark = pytest.mark.gpu

FIT_RTOL = 1e-5
_fp = C.POINTER(C.c_float)
_dp = C.POINTER(C.c_double)


def _noalloc(lib, desc, it, sigma, p0, n, w, feat, tgt, M):
    fit = np.zeros(2 * n, np.float64)
    why = C.create_string_buffer(256)
    ok = lib.ntcb_es_fitness_noalloc(C.byref(desc), it, sigma, p0, n, w.ctypes.data_as(_fp), feat.ctypes.data_as(_fp),
                                     tgt.ctypes.data_as(_fp), M, fit.ctypes.data_as(_dp), why, 256)
    return ok, why.value.decode(), fit


def _rel(a, b):
    return float(np.max(np.abs(a - b) / np.abs(b)))


@pytest.mark.parametrize("name", ["cfg2", "cfg3", "generic3"])
def test_noalloc_matches_trainer_and_oracle_twice(name, cuda_device):
    import torch
    lib = load_library()
    spec = spec_named(name)
    tgt_img = target_for(spec)
    z, p = spec.init_params()
    desc = spec.model_desc()
    orc = Oracle(spec, tgt_img)
    with Trainer() as tr:
        ok, why = tr.init(desc, z, p, tgt_img)
        assert ok, why
        N, M = 32, 512
        # two calls in a row (the array keeps the first call's contents), then sigma = 0 (no noise is generated or read)
        for call, (it, sigma, p0, n) in enumerate([(5, 0.02, 0, 32), (6, 0.02, 8, 16), (7, 0.0, 3, 5)]):
            fit_dev = torch.zeros(2 * n, dtype=torch.float64, device="cuda")
            tr.shard_mlp_eval(it, sigma, N, M, p0, p0 + n, fit_dev)
            torch.cuda.synchronize()
            ref = fit_dev.cpu().numpy()
            bidx = tr.debug_last_batch()
            feat = np.ascontiguousarray(np.stack([orc.features(z, i % spec.W, i // spec.W) for i in bidx]), np.float32)
            tgt = np.ascontiguousarray(tgt_img.reshape(-1, spec.nout)[bidx], np.float32)
            ok, why, fit = _noalloc(lib, desc, it, sigma, p0, n, p, feat, tgt, M)
            assert ok == 1, why
            assert _rel(fit, ref) < FIT_RTOL, f"call {call}: against the trainer"
            olp, olm = orc.es_fitness(p, z, spec.seed, it, sigma, p0, n, bidx)
            assert _rel(fit[0::2], olp) < FIT_RTOL and _rel(fit[1::2], olm) < FIT_RTOL, f"call {call}: against the oracle"
            if sigma == 0.0:
                assert np.array_equal(fit[0::2], fit[1::2])


def test_noalloc_refuses_bad_requests_without_exiting(cuda_device):
    lib = load_library()
    spec = spec_named("cfg2")
    desc = spec.model_desc()
    z, p = spec.init_params()
    M, n = 64, 100000
    feat = np.zeros((M, spec.nin), np.float32)
    tgt = np.zeros((M, spec.nout), np.float32)
    ok, why, _ = _noalloc(lib, desc, 1, 0.02, 0, n, p, feat, tgt, M)
    assert ok == 0 and "static maximum" in why
    fit = np.zeros(2, np.float64)
    buf = C.create_string_buffer(256)
    assert lib.ntcb_es_fitness_noalloc(C.byref(desc), 1, 0.02, 0, 1, p.ctypes.data_as(_fp), None, tgt.ctypes.data_as(_fp), M,
                                       fit.ctypes.data_as(_dp), buf, 256) == 0
    assert "null pointer" in buf.value.decode()
    ok, why, _ = _noalloc(lib, desc, 1, 0.02, 0, 0, p, feat, tgt, M)
    assert ok == 0 and "npairs" in why
    # the library still works after the refusals
    ok, why, fit = _noalloc(lib, desc, 1, 0.02, 0, 2, p, np.ones((M, spec.nin), np.float32), np.full((M, spec.nout), 0.5, np.float32), M)
    assert ok == 1, why
    assert np.all(np.isfinite(fit)) and np.all(fit >= 0)
