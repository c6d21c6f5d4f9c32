"""Bounded device waits of the peer exchange, and one process driving two GPUs.

* A peer that never arrives: two processes share one GPU and map each other's exchange buffers (CUDA IPC); only
  rank 0 runs an exchange (ntcb_p2p_barrier with a short poll limit), rank 1 never launches one. Rank 0's wait must
  run out, come back as device error word 2 within a bounded time, and leave the trainer usable. Only one rank ever
  has a waiting kernel in flight, so no two kernels on the GPU wait on each other. The reference has no multi-GPU
  path; on a runtime failure it prints and exits (cuda/ntc_cuda.cu:55-56), which is what the iteration's exchanges
  (the same kernel, the same error word) do at the next synchronising call.
* Two GPUs (skipped on one): the barrier completes on both ranks (error word 0), and trainers on two devices of one
  process both run the tensor-core kernels (their shared-memory opt-ins are per device) and the allocation-free
  entry point on either device."""
import json
import os
import socket
import time
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _barrier_rank(rank, world, port, out_dir, same_gpu, polls):
    import datetime
    import torch
    import torch.distributed as dist
    from neural_block_textures_b200 import Trainer
    from tests.helpers import spec_named, target_for
    dev = 0 if same_gpu else rank
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=datetime.timedelta(seconds=60))
    out = {}
    try:
        spec = spec_named("cfg2")
        z, p = spec.init_params()
        tr = Trainer()
        ok, why = tr.init(spec.model_desc(), z, p, target_for(spec))
        assert ok, why
        h = tr.p2p_export(world, rank, 64, 4, True)
        allh = [None] * world
        dist.all_gather_object(allh, h)
        tr.p2p_import(b"".join(allh), world, rank)
        dist.barrier()
        if same_gpu:
            if rank == 0:           # rank 1 never runs an exchange: rank 0's wait must run out
                t0 = time.perf_counter()
                out["code"] = tr.p2p_barrier(polls)
                out["seconds"] = time.perf_counter() - t0
                tr.mlp_step(1, 0.02, 0.0, 32, 256)       # the trainer still works, and its error word was cleared
                lp, lm = tr.debug_last_fitness()
                out["finite"] = bool(np.all(np.isfinite(lp)) and np.all(np.isfinite(lm)))
        else:
            t0 = time.perf_counter()
            out["code"] = tr.p2p_barrier(polls)
            out["seconds"] = time.perf_counter() - t0
        dist.barrier()
        tr.p2p_release()
        dist.barrier()
        tr.close()
        (Path(out_dir) / f"r{rank}.json").write_text(json.dumps(out))
    finally:
        dist.destroy_process_group()


def _run_ranks(tmp_path, same_gpu, polls):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_barrier_rank, args=(r, 2, port, str(tmp_path), same_gpu, polls)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=240)
    codes = [pr.exitcode for pr in procs]
    for pr in procs:
        if pr.is_alive():
            pr.kill()
    assert codes == [0, 0], codes
    return [json.loads((tmp_path / f"r{r}.json").read_text()) for r in range(2)]


def test_p2p_wait_runs_out_when_peer_never_arrives(tmp_path, cuda_device):
    r0, r1 = _run_ranks(tmp_path, True, 10000)
    assert r0["code"] == 2, r0
    assert r0["seconds"] < 20, r0
    assert r0["finite"], r0
    assert r1 == {}


def test_p2p_barrier_two_gpus(tmp_path, cuda_device):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    r0, r1 = _run_ranks(tmp_path, False, 0)
    assert r0["code"] == 0 and r1["code"] == 0, (r0, r1)


def test_two_devices_one_process(cuda_device):
    """Trainers on devices 0 and 1 in one process run the tensor-core population and latent kernels (each device
    makes its own shared-memory opt-in) with identical results, and the allocation-free entry runs on device 1
    after device 0."""
    import ctypes as C
    import torch
    from neural_block_textures_b200 import Trainer, load_library
    from oracle.oracle import Oracle
    from tests.helpers import spec_named, target_for
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    spec = spec_named("cfg2")
    tgt = target_for(spec)
    z, p = spec.init_params()
    res = []
    trs = []
    for dev in (0, 1):
        torch.cuda.set_device(dev)
        tr = Trainer()
        ok, why = tr.init(spec.model_desc(), z, p, tgt)
        assert ok, why
        trs.append(tr)
    for tr in trs:
        tr.mlp_step(3, 0.02, 0.005, 64, 1024)
        tr.lat_step(3, 0.05, 0.02, 4)
        tr.qat_search()
        res.append(tr.download_model())
    for tr in trs:
        tr.close()
    assert np.array_equal(res[0][0], res[1][0]) and np.array_equal(res[0][1], res[1][1])
    lib = load_library()
    orc = Oracle(spec, tgt)
    bidx = orc.draw_batch(spec.seed, 4, 256)
    feat = np.ascontiguousarray(np.stack([orc.features(z, i % spec.W, i // spec.W) for i in bidx]), np.float32)
    t = np.ascontiguousarray(tgt.reshape(-1, spec.nout)[bidx], np.float32)
    desc = spec.model_desc()
    fits = []
    for dev in (0, 1):
        torch.cuda.set_device(dev)
        fit = np.zeros(16, np.float64)
        why = C.create_string_buffer(256)
        ok = lib.ntcb_es_fitness_noalloc(C.byref(desc), 4, 0.02, 0, 8, p.ctypes.data_as(C.POINTER(C.c_float)),
                                         feat.ctypes.data_as(C.POINTER(C.c_float)), t.ctypes.data_as(C.POINTER(C.c_float)), 256,
                                         fit.ctypes.data_as(C.POINTER(C.c_double)), why, 256)
        assert ok == 1, why.value
        fits.append(fit)
    torch.cuda.set_device(0)
    assert np.array_equal(fits[0], fits[1])
