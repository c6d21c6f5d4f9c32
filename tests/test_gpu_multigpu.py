"""Population / weight (FD) / image / texel-row sharding over NCCL, through both drivers bench.py can use under
torchrun: ShardedES (per-phase entry points around torch.distributed all-gathers) and NativeShardedES (one
ntcb_shard_iteration call per iteration, in-place all-gathers on the library's own NCCL communicator, or its own
peer-memory exchange kernel over CUDA IPC mappings of every rank's exchange buffer). The ranks
must end with the same weights and latent as one GPU running the plain Trainer steps, bit for bit (every per-pair,
per-pixel and per-texel value is computed by the same kernels whichever rank computes it, and the gradient sums
keep their order). The 2-, 4- and 8-rank cases (64 pairs, 2 level-1 texel rows and 8 level-0 rows per rank at 8)
need as many GPUs and are skipped otherwise; the one-rank native cases run on one GPU."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N, M, K, ITERS = 512, 256, 4, 3   # 256 pairs per rank: the segment-aligned ES block exchange


def _spec():
    from neural_block_textures_b200.model import LevelSpec, ModelSpec
    return ModelSpec(64, 64, [LevelSpec(64, 64, 1, True), LevelSpec(16, 16, 2)], qat_bits=(2,), max_pairs=N, max_batch=M, seed=21)


def _target(spec):
    from neural_block_textures_b200 import synth
    return synth.to_target([synth.synth_rgb8(spec.W, spec.H, 9)])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir, driver="python"):
    import datetime
    import torch
    import torch.distributed as dist
    from neural_block_textures_b200 import Trainer
    from neural_block_textures_b200.shard import ShardedES
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        spec = _spec()
        z, p = spec.init_params()
        tr = Trainer()
        ok, why = tr.init(spec.model_desc(), z, p, _target(spec))
        assert ok, why
        stream = torch.cuda.Stream()
        tr.set_stream(stream.cuda_stream)
        L0 = spec.levels[0]
        if driver in ("native", "native_p2p"):
            from neural_block_textures_b200.shard import NativeShardedES
            nat = NativeShardedES(tr, dist, device="cuda", p2p=(N, K, True) if driver == "native_p2p" else None)
            assert nat.p2p == (driver == "native_p2p")
            ok, mx, lx, why = nat.plan(1, N, M, K, True)
            assert ok and mx == 1 and lx == 1, why
            for it in range(1, ITERS + 1):
                nat.iteration(it, 1, 0.02, 0.005, N, M, K, 0.05, 0.02, True)
            nat.iteration(ITERS + 1, 2, 1e-3, 0.005, N, M, 0, 0.0, 0.0, False)
            zz, pp = tr.download_model()
            nat.close()
        else:
            es = ShardedES(tr, dist, N, device="cuda", stream=stream, K=K, image=(spec.W, spec.H), level0=(L0.W, L0.H, L0.C),
                           P=spec.P)
            assert es.block > 0
            for it in range(1, ITERS + 1):
                es.step(it, 0.02, 0.005, M)
                es.lat_step(it, 0.05, 0.02, K)
                es.qat_search()
            es.fd_step(ITERS + 1, 1e-3, 0.005, M)
            zz, pp = tr.download_model()
        np.save(os.path.join(out_dir, f"z{rank}.npy"), zz)
        np.save(os.path.join(out_dir, f"p{rank}.npy"), pp)
        tr.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _one_gpu_reference():
    """Weights and latent after the plain single-GPU steps the sharded runs must reproduce."""
    from neural_block_textures_b200 import Trainer
    spec = _spec()
    z, p = spec.init_params()
    with Trainer() as tr:
        ok, why = tr.init(spec.model_desc(), z, p, _target(spec))
        assert ok, why
        for it in range(1, ITERS + 1):
            tr.mlp_step(it, 0.02, 0.005, N, M)
            tr.lat_step(it, 0.05, 0.02, K)
            tr.qat_search()
        tr.mlp_step_fd(ITERS + 1, 1e-3, 0.005, M)
        z1, p1 = tr.download_model()
    return z, p, z1, p1


def test_native_iteration_one_rank_matches_plain_steps(cuda_device):
    """ntcb_shard_iteration on a one-rank communicator (its all-gathers are identities) runs the same kernels as the
    plain steps; the result must be identical."""
    from neural_block_textures_b200 import Trainer
    from neural_block_textures_b200.trainer import Comm
    z, p, z1, p1 = _one_gpu_reference()
    spec = _spec()
    comm = Comm(Comm.unique_id(), 1, 0)
    try:
        with Trainer() as tr:
            ok, why = tr.init(spec.model_desc(), z, p, _target(spec))
            assert ok, why
            ok, mx, lx, why = tr.shard_iteration_plan(1, 0, 1, N, M, K, True)
            assert ok and mx == 1 and lx == 1, why
            for it in range(1, ITERS + 1):
                tr.shard_iteration(comm, it, 1, 0.02, 0.005, N, M, K, 0.05, 0.02, True)
            tr.shard_iteration(comm, ITERS + 1, 2, 1e-3, 0.005, N, M, 0, 0.0, 0.0, False)
            zz, pp = tr.download_model()
    finally:
        comm.close()
    assert np.array_equal(pp, p1) and np.array_equal(zz, z1)


def test_native_iteration_one_rank_other_exchanges(cuda_device):
    """The other exchange forms on a one-rank communicator, against the plain steps: the fitness-only MLP exchange
    (64 pairs, below the segment-block threshold) and the pixel-row latent exchange (two ES-trained levels), plus
    an FD iteration; both peer-exchange-free paths must reproduce the plain steps bit for bit."""
    from neural_block_textures_b200 import Trainer
    from neural_block_textures_b200.model import LevelSpec, ModelSpec
    from neural_block_textures_b200.trainer import Comm
    spec = ModelSpec(64, 64, [LevelSpec(32, 32, 4), LevelSpec(16, 16, 2)], max_pairs=64, max_batch=M, seed=22)
    tgt = _target(spec)
    n = 64

    def run(native):
        z, p = spec.init_params()
        with Trainer() as tr:
            ok, why = tr.init(spec.model_desc(), z, p, tgt)
            assert ok, why
            if native:
                ok, mx, lx, why = tr.shard_iteration_plan(1, 0, 1, n, M, K, False)
                assert ok and (mx, lx) == (2, 2), (mx, lx, why)
                for it in range(1, ITERS + 1):
                    tr.shard_iteration(comm, it, 1, 0.02, 0.005, n, M, K, 0.05, 0.02, False)
                tr.shard_iteration(comm, ITERS + 1, 2, 1e-3, 0.005, n, M, K, 0.05, 0.02, False)
            else:
                for it in range(1, ITERS + 1):
                    tr.mlp_step(it, 0.02, 0.005, n, M)
                    tr.lat_step(it, 0.05, 0.02, K)
                tr.mlp_step_fd(ITERS + 1, 1e-3, 0.005, M)
                tr.lat_step(ITERS + 1, 0.05, 0.02, K)
            return tr.download_model()

    comm = Comm(Comm.unique_id(), 1, 0)
    try:
        z1, p1 = run(False)
        zn, pn = run(True)
    finally:
        comm.close()
    assert np.array_equal(pn, p1) and np.array_equal(zn, z1)


def test_native_iteration_plan_refusals(cuda_device):
    """The plan names the exchange per phase and refuses ranks that cannot split the work evenly."""
    from neural_block_textures_b200 import Trainer
    spec = _spec()
    z, p = spec.init_params()
    with Trainer() as tr:
        ok, why = tr.init(spec.model_desc(), z, p, _target(spec))
        assert ok, why
        ok, mx, lx, _ = tr.shard_iteration_plan(2, 1, 1, N, M, K, True)
        assert ok and (mx, lx) == (1, 1)
        ok, mx, _, _ = tr.shard_iteration_plan(2, 0, 1, 96, M, K, True)      # 48 pairs per rank: fitness-only exchange
        assert ok and mx == 2
        ok, _, _, why = tr.shard_iteration_plan(3, 0, 1, N, M, K, True)      # 512 pairs over 3 ranks
        assert not ok and "split evenly" in why
        ok, _, _, why = tr.shard_iteration_plan(2, 0, 1, N, 10 * M, K, True)  # minibatch above the init size
        assert not ok and "minibatch" in why


@pytest.mark.parametrize("driver,world", [("python", 2), ("native", 2), ("native_p2p", 2), ("native_p2p", 4), ("native_p2p", 8)])
def test_sharding_matches_one_gpu(tmp_path, cuda_device, driver, world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, str(tmp_path), driver)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=300)
        assert pr.exitcode == 0
    z, p, z1, p1 = _one_gpu_reference()
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"p{r}.npy"), p1), f"rank {r} weights"
        assert np.array_equal(np.load(tmp_path / f"z{r}.npy"), z1), f"rank {r} latent"
    assert not np.array_equal(p1, p)
