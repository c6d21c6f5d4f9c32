"""The N > 1 host logic on CPU: two gloo ranks shard the ES population with ShardedES (the code bench.py
runs over NCCL on GPUs), all-gather the per-pair fitness and apply identical updates. The per-rank
evaluator here is the oracle (test infrastructure standing in for the GPU kernels); the test checks the
pair split, the gather order and that every rank ends with the single-process weights, bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from neural_block_textures_b200.shard import ShardedES, padded_range, pair_range

from .helpers import spec_named, target_for

N, M, SIGMA, LR, STEPS = 8, 128, 0.02, 0.005, 2


class OracleEvaluator:
    """shard_mlp_eval / shard_mlp_apply with the libntc_b200 contract, computed by the oracle on CPU."""

    def __init__(self, name):
        from oracle.oracle import Oracle
        self.spec = spec_named(name)
        self.z, self.p = self.spec.init_params()
        self.orc = Oracle(self.spec, target_for(self.spec))
        self.m = np.zeros_like(self.p); self.v = np.zeros_like(self.p); self.t = 0

    def shard_mlp_eval(self, it, sigma, N_, M_, p0, p1, fit):
        idx = self.orc.draw_batch(self.spec.seed, it, M_)
        lp, lm = self.orc.es_fitness(self.p, self.z, self.spec.seed, it, sigma, p0, p1 - p0, idx)
        fit[0::2] = torch.from_numpy(lp); fit[1::2] = torch.from_numpy(lm)

    def shard_mlp_apply(self, it, sigma, lr, N_, M_, fit_all):
        f = fit_all.numpy()
        g = self.orc.es_grad(self.spec.seed, it, sigma, f[0::2] - f[1::2])
        self.t += 1
        self.p, self.m, self.v = self.orc.adam(self.p, g, self.m, self.v, lr, self.t)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ev = OracleEvaluator("cfg2")
        es = ShardedES(ev, dist, N, device="cpu")
        for it in range(1, STEPS + 1):
            es.step(it, SIGMA, LR, M)
        np.save(os.path.join(out_dir, f"p{rank}.npy"), ev.p)
    finally:
        dist.destroy_process_group()


class PlumbingTrainer:
    """Writes known values into its own rows / texel rows and records what the exchange delivered."""
    W, H, LW, LH, LC, K, P = 12, 8, 6, 4, 2, 3, 11

    def shard_lat_eval(self, sigma, K, r0, r1, block):
        n = (r1 - r0) * self.W
        for k in range(K):
            for p in range(r0 * self.W, r1 * self.W):
                block[k * n + p - r0 * self.W] = 1000.0 * k + p

    def shard_lat_apply(self, it, sigma, lr, K, blocks, rows_per_block):
        # back to [K][W * H] planes: block b holds rows [b R, (b + 1) R) of every plane
        n = rows_per_block * self.W
        b = blocks.reshape(-1, K, n)
        self.dpix = b.permute(1, 0, 2).reshape(K, -1).clone()

    def shard_qat(self, t0, t1, l0):
        n = self.LW * self.LC
        for i in range(t0 * n, t1 * n):
            l0[i] = -1.0 - i

    def shard_qat_apply(self, l0_all):
        self.l0 = l0_all.clone()

    def shard_es_block_bytes(self, N, p0, p1):
        n = p1 - p0
        return (16 * n + 4 * (n // 64) * self.P + 15) // 16 * 16

    def shard_mlp_eval_grad(self, it, sigma, N, M, p0, p1, block):
        # fitness doubles: (10 i + 1, 10 i + 2) per pair i; segment floats: 100 seg + k
        n = p1 - p0
        f = block[: 16 * n].view(torch.float64)
        for i in range(p0, p1):
            f[2 * (i - p0)] = 10.0 * i + 1.0
            f[2 * (i - p0) + 1] = 10.0 * i + 2.0
        g = block[16 * n:16 * n + 4 * (n // 64) * self.P].view(torch.float32)
        for sg in range(n // 64):
            for k in range(self.P):
                g[sg * self.P + k] = 100.0 * (p0 // 64 + sg) + k

    def shard_mlp_apply_grad(self, it, sigma, lr, N, M, blocks, world):
        self.es_blocks = blocks.clone()

    def shard_fd_eval(self, it, h, M, j0, j1, fit):
        for j in range(j0, j1):
            fit[2 * (j - j0)] = 10.0 * j + 1.0
            fit[2 * (j - j0) + 1] = 10.0 * j + 2.0

    def shard_fd_apply(self, h, lr, fit_all):
        self.fd = fit_all[: 2 * self.P].clone()


def _plumbing_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t = PlumbingTrainer()
        es = ShardedES(t, dist, 4, device="cpu", K=t.K, image=(t.W, t.H), level0=(t.LW, t.LH, t.LC), P=t.P)
        es.lat_step(1, 0.05, 0.0, t.K)
        es.qat_search()
        es.fd_step(1, 1e-3, 0.0, 64)
        np.save(os.path.join(out_dir, f"f{rank}.npy"), t.fd.numpy())
        es2 = ShardedES(t, dist, 256, device="cpu")       # 128 pairs per rank: the segment-aligned block exchange
        assert es2.block > 0
        es2.step(1, 0.02, 0.0, 64)
        np.save(os.path.join(out_dir, f"b{rank}.npy"), t.es_blocks.numpy())
        np.save(os.path.join(out_dir, f"d{rank}.npy"), t.dpix.numpy())
        np.save(os.path.join(out_dir, f"l{rank}.npy"), t.l0.numpy())
    finally:
        dist.destroy_process_group()


def test_latent_qat_fd_sharding_plumbing(tmp_path):
    """Two gloo ranks: each fills only its own image rows / level-0 texel rows / FD weights (P = 11, uneven) /
    ES block (fitness + gradient segments + padding to 16 bytes); after the all-gathers every rank holds the whole arrays in order."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_plumbing_main, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    T = PlumbingTrainer
    want_d = np.array([[1000.0 * k + p for p in range(T.W * T.H)] for k in range(T.K)], np.float32)
    want_l = np.array([-1.0 - i for i in range(T.LW * T.LH * T.LC)], np.float32)
    want_f = np.array([10.0 * j + 1.0 + s for j in range(T.P) for s in range(2)])
    n = 128
    want_b = []
    for r in range(2):
        want_b.append(np.array([10.0 * i + 1.0 + s for i in range(r * n, (r + 1) * n) for s in range(2)]).view(np.uint8))
        want_b.append(np.array([100.0 * (r * n // 64 + sg) + k for sg in range(n // 64) for k in range(T.P)], np.float32).view(np.uint8))
        want_b.append(np.zeros((-(16 * n + 4 * (n // 64) * T.P)) % 16, np.uint8))   # the block's padding to 16 bytes
    want_b = np.concatenate(want_b)
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"d{r}.npy"), want_d)
        assert np.array_equal(np.load(tmp_path / f"l{r}.npy"), want_l)
        assert np.array_equal(np.load(tmp_path / f"f{r}.npy"), want_f)
        assert np.array_equal(np.load(tmp_path / f"b{r}.npy"), want_b)


def test_padded_range():
    assert [padded_range(11, 2, r) for r in range(2)] == [(0, 6, 6), (6, 11, 6)]
    assert [padded_range(10, 8, r)[:2] for r in range(8)] == [(0, 2), (2, 4), (4, 6), (6, 8), (8, 10), (10, 10), (10, 10), (10, 10)]


def test_pair_range():
    assert [pair_range(16, 4, r) for r in range(4)] == [(0, 4), (4, 8), (8, 12), (12, 16)]
    with pytest.raises(ValueError):
        pair_range(10, 4, 0)


def test_two_gloo_ranks_match_single_process(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    p0, p1 = np.load(tmp_path / "p0.npy"), np.load(tmp_path / "p1.npy")
    assert np.array_equal(p0, p1), "replicas stay bit-identical"
    ev = OracleEvaluator("cfg2")
    for it in range(1, STEPS + 1):
        fit = torch.zeros(2 * N, dtype=torch.float64)
        ev.shard_mlp_eval(it, SIGMA, N, M, 0, N, fit)
        ev.shard_mlp_apply(it, SIGMA, LR, N, M, fit)
    assert np.array_equal(p0, ev.p), "sharded == single process"
    assert not np.array_equal(p0, spec_named("cfg2").init_params()[1])


class RowsTrainer:
    """The texel-row latent exchange: each rank fills its own rows of a 12 x 8 x 2 level; install records the level."""
    LW, LH, LC, K = 12, 8, 2, 3

    def shard_lat_plan(self, world, rank):
        ta, tb = rank * self.LH // world, (rank + 1) * self.LH // world
        return (1, ta, tb, 0, 0, (tb - ta) * self.LW * self.LC)

    def shard_lat_step_rows(self, it, sigma, lr, K, world, rank, zblock):
        _, ta, tb, _, _, n = self.shard_lat_plan(world, rank)
        base = ta * self.LW * self.LC
        for i in range(n):
            zblock[i] = 0.5 * (base + i)

    def shard_lat_install(self, level, level_all):
        self.level = (level, level_all.clone())


def _rows_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t = RowsTrainer()
        es = ShardedES(t, dist, 4, device="cpu", K=t.K, image=(16, 16))
        assert es.lat_rows is not None
        es.lat_step(1, 0.05, 0.0, t.K)
        assert t.level[0] == 1
        np.save(os.path.join(out_dir, f"z{rank}.npy"), t.level[1].numpy())
    finally:
        dist.destroy_process_group()


def test_latent_texel_row_sharding_plumbing(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rows_main, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    T = RowsTrainer
    want = np.array([0.5 * i for i in range(T.LW * T.LH * T.LC)], np.float32)
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"z{r}.npy"), want)


# ---- NativeShardedES set-up and teardown (the host side of ntcb_comm_* / ntcb_p2p_*) with stand-ins for the
# library's communicator and trainer, so the hand-over of the NCCL id and the IPC handles runs on two gloo ranks.
class FakeComm:
    def __init__(self, uid, world, rank):
        self.uid, self.world, self.rank, self.closed = uid, world, rank, False

    @staticmethod
    def unique_id():
        return bytes(range(128))

    def close(self):
        self.closed = True


class FakeP2PTrainer:
    def __init__(self, fail_export=False):
        self.log = []
        self.fail_export = fail_export

    def p2p_export(self, world, rank, N, K, qat):
        self.log.append(("export", world, rank, N, K, qat))
        if self.fail_export:
            raise RuntimeError("ntcb_p2p_export: cudaIpcGetMemHandle failed")
        return bytes([rank + 1]) * 64

    def p2p_import(self, handles, world, rank):
        self.log.append(("import", world, rank))
        self.handles = handles

    def p2p_release(self):
        self.log.append(("release",))


def _native_setup_main(rank, world, port, out_dir):
    from neural_block_textures_b200.shard import NativeShardedES
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tr = FakeP2PTrainer()
        nat = NativeShardedES(tr, dist, device="cpu", p2p=(64, 4, True), comm_cls=FakeComm)
        comm = nat.comm
        nat.close()
        np.save(os.path.join(out_dir, f"uid{rank}.npy"), np.frombuffer(comm.uid, np.uint8))
        np.save(os.path.join(out_dir, f"handles{rank}.npy"), np.frombuffer(tr.handles, np.uint8))
        with open(os.path.join(out_dir, f"log{rank}.txt"), "w") as f:
            f.write(repr(tr.log) + "\n" + repr((comm.world, comm.rank, comm.closed, nat.p2p)))
    finally:
        dist.destroy_process_group()


def test_native_driver_setup_two_ranks(tmp_path):
    """Rank 0's NCCL id reaches every rank unchanged; the IPC handles come back concatenated in rank order;
    close() releases the peer mappings on every rank before the communicator goes."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_native_setup_main, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0
    want = bytes([1]) * 64 + bytes([2]) * 64
    for r in range(2):
        assert np.load(tmp_path / f"uid{r}.npy").tobytes() == bytes(range(128))
        assert np.load(tmp_path / f"handles{r}.npy").tobytes() == want
        log, state = (tmp_path / f"log{r}.txt").read_text().splitlines()
        assert log == repr([("export", 2, r, 64, 4, True), ("import", 2, r), ("release",)])
        assert state == repr((2, r, True, False))


def _native_fallback_main(rank, world, port, out_dir):
    from neural_block_textures_b200.shard import NativeShardedES
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tr = FakeP2PTrainer(fail_export=(rank == 1))
        nat = NativeShardedES(tr, dist, device="cpu", p2p=(64, 4, True), comm_cls=FakeComm)
        with open(os.path.join(out_dir, f"fb{rank}.txt"), "w") as f:
            f.write(repr(tr.log) + "\n" + repr((nat.p2p, bool(nat.p2p_why))))
        nat.close()
    finally:
        dist.destroy_process_group()


def test_native_driver_peer_exchange_all_or_none(tmp_path):
    """When one rank cannot set up the peer exchange, no rank uses it (all stay on NCCL) and nobody waits."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_native_fallback_main, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0
    for r in range(2):
        log, state = (tmp_path / f"fb{r}.txt").read_text().splitlines()
        assert state == repr((False, True))
        assert "import" not in log
