"""Sharding one ES training iteration over G ranks (one process and one GPU per rank).

* MLP ES step — the population: rank r evaluates the antithetic pairs [r N / G, (r + 1) N / G), regenerating
  their noise from the counter (no noise crosses the wire). When its range is aligned to the 64-pair gradient
  segments it also sums its own segments of the ES gradient and contributes one block: 2 doubles per pair
  (L+, L-) and P floats per segment; otherwise just the fitness. One all-gather gives every rank all blocks in
  pair order; each rank runs the identical segment sum (or full gradient) and Adam, so the weight replicas
  stay bit-identical without exchanging weights.
* Latent ES step — the image: rank r evaluates the K pairs' per-pixel loss differences for image rows
  [r H / G, (r + 1) H / G) into its block [K][rows W]; one all-gather of the blocks (rank order = row order)
  gives every rank all K planes, from which each rank runs the identical footprint gathers, Adam and snap.
* FD step — the weights: rank r evaluates the central differences of weights [r B, min((r + 1) B, P)) with
  B = ceil(P / G) (every rank also evaluates the unperturbed stats pair); one all-gather of the padded
  [G][B] fitness pairs leaves all P weights' (L+, L-) in weight order at the front, and every rank runs the
  identical FD gradient and Adam.
* Latent ES step, texel rows (one ES-trained level, no qes / DCT): rank r owns texel rows [r LH / G, (r + 1)
  LH / G) of the level, evaluates the pixel rows their footprints cover, gathers and Adam-updates only its own
  texels; one all-gather of the updated rows installs the whole level everywhere. This replaces the per-pixel
  planes (K W H floats) on the wire by the level (LW LH C floats) and shards the gather and Adam too.
* Selector search — level-0 texel rows: rank r searches rows [r LH / G, (r + 1) LH / G) (texels are
  independent); one all-gather of the level installs every rank's result everywhere.

The exchanges run over NCCL (NVLink) on GPUs, over gloo in the CPU tests.
"""
from __future__ import annotations

import contextlib


def pair_range(N: int, world: int, rank: int) -> tuple[int, int]:
    return even_range(N, world, rank, "pairs")


def padded_range(n: int, world: int, rank: int) -> tuple[int, int, int]:
    """[begin, end) of rank's block of ceil(n / world) items (the last blocks may be short or empty), and the
    block size. Blocks are gathered at a stride of the block size, so the n items come out in order at the front."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    per = -(-n // world)
    return min(rank * per, n), min((rank + 1) * per, n), per


def even_range(n: int, world: int, rank: int, what: str = "items") -> tuple[int, int]:
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    if n % world:
        raise ValueError(f"{n} {what} do not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


class ShardedES:
    """Drives a trainer's ntcb_shard_* entry points around the all-gathers.

    `trainer` is a neural_block_textures_b200.Trainer (or any object with the same methods); `dist` is
    torch.distributed with an initialised process group; `device` is where the exchange buffers live (the
    trainer's GPU, or "cpu" for a gloo group); `stream` (optional) is the CUDA stream the trainer launches on.
    `image` = (W, H) and `level0` = (LW, LH, LC) enable the sharded latent step and selector search; `P` (the
    weight count) enables the sharded FD step."""

    def __init__(self, trainer, dist, N: int, device="cuda", stream=None, K: int = 0, image=None, level0=None, P: int = 0):
        import torch
        self.t, self.dist, self.N = trainer, dist, N
        self.world, self.rank = dist.get_world_size(), dist.get_rank()
        self.p0, self.p1 = pair_range(N, self.world, self.rank)
        per = self.p1 - self.p0
        self.fit_local = torch.zeros(2 * per, dtype=torch.float64, device=device)
        self.fit_all = torch.zeros(2 * N, dtype=torch.float64, device=device)
        self.block = -1
        if hasattr(trainer, "shard_es_block_bytes"):
            self.block = trainer.shard_es_block_bytes(N, self.p0, self.p1)
        if self.block > 0:
            self.blk_local = torch.zeros(self.block, dtype=torch.uint8, device=device)
            self.blk_all = torch.zeros(self.block * self.world, dtype=torch.uint8, device=device)
        self.stream = stream
        self.dpix = None
        if image is not None and K > 0:
            W, H = image
            self.W = W
            self.r0, self.r1 = even_range(H, self.world, self.rank, "image rows")
            self.rows = self.r1 - self.r0
            self.dblock = torch.zeros(K * self.rows * W, dtype=torch.float32, device=device)
            self.dpix = torch.zeros(self.world * K * self.rows * W, dtype=torch.float32, device=device)
            self.K = K
        self.lat_rows = None
        if image is not None and K > 0 and hasattr(trainer, "shard_lat_plan"):
            plan = trainer.shard_lat_plan(self.world, self.rank)
            if plan is not None:
                self.lat_rows = plan
                n = plan[5]
                self.zblock = torch.zeros(n, dtype=torch.float32, device=device)
                self.zlevel = torch.zeros(n * self.world, dtype=torch.float32, device=device)
        self.l0 = None
        if level0 is not None:
            LW, LH, LC = level0
            self.tr0, self.tr1 = even_range(LH, self.world, self.rank, "level-0 texel rows")
            self.row_floats = LW * LC
            self.l0 = torch.zeros(LW * LH * LC, dtype=torch.float32, device=device)

        self.fd_local = None
        if P > 0:
            self.P = P
            self.j0, self.j1, per = padded_range(P, self.world, self.rank)
            self.fd_local = torch.zeros(2 * per, dtype=torch.float64, device=device)
            self.fd_all = torch.zeros(2 * per * self.world, dtype=torch.float64, device=device)

    def _ctx(self):
        import torch
        return torch.cuda.stream(self.stream) if self.stream is not None else contextlib.nullcontext()

    def step(self, it: int, sigma: float, lr: float, M: int) -> None:
        """One MLP ES step (mlp_step)."""
        if self.block > 0:
            self.t.shard_mlp_eval_grad(it, sigma, self.N, M, self.p0, self.p1, self.blk_local)
            with self._ctx():
                self.dist.all_gather_into_tensor(self.blk_all, self.blk_local)
            self.t.shard_mlp_apply_grad(it, sigma, lr, self.N, M, self.blk_all, self.world)
            return
        self.t.shard_mlp_eval(it, sigma, self.N, M, self.p0, self.p1, self.fit_local)
        with self._ctx():
            self.dist.all_gather_into_tensor(self.fit_all, self.fit_local)
        self.t.shard_mlp_apply(it, sigma, lr, self.N, M, self.fit_all)

    def fd_step(self, it: int, h: float, lr: float, M: int) -> None:
        """One FD step (mlp_step_fd)."""
        assert self.fd_local is not None
        self.t.shard_fd_eval(it, h, M, self.j0, self.j1, self.fd_local)
        with self._ctx():
            self.dist.all_gather_into_tensor(self.fd_all, self.fd_local)
        self.t.shard_fd_apply(h, lr, self.fd_all)

    def lat_step(self, it: int, sigma: float, lr: float, K: int) -> None:
        """One latent ES step (lat_step)."""
        assert self.dpix is not None and K == self.K
        if self.lat_rows is not None:
            self.t.shard_lat_step_rows(it, sigma, lr, K, self.world, self.rank, self.zblock)
            with self._ctx():
                self.dist.all_gather_into_tensor(self.zlevel, self.zblock)
            self.t.shard_lat_install(self.lat_rows[0], self.zlevel)
            return
        self.t.shard_lat_eval(sigma, K, self.r0, self.r1, self.dblock)
        with self._ctx():
            self.dist.all_gather_into_tensor(self.dpix, self.dblock)
        self.t.shard_lat_apply(it, sigma, lr, K, self.dpix, self.rows)

    def qat_search(self) -> None:
        """One selector search (qat_search)."""
        assert self.l0 is not None
        self.t.shard_qat(self.tr0, self.tr1, self.l0)
        a, b = self.tr0 * self.row_floats, self.tr1 * self.row_floats
        with self._ctx():
            self.dist.all_gather_into_tensor(self.l0, self.l0[a:b])
        self.t.shard_qat_apply(self.l0)


class NativeShardedES:
    """One ES training iteration per call in the library (ntcb_shard_iteration): the same per-rank work and
    exchanges as ShardedES, but every exchange is an in-place NCCL all-gather the library issues on the trainer's
    stream into the trainer's own buffers, on a communicator of its own. torch.distributed only carries the
    128-byte NCCL id from rank 0 to the others (any backend)."""

    def __init__(self, trainer, dist, device=None, p2p: tuple[int, int, bool] | None = None, comm_cls=None):
        """p2p = (N, K, qat): also set up the peer-memory exchanges (ntcb_p2p_export / import) for iterations with N
        ES pairs, K latent pairs and the selector search on or off; without it every exchange goes through NCCL.
        comm_cls: the communicator class (neural_block_textures_b200.trainer.Comm unless given)."""
        import torch
        from .trainer import Comm as _Comm
        Comm = comm_cls or _Comm
        self.t, self.dist = trainer, dist
        self.world, self.rank = dist.get_world_size(), dist.get_rank()
        uid = torch.zeros(128, dtype=torch.uint8, device=device or "cpu")
        if self.rank == 0:
            uid.copy_(torch.frombuffer(bytearray(Comm.unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        self.comm = Comm(bytes(uid.cpu().numpy().tobytes()), self.world, self.rank)
        self.p2p = False
        self.p2p_why = ""
        if p2p is not None and self.world > 1:
            # collective decision: every rank uses the peer exchange, or none does (NCCL then)
            N, K, qat = p2p
            try:
                mine = trainer.p2p_export(self.world, self.rank, N, K, qat)
            except RuntimeError as e:
                mine, self.p2p_why = None, str(e)
            allh = [None] * self.world
            dist.all_gather_object(allh, mine)
            ok = all(h is not None for h in allh)
            if ok:
                try:
                    trainer.p2p_import(b"".join(allh), self.world, self.rank)
                except RuntimeError as e:
                    ok, self.p2p_why = False, str(e)
            oks = [None] * self.world
            dist.all_gather_object(oks, ok)
            if all(oks):
                self.p2p = True
            else:
                if ok:
                    trainer.p2p_release()
                self.p2p_why = self.p2p_why or "another rank could not set up the peer exchange"

    def plan(self, mlp_mode: int, N: int, M: int, K: int, qat: bool):
        return self.t.shard_iteration_plan(self.world, self.rank, mlp_mode, N, M, K, qat)

    def iteration(self, it: int, mlp_mode: int, mlp_sigma: float, mlp_lr: float, N: int, M: int, K: int, lat_sigma: float,
                  lat_lr: float, qat: bool) -> None:
        """mlp_mode 1: mlp_step (sigma, lr, N pairs, M rows), 2: mlp_step_fd (h = mlp_sigma); then lat_step (K pairs; 0
        skips it) and, with qat, qat_search."""
        self.t.shard_iteration(self.comm, it, mlp_mode, mlp_sigma, mlp_lr, N, M, K, lat_sigma, lat_lr, qat)

    def close(self) -> None:
        """Collective: every rank unmaps its peers' exchange buffers, then all wait, so no buffer is freed while a
        peer still maps it; then the communicator goes."""
        if self.p2p:
            self.t.p2p_release()
            self.dist.barrier()
            self.p2p = False
        self.comm.close()
