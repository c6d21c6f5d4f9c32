"""Population sharding of the MLP ES step over G ranks (one process and one GPU per rank).

Rank r evaluates the antithetic pairs [r N / G, (r + 1) N / G) of every step, regenerating their noise from
the counter (no noise crosses the wire), and contributes 2 doubles per pair (L+, L-). One all-gather
(NCCL over NVLink on GPUs, gloo in the CPU tests) gives every rank the fitness of all N pairs in pair order,
from which each rank computes the identical ES gradient and Adam step, so the weight replicas stay
bit-identical without exchanging weights. The latent ES step and the selector search run as replicas.
"""
from __future__ import annotations


def pair_range(N: int, world: int, rank: int) -> tuple[int, int]:
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    if N % world:
        raise ValueError(f"{N} pairs do not split evenly over {world} ranks")
    per = N // world
    return rank * per, (rank + 1) * per


def _ptr(x):
    return x if isinstance(x, int) else x.data_ptr()


class ShardedES:
    """Drives trainer.shard_mlp_eval / shard_mlp_apply around one all-gather of the per-pair fitness.

    `trainer` is a neural_block_textures_b200.Trainer (or any object with the same two methods); `dist` is
    torch.distributed with an initialised process group; `device` is where the fitness buffers live (the
    trainer's GPU, or "cpu" for a gloo group)."""

    def __init__(self, trainer, dist, N: int, device="cuda", stream=None):
        import torch
        self.t, self.dist, self.N = trainer, dist, N
        self.world, self.rank = dist.get_world_size(), dist.get_rank()
        self.p0, self.p1 = pair_range(N, self.world, self.rank)
        per = self.p1 - self.p0
        self.fit_local = torch.zeros(2 * per, dtype=torch.float64, device=device)
        self.fit_all = torch.zeros(2 * N, dtype=torch.float64, device=device)
        self.stream = stream

    def step(self, it: int, sigma: float, lr: float, M: int) -> None:
        import contextlib
        import torch
        self.t.shard_mlp_eval(it, sigma, self.N, M, self.p0, self.p1, self.fit_local)
        ctx = torch.cuda.stream(self.stream) if self.stream is not None else contextlib.nullcontext()
        with ctx:
            self.dist.all_gather_into_tensor(self.fit_all, self.fit_local)
        self.t.shard_mlp_apply(it, sigma, lr, self.N, M, self.fit_all)
