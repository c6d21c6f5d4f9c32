"""Model descriptions for the B200 backend, built the way the reference trainer lays a model out.

ModelSpec holds what main.cpp derives from its options before it calls Trainer::init
(main.cpp:3478-3565, 3882-3912): the latent levels and their flat offsets, the positional inputs,
the MLP widths, loss weights, --qat / --qes / --dct-q settings and the buffer sizes. It produces
the ctypes ModelDesc, the QAT grid table and a seeded initial latent and MLP.

The five benchmark configurations (configs 1-5 of the benchmark definition) are in CONFIGS.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import abi

POS_KINDS = {"uv": 0, "lv1local": 1}


@dataclass
class LevelSpec:
    W: int
    H: int
    C: int
    nearest: bool = False

    @property
    def size(self) -> int:
        return self.W * self.H * self.C


def qat_grid_table() -> np.ndarray:
    """QAT_GRID[9][257] (main.cpp:2051-2057): grid value k of a B-bit channel is -1 + 2k / (2^B - 1),
    evaluated in float as the expression reads (2.0f * k, then / levels, then + -1.0f)."""
    g = np.zeros((9, 257), np.float32)
    for b in range(1, 9):
        levels = np.float32((1 << b) - 1)
        for k in range((1 << b)):
            g[b, k] = np.float32(-1.0) + (np.float32(2.0) * np.float32(k)) / levels
    return g


def qat_index(v: float, bits: int) -> int:
    """qat_index (main.cpp:2060-2064): lround((v + 1) / 2 * levels), clamped."""
    levels = (1 << bits) - 1
    x = (np.float32(v) + np.float32(1.0)) * np.float32(0.5) * np.float32(levels)
    k = int(np.floor(abs(float(x)) + 0.5)) * (1 if x >= 0 else -1)
    return max(0, min(levels, k))


def qat_index_array(v: np.ndarray, bits: int) -> np.ndarray:
    """qat_index of every element of v (the same float32 steps, lround as floor(|x| + 0.5) with the sign)."""
    levels = (1 << bits) - 1
    x = ((v.astype(np.float32) + np.float32(1.0)) * np.float32(0.5) * np.float32(levels)).astype(np.float64)
    k = np.floor(np.abs(x) + 0.5) * np.where(x >= 0, 1.0, -1.0)
    return np.clip(k, 0, levels).astype(np.int64)


@dataclass
class ModelSpec:
    W: int
    H: int
    levels: list[LevelSpec]
    T: int = 1
    hidden: tuple[int, ...] = (24, 24)
    pos: tuple[str, ...] = ("uv",)
    leak: float = 0.01
    clamp_out: bool = False
    weights: tuple[float, ...] | None = None
    qat_bits: tuple[int, ...] | None = None      # per level-0 channel
    qes_bits: tuple[int, ...] = (0, 0, 0)
    dct_q: tuple[int, ...] | None = None          # per level-0 channel quality (DCT-coded level 0)
    dct_dc_step: int = 4
    max_pairs: int = 64
    max_batch: int = 4096
    seed: int = 1
    _keep: list = field(default_factory=list, repr=False)

    @property
    def nout(self) -> int:
        return 3 * self.T

    @property
    def nin(self) -> int:
        return sum(L.C for L in self.levels) + 2 * len(self.pos)

    @property
    def offsets(self) -> list[int]:
        offs, o = [], 0
        for L in self.levels:
            offs.append(o)
            o += L.size
        return offs

    @property
    def nz(self) -> int:
        return sum(L.size for L in self.levels)

    @property
    def widths(self) -> list[int]:
        return [self.nin, *self.hidden, self.nout]

    @property
    def P(self) -> int:
        w = self.widths
        return sum(w[i] * w[i - 1] + w[i] for i in range(1, len(w)))

    @property
    def qat(self) -> int:
        return max(self.qat_bits) if self.qat_bits else 0

    @property
    def wts(self) -> tuple[float, ...]:
        return self.weights if self.weights is not None else (1.0,) * self.T

    @property
    def wsum(self) -> np.float32:
        s = np.float32(0.0)
        for w in self.wts:
            s = np.float32(s + np.float32(w))
        return s

    def model_desc(self) -> abi.ModelDesc:
        d = abi.ModelDesc()
        d.W, d.H, d.T = self.W, self.H, self.T
        d.nlev = len(self.levels)
        for l, (L, off) in enumerate(zip(self.levels, self.offsets)):
            d.lv[l].W, d.lv[l].H, d.lv[l].C, d.lv[l].off, d.lv[l].nearest = L.W, L.H, L.C, off, L.nearest
        d.npos = len(self.pos)
        for q, k in enumerate(self.pos):
            d.pos[q].kind = POS_KINDS[k]
        d.nin, d.nout = self.nin, self.nout
        d.nhidden = len(self.hidden)
        for l, h in enumerate(self.hidden):
            d.hidden[l] = h
        d.leak = self.leak
        d.clamp_out = self.clamp_out
        for c in range(abi.MAX_OUT):
            d.cw[c] = self.wts[c // 3] if c < self.nout else 0.0
        d.wsum = float(self.wsum)
        self._keep.clear()
        if self.qat_bits:
            for c, b in enumerate(self.qat_bits):
                d.qat_bits[c] = b
            d.qat = self.qat
            grid = qat_grid_table()
            self._keep.append(grid)
            d.qat_grid = grid.ctypes.data_as(C.POINTER(C.c_float))
        for l in range(min(3, len(self.qes_bits))):
            d.qes_bits[l] = self.qes_bits[l]
        if self.dct_q:
            from . import dct as _dct
            d.dct, d.dct_C, d.dct_N, d.dct_dc_step = 1, self.levels[0].C, 8, self.dct_dc_step
            for c, q in enumerate(self.dct_q):
                d.dct_q[c] = q
            basis, zz = _dct.basis_table(), _dct.zigzag_table()
            self._keep += [basis, zz]
            d.dct_basis = basis.ctypes.data_as(C.POINTER(C.c_float))
            d.dct_zigzag = zz.ctypes.data_as(C.POINTER(C.c_int))
        d.max_pairs, d.max_batch = self.max_pairs, self.max_batch
        d.seed = self.seed
        return d

    def init_params(self, lat_init: float = 0.1, seed: int | None = None) -> tuple[np.ndarray, np.ndarray]:
        """A seeded initial latent N(0, lat_init) (level 0 snapped to its --qat grid) and MLP (He init for
        hidden layers, sqrt(1 / fan_in) for the output, zero biases), as main.cpp:586-599 and 3539-3543
        describe them; the draws come from numpy, not from the reference's std::mt19937."""
        rng = np.random.default_rng(self.seed if seed is None else seed)
        z = (rng.standard_normal(self.nz) * lat_init).astype(np.float32)
        if self.qat_bits:
            grid = qat_grid_table()
            L0 = self.levels[0]
            z0 = z[: L0.size].reshape(-1, L0.C)
            for c, b in enumerate(self.qat_bits):
                z0[:, c] = grid[b, qat_index_array(z0[:, c], b)]
        if self.dct_q:
            L0 = self.levels[0]
            z[: L0.size] = np.clip(z[: L0.size], -1.0, 1.0)
        w = self.widths
        p = []
        for l in range(1, len(w)):
            last = l + 1 == len(w)
            s = np.sqrt(1.0 / w[l - 1]) if last else np.sqrt(2.0 / w[l - 1])
            p.append((rng.standard_normal(w[l] * w[l - 1]) * s).astype(np.float32))
            p.append(np.zeros(w[l], np.float32))
        return np.ascontiguousarray(z), np.ascontiguousarray(np.concatenate(p).astype(np.float32))


@dataclass
class TrainConfig:
    """One benchmark configuration: the model, the synthetic input and the ES hyper-parameters."""
    name: str
    spec: ModelSpec
    image_seed: int
    pairs: int                 # N (population 2N)
    batch: int = 4096          # M
    lat_pairs: int = 4         # K
    iters: int = 3000
    mlp_sigma: float = 0.02
    mlp_lr: float = 0.005
    lat_sigma: float = 0.05
    lat_lr: float = 0.02
    fd_start: float = 1.0      # fraction of iters at which FD replaces ES (>= 1 = never)
    fd_h: float = 1e-3
    cli: str = ""              # the reference CLI options that describe the same run

    def images(self) -> list[np.ndarray]:
        from . import synth
        if self.spec.T == 1:
            return [synth.synth_rgb8(self.spec.W, self.spec.H, self.image_seed)]
        return synth.synth_material(self.spec.W, self.spec.H, self.image_seed, self.spec.T)

    def target(self) -> np.ndarray:
        from . import synth
        return synth.to_target(self.images())

    def decodes_per_iter(self, fd: bool = False) -> dict[str, int]:
        """Candidate-pixel decodes of one iteration per phase (MLP ES 2N M, FD (2P + 2) M, latent 2K W H when a
        level is ES-trained, qat sum_c 2^B_c W H)."""
        s = self.spec
        out = {"mlp": (2 * s.P + 2) * self.batch if fd else 2 * self.pairs * self.batch}
        active = [l for l in range(len(s.levels)) if not (s.qat_bits and l == 0)]
        out["latent"] = 2 * self.lat_pairs * s.W * s.H if active else 0
        out["qat"] = sum(1 << b for b in s.qat_bits) * s.W * s.H if s.qat_bits else 0
        return out

    def flops_per_decode(self) -> int:
        w = self.spec.widths
        return 2 * sum(w[i] * w[i - 1] for i in range(1, len(w)))


def _cfg(n: int) -> TrainConfig:
    if n == 1:
        spec = ModelSpec(256, 256, [LevelSpec(64, 64, 4, False)], max_pairs=32, seed=1)
        return TrainConfig("cfg1_256_lat64x64x4_pairs32", spec, 1, pairs=32, iters=200,
                           cli="--latent 64 64 4 --mlp-pairs 32 --iters 200 --seed 1")
    if n == 2:
        spec = ModelSpec(512, 512, [LevelSpec(512, 512, 1, True), LevelSpec(128, 128, 2, False)], qat_bits=(2,),
                         max_pairs=4096, seed=2)
        return TrainConfig("cfg2_512_qat2_512x512x1_lat2_128x128x2_pop8192", spec, 2, pairs=4096, iters=8000, fd_start=0.5,
                           cli="--latent 512 512 1 --latent2 128 128 2 --filter nearest,bilinear --qat 2 --mlp-pairs 4096 "
                               "--iters 8000 --mlp-fd 0.5 --write-ntcb --seed 2")
    if n == 3:
        spec = ModelSpec(512, 512, [LevelSpec(512, 512, 2, True), LevelSpec(128, 128, 4, False)], T=4, qat_bits=(2, 2),
                         max_pairs=4096, seed=3)
        return TrainConfig("cfg3_4x512_qat2_512x512x2_lat2_128x128x4_pop8192", spec, 3, pairs=4096, iters=8000,
                           cli="--latent 512 512 2 --latent2 128 128 4 --filter nearest,bilinear --qat 2 --mlp-pairs 4096 "
                               "--iters 8000 --seed 3")
    if n == 4:
        spec = ModelSpec(1024, 1024, [LevelSpec(1024, 1024, 1, True), LevelSpec(256, 256, 2, False)], dct_q=(50,),
                         max_pairs=4096, seed=4)
        return TrainConfig("cfg4_1024_dct50_lat2_256x256x2_pop8192", spec, 4, pairs=4096, iters=4000,
                           cli="--latent 1024 1024 1 --latent2 256 256 2 --filter nearest,bilinear --dct-q 50 --mlp-pairs 4096 "
                               "--iters 4000 --seed 4")
    if n == 5:
        spec = ModelSpec(2048, 2048, [LevelSpec(1024, 1024, 2, True), LevelSpec(256, 256, 4, False)], qat_bits=(2, 2),
                         max_pairs=16384, seed=5)
        return TrainConfig("cfg5_2048_qat2_1024x1024x2_lat2_256x256x4_pop32768", spec, 5, pairs=16384, iters=1000,
                           cli="--latent 1024 1024 2 --latent2 256 256 4 --filter nearest,bilinear --qat 2 --mlp-pairs 16384 "
                               "--iters 1000 --seed 5")
    raise ValueError(f"no config {n}")


CONFIGS = {n: _cfg for n in range(1, 6)}


def config(n: int) -> TrainConfig:
    return _cfg(n)
