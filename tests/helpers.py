"""Small seeded test models shaped like the benchmark configurations, with their targets."""
from __future__ import annotations

import numpy as np

from neural_block_textures_b200 import model, synth
from neural_block_textures_b200.model import LevelSpec, ModelSpec


def spec_named(name: str) -> ModelSpec:
    """cfgN-like models at sizes the oracle evaluates in seconds."""
    if name == "cfg1":      # bilinear 4-channel level, uv: fixed shape (6, 24, 24, 3)
        return ModelSpec(64, 64, [LevelSpec(16, 16, 4)], max_pairs=64, max_batch=1024, seed=11)
    if name == "cfg2":      # nearest 2-bit qat level 0 at full res + bilinear level 1: (5, 24, 24, 3)
        return ModelSpec(64, 64, [LevelSpec(64, 64, 1, True), LevelSpec(16, 16, 2)], qat_bits=(2,), max_pairs=64,
                         max_batch=1024, seed=12)
    if name == "cfg3":      # 4-texture material: (8, 24, 24, 12)
        return ModelSpec(64, 64, [LevelSpec(64, 64, 2, True), LevelSpec(16, 16, 4)], T=4, qat_bits=(2, 2),
                         weights=(1.0, 2.0, 0.5, 1.0), max_pairs=64, max_batch=1024, seed=13)
    if name == "cfg5":      # level 0 at half resolution (2x2 cells): (8, 24, 24, 3)
        return ModelSpec(96, 64, [LevelSpec(48, 32, 2, True), LevelSpec(24, 16, 4)], qat_bits=(2, 2), max_pairs=64,
                         max_batch=1024, seed=15)
    if name == "generic":   # runtime-shaped kernels: 3 levels, one hidden layer of 20, lv1local, clamp output
        return ModelSpec(40, 36, [LevelSpec(20, 18, 3, True), LevelSpec(10, 9, 2), LevelSpec(5, 5, 2)], hidden=(20,),
                         pos=("uv", "lv1local"), clamp_out=True, qat_bits=(3, 1, 2), max_pairs=64, max_batch=512, seed=16)
    if name == "generic3":  # runtime-shaped, three hidden layers, odd widths, nearest level 1
        # 35 / 11 pixels per texel: no pixel centre lands exactly on a bilinear texel edge (at such ties the
        # reference's -ffast-math build attributes the pixel by its own rounding of (px + 0.5) / W).
        return ModelSpec(35, 29, [LevelSpec(11, 10, 3), LevelSpec(7, 5, 2, True)], hidden=(13, 9, 7), pos=("uv",),
                         leak=0.05, max_pairs=64, max_batch=512, seed=17)
    raise KeyError(name)


ALL_SPECS = ["cfg1", "cfg2", "cfg3", "cfg5", "generic", "generic3"]


def target_for(spec: ModelSpec, seed: int = 5) -> np.ndarray:
    if spec.T == 1:
        return synth.to_target([synth.synth_rgb8(spec.W, spec.H, seed)])
    return synth.to_target(synth.synth_material(spec.W, spec.H, seed, spec.T))


def active_mask(spec: ModelSpec) -> int:
    m = 0
    for l in range(len(spec.levels)):
        if not (spec.qat_bits and l == 0):
            m |= 1 << l
    return m


def rel_err(a, b) -> float:
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) / np.maximum(np.abs(b), 1e-300)))
