"""Records golden vectors from the reference's own CPU code (main.cpp compiled unmodified behind
oracle/ref_shim.cpp, built by `make -C oracle ref` from the read-only reference tree) for the small seeded
models of tests/helpers.py. Run here (where the reference tree exists):

    python tests/golden/make_golden.py

Writes tests/golden/ref_golden.npz. tests/test_oracle_pin.py checks the oracle restatement against it, and
the GPU tests can use it on a box that has no reference tree.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from neural_block_textures_b200.model import qat_grid_table  # noqa: E402
from oracle.oracle import RefSession, refcpu_lib  # noqa: E402
from tests.helpers import ALL_SPECS, active_mask, spec_named, target_for  # noqa: E402

OUT = Path(__file__).resolve().parent / "ref_golden.npz"
SIGMA, LAT_SIGMA, LR, FD_H = 0.02, 0.05, 0.005, 1e-3


def main() -> None:
    lib = refcpu_lib()
    lib.ref_set_threads(1)   # the CPU result is not bit-stable across thread counts; pin one
    g: dict[str, np.ndarray] = {}
    # noise: the reference's ntc_noise.h on the host
    keys = [(1, 2, 7, 3, 0), (12345678901, 1, 0, 0, 1 << 33), (2, 3, 99, 0, 17), (5, 4, 1, 2, 1000)]
    for n, (seed, stream, step, pair, i0) in enumerate(keys):
        g[f"noise{n}_key"] = np.array([seed, stream, step, pair, i0], np.uint64)
        g[f"noise{n}_u32"] = np.array([lib.ref_noise_u32(seed, stream, step, pair, i0 + i) for i in range(512)], np.uint32)
        gs = np.zeros(512, np.float32)
        import ctypes as C
        lib.ref_noise_gauss_block(seed, stream, step, pair, i0, 512, gs.ctypes.data_as(C.POINTER(C.c_float)))
        g[f"noise{n}_gauss"] = gs
    g["qat_grid"] = np.zeros((9, 257), np.float32)
    import ctypes as C
    lib.ref_qat_grid(g["qat_grid"].ctypes.data_as(C.POINTER(C.c_float)))
    for name in ALL_SPECS:
        spec = spec_named(name)
        tgt = target_for(spec)
        z, p = spec.init_params()
        s = RefSession(spec, tgt)
        s.set_model(z, p)
        pre = f"{name}_"
        g[pre + "z"], g[pre + "p"] = z, p
        g[pre + "decode"] = s.decode_full(p, z)
        idx = np.array([lib.ref_noise_u32(spec.seed, 3, 3, 0, k) for k in range(256)], np.uint64)
        idx = ((idx * np.uint64(spec.W * spec.H)) >> np.uint64(32)).astype(np.int32)
        g[pre + "batch"] = idx
        g[pre + "loss"] = np.array([s.loss_subset(p, idx)])
        lp, lm = s.es_fitness(3, SIGMA, 0, 8, idx)
        g[pre + "lp"], g[pre + "lm"] = lp, lm
        js = np.unique(np.array([(q * 7919) % spec.P for q in range(12)], np.int32))
        g[pre + "fd_js"] = js
        g[pre + "fd_dl"] = s.fd_dl(FD_H, idx, js)
        mask = active_mask(spec)
        if mask:
            g[pre + "latgrad"] = s.lat_step(4, LAT_SIGMA, 0.0)   # step 0, lr 0: the latent is unchanged
        if spec.qat_bits:
            s.qat_search()
            zq, _ = s.get_model()
            g[pre + "qat_z"] = zq
            s.set_model(z, p)
        # one full ES step (iteration 3, N 16, M 256, lr LR) through MlpTrainer::step
        s.set_model(z, p)
        s.mlp_step(3, 16, 256, SIGMA, LR)
        _, p1 = s.get_model()
        g[pre + "es_step_p"] = p1
        g[pre + "es_step_grad"] = s.mlp_grad()
        s.close()
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
