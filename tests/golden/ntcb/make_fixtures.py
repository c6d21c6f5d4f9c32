"""Records .ntcb containers written by the reference's own CPU trainer (main.cpp --write-ntcb, oracle/_ref/ntc_cpu)
on small seeded synthetic images, and what the reference's own standalone decoder (ntc_decode.cpp,
oracle/_ref/ntc_decode, `--exact`) and the trainer (recon_q_final.png) decode from them. Run here, where the
reference tree exists (`make -C oracle ref` first):

    python tests/golden/ntcb/make_fixtures.py

Writes tests/golden/ntcb/<name>.ntcb and <name>.npz (the decoder's RGB8 per texture, the trainer's
recon_q_final RGB8, the trainer's printed final PSNR line). Every case covers a coding mode or a header feature:
  qat_q8        level 0 --qat palette (mode 2) + level 1 post-hoc 8-bit grid (mode 0), the (5, 24, 24, 3) shape
  qes           two --qes grid levels (mode 1), bilinear, uv position, runtime-shaped MLP
  dct           DCT-coded level 0 (mode 3, dead-zone quantizer) + a --qes level 1, lv1local, a padded source
                (60 x 52 -> 64 x 56) so the crop is exercised
  dct2_dz0      two DCT channels at different qualities, plain-rounding quantizer (dct_flags 0)
  material      two textures (nout 6), --qat level 0 + post-hoc level 1
"""
from __future__ import annotations

import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[2]
sys.path.insert(0, str(ROOT))

from neural_block_textures_b200 import synth  # noqa: E402

REF = ROOT / "oracle" / "_ref"
COMMON = "--rng hash --threads 1 --print-every 1000000 --write-ntcb"
CASES = {
    "qat_q8": ([(64, 64, 3)], "--latent 64 64 1 --latent2 16 16 2 --filter nearest,bilinear --qat 2 --mlp-pairs 16 --iters 20 --seed 3"),
    "qes": ([(48, 40, 4)], "--latent 24 20 4 --latent2 12 10 3 --filter bilinear,bilinear --pos uv --qes 6,8 --qes-start 0 --mlp 17,17 "
                           "--mlp-pairs 16 --iters 20 --seed 4"),
    "dct": ([(60, 52, 5)], "--block 8 --latent 0 0 1 --latent2 0 0 4 --filter nearest,bilinear --pos lv1local --dct-deadzone 1 "
                           "--dct-shadow-pull 0 --dct-q 50 --dct-lambda 0 --dct-start 0 --qes 0,8 --qes-start 0 --mlp 17,17 "
                           "--leak 0.0009765625 --mlp-pairs 16 --iters 20 --seed 5"),
    "dct2_dz0": ([(64, 64, 6)], "--block 4 --latent 0 0 2 --latent2 0 0 4 --filter nearest,bilinear --pos lv1local --dct-deadzone 0 "
                                "--dct-shadow-pull 0 --dct-q 50,20 --dct-lambda 0 --dct-start 0 --qes 0,8 --qes-start 0 --mlp 27,27 "
                                "--leak 0.0009765625 --mlp-pairs 16 --iters 20 --seed 6"),
    "material": ([(64, 64, 7), (64, 64, 8)], "--latent 64 64 2 --latent2 16 16 4 --filter nearest,bilinear --qat 2 --mlp-pairs 16 "
                                             "--iters 20 --seed 7"),
}


def run_case(name: str, images, flags: str, tmp: Path) -> None:
    paths = []
    for i, (w, h, seed) in enumerate(images):
        p = tmp / f"{name}_{i}.png"
        synth.write_png(p, synth.synth_rgb8(w, h, seed))
        paths.append(str(p))
    out = tmp / name
    r = subprocess.run([str(REF / "ntc_cpu"), *paths, *flags.split(), *COMMON.split(), "--out", str(out)],
                       capture_output=True, text=True, timeout=600)
    if r.returncode != 0 or "[OK]" not in r.stdout:
        raise SystemExit(f"{name}: trainer failed\n{r.stdout[-3000:]}\n{r.stderr[-2000:]}")
    done = [ln for ln in r.stdout.splitlines() if ln.startswith("done:")]
    shutil.copy(out / "model.ntcb", HERE / f"{name}.ntcb")
    d = subprocess.run([str(REF / "ntc_decode"), str(out / "model.ntcb"), "-o", str(out / "dec"), "--exact", "--threads", "1"],
                       capture_output=True, text=True, timeout=600)
    if d.returncode != 0:
        raise SystemExit(f"{name}: ntc_decode failed\n{d.stdout[-3000:]}")
    T = len(images)
    dec = np.stack([synth.read_png(out / ("dec.png" if T == 1 else f"dec_t{t}.png")) for t in range(T)])
    recon = [synth.read_png(out / ("recon_q_final.png" if T == 1 else f"recon_q_final_t{t}.png")) for t in range(T)] \
        if (out / ("recon_q_final.png" if T == 1 else "recon_q_final_t0.png")).exists() else []
    np.savez_compressed(HERE / f"{name}.npz", decoder_rgb8=dec, trainer_rgb8=np.stack(recon) if recon else np.zeros(0, np.uint8),
                        done_line=np.array(done[-1] if done else ""))
    print(f"{name}: {(HERE / f'{name}.ntcb').stat().st_size} bytes, decode {dec.shape}")


def main() -> None:
    for b in ("ntc_cpu", "ntc_decode"):
        if not (REF / b).exists():
            raise SystemExit(f"oracle/_ref/{b} missing: run `make -C oracle ref` where the reference tree exists")
    with tempfile.TemporaryDirectory() as t:
        for name, (images, flags) in CASES.items():
            run_case(name, images, flags, Path(t))


if __name__ == "__main__":
    main()
