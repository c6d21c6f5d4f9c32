"""The reference's own GPU-vs-CPU harness (main.cpp --cuda-check, main.cpp:2983-3219) run on this backend.

oracle/_ref/ntc_new is the reference trainer main.cpp compiled unmodified and linked against
libntc_b200.so through include/ntc_cuda.h: its --cuda-check compares our kernels with the reference's
CPU code on identical inputs (decode, ES loss differences, FD differences, latent gradient, selector
search, --qes snap, DCT symbols / plane / codes, the DCT rate integers) and must print
`cuda-check: all passed`. The flag lines are the reference's canonical regression lines
(README.md:1117-1127) with seeded synthetic images in place of the reference's photographs.
"""
import subprocess
from pathlib import Path

import pytest

from neural_block_textures_b200 import synth

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
NTC_NEW = ROOT / "oracle" / "_ref" / "ntc_new"

LINES = {
    "qat31_nearest_lv1local": "{img} --latent 512 512 2 --latent2 128 128 4 --filter nearest,nearest --pos lv1local --qat 3,1 --mlp 36,36",
    "default_bilinear": "{img} --latent 64 64 4",
    "material_qat2": "{m1} {m2} {m3} {m4} --latent 512 512 3 --latent2 128 128 4 --filter nearest,nearest --pos lv1local --qat 2 --mlp 36,36",
    "qes_block": "{img} --block 8 --latent 0 0 1 --latent2 0 0 4 --filter nearest,bilinear --pos lv1local --qat 2 --qes 0,8 --qes-start 0 "
                 "--mlp 17,17 --leak 0.0009765625",
    "qes_two_levels": "{img} --latent 128 128 4 --latent2 32 32 4 --filter bilinear,bilinear --pos uv --qes 6,8 --qes-start 0 --mlp 17,17",
    "dct50": "{img} --block 8 --latent 0 0 1 --latent2 0 0 4 --filter nearest,bilinear --pos lv1local --dct-deadzone 1 --dct-shadow-pull 0 "
             "--dct-q 50 --dct-lambda 0 --dct-start 0 --qes 0,8 --qes-start 0 --mlp 17,17 --leak 0.0009765625",
    "dct_two_channels": "{m1} --block 4 --latent 0 0 2 --latent2 0 0 4 --filter nearest,bilinear --pos lv1local --dct-deadzone 1 "
                        "--dct-shadow-pull 0 --dct-q 50,20 --dct-lambda 0 --dct-start 0 --qes 0,8 --qes-start 0 --mlp 27,27 --leak 0.0009765625",
    "dct_lambda80": "{img} --block 8 --latent 0 0 1 --latent2 0 0 4 --filter nearest,bilinear --pos lv1local --dct-deadzone 1 --dct-shadow-pull 0 "
                    "--dct-q 50 --dct-start 0 --qes 0,8 --qes-start 0 --mlp 17,17 --leak 0.0009765625 --dct-lambda 80",
    "dct_lambda80_two_channels": "{m1} --block 4 --latent 0 0 2 --latent2 0 0 4 --filter nearest,bilinear --pos lv1local --dct-deadzone 1 "
                                 "--dct-shadow-pull 0 --dct-q 50,20 --dct-start 0 --qes 0,8 --qes-start 0 --mlp 27,27 --leak 0.0009765625 --dct-lambda 80",
    "dct_deadzone0": "{img} --block 8 --latent 0 0 1 --latent2 0 0 4 --filter nearest,bilinear --pos lv1local --dct-shadow-pull 0 --dct-q 50 "
                     "--dct-lambda 0 --dct-start 0 --qes 0,8 --qes-start 0 --mlp 17,17 --leak 0.0009765625 --dct-deadzone 0",
    # the benchmark's shapes (fixed-shape kernels): config 2 and config 3
    "cfg2_shape": "{img} --latent 512 512 1 --latent2 128 128 2 --filter nearest,bilinear --qat 2 --mlp-pairs 64",
    "cfg3_shape": "{m1} {m2} {m3} {m4} --latent 512 512 2 --latent2 128 128 4 --filter nearest,bilinear --qat 2 --mlp-pairs 64",
    # config 4 at its own size: 1024^2, DCT-coded level 0 at q 50 with the default widths, the default --dct-lambda recipe
    # (rate term in the latent gradient and truncation at snap), the default dead-zone and shadow pull; --dct-start 0 makes the
    # level live before the harness runs (at the config's default 0.5 the DCT checks would report "skipped")
    "cfg4_shape": "{img1024} --latent 1024 1024 1 --latent2 256 256 2 --filter nearest,bilinear --dct-q 50 --dct-start 0 --mlp-pairs 64",
    # config 5 at its own size: 2048^2, level 0 1024x1024x2 2-bit selectors (2x2-pixel cells), level 1 256x256x4
    "cfg5_shape": "{img2048} --latent 1024 1024 2 --latent2 256 256 4 --filter nearest,bilinear --qat 2 --mlp-pairs 64",
}


@pytest.fixture(scope="module")
def images(tmp_path_factory):
    d = tmp_path_factory.mktemp("imgs")
    paths = {"img": d / "synth512_s21.png", "img1024": d / "synth1024_s4.png", "img2048": d / "synth2048_s5.png"}
    synth.write_png(paths["img"], synth.synth_rgb8(512, 512, 21))
    synth.write_png(paths["img1024"], synth.synth_rgb8(1024, 1024, 4))
    synth.write_png(paths["img2048"], synth.synth_rgb8(2048, 2048, 5))
    for t, im in enumerate(synth.synth_material(512, 512, 31, 4)):
        paths[f"m{t + 1}"] = d / f"mat512_s31_t{t}.png"
        synth.write_png(paths[f"m{t + 1}"], im)
    return {k: str(v) for k, v in paths.items()}


@pytest.mark.parametrize("name", list(LINES))
def test_reference_cuda_check(name, images, tmp_path, cuda_device):
    if not NTC_NEW.exists():
        pytest.skip("oracle/_ref/ntc_new not built (needs the reference tree at build time)")
    args = LINES[name].format(**images).split()
    cmd = [str(NTC_NEW), *args, "--cuda", "--cuda-check", "--rng", "hash", "--iters", "5", "--print-every", "5", "--out", str(tmp_path)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert "cuda-check: all passed" in out, out[-4000:]
