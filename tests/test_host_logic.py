"""Host-side logic without a GPU: synthetic inputs, PNG round trip, model layout arithmetic, the DCT host
tables against the reference's own, the texel footprint ranges the latent gather relies on, and init()'s
envelope checks (which run before any CUDA call)."""
import ctypes as C
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from neural_block_textures_b200 import abi, dct, model, synth
from neural_block_textures_b200.model import LevelSpec, ModelSpec

ROOT = Path(__file__).resolve().parent.parent


def test_synth_is_deterministic_and_in_range():
    a = synth.synth_rgb8(96, 64, 7)
    b = synth.synth_rgb8(96, 64, 7)
    assert a.shape == (64, 96, 3) and a.dtype == np.uint8 and np.array_equal(a, b)
    assert not np.array_equal(a, synth.synth_rgb8(96, 64, 8))
    assert a.std() > 10, "not a flat image"
    mat = synth.synth_material(64, 64, 3, 4)
    assert len(mat) == 4 and all(m.shape == (64, 64, 3) for m in mat)
    t = synth.to_target(mat)
    assert t.shape == (64 * 64 * 12,) and t.min() >= 0 and t.max() <= 1
    assert t[3] == np.float32(mat[1][0, 0, 0]) / np.float32(255.0), "interleaved [r0 g0 b0 r1 ...]"


def test_png_round_trip(tmp_path):
    img = synth.synth_rgb8(37, 23, 5)
    synth.write_png(tmp_path / "a.png", img)
    assert np.array_equal(synth.read_png(tmp_path / "a.png"), img)


def test_reference_reads_our_png(tmp_path):
    """The reference CLI decodes the synthetic PNG (stb_image) to the same bytes: it prints its latent layout."""
    exe = ROOT / "oracle" / "_ref" / "ntc_cpu"
    if not exe.exists():
        pytest.skip("oracle/_ref/ntc_cpu not built")
    img = synth.synth_rgb8(64, 64, 3)
    synth.write_png(tmp_path / "s.png", img)
    r = subprocess.run([str(exe), str(tmp_path / "s.png"), "--iters", "0", "--latent", "16", "16", "4", "--out", str(tmp_path / "o"),
                        "--threads", "1"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "image    : 64x64" in r.stdout


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5])
def test_config_shapes(n):
    """The benchmark configurations' derived shapes (nin, P, population, decodes per iteration)."""
    cfg = model.config(n)
    s = cfg.spec
    expect = {1: (6, 843, 64, 1584), 2: (5, 819, 8192, 1536), 3: (8, 1116, 8192, 2112), 4: (5, 819, 8192, 1536),
              5: (8, 891, 32768, 1680)}[n]
    assert (s.nin, s.P, 2 * cfg.pairs, cfg.flops_per_decode()) == expect
    d = cfg.decodes_per_iter()
    if n == 2:
        assert d == {"mlp": 33554432, "latent": 2097152, "qat": 1048576}
    if n == 5:
        assert d == {"mlp": 134217728, "latent": 33554432, "qat": 33554432}


def test_model_desc_layout_values():
    s = ModelSpec(32, 16, [LevelSpec(32, 16, 2, True), LevelSpec(8, 4, 3)], T=2, qat_bits=(2, 3), weights=(1.0, 3.0))
    d = s.model_desc()
    assert (d.W, d.H, d.T, d.nlev, d.nin, d.nout) == (32, 16, 2, 2, 7, 6)
    assert d.lv[1].off == 32 * 16 * 2 and d.lv[0].nearest and not d.lv[1].nearest
    assert list(d.cw[:6]) == [1, 1, 1, 3, 3, 3] and d.wsum == 4.0
    assert d.qat == 3 and d.qat_bits[0] == 2 and d.qat_bits[1] == 3
    grid = np.ctypeslib.as_array(d.qat_grid, shape=(9 * 257,))
    assert grid[3 * 257 + 7] == 1.0 and grid[2 * 257] == -1.0
    z, p = s.init_params()
    assert z.size == s.nz and p.size == s.P
    g = model.qat_grid_table()
    z0 = z[: 32 * 16 * 2].reshape(-1, 2)
    assert np.isin(z0[:, 0], g[2, :4]).all() and np.isin(z0[:, 1], g[3, :8]).all(), "qat level starts on its grid"


def brute_ranges(npx: int, ntex: int, nearest: bool):
    """Pixel sets per texel from the reference's tap rule written out directly (main.cpp:512-531, 2015-2024)."""
    sets = [[] for _ in range(ntex)]
    f32 = np.float32
    for px in range(npx):
        u = f32(f32(px) + f32(0.5)) / f32(npx)
        if nearest:
            t = min(ntex - 1, max(0, int(np.floor(f32(u * f32(ntex))))))
            sets[t].append(px)
        else:
            x = np.float32(np.float64(u) * ntex - 0.5)      # exact product, one rounding: the fused form
            x0 = int(np.floor(x))
            t0, t1 = min(ntex - 1, max(0, x0)), min(ntex - 1, max(0, x0 + 1))
            sets[t0].append(px)
            if t1 != t0:
                sets[t1].append(px)
    return sets


@pytest.mark.parametrize("npx,ntex", [(512, 128), (512, 512), (2048, 256), (64, 16), (35, 11), (40, 5), (33, 7), (100, 100), (7, 20)])
@pytest.mark.parametrize("nearest", [False, True])
def test_footprint_ranges(npx, ntex, nearest):
    lib = abi.load_library()
    lo = np.zeros(ntex, np.int32); hi = np.zeros(ntex, np.int32)
    ok = lib.ntcb_footprint_ranges(npx, ntex, int(nearest), lo.ctypes.data_as(C.POINTER(C.c_int)), hi.ctypes.data_as(C.POINTER(C.c_int)))
    assert ok == 1, "contiguous footprints"
    for t, s in enumerate(brute_ranges(npx, ntex, nearest)):
        if s:
            assert (lo[t], hi[t]) == (s[0], s[-1] + 1) and s == list(range(s[0], s[-1] + 1))
        else:
            assert lo[t] >= hi[t], "a texel without pixels gets an empty range"


def test_dct_tables_match_reference():
    from oracle.oracle import refcpu_available, refcpu_lib
    if not refcpu_available():
        pytest.skip("reference build absent")
    lib = refcpu_lib()
    basis = np.zeros(64, np.float32); zz = np.zeros(64, np.int32); ak = np.zeros(16, np.float32)
    lib.ref_dct_tables(basis.ctypes.data_as(C.POINTER(C.c_float)), zz.ctypes.data_as(C.POINTER(C.c_int)), ak.ctypes.data_as(C.POINTER(C.c_float)))
    assert np.array_equal(dct.basis_table().view(np.uint32), basis.view(np.uint32))
    assert np.array_equal(dct.zigzag_table(), zz)
    assert np.array_equal(dct.ak_table().view(np.uint32), ak.view(np.uint32))
    for q in (1, 10, 20, 30, 49, 50, 51, 75, 90, 99, 100):
        st = np.zeros(16 * 64, np.int32)
        lib.ref_dct_build_steps(q, 4, st.ctypes.data_as(C.POINTER(C.c_int)))
        assert np.array_equal(dct.build_steps(q, 4).reshape(-1), st), f"q={q}"
        assert dct.quality_scale(q) == lib.ref_dct_quality_scale(q)
    for k in range(16):
        assert dct.gain_of_code(k) == lib.ref_dct_gain_of_code(k)


def _init_reason(spec_code: str) -> str:
    code = ("import sys; sys.path.insert(0, %r)\n"
            "from neural_block_textures_b200 import Trainer\n"
            "from neural_block_textures_b200.model import ModelSpec, LevelSpec\n"
            "import numpy as np\n"
            "s = %s\n"
            "z, p = s.init_params(); t = Trainer()\n"
            "ok, why = t.init(s.model_desc(), z, p, np.zeros(s.W * s.H * s.nout, np.float32)); print(ok, why)\n") % (str(ROOT), spec_code)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    return r.stdout


@pytest.mark.parametrize("spec_code,reason", [
    ("ModelSpec(16, 16, [LevelSpec(4, 4, 4)], hidden=(96, 96))", "64 units"),
    ("ModelSpec(16, 16, [LevelSpec(4, 4, 4)], hidden=(64, 64, 64, 64))", "12288 weights"),
    ("ModelSpec(16, 16, [LevelSpec(4, 4, 4)], T=5)", "outputs"),
    ("ModelSpec(16, 16, [LevelSpec(4, 4, 4)], qat_bits=(2, 2, 2, 2))", "nearest"),
    ("ModelSpec(16, 16, [LevelSpec(16, 16, 17, True), LevelSpec(4, 4, 2)])", "16 level-0 channels"),
    ("ModelSpec(20, 20, [LevelSpec(20, 20, 1, True)], dct_q=(50,))", "multiple of 8"),
])
def test_init_rejects_unsupported_models(spec_code, reason):
    """The reference's envelope (cuda/ntc_cuda.cu:751-785): init() returns false with a reason."""
    out = _init_reason(spec_code)
    assert out.startswith("False") and reason in out, out
