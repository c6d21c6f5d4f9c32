"""Test infrastructure (oracle), not product code.

ctypes access to
  * the plain-C restatement of the reference CPU path (oracle/_build/libntc_oracle.so, ntc_oracle.c), and
  * the reference's own CPU trainer compiled behind oracle/ref_shim.cpp (oracle/_ref/libntc_refcpu.so),
used only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs as the checker.
Both libraries are built by oracle/Makefile (`make oracle`, `make ref`).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libntc_oracle.so"
REFCPU_SO = HERE / "_ref" / "libntc_refcpu.so"
REFNOISE_SO = HERE / "_ref" / "libref_noise.so"

_fp = C.POINTER(C.c_float)
_dp = C.POINTER(C.c_double)
_ip = C.POINTER(C.c_int)


class OrLevel(C.Structure):
    _fields_ = [("W", C.c_int), ("H", C.c_int), ("C", C.c_int), ("nearest", C.c_int), ("off", C.c_longlong)]


class OrModel(C.Structure):
    _fields_ = [("W", C.c_int), ("H", C.c_int), ("nlev", C.c_int), ("lv", OrLevel * 3), ("npos", C.c_int),
                ("pos_kind", C.c_int * 16), ("nin", C.c_int), ("nout", C.c_int), ("nhidden", C.c_int),
                ("hidden", C.c_int * 8), ("leak", C.c_float), ("clamp_out", C.c_int), ("cw", C.c_float * 12),
                ("wsum", C.c_float), ("P", C.c_int)]


class OrDct(C.Structure):
    _fields_ = [("C", C.c_int), ("BW", C.c_int), ("BH", C.c_int), ("dc_step", C.c_int), ("deadzone", C.c_int),
                ("lo_w16", C.c_int), ("basis", C.c_float * 64), ("zigzag", C.c_int * 64)]


def f32p(a):
    return None if a is None else np.ascontiguousarray(a, np.float32).ctypes.data_as(_fp)


def build_oracle() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)


def oracle_lib() -> C.CDLL:
    if not ORACLE_SO.exists():
        build_oracle()
    lib = C.CDLL(str(ORACLE_SO))
    lib.or_mix64.restype = C.c_uint64; lib.or_mix64.argtypes = [C.c_uint64]
    lib.or_noise_u32.restype = C.c_uint32
    lib.or_noise_u32.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64]
    lib.or_gauss.restype = C.c_float
    lib.or_gauss.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64]
    lib.or_gauss_block.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64, C.c_size_t, _fp]
    lib.or_loss_subset.restype = C.c_double
    lib.or_qes_index.restype = C.c_int
    lib.or_dct_quantize_block.restype = C.c_int
    lib.or_dct_block_bits.restype = C.c_int
    lib.or_dct_rate_block.restype = C.c_int
    lib.or_dct_rate_block.argtypes = [C.c_void_p, C.c_void_p, C.c_longlong, C.c_int, _fp, _fp, C.c_float, C.c_float,
                                      C.c_void_p, C.c_void_p, _fp]
    return lib


def or_model_of(spec) -> OrModel:
    """The oracle's model struct for a neural_block_textures_b200.ModelSpec."""
    from neural_block_textures_b200.model import POS_KINDS
    m = OrModel()
    m.W, m.H, m.nlev = spec.W, spec.H, len(spec.levels)
    for l, (L, off) in enumerate(zip(spec.levels, spec.offsets)):
        m.lv[l].W, m.lv[l].H, m.lv[l].C, m.lv[l].nearest, m.lv[l].off = L.W, L.H, L.C, int(L.nearest), off
    m.npos = len(spec.pos)
    for q, k in enumerate(spec.pos):
        m.pos_kind[q] = POS_KINDS[k]
    m.nin, m.nout, m.nhidden = spec.nin, spec.nout, len(spec.hidden)
    for l, h in enumerate(spec.hidden):
        m.hidden[l] = h
    m.leak, m.clamp_out = spec.leak, int(spec.clamp_out)
    for c in range(12):
        m.cw[c] = spec.wts[c // 3] if c < spec.nout else 0.0
    m.wsum = float(spec.wsum)
    m.P = spec.P
    return m


class Oracle:
    """The C restatement bound to one model."""

    def __init__(self, spec, target: np.ndarray):
        self.lib = oracle_lib()
        self.spec = spec
        self.m = or_model_of(spec)
        self.mp = C.byref(self.m)
        self.tgt = np.ascontiguousarray(target, np.float32)

    def features(self, z, px, py):
        f = np.zeros(128, np.float32)
        self.lib.or_features(self.mp, f32p(z), C.c_int(int(px)), C.c_int(int(py)), f.ctypes.data_as(_fp))
        return f[: self.spec.nin].copy()

    def decode_full(self, p, z):
        img = np.zeros(self.spec.W * self.spec.H * self.spec.nout, np.float32)
        self.lib.or_decode_full(self.mp, f32p(p), f32p(z), img.ctypes.data_as(_fp))
        return img

    def decode_err(self, p, z):
        e = np.zeros(self.spec.W * self.spec.H, np.float32)
        self.lib.or_decode_err(self.mp, f32p(p), f32p(z), f32p(self.tgt), e.ctypes.data_as(_fp))
        return e

    def loss_subset(self, p, z, idx):
        idx = np.ascontiguousarray(idx, np.int32)
        return self.lib.or_loss_subset(self.mp, f32p(p), f32p(z), f32p(self.tgt), idx.ctypes.data_as(_ip), len(idx))

    def draw_batch(self, seed, it, M):
        out = np.zeros(M, np.int32)
        self.lib.or_draw_batch(C.c_uint64(seed), it, M, self.spec.W * self.spec.H, out.ctypes.data_as(_ip))
        return out

    def es_fitness(self, p, z, seed, it, sigma, pair0, npairs, idx):
        idx = np.ascontiguousarray(idx, np.int32)
        lp = np.zeros(npairs); lm = np.zeros(npairs)
        self.lib.or_es_fitness(self.mp, f32p(p), f32p(z), f32p(self.tgt), C.c_uint64(seed), it, C.c_float(sigma), pair0, npairs,
                               idx.ctypes.data_as(_ip), len(idx), lp.ctypes.data_as(_dp), lm.ctypes.data_as(_dp))
        return lp, lm

    def es_grad(self, seed, it, sigma, dl):
        dl = np.ascontiguousarray(dl, np.float64)
        g = np.zeros(self.spec.P, np.float32)
        self.lib.or_es_grad(self.mp, C.c_uint64(seed), it, C.c_float(sigma), len(dl), dl.ctypes.data_as(_dp), g.ctypes.data_as(_fp))
        return g

    def adam(self, theta, g, m, v, lr, t):
        th = np.ascontiguousarray(theta, np.float32).copy()
        mm = np.ascontiguousarray(m, np.float32).copy()
        vv = np.ascontiguousarray(v, np.float32).copy()
        self.lib.or_adam(th.ctypes.data_as(_fp), f32p(g), mm.ctypes.data_as(_fp), vv.ctypes.data_as(_fp), C.c_size_t(th.size),
                         C.c_float(lr), t)
        return th, mm, vv

    def fd_dl(self, p, z, idx, h, js):
        idx = np.ascontiguousarray(idx, np.int32)
        js = np.ascontiguousarray(js, np.int32)
        dl = np.zeros(len(js)); hh = np.zeros(len(js))
        self.lib.or_fd_dl(self.mp, f32p(p), f32p(z), f32p(self.tgt), idx.ctypes.data_as(_ip), len(idx), C.c_float(h),
                          js.ctypes.data_as(_ip), len(js), dl.ctypes.data_as(_dp), hh.ctypes.data_as(_dp))
        return dl, hh

    def lat_grad(self, p, zdec, seed, step, K, sigma, active_mask):
        g = np.zeros(self.spec.nz, np.float32)
        self.lib.or_lat_grad(self.mp, f32p(p), f32p(zdec), f32p(self.tgt), C.c_uint64(seed), step, K, C.c_float(sigma),
                             C.c_uint(active_mask), g.ctypes.data_as(_fp))
        return g

    def qat_search(self, p, z, bits, grid):
        z = np.ascontiguousarray(z, np.float32).copy()
        b = np.zeros(16, np.int32); b[: len(bits)] = bits
        self.lib.or_qat_search(self.mp, f32p(p), z.ctypes.data_as(_fp), f32p(self.tgt), b.ctypes.data_as(_ip),
                               f32p(np.ascontiguousarray(grid, np.float32).reshape(-1)))
        return z


def noise_u32(seed, stream, step, pair, index):
    return oracle_lib().or_noise_u32(C.c_uint64(seed), stream, step, pair, C.c_uint64(index))


def noise_gauss_block(seed, stream, step, pair, index0, n):
    out = np.zeros(n, np.float32)
    oracle_lib().or_gauss_block(C.c_uint64(seed), stream, step, pair, C.c_uint64(index0), n, out.ctypes.data_as(_fp))
    return out


# ------------------------------------------------------------------ the reference's own CPU code
def refcpu_available() -> bool:
    return REFCPU_SO.exists()


def refcpu_lib() -> C.CDLL:
    lib = C.CDLL(str(REFCPU_SO))
    lib.ref_session_new.restype = C.c_void_p
    lib.ref_session_new.argtypes = [C.c_int, C.c_int, C.c_int, _fp, _fp, C.c_int, _ip, _ip, _ip, _ip, C.c_int, _ip, C.c_char_p,
                                    C.c_float, C.c_int, C.c_int, _ip, C.c_uint]
    lib.ref_session_free.argtypes = [C.c_void_p]
    for n in ["ref_sizes", "ref_set_model", "ref_get_model", "ref_init_like_cli", "ref_features", "ref_decode_full",
              "ref_decode_err", "ref_mlp_reset_adam", "ref_last_batch", "ref_mlp_grad", "ref_lat_step", "ref_set_lat_step_no",
              "ref_qat_search", "ref_iteration", "ref_qes_fit_level", "ref_qes_tables", "ref_qes_refresh", "ref_get_zdec",
              "ref_dct_enable", "ref_dct_fit", "ref_dct_state", "ref_dct_shadow_pull", "ref_dct_analyze", "ref_dct_set_symbols"]:
        getattr(lib, n).argtypes = None
    lib.ref_init_like_cli.argtypes = [C.c_void_p, C.c_float]
    lib.ref_loss_subset.restype = C.c_double
    lib.ref_loss_subset.argtypes = [C.c_void_p, _fp, _ip, C.c_int]
    lib.ref_mlp_step.restype = C.c_double
    lib.ref_mlp_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, _dp]
    lib.ref_mlp_step_fd.restype = C.c_double
    lib.ref_mlp_step_fd.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_float, _dp]
    lib.ref_lat_step.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_float, _fp]
    lib.ref_lat_step_no.restype = C.c_int
    lib.ref_lat_step_no.argtypes = [C.c_void_p]
    lib.ref_set_lat_step_no.argtypes = [C.c_void_p, C.c_int]
    lib.ref_iteration.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, C.c_int, C.c_float, C.c_int,
                                  C.c_float, C.c_float]
    lib.ref_psnr_of_decode.restype = C.c_double
    lib.ref_psnr_of_decode.argtypes = [C.c_void_p, _fp]
    lib.ref_noise_u32.restype = C.c_uint32
    lib.ref_noise_u32.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64]
    lib.ref_noise_gauss.restype = C.c_float
    lib.ref_noise_gauss.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64]
    lib.ref_noise_gauss_block.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64, C.c_size_t, _fp]
    lib.ref_max_threads.restype = C.c_int
    lib.ref_set_threads.argtypes = [C.c_int]
    lib.ref_qes_index.restype = C.c_int
    lib.ref_qes_index.argtypes = [C.c_float, C.c_float, C.c_float, C.c_int]
    lib.ref_dct_quantize_block.restype = C.c_int
    lib.ref_dct_block_bits.restype = C.c_int
    lib.ref_dct_gain_of_code.restype = C.c_double
    lib.ref_dct_quality_scale.restype = C.c_float
    lib.ref_dct_enable.argtypes = [C.c_void_p, _ip, C.c_int, C.c_int, C.c_float, C.c_int, C.c_int, C.c_float]
    lib.ref_dct_fit.argtypes = [C.c_void_p, C.c_int]
    lib.ref_dct_shadow_pull.argtypes = [C.c_void_p, C.c_float]
    lib.ref_qes_fit_level.argtypes = [C.c_void_p, C.c_int, C.c_int]
    lib.ref_es_fitness.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_int, C.c_int, _ip, C.c_int, _dp, _dp]
    lib.ref_fd_dl.argtypes = [C.c_void_p, C.c_float, _ip, C.c_int, _ip, C.c_int, _dp]
    lib.ref_bitrate_stats.argtypes = [C.c_void_p, C.c_int, _dp, _fp]
    lib.ref_mse_of.restype = C.c_double
    lib.ref_mse_of.argtypes = [C.c_void_p, _fp, C.c_int, C.c_int, _dp]
    lib.ref_latent_stats.argtypes = [C.c_void_p, C.c_int, _fp]
    lib.ref_qes_tables.argtypes = [C.c_void_p, C.c_int, _fp, _fp, _fp, _fp]
    return lib


class RefSession:
    """The reference CPU trainer (main.cpp) for one model, through ref_shim.cpp."""

    def __init__(self, spec, target: np.ndarray):
        self.lib = refcpu_lib()
        self.spec = spec
        L = spec.levels
        ai = lambda xs: np.ascontiguousarray(xs, np.int32)
        self._keep = [ai([l.W for l in L]), ai([l.H for l in L]), ai([l.C for l in L]), ai([int(l.nearest) for l in L]),
                      ai(spec.hidden), ai(spec.qat_bits or [0]), np.ascontiguousarray(target, np.float32),
                      np.ascontiguousarray(spec.wts, np.float32)]
        ip = lambda a: a.ctypes.data_as(_ip)
        self.h = self.lib.ref_session_new(spec.W, spec.H, spec.T, f32p(self._keep[6]), f32p(self._keep[7]), len(L),
                                          ip(self._keep[0]), ip(self._keep[1]), ip(self._keep[2]), ip(self._keep[3]),
                                          len(spec.hidden), ip(self._keep[4]), ",".join(spec.pos).encode(), C.c_float(spec.leak),
                                          int(spec.clamp_out), spec.qat, ip(self._keep[5]), spec.seed)
        assert self.h, "ref_session_new failed"

    def close(self):
        if self.h:
            self.lib.ref_session_free(C.c_void_p(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_model(self, z, p):
        self.lib.ref_set_model(C.c_void_p(self.h), f32p(z), f32p(p))

    def get_model(self):
        z = np.zeros(self.spec.nz, np.float32); p = np.zeros(self.spec.P, np.float32)
        self.lib.ref_get_model(C.c_void_p(self.h), z.ctypes.data_as(_fp), p.ctypes.data_as(_fp))
        return z, p

    def features(self, z, px, py):
        f = np.zeros(128, np.float32)
        self.lib.ref_features(C.c_void_p(self.h), f32p(z), C.c_int(px), C.c_int(py), f.ctypes.data_as(_fp))
        return f[: self.spec.nin].copy()

    def decode_full(self, p=None, z=None):
        img = np.zeros(self.spec.W * self.spec.H * self.spec.nout, np.float32)
        self.lib.ref_decode_full(C.c_void_p(self.h), f32p(p), f32p(z), img.ctypes.data_as(_fp))
        return img

    def decode_err(self, p=None, z=None):
        e = np.zeros(self.spec.W * self.spec.H, np.float32)
        self.lib.ref_decode_err(C.c_void_p(self.h), f32p(p), f32p(z), e.ctypes.data_as(_fp))
        return e

    def loss_subset(self, p, idx):
        idx = np.ascontiguousarray(idx, np.int32)
        return self.lib.ref_loss_subset(C.c_void_p(self.h), f32p(p), idx.ctypes.data_as(_ip), len(idx))

    def es_fitness(self, it, sigma, pair0, npairs, idx):
        idx = np.ascontiguousarray(idx, np.int32)
        lp = np.zeros(npairs); lm = np.zeros(npairs)
        self.lib.ref_es_fitness(C.c_void_p(self.h), it, C.c_float(sigma), pair0, npairs, idx.ctypes.data_as(_ip), len(idx),
                                lp.ctypes.data_as(_dp), lm.ctypes.data_as(_dp))
        return lp, lm

    def fd_dl(self, h, idx, js):
        idx = np.ascontiguousarray(idx, np.int32); js = np.ascontiguousarray(js, np.int32)
        dl = np.zeros(len(js))
        self.lib.ref_fd_dl(C.c_void_p(self.h), C.c_float(h), idx.ctypes.data_as(_ip), len(idx), js.ctypes.data_as(_ip), len(js),
                           dl.ctypes.data_as(_dp))
        return dl

    def qes_fit_level(self, l, bits):
        self.lib.ref_qes_fit_level(C.c_void_p(self.h), l, bits)

    def mlp_step(self, it, N, M, sigma, lr):
        ds = C.c_double()
        l = self.lib.ref_mlp_step(C.c_void_p(self.h), it, N, M, C.c_float(sigma), C.c_float(lr), C.byref(ds))
        return l, ds.value

    def mlp_step_fd(self, it, M, h, lr):
        ds = C.c_double()
        l = self.lib.ref_mlp_step_fd(C.c_void_p(self.h), it, M, C.c_float(h), C.c_float(lr), C.byref(ds))
        return l, ds.value

    def last_batch(self, M):
        out = np.zeros(M, np.int32)
        self.lib.ref_last_batch(C.c_void_p(self.h), out.ctypes.data_as(_ip))
        return out

    def mlp_grad(self):
        g = np.zeros(self.spec.P, np.float32)
        self.lib.ref_mlp_grad(C.c_void_p(self.h), g.ctypes.data_as(_fp))
        return g

    def lat_step(self, K, sigma, lr):
        g = np.zeros(self.spec.nz, np.float32)
        self.lib.ref_lat_step(C.c_void_p(self.h), K, C.c_float(sigma), C.c_float(lr), g.ctypes.data_as(_fp))
        return g

    def qat_search(self):
        self.lib.ref_qat_search(C.c_void_p(self.h))

    def iteration(self, it, N, M, mlp_sigma, mlp_lr, fd, fd_h, K, lat_sigma, lat_lr):
        self.lib.ref_iteration(C.c_void_p(self.h), it, N, M, C.c_float(mlp_sigma), C.c_float(mlp_lr), int(fd), C.c_float(fd_h), K,
                               C.c_float(lat_sigma), C.c_float(lat_lr))

    def psnr_of_decode(self, img):
        return self.lib.ref_psnr_of_decode(C.c_void_p(self.h), f32p(img))

    def dct_probe_codes(self, q, dc_step: int = 4, deadzone: int = 0, lam: float = 0.0, rate_es: bool = False,
                        rate_trunc: bool = False, lambda_lo: float = 0.0):
        """The reference's own host probe: turn on the DCT-coded level 0 (ref_dct_enable, with the given dead-zone and
        --dct-lambda settings), fit the scale codes on the current model and decode buffer (Decoder::dct_fit_all),
        return the codes [block][channel]."""
        qa = np.ascontiguousarray(q, np.int32)
        self._dct = (dc_step, deadzone, lam, rate_es, rate_trunc)
        self.lib.ref_dct_enable(C.c_void_p(self.h), qa.ctypes.data_as(_ip), dc_step, deadzone, C.c_float(lam), int(rate_es),
                                int(rate_trunc), C.c_float(lambda_lo))
        self.lib.ref_dct_fit(C.c_void_p(self.h), 1)
        n = (self.spec.W // 8) * (self.spec.H // 8) * self.spec.levels[0].C
        code = np.zeros(n, np.uint8)
        self.lib.ref_dct_state(C.c_void_p(self.h), None, code.ctypes.data_as(C.POINTER(C.c_uint8)), None, None, None, None, None, None, None)
        return code

    def dct_full_state(self):
        """The session's DCT level after dct_probe_codes: (symbols int16 [block][channel][64], codes uint8, steps int32)."""
        nbc = (self.spec.W // 8) * (self.spec.H // 8) * self.spec.levels[0].C
        sym = np.zeros(nbc * 64, np.int16)
        code = np.zeros(nbc, np.uint8)
        step = np.zeros(self.spec.levels[0].C * 16 * 64, np.int32)
        self.lib.ref_dct_state(C.c_void_p(self.h), sym.ctypes.data_as(C.POINTER(C.c_int16)), code.ctypes.data_as(C.POINTER(C.c_uint8)),
                               step.ctypes.data_as(_ip), None, None, None, None, None, None)
        return sym, code, step

    def dct_desc_fields(self) -> dict:
        """The device description of the session's live DCT level as main.cpp's dct_desc_of builds it
        (main.cpp:2947-2956): geometry, rate flags, rate_scale, the host's lam_t16 bit patterns, lo_w16, dead-zone."""
        dc_step, deadzone, lam, rate_es, rate_trunc = self._dct
        lam_t16 = np.zeros(16, np.float32)
        lo = C.c_int()
        self.lib.ref_dct_state(C.c_void_p(self.h), None, None, None, None, lam_t16.ctypes.data_as(_fp), C.byref(lo), None, None, None)
        W, H = self.spec.W, self.spec.H
        rate_scale = np.float32(float(np.float32(lam)) / (16.0 * 65025.0 * W * H)) if rate_es else np.float32(0.0)
        return {"live": 1, "C": self.spec.levels[0].C, "BW": W // 8, "BH": H // 8, "N": 8, "dc_step": dc_step,
                "rate_es": int(rate_es), "rate_trunc": int(rate_trunc), "rate_scale": float(rate_scale), "lam_t16": lam_t16,
                "lo_w16": lo.value, "deadzone": int(deadzone)}

    def dct_shadow_pull(self, f: float) -> None:
        """The --dct-shadow-pull step on the host (main.cpp:4139-4146): z += f (zq - z) on level 0, then the re-snap."""
        self.lib.ref_dct_shadow_pull(C.c_void_p(self.h), C.c_float(f))

    def dct_set_symbols(self, sym, code):
        sym = np.ascontiguousarray(sym, np.int16)
        code = np.ascontiguousarray(code, np.uint8)
        self.lib.ref_dct_set_symbols(C.c_void_p(self.h), sym.ctypes.data_as(C.POINTER(C.c_int16)), code.ctypes.data_as(C.POINTER(C.c_uint8)))

    def dct_analyze(self):
        """dct_analyze as the progress print runs it: (raw, h0, ctx, header) bits."""
        out = np.zeros(4, np.float64)
        self.lib.ref_dct_analyze(C.c_void_p(self.h), out.ctypes.data_as(_dp))
        return tuple(float(v) for v in out)

    BITRATE_FIELDS = ("bpp_fp32", "bpp_q8", "bpp_q8_ent", "bpp_q8_ctx", "bpp_ctx_level0", "bpp_est", "bits_mlp",
                      "bits_raw_latent", "bits_header")

    def bitrate_stats(self, qbits: int = 8):
        """bitrate_stats as the progress print calls it (main.cpp:4171): (fields dict, quantized copy zq)."""
        out = np.zeros(9)
        zq = np.zeros(self.spec.nz, np.float32)
        self.lib.ref_bitrate_stats(C.c_void_p(self.h), qbits, out.ctypes.data_as(_dp), zq.ctypes.data_as(_fp))
        return dict(zip(self.BITRATE_FIELDS, out.tolist())), zq

    def mse_of(self, img, ew: int = 0, eh: int = 0):
        """mse_of (main.cpp:1764-1788) of an image against the session target: (weighted, per-texture array)."""
        tex = np.zeros(4)
        img = np.ascontiguousarray(img, np.float32)
        w = self.lib.ref_mse_of(C.c_void_p(self.h), img.ctypes.data_as(_fp), ew, eh, tex.ctypes.data_as(_dp))
        return w, tex[: self.spec.T].copy()

    def latent_stats(self, l: int):
        """latent_stats (main.cpp:2212-2217) of level l: (mean, sd, max) as float32."""
        msm = np.zeros(3, np.float32)
        self.lib.ref_latent_stats(C.c_void_p(self.h), l, msm.ctypes.data_as(_fp))
        return tuple(msm.tolist())

    def qes_tables(self, l: int, C_: int, bits: int):
        """The fitted --qes table of level l: (lo, hi, range, grid [C][2^bits])."""
        lo = np.zeros(C_, np.float32); hi = np.zeros(C_, np.float32); rg = np.zeros(C_, np.float32)
        grid = np.zeros(C_ << bits, np.float32)
        self.lib.ref_qes_tables(C.c_void_p(self.h), l, lo.ctypes.data_as(_fp), hi.ctypes.data_as(_fp), rg.ctypes.data_as(_fp),
                                grid.ctypes.data_as(_fp))
        return lo, hi, rg, grid

    def zdec(self):
        z = np.zeros(self.spec.nz, np.float32)
        self.lib.ref_get_zdec(C.c_void_p(self.h), z.ctypes.data_as(_fp))
        return z


def psnr_basisu(target: np.ndarray, img: np.ndarray, weights, wsum: float, T: int) -> float:
    """mse_of + psnr_of (main.cpp:1764-1790): 8-bit rounded (lround of clamp * 255), weighted per texture."""
    a = np.rint(np.clip(target.astype(np.float64), 0, 1) * 255.0)
    b = np.clip(img.astype(np.float32), 0, 1)
    b = np.floor(b.astype(np.float64) * np.float32(255.0) + 0.5)
    a = np.floor(np.clip(target, 0, 1).astype(np.float32) * np.float32(255.0) + np.float32(0.5)).astype(np.float64)
    d = (a - b).reshape(-1, T, 3)
    sse = (d * d).sum(axis=(0, 2))
    npix = d.shape[0]
    ws = sum(w * s for w, s in zip(weights, sse))
    mse = ws / (3.0 * wsum * npix)
    return 100.0 if mse <= 0 else min(100.0, max(0.0, 10.0 * np.log10(255.0 * 255.0 / mse)))
