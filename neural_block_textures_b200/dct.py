"""Host tables of the DCT-coded level 0 (--dct-q), computed from their definitions.

The reference stores them as literal float bit patterns (main.cpp:654-690) and uploads them to the
device; the device never recomputes them. Here they are derived from the same definitions:
  * basis B[u][x] = alpha(u) cos(pi (2x + 1) u / 16), alpha(0) = sqrt(1/8), alpha(u > 0) = sqrt(2/8),
    evaluated in double and rounded once to float;
  * the zigzag order (zigzag position -> natural index u * 8 + v) by anti-diagonals, odd diagonals reversed;
  * the per-code block scale A_k = 1 / g_k with g_k = (14 / 64) 2^(0.6 k), rounded once;
  * the JPEG Annex K luminance table (with the DC entry 4) and the libjpeg quality scaling, which give the
    integer step tables per (channel, code) (dct_build_steps, main.cpp:747-781, strict float order);
  * the --dct-lambda per-code thresholds lam_t16[k] = L / (16 g_k^2).
tests/test_dct_tables.py checks every table against the reference's own values.
"""
from __future__ import annotations

import math

import numpy as np

JPEG_LUMA = np.array([
    [4, 11, 10, 16, 24, 40, 51, 61],
    [12, 12, 14, 19, 26, 58, 60, 55],
    [14, 13, 16, 24, 40, 57, 69, 56],
    [14, 17, 22, 29, 51, 87, 80, 62],
    [18, 22, 37, 56, 68, 109, 103, 77],
    [24, 35, 55, 64, 81, 104, 113, 92],
    [49, 64, 78, 87, 103, 121, 120, 101],
    [72, 92, 95, 98, 112, 100, 103, 99],
], dtype=np.int32)

G_FLOOR = 14.0 / 64.0


def basis_table() -> np.ndarray:
    b = np.zeros(64, np.float32)
    for u in range(8):
        a = math.sqrt(1.0 / 8.0) if u == 0 else math.sqrt(2.0 / 8.0)
        for x in range(8):
            b[u * 8 + x] = np.float32(a * math.cos(math.pi * (2 * x + 1) * u / 16.0))
    return b


def zigzag_table() -> np.ndarray:
    out = []
    for s in range(15):
        xs, xe = (0, s) if s < 8 else (s - 7, 7)
        diag = [x + (s - x) * 8 for x in range(xs, xe + 1)]
        out += diag[::-1] if s & 1 else diag
    return np.array(out, np.int32)


def gain_of_code(k: int) -> float:
    return G_FLOOR * 2.0 ** (0.6 * k)


def ak_table() -> np.ndarray:
    return np.array([np.float32(1.0 / gain_of_code(k)) for k in range(16)], np.float32)


def quality_scale(q: int) -> np.float32:
    q = max(1, min(100, q))
    f32 = np.float32
    S = f32(5000.0) / f32(q) if q < 50 else f32(200.0) - f32(2.0) * f32(q)
    return f32(S * f32(1.0 / 100.0))


def build_steps(q: int, dc_step: int) -> np.ndarray:
    """The 16 step tables of one channel, [16][64] ints (dct_build_steps_scaled at N = 8)."""
    f32 = np.float32
    ak = ak_table()
    out = np.zeros((16, 64), np.int32)
    for k in range(16):
        ls = f32(quality_scale(q) * ak[k])
        for u in range(8):
            for v in range(8):
                if u == 0 and v == 0:
                    out[k, 0] = dc_step
                    continue
                if q >= 100:
                    out[k, u * 8 + v] = 1
                    continue
                i, j = min(f32(v), f32(7)), min(f32(u), f32(7))
                i0, j0 = int(i), int(j)
                i1, j1 = min(i0 + 1, 7), min(j0 + 1, 7)
                ti, tj = f32(i - f32(i0)), f32(j - f32(j0))
                a = f32(f32(f32(1) - ti) * f32(JPEG_LUMA[j0, i0])) + f32(ti * f32(JPEG_LUMA[j0, i1]))
                b = f32(f32(f32(1) - ti) * f32(JPEG_LUMA[j1, i0])) + f32(ti * f32(JPEG_LUMA[j1, i1]))
                base = f32(f32(f32(1) - tj) * a) + f32(tj * b)
                sf = f32(f32(base * ls) + f32(0.5))
                if not sf >= 1.0:
                    sf = f32(1.0)
                if sf > 1048576.0:
                    sf = f32(1048576.0)
                out[k, u * 8 + v] = max(1, int(sf))
    return out


def lambda_recipe(qs: list[int]) -> float:
    """The default --dct-lambda (main.cpp:3389-3392): min over the channels of min(0.5, 7.5 S(q)^2), in float."""
    L = np.float32(0.5)
    for q in qs:
        S = quality_scale(q)
        L = min(L, np.float32(np.float32(7.5) * S * S))
    return float(L)


def lam_t16(lam: float, rate_trunc: bool) -> np.ndarray:
    return np.array([np.float32(lam / (gain_of_code(k) ** 2 * 16.0)) if rate_trunc else 0.0 for k in range(16)], np.float32)
