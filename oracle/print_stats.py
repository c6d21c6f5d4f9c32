"""Test infrastructure (oracle), not product code.

A numpy restatement of the reference trainer's progress-print statistics (main.cpp:4155-4205), the checker of
ntcb_print_stats: bitrate_stats in its progress-print form (main.cpp:2272-2352, g_ctx_stats off), mse_of
(main.cpp:1764-1788), latent_stats (main.cpp:2212-2217), the --qat off-grid count (main.cpp:4196-4200) and the
totals of the DCT bit simulator (dct_analyze, main.cpp:1080-1175) that bitrate_stats charges a live DCT level 0.
The quantizers follow the reference's strict-FP forms (main.cpp:446-482): every float32 operation is one
IEEE operation here (numpy float32 arithmetic does not contract), and lround is computed in float64, where
|x| + 0.5 is exact for a float32 x. Pinned against the reference's own functions through
oracle/ref_shim.cpp (tests/test_print_stats.py).
"""
from __future__ import annotations

import math

import numpy as np

F32 = np.float32


def lround(x: np.ndarray) -> np.ndarray:
    """C lround of float32 values: half away from zero."""
    x = np.asarray(x, np.float64)
    return (np.sign(x) * np.floor(np.abs(x) + 0.5)).astype(np.int64)


def q8_index(z, lo, rng, levels):
    """q8_index (main.cpp:478-481): lround((z - lo) / range * levels), clamped."""
    r = ((np.asarray(z, F32) - F32(lo)) / F32(rng)) * F32(levels)
    return np.clip(lround(r), 0, levels)


def q8_value(k, lo, rng, levels):
    """q8_value (main.cpp:482): lo + k / (float)levels * range."""
    return F32(lo) + (np.asarray(k, F32) / F32(levels)) * F32(rng)


def qes_index(v, lo, rng, levels):
    """qes_index (main.cpp:448-453): round-half-even, clamped in float."""
    r = np.rint(((np.asarray(v, F32) - F32(lo)) / F32(rng)) * F32(levels))
    return np.where(r <= 0, 0, np.where(r >= levels, levels, r)).astype(np.int64)


def qat_index(v, bits):
    """qat_index (main.cpp:2060-2064): lround((v + 1) * 0.5 * levels), clamped."""
    levels = (1 << bits) - 1
    r = (np.asarray(v, F32) + F32(1.0)) * F32(0.5) * F32(levels)
    return np.clip(lround(r), 0, levels)


def _h0(hist: np.ndarray, ntex: float) -> float:
    """-sum hist[q] log2(hist[q] / ntex) over the nonzero bins in index order (main.cpp:2324-2326)."""
    h = 0.0
    for c in hist.tolist():
        if c:
            h -= c * math.log2(c / ntex)
    return h


def bitrate_stats(spec, z: np.ndarray, zdec: np.ndarray, P: int, level_bits, qes=None):
    """bitrate_stats (main.cpp:2272-2352) with g_ctx_stats off. level_bits[l] = lbits of continuous levels;
    qes = {level: (bits, lo[C], range[C])} for live --qes levels. Returns (fields dict, zq)."""
    npix = float(spec.W * spec.H)
    s = {"bits_mlp": P * 16.0, "bpp_fp32": (spec.nz * 32.0 + P * 32.0) / npix, "bpp_ctx_level0": 0.0}
    zq = np.zeros(spec.nz, np.float32)
    ent = header = raw = ctx = est = 0.0
    for l, (L, off) in enumerate(zip(spec.levels, spec.offsets)):
        fixed = l == 0 and bool(spec.qat_bits)
        q = None if (qes is None or fixed) else qes.get(l)
        lbits = level_bits[l]
        zl = z[off: off + L.size].reshape(L.H * L.W, L.C)
        zdl = zdec[off: off + L.size].reshape(L.H * L.W, L.C)
        ql = zq[off: off + L.size].reshape(L.H * L.W, L.C)
        ntex = float(L.W * L.H)
        if not fixed and q is None:
            raw += L.size * float(lbits)
        for c in range(L.C):
            bits = spec.qat_bits[c] if fixed else (q[0] if q is not None else lbits)
            levels = (1 << bits) - 1
            if fixed or q is not None:
                raw += ntex * float(bits)
            v = zl[:, c]
            if fixed:
                idx = qat_index(v, bits)
                ql[:, c] = v
            elif q is not None:
                idx = qes_index(v, q[1][c], q[2][c], levels)
                ql[:, c] = zdl[:, c]
            else:
                finite = v[~np.isnan(v)]
                lo = min(F32(1e30), finite.min()) if finite.size else F32(1e30)
                hi = max(F32(-1e30), finite.max()) if finite.size else F32(-1e30)
                rng = max(F32(hi - lo), F32(1e-6))
                idx = q8_index(v, lo, rng, levels)
                ql[:, c] = q8_value(idx, lo, rng, levels)
            h0 = _h0(np.bincount(idx, minlength=levels + 1), ntex)
            ent += h0
            ctx += h0
            if l == 0:
                s["bpp_ctx_level0"] += h0 / npix
                est += h0
            else:
                g = idx.reshape(L.H, L.W)
                lf = np.full_like(g, -1); lf[:, 1:] = g[:, :-1]
                up = np.full_like(g, -1); up[1:, :] = g[:-1, :]
                pred = np.where((lf >= 0) & (up >= 0), (lf + up) // 2, np.where(lf >= 0, lf, np.where(up >= 0, up, 0)))
                est += _h0(np.bincount(((g - pred) & levels).reshape(-1), minlength=levels + 1), ntex)
        if not fixed:
            header += L.C * 2 * 32.0
    s["bpp_q8"] = (raw + header + s["bits_mlp"]) / npix
    s["bpp_q8_ent"] = (ent + header + s["bits_mlp"]) / npix
    s["bpp_q8_ctx"] = (ctx + header + s["bits_mlp"]) / npix
    s["bpp_est"] = (est + header + s["bits_mlp"]) / npix
    s["bits_raw_latent"], s["bits_header"] = raw, header
    return s, zq


def mse_of(spec, target: np.ndarray, img: np.ndarray, ew: int = 0, eh: int = 0):
    """mse_of (main.cpp:1764-1788): 8-bit rounding of both images, integer squared error per texture over the
    extent ew x eh. Returns (weighted, per-texture array, the integer squared-error sums)."""
    W, H, T = spec.W, spec.H, spec.T
    ew = W if ew <= 0 or ew > W else ew
    eh = H if eh <= 0 or eh > H else eh
    def q8(a):
        a = np.asarray(a, F32).reshape(H, W, T, 3)[:eh, :ew]
        return lround(np.minimum(F32(1.0), np.maximum(F32(0.0), a)) * F32(255.0))
    d = q8(target) - q8(img)
    sse = (d * d).sum(axis=(0, 1, 3)).astype(np.float64)
    npe = float(ew * eh)
    tex = sse / (3.0 * npe)
    ws = 0.0
    for t in range(T):
        ws += float(F32(spec.wts[t])) * sse[t]
    return ws / (3.0 * float(spec.wsum) * npe), tex, sse


def latent_stats(zl: np.ndarray):
    """latent_stats (main.cpp:2212-2217): serial double sums, max |v|; (mean, sd, max) as float32 values."""
    v = np.asarray(zl, F32).astype(np.float64)
    n = float(v.size)
    s = float(np.cumsum(v)[-1]) if v.size else 0.0
    s2 = float(np.cumsum(v * v)[-1]) if v.size else 0.0
    mx = float(np.nanmax(np.abs(np.asarray(zl, F32)))) if v.size else 0.0
    mean = float(F32(s / n))
    sd = float(F32(math.sqrt(max(0.0, s2 / n - (s / n) * (s / n)))))
    return mean, sd, float(F32(max(mx, 0.0)))


def qat_off_grid(spec, z: np.ndarray, grid: np.ndarray) -> int:
    """Level-0 values whose --qat grid snap differs from the value (main.cpp:4196-4200)."""
    L = spec.levels[0]
    z0 = z[: L.size].reshape(-1, L.C)
    n = 0
    for c, b in enumerate(spec.qat_bits):
        n += int(np.sum(grid[b, qat_index(z0[:, c], b)] != z0[:, c]))
    return n


def dct_bits(sym: np.ndarray, code: np.ndarray, C: int, BW: int, BH: int, dc_step: int, zigzag: np.ndarray):
    """dct_analyze's (raw, h0, ctx, header) bit totals as the progress print runs it (main.cpp:1080-1175, g_ctx_stats
    off: the code plane's order-0 figure stands in for its context figure). sym: int16 [block][channel][64] in
    natural order, code: uint8 [block][channel], zigzag[p] = the natural index of zigzag position p. Per channel:
    the DC residual against the left block (the upper one in the first column, 0 first), the ACs as (run, |q|)
    tokens in zigzag order with the zigzag position of the previous nonzero as context, an EOB unless the last
    nonzero is at 63; each token charged -log2(count / total) of its symbol (summed here as count x code length)."""
    nb = BW * BH
    sym = np.asarray(sym, np.int64).reshape(nb, C, 64)
    cl0 = lambda c, t: -math.log2(c / t) if c and t else 0.0
    ent = lambda h, t: sum(float(v) * cl0(float(v), float(t)) for v in h if v)
    dc_raw_bits = 0
    while (1 << dc_raw_bits) < 512 // dc_step + 1:
        dc_raw_bits += 1
    raw = h0 = ctx = header = 0.0
    for c in range(C):
        run = np.zeros(65, np.int64); mag = np.zeros(257, np.int64)
        cr = np.zeros((64, 65), np.int64); cm = np.zeros((64, 257), np.int64)
        dcr = np.zeros(4097, np.int64); chist = np.zeros(16, np.int64)
        nrun = neob = 0
        for b in range(nb):
            s = sym[b, c]
            bx, by = b % BW, b // BW
            pred = sym[b - 1, c, 0] if bx > 0 else (sym[b - BW, c, 0] if by > 0 else 0)
            dcr[max(0, min(4096, int(s[0]) - int(pred) + 2048))] += 1
            chist[min(int(code[b * C + c]), 15)] += 1
            r = prev = lnz = 0
            for p in range(1, 64):
                q = int(s[zigzag[p]])
                if q == 0:
                    r += 1
                    continue
                m = min(256, abs(q))
                run[r] += 1; mag[m] += 1; cr[prev, r] += 1; cm[prev, m] += 1
                nrun += 1; lnz = p; prev = p; r = 0
            if lnz < 63:
                run[64] += 1; cr[prev, 64] += 1; neob += 1
        dc, cd = ent(dcr, nb), ent(chist, nb)
        run0, mag0 = ent(run, nrun + neob), ent(mag, nrun)
        runc = sum(ent(cr[k], cr[k].sum()) for k in range(64))
        magc = sum(ent(cm[k], cm[k].sum()) for k in range(64))
        raw += nb * dc_raw_bits + 16 * nrun + 7 * neob + 4 * nb + 96
        h0 += dc + run0 + mag0 + nrun + cd + 96
        ctx += dc + runc + magc + nrun + cd + 96
        header += 96
    return raw, h0, ctx, header
