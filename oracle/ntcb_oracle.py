"""Test infrastructure (oracle), not product code.

A Python restatement of reading the reference's .ntcb container (the layout of ntcb_read_header / ntcb_restore,
main.cpp:2521-2629 and 2762-2855: little-endian fields, LSB-first bit fields, 6-bit sync markers, the DC / run /
magnitude / sign / EOB token stream, fp16 weights), followed by the oracle's C decode (or_decode_full) and DCT
reconstruction (or_dct_recon_level0) and the reference's RGB8 rounding. The checker of the device decoder
(ntcb_decoder_*), pinned against the reference's own decoder output recorded in tests/golden/ntcb/.
"""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np

from neural_block_textures_b200 import dct
from neural_block_textures_b200.model import LevelSpec, ModelSpec

from .oracle import Oracle, OrDct, f32p, or_model_of
from .print_stats import lround, q8_value

SYNC_LEVEL, SYNC_CHANNEL, SYNC_MLP, SYNC_END = 0x2B, 0x16, 0x31, 0x0C


def _sync(base: int, level: int, channel: int) -> int:
    return (base + 13 * level + 7 * channel) & 63


class _BitStream:
    def __init__(self, data: bytes, begin: int, end: int):
        self.data, self.pos, self.end, self.acc, self.have = data, begin, end, 0, 0

    def get(self, n: int) -> int:
        while self.have < n:
            if self.pos >= self.end:
                raise ValueError("bit stream runs past its section")
            self.acc |= self.data[self.pos] << self.have
            self.pos += 1
            self.have += 8
        v = self.acc & ((1 << n) - 1)
        self.acc >>= n
        self.have -= n
        return v


def _half(h: int) -> np.float32:
    return np.frombuffer(struct.pack("<H", h), np.float16)[0].astype(np.float32)


def read(data: bytes):
    """Returns (header dict, ModelSpec, z, p). z holds every level; a DCT level 0 is reconstructed by the oracle."""
    u8 = lambda o: data[o]
    u16 = lambda o: struct.unpack_from("<H", data, o)[0]
    u32 = lambda o: struct.unpack_from("<I", data, o)[0]
    f32 = lambda o: struct.unpack_from("<f", data, o)[0]
    assert u32(0) == 0x6263746E
    h = {"version": u16(4), "H": u16(6), "img_w": u32(8), "img_h": u32(12), "src_w": u32(16), "src_h": u32(20),
         "T": u8(34), "nlevels": u8(35), "clamp": u8(37), "nhidden": u8(38), "leak": f32(40), "nin": u32(44), "nout": u32(48)}
    o = 52 + h["T"]
    hidden = [u16(o + 2 * i) for i in range(h["nhidden"])]
    o += 2 * h["nhidden"]
    poslen = u16(o)
    pos = data[o + 2: o + 2 + poslen].decode()
    o += 2 + poslen
    levels = []
    for _ in range(h["nlevels"]):
        L = {"W": u32(o), "H": u32(o + 4), "C": u16(o + 8), "nearest": u8(o + 10), "mode": u8(o + 11)}
        o += 12
        L["bits"] = list(data[o: o + L["C"]])
        o += L["C"]
        if L["mode"] == 3:
            L["dc_step"] = u8(o)
            o += 1
            L["deadzone"] = u8(o) & 1 if h["version"] >= 2 else 1
            o += 1 if h["version"] >= 2 else 0
            L["q"] = list(data[o: o + L["C"]])
            o += L["C"]
        if L["mode"] in (0, 1):
            L["lo"] = [np.float32(f32(o + 8 * c)) for c in range(L["C"])]
            L["hi"] = [np.float32(f32(o + 8 * c + 4)) for c in range(L["C"])]
            o += 8 * L["C"]
        if L["mode"] == 2:
            L["palette"] = []
            for c in range(L["C"]):
                n = 1 << L["bits"][c]
                L["palette"].append(np.frombuffer(data, np.float32, n, o).copy())
                o += 4 * n
        levels.append(L)
    assert o == h["H"]
    kinds = [k for k in pos.split(",") if k and k != "none"]
    spec = ModelSpec(h["img_w"], h["img_h"], [LevelSpec(L["W"], L["H"], L["C"], bool(L["nearest"])) for L in levels],
                     T=h["T"], hidden=tuple(hidden), pos=tuple(kinds), leak=float(np.float32(h["leak"])), clamp_out=bool(h["clamp"]))
    z = np.zeros(spec.nz, np.float32)
    pos_at = h["H"]
    dct_state = None
    for l, (L, off) in enumerate(zip(levels, spec.offsets)):
        kind, coding, lvl, res, blen = data[pos_at], data[pos_at + 1], data[pos_at + 2], data[pos_at + 3], u32(pos_at + 4)
        assert (kind, coding, lvl, res) == (1, 0, l, 0)
        body = pos_at + 8
        bs = _BitStream(data, body, body + blen)
        assert bs.get(6) == _sync(SYNC_LEVEL, l, 0)
        zl = z[off: off + L["W"] * L["H"] * L["C"]].reshape(L["H"] * L["W"], L["C"])
        if L["mode"] == 3:
            nb = (L["W"] // 8) * (L["H"] // 8)
            dcb = 0
            while (1 << dcb) < 512 // L["dc_step"] + 1:
                dcb += 1
            zz = dct.zigzag_table()
            sym = np.zeros((nb, L["C"], 64), np.int16)
            code = np.zeros((nb, L["C"]), np.uint8)
            for c in range(L["C"]):
                assert bs.get(6) == _sync(SYNC_CHANNEL, l, c)
                for b in range(nb):
                    code[b, c] = bs.get(4)
                for b in range(nb):
                    sym[b, c, 0] = bs.get(dcb)
                    p = 1
                    while p < 64:
                        run = bs.get(7)
                        if run == 64:
                            break
                        p += run
                        mag, sign = bs.get(8) + 1, bs.get(1)
                        sym[b, c, zz[p]] = -mag if sign else mag
                        p += 1
            dct_state = (L, sym, code)
        else:
            for c in range(L["C"]):
                b = L["bits"][c]
                idx = np.array([bs.get(b) for _ in range(L["W"] * L["H"])], np.int64)
                if L["mode"] == 2:
                    zl[:, c] = L["palette"][c][idx]
                else:
                    lo, hi = L["lo"][c], L["hi"][c]
                    rng = max(np.float32(hi - lo), np.float32(1e-6))
                    zl[:, c] = q8_value(idx, lo, rng, (1 << b) - 1)
        assert bs.get(6) == _sync(SYNC_END, l, 0)
        pos_at = body + blen
    kind, blen = data[pos_at], u32(pos_at + 4)
    assert kind == 2
    bs = _BitStream(data, pos_at + 8, pos_at + 8 + blen)
    assert bs.get(6) == _sync(SYNC_MLP, h["nlevels"], 0)
    p = np.array([_half(bs.get(16)) for _ in range(spec.P)], np.float32)
    assert bs.get(6) == _sync(SYNC_END, h["nlevels"], 0)
    assert pos_at + 8 + blen == len(data)
    if dct_state is not None:
        L, sym, code = dct_state
        T = OrDct()
        T.C, T.BW, T.BH, T.dc_step, T.deadzone, T.lo_w16 = L["C"], L["W"] // 8, L["H"] // 8, L["dc_step"], L["deadzone"], 0
        T.basis[:] = dct.basis_table().tolist()
        T.zigzag[:] = dct.zigzag_table().tolist()
        steps = np.concatenate([dct.build_steps(q, L["dc_step"]).reshape(-1) for q in L["q"]]).astype(np.int32)
        orc = Oracle(spec, np.zeros(spec.W * spec.H * spec.nout, np.float32))
        orc.lib.or_dct_recon_level0(C.byref(T), orc.mp, z.ctypes.data_as(C.POINTER(C.c_float)),
                                    np.ascontiguousarray(sym).ctypes.data_as(C.POINTER(C.c_int16)),
                                    np.ascontiguousarray(code).ctypes.data_as(C.POINTER(C.c_uint8)),
                                    steps.ctypes.data_as(C.POINTER(C.c_int)))
    return h, spec, z, p


def decode_rgb8(data: bytes) -> np.ndarray:
    """[T][src_h][src_w][3]: the oracle decode of the container, rounded as the reference writes its PNGs."""
    h, spec, z, p = read(data)
    orc = Oracle(spec, np.zeros(spec.W * spec.H * spec.nout, np.float32))
    img = orc.decode_full(p, z).reshape(spec.H, spec.W, spec.T, 3)[: h["src_h"], : h["src_w"]]
    q = lround(np.minimum(np.float32(1.0), np.maximum(np.float32(0.0), img)) * np.float32(255.0)).astype(np.uint8)
    return np.ascontiguousarray(q.transpose(2, 0, 1, 3))
