""".ntcb containers on the host (no GPU): the oracle reader against the reference's own decoder output, this
library's parser (ntcb_container_info) against the oracle, its refusals of damaged files, and the DCT tables the
device decoder builds against the pinned Python ones.

Fixtures: tests/golden/ntcb/*.ntcb written by the reference trainer (--write-ntcb) and *.npz with the reference
decoder's RGB8 (ntc_decode --exact) and the trainer's recon_q_final (tests/golden/ntcb/make_fixtures.py)."""
import struct
from pathlib import Path

import numpy as np
import pytest

from neural_block_textures_b200 import dct, ntcb
from oracle import ntcb_oracle

FIX = Path(__file__).resolve().parent / "golden" / "ntcb"
CASES = ["qat_q8", "qes", "dct", "dct2_dz0", "material"]
MODES = {"qat_q8": [2, 0], "qes": [1, 1], "dct": [3, 1], "dct2_dz0": [3, 1], "material": [2, 0]}


def _data(name: str) -> bytes:
    return (FIX / f"{name}.ntcb").read_bytes()


def _rehash(b: bytearray) -> bytes:
    """Rewrites file_bytes (offset 24) and the FNV-1a hash (offset 28, computed with itself read as zero)."""
    b[24:28] = struct.pack("<I", len(b))
    h = 2166136261
    for i, v in enumerate(b):
        h = ((h ^ (0 if 28 <= i < 32 else v)) * 16777619) & 0xFFFFFFFF
    b[28:32] = struct.pack("<I", h)
    return bytes(b)


@pytest.mark.parametrize("name", CASES)
def test_oracle_reader_matches_reference_decoder(name):
    g = np.load(FIX / f"{name}.npz")
    o = ntcb_oracle.decode_rgb8(_data(name))
    assert np.array_equal(o, g["decoder_rgb8"])
    assert np.array_equal(g["decoder_rgb8"], g["trainer_rgb8"]), "the reference's decoder and trainer agree"


@pytest.mark.parametrize("name", CASES)
def test_container_info_matches_oracle(name):
    data = _data(name)
    i = ntcb.container_info(data)
    h, spec, z, p = ntcb_oracle.read(data)
    assert (i.version, i.img_w, i.img_h, i.src_w, i.src_h, i.T) == (h["version"], h["img_w"], h["img_h"], h["src_w"], h["src_h"], spec.T)
    assert i.nlevels == len(spec.levels) and [i.lv_mode[l] for l in range(i.nlevels)] == MODES[name]
    for l, L in enumerate(spec.levels):
        assert (i.lv_W[l], i.lv_H[l], i.lv_C[l], bool(i.lv_nearest[l])) == (L.W, L.H, L.C, L.nearest)
    assert (i.nin, i.nout, i.nz, i.nweights) == (spec.nin, spec.nout, spec.nz, spec.P)
    assert list(i.hidden)[: i.nhidden] == list(spec.hidden)
    assert np.float32(i.leak) == np.float32(spec.leak) and bool(i.clamp_out) == spec.clamp_out


def _refused(data: bytes, what: str):
    with pytest.raises(ntcb.NtcbError, match=what):
        ntcb.container_info(data)


def test_container_refusals():
    data = _data("qat_q8")
    b = bytearray(data); b[len(b) // 2] ^= 0x10
    _refused(bytes(b), "hash")
    _refused(data[:-1], "file_bytes")
    _refused(b"xxxx" + data[4:], "magic")
    _refused(data[:6], "shorter than 8")
    b = bytearray(data); b[4] = 3
    _refused(_rehash(b), "version 3")
    _refused(_rehash(bytearray(data) + b"\0\0"), "trailing bytes")
    # the level-0 sync marker (first 6 bits of the first section body) flipped, the file re-hashed
    H = struct.unpack_from("<H", data, 6)[0]
    b = bytearray(data); b[H + 8] ^= 0x01
    _refused(_rehash(b), "sync marker mismatch before level 0")
    # a section header that names the wrong level
    b = bytearray(data); b[H + 2] = 1
    _refused(_rehash(b), "unexpected section header")
    # an activation other than leaky
    b = bytearray(data); b[36] = 1
    _refused(_rehash(b), "out of range")


def test_dct_container_refusals():
    data = _data("dct")
    i = ntcb.container_info(data)
    assert i.lv_mode[0] == 3
    # a run symbol of 63 (neither 0..62 nor the EOB 64) right after the first block's DC: find the level-0 body
    H = struct.unpack_from("<H", data, 6)[0]
    b = bytearray(data)
    b[H + 8 + 1] = 0xFF   # bits 8..15 of the body: the sync marker, channel marker and scale codes follow
    with pytest.raises(ntcb.NtcbError):
        ntcb.container_info(_rehash(b))


@pytest.mark.parametrize("q", [1, 20, 49, 50, 51, 90, 100])
def test_decoder_dct_tables_match_pinned_tables(q):
    basis, zz, steps = ntcb.dct_tables(q, 4)
    assert np.array_equal(basis.view(np.uint32), dct.basis_table().view(np.uint32))
    assert np.array_equal(zz, dct.zigzag_table())
    assert np.array_equal(steps, dct.build_steps(q, 4))
