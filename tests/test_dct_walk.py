"""The DCT kernels' truncation walk and token count (csrc/kernels_snap.cu: group_mask, quantize_group, mask_bits) run
over the block's 64-bit zigzag mask of nonzero ACs instead of over all 63 zigzag positions with a backward search
per nonzero, as the reference does (dct_truncate_block, main.cpp:850-869; dct_block_bits, main.cpp:829-848). This
checks on the host that both formulations make the same decisions and the same token counts on random blocks: the
reference's control flow restated position by position against the mask form (nearest nonzero below p from the
original mask, nearest kept nonzero above p as the walk's state, bits from the final mask), with the same float32
comparison dD < lam16 * saved. The device kernels themselves are held bit-exact to the reference's host code on the
GPU (tests/test_gpu_cuda_check.py DCT lines, tests/test_gpu_bench_shapes.py)."""
import numpy as np

from neural_block_textures_b200 import dct

ZZ = [int(x) for x in dct.zigzag_table()]
C_SIGN, C_EOB = 16, 32


def floor_log2(v: int) -> int:
    return v.bit_length() - 1 if v > 0 else 0


def c_run(r: int) -> int:
    return 16 * (2 * floor_log2(r + 1) + 1)


def c_mag(m: int) -> int:
    return 16 * (2 * floor_log2(m) + 1)


def lo_weight(tok: int, p: int, lo16: int) -> int:
    return (tok * lo16 + 8) >> 4 if p <= 2 else tok


def token(r: int, q: int, p: int, lo16: int) -> int:
    return lo_weight(c_run(r) + c_mag(min(256, abs(q))) + C_SIGN, p, lo16)


def below(lhs: np.float32, lam16: np.float32, saved: int) -> bool:
    return bool(lhs < np.float32(lam16 * np.float32(saved)))


def walk_positions(sym, dd, lam16, lo16):
    """main.cpp:850-869 restated: every zigzag position from 63 down, a backward search for the previous nonzero."""
    sym = list(sym)
    nt, nxt = 0, 64
    for p in range(63, 0, -1):
        k = ZZ[p]
        q = sym[k]
        if q == 0:
            continue
        prev = 0
        for j in range(p - 1, 0, -1):
            if sym[ZZ[j]] != 0:
                prev = j
                break
        r1 = p - prev - 1
        tok = token(r1, q, p, lo16)
        saved = tok - (C_EOB if p == 63 else 0) if nxt == 64 else tok + c_run(nxt - p - 1) - c_run(nxt - p - 1 + r1 + 1)
        if below(dd[k], lam16, saved):
            sym[k] = 0
            nt += 1
        else:
            nxt = p
    return sym, nt


def bits_positions(sym, lo16):
    """main.cpp:829-848 restated: zero runs counted position by position."""
    bits, run, lnz = 0, 0, 0
    for p in range(1, 64):
        q = sym[ZZ[p]]
        if q == 0:
            run += 1
            continue
        bits += token(run, q, p, lo16)
        lnz, run = p, 0
    return bits + (C_EOB if lnz < 63 else 0)


def walk_mask(sym, dd, lam16, lo16):
    """The kernels' form: the zigzag mask of nonzero ACs, its set bits walked from the top."""
    sym = list(sym)
    mask = 0
    for p in range(1, 64):
        if sym[ZZ[p]] != 0:
            mask |= 1 << p
    fin, m, nt, nxt = mask, mask, 0, 64
    while m:
        p = m.bit_length() - 1
        m &= ~(1 << p)
        prev = m.bit_length() - 1 if m else 0
        k = ZZ[p]
        r1 = p - prev - 1
        tok = token(r1, sym[k], p, lo16)
        saved = tok - (C_EOB if p == 63 else 0) if nxt == 64 else tok + c_run(nxt - p - 1) - c_run(nxt - p - 1 + r1 + 1)
        if below(dd[k], lam16, saved):
            sym[k] = 0
            fin &= ~(1 << p)
            nt += 1
        else:
            nxt = p
    return sym, nt, mask, fin


def bits_mask(sym, fin, lo16):
    bits, prevp, m = 0, 0, fin
    while m:
        p = (m & -m).bit_length() - 1
        m &= m - 1
        bits += token(p - prevp - 1, sym[ZZ[p]], p, lo16)
        prevp = p
    return bits + (C_EOB if prevp < 63 else 0)


def test_zigzag_is_a_permutation_from_dc():
    assert sorted(ZZ) == list(range(64)) and ZZ[0] == 0


def test_mask_walk_matches_position_walk():
    rng = np.random.default_rng(17)
    for trial in range(3000):
        density = rng.choice([0.02, 0.1, 0.3, 0.7, 1.0])
        sym = [int(v) for v in np.where(rng.random(64) < density, rng.integers(-300, 301, 64), 0)]
        if trial % 7 == 0:
            sym[ZZ[63]] = int(rng.integers(1, 4))       # zigzag 63 occupied: the EOB term of the last token
        dd = (rng.standard_normal(64) * rng.choice([1.0, 50.0, 2000.0])).astype(np.float32)
        lam16 = np.float32(rng.choice([0.0, 0.05, 0.5, 3.0, 40.0]))
        lo16 = int(rng.choice([8, 16, 24]))
        nz_before = sum(1 for k in range(1, 64) if sym[k] != 0)
        s_ref, nt_ref = walk_positions(sym, dd, lam16, lo16)
        s_msk, nt_msk, mask, fin = walk_mask(sym, dd, lam16, lo16)
        assert s_ref == s_msk and nt_ref == nt_msk, trial
        assert bin(mask).count("1") == nz_before, trial     # the kernels' pre-truncation count
        assert bits_positions(s_ref, lo16) == bits_mask(s_msk, fin, lo16), trial
        # the untruncated token count from the mask as well (the rate pass with lambda 0, the plane rebuild)
        assert bits_positions(list(sym), lo16) == bits_mask(list(sym), mask, lo16), trial


def test_empty_and_full_blocks():
    lo16 = 16
    empty = [0] * 64
    assert bits_positions(empty, lo16) == bits_mask(empty, 0, lo16) == C_EOB
    full = [1] * 64
    mask = sum(1 << p for p in range(1, 64))
    assert bits_positions(full, lo16) == bits_mask(full, mask, lo16)
    dd = np.full(64, -1.0, np.float32)                      # every zeroing lowers the distortion: all go
    s, nt, _, fin = walk_mask(full, dd, np.float32(1.0), lo16)
    assert nt == 63 and fin == 0 and s == walk_positions(full, dd, np.float32(1.0), lo16)[0]
