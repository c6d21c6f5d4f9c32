"""Seeded synthetic RGB8 test images (the reference trains on PNG photos; these stand in for them).

An image is the per-channel sum of 6 sinusoids of random orientation, frequency and phase, 4 octaves
of value noise and 20 hard-edged axis-aligned rectangles, clamped to 0..255. A material (several
textures sharing one UV) draws one base field and gives each texture its own random per-channel
affine remap plus independent noise. PNG read/write is plain zlib (no third-party codec).
"""
from __future__ import annotations

import struct
import zlib
from pathlib import Path

import numpy as np

# Distribution parameters (the generator's own choice; recorded here so the fixtures are reproducible).
N_SINES = 6
SINE_CYCLES = (1.0, 24.0)      # cycles across the image, uniform
SINE_AMP = 28.0                # per-channel amplitude std
NOISE_OCTAVES = 4
NOISE_BASE_CELLS = 4           # octave o has NOISE_BASE_CELLS * 2^o cells across
NOISE_AMP = 36.0               # octave o amplitude NOISE_AMP / 2^o
N_RECTS = 20
RECT_AMP = 45.0


def _value_noise(rng: np.random.Generator, W: int, H: int, cells: int) -> np.ndarray:
    g = rng.standard_normal((cells + 1, cells + 1, 3))
    x = (np.arange(W) + 0.5) / W * cells
    y = (np.arange(H) + 0.5) / H * cells
    x0 = np.minimum(np.floor(x).astype(int), cells - 1)
    y0 = np.minimum(np.floor(y).astype(int), cells - 1)
    fx = x - x0
    fy = y - y0
    sx = fx * fx * (3 - 2 * fx)
    sy = fy * fy * (3 - 2 * fy)
    # Interpolate along x on the (cells + 1) grid rows first, then pick and blend rows: every output element goes
    # through the same operations as a * (1 - sx) + b * sx per corner row, so the field is unchanged.
    sx = sx[None, :, None]
    gx = g[:, x0] * (1 - sx) + g[:, x0 + 1] * sx          # (cells + 1, W, 3)
    sy = sy[:, None, None]
    return gx[y0] * (1 - sy) + gx[y0 + 1] * sy


def base_field(W: int, H: int, seed: int) -> np.ndarray:
    """Float field (H, W, 3) before clamping, deterministic in (W, H, seed)."""
    rng = np.random.default_rng(seed)
    yy, xx = np.meshgrid(np.arange(H) + 0.5, np.arange(W) + 0.5, indexing="ij")
    img = np.full((H, W, 3), 128.0)
    for _ in range(N_SINES):
        th = rng.uniform(0, np.pi)
        cyc = rng.uniform(*SINE_CYCLES)
        ph = rng.uniform(0, 2 * np.pi)
        amp = rng.normal(0, SINE_AMP, 3)
        t = (xx * np.cos(th) / W + yy * np.sin(th) / H) * cyc * 2 * np.pi + ph
        img += np.sin(t)[..., None] * amp
    for o in range(NOISE_OCTAVES):
        img += _value_noise(rng, W, H, NOISE_BASE_CELLS << o) * (NOISE_AMP / (1 << o))
    for _ in range(N_RECTS):
        w = int(rng.integers(max(2, W // 32), max(3, W // 4)))
        h = int(rng.integers(max(2, H // 32), max(3, H // 4)))
        x0 = int(rng.integers(0, W - w + 1))
        y0 = int(rng.integers(0, H - h + 1))
        img[y0:y0 + h, x0:x0 + w] += rng.normal(0, RECT_AMP, 3)
    return img


def synth_rgb8(W: int, H: int, seed: int) -> np.ndarray:
    """One synthetic texture, uint8 (H, W, 3)."""
    return np.clip(np.rint(base_field(W, H, seed)), 0, 255).astype(np.uint8)


def synth_material(W: int, H: int, seed: int, T: int) -> list[np.ndarray]:
    """T textures sharing one base field: per texture a random per-channel affine remap plus noise."""
    base = base_field(W, H, seed)
    rng = np.random.default_rng(seed + 1_000_003)
    out = []
    for t in range(T):
        gain = rng.uniform(0.5, 1.5, 3)
        bias = rng.uniform(-40, 40, 3)
        noise = _value_noise(rng, W, H, 16) * 10.0 + rng.normal(0, 3.0, (H, W, 3))
        img = (base - 128.0) * gain + 128.0 + bias + noise
        out.append(np.clip(np.rint(img), 0, 255).astype(np.uint8))
    return out


def to_target(images: list[np.ndarray]) -> np.ndarray:
    """Interleaved float target (H*W*3T,) as the reference builds it: byte / 255.0f (main.cpp:319, 358-365)."""
    H, W, _ = images[0].shape
    f = np.stack([im.astype(np.float32) / np.float32(255.0) for im in images], axis=2)  # H, W, T, 3
    return np.ascontiguousarray(f.reshape(H * W * 3 * len(images)), dtype=np.float32)


def write_png(path: str | Path, rgb: np.ndarray) -> None:
    """8-bit RGB PNG, filter 0 on every row."""
    H, W, _ = rgb.shape
    raw = b"".join(b"\x00" + rgb[y].astype(np.uint8).tobytes() for y in range(H))

    def chunk(tag: bytes, data: bytes) -> bytes:
        return struct.pack(">I", len(data)) + tag + data + struct.pack(">I", zlib.crc32(tag + data) & 0xFFFFFFFF)

    png = b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", W, H, 8, 2, 0, 0, 0))
    png += chunk(b"IDAT", zlib.compress(raw, 6)) + chunk(b"IEND", b"")
    Path(path).write_bytes(png)


def read_png(path: str | Path) -> np.ndarray:
    """Reads the 8-bit RGB, non-interlaced PNGs write_png produces (all five filter types handled)."""
    data = Path(path).read_bytes()
    assert data[:8] == b"\x89PNG\r\n\x1a\n", "not a PNG"
    pos, idat, W, H = 8, b"", 0, 0
    while pos < len(data):
        n = struct.unpack(">I", data[pos:pos + 4])[0]
        tag = data[pos + 4:pos + 8]
        body = data[pos + 8:pos + 8 + n]
        if tag == b"IHDR":
            W, H, depth, ctype = struct.unpack(">IIBB", body[:10])
            assert depth == 8 and ctype == 2, "only 8-bit RGB"
        elif tag == b"IDAT":
            idat += body
        pos += 12 + n
    raw = zlib.decompress(idat)
    stride = W * 3
    out = np.zeros((H, stride), np.uint8)
    prev = np.zeros(stride, np.int32)
    for y in range(H):
        f = raw[y * (stride + 1)]
        line = np.frombuffer(raw[y * (stride + 1) + 1:(y + 1) * (stride + 1)], np.uint8).astype(np.int32)
        cur = np.zeros(stride, np.int32)
        for x in range(stride):
            a = cur[x - 3] if x >= 3 else 0
            b = prev[x]
            c = prev[x - 3] if x >= 3 else 0
            if f == 0:
                p = 0
            elif f == 1:
                p = a
            elif f == 2:
                p = b
            elif f == 3:
                p = (a + b) // 2
            else:
                pa, pb, pc = abs(b - c), abs(a - c), abs(a + b - 2 * c)
                p = a if pa <= pb and pa <= pc else (b if pb <= pc else c)
            cur[x] = (line[x] + p) & 0xFF
        out[y] = cur
        prev = cur
    return out.reshape(H, W, 3)
