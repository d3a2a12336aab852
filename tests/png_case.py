"""A small PNG writer for the decoder tests: any colour type and bit depth,
Adam7 interlacing, and every scanline filter (rows cycle through filter
types 0-4), so each decoding path is exercised with known pixels.  Also the
8-bit RGB the engine's decoder should produce from them."""
from __future__ import annotations

import struct
import zlib

import numpy as np

ADAM7 = [(0, 0, 8, 8), (4, 0, 8, 8), (0, 4, 4, 8), (2, 0, 4, 4), (0, 2, 2, 4), (1, 0, 2, 2),
         (0, 1, 1, 2)]
CHANNELS = {0: 1, 2: 3, 3: 1, 4: 2, 6: 4}


def _chunk(kind: bytes, body: bytes) -> bytes:
    return struct.pack(">I", len(body)) + kind + body + struct.pack(">I", zlib.crc32(kind + body))


def _pack_row(samples: np.ndarray, depth: int) -> bytes:
    if depth == 16:
        return samples.astype(">u2").tobytes()
    if depth == 8:
        return samples.astype(np.uint8).tobytes()
    per = 8 // depth
    out = bytearray((len(samples) + per - 1) // per)
    for i, v in enumerate(samples):
        out[i // per] |= int(v) << (8 - depth * (1 + i % per))
    return bytes(out)


def _paeth(a, b, c):
    p = a + b - c
    pa, pb, pc = abs(p - a), abs(p - b), abs(p - c)
    return a if pa <= pb and pa <= pc else (b if pb <= pc else c)


def _filter(rows, bpp):
    out = bytearray()
    prev = bytes(len(rows[0])) if rows else b""
    for y, row in enumerate(rows):
        f = y % 5
        out.append(f)
        for i, x in enumerate(row):
            a = row[i - bpp] if i >= bpp else 0
            b = prev[i]
            c = prev[i - bpp] if i >= bpp else 0
            pred = (0, a, b, (a + b) >> 1, _paeth(a, b, c))[f]
            out.append((x - pred) & 0xFF)
        prev = row
    return bytes(out)


def png_bytes(samples: np.ndarray, color: int, depth: int, interlace: bool = False,
              palette: np.ndarray | None = None) -> bytes:
    """samples: (h, w, channels) integers in [0, 2**depth)."""
    h, w = samples.shape[:2]
    ch = CHANNELS[color]
    samples = samples.reshape(h, w, ch)
    bpp = max(1, ch * depth // 8)
    passes = ADAM7 if interlace else [(0, 0, 1, 1)]
    raw = b""
    for x0, y0, dx, dy in passes:
        sub = samples[y0::dy, x0::dx]
        if sub.size == 0:
            continue
        rows = [_pack_row(sub[y].reshape(-1), depth) for y in range(sub.shape[0])]
        raw += _filter(rows, bpp)
    ihdr = struct.pack(">IIBBBBB", w, h, depth, color, 0, 0, 1 if interlace else 0)
    out = b"\x89PNG\r\n\x1a\n" + _chunk(b"IHDR", ihdr)
    if palette is not None:
        out += _chunk(b"PLTE", np.asarray(palette, np.uint8).tobytes())
    # split the stream over two IDAT chunks
    z = zlib.compress(raw, 6)
    half = len(z) // 2
    return out + _chunk(b"IDAT", z[:half]) + _chunk(b"IDAT", z[half:]) + _chunk(b"IEND", b"")


def expected_rgb8(samples: np.ndarray, color: int, depth: int, palette=None) -> np.ndarray:
    """(h, w, 3) bytes: high byte of 16-bit samples, low depths scaled to
    255, palette looked up, alpha composited over black ((c a + 127) / 255)."""
    h, w = samples.shape[:2]
    s = samples.reshape(h, w, CHANNELS[color]).astype(np.int64)
    if color == 3:
        return np.asarray(palette, np.uint8)[s[..., 0]]
    if depth == 16:
        s = s >> 8
    elif depth < 8:
        s = s * 255 // ((1 << depth) - 1)
    if color in (4, 6):
        c, a = s[..., :-1], s[..., -1:]
        s = (c * a + 127) // 255
    if s.shape[-1] == 1:
        s = np.repeat(s, 3, -1)
    return s.astype(np.uint8)


def random_samples(h: int, w: int, color: int, depth: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(0, 1 << depth, (h, w, CHANNELS[color]))
