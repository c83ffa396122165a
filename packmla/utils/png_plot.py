"""Dependency-free line charts written as PNG (numpy raster + zlib), for reports on hosts without matplotlib.

A chart is a white canvas with a plot frame, horizontal grid lines at "nice" y ticks, x ticks at the given
x values, one polyline with square markers per series, and tick labels drawn in a built-in 3x5 pixel font
(digits, '.', '-', '%').  Series colours are fixed by order.  The title, axis labels and the
colour -> series legend are stored as PNG tEXt chunks and returned, so a caller can print them beside the
image.
"""
from __future__ import annotations

import math
import struct
import zlib

import numpy as np

COLORS = ((31, 119, 180), (255, 127, 14), (44, 160, 44), (214, 39, 40), (148, 103, 189), (140, 86, 75))
COLOR_NAMES = ("blue", "orange", "green", "red", "purple", "brown")

_FONT = {  # 3 x 5 glyphs, rows top to bottom, bit 2 = left column
    "0": (7, 5, 5, 5, 7), "1": (2, 6, 2, 2, 7), "2": (7, 1, 7, 4, 7), "3": (7, 1, 7, 1, 7), "4": (5, 5, 7, 1, 1),
    "5": (7, 4, 7, 1, 7), "6": (7, 4, 7, 5, 7), "7": (7, 1, 1, 1, 1), "8": (7, 5, 7, 5, 7), "9": (7, 5, 7, 1, 7),
    ".": (0, 0, 0, 0, 2), "-": (0, 0, 7, 0, 0), "%": (5, 1, 2, 4, 5), " ": (0, 0, 0, 0, 0),
}


def _chunk(kind: bytes, data: bytes) -> bytes:
    return struct.pack(">I", len(data)) + kind + data + struct.pack(">I", zlib.crc32(kind + data) & 0xFFFFFFFF)


def encode_png(img: np.ndarray, text: dict | None = None) -> bytes:
    """RGB uint8 [H, W, 3] -> PNG bytes (8-bit truecolour, filter 0, tEXt chunks from `text`)."""
    if img.dtype != np.uint8 or img.ndim != 3 or img.shape[2] != 3:
        raise ValueError("image must be uint8 [H, W, 3]")
    h, w, _ = img.shape
    raw = b"".join(b"\x00" + img[y].tobytes() for y in range(h))
    out = b"\x89PNG\r\n\x1a\n" + _chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, 8, 2, 0, 0, 0))
    for k, v in (text or {}).items():
        out += _chunk(b"tEXt", k.encode("latin-1") + b"\x00" + str(v).encode("latin-1", "replace"))
    return out + _chunk(b"IDAT", zlib.compress(raw, 9)) + _chunk(b"IEND", b"")


def _line(img, x0, y0, x1, y1, color, width=2):
    n = int(max(abs(x1 - x0), abs(y1 - y0))) + 1
    for t in np.linspace(0.0, 1.0, n):
        x, y = int(round(x0 + (x1 - x0) * t)), int(round(y0 + (y1 - y0) * t))
        img[max(0, y - width // 2):y + (width + 1) // 2, max(0, x - width // 2):x + (width + 1) // 2] = color


def _text(img, x, y, s, color=(0, 0, 0), scale=2):
    for ch in s:
        rows = _FONT.get(ch, _FONT[" "])
        for r, bits in enumerate(rows):
            for c in range(3):
                if bits >> (2 - c) & 1:
                    img[y + r * scale:y + (r + 1) * scale, x + c * scale:x + (c + 1) * scale] = color
        x += 4 * scale


def _nice_ticks(lo: float, hi: float, n: int = 5) -> list[float]:
    if hi <= lo:
        hi = lo + 1.0
    step = (hi - lo) / n
    mag = 10 ** math.floor(math.log10(step))
    step = min((m * mag for m in (1, 2, 5, 10) if m * mag >= step), default=10 * mag)
    start = math.floor(lo / step) * step
    ticks, v = [], start
    while not ticks or ticks[-1] < hi - 1e-9 * step:  # the last tick covers the largest value
        ticks.append(round(v, 10))
        v += step
    return ticks


def _fmt(v: float) -> str:
    s = f"{v:.3g}"
    return s if "e" not in s else f"{v:.1f}"


def line_chart(path, xs: list[float], series: dict[str, list[float]], title: str = "", xlabel: str = "",
               ylabel: str = "", size: tuple[int, int] = (800, 500)) -> dict:
    """Write a line chart of `series` (name -> y values at `xs`) to `path`; returns the legend
    {name: colour name} and the axis ranges."""
    if len(series) > len(COLORS):
        raise ValueError(f"at most {len(COLORS)} series")
    W, H = size
    img = np.full((H, W, 3), 255, dtype=np.uint8)
    left, right, top, bottom = 70, 20, 20, 50
    ys = [v for vals in series.values() for v in vals]
    yt = _nice_ticks(min(ys), max(ys))
    ylo, yhi = yt[0], yt[-1]
    xlo, xhi = min(xs), max(xs)
    xhi = xhi if xhi > xlo else xlo + 1

    def px(x):
        return left + (x - xlo) / (xhi - xlo) * (W - left - right)

    def py(y):
        return H - bottom - (y - ylo) / (yhi - ylo) * (H - top - bottom)

    for t in yt:  # grid and y tick labels
        _line(img, left, py(t), W - right, py(t), (225, 225, 225), 1)
        label = _fmt(t)
        _text(img, max(0, left - 8 - 8 * len(label)), int(py(t)) - 5, label)
    for x in xs:  # x ticks and labels
        _line(img, px(x), H - bottom, px(x), H - bottom + 6, (0, 0, 0), 1)
        label = _fmt(x)
        _text(img, int(px(x)) - 4 * len(label), H - bottom + 12, label)
    _line(img, left, top, left, H - bottom, (0, 0, 0), 2)  # frame
    _line(img, left, H - bottom, W - right, H - bottom, (0, 0, 0), 2)
    legend = {}
    for (name, vals), color, cname in zip(series.items(), COLORS, COLOR_NAMES):
        pts = [(px(x), py(y)) for x, y in zip(xs, vals)]
        for (x0, y0), (x1, y1) in zip(pts, pts[1:]):
            _line(img, x0, y0, x1, y1, color, 2)
        for x, y in pts:
            img[int(y) - 3:int(y) + 4, int(x) - 3:int(x) + 4] = color
        legend[name] = cname
    text = {"Title": title, "X-Axis": xlabel, "Y-Axis": ylabel,
            "Legend": ", ".join(f"{n}={c}" for n, c in legend.items())}
    with open(path, "xb") as f:
        f.write(encode_png(img, text))
    return {"legend": legend, "y_range": [ylo, yhi], "x_range": [xlo, xhi]}


def read_png(path) -> tuple[np.ndarray, dict]:
    """Decode a PNG written by `encode_png` (RGB, filter 0): (image, tEXt entries)."""
    data = open(path, "rb").read()
    if data[:8] != b"\x89PNG\r\n\x1a\n":
        raise ValueError("not a PNG")
    pos, idat, text, w, h = 8, b"", {}, 0, 0
    while pos < len(data):
        n = struct.unpack(">I", data[pos:pos + 4])[0]
        kind, body = data[pos + 4:pos + 8], data[pos + 8:pos + 8 + n]
        if zlib.crc32(kind + body) & 0xFFFFFFFF != struct.unpack(">I", data[pos + 8 + n:pos + 12 + n])[0]:
            raise ValueError(f"bad CRC in {kind!r}")
        if kind == b"IHDR":
            w, h = struct.unpack(">II", body[:8])
        elif kind == b"IDAT":
            idat += body
        elif kind == b"tEXt":
            k, v = body.split(b"\x00", 1)
            text[k.decode("latin-1")] = v.decode("latin-1")
        pos += 12 + n
    raw = zlib.decompress(idat)
    rows = np.frombuffer(raw, dtype=np.uint8).reshape(h, 1 + 3 * w)
    if bool((rows[:, 0] != 0).any()):
        raise ValueError("only filter type 0 is supported")
    return rows[:, 1:].reshape(h, w, 3).copy(), text
