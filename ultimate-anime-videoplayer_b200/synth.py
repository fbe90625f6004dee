"""Seeded synthetic anime-like frames (the contract's stand-in for real video: no dataset is used).

A frame is a smooth colour gradient, overlaid with flat colour cells (a Voronoi partition, a fraction
of the cells painted flat) and 1-pixel dark line edges (random polylines), values in [0, 1].
RIFE pairs: frame B is frame A moved by a seeded per-region translation of up to 24 pixels.
"""
from __future__ import annotations

import numpy as np


def _gradient(rng, h, w):
    ys = np.linspace(0.0, 1.0, h, dtype=np.float32)[:, None]
    xs = np.linspace(0.0, 1.0, w, dtype=np.float32)[None, :]
    out = np.empty((3, h, w), np.float32)
    for c in range(3):
        a, bx, by = rng.uniform(0.15, 0.6), rng.uniform(-0.3, 0.3), rng.uniform(-0.3, 0.3)
        fx, fy, ph = rng.uniform(0.5, 2.0), rng.uniform(0.5, 2.0), rng.uniform(0, 2 * np.pi)
        out[c] = a + bx * xs + by * ys + 0.08 * np.sin(2 * np.pi * (fx * xs + fy * ys) + ph)
    return out


def _cells(rng, h, w, n_cells):
    """Label of the nearest seed point for every pixel, computed on a 1/4 grid then upsampled."""
    gh, gw = max(1, h // 4), max(1, w // 4)
    sy = rng.uniform(0, gh, n_cells).astype(np.float32)
    sx = rng.uniform(0, gw, n_cells).astype(np.float32)
    yy = np.arange(gh, dtype=np.float32)[:, None, None]
    xx = np.arange(gw, dtype=np.float32)[None, :, None]
    lab = np.argmin((yy - sy) ** 2 + (xx - sx) ** 2, axis=2)
    lab = np.repeat(np.repeat(lab, 4, axis=0), 4, axis=1)
    return np.pad(lab, ((0, max(0, h - lab.shape[0])), (0, max(0, w - lab.shape[1]))), mode="edge")[:h, :w]


def _lines(rng, img, n_lines):
    _, h, w = img.shape
    for _ in range(n_lines):
        x, y = rng.uniform(0, w), rng.uniform(0, h)
        dark = rng.uniform(0.02, 0.12)
        for _seg in range(int(rng.integers(2, 6))):
            ang, length = rng.uniform(0, 2 * np.pi), rng.uniform(0.05, 0.3) * max(h, w)
            x1, y1 = x + length * np.cos(ang), y + length * np.sin(ang)
            t = np.linspace(0.0, 1.0, int(length * 2) + 2)
            px = np.clip(np.round(x + (x1 - x) * t).astype(np.int64), 0, w - 1)
            py = np.clip(np.round(y + (y1 - y) * t).astype(np.int64), 0, h - 1)
            img[:, py, px] = dark
            x, y = float(np.clip(x1, 0, w - 1)), float(np.clip(y1, 0, h - 1))


def anime_frame(h, w, seed):
    rng = np.random.default_rng(seed)
    img = _gradient(rng, h, w)
    n_cells = max(4, (h * w) // 40000)
    lab = _cells(rng, h, w, n_cells)
    flat = rng.random(n_cells) < 0.6
    colours = rng.uniform(0.05, 0.95, (n_cells, 3)).astype(np.float32)
    mask = flat[lab]
    for c in range(3):
        img[c] = np.where(mask, colours[lab, c], img[c])
    _lines(rng, img, max(3, (h + w) // 40))
    return np.clip(img, 0.0, 1.0)


def anime_frames(n, h, w, seed=0):
    return np.stack([anime_frame(h, w, seed * 1000 + i) for i in range(n)]).astype(np.float32)


def shifted_pair(h, w, seed, max_shift=24.0, regions=(3, 4)):
    """(A, B): B = A translated per region (a regions[0] x regions[1] grid), shifts up to max_shift
    pixels, integer or sub-pixel, bilinear with border clamp."""
    rng = np.random.default_rng(seed)
    a = anime_frame(h, w, seed)
    ry = np.minimum(np.arange(h) * regions[0] // h, regions[0] - 1)
    rx = np.minimum(np.arange(w) * regions[1] // w, regions[1] - 1)
    shifts = rng.uniform(-max_shift, max_shift, (regions[0], regions[1], 2)).astype(np.float32)
    dx = shifts[ry[:, None], rx[None, :], 0]
    dy = shifts[ry[:, None], rx[None, :], 1]
    sx = np.clip(np.arange(w, dtype=np.float32)[None, :] - dx, 0, w - 1)
    sy = np.clip(np.arange(h, dtype=np.float32)[:, None] - dy, 0, h - 1)
    x0, y0 = np.floor(sx).astype(np.int64), np.floor(sy).astype(np.int64)
    x1, y1 = np.minimum(x0 + 1, w - 1), np.minimum(y0 + 1, h - 1)
    fx, fy = sx - x0, sy - y0
    b = (a[:, y0, x0] * (1 - fx) + a[:, y0, x1] * fx) * (1 - fy) + (a[:, y1, x0] * (1 - fx) + a[:, y1, x1] * fx) * fy
    return a.astype(np.float32), b.astype(np.float32)
