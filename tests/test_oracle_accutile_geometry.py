"""Geometric check of the oracle's AccuTile intersection (IntersectTile.cu:195-253,
restated in oracle/gsb_oracle.c): the tiles a splat is assigned to are exactly the
tiles whose rectangle meets its ellipse d^T [[a, b], [b, c]] d <= t, with
t = min(3.33^2, 2 ln(255 o)), computed here in float64 by minimising the
quadratic over each tile rectangle. Tiles whose minimum lies within 1e-4
(relative) of t may go either way (the kernel's float32 rounding). CPU only."""

import math

import numpy as np

from oracle import oracle as O


def rect_min(A, B, C, mx, my, x0, x1, y0, y1):
    """Minimum of A dx^2 + 2 B dx dy + C dy^2 over the rectangle (d = p - m)."""
    if x0 <= mx <= x1 and y0 <= my <= y1:
        return 0.0
    best = math.inf
    for x in (x0, x1):  # vertical edges: minimise over y
        dx = x - mx
        dy = min(max(-B * dx / C, y0 - my), y1 - my)
        best = min(best, A * dx * dx + 2 * B * dx * dy + C * dy * dy)
    for y in (y0, y1):
        dy = y - my
        dx = min(max(-B * dy / A, x0 - mx), x1 - mx)
        best = min(best, A * dx * dx + 2 * B * dx * dy + C * dy * dy)
    return best


def test_accutile_tiles_are_the_ellipse_tiles():
    rng = np.random.default_rng(17)
    W, H, ts = 320, 240, 16
    tw, th = math.ceil(W / ts), math.ceil(H / ts)
    N = 1500
    m2 = np.stack([rng.uniform(-20, W + 20, N), rng.uniform(-20, H + 20, N)], -1).astype(np.float32)
    # 2D covariances with radii 0.5..40 px and random orientation
    ang = rng.uniform(0, np.pi, N)
    s1, s2 = np.exp(rng.uniform(np.log(0.5), np.log(40), (2, N)))
    c, s = np.cos(ang), np.sin(ang)
    cov = np.stack([[c * c * s1**2 + s * s * s2**2, c * s * (s1**2 - s2**2)],
                    [c * s * (s1**2 - s2**2), s * s * s1**2 + c * c * s2**2]]).transpose(2, 0, 1)
    inv = np.linalg.inv(cov)
    conics = np.stack([inv[:, 0, 0], inv[:, 0, 1], inv[:, 1, 1]], -1).astype(np.float32)
    op = rng.uniform(0.01, 1.0, N).astype(np.float32)
    radii = np.ceil(3.33 * np.sqrt(np.stack([cov[:, 0, 0], cov[:, 1, 1]], -1))).astype(np.int32)
    dep = rng.uniform(1, 5, N).astype(np.float32)
    _, keys, fids = O.isect_tiles(m2[None], radii[None], dep[None], ts, tw, th, conics=conics[None],
                                  opacities=op[None])
    tile_bits = (tw * th).bit_length()
    got = {}
    for k, g in zip(keys.tolist(), fids.tolist()):
        got.setdefault(g, set()).add((k >> 32) & ((1 << tile_bits) - 1))
    n_tiles_checked = ambiguous = 0
    for g in range(N):
        A, B, Cc = (float(v) for v in conics[g])
        mx, my = float(m2[g, 0]), float(m2[g, 1])
        t = min(3.33 * 3.33, 2.0 * math.log(float(op[g]) * 255.0))
        mine = got.get(g, set())
        for ty in range(th):
            for tx in range(tw):
                f = rect_min(A, B, Cc, mx, my, tx * ts, tx * ts + ts, ty * ts, ty * ts + ts)
                inside = f <= t
                n_tiles_checked += 1
                if abs(f - t) <= 1e-4 * max(t, 1e-6):
                    ambiguous += 1
                    continue
                assert inside == ((ty * tw + tx) in mine), (g, tx, ty, f, t)
    assert sum(len(v) for v in got.values()) > 5000
    assert ambiguous < 1e-3 * n_tiles_checked
