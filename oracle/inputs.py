"""Seeded synthetic Q/K/V of the BASELINE configs (test infrastructure only).

The reference measures on no public dataset; these generators are the whole
workload.  Distributions (values drawn in float32, then rounded to bf16):

* Q ~ N(0, 1).
* K = N(0, 1) + a per-(b, h) per-channel offset o[d] ~ N(0, sigma=2).
* V: 64 cluster centres C ~ N(0, 1) per (b, h); token = C[randint(64)] +
  0.3 N(0, 1); tokens then shuffled.
* ``spatial=(T, Hg, W)``: tokens sit on a T x Hg x W grid; a
  smooth positional field (8 separable low-frequency cosines projected to D by
  a seeded Gaussian, RMS 0.5) is added to Q and K, and V's centre is chosen by
  the token's spatial region (4 x 4 x 4 regions), so routing is non-trivial.
* ``cfg_pair``: batch 1 = batch 0 + 0.05 N(0, 1).
"""

from __future__ import annotations

import hashlib
from typing import Optional, Tuple

import numpy as np

from .vc_oracle import bf16_round


def _positional_field(rng, grid: Tuple[int, int, int], d: int) -> np.ndarray:
    t, hg, w = grid
    tt, hh, ww = np.meshgrid(np.arange(t), np.arange(hg), np.arange(w), indexing="ij")
    feats = []
    for _ in range(8):
        ft, fh, fw = rng.uniform(0.0, 2.0, size=3)
        ph = rng.uniform(0, 2 * np.pi, size=3)
        f = (np.cos(np.pi * ft * tt / max(t, 1) + ph[0]) * np.cos(np.pi * fh * hh / max(hg, 1) + ph[1])
             * np.cos(np.pi * fw * ww / max(w, 1) + ph[2]))
        feats.append(f.reshape(-1))
    feats = np.stack(feats, axis=-1).astype(np.float32)               # (N, 8)
    proj = rng.standard_normal((8, d)).astype(np.float32)
    p = feats @ proj
    p *= 0.5 / max(float(np.sqrt(np.mean(p.astype(np.float64) ** 2))), 1e-12)
    return p.astype(np.float32)


def make_qkv(b: int, h: int, n: int, d: int = 128, seed: int = 0, centres: int = 64,
             spatial: Optional[Tuple[int, int, int]] = None, cfg_pair: bool = False):
    """-> (q, k, v) float32 arrays of shape (B, H, N, D) holding bf16 values."""
    rng = np.random.default_rng(seed)
    g = h if cfg_pair else b * h
    q = rng.standard_normal((g, n, d), dtype=np.float32)
    off = (2.0 * rng.standard_normal((g, 1, d), dtype=np.float32)).astype(np.float32)
    k = (rng.standard_normal((g, n, d), dtype=np.float32) + off).astype(np.float32)
    c = rng.standard_normal((g, centres, d), dtype=np.float32)
    if spatial is not None:
        t, hg, w = spatial
        assert t * hg * w == n, "spatial grid must cover N tokens"
        tt, hh, ww = np.meshgrid(np.arange(t), np.arange(hg), np.arange(w), indexing="ij")
        reg = ((tt * 4) // t) * 16 + ((hh * 4) // hg) * 4 + (ww * 4) // w
        lab = np.broadcast_to((reg.reshape(-1) % centres)[None, :], (g, n))
        pos = _positional_field(rng, spatial, d)
        q = (q + pos[None]).astype(np.float32)
        k = (k + pos[None]).astype(np.float32)
    else:
        lab = rng.integers(0, centres, size=(g, n))
    v = np.take_along_axis(c, lab[..., None], axis=1)
    v = (v + 0.3 * rng.standard_normal((g, n, d), dtype=np.float32)).astype(np.float32)
    if spatial is None:
        for gi in range(g):
            v[gi] = v[gi, rng.permutation(n)]
    if cfg_pair:
        q = np.concatenate([q, q + 0.05 * rng.standard_normal(q.shape, dtype=np.float32)], 0)
        k = np.concatenate([k, k + 0.05 * rng.standard_normal(k.shape, dtype=np.float32)], 0)
        v = np.concatenate([v, v + 0.05 * rng.standard_normal(v.shape, dtype=np.float32)], 0)
        b = 2
    shape = (b, h, n, d)
    return (bf16_round(q).reshape(shape), bf16_round(k).reshape(shape),
            bf16_round(v).reshape(shape))


def digest(*arrays) -> str:
    """Short content hash used to check that regenerated inputs match a fixture."""
    hsh = hashlib.sha256()
    for a in arrays:
        hsh.update(np.ascontiguousarray(a).tobytes())
    return hsh.hexdigest()[:16]
