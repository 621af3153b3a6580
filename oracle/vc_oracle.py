"""CPU restatement of the VC-Attention hot path of bingling360/comfyui_vc_attention.

TEST INFRASTRUCTURE ONLY.  This module is the checker: it is imported by
``tests/``, by ``__graft_entry__.smoke()`` and by the CPU-baseline legs of
``bench.py``.  The product package ``comfyui_vc_attention_b200`` never
imports, links or executes anything under ``oracle/``.

Parity pinning
--------------
``tests/golden/make_golden.py`` imports the reference package read-only and
records its outputs on seeded inputs into ``tests/golden/*.npz``;
``tests/test_oracle_golden.py`` checks every function below against those
vectors.  Where the reference's result depends on an unspecified floating-point
summation order (torch CPU cascade sums, oneDNN bf16 GEMM), this module fixes
one order and says which; the golden test then bounds the disagreement and
checks that every disagreement sits on a rounding tie.

Conventions: every tensor is a numpy array.  Floating arithmetic is float32
unless stated; numpy float32 ops are IEEE correctly rounded and never fused,
which is what makes the restatement reproducible on the GPU with ``__f*_rn``
intrinsics.  bf16 values are carried as float32 arrays holding bf16-exact
values (``bf16_round``) or as uint16 bit patterns.
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Sequence, Tuple

import numpy as np

F32 = np.float32
LOG2E = 1.4426950408889634          # expcast.py:47
E4M3_MAX = 448.0                    # quant.py:42
E4M3_MIN_NORMAL = 2.0 ** -6         # quant.py:43
FP4_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float32)   # quant.py:46
_FP4_BREAKS = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)  # quant.py:49
P_SCALE = 448.0                     # triton_attn.py:83
TINY = F32(1e-30)                   # clamp(min=1e-30) used throughout quant.py


# ---------------------------------------------------------------------------
# bf16 helpers
# ---------------------------------------------------------------------------

def f32_to_bf16_bits(x) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit pattern (uint16)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def bf16_bits_to_f32(h) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def mean_f32(x: np.ndarray, axis: int, count: Optional[int] = None) -> np.ndarray:
    """Mean with one rounding of the sum: fp32(sum in float64) / count in fp32.

    The reference uses torch's CPU cascade sum (order unspecified).  This build
    fixes the correctly rounded sum; the GPU kernels accumulate in float64 and
    round once, so the two agree bit for bit.
    """
    s = np.sum(x.astype(np.float64), axis=axis, keepdims=True).astype(np.float32)
    n = x.shape[axis] if count is None else count
    return (s / F32(n)).astype(np.float32)


# ---------------------------------------------------------------------------
# E4M3 / E2M1 codecs  (quant.py)
# ---------------------------------------------------------------------------

def e4m3_encode(x) -> np.ndarray:
    """RNE, saturating E4M3 encoder.  Restates quant.py:56-84 bit for bit."""
    a = np.asarray(x, dtype=np.float32)
    sign = (a < 0).astype(np.int64)
    a = np.minimum(np.abs(a), F32(E4M3_MAX))
    frac, exp = np.frexp(a)
    frac = frac.astype(np.float32)
    exp = exp.astype(np.int64)
    is_sub = a < F32(E4M3_MIN_NORMAL)
    code_sub = np.clip(np.round(a * F32(512.0)), 0, 8).astype(np.int64)
    mant = np.round(frac * F32(16.0) - F32(8.0))
    carry = mant >= 8.0
    mant = np.where(carry, mant - 8.0, mant)
    exp = np.where(carry, exp + 1, exp)
    exp = np.where(is_sub, 0, exp)
    e_field = np.clip((exp - 1) + 7, 1, 15)
    code_n = (e_field << 3) | np.clip(mant, 0, 7).astype(np.int64)
    code = np.where(is_sub, code_sub, code_n)
    code = (code & 0x7F) | (sign << 7)
    return code.astype(np.uint8)


def e4m3_decode(code) -> np.ndarray:
    """quant.py:87-100 (0x7F/0xFF decode to +-448)."""
    c = np.asarray(code).astype(np.int64) & 0xFF
    sign = ((c >> 7) & 1) * -2.0 + 1.0
    e = (c >> 3) & 0xF
    m = c & 0x7
    val_sub = m.astype(np.float32) * F32(2.0 ** -9)
    val_norm = (F32(1.0) + m.astype(np.float32) / F32(8.0)) * np.power(
        F32(2.0), (e - 7).astype(np.float32))
    val = np.where(e == 0, val_sub, val_norm).astype(np.float32)
    val = np.where((e == 15) & (m == 7), F32(E4M3_MAX), val)
    return (val * sign.astype(np.float32)).astype(np.float32)


def fp4_encode(x) -> np.ndarray:
    """RNE E2M1 codes 0..15, bit 3 = sign.  quant.py:144-161."""
    a = np.asarray(x, dtype=np.float32)
    sign = (a < 0).astype(np.int64)
    a = np.abs(a)
    idx = np.searchsorted(_FP4_BREAKS, a, side="left").astype(np.int64)
    nbrk = len(_FP4_BREAKS)
    in_range = idx < nbrk
    safe = np.minimum(idx, nbrk - 1)
    tie = in_range & (a == _FP4_BREAKS[safe]) & ((safe & 1) != 0)
    idx = np.clip(np.where(tie, idx + 1, idx), 0, 7)
    return ((sign << 3) | idx).astype(np.uint8)


def fp4_decode(code) -> np.ndarray:
    """quant.py:164-169."""
    c = np.asarray(code).astype(np.int64) & 0xF
    sign = ((c >> 3) & 1) * -2.0 + 1.0
    return (FP4_VALUES[c & 0x7] * sign).astype(np.float32)


def quantize_e4m3_rows(x: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """Per-row (last axis) symmetric E4M3.  quant.py:107-126 with dim=-1.

    scale = max(amax, 1e-30) / 448 ; code = e4m3(x / scale); both fp32 IEEE.
    Returns (codes uint8 same shape, scale float32 shape[:-1]).
    """
    amax = np.max(np.abs(x), axis=-1, keepdims=True).astype(np.float32)
    scale = (np.maximum(amax, TINY) / F32(E4M3_MAX)).astype(np.float32)
    codes = e4m3_encode((x / scale).astype(np.float32))
    return codes, scale[..., 0]


def quantize_e4m3_blocks(x: np.ndarray, block_rows: int) -> Tuple[np.ndarray, np.ndarray]:
    """Per-(block of rows) x per-channel E4M3.  quant.py:219-237.

    x: (G, N, D) with N % block_rows == 0 -> (codes (G,N,D), scale (G,NB,D)).
    """
    g, n, d = x.shape
    xb = x.reshape(g, n // block_rows, block_rows, d)
    amp = np.maximum(np.max(np.abs(xb), axis=2), TINY).astype(np.float32)
    scale = (amp / F32(E4M3_MAX)).astype(np.float32)
    codes = e4m3_encode((xb / scale[:, :, None, :]).astype(np.float32))
    return codes.reshape(g, n, d), scale


def dequantize_e4m3_blocks(codes, scale, block_rows):
    g, n, d = codes.shape
    s = np.repeat(scale, block_rows, axis=1)
    return (e4m3_decode(codes) * s).astype(np.float32)


def quantize_nvfp4(x: np.ndarray, block: int = 16):
    """NVFP4 over the flattened tensor: E2M1 codes, per-16 E4M3 micro codes and
    one fp32 tensor scale g.  quant.py:172-204.  Codes are one per element
    (unpacked); ``pack_nibbles`` packs them low-nibble-first.
    """
    flat = np.asarray(x, np.float32).reshape(-1)
    n = flat.size
    pad = (-n) % block
    if pad:
        flat = np.concatenate([flat, np.zeros(pad, np.float32)])
    blocks = flat.reshape(-1, block)
    g = F32(max(F32(np.max(np.abs(blocks))), TINY) / F32(6.0 * E4M3_MAX))
    g = max(g, TINY)
    amax_b = np.maximum(np.max(np.abs(blocks), axis=1, keepdims=True), TINY).astype(np.float32)
    micro = ((amax_b / F32(6.0)) / g).astype(np.float32)
    micro_code = e4m3_encode(np.minimum(micro, F32(E4M3_MAX)))
    micro_val = e4m3_decode(micro_code)
    q = fp4_encode((blocks / np.maximum(g * micro_val, TINY)).astype(np.float32))
    return q.reshape(-1)[:n], micro_code.reshape(-1), F32(g)


def dequantize_nvfp4(codes, micro_code, g, block=16):
    micro_val = e4m3_decode(micro_code).astype(np.float32)
    return (fp4_decode(codes) * (np.repeat(micro_val, block)[: codes.size] * F32(g))).astype(np.float32)


def pack_nibbles(codes: np.ndarray) -> np.ndarray:
    """(..., D) uint8 4-bit codes -> (..., D//2); low nibble = even element
    (triton_attn.py:197)."""
    c = codes.astype(np.uint8)
    return ((c[..., 0::2] & 0xF) | ((c[..., 1::2] & 0xF) << 4)).astype(np.uint8)


# ---------------------------------------------------------------------------
# Hadamard  (hadamard.py:37-65)
# ---------------------------------------------------------------------------

def fwht(x: np.ndarray) -> np.ndarray:
    """fp32 butterfly: stage h maps (x[i], x[i+h]) -> (x[i]+x[i+h], x[i]-x[i+h]),
    then one IEEE division by fp32(sqrt(d)).  Bit-identical to hadamard.py:37-65.
    """
    d = x.shape[-1]
    if d & (d - 1):
        raise ValueError(f"Hadamard transform needs a power-of-two dim, got {d}")
    batch = x.shape[:-1]
    out = np.asarray(x, np.float32)
    h = 1
    while h < d:
        o = out.reshape(*batch, -1, 2, h)
        a = o[..., 0, :]
        b = o[..., 1, :]
        out = np.concatenate((a + b, a - b), axis=-1)
        h *= 2
    out = out.reshape(x.shape)
    return (out / F32(math.sqrt(d))).astype(np.float32)


# ---------------------------------------------------------------------------
# V-Smooth k-means  (grouping.py)
# ---------------------------------------------------------------------------

def num_clusters(n: int, block_rows: int, max_clusters: int = 1024) -> int:
    """grouping.py:66-68."""
    k = max(1, (n + block_rows - 1) // block_rows)
    return min(k, max_clusters, n)


def linspace_f32(start: float, end: float, steps: int) -> np.ndarray:
    """torch.linspace in float32: step = (end-start)/(steps-1) in fp32, lower half
    fma(step, i, start), upper half fma(-step, steps-1-i, end), each rounded once
    (the form torch's CPU kernel evaluates; pinned by tests against torch)."""
    if steps == 1:
        return np.array([start], np.float32)
    s0, s1 = F32(start), F32(end)
    step = F32(F32(s1 - s0) / F32(steps - 1))
    i = np.arange(steps)
    lo = (np.float64(step) * i + np.float64(s0)).astype(np.float32)
    hi = (np.float64(s1) - np.float64(step) * (steps - 1 - i)).astype(np.float32)
    return np.where(i < steps // 2, lo, hi).astype(np.float32)


def seed_indices(n: int, k: int, init_samples: int = 4) -> Tuple[np.ndarray, int]:
    """Token indices and samples-per-centroid of grouping.py:71-83."""
    m = min(n, k * init_samples)
    idx = np.round(linspace_f32(0.0, float(n - 1), m)).astype(np.int64)
    m_per = max(1, m // k)
    return idx[: m_per * k], m_per


def seed_centroids(vb: np.ndarray, k: int, init_samples: int = 4) -> np.ndarray:
    """Strided-subsample seeding, grouping.py:71-83.  bf16 mean = fp32 sum of the
    m_per samples / m_per, rounded to bf16 (probed against torch)."""
    g, n, d = vb.shape
    idx, m_per = seed_indices(n, k, init_samples)
    sub = vb[:, idx, :].reshape(g, k, m_per, d)
    s = np.sum(sub.astype(np.float64), axis=2).astype(np.float32)
    return bf16_round(s / F32(m_per))


def sq_norms_f32(cb: np.ndarray) -> np.ndarray:
    """|c|^2 per centroid: sequential fp32 sum over channels of exact squares."""
    acc = np.zeros(cb.shape[:-1], np.float32)
    for j in range(cb.shape[-1]):
        acc = (acc + cb[..., j] * cb[..., j]).astype(np.float32)
    return acc


def assign(vb: np.ndarray, cb: np.ndarray) -> np.ndarray:
    """Nearest-centroid labels, grouping.py:86-100.

    sim = bf16(v.c) * 2 - |c|^2 (fp32), label = first argmax.  The bf16 GEMM's
    fp32 accumulation order is fixed here as sequential over channels
    (bf16 x bf16 products are exact in fp32, so this equals an FMA chain).
    """
    g, n, d = vb.shape
    c2 = sq_norms_f32(cb)                                  # (G, K)
    acc = np.zeros((g, n, cb.shape[1]), np.float32)
    for j in range(d):
        acc = (acc + vb[:, :, j:j + 1] * cb[:, None, :, j]).astype(np.float32)
    sim = (bf16_round(acc) * F32(2.0) - c2[:, None, :]).astype(np.float32)
    return np.argmax(sim, axis=-1).astype(np.int32)


def update_centroids(vb: np.ndarray, labels: np.ndarray, k: int,
                     init_samples: int = 4) -> np.ndarray:
    """grouping.py:103-124: fp32 sums in token order (index_add_), clamp(count,1),
    divide, re-seed clusters with count <= 1, round to bf16."""
    g, n, d = vb.shape
    out = np.zeros((g, k, d), np.float32)
    cnt = np.zeros((g, k), np.float32)
    for gi in range(g):
        lab = labels[gi]
        order = np.argsort(lab, kind="stable")
        sl = lab[order]
        bounds = np.searchsorted(sl, np.arange(k + 1))
        for c in range(k):
            a, b = bounds[c], bounds[c + 1]
            cnt[gi, c] = b - a
            if b > a:
                out[gi, c] = np.cumsum(vb[gi, order[a:b]], axis=0, dtype=np.float32)[-1]
    cntc = np.maximum(cnt, F32(1.0))
    new = (out / cntc[:, :, None]).astype(np.float32)
    empty = cntc <= 1.0
    if empty.any():
        filler = seed_centroids(vb, k, init_samples)
        new = np.where(empty[:, :, None], filler, new)
    return bf16_round(new)


def kmeans(vb: np.ndarray, k: int, iters: int, warm: Optional[np.ndarray] = None,
           warm_iters: int = 2, init_samples: int = 4):
    """grouping.py:127-147.  vb must hold bf16 values.  -> (labels, centroids)."""
    if warm is None:
        c = seed_centroids(vb, k, init_samples)
        n_it = iters
    else:
        c = bf16_round(warm)
        n_it = warm_iters
    labels = None
    for _ in range(n_it):
        labels = assign(vb, c)
        c = update_centroids(vb, labels, k, init_samples)
    labels = assign(vb, c)
    return labels, c


def build_permutation(vb: np.ndarray, block_rows: int = 128, iters: int = 3,
                      max_clusters: int = 1024, warm: Optional[np.ndarray] = None,
                      warm_iters: int = 2, tags: Optional[np.ndarray] = None,
                      modality_aware: bool = False, valid_len: Optional[int] = None):
    """grouping.py:150-186 -> (perm int32 (G,N), centroids, k)."""
    g, n, d = vb.shape
    k = num_clusters(n, block_rows, max_clusters)
    labels, cent = kmeans(vb, k, iters, warm, warm_iters)
    key = labels.astype(np.int64)
    if modality_aware and tags is not None:
        tag = np.maximum(np.asarray(tags, np.int64), -1)
        tag = np.where(tag < 0, 8, tag)
        key = tag[None, :] * (k + 1) + key
    if valid_len is not None and valid_len < n:
        is_pad = (np.arange(n) >= valid_len).astype(np.int64)
        key = key + is_pad[None, :] * (16 * (k + 1))
    perm = np.argsort(key, axis=-1, kind="stable").astype(np.int32)
    return perm, cent, k, labels


# ---------------------------------------------------------------------------
# prepare  (triton_attn.py:504-579) + routing statistics (:716-735)
# ---------------------------------------------------------------------------

def gather_rows(x: np.ndarray, perm: Optional[np.ndarray]) -> np.ndarray:
    if perm is None:
        return x
    p = np.asarray(perm, np.int64)
    if p.shape[0] == 1 and x.shape[0] > 1:
        p = np.broadcast_to(p, (x.shape[0], x.shape[1]))
    return np.take_along_axis(x, p[:, :, None], axis=1)


def prepare(q, k, v, perm=None, block_rows=128, hadamard=True, smooth_k=True) -> Dict[str, np.ndarray]:
    """Byte oracle of the Prepared layout (triton_attn.py:504-579).

    q, k, v: (G, N, D) float32 (bf16-exact values).  Means (K token mean,
    V block mean) use ``mean_f32`` (one rounding).  Returns a dict with the
    Prepared fields as (G, ...) arrays plus the float intermediates the
    routing statistics need (q_t, k_t padded).
    """
    g, n, d = q.shape
    n_pad = -(-n // block_rows) * block_rows
    nb = n_pad // block_rows
    qf = np.asarray(q, np.float32)
    kf = gather_rows(np.asarray(k, np.float32), perm)
    vf = gather_rows(np.asarray(v, np.float32), perm)
    q_t = fwht(qf) if hadamard else qf
    k_t = fwht(kf) if hadamard else kf
    if smooth_k:
        k_t = (k_t - mean_f32(k_t, axis=1)).astype(np.float32)
    q_codes, q_scale = quantize_e4m3_rows(q_t)
    k_codes, k_scale = quantize_e4m3_rows(k_t)
    pad = n_pad - n

    def padrows(x):
        if not pad:
            return x
        z = np.zeros((g, pad) + x.shape[2:], x.dtype)
        return np.concatenate([x, z], axis=1)

    vf_p = padrows(vf)
    vb = vf_p.reshape(g, nb, block_rows, d)
    mu = mean_f32(vb, axis=2)[:, :, 0, :]                           # (G, NB, D)
    resid = (vb - mu[:, :, None, :]).astype(np.float32).reshape(g, n_pad, d)
    v_codes, v_scale = quantize_e4m3_blocks(resid, block_rows)
    return {
        "q": padrows(q_codes), "q_scale": padrows(q_scale),
        "k": padrows(k_codes), "k_scale": padrows(k_scale),
        "v": v_codes, "v_scale": v_scale,
        "mu": (mu / v_scale).astype(np.float32),
        "mean": mu, "n_pad": n_pad,
        "q_t": padrows(q_t), "k_t": padrows(k_t),
    }


def nvfp4_per_head(x_t: np.ndarray):
    """NVFP4 of a (G, NP, D) tensor with one tensor scale per (b, h):
    quant.py:172-204 applied to each head's row-major (NP, D) slab.
    -> (packed (G,NP,D/2) uint8, micro (G,NP,D/16) uint8, g (G,) fp32)."""
    G, NP, D = x_t.shape
    packed = np.zeros((G, NP, D // 2), np.uint8)
    micro = np.zeros((G, NP, D // 16), np.uint8)
    gs = np.zeros((G,), np.float32)
    for i in range(G):
        c, m, gg = quantize_nvfp4(x_t[i])
        packed[i] = pack_nibbles(c.reshape(NP, D))
        micro[i] = m.reshape(NP, D // 16)
        gs[i] = gg
    return packed, micro, gs


def route_stats(prep: Dict[str, np.ndarray], block_rows: int, q_block: int,
                tau: float, scale: float) -> Dict[str, np.ndarray]:
    """Routing statistics of triton_attn.py:716-735 on the tensors prepare()
    quantises, with every mean and dot rounded once (float64 accumulation).

    k_mean (G,NB,D), v_mean (G,NB,D), thresh (G,NQB).
    thresh = mean_j(P) + tau * std_pop_j(P), P = (q_cent . k_mean) * scale.
    """
    q_t, k_t = prep["q_t"], prep["k_t"]
    g, n_pad, d = k_t.shape
    nb = n_pad // block_rows
    nqb = n_pad // q_block
    k_mean = mean_f32(k_t.reshape(g, nb, block_rows, d), axis=2)[:, :, 0, :]
    q_cent = mean_f32(q_t.reshape(g, nqb, q_block, d), axis=2)[:, :, 0, :]
    dots = np.einsum("gid,gjd->gij", q_cent.astype(np.float64), k_mean.astype(np.float64))
    proxy = (dots.astype(np.float32) * F32(scale)).astype(np.float32)
    mean = mean_f32(proxy, axis=2)
    dev = (proxy - mean).astype(np.float32)
    var = mean_f32((dev * dev).astype(np.float32), axis=2)
    thr = (mean + F32(tau) * np.sqrt(var).astype(np.float32)).astype(np.float32)
    return {"k_mean": k_mean, "v_mean": prep["mean"], "thresh": thr[:, :, 0]}


def route_mask(prep: Dict[str, np.ndarray], stats: Dict[str, np.ndarray], n: int,
               block_rows: int, q_block: int, scale: float, local_blocks: int = 1,
               sink_blocks: int = 0) -> Tuple[np.ndarray, np.ndarray]:
    """Block routing of triton_attn.py:449-459, restated with one rounding per
    reduction.  Per q-block i and KV block j:

      w_r   = fp32(qs_r * scale)
      qbar  = fp32( sum_r fp32(q8_r * w_r) )             (rows of q-block i)
      score = fp32( qbar . bf16(k_mean_j) ) / q_block    (fp32 division)
      keep  = score > thresh_i  or |i*q_block//BR - j| <= local  or  j < sink

    The reference kernel forms the same row-mean of the per-row proxy
    (q8_r . bf16(k_mean_j)) * qs_r * scale with an unspecified fp32 tree sum;
    this restatement fixes a single rounding of the sum.
    Returns (keep bool (G,NQB,NB), score fp32 (G,NQB,NB)).
    """
    q8 = e4m3_decode(prep["q"])                       # (G, NP, D)
    qs = prep["q_scale"]                              # (G, NP)
    g, n_pad, d = q8.shape
    nb = n_pad // block_rows
    nqb = n_pad // q_block
    w = (qs * F32(scale)).astype(np.float32)
    prod = (q8 * w[:, :, None]).astype(np.float32)
    qbar = np.sum(prod.reshape(g, nqb, q_block, d).astype(np.float64), axis=2).astype(np.float32)
    kmb = bf16_round(stats["k_mean"])
    dots = np.einsum("gid,gjd->gij", qbar.astype(np.float64), kmb.astype(np.float64)).astype(np.float32)
    score = (dots / F32(q_block)).astype(np.float32)
    qi = np.arange(nqb)[:, None]
    kj = np.arange(nb)[None, :]
    qb_kv = (qi * q_block) // block_rows
    keep = (score > stats["thresh"][:, :, None]) | (np.abs(qb_kv - kj) <= local_blocks)[None] \
        | (kj < sink_blocks)[None]
    return keep, score


# ---------------------------------------------------------------------------
# ExpCast  (expcast.py:52-70)
# ---------------------------------------------------------------------------

def expcast_codes(s: np.ndarray, m: np.ndarray, beta: float = -0.35) -> np.ndarray:
    """u = (s - m) * LOG2E + 8 ; c = u * 8 + (56 + beta) ; clamp(round_even(c), 0, 120)."""
    u = ((np.asarray(s, np.float32) - np.asarray(m, np.float32)[..., None]) * F32(LOG2E)
         + F32(8.0)).astype(np.float32)
    c = (u * F32(8.0) + F32(56.0 + beta)).astype(np.float32)
    return np.clip(np.round(c), 0, 120).astype(np.uint8)


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------

def attention_reference(q, k, v, perm=None, block_rows=128, block_m=64, expcast=False,
                        beta=-0.35, scale=None, vsmooth=True, hadamard=True,
                        smooth_k=True, q_rows=None, valid_len=None) -> np.ndarray:
    """vc_attention_reference (kernels/reference.py:162-294), backend fp8, in
    fp32 value units.  q,k,v: (G,N,D) float32.  Returns (G,N,D) float32, or
    (G,q_rows,D) when only the first ``q_rows`` query rows are wanted (the
    CPU-baseline sample; every query row costs the same).  ``valid_len``
    (reference.py:197, 251-256): keys at permuted positions >= valid_len are
    masked out (score -1e30), like the zero padding past N.
    """
    g, n, d = q.shape
    if scale is None:
        scale = d ** -0.5
    kf = gather_rows(np.asarray(k, np.float32), perm)
    vf = gather_rows(np.asarray(v, np.float32), perm)
    n_pad = -(-n // block_rows) * block_rows
    pad = n_pad - n
    if pad:
        z = np.zeros((g, pad, d), np.float32)
        kf = np.concatenate([kf, z], 1)
        vf = np.concatenate([vf, z], 1)
    nb = n_pad // block_rows
    if vsmooth:
        vb = vf.reshape(g, nb, block_rows, d)
        mu = mean_f32(vb, axis=2)[:, :, 0, :]
        resid = (vb - mu[:, :, None, :]).astype(np.float32).reshape(g, n_pad, d)
    else:
        mu, resid = None, vf
    vc, vsc = quantize_e4m3_blocks(resid, block_rows)
    v_hat = dequantize_e4m3_blocks(vc, vsc, block_rows)
    qf = np.asarray(q, np.float32)
    q_t = fwht(qf) if hadamard else qf
    k_t = fwht(kf) if hadamard else kf
    if smooth_k:
        k_t = (k_t - mean_f32(k_t, axis=1)).astype(np.float32)   # over n_pad rows (reference.py:236)
    qc, qsc = quantize_e4m3_rows(q_t)
    kc, ksc = quantize_e4m3_rows(k_t)
    q_hat = (e4m3_decode(qc) * qsc[..., None]).astype(np.float32)
    k_hat = (e4m3_decode(kc) * ksc[..., None]).astype(np.float32)
    inv_p = F32(1.0 / P_SCALE)
    n_out = n if q_rows is None else min(n, q_rows)
    out = np.zeros((g, n_out, d), np.float32)
    for sm in range(0, n_out, block_m):
        em = min(n_out, sm + block_m)
        qb = (q_hat[:, sm:em, :] * F32(scale)).astype(np.float32)
        mb = np.full((g, em - sm), -np.inf, np.float32)
        lb = np.zeros((g, em - sm), np.float32)
        ab = np.zeros((g, em - sm, d), np.float32)
        for j in range(nb):
            js, je = j * block_rows, (j + 1) * block_rows
            s = np.matmul(qb, k_hat[:, js:je, :].transpose(0, 2, 1)).astype(np.float32)
            n_valid = n if valid_len is None else valid_len
            if n_valid < n_pad:
                s = np.where((np.arange(js, je) >= n_valid)[None, None, :], F32(-1e30), s)
            m_new = np.maximum(mb, s.max(-1))
            m_new = np.where(np.isneginf(m_new), F32(0), m_new).astype(np.float32)
            if expcast:
                p = (e4m3_decode(expcast_codes(s, m_new, beta)) / F32(256.0)).astype(np.float32)
            else:
                e = np.exp2(((s - m_new[..., None]) * F32(LOG2E)).astype(np.float32)).astype(np.float32)
                p = (e4m3_decode(e4m3_encode((e / inv_p).astype(np.float32))) * inv_p).astype(np.float32)
            p = np.where(p < 0, F32(0), p)
            with np.errstate(over="ignore", invalid="ignore"):
                alpha = np.exp2(((mb - m_new) * F32(LOG2E)).astype(np.float32)).astype(np.float32)
            alpha = np.where(np.isneginf(mb), F32(0), alpha)
            r = p.sum(-1, dtype=np.float32)
            ab = (ab * alpha[..., None] + np.matmul(p, v_hat[:, js:je, :])).astype(np.float32)
            if mu is not None:
                ab = (ab + r[..., None] * mu[:, j, None, :]).astype(np.float32)
            lb = (lb * alpha + r).astype(np.float32)
            mb = m_new
        out[:, sm:em, :] = ab / np.maximum(lb, TINY)[..., None]
    return out


def _exact_tile(q8s, qs_rows, k8_blk, ks_blk, v8_blk, vs_row, mu_row, valid, sm_scale,
                m_i, l_i, acc, expcast, beta):
    """One exact KV tile in code units (triton_attn.py:254-318 == :324-382):
    s = dot(q8, k8) * (qs*ks) * sm_scale ; P as E4M3 (exp2*448 cast or ExpCast);
    r = sum(P)/448 ; acc = alpha*acc + (P@V8)*vs/448 + r*mu*vs ; l = alpha*l + r.
    """
    s_dot = np.matmul(q8s, k8_blk.T).astype(np.float32)
    s = (s_dot * (qs_rows[:, None] * ks_blk[None, :]).astype(np.float32)).astype(np.float32)
    s = (s * F32(sm_scale)).astype(np.float32)
    return _tile_from_scores(s, v8_blk, vs_row, mu_row, valid, m_i, l_i, acc, expcast, beta)


def _tile_softmax(s, valid, m_i, expcast, beta):
    """Online max, rescale factor and P values of one tile's scores
    (triton_attn.py:272-295): returns (m_new, alpha, p8)."""
    s = np.where(valid[None, :], s, F32(-1e30))
    m_new = np.maximum(m_i, s.max(-1))
    m_new = np.where(np.isneginf(m_new), F32(0), m_new).astype(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        alpha = np.exp2(((m_i - m_new) * F32(LOG2E)).astype(np.float32)).astype(np.float32)
    alpha = np.where(np.isneginf(m_i), F32(0), alpha)
    if expcast:
        p8 = e4m3_decode(expcast_codes(s, m_new, beta))
    else:
        e = np.exp2(((s - m_new[:, None]) * F32(LOG2E)).astype(np.float32)).astype(np.float32)
        p8 = e4m3_decode(e4m3_encode((e * F32(P_SCALE)).astype(np.float32)))
    return m_new, alpha, p8


def _tile_from_scores(s, v8_blk, vs_row, mu_row, valid, m_i, l_i, acc, expcast, beta):
    """The part of the exact tile after the scores: online max, P bytes, row
    sum and the V-Smooth accumulation (triton_attn.py:272-318)."""
    m_new, alpha, p8 = _tile_softmax(s, valid, m_i, expcast, beta)
    r = (p8.sum(-1, dtype=np.float32) / F32(P_SCALE)).astype(np.float32)
    tile = np.matmul(p8, v8_blk).astype(np.float32)
    acc = (acc * alpha[:, None]).astype(np.float32)
    acc = (acc + tile * (vs_row / F32(P_SCALE))[None, :]).astype(np.float32)
    acc = (acc + r[:, None] * (mu_row * vs_row)[None, :]).astype(np.float32)
    l_i = (l_i * alpha + r).astype(np.float32)
    return m_new, l_i, acc


def _row_starts(n: int, block_m: int, row_blocks: Optional[Sequence[int]]):
    """(index, first row) of the block_m-row query blocks to evaluate: all of
    them, or only ``row_blocks`` (rows of the others stay zero)."""
    nqb = -(-n // block_m)
    idx = range(nqb) if row_blocks is None else sorted(set(int(i) for i in row_blocks))
    return [(i, i * block_m) for i in idx if 0 <= i < nqb]


def attention_codes(prep: Dict[str, np.ndarray], n: int, block_rows: int, block_m: int,
                    sm_scale: float, expcast: bool = False, beta: float = -0.35,
                    row_blocks: Optional[Sequence[int]] = None,
                    kv_len: Optional[Sequence[int]] = None,
                    kv_piece_tiles: Optional[int] = None) -> np.ndarray:
    """The fused kernel's arithmetic in code units (triton_attn.py:203-322):
    s = dot(q8,k8) * (qs*ks) * sm_scale ; P as E4M3 (exp2*448 cast or ExpCast);
    r = sum(P)/448 ; acc = alpha*acc + (P@V8)*vs/448 + r*mu*vs ; O = acc/l.
    Consumes prepare() output; returns (G, N, D) float32.  ``row_blocks``
    restricts the evaluation to those query blocks (full-size spot checks).
    ``kv_len`` (G,): per head, only keys below it take part (key padding,
    reference.py valid_len); KV tiles entirely past it are not visited, which
    leaves every value as if they had been visited with all keys masked.
    ``kv_piece_tiles`` (this build's split of the KV axis, no counterpart in
    the reference): the KV tiles run in pieces of that many tiles, each piece
    from a fresh running max, sum and accumulator (its P bytes relative to its
    own max), and the pieces combine as O = sum_p w_p acc_p / sum_p w_p l_p
    with w_p = exp2((m_p - max_p m_p) log2e).
    """
    q8 = e4m3_decode(prep["q"])
    k8 = e4m3_decode(prep["k"])
    v8 = e4m3_decode(prep["v"])
    qs, ks, vs, mu = prep["q_scale"], prep["k_scale"], prep["v_scale"], prep["mu"]
    g, n_pad, d = q8.shape
    nb = n_pad // block_rows
    out = np.zeros((g, n, d), np.float32)
    for gi in range(g):
        for _, sm in _row_starts(n, block_m, row_blocks):
            em = min(n, sm + block_m)
            rows = em - sm
            kv = n if kv_len is None else max(1, min(n, int(kv_len[gi])))
            tiles = -(-kv // block_rows)
            step = tiles if kv_piece_tiles is None else int(kv_piece_tiles)
            parts = []
            for j0 in range(0, tiles, step):
                m_i = np.full(rows, -np.inf, np.float32)
                l_i = np.zeros(rows, np.float32)
                acc = np.zeros((rows, d), np.float32)
                for j in range(j0, min(tiles, j0 + step)):
                    js, je = j * block_rows, (j + 1) * block_rows
                    m_i, l_i, acc = _exact_tile(
                        q8[gi, sm:em], qs[gi, sm:em], k8[gi, js:je], ks[gi, js:je], v8[gi, js:je],
                        vs[gi, j], mu[gi, j], np.arange(js, je) < kv, sm_scale, m_i, l_i, acc,
                        expcast, beta)
                parts.append((m_i, l_i, acc))
            if len(parts) == 1:
                out[gi, sm:em] = acc / l_i[:, None]
                continue
            mx = np.max(np.stack([pm for pm, _, _ in parts]), axis=0)
            num = np.zeros((rows, d), np.float64)
            den = np.zeros(rows, np.float64)
            for pm, pl, pa in parts:
                w = np.exp2((pm.astype(np.float64) - mx) * LOG2E)
                num += w[:, None] * pa
                den += w * pl
            out[gi, sm:em] = (num / den[:, None]).astype(np.float32)
    return out


def attention_codes_units(prep: Dict[str, np.ndarray], n: int, block_rows: int, block_m: int,
                          sm_scale: float, expcast: bool = False, beta: float = -0.35,
                          floor_exp: int = -120) -> np.ndarray:
    """attention_codes (triton_attn.py:203-322) with the output accumulated the
    way a kernel that lets the P.V tensor-core MMA add into O itself must: in
    units of the current value block's scale.  With u_j = max(vs_j, floor) per
    channel, O_hat holds acc * 448 / u_j; before block j's P.V it gets block
    j-1's mean term R_{j-1} * mu_{j-1} and the factor alpha_j * u_{j-1} / u_j,
    then the MMA adds P_j . V8_j unscaled; the output is O_hat * u_last / 448 / l.
    floor = max|V_c| * 448 * 2^floor_exp per channel keeps O_hat finite when a
    block's scale sits at the amax clamp (a constant channel); such a block's
    codes are then counted at the floor's scale.  The result differs from
    attention_codes only by float32 rounding (and, for floored blocks, by at
    most 448 * 2^floor_exp of max|V_c|).  Returns (G, N, D) float32.
    """
    q8 = e4m3_decode(prep["q"])
    k8 = e4m3_decode(prep["k"])
    v8 = e4m3_decode(prep["v"])
    qs, ks, vs, mu = prep["q_scale"], prep["k_scale"], prep["v_scale"], prep["mu"]
    g, n_pad, d = q8.shape
    nb = n_pad // block_rows
    out = np.zeros((g, n, d), np.float32)
    for gi in range(g):
        # max |V_c| over the head: |mean| + the residual bound 448 * scale
        vmax = np.max(np.abs(mu[gi] * vs[gi]) + F32(P_SCALE) * vs[gi], axis=0).astype(np.float32)
        floor = (vmax * F32(P_SCALE) * F32(2.0 ** floor_exp)).astype(np.float32)
        for _, sm in _row_starts(n, block_m, None):
            em = min(n, sm + block_m)
            rows = em - sm
            m_i = np.full(rows, -np.inf, np.float32)
            l_i = np.zeros(rows, np.float32)
            oh = np.zeros((rows, d), np.float32)
            u_prev = r_prev = mu_prev = None
            for j in range(nb):
                js, je = j * block_rows, (j + 1) * block_rows
                sd = np.matmul(q8[gi, sm:em], k8[gi, js:je].T).astype(np.float32)
                sc = (sd * (qs[gi, sm:em, None] * ks[gi, None, js:je]).astype(np.float32)).astype(np.float32)
                sc = (sc * F32(sm_scale)).astype(np.float32)
                m_new, alpha, p8 = _tile_softmax(sc, np.arange(js, je) < n, m_i, expcast, beta)
                r = p8.sum(-1, dtype=np.float32)                 # un-normalised row sum
                u = np.maximum(vs[gi, j], floor).astype(np.float32)
                if u_prev is not None:
                    oh = (oh + (r_prev[:, None] * mu_prev[None, :]).astype(np.float32)).astype(np.float32)
                    f = (alpha[:, None] * (u_prev / u).astype(np.float32)[None, :]).astype(np.float32)
                    oh = (oh * f).astype(np.float32)
                else:
                    oh = (oh * alpha[:, None]).astype(np.float32)
                oh = (oh + np.matmul(p8, v8[gi, js:je]).astype(np.float32)).astype(np.float32)
                l_i = (l_i * alpha + (r / F32(P_SCALE)).astype(np.float32)).astype(np.float32)
                # mu is in units of vs_j; in units of u_j it carries vs_j / u_j
                u_prev, r_prev, m_i = u, r, m_new
                mu_prev = (mu[gi, j] * (vs[gi, j] / u).astype(np.float32)).astype(np.float32)
            oh = (oh + (r_prev[:, None] * mu_prev[None, :]).astype(np.float32)).astype(np.float32)
            o = (oh * (u_prev / F32(P_SCALE)).astype(np.float32)[None, :]).astype(np.float32)
            out[gi, sm:em] = (o / l_i[:, None]).astype(np.float32)
    return out


def attention_codes_nvfp4(prep: Dict[str, np.ndarray], n: int, block_rows: int, block_m: int,
                          sm_scale: float, expcast: bool = False, beta: float = -0.35,
                          row_blocks: Optional[Sequence[int]] = None) -> np.ndarray:
    """NVFP4-QK variant of attention_codes (triton_attn.py:227-239, 263-271 with
    the tensor-scaled NVFP4 of quant.py:172-204): Q and K are the NVFP4 codes
    of the rotated (and smoothed) rows with one tensor scale per head,
    s = dot(q4 * micro_q, k4 * micro_k) * fp32(fp32(g_q * g_k) * sm_scale)
    (the block-scaled MMA's product, then one scale for the whole head); P and
    V stay FP8 exactly as in attention_codes.  Returns (G, N, D) float32;
    ``row_blocks`` restricts the evaluation to those query blocks.
    """
    def deq(x_t):
        packed, micro, gs = nvfp4_per_head(x_t)
        g_, np_, dh = packed.shape
        codes = np.stack([packed & 0xF, packed >> 4], axis=-1).reshape(g_, np_, dh * 2)
        vals = fp4_decode(codes).astype(np.float32) * np.repeat(e4m3_decode(micro).astype(np.float32), 16, axis=-1)
        return vals.astype(np.float32), gs
    q4, gq = deq(prep["q_t"])
    k4, gk = deq(prep["k_t"])
    v8 = e4m3_decode(prep["v"])
    vs, mu = prep["v_scale"], prep["mu"]
    g, n_pad, d = q4.shape
    nb = n_pad // block_rows
    out = np.zeros((g, n, d), np.float32)
    for gi in range(g):
        c = F32(F32(gq[gi] * gk[gi]) * F32(sm_scale))
        for _, sm in _row_starts(n, block_m, row_blocks):
            em = min(n, sm + block_m)
            rows = em - sm
            m_i = np.full(rows, -np.inf, np.float32)
            l_i = np.zeros(rows, np.float32)
            acc = np.zeros((rows, d), np.float32)
            for j in range(nb):
                js, je = j * block_rows, (j + 1) * block_rows
                s = (np.matmul(q4[gi, sm:em], k4[gi, js:je].T).astype(np.float32) * c).astype(np.float32)
                m_i, l_i, acc = _tile_from_scores(s, v8[gi, js:je], vs[gi, j], mu[gi, j], np.arange(js, je) < n,
                                                  m_i, l_i, acc, expcast, beta)
            out[gi, sm:em] = acc / l_i[:, None]
    return out


def attention_sparse_codes(prep, stats, keep, n, block_rows, block_m, sm_scale,
                           group=16, expcast=False, beta=-0.35, row_blocks=None) -> np.ndarray:
    """Sparse kernel arithmetic (triton_attn.py:384-501) driven by a given
    routing mask ``keep`` (G, NP/block_m, NB).  Per KV group of ``group``
    blocks: approximated blocks are folded first with their per-row proxy
    score s_ap = (q8 . bf16(k_mean)) * qs * sm_scale, weighted by the block's
    real length, against bf16(p_ap) @ bf16(v_mean); kept blocks then run the
    exact tile in ascending order.  ``row_blocks`` restricts the evaluation
    to those query blocks.
    """
    q8 = e4m3_decode(prep["q"])
    k8 = e4m3_decode(prep["k"])
    v8 = e4m3_decode(prep["v"])
    qs, ks, vs, mu = prep["q_scale"], prep["k_scale"], prep["v_scale"], prep["mu"]
    kmb = bf16_round(stats["k_mean"])
    vmb = bf16_round(stats["v_mean"])
    g, n_pad, d = q8.shape
    nb = n_pad // block_rows
    out = np.zeros((g, n, d), np.float32)
    for gi in range(g):
        for qi, sm in _row_starts(n, block_m, row_blocks):
            em = min(n, sm + block_m)
            rows = em - sm
            m_i = np.full(rows, -np.inf, np.float32)
            l_i = np.zeros(rows, np.float32)
            acc = np.zeros((rows, d), np.float32)
            q8s = q8[gi, sm:em]
            qsc = (qs[gi, sm:em] * F32(sm_scale)).astype(np.float32)
            for g0 in range(0, nb, group):
                blks = np.arange(g0, min(nb, g0 + group))
                kp = keep[gi, qi, blks]
                proxy = (np.matmul(q8s, kmb[gi, blks].T).astype(np.float32) * qsc[:, None]).astype(np.float32)
                approx = ~kp
                if approx.any():
                    s_ap = np.where(approx[None, :], proxy, -np.inf).astype(np.float32)
                    m_new = np.maximum(m_i, s_ap.max(-1))
                    m_new = np.where(np.isneginf(m_new), F32(0), m_new).astype(np.float32)
                    with np.errstate(over="ignore", invalid="ignore"):
                        alpha = np.exp2(((m_i - m_new) * F32(LOG2E)).astype(np.float32)).astype(np.float32)
                        alpha = np.where(np.isneginf(m_i), F32(0), alpha)
                        p_ap = np.exp2(((s_ap - m_new[:, None]) * F32(LOG2E)).astype(np.float32)).astype(np.float32)
                    p_ap = np.where(approx[None, :], p_ap, F32(0))
                    lengths = np.minimum(block_rows, n - blks * block_rows).astype(np.float32)
                    p_ap = (p_ap * lengths[None, :]).astype(np.float32)
                    acc = (acc * alpha[:, None] + np.matmul(bf16_round(p_ap), vmb[gi, blks])).astype(np.float32)
                    l_i = (l_i * alpha + p_ap.sum(-1, dtype=np.float32)).astype(np.float32)
                    m_i = m_new
                for bj in blks[kp]:
                    js, je = bj * block_rows, (bj + 1) * block_rows
                    m_i, l_i, acc = _exact_tile(
                        q8s, qs[gi, sm:em], k8[gi, js:je], ks[gi, js:je], v8[gi, js:je],
                        vs[gi, bj], mu[gi, bj], np.arange(js, je) < n, sm_scale, m_i, l_i,
                        acc, expcast, beta)
            out[gi, sm:em] = acc / l_i[:, None]
    return out


def sdpa_f32(q, k, v, scale=None) -> np.ndarray:
    """Exact softmax attention in float64, returned as float32 (the PSNR target)."""
    g, n, d = q.shape
    if scale is None:
        scale = d ** -0.5
    out = np.zeros((g, n, d), np.float32)
    for gi in range(g):
        s = (q[gi].astype(np.float64) @ k[gi].astype(np.float64).T) * scale
        s -= s.max(-1, keepdims=True)
        p = np.exp(s)
        out[gi] = ((p @ v[gi].astype(np.float64)) / p.sum(-1, keepdims=True)).astype(np.float32)
    return out


def psnr(out, ref) -> float:
    """Peak-power PSNR of tests/bench_attention.py:55-57."""
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    mse = np.mean((out - ref) ** 2)
    return float(10 * np.log10(np.max(ref ** 2) / max(mse, 1e-30)))


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
