"""Fused VC-Attention on B200: host side of the libvcattn.so kernels.

Interface of the reference's vc_attention/kernels/triton_attn.py
(``TritonConfig`` :93-129, ``Prepared`` :140-165, ``prepare`` :504-579,
``restore`` :582-598, ``vc_attention_triton`` :757-855).  The reference name
``vc_attention_triton`` is kept as an alias of ``vc_attention_cuda`` so the
router calls it unchanged; there is no Triton and no CPU fallback here: a
failure raises, and the router (patch.py) turns that into "defer to the
original attention".

Per call (all on the current CUDA stream, no host synchronisation):
  1. vcattn_prepare_fp8 : permute K/V, Hadamard-rotate Q/K, subtract the K
     token mean, per-token E4M3 Q/K, V block demean + per-(block, channel)
     E4M3, and (sparse) the routing statistics;
  2. vcattn_route_mask  : the tau block mask (sparse only);
  3. vcattn_attn_fp8[_sparse] : the fused attention kernel.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import NamedTuple, Optional

import torch

from .. import _native as N
from ..grouping import _dtype_code, as_bhnd

__all__ = ["TritonConfig", "Prepared", "has_triton", "has_kernel", "prepare", "prepare_for", "slice_prepared",
           "restore", "vc_attention_host", "vc_attention_cuda", "vc_attention_triton", "route_mask"]

LOG2E = 1.4426950408889634
P_SCALE = 448.0


@dataclass
class TritonConfig:
    """Launch configuration (field names of triton_attn.py:93-129).

    block_m     rows per routing query block of the sparse path (the dense
                kernel's own tile is fixed by the kernel).
    block_n     KV tile == value block rows (64 or 128).
    num_warps / num_stages  accepted for interface parity, unused.
    pv_fp8      accepted; PV is always FP8 E4M3 here.
    expcast_exact  (this build) with enable_expcast, the dense tcgen05 kernel
                evaluates ExpCast in expcast.py's operation order instead of
                the one-FMA form (slower; for parity runs).
    kv_split    (this build) dense tcgen05 kernel: 1 = no split (default),
                0 = split the query tiles of a last partial wave of CTAs over
                their KV tiles when that wave would fill at most half of the
                SMs, k >= 2 = every query tile in k KV pieces
                (vcattn_attn_fp8_split; split tiles round P relative to each
                piece's own max).
    """
    block_m: int = 64
    block_n: int = 128
    num_warps: int = 4
    num_stages: int = 2
    enable_expcast: bool = False
    expcast_beta: float = -0.35
    pv_fp8: Optional[bool] = None
    qk_fp4: bool = False
    sparse: bool = False
    tau: float = 1.3
    local_blocks: int = 1
    sink_blocks: int = 0
    group: int = 16
    expcast_exact: bool = False
    kv_split: int = 1


class Prepared(NamedTuple):
    """Kernel operands (layout of triton_attn.py:140-165)."""
    q: torch.Tensor            # (B, H, NP, D) float8_e4m3fn
    q_scale: torch.Tensor      # (B, H, NP) fp32
    k: torch.Tensor            # (B, H, NP, D) float8_e4m3fn (permuted)
    k_scale: torch.Tensor      # (B, H, NP) fp32
    v: Optional[torch.Tensor]  # (B, H, NP, D) float8_e4m3fn residual codes (permuted)
    v_scale: torch.Tensor      # (B, H, NB, D) fp32
    mu: torch.Tensor           # (B, H, NB, D) fp32 block mean / v_scale
    n_pad: int
    q4: Optional[torch.Tensor] = None        # (B, H, NP, D/2) uint8 E2M1 pairs, low nibble first
    q4_scale: Optional[torch.Tensor] = None  # (B, H, NP, D/16) uint8 E4M3 micro scales
    k4: Optional[torch.Tensor] = None        # (B, H, NP, D/2) token-major (the reference: K-first)
    k4_scale: Optional[torch.Tensor] = None  # (B, H, NP, D/16)
    k_mean: Optional[torch.Tensor] = None   # (B, H, NB, D) fp32
    v_mean: Optional[torch.Tensor] = None   # (B, H, NB, D) fp32
    thresh: Optional[torch.Tensor] = None   # (B, H, NQB) fp32
    n_qblk: int = 0
    # build-specific operands
    v_t: Optional[torch.Tensor] = None      # (G, NB, D, block_rows) uint8 V codes, block-transposed
    ap_tiles: Optional[torch.Tensor] = None  # (G, ceil(NB/16), 8192) uint8 bf16 proxy tiles (tcgen05 sparse)
    q_cent: Optional[torch.Tensor] = None   # (G, NQB, D) fp32
    q_bar: Optional[torch.Tensor] = None    # (G, NQB, D) fp32
    keep: Optional[torch.Tensor] = None     # (G, NQB, NB) uint8 routing mask
    block_rows: int = 128
    v_mma_order: bool = False               # v rows in the tcgen05 kernel's key order
    q4_g: Optional[torch.Tensor] = None     # (G,) fp32 NVFP4 tensor scale per head
    k4_g: Optional[torch.Tensor] = None
    q4_sf_mma: Optional[torch.Tensor] = None  # (G, NP/128, D/64, 512) micro scales in MMA atom order
    k4_sf_mma: Optional[torch.Tensor] = None


def has_kernel() -> bool:
    """True when libvcattn.so is loaded and a CUDA device is visible."""
    return N.available() and torch.cuda.is_available()


# The reference's name for "the fused kernel can run".
has_triton = has_kernel


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _check_qkv(q, k, v):
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("VC-Attention kernels need CUDA tensors (this build has no CPU path)")
    if q.shape != k.shape or q.shape != v.shape or q.dim() != 4:
        raise ValueError(f"q, k, v must share a (B, H, N, D) shape, got {tuple(q.shape)}, "
                         f"{tuple(k.shape)}, {tuple(v.shape)}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, v must share a dtype")
    if q.shape[-1] not in (64, 128):
        raise ValueError(f"head_dim must be 64 or 128, got {q.shape[-1]}")


def prepare(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, perm: Optional[torch.Tensor] = None,
            block_rows: int = 128, hadamard: bool = True, smooth_k: bool = True, *,
            sparse: bool = False, tau: float = 1.3, q_block: int = 64,
            scale: Optional[float] = None, want_v: bool = True, want_v_t: bool = False,
            local_blocks: int = 1, sink_blocks: int = 0, v_mma_order: Optional[bool] = None,
            qk_fp4: bool = False, fp8_qk: bool = True) -> Prepared:
    """Quantise and permute Q/K/V into the kernel layout (triton_attn.py:504-579).

    Byte-identical to the reference's portable ``prepare`` on the codes; the
    scales that depend on a token/block mean differ from it only in the last
    bits (the mean is rounded once here).  With ``sparse=True`` the routing
    statistics and the block mask are produced as well; with ``qk_fp4=True``
    the NVFP4 Q/K of quant.py:172-204 (one tensor scale per head) too, and
    ``fp8_qk=False`` then leaves out the E4M3 Q/K codes (``q``, ``k`` None).
    """
    _check_qkv(q, k, v)
    lib = N.lib()
    b, h, n, d = q.shape
    g = b * h
    dev = q.device
    n_pad = -(-n // block_rows) * block_rows
    nb = n_pad // block_rows
    qv, _, _, _, _ = as_bhnd(q)
    kv, _, _, _, _ = as_bhnd(k)
    vv, _, _, _, _ = as_bhnd(v)
    dt = _dtype_code(qv._keep)
    if _dtype_code(kv._keep) != dt or _dtype_code(vv._keep) != dt:
        raise ValueError("q, k, v must share a dtype")
    perm_t = None
    perm_rows = 0
    if perm is not None:
        perm_t = perm.to(device=dev, dtype=torch.int32).contiguous()
        if perm_t.dim() != 2 or perm_t.shape[1] != n or perm_t.shape[0] not in (1, g):
            raise ValueError(f"perm must be (G, N) or (1, N), got {tuple(perm_t.shape)}")
        perm_rows = perm_t.shape[0]
    u8 = torch.uint8
    if not fp8_qk and (sparse or not qk_fp4):
        raise ValueError("fp8_qk=False is only for the NVFP4 QK path (qk_fp4=True, dense)")
    q8 = torch.empty((g, n_pad, d), dtype=u8, device=dev) if fp8_qk else None
    k8 = torch.empty((g, n_pad, d), dtype=u8, device=dev) if fp8_qk else None
    v8 = torch.empty((g, n_pad, d), dtype=u8, device=dev) if want_v else None
    v8t = torch.empty((g, nb, d, block_rows), dtype=u8, device=dev) if want_v_t else None
    qs = torch.empty((g, n_pad), dtype=torch.float32, device=dev) if fp8_qk else None
    ks = torch.empty((g, n_pad), dtype=torch.float32, device=dev) if fp8_qk else None
    vs = torch.empty((g, nb, d), dtype=torch.float32, device=dev)
    mu = torch.empty((g, nb, d), dtype=torch.float32, device=dev)
    flags = (N.HADAMARD if hadamard else 0) | (N.SMOOTH_K if smooth_k else 0)
    if v_mma_order is None:
        v_mma_order = sparse   # the order the matching tcgen05 kernel reads
    v_mma_order = bool(v_mma_order and want_v)
    if v_mma_order:
        flags |= N.V_MMA_ORDER
    sc = scale if scale is not None else d ** -0.5
    route = None
    k_mean = v_mean = q_cent = q_bar = None
    if sparse:
        if n_pad % q_block:
            raise ValueError("n_pad must be a multiple of q_block for routing")
        nqb = n_pad // q_block
        k_mean = torch.empty((g, nb, d), dtype=torch.float32, device=dev)
        v_mean = torch.empty((g, nb, d), dtype=torch.float32, device=dev)
        q_cent = torch.empty((g, nqb, d), dtype=torch.float32, device=dev)
        q_bar = torch.empty((g, nqb, d), dtype=torch.float32, device=dev)
        route = N.RouteStats(q_block, k_mean.data_ptr(), q_cent.data_ptr(), q_bar.data_ptr(),
                             v_mean.data_ptr(), float(sc))
    ws_bytes = lib.vcattn_prepare_workspace_bytes(g, n, d)
    ws = torch.empty(ws_bytes, dtype=u8, device=dev)
    N.check("vcattn_prepare_fp8", lib.vcattn_prepare_fp8(
        qv, kv, vv, dt, b, h, n, d, _ptr(perm_t), perm_rows, block_rows, flags,
        _ptr(q8), _ptr(qs), _ptr(k8), _ptr(ks), _ptr(v8), vs.data_ptr(),
        mu.data_ptr(), _ptr(v8t), route, ws.data_ptr(), ws_bytes, _stream(q)))
    q4 = q4s = k4 = k4s = q4g = k4g = q4sf = k4sf = None
    if qk_fp4:
        q4 = torch.empty((g, n_pad, d // 2), dtype=u8, device=dev)
        k4 = torch.empty((g, n_pad, d // 2), dtype=u8, device=dev)
        q4s = torch.empty((g, n_pad, d // 16), dtype=u8, device=dev)
        k4s = torch.empty((g, n_pad, d // 16), dtype=u8, device=dev)
        q4g = torch.empty((g,), dtype=torch.float32, device=dev)
        k4g = torch.empty((g,), dtype=torch.float32, device=dev)
        tiles = -(-n_pad // 128)
        q4sf = torch.empty((g, tiles, d // 64, 512), dtype=u8, device=dev)
        k4sf = torch.empty((g, tiles, d // 64, 512), dtype=u8, device=dev)
        N.check("vcattn_prepare_nvfp4", lib.vcattn_prepare_nvfp4(
            qv, kv, dt, b, h, n, d, _ptr(perm_t), perm_rows, block_rows, flags & ~N.V_MMA_ORDER,
            q4.data_ptr(), q4s.data_ptr(), q4g.data_ptr(), k4.data_ptr(), k4s.data_ptr(), k4g.data_ptr(),
            q4sf.data_ptr(), k4sf.data_ptr(), ws.data_ptr(), ws_bytes, _stream(q)))
    keep = thresh = ap_tiles = None
    nqb = 0
    if sparse:
        nqb = n_pad // q_block
        keep, thresh = route_mask(route, g, n, n_pad, d, block_rows, tau, local_blocks, sink_blocks,
                                  sc, dev, q)
        if d in (64, 128) and block_rows in (64, 128):
            ap_tiles = torch.empty((g, -(-nb // 16), 8192), dtype=u8, device=dev)
            N.check("vcattn_route_tiles", lib.vcattn_route_tiles(
                k_mean.data_ptr(), v_mean.data_ptr(), g, n_pad, d, block_rows, ap_tiles.data_ptr(), _stream(q)))
    f8 = torch.float8_e4m3fn
    return Prepared(
        q=None if q8 is None else q8.view(f8).view(b, h, n_pad, d),
        q_scale=None if qs is None else qs.view(b, h, n_pad),
        k=None if k8 is None else k8.view(f8).view(b, h, n_pad, d),
        k_scale=None if ks is None else ks.view(b, h, n_pad),
        v=None if v8 is None else v8.view(f8).view(b, h, n_pad, d),
        v_scale=vs.view(b, h, nb, d), mu=mu.view(b, h, nb, d), n_pad=n_pad,
        k_mean=None if k_mean is None else k_mean.view(b, h, nb, d),
        v_mean=None if v_mean is None else v_mean.view(b, h, nb, d),
        thresh=None if thresh is None else thresh.view(b, h, nqb), n_qblk=nqb,
        v_t=v8t, q_cent=q_cent, q_bar=q_bar, keep=keep, block_rows=block_rows, v_mma_order=v_mma_order,
        ap_tiles=ap_tiles,
        q4=None if q4 is None else q4.view(b, h, n_pad, d // 2),
        q4_scale=None if q4s is None else q4s.view(b, h, n_pad, d // 16),
        k4=None if k4 is None else k4.view(b, h, n_pad, d // 2),
        k4_scale=None if k4s is None else k4s.view(b, h, n_pad, d // 16), q4_g=q4g, k4_g=k4g,
        q4_sf_mma=q4sf, k4_sf_mma=k4sf)


def route_mask(route: "N.RouteStats", g: int, n: int, n_pad: int, d: int, block_rows: int, tau: float,
               local_blocks: int, sink_blocks: int, sm_scale: float, dev, like: torch.Tensor):
    nqb = n_pad // route.q_block
    nb = n_pad // block_rows
    keep = torch.empty((g, nqb, nb), dtype=torch.uint8, device=dev)
    thresh = torch.empty((g, nqb), dtype=torch.float32, device=dev)
    lib = N.lib()
    N.check("vcattn_route_mask", lib.vcattn_route_mask(
        route, g, n, n_pad, d, block_rows, float(tau), int(local_blocks), int(sink_blocks),
        float(sm_scale), keep.data_ptr(), thresh.data_ptr(), _stream(like)))
    return keep, thresh


def mma_key_slot(r: torch.Tensor) -> torch.Tensor:
    """Slot of value-block row r under VCATTN_V_MMA_ORDER (its own inverse)."""
    return (r & ~31) | (((r >> 1) & 3) << 3) | (((r >> 3) & 3) << 1) | (r & 1)


def v_natural(p: Prepared) -> torch.Tensor:
    """V codes (uint8) in token order, whichever order ``p.v`` is stored in."""
    v = p.v.view(torch.uint8)
    if not p.v_mma_order:
        return v
    idx = mma_key_slot(torch.arange(v.shape[-2], device=v.device))
    return v.index_select(-2, idx)


def restore(p: Prepared, block_rows: int = 128):
    """Dequantise a Prepared back to value/score units (tests; triton_attn.py:582-598)."""
    from ..quant import e4m3_decode
    b, h, np_, d = p.q.shape
    g = b * h
    qd = e4m3_decode(p.q.view(torch.uint8).reshape(g, np_, d)) * p.q_scale.reshape(g, np_, 1)
    kd = e4m3_decode(p.k.view(torch.uint8).reshape(g, np_, d)) * p.k_scale.reshape(g, np_, 1)
    vs = p.v_scale.reshape(g, -1, d).repeat_interleave(block_rows, dim=1)
    vd = e4m3_decode(v_natural(p).reshape(g, np_, d)) * vs
    vd = vd + p.mu.reshape(g, -1, d).repeat_interleave(block_rows, dim=1) * vs
    return qd, kd, vd


def _out_view(q: torch.Tensor, dtype: torch.dtype):
    """Output buffer in the input's token layout: a transposed (B, N, H, D)
    input (the ComfyUI 3-D path) gets a (B, N, H, D) buffer, so the caller's
    transpose-back is free."""
    b, h, n, d = q.shape
    if q.stride(-1) == 1 and q.stride(1) == d and q.stride(2) == h * d:
        buf = torch.empty((b, n, h, d), dtype=dtype, device=q.device)
        return buf.transpose(1, 2)
    return torch.empty((b, h, n, d), dtype=dtype, device=q.device)


def vc_attention_cuda(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      perm: Optional[torch.Tensor] = None, cfg: Optional[TritonConfig] = None,
                      scale: Optional[float] = None, kv_len: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused VC-Attention (triton_attn.py:757-855 semantics, no fallback).

    q, k, v: (B, H, N, D) CUDA bf16/fp16/fp32 (strided views accepted);
    perm: (G, N) or (1, N) int32 V-Smooth permutation or None.
    kv_len: None, or a (B,) int32 CUDA tensor: in batch entry b only the
    first kv_len[b] keys of the permuted order take part (key padding,
    reference.py ``valid_len``); the permutation must have sorted the
    excluded keys to the tail.  Dense FP8 only.
    Returns (B, H, N, D) in q.dtype.
    """
    return _attention_into(q, k, v, perm, cfg, scale, None, kv_len)


def _call_config(cfg, d):
    cfg = cfg or TritonConfig()
    if cfg.qk_fp4 and cfg.sparse:
        cfg = TritonConfig(**{**cfg.__dict__, "qk_fp4": False})
    if cfg.qk_fp4 and (d != 128 or cfg.block_n != 128):
        raise ValueError("the NVFP4 QK kernel needs D = 128 and block_n = 128")
    return cfg


def prepare_for(q, k, v, perm, cfg: Optional[TritonConfig] = None, scale: Optional[float] = None) -> Prepared:
    """The operands vc_attention_cuda prepares for ``cfg`` (the kernel family
    that will read them decides the V layout)."""
    _check_qkv(q, k, v)
    b, h, n, d = q.shape
    cfg = _call_config(cfg, d)
    if scale is None:
        scale = d ** -0.5
    br = cfg.block_n
    sparse = bool(cfg.sparse)
    fp4 = bool(cfg.qk_fp4)
    use_tc = (not sparse) or sparse_tc_applies(d, br, cfg.block_m, cfg.group, n)
    return prepare(q, k, v, perm, block_rows=br, hadamard=True, smooth_k=True, sparse=sparse,
                   tau=cfg.tau, q_block=cfg.block_m, scale=scale, want_v=use_tc, want_v_t=not use_tc,
                   local_blocks=cfg.local_blocks, sink_blocks=cfg.sink_blocks, qk_fp4=fp4, fp8_qk=not fp4)


_BH_FIELDS = ("q", "q_scale", "k", "k_scale", "v", "v_scale", "mu", "q4", "q4_scale", "k4", "k4_scale",
              "k_mean", "v_mean", "thresh")
_G_FIELDS = ("v_t", "ap_tiles", "q_cent", "q_bar", "keep", "q4_g", "k4_g", "q4_sf_mma", "k4_sf_mma")


def slice_prepared(p: Prepared, i: int) -> Prepared:
    """Batch entry ``i`` of a Prepared as a Prepared of batch 1 (views, no copy)."""
    b, h = (p.q if p.q is not None else p.v).shape[:2]
    upd = {}
    for name in _BH_FIELDS:
        t = getattr(p, name)
        if t is not None:
            upd[name] = t[i:i + 1]
    for name in _G_FIELDS:
        t = getattr(p, name)
        if t is not None:
            upd[name] = t[i * h:(i + 1) * h]
    return p._replace(**upd)


def _attention_into(q, k, v, perm, cfg, scale, out, kv_len=None):
    """vc_attention_cuda writing into ``out`` ((B, H, N, D) view of q's dtype,
    d contiguous), or into a new buffer when ``out`` is None."""
    _check_qkv(q, k, v)
    b, h, n, d = q.shape
    cfg = _call_config(cfg, d)
    if scale is None:
        scale = d ** -0.5
    p = prepare_for(q, k, v, perm, cfg, scale)
    if out is None:
        out = _out_view(q, q.dtype)
    elif out.shape != q.shape or out.dtype != q.dtype or out.stride(-1) != 1:
        raise ValueError("out must be a (B, H, N, D) view of q's dtype with d contiguous")
    return attention_prepared(p, n, out, scale, cfg, kv_len=kv_len)


def attention_prepared(p: Prepared, n: int, out: torch.Tensor, scale: float,
                       cfg: TritonConfig, kernel: str = "auto",
                       kv_len: Optional[torch.Tensor] = None, kv_split: Optional[int] = None) -> torch.Tensor:
    """Run the attention kernel on prepared operands, writing into ``out``.

    kernel: "tc" (tcgen05, needs ``p.v``), "mma" (register MMA,
    needs ``p.v_t``) or "auto" (tcgen05 whenever it applies), for the dense
    and the sparse path alike.  ``kv_len`` ((B,) int32 on the device) runs
    the key-padding masked dense tcgen05 kernel (vcattn_attn_fp8_masked).
    ``kv_split`` overrides ``cfg.kv_split`` for the dense tcgen05 kernel.
    """
    lib = N.lib()
    b, h, n_pad, d = (p.q if p.q is not None else p.v).shape
    flags = N.EXPCAST if cfg.enable_expcast else 0
    if cfg.enable_expcast and cfg.expcast_exact:
        flags |= N.EXPCAST_EXACT
    odt = _dtype_code(out)
    st = _stream(out)
    if kv_len is not None:
        if cfg.sparse or cfg.qk_fp4 or p.v is None or p.v_mma_order or kernel not in ("auto", "tc"):
            raise ValueError("masked attention runs on the dense FP8 tcgen05 kernel (token-order V)")
        kl = kv_len.to(device=out.device, dtype=torch.int32).contiguous()
        if kl.shape != (b,):
            raise ValueError(f"kv_len must be ({b},), got {tuple(kl.shape)}")
        N.check("vcattn_attn_fp8_masked", lib.vcattn_attn_fp8_masked(
            p.q.view(torch.uint8).data_ptr(), p.q_scale.data_ptr(), p.k.view(torch.uint8).data_ptr(),
            p.k_scale.data_ptr(), p.v.view(torch.uint8).data_ptr(), p.v_scale.data_ptr(), p.mu.data_ptr(),
            kl.data_ptr(), b, h, n, n_pad, d, p.block_rows, float(scale), flags, float(cfg.expcast_beta),
            out.data_ptr(), odt, out.stride(0), out.stride(1), out.stride(2), st))
        return out
    if cfg.qk_fp4 and not cfg.sparse:
        if p.q4 is None or p.v is None or p.v_mma_order:
            raise ValueError("the NVFP4 kernel needs prepare(qk_fp4=True, want_v=True, v_mma_order=False)")
        N.check("vcattn_attn_nvfp4", lib.vcattn_attn_nvfp4(
            p.q4.data_ptr(), p.q4_sf_mma.data_ptr(), p.q4_g.data_ptr(), p.k4.data_ptr(), p.k4_sf_mma.data_ptr(),
            p.k4_g.data_ptr(), p.v.view(torch.uint8).data_ptr(), p.v_scale.data_ptr(), p.mu.data_ptr(),
            b, h, n, n_pad, d, p.block_rows, float(scale), flags, float(cfg.expcast_beta), out.data_ptr(), odt,
            out.stride(0), out.stride(1), out.stride(2), st))
        return out
    if p.q is None or p.k is None:
        raise ValueError("the FP8 kernels need the E4M3 Q/K codes (prepare with fp8_qk=True)")
    q8 = p.q.view(torch.uint8)
    k8 = p.k.view(torch.uint8)
    if cfg.sparse:
        if kernel == "auto":
            kernel = "tc" if (p.v is not None and p.v_mma_order and p.ap_tiles is not None and
                              sparse_tc_applies(d, p.block_rows, cfg.block_m, cfg.group, n_pad)) else "mma"
        if kernel == "tc":
            if p.v is None or not p.v_mma_order or p.ap_tiles is None:
                raise ValueError("the tcgen05 sparse kernel reads V codes in its key order and the proxy "
                                 "tiles (want_v=True, v_mma_order=True, D and block_rows in {64, 128})")
            N.check("vcattn_attn_fp8_sparse_tc", lib.vcattn_attn_fp8_sparse_tc(
                q8.data_ptr(), p.q_scale.data_ptr(), k8.data_ptr(), p.k_scale.data_ptr(),
                p.v.view(torch.uint8).data_ptr(), p.v_scale.data_ptr(), p.mu.data_ptr(), p.ap_tiles.data_ptr(),
                p.keep.data_ptr(), cfg.block_m, cfg.group, b, h, n, n_pad, d,
                p.block_rows, float(scale), flags, float(cfg.expcast_beta), out.data_ptr(), odt,
                out.stride(0), out.stride(1), out.stride(2), st))
            return out
        if p.v_t is None:
            raise ValueError("the sparse kernel needs the block-transposed V codes (want_v_t=True)")
        N.check("vcattn_attn_fp8_sparse", lib.vcattn_attn_fp8_sparse(
            q8.data_ptr(), p.q_scale.data_ptr(), k8.data_ptr(), p.k_scale.data_ptr(),
            p.v_t.data_ptr(), p.v_scale.data_ptr(), p.mu.data_ptr(), p.k_mean.data_ptr(),
            p.v_mean.data_ptr(), p.keep.data_ptr(), cfg.block_m, cfg.group, b, h, n, n_pad, d,
            p.block_rows, float(scale), flags, float(cfg.expcast_beta), out.data_ptr(), odt,
            out.stride(0), out.stride(1), out.stride(2), st))
        return out
    if kernel == "auto":
        kernel = "tc" if (p.v is not None and not p.v_mma_order) else "mma"
    if kernel == "tc":
        if p.v is None or p.v_mma_order:
            raise ValueError("the dense tcgen05 kernel reads V codes in token order (want_v=True, v_mma_order=False)")
        split = cfg.kv_split if kv_split is None else int(kv_split)
        ws_bytes = lib.vcattn_attn_split_workspace_bytes(b, h, n, n_pad, d, p.block_rows, split)
        if ws_bytes == 0:
            N.check("vcattn_attn_fp8", lib.vcattn_attn_fp8(
                q8.data_ptr(), p.q_scale.data_ptr(), k8.data_ptr(), p.k_scale.data_ptr(),
                p.v.view(torch.uint8).data_ptr(), p.v_scale.data_ptr(), p.mu.data_ptr(), b, h, n, n_pad, d,
                p.block_rows, float(scale), flags, float(cfg.expcast_beta), out.data_ptr(), odt,
                out.stride(0), out.stride(1), out.stride(2), st))
        else:
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=out.device)
            N.check("vcattn_attn_fp8_split", lib.vcattn_attn_fp8_split(
                q8.data_ptr(), p.q_scale.data_ptr(), k8.data_ptr(), p.k_scale.data_ptr(),
                p.v.view(torch.uint8).data_ptr(), p.v_scale.data_ptr(), p.mu.data_ptr(), b, h, n, n_pad, d,
                p.block_rows, float(scale), flags, float(cfg.expcast_beta), out.data_ptr(), odt,
                out.stride(0), out.stride(1), out.stride(2), split, ws.data_ptr(), ws_bytes, st))
    else:
        if p.v_t is None:
            raise ValueError("the register-MMA kernel needs the block-transposed V codes (want_v_t=True)")
        N.check("vcattn_attn_fp8_mma", lib.vcattn_attn_fp8_mma(
            q8.data_ptr(), p.q_scale.data_ptr(), k8.data_ptr(), p.k_scale.data_ptr(),
            p.v_t.data_ptr(), p.v_scale.data_ptr(), p.mu.data_ptr(), b, h, n, n_pad, d,
            p.block_rows, float(scale), flags, float(cfg.expcast_beta), out.data_ptr(), odt,
            out.stride(0), out.stride(1), out.stride(2), st))
    return out


def sparse_tc_applies(d: int, block_rows: int, q_block: int, group: int, n: int) -> bool:
    """Whether the tcgen05 sparse kernel takes this shape (two 64-row routing
    blocks per CTA, head dim and value block of 64 or 128, groups of 16, at
    most 1024 KV tiles)."""
    nb = -(-n // block_rows)
    return (d in (64, 128) and block_rows in (64, 128) and q_block == 64 and group == 16
            and nb + -(-nb // 16) <= 1088)


def attention_status(reset: bool = True):
    """(code, where, block) of the tcgen05 kernels' device status word; code 0
    means every bounded wait completed.  Synchronises the device."""
    import ctypes
    code, where, block = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    lib = N.lib()
    N.check("vcattn_attn_status", lib.vcattn_attn_status(ctypes.byref(code), ctypes.byref(where),
                                                          ctypes.byref(block), 1 if reset else 0))
    return code.value, where.value, block.value


_HOST_STREAMS = {}


def _host_streams(dev: torch.device):
    """The copy-in, compute and copy-out streams of vc_attention_host, one set
    per device for the process: the caching allocator keeps freed blocks per
    stream, so fresh streams on every call would re-allocate (and free) the
    prepared operands each time."""
    key = dev.index
    if key not in _HOST_STREAMS:
        _HOST_STREAMS[key] = tuple(torch.cuda.Stream(dev) for _ in range(3))
    return _HOST_STREAMS[key]


def _chunk_bounds(g: int, c: int):
    """Unit ranges [lo, hi) for vc_attention_host: chunks of c units, with the
    last c (or fewer) units split into shrinking pieces (c=4: ..., 4, 2, 1, 1)
    so that the work left after the final copy-in, one piece's compute and
    copy-out, is small."""
    out, lo = [], 0
    while g - lo > c:
        out.append((lo, lo + c))
        lo += c
    while lo < g:
        r = g - lo
        s = r // 2 if r > 1 else 1
        out.append((lo, lo + s))
        lo += s
    return out


def vc_attention_host(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      perm: Optional[torch.Tensor] = None, cfg: Optional[TritonConfig] = None,
                      scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                      chunk_heads: Optional[int] = None, device=None) -> torch.Tensor:
    """VC-Attention of host-resident (B, H, N, D) tensors on one GPU.

    The path is independent per (b, h) unit, so the units are streamed in
    chunks of ``chunk_heads``: while chunk i is prepared and attended on one
    stream, chunk i+1 is copied in and chunk i-1 copied out on two others
    (double-buffered device slabs), so the host<->device transfers overlap the
    compute and each other.  q, k, v: contiguous (pinned for overlap) host
    tensors; perm: (G, N) or (1, N) int32 on the device, or None; out: a host
    tensor of q's shape and dtype (allocated pinned when None).  The call
    returns once ``out`` holds the result.
    """
    cfg = cfg or TritonConfig()
    if q.is_cuda or k.is_cuda or v.is_cuda:
        raise ValueError("vc_attention_host takes host tensors; use vc_attention_cuda for device tensors")
    if q.shape != k.shape or q.shape != v.shape or q.dim() != 4 or q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, v must share a (B, H, N, D) shape and dtype")
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
        raise ValueError("q, k, v must be contiguous (B, H, N, D) host tensors")
    b, h, n, d = q.shape
    g = b * h
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    if out.shape != q.shape or out.dtype != q.dtype or out.is_cuda or not out.is_contiguous():
        raise ValueError("out must be a contiguous host tensor of q's shape and dtype")
    c = chunk_heads or max(1, -(-g // 14))   # ~14 chunks: the copies dominate, keep the pipe full
    # chunks overlap one another, so no chunk's last wave is the call's tail:
    # no KV split (the output equals per-unit device calls bit for bit)
    cfg = replace(cfg, kv_split=1)
    if scale is None:
        scale = d ** -0.5
    src = [t.reshape(g, n, d) for t in (q, k, v)]
    dst = out.reshape(g, n, d)
    cur = torch.cuda.current_stream(dev)
    s_in, s_comp, s_out = _host_streams(dev)
    for st in (s_in, s_comp, s_out):
        st.wait_stream(cur)
    slab_in = [[torch.empty((c, n, d), dtype=q.dtype, device=dev) for _ in range(3)] for _ in range(2)]
    slab_out = [torch.empty((c, n, d), dtype=q.dtype, device=dev) for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]
    for i, (lo, hi) in enumerate(_chunk_bounds(g, c)):
        u, slot = hi - lo, i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(comp_done[slot])     # chunk i-2 no longer reads this slab
            for t_h, t_d in zip(src, slab_in[slot]):
                t_d[:u].copy_(t_h[lo:hi], non_blocking=True)
            in_ready[slot].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(in_ready[slot])
            if i >= 2:
                s_comp.wait_event(out_done[slot])    # chunk i-2's result copied out
            qd, kd, vd = (t[:u].unsqueeze(0) for t in slab_in[slot])
            pl = None if perm is None else (perm if perm.shape[0] == 1 else perm[lo:hi])
            _attention_into(qd, kd, vd, pl, cfg, scale, slab_out[slot][:u].unsqueeze(0))
            comp_done[slot].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done[slot])
            dst[lo:hi].copy_(slab_out[slot][:u], non_blocking=True)
            out_done[slot].record(s_out)
    for st in (s_in, s_comp, s_out):
        cur.wait_stream(st)
    s_out.synchronize()
    return out


vc_attention_triton = vc_attention_cuda
