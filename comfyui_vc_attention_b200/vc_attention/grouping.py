"""V-Smooth grouping on the GPU: k-means over value tokens and the stable
label sort that yields the K/V permutation.

Interface of the reference's vc_attention/grouping.py:40-191
(``GroupingConfig``, ``GroupingResult``, ``kmeans``, ``build_permutation``,
``apply_permutation``); the work runs in ``vcattn_kmeans`` (libvcattn.so):
seeding, Lloyd iterations (assign + update) and the final sort are all device
kernels, with no host synchronisation.

Permuting K and V together leaves softmax(QK^T)V unchanged; it only groups
similar value rows into the same quantisation block so that the block-mean
subtraction leaves a small residual.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import _native as N

__all__ = ["GroupingConfig", "GroupingResult", "kmeans", "build_permutation", "apply_permutation",
           "num_clusters"]


@dataclass
class GroupingConfig:
    block_rows: int = 128
    iters: int = 3
    warm_iters: int = 2
    init_samples_per_centroid: int = 4
    max_clusters: int = 1024
    chunk: int = 8192              # kept for interface parity; the kernel is not chunked
    modality_aware: bool = False
    scope: str = "per_head"
    dtype: torch.dtype = torch.bfloat16


@dataclass
class GroupingResult:
    perm: torch.Tensor                      # (G, N) int32
    centroids: Optional[torch.Tensor]       # (G, k, D) bf16
    k: int
    labels: Optional[torch.Tensor] = None   # (G, N) int32


def num_clusters(n: int, cfg: GroupingConfig) -> int:
    """min(ceil(n / block_rows), max_clusters, n), at least 1."""
    k = max(1, (n + cfg.block_rows - 1) // cfg.block_rows)
    return min(k, cfg.max_clusters, n)


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return N.DTYPE_BF16
    if t.dtype == torch.float16:
        return N.DTYPE_F16
    if t.dtype == torch.float32:
        return N.DTYPE_F32
    raise TypeError(f"unsupported dtype {t.dtype}")


def as_bhnd(x: torch.Tensor) -> Tuple[N.BHND, int, int, int, int]:
    """A (B,H,N,D) or (G,N,D) tensor as a vcattn_bhnd view without copying
    when its last dim is contiguous and its strides are 16-byte multiples."""
    if x.dim() == 3:
        x = x.unsqueeze(0)
    if x.dim() != 4:
        raise ValueError("expected a (B, H, N, D) or (G, N, D) tensor")
    esz = x.element_size()
    ok = (x.stride(-1) == 1 and x.data_ptr() % 16 == 0
          and all((s * esz) % 16 == 0 for s in x.stride()[:3]))
    if not ok:
        x = x.contiguous()
    b, h, n, d = x.shape
    v = N.BHND(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2))
    v._keep = x   # the view must outlive the call
    return v, b, h, n, d


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def kmeans(v: torch.Tensor, k: int, cfg: GroupingConfig,
           centroids: Optional[torch.Tensor] = None,
           key_offset: Optional[torch.Tensor] = None, nkeys: int = 0):
    """Batched k-means over (G, N, D) [or (B, H, N, D)] value rows on the GPU.

    Returns (labels (G,N) int32, centroids (G,k,D) bf16, perm (G,N) int32).
    ``perm`` is the stable argsort of label + key_offset.
    """
    if not v.is_cuda:
        raise RuntimeError("kmeans runs on CUDA tensors only (no CPU implementation)")
    lib = N.lib()
    view, b, h, n, d = as_bhnd(v)
    g = b * h
    iters = cfg.iters if centroids is None else cfg.warm_iters
    nk = nkeys if key_offset is not None else k
    ws_bytes = lib.vcattn_kmeans_workspace_bytes(g, n, d, k, nk)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=v.device)
    cent = torch.empty((g, k, d), dtype=torch.bfloat16, device=v.device)
    perm = torch.empty((g, n), dtype=torch.int32, device=v.device)
    labels = torch.empty((g, n), dtype=torch.int32, device=v.device)
    warm = None
    if centroids is not None:
        warm = centroids.to(device=v.device, dtype=torch.bfloat16).reshape(g, k, d).contiguous()
    koff = None
    if key_offset is not None:
        koff = key_offset.to(device=v.device, dtype=torch.int32).contiguous()
    N.check("vcattn_kmeans", lib.vcattn_kmeans(
        view, _dtype_code(view._keep), b, h, n, d, k, iters,
        warm.data_ptr() if warm is not None else None,
        koff.data_ptr() if koff is not None else None, nk,
        cent.data_ptr(), perm.data_ptr(), labels.data_ptr(),
        ws.data_ptr(), ws_bytes, _stream(v)))
    return labels, cent, perm


def build_permutation(v: torch.Tensor, cfg: GroupingConfig, tags: Optional[torch.Tensor] = None,
                      centroids: Optional[torch.Tensor] = None,
                      valid_len: Optional[int] = None,
                      pad_mask: Optional[torch.Tensor] = None) -> GroupingResult:
    """V-Smooth permutation of one value tensor (G, N, D).

    ``tags`` (N,) modality tags are a secondary key when ``cfg.modality_aware``
    (pad tag -1 sorts last); rows >= ``valid_len`` are pushed to the tail.
    ``pad_mask`` (N,) bool (this build; may live on the device) generalises
    ``valid_len`` to any set of padding rows: they get the same pad key
    (grouping.py:181-183), so they sort to the tail in their original order.
    """
    if v.dim() == 4:
        v = v.reshape(-1, v.shape[-2], v.shape[-1]) if not v.is_contiguous() else v.view(-1, v.shape[-2], v.shape[-1])
    g, n, d = v.shape
    k = num_clusters(n, cfg)
    if pad_mask is not None:
        if valid_len is not None:
            raise ValueError("give valid_len or pad_mask, not both")
        if pad_mask.shape != (n,):
            raise ValueError(f"pad_mask must be ({n},)")
        off = pad_mask.to(device=v.device, dtype=torch.int32) * (16 * (k + 1))
        nkeys = 16 * (k + 1) + k
        if cfg.modality_aware and tags is not None:
            tag = tags.detach().to(v.device, torch.int64).clamp(min=-1)
            tag = torch.where(tag < 0, torch.full_like(tag, 8), tag)
            off = off + (tag * (k + 1)).to(torch.int32)
            nkeys += 8 * (k + 1)
        labels, cent, perm = kmeans(v, k, cfg, centroids, off, nkeys)
        return GroupingResult(perm=perm, centroids=cent, k=k, labels=labels)
    key_offset = None
    nkeys = k
    if (cfg.modality_aware and tags is not None) or (valid_len is not None and valid_len < n):
        off = torch.zeros(n, dtype=torch.int64)
        nkeys = k
        if cfg.modality_aware and tags is not None:
            tag = tags.detach().to("cpu", torch.int64).clamp(min=-1)
            tag = torch.where(tag < 0, torch.full_like(tag, 8), tag)
            off = off + tag * (k + 1)
            nkeys = max(nkeys, int(off.max()) + k)
        if valid_len is not None and valid_len < n:
            is_pad = (torch.arange(n) >= valid_len).to(torch.int64)
            off = off + is_pad * (16 * (k + 1))
            nkeys = max(nkeys, int(off.max()) + k)
        key_offset = off.to(torch.int32)
    labels, cent, perm = kmeans(v, k, cfg, centroids, key_offset, nkeys)
    return GroupingResult(perm=perm, centroids=cent, k=k, labels=labels)


def apply_permutation(x: torch.Tensor, perm: torch.Tensor) -> torch.Tensor:
    """Gather ``x`` (..., N, D) along the token axis with ``perm`` (G, N)."""
    return x.gather(-2, perm.to(torch.int64).unsqueeze(-1).expand_as(x))
