"""ExpCast-FP8 on the GPU (interface of the reference's vc_attention/expcast.py).

An E4M3 byte is close to an affine function of log2 of its value, so the
probability byte of a score s against the running row maximum m is written
without an exponential:

    u    = (s - m) * log2(e) + 8          (row maximum lands on 2^8 = 256)
    code = clamp(round_even(8 * u + 56 + beta), 0, 120)

``expcast_codes(..., exact=True)`` evaluates the operation sequence above;
``exact=False`` runs the attention kernels' own device routine (one saturating
FMA per code with the per-row constants folded, rounded by a magic add).
"""

from __future__ import annotations

import torch

from . import _native as N

__all__ = ["LOG2E", "DEFAULT_BETA", "expcast_codes", "expcast_probabilities"]

LOG2E = 1.4426950408889634
DEFAULT_BETA = -0.35


def expcast_codes(s: torch.Tensor, m: torch.Tensor, beta: float = DEFAULT_BETA,
                  exact: bool = True) -> torch.Tensor:
    """(M, N) scores and (M,) running maxima -> (M, N) uint8 E4M3 codes of p * 256."""
    if not s.is_cuda:
        raise RuntimeError("expcast_codes runs on CUDA tensors only")
    s2 = s.detach().to(torch.float32).reshape(-1, s.shape[-1]).contiguous()
    m2 = m.detach().to(torch.float32).reshape(-1).contiguous()
    if m2.numel() != s2.shape[0]:
        raise ValueError("m must hold one maximum per score row")
    out = torch.empty(s2.shape, dtype=torch.uint8, device=s.device)
    lib = N.lib()
    N.check("vcattn_expcast_codes", lib.vcattn_expcast_codes(
        s2.data_ptr(), m2.data_ptr(), s2.shape[0], s2.shape[1], float(beta), 1 if exact else 0,
        out.data_ptr(), torch.cuda.current_stream(s.device).cuda_stream))
    return out.reshape(s.shape)


def expcast_probabilities(s: torch.Tensor, m: torch.Tensor, beta: float = DEFAULT_BETA) -> torch.Tensor:
    """Decoded p * 256 values."""
    from .quant import e4m3_decode
    return e4m3_decode(expcast_codes(s, m, beta))
