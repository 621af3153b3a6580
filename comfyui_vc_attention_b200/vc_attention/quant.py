"""E4M3 / E2M1 codecs on the GPU (interface of the reference's
vc_attention/quant.py:56-169 for the formats this path uses).

Encoders run the same device conversions the prepare and attention kernels
use (``cvt.rn.satfinite`` E4M3 / E2M1, with +-0 canonicalised to code 0 as the
reference encoder does); decoders are table lookups.
"""

from __future__ import annotations

import torch

from . import _native as N

__all__ = ["E4M3_MAX", "E4M3_MIN_NORMAL", "FP4_VALUES", "e4m3_encode", "e4m3_decode",
           "fp4_encode", "fp4_decode"]

E4M3_MAX = 448.0
E4M3_MIN_NORMAL = 2.0 ** -6
FP4_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)

_E4M3_TABLE = {}


def _e4m3_table(device) -> torch.Tensor:
    key = str(device)
    if key not in _E4M3_TABLE:
        c = torch.arange(256, dtype=torch.int64)
        sign = 1.0 - 2.0 * ((c >> 7) & 1).to(torch.float32)
        e = (c >> 3) & 0xF
        m = (c & 7).to(torch.float32)
        val = torch.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * torch.pow(2.0, (e - 7).to(torch.float32)))
        val = torch.where((e == 15) & ((c & 7) == 7), torch.full_like(val, E4M3_MAX), val)
        _E4M3_TABLE[key] = (val * sign).to(device)
    return _E4M3_TABLE[key]


def _run_encoder(fn: str, x: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda:
        raise RuntimeError(f"{fn} runs on CUDA tensors only")
    xf = x.detach().to(torch.float32).contiguous()
    out = torch.empty(xf.shape, dtype=torch.uint8, device=x.device)
    lib = N.lib()
    N.check(fn, getattr(lib, fn)(xf.data_ptr(), xf.numel(), out.data_ptr(),
                                 torch.cuda.current_stream(x.device).cuda_stream))
    return out


def e4m3_encode(x: torch.Tensor) -> torch.Tensor:
    """RNE, saturating E4M3 codes (uint8)."""
    return _run_encoder("vcattn_e4m3_encode", x)


def e4m3_decode(code: torch.Tensor) -> torch.Tensor:
    """E4M3 codes -> float32 (0x7F / 0xFF decode to +-448)."""
    return _e4m3_table(code.device)[code.to(torch.int64) & 0xFF]


def fp4_encode(x: torch.Tensor) -> torch.Tensor:
    """RNE E2M1 codes 0..15 (bit 3 = sign), one per byte."""
    return _run_encoder("vcattn_fp4_encode", x)


def fp4_decode(code: torch.Tensor) -> torch.Tensor:
    table = torch.tensor(FP4_VALUES, dtype=torch.float32, device=code.device)
    c = code.to(torch.int64) & 0xF
    return table[c & 7] * (1.0 - 2.0 * ((c >> 3) & 1).to(torch.float32))
