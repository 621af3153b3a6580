"""Device profile and backend names (the reference's vc_attention/device.py
interface, narrowed to what this build runs).

This build has exactly one implementation: the sm_100a kernels of
libvcattn.so.  ``detect_profile`` reports the GPU; ``resolve_backend`` maps
the node's backend choices onto the two variants that kernel offers:

  * "fp8"   : FP8 E4M3 QK^T and PV (auto, fp8, int4, reference);
  * "nvfp4" : NVFP4 QK^T with FP8 PV.

"int4" maps to "fp8" because Blackwell datacenter parts have no INT4 MMA (the
reference does the same for sm >= 10.0).  "reference" maps to "fp8": the
CUDA prepare reproduces the portable reference's quantisation byte for byte,
so there is no separate slow path to select.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch

__all__ = ["DeviceProfile", "detect_profile", "resolve_backend", "is_supported"]


@dataclass(frozen=True)
class DeviceProfile:
    name: str
    sm: Tuple[int, int]
    has_fp8: bool
    has_fp4: bool
    softmax_bound: bool
    recommended_bits: int
    recommended_expcast: bool

    def describe(self) -> str:
        return (f"{self.name} (sm_{self.sm[0]}{self.sm[1]}): fp8={self.has_fp8}, fp4={self.has_fp4}, "
                f"recommended={self.recommended_bits}-bit, expcast={self.recommended_expcast}")

    def expectation_note(self) -> str:
        if is_supported(self):
            return ("B200 (sm_100a): fused tcgen05/TMA FP8 VC-Attention kernels; "
                    "NVFP4 QK^T optional.")
        return "not an sm_100 GPU: the node defers to native attention (inactive)."


def is_supported(profile: "DeviceProfile") -> bool:
    return profile.sm[0] == 10


def detect_profile(device: Optional[torch.device] = None) -> DeviceProfile:
    if device is None:
        device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    if device.type != "cuda" or not torch.cuda.is_available():
        return DeviceProfile("CPU", (0, 0), False, False, False, 8, False)
    major, minor = torch.cuda.get_device_capability(device)
    name = torch.cuda.get_device_name(device)
    dc = major == 10
    # Datacenter Blackwell doubled tensor throughput without doubling the
    # exponential unit, so the 8-bit path is softmax-bound and ExpCast pays.
    return DeviceProfile(name, (major, minor), major >= 9 or (major, minor) == (8, 9), dc or major == 12,
                         dc, 8, dc)


def resolve_backend(requested: str, profile: Optional[DeviceProfile] = None) -> str:
    """auto | fp8 | nvfp4 | fp4 | int4 | reference  ->  fp8 | nvfp4."""
    req = (requested or "auto").lower()
    if req in ("nvfp4", "fp4"):
        return "nvfp4"
    return "fp8"
