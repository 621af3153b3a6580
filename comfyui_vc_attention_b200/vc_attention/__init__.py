"""VC-Attention for MiniMax-H3 on B200: V-Smooth (k-means value grouping,
block demean, mean restored from the softmax row sum) + ExpCast-FP8, with
fused tau block sparsity, as sm_100a CUDA kernels behind the reference
package's Python interface.

Quick start::

    from comfyui_vc_attention_b200.vc_attention.patch import install, VCAttentionConfig
    install(VCAttentionConfig(backend="auto"))
"""

from .device import DeviceProfile, detect_profile, resolve_backend  # noqa: F401
from .grouping import GroupingConfig, build_permutation  # noqa: F401
from .h3 import H3, TAG, H3Profile, estimate_tokens, recommended_config  # noqa: F401
from .kernels.cuda_attn import vc_attention_cuda, vc_attention_host, vc_attention_triton  # noqa: F401
from .schedule import GroupSchedule, PermutationCache, StepTracker  # noqa: F401

__all__ = [
    "DeviceProfile", "detect_profile", "resolve_backend",
    "GroupingConfig", "build_permutation",
    "H3", "H3Profile", "TAG", "estimate_tokens", "recommended_config",
    "GroupSchedule", "PermutationCache", "StepTracker",
    "vc_attention_triton", "vc_attention_cuda", "vc_attention_host",
]
