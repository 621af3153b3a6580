"""ComfyUI custom node package: VC-Attention for MiniMax-H3 on B200 (sm_100a).

Copy (or symlink) this folder into ``ComfyUI/custom_nodes/`` after building
the CUDA library with ``python -m comfyui_vc_attention_b200.build``.
"""

from .nodes import (  # noqa: F401
    NODE_CLASS_MAPPINGS,
    NODE_DISPLAY_NAME_MAPPINGS,
    VCAttentionDisable,
    VCAttentionMiniMaxH3,
)

__all__ = ["NODE_CLASS_MAPPINGS", "NODE_DISPLAY_NAME_MAPPINGS", "VCAttentionMiniMaxH3",
           "VCAttentionDisable"]
