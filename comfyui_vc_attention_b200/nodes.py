"""ComfyUI nodes (behaviour and inputs of the reference's nodes.py:34-243).

``VC Attention (MiniMax-H3)`` installs the router with the H3 defaults;
``VC Attention Disable`` restores the original attention.  The patch is
process-global until disabled.
"""

from __future__ import annotations

from .vc_attention.device import detect_profile, resolve_backend
from .vc_attention.h3 import recommended_config
from .vc_attention.patch import VCAttentionConfig, install, kernel_status, uninstall

CATEGORY = "vc_attention"


class VCAttentionMiniMaxH3:
    """Low-bit attention for MiniMax-H3: V-Smooth grouping, FP8/NVFP4 QK^T,
    ExpCast FP8 softmax, FP8 PV with block-mean restoration and fused tau
    block sparsity, on B200 (sm_100a) CUDA kernels."""

    @classmethod
    def INPUT_TYPES(cls):
        h3 = recommended_config(total_steps=8)
        return {
            "required": {
                "model": ("MODEL", {"tooltip": "The diffusion model to patch."}),
                "backend": (["auto", "nvfp4", "fp8", "int4", "reference"],
                            {"default": "auto",
                             "tooltip": "fp8: FP8 QK^T and PV. nvfp4: NVFP4 QK^T with FP8 PV. "
                                        "auto/int4/reference run fp8 on B200."}),
                "enable_vsmooth": ("BOOLEAN", {"default": True,
                                               "tooltip": "V-Smooth: k-means grouping + block demean."}),
                "enable_expcast": ("BOOLEAN", {"default": False,
                                               "tooltip": "ExpCast-FP8: write the probability byte "
                                                          "with one FMA instead of exp2 + cast."}),
                "total_steps": ("INT", {"default": 8, "min": 1, "max": 200,
                                        "tooltip": "Denoising steps; grouping runs on the first 25%."}),
                "block_rows": ("INT", {"default": h3["block_rows"], "min": 16, "max": 256, "step": 16,
                                       "tooltip": "Value rows per quantisation block (64 or 128 on B200)."}),
                "min_tokens": ("INT", {"default": 8192, "min": 512, "max": 1 << 20, "step": 512,
                                       "tooltip": "Skip VC-Attention below this sequence length."}),
                "enable_sparsity": ("BOOLEAN", {"default": True,
                                                "tooltip": "Fused tau block sparsity: KV blocks under "
                                                           "the proxy threshold use their block mean."}),
            },
            "optional": {
                "tau": ("FLOAT", {"default": 1.3, "min": 0.0, "max": 8.0, "step": 0.1,
                                  "tooltip": "Routing threshold in std-devs above the mean proxy."}),
                "sparsity_min_tokens": ("INT", {"default": 8192, "min": 1024, "max": 1 << 20, "step": 512,
                                                "tooltip": "Sparsity is off below this length."}),
                "sink_tokens": ("INT", {"default": 512, "min": 0, "max": 8192, "step": 128,
                                        "tooltip": "Leading tokens always kept exact."}),
                "local_blocks": ("INT", {"default": 1, "min": 0, "max": 8,
                                         "tooltip": "+/-N KV blocks around each query block kept exact."}),
                "group_fraction": ("FLOAT", {"default": 0.25, "min": 0.0, "max": 1.0, "step": 0.05,
                                             "tooltip": "Fraction of steps that run k-means."}),
                "reuse_every": ("INT", {"default": 4, "min": 1, "max": 64,
                                        "tooltip": "Reuse one permutation for this many steps."}),
                "kmeans_iters": ("INT", {"default": 3, "min": 1, "max": 16,
                                         "tooltip": "Lloyd iterations on a cold start."}),
                "modality_aware": ("BOOLEAN", {"default": False,
                                               "tooltip": "Use the H3 modality tag as the primary sort key."}),
                "override_priority": (["front", "defer"],
                                      {"default": "front",
                                       "tooltip": "front: chain in front of another attention override; "
                                                  "defer: stay out when one is installed."}),
            },
        }

    RETURN_TYPES = ("MODEL",)
    RETURN_NAMES = ("model",)
    FUNCTION = "apply"
    CATEGORY = CATEGORY
    DESCRIPTION = ("VC-Attention adapted to MiniMax-H3 on B200: V-Smooth value grouping plus low-bit "
                   "QK/PV with fused tau block sparsity. Training-free; no checkpoint changes.")

    def apply(self, model, backend="auto", enable_vsmooth=True, enable_expcast=False, total_steps=8,
              block_rows=128, min_tokens=8192, enable_sparsity=True, tau=1.3, sparsity_min_tokens=8192,
              sink_tokens=512, local_blocks=1, group_fraction=0.25, reuse_every=4, kmeans_iters=3,
              modality_aware=False, override_priority="defer"):
        profile = detect_profile()
        resolved = resolve_backend(backend, profile)
        cfg = VCAttentionConfig(
            enabled=True, backend=backend, enable_vsmooth=enable_vsmooth,
            enable_expcast=bool(enable_expcast and resolved == "fp8"),
            block_rows=int(block_rows), min_tokens=int(min_tokens),
            enable_sparsity=bool(enable_sparsity), tau=float(tau),
            sparsity_min_tokens=int(sparsity_min_tokens), sink_tokens=int(sink_tokens),
            local_blocks=int(local_blocks), kmeans_iters=int(kmeans_iters),
            modality_aware=bool(modality_aware), group_fraction=float(group_fraction),
            reuse_every=int(reuse_every), total_steps_hint=int(total_steps),
            override_priority=str(override_priority))
        runtime = install(cfg, model=model)
        runtime.reset()
        status = kernel_status()
        print(f"[VC-Attention] {profile.describe()}\n"
              f"[VC-Attention] backend={resolved} vsmooth={cfg.enable_vsmooth} "
              f"expcast={cfg.enable_expcast} block_rows={cfg.block_rows} grouping on steps "
              f"0..{max(0, runtime.schedule.group_steps(total_steps) - 1)} of {total_steps}\n"
              f"[VC-Attention] sparsity={cfg.enable_sparsity} tau={cfg.tau} (on from "
              f"{cfg.sparsity_min_tokens} tokens; sink {cfg.sink_tokens}, local +/-{cfg.local_blocks} blocks)\n"
              f"[VC-Attention] {status}\n[VC-Attention] {profile.expectation_note()}")
        if "inactive" in status:
            print("[VC-Attention] Nothing will be accelerated; sampling runs at native speed.")
        return (model,)


class VCAttentionDisable:
    """Restore the original attention implementation."""

    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"model": ("MODEL",)}}

    RETURN_TYPES = ("MODEL",)
    RETURN_NAMES = ("model",)
    FUNCTION = "apply"
    CATEGORY = CATEGORY

    def apply(self, model):
        uninstall()
        print("[VC-Attention] restored the original attention")
        return (model,)


NODE_CLASS_MAPPINGS = {
    "VCAttentionMiniMaxH3": VCAttentionMiniMaxH3,
    "VCAttentionDisable": VCAttentionDisable,
}

NODE_DISPLAY_NAME_MAPPINGS = {
    "VCAttentionMiniMaxH3": "VC Attention (MiniMax-H3)",
    "VCAttentionDisable": "VC Attention Disable",
}
