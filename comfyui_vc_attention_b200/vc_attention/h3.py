"""MiniMax-H3 facts the node defaults are derived from (behaviour of the
reference's vc_attention/h3.py:46-155).

H3 runs 50 DiT blocks of full self-attention over one packed sequence of text,
video and audio rows: 56 heads x head_dim 128, no GQA.  The V-Smooth value
block is 128 rows (= head_dim), and the deployed schedule is an 8-step
distilled LoRA.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Tuple

__all__ = ["H3Profile", "H3", "TAG", "estimate_tokens", "recommended_config"]


@dataclass(frozen=True)
class H3Profile:
    num_attention_heads: int = 56
    attention_head_dim: int = 128
    hidden_size: int = 5376
    num_layers: int = 50
    num_refiner_layers: int = 2
    ffn_dim: int = 14336
    in_channels: int = 24
    audio_in_channels: int = 32
    patch_size: Tuple[int, int, int] = (1, 2, 2)
    text_dim: int = 5120
    freq_dim: int = 256
    time_embed_hidden_dim: int = 5376
    time_embed_dim: int = 2688
    rope_freq_dim: int = 16
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    qk_norm_eps: float = 1e-5
    final_norm_eps: float = 1e-5
    vae_spatial: int = 16
    vae_temporal: int = 4
    vae_channels: int = 24
    audio_latent_rate_hz: float = 40.0
    video_fps: float = 24.0

    @property
    def qkv_dim(self) -> int:
        return self.num_attention_heads * self.attention_head_dim

    @property
    def rope_dims(self) -> int:
        """MM-RoPE rotates 2 * 3 * rope_freq_dim channels of each head."""
        return 6 * self.rope_freq_dim

    @property
    def unrotated_dims(self) -> int:
        return self.attention_head_dim - self.rope_dims


H3 = H3Profile()


class TAG:
    """Modality tag of each row of the packed sequence."""
    VIDEO = 0
    TEXT = 1
    AUDIO = 2
    PAD = -1


def estimate_tokens(frames: int, height: int, width: int, audio_seconds: float = 0.0,
                    text_tokens: int = 1024, conditioning_rows: int = 0,
                    profile: H3Profile = H3) -> Dict[str, object]:
    """Row counts of one clip's packed sequence: the VAE divides time by 4
    (causal: ceil) and space by 16, the 1x2x2 patchify space by 2 more."""
    lt = -(-frames // profile.vae_temporal)
    lh = height // (profile.vae_spatial * profile.patch_size[1])
    lw = width // (profile.vae_spatial * profile.patch_size[2])
    video = lt * lh * lw
    audio = int(round(audio_seconds * profile.audio_latent_rate_hz)) if audio_seconds else 0
    return {
        "video": video,
        "audio": audio,
        "text": text_tokens,
        "conditioning": conditioning_rows,
        "total": video + audio + text_tokens + conditioning_rows,
        "latent_grid": (lt, lh, lw),
    }


def recommended_config(profile: H3Profile = H3, total_steps: int = 8) -> Dict[str, object]:
    """Node defaults for H3: group on the first 25% of steps, reuse for 4."""
    group_steps = max(1, -(-int(total_steps * 0.25) // 1))
    return {
        "block_rows": 128,
        "heads": profile.num_attention_heads,
        "head_dim": profile.attention_head_dim,
        "group_fraction": 0.25,
        "group_steps": group_steps,
        "reuse_every": 4,
        "modality_aware": True,
        "min_tokens": 8192,
    }
