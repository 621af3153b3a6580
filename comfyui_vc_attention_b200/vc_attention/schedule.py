"""Grouping schedule, step counter and permutation cache.

Host bookkeeping around the grouping kernel (behaviour of the reference's
vc_attention/schedule.py:27-115).  k-means runs on the first
``group_fraction`` of the denoising steps and its permutation is recomputed
every ``reuse_every`` steps; in between the cached permutation (and the
centroids that produced it, for a warm start) is reused.  With the deployed
8-step MiniMax-H3 schedule that is ceil(8 * 0.25) = 2 grouping steps inside
one 4-step window: one k-means pass at step 0, reused at step 1.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Optional, Tuple

__all__ = ["GroupSchedule", "StepTracker", "PermutationCache", "TauSchedule"]


@dataclass
class GroupSchedule:
    group_fraction: float = 0.25
    reuse_every: int = 4
    total_steps_hint: int = 8
    min_tokens: int = 8192

    def group_steps(self, total_steps: Optional[int] = None) -> int:
        """Number of leading steps that group: max(1, ceil(round(total * fraction)))."""
        total = total_steps or self.total_steps_hint
        n = round(total * self.group_fraction)
        return max(1, int(-(-n // 1)))

    def should_group(self, step_index: int, total_steps: Optional[int] = None) -> bool:
        return step_index < self.group_steps(total_steps)

    def should_recompute(self, step_index: int) -> bool:
        return step_index % max(1, self.reuse_every) == 0

    def window_index(self, step_index: int) -> int:
        return step_index // max(1, self.reuse_every)


@dataclass
class StepTracker:
    """Counts denoiser forward calls; one call is one denoising step (CFG is a
    batch duplication inside the call, not a second call)."""

    total_steps_hint: int = 8
    index: int = -1
    total_steps: Optional[int] = None
    _installed: bool = field(default=False, repr=False)

    def reset(self) -> None:
        self.index = -1
        self.total_steps = None

    def begin_step(self) -> int:
        self.index += 1
        return self.index

    def observe_total(self, total: int) -> None:
        if total and total > 0:
            self.total_steps = int(total)

    @property
    def current(self) -> int:
        return self.index if self.index > 0 else 0


class PermutationCache:
    """FIFO cache of (permutation, centroids) keyed by (window, tokens, heads).

    The tensors stay on the device: one entry is G * N int32 (about 16 MB for
    56 heads x 73.5K tokens) plus the bf16 centroids.
    """

    def __init__(self, max_entries: int = 8):
        self.max_entries = max_entries
        self._store: "OrderedDict[Tuple[int, int, int], tuple]" = OrderedDict()
        self.hits = 0
        self.misses = 0

    @staticmethod
    def key(bucket: int, n_tokens: int, n_heads: int) -> Tuple[int, int, int]:
        return (bucket, n_tokens, n_heads)

    def get(self, bucket: int, n_tokens: int, n_heads: int):
        item = self._store.get(self.key(bucket, n_tokens, n_heads))
        if item is None:
            self.misses += 1
        else:
            self.hits += 1
        return item

    def put(self, bucket: int, n_tokens: int, n_heads: int, perm, centroids) -> None:
        k = self.key(bucket, n_tokens, n_heads)
        if k not in self._store and len(self._store) >= self.max_entries:
            self._store.popitem(last=False)
        self._store[k] = (perm, centroids)

    def clear(self) -> None:
        self._store.clear()
        self.hits = 0
        self.misses = 0

    def __len__(self) -> int:
        return len(self._store)


@dataclass
class TauSchedule:
    """The sparsity threshold across denoising steps: the schedule Sol-Attn
    uses, which the reference plans but does not build
    (PLAN_sparse_fusion.md:115-118): the first ``dense_steps`` steps run
    dense, then tau falls linearly from ``tau_start`` at the first sparse step
    to ``tau_end`` at the last step (a larger tau keeps fewer blocks)."""

    tau_start: float = 1.0
    tau_end: float = 2.0
    dense_steps: int = 0

    def tau(self, step_index: int, total_steps: Optional[int]) -> Optional[float]:
        """tau for this step, or None for a dense step."""
        if step_index < self.dense_steps:
            return None
        total = max(total_steps or 0, step_index + 1)
        span = total - 1 - self.dense_steps
        if span <= 0:
            return float(self.tau_end)
        t = min(1.0, (step_index - self.dense_steps) / span)
        return float(self.tau_start + (self.tau_end - self.tau_start) * t)

