"""The output accumulated in value-block-scale units (CPU).

A kernel whose P.V tensor-core MMA adds into the output accumulator itself
has to keep that accumulator in units of the current value block's per-channel
scale, rescaling it by alpha * vs_{j-1} / vs_j between blocks.
``oracle.attention_codes_units`` restates that order of operations; these
tests check it against ``attention_codes`` (the order the shipped kernels use),
including value blocks whose channel scale sits at the amax clamp, where the
unit needs its own floor to keep the accumulator finite.
"""

import numpy as np
import pytest

from oracle import vc_oracle as O


def _inputs(seed, degenerate):
    rng = np.random.default_rng(seed)
    g, n, d = 2, 1000, 128
    q = rng.standard_normal((g, n, d)).astype(np.float32)
    k = (rng.standard_normal((g, n, d)) + rng.normal(0, 2, (g, 1, d))).astype(np.float32)
    centres = rng.standard_normal((g, 64, d))
    v = (centres[:, rng.integers(0, 64, n)] + 0.3 * rng.standard_normal((g, n, d))).astype(np.float32)
    if degenerate:
        v[:, 128:256, 5] = 3.0                 # one block's channel is constant: residual 0
        v[:, 256:384, :] = v[:, 256:257, :]    # one block of identical rows
        perm = np.tile(np.arange(n, dtype=np.int32), (g, 1))   # keep the blocks intact
    else:
        perm = np.stack([rng.permutation(n) for _ in range(g)]).astype(np.int32)
    q, k, v = (O.bf16_round(x) for x in (q, k, v))
    return O.prepare(q, k, v, perm, block_rows=128), n, d


@pytest.mark.parametrize("degenerate", [False, True])
@pytest.mark.parametrize("expcast", [False, True])
def test_block_scale_units_match_the_kernel_order(degenerate, expcast):
    prep, n, d = _inputs(5 + int(degenerate), degenerate)
    if degenerate:
        assert float(prep["v_scale"].min()) < 1e-30      # a scale at the amax clamp
    ref = O.attention_codes(prep, n, 128, 128, d ** -0.5, expcast=expcast)
    got = O.attention_codes_units(prep, n, 128, 128, d ** -0.5, expcast=expcast)
    assert np.isfinite(got).all()
    assert O.rel_l2(got, ref) <= 1e-5


def test_unit_floor_keeps_large_values_finite():
    """With |V| in the thousands, a block scale at the amax clamp would push
    the accumulator past float32 (acc * 448 / 2.2e-33); the per-channel unit
    floor keeps it finite and the result still matches."""
    rng = np.random.default_rng(9)
    g, n, d = 1, 512, 128
    q = O.bf16_round(rng.standard_normal((g, n, d)).astype(np.float32))
    k = O.bf16_round(rng.standard_normal((g, n, d)).astype(np.float32))
    v = O.bf16_round((rng.standard_normal((g, n, d)) * 4096).astype(np.float32))
    v[:, 128:256, 7] = 3000.0
    prep = O.prepare(q, k, v, np.arange(n, dtype=np.int32)[None], block_rows=128)
    assert float(prep["v_scale"].min()) < 1e-30
    ref = O.attention_codes(prep, n, 128, 128, d ** -0.5, expcast=True)
    got = O.attention_codes_units(prep, n, 128, 128, d ** -0.5, expcast=True)
    assert np.isfinite(got).all() and O.rel_l2(got, ref) <= 1e-5
    with np.errstate(over="ignore", invalid="ignore"):
        unfloored = O.attention_codes_units(prep, n, 128, 128, d ** -0.5, expcast=True, floor_exp=-1000)
    assert not np.isfinite(unfloored).all()
