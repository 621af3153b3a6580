"""Query tiles split over their KV tiles (vcattn_attn_fp8_split).

A split query tile runs as several CTAs, each over a contiguous range of KV
tiles with its own running max, and a combine kernel merges the partials.
The reference has no such split (its grid is one program per query block,
triton_attn.py:804); the oracle restates it as attention_codes with
``kv_piece_tiles`` (each piece's P bytes rounded relative to its own max,
pieces combined with exp2 weights), so split tiles are checked against that
arithmetic and unsplit tiles stay bit-identical to the unsplit kernel.
"""

import numpy as np
import pytest
import torch

from oracle import vc_oracle as O
from oracle.inputs import make_qkv

pytestmark = pytest.mark.gpu

REL_L2_CODES = 1e-3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from comfyui_vc_attention_b200.vc_attention import _native as N
    N.lib()
    return torch.device("cuda:0")


def _run(q, k, v, perm, br, dev, kv_split, expcast=False):
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                          attention_status, prepare)
    t = [torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(torch.bfloat16) for a in (q, k, v)]
    p = prepare(*t, torch.from_numpy(perm).to(dev), block_rows=br, want_v=True)
    b, h, n, d = q.shape
    out = torch.empty((b, h, n, d), dtype=torch.float32, device=dev)
    attention_prepared(p, n, out, d ** -0.5, TritonConfig(block_n=br, enable_expcast=expcast), kernel="tc",
                       kv_split=kv_split)
    torch.cuda.synchronize()
    assert attention_status() == (0, 0, 0)
    return out.cpu().numpy().reshape(b * h, n, d)


def _pieces(tiles, want):
    want = min(want, tiles, 32)
    tp = -(-tiles // want)
    return tp, -(-tiles // tp)


@pytest.mark.parametrize("n,br,d,k,expcast", [(1024, 128, 128, 2, True), (1000, 64, 128, 3, False),
                                              (700, 128, 64, 4, True), (2048, 64, 64, 5, True),
                                              (1536, 128, 128, 32, False)])
def test_forced_split_matches_oracle(dev, n, br, d, k, expcast):
    """Every query tile in k pieces: the output equals the oracle of the split
    arithmetic, and stays as close to fp32 SDPA as the unsplit kernel."""
    h = 2
    q, k_, v = make_qkv(1, h, n, d, seed=n + k)
    perm = np.stack([np.random.default_rng(90 + i).permutation(n) for i in range(h)]).astype(np.int32)
    got = _run(q, k_, v, perm, br, dev, k, expcast)
    tiles = -(-n // br)
    tp, pieces = _pieces(tiles, k)
    assert pieces >= 2
    qg, kg, vg = (a.reshape(h, n, d) for a in (q, k_, v))
    prep = O.prepare(qg, kg, vg, perm, block_rows=br)
    ref = O.attention_codes(prep, n, br, 64, d ** -0.5, expcast=expcast, kv_piece_tiles=tp)
    assert O.rel_l2(got, ref) <= REL_L2_CODES
    whole = _run(q, k_, v, perm, br, dev, 1, expcast)
    sd = O.sdpa_f32(qg, kg, vg)
    assert abs(O.psnr(got, sd) - O.psnr(whole, sd)) <= 0.3


def test_auto_split_of_the_last_partial_wave(dev):
    """More CTAs than SMs with a short last wave: only that wave's query tiles
    are split (pieces chosen from the SM count); every other tile is
    bit-identical to the unsplit kernel, the split ones match the oracle."""
    from comfyui_vc_attention_b200.vc_attention import _native as N
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    h, d, br = 2, 128, 128
    qt = nsm // 2 + 1                       # query tiles per head: 2 * qt = nsm + 2 CTAs
    n = qt * 128
    ctas = h * qt
    r = ctas % nsm
    assert ctas > nsm and 0 < r <= nsm // 2
    tiles = -(-n // br)
    tp, pieces = _pieces(tiles, nsm // r)
    lib = N.lib()
    assert lib.vcattn_attn_split_workspace_bytes(1, h, n, n, d, br, 0) == r * pieces * 128 * (d + 2) * 4
    q, k, v = make_qkv(1, h, n, d, seed=5)
    perm = np.stack([np.random.default_rng(7 + i).permutation(n) for i in range(h)]).astype(np.int32)
    auto = _run(q, k, v, perm, br, dev, 0, True)
    whole = _run(q, k, v, perm, br, dev, 1, True)
    split_rows = slice(n - r * 128, n)          # the last r query tiles of the last head
    assert np.array_equal(auto[0], whole[0])
    assert np.array_equal(auto[1, : n - r * 128], whole[1, : n - r * 128])
    assert not np.array_equal(auto[1, split_rows], whole[1, split_rows])
    qg, kg, vg = (a.reshape(h, n, d) for a in (q, k, v))
    prep = O.prepare(qg, kg, vg, perm, block_rows=br)
    blocks = list(range((n - r * 128) // 64, n // 64))
    head1 = {key: (val[1:2] if isinstance(val, np.ndarray) else val) for key, val in prep.items()}
    ref = O.attention_codes(head1, n, br, 64, d ** -0.5, expcast=True, row_blocks=blocks, kv_piece_tiles=tp)
    assert O.rel_l2(auto[1, split_rows], ref[0, split_rows]) <= REL_L2_CODES
