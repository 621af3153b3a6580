"""Key-padding (masked) attention on the GPU.

The reference defines key padding through ``valid_len``: build_permutation
gives padding rows a pad key so they sort to the tail of the V-Smooth
permutation (grouping.py:176-183), and vc_attention_reference masks the keys
at permuted positions >= valid_len (reference.py:162-294).  Its Triton path
does not run masked attention (README.md:514-515); here the dense tcgen05
kernel stops at a per-batch key count (vcattn_attn_fp8_masked) and the router
accepts key-padding masks.  tests/golden/masked.npz holds the reference's own
permutation and outputs.
"""

import os

import numpy as np
import pytest
import torch

from oracle import vc_oracle as O
from oracle.inputs import digest, make_qkv

pytestmark = pytest.mark.gpu

REL_L2_REF = 2e-3
REL_L2_CODES = 1e-3
PSNR_DB = 0.3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from comfyui_vc_attention_b200.vc_attention import _native as N
    N.lib()
    return torch.device("cuda:0")


def _bf16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(torch.bfloat16)


def _masked_gpu(q, k, v, perm, kv_len, dev, expcast=False):
    """The masked kernel on prepared operands, fp32 output."""
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                          attention_status, prepare_for)
    qt, kt, vt = _bf16(q, dev), _bf16(k, dev), _bf16(v, dev)
    cfg = TritonConfig(block_n=128, enable_expcast=expcast)
    p = prepare_for(qt, kt, vt, torch.from_numpy(np.ascontiguousarray(perm)).to(dev), cfg)
    out = torch.empty(qt.shape, dtype=torch.float32, device=dev)
    attention_prepared(p, qt.shape[2], out, qt.shape[3] ** -0.5, cfg,
                       kv_len=torch.tensor(kv_len, dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert attention_status() == (0, 0, 0)
    return out.cpu().numpy()


@pytest.mark.parametrize("expcast", [False, True])
def test_masked_attention_matches_reference(dev, expcast):
    from comfyui_vc_attention_b200.vc_attention.grouping import GroupingConfig, build_permutation
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "masked.npz"))
    h, n, d = 2, 1024, 128
    q, k, v = make_qkv(1, h, n, d, seed=9)
    assert digest(q, k, v) == str(g["digest"])
    vl = int(g["valid_len"])
    # the GPU permutation with the reference's pad key equals the reference's
    res = build_permutation(_bf16(v, dev).reshape(h, n, d), GroupingConfig(block_rows=128, iters=3), valid_len=vl)
    np.testing.assert_array_equal(res.perm.cpu().numpy(), g["perm"])
    keep = torch.zeros(n, dtype=torch.bool)
    keep[:vl] = True
    pad = (~keep).to(dev)
    res2 = build_permutation(_bf16(v, dev).reshape(h, n, d), GroupingConfig(block_rows=128, iters=3), pad_mask=pad)
    np.testing.assert_array_equal(res2.perm.cpu().numpy(), g["perm"])
    got = _masked_gpu(q, k, v, g["perm"], [vl], dev, expcast=expcast).reshape(h, n, d)
    name = "expcast" if expcast else "plain"
    ref = g[f"out_{name}"].reshape(h, n, d)
    assert O.rel_l2(got, ref) <= REL_L2_REF
    qg, kg, vg = (a.reshape(h, n, d) for a in (q, k, v))
    prep = O.prepare(qg, kg, vg, g["perm"], block_rows=128)
    codes = O.attention_codes(prep, n, 128, 128, d ** -0.5, expcast=expcast, kv_len=[vl, vl])
    assert O.rel_l2(got, codes) <= REL_L2_CODES
    sd = torch.nn.functional.scaled_dot_product_attention(
        *(torch.from_numpy(a.reshape(1, h, n, d)) for a in (q, k, v)), attn_mask=keep[None, None, None, :])
    sd = sd.numpy().reshape(h, n, d)
    assert abs(O.psnr(got, sd) - float(g[f"psnr_{name}"])) <= PSNR_DB


def test_masked_attention_per_batch_and_ragged(dev):
    """Different key counts per batch entry, counts inside a tile and at a
    tile edge, N not a multiple of the block; against the code-unit oracle."""
    b, h, n, d = 3, 2, 1000, 128
    q, k, v = make_qkv(b, h, n, d, seed=31)
    perm = np.stack([np.random.default_rng(40 + i).permutation(n) for i in range(b * h)]).astype(np.int32)
    kv = [333, 1000, 256]
    got = _masked_gpu(q, k, v, perm, kv, dev).reshape(b * h, n, d)
    prep = O.prepare(*(a.reshape(b * h, n, d) for a in (q, k, v)), perm, block_rows=128)
    codes = O.attention_codes(prep, n, 128, 128, d ** -0.5, kv_len=[kv[i // h] for i in range(b * h)])
    assert O.rel_l2(got, codes) <= REL_L2_CODES


def test_router_takes_key_padding_masks(dev):
    """runtime.attention with a boolean key-padding mask (scattered masked
    keys, different per batch entry) runs the masked kernel and agrees with
    SDPA under the same mask; a mask that varies by query still defers."""
    from comfyui_vc_attention_b200.vc_attention.patch import VCAttentionConfig, VCAttentionRuntime
    b, h, n, d = 2, 4, 2048, 128
    q, k, v = (_bf16(a, dev) for a in make_qkv(b, h, n, d, seed=33))
    rng = np.random.default_rng(3)
    keep = torch.from_numpy(rng.random((b, n)) > 0.3)
    keep[1, 1500:] = False
    mask = keep[:, None, None, :].to(dev)
    rt = VCAttentionRuntime(VCAttentionConfig(min_tokens=1024, enable_sparsity=True))
    out = rt.attention(q, k, v, attn_mask=mask)
    assert out is not None and out.dtype == torch.bfloat16 and rt.stats["used"] == 1
    sd = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), attn_mask=mask)
    assert O.psnr(out.float().cpu().numpy(), sd.cpu().numpy()) > 35.0
    again = rt.attention(q, k, v, attn_mask=mask)               # cached permutation, same result
    assert torch.equal(again, out)
    per_query = torch.ones(b, 1, n, n, dtype=torch.bool, device=dev)
    assert rt.attention(q, k, v, attn_mask=per_query) is None
