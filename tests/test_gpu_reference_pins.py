"""GPU results against fixtures made by the reference's own code.

tests/golden/sparse_ref.npz and nvfp4_ref.npz were written by
tests/golden/make_golden.py, which ran the reference package on CPU:

* its routing rule (kernels/triton_attn.py:449-459) on the portable
  ``prepare()`` codes with the statistics formula of :716-735, and the same
  rule on ``_prepare_fast`` (the bf16 prepare of its GPU path);
* ``simulate()`` of tests/_probe35_phase3.py:45-114, the reference's ground
  truth for its fused sparse kernel;
* ``vc_attention_reference`` with backend "nvfp4" and "fp8"
  (kernels/reference.py:162-294).

Also here: the ExpCast bytes of the attention kernels' own device routine and
the dense kernel's exact-ExpCast variant.
"""

import numpy as np
import pytest
import torch

from oracle import vc_oracle as O
from oracle.inputs import digest, make_qkv
from tests.test_oracle_golden import SPARSE_CASES, TIE_FAST, TIE_PREP, mask_agreement, sparse_case

pytestmark = pytest.mark.gpu

SIM_REL_L2 = 5e-2      # the reference probe's own kernel-vs-simulation gate (_probe35_phase3.py:140)
PSNR_DB = 0.3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from comfyui_vc_attention_b200.vc_attention import _native as N
    N.lib()
    return torch.device("cuda:0")


def _golden(name):
    import os
    return np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", name))


def _bf16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(torch.bfloat16)


def _prep(q, k, v, perm, dev, **kw):
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import prepare
    return prepare(_bf16(q, dev), _bf16(k, dev), _bf16(v, dev),
                   torch.from_numpy(np.ascontiguousarray(perm)).to(dev), **kw)


# ---------------------------------------------------------------- ExpCast ---

def test_kernel_expcast_routine_bytes_vs_reference(dev):
    """The one-FMA ExpCast routine the attention kernels run (tc::expcast4
    with the kernel's folding of the per-row constants) against the
    reference's expcast_codes bytes: at least 99 % identical, never more than
    one code apart."""
    from comfyui_vc_attention_b200.vc_attention.expcast import expcast_codes
    c = _golden("codecs.npz")
    s = torch.from_numpy(c["ec_s"]).to(dev)
    m = torch.from_numpy(c["ec_m"]).to(dev)
    fast = expcast_codes(s, m, exact=False).cpu().numpy().astype(np.int32)
    ref = c["ec_codes"].astype(np.int32)
    diff = np.abs(fast - ref)
    assert diff.max() <= 1
    assert (diff == 0).mean() >= 0.99


@pytest.mark.parametrize("n,br", [(1024, 128), (1000, 64)])
def test_dense_exact_expcast_matches_oracle(dev, n, br):
    """VCATTN_EXPCAST_EXACT: the dense tcgen05 kernel writes the P bytes in
    expcast.py's operation order, so its output follows the oracle of that
    arithmetic to fp32 accumulation noise (rel-L2 <= 1e-5)."""
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                          attention_status)
    h = 2
    q, k, v = make_qkv(1, h, n, 128, seed=21)
    perm = np.stack([np.random.default_rng(30 + i).permutation(n) for i in range(h)]).astype(np.int32)
    p = _prep(q, k, v, perm, dev, block_rows=br, want_v=True)
    out = torch.empty((1, h, n, 128), dtype=torch.float32, device=dev)
    cfg = TritonConfig(block_n=br, enable_expcast=True, expcast_exact=True)
    attention_prepared(p, n, out, 128 ** -0.5, cfg, kernel="tc")
    torch.cuda.synchronize()
    assert attention_status() == (0, 0, 0)
    got = out.cpu().numpy().reshape(h, n, 128)
    qg, kg, vg = (a.reshape(h, n, 128) for a in (q, k, v))
    prep = O.prepare(qg, kg, vg, perm, block_rows=br)
    ref = O.attention_codes(prep, n, br, 128, 128 ** -0.5, expcast=True)
    assert O.rel_l2(got, ref) <= 1e-5


# ------------------------------------------------------- routing & sparse ---

@pytest.mark.parametrize("name", list(SPARSE_CASES))
def test_gpu_route_mask_vs_reference_routing(dev, name):
    """The GPU's block mask against the reference's routing decisions: every
    disagreement is a tie within the stated margin of the reference's
    threshold, and at least 99.9 % of the decisions agree (both for the
    portable-prepare routing and for the bf16 fast prepare of the reference's
    GPU path)."""
    g = _golden("sparse_ref.npz")
    q, k, v = sparse_case(g, name)
    h, n, _ = q.shape
    p = _prep(q[None], k[None], v[None], g[f"{name}_perm"], dev, block_rows=128, sparse=True, tau=1.3,
              q_block=64, want_v=True)
    keep = p.keep.cpu().numpy().astype(bool)
    agree, margins = mask_agreement(keep, g, name, "prep", TIE_PREP)
    agree_f, margins_f = mask_agreement(keep, g, name, "fast", TIE_FAST)
    print(f"{name}: agreement with the reference routing {agree:.5f} (ties {margins}), "
          f"with its fast-prepare routing {agree_f:.5f} (ties {margins_f})")
    assert agree >= 0.999 and agree_f >= 0.999


def test_gpu_sparse_vs_reference_simulation(dev):
    """The tcgen05 sparse kernel's output against the reference's own sparse
    simulation: rel-L2 within the reference probe's 5e-2 gate and PSNR
    against fp32 SDPA within 0.3 dB of the simulation's."""
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                          attention_status)
    g = _golden("sparse_ref.npz")
    q, k, v = sparse_case(g, "s2k")
    h, n, d = q.shape
    p = _prep(q[None], k[None], v[None], g["s2k_perm"], dev, block_rows=128, sparse=True, tau=1.3,
              q_block=64, want_v=True)
    out = torch.empty((1, h, n, d), dtype=torch.float32, device=dev)
    cfg = TritonConfig(block_m=64, block_n=128, sparse=True, tau=1.3)
    attention_prepared(p, n, out, d ** -0.5, cfg, kernel="tc")
    torch.cuda.synchronize()
    assert attention_status() == (0, 0, 0)
    got = out.cpu().numpy().reshape(h, n, d)
    sim = g["s2k_sim_out"].astype(np.float32).reshape(h, n, d)
    rel = O.rel_l2(got, sim)
    sd = O.sdpa_f32(q, k, v)
    ps, ps_sim = O.psnr(got, sd), float(g["s2k_sim_psnr"])
    print(f"sparse vs reference simulation: rel-L2 {rel:.3e}, PSNR {ps:.2f} dB (simulation {ps_sim:.2f} dB), "
          f"keep {float(p.keep.float().mean()):.4f} (simulation {float(g['s2k_sim_keep']):.4f})")
    assert rel <= SIM_REL_L2
    assert abs(ps - ps_sim) <= PSNR_DB


# ------------------------------------------------------------------ NVFP4 ---

def test_gpu_nvfp4_and_fp8_vs_reference_backends(dev):
    """configs[3] semantics on a small shape: the NVFP4-QK kernel and the
    dense FP8 kernel against the reference's own ``vc_attention_reference``
    with backend "nvfp4" (Q/K, V and P all NVFP4 with 16-token micro scales)
    and "fp8", each measured as PSNR against fp32 SDPA.  The FP8 kernel is
    held to the north-star tolerance (within 0.3 dB of the reference's fp8
    PSNR, rel-L2 <= 2e-3 against its output); the NVFP4-QK kernel, which
    keeps P and V in FP8, must not fall below the reference's nvfp4 PSNR."""
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_status,
                                                                          vc_attention_cuda)
    g = _golden("nvfp4_ref.npz")
    h, n, d = 2, 2048, 128
    q, k, v = make_qkv(1, h, n, d, seed=8)
    assert digest(q, k, v) == str(g["digest"])
    perm = torch.from_numpy(g["perm"]).to(dev)
    qt, kt, vt = _bf16(q, dev), _bf16(k, dev), _bf16(v, dev)
    sd = O.sdpa_f32(*(a.reshape(h, n, d) for a in (q, k, v)))
    res = {}
    for name, cfg in (("nvfp4", TritonConfig(block_n=128, qk_fp4=True)), ("fp8", TritonConfig(block_n=128))):
        out = vc_attention_cuda(qt, kt, vt, perm, cfg)
        torch.cuda.synchronize()
        assert attention_status() == (0, 0, 0)
        res[name] = out.float().cpu().numpy().reshape(h, n, d)
    ps = {name: O.psnr(o, sd) for name, o in res.items()}
    ref_ps = {name: float(g[f"{name}_psnr"]) for name in ("nvfp4", "fp8")}
    print(f"PSNR vs fp32 SDPA: NVFP4-QK kernel {ps['nvfp4']:.2f} dB (reference nvfp4 backend "
          f"{ref_ps['nvfp4']:.2f} dB); FP8 kernel {ps['fp8']:.2f} dB (reference fp8 {ref_ps['fp8']:.2f} dB)")
    assert ps["nvfp4"] >= ref_ps["nvfp4"] - PSNR_DB
    assert abs(ps["fp8"] - ref_ps["fp8"]) <= PSNR_DB
    ref_fp8 = g["fp8_out"].astype(np.float32).reshape(h, n, d)
    assert O.rel_l2(res["fp8"], ref_fp8) <= 2e-3
