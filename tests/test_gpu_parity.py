"""GPU parity: the sm_100a kernels of libvcattn.so against the CPU oracle.

Bit-exact: E4M3/E2M1 encoders, ExpCast bytes (reference operation order),
k-means labels / centroids / permutation, prepared Q/K/V codes and scales.
Tolerance (attention output, fp32 accumulation order differs): rel-L2 <= 2e-3
against the reference's portable path and PSNR vs fp32 SDPA within 0.3 dB of
the reference's own PSNR; a tighter 1e-3 against the oracle of the kernel's
own code-unit arithmetic.
"""

import functools
import os

import numpy as np
import pytest
import torch

from oracle import vc_oracle as O
from oracle.inputs import digest, make_qkv

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
REL_L2_REF = 2e-3        # north-star tolerance vs the reference's portable path
PSNR_DB = 0.3
REL_L2_CODES = 1e-3      # vs the oracle of the kernel's own arithmetic


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from comfyui_vc_attention_b200.vc_attention import _native as N
    N.lib()   # raises if the library is missing: a GPU box must have it
    return torch.device("cuda:0")


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t.to(dtype) if dtype is not None else t


def _bf16(a, dev):
    return _t(a, dev, torch.bfloat16)


# ---------------------------------------------------------------- codecs ----

def test_e4m3_encoder_bit_exact(dev):
    from comfyui_vc_attention_b200.vc_attention.quant import e4m3_encode
    c = _load("codecs.npz")
    got = e4m3_encode(_t(c["e4m3_x"], dev)).cpu().numpy()
    assert np.array_equal(got, c["e4m3_codes"])
    # every fp32 bit pattern class near E4M3 ties / subnormals / saturation
    rng = np.random.default_rng(11)
    x = np.concatenate([rng.standard_normal(200000).astype(np.float32) * 50,
                        rng.standard_normal(100000).astype(np.float32) * 1e-2,
                        (np.arange(-4000, 4000, dtype=np.float32) / 16.0)])
    assert np.array_equal(e4m3_encode(_t(x, dev)).cpu().numpy(), O.e4m3_encode(x))


def test_fp4_encoder_bit_exact(dev):
    from comfyui_vc_attention_b200.vc_attention.quant import fp4_encode
    c = _load("codecs.npz")
    assert np.array_equal(fp4_encode(_t(c["fp4_x"], dev)).cpu().numpy(), c["fp4_codes"])
    x = (np.arange(-1000, 1000, dtype=np.float32) / 128.0)
    assert np.array_equal(fp4_encode(_t(x, dev)).cpu().numpy(), O.fp4_encode(x))


def test_expcast_bytes_bit_exact(dev):
    from comfyui_vc_attention_b200.vc_attention.expcast import expcast_codes
    c = _load("codecs.npz")
    s, m = _t(c["ec_s"], dev), _t(c["ec_m"], dev)
    exact = expcast_codes(s, m, exact=True).cpu().numpy()
    assert np.array_equal(exact, c["ec_codes"])
    fast = expcast_codes(s, m, exact=False).cpu().numpy().astype(np.int32)
    diff = np.abs(fast - exact.astype(np.int32))
    assert diff.max() <= 1
    assert (diff == 0).mean() >= 0.99


# --------------------------------------------------------------- k-means ----

def test_kmeans_config0_bit_exact(dev):
    from comfyui_vc_attention_b200.vc_attention.grouping import GroupingConfig, build_permutation
    g = _load("config0.npz")
    q, k, v = make_qkv(1, 2, 1024, 128, seed=0)
    assert digest(q, k, v) == str(g["inputs_digest"])
    res = build_permutation(_bf16(v.reshape(2, 1024, 128), dev), GroupingConfig(block_rows=64, iters=10))
    assert res.k == 16
    assert np.array_equal(res.perm.cpu().numpy(), g["perm"])
    assert np.array_equal(res.centroids.float().cpu().numpy(), g["centroids"])
    assert np.array_equal(res.labels.cpu().numpy(), g["labels"])


def test_kmeans_k64_bit_exact(dev):
    from comfyui_vc_attention_b200.vc_attention.grouping import GroupingConfig, build_permutation
    g = _load("kmeans64.npz")
    q, k, v = make_qkv(1, 2, 4096, 128, seed=1)
    res = build_permutation(_bf16(v.reshape(2, 4096, 128), dev),
                            GroupingConfig(block_rows=64, iters=3, max_clusters=64))
    assert res.k == 64
    assert np.array_equal(res.perm.cpu().numpy(), g["perm"])
    assert np.array_equal(res.centroids.float().cpu().numpy(), g["centroids"])


@pytest.mark.parametrize("n,k_clusters,iters", [(1000, 8, 3), (3000, 200, 2), (257, 3, 4)])
def test_kmeans_matches_oracle(dev, n, k_clusters, iters):
    from comfyui_vc_attention_b200.vc_attention.grouping import GroupingConfig, build_permutation
    q, k, v = make_qkv(1, 3, n, 128, seed=n)
    vb = v.reshape(3, n, 128)
    br = max(1, -(-n // k_clusters))
    perm_o, cent_o, kk, lab_o = O.build_permutation(vb, block_rows=br, iters=iters)
    res = build_permutation(_bf16(vb, dev), GroupingConfig(block_rows=br, iters=iters))
    assert res.k == kk
    assert np.array_equal(res.labels.cpu().numpy(), lab_o)
    assert np.array_equal(res.centroids.float().cpu().numpy(), cent_o)
    assert np.array_equal(res.perm.cpu().numpy(), perm_o)


def test_kmeans_warm_start_and_keys(dev):
    """Warm-started centroids and the modality / padding sort keys."""
    from comfyui_vc_attention_b200.vc_attention.grouping import GroupingConfig, build_permutation
    n = 2048
    q, k, v = make_qkv(1, 2, n, 128, seed=5)
    vb = v.reshape(2, n, 128)
    _, cent0, kk, _ = O.build_permutation(vb, block_rows=128, iters=2)
    tags = np.zeros(n, np.int64)
    tags[:128] = 1
    tags[128:384] = 2
    tags[-100:] = -1
    perm_o, cent_o, _, lab_o = O.build_permutation(vb, block_rows=128, iters=1, warm=cent0, warm_iters=2,
                                                   tags=tags, modality_aware=True, valid_len=n - 50)
    cfg = GroupingConfig(block_rows=128, iters=1, warm_iters=2, modality_aware=True)
    res = build_permutation(_bf16(vb, dev), cfg, tags=torch.from_numpy(tags),
                            centroids=_bf16(cent0, dev), valid_len=n - 50)
    assert np.array_equal(res.centroids.float().cpu().numpy(), cent_o)
    assert np.array_equal(res.perm.cpu().numpy(), perm_o)


def test_kmeans_input_layouts_agree(dev):
    """fp32 input and a strided (B, N, H, D)-backed view give the bf16 result."""
    from comfyui_vc_attention_b200.vc_attention.grouping import GroupingConfig, kmeans
    n = 1536
    q, k, v = make_qkv(1, 4, n, 128, seed=9)
    vt = _bf16(v, dev)                                           # (1, 4, n, 128)
    cfg = GroupingConfig(block_rows=128, iters=3)
    lab_a, cent_a, perm_a = kmeans(vt, 12, cfg)
    strided = vt.transpose(1, 2).contiguous().transpose(1, 2)    # same values, (B,N,H,D) memory
    lab_b, cent_b, perm_b = kmeans(strided, 12, cfg)
    lab_c, cent_c, perm_c = kmeans(vt.float(), 12, cfg)
    for lab, cent, perm in ((lab_b, cent_b, perm_b), (lab_c, cent_c, perm_c)):
        assert torch.equal(lab, lab_a) and torch.equal(cent, cent_a) and torch.equal(perm, perm_a)


@pytest.mark.parametrize("n,k_clusters,iters", [(16384, 512, 2), (5000, 300, 1), (4096, 1000, 1), (3000, 37, 2)])
def test_kmeans_tensor_core_assign_equals_cuda_core(dev, n, k_clusters, iters, monkeypatch):
    """bf16 D=128 input takes the tcgen05 assignment (certified argmax); the
    CUDA-core assignment (VCATTN_KMEANS_SIMT=1) is the definition it must
    reproduce: labels, centroids and permutation bit for bit, for k in one
    chunk, two chunks and two TMEM passes, and a head against the oracle."""
    from comfyui_vc_attention_b200.vc_attention.grouping import GroupingConfig, build_permutation
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import attention_status
    q, k, v = make_qkv(1, 2, n, 128, seed=n + k_clusters)
    vt = _bf16(v.reshape(2, n, 128), dev)
    br = max(1, n // k_clusters)          # ceil(n / br) >= k_clusters: k = max_clusters
    cfg = GroupingConfig(block_rows=br, iters=iters, max_clusters=k_clusters)
    res_tc = build_permutation(vt, cfg)
    assert attention_status() == (0, 0, 0), "a bounded wait of the tensor-core assignment expired"
    monkeypatch.setenv("VCATTN_KMEANS_SIMT", "1")
    res_ref = build_permutation(vt, cfg)
    assert res_tc.k == res_ref.k == k_clusters
    assert torch.equal(res_tc.labels, res_ref.labels)
    assert torch.equal(res_tc.centroids, res_ref.centroids)
    assert torch.equal(res_tc.perm, res_ref.perm)
    if n <= 5000:
        perm_o, cent_o, _, lab_o = O.build_permutation(v.reshape(2, n, 128)[:1], block_rows=br, iters=iters,
                                                       max_clusters=k_clusters)
        assert np.array_equal(res_tc.labels[:1].cpu().numpy(), lab_o)
        assert np.array_equal(res_tc.perm[:1].cpu().numpy(), perm_o)


# --------------------------------------------------------------- prepare ----

def _prep_gpu(q, k, v, perm, br, dev, **kw):
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import prepare
    return prepare(_bf16(q, dev), _bf16(k, dev), _bf16(v, dev),
                   None if perm is None else _t(perm, dev), block_rows=br, **kw)


def _assert_prepare_equal(p, ref, g_shape):
    G = g_shape
    np.testing.assert_array_equal(p.q.view(torch.uint8).reshape(G, -1, p.q.shape[-1]).cpu().numpy(), ref["q"])
    np.testing.assert_array_equal(p.k.view(torch.uint8).reshape(G, -1, p.k.shape[-1]).cpu().numpy(), ref["k"])
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import v_natural
    np.testing.assert_array_equal(v_natural(p).reshape(G, -1, p.v.shape[-1]).cpu().numpy(), ref["v"])
    for f in ("q_scale", "k_scale", "v_scale", "mu"):
        got = getattr(p, f).reshape(ref[f].shape).cpu().numpy()
        np.testing.assert_array_equal(got, ref[f], err_msg=f)


def test_prepare_config0_bit_exact(dev):
    g = _load("config0.npz")
    q, k, v = make_qkv(1, 2, 1024, 128, seed=0)
    q, k, v = (a.reshape(1, 2, 1024, 128) for a in (q, k, v))
    p = _prep_gpu(q, k, v, g["perm"], 64, dev, want_v_t=True, v_mma_order=True)
    ref = O.prepare(q.reshape(2, 1024, 128), k.reshape(2, 1024, 128), v.reshape(2, 1024, 128),
                    g["perm"], block_rows=64)
    _assert_prepare_equal(p, ref, 2)
    # codes equal the reference's own prepare() bytes
    assert np.array_equal(p.q.view(torch.uint8).cpu().numpy().reshape(g["q8"].shape), g["q8"])
    assert np.array_equal(p.k.view(torch.uint8).cpu().numpy().reshape(g["k8"].shape), g["k8"])
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import v_natural
    assert p.v_mma_order
    assert np.array_equal(v_natural(p).cpu().numpy().reshape(g["v8"].shape), g["v8"])
    # block-transposed V holds the same codes
    vt = p.v_t.cpu().numpy()                                   # (G, NB, D, BR)
    v8 = ref["v"].reshape(2, 16, 64, 128).transpose(0, 1, 3, 2)
    assert np.array_equal(vt, v8)


@pytest.mark.parametrize("n,br,h", [(200, 128, 2), (1000, 128, 3), (333, 64, 2), (64, 64, 1)])
def test_prepare_ragged_bit_exact(dev, n, br, h):
    q, k, v = make_qkv(1, h, n, 128, seed=n + br)
    rng = np.random.default_rng(n)
    perm = np.stack([rng.permutation(n) for _ in range(h)]).astype(np.int32)
    p = _prep_gpu(q, k, v, perm, br, dev)
    ref = O.prepare(q.reshape(h, n, 128), k.reshape(h, n, 128), v.reshape(h, n, 128), perm, block_rows=br)
    assert p.n_pad == ref["n_pad"]
    _assert_prepare_equal(p, ref, h)


def test_prepare_head_dim_64_and_shared_perm(dev):
    n, h = 500, 2
    q, k, v = make_qkv(1, h, n, 64, seed=4)
    perm = np.random.default_rng(3).permutation(n).astype(np.int32)[None, :]
    p = _prep_gpu(q, k, v, perm, 128, dev)
    ref = O.prepare(q.reshape(h, n, 64), k.reshape(h, n, 64), v.reshape(h, n, 64), perm, block_rows=128)
    _assert_prepare_equal(p, ref, h)


def test_prepare_without_hadamard_or_smoothing(dev):
    n, h = 300, 2
    q, k, v = make_qkv(1, h, n, 128, seed=8)
    p = _prep_gpu(q, k, v, None, 128, dev, hadamard=False, smooth_k=False)
    ref = O.prepare(q.reshape(h, n, 128), k.reshape(h, n, 128), v.reshape(h, n, 128), None,
                    block_rows=128, hadamard=False, smooth_k=False)
    _assert_prepare_equal(p, ref, h)


# ------------------------------------------------------------- attention ----

def _attn_gpu(q, k, v, perm, br, dev, expcast=False, out_dtype=torch.float32, kernel="mma"):
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig,
                                                                          attention_prepared,
                                                                          attention_status)
    p = _prep_gpu(q, k, v, perm, br, dev, want_v=True, want_v_t=True)
    b, h, n, d = q.shape
    out = torch.empty((b, h, n, d), dtype=out_dtype, device=dev)
    cfg = TritonConfig(block_n=br, enable_expcast=expcast)
    attention_prepared(p, n, out, d ** -0.5, cfg, kernel=kernel)
    torch.cuda.synchronize()
    if kernel == "tc":
        assert attention_status() == (0, 0, 0), "a bounded wait of the tcgen05 kernel expired"
    return out.float().cpu().numpy().reshape(b * h, n, d)


def _kernels(d):
    return ["tc", "mma"]


@pytest.mark.parametrize("kernel", ["tc", "mma"])
@pytest.mark.parametrize("expcast", [False, True])
def test_attention_config0(dev, expcast, kernel):
    g = _load("config0.npz")
    q, k, v = make_qkv(1, 2, 1024, 128, seed=0)
    got = _attn_gpu(q, k, v, g["perm"], 64, dev, expcast=expcast, kernel=kernel)
    G = 2
    qg, kg, vg = (a.reshape(G, 1024, 128) for a in (q, k, v))
    ref = g["out_expcast" if expcast else "out_plain"].reshape(G, 1024, 128)
    assert O.rel_l2(got, ref) <= REL_L2_REF
    prep = O.prepare(qg, kg, vg, g["perm"], block_rows=64)
    codes = O.attention_codes(prep, 1024, 64, 128, 128 ** -0.5, expcast=expcast)
    assert O.rel_l2(got, codes) <= REL_L2_CODES
    sd = O.sdpa_f32(qg, kg, vg)
    assert abs(O.psnr(got, sd) - O.psnr(ref, sd)) <= PSNR_DB


@pytest.mark.parametrize("n,br,d,h", [(200, 128, 128, 2), (1000, 64, 128, 2), (700, 128, 64, 3),
                                      (64, 64, 128, 1), (2048, 128, 128, 2), (300, 128, 128, 2),
                                      (600, 128, 128, 1)])
@pytest.mark.parametrize("kernel", ["tc", "mma"])
def test_attention_shapes(dev, n, br, d, h, kernel):
    """Ragged N, head_dim 64, single tile.  For N not a multiple of the block,
    the reference's prepare() takes the K token mean over N rows while its
    vc_attention_reference takes it over the padded rows; the kernel follows
    prepare() (whose bytes it reproduces), so the tight check is against the
    code-unit oracle on those bytes and the reference path is compared by
    PSNR (and by rel-L2 when the two definitions coincide)."""
    q, k, v = make_qkv(1, h, n, d, seed=n + d)
    qg, kg, vg = (a.reshape(h, n, d) for a in (q, k, v))
    perm = np.stack([np.random.default_rng(i).permutation(n) for i in range(h)]).astype(np.int32)
    if kernel not in _kernels(d):
        pytest.skip("the tcgen05 kernel is built for head_dim 128")
    got = _attn_gpu(q, k, v, perm, br, dev, kernel=kernel)
    prep = O.prepare(qg, kg, vg, perm, block_rows=br)
    codes = O.attention_codes(prep, n, br, 64, d ** -0.5)
    assert O.rel_l2(got, codes) <= REL_L2_CODES
    ref = O.attention_reference(qg, kg, vg, perm, block_rows=br, block_m=64)
    if n % br == 0:
        assert O.rel_l2(got, ref) <= REL_L2_REF
    sd = O.sdpa_f32(qg, kg, vg)
    assert abs(O.psnr(got, sd) - O.psnr(ref, sd)) <= PSNR_DB


def test_attention_bf16_output_and_layouts(dev):
    """Product entry point: bf16 in/out, 4-D and 3-D ComfyUI layouts agree."""
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import TritonConfig, vc_attention_cuda
    n, h, d = 1024, 4, 128
    q, k, v = make_qkv(1, h, n, d, seed=21)
    qt, kt, vt = _bf16(q, dev), _bf16(k, dev), _bf16(v, dev)
    perm = torch.stack([torch.randperm(n, generator=torch.Generator().manual_seed(i)) for i in range(h)])
    perm = perm.to(torch.int32).to(dev)
    cfg = TritonConfig(block_n=128)
    o4 = vc_attention_cuda(qt, kt, vt, perm, cfg)
    assert o4.dtype == torch.bfloat16 and o4.shape == (1, h, n, d)
    # (B, N, H*D) memory viewed as (B, H, N, D): no copy on the way in or out
    q3 = qt.transpose(1, 2).contiguous().transpose(1, 2)
    k3 = kt.transpose(1, 2).contiguous().transpose(1, 2)
    v3 = vt.transpose(1, 2).contiguous().transpose(1, 2)
    o3 = vc_attention_cuda(q3, k3, v3, perm, cfg)
    assert torch.equal(o3, o4)
    assert o3.transpose(1, 2).is_contiguous()
    ref = O.attention_reference(q.reshape(h, n, d), k.reshape(h, n, d), v.reshape(h, n, d),
                                perm.cpu().numpy(), block_rows=128)
    got = o4.float().cpu().numpy().reshape(h, n, d)
    assert O.rel_l2(got, O.bf16_round(ref)) <= REL_L2_REF


def test_router_routes_and_defers(dev):
    """SDPA hook: large calls go through the kernels, a host-injected kernel
    failure defers to the original attention, uninstall restores it."""
    import torch.nn.functional as F
    from comfyui_vc_attention_b200.vc_attention import _native as N
    from comfyui_vc_attention_b200.vc_attention.patch import (VCAttentionConfig, get_runtime, install,
                                                              uninstall)
    orig = F.scaled_dot_product_attention
    n, h, d = 1024, 2, 128
    q, k, v = make_qkv(1, h, n, d, seed=31)
    qt, kt, vt = _bf16(q, dev), _bf16(k, dev), _bf16(v, dev)
    try:
        rt = install(VCAttentionConfig(min_tokens=512, enable_sparsity=False))
        rt.begin_step()
        out = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt)
        assert rt.stats["used"] == 1 and rt.stats["grouped"] == 1
        sd = O.sdpa_f32(q.reshape(h, n, d), k.reshape(h, n, d), v.reshape(h, n, d))
        assert O.psnr(out.float().cpu().numpy().reshape(h, n, d), sd) > 35.0
        N.inject_fault("vcattn_attn_fp8")
        try:
            out2 = torch.nn.functional.scaled_dot_product_attention(qt, kt, vt)
        finally:
            N.inject_fault(None)
        assert torch.equal(out2, orig(qt, kt, vt))
        assert get_runtime().stats["used"] == 2
    finally:
        uninstall()
    assert F.scaled_dot_product_attention is orig


# ------------------------------------------------------- block-sparse path ----

def _sparse_case(n=1024, h=2, seed=3, grid=(4, 16, 16)):
    q, k, v = make_qkv(1, h, n, 128, seed=seed, spatial=grid)
    G = h
    vb = v.reshape(G, n, 128)
    perm, _, _, _ = O.build_permutation(vb, block_rows=128, iters=3)
    return q, k, v, perm


@pytest.mark.parametrize("tau,local,sink", [(1.3, 1, 0), (0.5, 0, 1), (2.0, 1, 2)])
def test_route_mask_bit_exact(dev, tau, local, sink):
    n, h, br, qb = 1024, 2, 128, 64
    q, k, v, perm = _sparse_case(n, h)
    sc = 128 ** -0.5
    p = _prep_gpu(q, k, v, perm, br, dev, sparse=True, tau=tau, q_block=qb, want_v_t=True,
                  local_blocks=local, sink_blocks=sink)
    prep = O.prepare(q.reshape(h, n, 128), k.reshape(h, n, 128), v.reshape(h, n, 128), perm, block_rows=br)
    st = O.route_stats(prep, br, qb, tau, sc)
    keep, score = O.route_mask(prep, st, n, br, qb, sc, local_blocks=local, sink_blocks=sink)
    assert np.array_equal(p.k_mean.reshape(st["k_mean"].shape).cpu().numpy(), st["k_mean"])
    assert np.array_equal(p.v_mean.reshape(st["v_mean"].shape).cpu().numpy(), st["v_mean"])
    assert np.array_equal(p.thresh.reshape(st["thresh"].shape).cpu().numpy(), st["thresh"])
    got = p.keep.cpu().numpy().astype(bool)
    assert np.array_equal(got, keep)
    assert 0.0 < keep.mean() < 1.0, "routing must be non-trivial on the spatial inputs"


def _sparse_gpu(q, k, v, perm, dev, tau, local=1, sink=0, expcast=False, out_dtype=torch.float32, kernel="mma",
                br=128):
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                           attention_status)
    b, h, n, d = q.shape
    tc = kernel == "tc"
    p = _prep_gpu(q, k, v, perm, br, dev, sparse=True, tau=tau, q_block=64, want_v_t=not tc, want_v=tc,
                  local_blocks=local, sink_blocks=sink)
    out = torch.empty((b, h, n, d), dtype=out_dtype, device=dev)
    cfg = TritonConfig(block_m=64, block_n=br, sparse=True, tau=tau, local_blocks=local, sink_blocks=sink,
                       enable_expcast=expcast)
    attention_prepared(p, n, out, d ** -0.5, cfg, kernel=kernel)
    torch.cuda.synchronize()
    if tc:
        assert attention_status() == (0, 0, 0), "a bounded wait of the tcgen05 sparse kernel expired"
    return out.float().cpu().numpy().reshape(b * h, n, d), p


def _route_tiles_np(k_mean, v_mean):
    """Expected bytes of vcattn_route_tiles: per (head, group of 16 blocks) an
    8 KB tile, bf16(k_mean) K-major then bf16(v_mean) MN-major with rows in
    the proxy MMA's key order, both in the 128-byte swizzle."""
    g, nb, d = k_mean.shape
    ng = -(-nb // 16)
    out = np.zeros((g, ng, 8192), np.uint8)
    kb = O.f32_to_bf16_bits(k_mean).astype(np.uint16)
    vb = O.f32_to_bf16_bits(v_mean).astype(np.uint16)

    def sw(r, c):
        return r * 128 + ((((c >> 4) ^ (r & 7)) & 7) << 4) + (c & 15)

    def blk_of(kpos):
        return 2 * (kpos >> 2) + (kpos & 3) if (kpos & 3) < 2 else 8 + 2 * (kpos >> 2) + (kpos & 3) - 2

    for gi in range(g):
        for gr in range(ng):
            t = out[gi, gr]
            for which, src in ((0, kb), (1, vb)):
                for r in range(16):
                    blk = gr * 16 + (r if which == 0 else blk_of(r))
                    if blk >= nb:
                        continue
                    for ch in range(d):
                        half, c = ch // 64, (ch % 64) * 2
                        off = which * 4096 + half * 2048 + sw(r, c)
                        val = int(src[gi, blk, ch])
                        t[off] = val & 0xFF
                        t[off + 1] = val >> 8
    return out


def test_route_tiles_layout(dev):
    n, h = 2500, 2     # 20 blocks: a full and a partial group
    q, k, v = make_qkv(1, h, n, 128, seed=5)
    perm = np.stack([np.random.default_rng(i).permutation(n) for i in range(h)]).astype(np.int32)
    p = _prep_gpu(q, k, v, perm, 128, dev, sparse=True, tau=1.3, q_block=64, want_v=True)
    assert p.ap_tiles is not None
    nb = p.k_mean.shape[-2]
    want = _route_tiles_np(p.k_mean.reshape(h, nb, 128).cpu().numpy(), p.v_mean.reshape(h, nb, 128).cpu().numpy())
    np.testing.assert_array_equal(p.ap_tiles.cpu().numpy(), want)


@pytest.mark.parametrize("kernel", ["tc", "mma"])
@pytest.mark.parametrize("expcast", [False, True])
def test_sparse_attention_matches_oracle(dev, expcast, kernel):
    n, h = 1024, 2
    q, k, v, perm = _sparse_case(n, h)
    got, p = _sparse_gpu(q, k, v, perm, dev, tau=1.3, expcast=expcast, kernel=kernel)
    qg, kg, vg = (a.reshape(h, n, 128) for a in (q, k, v))
    prep = O.prepare(qg, kg, vg, perm, block_rows=128)
    st = O.route_stats(prep, 128, 64, 1.3, 128 ** -0.5)
    keep = p.keep.cpu().numpy().astype(bool)
    ref = O.attention_sparse_codes(prep, st, keep, n, 128, 64, 128 ** -0.5, group=16, expcast=expcast)
    assert O.rel_l2(got, ref) <= REL_L2_CODES
    sd = O.sdpa_f32(qg, kg, vg)
    assert O.psnr(got, sd) > 20.0


@pytest.mark.parametrize("kernel", ["tc", "mma"])
def test_sparse_keep_all_equals_dense(dev, kernel):
    """tau -> -inf keeps every block: the sparse kernel must reproduce the
    dense kernel of the same family bit for bit (exact tiles, same order)."""
    n, h = 1024, 2
    q, k, v, perm = _sparse_case(n, h)
    sparse, p = _sparse_gpu(q, k, v, perm, dev, tau=-1000.0, kernel=kernel)
    assert p.keep.bool().all()
    dense = _attn_gpu(q, k, v, perm, 128, dev, kernel=kernel)
    assert np.array_equal(sparse, dense)


@pytest.mark.parametrize("kernel", ["tc", "mma"])
def test_sparse_ragged_and_multi_group(dev, kernel):
    """N not a multiple of the block, more than one 16-block group."""
    n, h = 2500, 2
    q, k, v = make_qkv(1, h, n, 128, seed=12)
    perm = np.stack([np.random.default_rng(i).permutation(n) for i in range(h)]).astype(np.int32)
    got, p = _sparse_gpu(q, k, v, perm, dev, tau=0.8, local=0, kernel=kernel)
    qg, kg, vg = (a.reshape(h, n, 128) for a in (q, k, v))
    prep = O.prepare(qg, kg, vg, perm, block_rows=128)
    st = O.route_stats(prep, 128, 64, 0.8, 128 ** -0.5)
    keep_o, _ = O.route_mask(prep, st, n, 128, 64, 128 ** -0.5, local_blocks=0)
    keep = p.keep.cpu().numpy().astype(bool)
    assert np.array_equal(keep, keep_o)
    ref = O.attention_sparse_codes(prep, st, keep, n, 128, 64, 128 ** -0.5, group=16)
    assert O.rel_l2(got, ref) <= REL_L2_CODES


_SPARSE_SHAPES = [(1024, 64, 128, 1.3), (1024, 128, 64, 1.3), (1000, 64, 64, 0.8), (2048, 64, 128, 0.8),
                  (2500, 128, 64, 0.8)]


def _sparse_shape_case(n, br, d):
    grid = {1024: (4, 16, 16), 2048: (8, 16, 16)}.get(n)
    q, k, v = make_qkv(1, 2, n, d, seed=n + d + br, spatial=grid)
    perm = np.stack([np.random.default_rng(70 + i).permutation(n) for i in range(2)]).astype(np.int32)
    return q, k, v, perm


@pytest.mark.parametrize("n,br,d,tau", _SPARSE_SHAPES)
@pytest.mark.parametrize("kernel", ["tc", "mma"])
def test_sparse_shapes(dev, n, br, d, tau, kernel):
    """Value blocks of 64 keys and head dim 64 (one and two 16-block groups,
    ragged N) on both sparse kernels: the GPU routing mask equals the
    oracle's, and the output matches the oracle driven by that mask."""
    h = 2
    q, k, v, perm = _sparse_shape_case(n, br, d)
    got, p = _sparse_gpu(q, k, v, perm, dev, tau=tau, kernel=kernel, br=br)
    qg, kg, vg = (a.reshape(h, n, d) for a in (q, k, v))
    prep = O.prepare(qg, kg, vg, perm, block_rows=br)
    sc = d ** -0.5
    st = O.route_stats(prep, br, 64, tau, sc)
    keep_o, _ = O.route_mask(prep, st, n, br, 64, sc, local_blocks=1)
    keep = p.keep.cpu().numpy().astype(bool)
    assert np.array_equal(keep, keep_o)
    assert 0.0 < keep.mean() < 1.0
    ref = O.attention_sparse_codes(prep, st, keep, n, br, 64, sc, group=16)
    assert O.rel_l2(got, ref) <= REL_L2_CODES


@pytest.mark.parametrize("n,br,d", [(1024, 64, 128), (1024, 128, 64), (1000, 64, 64)])
def test_sparse_tc_keep_all_equals_dense_shapes(dev, n, br, d):
    """Every block kept: the tcgen05 sparse kernel at 64-key value blocks and
    head dim 64 equals the dense tcgen05 kernel of the same shape bit for bit."""
    q, k, v, perm = _sparse_shape_case(n, br, d)
    sparse, p = _sparse_gpu(q, k, v, perm, dev, tau=-1000.0, kernel="tc", br=br)
    assert p.keep.bool().all()
    dense = _attn_gpu(q, k, v, perm, br, dev, kernel="tc")
    assert np.array_equal(sparse, dense)


# ------------------------------------------------------------ NVFP4 Q / K ----

@pytest.mark.parametrize("n,d,br", [(1024, 128, 128), (1000, 128, 128), (700, 64, 64)])
def test_prepare_nvfp4_bit_exact(dev, n, d, br):
    """E2M1 codes, E4M3 micro scales and the per-head tensor scale equal the
    oracle's quant.py:172-204 on each head's rotated (and smoothed) slab."""
    h = 2
    q, k, v = make_qkv(1, h, n, d, seed=7)
    perm = np.stack([np.random.default_rng(i).permutation(n) for i in range(h)]).astype(np.int32)
    p = _prep_gpu(q, k, v, perm, br, dev, qk_fp4=True)
    ref = O.prepare(q.reshape(h, n, d), k.reshape(h, n, d), v.reshape(h, n, d), perm, block_rows=br)
    n_pad = p.n_pad
    for name, pk, ps, pg in (("q_t", p.q4, p.q4_scale, p.q4_g), ("k_t", p.k4, p.k4_scale, p.k4_g)):
        packed, micro, gs = O.nvfp4_per_head(ref[name])
        np.testing.assert_array_equal(pk.reshape(h, n_pad, d // 2).cpu().numpy(), packed, err_msg=name)
        np.testing.assert_array_equal(ps.reshape(h, n_pad, d // 16).cpu().numpy(), micro, err_msg=name)
        np.testing.assert_array_equal(pg.cpu().numpy(), gs, err_msg=name)


@pytest.mark.parametrize("n,expcast", [(1024, False), (1024, True), (1000, True)])
def test_attention_nvfp4_matches_oracle(dev, n, expcast):
    """NVFP4 QK^T (block-scaled tcgen05 MMA) + FP8 PV against the oracle of
    the same arithmetic (Q/K dequantised from NVFP4, P/V FP8)."""
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                          attention_status)
    h = 2
    q, k, v = make_qkv(1, h, n, 128, seed=11)
    perm = np.stack([np.random.default_rng(i).permutation(n) for i in range(h)]).astype(np.int32)
    p = _prep_gpu(q, k, v, perm, 128, dev, qk_fp4=True, want_v=True, v_mma_order=False)
    out = torch.empty((1, h, n, 128), dtype=torch.float32, device=dev)
    cfg = TritonConfig(block_n=128, enable_expcast=expcast, qk_fp4=True)
    attention_prepared(p, n, out, 128 ** -0.5, cfg)
    torch.cuda.synchronize()
    assert attention_status() == (0, 0, 0)
    got = out.cpu().numpy().reshape(h, n, 128)
    qg, kg, vg = (a.reshape(h, n, 128) for a in (q, k, v))
    prep = O.prepare(qg, kg, vg, perm, block_rows=128)
    ref = O.attention_codes_nvfp4(prep, n, 128, 128, 128 ** -0.5, expcast=expcast)
    assert O.rel_l2(got, ref) <= REL_L2_CODES
    assert O.psnr(got, O.sdpa_f32(qg, kg, vg)) > 20.0


def test_vc_attention_cuda_nvfp4_entry_point(dev):
    """The public entry point with TritonConfig(qk_fp4=True), bf16 in / out."""
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import TritonConfig, vc_attention_cuda
    h, n = 2, 1024
    q, k, v = make_qkv(1, h, n, 128, seed=12)
    perm = np.stack([np.random.default_rng(10 + i).permutation(n) for i in range(h)]).astype(np.int32)
    out = vc_attention_cuda(_bf16(q, dev), _bf16(k, dev), _bf16(v, dev), _t(perm, dev),
                            TritonConfig(block_n=128, enable_expcast=True, qk_fp4=True))
    torch.cuda.synchronize()
    got = out.float().cpu().numpy().reshape(h, n, 128)
    qg, kg, vg = (a.reshape(h, n, 128) for a in (q, k, v))
    ref = O.attention_codes_nvfp4(O.prepare(qg, kg, vg, perm, block_rows=128), n, 128, 128, 128 ** -0.5,
                                  expcast=True)
    assert O.rel_l2(got, ref) <= 5e-3      # bf16 output rounding


# ------------------------------------------------- host-tensor entry point ----

@pytest.mark.parametrize("sparse", [False, True])
def test_vc_attention_host_matches_device_call(dev, sparse):
    """The chunk-pipelined host entry point gives the device call's bytes
    (units are independent; 6 heads in chunks of 4, 1 and 1)."""
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, vc_attention_cuda,
                                                                           vc_attention_host)
    b, h, n, d = 1, 6, 1024, 128
    q, k, v = make_qkv(b, h, n, d, seed=31)
    qt, kt, vt = _bf16(q, dev), _bf16(k, dev), _bf16(v, dev)
    perm = torch.stack([torch.randperm(n, generator=torch.Generator().manual_seed(i)) for i in range(h)])
    perm = perm.to(torch.int32).to(dev)
    cfg = TritonConfig(block_m=64, block_n=128, sparse=sparse, tau=1.3, enable_expcast=True)
    want = vc_attention_cuda(qt, kt, vt, perm, cfg).cpu()
    qh, kh, vh = (t.cpu().pin_memory() for t in (qt, kt, vt))
    got = vc_attention_host(qh, kh, vh, perm, cfg, chunk_heads=4)
    assert not got.is_cuda and got.shape == want.shape
    assert torch.equal(got, want)


# ------------------------------------------- BASELINE full sizes (56 x 16K) ----
#
# configs[1] (dense, ExpCast) and configs[2] (tau = 1.3 sparse) at their own
# shape, B=1, H=56, N=16384, D=128, V-Smooth k=64.  The GPU runs every head;
# the oracle re-derives sampled heads (k-means permutation, prepared codes,
# routing statistics and mask: bit-exact) and sampled 64-row query blocks of
# the output (rel-L2 <= REL_L2_CODES).  Size-independent properties cover the
# rest: every permutation row is a permutation, the output is finite, and the
# sparse kernel with every block kept equals the dense kernel bit for bit.

FULL_H, FULL_N, FULL_D = 56, 16384, 128
FULL_HEADS = [0, 37]
FULL_ROW_BLOCKS = [0, 97, 255]


@functools.lru_cache(maxsize=2)
def _full_pipeline(dev, spatial, seed):
    """Inputs (host and device) and the GPU permutation, shared by the tests
    of one config (generating 3 x 117M seeded values takes most of a minute)."""
    from comfyui_vc_attention_b200.vc_attention.grouping import GroupingConfig, build_permutation
    q, k, v = make_qkv(1, FULL_H, FULL_N, FULL_D, seed=seed, spatial=spatial)
    qt, kt, vt = _bf16(q, dev), _bf16(k, dev), _bf16(v, dev)
    res = build_permutation(vt.view(FULL_H, FULL_N, FULL_D),
                            GroupingConfig(block_rows=128, iters=3, max_clusters=64))
    assert res.k == 64
    perm = res.perm
    srt = torch.sort(perm.long(), dim=-1).values
    assert torch.equal(srt, torch.arange(FULL_N, device=dev).expand_as(srt)), "a row is not a permutation"
    return q, k, v, qt, kt, vt, perm.cpu().numpy()


def _oracle_heads(q, k, v, gpu_perm, heads):
    """Oracle permutation and prepare() of the sampled heads."""
    sel = (lambda a: a.reshape(FULL_H, FULL_N, FULL_D)[heads])
    qh, kh, vh = sel(q), sel(k), sel(v)
    for i, hh in enumerate(heads):
        perm_o, _, kc, _ = O.build_permutation(vh[i:i + 1], block_rows=128, iters=3, max_clusters=64)
        assert kc == 64
        np.testing.assert_array_equal(gpu_perm[hh], perm_o[0], err_msg=f"k-means permutation, head {hh}")
    return O.prepare(qh, kh, vh, gpu_perm[heads], block_rows=128)


def _assert_prepare_heads(p, ref, heads):
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import v_natural
    d = p.q.shape[-1]
    np.testing.assert_array_equal(p.q.view(torch.uint8).reshape(FULL_H, -1, d)[heads].cpu().numpy(), ref["q"])
    np.testing.assert_array_equal(p.k.view(torch.uint8).reshape(FULL_H, -1, d)[heads].cpu().numpy(), ref["k"])
    np.testing.assert_array_equal(v_natural(p).reshape(FULL_H, -1, d)[heads].cpu().numpy(), ref["v"])
    for f in ("q_scale", "k_scale", "v_scale", "mu"):
        got = getattr(p, f).reshape((FULL_H,) + ref[f].shape[1:])[heads].cpu().numpy()
        np.testing.assert_array_equal(got, ref[f], err_msg=f)


def _rows(a, heads):
    """(len(heads), rows of FULL_ROW_BLOCKS, D) slice of a (G, N, D) array."""
    idx = np.concatenate([np.arange(i * 64, (i + 1) * 64) for i in FULL_ROW_BLOCKS])
    return a[heads][:, idx]


def test_full_size_config1_dense(dev):
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                           attention_status, prepare)
    q, k, v, qt, kt, vt, perm = _full_pipeline(dev, None, seed=7)
    p = prepare(qt, kt, vt, _t(perm, dev), block_rows=128, want_v=True)
    sc = FULL_D ** -0.5
    out = torch.empty((1, FULL_H, FULL_N, FULL_D), dtype=torch.float32, device=dev)
    attention_prepared(p, FULL_N, out, sc, TritonConfig(block_n=128, enable_expcast=True), kernel="tc")
    torch.cuda.synchronize()
    assert attention_status() == (0, 0, 0), "a bounded wait of the tcgen05 kernel expired"
    assert bool(torch.isfinite(out).all())
    got = out.reshape(FULL_H, FULL_N, FULL_D).cpu().numpy()

    ref = _oracle_heads(q, k, v, perm, FULL_HEADS)
    _assert_prepare_heads(p, ref, FULL_HEADS)
    codes = O.attention_codes(ref, FULL_N, 128, 64, sc, expcast=True, row_blocks=FULL_ROW_BLOCKS)
    assert O.rel_l2(_rows(got, FULL_HEADS), _rows(codes, slice(None))) <= REL_L2_CODES
    # against fp32 SDPA on the same rows (all 16384 keys)
    qh = q.reshape(FULL_H, FULL_N, FULL_D)[FULL_HEADS]
    idx = np.concatenate([np.arange(i * 64, (i + 1) * 64) for i in FULL_ROW_BLOCKS])
    sd = O.sdpa_f32(qh[:, idx], k.reshape(FULL_H, FULL_N, FULL_D)[FULL_HEADS],
                    v.reshape(FULL_H, FULL_N, FULL_D)[FULL_HEADS])
    assert O.psnr(_rows(got, FULL_HEADS), sd) > 30.0


def test_full_size_config2_sparse(dev):
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                           attention_status, prepare)
    q, k, v, qt, kt, vt, perm = _full_pipeline(dev, (16, 32, 32), seed=9)
    sc, tau = FULL_D ** -0.5, 1.3
    pt = _t(perm, dev)
    p = prepare(qt, kt, vt, pt, block_rows=128, sparse=True, tau=tau, q_block=64, want_v=True)
    cfg = TritonConfig(block_m=64, block_n=128, sparse=True, tau=tau, enable_expcast=True)
    out = torch.empty((1, FULL_H, FULL_N, FULL_D), dtype=torch.float32, device=dev)
    attention_prepared(p, FULL_N, out, sc, cfg, kernel="tc")
    torch.cuda.synchronize()
    assert attention_status() == (0, 0, 0), "a bounded wait of the tcgen05 sparse kernel expired"
    assert bool(torch.isfinite(out).all())
    keep_all = p.keep.cpu().numpy().astype(bool)
    assert 0.02 < 1.0 - keep_all.mean() < 0.98, "routing must skip some blocks and keep some"
    got = out.reshape(FULL_H, FULL_N, FULL_D).cpu().numpy()

    ref = _oracle_heads(q, k, v, perm, FULL_HEADS)
    _assert_prepare_heads(p, ref, FULL_HEADS)
    st = O.route_stats(ref, 128, 64, tau, sc)
    keep_o, _ = O.route_mask(ref, st, FULL_N, 128, 64, sc)
    nb = FULL_N // 128
    for f, shp in (("k_mean", (nb, FULL_D)), ("v_mean", (nb, FULL_D)), ("thresh", (FULL_N // 64,))):
        np.testing.assert_array_equal(getattr(p, f).reshape((FULL_H,) + shp)[FULL_HEADS].cpu().numpy(), st[f],
                                      err_msg=f)
    np.testing.assert_array_equal(keep_all[FULL_HEADS], keep_o)
    codes = O.attention_sparse_codes(ref, st, keep_o, FULL_N, 128, 64, sc, group=16, expcast=True,
                                     row_blocks=FULL_ROW_BLOCKS)
    assert O.rel_l2(_rows(got, FULL_HEADS), _rows(codes, slice(None))) <= REL_L2_CODES


def test_full_size_sparse_keep_all_equals_dense(dev):
    """tau -> -inf at configs[2]'s shape: all 56 x 256 x 128 blocks kept, the
    sparse kernel's output equals the dense kernel's bit for bit."""
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                           attention_status, prepare)
    q, k, v, qt, kt, vt, perm = _full_pipeline(dev, (16, 32, 32), seed=9)
    pt, sc = _t(perm, dev), FULL_D ** -0.5
    ps = prepare(qt, kt, vt, pt, block_rows=128, sparse=True, tau=-1000.0, q_block=64, want_v=True)
    assert bool(ps.keep.bool().all())
    o_s = torch.empty((1, FULL_H, FULL_N, FULL_D), dtype=torch.bfloat16, device=dev)
    attention_prepared(ps, FULL_N, o_s, sc, TritonConfig(block_m=64, block_n=128, sparse=True, tau=-1000.0,
                                                        enable_expcast=True), kernel="tc")
    del ps
    pd = prepare(qt, kt, vt, pt, block_rows=128, want_v=True)
    o_d = torch.empty_like(o_s)
    attention_prepared(pd, FULL_N, o_d, sc, TritonConfig(block_n=128, enable_expcast=True), kernel="tc",
                       kv_split=1)
    torch.cuda.synchronize()
    assert attention_status() == (0, 0, 0)
    assert torch.equal(o_s, o_d)


# ------------------------------------ per-head full size, N = 65536, k = 512 ----
#
# configs[3] / configs[4] / the N = 65536 case of configs[2] run 65536 tokens
# per head with V-Smooth k = 512.  Two heads of that size carry the per-head
# work of the 56-head calls; the GPU permutation (tensor-core k-means, checked
# against the oracle at smaller sizes) feeds both sides, and the oracle checks
# the prepared codes bit for bit and three query blocks of each output.

N64K, H64K = 65536, 2


def _perm64k(vt):
    from comfyui_vc_attention_b200.vc_attention.grouping import GroupingConfig, build_permutation
    res = build_permutation(vt.view(H64K, N64K, 128), GroupingConfig(block_rows=128, iters=3, max_clusters=512))
    assert res.k == 512
    srt = torch.sort(res.perm.long(), dim=-1).values
    assert torch.equal(srt, torch.arange(N64K, device=vt.device).expand_as(srt))
    return res.perm


def test_n65536_dense_fp8_and_nvfp4(dev):
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                           attention_status, prepare)
    q, k, v = make_qkv(1, H64K, N64K, 128, seed=31)
    qt, kt, vt = _bf16(q, dev), _bf16(k, dev), _bf16(v, dev)
    perm = _perm64k(vt)
    sc = 128 ** -0.5
    qg, kg, vg = (a.reshape(H64K, N64K, 128) for a in (q, k, v))
    ref = O.prepare(qg, kg, vg, perm.cpu().numpy(), block_rows=128)
    # FP8 (configs[3] FP8 line, configs[4] dense)
    p = prepare(qt, kt, vt, perm, block_rows=128, want_v=True)
    np.testing.assert_array_equal(p.q.view(torch.uint8).reshape(H64K, -1, 128).cpu().numpy(), ref["q"])
    np.testing.assert_array_equal(p.k.view(torch.uint8).reshape(H64K, -1, 128).cpu().numpy(), ref["k"])
    np.testing.assert_array_equal(p.v.view(torch.uint8).reshape(H64K, -1, 128).cpu().numpy(), ref["v"])
    out = torch.empty((1, H64K, N64K, 128), dtype=torch.float32, device=dev)
    attention_prepared(p, N64K, out, sc, TritonConfig(block_n=128, enable_expcast=True), kernel="tc")
    torch.cuda.synchronize()
    assert attention_status() == (0, 0, 0)
    got = out.reshape(H64K, N64K, 128).cpu().numpy()
    blocks = [0, 511, 1023]
    rows = np.concatenate([np.arange(i * 64, (i + 1) * 64) for i in blocks])
    codes = O.attention_codes(ref, N64K, 128, 64, sc, expcast=True, row_blocks=blocks)
    assert O.rel_l2(got[:, rows], codes[:, rows]) <= REL_L2_CODES
    del p
    # NVFP4 QK^T
    p4 = prepare(qt, kt, vt, perm, block_rows=128, want_v=True, qk_fp4=True, fp8_qk=False)
    attention_prepared(p4, N64K, out, sc, TritonConfig(block_n=128, enable_expcast=True, qk_fp4=True))
    torch.cuda.synchronize()
    assert attention_status() == (0, 0, 0)
    got4 = out.reshape(H64K, N64K, 128).cpu().numpy()
    blocks4 = [0, 255, 511]
    rows4 = np.concatenate([np.arange(i * 128, (i + 1) * 128) for i in blocks4])
    codes4 = O.attention_codes_nvfp4(ref, N64K, 128, 128, sc, expcast=True, row_blocks=blocks4)
    assert O.rel_l2(got4[:, rows4], codes4[:, rows4]) <= REL_L2_CODES


def test_n65536_sparse_on_the_64x32x32_grid(dev):
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                           attention_status, prepare)
    q, k, v = make_qkv(1, H64K, N64K, 128, seed=33, spatial=(64, 32, 32))
    qt, kt, vt = _bf16(q, dev), _bf16(k, dev), _bf16(v, dev)
    perm = _perm64k(vt)
    sc, tau = 128 ** -0.5, 1.3
    p = prepare(qt, kt, vt, perm, block_rows=128, sparse=True, tau=tau, q_block=64, want_v=True)
    out = torch.empty((1, H64K, N64K, 128), dtype=torch.float32, device=dev)
    attention_prepared(p, N64K, out, sc, TritonConfig(block_m=64, block_n=128, sparse=True, tau=tau,
                                                     enable_expcast=True), kernel="tc")
    torch.cuda.synchronize()
    assert attention_status() == (0, 0, 0)
    qg, kg, vg = (a.reshape(H64K, N64K, 128) for a in (q, k, v))
    ref = O.prepare(qg, kg, vg, perm.cpu().numpy(), block_rows=128)
    st = O.route_stats(ref, 128, 64, tau, sc)
    keep_o, _ = O.route_mask(ref, st, N64K, 128, 64, sc)
    keep = p.keep.cpu().numpy().astype(bool).reshape(keep_o.shape)
    np.testing.assert_array_equal(keep, keep_o)
    assert 0.5 < 1.0 - keep.mean() < 0.99
    got = out.reshape(H64K, N64K, 128).cpu().numpy()
    blocks = [0, 511, 1023]
    rows = np.concatenate([np.arange(i * 64, (i + 1) * 64) for i in blocks])
    codes = O.attention_sparse_codes(ref, st, keep_o, N64K, 128, 64, sc, group=16, expcast=True, row_blocks=blocks)
    assert O.rel_l2(got[:, rows], codes[:, rows]) <= REL_L2_CODES
