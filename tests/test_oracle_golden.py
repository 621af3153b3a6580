"""Pin the CPU oracle to the reference implementation's own outputs.

tests/golden/*.npz were produced by tests/golden/make_golden.py, which ran the
reference package (bingling360/comfyui_vc_attention) on the seeded inputs of
oracle/inputs.py.  Every byte-level quantity (E4M3/E2M1 codes, ExpCast bytes,
Hadamard outputs, k-means labels / centroids / permutation, prepared Q/K/V
codes) must match exactly.  Two scales are derived from a mean whose fp32
summation order the reference leaves to torch (cascade sum); the oracle rounds
that sum once, so those two are checked to a few ulps and their codes exactly.
"""

import os

import numpy as np
import pytest

from oracle import vc_oracle as O
from oracle.inputs import digest, make_qkv

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def _ulps(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(a - b)


@pytest.fixture(scope="module")
def codecs():
    return _load("codecs.npz")


@pytest.fixture(scope="module")
def c0():
    g = _load("config0.npz")
    q, k, v = make_qkv(1, 2, 1024, 128, seed=0)
    assert digest(q, k, v) == str(g["inputs_digest"]), "regenerated inputs differ from the fixture's"
    return g, q.reshape(2, 1024, 128), k.reshape(2, 1024, 128), v.reshape(2, 1024, 128)


def test_e4m3_encode_matches_reference(codecs):
    assert np.array_equal(O.e4m3_encode(codecs["e4m3_x"]), codecs["e4m3_codes"])


def test_e4m3_known_bytes():
    # test_quant.py:43-46 of the reference
    known = {1.0: 56, 2.0: 64, 0.5: 48, 4.0: 72, 256.0: 120, 448.0: 126, 0.0: 0}
    for val, byte in known.items():
        assert int(O.e4m3_encode(np.array([val], np.float32))[0]) == byte


def test_e4m3_roundtrip_bound(codecs):
    x = codecs["e4m3_x"]
    d = O.e4m3_decode(O.e4m3_encode(x))
    normal = np.abs(x) >= 2.0 ** -6
    normal &= np.abs(x) <= 448.0
    rel = np.abs(d - x)[normal] / np.abs(x)[normal]
    assert rel.max() <= 2.0 ** -4 + 1e-6


def test_fp4_encode_matches_reference(codecs):
    assert np.array_equal(O.fp4_encode(codecs["fp4_x"]), codecs["fp4_codes"])


def test_fp4_ties_to_even():
    ties = {0.25: 0.0, 0.75: 1.0, 1.25: 1.0, 1.75: 2.0, 2.5: 2.0, 3.5: 4.0, 5.0: 4.0}
    for t, want in ties.items():
        assert float(O.fp4_decode(O.fp4_encode(np.array([t], np.float32)))[0]) == want


def test_nvfp4_matches_reference(codecs):
    c, m, g = O.quantize_nvfp4(codecs["nv_x"].reshape(-1))
    assert np.array_equal(c, codecs["nv_codes"])
    assert np.array_equal(m, codecs["nv_micro"])
    assert np.float32(g) == codecs["nv_g"]


def test_expcast_matches_reference(codecs):
    got = O.expcast_codes(codecs["ec_s"], codecs["ec_m"])
    assert np.array_equal(got, codecs["ec_codes"])
    # row maximum lands on byte 120 = 2^8 (test_quant.py:130-132)
    assert np.all(got.max(axis=1) == 120)


def test_fwht_matches_reference(codecs):
    assert np.array_equal(O.fwht(codecs["fw_x"]), codecs["fw_out"])


def test_linspace_matches_torch(codecs):
    sizes = [(1024, 64), (16384, 256), (1000, 32), (65536, 4096), (777, 100), (65536, 256),
             (16384, 4096), (4096, 256), (200, 64), (5, 5)]
    off = 0
    for (n, m), sz in zip(sizes, codecs["lin_sizes"]):
        got = np.round(O.linspace_f32(0, n - 1, m)).astype(np.int64)
        assert np.array_equal(got, codecs["lin_idx"][off:off + sz]), (n, m)
        off += sz


def test_kmeans_steps_match_reference(c0):
    g, q, k, v = c0
    kk = int(g["k"])
    assert kk == 16
    assert np.array_equal(O.seed_centroids(v, kk), g["seeds"])
    assert np.array_equal(O.assign(v, g["seeds"]), g["lab0"])
    assert np.array_equal(O.update_centroids(v, g["lab0"], kk), g["cent1"])


def test_build_permutation_matches_reference(c0):
    g, q, k, v = c0
    perm, cent, kk, labels = O.build_permutation(v, block_rows=64, iters=10)
    assert kk == int(g["k"])
    assert np.array_equal(perm, g["perm"])
    assert np.array_equal(cent, g["centroids"])
    assert np.array_equal(labels, g["labels"])


def test_build_permutation_k64_matches_reference():
    g = _load("kmeans64.npz")
    q, k, v = make_qkv(1, 2, 4096, 128, seed=1)
    assert digest(q, k, v) == str(g["inputs_digest"])
    perm, cent, kk, _ = O.build_permutation(v.reshape(2, 4096, 128), block_rows=64, iters=3,
                                            max_clusters=64)
    assert kk == int(g["k"]) == 64
    assert np.array_equal(perm, g["perm"])
    assert np.array_equal(cent, g["centroids"])


def _check_prepare(prep, g, G):
    for f, gf in [("q", "q8"), ("k", "k8"), ("v", "v8"), ("q_scale", "qs"), ("v_scale", "vs")]:
        assert np.array_equal(prep[f], g[gf].reshape(prep[f].shape)), f
    # k_scale: amax of (K - token mean); the reference's mean is a cascade sum
    ks_ulps = _ulps(prep["k_scale"], g["ks"].reshape(prep["k_scale"].shape))
    assert ks_ulps.max() <= 8, ks_ulps.max()
    # mu = block mean / v_scale: compare the restored block mean in absolute terms
    vs = prep["v_scale"]
    mean_ref = g["mu"].reshape(prep["mu"].shape) * vs
    mean_got = prep["mu"] * vs
    assert np.abs(mean_ref - mean_got).max() <= 1e-6 * max(1.0, float(np.abs(mean_ref).max()))


def test_prepare_matches_reference(c0):
    g, q, k, v = c0
    prep = O.prepare(q, k, v, g["perm"], block_rows=64)
    _check_prepare(prep, g, 2)


def test_prepare_ragged_matches_reference():
    g = _load("ragged.npz")
    q, k, v = make_qkv(1, 2, 200, 128, seed=2)
    assert digest(q, k, v) == str(g["inputs_digest"])
    prep = O.prepare(q.reshape(2, 200, 128), k.reshape(2, 200, 128), v.reshape(2, 200, 128),
                     g["perm"], block_rows=128)
    assert prep["n_pad"] == 256
    _check_prepare(prep, g, 2)
    # padding rows carry zero codes and zero scales
    assert not prep["q"][:, 200:].any() and not prep["q_scale"][:, 200:].any()
    out = O.attention_reference(q.reshape(2, 200, 128), k.reshape(2, 200, 128),
                                v.reshape(2, 200, 128), g["perm"], block_rows=128, block_m=64)
    assert O.rel_l2(out, g["out"].reshape(out.shape)) <= 1e-4


def test_attention_oracles_match_reference(c0):
    g, q, k, v = c0
    ref = g["out_plain"].reshape(q.shape)
    ref_ec = g["out_expcast"].reshape(q.shape)
    out = O.attention_reference(q, k, v, g["perm"], block_rows=64, block_m=128)
    assert O.rel_l2(out, ref) <= 2e-4
    out_ec = O.attention_reference(q, k, v, g["perm"], block_rows=64, block_m=128, expcast=True)
    assert O.rel_l2(out_ec, ref_ec) <= 2e-4
    prep = O.prepare(q, k, v, g["perm"], block_rows=64)
    codes = O.attention_codes(prep, 1024, 64, 128, 128 ** -0.5)
    assert O.rel_l2(codes, ref) <= 2e-3
    sd = O.sdpa_f32(q, k, v)
    assert abs(O.psnr(codes, sd) - O.psnr(ref, sd)) <= 0.3


def test_route_stats_close_to_reference():
    """The reference's routing statistics come from its bf16 fast prepare; the
    oracle's from the fp32 portable prepare, so they agree to bf16 precision."""
    g = _load("route.npz")
    q, k, v = make_qkv(1, 2, 1024, 128, seed=3, spatial=(4, 16, 16))
    assert digest(q, k, v) == str(g["inputs_digest"])
    prep = O.prepare(q.reshape(2, 1024, 128), k.reshape(2, 1024, 128), v.reshape(2, 1024, 128),
                     g["perm"], block_rows=128)
    st = O.route_stats(prep, 128, 64, 1.3, 128 ** -0.5)
    km_ref = g["k_mean"].reshape(st["k_mean"].shape)
    assert O.rel_l2(st["k_mean"], km_ref) <= 5e-2   # block means of bf16 values, with cancellation
    vm_ref = g["v_mean"].reshape(st["v_mean"].shape)
    assert O.rel_l2(st["v_mean"], vm_ref) <= 1e-2
    th_ref = g["thresh"].reshape(st["thresh"].shape)
    assert np.abs(st["thresh"] - th_ref).max() <= 0.05 * max(1.0, float(np.abs(th_ref).max()))


def test_sparse_oracle_keep_all_equals_dense(c0):
    """All blocks kept -> the sparse algorithm is the dense one (probe33 gate)."""
    g, q, k, v = c0
    prep = O.prepare(q, k, v, g["perm"], block_rows=64)
    st = O.route_stats(prep, 64, 64, 1.3, 128 ** -0.5)
    keep = np.ones((2, 1024 // 64, 1024 // 64), bool)
    dense = O.attention_codes(prep, 1024, 64, 64, 128 ** -0.5)
    sparse = O.attention_sparse_codes(prep, st, keep, 1024, 64, 64, 128 ** -0.5)
    assert np.array_equal(dense, sparse)


def test_attention_codes_nvfp4_close_to_float64():
    """The NVFP4-QK restatement equals a float64 evaluation of the same
    definition (dequantised NVFP4 Q/K, FP8 P and V) to fp32 rounding, and
    stays close to exact attention on small inputs."""
    import numpy as np
    from oracle.inputs import make_qkv
    q, k, v = make_qkv(1, 1, 256, 128, seed=3)
    perm = np.arange(256, dtype=np.int32)[None]
    prep = O.prepare(q.reshape(1, 256, 128), k.reshape(1, 256, 128), v.reshape(1, 256, 128), perm, block_rows=128)
    out = O.attention_codes_nvfp4(prep, 256, 128, 128, 128 ** -0.5)
    fp8 = O.attention_codes(prep, 256, 128, 128, 128 ** -0.5)
    sd = O.sdpa_f32(q.reshape(1, 256, 128), k.reshape(1, 256, 128), v.reshape(1, 256, 128))
    assert np.isfinite(out).all()
    assert O.rel_l2(out, sd) < 0.1
    assert O.rel_l2(out, fp8) < 0.1
    assert O.psnr(out, sd) > 20.0


# ---------------------------------------------------------------------------
# Routing mask and sparse output against the reference's own code
# (tests/golden/sparse_ref.npz, written by make_golden.py --only sparse)
# ---------------------------------------------------------------------------
SPARSE_CASES = {"s2k": (2, 2048, (8, 16, 16), 5), "s4k": (4, 4096, (16, 16, 16), 6)}
# A routing decision may differ from the reference's only at a tie: the
# reference sums the per-row proxies and the statistics in fp32 (torch's
# order), the oracle rounds each sum once.  Measured: the scores agree to
# 3.4e-5 and the thresholds to 2.4e-7 (max |score| 2.6).  Against _prepare_fast
# (bf16 Hadamard and divide) they agree to 6.1e-3 and 3.1e-3.
TIE_PREP = 2e-4       # |score - thresh| of a disagreement, portable-prepare routing
TIE_FAST = 2e-2       # the same against the bf16 fast-prepare routing


@pytest.fixture(scope="module")
def sparse_ref():
    return _load("sparse_ref.npz")


def sparse_case(g, name):
    h, n, grid, seed = SPARSE_CASES[name]
    q, k, v = make_qkv(1, h, n, 128, seed=seed, spatial=grid)
    assert digest(q, k, v) == str(g[f"{name}_digest"]), "regenerated inputs differ from the fixture's"
    return q.reshape(h, n, 128), k.reshape(h, n, 128), v.reshape(h, n, 128)


def mask_agreement(keep, g, name, tag, tie):
    """Fraction of routing decisions equal to the reference's; every
    disagreement must sit within ``tie`` of the reference's threshold."""
    kr = g[f"{name}_keep_{tag}"].astype(bool)
    sr = g[f"{name}_score_{tag}"]
    tr = g[f"{name}_thresh_{tag}"]
    keep = np.asarray(keep, bool).reshape(kr.shape)
    dis = np.argwhere(keep != kr)
    margins = [float(sr[a, i, j] - tr[a, i]) for a, i, j in dis]
    assert all(abs(m) <= tie for m in margins), f"{name}/{tag}: non-tie disagreements {margins}"
    return float((keep == kr).mean()), margins


@pytest.mark.parametrize("name", list(SPARSE_CASES))
def test_route_mask_matches_reference_routing(sparse_ref, name):
    """The oracle's mask (the GPU's, bit for bit) against the reference's
    routing rule (triton_attn.py:449-459) run by the reference's own torch code
    on the portable prepare's codes, and on _prepare_fast's."""
    q, k, v = sparse_case(sparse_ref, name)
    n = q.shape[1]
    prep = O.prepare(q, k, v, sparse_ref[f"{name}_perm"], block_rows=128)
    st = O.route_stats(prep, 128, 64, 1.3, 128 ** -0.5)
    keep, _ = O.route_mask(prep, st, n, 128, 64, 128 ** -0.5)
    agree, _ = mask_agreement(keep, sparse_ref, name, "prep", TIE_PREP)
    assert agree >= 0.999
    agree_f, _ = mask_agreement(keep, sparse_ref, name, "fast", TIE_FAST)
    assert agree_f >= 0.999
    assert 0.05 < keep.mean() < 0.6     # routing is non-trivial on these inputs


def test_sparse_oracle_matches_reference_simulation(sparse_ref):
    """The oracle's sparse-kernel arithmetic against simulate() of the
    reference's tests/_probe35_phase3.py:45-114 (its ground truth for the
    fused sparse kernel): rel-L2 within the probe's own 5e-2 gate, and PSNR
    against fp32 SDPA within 0.3 dB of the simulation's."""
    q, k, v = sparse_case(sparse_ref, "s2k")
    n = q.shape[1]
    prep = O.prepare(q, k, v, sparse_ref["s2k_perm"], block_rows=128)
    st = O.route_stats(prep, 128, 64, 1.3, 128 ** -0.5)
    keep, _ = O.route_mask(prep, st, n, 128, 64, 128 ** -0.5)
    out = O.attention_sparse_codes(prep, st, keep, n, 128, 64, 128 ** -0.5)
    sim = sparse_ref["s2k_sim_out"].astype(np.float32).reshape(out.shape)
    assert O.rel_l2(out, sim) <= 5e-2
    sd = O.sdpa_f32(q, k, v)
    assert abs(O.psnr(out, sd) - float(sparse_ref["s2k_sim_psnr"])) <= 0.3


# ---------------------------------------------------------------------------
# Key padding (valid_len) against the reference (tests/golden/masked.npz)
# ---------------------------------------------------------------------------

def test_masked_attention_oracle_matches_reference():
    """reference.py's valid_len: keys at permuted positions >= valid_len take
    no part; the permutation (build_permutation(valid_len=...)) has sorted the
    padding rows to the tail.  The oracle's permutation with the same pad key
    and its attention both match the reference."""
    g = _load("masked.npz")
    h, n, d = 2, 1024, 128
    q, k, v = make_qkv(1, h, n, d, seed=9)
    assert digest(q, k, v) == str(g["digest"])
    vl = int(g["valid_len"])
    qg, kg, vg = (a.reshape(h, n, d) for a in (q, k, v))
    perm, _, _, _ = O.build_permutation(vg, block_rows=128, iters=3, valid_len=vl)
    assert np.array_equal(perm, g["perm"])
    assert (g["perm"][:, vl:] >= vl).all()          # padding rows sit at the tail
    for name, ec in (("plain", False), ("expcast", True)):
        out = O.attention_reference(qg, kg, vg, g["perm"], block_rows=128, block_m=64, expcast=ec, valid_len=vl)
        assert O.rel_l2(out, g[f"out_{name}"].reshape(out.shape)) <= 2e-4
    prep = O.prepare(qg, kg, vg, g["perm"], block_rows=128)
    codes = O.attention_codes(prep, n, 128, 64, d ** -0.5, kv_len=[vl, vl])
    assert O.rel_l2(codes, g["out_plain"].reshape(codes.shape)) <= 2e-3
