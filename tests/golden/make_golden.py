"""Generate the golden vectors that pin the oracle to the reference.

Run once, where the reference package is importable (read-only source tree):

    python tests/golden/make_golden.py [--reference PATH]

It imports bingling360/comfyui_vc_attention (``vc_attention``), runs the
reference's own functions on seeded inputs from ``oracle/inputs.py`` and writes
``tests/golden/*.npz``.  Inputs are not stored; each fixture stores a digest of
them and the tests regenerate and check it.  Nothing at test time reads the
reference tree.
"""

from __future__ import annotations

import argparse
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.inputs import digest, make_qkv  # noqa: E402


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VC_REFERENCE", "/root/reference"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    from vc_attention import quant as Q
    from vc_attention.expcast import expcast_codes, standard_codes
    from vc_attention.grouping import (GroupingConfig, _assign, _seed_centroids,
                                       _update_centroids, build_permutation)
    from vc_attention.hadamard import fwht
    from vc_attention.kernels.reference import RefConfig, vc_attention_reference
    from vc_attention.kernels.triton_attn import _prepare_fast, prepare

    torch.set_num_threads(max(1, os.cpu_count() or 1))

    # ---------------- codecs, fwht, linspace ----------------
    g = torch.Generator().manual_seed(0)
    specials = torch.tensor(
        [0.0, -0.0, 1.0, 2.0, 0.5, 4.0, 256.0, 448.0, 449.0, 464.0, 480.0, 1000.0, -448.0,
         2 ** -6, 2 ** -7, 2 ** -9, 2 ** -10, 3 * 2 ** -10, 1.0625, 1.1875, -1.0625, 432.0,
         -1e-5, 1e-5, 5 * 2 ** -11, 7 * 2 ** -11], dtype=torch.float32)
    x = torch.cat([specials, torch.randn(20000, generator=g) * 3.0,
                   torch.randn(5000, generator=g) * 1e-3])
    fp4x = torch.cat([torch.tensor([0.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 7.0,
                                    -0.25, -0.75, -5.0, 0.1, -0.1]),
                      torch.randn(5000, generator=g) * 2.0])
    nv = torch.randn(4, 256, generator=g) * 0.7
    nv_codes, nv_micro, nv_g = Q.quantize_nvfp4(nv.reshape(-1), block=16)
    qq = torch.randn(128, 128, generator=g)
    kk = torch.randn(512, 128, generator=g)
    s = (qq @ kk.T) / (128 ** 0.5)
    m = s.amax(dim=-1)
    fw = torch.randn(64, 128, generator=g) * 2.0
    lin = []
    for n_, m_ in [(1024, 64), (16384, 256), (1000, 32), (65536, 4096), (777, 100),
                   (65536, 256), (16384, 4096), (4096, 256), (200, 64), (5, 5)]:
        lin.append(torch.linspace(0, n_ - 1, m_).round().long().numpy())
    np.savez_compressed(
        os.path.join(HERE, "codecs.npz"),
        e4m3_x=x.numpy(), e4m3_codes=Q.e4m3_encode(x).numpy(),
        fp4_x=fp4x.numpy(), fp4_codes=Q.fp4_encode(fp4x).numpy(),
        nv_x=nv.numpy(), nv_codes=nv_codes.numpy(), nv_micro=nv_micro.numpy().reshape(-1),
        nv_g=np.float32(nv_g),
        ec_s=s.numpy(), ec_m=m.numpy(), ec_codes=expcast_codes(s, m).numpy(),
        ec_std=standard_codes(s, m).numpy(),
        fw_x=fw.numpy(), fw_out=fwht(fw).numpy(),
        lin_idx=np.concatenate(lin), lin_sizes=np.array([len(a) for a in lin]),
    )

    # ---------------- k-means, prepare, attention ----------------
    B, H, N, D = 1, 2, 1024, 128
    q, k, v = make_qkv(B, H, N, D, seed=0)
    qt, kt, vt = (torch.from_numpy(a).to(torch.bfloat16) for a in (q, k, v))
    G = B * H
    gcfg = GroupingConfig(block_rows=64, iters=10)
    v_b = vt.reshape(G, N, D)
    res = build_permutation(v_b, gcfg)
    kk_ = res.k
    seeds = _seed_centroids(v_b, kk_, gcfg)
    lab0 = _assign(v_b, seeds, gcfg)
    cent1 = _update_centroids(v_b, lab0, kk_, gcfg)
    lab_final = _assign(v_b, res.centroids, gcfg)
    perm = res.perm
    prep = prepare(qt, kt, vt, perm, block_rows=64)
    ref_plain = vc_attention_reference(
        qt.float(), kt.float(), vt.float(),
        RefConfig(backend="fp8", block_rows=64, block_m=128, enable_vsmooth=True,
                  enable_expcast=False), perm=perm)
    ref_ec = vc_attention_reference(
        qt.float(), kt.float(), vt.float(),
        RefConfig(backend="fp8", block_rows=64, block_m=128, enable_vsmooth=True,
                  enable_expcast=True), perm=perm)
    np.savez_compressed(
        os.path.join(HERE, "config0.npz"),
        inputs_digest=np.array(digest(q, k, v)), k=np.int32(kk_),
        seeds=seeds.float().numpy(), lab0=lab0.numpy(), cent1=cent1.float().numpy(),
        centroids=res.centroids.float().numpy(), labels=lab_final.numpy(),
        perm=perm.numpy(),
        q8=prep.q.view(torch.uint8).numpy(), qs=prep.q_scale.numpy(),
        k8=prep.k.view(torch.uint8).numpy(), ks=prep.k_scale.numpy(),
        v8=prep.v.view(torch.uint8).numpy(), vs=prep.v_scale.numpy(), mu=prep.mu.numpy(),
        out_plain=ref_plain.numpy(), out_expcast=ref_ec.numpy(),
    )

    # ---------------- k=64 grouping (configs[1] semantics, smaller N) ----------------
    q2, k2, v2 = make_qkv(1, 2, 4096, D, seed=1)
    v2b = torch.from_numpy(v2).to(torch.bfloat16).reshape(2, 4096, D)
    res2 = build_permutation(v2b, GroupingConfig(block_rows=64, iters=3, max_clusters=64))
    np.savez_compressed(
        os.path.join(HERE, "kmeans64.npz"),
        inputs_digest=np.array(digest(q2, k2, v2)), k=np.int32(res2.k),
        perm=res2.perm.numpy(), centroids=res2.centroids.float().numpy())

    # ---------------- ragged prepare (N not a multiple of block_rows) ----------------
    q3, k3, v3 = make_qkv(1, 2, 200, D, seed=2)
    q3t, k3t, v3t = (torch.from_numpy(a).to(torch.bfloat16) for a in (q3, k3, v3))
    perm3 = torch.stack([torch.randperm(200, generator=torch.Generator().manual_seed(7 + i))
                         for i in range(2)]).to(torch.int32)
    p3 = prepare(q3t, k3t, v3t, perm3, block_rows=128)
    ref3 = vc_attention_reference(
        q3t.float(), k3t.float(), v3t.float(),
        RefConfig(backend="fp8", block_rows=128, block_m=64, enable_vsmooth=True), perm=perm3)
    np.savez_compressed(
        os.path.join(HERE, "ragged.npz"),
        inputs_digest=np.array(digest(q3, k3, v3)), perm=perm3.numpy(),
        q8=p3.q.view(torch.uint8).numpy(), qs=p3.q_scale.numpy(),
        k8=p3.k.view(torch.uint8).numpy(), ks=p3.k_scale.numpy(),
        v8=p3.v.view(torch.uint8).numpy(), vs=p3.v_scale.numpy(), mu=p3.mu.numpy(),
        out=ref3.numpy())

    # ---------------- routing statistics (configs[2] semantics, small grid) ----------------
    q4, k4, v4 = make_qkv(1, 2, 1024, D, seed=3, spatial=(4, 16, 16))
    q4t, k4t, v4t = (torch.from_numpy(a).to(torch.bfloat16) for a in (q4, k4, v4))
    perm4 = build_permutation(v4t.reshape(2, 1024, D), GroupingConfig(block_rows=128, iters=3)).perm
    pf = _prepare_fast(q4t, k4t, v4t, perm4, block_rows=128, hadamard=True, smooth_k=True,
                       sparse=True, tau=1.3, q_block=64, scale=D ** -0.5)
    np.savez_compressed(
        os.path.join(HERE, "route.npz"),
        inputs_digest=np.array(digest(q4, k4, v4)), perm=perm4.numpy(),
        k_mean=pf.k_mean.numpy(), v_mean=pf.v_mean.numpy(), thresh=pf.thresh.numpy())

    print("golden vectors written to", HERE)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f"  {f}: {os.path.getsize(os.path.join(HERE, f)) / 1024:.0f} KiB")
    return 0


if __name__ == "__main__":
    sys.exit(main())
