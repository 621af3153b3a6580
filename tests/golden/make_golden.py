"""Generate the golden vectors that pin the oracle to the reference.

Run once, where the reference package is importable (read-only source tree):

    python tests/golden/make_golden.py [--reference PATH] [--only base,sparse,nvfp4,masked]

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
    ap.add_argument("--only", default="",
                    help="comma-separated fixture groups to (re)write: base, sparse, nvfp4, masked (default all)")
    args = ap.parse_args()
    only = set(filter(None, args.only.split(",")))
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

    if not only or "sparse" in only:
        make_sparse(args.reference)
    if not only or "nvfp4" in only:
        make_nvfp4()
    if not only or "masked" in only:
        make_masked()
    if only and "base" not in only:
        return _report()

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

    return _report()


def _report() -> int:
    print("golden vectors written to", HERE)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f"  {f}: {os.path.getsize(os.path.join(HERE, f)) / 1024:.0f} KiB")
    return 0


def _psnr(out, ref) -> float:
    """PSNR of the reference's benchmark (tests/bench_attention.py:55-57)."""
    import torch
    mse = ((out.float() - ref.float()) ** 2).mean()
    return float(10 * torch.log10(ref.float().pow(2).max() / mse.clamp(min=1e-30)))


def _kernel_route(q8, qs, k_mean, thresh, n, block_rows, q_block, scale, local=1, sink=0):
    """The routing decision of the reference's sparse kernel
    (kernels/triton_attn.py:449-459), evaluated with the kernel's operand
    precisions: proxy = dot(bf16(q8), bf16(k_mean)) * (qs * sm_scale) per query
    row, its mean over the q_block rows against the block's threshold, plus the
    local window and the sink blocks.
    q8 (G, NP, D) float8_e4m3fn; qs (G, NP); k_mean (G, NB, D); thresh (G, NQB).
    -> (keep bool (G, NQB, NB), score (G, NQB, NB) fp32)."""
    import torch
    g, n_pad, d = q8.shape
    nb = n_pad // block_rows
    nqb = n_pad // q_block
    qb = q8.to(torch.bfloat16).float()
    kc = k_mean.to(torch.bfloat16).float()
    proxy = torch.bmm(qb, kc.transpose(1, 2)) * (qs.float() * scale).unsqueeze(-1)   # (G, NP, NB)
    score = proxy.reshape(g, nqb, q_block, nb).sum(dim=2) / q_block
    qi = torch.arange(nqb)[:, None]
    kj = torch.arange(nb)[None, :]
    qb_kv = (qi * q_block) // block_rows
    keep = (score > thresh.reshape(g, nqb, 1)) | ((qb_kv - kj).abs() <= local)[None] | (kj < sink)[None]
    return keep, score


def _load_simulate(reference: str):
    """``simulate`` (and its helper ``dq_fp8``) of the reference's
    tests/_probe35_phase3.py, lifted out with ``ast`` so that the probe's own
    imports (ComfyUI, comfy_kitchen, a GPU) are never executed."""
    import ast

    import torch
    from vc_attention import quant as Q
    from vc_attention.kernels import triton_attn as T

    path = os.path.join(reference, "tests", "_probe35_phase3.py")
    tree = ast.parse(open(path).read(), filename=path)
    keep = [node for node in tree.body
            if isinstance(node, ast.FunctionDef) and node.name in ("simulate", "dq_fp8")]
    keep += [node for node in tree.body if isinstance(node, ast.Assign)
             and any(isinstance(t, ast.Tuple) and any(getattr(e, "id", "") == "BN" for e in t.elts)
                     for t in node.targets)]
    mod = ast.Module(body=keep, type_ignores=[])
    ns = {"torch": torch, "Q": Q, "T": T}
    exec(compile(mod, path, "exec"), ns)
    assert ns["BN"] == 128 and ns["QB"] == 64
    return ns["simulate"]


def make_sparse(reference: str) -> None:
    """sparse_ref.npz: the reference's own routing decisions and its own
    sparse-attention simulation on configs[2]-style inputs (spatial grid,
    V-Smooth k-means perm with block_rows 128, q_block 64, tau 1.3).

    Per case c:
      c_perm                 reference build_permutation (iters=3) perm
      c_keep_prep / _score_prep / _thresh_prep
          the kernel rule of triton_attn.py:449-459 applied to the portable
          prepare()'s Q codes and scales (:504-579) and to routing statistics
          computed by the formula of :716-735 from the same fp32 rotated Q/K
      c_keep_fast / _score_fast / _thresh_fast
          the same rule on _prepare_fast's outputs (:640-754: bf16 Hadamard,
          bf16 divide), i.e. the routing the reference's GPU path takes
      c_sim_out (fp16), c_sim_keep, c_sim_psnr
          simulate() of tests/_probe35_phase3.py:45-114 (the reference's ground
          truth for its sparse kernel) and its PSNR against fp32 SDPA
      c_dense_psnr           vc_attention_reference (fp8, ExpCast off) PSNR
    """
    import torch
    from vc_attention.grouping import GroupingConfig, build_permutation
    from vc_attention.hadamard import fwht
    from vc_attention.kernels.reference import RefConfig, vc_attention_reference
    from vc_attention.kernels.triton_attn import _prepare_fast, prepare

    simulate = _load_simulate(reference)
    D, BR, QB, TAU = 128, 128, 64, 1.3
    sc = D ** -0.5
    cases = {"s2k": (2, 2048, (8, 16, 16), 5, True), "s4k": (4, 4096, (16, 16, 16), 6, False)}
    out = {}
    for name, (H, n, grid, seed, with_sim) in cases.items():
        q, k, v = make_qkv(1, H, n, D, seed=seed, spatial=grid)
        qt, kt, vt = (torch.from_numpy(a).to(torch.bfloat16) for a in (q, k, v))
        G = H
        perm = build_permutation(vt.reshape(G, n, D), GroupingConfig(block_rows=BR, iters=3)).perm
        # portable prepare + the routing formula on its fp32 rotated tensors
        prep = prepare(qt, kt, vt, perm, block_rows=BR)
        qf = qt.reshape(G, n, D).float()
        kf = kt.reshape(G, n, D).float().gather(1, perm.to(torch.int64).unsqueeze(-1).expand(G, n, D))
        q_t, k_t = fwht(qf), fwht(kf)
        k_t = k_t - k_t.mean(dim=1, keepdim=True)
        nb, nqb = n // BR, n // QB
        k_mean = k_t.reshape(G, nb, BR, D).mean(dim=2)
        q_cent = q_t.reshape(G, nqb, QB, D).mean(dim=2)
        proxy = torch.matmul(q_cent, k_mean.transpose(-1, -2)) * sc
        thr = (proxy.mean(dim=-1, keepdim=True)
               + TAU * proxy.std(dim=-1, keepdim=True, unbiased=False)).reshape(G, nqb)
        keep_p, score_p = _kernel_route(prep.q.reshape(G, n, D), prep.q_scale.reshape(G, n), k_mean, thr,
                                        n, BR, QB, sc)
        # the GPU path of the reference: _prepare_fast
        pf = _prepare_fast(qt, kt, vt, perm, block_rows=BR, hadamard=True, smooth_k=True, sparse=True,
                           tau=TAU, q_block=QB, scale=sc)
        keep_f, score_f = _kernel_route(pf.q.reshape(G, n, D), pf.q_scale.reshape(G, n),
                                        pf.k_mean.reshape(G, nb, D), pf.thresh.reshape(G, nqb), n, BR, QB, sc)
        out.update({f"{name}_digest": np.array(digest(q, k, v)), f"{name}_perm": perm.numpy(),
                    f"{name}_keep_prep": keep_p.numpy(), f"{name}_score_prep": score_p.numpy(),
                    f"{name}_thresh_prep": thr.numpy(),
                    f"{name}_keep_fast": keep_f.numpy(), f"{name}_score_fast": score_f.numpy(),
                    f"{name}_thresh_fast": pf.thresh.reshape(G, nqb).numpy()})
        agree = float((keep_p == keep_f).float().mean())
        print(f"  {name}: keep(prep) {float(keep_p.float().mean()):.4f}  keep(fast) "
              f"{float(keep_f.float().mean()):.4f}  agreement {agree:.4f}")
        if with_sim:
            sim, ratio = simulate(qt.float(), kt.float(), vt.float(), perm, TAU, sc)
            sd = torch.nn.functional.scaled_dot_product_attention(qt.float(), kt.float(), vt.float())
            dense = vc_attention_reference(qt.float(), kt.float(), vt.float(),
                                           RefConfig(backend="fp8", block_rows=BR, block_m=QB,
                                                     enable_vsmooth=True), perm=perm)
            out.update({f"{name}_sim_out": sim.numpy().astype(np.float16),
                        f"{name}_sim_keep": np.float32(ratio),
                        f"{name}_sim_psnr": np.float32(_psnr(sim, sd)),
                        f"{name}_dense_psnr": np.float32(_psnr(dense, sd))})
            print(f"  {name}: simulate keep {ratio:.4f}  PSNR sim {_psnr(sim, sd):.2f} dB  "
                  f"dense {_psnr(dense, sd):.2f} dB")
    np.savez_compressed(os.path.join(HERE, "sparse_ref.npz"), **out)


def make_nvfp4() -> None:
    """nvfp4_ref.npz: the reference's own nvfp4 backend
    (kernels/reference.py:112-116, 135-152: Q/K, V and P quantised to NVFP4
    with per-16-token microscales) and its fp8 backend on the same seeded
    configs[3]-distributed inputs, with their PSNRs against fp32 SDPA."""
    import torch
    from vc_attention.grouping import GroupingConfig, build_permutation
    from vc_attention.kernels.reference import RefConfig, vc_attention_reference

    H, n, D, BR = 2, 2048, 128, 128
    q, k, v = make_qkv(1, H, n, D, seed=8)
    qt, kt, vt = (torch.from_numpy(a).to(torch.bfloat16) for a in (q, k, v))
    perm = build_permutation(vt.reshape(H, n, D), GroupingConfig(block_rows=BR, iters=3)).perm
    sd = torch.nn.functional.scaled_dot_product_attention(qt.float(), kt.float(), vt.float())
    res = {"digest": np.array(digest(q, k, v)), "perm": perm.numpy()}
    for backend in ("nvfp4", "fp8"):
        o = vc_attention_reference(qt.float(), kt.float(), vt.float(),
                                   RefConfig(backend=backend, block_rows=BR, block_m=64, enable_vsmooth=True),
                                   perm=perm)
        res[f"{backend}_out"] = o.numpy().astype(np.float16)
        res[f"{backend}_psnr"] = np.float32(_psnr(o, sd))
        print(f"  reference backend {backend}: PSNR {_psnr(o, sd):.2f} dB")
    np.savez_compressed(os.path.join(HERE, "nvfp4_ref.npz"), **res)



def make_masked() -> None:
    """masked.npz: key padding as the reference defines it.  build_permutation
    with valid_len (grouping.py:150-186: padding rows get the pad key and sort
    to the tail) and vc_attention_reference with the same valid_len
    (reference.py:162-294: keys at permuted positions >= valid_len masked),
    plain and ExpCast, with their PSNR against fp32 SDPA whose boolean mask
    drops the same keys (tokens >= valid_len in the original order)."""
    import torch
    from vc_attention.grouping import GroupingConfig, build_permutation
    from vc_attention.kernels.reference import RefConfig, vc_attention_reference

    H, n, D, BR, VL = 2, 1024, 128, 128, 800
    q, k, v = make_qkv(1, H, n, D, seed=9)
    qt, kt, vt = (torch.from_numpy(a).to(torch.bfloat16) for a in (q, k, v))
    perm = build_permutation(vt.reshape(H, n, D), GroupingConfig(block_rows=BR, iters=3), valid_len=VL).perm
    keep = torch.arange(n) < VL
    sd = torch.nn.functional.scaled_dot_product_attention(qt.float(), kt.float(), vt.float(),
                                                          attn_mask=keep[None, None, None, :])
    res = {"digest": np.array(digest(q, k, v)), "perm": perm.numpy(), "valid_len": np.int32(VL)}
    for name, ec in (("plain", False), ("expcast", True)):
        o = vc_attention_reference(qt.float(), kt.float(), vt.float(),
                                   RefConfig(backend="fp8", block_rows=BR, block_m=64, enable_vsmooth=True,
                                             enable_expcast=ec), perm=perm, valid_len=VL)
        res[f"out_{name}"] = o.numpy()
        res[f"psnr_{name}"] = np.float32(_psnr(o, sd))
        print(f"  masked reference ({name}): PSNR {_psnr(o, sd):.2f} dB vs masked SDPA")
    np.savez_compressed(os.path.join(HERE, "masked.npz"), **res)

if __name__ == "__main__":
    sys.exit(main())