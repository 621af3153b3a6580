"""Time the reference's own CPU code against the numpy port on the same inputs.

Test infrastructure, run only where the reference package is importable (its
source tree is read-only and never travels to a GPU box):

    python oracle/calibrate_reference.py [--reference PATH] [--n 2048] [--reps 2]

The reference is pure Python/PyTorch and ships no build recipe (no setup.py or
pyproject.toml), so it cannot be installed or carried to the GPU box; the
benchmark's CPU arm therefore runs the port (``oracle/vc_oracle.py``).  This
script measures, on one head at configs[1]'s distributions, the reference's
``build_permutation`` (grouping.py:150) + ``vc_attention_reference``
(kernels/reference.py:162, backend fp8, V-Smooth, ExpCast) with torch using
every host core, and the port's ``build_permutation`` + ``attention_reference``
on the same seeded inputs.  It writes ``oracle/reference_cpu_calibration.json``;
``bench.py --impl reference`` reports that file beside its own timing so the
port's number can be read against the reference's own code.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)

OUT = os.path.join(HERE, "reference_cpu_calibration.json")


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VC_REFERENCE", "/root/reference"))
    ap.add_argument("--n", type=int, default=2048)
    ap.add_argument("--reps", type=int, default=2)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    from vc_attention.grouping import GroupingConfig, build_permutation
    from vc_attention.kernels.reference import RefConfig, vc_attention_reference

    from oracle import vc_oracle as O
    from oracle.inputs import make_qkv

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    N, D, BR, BM = args.n, 128, 128, 64
    q, k, v = make_qkv(1, 1, N, D, seed=0)
    qt, kt, vt = (torch.from_numpy(a).to(torch.bfloat16) for a in (q, k, v))
    cfg = RefConfig(backend="fp8", block_rows=BR, block_m=BM, enable_vsmooth=True, enable_expcast=True)

    def run_ref():
        res = build_permutation(vt.reshape(1, N, D).float(), GroupingConfig(block_rows=BR, iters=3))
        perm = res[0] if isinstance(res, tuple) else getattr(res, "perm", res)
        return vc_attention_reference(qt.float(), kt.float(), vt.float(), cfg, perm=perm.reshape(1, N))

    def run_port():
        perm, _, _, _ = O.build_permutation(v.reshape(1, N, D), block_rows=BR, iters=3)
        return O.attention_reference(q.reshape(1, N, D), k.reshape(1, N, D), v.reshape(1, N, D), perm,
                                     block_rows=BR, block_m=BM, expcast=True)

    def best(fn):
        fn()
        ts = []
        for _ in range(args.reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return min(ts)

    t_ref = best(run_ref)
    t_port = best(run_port)
    rec = {
        "what": "one head, N=%d, D=128, k-means (3 iters) + fp8 VC-Attention with V-Smooth and ExpCast" % N,
        "reference_s": round(t_ref, 4),
        "port_s": round(t_port, 4),
        "reference_over_port": round(t_ref / t_port, 3),
        "cores": cores,
        "torch_threads": torch.get_num_threads(),
        "where": "build container (CPU only), reference imported read-only",
    }
    with open(OUT, "w") as f:
        json.dump(rec, f, indent=1)
        f.write("\n")
    print(json.dumps(rec))
    return 0


if __name__ == "__main__":
    sys.exit(main())
