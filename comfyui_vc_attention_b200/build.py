"""Build libvcattn.so in-tree with nvcc for sm_100a.

    python -m comfyui_vc_attention_b200.build [--force] [--jobs N]

Each ``csrc/*.cu`` compiles to an object under ``_build/`` (in parallel) and
the objects link into ``comfyui_vc_attention_b200/libvcattn.so``.  The library
exports only the C ABI of ``include/vcattn.h``; it does not link against torch.
A source is recompiled when it, or any header, is newer than its object.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(REPO, "_build")
LIB = os.path.join(PKG, "libvcattn.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers_mtime() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src: str, obj: str, extra) -> str:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr}\n{r.stdout}")
    return r.stderr


def build(force: bool = False, jobs: int = 0, verbose: bool = False, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr = _headers_mtime()
    todo = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr):
            todo.append((s, o))
    if todo:
        jobs = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            futs = {ex.submit(_compile, s, o, list(extra)): s for s, o in todo}
            for f in cf.as_completed(futs):
                msg = f.result()
                if verbose and msg.strip():
                    print(f"[{os.path.basename(futs[f])}]\n{msg}", file=sys.stderr)
    if todo or not os.path.exists(LIB):
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", LIB + ".tmp"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}\n{r.stdout}")
        os.replace(LIB + ".tmp", LIB)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_info else []
    print(build(force=args.force or args.ptxas_info, jobs=args.jobs,
                verbose=args.verbose or args.ptxas_info, extra=extra))
    return 0


if __name__ == "__main__":
    sys.exit(main())
