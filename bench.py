#!/usr/bin/env python
"""VC-Attention hot-path benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c1|c3|c2]

Workload (N=1 headline): B=1, H=56, N=16384, D=128 bf16,
dense FP8 VC-Attention with ExpCast, Hadamard and a V-Smooth permutation from
k-means with k=64.  One "step" is one call of the hot path on one batch:
prepare (permute, rotate, smooth, quantise) + the fused attention kernel, the
permutation precomputed (it is cached across layers and steps by the runtime;
its k-means time is reported separately as ``kmeans_ms``).

``value`` = effective TFLOPS over all ranks, 4*B*H*N^2*D per call / time, with
inputs resident in HBM; ``e2e`` = the same through the public entry point with
pinned-host inputs copied in and the output copied back inside the timed
region.  Multi-GPU runs (torchrun, one rank per GPU) split the same job's
(batch, head) units over the ranks (strong scaling: the total work is the
N=1 workload's) and NCCL all-gathers assemble the full output on every rank,
in rounds that overlap the remaining compute; the time is the max over
ranks.  ``--replicas`` instead gives every rank its own full-size copy of
the workload (weak scaling, no collective).

``--impl reference`` times the reference's CPU algorithm (the oracle
restatement of vc_attention_reference, oracle/) on the host cores on a
bounded sample of the same workload (one head x a block of query rows per
step, timed as it runs), and reports beside it the committed timing of the
reference's own code against that restatement on the same inputs
(oracle/reference_cpu_calibration.json).
"""

from __future__ import annotations

import argparse
import math
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ms/call & effective TFLOPS, 56h D=128 at 16K/64K tokens; PSNR vs fp32 SDPA"
UNIT = "TFLOPS (effective, 4*B*H*N^2*D per call)"

WORKLOADS = {
    "c1": dict(desc="configs[1]: dense FP8 VC-Attention, B1 H56 N16384 D128, ExpCast on, Hadamard on, "
                    "V-Smooth k=64", B=1, H=56, N=16384, D=128, expcast=True, sparse=False, k=64,
               block_rows=128, spatial=None),
    "c1h16": dict(desc="profiling slice of configs[1]: B1 H16 N16384 D128, ExpCast on, V-Smooth k=64",
                  B=1, H=16, N=16384, D=128, expcast=True, sparse=False, k=64, block_rows=128,
                  spatial=None),
    "c3": dict(desc="dense FP8 VC-Attention, B1 H56 N65536 D128, ExpCast on, V-Smooth k=512",
               B=1, H=56, N=65536, D=128, expcast=True, sparse=False, k=512, block_rows=128, spatial=None),
    "c3h8": dict(desc="profiling slice of the N=65536 dense shape: B1 H8 N65536 D128, ExpCast on, V-Smooth k=512",
                 B=1, H=8, N=65536, D=128, expcast=True, sparse=False, k=512, block_rows=128, spatial=None),
    "c3nv": dict(desc="configs[3]: NVFP4 QK^T (E2M1, E4M3 per-16 scales, fp32 tensor scale per head) + FP8 PV, "
                      "B1 H56 N65536 D128, ExpCast on, V-Smooth k=512", B=1, H=56, N=65536, D=128, expcast=True,
                 sparse=False, k=512, block_rows=128, spatial=None, qk_fp4=True),
    "c1nv": dict(desc="NVFP4 QK^T + FP8 PV at the configs[1] shape: B1 H56 N16384 D128, ExpCast on, V-Smooth k=64",
                 B=1, H=56, N=16384, D=128, expcast=True, sparse=False, k=64, block_rows=128, spatial=None,
                 qk_fp4=True),
    "c1d64": dict(desc="head dim 64 at the configs[1] width: dense FP8 VC-Attention, B1 H112 N16384 D64, ExpCast on, "
                       "V-Smooth k=64", B=1, H=112, N=16384, D=64, expcast=True, sparse=False, k=64, block_rows=128,
                  spatial=None),
    "c1nvh16": dict(desc="profiling slice of the NVFP4 QK^T path at the configs[1] shape: B1 H16 N16384 D128",
                    B=1, H=16, N=16384, D=128, expcast=True, sparse=False, k=64, block_rows=128, spatial=None,
                    qk_fp4=True),
    "c4": dict(desc="configs[4]: dense FP8 VC-Attention, B2 (CFG pair) H56 N65536 D128, (batch, head) units "
                    "sharded over the ranks, NCCL all-gather of the bf16 output, ExpCast on, V-Smooth k=512",
               B=2, H=56, N=65536, D=128, expcast=True, sparse=False, k=512, block_rows=128, spatial=None,
               sharded=True, cfg_pair=True),
    "c2h16": dict(desc="profiling slice of configs[2]: tau=1.3 block-sparse, B1 H16 N16384 D128, 16x32x32 grid",
                  B=1, H=16, N=16384, D=128, expcast=True, sparse=True, k=64, block_rows=128,
                  spatial=(16, 32, 32), tau=1.3),
    "c2l": dict(desc="configs[2] at N=65536: block-sparse FP8 VC-Attention, tau=1.3, B1 H56 N65536 D128 on a "
                     "64x32x32 grid, ExpCast on, V-Smooth k=512", B=1, H=56, N=65536, D=128, expcast=True,
                sparse=True, k=512, block_rows=128, spatial=(64, 32, 32), tau=1.3),
    "c2b64": dict(desc="configs[2] with 64-key value blocks: block-sparse FP8 VC-Attention, tau=1.3, B1 H56 "
                       "N16384 D128 on a 16x32x32 grid, block_rows 64, ExpCast on, V-Smooth k=64", B=1, H=56,
                  N=16384, D=128, expcast=True, sparse=True, k=64, block_rows=64, spatial=(16, 32, 32), tau=1.3),
    "c2d64": dict(desc="configs[2] with head dim 64 at the same width: block-sparse FP8 VC-Attention, tau=1.3, "
                       "B1 H112 N16384 D64 on a 16x32x32 grid, ExpCast on, V-Smooth k=64", B=1, H=112, N=16384,
                  D=64, expcast=True, sparse=True, k=64, block_rows=128, spatial=(16, 32, 32), tau=1.3),
    "c2": dict(desc="configs[2]: block-sparse FP8 VC-Attention, tau=1.3, B1 H56 N16384 D128 on a 16x32x32 "
                    "grid, ExpCast on, V-Smooth k=64", B=1, H=56, N=16384, D=128, expcast=True, sparse=True,
               k=64, block_rows=128, spatial=(16, 32, 32), tau=1.3),
}


def flops_per_call(w) -> float:
    return 4.0 * w["B"] * w["H"] * float(w["N"]) ** 2 * w["D"]


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            mp = json.load(f)
        return mp, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# --------------------------------------------------------------- clocks ----

class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self._t.join(timeout=2)
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes),
                "reasons": sorted(reasons), "samples": len(sms)}


# ------------------------------------------------------------ GPU inputs ----

def make_inputs_gpu(w, seed, dev):
    """Seeded Q/K/V of the configs' distributions, generated on the device."""
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    G, N, D = w["B"] * w["H"], w["N"], w["D"]
    q = torch.randn((G, N, D), generator=g, device=dev)
    k = torch.randn((G, N, D), generator=g, device=dev) + 2.0 * torch.randn((G, 1, D), generator=g, device=dev)
    cent = torch.randn((G, 64, D), generator=g, device=dev)
    if w.get("spatial"):
        # tokens on a T x Hg x W grid; a smooth positional field
        # (8 separable low-frequency cosines projected to D, RMS 0.5) is shared
        # by Q and K; V's centre is the token's region (4 x 4 x 4 regions)
        t, hg, wd = w["spatial"]
        tt, hh, ww = torch.meshgrid(torch.arange(t, device=dev), torch.arange(hg, device=dev),
                                    torch.arange(wd, device=dev), indexing="ij")
        fr = torch.rand((8, 3), generator=g, device=dev) * 2.0
        ph = torch.rand((8, 3), generator=g, device=dev) * (2 * math.pi)
        feats = torch.stack([torch.cos(math.pi * fr[i, 0] * tt / t + ph[i, 0])
                             * torch.cos(math.pi * fr[i, 1] * hh / hg + ph[i, 1])
                             * torch.cos(math.pi * fr[i, 2] * ww / wd + ph[i, 2]) for i in range(8)], -1)
        pos = feats.reshape(N, 8) @ torch.randn((8, D), generator=g, device=dev)
        pos = pos * (0.5 / pos.pow(2).mean().sqrt().clamp_min(1e-12))
        q = q + pos
        k = k + pos
        reg = ((tt * 4) // t) * 16 + ((hh * 4) // hg) * 4 + (ww * 4) // wd
        lab = (reg.reshape(1, N) % 64).expand(G, N)
    else:
        lab = torch.randint(0, 64, (G, N), generator=g, device=dev)
    v = torch.gather(cent, 1, lab.unsqueeze(-1).expand(G, N, D))
    v = v + 0.3 * torch.randn((G, N, D), generator=g, device=dev)
    if w.get("cfg_pair"):
        # batch 1 = batch 0 + 0.05 N(0, 1)
        half = G // 2
        q[half:] = q[:half] + 0.05 * torch.randn((half, N, D), generator=g, device=dev)
        k[half:] = k[:half] + 0.05 * torch.randn((half, N, D), generator=g, device=dev)
        v[half:] = v[:half] + 0.05 * torch.randn((half, N, D), generator=g, device=dev)
    shape = (w["B"], w["H"], N, D)
    out = [t.to(torch.bfloat16).reshape(shape).contiguous() for t in (q, k, v)]
    del q, k, v, cent, lab
    return out


def psnr_vs_sdpa(out, q, k, v, heads_per_chunk=8):
    import torch
    import torch.nn.functional as F
    num = 0.0
    peak = 0.0
    cnt = 0
    H = q.shape[1]
    for h0 in range(0, H, heads_per_chunk):
        sl = slice(h0, min(H, h0 + heads_per_chunk))
        ref = F.scaled_dot_product_attention(q[:, sl].float(), k[:, sl].float(), v[:, sl].float())
        num += float(((out[:, sl].float() - ref) ** 2).sum())
        peak = max(peak, float((ref ** 2).max()))
        cnt += ref.numel()
        del ref
    import math
    return 10 * math.log10(peak / max(num / cnt, 1e-30))


# --------------------------------------------------------- CPU baseline ----

def cpu_sample(w, q_rows, seed=0):
    """Reference CPU algorithm (oracle restatement of vc_attention_reference,
    with the oracle's k-means permutation) on one head and the first q_rows
    query rows at full N.  Returns (seconds, extrapolated ms per full call)."""
    import numpy as np
    from oracle import vc_oracle as O
    rng = np.random.default_rng(seed)
    N, D = w["N"], w["D"]
    q = O.bf16_round(rng.standard_normal((1, N, D), dtype=np.float32))
    k = O.bf16_round(rng.standard_normal((1, N, D), dtype=np.float32)
                     + 2.0 * rng.standard_normal((1, 1, D), dtype=np.float32))
    c = rng.standard_normal((1, 64, D), dtype=np.float32)
    v = O.bf16_round(c[:, rng.integers(0, 64, N)] + 0.3 * rng.standard_normal((1, N, D), dtype=np.float32))
    perm = np.argsort(rng.integers(0, w["k"], (1, N)), axis=-1, kind="stable").astype(np.int32)
    t0 = time.perf_counter()
    O.attention_reference(q, k, v, perm, block_rows=w["block_rows"], block_m=64, expcast=w["expcast"],
                          q_rows=q_rows)
    dt = time.perf_counter() - t0
    scale = (w["B"] * w["H"]) * (N / q_rows)
    return dt, dt * scale * 1e3


def reference_calibration():
    """oracle/reference_cpu_calibration.json: the reference's own CPU code
    timed against this port on the same one-head inputs (made where the
    reference is importable by oracle/calibrate_reference.py), or None."""
    try:
        with open(os.path.join(ROOT, "oracle", "reference_cpu_calibration.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def run_reference_arm(args, w, rank):
    """The reference's CPU algorithm on the host cores: each step is one head x
    cpu_rows query rows x all N keys of the workload (prepare of that head
    included), timed as it runs; ``value`` is that sample's attention FLOPs
    over its time, the same rate a whole call would run at (every head and
    query row block costs the same)."""
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    q_rows = args.cpu_rows
    for _ in range(args.warmup):
        cpu_sample(w, q_rows)
    secs, extrap = [], []
    for i in range(args.steps):
        dt, ms = cpu_sample(w, q_rows, seed=i)
        secs.append(dt)
        extrap.append(ms)
    dt = statistics.mean(secs)
    ms_call = statistics.mean(extrap)
    val = 4.0 * q_rows * float(w["N"]) * w["D"] / dt / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp8-e4m3 (fp32 accumulate, CPU emulation)",
        "data": "synthetic (seeded configs[1] distributions)",
        "config": {"workload": w["desc"], "q_rows_sampled": q_rows, "heads_sampled": 1},
        "ms_per_call_extrapolated": ms_call,
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"oracle vc_attention_reference, 1 head x {q_rows} query rows x "
                                   f"{w['N']} keys per step (a full call is {w['B'] * w['H']} heads x "
                                   f"{w['N'] // q_rows} such blocks: {ms_call / 1e3:.0f} s)",
                         "reference_calibration": reference_calibration()},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------- main ----

def _default_chunk(w, world):
    """Units per rank per all-gather round: a divisor of the rank's unit count
    (every round gives every rank the same work) leaving at least four
    rounds, so that each gather hides under the next rounds' attention; with
    the rounds on two alternating streams their grid tails overlap, so larger
    rounds buy nothing beyond that."""
    G = w["B"] * w["H"]
    per_rank = -(-G // world)
    cands = [c for c in range(1, per_rank + 1) if per_rank % c == 0 and per_rank // c >= 4]
    return max(cands) if cands else 1


def run_sharded(args, w, rank, world, local) -> int:
    """The job's (batch, head) units split over the ranks (strong scaling:
    the total work is the single-GPU workload's), each rank running prepare +
    attention on its units and NCCL all-gathers assembling the full bf16
    output on every rank.  The units are dealt in rounds; each round's
    all-gather overlaps the next round's compute.  configs[4] always runs
    here; the other workloads run here when N > 1."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        # The gathers run on a high-priority NCCL stream: when an attention
        # CTA retires, a waiting NCCL CTA gets the SM first.
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = not args.nccl_normal_priority
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev, pg_options=opts)
    from comfyui_vc_attention_b200.vc_attention import _native as N
    from comfyui_vc_attention_b200.vc_attention.grouping import GroupingConfig, build_permutation
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_status,
                                                                          vc_attention_cuda, vc_attention_host)
    from comfyui_vc_attention_b200.vc_attention.sharded import rank_units, vc_attention_sharded
    N.lib()
    q, k, v = make_inputs_gpu(w, 1234, dev)          # the same inputs on every rank
    B, H, NT, D = q.shape
    G = B * H
    chunk = (args.chunk or _default_chunk(w, world)) if world > 1 else None
    mine = rank_units(G, world, rank, chunk)
    n_mine = sum(hi - lo for lo, hi in mine)
    perm = torch.zeros((G, NT), dtype=torch.int32, device=dev)
    gcfg = GroupingConfig(block_rows=w["block_rows"], iters=3, max_clusters=w["k"])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for lo, hi in mine:
        perm[lo:hi] = build_permutation(v.view(G, NT, D)[lo:hi], gcfg).perm
    e1.record()
    torch.cuda.synchronize()
    kmeans_ms = e0.elapsed_time(e1)
    cfg = TritonConfig(block_n=w["block_rows"], enable_expcast=w["expcast"], sparse=w["sparse"],
                       tau=w.get("tau", 1.3), qk_fp4=w.get("qk_fp4", False))
    scale = D ** -0.5

    transport, transport_note = args.gather, None
    if world > 1 and transport == "peer":
        # the symmetric-memory rendezvous happens on the first call; if it
        # raises on any rank, every rank takes the NCCL gathers instead
        ok = 1.0
        try:
            vc_attention_sharded(q, k, v, perm, cfg, scale, gather=True, chunk=chunk,
                                 overlap_rounds=not args.serial_rounds, transport="peer")
            torch.cuda.synchronize()
        except Exception as e:  # reported in the JSON line
            ok, transport_note = 0.0, f"peer transport unavailable ({type(e).__name__}: {str(e)[:160]})"
        flag = torch.tensor([ok], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if float(flag.item()) < 1.0:
            transport = "nccl"
            transport_note = transport_note or "peer transport failed on another rank"

    def step(gather=True):
        return vc_attention_sharded(q, k, v, perm, cfg, scale, gather=gather, chunk=chunk,
                                    overlap_rounds=not args.serial_rounds, transport=transport)

    for _ in range(max(3, args.warmup)):
        out = step()
    torch.cuda.synchronize()

    # One step per CUDA graph replay (all rounds, both compute streams and
    # the NCCL all-gathers captured): a round's host work (argument checks,
    # tensor-map encoding, allocator calls) is of the order of its GPU time
    # once a rank holds only a few heads.
    graphs = {}
    if not args.eager:
        for gather in (True, False):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                res_g = step(gather)
            graphs[gather] = (gr, res_g)
        torch.cuda.synchronize()

    def run(gather=True):
        if graphs:
            graphs[gather][0].replay()
            return graphs[gather][1]
        return step(gather)

    for _ in range(2):
        out = run()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    t0.record()
    for _ in range(args.steps):
        out = run()
    t1.record()
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / args.steps
    # the same units without the all-gathers: the compute share of a step
    t2, t3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t2.record()
    for _ in range(args.steps):
        run(False)
    t3.record()
    torch.cuda.synchronize()
    ms_compute = t2.elapsed_time(t3) / args.steps
    if world > 1:
        t = torch.tensor([ms, ms_compute], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_compute = (float(x) for x in t.tolist())
    fl = flops_per_call(w)
    value = fl / (ms / 1e3) / 1e12

    # ---- the sharded output equals single-GPU calls (not timed) ----------
    # Heads are independent and every kernel is deterministic, so a sampled
    # unit recomputed alone on this GPU (its permutation rebuilt here) must
    # equal the gathered output bit for bit.
    check_units = sorted({0, G // 2 + 1, G - 1})
    mismatches = 0
    for u in check_units:
        pu = build_permutation(v.view(G, NT, D)[u:u + 1], gcfg).perm
        ou = vc_attention_cuda(q.view(G, NT, D)[u:u + 1].unsqueeze(0), k.view(G, NT, D)[u:u + 1].unsqueeze(0),
                               v.view(G, NT, D)[u:u + 1].unsqueeze(0), pu, cfg, scale)
        if not torch.equal(ou.reshape(NT, D), out.reshape(G, NT, D)[u]):
            mismatches += 1
    torch.cuda.synchronize()
    status = attention_status()

    # ---- e2e: each rank streams its own units from pinned host memory
    # through the public host entry point and writes their output rows back
    # to the host (no device all-gather: the host receives every unit once)
    q_h = [q.view(G, NT, D)[lo:hi].unsqueeze(0).cpu().pin_memory() for lo, hi in mine]
    k_h = [k.view(G, NT, D)[lo:hi].unsqueeze(0).cpu().pin_memory() for lo, hi in mine]
    v_h = [v.view(G, NT, D)[lo:hi].unsqueeze(0).cpu().pin_memory() for lo, hi in mine]
    o_h = [torch.empty_like(t).pin_memory() for t in q_h]
    p_d = [perm[lo:hi] for lo, hi in mine]

    def e2e_step():
        for qq, kk, vv, oo, pp in zip(q_h, k_h, v_h, o_h, p_d):
            vc_attention_host(qq, kk, vv, pp, cfg, scale, out=oo)

    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = 3
    a.record()
    for _ in range(e2e_steps):
        e2e_step()
    b_.record()
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b_) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms, float(mismatches), float(status[0])], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms, mismatches, st_code = float(t[0]), int(t[1]), int(t[2])
    else:
        st_code = status[0]
    psnr = None
    if rank == 0 and not args.no_psnr and NT <= 16384:
        psnr = psnr_vs_sdpa(out, q, k, v)
    peaks, peak_kind = measured_peaks()
    fp8_peak = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    rounds = len(mine)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp8-e4m3 (fp32 accumulate)",
            "data": "synthetic (seeded configs distributions, generated on device)",
            "config": {"workload": w["desc"], "B": B, "H": H, "N": NT, "D": D, "block_rows": w["block_rows"],
                       "kmeans_k": w["k"], "expcast": w["expcast"], "sparse": w["sparse"],
                       "units_per_rank": n_mine,
                       "parallelism": (f"(batch, head) units over {world} ranks (strong scaling), dealt in "
                                       f"{rounds} rounds of {chunk} per rank, prepared once per rank; each "
                                       + (f"round's bf16 output slice pushed to every peer's symmetric-memory "
                                          f"buffer by copy-engine copies (no SMs), one NCCL all-reduce at the end"
                                          if transport == "peer" else
                                          f"round's NCCL all-gather of the bf16 output (high-priority stream: "
                                          f"{not args.nccl_normal_priority})")
                                       + f"; overlaps the next round's attention "
                                       f"(rounds on two streams: {not args.serial_rounds})"
                                       if world > 1 else "one GPU"),
                       "l2": "inputs larger than L2"},
            "ms_compute": ms_compute, "ms_gather_exposed": max(0.0, ms - ms_compute), "kmeans_ms": kmeans_ms,
            "gather_transport": transport if world > 1 else None, "gather_transport_note": transport_note,
            "host_enqueue_ms": host_ms, "cuda_graph": bool(graphs),
            "psnr_db": psnr,
            "sharded_equals_single_gpu": {"units_checked": check_units, "mismatches": mismatches,
                                          "device_status": st_code},
            "roofline": {"bound": "tensor", "achieved": value / world, "peak": fp8_peak, "unit": "TFLOP/s",
                         "frac": value / world / fp8_peak, "traffic": None,
                         "kernel": "whole step per GPU (prepare + attention + all-gather)",
                         "peak_note": f"dense FP8 = 2 x {peak_kind} bf16 burst"},
            "e2e": {"value": fl / (e2e_ms / 1e3) / 1e12, "unit": UNIT, "ms_per_call": e2e_ms,
                    "h2d_bytes_per_step": 3 * G * NT * D * q.element_size(),
                    "d2h_bytes_per_step": G * NT * D * q.element_size(),
                    "note": "all ranks together; each rank copies only its own units"},
            "gpu_launches": (5 + 1) * rounds * args.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    graphs.clear()          # graphs holding NCCL calls go before the process group
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c1", choices=sorted(WORKLOADS))
    ap.add_argument("--cpu-rows", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--chunk", type=int, default=0, help="units per rank per all-gather round (N > 1)")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: independent full-size replicas per rank instead of the sharded split")
    ap.add_argument("--no-psnr", action="store_true")
    ap.add_argument("--kernel", default="auto", choices=["auto", "tc", "mma"],
                    help="attention kernel of the timed device step: tcgen05, the register-MMA comparison "
                         "kernel, or auto (tcgen05 wherever it applies)")
    ap.add_argument("--kv-split", type=int, default=1,
                    help="dense kernel KV split: 1 = none, 0 = the last partial wave (auto), k = k pieces")
    ap.add_argument("--eager", action="store_true", help="N > 1: launch every round eagerly (no CUDA graph)")
    ap.add_argument("--serial-rounds", action="store_true",
                    help="N > 1: rounds in order on one stream (default: two alternating streams)")
    ap.add_argument("--nccl-normal-priority", action="store_true", help="N > 1: NCCL on a normal-priority stream")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="N > 1: output all-gather by copy-engine pushes into the peers' symmetric-memory "
                         "buffers (peer) or by one NCCL all-gather per round (nccl)")
    ap.add_argument("--profile", action="store_true",
                    help="timed steps only (no e2e, PSNR or CPU baseline): the command profiled by ncu")
    args = ap.parse_args()
    w = WORKLOADS[args.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference_arm(args, w, rank)
    if w.get("sharded") or (world > 1 and not args.replicas):
        return run_sharded(args, w, rank, world, local)

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from comfyui_vc_attention_b200.vc_attention import _native as N
    from comfyui_vc_attention_b200.vc_attention.grouping import GroupingConfig, build_permutation
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import (TritonConfig, attention_prepared,
                                                                          prepare, vc_attention_cuda, sparse_tc_applies,
                                                                          vc_attention_host)
    N.lib()

    q, k, v = make_inputs_gpu(w, 1234 + rank, dev)
    B, H, NT, D = q.shape
    G = B * H
    # k-means permutation (timed once, reported separately)
    gcfg = GroupingConfig(block_rows=w["block_rows"], iters=3, max_clusters=w["k"])
    build_permutation(v.view(G, NT, D), gcfg)      # warm
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    res = build_permutation(v.view(G, NT, D), gcfg)
    e1.record()
    torch.cuda.synchronize()
    kmeans_ms = e0.elapsed_time(e1)
    perm = res.perm
    cfg = TritonConfig(block_n=w["block_rows"], enable_expcast=w["expcast"], sparse=w["sparse"],
                       tau=w.get("tau", 1.3), qk_fp4=w.get("qk_fp4", False), kv_split=args.kv_split)
    scale = D ** -0.5
    out = torch.empty_like(q)
    # tcgen05 kernels read V in their key order; the register-MMA sparse
    # kernel (other shapes) reads the block-transposed copy.
    sparse_tc = cfg.sparse and sparse_tc_applies(D, w["block_rows"], cfg.block_m, cfg.group, NT)
    want_v = ((not cfg.sparse) or sparse_tc) and args.kernel != "mma"

    def step(evs=None):
        if evs is not None:
            evs[0].record()
        p = prepare(q, k, v, perm, block_rows=w["block_rows"], hadamard=True, smooth_k=True,
                    sparse=cfg.sparse, tau=cfg.tau, q_block=cfg.block_m, scale=scale,
                    want_v=want_v, want_v_t=not want_v, local_blocks=cfg.local_blocks,
                    sink_blocks=cfg.sink_blocks, qk_fp4=cfg.qk_fp4, fp8_qk=not cfg.qk_fp4)
        if evs is not None:
            evs[1].record()
        attention_prepared(p, NT, out, scale, cfg, kernel=args.kernel)
        if evs is not None:
            evs[2].record()
        return p

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local if "CUDA_VISIBLE_DEVICES" not in os.environ else local)
    clocks.start()
    time.sleep(0.3)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t_start.record()
    for i in range(args.steps):
        step(evs[i])
    t_end.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    total_ms = t_start.elapsed_time(t_end)
    prep_ms = statistics.mean(evs[i][0].elapsed_time(evs[i][1]) for i in range(args.steps))
    attn_ms = statistics.mean(evs[i][1].elapsed_time(evs[i][2]) for i in range(args.steps))
    if world > 1:
        t = torch.tensor([total_ms, attn_ms, prep_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, attn_ms, prep_ms = (float(x) for x in t.tolist())
    ms_per_step = total_ms / args.steps
    fl = flops_per_call(w)
    value = world * fl / (ms_per_step / 1e3) / 1e12

    if args.profile:
        if rank == 0:
            print(json.dumps({"profile": args.workload, "ms_per_step": ms_per_step, "ms_prepare": prep_ms,
                              "ms_attention": attn_ms}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return 0

    # ---- end to end through the public entry point, host buffers ----------
    # vc_attention_host streams head chunks: copy-in, prepare + attention and
    # copy-out of consecutive chunks overlap on three streams.
    q_h = q.cpu().pin_memory()
    k_h = k.cpu().pin_memory()
    v_h = v.cpu().pin_memory()
    o_h = torch.empty(q.shape, dtype=q.dtype).pin_memory()

    def e2e_step():
        vc_attention_host(q_h, k_h, v_h, perm, cfg, scale, out=o_h)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, args.steps // 2)
    a.record()
    for _ in range(e2e_steps):
        e2e_step()
    b_.record()
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b_) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = 3 * q.numel() * q.element_size()
    d2h = q.numel() * q.element_size()
    del q_h, k_h, v_h

    # ---- fidelity (not timed) ---------------------------------------------
    psnr = None
    if rank == 0:
        step()
        torch.cuda.synchronize()
        psnr = psnr_vs_sdpa(out, q, k, v)

    peaks, peak_kind = measured_peaks()
    fp8_peak = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    keep_frac = None
    sparse_stats = None
    if w["sparse"]:
        pk = step()
        torch.cuda.synchronize()
        keep_frac = float(pk.keep.float().mean())
        kp = pk.keep.view(G, -1, 2, pk.keep.shape[-1]).bool()
        union = kp[:, :, 0] | kp[:, :, 1]           # tiles run by the tcgen05 CTA of two query blocks
        nbk = kp.shape[-1]
        pad = (-nbk) % 16                            # blocks past the end are never approximated
        kpp = torch.nn.functional.pad(kp.to(torch.uint8), (0, pad), value=1).bool()
        appx = (~kpp).view(G, kp.shape[1], 2, -1, 16).any(-1).any(2)   # groups with a proxy fold
        sparse_stats = {"union_fraction": float(union.float().mean()),
                        "proxy_groups_per_cta": float(appx.float().sum(-1).mean())}
        del kpp
        del pk, kp, union, appx
    # executed work of the attention kernel: dense tiles, or the kept tiles
    # plus the block-mean proxy of the skipped ones (2*N*NB*D per head each way)
    fl_exec = fl if keep_frac is None else (keep_frac * fl + 4.0 * G * NT * (NT // w["block_rows"]) * D)
    attn_tflops = fl_exec / (attn_ms / 1e3) / 1e12
    traffic = None   # DRAM bytes per attention launch from the committed ncu summary
    for tname in ("attn_tc_c1.md", "attn_tc_sparse_c2.md"):
        tpath = os.path.join(ROOT, "profiles", tname)
        if os.path.exists(tpath):
            with open(tpath) as f:
                for ln in f:
                    if ln.startswith(f"traffic_bytes_per_launch {args.workload}:"):
                        traffic = int(ln.split(":")[1])
    prep_bytes = (6 * G * NT * D + 3 * G * NT * D + 8 * G * NT + 8 * G * (NT // w["block_rows"]) * D
                  + 4 * G * NT)
    launches_per_step = 5 + 1
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp8-e4m3 (fp32 accumulate)",
        "data": "synthetic (seeded configs[1] distributions, generated on device)",
        "config": {"workload": w["desc"], "B": B, "H": H, "N": NT, "D": D, "block_rows": w["block_rows"],
                   "kmeans_k": res.k, "expcast": w["expcast"], "sparse": w["sparse"], "kv_split": args.kv_split,
                   "kernel": args.kernel,
                   "parallelism": (f"(batch, head) units x{world} ranks, independent replicas, no collective"
                                   if world > 1 else "one GPU"),
                   "l2": "inputs larger than L2 (Q/K/V 235 MB each)",
                   "keep_fraction": keep_frac,
                   "block_skip_ratio": None if keep_frac is None else 1.0 - keep_frac,
                   "sparse_cta_work": sparse_stats},
        "ms_prepare": prep_ms, "ms_attention": attn_ms, "kmeans_ms": kmeans_ms, "psnr_db": psnr,
        "roofline": {"bound": "tensor", "achieved": attn_tflops, "peak": fp8_peak, "unit": "TFLOP/s",
                     "frac": attn_tflops / fp8_peak, "traffic": traffic,
                     "kernel": ("attn_tc_sparse_kernel (tcgen05, tau-routed)" if sparse_tc and want_v
                                else "attn_sparse_kernel (mma.sync, tau-routed)" if w["sparse"]
                                else "attn_tc_kernel<NVFP4 QK> (tcgen05 mxf4nvf4 + f8f6f4)" if w.get("qk_fp4")
                                else "attn_mma_kernel (mma.sync comparison kernel)" if args.kernel == "mma"
                                else "attn_tc_kernel (tcgen05)"),
                     "flops": ("executed (kept tiles + proxy)" if w["sparse"] else "dense"),
                     "peak_note": f"dense FP8 = 2 x {peak_kind} bf16 burst ({peaks.get('bf16_tflops')} TF/s)"},
        "prepare_roofline": {"bound": "hbm", "achieved": prep_bytes / (prep_ms / 1e3) / 1e9,
                             "peak": float(peaks.get("hbm_gbs", 6650.0)), "unit": "GB/s",
                             "frac": prep_bytes / (prep_ms / 1e3) / 1e9 / float(peaks.get("hbm_gbs", 6650.0))},
        "e2e": {"value": world * fl / (e2e_ms / 1e3) / 1e12, "unit": UNIT, "ms_per_call": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, ms_cpu = cpu_sample(w, args.cpu_rows)
        line["cpu_baseline"] = {
            "value": fl / (ms_cpu / 1e3) / 1e12, "unit": UNIT, "cores": os.cpu_count() or 1,
            "kind": "port", "ms_per_call_extrapolated": ms_cpu, "sample_seconds": dt,
            "sample": f"oracle vc_attention_reference, 1 head x {args.cpu_rows} query rows x {NT} keys, "
                      f"extrapolated x{G} heads x {NT // args.cpu_rows} row blocks",
            "reference_calibration": reference_calibration()}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
