#!/usr/bin/env python
"""Benchmark of the B200 PP-DocLayoutV3 hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload forward|msda|gemm] [--pages P] [--gemm M,N,K,P]
                    [--capture-once]

Workloads
  forward  (default) config 3 of the baseline: the full PP-DocLayoutV3 forward
           plus the postprocess on 800x800 pages, FP32, 8 pages per GPU per
           step, replayed from its CUDA graph with the inputs in HBM.  `value`
           is pages/s; `e2e` is ppdl_infer_batch with host images in and
           detections + masks out; `stages` / `top_steps` / `roofline` come
           from the per-step device profile (ppdl_profile_steps); the CPU
           baseline is the oracle's restatement of the forward on the host
           threads.  The per-step working set (~6 GB) is larger than L2.
  msda     config 1 of the baseline: the MSDeformAttn operator alone, FP32,
           value [B,13125,8,32] ~ N(0,1), sampling locations
           [B,300,8,3,4,2] ~ U[0,1], weights softmax(N(0,1)) over 12, at
           B = 32 pages per GPU (the largest of the B sweep {1,8,32}; the
           smaller B are parity-test cases).  One step = one launch over the
           batch.  The 430 MB value tensor is larger than the 126 MB L2, so
           nothing stays cached between steps.
  gemm     the forward's dominant kernel alone: ppdl_gemm_tf32x3 (3xTF32 on
           tcgen05) on one shape, default the 200x200-plane 1x1 conv 1024 ->
           256 over 8 pages.

`--capture-once` (forward): set up, run one eager forward and exit — the
launch sequence of one forward, for profiler captures.

Multi-GPU: one process per GPU (torchrun), every rank runs its own pages
(weak scaling, no data-path collective); the timed region is bracketed by a
gloo barrier + device synchronise and the slowest rank's time is reported.

`--impl reference` times the reference's CPU path of the workload on all
host cores, rank 0 only: for the forward the oracle's restatement (the
reference's ggml CPU graph cannot be built here), for msda the reference's
own op_msdeform (src/ppdoclayout.cpp:142-198, compiled from the reference
sources into oracle/_ref/, or the oracle restatement when that build is
absent).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "ppdoclayout-ggml_b200"))

METRIC = "pages/s @800² FP32 at 1/2/4/8 B200; MSDeformAttn HBM GB/s; conv TFLOPS"


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms during the
    timed region (a 20-step forward region lasts about 0.3 s)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.06)  # the sample in flight at the end of the region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self._t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- distributed
def dist_setup(args, timeout_s: float = 120.0):
    """Rank layout from the torchrun environment; a gloo group (timing
    barrier and max/sum reductions only) when there are several ranks.  The
    group timeout bounds every collective, so a rank that died makes the
    others fail instead of waiting."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s))
        pg = dist
    return world, rank, local, pg


def barrier(pg):
    if pg is not None:
        pg.barrier()


def max_over_ranks(pg, v: float) -> float:
    if pg is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(pg, v: float) -> float:
    if pg is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    pg.all_reduce(t, op=pg.ReduceOp.SUM)
    return float(t.item())


def job_rate(units_per_rank_step: float, steps: int, world: int, ms_max: float) -> float:
    """Whole-job throughput: the units all ranks processed divided by the
    slowest rank's device time (weak scaling: every rank does the same work)."""
    return units_per_rank_step * steps * world / (ms_max / 1e3)


# ------------------------------------------------------------------ MSDA (cfg 1)
MSDA_B = 32
NQ, NTOK = 300, 13125
LVL = ((100, 100, 0), (50, 50, 10000), (25, 25, 12500))


def msda_inputs_torch(B, seed, device):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    val = torch.randn((B, NTOK, 8, 32), generator=g, device=device, dtype=torch.float32)
    loc = torch.rand((B, NQ, 8, 3, 4, 2), generator=g, device=device, dtype=torch.float32)
    lg = torch.randn((B, NQ, 8, 12), generator=g, device=device, dtype=torch.float32)
    w = torch.softmax(lg, dim=-1).contiguous()
    return val, loc, w


def msda_algorithmic_bytes(loc, w):
    """128 B per unique (page, head, level-token) value row touched by an
    in-bounds corner with non-zero weight, plus the loc, weight and output
    bytes.  Computed on the device with the kernel's tap rule."""
    import torch
    B = loc.shape[0]
    keys = []
    for l, (W, H, st) in enumerate(LVL):
        lx = loc[:, :, :, l, :, 0]
        ly = loc[:, :, :, l, :, 1]
        fx = lx * W - 0.5
        fy = ly * H - 0.5
        x0 = torch.floor(fx)
        y0 = torch.floor(fy)
        tx, ty = fx - x0, fy - y0
        x0 = x0.long()
        y0 = y0.long()
        wl = w[:, :, :, l * 4:(l + 1) * 4]
        for k in range(4):
            dx, dy = k & 1, k >> 1
            cw = (tx if dx else 1 - tx) * (ty if dy else 1 - ty)
            xx, yy = x0 + dx, y0 + dy
            ok = (xx >= 0) & (xx < W) & (yy >= 0) & (yy < H) & (cw != 0) & (wl != 0)
            b = torch.arange(B, device=loc.device).view(B, 1, 1, 1).expand_as(xx)
            h = torch.arange(8, device=loc.device).view(1, 1, 8, 1).expand_as(xx)
            tok = st + yy * W + xx
            key = (b * 8 + h) * NTOK + tok
            keys.append(key[ok])
    uniq = torch.unique(torch.cat(keys)).numel()
    out_b = B * NQ * 256 * 4
    return uniq * 128 + loc.numel() * 4 + w.numel() * 4 + out_b, uniq


def run_msda(args, world, rank, local, pg):
    import torch
    import ppdl
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    B = MSDA_B
    val, loc, w = msda_inputs_torch(B, 1234 + rank, dev)
    out = torch.empty((B, NQ, 256), device=dev, dtype=torch.float32)
    stream = torch.cuda.Stream(device=dev)
    desc = ppdl.make_desc(ppdl.OP_MSDEF, out, [val, loc, w], params=[1],
                          dst_ne=[256, NQ, B], src_ne=[[256, NTOK, B], [192, NQ, B], [96, NQ, B]])
    L = ppdl.lib()
    sp = C.c_void_p(stream.cuda_stream)

    def step():
        st = L.ppdl_op_launch(C.byref(desc), sp)
        if st != 0:
            raise RuntimeError(ppdl.last_error())

    alg_bytes, uniq_rows = msda_algorithmic_bytes(loc, w)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize(dev)

    K = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(K)]
    clocks = ClockSampler(local)
    barrier(pg)
    torch.cuda.synchronize(dev)
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(K):
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(pg)
    clk = clocks.stop()
    total_ms = t0.elapsed_time(t1)
    kern_ms = sum(a.elapsed_time(b) for a, b in ev) / K
    total_ms_max = max_over_ranks(pg, total_ms)
    pages = B * K * world
    value = pages / (total_ms_max / 1e3)

    # ---- e2e: same op through the C ABI with host buffers (H2D + launch + D2H)
    hv = val.cpu().pin_memory()
    hl = loc.cpu().pin_memory()
    hw = w.cpu().pin_memory()
    ho = torch.empty(out.shape, dtype=torch.float32).pin_memory()
    h2d = (hv.numel() + hl.numel() + hw.numel()) * 4
    d2h = ho.numel() * 4

    def e2e_step():
        with torch.cuda.stream(stream):
            val.copy_(hv, non_blocking=True)
            loc.copy_(hl, non_blocking=True)
            w.copy_(hw, non_blocking=True)
            step()
            ho.copy_(out, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier(pg)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e2e_steps = max(3, min(K, 10))
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(pg)
    e2e_ms = max_over_ranks(pg, e0.elapsed_time(e1))
    e2e_val = B * e2e_steps * world / (e2e_ms / 1e3)

    hbm, _, peak_kind = _peaks()
    achieved = alg_bytes / (kern_ms / 1e3) / 1e9
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "pages/s (MSDeformAttn op, config 1)",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms_max / K, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded torch RNG, per-rank seed)",
        "config": {"workload": "config 1: MSDeformAttn, canonical form, B=32 pages per GPU",
                   "pages_per_gpu_per_step": B, "queries": NQ, "heads": 8, "levels": 3,
                   "points": 4, "l2": "inputs (430 MB value) larger than L2",
                   "parallelism": f"dp{world} (pages sharded, no collective)"},
        "msda_gbs": round(achieved, 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                     "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_kind": f"{peak_kind} burst copy",
                     "algorithmic_bytes_per_launch": alg_bytes,
                     "unique_value_rows": uniq_rows,
                     "kernel_ms": round(kern_ms, 5), "traffic": None},
        "e2e": {"value": round(e2e_val, 1), "unit": "pages/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "ppdl_op_launch(op 2) with pinned host buffers, copies in the timed region"},
        "gpu_launches": K,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_msda(budget_s=args.cpu_seconds)
    return line


def cpu_baseline_msda(budget_s=10.0, sample_pages=None):
    """The reference CPU op (or the oracle port) over a bounded sample of the
    config-1 workload, all host threads; pages/s."""
    import numpy as np
    import oracle
    nth = os.cpu_count() or 1
    rng = np.random.default_rng(7)
    pages = []
    for _ in range(2):
        val = rng.standard_normal((NTOK, 256), dtype=np.float32)
        loc = rng.uniform(0, 1, (NQ, 192)).astype(np.float32)
        lg = rng.standard_normal((NQ, 8, 12)).astype(np.float32)
        # the reference op consumes offsets + ref + logits; ref = (0,0,8,8)
        # makes its sampling location equal `loc` exactly
        ref = np.tile(np.array([0, 0, 8, 8], np.float32), (NQ, 1))
        pages.append((val, loc, lg.reshape(NQ, 96), ref))
    if oracle.ref_available():
        r = oracle.ref()
        kind = "reference"
        fn = lambda p: r.msdeform(p[0], p[1], p[2], p[3], nth=nth)  # noqa: E731
    else:
        o = oracle.oracle()
        kind = "port"
        fn = lambda p: o.msdeform(p[0][None], p[1][None], p[2][None], p[3][None])  # noqa: E731
    fn(pages[0])
    n, t0 = 0, time.perf_counter()
    while True:
        fn(pages[n % len(pages)])
        n += 1
        el = time.perf_counter() - t0
        if (sample_pages and n >= sample_pages) or (not sample_pages and el >= budget_s):
            break
    return {"value": round(n / el, 2), "unit": "pages/s", "cores": nth, "kind": kind,
            "sample": f"{n} pages of config 1 (B=1 each, 2 distinct seeded pages cycled) in "
                      f"{el:.1f} s; op_msdeform of src/ppdoclayout.cpp:142-198"}


# ------------------------------------------------------------ forward (cfg 3)
FWD_B = 8
GEMM_KINDS = ("gemm_1x1", "wg_madd", "gemm_implicit", "gemm_linear")
HBM_KINDS = ("wg_input", "wg_output", "dwconv", "msda", "mask_box", "glue", "postprocess", "topk",
             "im2col")
# FP32 CUDA-core work (q-k products, the stem's narrow convs): their FLOP rate, no roofline class
SIMT_KINDS = ("attention", "conv_direct")
# DRAM traffic of the tensor-core GEMM per page of one forward (sum over its
# launches of dram__bytes_read.sum + dram__bytes_write.sum), from an ncu
# capture of one eager forward at 2 pages; None until measured.
TC_GEMM_DRAM_BYTES_PER_PAGE = 1.2477e9  # 2.495 GB over the 166 launches of 2 pages


def _fwd_pages(rank, B):
    import numpy as np
    import synth
    return np.stack([synth.synth_page(1000 + rank * B + i) for i in range(B)])


def stage_summary(steps, B, hbm_gbs, tc_tflops):
    """Per kernel class: device ms, achieved TFLOP/s or GB/s and the
    fraction of the class's roofline."""
    out = {}
    for kind in sorted({s[1] for s in steps}):
        ss = [s for s in steps if s[1] == kind]
        ms = sum(s[2] for s in ss)
        fl = sum(s[3] for s in ss) * B
        by = sum(s[4] for s in ss) * B
        e = {"ms": round(ms, 4), "launch_groups": len(ss)}
        if kind in GEMM_KINDS and ms > 0:
            e["tflops"] = round(fl / (ms / 1e3) / 1e12, 2)
            e["frac_of_3xtf32"] = round(e["tflops"] / tc_tflops, 4)
        elif kind in SIMT_KINDS and ms > 0:
            e["tflops"] = round(fl / (ms / 1e3) / 1e12, 2)
        elif ms > 0:
            e["gbs"] = round(by / (ms / 1e3) / 1e9, 1)
            e["frac_of_hbm"] = round(e["gbs"] / hbm_gbs, 4)
        out[kind] = e
    return out


def run_forward(args, world, rank, local, pg):
    import numpy as np
    import torch
    import ppdl
    import synth
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    B = args.pages or FWD_B
    gguf = synth.cached_gguf(0)
    ctx = ppdl.Context(gguf, device=local, max_batch=B)
    pages = _fwd_pages(rank, B)
    hw = np.full((B, 2), 800, np.int32)
    d_img = torch.from_numpy(pages).to(dev)
    st = torch.cuda.ExternalStream(ctx.stream_ptr(), device=dev)
    if args.capture_once:
        torch.cuda.synchronize(dev)
        if ctx.infer_device_bits(d_img.data_ptr(), B, hw) != 0 or ctx.sync() != 0:
            raise RuntimeError("forward failed")
        return None

    def step():
        # the forward with its own mask output (packed, 1 bit per pixel)
        rc = ctx.infer_device_bits(d_img.data_ptr(), B, hw)
        if rc != 0:
            raise RuntimeError(f"ppdl_infer_device_bits returned {rc}")

    for _ in range(args.warmup):
        step()
    if ctx.sync() != 0:
        raise RuntimeError("forward failed")
    K = args.steps
    clocks = ClockSampler(local)
    barrier(pg)
    torch.cuda.synchronize(dev)
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(st)
    for _ in range(K):
        step()
    t1.record(st)
    torch.cuda.synchronize(dev)
    ctx.sync()
    barrier(pg)
    clk = clocks.stop()
    total_ms = t0.elapsed_time(t1)
    total_ms_max = max_over_ranks(pg, total_ms)
    value = job_rate(B, K, world, total_ms_max)

    # per-step device profile of one eager forward (kernel classes, roofline)
    steps = ctx.profile_steps(B)
    top = []
    for name, kind, ms, fl, by in sorted(steps, key=lambda s: -s[2])[:12]:
        e = {"step": name, "kind": kind, "ms": round(ms, 4)}
        if kind in GEMM_KINDS + SIMT_KINDS and ms > 0:
            e["tflops"] = round(fl * B / (ms / 1e3) / 1e12, 1)
        elif ms > 0:
            e["gbs"] = round(by * B / (ms / 1e3) / 1e9, 1)
        top.append(e)
    hbm, bf16, peak_kind = _peaks()
    tc = bf16 / 6.0  # 3xTF32: three TF32 products at half the BF16 rate
    stages = stage_summary(steps, B, hbm, tc)
    prof_ms = sum(s[2] for s in steps)
    conv_kinds = ("gemm_1x1", "wg_madd", "gemm_implicit", "wg_input", "wg_output", "dwconv")
    conv_ms = sum(stages[k]["ms"] for k in conv_kinds if k in stages)
    direct_conv_flops = 0.0
    for name, kind, ms, fl, by in steps:
        if kind == "wg_madd":
            # executed 2*36*T*IC*OC; the direct conv does 2*16T*9*IC*OC = 4x that
            direct_conv_flops += fl * 4.0
        elif kind in ("gemm_1x1", "gemm_implicit", "dwconv"):
            direct_conv_flops += fl
    # dominant kernel: the 3xTF32 tcgen05 GEMM, which every step of the GEMM
    # kinds launches once (1x1 convs, Winograd madd, im2col convs, linears)
    gsteps = [s for s in steps if s[1] in GEMM_KINDS]
    g_ms = sum(s[2] for s in gsteps)
    g_fl = sum(s[3] for s in gsteps) * B
    if g_ms <= 0:
        raise RuntimeError("per-step profile returned no GEMM time")
    achieved = g_fl / (g_ms / 1e3) / 1e12
    roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(tc, 1),
            "unit": "TFLOP/s", "frac": round(achieved / tc, 4),
            "peak_kind": f"{peak_kind} bf16 dense / 6 (3xTF32: three TF32 MMAs at half rate)",
            "kernel": "tc_gemm_kernel (3xTF32 tcgen05)", "launches_per_forward": len(gsteps),
            "kernel_ms_per_forward": round(g_ms, 4),
            "achieved_per_launch": "algorithmic FLOPs of the launches / their summed device time",
            "traffic": None}
    if TC_GEMM_DRAM_BYTES_PER_PAGE:
        # DRAM bytes per launch, from the ncu capture named beside the constant
        roof["traffic"] = round(TC_GEMM_DRAM_BYTES_PER_PAGE * B / max(1, len(gsteps)))
        roof["traffic_unit"] = "bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum)"
        roof["algorithmic_bytes_per_launch"] = round(
            sum(s[4] for s in gsteps) * B / max(1, len(gsteps)))

    # ---- e2e (headline): the pipelined public API, ppdl_submit_batch /
    # ppdl_wait_batch, with the pages in pinned host memory and the dets and
    # packed masks read back into the context's pinned result slots; two
    # batches in flight, so one batch's copies overlap the next one's
    # forward.  Timed by the host clock from a synchronised start to the
    # last wait (which returns once that batch's results are in host memory).
    h_pages = torch.from_numpy(pages).pin_memory().numpy()
    e2e_steps = max(3, K)
    for _ in range(2):
        ctx.wait(ctx.submit(h_pages, hw), B, copy=False)
    torch.cuda.synchronize(dev)
    barrier(pg)
    w0 = time.perf_counter()
    pending = []
    for _ in range(e2e_steps):
        pending.append(ctx.submit(h_pages, hw))
        if len(pending) == 2:
            ctx.wait(pending.pop(0), B, copy=False)
    for t in pending:
        ctx.wait(t, B, copy=False)
    e2e_ms = (time.perf_counter() - w0) * 1e3
    barrier(pg)
    e2e_ms = max_over_ranks(pg, e2e_ms)
    e2e_val = B * e2e_steps * world / (e2e_ms / 1e3)
    h2d = B * 3 * 800 * 800 * 4 + B * 8
    d2h = B * 300 * 7 * 4 + B * 300 * 1250 * 4

    # ---- e2e in the reference's result format: ppdl_infer_batch (one batch
    # at a time, int32 masks of 48 MB per page read back into pinned buffers)
    ctx.infer_batch(h_pages, hw, copy=False)
    barrier(pg)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    i32_steps = max(3, min(K, 5))
    e0.record(st)
    for _ in range(i32_steps):
        ctx.infer_batch(h_pages, hw, copy=False)
    e1.record(st)
    torch.cuda.synchronize(dev)
    barrier(pg)
    i32_ms = max_over_ranks(pg, e0.elapsed_time(e1))
    i32_val = B * i32_steps * world / (i32_ms / 1e3)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "pages/s",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms_max / K, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic pages (config 0 recipe, distinct seed per page) and seeded random "
                "weights (BN folded GGUF)",
        "config": {"workload": "config 3: full PP-DocLayoutV3 forward + postprocess, "
                               "800x800, 8 pages per GPU per step, CUDA-graph replay",
                   "pages_per_gpu_per_step": B,
                   "l2": "working set per step (~6 GB of activations) larger than L2",
                   "parallelism": f"dp{world} (pages sharded, weights replicated, no collective)"},
        "conv_tflops_direct": round(direct_conv_flops * B / (conv_ms / 1e3) / 1e12, 2)
        if conv_ms else None,
        "msda_gbs": stages.get("msda", {}).get("gbs"),
        "stages": stages,
        "top_steps": top,
        "profile_ms_per_step": round(prof_ms, 3),
        "roofline": roof,
        "e2e": {"value": round(e2e_val, 2), "unit": "pages/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "path": "ppdl_submit_batch / ppdl_wait_batch (pinned host pages in, dets + "
                        "packed masks out into pinned host buffers, two batches in flight; "
                        "host clock)"},
        "e2e_int32_masks": {"value": round(i32_val, 2), "unit": "pages/s",
                            "h2d_bytes_per_step": h2d,
                            "d2h_bytes_per_step": B * 300 * 7 * 4 + B * 300 * 40000 * 4,
                            "path": "ppdl_infer_batch (one batch at a time, dets + int32 masks "
                                    "of the reference's format)"},
        "gpu_launches": len(steps) * K,
        "clocks": clk,
    }
    ctx.close()
    if rank == 0 and world == 1 and not args.no_sweeps:
        # the metric's other two clauses, measured after the timed region:
        # MSDeformAttn HBM GB/s (config 1, B = 32) and conv TFLOPS (config 2);
        # and config 4 (2048 pages, 32 per batch) on this GPU
        line.update(kernel_sweeps(dev, hbm, tc))
        line["config4_stress_1gpu"] = config4_stress(dev, 1, 0, None)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_forward(gguf, budget_s=args.cpu_seconds)
        if not args.no_sweeps:
            line["reference_gpu_bar"] = reference_gpu_bar(dev, hbm)
    return line


# --------------------------------------------- per-kernel sweeps (configs 1, 2)
L2_FLUSH_BYTES = 256 << 20  # written, then another buffer read, between timed launches (L2 is 126 MB)


def _time_launches(fn, dev, iters=10, warmup=3, flush=True):
    """Mean device time (ms) of fn() over iters launches, CUDA events on the
    current stream around each launch, L2 flushed in between (untimed): a
    write of a buffer larger than L2, then a read of another one, so that the
    write's dirty lines go back to HBM before the timed launch rather than
    during it."""
    import torch
    buf = torch.empty(L2_FLUSH_BYTES // 4, device=dev) if flush else None
    rd = torch.ones(L2_FLUSH_BYTES // 4, device=dev) if flush else None
    acc = torch.empty((), device=dev) if flush else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    st = torch.cuda.current_stream(dev)
    tot = 0.0
    for _ in range(iters):
        if buf is not None:
            buf.fill_(1.0)
            torch.sum(rd, dim=0, out=acc)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        fn()
        b.record(st)
        b.synchronize()
        tot += a.elapsed_time(b)
    return tot / iters


CONFIG2 = [
    # (kind, IC, H, OC): config 2 of the baseline, NCHW, B in {1, 8}
    ("3x3-s1", 128, 200, 128), ("3x3-s1", 256, 100, 256), ("3x3-s1", 512, 50, 512),
    ("3x3-s1", 1024, 25, 1024),
    ("1x1", 512, 100, 256), ("1x1", 1024, 50, 256), ("1x1", 2048, 25, 256),
    ("3x3-s2", 128, 200, 256), ("3x3-s2", 512, 100, 512),
]


def _bind_conv_entries(L):
    import ctypes as C
    L.ppdl_conv3x3_wg4_workspace.argtypes = [C.c_int] * 5
    L.ppdl_conv3x3_wg4_workspace.restype = C.c_longlong
    L.ppdl_conv3x3_wg4_prepare.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    L.ppdl_conv3x3_wg4_run.argtypes = (
        [C.c_void_p] + [C.c_int] * 4 + [C.c_longlong, C.c_void_p, C.c_int, C.c_int,
                                        C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p])
    L.ppdl_tf32_split.argtypes = [C.c_void_p, C.c_longlong, C.c_void_p, C.c_void_p]
    L.ppdl_gemm_tf32x3_presplit.argtypes = ([C.c_int] * 4 + [C.c_void_p, C.c_int, C.c_longlong,
                                            C.c_longlong, C.c_void_p, C.c_void_p]
                                            + [C.c_longlong] * 3 + [C.c_void_p])
    L.ppdl_conv2d_tf32x3.argtypes = (
        [C.c_void_p] + [C.c_int] * 4 + [C.c_longlong, C.c_void_p, C.c_void_p]
        + [C.c_int] * 7 + [C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p])
    L.ppdl_conv2d_tf32x3_workspace.argtypes = [C.c_int] * 3
    L.ppdl_conv2d_tf32x3_workspace.restype = C.c_longlong


def _conv_case(L, g, dev, kind, IC, H, OC, Bc, stream, with_bar=False):
    """One config-2 conv: (launch closure, direct FLOPs, executed GEMM
    FLOPs[, cuBLAS FP32 SGEMM closure on the GEMM the reference runs])."""
    import torch
    import ppdl
    K = 1 if kind == "1x1" else 3
    S = 2 if kind == "3x3-s2" else 1
    OH = (H + 2 * (K // 2) - K) // S + 1
    x = torch.randn((Bc, IC, H, H), generator=g, device=dev)
    wt = torch.randn((OC, IC, K, K), generator=g, device=dev) * (2.0 / (IC * K * K)) ** 0.5
    bias = torch.randn((OC,), generator=g, device=dev) * 0.1
    y = torch.empty((Bc, OC, OH, OH), device=dev)
    direct = 2.0 * Bc * OH * OH * OC * IC * K * K
    bar = None
    if kind == "3x3-s1":
        # filter transform once (as at model load), then the conv
        work = torch.empty(L.ppdl_conv3x3_wg4_workspace(Bc, IC, OC, H, H), device=dev)
        ppdl.check(L.ppdl_conv3x3_wg4_prepare(wt.data_ptr(), IC, OC, work.data_ptr(), stream()))

        def f():
            ppdl.check(L.ppdl_conv3x3_wg4_run(x.data_ptr(), Bc, IC, H, H, IC * H * H,
                                              bias.data_ptr(), OC, 1, work.data_ptr(),
                                              y.data_ptr(), OC * H * H, stream()))
        T = ((H + 3) // 4) ** 2
        executed = 2.0 * 36 * Bc * T * IC * OC
        if with_bar:
            # the reference's op 12: 36 strided-batched SGEMMs per page
            ga = torch.randn((Bc * 36, T, IC), generator=g, device=dev)
            gb = torch.randn((IC, OC), generator=g, device=dev)
            bar = lambda: torch.matmul(ga, gb)  # noqa: E731
    elif kind == "1x1":
        M = H * H
        ws = torch.empty(2 * OC * IC, device=dev)
        ppdl.check(L.ppdl_tf32_split(wt.data_ptr(), OC * IC, ws.data_ptr(), stream()))

        def f():
            ppdl.check(L.ppdl_gemm_tf32x3_presplit(M, OC, IC, Bc, x.data_ptr(), 1, M, IC * M,
                                                   ws.data_ptr(), y.data_ptr(), 1, M, OC * M,
                                                   stream()))
        executed = direct
        if with_bar:
            w2, x2 = wt.view(OC, IC), x.view(Bc, IC, M)
            bar = lambda: torch.matmul(w2, x2)  # noqa: E731
    else:
        ws = torch.empty(L.ppdl_conv2d_tf32x3_workspace(IC, OC, 3), device=dev)

        def f():
            ppdl.check(L.ppdl_conv2d_tf32x3(x.data_ptr(), Bc, IC, H, H, IC * H * H, wt.data_ptr(),
                                            bias.data_ptr(), OC, 3, 2, 1, OH, OH, 1,
                                            ws.data_ptr(), y.data_ptr(), OC * OH * OH, stream()))
        executed = direct
        if with_bar:
            # the reference's im2col + mul_mat: the GEMM alone
            ga = torch.randn((Bc, OH * OH, IC * 9), generator=g, device=dev)
            gb = torch.randn((IC * 9, OC), generator=g, device=dev)
            bar = lambda: torch.matmul(ga, gb)  # noqa: E731
    if with_bar:
        return f, direct, executed, bar
    return f, direct, executed


def kernel_sweeps(dev, hbm, tc):
    """Config 1 (MSDeformAttn alone, canonical form, B = 32) and config 2
    (the conv sweep at B = 1 and 8) through this build's C ABI entry points
    — the kernels the forward runs — with cuBLAS FP32 SGEMM (TF32 off, the
    reference's GEMM mode, patches/ggml-ppdl.patch:14-16, 650-665, 787-802)
    timed on each conv's GEMM beside it as the same-box bar."""
    import ctypes as C
    import torch
    import ppdl
    L = ppdl.lib()
    stream = lambda: torch.cuda.current_stream(dev).cuda_stream  # noqa: E731
    out = {}
    # ---- config 1
    B = MSDA_B
    val, loc, w = msda_inputs_torch(B, 4321, dev)
    o = torch.empty((B, NQ, 256), device=dev)
    desc = ppdl.make_desc(ppdl.OP_MSDEF, o, [val, loc, w], params=[1],
                          dst_ne=[256, NQ, B], src_ne=[[256, NTOK, B], [192, NQ, B], [96, NQ, B]])
    alg, _ = msda_algorithmic_bytes(loc, w)
    ms = _time_launches(lambda: ppdl.check(L.ppdl_op_launch(C.byref(desc), C.c_void_p(stream()))),
                        dev)
    out["config1_msda"] = {"pages": B, "ms": round(ms, 5), "gbs": round(alg / ms / 1e6, 1),
                           "frac_of_hbm": round(alg / ms / 1e6 / hbm, 4),
                           "algorithmic_bytes": alg, "l2": "flushed between launches (256 MB write, then 256 MB read)"}
    del val, loc, w, o
    # ---- config 2
    _bind_conv_entries(L)
    tf32_was = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    rows = []
    g = torch.Generator(device=dev).manual_seed(99)
    try:
        for kind, IC, H, OC in CONFIG2:
            for Bc in (1, 8):
                f, direct, executed, bar = _conv_case(L, g, dev, kind, IC, H, OC, Bc, stream,
                                                      with_bar=True)
                ms = _time_launches(f, dev)
                ms_bar = _time_launches(bar, dev)
                rows.append({"conv": f"{kind} {H}x{H}x{IC}->{OC}", "pages": Bc,
                             "ms": round(ms, 4), "tflops_direct": round(direct / ms / 1e9, 2),
                             "tflops_executed": round(executed / ms / 1e9, 2),
                             "frac_of_3xtf32": round(executed / ms / 1e9 / tc, 4),
                             "sgemm_gemm_only_ms": round(ms_bar, 4),
                             "speedup_vs_sgemm": round(ms_bar / ms, 2)})
                del f, bar
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32_was
    out["config2_conv"] = rows
    out["config2_note"] = ("ms: this build's conv with its weights prepared beforehand as at model "
                           "load (Winograd: input transform + 36-plane GEMM + output transform; "
                           "1x1: the GEMM; k3-s2: windowed implicit GEMM, its weight split "
                           "included) with bias + ReLU; sgemm_gemm_only_ms: "
                           "cuBLAS FP32 SGEMM, TF32 off, on the GEMM the reference runs for that "
                           "conv (its transforms / im2col not counted); L2 flushed between "
                           "launches")
    return out


def reference_gpu_bar(dev, hbm):
    """The reference's own CUDA kernels for MSDeformAttn and mask->box
    (compiled for sm_100a from its ggml patch into oracle/_ref/, one launch
    per page as the reference runs them) timed beside this build's kernels
    on the same inputs: config 1 at B = 32 (in-model form with reference
    boxes (0, 0, 8, 8), so the sampling locations are the config's) and
    mask->box over 8 pages of 300 masks."""
    import ctypes as C
    import torch
    import ppdl
    so = os.path.join(ROOT, "oracle", "_ref", "librefkern.so")
    if not os.path.exists(so):
        return {"unavailable": "oracle/_ref/librefkern.so not built (needs the reference "
                               "checkout at build time)"}
    R = C.CDLL(so)
    R.refkern_msdeform.argtypes = [C.c_void_p] * 5 + [C.c_int, C.c_int, C.c_void_p]
    R.refkern_mask_box.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
    L = ppdl.lib()
    st = lambda: C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)  # noqa: E731
    B = MSDA_B
    g = torch.Generator(device=dev).manual_seed(4321)
    val = torch.randn((B, NTOK, 256), generator=g, device=dev)
    off = torch.rand((B, NQ, 192), generator=g, device=dev)
    lg = torch.randn((B, NQ, 96), generator=g, device=dev)
    ref = torch.tensor([0.0, 0.0, 8.0, 8.0], device=dev).repeat(B, NQ, 1).contiguous()
    o1 = torch.empty((B, NQ, 256), device=dev)
    o2 = torch.empty((B, NQ, 256), device=dev)
    desc = ppdl.make_desc(ppdl.OP_MSDEF, o1, [val, off, lg, ref], params=[0],
                          dst_ne=[256, NQ, B],
                          src_ne=[[256, NTOK, B], [192, NQ, B], [96, NQ, B], [4, NQ, B]])
    ours = _time_launches(lambda: ppdl.check(L.ppdl_op_launch(C.byref(desc), st())), dev)
    theirs = _time_launches(lambda: R.refkern_msdeform(val.data_ptr(), off.data_ptr(),
                                                       lg.data_ptr(), ref.data_ptr(),
                                                       o2.data_ptr(), NQ, B, st()), dev)
    torch.cuda.synchronize(dev)
    msda_diff = float((o1 - o2).abs().max())
    rows = 8 * NQ
    ml = torch.randn((rows, 40000), generator=g, device=dev) - 1.5
    b1 = torch.empty((rows, 4), device=dev)
    b2 = torch.empty((rows, 4), device=dev)
    mdesc = ppdl.make_desc(ppdl.OP_MASKBOX, b1, [ml], dst_ne=[4, rows], src_ne=[[40000, rows]])
    ours_mb = _time_launches(lambda: ppdl.check(L.ppdl_op_launch(C.byref(mdesc), st())), dev)
    theirs_mb = _time_launches(lambda: R.refkern_mask_box(ml.data_ptr(), b2.data_ptr(), rows,
                                                          st()), dev)
    torch.cuda.synchronize(dev)
    mb_bytes = rows * 40000 * 4
    return {
        "kind": "reference CUDA kernels (patches/ggml-ppdl.patch:212-312) compiled for sm_100a",
        "msda_config1_b32": {"ours_ms": round(ours, 5), "reference_ms": round(theirs, 5),
                             "speedup": round(theirs / ours, 2), "max_abs_diff": msda_diff},
        "mask_box_8_pages": {"ours_ms": round(ours_mb, 5), "reference_ms": round(theirs_mb, 5),
                             "ours_gbs": round(mb_bytes / ours_mb / 1e6, 1),
                             "reference_gbs": round(mb_bytes / theirs_mb / 1e6, 1),
                             "speedup": round(theirs_mb / ours_mb, 2),
                             "max_abs_diff": float((b1 - b2).abs().max())},
    }


def cpu_baseline_forward(gguf, budget_s=10.0, sample_pages=None):
    """The CPU restatement of the reference forward (torch-CPU FP32 dense
    ops + the C restatement of the hot-path ops) on all host threads."""
    import torch
    from oracle import model_ref
    import synth
    nth = os.cpu_count() or 1
    torch.set_num_threads(nth)
    m = model_ref.RefModel(model_ref.load_gguf(gguf))
    pages = [synth.synth_page(5000 + i) for i in range(2)]
    n, t0 = 0, time.perf_counter()
    while True:
        m.forward(pages[n % 2], 800, 800)
        n += 1
        el = time.perf_counter() - t0
        if (sample_pages and n >= sample_pages) or (not sample_pages and el >= budget_s):
            break
    return {"value": round(n / el, 3), "unit": "pages/s", "cores": nth, "kind": "port",
            "sample": f"{n} pages of config 0/3 (full forward + postprocess) in {el:.1f} s; the "
                      "reference ggml CPU path cannot be built here (ggml submodule absent)"}


def run_reference(args, world, rank):
    if rank != 0:
        return None
    if args.workload in ("gemm", "conv", "stress"):
        return {"impl": "reference", "unavailable": f"the {args.workload} workload is a kernel-level "
                "measurement of this build only (its same-box bar, cuBLAS FP32 SGEMM, is part of "
                "the forward workload's config2_conv); the reference arm times the forward"}
    if args.workload == "forward":
        import synth
        gguf = synth.cached_gguf(0)
        for _ in range(max(1, min(args.warmup, 1))):
            cpu_baseline_forward(gguf, sample_pages=1)
        per = []
        K = args.steps
        for _ in range(K):
            r = cpu_baseline_forward(gguf, sample_pages=1)
            per.append(1.0 / r["value"])
        tot = sum(per)
        v = K / tot
        return {
            "metric": METRIC, "impl": "reference", "value": round(v, 3), "unit": "pages/s",
            "n_gpus": world, "steps": K, "warmup": args.warmup,
            "ms_per_step": round(tot / K * 1e3, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic pages and seeded random weights",
            "config": {"workload": "config 3 forward, one page per step (bounded CPU sample)",
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": round(v, 3), "unit": "pages/s", "cores": r["cores"],
                             "kind": r["kind"], "sample": f"1 page per step x {K} steps"},
            "e2e": {"value": round(v, 3), "unit": "pages/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
    if args.workload == "msda":
        K = args.steps
        for _ in range(max(1, args.warmup)):
            cpu_baseline_msda(sample_pages=1)
        per_step = []
        for _ in range(K):
            r = cpu_baseline_msda(sample_pages=MSDA_B)
            per_step.append(MSDA_B / r["value"])
        tot = sum(per_step)
        v = MSDA_B * K / tot
        return {
            "metric": METRIC, "impl": "reference", "value": round(v, 2),
            "unit": "pages/s (MSDeformAttn op, config 1)", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(tot / K * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded numpy RNG)",
            "config": {"workload": "config 1: MSDeformAttn, B=32 pages per step",
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": round(v, 2), "unit": "pages/s", "cores": r["cores"],
                             "kind": r["kind"], "sample": f"{MSDA_B} pages per step x {K} steps"},
            "e2e": {"value": round(v, 2), "unit": "pages/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
    raise SystemExit(f"unknown workload {args.workload}")


# ------------------------------------------------- tensor-core GEMM, standalone
GEMM_SHAPE = (40000, 256, 1024, 8)  # 1x1 conv 1024 -> 256 on 200 x 200 planes, 8 pages


def run_gemm(args, world, rank, local, pg):
    """The dominant kernel alone: ppdl_gemm_tf32x3 (3xTF32 tcgen05) on one
    shape, A M-major (CHW activations), B [N][K] weights; each step is one
    launch over all pages (the weight split included, as the entry point does
    it per call).  Inputs are larger than L2."""
    import ctypes as C
    import torch
    import ppdl
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    M, N, K, B = (tuple(int(v) for v in args.gemm.split(",")) if args.gemm else GEMM_SHAPE)
    L = ppdl.lib()
    L.ppdl_gemm_tf32x3.argtypes = ([C.c_int] * 4 + [C.c_void_p, C.c_int, C.c_longlong,
                                   C.c_longlong, C.c_void_p, C.c_void_p, C.c_void_p]
                                   + [C.c_longlong] * 3 + [C.c_void_p])
    g = torch.Generator(device="cpu").manual_seed(7 + rank)
    A = torch.randn((B, K, M), generator=g).to(dev)
    W = (torch.randn((N, K), generator=g) / K ** 0.5).to(dev)
    ws = torch.empty(2 * N * K, device=dev)
    out = torch.empty((B, N, M), device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        rc = L.ppdl_gemm_tf32x3(M, N, K, B, A.data_ptr(), 1, M, M * K, W.data_ptr(),
                                ws.data_ptr(), out.data_ptr(), 1, M, M * N, stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"ppdl_gemm_tf32x3 returned {rc}: {ppdl.last_error()}")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    barrier(pg)
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(pg)
    clk = clocks.stop()
    ms = max_over_ranks(pg, t0.elapsed_time(t1)) / args.steps
    flops = 2.0 * M * N * K * B
    tflops = flops * world / (ms / 1e3) / 1e12
    hbm, bf16, peak_kind = _peaks()
    tc = bf16 / 6.0
    per_gpu = flops / (ms / 1e3) / 1e12
    return {
        "metric": "3xTF32 tensor-core GEMM TFLOP/s (dominant kernel of the forward, alone)",
        "value": round(tflops, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (3xTF32 on tcgen05)",
        "data": "seeded normal A, weights scaled by 1/sqrt(K)",
        "config": {"workload": f"ppdl_gemm_tf32x3 M={M} N={N} K={K} x {B} pages (CHW A)",
                   "l2": "inputs larger than L2", "parallelism": f"dp{world} (no collective)"},
        "roofline": {"bound": "tensor", "achieved": round(per_gpu, 2), "peak": round(tc, 1),
                     "unit": "TFLOP/s", "frac": round(per_gpu / tc, 4),
                     "peak_kind": f"{peak_kind} bf16 dense burst / 6 (3xTF32)",
                     "algorithmic_bytes": 4 * (M * K * B + M * N * B + 2 * N * K)},
        "gpu_launches": 2 * (args.steps),
        "clocks": clk,
    }


STRESS_PAGES, STRESS_B = 2048, 32


def _stage_of(names):
    """Stage of every plan step of the forward (by its position between
    landmark steps): backbone, encoder (AIFI, FPN/PAN, mask-feature head),
    selection (decoder input, two-stage query selection, initial boxes),
    decoder (the six layers), heads, postprocess."""
    first = {}
    for i, n in enumerate(names):
        first.setdefault(n, i)
    enc0, sel0 = first.get("enc_in0", 0), first.get("dec_in0", 0)
    dec_idx = [i for i, n in enumerate(names) if n.startswith("dec") and n[3:4].isdigit()]
    dec0, dec1 = (dec_idx[0], dec_idx[-1]) if dec_idx else (len(names), len(names))
    out = []
    for i, n in enumerate(names):
        if n == "postprocess":
            out.append("postprocess")
        elif i < enc0:
            out.append("backbone")
        elif i < sel0:
            out.append("encoder")
        elif i < dec0:
            out.append("selection")
        elif i <= dec1:
            out.append("decoder")
        else:
            out.append("heads")
    return out


def config4_stress(dev, world, rank, pg, total_pages=STRESS_PAGES, B=STRESS_B, ctx=None):
    """Config 4 of the baseline: total_pages pages split over the ranks, B
    per GPU per batch, through the pipelined host API (ppdl_submit_batch /
    ppdl_wait_batch: pinned pages in, dets + packed masks out, two batches in
    flight), timed by the host clock, slowest rank; plus the per-stage split
    of one batch (device time of the forward's steps, one after another, and
    the host<->device copies timed alone)."""
    import numpy as np
    import torch
    import ppdl
    import synth
    own = ctx is None
    if own:
        ctx = ppdl.Context(synth.cached_gguf(0), device=dev.index, max_batch=B)
    # a pool of 2B distinct seeded pages, cycled (generating 2048 pages on
    # the host would take minutes); each batch is B distinct pages
    pool = torch.from_numpy(np.stack([synth.synth_page(20000 + rank * 2 * B + i)
                                      for i in range(2 * B)])).pin_memory().numpy()
    hw = np.full((B, 2), 800, np.int32)
    halves = [pool[:B], pool[B:]]  # contiguous views of the pinned pool
    per_rank = (total_pages + world - 1) // world
    n_batches = (per_rank + B - 1) // B
    for i in range(2):
        ctx.wait(ctx.submit(halves[i], hw), B, copy=False)
    torch.cuda.synchronize(dev)
    barrier(pg)
    t0 = time.perf_counter()
    pending = []
    for i in range(n_batches):
        pending.append(ctx.submit(halves[i & 1], hw))
        if len(pending) == 2:
            ctx.wait(pending.pop(0), B, copy=False)
    for t in pending:
        ctx.wait(t, B, copy=False)
    wall = time.perf_counter() - t0
    barrier(pg)
    wall = max_over_ranks(pg, wall)
    pages = n_batches * B * world
    # per-stage split of one batch
    steps = ctx.profile_steps(B)
    stages = {}
    for st_name, (name, kind, ms, fl, by) in zip(_stage_of([x[0] for x in steps]), steps):
        stages[st_name] = stages.get(st_name, 0.0) + ms
    d_in = torch.empty((B, 3, 800, 800), device=dev)
    d_out = torch.empty(B * 300 * (7 + 1250), device=dev)
    h_out = torch.empty(d_out.shape, dtype=torch.float32).pin_memory()
    h_in = torch.from_numpy(halves[0])  # pinned (a view of the pinned pool)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    e[0].record()
    d_in.copy_(h_in, non_blocking=True)
    e[1].record()
    e[2].record()
    h_out.copy_(d_out, non_blocking=True)
    e[3].record()
    torch.cuda.synchronize(dev)
    stages["h2d"] = e[0].elapsed_time(e[1])
    stages["d2h"] = e[2].elapsed_time(e[3])
    if own:
        ctx.close()
    return {"pages": pages, "pages_per_gpu_per_batch": B, "batches_per_gpu": n_batches,
            "wall_s": round(wall, 3), "pages_per_s": round(pages / wall, 2),
            "stage_ms_per_batch": {k: round(v, 3) for k, v in stages.items()},
            "note": "pages cycled from a pool of 2B distinct seeded pages per rank; stage split: "
                    "device time of the forward's steps one after another (lower bounds; the "
                    "captured forward overlaps its three lanes) and the copies of one batch "
                    "timed alone (in the pipelined run they overlap the next batch's forward)"}


def run_stress(args, world, rank, local, pg):
    """--workload stress: config 4 on all ranks (torchrun for N GPUs)."""
    import torch
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    clocks = ClockSampler(local)
    clocks.start()
    r = config4_stress(dev, world, rank, pg, total_pages=args.stress_pages)
    clk = clocks.stop()
    return {
        "metric": METRIC, "value": r["pages_per_s"], "unit": "pages/s", "n_gpus": world,
        "steps": r["batches_per_gpu"], "warmup": 2,
        "ms_per_step": round(r["wall_s"] * 1e3 / r["batches_per_gpu"], 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic pages (config 0 recipe) and seeded random weights",
        "config": {"workload": f"config 4: {args.stress_pages} pages, {STRESS_B} per GPU per "
                               "batch, host pages in / dets + packed masks out",
                   "parallelism": f"dp{world} (pages sharded, no collective)"},
        "e2e": {"value": r["pages_per_s"], "unit": "pages/s",
                "h2d_bytes_per_step": STRESS_B * (3 * 800 * 800 * 4 + 8),
                "d2h_bytes_per_step": STRESS_B * 300 * (7 + 1250) * 4},
        "config4": r, "gpu_launches": r["batches_per_gpu"] * 338, "clocks": clk,
    }


def run_conv(args, world, rank, local, pg):
    """Config 2 of the baseline, one conv shape: the forward's conv path
    through the C ABI (Winograd F(4,3) for 3x3-s1, the 3xTF32 GEMM for 1x1,
    the windowed implicit GEMM for 3x3-s2), weights prepared beforehand as at
    model load (the k3-s2 entry splits its weights in the call), bias + ReLU.
    `value` is conv TFLOP/s on the direct-conv FLOPs 2*B*OH*OW*OC*IC*K^2;
    the L2 is flushed between launches."""
    import ctypes as C
    import torch
    import ppdl
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    kind, IC, H, OC, Bc = (args.conv.split(",") if args.conv else ("3x3-s1", 256, 100, 256, 8))
    IC, H, OC, Bc = int(IC), int(H), int(OC), int(Bc)
    if kind not in ("3x3-s1", "1x1", "3x3-s2"):
        raise SystemExit(f"--conv kind must be 3x3-s1, 1x1 or 3x3-s2, not {kind}")
    hbm, bf16, peak_kind = _peaks()
    tc = bf16 / 6.0
    L = ppdl.lib()
    _bind_conv_entries(L)
    stream = lambda: torch.cuda.current_stream(dev).cuda_stream  # noqa: E731
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    f, direct, executed = _conv_case(L, g, dev, kind, IC, H, OC, Bc, stream)
    for _ in range(args.warmup):
        f()
    torch.cuda.synchronize(dev)
    clocks = ClockSampler(local)
    barrier(pg)
    clocks.start()
    ms = _time_launches(f, dev, iters=args.steps, warmup=0)
    barrier(pg)
    clk = clocks.stop()
    ms = max_over_ranks(pg, ms)
    per_gpu = direct / ms / 1e9
    return {
        "metric": METRIC, "value": round(per_gpu * world, 2), "unit": "conv TFLOP/s (direct FLOPs)",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: activations N(0,1), Kaiming weights, bias N(0,0.1), ReLU",
        "config": {"workload": f"config 2: {kind} conv {H}x{H}x{IC}->{OC}, {Bc} pages",
                   "l2": "flushed between launches (256 MB write, then 256 MB read)", "parallelism": f"dp{world} (no collective)"},
        "roofline": {"bound": "tensor", "achieved": round(executed / ms / 1e9, 2),
                     "peak": round(tc, 1), "unit": "TFLOP/s",
                     "frac": round(executed / ms / 1e9 / tc, 4),
                     "peak_kind": f"{peak_kind} bf16 dense burst / 6 (3xTF32)",
                     "flops": "executed GEMM FLOPs (Winograd: 2*36*T*IC*OC per page)"},
        "gpu_launches": args.steps * (3 if kind == "3x3-s1" else (2 if kind == "3x3-s2" else 1)),
        "clocks": clk,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="forward",
                    choices=["forward", "msda", "gemm", "conv", "stress"])
    ap.add_argument("--stress-pages", type=int, default=STRESS_PAGES,
                    help="stress workload: pages in all (config 4: 2048)")
    ap.add_argument("--conv", default="",
                    help="conv workload: kind,IC,H,OC,pages with kind 3x3-s1, 1x1 or 3x3-s2 "
                         "(default 3x3-s1,256,100,256,8)")
    ap.add_argument("--gemm", default="",
                    help="gemm workload shape M,N,K,pages (default 40000,256,1024,8)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweeps", action="store_true",
                    help="forward workload: skip the config-1 / config-2 kernel sweeps")
    ap.add_argument("--pages", type=int, default=0,
                    help="pages per GPU per step of the forward workload (default 8, config 3); "
                         "smaller values are for profiler captures")
    ap.add_argument("--capture-once", action="store_true",
                    help="forward workload: set up, run one eager forward, print nothing and "
                         "exit (the launch sequence of one forward, for profiler captures)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    world, rank, local, pg = dist_setup(args)
    try:
        if args.impl == "reference":
            line = run_reference(args, world, rank)
        elif args.workload == "forward":
            line = run_forward(args, world, rank, local, pg)
        elif args.workload == "gemm":
            line = run_gemm(args, world, rank, local, pg)
        elif args.workload == "conv":
            line = run_conv(args, world, rank, local, pg)
        elif args.workload == "stress":
            line = run_stress(args, world, rank, local, pg)
        else:
            line = run_msda(args, world, rank, local, pg)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if pg is not None:
            pg.destroy_process_group()


if __name__ == "__main__":
    main()
