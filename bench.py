"""Benchmark of the attention-backward path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload flux|cross|fp16|video] [--no-cpu-baseline]

One step = one backward pass (dQ, dK, dV) over the workload's heads on each
GPU. The default workload is FLUX-like joint self-attention (M=N=4608, d=128,
24 heads, bf16). With N GPUs (launched under torchrun, one rank per GPU),
each rank runs its own 24-head shard of a 24*N-head batch (weak scaling: the
heads are independent, so there is no collective on the data path); NCCL
only gathers per-rank timings and output checksums after the timed region.

Reported (one JSON line from rank 0):
  value       counted TFLOP/s (8*M*N*d*heads, all ranks) / max-over-ranks
              device time of K back-to-back steps, inputs resident in HBM
              (P alone is 1.02 GB per GPU, far larger than the 126 MB L2, so
              no L2 flush is needed between steps; alternate steps also use
              two copies of the inputs, so no step starts on rows the step
              before it left in L2)
  e2e         the same metric through the reference-facing C-ABI call
              (fmha_bwd_full_py) with host buffers: pinned-host -> device
              copies of Q, K, V, P, dO and device -> host copies of dQ, dK, dV
              inside the timed region, every step
  roofline    the backward call (dq_kernel + dkv_kernel) against the
              tensor roofline: achieved = the algorithm's 8*M*N*d*heads
              FLOPs per call / ms_per_step, frac = achieved / the measured
              bf16 peak; traffic = both kernels' DRAM bytes per call (ncu),
              with its ratio to the algorithmic bytes; each kernel's own MMA
              work (6*M*N*d per head) and time under "kernels"
  strong      strong scaling on the long video workload (M=N=16384, d=128,
              40 heads): the 40 heads are split over the N ranks by
              workloads.head_range (40/20/10/5 heads per GPU at N=1/2/4/8),
              P generated per head on the device; per-rank and
              max-over-ranks ms, TFLOP/s and the fraction of the one-GPU
              roofline time
  cpu_baseline  the reference's own CPU backward (cpu_reference.hpp), timed
              on this host's cores on a bounded sample (rank 0, N=1 only)
  recompute_p   the same workload through fmha_bwd_full_lse (P formed on chip
              from the forward's LSE and O), after the timed region

--impl reference times the reference's CPU implementation of the path (the
reference's GPU code is HIP for gfx1100 and cannot run here) on the same
workload, metric and unit: each step is a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "fmha-bwd-gfx1100_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "bwd TFLOP/s (8·M·N·d·H/t) at M=N=4608,d=128,H=24; % of B200 bf16 peak"


def metric_name(w) -> str:
    """The headline metric string for the FLUX workload; the same metric at
    the other workloads' shapes otherwise."""
    if w.name == "flux":
        return METRIC
    return f"bwd TFLOP/s (8·M·N·d·H/t) at M={w.M},N={w.N},d={w.d},H={w.heads}; % of B200 bf16 peak"
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(key: str):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary
    (lines 'key: bytes'), or None."""
    try:
        with open(TRAFFIC_FILE) as f:
            for line in f:
                if ":" in line and not line.lstrip().startswith("#"):
                    k, v = line.rsplit(":", 1)
                    if k.strip() == key:
                        return float(v.split()[0])
    except OSError:
        pass
    return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    QUERY = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.path = os.path.join("/tmp", f"fmha_bench_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            args = ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                    "-lms", "100"]
            if self.uuid:
                args += ["-i", self.uuid]
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(args, stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    rows.append({"sm": float(parts[2]), "max": float(parts[3]),
                                 "power": float(parts[4]), "hw": parts[6], "hwt": parts[7],
                                 "swt": parts[8], "pcap": parts[9]})
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        reasons = set()
        for r in rows:
            if r["hw"] == "Active":
                reasons.add("hw_slowdown")
            if r["hwt"] == "Active":
                reasons.add("hw_thermal_slowdown")
            if r["swt"] == "Active":
                reasons.add("sw_thermal_slowdown")
            if r["pcap"] == "Active":
                reasons.add("sw_power_cap")
        loaded = [r["sm"] for r in rows if r["power"] > 200.0] or [r["sm"] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(r["max"] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows),
                "power_w_max": max(r["power"] for r in rows)}


# ------------------------------------------------------- CPU (reference) leg
def cpu_reference_sample(w, rows: int, threads: int, seed: int = 42):
    """Time the reference's own fmha_backward_cpu on `threads` heads of the
    workload, each restricted to its first `rows` query rows (all N keys, full
    d), one head per thread. Returns (flops, seconds, kind, cores)."""
    from oracle import oracle as O

    kind = "reference" if O.have_reference() else "port"
    Q, K, V, P, dO = O.make_inputs(rows, w.N, w.d, threads, w.dtype, seed=seed,
                                   do_std=w.do_std)
    t0 = time.perf_counter()
    if kind == "reference":
        O.reference_bwd(Q, K, V, P, dO, w.dtype, threads=threads)
    else:
        O.oracle_bwd(Q, K, V, P, dO, w.dtype, threads=threads)
    dt = time.perf_counter() - t0
    return 8.0 * rows * w.N * w.d * threads, dt, kind, threads


def launches_per_call(w, heads: int, sms: int) -> int:
    """Kernels one backward call launches: dq_kernel and dkv_kernel, each
    followed by its combine kernel when the library splits its tail items
    (the library's work-unit rule: items of 16+ steps; the tail split into
    q <= 4 parts of 8+ steps when that saves a tenth of an item time)."""
    def split(items: int, length: int) -> bool:
        if length < 16:
            return False
        tail = items % sms
        if tail == 0:
            return False
        best_q, best = 1, 1.0
        for q in range(2, 5):
            if length // q < 8:
                break
            cost = ((q * tail + sms - 1) // sms) / q
            if cost < best - 0.1:
                best, best_q = cost, q
        return best_q > 1

    mt, nt = -(-w.M // 128), -(-w.N // 128)
    return 2 + int(split(mt * heads, nt)) + int(split(nt * heads, mt))


def cpu_threads(w) -> int:
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    return max(1, min(n, w.heads))


# ------------------------------------------------------------------ helpers
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def run_reference_arm(args, w):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    threads = cpu_threads(w)
    rows = args.cpu_rows_per_step
    if rows <= 0:
        # size each step so the whole run (warm-up + timed) takes ~2 minutes
        fl, dt, _, _ = cpu_reference_sample(w, 16, threads)
        per_row = dt / 16.0
        budget = 120.0 / max(1, args.steps + args.warmup)
        rows = int(budget / max(per_row, 1e-9)) // 8 * 8
        rows = max(8, min(rows, 1024, w.M))
    for _ in range(args.warmup):
        cpu_reference_sample(w, rows, threads)
    times, flops, kind = [], 0.0, "reference"
    for _ in range(args.steps):
        fl, dt, kind, _ = cpu_reference_sample(w, rows, threads)
        times.append(dt)
        flops = fl
    total = sum(times)
    value = flops * len(times) / total / 1e12
    line = {
        "impl": "reference",
        "metric": metric_name(w), "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": w.dtype, "data": "synthetic",
        "config": {"workload": w.description, "M": w.M, "N": w.N, "d": w.d,
                   "heads_per_gpu": w.heads, "parallelism": "cpu threads over heads"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                         "sample": f"per step: first {rows} of {w.M} query rows x {w.N} keys x "
                                   f"d={w.d} for {threads} heads, one head per thread "
                                   "(reference fmha_backward_cpu, cpu_reference.hpp:74-126)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference's GPU path is HIP/rocWMMA for gfx1100 and cannot run on B200; "
                "its CPU implementation of the same path is the reference arm",
    }
    print(json.dumps(line), flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="flux")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-rows", type=int, default=2048,
                    help="query rows per head in the CPU baseline sample (0: all M rows); "
                         "2048 rows of 16 FLUX heads take about 15 s on 16 host cores")
    ap.add_argument("--lse-steps", type=int, default=200,
                    help="timed steps of the recompute-P entry (fmha_bwd_full_lse) on the "
                         "same workload, reported under 'recompute_p' (0: skip)")
    ap.add_argument("--strong-steps", type=int, default=5,
                    help="timed steps of the strong-scaling run on the video workload "
                         "(40 heads split over the ranks; 0: skip)")
    ap.add_argument("--cpu-rows-per-step", type=int, default=0,
                    help="query rows per head per step of the reference arm "
                         "(0: sized so the run takes about two minutes)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    import workloads

    w = workloads.WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference_arm(args, w)

    import torch
    import torch.distributed as dist

    import fmha_bwd_b200 as F

    rank, world, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)

    # ---- inputs: this rank's head shard of a (heads * world)-head batch
    heads = w.heads
    Q, K, V, P, dO = workloads.make_inputs(w, seed=42, device=dev, heads=heads,
                                           head_offset=rank * heads)
    dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)
    lib = F.load_library(w.torch_dtype)
    import ctypes

    ev_fn = lib.fmha_bwd_full_stream_events if w.dtype == "bf16" else \
        lib.fmha_bwd_full_fp16_stream_events
    ev_fn.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_int] * 4 + [ctypes.c_void_p,
                                                                   ctypes.c_void_p]
    ev_fn.restype = ctypes.c_int
    stream = torch.cuda.Stream(device=dev)
    # two copies of the inputs and outputs, used by alternate steps, so that
    # no step starts on rows the step before it left in L2
    sets = [(Q, K, V, P, dO, dQ, dK, dV),
            tuple(t.clone() for t in (Q, K, V, P, dO)) +
            tuple(torch.empty_like(t) for t in (dQ, dK, dV))]
    ptrs = [(s[5].data_ptr(), s[6].data_ptr(), s[7].data_ptr(), s[0].data_ptr(), s[1].data_ptr(),
             s[2].data_ptr(), s[3].data_ptr(), s[4].data_ptr(), w.M, w.N, w.d, heads) for s in sets]

    def step(events_arr=None, k=0):
        rc = ev_fn(*ptrs[k % 2], ctypes.c_void_p(stream.cuda_stream),
                   ctypes.cast(events_arr, ctypes.c_void_p) if events_arr is not None else None)
        if rc != 0:
            raise F.FmhaBwdError(rc, lib.fmha_bwd_last_error_message().decode())

    torch.cuda.synchronize(dev)
    for k in range(args.warmup):
        step(k=k)
    stream.synchronize()
    if lib.fmha_bwd_poll_device_status() != 0:
        raise RuntimeError("device status reported a wait timeout during warm-up")

    # per-step kernel-boundary events, to time the main kernel inside the run
    K_steps = args.steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K_steps)]
    ev_arrays = []
    for e4 in evs:
        for e in e4:
            e.record(stream)  # torch creates the CUDA event lazily, at first record
        if any(not e.cuda_event for e in e4):
            raise RuntimeError("could not create CUDA timing events")
        arr = (ctypes.c_void_p * 4)(*[e.cuda_event for e in e4])
        ev_arrays.append(arr)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)

    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    start.record(stream)
    for k in range(K_steps):
        step(ev_arrays[k], k)
    end.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    ms_total = start.elapsed_time(end)
    if lib.fmha_bwd_poll_device_status() != 0:
        raise RuntimeError("device status reported a wait timeout in the timed region")
    t_dq = [e[0].elapsed_time(e[1]) for e in evs]
    t_dkv = [e[1].elapsed_time(e[2]) for e in evs]

    # ---- gather timings and checksums (NCCL, after the timed region)
    checksum = float(dQ.float().sum().item() + dK.float().sum().item() + dV.float().sum().item())
    if world > 1:
        allt = workloads.gather_rank_stats(dist, [ms_total, statistics.mean(t_dkv), checksum],
                                           dev)
        ms_max = float(allt[:, 0].max())
        main_ms = float(allt[:, 1].max())
        checksums = [float(x) for x in allt[:, 2]]
    else:
        ms_max = ms_total
        main_ms = statistics.mean(t_dkv)
        checksums = [checksum]

    flops_rank = w.flops(heads)
    total_flops = flops_rank * world * K_steps
    value = total_flops / (ms_max * 1e-3) / 1e12
    ms_per_step = ms_max / K_steps

    # ---- e2e through the reference-facing call with host buffers. Every
    # step copies its inputs from pinned host memory, runs the synchronous
    # reference-facing call and copies its results back; steps are
    # pipelined as a user would: step k+1's inputs upload (copy stream, into
    # the other of two device input sets) while step k computes, and step
    # k's results download (a second copy stream, PCIe is full duplex) while
    # step k+1's inputs upload.
    e2e = None
    if args.e2e_steps > 0:
        hQ, hK, hV, hP, hdO = (t.cpu().pin_memory() for t in (Q, K, V, P, dO))
        hin = (hQ, hK, hV, hP, hdO)
        ohQ, ohK, ohV = (torch.empty_like(t, device="cpu").pin_memory() for t in (Q, K, V))
        dev_in = [[torch.empty_like(t) for t in (Q, K, V, P, dO)] for _ in range(2)]
        dev_out = [[torch.empty_like(t) for t in (Q, K, V)] for _ in range(2)]
        h2d = sum(t.numel() * t.element_size() for t in hin)
        d2h = sum(t.numel() * t.element_size() for t in (ohQ, ohK, ohV))
        full = lib.fmha_bwd_full_py if w.dtype == "bf16" else lib.fmha_bwd_full_fp16
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        main = torch.cuda.current_stream(dev)

        def upload(k):
            with torch.cuda.stream(s_in):
                for dst, src in zip(dev_in[k % 2], hin):
                    dst.copy_(src, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(s_in)
            return ev

        def e2e_run(n_steps):
            ev_in = upload(0)
            ev_out = [None, None]
            for k in range(n_steps):
                main.wait_event(ev_in)
                if ev_out[k % 2] is not None:
                    main.wait_event(ev_out[k % 2])  # step k-2's download done
                if k + 1 < n_steps:
                    ev_in = upload(k + 1)
                o, i = dev_out[k % 2], dev_in[k % 2]
                full(*(t.data_ptr() for t in o), *(t.data_ptr() for t in i), w.M, w.N, w.d, heads)
                done = torch.cuda.Event()
                done.record(main)
                s_out.wait_event(done)
                with torch.cuda.stream(s_out):
                    for dst, src in zip((ohQ, ohK, ohV), o):
                        dst.copy_(src, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_out)
                ev_out[k % 2] = ev
            for ev in ev_out:
                if ev is not None:
                    main.wait_event(ev)

        e2e_run(2)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record(main)
        s_in.wait_stream(main)
        s_out.wait_stream(main)
        e2e_run(args.e2e_steps)
        s1.record(main)
        torch.cuda.synchronize(dev)
        e2e_ms = s0.elapsed_time(s1)
        dQ2, dK2, dV2 = dev_out[(args.e2e_steps - 1) % 2]
        if lib.fmha_bwd_last_error() != 0:
            raise RuntimeError(lib.fmha_bwd_last_error_message().decode())
        # the host->device copies alone: this rank's pinned-host copy rate
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        c0.record()
        for _ in range(3):
            for dst, src in zip(dev_in[0], hin):
                dst.copy_(src, non_blocking=True)
        c1.record()
        torch.cuda.synchronize(dev)
        h2d_gbs = 3.0 * h2d / (c0.elapsed_time(c1) * 1e-3) / 1e9
        if world > 1:
            st = workloads.gather_rank_stats(dist, [e2e_ms, h2d_gbs], dev)
            e2e_ms = float(st[:, 0].max())
            h2d_rank = [float(x) for x in st[:, 1]]
        else:
            h2d_rank = [h2d_gbs]
        e2e = {"value": flops_rank * world * args.e2e_steps / (e2e_ms * 1e-3) / 1e12,
               "unit": "TFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": e2e_ms / args.e2e_steps,
               "h2d_gbs_per_rank": h2d_rank,
               "note": "host copies dominate (steps pipelined: uploads overlap the previous "
                       "step's compute and download); every rank's pinned buffers sit in one "
                       "host's memory, so the per-rank copy rate falls as ranks are added",
               "entry": "fmha_bwd_full_py" if w.dtype == "bf16" else "fmha_bwd_full_fp16"}
        if not torch.equal(dK2, dK) or not torch.equal(dV2, dV):
            raise RuntimeError("e2e outputs differ from the device-resident run")
        del hQ, hK, hV, hP, hdO, hin, ohQ, ohK, ohV, dQ2, dK2, dV2, dev_in, dev_out

    # ---- strong scaling: the long video workload's 40 heads split over the
    # ranks (workloads.head_range: 40/20/10/5 heads per GPU at 1/2/4/8 GPUs),
    # each rank generating its heads' inputs (P per head) on its own GPU
    strong = None
    if args.strong_steps > 0:
        wv = workloads.WORKLOADS["video"]
        h0, h1 = workloads.head_range(wv.heads, rank, world)
        nh = h1 - h0
        sstep = None
        if nh > 0:
            sQ, sK, sV, sP, sdO = workloads.make_inputs(wv, seed=42, device=dev, heads=nh,
                                                       head_offset=h0)
            so = (torch.empty_like(sQ), torch.empty_like(sK), torch.empty_like(sV))
            sptrs = (so[0].data_ptr(), so[1].data_ptr(), so[2].data_ptr(), sQ.data_ptr(),
                     sK.data_ptr(), sV.data_ptr(), sP.data_ptr(), sdO.data_ptr(), wv.M, wv.N,
                     wv.d, nh)

            def sstep():
                rc = ev_fn(*sptrs, ctypes.c_void_p(stream.cuda_stream), None)
                if rc != 0:
                    raise F.FmhaBwdError(rc, lib.fmha_bwd_last_error_message().decode())

            for _ in range(2):
                sstep()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        if sstep is not None:
            for _ in range(args.strong_steps):
                sstep()
        a1.record(stream)
        torch.cuda.synchronize(dev)
        if lib.fmha_bwd_poll_device_status() != 0:
            raise RuntimeError("device status reported a wait timeout in the strong-scaling run")
        ms_rank = a0.elapsed_time(a1) / args.strong_steps if sstep is not None else 0.0
        if world > 1:
            st = workloads.gather_rank_stats(dist, [ms_rank, nh], dev)
            ms_ranks = [float(x) for x in st[:, 0]]
            heads_ranks = [int(x) for x in st[:, 1]]
        else:
            ms_ranks, heads_ranks = [ms_rank], [nh]
        s_ms = max(ms_ranks)
        s_flops = wv.flops()
        peaks_s, _ = load_peaks()
        roof1_ms = s_flops / (float(peaks_s["bf16_tflops"]) * 1e12) * 1e3
        strong = {
            "workload": wv.description, "scaling": "strong", "total_heads": wv.heads,
            "heads_per_rank": heads_ranks, "ms_per_step_per_rank": ms_ranks,
            "ms_per_step": s_ms, "steps": args.strong_steps,
            "value": s_flops / (s_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "one_gpu_roofline_ms": roof1_ms,
            "frac_of_roofline": (roof1_ms / world) / s_ms,
        }
        if sstep is not None:
            del sQ, sK, sV, sP, sdO, so
        torch.cuda.empty_cache()

    # ---- the recompute-P entry on the same workload: P = exp(scale Q K^T - LSE)
    # formed on chip from the forward's LSE and O (scale = 1/sqrt(d), the
    # scale the synthetic P was made with), 14*M*N*d of MMA work per head.
    recompute_p = None
    if args.lse_steps > 0:
        import math

        scale = 1.0 / math.sqrt(w.d)
        LSE = torch.empty(heads, w.M, device=dev, dtype=torch.float32)
        Ofwd = torch.empty_like(Q)
        for h in range(heads):
            S = (Q[h].float() @ K[h].float().T) * scale
            LSE[h] = torch.logsumexp(S, dim=-1)
            Ofwd[h] = (torch.exp(S - LSE[h][:, None]) @ V[h].float()).to(Q.dtype)
            del S
        lse_out = (torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V))

        def lse_step():
            F.fmha_bwd_lse(Q, K, V, Ofwd, dO, LSE, scale, out=lse_out, stream=stream, sync=False)

        for _ in range(args.warmup):
            lse_step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        l0 = torch.cuda.Event(enable_timing=True)
        l1 = torch.cuda.Event(enable_timing=True)
        l0.record(stream)
        for _ in range(args.lse_steps):
            lse_step()
        l1.record(stream)
        torch.cuda.synchronize(dev)
        lse_ms = l0.elapsed_time(l1)
        if lib.fmha_bwd_poll_device_status() != 0:
            raise RuntimeError("device status reported a wait timeout in the recompute-P run")
        if world > 1:
            t = torch.tensor([lse_ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            lse_ms = float(t.item())
        # dV = P^T dO does not depend on D: it must agree with the P-reading run
        rel = float((lse_out[2].float() - dV.float()).norm() / dV.float().norm().clamp_min(1e-30))
        if not rel < 2e-2:
            raise RuntimeError(f"recompute-P dV differs from the P-reading run (rel-L2 {rel:.3g})")
        recompute_p = {
            "entry": "fmha_bwd_full_lse" if w.dtype == "bf16" else "fmha_bwd_full_fp16_lse",
            "value": flops_rank * world * args.lse_steps / (lse_ms * 1e-3) / 1e12,
            "unit": "TFLOP/s (same counted 8*M*N*d per head)",
            "ms_per_step": lse_ms / args.lse_steps, "steps": args.lse_steps,
            "mma_work_per_head": "14*M*N*d (adds S = Q K^T in both kernels; reads no P)",
            "dV_rel_l2_vs_P_path": rel,
        }
        del LSE, Ofwd, lse_out

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    peaks, peak_src = load_peaks()
    peak = float(peaks["bf16_tflops"])
    peak_sus = float(peaks.get("bf16_tflops_sustained", peak))
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    # the whole call (both kernels) against the tensor roofline: the
    # algorithm's 8*M*N*d FLOPs per head over the measured time per step
    achieved = flops_rank / (ms_per_step * 1e-3) / 1e12
    dq_ms = statistics.mean(t_dq)
    mma_flops = 0.75 * flops_rank  # each kernel issues 6*M*N*d of MMA work per head
    t_dq_traffic = load_traffic(f"dq_kernel:{w.name}")
    t_dkv_traffic = load_traffic(f"dkv_kernel:{w.name}")
    traffic = (t_dq_traffic + t_dkv_traffic
               if t_dq_traffic is not None and t_dkv_traffic is not None else None)
    alg_bytes = w.algorithmic_bytes(heads)
    roofline = {
        "kernel": "backward call: dq_kernel + dkv_kernel (8*M*N*d per head counted)",
        "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
        "frac": achieved / peak, "traffic": traffic,
        "algorithmic_bytes": alg_bytes,
        "traffic_over_algorithmic": traffic / alg_bytes if traffic else None,
        "bytes_roof_ms": alg_bytes / (hbm * 1e9) * 1e3,
        "flops_roof_ms": flops_rank / (peak * 1e12) * 1e3,
        "peak_source": f"{peak_src} (bf16 burst, MEASURED_PEAKS.json)" if peak_src == "measured"
        else "fallback 1.59 PFLOP/s",
        "frac_of_sustained": achieved / peak_sus,
        "kernels": {
            "dq_kernel": {"ms": dq_ms, "mma_tflops": mma_flops / (dq_ms * 1e-3) / 1e12,
                          "mma_frac": mma_flops / (dq_ms * 1e-3) / 1e12 / peak,
                          "traffic": t_dq_traffic},
            "dkv_kernel": {"ms": main_ms, "mma_tflops": mma_flops / (main_ms * 1e-3) / 1e12,
                           "mma_frac": mma_flops / (main_ms * 1e-3) / 1e12 / peak,
                           "traffic": t_dkv_traffic},
            "mma_work": "each kernel issues 6*M*N*d of MMA work per head (12 in all for the "
                        "8 counted): dP in both, then B = P K and A = E K in dq_kernel, dV "
                        "and dK in dkv_kernel",
        },
    }
    line = {
        "metric": metric_name(w), "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": K_steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": w.dtype, "data": "synthetic",
        "config": {"workload": w.description, "M": w.M, "N": w.N, "d": w.d,
                   "heads_per_gpu": heads, "total_heads": heads * world,
                   "parallelism": f"head-sharded x{world}, no data-path collective",
                   "l2": f"inputs larger than L2 (P is {P.numel() * P.element_size() / 1e9:.2f} GB "
                         "per GPU vs 126 MB L2), and alternate steps use two copies of the "
                         "inputs; no flush"},
        "e2e": e2e,
        "strong": strong,
        "recompute_p": recompute_p,
        "gpu_launches": launches_per_call(
            w, heads, torch.cuda.get_device_properties(dev).multi_processor_count) * K_steps,
        "roofline": roofline,
        "clocks": clocks,
        "checksums": checksums,
    }
    if world == 1 and not args.no_cpu_baseline:
        threads = cpu_threads(w)
        rows = args.cpu_rows if args.cpu_rows > 0 else w.M
        fl, dt, kind, cores = cpu_reference_sample(w, rows, threads)
        line["cpu_baseline"] = {
            "value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": kind,
            "sample": f"{rows} of {w.M} query rows x {w.N} keys x d={w.d} for {threads} of "
                      f"{w.heads} heads, one head per thread (reference fmha_backward_cpu), "
                      f"{dt:.1f} s",
        }
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
