"""Benchmark of the spTiles hot path on B200: matmul TFLOP/s and vector_add HBM GB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Under torchrun (N > 1) each rank drives one GPU; the work is sharded with the
library's partitioner (matmul by M-row blocks, vector_add by element range:
strong scaling, total work fixed) and the reported time is the maximum over
ranks of the device-timed region.  Rank 0 prints one JSON line.

Workloads (synthetic inputs of the configured shapes and distributions):
  matmul_f16     C[8192,8192] f32 = A f16 @ B f16, A,B ~ N(0, 0.1), seed 3   (default headline)
  matmul_bf16    C[32768,4096] bf16 = A bf16 @ B bf16 + bias, N(0, 0.05), seed 4
  matmul_fp32    C[1024,1024] = A @ B, f32 via 3xTF32, N(0, 1), seed 2
  vector_add_2d  C = A + B, f32 4096 x 4096, U[-1, 1), seed 1
  vector_add_1d  C = A + B, f32 2^20, U[-1, 1), seed 0
The default run also measures vector_add_2d and reports it under "vecadd".

A step is one call of the hot path over one batch.  Device time: CUDA events
on the stream the kernels run on, bracketed by a barrier and a synchronize.
Between timed steps either the inputs exceed the 126 MB L2 (matmul), or the
step rotates through enough buffer sets to exceed it (vector_add).

--impl reference times the reference's algorithm on the host cores instead:
the CPU restatement of its shader arithmetic (the reference itself cannot be
built or run here), on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "matmul TFLOP/s & vecadd HBM GB/s at 1/2/4/8 B200, % of roofline"
L2_BYTES = 126 * 1024 * 1024

WORKLOADS = {
    "matmul_f16": dict(kind="matmul", m=8192, n=8192, k=8192, dtype="f16", out="f32", bias=False, std=0.1, seed=3),
    "matmul_bf16": dict(kind="matmul", m=32768, n=4096, k=4096, dtype="bf16", out="bf16", bias=True, std=0.05,
                        seed=4),
    "matmul_fp32": dict(kind="matmul", m=1024, n=1024, k=1024, dtype="f32", out="f32", bias=False, std=1.0, seed=2),
    "vector_add_2d": dict(kind="vector_add", shape=(4096, 4096), seed=1),
    "vector_add_1d": dict(kind="vector_add", shape=(2 ** 20,), seed=0),
}


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--workload", default="matmul_f16", choices=sorted(WORKLOADS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-secondary", action="store_true", help="skip the vector_add measurement of the default run")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--replicate", choices=["fused", "nccl"], default=None,
                   help="matmul: every step leaves the full C on every rank. fused: the GEMM epilogue stores each "
                        "C chunk into every rank's copy over NVLink peer memory; nccl: the GEMM, then an NCCL "
                        "all-gather of the row blocks")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-sweep", action="store_true", help="vector_add_1d: skip the N = 2^20 .. 2^28 sweep")
    p.add_argument("--m", type=int, default=None,
                   help="matmul: rows of C in place of the configuration's M (a single GPU's share of a sharded "
                        "run, e.g. 1024 = 8192 / 8, for profiling)")
    p.add_argument("--sustain-steps", type=int, default=300,
                   help="matmul: after the timed steps, this many more back to back, reported under "
                        "'sustained' with their own clock record (0: skip)")
    p.add_argument("--timing", choices=["auto", "graph", "eager"], default="auto",
                   help="graph: replay the K timed steps from one CUDA graph (host launch overhead out of the "
                        "timed region); eager: launch every step from the host; auto: graph for the "
                        "launch-bound vector_add workloads, eager for the matmuls")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


def measured_peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def _traffic_line(key: str):
    """Fields of the summary line for `key`: key, bytes, read, write, note."""
    f = ROOT / "profiles" / "traffic_per_launch.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        parts = line.split(None, 4)
        if len(parts) >= 2 and parts[0] == key:
            return parts
    return None


def profile_traffic(key: str):
    """DRAM bytes (read + write) per launch from the committed ncu summary, if one exists."""
    parts = _traffic_line(key)
    if parts is None:
        return None
    try:
        return float(parts[1])
    except ValueError:
        return None


def profile_traffic_note(key: str):
    parts = _traffic_line(key)
    return parts[4].strip() if parts is not None and len(parts) > 4 else None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock, power and clock-event reasons through NVML while running."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples, self.power_w, self.reasons, self.max_mhz = [], [], 0, None
        self._stop = threading.Event()
        self._thread = None
        self.error = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # pragma: no cover - depends on the box
            self._nv = None
            self.error = str(e)
        self.period = period_s

    def _run(self):
        nv = self._nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= int(get_reasons(self._h))
                self.power_w.append(nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0)
            except Exception as e:  # pragma: no cover
                self.error = str(e)
                return
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self, ms_per_launch=None):
        """Median SM clock, the samples binned by 100 MHz, power, and (given the
        device time of one launch) the SM cycles one launch takes at that clock."""
        if self._nv is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": len(self.samples),
                    "note": self.error or "no samples"}
        bins = {}
        for mhz in self.samples:
            lo = int(mhz) // 100 * 100
            key = f"{lo}-{lo + 99}"
            bins[key] = bins.get(key, 0) + 1
        med = statistics.median(self.samples)
        out = {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "sm_mhz_min": min(self.samples),
               "reasons": [v for k, v in self.REASONS.items() if self.reasons & k], "samples": len(self.samples),
               "sm_mhz_bins": dict(sorted(bins.items())),
               "power_w_median": round(statistics.median(self.power_w), 1) if self.power_w else None,
               "power_w_max": round(max(self.power_w), 1) if self.power_w else None,
               "source": "NVML every 2 ms during the timed region"}
        if ms_per_launch:
            out["cycles_per_launch_at_median_mhz"] = int(ms_per_launch * 1e-3 * med * 1e6)
        return out


# ------------------------------------------------------------------ inputs
def torch_dtype(name):
    import torch
    return {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[name]


def make_matmul_inputs(wl, rows, device, seed_offset=0):
    """This rank's A rows, B and bias, generated on the device."""
    import torch
    g = torch.Generator(device=device).manual_seed(wl["seed"] * 1000 + seed_offset)
    dt = torch_dtype(wl["dtype"])
    a = (torch.randn((rows, wl["k"]), generator=g, device=device) * wl["std"]).to(dt)
    gb = torch.Generator(device=device).manual_seed(wl["seed"] * 1000 + 999)
    b = (torch.randn((wl["k"], wl["n"]), generator=gb, device=device) * wl["std"]).to(dt)
    bias = None
    if wl["bias"]:
        bias = (torch.rand(wl["n"], generator=gb, device=device) * 2 - 1).to(dt)
    return a, b, bias


def matmul_buffer_sets(wl, rows):
    """Buffer sets a matmul step rotates through: operands and C that fit in
    the L2 (fp32 1024^3: 12 MB) get enough copies that one pass over them
    exceeds twice the L2, so every step reads its inputs from HBM."""
    elem = {"f32": 4, "f16": 2, "bf16": 2}
    set_bytes = (rows * wl["k"] + wl["k"] * wl["n"]) * elem[wl["dtype"]] + rows * wl["n"] * elem[wl["out"]]
    if rows == 0 or set_bytes > L2_BYTES:
        return 1
    return min(64, 2 * L2_BYTES // set_bytes + 1)  # strictly more than twice the L2


def flops_of(wl, rows):
    f = 2.0 * rows * wl["n"] * wl["k"]
    if wl["bias"]:
        f += rows * wl["n"]
    return f


# ------------------------------------------------------------------ our arm
def gpu_spin(stream, cycles=2_000_000):
    """A ~1 ms busy kernel on `stream` (torch's spin kernel), so that the host
    can queue the next launches before the GPU reaches them; skipped where
    this torch has no such kernel."""
    import torch
    spin = getattr(torch.cuda, "_sleep", None)
    if spin is not None:
        with torch.cuda.stream(stream):
            spin(cycles)


def time_steps(fn, steps, warmup, stream, dist_on, graph=True, stats=None):
    """Device time (ms) of `steps` calls of `fn` after `warmup` calls.

    With ``graph`` the timed calls are captured once into a CUDA graph and
    the timed region is one replay of it: every step is still one full call
    of the hot path, but the host's per-call launch overhead leaves the
    timed region (what a launch-bound inner loop does in production).
    Without it and with ``stats``, the same steps run once more right after
    the timed region with an event between steps (events between launches
    would perturb the timed region itself), and each step's own device time
    is summarised into ``stats`` (first / last / min / median / max ms),
    which shows the clock settling under the power cap.
    Returns (ms, launches issued by the library for the timed steps).
    """
    import torch
    import torch.distributed as dist
    import sptiles_b200 as st
    for _ in range(warmup):
        fn(-1)
    torch.cuda.synchronize()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        before = st.kernel_launches()
        with torch.cuda.graph(g):
            for i in range(steps):
                fn(i)
        launches = st.kernel_launches() - before
        g.replay()  # upload the graph; untimed
        torch.cuda.synchronize()
    if dist_on:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream()
    if g is None:
        before = st.kernel_launches()
        # Keep the GPU busy (a spin of ~1 ms, before the start event) while the
        # host enqueues the first steps, so the timed region does not include
        # the GPU idling for the host's first launch: the steps still run back
        # to back as the host issues them, and the events bracket exactly them.
        gpu_spin(stream)
    start.record(stream)
    if g is not None:
        g.replay()
    else:
        for i in range(steps):
            fn(i)
    end.record(stream)
    torch.cuda.synchronize()
    if g is None:
        launches = st.kernel_launches() - before
        if stats is not None and steps > 1:
            # the per-step pass (untimed as a whole)
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
            gpu_spin(stream)
            ev[0].record(stream)
            for i in range(steps):
                fn(i)
                ev[i + 1].record(stream)
            torch.cuda.synchronize()
            per = [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]
            stats.update({"first": round(per[0], 5), "last": round(per[-1], 5), "min": round(min(per), 5),
                          "median": round(statistics.median(per), 5), "max": round(max(per), 5),
                          "how": "the same steps again after the timed region, an event between steps"})
    if dist_on:
        dist.barrier()
    del g
    return start.elapsed_time(end), launches


def use_graph(args, wl):
    if args.timing == "auto":
        return wl["kind"] == "vector_add"
    return args.timing == "graph"


def max_over_ranks(x, dist_on):
    if not dist_on:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, dist_on):
    if not dist_on:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def run_matmul(wl, args, rank, world, local, dist_on, peaks):
    import torch
    import sptiles_b200 as st
    from sptiles_b200.partition import gather_row_shards, matmul_row_shard

    dev = torch.device("cuda", local)
    r0, r1 = matmul_row_shard(wl["m"], world, rank)
    rows = r1 - r0
    a, b, bias = make_matmul_inputs(wl, rows, dev, seed_offset=rank)
    out_dt = torch_dtype(wl["out"])
    c = torch.empty((rows, wl["n"]), dtype=out_dt, device=dev)
    stream = torch.cuda.current_stream(dev)

    replicate = args.replicate if dist_on else None
    c_full = torch.empty((wl["m"], wl["n"]), dtype=out_dt, device=dev) if replicate else None
    if replicate == "nccl" and wl["m"] % (world * 128) == 0:
        # equal shards: the GEMM writes its rows of the full C and the NCCL
        # all-gather runs in place (as partition.sharded_matmul does)
        c = c_full[r0:r1]
    rep = None
    if replicate == "fused":
        from sptiles_b200.partition import ReplicatedOutput
        rep = ReplicatedOutput(wl["m"], wl["n"], out_dt)
    sets = 1 if replicate else matmul_buffer_sets(wl, rows)
    bufs = [(a, b, c)] + [(a.clone(), b.clone(), torch.empty_like(c)) for _ in range(sets - 1)]

    def step(i):
        if rep is not None:
            rep.matmul(a, b, bias)
            return
        if rows:
            aa, bb, cc = bufs[i % sets]
            st.matmul(aa, bb, bias, out=cc)
        if replicate:
            gather_rows()

    def gather_rows():
        if c_full is not None and c.data_ptr() == c_full[r0:r1].data_ptr():
            torch.distributed.all_gather_into_tensor(c_full, c, group=None)
        else:
            gather_row_shards(c, wl["m"], out=c_full)

    step_stats = {}
    with ClockSampler(local) as clk:
        ms, launches = time_steps(step, args.steps, args.warmup, stream, dist_on,
                                  graph=use_graph(args, wl) and not replicate, stats=step_stats)
    ms_max = max_over_ranks(ms, dist_on)
    sustained = None
    if getattr(args, "sustain_steps", 0) and not replicate:
        # the same steps back to back for a few hundred ms: the clock the
        # 1000 W cap settles at, beside the short timed region's burst figure
        n_s = args.sustain_steps
        sus_stats = {}
        with ClockSampler(local) as sclk:
            s_ms, _ = time_steps(step, n_s, 0, stream, dist_on, graph=False, stats=sus_stats)
        s_max = max_over_ranks(s_ms, dist_on)
        sustained = {"steps": n_s, "ms_per_step": round(s_max / n_s, 5),
                     "value": round(sum_over_ranks(flops_of(wl, rows), dist_on) * n_s / (s_max / 1e3) / 1e12, 3),
                     "step_ms": sus_stats, "clocks": sclk.summary(s_ms / n_s)}
    gather = None
    kernel_ms = ms  # this rank's device time of the GEMM launches alone
    if replicate:
        def gemm_only(_i):
            if rows:
                st.matmul(a, b, bias, out=c)

        def gather_only(_i):
            gather_rows()

        def gemm_then_nccl(_i):
            gemm_only(_i)
            gather_only(_i)
        kernel_ms, _ = time_steps(gemm_only, args.steps, 2, stream, dist_on, graph=False)
        g_ms, _ = time_steps(gather_only, args.steps, 2, stream, dist_on, graph=False)
        g_ms = max_over_ranks(g_ms, dist_on) / args.steps
        gemm_ms = max_over_ranks(kernel_ms, dist_on) / args.steps
        recv = (wl["m"] - rows) * wl["n"] * c.element_size()
        gather = {"mode": replicate, "step_ms": round(ms_max / args.steps, 4), "gemm_alone_ms": round(gemm_ms, 4),
                  "nccl_allgather_alone_ms": round(g_ms, 4), "bytes_received_per_rank": int(recv),
                  "nccl_GBps_per_rank": round(recv / (g_ms / 1e3) / 1e9, 1)}
        if replicate == "fused":
            n_ms, _ = time_steps(gemm_then_nccl, args.steps, 2, stream, dist_on, graph=False)
            gather["gemm_then_nccl_step_ms"] = round(max_over_ranks(n_ms, dist_on) / args.steps, 4)
            gather["how"] = ("the GEMM epilogue stores each C chunk into every rank's copy (CUDA IPC peer "
                             "pointers over NVLink), then a one-element NCCL all-reduce orders the ranks")
        else:
            gather["how"] = "the GEMM, then torch.distributed.all_gather_into_tensor (NCCL) of the C row blocks"
        gather["overhead_over_gemm_ms"] = round(ms_max / args.steps - gemm_ms, 4)
    total_flops = sum_over_ranks(flops_of(wl, rows), dist_on)
    value = total_flops * args.steps / (ms_max / 1e3) / 1e12
    per_launch_ms = kernel_ms / args.steps
    achieved = flops_of(wl, rows) / (per_launch_ms / 1e3) / 1e12 if rows else 0.0
    peak = peaks["bf16_tflops"]
    peak_sus = peaks.get("bf16_tflops_sustained") or peak
    if wl["dtype"] == "f32":
        peak = peaks["bf16_tflops"] / 2.0 / 3.0  # tf32 runs at half the 16-bit rate, 3 passes
        peak_sus = peak_sus / 2.0 / 3.0
    key = f"matmul_{wl['dtype']}_{wl['m']}x{wl['n']}x{wl['k']}"
    traffic = profile_traffic(key) if world == 1 else None  # captured on the 1-GPU workload
    plan = st.matmul_plan({"f16": 1, "bf16": 2, "f32": 0}[wl["dtype"]], rows or 1, wl["n"], wl["k"])
    roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4),
            "peak_note": ("of measured dense bf16 cuBLAS burst peak (fp16 has the same dense rate)"
                          if wl["dtype"] != "f32" else "of measured bf16 peak / 2 (tf32 rate) / 3 (3xTF32 passes)")
            if peaks["source"] == "measured" else "of fallback peak",
            "traffic": traffic, "ms_per_launch": round(per_launch_ms, 4),
            "kernel": "gemm_tc_pair_kernel" if plan["block_m"] == 256 else "gemm_tc_kernel",
            # the timed steps run back to back into the 1000 W cap: the measured
            # sustained (seconds-long cuBLAS loop) peak, for comparison
            "peak_sustained": round(peak_sus, 1), "frac_sustained": round(achieved / peak_sus, 4)}
    if traffic is not None:
        roof["traffic_note"] = profile_traffic_note(key)
    out = dict(value=value, ms_per_step=ms_max / args.steps, roofline=roof, gpu_launches=int(launches),
               clocks=clk.summary(ms / args.steps), plan=plan, rows=rows, allgather=gather)
    if step_stats:
        out["step_ms"] = step_stats
    if sustained:
        out["sustained"] = sustained
    if rep is not None:
        rep.close()
    del bufs[1:]
    if not args.no_e2e:
        out["e2e"] = e2e_matmul(wl, args, a, b, bias, out_dt, rows, dist_on)
    return out


def host_link_probe(dev, h2d_bytes, d2h_bytes, dist_on):
    """Pinned-memory copy rates of this box's host link, measured with the
    e2e step's own byte counts: H2D alone, D2H alone, and both at once on two
    streams (what a pipelined step overlaps).  With N ranks all ranks copy at
    once, as their e2e steps do.  Returns GB/s figures and the link-bound
    time of one step: max(H2D, D2H) bytes at the concurrent rates."""
    import torch
    nb_in, nb_out = max(h2d_bytes, 1 << 20), max(d2h_bytes, 1 << 20)
    h_in = torch.empty(nb_in, dtype=torch.uint8).pin_memory()
    h_out = torch.empty(nb_out, dtype=torch.uint8).pin_memory()
    d_in = torch.empty(nb_in, dtype=torch.uint8, device=dev)
    d_out = torch.empty(nb_out, dtype=torch.uint8, device=dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def timed(do_in, do_out, reps=3):
        """Best of `reps`: (wall s, H2D s, D2H s), the per-direction times from
        events on each copy stream, all started together."""
        best = (float("inf"), 0.0, 0.0)
        for _ in range(reps):
            torch.cuda.synchronize(dev)
            if dist_on:
                import torch.distributed as dist
                dist.barrier()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            t0 = time.perf_counter()
            if do_in:
                with torch.cuda.stream(s_in):
                    ev[0].record()
                    d_in.copy_(h_in, non_blocking=True)
                    ev[1].record()
            if do_out:
                with torch.cuda.stream(s_out):
                    ev[2].record()
                    h_out.copy_(d_out, non_blocking=True)
                    ev[3].record()
            torch.cuda.synchronize(dev)
            wall = time.perf_counter() - t0
            if wall < best[0]:
                best = (wall, ev[0].elapsed_time(ev[1]) / 1e3 if do_in else 0.0,
                        ev[2].elapsed_time(ev[3]) / 1e3 if do_out else 0.0)
        return best
    t_in, t_out, (t_both, t_in_c, t_out_c) = timed(True, False)[0], timed(False, True)[0], timed(True, True)
    bound_s = t_both if h2d_bytes and d2h_bytes else max(t_in * h2d_bytes / nb_in, t_out * d2h_bytes / nb_out)
    return {"h2d_GBps": round(nb_in / t_in / 1e9, 1), "d2h_GBps": round(nb_out / t_out / 1e9, 1),
            "both_GBps": round((nb_in + nb_out) / t_both / 1e9, 1),
            "h2d_GBps_concurrent": round(nb_in / max(t_in_c, 1e-9) / 1e9, 1),
            "d2h_GBps_concurrent": round(nb_out / max(t_out_c, 1e-9) / 1e9, 1),
            "ms_per_step": round(bound_s * 1e3, 3),
            "how": "pinned copies of this step's H2D and D2H byte counts on two streams at once (best of 3)"}


def growing_blocks_bound_ms(h2d_bytes, d2h_bytes, h2d_gbps, d2h_gbps):
    """Least time of a pipelined C = A @ B over the host link whose output can
    leave only after its inputs arrived.  Row blocks of A and column blocks of
    B arrive together, so after a fraction f of the input bytes a fraction f^2
    of C is computable (the most any order gives for that much input).  With
    the input done at T_in = in / r_in, the output's copy-out is limited by
    what is available until t* = r_out T_in^2 / (2 out), and by r_out after
    that: T = t* + out (1 - (t* / T_in)^2) / r_out (T = T_in when t* >= T_in)."""
    r_in, r_out = h2d_gbps * 1e9, d2h_gbps * 1e9
    t_in = h2d_bytes / r_in
    if d2h_bytes <= 0:
        return t_in * 1e3
    t_star = r_out * t_in * t_in / (2.0 * d2h_bytes)
    if t_star >= t_in:
        return t_in * 1e3
    return (t_star + d2h_bytes * (1.0 - (t_star / t_in) ** 2) / r_out) * 1e3


def e2e_matmul(wl, args, a, b, bias, out_dt, rows, dist_on):
    """Same metric through the public API on pinned host buffers (copies in the timed region).

    One GPU: sptiles_b200.matmul on host tensors (st_matmul_host).  N GPUs:
    partition.sharded_matmul_host on each rank (its rows of A, 1/N of B's
    rows copied and all-gathered over NVLink, its rows of C back).  Byte
    counts are the whole job's per step."""
    import torch
    import sptiles_b200 as st
    from sptiles_b200.partition import sharded_matmul_host
    ha = a.cpu().pin_memory()
    hb = b.cpu().pin_memory()
    hbias = bias.cpu().pin_memory() if bias is not None else None
    hc = torch.empty((rows, wl["n"]), dtype=out_dt).pin_memory()
    steps = max(1, min(args.steps, 10))

    def step():
        if dist_on:
            sharded_matmul_host(ha, hb, hbias, m_total=wl["m"], out=hc)
        elif rows:
            st.matmul(ha, hb, hbias, out=hc)  # returns once C is back in host memory
    for _ in range(2):
        step()
    if dist_on:
        import torch.distributed as dist
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = time.perf_counter() - t0
    dt = max_over_ranks(dt, dist_on)
    total_flops = sum_over_ranks(flops_of(wl, rows), dist_on)
    h2d = sum_over_ranks(ha.numel() * ha.element_size() + (hbias.numel() * hbias.element_size() if hbias is not None
                                                           else 0), dist_on) + hb.numel() * hb.element_size()
    d2h = sum_over_ranks(hc.numel() * hc.element_size(), dist_on)
    how = ("partition.sharded_matmul_host on each rank: its rows of A and 1/N of B's rows H2D, B all-gathered "
           "over NCCL, GEMM, its rows of C D2H" if dist_on else
           "sptiles_b200.matmul on pinned host tensors (st_matmul_host): H2D, kernel, D2H")
    value = total_flops * steps / dt / 1e12
    # per rank: its rows of A and its 1/N of B's rows in, its rows of C out
    world = torch.distributed.get_world_size() if dist_on else 1
    rank_h2d = ha.numel() * ha.element_size() + hb.numel() * hb.element_size() // world
    rank_d2h = hc.numel() * hc.element_size()
    link = host_link_probe(a.device, rank_h2d, rank_d2h, dist_on)
    bound_ms = max_over_ranks(link["ms_per_step"], dist_on)
    link["value"] = round(total_flops / (bound_ms / 1e3) / 1e12, 3)
    link["frac"] = round(value / link["value"], 4)
    # the same link with the dependency of C on A's rows and B's columns (one
    # GPU; with N ranks B's rows are all-gathered over NVLink, which the
    # growing-block model does not describe)
    if not dist_on:
        sched_ms = growing_blocks_bound_ms(rank_h2d, rank_d2h, link["h2d_GBps_concurrent"],
                                           link["d2h_GBps_concurrent"])
        link["schedule_ms_per_step"] = round(sched_ms, 3)
        link["schedule_value"] = round(total_flops / (sched_ms / 1e3) / 1e12, 3)
        link["schedule_frac"] = round(value / link["schedule_value"], 4)
        link["schedule_how"] = ("C's blocks leave only after their rows of A and columns of B arrived: with rows "
                                "and columns growing together, f of the input makes f^2 of C; time = input at "
                                "the concurrent H2D rate, output at the concurrent D2H rate under that "
                                "availability")
    return {"value": round(value, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "steps": steps, "how": how + " per step, host wall clock",
            "link_bound": link}


def vector_add_sweep(dev, peaks, exps=(20, 22, 24, 26, 28)):
    """1D add at N = 2^20 .. 2^28 fp32: HBM GB/s (12 bytes per element) and
    its fraction of the measured copy bandwidth.  Steps rotate through buffer
    sets totalling > 2x L2 (one set from 2^24 up: 201 MB and more), ~50 ms of
    graph-replayed steps per size after 3 warm-up steps."""
    import torch
    import sptiles_b200 as st
    rows = []
    for e in exps:
        n = 2 ** e
        sets = min(64, max(1, 2 * L2_BYTES // (12 * n) + 1))
        bufs = [(torch.rand(n, device=dev) * 2 - 1, torch.rand(n, device=dev) * 2 - 1, torch.empty(n, device=dev))
                for _ in range(sets)]
        steps = int(min(2000, max(20, 0.05 / (12 * n / (peaks["hbm_gbs"] * 1e9)))))

        def step(i, bufs=bufs, sets=sets):
            a, b, c = bufs[i % sets]
            st.vector_add(a, b, out=c)
        ms, _ = time_steps(step, steps, 3, torch.cuda.current_stream(dev), False, graph=True)
        gbs = 12 * n * steps / (ms / 1e3) / 1e9
        rows.append({"n": n, "GBps": round(gbs, 1), "frac": round(gbs / peaks["hbm_gbs"], 4), "steps": steps,
                     "buffer_sets": sets, "us_per_launch": round(ms / steps * 1e3, 2)})
        del bufs
        torch.cuda.empty_cache()
    return rows


def run_vector_add(wl, args, rank, world, local, dist_on, peaks):
    import torch
    import sptiles_b200 as st
    from sptiles_b200.partition import vector_add_shard

    dev = torch.device("cuda", local)
    total = math.prod(wl["shape"])
    e0, e1 = vector_add_shard(total, world, rank)
    n = e1 - e0
    bytes_per_step = 12 * n
    # enough buffer sets that one round trip exceeds twice the L2
    sets = max(1, 2 * L2_BYTES // max(1, bytes_per_step) + 1)
    sets = min(sets, 64)
    g = torch.Generator(device=dev).manual_seed(wl["seed"] * 1000 + rank)
    shape_local = (n,) if len(wl["shape"]) == 1 else None
    bufs = []
    for _ in range(sets):
        a = torch.rand(n, generator=g, device=dev) * 2 - 1
        b = torch.rand(n, generator=g, device=dev) * 2 - 1
        c = torch.empty(n, device=dev)
        if len(wl["shape"]) == 2 and world == 1:
            a, b, c = (x.view(wl["shape"]) for x in (a, b, c))
        bufs.append((a, b, c))
    stream = torch.cuda.current_stream(dev)

    def step(i):
        a, b, c = bufs[i % sets]
        st.vector_add(a, b, out=c)

    with ClockSampler(local) as clk:
        ms, launches = time_steps(step, args.steps, args.warmup, stream, dist_on, graph=use_graph(args, wl))
    ms_max = max_over_ranks(ms, dist_on)
    total_bytes = sum_over_ranks(bytes_per_step, dist_on)
    value = total_bytes * args.steps / (ms_max / 1e3) / 1e9
    achieved = bytes_per_step / (ms / args.steps / 1e3) / 1e9
    key = "vector_add_" + "x".join(str(s) for s in wl["shape"])
    roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 4),
            "peak_note": "of measured copy bandwidth" if peaks["source"] == "measured" else "of fallback",
            "traffic": profile_traffic(key), "kernel": "vadd_vec4_kernel",
            "ms_per_launch": round(ms / args.steps, 5)}
    if roof["traffic"] is not None:
        roof["traffic_note"] = profile_traffic_note(key)
    out = dict(value=value, ms_per_step=ms_max / args.steps, roofline=roof, gpu_launches=int(launches),
               clocks=clk.summary(ms / args.steps), sets=sets, elements=n)
    if len(wl["shape"]) == 1 and world == 1 and not args.no_sweep:
        del bufs
        out["sweep_1d"] = vector_add_sweep(dev, peaks)
        bufs = [(torch.rand(n, device=dev), torch.rand(n, device=dev), torch.empty(n, device=dev))]
    if not args.no_e2e:
        a, b, c = bufs[0]
        ha, hb = a.cpu().pin_memory(), b.cpu().pin_memory()
        hc = torch.empty_like(ha).pin_memory()
        steps = max(1, min(args.steps, 20))
        st.vector_add(ha, hb, out=hc)
        if dist_on:
            import torch.distributed as dist
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            st.vector_add(ha, hb, out=hc)
        dt = max_over_ranks(time.perf_counter() - t0, dist_on)
        e2e_value = total_bytes * steps / dt / 1e9
        link = host_link_probe(dev, 8 * n, 4 * n, dist_on)
        bound_ms = max_over_ranks(link["ms_per_step"], dist_on)
        link["value"] = round(total_bytes / (bound_ms / 1e3) / 1e9, 2)
        link["frac"] = round(e2e_value / link["value"], 4)
        out["e2e"] = {"value": round(e2e_value, 2), "unit": "GB/s",
                      "h2d_bytes_per_step": int(sum_over_ranks(8 * n, dist_on)),
                      "d2h_bytes_per_step": int(sum_over_ranks(4 * n, dist_on)), "steps": steps,
                      "how": "sptiles_b200.vector_add on pinned host tensors (st_vector_add_host), host wall clock",
                      "link_bound": link}
    return out


def extra_entry(name, wl, sub, sub_args, world, unit):
    """One configuration's measurement as a key of the bench line."""
    e = {"workload": name, "value": round(sub["value"], 3), "unit": unit, "steps": sub_args.steps,
         "warmup": sub_args.warmup, "ms_per_step": round(sub["ms_per_step"], 5), "roofline": sub["roofline"],
         "e2e": sub.get("e2e"), "gpu_launches": sub["gpu_launches"], "clocks": sub["clocks"],
         "config": config_of(name, wl, world, sub_args.timing)}
    for k in ("sweep_1d", "step_ms", "allgather"):
        if sub.get(k):
            e[k] = sub[k]
    if wl["kind"] == "matmul":
        e["config"]["tile"] = f"{sub['plan']['block_m']}x{sub['plan']['block_n']}x{sub['plan']['block_k']}"
    return e


def run_extras(args, rank, world, local, dist_on, peaks):
    """The other configurations, each with its own roofline and clock record.

    One GPU: vector_add 1D 2^20 (with the 2^20 .. 2^28 sweep), fp32 1024^3
    (3xTF32) and bf16 32768x4096x4096 + bias.  N GPUs: the bf16 + bias
    configuration M-row sharded with C replicated on every rank, by the GEMM
    epilogue's stores into every rank's copy (fused) and, timed beside it, by
    the GEMM followed by an NCCL all-gather.  Every rank runs the same steps."""
    out = {}
    if world == 1:
        plan = [("vector_add_1d", dict(steps=max(args.steps, 2000), warmup=max(args.warmup, 10), timing="graph")),
                ("matmul_fp32", dict(steps=max(args.steps, 500), warmup=max(args.warmup, 10), timing="graph")),
                ("matmul_bf16", dict(steps=args.steps, warmup=args.warmup, timing="eager"))]
    else:
        plan = [("matmul_bf16", dict(steps=args.steps, warmup=args.warmup, timing="eager", replicate="fused",
                                     no_e2e=True))]
    for name, over in plan:
        wl = WORKLOADS[name]
        sub_args = argparse.Namespace(**{**vars(args), "sustain_steps": 0, **over})
        if wl["kind"] == "matmul":
            sub = run_matmul(wl, sub_args, rank, world, local, dist_on, peaks)
            unit = "TFLOP/s"
        else:
            sub = run_vector_add(wl, sub_args, rank, world, local, dist_on, peaks)
            unit = "GB/s"
        key = name + ("_replicated" if over.get("replicate") else "")
        out[key] = extra_entry(name, wl, sub, sub_args, world, unit)
        if over.get("replicate"):
            out[key]["config"]["replicate_output"] = over["replicate"]
        import torch
        torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------ CPU side
class CpuMatmul:
    """The oracle (CPU restatement of the shader arithmetic) on row samples of a workload."""

    def __init__(self, wl, threads):
        import numpy as np
        import oracle
        self.wl, self.threads, self.oracle = wl, threads, oracle
        rng = np.random.default_rng(wl["seed"])
        k, n = wl["k"], wl["n"]
        self.bf = wl["dtype"] == "bf16"

        def gen(shape):
            x = (rng.standard_normal(shape, dtype=np.float32) * np.float32(wl["std"]))
            if wl["dtype"] == "f16":
                return x.astype(np.float16)
            if self.bf:
                return oracle.f32_to_bf16_bits(x).reshape(shape)
            return x

        self.gen = gen
        self.b = gen((k, n))
        self.bias = None
        if wl["bias"]:
            u = rng.uniform(-1, 1, n).astype(np.float32)
            self.bias = oracle.f32_to_bf16_bits(u) if self.bf else u
        self.a = gen((min(wl["m"], 256), k))
        self.out = {"f32": oracle.F32, "f16": oracle.F16, "bf16": oracle.BF16}[wl["out"]]

    def rows_for(self, budget_s):
        probe = max(self.threads, 8)
        t = self.run(probe)
        return int(max(1, min(self.wl["m"], budget_s / max(t / probe, 1e-9))))

    def run(self, rows):
        import numpy as np
        while self.a.shape[0] < rows:
            self.a = np.concatenate([self.a, self.gen((min(rows, self.wl["m"]) - self.a.shape[0], self.wl["k"]))])
        t, _ = self.oracle.time_matmul_rows(self.a[:rows], self.b, self.bias, bf16=self.bf, out_dtype=self.out,
                                            rows=rows, threads=self.threads)
        return t


class CpuVectorAdd:
    def __init__(self, wl):
        import numpy as np
        import oracle
        self.oracle = oracle
        n = math.prod(wl["shape"])
        rng = np.random.default_rng(wl["seed"])
        self.a = rng.uniform(-1, 1, n).astype(np.float32)
        self.b = rng.uniform(-1, 1, n).astype(np.float32)
        self.c = np.empty_like(self.a)
        self.n = n

    def reps_for(self, budget_s):
        return max(1, int(budget_s / max(self.oracle.time_vector_add(self.a, self.b, self.c, 1), 1e-6)))

    def run(self, reps):
        return self.oracle.time_vector_add(self.a, self.b, self.c, reps) * reps


def cpu_baseline(wl, budget_s=10.0):
    threads = os.cpu_count() or 1
    if wl["kind"] == "matmul":
        cm = CpuMatmul(wl, threads)
        rows = cm.rows_for(budget_s)
        t = cm.run(rows)
        v = flops_of(wl, rows) / t / 1e12
        return {"value": round(v, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                "sample": f"first {rows} of {wl['m']} rows of C ({rows}x{wl['n']}x{wl['k']}), {t:.1f} s, "
                          "oracle restatement of the shader arithmetic, -O3 -ffp-contract=off, "
                          f"{threads} threads; throughput extrapolates linearly in rows"}
    cv = CpuVectorAdd(wl)
    reps = cv.reps_for(budget_s)
    t = cv.run(reps)
    return {"value": round(12 * cv.n * reps / t / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{reps} full passes over {cv.n} elements, {t:.1f} s, one thread"}


def run_reference(args, rank, world):
    """The reference arm: its arithmetic on the host cores, rank 0 only."""
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    threads = os.cpu_count() or 1
    per_step_budget = max(0.3, min(4.0, 150.0 / max(1, args.steps + args.warmup)))
    vals, secs = [], []
    if wl["kind"] == "matmul":
        cm = CpuMatmul(wl, threads)
        rows = cm.rows_for(per_step_budget)
        for i in range(args.warmup + args.steps):
            t = cm.run(rows)
            if i >= args.warmup:
                vals.append(flops_of(wl, rows) / t / 1e12)
                secs.append(t)
        detail = (f"each step: first {rows} of {wl['m']} rows of C ({rows}x{wl['n']}x{wl['k']}) on {threads} "
                  "threads; CPU restatement of the shader arithmetic (-O3 -ffp-contract=off)")
        unit, cores = "TFLOP/s", threads
    else:
        cv = CpuVectorAdd(wl)
        reps = cv.reps_for(per_step_budget)
        for i in range(args.warmup + args.steps):
            t = cv.run(reps)
            if i >= args.warmup:
                vals.append(12 * cv.n * reps / t / 1e9)
                secs.append(t)
        detail = f"each step: {reps} passes over {cv.n} elements, one thread"
        unit, cores = "GB/s", 1
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(statistics.median(secs) * 1e3, 3),  # one bounded sample (see cpu_baseline)
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": wl.get("dtype", "f32"), "data": "synthetic",
        "config": {**_config_of(args.workload, wl, args.gpus),
                   "timed_region": "host wall clock per step, rank 0's host cores"},
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port", "sample": detail},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's SPIR-V runs through Vulkan, which is unavailable on this box, and its "
                "translator cannot be built here; this arm runs the CPU restatement of its shader arithmetic",
    }
    print(json.dumps(line), flush=True)
    return 0


def config_of(name, wl, n_gpus, timing="auto"):
    graph = (wl["kind"] == "vector_add") if timing == "auto" else timing == "graph"
    how = "one CUDA-graph replay of the K steps" if graph else "K host launches"
    cfg = _config_of(name, wl, n_gpus)
    cfg["timed_region"] = how
    return cfg


def _matmul_l2_note(wl, n_gpus):
    sets = matmul_buffer_sets(wl, -(-wl["m"] // n_gpus))
    if sets == 1:
        return "inputs exceed L2 (A + B + C per rank > 126 MB)"
    return f"steps rotate through {sets} buffer sets of A, B, C totalling > 2x L2"


def _config_of(name, wl, n_gpus):
    if wl["kind"] == "matmul":
        return {"workload": name, "M": wl["m"], "N": wl["n"], "K": wl["k"], "in_dtype": wl["dtype"],
                "out_dtype": wl["out"], "bias": wl["bias"], "parallelism": f"M-row shards x{n_gpus}",
                "l2": _matmul_l2_note(wl, n_gpus)}
    total = math.prod(wl["shape"])
    return {"workload": name, "shape": list(wl["shape"]), "dtype": "f32", "parallelism": f"element shards x{n_gpus}",
            "l2": "steps rotate through buffer sets totalling > 2x L2"}


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    import torch
    torch.cuda.set_device(local)
    dist_on = world > 1
    if dist_on:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    peaks = measured_peaks()
    wl = dict(WORKLOADS[args.workload])
    if args.m is not None and wl["kind"] == "matmul":
        wl["m"] = args.m
    try:
        if wl["kind"] == "matmul":
            res = run_matmul(wl, args, rank, world, local, dist_on, peaks)
        else:
            res = run_vector_add(wl, args, rank, world, local, dist_on, peaks)
        secondary, extras = None, None
        if args.workload == "matmul_f16" and not args.no_secondary:
            vw = WORKLOADS["vector_add_2d"]
            # a ~35 us step needs more steps for a timed region the clock sampler can see
            sub_args = argparse.Namespace(**{**vars(args), "steps": max(args.steps, 1000),
                                             "warmup": max(args.warmup, 10)})
            sub = run_vector_add(vw, sub_args, rank, world, local, dist_on, peaks)
            secondary = extra_entry("vector_add_2d", vw, sub, sub_args, world, "GB/s")
            extras = run_extras(args, rank, world, local, dist_on, peaks)
        cpu = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(wl)
        if rank == 0:
            line = {
                "metric": METRIC, "value": round(res["value"], 3),
                "unit": "TFLOP/s" if wl["kind"] == "matmul" else "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(res["ms_per_step"], 5), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": wl.get("dtype", "f32"),
                "data": "synthetic (seeded; shapes and distributions of the configuration)",
                "config": config_of(args.workload, wl, world, args.timing), "roofline": res["roofline"],
                "cpu_baseline": cpu, "e2e": res.get("e2e"), "gpu_launches": res["gpu_launches"],
                "clocks": res["clocks"],
            }
            if wl["kind"] == "matmul":
                line["config"]["tile"] = f"{res['plan']['block_m']}x{res['plan']['block_n']}x{res['plan']['block_k']}"
                line["config"]["ctas"] = res["plan"]["ctas"]
                if args.replicate and world > 1:
                    line["config"]["replicate_output"] = args.replicate
                    line["allgather"] = res.get("allgather")
            if secondary:
                line["vecadd"] = secondary
            if extras:
                line["configs"] = extras
            if res.get("step_ms"):
                line["step_ms"] = res["step_ms"]
            if res.get("sustained"):
                line["sustained"] = res["sustained"]
            if res.get("sweep_1d"):
                line["sweep_1d"] = res["sweep_1d"]
            print(json.dumps(line), flush=True)
    finally:
        if dist_on:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
