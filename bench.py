#!/usr/bin/env python3
"""Benchmark: generate fwd + d/dxi + d/dcov_vals points/s on B200 (BASELINE.json `metric`).

Workload (the configuration the metric is quoted on): N = 10^6 points,
D = 2, iid standard normal (numpy PCG64 seed 1 -- Julia's MersenneTwister streams are not
reproducible here), graph by the build_graph restatement with n0 = 1000, k = 8; RBF table
(variance 1, scale 0.3, 1000 bins over [1e-4, 10], jitter 1e-5) in float32; xi ~ N(0,1)
(seed 2), upstream cotangent vbar ~ N(0,1) (seed 3).  The calls run in the library's
asynchronous mode (set_synchronous(False): each call queues its work; every step ends with
prob.check(), which waits and raises the step's status).  One step = prob.update_vals(table) +
prob.prefactor() (queues the new table's factorisations; in the end-to-end leg they overlap the
upload of xi) + generate(prob, xi) + generate_grad_xi(prob, vbar) + generate_grad_vals(prob, xi, vbar), each
through the public API.  Re-setting the table makes every step factorise the dense block once,
as a step of an optimisation over the covariance does (the handle reuses the factor across the
three calls of a step, and would reuse it across steps if the table did not change).
value = N / step time (points per second through all three operations).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Under torchrun (N > 1) every rank runs the same single-GPU step on its own GPU (independent
fields on a replicated graph); value = N_points * ranks / max-over-ranks time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "graphgp.jl_b200"))

METRIC = "generate fwd+dxi+dcov_vals points/s"
UNIT = "points/s"
CONFIG = dict(N=1_000_000, D=2, n0=1000, k=8, seed_pts=1, seed_xi=2, seed_vb=3,
              kernel=dict(variance=1.0, scale=0.3, r_min=1e-4, r_max=10.0, n_bins=1000,
                          jitter=1e-5))
CFG_NAME = "config2: N=1e6 D=2 normal(seed 1) n0=1000 k=8 RBF(1,0.3,[1e-4,10],1000 bins,jitter 1e-5) f32"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu-case", action="store_true",
                    help="profiling case: one untimed step of the workload, no JSON line")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def make_inputs():
    import graphgp_b200 as gp
    c = CONFIG
    key = f"bench-config2-N{c['N']}-D{c['D']}-seed{c['seed_pts']}"
    g = gp.cached_graph(
        lambda: np.random.default_rng(c["seed_pts"]).standard_normal((c["N"], c["D"])),
        key, c["n0"], c["k"])
    kk = c["kernel"]
    bins, vals = gp.rbf_kernel(kk["variance"], kk["scale"], kk["r_min"], kk["r_max"],
                               kk["n_bins"], jitter=kk["jitter"])
    xi = np.random.default_rng(c["seed_xi"]).standard_normal(c["N"]).astype(np.float32)
    vb = np.random.default_rng(c["seed_vb"]).standard_normal(c["N"]).astype(np.float32)
    return g, bins.astype(np.float32), vals.astype(np.float32), xi, vb


# ---------------------------------------------------------------------------------------------
# CPU baseline: the oracle (C restatement of the reference's CPU path) on the host cores.
# ---------------------------------------------------------------------------------------------
def oracle_problem(g, bins, vals):
    from oracle import oracle as O
    return O.make_problem(g["coords"], g["neighbors"], g["offsets"], g["n0"],
                          np.float32(g["scale"]), bins, vals, g["indices"], np.float32)


def oracle_step(p, xi, vb):
    from oracle import oracle as O
    O.generate(p, xi)
    O.generate_grad_xi(p, vb)
    O.generate_grad_vals(p, xi, vb)


def cpu_info():
    model = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return os.cpu_count() or 1, model


def cpu_baseline(g, bins, vals, xi, vb, steps=1):
    cores, model = cpu_info()
    p = oracle_problem(g, bins, vals)
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        oracle_step(p, xi, vb)
        ts.append(time.perf_counter() - t0)
    t = statistics.median(ts)
    return dict(value=CONFIG["N"] / t, unit=UNIT, cores=cores, kind="port",
                sample=(f"full config-2 step (generate + grad_xi + grad_vals on all 1e6 points), "
                        f"{steps} run(s), median {t:.2f} s; C restatement of the reference's CPU "
                        f"path (OpenMP static chunks, {cores} threads for the per-point passes; "
                        f"the reverse sweeps are serial as in src/grad.jl and "
                        f"src/grad_generate_vals.jl); CPU: {model}"))


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    g, bins, vals, xi, vb = make_inputs()
    p = oracle_problem(g, bins, vals)
    for _ in range(args.warmup):
        oracle_step(p, xi, vb)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle_step(p, xi, vb)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    cores, model = cpu_info()
    val = CONFIG["N"] / dt
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": CFG_NAME, "points": CONFIG["N"]},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"full config-2 step per timed step; CPU: {model}"},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------
# GPU arm.
# ---------------------------------------------------------------------------------------------
class NvmlClockSampler:
    """SM clock and clock-event (throttle) reasons read through NVML every 5 ms on a thread
    during the timed region (a step takes a few ms, so nvidia-smi's 200 ms period would see
    none); the NVML device is matched to the CUDA device by PCI bus id.  Read-only."""

    def __init__(self, cuda_index: int):
        import pynvml
        self.nv = pynvml
        pynvml.nvmlInit()
        import torch
        pr = torch.cuda.get_device_properties(cuda_index)
        try:
            bus = "%08X:%02X:%02X.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            self.h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
        self.samples = []
        self.stop = None
        self.thread = None

    def _read(self):
        nv = self.nv
        sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
        rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        self.samples.append((sm, mx, rs))

    def __enter__(self):
        import threading
        self.stop = threading.Event()
        self._read()

        def loop():
            while not self.stop.wait(0.005):
                self._read()
        self.thread = threading.Thread(target=loop, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        self.stop.set()
        self.thread.join(timeout=5)
        self._read()

    def summary(self):
        nv = self.nv
        bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        reasons = sorted({n for _, _, r in self.samples for n, b in bits.items() if r & b})
        sm = [s for s, _, _ in self.samples]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(m for _, m, _ in self.samples) if self.samples else None,
                "reasons": reasons, "samples": len(sm), "source": "nvml"}


def clock_sampler(cuda_index: int):
    try:
        return NvmlClockSampler(cuda_index)
    except Exception:
        return ClockSampler(cuda_index)


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# DRAM bytes (read + write) per launch of the refine kernels at config 2, from one ncu capture
# each (`ncu --set full ... python bench.py --ncu-case`; summaries in profiles/).  Measured, not
# computed here: the bench itself never runs under a profiler.
NCU_TRAFFIC = {
    "grad_vals": (83.91e6 + 5.47e6, "profiles/k_grad_vals_config2.md"),
    "factor": (40.06e6 + 2.19e6, "profiles/k_factor_config2.md"),
    "sweep_fwdrev_all": (78.64e6 + 4.30e6, "profiles/k_sweep_fwdrev_all_config2.md"),
}


def algorithmic_bytes(kind: str, K: int, D: int, T: int = 4, I: int = 4) -> float:
    """Compulsory bytes per refined point of one kernel launch (no cache-reuse credit)."""
    coords = 4 * D * (K + 1)
    if kind == "factor":      # nbrs + joint coords in, mean_vec + std out
        return I * K + coords + T * K + T
    if kind == "grad_vals":   # nbrs + coords + vb[p] + xi[p] + v[nbr] in (histogram flush excluded)
        return I * K + coords + 2 * T + T * K
    if kind == "sweep_fwd":   # nbrs + mean_vec + std + xi + values[nbr] in, values[p] out
        return I * K + T * K + T + T + T * K + T
    if kind == "sweep_rev":   # nbrs + mean_vec + std + vb[p] in, xg[p] out, K atomics (RMW)
        return I * K + T * K + 2 * T + T + 2 * T * K
    if kind == "fused_fwd":   # the reference's fused forward: B_f = I*k + 4D(k+1) + T(k+2)
        return I * K + coords + T * (K + 2)
    if kind == "sweep_fwd_all":     # persistent forward sweep over all batches
        return algorithmic_bytes("sweep_fwd", K, D, T, I)
    if kind == "sweep_rev_all":     # persistent reverse sweep
        return algorithmic_bytes("sweep_rev", K, D, T, I)
    if kind == "sweep_fwdrev_all":  # both sweeps of generate_grad_vals in one kernel
        return algorithmic_bytes("sweep_fwd", K, D, T, I) + algorithmic_bytes("sweep_rev", K, D, T, I)
    return float("nan")


def run_b200(args):
    import torch
    import torch.distributed as dist

    import graphgp_b200 as gp
    from graphgp_b200 import _lib

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=600))

    g, bins, vals, xi_h, vb_h = make_inputs()
    N = CONFIG["N"]
    prob = gp.GraphGPProblem(g["coords"], g["neighbors"], g["offsets"], g["n0"],
                             np.float32(g["scale"]), bins, vals, g["indices"],
                             dtype=np.float32, device=dev)
    prob.handle  # upload + graph validation, untimed
    gp.set_synchronous(False)  # calls queue their work; each step's prob.check() waits
    xi = torch.from_numpy(xi_h).to(dev)
    vb = torch.from_numpy(vb_h).to(dev)
    vals_d = torch.from_numpy(vals).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2
    stream = torch.cuda.current_stream(dev)
    L = _lib.lib()

    def step():
        prob.update_vals(vals_d).prefactor()
        gp.generate(prob, xi)
        gp.generate_grad_xi(prob, vb)
        gp.generate_grad_vals(prob, xi, vb)
        prob.check()  # the step's status (asynchronous calls): a wait, inside the timed region

    def timed(fn, k):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(k)]
        for a, b in ev:
            flush.random_(0, 255)  # L2 flush between timed iterations (outside the events)
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize(dev)
        return [a.elapsed_time(b) for a, b in ev]

    def barrier():
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()

    if args.ncu_case:  # the same step once, for ncu captures (no timing, no output line)
        step()
        torch.cuda.synchronize(dev)
        prob.release()
        return 0

    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    launches0 = L.gpb2_launch_count()
    with clock_sampler(local) as cs:
        ms = timed(step, args.steps)
    barrier()
    launches = L.gpb2_launch_count() - launches0
    clocks = cs.summary()
    t_local = sum(ms)
    t_all = t_local
    if world > 1:
        tt = torch.tensor([t_local], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_all = float(tt.item())
    ms_per_step = t_all / args.steps
    value = N * world / (ms_per_step / 1e3)

    # Per-kernel durations: the same steps again with a CUDA event pair around every launch.
    L.gpb2_profile_reset()
    L.gpb2_profile_enable(1)
    timed(step, args.steps)
    L.gpb2_profile_enable(0)
    prof = _lib.profile_report()
    L.gpb2_profile_reset()
    M = N - g["n0"]
    K, D = CONFIG["k"], CONFIG["D"]
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    nonempty = int(np.sum(np.diff(g["offsets"]) > 0))
    per_batch = {"sweep_fwd", "sweep_rev", "fused_fwd"}

    def points_done(kind, cnt):  # a flat kernel covers M points per launch, a batch kernel M/sweep
        return M * (cnt / nonempty if kind in per_batch else cnt)

    def gbs(kind, cnt, ms):
        return algorithmic_bytes(kind, K, D) * points_done(kind, cnt) / (ms / 1e3) / 1e9

    refine_kinds = {k: v for k, v in prof.items() if not np.isnan(algorithmic_bytes(k, K, D))}
    kind, (cnt, tot_ms) = max(refine_kinds.items(), key=lambda kv: kv[1][1])
    achieved = gbs(kind, cnt, tot_ms)
    all_ms = sum(v[1] for v in prof.values())
    roofline = {"bound": "hbm", "kernel": kind, "achieved": achieved, "peak": peak,
                "unit": "GB/s", "frac": achieved / peak,
                "traffic": NCU_TRAFFIC[kind][0] if kind in NCU_TRAFFIC else None,
                "traffic_source": NCU_TRAFFIC[kind][1] if kind in NCU_TRAFFIC else None,
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if peaks
                else "fallback 6650 GB/s (of fallback)",
                "bytes_per_point": algorithmic_bytes(kind, K, D),
                "points_per_launch": points_done(kind, cnt) / cnt,
                "launches_per_step": cnt / args.steps,
                "ms_per_launch": tot_ms / cnt,
                "kernel_share_of_library_time": tot_ms / max(all_ms, 1e-9),
                "library_kernel_ms_per_step": all_ms / args.steps,
                "kernels": {k: {"launches": v[0], "ms": round(v[1], 4),
                                **({"GBps": round(gbs(k, v[0], v[1]), 1)} if k in refine_kinds
                                   else {})}
                            for k, v in prof.items()}}

    # End to end through the public API with host buffers: pinned xi/vbar in, results out.
    e2e = None
    if not args.no_e2e:
        xi_p = torch.from_numpy(xi_h).pin_memory()
        vb_p = torch.from_numpy(vb_h).pin_memory()
        out_f = torch.empty(N, dtype=torch.float32).pin_memory()
        out_x = torch.empty(N, dtype=torch.float32).pin_memory()
        out_d = torch.empty(prob.nbins(), dtype=torch.float32).pin_memory()
        vals_p = torch.from_numpy(vals).pin_memory()

        # Inputs land and results leave on a copy stream, overlapped with the compute stream:
        # the new table's factorisations run while xi uploads, vbar uploads during generate,
        # each result downloads during the next call.
        copy_s = torch.cuda.Stream(dev)
        x_d = torch.empty(N, dtype=torch.float32, device=dev)
        v_d = torch.empty(N, dtype=torch.float32, device=dev)
        vals_d = torch.empty(prob.nbins(), dtype=torch.float32, device=dev)

        def e2e_step():
            comp = torch.cuda.current_stream(dev)
            copy_s.wait_stream(comp)  # the previous step is done with the input buffers
            with torch.cuda.stream(copy_s):
                vals_d.copy_(vals_p, non_blocking=True)
                ev_t = copy_s.record_event()
            comp.wait_event(ev_t)
            prob.update_vals(vals_d).prefactor()
            # The large uploads go after the table's and the ladder's small ones: copies in the
            # same direction share the copy engine in issue order.
            with torch.cuda.stream(copy_s):
                x_d.copy_(xi_p, non_blocking=True)
                ev_x = copy_s.record_event()
                v_d.copy_(vb_p, non_blocking=True)
                ev_v = copy_s.record_event()
            comp.wait_event(ev_x)
            outs = []
            for name, fn in (("f", lambda: gp.generate(prob, x_d)),
                             ("x", lambda: gp.generate_grad_xi(prob, v_d)),
                             ("d", lambda: gp.generate_grad_vals(prob, x_d, v_d))):
                if name == "x":
                    comp.wait_event(ev_v)
                r = fn()
                ev = comp.record_event()
                with torch.cuda.stream(copy_s):
                    copy_s.wait_event(ev)
                    {"f": out_f, "x": out_x, "d": out_d}[name].copy_(r, non_blocking=True)
                    r.record_stream(copy_s)
                outs.append(r)
            comp.wait_stream(copy_s)  # the step ends when its last result has landed
            prob.check()

        for _ in range(2):
            e2e_step()
        barrier()
        ems = timed(e2e_step, args.steps)
        barrier()
        te = sum(ems)
        if world > 1:
            tt = torch.tensor([te], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            te = float(tt.item())
        e2e = {"value": N * world / (te / args.steps / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": 2 * N * 4 + 4 * prob.nbins(),
               "d2h_bytes_per_step": 2 * N * 4 + 4 * prob.nbins()}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(g, bins, vals, xi_h, vb_h, steps=1)

    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": CFG_NAME, "points": N, "refined": M,
                       "depth_batches": len(g["offsets"]) - 1,
                       "parallelism": "replicas" if world > 1 else "single",
                       "l2": "flushed between timed steps (256 MB write)"},
            "clocks": clocks, "gpu_launches": int(launches), "roofline": roofline,
            "e2e": e2e, "cpu_baseline": cpu,
            "step_ms_each": [round(x, 4) for x in ms],
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    prob.release()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
