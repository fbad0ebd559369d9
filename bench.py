#!/usr/bin/env python
"""Benchmark: CSR SpMV GFLOP/s (2*nnz/t) on B200, config 5 of the baseline.

Workload (the largest config; it fits one GPU):
64M x 64M CSR, 32 nnz/row (2^31 non-zeros), int64 row_ptr, int32 col, fp64,
70% of columns within +-4096 of the diagonal, 30% uniform; seeded synthetic
data (counter-based generator, seed 12345). One step = one iterated multiply
y <- A*y/||y|| over equal-nnz row shards: by default one fused kernel per rank
(rows stored straight into every rank's next x over NVLink, ||y||^2 reduced
in the kernel, alpha = 1/||x|| read on the device, the cross-rank step barrier in the kernel);
`--path nccl` runs the local SpMV + NCCL all-reduce/all-gather instead.
`scaling` is "strong": the matrix is fixed, N GPUs share it.

Timing: W warm-up steps, then K steps between barrier + synchronize, CUDA
events on the compute stream, max over ranks. Inputs (27 GB) are far larger
than L2 (126 MB), so no flush is needed between steps.

At N = 1 the line also carries `per_config`: configs 1-4 (and config 3 with
fp32 values) on one GPU, L2 warm and, for configs 1 and 3, cold; cuSPARSE on
the same arrays; and the reference's spmv_serial on this host.

`--impl reference` times the reference's own CPU SpMV (spmv_serial of
test/test_cdspmv.cpp:4-20, compiled from the reference sources into
oracle/_ref/libref.so) on a bounded row sample of the same workload, with
every host thread (row slices in parallel); rank 0 only. Its inputs come from
the oracle's own generator (oracle/gen_oracle.c), not from the library under
test. At N = 1 it adds `per_config`: the reference's own GPU path
(preFreeSpMV compiled for sm_100a) on configs 1-4 with its own cdTime and
cdPre.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SpMV GFLOP/s (2*nnz/t) and achieved HBM GB/s vs roofline"
WORKLOAD = "config5: 64Mx64M CSR, 32 nnz/row (2^31 nnz), int64 row_ptr, fp64, 70% band +-4096 / 30% uniform cols; 10-step power iteration y<-A*y/||y||"
SEED = 12345


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """SM clocks and throttle reasons of one GPU, polled through NVML every
    5 ms on a background thread while the timed region runs (read-only
    queries). Falls back to an `nvidia-smi -lms` subprocess without NVML."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, gpu_index: int, period_s: float = 0.005):
        self.gpu, self.period = gpu_index, period_s
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None

    def _poll(self, nv, hdl):
        while not self._stop.is_set():
            try:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(hdl, nv.NVML_CLOCK_SM)))
                get = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    nv.nvmlDeviceGetCurrentClocksThrottleReasons
                bits = get(hdl)
                for name, b in self.REASONS.items():
                    if bits & b:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        try:
            import pynvml as nv
            import torch
            nv.nvmlInit()
            # NVML numbers GPUs in its own order: find this CUDA device by PCI id
            p = torch.cuda.get_device_properties(self.gpu)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            hdl = nv.nvmlDeviceGetHandleByPciBusId(bus.encode())
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(hdl, nv.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._poll, args=(nv, hdl), daemon=True)
            self._thread.start()
        except Exception:  # noqa: BLE001
            self._thread = None
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": sorted(self.reasons), "source": "NVML, 5 ms polling"}


def traffic_per_row():
    """DRAM bytes per row of the config-5 kernel from the committed ncu capture
    (profiles/config5_spmv_traffic.json), or None."""
    p = os.path.join(ROOT, "profiles", "config5_spmv_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f).get("dram_bytes_per_row")


PER_CONFIGS = [(1, "f64"), (2, "f64"), (3, "f64"), (3, "f32"), (4, "f64")]


def compulsory_bytes(m, n, nnz, vbytes, ibytes):
    """nnz*(V+4) + (m+1)*R + n*V + m*V: the reference's data_origin1
    (test/test_cdspmv.cpp:305) with beta = 0."""
    return nnz * (vbytes + 4) + (m + 1) * ibytes + n * vbytes + m * vbytes


def reference_gpu_per_config(oracle, threads):
    """The reference's own GPU path (preFreeSpMV compiled unmodified for
    sm_100a, oracle/_ref/libref_gpu.so) on configs 1-4, fp64 (its only value
    type): its own cdTime (ms per multiply, 4000 launches after 200 warm-ups,
    L2 warm, src/spmv_kernel/preFreeSpMV.cu:604-650) and cdPre (its start-row
    pre-pass), and whether its y meets the tolerance against spmv_serial.
    Inputs from the oracle's generator."""
    if not oracle.ref_gpu_available():
        return {"unavailable": "oracle/_ref/libref_gpu.so not built"}
    out = {}
    for cfg in (1, 2, 3, 4):
        rp, col, val, x = oracle.gen_config(cfg, seed=SEED, threads=threads)
        m, n, z = len(rp) - 1, len(x), len(col)
        rp32 = rp.astype(np.int32)
        y, cd, pre = oracle.ref_gpu_prefree(val, rp32, col, x, m, n)
        ref = oracle.ref_serial_threaded(rp32, col, val, x, threads)
        a, comp = oracle.abs_comp(rp, col, val, x)
        _, _, nbad = oracle.tolerance_report(y, ref, a, 1e-12, y_comp=comp)
        B = compulsory_bytes(m, n, z, 8, 4)
        out[f"c{cfg}_f64"] = {"m": m, "nnz": z, "cdTime_us": cd * 1e3, "cdPre_us": pre * 1e3,
                              "gflops": 2 * z / (cd * 1e6), "alg_GBps": B / (cd * 1e6),
                              "rows_out_of_tolerance": nbad}
        del rp, rp32, col, val, x, y, ref, a, comp
    out["timing"] = "the reference's own cdTime / cdPre (preFreeSpMV.cu:604-650), L2 warm"
    return out


def run_reference(args, rank):
    """--impl reference: the reference's CPU spmv_serial on all host threads
    (the headline), plus at N = 1 the reference's own GPU path per config."""
    if rank != 0:
        return
    import oracle
    threads = os.cpu_count() or 1
    rows = 1 << 23                      # 2^28 non-zeros per sampled step
    rp, col, val, x = oracle.gen_config(5, seed=SEED, r0=0, r1=rows, threads=threads)
    rp32 = rp.astype(np.int32)
    kind = "reference" if oracle.ref_available() else "port"

    def one():
        if kind == "reference":
            return oracle.ref_serial_threaded(rp32, col, val, x, threads)
        return oracle.serial(rp, col, val, x)

    for _ in range(args.warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    dt = (time.perf_counter() - t0) / args.steps
    z = int(rp[-1])
    del rp, rp32, col, val, x
    v = 2.0 * z / dt / 1e9
    sample = (f"rows [0, 2^23) of config 5 ({z} nnz, x of 2^26) per step; "
              f"spmv_serial on {threads} equal-nnz row slices in parallel threads")
    per = None
    if int(os.environ.get("WORLD_SIZE", "1")) == 1 and not args.no_per_config:
        per = reference_gpu_per_config(oracle, threads)
    print(json.dumps({
        "metric": METRIC, "value": v, "unit": "GFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded generator, oracle/gen_oracle.c)", "impl": "reference",
        "config": {"workload": WORKLOAD, "parallelism": "host threads", "sample_rows": rows},
        "cpu_baseline": {"value": v, "unit": "GFLOP/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": v, "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "per_config": per,
    }), flush=True)


def _median(v):
    return float(statistics.median(v))


def time_graph_us(torch, fn, launches=200, repeats=5):
    """Per-launch µs of `fn` replayed back to back from one CUDA graph of
    `launches` calls (L2 warm, like the reference's launch loop): the median
    of `repeats` replays, CUDA events on the capturing stream."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(launches):
                fn()
        g.replay()
        ts = []
        for _ in range(repeats):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            g.replay()
            e1.record(s)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3 / launches)
    torch.cuda.current_stream().wait_stream(s)
    del g
    return _median(ts)


def time_cold_us(torch, fn, flush, reps=20):
    """Per-launch µs with L2 flushed before every launch: a write of `flush`
    (four times the L2 size) outside the timed events; median of `reps`."""
    st = torch.cuda.current_stream()
    for _ in range(3):
        fn()
    ts = []
    for i in range(reps):
        flush.fill_(i & 0xff)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        fn()
        e1.record(st)
        e1.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3)
    return _median(ts)


def per_config_block(pf, torch, dev, with_cpu: bool):
    """Configs 1-4 (config 3 also with fp32 values) on one GPU, each through
    the auto-selected variant: per-launch µs (L2 warm: median of 5 replays of
    200 launches; configs 1 and 3 also cold-L2), algorithmic GB/s and its
    fraction of the measured copy peak and of 8 TB/s; cuSPARSE CSR SpMV
    (torch sparse CSR, int32 indices) on the same device arrays; and, when
    with_cpu, the reference's spmv_serial (one thread, median of 3) on the
    same matrix on this host."""
    import oracle
    hbm_peak, peak_src = peaks()
    h = pf.Handle()
    flush = torch.empty(4 * 126 * 2**20 // 4, dtype=torch.int32, device=dev)  # 504 MB
    out = {}
    launches0 = pf.launch_count()
    for cfg, vname in PER_CONFIGS:
        vdt = {"f64": torch.float64, "f32": torch.float32}[vname]
        spec = pf.GenSpec(cfg=cfg, seed=SEED).resolved()
        rp, col, val = pf.gen_rows_device(spec, index_dtype=torch.int32, value_dtype=vdt,
                                          device=dev)
        x = pf.gen_x_device(spec, value_dtype=vdt, device=dev)
        y = torch.empty(spec.m, dtype=vdt, device=dev)
        z = col.numel()

        def ours():
            pf.spmv(h, spec.m, spec.n, z, rp, col, val, x, y)

        warm = time_graph_us(torch, ours)
        cold = time_cold_us(torch, ours, flush) if cfg in (1, 3) else None
        assert h.device_error() == 0, "device error word set"
        B = compulsory_bytes(spec.m, spec.n, z, val.element_size(), 4)
        e = {"m": spec.m, "nnz": z, "variant": "%s/%d" % h.choice(spec.m, z, rp, val.element_size()),
             "alg_bytes": B, "us": warm, "gflops": 2 * z / warm / 1e3,
             "alg_GBps": B / warm / 1e3, "frac_of_" + peak_src: B / warm / 1e3 / hbm_peak,
             "frac_of_8TBps": B / warm / 1e3 / 8000.0}
        if cold is not None:
            e["cold_l2_us"] = cold
            e["cold_l2_frac_of_" + peak_src] = B / cold / 1e3 / hbm_peak
        try:
            A = torch.sparse_csr_tensor(rp, col, val, size=(spec.m, spec.n))
            xv = x.unsqueeze(1)
            yv = torch.empty(spec.m, 1, dtype=vdt, device=dev)
            e["cusparse_us"] = time_graph_us(torch, lambda: torch.matmul(A, xv, out=yv))
            del A, xv, yv
        except RuntimeError as ex:
            e["cusparse_us"] = None
            e["cusparse_error"] = str(ex).splitlines()[0][:200]
        if with_cpu:
            hrp, hcol = rp.cpu().numpy(), col.cpu().numpy()
            hval = val.double().cpu().numpy()   # fp32 values widened: spmv_serial is fp64
            hx = x.double().cpu().numpy()
            kind = "reference" if oracle.ref_available() else "port"
            ts = []
            for _ in range(3):
                t0 = time.perf_counter()
                if kind == "reference":
                    oracle.ref_serial(hrp, hcol, hval, hx)
                else:
                    oracle.serial(hrp.astype(np.int64), hcol, hval, hx)
                ts.append(time.perf_counter() - t0)
            e["cpu_spmv_serial_ms"] = _median(ts) * 1e3
            e["cpu_gflops"] = 2 * z / _median(ts) / 1e9
            e["cpu_kind"] = kind
            del hrp, hcol, hval, hx
        out[f"c{cfg}_{vname}"] = e
        del rp, col, val, x, y
        torch.cuda.empty_cache()
    out["launches"] = int(pf.launch_count() - launches0)
    out["timing"] = ("ours and cuSPARSE: median of 5 replays of a 200-launch CUDA graph, L2 warm "
                     "(as the reference's 4000-launch loop); cold_l2: L2 flushed by a 504 MB "
                     "write before each launch, outside the events, median of 20")
    if with_cpu:
        out["cpu"] = {"cores": 1, "threads_available": os.cpu_count(),
                      "what": "the reference's spmv_serial (test/test_cdspmv.cpp:4-20), one "
                              "thread, median of 3; fp32 values widened to fp64"}
    h.close()
    del flush
    torch.cuda.empty_cache()
    return out


def run_kernel_mode(args):
    """--mode kernel: one config, one GPU, back-to-back multiplies of the
    device-resident matrix (L2 warm between launches, as in the reference's
    4000-launch loop, preFreeSpMV.cu:632-642). Prints one JSON line per
    config with the per-launch time, algorithmic GB/s and the fraction of the
    measured copy bandwidth. Used for the per-config table and ncu captures."""
    import torch
    pf = importlib.import_module("prefree-public_b200")
    hbm_peak, peak_src = peaks()
    h = pf.Handle()
    h.set_variant(args.variant)
    for cfg in [int(c) for c in args.config.split(",")]:
        for vname in args.dtype.split(","):
            vdt = {"f64": torch.float64, "f32": torch.float32, "f16": torch.float16,
                   "bf16": torch.bfloat16}[vname]
            gdt = vdt if vname in ("f64", "f32") else torch.float32  # generated, then rounded
            spec = pf.GenSpec(cfg=cfg, seed=SEED, m=args.rows, n=args.cols).resolved()
            idt = torch.int64 if (cfg == 5 or args.int64) else torch.int32
            rp, col, val = pf.gen_rows_device(spec, index_dtype=idt, value_dtype=gdt)
            val = val.to(vdt)
            z = col.numel()
            if args.k > 0:
                # SpMM: k dense columns (x and its rotations), Y m x k
                x0 = pf.gen_x_device(spec, value_dtype=gdt).to(vdt)
                x = torch.stack([torch.roll(x0, j) for j in range(args.k)], dim=1).contiguous()
                y = torch.empty(spec.m, args.k, dtype=vdt, device="cuda")
                del x0

                def one():
                    pf.spmm(h, spec.m, spec.n, z, rp, col, val, x, y)
            else:
                x = pf.gen_x_device(spec, value_dtype=gdt).to(vdt)
                y = torch.empty(spec.m, dtype=vdt, device="cuda")

                def one():
                    pf.spmv(h, spec.m, spec.n, z, rp, col, val, x, y)
            for _ in range(args.warmup):
                one()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            if args.graph:
                # the K launches replayed from one CUDA graph: back-to-back on
                # the GPU like the reference's C++ loop, without the Python
                # call overhead between launches (it exceeds a config-1 multiply)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for _ in range(args.steps):
                        one()
                g.replay()
                torch.cuda.synchronize()
                e0.record()
                g.replay()
                e1.record()
            else:
                e0.record()
                for _ in range(args.steps):
                    one()
                e1.record()
            torch.cuda.synchronize()
            assert h.device_error() == 0
            ms = e0.elapsed_time(e1) / args.steps
            kk = max(args.k, 1)
            vs = val.element_size()
            # compulsory bytes: A once, k columns of x and y
            B = (pf.compulsory_bytes(spec.m, spec.n, z, vs, rp.element_size())
                 + (kk - 1) * (spec.n + spec.m) * vs)
            print(json.dumps({"mode": "kernel", "config": cfg, "dtype": vname, "m": spec.m,
                              "n": spec.n, "nnz": z, "variant": args.variant, "k": args.k,
                              "us": ms * 1e3,
                              "gflops": 2 * z * kk / ms / 1e6, "alg_GBps": B / ms / 1e6,
                              "frac_of_" + peak_src: B / ms / 1e6 / hbm_peak,
                              "frac_of_8TBps": B / ms / 1e6 / 8000.0,
                              "launches": args.steps, "graph": bool(args.graph)}), flush=True)
            if args.graph:
                del g
            del rp, col, val, x, y
            torch.cuda.empty_cache()
    h.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip the per-config block (configs 1-4 on one GPU)")
    ap.add_argument("--path", default="fused", choices=["fused", "nccl"],
                    help="power mode: fused multiply + all-gather kernel, or SpMV + NCCL")
    ap.add_argument("--barrier", default="kernel", choices=["kernel", "host"],
                    help="fused path: step barrier inside the kernel (step counters) "
                         "or a symmetric-memory barrier launched between steps")
    ap.add_argument("--mode", default="power", choices=["power", "kernel"],
                    help="power: the config-5 power iteration (the benchmark line); "
                         "kernel: per-config single-GPU multiply timing")
    ap.add_argument("--config", default="1,2,3,4,5", help="kernel mode: configs")
    ap.add_argument("--dtype", default="f64", help="kernel mode: f64, f32, f16, bf16 (comma list)")
    ap.add_argument("--variant", type=int, default=0, help="kernel mode: 0 auto, or a forced pf_variant (1, 2, 4, 7)")
    ap.add_argument("--rows", type=int, default=0,
                    help="override m (kernel mode; power mode: profiling slice of config 5)")
    ap.add_argument("--cols", type=int, default=0, help="kernel mode: override n")
    ap.add_argument("--int64", action="store_true", help="kernel mode: int64 row_ptr")
    ap.add_argument("--k", type=int, default=0,
                    help="kernel mode: SpMM with k dense columns (0: SpMV)")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="kernel mode: launch from Python instead of replaying a CUDA graph")
    args = ap.parse_args()
    if args.mode == "kernel":
        run_kernel_mode(args)
        return
    assert args.warmup >= 3 or args.impl == "reference" or os.environ.get("PF_BENCH_ALLOW_SHORT"), \
        "at least 3 warm-up steps"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=dev)
    pf = importlib.import_module("prefree-public_b200")
    pfd = importlib.import_module("prefree-public_b200.dist")

    spec = pf.GenSpec(cfg=5, seed=SEED).resolved()
    if args.rows:
        # profiling case only: the first `rows` rows of config 5 (x keeps all
        # 2^26 columns, so the gathers behave as in the full matrix)
        spec = pf.GenSpec(cfg=5, seed=SEED, m=args.rows, n=spec.n).resolved()
    bounds = pfd.gen_bounds(pf, spec, world)
    r0, r1 = int(bounds[rank]), int(bounds[rank + 1])
    m_loc, n = r1 - r0, spec.n
    rp, col, val = pf.gen_rows_device(spec, r0, r1, index_dtype=torch.int64,
                                      value_dtype=torch.float64, device=dev)
    x = pf.gen_x_device(spec, value_dtype=torch.float64, device=dev)
    y = torch.empty(m_loc, dtype=torch.float64, device=dev)
    nnz_loc = col.numel()
    z_tot = torch.tensor([nnz_loc], dtype=torch.int64, device=dev)
    if world > 1:
        dist.all_reduce(z_tot)
    z_tot = int(z_tot.item())
    h = pf.Handle()
    stream = torch.cuda.current_stream(dev)
    ev_pairs = []

    def local_spmv(xf, yl, alpha):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        pf.spmv(h, m_loc, n, nnz_loc, rp, col, val, xf, yl, alpha, 0.0, stream=stream)
        e1.record(stream)
        ev_pairs.append((e0, e1))

    if args.path == "fused":
        # one kernel per step: rows go straight into every rank's next x over
        # NVLink, ||y||^2 is reduced in the kernel, and the kernel waits for
        # every rank's previous step (step counters) before reading x: steps
        # are launched back to back
        fused = pfd.FusedPowerIteration(pf, h, rp, col, val, x, bounds, rank, world,
                                        stream=stream)

        class _Step:
            def step(self):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                fp = fused.flag_ptrs.data_ptr() if (fused.flag_ptrs is not None
                                                    and args.barrier == "kernel") else 0
                pf.spmv_dist(h, m_loc, n, nnz_loc, rp, col, val, fused.xs[fused.k % 2],
                             fused.slots[fused.k % 2], world, rank,
                             fused.out_ptrs[(fused.k + 1) % 2].data_ptr(),
                             fused.slot_ptrs[(fused.k + 1) % 2].data_ptr(), int(bounds[rank]),
                             stream=stream, flag_ptrs_dev=fp, step=fused.k)
                e1.record(stream)
                ev_pairs.append((e0, e1))
                if fused.hdl is not None and not fp:
                    fused.hdl.barrier(channel=0)
                fused.k += 1
                return None
        it = _Step()
    else:
        it = pfd.PowerIteration(local_spmv, x, y, bounds, rank, world)
    for _ in range(args.warmup):
        it.step()
    torch.cuda.synchronize()
    ev_pairs.clear()

    # ---- timed region ------------------------------------------------------------
    if args.path == "fused":
        h.dist_wait_ns(reset=True)
    launches0 = pf.launch_count()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    # the clock sampler starts (NVML initialisation, milliseconds that differ
    # from rank to rank) before the barrier, so that every rank records its
    # start event right after leaving the same barrier
    with ClockSampler(local) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t_start.record(stream)
        for _ in range(args.steps):
            st = it.step()
        t_end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches = pf.launch_count() - launches0
    step_ms = t_start.elapsed_time(t_end) / args.steps
    dist_diag = None
    if args.path == "fused" and world > 1:
        # how long each rank's CTAs waited in the in-kernel step barrier, and
        # each rank's own kernel time: min / max over ranks
        wns, ctas = h.dist_wait_ns(reset=True)
        my_kern = sum(a.elapsed_time(b) for a, b in ev_pairs) / len(ev_pairs)
        d = torch.tensor([wns / max(ctas, 1) / args.steps / 1e3, my_kern], dtype=torch.float64,
                         device=dev)
        dmin, dmax = d.clone(), d.clone()
        dist.all_reduce(dmin, op=dist.ReduceOp.MIN)
        dist.all_reduce(dmax, op=dist.ReduceOp.MAX)
        dist_diag = {"barrier_wait_us_per_cta_step": {"min": float(dmin[0]), "max": float(dmax[0])},
                     "kernel_ms_per_rank": {"min": float(dmin[1]), "max": float(dmax[1])},
                     "ctas_per_rank": ctas}
    if args.path == "fused":
        final_nsq = fused.norm_sq()
    else:
        final_nsq = st.norm_sq
    kern_ms = sum(a.elapsed_time(b) for a, b in ev_pairs) / len(ev_pairs)
    stats = torch.tensor([step_ms, kern_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    step_ms, kern_ms = float(stats[0]), float(stats[1])
    assert h.device_error() == 0, "device error word set"
    final_norm = math.sqrt(final_nsq)

    # roofline of the SpMV kernel (rank with the slowest launch)
    alg_bytes = pf.compulsory_bytes(m_loc, n, nnz_loc, 8, 8)
    hbm_peak, peak_src = peaks()
    achieved = alg_bytes / (kern_ms * 1e-3) / 1e9
    tpr = traffic_per_row()
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "peak_source": peak_src,
                "traffic": (tpr * m_loc) if tpr else None,
                "algorithmic_bytes_per_launch": alg_bytes, "kernel_ms": kern_ms}

    # ---- e2e: the host-buffer C-ABI call, copies inside the timed region ----------
    e2e = None
    if not args.no_e2e:
        ks = args.e2e_steps or max(1, min(args.steps, 5))
        h_rp = torch.empty(rp.shape, dtype=torch.int64, pin_memory=True)
        h_col = torch.empty(col.shape, dtype=torch.int32, pin_memory=True)
        h_val = torch.empty(val.shape, dtype=torch.float64, pin_memory=True)
        h_x = torch.empty(x.shape, dtype=torch.float64, pin_memory=True)
        h_y = torch.empty(y.shape, dtype=torch.float64, pin_memory=True)
        h_rp.copy_(rp)
        h_col.copy_(col)
        h_val.copy_(val)
        h_x.copy_(x)
        he = pf.Handle()
        a_rp, a_col, a_val, a_x, a_y = (t.numpy() for t in (h_rp, h_col, h_val, h_x, h_y))
        pf.spmv_host(he, a_rp, a_col, a_val, a_x, a_y, stream=stream.cuda_stream)  # warm-up
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(ks):
            pf.spmv_host(he, a_rp, a_col, a_val, a_x, a_y, stream=stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        my_ms = e0.elapsed_time(e1) / ks
        my_h2d = h_rp.numel() * 8 + h_col.numel() * 4 + h_val.numel() * 8 + h_x.numel() * 8
        e_ms = torch.tensor([my_ms], dtype=torch.float64, device=dev)
        # per-rank host-to-device rate (the rank's shard and its own full x,
        # which every row of the shard may read): min and max over ranks
        rate = torch.tensor([my_h2d / (my_ms * 1e-3) / 1e9], dtype=torch.float64, device=dev)
        rate_min, rate_max = rate.clone(), rate.clone()
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
            dist.all_reduce(rate_min, op=dist.ReduceOp.MIN)
            dist.all_reduce(rate_max, op=dist.ReduceOp.MAX)
        h2d = torch.tensor([my_h2d, h_y.numel() * 8], dtype=torch.int64, device=dev)
        if world > 1:
            dist.all_reduce(h2d)
        e2e = {"value": 2.0 * z_tot / (float(e_ms) * 1e-3) / 1e9, "unit": "GFLOP/s",
               "h2d_bytes_per_step": int(h2d[0]), "d2h_bytes_per_step": int(h2d[1]),
               "ms_per_step": float(e_ms), "steps": ks,
               "h2d_GBps_per_rank": {"min": float(rate_min), "max": float(rate_max)},
               "call": "pf_spmv_host_f64_i64 per rank on its host shard (one multiply)"}
        he.close()
        del h_rp, h_col, h_val, h_x, h_y

    # ---- CPU baseline (rank 0, N = 1): the reference's spmv_serial, 1 thread -------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        rows = 1 << 21
        hrp = rp[:rows + 1].cpu().numpy()
        zc = int(hrp[-1])
        hcol = col[:zc].cpu().numpy()
        hval = val[:zc].cpu().numpy()
        x0 = pf.gen_x_device(spec, value_dtype=torch.float64, device=dev).cpu().numpy()
        kind = "reference" if oracle.ref_available() else "port"
        t0 = time.perf_counter()
        if kind == "reference":
            oracle.ref_serial(hrp.astype(np.int32), hcol, hval, x0)
        else:
            oracle.serial(hrp, hcol, hval, x0)
        dt = time.perf_counter() - t0
        cpu = {"value": 2.0 * zc / dt / 1e9, "unit": "GFLOP/s", "cores": 1, "kind": kind,
               "sample": f"rows [0, 2^21) of config 5 ({zc} nnz), one multiply, single thread "
                         "(spmv_serial is serial by construction)"}

    per = None
    if world == 1 and not args.no_per_config:
        per = per_config_block(pf, torch, dev, with_cpu=not args.no_cpu)

    if rank == 0:
        out = {
            "metric": METRIC, "value": 2.0 * z_tot / (step_ms * 1e-3) / 1e9, "unit": "GFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded counter-based generator; SuiteSparse files are not available)",
            "config": {"workload": WORKLOAD, "m": spec.m, "n": spec.n, "nnz": z_tot,
                       "index": "int64 row_ptr, int32 col", "parallelism": f"row shards x{world}",
                       "l2": "inputs (27 GB) larger than L2: no flush",
                       "step": ("fused: SpMV storing rows into every rank's next x over NVLink + in-kernel ||y||^2 + in-kernel cross-rank step barrier"
                                if args.path == "fused" else
                                "local SpMV + NCCL all-reduce ||y||^2 + NCCL all-gather y")},
            "gpu_launches": int(launches),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clocks.summary(),
            "check": {"final_norm_sq_of_y": final_nsq, "final_norm": final_norm},
            "per_config": per,
            "dist": dist_diag,
        }
        print(json.dumps(out), flush=True)
    h.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
