"""Benchmark of the enumerate + sparse-coarsen SpMM hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 5|4|3|2|1]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

Default workload (config 5, the largest single-GPU configuration): A is
16384 x 16384 fp32 at 95% sparsity (half the nonzeros in aligned 4x1
vertical runs, half unstructured, N(0, 0.02^2)), coarsened with
(kernel_m, kernel_n) = (4, 1); B is 16384 x 128 fp32 U(-1, 1), replicated.
A step is one C = A*B.  With N GPUs, A is row-partitioned at row-panel
boundaries (balanced by nonzeros), each rank multiplies its row block, and
the C row blocks are gathered with NCCL all-gather (strong scaling: the job's
work is fixed).

Metric: GFLOP/s = 2*nnz*N / time (whole job), time = max over ranks of the
CUDA-event time of the K timed steps; L2 (126 MB) is flushed before every
timed step by writing a 256 MiB buffer, then reading another 256 MiB buffer
(so the flush's dirty lines are written back before the events), outside the
timed events.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HBM_FALLBACK_GBS = 6650.0
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "dram_traffic.json")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", type=int, default=5, choices=[1, 2, 3, 4, 5])
    p.add_argument("--n-cols-b", type=int, default=None)
    p.add_argument("--kernel-m", default="4",
                   help="coarsening rows, or 'auto' to time kernel_m 1..6 per matrix and keep the fastest")
    p.add_argument("--kernel-n", type=int, default=1)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--sweep-small", action="store_true",
                   help="config 2 table: every sparsity x N in {1,2,4}, single warm launch, CUDA-graph "
                        "replay, and cuSPARSE (one JSON line with a 'sweep' list)")
    p.add_argument("--exchange", choices=["peer", "peer-barrier", "nccl"], default="peer",
                   help="N>1 row partition: C blocks stored to peers by the SpMM kernel itself over NVLink "
                        "(symmetric memory) and completion flags (peer) or a barrier (peer-barrier), or "
                        "gathered afterwards with NCCL all-gather (nccl)")
    p.add_argument("--dense-bf16", action="store_true",
                   help="opt-in: dense-tile plans on bf16 tiles (fp32 accumulation, looser error bound) "
                        "instead of 3xTF32; the default and the reference compute in fp32")
    p.add_argument("--values", choices=["f32", "f16", "bf16"], default="f32",
                   help="opt-in: small-B / SpMV plans (N in {1,2,4}) with A's values stored in 16 bits "
                        "(fp32 products and sums, looser error bound); the default and the reference use fp32")
    p.add_argument("--no-graph", action="store_true",
                   help="config 4: launch the batch directly instead of replaying its captured CUDA graph")
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="target CPU work of the bounded cpu_baseline sample")
    return p.parse_args()


# ---------------------------------------------------------------- inputs --

def workload(cfg: int, n_cols_b):
    """Returns (name, [(csr arrays, B)], kernel shapes) for the chosen config."""
    from sparse_computation_b200 import workloads as wl
    if cfg == 5:
        N = n_cols_b or 128
        a, B = wl.config5(n_cols_b=N)
        return f"config5: A 16384x16384 fp32 95% sparse (half 4x1 runs), B 16384x{N}", [(a, B)]
    if cfg == 1:
        a, B = wl.config1()
        return "config1: A 512x512 p=0.10, B 512x32", [(a, B)]
    if cfg == 2:
        N = n_cols_b or 4
        a, B = wl.config2(0.9, N)
        return f"config2: A 512x512 90% magnitude-pruned, B 512x{N}", [(a, B)]
    if cfg == 3:
        N = n_cols_b or 128
        return f"config3: A 2048x512 + 512x2048 90% Beta(2,18) rows, B Kx{N}", \
            [wl.config3((2048, 512), N), wl.config3((512, 2048), N)]
    N = n_cols_b or 128
    return f"config4: 96-matrix transformer-base stack 80%, B Kx{N}", [(a, B) for _, a, B in wl.config4(N)]


from sparse_computation_b200.partition import balanced_panel_cuts, lpt_assign, row_slice  # noqa: E402


def symmetric_buffer(shape, dev, dtype=None):
    """A buffer (float32 by default) allocated in torch symmetric memory
    (peer-mapped on every rank) and its rendezvous handle."""
    import torch
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem
    group = dist.group.WORLD
    try:
        symm_mem.enable_symm_mem_for_group(group.group_name)
    except Exception:
        pass
    t = symm_mem.empty(shape, dtype=dtype or torch.float32, device=dev)
    hdl = symm_mem.rendezvous(t, group.group_name)
    return t, hdl


# ---------------------------------------------------------------- clocks --

class ClockSampler:
    """Samples the SM clock and clock-event (throttle) reasons of the bench's
    GPU through NVML (read-only queries) every 5 ms; only samples taken while
    `timed` is set are summarised, so the record covers the timed region.
    Falls back to `nvidia-smi` polling when NVML is unavailable."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}

    def __init__(self, cuda_index: int):
        self.rows = []  # (sm_mhz, max_mhz, [reasons])
        self.timed = False
        self._stop = threading.Event()
        self._h = None
        self._nv = None
        try:
            import pynvml as nv
            import torch
            nv.nvmlInit()
            props = torch.cuda.get_device_properties(cuda_index)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            self._h = nv.nvmlDeviceGetHandleByPciBusId(bus)
            self._nv = nv
        except Exception:
            self._h = None
        self.idx = cuda_index
        self._t = threading.Thread(target=self._run, daemon=True)

    def _sample(self):
        if self._h is not None:
            nv = self._nv
            sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
            mx = nv.nvmlDeviceGetMaxClockInfo(self._h, nv.NVML_CLOCK_SM)
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            rs = [k for k, attr in self.REASONS.items() if bits & getattr(nv, attr)]
            return float(sm), float(mx), rs
        out = subprocess.run(["nvidia-smi", "-i", str(self.idx), "--query-gpu=clocks.sm,clocks.max.sm,"
                              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                              "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5).stdout
        f = [x.strip() for x in out.strip().split(",")]
        rs = [k for k, v in zip(self.REASONS, f[2:]) if v == "Active"]
        return float(f[0]), float(f[1]), rs

    def sample_now(self):
        """One synchronous sample (call while the GPU is busy with timed work)."""
        try:
            self.rows.append(self._sample())
        except Exception:
            pass

    def _run(self):
        period = 0.005 if self._h is not None else 0.2
        while not self._stop.is_set():
            try:
                if self.timed:
                    self.rows.append(self._sample())
            except Exception:
                pass
            self._stop.wait(period)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            try:
                self.rows.append(self._sample())
            except Exception:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock query unavailable"], "samples": 0}
        sm = [r[0] for r in self.rows]
        reasons = sorted({x for r in self.rows for x in r[2]})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(r[1] for r in self.rows), "reasons": reasons,
                "samples": len(self.rows), "source": "nvml" if self._h is not None else "nvidia-smi",
                "window": "timed region"}


def measured_peak_hbm():
    try:
        with open(PEAKS_FILE) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


def measured_traffic(workload_key):
    try:
        with open(TRAFFIC_FILE) as f:
            return json.load(f).get(workload_key)
    except Exception:
        return None


# ----------------------------------------------------------- CPU leg ----

def cpu_reference_rate(mats, seconds, threads):
    """Times the reference's spmm_csr_float (oracle/_ref, else the restated
    oracle) on a bounded row sample of the workload; returns (GFLOP/s, kind,
    sample description, threads)."""
    from oracle import cpu
    kind = "reference" if cpu.ref_available("libref_spmm.so") else "port"
    fn = cpu.ref_spmm_csr_float if kind == "reference" else None
    a, B = mats[0]
    m, n, ip, ix, dx = a
    ip32 = np.ascontiguousarray(ip, np.int32)
    ix32 = np.ascontiguousarray(ix, np.int32)
    dx32 = np.ascontiguousarray(dx, np.float32)
    N = B.shape[1]
    C = np.zeros((m, N), np.float32)

    def run_rows(r0, r1):
        if kind == "reference":
            fn(ip32, ix32, dx32, B, C, r0, r1)
        else:
            s = row_slice(a, r0, r1)
            cpu.spmm_csr_float(s[2], s[3], s[4], B, C[r0:r1])

    # Each thread walks 512-row blocks (thread t takes blocks t, t+T, ...,
    # wrapping around the matrix) until the deadline; the sample is what got
    # done in `seconds`.
    blk = 512
    nblk = (m + blk - 1) // blk
    done = [0] * threads
    deadline = time.perf_counter() + seconds

    def worker(t):
        b = t
        while time.perf_counter() < deadline:
            r0 = (b % nblk) * blk
            r1 = min(m, r0 + blk)
            run_rows(r0, r1)
            done[t] += int(ip[r1] - ip[r0])
            b += threads

    from concurrent.futures import ThreadPoolExecutor
    t0 = time.perf_counter()
    if threads == 1:
        worker(0)
    else:
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(worker, range(threads)))
    dt = time.perf_counter() - t0
    nnz = sum(done)
    gflops = 2.0 * nnz * N / dt / 1e9
    sample = (f"{nnz} nonzeros x N={N} in {dt:.2f} s: 512-row blocks of the {m}-row matrix "
              f"({len(ix)} nnz) visited in order")
    return gflops, kind, sample, dt


class L2Flush:
    """Clears L2 (126 MB) between timed steps, outside the events: a 256 MiB
    write (the required flush), then a 256 MiB read of another buffer so that
    the evicted dirty lines are written back here and the timed kernel starts
    on a clean L2 rather than paying for the flush's own write-back."""

    def __init__(self, dev):
        import torch
        self.w = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
        self.r = torch.zeros(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
        self.out = torch.empty(1, dtype=torch.float32, device=dev)

    def __call__(self):
        import torch
        self.w.zero_()
        torch.sum(self.r, dim=0, keepdim=True, out=self.out)


def cusparse_baseline(mats, dev, flush, args):
    """cuSPARSE CSR SpMM (through torch.sparse_csr_tensor @ dense, row-major B
    and C) on the same inputs and with the same timing method: a reported
    baseline, not part of the product path."""
    import torch
    try:
        As, Bs = [], []
        for a, B in mats:
            m, n, ip, ix, dx = a
            As.append(torch.sparse_csr_tensor(torch.from_numpy(ip.astype(np.int32)),
                                              torch.from_numpy(ix.astype(np.int32)),
                                              torch.from_numpy(dx.astype(np.float32)), size=(m, n)).to(dev))
            Bs.append(torch.from_numpy(B).to(dev))
        for _ in range(3):
            for A, B in zip(As, Bs):
                A @ B
        torch.cuda.synchronize()
        tot = 0.0
        steps = min(args.steps, 50)
        for _ in range(steps):
            flush()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for A, B in zip(As, Bs):
                A @ B
            e.record()
            e.synchronize()
            tot += s.elapsed_time(e)
        ms = tot / steps
        flops = 2.0 * sum(len(a[3]) * B.shape[1] for a, B in mats)
        return {"value": flops / (ms * 1e-3) / 1e9, "unit": "GFLOP/s", "ms_per_step": ms,
                "how": "torch.sparse_csr_tensor @ dense (cusparseSpMM, CSR int32, row-major)"}
    except Exception as ex:  # reported baseline only
        return {"unavailable": str(ex)[:200]}


def reference_gpu_baseline(mats, flush, args):
    """The reference's own GPU kernel for this product, compiled from its
    headers for sm_100a into oracle/_ref (a reported baseline, never the
    product path): SpMMFullRowPanelGeneralKernel4With2BlockCacheLess for N > 4
    (generated for coarsening (4, 2)), SpmvComplexPatternDecomposeByRowSeperated
    for N = 1 (coarsening (4, 1)).  Run as the reference's benchmark runs it --
    one .cfmtx read by its loader, C zeroed outside the timed region, one launch
    per step timed with CUDA events -- with the L2 flushed before each step like
    our kernel."""
    import tempfile

    import torch

    import sparse_computation_b200 as sc
    from oracle import cpu
    if len(mats) != 1:
        return {"unavailable": "single-matrix workloads only"}
    (m, n, ip, ix, dx), B = mats[0]
    N = B.shape[1]
    spmv = N == 1
    so = "libref_gpu_spmv.so" if spmv else "libref_gpu_spmm.so"
    if N not in (1, 128) and not (N > 4 and N % 32 == 0):
        return {"unavailable": f"the reference's generated kernels cover N = 1 and N > 4 (multiple of 32), not {N}"}
    if not cpu.ref_available(so):
        return {"unavailable": f"oracle/_ref/{so} not built (needs the reference sources at build time)"}
    L = cpu.ref_lib(so)
    pre = "ref_gpu_spmv_" if spmv else "ref_gpu_spmm_"
    fn = lambda name: getattr(L, pre + name)  # noqa: E731
    kn = 1 if spmv else 2
    cf = sc.csr_to_compressed_format_converter(sc.CSR.from_arrays(m, n, ip, ix, dx), 4, kn)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, f"matrix-4-{kn}.cfmtx")
        cf.write(path)
        Bc = np.ascontiguousarray(B[:, 0] if spmv else B, np.float32)
        h = fn("create")(os.fsencode(path), Bc.ctypes.data) if spmv else \
            fn("create")(os.fsencode(path), Bc.ctypes.data, N)
    if not h:
        return {"unavailable": "reference loader or upload failed"}
    try:
        # the reference library carries its own CUDA runtime: it launches on the
        # legacy default stream (as the reference does), timed on that stream
        st = torch.cuda.default_stream()
        sp = None
        fn("zero")(h, sp)
        rc = fn("run")(h, sp)
        if rc != 0:
            return {"unavailable": f"reference kernel launch failed (cudaError {rc})"}
        torch.cuda.synchronize()
        out = np.zeros((m, N), np.float32)
        fn("result")(h, out.ctypes.data)
        ref = cpu.spmm_csr_float(ip, ix, dx, B)
        scale = cpu.spmm_csr_abs(ip, ix, dx, B)
        rel = float(np.max(np.abs(out.astype(np.float64) - ref) / np.maximum(scale, 1e-30)))
        steps = max(3, min(args.steps, 20))
        tot = 0.0
        for _ in range(2):
            fn("zero")(h, sp)
            fn("run")(h, sp)
        for _ in range(steps):
            flush()
            fn("zero")(h, sp)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(st)
            fn("run")(h, sp)
            e.record(st)
            e.synchronize()
            tot += s.elapsed_time(e)
        ms = tot / steps
        return {"value": 2.0 * len(ix) * N / (ms * 1e-3) / 1e9, "unit": "GFLOP/s", "kernel_us": ms * 1e3,
                "coarsening": [4, kn], "max_err_over_abs_scale": rel,
                "how": ("reference SpmvComplexPatternDecomposeByRowSeperated" if spmv else
                        "reference SpMMFullRowPanelGeneralKernel4With2BlockCacheLess") +
                       " built from its header for sm_100a (oracle/_ref), atomics into a zeroed C, CUDA events"}
    finally:
        fn("free")(h)


def small_b_sweep(args):
    """512x512 magnitude-pruned weights (config 2) at every sparsity, N in
    {1, 2, 4}: our kernel as one warm launch (L2-resident, as in serving) and
    as 200 launches replayed from one CUDA graph, next to cuSPARSE CSR SpMM
    launched back to back."""
    import torch

    import sparse_computation_b200 as sc
    from sparse_computation_b200 import workloads as wl
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    reps = 200

    def events_ms(fn, n):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        fn()
        torch.cuda.synchronize()
        s.record()
        for _ in range(n):
            fn()
        e.record()
        e.synchronize()
        return s.elapsed_time(e) / n

    rows = []
    km = 4 if args.kernel_m == "auto" else int(args.kernel_m)
    for sp in wl.CONFIG2_SPARSITIES:
        for N in (1, 2, 4):
            a, B = wl.config2(sp, N)
            m, n, ip, ix, dx = a
            cf = sc.csr_to_compressed_format_converter(sc.CSR.from_arrays(*a), km, args.kernel_n)
            plan = sc.SpMMPlan(cf, N, device=0, flags={"f32": 0, "f16": sc.SC_PLAN_VALUES_F16,
                                                       "bf16": sc.SC_PLAN_VALUES_BF16}[args.values])
            Bt = torch.from_numpy(B).to(dev)
            C = torch.empty((m, N), device=dev)
            ours = events_ms(lambda: plan.spmm(Bt, C, stream=stream), reps)
            g = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(dev)
            with torch.cuda.stream(side):
                plan.spmm(Bt, C, stream=side)
                torch.cuda.synchronize()
                with torch.cuda.graph(g, stream=side):
                    for _ in range(reps):
                        plan.spmm(Bt, C, stream=side)
            graph = events_ms(g.replay, 5) / reps
            A = torch.sparse_csr_tensor(torch.from_numpy(ip.astype(np.int32)), torch.from_numpy(ix.astype(np.int32)),
                                        torch.from_numpy(dx.astype(np.float32)), size=(m, n)).to(dev)
            Bc = Bt if N > 1 else Bt.view(n, 1)
            cus = events_ms(lambda: A @ Bc, reps)
            fl = 2.0 * len(ix) * N
            rows.append({"sparsity": sp, "n_cols_b": N, "nnz": int(len(ix)),
                         "ours_us": ours * 1e3, "ours_graph_us": graph * 1e3, "cusparse_us": cus * 1e3,
                         "ours_gflops": fl / (ours * 1e-3) / 1e9, "ours_graph_gflops": fl / (graph * 1e-3) / 1e9,
                         "cusparse_gflops": fl / (cus * 1e-3) / 1e9, "speedup_vs_cusparse": cus / ours,
                         "graph_speedup_vs_cusparse": cus / graph})
    print(json.dumps({"metric": "SpMM GFLOP/s (2*nnz*N)", "unit": "GFLOP/s", "config": {
        "workload": "config2 sweep: A 512x512 magnitude-pruned N(0,0.05^2), B 512xN",
        "coarsening": [km, args.kernel_n], "values": args.values, "l2": "warm (L2-resident)"},
        "sweep": rows}), flush=True)


# ----------------------------------------------------------- reference ---

def run_reference(args, rank):
    if rank != 0:
        return
    name, mats = workload(args.config, args.n_cols_b)
    threads = len(os.sched_getaffinity(0))
    total_nnz = sum(len(a[3]) for a, _ in mats)
    N = mats[0][1].shape[1]
    # each step: a bounded sample (~0.25 s of all-core work)
    vals = []
    kind = sample = None
    for i in range(args.warmup + args.steps):
        g, kind, sample, dt = cpu_reference_rate(mats, 0.25, threads)
        if i >= args.warmup:
            vals.append(g)
    v = statistics.median(vals)
    line = {"metric": "SpMM GFLOP/s (2*nnz*N)", "value": v, "unit": "GFLOP/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 2.0 * total_nnz * N / (v * 1e9) * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)", "impl": "reference",
            "config": {"workload": name, "coarsening": None, "n_cols_b": N},
            "cpu_baseline": {"value": v, "unit": "GFLOP/s", "cores": threads, "kind": kind,
                             "sample": sample + f"; spmm_csr_float on {threads} threads over row blocks"},
            "e2e": {"value": v, "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ ours --

def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist

    import sparse_computation_b200 as sc

    sc.lib()  # builds libsc_b200.so in-tree when it is missing (ranks of one node build once)

    if args.sweep_small:
        small_b_sweep(args)
        return

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", device_id=dev)

    name, mats = workload(args.config, args.n_cols_b)
    auto_m = args.kernel_m == "auto"
    km, kn = (4 if auto_m else int(args.kernel_m)), args.kernel_n
    N = mats[0][1].shape[1]

    # ---- setup: this rank's row blocks, coarsening, plans (untimed)
    t_setup = time.perf_counter()
    layers = args.config == 4  # independent matrices: shard whole matrices, no collective
    jobs = []
    total_nnz = sum(len(a[3]) for a, _ in mats)
    tuned = {}

    def pick_m(i, a):
        """kernel_m of matrix i: fixed, or measured per matrix (--kernel-m auto)."""
        if not auto_m:
            return km
        if i not in tuned:
            from sparse_computation_b200 import tuning
            tuned[i] = tuning.autotune_kernel_m(sc.CSR.from_arrays(*a), N, device=local)[0]
        return tuned[i]

    plan_flags = (sc.SC_PLAN_DENSE_BF16 if args.dense_bf16 else 0) | \
        {"f32": 0, "f16": sc.SC_PLAN_VALUES_F16, "bf16": sc.SC_PLAN_VALUES_BF16}[args.values]
    if layers:
        owner = lpt_assign([len(a[3]) for a, _ in mats], world)
        mine = [i for i, r in enumerate(owner) if r == rank]
        for i in mine:
            a, B = mats[i]
            mk = pick_m(i, a)
            cf = sc.csr_to_compressed_format_converter(sc.CSR.from_arrays(*a), mk, kn)
            plan = sc.SpMMPlan(cf, N, device=local, flags=plan_flags)
            jobs.append({"km": mk, "plan": plan, "B": torch.from_numpy(B).to(dev), "rows": a[0], "max_rows": a[0],
                         "m": a[0], "nnz_local": len(a[3]), "Bhost": B, "cuts": None, "K": a[1],
                         "C": torch.empty((a[0], N), device=dev)})
    else:
        for i, (a, B) in enumerate(mats):
            m = a[0]
            mk = pick_m(i, a)
            cuts = balanced_panel_cuts(a[2], m, mk, world)
            p0, p1 = cuts[rank], cuts[rank + 1]
            r0, r1 = min(p0 * mk, m), min(p1 * mk, m)
            blk = row_slice(a, r0, r1)
            cf = sc.csr_to_compressed_format_converter(sc.CSR.from_arrays(*blk), mk, kn)
            plan = sc.SpMMPlan(cf, N, device=local, flags=plan_flags)
            max_rows = max(min(cuts[r + 1] * mk, m) - min(cuts[r] * mk, m) for r in range(world))
            j = {"km": mk, "plan": plan, "B": torch.from_numpy(B).to(dev), "rows": r1 - r0, "max_rows": max_rows,
                 "m": m, "nnz_local": len(blk[3]), "Bhost": B, "cuts": cuts, "K": a[1]}
            if world > 1 and args.exchange.startswith("peer"):
                full, hdl = symmetric_buffer((m, N), dev)
                j["full"], j["hdl"] = full, hdl
                j["C"] = full[r0:r1]
                j["peers"] = [int(hdl.buffer_ptrs[q]) + r0 * N * 4 for q in range(world) if q != rank]
                flags, fh = symmetric_buffer((world,), dev, torch.int32)
                flags.zero_()
                j["flags"], j["flag_ptrs"] = flags, [int(fh.buffer_ptrs[q]) + rank * 4 for q in range(world)]
                j["status"] = torch.zeros(1, dtype=torch.int32, device=dev)
                fh.barrier(channel=0)
            else:
                j["gather"] = torch.empty((world, max_rows, N), device=dev)
                j["C"] = j["gather"][rank, : j["rows"]] if world > 1 else torch.empty((j["rows"], N), device=dev)
            jobs.append(j)
    # one batched launch per kernel_m group of wide-B plans
    batches = []
    if len(jobs) > 1 and jobs[0]["plan"].info["kernel"] in (2, 3):
        for mk in sorted({j["km"] for j in jobs}):
            grp = [j for j in jobs if j["km"] == mk]
            bt = sc.SpMMBatch([j["plan"] for j in grp])
            bt.bind([j["B"] for j in grp], [j["C"] for j in grp])
            batches.append(bt)
    # config 4: each GPU's whole layer-stack product captured once into a CUDA
    # graph and replayed (one graph launch per step)
    graphs = []
    if layers and batches and not args.no_graph:
        graphs = [bt.capture(repeat=1) for bt in batches]
    t_setup = time.perf_counter() - t_setup

    peer_mode = world > 1 and not layers and args.exchange.startswith("peer")
    use_flags = args.exchange == "peer"
    epoch = [0]

    def launch_all(stream):
        if graphs:
            for g in graphs:
                g.launch(stream=stream)
        elif batches:
            for bt in batches:
                bt.spmm(stream=stream)  # every local matrix of one kernel_m in one kernel launch
        else:
            for j in jobs:
                if peer_mode:  # the kernel stores each C tile locally and into every peer's C
                    if use_flags:
                        epoch[0] += 1
                        j["plan"].spmm_peers(j["B"], j["C"], j["peers"], stream=stream, flag_ptrs=j["flag_ptrs"],
                                             epoch=epoch[0])
                    else:
                        j["plan"].spmm_peers(j["B"], j["C"], j["peers"], stream=stream)
                else:
                    j["plan"].spmm(j["B"], j["C"], stream=stream)

    def gather_all():
        if peer_mode:
            for j in jobs:
                if use_flags:  # every rank's last CTA has published its epoch here
                    sc.wait_flags(j["flags"].data_ptr(), world, epoch[0], j["status"].data_ptr(), stream)
                else:
                    j["hdl"].barrier(channel=0)  # all ranks' peer stores have landed
        elif world > 1 and not layers:
            for j in jobs:
                # in place: this rank's block already sits at its slot
                dist.all_gather_into_tensor(j["gather"], j["gather"][rank])

    stream = torch.cuda.current_stream(dev)
    flush = L2Flush(dev)

    def step():
        launch_all(stream)
        gather_all()

    kernel_events = []

    with ClockSampler(local) as clocks:
        for _ in range(args.warmup):
            flush()
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        clocks.timed = True
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        kstarts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        kends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        for i in range(args.steps):
            flush()
            starts[i].record(stream)
            kstarts[i].record(stream)
            launch_all(stream)
            kends[i].record(stream)
            gather_all()
            ends[i].record(stream)
        clocks.sample_now()  # the GPU is still working through the timed steps
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        clocks.timed = False
        step_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
        kern_ms = sum(s.elapsed_time(e) for s, e in zip(kstarts, kends)) / args.steps

        # ---- e2e: host B -> device, product, gather, C -> host
        e2e_steps = max(10, min(args.steps, 50))
        if world == 1 and len(jobs) == 1:
            j = jobs[0]
            hB = torch.from_numpy(j["Bhost"]).pin_memory()
            hC = torch.empty((j["rows"], N), dtype=torch.float32).pin_memory()
            hBn, hCn = hB.numpy(), hC.numpy()
            for _ in range(3):
                j["plan"].spmm_host(hBn, hCn, stream=stream)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(e2e_steps):
                j["plan"].spmm_host(hBn, hCn, stream=stream)  # sc_spmm_host: H2D, kernel, D2H, sync
            e2e_s = (time.perf_counter() - t0) / e2e_steps
            h2d = j["Bhost"].nbytes
            d2h = hC.numel() * 4
        else:
            hBs = [torch.from_numpy(j["Bhost"]).pin_memory() for j in jobs]
            hCs = [torch.empty((j["m"], N), dtype=torch.float32).pin_memory() for j in jobs]

            def e2e_step():
                for j, hB in zip(jobs, hBs):
                    j["B"].copy_(hB, non_blocking=True)
                launch_all(stream)
                gather_all()
                if layers:
                    for j, hC in zip(jobs, hCs):
                        hC.copy_(j["C"], non_blocking=True)
                elif rank == 0 and peer_mode:
                    for j, hC in zip(jobs, hCs):
                        hC.copy_(j["full"], non_blocking=True)
                elif rank == 0:
                    for j, hC in zip(jobs, hCs):
                        for r in range(world):
                            a0 = min(j["cuts"][r] * j["km"], j["m"])
                            a1 = min(j["cuts"][r + 1] * j["km"], j["m"])
                            src = j["gather"][r, : a1 - a0] if world > 1 else j["C"]
                            hC[a0:a1].copy_(src, non_blocking=True)
                torch.cuda.synchronize()

            for _ in range(3):
                e2e_step()
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            for _ in range(e2e_steps):
                e2e_step()
            e2e_s = (time.perf_counter() - t0) / e2e_steps
            h2d = sum(j["Bhost"].nbytes for j in jobs)
            d2h = sum(j["m"] * N * 4 for j in jobs) if (rank == 0 or layers) else 0

    exchange_status = 0
    if peer_mode and use_flags:
        exchange_status = max(int(j["status"].item()) for j in jobs)  # 5: a flag wait expired
    # ---- reduce over ranks (max time)
    t = torch.tensor([step_ms, kern_ms, e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms, kern_ms, e2e_s = t.tolist()
    flops = 2.0 * total_nnz * N
    ms_per_step = step_ms / args.steps
    value = flops / (ms_per_step * 1e-3) / 1e9
    e2e_value = flops / e2e_s / 1e9

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    # ---- roofline of the dominant kernel (the SpMM launch of this rank)
    # this rank's launch(es): values + B read once + C written once, per matrix
    alg_bytes = sum(4.0 * j["nnz_local"] + 4.0 * j["K"] * N + 4.0 * j["rows"] * N for j in jobs)
    peak, peak_kind = measured_peak_hbm()
    achieved = alg_bytes / (kern_ms * 1e-3) / 1e9
    props = torch.cuda.get_device_properties(dev)
    clk = clocks.summary()
    sm_max = clk["sm_max_mhz"] or 1965.0
    fp32_peak = props.multi_processor_count * 128 * 2 * sm_max * 1e6 / 1e12
    local_flops = 2.0 * sum(j["nnz_local"] for j in jobs) * N
    traffic = measured_traffic(f"config{args.config}_n{N}_m{km}_{kn}_gpus{world}")
    # L1/shared data-pipe bound of the gather kernel (wide-B plans): every
    # (panel, column) entry loads one N-float B row (ceil(4N/128) wavefronts of
    # 128 bytes) plus ~1 wavefront for its record; the pipe moves one wavefront
    # per cycle per SM
    wide_entries = sum(j["plan"].info["entries"] for j in jobs if j["plan"].info["kernel"] == 2)
    gather_us = (wide_entries * (-(-4 * N // 128) + 1) / (props.multi_processor_count * sm_max * 1e6) * 1e6
                 if wide_entries else None)
    info = jobs[0]["plan"].info

    line = {
        "metric": "SpMM GFLOP/s (2*nnz*N)", "value": value, "unit": "GFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": ("bf16 tiles, f32 accumulate" if any(j["plan"].info["dense_bf16"] for j in jobs) else
                  {0: "f32", 1: "f16 values, f32 accumulate", 2: "bf16 values, f32 accumulate"}[
                      max(j["plan"].info["value_type"] for j in jobs)]),
        "data": "synthetic (seeded)",
        "config": {"workload": name,
                   "coarsening": ([km, kn] if not auto_m else
                                  {"kernel_m": "auto (measured per matrix)", "chosen": sorted({j["km"] for j in jobs}),
                                   "kernel_n": kn}),
                   "n_cols_b": N, "nnz": total_nnz,
                   "exchange": args.exchange if world > 1 and not layers else None,
                   "parallelism": ("1 GPU" if world == 1 else
                                   f"whole matrices sharded over {world} GPUs (LPT by nnz), no collective"
                                   if layers else
                                   (f"row-partition x{world}; SpMM kernel stores C tiles into every peer over "
                                    "NVLink (symmetric memory) + one barrier" if peer_mode else
                                    f"row-partition x{world} + NCCL all-gather of C")),
                   "launches_per_step": len(batches) if batches else len(jobs),
                   "cuda_graph": bool(graphs),
                   "l2": "flushed before every timed step (256 MiB write, then a 256 MiB read of another buffer so the "
                         "flush's dirty lines are written back; outside the events)",
                   "plan": {k: info[k] for k in ("entries", "items", "kernel", "warps_per_panel",
                                                 "device_bytes")}},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_kind, "traffic": traffic,
                     "kernel_us": kern_ms * 1e3,
                     "algorithmic_bytes": alg_bytes,
                     "fp32_tflops": local_flops / (kern_ms * 1e-3) / 1e12,
                     "fp32_peak_tflops": fp32_peak,
                     "fp32_frac": local_flops / (kern_ms * 1e-3) / 1e12 / fp32_peak,
                     "gather_bound_us": gather_us,
                     "gather_frac": (gather_us / (kern_ms * 1e3)) if gather_us else None},
        "e2e": {"value": e2e_value, "unit": "GFLOP/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_s * 1e3},
        "gpu_launches": args.steps * (len(batches) if batches else len(jobs)) * (2 if peer_mode and use_flags else 1),
        "exchange_status": exchange_status,
        "clocks": clk,
        "setup_s": t_setup,
    }
    if world == 1:
        line["cusparse"] = cusparse_baseline(mats, dev, flush, args)
        try:
            line["reference_gpu"] = reference_gpu_baseline(mats, flush, args)
        except Exception as ex:  # reported baseline only
            line["reference_gpu"] = {"unavailable": f"{type(ex).__name__}: {ex}"[:200]}
    if world == 1 and not args.no_cpu_baseline:
        g, kind, sample, dt = cpu_reference_rate(mats, args.cpu_seconds, 1)
        line["cpu_baseline"] = {"value": g, "unit": "GFLOP/s", "cores": 1, "kind": kind,
                                "sample": sample + "; serial spmm_csr_float as in the reference"}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
