#!/usr/bin/env python
"""Benchmark of the packed PentaLinear path on B200.

Workload (headline): 70B-class decode GEMV -- the packed layers K->N =
8192->28672 and 28672->8192 at batch M in {1, 8, 64} (bf16 activations,
N(0,1); weights N(0,0.02) absmean-quantised and packed).  One step runs the
six (shape, M) products once.  The metric is HBM GB/s of algorithmic bytes
(4*N*ceil(K/10) packed weight bytes + 2*M*K activation bytes + 2*M*N output
bytes per product) divided by device time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's own CPU kernel (penta_avx2.c compiled
from source into oracle/_ref/, or the oracle port when it is absent) on the
same workload with all host threads, on a bounded row sample per step.

At N > 1 (torchrun) every layer is sharded by output rows over the ranks: each
rank's GEMM stores its output columns straight into every GPU's full-output
buffer (CUDA IPC peer mappings over NVLink) and a cross-GPU barrier kernel
ends each product, so every GPU holds the whole output (strong scaling: the
total work is fixed).  The sharded outputs are checked against the unsharded
product on every rank.

The printed JSON line carries the device-timed value, an end-to-end number
through the public API with host buffers, the roofline of the dqmm kernel, a
CPU baseline, kernel-launch counts and the SM clocks sampled during timing.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "pentanet-v1.0_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "PentaLinear GEMV HBM GB/s & GEMM int8 TOPS vs roofline; 124M fwd tokens/s"
SHAPES = [(8192, 28672), (28672, 8192)]   # (K, N)
BATCHES = [1, 8, 64]
COPIES = 4                                  # weight copies per shape, rotated (4 x 2 x 94 MB >> L2)
FALLBACK_HBM_GBS = 6650.0


PREFILL_SHAPES = [(4096, 4096), (4096, 11008), (11008, 4096)]   # (K, N), 7B-class layers
PREFILL_COPIES = 6
PREFILL_M = 4096


def k_packs(K: int) -> int:
    return (K + 9) // 10


def alg_bytes(M: int, K: int, N: int) -> int:
    return 4 * N * k_packs(K) + 2 * M * K + 2 * M * N


def launches_per_step():
    return [(M, K, N) for M in BATCHES for (K, N) in SHAPES]


def step_bytes(world: int = 1) -> int:
    # algorithmic bytes of the whole (unsharded) layer products
    return sum(alg_bytes(M, K, N) for (M, K, N) in launches_per_step())


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d.get("bf16_tflops", 0)),
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": 1590.0, "source": "fallback"}


def kernel_source_sha() -> str:
    """sha256 of the decode GEMM's sources (the kernel an ncu capture describes)."""
    import hashlib
    h = hashlib.sha256()
    for f in ("pn_dqmm.cu", "pn_common.cuh"):
        with open(os.path.join(PKG, "csrc", f), "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()[:16]


def profile_traffic():
    """DRAM bytes per launch of the dqmm kernel from the committed ncu summary,
    used only when the summary was captured from the current kernel source
    (its `kernel_source_sha:` line); returns (bytes or None, source note)."""
    path = os.path.join(ROOT, "profiles", "dqmm_gemv_70b_decode.md")
    if not os.path.exists(path):
        return None, "no ncu summary"
    traffic = sha = None
    for line in open(path):
        if line.startswith("traffic_bytes_per_launch_full_size:"):
            try:
                traffic = float(line.split(":", 1)[1].strip())
            except ValueError:
                traffic = None
        if line.startswith("kernel_source_sha:"):
            sha = line.split(":", 1)[1].strip()
    if sha != kernel_source_sha():
        return None, "profiles/dqmm_gemv_70b_decode.md was captured from another kernel source: not used"
    return traffic, f"ncu capture of this kernel source ({sha}), profiles/dqmm_gemv_70b_decode.md"


# --------------------------------------------------------------- clocks ----

class ClockSampler:
    """Samples SM clock and throttle reasons with NVML (every ~1 ms) from the
    start of the warm-up to the end of the per-launch timing; `window` marks
    the timed region so the summary can say how many samples fell inside it."""

    def __init__(self, device_indices):
        self.samples = []
        self.ok = False
        self._stop = threading.Event()
        self._th = None
        self.max_mhz = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.handles = [nv.nvmlDeviceGetHandleByIndex(i) for i in device_indices]
            self.max_mhz = max(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM) for h in self.handles)
            self.ok = True
        except Exception:  # NVML unavailable: report no clocks rather than guess
            self.ok = False

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            for h in self.handles:
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((time.time(), sm, reasons))
                except Exception:
                    pass
            time.sleep(0.001)

    def start(self):
        if self.ok:
            self._th = threading.Thread(target=self._run, daemon=True)
            self._th.start()

    def stop(self):
        if self._th:
            self._stop.set()
            self._th.join()

    window = None

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        nv = self.nv
        names = {
            "gpu_idle": getattr(nv, "nvmlClocksEventReasonGpuIdle", 0x1),
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        seen = set()
        for _, _, r in self.samples:
            for k, bit in names.items():
                if k != "gpu_idle" and r & bit:
                    seen.add(k)
        inside = [s for t, s, _ in self.samples if self.window and self.window[0] <= t <= self.window[1]]
        return {"sm_mhz": statistics.median(s for _, s, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(seen), "samples": len(self.samples),
                "samples_in_timed_region": len(inside),
                "sm_mhz_timed_region": statistics.median(inside) if inside else None,
                "sampled": "warm-up, timed region and per-launch timing, every ~1 ms"}


# ------------------------------------------------------- CPU reference -----

def host_cpu() -> dict:
    """Host CPU facts recorded beside every CPU number."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return {"cpu_model": model, "affinity_cores": cores, "env_OMP_NUM_THREADS": os.environ.get("OMP_NUM_THREADS")}


def _timed_reps(fn, reps: int, warmup: int, budget_s: float):
    """Run fn `warmup` times, then up to `reps` times or until budget_s has
    passed (at least once); returns (seconds per rep, reps run)."""
    for _ in range(warmup):
        fn()
    n = 0
    t0 = time.perf_counter()
    while True:
        fn()
        n += 1
        dt = time.perf_counter() - t0
        if n >= reps or dt >= budget_s:
            return dt / n, n


def cpu_reference_rate(sample_rows: int, reps: int, warmup: int, seed: int = 0, budget_s: float = 20.0):
    """The reference's CPU kernel (penta_matmul_avx2 over int8 weights from
    penta_unpack_3bit, as penta_avx2_wrapper.py:37-94 runs it) on the six
    products, restricted to the first `sample_rows` output rows of each layer,
    with every host core the process may use (OpenMP threads set explicitly:
    launchers such as torchrun export OMP_NUM_THREADS=1).
    Returns a dict: value (GB/s of algorithmic bytes), seconds per sample,
    kind, cores (threads used), sample description, reps, host facts."""
    import numpy as np
    import torch
    from oracle import oracle as orc

    kind = "reference" if orc.ref_avx2_available() else "port"
    host = host_cpu()
    cores = host["affinity_cores"]
    threads = orc.ref_omp_threads(cores) if kind == "reference" else 1
    g = torch.Generator().manual_seed(seed)
    layers = {}
    for (K, N) in SHAPES:
        n = min(sample_rows, N)
        w = (torch.randn(n, K, generator=g) * 0.02).numpy()
        packed, _, gamma = orc.quantize_pack(w)
        w8 = orc.ref_avx2_unpack(packed, K) if kind == "reference" else orc.unpack(packed, K)
        layers[(K, N)] = (w8, gamma, n, packed)
    xs = {(M, K): torch.randn(M, K, generator=g).to(torch.bfloat16).float().numpy()
          for (M, K, _) in launches_per_step()}
    outs = {(M, K, N): np.empty((M, layers[(K, N)][2]), dtype=np.float32) for (M, K, N) in launches_per_step()}

    def one():
        for (M, K, N) in launches_per_step():
            w8, gamma, n, _ = layers[(K, N)]
            if kind == "reference":
                orc.ref_avx2_linear(xs[(M, K)], w8, gamma, outs[(M, K, N)])
            else:
                outs[(M, K, N)][...] = orc.matmul_f32(xs[(M, K)], w8, gamma)

    dt, n_reps = _timed_reps(one, reps, warmup, budget_s)
    sample_bytes = sum(alg_bytes(M, K, layers[(K, N)][2]) for (M, K, N) in launches_per_step())
    desc = (f"rows 0..{sample_rows} of each layer (of 28672 / 8192), all six (shape, M) products per step; "
            f"{'penta_matmul_avx2 (-O3 -mavx2 -mfma -fopenmp)' if kind == 'reference' else 'scalar oracle port'}"
            f"; {n_reps} timed reps after {warmup} warm-up")
    res = {"value": round(sample_bytes / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": kind,
           "sample": desc, "s_per_sample": round(dt, 4), "reps": n_reps,
           "threads": {"omp_max_threads": threads, "torch": torch.get_num_threads()}, **host}
    return res, layers, xs


def cpu_numba_rate(layers, xs, reps: int, warmup: int, budget_s: float = 10.0):
    """The reference's numba kernel (penta_linear_cpu, penta_kernel_cpu.py:63-101,
    restated in oracle/numba_port.py: per-call unpack of the packed words, then
    the five-way add/subtract loop parallel over output rows) on the same
    sample as the AVX2 leg, all host cores."""
    import torch
    from oracle import numba_port as nbp
    if not nbp.AVAILABLE:
        return {"unavailable": "numba not importable"}
    threads = nbp.threads(host_cpu()["affinity_cores"])
    tl = {k: torch.from_numpy(v[3]) for k, v in layers.items()}
    tx = {k: torch.from_numpy(v) for k, v in xs.items()}

    def one():
        for (M, K, N) in launches_per_step():
            nbp.penta_linear_cpu(tx[(M, K)], tl[(K, N)], layers[(K, N)][1], K)

    one()  # JIT compile (and warm-up) outside the timing
    dt, n_reps = _timed_reps(one, reps, 0, budget_s)
    sample_bytes = sum(alg_bytes(M, K, layers[(K, N)][2]) for (M, K, N) in launches_per_step())
    return {"value": round(sample_bytes / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": "same rows and products as the AVX2 leg; numba restatement of penta_linear_cpu "
                      f"(per-call unpack included); {n_reps} timed reps",
            "s_per_sample": round(dt, 4)}


def cpu_int_mm_rate(reps: int, warmup: int, rows: int = 512, budget_s: float = 10.0):
    """The reference's CPU int8 line for the 7B-class prefill shapes
    (penta_avx2_wrapper.py:130-131,137,147: torch._int_mm of per-tensor int8
    activations and int8 weights, then the float rescale) at M = 4096 on the
    first `rows` output rows of each layer; TOP/s of 2*M*rows*K."""
    import torch
    threads = torch.get_num_threads()
    torch.set_num_threads(host_cpu()["affinity_cores"])
    g = torch.Generator().manual_seed(5)
    cases = []
    for (K, N) in PREFILL_SHAPES:
        x = torch.randn(PREFILL_M, K, generator=g)
        w8 = torch.randint(-2, 3, (rows, K), generator=g, dtype=torch.int8)
        xs = x.abs().max() / 127.0
        x8 = (x / xs).round().clamp(-128, 127).to(torch.int8)
        cases.append((x8, w8.t(), float(xs) * 0.02))

    def one():
        for (x8, wt, sc) in cases:
            torch._int_mm(x8, wt).float() * sc

    try:
        dt, n_reps = _timed_reps(one, reps, warmup, budget_s)
    except RuntimeError as e:  # no CPU _int_mm kernel in this torch build
        torch.set_num_threads(threads)
        return {"unavailable": str(e).splitlines()[0][:200]}
    ops = sum(2.0 * PREFILL_M * rows * K for (K, N) in PREFILL_SHAPES)
    used = torch.get_num_threads()
    torch.set_num_threads(threads)
    return {"value": round(ops / dt / 1e12, 4), "unit": "TOP/s", "cores": used, "kind": "port",
            "sample": f"M={PREFILL_M}, first {rows} output rows of 4096->4096, 4096->11008, 11008->4096; "
                      f"torch._int_mm as penta_avx2_wrapper.py runs it; {n_reps} timed reps",
            "s_per_sample": round(dt, 4)}


def cpu_legs(reps: int, warmup: int) -> dict:
    rows = int(os.environ.get("PN_REF_ROWS", "2048"))
    res, layers, xs = cpu_reference_rate(rows, reps, warmup)
    res["legs"] = {"numba_penta_linear_cpu": cpu_numba_rate(layers, xs, reps, warmup),
                   "int_mm_prefill_7b": cpu_int_mm_rate(reps, warmup)}
    return res


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the CPU reference runs once per node, on rank 0
    rows = int(os.environ.get("PN_REF_ROWS", "2048"))
    res, _, _ = cpu_reference_rate(rows, max(1, args.steps), args.warmup)
    rate = res["value"]
    line = {"metric": METRIC, "value": rate, "unit": "GB/s", "n_gpus": args.gpus, "steps": res["reps"],
            "warmup": args.warmup, "ms_per_step": round(res["s_per_sample"] * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "70B-class decode GEMV: K->N 8192->28672 and 28672->8192, M in {1,8,64}",
                       "sample": res["sample"]},
            "cpu_baseline": res,
            "e2e": {"value": rate, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ our arm -----

def decode_kernel_label() -> str:
    """Which dqmm instantiations run the decode products (limb path up to the
    library's current limit, kind::f16 above it)."""
    import penta_native as nat
    lim = nat.load().pn_set_limb_max_tokens(-1)
    parts = [f"pn::dqmm_kernel<L8, 4M columns> + limb_x_kernel for M <= {lim}"] if lim > 0 else []
    parts.append("pn::dqmm_kernel<F16, BT> + permute_x_kernel" + (f" for M > {lim}" if lim > 0 else ""))
    return "; ".join(parts)


def run_profile_case(args):
    """Small case for ncu --set full: both 70B-class layers (94 MB packed each,
    one copy), one launch each at M = 1, 8, 64, after three warm-up launches."""
    import torch
    import penta_kernel as pk
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(1234)
    layers = []
    for (K, N) in SHAPES:
        w = torch.randn(N, K, device=dev, generator=gen) * 0.02
        packed, _, s = pk.quantize_and_pack(w)
        del w
        layers.append((K, N, packed, s))
    torch.cuda.empty_cache()
    xs = {(M, K): torch.randn(M, K, device=dev, generator=gen).to(torch.bfloat16)
          for M in BATCHES for (K, _, _, _) in layers}
    K0, _, p0, s0 = layers[0]
    for _ in range(3):
        pk.penta_linear(xs[(1, K0)], p0, s0, K0)
    for (K, N, packed, s) in layers:
        for M in BATCHES:
            pk.penta_linear(xs[(M, K)], packed, s, K)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": "dqmm 8192->28672 and 28672->8192", "warmup_launches": 3,
                      "launches": len(layers) * len(BATCHES)}))


def _graph_time(fn, n_launch: int) -> float:
    """Seconds per call of fn(i), i = 0..n_launch-1, from one CUDA graph replay."""
    import torch
    for i in range(2):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n_launch):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / n_launch * 1e-3


def _max_over_ranks(v: float, world: int, dev) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def prefill_int8(dev, gen, peaks, world: int = 1, rank: int = 0):
    """Secondary measurement: the int8 prefill GEMM (per-token int8 activations
    x packed weights on the int8 tensor cores) at M = 4096 on the 7B-class
    layer shapes.  Reports the GEMM alone (activations already quantised) and
    with the activation quantiser, each from CUDA graphs of 12 launches that
    rotate over PREFILL_COPIES copies of weights and activations (more than L2
    between two uses of a copy).  Weights are in the layer's resident layout
    (rows at a 16-byte stride, penta_kernel.pad_packed).

    At N > 1 every layer is column-sharded: rank r holds the packed rows
    shard_range(N, r, world) (its output columns) and computes its (M, N/P)
    block; the times are the max over ranks and the value counts the whole
    layer's 2*M*N*K.  `with_all_gather` adds the NCCL all-gather of the output
    blocks into the full (M, N) result (penta_dist.gather_columns, eager), and
    the gathered result is compared bit for bit with the unsharded product."""
    import torch
    import penta_kernel as pk
    import penta_dist as pd
    rows = []
    tot_ops = tot_gemm = tot_e2e = tot_gather = 0.0
    n_launch = 2 * PREFILL_COPIES
    parity = True
    for (K, N) in PREFILL_SHAPES:
        lo, hi = pd.shard_range(N, rank, world)
        packs, xs, xqs = [], [], []
        full0 = None
        for c in range(PREFILL_COPIES):
            w = torch.randn(N, K, device=dev, generator=gen) * 0.02
            packed, _, s = pk.quantize_and_pack(w)
            del w
            if c == 0 and world > 1:
                full0 = (pk.pad_packed(packed), s)
            packs.append((pk.pad_packed(packed[lo:hi].contiguous()), s))
            del packed
            x = torch.randn(PREFILL_M, K, device=dev, generator=gen).to(torch.bfloat16)
            xs.append(x)
            xqs.append(pk.quantize_activations_i8(x))
        torch.cuda.synchronize()

        def gemm(i):
            xq, s_x, rowsum = xqs[i % PREFILL_COPIES]
            pw, s = packs[i % PREFILL_COPIES]
            return pk.penta_linear_i8_prequant(xq, s_x, rowsum, K, pw, s)

        def full(i):
            pw, s = packs[i % PREFILL_COPIES]
            return pk.penta_linear_i8(xs[i % PREFILL_COPIES], pw, s, K)

        t_gemm = _max_over_ranks(_graph_time(gemm, n_launch), world, dev)
        t_full = _max_over_ranks(_graph_time(full, n_launch), world, dev)
        row = {"M": PREFILL_M, "K": K, "N": N, "cols_local": hi - lo, "gemm_us": round(t_gemm * 1e6, 1),
               "with_quant_us": round(t_full * 1e6, 1)}
        ops = 2.0 * PREFILL_M * N * K
        if world > 1:
            import torch.distributed as dist
            y_full = torch.empty(PREFILL_M, N, dtype=torch.bfloat16, device=dev)
            for i in range(2):
                pd.gather_columns(gemm(i), N, world, out=y_full)
            torch.cuda.synchronize()
            dist.barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(n_launch):
                pd.gather_columns(gemm(i), N, world, out=y_full)
            e1.record()
            torch.cuda.synchronize()
            t_gather = _max_over_ranks(e0.elapsed_time(e1) / n_launch * 1e-3, world, dev)
            row["with_all_gather_us"] = round(t_gather * 1e6, 1)
            tot_gather += t_gather
            # parity: the gathered columns equal the unsharded product bit for bit
            pd.gather_columns(gemm(0), N, world, out=y_full)
            xq, s_x, rowsum = xqs[0]
            want = pk.penta_linear_i8_prequant(xq, s_x, rowsum, K, full0[0], full0[1])
            ok = torch.tensor([1 if torch.equal(y_full, want) else 0], device=dev)
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            row["parity"] = "bit-exact" if int(ok.item()) == 1 else "MISMATCH"
            parity = parity and int(ok.item()) == 1
            del y_full, want
        row["tops"] = round(ops / t_gemm / 1e12, 1)
        tot_ops += ops
        tot_gemm += t_gemm
        tot_e2e += t_full
        rows.append(row)
        del packs, xs, xqs, full0
        torch.cuda.empty_cache()
    peak = 2.0 * peaks["bf16_tflops"] * world
    res = {"workload": f"int8 prefill GEMM, M={PREFILL_M}, K->N 4096->4096, 4096->11008, 11008->4096"
                       + (f", output columns sharded over {world} GPUs" if world > 1 else ""),
           "inputs": f"{PREFILL_COPIES} copies of weights and activations rotated (larger than L2 between uses)",
           "value": round(tot_ops / tot_gemm / 1e12, 1), "unit": "TOPS",
           "with_activation_quant": round(tot_ops / tot_e2e / 1e12, 1),
           "roofline": {"bound": "tensor", "achieved": round(tot_ops / tot_gemm / 1e12, 1), "peak": round(peak, 1),
                        "unit": "TOP/s", "frac": round(tot_ops / tot_gemm / 1e12 / peak, 4),
                        "peak_source": "2 x measured dense bf16 (MEASURED_PEAKS.json) per GPU x GPUs; B200's "
                                       "dense int8 rate is twice its bf16 rate", "kernel": "pn::dqmm_kernel<I8, 256>"},
           "per_shape": rows}
    if world > 1:
        res["with_all_gather"] = round(tot_ops / tot_gather / 1e12, 1)
        res["per_gpu_tops"] = round(tot_ops / tot_gemm / 1e12 / world, 1)
        res["parity"] = "bit-exact" if parity else "MISMATCH"
    return res


def pack_secondary(dev, peaks):
    """Secondary measurement: quantise + 3-bit pack of the 70B-class fp32
    master weights on the device (pn_absmean_scale, then pn_quantize_pack,
    gamma kept on the device), and the pack kernel alone with gamma given.
    Algorithmic bytes: one read of W (4 N K) + the packed words (4 N K_packs);
    the two-pass form reads W twice."""
    import torch
    import penta_kernel as pk
    import penta_native as nat
    L = nat.load()
    res = {"workload": "quantize_and_pack of fp32 W 28672x8192 and 8192x28672 (940 MB each)", "unit": "GB/s"}
    per = []
    tot_b = tot_two = tot_one = 0.0
    for (N, K) in ((28672, 8192), (8192, 28672)):
        g = torch.Generator(device=dev).manual_seed(N)
        w = torch.randn(N, K, device=dev, generator=g) * 0.02
        kp = (K + 9) // 10
        packed = torch.empty(N, kp, dtype=torch.int32, device=dev)
        d_scale = torch.empty((), dtype=torch.float32, device=dev)
        ws = torch.empty(int(L.pn_absmean_workspace_size()), dtype=torch.uint8, device=dev)
        sp = torch.cuda.current_stream(dev).cuda_stream

        def absmean():
            nat.check(L.pn_absmean_scale(w.data_ptr(), nat.PN_F32, N * K, d_scale.data_ptr(), ws.data_ptr(),
                                         ws.numel(), sp), "pn_absmean_scale")

        def pack():
            nat.check(L.pn_quantize_pack(w.data_ptr(), nat.PN_F32, N, K, d_scale.data_ptr(), packed.data_ptr(), sp),
                      "pn_quantize_pack")

        def timed(fn, reps=5):
            fn()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / reps * 1e-3

        t_two = timed(lambda: (absmean(), pack()))
        t_one = timed(pack)
        b = 4.0 * N * K + 4.0 * N * kp
        want, _, _ = pk.quantize_and_pack(w)
        assert torch.equal(packed, want), "device-scale pack differs from quantize_and_pack"
        per.append({"N": N, "K": K, "us_scale_and_pack": round(t_two * 1e6, 1), "us_pack": round(t_one * 1e6, 1)})
        tot_b += b
        tot_two += t_two
        tot_one += t_one
        del w, packed
        torch.cuda.empty_cache()
    res["value"] = round(tot_b / tot_two / 1e9, 1)
    res["pack_only"] = round(tot_b / tot_one / 1e9, 1)
    res["roofline"] = {"bound": "hbm", "achieved": res["value"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                       "frac": round(res["value"] / peaks["hbm_gbs"], 4),
                       "frac_pack_only": round(res["pack_only"] / peaks["hbm_gbs"], 4),
                       "kernel": "pn::absmean_partial/final + pn::quantize_pack_kernel<float>"}
    res["per_shape"] = per
    return res


def gpt_roofline(gpt: dict, peaks: dict, world: int) -> dict:
    """Tensor roofline of the bf16 PentaGPT-124M forward.  Algorithmic FLOPs
    per forward of B x T tokens: the four projections of each of the 12
    layers, 2 (3 + 1 + 4 + 4) d^2 per token (d = 768); causal attention,
    QK^T and AV over the T/2 earlier positions on average, 2 T d per token
    per layer; the tied lm_head on the last position of each sequence,
    2 d V (V = 50257)."""
    B, T, d, L, V = 32, 1024, 768, 12, 50257
    proj = 2.0 * (3 + 1 + 4 + 4) * d * d * L * B * T
    attn = 2.0 * T * d * L * B * T
    head = 2.0 * d * V * B
    flops = proj + attn + head
    achieved = flops / (gpt["bf16"]["ms_per_forward"] * 1e-3) / 1e12
    peak = peaks["bf16_tflops"] * world
    return {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4), "flops_per_forward": flops,
            "peak_source": "measured dense bf16 (MEASURED_PEAKS.json) per GPU x GPUs"
                           if peaks.get("source") != "fallback" else "fallback",
            "note": "projections run as packed-weight bf16 products, attention as torch SDPA"}


def pentagpt_forward(dev, world: int = 1, rank: int = 0):
    """Secondary measurement: PentaGPT-124M forward (prefill) tokens/s -- 12
    layers, d 768, every projection packed, batch 32 x 1024 random token ids,
    random weights from seed 42; last-position logits as the reference's
    inference forward.  bf16 projections (the parity path) and the per-token
    int8 projections.  At N > 1 the batch is split over the ranks (pure
    replicas, 32/N sequences each, no collective); the time is the max over
    ranks and the value counts all 32 x 1024 tokens."""
    import torch
    from pentagpt import PentaGPTFast
    B, T = 32, 1024
    idx_all = torch.randint(0, 50257, (B, T), generator=torch.Generator().manual_seed(42))
    per = B // world
    idx = idx_all[rank * per:(rank + 1) * per].to(dev)
    res = {"workload": "PentaGPT-124M forward, batch 32 x seq 1024, random init seed 42"
                       + (f", batch split over {world} GPUs ({per} sequences each)" if world > 1 else ""),
           "unit": "tokens/s"}
    for name, aq in (("bf16", None), ("int8", "int8")):
        model = PentaGPTFast.random(seed=42, device=dev, act_quant=aq)
        model(idx)
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        reps = 5
        e0.record()
        for _ in range(reps):
            model(idx)
        e1.record()
        torch.cuda.synchronize()
        ms = _max_over_ranks(e0.elapsed_time(e1) / reps, world, dev)
        res[name] = {"tokens_per_s": round(per * world * T / (ms * 1e-3)), "ms_per_forward": round(ms, 2)}
        del model
        torch.cuda.empty_cache()
    res["value"] = res["bf16"]["tokens_per_s"]
    return res


def run_profile_gpt(args):
    """PentaGPT-124M bf16 forward (batch 32 x 1024), three calls, for a launch
    list of one forward under ncu (skip the first two calls' launches)."""
    import torch
    from pentagpt import PentaGPTFast
    dev = torch.device("cuda", 0)
    idx = torch.randint(0, 50257, (32, 1024), generator=torch.Generator().manual_seed(42)).to(dev)
    model = PentaGPTFast.random(seed=42, device=dev)
    for _ in range(3):
        model(idx)
    torch.cuda.synchronize()
    print(json.dumps({"profile": "pentagpt_124m_fwd", "forwards": 3}))


def run_profile_epilogue(args):
    """The PentaGPT c_fc product (M 32768, K 768 -> N 3072, bf16) without and
    with the GELU fused into its epilogue, three times each, alternating (for
    ncu: skip 4 dqmm launches, capture 2)."""
    import torch
    import penta_kernel as pk
    dev = torch.device("cuda", 0)
    M, N, K = 32768, 3072, 768
    g = torch.Generator(device=dev).manual_seed(1)
    packed, _, gamma = pk.quantize_and_pack(torch.randn(N, K, device=dev, generator=g) * 0.02)
    packed = pk.pad_packed(packed)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    for _ in range(3):
        pk.penta_linear(x, packed, gamma, K)
        pk.penta_linear(x, packed, gamma, K, act="gelu")
    torch.cuda.synchronize()
    print(json.dumps({"profile": "c_fc plain / fused gelu", "M": M, "N": N, "K": K}))


def run_profile_gemv(args):
    """Small case for ncu: the CUDA-core decode GEMV (opt-in path) on the
    8192->28672 layer at M = 1, three warm-up launches and one measured."""
    import torch
    import penta_kernel as pk
    import penta_native as nat
    nat.load().pn_set_gemv_max_tokens(8)
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(1)
    K, N = 8192, 28672
    w = torch.randn(N, K, device=dev, generator=gen) * 0.02
    packed, _, s = pk.quantize_and_pack(w)
    del w
    x = torch.randn(1, K, device=dev, generator=gen).to(torch.bfloat16)
    for _ in range(4):
        pk.penta_linear(x, packed, s, K)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": "CUDA-core GEMV 8192->28672, M=1", "warmup_launches": 3, "launches": 1}))


def run_profile_prefill(args):
    """Small case for ncu: the int8 prefill GEMM at M = 4096, K = N = 4096,
    three warm-up launches and one measured launch (activations quantised
    beforehand)."""
    import torch
    import penta_kernel as pk
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(1234)
    K = N = M = 4096
    w = torch.randn(N, K, device=dev, generator=gen) * 0.02
    packed, _, s = pk.quantize_and_pack(w)
    packed = pk.pad_packed(packed)
    del w
    x = torch.randn(M, K, device=dev, generator=gen).to(torch.bfloat16)
    xq, s_x, rowsum = pk.quantize_activations_i8(x)
    for _ in range(4):
        pk.penta_linear_i8_prequant(xq, s_x, rowsum, K, packed, s)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": "int8 prefill 4096x4096x4096", "warmup_launches": 3, "launches": 1}))


def run_ours(args):
    import torch
    import torch.distributed as dist

    import penta_kernel as pk
    import penta_dist as pd

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    # ---- weights: quantise + pack each full layer on the GPU, keep this rank's rows
    # (and, at N > 1, the whole packed layer for the parity check of the sharded outputs)
    gen = torch.Generator(device=dev).manual_seed(1234)
    packed = {}
    scales = {}
    full = {}
    for (K, N) in SHAPES:
        w = torch.randn(N, K, device=dev, generator=gen) * 0.02
        p, _, s = pk.quantize_and_pack(w)
        del w
        lo, hi = pd.shard_range(N, rank, world)
        base = p[lo:hi].contiguous()
        if world > 1:
            full[(K, N)] = p
        del p
        packed[(K, N)] = [base] + [base.clone() for _ in range(COPIES - 1)]
        scales[(K, N)] = s
    torch.cuda.synchronize()
    xs = {(M, K): torch.randn(M, K, device=dev, generator=gen).to(torch.bfloat16) for (M, K, _) in launches_per_step()}

    seq = launches_per_step()
    # N > 1: each product's GEMM stores its output columns into every GPU's
    # full-output buffer (peer memory), then a cross-GPU barrier kernel.  Four
    # buffer sets: the end-to-end graph gives each of its four steps its own.
    peers = pd.PeerGroup() if world > 1 else None
    outs_sets = [[peers.buffer((M, N), torch.bfloat16) for (M, K, N) in seq] for _ in range(4)] if peers else None
    col0 = {(K, N): pd.shard_range(N, rank, world)[0] for (K, N) in SHAPES}

    def product(l: int, c: int, barrier: bool = True, x=None, bufset: int = 0):
        M, K, N = seq[l]
        xin = xs[(M, K)] if x is None else x
        if peers is None:
            return pk.penta_linear(xin, packed[(K, N)][c], scales[(K, N)], K)
        out = outs_sets[bufset][l]
        pd.linear_peers(xin, packed[(K, N)][c], scales[(K, N)], K, col0[(K, N)], out[1], N)
        if barrier:
            peers.barrier()
        return out[0]

    def run_step(i: int):
        for l, (M, K, N) in enumerate(seq):
            product(l, ((6 * i + l) // 2) % COPIES)

    for i in range(3):
        run_step(i)
    torch.cuda.synchronize()

    # One CUDA graph per step phase removes host launch cost (at N > 1 the
    # graphs hold the GEMMs and the cross-GPU barrier kernels, no NCCL calls).
    graphs = []
    for ph in range(4):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run_step(ph)
        graphs.append(g)
    torch.cuda.synchronize()

    def step(i):
        graphs[i % 4].replay()

    sampler = ClockSampler([local] if world == 1 else list(range(torch.cuda.device_count()))[:world]) \
        if rank == 0 else None
    if sampler:
        sampler.start()
    for i in range(args.warmup):
        step(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    h0 = time.time()
    t0.record(stream)
    for i in range(args.steps):
        step(i)
    t1.record(stream)
    torch.cuda.synchronize()
    h1 = time.time()
    if sampler:
        sampler.window = (h0, h1)
    if world > 1:
        dist.barrier()
    ms = _max_over_ranks(t0.elapsed_time(t1), world, dev)
    ms_per_step = ms / args.steps
    value = step_bytes() * args.steps / (ms * 1e-3) / 1e9

    # ---- per-launch kernel durations (roofline): each (shape, M) alone, 20 launches, rotating copies
    per = []
    for l, (M, K, N) in enumerate(seq):
        n_loc = packed[(K, N)][0].shape[0]
        reps = 20
        # the local GEMM alone (its peer stores included, no barrier)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for r in range(reps):
                product(l, r % COPIES, barrier=False)
        g.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        dur = e0.elapsed_time(e1) / reps
        del g
        b = alg_bytes(M, K, n_loc)
        per.append({"M": M, "K": K, "N": N, "rows_local": n_loc, "us": round(dur * 1e3, 2),
                    "gbs": round(b / (dur * 1e-3) / 1e9, 1)})
    if sampler:
        sampler.stop()
    peaks = measured_peaks()
    tot_b = sum(alg_bytes(p["M"], p["K"], p["rows_local"]) for p in per)
    tot_t = sum(p["us"] for p in per) * 1e-6
    achieved = tot_b / tot_t / 1e9
    traffic, traffic_src = profile_traffic()

    # ---- parity of the timed path: every product as the step runs it, against
    # the unsharded product of the whole layer (N > 1: on every rank, the full
    # output assembled by the peer stores; sharding changes the k split of the
    # tiles, hence the fp32 summation order: within one bf16 ulp)
    parity = check_parity(pk, seq, product, xs, packed, full, scales, world, dev)

    # ---- end to end through the public API with host buffers (pinned).
    # Host -> device copies on one stream, the products on the compute stream
    # (penta_linear; at N > 1 penta_dist.linear_peers + the cross-GPU barrier),
    # device -> host copies on a third, joined per product by events, so the
    # copy engines and the SMs work on different products at once (as a
    # serving loop overlaps them); every step moves all its inputs and outputs.
    # At N > 1 the products write fixed peer buffers, so each step has its own
    # buffer set and the compute stream waits for the step's device -> host
    # copies before the next step's first barrier (no rank overwrites a buffer
    # that another rank is still copying out).
    xh = {k: v.cpu().pin_memory() for k, v in xs.items()}
    yh = {(M, K, N): torch.empty(M, N, dtype=torch.bfloat16).pin_memory() for (M, K, N) in seq}
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    xd_l = [torch.empty(M, K, dtype=torch.bfloat16, device=dev) for (M, K, N) in seq]
    ev_in = [torch.cuda.Event() for _ in seq]    # x of product l on the device
    ev_out = [torch.cuda.Event() for _ in seq]   # product l done (its x buffer free, its y ready)

    def e2e_step(i, first=False, capturing=False):
        cs = torch.cuda.current_stream()
        with torch.cuda.stream(h2d_s):
            for l, (M, K, N) in enumerate(seq):
                if not first:
                    h2d_s.wait_event(ev_out[l])  # the previous step's product l has read xd_l[l]
                xd_l[l].copy_(xh[(M, K)], non_blocking=True)
                ev_in[l].record(h2d_s)
        ys = []
        for l, (M, K, N) in enumerate(seq):
            cs.wait_event(ev_in[l])
            ys.append(product(l, ((6 * i + l) // 2) % COPIES, x=xd_l[l], bufset=i % 4))
            ev_out[l].record(cs)
        with torch.cuda.stream(d2h_s):
            for l, (M, K, N) in enumerate(seq):
                d2h_s.wait_event(ev_out[l])
                yh[(M, K, N)].copy_(ys[l], non_blocking=True)
                if peers is None and not capturing:
                    ys[l].record_stream(d2h_s)
        if peers is not None:
            cs.wait_stream(d2h_s)

    def check_host_outputs(i):
        bad = 0
        for l, (M, K, N) in enumerate(seq):
            c = ((6 * i + l) // 2) % COPIES
            if peers is None:
                want = pk.penta_linear(xd_l[l], packed[(K, N)][c], scales[(K, N)], K).cpu()
                bad += 0 if torch.equal(yh[(M, K, N)], want) else 1
            else:  # copies hold the same rows; the whole layer's product, one bf16 ulp
                want = pk.penta_linear(xd_l[l], full[(K, N)], scales[(K, N)], K).cpu()
                bad += 0 if within_bf16_ulp(yh[(M, K, N)], want) else 1
        return bad

    e2e_steps = max(1, min(args.steps, 200))
    for i in range(3):
        e2e_step(i, first=(i == 0))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    h2d_s.wait_stream(stream)
    d2h_s.wait_stream(stream)
    for i in range(e2e_steps):
        e2e_step(i)
    stream.wait_stream(h2d_s)
    stream.wait_stream(d2h_s)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), world, dev)
    bad = check_host_outputs(e2e_steps - 1)
    e2e_eager = step_bytes() * e2e_steps / (e2e_ms * 1e-3) / 1e9
    h2d = sum(2 * M * K for (M, K, N) in seq)
    d2h = sum(2 * M * N for (M, K, N) in seq)

    # The same calls and copies captured once into a CUDA graph (four steps,
    # so the weight-copy rotation is kept) and replayed: what a serving loop
    # that graphs its decode step gets, without the eager loop's host time.
    # Every replayed step still copies all inputs in and all outputs out.
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    g_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_e2e, stream=cap):
        h2d_s.wait_stream(cap)
        d2h_s.wait_stream(cap)
        for i in range(4):
            e2e_step(i, first=(i == 0), capturing=True)
        cap.wait_stream(h2d_s)
        cap.wait_stream(d2h_s)
    reps = max(1, e2e_steps // 4)
    for _ in range(2):
        g_e2e.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(stream)
    for _ in range(reps):
        g_e2e.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_graph = step_bytes() * 4 * reps / (_max_over_ranks(e0.elapsed_time(e1), world, dev) * 1e-3) / 1e9
    bad += check_host_outputs(3)
    del g_e2e
    if world > 1:
        t = torch.tensor([bad], device=dev)
        dist.all_reduce(t)
        bad = int(t.item())
    if bad:
        raise SystemExit(f"end-to-end host outputs differ from the product in {bad} cases")
    e2e_val = e2e_graph

    prefill = gpt = packsec = None
    if not args.no_prefill:
        prefill = prefill_int8(dev, gen, peaks, world, rank)
        gpt = pentagpt_forward(dev, world, rank)
        gpt["roofline"] = gpt_roofline(gpt, peaks, world)
        if world == 1:
            packsec = pack_secondary(dev, peaks)
    if prefill is not None and prefill.get("parity", "bit-exact") != "bit-exact":
        raise SystemExit("sharded int8 prefill output differs from the unsharded product")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_legs(max(1, args.steps), args.warmup)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "70B-class decode GEMV: K->N 8192->28672 and 28672->8192, M in {1,8,64}",
                       "weights": "N(0,0.02) absmean-quantised, 3-bit packed (94 MB per matrix)",
                       "activations": "bf16 N(0,1)",
                       "l2": f"inputs larger than L2: {COPIES} weight copies per shape rotated "
                             f"({COPIES * 2 * 94} MB); a buffer is reused after >= 7 other 94 MB launches",
                       "parallelism": "single GPU" if world == 1 else
                       f"output rows sharded x{world}; outputs stored into every GPU's buffer by the GEMM "
                       f"(NVLink peer stores) + cross-GPU barrier kernel",
                       "timing": "CUDA graphs of one step"},
            "parity": parity,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                         "traffic_source": traffic_src,
                         "peak_source": peaks["source"], "kernel": decode_kernel_label(),
                         "per_launch": per},
            "e2e": {"value": round(e2e_val, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps, "eager_value": round(e2e_eager, 1),
                    "graphed": True,
                    "path": ("penta_kernel.penta_linear" if world == 1 else
                             "penta_dist.linear_peers + PeerGroup.barrier (outputs in every GPU's buffer)")
                            + " on the compute stream, pinned host->device and device->host copies of every "
                              "product's x and y on two other streams, joined per product by events; value: "
                              "those calls captured in a CUDA graph of four steps and replayed, eager_value: "
                              "the eager loop; the host outputs of the last step of each are checked"},
            "cpu_baseline": cpu,
            # per product: the activation re-layout kernel and the dqmm kernel
            # (+ the cross-GPU barrier kernel when sharded)
            "gpu_launches": (2 if world == 1 else 3) * len(seq) * args.steps,
            "secondary": {"prefill_int8": prefill, "pentagpt_124m_fwd": gpt, "quantize_pack": packsec},
            "clocks": sampler.summary() if sampler else None,
        }
        print(json.dumps(line), flush=True)

    graphs.clear()
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        peers.close()
        dist.destroy_process_group()


def within_bf16_ulp(y, want) -> bool:
    """|y - want| <= one bf16 ulp of want (+1e-6) elementwise (both bf16 tensors)."""
    import torch
    a = y.float().double()
    b = want.float().double()
    ulp = torch.ldexp(torch.ones_like(b), (torch.frexp(b.abs().clamp(min=1e-30))[1] - 8))
    return bool(((a - b).abs() <= ulp + 1e-6).all())


def check_parity(pk, seq, product, xs, packed, full, scales, world, dev) -> str:
    """At N > 1: runs every product of the step once more as the timed path
    runs it (sharded GEMM, peer stores, barrier) and compares the full output
    on every rank with the unsharded product of the whole layer; exits non-zero
    on a mismatch."""
    import torch
    if world == 1:
        return "n/a at N = 1: the unsharded path (tests/test_linear_gpu.py checks it against the oracle)"
    bad = []
    for l, (M, K, N) in enumerate(seq):
        y = product(l, 0).clone()
        torch.cuda.synchronize()
        ok = within_bf16_ulp(y, pk.penta_linear(xs[(M, K)], full[(K, N)], scales[(K, N)], K))
        if not ok:
            bad.append(l)
    n_bad = len(bad)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([n_bad], device=dev)
        dist.all_reduce(t)
        n_bad = int(t.item())
    if n_bad:
        raise SystemExit(f"sharded output parity failed: {n_bad} (product, rank) cases, here {bad}")
    return (f"ok: on all {world} ranks the full output of each of the six products, assembled by the "
            f"peer stores, is within one bf16 ulp of the unsharded product")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-prefill", action="store_true", help="skip the int8 prefill secondary measurement")
    ap.add_argument("--profile", action="store_true", help="small fixed case for ncu captures")
    ap.add_argument("--profile-prefill", action="store_true", help="int8 prefill case for ncu captures")
    ap.add_argument("--profile-gemv", action="store_true", help="CUDA-core decode GEMV case for ncu captures")
    ap.add_argument("--profile-gpt", action="store_true", help="PentaGPT-124M forward for ncu launch lists")
    ap.add_argument("--profile-epilogue", action="store_true", help="plain vs fused-GELU product for ncu")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.profile_gpt:
        run_profile_gpt(args)
        return
    if args.profile_epilogue:
        run_profile_epilogue(args)
        return
    if args.profile_prefill:
        run_profile_prefill(args)
        return
    if args.profile_gemv:
        run_profile_gemv(args)
        return
    if args.profile:
        run_profile_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
