#!/usr/bin/env python
"""Benchmark of the bf16 GEMM hot path: C = A . B^T, bf16 in/out, fp32 accumulate.

One step = one GEMM over one batch of synthetic operands already resident in
HBM.  Default workload (N=1): M = N = K = 8192, U[-1, 1] operands, the
configuration the reference publishes its headline TFLOPS on.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                  [--impl ours|reference] [--allgather] [--no-cublas]
                  [--no-cpu-baseline] [--no-e2e]

Multi-GPU (launched by torchrun, one process per GPU): the GEMM is sharded
along N.  Every rank holds A, its rows of B and its columns of C; there is
no collective on the compute path.  For "square8192" each rank owns a fixed
8192-column shard (global N = 8192 * world: weak scaling); for "square16384"
and "mlp" the global N is fixed and split (strong scaling).  --allgather adds
a separately timed NCCL all-gather of the C shards.

Every run also carries a "strong16384" block (skip with --no-strong): the
16384^3 GEMM split along N over all ranks (strong scaling; at one GPU the
whole 16384^3), its separately timed NCCL all-gather of C and the GEMM with
the all-gather fused into its epilogue (checked bit for bit against a
single-GPU GEMM first), and its end-to-end rate from host memory, where each
rank uploads only its share of A's rows and gathers the rest over NVLink;
and a "strong_mlp" block: the MLP projection 16384 x 14336 x 4096 split the
same way (configs[3] of the benchmark at 8 GPUs).

--impl reference times the reference implementation of the path on the
host CPU cores: the reference project has no CPU GEMM of its own, so this
arm runs the C restatement of its arithmetic (oracle/, multithreaded fp32)
on a bounded row sample of the same workload.  When the reference's own
B200 kernel was built from its sources (oracle/_ref/libref_gemm.so) and a
GPU is present, the line also carries "reference_kernel": that kernel timed
on the same shape and operand distribution, exactly like `value`.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

WORKLOADS = {
    # name: global shape, operand distribution, how N>1 shards it
    "square8192": dict(M=8192, N=8192, K=8192, dist="uniform", scaling="weak"),
    "square16384": dict(M=16384, N=16384, K=16384, dist="normal", scaling="strong"),
    # one GPU's part of square16384 on 8 GPUs (N = 16384 / 8 columns)
    "shard16384x8": dict(M=16384, N=2048, K=16384, dist="normal", scaling="weak"),
    "mlp": dict(M=16384, N=14336, K=4096, dist="mlp", scaling="strong"),
    # one GPU's part of mlp on 8 GPUs (N = 14336 / 8 columns)
    "mlp_shard8": dict(M=16384, N=1792, K=4096, dist="mlp", scaling="weak"),
    # Decode shapes run as a decoder runs them: back to back, each step on the
    # next of `weights` weight matrices (B), whose total exceeds twice L2, with
    # the small-M kernels' launch overlap (B200GEMM_PDL_WEIGHTS_EARLY).
    "decode": dict(M=128, N=8192, K=8192, dist="normal", scaling="strong", bound="hbm", weights=8),
    # the MLP config's down projection (K = 14336 -> N = 4096) at 128 tokens
    "decode_down": dict(M=128, N=4096, K=14336, dist="normal", scaling="strong", bound="hbm", weights=8),
    "square512": dict(M=512, N=512, K=512, dist="normal", scaling="strong"),
}
METRIC = "bf16 GEMM TFLOPS @8192^3 (1 GPU) + N-GPU aggregate"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
SPEC_PEAKS = {"hbm_gbs": 8000.0, "bf16_tflops": 2250.0}  # public dense figures, for context


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--workload", default="square8192", choices=sorted(WORKLOADS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference", "cublaslt"],
                   help="ours: this library; reference: the reference arithmetic on the host CPU; "
                        "cublaslt: torch.matmul with the cuBLASLt backend on the same operands")
    p.add_argument("--tile-width", type=int, default=0, choices=[0, 512, 448, 256, 224, 192, 128],
                   help="force the output tile width (0 = the library's per-shape choice)")
    p.add_argument("--order", default="default", choices=["default", "hilbert", "bands"])
    p.add_argument("--band", type=int, default=16, help="tile-rows per band for --order bands")
    p.add_argument("--seed", type=int, default=1)
    p.add_argument("--allgather", action="store_true",
                   help="also time an NCCL all-gather of the C shards (separately)")
    p.add_argument("--fused-allgather", action="store_true",
                   help="also time the GEMM with the all-gather fused into its epilogue")
    p.add_argument("--epilogue", default=None, choices=["relu", "gelu", "gelu_tanh", "silu"],
                   help="also time GEMM + bias + this activation fused into the epilogue, against "
                        "cuBLASLt's fused bias+GELU/ReLU epilogue and the unfused torch sequence")
    p.add_argument("--no-cublas", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-strong", action="store_true", help="skip the strong16384 and strong_mlp blocks")
    p.add_argument("--no-numa-bind", action="store_true",
                   help="do not move each rank onto the CPUs of its GPU's NUMA node")
    p.add_argument("--cpu-seconds", type=float, default=10.0,
                   help="target CPU time of the cpu_baseline sample")
    return p.parse_args(argv)


# --------------------------------------------------------------------------- helpers
def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return d, "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(workload: str):
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary."""
    path = ROOT / "profiles" / "ncu_traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        fields = dict(kv.split("=", 1) for kv in line.split() if "=" in kv)
        if fields.get("workload") == workload and "dram_bytes_per_launch" in fields:
            return float(fields["dram_bytes_per_launch"])
    return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._period = period_s
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0}
        names = [n for n, bit in self.REASONS.items() if self.reasons & bit]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


def shard_shape(w, world: int, rank: int):
    """Per-rank (M, N_local, K, n0) for a workload under N-sharding."""
    from b200_gemm_b200.shard import column_shard

    M, N, K = w["M"], w["N"], w["K"]
    if w["scaling"] == "weak":
        return M, N, K, rank * N
    n0, n1 = column_shard(N, world, rank)
    return M, n1 - n0, K, n0


def time_steps(torch, step, steps, flush, stream, dev, barrier, per_step=None, between=True):
    """Device milliseconds for `steps` calls of `step` on `stream`.

    Operands far larger than L2: back-to-back steps, an event between every
    two (the total runs from the first event to the last), or with
    between=False only around the whole run (an event between two launches
    would keep the second from overlapping the first).  Otherwise a 256 MB
    buffer is overwritten before every step (outside the timed pair, per-step
    events) so no step starts with its operands in L2.  The per-step times go
    into `per_step` when a list is given."""
    if not flush:
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1 if between else 2)]
        barrier()
        evs[0].record(stream)
        for i in range(steps):
            step()
            if between:
                evs[i + 1].record(stream)
        if not between:
            evs[1].record(stream)
        barrier()
        if per_step is not None and between:
            per_step.extend(evs[i].elapsed_time(evs[i + 1]) for i in range(steps))
        return evs[0].elapsed_time(evs[-1])
    scratch = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(steps)]
    barrier()
    for e0, e1 in pairs:
        scratch.zero_()
        e0.record(stream)
        step()
        e1.record(stream)
    barrier()
    times = [e0.elapsed_time(e1) for e0, e1 in pairs]
    if per_step is not None:
        per_step.extend(times)
    del scratch
    return sum(times)


def time_epilogue(gemm, torch, A, B, C, args, flush, stream, dev, barrier, flops):
    """GEMM + bias + activation: ours fused (b200gemm_bf16_nt_epilogue), cuBLASLt's
    fused epilogue (torch._addmm_activation: bias + GELU(tanh) or ReLU), and the
    unfused torch sequence (matmul, then bias + activation kernels)."""
    import torch.nn.functional as F

    act = args.epilogue
    N = B.shape[0]
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 7)
    bias = (torch.randn(N, generator=g, device=dev) * 0.1).to(torch.bfloat16)
    out = torch.empty_like(C)
    steps = max(3, min(args.steps, 20))
    res = {"activation": act, "bias": True, "steps": steps}

    def tflops(ms):
        return flops / (ms / 1e3 / steps) / 1e12

    ours = lambda: gemm.bf16_nt_epilogue(A, B, bias=bias, activation=act, out=out)  # noqa: E731
    for _ in range(3):
        ours()
    barrier()
    res["ours_tflops"] = tflops(time_steps(torch, ours, steps, flush, stream, dev, barrier))
    torch.backends.cuda.preferred_blas_library("cublaslt")
    Bt = B.t()
    if act in ("relu", "gelu_tanh"):
        lt = lambda: torch._addmm_activation(bias, A, Bt, use_gelu=(act != "relu"))  # noqa: E731
        for _ in range(3):
            lt()
        barrier()
        res["cublaslt_fused_tflops"] = tflops(time_steps(torch, lt, steps, flush, stream, dev, barrier))
    fn = {"relu": F.relu, "gelu": F.gelu, "silu": F.silu,
          "gelu_tanh": lambda x: F.gelu(x, approximate="tanh")}[act]
    unfused = lambda: fn(torch.matmul(A, Bt) + bias)  # noqa: E731
    for _ in range(3):
        unfused()
    barrier()
    res["unfused_torch_tflops"] = tflops(time_steps(torch, unfused, steps, flush, stream, dev, barrier))
    res["how"] = ("TFLOPS of the GEMM flops (2MNK) per step, steps timed like `value`; cuBLASLt fused = "
                  "torch._addmm_activation (cuBLASLt bias+GELU(tanh)/ReLU epilogue), unfused = "
                  "torch.matmul then bias add and activation as separate kernels")
    return res


def launch_shape(gemm, M, N, K, info, library_arm):
    """Grid geometry of our kernel for this shape (what the library's plan says)."""
    if library_arm:
        return None
    plan = gemm.plan(M, N, K)
    if plan["kernel"] == "small_m":  # CTA pairs of 256 rows of B, clusters of 2 x split
        split = plan["small_m_split"]
        return dict(info, kernel="small_m", ctas=plan["tiles"] * 2 * split, threads_per_cta=192,
                    cluster=2 * split)
    if plan["kernel"] == "small_m_1cta":  # CTAs of 128 rows of B, clusters of split
        split = plan["small_m_split"]
        return dict(info, kernel="small_m_1cta", ctas=plan["tiles"] * split, threads_per_cta=192,
                    cluster=split)
    return dict(info, kernel="tiled", clusters=plan["clusters"], tiles=plan["tiles"],
                threads_per_cta=320 if plan["tile_width"] > 256 else 192, cluster=2)


def roofline(w, M, N, K, ms_per_launch, peaks, peak_kind, traffic):
    """Roofline entry for the dominant kernel.  Tensor-bound shapes report
    TFLOP/s against the measured bf16 GEMM peak; HBM-bound shapes (small M)
    report algorithmic GB/s against the measured copy bandwidth."""
    flops = 2.0 * M * N * K
    alg_bytes = 2.0 * (M * K + N * K + M * N)
    if w.get("bound") == "hbm":
        achieved = alg_bytes / (ms_per_launch / 1e3) / 1e9
        peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_kind": f"{peak_kind} hbm_gbs (copy)",
                "frac_of_spec": achieved / SPEC_PEAKS["hbm_gbs"],
                "traffic": traffic, "algorithmic_bytes": alg_bytes,
                "tflops": flops / (ms_per_launch / 1e3) / 1e12}
    achieved = flops / (ms_per_launch / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    sustained = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak, "peak_kind": f"{peak_kind} bf16_tflops (burst)",
            "frac_of_sustained": achieved / sustained, "frac_of_spec": achieved / SPEC_PEAKS["bf16_tflops"],
            "traffic": traffic, "algorithmic_bytes": alg_bytes}


# ------------------------------------------------------------------ reference arm
def cpu_rows_for(seconds: float, N: int, K: int, threads: int, probe_rate_flops: float) -> int:
    rows = int(seconds * probe_rate_flops / (2.0 * N * K))
    return max(2, rows)


def time_cpu_gemm(A_bits, B_bits, rows: int, threads: int = 0):
    from oracle import oracle

    t0 = time.perf_counter()
    _, used = oracle.gemm_f32_cpu(A_bits, B_bits, 0, rows, threads)
    dt = time.perf_counter() - t0
    return dt, used


def cpu_sample_operands(w, seed: int, rows: int):
    from b200_gemm_b200 import data

    # Only the first `rows` rows of A are needed; B is full size.
    A, B = data.host_operands(rows, w["N"], w["K"], w["dist"], seed=seed)
    return A, B


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(w, seed: int, target_s: float):
    """Multithreaded fp32 CPU GEMM on a row sample of the workload."""
    from oracle import oracle

    N, K = w["N"], w["K"]
    # Calibrate on enough rows to occupy every thread (a few rows measure
    # thread start-up, not the GEMM), then size the sample from that rate.
    probe_rows = min(w["M"], 8 * max(1, os.cpu_count() or 1))
    A, B = cpu_sample_operands(w, seed, max(probe_rows, 256))
    dt, used = time_cpu_gemm(A, B, probe_rows)
    rate = 2.0 * probe_rows * N * K / max(dt, 1e-9)
    rows = cpu_rows_for(target_s, N, K, used, rate)
    if rows * 2 >= w["M"]:
        rows = w["M"]  # within twice the target: run the whole workload, no extrapolation
    rows = min(rows, w["M"])
    if rows > A.shape[0]:
        A, B = cpu_sample_operands(w, seed, rows)
    dt, used = time_cpu_gemm(A, B, rows)
    tflops = 2.0 * rows * N * K / dt / 1e12
    full_s = 2.0 * w["M"] * N * K / (tflops * 1e12)
    sample = (f"the whole workload ({w['M']} x {N} x {K}) in {dt:.2f} s, fp32 accumulate" if rows == w["M"] else
              f"{rows} of {w['M']} rows of C (full N={N}, K={K}) in {dt:.2f} s, fp32 accumulate; "
              f"the whole workload at this rate (linear in M) would take {full_s:.1f} s")
    return {"value": tflops, "unit": "TFLOPS", "cores": used, "kind": "port",
            "sample": sample,
            "seconds": dt, "ncpus": oracle.num_cpus(), "cpu_model": cpu_model()}


def bench_config(args, w, world: int, rank: int = 0, library_arm: bool = False):
    """The `config` object of the JSON line, identical for both arms of a run
    (the reference arm computes it for the same --gpus N without a GPU)."""
    M, Nl, K, _ = shard_shape(w, world, rank)
    nw = w.get("weights", 1)
    operand_bytes = (M * K + nw * Nl * K) * 2
    flush = operand_bytes < 2 * L2_BYTES
    cfg = {"workload": args.workload, "M": M, "N_per_gpu": Nl, "K": K,
           "N_global": Nl * world if w["scaling"] == "weak" else w["N"],
           "dist": w["dist"], "seed": args.seed,
           "parallelism": f"N-sharded x{world}, A replicated, no collective",
           "l2": ("operands %.0f MB > 2x L2 (126 MB): back-to-back steps, no flush"
                  % (operand_bytes / 1e6)) if not flush else
                 ("operands %.0f MB < 2x L2: 256 MB L2 flush before each step, "
                  "per-step CUDA events" % (operand_bytes / 1e6))}
    if nw > 1:
        cfg["weights"] = (f"{nw} weight matrices B rotate, step i uses B[i mod {nw}]; CUDA events "
                          "only around the whole run")
        cfg["launch_overlap"] = None if library_arm else "B200GEMM_PDL_WEIGHTS_EARLY"
    return cfg, flush


def reference_kernel_leg(args, w, steps: int, warmup: int):
    """The reference's own B200 kernel, runKernel1 (b200_kernels/matmul_1.cuh:
    386-418), built from its sources into oracle/_ref/libref_gemm.so, on the
    workload's per-GPU shape and operand distribution, timed exactly like
    `value` (back-to-back launches, CUDA events, same L2 rule).  Its result
    is checked against cuBLASLt first.  None when the library or a GPU is
    missing, or the shape is outside what the reference supports (M, N
    multiples of 256, K a multiple of 64)."""
    lib_path = ROOT / "oracle" / "_ref" / "libref_gemm.so"
    M, N, K = w["M"], w["N"], w["K"]
    if w.get("weights", 1) > 1 or M % 256 or N % 256 or K % 64:
        return None
    if not lib_path.exists():
        return {"unavailable": "oracle/_ref/libref_gemm.so not built (needs the reference sources at build time)"}
    try:
        import torch
    except Exception:
        return None
    if not torch.cuda.is_available():
        return None
    import ctypes

    from b200_gemm_b200 import data

    lib = ctypes.CDLL(str(lib_path))
    lib.ref_run_kernel1.restype = ctypes.c_int
    lib.ref_run_kernel1.argtypes = [ctypes.c_int] * 3 + [ctypes.c_void_p] * 3
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    A, B = data.device_operands(M, N, K, w["dist"], seed=args.seed, device=dev)
    C = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    a, b, c = A.data_ptr(), B.data_ptr(), C.data_ptr()

    def step():
        rc = lib.ref_run_kernel1(M, N, K, a, b, c)
        if rc != 0:
            raise RuntimeError(f"reference kernel launch: CUDA error {rc}")

    step()
    torch.backends.cuda.preferred_blas_library("cublaslt")
    R = torch.matmul(A, B.t())
    torch.cuda.synchronize()
    ok = bool(((C.float() - R.float()).abs() <= 2.0 ** -7 * (R.float().abs() + 1.0)).all())
    del R
    for _ in range(max(3, warmup)):
        step()
    stream = torch.cuda.current_stream(dev)
    flush = (M * K + N * K) * 2 < 2 * L2_BYTES
    with ClockSampler(0) as clocks:
        ms = time_steps(torch, step, steps, flush, stream, dev, torch.cuda.synchronize)
    return {"value": 2.0 * M * N * K / (ms / 1e3 / steps) / 1e12, "unit": "TFLOPS",
            "ms_per_launch": ms / steps, "steps": steps, "shape": [M, N, K],
            "matches_cublaslt": ok, "clocks": clocks.summary(),
            "how": "reference runKernel1 built from its sources (oracle/_ref/libref_gemm.so), one GPU, "
                   "same operands and timing rule as `value` of the GPU arm"}


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0  # the CPU arm runs on rank 0 only
    from oracle import oracle

    N, K = w["N"], w["K"]
    A, B = cpu_sample_operands(w, args.seed, 4)
    dt, used = time_cpu_gemm(A, B, 4)
    rate = 2.0 * 4 * N * K / max(dt, 1e-9)
    total_budget = 150.0  # seconds for warmup + steps
    per_step = max(0.2, min(5.0, total_budget / max(1, args.steps + args.warmup)))
    rows = min(w["M"], cpu_rows_for(per_step, N, K, used, rate))
    A, B = cpu_sample_operands(w, args.seed, rows)
    for _ in range(args.warmup):
        time_cpu_gemm(A, B, rows)
    times = []
    for _ in range(args.steps):
        dt, used = time_cpu_gemm(A, B, rows)
        times.append(dt)
    total = sum(times)
    flops = 2.0 * rows * N * K * args.steps
    value = flops / total / 1e12
    config, _ = bench_config(args, w, max(1, args.gpus))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": w["scaling"] if world > 1 else "weak", "vs_baseline": None,
        "dtype": "f32 (bf16 inputs widened)", "data": "synthetic", "config": config,
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": used, "kind": "port",
                         "sample": f"{rows} of {w['M']} rows of C per step (full N, K), "
                                   "C restatement of the reference arithmetic, fp32 accumulate; "
                                   "the rate extrapolates linearly in M to the whole workload",
                         "rows_per_step": rows,
                         "ncpus": oracle.num_cpus(), "cpu_model": cpu_model()},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    rk = reference_kernel_leg(args, w, max(3, args.steps), args.warmup)
    if rk is not None:
        line["reference_kernel"] = rk
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------ GPU arm
def run_ours(args, w):
    import torch
    import torch.distributed as dist

    from b200_gemm_b200 import Gemm, _lib, data

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    distributed = world > 1
    from b200_gemm_b200 import shard

    # Pinned host buffers (e2e legs) go to the GPU's own NUMA node; the CPU
    # baseline gets the whole machine back before it runs.
    all_cpus = os.sched_getaffinity(0)
    numa_cpus = None if args.no_numa_bind else shard.bind_to_gpu_numa_node(local)
    if distributed:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    def barrier():
        if distributed:
            dist.barrier()
        torch.cuda.synchronize()

    M, Nl, K, n0 = shard_shape(w, world, rank)
    flops_rank = 2.0 * M * Nl * K
    # Operands: A replicated (same seed everywhere), B rows [n0, n0 + Nl).
    A, _ = data.device_operands(M, 8, K, w["dist"], seed=args.seed, device=dev)
    _, B = data.device_operands(8, Nl, K, w["dist"], seed=args.seed + 1 + n0, device=dev)
    # Decode workloads: step i multiplies by weight matrix i mod nw.
    nw = w.get("weights", 1)
    Bs = [B] + [data.device_operands(8, Nl, K, w["dist"], seed=args.seed + 1 + n0 + 7919 * j, device=dev)[1]
                for j in range(1, nw)]
    C = torch.empty(M, Nl, dtype=torch.bfloat16, device=dev)
    gemm = Gemm(local)
    if nw > 1:
        gemm.set_pdl(_lib.PDL_WEIGHTS_EARLY)  # B is never written by the kernel before
    if args.tile_width:
        gemm.set_tile_width(args.tile_width)
    if args.order != "default":
        gemm.set_schedule(_lib.ORDER_HILBERT if args.order == "hilbert" else _lib.ORDER_BANDS, args.band)
    stream = torch.cuda.current_stream(dev)
    sptr = int(stream.cuda_stream)
    a_ptr, c_ptr = A.data_ptr(), C.data_ptr()
    b_ptrs = [b.data_ptr() for b in Bs]
    turn = [0]

    def step():
        rc = gemm.bf16_nt_ptr(M, Nl, K, a_ptr, b_ptrs[turn[0] % nw], c_ptr, Nl, sptr)
        turn[0] += 1
        if rc != _lib.OK:
            raise RuntimeError(_lib.strerror(rc))

    library_arm = args.impl == "cublaslt"
    if library_arm:
        # Comparison arm: the same operands through cuBLASLt (no kernel of ours runs).
        torch.backends.cuda.preferred_blas_library("cublaslt")
        Bts = [b.t() for b in Bs]

        def step():  # noqa: F811
            torch.matmul(A, Bts[turn[0] % nw], out=C)
            turn[0] += 1

    for _ in range(max(3, args.warmup)):
        step()
    barrier()
    st, detail = gemm.last_device_status()
    if st != _lib.OK:
        raise RuntimeError(f"device status {st} {detail}")

    operand_bytes = (M * K + nw * Nl * K) * 2
    flush = operand_bytes < 2 * L2_BYTES
    between = nw == 1
    with ClockSampler(local) as clocks:
        step_ms = []
        ms = time_steps(torch, step, args.steps, flush, stream, dev, barrier, step_ms, between)
    st, detail = gemm.last_device_status()
    if st != _lib.OK:
        raise RuntimeError(f"device status {st} {detail}")
    ms_max = ms
    if distributed:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    per_step_s = ms_max / 1e3 / args.steps
    total_flops = flops_rank * world  # every rank does the same amount of work
    value = total_flops / per_step_s / 1e12
    kernel_tflops = flops_rank / (ms / 1e3 / args.steps) / 1e12

    extra = {}
    # ------------------------------------------------ cuBLASLt on the same box
    if not args.no_cublas and not library_arm:
        torch.backends.cuda.preferred_blas_library("cublaslt")
        Cr = torch.empty_like(C)
        Bts = [b.t() for b in Bs]
        cturn = [0]

        def cub_step():
            torch.matmul(A, Bts[cturn[0] % nw], out=Cr)
            cturn[0] += 1

        for _ in range(max(3, args.warmup)):
            cub_step()
        barrier()
        cms = time_steps(torch, cub_step, args.steps, flush, stream, dev, barrier, None, between)
        extra["cublaslt"] = {"value": flops_rank / (cms / 1e3 / args.steps) / 1e12, "unit": "TFLOPS",
                             "per_gpu": True, "how": "torch.matmul, preferred_blas_library=cublaslt; "
                                                     "timed exactly like `value` (same L2 rule)"}
        del Cr

    # ------------------------------- GEMM + bias + activation in the epilogue
    if args.epilogue and not library_arm:
        one_b_flush = (M * K + Nl * K) * 2 < 2 * L2_BYTES  # this leg uses one B
        extra["epilogue"] = time_epilogue(gemm, torch, A, B, C, args, one_b_flush, stream, dev, barrier,
                                          flops_rank)

    # ---------------------------------------- optional all-gather of C shards
    if args.allgather and distributed:
        gathered = torch.empty(world * M * Nl, dtype=torch.bfloat16, device=dev)
        flat = C.view(-1)
        for _ in range(3):
            dist.all_gather_into_tensor(gathered, flat)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        reps = max(3, min(args.steps, 20))
        for _ in range(reps):
            dist.all_gather_into_tensor(gathered, flat)
        e1.record(stream)
        barrier()
        ag_ms = e0.elapsed_time(e1) / reps
        t = torch.tensor([ag_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ag_ms = float(t.item())
        nbytes = gathered.numel() * 2
        extra["allgather"] = {"ms": ag_ms, "bytes_per_rank_out": nbytes,
                              "algbw_gbs": nbytes / (ag_ms / 1e3) / 1e9,
                              "layout": "shard-major [world][M][N/world]", "timed_separately": True}
        del gathered

    # ------------------------------- GEMM with the all-gather in its epilogue
    if args.fused_allgather and distributed:
        from b200_gemm_b200 import shard

        fused = shard.FusedAllGather(gemm, M, Nl * world if w["scaling"] == "weak" else w["N"])
        if fused.n1 - fused.n0 == Nl:
            B_loc = B  # this rank's rows of B are exactly its column block
            fstep = lambda: fused.run(A, B_loc, sptr)  # noqa: E731
            for _ in range(3):
                fstep()
            barrier()
            fms = time_steps(torch, fstep, max(3, min(args.steps, 20)), False, stream, dev, barrier)
            t = torch.tensor([fms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            reps = max(3, min(args.steps, 20))
            fms = float(t.item()) / reps
            extra["fused_allgather"] = {
                "ms": fms, "tflops_aggregate": total_flops / (fms / 1e3) / 1e12,
                "gemm_only_ms": ms_max / args.steps,
                "bytes_to_peers_per_rank": 2 * M * Nl * (world - 1),
                "how": "b200gemm_bf16_nt_allgather: epilogue stores each C chunk to all peers' "
                       "full C over NVLink (IPC-mapped), timed with CUDA events, max over ranks"}
        fused.close()

    # ----------------------------------------------------- end to end (host)
    if not args.no_e2e and not library_arm:
        e2e = run_e2e(gemm, torch, dev, stream, M, Nl, K, A, B, args, barrier, distributed, world)
        extra["e2e"] = e2e

    del A, B, C, Bs
    # ------------------------------------ 16384^3 split over all ranks (strong)
    if not args.no_strong and not library_arm:
        torch.cuda.empty_cache()
        extra["strong16384"] = run_strong16384(gemm, torch, dev, stream, args, barrier, distributed,
                                               world, rank)
        torch.cuda.empty_cache()
        extra["strong_mlp"] = run_strong_mlp(gemm, torch, dev, stream, args, barrier, distributed, world, rank)
    info = gemm.device_info()
    result = None
    if rank == 0:
        peaks, peak_kind = load_peaks()
        traffic = None if library_arm else load_traffic(args.workload)
        result = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": w["scaling"] if world > 1 else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": bench_config(args, w, world, rank, library_arm)[0],
            "gpu_launches": 0 if library_arm else args.steps,
            "launch": launch_shape(gemm, M, Nl, K, info, library_arm),
            "roofline": roofline(w, M, Nl, K, ms / args.steps, peaks, peak_kind, traffic),
            "per_launch_ms": ({"mean": ms / args.steps, "median": statistics.median(step_ms),
                               "best": min(step_ms), "worst": max(step_ms),
                               "how": "CUDA events between consecutive launches (rank 0)"} if step_ms else
                              {"mean": ms / args.steps, "how": "events around the whole run only"}),
            "clocks": clocks.summary(),
        }
        result.update(extra)
        if library_arm:
            result["impl"] = "cublaslt"
            result["tile_width"] = None
        else:
            plan = gemm.plan(M, Nl, K)
            result["kernel"] = plan["kernel"]
            result["tile_width"] = plan["tile_width"] if plan["kernel"] == "tiled" else None
            if plan["kernel"].startswith("small_m"):
                result["small_m_split"] = plan["small_m_split"]
        if numa_cpus is not None:
            result["host_cpus"] = {"bound_to_gpu_numa_node": True, "cpus": len(numa_cpus)}
        if not args.no_cpu_baseline and not library_arm:
            os.sched_setaffinity(0, all_cpus)
            result["cpu_baseline"] = cpu_baseline(w, args.seed, args.cpu_seconds)
    gemm.close()
    if distributed:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


def time_e2e(torch, dev, stream, step, steps, barrier, distributed):
    """Device ms for `steps` calls of step(i, stream_i), the calls alternating
    between `stream` and a second stream, as independent requests would
    arrive (calls on one stream run one after the other); CUDA events on
    `stream`, which waits for the other stream before the end event; max
    over ranks."""
    streams = [stream, torch.cuda.Stream(device=dev)]
    for i in range(3):
        step(i, streams[i % 2])
    streams[0].wait_stream(streams[1])
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    streams[1].wait_event(e0)
    for i in range(steps):
        step(i, streams[i % 2])
    streams[0].wait_stream(streams[1])
    e1.record(stream)
    barrier()
    ms = e0.elapsed_time(e1)
    if distributed:
        import torch.distributed as dist

        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def host_e2e(gemm, torch, dev, stream, M, Nl, K, A, B, steps, barrier, distributed, world):
    """One rank's end-to-end GEMM from pinned host memory, through the
    library's public host-buffer paths:
      * one GPU: b200gemm_bf16_nt_host (C-ABI) with host A, B and C, which
        copies them in and out by row chunks overlapped with the GEMMs;
      * N GPUs: shard.ShardedHostGemm, where each rank holds and uploads only
        its 1/N of A's rows plus its own B rows, gathers the rest of A from
        the other ranks over NVLink (one NCCL all-gather), runs the GEMM
        through the C-ABI and copies its C columns out.
    Returns (ms for `steps` calls, max over ranks; h2d bytes; d2h bytes) per
    rank and call."""
    from b200_gemm_b200 import _lib, shard

    hB = torch.empty(Nl, K, dtype=torch.bfloat16, pin_memory=True)
    hC = torch.empty(M, Nl, dtype=torch.bfloat16, pin_memory=True)
    hB.copy_(B)
    if world == 1:
        hA = torch.empty(M, K, dtype=torch.bfloat16, pin_memory=True)
        hA.copy_(A)

        def step(i, s):
            gemm.bf16_nt_host(hA, hB, out=hC, stream=s)

        up, down = 2 * (M * K + Nl * K), 2 * M * Nl
    else:
        def gemm_fn(A_full, Bd, Cd, s):
            return gemm.bf16_nt_ptr(M, Nl, K, A_full.data_ptr(), Bd.data_ptr(), Cd.data_ptr(), Nl,
                                    int(s.cuda_stream))

        hg = shard.ShardedHostGemm(M, Nl, K, gemm_fn, dev)
        hA_rows = torch.empty(hg.r1 - hg.r0, K, dtype=torch.bfloat16, pin_memory=True)
        hA_rows.copy_(A[hg.r0:hg.r1])

        def step(i, s):
            hg.run(hA_rows, hB, hC, s)

        up, down = hg.bytes_per_call()
    ms = time_e2e(torch, dev, stream, step, steps, barrier, distributed)
    st, detail = gemm.last_device_status()
    if st != _lib.OK:
        raise RuntimeError(f"device status {st} {detail}")
    return ms, up, down


def run_e2e(gemm, torch, dev, stream, M, Nl, K, A, B, args, barrier, distributed, world):
    """Same metric through the public host-buffer entry points (host_e2e)."""
    steps = max(3, min(args.steps, 20))
    ms, up, down = host_e2e(gemm, torch, dev, stream, M, Nl, K, A, B, steps, barrier, distributed, world)
    value = 2.0 * M * Nl * K * world / (ms / 1e3 / steps) / 1e12
    how = ("pinned host A,B,C through b200gemm_bf16_nt_host (row-chunked; H2D, GEMM and D2H overlapped on "
           "three streams)" if world == 1 else
           "shard.ShardedHostGemm: each rank uploads its 1/N of A's rows and its B rows from pinned host "
           "memory, one NCCL all-gather assembles A over NVLink, GEMM through the C-ABI, C columns copied "
           "back to pinned host memory")
    return {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": up * world,
            "d2h_bytes_per_step": down * world, "per_rank_h2d_bytes": up, "per_rank_d2h_bytes": down,
            "steps": steps,
            "how": how + "; steps alternate between two caller streams; CUDA events on the first, which "
                         "waits for the second before the end event; max over ranks"}


def strong_gemm(gemm, torch, dev, stream, args, barrier, distributed, world, rank, M, N, K, dist_name,
                seed):
    """C = A . B^T split along N over all ranks (strong scaling; at one GPU
    the whole GEMM): B and C column-sharded, A replicated, no collective.
    Returns (result dict, A, B_local, B_full, C_local, ms for the steps, steps)."""
    import torch.distributed as dist

    from b200_gemm_b200 import _lib, data, shard

    n0, n1 = shard.column_shard(N, world, rank)
    Nl = n1 - n0
    flops = 2.0 * M * N * K
    A, B_full = data.device_operands(M, N, K, dist_name, seed=seed, device=dev)
    B = B_full[n0:n1].contiguous() if Nl != N else B_full
    C = torch.empty(M, Nl, dtype=torch.bfloat16, device=dev)
    sptr = int(stream.cuda_stream)
    a, b, c = A.data_ptr(), B.data_ptr(), C.data_ptr()

    def step():
        rc = gemm.bf16_nt_ptr(M, Nl, K, a, b, c, Nl, sptr)
        if rc != _lib.OK:
            raise RuntimeError(_lib.strerror(rc))

    steps = max(5, min(args.steps, 20))
    for _ in range(3):
        step()
    barrier()
    ms = time_steps(torch, step, steps, False, stream, dev, barrier)
    if distributed:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    st, detail = gemm.last_device_status()
    if st != _lib.OK:
        raise RuntimeError(f"device status {st} {detail}")
    plan = gemm.plan(M, Nl, K)
    res = {"M": M, "N": N, "K": K, "N_per_gpu": Nl, "n_gpus": world, "dist": dist_name,
           "scaling": "strong", "steps": steps, "ms_per_step": ms / steps,
           "value": flops / (ms / 1e3 / steps) / 1e12, "unit": "TFLOPS",
           "tile_width": plan["tile_width"], "tail_split": plan["tail_split"],
           "how": "B and C column-sharded (shard.column_shard), A replicated, no collective; back-to-back "
                  "launches, CUDA events, max over ranks; value = 2MNK / per-step time"}
    return res, A, B, B_full, C, ms, steps


def run_strong_mlp(gemm, torch, dev, stream, args, barrier, distributed, world, rank):
    """the MLP projection 16384 x 14336 x 4096 (A ~ N(0,1)
    activations, B ~ N(0,0.02) weights) split along N over all ranks."""
    res, A, B, B_full, C, _, _ = strong_gemm(gemm, torch, dev, stream, args, barrier, distributed, world,
                                             rank, 16384, 14336, 4096, "mlp", args.seed + 200)
    del A, B, B_full, C
    return res


def run_strong16384(gemm, torch, dev, stream, args, barrier, distributed, world, rank):
    """The north-star scaling configuration: C = A . B^T at M = N = K = 16384
    (N(0,1) operands), B and C column-sharded over all ranks, A replicated
    (at one GPU the whole GEMM).  Times the GEMM (max over ranks, aggregate
    TFLOPS), the NCCL all-gather of the C shards separately, the GEMM with
    the all-gather fused into its epilogue (P2P stores and NVLink multicast;
    each first checked bit for bit on every rank against a one-GPU 16384^3
    GEMM), and the end-to-end rate from pinned host memory (host_e2e)."""
    import torch.distributed as dist

    from b200_gemm_b200 import _lib, shard

    M = N = K = 16384
    flops = 2.0 * M * N * K
    res, A, B, B_full, C, ms, steps = strong_gemm(gemm, torch, dev, stream, args, barrier, distributed,
                                                  world, rank, M, N, K, "normal", args.seed + 100)
    Nl = res["N_per_gpu"]
    sptr = int(stream.cuda_stream)

    def max_ms(v):
        if not distributed:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    reps = max(3, min(args.steps, 20))
    if distributed:
        gathered = torch.empty(world * M * Nl, dtype=torch.bfloat16, device=dev)
        flat = C.view(-1)
        for _ in range(3):
            dist.all_gather_into_tensor(gathered, flat)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            dist.all_gather_into_tensor(gathered, flat)
        e1.record(stream)
        barrier()
        ag_ms = max_ms(e0.elapsed_time(e1) / reps)
        nbytes = gathered.numel() * 2
        res["allgather"] = {"ms": ag_ms, "bytes_out_per_rank": nbytes,
                            "busbw_gbs": nbytes * (world - 1) / world / (ag_ms / 1e3) / 1e9,
                            "gemm_plus_allgather_ms": ms / steps + ag_ms,
                            "how": "NCCL all_gather_into_tensor of the C shards (shard-major), timed "
                                   "separately from the GEMM, CUDA events, max over ranks"}
        del gathered
        full = gemm.bf16_nt(A, B_full)  # the one-GPU 16384^3 result every rank's gathered C must equal
        torch.cuda.synchronize()

        def fused_leg(fused, how):
            fused.C.fill_(float("nan"))
            barrier()
            rc = fused.run(A, B, sptr)
            barrier()
            same = torch.tensor([1 if rc == _lib.OK and torch.equal(
                fused.view().view(torch.int16), full.view(torch.int16)) else 0], device=dev)
            dist.all_reduce(same, op=dist.ReduceOp.MIN)
            fstep = lambda: fused.run(A, B, sptr)  # noqa: E731
            for _ in range(3):
                fstep()
            barrier()
            fms = max_ms(time_steps(torch, fstep, reps, False, stream, dev, barrier)) / reps
            return {"ms": fms, "bit_exact": bool(same.item()), "tflops_aggregate": flops / (fms / 1e3) / 1e12,
                    "vs_gemm_plus_allgather": (ms / steps + ag_ms) / fms, "how": how}

        fused = shard.FusedAllGather(gemm, M, N)
        try:
            res["fused_allgather"] = fused_leg(
                fused, "b200gemm_bf16_nt_allgather: the epilogue writes each C chunk into every rank's "
                       "full-width C over NVLink (IPC-mapped peer stores); bit_exact: every rank's gathered "
                       "C equals its own one-GPU 16384^3 GEMM, bit for bit")
        finally:
            barrier()
            fused.close()
            del fused
        try:
            mc = shard.MulticastAllGather(gemm, M, N)
        except RuntimeError as e:
            res["fused_allgather_multicast"] = {"unavailable": str(e)}
            mc = None
        if mc is not None:
            try:
                res["fused_allgather_multicast"] = fused_leg(
                    mc, "b200gemm_bf16_nt_allgather_multicast: the epilogue writes each C chunk once with "
                        "multimem.st to an NVLink multicast mapping of every rank's C (torch symmetric "
                        "memory), NVSwitch replicates it; bit_exact as for fused_allgather")
            finally:
                barrier()
                mc.close()
                del mc
        del full
    st, detail = gemm.last_device_status()
    if st != _lib.OK:
        raise RuntimeError(f"device status {st} {detail}")
    if not args.no_e2e:
        e_steps = max(3, min(args.steps, 10))
        del C
        ems, up, down = host_e2e(gemm, torch, dev, stream, M, Nl, K, A, B, e_steps, barrier, distributed,
                                 world)
        res["e2e"] = {"value": flops / (ems / 1e3 / e_steps) / 1e12, "unit": "TFLOPS", "steps": e_steps,
                      "h2d_bytes_per_step": up * world, "d2h_bytes_per_step": down * world,
                      "per_rank_h2d_bytes": up, "per_rank_d2h_bytes": down,
                      "how": "host_e2e: one GPU b200gemm_bf16_nt_host; N GPUs shard.ShardedHostGemm (each "
                             "rank uploads 1/N of A's rows and its B rows, NCCL all-gather of A over "
                             "NVLink, GEMM, C columns back to host); max over ranks"}
    return res


def main(argv=None):
    args = parse_args(argv)
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference(args, w)
    return run_ours(args, w)


if __name__ == "__main__":
    sys.exit(main())
