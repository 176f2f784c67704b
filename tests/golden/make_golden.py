"""Generate golden fixtures from the reference project's own kernel.

Runs on a B200 host with oracle/_ref/libref_gemm.so (the reference launcher
runKernel1 from b200_kernels/matmul_1.cuh, built from its sources by
`make -C oracle ref`).  For every case the operands are regenerated from
(shape, distribution, seed) with b200_gemm_b200.data.host_operands, the
reference kernel computes C, and the bf16 output bits are saved as
<outdir>/<case>.npz.  The reference caches its tensor maps keyed on M only
(matmul_1.cuh:390), so each case runs in a fresh process.

    python tests/golden/make_golden.py <outdir>
    python tests/golden/make_golden.py time 8192     # reference kernel TFLOPS

The reference only supports M, N multiples of 256 and K multiples of 64,
so the cases respect that.
"""
from __future__ import annotations

import ctypes
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

CASES = {
    "ref_512x512x512_normal_s0": (512, 512, 512, "normal", 0),
    "ref_256x512x128_uniform_s1": (256, 512, 128, "uniform", 1),
    "ref_768x256x320_mlp_s2": (768, 256, 320, "mlp", 2),
}


def run_case(name: str, outdir: Path) -> None:
    import torch

    from b200_gemm_b200 import data

    M, N, K, dist, seed = CASES[name]
    A_bits, B_bits = data.host_operands(M, N, K, dist, seed)
    lib = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libref_gemm.so"))
    lib.ref_run_kernel1.restype = ctypes.c_int
    lib.ref_run_kernel1.argtypes = [ctypes.c_int] * 3 + [ctypes.c_void_p] * 3
    dev = lambda b: torch.from_numpy(b.view(np.int16)).cuda()
    A, B = dev(A_bits), dev(B_bits)
    C = torch.zeros(M, N, dtype=torch.int16, device="cuda")
    rc = lib.ref_run_kernel1(M, N, K, A.data_ptr(), B.data_ptr(), C.data_ptr())
    torch.cuda.synchronize()
    if rc != 0:
        raise SystemExit(f"{name}: reference launch returned CUDA error {rc}")
    out = C.cpu().numpy().view(np.uint16)
    np.savez_compressed(outdir / f"{name}.npz", C=out, M=M, N=N, K=K, dist=dist, seed=seed,
                        source="reference runKernel1 (b200_kernels/matmul_1.cuh) on B200")
    print(f"{name}: ok")


def time_reference(size: int, reps: int = 20) -> None:
    """Throughput of the reference kernel itself at size^3 (U[-1,1] operands),
    back-to-back launches timed with CUDA events, as its bench does
    (matmul_b200.cu:139-153).  Printed as one JSON line."""
    import json

    import torch

    from b200_gemm_b200 import data

    lib = ctypes.CDLL(str(ROOT / "oracle" / "_ref" / "libref_gemm.so"))
    lib.ref_run_kernel1.restype = ctypes.c_int
    lib.ref_run_kernel1.argtypes = [ctypes.c_int] * 3 + [ctypes.c_void_p] * 3
    A, B = data.device_operands(size, size, size, "uniform", seed=1)
    C = torch.empty(size, size, dtype=torch.bfloat16, device="cuda")
    run = lambda: lib.ref_run_kernel1(size, size, size, A.data_ptr(), B.data_ptr(), C.data_ptr())
    for _ in range(3):
        if run() != 0:
            raise SystemExit("reference launch failed")
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    ref = torch.matmul(A, B.t())
    ok = bool(((C.float() - ref.float()).abs() <= 2.0 ** -7 * (ref.float().abs() + 1.0)).all())
    print(json.dumps({"kernel": "reference runKernel1", "size": size, "ms": ms,
                      "tflops": 2.0 * size ** 3 / ms / 1e9, "matches_cublaslt": ok}))


def main() -> int:
    if len(sys.argv) > 1 and sys.argv[1] == "time":
        time_reference(int(sys.argv[2]) if len(sys.argv) > 2 else 8192)
        return 0
    outdir = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent
    outdir.mkdir(parents=True, exist_ok=True)
    if len(sys.argv) > 2:
        run_case(sys.argv[2], outdir)
        return 0
    for name in CASES:
        subprocess.run([sys.executable, __file__, str(outdir), name], check=True, timeout=300)
    return 0


if __name__ == "__main__":
    sys.exit(main())
