"""The C++ drop-in, run from C++.

1. b200_gemm_b200/lib/gemm_bench: the reference bench loop rebuilt on this
   library (fill, verify kernel 0 = cuBLASLt and kernel 2 = runKernel2 with a
   relative tolerance, time back-to-back launches), at 512^3, 8192^3 and a
   ragged shape.  It exits non-zero on a divergence or a failed launch.
2. oracle/_ref/matmul_b200_dropin: the reference's own bench
   (matmul_b200.cu:28-38, 44-166) with the edits INTEGRATION.md prints
   applied (include b200gemm.hpp, `case 2: runKernel2(...)`, kernel list
   {0, 1, 2}), built against libb200gemm.so by `make -C oracle dropin`.  It
   runs cuBLAS, the reference kernel runKernel1 and this library's kernel in
   one process on its 8192^3 N(0,1) operands.  Its check is an absolute 0.1
   on the bf16 difference to cuBLAS (include/utils.cuh:31-41), which one
   bf16 rounding step already exceeds at |C| >= 32; so the test requires
   kernel 2's first reported divergence, if any, to be within
   2^-7 (|ref| + 1), the tolerance of the other tests.
"""
import re
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
BENCH = ROOT / "b200_gemm_b200" / "lib" / "gemm_bench"
DROPIN = ROOT / "oracle" / "_ref" / "matmul_b200_dropin"
PERF = re.compile(r"Average elapsed time: \(\s*([0-9.]+)\) s, performance: \(\s*([0-9.]+)\) TFLOPS")
DIVERGE = re.compile(r"Divergence! Should\s*(-?[0-9.]+), Is\s*(-?[0-9.]+)")


def _sections(out: str):
    """{kernel number: text of its section} of the bench output."""
    parts = re.split(r"^KERNEL (\d+)\s*$", out, flags=re.M)
    return {int(parts[i]): parts[i + 1] for i in range(1, len(parts) - 1, 2)}


@pytest.mark.parametrize("args", [["512", "512", "512", "20"], ["8192", "8192", "8192", "8"],
                                  ["1000", "1528", "520", "20"]], ids=["512", "8192", "ragged"])
def test_gemm_bench_cpp(args):
    from b200_gemm_b200 import build

    build.build_bench()
    r = subprocess.run([str(BENCH), *args], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.returncode, r.stdout[-2000:], r.stderr[-2000:])
    sec = _sections(r.stdout)
    assert sorted(sec) == [0, 2], r.stdout
    for k in (0, 2):
        assert "Divergence" not in sec[k], sec[k]
        m = PERF.search(sec[k])
        assert m and float(m.group(2)) > 0, sec[k]


def test_reference_bench_with_runkernel2():
    if not DROPIN.exists():
        pytest.skip("oracle/_ref/matmul_b200_dropin not built: it needs the reference sources at build "
                    "time (B200GEMM_REFERENCE_DIR, make -C oracle dropin)")
    r = subprocess.run([str(DROPIN)], capture_output=True, text=True, timeout=900, cwd=DROPIN.parent)
    assert r.returncode == 0, (r.returncode, r.stdout[-2000:], r.stderr[-2000:])
    sec = _sections(r.stdout)
    assert sorted(sec) == [0, 1, 2], r.stdout
    tflops = {}
    for k in (0, 1, 2):
        m = PERF.search(sec[k])
        assert m, sec[k]
        tflops[k] = float(m.group(2))
        assert tflops[k] > 0
    assert "[b200gemm]" not in r.stderr, r.stderr  # runKernel2 reported no error status
    d = DIVERGE.search(sec[2])
    if d:
        should, got = float(d.group(1)), float(d.group(2))
        # the printout keeps two decimals: allow their rounding on top of the tolerance
        assert abs(should - got) <= 2.0 ** -7 * (abs(should) + 1.0) + 0.01, sec[2]
    print(f"reference bench, 8192^3: cuBLAS {tflops[0]:.1f}, runKernel1 {tflops[1]:.1f}, "
          f"runKernel2 {tflops[2]:.1f} TFLOPS")
