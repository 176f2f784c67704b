// TEST INFRASTRUCTURE ONLY.  Exposes the reference project's own B200
// launcher, runKernel1 (b200_kernels/matmul_1.cuh:386-418), compiled from its
// sources, through a C symbol so tests/golden/make_golden.py can record its
// outputs as golden fixtures.  Nothing of the reference is copied here; the
// header is included from the reference tree at build time (oracle/Makefile).
#include "b200_kernels/matmul_1.cuh"

extern "C" int ref_run_kernel1(int M, int N, int K, void* A, void* B, void* C) {
  runKernel1(M, N, K, static_cast<bf16*>(A), static_cast<bf16*>(B), static_cast<bf16*>(C), nullptr);
  return static_cast<int>(cudaGetLastError());
}
