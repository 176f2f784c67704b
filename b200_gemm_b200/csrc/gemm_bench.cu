// C++ driver with the shape of the reference bench (matmul_b200.cu:44-166):
// fill A and B with N(0,1) bf16 on the host, verify each kernel against
// cuBLASLt, then time back-to-back launches with CUDA events and print TFLOPS.
//
//   gemm_bench [M N K] [reps]        (default 8192 8192 8192, 8 reps)
//
// Kernel 0 is cuBLASLt (the reference's comparator, matmul_b200.cu:13-26,
// rewritten with the operand order that is correct for non-square shapes);
// kernel 2 is this library through runKernel2, the drop-in for runKernel1.
// Differences from the reference bench: the tolerance is |err| <= 2^-7
// (|ref| + 1) instead of an absolute 0.1 (include/utils.cuh:31-41), failures
// set the exit code, and there is no 5 s sleep between kernels.
#include <cublasLt.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "b200gemm.hpp"

using bf16 = __nv_bfloat16;

#define CHECK_CUDA(x)                                                                   \
  do {                                                                                  \
    cudaError_t e_ = (x);                                                               \
    if (e_ != cudaSuccess) {                                                            \
      std::fprintf(stderr, "%s:%d %s\n", __FILE__, __LINE__, cudaGetErrorString(e_));   \
      return 2;                                                                         \
    }                                                                                   \
  } while (0)

namespace {

cublasLtHandle_t g_lt;
void* g_workspace = nullptr;
constexpr size_t kWorkspace = 32u << 20;

// C (M x N, row-major) = A (M x K, row-major) . B (N x K, row-major)^T.
// In cuBLASLt's column-major terms that is C^T (N x M) = B (N x K) . A^T,
// i.e. op(B) = B^T stored K x N with ld K, op(A) = A stored K x M with ld K.
int run_cublaslt(int M, int N, int K, const bf16* A, const bf16* B, bf16* C) {
  cublasLtMatmulDesc_t op;
  cublasLtMatrixLayout_t la, lb, lc;
  cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
  cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F);
  cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof(ta));
  cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof(tb));
  cublasLtMatrixLayoutCreate(&la, CUDA_R_16BF, K, N, K);  // B as K x N column-major
  cublasLtMatrixLayoutCreate(&lb, CUDA_R_16BF, K, M, K);  // A as K x M column-major
  cublasLtMatrixLayoutCreate(&lc, CUDA_R_16BF, N, M, N);  // C^T as N x M column-major
  cublasLtMatmulPreference_t pref;
  cublasLtMatmulPreferenceCreate(&pref);
  cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &kWorkspace,
                                       sizeof(kWorkspace));
  cublasLtMatmulHeuristicResult_t heur;
  int found = 0;
  cublasLtMatmulAlgoGetHeuristic(g_lt, op, la, lb, lc, lc, pref, 1, &heur, &found);
  float alpha = 1.f, beta = 0.f;
  int rc = 1;
  if (found > 0) {
    rc = cublasLtMatmul(g_lt, op, &alpha, B, la, A, lb, &beta, C, lc, C, lc, &heur.algo,
                        g_workspace, kWorkspace, 0) == CUBLAS_STATUS_SUCCESS
             ? 0
             : 1;
  }
  cublasLtMatmulPreferenceDestroy(pref);
  cublasLtMatrixLayoutDestroy(la);
  cublasLtMatrixLayoutDestroy(lb);
  cublasLtMatrixLayoutDestroy(lc);
  cublasLtMatmulDescDestroy(op);
  return rc;
}

int run_kernel(int kernel_num, int M, int N, int K, bf16* A, bf16* B, bf16* C) {
  switch (kernel_num) {
    case 0: return run_cublaslt(M, N, K, A, B, C);
    case 2: runKernel2(M, N, K, A, B, C, nullptr); return 0;
    default: return 1;
  }
}

}  // namespace

int main(int argc, char** argv) {
  long M = 8192, N = 8192, K = 8192;
  int reps = 8;
  if (argc >= 4) {
    M = std::atol(argv[1]);
    N = std::atol(argv[2]);
    K = std::atol(argv[3]);
  }
  if (argc >= 5) reps = std::atoi(argv[4]);
  cublasLtCreate(&g_lt);
  CHECK_CUDA(cudaMalloc(&g_workspace, kWorkspace));

  std::vector<bf16> hA(M * K), hB(N * K), hC(M * N), hR(M * N);
  std::default_random_engine gen(69);
  std::normal_distribution<float> dist(0.f, 1.f);
  for (auto& x : hA) x = __float2bfloat16_rn(dist(gen));
  for (auto& x : hB) x = __float2bfloat16_rn(dist(gen));
  bf16 *dA, *dB, *dC, *dR;
  CHECK_CUDA(cudaMalloc(&dA, sizeof(bf16) * M * K));
  CHECK_CUDA(cudaMalloc(&dB, sizeof(bf16) * N * K));
  CHECK_CUDA(cudaMalloc(&dC, sizeof(bf16) * M * N));
  CHECK_CUDA(cudaMalloc(&dR, sizeof(bf16) * M * N));
  CHECK_CUDA(cudaMemcpy(dA, hA.data(), sizeof(bf16) * M * K, cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMemcpy(dB, hB.data(), sizeof(bf16) * N * K, cudaMemcpyHostToDevice));

  cudaEvent_t start, stop;
  cudaEventCreate(&start);
  cudaEventCreate(&stop);
  int failures = 0;
  for (int kernel_num : {0, 2}) {
    std::printf("KERNEL %d\n", kernel_num);
    CHECK_CUDA(cudaMemset(dC, 0, sizeof(bf16) * M * N));
    CHECK_CUDA(cudaMemset(dR, 0, sizeof(bf16) * M * N));
    if (run_kernel(0, M, N, K, dA, dB, dR) != 0 || run_kernel(kernel_num, M, N, K, dA, dB, dC) != 0) {
      std::printf("launch failed\n");
      return 2;
    }
    CHECK_CUDA(cudaDeviceSynchronize());
    CHECK_CUDA(cudaMemcpy(hC.data(), dC, sizeof(bf16) * M * N, cudaMemcpyDeviceToHost));
    CHECK_CUDA(cudaMemcpy(hR.data(), dR, sizeof(bf16) * M * N, cudaMemcpyDeviceToHost));
    for (long i = 0; i < M * N; ++i) {
      const double r = __bfloat162float(hR[i]), c = __bfloat162float(hC[i]);
      if (!(std::fabs(r - c) <= std::ldexp(1.0, -7) * (std::fabs(r) + 1.0))) {
        std::printf("Divergence! Should %5.2f, Is %5.2f at %ld\n", r, c, i);
        ++failures;
        break;
      }
    }
    CHECK_CUDA(cudaEventRecord(start));
    for (int j = 0; j < reps; ++j) run_kernel(kernel_num, M, N, K, dA, dB, dC);
    CHECK_CUDA(cudaEventRecord(stop));
    CHECK_CUDA(cudaEventSynchronize(stop));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, start, stop);
    const double flops = 2.0 * M * N * K;
    std::printf("Average elapsed time: (%7.6f) s, performance: (%7.1f) TFLOPS. size: (%ld).\n\n",
                ms / 1e3 / reps, reps * flops * 1e-9 / ms, M);
  }
  cudaFree(dA);
  cudaFree(dB);
  cudaFree(dC);
  cudaFree(dR);
  cudaFree(g_workspace);
  cublasLtDestroy(g_lt);
  return failures == 0 ? 0 : 1;
}
