// Library comparison rows for gemm_bench (measured beside our kernels, never on our path).
// Same semantics as the reference's rows (src/reference.cu:4-11, src/cublas_tc.cu:15-47,
// src/cublaslt_fp8.cu:32-94): inputs staged once per pointer outside the timed loop, the
// handle and descriptors created once, row-major C computed as column-major C^T.
//   cublas            cublasSgemm, FP32 (correctness reference of the driver)
//   cublas_tc         cublasGemmEx FP16 in, FP32 compute and out
//   cublaslt_fp8      cublasLtMatmul E4M3 "TN", FP32 out, no scales
//   cublaslt_fp8_amax cublasLtMatmul E4M3 with per-tensor scale pointers (amax/448), BF16 out
//   cublaslt_mxfp4    cublasLtMatmul E2M1 with VEC32_UE8M0 block scales, BF16 out (cuBLASLt 12.9.1
//                     rejects this combination of precisions; the row then reports unavailable)
#include <cublasLt.h>
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

#include "bwgemm.h"

bool g_row_unavailable = false;  // set by a row that cannot run on this device / shape

namespace {

#define CK(call)                                                                                \
  do {                                                                                          \
    cudaError_t e_ = (call);                                                                    \
    if (e_ != cudaSuccess) {                                                                    \
      fprintf(stderr, "CUDA %s:%d: %s\n", __FILE__, __LINE__, cudaGetErrorString(e_));          \
      exit(1);                                                                                  \
    }                                                                                           \
  } while (0)
#define BK(call)                                                        \
  do {                                                                  \
    if ((call) != BW_OK) {                                              \
      fprintf(stderr, "%s: %s\n", #call, bw_last_error_string());       \
      exit(1);                                                          \
    }                                                                   \
  } while (0)

cublasHandle_t handle() {
  static cublasHandle_t h = nullptr;
  if (!h) cublasCreate(&h);
  return h;
}
cublasLtHandle_t lt_handle() {
  static cublasLtHandle_t h = nullptr;
  if (!h) cublasLtCreate(&h);
  return h;
}
void* lt_workspace(size_t* bytes) {
  static void* ws = nullptr;
  constexpr size_t kBytes = 64u << 20;
  if (!ws) CK(cudaMalloc(&ws, kBytes));
  *bytes = kBytes;
  return ws;
}

// Staged operands, cached by source pointer and shape.
struct Staged {
  void *A = nullptr, *B = nullptr, *C16 = nullptr;
  uint8_t *sfa = nullptr, *sfb = nullptr;
  float* sc = nullptr;
  const float *srcA = nullptr, *srcB = nullptr;
  int M = 0, N = 0, K = 0;
  bool fresh(int m, int n, int k) {
    if (m == M && n == N && k == K && A) return false;
    cudaFree(A); cudaFree(B); cudaFree(C16); cudaFree(sfa); cudaFree(sfb); cudaFree(sc);
    A = B = C16 = nullptr; sfa = sfb = nullptr; sc = nullptr; srcA = srcB = nullptr;
    M = m; N = n; K = k;
    return true;
  }
};

struct LtPlan {
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
  cublasLtMatmulHeuristicResult_t heur{};
  bool ok = false;
  int M = 0, N = 0, K = 0;
};

void lt_run(LtPlan& pl, const void* X, const void* Y, void* C) {
  if (!pl.ok) {
    g_row_unavailable = true;
    return;
  }
  size_t wsb = 0;
  void* ws = lt_workspace(&wsb);
  float alpha = 1.f, beta = 0.f;
  cublasStatus_t st = cublasLtMatmul(lt_handle(), pl.op, &alpha, X, pl.la, Y, pl.lb, &beta, C, pl.lc, C, pl.lc,
                                     &pl.heur.algo, ws, wsb, nullptr);
  if (st != CUBLAS_STATUS_SUCCESS) fprintf(stderr, "cublasLtMatmul failed: %d\n", static_cast<int>(st));
}

// C^T [N x M] (col-major) = op(X) op(Y), X = Bt seen as col-major K x N (op T), Y = A seen as
// col-major K x M (op N): both operands K-contiguous ("TN").
void lt_plan(LtPlan& pl, cudaDataType_t ab, cudaDataType_t cd, int M, int N, int K, const float* sa, const float* sb,
             const uint8_t* sfa, const uint8_t* sfb) {
  if (pl.op) {
    cublasLtMatmulDescDestroy(pl.op);
    cublasLtMatrixLayoutDestroy(pl.la);
    cublasLtMatrixLayoutDestroy(pl.lb);
    cublasLtMatrixLayoutDestroy(pl.lc);
  }
  cublasLtMatmulDescCreate(&pl.op, CUBLAS_COMPUTE_32F, CUDA_R_32F);
  cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
  cublasLtMatmulDescSetAttribute(pl.op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof(ta));
  cublasLtMatmulDescSetAttribute(pl.op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof(tb));
  if (sa && sb) {
    cublasLtMatmulDescSetAttribute(pl.op, CUBLASLT_MATMUL_DESC_A_SCALE_POINTER, &sb, sizeof(sb));
    cublasLtMatmulDescSetAttribute(pl.op, CUBLASLT_MATMUL_DESC_B_SCALE_POINTER, &sa, sizeof(sa));
  }
  if (sfa && sfb) {
    cublasLtMatmulMatrixScale_t mode = CUBLASLT_MATMUL_MATRIX_SCALE_VEC32_UE8M0;
    cublasLtMatmulDescSetAttribute(pl.op, CUBLASLT_MATMUL_DESC_A_SCALE_MODE, &mode, sizeof(mode));
    cublasLtMatmulDescSetAttribute(pl.op, CUBLASLT_MATMUL_DESC_B_SCALE_MODE, &mode, sizeof(mode));
    cublasLtMatmulDescSetAttribute(pl.op, CUBLASLT_MATMUL_DESC_A_SCALE_POINTER, &sfb, sizeof(sfb));
    cublasLtMatmulDescSetAttribute(pl.op, CUBLASLT_MATMUL_DESC_B_SCALE_POINTER, &sfa, sizeof(sfa));
  }
  cublasLtMatrixLayoutCreate(&pl.la, ab, K, N, K);
  cublasLtMatrixLayoutCreate(&pl.lb, ab, K, M, K);
  cublasLtMatrixLayoutCreate(&pl.lc, cd, N, M, N);
  cublasLtMatmulPreference_t pref;
  cublasLtMatmulPreferenceCreate(&pref);
  size_t wsb = 0;
  lt_workspace(&wsb);
  cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &wsb, sizeof(wsb));
  int found = 0;
  cublasLtMatmulAlgoGetHeuristic(lt_handle(), pl.op, pl.la, pl.lb, pl.lc, pl.lc, pref, 1, &pl.heur, &found);
  cublasLtMatmulPreferenceDestroy(pref);
  pl.ok = found > 0;
  if (!pl.ok) fprintf(stderr, "cuBLASLt found no algorithm for this row (%dx%dx%d)\n", M, N, K);
  pl.M = M; pl.N = N; pl.K = K;
}

__global__ void k_widen(const __nv_bfloat16* __restrict__ s, float* __restrict__ d, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    d[i] = __bfloat162float(s[i]);
}

Staged g_tc, g_fp8, g_fp8a, g_mx;
LtPlan p_fp8, p_fp8a, p_mx;

}  // namespace

void launch_cublas(const float* A, const float* B, float* C, int M, int N, int K) {
  float al = 1.f, be = 0.f;
  cublasSgemm(handle(), CUBLAS_OP_N, CUBLAS_OP_N, N, M, K, &al, B, N, A, K, &be, C, N);
}

void launch_cublas_tc(const float* A, const float* B, float* C, int M, int N, int K) {
  Staged& s = g_tc;
  if (s.fresh(M, N, K)) {
    CK(cudaMalloc(&s.A, size_t(M) * K * 2));
    CK(cudaMalloc(&s.B, size_t(K) * N * 2));
  }
  if (A != s.srcA) { BK(bw_quantize_f16(A, s.A, (long long)M * K, nullptr)); s.srcA = A; }
  if (B != s.srcB) { BK(bw_quantize_f16(B, s.B, (long long)K * N, nullptr)); s.srcB = B; }
  float al = 1.f, be = 0.f;
  cublasGemmEx(handle(), CUBLAS_OP_N, CUBLAS_OP_N, N, M, K, &al, s.B, CUDA_R_16F, N, s.A, CUDA_R_16F, K, &be, C,
               CUDA_R_32F, N, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
}

void launch_cublaslt_fp8(const float* A, const float* B, float* C, int M, int N, int K) {
  Staged& s = g_fp8;
  if (s.fresh(M, N, K)) {
    CK(cudaMalloc(&s.A, size_t(M) * K));
    CK(cudaMalloc(&s.B, size_t(K) * N));
    lt_plan(p_fp8, CUDA_R_8F_E4M3, CUDA_R_32F, M, N, K, nullptr, nullptr, nullptr, nullptr);
  }
  if (A != s.srcA) { BK(bw_quantize_fp8(A, (uint8_t*)s.A, nullptr, M, K, 0, BW_SCALE_NONE, nullptr)); s.srcA = A; }
  if (B != s.srcB) { BK(bw_quantize_fp8(B, (uint8_t*)s.B, nullptr, K, N, 1, BW_SCALE_NONE, nullptr)); s.srcB = B; }
  lt_run(p_fp8, s.B, s.A, C);
}

void launch_cublaslt_fp8_amax(const float* A, const float* B, float*, int M, int N, int K) {
  Staged& s = g_fp8a;
  if (s.fresh(M, N, K)) {
    CK(cudaMalloc(&s.A, size_t(M) * K));
    CK(cudaMalloc(&s.B, size_t(K) * N));
    CK(cudaMalloc(&s.sc, 2 * sizeof(float)));
    CK(cudaMalloc(&s.C16, size_t(M) * N * 2));
    lt_plan(p_fp8a, CUDA_R_8F_E4M3, CUDA_R_16BF, M, N, K, s.sc, s.sc + 1, nullptr, nullptr);
  }
  if (A != s.srcA) { BK(bw_quantize_fp8(A, (uint8_t*)s.A, s.sc, M, K, 0, BW_SCALE_AMAX, nullptr)); s.srcA = A; }
  if (B != s.srcB) { BK(bw_quantize_fp8(B, (uint8_t*)s.B, s.sc + 1, K, N, 1, BW_SCALE_AMAX, nullptr)); s.srcB = B; }
  lt_run(p_fp8a, s.B, s.A, s.C16);
}
void finalize_cublaslt_fp8_amax(float* C, int M, int N) {
  k_widen<<<1184, 256>>>(static_cast<const __nv_bfloat16*>(g_fp8a.C16), C, (long long)M * N);
}

void launch_cublaslt_mxfp4(const float* A, const float* B, float*, int M, int N, int K) {
  Staged& s = g_mx;
  if (s.fresh(M, N, K)) {
    CK(cudaMalloc(&s.A, size_t(M) * K / 2));
    CK(cudaMalloc(&s.B, size_t(K) * N / 2));
    CK(cudaMalloc(&s.sfa, bw_sf_bytes(M, K)));
    CK(cudaMalloc(&s.sfb, bw_sf_bytes(N, K)));
    CK(cudaMalloc(&s.C16, size_t(M) * N * 2));
    lt_plan(p_mx, CUDA_R_4F_E2M1, CUDA_R_16BF, M, N, K, nullptr, nullptr, s.sfa, s.sfb);
  }
  if (A != s.srcA) { BK(bw_quantize_mxfp4(A, (uint8_t*)s.A, s.sfa, M, K, 0, BW_MX_BLOCK32, nullptr)); s.srcA = A; }
  if (B != s.srcB) { BK(bw_quantize_mxfp4(B, (uint8_t*)s.B, s.sfb, K, N, 1, BW_MX_BLOCK32, nullptr)); s.srcB = B; }
  lt_run(p_mx, s.B, s.A, s.C16);
}
void finalize_cublaslt_mxfp4(float* C, int M, int N) {
  k_widen<<<1184, 256>>>(static_cast<const __nv_bfloat16*>(g_mx.C16), C, (long long)M * N);
}
