// Reference-signature launchers over the C ABI.
//
// The reference registers every kernel as
//     void launch_<name>(const float* A, const float* B, float* C, int M, int N, int K)
// (src/main.cu:18-39): A (MxK), B (KxN) and C (MxN) are FP32 row-major device buffers, and
// each launcher stages (casts / quantises) its inputs into launcher-owned buffers that are
// cached by pointer identity and shape, so repeated timed calls only run the GEMM
// (src/gemm_mma.cu:152-168, src/gemm_mma_fp8.cu:230-264). These launchers keep that contract
// and route the GEMM through bw_gemm_* (tcgen05 kernels). Errors print the library's message
// and exit(1), as the reference's CUDA_CHECK does (include/util.cuh:7-8).
//
// Rows with reference semantics (same quantisation and unscale as the reference's rows):
//   tc_f16     fp32 -> fp16 (RNE), C = A x B in FP32                    (mma_warptile / wmma)
//   tc_fp8     e4m3(x) unscaled, FP32 out                                (mma_fp8)
//   tc_fp4     e2m1(8x), result x 1/64                                   (mma_fp4)
//   tc_mxfp4   packed e2m1(8x), all block scales 2^0, result x 1/64      (mma_mxfp4)
// Rows with the BASELINE behaviour (per-tensor / per-block scales, BF16 out; the BF16 result
// is widened into C by the row's finalize hook, outside the timed loop):
//   tc_fp8_amax    s = amax/448 per tensor
//   tc_fp4_amax    s = amax/6 per tensor
//   tc_mxfp4_b32   UE8M0 scale per 32 K elements, e = floor(log2 amax) - 2
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

#include "bwgemm.h"

namespace {

void die(const char* what) {
  fprintf(stderr, "%s: %s\n", what, bw_last_error_string());
  exit(1);
}
#define BW_OR_DIE(call)                 \
  do {                                  \
    if ((call) != BW_OK) die(#call);    \
  } while (0)
#define CUDA_OR_DIE(call)                                                        \
  do {                                                                           \
    cudaError_t e_ = (call);                                                     \
    if (e_ != cudaSuccess) {                                                     \
      fprintf(stderr, "CUDA %s:%d: %s\n", __FILE__, __LINE__, cudaGetErrorString(e_)); \
      exit(1);                                                                   \
    }                                                                            \
  } while (0)

// One staging cache per launcher: quantised A, quantised (transposed) B, scales, and for
// BF16 rows the BF16 result. Re-staged when the input pointer or the shape changes.
struct Stage {
  void* A = nullptr;
  void* B = nullptr;
  uint8_t* sfa = nullptr;
  uint8_t* sfb = nullptr;
  float* scales = nullptr;  // [0] = scale_a, [1] = scale_b
  void* Cbf16 = nullptr;
  const float* srcA = nullptr;
  const float* srcB = nullptr;
  int M = 0, N = 0, K = 0;

  void reset_if_shape(int m, int n, int k) {
    if (m == M && n == N && k == K) return;
    cudaFree(A); cudaFree(B); cudaFree(sfa); cudaFree(sfb); cudaFree(scales); cudaFree(Cbf16);
    A = B = Cbf16 = nullptr;
    sfa = sfb = nullptr;
    scales = nullptr;
    srcA = srcB = nullptr;
    M = m; N = n; K = k;
  }
};

enum class Row { F16, FP8, FP4, MXFP4, FP8_AMAX, FP4_AMAX, MXFP4_B32 };
Stage g_stage[7];

void stage_inputs(Row row, const float* A, const float* B, int M, int N, int K) {
  Stage& s = g_stage[static_cast<int>(row)];
  s.reset_if_shape(M, N, K);
  const size_t mk = size_t(M) * K, kn = size_t(K) * N;
  if (!s.A) {
    switch (row) {
      case Row::F16:
        CUDA_OR_DIE(cudaMalloc(&s.A, mk * 2));
        CUDA_OR_DIE(cudaMalloc(&s.B, kn * 2));
        break;
      case Row::FP8:
      case Row::FP8_AMAX:
        CUDA_OR_DIE(cudaMalloc(&s.A, mk));
        CUDA_OR_DIE(cudaMalloc(&s.B, kn));
        break;
      default:  // packed fp4
        CUDA_OR_DIE(cudaMalloc(&s.A, mk / 2));
        CUDA_OR_DIE(cudaMalloc(&s.B, kn / 2));
        CUDA_OR_DIE(cudaMalloc(&s.sfa, bw_sf_bytes(M, K)));
        CUDA_OR_DIE(cudaMalloc(&s.sfb, bw_sf_bytes(N, K)));
        break;
    }
    CUDA_OR_DIE(cudaMalloc(&s.scales, 2 * sizeof(float)));
    CUDA_OR_DIE(cudaMalloc(&s.Cbf16, size_t(M) * N * 2));
    if (row == Row::MXFP4) {
      // reference mxfp4: x8 on both operands, unscaled by 1/64 in the epilogue
      const float eighth[2] = {0.125f, 0.125f};
      CUDA_OR_DIE(cudaMemcpy(s.scales, eighth, sizeof(eighth), cudaMemcpyHostToDevice));
    }
  }
  auto q = [&](const float* src, bool is_b) {
    void* dst = is_b ? s.B : s.A;
    const int rows = is_b ? K : M, cols = is_b ? N : K;
    float* sc = s.scales + (is_b ? 1 : 0);
    uint8_t* sf = is_b ? s.sfb : s.sfa;
    switch (row) {
      case Row::F16: BW_OR_DIE(bw_quantize_f16(src, dst, (long long)rows * cols, nullptr)); break;
      case Row::FP8:
        BW_OR_DIE(bw_quantize_fp8(src, static_cast<uint8_t*>(dst), sc, rows, cols, is_b, BW_SCALE_NONE, nullptr));
        break;
      case Row::FP8_AMAX:
        BW_OR_DIE(bw_quantize_fp8(src, static_cast<uint8_t*>(dst), sc, rows, cols, is_b, BW_SCALE_AMAX, nullptr));
        break;
      case Row::FP4:
        BW_OR_DIE(bw_quantize_fp4(src, static_cast<uint8_t*>(dst), sc, rows, cols, is_b, BW_SCALE_FIXED8,
                                  BW_FP4_PACKED, nullptr));
        break;
      case Row::FP4_AMAX:
        BW_OR_DIE(bw_quantize_fp4(src, static_cast<uint8_t*>(dst), sc, rows, cols, is_b, BW_SCALE_AMAX,
                                  BW_FP4_PACKED, nullptr));
        break;
      case Row::MXFP4:
        BW_OR_DIE(bw_quantize_mxfp4(src, static_cast<uint8_t*>(dst), sf, rows, cols, is_b, BW_MX_UNIT_FIXED8, nullptr));
        break;
      case Row::MXFP4_B32:
        BW_OR_DIE(bw_quantize_mxfp4(src, static_cast<uint8_t*>(dst), sf, rows, cols, is_b, BW_MX_BLOCK32, nullptr));
        break;
    }
  };
  if (A != s.srcA) { q(A, false); s.srcA = A; }
  if (B != s.srcB) { q(B, true); s.srcB = B; }
}

__global__ void k_widen_bf16(const __nv_bfloat16* __restrict__ src, float* __restrict__ dst, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = __bfloat162float(src[i]);
}

void widen(Row row, float* C, int M, int N) {
  const Stage& s = g_stage[static_cast<int>(row)];
  const long long n = (long long)M * N;
  k_widen_bf16<<<1184, 256>>>(static_cast<const __nv_bfloat16*>(s.Cbf16), C, n);
  CUDA_OR_DIE(cudaGetLastError());
}

}  // namespace

void launch_tc_f16(const float* A, const float* B, float* C, int M, int N, int K) {
  stage_inputs(Row::F16, A, B, M, N, K);
  const Stage& s = g_stage[static_cast<int>(Row::F16)];
  BW_OR_DIE(bw_gemm_f16(s.A, s.B, C, M, N, K, nullptr));
}

void launch_tc_fp8(const float* A, const float* B, float* C, int M, int N, int K) {
  stage_inputs(Row::FP8, A, B, M, N, K);
  const Stage& s = g_stage[static_cast<int>(Row::FP8)];
  BW_OR_DIE(bw_gemm_fp8(static_cast<uint8_t*>(s.A), static_cast<uint8_t*>(s.B), nullptr, nullptr, C, BW_OUT_F32, M,
                        N, K, nullptr));
}

void launch_tc_fp4(const float* A, const float* B, float* C, int M, int N, int K) {
  stage_inputs(Row::FP4, A, B, M, N, K);
  const Stage& s = g_stage[static_cast<int>(Row::FP4)];
  BW_OR_DIE(bw_gemm_fp4(static_cast<uint8_t*>(s.A), static_cast<uint8_t*>(s.B), s.scales, s.scales + 1, C,
                        BW_OUT_F32, M, N, K, nullptr));
}

void launch_tc_mxfp4(const float* A, const float* B, float* C, int M, int N, int K) {
  stage_inputs(Row::MXFP4, A, B, M, N, K);
  const Stage& s = g_stage[static_cast<int>(Row::MXFP4)];
  BW_OR_DIE(bw_gemm_mxfp4(static_cast<uint8_t*>(s.A), static_cast<uint8_t*>(s.B), s.sfa, s.sfb, s.scales,
                          s.scales + 1, C, BW_OUT_F32, M, N, K, nullptr));
}

void launch_tc_fp8_amax(const float* A, const float* B, float*, int M, int N, int K) {
  stage_inputs(Row::FP8_AMAX, A, B, M, N, K);
  const Stage& s = g_stage[static_cast<int>(Row::FP8_AMAX)];
  BW_OR_DIE(bw_gemm_fp8(static_cast<uint8_t*>(s.A), static_cast<uint8_t*>(s.B), s.scales, s.scales + 1, s.Cbf16,
                        BW_OUT_BF16, M, N, K, nullptr));
}
void finalize_tc_fp8_amax(float* C, int M, int N) { widen(Row::FP8_AMAX, C, M, N); }

void launch_tc_fp4_amax(const float* A, const float* B, float*, int M, int N, int K) {
  stage_inputs(Row::FP4_AMAX, A, B, M, N, K);
  const Stage& s = g_stage[static_cast<int>(Row::FP4_AMAX)];
  BW_OR_DIE(bw_gemm_fp4(static_cast<uint8_t*>(s.A), static_cast<uint8_t*>(s.B), s.scales, s.scales + 1, s.Cbf16,
                        BW_OUT_BF16, M, N, K, nullptr));
}
void finalize_tc_fp4_amax(float* C, int M, int N) { widen(Row::FP4_AMAX, C, M, N); }

void launch_tc_mxfp4_b32(const float* A, const float* B, float*, int M, int N, int K) {
  stage_inputs(Row::MXFP4_B32, A, B, M, N, K);
  const Stage& s = g_stage[static_cast<int>(Row::MXFP4_B32)];
  BW_OR_DIE(bw_gemm_mxfp4(static_cast<uint8_t*>(s.A), static_cast<uint8_t*>(s.B), s.sfa, s.sfb, nullptr, nullptr,
                          s.Cbf16, BW_OUT_BF16, M, N, K, nullptr));
}
void finalize_tc_mxfp4_b32(float* C, int M, int N) { widen(Row::MXFP4_B32, C, M, N); }
