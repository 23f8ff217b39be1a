// C-linkage shim over the reference's own launch_* entry points (src/main.cu:18-39) and its
// staging quantisers (src/gemm_mma_fp8.cu:37-80), so bench.py and the GPU tests can call the
// reference's stock kernels through ctypes. Compiled together with the reference's sources by
// oracle/build_ref.sh into oracle/_ref/libref_kernels.so. Test / baseline infrastructure only.
#include <cuda_runtime.h>
#include <cstdint>

void launch_wmma(const float*, const float*, float*, int, int, int);
void launch_mma_warptile(const float*, const float*, float*, int, int, int);
void launch_mma_fp8(const float*, const float*, float*, int, int, int);
void launch_cublas(const float*, const float*, float*, int, int, int);
void launch_cublas_tc(const float*, const float*, float*, int, int, int);
void launch_cublaslt_fp8(const float*, const float*, float*, int, int, int);

// The reference's quantisation kernels (defined in src/gemm_mma_fp8.cu, namespace lowprec).
namespace lowprec {
__global__ void q_fp8(const float* in, uint8_t* out, int n);
__global__ void q_fp8_t(const float* in, uint8_t* out, int K, int N);
__global__ void q_fp4(const float* in, uint8_t* out, int n, float scale);
__global__ void q_fp4_t(const float* in, uint8_t* out, int K, int N, float scale);
__global__ void q_mxfp4(const float* in, uint8_t* out, int n, float scale);
__global__ void q_mxfp4_t(const float* in, uint8_t* out, int K, int N, float scale);
}  // namespace lowprec

typedef void (*launch_fn)(const float*, const float*, float*, int, int, int);

static bool same(const char* a, const char* b) {
  while (*a && *a == *b) { ++a; ++b; }
  return *a == 0 && *b == 0;
}

extern "C" int ref_launch(const char* name, const float* A, const float* B, float* C, int M, int N, int K) {
  struct { const char* n; launch_fn f; } table[] = {
      {"wmma", launch_wmma},       {"mma_warptile", launch_mma_warptile}, {"mma_fp8", launch_mma_fp8},
      {"cublas", launch_cublas},   {"cublas_tc", launch_cublas_tc},       {"cublaslt_fp8", launch_cublaslt_fp8}};
  for (auto& e : table) {
    if (same(e.n, name)) {
      e.f(A, B, C, M, N, K);
      return static_cast<int>(cudaGetLastError());
    }
  }
  return -1;
}

// Runs one of the reference's staging kernels with the launch shapes its stage()
// (src/gemm_mma_fp8.cu:240-266) uses, on the legacy default stream. `in` is rows x cols FP32
// row-major; the "_t" forms write the cols x rows transpose (the reference's B -> Bt, with
// K = rows and N = cols). `scale` is the FP4 pre-scale (the reference passes 8).
extern "C" int ref_quant(const char* name, const float* in, uint8_t* out, int rows, int cols, float scale) {
  using namespace lowprec;
  const size_t n = static_cast<size_t>(rows) * cols;
  const int K = rows, N = cols;
  dim3 t2(16, 16), g2((K + 15) / 16, (N + 15) / 16);
  if (same(name, "q_fp8")) q_fp8<<<(int)((n + 255) / 256), 256>>>(in, out, (int)n);
  else if (same(name, "q_fp8_t")) q_fp8_t<<<g2, t2>>>(in, out, K, N);
  else if (same(name, "q_fp4")) q_fp4<<<(int)((n + 255) / 256), 256>>>(in, out, (int)n, scale);
  else if (same(name, "q_fp4_t")) q_fp4_t<<<g2, t2>>>(in, out, K, N, scale);
  else if (same(name, "q_mxfp4")) q_mxfp4<<<(int)((n / 2 + 255) / 256), 256>>>(in, out, (int)n, scale);
  else if (same(name, "q_mxfp4_t")) q_mxfp4_t<<<dim3((K / 2 + 15) / 16, (N + 15) / 16), t2>>>(in, out, K, N, scale);
  else return -1;
  return static_cast<int>(cudaGetLastError());
}
