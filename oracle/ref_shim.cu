// C-linkage shim over the reference's own launch_* entry points (src/main.cu:18-39), so
// bench.py and the GPU tests can call the reference's stock kernels through ctypes.
// Compiled together with the reference's sources by oracle/build_ref.sh into
// oracle/_ref/libref_kernels.so. Test / baseline infrastructure only.
#include <cuda_runtime.h>

void launch_wmma(const float*, const float*, float*, int, int, int);
void launch_mma_warptile(const float*, const float*, float*, int, int, int);
void launch_mma_fp8(const float*, const float*, float*, int, int, int);
void launch_cublas(const float*, const float*, float*, int, int, int);
void launch_cublas_tc(const float*, const float*, float*, int, int, int);
void launch_cublaslt_fp8(const float*, const float*, float*, int, int, int);

typedef void (*launch_fn)(const float*, const float*, float*, int, int, int);

extern "C" int ref_launch(const char* name, const float* A, const float* B, float* C, int M, int N, int K) {
  struct { const char* n; launch_fn f; } table[] = {
      {"wmma", launch_wmma},       {"mma_warptile", launch_mma_warptile}, {"mma_fp8", launch_mma_fp8},
      {"cublas", launch_cublas},   {"cublas_tc", launch_cublas_tc},       {"cublaslt_fp8", launch_cublaslt_fp8}};
  for (auto& e : table) {
    const char* a = e.n;
    const char* b = name;
    while (*a && *a == *b) { ++a; ++b; }
    if (*a == 0 && *b == 0) {
      e.f(A, B, C, M, N, K);
      return static_cast<int>(cudaGetLastError());
    }
  }
  return -1;
}
