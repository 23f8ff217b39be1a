// gemm_bench: correctness + throughput driver with the reference's command line and CSV.
//
//   gemm_bench [M] [N] [K] [out_csv] [kernels]          (src/main.cu:43-113)
//     out_csv defaults to results/bench.csv; kernels is an optional comma-separated filter.
//
// Same flow as the reference: FP32 inputs filled on the host, copied to the device, a
// cublasSgemm result as the correctness reference, then for every selected row one warm-up
// call and 10 timed calls (CUDA events on the legacy default stream), max |C - C_ref| and
// TFLOP/s = 2MNK / t. The CSV header and first ten columns are the reference's
// (device,sm,M,N,K,kernel,ms,tflops,pct_of_cublas,max_abs_err); a file created by this
// driver also gets pct_of_peak (of the nominal dense peak for the row's precision) and dtype,
// appended after max_abs_err so csv.DictReader consumers of the old columns keep working.
// An existing file with the reference's header receives reference-shaped rows only.
//
// Inputs (BW_INPUT_DIST): "ref" (default) = glibc rand() uniform[-0.5, 0.5] from the default
// seed, exactly the reference's fill_rand (include/util.cuh:17), so the max_abs_err column is
// comparable with the reference's; "uniform" = U[-1, 1] and "normal" = N(0, 1) from
// std::mt19937_64(BW_SEED, default 0x5EED). BW_ITERS changes the 10 timed calls.
//
// Rows: our tcgen05 kernels (tc_*), cuBLAS / cuBLASLt comparison rows, and - when
// oracle/_ref/libref_kernels.so is present (built from the reference's sources for sm_100a) -
// the reference's own kernels as ref_* rows.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "bwgemm.h"

using LaunchFn = void (*)(const float*, const float*, float*, int, int, int);
using FinalizeFn = void (*)(float*, int, int);

void launch_tc_f16(const float*, const float*, float*, int, int, int);
void launch_tc_fp8(const float*, const float*, float*, int, int, int);
void launch_tc_fp4(const float*, const float*, float*, int, int, int);
void launch_tc_mxfp4(const float*, const float*, float*, int, int, int);
void launch_tc_fp8_amax(const float*, const float*, float*, int, int, int);
void launch_tc_fp4_amax(const float*, const float*, float*, int, int, int);
void launch_tc_mxfp4_b32(const float*, const float*, float*, int, int, int);
void finalize_tc_fp8_amax(float*, int, int);
void finalize_tc_fp4_amax(float*, int, int);
void finalize_tc_mxfp4_b32(float*, int, int);
void launch_cublas(const float*, const float*, float*, int, int, int);
void launch_cublas_tc(const float*, const float*, float*, int, int, int);
void launch_cublaslt_fp8(const float*, const float*, float*, int, int, int);
void launch_cublaslt_fp8_amax(const float*, const float*, float*, int, int, int);
void launch_cublaslt_mxfp4(const float*, const float*, float*, int, int, int);
void finalize_cublaslt_fp8_amax(float*, int, int);
void finalize_cublaslt_mxfp4(float*, int, int);
extern bool g_row_unavailable;

#define CUDA_CHECK(x)                                                                   \
  do {                                                                                  \
    cudaError_t e = (x);                                                                \
    if (e != cudaSuccess) {                                                             \
      fprintf(stderr, "CUDA %s:%d: %s\n", __FILE__, __LINE__, cudaGetErrorString(e));   \
      exit(1);                                                                          \
    }                                                                                   \
  } while (0)

namespace {

struct Kern {
  std::string name;
  LaunchFn fn;
  FinalizeFn finalize;  // widens a BF16 result into C after timing (nullptr: C written directly)
  double peak_tflops;   // nominal dense B200 peak for the row's precision
  const char* dtype;
};

// Reference-kernel rows through oracle/_ref/libref_kernels.so (ref_launch(name, ...)).
using RefLaunch = int (*)(const char*, const float*, const float*, float*, int, int, int);
RefLaunch g_ref = nullptr;
std::string g_ref_name;
void ref_row(const float* A, const float* B, float* C, int M, int N, int K) {
  int rc = g_ref(g_ref_name.c_str(), A, B, C, M, N, K);
  if (rc != 0) fprintf(stderr, "reference launcher %s returned %d\n", g_ref_name.c_str(), rc);
}
std::vector<std::string> g_ref_names;
void ref_wmma(const float* A, const float* B, float* C, int M, int N, int K) { g_ref_name = "wmma"; ref_row(A, B, C, M, N, K); }
void ref_mma_warptile(const float* A, const float* B, float* C, int M, int N, int K) { g_ref_name = "mma_warptile"; ref_row(A, B, C, M, N, K); }
void ref_mma_fp8(const float* A, const float* B, float* C, int M, int N, int K) { g_ref_name = "mma_fp8"; ref_row(A, B, C, M, N, K); }

// The ref_* comparison rows exist only when BW_REF_LIB names a library exporting
// `int ref_launch(name, A, B, C, M, N, K)` (the reference's own launchers built from its
// sources); without it the driver runs our rows and the library rows alone.
void load_reference_rows(const char*) {
  const char* env = getenv("BW_REF_LIB");
  if (!env || !*env) return;
  void* h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
  if (!h) return;
  g_ref = reinterpret_cast<RefLaunch>(dlsym(h, "ref_launch"));
}

void fill(std::vector<float>& a, std::vector<float>& b) {
  const char* dist = getenv("BW_INPUT_DIST");
  const std::string d = dist ? dist : "ref";
  if (d == "ref") {  // include/util.cuh:17, called for hA then hB from the default seed
    for (auto& x : a) x = (rand() / (float)RAND_MAX) - 0.5f;
    for (auto& x : b) x = (rand() / (float)RAND_MAX) - 0.5f;
    return;
  }
  const char* seed_s = getenv("BW_SEED");
  std::mt19937_64 rng(seed_s ? strtoull(seed_s, nullptr, 0) : 0x5EEDull);
  if (d == "normal") {
    std::normal_distribution<float> nd(0.f, 1.f);
    for (auto& x : a) x = nd(rng);
    for (auto& x : b) x = nd(rng);
  } else {
    std::uniform_real_distribution<float> ud(-1.f, 1.f);
    for (auto& x : a) x = ud(rng);
    for (auto& x : b) x = ud(rng);
  }
}

}  // namespace

int main(int argc, char** argv) {
  const int M = argc > 1 ? atoi(argv[1]) : 4096, N = argc > 2 ? atoi(argv[2]) : 4096, K = argc > 3 ? atoi(argv[3]) : 4096;
  const char* out = argc > 4 ? argv[4] : "results/bench.csv";
  const char* filter = argc > 5 ? argv[5] : nullptr;
  const int iters = getenv("BW_ITERS") ? atoi(getenv("BW_ITERS")) : 10;
  const size_t szA = sizeof(float) * size_t(M) * K, szB = sizeof(float) * size_t(K) * N, szC = sizeof(float) * size_t(M) * N;
  std::vector<float> hA(size_t(M) * K), hB(size_t(K) * N), hRef(size_t(M) * N), hC(size_t(M) * N);
  fill(hA, hB);
  float *dA, *dB, *dC;
  CUDA_CHECK(cudaMalloc(&dA, szA));
  CUDA_CHECK(cudaMalloc(&dB, szB));
  CUDA_CHECK(cudaMalloc(&dC, szC));
  CUDA_CHECK(cudaMemcpy(dA, hA.data(), szA, cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(dB, hB.data(), szB, cudaMemcpyHostToDevice));
  cudaDeviceProp prop;
  CUDA_CHECK(cudaGetDeviceProperties(&prop, 0));
  const int sm = prop.major * 10 + prop.minor;
  if (bw_init(0) != BW_OK) {
    fprintf(stderr, "bw_init: %s\n", bw_last_error_string());
    return 1;
  }
  load_reference_rows(argv[0]);

  launch_cublas(dA, dB, dC, M, N, K);
  CUDA_CHECK(cudaDeviceSynchronize());
  CUDA_CHECK(cudaMemcpy(hRef.data(), dC, szC, cudaMemcpyDeviceToHost));

  std::vector<Kern> kerns = {
      {"tc_f16", launch_tc_f16, nullptr, 2250.0, "f16"},
      {"tc_fp8", launch_tc_fp8, nullptr, 4500.0, "e4m3"},
      {"tc_fp4", launch_tc_fp4, nullptr, 9000.0, "e2m1"},
      {"tc_mxfp4", launch_tc_mxfp4, nullptr, 9000.0, "e2m1"},
      {"tc_fp8_amax", launch_tc_fp8_amax, finalize_tc_fp8_amax, 4500.0, "e4m3"},
      {"tc_fp4_amax", launch_tc_fp4_amax, finalize_tc_fp4_amax, 9000.0, "e2m1"},
      {"tc_mxfp4_b32", launch_tc_mxfp4_b32, finalize_tc_mxfp4_b32, 9000.0, "e2m1"},
      {"cublas", launch_cublas, nullptr, 0.0, "f32"},
      {"cublas_tc", launch_cublas_tc, nullptr, 2250.0, "f16"},
      {"cublaslt_fp8", launch_cublaslt_fp8, nullptr, 4500.0, "e4m3"},
      {"cublaslt_fp8_amax", launch_cublaslt_fp8_amax, finalize_cublaslt_fp8_amax, 4500.0, "e4m3"},
      {"cublaslt_mxfp4", launch_cublaslt_mxfp4, finalize_cublaslt_mxfp4, 9000.0, "e2m1"},
  };
  if (g_ref) {
    kerns.push_back({"ref_wmma", ref_wmma, nullptr, 2250.0, "f16"});
    kerns.push_back({"ref_mma_warptile", ref_mma_warptile, nullptr, 2250.0, "f16"});
    kerns.push_back({"ref_mma_fp8", ref_mma_fp8, nullptr, 4500.0, "e4m3"});
  }
  auto selected = [&](const std::string& name) {
    if (!filter) return true;
    const std::string hay = std::string(",") + filter + ",", needle = "," + name + ",";
    return hay.find(needle) != std::string::npos;
  };

  struct Row { std::string name; float ms, tf; double err, pct_peak; const char* dtype; };
  std::vector<Row> rows;
  double cublas_tf = 0;
  cudaEvent_t e0, e1;
  CUDA_CHECK(cudaEventCreate(&e0));
  CUDA_CHECK(cudaEventCreate(&e1));
  for (auto& k : kerns) {
    if (!selected(k.name)) continue;
    g_row_unavailable = false;
    k.fn(dA, dB, dC, M, N, K);  // warm-up (and staging)
    CUDA_CHECK(cudaDeviceSynchronize());
    if (g_row_unavailable) {
      printf("%-18s unavailable on this device/shape (library found no algorithm)\n", k.name.c_str());
      continue;
    }
    CUDA_CHECK(cudaEventRecord(e0));
    for (int i = 0; i < iters; ++i) k.fn(dA, dB, dC, M, N, K);
    CUDA_CHECK(cudaEventRecord(e1));
    CUDA_CHECK(cudaEventSynchronize(e1));
    float ms = 0;
    CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
    ms /= iters;
    if (k.finalize) k.finalize(dC, M, N);
    CUDA_CHECK(cudaDeviceSynchronize());
    int st = 0;
    if (bw_device_status(nullptr, &st) != BW_OK) fprintf(stderr, "%s: device status %d\n", k.name.c_str(), st);
    CUDA_CHECK(cudaMemcpy(hC.data(), dC, szC, cudaMemcpyDeviceToHost));
    double err = 0;
    for (size_t i = 0; i < hC.size(); ++i) err = fmax(err, fabs((double)hC[i] - hRef[i]));
    const float tf = static_cast<float>(2.0 * M * N * K / (ms * 1e-3) / 1e12);
    if (k.name == "cublas") cublas_tf = tf;
    rows.push_back({k.name, ms, tf, err, k.peak_tflops > 0 ? 100.0 * tf / k.peak_tflops : 0.0, k.dtype});
  }

  const std::string ref_header = "device,sm,M,N,K,kernel,ms,tflops,pct_of_cublas,max_abs_err";
  const std::string ext_header = ref_header + ",pct_of_peak,dtype";
  bool exists = access(out, F_OK) == 0;
  bool extended = true;
  if (exists) {
    FILE* r = fopen(out, "r");
    char line[512] = {0};
    if (r && fgets(line, sizeof(line), r)) extended = std::string(line).rfind(ext_header, 0) == 0;
    if (r) fclose(r);
  }
  FILE* f = fopen(out, "a");
  if (!f) {
    fprintf(stderr, "cannot open %s for writing\n", out);
    return 1;
  }
  if (!exists) fprintf(f, "%s\n", ext_header.c_str());
  printf("M=%d N=%d K=%d on %s (sm_%d)\n", M, N, K, prop.name, sm);
  for (auto& r : rows) {
    const double pct = cublas_tf > 0 ? 100.0 * r.tf / cublas_tf : 0.0;
    printf("%-18s %8.3f ms  %8.2f TFLOP/s  %7.1f%% cuBLAS  %5.1f%% peak  maxerr=%.3g\n", r.name.c_str(), r.ms, r.tf,
           pct, r.pct_peak, r.err);
    fprintf(f, "\"%s\",%d,%d,%d,%d,%s,%.3f,%.2f,%.1f,%.3g", prop.name, sm, M, N, K, r.name.c_str(), r.ms, r.tf, pct,
            r.err);
    if (extended) fprintf(f, ",%.1f,%s", r.pct_peak, r.dtype);
    fprintf(f, "\n");
  }
  fclose(f);
  cudaFree(dA);
  cudaFree(dB);
  cudaFree(dC);
  return 0;
}
