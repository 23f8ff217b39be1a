// tc_rate_probe: tcgen05 tensor-core issue-rate probe (B200 analogue of the reference's
// mma_rate_probe, src/mma_rate_probe.cu:54-171, which measures register-resident mma.sync).
//
// One CTA per SM. Operands sit in shared memory (128B-swizzled K-major tiles filled with a
// fixed pattern) and are never reloaded; one elected thread issues `iters` x 4 back-to-back
// tcgen05.mma into a single TMEM accumulator, commits once, and waits (bounded) for
// completion. clock64() around issue..completion gives cycles on that SM, so
//     FLOP / SM / clk = 2 * M * N * K_per_instr * 4 * iters / cycles
// is independent of the (power-capped) SM clock; the wall time of the launch gives the
// achieved TFLOP/s and, combined with the cycle count, the effective SM clock.
//
// Variants: f16 (kind::f16, M128 N256 K16), e4m3 (kind::f8f6f4, K32), mxf4 (kind::mxf4
// block32, packed E2M1 with 2^0 scales, K64), f16x2 (cta_group::2, M256 N256 K16 per pair),
// mxf4 pairs (cta_group::2, M256 with N 256 / 128 / 192 / 224, K64).
//   tc_rate_probe [iters=4096] [reps=5] [csv_out]
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "bw_ptx.cuh"

using namespace bw;

namespace {

constexpr int kThreads = 128;
constexpr int kABytes = 128 * 128;   // 128 rows x 128 B
constexpr int kBBytes = 256 * 128;   // 256 rows x 128 B
constexpr int kSfBytes = 2 * 512;    // scale factors for mxf4: A + B atoms

// 0 f16, 1 e4m3, 2 mxf4, 3 f16 cta pair, mxf4 pairs: 4 N256, 5 N128, 6 N192, 7 N224
template <int VARIANT>
__global__ void __launch_bounds__(kThreads, 1) k_rate(int iters, unsigned long long* cycles, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kABytes;
  uint8_t* sSF = sB + kBBytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sSF + kSfBytes);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(slot + 1);
  const int warp = threadIdx.x >> 5;
  constexpr bool kPair = VARIANT >= 3;
  constexpr bool kMx = VARIANT == 2 || VARIANT >= 4;

  // Operand pattern: small values (0x3c/0x38 patterns are ~1.0 in f16/e4m3; nibbles 0x2 =
  // 1.0 in e2m1) so no lane produces Inf/NaN. Scale factors 0x7f = 2^0.
  for (int i = threadIdx.x; i < (kABytes + kBBytes) / 4; i += kThreads)
    reinterpret_cast<uint32_t*>(smem)[i] = kMx ? 0x22222222u : (VARIANT == 1 ? 0x38303830u : 0x3c003800u);
  for (int i = threadIdx.x; i < kSfBytes / 4; i += kThreads) reinterpret_cast<uint32_t*>(sSF)[i] = 0x7f7f7f7fu;
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    if constexpr (kPair) { tmem_alloc_pair(slot, 512); tmem_relinquish_pair(); }
    else { tmem_alloc(slot, 512); tmem_relinquish(); }
  }
  tc_fence_before();
  if constexpr (kPair) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  const bool issuer = threadIdx.x == 0 && (!kPair || cluster_ctarank() == 0);
  if (issuer) {
    const WaitCtl wc{abort_flag, status, 2000000000ull};
    const uint32_t a = smem_u32(sA), b = smem_u32(sB), sf = smem_u32(sSF);
    if constexpr (VARIANT == 2) {
      tmem_cp_32x128b_warpx4(tmem + 256, sdesc_noswz(sf, 16, 128));
      tmem_cp_32x128b_warpx4(tmem + 260, sdesc_noswz(sf + 512, 16, 128));
    }
    if constexpr (VARIANT >= 4) {  // SFA at column 256, SFB (two 128-row blocks) at 260 and 264
      tmem_cp_32x128b_warpx4_pair(tmem + 256, sdesc_noswz(sf, 16, 128));
      tmem_cp_32x128b_warpx4_pair(tmem + 260, sdesc_noswz(sf + 512, 16, 128));
      tmem_cp_32x128b_warpx4_pair(tmem + 264, sdesc_noswz(sf + 512, 16, 128));
    }
    const uint32_t idesc = VARIANT == 2   ? idesc_mxf4(128, 256, 0, 0)
                         : VARIANT == 4 ? idesc_mxf4(256, 256, 0, 0)
                         : VARIANT == 5 ? idesc_mxf4(256, 128, 0, 0)
                         : VARIANT == 6 ? idesc_mxf4(256, 192, 0, 0)
                         : VARIANT == 7 ? idesc_mxf4(256, 224, 0, 0)
                                        : idesc_dense(0, 0, false, kPair ? 256 : 128, 256);
    const long long t0 = clock64();
#pragma unroll 1
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t ad = sdesc_sw128(a + k * 32, 16, 1024);
        const uint64_t bd = sdesc_sw128(b + k * 32, 16, 1024);
        const uint32_t acc = (it | k) ? 1u : 0u;
        if constexpr (VARIANT == 0) umma_f16(tmem, ad, bd, idesc, acc);
        else if constexpr (VARIANT == 1) umma_f8f6f4(tmem, ad, bd, idesc, acc);
        else if constexpr (VARIANT == 2) umma_mxf4(tmem, ad, bd, idesc, tmem + 256, tmem + 260, acc);
        else if constexpr (VARIANT >= 4) umma_mxf4_pair(tmem, ad, bd, idesc, tmem + 256, tmem + 260, acc);
        else umma_f16_pair(tmem, ad, bd, idesc, acc);
      }
    }
    if constexpr (kPair) umma_commit_pair(smem_u32(bar));
    else umma_commit(bar);
    mbar_wait(bar, 0, wc, 21);
    cycles[blockIdx.x] = static_cast<unsigned long long>(clock64() - t0);
  }
  tc_fence_before();
  if constexpr (kPair) cluster_sync(); else __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    if constexpr (kPair) tmem_dealloc_pair(tmem, 512);
    else tmem_dealloc(tmem, 512);
  }
}

#define CK(x)                                                                           \
  do {                                                                                  \
    cudaError_t e = (x);                                                                \
    if (e != cudaSuccess) {                                                             \
      fprintf(stderr, "CUDA %s:%d: %s\n", __FILE__, __LINE__, cudaGetErrorString(e));   \
      exit(1);                                                                          \
    }                                                                                   \
  } while (0)

}  // namespace

int main(int argc, char** argv) {
  const int iters = argc > 1 ? atoi(argv[1]) : 4096;
  const int reps = argc > 2 ? atoi(argv[2]) : 5;
  const char* csv = argc > 3 ? argv[3] : nullptr;
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, 0));
  const int sms = prop.multiProcessorCount;
  // more shared memory than two CTAs can share, so every SM runs exactly one CTA
  const size_t smem = 120 * 1024;
  unsigned long long* dcyc;
  int* dstat;
  CK(cudaMalloc(&dcyc, sizeof(unsigned long long) * sms));
  CK(cudaMalloc(&dstat, sizeof(int)));
  CK(cudaMemset(dstat, 0, sizeof(int)));
  CK(cudaFuncSetAttribute(k_rate<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CK(cudaFuncSetAttribute(k_rate<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CK(cudaFuncSetAttribute(k_rate<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CK(cudaFuncSetAttribute(k_rate<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CK(cudaFuncSetAttribute(k_rate<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CK(cudaFuncSetAttribute(k_rate<5>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CK(cudaFuncSetAttribute(k_rate<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CK(cudaFuncSetAttribute(k_rate<7>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  constexpr int kVariants = 8;
  const char* names[kVariants] = {"f16_m128n256k16",       "e4m3_m128n256k32",      "mxf4_m128n256k64",
                                  "f16_pair_m256n256k16",  "mxf4_pair_m256n256k64", "mxf4_pair_m256n128k64",
                                  "mxf4_pair_m256n192k64", "mxf4_pair_m256n224k64"};
  const double kflop[kVariants] = {2.0 * 128 * 256 * 16, 2.0 * 128 * 256 * 32, 2.0 * 128 * 256 * 64,
                                   2.0 * 256 * 256 * 16, 2.0 * 256 * 256 * 64, 2.0 * 256 * 128 * 64,
                                   2.0 * 256 * 192 * 64, 2.0 * 256 * 224 * 64};
  FILE* f = csv ? fopen(csv, "w") : nullptr;
  if (f) fprintf(f, "variant,rep,ms,tflops,flop_per_sm_clk,sm_mhz_effective\n");
  printf("%-22s %4s %9s %9s %14s %10s\n", "variant", "rep", "ms", "TFLOP/s", "FLOP/SM/clk", "SM MHz");
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  std::vector<unsigned long long> cyc(sms);
  for (int rep = 0; rep < reps; ++rep) {
    for (int v = 0; v < kVariants; ++v) {
      const bool pair = v >= 3;
      const int grid = pair ? (sms / 2) * 2 : sms;
      auto launch = [&] {
        if (pair) {
          cudaLaunchConfig_t cfg = {};
          cfg.gridDim = dim3(grid);
          cfg.blockDim = dim3(kThreads);
          cfg.dynamicSmemBytes = smem;
          cudaLaunchAttribute at;
          at.id = cudaLaunchAttributeClusterDimension;
          at.val.clusterDim.x = 2;
          at.val.clusterDim.y = 1;
          at.val.clusterDim.z = 1;
          cfg.attrs = &at;
          cfg.numAttrs = 1;
          if (v == 3) CK(cudaLaunchKernelEx(&cfg, k_rate<3>, iters, dcyc, dstat));
          else if (v == 4) CK(cudaLaunchKernelEx(&cfg, k_rate<4>, iters, dcyc, dstat));
          else if (v == 5) CK(cudaLaunchKernelEx(&cfg, k_rate<5>, iters, dcyc, dstat));
          else if (v == 6) CK(cudaLaunchKernelEx(&cfg, k_rate<6>, iters, dcyc, dstat));
          else CK(cudaLaunchKernelEx(&cfg, k_rate<7>, iters, dcyc, dstat));
        } else if (v == 0) {
          k_rate<0><<<grid, kThreads, smem>>>(iters, dcyc, dstat);
        } else if (v == 1) {
          k_rate<1><<<grid, kThreads, smem>>>(iters, dcyc, dstat);
        } else {
          k_rate<2><<<grid, kThreads, smem>>>(iters, dcyc, dstat);
        }
        CK(cudaGetLastError());
      };
      launch();  // warm-up
      CK(cudaMemset(dcyc, 0, sizeof(unsigned long long) * sms));
      CK(cudaEventRecord(e0));
      launch();
      CK(cudaEventRecord(e1));
      CK(cudaEventSynchronize(e1));
      float ms = 0;
      CK(cudaEventElapsedTime(&ms, e0, e1));
      CK(cudaMemcpy(cyc.data(), dcyc, sizeof(unsigned long long) * sms, cudaMemcpyDeviceToHost));
      std::vector<double> per;
      for (int i = 0; i < grid; ++i)
        if (cyc[i]) per.push_back(cyc[i]);
      std::sort(per.begin(), per.end());
      const double med = per.empty() ? 0 : per[per.size() / 2];
      const int issuers = pair ? grid / 2 : grid;
      const double flop_instr = kflop[v] * 4.0 * iters;
      // per SM: a pair instruction's work is split over two SMs
      const double per_sm_clk = med > 0 ? flop_instr / med / (pair ? 2.0 : 1.0) : 0;
      const double tflops = flop_instr * issuers / (ms * 1e-3) / 1e12;
      const double mhz = med > 0 ? med / (ms * 1e3) : 0;
      printf("%-22s %4d %9.3f %9.1f %14.1f %10.0f\n", names[v], rep, ms, tflops, per_sm_clk, mhz);
      if (f) fprintf(f, "%s,%d,%.4f,%.2f,%.2f,%.1f\n", names[v], rep, ms, tflops, per_sm_clk, mhz);
    }
  }
  int st = 0;
  CK(cudaMemcpy(&st, dstat, sizeof(int), cudaMemcpyDeviceToHost));
  if (f) fclose(f);
  if (st) { fprintf(stderr, "probe wait budget expired (status %d)\n", st); return 2; }
  return 0;
}
