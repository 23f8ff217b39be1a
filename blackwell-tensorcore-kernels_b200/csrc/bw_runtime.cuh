// Host-side runtime shared by the library's translation units: per-thread error text,
// per-device state (SM count, device status word, workspace), TMA descriptor encoding
// through the driver entry point (no link-time dependency on libcuda).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/bwgemm.h"

namespace bw {

int set_error(int code, const char* fmt, ...);
int cuda_error(cudaError_t e, const char* what);
#define BW_CUDA(call)                                  \
  do {                                                 \
    cudaError_t e_ = (call);                           \
    if (e_ != cudaSuccess) return cuda_error(e_, #call); \
  } while (0)

struct DeviceState {
  bool ready = false;
  int sms = 0;
  int major = 0, minor = 0;
  int* status = nullptr;         // device status word (kernels' bounded waits report here)
  void* workspace = nullptr;     // small scratch for quantiser reductions
  size_t workspace_bytes = 0;
  struct SplitWs {               // FP32 split-K partial sums for BF16 outputs, one per stream
    void* stream = nullptr;
    float* buf = nullptr;
    size_t bytes = 0;
  };
  static constexpr int kSplitWs = 8;
  SplitWs splitk[kSplitWs];
};

// Ensures the current device is initialised; returns BW_OK or an error status.
int ensure_device(DeviceState** out);
unsigned long long wait_budget_ns();
// FP32 workspace of at least `bytes` private to `stream` on this device (grown on demand, kept
// until bw_shutdown); BW_ERR_UNSUPPORTED when every slot belongs to another stream.
int splitk_workspace(DeviceState& d, cudaStream_t stream, size_t bytes, float** out);
unsigned long long* trace_buffer(int ctas_needed);  // null unless bw_set_trace_buffer armed one

// 2-D row-major tensor map: dims {inner, outer}, box {box_inner, box_outer}, 128B swizzle.
int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// [world][M][N/world] -> row-major M x N for 4-byte (FP32) or 2-byte (BF16) elements.
int unshard_elems(const void* src, void* dst, int M, int N, int world, int elem_bytes, cudaStream_t stream);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace bw
