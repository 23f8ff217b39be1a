// Library runtime: device state, error reporting, TMA descriptor encoding.
// The reference reports errors by printing and exit(1) (include/util.cuh:7-8); here every
// failure becomes a status code plus a per-thread message (bw_last_error_string).
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "bw_ptx.cuh"
#include "bw_runtime.cuh"

namespace bw {

// Failure-detection self-test: one CTA waits on an mbarrier that nothing ever arrives at,
// through the same bounded wait the GEMM kernels use. The wait must give up after the budget,
// record the timeout in the device status word and return normally.
__global__ void k_selftest_bounded_wait(int* status, unsigned long long budget_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const WaitCtl wc{&abort_flag, status, budget_ns};
    mbar_wait(&bar, 0, wc, 99);
  }
}

namespace {
thread_local std::string g_err;
constexpr int kMaxDevices = 64;
DeviceState g_dev[kMaxDevices];
std::mutex g_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
unsigned long long g_budget_ns = 2000000000ull;
unsigned long long* g_trace = nullptr;
int g_trace_ctas = 0;
bool g_budget_from_env = false;
}  // namespace

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(BW_ERR_CUDA, "%s failed: %s", what, cudaGetErrorString(e));
}

unsigned long long* trace_buffer(int ctas_needed) {
  return (g_trace && ctas_needed <= g_trace_ctas) ? g_trace : nullptr;
}

unsigned long long wait_budget_ns() {
  if (!g_budget_from_env) {
    g_budget_from_env = true;
    if (const char* s = getenv("BW_WAIT_BUDGET_MS")) {
      long long ms = atoll(s);
      if (ms > 0) g_budget_ns = static_cast<unsigned long long>(ms) * 1000000ull;
    }
  }
  return g_budget_ns;
}

static int load_encode() {
  if (g_encode) return BW_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return set_error(BW_ERR_CUDA, "cannot resolve cuTensorMapEncodeTiled from the driver");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return BW_OK;
}

int ensure_device(DeviceState** out) {
  int dev = 0;
  BW_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(BW_ERR_INVALID, "device index %d out of range", dev);
  DeviceState& d = g_dev[dev];
  if (!d.ready) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!d.ready) {
      cudaDeviceProp prop;
      BW_CUDA(cudaGetDeviceProperties(&prop, dev));
      if (prop.major != 10 || prop.minor != 0)
        return set_error(BW_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                         prop.major, prop.minor);
      int r = load_encode();
      if (r != BW_OK) return r;
      d.sms = prop.multiProcessorCount;
      d.major = prop.major;
      d.minor = prop.minor;
      BW_CUDA(cudaMalloc(&d.status, sizeof(int)));
      BW_CUDA(cudaMemset(d.status, 0, sizeof(int)));
      d.workspace_bytes = 4096;
      BW_CUDA(cudaMalloc(&d.workspace, d.workspace_bytes));
      BW_CUDA(cudaMemset(d.workspace, 0, d.workspace_bytes));
      d.ready = true;
    }
  }
  *out = &d;
  return BW_OK;
}

int splitk_workspace(DeviceState& d, cudaStream_t stream, size_t bytes, float** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState::SplitWs* slot = nullptr;
  for (auto& w : d.splitk)
    if (w.buf && w.stream == static_cast<void*>(stream)) { slot = &w; break; }
  if (!slot)
    for (auto& w : d.splitk)
      if (!w.buf) { slot = &w; break; }
  if (!slot) return set_error(BW_ERR_UNSUPPORTED, "split-K workspaces of %d streams in use", DeviceState::kSplitWs);
  if (slot->bytes < bytes) {
    if (slot->buf) BW_CUDA(cudaFree(slot->buf));  // synchronising: no launch still uses it
    slot->buf = nullptr;
    slot->bytes = 0;
    BW_CUDA(cudaMalloc(&slot->buf, bytes));
    slot->bytes = bytes;
    slot->stream = stream;
  }
  *out = slot->buf;
  return BW_OK;
}

int make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  int r = load_encode();
  if (r != BW_OK) return r;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult cr = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS)
    return set_error(BW_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu stride %llu box %u x %u",
                     static_cast<int>(cr), (unsigned long long)inner, (unsigned long long)outer,
                     (unsigned long long)row_stride_bytes, box_inner, box_outer);
  return BW_OK;
}

}  // namespace bw

using namespace bw;

extern "C" {

const char* bw_last_error_string(void) { return g_err.c_str(); }

int bw_version(void) { return (0 << 16) | 3; }

int bw_init(int device) {
  BW_CUDA(cudaSetDevice(device));
  DeviceState* d;
  return ensure_device(&d);
}

int bw_num_sms(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
  return n;
}

int bw_device_state_ready(int device) {
  if (device < 0 || device >= kMaxDevices) return 0;
  return g_dev[device].ready ? 1 : 0;
}

int bw_shutdown(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  int cur = 0;
  cudaGetDevice(&cur);
  for (int i = 0; i < kMaxDevices; ++i) {
    DeviceState& d = g_dev[i];
    if (!d.ready) continue;
    cudaSetDevice(i);
    cudaFree(d.status);
    cudaFree(d.workspace);
    for (auto& w : d.splitk) cudaFree(w.buf);
    d = DeviceState{};
  }
  cudaSetDevice(cur);
  return BW_OK;
}

int bw_ipc_malloc(size_t bytes, void** ptr, void* handle_out) {
  if (!ptr || !handle_out || bytes == 0) return set_error(BW_ERR_INVALID, "bw_ipc_malloc: bad arguments");
  DeviceState* d;
  int r = ensure_device(&d);
  if (r != BW_OK) return r;
  BW_CUDA(cudaMalloc(ptr, bytes));
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return cuda_error(e, "cudaIpcGetMemHandle");
  }
  static_assert(sizeof(h) == BW_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  return BW_OK;
}

int bw_ipc_free(void* ptr) {
  if (!ptr) return BW_OK;
  BW_CUDA(cudaFree(ptr));
  return BW_OK;
}

int bw_ipc_open(const void* handle, void** peer_ptr) {
  if (!handle || !peer_ptr) return set_error(BW_ERR_INVALID, "bw_ipc_open: bad arguments");
  DeviceState* d;
  int r = ensure_device(&d);
  if (r != BW_OK) return r;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  BW_CUDA(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return BW_OK;
}

int bw_ipc_close(void* peer_ptr) {
  if (!peer_ptr) return BW_OK;
  BW_CUDA(cudaIpcCloseMemHandle(peer_ptr));
  return BW_OK;
}

int bw_device_status(void* stream, int* out_status) {
  if (!out_status) return set_error(BW_ERR_INVALID, "out_status is null");
  DeviceState* d;
  int r = ensure_device(&d);
  if (r != BW_OK) return r;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  BW_CUDA(cudaStreamSynchronize(s));
  int v = 0;
  BW_CUDA(cudaMemcpy(&v, d->status, sizeof(int), cudaMemcpyDeviceToHost));
  BW_CUDA(cudaMemset(d->status, 0, sizeof(int)));
  *out_status = v;
  if (v != 0) return set_error(BW_ERR_TIMEOUT, "kernel wait budget expired at site %d", v & 255);
  return BW_OK;
}

int bw_selftest_bounded_wait(unsigned long long budget_ns, void* stream) {
  if (budget_ns == 0 || budget_ns > 10000000000ull) return set_error(BW_ERR_INVALID, "budget must be in (0, 10 s]");
  DeviceState* d;
  int r = ensure_device(&d);
  if (r != BW_OK) return r;
  k_selftest_bounded_wait<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(d->status, budget_ns);
  BW_CUDA(cudaGetLastError());
  int st = 0;
  return bw_device_status(stream, &st);
}

int bw_set_trace_buffer(unsigned long long* dev_buf, int max_ctas) {
  if (dev_buf && max_ctas <= 0) return set_error(BW_ERR_INVALID, "max_ctas must be > 0");
  g_trace = dev_buf;
  g_trace_ctas = dev_buf ? max_ctas : 0;
  return BW_OK;
}

int bw_set_wait_budget_ns(unsigned long long ns) {
  if (ns == 0) return set_error(BW_ERR_INVALID, "wait budget must be > 0");
  wait_budget_ns();
  g_budget_ns = ns;
  return BW_OK;
}

}  // extern "C"
