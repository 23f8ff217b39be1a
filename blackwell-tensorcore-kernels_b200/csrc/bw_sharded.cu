// Single-process N-sharded GEMM over several GPUs of one node (bw_gemm_sharded).
//
// The reference runs one GPU (src/main.cu:47-111); the sharded form is new. Columns of B and C
// are independent, so shard r computes C_r = A x B[:, r*N/g : (r+1)*N/g] with the single-GPU
// kernels and no communication. A gathered C is an NCCL all-gather of the M x (N/g) shards
// (shard-major [g][M][N/g], since NCCL gathers contiguous chunks) into a per-device staging
// buffer, then a column unshard into row-major M x N.
//
// NCCL is loaded with dlopen on the first gather: a process that also runs torch.distributed
// already has libnccl.so.2 mapped and gets that copy, and the library itself keeps no
// link-time dependency on NCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "bw_runtime.cuh"

namespace bw {
namespace {

struct NcclApi {
  bool tried = false;
  bool ok = false;
  ncclResult_t (*comm_init_all)(ncclComm_t*, int, const int*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

struct CommSet {
  std::vector<int> devices;
  std::vector<ncclComm_t> comms;
};

struct Staging {
  void* ptr = nullptr;
  size_t bytes = 0;
};

std::mutex g_shard_mu;
NcclApi g_nccl;
std::vector<CommSet> g_comm_sets;
Staging g_staging[64];

int load_nccl() {
  if (g_nccl.tried) return g_nccl.ok ? BW_OK : set_error(BW_ERR_UNSUPPORTED, "NCCL could not be loaded");
  g_nccl.tried = true;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  if (!h) return set_error(BW_ERR_UNSUPPORTED, "gather needs libnccl.so.2: %s", dlerror());
  g_nccl.comm_init_all = reinterpret_cast<decltype(g_nccl.comm_init_all)>(dlsym(h, "ncclCommInitAll"));
  g_nccl.all_gather = reinterpret_cast<decltype(g_nccl.all_gather)>(dlsym(h, "ncclAllGather"));
  g_nccl.group_start = reinterpret_cast<decltype(g_nccl.group_start)>(dlsym(h, "ncclGroupStart"));
  g_nccl.group_end = reinterpret_cast<decltype(g_nccl.group_end)>(dlsym(h, "ncclGroupEnd"));
  g_nccl.error_string = reinterpret_cast<decltype(g_nccl.error_string)>(dlsym(h, "ncclGetErrorString"));
  g_nccl.ok = g_nccl.comm_init_all && g_nccl.all_gather && g_nccl.group_start && g_nccl.group_end &&
              g_nccl.error_string;
  return g_nccl.ok ? BW_OK : set_error(BW_ERR_UNSUPPORTED, "libnccl.so.2 lacks the collective entry points");
}

int nccl_error(ncclResult_t r, const char* what) {
  return set_error(BW_ERR_CUDA, "%s: %s", what, g_nccl.error_string ? g_nccl.error_string(r) : "NCCL error");
}

// Communicators over exactly this ordered device list (created once, kept for the process).
int comms_for(const std::vector<int>& devices, const std::vector<ncclComm_t>** out) {
  for (const CommSet& cs : g_comm_sets)
    if (cs.devices == devices) {
      *out = &cs.comms;
      return BW_OK;
    }
  CommSet cs;
  cs.devices = devices;
  cs.comms.resize(devices.size());
  const ncclResult_t r = g_nccl.comm_init_all(cs.comms.data(), static_cast<int>(devices.size()), devices.data());
  if (r != ncclSuccess) return nccl_error(r, "ncclCommInitAll");
  g_comm_sets.push_back(std::move(cs));
  *out = &g_comm_sets.back().comms;
  return BW_OK;
}

// Shard-major staging buffer on the current device, grown on demand.
int staging_for(int device, size_t bytes, void** out) {
  Staging& s = g_staging[device];
  if (s.bytes < bytes) {
    if (s.ptr) BW_CUDA(cudaFree(s.ptr));  // synchronising: no earlier gather still reads it
    s.ptr = nullptr;
    s.bytes = 0;
    BW_CUDA(cudaMalloc(&s.ptr, bytes));
    s.bytes = bytes;
  }
  *out = s.ptr;
  return BW_OK;
}

int validate(int dtype, int out_dtype, const bw_shard_t* shards, int ngpu, int M, int N, int K, int gather) {
  if (dtype < BW_DTYPE_F16 || dtype > BW_DTYPE_MXFP4) return set_error(BW_ERR_INVALID, "bad dtype %d", dtype);
  if (out_dtype != BW_OUT_F32 && out_dtype != BW_OUT_BF16) return set_error(BW_ERR_INVALID, "bad out_dtype %d", out_dtype);
  if (dtype == BW_DTYPE_F16 && out_dtype != BW_OUT_F32)
    return set_error(BW_ERR_INVALID, "the FP16 GEMM writes FP32 C (out_dtype BW_OUT_F32)");
  if (ngpu < 1 || ngpu > 64) return set_error(BW_ERR_INVALID, "ngpu=%d out of range", ngpu);
  if (!shards) return set_error(BW_ERR_INVALID, "shards is null");
  if (M < 0 || N < 0 || K < 0) return set_error(BW_ERR_INVALID, "negative size M=%d N=%d K=%d", M, N, K);
  if (N % ngpu != 0) return set_error(BW_ERR_INVALID, "N=%d is not divisible by ngpu=%d", N, ngpu);
  for (int r = 0; r < ngpu; ++r) {
    const bw_shard_t& s = shards[r];
    if (s.device < 0 || s.device >= 64) return set_error(BW_ERR_INVALID, "shard %d: device %d", r, s.device);
    for (int q = 0; q < r; ++q)
      if (shards[q].device == s.device) return set_error(BW_ERR_INVALID, "shards %d and %d share device %d", q, r, s.device);
    if (!s.A || !s.B || !s.C) return set_error(BW_ERR_INVALID, "shard %d: A, B or C is null", r);
    if (dtype == BW_DTYPE_MXFP4 && (!s.sfA || !s.sfB))
      return set_error(BW_ERR_INVALID, "shard %d: MXFP4 needs sfA and sfB", r);
    if (gather && !s.C_gathered) return set_error(BW_ERR_INVALID, "shard %d: gather needs C_gathered", r);
  }
  return BW_OK;
}

int shard_gemm(int dtype, int out_dtype, const bw_shard_t& s, int M, int ns, int K) {
  switch (dtype) {
    case BW_DTYPE_F16:
      return bw_gemm_f16(s.A, s.B, static_cast<float*>(s.C), M, ns, K, s.stream);
    case BW_DTYPE_FP8:
      return bw_gemm_fp8(static_cast<const uint8_t*>(s.A), static_cast<const uint8_t*>(s.B), s.scale_a, s.scale_b,
                         s.C, out_dtype, M, ns, K, s.stream);
    case BW_DTYPE_FP4:
      return bw_gemm_fp4(static_cast<const uint8_t*>(s.A), static_cast<const uint8_t*>(s.B), s.scale_a, s.scale_b,
                         s.C, out_dtype, M, ns, K, s.stream);
    default:
      return bw_gemm_mxfp4(static_cast<const uint8_t*>(s.A), static_cast<const uint8_t*>(s.B),
                           static_cast<const uint8_t*>(s.sfA), static_cast<const uint8_t*>(s.sfB), s.scale_a,
                           s.scale_b, s.C, out_dtype, M, ns, K, s.stream);
  }
}

}  // namespace
}  // namespace bw

using namespace bw;

extern "C" int bw_gemm_sharded(int dtype, int out_dtype, const bw_shard_t* shards, int ngpu, int M, int N, int K,
                               int gather) {
  int r = validate(dtype, out_dtype, shards, ngpu, M, N, K, gather);
  if (r != BW_OK) return r;
  int cur = 0;
  BW_CUDA(cudaGetDevice(&cur));
  const int ns = N / ngpu;
  const size_t elem = out_dtype == BW_OUT_F32 ? 4 : 2;
  // 1. the shards' GEMMs, each on its own device and stream (asynchronous)
  for (int i = 0; i < ngpu && r == BW_OK; ++i) {
    if (cudaSetDevice(shards[i].device) != cudaSuccess) {
      r = set_error(BW_ERR_CUDA, "cudaSetDevice(%d) failed", shards[i].device);
      break;
    }
    r = shard_gemm(dtype, out_dtype, shards[i], M, ns, K);
  }
  // 2. optional gather: all-gather into shard-major staging, then unshard into C_gathered
  if (r == BW_OK && gather && static_cast<long long>(M) * N > 0) {
    std::lock_guard<std::mutex> lk(g_shard_mu);
    if (ngpu == 1) {
      const bw_shard_t& s = shards[0];
      if (s.C_gathered != s.C && cudaSetDevice(s.device) == cudaSuccess &&
          cudaMemcpyAsync(s.C_gathered, s.C, elem * M * static_cast<size_t>(N), cudaMemcpyDeviceToDevice,
                          static_cast<cudaStream_t>(s.stream)) != cudaSuccess)
        r = set_error(BW_ERR_CUDA, "copy of the single shard failed");
    } else if ((r = load_nccl()) == BW_OK) {
      std::vector<int> devices(ngpu);
      for (int i = 0; i < ngpu; ++i) devices[i] = shards[i].device;
      const std::vector<ncclComm_t>* comms = nullptr;
      std::vector<void*> staging(ngpu, nullptr);
      r = comms_for(devices, &comms);
      for (int i = 0; i < ngpu && r == BW_OK; ++i) {
        if (cudaSetDevice(devices[i]) != cudaSuccess) r = set_error(BW_ERR_CUDA, "cudaSetDevice(%d)", devices[i]);
        else r = staging_for(devices[i], elem * M * static_cast<size_t>(N), &staging[i]);
      }
      if (r == BW_OK) {
        const ncclDataType_t dt = out_dtype == BW_OUT_F32 ? ncclFloat32 : ncclBfloat16;
        ncclResult_t nr = g_nccl.group_start();
        for (int i = 0; i < ngpu && nr == ncclSuccess; ++i)
          nr = g_nccl.all_gather(shards[i].C, staging[i], static_cast<size_t>(M) * ns, dt, (*comms)[i],
                                 static_cast<cudaStream_t>(shards[i].stream));
        const ncclResult_t ne = g_nccl.group_end();
        if (nr != ncclSuccess) r = nccl_error(nr, "ncclAllGather");
        else if (ne != ncclSuccess) r = nccl_error(ne, "ncclGroupEnd");
      }
      for (int i = 0; i < ngpu && r == BW_OK; ++i) {
        if (cudaSetDevice(devices[i]) != cudaSuccess) r = set_error(BW_ERR_CUDA, "cudaSetDevice(%d)", devices[i]);
        else r = unshard_elems(staging[i], shards[i].C_gathered, M, N, ngpu, static_cast<int>(elem),
                               static_cast<cudaStream_t>(shards[i].stream));
      }
    }
  }
  cudaSetDevice(cur);
  return r;
}
