/* bwgemm.h - C ABI of the B200 (sm_100a) tensor-core GEMM library.
 *
 * Every entry point returns an int status (BW_OK on success) instead of the reference's
 * CUDA_CHECK-then-exit(1) (include/util.cuh:7-8); bw_last_error_string() describes the
 * last failure on the calling thread. Pointers are plain device pointers, sizes are
 * plain ints, streams are passed as void* (a cudaStream_t; NULL = legacy default stream).
 * No call allocates per invocation; quantisers with a per-tensor scale use a small
 * library-owned device workspace created on first use of each device.
 *
 * Reference interfaces these replace (paths within waynehacking8/blackwell-tensorcore-kernels):
 *   launch_<name>(const float* A, const float* B, float* C, int M, int N, int K)
 *       src/main.cu:18-39 - FP32 device buffers; each launcher stages (casts/quantises)
 *       its inputs and then runs one kernel. The C++ wrappers with that exact signature
 *       live in csrc/bw_launchers.cu and call the functions below.
 *   gemm_mma_t / gemm_wmma_t  (src/gemm_mma.cu:23-141, src/gemm_wmma.cu:29-104)
 *       -> bw_gemm_f16
 *   gemm_lowprec_t<FP8|FP4|MXFP4> (src/gemm_mma_fp8.cu:89-223)
 *       -> bw_gemm_fp8, bw_gemm_fp4, bw_gemm_mxfp4
 *   f2h / f2h_mma (src/gemm_wmma.cu:106-108, src/gemm_mma.cu:147-150) -> bw_quantize_f16
 *   q_fp8 / q_fp8_t (src/gemm_mma_fp8.cu:37-45)                      -> bw_quantize_fp8
 *   q_fp4 / q_fp4_t (src/gemm_mma_fp8.cu:61-68)                      -> bw_quantize_fp4
 *   q_mxfp4 / q_mxfp4_t (src/gemm_mma_fp8.cu:70-80)                  -> bw_quantize_mxfp4
 */
#ifndef BWGEMM_H
#define BWGEMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum bw_status {
  BW_OK = 0,
  BW_ERR_INVALID = 1,     /* bad argument: null pointer, negative/unsupported size, misalignment */
  BW_ERR_CUDA = 2,        /* a CUDA runtime/driver call failed */
  BW_ERR_TIMEOUT = 3,     /* a kernel's bounded wait ran out (see bw_device_status) */
  BW_ERR_UNSUPPORTED = 4  /* device is not sm_100 or feature not built */
};

/* Output element type for the low-precision GEMMs. */
enum bw_out_dtype { BW_OUT_F32 = 0, BW_OUT_BF16 = 1 };

/* Per-tensor scale policy for the quantisers.
 *   BW_SCALE_NONE  : no scaling (reference q_fp8: __nv_fp8_e4m3(x), src/gemm_mma_fp8.cu:37-40)
 *   BW_SCALE_FIXED8: the reference FP4/MXFP4 staging, x * 8 (src/gemm_mma_fp8.cu:228)
 *   BW_SCALE_AMAX  : s = amax/448 (E4M3) or amax/6 (E2M1); q = cvt(x * (448/amax));
 *                    s is written to *scale_out so the GEMM epilogue multiplies it back. */
enum bw_scale_mode { BW_SCALE_NONE = 0, BW_SCALE_FIXED8 = 1, BW_SCALE_AMAX = 2 };

/* FP4 storage: packed two per byte (even k in the low nibble, as q_mxfp4), or the
 * reference's kind::f8f6f4 byte container (code << 2, one per byte, as q_fp4). */
enum bw_fp4_container { BW_FP4_PACKED = 0, BW_FP4_BYTE_SHL2 = 1 };

/* MXFP4 block-scale policy. */
enum bw_mx_mode {
  BW_MX_UNIT_FIXED8 = 0, /* reference: x*8, every UE8M0 scale = 0x7f (include/mma_ptx.cuh:146-148) */
  BW_MX_BLOCK32 = 1      /* e = floor(log2(amax of 32 K-contiguous values)) - 2; byte = e + 127 */
};

/* ---------------- runtime ---------------- */
int bw_init(int device);              /* select device, load driver entry points, query SMs */
int bw_shutdown(void);                /* free library-owned device memory on all devices */
const char* bw_last_error_string(void);
int bw_version(void);                 /* (major << 16) | minor */
int bw_num_sms(int device);
/* Diagnostic: 1 when the library has set up its state on `device` (status word and the
 * small workspace it cudaMallocs on a device's first use), else 0; allocates nothing and
 * makes no CUDA call. */
int bw_device_state_ready(int device);
/* Reads (after synchronising `stream`) and clears the device status word that kernels
 * set when a bounded wait expires: 0 = ok, else (BW_ERR_TIMEOUT << 8) | site. */
int bw_device_status(void* stream, int* out_status);
/* Arms (dev_buf != NULL) or disarms the wait-time trace: every later CTA-pair GEMM launch
 * with at most max_ctas CTAs writes 8 unsigned long long per CTA into dev_buf (device
 * memory owned by the caller): [0] kernel cycles, [1] MMA-thread cycles waiting for loaded
 * k-slabs, [2] MMA-thread cycles waiting for a free accumulator, [3] producer cycles
 * waiting for free slabs, [4] epilogue cycles waiting for a finished accumulator,
 * [5] epilogue busy cycles, [6] tiles, [7] k-slabs. Diagnostic; no reference counterpart. */
int bw_set_trace_buffer(unsigned long long* dev_buf, int max_ctas);
/* Failure-detection self-test (no reference counterpart: the reference exits on errors).
 * Launches one CTA that waits on an mbarrier nothing arrives at, through the same bounded
 * wait as the GEMM kernels; returns BW_ERR_TIMEOUT after about budget_ns with the device
 * status word cleared again, leaving the context usable. */
int bw_selftest_bounded_wait(unsigned long long budget_ns, void* stream);
/* Overrides the per-wait budget of every kernel (nanoseconds; default 2e9). */
int bw_set_wait_budget_ns(unsigned long long ns);

/* ---------------- GEMMs (C row-major, ldc = N) ---------------- */
/* C[M,N] (fp32) = A[M,K] (fp16, row-major) x B[K,N] (fp16, row-major).
 * Requires K % 8 == 0 and N % 8 == 0 (16-byte TMA row strides), 16-byte aligned pointers.
 * Replaces gemm_mma_t<128,128,32,64,64,2,1,1> (src/gemm_mma.cu:219-226). */
int bw_gemm_f16(const void* A, const void* B, float* C, int M, int N, int K, void* stream);

/* Same, with B given transposed (Bt[N,K] row-major, K-contiguous). */
int bw_gemm_f16_bt(const void* A, const void* Bt, float* C, int M, int N, int K, void* stream);

/* C[M,N] = (sum_k A[m,k] * Bt[n,k]) * scale_a * scale_b, E4M3 inputs, FP32 accumulate.
 * scale_a / scale_b are device pointers to one float each (NULL = 1.0).
 * out_dtype BW_OUT_F32 (reference, src/gemm_mma_fp8.cu:217-221) or BW_OUT_BF16.
 * Requires K % 16 == 0. */
int bw_gemm_fp8(const uint8_t* A, const uint8_t* Bt, const float* scale_a, const float* scale_b, void* C,
                int out_dtype, int M, int N, int K, void* stream);

/* Block-scaled packed E2M1: A[M,K/2], Bt[N,K/2] packed bytes; sfA / sfB UE8M0 in the 128x4
 * tiled layout (bw_sf_bytes / bw_sf_offset). Optional per-tensor scales as in bw_gemm_fp8.
 * Requires K % 32 == 0. */
int bw_gemm_mxfp4(const uint8_t* A, const uint8_t* Bt, const uint8_t* sfA, const uint8_t* sfB,
                  const float* scale_a, const float* scale_b, void* C, int out_dtype, int M, int N, int K,
                  void* stream);

/* Plain FP4 (E2M1, packed) with per-tensor scales only; every block scale is 2^0.
 * Replaces gemm_lowprec_t<FP4> (src/gemm_mma_fp8.cu:305-310), whose epilogue multiplies by
 * 1/64 (src/gemm_mma_fp8.cu:208): pass scale_a = scale_b = 1/8 for that behaviour.
 * Requires K % 32 == 0. */
int bw_gemm_fp4(const uint8_t* A, const uint8_t* Bt, const float* scale_a, const float* scale_b, void* C,
                int out_dtype, int M, int N, int K, void* stream);

/* ---------------- quantisers (device, src/dst device pointers) ---------------- */
/* fp32 -> fp16 round-to-nearest-even, n elements. */
int bw_quantize_f16(const float* src, void* dst, long long n, void* stream);
/* src is rows x cols fp32 row-major. transpose = 0: dst rows x cols; transpose = 1:
 * dst cols x rows (the reference's B -> Bt staging). E4M3 with satfinite. */
int bw_quantize_fp8(const float* src, uint8_t* dst, float* scale_out, int rows, int cols, int transpose,
                    int scale_mode, void* stream);
/* E2M1 by the reference rule (nearest level, ties to the smaller magnitude, > 6 -> 6,
 * NaN -> +0). Packed containers pair values along the contiguous dimension of dst. */
int bw_quantize_fp4(const float* src, uint8_t* dst, float* scale_out, int rows, int cols, int transpose,
                    int scale_mode, int container, void* stream);
/* bw_quantize_fp8 for callers that cannot allocate device memory (no counterpart in the
 * reference). Framework-hosted plugins may find the device memory already reserved by the
 * host's own allocator, and latency-bound serving loops may forbid allocation; bw_quantize_fp8 needs a small library-allocated
 * workspace for its amax reduction, this variant uses a fixed scratch array compiled into the
 * library (64 KiB per device, held until exit) and calls no allocating routine. Same
 * arguments and bit-identical results. Limit: rows * cols <= 134,217,728 elements, larger
 * inputs return BW_ERR_INVALID. The first call on each device looks the array up (make it
 * outside any stream capture). Calls share the array: calls that may overlap on the GPU
 * (unordered streams) race and must be serialised by the caller. It launches kernels, so call
 * it from an ordinary host thread, not from a host function / stream callback (CUDA forbids
 * runtime calls there). */
int bw_quantize_fp8_noalloc(const float* src, uint8_t* dst, float* scale_out, int rows, int cols, int transpose,
                            int scale_mode, void* stream);
/* Packed E2M1 plus UE8M0 scale factors along the contiguous (K) dimension of dst.
 * dst is (transpose ? cols : rows) x (K/2) where K = (transpose ? rows : cols); sf receives
 * bw_sf_bytes(outer, K) bytes in the tiled layout. */
int bw_quantize_mxfp4(const float* src, uint8_t* dst, uint8_t* sf, int rows, int cols, int transpose, int mode,
                      void* stream);

/* Tiled scale-factor layout (same as cuBLASLt VEC32_UE8M0): 128-row x 4-block atoms of
 * 512 B, atoms ordered K-group-fastest; within an atom row r, block j sits at
 * (r % 32) * 16 + (r / 32) * 4 + j. */
size_t bw_sf_bytes(int outer, int K);
size_t bw_sf_offset(int row, int kblock, int K);

/* ---------------- N-sharded multi-GPU GEMM helpers ---------------- */
/* Column sharding (one process per GPU) needs no new GEMM: rank r calls bw_gemm_* on its
 * shard B[:, r*N/world:(r+1)*N/world]. When a gathered C is requested, the host layer
 * all-gathers the M x (N/world) shards over NCCL, which yields a shard-major buffer
 * [world][M][N/world]; this permutes it into row-major M x N. */
int bw_unshard_columns(const float* C_shardmajor, float* C_rowmajor, int M, int N, int world, void* stream);
/* The same permutation for 2-byte elements (BF16 C). */
int bw_unshard_columns_bf16(const void* C_shardmajor, void* C_rowmajor, int M, int N, int world, void* stream);

/* Fused all-gather (one process per GPU). Every rank holds a row-major M x N_total C_full and the
 * peers' C_full opened through CUDA IPC (bw_ipc_*); rank r computes columns
 * [r*N_total/world, (r+1)*N_total/world) from its B shard, and its epilogue sends every staged
 * 32-row chunk of the result out through TMA stores to its own C_full and to each peer's, so
 * the NVLink transfer overlaps the math tile by tile. When all ranks' calls have completed (the
 * caller synchronises, then barriers across ranks) every C_full holds the whole product: no
 * separate collective, no unshard pass. peer_C_full[q] is rank q's buffer as mapped here (entry
 * [rank] is ignored). Needs 16-byte aligned buffers, column offset and row pitch. The per-rank
 * math is bw_gemm_f16 / bw_gemm_fp8 (B_shard: K x N_total/world FP16; Bt_shard: N_total/world x K). */
int bw_gemm_f16_allgather(const void* A, const void* B_shard, float* C_full, void* const* peer_C_full, int world,
                          int rank, int M, int N_total, int K, void* stream);
int bw_gemm_fp8_allgather(const uint8_t* A, const uint8_t* Bt_shard, const float* scale_a, const float* scale_b,
                          void* C_full, int out_dtype, void* const* peer_C_full, int world, int rank, int M,
                          int N_total, int K, void* stream);

/* Fused all-gather through NVSwitch multicast (one process per GPU, 1..8 ranks). C_multicast is
 * the multicast address of a row-major M x N_total buffer that every rank has bound to one
 * NVLink multicast object (e.g. torch symmetric memory's multicast_ptr); rank r computes columns
 * [r*N_total/world, (r+1)*N_total/world) and its epilogue writes each staged 32-row chunk once
 * with multimem.st, which NVSwitch replicates into every rank's buffer: one copy of the shard
 * leaves each GPU instead of world - 1. Completion as for bw_gemm_f16_allgather (synchronise,
 * then barrier across ranks). BW_MC_PLAIN=1 writes with plain stores instead, for checking the
 * indexing on one GPU with an ordinary buffer. No counterpart in the reference (single GPU). */
int bw_gemm_f16_allgather_multicast(const void* A, const void* B_shard, void* C_multicast, int world, int rank,
                                    int M, int N_total, int K, void* stream);
int bw_gemm_fp8_allgather_multicast(const uint8_t* A, const uint8_t* Bt_shard, const float* scale_a,
                                    const float* scale_b, void* C_multicast, int out_dtype, int world, int rank,
                                    int M, int N_total, int K, void* stream);

/* Device buffers shareable across processes (CUDA IPC, 64-byte handles): bw_ipc_malloc returns
 * the buffer (256-byte aligned) and its handle; another process maps it with bw_ipc_open. */
enum { BW_IPC_HANDLE_BYTES = 64 };
int bw_ipc_malloc(size_t bytes, void** ptr, void* handle_out);
int bw_ipc_free(void* ptr);
int bw_ipc_open(const void* handle, void** peer_ptr);
int bw_ipc_close(void* peer_ptr);

/* One process driving g GPUs of a node (the single-process form of the sharded run).
 * Shard r lives on `device` and holds the full A plus columns [r*N/g, (r+1)*N/g) of B in the
 * layout the dtype's single-GPU entry point takes:
 *   BW_DTYPE_F16    A M x K FP16, B K x (N/g) FP16 row-major; C FP32 (out_dtype BW_OUT_F32)
 *   BW_DTYPE_FP8    A M x K E4M3, Bt (N/g) x K E4M3, optional device scales; C FP32 or BF16
 *   BW_DTYPE_FP4    A, Bt packed E2M1 (K/2 bytes a row), optional device scales
 *   BW_DTYPE_MXFP4  as FP4 plus the tiled UE8M0 scale factors of A and of the Bt shard
 * C (M x N/g) is written on each device. With gather != 0 every C_gathered (M x N, row-major,
 * on its shard's device) receives the whole product: an NCCL all-gather of the shards
 * (ncclCommInitAll over the listed devices, cached; libnccl.so.2 is loaded on first use)
 * followed by a column unshard. Work is enqueued on each shard's stream; the call does not
 * synchronise. Replaces nothing in the reference (it runs on one GPU, src/main.cu:47-111).
 * Returns BW_ERR_INVALID for bad arguments before touching any device, BW_ERR_UNSUPPORTED when
 * a gather is requested and NCCL cannot be loaded. */
enum { BW_DTYPE_F16 = 0, BW_DTYPE_FP8 = 1, BW_DTYPE_FP4 = 2, BW_DTYPE_MXFP4 = 3 };
typedef struct {
  int device;
  const void* A;
  const void* B;
  const void* sfA;
  const void* sfB;
  const float* scale_a;
  const float* scale_b;
  void* C;
  void* C_gathered;
  void* stream;
} bw_shard_t;
int bw_gemm_sharded(int dtype, int out_dtype, const bw_shard_t* shards, int ngpu, int M, int N, int K, int gather);

#ifdef __cplusplus
}
#endif

#endif /* BWGEMM_H */
