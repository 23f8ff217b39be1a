// Device quantisers (the staging step in front of every GEMM) and small layout helpers.
//
// Element rules follow the reference bit for bit:
//   fp16: __float2half round-to-nearest-even            (src/gemm_mma.cu:147-150)
//   e4m3: __nv_fp8_e4m3(x), i.e. RNE with satfinite      (src/gemm_mma_fp8.cu:37-45)
//   e2m1: f32_to_e2m1, first strictly-nearest level of {0,.5,1,1.5,2,3,4,6} by fabsf
//         distance computed in fp32, sign bit iff v < 0   (src/gemm_mma_fp8.cu:47-58)
//   fp4 byte container: code << 2 (kind::f8f6f4 alignment) (src/gemm_mma_fp8.cu:61-68)
//   packed fp4: element 2i in the low nibble              (src/gemm_mma_fp8.cu:70-80)
// New behaviour (no reference counterpart): per-tensor amax scaling and UE8M0 block-32
// scales (e = floor(log2(block amax)) - 2).
#include <atomic>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "bw_e2m1.h"
#include "bw_runtime.cuh"

namespace bw {
namespace {

constexpr int kQThreads = 256;

__device__ __forceinline__ uint8_t e2m1_code(float v) { return bw_e2m1_code(v); }

__device__ __forceinline__ uint8_t e4m3_sat(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

// ---------------------------------------------------------------- fp16
__global__ void k_f32_to_f16(const float* __restrict__ src, __half* __restrict__ dst, long long n) {
  const long long n4 = n / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(src)[i];
    __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    uint2 o;
    o.x = *reinterpret_cast<uint32_t*>(&a);
    o.y = *reinterpret_cast<uint32_t*>(&b);
    reinterpret_cast<uint2*>(dst)[i] = o;
  }
  for (long long i = n4 * 4 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n; i += stride)
    dst[i] = __float2half_rn(src[i]);
}

// ---------------------------------------------------------------- amax
__global__ void k_amax(const float* __restrict__ src, long long n, unsigned* __restrict__ out) {
  float m = 0.f;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long t0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
    const long long n4 = n / 4;
    for (long long i = t0; i < n4; i += stride) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(src) + i);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
    }
    for (long long i = 4 * n4 + t0; i < n; i += stride) m = fmaxf(m, fabsf(src[i]));
  } else {
    for (long long i = t0; i < n; i += stride) m = fmaxf(m, fabsf(src[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float wm[kQThreads / 32];
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kQThreads / 32; ++w) m = fmaxf(m, wm[w]);
    atomicMax(out, __float_as_uint(m));  // non-negative floats order like their bits
  }
}

// Per-tensor multiplier and the scale handed to the GEMM epilogue.
//   NONE: q = cvt(x), s = 1. FIXED8: q = cvt(8x), s = 1/8. AMAX: q = cvt(x * (qmax/amax)),
//   s = amax/qmax (amax == 0 -> 1).
__device__ __forceinline__ void tensor_scale(int mode, const unsigned* amax_bits, float qmax, float& mul,
                                             float& s) {
  if (mode == BW_SCALE_FIXED8) { mul = 8.f; s = 0.125f; return; }
  if (mode == BW_SCALE_AMAX) {
    const float amax = __uint_as_float(*amax_bits);
    if (amax > 0.f && amax < INFINITY) { mul = qmax / amax; s = amax / qmax; return; }
  }
  mul = 1.f;
  s = 1.f;
}

// Quantise rows x cols fp32 into dst (rows x cols, or cols x rows when transposing).
// FMT 0 = e4m3 byte, 1 = e2m1 byte container (<<2), 2 = e2m1 packed pairs.
template <int FMT>
__device__ __forceinline__ uint8_t encode(float x) {
  if constexpr (FMT == 0) return e4m3_sat(x);
  else return e2m1_code(x);
}

template <int FMT>
__device__ __forceinline__ uint32_t encode_byte(float x) {
  const uint32_t c = encode<FMT>(x);
  return FMT == 1 ? (c << 2) : c;
}

// 16 consecutive values -> 16 code bytes (FMT 0/1) or 8 packed bytes (FMT 2).
template <int FMT>
__device__ __forceinline__ void encode16(const float (&v)[16], float mul, uint32_t (&w)[4]) {
  if constexpr (FMT == 2) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      w[q] = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) w[q] |= static_cast<uint32_t>(e2m1_code(v[8 * q + i] * mul)) << (4 * i);
    }
    w[2] = w[3] = 0;
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      w[q] = encode_byte<FMT>(v[4 * q] * mul) | (encode_byte<FMT>(v[4 * q + 1] * mul) << 8) |
             (encode_byte<FMT>(v[4 * q + 2] * mul) << 16) | (encode_byte<FMT>(v[4 * q + 3] * mul) << 24);
  }
}

// Row-major output: 16 elements per thread per step (four float4 loads, one 16- or 8-byte
// store) when src/dst alignment and n allow it; element-wise otherwise.
template <int FMT>
__global__ void k_quant_rowmajor(const float* __restrict__ src, uint8_t* __restrict__ dst, int rows, int cols,
                                 int mode, float qmax, const unsigned* amax_bits, float* scale_out) {
  float mul, s;
  tensor_scale(mode, amax_bits, qmax, mul, s);
  if (scale_out && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *scale_out = s;
  const long long n = static_cast<long long>(rows) * cols;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long t0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const bool vec = n % 16 == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(dst) & (FMT == 2 ? 7u : 15u)) == 0;
  if (vec) {
    for (long long i = t0; i < n / 16; i += stride) {
      float v[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 f = __ldcs(reinterpret_cast<const float4*>(src) + 4 * i + q);
        v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
      }
      uint32_t w[4];
      encode16<FMT>(v, mul, w);
      if constexpr (FMT == 2) reinterpret_cast<uint2*>(dst)[i] = make_uint2(w[0], w[1]);
      else reinterpret_cast<uint4*>(dst)[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    return;
  }
  if constexpr (FMT == 2) {
    const long long npairs = n / 2;  // cols is even: pairs never straddle rows
    for (long long i = t0; i < npairs; i += stride) {
      const float2 v = reinterpret_cast<const float2*>(src)[i];
      dst[i] = static_cast<uint8_t>(e2m1_code(v.x * mul) | (e2m1_code(v.y * mul) << 4));
    }
  } else {
    for (long long i = t0; i < n; i += stride) dst[i] = static_cast<uint8_t>(encode_byte<FMT>(src[i] * mul));
  }
}

// src rows x cols -> dst cols x rows. A CTA takes 128 src rows x 32 src columns: lane = column,
// warp w = rows r0 + 16w .. +15 (16 coalesced 128-byte row loads), so each thread ends with 16
// consecutive codes of one dst row and stores them as one 16-byte (8 packed bytes for FMT 2)
// store when rows % 16 == 0 and dst is aligned; byte stores otherwise.
constexpr int kQuantColsRows = 128;
inline unsigned transpose_grid_y(int rows) {
  const long long g = (static_cast<long long>(rows) + kQuantColsRows - 1) / kQuantColsRows;
  return static_cast<unsigned>(g < 65535 ? g : 65535);
}
template <int FMT>
__global__ void __launch_bounds__(256) k_quant_transpose(const float* __restrict__ src, uint8_t* __restrict__ dst,
                                                         int rows, int cols, int mode, float qmax,
                                                         const unsigned* amax_bits, float* scale_out) {
  float mul, s;
  tensor_scale(mode, amax_bits, qmax, mul, s);
  if (scale_out && blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *scale_out = s;
  const int c = blockIdx.x * 32 + (threadIdx.x & 31);
  if (c >= cols) return;
  const bool vec = rows % 16 == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
  // grid.y is capped at 65535: row groups beyond it are walked by a grid-stride loop
  for (long long rb = blockIdx.y; rb * kQuantColsRows < rows; rb += gridDim.y) {
    const int r0 = static_cast<int>(rb * kQuantColsRows) + 16 * (threadIdx.x >> 5);
    if (r0 >= rows) continue;
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = (r0 + i < rows) ? __ldcs(src + static_cast<size_t>(r0 + i) * cols + c) : 0.f;
    uint32_t w[4];
    encode16<FMT>(v, mul, w);
    if constexpr (FMT == 2) {
      uint8_t* row = dst + static_cast<size_t>(c) * (rows / 2);
      if (vec) {
        *reinterpret_cast<uint2*>(row + r0 / 2) = make_uint2(w[0], w[1]);
      } else {
        for (int i = 0; i < 16 && r0 + i < rows; i += 2)
          row[(r0 + i) / 2] = static_cast<uint8_t>(w[i / 8] >> (4 * (i % 8)));
      }
    } else {
      uint8_t* row = dst + static_cast<size_t>(c) * rows;
      if (vec) {
        *reinterpret_cast<uint4*>(row + r0) = make_uint4(w[0], w[1], w[2], w[3]);
      } else {
        for (int i = 0; i < 16 && r0 + i < rows; ++i) row[r0 + i] = static_cast<uint8_t>(w[i / 4] >> (8 * (i % 4)));
      }
    }
  }
}

// MXFP4 block scale: e = floor(log2(block amax)) - 2 read from the exponent field; zero and
// subnormal blocks clamp to e = -127 (byte 0). Returns the UE8M0 byte and the multiplier 2^-e.
__device__ __forceinline__ uint8_t mx_block_scale(float amax, int mode, float& mul) {
  if (mode != BW_MX_BLOCK32) {
    mul = 8.f;
    return 127;
  }
  const int biased = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFF);
  int e = (biased == 0) ? -127 : biased - 127 - 2;
  if (e < -127) e = -127;
  if (e > 127) e = 127;
  const int mexp = 127 - e;  // exponent field of 2^-e, in [0, 254]
  mul = (mexp >= 1) ? __uint_as_float(static_cast<uint32_t>(mexp) << 23) : 1.f;
  if (e == -127) mul = __uint_as_float(254u << 23);  // 2^127
  return static_cast<uint8_t>(e + 127);
}

__device__ __forceinline__ size_t sf_index(int o, int j, size_t kgroups) {
  const int r = o % 128;
  return ((static_cast<size_t>(o) / 128) * kgroups + j / 4) * 512 + (r % 32) * 16 + (r / 32) * 4 + (j % 4);
}

// MXFP4, K contiguous in src (outer x K row-major): one thread per 32-element block, eight
// float4 loads and one 16-byte store of its packed codes (a warp stores 512 contiguous bytes:
// the packed output is flat in the block index b = o * (K/32) + j). Measured faster than
// warp-cooperative forms that share a block across lanes (fewer instructions per element).
__global__ void __launch_bounds__(256) k_quant_mx_rows(const float4* __restrict__ src, uint4* __restrict__ dst,
                                                        uint8_t* __restrict__ sf, int nkb, int nblocks, int mode) {
  const unsigned kg = (static_cast<unsigned>(nkb) + 3u) / 4u;
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += gridDim.x * blockDim.x) {
    float4 x[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = __ldcs(src + static_cast<size_t>(b) * 8 + i);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(x[i].x), fabsf(x[i].y)), fmaxf(fabsf(x[i].z), fabsf(x[i].w))));
    float mul;
    const uint8_t byte = mx_block_scale(amax, mode, mul);
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 a = x[2 * q], c = x[2 * q + 1];
      w[q] = static_cast<uint32_t>(e2m1_code(a.x * mul)) | (static_cast<uint32_t>(e2m1_code(a.y * mul)) << 4) |
             (static_cast<uint32_t>(e2m1_code(a.z * mul)) << 8) | (static_cast<uint32_t>(e2m1_code(a.w * mul)) << 12) |
             (static_cast<uint32_t>(e2m1_code(c.x * mul)) << 16) | (static_cast<uint32_t>(e2m1_code(c.y * mul)) << 20) |
             (static_cast<uint32_t>(e2m1_code(c.z * mul)) << 24) | (static_cast<uint32_t>(e2m1_code(c.w * mul)) << 28);
    }
    dst[b] = make_uint4(w[0], w[1], w[2], w[3]);
    const unsigned o = static_cast<unsigned>(b) / static_cast<unsigned>(nkb);
    const unsigned j = static_cast<unsigned>(b) - o * static_cast<unsigned>(nkb);
    const unsigned r = o & 127u;
    sf[(static_cast<size_t>(o >> 7) * kg + (j >> 2)) * 512 + (r & 31u) * 16 + (r >> 5) * 4 + (j & 3u)] = byte;
  }
}

// MXFP4 from a K x outer source (the Bt operand built from row-major B): a CTA takes 32
// outer columns x 256 K. Warp w quantises K block w of the tile for 32 columns (lane = column,
// 32 coalesced 128-byte row loads), the packed blocks and scale bytes go through shared memory,
// and the tile leaves as 32 output rows x 128 contiguous bytes.
__global__ void __launch_bounds__(256) k_quant_mx_cols(const float* __restrict__ src, uint8_t* __restrict__ dst,
                                                       uint8_t* __restrict__ sf, int K, int outer, int mode) {
  __shared__ uint4 packed[32][9];  // [column][K block], padded
  __shared__ uint8_t scales[32][8];
  const int lane = threadIdx.x & 31, wk = threadIdx.x >> 5;
  const int o0 = blockIdx.x * 32, k0 = blockIdx.y * 256;
  const int nkb = K / 32;
  const int j = k0 / 32 + wk;  // this warp's K block
  const int o = o0 + lane;
  if (j < nkb && o < outer) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __ldg(src + static_cast<size_t>(j * 32 + i) * outer + o);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    float mul;
    scales[lane][wk] = mx_block_scale(amax, mode, mul);
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i / 8] |= static_cast<uint32_t>(e2m1_code(v[i] * mul)) << (4 * (i % 8));
    packed[lane][wk] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  __syncthreads();
  // 32 rows x 8 blocks of 16 bytes: thread t writes block t % 8 of row t / 8
  {
    const int r = threadIdx.x >> 3, c = threadIdx.x & 7;
    const int oo = o0 + r, jj = k0 / 32 + c;
    if (oo < outer && jj < nkb)
      *reinterpret_cast<uint4*>(dst + static_cast<size_t>(oo) * (K / 2) + static_cast<size_t>(jj) * 16) = packed[r][c];
  }
  // scale bytes: 4 consecutive K blocks of one row are one aligned 32-bit word of the layout
  if (threadIdx.x < 64) {
    const int r = threadIdx.x >> 1, g = threadIdx.x & 1;
    const int oo = o0 + r, jj = k0 / 32 + 4 * g;
    const size_t kg = (static_cast<size_t>(nkb) + 3) / 4;
    if (oo < outer && jj < nkb) {
      if (jj + 3 < nkb) {
        const uint32_t word = scales[r][4 * g] | (scales[r][4 * g + 1] << 8) | (scales[r][4 * g + 2] << 16) |
                              (static_cast<uint32_t>(scales[r][4 * g + 3]) << 24);
        *reinterpret_cast<uint32_t*>(sf + sf_index(oo, jj, kg)) = word;
      } else {
        for (int t = 0; t < 4 && jj + t < nkb; ++t) sf[sf_index(oo, jj + t, kg)] = scales[r][4 * g + t];
      }
    }
  }
}

template <typename T>
__global__ void k_unshard(const T* __restrict__ src, T* __restrict__ dst, int M, int N, int world) {
  const int ns = N / world;
  const long long total = static_cast<long long>(M) * N;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total; i += stride) {
    const long long m = i / N;
    const int c = static_cast<int>(i % N);
    const int r = c / ns, j = c % ns;
    dst[i] = src[(static_cast<long long>(r) * M + m) * ns + j];
  }
}

// Same permutation, 16 bytes per thread: blockIdx.y walks rows, x walks 16-byte column
// groups (a group never straddles two shards when a shard row is a multiple of 16 bytes).
template <typename T>
__global__ void k_unshard_vec(const T* __restrict__ src, T* __restrict__ dst, int M, int N, int world) {
  constexpr int V = 16 / sizeof(T);
  const int ns = N / world;
  const int groups = N / V;
  for (int m = blockIdx.y; m < M; m += gridDim.y) {
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < groups; j += gridDim.x * blockDim.x) {
      const int c = j * V;
      const int r = c / ns, cc = c - r * ns;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + (static_cast<size_t>(r) * M + m) * ns + cc));
      *reinterpret_cast<uint4*>(dst + static_cast<size_t>(m) * N + c) = v;
    }
  }
}

template <typename T>
int launch_unshard(const T* src, T* dst, int M, int N, int world, cudaStream_t s, const DeviceState& d);

int grid_for(long long n, const DeviceState& d) {
  long long g = (n + kQThreads - 1) / kQThreads;
  const long long cap = static_cast<long long>(d.sms) * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

template <typename T>
int launch_unshard(const T* src, T* dst, int M, int N, int world, cudaStream_t s, const DeviceState& d) {
  const int ns = N / world;
  const bool vec = (ns * sizeof(T)) % 16 == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0;
  if (vec) {
    const int groups = N / static_cast<int>(16 / sizeof(T));
    dim3 grid((groups + 255) / 256, M < 65535 ? M : 65535);
    k_unshard_vec<T><<<grid, 256, 0, s>>>(src, dst, M, N, world);
  } else {
    k_unshard<T><<<grid_for(static_cast<long long>(M) * N, d), kQThreads, 0, s>>>(src, dst, M, N, world);
  }
  BW_CUDA(cudaGetLastError());
  return BW_OK;
}

// Shared driver for the per-tensor quantisers (fp8 and fp4).
template <int FMT>
int quant_tensor(const float* src, uint8_t* dst, float* scale_out, int rows, int cols, int transpose, int mode,
                 float qmax, cudaStream_t s) {
  if (rows < 0 || cols < 0) return set_error(BW_ERR_INVALID, "negative size");
  if (mode != BW_SCALE_NONE && mode != BW_SCALE_FIXED8 && mode != BW_SCALE_AMAX)
    return set_error(BW_ERR_INVALID, "bad scale_mode %d", mode);
  const long long n = static_cast<long long>(rows) * cols;
  DeviceState* d;
  int r = ensure_device(&d);
  if (r != BW_OK) return r;
  if (n == 0) {
    if (scale_out) {
      const float one = 1.f;
      BW_CUDA(cudaMemcpyAsync(scale_out, &one, sizeof(float), cudaMemcpyHostToDevice, s));
    }
    return BW_OK;
  }
  if (!src || !dst) return set_error(BW_ERR_INVALID, "null src/dst");
  if (FMT == 2 && ((transpose ? rows : cols) % 2 != 0))
    return set_error(BW_ERR_INVALID, "packed fp4 needs an even contiguous dimension");
  if (FMT == 2 && !transpose && (reinterpret_cast<uintptr_t>(src) & 7u))
    return set_error(BW_ERR_INVALID, "packed fp4 source must be 8-byte aligned");
  unsigned* amax = static_cast<unsigned*>(d->workspace);
  if (mode == BW_SCALE_AMAX) {
    BW_CUDA(cudaMemsetAsync(amax, 0, sizeof(unsigned), s));
    k_amax<<<grid_for(n, *d), kQThreads, 0, s>>>(src, n, amax);
    BW_CUDA(cudaGetLastError());
  }
  if (transpose) {
    dim3 grid((cols + 31) / 32, transpose_grid_y(rows));
    k_quant_transpose<FMT><<<grid, 256, 0, s>>>(src, dst, rows, cols, mode, qmax, amax, scale_out);
  } else {
    k_quant_rowmajor<FMT><<<grid_for(FMT == 2 ? n / 2 : n, *d), kQThreads, 0, s>>>(src, dst, rows, cols, mode, qmax,
                                                                                  amax, scale_out);
  }
  BW_CUDA(cudaGetLastError());
  return BW_OK;
}

}  // namespace
}  // namespace bw

using namespace bw;

extern "C" {

int bw_quantize_f16(const float* src, void* dst, long long n, void* stream) {
  if (n < 0) return set_error(BW_ERR_INVALID, "negative n");
  if (n == 0) return BW_OK;
  if (!src || !dst) return set_error(BW_ERR_INVALID, "null src/dst");
  if (!aligned16(src) || (reinterpret_cast<uintptr_t>(dst) & 7u))
    return set_error(BW_ERR_INVALID, "src must be 16-byte and dst 8-byte aligned");
  DeviceState* d;
  int r = ensure_device(&d);
  if (r != BW_OK) return r;
  k_f32_to_f16<<<grid_for(n / 4 + 1, *d), kQThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      src, static_cast<__half*>(dst), n);
  BW_CUDA(cudaGetLastError());
  return BW_OK;
}

int bw_quantize_fp8(const float* src, uint8_t* dst, float* scale_out, int rows, int cols, int transpose,
                    int scale_mode, void* stream) {
  return quant_tensor<0>(src, dst, scale_out, rows, cols, transpose, scale_mode, 448.f,
                         static_cast<cudaStream_t>(stream));
}

int bw_quantize_fp4(const float* src, uint8_t* dst, float* scale_out, int rows, int cols, int transpose,
                    int scale_mode, int container, void* stream) {
  if (container == BW_FP4_PACKED)
    return quant_tensor<2>(src, dst, scale_out, rows, cols, transpose, scale_mode, 6.f,
                           static_cast<cudaStream_t>(stream));
  if (container == BW_FP4_BYTE_SHL2)
    return quant_tensor<1>(src, dst, scale_out, rows, cols, transpose, scale_mode, 6.f,
                           static_cast<cudaStream_t>(stream));
  return set_error(BW_ERR_INVALID, "bad fp4 container %d", container);
}

int bw_quantize_mxfp4(const float* src, uint8_t* dst, uint8_t* sf, int rows, int cols, int transpose, int mode,
                      void* stream) {
  if (rows < 0 || cols < 0) return set_error(BW_ERR_INVALID, "negative size");
  if (mode != BW_MX_UNIT_FIXED8 && mode != BW_MX_BLOCK32) return set_error(BW_ERR_INVALID, "bad mx mode %d", mode);
  const int K = transpose ? rows : cols;
  const int outer = transpose ? cols : rows;
  if (K % 32 != 0) return set_error(BW_ERR_INVALID, "mxfp4 needs K %% 32 == 0 (got %d)", K);
  if (static_cast<long long>(rows) * cols == 0) return BW_OK;
  if (!src || !dst || !sf) return set_error(BW_ERR_INVALID, "null src/dst/sf");
  if (!aligned16(src) || !aligned16(dst)) return set_error(BW_ERR_INVALID, "src and dst must be 16-byte aligned");
  DeviceState* d;
  int r = ensure_device(&d);
  if (r != BW_OK) return r;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  BW_CUDA(cudaMemsetAsync(sf, 0x7f, bw_sf_bytes(outer, K), s));
  if (transpose) {
    if ((K + 255) / 256 > 65535)
      return set_error(BW_ERR_INVALID, "mxfp4 transposed: K = %d exceeds the %d rows one launch covers", K, 65535 * 256);
    dim3 grid((outer + 31) / 32, (K + 255) / 256);
    k_quant_mx_cols<<<grid, 256, 0, s>>>(src, dst, sf, K, outer, mode);
  } else {
    const long long nblocks = static_cast<long long>(outer) * (K / 32);
    if (nblocks >= (1LL << 31) - 256) return set_error(BW_ERR_INVALID, "mxfp4: %lld blocks exceed the index range", nblocks);
    const long long ctas = (nblocks + 255) / 256;
    const long long cap = static_cast<long long>(d->sms) * 32;
    k_quant_mx_rows<<<static_cast<int>(ctas < cap ? ctas : cap), 256, 0, s>>>(
        reinterpret_cast<const float4*>(src), reinterpret_cast<uint4*>(dst), sf, K / 32, static_cast<int>(nblocks), mode);
  }
  BW_CUDA(cudaGetLastError());
  return BW_OK;
}

int bw_unshard_columns(const float* C_shardmajor, float* C_rowmajor, int M, int N, int world, void* stream) {
  if (M < 0 || N < 0 || world <= 0 || N % world != 0) return set_error(BW_ERR_INVALID, "bad unshard shape");
  if (static_cast<long long>(M) * N == 0) return BW_OK;
  if (!C_shardmajor || !C_rowmajor) return set_error(BW_ERR_INVALID, "null buffer");
  DeviceState* d;
  int r = ensure_device(&d);
  if (r != BW_OK) return r;
  return launch_unshard<float>(C_shardmajor, C_rowmajor, M, N, world, static_cast<cudaStream_t>(stream), *d);
}

int bw_unshard_columns_bf16(const void* C_shardmajor, void* C_rowmajor, int M, int N, int world, void* stream) {
  if (M < 0 || N < 0 || world <= 0 || N % world != 0) return set_error(BW_ERR_INVALID, "bad unshard shape");
  if (static_cast<long long>(M) * N == 0) return BW_OK;
  if (!C_shardmajor || !C_rowmajor) return set_error(BW_ERR_INVALID, "null buffer");
  return unshard_elems(C_shardmajor, C_rowmajor, M, N, world, 2, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace bw {
// [world][M][N/world] -> M x N for 4- or 2-byte elements (FP32 or BF16 C), on the current device.
int unshard_elems(const void* src, void* dst, int M, int N, int world, int elem_bytes, cudaStream_t stream) {
  if (elem_bytes == 4) return bw_unshard_columns(static_cast<const float*>(src), static_cast<float*>(dst), M, N, world, stream);
  if (elem_bytes != 2) return set_error(BW_ERR_INVALID, "unshard: element size %d", elem_bytes);
  if (M < 0 || N < 0 || world <= 0 || N % world != 0) return set_error(BW_ERR_INVALID, "bad unshard shape");
  if (static_cast<long long>(M) * N == 0) return BW_OK;
  DeviceState* d;
  int r = ensure_device(&d);
  if (r != BW_OK) return r;
  return launch_unshard<uint16_t>(static_cast<const uint16_t*>(src), static_cast<uint16_t*>(dst), M, N, world, stream, *d);
}
}  // namespace bw

// =========================================================================================
// bw_quantize_fp8_noalloc: the per-tensor E4M3 quantiser for callers that cannot allocate
// device memory. Some callers are not allowed to call cudaMalloc at all: plugins hosted by a
// framework whose own allocator has already reserved the device memory and must account for
// every byte, and serving loops with a no-allocation latency contract (a cudaMalloc can
// synchronise the device and take milliseconds). It still calls the CUDA runtime (kernel
// launches, and a symbol lookup on first use), so it must be called from an ordinary host
// thread, never from a host function or stream callback (CUDA forbids runtime calls there);
// a callback-driven design enqueues it from the thread that owns the stream. bw_quantize_fp8 needs a small device
// workspace for its amax reduction, which the library cudaMallocs on a device's first use;
// this variant keeps that scratch in a fixed array compiled into the library instead.
//
// Scratch: kNoAllocAmaxBlocks per-block maxima plus one result word, 64 KiB + 4 B in total,
// held by every device that loads the library until the process exits. One block reduces
// kNoAllocChunk input elements, so an input may hold at most
// kNoAllocAmaxBlocks * kNoAllocChunk = 134,217,728 elements; larger inputs are rejected with
// BW_ERR_INVALID before anything is launched. Every slot a call reads is written earlier in
// the same call, so nothing has to be cleared between calls. All calls on a device share the
// array: two calls whose kernels may overlap on the GPU (different streams without ordering)
// race on it and must be serialised by the caller.
//
// Set-up: the first call on each device looks up the array's device address with
// cudaGetSymbolAddress while that device is current (the array's name in host code is a host
// stand-in, not a device address). Make that first call outside any stream capture.
// Results are bit-identical to bw_quantize_fp8 (max is exact and order-independent).
// =========================================================================================
namespace bw {
namespace {

constexpr int kNoAllocAmaxBlocks = 16384;
constexpr int kNoAllocChunk = 8192;  // elements reduced by one block (32 per thread)
static __device__ __align__(256) unsigned g_noalloc_amax_scratch[kNoAllocAmaxBlocks + 1];

// Per-device cache of the set-up results. Two host threads making their first call on one
// device may both run the set-up; they store the same values, published with release order
// (the SM count before the address, so a thread that sees the address also sees the count).
std::atomic<void*> g_noalloc_scratch_addr[64] = {};
std::atomic<int> g_noalloc_sms[64] = {};

__global__ void k_amax_partial(const float* __restrict__ src, long long n, unsigned* __restrict__ partial) {
  const long long base = static_cast<long long>(blockIdx.x) * kNoAllocChunk;
  float m = 0.f;
  for (int i = threadIdx.x; i < kNoAllocChunk; i += kQThreads) {
    const long long j = base + i;
    if (j < n) m = fmaxf(m, fabsf(src[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float wm[kQThreads / 32];
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kQThreads / 32; ++w) m = fmaxf(m, wm[w]);
    partial[blockIdx.x] = __float_as_uint(m);
  }
}

__global__ void k_amax_final(const unsigned* __restrict__ partial, int nblocks, unsigned* __restrict__ out) {
  float m = 0.f;
  for (int i = threadIdx.x; i < nblocks; i += kQThreads) m = fmaxf(m, __uint_as_float(partial[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float wm[kQThreads / 32];
  if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kQThreads / 32; ++w) m = fmaxf(m, wm[w]);
    *out = __float_as_uint(m);
  }
}

__global__ void k_store_one(float* out) { *out = 1.f; }

// Once per device, with that device current: device address of the scratch array and the SM
// count (neither call allocates).
int noalloc_setup(int dev, unsigned** scratch, int* sms) {
  if (dev < 0 || dev >= 64) return set_error(BW_ERR_INVALID, "device index %d out of range", dev);
  void* addr = g_noalloc_scratch_addr[dev].load(std::memory_order_acquire);
  if (!addr) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_amax_scratch);
    if (e != cudaSuccess || !ptr) return cuda_error(e, "cudaGetSymbolAddress(no-alloc scratch)");
    int n = 0;
    BW_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    g_noalloc_sms[dev].store(n > 0 ? n : 1, std::memory_order_relaxed);
    g_noalloc_scratch_addr[dev].store(ptr, std::memory_order_release);
    addr = ptr;
  }
  *scratch = static_cast<unsigned*>(addr);
  *sms = g_noalloc_sms[dev].load(std::memory_order_relaxed);
  return BW_OK;
}

}  // namespace
}  // namespace bw

extern "C" int bw_quantize_fp8_noalloc(const float* src, uint8_t* dst, float* scale_out, int rows, int cols,
                                       int transpose, int scale_mode, void* stream) {
  using namespace bw;
  if (rows < 0 || cols < 0) return set_error(BW_ERR_INVALID, "negative size");
  if (scale_mode != BW_SCALE_NONE && scale_mode != BW_SCALE_FIXED8 && scale_mode != BW_SCALE_AMAX)
    return set_error(BW_ERR_INVALID, "bad scale_mode %d", scale_mode);
  const long long n = static_cast<long long>(rows) * cols;
  const long long limit = static_cast<long long>(kNoAllocAmaxBlocks) * kNoAllocChunk;
  if (n > limit)
    return set_error(BW_ERR_INVALID,
                     "bw_quantize_fp8_noalloc: %lld elements exceed its fixed scratch limit of %lld elements "
                     "(use bw_quantize_fp8)",
                     n, limit);
  if (n > 0 && (!src || !dst)) return set_error(BW_ERR_INVALID, "null src/dst");
  int dev = 0;
  BW_CUDA(cudaGetDevice(&dev));
  unsigned* scratch = nullptr;
  int sms = 1;
  int r = noalloc_setup(dev, &scratch, &sms);
  if (r != BW_OK) return r;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned* amax = scratch + kNoAllocAmaxBlocks;  // result word, written before it is read
  if (n == 0) {
    if (scale_out) {
      k_store_one<<<1, 1, 0, s>>>(scale_out);
      BW_CUDA(cudaGetLastError());
    }
    return BW_OK;
  }
  if (scale_mode == BW_SCALE_AMAX) {
    const int nblocks = static_cast<int>((n + kNoAllocChunk - 1) / kNoAllocChunk);
    k_amax_partial<<<nblocks, kQThreads, 0, s>>>(src, n, scratch);
    BW_CUDA(cudaGetLastError());
    k_amax_final<<<1, kQThreads, 0, s>>>(scratch, nblocks, amax);
    BW_CUDA(cudaGetLastError());
  }
  if (transpose) {
    dim3 grid((cols + 31) / 32, transpose_grid_y(rows));
    k_quant_transpose<0><<<grid, 256, 0, s>>>(src, dst, rows, cols, scale_mode, 448.f, amax, scale_out);
  } else {
    long long g = (n + kQThreads - 1) / kQThreads;
    if (g > static_cast<long long>(sms) * 16) g = static_cast<long long>(sms) * 16;
    k_quant_rowmajor<0><<<static_cast<int>(g), kQThreads, 0, s>>>(src, dst, rows, cols, scale_mode, 448.f, amax,
                                                                   scale_out);
  }
  BW_CUDA(cudaGetLastError());
  return BW_OK;
}
