/* bw_oracle.c - CPU restatement of the reference's GEMM path. TEST INFRASTRUCTURE ONLY:
 * used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the checker,
 * never by the library.
 *
 * What it restates (paths within waynehacking8/blackwell-tensorcore-kernels):
 *   fill_rand           include/util.cuh:17   rand()/RAND_MAX - 0.5 from glibc's default seed
 *   f2h (fp32->fp16)    src/gemm_wmma.cu:106  __float2half: round to nearest even
 *   q_fp8 / q_fp8_t     src/gemm_mma_fp8.cu:37-45   __nv_fp8_e4m3(x): RNE, satfinite (+-448)
 *   f32_to_e2m1         src/gemm_mma_fp8.cu:47-58   first strictly-nearest E2M1 level by
 *                                                   fp32 fabsf distance; sign bit iff v < 0
 *   q_fp4 / q_fp4_t     src/gemm_mma_fp8.cu:61-68   code << 2, one per byte, x * 8
 *   q_mxfp4 / _t        src/gemm_mma_fp8.cu:70-80   packed, even k in the low nibble, x * 8
 *   epilogue unscale    src/gemm_mma_fp8.cu:208     FP4/MXFP4 results * 1/64
 *   the GEMM itself     src/gemm_mma.cu:23-141      C = A x B, A MxK, B KxN row-major
 * The GEMM is accumulated in FP64 over the (exactly representable) dequantised inputs,
 * which is the correctness anchor the north star names. The reference's own check
 * (src/main.cu:57-59) compares against cublasSgemm on the unquantised inputs; the
 * reference-compat tests reproduce its committed max_abs_err column that way.
 *
 * The fp16 and e4m3 conversions are written here from the IEEE-754 / OCP FP8 definitions
 * and are pinned against CUDA's host conversion functions by oracle/pin_conversions.cpp.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ inputs */
void or_srand(unsigned seed) { srand(seed); }

/* include/util.cuh:17 - p[i] = rand()/(float)RAND_MAX - 0.5f, in call order. */
void or_ref_fill_rand(float* p, long n) {
  for (long i = 0; i < n; ++i) p[i] = (rand() / (float)RAND_MAX) - 0.5f;
}

/* ------------------------------------------------------------------ fp16 */
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t or_f32_to_f16(float f) {
  const uint32_t x = f2u(f);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u); /* NaN / Inf */
  const int exp = (int)(ax >> 23) - 127;
  if (exp > 15) return sign | 0x7c00u;                                          /* overflow */
  if (exp >= -14) {                                                             /* normal */
    uint32_t mant = ax & 0x7fffffu;
    uint32_t h = ((uint32_t)(exp + 15) << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1; /* may carry into Inf: correct */
    return sign | (uint16_t)h;
  }
  /* subnormal half: value = m * 2^-24 */
  if (exp < -25) return sign;
  const uint32_t mant = (ax & 0x7fffffu) | 0x800000u; /* 1.m * 2^23 */
  const int shift = -exp - 1;                          /* 24 - (exp + 24) - ... : bits to drop */
  /* value = mant * 2^(exp-23); in units of 2^-24: mant * 2^(exp+1) -> drop (-(exp+1)) bits */
  const int drop = shift;
  uint32_t h = mant >> (drop);
  const uint32_t rem = mant & ((1u << drop) - 1u);
  const uint32_t half = 1u << (drop - 1);
  if (rem > half || (rem == half && (h & 1u))) h += 1;
  return sign | (uint16_t)h;
}

float or_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const int e = (h >> 10) & 0x1f;
  const uint32_t m = h & 0x3ffu;
  if (e == 0x1f) return u2f(sign | 0x7f800000u | (m << 13));
  if (e == 0) {
    float v = (float)m * (1.0f / 16777216.0f);
    return sign ? -v : v;
  }
  return u2f(sign | ((uint32_t)(e - 15 + 127) << 23) | (m << 13));
}

/* ------------------------------------------------------------------ e4m3 (OCP, fn) */
/* Finite range +-448, no infinities, 0x7f/0xff = NaN. Saturating, round-nearest-even. */
uint8_t or_f32_to_e4m3_sat(float f) {
  const uint32_t x = f2u(f);
  const uint8_t sign = (uint8_t)((x >> 24) & 0x80u);
  const uint32_t ax = x & 0x7fffffffu;
  if (ax > 0x7f800000u) return 0x7f; /* NaN -> canonical NaN */
  if (ax >= 0x43e00000u) return sign | 0x7e; /* >= 448 (incl. Inf) saturates to 448 */
  const int exp = (int)(ax >> 23) - 127;
  if (exp >= -6) { /* normal e4m3: exponent field exp+7 in [1,15] */
    const uint32_t mant = ax & 0x7fffffu;
    uint32_t q = ((uint32_t)(exp + 7) << 3) | (mant >> 20);
    const uint32_t rem = mant & 0xfffffu;
    if (rem > 0x80000u || (rem == 0x80000u && (q & 1u))) q += 1;
    if (q > 0x7e) q = 0x7e; /* rounding past 448 (480 boundary is not reachable below 464) */
    return sign | (uint8_t)q;
  }
  /* subnormal: units of 2^-9 */
  if (exp < -11) {
    /* values below 2^-10 (half of the smallest subnormal) round to 0; exactly 2^-10 -> 0 (even) */
    return sign;
  }
  const uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
  const int drop = 23 - (exp + 9); /* value = mant * 2^(exp-23) = q * 2^-9 */
  uint32_t q = mant >> drop;
  const uint32_t rem = mant & ((1u << drop) - 1u);
  const uint32_t half = 1u << (drop - 1);
  if (rem > half || (rem == half && (q & 1u))) q += 1;
  return sign | (uint8_t)q; /* q == 8 carries into the smallest normal, which is correct */
}

float or_e4m3_to_f32(uint8_t c) {
  const int s = c & 0x80, e = (c >> 3) & 0xf, m = c & 7;
  float v;
  if (e == 0xf && m == 7) return NAN;
  if (e == 0) v = (float)m * (1.0f / 512.0f);
  else v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return s ? -v : v;
}

/* ------------------------------------------------------------------ e2m1 */
/* src/gemm_mma_fp8.cu:47-58, restated: distances are fp32 fabsf(a - level), the first
 * strictly smaller distance wins (ties keep the smaller level, NaN and huge |v| whose
 * distances all round to |v| keep level 0), sign bit set iff v < 0. */
uint8_t or_e2m1_code(float v) {
  static const float lv[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float a = fabsf(v);
  int best = 0;
  float bd = fabsf(a - lv[0]);
  for (int i = 1; i < 8; ++i) {
    const float d = fabsf(a - lv[i]);
    if (d < bd) { bd = d; best = i; }
  }
  return (uint8_t)((v < 0.f ? 8 : 0) | best);
}

float or_e2m1_to_f32(uint8_t code) {
  static const float lv[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float v = lv[code & 7];
  return (code & 8) ? -v : v;
}

/* ------------------------------------------------------------------ per-tensor scales */
/* Mirrors the library's policy: NONE mul=1 s=1; FIXED8 mul=8 s=1/8;
 * AMAX mul = qmax/amax, s = amax/qmax (fp32 division), amax==0 or non-finite -> 1. */
enum { OR_SCALE_NONE = 0, OR_SCALE_FIXED8 = 1, OR_SCALE_AMAX = 2 };

static float amax_of(const float* src, long n) {
  float m = 0.f;
  for (long i = 0; i < n; ++i) {
    const float a = fabsf(src[i]);
    if (a > m) m = a; /* NaN never compares greater: ignored, like fmaxf */
  }
  return m;
}

static void tensor_scale(int mode, const float* src, long n, float qmax, float* mul, float* s) {
  if (mode == OR_SCALE_FIXED8) { *mul = 8.f; *s = 0.125f; return; }
  if (mode == OR_SCALE_AMAX) {
    const float amax = amax_of(src, n);
    if (amax > 0.f && amax < INFINITY) { *mul = qmax / amax; *s = amax / qmax; return; }
  }
  *mul = 1.f;
  *s = 1.f;
}

/* Quantise rows x cols (row-major) to e4m3; transpose=1 writes cols x rows. */
void or_quant_fp8(const float* src, uint8_t* dst, float* scale_out, int rows, int cols, int transpose, int mode) {
  float mul, s;
  tensor_scale(mode, src, (long)rows * cols, 448.f, &mul, &s);
  if (scale_out) *scale_out = s;
  for (long r = 0; r < rows; ++r)
    for (long c = 0; c < cols; ++c) {
      const uint8_t q = or_f32_to_e4m3_sat(src[r * cols + c] * mul);
      if (transpose) dst[c * rows + r] = q;
      else dst[r * cols + c] = q;
    }
}

/* container 0 = packed pairs along the contiguous dim of dst; 1 = code << 2 per byte. */
void or_quant_fp4(const float* src, uint8_t* dst, float* scale_out, int rows, int cols, int transpose, int mode,
                  int container) {
  float mul, s;
  tensor_scale(mode, src, (long)rows * cols, 6.f, &mul, &s);
  if (scale_out) *scale_out = s;
  const long orows = transpose ? cols : rows, ocols = transpose ? rows : cols;
  if (container == 1) {
    for (long r = 0; r < orows; ++r)
      for (long c = 0; c < ocols; ++c) {
        const float x = transpose ? src[c * cols + r] : src[r * cols + c];
        dst[r * ocols + c] = (uint8_t)(or_e2m1_code(x * mul) << 2);
      }
  } else {
    for (long r = 0; r < orows; ++r)
      for (long c = 0; c < ocols; c += 2) {
        const float x0 = transpose ? src[c * cols + r] : src[r * cols + c];
        const float x1 = transpose ? src[(c + 1) * cols + r] : src[r * cols + c + 1];
        dst[r * (ocols / 2) + c / 2] = (uint8_t)(or_e2m1_code(x0 * mul) | (or_e2m1_code(x1 * mul) << 4));
      }
  }
}

/* Tiled UE8M0 layout: 128-row x 4-block atoms of 512 B, K-group fastest. */
long or_sf_bytes(int outer, int K) {
  const long rb = (outer + 127) / 128, kg = ((K + 31) / 32 + 3) / 4;
  return rb * kg * 512;
}
long or_sf_offset(int row, int kblock, int K) {
  const long kg = ((K + 31) / 32 + 3) / 4;
  const int r = row % 128;
  return ((long)(row / 128) * kg + kblock / 4) * 512 + (r % 32) * 16 + (r / 32) * 4 + (kblock % 4);
}

/* MXFP4: mode 0 = reference (x*8, all scales 0x7f); mode 1 = e = floor(log2(block amax)) - 2
 * clamped to [-127, 127], byte = e + 127, q = e2m1(x * 2^-e). K = contiguous dim of dst. */
void or_quant_mxfp4(const float* src, uint8_t* dst, uint8_t* sf, int rows, int cols, int transpose, int mode) {
  const int K = transpose ? rows : cols, outer = transpose ? cols : rows;
  memset(sf, 0x7f, (size_t)or_sf_bytes(outer, K));
  for (int o = 0; o < outer; ++o)
    for (int j = 0; j < K / 32; ++j) {
      float v[32];
      for (int i = 0; i < 32; ++i) v[i] = transpose ? src[(long)(j * 32 + i) * cols + o] : src[(long)o * K + j * 32 + i];
      float mul = 8.f;
      uint8_t byte = 127;
      if (mode == 1) {
        float amax = 0.f;
        for (int i = 0; i < 32; ++i) { const float a = fabsf(v[i]); if (a > amax) amax = a; }
        const int biased = (int)((f2u(amax) >> 23) & 0xff);
        int e = (biased == 0) ? -127 : biased - 129;
        if (e < -127) e = -127;
        if (e > 127) e = 127;
        byte = (uint8_t)(e + 127);
        mul = u2f((uint32_t)(127 - e) << 23); /* 2^-e, e in [-127, 126] */
      }
      for (int i = 0; i < 32; i += 2)
        dst[(long)o * (K / 2) + (j * 32 + i) / 2] =
            (uint8_t)(or_e2m1_code(v[i] * mul) | (or_e2m1_code(v[i + 1] * mul) << 4));
      sf[or_sf_offset(o, j, K)] = byte;
    }
}

/* UE8M0 byte -> 2^(byte-127) as float (byte 0 -> 2^-127 is subnormal; 255 = NaN). */
float or_ue8m0_to_f32(uint8_t b) {
  if (b == 255) return NAN;
  return ldexpf(1.0f, (int)b - 127);
}

/* Dequantise packed fp4 (+ optional sf) into floats: rows x K. */
void or_dequant_mxfp4(const uint8_t* q, const uint8_t* sf, float* out, int rows, int K) {
  for (long r = 0; r < rows; ++r)
    for (long k = 0; k < K; ++k) {
      const uint8_t byte = q[r * (K / 2) + k / 2];
      const uint8_t code = (k & 1) ? (byte >> 4) : (byte & 15);
      const float scale = sf ? or_ue8m0_to_f32(sf[or_sf_offset((int)r, (int)(k / 32), K)]) : 1.0f;
      out[r * K + k] = or_e2m1_to_f32(code) * scale;
    }
}

void or_dequant_fp8(const uint8_t* q, float* out, long n) {
  for (long i = 0; i < n; ++i) out[i] = or_e4m3_to_f32(q[i]);
}

void or_f32_to_f16_array(const float* src, uint16_t* dst, long n) {
  for (long i = 0; i < n; ++i) dst[i] = or_f32_to_f16(src[i]);
}
void or_f16_to_f32_array(const uint16_t* src, float* dst, long n) {
  for (long i = 0; i < n; ++i) dst[i] = or_f16_to_f32(src[i]);
}

/* ------------------------------------------------------------------ FP64 GEMM */
/* C[m][n] = sum_k A[m][k] * B(k, n), B(k, n) = b_trans ? B[n][k] : B[k][n]; inputs are
 * fp32 values (every quantised value is exact in fp32), accumulation in double.
 * Rows of C are split over `nthreads` pthreads; each thread walks k in blocks so the
 * working set of B stays in cache. */
typedef struct {
  const float* A;
  const double* Bd; /* K x N, double */
  double* C;
  int M, N, K, m0, m1;
} gemm_job;

static void* gemm_worker(void* arg) {
  gemm_job* j = (gemm_job*)arg;
  const int N = j->N, K = j->K;
  const int KB = 128, NB = 512;
  for (int m = j->m0; m < j->m1; ++m) memset(j->C + (long)m * N, 0, sizeof(double) * N);
  for (int n0 = 0; n0 < N; n0 += NB) {
    const int n1 = n0 + NB < N ? n0 + NB : N;
    for (int k0 = 0; k0 < K; k0 += KB) {
      const int k1 = k0 + KB < K ? k0 + KB : K;
      for (int m = j->m0; m < j->m1; ++m) {
        double* c = j->C + (long)m * N;
        const float* a = j->A + (long)m * K;
        for (int k = k0; k < k1; ++k) {
          const double av = (double)a[k];
          const double* b = j->Bd + (long)k * N;
          for (int n = n0; n < n1; ++n) c[n] += av * b[n];
        }
      }
    }
  }
  return 0;
}

int or_gemm_f64(const float* A, const float* B, double* C, int M, int N, int K, int b_trans, int nthreads) {
  if (M <= 0 || N <= 0) return 0;
  double* Bd = (double*)malloc(sizeof(double) * (size_t)K * N + 8);
  if (!Bd) return -1;
  for (long k = 0; k < K; ++k)
    for (long n = 0; n < N; ++n) Bd[k * N + n] = (double)(b_trans ? B[n * K + k] : B[k * N + n]);
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  int created[256];
  gemm_job jobs[256];
  const int per = (M + nthreads - 1) / nthreads;
  for (int t = 0; t < nthreads; ++t) {
    created[t] = 0;
    const int m0 = t * per, m1 = (t + 1) * per < M ? (t + 1) * per : M;
    if (m0 >= m1) continue;
    jobs[t] = (gemm_job){A, Bd, C, M, N, K, m0, m1};
    if (pthread_create(&th[t], 0, gemm_worker, &jobs[t]) == 0) created[t] = 1;
    else gemm_worker(&jobs[t]);
  }
  for (int t = 0; t < nthreads; ++t)
    if (created[t]) pthread_join(th[t], 0);
  free(Bd);
  return 0;
}

/* max |C - R| over n entries, C float, R double. */
double or_max_abs_diff_f32(const float* C, const double* R, long n) {
  double m = 0.0;
  for (long i = 0; i < n; ++i) {
    const double d = fabs((double)C[i] - R[i]);
    if (d > m || d != d) m = (d != d) ? INFINITY : d;
  }
  return m;
}
