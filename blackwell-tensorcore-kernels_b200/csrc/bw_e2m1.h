/* E2M1 encoding by the reference's rule (src/gemm_mma_fp8.cu:47-58): the first level of
 * {0, .5, 1, 1.5, 2, 3, 4, 6} whose fp32 distance |(|v|) - level| is strictly smallest, sign bit
 * (8) iff v < 0. Shared by the CUDA quantisers and the host-side exhaustive check.
 *
 * Fast form: for |v| < 2^25 the rule equals rounding half-down onto the level grid (the fp32
 * distances to the two nearest levels are exact there, by Sterbenz). Every midpoint
 * (.25 .75 1.25 1.75 2.5 3.5 5) has at most two mantissa bits, so with b = bits(|v|) - 1 (the
 * -1 sends a value exactly on a midpoint to the lower side) the code depends only on the
 * exponent and top two mantissa bits of b: 20 buckets from 0.25 to 8, read from a 3-bit-per-entry
 * table. Beyond 2^25 rounded distances tie in ways only the loop reproduces; Inf and NaN go
 * there too (they give level 0). Checked against the loop over all 2^32 inputs. */
#ifndef BW_E2M1_H
#define BW_E2M1_H
#include <stdint.h>
#include <math.h>

#if defined(__CUDACC__)
#define BW_E2M1_FN __host__ __device__ __forceinline__
#define BW_E2M1_SLOW_FN __host__ __device__ __noinline__
#else
#define BW_E2M1_FN static inline
#define BW_E2M1_SLOW_FN static
#endif

#define BW_E2M1_TABLE 0x0ffed6c8da489249ull /* code of bucket k in bits [3k, 3k+3), k = 0..19 */

/* The reference loop, kept out of line so the fast path is not if-converted around it. */
BW_E2M1_SLOW_FN int bw_e2m1_level_loop(float a) {
  const float lv[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  float bd = fabsf(a - lv[0]);
  int c = 0;
  for (int i = 1; i < 8; ++i) {
    const float d = fabsf(a - lv[i]);
    if (d < bd) {
      bd = d;
      c = i;
    }
  }
  return c;
}

BW_E2M1_FN uint8_t bw_e2m1_code(float v) {
  union {
    float f;
    uint32_t u;
  } x;
  x.f = v;
  const uint32_t ab = x.u & 0x7fffffffu;
  int c;
  if (ab >= 0x4C000000u) { /* |v| >= 2^25, Inf, NaN: the reference loop */
    c = bw_e2m1_level_loop(fabsf(v));
  } else if (ab <= 0x3E800000u) { /* |v| <= 0.25 */
    c = 0;
  } else {
    const uint32_t k = (ab - 1u - 0x3E800000u) >> 21;
    c = k >= 20u ? 7 : (int)((BW_E2M1_TABLE >> (3u * k)) & 7u);
  }
  return (uint8_t)((v < 0.f ? 8 : 0) | c);
}

#endif /* BW_E2M1_H */
