/* Test infrastructure: checks the library's fast E2M1 encoder (bucket table,
 * blackwell-tensorcore-kernels_b200/csrc/bw_e2m1.h, used by the CUDA quantisers) against the
 * oracle's restatement of the reference rule (or_e2m1_code, src/gemm_mma_fp8.cu:47-58) over
 * every 32-bit pattern with the given stride (1 = all 2^32). Exit status 0 iff they agree. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../blackwell-tensorcore-kernels_b200/csrc/bw_e2m1.h"

uint8_t or_e2m1_code(float v);

int main(int argc, char** argv) {
  const uint64_t stride = argc > 1 ? strtoull(argv[1], NULL, 10) : 1;
  uint64_t bad = 0, n = 0;
  for (uint64_t u = 0; u <= 0xFFFFFFFFull; u += stride) {
    const uint32_t b = (uint32_t)u;
    float v;
    memcpy(&v, &b, 4);
    ++n;
    if (bw_e2m1_code(v) != or_e2m1_code(v)) {
      if (bad < 8) printf("mismatch at %08x: fast %d, rule %d\n", b, bw_e2m1_code(v), or_e2m1_code(v));
      ++bad;
    }
  }
  printf("%llu inputs, %llu mismatches\n", (unsigned long long)n, (unsigned long long)bad);
  return bad != 0;
}
