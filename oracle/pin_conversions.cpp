// Pins the oracle's hand-written fp32->fp16 and fp32->e4m3(satfinite) conversions against
// CUDA's host-side conversion functions (the ones the reference calls: __float2half in
// src/gemm_wmma.cu:106-108 and __nv_fp8_e4m3(x) in src/gemm_mma_fp8.cu:37-45), and the
// decoders against each other. Test infrastructure, built and run by tests/test_oracle.py.
//   pin_conversions [stride]   checks every `stride`-th fp32 bit pattern (1 = all 2^32)
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

extern "C" {
uint16_t or_f32_to_f16(float);
float or_f16_to_f32(uint16_t);
uint8_t or_f32_to_e4m3_sat(float);
float or_e4m3_to_f32(uint8_t);
}

int main(int argc, char** argv) {
  const uint64_t stride = argc > 1 ? strtoull(argv[1], nullptr, 10) : 1;
  uint64_t checked = 0, bad16 = 0, bad8 = 0;
  for (uint64_t u = 0; u < (1ull << 32); u += stride) {
    float f;
    uint32_t x = static_cast<uint32_t>(u);
    memcpy(&f, &x, 4);
    __half h = __float2half_rn(f);
    uint16_t hb;
    memcpy(&hb, &h, 2);
    const uint16_t mine16 = or_f32_to_f16(f);
    const bool nan = (x & 0x7fffffffu) > 0x7f800000u;
    if (nan ? ((mine16 & 0x7fffu) <= 0x7c00u) : (mine16 != hb)) {
      if (bad16 < 5) printf("f16 mismatch x=%08x cuda=%04x mine=%04x\n", x, hb, mine16);
      ++bad16;
    }
    const uint8_t c8 = static_cast<uint8_t>(__nv_cvt_float_to_fp8(f, __NV_SATFINITE, __NV_E4M3));
    const uint8_t mine8 = or_f32_to_e4m3_sat(f);
    if (c8 != mine8) {
      if (bad8 < 5) printf("e4m3 mismatch x=%08x cuda=%02x mine=%02x\n", x, c8, mine8);
      ++bad8;
    }
    ++checked;
  }
  uint64_t baddec = 0;
  for (int c = 0; c < 256; ++c) {
    __nv_fp8_e4m3 v;
    v.__x = static_cast<__nv_fp8_storage_t>(c);
    const float a = static_cast<float>(v), b = or_e4m3_to_f32(static_cast<uint8_t>(c));
    if (!((a == b) || (a != a && b != b))) ++baddec;
  }
  for (uint32_t hbits = 0; hbits < 65536; ++hbits) {
    __half_raw r;
    r.x = static_cast<unsigned short>(hbits);
    const float a = __half2float(__half(r)), b = or_f16_to_f32(static_cast<uint16_t>(hbits));
    if (!((a == b) || (a != a && b != b))) ++baddec;
  }
  printf("checked=%llu f16_mismatch=%llu e4m3_mismatch=%llu decode_mismatch=%llu\n",
         (unsigned long long)checked, (unsigned long long)bad16, (unsigned long long)bad8,
         (unsigned long long)baddec);
  return (bad16 || bad8 || baddec) ? 1 : 0;
}
