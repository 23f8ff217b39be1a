// Column-panel tcgen05 GEMM for short-and-wide problems (M <= 256: decode-style 128 x 65536 x
// 8192), where the cost is reading B once from HBM.
//
// The output is cut into column panels of W columns; a CTA computes one panel for all MT (1 or
// 2) 128-row blocks of M at once (MT = ceil(M / 128)), so every B slab it loads feeds MT
// accumulators of W columns each (MT x W <= 512 = all of Tensor Memory). W is chosen on the
// host so the panels fill the SMs in as few, as full waves as possible (one wave for M <= 128
// and N <= 148 x 512). Each CTA runs over the whole K range: no split-K, so no zeroed C, no
// FP32 workspace and no reduction traffic, and every B byte is read exactly once. One CTA per
// SM (shared memory sizes it so).
//   warp 0      TMA producer: one elected lane streams A (MT x 128 x 128 B) and the B panel
//               (W x 128 B) per k-slab into a runtime-deep shared-memory ring.
//   warp 1      allocates Tensor Memory; one elected lane issues, per k-step and 128-row block,
//               one tcgen05.mma per 256-column chunk of the panel (N = 256 and W - 256 for
//               W > 256).
//   warps 2..5  epilogue once the last k-slab is in: tcgen05.ld 32 columns at a time, scale,
//               convert and store 256-bit pieces of each thread's row straight to C.
#pragma once
#include "bw_gemm_kernel.cuh"

namespace bw {

constexpr int kPanelMaxW = 512;
constexpr int kPanelMaxStages = 6;

struct PanelParams {
  int W;            // panel width (columns), multiple of 32 (64 for an N-major B)
  int panels;       // panels (= CTAs)
  int stages;       // shared-memory ring depth
  int stage_bytes;  // MT x 16 KB of A + W x 128 B of B, a multiple of 1024
  int b_box;        // rows per TMA box of a K-major B (W or W / 2)
};

// Dynamic shared memory of a panel launch: the ring, barriers, TMEM slot, abort flag, alignment.
__host__ __device__ constexpr int panel_smem_bytes(int stages, int stage_bytes) {
  return stages * stage_bytes + (2 * kPanelMaxStages + 2) * 8 + 16 + 1024;
}

template <Kind KIND, bool B_MN, Out OUT, int MT>
__global__ void __launch_bounds__(kThreads, 1)
    bw_tc_gemm_panel_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const GemmParams p, const PanelParams pp) {
  static_assert(KIND != Kind::MXF4, "panel kernel: dense kinds only");
  static_assert(MT == 1 || MT == 2, "one or two 128-row blocks of M");
  constexpr int KE = KindTraits<KIND>::kElemsPerSlab;
  constexpr int KX = KindTraits<KIND>::kCoordPerSlab;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + pp.stages * pp.stage_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kPanelMaxStages;
  uint64_t* accfull = bars + 2 * kPanelMaxStages;
  uint64_t* teardown = accfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(teardown + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int W = pp.W;
  const int col0 = blockIdx.x * W;
  const int nk = (p.K + KE - 1) / KE;
  const int S = pp.stages;
  const uint32_t tmem_cols = MT * W <= 256 ? 256u : 512u;
  const WaitCtl wc{abort_flag, p.status, p.budget_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    mbar_init(accfull, 1);
    mbar_init(teardown, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); }
  if (warp == 1) { tmem_alloc(tmem_slot, tmem_cols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol_a = l2_policy_evict_last();   // A is re-read by every panel
      const uint64_t pol_b = l2_policy_evict_first();  // each B byte is read once
      const uint32_t tx = static_cast<uint32_t>(pp.stage_bytes);
      int s = 0;
      uint32_t ph = 0;
      for (int kb = 0; kb < nk; ++kb) {
        if (!mbar_wait(&empty[s], ph ^ 1, wc, 41)) break;
        uint8_t* sA = smem + s * pp.stage_bytes;
        uint8_t* sB = sA + MT * kBM * kSlabBytes;
        mbar_arrive_expect_tx(&full[s], tx);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) tma_load_2d(&tmA, &full[s], sA + mt * kBM * kSlabBytes, kb * KX, mt * kBM, pol_a);
        if constexpr (B_MN) {
          for (int j = 0; j < W / 64; ++j)
            tma_load_2d(&tmB, &full[s], sB + j * 64 * kSlabBytes, col0 + 64 * j, kb * 64, pol_b);
        } else {
          for (int j = 0; j < W; j += pp.b_box)
            tma_load_2d(&tmB, &full[s], sB + j * kSlabBytes, kb * KX, col0 + j, pol_b);
        }
        if (++s == S) { s = 0; ph ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const int n1 = W > 256 ? W - 256 : 0;  // second chunk's width (0: one chunk)
      const uint32_t idesc0 = idesc_dense(KindTraits<KIND>::kFmt, KindTraits<KIND>::kFmt, B_MN, kBM, W > 256 ? 256 : W);
      const uint32_t idesc1 = idesc_dense(KindTraits<KIND>::kFmt, KindTraits<KIND>::kFmt, B_MN, kBM, n1 > 0 ? n1 : 16);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        if (!mbar_wait(&full[s], ph, wc, 42)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aaddr = smem_u32(smem + s * pp.stage_bytes);
        const uint32_t baddr = aaddr + MT * kBM * kSlabBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const uint64_t adesc = sdesc_sw128(aaddr + mt * kBM * kSlabBytes + k * 32, 16, 1024);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
              if (c == 1 && n1 == 0) break;
              uint64_t bdesc;
              // chunk c starts 256 columns in: 4 boxes of 64 columns (N-major) or 256 rows (K-major)
              if constexpr (B_MN) bdesc = sdesc_sw128(baddr + c * 4 * 64 * kSlabBytes + k * 16 * kSlabBytes,
                                                      64 * kSlabBytes, 1024);
              else bdesc = sdesc_sw128(baddr + c * 256 * kSlabBytes + k * 32, 16, 1024);
              const uint32_t d = tmem_base + mt * W + c * 256;
              if constexpr (KIND == Kind::F16) umma_f16(d, adesc, bdesc, c ? idesc1 : idesc0, acc);
              else umma_f8f6f4(d, adesc, bdesc, c ? idesc1 : idesc0, acc);
            }
          }
        }
        umma_commit(&empty[s]);
        if (++s == S) { s = 0; ph ^= 1; }
      }
      if (ok) umma_commit(accfull);
      umma_commit(teardown);
      mbar_wait(teardown, 0, WaitCtl{abort_flag, p.status, p.budget_ns}, 43);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    float alpha = 1.f;
    if (p.scale_a) alpha *= __ldg(p.scale_a);
    if (p.scale_b) alpha *= __ldg(p.scale_b);
    if (mbar_wait(accfull, 0, wc, 44)) {
      tc_fence_after();
      const bool stream_out = (p.hints & 2) != 0;
      const uint64_t pol = l2_policy_evict_first();
#pragma unroll 1
      for (int cc = 0; cc < MT * W; cc += 32) {
        const int mt = cc / W, c = cc - mt * W;  // accumulator mt holds rows [128 mt, 128 mt + 128)
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + mt * W;
        const int row = mt * kBM + q * 32 + lane;
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + c, r);
        tmem_ld_wait();
        const int col = col0 + c;
        if (row >= p.M || col >= p.N) continue;
        if constexpr (OUT == Out::F32) {
          float* dst = reinterpret_cast<float*>(p.C) + static_cast<size_t>(row) * p.ldc + col;
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            if (col + 8 * g >= p.N) break;
            uint32_t v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __float_as_uint(__uint_as_float(r[8 * g + j]) * alpha);
            if (stream_out) st_global_v8_hint(dst + 8 * g, v, pol);
            else st_global_v8(dst + 8 * g, v);
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<size_t>(row) * p.ldc + col;
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            if (col + 16 * g >= p.N) break;
            uint32_t v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[16 * g + 2 * j]) * alpha,
                                                       __uint_as_float(r[16 * g + 2 * j + 1]) * alpha);
              v[j] = *reinterpret_cast<uint32_t*>(&h);
            }
            if (col + 16 * g + 16 <= p.N) {
              if (stream_out) st_global_v8_hint(dst + 16 * g, v, pol);
              else st_global_v8(dst + 16 * g, v);
            } else {  // N % 16 == 8: the last group holds 8 valid columns
              *reinterpret_cast<uint4*>(dst + 16 * g) = make_uint4(v[0], v[1], v[2], v[3]);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

}  // namespace bw
