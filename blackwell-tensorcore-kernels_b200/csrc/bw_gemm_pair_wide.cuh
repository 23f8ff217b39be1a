// CTA-pair GEMM with 256 x 512 output tiles (FP16 and E4M3 operands).
//
// Same roles as bw_tc_gemm_pair_kernel (bw_gemm_pair.cuh): a cluster of two CTAs shares one tile,
// CTA r loads rows [128r, 128r+128) of A and 128 columns of each 256-column half of B, and the
// leader's MMA thread issues tcgen05.mma.cta_group::2 (M = 256, N = 256) twice per K step, once
// per N half. Per k-atom a CTA moves 16 KB of A and 32 KB of B for 2x the MMA work of the
// 256 x 256 tile (which moves 16 + 16 KB), i.e. 27% less L2 -> SM traffic per FLOP; under the
// power cap that traffic costs clock (removing half of B's traffic in an experiment raised the
// sustained FP16 rate by 5%).
//
// Tensor Memory holds one 512-column accumulator (the two halves side by side), so the epilogue
// cannot run behind a second buffer. Instead each half is released on its own: 8 epilogue warps
// (two per TMEM lane quarter, 128 columns each) drain half 0 into registers as soon as its last
// MMAs complete (accfull[0], committed before the last half-1 MMAs), free it (half_free[0]),
// store it, then drain and free half 1. The MMA thread starts the next tile's half-0 MMAs as
// soon as half 0 is free and waits for half 1 only before its first half-1 MMA.
// Stage = one K atom (A 16 KB + B 2 x 16 KB), 4 stages, 8 MMAs per stage.
#pragma once
#include "bw_gemm_kernel.cuh"

namespace bw {

constexpr int kWideThreads = 320;  // producer, MMA, 8 epilogue warps
constexpr int kWideStages = 4;

struct WideCfg {
  static constexpr int kABytes = 128 * kSlabBytes;      // this CTA's 128 rows x one K atom
  static constexpr int kBHalfBytes = 128 * kSlabBytes;  // this CTA's 128 columns of one N half
  static constexpr int kStageBytes = kABytes + 2 * kBHalfBytes;
  static constexpr int kBarOffset = kWideStages * kStageBytes;
  // full[S], empty[S], accfull[2], half_free[2], teardown
  static constexpr int kNumBars = 2 * kWideStages + 5;
  static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr int kTmemCols = 512;
};

template <Kind KIND, bool B_MN, Out OUT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kWideThreads, 1)
    bw_tc_gemm_pair_wide_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                const GemmParams p) {
  static_assert(KIND == Kind::F16 || KIND == Kind::F8, "dense FP16 / E4M3 operands");
  using Cfg = WideCfg;
  constexpr int KX = KindTraits<KIND>::kCoordPerSlab;
  constexpr int KE = KindTraits<KIND>::kElemsPerSlab;
  constexpr int TM = 256, TN = 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint64_t* full = bars;
  uint64_t* empty = bars + kWideStages;
  uint64_t* accfull = bars + 2 * kWideStages;  // [2]: N half h of the tile is complete
  uint64_t* half_free = accfull + 2;  // [2], on the leader: both CTAs' 8 epilogue warps arrive
  uint64_t* teardown = accfull + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t peer = rank ^ 1u;
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;
  const int tiles_m = (p.M + TM - 1) / TM;
  const int tiles_n = (p.N + TN - 1) / TN;
  const int num_tiles = tiles_m * tiles_n;
  const int nk = (p.K + KE - 1) / KE;
  const WaitCtl wc{abort_flag, p.status, p.budget_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWideStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&accfull[h], 1);
      mbar_init(&half_free[h], 2 * 8);
    }
    mbar_init(teardown, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); }
  if (warp == 1) { tmem_alloc_pair(tmem_slot, Cfg::kTmemCols); tmem_relinquish_pair(); }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      const uint64_t pol = (p.hints & 1) ? l2_policy_evict_last() : l2_policy_evict_normal();
      const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = cluster; t < num_tiles && ok; t += nclusters) {
        int tm, tn;
        tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn);
        const int arow = tm * TM + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, wc, 51)) { ok = false; break; }
          uint8_t* sA = smem + s * Cfg::kStageBytes;
          uint8_t* sB = sA + Cfg::kABytes;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * Cfg::kStageBytes);
          const uint32_t fb = full_leader + s * 8;
          tma_load_2d_pair(&tmA, fb, sA, kb * KX, arow, pol);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int bcol = tn * TN + 256 * h + static_cast<int>(rank) * 128;
            uint8_t* dst = sB + h * Cfg::kBHalfBytes;
            if constexpr (B_MN) {
              tma_load_2d_pair(&tmB, fb, dst, bcol, kb * 64, pol);
              tma_load_2d_pair(&tmB, fb, dst + 64 * kSlabBytes, bcol + 64, kb * 64, pol);
            } else {
              tma_load_2d_pair(&tmB, fb, dst, kb * KX, bcol, pol);
            }
          }
          if (++s == kWideStages) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only) ----------------
    if (leader && lane == 0) {
      const uint32_t idesc = idesc_dense(KindTraits<KIND>::kFmt, KindTraits<KIND>::kFmt, B_MN, 256, 256);
      const uint32_t empty_own = smem_u32(empty), empty_peer = mapa_shared(smem_u32(empty), peer);
      const uint32_t accfull_own = smem_u32(accfull), accfull_peer = mapa_shared(smem_u32(accfull), peer);
      int s = 0;
      uint32_t ph = 0;
      int local = 0;
      bool ok = true;
      for (int t = cluster; t < num_tiles && ok; t += nclusters, ++local) {
        const uint32_t fph = static_cast<uint32_t>(local & 1) ^ 1u;  // half_free phase of the previous tile
        for (int kb = 0; kb < nk && ok; ++kb) {
          if (!mbar_wait(&full[s], ph, wc, 52)) { ok = false; break; }
          tc_fence_after();
          const uint32_t aaddr = smem_u32(smem + s * Cfg::kStageBytes);
          const uint32_t baddr = aaddr + Cfg::kABytes;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (kb == 0) {  // this half of the accumulator must have been drained
              if (!mbar_wait(&half_free[h], fph, wc, 53)) { ok = false; break; }
              tc_fence_after();
            }
            const uint32_t d_tmem = tmem_base + 256 * h;
            const uint32_t bh = baddr + h * Cfg::kBHalfBytes;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
              const uint64_t adesc = sdesc_sw128(aaddr + k * 32, 16, 1024);
              uint64_t bdesc;
              if constexpr (B_MN) bdesc = sdesc_sw128(bh + k * 16 * kSlabBytes, 64 * kSlabBytes, 1024);
              else bdesc = sdesc_sw128(bh + k * 32, 16, 1024);
              if constexpr (KIND == Kind::F16) umma_f16_pair(d_tmem, adesc, bdesc, idesc, acc);
              else umma_f8f6f4_pair(d_tmem, adesc, bdesc, idesc, acc);
            }
            if (kb == nk - 1) {  // half h of the tile is final: its epilogue may start now
              umma_commit_pair(accfull_own + h * 8);
              umma_commit_pair(accfull_peer + h * 8);
            }
          }
          if (!ok) break;
          umma_commit_pair(empty_own + s * 8);
          umma_commit_pair(empty_peer + s * 8);
          if (++s == kWideStages) { s = 0; ph ^= 1; }
        }
      }
      umma_commit_pair(smem_u32(teardown));
      mbar_wait(teardown, 0, wc, 54);
    }
  } else {
    // ---------------- epilogue (warps 2..9 of both CTAs) ----------------
    const int q = warp & 3;            // TMEM lane quarter
    const int cpart = (warp - 2) >> 2; // which 128 columns of each half
    const uint32_t half_free_leader = mapa_shared(smem_u32(half_free), 0);
    float alpha = 1.f;
    if (p.scale_a) alpha *= __ldg(p.scale_a);
    if (p.scale_b) alpha *= __ldg(p.scale_b);
    int local = 0;
    for (int t = cluster; t < num_tiles; t += nclusters, ++local) {
      int tm, tn;
      tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn);
      const int row = tm * TM + static_cast<int>(rank) * 128 + q * 32 + lane;
      bool ok = true;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        if (!mbar_wait(&accfull[h], static_cast<uint32_t>(local & 1), wc, 55)) { ok = false; break; }
        tc_fence_after();
        const int cols = 256 * h + 128 * cpart;
        uint32_t r[128];
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + cols;
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(tbase + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * c]));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote_cta(half_free_leader + h * 8);  // the MMA may refill this half
        if (row >= p.M) continue;
        const int col0 = tn * TN + cols;
        if constexpr (OUT == Out::F32) {
          float* dst = reinterpret_cast<float*>(p.C) + static_cast<size_t>(row) * p.ldc + col0;
#pragma unroll
          for (int g = 0; g < 16; ++g) {
            if (col0 + 8 * g >= p.N) break;
            uint32_t v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __float_as_uint(__uint_as_float(r[8 * g + j]) * alpha);
            st_global_v8(dst + 8 * g, v);
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<size_t>(row) * p.ldc + col0;
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            if (col0 + 16 * g >= p.N) break;
            uint32_t v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(r[16 * g + 2 * j]) * alpha,
                                                        __uint_as_float(r[16 * g + 2 * j + 1]) * alpha);
              v[j] = *reinterpret_cast<uint32_t*>(&b2);
            }
            st_global_v8(dst + 16 * g, v);
          }
        }
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace bw
