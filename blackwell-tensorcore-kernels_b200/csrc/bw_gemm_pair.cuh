// CTA-pair (cta_group::2) variant of the persistent tcgen05 GEMM: 256 x 256 output tiles.
//
// A cluster of two CTAs on neighbouring SMs shares one 256 x 256 accumulator tile: CTA r
// loads rows [128r, 128r+128) of A and columns [128r, 128r+128) of B for every k-slab into
// its own shared memory (no multicast; each TMA load targets its own CTA), and the leader
// CTA's single MMA thread issues tcgen05.mma.cta_group::2 with M = 256, N = 256, which reads
// both CTAs' slabs and accumulates rows [128r, 128r+128) in CTA r's Tensor Memory. Per CTA
// and k-slab this moves 32 KB instead of the 48 KB of a 128 x 256 single-CTA tile for the
// same MMA work, which is what keeps the L2 -> SM feed below the tensor-core rate.
//
// Synchronisation:
//   full[s]    (leader)  producer of the leader expects both CTAs' bytes; both CTAs' TMA
//                        loads complete on it.
//   empty[s]   (each)    the leader's MMA thread commits to its own and to the peer's copy.
//   accfull[b] (each)    accumulator b ready: committed to both CTAs.
//   accempty[b](leader)  4 epilogue warps of each CTA arrive (8 arrivals).
// Every wait is bounded; all CTAs reach the closing cluster barrier on every path.
#pragma once
#include "bw_gemm_kernel.cuh"

namespace bw {

template <Kind KIND, int STAGES, bool DIRECT_EPI = false, int KSUB = 1, int TN = 256, int EPI_BUFS = 2>
struct PairCfg {
  static constexpr int kAtomBytes = 128 * kSlabBytes;  // 128 rows x one 128-byte swizzle atom of K
  static constexpr int kBAtomBytes = (TN / 2) * kSlabBytes;
  static constexpr int kABytes = KSUB * kAtomBytes;    // this CTA's 128 rows of A, KSUB atoms of K
  static constexpr int kBBytes = KSUB * kBAtomBytes;   // this CTA's TN/2 columns of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiOffset = STAGES * kStageBytes;
  // plain FP4 (kind::mxf4 with every block scale 2^0): 3 constant scale-factor atoms
  static constexpr int kEpiBufs = EPI_BUFS;  // staging buffers per epilogue warp (staged epilogue)
  static constexpr int kSfOffset = kEpiOffset + (DIRECT_EPI ? 0 : kEpiWarps * EPI_BUFS * kEpiBufBytes);
  static constexpr int kSfBytes = (KIND == Kind::MXF4) ? 3 * 512 : 0;
  static constexpr int kBarOffset = kSfOffset + kSfBytes;
  static_assert(TN % 32 == 0 && TN <= 256 && (KIND == Kind::MXF4 ? 2 * TN + 12 <= 512 : TN == 256), "tile N");
  static constexpr int kNumBars = 2 * STAGES + 2 * 2 + 1;
  static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr int kTmemCols = 512;  // two 256-column FP32 accumulators
};

template <Kind KIND, bool B_MN, int STAGES, Out OUT, bool DIRECT_EPI, int KSUB, int TN = 256, int EPI_BUFS = 2>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    bw_tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmC, const __grid_constant__ PeerMaps pm,
                           const GemmParams p) {
  using Cfg = PairCfg<KIND, STAGES, DIRECT_EPI, KSUB, TN, EPI_BUFS>;
  static_assert(!B_MN || TN == 256, "N-major B is loaded as 64-column boxes of a 256-wide tile");
  constexpr int KX = KindTraits<KIND>::kCoordPerSlab;          // tensor-map units per swizzle atom
  constexpr int KE = KindTraits<KIND>::kElemsPerSlab * KSUB;   // K elements per pipeline stage
  constexpr int TM = 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* accfull = bars + 2 * STAGES;
  uint64_t* accempty = bars + 2 * STAGES + 2;
  uint64_t* teardown = bars + 2 * STAGES + 4;
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
  const bool tracing = p.trace != nullptr;
  const long long t_start = clock64();
  unsigned long long tr_a = 0, tr_b = 0, tr_c = 0;  // role-specific wait counters

  if constexpr (KIND == Kind::MXF4) {
    uint32_t* sf = reinterpret_cast<uint32_t*>(smem + Cfg::kSfOffset);
    for (int i = threadIdx.x; i < Cfg::kSfBytes / 4; i += kThreads) sf[i] = 0x7f7f7f7fu;  // 2^0
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&accfull[b], 1); mbar_init(&accempty[b], 2 * kEpiWarps); }
    mbar_init(teardown, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); tma_prefetch_desc(&tmC); }
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
        const int bcol = tn * TN + static_cast<int>(rank) * (TN / 2);
        for (int kb = 0; kb < nk; ++kb) {
          const long long w0 = tracing ? clock64() : 0;
          if (!mbar_wait(&empty[s], ph ^ 1, wc, 11)) { ok = false; break; }
          if (tracing) tr_a += clock64() - w0;
          uint8_t* sA = smem + s * Cfg::kStageBytes;
          uint8_t* sB = sA + Cfg::kABytes;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * Cfg::kStageBytes);
          const uint32_t fb = full_leader + s * 8;
#pragma unroll
          for (int j = 0; j < KSUB; ++j) {
            const int ka = kb * KSUB + j;  // swizzle-atom index along K
            tma_load_2d_pair(&tmA, fb, sA + j * Cfg::kAtomBytes, ka * KX, arow, pol);
            if constexpr (B_MN) {
              tma_load_2d_pair(&tmB, fb, sB + j * Cfg::kAtomBytes, bcol, ka * 64, pol);
              tma_load_2d_pair(&tmB, fb, sB + j * Cfg::kAtomBytes + 64 * kSlabBytes, bcol + 64, ka * 64, pol);
            } else {
              tma_load_2d_pair(&tmB, fb, sB + j * Cfg::kBAtomBytes, ka * KX, bcol, pol);
            }
          }
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only) ----------------
    if (leader && lane == 0) {
      const uint32_t idesc = (KIND == Kind::MXF4) ? 0u
                             : idesc_dense(KindTraits<KIND>::kFmt, KindTraits<KIND>::kFmt, B_MN, 256, TN);
      const uint32_t tmem_sf = tmem_base + 2 * TN;  // plain FP4: SFA atom at +0, SFB blocks at +4, +8
      if constexpr (KIND == Kind::MXF4) {
        const uint32_t sf_s = smem_u32(smem + Cfg::kSfOffset);
#pragma unroll
        for (int a = 0; a < 3; ++a) tmem_cp_32x128b_warpx4_pair(tmem_sf + 4 * a, sdesc_noswz(sf_s + 512 * a, 16, 128));
      }
      const uint32_t empty_own = smem_u32(empty), empty_peer = mapa_shared(smem_u32(empty), peer);
      const uint32_t accfull_own = smem_u32(accfull), accfull_peer = mapa_shared(smem_u32(accfull), peer);
      int s = 0;
      uint32_t ph = 0;
      int local = 0;
      bool ok = true;
      for (int t = cluster; t < num_tiles && ok; t += nclusters, ++local) {
        const int b = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        const long long w1 = tracing ? clock64() : 0;
        if (!mbar_wait(&accempty[b], aph ^ 1, wc, 12)) { ok = false; break; }
        if (tracing) tr_b += clock64() - w1;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * TN;
        for (int kb = 0; kb < nk; ++kb) {
          const long long w2 = tracing ? clock64() : 0;
          if (!mbar_wait(&full[s], ph, wc, 13)) { ok = false; break; }
          if (tracing) { tr_a += clock64() - w2; ++tr_c; }
          tc_fence_after();
          const uint32_t aaddr = smem_u32(smem + s * Cfg::kStageBytes);
          const uint32_t baddr = aaddr + Cfg::kABytes;
#pragma unroll
          for (int kk = 0; kk < 4 * KSUB; ++kk) {
            const int j = kk >> 2, k = kk & 3;
            const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
            const uint64_t adesc = sdesc_sw128(aaddr + j * Cfg::kAtomBytes + k * 32, 16, 1024);
            uint64_t bdesc;
            if constexpr (B_MN)
              bdesc = sdesc_sw128(baddr + j * Cfg::kAtomBytes + k * 16 * kSlabBytes, 64 * kSlabBytes, 1024);
            else bdesc = sdesc_sw128(baddr + j * Cfg::kBAtomBytes + k * 32, 16, 1024);
            if constexpr (KIND == Kind::F16) umma_f16_pair(d_tmem, adesc, bdesc, idesc, acc);
            else if constexpr (KIND == Kind::F8) umma_f8f6f4_pair(d_tmem, adesc, bdesc, idesc, acc);
            else umma_mxf4_pair(d_tmem, adesc, bdesc, idesc_mxf4(256, TN, (2 * k) & 3, (2 * k) & 3), tmem_sf,
                                tmem_sf + 4, acc);
          }
          umma_commit_pair(empty_own + s * 8);
          umma_commit_pair(empty_peer + s * 8);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (ok) {
          umma_commit_pair(accfull_own + b * 8);
          umma_commit_pair(accfull_peer + b * 8);
        }
      }
      umma_commit_pair(smem_u32(teardown));
      mbar_wait(teardown, 0, wc, 14);
    }
  } else {
    // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
    const int q = warp & 3;
    const uint64_t store_pol = l2_policy_evict_first();
    uint8_t* wbuf = smem + Cfg::kEpiOffset + (warp - 2) * EPI_BUFS * kEpiBufBytes;
    int uses = 0;
    const uint32_t accempty_leader = mapa_shared(smem_u32(accempty), 0);
    float alpha = 1.f;
    if (p.scale_a) alpha *= __ldg(p.scale_a);
    if (p.scale_b) alpha *= __ldg(p.scale_b);
    int local = 0;
    for (int t = cluster; t < num_tiles; t += nclusters, ++local) {
      int tm, tn;
      tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn);
      const int b = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      const long long w3 = tracing ? clock64() : 0;
      if (!mbar_wait(&accfull[b], aph, wc, 15)) break;
      const long long w4 = tracing ? clock64() : 0;
      if (tracing) tr_a += w4 - w3;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * TN;
      auto release = [&] {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote_cta(accempty_leader + b * 8);
      };
      const int row0 = tm * TM + static_cast<int>(rank) * 128 + q * 32;
      if constexpr (DIRECT_EPI) epilogue_tile_direct<OUT, TN>(tbase, p, row0 + lane, tn * TN, alpha, release);
      else epilogue_tile<OUT, TN, decltype(release), EPI_BUFS>(tbase, &tmC, tn * TN, row0, alpha, wbuf, uses, lane, store_pol,
                                  (p.hints & 2) != 0, release, false, &pm, p.npeers, p.mc ? &p : nullptr);
      if (tracing) { tr_b += clock64() - w4; ++tr_c; }
    }
    if (lane == 0) bulk_wait_group<0>();
    if (p.mc) __threadfence_system();  // multicast stores performed before the grid completes
  }

  if (tracing && lane == 0) {
    unsigned long long* tr = p.trace + static_cast<size_t>(blockIdx.x) * kTraceWords;
    if (warp == 0) tr[3] = tr_a;
    if (warp == 1 && leader) { tr[1] = tr_a; tr[2] = tr_b; tr[7] = tr_c; }
    if (warp == 2) { tr[4] = tr_a; tr[5] = tr_b; tr[6] = tr_c; }
  }
  tc_fence_before();
  cluster_sync();
  if (tracing && threadIdx.x == 0) p.trace[static_cast<size_t>(blockIdx.x) * kTraceWords] = clock64() - t_start;
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace bw
