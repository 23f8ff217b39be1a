// CTA-pair block-scaled FP4 GEMM (kind::mxf4, E2M1 packed, UE8M0 per 32 K): 256 x 256 tiles.
//
// Replaces gemm_lowprec_t<MXFP4> / <FP4> (src/gemm_mma_fp8.cu:89-223, 305-317) for large
// problems. Structure as bw_tc_gemm_pair_kernel (bw_gemm_pair.cuh) with these differences:
//   * scale factors travel apart from A/B: a loader warp (both CTAs) TMA-loads each stage's SF
//     atoms - this CTA's 128 A rows and all 256 B rows of the tile, since both CTAs' tensor
//     cores scale the full N - into a 4-slot shared-memory ring (sf_full / sf_empty), and a
//     copier warp (leader) moves them with tcgen05.cp.cta_group::2 (each CTA from its own shared
//     memory) into one of kSfBufs TMEM column buffers (sf_ready / sf_free), so the copies run
//     ahead of the A/B data and the MMA thread issues only MMAs and commits;
//   * Tensor Memory holds one 256-column FP32 accumulator plus the scale-factor buffers (two
//     accumulators would leave no room), so 8 epilogue warps drain the accumulator into
//     registers (128 columns each), release it at once (CTA-scope arrive) and convert/store
//     while the next tile already accumulates.
// A/B stage = 2 K atoms (512 FP4 values): A 32 KB + B 32 KB per CTA, 3 stages; SF slot = SFA
// 2 KB + SFB 4 KB. With null scale-factor pointers (plain FP4, per-tensor scales only) the
// 0x7f-filled slot 0 is copied once and every block scale stays 2^0.
#pragma once
#include "bw_gemm_kernel.cuh"

namespace bw {

constexpr int kMxThreads = 384;  // producer, MMA, 8 epilogue warps, scale-factor copier and loader
constexpr int kMxKsub = 2;
constexpr int kMxStages = 3;     // A/B stages
constexpr int kMxSfSlots = 4;    // scale-factor stages in shared memory (run ahead of A/B)

// TN = 256: one 256-column accumulator, 8 epilogue warps drain it to registers.
// TN = 192: two 192-column accumulators (epilogue overlaps the next tile), 4 epilogue warps
//           with direct stores; a tile's B rows start at offset 0 or 64 inside a 128-row
//           scale-factor block, which shifts the SFB TMEM address by 0 or 2 columns.
template <int TN>
struct MxPairCfg {
  static_assert(TN == 192 || TN == 256, "block-scaled tile N");
  static constexpr int kAccBufs = TN == 192 ? 2 : 1;
  static constexpr int kAtom = 128 * kSlabBytes;           // 128 rows x 128 B
  static constexpr int kBAtom = (TN / 2) * kSlabBytes;     // this CTA's TN/2 rows of Bt
  static constexpr int kABytes = kMxKsub * kAtom;          // 32 KB
  static constexpr int kBBytes = kMxKsub * kBAtom;         // 32 or 24 KB
  static constexpr int kSfaBytes = kMxKsub * 1024;         // 2 SF atoms (512 B) per K atom of 256
  static constexpr int kSfbBytes = 2 * kSfaBytes;          // two 128-row blocks of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kSfSlotBytes = kSfaBytes + kSfbBytes;
  static constexpr int kSfRingOffset = kMxStages * kStageBytes;
  static constexpr int kBarOffset = kSfRingOffset + kMxSfSlots * kSfSlotBytes;
  static constexpr int kSfBufs = TN == 256 ? 3 : 2;         // TMEM scale-factor buffers
  // full[S], empty[S], accfull[2], accempty[2], teardown, sf_ready[kSfBufs], sf_free[kSfBufs],
  // sf_full[kMxSfSlots], sf_empty[kMxSfSlots]
  static constexpr int kNumBars = 2 * kMxStages + 5 + 2 * kSfBufs + 2 * kMxSfSlots;
  static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static constexpr int kSfaCols = 4 * kMxKsub * 2;          // 4 atoms per stage x 4 columns
  static constexpr int kSfbCols = 2 * kSfaCols;             // two row blocks
  static constexpr int kSfCols = kSfaCols + kSfbCols;       // 48 per buffer
  static constexpr int kSfBase = kAccBufs * TN;            // first scale-factor column
  static constexpr int kTmemCols = 512;
  static_assert(kSfBase + kSfBufs * kSfCols <= kTmemCols, "TMEM budget");
};

template <Out OUT, int TN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kMxThreads, 1)
    bw_tc_gemm_pair_mx_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                              const __grid_constant__ CUtensorMap tmSfa, const __grid_constant__ CUtensorMap tmSfb,
                              const GemmParams p) {
  using Cfg = MxPairCfg<TN>;
  constexpr int KX = 128;    // packed bytes per K atom (256 FP4 values)
  constexpr int KE = 256 * kMxKsub;
  constexpr int TM = 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint64_t* full = bars;
  uint64_t* empty = bars + kMxStages;
  uint64_t* accfull = bars + 2 * kMxStages;
  uint64_t* accempty = accfull + 2;
  uint64_t* teardown = accfull + 4;
  uint64_t* sf_ready = accfull + 5;                // [kSfBufs]: a stage's scale factors are in buffer b
  uint64_t* sf_free = sf_ready + Cfg::kSfBufs;     // [kSfBufs]: the MMAs reading buffer b have completed
  uint64_t* sf_full = sf_free + Cfg::kSfBufs;      // [slots] (leader): both CTAs' scale factors landed
  uint64_t* sf_empty = sf_full + kMxSfSlots;       // [slots] (each): the copies out of the slot are done
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
  const bool unit_sf = p.sfa == nullptr;
  const WaitCtl wc{abort_flag, p.status, p.budget_ns};
  const long long t_start = clock64();
  const bool tracing = p.trace != nullptr;
  unsigned long long tr_a = 0, tr_b = 0, tr_c = 0;
  long long t_commit = 0;

  // Scale-factor slot 0 starts at 2^0 (0x7f): the plain-FP4 path copies it once.
  if (unit_sf) {
    uint32_t* sf = reinterpret_cast<uint32_t*>(smem + Cfg::kSfRingOffset);
    for (int i = threadIdx.x; i < Cfg::kSfSlotBytes / 4; i += kMxThreads) sf[i] = 0x7f7f7f7fu;
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMxStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 2 * (TN == 192 ? 4 : 8));  // epilogue warps of both CTAs
    }
    mbar_init(teardown, unit_sf ? 1 : 2);  // MMA thread and scale-factor copier
    for (int b = 0; b < Cfg::kSfBufs; ++b) { mbar_init(&sf_ready[b], 1); mbar_init(&sf_free[b], 1); }
    for (int b = 0; b < kMxSfSlots; ++b) { mbar_init(&sf_full[b], 1); mbar_init(&sf_empty[b], 1); }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (!unit_sf) { tma_prefetch_desc(&tmSfa); tma_prefetch_desc(&tmSfb); }
  }
  if (warp == 1) { tmem_alloc_pair(tmem_slot, Cfg::kTmemCols); tmem_relinquish_pair(); }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // scale-factor buffer b: SFA at 256 + 48b (16 columns), SFB right after (32 columns)
  const uint32_t tmem_sfa = tmem_base + Cfg::kSfBase;
  const uint32_t tmem_sfb = tmem_sfa + Cfg::kSfaCols;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
      const uint32_t stage_tx = Cfg::kStageBytes;
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
          if (!mbar_wait(&empty[s], ph ^ 1, wc, 31)) { ok = false; break; }
          if (tracing) tr_a += clock64() - w0;
          uint8_t* sA = smem + s * Cfg::kStageBytes;
          uint8_t* sB = sA + Cfg::kABytes;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * stage_tx);
          const uint32_t fb = full_leader + s * 8;
#pragma unroll
          for (int j = 0; j < kMxKsub; ++j) {
            const int ka = kb * kMxKsub + j;
            tma_load_2d_pair(&tmA, fb, sA + j * Cfg::kAtom, ka * KX, arow, pol);
            tma_load_2d_pair(&tmB, fb, sB + j * Cfg::kBAtom, ka * KX, bcol, pol);
          }
          if (++s == kMxStages) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (leader && lane == 0) {
      const uint32_t empty_own = smem_u32(empty), empty_peer = mapa_shared(smem_u32(empty), peer);
      const uint32_t accfull_own = smem_u32(accfull), accfull_peer = mapa_shared(smem_u32(accfull), peer);
      int s = 0;
      uint32_t ph = 0;
      int local = 0;
      bool ok = true;
      bool sf_loaded = false;
      int sb = 0;         // scale-factor buffer of the next stage
      uint32_t sph = 0;   // its phase
      for (int t = cluster; t < num_tiles && ok; t += nclusters, ++local) {
        int tm, tn;
        tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn);
        (void)tm;
        const int ab = (Cfg::kAccBufs == 2) ? (local & 1) : 0;
        const uint32_t aph = static_cast<uint32_t>((Cfg::kAccBufs == 2 ? (local >> 1) : local) & 1);
        const uint32_t d_tmem = tmem_base + ab * TN;
        const uint32_t sfb_shift = static_cast<uint32_t>(((tn * TN) % 128) / 32);  // 0 or 2 columns
        const long long w1 = tracing ? clock64() : 0;
        if (!mbar_wait(&accempty[ab], aph ^ 1, wc, 32)) { ok = false; break; }
        if (tracing) { tr_b += clock64() - w1; if (t_commit) tr_c += clock64() - t_commit; }
        tc_fence_after();
        for (int kb = 0; kb < nk; ++kb) {
          const long long w2 = tracing ? clock64() : 0;
          if (!mbar_wait(&full[s], ph, wc, 33)) { ok = false; break; }
          if (tracing) tr_a += clock64() - w2;
          tc_fence_after();
          const uint32_t aaddr = smem_u32(smem + s * Cfg::kStageBytes);
          const uint32_t baddr = aaddr + Cfg::kABytes;
          uint32_t sfb_off = 0;  // column offset of the stage's scale-factor buffer
          if (unit_sf) {
            if (!sf_loaded) {  // plain FP4: the 0x7f scale-factor slot 0, copied once
              const uint32_t sfa_s = smem_u32(smem + Cfg::kSfRingOffset);
              const uint32_t sfb_s = sfa_s + Cfg::kSfaBytes;
#pragma unroll
              for (int a = 0; a < 4; ++a) {
                tmem_cp_32x128b_warpx4_pair(tmem_sfa + 4 * a, sdesc_noswz(sfa_s + 512 * a, 16, 128));
                tmem_cp_32x128b_warpx4_pair(tmem_sfb + 8 * a, sdesc_noswz(sfb_s + 512 * a, 16, 128));
                tmem_cp_32x128b_warpx4_pair(tmem_sfb + 8 * a + 4,
                                            sdesc_noswz(sfb_s + Cfg::kSfaBytes + 512 * a, 16, 128));
              }
              sf_loaded = true;
            }
          } else {
            // the copier warp has put this stage's scale factors into buffer sb
            if (!mbar_wait(&sf_ready[sb], sph, wc, 36)) { ok = false; break; }
            tc_fence_after();
            sfb_off = sb * Cfg::kSfCols;
          }
#pragma unroll
          for (int kk = 0; kk < 4 * kMxKsub; ++kk) {
            const int j = kk >> 2, k = kk & 3;
            const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
            const uint64_t adesc = sdesc_sw128(aaddr + j * Cfg::kAtom + k * 32, 16, 1024);
            const uint64_t bdesc = sdesc_sw128(baddr + j * Cfg::kBAtom + k * 32, 16, 1024);
            // MMA kk covers 64 K values = SF blocks 2kk, 2kk+1: atom kk/2, byte (2kk) % 4.
            const uint32_t sf_id = (2 * kk) & 3;
            const uint32_t atom = unit_sf ? 0u : static_cast<uint32_t>(kk >> 1);
            umma_mxf4_pair(d_tmem, adesc, bdesc, idesc_mxf4(256, TN, sf_id, sf_id),
                           tmem_sfa + sfb_off + 4 * atom, tmem_sfb + sfb_off + 8 * atom + sfb_shift, acc);
          }
          umma_commit_pair(empty_own + s * 8);
          umma_commit_pair(empty_peer + s * 8);
          if (!unit_sf) {
            umma_commit_pair(smem_u32(&sf_free[sb]));
            if (++sb == Cfg::kSfBufs) { sb = 0; sph ^= 1; }
          }
          if (++s == kMxStages) { s = 0; ph ^= 1; }
        }
        if (ok) {
          if (tracing) t_commit = clock64();
          umma_commit_pair(accfull_own + ab * 8);
          umma_commit_pair(accfull_peer + ab * 8);
        }
      }
      umma_commit_pair(smem_u32(teardown));
      mbar_wait(teardown, 0, wc, 34);
    }
  } else if (warp == 10) {
    // ---------------- scale-factor copier (leader only) ----------------
    // Moves each stage's scale factors shared memory -> TMEM (both CTAs, cta_group::2) into
    // one of kSfBufs column buffers, so the MMA thread issues only MMAs and commits. The
    // scale factors have their own shared-memory ring, so this runs ahead of the A/B data.
    if (leader && lane == 0 && !unit_sf) {
      const uint32_t sf_empty_own = smem_u32(sf_empty), sf_empty_peer = mapa_shared(smem_u32(sf_empty), peer);
      int s = 0;
      uint32_t ph = 0;
      int b = 0;
      uint32_t u = 0;
      bool ok = true;
      for (int t = cluster; t < num_tiles && ok; t += nclusters) {
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&sf_full[s], ph, wc, 37)) { ok = false; break; }
          if (!mbar_wait(&sf_free[b], u ^ 1, wc, 38)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sfa_s = smem_u32(smem + Cfg::kSfRingOffset + s * Cfg::kSfSlotBytes);
          const uint32_t sfb_s = sfa_s + Cfg::kSfaBytes;
          const uint32_t off = b * Cfg::kSfCols;
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            tmem_cp_32x128b_warpx4_pair(tmem_sfa + off + 4 * a, sdesc_noswz(sfa_s + 512 * a, 16, 128));
            tmem_cp_32x128b_warpx4_pair(tmem_sfb + off + 8 * a, sdesc_noswz(sfb_s + 512 * a, 16, 128));
            tmem_cp_32x128b_warpx4_pair(tmem_sfb + off + 8 * a + 4,
                                        sdesc_noswz(sfb_s + Cfg::kSfaBytes + 512 * a, 16, 128));
          }
          umma_commit_pair(smem_u32(&sf_ready[b]));
          umma_commit_pair(sf_empty_own + s * 8);   // slot s may be refilled (both CTAs)
          umma_commit_pair(sf_empty_peer + s * 8);
          if (++b == Cfg::kSfBufs) { b = 0; u ^= 1; }
          if (++s == kMxSfSlots) { s = 0; ph ^= 1; }
        }
      }
      umma_commit_pair(smem_u32(teardown));  // its commits to the peer land before teardown
    }
  } else if (warp == 11) {
    // ---------------- scale-factor loader (both CTAs) ----------------
    if (lane == 0 && !unit_sf) {
      const uint64_t pol = l2_policy_evict_last();
      const uint32_t sf_full_leader = mapa_shared(smem_u32(sf_full), 0);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = cluster; t < num_tiles && ok; t += nclusters) {
        int tm, tn;
        tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn);
        const int sfb_block = (tn * TN) / 128;  // first 128-row SF block the tile's B rows touch
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&sf_empty[s], ph ^ 1, wc, 39)) { ok = false; break; }
          uint8_t* sSfa = smem + Cfg::kSfRingOffset + s * Cfg::kSfSlotBytes;
          uint8_t* sSfb = sSfa + Cfg::kSfaBytes;
          if (leader) mbar_arrive_expect_tx(&sf_full[s], 2 * Cfg::kSfSlotBytes);
          const uint32_t fb = sf_full_leader + s * 8;
          // SF buffers viewed as rows of 256 B (an atom = 2 rows); a stage needs 4 atoms
          // (k groups 4kb..4kb+3) of one row block: one 8-row box. Boxes past the end of a
          // row block read the next block's scales for zero-filled K, past the buffer zeros.
          const int kg0 = kb * 4;
          tma_load_2d_pair(&tmSfa, fb, sSfa, 0, ((tm * 2 + static_cast<int>(rank)) * p.sf_kgroups + kg0) * 2, pol);
          tma_load_2d_pair(&tmSfb, fb, sSfb, 0, (sfb_block * p.sf_kgroups + kg0) * 2, pol);
          tma_load_2d_pair(&tmSfb, fb, sSfb + Cfg::kSfaBytes, 0, ((sfb_block + 1) * p.sf_kgroups + kg0) * 2, pol);
          if (++s == kMxSfSlots) { s = 0; ph ^= 1; }
        }
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int q = warp & 3;
    const uint32_t accempty_leader = mapa_shared(smem_u32(accempty), 0);
    float alpha = 1.f;
    if (p.scale_a) alpha *= __ldg(p.scale_a);
    if (p.scale_b) alpha *= __ldg(p.scale_b);
    if constexpr (TN == 192) {
      // warps 2..5: double-buffered accumulators, 32-byte direct stores (warps 6..9 idle)
      if (warp < 6) {
        int local = 0;
        for (int t = cluster; t < num_tiles; t += nclusters, ++local) {
          int tm, tn;
          tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn);
          const int ab = local & 1;
          const long long w3 = tracing ? clock64() : 0;
          if (!mbar_wait(&accfull[ab], static_cast<uint32_t>((local >> 1) & 1), wc, 35)) break;
          const long long w4 = tracing ? clock64() : 0;
          if (tracing) tr_a += w4 - w3;
          tc_fence_after();
          const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + ab * TN;
          const int row = tm * TM + static_cast<int>(rank) * 128 + q * 32 + lane;
          epilogue_tile_direct<OUT, TN>(tbase, p, row, tn * TN, alpha, [&] {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote_cta(accempty_leader + ab * 8);
          });
          if (tracing) tr_b += clock64() - w4;
        }
      }
    } else {
      // warps 2..9: lane quarter q, column half h; drain the single accumulator to registers
      const int h = (warp - 2) >> 2;
      // BF16 rows go out as 32-byte stores when C and its row pitch allow them
      const bool bf16_v8 = (reinterpret_cast<uintptr_t>(p.C) & 31u) == 0 && (p.ldc % 16) == 0;
      int local = 0;
      for (int t = cluster; t < num_tiles; t += nclusters, ++local) {
        int tm, tn;
        tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn);
        const long long w3 = tracing ? clock64() : 0;
        if (!mbar_wait(accfull, local & 1, wc, 35)) break;
        const long long w4 = tracing ? clock64() : 0;
        if (tracing) tr_a += w4 - w3;
        tc_fence_after();
        uint32_t r[128];
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + h * 128;
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(tbase + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * c]));
        tmem_ld_wait();
        if (tracing) tr_c += clock64() - w4;
        tc_fence_before();
        __syncwarp();
        // accumulator free: the next tile may start. The loads above have completed
        // (wait::ld), so a CTA-scope release suffices; a cluster-scope release here cost
        // about 1.5k cycles per tile with the MMA idle.
        if (lane == 0) mbar_arrive_remote_cta(accempty_leader);
        if (tracing) tr_b += clock64() - w4;  // drain time (TMEM -> registers)
        const int row = tm * TM + static_cast<int>(rank) * 128 + q * 32 + lane;
        if (row < p.M) {
          const int col0 = tn * TN + h * 128;
          if constexpr (OUT == Out::F32) {
#pragma unroll
            for (int g = 0; g < 16; ++g) {  // 16 groups of 8 columns, one 32-byte store each
              const int col = col0 + 8 * g;
              if (col >= p.N) break;
              float* dst = reinterpret_cast<float*>(p.C) + static_cast<size_t>(row) * p.ldc + col;
              uint32_t v[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) v[j] = __float_as_uint(__uint_as_float(r[8 * g + j]) * alpha);
              st_global_v8(dst, v);
            }
          } else {
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<size_t>(row) * p.ldc + col0;
#pragma unroll
            for (int g = 0; g < 8; ++g) {  // 8 groups of 16 columns
              const int col = col0 + 16 * g;
              if (col >= p.N) break;
              uint32_t v[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                __nv_bfloat162 b2 = __floats2bfloat162_rn(__uint_as_float(r[16 * g + 2 * j]) * alpha,
                                                          __uint_as_float(r[16 * g + 2 * j + 1]) * alpha);
                v[j] = *reinterpret_cast<uint32_t*>(&b2);
              }
              if (bf16_v8 && col + 16 <= p.N) {
                st_global_v8(dst + 16 * g, v);  // full 32-byte sector
              } else {
                *reinterpret_cast<uint4*>(dst + 16 * g) = make_uint4(v[0], v[1], v[2], v[3]);
                if (col + 8 < p.N) *reinterpret_cast<uint4*>(dst + 16 * g + 8) = make_uint4(v[4], v[5], v[6], v[7]);
              }
            }
          }
        }
      }
    }
  }

  if (tracing && lane == 0) {
    unsigned long long* tr = p.trace + static_cast<size_t>(blockIdx.x) * kTraceWords;
    if (warp == 0) tr[3] = tr_a;
    // words as in the other kernels except 6 (MMA thread: cycles from committing a finished
    // accumulator to seeing it free again) and 7 (epilogue: TMEM -> register drain cycles)
    if (warp == 1 && leader) { tr[1] = tr_a; tr[2] = tr_b; tr[6] = tr_c; }
    if (warp == 2) { tr[4] = tr_a; tr[5] = tr_b; tr[7] = tr_c; }
  }
  tc_fence_before();
  cluster_sync();
  if (p.trace && threadIdx.x == 0) p.trace[static_cast<size_t>(blockIdx.x) * kTraceWords] = clock64() - t_start;
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace bw
