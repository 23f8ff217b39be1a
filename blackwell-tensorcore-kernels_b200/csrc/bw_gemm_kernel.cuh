// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
// Replaces the reference's hot kernels:
//   gemm_mma_t      (src/gemm_mma.cu:23-141)      FP16 in / FP32 acc, A MxK, B KxN row-major
//   gemm_wmma_t     (src/gemm_wmma.cu:29-104)     same math through WMMA
//   gemm_lowprec_t  (src/gemm_mma_fp8.cu:89-223)  E4M3 / E2M1 / packed E2M1, "TN" layout
//
// One CTA per SM runs for the whole problem and walks output tiles of 128 x BN.
//   warp 0      TMA producer: one elected lane streams A/B k-slabs (128 B wide, 128B-swizzled)
//               into a STAGES-deep shared-memory ring guarded by full/empty mbarriers.
//   warp 1      allocates Tensor Memory; one elected lane issues tcgen05.mma for every
//               k-slab (4 MMAs of 32 bytes of K each) into one of ACC_BUFS TMEM accumulators
//               and commits slab release / accumulator-ready through tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld the 128 x BN FP32 accumulator (one row per thread),
//               release the TMEM buffer, scale, convert and store C.
// With ACC_BUFS = 2 the epilogue of tile i overlaps the main loop of tile i+1.
//
// Operand formats (KIND):
//   F16   A: MxK fp16 (K-major). B: KxN fp16 (N-major, B_MN = true) or NxK (B_MN = false).
//   F8    A: MxK e4m3, Bt: NxK e4m3 (both K-major).
//   MXF4  A: MxK/2 packed e2m1, Bt: NxK/2 packed e2m1, plus UE8M0 scale factors, one per
//         32 K elements, in the 128x4 tiled layout (see bw_sf_offset in bwgemm.h).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "bw_ptx.cuh"

namespace bw {

enum class Kind : int { F16 = 0, F8 = 1, MXF4 = 2 };
enum class Out : int { F32 = 0, BF16 = 1 };

constexpr int kBM = 128;          // rows of A per tile (one TMEM lane per row)
constexpr int kSlabBytes = 128;   // bytes of K per k-slab row (one 128B swizzle atom)
constexpr int kThreads = 192;     // 6 warps
constexpr int kEpiWarps = 4;
// Trace words per CTA (clock64 cycles unless noted): 0 total kernel cycles, 1 MMA waits on
// full slabs, 2 MMA waits on a free accumulator, 3 producer waits on empty slabs,
// 4 epilogue (warp 2) waits on a ready accumulator, 5 epilogue (warp 2) busy cycles,
// 6 tiles processed, 7 k-slabs issued by the MMA thread.
constexpr int kTraceWords = 8;
constexpr int kEpiBufBytes = 32 * 128;                   // per-warp staging buffer: 32 rows x 128 B
constexpr int kEpiBytes = kEpiWarps * 2 * kEpiBufBytes;  // two buffers per epilogue warp: 32 KB

template <Kind KIND>
struct KindTraits;
template <>
struct KindTraits<Kind::F16> {
  static constexpr int kElemsPerSlab = 64;  // 64 fp16 = 128 B
  static constexpr int kCoordPerSlab = 64;  // tensor-map units (elements) per slab
  static constexpr uint32_t kFmt = 0;       // F16
};
template <>
struct KindTraits<Kind::F8> {
  static constexpr int kElemsPerSlab = 128;  // 128 e4m3
  static constexpr int kCoordPerSlab = 128;
  static constexpr uint32_t kFmt = 0;        // E4M3
};
template <>
struct KindTraits<Kind::MXF4> {
  static constexpr int kElemsPerSlab = 256;  // 256 packed e2m1 = 128 B
  static constexpr int kCoordPerSlab = 128;  // the tensor map counts packed bytes
  static constexpr uint32_t kFmt = 1;
};

struct GemmParams {
  void* C;
  int M, N, K;
  int ldc;                     // elements between C rows
  const float* scale_a;        // optional per-tensor scales (device, may be null)
  const float* scale_b;
  const uint8_t* sfa;          // MXF4: A scale factors, tiled 128x4 layout
  const uint8_t* sfb;          // MXF4: B scale factors
  int sf_kgroups;              // MXF4: number of 4-block K groups per 128-row block
  int group_m;                 // raster: tile rows per group
  int splits;                  // single-CTA kernel: K splits per tile (>1: partials are TMA-reduce-added into zeroed C)
  int kb_per_split;            // k-slabs per split
  int hints;                   // bit 0: A/B loads evict_last (else evict_normal); bit 1: C stores evict_first;
                               // bit 2: B loads evict_first (single-CTA kernel)
  int* status;                 // device status word
  unsigned long long* trace;   // optional per-CTA wait-time trace (kTraceWords per CTA), or null
  unsigned long long budget_ns;
  // Fused all-gather (staged epilogue): peers[i] is another GPU's copy of C (opened through
  // CUDA IPC) at this shard's column offset; each staged chunk is also TMA-stored there.
  void* peers[7];
  int npeers;
  // Fused all-gather through NVSwitch multicast (staged epilogue): `mc` is the multicast
  // address of the M x ldc C that every rank has bound, at this shard's column offset; each
  // staged chunk is written once with multimem.st and lands in every rank's C. mc_plain = 1
  // writes it with plain stores instead (a single-GPU check of the same indexing).
  void* mc;
  int mc_plain;
};

template <Kind KIND, bool B_MN, int BN, int STAGES, int ACC_BUFS>
struct GemmCfg {
  static constexpr int kABytes = kBM * kSlabBytes;               // 16 KB
  static constexpr int kBBytes = BN * kSlabBytes;                // BN x 128 B
  static constexpr int kSfaBytes = (KIND == Kind::MXF4) ? 1024 : 0;        // 2 atoms of 512 B
  static constexpr int kSfbBytes = (KIND == Kind::MXF4) ? (BN / 128) * 1024 : 0;
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
  static constexpr int kAccCols = ACC_BUFS * BN;
  static constexpr int kSfaCols = (KIND == Kind::MXF4) ? 8 : 0;
  static constexpr int kSfbCols = (KIND == Kind::MXF4) ? 8 * (BN / 128) : 0;
  static constexpr int kNeedCols = kAccCols + kSfaCols + kSfbCols;
  static constexpr int kTmemCols = kNeedCols <= 32 ? 32 : kNeedCols <= 64 ? 64 : kNeedCols <= 128 ? 128
                                   : kNeedCols <= 256 ? 256 : 512;
  static_assert(kNeedCols <= 512, "TMEM budget exceeded");
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN");
  static_assert(KIND != Kind::MXF4 || BN % 128 == 0, "MXF4 tiles cover whole 128-row SF blocks");
  static constexpr int kEpiOffset = STAGES * kStageBytes;
  static constexpr int kBarOffset = kEpiOffset + kEpiBytes;
  // full[S], empty[S], accfull[ACC], accempty[ACC], teardown
  static constexpr int kNumBars = 2 * STAGES + 2 * ACC_BUFS + 1;
  static constexpr int kSmemBytes = kBarOffset + kNumBars * 8 + 16 + 1024;  // + align slack
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group_m, int& tm, int& tn) {
  const int per_group = group_m * tiles_n;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int gm = min(tiles_m - first_m, group_m);
  const int r = t - g * per_group;
  tm = first_m + r % gm;
  tn = r / gm;
}

// Epilogue of one warp for one accumulator tile: 32 TMEM lanes (= 32 output rows) x NCOLS
// FP32 columns. Each chunk (128 B per row: 32 fp32 or 64 bf16) goes registers -> one of the
// warp's two 4 KB staging buffers in shared memory, 128B-swizzled like the C tensor map so
// the 16-byte writes of a warp spread over all banks, and leaves through one TMA store
// (full 128 B lines; rows/columns outside C are clipped by the TMA unit). `release` runs
// once the last TMEM load of the tile has completed, so the MMA warp can reuse the buffer.

// Shared-memory-free epilogue: each thread writes its own row straight from registers with
// 256-bit stores, so every store fills whole 32-byte sectors. Needs 32-byte aligned C and
// N % 8 == 0 (checked on the host); used where the staging buffers would cost a pipeline stage.
template <Out OUT, int NCOLS, typename Release>
__device__ __forceinline__ void epilogue_tile_direct(uint32_t tbase, const GemmParams& p, int row, int col0,
                                                     float alpha, Release release) {
  static_assert(NCOLS % 32 == 0, "tile width must be whole 32-column chunks");
  const bool stream_out = (p.hints & 2) != 0;  // results go out with L2 evict-first priority
  const uint64_t pol = l2_policy_evict_first();
#pragma unroll 1
  for (int c = 0; c < NCOLS; c += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(tbase + c, r);
    tmem_ld_wait();
    if (c + 32 >= NCOLS) release();
    if (row >= p.M) continue;
    const int col = col0 + c;
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

// Tensor maps over the peers' copies of C for the fused all-gather (staged epilogue): each
// staged 32-row chunk leaves through one TMA store per destination, so the copy engine, not the
// epilogue warps, carries the NVLink traffic.
struct PeerMaps {
  CUtensorMap m[7];
};

// NB staging buffers per warp (a chunk's TMA stores must have read its buffer before the warp
// reuses it): more buffers keep more store bytes in flight, which is what a fused all-gather's
// remote stores need to cover the NVLink round trip.
template <Out OUT, int NCOLS, typename Release, int NB = 2>
__device__ __forceinline__ void epilogue_tile(uint32_t tbase, const CUtensorMap* tmC, int x0, int y0, float alpha,
                                              uint8_t* wbuf, int& uses, int lane, uint64_t store_policy,
                                              bool hinted, Release release, bool reduce_add = false,
                                              const PeerMaps* peer_maps = nullptr, int npeers = 0,
                                              const GemmParams* mcp = nullptr) {
  constexpr int kCols = (OUT == Out::F32) ? 32 : 64;  // columns per 128-byte row chunk
  static_assert(NCOLS % kCols == 0, "tile width must be whole 128-byte chunks");
  const uint32_t row_addr = smem_u32(wbuf) + lane * 128;
#pragma unroll 1
  for (int c = 0; c < NCOLS; c += kCols) {
    uint32_t r[kCols];
    tmem_ld_32x32b_x32(tbase + c, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
    if constexpr (kCols == 64) tmem_ld_32x32b_x32(tbase + c + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
    tmem_ld_wait();
    if (c + kCols >= NCOLS) release();
    const int bsel = uses % NB;
    if (uses >= NB) {
      if (lane == 0) bulk_wait_group_read<NB - 1>();
      __syncwarp();
    }
    const uint32_t base = row_addr + bsel * kEpiBufBytes;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t dst = base + ((j ^ (lane & 7)) << 4);
      if constexpr (OUT == Out::F32) {
        st_shared_v4(dst, __float_as_uint(__uint_as_float(r[4 * j]) * alpha),
                     __float_as_uint(__uint_as_float(r[4 * j + 1]) * alpha),
                     __float_as_uint(__uint_as_float(r[4 * j + 2]) * alpha),
                     __float_as_uint(__uint_as_float(r[4 * j + 3]) * alpha));
      } else {
        uint32_t w[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          __nv_bfloat162 v = __floats2bfloat162_rn(__uint_as_float(r[8 * j + 2 * h]) * alpha,
                                                   __uint_as_float(r[8 * j + 2 * h + 1]) * alpha);
          w[h] = *reinterpret_cast<uint32_t*>(&v);
        }
        st_shared_v4(dst, w[0], w[1], w[2], w[3]);
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (mcp != nullptr) {
      // Multicast gather: the warp copies the staged 32 x 128 B chunk out in 16-byte pieces,
      // 8 lanes per row (whole 128-byte lines), clipped to C like the TMA store would be.
      constexpr int kElemsPer16 = (OUT == Out::F32) ? 4 : 8;
      constexpr int kElemBytes = (OUT == Out::F32) ? 4 : 2;
      const uint32_t sbase = smem_u32(wbuf) + bsel * kEpiBufBytes;
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int li = it * 32 + lane;
        const int i = li >> 3, j = li & 7;
        const int row = y0 + i, col = x0 + c + j * kElemsPer16;
        if (row < mcp->M && col < mcp->N) {
          const uint4 v = ld_shared_v4(sbase + i * 128 + ((j ^ (i & 7)) << 4));
          char* dst = static_cast<char*>(mcp->mc) + (static_cast<size_t>(row) * mcp->ldc + col) * kElemBytes;
          if (mcp->mc_plain) st_global_v4(dst, v);
          else multimem_st_v4(dst, v);
        }
      }
      __syncwarp();
      ++uses;
      continue;
    }
    if (lane == 0) {
      if (reduce_add) tma_reduce_add_2d(tmC, wbuf + bsel * kEpiBufBytes, x0 + c, y0);
      else if (hinted) tma_store_2d_hint(tmC, wbuf + bsel * kEpiBufBytes, x0 + c, y0, store_policy);
      else tma_store_2d(tmC, wbuf + bsel * kEpiBufBytes, x0 + c, y0);
      for (int q = 0; q < npeers; ++q) tma_store_2d(&peer_maps->m[q], wbuf + bsel * kEpiBufBytes, x0 + c, y0);
      bulk_commit_group();
    }
    ++uses;
  }
}

template <Kind KIND, bool B_MN, int BN, int STAGES, int ACC_BUFS, Out OUT>
__global__ void __launch_bounds__(kThreads, 1)
    bw_tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
  using Cfg = GemmCfg<KIND, B_MN, BN, STAGES, ACC_BUFS>;
  constexpr int KE = KindTraits<KIND>::kElemsPerSlab;
  constexpr int KX = KindTraits<KIND>::kCoordPerSlab;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOffset);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* accfull = bars + 2 * STAGES;
  uint64_t* accempty = bars + 2 * STAGES + ACC_BUFS;
  uint64_t* teardown = bars + 2 * STAGES + 2 * ACC_BUFS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (p.M + kBM - 1) / kBM;
  const int tiles_n = (p.N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int nk_all = (p.K + KE - 1) / KE;
  // Work unit u = (tile u / splits, K split u % splits): k-slabs [kb0, kb1) of that tile.
  const int splits = p.splits > 1 ? p.splits : 1;
  const int kb_per = splits > 1 ? p.kb_per_split : nk_all;
  const int num_units = num_tiles * splits;
  const WaitCtl wc{abort_flag, p.status, p.budget_ns};

  if constexpr (KIND == Kind::MXF4) {
    // Scale-factor slots a tail slab does not refill must hold finite scales (they
    // multiply zero-filled operands); start them at 0x7f = 2^0.
    for (int s = 0; s < STAGES; ++s) {
      uint32_t* sf = reinterpret_cast<uint32_t*>(smem + s * Cfg::kStageBytes + Cfg::kABytes + Cfg::kBBytes);
      for (int i = threadIdx.x; i < (Cfg::kSfaBytes + Cfg::kSfbBytes) / 4; i += kThreads) sf[i] = 0x7f7f7f7fu;
    }
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < ACC_BUFS; ++b) { mbar_init(&accfull[b], 1); mbar_init(&accempty[b], kEpiWarps * 32); }
    mbar_init(teardown, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) { tma_prefetch_desc(&tmA); tma_prefetch_desc(&tmB); tma_prefetch_desc(&tmC); }
  if (warp == 1) { tmem_alloc(tmem_slot, Cfg::kTmemCols); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol_a = (p.hints & 1) ? l2_policy_evict_last() : l2_policy_evict_normal();
      const uint64_t pol_b = (p.hints & 4) ? l2_policy_evict_first() : pol_a;  // streamed-once B
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        int tm, tn;
        tile_coords(u / splits, tiles_m, tiles_n, p.group_m, tm, tn);
        const int kb0 = (u % splits) * kb_per, kb1 = min(nk_all, kb0 + kb_per);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, wc, 1)) { ok = false; break; }
          uint8_t* sA = smem + s * Cfg::kStageBytes;
          uint8_t* sB = sA + Cfg::kABytes;
          uint32_t tx = Cfg::kABytes + Cfg::kBBytes;
          uint32_t sfa_bytes = 0, sfb_rbs = 0;
          if (KIND == Kind::MXF4 && p.sfa != nullptr) {
            // A k-slab of 256 K covers SF groups 2kb, 2kb+1; the last slab may have only one,
            // and the last B tile may cover fewer than BN/128 row blocks.
            sfa_bytes = (2 * kb + 1 < p.sf_kgroups) ? 1024u : 512u;
            const int rb_total = (p.N + 127) / 128;
            sfb_rbs = min(BN / 128, rb_total - tn * (BN / 128));
            tx += sfa_bytes * (1 + sfb_rbs);
          }
          mbar_arrive_expect_tx(&full[s], tx);
          tma_load_2d(&tmA, &full[s], sA, kb * KX, tm * kBM, pol_a);
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(&tmB, &full[s], sB + j * 64 * kSlabBytes, tn * BN + 64 * j, kb * 64, pol_b);
          } else {
            tma_load_2d(&tmB, &full[s], sB, kb * KX, tn * BN, pol_b);
          }
          if (KIND == Kind::MXF4 && p.sfa != nullptr) {
            // Scale factors: tiled layout = [row block][k group of 4 SF][512 B]. One stage
            // covers 256 K = 8 SF per row = 2 k groups = 1 KB contiguous per row block.
            uint8_t* sSfa = sB + Cfg::kBBytes;
            uint8_t* sSfb = sSfa + Cfg::kSfaBytes;
            const size_t kg0 = static_cast<size_t>(kb) * 2;
            bulk_load(sSfa, p.sfa + (static_cast<size_t>(tm) * p.sf_kgroups + kg0) * 512, sfa_bytes, &full[s]);
            for (uint32_t rb = 0; rb < sfb_rbs; ++rb)
              bulk_load(sSfb + rb * 1024,
                        p.sfb + (static_cast<size_t>(tn * (BN / 128) + rb) * p.sf_kgroups + kg0) * 512, sfa_bytes,
                        &full[s]);
          }
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t idesc;
      if constexpr (KIND == Kind::MXF4) idesc = 0;  // built per k-step (scale-factor byte ids)
      else idesc = idesc_dense(KindTraits<KIND>::kFmt, KindTraits<KIND>::kFmt, B_MN, kBM, BN);
      const uint32_t tmem_sfa = tmem_base + Cfg::kAccCols;
      const uint32_t tmem_sfb = tmem_sfa + Cfg::kSfaCols;
      int s = 0;
      uint32_t ph = 0;
      int local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++local) {
        const int b = local % ACC_BUFS;
        const uint32_t aph = (local / ACC_BUFS) & 1;
        const int kb0 = (u % splits) * kb_per, kb1 = min(nk_all, kb0 + kb_per);
        if (!mbar_wait(&accempty[b], aph ^ 1, wc, 2)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[s], ph, wc, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t aaddr = smem_u32(smem + s * Cfg::kStageBytes);
          const uint32_t baddr = aaddr + Cfg::kABytes;
          if (KIND == Kind::MXF4 && (p.sfa != nullptr || (kb == kb0 && local == 0))) {
            // Per-slab scale factors; with no SF arrays (plain FP4) the 0x7f-filled slots are
            // copied once and every block scale stays 2^0.
            const uint32_t sfa_s = baddr + Cfg::kBBytes;
            const uint32_t sfb_s = sfa_s + Cfg::kSfaBytes;
            // 512 B atom = 32 rows x 16 B, no swizzle; replicated to the 4 lane quarters.
#pragma unroll
            for (int a = 0; a < 2; ++a) {
              tmem_cp_32x128b_warpx4(tmem_sfa + a * 4, sdesc_noswz(sfa_s + a * 512, 16, 128));
#pragma unroll
              for (int rb = 0; rb < BN / 128; ++rb)
                tmem_cp_32x128b_warpx4(tmem_sfb + a * (BN / 128) * 4 + rb * 4,
                                       sdesc_noswz(sfb_s + rb * 1024 + a * 512, 16, 128));
            }
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
            const uint64_t adesc = sdesc_sw128(aaddr + k * 32, 16, 1024);
            uint64_t bdesc;
            if constexpr (B_MN) bdesc = sdesc_sw128(baddr + k * 16 * kSlabBytes, 64 * kSlabBytes, 1024);
            else bdesc = sdesc_sw128(baddr + k * 32, 16, 1024);
            if constexpr (KIND == Kind::F16) {
              umma_f16(d_tmem, adesc, bdesc, idesc, acc);
            } else if constexpr (KIND == Kind::F8) {
              umma_f8f6f4(d_tmem, adesc, bdesc, idesc, acc);
            } else {
              // k-step k uses SF blocks 2k, 2k+1 = atom k/2, bytes (2k)%4 .. +1.
              const uint32_t sf_id = (2 * k) & 3;
              const uint32_t id = idesc_mxf4(kBM, BN, sf_id, sf_id);
              umma_mxf4(d_tmem, adesc, bdesc, id, tmem_sfa + (k >> 1) * 4,
                        tmem_sfb + (k >> 1) * (BN / 128) * 4, acc);
            }
          }
          umma_commit(&empty[s]);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (ok) umma_commit(&accfull[b]);
      }
      // Make sure every MMA this thread issued has retired before TMEM is released.
      umma_commit(teardown);
      mbar_wait(teardown, 0, WaitCtl{abort_flag, p.status, p.budget_ns}, 4);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;                  // TMEM lane quarter this warp may access
    const uint64_t store_pol = l2_policy_evict_first();
    uint8_t* wbuf = smem + Cfg::kEpiOffset + (warp - 2) * 2 * kEpiBufBytes;
    int uses = 0;
    float alpha = 1.f;
    if (p.scale_a) alpha *= __ldg(p.scale_a);
    if (p.scale_b) alpha *= __ldg(p.scale_b);
    int local = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++local) {
      int tm, tn;
      tile_coords(u / splits, tiles_m, tiles_n, p.group_m, tm, tn);
      const int b = local % ACC_BUFS;
      const uint32_t aph = (local / ACC_BUFS) & 1;
      if (!mbar_wait(&accfull[b], aph, wc, 5)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + b * BN;
      epilogue_tile<OUT, BN>(tbase, &tmC, tn * BN, tm * kBM + q * 32, alpha, wbuf, uses, lane, store_pol,
                             (p.hints & 2) != 0, [&] {
        tc_fence_before();
        mbar_arrive(&accempty[b]);
      }, splits > 1);
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace bw
