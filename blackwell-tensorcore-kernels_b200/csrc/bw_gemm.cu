// GEMM entry points of the C ABI: argument checks, TMA descriptors, tile-shape choice and
// launch of the persistent tcgen05 kernel (bw_gemm_kernel.cuh).
#include <cstdlib>

#include "bw_gemm_kernel.cuh"
#include "bw_gemm_pair.cuh"
#include "bw_gemm_pair_mx.cuh"
#include "bw_gemm_pair_wide.cuh"
#include "bw_gemm_panel.cuh"
#include "bw_runtime.cuh"

namespace bw {
namespace {

int env_int(const char* name, int dflt) {
  const char* s = getenv(name);
  if (!s || !*s) return dflt;
  return atoi(s);
}

template <Kind KIND, bool B_MN, int BN, int STAGES, int ACC_BUFS, Out OUT>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, GemmParams p, cudaStream_t stream,
           const DeviceState& d) {
  using Cfg = GemmCfg<KIND, B_MN, BN, STAGES, ACC_BUFS>;
  auto kern = bw_tc_gemm_kernel<KIND, B_MN, BN, STAGES, ACC_BUFS, OUT>;
  static bool attr_done[64] = {};
  int dev = 0;
  BW_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev & 63]) {
    BW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    attr_done[dev & 63] = true;
  }
  const int tiles = ((p.M + kBM - 1) / kBM) * ((p.N + BN - 1) / BN) * (p.splits > 1 ? p.splits : 1);
  int grid = tiles < d.sms ? tiles : d.sms;
  const int cap = env_int("BW_MAX_CTAS", 0);
  if (cap > 0 && grid > cap) grid = cap;
  p.trace = nullptr;  // the single-CTA kernel has no trace points
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, tc, p);
  BW_CUDA(cudaGetLastError());
  return BW_OK;
}

// Co-resident CTA pairs of a persistent `__cluster_dims__(2,1,1)` kernel (clusters must fit
// inside one GPC, so this can be below sms / 2); falls back to sms / 2 if the query fails.
template <typename Kernel>
int pair_clusters_resident(Kernel kern, int threads, int smem_bytes, const DeviceState& d) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (d.sms / 2), 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = d.sms / 2;
  }
  return n;
}

template <Kind KIND, bool B_MN, int STAGES, Out OUT, bool DIRECT_EPI, int KSUB, int TN = 256, int EPI_BUFS = 2>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, GemmParams p,
                cudaStream_t stream, const DeviceState& d, const PeerMaps* pm = nullptr) {
  static const PeerMaps no_peers{};
  using Cfg = PairCfg<KIND, STAGES, DIRECT_EPI, KSUB, TN, EPI_BUFS>;
  auto kern = bw_tc_gemm_pair_kernel<KIND, B_MN, STAGES, OUT, DIRECT_EPI, KSUB, TN, EPI_BUFS>;
  static bool attr_done[64] = {};
  int dev = 0;
  BW_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev & 63]) {
    BW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    attr_done[dev & 63] = true;
  }
  // Persistent grid: as many CTA pairs as can be co-resident (clusters must sit inside one
  // GPC, so this can be below sms/2).
  static int max_clusters[64] = {};
  if (max_clusters[dev & 63] == 0) {
    max_clusters[dev & 63] = pair_clusters_resident(kern, kThreads, Cfg::kSmemBytes, d);
  }
  const int tiles = ((p.M + 255) / 256) * ((p.N + TN - 1) / TN);
  const int resident = max_clusters[dev & 63];
  int clusters = tiles < resident ? tiles : resident;
  const int cap = env_int("BW_MAX_CTAS", 0);
  if (cap > 1 && clusters > cap / 2) clusters = cap / 2;
  p.trace = trace_buffer(2 * clusters);
  kern<<<2 * clusters, kThreads, Cfg::kSmemBytes, stream>>>(ta, tb, tc, pm ? *pm : no_peers, p);
  BW_CUDA(cudaGetLastError());
  return BW_OK;
}

// Pair kernels stage two 128-byte K atoms per pipeline stage (3 x 64 KB): the MMA thread then
// issues 8 MMAs per barrier round trip instead of 4, measured at 90-93% of the tcgen05 peak
// per clock versus 75% with one atom per stage. The epilogue stores 32-byte sectors straight
// from registers when C is 32-byte aligned (no staging shared memory), else stages through
// shared memory and TMA stores.
// Every 256-bit store must start on a 32-byte boundary: the base of C and every row pitch
// (N * element bytes) must be multiples of 32 (BF16 output therefore needs N % 16 == 0).
bool direct_epilogue_ok(const void* C, int N, int elem_bytes) {
  if (env_int("BW_EPI_DIRECT", 1) == 0) return false;
  return (reinterpret_cast<uintptr_t>(C) & 31u) == 0 && (static_cast<long long>(N) * elem_bytes) % 32 == 0;
}

// CTA pairs (256 x 256 tiles) when the problem fills at least most of the SM pairs.
bool use_pair(int M, int N, const DeviceState& d) {
  const int forced = env_int("BW_PAIR", -1);
  if (forced == 0) return false;
  if (forced == 1) return true;
  const long tiles = static_cast<long>((M + 255) / 256) * ((N + 255) / 256);
  return tiles >= d.sms / 4;  // e.g. 2048^3 (64 tiles): pair 828 vs single-CTA 691 TFLOP/s
}

// 256 x 512 tiles (bw_gemm_pair_wide.cuh): less L2 -> SM traffic per FLOP than 256 x 256.
template <Kind KIND, bool B_MN, Out OUT>
int launch_pair_wide(const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p, cudaStream_t stream,
                     const DeviceState& d) {
  auto kern = bw_tc_gemm_pair_wide_kernel<KIND, B_MN, OUT>;
  static bool attr_done[64] = {};
  static int max_clusters[64] = {};
  int dev = 0;
  BW_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev & 63]) {
    BW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, WideCfg::kSmemBytes));
    attr_done[dev & 63] = true;
    max_clusters[dev & 63] = pair_clusters_resident(kern, kWideThreads, WideCfg::kSmemBytes, d);
  }
  const int tiles = ((p.M + 255) / 256) * ((p.N + 511) / 512);
  const int resident = max_clusters[dev & 63];
  const int clusters = tiles < resident ? tiles : resident;
  p.trace = nullptr;
  kern<<<2 * clusters, kWideThreads, WideCfg::kSmemBytes, stream>>>(ta, tb, p);
  BW_CUDA(cudaGetLastError());
  return BW_OK;
}

template <Out OUT, int TN>
int launch_pair_mx(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tsa, const CUtensorMap& tsb,
                   GemmParams p, cudaStream_t stream, const DeviceState& d) {
  using Cfg = MxPairCfg<TN>;
  auto kern = bw_tc_gemm_pair_mx_kernel<OUT, TN>;
  static bool attr_done[64] = {};
  static int max_clusters[64] = {};
  int dev = 0;
  BW_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev & 63]) {
    BW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes));
    attr_done[dev & 63] = true;
    max_clusters[dev & 63] = pair_clusters_resident(kern, kMxThreads, Cfg::kSmemBytes, d);
  }
  const int tiles = ((p.M + 255) / 256) * ((p.N + TN - 1) / TN);
  const int resident = max_clusters[dev & 63];
  const int clusters = tiles < resident ? tiles : resident;
  p.trace = trace_buffer(2 * clusters);  // word 0 (kernel cycles) only
  kern<<<2 * clusters, kMxThreads, Cfg::kSmemBytes, stream>>>(ta, tb, tsa, tsb, p);
  BW_CUDA(cudaGetLastError());
  return BW_OK;
}

// Output tensor map for the TMA-store epilogue: 32 rows x 128 B boxes, 128B swizzle.
// C map with an explicit row pitch (elements), e.g. one column shard inside a wider C.
int make_c_map_ld(CUtensorMap* tc, void* C, int M, int N, int ld, int out_dtype) {
  if (out_dtype == BW_OUT_BF16)
    return make_tmap_2d(tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, C, N, M, uint64_t(ld) * 2, 64, 32);
  return make_tmap_2d(tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, C, N, M, uint64_t(ld) * 4, 32, 32);
}

int make_c_map(CUtensorMap* tc, void* C, int M, int N, int out_dtype) {
  if (out_dtype == BW_OUT_BF16)
    return make_tmap_2d(tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, C, N, M, uint64_t(N) * 2, 64, 32);
  return make_tmap_2d(tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, C, N, M, uint64_t(N) * 4, 32, 32);
}

// Fused all-gather of column shards: this rank's C columns start at col0 of a row-major
// M x ldc buffer, and the same bytes go to the same place in each peer's buffer.
struct GatherCtx {
  int ldc;
  int col0;
  int npeers;
  void* peers[7];
  void* mc = nullptr;  // multicast address of C_full (all ranks bound): replaces the peer stores
  int mc_plain = 0;
};

GemmParams base_params(const DeviceState& d, void* C, int M, int N, int K) {
  GemmParams p{};
  p.C = C;
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = N;
  p.group_m = env_int("BW_GROUP_M", 16);
  // bit 0: A and B tiles evict-last in L2 (re-read by neighbouring tiles); bit 2: B evict-first
  // instead, for M <= 256 where each B tile is read by one tile row (at most two)
  p.hints = env_int("BW_L2_HINTS", M <= 256 ? 5 : 1);
  p.splits = 1;
  p.kb_per_split = 0;
  if (p.group_m < 1) p.group_m = 1;
  p.status = d.status;
  p.budget_ns = wait_budget_ns();
  return p;
}

int check_common(const void* A, const void* B, const void* C, int M, int N, int K) {
  if (M < 0 || N < 0 || K < 0) return set_error(BW_ERR_INVALID, "negative size M=%d N=%d K=%d", M, N, K);
  if (M == 0 || N == 0) return BW_OK;
  if (!C) return set_error(BW_ERR_INVALID, "C is null");
  if (K > 0 && (!A || !B)) return set_error(BW_ERR_INVALID, "A or B is null");
  if (!aligned16(A) || !aligned16(B) || !aligned16(C))
    return set_error(BW_ERR_INVALID, "A, B and C must be 16-byte aligned");
  return BW_OK;
}

// Split-K for HBM-bound short-and-wide problems (M <= 256, e.g. the decode-style 128 x 65536):
// 128 x 256 single-CTA tiles split along K until there are >= 4 work units per SM, each split
// >= 8 k-slabs; partial tiles are added into C (zeroed first, in stream order) by the TMA
// reduce-add store. FP32 output only. Returns the split count (1 = no split).
// FP32 outputs add the partial tiles into C; BF16 outputs add them into an FP32 workspace that
// one conversion pass turns into C (BW_SPLITK_BF16=0 keeps BF16 outputs unsplit).
int choose_splits(int M, int N, int nk, int out_elem, const DeviceState& d) {
  const int forced = env_int("BW_SPLITK", -1);
  if (forced >= 1) return forced;
  if (forced == 0 || M > 256) return 1;
  if (out_elem != 4 && env_int("BW_SPLITK_BF16", 1) == 0) return 1;
  const long tiles = static_cast<long>((M + 127) / 128) * ((N + 255) / 256);
  int s = 1;
  while (s < 8 && tiles * s < 4L * d.sms && nk / (2 * s) >= 8) s *= 2;
  return s;
}

// Prefer 128 x 256 tiles; fall back to 128 x 128 when the wide tiles would leave SMs idle.
bool use_narrow(int M, int N, const DeviceState& d) {
  const int forced = env_int("BW_TILE_N", 0);
  if (forced == 128) return true;
  if (forced == 256) return false;
  const long tiles256 = static_cast<long>((M + 127) / 128) * ((N + 255) / 256);
  return tiles256 < d.sms;
}

// Column-panel kernel (bw_gemm_panel.cuh) for M <= 256: the panel width W (a multiple of 32,
// of 64 for an N-major B; MT x W <= 512 TMEM columns with MT = ceil(M / 128) accumulators) with
// the least work per SM, ceil(panels / SMs) x W (ties go to the wider panel), among widths of at
// least 96 x MT columns that keep 3/4 of the SMs busy; 0 when none exists or the kernel does not
// apply: M > 256, K < 512, C not 32-byte aligned per row (direct stores). Narrow panels lose
// because each CTA re-reads all MT x 128 rows of A (from L2) for its W columns of B: measured,
// 128 x 8192 x 8192 FP16 at W = 64 took 47.8 us against 31.9 us split-K, W = 112..448 were 8-38%
// faster than split-K, and 256 x 65536 x 8192 FP16 at W = 64 took 529 us against 280 us.
// BW_PANEL = 0 disables the kernel; 1 forces it wherever it can run (any width from 32 / 64 up,
// any number of panels); an explicit BW_SPLITK count selects split-K.
int panel_width(int M, int N, int K, bool gran64, const void* C, int elem, const DeviceState& d, int* mt) {
  const int forced = env_int("BW_PANEL", -1);
  if (forced == 0 || M > 256 || !direct_epilogue_ok(C, N, elem)) return 0;
  if (forced != 1 && env_int("BW_SPLITK", -1) >= 1) return 0;
  if (forced != 1 && K < 512) return 0;
  *mt = M > 128 ? 2 : 1;
  const int gran = gran64 ? 64 : 32;
  const int wmax = kPanelMaxW / *mt;
  const int wmin = forced == 1 ? gran : (96 * *mt + gran - 1) / gran * gran;
  long best_cost = -1;
  int W = 0;
  for (int w = wmin; w <= wmax; w += gran) {
    const long panels = (static_cast<long>(N) + w - 1) / w;
    if (forced != 1 && panels * 4 < 3L * d.sms) continue;
    const long cost = (panels + d.sms - 1) / d.sms * w;
    if (best_cost < 0 || cost <= best_cost) {
      best_cost = cost;
      W = w;
    }
  }
  return W;
}

template <Kind KIND, bool B_MN, Out OUT, int MT>
int launch_panel_mt(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int W, int b_box,
                    cudaStream_t stream) {
  auto kern = bw_tc_gemm_panel_kernel<KIND, B_MN, OUT, MT>;
  constexpr int kMaxSmem = 232448;
  static bool attr_done[64] = {};
  int dev = 0;
  BW_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev & 63]) {
    BW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
    attr_done[dev & 63] = true;
  }
  PanelParams pp;
  pp.W = W;
  pp.panels = (p.N + W - 1) / W;
  pp.stage_bytes = MT * kBM * kSlabBytes + W * kSlabBytes;
  pp.stages = (kMaxSmem - panel_smem_bytes(0, 0)) / pp.stage_bytes;
  if (pp.stages > kPanelMaxStages) pp.stages = kPanelMaxStages;
  if (pp.stages < 2) return set_error(BW_ERR_INVALID, "panel width %d leaves fewer than 2 stages", W);
  pp.b_box = b_box;
  kern<<<pp.panels, kThreads, panel_smem_bytes(pp.stages, pp.stage_bytes), stream>>>(ta, tb, p, pp);
  BW_CUDA(cudaGetLastError());
  return BW_OK;
}

template <Kind KIND, bool B_MN, Out OUT>
int launch_panel(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int W, int b_box, int mt,
                 cudaStream_t stream) {
  if (mt == 2) return launch_panel_mt<KIND, B_MN, OUT, 2>(ta, tb, p, W, b_box, stream);
  return launch_panel_mt<KIND, B_MN, OUT, 1>(ta, tb, p, W, b_box, stream);
}

// C (BF16) = workspace (FP32; scales already applied by the split-K epilogue), 8 per thread.
__global__ void k_f32_to_bf16(const float4* __restrict__ src, uint4* __restrict__ dst, long long n8) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n8; i += stride) {
    const float4 a = src[2 * i], b = src[2 * i + 1];
    __nv_bfloat162 h0 = __floats2bfloat162_rn(a.x, a.y), h1 = __floats2bfloat162_rn(a.z, a.w);
    __nv_bfloat162 h2 = __floats2bfloat162_rn(b.x, b.y), h3 = __floats2bfloat162_rn(b.z, b.w);
    dst[i] = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                        *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
  }
}

// Split-K launch of the single-CTA 128 x 256 kernel: partial tiles are TMA-reduce-added into C
// zeroed in stream order (FP32 C), or for BF16 C into a per-stream FP32 workspace that one
// conversion pass turns into C. BW_ERR_UNSUPPORTED (BF16 only) when every workspace slot
// belongs to another stream: the caller then runs unsplit.
template <Kind KIND, bool B_MN>
int launch_split(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, GemmParams p, void* C,
                 int out_dtype, cudaStream_t s, DeviceState& d) {
  const size_t mn = static_cast<size_t>(p.M) * p.N;
  if (out_dtype == BW_OUT_F32) {
    BW_CUDA(cudaMemsetAsync(C, 0, 4 * mn, s));
    return launch<KIND, B_MN, 256, 4, 2, Out::F32>(ta, tb, tc, p, s, d);
  }
  float* ws = nullptr;
  int r = splitk_workspace(d, s, 4 * mn, &ws);
  if (r != BW_OK) return r;
  CUtensorMap tw;
  if ((r = make_c_map(&tw, ws, p.M, p.N, BW_OUT_F32)) != BW_OK) return r;
  p.C = ws;
  BW_CUDA(cudaMemsetAsync(ws, 0, 4 * mn, s));
  if ((r = launch<KIND, B_MN, 256, 4, 2, Out::F32>(ta, tb, tw, p, s, d)) != BW_OK) return r;
  const long long n8 = static_cast<long long>(mn / 8);  // N % 8 == 0
  long long blocks = (n8 + 255) / 256;
  if (blocks > 8LL * d.sms) blocks = 8LL * d.sms;
  if (blocks < 1) blocks = 1;
  k_f32_to_bf16<<<static_cast<int>(blocks), 256, 0, s>>>(reinterpret_cast<const float4*>(ws), static_cast<uint4*>(C),
                                                          n8);
  BW_CUDA(cudaGetLastError());
  return BW_OK;
}

size_t out_elem_bytes(int out_dtype) { return out_dtype == BW_OUT_BF16 ? 2 : 4; }

// Even k-slab ranges with no empty split.
int set_splits(GemmParams& p, int splits, int nk) {
  if (splits < 1 || nk < 1) return set_error(BW_ERR_INVALID, "bad split-K configuration");
  p.kb_per_split = (nk + splits - 1) / splits;
  p.splits = (nk + p.kb_per_split - 1) / p.kb_per_split;
  return BW_OK;
}

// With a GatherCtx, C is the row-major M x g->ldc buffer that receives this rank's N columns at
// g->col0, and every peer receives the same: the CTA-pair kernel with the staged (TMA-store)
// epilogue and one extra tensor map per peer. TMA needs 16-byte aligned bases and row pitches.
int gather_check(const GatherCtx* g, const void* C, int N, int K, int elem) {
  if (!g) return BW_OK;
  if (K <= 0) return set_error(BW_ERR_INVALID, "fused gather needs K > 0");
  if (g->npeers < 0 || g->npeers > 7) return set_error(BW_ERR_INVALID, "fused gather: %d peers (at most 7)", g->npeers);
  const size_t off = static_cast<size_t>(g->col0) * elem;
  if (((reinterpret_cast<uintptr_t>(C) + off) & 15u) || (static_cast<size_t>(g->ldc) * elem) % 16 != 0 ||
      (static_cast<size_t>(N) * elem) % 16 != 0)
    return set_error(BW_ERR_INVALID, "fused gather needs 16-byte aligned C, column offset and row pitch");
  for (int i = 0; i < g->npeers; ++i)
    if (!g->peers[i] || (reinterpret_cast<uintptr_t>(g->peers[i]) & 15u))
      return set_error(BW_ERR_INVALID, "fused gather: peer buffer %d is null or not 16-byte aligned", i);
  return BW_OK;
}

// Fused gather with remote stores: 2 pipeline stages and 6 staging buffers per epilogue warp
// (24 KB of chunks in flight per warp instead of 8 KB) when BW_GATHER_STAGING=6, the default
// being decided by measurement; the multicast form keeps 3 stages (its stores do not hold
// the staging buffers).
bool gather_deep_staging(const GatherCtx* g) {
  if (!g || g->mc || g->npeers == 0) return false;
  return env_int("BW_GATHER_STAGING", 2) == 6;
}

void gather_apply(const GatherCtx* g, GemmParams& p, int elem) {
  if (!g) return;
  p.C = static_cast<char*>(p.C) + static_cast<size_t>(g->col0) * elem;
  p.ldc = g->ldc;
  p.npeers = g->npeers;
  for (int i = 0; i < g->npeers; ++i) p.peers[i] = static_cast<char*>(g->peers[i]) + static_cast<size_t>(g->col0) * elem;
  if (g->mc) {
    p.mc = static_cast<char*>(g->mc) + static_cast<size_t>(g->col0) * elem;
    p.mc_plain = g->mc_plain;
    p.C = nullptr;  // only multimem stores may touch a multicast address
  }
}

int gemm_f16_impl(const void* A, const void* B, float* C, int M, int N, int K, cudaStream_t s, bool b_mn,
                  const GatherCtx* g = nullptr) {
  int r = check_common(A, B, C, M, N, K);
  if (r != BW_OK || M == 0 || N == 0) return r;
  if (K % 8 != 0 || N % 8 != 0)
    return set_error(BW_ERR_INVALID, "fp16 GEMM needs K %% 8 == 0 and N %% 8 == 0 (got N=%d K=%d)", N, K);
  if ((r = gather_check(g, C, N, K, 4)) != BW_OK) return r;
  DeviceState* d;
  if ((r = ensure_device(&d)) != BW_OK) return r;
  if (K == 0) { BW_CUDA(cudaMemsetAsync(C, 0, sizeof(float) * size_t(M) * N, s)); return BW_OK; }
  int pmt = 1;
  if (const int pw = g ? 0 : panel_width(M, N, K, b_mn, C, 4, *d, &pmt)) {
    const int box = b_mn ? 64 : (pw <= 256 ? pw : pw / 2);
    CUtensorMap ta, tb;
    if ((r = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, A, K, M, uint64_t(K) * 2, 64, 128)) != BW_OK) return r;
    if (b_mn) r = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, B, N, K, uint64_t(N) * 2, 64, 64);
    else r = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, B, K, N, uint64_t(K) * 2, 64, box);
    if (r != BW_OK) return r;
    GemmParams p = base_params(*d, C, M, N, K);
    p.hints = env_int("BW_L2_HINTS", 0);
    if (b_mn) return launch_panel<Kind::F16, true, Out::F32>(ta, tb, p, pw, box, pmt, s);
    return launch_panel<Kind::F16, false, Out::F32>(ta, tb, p, pw, box, pmt, s);
  }
  const int splits = g ? 1 : choose_splits(M, N, (K + 63) / 64, 4, *d);
  const bool pair = g || (splits == 1 && use_pair(M, N, *d));
  const bool narrow = !pair && splits == 1 && use_narrow(M, N, *d);
  const int bn = pair ? 128 : narrow ? 128 : 256;
  CUtensorMap ta, tb;
  if ((r = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, A, K, M, uint64_t(K) * 2, 64, 128)) != BW_OK) return r;
  if (b_mn) r = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, B, N, K, uint64_t(N) * 2, 64, 64);
  else r = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, B, K, N, uint64_t(K) * 2, 64, bn);
  if (r != BW_OK) return r;
  CUtensorMap tc;
  if ((r = make_c_map(&tc, C, M, N, BW_OUT_F32)) != BW_OK) return r;
  GemmParams p = base_params(*d, C, M, N, K);
  gather_apply(g, p, 4);
  if (g) {
    PeerMaps pm{};
    CUtensorMap tcl;
    // With a multicast C the epilogue writes through multimem.st and no TMA store runs: the
    // C tensor map is a placeholder over A (local memory, never copied to or from).
    if (g->mc) r = make_c_map_ld(&tcl, const_cast<void*>(A), 8, 8, 8, BW_OUT_F32);
    else r = make_c_map_ld(&tcl, p.C, M, N, g->ldc, BW_OUT_F32);
    if (r != BW_OK) return r;
    for (int q = 0; q < p.npeers; ++q)
      if ((r = make_c_map_ld(&pm.m[q], p.peers[q], M, N, g->ldc, BW_OUT_F32)) != BW_OK) return r;
    if (gather_deep_staging(g))
      return launch_pair<Kind::F16, true, 2, Out::F32, false, 2, 256, 6>(ta, tb, tcl, p, s, *d, &pm);
    return launch_pair<Kind::F16, true, 3, Out::F32, false, 2>(ta, tb, tcl, p, s, *d, &pm);
  }
  if (pair) {
    if (direct_epilogue_ok(C, N, 4)) {
      if (env_int("BW_WIDE", 0) != 0) {
        if (b_mn) return launch_pair_wide<Kind::F16, true, Out::F32>(ta, tb, p, s, *d);
        return launch_pair_wide<Kind::F16, false, Out::F32>(ta, tb, p, s, *d);
      }
      if (b_mn) return launch_pair<Kind::F16, true, 3, Out::F32, true, 2>(ta, tb, tc, p, s, *d);
      return launch_pair<Kind::F16, false, 3, Out::F32, true, 2>(ta, tb, tc, p, s, *d);
    }
    if (b_mn) return launch_pair<Kind::F16, true, 3, Out::F32, false, 2>(ta, tb, tc, p, s, *d);
    return launch_pair<Kind::F16, false, 3, Out::F32, false, 2>(ta, tb, tc, p, s, *d);
  }
  if (splits > 1) {
    if ((r = set_splits(p, splits, (K + 63) / 64)) != BW_OK) return r;
    if (b_mn) return launch_split<Kind::F16, true>(ta, tb, tc, p, C, BW_OUT_F32, s, *d);
    return launch_split<Kind::F16, false>(ta, tb, tc, p, C, BW_OUT_F32, s, *d);
  }
  if (b_mn) {
    if (narrow) return launch<Kind::F16, true, 128, 6, 2, Out::F32>(ta, tb, tc, p, s, *d);
    return launch<Kind::F16, true, 256, 4, 2, Out::F32>(ta, tb, tc, p, s, *d);
  }
  if (narrow) return launch<Kind::F16, false, 128, 6, 2, Out::F32>(ta, tb, tc, p, s, *d);
  return launch<Kind::F16, false, 256, 4, 2, Out::F32>(ta, tb, tc, p, s, *d);
}

int gemm_fp8_impl(const uint8_t* A, const uint8_t* Bt, const float* sa, const float* sb, void* C, int out_dtype,
                  int M, int N, int K, cudaStream_t s, const GatherCtx* g = nullptr) {
  int r = check_common(A, Bt, C, M, N, K);
  if (r != BW_OK || M == 0 || N == 0) return r;
  if (out_dtype != BW_OUT_F32 && out_dtype != BW_OUT_BF16) return set_error(BW_ERR_INVALID, "bad out_dtype %d", out_dtype);
  if (K % 16 != 0) return set_error(BW_ERR_INVALID, "fp8 GEMM needs K %% 16 == 0 (got %d)", K);
  if (N % 8 != 0) return set_error(BW_ERR_INVALID, "fp8 GEMM needs N %% 8 == 0 (got %d)", N);
  if ((r = gather_check(g, C, N, K, static_cast<int>(out_elem_bytes(out_dtype)))) != BW_OK) return r;
  DeviceState* d;
  if ((r = ensure_device(&d)) != BW_OK) return r;
  if (K == 0) { BW_CUDA(cudaMemsetAsync(C, 0, out_elem_bytes(out_dtype) * size_t(M) * N, s)); return BW_OK; }
  int pmt = 1;
  if (const int pw = g ? 0 : panel_width(M, N, K, false, C, static_cast<int>(out_elem_bytes(out_dtype)), *d, &pmt)) {
    const int box = pw <= 256 ? pw : pw / 2;
    CUtensorMap ta, tb;
    if ((r = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, A, K, M, uint64_t(K), 128, 128)) != BW_OK) return r;
    if ((r = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, Bt, K, N, uint64_t(K), 128, box)) != BW_OK) return r;
    GemmParams p = base_params(*d, C, M, N, K);
    p.hints = env_int("BW_L2_HINTS", 0);
    p.scale_a = sa;
    p.scale_b = sb;
    if (out_dtype == BW_OUT_F32) return launch_panel<Kind::F8, false, Out::F32>(ta, tb, p, pw, box, pmt, s);
    return launch_panel<Kind::F8, false, Out::BF16>(ta, tb, p, pw, box, pmt, s);
  }
  const int splits = g ? 1 : choose_splits(M, N, (K + 127) / 128, static_cast<int>(out_elem_bytes(out_dtype)), *d);
  const bool pair = g || (splits == 1 && use_pair(M, N, *d));
  const bool narrow = !pair && splits == 1 && use_narrow(M, N, *d);
  const int bn = pair ? 128 : narrow ? 128 : 256;
  CUtensorMap ta, tb;
  if ((r = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, A, K, M, uint64_t(K), 128, 128)) != BW_OK) return r;
  if ((r = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, Bt, K, N, uint64_t(K), 128, bn)) != BW_OK) return r;
  CUtensorMap tc;
  if ((r = make_c_map(&tc, C, M, N, out_dtype)) != BW_OK) return r;
  GemmParams p = base_params(*d, C, M, N, K);
  gather_apply(g, p, static_cast<int>(out_elem_bytes(out_dtype)));
  p.scale_a = sa;
  p.scale_b = sb;
  if (g) {
    PeerMaps pm{};
    CUtensorMap tcl;
    if (g->mc) r = make_c_map_ld(&tcl, const_cast<uint8_t*>(A), 8, 8, 8, out_dtype);  // placeholder (see f16)
    else r = make_c_map_ld(&tcl, p.C, M, N, g->ldc, out_dtype);
    if (r != BW_OK) return r;
    for (int q = 0; q < p.npeers; ++q)
      if ((r = make_c_map_ld(&pm.m[q], p.peers[q], M, N, g->ldc, out_dtype)) != BW_OK) return r;
    if (gather_deep_staging(g)) {
      if (out_dtype == BW_OUT_F32)
        return launch_pair<Kind::F8, false, 2, Out::F32, false, 2, 256, 6>(ta, tb, tcl, p, s, *d, &pm);
      return launch_pair<Kind::F8, false, 2, Out::BF16, false, 2, 256, 6>(ta, tb, tcl, p, s, *d, &pm);
    }
    if (out_dtype == BW_OUT_F32) return launch_pair<Kind::F8, false, 3, Out::F32, false, 2>(ta, tb, tcl, p, s, *d, &pm);
    return launch_pair<Kind::F8, false, 3, Out::BF16, false, 2>(ta, tb, tcl, p, s, *d, &pm);
  }
  if (pair) {
    const bool direct = direct_epilogue_ok(C, N, static_cast<int>(out_elem_bytes(out_dtype)));
    if (direct && env_int("BW_WIDE", 0) != 0) {
      if (out_dtype == BW_OUT_F32) return launch_pair_wide<Kind::F8, false, Out::F32>(ta, tb, p, s, *d);
      return launch_pair_wide<Kind::F8, false, Out::BF16>(ta, tb, p, s, *d);
    }
    if (out_dtype == BW_OUT_F32) {
      if (direct) return launch_pair<Kind::F8, false, 3, Out::F32, true, 2>(ta, tb, tc, p, s, *d);
      return launch_pair<Kind::F8, false, 3, Out::F32, false, 2>(ta, tb, tc, p, s, *d);
    }
    if (direct) return launch_pair<Kind::F8, false, 3, Out::BF16, true, 2>(ta, tb, tc, p, s, *d);
    return launch_pair<Kind::F8, false, 3, Out::BF16, false, 2>(ta, tb, tc, p, s, *d);
  }
  if (splits > 1) {
    if ((r = set_splits(p, splits, (K + 127) / 128)) != BW_OK) return r;
    r = launch_split<Kind::F8, false>(ta, tb, tc, p, C, out_dtype, s, *d);
    if (r != BW_ERR_UNSUPPORTED) return r;
    p.splits = 1;  // BF16 C and no workspace slot for this stream: run unsplit
    p.kb_per_split = 0;
  }
  if (out_dtype == BW_OUT_F32) {
    if (narrow) return launch<Kind::F8, false, 128, 6, 2, Out::F32>(ta, tb, tc, p, s, *d);
    return launch<Kind::F8, false, 256, 4, 2, Out::F32>(ta, tb, tc, p, s, *d);
  }
  if (narrow) return launch<Kind::F8, false, 128, 6, 2, Out::BF16>(ta, tb, tc, p, s, *d);
  return launch<Kind::F8, false, 256, 4, 2, Out::BF16>(ta, tb, tc, p, s, *d);
}

int gemm_mxf4_impl(const uint8_t* A, const uint8_t* Bt, const uint8_t* sfa, const uint8_t* sfb, const float* sa,
                   const float* sb, void* C, int out_dtype, int M, int N, int K, cudaStream_t s, bool unit_sf) {
  int r = check_common(A, Bt, C, M, N, K);
  if (r != BW_OK || M == 0 || N == 0) return r;
  if (out_dtype != BW_OUT_F32 && out_dtype != BW_OUT_BF16) return set_error(BW_ERR_INVALID, "bad out_dtype %d", out_dtype);
  if (K % 32 != 0) return set_error(BW_ERR_INVALID, "fp4 GEMM needs K %% 32 == 0 (got %d)", K);
  if (N % 8 != 0) return set_error(BW_ERR_INVALID, "fp4 GEMM needs N %% 8 == 0 (got %d)", N);
  if (unit_sf) { sfa = nullptr; sfb = nullptr; }
  else if (K > 0 && (!sfa || !sfb)) return set_error(BW_ERR_INVALID, "scale-factor pointers are null");
  if (!unit_sf && K > 0 && (!aligned16(sfa) || !aligned16(sfb))) return set_error(BW_ERR_INVALID, "scale factors must be 16-byte aligned");
  DeviceState* d;
  if ((r = ensure_device(&d)) != BW_OK) return r;
  if (K == 0) { BW_CUDA(cudaMemsetAsync(C, 0, out_elem_bytes(out_dtype) * size_t(M) * N, s)); return BW_OK; }
  CUtensorMap ta, tb;
  if ((r = make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, A, K / 2, M, uint64_t(K / 2), 128, 128)) != BW_OK) return r;
  if ((r = make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, Bt, K / 2, N, uint64_t(K / 2), 128, 128)) != BW_OK) return r;
  CUtensorMap tc;
  if ((r = make_c_map(&tc, C, M, N, out_dtype)) != BW_OK) return r;
  GemmParams p = base_params(*d, C, M, N, K);
  p.scale_a = sa;
  p.scale_b = sb;
  p.sfa = sfa;
  p.sfb = sfb;
  p.sf_kgroups = ((K + 31) / 32 + 3) / 4;
  const bool pair_ok = env_int("BW_MX_PAIR", 1) != 0 && use_pair(M, N, *d) &&
                       (out_dtype == BW_OUT_BF16 || (reinterpret_cast<uintptr_t>(C) & 31u) == 0);
  if (pair_ok && unit_sf && direct_epilogue_ok(C, N, static_cast<int>(out_elem_bytes(out_dtype))) && env_int("BW_FP4_TN224", 1) != 0) {
    // plain FP4: constant 2^0 block scales need only 12 TMEM columns, which leaves room for two
    // 224-column accumulators - the double-buffered pair kernel with 256 x 224 tiles
    CUtensorMap ta2, tb2;
    if ((r = make_tmap_2d(&ta2, CU_TENSOR_MAP_DATA_TYPE_UINT8, A, K / 2, M, uint64_t(K / 2), 128, 128)) != BW_OK) return r;
    if ((r = make_tmap_2d(&tb2, CU_TENSOR_MAP_DATA_TYPE_UINT8, Bt, K / 2, N, uint64_t(K / 2), 128, 112)) != BW_OK) return r;
    if (out_dtype == BW_OUT_F32) return launch_pair<Kind::MXF4, false, 3, Out::F32, true, 2, 224>(ta2, tb2, tc, p, s, *d);
    return launch_pair<Kind::MXF4, false, 3, Out::BF16, true, 2, 224>(ta2, tb2, tc, p, s, *d);
  }
  if (pair_ok) {
    // 256 x 192 tiles (two accumulators, direct 32-byte stores) when C allows them, else
    // 256 x 256 with one accumulator drained to registers
    const bool narrow_mx = direct_epilogue_ok(C, N, static_cast<int>(out_elem_bytes(out_dtype))) &&
                           env_int("BW_MX_TN", 256) == 192;
    CUtensorMap ta2, tb2, tsa, tsb;
    if ((r = make_tmap_2d(&ta2, CU_TENSOR_MAP_DATA_TYPE_UINT8, A, K / 2, M, uint64_t(K / 2), 128, 128)) != BW_OK) return r;
    if ((r = make_tmap_2d(&tb2, CU_TENSOR_MAP_DATA_TYPE_UINT8, Bt, K / 2, N, uint64_t(K / 2), 128,
                          narrow_mx ? 96 : 128)) != BW_OK) return r;
    if (sfa) {
      // scale factors seen as rows of 256 bytes; one box = 8 rows = 4 atoms of 512 B
      const uint64_t ra = bw_sf_bytes(M, K) / 256, rb = bw_sf_bytes(N, K) / 256;
      if ((r = make_tmap_2d(&tsa, CU_TENSOR_MAP_DATA_TYPE_UINT8, sfa, 256, ra, 256, 256, 8,
                            CU_TENSOR_MAP_SWIZZLE_NONE)) != BW_OK) return r;
      if ((r = make_tmap_2d(&tsb, CU_TENSOR_MAP_DATA_TYPE_UINT8, sfb, 256, rb, 256, 256, 8,
                            CU_TENSOR_MAP_SWIZZLE_NONE)) != BW_OK) return r;
    } else {
      tsa = ta2;  // unused: plain FP4 keeps every block scale at 2^0
      tsb = tb2;
    }
    if (narrow_mx) {
      if (out_dtype == BW_OUT_F32) return launch_pair_mx<Out::F32, 192>(ta2, tb2, tsa, tsb, p, s, *d);
      return launch_pair_mx<Out::BF16, 192>(ta2, tb2, tsa, tsb, p, s, *d);
    }
    if (out_dtype == BW_OUT_F32) return launch_pair_mx<Out::F32, 256>(ta2, tb2, tsa, tsb, p, s, *d);
    return launch_pair_mx<Out::BF16, 256>(ta2, tb2, tsa, tsb, p, s, *d);
  }
  if (out_dtype == BW_OUT_F32) return launch<Kind::MXF4, false, 128, 5, 2, Out::F32>(ta, tb, tc, p, s, *d);
  return launch<Kind::MXF4, false, 128, 5, 2, Out::BF16>(ta, tb, tc, p, s, *d);
}

}  // namespace
}  // namespace bw

using namespace bw;

extern "C" {

int bw_gemm_f16(const void* A, const void* B, float* C, int M, int N, int K, void* stream) {
  return gemm_f16_impl(A, B, C, M, N, K, static_cast<cudaStream_t>(stream), true);
}

int bw_gemm_f16_bt(const void* A, const void* Bt, float* C, int M, int N, int K, void* stream) {
  return gemm_f16_impl(A, Bt, C, M, N, K, static_cast<cudaStream_t>(stream), false);
}

static int make_gather(GatherCtx* g, void* const* peer_C_full, int world, int rank, int N_total) {
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return set_error(BW_ERR_INVALID, "fused gather: rank %d of world %d (1..8 ranks)", rank, world);
  if (N_total % world != 0) return set_error(BW_ERR_INVALID, "N_total=%d not divisible by world=%d", N_total, world);
  if (world > 1 && !peer_C_full) return set_error(BW_ERR_INVALID, "fused gather: peer_C_full is null");
  g->ldc = N_total;
  g->col0 = rank * (N_total / world);
  g->npeers = 0;
  // Each staged chunk goes to the peers in this order. Rotated by rank (rank + 1, rank + 2, ...)
  // unless BW_PEER_ORDER=0 (0, 1, ..., every rank starting with the same peer).
  const bool rotate = env_int("BW_PEER_ORDER", 1) != 0;
  for (int i = 1; i <= world; ++i) {
    const int q = rotate ? (rank + i) % world : i - 1;
    if (q != rank) g->peers[g->npeers++] = peer_C_full[q];
  }
  return BW_OK;
}

int bw_gemm_f16_allgather(const void* A, const void* B_shard, float* C_full, void* const* peer_C_full, int world,
                          int rank, int M, int N_total, int K, void* stream) {
  GatherCtx g;
  int r = make_gather(&g, peer_C_full, world, rank, N_total);
  if (r != BW_OK) return r;
  return gemm_f16_impl(A, B_shard, C_full, M, N_total / world, K, static_cast<cudaStream_t>(stream), true, &g);
}

int bw_gemm_fp8_allgather(const uint8_t* A, const uint8_t* Bt_shard, const float* scale_a, const float* scale_b,
                          void* C_full, int out_dtype, void* const* peer_C_full, int world, int rank, int M,
                          int N_total, int K, void* stream) {
  GatherCtx g;
  int r = make_gather(&g, peer_C_full, world, rank, N_total);
  if (r != BW_OK) return r;
  return gemm_fp8_impl(A, Bt_shard, scale_a, scale_b, C_full, out_dtype, M, N_total / world, K,
                       static_cast<cudaStream_t>(stream), &g);
}

static int make_gather_mc(GatherCtx* g, void* C_multicast, int world, int rank, int N_total) {
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return set_error(BW_ERR_INVALID, "multicast gather: rank %d of world %d (1..8 ranks)", rank, world);
  if (N_total % world != 0) return set_error(BW_ERR_INVALID, "N_total=%d not divisible by world=%d", N_total, world);
  if (!C_multicast) return set_error(BW_ERR_INVALID, "multicast gather: C_multicast is null");
  g->ldc = N_total;
  g->col0 = rank * (N_total / world);
  g->npeers = 0;
  g->mc = C_multicast;
  g->mc_plain = env_int("BW_MC_PLAIN", 0) != 0 ? 1 : 0;
  return BW_OK;
}

int bw_gemm_f16_allgather_multicast(const void* A, const void* B_shard, void* C_multicast, int world, int rank,
                                    int M, int N_total, int K, void* stream) {
  GatherCtx g;
  int r = make_gather_mc(&g, C_multicast, world, rank, N_total);
  if (r != BW_OK) return r;
  return gemm_f16_impl(A, B_shard, static_cast<float*>(C_multicast), M, N_total / world, K,
                       static_cast<cudaStream_t>(stream), true, &g);
}

int bw_gemm_fp8_allgather_multicast(const uint8_t* A, const uint8_t* Bt_shard, const float* scale_a,
                                    const float* scale_b, void* C_multicast, int out_dtype, int world, int rank,
                                    int M, int N_total, int K, void* stream) {
  GatherCtx g;
  int r = make_gather_mc(&g, C_multicast, world, rank, N_total);
  if (r != BW_OK) return r;
  return gemm_fp8_impl(A, Bt_shard, scale_a, scale_b, C_multicast, out_dtype, M, N_total / world, K,
                       static_cast<cudaStream_t>(stream), &g);
}

int bw_gemm_fp8(const uint8_t* A, const uint8_t* Bt, const float* scale_a, const float* scale_b, void* C,
                int out_dtype, int M, int N, int K, void* stream) {
  return gemm_fp8_impl(A, Bt, scale_a, scale_b, C, out_dtype, M, N, K, static_cast<cudaStream_t>(stream));
}

int bw_gemm_mxfp4(const uint8_t* A, const uint8_t* Bt, const uint8_t* sfA, const uint8_t* sfB,
                  const float* scale_a, const float* scale_b, void* C, int out_dtype, int M, int N, int K,
                  void* stream) {
  return gemm_mxf4_impl(A, Bt, sfA, sfB, scale_a, scale_b, C, out_dtype, M, N, K, static_cast<cudaStream_t>(stream),
                        false);
}

int bw_gemm_fp4(const uint8_t* A, const uint8_t* Bt, const float* scale_a, const float* scale_b, void* C,
                int out_dtype, int M, int N, int K, void* stream) {
  return gemm_mxf4_impl(A, Bt, nullptr, nullptr, scale_a, scale_b, C, out_dtype, M, N, K,
                        static_cast<cudaStream_t>(stream), true);
}

size_t bw_sf_bytes(int outer, int K) {
  if (outer <= 0 || K <= 0) return 0;
  const size_t rb = (static_cast<size_t>(outer) + 127) / 128;
  const size_t kg = ((static_cast<size_t>(K) + 31) / 32 + 3) / 4;
  return rb * kg * 512;
}

size_t bw_sf_offset(int row, int kblock, int K) {
  const size_t kg = ((static_cast<size_t>(K) + 31) / 32 + 3) / 4;
  const size_t atom = (static_cast<size_t>(row) / 128) * kg + static_cast<size_t>(kblock) / 4;
  const int r = row % 128;
  return atom * 512 + (r % 32) * 16 + (r / 32) * 4 + (kblock % 4);
}

}  // extern "C"
