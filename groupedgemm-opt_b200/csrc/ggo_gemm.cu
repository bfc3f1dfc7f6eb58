// Host side of the grouped GEMM: tensor-map encoding, per-device caches, tile choice and the
// C-ABI entry points declared in include/ggo.h.
//
// Reference counterpart: csrc/grouped_gemm_kernel.cu:348-450 (grouped_gemm_forward) and :195-279
// (launch_grouped_gemm). Differences by design: the token counts stay on the device (no
// cudaStreamSynchronize), zero-token experts are skipped inside the kernel, and there is no
// per-group argument buffer to build or copy.
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>

#include "ggo.h"
#include "ggo_gemm.cuh"
#include "ggo_gemm_pair.cuh"
#include "ggo_gemm_wgrad.cuh"
#include "ggo_gemm_wgrad_pair.cuh"
#include "ggo_internal.h"

namespace ggo {

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::mutex g_mu;
EncodeTiledFn g_encode = nullptr;
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};

int get_encode(EncodeTiledFn* fn) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_encode) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !ptr)
      return GGO_ERR_CUDA;
    g_encode = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  *fn = g_encode;
  return GGO_OK;
}

// 2D K-major operand map: dims {K, rows}, box {64, box_rows}, 128-B swizzle, zero fill out of
// bounds.
int make_map_dt(CUtensorMap* m, const void* base, int64_t rows, int64_t k,
                CUtensorMapDataType dt, int elem_bytes, int box_rows, int box_cols) {
  EncodeTiledFn enc;
  if (int st = get_encode(&enc)) return st;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * elem_bytes};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? GGO_OK : cuda_fail(100000 + static_cast<int>(r));
}

int make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t k, bool bf16, int box_rows,
             int box_cols = kBK) {
  return make_map_dt(m, base, rows, k,
                     bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                     box_rows, box_cols);
}

// Operand map for 1-byte e4m3 data: rows of K bytes, boxes of 128 elements (128 B) x box_rows.
int make_map_fp8(CUtensorMap* m, const void* base, int64_t rows, int64_t k, int box_rows) {
  return make_map_dt(m, base, rows, k, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, box_rows, 128);
}

// Block-scale map (MX path): the UE8M0 scales as [atoms * 2, 256] bytes, no swizzle, boxes of
// one 512-B atom (2 x 256). Atoms past the end read as zeros.
int make_sf_map(CUtensorMap* m, const void* base, int64_t atoms) {
  EncodeTiledFn enc;
  if (int st = get_encode(&enc)) return st;
  const cuuint64_t dims[2] = {256, static_cast<cuuint64_t>(atoms > 0 ? 2 * atoms : 2)};
  const cuuint64_t strides[1] = {256};
  const cuuint32_t box[2] = {256, 2};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? GGO_OK : cuda_fail(100000 + static_cast<int>(r));
}

// Output map for the TMA-store epilogue: [rows, n_out] row-major, boxes of 32 rows x 64 columns
// (128 B, 128-B swizzle, matching the staging layout). Only for a plain (non-scattered) output.
int make_out_map(CUtensorMap* m, GemmParams* p, bool bf16) {
  memset(m, 0, sizeof(*m));
  p->use_tma_store = 0;
  if (p->out == nullptr || p->origin != nullptr) return GGO_OK;
  if (int st = make_map(m, p->out, p->rows, p->n_out, bf16, 32, 64)) return st;
  p->use_tma_store = 1;
  return GGO_OK;
}

// Per (device, kernel) one-time set-up: the dynamic shared-memory opt-in and, for cluster
// kernels, how many clusters can be resident at once.
std::map<std::pair<int, const void*>, int> g_kernel_slots;

template <typename Kern>
int kernel_setup(Kern kern, int smem, int dev, bool pair, int* resident) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto key = std::make_pair(dev, reinterpret_cast<const void*>(kern));
  auto it = g_kernel_slots.find(key);
  if (it == g_kernel_slots.end()) {
    if (cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem))
      return cuda_fail(e);
    int n = g_sm_count[dev];
    if (pair) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (g_sm_count[dev] / 2), 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = smem;
      n = 0;
      if (cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg)) return cuda_fail(e);
      if (n <= 0) return cuda_fail(static_cast<int>(cudaErrorInvalidConfiguration));
    }
    it = g_kernel_slots.emplace(key, n).first;
  }
  *resident = it->second;
  return GGO_OK;
}

// Weight map: K-major rows of K (boxes of 64 x box_rows), or for an MN-major operand
// (the dgrad form) [E * Kred rows, n_out columns] in 64 x 64 boxes.
template <bool BMN>
int make_b_map(CUtensorMap* m, const void* b, int64_t b_rows, const GemmParams& q, bool bf16,
               int box_rows) {
  if (BMN) return make_map(m, b, static_cast<int64_t>(q.num_experts) * q.k, q.n_out, bf16, 64, 64);
  return make_map(m, b, b_rows, q.k, bf16, box_rows);
}

template <int BN, int EPI, bool BF16, bool BMN = false, bool FP8 = false>
int launch(const void* a, const void* b, int64_t b_rows, const GemmParams& p, int dev,
           cudaStream_t stream) {
  CUtensorMap ma, mb, mc, mas;
  memset(&mas, 0, sizeof(mas));
  GemmParams q = p;
  if (FP8) {
    if (int st = make_map_fp8(&ma, a, q.rows, q.k, kBM)) return st;
    if (int st = make_map_fp8(&mb, b, b_rows, q.k, 128)) return st;
    q.skinny_max = 0;
  } else {
    if (int st = make_map(&ma, a, q.rows, q.k, BF16, kBM)) return st;
    if (int st = make_b_map<BMN>(&mb, b, b_rows, q, BF16, 128)) return st;
    if (BMN) {
      q.skinny_max = 0;
    } else if (q.skinny_max > 0) {  // input boxes of kSkinnyRows rows for the skinny tiles
      if (int st = make_map(&mas, a, q.rows, q.k, BF16, kSkinnyRows)) return st;
    }
  }
  if (int st = make_out_map(&mc, &q, BF16)) return st;
  auto kern = grouped_gemm_kernel<BN, EPI, BF16, BMN, FP8>;
  constexpr int smem = SmemLayout<BN>::kTotal;
  int sms = 0;
  if (int st = kernel_setup(kern, smem, dev, false, &sms)) return st;
  constexpr int out_bn = epi_glu(EPI) ? BN / 2 : BN;
  const int64_t n_tiles = (p.n_out + out_bn - 1) / out_bn;
  const int64_t ub = ((p.rows + kBM - 1) / kBM + p.num_segments) * n_tiles;  // tile upper bound
  const int grid = static_cast<int>(ub < sms ? ub : sms);
  if (grid <= 0) return GGO_OK;
  kern<<<grid, kThreads, smem, stream>>>(ma, mb, mc, mas, q);
  return check_launch();
}

// Block scales of an MX launch: base pointers and their sizes in 512-B atoms.
struct MxScales {
  const void* a = nullptr;
  int64_t a_atoms = 0;
  const void* b = nullptr;
  int64_t b_atoms = 0;
};

template <int BN, int EPI, bool BF16, bool BMN = false, bool FP8 = false, bool MX = false>
int launch_pair(const void* a, const void* b, int64_t b_rows, const GemmParams& p, int dev,
                cudaStream_t stream, const MxScales* mx = nullptr) {
  CUtensorMap ma, mb, mc, msa, msb;
  memset(&msa, 0, sizeof(msa));
  memset(&msb, 0, sizeof(msb));
  if (MX) {
    if (!mx) return GGO_ERR_INVALID_ARG;
    if (int st = make_sf_map(&msa, mx->a, mx->a_atoms)) return st;
    if (int st = make_sf_map(&msb, mx->b, mx->b_atoms)) return st;
  }
  GemmParams q = p;
  if (FP8) {
    if (int st = make_map_fp8(&ma, a, q.rows, q.k, 128)) return st;
    if (int st = make_map_fp8(&mb, b, b_rows, q.k, BN / 2)) return st;
  } else {
    if (int st = make_map(&ma, a, q.rows, q.k, BF16, 128)) return st;
    if (int st = make_b_map<BMN>(&mb, b, b_rows, q, BF16, BN / 2)) return st;
  }
  if (int st = make_out_map(&mc, &q, BF16)) return st;
  auto kern = grouped_gemm_pair_kernel<BN, EPI, BF16, BMN, FP8, MX>;
  constexpr int smem = PairLayout<BN, MX>::kTotal;
  int clusters = 0;
  if (int st = kernel_setup(kern, smem, dev, true, &clusters)) return st;
  constexpr int out_bn = epi_glu(EPI) ? BN / 2 : BN;
  const int64_t n_tiles = (p.n_out + out_bn - 1) / out_bn;
  const int64_t ub = ((p.rows + 255) / 256 + p.num_segments) * n_tiles;  // pair-tile upper bound
  const int64_t pairs = ub < clusters ? ub : clusters;
  if (pairs <= 0) return GGO_OK;
  kern<<<static_cast<int>(2 * pairs), kThreads, smem, stream>>>(ma, mb, mc, msa, msb, q);
  return check_launch();
}

// Pair-tile width. 256 is the default: measured on cfg2 under the 1 kW power cap, 256-wide tiles
// beat 224-wide ones per SM clock (0.87 vs 0.81 TFLOP/s per MHz) although the 224-wide grid has a
// fuller last wave; wider tiles move fewer operand bytes per FLOP, and energy per FLOP sets the
// clock the GPU can hold. GGO_PAIR_BN selects another width for experiments.
constexpr int kDefaultPairBN = 256;

template <int EPI, bool BF16>
int launch_pair_bn(int bn, const void* a, const void* b, int64_t b_rows, const GemmParams& p,
                   int dev, cudaStream_t stream) {
  switch (bn) {
    case 224: if constexpr (EPI == kEpiStore) return launch_pair<224, EPI, BF16>(a, b, b_rows, p, dev, stream); break;
    case 192: return launch_pair<192, EPI, BF16>(a, b, b_rows, p, dev, stream);
    case 160: if constexpr (EPI == kEpiStore) return launch_pair<160, EPI, BF16>(a, b, b_rows, p, dev, stream); break;
    case 128: return launch_pair<128, EPI, BF16>(a, b, b_rows, p, dev, stream);
    default: break;
  }
  return launch_pair<256, EPI, BF16>(a, b, b_rows, p, dev, stream);
}

// Tuning knobs, read on every call (cheap next to a launch): GGO_RASTER_GROUP_M (m-tiles per
// raster group, default 8) and GGO_PAIR_BN (force the CTA-pair tile width: 256/224/192/160/128).
int env_int(const char* name, int dflt) {
  const char* e = getenv(name);
  const int v = e ? atoi(e) : 0;
  return v > 0 ? v : dflt;
}
// m-tiles per raster group: as many as keep the group's A panels (tile_m x K bf16 each) within
// ~48 MB of L2, at most 16. Inside a group every weight column is streamed from HBM once, so
// taller groups re-read the weights less; beyond the L2 budget the A panels themselves thrash.
int raster_group_m(int64_t k, int tile_m) {
  const int64_t panel = static_cast<int64_t>(tile_m) * k * 2;
  int64_t g = (48ll << 20) / (panel > 0 ? panel : 1);
  g = g < 1 ? 1 : (g > 16 ? 16 : g);
  return env_int("GGO_RASTER_GROUP_M", static_cast<int>(g));
}

int device_setup(int* dev_out) {
  int dev;
  if (cudaError_t e = cudaGetDevice(&dev)) return cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return GGO_ERR_NO_DEVICE;
  // Bind the device's primary context to this thread: the tensor-map encoder is a driver call and
  // needs a current context, which a fresh thread (e.g. autograd's backward worker) lacks.
  if (cudaError_t e = cudaSetDevice(dev)) return cuda_fail(e);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sm_count[dev] == 0) {
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return GGO_ERR_CUDA;
    if (major != 10) return GGO_ERR_NO_DEVICE;
    g_sm_count[dev] = sms;
  }
  *dev_out = dev;
  return GGO_OK;
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// Kernel choice: 128 = single-CTA 128x128 tile, 256 = single-CTA 128x256 tile,
// 512 = CTA-pair 256x256 tile.
int choose_bn(int tile_config, int64_t rows, int64_t n, int num_segments, int sms) {
  switch (tile_config) {
    case GGO_TILE_PP_128x256x64:
      return 512;
    case GGO_TILE_CO_128x128x64:
    case GGO_TILE_PP_128x128x128:
      return 128;
    case GGO_TILE_CO_128x256x64:
      return 256;
    default: {  // AUTO / CuBLAS_Seq
      if (n <= 128) return 128;
      const int64_t m_tiles = (rows + kBM - 1) / kBM;
      const int64_t wide = m_tiles * ((n + 255) / 256);
      if (wide < sms) return 128;            // narrow tiles keep every SM busy
      // CTA pairs when segments average at least 192 rows (a 256-row tile is mostly full)
      if (rows >= 192 * static_cast<int64_t>(num_segments) && wide / 2 >= sms) return 512;
      return 256;
    }
  }
}

// Expert-parallel extensions of one call (see ggo_ep_grouped_gemm).
struct GemmExtras {
  int rows_is_bound = 0;
  const int32_t* origin = nullptr;
  void* const* peer_out = nullptr;
  int world = 1;
  // FP8 path: e4m3 operands, out = acc * row_scale[row] * col_scale[expert * n + col] in bf16
  int fp8 = 0;
  const float* row_scale = nullptr;
  const float* col_scale = nullptr;
  // MX path (with fp8): e4m3 operands with UE8M0 block scales (one per 32 K elements) in the
  // 128x4 blocked layout, applied by the tensor cores; out = the block-scaled product in bf16
  int mx = 0;
  const void* a_sf = nullptr;
  const void* b_sf = nullptr;
};

// MX tiles: CTA pairs of 256 x 256 with overlapping accumulators (TMEM columns 0-255 and
// 192-447; the scales in 448-511). SwiGLU weights for the MX path are blocked by kMxGluBlock
// output columns: [E, 2 * F_pad, K], F_pad = F rounded up to kMxGluBlock, block j = gate rows
// j*128.. then the matching up rows.
constexpr int kMxPairBN = 256;
constexpr int kMxGluBlock = kMxPairBN / 2;
int64_t mx_glu_rows(int64_t f) { return 2 * ((f + kMxGluBlock - 1) / kMxGluBlock) * kMxGluBlock; }
// 512-B scale atoms of `rows` rows in `segments` segments (each padded to 128 rows), K columns
int64_t mx_scale_atoms(int64_t rows, int64_t segments, int64_t k) {
  return ((rows + 127) / 128 + segments) * (k / 128);
}

int gemm_common(const void* input, const void* weights, void* output, const int64_t* counts,
                int num_segments, int num_experts, int64_t rows, int64_t n, int64_t k, int dtype,
                int tile_config, int sort_by_m, void* workspace, cudaStream_t stream, bool swiglu,
                const GemmExtras* ex = nullptr, bool bmn = false) {
  const bool scatter = ex && ex->origin;
  if (!input || !weights || (!output && !scatter) || !counts || !workspace)
    return GGO_ERR_INVALID_ARG;
  if (scatter) {
    if (ex->world < 1 || ex->world > 8) return GGO_ERR_INVALID_ARG;
    if (rows > 0x0fffffff) return GGO_ERR_SHAPE;  // origin words hold 28-bit row numbers
    for (int r = 0; r < ex->world; ++r)
      if (!ex->peer_out[r] || !aligned16(ex->peer_out[r])) return GGO_ERR_ALIGNMENT;
  }
  if (num_segments <= 0 || num_experts <= 0 || rows < 0 || n <= 0 || k <= 0)
    return GGO_ERR_INVALID_ARG;
  if (tile_config < 0 || tile_config > GGO_TILE_CUBLAS_SEQ) return GGO_ERR_INVALID_ARG;
  if (num_segments > kMaxSegments) return GGO_ERR_TOO_MANY_SEGMENTS;
  const bool fp8 = ex && ex->fp8;
  const bool mx = fp8 && ex->mx;
  if (fp8) {
    if (bmn || scatter) return GGO_ERR_INVALID_ARG;
    if (mx ? (!ex->a_sf || !ex->b_sf) : (!ex->row_scale || !ex->col_scale))
      return GGO_ERR_INVALID_ARG;
    dtype = GGO_DTYPE_BF16;  // e4m3 in, bf16 out
    if (k % (mx ? 128 : 16)) return GGO_ERR_ALIGNMENT;  // rows of K bytes; MX: whole scale atoms
    if (mx && (!aligned16(ex->a_sf) || !aligned16(ex->b_sf))) return GGO_ERR_ALIGNMENT;
  }
  if (dtype != GGO_DTYPE_BF16 && dtype != GGO_DTYPE_FP16) return GGO_ERR_DTYPE;
  if ((k % 8) || (n % 8)) return GGO_ERR_ALIGNMENT;
  if (!aligned16(input) || !aligned16(weights) || (output && !aligned16(output)) ||
      (reinterpret_cast<uintptr_t>(workspace) & 3u))
    return GGO_ERR_ALIGNMENT;
  const int64_t n_b = swiglu ? (mx ? mx_glu_rows(n) : 2 * n) : n;
  const int64_t b_rows = static_cast<int64_t>(num_experts) * n_b;
  if (rows > INT32_MAX || b_rows > INT32_MAX || k > INT32_MAX) return GGO_ERR_SHAPE;
  if (bmn && static_cast<int64_t>(num_experts) * k > INT32_MAX) return GGO_ERR_SHAPE;
  if (rows == 0) return GGO_OK;
  int dev;
  if (int st = device_setup(&dev)) return st;

  GemmParams p;
  p.counts = counts;
  p.num_segments = num_segments;
  p.num_experts = num_experts;
  p.rows = static_cast<int>(rows);
  p.n_out = static_cast<int>(n);
  p.n_b = static_cast<int>(n_b);
  p.k = static_cast<int>(k);
  p.sort_by_m = sort_by_m ? env_int("GGO_SEG_ORDER", 2) : 0;
  p.group_m = raster_group_m(k, 128);  // re-derived below for 256-row pair tiles
  // Test hook for the bounded waits: GGO_TEST_INJECT_STALL=1 makes the CTA that claims tile 0 leave
  // its first pipeline stage unarmed and lowers the wait limit to 2^24 cycles (~10 ms). The kernel then
  // records a timeout in the workspace and returns; nothing faults or hangs.
  p.inject_stall = env_int("GGO_TEST_INJECT_STALL", 0) > 0 ? 1 : 0;
  p.wait_limit = p.inject_stall ? (1ll << 24) : GGO_WAIT_LIMIT_CYCLES;
  p.split_mode = 0;
  p.split_tail_ntiles = 1;
  p.split_min_tiles = 0;
  p.glu_blocked = 0;
  // GGO_SKINNY_ROWS: row limit of the swapped-operand tiles (default 64, 0 disables)
  {
    const char* e = getenv("GGO_SKINNY_ROWS");
    const int v = e ? atoi(e) : kSkinnyRows;
    p.skinny_max = v < 0 ? 0 : (v > kSkinnyRows ? kSkinnyRows : v);
  }
  p.rows_is_bound = ex ? ex->rows_is_bound : 0;
  p.row_scale = fp8 ? ex->row_scale : nullptr;
  p.col_scale = fp8 ? ex->col_scale : nullptr;
  p.origin = scatter ? ex->origin : nullptr;
  for (int r = 0; r < 8; ++r) p.peer_out[r] = (scatter && r < ex->world) ? ex->peer_out[r] : nullptr;
  p.out = output;
  p.ws = static_cast<GgoWorkspace*>(workspace);
  const bool bf16 = dtype == GGO_DTYPE_BF16;
  int bn = choose_bn(tile_config, rows, swiglu ? 2 * n : n, num_segments, g_sm_count[dev]);
  if (mx) {  // CTA pairs only (no short-tail pass: its scales would need a second layout)
    MxScales sc;
    sc.a = ex->a_sf;
    sc.a_atoms = mx_scale_atoms(rows, num_segments, k);
    sc.b = ex->b_sf;
    sc.b_atoms = static_cast<int64_t>(num_experts) * ((n_b + 127) / 128) * (k / 128);
    // The kernel addresses scale atoms by 32-bit TMA row coordinates, two rows per atom. The
    // largest coordinate it forms is 2 * (block * (k / 128) + kb) with block at most one past the
    // last block (rank 1's half of a pair tile, the B tile's second block): bound that.
    const int64_t kgroups = k / 128;
    if (2 * (sc.a_atoms + kgroups) > INT32_MAX || 2 * (sc.b_atoms + kgroups) > INT32_MAX)
      return GGO_ERR_SHAPE;
    p.group_m = raster_group_m(k / 2, 256);
    p.glu_blocked = swiglu ? 1 : 0;
    return swiglu ? launch_pair<kMxPairBN, kEpiSwiGLU, true, false, true, true>(
                        input, weights, b_rows, p, dev, stream, &sc)
                  : launch_pair<kMxPairBN, kEpiStore, true, false, true, true>(
                        input, weights, b_rows, p, dev, stream, &sc);
  }
  if (fp8) {  // CTA-pair pass (+ short-tail pass) or single-CTA 128x256, scaled epilogue
    if (bn == 512) {
      const bool split = env_int("GGO_SPLIT_TAILS", 1) > 0;
      p.split_tail_ntiles = static_cast<int>((n + (swiglu ? 127 : 255)) / (swiglu ? 128 : 256));
      p.split_min_tiles = env_int("GGO_SPLIT_MIN_TILES", 2 * g_sm_count[dev]);
      GemmParams pp = p;
      pp.group_m = raster_group_m(k / 2, 256);  // k bytes: half the bf16 panel size
      pp.split_mode = split ? 1 : 0;
      const int st =
          swiglu ? launch_pair<256, kEpiScaledSwiGLU, true, false, true>(input, weights, b_rows,
                                                                         pp, dev, stream)
                 : launch_pair<256, kEpiScaled, true, false, true>(input, weights, b_rows, pp, dev,
                                                                   stream);
      if (st) return st;
      if (!split) return GGO_OK;
      p.split_mode = 2;
    }
    return swiglu
               ? launch<256, kEpiScaledSwiGLU, true, false, true>(input, weights, b_rows, p, dev,
                                                                  stream)
               : launch<256, kEpiScaled, true, false, true>(input, weights, b_rows, p, dev, stream);
  }
  if (bn == 512) {
    // CTA-pair pass over 256-row tiles, then (GGO_SPLIT_TAILS, default on) a single-CTA pass over
    // the segments' short tails (count mod 256 in 1..128), which would waste most of a pair tile.
    const bool split = env_int("GGO_SPLIT_TAILS", 1) > 0;
    p.split_tail_ntiles = static_cast<int>((n + (swiglu ? 127 : 255)) / (swiglu ? 128 : 256));
    p.split_min_tiles = env_int("GGO_SPLIT_MIN_TILES", 2 * g_sm_count[dev]);
    GemmParams pp = p;
    pp.group_m = raster_group_m(k, 256);
    pp.split_mode = split ? 1 : 0;
    int st;
    if (bmn)
      st = bf16 ? launch_pair<256, kEpiStore, true, true>(input, weights, b_rows, pp, dev, stream)
                : launch_pair<256, kEpiStore, false, true>(input, weights, b_rows, pp, dev, stream);
    else if (swiglu)
      st = bf16 ? launch_pair_bn<kEpiSwiGLU, true>(env_int("GGO_PAIR_BN", kDefaultPairBN), input,
                                                  weights, b_rows, pp, dev, stream)
                : launch_pair_bn<kEpiSwiGLU, false>(env_int("GGO_PAIR_BN", kDefaultPairBN), input,
                                                   weights, b_rows, pp, dev, stream);
    else
      st = bf16 ? launch_pair_bn<kEpiStore, true>(env_int("GGO_PAIR_BN", kDefaultPairBN), input,
                                                 weights, b_rows, pp, dev, stream)
                : launch_pair_bn<kEpiStore, false>(env_int("GGO_PAIR_BN", kDefaultPairBN), input,
                                                  weights, b_rows, pp, dev, stream);
    if (st || !split) return st;
    p.split_mode = 2;
    bn = 256;
  }
  if (bmn) {  // dgrad form: MN-major weights, plain epilogue
    if (bn == 256)
      return bf16 ? launch<256, kEpiStore, true, true>(input, weights, b_rows, p, dev, stream)
                  : launch<256, kEpiStore, false, true>(input, weights, b_rows, p, dev, stream);
    return bf16 ? launch<128, kEpiStore, true, true>(input, weights, b_rows, p, dev, stream)
                : launch<128, kEpiStore, false, true>(input, weights, b_rows, p, dev, stream);
  }
  if (swiglu)
    return bf16 ? launch<256, kEpiSwiGLU, true>(input, weights, b_rows, p, dev, stream)
                : launch<256, kEpiSwiGLU, false>(input, weights, b_rows, p, dev, stream);
  if (bn == 256)
    return bf16 ? launch<256, kEpiStore, true>(input, weights, b_rows, p, dev, stream)
                : launch<256, kEpiStore, false>(input, weights, b_rows, p, dev, stream);
  return bf16 ? launch<128, kEpiStore, true>(input, weights, b_rows, p, dev, stream)
              : launch<128, kEpiStore, false>(input, weights, b_rows, p, dev, stream);
}

template <int BN, bool BF16>
int launch_wgrad(const void* x, const void* dy, void* dw, const WgradParams& p, int dev,
                 cudaStream_t stream) {
  CUtensorMap mdy, mx, mw;
  if (int st = make_map(&mdy, dy, p.rows, p.n, BF16, 64, 64)) return st;
  if (int st = make_map(&mx, x, p.rows, p.k, BF16, 64, 64)) return st;
  if (int st = make_map(&mw, dw, static_cast<int64_t>(p.num_experts) * p.n, p.k, BF16, 32, 64))
    return st;
  auto kern = grouped_gemm_wgrad_kernel<BN, BF16>;
  constexpr int smem = WgradLayout<BN>::kTotal;
  int sms = 0;
  if (int st = kernel_setup(kern, smem, dev, false, &sms)) return st;
  const int64_t tiles = static_cast<int64_t>(p.num_experts) * ((p.n + 127) / 128) *
                        ((p.k + BN - 1) / BN);
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  kern<<<grid, kThreads, smem, stream>>>(mdy, mx, mw, p);
  return check_launch();
}

template <bool BF16>
int launch_wgrad_pair(const void* x, const void* dy, void* dw, const WgradParams& p, int dev,
                      cudaStream_t stream) {
  CUtensorMap mdy, mx, mw;
  if (int st = make_map(&mdy, dy, p.rows, p.n, BF16, 64, 64)) return st;
  if (int st = make_map(&mx, x, p.rows, p.k, BF16, 64, 64)) return st;
  if (int st = make_map(&mw, dw, static_cast<int64_t>(p.num_experts) * p.n, p.k, BF16, 32, 64))
    return st;
  auto kern = grouped_gemm_wgrad_pair_kernel<BF16>;
  constexpr int smem = WgradPairLayout::kTotal;
  int clusters = 0;
  if (int st = kernel_setup(kern, smem, dev, true, &clusters)) return st;
  const int64_t tiles = static_cast<int64_t>(p.num_experts) * ((p.n + 255) / 256) *
                        ((p.k + 255) / 256);
  const int64_t pairs = tiles < clusters ? tiles : clusters;
  kern<<<static_cast<int>(2 * pairs), kThreads, smem, stream>>>(mdy, mx, mw, p);
  return check_launch();
}

int wgrad_common(const void* x, const void* dy, void* dw, const int64_t* counts, int num_experts,
                 int64_t rows, int64_t n, int64_t k, int dtype, int sort_by_m, void* workspace,
                 cudaStream_t stream) {
  if (!x || !dy || !dw || !counts || !workspace) return GGO_ERR_INVALID_ARG;
  if (num_experts <= 0 || rows < 0 || n <= 0 || k <= 0) return GGO_ERR_INVALID_ARG;
  if (num_experts > kMaxSegments) return GGO_ERR_TOO_MANY_SEGMENTS;
  if (dtype != GGO_DTYPE_BF16 && dtype != GGO_DTYPE_FP16) return GGO_ERR_DTYPE;
  if ((k % 8) || (n % 8)) return GGO_ERR_ALIGNMENT;
  if (!aligned16(x) || !aligned16(dy) || !aligned16(dw)) return GGO_ERR_ALIGNMENT;
  if (rows > INT32_MAX || n > INT32_MAX || k > INT32_MAX ||
      static_cast<int64_t>(num_experts) * n > INT32_MAX)
    return GGO_ERR_SHAPE;
  int dev;
  if (int st = device_setup(&dev)) return st;
  WgradParams p;
  p.counts = counts;
  p.num_experts = num_experts;
  p.rows = static_cast<int>(rows);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.sort_by_m = sort_by_m ? 1 : 0;
  p.out = dw;
  p.ws = static_cast<GgoWorkspace*>(workspace);
  p.wait_limit = GGO_WAIT_LIMIT_CYCLES;
  // 256x256 CTA-pair tiles when they fill every SM pair, else single-CTA 128x256 tiles unless
  // those leave SMs idle. GGO_WGRAD_PAIR: 0 never pairs, 2 always pairs (tests).
  const int64_t wide = static_cast<int64_t>(num_experts) * ((n + 127) / 128) * ((k + 255) / 256);
  const bool bf16 = dtype == GGO_DTYPE_BF16;
  const int64_t pair_tiles =
      static_cast<int64_t>(num_experts) * ((n + 255) / 256) * ((k + 255) / 256);
  const char* pair_env = getenv("GGO_WGRAD_PAIR");
  const int pair_mode = pair_env ? atoi(pair_env) : 1;
  if (pair_mode == 2 || (pair_mode == 1 && pair_tiles >= g_sm_count[dev] / 2))
    return bf16 ? launch_wgrad_pair<true>(x, dy, dw, p, dev, stream)
                : launch_wgrad_pair<false>(x, dy, dw, p, dev, stream);
  if (wide >= g_sm_count[dev])
    return bf16 ? launch_wgrad<256, true>(x, dy, dw, p, dev, stream)
                : launch_wgrad<256, false>(x, dy, dw, p, dev, stream);
  return bf16 ? launch_wgrad<128, true>(x, dy, dw, p, dev, stream)
              : launch_wgrad<128, false>(x, dy, dw, p, dev, stream);
}

}  // namespace

// Scratch for ggo_grouped_gemm_noalloc: one workspace (tile counter, done counter, error word) in
// a file-scope device array, so that entry point never allocates. Every GPU that loads this
// library holds these 256 bytes until the process exits. Host code must not hand the symbol
// itself to a kernel (on the host it only names a stand-in); the device address comes from
// cudaGetSymbolAddress, looked up once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[GGO_WORKSPACE_BYTES];
static void* g_noalloc_ptr[kMaxDevices] = {nullptr};

int noalloc_scratch(void** out) {
  int dev;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GGO_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return GGO_ERR_CUDA;
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return GGO_OK;
}

}  // namespace ggo

extern "C" {

int ggo_version(void) { return 100; }

const char* ggo_status_string(int status) {
  switch (status) {
    case GGO_OK: return "ok";
    case GGO_ERR_INVALID_ARG: return "invalid argument";
    case GGO_ERR_SHAPE: return "unsupported shape";
    case GGO_ERR_DTYPE: return "unsupported dtype (expected bf16 or fp16)";
    case GGO_ERR_ALIGNMENT: return "misaligned pointer or K/N not a multiple of 8";
    case GGO_ERR_TOO_MANY_SEGMENTS: return "too many experts/segments (max 1024)";
    case GGO_ERR_CUDA: return "CUDA call failed";
    case GGO_ERR_NO_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    case GGO_ERR_DEVICE_TIMEOUT: return "a device-side wait timed out";
    case GGO_ERR_COUNT_MISMATCH: return "sum(tokens_per_expert) != total_tokens";
    case GGO_ERR_NEGATIVE_COUNT: return "negative entry in tokens_per_expert";
    default: return "unknown status";
  }
}

size_t ggo_workspace_size(void) { return sizeof(ggo::GgoWorkspace); }

int ggo_grouped_gemm(const void* input_dev, const void* weights_dev, void* output_dev,
                     const int64_t* tokens_per_expert_dev, int num_experts, int64_t total_tokens,
                     int64_t N, int64_t K, int dtype, int tile_config, int sort_by_m,
                     void* workspace_dev, cudaStream_t stream) {
  return ggo::gemm_common(input_dev, weights_dev, output_dev, tokens_per_expert_dev, num_experts,
                          num_experts, total_tokens, N, K, dtype, tile_config, sort_by_m,
                          workspace_dev, stream, false);
}

int ggo_grouped_gemm_segments(const void* input_dev, const void* weights_dev, void* output_dev,
                              const int64_t* tokens_per_segment_dev, int num_segments,
                              int num_experts, int64_t total_tokens, int64_t N, int64_t K,
                              int dtype, int tile_config, int sort_by_m, void* workspace_dev,
                              cudaStream_t stream) {
  return ggo::gemm_common(input_dev, weights_dev, output_dev, tokens_per_segment_dev,
                          num_segments, num_experts, total_tokens, N, K, dtype, tile_config,
                          sort_by_m, workspace_dev, stream, false);
}

int ggo_grouped_gemm_swiglu(const void* x_dev, const void* w_gate_up_dev, void* h_dev,
                            const int64_t* tokens_per_segment_dev, int num_segments,
                            int num_experts, int64_t total_tokens, int64_t F, int64_t K, int dtype,
                            int sort_by_m, void* workspace_dev, cudaStream_t stream) {
  return ggo::gemm_common(x_dev, w_gate_up_dev, h_dev, tokens_per_segment_dev, num_segments,
                          num_experts, total_tokens, F, K, dtype, GGO_TILE_AUTO, sort_by_m,
                          workspace_dev, stream, true);
}

int ggo_grouped_gemm_noalloc(const void* input_dev, const void* weights_dev, void* output_dev,
                             const int64_t* tokens_per_expert_dev, int num_experts,
                             int64_t total_tokens, int64_t N, int64_t K, int dtype,
                             int tile_config, int sort_by_m, cudaStream_t stream) {
  if (num_experts > GGO_NOALLOC_MAX_EXPERTS) return GGO_ERR_TOO_MANY_SEGMENTS;
  if (!input_dev || !weights_dev || !output_dev || !tokens_per_expert_dev)
    return GGO_ERR_INVALID_ARG;
  void* scratch = nullptr;
  if (int st = ggo::noalloc_scratch(&scratch)) return st;
  // The array keeps whatever the previous call left; start every call from zero (stream-ordered,
  // no allocation). This also discards any device-side error word of the previous call.
  if (cudaMemsetAsync(scratch, 0, GGO_WORKSPACE_BYTES, stream) != cudaSuccess) return GGO_ERR_CUDA;
  return ggo::gemm_common(input_dev, weights_dev, output_dev, tokens_per_expert_dev, num_experts,
                          num_experts, total_tokens, N, K, dtype, tile_config, sort_by_m, scratch,
                          stream, false);
}

int ggo_grouped_gemm_dgrad(const void* dy_dev, const void* weights_dev, void* dx_dev,
                           const int64_t* tokens_per_expert_dev, int num_experts,
                           int64_t total_tokens, int64_t N, int64_t K, int dtype, int tile_config,
                           int sort_by_m, void* workspace_dev, cudaStream_t stream) {
  // dx [T, K] = dy [T, N] @ W[e]: reduction over N, output width K, weights read MN-major
  return ggo::gemm_common(dy_dev, weights_dev, dx_dev, tokens_per_expert_dev, num_experts,
                          num_experts, total_tokens, K, N, dtype, tile_config, sort_by_m,
                          workspace_dev, stream, false, nullptr, true);
}

int ggo_grouped_gemm_wgrad(const void* x_dev, const void* dy_dev, void* dw_dev,
                           const int64_t* tokens_per_expert_dev, int num_experts,
                           int64_t total_tokens, int64_t N, int64_t K, int dtype, int sort_by_m,
                           void* workspace_dev, cudaStream_t stream) {
  return ggo::wgrad_common(x_dev, dy_dev, dw_dev, tokens_per_expert_dev, num_experts,
                           total_tokens, N, K, dtype, sort_by_m, workspace_dev, stream);
}

int ggo_grouped_gemm_fp8(const void* input_dev, const float* input_scale_dev,
                         const void* weights_dev, const float* weight_scale_dev, void* output_dev,
                         const int64_t* tokens_per_expert_dev, int num_experts,
                         int64_t total_tokens, int64_t N, int64_t K, int tile_config,
                         int sort_by_m, void* workspace_dev, cudaStream_t stream) {
  ggo::GemmExtras ex;
  ex.fp8 = 1;
  ex.row_scale = input_scale_dev;
  ex.col_scale = weight_scale_dev;
  return ggo::gemm_common(input_dev, weights_dev, output_dev, tokens_per_expert_dev, num_experts,
                          num_experts, total_tokens, N, K, GGO_DTYPE_BF16, tile_config, sort_by_m,
                          workspace_dev, stream, false, &ex);
}

int ggo_grouped_gemm_swiglu_fp8(const void* x_dev, const float* x_scale_dev,
                                const void* w_gate_up_dev, const float* w_scale_dev, void* h_dev,
                                const int64_t* tokens_per_segment_dev, int num_segments,
                                int num_experts, int64_t total_tokens, int64_t F, int64_t K,
                                int sort_by_m, void* workspace_dev, cudaStream_t stream) {
  ggo::GemmExtras ex;
  ex.fp8 = 1;
  ex.row_scale = x_scale_dev;
  ex.col_scale = w_scale_dev;
  return ggo::gemm_common(x_dev, w_gate_up_dev, h_dev, tokens_per_segment_dev, num_segments,
                          num_experts, total_tokens, F, K, GGO_DTYPE_BF16, GGO_TILE_AUTO,
                          sort_by_m, workspace_dev, stream, true, &ex);
}

size_t ggo_mxfp8_scale_bytes(int64_t rows, int num_segments, int64_t k) {
  if (rows < 0 || num_segments < 0 || k <= 0 || k % 128) return 0;
  return static_cast<size_t>(ggo::mx_scale_atoms(rows, num_segments, k)) * 512;
}

int64_t ggo_mxfp8_glu_rows(int64_t F) { return F > 0 ? ggo::mx_glu_rows(F) : 0; }

int ggo_grouped_gemm_mxfp8(const void* input_dev, const void* input_scale_dev,
                           const void* weights_dev, const void* weight_scale_dev, void* output_dev,
                           const int64_t* tokens_per_segment_dev, int num_segments,
                           int num_experts, int64_t total_tokens, int64_t N, int64_t K,
                           int sort_by_m, void* workspace_dev, cudaStream_t stream) {
  ggo::GemmExtras ex;
  ex.fp8 = 1;
  ex.mx = 1;
  ex.a_sf = input_scale_dev;
  ex.b_sf = weight_scale_dev;
  return ggo::gemm_common(input_dev, weights_dev, output_dev, tokens_per_segment_dev, num_segments,
                          num_experts, total_tokens, N, K, GGO_DTYPE_BF16, GGO_TILE_AUTO,
                          sort_by_m, workspace_dev, stream, false, &ex);
}

int ggo_grouped_gemm_swiglu_mxfp8(const void* x_dev, const void* x_scale_dev,
                                  const void* w_gate_up_dev, const void* w_scale_dev, void* h_dev,
                                  const int64_t* tokens_per_segment_dev, int num_segments,
                                  int num_experts, int64_t total_tokens, int64_t F, int64_t K,
                                  int sort_by_m, void* workspace_dev, cudaStream_t stream) {
  ggo::GemmExtras ex;
  ex.fp8 = 1;
  ex.mx = 1;
  ex.a_sf = x_scale_dev;
  ex.b_sf = w_scale_dev;
  return ggo::gemm_common(x_dev, w_gate_up_dev, h_dev, tokens_per_segment_dev, num_segments,
                          num_experts, total_tokens, F, K, GGO_DTYPE_BF16, GGO_TILE_AUTO,
                          sort_by_m, workspace_dev, stream, true, &ex);
}

int ggo_ep_grouped_gemm(const void* input_dev, const void* weights_dev, void* output_dev,
                        const int64_t* tokens_per_segment_dev, int num_segments, int num_experts,
                        int64_t capacity_rows, int64_t N, int64_t K, int dtype, int swiglu,
                        const int32_t* origin_dev, void* const* peer_out, int world_size,
                        int sort_by_m, void* workspace_dev, cudaStream_t stream) {
  ggo::GemmExtras ex;
  ex.rows_is_bound = 1;
  ex.origin = origin_dev;
  ex.peer_out = peer_out;
  ex.world = world_size;
  return ggo::gemm_common(input_dev, weights_dev, output_dev, tokens_per_segment_dev,
                          num_segments, num_experts, capacity_rows, N, K, dtype, GGO_TILE_AUTO,
                          sort_by_m, workspace_dev, stream, swiglu != 0, &ex);
}

int ggo_ipc_alloc(size_t bytes, void** ptr_out, void* handle_out) {
  if (!ptr_out || !handle_out || bytes == 0) return GGO_ERR_INVALID_ARG;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return GGO_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return GGO_ERR_CUDA;
  }
  memcpy(handle_out, &h, sizeof(h));
  *ptr_out = p;
  return GGO_OK;
}

int ggo_ipc_open(const void* handle, void** ptr_out) {
  if (!handle || !ptr_out) return GGO_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return GGO_ERR_CUDA;
  *ptr_out = p;
  return GGO_OK;
}

int ggo_ipc_close(void* peer_ptr) {
  return cudaIpcCloseMemHandle(peer_ptr) == cudaSuccess ? GGO_OK : GGO_ERR_CUDA;
}

int ggo_ipc_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? GGO_OK : GGO_ERR_CUDA; }

uint64_t ggo_kernel_launches(void) {
  return ggo::g_kernel_launches.load(std::memory_order_relaxed);
}

const char* ggo_last_cuda_error_string(void) {
  const int c = ggo::g_last_cuda_error;
  if (c == 0) return "no CUDA error recorded";
  if (c >= 100000) {
    static thread_local char buf[64];
    snprintf(buf, sizeof(buf), "CUDA driver error %d", c - 100000);
    return buf;
  }
  return cudaGetErrorString(static_cast<cudaError_t>(c));
}

int ggo_workspace_error(void* workspace_dev, cudaStream_t stream, int* status_out) {
  if (!workspace_dev || !status_out) return GGO_ERR_INVALID_ARG;
  int code = 0;
  auto* ws = static_cast<ggo::GgoWorkspace*>(workspace_dev);
  if (cudaMemcpyAsync(&code, &ws->error, sizeof(int), cudaMemcpyDeviceToHost, stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return GGO_ERR_CUDA;
  if (code != 0) {
    const int zero = 0;
    if (cudaMemcpyAsync(&ws->error, &zero, sizeof(int), cudaMemcpyHostToDevice, stream) !=
            cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
      return GGO_ERR_CUDA;
  }
  *status_out = ggo::device_error_to_status(code);
  return GGO_OK;
}

}  // extern "C"
