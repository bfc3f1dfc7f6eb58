// Persistent tcgen05 grouped GEMM for sm_100a.
//
//   out[r, :] = epilogue( in[r, :] @ W[expert(r)]^T ),  rows r grouped into contiguous segments.
//
// Replaces the CUTLASS SM90 Ptr-Array grouped GEMM of the reference
// (csrc/grouped_gemm_sm90.cuh:87-152, launched from csrc/grouped_gemm_kernel.cu:195-279) with a
// kernel built around B200 hardware:
//
//  * One flat tile pool across every segment. Each CTA computes the segment table (exclusive
//    prefix sums of the per-segment row counts, optional heavy-first order) from the DEVICE copy of
//    the counts, so the host never reads them (the reference copies them back and synchronises the
//    stream, grouped_gemm_kernel.cu:374-381). Tiles are claimed by atomic work stealing.
//  * No per-group tensor maps: all experts share K, so one 2D TMA map over in[T,K] and one over
//    W viewed as [E*N, K] serve every segment. Rows of a tile past its segment's end are loaded
//    (they belong to the next segment or are TMA zero-fill) and masked at the store.
//  * Warp specialisation: warp 0 = TMA producer, warp 1 = single-thread tcgen05.mma issuer,
//    warp 2 = TMEM allocator, warps 4..7 = epilogue (TMEM -> registers -> shared-memory staging
//    -> TMA stores; masked 16-byte stores where a warp's rows cross a segment boundary).
//    Two TMEM accumulators let the epilogue of tile i overlap the MMAs of tile i+1.
//  * Epilogues: plain store; SwiGLU (silu(gate) * up) for the fused-MoE gate/up projection, where
//    one 256-wide B tile holds 128 gate rows and the matching 128 up rows; row/column-scaled for
//    FP8 operands; and a scatter of each row to its source rank's buffer (expert parallelism).
//  * Operand forms: K-major weights (forward), MN-major weights read in place (dgrad), bf16/fp16
//    (kind::f16) or e4m3 (kind::f8f6f4).
//  * The CTA-pair variant (ggo_gemm_pair.cuh) shares the segment table, tile decode and epilogue.
//
// Every bulk-tensor load writes only the issuing CTA's shared memory, from this GPU's memory.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "ggo_ptx.cuh"

namespace ggo {

constexpr int kBM = 128;          // rows per tile (tcgen05 M)
constexpr int kBK = 64;           // K per pipeline stage: one 128-B swizzle atom of bf16
constexpr int kUmmaK = 16;        // K per tcgen05.mma kind::f16
constexpr int kMaxSegments = 1024;
constexpr int kSchedDepth = 4;
constexpr int kThreads = 256;

// kEpiScaled: out = acc * row_scale[row] * col_scale[expert * n_out + col] (the FP8 path).
// kEpiScaledSwiGLU: silu(gate * rs * cs_gate) * (up * rs * cs_up) (the FP8 gate/up projection).
enum EpiKind { kEpiStore = 0, kEpiSwiGLU = 1, kEpiScaled = 2, kEpiScaledSwiGLU = 3 };

// Epilogues whose B tile is [gate rows | up rows] and whose output is half the tile width.
__host__ __device__ constexpr bool epi_glu(int e) {
  return e == kEpiSwiGLU || e == kEpiScaledSwiGLU;
}

// Error codes written to GgoWorkspace::error (first error wins).
enum DevError {
  kDevOk = 0,
  kDevTimeoutProducer = 101,
  kDevTimeoutMma = 102,
  kDevTimeoutEpilogue = 103,
  kDevCountMismatch = 110,  // sum(counts) != rows of the input
  kDevNegativeCount = 111,
};

// 256 bytes of per-stream scratch. Must be zero before the first launch; each launch leaves the
// two counters at zero again (the last CTA to finish resets them). `error` is sticky.
struct GgoWorkspace {
  int tile_counter;
  int done_counter;
  int error;
  int pad[61];
};

struct GemmParams {
  const int64_t* counts;  // [num_segments] rows per segment, device memory
  int num_segments;       // <= kMaxSegments
  int num_experts;        // segment s multiplies by expert (s % num_experts)
  int rows;               // T = rows of `in` (and of `out`)
  int n_out;              // columns of `out` (N, or F for SwiGLU)
  int n_b;                // rows of one expert's W (N, or 2F for SwiGLU)
  int k;                  // K
  int sort_by_m;          // 0 segment order; 1 heaviest first; 2 heavy and light tiles interleaved
  int group_m;            // m-tiles per raster group (>= 1)
  void* out;              // [rows, n_out], bf16 or fp16
  int rows_is_bound;      // 1: `rows` is a capacity; counts may sum to less (no mismatch error)
  // Scatter epilogue (expert parallelism): when `origin` is set, output row r goes to
  // peer_out[origin[r] >> 28] + (origin[r] & 0x0fffffff) * n_out instead of out + r * n_out.
  const int32_t* origin;
  void* peer_out[8];
  int use_tma_store;      // 1: the output tensor map is valid (plain output, 64-column boxes)
  long long wait_limit;   // bounded-wait limit in SM cycles
  int inject_stall;       // test hook: the tile claimed first never gets its first stage armed
  const float* row_scale; // kEpiScaled: one scale per input row
  const float* col_scale; // kEpiScaled: [num_experts, n_out] scales
  int split_mode;         // 0 all rows; 1 pair pass (no short tails); 2 short tails only
  int split_tail_ntiles;  // column tiles of the tail pass (its output width / its tile width)
  int split_min_tiles;    // split only when the tail pass gets at least this many tiles
  // SwiGLU weight layout: 0 = all gate rows then all up rows; 1 = blocked, output columns
  // [n0, n0 + w) read weight rows [2 n0, 2 n0 + 2w): w gate rows then the w matching up rows,
  // w = the tile's output width (the layout the MX path's weight preparation writes)
  int glu_blocked;
  // Skinny tiles: a tile of at most this many rows (a short segment, or a segment's last rows)
  // runs with the operands swapped -- weight rows on the MMA's M side, the tile's rows on its N
  // side rounded up to 16 -- so the tensor cores do work for the rows that exist instead of a
  // 128-row block. 0 disables. Single-CTA kernel, bf16/fp16 K-major weights, plain or SwiGLU.
  int skinny_max;
  GgoWorkspace* ws;
};

constexpr int kSkinnyRows = 64;  // rows of the input box a skinny tile loads (its row limit)

struct TileInfo {
  int row0;    // first input row of the tile
  int rows;    // valid rows (<= kBM); 0 = no more work
  int n0;      // first output column
  int brow0;   // first W row of box 0 (and box 1 = brow1)
  int brow1;
  int seg;     // segment of the tile
  int skinny;  // 1: swapped-operand tile for a short row block (single-CTA kernel only)
  int pad;
};

template <int BN>
struct SmemLayout {
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  static constexpr int kABytes = kBM * kBK * 2;   // 16 KB
  static constexpr int kBBytes = BN * kBK * 2;    // 32 KB or 16 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTileBytes = kStages * kStageBytes;
  static constexpr int kStagingBytes = 4 * 4096;  // TMA-store staging, 4 KB per epilogue warp
  static constexpr int kTableBytes = 4 * kMaxSegments * 4 + 16;
  static constexpr int kMiscBytes = 1024;
  static constexpr int kTotal =
      1024 /*align slack*/ + kTileBytes + kStagingBytes + kTableBytes + kMiscBytes;
  static_assert(kTotal <= 227 * 1024, "shared memory budget");
};

// Sum of one int per thread over the CTA (all kThreads threads must call it). `partial` is
// kThreads / 32 ints of shared memory free for the duration of the call (no static shared memory:
// it would push the 1024-aligned dynamic region past the per-CTA limit).
__device__ __forceinline__ int block_sum(int v, int* partial) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = v;
  __syncthreads();
  int t = 0;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) t += partial[i];
  __syncthreads();
  return t;
}

// Builds, in shared memory, the segment table every CTA needs to map a flat tile index to work:
// clamped counts, exclusive row offsets (segment order), processing order (identity or heaviest
// first) and exclusive tile offsets (processing order); *total_tiles_s receives the tile count.
// Called by all kThreads threads of the CTA (contains __syncthreads).
template <int TILE_M, int OUT_BN>
__device__ __forceinline__ void build_segment_table(const GemmParams& p, uint8_t* tiles, int* t_cnt,
                                                    int* t_rowoff, int* t_order, int* t_tileoff,
                                                    int* total_tiles_s, int* err) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nseg = p.num_segments;
  // Segment table, computed redundantly by every CTA from the device counts.
  for (int s = threadIdx.x; s < nseg; s += kThreads) {
    long long c = p.counts[s];
    if (c < 0) {
      atomicCAS(err, 0, kDevNegativeCount);
      c = 0;
    }
    t_cnt[s] = c > p.rows ? p.rows : static_cast<int>(c);
  }
  __syncthreads();
  if (warp == 0) {  // exclusive prefix sum of rows, in segment order
    int carry = 0;
    for (int base = 0; base < nseg; base += 32) {
      const int s = base + lane;
      const int v = s < nseg ? t_cnt[s] : 0;
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (s < nseg) t_rowoff[s] = carry + x - v;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
    const bool bad = p.rows_is_bound ? carry > p.rows : carry != p.rows;
    if (lane == 0 && bad && blockIdx.x == 0) atomicCAS(err, 0, kDevCountMismatch);
  }
  if (p.split_mode) {
    // Split launch: a segment's last `small` rows (its count mod 256, when 1..128) go to a
    // 128-row single-CTA pass (mode 2); everything else to the 256-row pair pass (mode 1). Both
    // kernels take the same decision from the same counts: split only when the short tails make
    // at least p.split_min_tiles single-CTA tiles (a tail pass of whole waves), else the pair
    // pass keeps every row and the tail pass has nothing to do.
    __syncthreads();
    int mine = 0;
    for (int s = threadIdx.x; s < nseg; s += kThreads) {
      const int r = t_cnt[s] % 256;
      mine += (r > 0 && r <= 128) ? 1 : 0;
    }
    const int tails = block_sum(mine, t_tileoff);  // t_tileoff is filled later
    const bool split = static_cast<long long>(tails) * p.split_tail_ntiles >= p.split_min_tiles;
    for (int s = threadIdx.x; s < nseg; s += kThreads) {
      const int c = t_cnt[s];
      const int r = c % 256;
      const int small = (split && r > 0 && r <= 128) ? r : 0;
      if (p.split_mode == 1) {
        t_cnt[s] = c - small;
      } else {
        t_rowoff[s] += c - small;
        t_cnt[s] = small;
      }
    }
    __syncthreads();
  }
  // Processing order: identity, or heaviest segment first (ties by index) via a bitonic sort of
  // 64-bit keys held temporarily in the (still unused) operand tile buffers.
  if (p.sort_by_m && nseg > 1) {
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(tiles);
    int n2 = 1;
    while (n2 < nseg) n2 <<= 1;
    for (int i = threadIdx.x; i < n2; i += kThreads) {
      keys[i] = i < nseg ? (static_cast<unsigned long long>(0x7fffffff - t_cnt[i]) << 32) |
                               static_cast<unsigned>(i)
                         : ~0ull;
    }
    __syncthreads();
    for (int size = 2; size <= n2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = threadIdx.x; i < n2; i += kThreads) {
          const int j = i ^ stride;
          if (j > i) {
            const bool up = (i & size) == 0;
            const unsigned long long a = keys[i], b = keys[j];
            if ((a > b) == up) {
              keys[i] = b;
              keys[j] = a;
            }
          }
        }
        __syncthreads();
      }
    }
    for (int i = threadIdx.x; i < nseg; i += kThreads)
      t_order[i] = static_cast<int>(keys[i] & 0xffffffffu);
  } else {
    for (int i = threadIdx.x; i < nseg; i += kThreads) t_order[i] = i;
  }
  __syncthreads();
  const int n_tiles = (p.n_out + OUT_BN - 1) / OUT_BN;
  if (warp == 0) {  // exclusive prefix sum of tiles, in processing order
    int carry = 0;
    for (int base = 0; base < nseg; base += 32) {
      const int i = base + lane;
      const int v = i < nseg ? ((t_cnt[t_order[i]] + TILE_M - 1) / TILE_M) * n_tiles : 0;
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (i < nseg) t_tileoff[i] = carry + x - v;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) {
      t_tileoff[nseg] = carry;
      *total_tiles_s = carry;
    }
    // Tile-level interleave (sort_by_m == 2): the tiles of segments with at least one full row
    // block ("heavy", compute-bound) alternate with those of shorter segments ("light",
    // weight-streaming), so the tensor pipe and HBM work at the same time. total_tiles_s[1]
    // receives the heavy tile count (the processing order is heaviest first), -1 for no interleave.
    __syncwarp();
    int h = 0;
    if (p.sort_by_m == 2) {
      for (int base = 0; base < nseg; base += 32) {
        const int i = base + lane;
        const unsigned heavy = __ballot_sync(0xffffffffu, i < nseg && t_cnt[t_order[i]] >= TILE_M);
        h += __popc(heavy);
        if (heavy != 0xffffffffu) break;
      }
    }
    if (lane == 0) total_tiles_s[1] = (p.sort_by_m == 2 && h > 0 && h < nseg) ? t_tileoff[h] : -1;
  }
}

// Position in the heaviest-first tile order of the t-th claimed tile when heavy and light tiles
// alternate (`heavy` = heavy tile count, -1: no interleave): heavy tiles are [0, heavy), light
// ones [heavy, total); pairs (heavy i, light i) come first, then the longer list's remainder.
__device__ __forceinline__ int interleave_tile(int t, int heavy, int total) {
  if (heavy < 0) return t;
  const int light = total - heavy;
  const int m = heavy < light ? heavy : light;
  if (t < 2 * m) return (t & 1) ? heavy + (t >> 1) : (t >> 1);
  return heavy > light ? t - light : t;
}

// Maps flat tile index t (< total tiles) to its rows, output columns and weight rows.
// Tiles of one segment are rastered in groups of p.group_m m-tiles: inside a group the m index
// runs fastest, so concurrently running CTAs share the weight tile in L2.
// After an abort, waits (bounded by `limit` cycles per stage) for the bulk loads this producer
// issued into stages the MMA never consumed, so no copy is still landing in shared memory when the
// CTA exits. Stage s was last armed with phase parity bit s of `armed_par`.
template <int S>
__device__ __forceinline__ void drain_armed_stages(uint64_t* full_bar, uint32_t armed,
                                                   uint32_t armed_par, long long limit) {
  for (int s = 0; s < S; ++s) {
    if (!(armed >> s & 1u)) continue;
    const uint32_t a = smem_u32(&full_bar[s]);
    const uint32_t par = armed_par >> s & 1u;
    const long long t0 = clock64();
    while (!mbar_try_wait(a, par) && clock64() - t0 < limit) {
    }
  }
}

template <int TILE_M, int OUT_BN, int EPI, int B_HALF, bool BMN = false>
__device__ __forceinline__ TileInfo decode_tile(int t, const GemmParams& p, const int* t_cnt,
                                                const int* t_rowoff, const int* t_order,
                                                const int* t_tileoff) {
  const int nseg = p.num_segments;
  const int n_tiles = (p.n_out + OUT_BN - 1) / OUT_BN;
  int lo = 0, hi = nseg - 1;  // last position whose tile offset is <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (t_tileoff[mid] <= t) lo = mid; else hi = mid - 1;
  }
  const int seg = t_order[lo];
  const int local = t - t_tileoff[lo];
  const int mt = (t_cnt[seg] + TILE_M - 1) / TILE_M;
  const int gsz = p.group_m;
  const int group = local / (gsz * n_tiles);
  const int first_m = group * gsz;
  const int gm = min(gsz, mt - first_m);
  const int r = local - group * gsz * n_tiles;
  const int m_idx = first_m + r % gm;
  const int n_idx = r / gm;
  const int expert = seg % p.num_experts;
  TileInfo info;
  info.row0 = t_rowoff[seg] + m_idx * TILE_M;
  info.rows = min(TILE_M, t_cnt[seg] - m_idx * TILE_M);
  info.seg = seg;
  info.n0 = n_idx * OUT_BN;
  if (BMN) {
    // MN-major weights [E, Kred, n_out]: rows are the reduction index; the column is n0
    info.brow0 = expert * p.k;
    info.brow1 = info.brow0;
  } else if (epi_glu(EPI) && p.glu_blocked) {
    info.brow0 = expert * p.n_b + 2 * info.n0;  // gate rows, then the up rows of the same block
    info.brow1 = info.brow0 + B_HALF;
  } else if (epi_glu(EPI)) {
    info.brow0 = expert * p.n_b + info.n0;                 // gate rows
    info.brow1 = expert * p.n_b + (p.n_b >> 1) + info.n0;  // matching up rows
  } else {
    info.brow0 = expert * p.n_b + info.n0;
    info.brow1 = info.brow0 + B_HALF;  // second half of the B tile
  }
  return info;
}

__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf16) {
  if (bf16) {
    __nv_bfloat162 t2 = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&t2);
  }
  __half2 t2 = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&t2);
}

// 32 output columns of this thread's accumulator row, packed as 16 bf16x2/half2 words: TMEM
// columns [c, c+32) (plain), or silu(gate) * up from columns [c, c+32) and [BN/2 + c, ...).
template <int BN, int EPI, bool BF16>
__device__ __forceinline__ void load_out32(uint32_t t_row, int c, uint32_t (&o)[16], float rs = 1.f,
                                           const float* cs = nullptr, int cs_valid = 0,
                                           int cs_up_off = 0) {
  if (EPI == kEpiScaledSwiGLU) {
    uint32_t g[32], u[32];
    tmem_ld_32x32b_x32(t_row + c, g);
    tmem_ld_32x32b_x32(t_row + BN / 2 + c, u);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float y[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = 2 * i + e;
        const bool ok = j < cs_valid;
        const float gv = __uint_as_float(g[j]) * rs * (ok ? __ldg(cs + j) : 0.f);
        const float uv = __uint_as_float(u[j]) * rs * (ok ? __ldg(cs + cs_up_off + j) : 0.f);
        y[e] = gv / (1.0f + __expf(-gv)) * uv;
      }
      o[i] = pack2(y[0], y[1], BF16);
    }
  } else if (EPI == kEpiScaled) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(t_row + c, v);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float s0 = 2 * i < cs_valid ? __ldg(cs + 2 * i) : 0.f;
      const float s1 = 2 * i + 1 < cs_valid ? __ldg(cs + 2 * i + 1) : 0.f;
      o[i] = pack2(__uint_as_float(v[2 * i]) * rs * s0, __uint_as_float(v[2 * i + 1]) * rs * s1,
                   BF16);
    }
  } else if (EPI == kEpiStore) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(t_row + c, v);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i)
      o[i] = pack2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]), BF16);
  } else {
    uint32_t g[32], u[32];
    tmem_ld_32x32b_x32(t_row + c, g);
    tmem_ld_32x32b_x32(t_row + BN / 2 + c, u);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float y[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float gv = __uint_as_float(g[2 * i + e]);
        const float uv = __uint_as_float(u[2 * i + e]);
        y[e] = gv / (1.0f + __expf(-gv)) * uv;
      }
      o[i] = pack2(y[0], y[1], BF16);
    }
  }
}

// Epilogue of one warp's 32 accumulator rows (one row per thread, TMEM lane quarter `t_row`):
// output columns n0 + [0, OUTW), OUTW = BN (plain) or BN / 2 (SwiGLU). All 32 lanes must call it
// (tcgen05.ld is warp-collective).
//  * warp_tma: the warp's 32 rows all belong to the tile's segment and an output tensor map
//    exists. Each 64-column box is staged in `stage` (4 KB, 1024-B aligned, rows of 128 B with
//    the 128-B swizzle: 16-B chunk j of row r at chunk j ^ (r % 8), conflict-free) and written
//    with one TMA store; the box at x0 = n0 + c64, y0 = x_row0. Columns past n_out are clipped by
//    the tensor map.
//  * row_copy (scatter epilogue, rows going to scattered destinations, often another GPU): the
//    box is staged the same way, then copied out row by row -- eight lanes write one row's 128
//    contiguous bytes -- so each store instruction sends whole rows instead of 16-byte pieces of
//    32 different rows.
//  * otherwise each thread stores its own row with 16-byte stores, masked by row_ok and n_out.
template <int BN, int EPI, bool BF16, typename OutT>
__device__ __forceinline__ void store_tile_rows(uint32_t t_row, int n0, int n_out, bool row_ok,
                                                OutT* out_row, bool warp_tma,
                                                const CUtensorMap* tmC, uint8_t* stage,
                                                int x_row0, float rs = 1.f,
                                                const float* cs_row = nullptr,
                                                int cs_up_off = 0, bool row_copy = false,
                                                int first_box = 0, uint32_t release_bar = 0) {
  constexpr int OUTW = epi_glu(EPI) ? BN / 2 : BN;
  constexpr int kBoxes = (OUTW + 63) / 64;
  const int lane = threadIdx.x & 31;
  const uint32_t st_row = smem_u32(stage) + lane * 128;
  // Output boxes run from `first_box` round to first_box - 1. With `release_bar` (a cluster
  // address) the warp arrives on it once the first box's TMEM columns are read.
  auto release = [&]() {
    if (release_bar != 0u) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(release_bar);
    }
  };
  if (warp_tma && OUTW % 64 == 0) {
    // TMA-store path, software-pipelined: box i+1 is read from TMEM (and converted) while the
    // bulk store of box i still reads the staging buffer, so the two latencies overlap instead of
    // adding up box after box.
    uint32_t o[32];
    const int f64 = 64 * first_box;
    load_out32<BN, EPI, BF16>(t_row, f64, *reinterpret_cast<uint32_t(*)[16]>(o), rs,
                              cs_row ? cs_row + n0 + f64 : nullptr, n_out - (n0 + f64), cs_up_off);
    load_out32<BN, EPI, BF16>(t_row, f64 + 32, *reinterpret_cast<uint32_t(*)[16]>(o + 16), rs,
                              cs_row ? cs_row + n0 + f64 + 32 : nullptr, n_out - (n0 + f64 + 32),
                              cs_up_off);
    release();
#pragma unroll 1
    for (int b = 0; b < kBoxes; ++b) {
      const int c64 = 64 * ((first_box + b) % kBoxes);
      // the previous box's store -- for box 0 the last store of this warp's previous tile -- has
      // finished reading the staging buffer
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t chunk = static_cast<uint32_t>(q ^ (lane & 7));
        st_shared_v4(st_row + chunk * 16, o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmC, stage, n0 + c64, x_row0);
        bulk_commit();
      }
      const int nx = 64 * ((first_box + b + 1) % kBoxes);
      if (b + 1 < kBoxes) {
        load_out32<BN, EPI, BF16>(t_row, nx, *reinterpret_cast<uint32_t(*)[16]>(o), rs,
                                  cs_row ? cs_row + n0 + nx : nullptr, n_out - (n0 + nx),
                                  cs_up_off);
        load_out32<BN, EPI, BF16>(t_row, nx + 32, *reinterpret_cast<uint32_t(*)[16]>(o + 16), rs,
                                  cs_row ? cs_row + n0 + nx + 32 : nullptr,
                                  n_out - (n0 + nx + 32), cs_up_off);
      }
    }
    return;
  }
  const bool staged = warp_tma || row_copy;
#pragma unroll 1
  for (int b = 0; b < kBoxes; ++b) {
    const int c64 = 64 * ((first_box + b) % kBoxes);
    if (warp_tma) {  // the previous box's store (for box 0: of the previous tile) has read it
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
    }
#pragma unroll 1
    for (int s = 0; s < 2; ++s) {
      const int c = c64 + 32 * s;
      if (c >= OUTW) break;
      uint32_t o[16];
      load_out32<BN, EPI, BF16>(t_row, c, o, rs, cs_row ? cs_row + n0 + c : nullptr,
                                n_out - (n0 + c), cs_up_off);
      if (staged) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t chunk = static_cast<uint32_t>((4 * s + q) ^ (lane & 7));
          st_shared_v4(st_row + chunk * 16, o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
        }
      } else if (row_ok) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int col = n0 + c + 8 * q;
          if (col < n_out)
            *reinterpret_cast<uint4*>(out_row + col) =
                make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
        }
      }
    }
    if (b == 0) release();
    if (warp_tma) {
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmC, stage, n0 + c64, x_row0);
        bulk_commit();
      }
    } else if (row_copy) {
      __syncwarp();
      const int box_cols = OUTW - c64 < 64 ? OUTW - c64 : 64;
      const int chunk = lane & 7;
      const uint32_t base = smem_u32(stage);
#pragma unroll 1
      for (int it = 0; it < 8; ++it) {
        const int row = it * 4 + (lane >> 3);
        const unsigned long long rp =
            __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(out_row), row);
        const int rok = __shfl_sync(0xffffffffu, row_ok ? 1 : 0, row);
        const int col = n0 + c64 + chunk * 8;
        if (rok && chunk * 8 < box_cols && col < n_out) {
          const uint4 v = ld_shared_v4(base + row * 128 + ((chunk ^ (row & 7)) * 16));
          *reinterpret_cast<uint4*>(reinterpret_cast<OutT*>(rp) + col) = v;
        }
      }
      __syncwarp();  // the next box reuses the staging buffer
    }
  }
}

// Destination of accumulator row r_local of a tile: the local output row, or (scatter epilogue)
// the row on the source rank given by `origin`, through that rank's peer mapping.
template <typename OutT>
__device__ __forceinline__ OutT* output_row(const GemmParams& p, const TileInfo& info, int r_local,
                                            bool row_ok) {
  const int r = info.row0 + r_local;
  if (p.origin == nullptr || !row_ok)
    return reinterpret_cast<OutT*>(p.out) + static_cast<size_t>(r) * p.n_out;
  const int o = p.origin[r];  // (source rank << 28) | row on the source rank
  return reinterpret_cast<OutT*>(p.peer_out[(o >> 28) & 7]) +
         static_cast<size_t>(o & 0x0fffffff) * p.n_out;
}

// Epilogue of a skinny (swapped-operand) tile. The accumulator is transposed: TMEM lane = weight
// row, column = the tile's input row. The warp holding lanes [32 ew, 32 ew + 32) of weight half h
// (TMEM columns [128 h, 128 h + 64)) owns output columns n0 + 128 h + 32 ew + lane (plain), or
// n0 + 32 ew + lane with gate in half 0 and up in half 1 (SwiGLU). For every input row of the
// tile the 32 lanes store 32 consecutive output columns (64 contiguous bytes). All 32 lanes must
// call it (tcgen05.ld is warp-collective).
template <int BN, int EPI, bool BF16, typename OutT>
__device__ __forceinline__ void store_skinny(uint32_t t_row, const GemmParams& p,
                                             const TileInfo& info, int ew) {
  const int lane = threadIdx.x & 31;
  constexpr int kHalves = epi_glu(EPI) ? 1 : BN / 128;
#pragma unroll 1
  for (int h = 0; h < kHalves; ++h) {
    const int col = info.n0 + 128 * h + 32 * ew + lane;
    const bool col_ok = col < p.n_out;
#pragma unroll 1
    for (int cb = 0; cb < info.rows; cb += 32) {
      uint32_t v[32];
      uint32_t u[32];
      tmem_ld_32x32b_x32(t_row + 128 * h + cb, v);
      if (epi_glu(EPI)) tmem_ld_32x32b_x32(t_row + 128 + cb, u);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int r = cb + j;
        const bool ok = r < info.rows && info.row0 + r < p.rows;
        float y = __uint_as_float(v[j]);
        if (epi_glu(EPI)) y = y / (1.0f + __expf(-y)) * __uint_as_float(u[j]);
        OutT* dst = output_row<OutT>(p, info, r, ok);
        if (ok && col_ok) dst[col] = static_cast<OutT>(y);
      }
    }
  }
}

template <int BN, int EPI, bool BF16, bool BMN = false, bool FP8 = false>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC,
                        const __grid_constant__ CUtensorMap tmAs, const GemmParams p) {
  using L = SmemLayout<BN>;
  constexpr int S = L::kStages;
  constexpr int kTmemCols = 2 * BN;             // two accumulators
  constexpr int kOutBN = epi_glu(EPI) ? BN / 2 : BN;
  constexpr bool kTmaStoreOk = kOutBN % 64 == 0;  // output boxes are 64 columns wide
  // skinny tiles: tmAs is the input map with kSkinnyRows-row boxes
  constexpr bool kSkinnyOk = !FP8 && !BMN && (EPI == kEpiStore || EPI == kEpiSwiGLU);
  constexpr int kSkinnyABytes = kSkinnyRows * kBK * 2;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* tiles = smem;
  uint8_t* staging = smem + L::kTileBytes;
  int* t_cnt = reinterpret_cast<int*>(smem + L::kTileBytes + L::kStagingBytes);
  int* t_rowoff = t_cnt + kMaxSegments;
  int* t_order = t_rowoff + kMaxSegments;
  int* t_tileoff = t_order + kMaxSegments;  // kMaxSegments + 1 entries
  uint8_t* misc = smem + L::kTileBytes + L::kStagingBytes + L::kTableBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(misc);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* accf_bar = empty_bar + S;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* schf_bar = acce_bar + 2;
  uint64_t* sche_bar = schf_bar + kSchedDepth;
  TileInfo* ring = reinterpret_cast<TileInfo*>(sche_bar + kSchedDepth);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring + kSchedDepth);
  int* total_tiles_s = reinterpret_cast<int*>(tmem_slot + 1);
  WaitGuard* guard = reinterpret_cast<WaitGuard*>(tmem_slot + 4);  // 16-byte aligned

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = &p.ws->error;

  // ------------------------------------------------------------------ set-up
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf_bar[i], 1);
      mbar_init(&acce_bar[i], 4);
    }
    for (int i = 0; i < kSchedDepth; ++i) {
      mbar_init(&schf_bar[i], 1);
      mbar_init(&sche_bar[i], 1 + 4);
    }
    guard->abort = 0;
    guard->limit = p.wait_limit;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }

  build_segment_table<kBM, kOutBN>(p, tiles, t_cnt, t_rowoff, t_order, t_tileoff, total_tiles_s, err);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = *total_tiles_s;
  const int heavy_tiles = total_tiles_s[1];
  // K elements per pipeline stage: one 128-B swizzle row (64 bf16/fp16 or 128 e4m3)
  constexpr int kStageK = FP8 ? 128 : kBK;
  const int num_kb = (p.k + kStageK - 1) / kStageK;

  if (warp == 0) {
    // -------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0, phase = 0, q = 0, qphase = 0;
      uint32_t armed = 0, armed_par = 0;  // stages whose loads were issued, and their parity
      while (true) {
        const int t = atomicAdd(&p.ws->tile_counter, 1);
        TileInfo info;
        info.rows = 0;
        if (t < total_tiles)
          info = decode_tile<kBM, kOutBN, EPI, 128, BMN>(interleave_tile(t, heavy_tiles, total_tiles),
                                                        p, t_cnt, t_rowoff, t_order, t_tileoff);
        info.skinny = (kSkinnyOk && info.rows > 0 && info.rows <= p.skinny_max) ? 1 : 0;
        if (!mbar_wait(&sche_bar[q], qphase ^ 1, guard, err, kDevTimeoutProducer)) break;
        ring[q] = info;
        mbar_arrive(&schf_bar[q]);
        if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
        if (info.rows == 0) break;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, guard, err, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          // test hook: the CTA that claimed tile 0 leaves that tile's first stage unarmed, so its
          // MMA's bounded wait expires
          const bool skip = p.inject_stall && t == 0 && kb == 0;
          if (!skip) {
            uint8_t* a_dst = tiles + stage * L::kStageBytes;
            uint8_t* b_dst = a_dst + L::kABytes;
            if (kSkinnyOk && info.skinny) {  // only the tile's first kSkinnyRows input rows
              mbar_arrive_expect_tx(&full_bar[stage], kSkinnyABytes + L::kBBytes);
              tma_load_2d(a_dst, &tmAs, &full_bar[stage], kb * kStageK, info.row0);
            } else {
              mbar_arrive_expect_tx(&full_bar[stage], L::kStageBytes);
              tma_load_2d(a_dst, &tmA, &full_bar[stage], kb * kStageK, info.row0);
            }
            if (BMN) {  // BN/64 boxes of [64 reduction rows][64 output columns]
#pragma unroll
              for (int i = 0; i < BN / 64; ++i)
                tma_load_2d(b_dst + i * 8192, &tmB, &full_bar[stage], info.n0 + 64 * i,
                            info.brow0 + kb * kBK);
            } else {
              tma_load_2d(b_dst, &tmB, &full_bar[stage], kb * kStageK, info.brow0);
              if (BN == 256)
                tma_load_2d(b_dst + 128 * 128, &tmB, &full_bar[stage], kb * kStageK, info.brow1);
            }
            armed |= 1u << stage;
            armed_par = (armed_par & ~(1u << stage)) | (static_cast<uint32_t>(phase) << stage);
          }
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      if (guard->abort) drain_armed_stages<S>(full_bar, armed, armed_par, guard->limit);
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      // e4m3 operands are format 0 of kind::f8f6f4, the same bits as f16 in kind::f16
      constexpr uint32_t idesc = idesc_f16(kBM, BN, FP8 ? false : BF16, BMN);
      int stage = 0, phase = 0, q = 0, qphase = 0, acc = 0, aphase = 0;
      const uint32_t tiles_addr = smem_u32(tiles);
      while (true) {
        if (!mbar_wait(&schf_bar[q], qphase, guard, err, kDevTimeoutMma)) break;
        const bool valid = ring[q].rows > 0;
        const bool skinny = kSkinnyOk && ring[q].skinny;
        // skinny: M = 128 weight rows per MMA, N = the tile's rows rounded up to 16
        const uint32_t idesc_s = idesc_f16(kBM, (ring[q].rows + 15) & ~15, BF16, false);
        mbar_arrive(&sche_bar[q]);
        if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
        if (!valid) break;
        if (!mbar_wait(&acce_bar[acc], aphase ^ 1, guard, err, kDevTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, guard, err, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = tiles_addr + stage * L::kStageBytes;
          const uint64_t adesc = sdesc_sw128_kmajor(a_addr);
          const uint64_t bdesc = BMN ? sdesc_sw128_mnmajor(a_addr + L::kABytes, 8192)
                                     : sdesc_sw128_kmajor(a_addr + L::kABytes);
          // per 16-element K step: A (K-major) advances 32 B inside its swizzle atom; a K-major
          // B likewise, an MN-major B by 16 rows of 128 B (two 8-row atoms)
          constexpr uint64_t kBStep = BMN ? (2048 >> 4) : 2;
          if (kSkinnyOk && skinny) {
            // weights (the B slot, 128 rows per half) as the M-side operand, the tile's rows
            // (the A slot) as the N side; half h accumulates into TMEM columns [128 h, ...)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
              for (int h = 0; h < BN / 128; ++h)
                mma_f16_ss(d_tmem + 128 * h,
                           sdesc_sw128_kmajor(a_addr + L::kABytes + h * 16384) + 2 * kk,
                           adesc + 2 * kk, idesc_s, (kb | kk) != 0);
            }
            mma_commit(&empty_bar[stage]);
            if (++stage == S) { stage = 0; phase ^= 1; }
            continue;
          }
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {  // four 32-byte K steps per 128-byte stage row
            if (FP8)
              mma_f8_ss(d_tmem, adesc + 2 * kk, bdesc + kBStep * kk, idesc, (kb | kk) != 0);
            else
              mma_f16_ss(d_tmem, adesc + 2 * kk, bdesc + kBStep * kk, idesc, (kb | kk) != 0);
          }
          mma_commit(&empty_bar[stage]);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(&accf_bar[acc]);
        if (++acc == 2) { acc = 0; aphase ^= 1; }
      }
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- epilogue
    const int ew = warp - 4;  // TMEM lane quarter this warp may access
    int q = 0, qphase = 0, acc = 0, aphase = 0;
    while (true) {
      if (!mbar_wait(&schf_bar[q], qphase, guard, err, kDevTimeoutEpilogue)) break;
      const TileInfo info = ring[q];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sche_bar[q]);
      if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
      if (info.rows == 0) break;
      if (!mbar_wait(&accf_bar[acc], aphase, guard, err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int r_local = ew * 32 + lane;
      const bool row_ok = r_local < info.rows && info.row0 + r_local < p.rows;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + acc * BN;
      using OutT = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      if (kSkinnyOk && info.skinny) {
        store_skinny<BN, EPI, BF16, OutT>(t_row, p, info, ew);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce_bar[acc]);
        if (++acc == 2) { acc = 0; aphase ^= 1; }
        continue;
      }
      OutT* out_row = output_row<OutT>(p, info, r_local, row_ok);
      const bool warp_tma = kTmaStoreOk && p.use_tma_store && ew * 32 + 32 <= info.rows;
      constexpr bool kScaled = EPI == kEpiScaled || EPI == kEpiScaledSwiGLU;
      const float rs = (kScaled && row_ok) ? __ldg(p.row_scale + info.row0 + r_local) : 1.f;
      // column scales: one per weight row, [E, n_b] (gate rows then up rows for SwiGLU)
      const float* cs_row =
          kScaled ? p.col_scale + static_cast<size_t>(info.seg % p.num_experts) * p.n_b : nullptr;
      store_tile_rows<BN, EPI, BF16>(t_row, info.n0, p.n_out, row_ok, out_row, warp_tma, &tmC,
                                     staging + ew * 4096, info.row0 + ew * 32, rs, cs_row,
                                     p.n_b / 2, p.origin != nullptr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce_bar[acc]);
      if (++acc == 2) { acc = 0; aphase ^= 1; }
    }
  }

  // ------------------------------------------------------------------ tear-down
  if (p.origin) __threadfence_system();  // scattered rows visible to the peers before exit
  if (warp >= 4 && lane == 0) bulk_wait_all();  // TMA stores done before shared memory goes
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(&p.ws->done_counter, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      atomicExch(&p.ws->tile_counter, 0);
      atomicExch(&p.ws->done_counter, 0);
    }
  }
}

}  // namespace ggo
