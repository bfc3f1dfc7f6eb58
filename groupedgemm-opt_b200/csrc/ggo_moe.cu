// Fused-MoE data-movement kernels: router top-k, deterministic permute/gather, weighted combine.
//
// The reference has no router, permute or combine: its "fused MoE" entry point
// (grouped_gemm_opt/triton_fused_moe.py:81-150) gathers through an identity `sorted_ids` and
// computes the plain grouped GEMM. These kernels are the stages the layer needs around the
// grouped GEMMs (ggo_gemm.cu), all stream-ordered and free of host synchronisation.
//
// Determinism: the only atomics are per-block expert histograms (order-independent sums). Sorted
// positions come from per-block offsets (an exclusive scan over blocks) plus in-block ranks from
// one warp walking the block's (token, slot) entries in order, so every position is a pure
// function of the routing: expert-major, then token index.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "ggo.h"
#include "ggo_internal.h"

namespace ggo {
namespace {

constexpr int kRouteTokens = 32;   // tokens per route/dispatch block
constexpr int kMaxPeers = 8;       // expert-parallel ranks a dispatch can address
constexpr int kRouteThreads = 256;
constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 16;

// Monotone float -> uint32 map (larger float -> larger key); 0 is below every real key and marks
// an expert already chosen.
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t b = __float_as_uint(f);
  const uint32_t k = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return k == 0 ? 1u : k;
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);
}

// grid = ceil(T / kRouteTokens); dynamic smem = (8 warps * E + E) * 4 bytes.
__global__ void __launch_bounds__(kRouteThreads)
    route_kernel(const float* __restrict__ logits, int T, int E, int K,
                 int32_t* __restrict__ topk_ids, float* __restrict__ topk_w,
                 int* __restrict__ block_counts) {
  extern __shared__ uint32_t rsm[];
  uint32_t* hist = rsm;                     // [E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t* keys = rsm + E + warp * E;      // [E] per warp
  for (int e = threadIdx.x; e < E; e += kRouteThreads) hist[e] = 0;
  __syncthreads();
  const int t0 = blockIdx.x * kRouteTokens;
  for (int tl = warp; tl < kRouteTokens; tl += kRouteThreads / 32) {
    const int t = t0 + tl;
    if (t >= T) break;
    const float* row = logits + static_cast<size_t>(t) * E;
    for (int e = lane; e < E; e += 32) keys[e] = fkey(row[e]);
    __syncwarp();
    float vals[kMaxTopK];
    int ids[kMaxTopK];
    for (int j = 0; j < K; ++j) {
      // (key, lower index wins) packed so that a plain max picks the right element
      unsigned long long best = 0;
      for (int e = lane; e < E; e += 32) {
        const unsigned long long c =
            (static_cast<unsigned long long>(keys[e]) << 32) | (0xffffffffu - static_cast<uint32_t>(e));
        best = c > best ? c : best;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      const int id = static_cast<int>(0xffffffffu - static_cast<uint32_t>(best & 0xffffffffu));
      ids[j] = id;
      vals[j] = fkey_inv(static_cast<uint32_t>(best >> 32));
      __syncwarp();
      if (lane == 0) keys[id] = 0;
      __syncwarp();
    }
    if (lane == 0) {
      // softmax over the selected logits (vals[0] is the maximum)
      float s = 0.f, ex[kMaxTopK];
      for (int j = 0; j < K; ++j) {
        ex[j] = expf(vals[j] - vals[0]);
        s += ex[j];
      }
      const float inv = 1.0f / s;
      for (int j = 0; j < K; ++j) {
        topk_ids[static_cast<size_t>(t) * K + j] = ids[j];
        topk_w[static_cast<size_t>(t) * K + j] = ex[j] * inv;
        atomicAdd(&hist[ids[j]], 1u);
      }
    }
    __syncwarp();
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kRouteThreads)
    block_counts[static_cast<size_t>(blockIdx.x) * E + e] = static_cast<int>(hist[e]);
}

// One block of 1024 threads. Turns block_counts[b][e] into absolute start rows (in place),
// writes tokens_per_expert and the exclusive start row of every expert (expert_start[E], stored
// right after the nblocks x E table). Each expert's column of the table is split into
// P = 1024 / E contiguous block ranges, one per thread: range sums, a per-expert scan of the P
// partial sums, a scan over experts, then every thread rewrites its range.
__global__ void __launch_bounds__(1024)
    route_scan_kernel(int* __restrict__ block_counts, int nblocks, int E,
                      int64_t* __restrict__ tpe) {
  __shared__ int part[1024];   // [E][P] range sums, then exclusive range offsets within expert
  __shared__ int tot[kMaxExperts];
  int* expert_start = block_counts + static_cast<size_t>(nblocks) * E;
  const int P = max(1, 1024 / E);
  const int tid = threadIdx.x;
  const int e = tid / P, q = tid % P;
  const bool active = e < E;
  const int per = (nblocks + P - 1) / P;
  const int b0 = min(nblocks, q * per), b1 = min(nblocks, b0 + per);
  int sum = 0;
  if (active)
    for (int b = b0; b < b1; ++b) sum += block_counts[static_cast<size_t>(b) * E + e];
  part[tid] = sum;
  __syncthreads();
  if (tid < E) {  // exclusive scan of expert tid's P range sums
    int run = 0;
    for (int j = 0; j < P; ++j) {
      const int v = part[tid * P + j];
      part[tid * P + j] = run;
      run += v;
    }
    tot[tid] = run;
  }
  __syncthreads();
  // exclusive scan over experts (E <= 1024): inclusive Hillis-Steele on a copy
  __shared__ int inc[kMaxExperts];
  if (tid < kMaxExperts) inc[tid] = tid < E ? tot[tid] : 0;
  __syncthreads();
  for (int o = 1; o < kMaxExperts; o <<= 1) {
    const int v = (tid < kMaxExperts && tid >= o) ? inc[tid - o] : 0;
    __syncthreads();
    if (tid < kMaxExperts) inc[tid] += v;
    __syncthreads();
  }
  if (tid < E) {
    tpe[tid] = tot[tid];
    expert_start[tid] = inc[tid] - tot[tid];
  }
  if (active) {
    int run = inc[e] - tot[e] + part[tid];
    for (int b = b0; b < b1; ++b) {
      const size_t i = static_cast<size_t>(b) * E + e;
      const int c = block_counts[i];
      block_counts[i] = run;
      run += c;
    }
  }
}

// Where dispatched rows go. world == 1: recv[0] is the local expert-sorted buffer and a row's
// destination is its sorted position. world > 1 (expert parallelism): rank r owns experts
// [r*el, (r+1)*el); recv[r] is rank r's receive buffer (a peer mapping for r != rank) laid out
// expert-major, [local expert][source rank], with sizes from counts_all [world][E] (every rank's
// tokens_per_expert), so each local expert is one contiguous segment; origin[r][dst] receives
// (source rank << 28) | the row's sorted position on the source (where its result goes back).
template <typename T16>
struct DispatchTargets {
  int world;
  int rank;
  int el;
  const int64_t* counts_all;
  T16* recv[kMaxPeers];
  int32_t* origin[kMaxPeers];
};

// grid = ceil(T / kRouteTokens). Sorted positions by one warp (deterministic in-block ranks),
// destination rows from per-expert bases, then the row copy by all warps (each token's row read
// once, written top_k times, four 16-byte chunks in flight per lane).
template <typename T16>
__global__ void __launch_bounds__(kRouteThreads)
    dispatch_kernel(const T16* __restrict__ x, int T, int H, int E, int K,
                    const int32_t* __restrict__ topk_ids, const int* __restrict__ block_offsets,
                    const int* __restrict__ expert_start, const DispatchTargets<T16> tg,
                    int32_t* __restrict__ sorted_token, int32_t* __restrict__ slot_pos) {
  extern __shared__ int psm[];
  int* off = psm;             // [E] running sorted position per expert (this block)
  int* dbase = psm + E;       // [E] destination row of the expert's first row from this rank
  int* pos = dbase + E;       // [kRouteTokens * K] sorted position per entry
  int* drow = pos + kRouteTokens * K;  // [kRouteTokens * K] destination row per entry
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kRouteTokens;
  const int ntok = min(kRouteTokens, T - t0);
  const int nent = ntok * K;
  for (int e = threadIdx.x; e < E; e += kRouteThreads) {
    off[e] = block_offsets[static_cast<size_t>(blockIdx.x) * E + e];
    if (tg.world == 1) {
      dbase[e] = expert_start[e];
    } else {
      // owner's receive buffer is expert-major: all rows of its lower local experts (from every
      // source), then this expert's rows from lower source ranks
      const int r = e / tg.el, le = e % tg.el;
      long long b = 0;
      for (int j = 0; j < le; ++j)
        for (int s = 0; s < tg.world; ++s)
          b += tg.counts_all[static_cast<size_t>(s) * E + r * tg.el + j];
      for (int s = 0; s < tg.rank; ++s) b += tg.counts_all[static_cast<size_t>(s) * E + e];
      dbase[e] = static_cast<int>(b);
    }
  }
  __syncthreads();
  if (warp == 0) {
    const int32_t* ids = topk_ids + static_cast<size_t>(t0) * K;
    for (int base = 0; base < nent; base += 32) {
      const int i = base + lane;
      const bool valid = i < nent;
      const unsigned vmask = __ballot_sync(0xffffffffu, valid);
      if (valid) {
        const int id = ids[i];
        const unsigned peers = __match_any_sync(vmask, id);
        const int rank_in = __popc(peers & ((1u << lane) - 1u));
        const int b = off[id];
        __syncwarp(vmask);
        if (lane == __ffs(peers) - 1) off[id] = b + __popc(peers);
        const int ps = b + rank_in;
        pos[i] = ps;
        const int d = dbase[id] + (ps - expert_start[id]);
        drow[i] = d;
        slot_pos[static_cast<size_t>(t0) * K + i] = ps;
        if (sorted_token) sorted_token[ps] = t0 + i / K;
        // origin word: source rank in bits 28..30, sorted position on the source below
        if (tg.world > 1) tg.origin[id / tg.el][d] = (tg.rank << 28) | ps;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  const int vec = H / 8;  // 16-byte chunks per row
  for (int tl = warp; tl < ntok; tl += kRouteThreads / 32) {
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t0 + tl) * H);
    for (int c0 = lane; c0 < vec; c0 += 32 * 4) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + 32 * u;
        if (c < vec) v[u] = src[c];
      }
      for (int j = 0; j < K; ++j) {
        const int e = tl * K + j;
        const int r = tg.world > 1 ? topk_ids[static_cast<size_t>(t0) * K + e] / tg.el : 0;
        uint4* dst = reinterpret_cast<uint4*>(tg.recv[r] + static_cast<size_t>(drow[e]) * H);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + 32 * u;
          if (c < vec) dst[c] = v[u];
        }
      }
    }
  }
  if (tg.world > 1) __threadfence_system();
}

template <typename T16>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const T16* h = reinterpret_cast<const T16*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = static_cast<float>(h[i]);
}

// One warp per token; fp32 accumulation in fixed slot order.
template <typename T16>
__global__ void __launch_bounds__(256)
    combine_kernel(const T16* __restrict__ ys, const float* __restrict__ w,
                   const int32_t* __restrict__ slot_pos, int T, int H, int K,
                   T16* __restrict__ out, const int* __restrict__ err) {
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const int vec = H / 8;
  if (err != nullptr && *reinterpret_cast<const volatile int*>(err) != 0) {
    // the data this token's rows came from is incomplete: hand back NaN, never stale numbers
    uint4 nan4;
    T16* nh = reinterpret_cast<T16*>(&nan4);
#pragma unroll
    for (int i = 0; i < 8; ++i) nh[i] = static_cast<T16>(__int_as_float(0x7fc00000));
    uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H);
    for (int c = lane; c < vec; c += 32) dst[c] = nan4;
    return;
  }
  int ps[kMaxTopK];
  float wt[kMaxTopK];
  for (int j = 0; j < K; ++j) {
    ps[j] = slot_pos[static_cast<size_t>(t) * K + j];
    wt[j] = w[static_cast<size_t>(t) * K + j];
  }
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H);
  for (int c = lane; c < vec; c += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < K; ++j) {
      const uint4 v = reinterpret_cast<const uint4*>(ys + static_cast<size_t>(ps[j]) * H)[c];
      float f[8];
      unpack8<T16>(v, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(wt[j], f[i], acc[i]);
    }
    uint4 o;
    T16* oh = reinterpret_cast<T16*>(&o);
#pragma unroll
    for (int i = 0; i < 8; ++i) oh[i] = static_cast<T16>(acc[i]);
    dst[c] = o;
  }
}

// Per-row e4m3 quantisation: scale[r] = max|x[r,:]| / 448 (1 for an all-zero row) and
// q[r,c] = e4m3(x[r,c] / scale[r]) rounded to nearest, saturating. One warp per row.
template <typename T16>
__global__ void __launch_bounds__(256)
    quantize_rows_fp8_kernel(const T16* __restrict__ x, int rows, int cols,
                             uint8_t* __restrict__ q, float* __restrict__ scale) {
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const T16* xr = x + static_cast<size_t>(r) * cols;
  const int vec = cols / 8;
  float amax = 0.f;
  for (int c = lane; c < vec; c += 32) {
    float f[8];
    unpack8<T16>(reinterpret_cast<const uint4*>(xr)[c], f);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = amax > 0.f ? amax / 448.f : 1.f;
  if (lane == 0) scale[r] = s;
  uint8_t* qr = q + static_cast<size_t>(r) * cols;
  for (int c = lane; c < vec; c += 32) {
    float f[8];
    unpack8<T16>(reinterpret_cast<const uint4*>(xr)[c], f);
    uint32_t w[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_fp8x2_storage_t lo =
          __nv_cvt_float2_to_fp8x2(make_float2(f[4 * h] / s, f[4 * h + 1] / s), __NV_SATFINITE,
                                   __NV_E4M3);
      const __nv_fp8x2_storage_t hi =
          __nv_cvt_float2_to_fp8x2(make_float2(f[4 * h + 2] / s, f[4 * h + 3] / s),
                                   __NV_SATFINITE, __NV_E4M3);
      w[h] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
    reinterpret_cast<uint2*>(qr)[c] = make_uint2(w[0], w[1]);
  }
}

// The same quantisation with one 256-thread block per row and the row held in registers
// (cols <= kFp8RowRegCols): one HBM read of the row instead of a read for the amax and a second
// for the conversion, and 8 independent 16-byte loads per thread in flight.
constexpr int kFp8RowVecPerThread = 8;
constexpr int kFp8RowRegCols = 256 * kFp8RowVecPerThread * 8;  // 16384

template <typename T16>
__global__ void __launch_bounds__(256)
    quantize_rows_fp8_reg_kernel(const T16* __restrict__ x, int cols, uint8_t* __restrict__ q,
                                 float* __restrict__ scale) {
  __shared__ float s_max[8];
  const int r = blockIdx.x;
  const int vec = cols / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(r) * cols);
  uint4 v[kFp8RowVecPerThread];
#pragma unroll
  for (int i = 0; i < kFp8RowVecPerThread; ++i) {
    const int c = threadIdx.x + i * 256;
    v[i] = c < vec ? xr[c] : make_uint4(0, 0, 0, 0);
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kFp8RowVecPerThread; ++i) {
    float f[8];
    unpack8<T16>(v[i], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = amax;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < 8; ++w) amax = fmaxf(amax, s_max[w]);
  const float s = amax > 0.f ? amax / 448.f : 1.f;
  if (threadIdx.x == 0) scale[r] = s;
  // x / s, correctly rounded, without a division per element (Markstein, IBM J. Res. Dev. 34(1),
  // 1990): with y = RN(1/s) and q0 = RN(x y), the fma residual r = x - s q0 is exact and
  // RN(q0 + r y) = RN(x / s) when no underflow occurs; |x / s| <= 448 here, and quotients small
  // enough to underflow round to zero in e4m3 either way.
  const float y = __frcp_rn(s);
  uint2* qr = reinterpret_cast<uint2*>(q + static_cast<size_t>(r) * cols);
#pragma unroll
  for (int i = 0; i < kFp8RowVecPerThread; ++i) {
    const int c = threadIdx.x + i * 256;
    if (c >= vec) break;
    float f[8];
    unpack8<T16>(v[i], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float q0 = f[e] * y;
      f[e] = fmaf(fmaf(-s, q0, f[e]), y, q0);
    }
    uint32_t w[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
          make_float2(f[4 * h], f[4 * h + 1]), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
          make_float2(f[4 * h + 2], f[4 * h + 3]), __NV_SATFINITE, __NV_E4M3);
      w[h] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    }
    qr[c] = make_uint2(w[0], w[1]);
  }
}

// ---------------------------------------------------------------- MX (block-scaled) quantisation
// OCP MX e4m3 with UE8M0 scales, one per 32 consecutive elements of a row. For each group of 32:
// amax = max |x|, E = floor(log2 amax), scale exponent X = E - 8, plus 1 when amax / 2^E > 1.75
// (so amax / 2^X <= 448, the largest e4m3 value: nothing clips), clamped to [-127, 127] (a zero
// group gets -127); q = e4m3 round-to-nearest-even of x * 2^-X (exact power-of-two scaling).
// Scales go to the 128x4 blocked layout the block-scaled tensor-core MMA reads: segment s's rows
// start a fresh 128-row block after the blocks of segments < s; block b and K group g (128
// elements, 4 scales) form the 512-B atom b * K/128 + g, in which row r (0..127) and scale j
// (0..3) sit at byte (r % 32) * 16 + (r / 32) * 4 + j. Bytes of padding rows are not written.
constexpr int kMxMaxSegments = 1024;

// One warp per row (grid-stride over rows). Lane l converts 8 consecutive elements per step, so a
// 32-element group is four lanes and one warp step covers 256 elements with fully coalesced 16-B
// loads and 8-B stores; the group amax is two shuffles. The row's segment, scale block and row in
// block are found once per row.
template <typename T16>
__global__ void __launch_bounds__(256)
    quantize_mxfp8_kernel(const T16* __restrict__ x, const int64_t* __restrict__ counts, int nseg,
                          int rows, int k, uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  __shared__ int s_rowoff[kMxMaxSegments + 1];
  __shared__ int s_blkoff[kMxMaxSegments];
  if (threadIdx.x < 32) {  // exclusive prefix sums of rows and 128-row blocks, segment order
    const int lane = threadIdx.x;
    int carry = 0, bcarry = 0;
    for (int base = 0; base < nseg; base += 32) {
      const int s = base + lane;
      long long c = s < nseg ? counts[s] : 0;
      c = c < 0 ? 0 : (c > rows ? rows : c);
      const int v = static_cast<int>(c), b = (v + 127) / 128;
      int xs = v, ys = b;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int xu = __shfl_up_sync(0xffffffffu, xs, o);
        const int yu = __shfl_up_sync(0xffffffffu, ys, o);
        if (lane >= o) {
          xs += xu;
          ys += yu;
        }
      }
      if (s < nseg) {
        s_rowoff[s] = carry + xs - v;
        s_blkoff[s] = bcarry + ys - b;
      }
      carry += __shfl_sync(0xffffffffu, xs, 31);
      bcarry += __shfl_sync(0xffffffffu, ys, 31);
    }
    if (lane == 0) s_rowoff[nseg] = carry;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int kg = k / 128;
  const int covered = s_rowoff[nseg];
  const int nwarps = gridDim.x * 8;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += nwarps) {
    // scale-block coordinates of row r (rows past the counted ones get no scale bytes)
    size_t sf_row = 0;
    const bool has_sf = r < covered;
    if (has_sf) {
      int lo = 0, hi = nseg - 1;  // the last segment starting at or before r is r's segment
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_rowoff[mid] <= r) lo = mid; else hi = mid - 1;
      }
      const int rl = r - s_rowoff[lo];
      const int rr = rl & 127;
      sf_row = static_cast<size_t>(s_blkoff[lo] + rl / 128) * kg * 512 + (rr & 31) * 16 +
               (rr >> 5) * 4;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(r) * k);
    uint2* dst = reinterpret_cast<uint2*>(q + static_cast<size_t>(r) * k);
    const int vec = k / 8;
    // every lane runs every step (the shuffles need the whole warp); vec is a multiple of 16, so
    // a step's inactive lanes are whole groups
#pragma unroll 2
    for (int c0 = 0; c0 < vec; c0 += 32) {
      const int c = c0 + lane;  // 8-element chunk; group j = c / 4
      const bool active = c < vec;
      float f[8];
      unpack8<T16>(active ? src[c] : make_uint4(0, 0, 0, 0), f);
      float amax = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const uint32_t bits = __float_as_uint(amax);
      const int eb = static_cast<int>((bits >> 23) & 0xFFu);
      int xe = eb == 0 ? -127 : eb - 127 - 8 + ((bits & 0x7FFFFFu) > 0x600000u ? 1 : 0);
      xe = xe < -127 ? -127 : (xe > 127 ? 127 : xe);
      const float inv = xe <= 126 ? __uint_as_float(static_cast<uint32_t>(127 - xe) << 23)
                                  : __uint_as_float(1u << 22);  // 2^-127
      uint32_t w[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(
            make_float2(f[4 * h] * inv, f[4 * h + 1] * inv), __NV_SATFINITE, __NV_E4M3);
        const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
            make_float2(f[4 * h + 2] * inv, f[4 * h + 3] * inv), __NV_SATFINITE, __NV_E4M3);
        w[h] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
      }
      if (!active) continue;
      dst[c] = make_uint2(w[0], w[1]);
      const int j = c >> 2;
      if (has_sf && (c & 3) == 0)
        sf[sf_row + static_cast<size_t>(j >> 2) * 512 + (j & 3)] = static_cast<uint8_t>(xe + 127);
    }
  }
}

// ---------------------------------------------------------------- expert-parallel signalling
// Each rank owns an IPC-shared sync board: counts [kMaxPeers][E] int64 (every rank's
// tokens_per_expert, written by that rank) and flags [kEpSlots][kMaxPeers] int64 (per phase, the
// last layer epoch each rank has completed). A rank posts by storing into every peer's board;
// a rank waits by polling its own board. Epochs only grow, so no reset is needed.
constexpr int kEpSlots = 4;

struct PeerBoards {
  int64_t* board[kMaxPeers];
};

// Stores this rank's tokens_per_expert into row `rank` of every peer's counts board, then (after a
// system-scope fence) its epoch into every peer's flags[slot][rank]. One block.
__global__ void ep_publish_counts_kernel(const int64_t* __restrict__ tpe, PeerBoards pb, int world,
                                         int rank, int E, int slot, long long epoch) {
  for (int r = 0; r < world; ++r)
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      pb.board[r][static_cast<size_t>(rank) * E + e] = tpe[e];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world) {
    volatile long long* f = reinterpret_cast<volatile long long*>(
        pb.board[threadIdx.x] + static_cast<size_t>(kMaxPeers) * E + slot * kMaxPeers + rank);
    *f = epoch;
  }
}

// After the previous kernels on this stream (which fenced their peer stores), tells every peer
// that this rank finished phase `slot` of layer `epoch`.
__global__ void ep_signal_kernel(PeerBoards pb, int world, int rank, int E, int slot,
                                 long long epoch) {
  __threadfence_system();
  if (threadIdx.x < world) {
    volatile long long* f = reinterpret_cast<volatile long long*>(
        pb.board[threadIdx.x] + static_cast<size_t>(kMaxPeers) * E + slot * kMaxPeers + rank);
    *f = epoch;
  }
}

// Waits until every rank has posted `epoch` for `slot` in this rank's own board. Bounded: after
// `limit` cycles it records kErrEpTimeout in *err and returns (the data of the phase is then
// incomplete and the host reports the error).
__global__ void ep_wait_kernel(const int64_t* __restrict__ own_board, int world, int E, int slot,
                               long long epoch, int* err, long long limit) {
  // an earlier phase already failed: this layer's data is void, do not wait out another limit
  const bool failed = *reinterpret_cast<const volatile int*>(err) != 0;
  if (threadIdx.x < world && !failed) {
    const volatile long long* f = reinterpret_cast<const volatile long long*>(
        own_board + static_cast<size_t>(kMaxPeers) * E + slot * kMaxPeers + threadIdx.x);
    const long long t0 = clock64();
    while (*f < epoch) {
      if (clock64() - t0 > limit) {
        atomicCAS(err, 0, 104);  // device error code: expert-parallel peer wait timed out
        break;
      }
    }
  }
  __threadfence_system();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int nblocks_for(int64_t T) { return static_cast<int>((T + kRouteTokens - 1) / kRouteTokens); }

template <typename T16>
void launch_dispatch(const void* x, int T, int H, int E, int K, const int32_t* ids,
                     const int* bo, const int* es, const int64_t* counts_all, int world, int rank,
                     void* const* recv, int32_t* const* origin, int32_t* stok, int32_t* spos,
                     cudaStream_t stream) {
  DispatchTargets<T16> tg;
  tg.world = world;
  tg.rank = rank;
  tg.el = E / world;
  tg.counts_all = counts_all;
  for (int r = 0; r < kMaxPeers; ++r) {
    tg.recv[r] = r < world ? static_cast<T16*>(recv[r]) : nullptr;
    tg.origin[r] = r < world ? origin[r] : nullptr;
  }
  const int nb = nblocks_for(T);
  const size_t smem = (2 * static_cast<size_t>(E) + 2 * kRouteTokens * K) * 4;
  dispatch_kernel<T16><<<nb, kRouteThreads, smem, stream>>>(
      static_cast<const T16*>(x), T, H, E, K, ids, bo, es, tg, stok, spos);
}

int dispatch_common(const void* x, int64_t num_tokens, int64_t hidden, int E, int K,
                    const int32_t* ids, const void* scratch, const int64_t* counts_all, int world,
                    int rank, void* const* recv, int32_t* const* origin, int32_t* stok,
                    int32_t* spos, int dtype, cudaStream_t stream) {
  if (!x || !ids || !spos || !scratch) return GGO_ERR_INVALID_ARG;
  if (num_tokens < 0 || hidden <= 0 || E <= 0 || E > kMaxExperts || K <= 0 || K > kMaxTopK)
    return GGO_ERR_INVALID_ARG;
  if (dtype != GGO_DTYPE_BF16 && dtype != GGO_DTYPE_FP16) return GGO_ERR_DTYPE;
  if (hidden % 8 || !aligned16(x)) return GGO_ERR_ALIGNMENT;
  for (int r = 0; r < world; ++r)
    if (!aligned16(recv[r])) return GGO_ERR_ALIGNMENT;
  if (num_tokens * K > INT32_MAX || hidden > INT32_MAX) return GGO_ERR_SHAPE;
  const int T = static_cast<int>(num_tokens);
  const int nb = nblocks_for(T);
  if (nb == 0) return GGO_OK;
  const int* bo = static_cast<const int*>(scratch);
  const int* es = bo + static_cast<size_t>(nb) * E;
  if (dtype == GGO_DTYPE_BF16)
    launch_dispatch<__nv_bfloat16>(x, T, static_cast<int>(hidden), E, K, ids, bo, es, counts_all,
                                   world, rank, recv, origin, stok, spos, stream);
  else
    launch_dispatch<__half>(x, T, static_cast<int>(hidden), E, K, ids, bo, es, counts_all, world,
                            rank, recv, origin, stok, spos, stream);
  return ggo::check_launch();
}

}  // namespace
}  // namespace ggo

extern "C" {

size_t ggo_moe_route_scratch_bytes(int64_t num_tokens, int num_experts) {
  if (num_tokens <= 0 || num_experts <= 0) return 16;
  return (static_cast<size_t>(ggo::nblocks_for(num_tokens)) + 1) * num_experts * sizeof(int);
}

int ggo_moe_route(const float* logits_dev, int64_t num_tokens, int num_experts, int top_k,
                  int32_t* topk_ids_dev, float* topk_weights_dev,
                  int64_t* tokens_per_expert_dev, void* scratch_dev, cudaStream_t stream) {
  if (!logits_dev || !topk_ids_dev || !topk_weights_dev || !tokens_per_expert_dev || !scratch_dev)
    return GGO_ERR_INVALID_ARG;
  if (num_tokens < 0 || num_experts <= 0 || num_experts > ggo::kMaxExperts || top_k <= 0 ||
      top_k > ggo::kMaxTopK || top_k > num_experts)
    return GGO_ERR_INVALID_ARG;
  if (num_tokens * top_k > INT32_MAX) return GGO_ERR_SHAPE;
  const int T = static_cast<int>(num_tokens);
  const int nb = ggo::nblocks_for(T);
  int* bc = static_cast<int*>(scratch_dev);
  if (nb > 0) {
    const size_t smem = static_cast<size_t>(num_experts) * (1 + ggo::kRouteThreads / 32) * 4;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(ggo::route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return GGO_ERR_CUDA;
    ggo::route_kernel<<<nb, ggo::kRouteThreads, smem, stream>>>(
        logits_dev, T, num_experts, top_k, topk_ids_dev, topk_weights_dev, bc);
  }
  ggo::route_scan_kernel<<<1, 1024, 0, stream>>>(bc, nb, num_experts, tokens_per_expert_dev);
  return ggo::check_launch();
}

int ggo_moe_permute(const void* x_dev, int64_t num_tokens, int64_t hidden, int num_experts,
                    int top_k, const int32_t* topk_ids_dev, void* x_sorted_dev,
                    int32_t* sorted_token_dev, int32_t* slot_pos_dev, void* scratch_dev,
                    int dtype, cudaStream_t stream) {
  if (!x_sorted_dev || !sorted_token_dev) return GGO_ERR_INVALID_ARG;
  void* recv[1] = {x_sorted_dev};
  int32_t* origin[1] = {nullptr};
  return ggo::dispatch_common(x_dev, num_tokens, hidden, num_experts, top_k, topk_ids_dev,
                              scratch_dev, nullptr, 1, 0, recv, origin, sorted_token_dev,
                              slot_pos_dev, dtype, stream);
}

int ggo_ep_dispatch(const void* x_dev, int64_t num_tokens, int64_t hidden, int num_experts,
                    int top_k, const int32_t* topk_ids_dev, const void* scratch_dev,
                    const int64_t* counts_all_dev, int world_size, int rank,
                    void* const* recv_rows, int32_t* const* recv_origin, int32_t* slot_pos_dev,
                    int dtype, cudaStream_t stream) {
  if (world_size < 1 || world_size > ggo::kMaxPeers || rank < 0 || rank >= world_size ||
      !counts_all_dev || !recv_rows || !recv_origin || num_experts % world_size)
    return GGO_ERR_INVALID_ARG;
  for (int r = 0; r < world_size; ++r)
    if (!recv_rows[r] || !recv_origin[r]) return GGO_ERR_INVALID_ARG;
  return ggo::dispatch_common(x_dev, num_tokens, hidden, num_experts, top_k, topk_ids_dev,
                              scratch_dev, counts_all_dev, world_size, rank, recv_rows,
                              recv_origin, nullptr, slot_pos_dev, dtype, stream);
}

int ggo_quantize_fp8_rows(const void* x_dev, int64_t rows, int64_t cols, int dtype, void* q_dev,
                          float* scale_dev, cudaStream_t stream) {
  if (!x_dev || !q_dev || !scale_dev || rows < 0 || cols <= 0) return GGO_ERR_INVALID_ARG;
  if (dtype != GGO_DTYPE_BF16 && dtype != GGO_DTYPE_FP16) return GGO_ERR_DTYPE;
  if (cols % 16 || !ggo::aligned16(x_dev) || !ggo::aligned16(q_dev)) return GGO_ERR_ALIGNMENT;
  if (rows > INT32_MAX || cols > INT32_MAX) return GGO_ERR_SHAPE;
  if (rows == 0) return GGO_OK;
  if (cols <= ggo::kFp8RowRegCols) {  // the row fits in the block's registers
    const int grid = static_cast<int>(rows);
    if (dtype == GGO_DTYPE_BF16)
      ggo::quantize_rows_fp8_reg_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(x_dev), static_cast<int>(cols),
          static_cast<uint8_t*>(q_dev), scale_dev);
    else
      ggo::quantize_rows_fp8_reg_kernel<__half><<<grid, 256, 0, stream>>>(
          static_cast<const __half*>(x_dev), static_cast<int>(cols), static_cast<uint8_t*>(q_dev),
          scale_dev);
    return ggo::check_launch();
  }
  const int grid = static_cast<int>((rows + 7) / 8);
  if (dtype == GGO_DTYPE_BF16)
    ggo::quantize_rows_fp8_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x_dev), static_cast<int>(rows), static_cast<int>(cols),
        static_cast<uint8_t*>(q_dev), scale_dev);
  else
    ggo::quantize_rows_fp8_kernel<__half><<<grid, 256, 0, stream>>>(
        static_cast<const __half*>(x_dev), static_cast<int>(rows), static_cast<int>(cols),
        static_cast<uint8_t*>(q_dev), scale_dev);
  return ggo::check_launch();
}

int ggo_quantize_mxfp8(const void* x_dev, int dtype, const int64_t* counts_dev, int num_segments,
                       int64_t rows, int64_t k, void* q_dev, void* scale_dev,
                       cudaStream_t stream) {
  if (!x_dev || !counts_dev || !q_dev || !scale_dev || rows < 0 || k <= 0)
    return GGO_ERR_INVALID_ARG;
  if (num_segments <= 0) return GGO_ERR_INVALID_ARG;
  if (num_segments > ggo::kMxMaxSegments) return GGO_ERR_TOO_MANY_SEGMENTS;
  if (dtype != GGO_DTYPE_BF16 && dtype != GGO_DTYPE_FP16) return GGO_ERR_DTYPE;
  if (k % 128 || !ggo::aligned16(x_dev) || !ggo::aligned16(q_dev)) return GGO_ERR_ALIGNMENT;
  if (rows > INT32_MAX || k > INT32_MAX) return GGO_ERR_SHAPE;
  if (rows == 0) return GGO_OK;
  const long long want = (rows + 7) / 8;  // one warp per row, grid-stride beyond 4096 blocks
  const int grid = static_cast<int>(want < 4096 ? want : 4096);
  if (dtype == GGO_DTYPE_BF16)
    ggo::quantize_mxfp8_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x_dev), counts_dev, num_segments,
        static_cast<int>(rows), static_cast<int>(k), static_cast<uint8_t*>(q_dev),
        static_cast<uint8_t*>(scale_dev));
  else
    ggo::quantize_mxfp8_kernel<__half><<<grid, 256, 0, stream>>>(
        static_cast<const __half*>(x_dev), counts_dev, num_segments, static_cast<int>(rows),
        static_cast<int>(k), static_cast<uint8_t*>(q_dev), static_cast<uint8_t*>(scale_dev));
  return ggo::check_launch();
}

size_t ggo_ep_board_bytes(int num_experts) {
  return (static_cast<size_t>(ggo::kMaxPeers) * num_experts +
          static_cast<size_t>(ggo::kEpSlots) * ggo::kMaxPeers) * sizeof(int64_t);
}

static int ep_boards(int64_t* const* boards, int world, ggo::PeerBoards* pb) {
  if (!boards || world < 1 || world > ggo::kMaxPeers) return GGO_ERR_INVALID_ARG;
  for (int r = 0; r < ggo::kMaxPeers; ++r) pb->board[r] = r < world ? boards[r] : nullptr;
  for (int r = 0; r < world; ++r)
    if (!boards[r]) return GGO_ERR_INVALID_ARG;
  return GGO_OK;
}

int ggo_ep_publish_counts(const int64_t* tokens_per_expert_dev, int64_t* const* boards,
                          int world_size, int rank, int num_experts, int slot, int64_t epoch,
                          cudaStream_t stream) {
  ggo::PeerBoards pb;
  if (int st = ep_boards(boards, world_size, &pb)) return st;
  if (!tokens_per_expert_dev || rank < 0 || rank >= world_size || num_experts <= 0 || slot < 0 ||
      slot >= ggo::kEpSlots)
    return GGO_ERR_INVALID_ARG;
  ggo::ep_publish_counts_kernel<<<1, 256, 0, stream>>>(tokens_per_expert_dev, pb, world_size,
                                                        rank, num_experts, slot, epoch);
  return ggo::check_launch();
}

int ggo_ep_signal(int64_t* const* boards, int world_size, int rank, int num_experts, int slot,
                  int64_t epoch, cudaStream_t stream) {
  ggo::PeerBoards pb;
  if (int st = ep_boards(boards, world_size, &pb)) return st;
  if (rank < 0 || rank >= world_size || num_experts <= 0 || slot < 0 || slot >= ggo::kEpSlots)
    return GGO_ERR_INVALID_ARG;
  ggo::ep_signal_kernel<<<1, 32, 0, stream>>>(pb, world_size, rank, num_experts, slot, epoch);
  return ggo::check_launch();
}

int ggo_ep_wait(const int64_t* own_board, int world_size, int num_experts, int slot,
                int64_t epoch, void* workspace_dev, int64_t limit_cycles, cudaStream_t stream) {
  if (!own_board || !workspace_dev || world_size < 1 || world_size > ggo::kMaxPeers ||
      num_experts <= 0 || slot < 0 || slot >= ggo::kEpSlots || limit_cycles <= 0)
    return GGO_ERR_INVALID_ARG;
  int* err = static_cast<int*>(workspace_dev) + 2;  // GgoWorkspace::error
  ggo::ep_wait_kernel<<<1, 32, 0, stream>>>(own_board, world_size, num_experts, slot, epoch, err,
                                            limit_cycles);
  return ggo::check_launch();
}

int ggo_moe_combine(const void* y_sorted_dev, const float* topk_weights_dev,
                    const int32_t* slot_pos_dev, int64_t num_tokens, int64_t hidden, int top_k,
                    void* out_dev, int dtype, cudaStream_t stream) {
  return ggo_moe_combine_checked(y_sorted_dev, topk_weights_dev, slot_pos_dev, num_tokens, hidden,
                                 top_k, out_dev, dtype, nullptr, stream);
}

int ggo_moe_combine_checked(const void* y_sorted_dev, const float* topk_weights_dev,
                            const int32_t* slot_pos_dev, int64_t num_tokens, int64_t hidden,
                            int top_k, void* out_dev, int dtype, const void* workspace_dev,
                            cudaStream_t stream) {
  // GgoWorkspace::error is the third int of the workspace
  const int* err = workspace_dev ? static_cast<const int*>(workspace_dev) + 2 : nullptr;
  if (!y_sorted_dev || !topk_weights_dev || !slot_pos_dev || !out_dev) return GGO_ERR_INVALID_ARG;
  if (num_tokens < 0 || hidden <= 0 || top_k <= 0 || top_k > ggo::kMaxTopK)
    return GGO_ERR_INVALID_ARG;
  if (dtype != GGO_DTYPE_BF16 && dtype != GGO_DTYPE_FP16) return GGO_ERR_DTYPE;
  if (hidden % 8 || !ggo::aligned16(y_sorted_dev) || !ggo::aligned16(out_dev))
    return GGO_ERR_ALIGNMENT;
  if (num_tokens * top_k > INT32_MAX || hidden > INT32_MAX) return GGO_ERR_SHAPE;
  const int T = static_cast<int>(num_tokens);
  if (T == 0) return GGO_OK;
  const int grid = (T + 7) / 8;
  if (dtype == GGO_DTYPE_BF16) {
    ggo::combine_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(y_sorted_dev), topk_weights_dev, slot_pos_dev, T,
        static_cast<int>(hidden), top_k, static_cast<__nv_bfloat16*>(out_dev), err);
  } else {
    ggo::combine_kernel<__half><<<grid, 256, 0, stream>>>(
        static_cast<const __half*>(y_sorted_dev), topk_weights_dev, slot_pos_dev, T,
        static_cast<int>(hidden), top_k, static_cast<__half*>(out_dev), err);
  }
  return ggo::check_launch();
}

}  // extern "C"
