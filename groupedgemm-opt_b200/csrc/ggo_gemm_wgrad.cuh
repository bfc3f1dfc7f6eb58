// Backward weight gradient of the grouped GEMM, persistent tcgen05 kernel for sm_100a:
//
//   dW[e] (N x K) = dY_e^T (N x M_e) @ X_e (M_e x K)     for every expert e,
//
// where X_e / dY_e are expert e's M_e consecutive rows of x [T, K] / dy [T, N]. The reduction runs
// over each expert's own (ragged) token range. No reference counterpart (the reference is
// forward-only).
//
// Both operands are MN-major in memory and are TMA-loaded in place as 64 x 64 boxes (64 tokens x
// 64 output rows or columns, 128-B swizzle). The last 64-token block of an expert may contain
// the next expert's tokens: the MMA warp zeroes those token rows in shared memory (whole 128-B
// rows, so the swizzle is irrelevant) before the final MMAs. Experts with no tokens get zero
// gradients. Tiles are 128 (rows of dW) x BN (columns), claimed from an atomic counter,
// heaviest expert first (tile cost is proportional to M_e).
#pragma once

#include "ggo_gemm.cuh"

namespace ggo {

struct WgradParams {
  const int64_t* counts;  // [E] tokens per expert (device)
  int num_experts;
  int rows;               // T
  int n;                  // N: rows of each dW[e]
  int k;                  // K: columns of dW[e]
  int sort_by_m;
  void* out;              // dW [E, N, K]
  GgoWorkspace* ws;
  long long wait_limit;
};

template <int BN>
struct WgradLayout {
  static constexpr int kABytes = 128 * kBK * 2;  // two 64x64 boxes: 128 dW rows x 64 tokens
  static constexpr int kBBytes = BN * kBK * 2;   // BN/64 boxes: BN dW columns x 64 tokens
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (BN == 256) ? 4 : 6;
  static constexpr int kTileBytes = kStages * kStageBytes;
  static constexpr int kStagingBytes = 4 * 4096;
  static constexpr int kTableBytes = 4 * kMaxSegments * 4 + 16;
  static constexpr int kMiscBytes = 1024;
  static constexpr int kTotal =
      1024 + kTileBytes + kStagingBytes + kTableBytes + kMiscBytes;
  static_assert(kTotal <= 227 * 1024, "shared memory budget");
};

struct WgradTile {
  int m0;      // first dW row (within the expert)
  int rows;    // valid dW rows (<= 128); 0 = no more work
  int n0;      // first dW column
  int expert;
  int tok0;    // first token row of the expert
  int ntok;    // tokens of the expert
  int pad[2];
};

template <int BN, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_wgrad_kernel(const __grid_constant__ CUtensorMap tmDY,
                              const __grid_constant__ CUtensorMap tmX,
                              const __grid_constant__ CUtensorMap tmW, const WgradParams p) {
  using L = WgradLayout<BN>;
  constexpr int S = L::kStages;
  constexpr int kTmemCols = 2 * BN;
  using OutT = typename std::conditional<BF16, __nv_bfloat16, __half>::type;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* tiles = smem;
  uint8_t* staging = smem + L::kTileBytes;
  int* t_cnt = reinterpret_cast<int*>(smem + L::kTileBytes + L::kStagingBytes);
  int* t_rowoff = t_cnt + kMaxSegments;
  int* t_order = t_rowoff + kMaxSegments;
  uint8_t* misc = smem + L::kTileBytes + L::kStagingBytes + L::kTableBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(misc);
  uint64_t* empty_bar = full_bar + S;
  uint64_t* accf_bar = empty_bar + S;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* schf_bar = acce_bar + 2;
  uint64_t* sche_bar = schf_bar + kSchedDepth;
  WgradTile* ring = reinterpret_cast<WgradTile*>(sche_bar + kSchedDepth);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring + kSchedDepth);
  WaitGuard* guard = reinterpret_cast<WaitGuard*>(tmem_slot + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = &p.ws->error;
  const int E = p.num_experts;

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
    tma_prefetch_desc(&tmDY);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  // expert table: clamped counts, token offsets, heaviest-first order
  for (int e = threadIdx.x; e < E; e += kThreads) {
    long long c = p.counts[e];
    if (c < 0) {
      atomicCAS(err, 0, kDevNegativeCount);
      c = 0;
    }
    t_cnt[e] = c > p.rows ? p.rows : static_cast<int>(c);
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < E; base += 32) {
      const int s = base + lane;
      const int v = s < E ? t_cnt[s] : 0;
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (s < E) t_rowoff[s] = carry + x - v;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0 && carry != p.rows && blockIdx.x == 0) atomicCAS(err, 0, kDevCountMismatch);
  }
  if (p.sort_by_m && E > 1) {  // rank of expert e in descending-count order (ties by index)
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += kThreads) {
      int r = 0;
      const int ce = t_cnt[e];
      for (int j = 0; j < E; ++j) r += (t_cnt[j] > ce) || (t_cnt[j] == ce && j < e);
      t_order[r] = e;
    }
  } else {
    for (int e = threadIdx.x; e < E; e += kThreads) t_order[e] = e;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int mt = (p.n + 127) / 128;
  const int nt = (p.k + BN - 1) / BN;
  const int per_expert = mt * nt;
  const int total_tiles = per_expert * E;

  if (warp == 0) {
    // -------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0, phase = 0, q = 0, qphase = 0;
      uint32_t armed = 0, armed_par = 0;
      while (true) {
        const int t = atomicAdd(&p.ws->tile_counter, 1);
        WgradTile info;
        info.rows = 0;
        if (t < total_tiles) {
          const int e = t_order[t / per_expert];
          const int local = t % per_expert;
          const int m_idx = local % mt, n_idx = local / mt;
          info.m0 = m_idx * 128;
          info.rows = min(128, p.n - info.m0);
          info.n0 = n_idx * BN;
          info.expert = e;
          info.tok0 = t_rowoff[e];
          info.ntok = t_cnt[e];
        }
        if (!mbar_wait(&sche_bar[q], qphase ^ 1, guard, err, kDevTimeoutProducer)) break;
        ring[q] = info;
        mbar_arrive(&schf_bar[q]);
        if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
        if (info.rows == 0) break;
        const int nkb = (info.ntok + kBK - 1) / kBK;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, guard, err, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = tiles + stage * L::kStageBytes;
          uint8_t* b_dst = a_dst + L::kABytes;
          const int y = info.tok0 + kb * kBK;
          mbar_arrive_expect_tx(&full_bar[stage], L::kStageBytes);
#pragma unroll
          for (int i = 0; i < 2; ++i)  // dY columns m0.. (dW rows) x 64 tokens
            tma_load_2d(a_dst + i * 8192, &tmDY, &full_bar[stage], info.m0 + 64 * i, y);
#pragma unroll
          for (int i = 0; i < BN / 64; ++i)  // X columns n0.. (dW columns) x 64 tokens
            tma_load_2d(b_dst + i * 8192, &tmX, &full_bar[stage], info.n0 + 64 * i, y);
          armed |= 1u << stage;
          armed_par = (armed_par & ~(1u << stage)) | (static_cast<uint32_t>(phase) << stage);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      if (guard->abort) drain_armed_stages<S>(full_bar, armed, armed_par, guard->limit);
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA warp (lane 0 issues)
    constexpr uint32_t idesc = idesc_f16(128, BN, BF16, true) | (1u << 15);  // A and B MN-major
    int stage = 0, phase = 0, q = 0, qphase = 0, acc = 0, aphase = 0;
    const uint32_t tiles_addr = smem_u32(tiles);
    while (true) {
      if (!mbar_wait(&schf_bar[q], qphase, guard, err, kDevTimeoutMma)) break;
      const WgradTile info = ring[q];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sche_bar[q]);
      if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
      if (info.rows == 0) break;
      if (!mbar_wait(&acce_bar[acc], aphase ^ 1, guard, err, kDevTimeoutMma)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      const int nkb = (info.ntok + kBK - 1) / kBK;
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, guard, err, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        const int valid = min(kBK, info.ntok - kb * kBK);  // tokens of this expert in the block
        const uint32_t a_addr = tiles_addr + stage * L::kStageBytes;
        if (valid < kBK) {
          // zero token rows [valid, 64) of every box (2 A boxes + BN/64 B boxes, 128 B a row)
          constexpr int kBoxes = 2 + BN / 64;
          const int zrows = kBK - valid;
          for (int i = lane; i < kBoxes * zrows * 8; i += 32) {
            const int box = i / (zrows * 8), rem = i % (zrows * 8);
            const uint32_t addr = a_addr + box * 8192 + (valid + rem / 8) * 128 + (rem % 8) * 16;
            st_shared_v4(addr, 0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t adesc = sdesc_sw128_mnmajor(a_addr, 8192);
          const uint64_t bdesc = sdesc_sw128_mnmajor(a_addr + L::kABytes, 8192);
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk)
            mma_f16_ss(d_tmem, adesc + 128 * kk, bdesc + 128 * kk, idesc, (kb | kk) != 0);
          mma_commit(&empty_bar[stage]);
        }
        __syncwarp();
        if (++stage == S) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (lane == 0) {
        if (nkb > 0) mma_commit(&accf_bar[acc]);
        else mbar_arrive(&accf_bar[acc]);  // no tokens: the epilogue writes zeros
      }
      __syncwarp();
      if (++acc == 2) { acc = 0; aphase ^= 1; }
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- epilogue
    const int ew = warp - 4;
    int q = 0, qphase = 0, acc = 0, aphase = 0;
    while (true) {
      if (!mbar_wait(&schf_bar[q], qphase, guard, err, kDevTimeoutEpilogue)) break;
      const WgradTile info = ring[q];
      __syncwarp();
      if (lane == 0) mbar_arrive(&sche_bar[q]);
      if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
      if (info.rows == 0) break;
      if (!mbar_wait(&accf_bar[acc], aphase, guard, err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int r_local = ew * 32 + lane;
      const bool row_ok = r_local < info.rows;
      const int grow = info.expert * p.n + info.m0;  // row of dW viewed as [E*N, K]
      OutT* out_row = reinterpret_cast<OutT*>(p.out) + static_cast<size_t>(grow + r_local) * p.k;
      const bool warp_tma = ew * 32 + 32 <= info.rows;
      if (info.ntok > 0) {
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + acc * BN;
        store_tile_rows<BN, kEpiStore, BF16>(t_row, info.n0, p.k, row_ok, out_row, warp_tma,
                                             &tmW, staging + ew * 4096, grow + ew * 32);
      } else if (row_ok) {  // expert without tokens: zero gradient
        for (int c = 0; c < BN; c += 8)
          if (info.n0 + c < p.k)
            *reinterpret_cast<uint4*>(out_row + info.n0 + c) = make_uint4(0u, 0u, 0u, 0u);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce_bar[acc]);
      if (++acc == 2) { acc = 0; aphase ^= 1; }
    }
  }

  if (warp >= 4 && lane == 0) bulk_wait_all();
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
