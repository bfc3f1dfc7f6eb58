// CTA-pair (cta_group::2) form of the weight-gradient kernel of ggo_gemm_wgrad.cuh:
//
//   dW[e] (N x K) = dY_e^T (N x M_e) @ X_e (M_e x K),  256 x 256 tiles of dW per CTA pair.
//
// Each CTA of the pair loads, per 64-token K step, its 128 rows of the tile's dY^T panel and its
// 128 columns of the X panel (two 64 x 64 MN-major boxes each, 32 KB) into its own shared memory;
// one thread of the even CTA issues tcgen05.mma.cta_group::2 (M = 256, N = 256), which reads A
// rows and the B half from each CTA and accumulates each CTA's 128 dW rows into that CTA's TMEM.
// Per SM this moves 32 KB of operands per K step instead of the single-CTA tile's 48 KB for the
// same MMA work: the L2 -> SM traffic that bounds the single-CTA main loop drops by a third.
//
// Full 64-token blocks are loaded as the forward pair kernel loads its operands: both CTAs' bytes
// complete on the leader's `full_bar`. The last block of an expert may hold the next expert's
// tokens, and both CTAs hold token rows of both operands, so both must zero them before the pair
// MMA reads the block: for such a partial block each CTA counts its own loads on its own
// `full_bar`, warp 1 of each CTA waits on it, zeroes the foreign token rows of its boxes, fences
// the async proxy and arrives on the leader's `ready_bar`, and the leader's MMA thread waits for
// both arrivals. Only the partial blocks pay for that handshake.
// Every bulk-tensor load writes only the issuing CTA's shared memory, from this GPU's memory.
#pragma once

#include "ggo_gemm_wgrad.cuh"

namespace ggo {

struct WgradPairLayout {
  static constexpr int kABytes = 128 * kBK * 2;  // this CTA's 128 dW rows x 64 tokens (2 boxes)
  static constexpr int kBBytes = 128 * kBK * 2;  // this CTA's 128 dW columns x 64 tokens
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = 6;
  static constexpr int kTileBytes = kStages * kStageBytes;
  static constexpr int kStagingBytes = 4 * 4096;
  static constexpr int kTableBytes = 3 * kMaxSegments * 4 + 16;
  static constexpr int kMiscBytes = 1024;
  static constexpr int kTotal = 1024 + kTileBytes + kStagingBytes + kTableBytes + kMiscBytes;
  static_assert(kTotal <= 227 * 1024, "shared memory budget");
};

template <bool BF16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    grouped_gemm_wgrad_pair_kernel(const __grid_constant__ CUtensorMap tmDY,
                                   const __grid_constant__ CUtensorMap tmX,
                                   const __grid_constant__ CUtensorMap tmW, const WgradParams p) {
  using L = WgradPairLayout;
  constexpr int S = L::kStages;
  constexpr int BN = 256;                // dW columns per pair tile (128 per CTA's B half)
  constexpr int kAccStride = 256;
  constexpr int kTmemCols = 512;
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
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(misc);  // own loads landed (each CTA)
  uint64_t* ready_bar = full_bar + S;                        // leader: both CTAs' stage ready
  uint64_t* empty_bar = ready_bar + S;                       // both: the pair MMA retired
  uint64_t* accf_bar = empty_bar + S;
  uint64_t* acce_bar = accf_bar + 2;
  uint64_t* schf_bar = acce_bar + 2;
  uint64_t* sche_bar = schf_bar + kSchedDepth;
  WgradTile* ring = reinterpret_cast<WgradTile*>(sche_bar + kSchedDepth);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring + kSchedDepth);
  WaitGuard* guard = reinterpret_cast<WaitGuard*>(tmem_slot + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  int* err = &p.ws->error;
  const int E = p.num_experts;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);    // this CTA's expect_tx arrive + its bytes
      mbar_init(&ready_bar[i], 2);   // leader: warp 1 of each CTA
      mbar_init(&empty_bar[i], 1);   // both: one two-CTA commit per use
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf_bar[i], 1);    // both: one two-CTA commit (or arrive) per tile
      mbar_init(&acce_bar[i], 8);    // leader: 4 epilogue warps x 2 CTAs
    }
    for (int i = 0; i < kSchedDepth; ++i) {
      mbar_init(&schf_bar[i], 1);    // both: the leader producer
      // leader: its warp 1 and 4 epilogue warps; the peer's producer, warp 1 and 4 epilogue warps
      mbar_init(&sche_bar[i], 1 + 4 + 1 + 1 + 4);
    }
    guard->abort = 0;
    guard->limit = p.wait_limit;
    fence_barrier_init();
    tma_prefetch_desc(&tmDY);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  // expert table: clamped counts, token offsets, heaviest-first order (as the single-CTA kernel)
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
  if (p.sort_by_m && E > 1) {
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
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int mt = (p.n + 255) / 256;
  const int nt = (p.k + BN - 1) / BN;
  const int per_expert = mt * nt;
  const int total_tiles = per_expert * E;

  if (warp == 0) {
    // -------------------------------------------------------------- TMA producers (both CTAs)
    if (lane == 0) {
      int stage = 0, phase = 0, q = 0, qphase = 0;
      uint32_t own_par = 0;               // peer: parity of its own full_bar per stage
      uint32_t armed = 0, armed_par = 0;  // stages this CTA armed on its own full_bar
      while (true) {
        WgradTile info;
        if (leader) {
          const int t = atomicAdd(&p.ws->tile_counter, 1);
          info.rows = 0;
          if (t < total_tiles) {
            const int e = t_order[t / per_expert];
            const int local = t % per_expert;
            const int m_idx = local % mt, n_idx = local / mt;
            info.m0 = m_idx * 256;
            info.rows = min(256, p.n - info.m0);
            info.n0 = n_idx * BN;
            info.expert = e;
            info.tok0 = t_rowoff[e];
            info.ntok = t_cnt[e];
          }
          if (!mbar_wait_cluster(&sche_bar[q], qphase ^ 1, guard, err, kDevTimeoutProducer))
            break;
          ring[q] = info;
          const uint32_t pr = mapa_shared(&ring[q], 1);
          st_cluster_v4(pr, info.m0, info.rows, info.n0, info.expert);
          st_cluster_v4(pr + 16, info.tok0, info.ntok, 0, 0);
          mbar_arrive(&schf_bar[q]);
          mbar_arrive_cluster(mapa_shared(&schf_bar[q], 1));
        } else {
          if (!mbar_wait_cluster(&schf_bar[q], qphase, guard, err, kDevTimeoutProducer)) break;
          info = ring[q];
          mbar_arrive_cluster(mapa_shared(&sche_bar[q], 0));
        }
        if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
        if (info.rows == 0) break;
        const int nkb = (info.ntok + kBK - 1) / kBK;
        const int a_col = info.m0 + static_cast<int>(rank) * 128;  // this CTA's dW rows
        const int b_col = info.n0 + static_cast<int>(rank) * 128;  // this CTA's dW columns
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_cluster(&empty_bar[stage], phase ^ 1, guard, err,
                                 kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = tiles + stage * L::kStageBytes;
          uint8_t* b_dst = a_dst + L::kABytes;
          const int y = info.tok0 + kb * kBK;
          const bool partial = info.ntok - kb * kBK < kBK;
          if (!partial) {  // both CTAs' bytes on the leader's barrier
            if (leader) {
              mbar_arrive_expect_tx(&full_bar[stage], 2 * L::kStageBytes);
              armed |= 1u << stage;
              armed_par = (armed_par & ~(1u << stage)) | (static_cast<uint32_t>(phase) << stage);
            }
            const uint32_t fb = mapa_shared(&full_bar[stage], 0);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              tma_load_2d_pair(a_dst + i * 8192, &tmDY, fb, a_col + 64 * i, y);
              tma_load_2d_pair(b_dst + i * 8192, &tmX, fb, b_col + 64 * i, y);
            }
          } else {  // each CTA's bytes on its own barrier, for its relay to zero
            const uint32_t par = leader ? static_cast<uint32_t>(phase) : (own_par >> stage) & 1u;
            mbar_arrive_expect_tx(&full_bar[stage], L::kStageBytes);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              tma_load_2d(a_dst + i * 8192, &tmDY, &full_bar[stage], a_col + 64 * i, y);
              tma_load_2d(b_dst + i * 8192, &tmX, &full_bar[stage], b_col + 64 * i, y);
            }
            armed |= 1u << stage;
            armed_par = (armed_par & ~(1u << stage)) | (par << stage);
            if (!leader) own_par ^= 1u << stage;
          }
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      if (guard->abort) drain_armed_stages<S>(full_bar, armed, armed_par, guard->limit);
    }
  } else if (warp == 1) {
    // ---------------------------- relay of partial blocks (both CTAs) + MMA issuer (leader)
    constexpr uint32_t idesc = idesc_f16(256, BN, BF16, true) | (1u << 15);  // A, B MN-major
    int stage = 0, phase = 0, q = 0, qphase = 0, acc = 0, aphase = 0;
    uint32_t own_par = 0;    // peer: parity of its own full_bar per stage (partial blocks only)
    uint32_t ready_par = 0;  // leader: parity of ready_bar per stage
    const uint32_t tiles_addr = smem_u32(tiles);
    while (true) {
      if (!mbar_wait_cluster(&schf_bar[q], qphase, guard, err, kDevTimeoutMma)) break;
      const WgradTile info = ring[q];
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&sche_bar[q]);
        else mbar_arrive_cluster(mapa_shared(&sche_bar[q], 0));
      }
      if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
      if (info.rows == 0) break;
      const int nkb = (info.ntok + kBK - 1) / kBK;
      bool ok = true;
      if (leader && lane == 0) {
        if (!mbar_wait_cluster(&acce_bar[acc], aphase ^ 1, guard, err, kDevTimeoutMma)) ok = false;
        tc_fence_after();
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      const uint32_t d_tmem = tmem_base + acc * kAccStride;
      for (int kb = 0; kb < nkb; ++kb) {
        const int valid = info.ntok - kb * kBK;
        const uint32_t s_addr = tiles_addr + stage * L::kStageBytes;
        if (valid < kBK) {
          // relay: this CTA's loads of the block landed; zero token rows [valid, 64) of its
          // four boxes (whole 128-B rows), then tell the leader
          const uint32_t par = leader ? static_cast<uint32_t>(phase) : (own_par >> stage) & 1u;
          if (!leader) own_par ^= 1u << stage;
          if (!mbar_wait(&full_bar[stage], par, guard, err, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          const int zrows = kBK - valid;
          for (int i = lane; i < 4 * zrows * 8; i += 32) {
            const int box = i / (zrows * 8), rem = i % (zrows * 8);
            const uint32_t addr = s_addr + box * 8192 + (valid + rem / 8) * 128 + (rem % 8) * 16;
            st_shared_v4(addr, 0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(&ready_bar[stage], 0));
        }
        if (leader && lane == 0) {
          bool got;
          if (valid < kBK) {
            got = mbar_wait_cluster(&ready_bar[stage], (ready_par >> stage) & 1u, guard, err,
                                    kDevTimeoutMma);
            ready_par ^= 1u << stage;
          } else {
            got = mbar_wait_cluster(&full_bar[stage], phase, guard, err, kDevTimeoutMma);
          }
          if (!got) {
            ok = false;
          } else {
            tc_fence_after();
            const uint64_t adesc = sdesc_sw128_mnmajor(s_addr, 8192);
            const uint64_t bdesc = sdesc_sw128_mnmajor(s_addr + L::kABytes, 8192);
#pragma unroll
            for (int kk = 0; kk < kBK / kUmmaK; ++kk)
              mma_f16_ss_pair(d_tmem, adesc + 128 * kk, bdesc + 128 * kk, idesc,
                              (kb | kk) != 0);
            mma_commit_pair(&empty_bar[stage], 0x3);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (++stage == S) { stage = 0; phase ^= 1; }
        if (!ok) break;
      }
      if (!ok) break;
      if (leader && lane == 0) {
        if (nkb > 0) {
          mma_commit_pair(&accf_bar[acc], 0x3);
        } else {  // no tokens: both epilogues write zeros
          mbar_arrive(&accf_bar[acc]);
          mbar_arrive_cluster(mapa_shared(&accf_bar[acc], 1));
        }
      }
      __syncwarp();
      if (++acc == 2) { acc = 0; aphase ^= 1; }
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- epilogue (both CTAs)
    const int ew = warp - 4;
    int q = 0, qphase = 0, acc = 0, aphase = 0;
    while (true) {
      if (!mbar_wait_cluster(&schf_bar[q], qphase, guard, err, kDevTimeoutEpilogue)) break;
      const WgradTile info = ring[q];
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&sche_bar[q]);
        else mbar_arrive_cluster(mapa_shared(&sche_bar[q], 0));
      }
      if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
      if (info.rows == 0) break;
      if (!mbar_wait_cluster(&accf_bar[acc], aphase, guard, err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int r_local = static_cast<int>(rank) * 128 + ew * 32 + lane;  // dW row in the tile
      const bool row_ok = r_local < info.rows;
      const int grow = info.expert * p.n + info.m0;  // row of dW viewed as [E*N, K]
      OutT* out_row = reinterpret_cast<OutT*>(p.out) + static_cast<size_t>(grow + r_local) * p.k;
      const int wrow0 = static_cast<int>(rank) * 128 + ew * 32;
      const bool warp_tma = wrow0 + 32 <= info.rows;
      if (info.ntok > 0) {
        const uint32_t t_row =
            tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + acc * kAccStride;
        store_tile_rows<BN, kEpiStore, BF16>(t_row, info.n0, p.k, row_ok, out_row, warp_tma,
                                             &tmW, staging + ew * 4096, grow + wrow0);
      } else if (row_ok) {  // expert without tokens: zero gradient
        for (int c = 0; c < BN; c += 8)
          if (info.n0 + c < p.k)
            *reinterpret_cast<uint4*>(out_row + info.n0 + c) = make_uint4(0u, 0u, 0u, 0u);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(&acce_bar[acc], 0));
      if (++acc == 2) { acc = 0; aphase ^= 1; }
    }
  }

  // ------------------------------------------------------------------ tear-down
  if (warp >= 4 && lane == 0) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no remote arrive or ring store may target a CTA that has exited
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
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
