// CTA-pair (cta_group::2) variant of the persistent grouped GEMM: 256 x 256 output tiles.
//
// A cluster of two CTAs on two SMs computes one 256-row tile. Each CTA TMA-loads its own 128 A
// rows and its own half (128 rows) of the B tile; one thread of the even CTA issues
// tcgen05.mma.cta_group::2 with M = 256, which reads A and the B halves from both CTAs' shared
// memory and accumulates each CTA's 128 rows into that CTA's TMEM. Per SM this moves 32 KB per
// 64-deep K step instead of 48 KB for a 128 x 256 single-CTA tile: the L2 -> SM operand traffic
// that bounds the single-CTA kernel drops by a third.
//
// Every bulk-tensor load lands in the issuing CTA's own shared memory (no broadcast); only its
// completion is counted on the leader's barrier (the cta_group::2 form of the bulk-tensor load).
// One tcgen05.commit with a two-CTA mask signals both CTAs' barriers when MMAs retire.
//
// Scheduling: the leader's producer claims a tile from the global atomic counter, decodes it and
// writes it into both CTAs' tile rings (distributed shared memory). Consumers of a ring slot in
// both CTAs release it on the leader's barrier.
#pragma once

#include "ggo_gemm.cuh"

namespace ggo {

template <int BN, bool MX = false>
struct PairLayout {
  static constexpr int kABytes = 128 * kBK * 2;       // this CTA's 128 A rows
  static constexpr int kBBytes = (BN / 2) * kBK * 2;  // this CTA's half of the BN-row B tile
  // MX: this CTA's A scales (one 512-B atom: 128 rows x 4 K groups of 32) and the scales of the
  // weight rows from the 128-row block where the tile's B rows start (kSfbAtoms atoms: a width
  // that is a multiple of 128 starts on a block, a multiple of 64 0 or 64 rows into one), behind
  // the B half
  static constexpr int kSfbAtoms = BN % 128 == 0 ? BN / 128 : (64 + BN + 127) / 128;
  static constexpr int kSfBytes = MX ? (1 + kSfbAtoms) * 512 : 0;
  static constexpr int kTxBytes = kABytes + kBBytes + kSfBytes;  // one CTA's loads per stage
  static constexpr int kStageBytes = (kTxBytes + 1023) / 1024 * 1024;  // 1024-B aligned stages
  static constexpr int kStagingBytes = 4 * 4096;  // TMA-store staging, 4 KB per epilogue warp
  // segment tables: counts, row offsets, order, tile offsets (+1), and for MX the scale blocks
  static constexpr int kTableBytes = MX ? 5 * kMaxSegments * 4 + 32 : 4 * kMaxSegments * 4 + 16;
  static constexpr int kMiscBytes = 1024;
  // as many stages (<= 8) as fit in the 227 KB a CTA may use, after everything else
  static constexpr int kRingBudget = 227 * 1024 - 1024 - kStagingBytes - kTableBytes - kMiscBytes;
  static constexpr int kStages = (kRingBudget / kStageBytes) > 8 ? 8 : (kRingBudget / kStageBytes);
  static constexpr int kTileBytes = kStages * kStageBytes;
  static constexpr int kTotal = 1024 + kTileBytes + kStagingBytes + kTableBytes + kMiscBytes;
  static_assert(kTotal <= 227 * 1024, "shared memory budget");
};

// MX = block-scaled e4m3 (kind::mxf8f6f4): tmSFA / tmSFB view the UE8M0 scales of A and B as
// [atoms * 2, 256] bytes (512-B atoms of 128 rows x 4 scales, the 128x4 blocked layout: a
// segment's rows start on a fresh 128-row block, atom (block, K group) at block * K/128 + group).
template <int BN, int EPI, bool BF16, bool BMN = false, bool FP8 = false, bool MX = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                             const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmC,
                             const __grid_constant__ CUtensorMap tmSFA,
                             const __grid_constant__ CUtensorMap tmSFB, const GemmParams p) {
  using L = PairLayout<BN, MX>;
  // MX: the scales of consecutive K steps rotate through 16-column TMEM slots (A: 4 columns, B:
  // 4 per atom) in the gaps beside the two accumulators (columns BN..255 and 256+BN..511), so
  // copying one step's scales never waits for the MMAs still reading the previous step's.
  // The block-scaled pair MMA is used only with N in {64, 128, 192, 256} and with B's scales
  // starting 0 or 2 TMEM words (0 or 64 weight rows) into a 128-row scale block: tiles start at
  // multiples of their width inside an expert, so a width in {64, 128, 192} gives exactly those
  // offsets (256 leaves no TMEM columns for the scale slots). A 224-wide variant (N = 224, offsets
  // 1 and 3) stopped with a misaligned-address error and is not built.
  static_assert(!MX || (FP8 && !BMN && (BN == 64 || BN == 128 || BN == 192 || BN == 256)),
                "MX tile width");
  static_assert(!MX || 4 + 4 * L::kSfbAtoms <= 16, "scale slot width");
  // MX with 256-wide tiles: the two accumulators overlap by 64 TMEM columns (columns 0-255 and
  // 192-447), which leaves columns 448-511 for four scale slots. The epilogue reads the overlapped
  // 64 columns of a tile first and then releases the next tile's MMAs (which overwrite them), and
  // drains the other 192 columns while those MMAs run.
  constexpr bool kOverlap = MX && BN == 256;
  constexpr uint32_t kSfSlotsPerGap = kOverlap ? 4 : (256 - BN) / 16;
  constexpr uint32_t kSfSlots = kOverlap ? 4 : 2 * kSfSlotsPerGap;
  static_assert(!MX || kSfSlots >= 2, "scale slots");
  constexpr int S = L::kStages;
  // BN = N of the pair tile = columns of each CTA's accumulator (multiple of 32, <= 256)
  static_assert(BN % 32 == 0 && BN <= 256 && (EPI == kEpiStore || BN % 64 == 0), "tile width");
  constexpr int kTileM = 256;
  constexpr int kAccStride = kOverlap ? 192 : 256;  // TMEM columns between the accumulators
  constexpr int kTmemCols = 512;
  constexpr int kOutBN = (EPI == kEpiSwiGLU) ? BN / 2 : BN;
  constexpr bool kTmaStoreOk = kOutBN % 64 == 0;  // output boxes are 64 columns wide

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* tiles = smem;
  uint8_t* staging = smem + L::kTileBytes;
  int* t_cnt = reinterpret_cast<int*>(smem + L::kTileBytes + L::kStagingBytes);
  int* t_rowoff = t_cnt + kMaxSegments;
  int* t_order = t_rowoff + kMaxSegments;
  int* t_tileoff = t_order + kMaxSegments;
  int* t_sfoff = t_tileoff + kMaxSegments + 4;  // MX only: first 128-row scale block per segment
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
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  int* err = &p.ws->error;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);    // leader: its expect_tx arrive + both CTAs' bytes
      mbar_init(&empty_bar[i], 1);   // both: one two-CTA commit per use
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf_bar[i], 1);    // both: one two-CTA commit per tile
      mbar_init(&acce_bar[i], 8);    // leader: 4 epilogue warps x 2 CTAs
    }
    for (int i = 0; i < kSchedDepth; ++i) {
      mbar_init(&schf_bar[i], 1);              // both: the leader producer
      mbar_init(&sche_bar[i], 1 + 4 + 1 + 4);  // leader: MMA, 4+4 epilogue warps, peer producer
    }
    guard->abort = 0;
    guard->limit = p.wait_limit;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  build_segment_table<kTileM, kOutBN>(p, tiles, t_cnt, t_rowoff, t_order, t_tileoff,
                                      total_tiles_s, err);
  if (MX && warp == 1) {  // exclusive prefix sum of 128-row scale blocks, in segment order
    const int nseg = p.num_segments;
    int carry = 0;
    for (int base = 0; base < nseg; base += 32) {
      const int s = base + lane;
      const int v = s < nseg ? (t_cnt[s] + 127) / 128 : 0;
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (s < nseg) t_sfoff[s] = carry + x - v;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = *total_tiles_s;
  const int heavy_tiles = total_tiles_s[1];
  constexpr int kStageK = FP8 ? 128 : kBK;  // K elements per stage (one 128-B swizzle row)
  const int num_kb = (p.k + kStageK - 1) / kStageK;

  if (warp == 0) {
    // -------------------------------------------------------------- TMA producers (both CTAs)
    if (lane == 0) {
      int stage = 0, phase = 0, q = 0, qphase = 0;
      uint32_t armed = 0, armed_par = 0;  // leader: stages armed, and their parity
      while (true) {
        TileInfo info;
        bool stall_tile = false;  // test hook: this pair claimed tile 0
        if (leader) {
          const int t = atomicAdd(&p.ws->tile_counter, 1);
          stall_tile = t == 0;
          info.rows = 0;
          if (t < total_tiles)
            info = decode_tile<kTileM, kOutBN, EPI, BN / 2, BMN>(
                interleave_tile(t, heavy_tiles, total_tiles), p, t_cnt, t_rowoff, t_order,
                                                               t_tileoff);
          if (!mbar_wait_cluster(&sche_bar[q], qphase ^ 1, guard, err, kDevTimeoutProducer))
            break;
          ring[q] = info;
          const uint32_t pr = mapa_shared(&ring[q], 1);
          st_cluster_v4(pr, info.row0, info.rows, info.n0, info.brow0);
          st_cluster_v4(pr + 16, info.brow1, info.seg, 0, 0);
          mbar_arrive(&schf_bar[q]);
          mbar_arrive_cluster(mapa_shared(&schf_bar[q], 1));
        } else {
          if (!mbar_wait_cluster(&schf_bar[q], qphase, guard, err, kDevTimeoutProducer))
            break;
          info = ring[q];
          mbar_arrive_cluster(mapa_shared(&sche_bar[q], 0));
        }
        if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
        if (info.rows == 0) break;
        const int a_row = info.row0 + static_cast<int>(rank) * 128;
        const int b_row = leader ? info.brow0 : info.brow1;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_cluster(&empty_bar[stage], phase ^ 1, guard, err,
                                 kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          // test hook: the leader of the pair that claimed tile 0 leaves its first stage unarmed
          const bool skip = p.inject_stall && stall_tile && kb == 0;
          if (!skip) {
            uint8_t* a_dst = tiles + stage * L::kStageBytes;
            uint8_t* b_dst = a_dst + L::kABytes;
            if (leader) {
              mbar_arrive_expect_tx(&full_bar[stage], 2 * L::kTxBytes);
              armed |= 1u << stage;
              armed_par = (armed_par & ~(1u << stage)) | (static_cast<uint32_t>(phase) << stage);
            }
            const uint32_t fb = mapa_shared(&full_bar[stage], 0);
            tma_load_2d_pair(a_dst, &tmA, fb, kb * kStageK, a_row);
            if (BMN) {  // this CTA's BN/2 output columns as 64-column boxes
#pragma unroll
              for (int i = 0; i < BN / 128; ++i)
                tma_load_2d_pair(b_dst + i * 8192, &tmB, fb,
                                 info.n0 + static_cast<int>(rank) * (BN / 2) + 64 * i,
                                 info.brow0 + kb * kBK);
            } else {
              tma_load_2d_pair(b_dst, &tmB, fb, kb * kStageK, b_row);
            }
            if (MX) {
              uint8_t* sf_dst = b_dst + L::kBBytes;
              const int seg = info.seg;
              const int blk_a = t_sfoff[seg] + (info.row0 - t_rowoff[seg]) / 128 +
                                static_cast<int>(rank);
              tma_load_2d_pair(sf_dst, &tmSFA, fb, 0, 2 * (blk_a * num_kb + kb));
              // both CTAs hold the scales of all the tile's weight rows (the MMA reads B's
              // scales from each CTA's own TMEM)
              const int w_row = epi_glu(EPI) ? 2 * info.n0 : info.n0;  // within the expert
              const int blk_b = (seg % p.num_experts) * ((p.n_b + 127) / 128) + w_row / 128;
#pragma unroll
              for (int i = 0; i < L::kSfbAtoms; ++i)
                tma_load_2d_pair(sf_dst + 512 * (i + 1), &tmSFB, fb, 0,
                                 2 * ((blk_b + i) * num_kb + kb));
            }
          }
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      // the leader's barriers count both CTAs' bytes; the final cluster barrier keeps the peer
      // resident until this drain is over
      if (leader && guard->abort) drain_armed_stages<S>(full_bar, armed, armed_par, guard->limit);
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA issuer (leader only)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16(kTileM, BN, FP8 ? false : BF16, BMN);
      static_assert(!BMN || (BN / 2) % 64 == 0, "MN-major B halves are whole 64-column boxes");
      int stage = 0, phase = 0, q = 0, qphase = 0, acc = 0, aphase = 0;
      uint32_t sf_slot = 0;  // MX: scale slot of the next K step
      int tiles_done = 0;    // overlapped accumulators: tiles issued so far
      const uint32_t tiles_addr = smem_u32(tiles);
      while (true) {
        if (!mbar_wait_cluster(&schf_bar[q], qphase, guard, err, kDevTimeoutMma)) break;
        const bool valid = ring[q].rows > 0;
        const int n0 = ring[q].n0;
        mbar_arrive(&sche_bar[q]);
        if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
        if (!valid) break;
        if (kOverlap) {
          // the previous tile's overlapped columns are read (and, the epilogue being in tile
          // order, every column of the tile before it); acce_bar[0] completes once per tile
          if (tiles_done > 0 && !mbar_wait_cluster(&acce_bar[0], (tiles_done - 1) & 1, guard, err,
                                                   kDevTimeoutMma))
            break;
          ++tiles_done;
        } else if (!mbar_wait_cluster(&acce_bar[acc], aphase ^ 1, guard, err, kDevTimeoutMma)) {
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccStride;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_cluster(&full_bar[stage], phase, guard, err, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = tiles_addr + stage * L::kStageBytes;
          const uint64_t adesc = sdesc_sw128_kmajor(a_addr);
          const uint64_t bdesc = BMN ? sdesc_sw128_mnmajor(a_addr + L::kABytes, 8192)
                                     : sdesc_sw128_kmajor(a_addr + L::kABytes);
          constexpr uint64_t kBStep = BMN ? (2048 >> 4) : 2;
          if constexpr (MX) {
            // scales of this stage into TMEM (in order with the MMAs below and the previous
            // stage's): A's 128 rows, then B's rows as kSfbAtoms 4-column atoms
            const uint32_t sf_addr = a_addr + L::kABytes + L::kBBytes;
            const uint32_t kSfaCol = kOverlap ? 448u + 16u * sf_slot
                                     : sf_slot < kSfSlotsPerGap
                                         ? BN + 16u * sf_slot
                                         : 256u + BN + 16u * (sf_slot - kSfSlotsPerGap);
            const uint32_t kSfbCol = kSfaCol + 4;
            if (++sf_slot == kSfSlots) sf_slot = 0;
            tmem_cp_32x128b_x4_pair(tmem_base + kSfaCol, sdesc_rows16(sf_addr));
#pragma unroll
            for (int i = 0; i < L::kSfbAtoms; ++i)
              tmem_cp_32x128b_x4_pair(tmem_base + kSfbCol + 4 * i,
                                      sdesc_rows16(sf_addr + 512 * (i + 1)));
            // weight row w of the tile has its scales in column (first row % 128 + w) / 32
            const uint32_t sfb_col =
                kSfbCol + static_cast<uint32_t>(((epi_glu(EPI) ? 2 * n0 : n0) & 127) >> 5);
            constexpr uint32_t kIdesc = idesc_mxf8(kTileM, BN);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)  // K step kk uses scale byte kk of each TMEM word
              mma_mxf8_ss_pair(d_tmem, adesc + 2 * kk, bdesc + 2 * kk,
                               idesc_sf_ids(kIdesc, kk, kk),
                               (tmem_base + kSfaCol) | (static_cast<uint32_t>(kk) << 30),
                               (tmem_base + sfb_col) | (static_cast<uint32_t>(kk) << 30),
                               (kb | kk) != 0);
          } else {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {  // four 32-byte K steps per 128-byte stage row
            if (FP8)
              mma_f8_ss_pair(d_tmem, adesc + 2 * kk, bdesc + kBStep * kk, idesc, (kb | kk) != 0);
            else
              mma_f16_ss_pair(d_tmem, adesc + 2 * kk, bdesc + kBStep * kk, idesc, (kb | kk) != 0);
          }
          }
          mma_commit_pair(&empty_bar[stage], 0x3);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit_pair(&accf_bar[acc], 0x3);
        if (++acc == 2) { acc = 0; aphase ^= 1; }
      }
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- epilogue (both CTAs)
    const int ew = warp - 4;
    int q = 0, qphase = 0, acc = 0, aphase = 0;
    using OutT = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    while (true) {
      if (!mbar_wait_cluster(&schf_bar[q], qphase, guard, err, kDevTimeoutEpilogue)) break;
      const TileInfo info = ring[q];
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(&sche_bar[q], 0));
      if (++q == kSchedDepth) { q = 0; qphase ^= 1; }
      if (info.rows == 0) break;
      if (!mbar_wait_cluster(&accf_bar[acc], aphase, guard, err, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int r_local = static_cast<int>(rank) * 128 + ew * 32 + lane;
      const bool row_ok = r_local < info.rows && info.row0 + r_local < p.rows;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + acc * kAccStride;
      OutT* out_row = output_row<OutT>(p, info, r_local, row_ok);
      const int wrow0 = static_cast<int>(rank) * 128 + ew * 32;
      const bool warp_tma = kTmaStoreOk && p.use_tma_store && wrow0 + 32 <= info.rows;
      constexpr bool kScaled = EPI == kEpiScaled || EPI == kEpiScaledSwiGLU;
      const float rs = (kScaled && row_ok) ? __ldg(p.row_scale + info.row0 + r_local) : 1.f;
      // column scales: one per weight row, [E, n_b] (gate rows then up rows for SwiGLU)
      const float* cs_row =
          kScaled ? p.col_scale + static_cast<size_t>(info.seg % p.num_experts) * p.n_b : nullptr;
      // overlapped accumulators: the columns shared with the other accumulator first (the last
      // 64 of accumulator 0, the first 64 of accumulator 1), then release the next tile's MMAs
      constexpr int kBoxes = (EPI == kEpiSwiGLU ? BN / 2 : BN) / 64;
      store_tile_rows<BN, EPI, BF16>(t_row, info.n0, p.n_out, row_ok, out_row, warp_tma, &tmC,
                                     staging + ew * 4096, info.row0 + wrow0, rs, cs_row,
                                     p.n_b / 2, p.origin != nullptr,
                                     kOverlap ? (acc == 0 ? kBoxes - 1 : 0) : 0,
                                     kOverlap ? mapa_shared(&acce_bar[0], 0) : 0u);
      tc_fence_before();
      __syncwarp();
      if (!kOverlap && lane == 0) mbar_arrive_cluster(mapa_shared(&acce_bar[acc], 0));
      if (++acc == 2) { acc = 0; aphase ^= 1; }
    }
  }

  // ------------------------------------------------------------------ tear-down
  if (p.origin) __threadfence_system();  // scattered rows visible to the peers before exit
  if (warp >= 4 && lane == 0) bulk_wait_all();  // TMA stores done before shared memory goes
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
