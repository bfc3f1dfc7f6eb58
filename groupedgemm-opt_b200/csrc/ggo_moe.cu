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

#include "ggo.h"

namespace ggo {
namespace {

constexpr int kRouteTokens = 128;  // tokens per route/permute block
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

// One block of 1024 threads. Turns block_counts[b][e] into absolute start rows (in place) and
// writes tokens_per_expert.
__global__ void __launch_bounds__(1024)
    route_scan_kernel(int* __restrict__ block_counts, int nblocks, int E,
                      int64_t* __restrict__ tpe) {
  __shared__ int tot[kMaxExperts];
  const int e = threadIdx.x;
  int sum = 0;
  if (e < E)
    for (int b = 0; b < nblocks; ++b) sum += block_counts[static_cast<size_t>(b) * E + e];
  tot[e] = e < E ? sum : 0;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {  // inclusive Hillis-Steele scan
    const int v = e >= o ? tot[e - o] : 0;
    __syncthreads();
    tot[e] += v;
    __syncthreads();
  }
  if (e < E) {
    int run = tot[e] - sum;  // exclusive start of expert e
    tpe[e] = sum;
    for (int b = 0; b < nblocks; ++b) {
      const size_t i = static_cast<size_t>(b) * E + e;
      const int c = block_counts[i];
      block_counts[i] = run;
      run += c;
    }
  }
}

// grid = ceil(T / kRouteTokens). Positions by one warp, row gather by all warps.
template <typename T16>
__global__ void __launch_bounds__(kRouteThreads)
    permute_kernel(const T16* __restrict__ x, int T, int H, int E, int K,
                   const int32_t* __restrict__ topk_ids, const int* __restrict__ block_offsets,
                   T16* __restrict__ xs, int32_t* __restrict__ sorted_token,
                   int32_t* __restrict__ slot_pos) {
  extern __shared__ int psm[];
  int* off = psm;        // [E]
  int* pos = psm + E;    // [kRouteTokens * K]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kRouteTokens;
  const int ntok = min(kRouteTokens, T - t0);
  const int nent = ntok * K;
  for (int e = threadIdx.x; e < E; e += kRouteThreads)
    off[e] = block_offsets[static_cast<size_t>(blockIdx.x) * E + e];
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
        const int rank = __popc(peers & ((1u << lane) - 1u));
        const int b = off[id];
        __syncwarp(vmask);
        if (lane == __ffs(peers) - 1) off[id] = b + __popc(peers);
        const int ps = b + rank;
        pos[i] = ps;
        const int t = t0 + i / K;
        slot_pos[static_cast<size_t>(t0) * K + i] = ps;
        sorted_token[ps] = t;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  const int vec = H / 8;  // 16-byte chunks per row
  for (int tl = warp; tl < ntok; tl += kRouteThreads / 32) {
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t0 + tl) * H);
    for (int c = lane; c < vec; c += 32) {
      const uint4 v = src[c];
      for (int j = 0; j < K; ++j) {
        uint4* dst = reinterpret_cast<uint4*>(xs + static_cast<size_t>(pos[tl * K + j]) * H);
        dst[c] = v;
      }
    }
  }
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
                   T16* __restrict__ out) {
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const int vec = H / 8;
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

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int nblocks_for(int64_t T) { return static_cast<int>((T + kRouteTokens - 1) / kRouteTokens); }

}  // namespace
}  // namespace ggo

extern "C" {

size_t ggo_moe_route_scratch_bytes(int64_t num_tokens, int num_experts) {
  if (num_tokens <= 0 || num_experts <= 0) return 16;
  return static_cast<size_t>(ggo::nblocks_for(num_tokens)) * num_experts * sizeof(int);
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
  return cudaGetLastError() == cudaSuccess ? GGO_OK : GGO_ERR_CUDA;
}

int ggo_moe_permute(const void* x_dev, int64_t num_tokens, int64_t hidden, int num_experts,
                    int top_k, const int32_t* topk_ids_dev, void* x_sorted_dev,
                    int32_t* sorted_token_dev, int32_t* slot_pos_dev, void* scratch_dev,
                    int dtype, cudaStream_t stream) {
  if (!x_dev || !topk_ids_dev || !x_sorted_dev || !sorted_token_dev || !slot_pos_dev ||
      !scratch_dev)
    return GGO_ERR_INVALID_ARG;
  if (num_tokens < 0 || hidden <= 0 || num_experts <= 0 || num_experts > ggo::kMaxExperts ||
      top_k <= 0 || top_k > ggo::kMaxTopK)
    return GGO_ERR_INVALID_ARG;
  if (dtype != GGO_DTYPE_BF16 && dtype != GGO_DTYPE_FP16) return GGO_ERR_DTYPE;
  if (hidden % 8 || !ggo::aligned16(x_dev) || !ggo::aligned16(x_sorted_dev))
    return GGO_ERR_ALIGNMENT;
  if (num_tokens * top_k > INT32_MAX || hidden > INT32_MAX) return GGO_ERR_SHAPE;
  const int T = static_cast<int>(num_tokens);
  const int nb = ggo::nblocks_for(T);
  if (nb == 0) return GGO_OK;
  const size_t smem = (static_cast<size_t>(num_experts) + ggo::kRouteTokens * top_k) * 4;
  const int* bo = static_cast<const int*>(scratch_dev);
  if (dtype == GGO_DTYPE_BF16) {
    ggo::permute_kernel<__nv_bfloat16><<<nb, ggo::kRouteThreads, smem, stream>>>(
        static_cast<const __nv_bfloat16*>(x_dev), T, static_cast<int>(hidden), num_experts, top_k,
        topk_ids_dev, bo, static_cast<__nv_bfloat16*>(x_sorted_dev), sorted_token_dev,
        slot_pos_dev);
  } else {
    ggo::permute_kernel<__half><<<nb, ggo::kRouteThreads, smem, stream>>>(
        static_cast<const __half*>(x_dev), T, static_cast<int>(hidden), num_experts, top_k,
        topk_ids_dev, bo, static_cast<__half*>(x_sorted_dev), sorted_token_dev, slot_pos_dev);
  }
  return cudaGetLastError() == cudaSuccess ? GGO_OK : GGO_ERR_CUDA;
}

int ggo_moe_combine(const void* y_sorted_dev, const float* topk_weights_dev,
                    const int32_t* slot_pos_dev, int64_t num_tokens, int64_t hidden, int top_k,
                    void* out_dev, int dtype, cudaStream_t stream) {
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
        static_cast<int>(hidden), top_k, static_cast<__nv_bfloat16*>(out_dev));
  } else {
    ggo::combine_kernel<__half><<<grid, 256, 0, stream>>>(
        static_cast<const __half*>(y_sorted_dev), topk_weights_dev, slot_pos_dev, T,
        static_cast<int>(hidden), top_k, static_cast<__half*>(out_dev));
  }
  return cudaGetLastError() == cudaSuccess ? GGO_OK : GGO_ERR_CUDA;
}

}  // extern "C"
