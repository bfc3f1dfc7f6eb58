// grouped_gemm_opt._C: thin PyTorch binding over the C ABI of libggo_b200.so (include/ggo.h).
//
// Replaces the reference binding csrc/torch_ext.cpp:1-27 and the torch-facing half of
// csrc/grouped_gemm_kernel.cu:348-450. This file only validates tensors, allocates outputs and
// per-stream workspaces through the torch caching allocator, and maps status codes to
// RuntimeError. All arithmetic happens in the CUDA kernels behind the C ABI.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>
#include <array>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "ggo.h"

namespace {

void check_status(int st, const char* what) {
  TORCH_CHECK(st == GGO_OK, what, " failed: ", ggo_status_string(st), " (status ", st, ")",
              st == GGO_ERR_CUDA ? std::string(": ") + ggo_last_cuda_error_string()
                                 : std::string());
}

int dtype_code(const torch::Tensor& t) {
  if (t.scalar_type() == torch::kBFloat16) return GGO_DTYPE_BF16;
  if (t.scalar_type() == torch::kHalf) return GGO_DTYPE_FP16;
  TORCH_CHECK(false, "Unsupported dtype: ", t.scalar_type());
  return -1;
}

// One zero-initialised workspace per (device, stream); kept for the life of the process.
std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, torch::Tensor> g_ws;

void* workspace_for(const torch::Device& dev, cudaStream_t stream) {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  auto key = std::make_pair(static_cast<int>(dev.index()), stream);
  auto it = g_ws.find(key);
  if (it == g_ws.end()) {
    auto t = torch::zeros({static_cast<int64_t>(ggo_workspace_size())},
                          torch::TensorOptions().dtype(torch::kUInt8).device(dev));
    it = g_ws.emplace(key, t).first;
  }
  return it->second.data_ptr();
}

torch::Tensor counts_on_device(const torch::Tensor& counts, const torch::Device& dev) {
  auto c = counts.to(torch::kInt64);
  if (!c.is_cuda() || c.device() != dev) c = c.to(dev, /*non_blocking=*/true);
  return c.contiguous();
}

void check_operands(const torch::Tensor& input, const torch::Tensor& weights) {
  TORCH_CHECK(input.is_cuda(), "input must be on CUDA");
  TORCH_CHECK(weights.is_cuda(), "weights must be on CUDA");
  TORCH_CHECK(input.dim() == 2, "input must be 2D [total_tokens, K]");
  TORCH_CHECK(weights.dim() == 3, "weights must be 3D [num_experts, N, K]");
  TORCH_CHECK(input.size(1) == weights.size(2), "K mismatch: input=", input.size(1),
              " vs weights=", weights.size(2));
  TORCH_CHECK(input.is_contiguous() && weights.is_contiguous(),
              "input and weights must be contiguous");
  TORCH_CHECK(input.scalar_type() == weights.scalar_type(), "input/weights dtype mismatch");
  TORCH_CHECK(input.device() == weights.device(), "input/weights on different devices");
}

// grouped_gemm_opt_forward(input, weights, tokens_per_expert, tile_config=4, sort_by_m=True)
// (reference csrc/torch_ext.cpp:19-27). Counts may be on the CPU or the GPU; on the GPU nothing
// synchronises.
torch::Tensor grouped_gemm_segments(const torch::Tensor& input, const torch::Tensor& weights,
                                    const torch::Tensor& counts, int64_t num_experts,
                                    int64_t tile_config, bool sort_by_m) {
  check_operands(input, weights);
  TORCH_CHECK(counts.dim() == 1, "tokens_per_expert must be 1D");
  c10::cuda::CUDAGuard guard(input.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t T = input.size(0), K = input.size(1), N = weights.size(1);
  auto out = torch::empty({T, N}, input.options());
  if (T == 0) return out;
  auto c = counts_on_device(counts, input.device());
  const int st = ggo_grouped_gemm_segments(
      input.data_ptr(), weights.data_ptr(), out.data_ptr(), c.data_ptr<int64_t>(),
      static_cast<int>(c.size(0)), static_cast<int>(num_experts), T, N, K, dtype_code(input),
      static_cast<int>(tile_config), sort_by_m ? 1 : 0, workspace_for(input.device(), stream),
      stream);
  check_status(st, "grouped GEMM");
  return out;
}

torch::Tensor grouped_gemm_forward(const torch::Tensor& input, const torch::Tensor& weights,
                                   const torch::Tensor& tokens_per_expert, int64_t tile_config,
                                   bool sort_by_m) {
  check_operands(input, weights);
  TORCH_CHECK(tokens_per_expert.dim() == 1 && tokens_per_expert.size(0) == weights.size(0),
              "tokens_per_expert must be 1D with num_experts entries");
  return grouped_gemm_segments(input, weights, tokens_per_expert, weights.size(0), tile_config,
                               sort_by_m);
}

// dx = dy @ W[e] per expert segment (weights [E, N, K], dy [T, N] -> dx [T, K]).
torch::Tensor grouped_gemm_dgrad(const torch::Tensor& dy, const torch::Tensor& weights,
                                 const torch::Tensor& tokens_per_expert, int64_t tile_config,
                                 bool sort_by_m) {
  TORCH_CHECK(dy.is_cuda() && weights.is_cuda(), "dy and weights must be on CUDA");
  TORCH_CHECK(dy.dim() == 2 && weights.dim() == 3, "dy [T, N], weights [E, N, K]");
  TORCH_CHECK(dy.size(1) == weights.size(1), "N mismatch: dy=", dy.size(1), " vs weights=",
              weights.size(1));
  TORCH_CHECK(dy.is_contiguous() && weights.is_contiguous(), "dy and weights must be contiguous");
  TORCH_CHECK(dy.scalar_type() == weights.scalar_type(), "dy/weights dtype mismatch");
  TORCH_CHECK(tokens_per_expert.dim() == 1 && tokens_per_expert.size(0) == weights.size(0),
              "tokens_per_expert must be 1D with num_experts entries");
  c10::cuda::CUDAGuard guard(dy.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t T = dy.size(0), N = weights.size(1), K = weights.size(2);
  auto dx = torch::empty({T, K}, dy.options());
  if (T == 0) return dx;
  auto c = counts_on_device(tokens_per_expert, dy.device());
  const int st = ggo_grouped_gemm_dgrad(
      dy.data_ptr(), weights.data_ptr(), dx.data_ptr(), c.data_ptr<int64_t>(),
      static_cast<int>(weights.size(0)), T, N, K, dtype_code(dy), static_cast<int>(tile_config),
      sort_by_m ? 1 : 0, workspace_for(dy.device(), stream), stream);
  check_status(st, "grouped GEMM dgrad");
  return dx;
}

// dw[e] = dy_e^T @ x_e per expert (x [T, K], dy [T, N] -> dw [E, N, K]).
torch::Tensor grouped_gemm_wgrad(const torch::Tensor& x, const torch::Tensor& dy,
                                 const torch::Tensor& tokens_per_expert, bool sort_by_m) {
  TORCH_CHECK(x.is_cuda() && dy.is_cuda(), "x and dy must be on CUDA");
  TORCH_CHECK(x.dim() == 2 && dy.dim() == 2 && x.size(0) == dy.size(0),
              "x [T, K] and dy [T, N] with the same rows");
  TORCH_CHECK(x.is_contiguous() && dy.is_contiguous(), "x and dy must be contiguous");
  TORCH_CHECK(x.scalar_type() == dy.scalar_type(), "x/dy dtype mismatch");
  TORCH_CHECK(tokens_per_expert.dim() == 1, "tokens_per_expert must be 1D");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t T = x.size(0), K = x.size(1), N = dy.size(1), E = tokens_per_expert.size(0);
  auto dw = torch::empty({E, N, K}, x.options());
  auto c = counts_on_device(tokens_per_expert, x.device());
  const int st = ggo_grouped_gemm_wgrad(x.data_ptr(), dy.data_ptr(), dw.data_ptr(),
                                        c.data_ptr<int64_t>(), static_cast<int>(E), T, N, K,
                                        dtype_code(x), sort_by_m ? 1 : 0,
                                        workspace_for(x.device(), stream), stream);
  check_status(st, "grouped GEMM wgrad");
  return dw;
}

// Row-wise e4m3 quantisation: returns (q float8_e4m3fn [rows, cols], scale fp32 [rows]).
std::tuple<torch::Tensor, torch::Tensor> quantize_fp8_rows(const torch::Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() >= 2, "x must be contiguous CUDA");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t cols = x.size(-1), rows = x.numel() / cols;
  auto q = torch::empty(x.sizes(), x.options().dtype(torch::kFloat8_e4m3fn));
  auto sizes = x.sizes().vec();
  sizes.pop_back();
  auto s = torch::empty(sizes, x.options().dtype(torch::kFloat32));
  check_status(ggo_quantize_fp8_rows(x.data_ptr(), rows, cols, dtype_code(x), q.data_ptr(),
                                     s.data_ptr<float>(), stream),
               "fp8 quantisation");
  return {q, s};
}

// FP8 grouped GEMM: out bf16 [T, N] = (a_q @ w_q[e]^T) * a_scale[row] * w_scale[e, col].
torch::Tensor grouped_gemm_fp8(const torch::Tensor& a_q, const torch::Tensor& a_scale,
                               const torch::Tensor& w_q, const torch::Tensor& w_scale,
                               const torch::Tensor& tokens_per_expert, int64_t tile_config,
                               bool sort_by_m) {
  TORCH_CHECK(a_q.is_cuda() && w_q.is_cuda() && a_q.dim() == 2 && w_q.dim() == 3,
              "a_q [T, K] and w_q [E, N, K] CUDA tensors");
  TORCH_CHECK(a_q.scalar_type() == torch::kFloat8_e4m3fn &&
                  w_q.scalar_type() == torch::kFloat8_e4m3fn, "operands must be float8_e4m3fn");
  TORCH_CHECK(a_q.size(1) == w_q.size(2), "K mismatch");
  TORCH_CHECK(a_q.is_contiguous() && w_q.is_contiguous(), "operands must be contiguous");
  TORCH_CHECK(a_scale.scalar_type() == torch::kFloat32 && a_scale.numel() == a_q.size(0) &&
                  a_scale.is_contiguous(), "a_scale must be fp32 [T]");
  TORCH_CHECK(w_scale.scalar_type() == torch::kFloat32 &&
                  w_scale.numel() == w_q.size(0) * w_q.size(1) && w_scale.is_contiguous(),
              "w_scale must be fp32 [E, N]");
  c10::cuda::CUDAGuard guard(a_q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t T = a_q.size(0), K = a_q.size(1), E = w_q.size(0), N = w_q.size(1);
  auto out = torch::empty({T, N}, a_q.options().dtype(torch::kBFloat16));
  if (T == 0) return out;
  auto c = counts_on_device(tokens_per_expert, a_q.device());
  const int st = ggo_grouped_gemm_fp8(
      a_q.data_ptr(), a_scale.data_ptr<float>(), w_q.data_ptr(), w_scale.data_ptr<float>(),
      out.data_ptr(), c.data_ptr<int64_t>(), static_cast<int>(E), T, N, K,
      static_cast<int>(tile_config), sort_by_m ? 1 : 0, workspace_for(a_q.device(), stream),
      stream);
  check_status(st, "fp8 grouped GEMM");
  return out;
}

// FP8 gate/up SwiGLU grouped GEMM: h bf16 [T, F].
torch::Tensor grouped_gemm_swiglu_fp8(const torch::Tensor& x_q, const torch::Tensor& x_scale,
                                      const torch::Tensor& w_q, const torch::Tensor& w_scale,
                                      const torch::Tensor& counts, int64_t num_experts,
                                      bool sort_by_m) {
  TORCH_CHECK(x_q.is_cuda() && w_q.is_cuda() && x_q.dim() == 2 && w_q.dim() == 3,
              "x_q [T, K] and w_q [E, 2F, K] CUDA tensors");
  TORCH_CHECK(x_q.scalar_type() == torch::kFloat8_e4m3fn &&
                  w_q.scalar_type() == torch::kFloat8_e4m3fn, "operands must be float8_e4m3fn");
  TORCH_CHECK(x_q.size(1) == w_q.size(2) && w_q.size(1) % 2 == 0, "shape mismatch");
  TORCH_CHECK(x_q.is_contiguous() && w_q.is_contiguous(), "operands must be contiguous");
  TORCH_CHECK(x_scale.scalar_type() == torch::kFloat32 && x_scale.numel() == x_q.size(0) &&
                  w_scale.scalar_type() == torch::kFloat32 &&
                  w_scale.numel() == w_q.size(0) * w_q.size(1) && x_scale.is_contiguous() &&
                  w_scale.is_contiguous(),
              "scales: fp32 [T] and [E, 2F]");
  c10::cuda::CUDAGuard guard(x_q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t T = x_q.size(0), K = x_q.size(1), F = w_q.size(1) / 2;
  auto h = torch::empty({T, F}, x_q.options().dtype(torch::kBFloat16));
  if (T == 0) return h;
  auto c = counts_on_device(counts, x_q.device());
  const int st = ggo_grouped_gemm_swiglu_fp8(
      x_q.data_ptr(), x_scale.data_ptr<float>(), w_q.data_ptr(), w_scale.data_ptr<float>(),
      h.data_ptr(), c.data_ptr<int64_t>(), static_cast<int>(c.size(0)),
      static_cast<int>(num_experts), T, F, K, sort_by_m ? 1 : 0,
      workspace_for(x_q.device(), stream), stream);
  check_status(st, "fp8 gate/up SwiGLU grouped GEMM");
  return h;
}

// MX quantisation of x [..., K] whose rows form segments of `counts` rows: returns (q
// float8_e4m3fn, same shape, UE8M0 scales uint8 [ggo_mxfp8_scale_bytes] in the blocked layout;
// padding bytes zero).
std::tuple<torch::Tensor, torch::Tensor> quantize_mxfp8(const torch::Tensor& x,
                                                        const torch::Tensor& counts) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.dim() >= 2, "x must be contiguous CUDA");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t k = x.size(-1), rows = x.numel() / k;
  auto c = counts_on_device(counts, x.device());
  const int nseg = static_cast<int>(c.numel());
  const size_t sb = ggo_mxfp8_scale_bytes(rows, nseg, k);
  TORCH_CHECK(sb > 0 || rows == 0, "K must be a multiple of 128");
  auto q = torch::empty(x.sizes(), x.options().dtype(torch::kFloat8_e4m3fn));
  auto sf = torch::zeros({static_cast<int64_t>(sb)}, x.options().dtype(torch::kUInt8));
  check_status(ggo_quantize_mxfp8(x.data_ptr(), dtype_code(x), c.data_ptr<int64_t>(), nseg, rows,
                                  k, q.data_ptr(), sf.data_ptr(), stream),
               "mxfp8 quantisation");
  return {q, sf};
}

void check_mx_operands(const torch::Tensor& a_q, const torch::Tensor& a_sf,
                       const torch::Tensor& w_q, const torch::Tensor& w_sf, int64_t nseg) {
  TORCH_CHECK(a_q.is_cuda() && w_q.is_cuda() && a_q.dim() == 2 && w_q.dim() == 3,
              "a_q [T, K] and w_q [E, N, K] CUDA tensors");
  TORCH_CHECK(a_q.scalar_type() == torch::kFloat8_e4m3fn &&
                  w_q.scalar_type() == torch::kFloat8_e4m3fn, "operands must be float8_e4m3fn");
  TORCH_CHECK(a_q.size(1) == w_q.size(2), "K mismatch");
  TORCH_CHECK(a_q.is_contiguous() && w_q.is_contiguous() && a_sf.is_contiguous() &&
                  w_sf.is_contiguous(), "operands must be contiguous");
  TORCH_CHECK(a_sf.scalar_type() == torch::kUInt8 && w_sf.scalar_type() == torch::kUInt8,
              "scales must be uint8 (UE8M0)");
  const int64_t T = a_q.size(0), K = a_q.size(1), E = w_q.size(0), N = w_q.size(1);
  TORCH_CHECK(a_sf.numel() >= static_cast<int64_t>(ggo_mxfp8_scale_bytes(T, nseg, K)),
              "input scales smaller than ggo_mxfp8_scale_bytes(T, segments, K)");
  TORCH_CHECK(w_sf.numel() >= E * ((N + 127) / 128) * (K / 128) * 512,
              "weight scales smaller than E * ceil(N / 128) * K / 128 atoms");
}

// MXFP8 grouped GEMM: out bf16 [T, N].
torch::Tensor grouped_gemm_mxfp8(const torch::Tensor& a_q, const torch::Tensor& a_sf,
                                 const torch::Tensor& w_q, const torch::Tensor& w_sf,
                                 const torch::Tensor& counts, int64_t num_experts,
                                 bool sort_by_m) {
  check_mx_operands(a_q, a_sf, w_q, w_sf, counts.numel());
  c10::cuda::CUDAGuard guard(a_q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t T = a_q.size(0), K = a_q.size(1), N = w_q.size(1);
  auto out = torch::empty({T, N}, a_q.options().dtype(torch::kBFloat16));
  if (T == 0) return out;
  auto c = counts_on_device(counts, a_q.device());
  const int st = ggo_grouped_gemm_mxfp8(
      a_q.data_ptr(), a_sf.data_ptr(), w_q.data_ptr(), w_sf.data_ptr(), out.data_ptr(),
      c.data_ptr<int64_t>(), static_cast<int>(c.numel()), static_cast<int>(num_experts), T, N, K,
      sort_by_m ? 1 : 0, workspace_for(a_q.device(), stream), stream);
  check_status(st, "mxfp8 grouped GEMM");
  return out;
}

// MXFP8 gate/up SwiGLU grouped GEMM over the blocked gate/up weight [E, glu_rows(F), K]: h [T, F].
torch::Tensor grouped_gemm_swiglu_mxfp8(const torch::Tensor& x_q, const torch::Tensor& x_sf,
                                        const torch::Tensor& w_q, const torch::Tensor& w_sf,
                                        const torch::Tensor& counts, int64_t num_experts,
                                        int64_t F, bool sort_by_m) {
  check_mx_operands(x_q, x_sf, w_q, w_sf, counts.numel());
  TORCH_CHECK(F > 0 && w_q.size(1) == ggo_mxfp8_glu_rows(F),
              "w_q must be the blocked gate/up weight [E, ggo_mxfp8_glu_rows(F), K]");
  c10::cuda::CUDAGuard guard(x_q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t T = x_q.size(0), K = x_q.size(1);
  auto h = torch::empty({T, F}, x_q.options().dtype(torch::kBFloat16));
  if (T == 0) return h;
  auto c = counts_on_device(counts, x_q.device());
  const int st = ggo_grouped_gemm_swiglu_mxfp8(
      x_q.data_ptr(), x_sf.data_ptr(), w_q.data_ptr(), w_sf.data_ptr(), h.data_ptr(),
      c.data_ptr<int64_t>(), static_cast<int>(c.numel()), static_cast<int>(num_experts), T, F, K,
      sort_by_m ? 1 : 0, workspace_for(x_q.device(), stream), stream);
  check_status(st, "mxfp8 gate/up SwiGLU grouped GEMM");
  return h;
}

torch::Tensor grouped_gemm_swiglu(const torch::Tensor& x, const torch::Tensor& w_gate_up,
                                  const torch::Tensor& counts, int64_t num_experts,
                                  bool sort_by_m) {
  check_operands(x, w_gate_up);
  TORCH_CHECK(w_gate_up.size(1) % 2 == 0, "w_gate_up must have 2F rows per expert");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t T = x.size(0), K = x.size(1), F = w_gate_up.size(1) / 2;
  auto h = torch::empty({T, F}, x.options());
  if (T == 0) return h;
  auto c = counts_on_device(counts, x.device());
  const int st = ggo_grouped_gemm_swiglu(
      x.data_ptr(), w_gate_up.data_ptr(), h.data_ptr(), c.data_ptr<int64_t>(),
      static_cast<int>(c.size(0)), static_cast<int>(num_experts), T, F, K, dtype_code(x),
      sort_by_m ? 1 : 0, workspace_for(x.device(), stream), stream);
  check_status(st, "gate/up SwiGLU grouped GEMM");
  return h;
}

// Router: returns (topk_ids int32 [T,k], topk_weights fp32 [T,k], tokens_per_expert int64 [E],
// scratch int32) -- scratch carries the per-block offsets to moe_permute.
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor> moe_route(
    const torch::Tensor& logits, int64_t top_k) {
  TORCH_CHECK(logits.is_cuda() && logits.dim() == 2, "router_logits must be a 2D CUDA tensor");
  c10::cuda::CUDAGuard guard(logits.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  auto lg = logits.to(torch::kFloat32).contiguous();
  const int64_t T = lg.size(0), E = lg.size(1);
  auto i32 = torch::TensorOptions().dtype(torch::kInt32).device(lg.device());
  auto ids = torch::empty({T, top_k}, i32);
  auto w = torch::empty({T, top_k}, lg.options());
  auto tpe = torch::empty({E}, torch::TensorOptions().dtype(torch::kInt64).device(lg.device()));
  const int64_t sb = static_cast<int64_t>(ggo_moe_route_scratch_bytes(T, static_cast<int>(E)));
  auto scratch = torch::empty({(sb + 3) / 4}, i32);
  const int st = ggo_moe_route(lg.data_ptr<float>(), T, static_cast<int>(E),
                               static_cast<int>(top_k), ids.data_ptr<int32_t>(),
                               w.data_ptr<float>(), tpe.data_ptr<int64_t>(), scratch.data_ptr(),
                               stream);
  check_status(st, "MoE router");
  return {ids, w, tpe, scratch};
}

// Permute: returns (x_sorted [T*k,H], sorted_token int32 [T*k], slot_pos int32 [T*k]).
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> moe_permute(
    const torch::Tensor& x, const torch::Tensor& topk_ids, const torch::Tensor& scratch,
    int64_t num_experts) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "hidden must be 2D contiguous CUDA");
  TORCH_CHECK(topk_ids.scalar_type() == torch::kInt32 && topk_ids.is_contiguous(),
              "topk_ids must be contiguous int32");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t T = x.size(0), H = x.size(1), k = topk_ids.size(1);
  auto xs = torch::empty({T * k, H}, x.options());
  auto i32 = torch::TensorOptions().dtype(torch::kInt32).device(x.device());
  auto stok = torch::empty({T * k}, i32);
  auto spos = torch::empty({T * k}, i32);
  const int st = ggo_moe_permute(x.data_ptr(), T, H, static_cast<int>(num_experts),
                                 static_cast<int>(k), topk_ids.data_ptr<int32_t>(), xs.data_ptr(),
                                 stok.data_ptr<int32_t>(), spos.data_ptr<int32_t>(),
                                 scratch.data_ptr(), dtype_code(x), stream);
  check_status(st, "MoE permute");
  return {xs, stok, spos};
}

torch::Tensor moe_combine(const torch::Tensor& y_sorted, const torch::Tensor& topk_weights,
                          const torch::Tensor& slot_pos, bool checked) {
  TORCH_CHECK(y_sorted.is_cuda() && y_sorted.dim() == 2 && y_sorted.is_contiguous(),
              "y_sorted must be 2D contiguous CUDA");
  TORCH_CHECK(topk_weights.scalar_type() == torch::kFloat32 && topk_weights.is_contiguous(),
              "topk_weights must be contiguous fp32");
  TORCH_CHECK(slot_pos.scalar_type() == torch::kInt32 && slot_pos.is_contiguous(),
              "slot_pos must be contiguous int32");
  c10::cuda::CUDAGuard guard(y_sorted.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t T = topk_weights.size(0), k = topk_weights.size(1), H = y_sorted.size(1);
  auto out = torch::empty({T, H}, y_sorted.options());
  // checked: NaN output when the stream's workspace error word is set (an expired peer wait)
  const int st = ggo_moe_combine_checked(
      y_sorted.data_ptr(), topk_weights.data_ptr<float>(), slot_pos.data_ptr<int32_t>(), T, H,
      static_cast<int>(k), out.data_ptr(), dtype_code(y_sorted),
      checked ? workspace_for(y_sorted.device(), stream) : nullptr, stream);
  check_status(st, "MoE combine");
  return out;
}

// Reads and clears the device-side error word of the current stream's workspace (synchronises).
int64_t workspace_error(int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  int code = 0;
  const int st = ggo_workspace_error(
      workspace_for(torch::Device(torch::kCUDA, static_cast<c10::DeviceIndex>(device)), stream),
      stream, &code);
  check_status(st, "workspace error read");
  return code;
}

// ------------------------------------------------------------------ host-buffer pipeline
// Three persistent non-blocking streams per device: copies in, grouped GEMMs, copies out.
std::mutex g_side_mu;
std::map<int, std::array<cudaStream_t, 3>> g_side_streams;

std::array<cudaStream_t, 3> side_streams(int dev) {
  std::lock_guard<std::mutex> lk(g_side_mu);
  auto it = g_side_streams.find(dev);
  if (it == g_side_streams.end()) {
    std::array<cudaStream_t, 3> s{};
    for (auto& x : s)
      TORCH_CHECK(cudaStreamCreateWithFlags(&x, cudaStreamNonBlocking) == cudaSuccess,
                  "stream creation failed");
    it = g_side_streams.emplace(dev, s).first;
  }
  return it->second;
}

// Grouped GEMM on host-resident activations (see grouped_gemm_opt_host): expert groups of about
// T/chunks rows are copied in, multiplied and copied back on three streams so the stages of
// consecutive groups overlap. Inputs/outputs should be pinned for the copies to be asynchronous.
// All work is joined back to the current stream before returning (nothing waits on the host).
torch::Tensor grouped_gemm_host(const torch::Tensor& input, const torch::Tensor& weights,
                                const torch::Tensor& tokens_per_expert, torch::Tensor out,
                                int64_t tile_config, bool sort_by_m, int64_t chunks) {
  TORCH_CHECK(!input.is_cuda() && input.dim() == 2 && input.is_contiguous(),
              "input must be a contiguous 2D host tensor");
  TORCH_CHECK(weights.is_cuda() && weights.dim() == 3 && weights.is_contiguous(),
              "weights must be a contiguous 3D CUDA tensor");
  TORCH_CHECK(input.size(1) == weights.size(2), "K mismatch");
  TORCH_CHECK(input.scalar_type() == weights.scalar_type(), "input/weights dtype mismatch");
  auto tpe = tokens_per_expert.to(torch::kInt64).cpu().contiguous();
  const int64_t T = input.size(0), K = input.size(1), E = weights.size(0), N = weights.size(1);
  TORCH_CHECK(tpe.numel() == E, "tokens_per_expert must have num_experts entries");
  const int64_t* c = tpe.data_ptr<int64_t>();
  int64_t total = 0;
  for (int64_t e = 0; e < E; ++e) total += c[e];
  TORCH_CHECK(total == T, "sum(tokens_per_expert)=", total, " != total_tokens=", T);
  TORCH_CHECK(out.defined() && !out.is_cuda() && out.is_contiguous() && out.size(0) == T &&
                  out.size(1) == N && out.scalar_type() == input.scalar_type(),
              "out must be a contiguous host tensor [T, N] of the input dtype");
  if (T == 0) return out;
  c10::cuda::CUDAGuard guard(weights.device());
  const int dev = weights.device().index();
  cudaStream_t cur = at::cuda::getCurrentCUDAStream();
  auto ss = side_streams(dev);
  cudaStream_t s_in = ss[0], s_mm = ss[1], s_out = ss[2];
  const size_t esz = input.element_size();
  auto dopt = input.options().device(weights.device());
  auto d_x = torch::empty({T, K}, dopt);
  auto d_y = torch::empty({T, N}, dopt);
  auto d_c = torch::empty({E}, torch::TensorOptions().dtype(torch::kInt64).device(weights.device()));
  std::vector<cudaEvent_t> evs;
  auto event = [&](cudaStream_t s) {
    cudaEvent_t ev;
    TORCH_CHECK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) == cudaSuccess, "event");
    TORCH_CHECK(cudaEventRecord(ev, s) == cudaSuccess, "event record");
    evs.push_back(ev);
    return ev;
  };
  cudaEvent_t e0 = event(cur);
  for (cudaStream_t s : {s_in, s_mm, s_out}) cudaStreamWaitEvent(s, e0, 0);
  TORCH_CHECK(cudaMemcpyAsync(d_c.data_ptr(), c, E * 8, cudaMemcpyHostToDevice, s_in) ==
                  cudaSuccess, "count copy");
  const int64_t nch = std::max<int64_t>(1, chunks);
  int64_t e_begin = 0, row = 0;
  const int dt = dtype_code(input);
  void* ws = workspace_for(weights.device(), s_mm);
  for (int64_t ch = 0; ch < nch && e_begin < E; ++ch) {
    // next group: experts until the group holds about T / nch rows (the last takes the rest)
    int64_t e_end = e_begin, rows = 0;
    const int64_t target = (T * (ch + 1)) / nch - row;
    while (e_end < E && (rows < target || ch == nch - 1)) rows += c[e_end++];
    if (rows == 0) { e_begin = e_end; continue; }
    const char* src = static_cast<const char*>(input.data_ptr()) + row * K * esz;
    char* dx = static_cast<char*>(d_x.data_ptr()) + row * K * esz;
    char* dy = static_cast<char*>(d_y.data_ptr()) + row * N * esz;
    TORCH_CHECK(cudaMemcpyAsync(dx, src, rows * K * esz, cudaMemcpyHostToDevice, s_in) ==
                    cudaSuccess, "input copy");
    cudaStreamWaitEvent(s_mm, event(s_in), 0);
    const char* wptr = static_cast<const char*>(weights.data_ptr()) + e_begin * N * K * esz;
    const int st = ggo_grouped_gemm_segments(
        dx, wptr, dy, d_c.data_ptr<int64_t>() + e_begin, static_cast<int>(e_end - e_begin),
        static_cast<int>(e_end - e_begin), rows, N, K, dt, static_cast<int>(tile_config),
        sort_by_m ? 1 : 0, ws, s_mm);
    check_status(st, "grouped GEMM (host pipeline)");
    cudaStreamWaitEvent(s_out, event(s_mm), 0);
    char* dst = static_cast<char*>(out.data_ptr()) + row * N * esz;
    TORCH_CHECK(cudaMemcpyAsync(dst, dy, rows * N * esz, cudaMemcpyDeviceToHost, s_out) ==
                    cudaSuccess, "output copy");
    row += rows;
    e_begin = e_end;
  }
  for (cudaStream_t s : {s_in, s_mm, s_out}) cudaStreamWaitEvent(cur, event(s), 0);
  for (cudaEvent_t ev : evs) cudaEventDestroy(ev);
  // the device buffers are freed to the caching allocator on `cur`, which now waits for all
  // side-stream work, so they cannot be reused early
  return out;
}

// ------------------------------------------------------------------ expert parallelism (IPC)
// Allocates `nbytes` of device memory shareable with the other processes of the node; returns
// (address, 64-byte handle).
std::tuple<int64_t, py::bytes> ipc_alloc(int64_t nbytes) {
  void* p = nullptr;
  char h[GGO_IPC_HANDLE_BYTES];
  check_status(ggo_ipc_alloc(static_cast<size_t>(nbytes), &p, h), "IPC alloc");
  return {reinterpret_cast<int64_t>(p), py::bytes(h, GGO_IPC_HANDLE_BYTES)};
}

int64_t ipc_open(py::bytes handle) {
  std::string h = handle;
  TORCH_CHECK(h.size() == GGO_IPC_HANDLE_BYTES, "bad IPC handle size");
  void* p = nullptr;
  check_status(ggo_ipc_open(h.data(), &p), "IPC open");
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { check_status(ggo_ipc_close(reinterpret_cast<void*>(ptr)), "IPC close"); }
void ipc_free(int64_t ptr) { check_status(ggo_ipc_free(reinterpret_cast<void*>(ptr)), "IPC free"); }

// Non-owning tensor view of device memory at `ptr` (the caller keeps the memory alive).
torch::Tensor tensor_view(int64_t ptr, std::vector<int64_t> shape, torch::Dtype dtype,
                          int64_t device) {
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA,
                                                        static_cast<c10::DeviceIndex>(device));
  return torch::from_blob(reinterpret_cast<void*>(ptr), shape, opts);
}

// Expert-parallel dispatch; returns slot_pos [T*k] int32.
torch::Tensor ep_dispatch(const torch::Tensor& x, const torch::Tensor& topk_ids,
                          const torch::Tensor& scratch, const torch::Tensor& counts_all,
                          int64_t rank, std::vector<int64_t> recv_ptrs,
                          std::vector<int64_t> origin_ptrs) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "hidden must be 2D contiguous CUDA");
  TORCH_CHECK(counts_all.scalar_type() == torch::kInt64 && counts_all.dim() == 2 &&
                  counts_all.is_contiguous(), "counts_all must be contiguous int64 [world, E]");
  const int world = static_cast<int>(recv_ptrs.size());
  TORCH_CHECK(world == static_cast<int>(origin_ptrs.size()) && world == counts_all.size(0) &&
                  world <= GGO_MAX_EP_RANKS, "one receive buffer and origin buffer per rank");
  c10::cuda::CUDAGuard guard(x.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t T = x.size(0), H = x.size(1), k = topk_ids.size(1);
  auto spos = torch::empty({T * k}, torch::TensorOptions().dtype(torch::kInt32).device(x.device()));
  std::vector<void*> recv(world);
  std::vector<int32_t*> orig(world);
  for (int r = 0; r < world; ++r) {
    recv[r] = reinterpret_cast<void*>(recv_ptrs[r]);
    orig[r] = reinterpret_cast<int32_t*>(origin_ptrs[r]);
  }
  const int st = ggo_ep_dispatch(x.data_ptr(), T, H, static_cast<int>(counts_all.size(1)),
                                 static_cast<int>(k), topk_ids.data_ptr<int32_t>(),
                                 scratch.data_ptr(), counts_all.data_ptr<int64_t>(), world,
                                 static_cast<int>(rank), recv.data(), orig.data(),
                                 spos.data_ptr<int32_t>(), dtype_code(x), stream);
  check_status(st, "expert-parallel dispatch");
  return spos;
}

// Grouped GEMM over a capacity-sized receive buffer. Returns the output [capacity, N] unless the
// scatter epilogue is used (origin given), in which case results go to peer_out and an empty
// tensor is returned.
torch::Tensor ep_grouped_gemm(const torch::Tensor& input, const torch::Tensor& weights,
                              const torch::Tensor& seg_counts, int64_t num_experts, bool swiglu,
                              c10::optional<torch::Tensor> origin,
                              std::vector<int64_t> peer_out, bool sort_by_m) {
  check_operands(input, weights);
  c10::cuda::CUDAGuard guard(input.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int64_t cap = input.size(0), K = input.size(1);
  const int64_t N = swiglu ? weights.size(1) / 2 : weights.size(1);
  torch::Tensor out;
  const int32_t* org = nullptr;
  std::vector<void*> peers(peer_out.size());
  for (size_t r = 0; r < peer_out.size(); ++r) peers[r] = reinterpret_cast<void*>(peer_out[r]);
  if (origin.has_value()) {
    TORCH_CHECK(origin->scalar_type() == torch::kInt32 && origin->numel() >= cap,
                "origin must be int32 with one entry per row");
    org = origin->data_ptr<int32_t>();
    out = torch::empty({0, N}, input.options());
  } else {
    out = torch::empty({cap, N}, input.options());
  }
  if (cap == 0) return out;
  auto c = counts_on_device(seg_counts, input.device());
  const int st = ggo_ep_grouped_gemm(
      input.data_ptr(), weights.data_ptr(), org ? nullptr : out.data_ptr(),
      c.data_ptr<int64_t>(), static_cast<int>(c.size(0)), static_cast<int>(num_experts), cap, N,
      K, dtype_code(input), swiglu ? 1 : 0, org, peers.data(), static_cast<int>(peers.size()),
      sort_by_m ? 1 : 0, workspace_for(input.device(), stream), stream);
  check_status(st, "expert-parallel grouped GEMM");
  return out;
}

// ------------------------------------------------------------------ EP device-side signalling
std::vector<int64_t*> board_ptrs(const std::vector<int64_t>& v) {
  std::vector<int64_t*> out(v.size());
  for (size_t i = 0; i < v.size(); ++i) out[i] = reinterpret_cast<int64_t*>(v[i]);
  return out;
}

void ep_publish_counts(const torch::Tensor& tpe, std::vector<int64_t> boards, int64_t rank,
                       int64_t slot, int64_t epoch) {
  TORCH_CHECK(tpe.is_cuda() && tpe.scalar_type() == torch::kInt64 && tpe.is_contiguous(),
              "tokens_per_expert must be contiguous int64 CUDA");
  c10::cuda::CUDAGuard guard(tpe.device());
  auto b = board_ptrs(boards);
  check_status(ggo_ep_publish_counts(tpe.data_ptr<int64_t>(), b.data(),
                                     static_cast<int>(b.size()), static_cast<int>(rank),
                                     static_cast<int>(tpe.numel()), static_cast<int>(slot), epoch,
                                     at::cuda::getCurrentCUDAStream()),
               "EP count publish");
}

void ep_signal(std::vector<int64_t> boards, int64_t rank, int64_t num_experts, int64_t slot,
               int64_t epoch, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  auto b = board_ptrs(boards);
  check_status(ggo_ep_signal(b.data(), static_cast<int>(b.size()), static_cast<int>(rank),
                             static_cast<int>(num_experts), static_cast<int>(slot), epoch,
                             at::cuda::getCurrentCUDAStream()),
               "EP signal");
}

void ep_wait(int64_t own_board, int64_t world, int64_t num_experts, int64_t slot, int64_t epoch,
             int64_t limit_cycles, int64_t device) {
  const torch::Device dev(torch::kCUDA, static_cast<c10::DeviceIndex>(device));
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(ggo_ep_wait(reinterpret_cast<const int64_t*>(own_board), static_cast<int>(world),
                           static_cast<int>(num_experts), static_cast<int>(slot), epoch,
                           workspace_for(dev, stream), limit_cycles, stream),
               "EP wait");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("grouped_gemm_opt_forward", &grouped_gemm_forward,
        "Persistent tcgen05 grouped GEMM for MoE (sm_100a)", py::arg("input"),
        py::arg("weights"), py::arg("tokens_per_expert"), py::arg("tile_config") = 4,
        py::arg("sort_by_m") = true);
  m.def("grouped_gemm_segments", &grouped_gemm_segments, py::arg("input"), py::arg("weights"),
        py::arg("tokens_per_segment"), py::arg("num_experts"), py::arg("tile_config") = 4,
        py::arg("sort_by_m") = true);
  m.def("grouped_gemm_dgrad", &grouped_gemm_dgrad, py::arg("dy"), py::arg("weights"),
        py::arg("tokens_per_expert"), py::arg("tile_config") = 4, py::arg("sort_by_m") = true);
  m.def("grouped_gemm_wgrad", &grouped_gemm_wgrad, py::arg("x"), py::arg("dy"),
        py::arg("tokens_per_expert"), py::arg("sort_by_m") = true);
  m.def("quantize_fp8_rows", &quantize_fp8_rows, py::arg("x"));
  m.def("quantize_mxfp8", &quantize_mxfp8, py::arg("x"), py::arg("counts"));
  m.def("grouped_gemm_mxfp8", &grouped_gemm_mxfp8, py::arg("input_q"), py::arg("input_scale"),
        py::arg("weights_q"), py::arg("weight_scale"), py::arg("counts"), py::arg("num_experts"),
        py::arg("sort_by_m") = true);
  m.def("grouped_gemm_swiglu_mxfp8", &grouped_gemm_swiglu_mxfp8, py::arg("x_q"),
        py::arg("x_scale"), py::arg("w_q"), py::arg("w_scale"), py::arg("counts"),
        py::arg("num_experts"), py::arg("F"), py::arg("sort_by_m") = true);
  m.def("mxfp8_glu_rows", [](int64_t f) { return ggo_mxfp8_glu_rows(f); });
  m.def("mxfp8_scale_bytes", [](int64_t rows, int64_t nseg, int64_t k) {
    return static_cast<int64_t>(ggo_mxfp8_scale_bytes(rows, static_cast<int>(nseg), k));
  });
  m.def("grouped_gemm_swiglu_fp8", &grouped_gemm_swiglu_fp8, py::arg("x_q"), py::arg("x_scale"),
        py::arg("w_gate_up_q"), py::arg("w_scale"), py::arg("tokens_per_segment"),
        py::arg("num_experts"), py::arg("sort_by_m") = true);
  m.def("grouped_gemm_fp8", &grouped_gemm_fp8, py::arg("input_q"), py::arg("input_scale"),
        py::arg("weights_q"), py::arg("weight_scale"), py::arg("tokens_per_expert"),
        py::arg("tile_config") = 4, py::arg("sort_by_m") = true);
  m.def("grouped_gemm_swiglu", &grouped_gemm_swiglu, py::arg("x"), py::arg("w_gate_up"),
        py::arg("tokens_per_segment"), py::arg("num_experts"), py::arg("sort_by_m") = true);
  m.def("moe_route", &moe_route, py::arg("router_logits"), py::arg("top_k"));
  m.def("moe_permute", &moe_permute, py::arg("hidden"), py::arg("topk_ids"), py::arg("scratch"),
        py::arg("num_experts"));
  m.def("moe_combine", &moe_combine, py::arg("y_sorted"), py::arg("topk_weights"),
        py::arg("slot_pos"), py::arg("checked") = false);
  m.def("workspace_error", &workspace_error, py::arg("device") = 0);
  m.def("abi_version", []() { return ggo_version(); });
  m.def("kernel_launches", []() { return static_cast<int64_t>(ggo_kernel_launches()); });
  m.def("grouped_gemm_host", &grouped_gemm_host, py::arg("input"), py::arg("weights"),
        py::arg("tokens_per_expert"), py::arg("out"), py::arg("tile_config") = 4,
        py::arg("sort_by_m") = true, py::arg("chunks") = 4);
  m.def("ep_board_bytes", [](int64_t e) { return static_cast<int64_t>(ggo_ep_board_bytes(static_cast<int>(e))); });
  m.def("ep_publish_counts", &ep_publish_counts, py::arg("tokens_per_expert"), py::arg("boards"),
        py::arg("rank"), py::arg("slot"), py::arg("epoch"));
  m.def("ep_signal", &ep_signal, py::arg("boards"), py::arg("rank"), py::arg("num_experts"),
        py::arg("slot"), py::arg("epoch"), py::arg("device"));
  m.def("ep_wait", &ep_wait, py::arg("own_board"), py::arg("world"), py::arg("num_experts"),
        py::arg("slot"), py::arg("epoch"), py::arg("limit_cycles"), py::arg("device"));
  m.def("ipc_alloc", &ipc_alloc, py::arg("nbytes"));
  m.def("ipc_open", &ipc_open, py::arg("handle"));
  m.def("ipc_close", &ipc_close, py::arg("ptr"));
  m.def("ipc_free", &ipc_free, py::arg("ptr"));
  m.def("tensor_view", &tensor_view, py::arg("ptr"), py::arg("shape"), py::arg("dtype"),
        py::arg("device"));
  m.def("ep_dispatch", &ep_dispatch, py::arg("hidden"), py::arg("topk_ids"), py::arg("scratch"),
        py::arg("counts_all"), py::arg("rank"), py::arg("recv_ptrs"), py::arg("origin_ptrs"));
  m.def("ep_grouped_gemm", &ep_grouped_gemm, py::arg("input"), py::arg("weights"),
        py::arg("seg_counts"), py::arg("num_experts"), py::arg("swiglu"), py::arg("origin"),
        py::arg("peer_out"), py::arg("sort_by_m") = true);
}
