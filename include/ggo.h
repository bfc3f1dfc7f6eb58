/*
 * ggo.h - C ABI of the B200-native (sm_100a) MoE grouped-GEMM library.
 *
 * Plain pointers, sizes and a cudaStream_t; no PyTorch types. Every pointer argument named
 * *_dev is device memory. Every call is stream-ordered on `stream` and never synchronises the
 * host unless its comment says so. Return value: GGO_OK (0) or one of the GGO_ERR_* codes;
 * ggo_status_string() turns a code into a message.
 *
 * Reference interfaces these entry points replace (paths inside jeshxxx/GroupedGEMM-OPT):
 *   csrc/grouped_gemm.h:21-26          grouped_gemm::grouped_gemm_forward
 *   csrc/grouped_gemm_kernel.cu:348-450 host dispatch (count copy, zero filter, tile choice)
 *   csrc/grouped_gemm_kernel.cu:195-279 launch_grouped_gemm<Kernel> (CUTLASS device adapter)
 *   csrc/torch_ext.cpp:19-27           pybind grouped_gemm_opt_forward
 *   grouped_gemm_opt/triton_fused_moe.py:104-150  the fused-MoE entry point
 */
#ifndef GGO_H_
#define GGO_H_

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ----------------------------------------------------------------- status codes */
#define GGO_OK 0
#define GGO_ERR_INVALID_ARG 1     /* null pointer, negative size, bad enum value          */
#define GGO_ERR_SHAPE 2           /* K mismatch / dimension out of the supported range     */
#define GGO_ERR_DTYPE 3           /* dtype other than GGO_DTYPE_BF16 / GGO_DTYPE_FP16      */
#define GGO_ERR_ALIGNMENT 4       /* pointer not 16-B aligned, K or N not a multiple of 8  */
#define GGO_ERR_TOO_MANY_SEGMENTS 5 /* num_segments > GGO_MAX_SEGMENTS                     */
#define GGO_ERR_CUDA 6            /* a CUDA runtime/driver call failed                     */
#define GGO_ERR_NO_DEVICE 7       /* device is not sm_100 (B200 class)                     */
#define GGO_ERR_DEVICE_TIMEOUT 8  /* a kernel's bounded wait expired (read back by ggo_workspace_error) */
#define GGO_ERR_COUNT_MISMATCH 9  /* sum(tokens_per_expert) != total_tokens (detected on device) */
#define GGO_ERR_NEGATIVE_COUNT 10 /* a token count was negative (detected on device)       */

#define GGO_DTYPE_BF16 0
#define GGO_DTYPE_FP16 1

#define GGO_MAX_SEGMENTS 1024
#define GGO_WORKSPACE_BYTES 256

/* TileConfig values, identical to the reference enum (csrc/grouped_gemm.h:8-19,
 * grouped_gemm_opt/ops.py:23-28). On sm_100a they select:
 *   0 Co_128x128x64  -> single-CTA 128x128 tcgen05 tile, 6-stage TMA ring
 *   1 Co_128x256x64  -> single-CTA 128x256 tile, 4-stage ring
 *   2 PP_128x128x128 -> single-CTA 128x128 tile (as 0)
 *   3 PP_128x256x64  -> CTA pair (cta_group::2), 256x256 tile, 6-stage ring, plus a single-CTA
 *                       pass over short segment tails when they fill two waves
 *   4 AUTO           -> device-free choice: 128x128 when wider tiles leave SMs idle, the CTA pair
 *                       when segments average >= 192 rows, else 128x256
 *   5 CuBLAS_Seq     -> accepted for API compatibility; runs the AUTO choice (no library GEMM) */
#define GGO_TILE_CO_128x128x64 0
#define GGO_TILE_CO_128x256x64 1
#define GGO_TILE_PP_128x128x128 2
#define GGO_TILE_PP_128x256x64 3
#define GGO_TILE_AUTO 4
#define GGO_TILE_CUBLAS_SEQ 5

/* After a call returned GGO_ERR_CUDA: the CUDA error it met, as text (this thread's last). */
const char* ggo_last_cuda_error_string(void);

/* Number of kernels this library has launched in this process (for launch accounting). */
uint64_t ggo_kernel_launches(void);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int ggo_version(void);

/* Human-readable message for a status code (static storage, never NULL). */
const char* ggo_status_string(int status);

/* Bytes of scratch one in-flight call needs (GGO_WORKSPACE_BYTES). The caller allocates it in
 * device memory, zero-fills it ONCE, and reuses it for every later call on the same stream; calls
 * that may run concurrently (different streams) need distinct workspaces. */
size_t ggo_workspace_size(void);

/* Grouped GEMM, the replacement of grouped_gemm::grouped_gemm_forward
 * (reference csrc/grouped_gemm.h:21-26, csrc/grouped_gemm_kernel.cu:348-450):
 *
 *   output[r, :] = input[r, :] @ weights[e(r)]^T
 *
 * input_dev   [total_tokens, K]   row-major, rows sorted by expert
 * weights_dev [num_experts, N, K] row-major (torch.nn.Linear layout per expert)
 * output_dev  [total_tokens, N]   written for every row that belongs to an expert
 * tokens_per_expert_dev [num_experts] int64, DEVICE memory: read only by the kernel, so the host
 *             never waits for it (the reference copies it to the host and synchronises).
 * Experts with zero tokens are skipped on the device with no weight copy. sum(tokens) must equal
 * total_tokens; a mismatch is recorded in the workspace (GGO_ERR_COUNT_MISMATCH via
 * ggo_workspace_error) and rows outside [0, total_tokens) are never read or written.
 * K and N must be multiples of 8; pointers 16-byte aligned. */
int ggo_grouped_gemm(const void* input_dev, const void* weights_dev, void* output_dev,
                     const int64_t* tokens_per_expert_dev, int num_experts, int64_t total_tokens,
                     int64_t N, int64_t K, int dtype, int tile_config, int sort_by_m,
                     void* workspace_dev, cudaStream_t stream);

/* Generalised form used by expert parallelism: `num_segments` contiguous row segments, segment s
 * multiplied by expert (s % num_experts). With num_segments == num_experts it equals
 * ggo_grouped_gemm. After an all-to-all the received rows are [source rank][local expert], i.e.
 * exactly this layout with num_segments = world_size * local_experts. No reference counterpart
 * (the reference is single-device). */
int ggo_grouped_gemm_segments(const void* input_dev, const void* weights_dev, void* output_dev,
                              const int64_t* tokens_per_segment_dev, int num_segments,
                              int num_experts, int64_t total_tokens, int64_t N, int64_t K,
                              int dtype, int tile_config, int sort_by_m, void* workspace_dev,
                              cudaStream_t stream);

/* Backward, input gradient of the grouped GEMM (no reference counterpart: the reference is
 * forward-only):
 *   dx[r, :] = dy[r, :] @ weights[e(r)]        dy [T, N], weights [E, N, K], dx [T, K]
 * The weights are read in place (MN-major operand), no transposed copy. Same segment, count and
 * alignment rules as ggo_grouped_gemm; tile_config as there. */
int ggo_grouped_gemm_dgrad(const void* dy_dev, const void* weights_dev, void* dx_dev,
                           const int64_t* tokens_per_expert_dev, int num_experts,
                           int64_t total_tokens, int64_t N, int64_t K, int dtype, int tile_config,
                           int sort_by_m, void* workspace_dev, cudaStream_t stream);

/* Backward, weight gradient (no reference counterpart):
 *   dw[e] = dy_e^T @ x_e        x [T, K], dy [T, N], dw [E, N, K]
 * where x_e, dy_e are expert e's rows (segments given by tokens_per_expert, on the device). The
 * reduction runs over each expert's own tokens; experts with no tokens get dw[e] = 0. Both
 * operands are read in place. N and K multiples of 8. */
int ggo_grouped_gemm_wgrad(const void* x_dev, const void* dy_dev, void* dw_dev,
                           const int64_t* tokens_per_expert_dev, int num_experts,
                           int64_t total_tokens, int64_t N, int64_t K, int dtype, int sort_by_m,
                           void* workspace_dev, cudaStream_t stream);

/* FP8 grouped GEMM (no reference counterpart; the reference is bf16/fp16 only):
 *   out[r, n] = (sum_k a[r,k] * b[e(r),n,k]) * input_scale[r] * weight_scale[e(r), n]   (bf16)
 * input_dev [T, K] and weights_dev [E, N, K] are e4m3 bytes (tcgen05 kind::f8f6f4, fp32
 * accumulation); input_scale_dev [T] and weight_scale_dev [E, N] fp32 (see
 * ggo_quantize_fp8_rows). K a multiple of 16, N of 8. Same segment rules as ggo_grouped_gemm. */
int ggo_grouped_gemm_fp8(const void* input_dev, const float* input_scale_dev,
                         const void* weights_dev, const float* weight_scale_dev, void* output_dev,
                         const int64_t* tokens_per_expert_dev, int num_experts,
                         int64_t total_tokens, int64_t N, int64_t K, int tile_config,
                         int sort_by_m, void* workspace_dev, cudaStream_t stream);

/* FP8 gate/up grouped GEMM with the SwiGLU epilogue (no reference counterpart):
 *   h[r, f] = silu(g * s_x[r] * s_w[e, f]) * (u * s_x[r] * s_w[e, F + f])  (bf16 out)
 * with g / u the e4m3 dot products of x row r with weight rows f / F + f. x [T, K] and
 * w_gate_up [E, 2F, K] e4m3; x_scale [T], w_scale [E, 2F] fp32. Segment semantics as
 * ggo_grouped_gemm_segments. K a multiple of 16, F of 8. */
int ggo_grouped_gemm_swiglu_fp8(const void* x_dev, const float* x_scale_dev,
                                const void* w_gate_up_dev, const float* w_scale_dev, void* h_dev,
                                const int64_t* tokens_per_segment_dev, int num_segments,
                                int num_experts, int64_t total_tokens, int64_t F, int64_t K,
                                int sort_by_m, void* workspace_dev, cudaStream_t stream);

/* Row-wise e4m3 quantisation of a bf16/fp16 matrix [rows, cols]: scale_dev[r] =
 * max|x[r,:]| / 448 (1 for an all-zero row), q_dev[r,c] = e4m3(x[r,c] / scale[r]) rounded to
 * nearest with saturation. Weights [E, N, K] quantise per output channel as rows = E*N.
 * cols a multiple of 16. */
int ggo_quantize_fp8_rows(const void* x_dev, int64_t rows, int64_t cols, int dtype, void* q_dev,
                          float* scale_dev, cudaStream_t stream);

/* MXFP8: block-scaled e4m3 in the OCP MX layout (no reference counterpart). Every 32 consecutive
 * K elements of a row share one UE8M0 scale 2^(byte - 127); the tensor cores apply both operands'
 * scales (tcgen05 kind::mxf8f6f4.block_scale) and accumulate in fp32. The GEMMs accept any UE8M0
 * scales; ggo_quantize_mxfp8 picks them with a non-saturating rule (below) that differs from the
 * OCP MX v1.0 reference rule (floor(log2 amax) - emax, then clamping), so its scale bytes can
 * differ from other MX producers' by one. The MXFP8 GEMMs always run 256 x 256 CTA-pair tiles:
 * they take no tile configuration.
 * Scale layout ("128x4 blocked"): the rows of each segment start a fresh 128-row block after the
 * blocks of the previous segments; block b and K group g (128 elements, 4 scales) form the 512-B
 * atom at byte (b * K/128 + g) * 512, inside which row r (0..127) and scale j (0..3) of the group
 * sit at byte (r % 32) * 16 + (r / 32) * 4 + j. Weights [E, N, K] are E segments of N rows. */

/* Bytes of the scale buffer for `rows` rows in `num_segments` segments, K columns (an upper bound
 * that needs no counts: ceil(rows / 128) + num_segments blocks). 0 if K is not a multiple of 128. */
size_t ggo_mxfp8_scale_bytes(int64_t rows, int num_segments, int64_t k);

/* MX quantisation of a bf16/fp16 matrix [rows, k] whose rows form consecutive segments of
 * counts_dev[s] rows (device int64; weights: num_segments = E, every count N). Per 32-element
 * group: X = floor(log2 amax) - 8, plus 1 when amax / 2^floor(log2 amax) > 1.75, clamped to
 * [-127, 127] (-127 for an all-zero group); scale byte X + 127; q = e4m3(x * 2^-X), round to
 * nearest even. q_dev [rows, k] e4m3 bytes; scale_dev ggo_mxfp8_scale_bytes() bytes (padding
 * bytes are left as they were). k a multiple of 128, at most 1024 segments. */
int ggo_quantize_mxfp8(const void* x_dev, int dtype, const int64_t* counts_dev, int num_segments,
                       int64_t rows, int64_t k, void* q_dev, void* scale_dev,
                       cudaStream_t stream);

/* MXFP8 grouped GEMM: out[r, n] = sum_k (a[r,k] 2^sa[r,k/32]) (b[e,n,k] 2^sb[e,n,k/32]) in bf16.
 * input_dev [T, K] and weights_dev [E, N, K] e4m3 with their scales from ggo_quantize_mxfp8
 * (the input quantised with these same segment counts). Segment s multiplies expert
 * s % num_experts. K a multiple of 128, N of 8. Runs 256 x 256 CTA-pair tiles. */
int ggo_grouped_gemm_mxfp8(const void* input_dev, const void* input_scale_dev,
                           const void* weights_dev, const void* weight_scale_dev, void* output_dev,
                           const int64_t* tokens_per_segment_dev, int num_segments,
                           int num_experts, int64_t total_tokens, int64_t N, int64_t K,
                           int sort_by_m, void* workspace_dev, cudaStream_t stream);

/* Rows per expert of the blocked gate/up weight the MXFP8 SwiGLU GEMM reads: 2 * F_pad with
 * F_pad = F rounded up to 128. Block j (rows 256j .. 256j+255) holds gate rows 128j .. 128j+127
 * then the matching up rows; rows past F are zero. */
int64_t ggo_mxfp8_glu_rows(int64_t F);

/* MXFP8 gate/up GEMM with the SwiGLU epilogue: h[r, f] = silu(g) * u, g / u the block-scaled
 * products of x row r with gate / up row f. w_gate_up_dev [E, ggo_mxfp8_glu_rows(F), K] e4m3 in the
 * blocked layout above, quantised as E segments of ggo_mxfp8_glu_rows(F) rows. h_dev [T, F] bf16. */
int ggo_grouped_gemm_swiglu_mxfp8(const void* x_dev, const void* x_scale_dev,
                                  const void* w_gate_up_dev, const void* w_scale_dev, void* h_dev,
                                  const int64_t* tokens_per_segment_dev, int num_segments,
                                  int num_experts, int64_t total_tokens, int64_t F, int64_t K,
                                  int sort_by_m, void* workspace_dev, cudaStream_t stream);

/* Fused-MoE stage 2: gate/up grouped GEMM with the SwiGLU epilogue.
 *   h[r, f] = silu(x[r,:] . Wgu[e, f, :]) * (x[r,:] . Wgu[e, F + f, :])
 * w_gate_up_dev [num_experts, 2F, K]: rows 0..F-1 gate, rows F..2F-1 up.
 * h_dev [total_tokens, F]. Segment semantics as ggo_grouped_gemm_segments. F multiple of 8.
 * Replaces the GEMM of grouped_gemm_opt/triton_fused_moe.py:16-78 plus the activation that the
 * reference leaves to the caller. */
int ggo_grouped_gemm_swiglu(const void* x_dev, const void* w_gate_up_dev, void* h_dev,
                            const int64_t* tokens_per_segment_dev, int num_segments,
                            int num_experts, int64_t total_tokens, int64_t F, int64_t K, int dtype,
                            int sort_by_m, void* workspace_dev, cudaStream_t stream);

/* Fused-MoE stage 1a: router. For every token t: the top_k largest logits (ties -> lower expert
 * index), softmax over those k values (fp32), written as topk_ids [T, top_k] int32 and
 * topk_weights [T, top_k] fp32, in descending-logit order. Also writes tokens_per_expert [E]
 * int64. logits fp32 [T, E]. E <= 1024, top_k <= 16, top_k <= E.
 * block_counts_dev needs ggo_moe_route_scratch_bytes(T, E) bytes. No reference counterpart. */
size_t ggo_moe_route_scratch_bytes(int64_t num_tokens, int num_experts);
int ggo_moe_route(const float* logits_dev, int64_t num_tokens, int num_experts, int top_k,
                  int32_t* topk_ids_dev, float* topk_weights_dev,
                  int64_t* tokens_per_expert_dev, void* scratch_dev, cudaStream_t stream);

/* Fused-MoE stage 1b: permute. Sorted order is expert-major, then token index (each token's k
 * experts are distinct, so the k-slot never ties). Writes
 *   x_sorted [T*top_k, H]  the gathered hidden rows,
 *   sorted_token [T*top_k] int32, the source token of each sorted row,
 *   slot_pos [T*top_k] int32, the sorted row of (token t, slot j) at index t*top_k + j.
 * Must be called with the scratch written by ggo_moe_route on the same stream. Deterministic
 * (no atomics on positions): bit-exact against any stable counting sort. */
int ggo_moe_permute(const void* x_dev, int64_t num_tokens, int64_t hidden, int num_experts,
                    int top_k, const int32_t* topk_ids_dev, void* x_sorted_dev,
                    int32_t* sorted_token_dev, int32_t* slot_pos_dev, void* scratch_dev,
                    int dtype, cudaStream_t stream);

/* Fused-MoE stage 4: top-k weighted combine.
 *   out[t, :] = sum_{j < top_k} topk_weights[t, j] * y_sorted[slot_pos[t*top_k + j], :]
 * accumulated in fp32 in fixed j order, rounded once to bf16/fp16. No atomics. */
int ggo_moe_combine(const void* y_sorted_dev, const float* topk_weights_dev,
                    const int32_t* slot_pos_dev, int64_t num_tokens, int64_t hidden, int top_k,
                    void* out_dev, int dtype, cudaStream_t stream);

/* ggo_moe_combine that refuses to hand back a result built from incomplete data: when the
 * workspace error word (see ggo_workspace_error) is non-zero as the kernel runs -- e.g. an
 * expert-parallel peer wait expired, so the receive/return buffers may hold a previous layer's
 * rows -- every output element is written as NaN instead. No host synchronisation. No reference
 * counterpart (the reference is single-device). */
int ggo_moe_combine_checked(const void* y_sorted_dev, const float* topk_weights_dev,
                            const int32_t* slot_pos_dev, int64_t num_tokens, int64_t hidden,
                            int top_k, void* out_dev, int dtype, const void* workspace_dev,
                            cudaStream_t stream);

/* ----------------------------------------------------------------- expert parallelism
 * The fused expert-parallel path over NVLink peer memory. None of these has a counterpart in the
 * reference, which is single-device. Buffers are shared between the ranks of one node through
 * CUDA IPC (ggo_ipc_*): every rank allocates its receive buffers, exchanges the 64-byte handles
 * (e.g. with an all_gather of bytes) and opens its peers' handles; kernels then load and store
 * peer memory directly. Ordering between ranks is the caller's: a collective (e.g. a one-element
 * NCCL all-reduce) after ggo_ep_dispatch and after the scattering GEMM. */
#define GGO_IPC_HANDLE_BYTES 64
#define GGO_MAX_EP_RANKS 8

/* cudaMalloc `bytes` and return its IPC handle (GGO_IPC_HANDLE_BYTES bytes into handle_out). */
int ggo_ipc_alloc(size_t bytes, void** ptr_out, void* handle_out);
/* Map a peer's buffer from its handle (peer access enabled lazily). */
int ggo_ipc_open(const void* handle, void** ptr_out);
int ggo_ipc_close(void* peer_ptr);
int ggo_ipc_free(void* ptr);

/* Expert-parallel dispatch: ggo_moe_permute that writes every routed row straight into the
 * receive buffer of the rank owning its expert (rank r owns experts [r*E/P, (r+1)*E/P)).
 * counts_all_dev [P, E] int64: every rank's tokens_per_expert (e.g. an all_gather of them).
 * recv_rows[r] / recv_origin[r]: rank r's receive rows [capacity, H] and origin [capacity] int32,
 * as mapped in this process (own buffers for r == rank). Received rows are laid out
 * expert-major, [local expert][source rank], so each local expert is one contiguous segment;
 * recv_origin holds (source rank << 28) | the row's sorted position on its source rank.
 * slot_pos_dev as in ggo_moe_permute. */
int ggo_ep_dispatch(const void* x_dev, int64_t num_tokens, int64_t hidden, int num_experts,
                    int top_k, const int32_t* topk_ids_dev, const void* scratch_dev,
                    const int64_t* counts_all_dev, int world_size, int rank,
                    void* const* recv_rows, int32_t* const* recv_origin, int32_t* slot_pos_dev,
                    int dtype, cudaStream_t stream);

/* Device-side signalling between the ranks of the fused expert-parallel path, replacing host
 * collectives. Every rank allocates a sync board of ggo_ep_board_bytes(E) bytes (zero-filled,
 * IPC-shared): counts [8][E] int64 (row r = rank r's tokens_per_expert) and flags [4][8] int64
 * (per phase slot, the last epoch each rank completed). boards[r] = rank r's board as mapped here.
 * Epochs must grow from layer to layer (start at 1).
 *   ggo_ep_publish_counts: write this rank's tokens_per_expert into every board, then post
 *                          `epoch` for `slot`.
 *   ggo_ep_signal:         post `epoch` for `slot` (after the peer stores of earlier kernels on
 *                          `stream`, which must end with a system-scope fence).
 *   ggo_ep_wait:           wait until every rank posted `epoch` for `slot` on this rank's board;
 *                          bounded by limit_cycles (SM clock), after which the workspace error
 *                          word records GGO_ERR_DEVICE_TIMEOUT (read it with ggo_workspace_error).
 *                          A wait that finds the error word already set returns at once, so one
 *                          expired wait does not make every later phase wait out its limit too. */
size_t ggo_ep_board_bytes(int num_experts);
int ggo_ep_publish_counts(const int64_t* tokens_per_expert_dev, int64_t* const* boards,
                          int world_size, int rank, int num_experts, int slot, int64_t epoch,
                          cudaStream_t stream);
int ggo_ep_signal(int64_t* const* boards, int world_size, int rank, int num_experts, int slot,
                  int64_t epoch, cudaStream_t stream);
int ggo_ep_wait(const int64_t* own_board, int world_size, int num_experts, int slot,
                int64_t epoch, void* workspace_dev, int64_t limit_cycles, cudaStream_t stream);

/* Grouped GEMM over a receive buffer of capacity_rows rows whose segment counts (device) may sum
 * to less. swiglu != 0: the gate/up SwiGLU form (N = F, weights [E, 2F, K]). With origin_dev set
 * (scatter epilogue), row r's result is stored to peer_out[origin_dev[r] >> 28] +
 * (origin_dev[r] & 0x0fffffff) * N, i.e. straight back to the source rank's buffer over
 * NVLink, and output_dev may be NULL. world_size = number of peer_out entries. */
int ggo_ep_grouped_gemm(const void* input_dev, const void* weights_dev, void* output_dev,
                        const int64_t* tokens_per_segment_dev, int num_segments, int num_experts,
                        int64_t capacity_rows, int64_t N, int64_t K, int dtype, int swiglu,
                        const int32_t* origin_dev, void* const* peer_out, int world_size,
                        int sort_by_m, void* workspace_dev, cudaStream_t stream);

/* Grouped GEMM that allocates nothing: same arguments, result and validation as
 * ggo_grouped_gemm, minus the workspace. It has no counterpart in the reference; it exists for
 * callers that cannot call cudaMalloc themselves or hand over a buffer -- code running while a
 * custom allocator must not be re-entered, plugins and hosts that give a kernel library no
 * allocator, or code that owns no device memory at all.
 * Its scratch is a fixed file-scope device array of GGO_WORKSPACE_BYTES (256 B) inside this
 * library, held by every GPU that loads the library until the process exits. That scratch covers
 * any problem with at most GGO_NOALLOC_MAX_EXPERTS experts; more experts are rejected with
 * GGO_ERR_TOO_MANY_SEGMENTS. The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call before any stream capture on that device.
 * Every call shares the one array and clears it on `stream` before its launch, so calls that
 * may overlap on the GPU (different streams, or other host threads) race and must be serialised
 * by the caller. Device-side errors (count mismatch, bounded-wait timeout) are not reported by
 * this entry point: the next call clears them. Calls no cudaMalloc, cudaFree or allocating
 * library routine. */
#define GGO_NOALLOC_MAX_EXPERTS GGO_MAX_SEGMENTS
int ggo_grouped_gemm_noalloc(const void* input_dev, const void* weights_dev, void* output_dev,
                             const int64_t* tokens_per_expert_dev, int num_experts,
                             int64_t total_tokens, int64_t N, int64_t K, int dtype,
                             int tile_config, int sort_by_m, cudaStream_t stream);

/* Reads (and clears) the sticky device error of a workspace. Synchronises `stream`.
 * Writes GGO_OK or a GGO_ERR_* code to *status_out. */
int ggo_workspace_error(void* workspace_dev, cudaStream_t stream, int* status_out);

#ifdef __cplusplus
}
#endif

#endif /* GGO_H_ */
