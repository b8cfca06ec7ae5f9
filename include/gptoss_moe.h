/*
 * gptoss_moe.h - C ABI of the B200 (sm_100a) GPT-OSS MXFP4 W4A8 mixture-of-experts
 * expert path (libgptoss_moe.so).
 *
 * Conventions for every entry point
 *   - Pointers are device pointers unless a parameter says "host".
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Work is enqueued on it;
 *     no entry point synchronises the stream unless its comment says so.
 *   - Return 0 on success, or a GPTOSS_ERR_* code; gptoss_last_error() then returns a
 *     message for the calling thread. No C++ exception crosses this boundary.
 *   - Tensors are dense and row-major ("contiguous"); shapes are given in elements.
 *   - FP8 activations are float8_e4m3fn bytes; MXFP4 weights are two E2M1 codes per
 *     byte (low nibble = even k); scales are UE8M0 bytes (value 2^(s-127)), one per 32
 *     consecutive k.
 *   - "Blocked" scales use the 128-row x 4-group atom layout of CUTLASS's
 *     Sm1xxBlockScaledConfig<32>::tile_atom_to_shape_SFA/SFB:
 *       off(r, g) = (r/128)*(G4*512) + (g/4)*512 + (r%32)*16 + ((r%128)/32)*4 + g%4
 *     with G4 = ceil(groups/4); a buffer for `rows` rows holds ceil(rows/128)*G4*512 bytes.
 *
 * Reference interfaces replaced are cited as path:line of evil0sheep/gpt-oss-mxfp4-compile.
 */
#ifndef GPTOSS_MOE_H
#define GPTOSS_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  GPTOSS_OK = 0,
  GPTOSS_ERR_INVALID_ARGUMENT = 1, /* bad shape / dtype / alignment (TORCH_CHECK in the reference) */
  GPTOSS_ERR_CUDA = 2,             /* a CUDA runtime or driver call failed */
  GPTOSS_ERR_NOT_IMPLEMENTED = 3,  /* a mode this build does not provide */
  GPTOSS_ERR_UNSUPPORTED_DEVICE = 4, /* not a compute-capability 10.x GPU */
  GPTOSS_ERR_WORKSPACE = 5         /* workspace smaller than gptoss_*_workspace_bytes() */
};

enum { GPTOSS_DTYPE_BF16 = 0, GPTOSS_DTYPE_F32 = 1 };

/* GEMM orientation: SWAP puts the weights on the MMA M side and multiplies 16-row
 * activation chunks; SWAP_WIDE does the same with 64-row chunks (16/32/64-row loads);
 * TOKENS_M puts the tokens on M. AUTO picks SWAP while the average expert holds <= 12
 * rows, SWAP_WIDE up to 80, else TOKENS_M (gptoss_fp4_group_mm: SWAP_WIDE up to 48).
 * Results agree to fp32 accumulation order. The stages of one forward (route_quant,
 * gemm1, gemm2) must be called with the same mode: it also selects the row layout of
 * the activation scales in the workspace. */
enum { GPTOSS_GEMM_AUTO = 0, GPTOSS_GEMM_TOKENS_M = 1, GPTOSS_GEMM_SWAP = 2, GPTOSS_GEMM_SWAP_WIDE = 3 };

/* The orientation a fused forward over `rows` assignments and `num_experts` experts runs
 * with for `gemm_mode` (AUTO resolved): GPTOSS_GEMM_TOKENS_M / _SWAP / _SWAP_WIDE, or -1 for
 * bad arguments. Host only. No counterpart in the reference. */
int gptoss_moe_gemm_layout(int gemm_mode, int64_t rows, int num_experts);

/* Message for the last failing call on this thread ("" if none). */
const char* gptoss_last_error(void);

/* ABI version of this header (bumped on any signature change; 2: gptoss_mma_peak takes a kind). */
int gptoss_abi_version(void);

/* Kernels this library has launched in this process, on every device (launch accounting
 * for benchmarks; no counterpart in the reference). */
uint64_t gptoss_kernel_launch_count(void);

/* Decode-sized fused forwards (gptoss_moe_layer_forward, gptoss_moe_experts_forward and
 * the no-allocation forward with at most 64 tokens, 256 assignments and 128 experts, on
 * the SWAP orientation) run as one persistent launch that streams the expert weights from
 * its first cycle and computes the routing on its idle warps (plus a one-CTA launch that
 * clears its synchronisation words). Its CTAs wait on each other, so it expects the whole
 * GPU (one CTA per SM). enable = 0 selects the three-launch path (routing prologue, GEMM1,
 * GEMM2) for those batches instead; outputs agree within the combine's bf16 atomics.
 * Process-wide; returns the previous setting. No counterpart in the reference. */
int gptoss_set_decode_layer_kernel(int enable);

/* Copies the 4-byte device status word that kernels set when a bounded wait times out
 * (0x101-0x104 GEMM roles, 0x106-0x108 the one-launch kernels, 0x301 a peer's flag), an
 * expert index is out of range (0x201) or an expert's scale offset is not 16-byte aligned
 * (0x109) -- 0 = ok -- into *status_host and clears it. Synchronises `stream`. */
int gptoss_read_status(int32_t* status_dev, int32_t* status_host, void* stream);

/* Replaces fused_moe_routing (kernels/matmul_mxfp4_cutlass.cu:1041-1095, registered as
 * cutlass::fused_moe_routing at kernels/cutlass_experts.py:168-188).
 * router_indices [T, top_k] int64, routing_weights [T, top_k] f32 ->
 * sorted_token_idx [T*top_k] int64, sorted_expert_idx [T*top_k] int64,
 * sorted_weights [T*top_k] f32, expert_counts [E] int32, expert_offsets [E] int32
 * (exclusive prefix of counts). Deterministic: inside an expert the assignments are in
 * ascending (token, k) order, i.e. torch.argsort(flat_expert, stable=True).
 * status_dev may be NULL; otherwise it records out-of-range expert indices. */
int gptoss_fused_moe_routing(const int64_t* router_indices, const float* routing_weights,
                             int64_t num_tokens, int top_k, int num_experts,
                             int64_t* sorted_token_idx, int64_t* sorted_expert_idx,
                             float* sorted_weights, int32_t* expert_counts,
                             int32_t* expert_offsets, int32_t* status_dev, void* stream);

/* Router (HF GptOssTopKRouter.forward, modeling_gpt_oss.py; the reference receives its
 * outputs in CutlassGptOssExperts.forward, kernels/cutlass_experts.py:376-391):
 * logits = bf16(hidden[T,H] . weight[E,H]^T + bias[E]) (fp32 accumulate), top-k
 * (ties -> lower expert index), softmax over the k logits rounded to bf16.
 * Outputs: router_indices [T,k] int64, router_scores [T,k] bf16 (may be NULL),
 * routing_weights_f32 [T,k] (the scores as f32, may be NULL), logits [T,E] bf16 (may be
 * NULL). hidden, weight, bias are bf16; H % 8 == 0; E <= 256; k <= 8. */
int gptoss_router_topk(const void* hidden, const void* weight, const void* bias,
                       int64_t num_tokens, int64_t hidden_size, int num_experts, int top_k,
                       int64_t* router_indices, void* router_scores,
                       float* routing_weights_f32, void* logits, void* stream);

/* Throughput probe of the block-scaled tensor-core MMAs the GEMMs issue: kind 0 =
 * tcgen05.mma kind::mxf8f6f4.block_scale (E4M3 x E2M1, UE8M0 1x32 scales, k block 128
 * codes, the W4A8 mode), kind 1 = kind::mxf4nvf4.block_scale.scale_vec::4X (E2M1 x E2M1,
 * UE4M3 1x16 scales, k block 256 codes, the W4A4 mode). One CTA per SM (pair = 0: M = 128)
 * or one CTA pair per two SMs (pair = 1: M = 256, cta_group::2), each issuing `iters` k
 * blocks of M x n into one accumulator from operands resident in shared memory (no memory
 * traffic). n: multiple of 16 in [16, 256]. FLOPs of one launch = (SMs, or SMs / 2 pairs) x
 * iters x 2 x M x n x (128 or 256 codes). The caller times it (CUDA events on `stream`). No
 * counterpart in the reference; it is the measured denominator of the tensor-bound GEMM
 * rooflines. */
int gptoss_mma_peak(int kind, int pair, int n, int iters, int32_t* status_dev, void* stream);

/* The second half of the router alone: top-k (ties -> lower expert index, NaN above every
 * number) and the softmax over the k values rounded to bf16, on given bf16 logits [T, E]
 * (E <= 256, k <= 8). Same device code as gptoss_router_topk. No counterpart in the
 * reference (its experts module receives the routing); for callers that run their own
 * router projection, and for checking the top-k bit for bit against given logits. */
int gptoss_router_topk_from_logits(const void* logits, int64_t num_tokens, int num_experts, int top_k,
                                   int64_t* router_indices, void* router_scores, float* routing_weights_f32,
                                   void* stream);

/* Replaces quantize_activations_to_fp8 (kernels/cutlass_experts.py:197-251):
 * x [M,K] (bf16 or f32, `dtype`) -> codes [M,K] e4m3 bytes + scales [M,K/32] UE8M0,
 * bit-identical to the reference. K % 32 == 0. */
int gptoss_quantize_fp8(const void* x, int dtype, int64_t rows, int64_t cols, uint8_t* codes,
                        uint8_t* scales, void* stream);

/* Replaces swiglu (kernels/cutlass_experts.py:258-276): x [rows, 2n] with gate on even
 * and up on odd columns -> out [rows, n]; gate clamped to <= limit, up to [-limit, limit],
 * out = gate * sigmoid(alpha * gate) * (up + 1). bf16 follows torch's per-op rounding. */
int gptoss_swiglu(const void* x, int dtype, int64_t rows, int64_t cols, void* out, float alpha,
                  float limit, void* stream);

/* Replaces convert_a_scales_for_w4a8 / convert_b_scales_for_w4a8
 * (kernels/matmul_mxfp4_cutlass.cu:666-759): row-major scales [rows, K/32] -> one
 * blocked buffer of blocked bytes (zero padded). `k` is the (padded) K the GEMM uses;
 * the mapping does not depend on M or N beyond `rows`. */
int gptoss_convert_scales_blocked(const uint8_t* scales_rowmajor, int64_t rows, int64_t k,
                                  uint8_t* blocked, int64_t blocked_bytes, void* stream);

/* Bytes one blocked buffer of `rows` rows needs for reduction depth k. Host only. */
int64_t gptoss_blocked_scales_bytes(int64_t rows, int64_t k);

/* Replaces batch_convert_a_scales_for_w4a8_gpu (kernels/matmul_mxfp4_cutlass.cu:912-1004)
 * without its host sync: per-expert blocked activation scales laid end to end, expert e
 * at sf_offsets[e] (bytes, written on the device). counts/offsets are [E] int32 device
 * arrays. `capacity` must be >= gptoss_batch_blocked_scales_capacity(total_rows, E, k). */
int gptoss_batch_convert_a_scales(const uint8_t* scales_rowmajor, const int32_t* expert_counts,
                                  const int32_t* expert_offsets, int num_experts, int64_t k,
                                  uint8_t* blocked, int64_t capacity, int32_t* sf_offsets,
                                  void* stream);
int64_t gptoss_batch_blocked_scales_capacity(int64_t total_rows, int num_experts, int64_t k);

/* Replaces cutlass_fp4_group_mm, W4A8 mode (kernels/matmul_mxfp4_cutlass.cu:1118-1171,
 * run_w4a8_group_mm_sm120 :471-655; op cutlass::fp4_group_mm, cutlass_experts.py:147-166):
 * for each expert e with m_e = problem_sizes[3e] rows:
 *   out[off_e + i, n] = bf16(alphas[e] * sum_k A[off_e + i, k] 2^(sfa) * B[e, n, k] 2^(sfb))
 * a [M, lda] e4m3 (lda <= K; columns past lda read as zero), b [E, N, K/2] packed E2M1
 * (K % 128 == 0), a_blockscale blocked per expert at sf_offsets[e] (bytes),
 * b_blockscales [E, ldb_blockscale] blocked per expert, alphas [E] f32,
 * problem_sizes [E,3] int32 (m_e, N, K), expert_offsets [E] int32, out [M, N] bf16.
 * Rows of `out` owned by no expert are left untouched. gemm_mode: GPTOSS_GEMM_*. */
int gptoss_fp4_group_mm(void* out, const uint8_t* a, int64_t m_total, int64_t lda,
                        const uint8_t* b, int num_experts, int64_t n, int64_t k,
                        const uint8_t* a_blockscale, const uint8_t* b_blockscales,
                        int64_t ldb_blockscale, const float* alphas,
                        const int32_t* problem_sizes, const int32_t* expert_offsets,
                        const int32_t* sf_offsets, int gemm_mode, int32_t* status_dev,
                        void* stream);

/* Replaces cutlass_fp4_group_mm, W4A4 mode (NVFP4 x NVFP4; kernels/matmul_mxfp4_cutlass.cu:
 * 1157-1162 dispatching to run_w4a4_original :180-356, pointer set-up :56-110): for each
 * expert e with m_e = problem_sizes[3e] rows,
 *   out[off_e + i, n] = bf16(alphas[e] * sum_k A[off_e + i, k] sfa(i, k/16) * B[e, n, k] sfb(n, k/16))
 * a [M, K/2] and b [E, N, K/2] packed E2M1 (low nibble = even k), K % 64 == 0, lda == K/2;
 * scales UE4M3 (float8_e4m3fn bytes with the sign bit clear), one per 16 codes, in the
 * blocked layout (128-row x 64-code atoms of 512 bytes): expert e's activation scales start
 * sf_offsets[e] ROWS into a_blockscale (sf_offsets[e] * K/16 bytes, a multiple of 16),
 * its weight scales at e * ldb_blockscale bytes (ldb >= the blocked size of N x K/16).
 * alphas [E] f32, expert_offsets [E] int32, out [M, N] bf16. tcgen05.mma kind::mxf4nvf4
 * block_scale scale_vec::4X on the tiles of gptoss_fp4_group_mm (same gemm_mode choice). */
int gptoss_fp4_group_mm_w4a4(void* out, const uint8_t* a, int64_t m_total, int64_t lda,
                             const uint8_t* b, int num_experts, int64_t n, int64_t k,
                             const uint8_t* a_blockscale, const uint8_t* b_blockscales,
                             int64_t ldb_blockscale, const float* alphas,
                             const int32_t* problem_sizes, const int32_t* expert_offsets,
                             const int32_t* sf_offsets, int gemm_mode, int32_t* status_dev,
                             void* stream);

/* Workspace (device bytes) for gptoss_moe_experts_forward / gptoss_moe_layer_forward. */
size_t gptoss_moe_workspace_bytes(int64_t num_tokens, int top_k, int num_experts,
                                  int64_t hidden_size, int64_t intermediate_size);

/* Replaces CutlassGptOssExperts.forward (kernels/cutlass_experts.py:376-452) as one
 * stream of kernels with no host synchronisation:
 *   route (stable counting sort) -> gather + FP8 quantise (blocked scales)
 *   -> GEMM1 (+bias, SwiGLU, FP8 requantise) -> GEMM2 (+bias, x routing weight,
 *   bf16 scatter-add into out).
 * hidden [T,H] bf16; router_indices [T,k] int64; routing_weights [T,k] f32;
 * gate_up_data [E, 2I, Kh/2] u8, gate_up_scales [E, ldb1] blocked, gate_up_bias [E,2I] f32;
 * down_data [E, H, Ki/2] u8, down_scales [E, ldb2] blocked, down_bias [E,H] f32;
 * Kh = pad128(H), Ki = pad128(I); out [T,H] bf16 (overwritten). swiglu: alpha, limit.
 * status_dev: NULL or a device int32 that records kernel timeouts / bad indices. */
int gptoss_moe_experts_forward(const void* hidden, const int64_t* router_indices,
                               const float* routing_weights, int64_t num_tokens, int top_k,
                               int num_experts, int64_t hidden_size, int64_t intermediate_size,
                               const uint8_t* gate_up_data, const uint8_t* gate_up_scales,
                               int64_t ldb_gate_up, const float* gate_up_bias,
                               const uint8_t* down_data, const uint8_t* down_scales,
                               int64_t ldb_down, const float* down_bias, float swiglu_alpha,
                               float swiglu_limit, void* out, void* workspace,
                               size_t workspace_bytes, int gemm_mode, int32_t* status_dev,
                               void* stream);

/* Router + experts (HF GptOssMLP.forward: router then experts): router_weight [E,H] bf16,
 * router_bias [E] bf16; writes router_indices [T,k] int64 and router_scores [T,k] bf16
 * (either may be NULL) and out [T,H] bf16. Same weights/workspace as above. */
int gptoss_moe_layer_forward(const void* hidden, const void* router_weight,
                             const void* router_bias, int64_t num_tokens, int top_k,
                             int num_experts, int64_t hidden_size, int64_t intermediate_size,
                             const uint8_t* gate_up_data, const uint8_t* gate_up_scales,
                             int64_t ldb_gate_up, const float* gate_up_bias,
                             const uint8_t* down_data, const uint8_t* down_scales,
                             int64_t ldb_down, const float* down_bias, float swiglu_alpha,
                             float swiglu_limit, void* out, int64_t* router_indices_out,
                             void* router_scores_out, void* workspace, size_t workspace_bytes,
                             int gemm_mode, int32_t* status_dev, void* stream);

/* The decoder block around the MoE layer, for stacks of layers (the reference's model runs
 * it as residual + mlp(post_attention_layernorm(hidden)), repro_compile_hftf.py:103-107
 * compiling the whole model): out = hidden + layer(RMSNorm(hidden)), RMSNorm as GptOssRMSNorm
 * (fp32 mean of squares, rsqrt(mean + norm_eps), times norm_weight [H] bf16, one rounding).
 * The norm and the residual copy are one kernel (gptoss_rmsnorm_residual) and GEMM2 adds the
 * expert outputs straight into the residual rows, so a block is the MoE kernels only. out
 * may alias hidden. workspace: gptoss_moe_block_workspace_bytes(). */
size_t gptoss_moe_block_workspace_bytes(int64_t num_tokens, int top_k, int num_experts,
                                        int64_t hidden_size, int64_t intermediate_size);
int gptoss_moe_block_forward(const void* hidden, const void* norm_weight, float norm_eps,
                             const void* router_weight, const void* router_bias, int64_t num_tokens,
                             int top_k, int num_experts, int64_t hidden_size,
                             int64_t intermediate_size, const uint8_t* gate_up_data,
                             const uint8_t* gate_up_scales, int64_t ldb_gate_up,
                             const float* gate_up_bias, const uint8_t* down_data,
                             const uint8_t* down_scales, int64_t ldb_down, const float* down_bias,
                             float swiglu_alpha, float swiglu_limit, void* out,
                             int64_t* router_indices_out, void* router_scores_out, void* workspace,
                             size_t workspace_bytes, int gemm_mode, int32_t* status_dev, void* stream);
/* xn = RMSNorm(x) as above; residual_out (may be NULL, may alias x) = a copy of x. */
int gptoss_rmsnorm_residual(const void* x, const void* weight, float eps, int64_t num_tokens,
                            int64_t hidden_size, void* xn, void* residual_out, void* stream);

/* ---- The expert forward as three stages on a shared workspace (same kernels as
 * gptoss_moe_experts_forward; used for per-stage timing and by expert parallelism,
 * which exchanges rows between the stages). */

/* Byte offsets of the workspace regions, in this order (GPTOSS_WS_* indices):
 * sorted_token i64[A], sorted_expert i64[A], sorted_weight f32[A], counts i32[E],
 * offsets i32[E], act_sf_offsets i32[E], inter_sf_offsets i32[E], act_codes u8[A,H],
 * act_scales (blocked), inter_codes u8[A,I], inter_scales (blocked), router_idx i64[A],
 * router_weights f32[A], total bytes. Host only. */
enum {
  GPTOSS_WS_SORTED_TOKEN = 0, GPTOSS_WS_SORTED_EXPERT, GPTOSS_WS_SORTED_WEIGHT, GPTOSS_WS_COUNTS,
  GPTOSS_WS_OFFSETS, GPTOSS_WS_ACT_SF_OFFSETS, GPTOSS_WS_INTER_SF_OFFSETS, GPTOSS_WS_ACT_CODES,
  GPTOSS_WS_ACT_SCALES, GPTOSS_WS_INTER_CODES, GPTOSS_WS_INTER_SCALES, GPTOSS_WS_ROUTER_IDX,
  GPTOSS_WS_ROUTER_WEIGHTS, GPTOSS_WS_TOTAL, GPTOSS_WS_NUM_REGIONS
};
int gptoss_moe_workspace_layout(int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size,
                                int64_t intermediate_size, int64_t* offsets_out /* host [14] */);

/* Stage 1 (fused_moe_routing + hidden[sorted_token] + quantize_activations_to_fp8 +
 * batch_convert_a_scales_for_w4a8_gpu, kernels/cutlass_experts.py:399-408 and
 * kernels/matmul_mxfp4_cutlass.cu:912-1004): fills the routing, act_codes and
 * act_scales regions and zeroes the padding of both blocked scale regions. */
int gptoss_moe_route_quant(const void* hidden, const int64_t* router_indices,
                           const float* routing_weights, int64_t num_tokens, int top_k,
                           int num_experts, int64_t hidden_size, int64_t intermediate_size,
                           void* workspace, size_t workspace_bytes, int gemm_mode,
                           int32_t* status_dev, void* stream);

/* Stage 2 (GEMM1 + bias + SwiGLU + requantisation, kernels/cutlass_experts.py:410-427):
 * reads act_codes/act_scales, writes inter_codes/inter_scales. */
int gptoss_moe_gemm1(int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size,
                     int64_t intermediate_size, const uint8_t* gate_up_data,
                     const uint8_t* gate_up_scales, int64_t ldb_gate_up, const float* gate_up_bias,
                     float swiglu_alpha, float swiglu_limit, void* workspace,
                     size_t workspace_bytes, int gemm_mode, int32_t* status_dev, void* stream);

/* Stage 3 (GEMM2 + bias, x routing weight, scatter-add, kernels/cutlass_experts.py:429-450):
 * ADDS into out [T,H] bf16 (zero it first for the reference's semantics, or pass a
 * residual to fuse the residual add). */
int gptoss_moe_gemm2(int64_t num_tokens, int top_k, int num_experts, int64_t hidden_size,
                     int64_t intermediate_size, const uint8_t* down_data,
                     const uint8_t* down_scales, int64_t ldb_down, const float* down_bias,
                     void* out, void* workspace, size_t workspace_bytes, int gemm_mode,
                     int32_t* status_dev, void* stream);

/* ---- Expert forward without any device allocation.
 *
 * No counterpart in the reference. Some callers cannot hand this library a workspace or let
 * it allocate one: runtimes that reserve all device memory up front behind their own pool
 * (an out-of-band cudaMalloc fails there), hosts that bind the C ABI through an FFI and have
 * no device allocator to call, and latency-critical loops that cannot pay for cudaMalloc /
 * cudaFree, which synchronise the device. For them this entry point runs the same kernels
 * as gptoss_moe_experts_forward with the workspace in a static device array of
 * GPTOSS_NOALLOC_SCRATCH_BYTES inside this library (every GPU that loads the library holds it
 * until the process exits). The array is reserved when the library's device code is loaded
 * onto a GPU, i.e. at this library's first CUDA call on that device, whichever entry point it
 * is: a runtime that reserves device memory up front must leave that many bytes free, or
 * that first call fails with an out-of-memory CUDA error. Batches whose workspace (gptoss_moe_workspace_bytes) exceeds that
 * size are rejected with GPTOSS_ERR_INVALID_ARGUMENT — at H = I = 2880 and 32 experts that
 * is about 2,400 token-expert assignments (600 tokens at top-4). The first call on a device
 * does a one-time set-up: it looks up the array's device address (cudaGetSymbolAddress, with
 * that device current) and caches it; make that first call before any stream capture
 * begins. All calls share the one
 * array and it keeps the previous call's contents; every region is rewritten before it is
 * read and the words that must start at zero are cleared by the call itself, but calls that
 * overlap on the GPU (other streams, other threads) race on it. Inputs, outputs and the status word are the caller's, exactly as in
 * gptoss_moe_experts_forward; no cudaMalloc, cudaFree or allocating library routine is called. */
#define GPTOSS_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
int gptoss_moe_experts_forward_noalloc(const void* hidden, const int64_t* router_indices,
                                       const float* routing_weights, int64_t num_tokens,
                                       int top_k, int num_experts, int64_t hidden_size,
                                       int64_t intermediate_size, const uint8_t* gate_up_data,
                                       const uint8_t* gate_up_scales, int64_t ldb_gate_up,
                                       const float* gate_up_bias, const uint8_t* down_data,
                                       const uint8_t* down_scales, int64_t ldb_down,
                                       const float* down_bias, float swiglu_alpha,
                                       float swiglu_limit, void* out, int gemm_mode,
                                       int32_t* status_dev, void* stream);

/* ---- Expert parallelism (one process per GPU, experts sharded by contiguous ranges).
 *
 * No counterpart in the reference, which runs on one GPU ("Expert parallelism not
 * implemented", kernels/cutlass_matmul_investigations.md:231). Rank r of W owns experts
 * [r*E/W, (r+1)*E/W). One layer is
 *   gptoss_ep_dispatch   -> send_counts, send_rows (quantised, ordered by destination rank)
 *   all-to-all of the counts, then of the rows (the caller's collective, e.g. NCCL)
 *   gptoss_ep_expert_forward on the received rows -> back_rows (weighted bf16, same order)
 *   all-to-all of back_rows with the splits reversed
 *   gptoss_ep_combine    -> out[t] = fp32 sum of token t's k rows (ascending expert), to bf16.
 * A row is gptoss_ep_row_bytes(H) bytes: FP8 codes [H], UE8M0 scales [H/32], padding, then
 * the local expert id (int32) and routing weight (f32) in its last 8 bytes. The codes and
 * scales are those gptoss_quantize_fp8 gives for the token's hidden row. */
int64_t gptoss_ep_row_bytes(int64_t hidden_size);
size_t gptoss_ep_dispatch_workspace_bytes(int64_t num_tokens, int top_k, int world_size);
/* router_indices hold GLOBAL expert ids; send_counts: [W] int32 rows per destination rank;
 * pos_of: [T*k] int32, row of send_rows that assignment i = t*k + j went to (the same row
 * of the returned back_rows).
 * capacity == 0: send_rows [T*k, row_bytes], compact, destination-major; the exchange
 *   needs send_counts on the host for its splits.
 * capacity >= T*k: send_rows [W*capacity, row_bytes], destination q's rows at
 *   [q*capacity, q*capacity + send_counts[q]), the rest marked empty (local expert -1);
 *   the exchange uses equal splits of capacity rows and no host-visible counts. */
int gptoss_ep_dispatch(const void* hidden, const int64_t* router_indices, const float* routing_weights,
                       int64_t num_tokens, int top_k, int num_experts, int world_size,
                       int64_t hidden_size, int64_t capacity, uint8_t* send_rows,
                       int32_t* send_counts, int32_t* pos_of, void* workspace,
                       size_t workspace_bytes, int32_t* status_dev, void* stream);
/* Received rows -> back_rows [num_rows, H] bf16, row r = routing weight x expert output of
 * row r (route sort by local expert, blocked-scale gather, GEMM1 + SwiGLU + requant,
 * GEMM2 + bias); empty rows (local expert -1) are skipped and come back as zeros. Weights
 * are this rank's [E/W, ...] slices; workspace = gptoss_moe_workspace_bytes(num_rows, 1,
 * E/W, H, I). Any other local expert id outside [0, E/W) sets *status_dev. */
int gptoss_ep_expert_forward(const uint8_t* recv_rows, int64_t num_rows, int num_local_experts,
                             int64_t hidden_size, int64_t intermediate_size,
                             const uint8_t* gate_up_data, const uint8_t* gate_up_scales,
                             int64_t ldb_gate_up, const float* gate_up_bias,
                             const uint8_t* down_data, const uint8_t* down_scales,
                             int64_t ldb_down, const float* down_bias, float swiglu_alpha,
                             float swiglu_limit, void* back_rows, void* workspace,
                             size_t workspace_bytes, int gemm_mode, int32_t* status_dev,
                             void* stream);
/* out [T, H] bf16 (overwritten): the k returned rows of each token summed in fp32 in
 * ascending global expert order and rounded to bf16 once -- the result of the reference's
 * scatter_add_ of expert-sorted bf16 rows into a zero bf16 tensor on the CPU
 * (kernels/cutlass_experts.py:445-450). */
int gptoss_ep_combine(const void* back_rows, int64_t num_back_rows, const int32_t* pos_of,
                      const int64_t* router_indices, int64_t num_tokens, int top_k,
                      int64_t hidden_size, void* out, void* stream);

/* ---- Expert parallelism over peer memory (one node; no collective library on the data
 * path). Each rank allocates one exchange buffer of gptoss_ep_p2p_buffer_bytes(W, cap, H)
 * with gptoss_ipc_alloc (zeroed; the handle goes to every other rank, which maps it with
 * gptoss_ipc_open), and passes its own base (`local_base`) and the W base addresses (its
 * own at index `rank`) as a device array `peer_bases`. Layout of a buffer: a 1 KB header of
 * flags and completion counters, receive rows [W][cap][row_bytes], return rows [W][cap][H]
 * bf16. One layer, with `epoch` = 1, 2, ... per call
 * and identical on every rank:
 *   gptoss_ep_p2p_dispatch        quantised rows stored straight into the owners' receive
 *                                 rows, then dispatch flag[rank] raised on every peer
 *                                 (one cluster launch up to 64 tokens x top-k <= 512);
 *   gptoss_ep_p2p_route_dispatch  the router (logits, top-k, softmax, as gptoss_router_topk)
 *                                 and the dispatch, one launch at decode sizes;
 *   gptoss_ep_p2p_expert_forward  waits for every sender's flag, runs the local experts,
 *                                 stores each output row into its source rank's return
 *                                 rows, raises return flag[W + rank] on every peer;
 *   gptoss_ep_p2p_combine         waits for every owner's return flag, sums each token's
 *                                 rows like gptoss_ep_combine.
 * Waits give up after 1 s and set *status_dev to 0x301. Buffers are reused across calls
 * without a barrier (see ep_p2p.cuh). No counterpart in the reference. */
int gptoss_ipc_handle_bytes(void);
int gptoss_ipc_alloc(size_t bytes, void** ptr, void* handle_out);
int gptoss_ipc_open(const void* handle, void** ptr);
int gptoss_ipc_close(void* ptr);
int gptoss_ipc_free(void* ptr);
size_t gptoss_ep_p2p_buffer_bytes(int world_size, int64_t capacity, int64_t hidden_size);
int gptoss_ep_p2p_dispatch(const void* hidden, const int64_t* router_indices, const float* routing_weights,
                           int64_t num_tokens, int top_k, int num_experts, int world_size, int rank,
                           int64_t hidden_size, int64_t capacity, void* local_base,
                           const uint64_t* peer_bases, int32_t epoch, int32_t* send_counts,
                           int32_t* pos_of, void* workspace, size_t workspace_bytes,
                           int32_t* status_dev, void* stream);
/* Router + dispatch: router_indices_out [T, k] i64, router_scores_out [T, k] bf16 (may be
 * NULL), routing_weights_out [T, k] f32 (the scores as f32); the rest as
 * gptoss_ep_p2p_dispatch. */
int gptoss_ep_p2p_route_dispatch(const void* hidden, const void* router_weight, const void* router_bias,
                                 int64_t num_tokens, int top_k, int num_experts, int world_size, int rank,
                                 int64_t hidden_size, int64_t capacity, void* local_base,
                                 const uint64_t* peer_bases, int32_t epoch, int64_t* router_indices_out,
                                 void* router_scores_out, float* routing_weights_out, int32_t* send_counts,
                                 int32_t* pos_of, void* workspace, size_t workspace_bytes,
                                 int32_t* status_dev, void* stream);
int gptoss_ep_p2p_expert_forward(void* local_base, int world_size, int rank, int64_t capacity,
                                 int32_t epoch, int num_local_experts, int64_t hidden_size,
                                 int64_t intermediate_size, const uint8_t* gate_up_data,
                                 const uint8_t* gate_up_scales, int64_t ldb_gate_up,
                                 const float* gate_up_bias, const uint8_t* down_data,
                                 const uint8_t* down_scales, int64_t ldb_down,
                                 const float* down_bias, float swiglu_alpha, float swiglu_limit,
                                 void* back_rows, const uint64_t* peer_bases, void* workspace,
                                 size_t workspace_bytes, int gemm_mode, int32_t* status_dev,
                                 void* stream);
int gptoss_ep_p2p_combine(const void* local_base, int world_size, int64_t capacity, int32_t epoch,
                          const int32_t* pos_of, const int64_t* router_indices, int64_t num_tokens,
                          int top_k, int64_t hidden_size, void* out, int32_t* status_dev,
                          void* stream);

/* The same expert-parallel step in ONE persistent launch (no counterpart in the reference,
 * which has no expert parallelism; it replaces the four calls above at decode sizes):
 * router (router_weight != NULL: logits, top-k, softmax as gptoss_router_topk, written to
 * router_indices_out / router_scores_out (may be NULL) / routing_weights_out) or the given
 * routing (router_weight == NULL: router_indices, routing_weights); the dispatch into the
 * owners' receive rows; the wait for every sender's flag; the local experts (the
 * num_experts / world_size experts of this rank, weights as gptoss_moe_experts_forward)
 * with each output row stored into its source rank's return rows; the return flags; the
 * wait for every owner's return flag and the combine into out [T, H] bf16. Same buffers,
 * row format, flags and epochs as the calls above; send_counts [W] and pos_of [T * top_k]
 * are written as gptoss_ep_p2p_dispatch writes them. workspace: at least
 * gptoss_moe_workspace_bytes(world_size * capacity, 1, num_experts / world_size, H, I).
 * Serves steps for which gptoss_ep_p2p_layer_fits() is 1 (T <= 64, T * top_k <= 256,
 * world_size * capacity <= 1024 received rows, few rows per local expert); every rank must
 * take it in the same step. gptoss_set_ep_layer_kernel(0) turns it off (returns the previous
 * setting). */
int gptoss_set_ep_layer_kernel(int enable);
int gptoss_ep_p2p_layer_fits(int64_t num_tokens, int top_k, int num_experts, int world_size,
                             int64_t hidden_size, int64_t intermediate_size, int64_t capacity);
int gptoss_ep_p2p_layer_forward(const void* hidden, const void* router_weight, const void* router_bias,
                                const int64_t* router_indices, const float* routing_weights,
                                int64_t num_tokens, int top_k, int num_experts, int world_size, int rank,
                                int64_t hidden_size, int64_t intermediate_size,
                                const uint8_t* gate_up_data, const uint8_t* gate_up_scales,
                                int64_t ldb_gate_up, const float* gate_up_bias, const uint8_t* down_data,
                                const uint8_t* down_scales, int64_t ldb_down, const float* down_bias,
                                float swiglu_alpha, float swiglu_limit, int64_t capacity, void* local_base,
                                const uint64_t* peer_bases, int32_t epoch, void* out,
                                int64_t* router_indices_out, void* router_scores_out,
                                float* routing_weights_out, int32_t* send_counts, int32_t* pos_of,
                                void* workspace, size_t workspace_bytes, int32_t* status_dev, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GPTOSS_MOE_H */
