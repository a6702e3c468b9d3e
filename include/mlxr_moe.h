/*
 * mlxr_moe.h — C ABI of the B200 (sm_100a) implementation of mlxr's MoE
 * block and its quantised-matmul op family.
 *
 * The boundary follows the reference's FFI contract for these ops
 * (crates/mlxr-sys -> mlx-c; wrapped by Guarded::try_from_op,
 * crates/mlxr/src/utils/guard.rs:31-51): every entry point returns an int
 * status, 0 on success; on failure a message is kept in a thread-local slot
 * and read back with mlxr_cu_last_error() (the reference's C error callback
 * into a thread-local, crates/mlxr/src/error.rs:229-290).
 *
 * Differences that follow from the device model:
 *  - Arrays are caller-owned device pointers plus explicit sizes; nothing is
 *    allocated on the compute path. Scratch comes from a caller-provided
 *    workspace (mlxr_cu_moe_workspace_size).
 *  - Work is queued asynchronously on the caller's stream (a cudaStream_t
 *    passed as void*; NULL = the legacy default stream). Errors detected on
 *    the device (a wait that timed out, an out-of-range expert index) land in
 *    a status word read by mlxr_cu_moe_status().
 *  - Only mode "affine" exists; bits in {2, 4, 8} for the op family, {4, 8}
 *    for the MoE block; group sizes {32, 64, 128} (block: 64).
 *
 * Array layouts match MLX's packing as consumed by the reference:
 *  packed weights uint32 [..., N, K*bits/32] with element j of a word at bits
 *  [bits*j, bits*j+bits); scales/biases [..., N, K/group_size] in the
 *  activation dtype (crates/mlxr/src/ops/quantization.rs:299-315 pins the
 *  shapes).
 */
#ifndef MLXR_MOE_H
#define MLXR_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLXR_CU_ABI_VERSION 2

#if defined(__GNUC__)
#define MLXR_CU_API __attribute__((visibility("default")))
#else
#define MLXR_CU_API
#endif

typedef enum mlxr_cu_status {
  MLXR_CU_OK = 0,
  MLXR_CU_ERR_INVALID_ARGUMENT = 1, /* bad shape, null pointer, bad index */
  MLXR_CU_ERR_UNSUPPORTED = 2,      /* bits / group size / mode not supported */
  MLXR_CU_ERR_CUDA = 3,             /* a CUDA runtime or driver call failed */
  MLXR_CU_ERR_WORKSPACE = 4,        /* workspace missing or too small */
  MLXR_CU_ERR_TIMEOUT = 5,          /* a device-side bounded wait expired */
  MLXR_CU_ERR_NCCL = 6,             /* a collective failed */
  MLXR_CU_ERR_DEVICE_INDEX = 7      /* the device saw an out-of-range index */
} mlxr_cu_status;

typedef enum mlxr_cu_dtype {
  MLXR_CU_BFLOAT16 = 0,
  MLXR_CU_FLOAT16 = 1,
  MLXR_CU_FLOAT32 = 2
} mlxr_cu_dtype;

/* ------------------------------------------------------------ errors -- */

/* Last error message of the calling thread, or NULL. Replaces the
 * thread-local LAST_MLX_ERROR slot (crates/mlxr/src/error.rs:239-290). */
MLXR_CU_API const char* mlxr_cu_last_error(void);
MLXR_CU_API void mlxr_cu_clear_error(void);
MLXR_CU_API int mlxr_cu_abi_version(void);

/* ---------------------------------------------------- the op family -- */

/* quantize (crates/mlxr/src/ops/quantization.rs:47-70 -> mlx_quantize):
 * w [rows, cols] in dtype -> wq uint32 [rows, cols*bits/32],
 * scales/biases [rows, cols/group_size] in dtype. mode must be "affine" or
 * NULL. group_size 0 / bits 0 select the reference defaults 64 / 4
 * (quantization.rs:11-13). The arithmetic is MLX's affine quantiser, so the
 * bytes match mlxr-convert output (crates/mlxr-convert/src/quantize.rs:44):
 * per group, the end of larger magnitude is the edge, the scale is
 * (max - min) / (2^bits - 1) (at least 1e-7) with the edge's sign flipped
 * (negative when the edge is the max), snapped to edge / rint(edge / scale)
 * so that 0 is exact, the bias is the edge (0 when rint(edge / scale) = 0),
 * and the codes rint((w - bias) / scale) clamped to [0, 2^bits - 1] come from
 * the fp32 pair before it is rounded to dtype. Halves round to even. */
MLXR_CU_API int mlxr_cu_quantize(const void* w, mlxr_cu_dtype dtype, int64_t rows, int64_t cols, int group_size, int bits,
                     const char* mode, uint32_t* wq, void* scales, void* biases, void* stream);

/* dequantize (quantization.rs:118-146 -> mlx_dequantize):
 * out[r][k] = scale * q + bias (fp32 fma), written in out_dtype. */
MLXR_CU_API int mlxr_cu_dequantize(const uint32_t* wq, const void* scales, const void* biases, mlxr_cu_dtype sb_dtype,
                       int64_t rows, int64_t cols, int group_size, int bits, const char* mode, void* out,
                       mlxr_cu_dtype out_dtype, void* stream);

/* quantized_matmul (quantization.rs:81-112 -> mlx_quantized_matmul;
 * QuantizedLinear::forward, crates/mlxr/src/layers/quantized.rs:356-371):
 * x [M, K] (x_dtype; scales/biases share it) times the dequantised w:
 *   transpose != 0: w packed [N, K*bits/32], out = x @ W^T
 *   transpose == 0: w packed [K, N*bits/32], out = x @ W
 * out [M, N] in x_dtype, fp32 accumulation. biases may not be NULL (affine). */
MLXR_CU_API int mlxr_cu_quantized_matmul(const void* x, mlxr_cu_dtype x_dtype, int64_t M, int64_t K, const uint32_t* w,
                             const void* scales, const void* biases, int64_t N, int transpose, int group_size,
                             int bits, const char* mode, void* out, void* stream);

/* gather_qmm (quantization.rs:171-221 -> mlx_gather_qmm):
 * out[p] = x[lhs[p]] @ dequant(w[rhs[p]])^T for p in [0, num_indices),
 * x [x_batch, M, K], w packed [w_batch, N, K*bits/32] (transpose) or
 * [w_batch, K, N*bits/32]; out [num_indices, M, N] in x_dtype. lhs / rhs may
 * be NULL, meaning the identity (MLX's broadcast of absent indices, flattened
 * by the caller). sorted_indices is the reference's hint (rhs sorted
 * ascending); results do not depend on it. */
MLXR_CU_API int mlxr_cu_gather_qmm(const void* x, mlxr_cu_dtype x_dtype, int64_t x_batch, int64_t M, int64_t K,
                       const uint32_t* w, const void* scales, const void* biases, int64_t w_batch, int64_t N,
                       const uint32_t* lhs_indices, const uint32_t* rhs_indices, int64_t num_indices, int transpose,
                       int group_size, int bits, const char* mode, int sorted_indices, void* out, void* stream);

/* gather_qmm with a caller-provided workspace (the same call as
 * mlxr_cu_gather_qmm, quantization.rs:171-221, as QuantizedSwitchLinear::apply
 * issues it, crates/mlxr-lm/src/nn/switch.rs:148-167). For bf16 x, transpose,
 * group_size 64, bits 4 or 8, K and N multiples of 128 and at most 1024
 * weight batches, the rows f = p * M + m are sorted by rhs[p] on the device
 * (counting sort, any index order), gathered (x[lhs[p]][m]) and multiplied on
 * the tensor cores by the block's grouped dequantising GEMM (tcgen05, fp32
 * accumulation, weights dequantised to bf16), then written back in index
 * order; every other shape runs mlxr_cu_gather_qmm unchanged (no workspace
 * used). Out-of-range indices are reported through mlxr_cu_op_status. The
 * workspace must be 256-byte aligned and at least
 * mlxr_cu_gather_qmm_workspace_size bytes (0 when the shape takes the
 * general kernel). */
MLXR_CU_API int mlxr_cu_gather_qmm_workspace_size(mlxr_cu_dtype x_dtype, int64_t x_batch, int64_t M, int64_t K,
                                                  int64_t w_batch, int64_t N, int64_t num_indices, int transpose,
                                                  int group_size, int bits, size_t* bytes);
MLXR_CU_API int mlxr_cu_gather_qmm_ws(const void* x, mlxr_cu_dtype x_dtype, int64_t x_batch, int64_t M, int64_t K,
                                      const uint32_t* w, const void* scales, const void* biases, int64_t w_batch,
                                      int64_t N, const uint32_t* lhs_indices, const uint32_t* rhs_indices,
                                      int64_t num_indices, int transpose, int group_size, int bits, const char* mode,
                                      int sorted_indices, void* out, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* quantized_matmul with a caller-provided workspace (QuantizedLinear::forward,
 * crates/mlxr/src/layers/quantized.rs:356-371): the one-matrix case of
 * mlxr_cu_gather_qmm_ws (x_batch 1, w_batch 1, one index, M rows); workspace
 * size from mlxr_cu_gather_qmm_workspace_size(x_dtype, 1, M, K, 1, N, 1, ...). */
MLXR_CU_API int mlxr_cu_quantized_matmul_ws(const void* x, mlxr_cu_dtype x_dtype, int64_t M, int64_t K,
                                            const uint32_t* w, const void* scales, const void* biases, int64_t N,
                                            int transpose, int group_size, int bits, const char* mode, void* out,
                                            void* workspace, size_t workspace_bytes, void* stream);

/* gather_mm (crates/mlxr/src/ops/arithmetic.rs:1577-1609 -> mlx_gather_mm):
 * out[p] = a[lhs[p]] @ b[rhs[p]], a [a_batch, M, K], b [b_batch, K, N], all in
 * dtype, fp32 accumulation. */
MLXR_CU_API int mlxr_cu_gather_mm(const void* a, const void* b, mlxr_cu_dtype dtype, int64_t a_batch, int64_t M, int64_t K,
                      int64_t b_batch, int64_t N, const uint32_t* lhs_indices, const uint32_t* rhs_indices,
                      int64_t num_indices, int sorted_indices, void* out, void* stream);

/* -------------------------------------------------------- MoE block -- */

/* Block dimensions (Qwen 3.5/3.6 text config fields,
 * crates/mlxr-lm/src/qwen3_5/text/config.rs:124-152). */
typedef struct mlxr_cu_moe_config {
  int32_t hidden_size;                     /* D */
  int32_t num_experts;                     /* E */
  int32_t num_experts_per_tok;             /* K */
  int32_t moe_intermediate_size;           /* I */
  int32_t shared_expert_intermediate_size; /* Is; 0 = no shared expert */
  int32_t group_size;                      /* 64 */
  int32_t bits;                            /* routed experts: 4 or 8 */
  int32_t shared_bits;                     /* shared expert: 4 or 8 */
  int32_t norm_topk_prob;                  /* 1 = renormalise top-k (moe.rs:136-138) */
  int32_t shared_gate_bits;                /* shared_expert_gate: 4 or 8; 0 = shared_bits. Converted
                                              checkpoints pin it at 8 (mlxr-convert/src/qwen3_5.rs:
                                              classify_default) while the body is 4-bit */
  int32_t model_kind;                      /* 0 = Qwen 3.5/3.6 MoE block (above); 1 = Gemma 4 MoE branch
                                              (crates/mlxr-lm/src/gemma4/text/text.rs:568-664, 901-916):
                                              RMS-normed router, top-k of the scores, softmax over the k
                                              times per-expert scales, experts on the RMS-normed input
                                              with a packed gate_up_proj and GeGLU; no shared expert
                                              (the layer's dense MLP is outside the branch) */
  float rms_norm_eps;                      /* model_kind 1: eps of both RMS norms (config rms_norm_eps) */
} mlxr_cu_moe_config;

/* One quantised projection: packed weight, scales, biases (bf16). */
typedef struct mlxr_cu_qlinear {
  const uint32_t* weight;
  const void* scales;
  const void* biases;
} mlxr_cu_qlinear;

/* Parameters of Qwen35MoeBlock (crates/mlxr-lm/src/qwen3_5/text/moe.rs:52-78):
 * router `gate` [E, D] bf16 (unquantised), `switch_mlp.{gate,up}_proj`
 * [E, I, D*b/32] and `down_proj` [E, D, I*b/32] with scales/biases
 * [E, N, Kin/64] bf16, and the optional shared expert
 * (`shared_expert.{gate,up,down}_proj`, `shared_expert_gate` [1, D]). */
typedef struct mlxr_cu_moe_weights {
  const void* router_weight; /* [E, D] bf16 */
  const float* router_bias;  /* [E] fp32 added to the logits, or NULL */
  mlxr_cu_qlinear switch_gate;
  mlxr_cu_qlinear switch_up;
  mlxr_cu_qlinear switch_down;
  mlxr_cu_qlinear shared_gate;
  mlxr_cu_qlinear shared_up;
  mlxr_cu_qlinear shared_down;
  mlxr_cu_qlinear shared_expert_gate;
  /* model_kind 1 (Gemma 4): router_weight = Router.proj [E, D] bf16 (router_bias NULL);
   * switch_gate_up = experts.switch_glu.gate_up_proj [E, 2I, D*b/32] (gate rows 0..I-1, up rows
   * I..2I-1 of each expert; nn/switch.rs:242-345); switch_down as above; the shared_* and
   * switch_gate / switch_up members are unused. */
  mlxr_cu_qlinear switch_gate_up;
  const void* router_norm;   /* [D] bf16: Router.scale * hidden_size^-0.5 (text.rs:628-639) */
  const void* expert_scale;  /* [E] bf16: Router.per_expert_scale */
  const void* experts_norm;  /* [D] bf16: pre_feedforward_layernorm_2.weight (text.rs:907-911) */
} mlxr_cu_moe_weights;

/* Optional routing outputs (any member may be NULL). indices/weights are the
 * top-k in rank order (prob desc, expert asc); counts/offsets describe the
 * stable expert-sorted order of the flat rows f = t*K + k (gather_sort,
 * crates/mlxr-lm/src/nn/switch.rs:499-512); sorted_rows[pos] = f and
 * inverse[f] = pos (scatter_unsort, switch.rs:514-517). */
typedef struct mlxr_cu_moe_routing {
  int32_t* indices;     /* [T, K] */
  void* weights;        /* [T, K] bf16 */
  int32_t* counts;      /* [E] */
  int32_t* offsets;     /* [E + 1] */
  int32_t* sorted_rows; /* [T*K] */
  int32_t* inverse;     /* [T*K] */
} mlxr_cu_moe_routing;

/* Bytes of device workspace mlxr_cu_moe_block_forward needs for num_tokens. */
MLXR_CU_API int mlxr_cu_moe_workspace_size(const mlxr_cu_moe_config* cfg, int64_t num_tokens, size_t* bytes);

/* Qwen35MoeBlock::forward (moe.rs:116-146) for x [T, D] bf16 -> out [T, D]
 * bf16: router -> permute -> grouped gate/up + SwiGLU -> grouped down ->
 * weighted combine (+ sigmoid-gated shared expert). Replaces the chain of
 * mlx_quantized_matmul / mlx_softmax_axis / mlx_argpartition_axis /
 * mlx_take_along_axis / mlx_gather_qmm calls the block issues
 * (SplitSwitchFfn::forward_with_combine, switch.rs:446-474). The workspace
 * must be 256-byte aligned and at least mlxr_cu_moe_workspace_size bytes. */
MLXR_CU_API int mlxr_cu_moe_block_forward(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, const void* x,
                              int64_t num_tokens, void* out, const mlxr_cu_moe_routing* routing, void* workspace,
                              size_t workspace_bytes, void* stream);

/* Allocation-free variant of mlxr_cu_moe_block_forward (no counterpart in
 * the reference, whose ops always allocate their outputs through MLX). For
 * callers that cannot allocate device memory at call time: a serving engine
 * that reserves nearly all HBM up front and forbids later cudaMalloc (or
 * cannot afford its implicit synchronisation), or a host runtime that binds
 * this library over a plain C ABI without a device allocator to pass in.
 * The caller passes inputs and outputs as for mlxr_cu_moe_block_forward; the
 * scratch is a fixed 24 MiB array inside the library, held by every GPU that
 * loads the library until the process exits. Requests needing more scratch
 * (beyond 321 tokens for a hidden-2048 / 128-expert / top-8 / 768 block,
 * 161 tokens for hidden 4096 / intermediate 1536)
 * fail with MLXR_CU_ERR_WORKSPACE. The first call on each device looks the
 * array's device address up (with that device current); make that first call
 * before any stream capture. All calls share the one array, so calls that
 * overlap on the GPU (different streams or threads) race: serialise them.
 * device_status (device int, may be NULL) receives the device-side status
 * word (0 ok, 1 wait timeout, 2 index out of range) when the forward ends;
 * it is written (by a copy queued on the stream) only when the call returns
 * MLXR_CU_OK, so after an error it still holds what it held before. The
 * array's address is cached per device and driver context. Nothing on this
 * path calls cudaMalloc, cudaFree or an allocating routine. */
MLXR_CU_API int mlxr_cu_moe_block_forward_noalloc(const mlxr_cu_moe_config* cfg,
                                                  const mlxr_cu_moe_weights* weights, const void* x,
                                                  int64_t num_tokens, void* out,
                                                  const mlxr_cu_moe_routing* routing, int* device_status,
                                                  void* stream);

/* Profiling hook (no counterpart in the reference, which times with Apple's
 * xctrace, justfile:96-142): with count = 7 events (cudaEvent_t as void*),
 * later mlxr_cu_moe_block_forward calls on this thread record events[i] on
 * their stream at stage boundaries: 0 start, 1 router done, 2 permute done,
 * 3 gate/up GEMM done, 4 down GEMM done, 5 shared expert done, 6 combine
 * done. count = 0 switches it off. */
MLXR_CU_API int mlxr_cu_moe_set_stage_events(void* const* events, int count);

/* Reads (synchronising on stream) the device status word of the last forward
 * that used this workspace: MLXR_CU_OK, MLXR_CU_ERR_TIMEOUT or
 * MLXR_CU_ERR_DEVICE_INDEX. */
MLXR_CU_API int mlxr_cu_moe_status(const void* workspace, void* stream);

/* Reads and clears (synchronising on stream) the device status word the op
 * family (quantize ... gather_mm) shares on the current device:
 * MLXR_CU_ERR_DEVICE_INDEX when an lhs/rhs index was outside its batch (the
 * affected output blocks are left unwritten). There is one such word per
 * device for all host threads and streams: when ops run concurrently on
 * several streams, a status raised by one of them may be reported to (and
 * cleared by) a caller checking another, so check it with those streams
 * serialised. The block entry points keep their status in their own
 * workspace instead. */
MLXR_CU_API int mlxr_cu_op_status(void* stream);

/* Router alone (moe.rs:123-138): logits = bf16(fp32(x . gate[e]) + bias[e])
 * where x . gate[e] is the exact dot product of the bf16 rows rounded once
 * to fp32 (the same value whatever the summation order; T > 256 runs it on
 * the int8 tensor cores), softmax (fp32 inside, bf16 probabilities), top-k by (prob desc,
 * expert asc), renormalised bf16 weights. logits / probs [T, E] bf16 may be
 * NULL. Bit-exact with the routing contract the oracle states.
 * model_kind 1 (Gemma 4, text.rs:622-664): x is the layer's h; logits are
 * the scores of its RMS-normed input, top-k by (score desc, expert asc),
 * weights = softmax over the k scores times per_expert_scale; probs is not
 * written (the branch has no softmax over all experts). */
MLXR_CU_API int mlxr_cu_moe_router(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, const void* x,
                       int64_t num_tokens, int32_t* indices, void* topk_weights, void* logits, void* probs,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Permute alone (gather_sort, switch.rs:499-512): stable sort of the flat
 * rows by expert; x_sorted [T*K, D] bf16 receives x[sorted_rows[pos] / K]. */
MLXR_CU_API int mlxr_cu_moe_permute(const mlxr_cu_moe_config* cfg, const int32_t* indices, int64_t num_tokens, const void* x,
                        int32_t* counts, int32_t* offsets, int32_t* sorted_rows, int32_t* inverse, void* x_sorted,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Routed experts alone (SplitSwitchFfn::forward, switch.rs:417-442: gather_qmm
 * gate_proj and up_proj, swiglu, gather_qmm down_proj, without the sort and
 * unsort): y_rows[r] = down_e(silu(gate_e(x_rows[r])) * up_e(x_rows[r])), the
 * un-weighted output of expert e = row_experts[r], for the T*K rows
 * (num_tokens = T). Rows may come in any order; the natural input is the
 * permute step's x_sorted with the sorted experts, which keeps the expert
 * order. The workspace is the block forward's (mlxr_cu_moe_workspace_size). */
MLXR_CU_API int mlxr_cu_moe_experts(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights,
                        const int32_t* row_experts, int64_t num_tokens, const void* x_rows, void* y_rows,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Combine alone (scatter_unsort and the weighted sum over k, switch.rs:437-439
 * and 223-234, plus the shared branch, qwen3_5/text/moe.rs:118-120,144):
 * out[t] = sum_k topk_weights[t,k] * y_sorted[inverse[t*K+k]] (fp32 in k order)
 * + sigmoid(x[t] . shared_expert_gate) * shared_expert(x[t]); x may be NULL
 * without a shared expert. An inverse entry outside [0, T*K) is reported by
 * mlxr_cu_moe_status as MLXR_CU_ERR_DEVICE_INDEX. */
MLXR_CU_API int mlxr_cu_moe_combine(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, const void* x,
                        int64_t num_tokens, const void* y_sorted, const int32_t* inverse,
                        const void* topk_weights, void* out, void* workspace, size_t workspace_bytes,
                        void* stream);

/* ---------------------------------------------- expert parallelism -- */
/* No counterpart in the reference, which runs the whole block on one device
 * (Qwen35MoeBlock::forward, crates/mlxr-lm/src/qwen3_5/text/moe.rs:116-146,
 * has no collective). The block's experts are spread over `world` ranks, one
 * process per GPU: expert e lives on rank placement[e] >> 16 as that rank's
 * local expert placement[e] & 0xFFFF (a device int32 table [E]; NULL means
 * rank e % world, local expert e / world); the router and the shared expert
 * are replicated. A step on each rank, with the caller doing the two
 * exchanges (e.g. NCCL all-to-all):
 *   1. mlxr_cu_moe_ep_dispatch: route this rank's T tokens; list one pair per
 *      (token, destination rank) holding one of the token's experts, sorted
 *      by rank then token, with the token's x row and K slots of (local
 *      expert << 16 | bf16 top-k weight) in k order (-1 = empty slot).
 *   2. exchange: pairs for rank r (x_send rows and meta_send rows) go to r.
 *   3. mlxr_cu_moe_ep_experts: the received pairs through this rank's
 *      experts; each pair is reduced to one partial row (sum of w * expert
 *      output over its slots).
 *   4. exchange back: the partial rows return to their senders, in the order
 *      they were sent.
 *   5. mlxr_cu_moe_ep_combine: out[t] = sum of t's partial rows (in the order
 *      of the k that first named each rank) + sigmoid gate * shared expert.
 * Routing is bit-identical to the one-device block; outputs differ from it
 * only by the bf16 rounding of each partial row. The three steps of a rank
 * share one workspace: dispatch clears its status word, experts and combine
 * add their device-side checks to it, and mlxr_cu_moe_status reads it after
 * combine. */

/* Workspace for all three steps of one rank: num_tokens of its own tokens,
 * up to max_recv_pairs received pairs carrying up to max_recv_rows filled
 * slots (bounds: world * num_tokens pairs; pairs * K rows); sized for any
 * placement. */
MLXR_CU_API int mlxr_cu_moe_ep_workspace_size(const mlxr_cu_moe_config* cfg, int world, int64_t num_tokens,
                                              int64_t max_recv_pairs, int64_t max_recv_rows, size_t* bytes);

/* Step 1. send_counts [world][2] int32: pairs and filled slots for each
 * destination rank. pair_pos [T*K] int32: send position of the pair of
 * (t, k) when k is the first of t's experts on its rank, else -1. x_send
 * [T * min(K, world), D] bf16 and meta_send [T * min(K, world), K] int32
 * receive the pairs in send order (the first sum(pairs) rows are written).
 * shared_gate [T] fp32 (sigmoid of the shared-expert gate; NULL without a
 * shared expert) is kept for step 5. */
MLXR_CU_API int mlxr_cu_moe_ep_dispatch(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, int world,
                                        const int32_t* placement, const void* x, int64_t num_tokens, int32_t* send_counts, int32_t* pair_pos,
                                        void* x_send, int32_t* meta_send, float* shared_gate, void* workspace,
                                        size_t workspace_bytes, void* stream);

/* Step 3. cfg is the full block's configuration; local_weights hold this
 * rank's num_local_experts experts in local order (switch_* members only). x_recv
 * [num_pairs, D] bf16 and meta_recv [num_pairs, K] int32 as received;
 * num_rows = the filled slots among them (the sum of the received
 * send_counts[.][1]). partial [num_pairs, D] bf16 out. */
MLXR_CU_API int mlxr_cu_moe_ep_experts(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* local_weights,
                                       int num_local_experts, const void* x_recv, const int32_t* meta_recv, int64_t num_pairs,
                                       int64_t num_rows, void* partial, void* workspace, size_t workspace_bytes,
                                       void* stream);

/* Step 5. partial_back [num_pairs, D] bf16: the partial rows of this rank's
 * pairs, in send order; pair_pos and shared_gate from step 1; weights for
 * the shared expert (full block). out [T, D] bf16. */
MLXR_CU_API int mlxr_cu_moe_ep_combine(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights,
                                       const void* x, int64_t num_tokens, const void* partial_back, int64_t num_pairs,
                                       const int32_t* pair_pos, const float* shared_gate, void* out,
                                       void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------- expert parallelism over peer memory -- */
/* The same steps as above with the exchange done by the kernels over NVLink
 * (no counterpart in the reference). Every rank creates a communicator with
 * an exchange buffer sized for `cap` tokens per rank, shares its CUDA IPC
 * handle (MLXR_CU_IPC_HANDLE_BYTES bytes) with the other ranks (e.g. through
 * a host all-gather) and connects with all handles in rank order. Per step,
 * with the same `epoch` on every rank (1, 2, 3, ...):
 *   dispatch_p2p: route; store each pair straight into its destination's
 *     buffer; publish counts and a flag there;
 *   experts_p2p: wait (bounded) for every rank's flag; run the received
 *     pairs through the local experts; store each partial row straight into
 *     its owner's buffer; publish a flag there;
 *   combine_p2p: the shared expert, then wait for every rank's flag and add
 *     up each token's partial rows.
 * No host synchronisation is needed between the steps. A rank that never
 * publishes makes the others' waits expire after 10 s with
 * MLXR_CU_ERR_TIMEOUT in the status word. A rank whose own status word is
 * already non-zero when it publishes (a wait of its own expired, or it
 * skipped a bad index) publishes a poisoned flag instead, and every rank that
 * waits on it records the failure (mlxr_cu_moe_status then returns
 * MLXR_CU_ERR_TIMEOUT with a message naming a failed peer) instead of using
 * the rows. epoch must be in [1, 2^31) and grow by step; the top bit marks
 * the poison. epoch 0 (every step of the comm, on every rank) selects a
 * device-resident step counter instead: dispatch_p2p advances it in the
 * comm's buffer before any kernel of the step reads it, so a step captured
 * in a CUDA graph replays with a new epoch each time. A comm uses one kind
 * of epoch for its whole life. Ranks must be on different GPUs. */
#define MLXR_CU_IPC_HANDLE_BYTES 64

MLXR_CU_API int mlxr_cu_ep_comm_create(int world, int rank, int64_t cap, int hidden, int k, void** comm,
                                       void* ipc_handle);
MLXR_CU_API int mlxr_cu_ep_comm_connect(void* comm, const void* ipc_handles);
MLXR_CU_API int mlxr_cu_ep_comm_destroy(void* comm);

/* Workspace for one rank's three peer-memory steps; expected_rows (the
 * filled slots a rank usually receives, e.g. T_total * K / world) picks the
 * tile widths; the buffers hold the worst case. */
MLXR_CU_API int mlxr_cu_moe_ep_p2p_workspace_size(const mlxr_cu_moe_config* cfg, const void* comm, int64_t num_tokens,
                                                  int num_local_experts, int64_t expected_rows, size_t* bytes);

/* pair_pos [T*K] int32 out: where each pair's partial row comes back;
 * shared_gate [T] fp32 out as for mlxr_cu_moe_ep_dispatch. */
MLXR_CU_API int mlxr_cu_moe_ep_dispatch_p2p(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights,
                                            void* comm, const int32_t* placement, const void* x, int64_t num_tokens,
                                            int32_t* pair_pos, float* shared_gate, uint32_t epoch, void* workspace,
                                            size_t workspace_bytes, void* stream);
MLXR_CU_API int mlxr_cu_moe_ep_experts_p2p(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* local_weights,
                                           int num_local_experts, void* comm, int64_t expected_rows, uint32_t epoch,
                                           void* workspace, size_t workspace_bytes, void* stream);
MLXR_CU_API int mlxr_cu_moe_ep_combine_p2p(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights,
                                           void* comm, const void* x, int64_t num_tokens, const int32_t* pair_pos,
                                           const float* shared_gate, void* out, uint32_t epoch, void* workspace,
                                           size_t workspace_bytes, void* stream);

/* ------------------------------------------------ synthetic inputs -- */

/* Seeded N(0, stddev^2) samples rounded to bf16: Philox4x32-10 keyed by
 * seed, counter (pair index, stream), Box-Muller in fp64 (the generator the
 * benchmark configurations are defined with). */
MLXR_CU_API int mlxr_cu_synth_normal_bf16(uint64_t seed, uint64_t stream_id, int64_t n, float stddev, void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MLXR_MOE_H */
