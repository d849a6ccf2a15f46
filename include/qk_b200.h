/*
 * qk_b200.h - C ABI of the B200 (sm_100a) packed-quant MoE and Q8 KV-cache kernels.
 *
 * Plain pointers and sizes only. All device pointers refer to memory of the CUDA
 * device that is current on the calling thread; every call is asynchronous on
 * `stream` and returns a qk_status. No call allocates device memory: scratch space
 * is passed in as `workspace` (size from the matching *_workspace_bytes query).
 *
 * Reference interfaces (AhmadSaeedZaidi/data-synth-tpu, paths under kaggle/) are
 * cited beside each entry point. BF16 values are passed as uint16_t storage bits.
 *
 * Quantisation type codes are GGML's type numbers (QK_TYPE_*), the numbering the
 * reference's GGUF reader uses (glm53_offload/gguf_quant.py:31-39).
 */
#ifndef QK_B200_H
#define QK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* qk_stream_t; /* a cudaStream_t; NULL = legacy default stream */

typedef enum qk_status {
  QK_OK = 0,
  QK_ERR_INVALID_ARGUMENT = 1, /* bad shape, size, stride or null pointer   */
  QK_ERR_UNSUPPORTED_TYPE = 2, /* quantisation type not handled by the call */
  QK_ERR_NONFINITE_SCALE = 3,  /* a block scale is inf/NaN (repack refuses) */
  QK_ERR_CUDA = 4,             /* a CUDA runtime call or launch failed       */
  QK_ERR_TIMEOUT = 5,          /* a bounded device wait gave up              */
  QK_ERR_WORKSPACE = 6         /* workspace pointer missing or too small     */
} qk_status;

enum {
  QK_TYPE_F32 = 0,
  QK_TYPE_F16 = 1,
  QK_TYPE_Q4_0 = 2,
  QK_TYPE_Q4_1 = 3,
  QK_TYPE_Q5_0 = 6,
  QK_TYPE_Q5_1 = 7,
  QK_TYPE_Q8_0 = 8,
  QK_TYPE_Q4_K = 12,
  QK_TYPE_Q5_K = 13,
  QK_TYPE_Q6_K = 14,
  QK_TYPE_IQ4_NL = 20,
  QK_TYPE_BF16 = 30
};

enum { QK_OUT_F32 = 0, QK_OUT_BF16 = 1 };
/* Flag for qk_dequantize_tiled's out_dtype: decode with the fused multiply-add form the
 * GEMM kernels run (same values; a zero may carry the other sign). */
enum { QK_DECODE_FUSED = 0x100 };

/* ---- library ---------------------------------------------------------------- */

/* Version string "qk_b200 <major>.<minor> sm_100a". */
const char* qk_version(void);
/* Human-readable text of the last error set on this host thread (or ""). */
const char* qk_last_error(void);
/* Number of kernels this library has launched in this process (all devices). */
uint64_t qk_launch_count(void);

/* ---- GGUF block decode -------------------------------------------------------
 * Replaces glm53_offload/gguf_quant.py:180-216 dequantize_rows(raw, qtype,
 * row_width, dtype) and qwen38_tpu/quant.py:15-55 (Q4_0/Q4_1/Q5_0/Q5_1/IQ4_NL).
 * raw: uint8 [rows, ceil(row_width / values_per_block), bytes_per_block].
 * out: [rows, row_width] FP32 or BF16 (RNE, precision.py:7-23). Bit-exact. */
int qk_dequantize_rows(const uint8_t* raw, int qtype, int64_t rows, int64_t row_width,
                       int out_dtype, void* out, qk_stream_t stream);

/* ---- tiled repack (lossless) -------------------------------------------------
 * Replaces packed_q6/layout.py:49-108 pack_q6 / unpack_q6: a byte-only repack of raw
 * GGUF rows into the B200 tile layout (64 rows x 256 values per tile, rows padded to
 * 64) read by qk_quant_gemm and qk_moe_forward. Q6_K, Q4_K, Q5_K, and Q8_0 and Q5_1
 * (eight 32-value blocks per 256-value tile column).
 * bad_scales (device int32, may be NULL): receives the count of non-finite FP16 block
 * scales (pack_q6 rejects those, layout.py:67-69); the host wrapper raises on > 0. */
int64_t qk_tiled_bytes(int qtype, int64_t rows, int64_t row_width);
int qk_repack_rows(const uint8_t* raw, int qtype, int64_t rows, int64_t row_width,
                   uint8_t* tiled, int32_t* bad_scales, qk_stream_t stream);
int qk_unpack_rows(const uint8_t* tiled, int qtype, int64_t rows, int64_t row_width,
                   uint8_t* raw, qk_stream_t stream);
/* The reference's own TPU input form of a Q6_K projection (packed_q6/layout.py:49-91,
 * PackedQ6.data / PackedQ6.scales, layout "q6_k_soa_n64_k256_v1") back to GGUF rows
 * raw [rows, ceil(input_features / 256), 210]: the inverse byte transform of pack_q6
 * (unpack_q6, layout.py:93-108), on the device. Feed the rows to qk_repack_rows. */
int qk_q6_soa_to_rows(const uint8_t* data, const uint8_t* scales, int64_t rows,
                      int64_t input_features, uint8_t* raw, qk_stream_t stream);
/* Decode of the tiled layout through the GEMM kernels' in-register fragment decoder:
 * bit-identical to qk_dequantize_rows on the raw rows (signed zeros included), or with
 * out_dtype | QK_DECODE_FUSED the exact arithmetic the GEMM kernels run. */
int qk_dequantize_tiled(const uint8_t* tiled, int qtype, int64_t rows, int64_t row_width,
                        int out_dtype, void* out, qk_stream_t stream);

/* ---- packed projection -------------------------------------------------------
 * Replaces packed_q6/kernel.py:98-148 q6_matmul(x, packed, scales, output_features):
 * out[M, N] (FP32) = bf16 x[M, K] @ bf16(decode(W))[N, K]^T, FP32 accumulation on the
 * tcgen05 tensor core. w_tiled: qk_repack_rows output for W (any tiled type). Ragged M, N
 * and K allowed. The workspace holds x repacked into the tensor core's operand tiles and
 * the FP32 partial sum of every 256-value K block, added in K order at the end. */
size_t qk_quant_gemm_workspace_bytes(int64_t M, int64_t K, int64_t N);
int qk_quant_gemm(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_tiled, int qtype,
                  int64_t N, float* out, void* workspace, size_t workspace_bytes,
                  qk_stream_t stream);

/* ---- W8A8 projection ------------------------------------------------------------
 * Replaces qwen38_tpu/compute.py:20-34 q8_matmul(x, packed, output_dtype): the int8_q8
 * policy's integer dot over Q8_0 weights. Per row of x and 32-value group the activations
 * are quantised to int8 (scale max|x| / 127, rint, clip +-127), the int32 dot with the
 * weight codes runs on the tcgen05 tensor core (kind::i8), and the groups are added in order
 * as (f32(partial) * act_scale) * weight_scale (compute.py:52-65). x: BF16 [M, K], K a
 * multiple of 32; w_tiled: qk_repack_rows output of Q8_0 W [N, K]; out: [M, N] FP32 or BF16
 * (out_dtype). The workspace (256-byte aligned) holds x's operand tiles, codes and scales. */
size_t qk_q8_matmul_workspace_bytes(int64_t M, int64_t K, int64_t N);
int qk_q8_matmul(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_tiled, int64_t N,
                 int out_dtype, void* out, void* workspace, size_t workspace_bytes,
                 qk_stream_t stream);

/* ---- dense BF16 projection (decode batches) -------------------------------------
 * Replaces qwen38_tpu/math.py:10-16 linear(x, weight) for BF16 operands, as the decoder's
 * attention projections call it (attention_cache.py:131-134 q|gate, k, v; :171 out):
 * y = bf16(x @ w^T) with FP32 accumulation. x: BF16 [M, K] (1 <= M <= 256, K a multiple of
 * 64); w: BF16 [N, K]; y: BF16 [M, N]. A tcgen05 pass that streams w once, its K dimension
 * split over the SMs with FP32 partials added in a fixed order; for 1 <= M <= 4 a GEMV (a warp
 * per output column, FP32 fused multiply-adds and a butterfly), which checks the workspace
 * argument but does not touch it. Both are tested against FP64 within one BF16 ulp plus the
 * FP32 accumulation bound. The workspace (256-byte aligned, qk_linear_bf16_workspace_bytes)
 * must be zeroed once before its first call; every call leaves it ready for the next. Calls
 * sharing a workspace must not overlap. */
size_t qk_linear_bf16_workspace_bytes(int64_t M, int64_t K, int64_t N);
int qk_linear_bf16(const uint16_t* x, int64_t M, int64_t K, const uint16_t* w, int64_t N,
                   uint16_t* y, void* workspace, size_t workspace_bytes, qk_stream_t stream);
/* No counterpart in the reference. QK_ERR_TIMEOUT if a bounded device wait of an earlier
 * qk_linear_bf16 call on this workspace gave up (its output is then not valid), else QK_OK;
 * clears the flag. Synchronises `stream`. */
int qk_linear_bf16_check(const void* workspace, qk_stream_t stream);

/* ---- router ------------------------------------------------------------------
 * Replaces the router of qwen38_tpu/math.py:277-281 (routes_and_shared):
 * probs = softmax(f32(x) @ f32(Wr)^T); (w, ids) = top_k(probs, k) (ties: lower index);
 * w = w / sum(w); w = bf16(active ? w : 0).
 * x: BF16 [T, H]; router_w: FP32 [E, H]; active: uint8 [T] or NULL (all active).
 * ids: int32 [T, k]; weights: BF16 [T, k]; probs (FP32 [T, E], may be NULL). */
int qk_router_topk(const uint16_t* x, const float* router_w, const uint8_t* active, int T, int H,
                   int E, int k, int32_t* ids, uint16_t* weights, float* probs, qk_stream_t stream);
/* Same selection from precomputed FP32 logits [T, E] (one warp per token). */
int qk_router_topk_logits(const float* logits, const uint8_t* active, int T, int E, int k,
                          int32_t* ids, uint16_t* weights, float* probs, qk_stream_t stream);
/* The router's FP32 logits alone (math.py:277-281's linear(f32(x), f32(Wr)), HIGHEST
 * precision): logits [T, E] = x @ router_w^T, spread over ceil(E / 4) x ceil(T / 8) CTAs with
 * the per-row summation order of qk_router_topk, so the values are identical to the ones it
 * selects from. Followed by qk_router_topk_logits it is qk_router_topk in two launches for
 * callers that own a [T, E] FP32 buffer (the router matrix is then read by ~E / 4 SMs instead
 * of one 8-CTA cluster per 8 tokens). */
int qk_router_logits(const uint16_t* x, const float* router_w, int T, int H, int E, float* logits,
                     qk_stream_t stream);
/* qk_router_topk_logits followed by the shared expert's route (math.py:282-283) in one launch:
 * ids_out / weights_out [T, k + 1] hold each token's k routes, then (shared_id,
 * bf16(sigmoid(bf16(h . shared_router)))); h: BF16 [T, H], shared_router: BF16 [H]. With
 * experts_per_rank > 0 routed expert e is written as (e / experts_per_rank) *
 * (experts_per_rank + 1) + e % experts_per_rank (the numbering of
 * qk_append_shared_route_ep). Bit-identical to qk_router_topk_logits followed by
 * qk_append_shared_route[_ep]. */
int qk_router_select_shared(const float* logits, const uint8_t* active, int T, int E, int k,
                            const uint16_t* h, const uint16_t* shared_router, int H,
                            int shared_id, int experts_per_rank, int32_t* ids_out,
                            uint16_t* weights_out, qk_stream_t stream);

/* ---- routed expert FFN -------------------------------------------------------
 * Replaces the function returned by qwen38_tpu/experts.py:17-140 expert_parallel(mesh,
 * gate_type, up_type, down_type, hidden, intermediate, ...) and
 * qwen38_tpu/grouped_experts.py:21-163, called as fn(gate, up, down, x, ids, weights)
 * (engine.py:199-201), for this rank's experts [first_expert, first_expert + num_experts).
 * gate/up: tiled bytes [num_experts, qk_tiled_bytes(type, intermediate, hidden)];
 * down: tiled bytes [num_experts, qk_tiled_bytes(type, hidden, intermediate)].
 * x: BF16 [B, hidden]; ids: int32 [B, top_k]; weights: BF16 [B, top_k].
 * out: BF16 [B, hidden] (out_dtype QK_OUT_BF16), or the FP32 sum over this rank's
 * experts (QK_OUT_F32) that an expert-parallel all-reduce adds (experts.py:130-131). */
typedef struct qk_moe_desc {
  int gate_type, up_type, down_type; /* gate == up: Q6_K, Q4_K or Q5_K; down: Q6_K,
                                        Q4_K, Q8_0 or Q5_1 (the reference
                                        checkpoints' types, checkpoints/q4.json, q6.json) */
  int hidden;                        /* multiple of 256                          */
  int intermediate;                  /* multiple of the down block: 256, or 32 (Q8_0, Q5_1) */
  int num_experts;                   /* experts held by this rank                */
  int first_expert;                  /* global id of this rank's first expert    */
  int top_k;                         /* routes per token                         */
  int compute;                       /* QK_COMPUTE_BF16 (0), or QK_COMPUTE_INT8_Q8: a
                                        Q8_0 down projection as the W8A8 integer dot of
                                        qwen38_tpu/compute.py:20-34 (tcgen05 kind::i8);
                                        other types compute as BF16 (experts.py:85-99) */
} qk_moe_desc;
enum { QK_COMPUTE_BF16 = 0, QK_COMPUTE_INT8_Q8 = 1 };

size_t qk_moe_workspace_bytes(const qk_moe_desc* desc, int max_tokens);
int qk_moe_forward(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up,
                   const uint8_t* down, const uint16_t* x, const int32_t* ids,
                   const uint16_t* weights, int B, int out_dtype, void* out, void* workspace,
                   size_t workspace_bytes, qk_stream_t stream);
/* qk_moe_forward that also records cudaEvent_t events[0..4] on `stream` before the
 * route, gate/up, down and combine launches and after the last one (NULL entries are
 * skipped): the per-kernel timing the benchmark reports. */
int qk_moe_forward_profiled(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up,
                            const uint8_t* down, const uint16_t* x, const int32_t* ids,
                            const uint16_t* weights, int B, int out_dtype, void* out,
                            void* workspace, size_t workspace_bytes, qk_stream_t stream,
                            void* const* events);
/* Tensor parallel inside the experts (grouped_experts.py:113-119, tensor_parallel > 1):
 * each tensor rank holds every expert's slice of I (desc->intermediate = I / tp, a
 * multiple of 256: whole down blocks, parallel.py:40-61). qk_moe_forward_tp_partial runs
 * route, dispatch, gate/up + SwiGLU and down for this slice and writes the FP32 down
 * projection of every route to y_routes [B * top_k, hidden] (16-byte aligned; rows of
 * merged or dropped routes are left as they were). The caller all-reduces y_routes over
 * the tensor ranks (the reference's psum before the BF16 rounding) and then calls
 * qk_moe_forward_tp_combine with the same workspace, which rounds each route's sum to
 * BF16 and adds f32(y) * f32(route weight) in ascending expert order. */
int qk_moe_forward_tp_partial(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up,
                              const uint8_t* down, const uint16_t* x, const int32_t* ids,
                              const uint16_t* weights, int B, float* y_routes, void* workspace,
                              size_t workspace_bytes, qk_stream_t stream);
int qk_moe_forward_tp_combine(const qk_moe_desc* desc, const float* y_routes, const int32_t* ids,
                              int B, int out_dtype, void* out, void* workspace,
                              size_t workspace_bytes, qk_stream_t stream);
/* BF16 (RNE) of an FP32 array: the cast after the expert-parallel all-reduce
 * (experts.py:131, psum(out).astype(x.dtype)). */
int qk_cast_f32_bf16(const float* in, uint16_t* out, int64_t n, qk_stream_t stream);
/* Status word the kernels of the last qk_moe_forward on `workspace` left behind:
 * 0, or QK_ERR_TIMEOUT when a bounded wait gave up. Synchronises `stream`. */
int qk_moe_check(const void* workspace, qk_stream_t stream);

/* ---- expert parallel with token dispatch ---------------------------------------
 * The dispatch / combine form of the expert-parallel layer that the reference expresses as
 * replicated tokens plus psum (qwen38_tpu/experts.py:130-131; placement parallel.py:64-87):
 * rank r owns experts [r * experts_per_rank, (r + 1) * experts_per_rank) and sends each
 * route's token row to the owning rank, which returns bf16(h Wd^T) for it.
 * qk_ep_plan: per token, routes naming the same expert merge into the first one with weight
 * bf16(sum) and zero-weight routes drop (experts.py:66-76); surviving routes are counting-
 * sorted by owning rank: send_counts [world], send_rows / send_expert [B * k] (token and
 * global expert of each send slot, rank-major), route_slot [B * k] (slot of route (b, j)
 * or -1), route_weight [B * k] (merged FP32 weight, 0 when dropped). */
int qk_ep_plan(const int32_t* ids, const uint16_t* weights, int B, int k, int experts_per_rank,
               int world, int32_t* send_counts, int32_t* send_rows, int32_t* send_expert,
               int32_t* route_slot, float* route_weight, qk_stream_t stream);
/* dst[i, :] = src[rows[i], :] for BF16 rows of `width` values (16-byte aligned). */
int qk_gather_rows(const uint16_t* src, const int32_t* rows, int64_t n, int64_t width, uint16_t* dst,
                   qk_stream_t stream);
/* out[b] = bf16 (or FP32 with QK_OUT_F32) of the FP32 sum over token b's surviving routes,
 * in ascending expert order, of f32(y[route_slot[b, j]]) * route_weight[b, j]
 * (experts.py:129-131). y: BF16 [slots, H], the returned expert outputs in send-slot order. */
int qk_ep_combine(const uint16_t* y, const int32_t* route_slot, const int32_t* ids,
                  const float* route_weight, int B, int k, int H, int out_dtype, void* out,
                  qk_stream_t stream);

/* ---- expert parallel over peer memory (no host synchronisation) ---------------------
 * The same layer as experts.py:61-131 with experts sharded over ranks (parallel.py:64-87)
 * and each rank keeping its own tokens. Every rank allocates one exchange region of
 * qk_ep_p2p_bytes() bytes (qk_device_alloc), clears its control words (qk_ep_p2p_reset),
 * exports it (qk_ipc_get_handle) and maps every peer's (qk_ipc_open_handle); `peers` is a
 * DEVICE array of `world` region pointers as mapped in this process (its own at [rank]).
 * A step is three stream-ordered calls on every rank, with the same max_tokens everywhere:
 * qk_ep_p2p_dispatch stores each token row once into every owner of one of its routed
 * experts (slot = token index, so no counts cross ranks); qk_ep_p2p_expert runs this rank's
 * experts over the received slots and stores each slot's FP32 partial (ascending expert
 * order) back into its source; qk_ep_p2p_combine adds a token's partials in ascending rank
 * order and rounds once to BF16 (experts.py:128-131: local sum, psum, cast). Waits on peers
 * are bounded; qk_ep_p2p_status reports one that gave up (QK_ERR_TIMEOUT). No call
 * allocates, and all sizes are fixed by (world, max_tokens), so a step can be captured in
 * a CUDA graph. */
size_t qk_ep_p2p_bytes(int world, int max_tokens, int hidden, int top_k);
int qk_ep_p2p_reset(void* region, qk_stream_t stream);
int qk_ep_p2p_status(const void* region, qk_stream_t stream);
int qk_ep_p2p_dispatch(void* const* peers, void* region, int world, int rank, int max_tokens,
                       int hidden, int top_k, int experts_per_rank, const uint16_t* x,
                       const int32_t* ids, const uint16_t* weights, int B, qk_stream_t stream);
/* desc: this rank's experts (num_experts = experts_per_rank, first_expert = rank *
 * experts_per_rank); workspace of qk_moe_workspace_bytes(desc, world * max_tokens). */
int qk_ep_p2p_expert(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up,
                     const uint8_t* down, void* const* peers, void* region, int world, int rank,
                     int max_tokens, void* workspace, size_t workspace_bytes, qk_stream_t stream);
/* qk_ep_p2p_expert with CUDA events (5, cudaEvent_t) recorded before the route kernel and
 * after the dispatch, gate/up, down and combine-and-return passes, as qk_moe_forward_profiled
 * does; for stage timing. */
int qk_ep_p2p_expert_profiled(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up,
                              const uint8_t* down, void* const* peers, void* region, int world, int rank,
                              int max_tokens, void* workspace, size_t workspace_bytes, qk_stream_t stream,
                              void* const* events);
int qk_ep_p2p_combine(void* region, int world, int rank, int max_tokens, int hidden, int top_k,
                      int experts_per_rank, const int32_t* ids, const uint16_t* weights, int B,
                      uint16_t* out, qk_stream_t stream);
/* Device memory another process of the node can map: cudaMalloc / cudaFree and the CUDA
 * IPC handle (64 bytes) of an allocation, opened with peer access enabled. */
int qk_device_alloc(size_t bytes, void** ptr);
int qk_device_free(void* ptr);
int qk_ipc_get_handle(void* ptr, uint8_t* handle64);
int qk_ipc_open_handle(const uint8_t* handle64, void** ptr);
int qk_ipc_close_handle(void* ptr);

/* ---- Q8 KV cache -------------------------------------------------------------
 * Cache layout is the reference's (attention_cache.py:26-43, engine.py:350-369):
 * codes int8 [B, T, kv_heads * head_dim]; scale planes BF16 [B * G, T] with
 * G = kv_heads * head_dim / group and group = min(32, head_dim) (config.py:91-93). */

/* attention_cache.py:15-23 quantize(x, group): x [rows, width] (BF16 or FP32 by
 * in_dtype QK_OUT_*); codes int8 [rows, width]; scales BF16 [rows, width / group]. */
int qk_kv_q8_quantize(const void* x, int in_dtype, int64_t rows, int width, int group,
                      int8_t* codes, uint16_t* scales, qk_stream_t stream);
/* attention_cache.py:26-43 write_quantized(cache, key, value, indices, active, c):
 * key/value [B, kv_heads, head_dim] (BF16 or FP32 by in_dtype); time [B] int32;
 * active uint8 [B] or NULL. In place. Negative times wrap once; out-of-range drop. */
int qk_kv_q8_append(const void* key, const void* value, int in_dtype, const int32_t* time,
                    const uint8_t* active, int8_t* k_codes, int8_t* v_codes, uint16_t* k_scale,
                    uint16_t* v_scale, int B, int T, int kv_heads, int head_dim,
                    qk_stream_t stream);
/* A prompt chunk of W tokens per cache row (the write of the chunked prefill,
 * engine.py:449-500 forward_chunk through attention_cache.py:26-43): key/value
 * [B * W, kv_heads, head_dim]; token j of row b is written at time start[b] + j. */
int qk_kv_q8_append_chunk(const void* key, const void* value, int in_dtype, const int32_t* start,
                          const uint8_t* active, int8_t* k_codes, int8_t* v_codes, uint16_t* k_scale,
                          uint16_t* v_scale, int B, int W, int T, int kv_heads, int head_dim,
                          qk_stream_t stream);
/* attention_cache.py:46-68 gather_scale_plane(plane, indices, groups): out BF16
 * [B, S, groups]; negative indices wrap once, then clamp (test_qwen38_kv_gather.py:22-32). */
int qk_kv_q8_gather_scales(const uint16_t* plane, const int32_t* indices, int B, int S,
                           int groups, int T, uint16_t* out, qk_stream_t stream);
/* attention_cache.py:71-81 read_quantized(cache, name, indices, c, dtype): out
 * [B, S, kv_heads, head_dim] FP32 or BF16 = compute_cast(code * scale). */
int qk_kv_q8_read(const int8_t* codes, const uint16_t* plane, const int32_t* indices, int B,
                  int S, int T, int kv_heads, int head_dim, int out_dtype, void* out,
                  qk_stream_t stream);

/* Decode attention over the Q8 cache, attention_cache.py:152-170 (step after the
 * cache write): GQA scores bf16(q.k), bf16(/sqrt(hd)), masked softmax, PV with FP32
 * accumulation, bf16, then bf16(o * bf16(sigmoid(gate))) when gate != NULL.
 * q: BF16 [B, hq, hd]; indices: int32 [B, S] cache times of the S slots (a page table
 * expands to indices[b, s] = page[b, s / P] * P + s % P); valid: uint8 [B, S] or NULL,
 * in which case slot s is valid iff s <= lengths[b]; out: BF16 [B, hq, hd].
 * Split-KV: one CTA per SM takes an equal, contiguous range of all pairs' 16-slot tiles; a
 * (b, kv head) pair cut by CTA boundaries leaves one partial (max, sum, out) per CTA in the
 * workspace for an LSE merge. It is at most 2 * SMs * kv * (16 + 8 * hd) * 4 bytes, whatever
 * B and S are. */
size_t qk_kv_q8_attention_workspace_bytes(int B, int S, int hq, int kv_heads, int head_dim);
int qk_kv_q8_decode_attention(const uint16_t* q, const int8_t* k_codes, const int8_t* v_codes,
                              const uint16_t* k_scale, const uint16_t* v_scale,
                              const int32_t* indices, const uint8_t* valid,
                              const int32_t* lengths, const uint16_t* gate, int B, int S, int T,
                              int hq, int kv_heads, int head_dim, uint16_t* out, void* workspace,
                              size_t workspace_bytes, qk_stream_t stream);

/* Time-sharded decode attention: the cache's time axis split over ranks, as the reference
 * shards it (engine.py:350-369, P(None, "expert", ...) on the time axis of the codes and
 * the scale planes, with attention_cache.py:152-170 reduced over the shards by SPMD).
 * qk_kv_q8_decode_attention_partial runs the same split-KV kernel over this rank's slots
 * and writes, in place of the BF16 output, one partial set (16-byte aligned, FP32):
 * B * hq * head_dim unnormalised outputs, then B * hq pairs (max score, sum of
 * exp(score - max)); a row with no valid slot has max -inf and sum 0. Same workspace as
 * qk_kv_q8_decode_attention. */
int qk_kv_q8_decode_attention_partial(const uint16_t* q, const int8_t* k_codes,
                                      const int8_t* v_codes, const uint16_t* k_scale,
                                      const uint16_t* v_scale, const int32_t* indices,
                                      const uint8_t* valid, const int32_t* lengths, int B, int S,
                                      int T, int hq, int kv_heads, int head_dim, float* partial,
                                      void* workspace, size_t workspace_bytes, qk_stream_t stream);
/* Log-sum-exp combine of R consecutive partial sets (e.g. all-gathered from R ranks, rank
 * order = time order), merged in set order, then the output rule of
 * attention_cache.py:169-170: out = bf16(bf16(o) * bf16(sigmoid(gate))) when gate != NULL.
 * out: BF16 [B, hq, head_dim]. */
int qk_kv_q8_attention_combine(const float* parts, int R, int B, int hq, int head_dim,
                               const uint16_t* gate, uint16_t* out, qk_stream_t stream);

/* ---- sparse token selection (QSA indexer) -------------------------------------
 * Replaces the selection half of attention_cache.py:84-125 select_tokens, once the block
 * keys are current. qk_qsa_block_scores: query BF16 [B, heads, dim] (normed, rotated),
 * keys BF16 [B, blocks, dim] (16-byte aligned), lengths int32 [B] -> scores FP32
 * [B, blocks] = sum_h relu(q_h . k_t) / sqrt(dim) for t < (lengths + 1) / ratio, else -inf
 * (:100-114). heads <= 8, dim in {64, 128, 256}. qk_qsa_select: top K = min(budget / ratio,
 * blocks) blocks per row (lax.top_k order: score descending, ties to the lower block) ->
 * indices int32 / valid uint8 [B, K * ratio + ratio - 1]: the selected blocks' tokens, then
 * the ratio - 1 tail tokens, invalid entries index 0 (:115-124). blocks <= 16384, K <= 1024. */
int qk_qsa_block_scores(const uint16_t* query, const uint16_t* keys, const int32_t* lengths, int B,
                        int heads, int dim, int blocks, int ratio, float* scores,
                        qk_stream_t stream);
int qk_qsa_select(const float* scores, const int32_t* lengths, int B, int blocks, int ratio,
                  int budget, int32_t* indices, uint8_t* valid, qk_stream_t stream);
/* The key-maintenance half of select_tokens (attention_cache.py:86-99). Rotary (math.py:
 * 231-243) with three position components: pair i (i < rotary / 2) turns by
 * positions[b, axis[i]] * inv_freq[i], cosine and sine rounded to BF16.
 * qk_qsa_update_keys: raw_k BF16 [B, dim] (linear(x, index_k)); for active rows (active
 * uint8 [B] or NULL) writes it to tail BF16 [B, ratio, dim] at slot lengths % ratio, copies
 * positions int32 [B, 3] to starts [B, 3] on slot 0, pools the tail (FP32 mean, BF16),
 * normalises (k_norm) and rotates it at the block start, and on slot ratio - 1 stores it to
 * keys BF16 [B, blocks, dim] at block lengths / ratio. qk_qsa_query: raw_q BF16
 * [B, heads, dim] (linear(x, index_q)) -> query = rope(rms(raw_q, q_norm), positions). */
int qk_qsa_update_keys(const uint16_t* raw_k, const int32_t* lengths, const int32_t* positions,
                       const uint8_t* active, const uint16_t* k_norm, float eps, const float* inv_freq,
                       const int32_t* axis, int rotary, int B, int ratio, int dim, int blocks,
                       uint16_t* tail, int32_t* starts, uint16_t* keys, qk_stream_t stream);
int qk_qsa_query(const uint16_t* raw_q, const int32_t* positions, const uint16_t* q_norm, float eps,
                 const float* inv_freq, const int32_t* axis, int rotary, int B, int heads, int dim,
                 uint16_t* query, qk_stream_t stream);

/* ---- decoder-layer glue around the path -----------------------------------------
 * The per-token steps on either side of the routed FFN and the decode attention in a
 * decoder layer, one launch each over all rows (BF16 storage bits throughout). */

/* qwen38_tpu/math.py:27-31 rms(x, gamma, eps): out = bf16(x * rsqrt(mean(x^2) + eps) *
 * gamma) per row of `width` values. */
int qk_rms_norm(const uint16_t* x, const uint16_t* gamma, int rows, int width, float eps,
                uint16_t* out, qk_stream_t stream);
/* qwen38_tpu/attention_cache.py:129-135 (q/gate split, q_norm / k_norm rms, rope of
 * math.py:231-243 with one position per row for every rotary section). qkv: the fused
 * projection rows [B, hq * (q hd | gate hd) + kv * hd (k) + kv * hd (v)]; inv_freq: FP32
 * [rotary_dim / 2]; positions: int32 [B]. Outputs q, gate [B, hq, hd], k, v [B, kv, hd]. */
int qk_qk_norm_rope(const uint16_t* qkv, const uint16_t* q_norm, const uint16_t* k_norm,
                    const float* inv_freq, const int32_t* positions, int B, int hq, int kv,
                    int head_dim, int rotary_dim, float eps, uint16_t* q_out,
                    uint16_t* gate_out, uint16_t* k_out, uint16_t* v_out, qk_stream_t stream);
/* The residual add followed by the next RMSNorm (math.py:27-31), one launch: x_out =
 * bf16(x + y) [rows, width] (x_out may alias x), out = rms(x_out, gamma, eps). Bit-identical
 * to qk_residual_add then qk_rms_norm. */
int qk_residual_rms_norm(const uint16_t* x, const uint16_t* y, const uint16_t* gamma, int rows,
                         int width, float eps, uint16_t* x_out, uint16_t* out,
                         qk_stream_t stream);
/* out = bf16(x + y) over n BF16 values (out may alias x): the residual add. */
int qk_residual_add(const uint16_t* x, const uint16_t* y, int64_t n, uint16_t* out,
                    qk_stream_t stream);
/* The shared expert as one more route (math.py:282-283): ids_out / weights_out [B, k + 1]
 * are the k routes of each row followed by (shared_id, bf16(sigmoid(bf16(h . shared_router)))),
 * so one qk_moe_forward over routed + shared experts applies the shared expert's gate. */
int qk_append_shared_route(const int32_t* ids, const uint16_t* weights, int B, int k,
                           const uint16_t* h, const uint16_t* shared_router, int H,
                           int shared_id, int32_t* ids_out, uint16_t* weights_out,
                           qk_stream_t stream);
/* The expert-parallel form of qk_append_shared_route: every rank holds its slice of
 * experts_per_rank routed experts followed by its own copy of the shared expert, so routed id
 * e becomes (e / experts_per_rank) * (experts_per_rank + 1) + e % experts_per_rank and the
 * shared route names this rank's copy, rank * (experts_per_rank + 1) + experts_per_rank
 * (math.py:282-283 with the experts placed as parallel.py:64-87 places them). */
int qk_append_shared_route_ep(const int32_t* ids, const uint16_t* weights, int B, int k,
                              const uint16_t* h, const uint16_t* shared_router, int H,
                              int experts_per_rank, int rank, int32_t* ids_out,
                              uint16_t* weights_out, qk_stream_t stream);

/* qwen38_tpu/run.py:46-55 checked_argmax(logits): out int32 [B, 2] = (argmax over the V
 * logits of the row - the first maximum, a NaN counting as the maximum, as jnp.argmax -
 * and the number of non-finite logits in the row). logits: [B, V] FP32 or BF16 (in_dtype
 * QK_OUT_F32 / QK_OUT_BF16). */
int qk_checked_argmax(const void* logits, int in_dtype, int B, int64_t V, int32_t* out,
                      qk_stream_t stream);

/* No counterpart in the reference. QK_ERR_TIMEOUT if a bounded device wait of an earlier
 * qk_kv_q8_decode_attention on this device gave up (its output is then not valid), else
 * QK_OK; clears the flag. Synchronises `stream`. */
int qk_kv_q8_attention_check(qk_stream_t stream);

/* Replaces the FP32 elementary functions of qwen38_tpu/numerics.py:13-51 (exp, divide,
 * sigmoid, softmax) as the kernels compute them, for the reference's FP64 validation
 * (numerics_validation.py:12-74, 5e-7 relative budget). Elementwise over n FP32 values:
 * out = exp(a), sigmoid(a), a / b (b read only by QK_NUM_DIVIDE), or the SwiGLU
 * activation bf16(bf16(a) * sigmoid(bf16(a))); QK_NUM_SOFTMAX normalises rows of row_len
 * values (n a multiple of row_len) exactly as the router kernel does. */
enum { QK_NUM_EXP = 0, QK_NUM_SIGMOID = 1, QK_NUM_DIVIDE = 2, QK_NUM_SOFTMAX = 3, QK_NUM_SILU_BF16 = 4 };
int qk_numerics(int op, const float* a, const float* b, float* out, int64_t n, int row_len,
                qk_stream_t stream);

/* No counterpart in the reference. qk_kv_q8_decode_attention without a workspace, for
 * callers that cannot provide device memory at the call. The split scratch is a fixed
 * 16 MiB array in the library's device image (QK_ATTN_STATIC_SCRATCH_BYTES). A geometry
 * whose qk_kv_q8_attention_workspace_bytes() exceeds it returns QK_ERR_WORKSPACE and
 * runs nothing: the need is 2 * SMs * kv_heads * (16 + 8 * head_dim) * 4 bytes, so on a
 * 148-SM B200 kv_heads * head_dim >= 2048 is refused. The first call on a device looks up the array's address, so make it
 * before any stream capture. The scratch is shared per device, so overlapping calls
 * (other streams or threads) race on it; calls in order on one stream are safe. */
#define QK_ATTN_STATIC_SCRATCH_BYTES (16u << 20)
int qk_kv_q8_decode_attention_noalloc(const uint16_t* q, const int8_t* k_codes,
                                      const int8_t* v_codes, const uint16_t* k_scale,
                                      const uint16_t* v_scale, const int32_t* indices,
                                      const uint8_t* valid, const int32_t* lengths,
                                      const uint16_t* gate, int B, int S, int T, int hq,
                                      int kv_heads, int head_dim, uint16_t* out,
                                      qk_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* QK_B200_H */
