/*
 * lightning_router.h -- C ABI of the B200 (sm_100a) MoE-layer hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream, is
 * stream-ordered, never allocates or frees device memory (scratch is passed in
 * as a workspace whose size is reported by a *_workspace_bytes query), and
 * returns 0 on success or a negative LR_* status (see lr_status_string).
 * Device-detected contract violations (an expert id out of range, a pipeline
 * wait that ran out of time) are OR-ed into the optional `err` word, which the
 * caller reads back when it chooses.
 *
 * Each entry point names the reference (AlexanderLeonida/LLM-Serving-Kernel-
 * Optimization) interface it replaces.
 */
#ifndef LIGHTNING_ROUTER_H
#define LIGHTNING_ROUTER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct CUstream_st;
typedef struct CUstream_st* lr_stream_t; /* == cudaStream_t */

/* ---- status ------------------------------------------------------------ */
#define LR_OK 0
#define LR_ERR_INVALID_ARGUMENT (-1)
#define LR_ERR_UNSUPPORTED (-2)
#define LR_ERR_CUDA (-3)
#define LR_ERR_WORKSPACE (-4)
#define LR_ERR_NO_DEVICE (-5)
#define LR_ERR_TOO_LARGE (-6) /* exceeds the fixed scratch of the allocation-free entry point */

/* bits OR-ed into the device `err` word */
#define LR_DEVERR_BAD_EXPERT 0x1     /* an expert id outside [0, E) */
#define LR_DEVERR_BAD_TOKEN 0x2      /* a source token outside [0, T) */
#define LR_DEVERR_PIPE_TIMEOUT 0x4   /* a GEMM pipeline wait ran out of time */
#define LR_DEVERR_BAD_SEGMENT 0x8    /* a GEMM row segment outside the row range */
#define LR_DEVERR_PEER_TIMEOUT 0x10  /* another rank's exchange flag did not arrive in time */

const char* lr_status_string(int status);
int lr_abi_version(void);
/* Last CUDA runtime error seen by an entry point on this thread (0 if none). */
int lr_last_cuda_error(void);

/* ---- gate projection --------------------------------------------------- */
/* logits[T,E] (fp32) = h[T,d] (fp16) . wg[E,d]^T (fp16) (+ bias[E] fp32).
 * Replaces TopKGating.gate_proj, lightning_router/models/gating.py:46,69.
 * Limits: d % 16 == 0, 1 <= E <= 256.                                      */
int lr_gate_logits(const void* h, const void* wg, const float* bias, int T, int d, int E,
                   float* logits, lr_stream_t stream);

/* ---- gating + dispatch -------------------------------------------------- */
size_t lr_route_workspace_bytes(int num_tokens, int top_k, int num_experts);

/* Fused top-k softmax gating and capacity-masked dispatch from fp32 logits.
 * Replaces TopKGating.forward (lightning_router/models/gating.py:48-101)
 * followed by expert_routing_forward (lightning_router/kernels/expert_routing.py:164-230).
 * Slot s = t*k + j, j in descending-logit order (ties: lowest expert index).
 * Outputs (S = T*k):
 *   expert_ids[S] int32, gate_weights[S] fp32, token_indices[S] int32 (nullable),
 *   offsets[E+1] int32 (UNCAPPED CSR, as the reference), kept_counts[E] int32,
 *   aux_loss[1] fp32 (nullable; Switch load-balancing loss, gating.py:91-99),
 *   permuted[S,d] fp16 (nullable => routing only), routing_w[S] fp32,
 *   source_idx[S] int32, slot_pos[S] int32 (row of each slot or -1 if dropped).
 * Rows of expert e occupy [offsets[e], offsets[e+1]); the first kept_counts[e]
 * are its kept slots in slot order.  A dropped slot's row has routing_w = 0,
 * source_idx = its token and (if fill_dropped) zeros.
 * Limits: E <= 64, 1 <= k <= min(E, 8), d % 8 == 0.                        */
int lr_topk_gating_dispatch(const void* x, const float* logits, int T, int d, int E, int k,
                            int capacity, float load_balance_weight, int fill_dropped,
                            int32_t* expert_ids, float* gate_weights, int32_t* token_indices,
                            int32_t* offsets, int32_t* kept_counts, float* aux_loss,
                            void* permuted, float* routing_w, int32_t* source_idx,
                            int32_t* slot_pos, void* workspace, size_t workspace_bytes,
                            int32_t* err, lr_stream_t stream);

/* Gate projection + lr_topk_gating_dispatch in one call (the reference's
 * TopKGating.forward from hidden states, gating.py:48-101, then
 * expert_routing_forward).  x[T,d] fp16 is both the gate input and the rows
 * to permute; gate_weight[E,d] fp16, bias[E] fp32 (nullable); logits[T,E]
 * fp32 receives the logits.  Other arguments and outputs as
 * lr_topk_gating_dispatch.  For T <= 256 the projection, top-k, ranks,
 * offsets and aux loss run in one launch and the row copy in a second; the
 * logits are bit-identical to lr_gate_logits.  Larger T runs lr_gate_logits
 * then lr_topk_gating_dispatch.  The workspace is
 * lr_gate_dispatch_workspace_bytes(T, k, E).
 * Limits: d % 16 == 0, E <= 64, 1 <= k <= min(E, 8); x, gate_weight and
 * permuted 16-byte aligned.                                                */
size_t lr_gate_dispatch_workspace_bytes(int num_tokens, int top_k, int num_experts);
int lr_gate_topk_gating_dispatch(const void* x, const void* gate_weight, const float* bias, int T,
                                 int d, int E, int k, int capacity, float load_balance_weight,
                                 int fill_dropped, float* logits, int32_t* expert_ids,
                                 float* gate_weights, int32_t* token_indices, int32_t* offsets,
                                 int32_t* kept_counts, float* aux_loss, void* permuted,
                                 float* routing_w, int32_t* source_idx, int32_t* slot_pos,
                                 void* workspace, size_t workspace_bytes, int32_t* err,
                                 lr_stream_t stream);

/* The two phases of lr_topk_gating_dispatch, for expert-parallel callers that
 * exchange per-expert counts between them.
 * lr_topk_route: gating, slot ranks inside their 256-token route blocks (left in
 * slot_pos), local uncapped CSR `offsets`, kept_counts = min(count, capacity),
 * the local aux loss and, if prob_sums != NULL, the per-expert sums of softmax
 * probabilities over the T tokens (fp64).  The workspace carries the per-block
 * bases to lr_permute_tokens and must not be reused in between.
 * lr_permute_tokens: a slot whose rank inside this shard's expert segment is r
 * is kept iff rank_base[e] + r < capacity (rank_base NULL => 0; rank_base[e] =
 * slots of expert e in lower shards, so capacity follows the global slot
 * order) and goes to row row_offsets[e] + r.  With compact != 0 dropped slots
 * get no row (row_offsets then spans kept rows only) and slot_pos = -1.      */
int lr_topk_route(const float* logits, int T, int E, int k, int capacity,
                  float load_balance_weight, int32_t* expert_ids, float* gate_weights,
                  int32_t* token_indices, int32_t* offsets, int32_t* kept_counts,
                  float* aux_loss, double* prob_sums, int32_t* slot_pos, void* workspace,
                  size_t workspace_bytes, int32_t* err, lr_stream_t stream);
int lr_permute_tokens(const void* x, int T, int d, int E, int k, int capacity,
                      const int32_t* expert_ids, const float* gate_weights,
                      const int32_t* row_offsets, const int32_t* rank_base, int compact,
                      int fill_dropped, int32_t* slot_pos, void* permuted, float* routing_w,
                      int32_t* source_idx, const void* workspace, size_t workspace_bytes,
                      lr_stream_t stream);

/* Allocation-free variant of lr_topk_gating_dispatch (no counterpart in the
 * reference).  Same arguments and results, minus the workspace.  It is for
 * callers that cannot allocate device memory: a serving host that owns all of
 * it and passes this library pre-sized input and output buffers but no
 * allocator, or a latency-critical loop where cudaMalloc, which synchronises
 * the device, is not allowed.  Its scratch is a 1 MiB file-scope device array
 * inside this library, held by every GPU that loads the library until the
 * process exits, so 256 + 16 * ceil(T/256) * E bytes (each part rounded up to
 * 256) must fit in 1 MiB: about 2 M tokens at E = 8, about 260 K tokens at
 * E = 64.  Larger sizes return LR_ERR_TOO_LARGE before any work is queued.
 * The first call on a device looks the array's device address up
 * (cudaGetSymbolAddress) with that device current, and so does the first call
 * after the device's context changed (a cudaDeviceReset); make such a call
 * before any stream capture begins.  Every call uses the same array and clears the
 * part that must start at zero, so calls that overlap on the GPU (other
 * streams, other host threads) race and must be serialised by the caller.
 * It allocates and frees nothing.                                          */
int lr_topk_gating_dispatch_noalloc(const void* x, const float* logits, int T, int d, int E,
                                    int k, int capacity, float load_balance_weight,
                                    int fill_dropped, int32_t* expert_ids, float* gate_weights,
                                    int32_t* token_indices, int32_t* offsets,
                                    int32_t* kept_counts, float* aux_loss, void* permuted,
                                    float* routing_w, int32_t* source_idx, int32_t* slot_pos,
                                    int32_t* err, lr_stream_t stream);

size_t lr_dispatch_workspace_bytes(int num_slots, int num_experts);

/* Dispatch of precomputed slots (expert id, gate weight, source token per slot).
 * Replaces expert_routing_forward, lightning_router/kernels/expert_routing.py:164-230.
 * Same output layout as lr_topk_gating_dispatch.  Limits: E <= 1024, d % 8 == 0. */
int lr_expert_routing_forward(const void* tokens, const int32_t* expert_ids,
                              const float* gate_weights, const int32_t* token_indices,
                              int T, int d, int S, int E, int capacity, int fill_dropped,
                              void* permuted, int32_t* offsets, float* routing_w,
                              int32_t* source_idx, int32_t* kept_counts, int32_t* slot_pos,
                              void* workspace, size_t workspace_bytes, int32_t* err,
                              lr_stream_t stream);

/* ---- combine ------------------------------------------------------------- */
/* out[t,:] = fp16( sum_j gate_weights[t*k+j] * y[slot_pos[t*k+j], :] ) over kept
 * slots, fp32 accumulation in slot order, one store per element, no atomics.
 * Replaces the gather of lightning_router/kernels/expert_routing.py:238-298 on
 * the layer path (lightning_router/models/moe_layer.py:126).  d % 8 == 0.  */
int lr_combine(const void* y, const float* gate_weights, const int32_t* slot_pos,
               int T, int k, int d, void* out, lr_stream_t stream);

size_t lr_gather_workspace_bytes(int num_rows, int num_tokens);

/* Row-wise weighted gather back to token order for arbitrary (rows -> token)
 * maps: out[src[r]] += w[r] * y[r] over rows with w[r] != 0, fp32 accumulation
 * in ascending row order per token, one fp16 store per element.
 * Replaces expert_routing_gather, lightning_router/kernels/expert_routing.py:274-298. */
int lr_expert_routing_gather(const void* y, const float* routing_w, const int32_t* source_idx,
                             int R, int d, int T, void* out, void* workspace,
                             size_t workspace_bytes, int32_t* err, lr_stream_t stream);

/* ---- W4A16 GEMM -------------------------------------------------------- */
/* Packed INT4 format (lightning_router/quantization/pack_weights.py:23-130):
 * qweight (K, N/8) int32, nibble i of word j = column 8j+i; scales (K/g, N)
 * fp16; zeros (K/g, N/8) int32 packed like qweight; w = fp16(scale*(q-zero)). */

#define LR_FFN_MODE_PLAIN 0   /* C = A . W                                   */
#define LR_FFN_MODE_SILU 1    /* C = silu(A . W)                             */
#define LR_FFN_MODE_SWIGLU 2  /* C = silu(A . Wgate) * (A . Wup)             */

/* One expert's matrices: index 0 gate, 1 up, 2 down (gate unused when not gated). */
typedef struct lr_expert_weights {
  const int32_t* qweight[3];
  const void* scales[3];
  const int32_t* zeros[3];
} lr_expert_weights;

/* Host-side encoding of the per-expert weight table (TMA descriptors and
 * pointers).  Writes `lr_weight_table_bytes(E)` bytes into `host_table`
 * (128-byte aligned host memory); the caller copies it to a 128-byte aligned
 * device buffer once per weight set.  No CUDA calls besides descriptor encoding.
 * Accepts every shape of the packed format: K % group_size == 0, N % 8 == 0
 * (reference lightning_router/quantization/pack_weights.py:44-45).          */
size_t lr_weight_table_bytes(int num_experts);
int lr_encode_weight_table(const lr_expert_weights* experts, int E, int d_model, int d_ff,
                           int group_size, int gated, void* host_table, size_t table_bytes);

/* Workspace of lr_grouped_w4a16_gemm: 0 when the call needs none.  Superseded
 * by lr_grouped_w4a16_workspace_bytes (ABI 3); kept for ABI 2 callers.        */
size_t lr_grouped_gemm_workspace_bytes(int num_experts);

/* Workspace (bytes, 128-byte aligned) that lets lr_grouped_w4a16_gemm take its
 * 8-bit path for this shape: expert segments of at most 32 rows with
 * K % 128 == 0, group_size % 128 == 0 and N % 32 == 0 (decode).  There the
 * token rows are written as two signed 8-bit terms per 128-k block
 * (x ~ sigma * (a1 + a2/256), sigma = max|x|/127 of the block; error at most
 * sigma/512, sigma/256 where the second term saturates) and the INT4 codes enter the tensor core as unsigned bytes; the
 * group scale and zero are applied in fp32 per 128-k block.  Returns 0 for
 * shapes that do not take that path.  Without the workspace the same call
 * runs the fp16-operand kernel.                                               */
size_t lr_grouped_w4a16_workspace_bytes(int num_experts, int R, int K, int N, int group_size,
                                        int max_rows_per_expert);

/* Grouped W4A16 GEMM.  For each expert e, rows
 * [seg_start[e], seg_start[e] + seg_len[e]) of A (R x K fp16, row-major)
 * are multiplied with matrix `mat` (or gate/up for SWIGLU) of expert e and
 * written to the same rows of C (R x N_out fp16).  seg_* live on the device.
 * `max_rows_per_expert` bounds seg_len (selects the token tile); seg_len
 * beyond it is clamped and flagged.  `group_size` is the one the table was
 * encoded with.  The kernel follows the shape: tcgen05 on 8-bit operands for
 * segments of at most 32 rows when the workspace holds
 * lr_grouped_w4a16_workspace_bytes(...) bytes; tcgen05 on fp16 operands (tokens
 * the UMMA M operand) when K % 64 == 0, group_size % 64 == 0 and N % 32 == 0; mma.sync
 * with the weights as the M operand when K % 8 == 0, N % 32 == 0 and
 * group_size is a power of two >= 16; otherwise CUDA cores.  A needs 2-byte,
 * C 16-byte alignment.
 * Replaces ExpertGroup.forward / ExpertFFN._qmatmul + quantized_matmul
 * (lightning_router/models/experts.py:58-121, kernels/quantized_matmul.py:122-173). */
int lr_grouped_w4a16_gemm(const void* device_table, int E, int mode, int mat,
                          const void* A, int R, int K, int N, int group_size,
                          const int32_t* seg_start, const int32_t* seg_len,
                          int max_rows_per_expert, void* C, void* workspace,
                          size_t workspace_bytes, int32_t* err, lr_stream_t stream);

/* Single W4A16 GEMM C[M,N] = A[M,K] . dequant(qweight) (fp16 out).
 * Replaces quantized_matmul, lightning_router/kernels/quantized_matmul.py:122-173.
 * `device_table` holds one expert entry encoded with gated = 0 whose matrix 2
 * is (qweight, scales, zeros) with K = d_ff, N = d_model.                     */
int lr_quantized_matmul(const void* device_table, const void* A, int M, int K, int N,
                        int group_size, void* C, void* workspace, size_t workspace_bytes,
                        int32_t* err, lr_stream_t stream);

/* ---- expert-parallel exchange over NVLink peer memory --------------------
 * Replaces the all-GPU expert execution + host all-reduce of the reference's
 * serving worker (lightning_router/serving/worker.py:156-186) for one process
 * per GPU.  Rank r owns experts [r*E/G, (r+1)*E/G).  The caller keeps five
 * buffers per rank mapped by every other rank (lr_ipc_*): the rank's tokens,
 * the row -> token map of its uncapped expert segments (source_idx of
 * lr_permute_tokens without rows), the expert-output rows it computes, a
 * statistics table (G rows of 1 + 2E doubles) and 2G int32 flags (zeroed
 * once); peer_* are device arrays of the G ranks' addresses of such a buffer.
 * A step is: lr_ep_publish -> lr_ep_plan_wait -> lr_ep_gather -> expert GEMMs
 * -> lr_ep_signal -> lr_ep_combine, with `epoch` = 1, 2, ... the step number
 * (the same on every rank).  The flags order every cross-GPU read after the
 * matching writes and every overwrite after the matching reads; each wait is
 * bounded (LR_DEVERR_PEER_TIMEOUT).  lr_ep_plan / lr_ep_plan_tokens plan from
 * counts the caller gathered itself (an NCCL exchange).                      */

/* Number of int32 entries of an exchange plan. */
int lr_ep_plan_size(int world, int num_experts);

/* plan from counts[G][E] (slots of each expert on each rank, uncapped): the
 * global slot-order capacity (kept(r, e) = clamp(C - sum_{r'<r} counts[r'][e],
 * 0, counts[r][e]), the single-GPU rule), the owner's segments [local expert]
 * [source rank] and where this rank's kept rows land at every owner.
 * Limits: G * E <= 4096.                                                     */
int lr_ep_plan(const int32_t* counts, int world, int num_experts, int rank, int capacity,
               int32_t* plan, int32_t* err, lr_stream_t stream);

/* lr_ep_plan with the capacity computed on the device from the G ranks' token
 * counts (shard_tokens, int32 [G]): C = max(int((top_k * sum T_r / E) *
 * capacity_factor), 1) in double precision, the single-GPU formula (reference
 * kernels/expert_routing.py:196-197), so shards may differ in size from rank
 * to rank and from step to step with no host round trip.  max_capacity is
 * the largest C the caller's buffers hold; a larger C is clipped to it and
 * flagged in err.  The plan's last entry holds the C it applied.             */
int lr_ep_plan_tokens(const int32_t* counts, const int32_t* shard_tokens, int world,
                      int num_experts, int top_k, double capacity_factor, int rank,
                      int max_capacity, int32_t* plan, int32_t* err, lr_stream_t stream);

/* Writes this rank's statistics row (num_tokens, per-expert counts from the
 * CSR offsets, per-expert probability sums; zeros when num_tokens == 0) into
 * slot `rank` of every rank's table, then raises its stats flag (flags[rank])
 * on every rank with the value epoch.                                        */
int lr_ep_publish(const uint64_t* peer_stats, const uint64_t* peer_flags, const int32_t* offsets,
                  const double* prob_sums, int num_tokens, int world, int num_experts, int rank,
                  int epoch, lr_stream_t stream);

/* Waits (bounded) until every rank's stats flag reached epoch, then plans as
 * lr_ep_plan_tokens from the table (capacity from the summed token counts,
 * clipped to max_capacity) and writes the whole job's auxiliary loss
 * (reference lightning_router/models/gating.py:91-99).  A flag that does not
 * arrive sets LR_DEVERR_PEER_TIMEOUT and yields a plan that keeps no rows.   */
int lr_ep_plan_wait(const double* stats, const int32_t* flags, int world, int num_experts,
                    int rank, int top_k, double capacity_factor, int max_capacity,
                    float load_balance_weight, int epoch, int32_t* plan, float* aux_loss,
                    int32_t* err, lr_stream_t stream);

/* After this rank's expert GEMMs: raises its outputs flag (flags[G + rank]) on
 * every rank with the value epoch.                                           */
int lr_ep_signal(const uint64_t* peer_flags, int world, int rank, int epoch, lr_stream_t stream);

/* Expert owner: rows of its segments <- the kept token rows, read from the
 * source ranks' token buffers (tokens < max_tokens, map entries < max_slots).
 * out has rows_max = E/G * capacity rows of d fp16; rows past the segments are
 * not written.                                                               */
int lr_ep_gather(const uint64_t* peer_tokens, const uint64_t* peer_source_idx,
                 const int32_t* plan, int world, int num_experts, int rank, int max_tokens,
                 int max_slots, int d, int rows_max, void* out, int32_t* err,
                 lr_stream_t stream);

/* Token owner: out[t,:] = fp16( sum_j gate_weights[t*k+j] * y_owner[row, :] )
 * over the kept slots in slot order (fp32), y read from the owners' expert
 * output buffers; slot_pos holds each slot's uncapped local row.  With
 * ready_flags (this rank's flags + G) it first waits (bounded) until every
 * rank's outputs flag reached epoch; without, the caller orders the reads.   */
int lr_ep_combine(const uint64_t* peer_outputs, const int32_t* plan, const int32_t* expert_ids,
                  const float* gate_weights, const int32_t* slot_pos, int T, int k, int world,
                  int num_experts, int d, int rows_max, void* out, const int32_t* ready_flags,
                  int epoch, int32_t* err, lr_stream_t stream);

/* CUDA IPC of a device buffer: export writes a 64-byte handle of the buffer's
 * allocation and the buffer's offset in it; import (in another process) maps
 * the allocation and returns the buffer address (+ the mapping base, which
 * lr_ipc_close unmaps).                                                      */
int lr_ipc_export(const void* ptr, void* handle, uint64_t* offset);
int lr_ipc_import(const void* handle, uint64_t offset, void** ptr, void** base);
int lr_ipc_close(void* base);

#ifdef __cplusplus
}
#endif

#endif /* LIGHTNING_ROUTER_H */
