/*
 * swiftmoe.h -- C ABI of the B200 (sm_100a) MoE-layer forward library (libswiftmoe.so).
 *
 * Every entry point takes plain device pointers and sizes, enqueues its work on the
 * given CUDA stream and returns an int status (SMOE_OK or a negative SMOE_ERR_*).
 * Nothing allocates device memory except smoe_ep_* (the expert-parallel exchange
 * buffers) ; scratch space is passed in by the caller and sized by the matching
 * *_workspace_size() query.  No call synchronises the host with the device unless its
 * comment says so.
 *
 * Each entry point names the SwiftMoE reference code it replaces (file:line in the
 * reference project).  Tensor layouts are row-major; "[A, B]" means B is contiguous.
 */
#ifndef SWIFTMOE_H_
#define SWIFTMOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* smoe_stream_t; /* == cudaStream_t */

#if defined(__GNUC__)
#define SMOE_API __attribute__((visibility("default")))
#else
#define SMOE_API
#endif

/* ----------------------------------------------------------------------------- status */
#define SMOE_OK 0
#define SMOE_ERR_INVALID (-1)     /* bad argument: null pointer, bad size, k > E, ... */
#define SMOE_ERR_CUDA (-2)        /* a CUDA runtime / driver call failed               */
#define SMOE_ERR_TIMEOUT (-3)     /* a device-side bounded wait gave up                */
#define SMOE_ERR_UNSUPPORTED (-4) /* valid but unsupported shape / dtype combination   */
#define SMOE_ERR_WORKSPACE (-5)   /* workspace too small                               */
#define SMOE_ERR_TOO_LARGE (-6)   /* size beyond a fixed, documented maximum           */

/* ------------------------------------------------------------------------------ dtypes */
#define SMOE_F32 0
#define SMOE_F16 1
#define SMOE_BF16 2
/* smoe_layer_args.dtype only: an fp32 layer whose routed expert weights (w1, w3, w2 or
 * w_lin) are given split by smoe_tf32_split_weights, [E, N, 3K] instead of [E, N, K]
 * (the shared expert's stay plain).  The layer then skips splitting them on every call;
 * it needs d_model % 8 == 0 and d_ff % 8 == 0 (else SMOE_ERR_UNSUPPORTED).             */
#define SMOE_F32_SPLITW 16

/* ----------------------------------------------------------------------- expert kinds */
#define SMOE_EXPERT_LINEAR 0 /* y = x W_e^T           (one bias-free d x d linear)      */
#define SMOE_EXPERT_SWIGLU 1 /* y = w2(silu(w1 x) * w3 x)                               */

SMOE_API const char* smoe_version(void);
SMOE_API const char* smoe_status_string(int status);
/* Number of SMs of the current device (used to size persistent grids). */
SMOE_API int smoe_device_sm_count(void);
/* Read and clear the device-side error word set by bounded waits inside kernels.
 * Synchronises the stream.  *flag receives 0 when no wait timed out. */
SMOE_API int smoe_read_device_error(int* flag, smoe_stream_t stream);
/* Self-test of the give-up path every bounded device wait of this library takes: one
 * thread waits on a shared-memory mbarrier that nothing arrives at, with a time limit
 * of limit_ns (0 < limit_ns <= 1 s) instead of the kernels' 2 s.  When the limit runs
 * out the wait returns, the kernel stores 1 in *gave_up (device int) and records the
 * timeout in the error word (smoe_read_device_error then reports 1), and the context
 * stays usable.  No counterpart in the reference (its kernels have no bounded waits). */
SMOE_API int smoe_selftest_wait_timeout(uint64_t limit_ns, int* gave_up, smoe_stream_t stream);

/* ------------------------------------------------------------------------------ router
 * logits[t,e] = sum_i x[t,i] * wg[e,i] (+ logit_bias[e]) accumulated in fp32; top-k over
 * e with ties to the LOWER expert index and NaN ranked highest; w = softmax of the k
 * selected logits (fp32).  Outputs idx [T,k] int32 (values descending), w [T,k] fp32,
 * and, when logits_out != NULL, the fp32 gate logits [T,E] before logit_bias is added.
 * k <= min(E, 32), E <= 1024.
 * Replaces: models/ultimate_moe.py:34-101 (fused_router_dispatch_kernel), :288-295
 * (torch routing fallback) and models/baseline_moe.py:56-67 (_route_tokens).        */
SMOE_API int smoe_router_fwd(const void* x, const void* wg, int dtype, const float* logit_bias,
                     int T, int d, int E, int k, int32_t* idx, float* w, float* logits_out,
                     void* workspace, size_t workspace_bytes, smoe_stream_t stream);
SMOE_API size_t smoe_router_workspace_size(int T, int d, int E, int dtype);

/* Top-k + softmax from given fp32 logits [T,E] (bit-exact routing entry point).
 * Replaces: torch.topk + torch.softmax at models/baseline_moe.py:62-65 and
 * models/ultimate_moe.py:290-291.                                                    */
SMOE_API int smoe_topk_from_logits(const float* logits, int T, int E, int k, int32_t* idx, float* w,
                          smoe_stream_t stream);

/* ---------------------------------------------------------------------- dispatch plan
 * Groups the T*k (token, slot) pairs by expert in index order (token-major, then slot)
 * without any host round trip.  Outputs:
 *   expert_counts [E]   : rows routed to each expert (before the capacity cut)
 *   expert_offsets[E+1] : start row of each expert's segment (exclusive scan of the kept
 *                         counts, each rounded up to row_align); [E] = total rows
 *   slot_row  [T*k]     : destination row of every slot, -1 when dropped by capacity
 *                         or skipped (an idx entry of -1 marks a slot to skip)
 *   row_token [rows_cap]: source token of every row, -1 for alignment padding
 * capacity <= 0 means unlimited; otherwise at most `capacity` rows per expert are kept,
 * the lowest (token, slot) indices winning.  rows_cap must be >= smoe_plan_rows_cap().
 * Replaces: bincount / argsort / repeat_interleave bookkeeping at
 * models/ultimate_moe.py:118-125 and :224-231, models/baseline_moe.py:80-98.        */
SMOE_API size_t smoe_plan_workspace_size(int T, int k, int E);
SMOE_API int64_t smoe_plan_rows_cap(int T, int k, int E, int capacity, int row_align);
SMOE_API int smoe_dispatch_plan(const int32_t* idx, int T, int k, int E, int capacity, int row_align,
                       int32_t* expert_counts, int32_t* expert_offsets, int32_t* slot_row,
                       int32_t* row_token, int64_t rows_cap, void* workspace,
                       size_t workspace_bytes, smoe_stream_t stream);

/* Allocation-free variant of smoe_dispatch_plan.  No counterpart in the reference.
 * For callers that cannot allocate device memory at all -- e.g. a host that owns every
 * byte of device memory in its own arena or caching allocator, where a cudaMalloc from
 * a library would bypass that budget and synchronise the device mid-step.  It takes no
 * workspace and allocates nothing: its scratch (per-block histograms and bases) is a
 * fixed 512 KiB static device array inside the library, held by every GPU that loads
 * the library until the process exits.  Same inputs, outputs and results as
 * smoe_dispatch_plan.  Limits: T*k <= SMOE_NOALLOC_PLAN_MAX_SLOTS and
 * E <= SMOE_NOALLOC_PLAN_MAX_EXPERTS, else SMOE_ERR_TOO_LARGE and nothing is launched.
 * The first call on a device resolves the scratch array's device address with that
 * device current (cudaGetSymbolAddress); make that first call before any stream
 * capture.  All calls share the one scratch array, so calls that overlap on the GPU
 * (other streams, other host threads) race and must be serialised by the caller.     */
#define SMOE_NOALLOC_PLAN_MAX_SLOTS (1 << 19)
#define SMOE_NOALLOC_PLAN_MAX_EXPERTS 256
SMOE_API int smoe_dispatch_plan_noalloc(const int32_t* idx, int T, int k, int E, int capacity,
                                        int row_align, int32_t* expert_counts,
                                        int32_t* expert_offsets, int32_t* slot_row,
                                        int32_t* row_token, int64_t rows_cap,
                                        smoe_stream_t stream);

/* rows[r,:] = x[row_token[r],:] for expert_offsets[0] <= r < expert_offsets[E] (zero
 * rows for token -1).  A plan's offsets start at 0; passing a slice of them (E experts
 * starting at some expert) fills only that range of rows, at their plan positions.
 * Replaces: x.repeat_interleave(2)[sort_idx] and recv_x[expert_order]
 * (models/ultimate_moe.py:123,225).                                                  */
SMOE_API int smoe_permute_rows(const void* x, int dtype, int T, int d, const int32_t* row_token,
                      const int32_t* expert_offsets, int E, int64_t rows_cap, void* rows,
                      smoe_stream_t stream);

/* out[t,:] = sum_{j<k} w[t,j] * y[slot_row[t,j],:] (slots in order 0..k-1, fp32
 * accumulation, dropped slots skipped) + (shared ? shared[t,:] : 0).
 * Replaces: combined_x[sort_idx_rev].view(M,2,d).sum(dim=1) and the gate weighting
 * (models/ultimate_moe.py:154-155,245; models/baseline_moe.py:162,188-189).         */
SMOE_API int smoe_combine(const void* y, int dtype, const int32_t* slot_row, const float* w, int T,
                 int k, int d, const void* shared, void* out, smoe_stream_t stream);

/* --------------------------------------------------------------------- expert GEMMs
 * Grouped GEMM over G groups of rows.  Group g owns rows [offsets[g], offsets[g+1]) of
 * A [rows_cap, K] -- or [offsets[g], ends[g]) when `ends` is not NULL -- and multiplies
 * them by B_g^T where B is [G, N, K] (nn.Linear layout, K contiguous).  offsets / ends
 * live in device memory and are read by the kernel; ranges are clamped to [0, rows_cap]
 * and only the rows of a group's range are written.
 *   epilogue SMOE_EPI_STORE  : C[r, n] = acc                       (C is [rows_cap, N])
 *   epilogue SMOE_EPI_SWIGLU : C[r, n] = silu(A B1_g^T) * (A B3_g^T) (B3 = B2 arg, C [rows_cap, N])
 * bf16 / fp16 run on tcgen05 tensor cores (TMEM accumulators, TMA-fed shared memory,
 * requires K % 8 == 0 and N % 8 == 0), except batches of at most 2 rows, which stream the
 * weights of the groups that have rows on the SIMT pipes (one warp per output column);
 * fp32 keeps fp32 accuracy: on the tf32 tensor cores with split operands (3xTF32: each
 * value = its tf32 rounding + the remainder, three tf32 products summed in fp32) when
 * K % 4 == 0 and N % 8 == 0, else on FFMA (SIMT).
 * C may be fp32 for the bf16/fp16 STORE epilogue when out_dtype == SMOE_F32.
 * Replaces: the per-expert loop of torch.mm at models/ultimate_moe.py:237-250 and
 * nn.Linear experts at models/baseline_moe.py:151-162.                               */
#define SMOE_EPI_STORE 0
#define SMOE_EPI_SWIGLU 1
#define SMOE_EPI_GATEUP 3 /* C[r, n] = A B1_g^T, C[r, N + n] = A B3_g^T (C is [rows_cap, 2N]) */
SMOE_API int smoe_grouped_gemm(const void* A, const void* B, const void* B3, void* C, int dtype,
                      int out_dtype, int epilogue, const int32_t* offsets, const int32_t* ends,
                      int G, int64_t rows_cap, int N, int K, smoe_stream_t stream);
/* The same grouped GEMM with output row r written at the address row_ptrs[r] (device
 * array of rows_cap addresses, 16-byte aligned; 0 skips the row) instead of C + r*N.
 * The addresses may lie in another GPU's memory (IPC-opened peer buffers): the
 * epilogue then stores the expert outputs straight into the source ranks' return
 * buffers over NVLink, tile by tile while the GEMM runs, and fences them at system
 * scope before the kernel exits.  Replaces the return all_to_all_single that follows
 * the expert loop in models/ultimate_moe.py:152 (MoEAsyncCommHandler.combine_async). */
SMOE_API int smoe_grouped_gemm_rows(const void* A, const void* B, const void* B3, const uint64_t* row_ptrs,
                                    int dtype, int out_dtype, int epilogue, const int32_t* offsets,
                                    const int32_t* ends, int G, int64_t rows_cap, int N, int K,
                                    smoe_stream_t stream);

/* out[r, :] = [lo(w[r, :]) | hi(w[r, :]) | hi(w[r, :])] for `rows` fp32 rows of K (K % 4
 * == 0, 16-byte aligned): hi = the tf32 rounding (to nearest, ties away from zero), lo =
 * the exact remainder -- the weight layout the fp32 grouped GEMMs run on the tf32 tensor
 * cores (three tf32 products per fp32 product).  A layer that keeps this copy of its
 * weights passes dtype SMOE_F32_SPLITW to smoe_layer_fwd.  No counterpart in the
 * reference (its fp32 experts are torch.mm / nn.Linear, models/ultimate_moe.py:237-250). */
SMOE_API int smoe_tf32_split_weights(const float* w, float* out, int64_t rows, int K, smoe_stream_t stream);

/* dst[g, c, r] = src[g, r, c] for G matrices of [R, C] (weight relayout, e.g. the
 * reference's x@W expert_weights [E, d_in, d_out] -> nn.Linear layout [E, d_out, d_in]). */
SMOE_API int smoe_transpose_batched(const void* src, void* dst, int dtype, int G, int R, int C,
                           smoe_stream_t stream);

/* dst[r,:] = src[index[r],:] for r < n_rows, zero rows where index[r] is -1.
 * Replaces: combined_x[sort_idx_rev] / expert_out[argsort(expert_order)] gathers
 * (models/ultimate_moe.py:154,252).                                                  */
SMOE_API int smoe_gather_rows(const void* src, int dtype, int d, const int32_t* index, int64_t n_rows,
                              void* dst, smoe_stream_t stream);

/* ------------------------------------------------------------ expert parallelism
 * Receive side of the dispatch all-to-all: rows arrive grouped by source rank, then by
 * local expert (recv_counts is [ws, E_l], row-major).  Builds the expert-major layout
 * the grouped GEMM consumes, applying the capacity cut in (source rank, token, slot)
 * order:
 *   expert_counts [E_l]   rows received per local expert (before the cut)
 *   expert_offsets[E_l+1] start row of each local expert; [E_l] = total kept rows
 *   row_src [>= n_recv]   received row that feeds each expert row
 *   recv_dst[n_recv]      expert row of each received row, -1 when dropped
 * pos_base [ws, E_l] (device, may be NULL): position, in expert le's global
 * (source rank, token, slot) order, of the first row of segment (s, le) -- used when a
 * batch is exchanged in token chunks, so the capacity cut stays the whole batch's.
 * NULL means the segments of this call are the whole batch.
 * Replaces: the receive-side bookkeeping of models/ultimate_moe.py:128-141 and the
 * regrouping by local expert at :224-231.                                             */
SMOE_API size_t smoe_ep_regroup_workspace_size(int ws, int E_l);
SMOE_API int smoe_ep_regroup_plan(const int32_t* recv_counts, int ws, int E_l, int capacity,
                                  const int32_t* pos_base, int64_t n_recv, int32_t* expert_counts,
                                  int32_t* expert_offsets, int32_t* row_src, int32_t* recv_dst,
                                  void* workspace, size_t workspace_bytes, smoe_stream_t stream);
/* Return addresses of the expert-parallel combine.  The receive buffer holds n_src
 * source segments: received row r with seg_table[s] <= r < seg_table[s+1] came from
 * source s and goes back to row r - seg_table[s] of that source's return region, whose
 * address is seg_table[n_src + 1 + s] (an int64 holding a device address, usually in
 * the source GPU's memory; 16-byte aligned, as is row_bytes).  seg_table is a device
 * array of 2 * n_src + 1 int64.  Writes row_ptrs[i] for the expert rows i < rows_cap
 * (0 past expert_offsets[E_l]) for smoe_grouped_gemm_rows, and writes zero rows at the
 * destinations of received rows the capacity dropped (recv_dst < 0), so the source's
 * combine adds nothing for those slots.  row_src NULL: expert row i is received row i
 * (the senders placed their rows in expert-major order; rows_cap <= n_recv); recv_dst
 * NULL: nothing was dropped.  Replaces, with the GEMM above, the return path of
 * models/ultimate_moe.py:152,224-231.                                                 */
/* ------------------------------------------------- expert-parallel exchange on device
 * The per-forward bookkeeping of the exchange without a host round trip (the reference
 * reads the counts on the host: models/ultimate_moe.py:128-137, and sends three
 * payloads: :139-141).  counts_all [ws][E] (device): rows each rank routes to each
 * global expert (every rank's plan counts, all-gathered); experts live in contiguous
 * blocks of E_l = E/ws per rank.  The capacity cut keeps, per expert, the first
 * `capacity` rows in (source rank, token, slot) order (0 = no cut).
 * smoe_ep_layout (one block; ws*E <= 8192) writes this rank's
 *   send_addr[E]      byte address, in the owner's receive buffer (recv_base[owner],
 *                     this GPU's mapping of it), of this rank's first row for expert e;
 *                     0 for its own experts
 *   keep[E]           rows of this rank's segment for expert e kept by the cut
 *   recv_offsets[E_l+1] expert offsets of its own receive buffer, which holds the other
 *                     ranks' rows expert-major (local expert, source rank, token, slot)
 *   seg_table[2*E_l*ws+1] the received segments in (local expert, source) order: first
 *                     receive row of each, the row total, then the byte address of each
 *                     segment's first row in the source's return buffer (ret_base[s]),
 *                     which has the source's send layout -- the format of
 *                     smoe_ep_return_rows (row_src = recv_dst = NULL)
 * If any rank's receive rows would exceed recv_rows_max, every rank (all compute the
 * same counts) sends and computes nothing and the device error word is set (4).
 * smoe_ep_send_rows: every row i of the send layout (expert_offsets [E+1] of this rank's
 * dispatch plan over global experts; row_token from the same plan) outside this rank's
 * own experts [own_first, own_first+own_count) is read from x[row_token[i]] and stored
 * at send_addr[e] + p*row_bytes (p = position in expert e's segment) when p < keep[e]:
 * the permute and the dispatch all-to-all in one kernel, writing straight into the
 * peers' memory (CUDA IPC mappings, NVLink).  row_bytes % 16 == 0; rows_cap bounds the
 * rows of the layout (expert_offsets[E] <= rows_cap).  Order the receivers after it
 * with a collective on the same stream.
 * smoe_ep_drop_slots: slot_row[s] = -1 for the slots the cut dropped (row position in
 * its expert's segment >= keep[e]), so that smoe_combine skips them.
 * flags SMOE_EP_LAYOUT_ROTATED (token dedup; E == ws "experts" = ranks, no capacity):
 * every source s lays out its rows in its rotated rank order (destination (s + g) % ws
 * for group g, its own rank first) and counts_all holds those groups' counts; send_addr
 * and keep come out in this rank's rotated group order, the return table in rank order.
 * smoe_ep_clear_tail: idx [rows_cap, k] slots of rows r >= *n_rows set to -1 (received
 * rows past this step's count).  smoe_store_rows: src row r (r < n_rows) to the address
 * row_ptrs[r] (0 = skip; 16-byte aligned, possibly another GPU's memory).
 * smoe_copy_rows_count: dst rows [0, *n_rows) = src rows, n_rows in device memory.
 * Replace, for token dedup: the host-side sizing and per-peer copies of the
 * (token, rank) rows and their slot metadata (models/ultimate_moe.py:128-141).       */
SMOE_API int smoe_ep_clear_tail(int32_t* idx, const int32_t* n_rows, int64_t rows_cap, int k, smoe_stream_t stream);
SMOE_API int smoe_store_rows(const void* src, int64_t row_bytes, const uint64_t* row_ptrs, int64_t n_rows,
                             smoe_stream_t stream);
SMOE_API int smoe_copy_rows_count(void* dst, const void* src, int64_t row_bytes, const int32_t* n_rows,
                                  int64_t rows_cap, smoe_stream_t stream);
#define SMOE_EP_LAYOUT_ROTATED 1 /* flags of smoe_ep_layout: token dedup's rotated layouts */
SMOE_API int smoe_ep_layout(const int32_t* counts_all, int ws, int E, int rank, int capacity,
                            const uint64_t* recv_base, const uint64_t* ret_base, int64_t row_bytes,
                            int64_t recv_rows_max, uint64_t* send_addr, int32_t* keep, int32_t* recv_offsets,
                            int64_t* seg_table, int flags, smoe_stream_t stream);
SMOE_API int smoe_ep_send_rows(const void* x, int64_t row_bytes, const int32_t* row_token,
                               const int32_t* expert_offsets, int E, int own_first, int own_count,
                               const uint64_t* send_addr, const int32_t* keep, int64_t rows_cap,
                               smoe_stream_t stream);
SMOE_API int smoe_ep_drop_slots(const int32_t* idx, int64_t n_slots, const int32_t* expert_offsets, int E,
                                const int32_t* keep, int32_t* slot_row, smoe_stream_t stream);

/* Expert-parallel token dedup (top-k with several experts per rank).  A token whose
 * slots go to several experts of one rank is sent to that rank once:
 *   smoe_ep_dedup_ranks: ridx[T, k] = destination rank of each slot in this rank's
 *     rotated order ((e / E_l - rank + ws) % ws; this rank first) for the first slot of
 *     the token bound for that rank, -1 for its later slots to the same rank.  A
 *     smoe_dispatch_plan over ridx with ws experts (-1 = skipped slot) lays out the sent
 *     rows: one per (token, rank), grouped by rotated rank, token order.
 *   smoe_ep_dedup_meta: for each sent row p (= slot_row of a first slot): meta_e[p, j] =
 *     the local expert of slot j if it goes to the row's rank, else -1, and
 *     meta_w[p, j] its gate weight (0 else), in slot order; own_e [T, k] holds the same
 *     for this rank's own rows (rows [0, own_count[0]), own_count = the plan's
 *     counts[0], device) and -1 in rows [own_count[0], T).
 * The receiver plans over meta_e (local experts, -1 skipped), runs the experts and
 * returns ONE weighted partial sum per received row (smoe_combine over meta_w); the
 * sender adds the partial sums of its token's ranks.  Replaces the per-(token, slot)
 * replication of models/ultimate_moe.py:123 (`repeat_interleave`) and its payload
 * all_to_all_single (:139-141).                                                       */
SMOE_API int smoe_ep_dedup_ranks(const int32_t* idx, int64_t T, int k, int E_l, int ws, int rank, int32_t* ridx,
                                 smoe_stream_t stream);
SMOE_API int smoe_ep_dedup_meta(const int32_t* idx, const float* w, const int32_t* ridx, const int32_t* slot_row,
                                const int32_t* own_count, int64_t T, int k, int E_l, int ws, int32_t* meta_e,
                                float* meta_w, int32_t* own_e, smoe_stream_t stream);
SMOE_API int smoe_ep_return_rows(const int32_t* row_src, const int32_t* expert_offsets, int E_l,
                                 const int32_t* recv_dst, int64_t n_recv, const int64_t* seg_table, int n_src,
                                 int64_t row_bytes, uint64_t* row_ptrs, int64_t rows_cap, smoe_stream_t stream);

/* Expert-parallel exchange buffers.  These are the only allocations of the library:
 * each rank allocates its receive / return buffers once (grown when a batch needs
 * more), exports a CUDA IPC handle, and every rank opens every peer's buffer, so rows
 * move with plain device-to-device copies over NVLink (copy engines, no SMs), in the
 * place of the reference's payload all_to_all_single calls
 * (models/ultimate_moe.py:139-141,152).  ipc_handle points to 64 bytes.             */
#define SMOE_IPC_HANDLE_BYTES 64
SMOE_API int smoe_ep_buffer_create(size_t bytes, void** dev_ptr, void* ipc_handle);
SMOE_API int smoe_ep_buffer_destroy(void* dev_ptr);
SMOE_API int smoe_ep_peer_open(const void* ipc_handle, void** peer_ptr);
SMOE_API int smoe_ep_peer_close(void* peer_ptr);
/* n device-to-device copies dst[i] <- src[i] (bytes[i]) on the stream, in order; the
 * pointers may be IPC-opened peer buffers.  One cudaMemcpyAsync per segment.         */
SMOE_API int smoe_copy_segments(void* const* dst, const void* const* src, const size_t* bytes, int n,
                                smoe_stream_t stream);

/* -------------------------------------------------------------------- whole layer
 * One-GPU MoE forward: router -> plan -> permute -> expert FFN -> combine (+ shared
 * expert).  Replaces UltimateMoE.forward (models/ultimate_moe.py:254-342) and
 * StandardMoE.forward (models/baseline_moe.py:191-213) at world size 1.             */
typedef struct smoe_layer_args {
  int32_t tokens, d_model, num_experts, top_k;
  int32_t expert_type; /* SMOE_EXPERT_*                                              */
  int32_t d_ff;        /* SwiGLU hidden size (ignored for linear)                    */
  int32_t dtype;       /* SMOE_F32 / SMOE_F16 / SMOE_BF16                             */
  int32_t capacity;    /* rows per expert, <= 0 = unlimited                           */
  int32_t num_shared;  /* 0 or 1 always-on SwiGLU shared expert                       */
  int32_t d_ff_shared;
  const void* x;          /* [T, d]                                                   */
  const void* gate_w;     /* [E, d]                                                   */
  const float* logit_bias; /* [E] or NULL                                              */
  const void* w1;         /* SwiGLU [E, F, d]                                          */
  const void* w3;         /* SwiGLU [E, F, d]                                          */
  const void* w2;         /* SwiGLU [E, d, F]                                          */
  const void* w_lin;      /* linear [E, d_out, d_in]                                   */
  const void* sw1;        /* shared [F_s, d]                                           */
  const void* sw3;        /* shared [F_s, d]                                           */
  const void* sw2;        /* shared [d, F_s]                                           */
  void* out;              /* [T, d]                                                    */
  int32_t* topk_idx;      /* optional [T, k] output (NULL: kept in workspace)          */
  float* topk_w;          /* optional [T, k] output                                    */
  int32_t* expert_counts; /* optional [E] output                                       */
  void* workspace;
  size_t workspace_bytes;
  /* Optional cudaEvent_t handles (from smoe_event_create) recorded on the stream at the
   * stage boundaries: [0] start, [1] router done, [2] dispatch plan + permute done,
   * [3] expert GEMM 1 done, [4] expert GEMM 2 + shared expert done, [5] combine done.
   * NULL entries are skipped.                                                          */
  void* stage_events[6];
} smoe_layer_args;

/* Timing events usable in smoe_layer_args.stage_events (cudaEventDefault flags).
 * smoe_event_elapsed waits for `end` and returns the milliseconds between the two.   */
SMOE_API int smoe_event_create(void** event);
SMOE_API int smoe_event_destroy(void* event);
SMOE_API int smoe_event_record(void* event, smoe_stream_t stream);
SMOE_API int smoe_event_elapsed(void* start, void* end, float* ms);

SMOE_API size_t smoe_layer_workspace_size(const smoe_layer_args* a);
SMOE_API int smoe_layer_fwd(const smoe_layer_args* a, smoe_stream_t stream);

/* --------------------------------------------------------------- layer backward
 * Gradients of smoe_layer_fwd's output (16-bit layers, SwiGLU or linear experts, one
 * GPU) with respect to x, the gate and every expert weight.  The reference is forward-only; these are the
 * gradients of its forward (models/baseline_moe.py:56-189 with SwiGLU experts,
 * post-weighting, k slots summed, capacity drops contributing zero, softmax over the k
 * selected logits).  The routing, the gate/up pre-activations and the per-slot outputs
 * are recomputed from x (nothing is kept from the forward).  Weights as in the forward,
 * plus two K-major copies the dgrad GEMMs read (make them once per weight update with
 * smoe_transpose_batched):  w2t [E, F, d] = w2 transposed;  w13t [E, d, 2F] = the
 * transpose of [w1; w3] stacked along F.  Gradients (fp32) go to
 *   dx [T, d] (dtype), dgate [E, d], dw13 [E, 2F, d] (each expert's dW1 rows, then its
 *   dW3 rows), dw2 [E, d, F], and for the shared expert dsw13 [2F_s, d], dsw2 [d, F_s].
 * No counterpart in the reference (forward-only).                                     */
typedef struct smoe_layer_bwd_args {
  int32_t tokens, d_model, num_experts, top_k;
  int32_t d_ff, dtype, capacity;
  int32_t num_shared, d_ff_shared;
  const void* x;           /* [T, d]                          */
  const void* dout;        /* [T, d] gradient of the output   */
  const void* gate_w;      /* [E, d]                          */
  const float* logit_bias; /* [E] or NULL                     */
  const void* w1;          /* [E, F, d]                       */
  const void* w3;          /* [E, F, d]                       */
  const void* w2t;         /* [E, F, d]                       */
  const void* w13t;        /* [E, d, 2F]                      */
  const void* sw1;         /* shared [F_s, d]                 */
  const void* sw3;         /* shared [F_s, d]                 */
  const void* sw2t;        /* shared [F_s, d] (sw2 transposed) */
  const void* sw13t;       /* shared [d, 2F_s]                */
  void* dx;
  float* dgate;
  float* dw13;
  float* dw2;
  float* dsw13;
  float* dsw2;
  void* workspace;
  size_t workspace_bytes;
  /* Linear experts (expert_type SMOE_EXPERT_LINEAR, y = x Wl^T with Wl [d_out, d_in]):
   * w_lin_t [E, d_in, d_out] = Wl transposed (UltimateMoE's x @ W parameter as it is);
   * dw_lin [E, d_out, d_in] fp32, or [E, d_in, d_out] when dw_lin_transposed != 0.
   * The SwiGLU fields are then unused (d_ff ignored).                                */
  int32_t expert_type;
  int32_t dw_lin_transposed;
  const void* w_lin_t;
  float* dw_lin;
} smoe_layer_bwd_args;
SMOE_API size_t smoe_layer_bwd_workspace_size(const smoe_layer_bwd_args* a);
SMOE_API int smoe_layer_bwd(const smoe_layer_bwd_args* a, smoe_stream_t stream);

/* Weight-gradient GEMM grouped along K: for g < G,
 *   C[g][m][n] = sum over k in [k_offsets[g], k_offsets[g+1]) of A[m][k] * B[n][k],
 * A [M, K] and B [N, K] 16-bit, K-major with row strides lda, ldb >= K elements (multiples
 * of 8); C [G, M, N] fp32.  Group starts must be multiples of 64 (a dispatch plan with
 * row_align 64 gives that; a start that is not is reported in the device error word, 5);
 * a group without rows gets zeros.  Replaces the weight gradients autograd would take
 * through the reference's per-expert Linear / torch.mm (models/baseline_moe.py:155-162,
 * models/ultimate_moe.py:245-249).                                                     */
SMOE_API int smoe_wgrad_gemm(const void* A, int64_t lda, const void* B, int64_t ldb, int dtype,
                             const int32_t* k_offsets, int G, int M, int N, int64_t K, float* C,
                             smoe_stream_t stream);
/* The same with the operands given as rows of K: A [K, lda] (its first M columns) and
 * B [K, ldb] (first N columns), row-major -- e.g. the routed rows themselves, grouped by
 * expert -- read as MN-major tensor-core tiles, with no transposed copy.  M, N, lda, ldb
 * multiples of 8; rows from K on read as zeros.                                        */
SMOE_API int smoe_wgrad_gemm_rows(const void* A, int64_t lda, const void* B, int64_t ldb, int dtype,
                                  const int32_t* k_offsets, int G, int M, int N, int64_t K, float* C,
                                  smoe_stream_t stream);

/* ---- The layer backward in pieces, for expert parallelism: the routed rows' part runs on
 * the rank that owns their experts, the tokens' part on the tokens' own rank.  The
 * reference is forward-only; these differentiate its forward (models/baseline_moe.py:
 * 56-189, models/ultimate_moe.py:222-252, 288-295), as smoe_layer_bwd does in one call.
 *
 * SwiGLU rows, in place: ab[r] = [a | b] (pre-activations, [rows, 2F]) -> [da | db];
 * g[r] (the gradient reaching h before the gate weight, dout_r W2, [rows, F]) -> w_r * h;
 * dw_row[r] = <g_r, h_r> fp32 (the gate weight's gradient; may be NULL).  Rows r <
 * *n_rows (n_rows NULL: all rows_cap); row_w NULL means w = 1.  16-bit, F % 8 == 0.     */
SMOE_API int smoe_swiglu_bwd(void* ab, void* g, const float* row_w, const int32_t* n_rows, int64_t rows_cap,
                             int F, int dtype, float* dw_row, smoe_stream_t stream);
/* Linear-expert rows, in place: dw_row[r] = <g_r, x_r> (g = dout_r Wl), g[r] -> w_r g_r
 * (the rows' input gradient), dr[r] -> w_r dr_r (their output gradient).  d % 8 == 0.   */
SMOE_API int smoe_linear_bwd(void* g, const void* xr, void* dr, const float* row_w, const int32_t* n_rows,
                             int64_t rows_cap, int d, int dtype, float* dw_row, smoe_stream_t stream);
/* dx[t] = sum_j dxr[slot_row[t,j]] (kept slots) + dxs[t] (shared expert, may be NULL) +
 * sum_j dsel_tj Wg[idx[t,j]], one rounding; dsel_tj = w_tj (dw_tj - sum_j' w_tj' dw_tj'),
 * dw_tj = dw_row[slot_row[t,j]] (0 for dropped slots), the softmax-over-top-k backward of
 * the router.  dsel_row (may be NULL) gets dsel_tj at slot_row_full[t,j] (a plan over
 * every slot) for smoe_router_dwg.                                                      */
SMOE_API int smoe_moe_bwd_dx(const void* dxr, const int32_t* slot_row, const int32_t* idx, const float* w,
                             const float* dw_row, const void* gate_w, const void* dxs, int T, int k, int d,
                             int dtype, void* dx, const int32_t* slot_row_full, float* dsel_row,
                             smoe_stream_t stream);
/* Gate gradient dgate[e] = sum over the rows r of expert e in a plan over every slot
 * (offsets_full [E+1], row_token_full) of dsel_row[r] * x[row_token_full[r]], fp32 [E, d],
 * summed in a fixed order.                                                              */
SMOE_API size_t smoe_router_dwg_workspace_size(int d, int E);
SMOE_API int smoe_router_dwg(const void* x, const int32_t* row_token_full, const int32_t* offsets_full,
                             const float* dsel_row, int d, int E, int dtype, float* dgate, void* workspace,
                             size_t workspace_bytes, smoe_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* SWIFTMOE_H_ */
