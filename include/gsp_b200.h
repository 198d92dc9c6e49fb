/*
 * gsp_b200.h -- C ABI of the B200 (sm_100a) grammar-conditioned LM-head library.
 *
 * Drop-in device layer for the GSP decode-time LM head: inputs are decode
 * hidden states [B, H], the LM-head weight W [V, H] (row-major) and a packed
 * int32 grammar bitmask [B, >= ceil(V/32)] (LSB-first: token v is legal iff bit
 * v%32 of word v/32 is set). Outputs are vocab-shaped logits with -inf on
 * illegal tokens, or compact legal logits with their token ids, plus a fused
 * greedy top-1 per request (ties to the lowest vocabulary index).
 *
 * Conventions for every entry point:
 *   - All tensor pointers are device pointers (cudaMalloc / torch CUDA memory).
 *   - Strides are in ELEMENTS of the pointed-to type and refer to the row
 *     (outer) dimension; the inner dimension is contiguous.
 *   - `stream` is a cudaStream_t handle passed as void* (NULL = legacy default
 *     stream). Every call is asynchronous on that stream: no host sync.
 *   - `dtype`: GSP_DTYPE_F16, GSP_DTYPE_BF16 or GSP_DTYPE_F32; hidden, weight
 *     and the logits share it. Accumulation is fp32, rounded once to `dtype`.
 *     The reference's wrappers take any floating dtype (the output dtype is
 *     the hidden dtype, gsp/triton_runtime.py:111; gsp/runtime.py:46-51 is a
 *     plain F.linear). fp32 runs on the row-sparse kernels only: the block and
 *     dense entry points given GSP_DTYPE_F32 run the row-sparse kernel (same
 *     outputs), and the sampler, adaptive and grouped entry points return
 *     GSP_ERR_UNSUPPORTED for it.
 *   - `vocab_offset` shifts the token ids reported in top_index / compact ids,
 *     for a weight that is one contiguous row shard of a larger vocabulary.
 *   - Optional outputs may be NULL.
 *   - `workspace` must be at least gsp_workspace_bytes(batch, vocab) bytes,
 *     zero-filled once before first use; every call leaves it zero-filled
 *     again. Calls that run concurrently must not share one workspace.
 *     Exception: bytes 4..7 hold an int32 error word that kernels set (and
 *     never clear) when a bounded wait ran out instead of hanging: 1 a
 *     multi-CTA kernel's wait for its CTAs' counts, flags or pipeline stages,
 *     2 a corrupt unit code found (stale state from an earlier failed call),
 *     3 the cross-rank top-1 exchange, 4 the single-GPU top-1 slot merge
 *     (then no token is reported: top_index -1). After a non-zero word the
 *     caller re-zeroes the whole workspace before its next call.
 *   - Returns GSP_OK or a negative GSP_ERR_* code; no exception or abort
 *     crosses the ABI. gsp_last_error() describes the last failure on the
 *     calling host thread.
 *
 * Top-1 keys (top_key outputs) are signed-orderable int64 values: a larger key
 * is a larger rounded logit, or the same logit at a lower token id. A plain
 * integer MAX reduction over keys from vocabulary shards therefore yields the
 * global greedy token; gsp_top1_from_keys decodes a key.
 */
#ifndef GSP_B200_H_
#define GSP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GSP_ABI_VERSION 1

#define GSP_OK 0
#define GSP_ERR_INVALID_ARGUMENT (-1)
#define GSP_ERR_UNSUPPORTED (-2)
#define GSP_ERR_WORKSPACE (-3)
#define GSP_ERR_CUDA (-4)

#define GSP_DTYPE_F16 0
#define GSP_DTYPE_BF16 1
#define GSP_DTYPE_F32 2

/* Rows of one vocabulary tile for the block and dense GEMM paths and for the
 * active-tile statistics. */
#define GSP_TILE_ROWS 128

int32_t gsp_abi_version(void);
const char* gsp_status_string(int32_t status);
const char* gsp_last_error(void);

/* Bytes of workspace any entry point below needs for (batch, vocab). */
size_t gsp_workspace_bytes(int32_t batch, int32_t vocab);

/*
 * Row-sparse (direct-bitmask) projection: only legal rows of W are read.
 * Replaces gsp/triton_runtime.py:61-125 (bitmask_sparse_logits) and its kernel
 * gsp/triton_runtime.py:15-58 (_bitmask_sparse_lm_head_kernel).
 * bitmask == NULL means every token is legal. bitmask_row_stride may be 0 to
 * share one mask row across the batch. logits [batch, vocab] may be NULL when
 * only the top-1 outputs are wanted.
 */
int32_t gsp_row_sparse_logits(const void* hidden, int64_t hidden_row_stride,
                              const void* weight, int64_t weight_row_stride,
                              const int32_t* bitmask, int64_t bitmask_row_stride,
                              int32_t batch, int32_t vocab, int32_t hidden_dim,
                              int32_t dtype, int64_t vocab_offset, void* logits,
                              int64_t logits_row_stride, float* top_value,
                              int64_t* top_index, int64_t* top_key, void* workspace,
                              size_t workspace_bytes, void* stream);

/*
 * Compact legal logits: request b's legal tokens, in increasing token order,
 * occupy positions [request_offsets[b], request_offsets[b+1]) of
 * compact_logits / compact_ids. request_offsets ([batch+1]) is always written;
 * entries past `capacity` are not. Replaces gsp/runtime.py:9-51
 * (constrained_projection / ProjectionResult, mode "sparse-gather" and
 * "dense-selected") for bitmask-described legal sets.
 */
int32_t gsp_row_sparse_compact(const void* hidden, int64_t hidden_row_stride,
                               const void* weight, int64_t weight_row_stride,
                               const int32_t* bitmask, int64_t bitmask_row_stride,
                               int32_t batch, int32_t vocab, int32_t hidden_dim,
                               int32_t dtype, int64_t vocab_offset, void* compact_logits,
                               int64_t* compact_ids, int64_t capacity,
                               int64_t* request_offsets, float* top_value,
                               int64_t* top_index, int64_t* top_key, void* workspace,
                               size_t workspace_bytes, void* stream);

/*
 * Token-id list -> packed bitmask [ceil(vocab/32)] (duplicates collapse, the
 * ids come out sorted). stats[0] = number of distinct in-range ids,
 * stats[1] = number of ids outside [0, vocab). Both outputs are cleared by the
 * call. Replaces the id handling of gsp/runtime.py:35-43.
 */
int32_t gsp_ids_to_bitmask(const int64_t* ids, int64_t count, int32_t vocab,
                           int32_t* bitmask, int64_t* stats, void* stream);

/*
 * Per-request density statistics computed on the device: legal token counts,
 * full (-1) word counts (the signal of gsp/triton_runtime.py:310-321) and the
 * number of GSP_TILE_ROWS-row tiles holding any legal token of any request.
 * Outputs may be NULL; active_tiles is a single int32.
 */
int32_t gsp_mask_stats(const int32_t* bitmask, int64_t bitmask_row_stride,
                       int32_t batch, int32_t vocab, int32_t* legal_counts,
                       int32_t* full_words, int32_t* active_tiles, void* stream);

/*
 * Grammar-aware block GEMM: tensor-core (tcgen05) projection of only the
 * GSP_TILE_ROWS-row vocabulary tiles that hold a legal token of any request in
 * the batch, with the -inf mask and top-1 fused into the epilogue.
 * Replaces gsp/triton_runtime.py:212-258 (bitmask_block_gemm_logits) and its
 * kernel gsp/triton_runtime.py:147-209.
 */
int32_t gsp_block_gemm_logits(const void* hidden, int64_t hidden_row_stride,
                              const void* weight, int64_t weight_row_stride,
                              const int32_t* bitmask, int64_t bitmask_row_stride,
                              int32_t batch, int32_t vocab, int32_t hidden_dim,
                              int32_t dtype, int64_t vocab_offset, void* logits,
                              int64_t logits_row_stride, float* top_value,
                              int64_t* top_index, int64_t* top_key, void* workspace,
                              size_t workspace_bytes, void* stream);

/*
 * Dense tensor-core projection of every vocabulary tile with the grammar mask
 * and top-1 fused into the epilogue (bitmask may be NULL: no mask).
 * Replaces gsp/triton_runtime.py:285-308 (dense_masked_logits: F.linear
 * followed by xgrammar's apply_token_bitmask_inplace).
 */
int32_t gsp_dense_masked_logits(const void* hidden, int64_t hidden_row_stride,
                                const void* weight, int64_t weight_row_stride,
                                const int32_t* bitmask, int64_t bitmask_row_stride,
                                int32_t batch, int32_t vocab, int32_t hidden_dim,
                                int32_t dtype, int64_t vocab_offset, void* logits,
                                int64_t logits_row_stride, float* top_value,
                                int64_t* top_index, int64_t* top_key, void* workspace,
                                size_t workspace_bytes, void* stream);

/*
 * Allocation-free variant of gsp_row_sparse_logits, for callers that cannot
 * allocate device memory at all (a plugin inside a serving engine that owns
 * every byte of device memory through its own pool, or an FFI binding that is
 * handed only the input and output buffers). It takes the same arguments minus
 * the workspace: the scratch (top-1 keys, and the slice counts, flags and
 * unit list of the multi-request kernel; 4.3 MB) lives in a fixed array inside
 * the library, kept on every GPU that loads it until exit, so batch must be
 * <= GSP_STATIC_MAX_BATCH and vocab <= GSP_STATIC_MAX_VOCAB (larger sizes fail
 * with GSP_ERR_INVALID_ARGUMENT and a message in gsp_last_error()).
 * The first call on each device (and CUDA context) looks up the array's
 * device address (cudaGetSymbolAddress) with that device current; make that
 * first call before any stream capture. Each call first launches a small
 * clearing kernel on `stream` that zeroes the scratch it needs (no memory is
 * allocated), then the projection. All calls share the one array: calls that
 * may run at the same time on the GPU (other streams, other host threads)
 * race on it and must be serialised by the caller. A kernel that gave up a
 * bounded wait leaves an error word in the array; it is kept across calls
 * until gsp_row_sparse_static_error reads it.
 * No counterpart in the reference.
 */
#define GSP_STATIC_MAX_BATCH 1024
#define GSP_STATIC_MAX_VOCAB 1048576
int32_t gsp_row_sparse_logits_static(const void* hidden, int64_t hidden_row_stride,
                                     const void* weight, int64_t weight_row_stride,
                                     const int32_t* bitmask, int64_t bitmask_row_stride,
                                     int32_t batch, int32_t vocab, int32_t hidden_dim,
                                     int32_t dtype, int64_t vocab_offset, void* logits,
                                     int64_t logits_row_stride, float* top_value,
                                     int64_t* top_index, int64_t* top_key, void* stream);

/*
 * Reads and clears the error word of gsp_row_sparse_logits_static's scratch on
 * the current device: *error = 0 when every call since the last read ran to
 * completion, else the code of the first wait that gave up (4: a row copy did
 * not land). Synchronises `stream` (call it after the calls to be checked have
 * been issued on that stream); when the word was set, re-zeroes the whole
 * scratch array on `stream`. Allocates nothing. No counterpart in the
 * reference.
 */
int32_t gsp_row_sparse_static_error(int32_t* error, void* stream);

/*
 * Decode top-1 keys (e.g. after an integer MAX all-reduce across vocabulary
 * shards) into the rounded logit value and the token id. No reference
 * counterpart: the reference is single-GPU and takes logits.argmax(-1)
 * (benchmarks/qwen35_adaptive_paired.py:94).
 */
int32_t gsp_top1_from_keys(const int64_t* keys, int32_t batch, float* top_value,
                           int64_t* top_index, void* stream);

/*
 * Fused grammar-conditioned sampler (row-sparse path): the projection of
 * gsp_row_sparse_logits reduced on chip to sampling statistics; logits are
 * optional (NULL: no vocabulary-shaped output is written at all). Per request
 * b, with x_v the legal logits rounded to `dtype`:
 *   sample_index[b]     = argmax over legal v of x_v / T + g_v, ties to the
 *                         lowest id (0 if no token is legal), where
 *                         g_v = -log(-log(u_v)) and u_v =
 *                         ((Philox4x32-10(counter {v, offset lo, offset hi, 0},
 *                         key {seeds[b] lo, seeds[b] hi}).word0 >> 8) + 0.5) / 2^24,
 *                         all in fp32: an exact draw from softmax(x / T) over the
 *                         legal tokens (Gumbel-max), reproducible from
 *                         (seeds[b], offset, v);
 *   sample_logsumexp[b] = log sum over legal v of exp(x_v / T) (optional;
 *                         -inf if no token is legal), so the sampled token's
 *                         log-probability is x / T - sample_logsumexp; its
 *                         partial sums merge in arrival order, so repeated calls
 *                         agree to fp32 rounding (the sampled ids bit for bit);
 *   sample_key[b]       = the winning perturbed score and id as a signed-
 *                         orderable top-1 key (optional): the noise is keyed by
 *                         the GLOBAL token id (vocab_offset + v), so for row
 *                         shards of one vocabulary the integer MAX of the
 *                         shards' keys is the whole vocabulary's draw
 *                         (gsp_top1_from_keys decodes it), and
 *                         gsp_merge_logsumexp combines their log-sum-exps;
 *   top_value / top_index / top_key: the greedy top-1, as in
 *                         gsp_row_sparse_logits.
 * temperature > 0 and finite; seeds is a device array [batch]; offset is the
 * caller's step counter (use a new one per step). The workspace must hold
 * gsp_workspace_bytes(batch, vocab) bytes. No counterpart in the reference
 * (its paper, paper/draft.md section 6.4, names this as the next step).
 */
int32_t gsp_row_sparse_sample(const void* hidden, int64_t hidden_row_stride,
                              const void* weight, int64_t weight_row_stride,
                              const int32_t* bitmask, int64_t bitmask_row_stride,
                              int32_t batch, int32_t vocab, int32_t hidden_dim,
                              int32_t dtype, int64_t vocab_offset, void* logits,
                              int64_t logits_row_stride, float temperature,
                              const uint64_t* seeds, uint64_t offset,
                              int64_t* sample_index, float* sample_logsumexp,
                              int64_t* sample_key, float* top_value, int64_t* top_index,
                              int64_t* top_key, void* workspace, size_t workspace_bytes,
                              void* stream);

/*
 * The same fused sampler on any route (GSP_ROUTE_*): row-sparse runs
 * gsp_row_sparse_sample; block-sparse and dense-mask run the tensor-core
 * projection with the sampler in its epilogue (Gumbel noise only for the legal
 * entries of the tiles it computes, per-request winning keys and (max, sum of
 * exp) partials merged by the last CTA). Same arguments and contract as
 * gsp_row_sparse_sample, so the same (seeds, offset) give the same tokens on
 * every route up to the last-bit differences of the routes' fp32 summation
 * order (a draw whose two best perturbed scores lie that close may differ).
 * No counterpart in the reference (paper/draft.md section 6.4).
 */
int32_t gsp_sample(int32_t route, const void* hidden, int64_t hidden_row_stride,
                   const void* weight, int64_t weight_row_stride,
                   const int32_t* bitmask, int64_t bitmask_row_stride,
                   int32_t batch, int32_t vocab, int32_t hidden_dim,
                   int32_t dtype, int64_t vocab_offset, void* logits,
                   int64_t logits_row_stride, float temperature,
                   const uint64_t* seeds, uint64_t offset, int64_t* sample_index,
                   float* sample_logsumexp, int64_t* sample_key,
                   float* top_value, int64_t* top_index, int64_t* top_key,
                   void* workspace, size_t workspace_bytes, void* stream);

/* out[b] = log sum over r < parts of exp(lse[r * batch + b]) (-inf when every
 * part is -inf): merges per-shard log-sum-exps of a vocabulary-parallel
 * sampler step (device arrays). No counterpart in the reference. */
int32_t gsp_merge_logsumexp(const float* lse, int32_t parts, int32_t batch, float* out, void* stream);

/*
 * Vocabulary-parallel head: top-1 merged across ranks inside the kernel.
 *
 * One process per GPU on one node, up to GSP_MAX_PEERS ranks; rank r holds a
 * contiguous row shard of W (vocab_offset = its first global row) and the
 * matching words of every request's mask. Set-up, once per rank:
 *   1. gsp_peer_exchange_alloc(gsp_peer_exchange_bytes(R, max_batch), &buf,
 *      handle): device memory (zeroed) and its IPC handle;
 *   2. send the GSP_IPC_HANDLE_BYTES handle to every other rank over any host
 *      channel (torch.distributed, a socket, ...);
 *   3. gsp_peer_exchange_open(handle_q, &peer_q) for every other rank q
 *      (peer access over NVLink is enabled by the mapping).
 * Then every call of gsp_vocab_parallel_logits with peer_buffers[q] = rank q's
 * buffer as mapped here (peer_buffers[rank] = buf) ends, inside the projection
 * kernel, with an exchange over peer memory: the last CTA stores the rank's
 * per-request top-1 keys into every rank's buffer, raises its flag there,
 * waits for the other ranks' flags for at most wait_us microseconds (<= 0:
 * 250,000) and writes the GLOBAL top-1 (global token ids) to top_value /
 * top_index / top_key. Logits, when given, are this rank's shard only. No
 * collective library call and no extra launch is involved, so the call can be
 * captured in a CUDA graph. Every rank must make the same sequence of calls
 * with the same route and batch. A wait that runs out reports no token for
 * the call: every top_index is -1 (top_value NaN, top_key INT64_MIN), never a
 * merge of the keys that happened to arrive, and the workspace error word is
 * set to 3. The group must then re-synchronise before its next call: every
 * rank, once its calls have completed, calls gsp_peer_exchange_reset on its
 * own buffer and re-zeroes its workspace, with a host barrier between the
 * ranks before and after. route is one of
 * GSP_ROUTE_*; world_size 1 runs the plain projection. total_vocab is the
 * whole head's vocabulary, the same on every rank (below 2^24 - 1 each key
 * travels as one self-tagged store; larger heads add a fence and a flag).
 * Replaces NCCL all-gather of (max, index) pairs; the reference is
 * single-GPU and has no counterpart.
 */
#define GSP_MAX_PEERS 8
#define GSP_IPC_HANDLE_BYTES 64
#define GSP_ROUTE_ROW_SPARSE 0
#define GSP_ROUTE_BLOCK_SPARSE 1
#define GSP_ROUTE_DENSE_MASK 2

size_t gsp_peer_exchange_bytes(int32_t world_size, int32_t max_batch);
int32_t gsp_peer_exchange_alloc(size_t bytes, void** buffer, void* ipc_handle);
int32_t gsp_peer_exchange_open(const void* ipc_handle, void** peer_buffer);
int32_t gsp_peer_exchange_close(void* peer_buffer);
int32_t gsp_peer_exchange_free(void* buffer);
/* Zeroes this rank's own exchange buffer (epoch, flags, keys) on the legacy
 * stream and waits for it: the re-synchronisation after a wait ran out. */
int32_t gsp_peer_exchange_reset(void* buffer, int32_t world_size, int32_t max_batch);
int32_t gsp_vocab_parallel_logits(int32_t route, const void* hidden, int64_t hidden_row_stride,
                                  const void* weight, int64_t weight_row_stride,
                                  const int32_t* bitmask, int64_t bitmask_row_stride,
                                  int32_t batch, int32_t vocab, int32_t hidden_dim,
                                  int32_t dtype, int64_t vocab_offset, void* logits,
                                  int64_t logits_row_stride, float* top_value,
                                  int64_t* top_index, int64_t* top_key, void* workspace,
                                  size_t workspace_bytes, void* const* peer_buffers,
                                  int32_t rank, int32_t world_size, int32_t max_batch,
                                  int64_t total_vocab, int64_t wait_us, void* stream);

/* ---- Device-side route choice (adaptive_grammar_logits without a host
 * round trip) ----------------------------------------------------------------
 * Route cost model (the reference's dispatcher, gsp/triton_runtime.py:324-353,
 * chooses from a host-side full-word fraction; this model costs each route as
 * a fixed latency plus its bytes at that kernel's measured B200 rate):
 *   row   = row_sparse_fixed_us + (legal_total * H * e + B * V * e) / (hbm_gbs * 1e3)
 *   block = max(block_floor_us, block_fixed_us + min(128 * active_tiles, V) * H * e / (block_gbs * 1e3))
 *   dense = dense_fixed_us + V * H * e / (dense_gbs * 1e3)
 * (us; e = element bytes). The cheapest wins; on equal cost block-sparse,
 * then dense-mask, then row-sparse. Batch 1 is always row-sparse.
 * gsp_default_route_cost fills the B200 calibration; gsp_choose_route applies
 * the model on the host (the device selector runs the same code).
 */
typedef struct gsp_route_cost {
  double hbm_gbs;
  double row_sparse_fixed_us;
  double block_floor_us;
  double block_fixed_us;
  double block_gbs;
  double dense_fixed_us;
  double dense_gbs;
  double group_split_fixed_us; /* lane-group split overhead (gsp_group_plan) */
} gsp_route_cost;

void gsp_default_route_cost(gsp_route_cost* cost);
int32_t gsp_choose_route(int32_t batch, int32_t vocab, int32_t hidden_dim, int32_t elem_bytes,
                         int64_t legal_total, int64_t active_tiles, const gsp_route_cost* cost);

/* Masked logits and fused top-1 with the route chosen ON THE DEVICE from the
 * mask: one selector kernel counts the batch's legal tokens and active
 * 128-row tiles, applies the cost model (cost NULL = defaults) and picks
 * GSP_ROUTE_ROW_SPARSE / _BLOCK_SPARSE / _DENSE_MASK.
 *  - Stream being captured into a CUDA graph: the call adds the selector
 *    kernel and a SWITCH conditional node whose three bodies hold the three
 *    routes' launches; the selector sets the switch with
 *    cudaGraphSetConditional, so every replay runs only the chosen route and
 *    the host never waits. Body launches are recorded from this call's
 *    pointers. Restrictions of conditional nodes apply to the enclosing graph
 *    (it cannot be cloned or nested as a child graph). Run each route's first
 *    call (or this call once) outside capture so that kernel attributes are
 *    set.
 *  - Otherwise (eager): the selector runs, the route is read back (one 4-byte
 *    device-to-host copy and a stream synchronisation) and the chosen route
 *    is launched.
 * route_out (device int32, optional) receives the route of each call;
 * route_host (host, optional) receives it in eager mode and -1 under
 * capture. bitmask is required; batch >= 1; the workspace must hold
 * gsp_workspace_bytes(batch, vocab) bytes. Extension beyond the reference.
 */
int32_t gsp_adaptive_logits(const void* hidden, int64_t hidden_row_stride, const void* weight,
                            int64_t weight_row_stride, const int32_t* bitmask,
                            int64_t bitmask_row_stride, int32_t batch, int32_t vocab,
                            int32_t hidden_dim, int32_t dtype, void* logits,
                            int64_t logits_row_stride, float* top_value, int64_t* top_index,
                            const gsp_route_cost* cost, int32_t* route_out, int32_t* route_host,
                            void* workspace, size_t workspace_bytes, void* stream);

/* ---- Lane grouping by density class -----------------------------------------
 * The reference's roadmap (paper/draft.md:264-270) proposes grouping requests
 * so that permissive lanes do not activate tiles for constrained ones.
 * gsp_group_plan profiles every request on the device (legal tokens, active
 * 128-row tiles), orders the requests by the fill of their active tiles
 * (legal / (128 x tiles); scattered lanes first), finds for every tile the
 * first and last position in that order of a request that touches it, and
 * costs every split "first k positions | the rest" with each group on its
 * cheapest route (the cost model above, plus group_split_fixed_us and, with
 * logits, the un-permute of the logits rows at hbm_gbs) against the best
 * single route. plan: device int32 [gsp_group_plan_words(batch)], layout
 *   [0] k (0: no split), [1] route of positions [0, k), [2] route of [k, B),
 *   [3] best single route, [4] its modelled ns, [5] the split's modelled ns
 *   (-1: none), [6..16) reserved, then order[B] (position -> request) and
 *   inverse[B] (request -> position), then per-request and per-position
 *   statistics. batch <= GSP_GROUP_MAX_BATCH. No workspace; asynchronous.
 * gsp_gather_rows copies dst row i = src row rows[i] (device int32 rows) for
 * permuting hidden states, masks, logits and top-1 rows.
 */
/* SM-driven asynchronous copy of `bytes` bytes between any two addresses the
 * device can reach: device memory, or pinned host memory (cudaHostAlloc /
 * cudaMallocHost, which unified addressing maps into the device's address
 * space). For a decode step's small inputs (a mask row and a hidden state,
 * tens of KB) it avoids the fixed latency of a copy-engine transfer; the
 * projection entries can likewise write top_value / top_index straight into
 * pinned host memory. 16-byte units when both addresses are 16-byte aligned.
 * No counterpart in the reference (its decode loop copies with torch). */
int32_t gsp_copy_bytes(void* dst, const void* src, size_t bytes, void* stream);

/* One decode step from host inputs in one call: gsp_copy_bytes of
 * input_bytes from host_inputs (pinned host memory: the step's packed mask
 * and hidden state) to device_inputs, then gsp_row_sparse_logits with the
 * remaining arguments, whose hidden and bitmask point into device_inputs and
 * whose top_value / top_index may point into pinned host memory. Every
 * argument is checked before anything is queued. The decode loop's mask copy
 * (gsp/triton_runtime.py:133-144) and head call
 * (benchmarks/qwen35_adaptive_paired.py:63-94) in one crossing of the ABI. */
int32_t gsp_row_sparse_step(const void* host_inputs, size_t input_bytes, void* device_inputs,
                            const void* hidden, int64_t hidden_row_stride,
                            const void* weight, int64_t weight_row_stride,
                            const int32_t* bitmask, int64_t bitmask_row_stride,
                            int32_t batch, int32_t vocab, int32_t hidden_dim,
                            int32_t dtype, int64_t vocab_offset, void* logits,
                            int64_t logits_row_stride, float* top_value,
                            int64_t* top_index, int64_t* top_key, void* workspace,
                            size_t workspace_bytes, void* stream);

/* The same step recorded once as a CUDA graph (copy node + projection; the
 * projection's launch overlaps the copy through a programmatic edge), for a
 * decode loop that repeats it on the same device buffers: create takes
 * gsp_row_sparse_step's arguments without the stream (host_inputs names the
 * pinned row recorded; nothing runs at create), launch replays the graph on
 * `stream` with one driver call, first pointing the copy at host_inputs when
 * given (a pinned row of the recorded size and 16-byte alignment). Launches
 * of one handle must not overlap (they share the workspace and buffers).
 * Extends the decode loop's copy + head call
 * (benchmarks/qwen35_adaptive_paired.py:63-94); no Triton counterpart. */
int32_t gsp_step_graph_create(void** handle, const void* host_inputs, size_t input_bytes,
                              void* device_inputs, const void* hidden, int64_t hidden_row_stride,
                              const void* weight, int64_t weight_row_stride,
                              const int32_t* bitmask, int64_t bitmask_row_stride,
                              int32_t batch, int32_t vocab, int32_t hidden_dim,
                              int32_t dtype, int64_t vocab_offset, void* logits,
                              int64_t logits_row_stride, float* top_value,
                              int64_t* top_index, int64_t* top_key, void* workspace,
                              size_t workspace_bytes);
int32_t gsp_step_graph_launch(void* handle, const void* host_inputs, void* stream);
int32_t gsp_step_graph_destroy(void* handle);

#define GSP_GROUP_MAX_BATCH 256
size_t gsp_group_plan_words(int32_t batch);
int32_t gsp_group_plan(const int32_t* bitmask, int64_t bitmask_row_stride, int32_t batch, int32_t vocab,
                       int32_t hidden_dim, int32_t elem_bytes, int32_t with_logits, const gsp_route_cost* cost,
                       int32_t* plan, void* stream);
int32_t gsp_gather_rows(const void* src, int64_t src_row_stride_bytes, const int32_t* rows, int32_t n,
                        int64_t row_bytes, void* dst, int64_t dst_row_stride_bytes, void* stream);

/* The whole grouped projection in one call: gsp_group_plan, a 32-byte
 * read-back of the plan header (the call waits for it: not capturable), then
 * either the best single route on the caller's buffers, or a split: hidden
 * and mask rows gathered into group order, each group's route, logits and
 * top-1 rows permuted back. Results equal the chosen routes' outputs.
 * scratch: gsp_grouped_scratch_bytes(batch, vocab, hidden_dim, logits != NULL)
 * bytes of device memory, 256-byte aligned (contents not preserved);
 * workspace as for the other entries; plan_header (host int32 [8], optional)
 * receives the plan header. batch <= GSP_GROUP_MAX_BATCH.
 */
size_t gsp_grouped_scratch_bytes(int32_t batch, int32_t vocab, int32_t hidden_dim, int32_t with_logits);
int32_t gsp_grouped_logits(const void* hidden, int64_t hidden_row_stride, const void* weight,
                           int64_t weight_row_stride, const int32_t* bitmask, int64_t bitmask_row_stride,
                           int32_t batch, int32_t vocab, int32_t hidden_dim, int32_t dtype, void* logits,
                           int64_t logits_row_stride, float* top_value, int64_t* top_index,
                           const gsp_route_cost* cost, int32_t* plan_header, void* scratch, size_t scratch_bytes,
                           void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GSP_B200_H_ */
