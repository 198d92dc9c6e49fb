// Internal launch interfaces shared by the kernel translation units and the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gsp {

// Ranks of one vocabulary-parallel group whose projection kernels merge their
// top-1 keys over peer memory (one process per GPU, one node).
constexpr int kMaxPeers = 8;

// Exchange buffer of one rank (gsp_peer_exchange_alloc): [0] epoch (calls
// completed), [128 + 128 q] flag written by rank q (one line per writer),
// [kPeerKeysOffset] keys[2][world][max_batch] (double-buffered by epoch
// parity), written by the ranks over NVLink.
constexpr size_t kPeerKeysOffset = 128 + 128 * kMaxPeers;

constexpr size_t peer_exchange_bytes_for(size_t world, size_t max_batch) {
  return (kPeerKeysOffset + 2 * world * max_batch * 8 + 255) / 256 * 256;
}

struct PeerExchange {
  unsigned char* buf[kMaxPeers];  // rank q's exchange buffer as mapped in this process
  int rank;
  int world;       // < 2: no exchange
  int max_batch;   // key slots per rank
  int batch_base;  // slot of this launch's request 0 (batch chunks of the block path)
  int tagged;      // global token ids < 2^24 - 1: one self-tagged store per key, no flag
  int64_t wait_ns; // how long the last CTA waits for the other ranks' keys before it gives up
};

constexpr int64_t kDefaultPeerWaitUs = 250000;

// Parameters of the row-sparse kernel (one launch covers every request).
struct RowSparseParams {
  const void* hidden;
  int64_t hidden_stride;
  const void* weight;
  int64_t weight_stride;
  const uint32_t* mask;  // nullptr: every token legal
  int64_t mask_stride;   // words; 0 broadcasts row 0
  int batch;
  int vocab;
  int hidden_dim;
  int nw;  // ceil(vocab / 32)
  int64_t vocab_offset;
  // full logits [batch, vocab] (optional)
  void* logits;
  int64_t logits_stride;
  // compact output (optional)
  void* compact;
  int64_t* compact_ids;
  int64_t capacity;
  int64_t* offsets;  // [batch + 1]
  // top-1 (optional; all three may be null)
  float* top_value;
  int64_t* top_index;
  int64_t* top_key;
  // workspace: per-request keys + arrival ticket (zero on entry and exit)
  unsigned long long* keys;
  unsigned int* ticket;
  int* error;  // set non-zero when a bounded wait gave up (never cleared by kernels)
  // cooperative kernel (all zero on entry and exit): per-CTA slice popcounts,
  // the number of CTAs that have published theirs, per-CTA "units listed"
  // flags (one per kFlagStride words, so pollers of different flags never
  // share a cache line), and the list of (request, row) unit codes in rank
  // order, room for list_cap units
  unsigned int* slice_counts;
  unsigned int* published;
  unsigned int* slice_ready;
  uint32_t* unit_list;
  int64_t list_cap;
  PeerExchange peers;  // cross-rank top-1 merge (world < 2: none)
  // fused sampler (sample_index != nullptr; contract in gsp_sampler.cuh)
  int64_t* sample_index;             // [batch] sampled global token ids
  float* sample_lse;                 // [batch] log-sum-exp of legal logits * inv_temp (optional)
  int64_t* sample_key;               // [batch] signed-orderable winning key (optional)
  const uint64_t* seeds;             // [batch] per-request generator keys
  uint64_t offset;                   // step counter
  float inv_temp;                    // 1 / temperature
  unsigned long long* sample_keys;   // workspace [batch]
  unsigned long long* stat_partials; // workspace [batch][kMaxSlices]
};

// Parameters of the tensor-core block / dense projection.
struct BlockGemmParams {
  const void* hidden;
  int64_t hidden_stride;
  const void* weight;
  int64_t weight_stride;
  const uint32_t* mask;  // nullptr: every token legal
  int64_t mask_stride;
  int batch;
  int vocab;
  int hidden_dim;
  int nw;
  int64_t vocab_offset;
  void* logits;
  int64_t logits_stride;
  float* top_value;
  int64_t* top_index;
  int64_t* top_key;
  unsigned long long* keys;
  unsigned int* ticket;
  int* error;
  int32_t* tile_list;     // workspace: compacted active tile ids
  int32_t* tile_counts;   // workspace: per-builder-block active tile counts
  int dense;              // 1: every tile is projected (dense_masked_logits)
  int no_pdl;             // 1: launch the projection without programmatic dependent launch
  PeerExchange peers;     // cross-rank top-1 merge (world < 2: none)
  // fused sampler (sample_index != nullptr; contract in gsp_sampler.cuh)
  int64_t* sample_index;
  float* sample_lse;
  int64_t* sample_key;
  const uint64_t* seeds;
  uint64_t offset;
  float inv_temp;
  unsigned long long* sample_keys;    // workspace [batch]
  unsigned long long* stat_partials;  // workspace [batch][kMaxSlices]
};

// Workspace layout (fixed offsets first, so calls with different batch sizes
// can share one buffer): [0] arrival ticket, [4] error word, [8..32) the
// device route selector's state (its ticket, active-tile count, legal-token
// total, route word), [32] per-request top-1 keys, then the tile lists of the block / dense path, the per-CTA slice
// counts and flags and the unit list of the cooperative row-sparse kernel.
// Every kernel leaves all of it zero except the error word (calls of other
// sizes carve the same bytes differently, so nothing may be left behind). A
// launch that set the error word may have left state behind: the caller
// re-zeroes such a workspace before reusing it.
constexpr size_t kKeysOffset = 32;

struct Workspace {
  unsigned long long* keys;
  unsigned int* route_ticket;       // [8]
  unsigned int* route_active;       // [12] active 128-row tiles
  unsigned long long* route_legal;  // [16] legal tokens over the batch
  int* route_word;                  // [24] chosen route (eager calls read it back)
  unsigned int* ticket;
  int* error;
  int32_t* tile_list;
  int32_t* tile_counts;
  unsigned int* slice_counts;
  unsigned int* published;
  unsigned int* slice_ready;
  uint32_t* unit_list;
  int64_t list_cap;
  unsigned long long* sample_keys;
  unsigned long long* stat_partials;
};

// Active-tile builder granularity: tiles per builder block (one count each).
constexpr int kBuilderTiles = 32;
// Upper bound on the grid of the cooperative row-sparse kernel (one slice
// count per CTA).
constexpr int kMaxSlices = 512;
// Words between consecutive slice flags (one 128-byte line each).
constexpr int kFlagStride = 32;
// Units the cooperative kernel's list holds at most (4 bytes each).
constexpr size_t kUnitListMax = size_t(1) << 20;

constexpr size_t unit_list_cap(size_t batch, size_t vocab) {
  return batch * vocab < kUnitListMax ? batch * vocab : kUnitListMax;
}

constexpr size_t align256c(size_t x) { return (x + 255) / 256 * 256; }

// Workspace bytes for (batch, vocab) of every call but the sampler: ticket +
// error word + one 64-bit key per request, the compacted active-tile list, the
// per-builder-block counts, the slice counts and flags, and the unit list.
constexpr size_t row_sparse_workspace_bytes_for(size_t batch, size_t vocab) {
  return align256c(kKeysOffset + 8 * batch) + align256c(4 * ((vocab + 127) / 128)) +
         align256c(4 * (((vocab + 127) / 128 + kBuilderTiles - 1) / kBuilderTiles)) + align256c(4 * kMaxSlices + 256) +
         align256c(4 * kMaxSlices * kFlagStride) + align256c(4 * unit_list_cap(batch, vocab));
}

// ... plus the sampler's per-request keys and per-CTA (max, sum) partials.
constexpr size_t workspace_bytes_for(size_t batch, size_t vocab) {
  return row_sparse_workspace_bytes_for(batch, vocab) + align256c(8 * batch) + align256c(8 * kMaxSlices * batch);
}

size_t workspace_bytes(int batch, int vocab);
size_t row_sparse_workspace_bytes(int batch, int vocab);
Workspace carve_workspace(void* base, int batch, int vocab);

int num_sms(int device);

// Records `code` with a printf-style message as the calling thread's
// gsp_last_error() and returns `code`.
int32_t record_error(int32_t code, const char* fmt, ...);

// Raises cudaFuncAttributeMaxDynamicSharedMemorySize of `func` on `device` to at
// least `bytes` (thread-safe; a no-op when the current setting suffices).
cudaError_t raise_smem_limit(const void* func, size_t bytes, int device);

// Each launcher returns a cudaError_t value (cudaSuccess == 0). dtype: 0 fp16,
// 1 bf16, 2 fp32 (row-sparse kernels only).
cudaError_t launch_row_sparse(const RowSparseParams& p, int dtype, cudaStream_t stream);
cudaError_t launch_ids_to_bitmask(const int64_t* ids, int64_t count, int vocab, uint32_t* mask,
                                  unsigned long long* stats, cudaStream_t stream);
cudaError_t launch_mask_stats(const uint32_t* mask, int64_t stride, int batch, int vocab,
                              int32_t* legal_counts, int32_t* full_words, int32_t* active_tiles,
                              cudaStream_t stream);
cudaError_t launch_copy_bytes(void* dst, const void* src, size_t bytes, cudaStream_t stream);
// The copy kernel launch_copy_bytes uses (arguments: dst, src, bytes, vec16),
// for finding its node in a captured graph.
const void* copy_bytes_kernel_fn();
cudaError_t launch_merge_logsumexp(const float* lse, int parts, int batch, float* out, cudaStream_t stream);
cudaError_t launch_top1_from_keys(const int64_t* keys, int batch, float* top_value,
                                  int64_t* top_index, cudaStream_t stream);
cudaError_t launch_block_gemm(const BlockGemmParams& p, int dtype, cudaStream_t stream);

// ---- device-side route choice ----------------------------------------------
// Route cost model (mirrors gsp_route_cost): each route is a fixed latency plus
// its bytes at the rate measured for its kernel on B200.
struct RouteCost {
  double hbm_gbs;              // legal rows and logits of the row-sparse kernels
  double row_sparse_fixed_us;  // launch, mask scan / slice-count exchange, top-1 merge
  double block_floor_us;       // tile builder + tensor-core pipeline: least a block call costs
  double block_fixed_us;
  double block_gbs;            // effective rate over the active tiles
  double dense_fixed_us;
  double dense_gbs;
  double group_split_fixed_us; // a lane-group split: row gathers, second route launch, un-permute
};
constexpr RouteCost kB200RouteCost = {6000.0, 9.0, 24.0, 10.0, 3800.0, 5.0, 6000.0, 10.0};

// Cheapest route for `batch` requests with these statistics: 0 row-sparse,
// 1 block-sparse, 2 dense-mask; its modelled time (us) in *cost_us. Same
// arithmetic (doubles, in this order) and tie order (block, dense, row) as
// the Python choose_route. Batch 1 is row-sparse; batch 0 costs nothing.
__host__ __device__ inline int best_route_by_cost(int batch, int vocab, int hidden_dim, int elem_bytes,
                                                  long long legal_total, long long active_tiles, const RouteCost& c,
                                                  double* cost_us) {
  const long long row_bytes = (long long)hidden_dim * elem_bytes;
  const long long out_bytes = (long long)batch * vocab * elem_bytes;
  const double t_row = c.row_sparse_fixed_us + (double)(legal_total * row_bytes + out_bytes) / (c.hbm_gbs * 1e3);
  if (batch <= 1) {
    if (cost_us) *cost_us = batch <= 0 ? 0.0 : t_row;
    return 0;
  }
  long long rows = active_tiles * 128;
  if (rows > vocab) rows = vocab;
  double t_block = c.block_fixed_us + (double)(rows * row_bytes) / (c.block_gbs * 1e3);
  if (c.block_floor_us > t_block) t_block = c.block_floor_us;
  const double t_dense = c.dense_fixed_us + (double)((long long)vocab * row_bytes) / (c.dense_gbs * 1e3);
  int best = 1;
  double bt = t_block;
  if (t_dense < bt) { best = 2; bt = t_dense; }
  if (t_row < bt) { best = 0; bt = t_row; }
  if (cost_us) *cost_us = bt;
  return best;
}

__host__ __device__ inline int choose_route_by_cost(int batch, int vocab, int hidden_dim, int elem_bytes,
                                                    long long legal_total, long long active_tiles,
                                                    const RouteCost& c) {
  return best_route_by_cost(batch, vocab, hidden_dim, elem_bytes, legal_total, active_tiles, c, nullptr);
}

struct RouteSelectParams {
  const uint32_t* mask;
  int64_t mask_stride;
  int batch, vocab, nw, ntiles, hidden_dim, elem_bytes;
  RouteCost cost;
  unsigned int* ticket;            // workspace: selector arrival ticket
  unsigned int* active;            // workspace: active-tile count
  unsigned long long* legal;       // workspace: legal-token total
  int* route_word;                 // workspace route word (eager calls), or nullptr
  int32_t* route_out;              // caller's device route, or nullptr
  cudaGraphConditionalHandle handle;
  int has_handle;                  // set the SWITCH node's value
};

// Selector: legal tokens and active tiles of the batch, then (last block) the
// cost model; leaves its workspace counters zero.
cudaError_t launch_route_select(const RouteSelectParams& p, cudaStream_t stream);

// ---- lane grouping by density class ----------------------------------------
// Plan buffer (caller's int32 [kPlanHeader + 6 * batch], zeroed by the
// launcher): header [0] k = requests of group A (0: no split), [1] route of
// group A, [2] route of group B, [3] best single route, [4] its modelled ns,
// [5] the chosen split's modelled ns (-1 without a split), [6] [7] arrival
// tickets; then order[B] (position -> request, ascending fill), inverse[B],
// legal[B], tiles[B], hist_min[B], hist_max[B].
constexpr int kPlanHeader = 16;
constexpr int kGroupMaxBatch = 256;

struct GroupPlanParams {
  const uint32_t* mask;
  int64_t mask_stride;
  int batch, vocab, nw, ntiles, hidden_dim, elem_bytes, with_logits;
  RouteCost cost;
  int32_t* plan;
};

cudaError_t launch_group_plan(const GroupPlanParams& p, cudaStream_t stream);
cudaError_t launch_gather_rows(const void* src, int64_t src_stride, const int32_t* rows, int n, int64_t row_bytes,
                               void* dst, int64_t dst_stride, cudaStream_t stream);

// Number of builder blocks used by the active-tile builder for `vocab`.
int tile_builder_blocks(int vocab);

}  // namespace gsp
