// extern "C" entry points declared in include/gsp_b200.h: argument validation,
// workspace carving and dispatch to the kernel launchers. No exception, abort
// or host synchronisation happens here.
#include <cstdarg>
#include <cstdio>
#include <cmath>
#include <cstring>
#include <mutex>

#include "../../include/gsp_b200.h"
#include "gsp_internal.h"

namespace gsp {
namespace {

thread_local char g_last_error[512] = "";
// Set while this thread records a conditional node's body (see kConditionalBodyPdl).
thread_local bool tl_no_pdl = false;

int32_t fail(int32_t code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int32_t cuda_status(cudaError_t err, const char* where) {
  if (err == cudaSuccess) return GSP_OK;
  return fail(GSP_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorName(err), cudaGetErrorString(err));
}

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

int tile_builder_blocks(int vocab) {
  const int ntiles = (vocab + GSP_TILE_ROWS - 1) / GSP_TILE_ROWS;
  return (ntiles + kBuilderTiles - 1) / kBuilderTiles;
}

size_t workspace_bytes(int batch, int vocab) { return workspace_bytes_for((size_t)batch, (size_t)vocab); }
size_t row_sparse_workspace_bytes(int batch, int vocab) {
  return row_sparse_workspace_bytes_for((size_t)batch, (size_t)vocab);
}

Workspace carve_workspace(void* base, int batch, int vocab) {
  const int ntiles = (vocab + GSP_TILE_ROWS - 1) / GSP_TILE_ROWS;
  char* p = static_cast<char*>(base);
  Workspace w;
  w.ticket = reinterpret_cast<unsigned int*>(p);
  w.error = reinterpret_cast<int*>(p + 4);
  w.route_ticket = reinterpret_cast<unsigned int*>(p + 8);
  w.route_active = reinterpret_cast<unsigned int*>(p + 12);
  w.route_legal = reinterpret_cast<unsigned long long*>(p + 16);
  w.route_word = reinterpret_cast<int*>(p + 24);
  w.keys = reinterpret_cast<unsigned long long*>(p + kKeysOffset);
  p += align256(kKeysOffset + sizeof(unsigned long long) * (size_t)batch);
  w.tile_list = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * (size_t)ntiles);
  w.tile_counts = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * (size_t)((ntiles + kBuilderTiles - 1) / kBuilderTiles));
  w.slice_counts = reinterpret_cast<unsigned int*>(p);
  w.published = reinterpret_cast<unsigned int*>(p + sizeof(unsigned int) * kMaxSlices + 128);
  p += align256(sizeof(unsigned int) * kMaxSlices + 256);
  w.slice_ready = reinterpret_cast<unsigned int*>(p);
  p += align256(sizeof(unsigned int) * kMaxSlices * kFlagStride);
  w.unit_list = reinterpret_cast<uint32_t*>(p);
  w.list_cap = (int64_t)unit_list_cap((size_t)batch, (size_t)vocab);
  p += align256(sizeof(uint32_t) * (size_t)w.list_cap);
  w.sample_keys = reinterpret_cast<unsigned long long*>(p);
  p += align256(sizeof(unsigned long long) * (size_t)batch);
  w.stat_partials = reinterpret_cast<unsigned long long*>(p);
  return w;
}

int num_sms(int device) {
  static int cache[128] = {0};
  if (device < 0 || device >= 128) return 148;
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    cache[device] = n;
  }
  return cache[device];
}

int32_t record_error(int32_t code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

cudaError_t raise_smem_limit(const void* func, size_t bytes, int device) {
  struct Entry {
    const void* func;
    int device;
    int bytes;
  };
  static std::mutex mu;
  static Entry table[256];
  static int used = 0;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i) {
    if (table[i].func == func && table[i].device == device) {
      if ((int)bytes <= table[i].bytes) return cudaSuccess;
      cudaError_t err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
      if (err == cudaSuccess) table[i].bytes = (int)bytes;
      return err;
    }
  }
  cudaError_t err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (err == cudaSuccess && used < 256) table[used++] = Entry{func, device, (int)bytes};
  return err;
}

namespace {

// Checks shared by every projection entry point.
int32_t validate_projection(const char* fn, const void* hidden, int64_t hidden_row_stride,
                            const void* weight, int64_t weight_row_stride, const int32_t* bitmask,
                            int64_t bitmask_row_stride, int32_t batch, int32_t vocab,
                            int32_t hidden_dim, int32_t dtype, const void* logits,
                            int64_t logits_row_stride) {
  if (!hidden || !weight) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: hidden and weight must be non-null", fn);
  if (batch < 1 || vocab < 1 || hidden_dim < 1)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: batch, vocab and hidden_dim must be positive", fn);
  if (dtype != GSP_DTYPE_F16 && dtype != GSP_DTYPE_BF16 && dtype != GSP_DTYPE_F32)
    return fail(GSP_ERR_UNSUPPORTED, "%s: dtype must be GSP_DTYPE_F16, GSP_DTYPE_BF16 or GSP_DTYPE_F32", fn);
  if (batch > 1 && hidden_row_stride < hidden_dim)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: hidden_row_stride < hidden_dim", fn);
  if (vocab > 1 && weight_row_stride < hidden_dim)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: weight_row_stride < hidden_dim", fn);
  const int64_t nw = (vocab + 31) / 32;
  if (bitmask && batch > 1 && bitmask_row_stride != 0 && bitmask_row_stride < nw)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: bitmask_row_stride must be 0 or >= ceil(vocab/32)", fn);
  if (bitmask_row_stride < 0) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: negative bitmask_row_stride", fn);
  if (logits && batch > 1 && logits_row_stride < vocab)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: logits_row_stride < vocab", fn);
  if ((uint64_t)batch * (uint64_t)nw * 32ull > 0xffffffffull)
    return fail(GSP_ERR_UNSUPPORTED, "%s: batch * vocab too large (limit 2^32 tokens)", fn);
  return GSP_OK;
}

// full: the call uses the sampler's part of the workspace too.
int32_t check_workspace(const char* fn, bool needed, void* workspace, size_t bytes, int32_t batch,
                        int32_t vocab, bool full = false) {
  if (!needed) return GSP_OK;
  if (!workspace) return fail(GSP_ERR_WORKSPACE, "%s: workspace is required for this call", fn);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(GSP_ERR_WORKSPACE, "%s: workspace must be 256-byte aligned", fn);
  const size_t need = full ? workspace_bytes(batch, vocab) : row_sparse_workspace_bytes(batch, vocab);
  if (bytes < need)
    return fail(GSP_ERR_WORKSPACE, "%s: workspace has %zu bytes, needs %zu", fn, bytes, need);
  return GSP_OK;
}

RowSparseParams make_row_sparse(const void* hidden, int64_t hidden_row_stride, const void* weight,
                                int64_t weight_row_stride, const int32_t* bitmask,
                                int64_t bitmask_row_stride, int32_t batch, int32_t vocab,
                                int32_t hidden_dim, int64_t vocab_offset) {
  RowSparseParams p;
  std::memset(&p, 0, sizeof(p));
  p.hidden = hidden;
  p.hidden_stride = batch > 1 ? hidden_row_stride : hidden_dim;
  p.weight = weight;
  p.weight_stride = vocab > 1 ? weight_row_stride : hidden_dim;
  p.mask = reinterpret_cast<const uint32_t*>(bitmask);
  p.mask_stride = batch > 1 ? bitmask_row_stride : 0;
  p.batch = batch;
  p.vocab = vocab;
  p.hidden_dim = hidden_dim;
  p.nw = (vocab + 31) / 32;
  p.vocab_offset = vocab_offset;
  return p;
}

void attach_workspace(RowSparseParams& p, void* workspace) {
  const Workspace w = carve_workspace(workspace, p.batch, p.vocab);
  p.keys = w.keys;
  p.ticket = w.ticket;
  p.error = w.error;
  p.slice_counts = w.slice_counts;
  p.published = w.published;
  p.slice_ready = w.slice_ready;
  p.unit_list = w.unit_list;
  p.list_cap = w.list_cap;
  p.sample_keys = w.sample_keys;
  p.stat_partials = w.stat_partials;
}

int32_t projection_common(const char* fn, bool tensor_core, int dense, const void* hidden,
                          int64_t hidden_row_stride, const void* weight, int64_t weight_row_stride,
                          const int32_t* bitmask, int64_t bitmask_row_stride, int32_t batch,
                          int32_t vocab, int32_t hidden_dim, int32_t dtype, int64_t vocab_offset,
                          void* logits, int64_t logits_row_stride, float* top_value,
                          int64_t* top_index, int64_t* top_key, void* workspace,
                          size_t workspace_bytes_, void* stream, const PeerExchange* peers = nullptr) {
  int32_t st = validate_projection(fn, hidden, hidden_row_stride, weight, weight_row_stride, bitmask,
                                   bitmask_row_stride, batch, vocab, hidden_dim, dtype, logits,
                                   logits_row_stride);
  if (st != GSP_OK) return st;
  const bool want_top = top_value || top_index || top_key;
  st = check_workspace(fn, want_top || tensor_core, workspace, workspace_bytes_, batch, vocab);
  if (st != GSP_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // fp32: the tensor-core kernels take half-precision operands, so the block
  // and dense routes run the row-sparse kernel (same outputs: legal rows dotted
  // in fp32, -inf elsewhere; the dense route with no mask projects every row)
  if (!tensor_core || dtype == GSP_DTYPE_F32) {
    RowSparseParams p = make_row_sparse(hidden, hidden_row_stride, weight, weight_row_stride,
                                        bitmask, bitmask_row_stride, batch, vocab, hidden_dim,
                                        vocab_offset);
    p.logits = logits;
    p.logits_stride = batch > 1 ? logits_row_stride : vocab;
    p.top_value = top_value;
    p.top_index = top_index;
    p.top_key = top_key;
    if (workspace) attach_workspace(p, workspace);
    if (peers) p.peers = *peers;
    return cuda_status(launch_row_sparse(p, dtype, s), fn);
  }
  BlockGemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.hidden = hidden;
  p.hidden_stride = batch > 1 ? hidden_row_stride : hidden_dim;
  p.weight = weight;
  p.weight_stride = vocab > 1 ? weight_row_stride : hidden_dim;
  p.mask = reinterpret_cast<const uint32_t*>(bitmask);
  p.mask_stride = batch > 1 ? bitmask_row_stride : 0;
  p.batch = batch;
  p.vocab = vocab;
  p.hidden_dim = hidden_dim;
  p.nw = (vocab + 31) / 32;
  p.vocab_offset = vocab_offset;
  p.logits = logits;
  p.logits_stride = batch > 1 ? logits_row_stride : vocab;
  p.top_value = top_value;
  p.top_index = top_index;
  p.top_key = top_key;
  Workspace w = carve_workspace(workspace, batch, vocab);
  p.keys = w.keys;
  p.ticket = w.ticket;
  p.error = w.error;
  p.tile_list = w.tile_list;
  p.tile_counts = w.tile_counts;
  p.dense = dense || bitmask == nullptr;
  p.no_pdl = tl_no_pdl ? 1 : 0;
  if (peers) p.peers = *peers;
  return cuda_status(launch_block_gemm(p, dtype, s), fn);
}

// ---- device-side route choice ---------------------------------------------
// Programmatic dependent launch between the tile builder and the projection
// inside a conditional node's body.
constexpr bool kConditionalBodyPdl = true;

int32_t route_call(const char* fn, int route, const void* hidden, int64_t hidden_row_stride, const void* weight,
                   int64_t weight_row_stride, const int32_t* bitmask, int64_t bitmask_row_stride, int32_t batch,
                   int32_t vocab, int32_t hidden_dim, int32_t dtype, void* logits, int64_t logits_row_stride,
                   float* top_value, int64_t* top_index, void* workspace, size_t workspace_bytes_, void* stream) {
  const bool tc = route != GSP_ROUTE_ROW_SPARSE;
  return projection_common(fn, tc, route == GSP_ROUTE_DENSE_MASK ? 1 : 0, hidden, hidden_row_stride, weight,
                           weight_row_stride, bitmask, bitmask_row_stride, batch, vocab, hidden_dim, dtype, 0, logits,
                           logits_row_stride, top_value, top_index, nullptr, workspace, workspace_bytes_, stream);
}

// One non-blocking stream per device for recording conditional bodies; the
// mutex also serialises body recording between threads.
std::mutex g_body_mu;
cudaStream_t body_stream(int device) {
  static cudaStream_t streams[128] = {};
  if (device < 0 || device >= 128) return nullptr;
  if (!streams[device] && cudaStreamCreateWithFlags(&streams[device], cudaStreamNonBlocking) != cudaSuccess)
    streams[device] = nullptr;
  return streams[device];
}

}  // namespace
}  // namespace gsp

using namespace gsp;

extern "C" {

int32_t gsp_abi_version(void) { return GSP_ABI_VERSION; }

const char* gsp_status_string(int32_t status) {
  switch (status) {
    case GSP_OK: return "GSP_OK";
    case GSP_ERR_INVALID_ARGUMENT: return "GSP_ERR_INVALID_ARGUMENT";
    case GSP_ERR_UNSUPPORTED: return "GSP_ERR_UNSUPPORTED";
    case GSP_ERR_WORKSPACE: return "GSP_ERR_WORKSPACE";
    case GSP_ERR_CUDA: return "GSP_ERR_CUDA";
    default: return "GSP_ERR_UNKNOWN";
  }
}

const char* gsp_last_error(void) { return g_last_error; }

size_t gsp_workspace_bytes(int32_t batch, int32_t vocab) {
  if (batch < 1 || vocab < 1) return 0;
  return workspace_bytes(batch, vocab);
}

int32_t gsp_row_sparse_logits(const void* hidden, int64_t hidden_row_stride, const void* weight,
                              int64_t weight_row_stride, const int32_t* bitmask,
                              int64_t bitmask_row_stride, int32_t batch, int32_t vocab,
                              int32_t hidden_dim, int32_t dtype, int64_t vocab_offset, void* logits,
                              int64_t logits_row_stride, float* top_value, int64_t* top_index,
                              int64_t* top_key, void* workspace, size_t workspace_bytes_,
                              void* stream) {
  return projection_common("gsp_row_sparse_logits", false, 0, hidden, hidden_row_stride, weight,
                           weight_row_stride, bitmask, bitmask_row_stride, batch, vocab, hidden_dim,
                           dtype, vocab_offset, logits, logits_row_stride, top_value, top_index,
                           top_key, workspace, workspace_bytes_, stream);
}

int32_t gsp_row_sparse_compact(const void* hidden, int64_t hidden_row_stride, const void* weight,
                               int64_t weight_row_stride, const int32_t* bitmask,
                               int64_t bitmask_row_stride, int32_t batch, int32_t vocab,
                               int32_t hidden_dim, int32_t dtype, int64_t vocab_offset,
                               void* compact_logits, int64_t* compact_ids, int64_t capacity,
                               int64_t* request_offsets, float* top_value, int64_t* top_index,
                               int64_t* top_key, void* workspace, size_t workspace_bytes_,
                               void* stream) {
  const char* fn = "gsp_row_sparse_compact";
  int32_t st = validate_projection(fn, hidden, hidden_row_stride, weight, weight_row_stride, bitmask,
                                   bitmask_row_stride, batch, vocab, hidden_dim, dtype, nullptr, 0);
  if (st != GSP_OK) return st;
  if (capacity < 0) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: negative capacity", fn);
  if (capacity > 0 && (!compact_logits || !compact_ids))
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: compact_logits and compact_ids are required", fn);
  if (!request_offsets) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: request_offsets is required", fn);
  const bool want_top = top_value || top_index || top_key;
  st = check_workspace(fn, want_top, workspace, workspace_bytes_, batch, vocab);
  if (st != GSP_OK) return st;
  RowSparseParams p = make_row_sparse(hidden, hidden_row_stride, weight, weight_row_stride, bitmask,
                                      bitmask_row_stride, batch, vocab, hidden_dim, vocab_offset);
  p.compact = capacity > 0 ? compact_logits : nullptr;
  p.compact_ids = compact_ids;
  p.capacity = capacity;
  p.offsets = request_offsets;
  p.top_value = top_value;
  p.top_index = top_index;
  p.top_key = top_key;
  if (workspace) attach_workspace(p, workspace);
  return cuda_status(launch_row_sparse(p, dtype, static_cast<cudaStream_t>(stream)), fn);
}

int32_t gsp_ids_to_bitmask(const int64_t* ids, int64_t count, int32_t vocab, int32_t* bitmask,
                           int64_t* stats, void* stream) {
  const char* fn = "gsp_ids_to_bitmask";
  if (vocab < 1) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: vocab must be positive", fn);
  if (count < 0 || (count > 0 && !ids)) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: bad ids", fn);
  if (!bitmask || !stats) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: bitmask and stats are required", fn);
  return cuda_status(launch_ids_to_bitmask(ids, count, vocab, reinterpret_cast<uint32_t*>(bitmask),
                                           reinterpret_cast<unsigned long long*>(stats),
                                           static_cast<cudaStream_t>(stream)),
                     fn);
}

int32_t gsp_mask_stats(const int32_t* bitmask, int64_t bitmask_row_stride, int32_t batch,
                       int32_t vocab, int32_t* legal_counts, int32_t* full_words,
                       int32_t* active_tiles, void* stream) {
  const char* fn = "gsp_mask_stats";
  if (!bitmask) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: bitmask is required", fn);
  if (batch < 1 || vocab < 1) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: batch and vocab must be positive", fn);
  const int64_t nw = (vocab + 31) / 32;
  if (batch > 1 && bitmask_row_stride != 0 && bitmask_row_stride < nw)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: bitmask_row_stride must be 0 or >= ceil(vocab/32)", fn);
  if (bitmask_row_stride < 0) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: negative bitmask_row_stride", fn);
  return cuda_status(launch_mask_stats(reinterpret_cast<const uint32_t*>(bitmask),
                                       batch > 1 ? bitmask_row_stride : 0, batch, vocab,
                                       legal_counts, full_words, active_tiles,
                                       static_cast<cudaStream_t>(stream)),
                     fn);
}

int32_t gsp_block_gemm_logits(const void* hidden, int64_t hidden_row_stride, const void* weight,
                              int64_t weight_row_stride, const int32_t* bitmask,
                              int64_t bitmask_row_stride, int32_t batch, int32_t vocab,
                              int32_t hidden_dim, int32_t dtype, int64_t vocab_offset, void* logits,
                              int64_t logits_row_stride, float* top_value, int64_t* top_index,
                              int64_t* top_key, void* workspace, size_t workspace_bytes_,
                              void* stream) {
  return projection_common("gsp_block_gemm_logits", true, 0, hidden, hidden_row_stride, weight,
                           weight_row_stride, bitmask, bitmask_row_stride, batch, vocab, hidden_dim,
                           dtype, vocab_offset, logits, logits_row_stride, top_value, top_index,
                           top_key, workspace, workspace_bytes_, stream);
}

int32_t gsp_dense_masked_logits(const void* hidden, int64_t hidden_row_stride, const void* weight,
                                int64_t weight_row_stride, const int32_t* bitmask,
                                int64_t bitmask_row_stride, int32_t batch, int32_t vocab,
                                int32_t hidden_dim, int32_t dtype, int64_t vocab_offset,
                                void* logits, int64_t logits_row_stride, float* top_value,
                                int64_t* top_index, int64_t* top_key, void* workspace,
                                size_t workspace_bytes_, void* stream) {
  return projection_common("gsp_dense_masked_logits", true, 1, hidden, hidden_row_stride, weight,
                           weight_row_stride, bitmask, bitmask_row_stride, batch, vocab, hidden_dim,
                           dtype, vocab_offset, logits, logits_row_stride, top_value, top_index,
                           top_key, workspace, workspace_bytes_, stream);
}

int32_t gsp_top1_from_keys(const int64_t* keys, int32_t batch, float* top_value, int64_t* top_index,
                           void* stream) {
  const char* fn = "gsp_top1_from_keys";
  if (!keys || batch < 1) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: keys and batch are required", fn);
  return cuda_status(
      launch_top1_from_keys(keys, batch, top_value, top_index, static_cast<cudaStream_t>(stream)),
      fn);
}

// The fused sampler on any route: validation shared by the entry points, then
// the row-sparse kernels (route 0) or the tensor-core kernels (1 block-sparse,
// 2 dense) with the sampler in their epilogue.
static int32_t sample_common(const char* fn, int32_t route, const void* hidden, int64_t hidden_row_stride,
                      const void* weight, int64_t weight_row_stride, const int32_t* bitmask,
                      int64_t bitmask_row_stride, int32_t batch, int32_t vocab, int32_t hidden_dim, int32_t dtype,
                      int64_t vocab_offset, void* logits, int64_t logits_row_stride, float temperature,
                      const uint64_t* seeds, uint64_t offset, int64_t* sample_index, float* sample_logsumexp,
                      int64_t* sample_key, float* top_value, int64_t* top_index, int64_t* top_key, void* workspace,
                      size_t workspace_bytes_, void* stream) {
  if (route != GSP_ROUTE_ROW_SPARSE && route != GSP_ROUTE_BLOCK_SPARSE && route != GSP_ROUTE_DENSE_MASK)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: unknown route %d", fn, route);
  int32_t st = validate_projection(fn, hidden, hidden_row_stride, weight, weight_row_stride, bitmask,
                                   bitmask_row_stride, batch, vocab, hidden_dim, dtype, logits, logits_row_stride);
  if (st != GSP_OK) return st;
  if (dtype == GSP_DTYPE_F32) return fail(GSP_ERR_UNSUPPORTED, "%s: the sampler takes GSP_DTYPE_F16 or GSP_DTYPE_BF16", fn);
  if (!(temperature > 0.f) || !std::isfinite(temperature))
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: temperature must be positive and finite", fn);
  if (!seeds || !sample_index) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: seeds and sample_index are required", fn);
  st = check_workspace(fn, true, workspace, workspace_bytes_, batch, vocab, true);
  if (st != GSP_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (route == GSP_ROUTE_ROW_SPARSE) {
    RowSparseParams p = make_row_sparse(hidden, hidden_row_stride, weight, weight_row_stride, bitmask,
                                        bitmask_row_stride, batch, vocab, hidden_dim, vocab_offset);
    p.logits = logits;
    p.logits_stride = batch > 1 ? logits_row_stride : vocab;
    p.top_value = top_value;
    p.top_index = top_index;
    p.top_key = top_key;
    attach_workspace(p, workspace);
    p.sample_index = sample_index;
    p.sample_lse = sample_logsumexp;
    p.sample_key = sample_key;
    p.seeds = seeds;
    p.offset = offset;
    p.inv_temp = 1.0f / temperature;
    return cuda_status(launch_row_sparse(p, dtype, s), fn);
  }
  BlockGemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.hidden = hidden;
  p.hidden_stride = batch > 1 ? hidden_row_stride : hidden_dim;
  p.weight = weight;
  p.weight_stride = vocab > 1 ? weight_row_stride : hidden_dim;
  p.mask = reinterpret_cast<const uint32_t*>(bitmask);
  p.mask_stride = batch > 1 ? bitmask_row_stride : 0;
  p.batch = batch;
  p.vocab = vocab;
  p.hidden_dim = hidden_dim;
  p.nw = (vocab + 31) / 32;
  p.vocab_offset = vocab_offset;
  p.logits = logits;
  p.logits_stride = batch > 1 ? logits_row_stride : vocab;
  p.top_value = top_value;
  p.top_index = top_index;
  p.top_key = top_key;
  Workspace w = carve_workspace(workspace, batch, vocab);
  p.keys = w.keys;
  p.ticket = w.ticket;
  p.error = w.error;
  p.tile_list = w.tile_list;
  p.tile_counts = w.tile_counts;
  p.dense = route == GSP_ROUTE_DENSE_MASK || bitmask == nullptr;
  p.no_pdl = tl_no_pdl ? 1 : 0;
  p.sample_index = sample_index;
  p.sample_lse = sample_logsumexp;
  p.sample_key = sample_key;
  p.seeds = seeds;
  p.offset = offset;
  p.inv_temp = 1.0f / temperature;
  p.sample_keys = w.sample_keys;
  p.stat_partials = w.stat_partials;
  return cuda_status(launch_block_gemm(p, dtype, s), fn);
}

int32_t gsp_row_sparse_sample(const void* hidden, int64_t hidden_row_stride, const void* weight,
                              int64_t weight_row_stride, const int32_t* bitmask, int64_t bitmask_row_stride,
                              int32_t batch, int32_t vocab, int32_t hidden_dim, int32_t dtype,
                              int64_t vocab_offset, void* logits, int64_t logits_row_stride, float temperature,
                              const uint64_t* seeds, uint64_t offset, int64_t* sample_index,
                              float* sample_logsumexp, int64_t* sample_key, float* top_value, int64_t* top_index,
                              int64_t* top_key, void* workspace, size_t workspace_bytes_, void* stream) {
  return sample_common("gsp_row_sparse_sample", GSP_ROUTE_ROW_SPARSE, hidden, hidden_row_stride, weight,
                       weight_row_stride, bitmask, bitmask_row_stride, batch, vocab, hidden_dim, dtype, vocab_offset,
                       logits, logits_row_stride, temperature, seeds, offset, sample_index, sample_logsumexp,
                       sample_key, top_value, top_index, top_key, workspace, workspace_bytes_, stream);
}

int32_t gsp_sample(int32_t route, const void* hidden, int64_t hidden_row_stride, const void* weight,
                   int64_t weight_row_stride, const int32_t* bitmask, int64_t bitmask_row_stride, int32_t batch,
                   int32_t vocab, int32_t hidden_dim, int32_t dtype, int64_t vocab_offset, void* logits,
                   int64_t logits_row_stride, float temperature, const uint64_t* seeds, uint64_t offset,
                   int64_t* sample_index, float* sample_logsumexp, int64_t* sample_key, float* top_value,
                   int64_t* top_index, int64_t* top_key, void* workspace, size_t workspace_bytes_, void* stream) {
  return sample_common("gsp_sample", route, hidden, hidden_row_stride, weight, weight_row_stride, bitmask,
                       bitmask_row_stride, batch, vocab, hidden_dim, dtype, vocab_offset, logits, logits_row_stride,
                       temperature, seeds, offset, sample_index, sample_logsumexp, sample_key, top_value, top_index,
                       top_key, workspace, workspace_bytes_, stream);
}

int32_t gsp_vocab_parallel_logits(int32_t route, const void* hidden, int64_t hidden_row_stride,
                                  const void* weight, int64_t weight_row_stride, const int32_t* bitmask,
                                  int64_t bitmask_row_stride, int32_t batch, int32_t vocab,
                                  int32_t hidden_dim, int32_t dtype, int64_t vocab_offset, void* logits,
                                  int64_t logits_row_stride, float* top_value, int64_t* top_index,
                                  int64_t* top_key, void* workspace, size_t workspace_bytes_,
                                  void* const* peer_buffers, int32_t rank, int32_t world_size,
                                  int32_t max_batch, int64_t total_vocab, int64_t wait_us, void* stream) {
  const char* fn = "gsp_vocab_parallel_logits";
  if (route != GSP_ROUTE_ROW_SPARSE && route != GSP_ROUTE_BLOCK_SPARSE && route != GSP_ROUTE_DENSE_MASK)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: unknown route %d", fn, route);
  if (world_size < 1 || world_size > kMaxPeers || rank < 0 || rank >= world_size)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: rank %d / world size %d (at most %d ranks)", fn, rank,
                world_size, kMaxPeers);
  if (!top_value && !top_index && !top_key)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: the exchange merges top-1; give top_value, top_index or top_key", fn);
  PeerExchange x;
  std::memset(&x, 0, sizeof(x));
  x.rank = rank;
  x.world = world_size;
  x.max_batch = max_batch;
  x.wait_ns = (wait_us > 0 ? wait_us : kDefaultPeerWaitUs) * 1000;
  if (vocab_offset < 0 || vocab_offset + (int64_t)vocab > total_vocab)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: shard [%lld, %lld) outside the head's %lld tokens", fn,
                (long long)vocab_offset, (long long)(vocab_offset + vocab), (long long)total_vocab);
  x.tagged = total_vocab < (int64_t)0xFFFFFF;  // the same on every rank
  if (world_size > 1) {
    if (!peer_buffers) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: peer_buffers is required", fn);
    if (batch > max_batch)
      return fail(GSP_ERR_INVALID_ARGUMENT, "%s: batch %d exceeds the exchange's max_batch %d", fn, batch, max_batch);
    for (int q = 0; q < world_size; ++q) {
      if (!peer_buffers[q]) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: peer_buffers[%d] is NULL", fn, q);
      x.buf[q] = static_cast<unsigned char*>(peer_buffers[q]);
    }
  }
  const bool tc = route != GSP_ROUTE_ROW_SPARSE;
  return projection_common(fn, tc, route == GSP_ROUTE_DENSE_MASK ? 1 : 0, hidden, hidden_row_stride, weight,
                           weight_row_stride, bitmask, bitmask_row_stride, batch, vocab, hidden_dim, dtype, vocab_offset, logits,
                           logits_row_stride, top_value, top_index, top_key, workspace, workspace_bytes_,
                           stream, &x);
}

void gsp_default_route_cost(gsp_route_cost* cost) {
  if (!cost) return;
  cost->hbm_gbs = kB200RouteCost.hbm_gbs;
  cost->row_sparse_fixed_us = kB200RouteCost.row_sparse_fixed_us;
  cost->block_floor_us = kB200RouteCost.block_floor_us;
  cost->block_fixed_us = kB200RouteCost.block_fixed_us;
  cost->block_gbs = kB200RouteCost.block_gbs;
  cost->dense_fixed_us = kB200RouteCost.dense_fixed_us;
  cost->dense_gbs = kB200RouteCost.dense_gbs;
  cost->group_split_fixed_us = kB200RouteCost.group_split_fixed_us;
}

static RouteCost to_route_cost(const gsp_route_cost* c) {
  if (!c) return kB200RouteCost;
  return RouteCost{c->hbm_gbs, c->row_sparse_fixed_us, c->block_floor_us, c->block_fixed_us,
                   c->block_gbs, c->dense_fixed_us, c->dense_gbs, c->group_split_fixed_us};
}

int32_t gsp_choose_route(int32_t batch, int32_t vocab, int32_t hidden_dim, int32_t elem_bytes, int64_t legal_total,
                         int64_t active_tiles, const gsp_route_cost* cost) {
  if (batch < 1 || vocab < 1 || hidden_dim < 1 || elem_bytes < 1 || legal_total < 0 || active_tiles < 0)
    return fail(GSP_ERR_INVALID_ARGUMENT, "gsp_choose_route: sizes and counts must be positive");
  return choose_route_by_cost(batch, vocab, hidden_dim, elem_bytes, legal_total, active_tiles, to_route_cost(cost));
}

int32_t gsp_adaptive_logits(const void* hidden, int64_t hidden_row_stride, const void* weight,
                            int64_t weight_row_stride, const int32_t* bitmask, int64_t bitmask_row_stride,
                            int32_t batch, int32_t vocab, int32_t hidden_dim, int32_t dtype, void* logits,
                            int64_t logits_row_stride, float* top_value, int64_t* top_index,
                            const gsp_route_cost* cost, int32_t* route_out, int32_t* route_host, void* workspace,
                            size_t workspace_bytes_, void* stream) {
  const char* fn = "gsp_adaptive_logits";
  if (route_host) *route_host = -1;
  int32_t st = validate_projection(fn, hidden, hidden_row_stride, weight, weight_row_stride, bitmask,
                                   bitmask_row_stride, batch, vocab, hidden_dim, dtype, logits, logits_row_stride);
  if (st != GSP_OK) return st;
  if (dtype == GSP_DTYPE_F32)
    return fail(GSP_ERR_UNSUPPORTED, "%s: fp32 has one route (row-sparse); call gsp_row_sparse_logits", fn);
  if (!bitmask) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: bitmask is required", fn);
  st = check_workspace(fn, true, workspace, workspace_bytes_, batch, vocab);
  if (st != GSP_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  if (batch == 1) {  // always row-sparse
    if (route_out && (err = cudaMemsetAsync(route_out, 0, sizeof(int32_t), s)) != cudaSuccess)
      return cuda_status(err, fn);
    if (route_host) *route_host = GSP_ROUTE_ROW_SPARSE;
    return route_call(fn, GSP_ROUTE_ROW_SPARSE, hidden, hidden_row_stride, weight, weight_row_stride, bitmask,
                      bitmask_row_stride, batch, vocab, hidden_dim, dtype, logits, logits_row_stride, top_value,
                      top_index, workspace, workspace_bytes_, stream);
  }
  const Workspace w = carve_workspace(workspace, batch, vocab);
  RouteSelectParams sel;
  std::memset(&sel, 0, sizeof(sel));
  sel.mask = reinterpret_cast<const uint32_t*>(bitmask);
  sel.mask_stride = bitmask_row_stride;
  sel.batch = batch;
  sel.vocab = vocab;
  sel.nw = (vocab + 31) / 32;
  sel.ntiles = (vocab + GSP_TILE_ROWS - 1) / GSP_TILE_ROWS;
  sel.hidden_dim = hidden_dim;
  sel.elem_bytes = 2;
  sel.cost = to_route_cost(cost);
  sel.ticket = w.route_ticket;
  sel.active = w.route_active;
  sel.legal = w.route_legal;
  sel.route_out = route_out;

  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if ((err = cudaStreamIsCapturing(s, &cs)) != cudaSuccess) return cuda_status(err, fn);
  if (cs == cudaStreamCaptureStatusInvalidated)
    return fail(GSP_ERR_CUDA, "%s: the stream's capture has been invalidated", fn);

  if (cs == cudaStreamCaptureStatusNone) {
    // eager: selector, 4-byte read-back, chosen route
    sel.route_word = w.route_word;
    if ((err = launch_route_select(sel, s)) != cudaSuccess) return cuda_status(err, fn);
    int32_t route = -1;
    if ((err = cudaMemcpyAsync(&route, w.route_word, sizeof(int32_t), cudaMemcpyDeviceToHost, s)) != cudaSuccess ||
        (err = cudaMemsetAsync(w.route_word, 0, sizeof(int32_t), s)) != cudaSuccess ||
        (err = cudaStreamSynchronize(s)) != cudaSuccess)
      return cuda_status(err, fn);
    if (route < GSP_ROUTE_ROW_SPARSE || route > GSP_ROUTE_DENSE_MASK)
      return fail(GSP_ERR_CUDA, "%s: the route selector returned %d", fn, route);
    if (route_host) *route_host = route;
    return route_call(fn, route, hidden, hidden_row_stride, weight, weight_row_stride, bitmask, bitmask_row_stride,
                      batch, vocab, hidden_dim, dtype, logits, logits_row_stride, top_value, top_index, workspace,
                      workspace_bytes_, stream);
  }

  // capture: selector kernel -> SWITCH node {row-sparse, block-sparse, dense-mask}
  int device = 0;
  if ((err = cudaGetDevice(&device)) != cudaSuccess) return cuda_status(err, fn);
  cudaGraph_t graph = nullptr;
  const cudaGraphNode_t* deps = nullptr;
  size_t ndeps = 0;
  if ((err = cudaStreamGetCaptureInfo(s, &cs, nullptr, &graph, &deps, &ndeps)) != cudaSuccess)
    return cuda_status(err, fn);
  cudaGraphConditionalHandle handle;
  if ((err = cudaGraphConditionalHandleCreate(&handle, graph, 0, cudaGraphCondAssignDefault)) != cudaSuccess)
    return cuda_status(err, fn);
  sel.handle = handle;
  sel.has_handle = 1;
  if ((err = launch_route_select(sel, s)) != cudaSuccess) return cuda_status(err, fn);
  if ((err = cudaStreamGetCaptureInfo(s, &cs, nullptr, &graph, &deps, &ndeps)) != cudaSuccess)
    return cuda_status(err, fn);
  // (the struct's union has no default constructor: zero-filled storage)
  alignas(cudaGraphNodeParams) unsigned char np_storage[sizeof(cudaGraphNodeParams)] = {};
  cudaGraphNodeParams& np = *reinterpret_cast<cudaGraphNodeParams*>(np_storage);
  np.type = cudaGraphNodeTypeConditional;
  np.conditional.handle = handle;
  np.conditional.type = cudaGraphCondTypeSwitch;
  np.conditional.size = 3;
  cudaGraphNode_t node;
  if ((err = cudaGraphAddNode(&node, graph, deps, ndeps, &np)) != cudaSuccess) return cuda_status(err, fn);
  {
    std::lock_guard<std::mutex> lock(g_body_mu);
    cudaStream_t bs = body_stream(device);
    if (!bs) return fail(GSP_ERR_CUDA, "%s: could not create the body-recording stream", fn);
    for (int r = GSP_ROUTE_ROW_SPARSE; r <= GSP_ROUTE_DENSE_MASK; ++r) {
      if ((err = cudaStreamBeginCaptureToGraph(bs, np.conditional.phGraph_out[r], nullptr, nullptr, 0,
                                               cudaStreamCaptureModeRelaxed)) != cudaSuccess)
        return cuda_status(err, fn);
      tl_no_pdl = !kConditionalBodyPdl;
      st = route_call(fn, r, hidden, hidden_row_stride, weight, weight_row_stride, bitmask, bitmask_row_stride,
                      batch, vocab, hidden_dim, dtype, logits, logits_row_stride, top_value, top_index, workspace,
                      workspace_bytes_, bs);
      tl_no_pdl = false;
      cudaGraph_t body = nullptr;
      err = cudaStreamEndCapture(bs, &body);
      if (st != GSP_OK) return st;
      if (err != cudaSuccess) return cuda_status(err, fn);
    }
  }
  if ((err = cudaStreamUpdateCaptureDependencies(s, &node, 1, cudaStreamSetCaptureDependencies)) != cudaSuccess)
    return cuda_status(err, fn);
  return GSP_OK;
}

int32_t gsp_merge_logsumexp(const float* lse, int32_t parts, int32_t batch, float* out, void* stream) {
  const char* fn = "gsp_merge_logsumexp";
  if (parts < 1 || batch < 1) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: parts and batch must be positive", fn);
  if (!lse || !out) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: lse and out are required", fn);
  return cuda_status(launch_merge_logsumexp(lse, parts, batch, out, static_cast<cudaStream_t>(stream)), fn);
}

int32_t gsp_copy_bytes(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return GSP_OK;
  if (!dst || !src) return fail(GSP_ERR_INVALID_ARGUMENT, "gsp_copy_bytes: dst and src are required");
  return cuda_status(launch_copy_bytes(dst, src, bytes, static_cast<cudaStream_t>(stream)), "gsp_copy_bytes");
}

int32_t gsp_row_sparse_step(const void* host_inputs, size_t input_bytes, void* device_inputs, const void* hidden,
                            int64_t hidden_row_stride, const void* weight, int64_t weight_row_stride,
                            const int32_t* bitmask, int64_t bitmask_row_stride, int32_t batch, int32_t vocab,
                            int32_t hidden_dim, int32_t dtype, int64_t vocab_offset, void* logits,
                            int64_t logits_row_stride, float* top_value, int64_t* top_index, int64_t* top_key,
                            void* workspace, size_t workspace_bytes_, void* stream) {
  const char* fn = "gsp_row_sparse_step";
  if (input_bytes > 0 && (!host_inputs || !device_inputs))
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: host_inputs and device_inputs are required", fn);
  // validated before the copy is queued, so a failed call queues nothing
  int32_t st = validate_projection(fn, hidden, hidden_row_stride, weight, weight_row_stride, bitmask,
                                   bitmask_row_stride, batch, vocab, hidden_dim, dtype, logits, logits_row_stride);
  if (st != GSP_OK) return st;
  st = check_workspace(fn, top_value || top_index || top_key, workspace, workspace_bytes_, batch, vocab);
  if (st != GSP_OK) return st;
  if (input_bytes > 0) {
    st = cuda_status(launch_copy_bytes(device_inputs, host_inputs, input_bytes, static_cast<cudaStream_t>(stream)),
                     fn);
    if (st != GSP_OK) return st;
  }
  return projection_common(fn, false, 0, hidden, hidden_row_stride, weight, weight_row_stride, bitmask,
                           bitmask_row_stride, batch, vocab, hidden_dim, dtype, vocab_offset, logits, logits_row_stride,
                           top_value, top_index, top_key, workspace, workspace_bytes_, stream);
}

size_t gsp_group_plan_words(int32_t batch) {
  if (batch < 1) return 0;
  return (size_t)kPlanHeader + 6 * (size_t)batch;
}

int32_t gsp_group_plan(const int32_t* bitmask, int64_t bitmask_row_stride, int32_t batch, int32_t vocab,
                       int32_t hidden_dim, int32_t elem_bytes, int32_t with_logits, const gsp_route_cost* cost,
                       int32_t* plan, void* stream) {
  const char* fn = "gsp_group_plan";
  if (!bitmask || !plan) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: bitmask and plan are required", fn);
  if (batch < 1 || batch > kGroupMaxBatch || vocab < 1 || hidden_dim < 1 || elem_bytes < 1)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: batch must be in [1, %d]; vocab, hidden_dim, elem_bytes positive", fn,
                kGroupMaxBatch);
  const int64_t nw = (vocab + 31) / 32;
  if (batch > 1 && bitmask_row_stride < nw)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: bitmask_row_stride must be >= ceil(vocab/32)", fn);
  GroupPlanParams p;
  std::memset(&p, 0, sizeof(p));
  p.mask = reinterpret_cast<const uint32_t*>(bitmask);
  p.mask_stride = batch > 1 ? bitmask_row_stride : 0;
  p.batch = batch;
  p.vocab = vocab;
  p.nw = (int)nw;
  p.ntiles = (vocab + GSP_TILE_ROWS - 1) / GSP_TILE_ROWS;
  p.hidden_dim = hidden_dim;
  p.elem_bytes = elem_bytes;
  p.with_logits = with_logits ? 1 : 0;
  p.cost = to_route_cost(cost);
  p.plan = plan;
  return cuda_status(launch_group_plan(p, static_cast<cudaStream_t>(stream)), fn);
}

int32_t gsp_gather_rows(const void* src, int64_t src_row_stride_bytes, const int32_t* rows, int32_t n,
                        int64_t row_bytes, void* dst, int64_t dst_row_stride_bytes, void* stream) {
  const char* fn = "gsp_gather_rows";
  if (n < 0 || row_bytes < 0) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: negative size", fn);
  if (n == 0 || row_bytes == 0) return GSP_OK;
  if (!src || !dst || !rows) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: src, rows and dst are required", fn);
  if (dst_row_stride_bytes < row_bytes)
    return fail(GSP_ERR_INVALID_ARGUMENT, "%s: dst_row_stride_bytes < row_bytes", fn);
  return cuda_status(launch_gather_rows(src, src_row_stride_bytes, rows, n, row_bytes, dst, dst_row_stride_bytes,
                                        static_cast<cudaStream_t>(stream)), fn);
}

struct GroupedScratch {
  int32_t* plan;
  void* hidden;
  uint32_t* mask;
  void* logits;
  float* top_value;
  int64_t* top_index;
  size_t total;
};

static GroupedScratch carve_grouped(void* base, int batch, int vocab, int hidden_dim, bool with_logits) {
  char* p = static_cast<char*>(base);
  GroupedScratch g;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t at = off; off += align256(bytes); return p ? p + at : nullptr; };
  g.plan = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * ((size_t)kPlanHeader + 6 * (size_t)batch)));
  g.hidden = take(2 * (size_t)batch * hidden_dim);
  g.mask = reinterpret_cast<uint32_t*>(take(4 * (size_t)batch * ((vocab + 31) / 32)));
  g.logits = with_logits ? take(2 * (size_t)batch * vocab) : nullptr;
  g.top_value = reinterpret_cast<float*>(take(4 * (size_t)batch));
  g.top_index = reinterpret_cast<int64_t*>(take(8 * (size_t)batch));
  g.total = off;
  return g;
}

size_t gsp_grouped_scratch_bytes(int32_t batch, int32_t vocab, int32_t hidden_dim, int32_t with_logits) {
  if (batch < 1 || vocab < 1 || hidden_dim < 1) return 0;
  return carve_grouped(nullptr, batch, vocab, hidden_dim, with_logits != 0).total;
}

int32_t gsp_grouped_logits(const void* hidden, int64_t hidden_row_stride, const void* weight,
                           int64_t weight_row_stride, const int32_t* bitmask, int64_t bitmask_row_stride,
                           int32_t batch, int32_t vocab, int32_t hidden_dim, int32_t dtype, void* logits,
                           int64_t logits_row_stride, float* top_value, int64_t* top_index,
                           const gsp_route_cost* cost, int32_t* plan_header, void* scratch, size_t scratch_bytes,
                           void* workspace, size_t workspace_bytes_, void* stream) {
  const char* fn = "gsp_grouped_logits";
  int32_t st = validate_projection(fn, hidden, hidden_row_stride, weight, weight_row_stride, bitmask,
                                   bitmask_row_stride, batch, vocab, hidden_dim, dtype, logits, logits_row_stride);
  if (st != GSP_OK) return st;
  if (dtype == GSP_DTYPE_F32)
    return fail(GSP_ERR_UNSUPPORTED, "%s: fp32 has one route (row-sparse); call gsp_row_sparse_logits", fn);
  if (!bitmask) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: bitmask is required", fn);
  if (batch > kGroupMaxBatch) return fail(GSP_ERR_INVALID_ARGUMENT, "%s: batch %d > %d", fn, batch, kGroupMaxBatch);
  st = check_workspace(fn, true, workspace, workspace_bytes_, batch, vocab);
  if (st != GSP_OK) return st;
  const GroupedScratch g = carve_grouped(scratch, batch, vocab, hidden_dim, logits != nullptr);
  if (!scratch || (reinterpret_cast<uintptr_t>(scratch) & 255) != 0 || scratch_bytes < g.total)
    return fail(GSP_ERR_WORKSPACE, "%s: scratch must be 256-byte aligned with %zu bytes", fn, g.total);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if ((err = cudaStreamIsCapturing(s, &cs)) != cudaSuccess) return cuda_status(err, fn);
  if (cs != cudaStreamCaptureStatusNone)
    return fail(GSP_ERR_UNSUPPORTED, "%s: reads its plan back, so it cannot be captured in a graph", fn);
  // plan
  const int32_t with_logits = logits != nullptr;
  st = gsp_group_plan(bitmask, bitmask_row_stride, batch, vocab, hidden_dim, 2, with_logits, cost, g.plan, stream);
  if (st != GSP_OK) return st;
  static thread_local int32_t* hdr = nullptr;  // pinned, one per host thread
  if (!hdr && (err = cudaMallocHost(&hdr, 8 * sizeof(int32_t))) != cudaSuccess) {
    hdr = nullptr;
    return cuda_status(err, fn);
  }
  if ((err = cudaMemcpyAsync(hdr, g.plan, 8 * sizeof(int32_t), cudaMemcpyDeviceToHost, s)) != cudaSuccess ||
      (err = cudaStreamSynchronize(s)) != cudaSuccess)
    return cuda_status(err, fn);
  if (plan_header) std::memcpy(plan_header, hdr, 8 * sizeof(int32_t));
  const int k = hdr[0];
  if (k <= 0 || k >= batch)  // one route on the caller's buffers
    return route_call(fn, hdr[3], hidden, hidden_row_stride, weight, weight_row_stride, bitmask, bitmask_row_stride,
                      batch, vocab, hidden_dim, dtype, logits, logits_row_stride, top_value, top_index, workspace,
                      workspace_bytes_, stream);
  // split: rows into group order, two routes, rows back
  const int32_t* order = g.plan + kPlanHeader;
  const int32_t* inverse = order + batch;
  const int64_t nw = (vocab + 31) / 32;
  const int64_t hbytes = 2 * (int64_t)hidden_dim;
  if ((err = launch_gather_rows(hidden, 2 * hidden_row_stride, order, batch, hbytes, g.hidden, hbytes, s)) !=
          cudaSuccess ||
      (err = launch_gather_rows(bitmask, 4 * bitmask_row_stride, order, batch, 4 * nw, g.mask, 4 * nw, s)) !=
          cudaSuccess)
    return cuda_status(err, fn);
  const int lo[2] = {0, k}, hi[2] = {k, batch}, route[2] = {hdr[1], hdr[2]};
  for (int i = 0; i < 2; ++i) {
    const int n = hi[i] - lo[i];
    st = route_call(fn, route[i], static_cast<const char*>(g.hidden) + (size_t)lo[i] * hbytes, hidden_dim, weight,
                    weight_row_stride, reinterpret_cast<const int32_t*>(g.mask + (size_t)lo[i] * nw), nw, n, vocab,
                    hidden_dim, dtype,
                    g.logits ? static_cast<char*>(g.logits) + (size_t)lo[i] * vocab * 2 : nullptr, vocab,
                    g.top_value + lo[i], g.top_index + lo[i], workspace, workspace_bytes_, stream);
    if (st != GSP_OK) return st;
  }
  if (logits &&
      (err = launch_gather_rows(g.logits, 2 * (int64_t)vocab, inverse, batch, 2 * (int64_t)vocab, logits,
                                2 * (batch > 1 ? logits_row_stride : vocab), s)) != cudaSuccess)
    return cuda_status(err, fn);
  if (top_value && (err = launch_gather_rows(g.top_value, 4, inverse, batch, 4, top_value, 4, s)) != cudaSuccess)
    return cuda_status(err, fn);
  if (top_index && (err = launch_gather_rows(g.top_index, 8, inverse, batch, 8, top_index, 8, s)) != cudaSuccess)
    return cuda_status(err, fn);
  return GSP_OK;
}

}  // extern "C"
