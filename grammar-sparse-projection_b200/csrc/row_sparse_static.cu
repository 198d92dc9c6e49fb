// gsp_row_sparse_logits_static: the row-sparse projection for callers that
// cannot allocate device memory.
//
// Some callers cannot call cudaMalloc or any allocator: a plugin inside a
// serving engine that owns every byte of device memory through its own pool,
// an FFI binding that is handed only the input and output buffers, or a
// runtime that forbids allocation on its decode path. gsp_row_sparse_logits
// needs a caller-provided workspace for its cross-CTA top-1 merge and, for
// large batches, its cross-CTA unit exchange; this
// variant instead uses the file-scope device array below, which the library
// carries for every GPU that loads it until the process exits.
//
// The array's name, used in host code, is only a host-side stand-in, not a
// device address. The first call on each device therefore looks up the
// array's device address with cudaGetSymbolAddress while that device is
// current and caches it; that first call should come before any stream
// capture. Every call clears the part of the array that must start at zero
// (cudaMemsetAsync on the caller's stream, not an allocation) and then runs
// the ordinary row-sparse kernel on it. All calls share the one array, so
// calls whose executions overlap on the GPU (different streams, or several
// host threads) race on it and must be serialised by the caller.
#include <mutex>

#include "../../include/gsp_b200.h"
#include "gsp_internal.h"

namespace gsp {
namespace {

// Scratch for batch <= GSP_STATIC_MAX_BATCH and vocab <= GSP_STATIC_MAX_VOCAB:
// the same layout as the caller-provided workspace (ticket, error word, one
// 64-bit top-1 key per request, tile lists, and the multi-request kernel's
// slice counts, flags and 1M-entry unit list; not the sampler's part), sized
// for those maxima (4,304,384 bytes).
constexpr size_t kStaticScratchBytes = row_sparse_workspace_bytes_for(GSP_STATIC_MAX_BATCH, GSP_STATIC_MAX_VOCAB);

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 128;
std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_static_scratch on the current device (looked up once).
cudaError_t scratch_on_current_device(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (err != cudaSuccess) return err;
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace gsp

extern "C" int32_t gsp_row_sparse_logits_static(const void* hidden, int64_t hidden_row_stride,
                                                const void* weight, int64_t weight_row_stride,
                                                const int32_t* bitmask, int64_t bitmask_row_stride,
                                                int32_t batch, int32_t vocab, int32_t hidden_dim,
                                                int32_t dtype, int64_t vocab_offset, void* logits,
                                                int64_t logits_row_stride, float* top_value,
                                                int64_t* top_index, int64_t* top_key, void* stream) {
  using namespace gsp;
  if (batch > GSP_STATIC_MAX_BATCH || vocab > GSP_STATIC_MAX_VOCAB) {
    return record_error(GSP_ERR_INVALID_ARGUMENT,
                        "gsp_row_sparse_logits_static: batch %d / vocab %d exceed the static scratch limits "
                        "(batch <= %d, vocab <= %d); use gsp_row_sparse_logits with a workspace",
                        batch, vocab, GSP_STATIC_MAX_BATCH, GSP_STATIC_MAX_VOCAB);
  }
  void* scratch = nullptr;
  cudaError_t err = scratch_on_current_device(&scratch);
  if (err != cudaSuccess) {
    return record_error(GSP_ERR_CUDA,
                        "gsp_row_sparse_logits_static: cudaGetSymbolAddress of the static scratch failed: %s",
                        cudaGetErrorString(err));
  }
  if (batch >= 1) {
    // ticket, error word and this call's keys must start at zero
    err = cudaMemsetAsync(scratch, 0, kKeysOffset + 8 * (size_t)batch, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) {
      return record_error(GSP_ERR_CUDA, "gsp_row_sparse_logits_static: clearing the static scratch failed: %s",
                          cudaGetErrorString(err));
    }
  }
  return gsp_row_sparse_logits(hidden, hidden_row_stride, weight, weight_row_stride, bitmask, bitmask_row_stride,
                               batch, vocab, hidden_dim, dtype, vocab_offset, logits, logits_row_stride, top_value,
                               top_index, top_key, scratch, kStaticScratchBytes, stream);
}
