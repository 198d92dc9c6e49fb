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
// device address. The first call on each device (and in each CUDA context of
// that device) therefore looks up the array's device address with
// cudaGetSymbolAddress while that device is current and caches it; that first
// call should come before any stream capture. Every call first runs a small
// clearing kernel on the caller's stream (a launch, not an allocation) that
// zeroes the part of the array that must start at zero, and then runs the
// ordinary row-sparse kernel on it. All calls share the one array, so calls
// whose executions overlap on the GPU (different streams, or several host
// threads) race on it and must be serialised by the caller.
//
// Errors: a kernel that gives up a bounded wait records a non-zero error word
// in the array. That word survives later calls (the clearing kernel keeps it)
// until gsp_row_sparse_static_error() reads it; while it is set, every call's
// clearing kernel re-zeroes the whole array except the word, because the
// failed launch may have left counters or flags behind.
#include <cuda.h>

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
static_assert(kStaticScratchBytes % 16 == 0, "the clearing kernel stores 16-byte words");

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Zeroes what a call needs zero: the arrival ticket, the route selector's
// state and this call's top-1 keys. When the error word is set, every other
// byte of the array too (the failed launch may have left any of them behind;
// calls of other sizes carve the array differently). The error word is kept.
__global__ void static_clear_kernel(unsigned char* scratch, int batch) {
  const int* error = reinterpret_cast<const int*>(scratch + 4);
  const bool dirty = *reinterpret_cast<const volatile int*>(error) != 0;
  if (!dirty) {
    if (blockIdx.x != 0) return;
    const size_t n = (kKeysOffset + 8 * (size_t)batch) / 4;
    uint32_t* w = reinterpret_cast<uint32_t*>(scratch);
    for (size_t i = threadIdx.x; i < n; i += blockDim.x)
      if (i != 1) w[i] = 0u;
    return;
  }
  const size_t n16 = kStaticScratchBytes / 16;
  uint4* v = reinterpret_cast<uint4*>(scratch);
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x) {
    if (i == 0) {
      reinterpret_cast<uint32_t*>(scratch)[0] = 0u;  // ticket; [1] is the error word
      reinterpret_cast<uint32_t*>(scratch)[2] = 0u;
      reinterpret_cast<uint32_t*>(scratch)[3] = 0u;
    } else {
      v[i] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// The calling thread's current CUDA context, through the driver entry point
// the runtime hands out (no link-time dependency on the driver library).
CUcontext current_context() {
  using CtxGetCurrent = CUresult (*)(CUcontext*);
  static CtxGetCurrent fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrent>(p);
  }();
  CUcontext c = nullptr;
  if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

constexpr int kMaxDevices = 128;
std::mutex g_setup_mu;
struct ScratchAddress {
  CUcontext ctx;
  void* ptr;
};
ScratchAddress g_scratch[kMaxDevices] = {};

// Device address of g_static_scratch on the current device, looked up once per
// device and context (a device whose context was reset and re-created gets a
// fresh lookup: the old address belonged to the old context).
cudaError_t scratch_on_current_device(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch[dev].ptr == nullptr || ctx == nullptr || g_scratch[dev].ctx != ctx) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (err != cudaSuccess) return err;
    g_scratch[dev].ptr = ptr;
    g_scratch[dev].ctx = current_context();
  }
  *out = g_scratch[dev].ptr;
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
    int dev = 0;
    cudaGetDevice(&dev);
    static_clear_kernel<<<num_sms(dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<unsigned char*>(scratch), batch);
    err = cudaGetLastError();
    if (err != cudaSuccess) {
      return record_error(GSP_ERR_CUDA, "gsp_row_sparse_logits_static: clearing the static scratch failed: %s",
                          cudaGetErrorString(err));
    }
  }
  return gsp_row_sparse_logits(hidden, hidden_row_stride, weight, weight_row_stride, bitmask, bitmask_row_stride,
                               batch, vocab, hidden_dim, dtype, vocab_offset, logits, logits_row_stride, top_value,
                               top_index, top_key, scratch, kStaticScratchBytes, stream);
}

extern "C" int32_t gsp_row_sparse_static_error(int32_t* error, void* stream) {
  using namespace gsp;
  if (error == nullptr) return record_error(GSP_ERR_INVALID_ARGUMENT, "gsp_row_sparse_static_error: error is NULL");
  *error = 0;
  void* scratch = nullptr;
  cudaError_t err = scratch_on_current_device(&scratch);
  if (err != cudaSuccess) {
    return record_error(GSP_ERR_CUDA,
                        "gsp_row_sparse_static_error: cudaGetSymbolAddress of the static scratch failed: %s",
                        cudaGetErrorString(err));
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t word = 0;
  if ((err = cudaMemcpyAsync(&word, static_cast<unsigned char*>(scratch) + 4, sizeof(word), cudaMemcpyDeviceToHost,
                             s)) != cudaSuccess ||
      (err = cudaStreamSynchronize(s)) != cudaSuccess) {
    return record_error(GSP_ERR_CUDA, "gsp_row_sparse_static_error: reading the error word failed: %s",
                        cudaGetErrorString(err));
  }
  if (word != 0) {
    // the whole array back to zero, error word included, for the next call
    if ((err = cudaMemsetAsync(scratch, 0, kStaticScratchBytes, s)) != cudaSuccess) {
      return record_error(GSP_ERR_CUDA, "gsp_row_sparse_static_error: clearing the static scratch failed: %s",
                          cudaGetErrorString(err));
    }
  }
  *error = word;
  return GSP_OK;
}
