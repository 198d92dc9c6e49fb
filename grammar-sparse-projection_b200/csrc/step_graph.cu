// gsp_step_graph_*: a decode step from pinned host inputs (gsp_row_sparse_step:
// the SM copy of the step's packed mask and hidden state, then the row-sparse
// projection) recorded once as a CUDA graph and replayed with one
// cudaGraphLaunch per step. Each launch may name another pinned source row of
// the same size and alignment: the copy node's source pointer is updated in
// the instantiated graph (cudaGraphExecKernelNodeSetParams) before the launch.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <new>

#include "../../include/gsp_b200.h"
#include "gsp_internal.h"

namespace gsp {
namespace {

struct StepGraph {
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaGraphNode_t copy_node = nullptr;
  unsigned char* dst = nullptr;
  const unsigned char* src = nullptr;
  size_t bytes = 0;
  int vec16 = 0;
  dim3 grid, block;
};

void destroy(StepGraph* g) {
  if (!g) return;
  if (g->exec) cudaGraphExecDestroy(g->exec);
  if (g->graph) cudaGraphDestroy(g->graph);
  delete g;
}

}  // namespace
}  // namespace gsp

using namespace gsp;

extern "C" {

int32_t gsp_step_graph_create(void** handle, const void* host_inputs, size_t input_bytes, void* device_inputs,
                              const void* hidden, int64_t hidden_row_stride, const void* weight,
                              int64_t weight_row_stride, const int32_t* bitmask, int64_t bitmask_row_stride,
                              int32_t batch, int32_t vocab, int32_t hidden_dim, int32_t dtype, int64_t vocab_offset,
                              void* logits, int64_t logits_row_stride, float* top_value, int64_t* top_index,
                              int64_t* top_key, void* workspace, size_t workspace_bytes) {
  const char* fn = "gsp_step_graph_create";
  if (!handle) return record_error(GSP_ERR_INVALID_ARGUMENT, "%s: handle is NULL", fn);
  *handle = nullptr;
  if (input_bytes == 0 || !host_inputs || !device_inputs)
    return record_error(GSP_ERR_INVALID_ARGUMENT, "%s: host_inputs, input_bytes and device_inputs are required", fn);
  StepGraph* g = new (std::nothrow) StepGraph();
  if (!g) return record_error(GSP_ERR_INVALID_ARGUMENT, "%s: out of host memory", fn);
  cudaStream_t s = nullptr;
  cudaError_t err = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (err != cudaSuccess) {
    destroy(g);
    return record_error(GSP_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(err));
  }
  err = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
  int32_t st = GSP_OK;
  if (err == cudaSuccess) {
    st = gsp_row_sparse_step(host_inputs, input_bytes, device_inputs, hidden, hidden_row_stride, weight,
                             weight_row_stride, bitmask, bitmask_row_stride, batch, vocab, hidden_dim, dtype,
                             vocab_offset, logits, logits_row_stride, top_value, top_index, top_key, workspace,
                             workspace_bytes, s);
    const cudaError_t end = cudaStreamEndCapture(s, &g->graph);
    if (err == cudaSuccess) err = end;
  }
  cudaStreamDestroy(s);
  if (st != GSP_OK) {  // the step's own message is in gsp_last_error
    destroy(g);
    return st;
  }
  if (err != cudaSuccess) {
    destroy(g);
    return record_error(GSP_ERR_CUDA, "%s: capture failed: %s", fn, cudaGetErrorString(err));
  }
  // the copy node (the one kernel node running copy_bytes_kernel)
  size_t n = 0;
  cudaGraphGetNodes(g->graph, nullptr, &n);
  cudaGraphNode_t nodes[16];
  if (n > 16) n = 16;
  cudaGraphGetNodes(g->graph, nodes, &n);
  for (size_t i = 0; i < n && !g->copy_node; ++i) {
    cudaGraphNodeType type;
    if (cudaGraphNodeGetType(nodes[i], &type) != cudaSuccess || type != cudaGraphNodeTypeKernel) continue;
    cudaKernelNodeParams kp;
    if (cudaGraphKernelNodeGetParams(nodes[i], &kp) != cudaSuccess) continue;
    if (kp.func != copy_bytes_kernel_fn()) continue;
    g->copy_node = nodes[i];
    g->grid = kp.gridDim;
    g->block = kp.blockDim;
    std::memcpy(&g->dst, kp.kernelParams[0], sizeof(g->dst));
    std::memcpy(&g->src, kp.kernelParams[1], sizeof(g->src));
    std::memcpy(&g->bytes, kp.kernelParams[2], sizeof(g->bytes));
    std::memcpy(&g->vec16, kp.kernelParams[3], sizeof(g->vec16));
  }
  if (!g->copy_node) {
    destroy(g);
    return record_error(GSP_ERR_CUDA, "%s: no copy node in the captured step", fn);
  }
  err = cudaGraphInstantiate(&g->exec, g->graph, 0);
  if (err != cudaSuccess) {
    destroy(g);
    return record_error(GSP_ERR_CUDA, "%s: instantiate: %s", fn, cudaGetErrorString(err));
  }
  *handle = g;
  return GSP_OK;
}

int32_t gsp_step_graph_launch(void* handle, const void* host_inputs, void* stream) {
  const char* fn = "gsp_step_graph_launch";
  StepGraph* g = static_cast<StepGraph*>(handle);
  if (!g) return record_error(GSP_ERR_INVALID_ARGUMENT, "%s: handle is NULL", fn);
  if (host_inputs && host_inputs != g->src) {
    const int vec16 = ((reinterpret_cast<uintptr_t>(g->dst) | reinterpret_cast<uintptr_t>(host_inputs)) & 15) == 0;
    if (vec16 != g->vec16)
      return record_error(GSP_ERR_INVALID_ARGUMENT, "%s: host_inputs must have the recorded row's 16-byte alignment",
                          fn);
    const unsigned char* src = static_cast<const unsigned char*>(host_inputs);
    void* args[4] = {&g->dst, &src, &g->bytes, &g->vec16};
    cudaKernelNodeParams kp;
    std::memset(&kp, 0, sizeof(kp));
    kp.func = const_cast<void*>(copy_bytes_kernel_fn());
    kp.gridDim = g->grid;
    kp.blockDim = g->block;
    kp.sharedMemBytes = 0;
    kp.kernelParams = args;
    const cudaError_t err = cudaGraphExecKernelNodeSetParams(g->exec, g->copy_node, &kp);
    if (err != cudaSuccess) return record_error(GSP_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(err));
    g->src = src;
  }
  const cudaError_t err = cudaGraphLaunch(g->exec, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return record_error(GSP_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(err));
  return GSP_OK;
}

int32_t gsp_step_graph_destroy(void* handle) {
  destroy(static_cast<StepGraph*>(handle));
  return GSP_OK;
}

}  // extern "C"
