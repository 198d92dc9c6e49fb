// Bitmask utilities: token-id list -> bitmask, per-request density statistics,
// the device route selector, and top-1 key decoding.
#include <algorithm>

#include "gsp_common.cuh"
#include "gsp_internal.h"

namespace gsp {
namespace {

// ids -> packed LSB-first bitmask (gsp/runtime.py:35-43: range check, dedup and
// sort are all implied by setting bits). stats[0] counts ids whose bit was
// newly set (distinct ids), stats[1] ids outside [0, vocab).
__global__ void ids_to_bitmask_kernel(const int64_t* __restrict__ ids, int64_t count, int vocab,
                                      uint32_t* __restrict__ mask,
                                      unsigned long long* __restrict__ stats) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  unsigned fresh = 0, bad = 0;
  if (i < count) {
    const int64_t id = ids[i];
    if (id < 0 || id >= vocab) {
      bad = 1;
    } else {
      const uint32_t bit = 1u << (uint32_t)(id & 31);
      const uint32_t old = atomicOr(mask + (id >> 5), bit);
      fresh = (old & bit) ? 0u : 1u;
    }
  }
  const unsigned nf = __reduce_add_sync(FULL_MASK, fresh);
  const unsigned nb = __reduce_add_sync(FULL_MASK, bad);
  if ((threadIdx.x & 31) == 0) {
    if (nf) atomicAdd(stats + 0, (unsigned long long)nf);
    if (nb) atomicAdd(stats + 1, (unsigned long long)nb);
  }
}

constexpr int kStatThreads = 256;
constexpr int kWordsPerThread = 4;

// Per request: legal tokens (popcount, bits >= vocab ignored) and full words
// (word == -1, the signal of gsp/triton_runtime.py:319).
__global__ void request_stats_kernel(const uint32_t* __restrict__ mask, int64_t stride, int vocab,
                                     int nw, int32_t* legal_counts, int32_t* full_words) {
  const int b = blockIdx.y;
  const int w0 = (blockIdx.x * kStatThreads + threadIdx.x) * kWordsPerThread;
  int legal = 0, full = 0;
#pragma unroll
  for (int j = 0; j < kWordsPerThread; ++j) {
    const int w = w0 + j;
    if (w < nw) {
      const uint32_t word = __ldg(mask + (int64_t)b * stride + w);
      legal += __popc(tail_clip(word, w, vocab));
      full += (word == 0xffffffffu);
    }
  }
  legal = __reduce_add_sync(FULL_MASK, legal);
  full = __reduce_add_sync(FULL_MASK, full);
  __shared__ int s_legal[kStatThreads / 32], s_full[kStatThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { s_legal[warp] = legal; s_full[warp] = full; }
  __syncthreads();
  if (threadIdx.x == 0) {
    int a = 0, f = 0;
    for (int i = 0; i < kStatThreads / 32; ++i) { a += s_legal[i]; f += s_full[i]; }
    if (legal_counts && a) atomicAdd(legal_counts + b, a);
    if (full_words && f) atomicAdd(full_words + b, f);
  }
}

// Tiles of 128 rows (4 words) with any legal token in any request.
__global__ void active_tile_count_kernel(const uint32_t* __restrict__ mask, int64_t stride,
                                         int batch, int vocab, int nw, int ntiles,
                                         int32_t* active_tiles) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  int active = 0;
  if (t < ntiles) {
    uint32_t any = 0;
    for (int b = 0; b < batch && !any; ++b) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int w = t * 4 + j;
        if (w < nw) any |= tail_clip(__ldg(mask + (int64_t)b * stride + w), w, vocab);
      }
    }
    active = any != 0;
  }
  active = __reduce_add_sync(FULL_MASK, active);
  if ((threadIdx.x & 31) == 0 && active) atomicAdd(active_tiles, active);
}

constexpr int kRouteTiles = 8;      // 128-row tiles per selector block
constexpr int kRouteThreads = 256;  // 32 request groups x 8 tiles

// Device route selector: each block ORs and counts the mask words of
// kRouteTiles tiles over every request (thread: tile tid % 8, requests
// tid / 8, +32, ...: a warp reads 4 requests x 128 contiguous bytes), adds its
// legal tokens and active tiles to the workspace counters; the last block to
// arrive applies the cost model, publishes the route and returns the counters
// to zero. One block per 8 tiles spreads the mask read over every SM.
__global__ void __launch_bounds__(kRouteThreads) route_select_kernel(const RouteSelectParams p) {
  __shared__ uint32_t s_act[kRouteThreads / 32][kRouteTiles];
  __shared__ unsigned int s_legal[kRouteThreads / 32];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lt = tid % kRouteTiles, grp = tid / kRouteTiles;
  constexpr int kGroups = kRouteThreads / kRouteTiles;
  const int t = blockIdx.x * kRouteTiles + lt;
  uint32_t any = 0u;
  unsigned int legal = 0u;
  if (t < p.ntiles) {
#pragma unroll 2
    for (int b = grp; b < p.batch; b += kGroups) {
      const uint32_t* row = p.mask + (int64_t)b * p.mask_stride;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int w = t * 4 + j;
        if (w < p.nw) {
          const uint32_t x = tail_clip(__ldg(row + w), w, p.vocab);
          any |= x;
          legal += __popc(x);
        }
      }
    }
  }
  // a warp holds 4 request groups of the same 8 tiles: OR them by tile
  any |= __shfl_xor_sync(FULL_MASK, any, 8);
  any |= __shfl_xor_sync(FULL_MASK, any, 16);
  legal = __reduce_add_sync(FULL_MASK, legal);
  if (lane < kRouteTiles) s_act[warp][lane] = any;
  if (lane == 0) s_legal[warp] = legal;
  __syncthreads();
  if (tid == 0) {
    unsigned long long sum = 0;
    for (int i = 0; i < kRouteThreads / 32; ++i) sum += s_legal[i];
    unsigned int act = 0;
    for (int j = 0; j < kRouteTiles; ++j) {
      uint32_t a = 0u;
      for (int i = 0; i < kRouteThreads / 32; ++i) a |= s_act[i][j];
      act += a != 0u;
    }
    if (sum) atomicAdd(p.legal, sum);
    if (act) atomicAdd(p.active, act);
    __threadfence();
    s_last = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last || tid != 0) return;
  __threadfence();
  const unsigned long long legal_total = atomicExch(p.legal, 0ull);
  const unsigned int active = atomicExch(p.active, 0u);
  atomicExch(p.ticket, 0u);
  const int route = choose_route_by_cost(p.batch, p.vocab, p.hidden_dim, p.elem_bytes, (long long)legal_total,
                                         (long long)active, p.cost);
  if (p.has_handle) cudaGraphSetConditional(p.handle, (unsigned int)route);
  if (p.route_out) *p.route_out = route;
  if (p.route_word) *p.route_word = route;
}

// out[b] = log sum_r exp(lse[r][b]), max-shifted; -inf when every part is.
__global__ void merge_logsumexp_kernel(const float* __restrict__ lse, int parts, int batch, float* __restrict__ out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  float m = -INFINITY;
  for (int r = 0; r < parts; ++r) m = fmaxf(m, lse[(size_t)r * batch + b]);
  if (m == -INFINITY) {
    out[b] = -INFINITY;
    return;
  }
  float s = 0.f;
  for (int r = 0; r < parts; ++r) s += expf(lse[(size_t)r * batch + b] - m);
  out[b] = m + logf(s);
}

__global__ void top1_from_keys_kernel(const int64_t* __restrict__ keys, int batch,
                                      float* top_value, int64_t* top_index) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const unsigned long long k = key_from_signed(keys[b]);
  if (top_value) top_value[b] = key_value(k);
  if (top_index) top_index[b] = key_index(k);
}

// SM-driven copy of `bytes` bytes between device-accessible addresses (device
// memory, or pinned host memory under unified addressing): each thread moves
// 16-byte units (bytes past the last whole unit one at a time).
__global__ void copy_bytes_kernel(unsigned char* __restrict__ dst, const unsigned char* __restrict__ src,
                                  size_t bytes, int vec16) {
  // the next kernel (a projection reading these bytes) may launch now; its
  // griddepcontrol.wait still waits for this copy to complete
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t done = 0;
  if (vec16) {
    const size_t units = bytes / 16;
    for (size_t i = tid; i < units; i += stride)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
    done = units * 16;
  }
  for (size_t i = done + tid; i < bytes; i += stride) dst[i] = src[i];
}

}  // namespace

const void* copy_bytes_kernel_fn() { return reinterpret_cast<const void*>(copy_bytes_kernel); }

cudaError_t launch_copy_bytes(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
  if (bytes == 0) return cudaSuccess;
  const int vec16 = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0;
  const size_t units = vec16 ? (bytes + 15) / 16 : bytes;
  const int threads = 256;
  const size_t blocks = std::min<size_t>((units + threads - 1) / threads, 1184);
  copy_bytes_kernel<<<(unsigned)blocks, threads, 0, stream>>>(static_cast<unsigned char*>(dst),
                                                             static_cast<const unsigned char*>(src), bytes, vec16);
  return cudaGetLastError();
}

cudaError_t launch_ids_to_bitmask(const int64_t* ids, int64_t count, int vocab, uint32_t* mask,
                                  unsigned long long* stats, cudaStream_t stream) {
  const int nw = (vocab + 31) / 32;
  cudaError_t err = cudaMemsetAsync(mask, 0, sizeof(uint32_t) * (size_t)nw, stream);
  if (err != cudaSuccess) return err;
  err = cudaMemsetAsync(stats, 0, 2 * sizeof(unsigned long long), stream);
  if (err != cudaSuccess) return err;
  if (count == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks = (count + threads - 1) / threads;
  ids_to_bitmask_kernel<<<(unsigned)blocks, threads, 0, stream>>>(ids, count, vocab, mask, stats);
  return cudaGetLastError();
}

cudaError_t launch_mask_stats(const uint32_t* mask, int64_t stride, int batch, int vocab,
                              int32_t* legal_counts, int32_t* full_words, int32_t* active_tiles,
                              cudaStream_t stream) {
  const int nw = (vocab + 31) / 32;
  cudaError_t err;
  if (legal_counts) {
    err = cudaMemsetAsync(legal_counts, 0, sizeof(int32_t) * batch, stream);
    if (err != cudaSuccess) return err;
  }
  if (full_words) {
    err = cudaMemsetAsync(full_words, 0, sizeof(int32_t) * batch, stream);
    if (err != cudaSuccess) return err;
  }
  if (legal_counts || full_words) {
    dim3 grid((nw + kStatThreads * kWordsPerThread - 1) / (kStatThreads * kWordsPerThread), batch);
    request_stats_kernel<<<grid, kStatThreads, 0, stream>>>(mask, stride, vocab, nw, legal_counts,
                                                            full_words);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
  }
  if (active_tiles) {
    err = cudaMemsetAsync(active_tiles, 0, sizeof(int32_t), stream);
    if (err != cudaSuccess) return err;
    const int ntiles = (vocab + 127) / 128;
    active_tile_count_kernel<<<(ntiles + 255) / 256, 256, 0, stream>>>(mask, stride, batch, vocab,
                                                                       nw, ntiles, active_tiles);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
  }
  return cudaSuccess;
}

cudaError_t launch_route_select(const RouteSelectParams& p, cudaStream_t stream) {
  const int blocks = (p.ntiles + kRouteTiles - 1) / kRouteTiles;
  route_select_kernel<<<blocks, kRouteThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_merge_logsumexp(const float* lse, int parts, int batch, float* out, cudaStream_t stream) {
  merge_logsumexp_kernel<<<(batch + 127) / 128, 128, 0, stream>>>(lse, parts, batch, out);
  return cudaGetLastError();
}

cudaError_t launch_top1_from_keys(const int64_t* keys, int batch, float* top_value,
                                  int64_t* top_index, cudaStream_t stream) {
  top1_from_keys_kernel<<<(batch + 127) / 128, 128, 0, stream>>>(keys, batch, top_value, top_index);
  return cudaGetLastError();
}

}  // namespace gsp
