// Lane grouping by density class, planned on the device.
//
// The reference leaves this as future work (paper/draft.md:264-270): one
// permissive request activates vocabulary tiles for every constrained request
// batched with it, so a mixed batch can cost as much as a dense one. The plan
// here splits the batch into two groups, each projected on its own cheapest
// route:
//
//  * request_profile_kernel: per request, legal tokens and active 128-row
//    tiles (blocks of 8 tiles; per-request shared-memory sums, one global
//    atomic per request and block). Its last block orders the requests by the
//    fill of their active tiles, legal / (128 x tiles), ascending: scattered
//    lanes (a legal token here and there, one per tile) first, clustered and
//    permissive lanes last; requests without a legal token lead.
//  * group_footprint_kernel: for every tile, the first and last position in
//    that order of a request with a legal token in it; histograms of both give
//    the active tiles of every prefix group (positions < k) and suffix group
//    (positions >= k). Its last block costs every split k with the route cost
//    model against the best single route and writes the plan.
//
// Both kernels read the mask once (L2-resident after the first); the plan is
// a few hundred int32 the host reads back before launching the groups.
#include <algorithm>
#include <climits>
#include <type_traits>

#include "gsp_common.cuh"
#include "gsp_internal.h"

namespace gsp {
namespace {

constexpr int kPlanTiles = 8;
constexpr int kPlanThreads = 256;
constexpr int kPlanGroups = kPlanThreads / kPlanTiles;  // request groups per block

struct PlanView {
  int32_t* hdr;
  int32_t* order;
  int32_t* inverse;
  int32_t* legal;
  int32_t* tiles;
  int32_t* hist_min;
  int32_t* hist_max;
};

__device__ __forceinline__ PlanView plan_view(int32_t* plan, int batch) {
  PlanView v;
  v.hdr = plan;
  v.order = plan + kPlanHeader;
  v.inverse = v.order + batch;
  v.legal = v.inverse + batch;
  v.tiles = v.legal + batch;
  v.hist_min = v.tiles + batch;
  v.hist_max = v.hist_min + batch;
  return v;
}

// OR of tile t's four mask words of request b (bits past the vocabulary cleared).
__device__ __forceinline__ uint32_t tile_bits(const GroupPlanParams& p, int b, int t) {
  const uint32_t* row = p.mask + (int64_t)b * p.mask_stride;
  uint32_t x = 0u;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int w = t * 4 + j;
    if (w < p.nw) x |= tail_clip(__ldg(row + w), w, p.vocab);
  }
  return x;
}

__device__ __forceinline__ int tile_popc(const GroupPlanParams& p, int b, int t) {
  const uint32_t* row = p.mask + (int64_t)b * p.mask_stride;
  int n = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int w = t * 4 + j;
    if (w < p.nw) n += __popc(tail_clip(__ldg(row + w), w, p.vocab));
  }
  return n;
}

__global__ void __launch_bounds__(kPlanThreads) request_profile_kernel(const GroupPlanParams p) {
  __shared__ int s_legal[kGroupMaxBatch];
  __shared__ int s_tiles[kGroupMaxBatch];
  __shared__ int s_last;
  const int tid = threadIdx.x;
  const int lt = tid % kPlanTiles, grp = tid / kPlanTiles;
  const int t = blockIdx.x * kPlanTiles + lt;
  const PlanView v = plan_view(p.plan, p.batch);
  for (int b = tid; b < p.batch; b += kPlanThreads) s_legal[b] = s_tiles[b] = 0;
  __syncthreads();
  if (t < p.ntiles) {
    for (int b = grp; b < p.batch; b += kPlanGroups) {
      const int n = tile_popc(p, b, t);
      if (n) {
        atomicAdd(&s_legal[b], n);
        atomicAdd(&s_tiles[b], 1);
      }
    }
  }
  __syncthreads();
  for (int b = tid; b < p.batch; b += kPlanThreads) {
    if (s_legal[b]) {
      atomicAdd(v.legal + b, s_legal[b]);
      atomicAdd(v.tiles + b, s_tiles[b]);
    }
  }
  // the barrier orders every thread's atomics before thread 0's fence and ticket
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(reinterpret_cast<unsigned int*>(v.hdr + 6), 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // order by fill (legal / (128 tiles)), ascending; ties by request index
  __shared__ double s_fill[kGroupMaxBatch];
  for (int b = tid; b < p.batch; b += kPlanThreads) {
    const int lb = __ldcg(v.legal + b), tb = __ldcg(v.tiles + b);
    s_fill[b] = tb ? (double)lb / (128.0 * tb) : -1.0;
  }
  __syncthreads();
  for (int b = tid; b < p.batch; b += kPlanThreads) {
    const double fb = s_fill[b];
    int rank = 0;
    for (int j = 0; j < p.batch; ++j) rank += (s_fill[j] < fb) || (s_fill[j] == fb && j < b);
    v.order[rank] = b;
    v.inverse[b] = rank;
  }
}

__global__ void __launch_bounds__(kPlanThreads) group_footprint_kernel(const GroupPlanParams p) {
  __shared__ int s_min[kPlanTiles];
  __shared__ int s_max[kPlanTiles];
  __shared__ int s_last;
  const int tid = threadIdx.x;
  const int lt = tid % kPlanTiles, grp = tid / kPlanTiles;
  const int t = blockIdx.x * kPlanTiles + lt;
  const PlanView v = plan_view(p.plan, p.batch);
  if (tid < kPlanTiles) {
    s_min[tid] = INT_MAX;
    s_max[tid] = -1;
  }
  __syncthreads();
  int lo = INT_MAX, hi = -1;
  if (t < p.ntiles) {
    for (int b = grp; b < p.batch; b += kPlanGroups) {
      if (tile_bits(p, b, t)) {
        const int pos = __ldcg(v.inverse + b);
        lo = min(lo, pos);
        hi = max(hi, pos);
      }
    }
  }
  // lanes l, l^8, l^16, l^24 of a warp hold the same tile
  lo = min(lo, __shfl_xor_sync(FULL_MASK, lo, 8));
  lo = min(lo, __shfl_xor_sync(FULL_MASK, lo, 16));
  hi = max(hi, __shfl_xor_sync(FULL_MASK, hi, 8));
  hi = max(hi, __shfl_xor_sync(FULL_MASK, hi, 16));
  if ((tid & 31) < kPlanTiles && hi >= 0) {
    atomicMin(&s_min[lt], lo);
    atomicMax(&s_max[lt], hi);
  }
  __syncthreads();
  if (tid < kPlanTiles && s_max[tid] >= 0) {
    atomicAdd(v.hist_min + s_min[tid], 1);
    atomicAdd(v.hist_max + s_max[tid], 1);
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(reinterpret_cast<unsigned int*>(v.hdr + 7), 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // cost every split k (positions [0, k) | [k, B)): prefix sums in shared
  // memory, one thread per k, then the first k of least cost
  __shared__ long long s_legal_pre[kGroupMaxBatch + 1];
  __shared__ int s_amin_pre[kGroupMaxBatch + 1], s_amax_pre[kGroupMaxBatch + 1];
  __shared__ double s_cost[kGroupMaxBatch];
  __shared__ int s_ra[kGroupMaxBatch], s_rb[kGroupMaxBatch];
  const int B = p.batch;
  for (int i = tid; i < B; i += kPlanThreads) {
    s_legal_pre[i + 1] = __ldcg(v.legal + __ldcg(v.order + i));
    s_amin_pre[i + 1] = __ldcg(v.hist_min + i);
    s_amax_pre[i + 1] = __ldcg(v.hist_max + i);
  }
  __syncthreads();
  if (tid == 0) {
    s_legal_pre[0] = 0;
    s_amin_pre[0] = s_amax_pre[0] = 0;
    for (int i = 1; i <= B; ++i) {
      s_legal_pre[i] += s_legal_pre[i - 1];
      s_amin_pre[i] += s_amin_pre[i - 1];
      s_amax_pre[i] += s_amax_pre[i - 1];
    }
  }
  __syncthreads();
  const long long legal_total = s_legal_pre[B], active_total = s_amax_pre[B];
  const double unpermute = p.with_logits
      ? 2.0 * (double)((long long)B * p.vocab * p.elem_bytes) / (p.cost.hbm_gbs * 1e3) : 0.0;
  for (int k = 1 + tid; k < B; k += kPlanThreads) {
    const long long la = s_legal_pre[k];
    double ta, tb;
    s_ra[k] = best_route_by_cost(k, p.vocab, p.hidden_dim, p.elem_bytes, la, s_amin_pre[k], p.cost, &ta);
    s_rb[k] = best_route_by_cost(B - k, p.vocab, p.hidden_dim, p.elem_bytes, legal_total - la,
                                 active_total - s_amax_pre[k], p.cost, &tb);
    s_cost[k] = ta + tb + p.cost.group_split_fixed_us + unpermute;
  }
  __syncthreads();
  if (tid != 0) return;
  double t_single;
  const int single = best_route_by_cost(B, p.vocab, p.hidden_dim, p.elem_bytes, legal_total, active_total, p.cost,
                                        &t_single);
  double best_t = t_single;
  int best_k = 0, best_a = single, best_b = single;
  for (int k = 1; k < B; ++k) {
    if (s_cost[k] < best_t) {
      best_t = s_cost[k];
      best_k = k;
      best_a = s_ra[k];
      best_b = s_rb[k];
    }
  }
  v.hdr[0] = best_k;
  v.hdr[1] = best_a;
  v.hdr[2] = best_b;
  v.hdr[3] = single;
  v.hdr[4] = (int32_t)fmin(t_single * 1e3, 2.0e9);
  v.hdr[5] = best_k ? (int32_t)fmin(best_t * 1e3, 2.0e9) : -1;
}

// dst row i = src row rows[i]; `vec` bytes per access (16, 8, 4 or 1).
template <int kVec>
__global__ void gather_rows_kernel(const unsigned char* __restrict__ src, int64_t src_stride,
                                   const int32_t* __restrict__ rows, int64_t row_bytes,
                                   unsigned char* __restrict__ dst, int64_t dst_stride) {
  using V = typename std::conditional<kVec == 16, uint4,
            typename std::conditional<kVec == 8, uint2,
            typename std::conditional<kVec == 4, uint32_t, unsigned char>::type>::type>::type;
  const int i = blockIdx.y;
  const int64_t r = rows[i];
  const V* s = reinterpret_cast<const V*>(src + r * src_stride);
  V* d = reinterpret_cast<V*>(dst + (int64_t)i * dst_stride);
  const int64_t n = row_bytes / kVec;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x)
    d[j] = s[j];
}

}  // namespace

cudaError_t launch_group_plan(const GroupPlanParams& p, cudaStream_t stream) {
  const size_t words = kPlanHeader + 6 * (size_t)p.batch;
  cudaError_t err = cudaMemsetAsync(p.plan, 0, words * sizeof(int32_t), stream);
  if (err != cudaSuccess) return err;
  const int blocks = (p.ntiles + kPlanTiles - 1) / kPlanTiles;
  request_profile_kernel<<<blocks, kPlanThreads, 0, stream>>>(p);
  if ((err = cudaGetLastError()) != cudaSuccess) return err;
  group_footprint_kernel<<<blocks, kPlanThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const void* src, int64_t src_stride, const int32_t* rows, int n, int64_t row_bytes,
                               void* dst, int64_t dst_stride, cudaStream_t stream) {
  if (n <= 0 || row_bytes <= 0) return cudaSuccess;
  const uint64_t bits = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) |
                        (uint64_t)src_stride | (uint64_t)dst_stride | (uint64_t)row_bytes;
  const int vec = (bits & 15) == 0 ? 16 : (bits & 7) == 0 ? 8 : (bits & 3) == 0 ? 4 : 1;
  const int64_t units = row_bytes / vec;
  const int threads = 256;
  const int64_t gx = std::min<int64_t>((units + threads - 1) / threads, 64);
  const dim3 grid((unsigned)std::max<int64_t>(gx, 1), (unsigned)n);
  auto s = static_cast<const unsigned char*>(src);
  auto d = static_cast<unsigned char*>(dst);
  switch (vec) {
    case 16: gather_rows_kernel<16><<<grid, threads, 0, stream>>>(s, src_stride, rows, row_bytes, d, dst_stride); break;
    case 8: gather_rows_kernel<8><<<grid, threads, 0, stream>>>(s, src_stride, rows, row_bytes, d, dst_stride); break;
    case 4: gather_rows_kernel<4><<<grid, threads, 0, stream>>>(s, src_stride, rows, row_bytes, d, dst_stride); break;
    default: gather_rows_kernel<1><<<grid, threads, 0, stream>>>(s, src_stride, rows, row_bytes, d, dst_stride);
  }
  return cudaGetLastError();
}

}  // namespace gsp
