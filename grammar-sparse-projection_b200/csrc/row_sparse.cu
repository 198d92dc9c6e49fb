// Row-sparse (direct-bitmask) LM-head projection for sm_100a.
//
// Behaviour follows gsp/triton_runtime.py:15-58 (_bitmask_sparse_lm_head_kernel):
// out[b, v] = sum_k W[v, k] * h[b, k] (fp32 accumulate, rounded to the input
// dtype) when token v is legal for request b, else -inf. Only legal rows of W
// are read.
//
// B200 design (one persistent launch, one CTA per SM):
//   1. every CTA scans the packed bitmask (a few tens of KB, L2-resident after
//      the first touch) with per-thread popcounts and one block-wide scan, so it
//      knows the global rank of every legal (request, row) unit without a
//      second launch;
//   2. CTA c takes the units of rank [c*U/G, (c+1)*U/G): the legal rows are
//      split evenly across SMs whatever their layout in the vocabulary
//      (uniform or clustered runs), in rounds of at most kListCap units;
//   3. each warp streams whole rows (H/8 16-byte lanes, up to two rows in flight
//      per warp) with L1-bypassing vector loads, dots them against the hidden
//      state staged in shared memory by cp.async, and reduces with shuffles;
//   4. the CTA writes -inf over the illegal entries of its slice of the output
//      (16-byte stores where eight neighbours are illegal);
//   5. greedy top-1: packed (rounded value, inverted index) keys are reduced in
//      shared memory, merged with one global atomicMax per request, and the
//      last CTA to arrive decodes them and re-zeroes the workspace. No CTA ever
//      waits on another.
#include "gsp_common.cuh"
#include "gsp_internal.h"

namespace gsp {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kListCap = 2048;   // units extracted per round
constexpr int kUnroll = 8;       // 16-byte loads per lane per pass over a row
constexpr size_t kHiddenSmemMax = 64 * 1024;

struct SmemLayout {
  size_t list, keys, warp, misc, hidden, total;
};

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline SmemLayout smem_layout(int batch, int hidden_dim, bool h_in_smem) {
  SmemLayout l;
  l.list = 0;
  l.keys = align_up(l.list + sizeof(uint32_t) * kListCap, 16);
  l.warp = align_up(l.keys + sizeof(unsigned long long) * batch, 16);
  l.misc = align_up(l.warp + sizeof(uint32_t) * 32, 16);
  l.hidden = align_up(l.misc + 16, 128);
  l.total = l.hidden + (h_in_smem ? sizeof(uint16_t) * (size_t)batch * hidden_dim : 0);
  return l;
}

__device__ __forceinline__ void cp_async_16(void* smem, const void* gmem) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}

template <typename T, bool kVec, bool kHiddenInSmem>
__global__ void __launch_bounds__(kThreads, 1) row_sparse_kernel(const RowSparseParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const SmemLayout L = smem_layout(p.batch, p.hidden_dim, kHiddenInSmem);
  uint32_t* s_list = reinterpret_cast<uint32_t*>(smem + L.list);
  unsigned long long* s_keys = reinterpret_cast<unsigned long long*>(smem + L.keys);
  uint32_t* s_warp = reinterpret_cast<uint32_t*>(smem + L.warp);
  int* s_misc = reinterpret_cast<int*>(smem + L.misc);
  uint16_t* s_h = reinterpret_cast<uint16_t*>(smem + L.hidden);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, cta = blockIdx.x;
  const int B = p.batch, V = p.vocab, H = p.hidden_dim, nw = p.nw;
  const bool want_top = (p.top_value != nullptr) | (p.top_index != nullptr) | (p.top_key != nullptr);

  // ---- phase 0: hidden states -> shared memory (asynchronous) -------------
  if (kHiddenInSmem) {
    const int vpr = H / 8;  // kVec guarantees H % 8 == 0 and 16-byte alignment
    const uint16_t* hsrc = static_cast<const uint16_t*>(p.hidden);
    for (int i = tid; i < B * vpr; i += kThreads) {
      int b = i / vpr, j = i - b * vpr;
      cp_async_16(s_h + (size_t)b * H + j * 8, hsrc + (size_t)b * p.hidden_stride + j * 8);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int b = tid; b < B; b += kThreads) s_keys[b] = 0ull;

  // ---- phase 1: popcount scan over the flat (request, word) space ---------
  const int64_t F = p.mask ? (int64_t)B * nw : 0;
  const int S = p.mask ? (int)((F + kThreads - 1) / kThreads) : 0;
  const int64_t f0 = p.mask ? min((int64_t)tid * S, F) : 0;
  const int64_t f1 = p.mask ? min(f0 + S, F) : 0;
  uint32_t cnt = 0;
  if (p.mask && f0 < f1) {
    int b = (int)(f0 / nw), w = (int)(f0 - (int64_t)b * nw);
    const uint32_t* row = p.mask + (int64_t)b * p.mask_stride;
    if ((f1 - 1) / nw == b) {  // segment inside one request: independent loads
      const int n = (int)(f1 - f0);
#pragma unroll 8
      for (int j = 0; j < n; ++j) cnt += __popc(tail_clip(__ldg(row + w + j), w + j, V));
    } else {
      for (int64_t f = f0; f < f1; ++f) {
        cnt += __popc(tail_clip(__ldg(row + w), w, V));
        if (++w == nw) { w = 0; ++b; row = p.mask + (int64_t)b * p.mask_stride; }
      }
    }
  }
  uint32_t incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t t = __shfl_up_sync(FULL_MASK, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t x = lane < kWarps ? s_warp[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t t = __shfl_up_sync(FULL_MASK, x, o);
      if (lane >= o) x += t;
    }
    if (lane < kWarps) s_warp[lane] = x;
  }
  __syncthreads();
  const uint32_t excl = incl - cnt + (warp > 0 ? s_warp[warp - 1] : 0u);
  const uint64_t total = p.mask ? (uint64_t)s_warp[kWarps - 1] : (uint64_t)B * V;

  // Request offsets of the compact layout: written by CTA 0 only.
  if (p.offsets != nullptr && cta == 0) {
    if (p.mask) {
      if (f0 < f1) {
        int b = (int)(f0 / nw), w = (int)(f0 - (int64_t)b * nw);
        uint32_t run = excl;
        for (int64_t f = f0; f < f1; ++f) {
          if (w == 0) p.offsets[b] = run;
          run += __popc(tail_clip(__ldg(p.mask + (int64_t)b * p.mask_stride + w), w, V));
          if (++w == nw) { w = 0; ++b; }
        }
      }
    } else {
      for (int b = tid; b < B; b += kThreads) p.offsets[b] = (int64_t)b * V;
    }
    if (tid == 0) p.offsets[B] = (int64_t)total;
  }

  const uint64_t lo = total * (uint64_t)cta / (uint64_t)G;
  const uint64_t hi = total * (uint64_t)(cta + 1) / (uint64_t)G;
  const uint32_t code_stride = (uint32_t)nw * 32u;  // unit code = b * code_stride + v

  if (kHiddenInSmem) {
    asm volatile("cp.async.wait_all;" ::: "memory");
  }
  __syncthreads();

  for (uint64_t rbase = lo; rbase < hi; rbase += kListCap) {
    const uint64_t rend = min(hi, rbase + (uint64_t)kListCap);
    const int n = (int)(rend - rbase);
    // ---- phase 2: extract the units of rank [rbase, rend) -----------------
    if (p.mask) {
      if ((uint64_t)excl < rend && (uint64_t)excl + cnt > rbase) {
        int b = (int)(f0 / nw), w = (int)(f0 - (int64_t)b * nw);
        uint64_t r = excl;
        for (int64_t f = f0; f < f1 && r < rend; ++f) {
          uint32_t word = tail_clip(__ldg(p.mask + (int64_t)b * p.mask_stride + w), w, V);
          uint32_t pc = __popc(word);
          if (r + pc > rbase) {
            while (word) {
              int bit = __ffs(word) - 1;
              word &= word - 1;
              if (r >= rbase && r < rend)
                s_list[r - rbase] = (uint32_t)b * code_stride + (uint32_t)(w * 32 + bit);
              ++r;
            }
          } else {
            r += pc;
          }
          if (++w == nw) { w = 0; ++b; }
        }
      }
    } else {
      for (int i = tid; i < n; i += kThreads) {
        uint64_t r = rbase + i;
        uint32_t b = (uint32_t)(r / (uint64_t)V), v = (uint32_t)(r - (uint64_t)b * V);
        s_list[i] = b * code_stride + v;
      }
    }
    __syncthreads();

    // ---- phase 3: stream legal rows, up to two per warp in flight -----------
    for (int i = warp; i < n; i += 2 * kWarps) {
      const int j = i + kWarps;
      const bool has2 = j < n;
      const uint32_t ca = s_list[i], cb = has2 ? s_list[j] : ca;
      const int ba = (int)(ca / code_stride), va = (int)(ca - (uint32_t)ba * code_stride);
      const int bb = (int)(cb / code_stride), vb = (int)(cb - (uint32_t)bb * code_stride);
      const uint16_t* wa = static_cast<const uint16_t*>(p.weight) + (int64_t)va * p.weight_stride;
      const uint16_t* wb = static_cast<const uint16_t*>(p.weight) + (int64_t)vb * p.weight_stride;
      float acc_a = 0.f, acc_b = 0.f;
      if (kVec) {
        const int nvec = H / 8;
        const uint16_t* ha;
        const uint16_t* hb;
        if (kHiddenInSmem) {
          ha = s_h + (size_t)ba * H;
          hb = s_h + (size_t)bb * H;
        } else {
          ha = static_cast<const uint16_t*>(p.hidden) + (int64_t)ba * p.hidden_stride;
          hb = static_cast<const uint16_t*>(p.hidden) + (int64_t)bb * p.hidden_stride;
        }
        for (int base = 0; base < nvec; base += 32 * kUnroll) {
          uint4 ra[kUnroll], rb[kUnroll];
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            const int e = base + u * 32 + lane;
            ra[u] = e < nvec ? ld_stream_v4(wa + e * 8) : make_uint4(0, 0, 0, 0);
            rb[u] = (has2 && e < nvec) ? ld_stream_v4(wb + e * 8) : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            const int e = base + u * 32 + lane;
            if (e < nvec) {
              uint4 xa, xb;
              if (kHiddenInSmem) {
                xa = reinterpret_cast<const uint4*>(ha)[e];
                xb = reinterpret_cast<const uint4*>(hb)[e];
              } else {
                xa = __ldg(reinterpret_cast<const uint4*>(ha) + e);
                xb = __ldg(reinterpret_cast<const uint4*>(hb) + e);
              }
              acc_a = dot8<T>(ra[u], xa, acc_a);
              if (has2) acc_b = dot8<T>(rb[u], xb, acc_b);
            }
          }
        }
      } else {
        const uint16_t* ha = static_cast<const uint16_t*>(p.hidden) + (int64_t)ba * p.hidden_stride;
        const uint16_t* hb = static_cast<const uint16_t*>(p.hidden) + (int64_t)bb * p.hidden_stride;
        for (int k = lane; k < H; k += 32) {
          acc_a = fmaf(DTypeTraits<T>::bits_to_float(__ldg(wa + k)),
                       DTypeTraits<T>::bits_to_float(__ldg(ha + k)), acc_a);
          if (has2)
            acc_b = fmaf(DTypeTraits<T>::bits_to_float(__ldg(wb + k)),
                         DTypeTraits<T>::bits_to_float(__ldg(hb + k)), acc_b);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        acc_a += __shfl_xor_sync(FULL_MASK, acc_a, o);
        acc_b += __shfl_xor_sync(FULL_MASK, acc_b, o);
      }
      if (lane < 2 && (lane == 0 || has2)) {
        const int b = lane == 0 ? ba : bb;
        const int v = lane == 0 ? va : vb;
        const float acc = lane == 0 ? acc_a : acc_b;
        const uint64_t rank = rbase + (uint64_t)(lane == 0 ? i : j);
        const uint16_t bits = DTypeTraits<T>::round_bits(acc);
        if (p.logits) static_cast<uint16_t*>(p.logits)[(int64_t)b * p.logits_stride + v] = bits;
        if (p.compact && rank < (uint64_t)p.capacity) {
          static_cast<uint16_t*>(p.compact)[rank] = bits;
          p.compact_ids[rank] = p.vocab_offset + v;
        }
        if (want_top) {
          const unsigned long long key =
              top1_key(DTypeTraits<T>::bits_to_float(bits), (uint64_t)(p.vocab_offset + v));
          atomicMax(&s_keys[b], key);
        }
      }
    }
    __syncthreads();
  }

  // ---- phase 4: -inf over the illegal entries of this CTA's output slice ---
  if (p.logits && p.mask) {
    const int64_t FW = (int64_t)B * nw;
    const int64_t w_lo = FW * cta / G, w_hi = FW * (cta + 1) / G;
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.logits) & 15) == 0) && (p.logits_stride % 8 == 0);
    const uint16_t ninf = DTypeTraits<T>::kNegInfBits;
    for (int64_t g = w_lo * 4 + tid; g < w_hi * 4; g += kThreads) {
      const int64_t f = g >> 2;
      const int q = (int)(g & 3);
      const int b = (int)(f / nw), w = (int)(f - (int64_t)b * nw);
      const uint32_t word = __ldg(p.mask + (int64_t)b * p.mask_stride + w);
      const uint32_t byte = (word >> (q * 8)) & 0xffu;
      const int row0 = w * 32 + q * 8;
      if (row0 >= V || byte == 0xffu) continue;
      uint16_t* dst = static_cast<uint16_t*>(p.logits) + (int64_t)b * p.logits_stride + row0;
      if (byte == 0u && vec_ok && row0 + 8 <= V) {
        const uint32_t x = (uint32_t)ninf | ((uint32_t)ninf << 16);
        *reinterpret_cast<uint4*>(dst) = make_uint4(x, x, x, x);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (!((byte >> e) & 1u) && row0 + e < V) dst[e] = ninf;
      }
    }
  }

  // ---- phase 5: cross-CTA top-1 merge (last CTA decodes) -------------------
  if (want_top) {
    __syncthreads();
    for (int b = tid; b < B; b += kThreads) {
      const unsigned long long k = s_keys[b];
      if (k != 0ull) atomicMax(p.keys + b, k);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const unsigned int t = atomicAdd(p.ticket, 1u);
      s_misc[0] = (t == (unsigned int)(G - 1));
    }
    __syncthreads();
    if (s_misc[0]) {
      __threadfence();
      for (int b = tid; b < B; b += kThreads) {
        const unsigned long long k = atomicExch(p.keys + b, 0ull);
        if (p.top_value) p.top_value[b] = key_value(k);
        if (p.top_index) p.top_index[b] = key_index(k);
        if (p.top_key) p.top_key[b] = key_to_signed(k);
      }
      if (tid == 0) atomicExch(p.ticket, 0u);
    }
  }
}

template <typename T, bool kVec, bool kHiddenInSmem>
cudaError_t launch_variant(const RowSparseParams& p, cudaStream_t stream) {
  const SmemLayout L = smem_layout(p.batch, p.hidden_dim, kHiddenInSmem);
  auto kernel = row_sparse_kernel<T, kVec, kHiddenInSmem>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)L.total);
  if (err != cudaSuccess) return err;
  int dev = 0;
  err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  const int grid = num_sms(dev);
  kernel<<<grid, kThreads, L.total, stream>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_typed(const RowSparseParams& p, cudaStream_t stream) {
  const bool vec = (p.hidden_dim % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.weight) & 15) == 0) && (p.weight_stride % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(p.hidden) & 15) == 0) &&
                   (p.batch == 1 || p.hidden_stride % 8 == 0);
  const bool h_smem = vec && (sizeof(uint16_t) * (size_t)p.batch * p.hidden_dim <= kHiddenSmemMax);
  if (vec && h_smem) return launch_variant<T, true, true>(p, stream);
  if (vec) return launch_variant<T, true, false>(p, stream);
  return launch_variant<T, false, false>(p, stream);
}

}  // namespace

cudaError_t launch_row_sparse(const RowSparseParams& p, int dtype, cudaStream_t stream) {
  if (dtype == 1) return launch_typed<__nv_bfloat16>(p, stream);
  return launch_typed<__half>(p, stream);
}

}  // namespace gsp
