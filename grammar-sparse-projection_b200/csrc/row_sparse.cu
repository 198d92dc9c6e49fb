// Row-sparse (direct-bitmask) LM-head projection for sm_100a.
//
// Behaviour follows gsp/triton_runtime.py:15-58 (_bitmask_sparse_lm_head_kernel):
// out[b, v] = sum_k W[v, k] * h[b, k] (fp32 accumulate, rounded to the input
// dtype) when token v is legal for request b, else -inf. Only legal rows of W
// are read.
//
// Two kernels, one persistent CTA per SM each. Units are (request, legal row)
// pairs in request-major, row-ascending order; CTA c owns the units of rank
// [c*U/G, (c+1)*U/G), so legal rows are split evenly across SMs whether they
// are spread uniformly or packed into a few runs.
//
// row_sparse_staged_kernel (fast path: 16-byte aligned operands, mask and
// hidden states fit in shared memory)
//   0. warp 0 decodes the CTA's own slice of the mask and fires
//      cp.async.bulk.prefetch.L2 for up to kPrefetchCap legal rows of it, so
//      the DRAM and address-translation latency of those rows overlaps the
//      scan (under uniform masks they are the rows the CTA ends up owning);
//   1. the CTA copies the whole packed mask (tail bits cleared) and the hidden
//      states into shared memory with coalesced 16-byte loads: one round trip;
//   2. one bank-conflict-free pass (warp-contiguous words, lane-strided)
//      writes every word's warp-local exclusive popcount prefix; a 16-entry
//      scan of the warp totals turns them into global ranks;
//   3. every thread checks its warp's words against the CTA's rank range and
//      emits the units of the overlapping words into a shared list;
//   4. each warp streams two whole rows at a time with L1-bypassing 16-byte
//      loads, dots them against h in shared memory and reduces with shuffles;
//   5. -inf is written over the illegal entries of the CTA's slice of the output;
//   6. greedy top-1 keys (rounded value, inverted index) are kept per warp,
//      merged in shared memory and then with one global atomicMax per request;
//      the last CTA to arrive decodes them and re-zeroes the workspace.
//
// row_sparse_direct_kernel (generic path: any alignment, H % 8 != 0, masks too
// large for shared memory): the same decomposition, reading the mask and the
// hidden states from global memory.
//
// No CTA ever waits on another; there is no spin-wait in either kernel.
#include "gsp_async.cuh"
#include "gsp_common.cuh"
#include "gsp_internal.h"

namespace gsp {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kListCap = 2048;      // units extracted per round
constexpr int kUnroll = 8;          // 16-byte loads per lane per pass over a row
constexpr int kPrefetchCap = 32;    // rows per CTA prefetched into L2 before the scan
constexpr size_t kStagedSmemMax = 200 * 1024;  // mask + prefix + hidden + list

__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------------------------
// shared pieces
// ---------------------------------------------------------------------------
// Running per-warp top-1 candidate: one shared-memory atomic per run of units
// of the same request instead of one per unit.
struct RunningTop {
  unsigned long long key = 0ull;
  int b = -1;
  __device__ __forceinline__ void flush(unsigned long long* s_keys) {
    if (b >= 0 && key != 0ull) atomicMax(&s_keys[b], key);
    key = 0ull;
    b = -1;
  }
  __device__ __forceinline__ void add(int req, unsigned long long k, unsigned long long* s_keys) {
    if (req != b) {
      flush(s_keys);
      b = req;
    }
    key = k > key ? k : key;
  }
};

template <typename T>
__device__ __forceinline__ void emit_unit(const RowSparseParams& p, int b, int v, uint64_t rank, float acc,
                                          bool want_top, RunningTop& top, unsigned long long* s_keys) {
  const uint16_t bits = DTypeTraits<T>::round_bits(acc);
  if (p.logits) static_cast<uint16_t*>(p.logits)[(int64_t)b * p.logits_stride + v] = bits;
  if (p.compact && rank < (uint64_t)p.capacity) {
    static_cast<uint16_t*>(p.compact)[rank] = bits;
    p.compact_ids[rank] = p.vocab_offset + v;
  }
  if (want_top)
    top.add(b, top1_key(DTypeTraits<T>::bits_to_float(bits), (uint64_t)(p.vocab_offset + v)), s_keys);
}

// Cross-CTA top-1 merge: each CTA folds its shared-memory keys into the
// workspace with atomicMax; the CTA that draws the last ticket decodes them and
// re-zeroes keys and ticket for the next call. Nobody waits on anybody.
__device__ __forceinline__ void finalize_top1(const RowSparseParams& p, unsigned long long* s_keys, int* s_flag) {
  const int tid = threadIdx.x;
  __syncthreads();
  bool did = false;
  for (int b = tid; b < p.batch; b += blockDim.x) {
    const unsigned long long k = s_keys[b];
    if (k != 0ull) {
      atomicMax(p.keys + b, k);
      did = true;
    }
  }
  if (did) __threadfence();  // only the threads that published keys need the fence
  __syncthreads();
  if (tid == 0) {
    const unsigned int t = atomicAdd(p.ticket, 1u);
    *s_flag = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (*s_flag) {
    __threadfence();
    for (int b = tid; b < p.batch; b += blockDim.x) {
      const unsigned long long k = atomicExch(p.keys + b, 0ull);
      if (p.top_value) p.top_value[b] = key_value(k);
      if (p.top_index) p.top_index[b] = key_index(k);
      if (p.top_key) p.top_key[b] = key_to_signed(k);
    }
    if (tid == 0) atomicExch(p.ticket, 0u);
  }
}

// -inf over the illegal entries of flat words [w_lo, w_hi). word_of(f, b, w)
// returns the word with bits at or beyond `vocab` already cleared or not; rows
// beyond `vocab` are never written either way.
template <typename T, typename WordFn>
__device__ __forceinline__ void fill_illegal(const RowSparseParams& p, int64_t w_lo, int64_t w_hi, WordFn word_of) {
  const int V = p.vocab, nw = p.nw;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.logits) & 15) == 0) && (p.logits_stride % 8 == 0);
  const uint16_t ninf = DTypeTraits<T>::kNegInfBits;
  for (int64_t g = w_lo * 4 + threadIdx.x; g < w_hi * 4; g += blockDim.x) {
    const int64_t f = g >> 2;
    const int q = (int)(g & 3);
    const int b = (int)(f / nw), w = (int)(f - (int64_t)b * nw);
    const uint32_t byte = (word_of(f, b, w) >> (q * 8)) & 0xffu;
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

// Streams units s_list[0, n) (two rows per warp in flight) and emits them.
template <typename T, bool kHSmem>
__device__ __forceinline__ void stream_rows(const RowSparseParams& p, const uint32_t* s_list, int n, uint64_t rbase,
                                            uint32_t code_stride, const uint16_t* s_h, bool want_top,
                                            unsigned long long* s_keys) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = p.hidden_dim, nvec = H / 8;
  RunningTop top;
  for (int i = warp; i < n; i += 2 * kWarps) {
    const int j = i + kWarps;
    const bool has2 = j < n;
    const uint32_t ca = s_list[i], cb = has2 ? s_list[j] : ca;
    const int ba = (int)(ca / code_stride), va = (int)(ca - (uint32_t)ba * code_stride);
    const int bb = (int)(cb / code_stride), vb = (int)(cb - (uint32_t)bb * code_stride);
    const uint16_t* wa = static_cast<const uint16_t*>(p.weight) + (int64_t)va * p.weight_stride;
    const uint16_t* wb = static_cast<const uint16_t*>(p.weight) + (int64_t)vb * p.weight_stride;
    const uint4* ha = kHSmem ? reinterpret_cast<const uint4*>(s_h + (size_t)ba * H)
                             : reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.hidden) +
                                                              (int64_t)ba * p.hidden_stride);
    const uint4* hb = kHSmem ? reinterpret_cast<const uint4*>(s_h + (size_t)bb * H)
                             : reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.hidden) +
                                                              (int64_t)bb * p.hidden_stride);
    float acc_a = 0.f, acc_b = 0.f;
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
          acc_a = dot8<T>(ra[u], kHSmem ? ha[e] : __ldg(ha + e), acc_a);
          if (has2) acc_b = dot8<T>(rb[u], kHSmem ? hb[e] : __ldg(hb + e), acc_b);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc_a += __shfl_xor_sync(FULL_MASK, acc_a, o);
      acc_b += __shfl_xor_sync(FULL_MASK, acc_b, o);
    }
    if (lane == 0) emit_unit<T>(p, ba, va, rbase + (uint64_t)i, acc_a, want_top, top, s_keys);
    if (lane == 1 && has2) emit_unit<T>(p, bb, vb, rbase + (uint64_t)j, acc_b, want_top, top, s_keys);
  }
  if (lane < 2) top.flush(s_keys);
}

// Scalar fallback of stream_rows (any alignment, any H).
template <typename T>
__device__ __forceinline__ void stream_rows_scalar(const RowSparseParams& p, const uint32_t* s_list, int n,
                                                   uint64_t rbase, uint32_t code_stride, bool want_top,
                                                   unsigned long long* s_keys) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = p.hidden_dim;
  RunningTop top;
  for (int i = warp; i < n; i += kWarps) {
    const uint32_t c = s_list[i];
    const int b = (int)(c / code_stride), v = (int)(c - (uint32_t)b * code_stride);
    const uint16_t* w = static_cast<const uint16_t*>(p.weight) + (int64_t)v * p.weight_stride;
    const uint16_t* h = static_cast<const uint16_t*>(p.hidden) + (int64_t)b * p.hidden_stride;
    float acc = 0.f;
    for (int k = lane; k < H; k += 32)
      acc = fmaf(DTypeTraits<T>::bits_to_float(__ldg(w + k)), DTypeTraits<T>::bits_to_float(__ldg(h + k)), acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(FULL_MASK, acc, o);
    if (lane == 0) emit_unit<T>(p, b, v, rbase + (uint64_t)i, acc, want_top, top, s_keys);
  }
  if (lane == 0) top.flush(s_keys);
}

// ===========================================================================
// staged kernel
// ===========================================================================
struct StagedLayout {
  size_t list, keys, warp, misc, mask, prefix, hidden, total;
};

__host__ __device__ inline StagedLayout staged_layout(int batch, int hidden_dim, int nw, bool has_mask) {
  StagedLayout l;
  const size_t F = has_mask ? (size_t)batch * nw : 0;
  size_t off = 0;
  l.list = off;
  off += 4 * (size_t)kListCap;
  l.keys = align_up(off, 16);
  off = l.keys + 8 * (size_t)batch;
  l.warp = align_up(off, 16);
  off = l.warp + 4 * 32;
  l.misc = align_up(off, 16);
  off = l.misc + 16;
  l.mask = align_up(off, 16);
  off = l.mask + 4 * F;
  l.prefix = align_up(off, 16);
  off = l.prefix + 4 * F;
  l.hidden = align_up(off, 16);
  off = l.hidden + 2 * (size_t)batch * hidden_dim;
  l.total = align_up(off, 128);
  return l;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) row_sparse_staged_kernel(const RowSparseParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const bool has_mask = p.mask != nullptr;
  const StagedLayout L = staged_layout(p.batch, p.hidden_dim, p.nw, has_mask);
  uint32_t* s_list = reinterpret_cast<uint32_t*>(smem + L.list);
  unsigned long long* s_keys = reinterpret_cast<unsigned long long*>(smem + L.keys);
  uint32_t* s_warp = reinterpret_cast<uint32_t*>(smem + L.warp);
  int* s_misc = reinterpret_cast<int*>(smem + L.misc);
  uint32_t* s_mask = reinterpret_cast<uint32_t*>(smem + L.mask);
  uint32_t* s_prefix = reinterpret_cast<uint32_t*>(smem + L.prefix);
  uint16_t* s_h = reinterpret_cast<uint16_t*>(smem + L.hidden);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, cta = blockIdx.x;
  const int B = p.batch, V = p.vocab, H = p.hidden_dim, nw = p.nw;
  const int nvec = H / 8;
  const bool want_top = (p.top_value != nullptr) | (p.top_index != nullptr) | (p.top_key != nullptr);
  const int F = has_mask ? B * nw : 0;  // < 2^27: batch * nw * 32 < 2^32 is checked on the host
  const int w_lo = (int)((int64_t)F * cta / G), w_hi = (int)((int64_t)F * (cta + 1) / G);
  const uint32_t tail_keep = (V & 31) ? ((1u << (V & 31)) - 1u) : 0xffffffffu;

  // ---- 0. L2 prefetch of the legal rows in this CTA's own slice ------------
  if (has_mask && warp == 0) {
    int issued = 0;
    for (int f0 = w_lo; f0 < w_hi && issued < kPrefetchCap; f0 += 32) {
      const int f = f0 + lane;
      uint32_t word = 0;
      int w = 0;
      if (f < w_hi) {
        const int b = f / nw;
        w = f - b * nw;
        word = __ldg(p.mask + (int64_t)b * p.mask_stride + w);
        if (w == nw - 1) word &= tail_keep;
      }
      const uint32_t pc = __popc(word);
      uint32_t before = pc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(FULL_MASK, before, o);
        if (lane >= o) before += t;
      }
      before -= pc;  // exclusive prefix within this group of 32 words
      while (word && issued + (int)before < kPrefetchCap) {
        const int bit = __ffs(word) - 1;
        word &= word - 1;
        bulk_prefetch_l2(static_cast<const uint16_t*>(p.weight) + (int64_t)(w * 32 + bit) * p.weight_stride,
                         (uint32_t)H * 2u);
        ++before;
      }
      issued += (int)__shfl_sync(FULL_MASK, before, 31);
    }
  }

  // ---- 1. mask (tail bits cleared) and hidden states -> shared memory ------
  if (has_mask) {
    const bool vec = ((reinterpret_cast<uintptr_t>(p.mask) & 15) == 0) && (nw % 4 == 0) &&
                     (B == 1 || p.mask_stride % 4 == 0);
    if (vec) {
      const int q = nw / 4;
      for (int i = tid; i < B * q; i += kThreads) {
        const int b = i / q, j = i - b * q;
        uint4 v = __ldg(reinterpret_cast<const uint4*>(p.mask + (int64_t)b * p.mask_stride) + j);
        if (j == q - 1) v.w &= tail_keep;
        reinterpret_cast<uint4*>(s_mask)[i] = v;
      }
    } else {
      for (int i = tid; i < F; i += kThreads) {
        const int b = i / nw, w = i - b * nw;
        const uint32_t v = __ldg(p.mask + (int64_t)b * p.mask_stride + w);
        s_mask[i] = (w == nw - 1) ? (v & tail_keep) : v;
      }
    }
  }
  for (int i = tid; i < B * nvec; i += kThreads) {
    const int b = i / nvec, j = i - b * nvec;
    reinterpret_cast<uint4*>(s_h)[i] = __ldg(
        reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.hidden) + (int64_t)b * p.hidden_stride) + j);
  }
  for (int b = tid; b < B; b += kThreads) s_keys[b] = 0ull;
  __syncthreads();

  // ---- 2. one-pass scan: warp-local exclusive prefixes, then warp bases ----
  const int per_warp = ((F + kWarps * 32 - 1) / (kWarps * 32)) * 32;
  const int wbeg = min(warp * per_warp, F), wend = min(wbeg + per_warp, F);
  {
    uint32_t run = 0;
    for (int f0 = wbeg; f0 < wend; f0 += 32) {
      const int f = f0 + lane;
      const uint32_t pc = f < wend ? __popc(s_mask[f]) : 0u;
      uint32_t incl = pc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(FULL_MASK, incl, o);
        if (lane >= o) incl += t;
      }
      if (f < wend) s_prefix[f] = run + incl - pc;
      run += __shfl_sync(FULL_MASK, incl, 31);
    }
    if (lane == 0) s_warp[warp] = run;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t x = lane < kWarps ? s_warp[lane] : 0u;
    uint32_t incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(FULL_MASK, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane < kWarps) s_warp[lane] = incl - x;        // exclusive base of warp `lane`
    if (lane == kWarps - 1) s_misc[2] = (int)incl;      // total legal units
  }
  __syncthreads();
  const uint32_t my_base = s_warp[warp];
  const uint64_t total = has_mask ? (uint64_t)(uint32_t)s_misc[2] : (uint64_t)B * V;
  if (p.offsets != nullptr && cta == 0) {
    for (int b = tid; b < B; b += kThreads) {
      if (has_mask) {
        const int f = b * nw;
        p.offsets[b] = (int64_t)s_prefix[f] + s_warp[f / per_warp];
      } else {
        p.offsets[b] = (int64_t)b * V;
      }
    }
    if (tid == 0) p.offsets[B] = (int64_t)total;
  }

  const uint64_t lo = total * (uint64_t)cta / (uint64_t)G;
  const uint64_t hi = total * (uint64_t)(cta + 1) / (uint64_t)G;
  const uint32_t code_stride = (uint32_t)nw * 32u;

  for (uint64_t rbase = lo; rbase < hi; rbase += kListCap) {
    const uint64_t rend = min(hi, rbase + (uint64_t)kListCap);
    const int n = (int)(rend - rbase);
    // ---- 3. extraction over the warp's own words --------------------------
    if (has_mask) {
      const uint32_t rb32 = (uint32_t)rbase, re32 = (uint32_t)rend;  // ranks < 2^32
      for (int f = wbeg + lane; f < wend; f += 32) {
        const uint32_t pre = s_prefix[f] + my_base;
        if (pre >= re32) break;  // prefixes grow along the warp's run
        uint32_t word = s_mask[f];
        if (pre + __popc(word) <= rb32) continue;
        const int b = f / nw, w = f - b * nw;
        uint32_t r = pre;
        while (word) {
          const int bit = __ffs(word) - 1;
          word &= word - 1;
          if (r >= rb32 && r < re32) s_list[r - rb32] = (uint32_t)b * code_stride + (uint32_t)(w * 32 + bit);
          ++r;
        }
      }
    } else {
      for (int i = tid; i < n; i += kThreads) {
        const uint64_t r = rbase + i;
        const uint32_t b = (uint32_t)(r / (uint64_t)V), v = (uint32_t)(r - (uint64_t)b * V);
        s_list[i] = b * code_stride + v;
      }
    }
    __syncthreads();
    // ---- 4. stream the rows ------------------------------------------------
    stream_rows<T, true>(p, s_list, n, rbase, code_stride, s_h, want_top, s_keys);
    __syncthreads();
  }

  // ---- 5. -inf over the illegal entries of this CTA's output slice ---------
  if (p.logits && has_mask) fill_illegal<T>(p, w_lo, w_hi, [&](int64_t f, int, int) { return s_mask[f]; });
  // ---- 6. top-1 ------------------------------------------------------------
  if (want_top) finalize_top1(p, s_keys, s_misc);
}

// ===========================================================================
// direct kernel (generic fallback)
// ===========================================================================
struct DirectLayout {
  size_t list, keys, warp, misc, total;
};

__host__ __device__ inline DirectLayout direct_layout(int batch) {
  DirectLayout l;
  l.list = 0;
  l.keys = align_up(l.list + sizeof(uint32_t) * kListCap, 16);
  l.warp = align_up(l.keys + sizeof(unsigned long long) * batch, 16);
  l.misc = align_up(l.warp + sizeof(uint32_t) * 32, 16);
  l.total = align_up(l.misc + 16, 128);
  return l;
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(kThreads, 1) row_sparse_direct_kernel(const RowSparseParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const DirectLayout L = direct_layout(p.batch);
  uint32_t* s_list = reinterpret_cast<uint32_t*>(smem + L.list);
  unsigned long long* s_keys = reinterpret_cast<unsigned long long*>(smem + L.keys);
  uint32_t* s_warp = reinterpret_cast<uint32_t*>(smem + L.warp);
  int* s_misc = reinterpret_cast<int*>(smem + L.misc);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = gridDim.x, cta = blockIdx.x;
  const int B = p.batch, V = p.vocab, nw = p.nw;
  const bool want_top = (p.top_value != nullptr) | (p.top_index != nullptr) | (p.top_key != nullptr);
  for (int b = tid; b < B; b += kThreads) s_keys[b] = 0ull;

  // per-thread contiguous segments of the flat (request, word) space
  const int64_t F = p.mask ? (int64_t)B * nw : 0;
  const int S = p.mask ? (int)((F + kThreads - 1) / kThreads) : 0;
  const int64_t f0 = p.mask ? min((int64_t)tid * S, F) : 0;
  const int64_t f1 = p.mask ? min(f0 + S, F) : 0;
  uint32_t cnt = 0;
  if (p.mask && f0 < f1) {
    int b = (int)(f0 / nw), w = (int)(f0 - (int64_t)b * nw);
    for (int64_t f = f0; f < f1; ++f) {
      cnt += __popc(tail_clip(__ldg(p.mask + (int64_t)b * p.mask_stride + w), w, V));
      if (++w == nw) { w = 0; ++b; }
    }
  }
  uint32_t incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(FULL_MASK, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t x = lane < kWarps ? s_warp[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(FULL_MASK, x, o);
      if (lane >= o) x += t;
    }
    if (lane < kWarps) s_warp[lane] = x;
  }
  __syncthreads();
  const uint32_t excl = incl - cnt + (warp > 0 ? s_warp[warp - 1] : 0u);
  const uint64_t total = p.mask ? (uint64_t)s_warp[kWarps - 1] : (uint64_t)B * V;

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
  const uint32_t code_stride = (uint32_t)nw * 32u;

  for (uint64_t rbase = lo; rbase < hi; rbase += kListCap) {
    const uint64_t rend = min(hi, rbase + (uint64_t)kListCap);
    const int n = (int)(rend - rbase);
    if (p.mask) {
      if ((uint64_t)excl < rend && (uint64_t)excl + cnt > rbase) {
        int b = (int)(f0 / nw), w = (int)(f0 - (int64_t)b * nw);
        uint64_t r = excl;
        for (int64_t f = f0; f < f1 && r < rend; ++f) {
          uint32_t word = tail_clip(__ldg(p.mask + (int64_t)b * p.mask_stride + w), w, V);
          const uint32_t pc = __popc(word);
          if (r + pc > rbase) {
            while (word) {
              const int bit = __ffs(word) - 1;
              word &= word - 1;
              if (r >= rbase && r < rend) s_list[r - rbase] = (uint32_t)b * code_stride + (uint32_t)(w * 32 + bit);
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
        const uint64_t r = rbase + i;
        const uint32_t b = (uint32_t)(r / (uint64_t)V), v = (uint32_t)(r - (uint64_t)b * V);
        s_list[i] = b * code_stride + v;
      }
    }
    __syncthreads();
    if (kVec)
      stream_rows<T, false>(p, s_list, n, rbase, code_stride, nullptr, want_top, s_keys);
    else
      stream_rows_scalar<T>(p, s_list, n, rbase, code_stride, want_top, s_keys);
    __syncthreads();
  }

  if (p.logits && p.mask) {
    const int64_t w_lo = F * cta / G, w_hi = F * (cta + 1) / G;
    fill_illegal<T>(p, w_lo, w_hi, [&](int64_t, int b, int w) {
      return __ldg(p.mask + (int64_t)b * p.mask_stride + w);
    });
  }
  if (want_top) finalize_top1(p, s_keys, s_misc);
}

// ===========================================================================
// launch
// ===========================================================================
template <typename T>
cudaError_t launch_typed(const RowSparseParams& p, cudaStream_t stream) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  const int grid = num_sms(dev);
  const bool vec = (p.hidden_dim % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.weight) & 15) == 0) &&
                   (p.weight_stride % 8 == 0) && ((reinterpret_cast<uintptr_t>(p.hidden) & 15) == 0) &&
                   (p.batch == 1 || p.hidden_stride % 8 == 0);
  if (vec) {
    const StagedLayout L = staged_layout(p.batch, p.hidden_dim, p.nw, p.mask != nullptr);
    if (L.total <= kStagedSmemMax) {
      auto k = row_sparse_staged_kernel<T>;
      if ((err = raise_smem_limit(reinterpret_cast<const void*>(k), L.total, dev)) != cudaSuccess) return err;
      k<<<grid, kThreads, L.total, stream>>>(p);
      return cudaGetLastError();
    }
  }
  const DirectLayout L = direct_layout(p.batch);
  if (vec) {
    auto k = row_sparse_direct_kernel<T, true>;
    if ((err = raise_smem_limit(reinterpret_cast<const void*>(k), L.total, dev)) != cudaSuccess) return err;
    k<<<grid, kThreads, L.total, stream>>>(p);
  } else {
    auto k = row_sparse_direct_kernel<T, false>;
    if ((err = raise_smem_limit(reinterpret_cast<const void*>(k), L.total, dev)) != cudaSuccess) return err;
    k<<<grid, kThreads, L.total, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_row_sparse(const RowSparseParams& p, int dtype, cudaStream_t stream) {
  if (dtype == 1) return launch_typed<__nv_bfloat16>(p, stream);
  return launch_typed<__half>(p, stream);
}

}  // namespace gsp
