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
// row_sparse_staged_kernel (fast path: 16-byte aligned operands, at most
// 16,384 mask words, i.e. B * ceil(V/32) <= 16384)
//   1. every thread loads 16 or 32 consecutive words of the flat (request,
//      word) mask into registers with 16-byte loads (one round trip), and the
//      hidden states go to shared memory;
//   2. (no prefetch: prefetching the CTA's own legal rows into L2 before the
//      scan was measured slower than not doing it);
//   3. the words and their rank prefixes (relative to the thread's warp) are
//      staged in shared memory with 16-byte stores before the first barrier;
//      one scan of the 16 warp totals gives the warps' bases;
//   4. -inf is written over the illegal entries of the CTA's slice of the
//      output;
//   5. greedy: each warp takes pairs of the CTA's units, whose codes its two
//      half-warps resolve by ballots over the staged prefixes (warp, thread,
//      word, bit), the next pair's while the current rows load; sampler: the
//      two threads holding the CTA's first and last rank publish themselves
//      and every thread lists the units of one word of theirs;
//   6. each warp streams two whole rows at a time with L1-bypassing 16-byte
//      loads, dots them against h in shared memory and reduces with shuffles;
//   7. greedy top-1 keys (rounded value, inverted index) are kept per warp and
//      merged in shared memory; small batches then use the polled merge
//      (self-tagged per-CTA slots read by the last CTA), others one global
//      atomicMax per request and an arrival ticket whose last holder decodes.
//
// row_sparse_direct_kernel (generic path: any alignment, H % 8 != 0, masks too
// large for shared memory): the same decomposition, reading the mask and the
// hidden states from global memory.
//
// row_sparse_coop_kernel (masks of more than 16,384 words, workspace given):
// launched cooperatively; each CTA scans only its own slice of the mask,
// publishes its popcount and waits (bounded; on time-out it sets the
// workspace error word and skips its units) for the other CTAs' counts.
//
// In the staged and direct kernels no CTA ever waits on another.
#include "gsp_async.cuh"
#include "gsp_common.cuh"
#include "gsp_internal.h"
#include "gsp_peer.cuh"
#include "gsp_sampler.cuh"

namespace gsp {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kListCap = 2048;      // units extracted per round
constexpr int kUnroll = 8;          // 16-byte loads per lane per pass over a row
constexpr size_t kStagedSmemMax = 200 * 1024;  // list + keys + mask slice + hidden states
// Masks of more flat (request, word) entries than this take the cooperative
// kernel when a workspace is given.
// (batch 2 at V=248,320, 15,520 words, measured 14.2 us on the staged kernel
// against 16.1 us on the cooperative one.)
constexpr int64_t kCoopMinWords = 16384;
// Logits bytes per CTA above which the cooperative kernel writes its -inf
// fill during the count wait rather than after publishing its units.
constexpr int64_t kEarlyFillBytes = 64 * 1024;

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

// Shared-memory state of the fused sampler (kSample kernels): per request the
// running Gumbel-max key, the (max, sum) pair of the scaled logits, and the
// generator key. The three arrays follow the top-1 keys in the CTA's keys
// region ([4 * batch] 64-bit words).
struct SampleSmem {
  unsigned long long* keys;   // [B] running Gumbel-max keys
  unsigned long long* stats;  // [B] the CTA's (max, sum) pairs so far
  const uint64_t* seeds;      // [B]
  float* noise;               // [kListCap] Gumbel noise of the round's units
  float* y;                   // [kListCap] scaled logits of the round's units
  unsigned int* rmax;         // [B] the round's max per request (ordered bits)
  float* rsum;                // [B] the round's sum of exp(y - rmax) per request
};

__device__ __forceinline__ SampleSmem sample_smem(unsigned long long* s_keys, int batch) {
  float* noise = reinterpret_cast<float*>(s_keys + 4 * batch);
  unsigned int* rmax = reinterpret_cast<unsigned int*>(noise + 2 * kListCap);
  return SampleSmem{s_keys + batch, s_keys + 2 * batch, reinterpret_cast<const uint64_t*>(s_keys + 3 * batch),
                    noise, noise + kListCap, rmax, reinterpret_cast<float*>(rmax + batch)};
}

// Bytes of a kernel's keys region: top-1 keys and the sampler's arrays.
__host__ __device__ inline size_t keys_region_bytes(int batch) { return 40 * (size_t)batch + 8 * (size_t)kListCap; }

// Initialises the CTA's sampler state (call before the first __syncthreads).
__device__ __forceinline__ void sample_smem_init(const RowSparseParams& p, unsigned long long* s_keys) {
  const SampleSmem ss = sample_smem(s_keys, p.batch);
  for (int b = threadIdx.x; b < p.batch; b += blockDim.x) {
    ss.keys[b] = 0ull;
    ss.stats[b] = empty_stats();
    s_keys[3 * p.batch + b] = p.seeds[b];
    ss.rmax[b] = 0u;
    ss.rsum[b] = 0.f;
  }
}

// Running per-lane sampler state of one request run.
struct RunningSample {
  RunningTop key;
};

// After a round's units are streamed (their scaled logits in ss.y): the
// round's (max, sum) per request with native shared-memory atomics (a 32-bit
// max of ordered bits, then float adds of exp(y - max)), folded into the
// CTA's running pair by one thread per request. Contains three __syncthreads
// and must be reached by the whole CTA.
template <bool kSample>
__device__ __forceinline__ void round_stats(const SampleSmem& ss, const uint32_t* s_list, int n,
                                            uint32_t code_stride) {
  if constexpr (kSample) {
    // Units are sorted by request, so a warp's 32 consecutive units hold a few
    // contiguous runs of one request each: reduce each run in the warp, then
    // one atomic per run (all units of a CTA usually share one or two
    // requests, and same-address shared atomics serialise).
    const int lane = threadIdx.x & 31;
    __syncthreads();
    for (int base = (int)(threadIdx.x & ~31u); base < n; base += blockDim.x) {
      const int i = base + lane;
      const bool valid = i < n;
      const int b = valid ? (int)(s_list[i] / code_stride) : -1 - lane;  // invalid lanes: runs of their own
      const unsigned run = __match_any_sync(FULL_MASK, b);
      const unsigned mx = __reduce_max_sync(run, valid ? ordered_bits(ss.y[i]) : 0u);
      if (valid && lane == __ffs(run) - 1) atomicMax(&ss.rmax[b], mx);
    }
    __syncthreads();
    for (int base = (int)(threadIdx.x & ~31u); base < n; base += blockDim.x) {
      const int i = base + lane;
      const bool valid = i < n;
      const int b = valid ? (int)(s_list[i] / code_stride) : -1 - lane;
      float e = valid ? __expf(ss.y[i] - from_ordered_bits(ss.rmax[b])) : 0.f;
      // suffix sums within each contiguous run; its first lane ends with the run's sum
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float e2 = __shfl_down_sync(FULL_MASK, e, o);
        const int b2 = __shfl_down_sync(FULL_MASK, b, o);
        if (lane + o < 32 && b2 == b) e += e2;
      }
      const int bp = __shfl_up_sync(FULL_MASK, b, 1);
      if (valid && (lane == 0 || bp != b)) atomicAdd(&ss.rsum[b], e);
    }
    __syncthreads();
    const int b0 = (int)(s_list[0] / code_stride), b1 = (int)(s_list[n - 1] / code_stride);
    for (int b = b0 + (int)threadIdx.x; b <= b1; b += blockDim.x) {
      if (ss.rsum[b] > 0.f) {
        float m = stats_m(ss.stats[b]), sum = stats_s(ss.stats[b]);
        merge_stats(m, sum, from_ordered_bits(ss.rmax[b]), ss.rsum[b]);
        ss.stats[b] = pack_stats(m, sum);
      }
      ss.rmax[b] = 0u;
      ss.rsum[b] = 0.f;
    }
  }
}

// ui: the unit's index in the round (its slot in the sampler's per-unit arrays).
template <typename T, bool kSample>
__device__ __forceinline__ void emit_unit(const RowSparseParams& p, int b, int v, uint64_t rank, float acc,
                                          bool want_top, RunningTop& top, unsigned long long* s_keys,
                                          RunningSample& rs, int ui) {
  using Bits = typename DTypeTraits<T>::Bits;
  const Bits bits = DTypeTraits<T>::round_bits(acc);
  if (p.logits) static_cast<Bits*>(p.logits)[(int64_t)b * p.logits_stride + v] = bits;
  if (p.compact && rank < (uint64_t)p.capacity) {
    static_cast<Bits*>(p.compact)[rank] = bits;
    p.compact_ids[rank] = p.vocab_offset + v;
  }
  if (want_top)
    top.add(b, top1_key(DTypeTraits<T>::bits_to_float(bits), (uint64_t)(p.vocab_offset + v)), s_keys);
  if constexpr (kSample) {
    // the sampler's arrays are derived here, not held across the row loop
    const SampleSmem ss = sample_smem(s_keys, p.batch);
    const float y = DTypeTraits<T>::bits_to_float(bits) * p.inv_temp;
    ss.y[ui] = y;
    rs.key.add(b, top1_key(y + ss.noise[ui], (uint64_t)(p.vocab_offset + v)), ss.keys);
  }
}

// Gumbel noise of the round's units s_list[0, n), one unit per thread, into
// ss.noise (kSample kernels; between the two __syncthreads that bracket the
// round's list and its streaming).
template <bool kSample>
__device__ __forceinline__ void round_noise(const RowSparseParams& p, const SampleSmem& ss, const uint32_t* s_list,
                                            int n, uint32_t code_stride) {
  if constexpr (kSample) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t c = s_list[i];
      const int b = (int)(c / code_stride), v = (int)(c - (uint32_t)b * code_stride);
      ss.noise[i] = gumbel_noise(ss.seeds[b], p.offset, (uint64_t)(p.vocab_offset + v));
    }
    __syncthreads();
  }
}

// Every CTA: publishes its sampler state (sample keys by atomicMax, its (max,
// sum) partials into its own row of the workspace). Followed by the ticket.
__device__ __forceinline__ bool sample_publish(const RowSparseParams& p, const SampleSmem& ss) {
  bool did = false;
  for (int b = threadIdx.x; b < p.batch; b += blockDim.x) {
    const unsigned long long k = ss.keys[b];
    if (k != 0ull) atomicMax(p.sample_keys + b, k);
    p.stat_partials[(size_t)b * kMaxSlices + blockIdx.x] = ss.stats[b];  // request-major
    did = true;
  }
  return did;
}

// Last CTA: sampled ids and log-sum-exp per request; re-zeroes the sampler's
// workspace (sampler_finish in gsp_sampler.cuh).
__device__ __forceinline__ void sample_finish(const RowSparseParams& p) {
  sampler_finish(p.sample_keys, p.stat_partials, p.batch, (int)gridDim.x, p.sample_index, p.sample_key, p.sample_lse);
}

// Last CTA: takes the merged keys out of the workspace (re-zeroing it), merges
// them across the ranks of a vocabulary-parallel group when one is given, and
// writes the decoded top-1. All threads of the CTA call it.
__device__ __forceinline__ void decode_top1(const RowSparseParams& p, unsigned long long* s_keys, uint32_t* s_word) {
  const int tid = threadIdx.x;
  bool ok = true;
  if (p.peers.world > 1) {
    for (int b = tid; b < p.batch; b += blockDim.x) s_keys[b] = atomicExch(p.keys + b, 0ull);
    ok = peer_exchange_keys(p.peers, s_keys, p.batch, s_word, p.error);
  }
  for (int b = tid; b < p.batch; b += blockDim.x) {
    const unsigned long long k = p.peers.world > 1 ? s_keys[b] : atomicExch(p.keys + b, 0ull);
    store_top1(p.top_value, p.top_index, p.top_key, b, k, ok);
  }
}

// Cross-CTA top-1 merge: each CTA folds its shared-memory keys into the
// workspace with atomicMax; the CTA that draws the last ticket decodes them and
// re-zeroes keys and ticket for the next call. Nobody waits on anybody.
template <bool kSample>
__device__ __forceinline__ void finalize_top1(const RowSparseParams& p, unsigned long long* s_keys, int* s_flag,
                                              bool want_top) {
  const int tid = threadIdx.x;
  __syncthreads();
  bool did = false;
  if (want_top) {
    for (int b = tid; b < p.batch; b += blockDim.x) {
      const unsigned long long k = s_keys[b];
      if (k != 0ull) {
        atomicMax(p.keys + b, k);
        did = true;
      }
    }
  }
  if constexpr (kSample) did |= sample_publish(p, sample_smem(s_keys, p.batch));
  if (did) __threadfence();  // only the threads that published keys need the fence
  __syncthreads();
  if (tid == 0) {
    const unsigned int t = atomicAdd(p.ticket, 1u);
    *s_flag = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (*s_flag) {
    __threadfence();
    if (want_top) decode_top1(p, s_keys, reinterpret_cast<uint32_t*>(s_flag + 1));
    if constexpr (kSample) sample_finish(p);
    if (tid == 0) atomicExch(p.ticket, 0u);
  }
}

// ---------------------------------------------------------------------------
// Polled cross-CTA top-1 merge (greedy kernels, small batches).
//
// The ticket merge above costs three dependent L2 round trips on the last
// CTA's path (atomicMax + fence, ticket, key read). Here every CTA but the
// decoder (the last block index) stores its per-request keys as self-tagged
// 8-byte words into its own slots, [batch][grid] in the workspace's unit-list
// region, and leaves: no fence, no ticket. Bits 24..31 of a key are always set
// while every global token id is below 2^24 - 1 (the low word is
// 0xffffffff - id), so they carry a fixed non-zero tag; the empty key travels
// as the tag alone. The decoder, after its own rows, polls the slots until
// each carries the tag, folds them into its shared-memory keys, re-zeroes
// them and writes the top-1. Only the decoder waits, and only on CTAs that
// never wait, so the merge needs no co-residency guarantee; the wait is still
// bounded (error word 4 and no token reported when it runs out, after which
// the caller re-zeroes the workspace).
// ---------------------------------------------------------------------------
constexpr int kPolledMaxBatch = 8;
constexpr uint32_t kSlotTag = 0x5Au;
constexpr int64_t kSlotWaitNs = 200000000;  // 0.2 s
constexpr uint32_t kSlotPollLimit = 1u << 22;

__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Whether this launch merges its top-1 keys by polled slots (uniform across
// the grid; the host's workspace carve gives unit_list/list_cap).
__device__ __forceinline__ bool polled_merge_ok(const RowSparseParams& p) {
  return p.unit_list != nullptr && p.batch <= kPolledMaxBatch &&
         (uint64_t)p.vocab_offset + (uint64_t)p.vocab < (1ull << 24) - 1 &&
         8ull * gridDim.x * (uint64_t)p.batch <= 4ull * (uint64_t)p.list_cap;
}

// All threads of every CTA call it after their units; s_keys[0, batch) holds
// the CTA's keys. s_word: one word of shared memory.
__device__ __forceinline__ void finalize_top1_polled(const RowSparseParams& p, unsigned long long* s_keys,
                                                     uint32_t* s_word) {
  const int tid = threadIdx.x, G = gridDim.x, B = p.batch;
  unsigned long long* slots = reinterpret_cast<unsigned long long*>(p.unit_list);
  __syncthreads();  // every warp's running key is in s_keys
  if ((int)blockIdx.x != G - 1) {
    for (int b = tid; b < B; b += blockDim.x) st_relaxed_gpu_u64(slots + (size_t)b * G + blockIdx.x, tag_key(s_keys[b], kSlotTag));
    // This CTA is done: a programmatic dependent of this kernel may be
    // scheduled once every CTA has got here (or exited). Its
    // griddepcontrol.wait still waits for this whole grid and its memory.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    return;
  }
  // the decoder's rows are done too; every other CTA it waits for has run
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  bool late = false;
  const uint64_t t0 = globaltimer_ns();
  for (int i = tid; i < B * (G - 1); i += blockDim.x) {
    const int b = i / (G - 1), c = i - b * (G - 1);
    unsigned long long* s = slots + (size_t)b * G + c;
    bool ok = false;
    unsigned long long w = 0ull;
    for (uint32_t it = 0; it < kSlotPollLimit; ++it) {
      w = ld_relaxed_gpu_u64(s);
      if (tag_is(w, kSlotTag)) {
        ok = true;
        break;
      }
      // the timer is read on every 32nd poll only: a read between two polls
      // delays the next one
      if ((it & 31u) == 31u && (int64_t)(globaltimer_ns() - t0) > kSlotWaitNs) break;
    }
    if (ok) {
      const unsigned long long k = untag_key(w);
      if (k != 0ull) atomicMax(&s_keys[b], k);
      *s = 0ull;
    } else {
      late = true;
    }
  }
  const bool failed = __syncthreads_or(late);
  if (failed && tid == 0 && p.error) atomicExch(p.error, 4);
  bool ok = !failed;
  if (p.peers.world > 1) ok = peer_exchange_keys(p.peers, s_keys, B, s_word, p.error) && ok;
  for (int b = tid; b < B; b += blockDim.x) store_top1(p.top_value, p.top_index, p.top_key, b, s_keys[b], ok);
}

// -inf over the illegal entries of flat words [w_lo, w_hi). word_of(f, b, w)
// returns the word with bits at or beyond `vocab` already cleared or not; rows
// beyond `vocab` are never written either way.
// Threads [t0, t0 + nt) of the CTA take part (default: all of them).
// I: the index type of the loop (32-bit whenever the byte count allows).
template <typename T, typename I, typename WordFn>
__device__ __forceinline__ void fill_illegal_range(const RowSparseParams& p, I w_lo, I w_hi, WordFn word_of, int me,
                                                   int nt) {
  const int V = p.vocab, nw = p.nw;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.logits) & 15) == 0) && (p.logits_stride % 8 == 0);
  using Bits = typename DTypeTraits<T>::Bits;
  const Bits ninf = DTypeTraits<T>::kNegInfBits;
  for (I g = w_lo * 4 + me; g < w_hi * 4; g += nt) {
    const I f = g >> 2;
    const int q = (int)(g & 3);
    const int b = p.batch == 1 ? 0 : (int)(f / nw), w = (int)(f - (I)b * nw);
    const uint32_t byte = (word_of(f, b, w) >> (q * 8)) & 0xffu;
    const int row0 = w * 32 + q * 8;
    if (row0 >= V || byte == 0xffu) continue;
    Bits* dst = static_cast<Bits*>(p.logits) + (int64_t)b * p.logits_stride + row0;
    if (byte == 0u && vec_ok && row0 + 8 <= V) {
      if constexpr (sizeof(Bits) == 2) {
        const uint32_t x = (uint32_t)ninf | ((uint32_t)ninf << 16);
        *reinterpret_cast<uint4*>(dst) = make_uint4(x, x, x, x);
      } else {
        reinterpret_cast<uint4*>(dst)[0] = make_uint4(ninf, ninf, ninf, ninf);
        reinterpret_cast<uint4*>(dst)[1] = make_uint4(ninf, ninf, ninf, ninf);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (!((byte >> e) & 1u) && row0 + e < V) dst[e] = ninf;
    }
  }
}

template <typename T, typename WordFn>
__device__ __forceinline__ void fill_illegal(const RowSparseParams& p, int64_t w_lo, int64_t w_hi, WordFn word_of,
                                             int t0 = 0, int nt = 0) {
  if (nt == 0) nt = blockDim.x;
  const int me = (int)threadIdx.x - t0;
  if (me < 0 || me >= nt) return;
  if (w_hi * 4 + nt < (int64_t)INT32_MAX)
    fill_illegal_range<T, int>(p, (int)w_lo, (int)w_hi, word_of, me, nt);
  else
    fill_illegal_range<T, int64_t>(p, w_lo, w_hi, word_of, me, nt);
}

// Streams units s_list[0, n) (two rows per warp in flight) and emits them.
// With kHSmem, s_h holds the hidden rows of requests b0, b0 + 1, ... .
template <typename T, bool kHSmem, bool kSample>
__device__ __forceinline__ void stream_rows(const RowSparseParams& p, const uint32_t* s_list, int n, uint64_t rbase,
                                            uint32_t code_stride, const void* s_h, int b0, bool want_top,
                                            unsigned long long* s_keys) {
  using Bits = typename DTypeTraits<T>::Bits;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = p.hidden_dim, nvec = H / DTypeTraits<T>::kPerVec;
  RunningTop top;
  RunningSample rs;
  for (int i = warp; i < n; i += 2 * kWarps) {
    const int j = i + kWarps;
    const bool has2 = j < n;
    const uint32_t ca = s_list[i], cb = has2 ? s_list[j] : ca;
    const int ba = (int)(ca / code_stride), va = (int)(ca - (uint32_t)ba * code_stride);
    const int bb = (int)(cb / code_stride), vb = (int)(cb - (uint32_t)bb * code_stride);
    const uint4* wa = reinterpret_cast<const uint4*>(static_cast<const Bits*>(p.weight) + (int64_t)va * p.weight_stride);
    const uint4* wb = reinterpret_cast<const uint4*>(static_cast<const Bits*>(p.weight) + (int64_t)vb * p.weight_stride);
    const uint4* ha = kHSmem ? reinterpret_cast<const uint4*>(static_cast<const Bits*>(s_h) + (size_t)(ba - b0) * H)
                             : reinterpret_cast<const uint4*>(static_cast<const Bits*>(p.hidden) +
                                                              (int64_t)ba * p.hidden_stride);
    const uint4* hb = kHSmem ? reinterpret_cast<const uint4*>(static_cast<const Bits*>(s_h) + (size_t)(bb - b0) * H)
                             : reinterpret_cast<const uint4*>(static_cast<const Bits*>(p.hidden) +
                                                              (int64_t)bb * p.hidden_stride);
    float acc_a = 0.f, acc_b = 0.f;
    for (int base = 0; base < nvec; base += 32 * kUnroll) {
      uint4 ra[kUnroll], rb[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int e = base + u * 32 + lane;
        ra[u] = e < nvec ? ld_stream_v4(wa + e) : make_uint4(0, 0, 0, 0);
        rb[u] = (has2 && e < nvec) ? ld_stream_v4(wb + e) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int e = base + u * 32 + lane;
        if (e < nvec) {
          acc_a = dot_vec<T>(ra[u], kHSmem ? ha[e] : __ldg(ha + e), acc_a);
          if (has2) acc_b = dot_vec<T>(rb[u], kHSmem ? hb[e] : __ldg(hb + e), acc_b);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc_a += __shfl_xor_sync(FULL_MASK, acc_a, o);
      acc_b += __shfl_xor_sync(FULL_MASK, acc_b, o);
    }
    if (lane == 0) emit_unit<T, kSample>(p, ba, va, rbase + (uint64_t)i, acc_a, want_top, top, s_keys, rs, i);
    if (lane == 1 && has2) emit_unit<T, kSample>(p, bb, vb, rbase + (uint64_t)j, acc_b, want_top, top, s_keys, rs, j);
  }
  if (lane < 2) {
    top.flush(s_keys);
    if constexpr (kSample) rs.key.flush(s_keys + p.batch);
  }
}

// Scalar fallback of stream_rows (any alignment, any H).
template <typename T, bool kSample>
__device__ __forceinline__ void stream_rows_scalar(const RowSparseParams& p, const uint32_t* s_list, int n,
                                                   uint64_t rbase, uint32_t code_stride, bool want_top,
                                                   unsigned long long* s_keys) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = p.hidden_dim;
  RunningTop top;
  RunningSample rs;
  for (int i = warp; i < n; i += kWarps) {
    const uint32_t c = s_list[i];
    const int b = (int)(c / code_stride), v = (int)(c - (uint32_t)b * code_stride);
    using Bits = typename DTypeTraits<T>::Bits;
    const Bits* w = static_cast<const Bits*>(p.weight) + (int64_t)v * p.weight_stride;
    const Bits* h = static_cast<const Bits*>(p.hidden) + (int64_t)b * p.hidden_stride;
    float acc = 0.f;
    for (int k = lane; k < H; k += 32)
      acc = fmaf(DTypeTraits<T>::bits_to_float(__ldg(w + k)), DTypeTraits<T>::bits_to_float(__ldg(h + k)), acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(FULL_MASK, acc, o);
    if (lane == 0) emit_unit<T, kSample>(p, b, v, rbase + (uint64_t)i, acc, want_top, top, s_keys, rs, i);
  }
  if (lane == 0) {
    top.flush(s_keys);
    if constexpr (kSample) rs.key.flush(s_keys + p.batch);
  }
}

// Block-wide exclusive scan of one value per thread (kThreads threads);
// writes the block total to *total. Contains two __syncthreads.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* s_warp, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
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
  *total = s_warp[kWarps - 1];
  return incl - v + (warp > 0 ? s_warp[warp - 1] : 0u);
}

// Slot of flat word f in the transposed staging layout (kWpt words per thread,
// 16-byte vector v of thread t at vector index v * kThreads + t).
template <int kWpt>
__device__ __forceinline__ int staged_index(int f) {
  const int t = f / kWpt, r = f - t * kWpt;
  return ((r >> 2) * kThreads + t) * 4 + (r & 3);
}

// Unit code (request * code_stride + row) of rank r, resolved by the 16 lanes
// of one half-warp at once (both halves call it together, each for its own
// rank; r below the block total). Four levels, each a shared-memory read per
// lane and a ballot: the warp of the block scan that holds r (16 inclusive
// warp prefixes s_wincl), the thread within that warp (its 32 exclusive
// prefixes s_excl, relative to the warp's first rank), the word within that
// thread's kWpt staged words (their exclusive prefixes s_pre, also relative
// to the warp), the bit within the word. A single lane searching
// alone spent about 1,700 cycles in dependent steps; this takes a few
// ballots.
template <int kWpt>
__device__ __forceinline__ uint32_t code_of_rank_halfwarp(uint32_t r, const uint32_t* s_wincl, const uint32_t* s_excl,
                                                          const uint32_t* s_words, const uint32_t* s_pre, int batch,
                                                          int nw, uint32_t code_stride) {
  const int lane = threadIdx.x & 31, hl = lane & 15, sh = lane & 16;
  // level 1: warps whose inclusive prefix is <= r lie wholly below rank r
  const unsigned m1 = __ballot_sync(FULL_MASK, s_wincl[hl] <= r);
  const int W = __popc((m1 >> sh) & 0xffffu);
  r -= W > 0 ? s_wincl[W - 1] : 0u;  // rank within warp W (s_excl and s_pre are warp-relative)
  // level 2: threads of warp W whose first rank is <= r; the last one holds r
  const unsigned m2a = __ballot_sync(FULL_MASK, s_excl[32 * W + hl] <= r);
  const unsigned m2b = __ballot_sync(FULL_MASK, s_excl[32 * W + 16 + hl] <= r);
  const int t = 32 * W + __popc((m2a >> sh) & 0xffffu) + __popc((m2b >> sh) & 0xffffu) - 1;
  // level 3: the last non-empty word of thread t that starts at or below r
  int q = -1;
  uint32_t word = 0u, base = 0u;
#pragma unroll
  for (int part = 0; part < kWpt / 16; ++part) {
    const int si = staged_index<kWpt>(t * kWpt + 16 * part + hl);
    const uint32_t wd = s_words[si], pre = s_pre[si];
    const unsigned m3 = (__ballot_sync(FULL_MASK, wd != 0u && pre <= r) >> sh) & 0xffffu;
    const int src = m3 ? 31 - __clz(m3) : -1;
    const uint32_t w_src = __shfl_sync(FULL_MASK, wd, sh + (src < 0 ? 0 : src));
    const uint32_t p_src = __shfl_sync(FULL_MASK, pre, sh + (src < 0 ? 0 : src));
    if (src >= 0) {
      q = 16 * part + src;
      word = w_src;
      base = p_src;
    }
  }
  // level 4: the set bit of that word whose rank is r (lane hl tests bits hl and hl + 16)
  const uint32_t below_lo = word & ((1u << hl) - 1u);
  const uint32_t below_hi = word & ((1u << (hl + 16)) - 1u);
  const bool is_lo = ((word >> hl) & 1u) && base + (uint32_t)__popc(below_lo) == r;
  const bool is_hi = ((word >> (hl + 16)) & 1u) && base + (uint32_t)__popc(below_hi) == r;
  const unsigned m4lo = (__ballot_sync(FULL_MASK, is_lo) >> sh) & 0xffffu;
  const unsigned m4hi = (__ballot_sync(FULL_MASK, is_hi) >> sh) & 0xffffu;
  const int bit = m4lo ? __ffs(m4lo) - 1 : 16 + __ffs(m4hi) - 1;
  const int f = t * kWpt + (q < 0 ? 0 : q);
  const int b = batch == 1 ? 0 : f / nw, w = f - b * nw;
  return (uint32_t)b * code_stride + (uint32_t)(w * 32 + bit);
}

// Greedy streaming of the CTA's units of rank [rbase, rbase + n) with no unit
// list: warp w takes the pairs (w + 32k, w + 32k + 16); its two half-warps
// resolve a pair's two codes (code_of_rank_halfwarp; without a mask the code
// follows from the rank). The codes of the next pair are resolved while the
// current pair's row loads are in flight, so only the first pair's search is
// on the critical path.
template <int kWpt>
__device__ __forceinline__ uint32_t pair_code(const RowSparseParams& p, uint64_t rbase, int i, bool has2, bool has_mask,
                                              const uint32_t* s_wincl, const uint32_t* s_excl,
                                              const uint32_t* s_words, const uint32_t* s_pre, uint32_t code_stride) {
  const int lane = threadIdx.x & 31;
  const uint64_t r = rbase + (uint64_t)((lane >= 16 && has2) ? i + kWarps : i);
  if (has_mask)
    return code_of_rank_halfwarp<kWpt>((uint32_t)r, s_wincl, s_excl, s_words, s_pre, p.batch, p.nw, code_stride);
  const uint32_t b = (uint32_t)(r / (uint64_t)p.vocab);
  return b * code_stride + (uint32_t)(r - (uint64_t)b * p.vocab);
}

template <typename T, int kWpt>
__device__ __forceinline__ void stream_rows_ranked(const RowSparseParams& p, uint64_t rbase, int n, bool has_mask,
                                                   const uint32_t* s_wincl, const uint32_t* s_excl,
                                                   const uint32_t* s_words, const uint32_t* s_pre,
                                                   uint32_t code_stride, const void* s_h, bool want_top,
                                                   unsigned long long* s_keys) {
  using Bits = typename DTypeTraits<T>::Bits;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = p.hidden_dim, nvec = H / DTypeTraits<T>::kPerVec;
  RunningTop top;
  RunningSample rs;
  int i = warp;
  uint32_t my_code = i < n ? pair_code<kWpt>(p, rbase, i, i + kWarps < n, has_mask, s_wincl, s_excl, s_words, s_pre,
                                             code_stride)
                           : 0u;
  while (i < n) {
    const int j = i + kWarps;
    const bool has2 = j < n;
    const int i_next = i + 2 * kWarps;
    const uint32_t ca = __shfl_sync(FULL_MASK, my_code, 0);
    const uint32_t cb = __shfl_sync(FULL_MASK, my_code, 16);
    const int ba = (int)(ca / code_stride), va = (int)(ca - (uint32_t)ba * code_stride);
    const int bb = (int)(cb / code_stride), vb = (int)(cb - (uint32_t)bb * code_stride);
    const uint4* wa = reinterpret_cast<const uint4*>(static_cast<const Bits*>(p.weight) + (int64_t)va * p.weight_stride);
    const uint4* wb = reinterpret_cast<const uint4*>(static_cast<const Bits*>(p.weight) + (int64_t)vb * p.weight_stride);
    const uint4* ha = reinterpret_cast<const uint4*>(static_cast<const Bits*>(s_h) + (size_t)ba * H);
    const uint4* hb = reinterpret_cast<const uint4*>(static_cast<const Bits*>(s_h) + (size_t)bb * H);
    float acc_a = 0.f, acc_b = 0.f;
    for (int base = 0; base < nvec; base += 32 * kUnroll) {
      uint4 ra[kUnroll], rb[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int e = base + u * 32 + lane;
        ra[u] = e < nvec ? ld_stream_v4(wa + e) : make_uint4(0, 0, 0, 0);
        rb[u] = (has2 && e < nvec) ? ld_stream_v4(wb + e) : make_uint4(0, 0, 0, 0);
      }
      if (base == 0 && i_next < n)  // next pair's codes while these loads are in flight
        my_code = pair_code<kWpt>(p, rbase, i_next, i_next + kWarps < n, has_mask, s_wincl, s_excl, s_words, s_pre,
                                  code_stride);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int e = base + u * 32 + lane;
        if (e < nvec) {
          acc_a = dot_vec<T>(ra[u], ha[e], acc_a);
          if (has2) acc_b = dot_vec<T>(rb[u], hb[e], acc_b);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc_a += __shfl_xor_sync(FULL_MASK, acc_a, o);
      acc_b += __shfl_xor_sync(FULL_MASK, acc_b, o);
    }
    if (lane == 0) emit_unit<T, false>(p, ba, va, rbase + (uint64_t)i, acc_a, want_top, top, s_keys, rs, 0);
    if (lane == 1 && has2) emit_unit<T, false>(p, bb, vb, rbase + (uint64_t)j, acc_b, want_top, top, s_keys, rs, 0);
    i = i_next;
  }
  if (lane < 2) top.flush(s_keys);
}

// ===========================================================================
// staged kernel
// ===========================================================================
struct StagedLayout {
  size_t list, keys, warp, misc, excl, words, pre, hidden, total;
};

// `words` = number of mask words staged (kThreads * words per thread).
__host__ __device__ inline StagedLayout staged_layout(int batch, int hidden_dim, int words, int elem_bytes) {
  StagedLayout l;
  size_t off = 0;
  l.list = off;
  off += 4 * (size_t)kListCap;
  l.keys = align_up(off, 16);
  off = l.keys + keys_region_bytes(batch);
  l.warp = align_up(off, 16);
  off = l.warp + 4 * 32;
  l.misc = align_up(off, 16);
  off = l.misc + 16;
  l.excl = align_up(off, 16);
  off = l.excl + 4 * (size_t)kThreads;
  l.words = align_up(off, 16);
  off = l.words + 4 * (size_t)words;
  l.pre = align_up(off, 16);
  off = l.pre + 4 * (size_t)words;
  l.hidden = align_up(off, 16);
  off = l.hidden + (size_t)elem_bytes * batch * hidden_dim;
  l.total = align_up(off, 128);
  return l;
}


// kV 16-byte mask vectors (4 * kV words) per thread: the whole flat
// (request, word) mask lives in the CTA's registers, kThreads * 4 * kV words.
template <typename T, int kV, bool kSample>
__global__ void __launch_bounds__(kThreads, 1) row_sparse_staged_kernel(const RowSparseParams p) {
  constexpr int kWpt = 4 * kV;  // words per thread
  // Launched with programmatic dependent launch allowed: the CTAs may be
  // resident while the previous kernel in the stream (an input copy) still
  // runs; nothing is read or written before that kernel has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  extern __shared__ __align__(1024) unsigned char smem[];
  using Bits = typename DTypeTraits<T>::Bits;
  const StagedLayout L = staged_layout(p.batch, p.hidden_dim, kThreads * kWpt, (int)sizeof(Bits));
  uint32_t* s_list = reinterpret_cast<uint32_t*>(smem + L.list);
  unsigned long long* s_keys = reinterpret_cast<unsigned long long*>(smem + L.keys);
  uint32_t* s_warp = reinterpret_cast<uint32_t*>(smem + L.warp);
  int* s_misc = reinterpret_cast<int*>(smem + L.misc);
  uint32_t* s_words = reinterpret_cast<uint32_t*>(smem + L.words);
  uint32_t* s_pre = reinterpret_cast<uint32_t*>(smem + L.pre);
  uint32_t* s_excl = reinterpret_cast<uint32_t*>(smem + L.excl);
  Bits* s_h = reinterpret_cast<Bits*>(smem + L.hidden);

  const int tid = threadIdx.x;
  const int G = gridDim.x, cta = blockIdx.x;
  const int B = p.batch, V = p.vocab, H = p.hidden_dim, nw = p.nw;
  const int nvec = H / DTypeTraits<T>::kPerVec;
  const bool has_mask = p.mask != nullptr;
  const bool want_top = (p.top_value != nullptr) | (p.top_index != nullptr) | (p.top_key != nullptr);
  const int F = has_mask ? B * nw : 0;  // <= kThreads * kWpt (checked on the host)
  const int w_lo = (int)((int64_t)F * cta / G), w_hi = (int)((int64_t)F * (cta + 1) / G);
  const uint32_t tail_keep = (V & 31) ? ((1u << (V & 31)) - 1u) : 0xffffffffu;
  const int f0 = tid * kWpt;  // this thread's words: flat [f0, f0 + kWpt)

  // ---- 1. loads: this thread's mask words (registers), hidden states (smem).
  //         Every load of the phase is issued before any result is used, so
  //         the phase costs one round trip, not one per load. -----------------
  const int hvec = B * nvec;
  uint4 hx = make_uint4(0, 0, 0, 0);
  if (tid < hvec) {
    const int b = tid / nvec, j = tid - b * nvec;
    hx = __ldg(reinterpret_cast<const uint4*>(static_cast<const Bits*>(p.hidden) + (int64_t)b * p.hidden_stride) + j);
  }
  uint32_t wd[kWpt];
  if (has_mask) {
    const bool vec = ((reinterpret_cast<uintptr_t>(p.mask) & 15) == 0) && (nw % 4 == 0) &&
                     (B == 1 || p.mask_stride % 4 == 0);
    if (vec) {
      uint4 x[kV];
      bool tail[kV];
#pragma unroll
      for (int v = 0; v < kV; ++v) {
        const int f = f0 + 4 * v;
        x[v] = make_uint4(0, 0, 0, 0);
        tail[v] = false;
        if (f < F) {
          const int b = B == 1 ? 0 : f / nw, w = f - b * nw;  // w % 4 == 0
          tail[v] = (w == nw - 4);
          x[v] = __ldg(reinterpret_cast<const uint4*>(p.mask + (int64_t)b * p.mask_stride + w));
        }
      }
#pragma unroll
      for (int v = 0; v < kV; ++v) {
        wd[4 * v] = x[v].x;
        wd[4 * v + 1] = x[v].y;
        wd[4 * v + 2] = x[v].z;
        wd[4 * v + 3] = tail[v] ? (x[v].w & tail_keep) : x[v].w;
      }
    } else {
      bool tail[kWpt];
#pragma unroll
      for (int j = 0; j < kWpt; ++j) {
        const int f = f0 + j;
        wd[j] = 0u;
        tail[j] = false;
        if (f < F) {
          const int b = B == 1 ? 0 : f / nw, w = f - b * nw;
          tail[j] = (w == nw - 1);
          wd[j] = __ldg(p.mask + (int64_t)b * p.mask_stride + w);
        }
      }
#pragma unroll
      for (int j = 0; j < kWpt; ++j)
        if (tail[j]) wd[j] &= tail_keep;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kWpt; ++j) wd[j] = 0u;
  }
  if (tid < hvec) reinterpret_cast<uint4*>(s_h)[tid] = hx;
  for (int i = tid + kThreads; i < hvec; i += kThreads) {
    const int b = i / nvec, j = i - b * nvec;
    reinterpret_cast<uint4*>(s_h)[i] = __ldg(
        reinterpret_cast<const uint4*>(static_cast<const Bits*>(p.hidden) + (int64_t)b * p.hidden_stride) + j);
  }
  for (int b = tid; b < B; b += kThreads) s_keys[b] = 0ull;
  if constexpr (kSample) sample_smem_init(p, s_keys);

  // ---- 2. per-thread counts; words and warp-relative rank prefixes staged ---
  // The words and their exclusive rank prefixes go to shared memory before
  // the scan's first barrier, so that extraction and the -inf fill can run one
  // word per thread without a barrier of their own. The prefixes are relative
  // to the thread's warp (the warp's base is known only after the scan):
  // s_excl[t] is thread t's first rank within its warp, s_pre the same per
  // word; s_warp ends as the inclusive prefix of the warp totals. Layout of
  // the words: the 16-byte vector v of thread t at vector index
  // v * kThreads + t (conflict-free stores); staged_index() maps a flat word
  // index to its slot.
  uint32_t pc[kWpt];
  uint32_t cnt = 0;
#pragma unroll
  for (int j = 0; j < kWpt; ++j) {
    pc[j] = __popc(wd[j]);
    cnt += pc[j];
  }
  uint32_t incl_w = cnt;  // inclusive scan within the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(FULL_MASK, incl_w, o);
    if ((tid & 31) >= o) incl_w += t;
  }
  const uint32_t excl_w = incl_w - cnt;
  if ((tid & 31) == 31) s_warp[tid >> 5] = incl_w;
  s_excl[tid] = excl_w;
  if (has_mask) {
    uint32_t run = excl_w;
#pragma unroll
    for (int v = 0; v < kV; ++v) {
      uint4 pr;
      pr.x = run;
      run += pc[4 * v];
      pr.y = run;
      run += pc[4 * v + 1];
      pr.z = run;
      run += pc[4 * v + 2];
      pr.w = run;
      run += pc[4 * v + 3];
      reinterpret_cast<uint4*>(s_words)[v * kThreads + tid] = make_uint4(wd[4 * v], wd[4 * v + 1], wd[4 * v + 2], wd[4 * v + 3]);
      reinterpret_cast<uint4*>(s_pre)[v * kThreads + tid] = pr;
    }
  }
  // ---- 3. scan of the warp totals --------------------------------------------
  __syncthreads();
  if (tid < 32) {
    uint32_t x = tid < kWarps ? s_warp[tid] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(FULL_MASK, x, o);
      if (tid >= o) x += t;
    }
    if (tid < kWarps) s_warp[tid] = x;
  }
  __syncthreads();
  const uint32_t warp_base = (tid >> 5) > 0 ? s_warp[(tid >> 5) - 1] : 0u;
  const uint32_t excl = warp_base + excl_w;  // this thread's first rank
  const uint32_t tot = s_warp[kWarps - 1];
  const uint64_t total = has_mask ? (uint64_t)tot : (uint64_t)B * V;
  if (p.offsets != nullptr && cta == 0) {
    if (has_mask) {
      uint32_t run = excl;
#pragma unroll
      for (int j = 0; j < kWpt; ++j) {
        const int f = f0 + j;
        if (f < F && f % nw == 0) p.offsets[f / nw] = run;
        run += __popc(wd[j]);
      }
    } else {
      for (int b = tid; b < B; b += kThreads) p.offsets[b] = (int64_t)b * V;
    }
    if (tid == 0) p.offsets[B] = (int64_t)total;
  }

  // -inf over the illegal entries of this CTA's output slice, issued before
  // the rows so that the stores drain while the row loads are in flight
  if (p.logits && has_mask)
    fill_illegal<T>(p, w_lo, w_hi, [&](int64_t f, int, int) { return s_words[staged_index<kWpt>((int)f)]; });
  // this CTA's ranks [lo, hi) (32-bit arithmetic whenever it cannot overflow)
  uint64_t lo, hi;
  if (total <= 0xffffffffull / (uint64_t)G) {
    lo = (uint32_t)total * (uint32_t)cta / (uint32_t)G;
    hi = (uint32_t)total * (uint32_t)(cta + 1) / (uint32_t)G;
  } else {
    lo = total * (uint64_t)cta / (uint64_t)G;
    hi = total * (uint64_t)(cta + 1) / (uint64_t)G;
  }
  const uint32_t code_stride = (uint32_t)nw * 32u;
  if constexpr (!kSample) {
    // greedy: the half-warps resolve each pair's units from the prefixes, no unit list
    stream_rows_ranked<T, kWpt>(p, lo, (int)(hi - lo), has_mask, s_warp, s_excl, s_words, s_pre, code_stride, s_h,
                                want_top, s_keys);
  } else {
  for (uint64_t rbase = lo; rbase < hi; rbase += kListCap) {
    const uint64_t rend = min(hi, rbase + (uint64_t)kListCap);
    const int n = (int)(rend - rbase);
    // ---- 4. extraction: the threads holding ranks rbase and rend - 1 publish
    //         themselves (a register test, no per-word search), then every
    //         thread takes one word of their words and lists its units ------
    if (has_mask) {
      const uint32_t rb32 = (uint32_t)rbase, re32 = (uint32_t)rend;  // ranks < 2^32
      if (excl <= rb32 && rb32 < excl + cnt) s_misc[2] = tid;
      if (excl <= re32 - 1 && re32 - 1 < excl + cnt) s_misc[3] = tid;
      __syncthreads();
      const int fa = s_misc[2] * kWpt, fb = s_misc[3] * kWpt + kWpt;
      for (int f = fa + tid; f < fb; f += kThreads) {
        const int si = staged_index<kWpt>(f);
        uint32_t word = s_words[si];
        const int fw = (f / kWpt) >> 5;  // warp of the thread holding word f
        uint32_t r = s_pre[si] + (fw > 0 ? s_warp[fw - 1] : 0u);
        if (word == 0u || r >= re32 || r + (uint32_t)__popc(word) <= rb32) continue;
        const int b = B == 1 ? 0 : f / nw, w = f - b * nw;
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
    round_noise<kSample>(p, sample_smem(s_keys, B), s_list, n, code_stride);
    // ---- 5. stream the rows ------------------------------------------------
    stream_rows<T, true, kSample>(p, s_list, n, rbase, code_stride, s_h, 0, want_top, s_keys);
    round_stats<kSample>(sample_smem(s_keys, B), s_list, n, code_stride);
    __syncthreads();
  }
  }

  // ---- 7. top-1 ------------------------------------------------------------
  if (!kSample && want_top && polled_merge_ok(p))
    finalize_top1_polled(p, s_keys, reinterpret_cast<uint32_t*>(s_misc + 1));
  else
    finalize_top1<kSample>(p, s_keys, s_misc, want_top);
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
  l.warp = align_up(l.keys + keys_region_bytes(batch), 16);
  l.misc = align_up(l.warp + sizeof(uint32_t) * 32, 16);
  l.total = align_up(l.misc + 16, 128);
  return l;
}

template <typename T, bool kVec, bool kSample>
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
  if constexpr (kSample) sample_smem_init(p, s_keys);

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
    round_noise<kSample>(p, sample_smem(s_keys, B), s_list, n, code_stride);
    if (kVec)
      stream_rows<T, false, kSample>(p, s_list, n, rbase, code_stride, nullptr, 0, want_top, s_keys);
    else
      stream_rows_scalar<T, kSample>(p, s_list, n, rbase, code_stride, want_top, s_keys);
    round_stats<kSample>(sample_smem(s_keys, B), s_list, n, code_stride);
    __syncthreads();
  }

  if (p.logits && p.mask) {
    const int64_t w_lo = F * cta / G, w_hi = F * (cta + 1) / G;
    fill_illegal<T>(p, w_lo, w_hi, [&](int64_t, int b, int w) {
      return __ldg(p.mask + (int64_t)b * p.mask_stride + w);
    });
  }
  if (want_top || kSample) finalize_top1<kSample>(p, s_keys, s_misc, want_top);
}

// ===========================================================================
// cooperative kernel (masks too large for one CTA to scan: B * ceil(V/32) >
// 16,384 words)
// ===========================================================================
// The flat mask is cut into G equal word slices, one per CTA. Each CTA counts
// the legal units of its own slice and publishes the count; after a bounded
// wait for all G counts every CTA knows each slice's rank base and takes the
// units of rank [c*U/G, (c+1)*U/G), which it gets from the owners of the
// slices through a unit list in the workspace (list mode) or by re-scanning
// those slices. The mask is read from DRAM once in total, not G times.
constexpr int kCoopWpt = 8;                  // words per thread per chunk scan
constexpr int kChunk = kThreads * kCoopWpt;  // mask words per chunk scan
constexpr uint32_t kSliceSpinLimit = 1u << 20;
static_assert(kMaxSlices <= kThreads, "one slice count per thread");

constexpr int kHStageBytes = 64 * 1024;  // hidden rows of the requests one list round touches

struct CoopLayout {
  size_t list, keys, warp, misc, cnt, base, words, pre, hidden, total;
};

__host__ __device__ inline CoopLayout coop_layout(int batch) {
  CoopLayout l;
  size_t off = 0;
  l.list = off;
  off += 4 * (size_t)kListCap;
  l.keys = align_up(off, 16);
  off = l.keys + keys_region_bytes(batch);
  l.warp = align_up(off, 16);
  off = l.warp + 4 * 32;
  l.misc = align_up(off, 16);
  off = l.misc + 16;
  l.cnt = align_up(off, 16);
  off = l.cnt + 4 * (size_t)kMaxSlices;
  l.base = align_up(off, 16);
  off = l.base + 4 * (size_t)kMaxSlices;
  l.words = align_up(off, 16);
  off = l.words + 4 * (size_t)kChunk;
  l.pre = align_up(off, 16);
  off = l.pre + 4 * (size_t)kChunk;
  l.hidden = align_up(off, 16);
  off = l.hidden + kHStageBytes;
  l.total = align_up(off, 128);
  return l;
}

// Loads flat mask words [c0, c0 + n) (n <= kChunk; bits beyond the vocabulary
// cleared) into s_words with coalesced loads and their exclusive popcount
// prefixes (relative to c0) into s_pre; returns the chunk's popcount. Holds a
// __syncthreads before its first shared-memory write and after its last, so
// callers may reuse the buffers around it.
__device__ __forceinline__ uint32_t scan_chunk(const RowSparseParams& p, int c0, int n, uint32_t* s_words,
                                               uint32_t* s_pre, uint32_t* s_warp) {
  const int tid = threadIdx.x, nw = p.nw, V = p.vocab;
  const uint32_t tail_keep = (V & 31) ? ((1u << (V & 31)) - 1u) : 0xffffffffu;
  uint32_t ld[kCoopWpt];
#pragma unroll
  for (int j = 0; j < kCoopWpt; ++j) {  // all loads in flight at once
    const int i = tid + j * kThreads;
    ld[j] = 0u;
    if (i < n) {
      const int f = c0 + i;
      const int b = f / nw, w = f - b * nw;
      ld[j] = __ldg(p.mask + (int64_t)b * p.mask_stride + w);
      if (w == nw - 1) ld[j] &= tail_keep;
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kCoopWpt; ++j)
    if (tid + j * kThreads < n) s_words[tid + j * kThreads] = ld[j];
  __syncthreads();
  const int i0 = tid * kCoopWpt;
  const uint4 x0 = reinterpret_cast<const uint4*>(s_words + i0)[0];
  const uint4 x1 = reinterpret_cast<const uint4*>(s_words + i0)[1];
  const uint32_t xs[kCoopWpt] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
  uint32_t pc[kCoopWpt], cnt = 0;
#pragma unroll
  for (int j = 0; j < kCoopWpt; ++j) {
    pc[j] = (i0 + j < n) ? (uint32_t)__popc(xs[j]) : 0u;
    cnt += pc[j];
  }
  uint32_t tot;
  uint32_t run = block_exclusive_scan(cnt, s_warp, &tot);
  uint32_t pre[kCoopWpt];
#pragma unroll
  for (int j = 0; j < kCoopWpt; ++j) {
    pre[j] = run;
    run += pc[j];
  }
  reinterpret_cast<uint4*>(s_pre + i0)[0] = make_uint4(pre[0], pre[1], pre[2], pre[3]);
  reinterpret_cast<uint4*>(s_pre + i0)[1] = make_uint4(pre[4], pre[5], pre[6], pre[7]);
  __syncthreads();
  return tot;
}

// Stages the hidden rows of the requests s_list[0, n) touches in s_h (when
// they fit; reused across rounds) and streams the units. Every unit code is
// checked first (request < B, row < V): a round holding any other code (which
// only a workspace left dirty by an earlier failed launch can produce) sets
// the error word and is skipped, so no address is ever formed from it.
template <typename T, bool kSample>
__device__ __forceinline__ void coop_stream_round(const RowSparseParams& p, const uint32_t* s_list, int n,
                                                  uint32_t rbase, uint32_t code_stride, void* s_h, int& h_lo,
                                                  int& h_hi, bool want_top, unsigned long long* s_keys) {
  const int tid = threadIdx.x, H = p.hidden_dim;
  bool bad = false;
  for (int i = tid; i < n; i += kThreads) {
    const uint32_t code = s_list[i];
    const uint32_t b = code / code_stride;
    bad |= (b >= (uint32_t)p.batch) || (code - b * code_stride >= (uint32_t)p.vocab);
  }
  if (__syncthreads_or(bad)) {
    if (tid == 0 && p.error) atomicExch(p.error, 2);
    return;
  }
  round_noise<kSample>(p, sample_smem(s_keys, p.batch), s_list, n, code_stride);
  const int rb0 = (int)(s_list[0] / code_stride), rb1 = (int)(s_list[n - 1] / code_stride);
  using Bits = typename DTypeTraits<T>::Bits;
  if ((size_t)(rb1 - rb0 + 1) * H * sizeof(Bits) <= (size_t)kHStageBytes) {
    if (rb0 < h_lo || rb1 >= h_hi) {
      const int nvec = H / DTypeTraits<T>::kPerVec;
      for (int i = tid; i < (rb1 - rb0 + 1) * nvec; i += kThreads) {
        const int b = rb0 + i / nvec, j = i - (i / nvec) * nvec;
        reinterpret_cast<uint4*>(s_h)[i] = __ldg(
            reinterpret_cast<const uint4*>(static_cast<const Bits*>(p.hidden) + (int64_t)b * p.hidden_stride) + j);
      }
      h_lo = rb0;
      h_hi = rb1 + 1;
      __syncthreads();
    }
    stream_rows<T, true, kSample>(p, s_list, n, rbase, code_stride, s_h, h_lo, want_top, s_keys);
  } else {
    stream_rows<T, false, kSample>(p, s_list, n, rbase, code_stride, nullptr, 0, want_top, s_keys);
  }
  round_stats<kSample>(sample_smem(s_keys, p.batch), s_list, n, code_stride);
}

// Bounded wait (one polling thread per flag) until *flag != 0; returns the
// value seen, 0 on time-out.
__device__ __forceinline__ uint32_t wait_flag(const uint32_t* flag) {
  uint32_t v = 0;
  for (uint32_t i = 0; i < kSliceSpinLimit; ++i) {
    v = ld_acquire_gpu(flag);
    if (v != 0u) break;
    __nanosleep(32);
  }
  return v;
}

// End of the cooperative kernel: top-1 keys folded into the workspace, one
// ticket per CTA; the last CTA decodes the keys and re-zeroes slice counts,
// flags and ticket (every CTA has passed both of its waits by then).
template <bool kSample>
__device__ __forceinline__ void coop_finish(const RowSparseParams& p, unsigned long long* s_keys, int* s_flag,
                                            bool want_top) {
  const int tid = threadIdx.x, G = gridDim.x;
  __syncthreads();
  bool did = false;
  if (want_top) {
    for (int b = tid; b < p.batch; b += blockDim.x) {
      const unsigned long long k = s_keys[b];
      if (k != 0ull) {
        atomicMax(p.keys + b, k);
        did = true;
      }
    }
  }
  if constexpr (kSample) did |= sample_publish(p, sample_smem(s_keys, p.batch));
  if (did) __threadfence();
  __syncthreads();
  if (tid == 0) *s_flag = (atomicAdd(p.ticket, 1u) == (unsigned)G - 1u);
  __syncthreads();
  if (*s_flag) {
    __threadfence();
    if (want_top) decode_top1(p, s_keys, reinterpret_cast<uint32_t*>(s_flag + 1));
    if constexpr (kSample) sample_finish(p);
    for (int c = tid; c < G; c += blockDim.x) {
      p.slice_counts[c] = 0u;
      p.slice_ready[(size_t)c * kFlagStride] = 0u;
    }
    if (tid == 0) {
      *p.published = 0u;
      atomicExch(p.ticket, 0u);
    }
  }
}

// Launched cooperatively (every CTA co-resident), grid <= kMaxSlices, with a
// zeroed workspace; 16-byte aligned weight and hidden rows, H % 8 == 0.
//
// List mode (every slice fits one chunk scan and the batch has at most
// list_cap units): after the counts, each CTA writes the unit codes of its own
// slice, still in shared memory, into the workspace list at the slice's rank
// base and raises its slice flag; each CTA then waits only for the flags of
// the slices its rank range draws from and reads its units from the list.
// No mask word is read twice and nothing waits on memory once rows stream.
// Otherwise each CTA re-scans (from L2) the slices its rank range overlaps.
template <typename T, bool kSample>
__global__ void __launch_bounds__(kThreads, 1) row_sparse_coop_kernel(const RowSparseParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  const CoopLayout L = coop_layout(p.batch);
  uint32_t* s_list = reinterpret_cast<uint32_t*>(smem + L.list);
  unsigned long long* s_keys = reinterpret_cast<unsigned long long*>(smem + L.keys);
  uint32_t* s_warp = reinterpret_cast<uint32_t*>(smem + L.warp);
  int* s_misc = reinterpret_cast<int*>(smem + L.misc);
  uint32_t* s_cnt = reinterpret_cast<uint32_t*>(smem + L.cnt);
  uint32_t* s_base = reinterpret_cast<uint32_t*>(smem + L.base);
  uint32_t* s_words = reinterpret_cast<uint32_t*>(smem + L.words);
  uint32_t* s_pre = reinterpret_cast<uint32_t*>(smem + L.pre);
  void* s_h = smem + L.hidden;

  const int tid = threadIdx.x, G = gridDim.x, cta = blockIdx.x;
  const int B = p.batch, nw = p.nw, F = B * nw;
  const bool want_top = (p.top_value != nullptr) | (p.top_index != nullptr) | (p.top_key != nullptr);
  auto slice_lo = [&](int s) { return (int)((int64_t)F * s / G); };
  const int my_lo = slice_lo(cta), my_hi = slice_lo(cta + 1);
  const int max_slice = (F + G - 1) / G;  // every slice holds at most this many words
  for (int b = tid; b < B; b += kThreads) s_keys[b] = 0ull;
  if constexpr (kSample) sample_smem_init(p, s_keys);
  if (tid == 0) s_misc[0] = 0;

  // ---- 1. popcount of this CTA's slice, published to the grid --------------
  // (slice, chunk) currently held in s_words / s_pre, and its popcount
  int held_slice = -1, held_chunk = -1;
  uint32_t held_total = 0;
  uint32_t mine = 0;
  for (int c0 = my_lo, ch = 0; c0 < my_hi; c0 += kChunk, ++ch) {
    held_total = scan_chunk(p, c0, min(kChunk, my_hi - c0), s_words, s_pre, s_warp);
    held_slice = cta;
    held_chunk = ch;
    mine += held_total;
  }
  if (tid == 0) {
    p.slice_counts[cta] = mine;
    __threadfence();
    atom_add_release_gpu(p.published, 1u);
  }
  // While the other counts arrive, warps 1.. (warp 0 holds the poller) could
  // write -inf over the own slice's illegal entries; in list mode the fence
  // that publishes the CTA's units then waits for those stores too. So the
  // fill is issued here only when it is large (more than kEarlyFillBytes of
  // logits per CTA, where it would delay the rows more than the fence);
  // otherwise it runs beside the flag waits (list mode) or after the rows.
  // (Measured, V=248,320: deferred, batch 4 / 8 / 16 gained 0.3-0.5 us and
  // batch 32 lost 0.4 us.) Prefetching the slice's legal rows into L2 during
  // the count wait did not shorten the kernel.
  const int pollers = 32;
  const bool filled_early = p.logits != nullptr && max_slice <= kChunk &&
                            (int64_t)B * p.vocab * (int64_t)sizeof(typename DTypeTraits<T>::Bits) >
                                (int64_t)kEarlyFillBytes * G;
  if (filled_early && my_hi > my_lo)
    fill_illegal<T>(p, my_lo, my_hi, [&](int64_t f, int, int) { return s_words[f - my_lo]; }, pollers,
                    kThreads - pollers);

  // ---- 2. bounded wait for every slice count; rank base of each slice ------
  // (one poller per CTA on the published counter, then one load per count)
  if (tid == 0) {
    uint32_t v = 0;
    for (uint32_t i = 0; i < kSliceSpinLimit; ++i) {
      v = ld_acquire_gpu(p.published);
      if (v >= (uint32_t)G) break;
      __nanosleep(64);
    }
    if (v < (uint32_t)G) {
      if (p.error) atomicExch(p.error, 1);
      s_misc[0] = 1;
    }
  }
  __syncthreads();
  const uint32_t c = (tid < G && s_misc[0] == 0) ? __ldcg(p.slice_counts + tid) : 0u;
  uint32_t total;
  const uint32_t base = block_exclusive_scan(tid < G ? c : 0u, s_warp, &total);
  if (tid < G) {
    s_cnt[tid] = c;
    s_base[tid] = base;
  }
  __syncthreads();
  bool aborted = s_misc[0] != 0;

  const uint32_t lo = aborted ? 0u : (uint32_t)((uint64_t)total * cta / G);
  const uint32_t hi = aborted ? 0u : (uint32_t)((uint64_t)total * (cta + 1) / G);
  const uint32_t code_stride = (uint32_t)nw * 32u;
  const bool list_mode = max_slice <= kChunk && (int64_t)total <= p.list_cap;
  int h_lo = 0, h_hi = 0;  // requests whose hidden rows are in s_h

  if (list_mode) {
    // ---- 3. own units -> list at the slice's rank base; flag ---------------
    if (!aborted) {
      const uint32_t sb = s_base[cta];
      for (int i = tid; i < my_hi - my_lo; i += kThreads) {
        uint32_t word = s_words[i];
        uint32_t r = sb + s_pre[i];
        const int f = my_lo + i;
        const int b = f / nw, w = f - b * nw;
        if (p.offsets != nullptr && w == 0) p.offsets[b] = (int64_t)r;
        while (word) {
          const int bit = __ffs(word) - 1;
          word &= word - 1;
          p.unit_list[r++] = (uint32_t)b * code_stride + (uint32_t)(w * 32 + bit);
        }
      }
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        st_release_gpu(p.slice_ready + (size_t)cta * kFlagStride, 1u);
      }
    }
    // the -inf fill of the own slice runs beside the flag waits (threads below
    // the first whole warp past the grid poll flags, the others fill)
    if (p.logits != nullptr && !filled_early && my_hi > my_lo && !aborted) {
      const int t0 = (G + 31) / 32 * 32 < kThreads ? (G + 31) / 32 * 32 : 0;
      fill_illegal<T>(p, my_lo, my_hi, [&](int64_t f, int, int) { return s_words[f - my_lo]; }, t0, kThreads - t0);
    }
    // ---- 4. wait for the slices this CTA's ranks come from; stream ---------
    if (lo < hi) {
      if (tid < G) {
        const uint32_t sb = s_base[tid], sc = s_cnt[tid];
        if (sc != 0u && sb < hi && sb + sc > lo && wait_flag(p.slice_ready + (size_t)tid * kFlagStride) == 0u) {
          if (p.error) atomicExch(p.error, 1);
          s_misc[0] = 1;
        }
      }
      __syncthreads();
      aborted = s_misc[0] != 0;
    }
    for (uint32_t rbase = lo; rbase < hi && !aborted; rbase += kListCap) {
      const int n = (int)(min(hi, rbase + (uint32_t)kListCap) - rbase);
      // read the units and re-zero them: each entry is written by one owner
      // and read by one CTA, so the list is all zero again on exit
      for (int i = tid; i < n; i += kThreads) {
        s_list[i] = __ldcg(p.unit_list + rbase + i);
        p.unit_list[rbase + i] = 0u;
      }
      __syncthreads();
      coop_stream_round<T, kSample>(p, s_list, n, rbase, code_stride, s_h, h_lo, h_hi, want_top, s_keys);
      __syncthreads();
    }
  } else {
    // ---- 3'. re-scan the slices each round of ranks overlaps ---------------
    for (uint32_t rbase = lo; rbase < hi; rbase += kListCap) {
      const uint32_t rend = min(hi, rbase + (uint32_t)kListCap);
      for (int s = 0; s < G; ++s) {
        const uint32_t sb = s_base[s], sc = s_cnt[s];
        if (sb >= rend) break;
        if (sc == 0u || sb + sc <= rbase) continue;
        const int s_lo = slice_lo(s), s_hi = slice_lo(s + 1);
        uint32_t run = sb;
        for (int c0 = s_lo, ch = 0; c0 < s_hi && run < rend; c0 += kChunk, ++ch) {
          const int n = min(kChunk, s_hi - c0);
          if (held_slice != s || held_chunk != ch) {
            held_total = scan_chunk(p, c0, n, s_words, s_pre, s_warp);
            held_slice = s;
            held_chunk = ch;
          }
          if (run + held_total > rbase) {
            for (int i = tid; i < n; i += kThreads) {
              uint32_t word = s_words[i];
              uint32_t r = run + s_pre[i];
              if (word == 0u || r >= rend || r + (uint32_t)__popc(word) <= rbase) continue;
              const int f = c0 + i;
              const int b = f / nw, w = f - b * nw;
              while (word) {
                const int bit = __ffs(word) - 1;
                word &= word - 1;
                if (r >= rbase && r < rend) s_list[r - rbase] = (uint32_t)b * code_stride + (uint32_t)(w * 32 + bit);
                ++r;
              }
            }
          }
          run += held_total;
        }
      }
      __syncthreads();
      coop_stream_round<T, kSample>(p, s_list, (int)(rend - rbase), rbase, code_stride, s_h, h_lo, h_hi, want_top,
                                    s_keys);
      __syncthreads();
    }
    // ---- 4'. own slice: request offsets (compact output), -inf fill ---------
    if ((p.logits != nullptr && !filled_early) || p.offsets != nullptr) {
      uint32_t run = s_base[cta];
      for (int c0 = my_lo, ch = 0; c0 < my_hi; c0 += kChunk, ++ch) {
        const int n = min(kChunk, my_hi - c0);
        if (held_slice != cta || held_chunk != ch) {
          held_total = scan_chunk(p, c0, n, s_words, s_pre, s_warp);
          held_slice = cta;
          held_chunk = ch;
        }
        if (p.offsets != nullptr) {
          for (int i = tid; i < n; i += kThreads) {
            const int f = c0 + i;
            if (f % nw == 0) p.offsets[f / nw] = (int64_t)(run + s_pre[i]);
          }
        }
        if (p.logits != nullptr && !filled_early)
          fill_illegal<T>(p, c0, c0 + n, [&](int64_t f, int, int) { return s_words[f - c0]; });
        run += held_total;
      }
    }
  }
  if (p.offsets != nullptr && cta == 0 && tid == 0) p.offsets[B] = (int64_t)total;

  // ---- 5. top-1, workspace reset ------------------------------------------
  coop_finish<kSample>(p, s_keys, s_misc + 2, want_top);
}

// ===========================================================================
// launch
// ===========================================================================
template <typename T, bool kSample>
cudaError_t launch_typed(const RowSparseParams& p, cudaStream_t stream) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  const int grid = num_sms(dev);
  constexpr int kPV = DTypeTraits<T>::kPerVec;
  const bool vec = (p.hidden_dim % kPV == 0) && ((reinterpret_cast<uintptr_t>(p.weight) & 15) == 0) &&
                   (p.weight_stride % kPV == 0) && ((reinterpret_cast<uintptr_t>(p.hidden) & 15) == 0) &&
                   (p.batch == 1 || p.hidden_stride % kPV == 0);
  const int64_t F64 = p.mask ? (int64_t)p.batch * p.nw : 0;
  if (vec && F64 > kCoopMinWords && p.slice_counts != nullptr && p.published != nullptr && p.slice_ready != nullptr &&
      F64 * 32 < (int64_t)1 << 32) {
    const CoopLayout L = coop_layout(p.batch);
    if (L.total <= kStagedSmemMax) {
      auto k = row_sparse_coop_kernel<T, kSample>;
      if ((err = raise_smem_limit(reinterpret_cast<const void*>(k), L.total, dev)) != cudaSuccess) return err;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)min(grid, kMaxSlices));
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = L.total;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      return cudaLaunchKernelEx(&cfg, k, p);
    }
  }
  if (vec) {
    const int F = p.mask ? p.batch * p.nw : 0;
    const int wpt = F <= kThreads * 16 ? 16 : 32;
    const StagedLayout L = staged_layout(p.batch, p.hidden_dim, kThreads * wpt, (int)sizeof(typename DTypeTraits<T>::Bits));
    if (L.total <= kStagedSmemMax && F <= kThreads * 32) {
      auto k = wpt == 16 ? row_sparse_staged_kernel<T, 4, kSample> : row_sparse_staged_kernel<T, 8, kSample>;
      if ((err = raise_smem_limit(reinterpret_cast<const void*>(k), L.total, dev)) != cudaSuccess) return err;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)grid);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = L.total;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      return cudaLaunchKernelEx(&cfg, k, p);
    }
  }
  const DirectLayout L = direct_layout(p.batch);
  if (vec) {
    auto k = row_sparse_direct_kernel<T, true, kSample>;
    if ((err = raise_smem_limit(reinterpret_cast<const void*>(k), L.total, dev)) != cudaSuccess) return err;
    k<<<grid, kThreads, L.total, stream>>>(p);
  } else {
    auto k = row_sparse_direct_kernel<T, false, kSample>;
    if ((err = raise_smem_limit(reinterpret_cast<const void*>(k), L.total, dev)) != cudaSuccess) return err;
    k<<<grid, kThreads, L.total, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_row_sparse(const RowSparseParams& p, int dtype, cudaStream_t stream) {
  const bool sample = p.sample_index != nullptr;
  if (dtype == 2) {
    if (sample) return cudaErrorNotSupported;  // the sampler takes half-precision inputs only
    return launch_typed<float, false>(p, stream);
  }
  if (dtype == 1) return sample ? launch_typed<__nv_bfloat16, true>(p, stream) : launch_typed<__nv_bfloat16, false>(p, stream);
  return sample ? launch_typed<__half, true>(p, stream) : launch_typed<__half, false>(p, stream);
}

}  // namespace gsp
