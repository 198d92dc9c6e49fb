// Grammar-aware block GEMM and dense masked GEMM on sm_100a tensor cores.
//
// Behaviour follows gsp/triton_runtime.py:147-209 (_bitmask_block_gemm_kernel):
// logits[b, v] = sum_k W[v, k] h[b, k] (fp32 accumulate, rounded to the input
// dtype) where token v is legal for request b, -inf elsewhere; only vocabulary
// tiles holding a legal token of some request are multiplied. The dense route
// (gsp/triton_runtime.py:285-308, F.linear + xgrammar mask) is the same kernel
// over every tile.
//
// Two launches:
//  * tile_builder_kernel: for every 128-row vocabulary tile, OR of the batch's
//    mask words (4 words per request); active tile ids are compacted per
//    builder block of kBuilderTiles tiles. Skipped in dense mode.
//  * tc_projection_kernel: one persistent CTA per SM, 10 warps.
//      warp 0      one lane issues TMA loads of the W tile (128 rows x 64 K,
//                  128-byte swizzle) and of h (Npad rows x 64 K) into a ring of
//                  shared-memory stages;
//      warp 1      allocates TMEM; one lane issues tcgen05.mma (M=128 vocabulary
//                  rows, N = batch padded to a multiple of 32, K = 16 per
//                  instruction) into one of 4 TMEM accumulators (2 when
//                  N > 128), committing each stage back to the producer and
//                  each tile to the epilogue;
//      warps 2-9   epilogue, two warps per TMEM lane quadrant splitting the
//                  accumulator's columns: first -inf over every request's
//                  outputs in the inactive tiles (block mode; while the first
//                  accumulator is computed), then per tile tcgen05.ld of the
//                  accumulator (one TMEM lane = one vocabulary row per thread),
//                  mask bit (words loaded before the accumulator wait),
//                  rounding, -inf, logits stores coalesced along the
//                  vocabulary, and 32-bit warp-local top-1 keys (16-bit value
//                  order + row) reduced across the warp's 32 rows with a
//                  transpose-reduce, widened to 64-bit global keys once per
//                  request.
//    Tiles are taken from the compacted list round-robin by CTA; at set-up a
//    CTA copies the whole list into its (still idle) A stages in the same
//    round trip as the per-builder-block counts and picks its own tiles out
//    of it. The cross-CTA top-1 merge is the last-arrival ticket scheme of
//    the row-sparse kernel's batched path.
//
// "Swap-AB": the vocabulary is the MMA's M dimension and the (small) batch its N
// dimension, so a batch of 2..256 requests fills a 128 x N tile.
//
// Every wait is bounded; a timed-out wait sets the workspace error word and the
// kernel drains its copies and tensor-core work before returning.
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "gsp_async.cuh"
#include "gsp_common.cuh"
#include "gsp_internal.h"
#include "gsp_peer.cuh"
#include "gsp_sampler.cuh"
#include "gsp_tcgen05.cuh"

namespace gsp {
namespace {

constexpr int kTileRows = 128;
constexpr int kTileK = 64;  // K elements per stage: one 128-byte swizzle row
constexpr int kEpilogueWarps = 8;  // two per TMEM lane quadrant
constexpr int kGemmThreads = 32 * (2 + kEpilogueWarps);
constexpr int kMaxNpad = 256;
constexpr int kMaxAcc = 4;          // TMEM accumulators (4 when npad <= 128, else 2)
constexpr int kMaxUnits = kMaxNpad / 64;  // 32-column units per epilogue warp
constexpr int kMaxStages = 8;
constexpr int kMaxMine = 64;  // tiles per CTA that the set-up can list in shared memory
constexpr uint32_t kABytes = kTileRows * kTileK * 2;  // 16 KB

struct GemmConfig {
  int npad;      // batch padded to a multiple of 32 (<= 256)
  int stages;
  int kblocks;   // ceil(H / 64)
  int ntiles;    // ceil(V / 128)
  int nbuild;    // builder blocks (block mode)
  int acc_shift; // log2 of the accumulator count
  int stage_list; // block mode: the set-up copies the tile list into shared memory
  uint32_t tmem_cols;
  uint32_t idesc;
};

struct GemmLayout {
  size_t a, b, bars, tmem, keys, skeys, stats, pref, mine, misc, total;
};

__host__ __device__ inline size_t align_to(size_t x, size_t a) { return (x + a - 1) / a * a; }

__host__ __device__ inline GemmLayout gemm_layout(int npad, int stages, int nbuild) {
  GemmLayout l;
  size_t off = 0;
  l.a = off;
  off += (size_t)stages * kABytes;
  l.b = align_to(off, 1024);
  off = l.b + (size_t)stages * npad * kTileK * 2;
  l.bars = align_to(off, 16);
  off = l.bars + 8 * (2 * (size_t)stages + 2 * kMaxAcc);
  l.tmem = align_to(off, 16);
  off = l.tmem + 16;
  l.keys = align_to(off, 16);
  off = l.keys + 8 * (size_t)kMaxNpad;
  l.skeys = align_to(off, 16);  // sampler: the CTA's winning perturbed key per request
  off = l.skeys + 8 * (size_t)kMaxNpad;
  l.stats = align_to(off, 16);  // sampler: the CTA's (max, sum) pair per request
  off = l.stats + 8 * (size_t)kMaxNpad;
  l.pref = align_to(off, 16);
  off = l.pref + 4 * ((size_t)nbuild + 1);
  l.mine = align_to(off, 16);  // this CTA's tile ids (block mode, stage_list)
  off = l.mine + 4 * (size_t)kMaxMine;
  l.misc = align_to(off, 16);
  off = l.misc + 16;
  l.total = align_to(off, 1024);
  return l;
}

// Slot of compacted position `pos` in the workspace tile list (block mode).
__device__ __forceinline__ int list_slot(const GemmConfig& c, const int* s_pref, int pos) {
  int lo = 0, hi = c.nbuild;  // find j with s_pref[j] <= pos < s_pref[j + 1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (s_pref[mid] <= pos) lo = mid; else hi = mid;
  }
  return lo * kBuilderTiles + (pos - s_pref[lo]);
}

// Tile id of compacted position `pos`, the CTA's i-th tile.
__device__ __forceinline__ int tile_at(const BlockGemmParams& p, const GemmConfig& c, const int* s_pref,
                                       const int* s_mine, int pos, int i) {
  if (p.dense) return pos;
  return c.stage_list ? s_mine[i] : p.tile_list[list_slot(c, s_pref, pos)];
}

// -inf over every request's outputs in the inactive 128-row tiles
// t = cta + G * (ew + kEpilogueWarps j) (block mode): a tile is inactive when
// no request has a legal token in it, the same test the builder applies. Run
// by the epilogue warps (ew = 0..kEpilogueWarps-1) before their first
// accumulator arrives.
template <typename T>
__device__ __forceinline__ void fill_inactive_tiles(const BlockGemmParams& p, int ntiles, int cta, int G, int ew,
                                                    int lane) {
  const int V = p.vocab, nw = p.nw, B = p.batch;
  const uint16_t ninf = DTypeTraits<T>::kNegInfBits;
  const uint32_t x = (uint32_t)ninf | ((uint32_t)ninf << 16);
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(p.logits) & 15) == 0) && (p.logits_stride % 8 == 0);
  for (int t = cta + ew * G; t < ntiles; t += kEpilogueWarps * G) {
    uint32_t any = 0u;
    for (int b = lane; b < B; b += 32) {
      const uint32_t* row = p.mask + (int64_t)b * p.mask_stride;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int w = t * 4 + j;
        if (w < nw) any |= tail_clip(__ldg(row + w), w, V);
      }
    }
    if (__any_sync(FULL_MASK, any != 0u)) continue;
    const int r0 = t * kTileRows;
    uint16_t* base = static_cast<uint16_t*>(p.logits) + r0;
    if (vec_ok && r0 + kTileRows <= V) {
      // 256 B per request: lanes 0-15 take request b, lanes 16-31 request b + 1
      for (int b = lane >> 4; b < B; b += 2)
        reinterpret_cast<uint4*>(base + (int64_t)b * p.logits_stride)[lane & 15] = make_uint4(x, x, x, x);
    } else {
      for (int b = 0; b < B; ++b)
        for (int r = lane; r < kTileRows && r0 + r < V; r += 32) base[(int64_t)b * p.logits_stride + r] = ninf;
    }
  }
}

// First request column of epilogue unit u of the quadrant's warp `half`.
__device__ __forceinline__ int unit_col(bool narrow, int half, int u) {
  return narrow ? 16 * half : 32 * (half + 2 * u);
}

// Warp-local top-1 key of a rounded 16-bit value at row `lane` of the warp's
// 32 rows: an order-preserving map of the 16-bit pattern (sign-magnitude to
// biased, -0 and +0 equal, every legal value >= 0x0001) in the high half, and
// 0xffff - lane in the low half so that the lower row wins ties. 0 means "no
// legal token". Ordering equals that of top1_key on the widened value.
__device__ __forceinline__ uint32_t warp_key16(uint32_t bits, uint32_t low) {
  const uint32_t o = (bits & 0x8000u) ? 0x8000u - (bits & 0x7fffu) : (bits | 0x8000u);
  return (o << 16) | low;
}

// Widen a warp_key16 of the warp whose first row is `row_base` (global
// vocabulary id) to a global top1_key and keep the larger.
template <typename T>
__device__ __forceinline__ unsigned long long merge_unit_key(unsigned long long running, uint32_t k, int64_t row_base) {
  if (k == 0u) return running;
  const uint32_t o = k >> 16;
  const uint32_t bits = o >= 0x8000u ? (o & 0x7fffu) : (0x8000u | (0x8000u - o));
  const uint32_t r = 0xffffu - (k & 0xffffu);
  const unsigned long long key =
      top1_key(DTypeTraits<T>::bits_to_float((uint16_t)bits), (uint64_t)(row_base + (int64_t)r));
  return key > running ? key : running;
}

// Sampler state of one epilogue unit (kSample kernels): its requests' seeds and
// the CTA's per-request accumulators in shared memory, all offset to the
// unit's first column, and the global token id of this lane's row.
struct UnitSampler {
  const uint64_t* seeds;
  unsigned long long* skeys;
  unsigned long long* stats;
  uint64_t offset;
  float inv_temp;
  int64_t global_row;
};

// Fused sampler, one accumulator column jj of the warp's 32 rows (the contract
// of gsp_sampler.cuh): the legal rows' perturbed scores x * inv_temp + Gumbel
// noise keyed by (seed, step, global id), their warp maximum as a top-1 key
// (ties to the lower id), and the warp's (max, sum of exp) pair of the scaled
// logits, folded into the CTA's shared accumulators by lane 0 (one shared
// atomicMax and one compare-and-swap merge per warp and column). Columns with
// no legal row in the warp cost one ballot. Called by all 32 lanes.
template <typename T>
__device__ __forceinline__ void sample_column(const UnitSampler& su, int jj, bool legal, uint16_t bits) {
  if (__ballot_sync(FULL_MASK, legal) == 0u) return;
  const float y = legal ? DTypeTraits<T>::bits_to_float(bits) * su.inv_temp : -INFINITY;
  unsigned long long sk = 0ull;
  if (legal)
    sk = top1_key(y + gumbel_noise_outlined(su.seeds[jj], su.offset, (uint64_t)su.global_row),
                  (uint64_t)su.global_row);
  sk = warp_max_u64(sk);
  const float m = from_ordered_bits(__reduce_max_sync(FULL_MASK, legal ? ordered_bits(y) : 0u));
  float e = legal ? __expf(y - m) : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(FULL_MASK, e, o);
  if ((threadIdx.x & 31) == 0) {
    atomicMax(&su.skeys[jj], sk);
    unsigned long long old = su.stats[jj], assumed;
    do {
      assumed = old;
      float mm = stats_m(assumed), ss = stats_s(assumed);
      merge_stats(mm, ss, m, e);
      old = atomicCAS(&su.stats[jj], assumed, pack_stats(mm, ss));
    } while (old != assumed);
  }
}

// One epilogue unit: kCols accumulator columns (requests b0 .. b0 + kCols - 1)
// of this warp's 32 TMEM lanes (one vocabulary row per thread). Rounds to the
// logits dtype, applies the mask bit (word_l: this lane's mask word for
// request b0 + lane % kCols), stores the row's logits (-inf where illegal) and
// returns in lane l < kCols the warp_key16 maximum over the 32 rows for
// request b0 + l. With kSample, also feeds every column to sample_column.
template <typename T, int kCols, bool kSample>
__device__ __forceinline__ uint32_t epilogue_unit(uint32_t taddr, uint32_t word_l, int b0, int B, bool row_ok,
                                                  bool store, uint16_t* out, int64_t stride, int lane,
                                                  const UnitSampler& su) {
  uint32_t v[kCols];
  if constexpr (kCols == 32) tmem_ld32(taddr, v);
  else tmem_ld16(taddr, v);
  tmem_ld_wait();
  const uint16_t ninf = DTypeTraits<T>::kNegInfBits;
  const uint32_t lanebit = row_ok ? (1u << lane) : 0u;
  const uint32_t low = 0xffffu - (uint32_t)lane;
  uint32_t key[kCols];
  if (b0 + kCols <= B) {
#pragma unroll
    for (int jj = 0; jj < kCols; ++jj) {
      const bool legal = (__shfl_sync(FULL_MASK, word_l, jj) & lanebit) != 0u;
      const uint16_t bits = legal ? DTypeTraits<T>::round_bits(__uint_as_float(v[jj])) : ninf;
      if (store) out[jj * stride] = bits;
      key[jj] = legal ? warp_key16(bits, low) : 0u;
      if constexpr (kSample) sample_column<T>(su, jj, legal, bits);
    }
  } else {
#pragma unroll
    for (int jj = 0; jj < kCols; ++jj) {
      const bool legal = (__shfl_sync(FULL_MASK, word_l, jj) & lanebit) != 0u;  // word is 0 past B
      const uint16_t bits = legal ? DTypeTraits<T>::round_bits(__uint_as_float(v[jj])) : ninf;
      if (store && b0 + jj < B) out[jj * stride] = bits;
      key[jj] = legal ? warp_key16(bits, low) : 0u;
      if constexpr (kSample) sample_column<T>(su, jj, legal, bits);
    }
  }
  // transpose-reduce: lane l ends with the maximum over the 32 rows of
  // column l % kCols
#pragma unroll
  for (int h = kCols / 2; h >= 1; h >>= 1) {
    const bool upper = (lane & h) != 0;
#pragma unroll
    for (int j = 0; j < h; ++j) {
      const uint32_t send = upper ? key[j] : key[j + h];
      const uint32_t keep = upper ? key[j + h] : key[j];
      const uint32_t recv = __shfl_xor_sync(FULL_MASK, send, h);
      key[j] = keep > recv ? keep : recv;
    }
  }
  if constexpr (kCols == 16) {
    const uint32_t other = __shfl_xor_sync(FULL_MASK, key[0], 16);
    key[0] = key[0] > other ? key[0] : other;
  }
  return key[0];
}

// kNarrow: the batch pads to 32 columns (one 16-column unit per epilogue warp).
// kSample: the fused sampler (p.sample_index != nullptr) runs in the epilogue.
template <typename T, bool kNarrow, bool kSample>
__global__ void __launch_bounds__(kGemmThreads, 1)
    tc_projection_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_h,
                         const BlockGemmParams p, const GemmConfig c) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 128-byte-swizzled TMA tiles need 1024-byte alignment; the launch reserves
  // 1 KB of slack for this round-up.
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const GemmLayout L = gemm_layout(c.npad, c.stages, c.nbuild);
  unsigned char* s_a = smem + L.a;
  unsigned char* s_b = smem + L.b;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + c.stages;
  uint64_t* tfull = empty + c.stages;  // [kMaxAcc]
  uint64_t* tempty = tfull + kMaxAcc;  // [kMaxAcc]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L.tmem);
  unsigned long long* s_keys = reinterpret_cast<unsigned long long*>(smem + L.keys);
  unsigned long long* s_skeys = reinterpret_cast<unsigned long long*>(smem + L.skeys);
  unsigned long long* s_stats = reinterpret_cast<unsigned long long*>(smem + L.stats);
  int* s_pref = reinterpret_cast<int*>(smem + L.pref);
  int* s_mine = reinterpret_cast<int*>(smem + L.mine);
  int* s_misc = reinterpret_cast<int*>(smem + L.misc);  // [0] abort, [1] last-CTA flag
  volatile int* abort_flag = s_misc;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int B = p.batch, V = p.vocab;
  const bool want_top = (p.top_value != nullptr) | (p.top_index != nullptr) | (p.top_key != nullptr);

  // ---- set-up -------------------------------------------------------------
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_h);
    for (int s = 0; s < c.stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int a = 0; a < kMaxAcc; ++a) {
      mbar_init(tfull + a, 1);
      mbar_init(tempty + a, kEpilogueWarps);  // one arrival per epilogue warp
    }
    fence_mbar_init();
    s_misc[0] = 0;
    s_misc[1] = 0;
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, c.tmem_cols);
    tmem_relinquish();
  }
  for (int i = tid; i < kMaxNpad; i += kGemmThreads) s_keys[i] = 0ull;
  if constexpr (kSample) {
    for (int i = tid; i < kMaxNpad; i += kGemmThreads) {
      s_skeys[i] = 0ull;
      s_stats[i] = empty_stats();
    }
  }
  // Everything above overlaps the tile builder; from here on its outputs (and
  // the inactive-tile -inf fill) are complete and visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (!p.dense && c.stage_list && warp != 2) {
    // The whole compacted list into shared memory, in the same round trip as
    // the counts that warp 2 reads (the A stages are idle until the
    // producer's first copy); the CTA picks its own tiles out of it below.
    int* s_list = reinterpret_cast<int*>(s_a);
    const int t = warp < 2 ? tid : tid - 32, nt = kGemmThreads - 32;
    const int n = c.ntiles;
    if ((reinterpret_cast<uintptr_t>(p.tile_list) & 15) == 0) {
      const int4* src = reinterpret_cast<const int4*>(p.tile_list);
      int4* dst = reinterpret_cast<int4*>(s_list);
      const int n4 = n / 4;
      for (int i0 = t; i0 < n4; i0 += 4 * nt) {
        int4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (i0 + u * nt < n4) v[u] = src[i0 + u * nt];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (i0 + u * nt < n4) dst[i0 + u * nt] = v[u];
      }
      for (int j = n4 * 4 + t; j < n; j += nt) s_list[j] = p.tile_list[j];
    } else {
      for (int j = t; j < n; j += nt) s_list[j] = p.tile_list[j];
    }
  }
  if (!p.dense && warp == 2) {
    // exclusive prefix of the builder blocks' active-tile counts; up to 256
    // counts are loaded before the first is used (one round trip)
    constexpr int kPre = 8;
    int carry = 0;
    for (int j00 = 0; j00 < c.nbuild; j00 += 32 * kPre) {
      int v[kPre];
#pragma unroll
      for (int u = 0; u < kPre; ++u) {
        const int j = j00 + u * 32 + lane;
        v[u] = j < c.nbuild ? p.tile_counts[j] : 0;
      }
#pragma unroll
      for (int u = 0; u < kPre; ++u) {
        const int j = j00 + u * 32 + lane;
        int incl = v[u];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(FULL_MASK, incl, o);
          if (lane >= o) incl += t;
        }
        if (j < c.nbuild) s_pref[j] = carry + incl - v[u];
        carry += __shfl_sync(FULL_MASK, incl, 31);
      }
    }
    if (lane == 0) s_pref[c.nbuild] = carry;
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *s_tmem;
  const int total = p.dense ? c.ntiles : s_pref[c.nbuild];
  if (!p.dense && c.stage_list) {
    // this CTA's tiles, compacted positions cta, cta + G, ..., in order
    const int* s_list = reinterpret_cast<const int*>(s_a);
    for (int j = tid; j < c.nbuild; j += kGemmThreads) {
      const int base = s_pref[j], cnt = s_pref[j + 1] - base;
      int k = (cta - base) % G;
      if (k < 0) k += G;
      for (; k < cnt; k += G) s_mine[(base + k) / G] = s_list[j * kBuilderTiles + k];
    }
    // order these generic accesses of the A stages before the producer's
    // first TMA write into them
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
  }

  if (warp == 0) {
    // ---- TMA producer -------------------------------------------------------
    if (lane == 0) {
      uint32_t g = 0;
      for (int pos = cta, i = 0; pos < total && !*abort_flag; pos += G, ++i) {
        const int tile = tile_at(p, c, s_pref, s_mine, pos, i);
        for (int kb = 0; kb < c.kblocks; ++kb, ++g) {
          const int s = (int)(g % (uint32_t)c.stages);
          const uint32_t use = g / (uint32_t)c.stages;
          if (use > 0 && !mbar_wait(empty + s, (use - 1) & 1u, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(full + s, kABytes + (uint32_t)c.npad * kTileK * 2u);
          tma_load_2d(s_a + (size_t)s * kABytes, &tmap_w, kb * kTileK, tile * kTileRows, full + s);
          tma_load_2d(s_b + (size_t)s * c.npad * kTileK * 2, &tmap_h, kb * kTileK, 0, full + s);
        }
      }
      // Let every issued copy land before the CTA can exit: the stage ring is
      // fully consumed on the normal path; after an abort, wait for each
      // stage's last phase (bounded).
      if (*abort_flag) {
        const uint32_t issued = g;
        for (uint32_t k = issued > (uint32_t)c.stages ? issued - c.stages : 0; k < issued; ++k)
          mbar_wait(full + (k % (uint32_t)c.stages), (k / (uint32_t)c.stages) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ---------------------------------------------------------
    if (lane == 0) {
      uint32_t g = 0;
      int last_stage = -1;
      uint32_t last_use = 0;
      int i = 0;
      for (int pos = cta; pos < total && !*abort_flag; pos += G, ++i) {
        const int acc = i & ((1 << c.acc_shift) - 1);
        const uint32_t ause = (uint32_t)(i >> c.acc_shift);
        if (ause > 0 && !mbar_wait(tempty + acc, (ause - 1) & 1u, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after_sync();
        const uint32_t d = tmem_base + (uint32_t)(acc * c.npad);
        bool ok = true;
        for (int kb = 0; kb < c.kblocks; ++kb, ++g) {
          const int s = (int)(g % (uint32_t)c.stages);
          const uint32_t use = g / (uint32_t)c.stages;
          if (!mbar_wait(full + s, use & 1u, abort_flag)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint64_t ad = tc_desc_sw128(s_a + (size_t)s * kABytes);
          const uint64_t bd = tc_desc_sw128(s_b + (size_t)s * c.npad * kTileK * 2);
#pragma unroll
          for (int k = 0; k < kTileK / 16; ++k)
            tc_mma_f16(d, ad + 2ull * k, bd + 2ull * k, c.idesc, (kb | k) != 0);
          tc_commit(empty + s);  // stage s is free once these MMAs complete
          last_stage = s;
          last_use = use;
        }
        if (!ok) break;
        tc_commit(tfull + acc);  // accumulator `acc` is complete
      }
      // all tensor-core work of this CTA has finished once the last stage
      // commit has arrived
      if (last_stage >= 0) mbar_wait(empty + last_stage, last_use & 1u, nullptr);
    }
  } else {
    // ---- epilogue: warps 2..9; warp w reads TMEM lane quadrant w % 4 -------
    // The quadrant's two warps split the accumulator's columns: 16 each when
    // the batch pads to 32, else alternating 32-column units.
    const int ew = warp - 2;
    const int q = warp & 3;
    const int half = ew >> 2;
    constexpr bool narrow = kNarrow;
    const int nunits = narrow ? 1 : (c.npad / 32 - half + 1) / 2;
    if (!p.dense && p.logits) fill_inactive_tiles<T>(p, c.ntiles, cta, G, ew, lane);
    unsigned long long running[kMaxUnits];  // lane l: best key of the unit's request l
#pragma unroll
    for (int u = 0; u < kMaxUnits; ++u) running[u] = 0ull;
    const int ulane = narrow ? (lane & 15) : lane;  // request column a lane's mask word serves
    int i = 0;
    for (int pos = cta; pos < total; pos += G, ++i) {
      const int acc = i & ((1 << c.acc_shift) - 1);
      const uint32_t ause = (uint32_t)(i >> c.acc_shift);
      const int tile = tile_at(p, c, s_pref, s_mine, pos, i);
      const int row0 = tile * kTileRows + q * 32;
      const int word_idx = tile * 4 + q;  // mask word holding this warp's 32 rows
      // mask words first: their loads overlap the wait for the accumulator
      uint32_t words[kMaxUnits];
#pragma unroll
      for (int u = 0; u < kMaxUnits; ++u) {
        words[u] = 0u;
        const int b = unit_col(narrow, half, u) + ulane;
        if (u < nunits && b < B) {
          if (!p.mask) words[u] = 0xffffffffu;
          else if (word_idx < p.nw) words[u] = __ldg(p.mask + (int64_t)b * p.mask_stride + word_idx);
        }
      }
      const bool ok = mbar_wait(tfull + acc, ause & 1u, abort_flag);
      __syncwarp();
      if (!ok) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      tc_fence_after_sync();
      const int row = row0 + lane;
      const bool row_ok = row < V;
      const bool store = row_ok && p.logits != nullptr;
      const uint32_t tcol = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * c.npad);
      uint16_t* out = static_cast<uint16_t*>(p.logits) + row;
      if constexpr (narrow) {
        const int b0 = 16 * half;
        UnitSampler su{};
        if constexpr (kSample)
          su = UnitSampler{p.seeds + b0, s_skeys + b0, s_stats + b0, p.offset, p.inv_temp, p.vocab_offset + row};
        const uint32_t k = epilogue_unit<T, 16, kSample>(tcol + (uint32_t)b0, words[0], b0, B, row_ok, store,
                                                 out + (int64_t)b0 * p.logits_stride, p.logits_stride, lane, su);
        running[0] = merge_unit_key<T>(running[0], k, p.vocab_offset + row0);
      } else {
#pragma unroll
        for (int u = 0; u < kMaxUnits; ++u) {
          if (u < nunits) {
            const int b0 = unit_col(false, half, u);
            UnitSampler su{};
            if constexpr (kSample)
              su = UnitSampler{p.seeds + b0, s_skeys + b0, s_stats + b0, p.offset, p.inv_temp, p.vocab_offset + row};
            const uint32_t k = epilogue_unit<T, 32, kSample>(tcol + (uint32_t)b0, words[u], b0, B, row_ok, store,
                                                     out + (int64_t)b0 * p.logits_stride, p.logits_stride, lane, su);
            running[u] = merge_unit_key<T>(running[u], k, p.vocab_offset + row0);
          }
        }
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + acc);
    }
    if (want_top) {
#pragma unroll
      for (int u = 0; u < kMaxUnits; ++u) {
        const int b = unit_col(narrow, half, u) + lane;
        if (u < nunits && lane < (narrow ? 16 : 32) && b < B && running[u] != 0ull) atomicMax(&s_keys[b], running[u]);
      }
    }
  }

  // ---- teardown: TMEM free, error report, top-1 merge ---------------------
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, c.tmem_cols);
  }
  if (*abort_flag) {
    if (tid == 0 && p.error) atomicExch(p.error, 1);
    return;
  }
  // The workspace must be left zero-filled for the next call, whatever its
  // batch and vocabulary: clear the tile-list slots this CTA consumed (every
  // reader of them is in this CTA and past the barrier above); the last CTA
  // clears the per-builder-block counts, which every CTA read at set-up.
  if (!p.dense)
    for (int pos = cta + tid * G; pos < total; pos += G * kGemmThreads) p.tile_list[list_slot(c, s_pref, pos)] = 0;
  if (!want_top && p.dense && !kSample) return;
  bool did = false;
  if (want_top) {
    for (int b = tid; b < B; b += kGemmThreads) {
      const unsigned long long k = s_keys[b];
      if (k != 0ull) {
        atomicMax(p.keys + b, k);
        did = true;
      }
    }
  }
  if constexpr (kSample) {  // the CTA's sample keys and (max, sum) partials (request-major rows)
    for (int b = tid; b < B; b += kGemmThreads) {
      if (s_skeys[b] != 0ull) atomicMax(p.sample_keys + b, s_skeys[b]);
      p.stat_partials[(size_t)b * kMaxSlices + cta] = s_stats[b];
      did = true;
    }
  }
  if (did) __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int t = atomicAdd(p.ticket, 1u);
    s_misc[1] = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (s_misc[1]) {
    __threadfence();
    if (want_top) {
      bool ok = true;
      if (p.peers.world > 1) {  // merge across the ranks of a vocabulary-parallel group
        for (int b = tid; b < B; b += kGemmThreads) s_keys[b] = atomicExch(p.keys + b, 0ull);
        ok = peer_exchange_keys(p.peers, s_keys, B, reinterpret_cast<uint32_t*>(s_misc + 2), p.error);
      }
      for (int b = tid; b < B; b += kGemmThreads) {
        const unsigned long long k = p.peers.world > 1 ? s_keys[b] : atomicExch(p.keys + b, 0ull);
        store_top1(p.top_value, p.top_index, p.top_key, b, k, ok);
      }
    }
    if constexpr (kSample)
      sampler_finish(p.sample_keys, p.stat_partials, B, G, p.sample_index, p.sample_key, p.sample_lse);
    if (!p.dense)
      for (int j = tid; j < c.nbuild; j += kGemmThreads) p.tile_counts[j] = 0;
    if (tid == 0) atomicExch(p.ticket, 0u);
  }
}

// ---------------------------------------------------------------------------
// active-tile builder
// ---------------------------------------------------------------------------
constexpr int kBuilderThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kBuilderThreads) tile_builder_kernel(const BlockGemmParams p, int ntiles) {
  __shared__ uint32_t s_act[kBuilderTiles];
  const int tid = threadIdx.x;
  const int t0 = blockIdx.x * kBuilderTiles;
  const int V = p.vocab, nw = p.nw, B = p.batch;
  // The projection kernel may start its set-up now (programmatic dependent
  // launch): its CTAs fit beside these blocks, and its griddepcontrol.wait
  // still waits for this grid to finish and its writes to be visible.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tid < kBuilderTiles) s_act[tid] = 0u;
  __syncthreads();

  // thread (tile = tid % 32, group = tid / 32) ORs the 4 words of requests
  // group, group + 8, ... for its tile: loads are independent, one round trip.
  {
    const int lt = tid % kBuilderTiles, grp = tid / kBuilderTiles;
    const int groups = kBuilderThreads / kBuilderTiles;
    const int t = t0 + lt;
    uint32_t any = 0u;
    if (t < ntiles && t * 4 + 4 <= nw && (reinterpret_cast<uintptr_t>(p.mask) & 15) == 0 && p.mask_stride % 4 == 0) {
      // the tile's 4 words as one 16-byte load per request: a warp reads 512
      // contiguous bytes per request
#pragma unroll 4
      for (int b = grp; b < B; b += groups) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(p.mask + (int64_t)b * p.mask_stride + t * 4));
        any |= tail_clip(q.x, t * 4, V) | tail_clip(q.y, t * 4 + 1, V) | tail_clip(q.z, t * 4 + 2, V) |
               tail_clip(q.w, t * 4 + 3, V);
      }
    } else if (t < ntiles) {
#pragma unroll 4
      for (int b = grp; b < B; b += groups) {
        const uint32_t* row = p.mask + (int64_t)b * p.mask_stride;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int w = t * 4 + j;
          if (w < nw) any |= tail_clip(__ldg(row + w), w, V);
        }
      }
    }
    if (any) atomicOr(&s_act[lt], 1u);
  }
  __syncthreads();
  if (tid < 32) {
    const int t = t0 + tid;
    const bool valid = t < ntiles;
    const bool act = valid && s_act[tid] != 0u;
    const unsigned am = __ballot_sync(FULL_MASK, act);
    const unsigned below = (1u << tid) - 1u;
    if (act) p.tile_list[t0 + __popc(am & below)] = t;
    if (tid == 0) p.tile_counts[blockIdx.x] = __popc(am);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D K-major tensor map [rows, H] with a (64 x box_rows) box and 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, int bf16, uint64_t rows, uint64_t cols, uint64_t row_stride_elems,
              uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_stride_elems * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kTileK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int smem_optin(int dev) {
  int v = 0;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0)
    v = 227 * 1024;
  return v;
}

template <typename T>
cudaError_t launch_chunk(const BlockGemmParams& p, int dev, cudaStream_t stream) {
  GemmConfig c;
  c.npad = ((p.batch + 31) / 32) * 32;
  c.kblocks = (p.hidden_dim + kTileK - 1) / kTileK;
  c.ntiles = (p.vocab + kTileRows - 1) / kTileRows;
  c.nbuild = (c.ntiles + kBuilderTiles - 1) / kBuilderTiles;
  // 4 accumulators let the MMA run up to 3 tiles ahead of the epilogue; TMEM
  // holds 512 fp32 columns per SM
  c.acc_shift = c.npad <= 128 ? 2 : 1;
  uint32_t cols = 32;
  while (cols < ((uint32_t)c.npad << c.acc_shift)) cols <<= 1;
  c.tmem_cols = cols;
  c.idesc = tc_idesc_f16((uint32_t)c.npad, sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value);
  c.stage_list = 0;
  const size_t stage_bytes = kABytes + (size_t)c.npad * kTileK * 2;
  const size_t fixed = gemm_layout(c.npad, 0, c.nbuild).total + 1024 + 2048;
  c.stages = (int)std::min<size_t>(kMaxStages, ((size_t)smem_optin(dev) - fixed) / stage_bytes);
  if (c.stages < 2) return cudaErrorInvalidConfiguration;
  const GemmLayout L = gemm_layout(c.npad, c.stages, c.nbuild);
  const int G = num_sms(dev);
  // the whole list fits the A stages and each CTA's share fits s_mine
  c.stage_list = (size_t)c.ntiles * 4 <= (size_t)c.stages * kABytes && (c.ntiles + G - 1) / G <= kMaxMine;

  const int bf16 = std::is_same<T, __nv_bfloat16>::value ? 1 : 0;
  CUtensorMap tw, th;
  if (!make_map(&tw, p.weight, bf16, (uint64_t)p.vocab, (uint64_t)p.hidden_dim, (uint64_t)p.weight_stride, kTileRows) ||
      !make_map(&th, p.hidden, bf16, (uint64_t)p.batch, (uint64_t)p.hidden_dim, (uint64_t)p.hidden_stride,
                (uint32_t)c.npad))
    return cudaErrorInvalidValue;

  cudaError_t err;
  if (!p.dense) {
    tile_builder_kernel<T><<<c.nbuild, kBuilderThreads, 0, stream>>>(p, c.ntiles);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  }
  const bool sample = p.sample_index != nullptr;
  auto k = c.npad == 32 ? (sample ? tc_projection_kernel<T, true, true> : tc_projection_kernel<T, true, false>)
                        : (sample ? tc_projection_kernel<T, false, true> : tc_projection_kernel<T, false, false>);
  const size_t smem_bytes = L.total + 1024;
  if ((err = raise_smem_limit(reinterpret_cast<const void*>(k), smem_bytes, dev)) != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (p.dense || p.no_pdl) ? 0 : 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, tw, th, p, c);
}

template <typename T>
cudaError_t launch_typed(const BlockGemmParams& p0, cudaStream_t stream) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  // TMA needs 16-byte aligned bases and row pitches; otherwise the row-sparse
  // kernel computes the same outputs (every legal row, -inf elsewhere).
  const bool tma_ok = (p0.hidden_dim % 8 == 0) && ((reinterpret_cast<uintptr_t>(p0.weight) & 15) == 0) &&
                      (p0.weight_stride % 8 == 0) && ((reinterpret_cast<uintptr_t>(p0.hidden) & 15) == 0) &&
                      (p0.batch == 1 || p0.hidden_stride % 8 == 0);
  if (!tma_ok) {
    RowSparseParams r{};
    r.hidden = p0.hidden;
    r.hidden_stride = p0.hidden_stride;
    r.weight = p0.weight;
    r.weight_stride = p0.weight_stride;
    r.mask = p0.mask;
    r.mask_stride = p0.mask_stride;
    r.batch = p0.batch;
    r.vocab = p0.vocab;
    r.hidden_dim = p0.hidden_dim;
    r.nw = p0.nw;
    r.vocab_offset = p0.vocab_offset;
    r.logits = p0.logits;
    r.logits_stride = p0.logits_stride;
    r.top_value = p0.top_value;
    r.top_index = p0.top_index;
    r.top_key = p0.top_key;
    r.keys = p0.keys;
    r.ticket = p0.ticket;
    r.error = p0.error;
    r.peers = p0.peers;
    r.sample_index = p0.sample_index;
    r.sample_lse = p0.sample_lse;
    r.sample_key = p0.sample_key;
    r.seeds = p0.seeds;
    r.offset = p0.offset;
    r.inv_temp = p0.inv_temp;
    r.sample_keys = p0.sample_keys;
    r.stat_partials = p0.stat_partials;
    return launch_row_sparse(r, std::is_same<T, __nv_bfloat16>::value ? 1 : 0, stream);
  }
  // Batches above kMaxNpad run as consecutive chunks of requests.
  for (int b0 = 0; b0 < p0.batch; b0 += kMaxNpad) {
    BlockGemmParams p = p0;
    const int nb = std::min(kMaxNpad, p0.batch - b0);
    p.batch = nb;
    p.hidden = static_cast<const uint16_t*>(p0.hidden) + (int64_t)b0 * p0.hidden_stride;
    if (p0.mask) p.mask = p0.mask + (int64_t)b0 * p0.mask_stride;
    if (p0.logits) p.logits = static_cast<uint16_t*>(p0.logits) + (int64_t)b0 * p0.logits_stride;
    if (p0.top_value) p.top_value = p0.top_value + b0;
    if (p0.top_index) p.top_index = p0.top_index + b0;
    if (p0.top_key) p.top_key = p0.top_key + b0;
    p.keys = p0.keys + b0;
    p.peers.batch_base = p0.peers.batch_base + b0;
    if (p0.sample_index) {
      p.sample_index = p0.sample_index + b0;
      if (p0.sample_lse) p.sample_lse = p0.sample_lse + b0;
      if (p0.sample_key) p.sample_key = p0.sample_key + b0;
      p.seeds = p0.seeds + b0;
      p.sample_keys = p0.sample_keys + b0;
      p.stat_partials = p0.stat_partials + (size_t)b0 * kMaxSlices;
    }
    if ((err = launch_chunk<T>(p, dev, stream)) != cudaSuccess) return err;
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_block_gemm(const BlockGemmParams& p, int dtype, cudaStream_t stream) {
  if (dtype == 1) return launch_typed<__nv_bfloat16>(p, stream);
  return launch_typed<__half>(p, stream);
}

}  // namespace gsp
