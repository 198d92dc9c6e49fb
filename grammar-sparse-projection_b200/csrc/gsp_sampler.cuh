// Fused grammar-conditioned sampler: the sampling contract and its device
// helpers.
//
// For request b with legal tokens L_b, rounded logits x_v (the values the
// materialised logits would hold), temperature T = 1 / inv_temp, seed k_b and
// step counter `offset`:
//
//   u_v  = ((philox4x32_10({v, offset_lo, offset_hi, 0}, {k_lo, k_hi}).x >> 8) + 0.5) * 2^-24
//   g_v  = -log(-log(u_v))                         (standard Gumbel noise)
//   s_v  = x_v * inv_temp + g_v                     (all in fp32)
//   sample_b = argmax_{v in L_b} s_v                (ties to the lowest id)
//   lse_b    = log sum_{v in L_b} exp(x_v * inv_temp)
//
// By the Gumbel-max property, sample_b is distributed exactly as softmax of
// x * inv_temp over the legal tokens; lse_b gives the sampled token's log
// probability, x * inv_temp - lse_b. u_v takes 2^24 values strictly inside
// (0, 1), each exact in fp32. v is the global token id (vocab_offset + row).
//
// Philox4x32-10 is the counter-based generator of Salmon, Moraes, Dror and
// Shaw, "Parallel random numbers: as easy as 1, 2, 3" (SC 2011): ten rounds
// of two 32x32 -> 64-bit multiplies with the published multipliers, the key
// bumped by the published Weyl constants between rounds.
#pragma once

#include <stdint.h>

#include "gsp_common.cuh"
#include "gsp_internal.h"

namespace gsp {

__host__ __device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;  // round multipliers
  constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;  // key schedule
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)kM0 * c[0], p1 = (uint64_t)kM1 * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    c[1] = (uint32_t)p1;
    c[3] = (uint32_t)p0;
    c[0] = n0;
    c[2] = n2;
    k0 += kW0;
    k1 += kW1;
  }
}

// Gumbel noise of token `v` for a request with key `seed` at step `offset`.
__device__ __forceinline__ float gumbel_noise(uint64_t seed, uint64_t offset, uint64_t v) {
  uint32_t c[4] = {(uint32_t)v, (uint32_t)offset, (uint32_t)(offset >> 32), 0u};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  const float u = ((float)(c[0] >> 8) + 0.5f) * 5.9604644775390625e-8f;  // 2^-24
  return -logf(-logf(u));
}

// (running max m, sum of exp(y - m)) packed as two floats: hi word m, lo word s.
// The empty pair is (-inf, 0).
__device__ __forceinline__ unsigned long long pack_stats(float m, float s) {
  return ((unsigned long long)__float_as_uint(m) << 32) | (unsigned long long)__float_as_uint(s);
}
__device__ __forceinline__ float stats_m(unsigned long long w) { return __uint_as_float((uint32_t)(w >> 32)); }
__device__ __forceinline__ float stats_s(unsigned long long w) { return __uint_as_float((uint32_t)w); }
__device__ __forceinline__ unsigned long long empty_stats() { return pack_stats(-INFINITY, 0.f); }

// Merge of two (m, s) pairs: max of the maxima, sums rescaled to it.
__device__ __forceinline__ void merge_stats(float& m, float& s, float m2, float s2) {
  if (s2 == 0.f) return;
  if (s == 0.f) {
    m = m2;
    s = s2;
    return;
  }
  const float mm = fmaxf(m, m2);
  s = s * __expf(m - mm) + s2 * __expf(m2 - mm);
  m = mm;
}

// The same noise through one out-of-line copy, for kernels that call it at many
// unrolled sites (the tensor-core epilogue's columns).
static __device__ __noinline__ float gumbel_noise_outlined(uint64_t seed, uint64_t offset, uint64_t v) {
  return gumbel_noise(seed, offset, v);
}

// Last CTA of a sampling launch of G CTAs: takes the per-request winning
// sample keys out of the workspace (re-zeroing them) into sample_index /
// sample_key, and merges the CTAs' (max, sum) partials (request-major rows of
// kMaxSlices) into sample_lse (re-zeroing them). The ids take one thread per
// request; the log-sum-exp a warp per request, its lanes loading the G partials
// (each load instruction coalesced) eight at a time, then merging across the
// warp with shuffles. All threads of the CTA call it.
__device__ __forceinline__ void sampler_finish(unsigned long long* sample_keys, unsigned long long* stat_partials,
                                               int B, int G, int64_t* sample_index, int64_t* sample_key,
                                               float* sample_lse) {
  constexpr int kChunkLoads = 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const unsigned long long k = atomicExch(sample_keys + b, 0ull);
    sample_index[b] = key_index(k);
    if (sample_key) sample_key[b] = key_to_signed(k);
  }
  for (int b = warp; b < B; b += nwarps) {
    float m = -INFINITY, sum = 0.f;
    for (int c0 = 0; c0 < G; c0 += 32 * kChunkLoads) {
      unsigned long long x[kChunkLoads];
#pragma unroll
      for (int k = 0; k < kChunkLoads; ++k) {
        const int c = c0 + lane + 32 * k;
        x[k] = c < G ? __ldcg(stat_partials + (size_t)b * kMaxSlices + c) : empty_stats();
      }
#pragma unroll
      for (int k = 0; k < kChunkLoads; ++k) {
        const int c = c0 + lane + 32 * k;
        if (c < G) stat_partials[(size_t)b * kMaxSlices + c] = 0ull;
        merge_stats(m, sum, stats_m(x[k]), stats_s(x[k]));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(FULL_MASK, m, o), s2 = __shfl_xor_sync(FULL_MASK, sum, o);
      merge_stats(m, sum, m2, s2);
    }
    if (lane == 0 && sample_lse) sample_lse[b] = sum > 0.f ? m + logf(sum) : -INFINITY;
  }
}

}  // namespace gsp
