// Cross-rank top-1 merge over NVLink peer memory, run by the last CTA of a
// projection kernel on every rank of a vocabulary-parallel group.
//
// Each rank's exchange buffer (layout in gsp_internal.h) is mapped into every
// other rank's process. For call number e (the buffer's epoch + 1) the last
// CTA of rank r
//   1. stores its per-request keys into slot [e & 1][r] of EVERY rank's buffer
//      (plain stores to peer memory), fences at system scope and raises flag r
//      of every rank's buffer to e (release, system scope);
//   2. waits, bounded, until each of its own flags has reached e (a flag may
//      already hold e + 1: the writer finished this call and started the next);
//   3. takes the MAX of the R keys per request and records e as its epoch.
// When every global token id is below 2^24 - 1 (x.tagged), steps 1-2 need no
// fence and no flag: bits 24..31 of a key are then always set (the low word is
// 0xffffffff - id), so they are replaced by the low 8 bits of e and each key
// travels as one self-tagged 8-byte store; the reader polls each slot until it
// carries tag e. The empty key (no legal token) travels as tag e alone.
// A rank can run at most one call ahead of the slowest peer (it cannot finish
// call e + 1 before every peer has written its e + 1 keys, which each peer does
// only after reading its call-e keys), so two key buffers suffice. All ranks
// must make the same sequence of calls. Only plain peer loads and stores are used.
#pragma once

#include <stdint.h>

#include "gsp_common.cuh"
#include "gsp_internal.h"

namespace gsp {

// Waits end after x.wait_ns of %globaltimer time; the poll count is capped as
// well (2^26 polls with a >= 32 ns back-off, over two seconds), so a wait ends
// even if the timer were not to advance.
constexpr uint32_t kPeerSpinLimit = 1u << 26;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

constexpr unsigned long long kTagMask = 0xFF000000ull;

__device__ __forceinline__ unsigned long long tag_key(unsigned long long k, uint32_t e) {
  return (k & ~kTagMask) | ((unsigned long long)(e & 0xFFu) << 24);
}
__device__ __forceinline__ bool tag_is(unsigned long long w, uint32_t e) {
  return ((w >> 24) & 0xFFu) == (e & 0xFFu);
}
__device__ __forceinline__ unsigned long long untag_key(unsigned long long w) {
  const unsigned long long k = w & ~kTagMask;
  return (k & 0xFFFFFFull) == 0ull ? 0ull : (k | kTagMask);  // low 24 bits 0: the empty key
}

__device__ __forceinline__ unsigned long long* peer_key_slot(const PeerExchange& x, int q, int parity, int src) {
  return reinterpret_cast<unsigned long long*>(x.buf[q] + kPeerKeysOffset) +
         ((size_t)parity * x.world + src) * x.max_batch + x.batch_base;
}

// Called by every thread of ONE CTA with the rank's merged keys in
// s_keys[0, batch); leaves the group's merged keys there and returns true.
// s_word is one word of shared memory. A wait that runs out sets *error (when
// given) to 3 and returns false on every thread: the keys are then not the
// group's, and the caller reports no top-1 for the call (its epoch is still
// recorded, so the host must re-synchronise the group's buffers before the
// next call).
__device__ __forceinline__ bool peer_exchange_keys(const PeerExchange& x, unsigned long long* s_keys, int batch,
                                                   uint32_t* s_word, int* error) {
  const int tid = threadIdx.x, nt = blockDim.x;
  unsigned char* self = x.buf[x.rank];
  uint32_t* epoch = reinterpret_cast<uint32_t*>(self);
  if (tid == 0) *s_word = *reinterpret_cast<volatile uint32_t*>(epoch) + 1u;
  __syncthreads();
  const uint32_t e = *s_word;
  const int par = (int)(e & 1u);
  bool late = false;
  if (x.tagged) {
    for (int i = tid; i < x.world * batch; i += nt) {
      const int q = i / batch, b = i - q * batch;
      st_relaxed_sys_u64(peer_key_slot(x, q, par, x.rank) + b, tag_key(s_keys[b], e));
    }
    for (int i = tid; i < x.world * batch; i += nt) {
      const int q = i / batch, b = i - q * batch;
      const unsigned long long* slot = peer_key_slot(x, x.rank, par, q) + b;
      bool ok = false;
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t it = 0; it < kPeerSpinLimit; ++it) {
        if (tag_is(ld_relaxed_sys_u64(slot), e)) {
          ok = true;
          break;
        }
        if ((int64_t)(globaltimer_ns() - t0) > x.wait_ns) break;
        __nanosleep(32);
      }
      if (!ok) {
        late = true;
        if (error) atomicExch(error, 3);
      }
    }
    const bool failed = __syncthreads_or(late);
    for (int b = tid; b < batch; b += nt) {
      unsigned long long k = 0ull;
      for (int q = 0; q < x.world; ++q) {
        const unsigned long long v = untag_key(ld_relaxed_sys_u64(peer_key_slot(x, x.rank, par, q) + b));
        k = v > k ? v : k;
      }
      s_keys[b] = k;
    }
    if (tid == 0) *reinterpret_cast<volatile uint32_t*>(epoch) = e;
    __syncthreads();
    return !failed;
  }
  for (int i = tid; i < x.world * batch; i += nt) {
    const int q = i / batch, b = i - q * batch;
    peer_key_slot(x, q, par, x.rank)[b] = s_keys[b];
  }
  if (tid < x.world * batch) __threadfence_system();  // only the threads that stored keys
  __syncthreads();
  if (tid < x.world) st_release_sys(reinterpret_cast<uint32_t*>(x.buf[tid] + 128 + 128 * x.rank), e);
  if (tid < x.world) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(self + 128 + 128 * tid);
    bool ok = false;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < kPeerSpinLimit; ++i) {
      if ((int32_t)(ld_acquire_sys(f) - e) >= 0) {
        ok = true;
        break;
      }
      if ((int64_t)(globaltimer_ns() - t0) > x.wait_ns) break;
      __nanosleep(64);
    }
    if (!ok) {
      late = true;
      if (error) atomicExch(error, 3);
    }
  }
  const bool failed = __syncthreads_or(late);
  for (int b = tid; b < batch; b += nt) {
    unsigned long long k = 0ull;
    for (int q = 0; q < x.world; ++q) {
      const unsigned long long v = ld_relaxed_sys_u64(peer_key_slot(x, x.rank, par, q) + b);
      k = v > k ? v : k;
    }
    s_keys[b] = k;
  }
  if (tid == 0) *reinterpret_cast<volatile uint32_t*>(epoch) = e;
  __syncthreads();
  return !failed;
}

// Writes request b's decoded top-1 from its merged key k. With ok false (a
// cross-rank wait ran out) no token is reported: index -1, value NaN, key
// INT64_MIN, which a caller tells apart from every real result.
__device__ __forceinline__ void store_top1(float* top_value, int64_t* top_index, int64_t* top_key, int b,
                                           unsigned long long k, bool ok) {
  if (top_value) top_value[b] = ok ? key_value(k) : __int_as_float(0x7fc00000);
  if (top_index) top_index[b] = ok ? key_index(k) : -1;
  if (top_key) top_key[b] = ok ? key_to_signed(k) : INT64_MIN;
}

}  // namespace gsp
