// Shared device helpers for the grammar-conditioned LM-head kernels (sm_100a).
//
// Conventions shared by every kernel in this library:
//   * Grammar bitmask: int32 words, LSB-first; token v of request b is legal iff
//     bit (v % 32) of word mask[b * mask_stride + v / 32] is set (gsp/triton_runtime.py:33-35).
//     Bits at or beyond `vocab` in the last word are ignored (triton_runtime.py:30,35).
//   * Logits are accumulated in fp32 and rounded once to the input dtype
//     (triton_runtime.py:38,54,56). Illegal entries hold -inf.
//   * Greedy top-1 is reduced on the *rounded* output values, ties to the lowest
//     vocabulary index, i.e. exactly torch.argmax over the materialised logits.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

namespace gsp {

constexpr unsigned FULL_MASK = 0xffffffffu;

template <typename T>
struct DTypeTraits;

// Bits: the storage word of one element; kPerVec: elements per 16-byte vector.
template <>
struct DTypeTraits<__half> {
  using Bits = uint16_t;
  static constexpr int kPerVec = 8;
  static constexpr uint16_t kNegInfBits = 0xFC00u;
  static __device__ __forceinline__ float2 pair_to_float2(uint32_t v) {
    __half2 h;
    *reinterpret_cast<uint32_t*>(&h) = v;
    return __half22float2(h);
  }
  static __device__ __forceinline__ uint16_t round_bits(float f) {
    return __half_as_ushort(__float2half_rn(f));
  }
  static __device__ __forceinline__ float bits_to_float(uint16_t u) {
    return __half2float(__ushort_as_half(u));
  }
};

template <>
struct DTypeTraits<__nv_bfloat16> {
  using Bits = uint16_t;
  static constexpr int kPerVec = 8;
  static constexpr uint16_t kNegInfBits = 0xFF80u;
  static __device__ __forceinline__ float2 pair_to_float2(uint32_t v) {
    // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 word.
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  }
  static __device__ __forceinline__ uint16_t round_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
  static __device__ __forceinline__ float bits_to_float(uint16_t u) {
    return __uint_as_float(static_cast<uint32_t>(u) << 16);
  }
};

// fp32 inputs (the reference's wrappers accept them: the output dtype is the
// hidden dtype, gsp/triton_runtime.py:111): products accumulate in fp32 and the
// output is the fp32 sum itself.
template <>
struct DTypeTraits<float> {
  using Bits = uint32_t;
  static constexpr int kPerVec = 4;
  static constexpr uint32_t kNegInfBits = 0xFF800000u;
  static __device__ __forceinline__ uint32_t round_bits(float f) { return __float_as_uint(f); }
  static __device__ __forceinline__ float bits_to_float(uint32_t u) { return __uint_as_float(u); }
};

// Order-preserving map float -> uint32 (total order on non-NaN values).
// +0 and -0 are canonicalised so that they compare equal, as in torch.argmax.
__device__ __forceinline__ uint32_t ordered_bits(float f) {
  if (f == 0.0f) f = 0.0f;
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float from_ordered_bits(uint32_t o) {
  uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
  return __uint_as_float(u);
}

// Packed top-1 key: larger value wins, then the lower global index wins.
// Key 0 means "no legal token seen".
__device__ __forceinline__ unsigned long long top1_key(float rounded_value,
                                                       uint64_t global_index) {
  return (static_cast<unsigned long long>(ordered_bits(rounded_value)) << 32) |
         static_cast<unsigned long long>(0xffffffffu - static_cast<uint32_t>(global_index));
}

__device__ __forceinline__ float key_value(unsigned long long key) {
  if (key == 0ull) return -__int_as_float(0x7f800000);  // -inf
  return from_ordered_bits(static_cast<uint32_t>(key >> 32));
}

__device__ __forceinline__ int64_t key_index(unsigned long long key) {
  if (key == 0ull) return 0;  // torch.argmax of an all -inf row is 0
  return static_cast<int64_t>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffull));
}

// Keys exported across the C-ABI are signed-orderable int64 so that a plain
// integer MAX all-reduce (NCCL/gloo) merges vocabulary shards.
__device__ __forceinline__ int64_t key_to_signed(unsigned long long key) {
  return static_cast<int64_t>(key ^ 0x8000000000000000ull);
}
__device__ __forceinline__ unsigned long long key_from_signed(int64_t k) {
  return static_cast<unsigned long long>(k) ^ 0x8000000000000000ull;
}

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int lane_mask) {
  uint32_t lo = static_cast<uint32_t>(v), hi = static_cast<uint32_t>(v >> 32);
  lo = __shfl_xor_sync(FULL_MASK, lo, lane_mask);
  hi = __shfl_xor_sync(FULL_MASK, hi, lane_mask);
  return (static_cast<unsigned long long>(hi) << 32) | lo;
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long other = shfl_xor_u64(v, o);
    v = other > v ? other : v;
  }
  return v;
}

// Streaming 16-byte load of weight rows: read once, keep out of L1.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Legal-bit word for (request row pointer, word index), with bits >= vocab cleared.
__device__ __forceinline__ uint32_t tail_clip(uint32_t word, int word_index, int vocab) {
  int rows_left = vocab - word_index * 32;
  if (rows_left >= 32) return word;
  if (rows_left <= 0) return 0u;
  return word & ((1u << rows_left) - 1u);
}

template <typename T>
__device__ __forceinline__ float dot8(uint4 w, uint4 h, float acc) {
  float2 a, b;
  a = DTypeTraits<T>::pair_to_float2(w.x); b = DTypeTraits<T>::pair_to_float2(h.x);
  acc = fmaf(a.x, b.x, acc); acc = fmaf(a.y, b.y, acc);
  a = DTypeTraits<T>::pair_to_float2(w.y); b = DTypeTraits<T>::pair_to_float2(h.y);
  acc = fmaf(a.x, b.x, acc); acc = fmaf(a.y, b.y, acc);
  a = DTypeTraits<T>::pair_to_float2(w.z); b = DTypeTraits<T>::pair_to_float2(h.z);
  acc = fmaf(a.x, b.x, acc); acc = fmaf(a.y, b.y, acc);
  a = DTypeTraits<T>::pair_to_float2(w.w); b = DTypeTraits<T>::pair_to_float2(h.w);
  acc = fmaf(a.x, b.x, acc); acc = fmaf(a.y, b.y, acc);
  return acc;
}

// fp32 dot of one 16-byte vector of weights with one of hidden states
// (8 half-precision or 4 fp32 elements), accumulated into acc in element order.
template <typename T>
__device__ __forceinline__ float dot_vec(uint4 w, uint4 h, float acc) {
  if constexpr (std::is_same<T, float>::value) {
    acc = fmaf(__uint_as_float(w.x), __uint_as_float(h.x), acc);
    acc = fmaf(__uint_as_float(w.y), __uint_as_float(h.y), acc);
    acc = fmaf(__uint_as_float(w.z), __uint_as_float(h.z), acc);
    acc = fmaf(__uint_as_float(w.w), __uint_as_float(h.w), acc);
    return acc;
  } else {
    return dot8<T>(w, h, acc);
  }
}

}  // namespace gsp
