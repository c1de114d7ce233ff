// ssa_common.cuh -- shared device helpers for the sm_100a sparse-attention kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ssa {

constexpr int kDtF32 = 0;
constexpr int kDtBF16 = 1;

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) {
  return __uint_as_float(bits16 << 16);
}

// fp32 -> bf16 round-to-nearest-even (the rounding torch's .to(bfloat16) uses);
// NaN is kept quiet.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

__device__ __forceinline__ float round_bf16(float f) {
  return bf16_bits_to_f32(f32_to_bf16_bits(f));
}

// Packed fp32 pairs (low element in the low word) and the sm_100 paired
// FMA, d = a * b + c on both halves.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  unsigned long long d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Philox4x32-10, the counter-based generator of Salmon, Moraes, Dror and
// Shaw, "Parallel random numbers: as easy as 1, 2, 3" (SC'11): ten rounds of
// two 32x32->64 multiplies and a Weyl-sequence key schedule.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
  constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u;  // round multipliers
  constexpr uint32_t kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;  // key increments
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(kM0, c.x), lo0 = kM0 * c.x;
    const uint32_t hi1 = __umulhi(kM1, c.z), lo1 = kM1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += kW0;
    k.y += kW1;
  }
  return c;
}

// Dropout keep decision of element e (row * Kn + slot): Philox word e % 4 of
// counter (e / 4, e >> 34, offset) under key seed, kept iff >= thresh.
__device__ __forceinline__ bool dropout_keep(unsigned long long e, unsigned long long seed,
                                             unsigned long long offset, uint32_t thresh) {
  const uint4 r = philox4x32_10(make_uint4((uint32_t)(e >> 2), (uint32_t)(e >> 34), (uint32_t)offset,
                                           (uint32_t)(offset >> 32)),
                                make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
  const uint32_t w = (e & 3) == 0 ? r.x : (e & 3) == 1 ? r.y : (e & 3) == 2 ? r.z : r.w;
  return w >= thresh;
}

// Four consecutive elements starting at element i of a row, widened to fp32.
// The caller guarantees 16-byte (fp32) / 8-byte (bf16) alignment of row + i.
template <int DT>
__device__ __forceinline__ float4 load4(const void* row, int i) {
  if constexpr (DT == kDtF32) {
    return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(row) + i));
  } else {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(row) + i));
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
  }
}

// Eight consecutive elements (16 B of bf16 or 32 B of fp32).
template <int DT>
__device__ __forceinline__ void load8(const void* row, int i, float* o) {
  if constexpr (DT == kDtF32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(row) + i);
    const float4 a = __ldg(p), b = __ldg(p + 1);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  } else {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(row) + i));
    o[0] = __uint_as_float(u.x << 16); o[1] = __uint_as_float(u.x & 0xffff0000u);
    o[2] = __uint_as_float(u.y << 16); o[3] = __uint_as_float(u.y & 0xffff0000u);
    o[4] = __uint_as_float(u.z << 16); o[5] = __uint_as_float(u.z & 0xffff0000u);
    o[6] = __uint_as_float(u.w << 16); o[7] = __uint_as_float(u.w & 0xffff0000u);
  }
}

template <int DT>
__device__ __forceinline__ float load1(const void* row, int i) {
  if constexpr (DT == kDtF32) return __ldg(static_cast<const float*>(row) + i);
  else return bf16_bits_to_f32(__ldg(static_cast<const uint16_t*>(row) + i));
}

template <int DT>
__device__ __forceinline__ void store1(void* row, int i, float v) {
  if constexpr (DT == kDtF32) static_cast<float*>(row)[i] = v;
  else static_cast<uint16_t*>(row)[i] = f32_to_bf16_bits(v);
}

template <int DT>
__device__ __forceinline__ const void* row_ptr(const void* base, int64_t elem_off) {
  if constexpr (DT == kDtF32) return static_cast<const float*>(base) + elem_off;
  else return static_cast<const uint16_t*>(base) + elem_off;
}

template <int DT>
__device__ __forceinline__ void* row_ptr_mut(void* base, int64_t elem_off) {
  if constexpr (DT == kDtF32) return static_cast<float*>(base) + elem_off;
  else return static_cast<uint16_t*>(base) + elem_off;
}

}  // namespace ssa
