// ssa_tcgen05.cuh -- device helpers for the tensor-core (tcgen05) kernels:
// mbarriers with bounded waits, TMA and bulk copies into shared memory,
// UMMA shared-memory and instruction descriptors, tcgen05.mma / commit, and
// TMEM loads. Shared by the candidate scan (ssa_select_tc.cu) and the
// tensor-core hash (ssa_hash_tc.cu).
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "ssa_internal.h"

namespace ssa {

// First error code a wait of this file's kernels recorded; 0 = none. Every
// file that includes this header has its own copy, read by tc_read_error;
// ssa_device_error reports the first nonzero one of all of them.
static __device__ int g_tc_error = 0;

static inline int tc_read_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
  }
  return v;
}

// 4-D bf16 tensor map {d, heads, rows, batch} with element strides
// {sh, sn, sb}; box {64, 1, 128, 1}, 128-byte swizzle, zero fill out of
// bounds. False when the driver entry point is missing or rejects the map.
bool tc_make_map(CUtensorMap* m, const void* base, int d, int heads, int rows, int batch, int64_t sh, int64_t sn,
                 int64_t sb);
bool tc_encode_available();
// 2-D bf16 tensor map {inner, outer} with a row pitch of `pitch` elements;
// box {64, 128}, 128-byte swizzle, zero fill out of bounds.
bool tc_make_map_2d(CUtensorMap* m, const void* base, int64_t inner, int64_t outer, int64_t pitch);

namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: `limit` polls (2^24 by default: a few seconds at most),
// then flag the error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int code, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try(bar, parity)) return true;
    if (*abort) return false;
    if (i > 2048) __nanosleep(64);
  }
  *abort = 1;
  atomicCAS(&g_tc_error, 0, code);
  return false;
}

// Warp-uniform version: every lane waits, and the warp proceeds only if all
// lanes saw the phase complete (so .sync.aligned TMEM loads never diverge).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort,
                                               int code, uint32_t limit) {
  const bool ok = mbar_wait(bar, parity, abort, code, limit);
  return __all_sync(0xffffffffu, ok);
}

// Bounded wait that ignores the abort flag: used to let TMA copies already
// issued land before the CTA exits.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < (1u << 24); ++i) {
    if (mbar_try(bar, parity)) return;
    if (i > 2048) __nanosleep(64);
  }
  atomicCAS(&g_tc_error, 0, 17);
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Tiled store shared -> global (bulk group of the issuing thread). The
// coordinates are never negative.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The issuing thread's bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// ... and have completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Makes this thread's shared-memory writes visible to the async proxy
// (tensor-core operands, TMA stores).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Plain bulk copy global -> shared (16-byte aligned addresses, size a
// multiple of 16), completing on the mbarrier's transaction count.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// K-major, SWIZZLE_128B operand descriptor (canonical layout: 8-row groups of
// 128-byte rows, 1024 bytes apart; LBO unused for this layout = 1).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both
// K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D (+)= A * B^T on the tensor cores, issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// One fp32 column of this thread's TMEM lane.
__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  return __uint_as_float(r);
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// a[j] for a dynamic j in [0, 32) without indexing the register array
// (which would move it to local memory): a 5-level select tree.
__device__ __forceinline__ float pick32(const float* a, int j) {
  float b16[16], b8[8], b4[4], b2[2];
#pragma unroll
  for (int i = 0; i < 16; ++i) b16[i] = (j & 16) ? a[i + 16] : a[i];
#pragma unroll
  for (int i = 0; i < 8; ++i) b8[i] = (j & 8) ? b16[i + 8] : b16[i];
#pragma unroll
  for (int i = 0; i < 4; ++i) b4[i] = (j & 4) ? b8[i + 4] : b8[i];
#pragma unroll
  for (int i = 0; i < 2; ++i) b2[i] = (j & 2) ? b4[i + 2] : b4[i];
  return (j & 1) ? b2[1] : b2[0];
}

}  // namespace tc
}  // namespace ssa
