// ssa_select_tc.cu -- tensor-core (tcgen05) candidate scan for bf16 inputs.
//
// Same selection as k_select_merge (ssa_graph.cu), but the q.k scores come
// from 5th-generation tensor cores instead of per-candidate FMA loops:
//
//   warp 4 (one lane)  TMA: the CTA's 128-row q tile once, then 128-key tiles
//                      of K into a 2-stage ring (SWIZZLE_128B, K-major).
//   warp 5             allocates 256 TMEM columns; one lane issues
//                      tcgen05.mma (M=128, N=128, K=16, bf16 in, fp32 out)
//                      for S = Q K^T into one of two TMEM accumulators, and
//                      tcgen05.commit releases the K stage and publishes S.
//   warps 0-3          thread per query row (TMEM lane = row): tcgen05.ld the
//                      row's 128 scores, OR the row's bucket masks for the
//                      tile, and push candidates that beat the heap minimum
//                      into the row's shared-memory top-A heap; then the
//                      special-key replay and the merge, as in ssa_graph.cu.
//
// bf16 x bf16 products are exact in fp32, so tensor-core scores differ from
// the reference's fp32 sums only by accumulation order (rescore ties).
// Every wait on an mbarrier is bounded: on timeout the kernel records an
// error code (ssa_device_error) and the pipeline drains and returns.
#include <cuda.h>

#include "ssa_common.cuh"
#include "ssa_internal.h"
#include "ssa_select_common.cuh"

namespace ssa {

__device__ int g_ssa_device_error = 0;

namespace tc {

constexpr int ROWS = 128;   // query rows per CTA (MMA M, TMEM lanes)
constexpr int NKEY = 128;   // keys per tile (MMA N)
constexpr int STAGES = 2;   // K-tile ring
constexpr int THREADS = 192;

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

// Bounded wait: about a few seconds at most, then flag the error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int code) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (mbar_try(bar, parity)) return true;
    if (*abort) return false;
    if (i > 64) __nanosleep(256);
  }
  *abort = 1;
  atomicCAS(&g_ssa_device_error, 0, code);
  return false;
}

// Warp-uniform version: every lane waits, and the warp proceeds only if all
// lanes saw the phase complete (so .sync.aligned TMEM loads never diverge).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort,
                                               int code) {
  const bool ok = mbar_wait(bar, parity, abort, code);
  return __all_sync(0xffffffffu, ok);
}

// Bounded wait that ignores the abort flag: used to let TMA copies already
// issued land before the CTA exits.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (mbar_try(bar, parity)) return;
    if (i > 64) __nanosleep(256);
  }
  atomicCAS(&g_ssa_device_error, 0, 17);
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// K-major, SWIZZLE_128B operand descriptor (canonical layout: 8-row groups of
// 128-byte rows, 1024 bytes apart; LBO unused for this layout = 1).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both
// K-major, M = 128, N = NKEY.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NKEY >> 3) << 17) |
                            ((uint32_t)(ROWS >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc));
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

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct SmemPlan {
  uint32_t q, k, heap_s, heap_k, tids, gs, bars, tmem_slot, total;
};

__host__ __device__ inline SmemPlan plan(int D, int A, int NT, int G, int key_bytes) {
  SmemPlan p;
  uint32_t off = 0;
  auto take = [&](uint32_t bytes, uint32_t align) {
    off = (off + align - 1) / align * align;
    const uint32_t o = off;
    off += bytes;
    return o;
  };
  const uint32_t atoms = (uint32_t)D / 64;
  p.q = take(atoms * ROWS * 128, 1024);
  p.k = take(STAGES * atoms * NKEY * 128, 1024);
  p.heap_s = take((uint32_t)A * ROWS * 4, 16);
  p.heap_k = take((uint32_t)A * ROWS * key_bytes, 16);
  p.tids = take((uint32_t)NT * ROWS * 2, 16);
  p.gs = take((uint32_t)(G + 1) * 4, 16);
  p.bars = take(16 * 8, 8);
  p.tmem_slot = take(16, 16);
  p.total = off + 1024;  // slack to realign the dynamic base to 1024 bytes
  return p;
}

}  // namespace tc

template <int D, typename KT>
__global__ void __launch_bounds__(tc::THREADS, 1)
    k_select_tc(GraphDev g, int mode, const __grid_constant__ CUtensorMap qmap,
                const __grid_constant__ CUtensorMap kmap) {
  using namespace tc;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int ATOMS = D / 64;
  const SmemPlan sp = plan(D, g.A, g.NT, g.G, (int)sizeof(KT));
  unsigned char* qs = smem + sp.q;
  unsigned char* ks = smem + sp.k;
  float* hs = reinterpret_cast<float*>(smem + sp.heap_s);
  KT* hk = reinterpret_cast<KT*>(smem + sp.heap_k);
  uint16_t* tids = reinterpret_cast<uint16_t*>(smem + sp.tids);
  int32_t* gs = reinterpret_cast<int32_t*>(smem + sp.gs);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + sp.bars);
  uint64_t* kfull = bars;           // [2] K stage loaded (TMA tx)
  uint64_t* kempty = bars + 2;      // [2] K stage consumed (MMA commit)
  uint64_t* sfull = bars + 4;       // [2] S accumulator ready (MMA commit)
  uint64_t* sempty = bars + 6;      // [2] S accumulator drained (4 epilogue warps)
  uint64_t* qfull = bars + 8;       // q tile loaded
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 9);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + sp.tmem_slot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / g.H, h = bh % g.H;
  const int gk = h / g.rep;
  const int bg = b * g.n_kv + gk;
  const int n0 = blockIdx.x * ROWS;
  const int n_hi = min(g.N, n0 + ROWS) - 1;
  const int nkt = g.causal ? min((g.M + NKEY - 1) / NKEY, (n_hi >> 7) + 1) : (g.M + NKEY - 1) / NKEY;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(kfull + i, 1);
      mbar_init(kempty + i, 1);
      mbar_init(sfull + i, 1);
      mbar_init(sempty + i, 4);
    }
    mbar_init(qfull, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // sorted unique globals for the merge
    int ng = 0;
    for (int i = 0; i < g.G; ++i) {
      const int v = g.glob[i];
      bool dup = false;
      for (int z = 0; z < ng; ++z) dup |= gs[z] == v;
      if (dup) continue;
      int j = ng - 1;
      while (j >= 0 && gs[j] > v) { gs[j + 1] = gs[j]; --j; }
      gs[j + 1] = v;
      ++ng;
    }
    gs[g.G] = ng;
  }
  if (warp == 5) {  // TMEM: 2 accumulators x NKEY fp32 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(2 * NKEY));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_expect_tx(qfull, ATOMS * ROWS * 128);
      for (int a = 0; a < ATOMS; ++a)
        tma_load_4d(qs + a * ROWS * 128, &qmap, qfull, a * 64, h, n0, b);
      int issued = 0;
      for (int kt = 0; kt < nkt; ++kt) {
        const int s = kt & 1;
        if (!mbar_wait(kempty + s, ((kt >> 1) & 1) ^ 1, abort_flag, 11)) break;
        mbar_expect_tx(kfull + s, ATOMS * NKEY * 128);
        for (int a = 0; a < ATOMS; ++a)
          tma_load_4d(ks + (s * ATOMS + a) * NKEY * 128, &kmap, kfull + s, a * 64, gk, kt * NKEY, b);
        issued = kt + 1;
      }
      // Do not leave while copies are in flight: the last two issued stages
      // (and the q tile) must have landed before the CTA's shared memory goes.
      mbar_drain(qfull, 0);
      for (int kt = max(0, issued - 2); kt < issued; ++kt) mbar_drain(kfull + (kt & 1), (kt >> 1) & 1);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && mbar_wait(qfull, 0, abort_flag, 13)) {
      const uint32_t qa = smem_u32(qs);
      for (int kt = 0; kt < nkt; ++kt) {
        const int s = kt & 1;
        if (!mbar_wait(kfull + s, (kt >> 1) & 1, abort_flag, 14)) break;
        if (!mbar_wait(sempty + s, ((kt >> 1) & 1) ^ 1, abort_flag, 15)) break;
        tc_fence_after();
        const uint32_t ka = smem_u32(ks + s * ATOMS * NKEY * 128);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (ROWS * 128) + (kk & 3) * 32;
          const uint32_t offk = (kk >> 2) * (NKEY * 128) + (kk & 3) * 32;
          umma_bf16(tmem + s * NKEY, umma_desc(qa + off), umma_desc(ka + offk), kk > 0);
        }
        umma_commit(kempty + s);
        umma_commit(sfull + s);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int t = threadIdx.x;  // row within the tile; TMEM lane
    const int n = n0 + t;
    const bool act = n < g.N;
    bool any_empty = false;
    if (act) {
      float q[D];
      const void* qrow = row_ptr<kDtBF16>(g.q, b * g.q_sb + h * g.q_sh + (int64_t)n * g.q_sn);
#pragma unroll
      for (int i = 0; i < D; i += 4) {
        const float4 x = load4<kDtBF16>(qrow, i);
        q[i] = x.x; q[i + 1] = x.y; q[i + 2] = x.z; q[i + 3] = x.w;
      }
      any_empty = hash_row_ids<D>(g, q, bg, tids, ROWS, t);
    }
    RowHeap<KT> heap{hs, hk, ROWS, t};
    int cnt = 0;
    float thr = -INFINITY;
    const unsigned long long* bmg = g.bmap + (int64_t)bg * g.Wpad * g.R * g.NB;
    for (int kt = 0; kt < nkt; ++kt) {
      const int s = kt & 1;
      if (!mbar_wait_warp(sfull + s, (kt >> 1) & 1, abort_flag, 16)) break;
      tc_fence_after();
      float sc[NKEY];
      const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + s * NKEY;
#pragma unroll
      for (int c = 0; c < NKEY / 32; ++c) tmem_ld32(ta + c * 32, sc + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sempty + s);
      if (!act) continue;
      const int key0 = kt * NKEY;
      unsigned long long w[2];
#pragma unroll
      for (int hw = 0; hw < 2; ++hw) {
        const unsigned long long* bm = bmg + (int64_t)(2 * kt + hw) * g.R * g.NB;
        unsigned long long x = 0ull;
        for (int tt = 0; tt < g.NT; ++tt) x |= __ldg(bm + (tt / (1 + g.Te)) * g.NB + tids[tt * ROWS + t]);
        x &= ~__ldg(g.pmask + (int64_t)bg * g.Wpad + 2 * kt + hw);
        if (g.causal) {
          const int lim = n - (key0 + 64 * hw);
          if (lim <= 0) x = 0ull;
          else if (lim < 64) x &= (1ull << lim) - 1ull;
        }
        w[hw] = x;
      }
#pragma unroll
      for (int hw = 0; hw < 2; ++hw) {
        const unsigned long long x = w[hw];
        if (!x) continue;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float v = sc[hw * 64 + j];
          if (((x >> j) & 1ull) && v > thr) {
            if (cnt < g.A) {
              heap.set(cnt, v, key0 + hw * 64 + j);
              if (++cnt == g.A) {
                heap.heapify_score(g.A);
                thr = heap.sc(0);
              }
            } else {
              heap.sift_score(0, g.A, v, key0 + hw * 64 + j);
              thr = heap.sc(0);
            }
          }
        }
      }
    }
    if (act && !*abort_flag) finish_row<kDtBF16, D, KT>(g, mode, heap, cnt, tids, ROWS, t, gs, bh, b, h,
                                                        gk, bg, n, any_empty);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * NKEY));
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 4-D bf16 map {d, heads, rows, batch} with byte strides {sh, sn, sb}; box
// {64, 1, 128, 1}, 128-byte swizzle, zero fill out of bounds.
static bool make_map(CUtensorMap* m, const void* base, int d, int heads, int rows, int batch,
                     int64_t sh, int64_t sn, int64_t sb) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)heads, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)sh * 2, (cuuint64_t)sn * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool select_tc_supported(const GraphDev& g) {
  if (g.dtype != kDtBF16 || (g.d != 64 && g.d != 128)) return false;
  // TMA: 16-byte aligned base and strides
  auto al = [](int64_t s) { return (s * 2) % 16 == 0; };
  if (!al(g.q_sh) || !al(g.q_sn) || !al(g.q_sb) || !al(g.k_sh) || !al(g.k_sm) || !al(g.k_sb)) return false;
  if ((reinterpret_cast<uintptr_t>(g.q) % 16) || (reinterpret_cast<uintptr_t>(g.k) % 16)) return false;
  const tc::SmemPlan sp = tc::plan(g.d, g.A, g.NT, g.G, g.M <= 65536 ? 2 : 4);
  if (sp.total > 227 * 1024) return false;
  return encode_fn() != nullptr;
}

template <int D, typename KT>
static cudaError_t launch_tc_t(const GraphDev& g, int mode, cudaStream_t st) {
  CUtensorMap qmap, kmap;
  // q (B, H, N, d): dims {d, H, N, B}; k (B, n_kv, M, d): dims {d, n_kv, M, B}
  if (!make_map(&qmap, g.q, g.d, g.H, g.N, g.B, g.q_sh, g.q_sn, g.q_sb)) return cudaErrorInvalidValue;
  if (!make_map(&kmap, g.k, g.d, g.n_kv, g.M, g.B, g.k_sh, g.k_sm, g.k_sb)) return cudaErrorInvalidValue;
  const tc::SmemPlan sp = tc::plan(D, g.A, g.NT, g.G, (int)sizeof(KT));
  auto fn = k_select_tc<D, KT>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sp.total);
  if (e != cudaSuccess) return e;
  dim3 grid((g.N + tc::ROWS - 1) / tc::ROWS, g.B * g.H);
  fn<<<grid, tc::THREADS, sp.total, st>>>(g, mode, qmap, kmap);
  return cudaGetLastError();
}

cudaError_t launch_select_tc(const GraphDev& g, int mode, cudaStream_t st) {
  const bool k16 = g.M <= 65536;
  if (g.d == 64) return k16 ? launch_tc_t<64, uint16_t>(g, mode, st) : launch_tc_t<64, uint32_t>(g, mode, st);
  return k16 ? launch_tc_t<128, uint16_t>(g, mode, st) : launch_tc_t<128, uint32_t>(g, mode, st);
}

int read_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_ssa_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_ssa_device_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace ssa
