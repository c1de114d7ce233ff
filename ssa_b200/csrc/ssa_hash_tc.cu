// ssa_hash_tc.cu -- tensor-core (tcgen05) LSH hash of bf16 keys and queries.
//
// The hash of a row x is, per round r and hyperplane j, the sign of the fp32
// projection x . P[r][j] (sparse_attention.py:588-591), and for queries the
// multi-probe ids flip the planes with the smallest |projection| (:599-646).
// The FMA kernels (k_hash_keys, k_hash_queries) compute every projection in
// one fixed fp32 order; this file computes the same projections on the
// tensor cores and falls back to that fp32 order only where the tensor-core
// value could decide differently:
//
//   * every fp32 hyperplane element is split into three bf16 pieces
//     (hi + mid + lo, exact to about 2^-27 relative), so x . P is three
//     bf16 GEMMs with fp32 accumulation, D = X [hi mid lo]^T, and bf16 x
//     bf16 products are exact;
//   * the tensor-core value v and the fp32-order value v' of a projection
//     differ by less than eps = c * |x|_2 * max_j |P[r][j]|_2 (c = 2^-14 by
//     default: about eight times a worst-case bound on both summation errors
//     for the head dims served, 64 and 128). A round whose every |v| > eps
//     -- and, with probes, whose Te + 1 smallest |v| are more than 2 eps
//     apart -- has the same sign bits and probe order as the fp32 order.
//     Every other (row, round) is recomputed in the fp32 order from the row
//     in global memory (warp-cooperative, four lanes per item), bit-identical
//     to the FMA kernels. So the ids equal the FMA kernels' everywhere.
//
// k_hash_tc: persistent CTAs (one per SM; two for head dim 64 when only two
// epilogue groups fit), 128-row tiles of one (batch, head) slice, round-robin
// over the CTAs:
//
//   TMA warp (one lane)  bulk-copies the hyperplane pieces once (an image in
//                        the UMMA SWIZZLE_128B K-major layout that
//                        k_hash_planes writes), then TMA-loads 128-row tiles
//                        into a 2-4 stage ring.
//   MMA warp             allocates TMEM (one accumulator per epilogue group,
//                        8 or 16 columns per round) and issues the 3 * d / 16
//                        MMAs of a tile (M = 128, N = 8 R or 16 R, K = 16).
//   NG epilogue groups   four warps each, taking tiles in turn; thread per row
//                        (TMEM lane = row): row norm from the staged tile, ids
//                        and certification per round, then the outputs --
//                        queries: qids per (round, probe) slot and qempty;
//                        keys: kcode, the member-mask block and pmax (as
//                        k_hash_keys). Uncertified (row, round) items go to
//                        the CTA's own queue segment, which its epilogue
//                        warps recompute after the CTA's last tile.
//
// k_proj_hash (further below) is the fused QKV projection whose epilogue
// runs the same per-row hashing on its freshly rounded q / k tiles.
//
// Every wait on an mbarrier is bounded (GraphDev::wait_limit); a group
// decides together (barrier vote) to stop when one of its waits ran out.
#include <cuda.h>
#include <cuda_bf16.h>

#include "ssa_common.cuh"
#include "ssa_internal.h"
#include "ssa_select_common.cuh"
#include "ssa_tcgen05.cuh"

namespace ssa {

// (row, round) items recomputed in the fp32 order since the last read.
static __device__ unsigned long long g_hash_recomputed = 0ull;

namespace htc {

constexpr int ROWS = 128;      // rows per tile (MMA M, TMEM lanes)
// Hash kernel: NG epilogue groups of four warps, then the TMA and MMA warps.
__host__ __device__ constexpr int hash_threads(int NG) { return 32 * (4 * NG + 2); }
constexpr int kPieces = 3;     // bf16 pieces of an fp32 hyperplane element
constexpr int kMaxR = 16;

// TMEM columns (and B rows) per round: the p <= 12 planes, zero padded to 8
// or 16; N = rounds * that, rounded up to a multiple of 16 (<= 256).
__host__ __device__ inline int round_cols(int p) { return p <= 8 ? 8 : 16; }
__host__ __device__ inline int n_cols(int R, int p) { return (round_cols(p) * R + 15) / 16 * 16; }

struct Plan {
  uint32_t pl, a, pn, blk, bars, tmem_slot, total;
  int stages, np, tmem_cols;
  bool blk_on;  // keys: the tile's member-mask block is built in shared memory
};

// Keys: a 128-key tile owns one (round, bucket) block of member masks,
// R * NB * 16 bytes; built in shared memory (then stored whole) when at most
// this size, else set with global atomics.
constexpr uint32_t kBlkMax = 8 * 1024;

__host__ __device__ inline uint32_t planes_bytes(int D, int R, int p) {
  return (uint32_t)kPieces * (uint32_t)(D / 64) * (uint32_t)n_cols(R, p) * 128u;
}

// Epilogue groups of the hash kernel: four (one CTA per SM) when their
// accumulators fit TMEM, else two (two CTAs per SM where they fit).
__host__ __device__ inline int hash_groups(const GraphDev& g) { return 4 * n_cols(g.R, g.p) <= 512 ? 4 : 2; }

__host__ __device__ inline Plan plan_stages(int D, const GraphDev& g, bool keys, int stages, int NG) {
  Plan p;
  uint32_t off = 0;
  auto take = [&](uint32_t bytes, uint32_t align) {
    off = (off + align - 1) / align * align;
    const uint32_t o = off;
    off += bytes;
    return o;
  };
  p.np = n_cols(g.R, g.p);
  p.pl = take(planes_bytes(D, g.R, g.p), 1024);
  p.a = take((uint32_t)stages * (uint32_t)(D / 64) * ROWS * 128, 1024);
  p.pn = take(kMaxR * 4 + 16, 16);                                    // [R] max_j |P[r][j]|_2, queue count
  const uint32_t blk = (uint32_t)g.R * (uint32_t)g.NB * 16u;
  p.blk_on = keys && blk <= kBlkMax;
  p.blk = take(p.blk_on ? (uint32_t)NG * blk : 0u, 16);                // [group][R][NB] 4 x u32
  p.bars = take(24 * 8, 8);
  p.tmem_slot = take(16, 16);
  p.total = off + 1024;  // the base is rounded up to 1024 bytes in the kernel
  p.stages = stages;
  int cols = 32;
  while (cols < NG * p.np) cols <<= 1;
  p.tmem_cols = cols;
  return p;
}

// Four groups: the deepest ring (4 .. 2 stages) that fits. Two groups: the
// deepest that keeps two CTAs per SM (shared memory and TMEM), else one.
__host__ __device__ inline Plan plan(int D, const GraphDev& g, bool keys, int NG) {
  if (NG == 2)
    for (int st = 4; st >= 2; --st) {
      const Plan p = plan_stages(D, g, keys, st, NG);
      if (p.total <= 113 * 1024 && p.tmem_cols <= 256) return p;
    }
  for (int st = 4; st > 2; --st) {
    const Plan p = plan_stages(D, g, keys, st, NG);
    if (p.total <= 227 * 1024) return p;
  }
  return plan_stages(D, g, keys, 2, NG);
}

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Waits for this thread's outstanding TMEM loads; the empty asm statements
// then redefine v[0..N), so nothing reads those registers before the wait.
template <int N>
__device__ __forceinline__ void tmem_wait_regs(float* v) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+f"(v[i]));
}

// Named-barrier vote over the 128 threads of an epilogue group: true if any
// thread passes `pred`.
__device__ __forceinline__ bool group_any(bool pred, int bar_id) {
  uint32_t any;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(any)
      : "r"(pred ? 1u : 0u), "r"(bar_id)
      : "memory");
  return any != 0;
}

__device__ __forceinline__ void group_sync(int bar_id) {
  asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
}

}  // namespace htc

// ---------------------------------------------------------------------------
// Hyperplane pieces in the B-operand layout, and the hyperplane norms
// ---------------------------------------------------------------------------
// Element t of B row n = RC r + j (hyperplane j of round r, RC =
// round_cols(p); rows j >= p and n >= RC R are zero) for piece c lives in the
// K-block t / 64 of that piece: byte ((c * KB + t / 64) * NP + n) * 128 +
// (chunk ^ (n % 8)) * 16 + (t % 8) * 2, chunk = (t % 64) / 8 (UMMA
// SWIZZLE_128B, K-major: 8-row groups 1024 bytes apart). The last R * p
// warps of the grid write pnorm[r * p + j] = |P[r][j]|_2 (rounded up).
__global__ void __launch_bounds__(256) k_hash_planes(const float* __restrict__ rp, int R, int max_p, int p, int d,
                                                     int D, int img_blocks, uint16_t* __restrict__ img,
                                                     float* __restrict__ pnorm) {
  const int KB = D / 64, RC = htc::round_cols(p), NP = htc::n_cols(R, p);
  if ((int)blockIdx.x >= img_blocks) {
    const int w = ((int)blockIdx.x - img_blocks) * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (w >= R * p) return;
    const float* pl = rp + ((int64_t)(w / p) * max_p + (w % p)) * d;
    float s = 0.f;
    for (int t = lane; t < d; t += 32) s = fmaf(pl[t], pl[t], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    // a relative 2^-12 margin covers the rounding of this sum and sqrt
    if (lane == 0) pnorm[w] = sqrtf(s) * (1.f + 1.f / 4096.f);
    return;
  }
  const int64_t total = (int64_t)htc::kPieces * KB * NP * 64;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int tt = (int)(i % 64);
  int64_t rest = i / 64;
  const int n = (int)(rest % NP);
  rest /= NP;
  const int kb = (int)(rest % KB);
  const int c = (int)(rest / KB);
  const int r = n / RC, j = n % RC, t = kb * 64 + tt;
  float x = 0.f;
  if (r < R && j < p && t < d) x = __ldg(rp + ((int64_t)r * max_p + j) * d + t);
  const __nv_bfloat16 hi = __float2bfloat16_rn(x);
  const float r1 = x - __bfloat162float(hi);
  const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(mid);
  const __nv_bfloat16 lo = __float2bfloat16_rn(r2);
  const __nv_bfloat16 v = c == 0 ? hi : (c == 1 ? mid : lo);
  const int64_t byte = ((int64_t)(c * KB + kb) * NP + n) * 128 + ((((tt >> 3) ^ (n & 7)) << 4) | ((tt & 7) << 1));
  img[byte >> 1] = __bfloat16_as_ushort(v);
}

// ---------------------------------------------------------------------------
// Ids of one row from its tensor-core projections (TMEM lane = row)
// ---------------------------------------------------------------------------
struct HashRow {
  const float* s_pn;       // [R] max_j |P[r][j]|_2 (shared memory)
  float xn;                // |x|_2 of the row (rounded up)
  bool act;                // a real row (the tile may run past the slice)
  uint32_t rowid;          // queries: B*H*N row; keys: bg * M + key
  int bg, n, r0, lane, wq; // kv slice, row within it, tile start, lane, warp of the group
  uint4* blk;              // keys: the tile's member-mask block (shared), if blk_on
  bool blk_on;
  bool with_empty;         // queries: OR of the certified slots' empty buckets
  float* dump;             // testing: this row's projections, or null
  uint32_t* gq;            // queue of flagged (row << 4 | round) items, and its counter
  unsigned int* gcount;
};

template <int D, bool KEYS>
__device__ void fixup_items(const GraphDev& g, const uint32_t* q, unsigned int count, int64_t gw, int64_t nw);

// Projection columns in batches of BW (TMEM lane = row; round r at columns
// RC r .. RC r + p - 1 of ta). Per round: sign bits, certification (every
// |v| > eps, and with probes the Te + 1 smallest |v| 2 eps apart), probe ids;
// certified rounds write their outputs (queries: qids; keys: kcode, the
// member masks, pmax), the others go to the fixup queue. `v` holds the first
// batch already requested when `preloaded`. Returns whether a certified
// slot's bucket is empty (queries, with_empty).
template <bool KEYS, int RC, int BW>
__device__ __forceinline__ bool hash_rows(const GraphDev& g, const HashRow& c, uint32_t ta, int NP, float (&v)[BW],
                                          bool preloaded) {
  using namespace tc;
  using namespace htc;
  const int Te = KEYS ? 0 : g.Te;
  const int64_t total = (int64_t)g.B * g.H * g.N;
  bool empty = false;
  auto round_ids = [&](const float* vr, int r) {
    const float eps = g.hash_eps * c.xn * c.s_pn[r];
    uint32_t id = 0;
    bool bad = false;
    float av[RC];
#pragma unroll
    for (int j = 0; j < RC; ++j) {
      if (j < g.p) {
        id |= (vr[j] > 0.f ? 1u : 0u) << j;  // proj > 0, strict (:589)
        av[j] = fabsf(vr[j]);
        bad |= !(av[j] > eps);
        if (c.dump) c.dump[r * g.p + j] = vr[j];
      } else {
        av[j] = INFINITY;
      }
    }
    uint32_t pid = 0;  // probe t's plane in bits 4t .. 4t+3
    if (!KEYS && Te > 0 && !bad) {
      // probes flip the planes of the Te smallest |proj| (ties: lower
      // plane); certified when the Te + 1 smallest are 2 eps apart
      uint32_t used = 0;
      float prev = 0.f;
      for (int tt = 0; tt <= Te; ++tt) {
        int best = -1;
        float bmag = INFINITY;
#pragma unroll
        for (int j = 0; j < RC; ++j)
          if (j < g.p && !((used >> j) & 1u) && (best < 0 || av[j] < bmag)) {
            best = j;
            bmag = av[j];
          }
        if (best < 0) break;
        if (tt > 0 && !(bmag - prev > 2.f * eps)) bad = true;
        used |= 1u << best;
        prev = bmag;
        if (tt < Te) pid |= (uint32_t)best << (4 * tt);
      }
    }
    if (c.act && bad) c.gq[atomicAdd(c.gcount, 1u)] = (c.rowid << 4) | (uint32_t)r;
    const bool cert = c.act && !bad;
    if constexpr (KEYS) {
      // as k_hash_keys: 32 consecutive keys per warp (a quarter of the
      // tile's 128-bit member masks), one mask per bucket present
      const unsigned cmask = __ballot_sync(0xffffffffu, cert);
      if (cert) {
        g.kcode[((int64_t)c.bg * g.R + r) * g.M + c.n] = (uint16_t)id;
        const unsigned peers = __match_any_sync(cmask, id);
        if (c.lane == __ffs(peers) - 1) {
          if (c.blk_on) {
            reinterpret_cast<uint32_t*>(c.blk)[(r * g.NB + (int)id) * 4 + c.wq] = peers;
          } else {
            const int wbase = c.r0 + c.wq * 32;
            atomicOr(&g.bmap[bmap_idx(g, c.bg, wbase >> 6, r, (int)id)], (unsigned long long)peers << (wbase & 63));
          }
        }
        // perm[M-1] of the stable sort = largest key of the highest bucket
        const uint32_t mx = __reduce_max_sync(cmask, (id << 20) | (uint32_t)c.n);
        if (c.lane == __ffs(cmask) - 1) atomicMax(&g.pmax[c.bg * g.R + r], mx);
      }
    } else if (cert) {
      const int s0 = r * (1 + Te);
      const uint32_t base = (uint32_t)(r * g.NB);
      const int32_t* bs = g.bsize + ((int64_t)c.bg * g.R + r) * g.NB;
      g.qids[(int64_t)s0 * total + c.rowid] = (uint16_t)(base + id);
      if (c.with_empty) empty |= __ldg(bs + id) == 0;
      for (int tt = 0; tt < Te; ++tt) {
        const uint32_t pid_t = id ^ (1u << ((pid >> (4 * tt)) & 15u));
        g.qids[(int64_t)(s0 + 1 + tt) * total + c.rowid] = (uint16_t)(base + pid_t);
        if (c.with_empty) empty |= __ldg(bs + pid_t) == 0;
      }
    }
  };
#pragma unroll 1
  for (int cb = 0; cb < NP; cb += BW) {
    if (cb > 0 || !preloaded) {
#pragma unroll
      for (int q = 0; q < BW / 16; ++q)
        if (cb + 16 * q < NP) tmem_ld16(ta + cb + 16 * q, v + 16 * q);
    }
    tmem_wait_regs<BW>(v);
#pragma unroll
    for (int rr = 0; rr < BW / RC; ++rr) {
      const int r = cb / RC + rr;
      if (r < g.R) round_ids(v + rr * RC, r);
    }
  }
  return empty;
}

// Stores a tile's member-mask block (it owns the block) and clears the
// shared copy; the group's 128 threads, between two group barriers.
__device__ __forceinline__ void store_mask_block(const GraphDev& g, uint4* blk, int bg, int r0, int t,
                                                 int bar_id) {
  const int nblk = g.R * g.NB;
  htc::group_sync(bar_id);
  uint4* gb = reinterpret_cast<uint4*>(g.bmap + bmap_idx(g, bg, r0 >> 6, 0, 0));
  for (int e = t; e < nblk; e += htc::ROWS) {
    gb[e] = blk[e];
    blk[e] = make_uint4(0u, 0u, 0u, 0u);
  }
  htc::group_sync(bar_id);
}

// ---------------------------------------------------------------------------
// The hash kernel
// ---------------------------------------------------------------------------
// KEYS: rows are the keys of (batch, kv head) slices (M each); else the
// queries of (batch, head) slices (N each).
template <int D, bool KEYS, int RC, int NG>
__global__ void __launch_bounds__(htc::hash_threads(NG), NG == 2 ? 2 : 1)
    k_hash_tc(GraphDev g, const __grid_constant__ CUtensorMap xmap) {
  using namespace tc;
  using namespace htc;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int KB = D / 64;
  const Plan sp = plan(D, g, KEYS, NG);
  constexpr int WTMA = 4 * NG, WMMA = 4 * NG + 1;  // producer and MMA warps
  const int NS = sp.stages, NP = sp.np;
  const uint32_t idesc = idesc_bf16(ROWS, NP);
  unsigned char* pls = smem + sp.pl;
  unsigned char* as = smem + sp.a;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + sp.bars);
  uint64_t* sfull = bars;          // [NS] row tile loaded (TMA tx)
  uint64_t* sfree = bars + 4;      // [NS] row tile read (the epilogue group's 4 warps)
  uint64_t* afull = bars + 8;      // [NG] projections ready (MMA commit)
  uint64_t* afree = bars + 12;     // [NG] projections read (the group's 4 warps)
  uint64_t* pfull = bars + 16;     // hyperplane pieces loaded
  uint64_t* mma_done = bars + 17;  // every MMA issued has completed
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 18);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + sp.tmem_slot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int L = KEYS ? g.M : g.N;             // rows per slice
  const int heads = KEYS ? g.n_kv : g.H;
  const int tps = (L + ROWS - 1) / ROWS;      // tiles per slice
  const int64_t ntiles = (int64_t)g.B * heads * tps;
  const int ntl = blockIdx.x < ntiles ? (int)((ntiles - 1 - blockIdx.x) / gridDim.x) + 1 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(sfull + i, 1);
      mbar_init(sfree + i, 4);
    }
    for (int i = 0; i < NG; ++i) {
      mbar_init(afull + i, 1);
      mbar_init(afree + i, 4);
    }
    mbar_init(pfull, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == WMMA) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(sp.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == WTMA) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && ntl > 0) {
      const uint32_t pbytes = planes_bytes(D, g.R, g.p);
      mbar_expect_tx(pfull, pbytes);
      bulk_load(pls, g.hpl, pbytes, pfull);
      int issued = 0;
      for (int i = 0; i < ntl; ++i) {
        const int64_t T = blockIdx.x + (int64_t)i * gridDim.x;
        const int slice = (int)(T / tps), r0 = (int)(T % tps) * ROWS;
        const int b = slice / heads, h = slice % heads;
        const int s = i % NS;
        if (!mbar_wait(sfree + s, ((i / NS) & 1) ^ 1, abort_flag, 21, g.wait_limit)) break;
        mbar_expect_tx(sfull + s, KB * ROWS * 128);
        for (int a = 0; a < KB; ++a) tma_load_4d(as + (s * KB + a) * ROWS * 128, &xmap, sfull + s, a * 64, h, r0, b);
        issued = i + 1;
      }
      mbar_drain(pfull, 0);
      for (int i = max(0, issued - NS); i < issued; ++i) mbar_drain(sfull + i % NS, (i / NS) & 1);
    }
  } else if (warp == WMMA) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && ntl > 0 && mbar_wait(pfull, 0, abort_flag, 22, g.wait_limit)) {
      const uint32_t pa = smem_u32(pls);
      int issued_mma = 0;
      for (int i = 0; i < ntl; ++i) {
        const int s = i % NS, ab = i % NG;
        if (!mbar_wait(sfull + s, (i / NS) & 1, abort_flag, 23, g.wait_limit)) break;
        if (!mbar_wait(afree + ab, ((i / NG) & 1) ^ 1, abort_flag, 24, g.wait_limit)) break;
        tc_fence_after();
        const uint32_t xa = smem_u32(as + s * KB * ROWS * 128);
#pragma unroll
        for (int c = 0; c < kPieces; ++c)
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t offa = (kk >> 2) * (ROWS * 128) + (kk & 3) * 32;
            const uint32_t offb = (uint32_t)(c * KB + (kk >> 2)) * (uint32_t)NP * 128u + (kk & 3) * 32;
            umma_bf16(tmem + ab * NP, umma_desc(xa + offa), umma_desc(pa + offb), idesc, (c | kk) != 0);
          }
        umma_commit(afull + ab);
        issued_mma = i + 1;
      }
      if (issued_mma) {
        umma_commit(mma_done);
        mbar_drain(mma_done, 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int grp = warp >> 2, wq = warp & 3;
    const int t = wq * 32 + lane;
    const int bar_id = 1 + grp;
    float* s_pn = reinterpret_cast<float*>(smem + sp.pn);
    const int nblk = g.R * g.NB;  // entries of a key tile's mask block
    uint4* blk = reinterpret_cast<uint4*>(smem + sp.blk) + grp * nblk;
    const bool blk_on = KEYS && sp.blk_on;  // the group shares the block: group barriers
    if (blk_on)
      for (int e = t; e < nblk; e += ROWS) blk[e] = make_uint4(0u, 0u, 0u, 0u);
    if (threadIdx.x < g.R) {  // per round, max_j |P[r][j]|_2
      float m = 0.f;
      for (int j = 0; j < g.p; ++j) m = fmaxf(m, __ldg(g.pnorm + threadIdx.x * g.p + j));
      s_pn[threadIdx.x] = m;
    }
    // Flagged (row, round) items: this CTA's own segment of the queue (at most
    // its tiles' rows x R items), recomputed by the epilogue after its tiles.
    unsigned int* qcount = reinterpret_cast<unsigned int*>(s_pn + kMaxR);
    const int64_t seg_cap = ((ntiles + gridDim.x - 1) / gridDim.x) * (int64_t)ROWS * g.R;
    uint32_t* qseg = (KEYS ? g.hq_keys : g.hq_rows) + (int64_t)blockIdx.x * seg_cap;
    if (threadIdx.x == 0) *qcount = 0u;
    asm volatile("bar.sync 5, %0;" ::"r"(NG * 128) : "memory");  // every group
    for (int i = grp; i < ntl; i += NG) {
      const int64_t T = blockIdx.x + (int64_t)i * gridDim.x;
      const int slice = (int)(T / tps), r0 = (int)(T % tps) * ROWS;
      const int b = slice / heads, h = slice % heads;
      const int bg = KEYS ? slice : b * g.n_kv + h / g.rep;
      const int n = r0 + t;
      const bool act = n < L;
      const int s = i % NS, ab = grp;
      // The tile's load (sfull, long complete: the MMA waited on it) makes
      // its shared-memory rows visible to this thread for the norm below.
      const bool ok = mbar_wait_warp(afull + ab, (i / NG) & 1, abort_flag, 25, g.wait_limit) &&
                      mbar_wait_warp(sfull + s, (i / NS) & 1, abort_flag, 26, g.wait_limit);
      if (blk_on ? group_any(!ok, bar_id) : !ok) break;
      tc_fence_after();
      const uint32_t ta = tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(ab * NP);
      // Projection columns in batches of BW; the first batch is read while
      // the row norm is computed.
      constexpr int BW = 32;  // registers: two CTAs per SM
      float v[BW];
#pragma unroll
      for (int q = 0; q < BW / 16; ++q)
        if (16 * q < NP) tmem_ld16(ta + 16 * q, v + 16 * q);
      // |x|_2 of this row from the staged tile (chunks visited in swizzled
      // order so that eight consecutive rows hit eight bank groups).
      float nrm2 = 0.f;
      {
        const unsigned char* rowp = as + (size_t)s * KB * ROWS * 128 + (size_t)t * 128;
#pragma unroll
        for (int a = 0; a < KB; ++a)
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 u4 = *reinterpret_cast<const uint4*>(rowp + a * ROWS * 128 + ((c ^ (t & 7)) << 4));
            const uint32_t w[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float lo = __uint_as_float(w[e] << 16), hi = __uint_as_float(w[e] & 0xFFFF0000u);
              nrm2 = fmaf(lo, lo, nrm2);
              nrm2 = fmaf(hi, hi, nrm2);
            }
          }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(sfree + s);
      const float xn = sqrtf(nrm2) * (1.f + 1.f / 4096.f);  // covers this sum's rounding
      HashRow hr;
      hr.s_pn = s_pn;
      hr.xn = xn;
      hr.act = act;
      hr.rowid = (uint32_t)((int64_t)slice * L + n);  // queries: B*H*N row; keys: bg * M + key
      hr.bg = bg;
      hr.n = n;
      hr.r0 = r0;
      hr.lane = lane;
      hr.wq = wq;
      hr.blk = blk;
      hr.blk_on = blk_on;
      hr.with_empty = true;
      hr.dump = (!KEYS && g.hash_dump && act) ? g.hash_dump + (int64_t)hr.rowid * g.R * g.p : nullptr;
      hr.gq = qseg;
      hr.gcount = qcount;
      const bool empty = hash_rows<KEYS, RC, BW>(g, hr, ta, NP, v, true);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(afree + ab);
      if (!KEYS && act) g.qempty[hr.rowid] = empty ? 1 : 0;  // the recompute below adds the flagged rounds
      if (blk_on) store_mask_block(g, blk, bg, r0, t, bar_id);
    }
    // The flagged items of this CTA's tiles (whose mask blocks it has
    // stored), eight per warp pass in the fp32 order of the FMA kernels.
    asm volatile("bar.sync 5, %0;" ::"r"(NG * 128) : "memory");
    const unsigned int nq = *qcount;
    if (!*abort_flag) fixup_items<D, KEYS>(g, qseg, nq, warp, NG * 4);
    if (threadIdx.x == 0 && nq) atomicAdd(&g_hash_recomputed, (unsigned long long)nq);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == WMMA) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(sp.tmem_cols));
  }
}

// ---------------------------------------------------------------------------
// Fused QKV projection + hash
// ---------------------------------------------------------------------------
// out = x W^T for W = [Wq; Wk; Wv] (the projections feeding the graph build,
// sparse_attention.py:1484-1486), bf16 with fp32 accumulation, in 128 x 256
// tiles, persistent CTAs taking tiles column-fastest (a row block of x stays
// in L2 while W streams from L2):
//
//   warp 4 (one lane)  TMA: the hyperplane pieces once, then 64-wide K slices
//                      of the x (128 rows) and W (256 rows) tiles into a ring.
//   warp 5             tcgen05.mma 128 x 256 x 16 into one of two TMEM
//                      accumulators (256 columns each); commits free ring
//                      slots and publish finished tiles.
//   warps 0-3          thread per row, head by head: the head's columns
//                      rounded to bf16 into a staging tile (SWIZZLE_128B,
//                      K-major: the TMA-store source and the hash MMA's A
//                      operand), one TMA store, and for a q or k head the
//                      hash MMA -- issued by thread 0 into the head's
//                      just-drained accumulator columns -- then hash_rows:
//                      query slots, or key codes / member masks / pad keys.
//                      qempty is left to the graph build (it needs the bucket
//                      sizes of every key).
// The epilogue of tile i overlaps the mainloop of tile i + 1.
namespace prj {
constexpr int TN = 256;        // tile columns (MMA N)
constexpr int THREADS = 192;   // warps 0-3 epilogue, 4 TMA, 5 MMA
constexpr uint32_t kStage = (128 + TN) * 128;  // x 128 x 64 + W 256 x 64 bf16
struct Plan {
  uint32_t pl, ring, stg, pn, bars, tmem_slot, total;
  int stages, np;
};
__host__ __device__ inline Plan plan(int D, const GraphDev& g) {
  Plan p;
  uint32_t off = 0;
  auto take = [&](uint32_t bytes, uint32_t align) {
    off = (off + align - 1) / align * align;
    const uint32_t o = off;
    off += bytes;
    return o;
  };
  p.np = htc::n_cols(g.R, g.p);
  p.pl = take(htc::planes_bytes(D, g.R, g.p), 1024);
  p.stg = take((uint32_t)htc::ROWS * D * 2, 1024);  // one head: D / 64 atoms of 128 x 64
  const uint32_t tail = htc::kMaxR * 4 + 24 * 8 + 16 + 1024 + 64;
  int st = 4;
  while (st > 2 && ((off + 1023) / 1024 * 1024) + (uint32_t)st * kStage + tail > 227u * 1024u) --st;
  p.stages = st;
  p.ring = take((uint32_t)st * kStage, 1024);
  p.pn = take(htc::kMaxR * 4, 16);
  p.bars = take(24 * 8, 8);
  p.tmem_slot = take(16, 16);
  p.total = off + 1024;
  return p;
}
}  // namespace prj

template <int D, int RC>
__global__ void __launch_bounds__(prj::THREADS, 1)
    k_proj_hash(GraphDev g, ProjDev pd, const __grid_constant__ CUtensorMap xmap,
                const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap omap) {
  using namespace tc;
  using namespace htc;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int KB = D / 64;
  const prj::Plan sp = prj::plan(D, g);
  const int NS = sp.stages, NP = sp.np;
  const uint32_t idesc_g = idesc_bf16(ROWS, prj::TN);
  const uint32_t idesc_h = idesc_bf16(ROWS, NP);
  unsigned char* pls = smem + sp.pl;
  unsigned char* ring = smem + sp.ring;
  unsigned char* stg = smem + sp.stg;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + sp.bars);
  uint64_t* sfull = bars;          // [NS] K slice loaded (TMA tx)
  uint64_t* sfree = bars + 4;      // [NS] K slice consumed (MMA commit)
  uint64_t* afull = bars + 8;      // [2] tile accumulator ready
  uint64_t* afree = bars + 10;     // [2] tile accumulator drained (the 4 epilogue warps)
  uint64_t* hfull = bars + 12;     // hash projections ready (thread 0's commit)
  uint64_t* pfull = bars + 13;     // hyperplane pieces loaded
  uint64_t* mma_done = bars + 14;  // every mainloop MMA has completed
  uint64_t* hdone = bars + 15;     // every hash MMA has completed
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 16);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + sp.tmem_slot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncol = (pd.n_out + prj::TN - 1) / prj::TN;
  const int nheads = g.H + 2 * g.n_kv;
  const int64_t ntiles = (int64_t)(pd.rows / ROWS) * ncol;
  const int ntl = blockIdx.x < ntiles ? (int)((ntiles - 1 - blockIdx.x) / gridDim.x) + 1 : 0;
  const int nk = pd.dm / 64;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(sfull + i, 1);
      mbar_init(sfree + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(afull + i, 1);
      mbar_init(afree + i, 4);
    }
    mbar_init(hfull, 1);
    mbar_init(pfull, 1);
    mbar_init(mma_done, 1);
    mbar_init(hdone, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 5) {  // two 256-column accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && ntl > 0) {
      const uint32_t pbytes = planes_bytes(D, g.R, g.p);
      mbar_expect_tx(pfull, pbytes);
      bulk_load(pls, g.hpl, pbytes, pfull);
      int64_t c = 0, issued = 0;
      bool stop = false;
      for (int i = 0; i < ntl && !stop; ++i) {
        const int64_t T = blockIdx.x + (int64_t)i * gridDim.x;
        const int row0 = (int)(T / ncol) * ROWS, col0 = (int)(T % ncol) * prj::TN;
        for (int kc = 0; kc < nk; ++kc, ++c) {
          const int s = (int)(c % NS);
          if (!mbar_wait(sfree + s, (uint32_t)((c / NS) & 1) ^ 1u, abort_flag, 31, g.wait_limit)) {
            stop = true;
            break;
          }
          unsigned char* st = ring + (size_t)s * prj::kStage;
          mbar_expect_tx(sfull + s, prj::kStage);
          tma_load_2d(st, &xmap, sfull + s, kc * 64, row0);
          tma_load_2d(st + 16384, &wmap, sfull + s, kc * 64, col0);  // W rows col0 .. +127
          tma_load_2d(st + 32768, &wmap, sfull + s, kc * 64, col0 + 128);  // +128 .. +255 (zero past n_out)
          issued = c + 1;
        }
      }
      mbar_drain(pfull, 0);
      for (int64_t q = issued - NS > 0 ? issued - NS : 0; q < issued; ++q)
        mbar_drain(sfull + q % NS, (uint32_t)((q / NS) & 1));
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && ntl > 0) {
      int64_t c = 0;
      int issued_mma = 0;
      bool stop = false;
      for (int i = 0; i < ntl && !stop; ++i) {
        const int ab = i & 1;
        if (!mbar_wait(afree + ab, ((i >> 1) & 1) ^ 1, abort_flag, 32, g.wait_limit)) break;
        tc_fence_after();
        for (int kc = 0; kc < nk; ++kc, ++c) {
          const int s = (int)(c % NS);
          if (!mbar_wait(sfull + s, (uint32_t)((c / NS) & 1), abort_flag, 33, g.wait_limit)) {
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t xa = smem_u32(ring + (size_t)s * prj::kStage), wa = xa + 16384;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + ab * prj::TN, umma_desc(xa + kk * 32), umma_desc(wa + kk * 32), idesc_g,
                      (kc | kk) != 0);
          umma_commit(sfree + s);
          issued_mma = 1;
        }
        if (!stop) umma_commit(afull + ab);
      }
      if (issued_mma) {
        umma_commit(mma_done);
        mbar_drain(mma_done, 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int t = threadIdx.x;  // row of the tile (TMEM lane)
    const int bar_id = 1;
    float* s_pn = reinterpret_cast<float*>(smem + sp.pn);
    if (t < g.R) {
      float m = 0.f;
      for (int j = 0; j < g.p; ++j) m = fmaxf(m, __ldg(g.pnorm + t * g.p + j));
      s_pn[t] = m;
    }
    const bool planes_ok = ntl == 0 || mbar_wait_warp(pfull, 0, abort_flag, 34, g.wait_limit);
    group_sync(bar_id);
    const uint32_t lrow = (uint32_t)(warp * 32) << 16;
    int nh = 0;  // hash MMAs issued (hfull phase)
    bool stored = false;
    for (int i = 0; i < ntl && planes_ok; ++i) {
      const int64_t T = blockIdx.x + (int64_t)i * gridDim.x;
      const int row0 = (int)(T / ncol) * ROWS, col0 = (int)(T % ncol) * prj::TN;
      const int ab = i & 1;
      const bool ok = mbar_wait_warp(afull + ab, (i >> 1) & 1, abort_flag, 35, g.wait_limit);
      if (group_any(!ok, bar_id)) break;
      tc_fence_after();
      const uint32_t acc = tmem + lrow + (uint32_t)(ab * prj::TN);
      const int b = row0 / g.N, n0 = row0 % g.N;  // N % 128 == 0: one batch element per tile
      bool aborted = false;
      for (int hh = 0; hh < prj::TN / D; ++hh) {
        const int hd = (col0 + hh * D) / D;
        if (hd >= nheads) break;  // past the last head (uniform)
        // The previous TMA store has read the staging tile.
        if (t == 0 && stored) bulk_wait_read();
        group_sync(bar_id);
        // Head columns -> bf16 (round to nearest) -> staging (row t: atom a at
        // a * 16 KB, 16-byte chunk c at (c ^ (t & 7)) * 16), and the squared
        // norm of the row's bf16 values.
        float nrm2 = 0.f;
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) {
          float f[32];
          tmem_ld32(acc + hh * D + cc * 32, f);
          tmem_wait_ld();
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
            w[e] = *reinterpret_cast<const uint32_t*>(&b2);
            const float lo = __uint_as_float(w[e] << 16), hi = __uint_as_float(w[e] & 0xFFFF0000u);
            nrm2 = fmaf(lo, lo, fmaf(hi, hi, nrm2));
          }
          unsigned char* rowp = stg + (cc >> 1) * (ROWS * 128) + t * 128;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int ch = (cc & 1) * 4 + u;
            *reinterpret_cast<uint4*>(rowp + ((ch ^ (t & 7)) << 4)) =
                make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
          }
        }
        tc_fence_before();
        fence_async_smem();
        group_sync(bar_id);
        if (t == 0) {
#pragma unroll
          for (int a = 0; a < KB; ++a) tma_store_2d(&omap, stg + a * ROWS * 128, col0 + hh * D + a * 64, row0);
          bulk_commit();
          stored = true;
        }
        if (hd >= g.H + g.n_kv) continue;  // a v head: no hash
        const bool key = hd >= g.H;
        // Hash MMA into the head's drained accumulator columns (NP <= D).
        const uint32_t hcol = tmem + (uint32_t)(ab * prj::TN + hh * D);
        if (t == 0) {
          tc_fence_after();
          const uint32_t xa = smem_u32(stg), pa = smem_u32(pls);
#pragma unroll
          for (int c = 0; c < kPieces; ++c)
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t offa = (kk >> 2) * (ROWS * 128) + (kk & 3) * 32;
              const uint32_t offb = (uint32_t)(c * KB + (kk >> 2)) * (uint32_t)NP * 128u + (kk & 3) * 32;
              umma_bf16(hcol, umma_desc(xa + offa), umma_desc(pa + offb), idesc_h, (c | kk) != 0);
            }
          umma_commit(hfull);
        }
        const bool hok = mbar_wait_warp(hfull, nh & 1, abort_flag, 36, g.wait_limit);
        ++nh;
        if (group_any(!hok, bar_id)) {
          aborted = true;
          break;
        }
        tc_fence_after();
        HashRow hr;
        hr.s_pn = s_pn;
        hr.xn = sqrtf(nrm2) * (1.f + 1.f / 4096.f);
        hr.act = true;
        hr.n = n0 + t;
        hr.r0 = n0;
        hr.lane = lane;
        hr.wq = warp;
        hr.blk = nullptr;
        hr.blk_on = false;
        hr.with_empty = false;
        hr.dump = nullptr;
        hr.gq = key ? g.hq_keys : g.hq_rows;
        hr.gcount = g.hq_count + (key ? 0 : 1);
        float v[32];
        if (key) {
          hr.bg = b * g.n_kv + (hd - g.H);
          hr.rowid = (uint32_t)((int64_t)hr.bg * g.M + hr.n);
          hash_rows<true, RC, 32>(g, hr, hcol + lrow, NP, v, false);
        } else {
          hr.bg = b * g.n_kv + hd / g.rep;
          hr.rowid = (uint32_t)(((int64_t)b * g.H + hd) * g.N + hr.n);
          hash_rows<false, RC, 32>(g, hr, hcol + lrow, NP, v, false);
        }
        tc_fence_before();
      }
      if (aborted) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(afree + ab);  // every column of the accumulator has been read
    }
    if (t == 0) {
      if (stored) bulk_wait_all();
      if (nh) {  // the hash MMAs have completed before TMEM is freed
        umma_commit(hdone);
        mbar_drain(hdone, 0);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// qempty[row] = some (round, probe) bucket of the row is empty, from qids and
// the bucket sizes (the fused projection writes qids before the sizes exist).
__global__ void __launch_bounds__(256) k_qempty(GraphDev g) {
  const int64_t total = (int64_t)g.B * g.H * g.N;
  for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < total;
       row += (int64_t)gridDim.x * blockDim.x) {
    const int bh = (int)(row / g.N);
    const int b = bh / g.H, h = bh % g.H;
    const int32_t* bs = g.bsize + (int64_t)(b * g.n_kv + h / g.rep) * g.R * g.NB;
    bool empty = false;
    for (int t0 = 0; t0 < g.NT; t0 += 8) {
      int32_t bz[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) bz[u] = t0 + u < g.NT ? __ldg(bs + g.qids[(int64_t)(t0 + u) * total + row]) : 1;
#pragma unroll
      for (int u = 0; u < 8; ++u) empty |= bz[u] == 0;
    }
    g.qempty[row] = empty ? 1 : 0;
  }
}

// ---------------------------------------------------------------------------
// Exact recompute of the flagged (row, round) items
// ---------------------------------------------------------------------------
// Eight items per warp pass, four lanes each, in the fp32 order of the FMA
// kernels (proj_planes_x4), so every id equals theirs. Queries: the round's
// (1 + Te) slot ids, and qempty[row] = 1 if one of those buckets is empty (the
// hash kernel wrote qempty from the other rounds). Keys: kcode, the member
// bit and the pad-key maximum -- after the hash kernel stored its mask blocks.
template <int D, bool KEYS>
__device__ void fixup_items(const GraphDev& g, const uint32_t* q, unsigned int count, int64_t gw, int64_t nw) {
  const int lane = threadIdx.x & 31, sub = lane & 3;
  const int Te = KEYS ? 0 : g.Te;
  const int64_t total = (int64_t)g.B * g.H * g.N;
  for (int64_t base = gw * 8; base < (int64_t)count; base += nw * 8) {
    const int64_t qi = base + (lane >> 2);
    const bool live = qi < (int64_t)count;
    const uint32_t item = live ? q[qi] : 0u;
    const uint32_t rowid = item >> 4;
    const int r = (int)(item & 15u);
    int bg, b, h;
    int64_t n;
    const void* rowp;
    if (KEYS) {
      bg = (int)(rowid / (uint32_t)g.M);
      n = rowid - (uint32_t)bg * (uint32_t)g.M;
      b = bg / g.n_kv;
      h = bg % g.n_kv;
      rowp = row_ptr<kDtBF16>(g.k, b * g.k_sb + h * g.k_sh + n * g.k_sm);
    } else {
      const int bh = (int)(rowid / (uint32_t)g.N);
      n = rowid - (uint32_t)bh * (uint32_t)g.N;
      b = bh / g.H;
      h = bh % g.H;
      bg = b * g.n_kv + h / g.rep;
      rowp = row_ptr<kDtBF16>(g.q, b * g.q_sb + h * g.q_sh + n * g.q_sn);
    }
    float xs[D / 4];
    load_slice_x4<kDtBF16, D>(rowp, g.d, sub, live, xs);
    float pv[12];
    uint32_t id = 0;
#pragma unroll
    for (int j = 0; j < 12; ++j) pv[j] = 0.f;
    for_round_projections_x4<D, false, 1>(xs, g.rp + (int64_t)r * g.max_p * g.d, g.d, g.p, sub,
                                          [&](int j, int, float v) {
                                            if (v > 0.f) id |= 1u << j;  // proj > 0, strict (:589)
                                            pv[j] = v;
                                          });
    if (!live || sub != 0) continue;
    if (KEYS) {
      g.kcode[((int64_t)bg * g.R + r) * g.M + n] = (uint16_t)id;
      atomicOr(&g.bmap[bmap_idx(g, bg, (int)(n >> 6), r, (int)id)], 1ull << (n & 63));
      atomicMax(&g.pmax[bg * g.R + r], (id << 20) | (uint32_t)n);
    } else {
      // Before the bucket sizes exist (fused projection) qempty is left to k_qempty.
      const int32_t* bs = g.prehashed ? nullptr : g.bsize + ((int64_t)bg * g.R + r) * g.NB;
      const int s0 = r * (1 + Te);
      g.qids[(int64_t)s0 * total + rowid] = (uint16_t)(r * g.NB + id);
      bool empty = bs && __ldg(bs + id) == 0;
      uint32_t used = 0;
      for (int tt = 0; tt < Te; ++tt) {  // as k_hash_queries
        int best = -1;
        float bmag = 0.f;
#pragma unroll
        for (int j = 0; j < 12; ++j) {
          if (j < g.p && !((used >> j) & 1u)) {
            const float a = fabsf(pv[j]);
            if (best < 0 || a < bmag) { best = j; bmag = a; }
          }
        }
        used |= 1u << best;
        const uint32_t pid = id ^ (1u << best);
        g.qids[(int64_t)(s0 + 1 + tt) * total + rowid] = (uint16_t)(r * g.NB + pid);
        empty |= bs && __ldg(bs + pid) == 0;
      }
      if (empty) g.qempty[rowid] = 1;
    }
  }
}

// The fused projection's flagged items (one global queue per kind).
template <int D, bool KEYS>
__global__ void __launch_bounds__(256) k_hash_fixup(GraphDev g) {
  const unsigned int count = g.hq_count[KEYS ? 0 : 1];
  if (blockIdx.x == 0 && threadIdx.x == 0 && count) atomicAdd(&g_hash_recomputed, (unsigned long long)count);
  fixup_items<D, KEYS>(g, KEYS ? g.hq_keys : g.hq_rows, count,
                       ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5, ((int64_t)gridDim.x * blockDim.x) >> 5);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
bool hash_tc_supported(const GraphDev& g) {
  if (g.dtype != kDtBF16 || (g.d != 64 && g.d != 128)) return false;
  if (g.R > htc::kMaxR || g.p > 12) return false;
  // queue items (row << 4 | round) in 32 bits
  if ((int64_t)g.B * g.H * g.N >= (int64_t(1) << 28) || (int64_t)g.B * g.n_kv * g.M >= (int64_t(1) << 28)) return false;
  auto al = [](int64_t s) { return (s * 2) % 16 == 0; };
  if (!al(g.q_sh) || !al(g.q_sn) || !al(g.q_sb) || !al(g.k_sh) || !al(g.k_sm) || !al(g.k_sb)) return false;
  const int NG = htc::hash_groups(g);
  if (htc::plan(g.d, g, false, NG).total > 227 * 1024 || htc::plan(g.d, g, true, NG).total > 227 * 1024) return false;
  if (NG * htc::n_cols(g.R, g.p) > 512) return false;
  return tc_encode_available();
}

size_t hash_tc_planes_bytes(const GraphDev& g) { return htc::planes_bytes(g.d, g.R, g.p); }

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
  }
  return n;
}

cudaError_t launch_hash_planes(const GraphDev& g, cudaStream_t st) {
  const int D = g.d;
  const int64_t elems = (int64_t)htc::kPieces * (D / 64) * htc::n_cols(g.R, g.p) * 64;
  const int img_blocks = (int)((elems + 255) / 256);
  const int norm_blocks = (g.R * g.p + 7) / 8;  // a warp per hyperplane
  k_hash_planes<<<img_blocks + norm_blocks, 256, 0, st>>>(g.rp, g.R, g.max_p, g.p, g.d, D, img_blocks, g.hpl,
                                                           g.pnorm);
  note_launch();
  return cudaGetLastError();
}

template <int D, bool KEYS, int RC, int NG>
static cudaError_t launch_hash_tc_t(const GraphDev& g, cudaStream_t st) {
  CUtensorMap map;
  const bool ok = KEYS ? tc_make_map(&map, g.k, g.d, g.n_kv, g.M, g.B, g.k_sh, g.k_sm, g.k_sb)
                       : tc_make_map(&map, g.q, g.d, g.H, g.N, g.B, g.q_sh, g.q_sn, g.q_sb);
  if (!ok) return cudaErrorInvalidValue;
  const htc::Plan sp = htc::plan(D, g, KEYS, NG);
  auto fn = k_hash_tc<D, KEYS, RC, NG>;
  constexpr int threads = htc::hash_threads(NG);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sp.total);
  if (e != cudaSuccess) return e;
  const int L = KEYS ? g.M : g.N, heads = KEYS ? g.n_kv : g.H;
  const int64_t ntiles = (int64_t)g.B * heads * ((L + htc::ROWS - 1) / htc::ROWS);
  // Resident CTAs per SM: registers and shared memory (occupancy query) and
  // TMEM (512 columns) allow.
  int occ = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, threads, sp.total) != cudaSuccess) occ = 1;
  const int per_sm = std::max(1, std::min(occ, 512 / sp.tmem_cols));
  const int64_t grid = std::min<int64_t>(ntiles, (int64_t)sm_count() * per_sm);
  if (grid <= 0) return cudaSuccess;
  fn<<<(unsigned)grid, threads, sp.total, st>>>(g, map);
  note_launch();
  return cudaGetLastError();
}

template <int RC, int NG>
static cudaError_t launch_hash_tc_rc(const GraphDev& g, bool keys, cudaStream_t st) {
  if (g.d == 64) return keys ? launch_hash_tc_t<64, true, RC, NG>(g, st) : launch_hash_tc_t<64, false, RC, NG>(g, st);
  return keys ? launch_hash_tc_t<128, true, RC, NG>(g, st) : launch_hash_tc_t<128, false, RC, NG>(g, st);
}

cudaError_t launch_hash_tc(const GraphDev& g, bool keys, cudaStream_t st) {
  const bool rc8 = htc::round_cols(g.p) == 8;
  if (htc::hash_groups(g) == 4)
    return rc8 ? launch_hash_tc_rc<8, 4>(g, keys, st) : launch_hash_tc_rc<16, 4>(g, keys, st);
  return rc8 ? launch_hash_tc_rc<8, 2>(g, keys, st) : launch_hash_tc_rc<16, 2>(g, keys, st);
}

bool proj_hash_supported(const GraphDev& g, int dm) {
  if (!hash_tc_supported(g) || g.is_cross || g.M != g.N || g.N % 128 != 0) return false;
  if (dm < 64 || dm % 64 != 0) return false;
  if ((int64_t)g.B * g.N >= (int64_t(1) << 31)) return false;
  const prj::Plan sp = prj::plan(g.d, g);
  // the hash accumulates in the head's drained accumulator columns
  if (sp.total > 227 * 1024 || sp.np > g.d) return false;
  return true;
}

template <int D, int RC>
static cudaError_t launch_proj_t(const GraphDev& g, const ProjDev& pd, cudaStream_t st) {
  CUtensorMap xmap, wmap, omap;
  if (!tc_make_map_2d(&xmap, pd.x, pd.dm, pd.rows, pd.dm) || !tc_make_map_2d(&wmap, pd.w, pd.dm, pd.n_out, pd.dm) ||
      !tc_make_map_2d(&omap, pd.out, pd.n_out, pd.rows, pd.n_out))
    return cudaErrorInvalidValue;
  const prj::Plan sp = prj::plan(D, g);
  auto fn = k_proj_hash<D, RC>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sp.total);
  if (e != cudaSuccess) return e;
  const int64_t ntiles = (int64_t)(pd.rows / htc::ROWS) * ((pd.n_out + prj::TN - 1) / prj::TN);
  const int64_t grid = std::min<int64_t>(ntiles, sm_count());
  fn<<<(unsigned)grid, prj::THREADS, sp.total, st>>>(g, pd, xmap, wmap, omap);
  note_launch();
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  GraphDev f = g;
  f.prehashed = 1;
  k_hash_fixup<D, true><<<2 * sm_count(), 256, 0, st>>>(f);
  note_launch();
  k_hash_fixup<D, false><<<2 * sm_count(), 256, 0, st>>>(f);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_proj_hash(const GraphDev& g, const ProjDev& pd, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(static_cast<char*>(g.ws) + g.zero_off, 0, g.zero_bytes, st);
  if (e != cudaSuccess) return e;
  if ((e = launch_hash_planes(g, st)) != cudaSuccess) return e;
  const bool rc8 = htc::round_cols(g.p) == 8;
  if (g.d == 64) return rc8 ? launch_proj_t<64, 8>(g, pd, st) : launch_proj_t<64, 16>(g, pd, st);
  return rc8 ? launch_proj_t<128, 8>(g, pd, st) : launch_proj_t<128, 16>(g, pd, st);
}

cudaError_t launch_qempty(const GraphDev& g, cudaStream_t st) {
  const int64_t total = (int64_t)g.B * g.H * g.N;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 8 * sm_count());
  k_qempty<<<blocks, 256, 0, st>>>(g);
  note_launch();
  return cudaGetLastError();
}

int read_hash_tc_error(int clear) { return tc_read_error(clear); }

unsigned long long read_hash_recomputed(int clear) {
  unsigned long long v = 0ull;
  if (cudaMemcpyFromSymbol(&v, g_hash_recomputed, sizeof(v)) != cudaSuccess) return ~0ull;
  if (clear && v) {
    const unsigned long long z = 0ull;
    cudaMemcpyToSymbol(g_hash_recomputed, &z, sizeof(z));
  }
  return v;
}

}  // namespace ssa
