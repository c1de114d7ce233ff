// ssa_select_tc.cu -- tensor-core (tcgen05) candidate scan for bf16 inputs.
//
// Computes the same candidate scores as k_select_merge (ssa_graph.cu), with
// 5th-generation tensor cores instead of per-candidate FMA loops. One CTA
// per 128-row query tile:
//
//   warp 8 (one lane)  TMA: the q tile once, then 128-key tiles of K into a
//                      ring of up to 4 stages (SWIZZLE_128B, K-major), and a
//                      bulk copy of each key tile's member-mask block (all
//                      rounds and buckets, R * NB * 16 bytes) into a second
//                      ring when that block is at most 8 KB.
//   warp 9             allocates 256 TMEM columns; one lane issues
//                      tcgen05.mma (M=128, N=128, K=16, bf16 in, fp32 out)
//                      for S = Q K^T into one of two TMEM accumulators, and
//                      tcgen05.commit releases the K stage and publishes S.
//   warps 0-7          two groups of four, alternating key tiles; thread per
//                      query row (TMEM lane = row): OR the row's bucket masks
//                      for the tile, tcgen05.ld the row's 128 scores, and
//                      write to the row's global buffer: in the sample pass
//                      the upper 16 bits of every score of the tile plus its
//                      candidate masks, in the full pass the (key, score)
//                      pairs of candidates with score >= tau.
//
// fp32 inputs are scanned as three bf16 pieces per operand (six products).
// bf16 x bf16 products are exact in fp32, so tensor-core scores differ from
// the reference's fp32 sums only by accumulation order (rescore ties).
// Every wait on an mbarrier is bounded: on timeout the kernel records an
// error code (ssa_device_error) and the pipeline drains and returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include "ssa_common.cuh"
#include "ssa_internal.h"
#include "ssa_select_common.cuh"
#include "ssa_tcgen05.cuh"

namespace ssa {

namespace tc {

constexpr int ROWS = 128;   // query rows per CTA (MMA M, TMEM lanes)
constexpr int NKEY = 128;   // keys per tile (MMA N)
constexpr int THREADS = 320;  // warps 0-7 epilogue (two groups), 8 TMA, 9 MMA

// Scores S = Q K^T: M = 128 query rows, N = 128 keys.
constexpr uint32_t kIdesc = idesc_bf16(ROWS, NKEY);

struct SmemPlan {
  uint32_t q, k, bm, toff, bars, tmem_slot, pads, total;
  int stages, bstages;
  uint32_t bm_bytes;
};

// Bytes of one key tile's member masks for all (round, bucket) pairs; the
// scan stages them in shared memory when they are at most 8 KB.
__host__ __device__ inline uint32_t bm_tile_bytes(const GraphDev& g) {
  return (uint32_t)g.R * (uint32_t)g.NB * 16u;
}

// fp32 inputs are scanned as three bf16 pieces per operand (x = hi + mid +
// lo); bf16 inputs as themselves.
__host__ __device__ inline int scan_pieces(const GraphDev& g) { return g.dtype == kDtF32 ? 3 : 1; }

__host__ __device__ inline SmemPlan plan_stages(int D, int NT, int stages, uint32_t bm_bytes, int bstages,
                                                int P) {
  SmemPlan p;
  uint32_t off = 0;
  auto take = [&](uint32_t bytes, uint32_t align) {
    off = (off + align - 1) / align * align;
    const uint32_t o = off;
    off += bytes;
    return o;
  };
  const uint32_t atoms = (uint32_t)D / 64;
  p.q = take((uint32_t)P * atoms * ROWS * 128, 1024);
  p.k = take((uint32_t)stages * P * atoms * NKEY * 128, 1024);
  p.bm = take((uint32_t)bstages * bm_bytes, 128);
  p.toff = take((uint32_t)NT * ROWS * 2, 16);
  p.bars = take(24 * 8, 8);
  p.tmem_slot = take(16, 16);
  p.pads = take(64 * 4 + 16 * 4, 16);  // pad keys perm_r[M-1] of the slice's rounds (R <= 64),
                                       // then a bitmap of the key tiles holding one (M <= 65536)
  // At least 80 KB per CTA so that at most two CTAs share an SM: two CTAs
  // use all 512 TMEM columns, a third would wait in tcgen05.alloc.
  uint32_t total = off + 1024;
  if (total < 80 * 1024) total = 80 * 1024;
  p.total = total;
  p.stages = stages;
  p.bstages = bstages;
  p.bm_bytes = bstages ? bm_bytes : 0u;
  return p;
}

// The deepest K ring (up to 4 stages) that keeps two CTAs per SM (one with
// fp32 pieces), with a 3-stage (else 2-stage) ring of mask blocks when those
// are staged.
__host__ __device__ inline SmemPlan plan(int D, const GraphDev& g) {
  const uint32_t bmb = bm_tile_bytes(g);
  const bool staged = bmb <= 8192u;
  const int P = scan_pieces(g);
  const uint32_t budget = P == 1 ? 113 * 1024 : 227 * 1024;
  for (int bst = staged ? 3 : 0; bst >= (staged ? 2 : 0); --bst)
    for (int st = 4; st >= 2; --st) {
      const SmemPlan p = plan_stages(D, g.NT, st, bmb, bst, P);
      if (p.total <= budget) return p;
    }
  return plan_stages(D, g.NT, 2, bmb, 0, P);
}

}  // namespace tc

// Candidate scan. pass 0 (sample): key tiles 0, s, 2s, ..., one record of
// upper score halves and candidate masks per tile; pass 1 (full): all key
// tiles, candidates with score >= tau[row] are kept as (key, score) pairs in
// the half of the row's buffer that belongs to the tile's epilogue group.
// rcnt[row][group] counts the candidates seen (pass 0) or kept (pass 1; above
// half the buffer means overflow).
template <int D, int PASS, int P>
__global__ void __launch_bounds__(tc::THREADS, P == 1 ? 2 : 1)
    k_scan_tc(GraphDev g, const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap) {
  using namespace tc;
  constexpr int pass = PASS;  // one instantiation per pass
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int ATOMS = D / 64;
  const SmemPlan sp = plan(D, g);
  const int NS = sp.stages;
  const int NB_ST = sp.bstages;     // 0: masks read from global memory
  const uint32_t bmb = sp.bm_bytes;
  unsigned char* qs = smem + sp.q;
  unsigned char* ks = smem + sp.k;
  unsigned char* bms = smem + sp.bm;
  uint16_t* toff = reinterpret_cast<uint16_t*>(smem + sp.toff);  // [NT][ROWS] r * NB + bucket
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + sp.bars);
  uint64_t* kfull = bars;           // [NS] K stage loaded (TMA tx)
  uint64_t* kempty = bars + 4;      // [NS] K stage consumed (MMA commit)
  uint64_t* sfull = bars + 8;       // [2] S accumulator ready (MMA commit)
  uint64_t* sempty = bars + 10;     // [2] S accumulator drained (its group's 4 warps)
  uint64_t* qfull = bars + 12;      // q tile loaded
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 13);
  uint64_t* bfull = bars + 14;      // [NB_ST] mask block loaded (bulk tx)
  uint64_t* bempty = bars + 18;     // [NB_ST] mask block read (the reading group's 4 warps)
  uint64_t* mma_done = bars + 22;   // every MMA issued has completed (before TMEM is freed)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + sp.tmem_slot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Causal: a row tile's work grows with its position. In a full pass of a
  // few waves (a sharded rank's slice) the CTAs are taken in groups of up to
  // 8 heads (whose K stays in L2 together); within a group in order of
  // decreasing row tile, all its heads per tile, so the heaviest tiles start
  // first and light ones fill the last wave. (Measured on a c2 rank's slice:
  // full pass 0.48 -> 0.43 ms; with many waves, and in the sample pass, the
  // launch order is as fast or faster.)
  int bh = blockIdx.y, bx = blockIdx.x;
  if (pass == 1 && g.causal && gridDim.x * gridDim.y <= 1200) {
    int G = 8;
    while (gridDim.y % G) G >>= 1;
    const int L = blockIdx.y * gridDim.x + blockIdx.x;  // launch order
    const int per = G * gridDim.x, r = L % per;
    bh = (L / per) * G + r % G;
    bx = gridDim.x - 1 - r / G;
  }
  const int b = bh / g.H, h = bh % g.H;
  const int gk = h / g.rep;
  const int bg = b * g.n_kv + gk;
  const int n0 = bx * ROWS;
  const int n_hi = min(g.N, n0 + ROWS) - 1;
  const int nkt_all =
      g.causal ? min((g.M + NKEY - 1) / NKEY, ((g.row0 + n_hi) >> 7) + 1) : (g.M + NKEY - 1) / NKEY;
  const int step = pass == 0 ? g.sample_s : 1;
  const int ntl = (nkt_all + step - 1) / step;  // tiles this CTA visits: 0, step, 2*step, ...

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(kfull + i, 1);
      mbar_init(kempty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(sfull + i, 1);
      mbar_init(sempty + i, 4);
    }
    for (int i = 0; i < NB_ST; ++i) {
      mbar_init(bfull + i, 1);
      mbar_init(bempty + i, 4);
    }
    mbar_init(qfull, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 9) {  // TMEM: 2 accumulators x NKEY fp32 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(2 * NKEY));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      // pieces c of q / k are batch entries c * B + b of the piece buffers
      mbar_expect_tx(qfull, P * ATOMS * ROWS * 128);
      for (int c = 0; c < P; ++c)
        for (int a = 0; a < ATOMS; ++a)
          tma_load_4d(qs + (c * ATOMS + a) * ROWS * 128, &qmap, qfull, a * 64, h, n0, c * g.B + b);
      int issued = 0, issued_b = 0;
      const unsigned long long* bmg = g.bmap + bmap_idx(g, bg, 0, 0, 0);
      for (int i = 0; i < ntl; ++i) {
        const int s = i % NS;
        if (!mbar_wait(kempty + s, ((i / NS) & 1) ^ 1, abort_flag, 11, g.wait_limit)) break;
        mbar_expect_tx(kfull + s, P * ATOMS * NKEY * 128);
        for (int c = 0; c < P; ++c)
          for (int a = 0; a < ATOMS; ++a)
            tma_load_4d(ks + ((s * P + c) * ATOMS + a) * NKEY * 128, &kmap, kfull + s, a * 64, gk,
                        i * step * NKEY, c * g.B + b);
        issued = i + 1;
        if (NB_ST) {
          const int sb2 = i % NB_ST;
          if (!mbar_wait(bempty + sb2, ((i / NB_ST) & 1) ^ 1, abort_flag, 18, g.wait_limit)) break;
          mbar_expect_tx(bfull + sb2, bmb);
          bulk_load(bms + sb2 * bmb, bmg + (int64_t)(i * step) * g.R * g.NB * 2, bmb, bfull + sb2);
          issued_b = i + 1;
        }
      }
      // Do not leave while copies are in flight.
      mbar_drain(qfull, 0);
      for (int i = max(0, issued - NS); i < issued; ++i) mbar_drain(kfull + i % NS, (i / NS) & 1);
      for (int i = max(0, issued_b - NB_ST); i < issued_b; ++i) mbar_drain(bfull + i % NB_ST, (i / NB_ST) & 1);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && mbar_wait(qfull, 0, abort_flag, 13, g.wait_limit)) {
      const uint32_t qa = smem_u32(qs);
      int issued_mma = 0;
      for (int i = 0; i < ntl; ++i) {
        const int s = i % NS, sb = i & 1;
        if (!mbar_wait(kfull + s, (i / NS) & 1, abort_flag, 14, g.wait_limit)) break;
        if (!mbar_wait(sempty + sb, ((i >> 1) & 1) ^ 1, abort_flag, 15, g.wait_limit)) break;
        tc_fence_after();
        const uint32_t ka = smem_u32(ks + s * P * ATOMS * NKEY * 128);
        // fp32: the six piece products down to 2^-16 relative (mid*mid,
        // hi*lo, lo*hi, hi*mid, mid*hi, hi*hi; each bf16 product exact in
        // fp32), smallest first; bf16: the one product.
        constexpr int NPAIR = P == 1 ? 1 : 6;
        constexpr int PA[6] = {1, 0, 2, 0, 1, 0}, PB[6] = {1, 2, 0, 1, 0, 0};
#pragma unroll
        for (int pr = 0; pr < NPAIR; ++pr) {
          const uint32_t qp = qa + (P == 1 ? 0 : PA[pr]) * ATOMS * ROWS * 128;
          const uint32_t kp = ka + (P == 1 ? 0 : PB[pr]) * ATOMS * NKEY * 128;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (ROWS * 128) + (kk & 3) * 32;
            const uint32_t offk = (kk >> 2) * (NKEY * 128) + (kk & 3) * 32;
            umma_bf16(tmem + sb * NKEY, umma_desc(qp + off), umma_desc(kp + offk), kIdesc, (pr | kk) > 0);
          }
        }
        umma_commit(kempty + s);
        umma_commit(sfull + sb);
        issued_mma = i + 1;
      }
      // The epilogue may have stopped early (a wait that ran out): wait for
      // the MMAs in flight before TMEM is freed.
      if (issued_mma) {
        umma_commit(mma_done);
        mbar_drain(mma_done, 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // Group grp (warps 4*grp .. 4*grp+3) takes the tiles i with i % 2 == grp,
    // i.e. accumulator grp; thread t of a group owns query row n0 + t (TMEM
    // lane t). Each group appends to its own half of the row's buffer.
    const int grp = warp >> 2;
    const int t = (warp & 3) * 32 + lane;
    const int n = n0 + t;
    const bool act = n < g.N;
    const int64_t row = (int64_t)bh * g.N + n;
    int* pads = reinterpret_cast<int*>(smem + sp.pads);
    if (act && grp == 0)
      for (int tt = 0; tt < g.NT; ++tt)
        toff[tt * ROWS + t] = g.qids[(int64_t)tt * ((int64_t)g.B * g.H * g.N) + row];
    uint32_t* padtiles = reinterpret_cast<uint32_t*>(pads + 64);
    if (pass == 1 && warp == 0) {
      if (lane < 16) padtiles[lane] = 0u;
      __syncwarp();
      for (int r = lane; r < g.R; r += 32) {
        const int pk = (int)(g.pmax[bg * g.R + r] & 0xFFFFFu);
        pads[r] = pk;
        atomicOr(&padtiles[(pk >> 7) >> 5], 1u << ((pk >> 7) & 31));
      }
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");  // both groups see the offsets (and pad keys)
    const float thr = (pass == 1 && act) ? g.tau[row] : -INFINITY;
    const int half_cap = g.capg >> 1;
    unsigned long long* bo = g.buf + row * g.capg;      // sample records (pass 0)
    unsigned long long* bh_out = bo + grp * half_cap;   // this group's half (pass 1)
    int cnt = 0;
    const uint4* bmg4 = reinterpret_cast<const uint4*>(g.bmap + bmap_idx(g, bg, 0, 0, 0));
    for (int i = grp; i < ntl; i += 2) {
      const int sb = grp;
      const int kt = i * step;
      const int key0 = kt * NKEY;
      // Candidate masks first: they overlap the wait for S. Each (round,
      // bucket) entry holds the tile's two 64-key words.
      unsigned long long w[2] = {0ull, 0ull};
      if (NB_ST) {
        const int sb2 = i % NB_ST;
        if (!mbar_wait_warp(bfull + sb2, (i / NB_ST) & 1, abort_flag, 19, g.wait_limit)) break;
        const uint4* bt = reinterpret_cast<const uint4*>(bms + sb2 * bmb);
        if (act)
          for (int tt = 0; tt < g.NT; ++tt) {
            const uint4 v = bt[toff[tt * ROWS + t]];
            w[0] |= ((unsigned long long)v.y << 32) | v.x;
            w[1] |= ((unsigned long long)v.w << 32) | v.z;
          }
        __syncwarp();
        if (lane == 0) mbar_arrive(bempty + sb2);
      } else if (act) {
        const uint4* bt = bmg4 + (int64_t)kt * g.R * g.NB;
        for (int tt = 0; tt < g.NT; ++tt) {
          const uint4 v = __ldg(bt + toff[tt * ROWS + t]);
          w[0] |= ((unsigned long long)v.y << 32) | v.x;
          w[1] |= ((unsigned long long)v.w << 32) | v.z;
        }
      }
      if (act) {
#pragma unroll
        for (int hw = 0; hw < 2; ++hw) {
          unsigned long long x = w[hw];
          x &= ~__ldg(g.pmask + (int64_t)bg * g.Wpad + 2 * kt + hw);
          if (g.causal) {
            const int lim = g.row0 + n - (key0 + 64 * hw);  // keys before the row's position
            if (lim <= 0) x = 0ull;
            else if (lim < 64) x &= (1ull << lim) - 1ull;
          }
          w[hw] = x;
        }
      }
      const bool pad_tile = pass == 1 && ((padtiles[kt >> 5] >> (kt & 31)) & 1u);
      // causal: the tile holds some row's own key (the last one or two tiles)
      const bool self_tile = pass == 1 && g.causal && key0 <= g.row0 + n_hi && key0 + NKEY > g.row0 + n0;
      if (!mbar_wait_warp(sfull + sb, (i >> 1) & 1, abort_flag, 16, g.wait_limit)) break;
      tc_fence_after();
      const uint32_t ta = tmem + ((uint32_t)((warp & 3) * 32) << 16) + sb * NKEY;
      unsigned char* tdst = reinterpret_cast<unsigned char*>(bo) + (size_t)i * kSampleTileBytes;
      const bool rec = pass == 0 && act && (size_t)(i + 1) * kSampleTileBytes <= (size_t)g.capg * 8;
      // In the tiles holding a row's own key (causal) or a pad key, the
      // scores of those keys -- which the scan leaves out but the selection
      // may need -- are read from the accumulator after the candidates, so
      // it is released only then.
      const bool capture = pass == 1 && (self_tile || pad_tile);
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 32-column chunks
        float sc[32];
        tmem_ld32(ta + c * 32, sc);
        tmem_wait_ld();
        if (c == 3 && !capture) {  // the accumulator can be reused once all columns are read
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(sempty + sb);
        }
        const uint32_t cm = (uint32_t)(w[c >> 1] >> ((c & 1) * 32));
        if (pass == 0) {
          // Sample pass: the upper 16 bits of all 32 scores (two per 32-bit
          // word, no compaction); the tile's candidate masks follow the 256
          // score bytes. The threshold stage reads the masks.
          if (rec) {
            uint4* dst = reinterpret_cast<uint4*>(tdst + c * 64);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 o;
              o.x = __byte_perm(__float_as_uint(sc[8 * v + 0]), __float_as_uint(sc[8 * v + 1]), 0x7632);
              o.y = __byte_perm(__float_as_uint(sc[8 * v + 2]), __float_as_uint(sc[8 * v + 3]), 0x7632);
              o.z = __byte_perm(__float_as_uint(sc[8 * v + 4]), __float_as_uint(sc[8 * v + 5]), 0x7632);
              o.w = __byte_perm(__float_as_uint(sc[8 * v + 6]), __float_as_uint(sc[8 * v + 7]), 0x7632);
              dst[v] = o;
            }
          }
          continue;
        }
        if (!cm) continue;
        const uint32_t kbase32 = (uint32_t)(key0 + c * 32);
        uint32_t h0 = 0, h1 = 0, h2 = 0, h3 = 0;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          h0 |= (sc[j] >= thr ? 1u : 0u) << j;
          h1 |= (sc[j + 1] >= thr ? 2u : 0u) << j;
          h2 |= (sc[j + 2] >= thr ? 4u : 0u) << j;
          h3 |= (sc[j + 3] >= thr ? 8u : 0u) << j;
        }
        uint32_t hit = (h0 | h1 | h2 | h3) & cm;
        while (hit) {
          const int j = __ffs(hit) - 1;
          hit &= hit - 1;
          if (cnt < half_cap)
            bh_out[cnt] = ((unsigned long long)(kbase32 + j) << 32) | __float_as_uint(pick32(sc, j));
          ++cnt;
        }
      }
      if (capture) {  // warp-uniform
        if (pad_tile)
          for (int r = 0; r < g.R; ++r) {
            const int jp = pads[r] - key0;  // the same column for every row
            if ((unsigned)jp < (unsigned)NKEY) {
              const float v = tmem_ld1(ta + jp);
              tmem_wait_ld();
              if (act) g.sspec[row * (g.R + 1) + r] = v;
            }
          }
        if (self_tile) {
          // lane L's own key is column cb + L of the tile
          const int cb = g.row0 + n0 + (warp & 3) * 32 - key0;
          const int ch0 = cb >= 0 ? (cb >> 5) : -1;
#pragma unroll 1
          for (int ch = ch0; ch <= ch0 + 1; ++ch) {
            if (ch < 0 || ch > 3) continue;
            float sc[32];
            tmem_ld32(ta + ch * 32, sc);
            tmem_wait_ld();
            const int js = cb + lane - ch * 32;
            if (act && (unsigned)js < 32u) g.sspec[row * (g.R + 1) + g.R] = pick32(sc, js);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sempty + sb);
      }
      if (pass == 0) {
        if (rec)
          *reinterpret_cast<uint4*>(tdst + 256) =
              make_uint4((uint32_t)w[0], (uint32_t)(w[0] >> 32), (uint32_t)w[1], (uint32_t)(w[1] >> 32));
        cnt += __popcll(w[0]) + __popcll(w[1]);
      }
    }
    if (act) g.rcnt[row * 2 + grp] = cnt;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
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

bool tc_encode_available() { return encode_fn() != nullptr; }

bool tc_make_map_2d(CUtensorMap* m, const void* base, int64_t inner, int64_t outer, int64_t pitch) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)pitch * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_make_map(CUtensorMap* m, const void* base, int d, int heads, int rows, int batch,
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

// fp32 q / k as three bf16 pieces each (hi = rn(x), mid = rn(x - hi),
// lo = rn(x - hi - mid)), in contiguous piece buffers [3 * B][heads][rows][d]
// that the scan's TMA maps read (piece c of batch b at batch index c * B + b).
__global__ void __launch_bounds__(256) k_split_pieces(const float* __restrict__ x, int B, int heads, int rows,
                                                      int d, int64_t sb, int64_t sh, int64_t sn,
                                                      uint16_t* __restrict__ out) {
  const int64_t total = (int64_t)B * heads * rows * d;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i % d);
    int64_t r = i / d;
    const int n = (int)(r % rows);
    r /= rows;
    const int h = (int)(r % heads);
    const int b = (int)(r / heads);
    const float v = __ldg(x + b * sb + h * sh + n * sn + t);
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(hi);
    const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
    const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
    out[i] = __bfloat16_as_ushort(hi);
    out[total + i] = __bfloat16_as_ushort(mid);
    out[2 * total + i] = __bfloat16_as_ushort(lo);
  }
}

bool select_tc_supported(const GraphDev& g) {
  // bf16 with head dim 64 / 128; fp32 (as bf16 pieces) with head dim 64
  if (g.dtype == kDtBF16 ? (g.d != 64 && g.d != 128) : g.d != 64) return false;
  if (g.M > 65536 || g.A > 1024) return false;
  if ((int64_t)g.B * g.H * g.N >= (int64_t(1) << 31)) return false;  // 32-bit row indices in k_rows
  if (g.R + 2 + (g.G < g.C ? g.G : g.C) > 32) return false;  // one special key per lane
  // TMA: 16-byte aligned strides (the base pointers are checked at launch)
  auto al = [](int64_t s) { return (s * 2) % 16 == 0; };
  if (g.dtype == kDtBF16 &&
      (!al(g.q_sh) || !al(g.q_sn) || !al(g.q_sb) || !al(g.k_sh) || !al(g.k_sm) || !al(g.k_sb)))
    return false;
  if ((int64_t)g.R * g.NB > 65535) return false;  // 16-bit mask-block offsets
  const tc::SmemPlan sp = tc::plan(g.d, g);
  if (sp.total > (tc::scan_pieces(g) == 1 ? 113u : 227u) * 1024) return false;
  if (rows_smem_bytes(g, 1) > 227 * 1024) return false;
  return tc_encode_available();
}

bool select_tc_pointers_ok(const GraphDev& g) {
  if (g.dtype == kDtF32) return true;  // the scan reads the piece buffers in the workspace
  return (reinterpret_cast<uintptr_t>(g.q) % 16) == 0 && (reinterpret_cast<uintptr_t>(g.k) % 16) == 0;
}

template <int D, int P>
static cudaError_t launch_scan_t(const GraphDev& g, int pass, const CUtensorMap& qmap,
                                 const CUtensorMap& kmap, cudaStream_t st) {
  const tc::SmemPlan sp = tc::plan(D, g);
  auto fn = pass == 0 ? k_scan_tc<D, 0, P> : k_scan_tc<D, 1, P>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sp.total);
  if (e != cudaSuccess) return e;
  dim3 grid((g.N + tc::ROWS - 1) / tc::ROWS, g.B * g.H);
  fn<<<grid, tc::THREADS, sp.total, st>>>(g, qmap, kmap);
  note_launch();
  return cudaGetLastError();
}

// hash queries -> sample scan -> thresholds -> full scan -> exact selection
// (+ merge). Rows flagged by the selection are recomputed afterwards by the
// exact FMA scan (launch_graph).
cudaError_t launch_select_tc(const GraphDev& g, int mode, cudaStream_t st) {
  CUtensorMap qmap, kmap;
  cudaError_t e;
  if (g.dtype == kDtF32) {
    // fp32: the scan reads bf16 pieces: (3 B, H, N, d) and (3 B, n_kv, M, d)
    const int64_t nq = (int64_t)g.B * g.H * g.N * g.d, nk = (int64_t)g.B * g.n_kv * g.M * g.d;
    k_split_pieces<<<(unsigned)std::min<int64_t>((nq + 255) / 256, 4096), 256, 0, st>>>(
        static_cast<const float*>(g.q), g.B, g.H, g.N, g.d, g.q_sb, g.q_sh, g.q_sn, g.qpc);
    note_launch();
    k_split_pieces<<<(unsigned)std::min<int64_t>((nk + 255) / 256, 4096), 256, 0, st>>>(
        static_cast<const float*>(g.k), g.B, g.n_kv, g.M, g.d, g.k_sb, g.k_sh, g.k_sm, g.kpc);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if (!tc_make_map(&qmap, g.qpc, g.d, g.H, g.N, 3 * g.B, g.N * (int64_t)g.d, g.d, (int64_t)g.H * g.N * g.d) ||
        !tc_make_map(&kmap, g.kpc, g.d, g.n_kv, g.M, 3 * g.B, g.M * (int64_t)g.d, g.d,
                     (int64_t)g.n_kv * g.M * g.d))
      return cudaErrorInvalidValue;
  } else {
    // q (B, H, N, d): dims {d, H, N, B}; k (B, n_kv, M, d): dims {d, n_kv, M, B}
    if (!tc_make_map(&qmap, g.q, g.d, g.H, g.N, g.B, g.q_sh, g.q_sn, g.q_sb)) return cudaErrorInvalidValue;
    if (!tc_make_map(&kmap, g.k, g.d, g.n_kv, g.M, g.B, g.k_sh, g.k_sm, g.k_sb)) return cudaErrorInvalidValue;
  }
  // Query ids: hashed here, or already written by the fused projection
  // (then only qempty, which needs the bucket sizes).
  e = g.prehashed ? launch_qempty(g, st) : (g.use_tc_hash ? launch_hash_tc(g, false, st) : launch_hash_queries(g, st));
  if (e != cudaSuccess) return e;
  stage_mark(kStageHashQueries, st);
  for (int pass = 0; pass < 2; ++pass) {
    e = g.dtype == kDtF32 ? launch_scan_t<64, 3>(g, pass, qmap, kmap, st)
        : g.d == 64       ? launch_scan_t<64, 1>(g, pass, qmap, kmap, st)
                          : launch_scan_t<128, 1>(g, pass, qmap, kmap, st);
    if (e != cudaSuccess) return e;
    stage_mark(pass == 0 ? kStageScanSample : kStageScanFull, st);
    if ((e = launch_rows(g, pass, mode, st)) != cudaSuccess) return e;
    stage_mark(pass == 0 ? kStageRowsThresh : kStageRowsFinal, st);
  }
  return cudaSuccess;
}

int read_device_error(int clear) {
  const int a = tc_read_error(clear);
  const int b = read_hash_tc_error(clear);
  if (a < 0 || b < 0) return -1;
  return a ? a : b;
}

}  // namespace ssa
