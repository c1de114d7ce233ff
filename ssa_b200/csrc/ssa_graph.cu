// ssa_graph.cu -- LSH neighbor-graph build for sm_100a.
//
// Replaces LSHGraphBuilder.forward + WindowGraphBuilder + GlobalGraphBuilder +
// merge_neighbors of the reference (sparse_attention.py:357-1089). The
// reference materialises, per query, R x (1 + probes) x C candidate slots,
// deduplicates them with two sorts, gathers every candidate key row and
// runs a chunked top-k. Here the same result is produced without ever
// materialising a candidate list:
//
//   1. k_hash_keys    per key row: R bucket ids (fp32 sign tests), and for
//                     every (64-key word, round, bucket) a 64-bit membership
//                     mask, built with warp match + one atomicOr per bucket.
//   2. k_bucket_trim  per (kv slice, round, bucket): keeps the first C members
//                     (ascending key index = the stable bucket order), records
//                     the bucket size and the C-th member, and marks the
//                     round's overflow pad key perm[M-1] (the largest key of
//                     the highest non-empty bucket).
//   3. k_select_merge per query row (one thread): hashes the query, ORs the
//                     masks of its R x (1+T) buckets into a 64-bit candidate
//                     word per 64-key tile, scores exactly those candidates
//                     from a shared-memory key tile and keeps the top-A in a
//                     shared-memory min-heap. The few keys whose eligibility
//                     is not plain membership (pad keys, causal self, empty-
//                     bucket fallbacks) are resolved by replaying the
//                     reference's slot order for that one key. Finally the
//                     LSH set is merged with the window and the globals
//                     (sorted, deduplicated, self first) straight into the
//                     neighbor output.
//
// Why this equals the reference: a candidate entry survives the reference's
// cross-round dedup iff it is valid and no earlier slot holds the same key.
// For an ordinary key x (not a pad key, not causal self, not an empty-bucket
// fallback of this row) every slot holding x is a valid bucket member, so x
// is eligible iff it is a member (rank < C) of at least one of the row's
// buckets -- exactly the OR of the masks. The special keys are replayed.
#include "ssa_common.cuh"
#include "ssa_internal.h"
#include "ssa_select_common.cuh"

namespace ssa {

// ---------------------------------------------------------------------------
// 1. Key hashing + bucket membership masks
// ---------------------------------------------------------------------------
// Four lanes per key row (each holds a quarter of the row, see
// proj_planes_x4), kHashRows<D> rows per four lanes: a warp hashes its 32
// keys 8 * kHashRows<D> at a time, staging the codes in shared memory, then
// lane L takes key L for the membership masks.
template <int DT, int D, bool SMEM>
__global__ void __launch_bounds__(256, 2) k_hash_keys(GraphDev g) {
  extern __shared__ __align__(16) float s_planes[];  // SMEM: R * p * d floats; then the codes
  const int bg = blockIdx.y;
  const int b = bg / g.n_kv, gk = bg % g.n_kv;
  const int pd = g.p * g.d;
  if (SMEM) {
    for (int i = threadIdx.x * 4; i < g.R * pd; i += blockDim.x * 4) {
      const int r = i / pd, rem = i - r * pd;
      *reinterpret_cast<float4*>(s_planes + i) =
          __ldg(reinterpret_cast<const float4*>(g.rp + (int64_t)r * g.max_p * g.d + rem));
    }
  }
  __shared__ uint32_t s_pmax[8][64];  // per warp and round (R <= 64): packed max, reduced per block
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane & 3;
  // [warp][R][32] codes of the warp's keys
  uint16_t* codes = reinterpret_cast<uint16_t*>(s_planes + (SMEM ? g.R * pd : 0)) + warp * g.R * 32;
  __syncthreads();
  const int wbase = (blockIdx.x * 8 + warp) * 32;  // first key of the warp (a multiple of 32)
  const void* kbase = row_ptr<DT>(g.k, b * g.k_sb + gk * g.k_sh);
  constexpr int RW = kHashRows<D>, EPL = D / 4;  // keys per four lanes
  for (int i = 0; i < 32 / (8 * RW); ++i) {
    float xs[RW * EPL];
#pragma unroll
    for (int w = 0; w < RW; ++w) {
      const int mk = wbase + i * 8 * RW + w * 8 + (lane >> 2);
      load_slice_x4<DT, D>(row_ptr<DT>(kbase, (int64_t)(mk < g.M ? mk : 0) * g.k_sm), g.d, sub, mk < g.M,
                           xs + w * EPL);
    }
    for (int r = 0; r < g.R; ++r) {
      uint32_t code[RW] = {};
      const float* pl = SMEM ? s_planes + r * pd : g.rp + (int64_t)r * g.max_p * g.d;
      for_round_projections_x4<D, SMEM, RW>(xs, pl, g.d, g.p, sub, [&](int j, int w, float s) {
        if (s > 0.f) code[w] |= 1u << j;  // proj > 0, strict (:589)
      });
      if (sub == 0)
#pragma unroll
        for (int w = 0; w < RW; ++w) codes[r * 32 + i * 8 * RW + w * 8 + (lane >> 2)] = (uint16_t)code[w];
    }
  }
  __syncwarp();
  const int m = wbase + lane;
  const bool act = m < g.M;
  const unsigned amask = __ballot_sync(0xffffffffu, act);
  for (int r = 0; r < g.R; ++r) {
    const uint32_t code = codes[r * 32 + lane];
    uint32_t mx = 0u;
    if (act) {
      g.kcode[((int64_t)bg * g.R + r) * g.M + m] = (uint16_t)code;
      const unsigned peers = __match_any_sync(amask, code);
      if (lane == __ffs(peers) - 1) {
        const unsigned long long bits = (unsigned long long)peers << (wbase & 63);
        atomicOr(&g.bmap[bmap_idx(g, bg, wbase >> 6, r, (int)code)], bits);
      }
      // perm[M-1] of the stable sort = largest key of the highest bucket.
      mx = __reduce_max_sync(amask, (code << 20) | (uint32_t)m);
    }
    if (lane == 0) s_pmax[warp][r] = mx;
  }
  // one atomicMax per block and round instead of one per warp
  __syncthreads();
  if (threadIdx.x < g.R) {
    uint32_t mx = 0u;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mx = max(mx, s_pmax[w][threadIdx.x]);
    atomicMax(&g.pmax[bg * g.R + threadIdx.x], mx);
  }
}

// ---------------------------------------------------------------------------
// 2. Keep the first C members of every bucket (stable order), sizes, C-th member
// ---------------------------------------------------------------------------
// One warp per (b, kv head, round, bucket): lane L owns a contiguous run of
// the bucket's 64-key mask words; a warp prefix sum of their popcounts gives
// every word's rank, so members past the first C are cleared in parallel.
// bsize = the bucket's full size; lastc = the key at rank min(size, C) - 1
// (-1 for an empty bucket). The first warp of each (b, kv head, round) also
// marks its pad key perm_r[M-1] in pmask.
__global__ void __launch_bounds__(256) k_bucket_trim(GraphDev g) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (wid >= (int64_t)g.B * g.n_kv * g.R * g.NB) return;
  const int u = (int)(wid % g.NB);
  const int64_t t = wid / g.NB;
  const int r = (int)(t % g.R), bg = (int)(t / g.R);
  const int wpl = (g.W + 31) / 32;
  const int w0 = min(lane * wpl, g.W), w1 = min(w0 + wpl, g.W);
  int cnt = 0;
  for (int w = w0; w < w1; ++w) cnt += __popcll(g.bmap[bmap_idx(g, bg, w, r, u)]);
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  const int size = __shfl_sync(0xffffffffu, incl, 31);
  const int keep_n = min(size, g.C);  // members that stay
  int run = incl - cnt;               // members before this lane's words
  int last = -1;
  if (run < keep_n || size > g.C) {
    for (int w = w0; w < w1; ++w) {
      unsigned long long* ptr = &g.bmap[bmap_idx(g, bg, w, r, u)];
      unsigned long long x = *ptr;
      if (!x) continue;
      const int c = __popcll(x);
      if (run >= g.C) {
        *ptr = 0ull;
      } else if (run + c > g.C) {
        int need = g.C - run;
        unsigned long long kept = 0ull;
        while (need--) {
          const unsigned long long lo = x & (~x + 1ull);
          kept |= lo;
          x ^= lo;
        }
        *ptr = kept;
        last = w * 64 + 63 - __clzll(kept);
      } else {
        last = w * 64 + 63 - __clzll(x);
      }
      run += c;
    }
  }
  // the bucket's last kept member lies in the highest lane that kept one
  const unsigned has = __ballot_sync(0xffffffffu, last >= 0);
  const int src = has ? 31 - __clz(has) : 0;
  last = __shfl_sync(0xffffffffu, last, src);
  if (lane == 0) {
    g.bsize[(bg * g.R + r) * g.NB + u] = size;
    g.lastc[(bg * g.R + r) * g.NB + u] = has ? last : -1;
    if (u == 0) {
      const uint32_t P = g.pmax[bg * g.R + r] & 0xFFFFFu;
      atomicOr(&g.pmask[(int64_t)bg * g.Wpad + (P >> 6)], 1ull << (P & 63));
    }
  }
}

// ---------------------------------------------------------------------------
// 3. Per-row selection (+ merge)
// ---------------------------------------------------------------------------
template <int DT, int D, typename KT>
__global__ void k_select_merge(GraphDev g, int mode) {
  // mode: 0 = build_graph (merge into nb/valid, optional lsh set out)
  //       1 = lsh_select (LSH output only, reference topk order)
  constexpr int KTILE = 64;
  constexpr int KS = D + 4;  // padded row stride (floats) of the key tile
  extern __shared__ __align__(16) unsigned char smem[];
  const int rows = blockDim.x;
  float* Ks = reinterpret_cast<float*>(smem);
  float* hs = Ks + KTILE * KS;
  KT* hk = reinterpret_cast<KT*>(hs + (size_t)g.A * rows);
  uint16_t* tids = reinterpret_cast<uint16_t*>(hk + (size_t)g.A * rows);
  int32_t* gs = reinterpret_cast<int32_t*>(
      (reinterpret_cast<uintptr_t>(tids + (size_t)g.NT * rows) + 3) & ~uintptr_t(3));

  const int bh = blockIdx.y;
  // As the exact fallback of the tensor-core path, only flagged 128-row tiles run.
  if (g.fallback_only && !g.tile_flags[(int64_t)bh * ((g.N + 127) / 128) + (blockIdx.x * rows) / 128]) return;
  const int b = bh / g.H, h = bh % g.H;
  const int gk = h / g.rep;
  const int bg = b * g.n_kv + gk;
  const int t = threadIdx.x;
  const int n = blockIdx.x * rows + t;
  const bool act = n < g.N;
  const int n_hi = min(g.N, (int)(blockIdx.x + 1) * rows) - 1;
  const int na = g.row0 + n;  // sequence position of this row

  // Sorted unique globals for the merge (only the set matters to it).
  if (t == 0) {
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

  float q[D];
#pragma unroll
  for (int i = 0; i < D; ++i) q[i] = 0.f;
  bool any_empty = false;
  if (act) {
    const void* qrow = row_ptr<DT>(g.q, b * g.q_sb + h * g.q_sh + (int64_t)n * g.q_sn);
#pragma unroll
    for (int i = 0; i < D; i += 4) {
      if (i < g.d) {
        const float4 x = load4<DT>(qrow, i);
        q[i] = x.x; q[i + 1] = x.y; q[i + 2] = x.z; q[i + 3] = x.w;
      }
    }
    any_empty = hash_row_ids<D>(g, q, bg, tids, rows, t);
  }

  // Dense candidate scan over 64-key tiles staged in shared memory; only the
  // row's candidates (OR of its bucket masks) are scored.
  RowHeap<KT> heap{hs, hk, rows, t};
  int cnt = 0;
  const int nkt = g.causal ? min(g.W, ((g.row0 + n_hi) >> 6) + 1) : g.W;
  const char* kbase = reinterpret_cast<const char*>(row_ptr<DT>(g.k, b * g.k_sb + gk * g.k_sh));
  for (int kt = 0; kt < nkt; ++kt) {
    const int key0 = kt * KTILE;
    __syncthreads();
    for (int e = t * 4; e < KTILE * D; e += rows * 4) {
      const int j = e / D, i = e - j * D;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (key0 + j < g.M && i < g.d)
        x = load4<DT>(row_ptr<DT>(kbase, (int64_t)(key0 + j) * g.k_sm), i);
      *reinterpret_cast<float4*>(Ks + j * KS + i) = x;
    }
    __syncthreads();
    if (!act) continue;
    unsigned long long w = 0ull;
    for (int tt = 0; tt < g.NT; ++tt) {
      const int r = tt / (1 + g.Te);
      w |= __ldg(&g.bmap[bmap_idx(g, bg, kt, r, tids[tt * rows + t])]);
    }
    w &= ~__ldg(g.pmask + (int64_t)bg * g.Wpad + kt);
    if (g.causal) {  // keys < na only; na itself is a special key
      const int lim = na - key0;
      if (lim <= 0) w = 0ull;
      else if (lim < 64) w &= (1ull << lim) - 1ull;
    }
    while (w) {
      const int j = __ffsll((long long)w) - 1;
      w &= w - 1ull;
      const float* kr = Ks + j * KS;
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
      for (int i = 0; i < D; i += 4) {
        const float4 x = *reinterpret_cast<const float4*>(kr + i);
        s0 = fmaf(q[i], x.x, s0);
        s1 = fmaf(q[i + 1], x.y, s1);
        s2 = fmaf(q[i + 2], x.z, s2);
        s3 = fmaf(q[i + 3], x.w, s3);
      }
      heap.push(cnt, g.A, (s0 + s1) + (s2 + s3), key0 + j);
    }
  }
  if (!act) return;
  finish_row<DT, D, KT>(g, mode, heap, cnt, tids, rows, t, gs, bh, b, h, gk, bg, n, na, any_empty);
}

// Standalone merge_neighbors (sparse_attention.py:966-1089) over explicit
// inputs: per row, the window row and the LSH row are sorted together
// (in-place heap sort, ascending) and merged with the sorted unique globals;
// entries equal to the row's self index are dropped, duplicates collapse,
// self (if any) takes slot 0 and everything is clamped to [0, true_max].
__device__ void int_sift(int32_t* a, int rows, int t, int i, int size, int x) {
  while (true) {
    const int l = 2 * i + 1;
    if (l >= size) break;
    int c = l;
    int cv = a[l * rows + t];
    if (l + 1 < size) {
      const int rv = a[(l + 1) * rows + t];
      if (rv > cv) { c = l + 1; cv = rv; }
    }
    if (cv > x) { a[i * rows + t] = cv; i = c; } else break;
  }
  a[i * rows + t] = x;
}

__global__ void k_merge_rows(MergeDev m) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int rows = blockDim.x;
  int32_t* buf = reinterpret_cast<int32_t*>(smem);
  int32_t* gs = buf + (size_t)(m.Kw + m.A) * rows;
  const int t = threadIdx.x;
  if (t == 0) {
    int ng = 0;
    for (int i = 0; i < m.G; ++i) {
      const int v = m.glob[i];
      bool dup = false;
      for (int z = 0; z < ng; ++z) dup |= gs[z] == v;
      if (dup) continue;
      int j = ng - 1;
      while (j >= 0 && gs[j] > v) { gs[j + 1] = gs[j]; --j; }
      gs[j + 1] = v;
      ++ng;
    }
    gs[m.G] = ng;
  }
  __syncthreads();
  const int64_t row = (int64_t)blockIdx.x * rows + t;
  if (row >= (int64_t)m.B * m.H * m.N) return;
  const int n = (int)(row % m.N);
  const int tm = *m.true_max;
  const int L = m.Kw + m.A;
  for (int j = 0; j < m.Kw; ++j) buf[j * rows + t] = m.win[(int64_t)n * m.Kw + j];
  for (int j = 0; j < m.A; ++j) buf[(m.Kw + j) * rows + t] = m.lsh[row * m.A + j];
  for (int i = L / 2 - 1; i >= 0; --i) int_sift(buf, rows, t, i, L, buf[i * rows + t]);
  for (int e = L - 1; e > 0; --e) {
    const int x = buf[e * rows + t];
    buf[e * rows + t] = buf[t];
    int_sift(buf, rows, t, 0, e, x);
  }
  int32_t* nbo = m.nb + row * m.Wout;
  uint8_t* vo = m.valid + row * m.Wout;
  int slot = 0;
  const bool has_self = m.self_idx != nullptr;
  const int self = has_self ? m.self_idx[row] : 0;
  if (has_self) {
    nbo[0] = self < 0 ? 0 : (self > tm ? tm : self);
    vo[0] = 1;
    slot = 1;
  }
  const int ng = gs[m.G];
  int il = 0, ig = 0;
  bool first = true;
  int last = 0;
  const int BIG = 0x7fffffff;
  while (slot < m.Wout) {
    const int vl = il < L ? buf[il * rows + t] : BIG;
    const int vg = ig < ng ? gs[ig] : BIG;
    const int v = min(vl, vg);
    if (il >= L && ig >= ng) break;
    if (v == vl && il < L) ++il; else ++ig;
    if ((!first && v == last) || (has_self && v == self)) continue;
    first = false;
    last = v;
    nbo[slot] = v < 0 ? 0 : (v > tm ? tm : v);
    vo[slot] = v <= tm;
    ++slot;
  }
  for (; slot < m.Wout; ++slot) {
    nbo[slot] = 0;
    vo[slot] = 0;
  }
}

// Query/key hash ids only (the reference's _hash), for the ssa_hash_ids API:
// the same four-lanes-per-row projections as the graph build's kernels, so
// the ids reported here are the ids the graph build uses.
template <int DT, int D>
__global__ void __launch_bounds__(256) k_hash_ids(const void* x, int B, int heads, int rows_n,
                                                  int d, int64_t sb, int64_t sh, int64_t sn,
                                                  const float* rp, int R, int max_p, int p,
                                                  int32_t* out) {
  constexpr int RW = kHashRows<D>, EPL = D / 4;  // rows per four lanes
  const int lane = threadIdx.x & 31, sub = lane & 3;
  const int64_t base = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * (8 * RW) + (lane >> 2);
  const int64_t total = (int64_t)B * heads * rows_n;
  int64_t obase[RW];
  int nn[RW];
  bool act[RW];
  float xs[RW * EPL];
#pragma unroll
  for (int w = 0; w < RW; ++w) {
    const int64_t i = base + 8 * w;
    act[w] = i < total;  // no early exit: the four lanes of a row shuffle together
    const int64_t ii = act[w] ? i : 0;
    nn[w] = (int)(ii % rows_n);
    const int64_t bh = ii / rows_n;
    const int b = (int)(bh / heads), h = (int)(bh % heads);
    obase[w] = bh * R;
    load_slice_x4<DT, D>(row_ptr<DT>(x, b * sb + h * sh + (int64_t)nn[w] * sn), d, sub, act[w], xs + w * EPL);
  }
  for (int r = 0; r < R; ++r) {
    uint32_t code[RW] = {};
    for_round_projections_x4<D, false, RW>(xs, rp + (int64_t)r * max_p * d, d, p, sub, [&](int j, int w, float s) {
      if (s > 0.f) code[w] |= 1u << j;
    });
#pragma unroll
    for (int w = 0; w < RW; ++w)
      if (act[w] && sub == 0) out[(obase[w] + r) * rows_n + nn[w]] = (int32_t)code[w];
  }
}

// ---------------------------------------------------------------------------
// neighbor_overlap (sparse_attention.py:1583-1615): per row, the number of
// valid A slots whose index is among the valid B slots, over |valid A| +
// |valid B| - that number (at least 1). One warp per row: B's valid indices
// staged in shared memory, each lane tests its A slots against all of them
// (broadcast reads, exact for any order and duplicates).
// ---------------------------------------------------------------------------
template <typename IT>
__global__ void __launch_bounds__(256) k_neighbor_overlap(const IT* nb_a, const uint8_t* va, const IT* nb_b,
                                                          const uint8_t* vb, int64_t rows, int K, float* out) {
  extern __shared__ __align__(16) long long s_b[];  // [8 warps][K]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= rows) return;
  long long* sb = s_b + (size_t)warp * K;
  const IT* ra = nb_a + row * K;
  const IT* rb = nb_b + row * K;
  int nbv = 0;  // valid B slots
  for (int j0 = 0; j0 < K; j0 += 32) {
    const int j = j0 + lane;
    const bool v = j < K && __ldg(vb + row * K + j);
    const unsigned m = __ballot_sync(0xffffffffu, v);
    if (v) sb[nbv + __popc(m & ((1u << lane) - 1u))] = (long long)__ldg(rb + j);
    nbv += __popc(m);
  }
  __syncwarp();
  int inter = 0, nav = 0;
  for (int j = lane; j < K; j += 32) {
    if (!__ldg(va + row * K + j)) continue;
    ++nav;
    const long long x = (long long)__ldg(ra + j);
    bool hit = false;
    for (int z = 0; z < nbv && !hit; ++z) hit = sb[z] == x;
    inter += hit ? 1 : 0;
  }
  inter = __reduce_add_sync(0xffffffffu, inter);
  nav = __reduce_add_sync(0xffffffffu, nav);
  if (lane == 0) out[row] = (float)inter / fmaxf((float)(nav + nbv - inter), 1.f);
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

#ifndef SSA_SAMPLE_DIV
#define SSA_SAMPLE_DIV 12
#endif
// The sample pass scores every (A / kSampleDiv)-th key tile.
constexpr int kSampleDiv = SSA_SAMPLE_DIV;

size_t graph_workspace_layout(GraphDev* g) {
  const int64_t BG = (int64_t)g->B * g->n_kv;
  const int64_t W = g->Wpad;
  const int64_t NB = int64_t(1) << g->p;
  const int64_t rows = (int64_t)g->B * g->H * g->N;
  g->capg = ((6 * g->A + 64) + 7) / 8 * 8;
  // Every s-th key tile is sampled (about kSampleDiv / A of them); the
  // sampled tiles' records must fit the row buffer.
  {
    const int tiles = (g->M + 127) / 128;
    const int fit = (int)((size_t)g->capg * 8 / kSampleTileBytes);
    int s = g->A / kSampleDiv > 1 ? g->A / kSampleDiv : 1;
    if (fit > 0 && (tiles + s - 1) / s > fit) s = (tiles + fit - 1) / fit;
    g->sample_s = s;
  }
  g->use_tc = select_tc_supported(*g) ? 1 : 0;
  if (g->use_tc_hash) g->use_tc_hash = hash_tc_supported(*g) ? 1 : 0;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t o_kcode = take(sizeof(uint16_t) * BG * g->R * g->M);
  const size_t o_zero_begin = off;
  const size_t o_bmap = take(sizeof(unsigned long long) * BG * W * g->R * NB);
  const size_t o_pmask = take(sizeof(unsigned long long) * BG * W);
  const size_t o_pmax = take(sizeof(uint32_t) * BG * g->R);
  const int64_t ntq = (g->N + 127) / 128;
  const size_t o_flags = take((size_t)g->B * g->H * ntq);
  const size_t o_hqc = take(2 * sizeof(unsigned int));
  const size_t o_zero_end = off;
  const size_t o_bsize = take(sizeof(int32_t) * BG * g->R * NB);
  const size_t o_lastc = take(sizeof(int32_t) * BG * g->R * NB);
  size_t o_hpl = 0, o_pnorm = 0, o_hqk = 0, o_hqr = 0;
  if (g->use_tc_hash) {
    o_hpl = take(hash_tc_planes_bytes(*g));
    o_pnorm = take(sizeof(float) * g->R * g->p);
    // per-CTA segments of ceil(tiles / CTAs) tiles' items: below 2 x tiles x 128 x R
    const int64_t tk = BG * ((g->M + 127) / 128), tq = (int64_t)g->B * g->H * ((g->N + 127) / 128);
    o_hqk = take(sizeof(uint32_t) * 2 * tk * 128 * g->R);
    o_hqr = take(sizeof(uint32_t) * 2 * tq * 128 * g->R);
  }
  size_t o_qids = 0, o_qempty = 0, o_tau = 0, o_rcnt = 0, o_buf = 0, o_sspec = 0;
  if (g->use_tc) {
    o_qids = take(sizeof(uint16_t) * rows * g->NT);
    o_qempty = take(rows);
    o_tau = take(sizeof(float) * rows);
    o_rcnt = take(sizeof(int32_t) * rows * 2);
    o_sspec = take(sizeof(float) * rows * (g->R + 1));
    o_buf = take(sizeof(unsigned long long) * rows * g->capg);
  }
  size_t o_qpc = 0, o_kpc = 0;
  if (g->use_tc && g->dtype == kDtF32) {
    o_qpc = take(sizeof(uint16_t) * 3 * rows * g->d);
    o_kpc = take(sizeof(uint16_t) * 3 * BG * g->M * g->d);
  }
  if (g->ws) {
    char* base = static_cast<char*>(g->ws);
    g->kcode = reinterpret_cast<uint16_t*>(base + o_kcode);
    g->bmap = reinterpret_cast<unsigned long long*>(base + o_bmap);
    g->pmask = reinterpret_cast<unsigned long long*>(base + o_pmask);
    g->pmax = reinterpret_cast<uint32_t*>(base + o_pmax);
    g->tile_flags = reinterpret_cast<uint8_t*>(base + o_flags);
    g->bsize = reinterpret_cast<int32_t*>(base + o_bsize);
    g->lastc = reinterpret_cast<int32_t*>(base + o_lastc);
    g->hq_count = reinterpret_cast<unsigned int*>(base + o_hqc);
    if (g->use_tc_hash) {
      g->hpl = reinterpret_cast<uint16_t*>(base + o_hpl);
      g->pnorm = reinterpret_cast<float*>(base + o_pnorm);
      g->hq_keys = reinterpret_cast<uint32_t*>(base + o_hqk);
      g->hq_rows = reinterpret_cast<uint32_t*>(base + o_hqr);
    }
    if (g->use_tc) {
      g->qids = reinterpret_cast<uint16_t*>(base + o_qids);
      g->qempty = reinterpret_cast<uint8_t*>(base + o_qempty);
      g->tau = reinterpret_cast<float*>(base + o_tau);
      g->rcnt = reinterpret_cast<int32_t*>(base + o_rcnt);
      g->sspec = reinterpret_cast<float*>(base + o_sspec);
      g->buf = reinterpret_cast<unsigned long long*>(base + o_buf);
      if (g->dtype == kDtF32) {
        g->qpc = reinterpret_cast<uint16_t*>(base + o_qpc);
        g->kpc = reinterpret_cast<uint16_t*>(base + o_kpc);
      }
    }
    g->zero_off = o_zero_begin;
    g->zero_bytes = o_zero_end - o_zero_begin;
  }
  return off;
}

static size_t select_smem(int D, int rows, int A, int NT, int G, int key_bytes) {
  return (size_t)64 * (D + 4) * 4 + (size_t)A * rows * (4 + key_bytes) +
         (size_t)NT * rows * 2 + 4 + (size_t)(G + 1) * 4 + 16;
}

int choose_select_rows(const GraphDev& g, int* rows_out, size_t* smem_out) {
  const int D = g.d <= 32 ? 32 : (g.d <= 64 ? 64 : 128);
  const int kb = g.M <= 65536 ? 2 : 4;
  const size_t budget2 = 113 * 1024, budget1 = 227 * 1024;
  for (int rows : {128, 64, 32}) {
    const size_t sm = select_smem(D, rows, g.A, g.NT, g.G, kb);
    if (sm <= budget2) { *rows_out = rows; *smem_out = sm; return 0; }
  }
  for (int rows : {64, 32}) {
    const size_t sm = select_smem(D, rows, g.A, g.NT, g.G, kb);
    if (sm <= budget1) { *rows_out = rows; *smem_out = sm; return 0; }
  }
  return 1;
}

template <typename F>
static cudaError_t set_smem(F* fn, size_t bytes) {
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <int DT, int D, typename KT>
static cudaError_t launch_select_t(const GraphDev& g, int mode, int rows, size_t smem,
                                   cudaStream_t st) {
  auto fn = k_select_merge<DT, D, KT>;
  cudaError_t e = set_smem(fn, smem);
  if (e != cudaSuccess) return e;
  dim3 grid((g.N + rows - 1) / rows, g.B * g.H);
  fn<<<grid, rows, smem, st>>>(g, mode);
  note_launch();
  return cudaGetLastError();
}

template <int DT>
static cudaError_t launch_select_dt(const GraphDev& g, int mode, int rows, size_t smem,
                                    cudaStream_t st) {
  const bool k16 = g.M <= 65536;
  if (g.d <= 32) return k16 ? launch_select_t<DT, 32, uint16_t>(g, mode, rows, smem, st)
                            : launch_select_t<DT, 32, uint32_t>(g, mode, rows, smem, st);
  if (g.d <= 64) return k16 ? launch_select_t<DT, 64, uint16_t>(g, mode, rows, smem, st)
                            : launch_select_t<DT, 64, uint32_t>(g, mode, rows, smem, st);
  return k16 ? launch_select_t<DT, 128, uint16_t>(g, mode, rows, smem, st)
             : launch_select_t<DT, 128, uint32_t>(g, mode, rows, smem, st);
}

cudaError_t launch_graph(const GraphDev& g_in, int mode, cudaStream_t st) {
  cudaError_t e;
  GraphDev g = g_in;
  if (!select_tc_pointers_ok(g)) g.use_tc_hash = 0;  // TMA needs 16-byte aligned rows
  stage_mark(kStageBegin, st);
  if (g.prehashed) {
    // ssa_qkv_proj_hash zeroed the workspace and wrote the key hash state.
  } else if ((e = cudaMemsetAsync(static_cast<char*>(g.ws) + g.zero_off, 0, g.zero_bytes, st)) != cudaSuccess) {
    return e;
  }
  if (g.prehashed) {
  } else if (g.use_tc_hash) {
    if ((e = launch_hash_planes(g, st)) != cudaSuccess) return e;
    if ((e = launch_hash_tc(g, true, st)) != cudaSuccess) return e;
  } else {
    const size_t planes = (size_t)g.R * g.p * g.d * sizeof(float);
    const bool smem = planes <= kHashPlaneSmemMax;
    const size_t sm = (smem ? planes : 0) + (size_t)8 * g.R * 32 * sizeof(uint16_t);
    dim3 grid((g.M + 255) / 256, g.B * g.n_kv);
    const bool f32 = g.dtype == kDtF32;
    auto fn = smem ? (g.d <= 64 ? (f32 ? k_hash_keys<kDtF32, 64, true> : k_hash_keys<kDtBF16, 64, true>)
                                : (f32 ? k_hash_keys<kDtF32, 128, true> : k_hash_keys<kDtBF16, 128, true>))
                   : (g.d <= 64 ? (f32 ? k_hash_keys<kDtF32, 64, false> : k_hash_keys<kDtBF16, 64, false>)
                                : (f32 ? k_hash_keys<kDtF32, 128, false> : k_hash_keys<kDtBF16, 128, false>));
    if ((e = set_smem(fn, sm)) != cudaSuccess) return e;
    fn<<<grid, 256, sm, st>>>(g);
    note_launch();
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  stage_mark(kStageHashKeys, st);
  {
    const int64_t warps = (int64_t)g.B * g.n_kv * g.R * g.NB;
    k_bucket_trim<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(g);
  }
  note_launch();
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  stage_mark(kStageBucketTrim, st);
  GraphDev f = g;
  if (g.use_tc && select_tc_pointers_ok(g)) {
    if ((e = launch_select_tc(g, mode, st)) != cudaSuccess) return e;
    f.fallback_only = 1;  // exact FMA scan for the tiles the selection flagged
  } else {
    for (int i = kStageHashQueries; i <= kStageRowsFinal; ++i) stage_mark(i, st);
    f.fallback_only = 0;
  }
  int rows;
  size_t smem;
  if (choose_select_rows(f, &rows, &smem)) return cudaErrorInvalidConfiguration;
  e = f.dtype == kDtF32 ? launch_select_dt<kDtF32>(f, mode, rows, smem, st)
                        : launch_select_dt<kDtBF16>(f, mode, rows, smem, st);
  stage_mark(kStageSelectFma, st);
  return e;
}

cudaError_t launch_merge(const MergeDev& m, cudaStream_t st) {
  int rows = 128;
  auto bytes = [&](int r) { return (size_t)(m.Kw + m.A) * r * 4 + (size_t)(m.G + 1) * 4; };
  while (bytes(rows) > 200 * 1024 && rows > 32) rows /= 2;
  if (bytes(rows) > 227 * 1024) return cudaErrorInvalidConfiguration;
  cudaError_t e = set_smem(k_merge_rows, bytes(rows));
  if (e != cudaSuccess) return e;
  const int64_t total = (int64_t)m.B * m.H * m.N;
  k_merge_rows<<<(unsigned)((total + rows - 1) / rows), rows, bytes(rows), st>>>(m);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_hash_ids(const void* x, int dtype, int B, int heads, int rows, int d,
                            int64_t sb, int64_t sh, int64_t sn, const float* rp, int R,
                            int max_p, int p, int32_t* out, cudaStream_t st) {
  const int64_t total = (int64_t)B * heads * rows;
  const int per_block = 64 * (d <= 64 ? kHashRows<64> : kHashRows<128>);  // 8 warps x 8 * RW rows
  const unsigned grid = (unsigned)((total + per_block - 1) / per_block);
  const bool f32 = dtype == kDtF32;
  auto fn = d <= 64 ? (f32 ? k_hash_ids<kDtF32, 64> : k_hash_ids<kDtBF16, 64>)
                    : (f32 ? k_hash_ids<kDtF32, 128> : k_hash_ids<kDtBF16, 128>);
  fn<<<grid, 256, 0, st>>>(x, B, heads, rows, d, sb, sh, sn, rp, R, max_p, p, out);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_neighbor_overlap(const void* nb_a, const uint8_t* va, const void* nb_b, const uint8_t* vb,
                                    int64_t rows, int K, int nb_i64, float* out, cudaStream_t st) {
  const size_t smem = (size_t)8 * K * sizeof(long long);
  const unsigned grid = (unsigned)((rows + 7) / 8);
  cudaError_t e;
  if (nb_i64) {
    if ((e = set_smem(k_neighbor_overlap<int64_t>, smem)) != cudaSuccess) return e;
    k_neighbor_overlap<int64_t><<<grid, 256, smem, st>>>(static_cast<const int64_t*>(nb_a), va,
                                                         static_cast<const int64_t*>(nb_b), vb, rows, K, out);
  } else {
    if ((e = set_smem(k_neighbor_overlap<int32_t>, smem)) != cudaSuccess) return e;
    k_neighbor_overlap<int32_t><<<grid, 256, smem, st>>>(static_cast<const int32_t*>(nb_a), va,
                                                         static_cast<const int32_t*>(nb_b), vb, rows, K, out);
  }
  note_launch();
  return cudaGetLastError();
}

}  // namespace ssa
