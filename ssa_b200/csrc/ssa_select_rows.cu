// ssa_select_rows.cu -- per-query-row stages of the tensor-core graph build.
//
//   k_hash_queries  thread per query row: the row's bucket id per (round,
//                   probe) slot and whether any of those buckets is empty.
//   k_rows          warp per query row, after a scan pass of k_scan_tc:
//     THRESH mode   from the sampled candidates, tau = the x-th largest score
//                   (x ~ 2A scaled by the sampled fraction of key tiles): a
//                   per-row threshold the full scan uses to keep only ~2A
//                   candidates.
//     FINAL mode    verifies that at least A candidates reached tau (then
//                   every top-A member did), adds the special keys (pad keys,
//                   causal self, empty-bucket fallbacks) after replaying the
//                   reference's slot order for each, selects the exact top-A
//                   by a 4-pass radix select, and writes the merged neighbor
//                   row (self, then ascending window/global/LSH keys) or the
//                   LSH row in the reference's topk order. A row that fails
//                   the verification, or overflowed its buffer, flags its
//                   query tile for the exact fallback scan (k_select_merge).
#include "ssa_common.cuh"
#include "ssa_internal.h"
#include "ssa_select_common.cuh"

namespace ssa {

// ---------------------------------------------------------------------------
// Query hashing
// ---------------------------------------------------------------------------
template <int DT, int D>
__global__ void __launch_bounds__(128) k_hash_queries(GraphDev g) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint16_t* tids = reinterpret_cast<uint16_t*>(smem);  // [NT][128]
  const int t = threadIdx.x;
  const int64_t row = (int64_t)blockIdx.x * 128 + t;
  const int64_t total = (int64_t)g.B * g.H * g.N;
  if (row >= total) return;
  const int n = (int)(row % g.N);
  const int64_t bh = row / g.N;
  const int b = (int)(bh / g.H), h = (int)(bh % g.H);
  const int bg = b * g.n_kv + h / g.rep;
  float q[D];
  const void* qrow = row_ptr<DT>(g.q, b * g.q_sb + h * g.q_sh + (int64_t)n * g.q_sn);
#pragma unroll
  for (int i = 0; i < D; i += 4) {
    if (i < g.d) {
      const float4 x = load4<DT>(qrow, i);
      q[i] = x.x; q[i + 1] = x.y; q[i + 2] = x.z; q[i + 3] = x.w;
    } else {
      q[i] = q[i + 1] = q[i + 2] = q[i + 3] = 0.f;
    }
  }
  const bool empty = hash_row_ids<D>(g, q, bg, tids, 128, t);
  for (int tt = 0; tt < g.NT; ++tt) g.qids[row * g.NT + tt] = tids[tt * 128 + t];
  g.qempty[row] = empty ? 1 : 0;
}

// ---------------------------------------------------------------------------
// Warp helpers
// ---------------------------------------------------------------------------
// Order-preserving map of a float to uint32 (ascending floats -> ascending
// unsigned); NaN-free inputs.
__device__ __forceinline__ uint32_t okey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float okey_inv(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// The kth largest (1-based, kth <= n) of sc[0..n) by a 4-pass, 8-bit radix
// select. Returns its order key T and, in *need, how many entries equal to T
// belong to the top kth. Warp-collective.
__device__ uint32_t warp_radix_kth(const float* sc, int n, int kth, uint32_t* hist, int* need_out) {
  const int lane = threadIdx.x & 31;
  uint32_t prefix = 0, pmask = 0;
  int need = kth;
  for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) hist[lane * 8 + j] = 0;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
      const uint32_t u = okey(sc[i]);
      if ((u & pmask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1u);
    }
    __syncwarp();
    // lane L owns bins 255-8L .. 248-8L (descending)
    uint32_t c[8];
    uint32_t tot = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = hist[255 - (lane * 8 + j)];
      tot += c[j];
    }
    uint32_t incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    uint32_t before = incl - tot;  // entries in higher bins than this lane's
    int found_bin = -1;
    uint32_t found_before = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (found_bin < 0 && before < (uint32_t)need && before + c[j] >= (uint32_t)need) {
        found_bin = 255 - (lane * 8 + j);
        found_before = before;
      }
      before += c[j];
    }
    const unsigned who = __ballot_sync(0xffffffffu, found_bin >= 0);
    const int src = __ffs(who) - 1;
    const int bin = __shfl_sync(0xffffffffu, found_bin, src);
    const uint32_t fb = __shfl_sync(0xffffffffu, found_before, src);
    need -= (int)fb;
    prefix |= (uint32_t)bin << shift;
    pmask |= 0xFFu << shift;
    __syncwarp();
  }
  *need_out = need;
  return prefix;
}

struct RowsSmem {
  float* sc;        // [cap] scores
  int32_t* ky;      // [cap] keys
  uint32_t* hist;   // [256]
  uint32_t* bits;   // [Mw] merge bitmap
  int32_t* spec;    // [64] special keys
  uint8_t* sflag;   // [64 * NT] replay flags
};

// ---------------------------------------------------------------------------
// k_rows
// ---------------------------------------------------------------------------
template <int DT, int D>
__global__ void __launch_bounds__(256) k_rows(GraphDev g, int stage, int mode) {
  // stage 0 = THRESH, 1 = FINAL
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cap = g.capg + 64;
  const int Mw = (g.M + 31) / 32;
  const size_t per_warp = (size_t)cap * 8 + 256 * 4 + (size_t)Mw * 4 + 64 * 4 + 64 * (size_t)g.NT;
  unsigned char* base = smem + warp * ((per_warp + 15) & ~size_t(15));
  RowsSmem S;
  S.sc = reinterpret_cast<float*>(base);
  S.ky = reinterpret_cast<int32_t*>(S.sc + cap);
  S.hist = reinterpret_cast<uint32_t*>(S.ky + cap);
  S.bits = S.hist + 256;
  S.spec = reinterpret_cast<int32_t*>(S.bits + Mw);
  S.sflag = reinterpret_cast<uint8_t*>(S.spec + 64);
  if (stage == 1)
    for (int i = lane; i < Mw; i += 32) S.bits[i] = 0;
  __syncwarp();

  const int64_t total = (int64_t)g.B * g.H * g.N;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp; row < total; row += nwarps) {
    const int n = (int)(row % g.N);
    const int64_t bh = row / g.N;
    const int b = (int)(bh / g.H), h = (int)(bh % g.H);
    const int gk = h / g.rep;
    const int bg = b * g.n_kv + gk;
    const int cnt_all = g.rcnt[row];
    const int c = min(cnt_all, g.capg);
    const unsigned long long* bo = g.buf + row * g.capg;
    if (stage == 0) {
      // ---- THRESH: tau = x-th largest sampled score ----------------------
      const int tiles_row = g.causal ? (n + 127) / 128 : (g.M + 127) / 128;
      const int sampled = tiles_row > 0 ? (tiles_row + g.sample_s - 1) / g.sample_s : 0;
      float tau = -INFINITY;
      if (sampled > 0 && tiles_row > 0) {
        // x ~ 3A scaled by the sampled fraction: about 3A candidates are
        // expected at or above tau, so fewer than A (the fallback case) is
        // a 3x deviation, and more than the buffer holds (6A+64) a 2x one.
        const int x = (int)(((int64_t)3 * g.A * sampled + tiles_row - 1) / tiles_row);
        if (x >= 1 && c >= x) {
          for (int i = lane; i < c; i += 32) S.sc[i] = __uint_as_float((uint32_t)bo[i]);
          __syncwarp();
          int need;
          const uint32_t T = warp_radix_kth(S.sc, c, x, S.hist, &need);
          tau = okey_inv(T);
        }
      }
      if (lane == 0) g.tau[row] = tau;
      __syncwarp();
      continue;
    }

    // ---- FINAL -------------------------------------------------------------
    const float tau = g.tau[row];
    const int ntq = (g.N + 127) / 128;
    if (cnt_all > g.capg || (tau > -INFINITY && cnt_all < g.A)) {
      if (lane == 0) g.tile_flags[bh * ntq + n / 128] = 1;  // exact fallback for this tile
      continue;
    }
    for (int i = lane; i < c; i += 32) {
      const unsigned long long e = bo[i];
      S.sc[i] = __uint_as_float((uint32_t)e);
      S.ky[i] = (int32_t)(e >> 32);
    }
    // Special keys: pad keys perm_r[M-1], causal self, empty-bucket fallbacks.
    const bool any_empty = g.qempty[row] != 0;
    const int lim_g = g.G < g.C ? g.G : g.C;
    // Candidate list at fixed positions, one per lane (the tensor-core path
    // requires R + min(G, C) + 2 <= 32): R pad keys, causal self, and (only if
    // a bucket of this row is empty) the fallback globals and key 0. A lane
    // keeps its entry unless it is out of range or repeats an earlier one;
    // kept entries are compacted in order.
    const int ncand = g.R + 1 + (any_empty ? lim_g + 1 : 0);
    int x = -1;
    if (lane < g.R) {
      x = (int)(g.pmax[bg * g.R + lane] & 0xFFFFFu);
      if (g.causal && x > n) x = -1;  // a future pad key never appears as itself
    } else if (lane == g.R) {
      x = g.causal ? n : -1;
    } else if (lane < ncand - 1) {
      x = g.glob[lane - g.R - 1];
    } else if (lane == ncand - 1 && any_empty) {
      x = g.G < g.C ? 0 : -1;
    }
    if (x >= g.M) x = -1;
    bool keep = x >= 0;
    for (int z = 0; z < 32; ++z) {
      const int y = __shfl_sync(0xffffffffu, x, z);
      if (z < lane && y == x) keep = false;
    }
    const unsigned km = __ballot_sync(0xffffffffu, keep);
    if (keep) S.spec[__popc(km & ((1u << lane) - 1u))] = x;
    const int nspec = __popc(km);
    __syncwarp();
    const uint16_t* tids = g.qids + row * g.NT;
    // Replay, lane-parallel over (key, slot) pairs: flag 1 = key's slot in
    // this (round, probe) bucket is a real member, 2 = it is the overflow pad,
    // 0 = absent (or the bucket is empty: handled as a third state 3 = present
    // via the empty-bucket fallback list).
    for (int p = lane; p < nspec * g.NT; p += 32) {
      const int i = p / g.NT, tt = p - i * g.NT;
      const int x = S.spec[i];
      const int r = tt / (1 + g.Te);
      const int u = tids[tt];
      // every load issued up front (no dependent chain)
      const int64_t tb = (int64_t)(bg * g.R + r) * g.NB + u;
      const int sz = __ldg(g.bsize + tb);
      const int lc = __ldg(g.lastc + tb);
      const uint32_t pm = __ldg(g.pmax + bg * g.R + r);
      const uint16_t code = __ldg(g.kcode + ((int64_t)bg * g.R + r) * g.M + x);
      const unsigned long long wbits =
          __ldg(&g.bmap[(((int64_t)bg * g.Wpad + (x >> 6)) * g.R + r) * g.NB + u]);
      const bool member = code == (uint16_t)u && ((wbits >> (x & 63)) & 1ull);
      uint8_t f = 0;
      if (sz == 0) {
        bool in = false;
        for (int cc = 0; cc < lim_g; ++cc) in |= g.glob[cc] == x;
        if (g.G < g.C && x == 0) in = true;
        f = in ? 3 : 0;
      } else {
        bool real;
        if (g.causal && x > n) real = false;
        else if (g.causal && x == n) real = lc > n || member;
        else real = member;
        if (real) f = 1;
        else if (sz < g.C) {
          int P = (int)(pm & 0xFFFFFu);
          if (g.causal && P > n) P = n;
          if (P == x) f = 2;
        }
      }
      S.sflag[p] = f;
    }
    __syncwarp();
    // Lane i decides special i: eligible iff its first appearance is valid.
    int add_key = -1;
    float add_score = 0.f;
    if (lane < nspec) {
      const int x = S.spec[lane];
      bool elig = false;
      for (int tt = 0; tt < g.NT; ++tt) {
        const uint8_t f = S.sflag[lane * g.NT + tt];
        if (f == 0) continue;
        elig = f != 2;
        break;
      }
      if (elig) {
        const bool scanned =
            !((__ldg(g.pmask + (int64_t)bg * g.Wpad + (x >> 6)) >> (x & 63)) & 1ull) && !(g.causal && x >= n);
        bool present = false;
        if (scanned)
          for (int z = 0; z < c && !present; ++z) present = S.ky[z] == x;
        if (!present) {
          const void* qrow = row_ptr<DT>(g.q, b * g.q_sb + h * g.q_sh + (int64_t)n * g.q_sn);
          const void* krow = row_ptr<DT>(g.k, b * g.k_sb + gk * g.k_sh + (int64_t)x * g.k_sm);
          float s0 = 0.f, s1 = 0.f;
          for (int i = 0; i < g.d; i += 4) {
            const float4 a = load4<DT>(qrow, i);
            const float4 kk = load4<DT>(krow, i);
            s0 = fmaf(a.x, kk.x, s0);
            s1 = fmaf(a.y, kk.y, s1);
            s0 = fmaf(a.z, kk.z, s0);
            s1 = fmaf(a.w, kk.w, s1);
          }
          add_key = x;
          add_score = s0 + s1;
        }
      }
    }
    const unsigned am = __ballot_sync(0xffffffffu, add_key >= 0);
    if (add_key >= 0) {
      const int pos = c + __popc(am & ((1u << lane) - 1u));
      S.sc[pos] = add_score;
      S.ky[pos] = add_key;
    }
    const int tot = c + __popc(am);
    __syncwarp();

    // Exact top-A (the whole pool when it has at most A entries).
    const int n_elig = min(tot, g.A);
    uint32_t T = 0;
    int need = 0;
    if (tot > g.A) T = warp_radix_kth(S.sc, tot, g.A, S.hist, &need);
    // Compact the selection to the front: keys > T, then `need` keys == T in
    // index order (ties are the reference's unspecified topk order).
    if (tot > g.A) {
      int wpos = 0, eq_seen = 0;
      // two sweeps keep the write position <= read position
      for (int i0 = 0; i0 < tot; i0 += 32) {
        const int i = i0 + lane;
        const bool in = i < tot;
        const uint32_t u = in ? okey(S.sc[i]) : 0u;
        const bool eq = in && u == T;
        const unsigned eqm = __ballot_sync(0xffffffffu, eq);
        const int eq_rank = eq_seen + __popc(eqm & ((1u << lane) - 1u));
        const bool sel = in && (u > T || (eq && eq_rank < need));
        const unsigned sm = __ballot_sync(0xffffffffu, sel);
        const float sv = in ? S.sc[i] : 0.f;
        const int kv = in ? S.ky[i] : 0;
        __syncwarp();
        if (sel) {
          const int dst = wpos + __popc(sm & ((1u << lane) - 1u));
          S.sc[dst] = sv;
          S.ky[dst] = kv;
        }
        __syncwarp();
        wpos += __popc(sm);
        eq_seen += __popc(eqm);
      }
    }
    __syncwarp();

    if (mode == 1) {
      // Reference topk order: descending score. Bitonic sort of n_elig
      // entries (padded to a power of two with -inf) in shared memory.
      int P2 = 32;
      while (P2 < n_elig) P2 <<= 1;
      for (int i = n_elig + lane; i < P2; i += 32) {
        S.sc[i] = -INFINITY;
        S.ky[i] = 0x7fffffff;
      }
      __syncwarp();
      for (int k2 = 2; k2 <= P2; k2 <<= 1) {
        for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1) {
          for (int i = lane; i < P2; i += 32) {
            const int ixj = i ^ j2;
            if (ixj > i) {
              const bool desc = (i & k2) == 0;
              const float a = S.sc[i], bb = S.sc[ixj];
              if ((a < bb) == desc) {
                S.sc[i] = bb;
                S.sc[ixj] = a;
                const int t0 = S.ky[i];
                S.ky[i] = S.ky[ixj];
                S.ky[ixj] = t0;
              }
            }
          }
          __syncwarp();
        }
      }
      int32_t* out = g.lsh + row * g.A;
      for (int j = lane; j < g.A; j += 32) out[j] = j < n_elig ? S.ky[j] : (j < g.G ? g.glob[j] : 0);
      __syncwarp();
      continue;
    }
    if (g.lsh) {
      int32_t* out = g.lsh + row * g.A;
      for (int j = lane; j < g.A; j += 32) out[j] = j < n_elig ? S.ky[j] : (j < g.G ? g.glob[j] : 0);
    }
    // Merge through a bitmap over [0, M): LSH keys, window, globals, key 0
    // from the fallback slots; self excluded, then emitted in ascending order.
    const bool add_zero = max(n_elig, g.G) < g.A;
    const int kw = g.is_cross ? 0 : 2 * g.window + 1;
    for (int j = lane; j < n_elig; j += 32) {
      const int x = S.ky[j];
      atomicOr(&S.bits[x >> 5], 1u << (x & 31));
    }
    for (int j = lane; j < kw; j += 32) {
      const int o = j - g.window;
      int idx = (g.causal && o > 0) ? n : n + o;
      idx = idx < 0 ? 0 : (idx > g.M - 1 ? g.M - 1 : idx);
      atomicOr(&S.bits[idx >> 5], 1u << (idx & 31));
    }
    for (int j = lane; j < g.G; j += 32) {
      const int x = min(max(g.glob[j], 0), g.M - 1);
      atomicOr(&S.bits[x >> 5], 1u << (x & 31));
    }
    if (add_zero && lane == 0) atomicOr(&S.bits[0], 1u);
    __syncwarp();
    if (!g.is_cross && lane == 0 && n < g.M) atomicAnd(&S.bits[n >> 5], ~(1u << (n & 31)));
    __syncwarp();
    int32_t* nbo = g.nb + row * g.Wout;
    uint8_t* vo = g.valid + row * g.Wout;
    const int s0 = g.is_cross ? 0 : 1;
    if (!g.is_cross && lane == 0) {
      nbo[0] = min(n, g.M - 1);
      vo[0] = 1;
    }
    // Lane L scans words [L*wpl, (L+1)*wpl); exclusive scan of popcounts.
    const int wpl = (Mw + 31) / 32;
    const int w0 = lane * wpl, w1 = min(Mw, w0 + wpl);
    int my = 0;
    for (int wd = w0; wd < w1; ++wd) my += __popc(S.bits[wd]);
    int incl = my;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int slot = s0 + incl - my;
    for (int wd = w0; wd < w1 && slot < g.Wout; ++wd) {
      uint32_t bw = S.bits[wd];
      while (bw && slot < g.Wout) {
        const int bit = __ffs(bw) - 1;
        bw &= bw - 1u;
        nbo[slot] = wd * 32 + bit;
        vo[slot] = 1;
        ++slot;
      }
    }
    const int total_set = __shfl_sync(0xffffffffu, incl, 31);
    for (int j = s0 + total_set + lane; j < g.Wout; j += 32) {
      nbo[j] = 0;
      vo[j] = 0;
    }
    __syncwarp();
    // clear the bitmap words this row touched
    for (int j = lane; j < n_elig; j += 32) S.bits[S.ky[j] >> 5] = 0;
    for (int j = lane; j < kw; j += 32) {
      const int o = j - g.window;
      int idx = (g.causal && o > 0) ? n : n + o;
      idx = idx < 0 ? 0 : (idx > g.M - 1 ? g.M - 1 : idx);
      S.bits[idx >> 5] = 0;
    }
    for (int j = lane; j < g.G; j += 32) S.bits[min(max(g.glob[j], 0), g.M - 1) >> 5] = 0;
    if (lane == 0) S.bits[0] = 0;
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
template <typename F>
static cudaError_t smem_attr(F* fn, size_t bytes) {
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

cudaError_t launch_hash_queries(const GraphDev& g, cudaStream_t st) {
  const int64_t rows = (int64_t)g.B * g.H * g.N;
  const unsigned grid = (unsigned)((rows + 127) / 128);
  const size_t sm = (size_t)g.NT * 128 * 2;
  cudaError_t e;
  if (g.d <= 64) {
    auto fn = g.dtype == kDtF32 ? k_hash_queries<kDtF32, 64> : k_hash_queries<kDtBF16, 64>;
    if ((e = smem_attr(fn, sm)) != cudaSuccess) return e;
    fn<<<grid, 128, sm, st>>>(g);
  } else {
    auto fn = g.dtype == kDtF32 ? k_hash_queries<kDtF32, 128> : k_hash_queries<kDtBF16, 128>;
    if ((e = smem_attr(fn, sm)) != cudaSuccess) return e;
    fn<<<grid, 128, sm, st>>>(g);
  }
  return cudaGetLastError();
}

size_t rows_smem_bytes(const GraphDev& g, int warps) {
  const int cap = g.capg + 64;
  const int Mw = (g.M + 31) / 32;
  const size_t per_warp = (size_t)cap * 8 + 256 * 4 + (size_t)Mw * 4 + 64 * 4 + 64 * (size_t)g.NT;
  return (size_t)warps * ((per_warp + 15) & ~size_t(15));
}

cudaError_t launch_rows(const GraphDev& g, int stage, int mode, cudaStream_t st) {
  int warps = 8;
  while (warps > 1 && rows_smem_bytes(g, warps) > 200 * 1024) warps >>= 1;
  const size_t sm = rows_smem_bytes(g, warps);
  if (sm > 227 * 1024) return cudaErrorInvalidConfiguration;
  const int64_t rows = (int64_t)g.B * g.H * g.N;
  int64_t blocks = (rows + warps - 1) / warps;
  if (blocks > 148 * 64) blocks = 148 * 64;
  cudaError_t e;
  auto fn = g.dtype == kDtF32 ? (g.d <= 64 ? k_rows<kDtF32, 64> : k_rows<kDtF32, 128>)
                              : (g.d <= 64 ? k_rows<kDtBF16, 64> : k_rows<kDtBF16, 128>);
  if ((e = smem_attr(fn, sm)) != cudaSuccess) return e;
  fn<<<(unsigned)blocks, warps * 32, sm, st>>>(g, stage, mode);
  return cudaGetLastError();
}

}  // namespace ssa
