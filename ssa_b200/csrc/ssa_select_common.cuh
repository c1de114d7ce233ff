// ssa_select_common.cuh -- per-query-row pieces shared by the two candidate
// scans (FMA scan in ssa_graph.cu, tensor-core scan in ssa_select_tc.cu):
// the shared-memory top-A heap, the query hash + multi-probe ids, the
// replay that decides the eligibility of the few "special" keys, and the
// row epilogue (special keys, fallback, merge with window and globals).
#pragma once

#include "ssa_common.cuh"
#include "ssa_internal.h"

namespace ssa {

// Shared-memory arrays are interleaved by row: element i of row t lives at
// [i * rows + t], so 32 threads touching their own element i hit 32 banks.
template <typename KT>
struct RowHeap {
  float* s;
  KT* k;
  int rows, t;
  __device__ float sc(int i) const { return s[i * rows + t]; }
  __device__ int key(int i) const { return (int)k[i * rows + t]; }
  __device__ void set(int i, float v, int kk) {
    s[i * rows + t] = v;
    k[i * rows + t] = (KT)kk;
  }
  // Min-heap on score: place (x, kx) at i and sift down within size.
  __device__ void sift_score(int i, int size, float x, int kx) {
    while (true) {
      const int l = 2 * i + 1;
      if (l >= size) break;
      int c = l;
      float cv = sc(l);
      if (l + 1 < size) {
        const float rv = sc(l + 1);
        if (rv < cv) { c = l + 1; cv = rv; }
      }
      if (cv < x) { set(i, cv, key(c)); i = c; } else break;
    }
    set(i, x, kx);
  }
  __device__ void heapify_score(int size) {
    for (int i = size / 2 - 1; i >= 0; --i) sift_score(i, size, sc(i), key(i));
  }
  // Max-heap on key (for an ascending in-place key sort).
  __device__ void sift_key(int i, int size, float x, int kx) {
    while (true) {
      const int l = 2 * i + 1;
      if (l >= size) break;
      int c = l;
      int cv = key(l);
      if (l + 1 < size) {
        const int rv = key(l + 1);
        if (rv > cv) { c = l + 1; cv = rv; }
      }
      if (cv > kx) { set(i, sc(c), cv); i = c; } else break;
    }
    set(i, x, kx);
  }
  __device__ void sort_keys_ascending(int size) {
    for (int i = size / 2 - 1; i >= 0; --i) sift_key(i, size, sc(i), key(i));
    for (int e = size - 1; e > 0; --e) {
      const float x = sc(e);
      const int kx = key(e);
      set(e, sc(0), key(0));
      sift_key(0, e, x, kx);
    }
  }
  // Descending by score (the reference's topk order): min-heap sort.
  __device__ void sort_scores_descending(int size, bool is_heap) {
    if (!is_heap) heapify_score(size);
    for (int e = size - 1; e > 0; --e) {
      const float x = sc(e);
      const int kx = key(e);
      set(e, sc(0), key(0));
      sift_score(0, e, x, kx);
    }
  }
  // Insert into a top-`cap` heap with `cnt` entries so far.
  __device__ void push(int& cnt, int cap, float v, int kk) {
    if (cnt < cap) {
      set(cnt, v, kk);
      if (++cnt == cap) heapify_score(cap);
    } else if (v > sc(0)) {
      sift_score(0, cap, v, kk);
    }
  }
};

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

__device__ __forceinline__ bool key_member(const GraphDev& g, int bg, int r, int u, int x) {
  if (x < 0 || x >= g.M) return false;
  if (g.kcode[((int64_t)bg * g.R + r) * g.M + x] != (uint16_t)u) return false;
  const unsigned long long w =
      __ldg(&g.bmap[bmap_idx(g, bg, x >> 6, r, u)]);
  return (w >> (x & 63)) & 1ull;
}

// Replays the reference's slot order (round-major, primary bucket then
// probes, slot c = 0..C-1) for one key x and reports whether x's FIRST slot
// is valid -- the cross-round dedup rule of sparse_attention.py:884-890.
// n is the query's sequence position.
__device__ inline bool replay_first_valid(const GraphDev& g, const uint16_t* tids, int rows, int t,
                                          int bg, int n, int x) {
  for (int tt = 0; tt < g.NT; ++tt) {
    const int r = tt / (1 + g.Te);
    const int u = tids[tt * rows + t];
    const int sz = g.bsize[(bg * g.R + r) * g.NB + u];
    if (sz == 0) {  // empty bucket: [glob..., 0, ...], all valid (:711-737)
      const int lim = g.G < g.C ? g.G : g.C;
      for (int c = 0; c < lim; ++c)
        if (g.glob[c] == x) return true;
      if (g.G < g.C && x == 0) return true;
      continue;
    }
    bool real;
    if (g.causal && x > n) real = false;  // future keys only appear as n
    else if (g.causal && x == n)          // n itself, or any future member mapped to n
      real = g.lastc[(bg * g.R + r) * g.NB + u] > n || key_member(g, bg, r, u, n);
    else
      real = key_member(g, bg, r, u, x);
    if (real) return true;
    if (sz < g.C) {  // overflow slots hold perm[M-1], invalid (:686-696)
      int P = (int)(g.pmax[bg * g.R + r] & 0xFFFFFu);
      if (g.causal && P > n) P = n;
      if (P == x) return false;
    }
  }
  return false;
}

template <int DT, int D>
__device__ __forceinline__ float dot_row_global(const float* q, const void* row, int d) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
  for (int i = 0; i < D; i += 4) {
    if (i < d) {
      const float4 x = load4<DT>(row, i);
      s0 = fmaf(q[i], x.x, s0);
      s1 = fmaf(q[i + 1], x.y, s1);
      s2 = fmaf(q[i + 2], x.z, s2);
      s3 = fmaf(q[i + 3], x.w, s3);
    }
  }
  return (s0 + s1) + (s2 + s3);
}

// Every hash projection (keys, queries, the FMA fallback scan, ssa_hash_ids)
// is summed in one fixed order, so the kernels that split a row over four
// lanes and the ones that keep it in one thread give bit-identical ids:
//   * element t belongs to slice (t / 4) % 4 -- slices interleave in groups
//     of four consecutive elements;
//   * within a slice, groups are taken in ascending order; of each group the
//     pairs (t, t+1) and (t+2, t+3) go through a paired fp32 FMA, so even
//     elements accumulate into the low half and odd ones into the high half;
//   * a slice's sum is low + high, and the projection is
//     (slice0 + slice1) + (slice2 + slice3).
// Elements at or past d are skipped.

// Projections of one row (x: D floats in registers) onto NBK hyperplanes pl,
// pl + d, ..., pl + (NBK-1) d, in the order above. The NBK chains only give
// the FMA pipe independent work; each result is the same as a lone one.
template <int NBK, int D, bool SMEM>
__device__ __forceinline__ void proj_planes(const float* x, const float* pl, int d, float* out) {
  unsigned long long s2[NBK][4];
#pragma unroll
  for (int k = 0; k < NBK; ++k)
#pragma unroll
    for (int s = 0; s < 4; ++s) s2[k][s] = 0ull;
#pragma unroll
  for (int t = 0; t < D; t += 4) {
    if (t < d) {
      const int s = (t >> 2) & 3;
      const unsigned long long xa = f2_pack(x[t], x[t + 1]), xb = f2_pack(x[t + 2], x[t + 3]);
#pragma unroll
      for (int k = 0; k < NBK; ++k) {
        const float4 w = SMEM ? *reinterpret_cast<const float4*>(pl + k * d + t)
                              : __ldg(reinterpret_cast<const float4*>(pl + k * d + t));
        s2[k][s] = f2_fma(xa, f2_pack(w.x, w.y), s2[k][s]);
        s2[k][s] = f2_fma(xb, f2_pack(w.z, w.w), s2[k][s]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < NBK; ++k) {
    float v[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      float lo, hi;
      f2_unpack(s2[k][s], lo, hi);
      v[s] = lo + hi;
    }
    out[k] = (v[0] + v[1]) + (v[2] + v[3]);
  }
}

// The same projections with each row split over four consecutive lanes: lane
// `sub` (0..3) holds slice `sub` of RW rows -- elements 16 i + 4 sub .. +3 --
// as xs[r * EPL + 4 i .. + 3] (EPL = D / 4 floats per row). Each lane sums
// its slices; two butterfly steps give every lane of the four (slice0 +
// slice1) + (slice2 + slice3), bit-identical to proj_planes. Each hyperplane
// element loaded serves RW rows. out[r * NBK + k]. All 32 lanes of the warp
// must call it together.
template <int NBK, int D, bool SMEM, int RW>
__device__ __forceinline__ void proj_planes_x4(const float* xs, const float* pl, int d, int sub, float* out) {
  constexpr int EPL = D / 4;
  unsigned long long s2[RW * NBK];
#pragma unroll
  for (int k = 0; k < RW * NBK; ++k) s2[k] = 0ull;
#pragma unroll
  for (int i = 0; i < EPL; i += 4) {
    const int t = 4 * i + 4 * sub;  // element index of xs[r * EPL + i]
    if (t < d) {
#pragma unroll
      for (int k = 0; k < NBK; ++k) {
        const float4 w = SMEM ? *reinterpret_cast<const float4*>(pl + k * d + t)
                              : __ldg(reinterpret_cast<const float4*>(pl + k * d + t));
        const unsigned long long wa = f2_pack(w.x, w.y), wb = f2_pack(w.z, w.w);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
          s2[r * NBK + k] = f2_fma(f2_pack(xs[r * EPL + i], xs[r * EPL + i + 1]), wa, s2[r * NBK + k]);
          s2[r * NBK + k] = f2_fma(f2_pack(xs[r * EPL + i + 2], xs[r * EPL + i + 3]), wb, s2[r * NBK + k]);
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < RW * NBK; ++k) {
    float lo, hi;
    f2_unpack(s2[k], lo, hi);
    float v = lo + hi;
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    out[k] = v;
  }
}

// Lane `sub`'s slice of a row (elements 16 i + 4 sub .. +3, zero at or past
// d) into xs[EPL]. Rows are 8-byte (bf16) / 16-byte (fp32) aligned and d is
// a multiple of 4, so every group of four is one aligned load.
template <int DT, int D>
__device__ __forceinline__ void load_slice_x4(const void* row, int d, int sub, bool act, float* xs) {
#pragma unroll
  for (int i = 0; i < D / 4; i += 4) {
    const int t = 4 * i + 4 * sub;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (act && t < d) v = load4<DT>(row, t);
    xs[i] = v.x; xs[i + 1] = v.y; xs[i + 2] = v.z; xs[i + 3] = v.w;
  }
}

// f(j, r, proj) for hyperplanes j = 0 .. p-1 of one round and rows r < RW,
// each row split over four lanes (see proj_planes_x4), two hyperplanes per
// pass. j and r are compile-time indices in f, so f may write register
// arrays at [j] / [r].
template <int D, bool SMEM, int RW, typename F>
__device__ __forceinline__ void for_round_projections_x4(const float* xs, const float* pl, int d, int p, int sub,
                                                         F&& f) {
#pragma unroll
  for (int j = 0; j < 12; j += 2) {
    if (j + 2 <= p) {
      float o[2 * RW];
      proj_planes_x4<2, D, SMEM, RW>(xs, pl + (size_t)j * d, d, sub, o);
#pragma unroll
      for (int r = 0; r < RW; ++r) {
        f(j, r, o[r * 2]);
        f(j + 1, r, o[r * 2 + 1]);
      }
    } else if (j < p) {
      float o[RW];
      proj_planes_x4<1, D, SMEM, RW>(xs, pl + (size_t)j * d, d, sub, o);
#pragma unroll
      for (int r = 0; r < RW; ++r) f(j, r, o[r]);
    }
  }
}

// f(j, proj_j) for the hyperplanes j = 0 .. p-1 of one round (hyperplane j
// at pl + j d): four per pass while four remain, then two, then one.
template <int D, bool SMEM, typename F>
__device__ __forceinline__ void for_round_projections(const float* x, const float* pl, int d, int p, F&& f) {
  int j = 0;
  for (; j + 4 <= p; j += 4) {
    float o[4];
    proj_planes<4, D, SMEM>(x, pl + (size_t)j * d, d, o);
#pragma unroll
    for (int k = 0; k < 4; ++k) f(j + k, o[k]);
  }
  if (j + 2 <= p) {
    float o[2];
    proj_planes<2, D, SMEM>(x, pl + (size_t)j * d, d, o);
    f(j, o[0]);
    f(j + 1, o[1]);
    j += 2;
  }
  if (j < p) {
    float o[1];
    proj_planes<1, D, SMEM>(x, pl + (size_t)j * d, d, o);
    f(j, o[0]);
  }
}

// The row's bucket id per (round, probe) slot into tids (sign tests in fp32,
// sparse_attention.py:559-597; step-wise multi-probe, :599-646: probe t flips
// the bit with the t-th smallest |proj| of the ORIGINAL id, ties in plane
// order). Returns whether any of those buckets is empty.
// Bucket ids of one row (q in registers) for every (round, probe) slot:
// tids[(r * (1 + Te) + probe) * rows + t]; returns whether any of those
// buckets is empty. Hyperplane j of round r is rp + (r * max_p + j) * d.
template <int D>
__device__ inline bool hash_row_ids(const GraphDev& g, const float* q, int bg, uint16_t* tids, int rows, int t) {
  for (int r = 0; r < g.R; ++r) {
    float proj[12];  // registers: written and read with static indices only
#pragma unroll
    for (int j = 0; j < 12; ++j) proj[j] = 0.f;
    uint32_t id = 0;
    for_round_projections<D, false>(q, g.rp + (int64_t)r * g.max_p * g.d, g.d, g.p, [&](int j, float s) {
      if (s > 0.f) id |= 1u << j;
      if (g.Te > 0) {
#pragma unroll
        for (int jj = 0; jj < 12; ++jj)
          if (jj == j) proj[jj] = s;
      }
    });
    tids[(r * (1 + g.Te)) * rows + t] = (uint16_t)id;
    uint32_t used = 0;
    for (int tt = 0; tt < g.Te; ++tt) {
      int best = -1;
      float bmag = 0.f;
#pragma unroll
      for (int j = 0; j < 12; ++j) {
        if (j < g.p && !((used >> j) & 1u)) {
          const float a = fabsf(proj[j]);
          if (best < 0 || a < bmag) { best = j; bmag = a; }
        }
      }
      used |= 1u << best;
      tids[(r * (1 + g.Te) + 1 + tt) * rows + t] = (uint16_t)(id ^ (1u << best));
    }
  }
  bool any_empty = false;
  for (int tt = 0; tt < g.NT; ++tt) {
    const int r = tt / (1 + g.Te);
    if (g.bsize[(bg * g.R + r) * g.NB + tids[tt * rows + t]] == 0) any_empty = true;
  }
  return any_empty;
}

// Row epilogue after the candidate scan: the special keys (pad keys perm_r[M-1],
// causal self, and -- when one of the row's buckets is empty -- the empty-
// bucket fallback entries) are replayed and, if eligible, scored and pushed;
// then either the LSH selection is written in the reference's topk order
// (mode 1) or merged with the window and the globals into the neighbor row
// (mode 0).
template <int DT, int D, typename KT>
__device__ inline void finish_row(const GraphDev& g, int mode, RowHeap<KT>& heap, int& cnt,
                                  const uint16_t* tids, int rows, int t, const int32_t* gs, int bh,
                                  int b, int h, int gk, int bg, int n, int na, bool any_empty) {
  // n: the row within q and the outputs; na = g.row0 + n: its sequence
  // position (causal limit, window, self).
  const char* kbase = reinterpret_cast<const char*>(row_ptr<DT>(g.k, b * g.k_sb + gk * g.k_sh));
  const int lim_g = g.G < g.C ? g.G : g.C;
  const int nspec = g.R + 1 + (any_empty ? lim_g + 1 : 0);
  auto spec_at = [&](int i) -> int {
    if (i < g.R) return (int)(g.pmax[bg * g.R + i] & 0xFFFFFu);
    if (i == g.R) return g.causal ? na : -1;
    i -= g.R + 1;
    if (i < lim_g) return g.glob[i];
    return g.G < g.C ? 0 : -1;
  };
  bool have_q = false;
  float q[D];
  for (int i = 0; i < nspec; ++i) {
    const int x = spec_at(i);
    if (x < 0 || x >= g.M) continue;  // not a key of this sequence (e.g. self when N > M)
    if (i < g.R && g.causal && x > na) continue;  // a future pad key never appears as itself
    bool dup = false;
    for (int z = 0; z < i && !dup; ++z) dup = spec_at(z) == x;
    if (dup) continue;
    if (!replay_first_valid(g, tids, rows, t, bg, na, x)) continue;
    // Keys the scan may already have taken: not a pad key, not causal self.
    const bool scanned = !((__ldg(g.pmask + (int64_t)bg * g.Wpad + (x >> 6)) >> (x & 63)) & 1ull) &&
                         !(g.causal && x >= na);
    if (scanned) {
      bool present = false;
      for (int z = 0; z < cnt && !present; ++z) present = heap.key(z) == x;
      if (present) continue;
    }
    if (!have_q) {
      const void* qrow = row_ptr<DT>(g.q, b * g.q_sb + h * g.q_sh + (int64_t)n * g.q_sn);
#pragma unroll
      for (int c = 0; c < D; c += 4) {
        if (c < g.d) {
          const float4 v = load4<DT>(qrow, c);
          q[c] = v.x; q[c + 1] = v.y; q[c + 2] = v.z; q[c + 3] = v.w;
        } else {
          q[c] = q[c + 1] = q[c + 2] = q[c + 3] = 0.f;
        }
      }
      have_q = true;
    }
    heap.push(cnt, g.A, dot_row_global<DT, D>(q, row_ptr<DT>(kbase, (int64_t)x * g.k_sm), g.d), x);
  }

  // Slots the reference fills from -inf scores get glob[j] (j < G) else 0
  // (:948-957); only the set matters to the merge, where the globals are
  // present anyway, so the merge adds just key 0 when such a slot exists.
  const bool add_zero = max(cnt, g.G) < g.A;
  if (mode == 1) {
    heap.sort_scores_descending(cnt, cnt == g.A);
    int32_t* out = g.lsh + ((int64_t)bh * g.N + n) * g.A;
    for (int j = 0; j < g.A; ++j) out[j] = j < cnt ? heap.key(j) : (j < g.G ? g.glob[j] : 0);
    return;
  }
  if (g.lsh) {
    int32_t* out = g.lsh + ((int64_t)bh * g.N + n) * g.A;
    for (int j = 0; j < g.A; ++j) out[j] = j < cnt ? heap.key(j) : (j < g.G ? g.glob[j] : 0);
  }
  heap.sort_keys_ascending(cnt);
  // Three-way merge of ascending streams: LSH keys, the window, the globals
  // (+ key 0 from the fallback). Self is excluded and takes slot 0 (:1043-1076).
  int32_t* nbo = g.nb + ((int64_t)bh * g.N + n) * g.Wout;
  uint8_t* vo = g.valid + ((int64_t)bh * g.N + n) * g.Wout;
  int slot = 0;
  if (!g.is_cross) {
    nbo[0] = min(na, g.M - 1);  // merge's final clamp to the true maximum index
    vo[0] = 1;
    slot = 1;
  }
  const int ng = gs[g.G];
  const int kw = g.is_cross ? 0 : 2 * g.window + 1;
  int il = 0, iw = 0, ig = 0;
  bool zero_pending = add_zero;
  int last = -1;
  const int BIG = 0x7fffffff;
  while (slot < g.Wout) {
    const int vl = il < cnt ? heap.key(il) : BIG;
    int vw = BIG;
    if (iw < kw) {
      const int o = iw - g.window;
      int idx = (g.causal && o > 0) ? na : na + o;
      idx = idx < 0 ? 0 : (idx > g.M - 1 ? g.M - 1 : idx);
      vw = idx;
    }
    const int vg = ig < ng ? gs[ig] : BIG;
    const int vz = zero_pending ? 0 : BIG;
    const int v = min(min(vl, vw), min(vg, vz));
    if (v == BIG) break;
    if (v == vl) ++il;
    else if (v == vw) ++iw;
    else if (v == vg) ++ig;
    else zero_pending = false;
    if (v == last || (!g.is_cross && v == na)) continue;
    last = v;
    nbo[slot] = v;
    vo[slot] = 1;
    ++slot;
  }
  for (; slot < g.Wout; ++slot) {
    nbo[slot] = 0;
    vo[slot] = 0;
  }
}

}  // namespace ssa
