// ssa_select_rows.cu -- per-query-row stages of the tensor-core graph build.
//
//   k_hash_queries  four lanes per query row: the row's bucket id per
//                   (round, probe) slot and whether any of those buckets is
//                   empty.
//   k_rows          warp per query row, after a scan pass of k_scan_tc:
//     THRESH mode   from the sampled candidates, tau = the x-th largest score
//                   (x ~ 3A scaled by the sampled fraction of key tiles),
//                   rounded down to its upper 16 bits: a per-row threshold
//                   the full scan uses to keep only ~3A candidates.
//     FINAL mode    verifies that at least A candidates reached tau (then
//                   every top-A member did), adds the special keys (pad keys,
//                   causal self, empty-bucket fallbacks) after replaying the
//                   reference's slot order for each, selects the exact top-A
//                   by range-narrowing histograms, and writes the merged neighbor
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
// Four lanes per query row (each holds a quarter of the row, see
// proj_planes_x4) and two rows per four lanes, sixteen rows per warp: each
// hyperplane element read from shared memory serves two rows. Lane 0 of each
// row's four writes its (round, probe) bucket offsets and the empty-bucket
// flag.
template <int DT, int D, bool SMEM>
__global__ void __launch_bounds__(256, 2) k_hash_queries(GraphDev g) {
  constexpr int RW = 2, EPL = D / 4;  // the probes' projections take registers too: two rows
  extern __shared__ __align__(16) float s_planes[];  // SMEM: R * p hyperplanes of d floats
  const int pd = g.p * g.d;
  if (SMEM) {
    for (int i = threadIdx.x * 4; i < g.R * pd; i += blockDim.x * 4) {
      const int r = i / pd, rem = i - r * pd;
      *reinterpret_cast<float4*>(s_planes + i) =
          __ldg(reinterpret_cast<const float4*>(g.rp + (int64_t)r * g.max_p * g.d + rem));
    }
    __syncthreads();
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane & 3;
  const int64_t total = (int64_t)g.B * g.H * g.N;
  const int64_t base = ((int64_t)blockIdx.x * 8 + warp) * (8 * RW) + (lane >> 2);
  int64_t rows[RW];
  int bgs[RW];
  bool writer[RW], empty[RW];
  float xs[RW * EPL];
#pragma unroll
  for (int w = 0; w < RW; ++w) {
    rows[w] = base + 8 * w;
    const bool act = rows[w] < total;  // no early exit: the four lanes of a row shuffle together
    const int64_t rr = act ? rows[w] : 0;
    const int n = (int)(rr % g.N);
    const int64_t bh = rr / g.N;
    const int b = (int)(bh / g.H), h = (int)(bh % g.H);
    bgs[w] = b * g.n_kv + h / g.rep;
    writer[w] = act && sub == 0;
    empty[w] = false;
    load_slice_x4<DT, D>(row_ptr<DT>(g.q, b * g.q_sb + h * g.q_sh + (int64_t)n * g.q_sn), g.d, sub, act,
                         xs + w * EPL);
  }
  for (int rd = 0; rd < g.R; ++rd) {
    float proj[RW][12];
    uint32_t id[RW];
#pragma unroll
    for (int w = 0; w < RW; ++w) {
      id[w] = 0;
#pragma unroll
      for (int j = 0; j < 12; ++j) proj[w][j] = 0.f;
    }
    const float* pl = SMEM ? s_planes + rd * pd : g.rp + (int64_t)rd * g.max_p * g.d;
    for_round_projections_x4<D, SMEM, RW>(xs, pl, g.d, g.p, sub, [&](int j, int w, float v) {
      if (v > 0.f) id[w] |= 1u << j;  // proj > 0, strict (:589)
      proj[w][j] = v;
    });
#pragma unroll
    for (int w = 0; w < RW; ++w) {
      if (!writer[w]) continue;
      // primary bucket, then probe t flips the bit with the t-th smallest
      // |proj| of the original id, ties in plane order (:599-646)
      const int32_t* bs = g.bsize + (int64_t)(bgs[w] * g.R + rd) * g.NB;
      const int tt0 = rd * (1 + g.Te);
      g.qids[(int64_t)tt0 * total + rows[w]] = (uint16_t)(rd * g.NB + id[w]);
      empty[w] |= __ldg(bs + id[w]) == 0;
      uint32_t used = 0;
      for (int t = 0; t < g.Te; ++t) {
        int best = -1;
        float bmag = 0.f;
#pragma unroll
        for (int j = 0; j < 12; ++j) {
          if (j < g.p && !((used >> j) & 1u)) {
            const float a = fabsf(proj[w][j]);
            if (best < 0 || a < bmag) { best = j; bmag = a; }
          }
        }
        used |= 1u << best;
        const uint32_t pid = id[w] ^ (1u << best);
        g.qids[(int64_t)(tt0 + 1 + t) * total + rows[w]] = (uint16_t)(rd * g.NB + pid);
        empty[w] |= __ldg(bs + pid) == 0;
      }
    }
  }
#pragma unroll
  for (int w = 0; w < RW; ++w)
    if (writer[w]) g.qempty[rows[w]] = empty[w] ? 1 : 0;
}

// ---------------------------------------------------------------------------
// Warp helpers
// ---------------------------------------------------------------------------

// The kth largest 16-bit order key among the candidates of a row's sample:
// ntiles records of kSampleTileBytes (128 upper score halves, then the 128-bit
// candidate mask). 2-pass, 8-bit radix select; lane L reads scores 4L..4L+3
// of each record. The first pass reads the records and keeps each lane's
// candidate keys (up to kThreshCache of them) in `cache` ([kThreshCache][32]),
// so the second pass reads shared memory, not the records again.
constexpr int kThreshCache = 64;

__device__ __forceinline__ void hist_find(uint32_t* hist, int need, int* bin_out, int* before_out) {
  const int lane = threadIdx.x & 31;
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
  uint32_t before = incl - tot;
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
  const int src_lane = __ffs(who) - 1;  // exists: the histogram holds at least `need` entries
  *bin_out = __shfl_sync(0xffffffffu, found_bin, src_lane);
  *before_out = (int)__shfl_sync(0xffffffffu, found_before, src_lane);
}

// Reads every candidate's 16-bit order key of the sample (lane L: scores
// 4L..4L+3 of each record) and calls f(u) for each.
template <typename F>
__device__ __forceinline__ void for_sample_keys(const unsigned char* base, int ntiles, F&& f) {
  const int lane = threadIdx.x & 31;
  for (int j0 = 0; j0 < ntiles; j0 += 4) {
    uint2 kv[4];
    uint32_t mw[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {  // four records' loads in flight before any use
      const unsigned char* tb = base + (size_t)(j0 + u) * kSampleTileBytes;
      const bool in = j0 + u < ntiles;
      kv[u] = in ? *reinterpret_cast<const uint2*>(tb + 8 * lane) : make_uint2(0u, 0u);
      mw[u] = in ? *reinterpret_cast<const uint32_t*>(tb + 256 + 4 * (lane >> 3)) : 0u;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t m4 = (mw[u] >> ((4 * lane) & 31)) & 0xFu;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if ((m4 >> q) & 1u) {
          const uint32_t h = ((q < 2 ? kv[u].x : kv[u].y) >> (16 * (q & 1))) & 0xFFFFu;
          f((h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u));  // okey of the upper half
        }
      }
    }
  }
}

__device__ uint32_t warp_sample_kth(const unsigned char* base, int ntiles, int kth, uint32_t* hist,
                                    uint16_t* cache) {
  const int lane = threadIdx.x & 31;
  // Pass 1 (the records): this lane's candidates into the cache, and the
  // range [umin, umax] of all of them.
  int k = 0;
  uint32_t umin = 0xFFFFu, umax = 0u;
  for_sample_keys(base, ntiles, [&](uint32_t u) {
    if (k < kThreshCache) cache[k * 32 + lane] = (uint16_t)u;
    ++k;
    umin = min(umin, u);
    umax = max(umax, u);
  });
  umin = __reduce_min_sync(0xffffffffu, umin);
  umax = __reduce_max_sync(0xffffffffu, umax);
  if (umin == umax) return umin;
  const bool cached = !__any_sync(0xffffffffu, k > kThreshCache);
  const int kc = min(k, kThreshCache);
  // Pass 2: 256 bins of width 2^sh over [umin, umax] (spread over the range,
  // so the shared-memory atomics rarely collide).
  const uint32_t span1 = umax - umin;
  const int bl = 32 - __clz(span1);
  const int sh = bl > 8 ? bl - 8 : 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) hist[lane * 8 + j] = 0;
  __syncwarp();
  auto add_top = [&](uint32_t u) { atomicAdd(&hist[(u - umin) >> sh], 1u); };
  if (cached) {
    for (int t = 0; t < kc; ++t) add_top(cache[t * 32 + lane]);
  } else {
    for_sample_keys(base, ntiles, add_top);
  }
  __syncwarp();
  int bin, before;
  hist_find(hist, kth, &bin, &before);
  const uint32_t lo = umin + ((uint32_t)bin << sh);
  if (sh == 0) return lo;
  // Pass 3: the low sh bits of the keys in that bin.
  const int need = kth - before;
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 8; ++j) hist[lane * 8 + j] = 0;
  __syncwarp();
  const uint32_t lmask = (1u << sh) - 1u;
  auto add_low = [&](uint32_t u) {
    if (((u - umin) >> sh) == (uint32_t)bin) atomicAdd(&hist[(u - umin) & lmask], 1u);
  };
  if (cached) {
    for (int t = 0; t < kc; ++t) add_low(cache[t * 32 + lane]);
  } else {
    for_sample_keys(base, ntiles, add_low);
  }
  __syncwarp();
  int bin2, before2;
  hist_find(hist, need, &bin2, &before2);
  __syncwarp();
  return lo + (uint32_t)bin2;
}

// Descending bitonic sort of one value per lane.
__device__ __forceinline__ uint32_t warp_sort_desc(uint32_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k2 = 2; k2 <= 32; k2 <<= 1) {
#pragma unroll
    for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1) {
      const uint32_t o = __shfl_xor_sync(0xffffffffu, v, j2);
      const bool asc = (lane & k2) == 0, lower = (lane & j2) == 0;
      v = (lower != asc) ? min(v, o) : max(v, o);
    }
  }
  return v;
}

// Narrows [ulo, uhi] -- an order-key range of ok[0..n) holding the entry of
// rank `need` (1-based, from the top) among the entries inside the range --
// by rounds of 256-bin histograms of the entries in the range (bin width 2^s,
// s the smallest shift that fits it), keeping the bin that holds that rank and
// updating `need` to the rank within it. Stops when the range is a single key
// (returns 0) or its bin holds at most 32 entries (returns their count).
// Warp-collective.
__device__ int warp_narrow_kth(const uint32_t* ok, int n, uint32_t& ulo, uint32_t& uhi, int& need,
                               uint32_t* hist) {
  const int lane = threadIdx.x & 31;
  while (ulo != uhi) {
    const uint32_t span1 = uhi - ulo;  // span - 1
    const int bl = 32 - __clz(span1);
    const int sh = bl > 8 ? bl - 8 : 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) hist[lane * 8 + j] = 0;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
      const uint32_t u = ok[i];
      if (u >= ulo && u <= uhi) atomicAdd(&hist[(u - ulo) >> sh], 1u);
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
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    uint32_t before = incl - tot;  // entries in higher bins than this lane's
    int found_bin = -1;
    uint32_t found_before = 0, found_cnt = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (found_bin < 0 && before < (uint32_t)need && before + c[j] >= (uint32_t)need) {
        found_bin = 255 - (lane * 8 + j);
        found_before = before;
        found_cnt = c[j];
      }
      before += c[j];
    }
    const unsigned who = __ballot_sync(0xffffffffu, found_bin >= 0);
    const int src = __ffs(who) - 1;  // exists: the range holds at least `need` entries
    const uint32_t bin = (uint32_t)__shfl_sync(0xffffffffu, found_bin, src);
    need -= (int)__shfl_sync(0xffffffffu, found_before, src);
    const uint32_t cb = __shfl_sync(0xffffffffu, found_cnt, src);
    const uint32_t nlo = ulo + (bin << sh);
    const uint32_t nhi = (sh == 0) ? nlo : min(uhi, nlo + ((1u << sh) - 1u));
    ulo = nlo;
    uhi = nhi;
    __syncwarp();
    if (ulo != uhi && cb <= 32u) return (int)cb;
  }
  return 0;
}

// The key T of rank `need` among the cb (<= 32) entries of ok[0..n) inside
// [ulo, uhi], found by sorting them across the warp; *need_out = how many
// entries equal to T belong to the selection. `list` holds 32 entries.
// Warp-collective.
__device__ uint32_t warp_kth_in_bin(const uint32_t* ok, int n, uint32_t ulo, uint32_t uhi, int need, int cb,
                                    uint32_t* list, int* need_out) {
  const int lane = threadIdx.x & 31;
  int k = 0;
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int i = i0 + lane;
    uint32_t u = 0u;
    bool m = false;
    if (i < n) {
      u = ok[i];
      m = u >= ulo && u <= uhi;
    }
    const unsigned bm = __ballot_sync(0xffffffffu, m);
    if (m) list[k + __popc(bm & ((1u << lane) - 1u))] = u;
    k += __popc(bm);
  }
  __syncwarp();
  const uint32_t v = warp_sort_desc(lane < cb ? list[lane] : 0u);
  const uint32_t T = __shfl_sync(0xffffffffu, v, need - 1);
  const int gt = __popc(__ballot_sync(0xffffffffu, lane < cb && v > T));
  __syncwarp();
  *need_out = need - gt;
  return T;
}

struct RowsSmem {
  uint32_t* ok;     // [max(cap, Wout)] order keys of the scores; later the staged neighbor row
  uint16_t* ky;     // [cap] keys (the tensor-core path has M <= 65536)
  uint32_t* hist;   // [256]
  uint32_t* bits;   // [Mw] merge bitmap over [0, M)
  uint32_t* l1;     // [64] nonzero words of `bits`
  int32_t* spec;    // [64] special keys, then the ones that need a dot product
  uint8_t* sflag;   // [32 * NT] replay flags
};

// Shared-memory bytes per warp of k_rows: THRESH needs only the histogram.
__host__ __device__ inline size_t rows_warp_bytes(const GraphDev& g, int stage) {
  if (stage == 0) return 256 * 4 + kThreshCache * 32 * 2;
  const int cap = g.capg + 64;
  const int scn = cap > g.Wout ? cap : g.Wout;
  const int Mw = (g.M + 31) / 32;
  const size_t b = (size_t)scn * 4 + (((size_t)cap * 2 + 15) & ~size_t(15)) + 256 * 4 + (size_t)Mw * 4 +
                   64 * 4 + 64 * 4 + 32 * (size_t)g.NT;
  return (b + 15) & ~size_t(15);
}

// ---------------------------------------------------------------------------
// k_rows
// ---------------------------------------------------------------------------
// One instantiation per stage (0 = THRESH, 1 = FINAL) and output mode (FINAL:
// 0 = merged neighbor rows, 1 = LSH rows in topk order), so each kernel
// carries only its own code.
template <int DT, int D, int STAGE, int MODE>
__global__ void __launch_bounds__(128, 8) k_rows(GraphDev g) {
  constexpr int stage = STAGE, mode = MODE;
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cap = g.capg + 64;
  const int scn = cap > g.Wout ? cap : g.Wout;
  const int Mw = (g.M + 31) / 32;
  const int nl1 = (Mw + 31) / 32;
  unsigned char* base = smem + warp * rows_warp_bytes(g, stage);
  RowsSmem S;
  uint16_t* tcache = nullptr;
  if (stage == 0) {
    S.hist = reinterpret_cast<uint32_t*>(base);
    tcache = reinterpret_cast<uint16_t*>(S.hist + 256);
  } else {
    S.ok = reinterpret_cast<uint32_t*>(base);
    S.ky = reinterpret_cast<uint16_t*>(S.ok + scn);
    S.hist = reinterpret_cast<uint32_t*>(base + (size_t)scn * 4 + (((size_t)cap * 2 + 15) & ~size_t(15)));
    S.bits = S.hist + 256;
    S.l1 = S.bits + Mw;
    S.spec = reinterpret_cast<int32_t*>(S.l1 + 64);
    S.sflag = reinterpret_cast<uint8_t*>(S.spec + 64);
    for (int i = lane; i < Mw; i += 32) S.bits[i] = 0;
    for (int i = lane; i < 64; i += 32) S.l1[i] = 0;
  }
  __syncwarp();

  const int64_t total = (int64_t)g.B * g.H * g.N;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp; row < total; row += nwarps) {
    // 32-bit division: the tensor-core path has fewer than 2^31 rows.
    const uint32_t bh32 = (uint32_t)row / (uint32_t)g.N;
    const int n = (int)((uint32_t)row - bh32 * (uint32_t)g.N);  // row within q and the outputs
    const int na = g.row0 + n;        // its sequence position (causal limit, window, self)
    const int64_t bh = bh32;
    const int b = (int)(bh32 / (uint32_t)g.H), h = (int)(bh32 - (uint32_t)b * (uint32_t)g.H);
    const int gk = h / g.rep;
    const int bg = b * g.n_kv + gk;
    // Two scan groups (even / odd key tiles) each fill half of the buffer.
    const int half_cap = g.capg >> 1;
    const int cnt0 = g.rcnt[row * 2], cnt1 = g.rcnt[row * 2 + 1];
    const int cnt_all = cnt0 + cnt1;
    const unsigned long long* bo = g.buf + row * g.capg;
    if (stage == 0) {
      // ---- THRESH: tau = x-th largest sampled score ----------------------
      const int tiles_row = g.causal ? (na + 127) / 128 : (g.M + 127) / 128;
      const int sampled = tiles_row > 0 ? (tiles_row + g.sample_s - 1) / g.sample_s : 0;
      float tau = -INFINITY;
      if (sampled > 0 && tiles_row > 0) {
        // x ~ 3A scaled by the sampled fraction: about 3A candidates are
        // expected at or above tau, so fewer than A (the fallback case) is
        // a 3x deviation, and more than the buffer holds (6A+64) a 2x one.
        const int x = (int)(((int64_t)3 * g.A * sampled + tiles_row - 1) / tiles_row);
        // The sample holds the upper 16 bits of each score's order key, so
        // tau is rounded down to the lowest score sharing the x-th key: at
        // least x sampled scores are >= tau.
        const int fit = (int)((size_t)g.capg * 8 / kSampleTileBytes);
        if (x >= 1 && cnt_all >= x && sampled <= fit)
          tau = okey_inv(warp_sample_kth(reinterpret_cast<const unsigned char*>(bo), sampled, x, S.hist, tcache)
                         << 16);
      }
      if (lane == 0) g.tau[row] = tau;
      __syncwarp();
      continue;
    }

    // ---- FINAL -------------------------------------------------------------
    const float tau = g.tau[row];
    const int ntq = (g.N + 127) / 128;
    if (cnt0 > half_cap || cnt1 > half_cap || (tau > -INFINITY && cnt_all < g.A)) {
      if (lane == 0) g.tile_flags[bh * ntq + n / 128] = 1;  // exact fallback for this tile
      continue;
    }
    const int c = cnt_all;
    // The select's starting range is gathered on the way: the order keys at or
    // above lo = okey(tau) (count, min, max) and the min / max of all of them.
    const uint32_t lo = tau > -INFINITY ? okey(tau == 0.f ? -0.f : tau) : 0u;
    uint32_t mn1 = 0xFFFFFFFFu, mx1 = 0u, c1 = 0u, mn0 = 0xFFFFFFFFu, mx0 = 0u;
    auto note_key = [&](uint32_t u) {
      mn0 = min(mn0, u);
      mx0 = max(mx0, u);
      if (u >= lo) {
        mn1 = min(mn1, u);
        mx1 = max(mx1, u);
        ++c1;
      }
    };
    // Two entries per 16-byte load (each half starts 16-byte aligned; an odd
    // count's last load also reads the unused slot after it, inside the half),
    // four loads in flight per lane.
    for (int hf = 0; hf < 2; ++hf) {
      const int ch = hf ? cnt1 : cnt0;
      const ulonglong2* src = reinterpret_cast<const ulonglong2*>(bo + (hf ? half_cap : 0));
      const int base = hf ? cnt0 : 0;
      constexpr int U = 4;  // loads in flight per lane before any is used
      for (int p0 = lane; 2 * p0 < ch; p0 += 32 * U) {
        ulonglong2 e[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int pi = p0 + 32 * u;
          e[u] = 2 * pi < ch ? __ldcs(src + pi) : make_ulonglong2(0ull, 0ull);  // read once
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int pi = p0 + 32 * u;
          if (2 * pi < ch) {
            const uint32_t u0 = okey(__uint_as_float((uint32_t)e[u].x));
            S.ok[base + 2 * pi] = u0;
            S.ky[base + 2 * pi] = (uint16_t)(e[u].x >> 32);
            note_key(u0);
            if (2 * pi + 1 < ch) {
              const uint32_t u1 = okey(__uint_as_float((uint32_t)e[u].y));
              S.ok[base + 2 * pi + 1] = u1;
              S.ky[base + 2 * pi + 1] = (uint16_t)(e[u].y >> 32);
              note_key(u1);
            }
          }
        }
      }
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
    int xs = -1;
    if (lane < g.R) {
      xs = (int)(g.pmax[bg * g.R + lane] & 0xFFFFFu);
      if (g.causal && xs > na) xs = -1;  // a future pad key never appears as itself
    } else if (lane == g.R) {
      xs = g.causal ? na : -1;
    } else if (lane < ncand - 1) {
      xs = g.glob[lane - g.R - 1];
    } else if (lane == ncand - 1 && any_empty) {
      xs = g.G < g.C ? 0 : -1;
    }
    if (xs >= g.M) xs = -1;
    const unsigned same = __match_any_sync(0xffffffffu, xs);  // every lane takes part
    const bool keep = xs >= 0 && lane == __ffs(same) - 1;
    const unsigned km = __ballot_sync(0xffffffffu, keep);
    // key in the low 24 bits; above them 1 + the slot of its full-scan score
    // (pad key of round r: r; causal self: R), 0 if the scan keeps none
    const int src1 = lane <= g.R ? lane + 1 : 0;
    if (keep) S.spec[__popc(km & ((1u << lane) - 1u))] = xs | (src1 << 24);
    const int nspec = __popc(km);
    __syncwarp();
    const uint16_t* toffs = g.qids + row;  // slot tt at toffs[tt * total]: r * NB + bucket
    // Replay, lane-parallel over (key, slot) pairs: flag 1 = key's slot in
    // this (round, probe) bucket is a real member, 2 = it is the overflow pad,
    // 0 = absent (or the bucket is empty: handled as a third state 3 = present
    // via the empty-bucket fallback list). Four pairs per lane per step, all
    // loads issued before any is used.
    auto replay = [&](int p) -> uint8_t {
      const int i = p / g.NT, tt = p - i * g.NT;
      const int x = S.spec[i] & 0xFFFFFF;
      const int off = __ldg(toffs + (int64_t)tt * total);
      const int r = off >> g.p;
      const int u = off & (g.NB - 1);
      const int64_t tb = (int64_t)bg * g.R * g.NB + off;
      const int sz = __ldg(g.bsize + tb);
      const int lc = __ldg(g.lastc + tb);
      const uint32_t pm = __ldg(g.pmax + bg * g.R + r);
      const uint16_t code = __ldg(g.kcode + ((int64_t)bg * g.R + r) * g.M + x);
      const unsigned long long wbits =
          __ldg(&g.bmap[bmap_idx(g, bg, x >> 6, r, u)]);
      const bool member = code == (uint16_t)u && ((wbits >> (x & 63)) & 1ull);
      uint8_t f = 0;
      if (sz == 0) {
        bool in = false;
        for (int cc = 0; cc < lim_g; ++cc) in |= g.glob[cc] == x;
        if (g.G < g.C && x == 0) in = true;
        f = in ? 3 : 0;
      } else {
        bool real;
        if (g.causal && x > na) real = false;
        else if (g.causal && x == na) real = lc > na || member;
        else real = member;
        if (real) f = 1;
        else if (sz < g.C) {
          int P = (int)(pm & 0xFFFFFu);
          if (g.causal && P > na) P = na;
          if (P == x) f = 2;
        }
      }
      return f;
    };
    const int npairs = nspec * g.NT;
    for (int p0 = 0; p0 < npairs; p0 += 128) {
      uint8_t f[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int p = p0 + j * 32 + lane;
        f[j] = p < npairs ? replay(p) : 0;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int p = p0 + j * 32 + lane;
        if (p < npairs) S.sflag[p] = f[j];
      }
    }
    __syncwarp();
    // Lane i decides special i: eligible iff its first appearance is valid.
    // An eligible key that the scan did not already keep needs its score:
    // pad keys and causal self were scored by the full scan (sspec); any
    // other (an empty-bucket fallback) gets a dot product below.
    bool need_dot = false, captured = false;
    int xk = 0;
    if (lane < nspec) {
      const int e = S.spec[lane];
      xk = e & 0xFFFFFF;
      const int src = (e >> 24) - 1;
      bool elig = false;
      for (int tt = 0; tt < g.NT; ++tt) {
        const uint8_t f = S.sflag[lane * g.NT + tt];
        if (f == 0) continue;
        elig = f != 2;
        break;
      }
      if (elig) {
        const bool scanned =
            !((__ldg(g.pmask + (int64_t)bg * g.Wpad + (xk >> 6)) >> (xk & 63)) & 1ull) && !(g.causal && xk >= na);
        if (scanned) {
          bool present = false;
          for (int z = 0; z < c && !present; ++z) present = (int)S.ky[z] == xk;
          need_dot = !present;
        } else if (src >= 0) {
          captured = true;
        } else {
          need_dot = true;
        }
      }
    }
    // Captured scores go right after the buffered entries.
    const unsigned cpm = __ballot_sync(0xffffffffu, captured);
    if (captured) {
      const int src = (S.spec[lane] >> 24) - 1;
      const int pos = c + __popc(cpm & ((1u << lane) - 1u));
      const uint32_t u = okey(__ldg(g.sspec + row * (g.R + 1) + src));
      S.ok[pos] = u;
      S.ky[pos] = (uint16_t)xk;
      note_key(u);
    }
    const int cc = c + __popc(cpm);
    const unsigned dm = __ballot_sync(0xffffffffu, need_dot);
    const int ndot = __popc(dm);
    if (need_dot) S.spec[32 + __popc(dm & ((1u << lane) - 1u))] = xk;
    __syncwarp();
    // Scores of those keys: 8 lanes per key, D/8 elements per lane.
    if (ndot > 0) {
      constexpr int E = D / 8;
      const int grp = lane >> 3, sub = lane & 7;
      float qv[E];
      const void* qrow = row_ptr<DT>(g.q, b * g.q_sb + h * g.q_sh + (int64_t)n * g.q_sn);
#pragma unroll
      for (int e = 0; e < E; e += 8) {
        if (sub * E + e < g.d) {
          load8<DT>(qrow, sub * E + e, qv + e);
        } else {
#pragma unroll
          for (int z = 0; z < 8; ++z) qv[e + z] = 0.f;
        }
      }
      for (int j0 = 0; j0 < ndot; j0 += 4) {
        const int j = j0 + grp;
        float acc = 0.f;
        if (j < ndot) {
          const int x = S.spec[32 + j];
          const void* krow = row_ptr<DT>(g.k, b * g.k_sb + gk * g.k_sh + (int64_t)x * g.k_sm);
#pragma unroll
          for (int e = 0; e < E; e += 8) {
            if (sub * E + e < g.d) {
              float kv[8];
              load8<DT>(krow, sub * E + e, kv);
#pragma unroll
              for (int z = 0; z < 8; ++z) acc = fmaf(qv[e + z], kv[z], acc);
            }
          }
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        acc += __shfl_xor_sync(0xffffffffu, acc, 4);
        if (j < ndot && sub == 0) {
          const uint32_t u = okey(acc);
          S.ok[cc + j] = u;
          S.ky[cc + j] = (uint16_t)S.spec[32 + j];
          note_key(u);
        }
      }
    }
    const int tot = cc + ndot;
    __syncwarp();

    // Exact top-A (the whole pool when it has at most A entries). At least A
    // entries reached tau, so the A-th largest is >= tau and only those take
    // part in the select (all entries if fewer than A did).
    const int n_elig = min(tot, g.A);
    if (tot > g.A) {
      const bool above = (int)__reduce_add_sync(0xffffffffu, c1) >= g.A;
      uint32_t ulo = __reduce_min_sync(0xffffffffu, above ? mn1 : mn0);
      uint32_t uhi = __reduce_max_sync(0xffffffffu, above ? mx1 : mx0);
      int need = g.A;
      const int cb = warp_narrow_kth(S.ok, tot, ulo, uhi, need, S.hist);
      uint32_t* list_u = reinterpret_cast<uint32_t*>(S.spec);  // [32]; the special keys are done
      int wpos = 0;
      if (mode == 0 && cb > 0) {
        // One pass: entries above the bin go to the front; the bin's cb
        // entries are collected (index order), sorted to find the rank-`need`
        // key T, and the selected ones follow: those above T, then the first
        // entries equal to T.
        uint16_t* list_k = reinterpret_cast<uint16_t*>(S.spec + 32);
        int lc = 0;
        for (int i0 = 0; i0 < tot; i0 += 32) {
          const int i = i0 + lane;
          const bool in = i < tot;
          const uint32_t u = in ? S.ok[i] : 0u;
          const uint16_t kv = in ? S.ky[i] : 0;
          const bool top = in && u > uhi;
          const bool mid = in && u >= ulo && u <= uhi;
          const unsigned tm = __ballot_sync(0xffffffffu, top);
          const unsigned mm = __ballot_sync(0xffffffffu, mid);
          __syncwarp();
          if (top) {
            const int dst = wpos + __popc(tm & ((1u << lane) - 1u));
            S.ok[dst] = u;
            S.ky[dst] = kv;
          }
          if (mid) {
            const int li = lc + __popc(mm & ((1u << lane) - 1u));
            list_u[li] = u;
            list_k[li] = kv;
          }
          __syncwarp();
          wpos += __popc(tm);
          lc += __popc(mm);
        }
        const bool inl = lane < cb;
        const uint32_t lu = inl ? list_u[lane] : 0u;
        const uint32_t v = warp_sort_desc(lu);
        const uint32_t T = __shfl_sync(0xffffffffu, v, need - 1);
        const int need_eq = need - __popc(__ballot_sync(0xffffffffu, inl && v > T));
        const bool eq = inl && lu == T;
        const int eq_rank = __popc(__ballot_sync(0xffffffffu, eq) & ((1u << lane) - 1u));
        const bool sel = inl && (lu > T || (eq && eq_rank < need_eq));
        const unsigned sm = __ballot_sync(0xffffffffu, sel);
        if (sel) {
          const int dst = wpos + __popc(sm & ((1u << lane) - 1u));
          S.ok[dst] = lu;
          S.ky[dst] = list_k[lane];
        }
      } else {
        int need_t = need;
        const uint32_t T = cb > 0 ? warp_kth_in_bin(S.ok, tot, ulo, uhi, need, cb, list_u, &need_t) : ulo;
        // Compact the selection to the front: keys > T, then `need_t` keys
        // == T in index order (ties are the reference's unspecified topk order).
        int eq_seen = 0;
        for (int i0 = 0; i0 < tot; i0 += 32) {
          const int i = i0 + lane;
          const bool in = i < tot;
          const uint32_t u = in ? S.ok[i] : 0u;
          const uint16_t kv = in ? S.ky[i] : 0;
          const bool eq = in && u == T;
          const unsigned eqm = __ballot_sync(0xffffffffu, eq);
          const int eq_rank = eq_seen + __popc(eqm & ((1u << lane) - 1u));
          const bool sel = in && (u > T || (eq && eq_rank < need_t));
          const unsigned sm = __ballot_sync(0xffffffffu, sel);
          __syncwarp();
          if (sel) {
            const int dst = wpos + __popc(sm & ((1u << lane) - 1u));
            S.ok[dst] = u;
            S.ky[dst] = kv;
          }
          __syncwarp();
          wpos += __popc(sm);
          eq_seen += __popc(eqm);
        }
      }
    }
    __syncwarp();

    if (mode == 1) {
      // Reference topk order: descending score. Bitonic sort of n_elig
      // entries by order key (padded to a power of two with key 0, below
      // every score's) in shared memory.
      int P2 = 32;
      while (P2 < n_elig) P2 <<= 1;
      for (int i = n_elig + lane; i < P2; i += 32) {
        S.ok[i] = 0u;
        S.ky[i] = 0xFFFF;
      }
      __syncwarp();
      for (int k2 = 2; k2 <= P2; k2 <<= 1) {
        for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1) {
          for (int i = lane; i < P2; i += 32) {
            const int ixj = i ^ j2;
            if (ixj > i) {
              const bool desc = (i & k2) == 0;
              const uint32_t a = S.ok[i], bb = S.ok[ixj];
              if ((a < bb) == desc) {
                S.ok[i] = bb;
                S.ok[ixj] = a;
                const uint16_t t0 = S.ky[i];
                S.ky[i] = S.ky[ixj];
                S.ky[ixj] = t0;
              }
            }
          }
          __syncwarp();
        }
      }
      int32_t* out = g.lsh + row * g.A;
      for (int j = lane; j < g.A; j += 32) out[j] = j < n_elig ? (int)S.ky[j] : (j < g.G ? g.glob[j] : 0);
      __syncwarp();
      continue;
    }
    if (g.lsh) {
      int32_t* out = g.lsh + row * g.A;
      for (int j = lane; j < g.A; j += 32) out[j] = j < n_elig ? (int)S.ky[j] : (j < g.G ? g.glob[j] : 0);
    }
    // ---- merge: self, then the ascending union of window, globals, LSH keys
    // and key 0 from the fallback slots, self excluded. The window is a
    // contiguous key range [wlo, whi] (indices clamped to [0, M), causal
    // offsets > 0 mapped to self), so only the other keys go through a
    // bitmap; the window's keys then take consecutive slots after the
    // bitmap keys below wlo.
    const bool add_zero = max(n_elig, g.G) < g.A;
    const bool drop_self = !g.is_cross && na < g.M;
    int wlo = 1, whi = 0, nwin = 0;
    if (!g.is_cross) {
      wlo = min(max(na - g.window, 0), g.M - 1);
      whi = min(max(g.causal ? na : na + g.window, 0), g.M - 1);
      nwin = whi - wlo + 1 - ((drop_self && na >= wlo && na <= whi) ? 1 : 0);
    }
    int xhi = -1;  // largest key this lane marked
    auto mark = [&](int x) {
      if (x >= wlo && x <= whi) return;  // window key (or self inside it)
      if (drop_self && x == na) return;
      xhi = max(xhi, x);
      const uint32_t old = atomicOr(&S.bits[x >> 5], 1u << (x & 31));
      if (old == 0u) atomicOr(&S.l1[x >> 10], 1u << ((x >> 5) & 31));
    };
    for (int j = lane; j < n_elig; j += 32) mark(S.ky[j]);
    for (int j = lane; j < g.G; j += 32) mark(min(max(g.glob[j], 0), g.M - 1));
    if (add_zero && lane == 0) mark(0);
    __syncwarp();
    // Lane L owns bitmap words [L*wpl, (L+1)*wpl) of the words in use (up to
    // the largest marked key: under causal masking a row's keys lie below
    // its position, so the lanes share that prefix evenly) and visits the
    // nonzero ones through the summary words: count its keys (and those
    // below wlo), exclusive-scan across lanes, then emit.
    const int xmax = __reduce_max_sync(0xffffffffu, xhi);
    const int Mu = xmax >= 0 ? (xmax >> 5) + 1 : 0;
    const int wpl = (Mu + 31) / 32;
    const int w0 = min(lane * wpl, Mu), w1 = min(w0 + wpl, Mu);
    auto lane_words = [&](int l) -> uint32_t {
      uint32_t m1 = S.l1[l];
      const int lb = l * 32;
      if (w0 > lb) m1 &= ~((1u << (w0 - lb)) - 1u);
      if (w1 < lb + 32) m1 &= (1u << (w1 - lb)) - 1u;
      return m1;
    };
    int cnt = 0, below = 0;
    if (w0 < w1) {
      for (int l = w0 >> 5; l <= (w1 - 1) >> 5; ++l) {
        uint32_t m1 = lane_words(l);
        while (m1) {
          const int wd = l * 32 + __ffs(m1) - 1;
          m1 &= m1 - 1u;
          const uint32_t bw = S.bits[wd];
          cnt += __popc(bw);
          const int lo_rel = wlo - wd * 32;  // keys below wlo in this word
          if (lo_rel >= 32) below += __popc(bw);
          else if (lo_rel > 0) below += __popc(bw & ((1u << lo_rel) - 1u));
        }
      }
    }
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    const int nlg = __shfl_sync(0xffffffffu, incl, 31);
    const int nbelow = __reduce_add_sync(0xffffffffu, below);
    const int s0 = g.is_cross ? 0 : 1;
    int* stage_out = reinterpret_cast<int*>(S.ok);  // the scores are no longer needed
    __syncwarp();
    if (w0 < w1) {
      int rank = incl - cnt;
      for (int l = w0 >> 5; l <= (w1 - 1) >> 5; ++l) {
        uint32_t m1 = lane_words(l);
        while (m1) {
          const int wd = l * 32 + __ffs(m1) - 1;
          m1 &= m1 - 1u;
          uint32_t bw = S.bits[wd];
          S.bits[wd] = 0u;
          while (bw) {
            const int x = wd * 32 + __ffs(bw) - 1;
            bw &= bw - 1u;
            const int slot = s0 + rank + (x > whi ? nwin : 0);
            if (slot < g.Wout) stage_out[slot] = x;
            ++rank;
          }
        }
      }
    }
    __syncwarp();
    for (int j = lane; j < nwin; j += 32) {
      int x = wlo + j;
      if (drop_self && x >= na) ++x;  // skip self
      const int slot = s0 + nbelow + j;
      if (slot < g.Wout) stage_out[slot] = x;
    }
    if (s0 == 1 && lane == 0) stage_out[0] = min(na, g.M - 1);
    __syncwarp();
    const int total = min(s0 + nlg + nwin, g.Wout);
    int32_t* nbo = g.nb + row * g.Wout;
    uint8_t* vo = g.valid + row * g.Wout;
    if ((g.Wout & 3) == 0) {  // rows start 16-byte (nb) / 4-byte (valid) aligned: 4 slots per store
      for (int j = lane * 4; j < g.Wout; j += 128) {
        const int4 sv = *reinterpret_cast<const int4*>(stage_out + j);
        int4 o;
        o.x = j < total ? sv.x : 0;
        o.y = j + 1 < total ? sv.y : 0;
        o.z = j + 2 < total ? sv.z : 0;
        o.w = j + 3 < total ? sv.w : 0;
        *reinterpret_cast<int4*>(nbo + j) = o;
        const int nv = min(max(total - j, 0), 4);  // leading valid slots of the four
        *reinterpret_cast<uint32_t*>(vo + j) = nv >= 4 ? 0x01010101u : (0x01010101u & ((1u << (8 * nv)) - 1u));
      }
    } else {
      for (int j = lane; j < g.Wout; j += 32) {
        nbo[j] = j < total ? stage_out[j] : 0;
        vo[j] = j < total ? 1 : 0;
      }
    }
    for (int l = lane; l < nl1; l += 32) S.l1[l] = 0u;
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
  const unsigned grid = (unsigned)((rows + 127) / 128);  // 8 warps x 16 rows
  const size_t planes = (size_t)g.R * g.p * g.d * sizeof(float);
  const bool smem = planes <= kHashPlaneSmemMax;
  const size_t sm = smem ? planes : 0;
  cudaError_t e;
  auto run = [&](auto fn) {
    if ((e = smem_attr(fn, sm)) != cudaSuccess) return;
    fn<<<grid, 256, sm, st>>>(g);
    note_launch();
    e = cudaGetLastError();
  };
  const bool f32 = g.dtype == kDtF32;
  if (g.d <= 64) {
    if (smem) run(f32 ? k_hash_queries<kDtF32, 64, true> : k_hash_queries<kDtBF16, 64, true>);
    else run(f32 ? k_hash_queries<kDtF32, 64, false> : k_hash_queries<kDtBF16, 64, false>);
  } else {
    if (smem) run(f32 ? k_hash_queries<kDtF32, 128, true> : k_hash_queries<kDtBF16, 128, true>);
    else run(f32 ? k_hash_queries<kDtF32, 128, false> : k_hash_queries<kDtBF16, 128, false>);
  }
  return e;
}

size_t rows_smem_bytes(const GraphDev& g, int warps) { return (size_t)warps * rows_warp_bytes(g, 1); }

cudaError_t launch_rows(const GraphDev& g, int stage, int mode, cudaStream_t st) {
  constexpr int kWarps = 4;
  const size_t sm = (size_t)kWarps * rows_warp_bytes(g, stage);
  if (sm > 227 * 1024) return cudaErrorInvalidConfiguration;
  // bf16 with head dim 64 / 128, fp32 with 64 (the tensor-core path)
  const bool f32 = g.dtype == kDtF32;
  if (f32 && g.d != 64) return cudaErrorInvalidValue;
  auto pick = [&](auto d64, auto d128) { return g.d <= 64 ? d64 : d128; };
  auto fn = f32 ? (stage == 0 ? k_rows<kDtF32, 64, 0, 0> : mode == 0 ? k_rows<kDtF32, 64, 1, 0> : k_rows<kDtF32, 64, 1, 1>)
          : stage == 0 ? pick(k_rows<kDtBF16, 64, 0, 0>, k_rows<kDtBF16, 128, 0, 0>)
          : mode == 0  ? pick(k_rows<kDtBF16, 64, 1, 0>, k_rows<kDtBF16, 128, 1, 0>)
                       : pick(k_rows<kDtBF16, 64, 1, 1>, k_rows<kDtBF16, 128, 1, 1>);
  cudaError_t e;
  if ((e = smem_attr(fn, sm)) != cudaSuccess) return e;
  int per_sm = 0;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kWarps * 32, sm)) != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  int dev = 0, nsm = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  const int64_t rows = (int64_t)g.B * g.H * g.N;
  int64_t blocks = (rows + kWarps - 1) / kWarps;
  const int64_t resident = (int64_t)nsm * per_sm;
  if (blocks > resident) blocks = resident;
  fn<<<(unsigned)blocks, kWarps * 32, sm, st>>>(g);
  note_launch();
  return cudaGetLastError();
}

}  // namespace ssa
