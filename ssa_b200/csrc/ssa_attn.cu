// ssa_attn.cu -- gather attention over a neighbor graph, forward and backward.
//
// Forward replaces sparse_gather_attention (sparse_attention.py:1096-1199):
// for every (b, h, query) row, scores s_j = (q . k[nb_j]) * scale in fp32 over
// the Kn neighbor slots, invalid slots -> -inf, fp32 softmax, the weights cast
// to the value dtype (or kept fp32 with fp32_weights), weighted sum of v rows.
//
// One warp owns one row. The warp is split into four 8-lane groups; a group
// gathers one neighbor row per step, each lane moving a contiguous 32-byte
// slice (16 bf16 or 8 fp32 of a 128-wide head), so one warp instruction
// touches four full rows. Scores stay in shared memory (K <= a few hundred),
// which allows the exact two-pass softmax the reference computes. Rows are
// enumerated (b, kv-head, query, head-in-group) so that the heads sharing a
// kv head, and consecutive queries, run close together and re-hit L2/L1 for
// the shared window/global rows; the (b, kv-head) slices stream through L2
// one after another.
//
// Backward: per row, dq and the per-edge weights (value weight p, and
// scale * dS); then the inverted neighbor index -- the edges of each (batch,
// kv-head) slice stably sorted by key (a hand-written LSD radix sort, so
// within a key edges keep their row order) -- and the dk/dv sums over each
// key's sorted segment, in that order. No floating-point atomics: the result
// is bitwise reproducible. The index depends only on the graph, so layers
// that share a graph can build it once (ssa_attn_build_csr).

#include "ssa_common.cuh"
#include "ssa_internal.h"

namespace ssa {

// Sorted edges per warp in the dk / dv reduction.
constexpr int kDkdvChunk = 512;

__device__ __forceinline__ void decode_row(const AttnDev& a, int64_t i, int& b, int& h, int& n,
                                           int& g) {
  const int hh = (int)(i % a.rep);
  int64_t t = i / a.rep;
  n = (int)(t % a.N);
  t /= a.N;
  g = (int)(t % a.n_kv);
  b = (int)(t / a.n_kv);
  h = g * a.rep + hh;
}

template <typename IT>
__device__ __forceinline__ int load_nb(const void* nb, int64_t i) {
  return (int)__ldg(static_cast<const IT*>(nb) + i);
}

// A slot takes part only if it is valid and its index lies in [0, M): an
// out-of-range index (possible only from a caller-built graph) is treated as
// padding instead of being dereferenced.
template <typename IT>
__device__ __forceinline__ bool slot_ok(const AttnDev& a, const void* nbr, const uint8_t* vr, int j) {
  if (!__ldg(vr + j)) return false;
  const int64_t key = (int64_t)__ldg(static_cast<const IT*>(nbr) + j);
  return key >= 0 && key < a.M;
}

template <int DT, int EPL>
__device__ __forceinline__ void load_slice(const void* row, int e0, int d, float* o) {
#pragma unroll
  for (int c = 0; c < EPL; c += 4) {
    if (e0 + c < d) {
      const float4 x = load4<DT>(row, e0 + c);
      o[c] = x.x; o[c + 1] = x.y; o[c + 2] = x.z; o[c + 3] = x.w;
    } else {
      o[c] = o[c + 1] = o[c + 2] = o[c + 3] = 0.f;
    }
  }
}

template <int DT, int EPL, bool FP32W, typename IT>
__global__ void __launch_bounds__(256) k_attn_fwd(AttnDev a) {
  extern __shared__ __align__(16) float s_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * 8 + warp;
  if (i >= (int64_t)a.B * a.H * a.N) return;
  int b, h, n, g;
  decode_row(a, i, b, h, n, g);
  const int Kp = (a.Kn + 31) & ~31;
  float* s = s_all + warp * Kp;
  const int grp = lane >> 3, li = lane & 7, e0 = li * EPL;
  const int64_t row = ((int64_t)b * a.H + h) * a.N + n;
  const void* nbr = static_cast<const char*>(a.nb) + row * a.Kn * (int64_t)sizeof(IT);
  const uint8_t* vr = a.valid + row * a.Kn;
  const void* kb = row_ptr<DT>(a.k, b * a.k_sb + g * a.k_sh);
  const void* vb = row_ptr<DT>(a.v, b * a.v_sb + g * a.v_sh);

  float qv[EPL];
  load_slice<DT, EPL>(row_ptr<DT>(a.q, b * a.q_sb + h * a.q_sh + (int64_t)n * a.q_sn), e0, a.d, qv);

  const int iters = (a.Kn + 3) >> 2;
  // Pass 1: scores.
  for (int it = 0; it < iters; it += 2) {
    float part[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int j = (it + u) * 4 + grp;
      part[u] = 0.f;
      if (it + u < iters && j < a.Kn && slot_ok<IT>(a, nbr, vr, j)) {
        const int key = load_nb<IT>(nbr, j);
        float kv[EPL];
        load_slice<DT, EPL>(row_ptr<DT>(kb, (int64_t)key * a.k_sm), e0, a.d, kv);
        float acc = 0.f;
#pragma unroll
        for (int c = 0; c < EPL; ++c) acc = fmaf(qv[c], kv[c], acc);
        part[u] = acc;
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float x = part[u];
      x += __shfl_xor_sync(0xffffffffu, x, 1);
      x += __shfl_xor_sync(0xffffffffu, x, 2);
      x += __shfl_xor_sync(0xffffffffu, x, 4);
      const int j = (it + u) * 4 + grp;
      if (li == 0 && it + u < iters && j < a.Kn)
        s[j] = slot_ok<IT>(a, nbr, vr, j) ? x * a.scale : -INFINITY;
    }
  }
  __syncwarp();
  // Softmax in fp32 (:1167).
  float mx = -INFINITY;
  for (int j = lane; j < a.Kn; j += 32) mx = fmaxf(mx, s[j]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int j = lane; j < a.Kn; j += 32) {
    const float e = expf(s[j] - mx);
    s[j] = e;
    sum += e;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  for (int j = lane; j < a.Kn; j += 32) {
    float p = s[j] / sum;
    if (DT == kDtBF16 && !FP32W) p = round_bf16(p);  // attn.to(v.dtype) (:1190)
    if (a.drop_thresh) {  // F.dropout(attn, p) (:1193-1194), in the weights' dtype
      const bool keep = dropout_keep((unsigned long long)row * a.Kn + j, a.drop_seed, a.drop_offset,
                                     a.drop_thresh);
      p = keep ? ((DT == kDtBF16 && !FP32W) ? round_bf16(p * a.drop_scale) : p * a.drop_scale) : 0.f;
    }
    s[j] = p;
  }
  __syncwarp();
  // Pass 2: weighted sum of value rows.
  float acc[EPL];
#pragma unroll
  for (int c = 0; c < EPL; ++c) acc[c] = 0.f;
  for (int it = 0; it < iters; it += 2) {
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int j = (it + u) * 4 + grp;
      if (it + u < iters && j < a.Kn && slot_ok<IT>(a, nbr, vr, j)) {
        const int key = load_nb<IT>(nbr, j);
        const float p = s[j];
        float vv[EPL];
        load_slice<DT, EPL>(row_ptr<DT>(vb, (int64_t)key * a.v_sm), e0, a.d, vv);
#pragma unroll
        for (int c = 0; c < EPL; ++c) acc[c] = fmaf(p, vv[c], acc[c]);
      }
    }
  }
#pragma unroll
  for (int c = 0; c < EPL; ++c) {
    acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 8);
    acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 16);
  }
  if (grp == 0) {
    void* orow = row_ptr_mut<DT>(a.out, b * a.o_sb + h * a.o_sh + (int64_t)n * a.o_sn);
#pragma unroll
    for (int c = 0; c < EPL; ++c)
      if (e0 + c < a.d) store1<DT>(orow, e0 + c, acc[c]);
  }
  if (a.lse && lane == 0) a.lse[row] = mx + logf(sum);
}

// ---------------------------------------------------------------------------
// Forward, vectorised: used when every row slice is 16-byte aligned and the
// head dim is exactly 8 * EPL. The row's slot keys (-1 for slots that take
// no part) are staged in shared memory first, so no gather waits on an index
// load; each lane moves its 32-byte (bf16) or 64-byte (fp32) share of a row
// with 16-byte loads (interleaved words, see raw_load), and every 8-lane
// group keeps U rows in flight.
// ---------------------------------------------------------------------------
template <int DT, int EPL>
struct RawSlice {
  static constexpr int NW = (DT == kDtF32 ? EPL * 4 : EPL * 2) / 16;  // 16-byte words
  uint4 w[NW];
};

// Lane li of an 8-lane group holds the row's 16-byte words li, 8 + li,
// 16 + li, ...: load k of the four groups of a warp reads 128 contiguous
// bytes of each of its four rows, one cache line per row per load (a
// contiguous 32-byte slice per lane would touch two lines per row per load).
template <int DT, int EPL>
__device__ __forceinline__ void raw_load(const void* row, int li, RawSlice<DT, EPL>& r) {
  const uint4* p = static_cast<const uint4*>(row);
#pragma unroll
  for (int k = 0; k < RawSlice<DT, EPL>::NW; ++k) r.w[k] = __ldg(p + k * 8 + li);
}

// Row element of lane li's slice element c (the word layout of raw_load).
template <int DT, int EPL>
__device__ __forceinline__ int raw_elem(int li, int c) {
  constexpr int EW = DT == kDtF32 ? 4 : 8;  // elements per 16-byte word
  return ((c / EW) * 8 + li) * EW + c % EW;
}

// Stores lane li's slice (the word layout of raw_load) with 16-byte stores;
// bf16 values are rounded to nearest even.
template <int DT, int EPL>
__device__ __forceinline__ void raw_store(void* row, int li, const float* v) {
  uint4* p = static_cast<uint4*>(row);
#pragma unroll
  for (int k = 0; k < RawSlice<DT, EPL>::NW; ++k) {
    uint4 w;
    if constexpr (DT == kDtF32) {
      w = make_uint4(__float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]), __float_as_uint(v[4 * k + 2]),
                     __float_as_uint(v[4 * k + 3]));
    } else {
      const float* x = v + 8 * k;
      auto pk = [](float lo, float hi) { return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16); };
      w = make_uint4(pk(x[0], x[1]), pk(x[2], x[3]), pk(x[4], x[5]), pk(x[6], x[7]));
    }
    p[k * 8 + li] = w;
  }
}

// Reduce-scatter over an aligned 8-lane group (lane li = lane & 7): each lane
// holds partial sums part[0..7] of eight slots; halving exchanges with lanes
// li ^ 1, li ^ 2, li ^ 4, each lane keeping the half its bit selects, leave
// lane li with the group's full sum of slot li -- 7 shuffles for 8 slots,
// and the same additions in the same order as a full butterfly per slot.
__device__ __forceinline__ float group8_reduce_scatter(const float (&part)[8], int li) {
  const bool b0 = li & 1, b1 = li & 2, b2 = li & 4;
  float h4[4], h2[2];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float keep = b0 ? part[2 * t + 1] : part[2 * t];
    const float send = b0 ? part[2 * t] : part[2 * t + 1];
    h4[t] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
  }
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const float keep = b1 ? h4[2 * t + 1] : h4[2 * t];
    const float send = b1 ? h4[2 * t] : h4[2 * t + 1];
    h2[t] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  const float keep = b2 ? h2[1] : h2[0];
  return keep + __shfl_xor_sync(0xffffffffu, b2 ? h2[0] : h2[1], 4);
}

// Element c of a raw slice as fp32.
template <int DT, int EPL>
__device__ __forceinline__ float raw_at(const RawSlice<DT, EPL>& r, int c) {
  if constexpr (DT == kDtF32) {
    const uint4 w = r.w[c >> 2];
    const uint32_t u = (c & 3) == 0 ? w.x : (c & 3) == 1 ? w.y : (c & 3) == 2 ? w.z : w.w;
    return __uint_as_float(u);
  } else {
    const uint4 w = r.w[c >> 3];
    const int q = (c >> 1) & 3;
    const uint32_t u = q == 0 ? w.x : q == 1 ? w.y : q == 2 ? w.z : w.w;
    return __uint_as_float((c & 1) ? (u & 0xffff0000u) : (u << 16));
  }
}

// Elements 2*cp and 2*cp+1 of a raw slice as a packed fp32 pair.
template <int DT, int EPL>
__device__ __forceinline__ unsigned long long raw_pair(const RawSlice<DT, EPL>& r, int cp) {
  if constexpr (DT == kDtF32) {
    const uint4 w = r.w[cp >> 1];
    return (cp & 1) ? f2_pack(__uint_as_float(w.z), __uint_as_float(w.w))
                    : f2_pack(__uint_as_float(w.x), __uint_as_float(w.y));
  } else {
    const uint4 w = r.w[cp >> 2];
    const uint32_t u = (cp & 3) == 0 ? w.x : (cp & 3) == 1 ? w.y : (cp & 3) == 2 ? w.z : w.w;
    return f2_pack(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
  }
}

// 32-bit word cp (elements 2 cp, 2 cp + 1) of a raw bf16 slice.
template <int DT, int EPL>
__device__ __forceinline__ uint32_t raw_word(const RawSlice<DT, EPL>& r, int cp) {
  const uint4 w = r.w[cp >> 2];
  return (cp & 3) == 0 ? w.x : (cp & 3) == 1 ? w.y : (cp & 3) == 2 ? w.z : w.w;
}

#ifndef SSA_ATTN_MIXED_FMA
#define SSA_ATTN_MIXED_FMA 1
#endif

// lo += a.lo * b.lo, hi += a.hi * b.hi for packed bf16 pairs, with the
// sm_100 mixed-precision FMA (bf16 operands, fp32 accumulate): the products
// of bf16 values are exact in fp32, so this is bit for bit the fp32 FMA of
// the widened values -- without the widening instructions.
__device__ __forceinline__ void bf2_fma(uint32_t a, uint32_t b, float& lo, float& hi) {
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %2;\n\t"
      "mov.b32 {bl, bh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, al, bl, %0;\n\t"
      "fma.rn.f32.bf16 %1, ah, bh, %1;\n\t}"
      : "+f"(lo), "+f"(hi)
      : "r"(a), "r"(b));
}

// Occupancy over rows in flight: for bf16 d = 128, 2 rows per 8-lane group at
// 4 blocks (32 warps) per SM measured 5.90 ms at c2, against 6.25 ms for 4
// rows at 3 blocks (the gathers hit L2; more warps hide their latency better).
template <int DT, int EPL, bool FP32W, typename IT>
__global__ void __launch_bounds__(256, (EPL >= 16 ? (DT == kDtF32 ? 2 : 4) : 4)) k_attn_fwd_v16(AttnDev a) {
  constexpr int U = (EPL >= 16 && DT != kDtF32) ? 2 : 4;  // rows in flight per 8-lane group
  extern __shared__ __align__(16) float s_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * 8 + warp;
  if (i >= (int64_t)a.B * a.H * a.N) return;
  int b, h, n, g;
  decode_row(a, i, b, h, n, g);
  const int Kp = (a.Kn + 31) & ~31;
  float* s = s_all + warp * 2 * Kp;
  int* sk = reinterpret_cast<int*>(s + Kp);
  const int grp = lane >> 3, li = lane & 7;
  const int64_t row = ((int64_t)b * a.H + h) * a.N + n;
  const void* nbr = static_cast<const char*>(a.nb) + row * a.Kn * (int64_t)sizeof(IT);
  const uint8_t* vr = a.valid + row * a.Kn;
  const void* kb = row_ptr<DT>(a.k, b * a.k_sb + g * a.k_sh);
  const void* vb = row_ptr<DT>(a.v, b * a.v_sb + g * a.v_sh);

  // Slot keys padded to Kp with -1, so the loops below (steps of 4U <= 32)
  // need no bound test.
  for (int j = lane; j < Kp; j += 32) sk[j] = (j < a.Kn && slot_ok<IT>(a, nbr, vr, j)) ? load_nb<IT>(nbr, j) : -1;
  RawSlice<DT, EPL> qr;
  raw_load<DT, EPL>(row_ptr<DT>(a.q, b * a.q_sb + h * a.q_sh + (int64_t)n * a.q_sn), li, qr);
  unsigned long long q2[EPL / 2];
#pragma unroll
  for (int c = 0; c < EPL / 2; ++c) q2[c] = raw_pair<DT, EPL>(qr, c);
  __syncwarp();

  // Pass 1: scores, 8 slots per lane at a time (four steps of U = 2 rows in
  // flight per group when U = 2, two steps when U = 4), reduced over the
  // 8-lane group with group8_reduce_scatter.
  static_assert(8 % U == 0, "slots per block");
  for (int jb = 0; jb < a.Kn; jb += 32) {
    float part[8];
#pragma unroll
    for (int st = 0; st < 8 / U; ++st) {
      RawSlice<DT, EPL> kr[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        // a slot without a key reads key 0's row; its score is masked below
        const int key = max(sk[jb + (st * U + u) * 4 + grp], 0);
        raw_load<DT, EPL>(row_ptr<DT>(kb, (int64_t)key * a.k_sm), li, kr[u]);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float xl = 0.f, xh = 0.f;
        if constexpr (DT == kDtBF16 && SSA_ATTN_MIXED_FMA) {
#pragma unroll
          for (int c = 0; c < EPL / 2; ++c) bf2_fma(raw_word<DT, EPL>(qr, c), raw_word<DT, EPL>(kr[u], c), xl, xh);
        } else {
          unsigned long long x2 = 0ull;
#pragma unroll
          for (int c = 0; c < EPL / 2; ++c) x2 = f2_fma(q2[c], raw_pair<DT, EPL>(kr[u], c), x2);
          f2_unpack(x2, xl, xh);
        }
        part[st * U + u] = xl + xh;
      }
    }
    // slot m of the block (part[m]) is j = jb + m * 4 + grp; lane li ends
    // with slot li (sk and s hold Kp entries, a multiple of 32)
    const float x = group8_reduce_scatter(part, li);
    const int js = jb + li * 4 + grp;
    s[js] = sk[js] >= 0 ? x * a.scale : -INFINITY;
  }
  __syncwarp();
  // Softmax in fp32 (:1167).
  float mx = -INFINITY;
  for (int j = lane; j < a.Kn; j += 32) mx = fmaxf(mx, s[j]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int j = lane; j < a.Kn; j += 32) {
    const float e = expf(s[j] - mx);
    s[j] = e;
    sum += e;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  for (int j = lane; j < a.Kn; j += 32) {
    float p = s[j] / sum;
    if (DT == kDtBF16 && !FP32W) p = round_bf16(p);  // attn.to(v.dtype) (:1190)
    if (a.drop_thresh) {  // F.dropout(attn, p) (:1193-1194), in the weights' dtype
      const bool keep = dropout_keep((unsigned long long)row * a.Kn + j, a.drop_seed, a.drop_offset,
                                     a.drop_thresh);
      p = keep ? ((DT == kDtBF16 && !FP32W) ? round_bf16(p * a.drop_scale) : p * a.drop_scale) : 0.f;
    }
    s[j] = p;
  }
  __syncwarp();
  // Pass 2: weighted sum of value rows. With bf16 weights (the reference's
  // cast to v.dtype) the weight is a bf16 value too, so the mixed FMA applies.
  constexpr bool kMixedPV = DT == kDtBF16 && !FP32W && SSA_ATTN_MIXED_FMA;
  unsigned long long acc2[EPL / 2];
  float acc[EPL];
#pragma unroll
  for (int c = 0; c < EPL / 2; ++c) acc2[c] = 0ull;
#pragma unroll
  for (int c = 0; c < EPL; ++c) acc[c] = 0.f;
  for (int j0 = 0; j0 < a.Kn; j0 += 4 * U) {
    RawSlice<DT, EPL> vrw[U];
    float p[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * 4 + grp;
      const int key = sk[j];
      p[u] = key >= 0 ? s[j] : 0.f;
      // a slot without a key reads key 0's row with weight 0, as the
      // reference's gather of its padded index does
      raw_load<DT, EPL>(row_ptr<DT>(vb, (int64_t)max(key, 0) * a.v_sm), li, vrw[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if constexpr (kMixedPV) {
        const uint32_t pb = __float_as_uint(p[u]);
        const uint32_t pw = (pb >> 16) | (pb & 0xffff0000u);  // the weight in both bf16 halves
#pragma unroll
        for (int c = 0; c < EPL / 2; ++c) bf2_fma(pw, raw_word<DT, EPL>(vrw[u], c), acc[2 * c], acc[2 * c + 1]);
      } else {
        const unsigned long long pp = f2_pack(p[u], p[u]);
#pragma unroll
        for (int c = 0; c < EPL / 2; ++c) acc2[c] = f2_fma(pp, raw_pair<DT, EPL>(vrw[u], c), acc2[c]);
      }
    }
  }
  if constexpr (!kMixedPV) {
#pragma unroll
    for (int c = 0; c < EPL / 2; ++c) f2_unpack(acc2[c], acc[2 * c], acc[2 * c + 1]);
  }
#pragma unroll
  for (int c = 0; c < EPL; ++c) {
    acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 8);
    acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 16);
  }
  if (grp == 0) raw_store<DT, EPL>(row_ptr_mut<DT>(a.out, b * a.o_sb + h * a.o_sh + (int64_t)n * a.o_sn), li, acc);
  if (a.lse && lane == 0) a.lse[row] = mx + logf(sum);
}

// ---------------------------------------------------------------------------
// Backward, stage 1: per row -- dq, edge weights, edge keys.
// ---------------------------------------------------------------------------
template <int DT, int EPL, bool FP32W, typename IT>
__global__ void __launch_bounds__(256) k_attn_bwd_rows(AttnDev a) {
  extern __shared__ __align__(16) float s_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * 8 + warp;
  if (i >= (int64_t)a.B * a.H * a.N) return;
  int b, h, n, g;
  decode_row(a, i, b, h, n, g);
  const int Kp = (a.Kn + 31) & ~31;
  float* sp = s_all + warp * 2 * Kp;  // p_j
  float* sdp = sp + Kp;               // dP_j
  const int grp = lane >> 3, li = lane & 7, e0 = li * EPL;
  const int64_t row = ((int64_t)b * a.H + h) * a.N + n;
  const void* nbr = static_cast<const char*>(a.nb) + row * a.Kn * (int64_t)sizeof(IT);
  const uint8_t* vr = a.valid + row * a.Kn;
  const void* kb = row_ptr<DT>(a.k, b * a.k_sb + g * a.k_sh);
  const void* vb = row_ptr<DT>(a.v, b * a.v_sb + g * a.v_sh);
  const int64_t orow_off = b * a.o_sb + h * a.o_sh + (int64_t)n * a.o_sn;

  float qv[EPL], gv[EPL];
  load_slice<DT, EPL>(row_ptr<DT>(a.q, b * a.q_sb + h * a.q_sh + (int64_t)n * a.q_sn), e0, a.d, qv);
  load_slice<DT, EPL>(row_ptr<DT>(a.dO, orow_off), e0, a.d, gv);
  const float lse = a.lse_in[row];
  const int iters = (a.Kn + 3) >> 2;
  for (int it = 0; it < iters; ++it) {
    const int j = it * 4 + grp;
    float ps = 0.f, pd = 0.f;
    const bool ok = j < a.Kn && slot_ok<IT>(a, nbr, vr, j);
    if (ok) {
      const int key = load_nb<IT>(nbr, j);
      float kv[EPL], vv[EPL];
      load_slice<DT, EPL>(row_ptr<DT>(kb, (int64_t)key * a.k_sm), e0, a.d, kv);
      load_slice<DT, EPL>(row_ptr<DT>(vb, (int64_t)key * a.v_sm), e0, a.d, vv);
#pragma unroll
      for (int c = 0; c < EPL; ++c) {
        ps = fmaf(qv[c], kv[c], ps);
        pd = fmaf(gv[c], vv[c], pd);
      }
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      ps += __shfl_xor_sync(0xffffffffu, ps, o);
      pd += __shfl_xor_sync(0xffffffffu, pd, o);
    }
    if (li == 0 && j < a.Kn) {
      sp[j] = ok ? expf(ps * a.scale - lse) : 0.f;
      sdp[j] = ok ? pd : 0.f;
    }
  }
  __syncwarp();
  // Dropout: the gradient reaching the pre-dropout weights is dO.v_j scaled
  // by 1/(1-p) where the weight was kept, 0 where it was dropped. Keep bits
  // of slots lane, lane + 32, ... stay in a register for the edge loop.
  uint32_t keep_bits = 0xFFFFFFFFu;
  if (a.drop_thresh) {
    keep_bits = 0u;
    for (int j = lane, kk = 0; j < a.Kn; j += 32, ++kk) {
      const bool keep = dropout_keep((unsigned long long)row * a.Kn + j, a.drop_seed, a.drop_offset,
                                     a.drop_thresh);
      if (keep && kk < 32) keep_bits |= 1u << kk;
      sdp[j] = keep ? sdp[j] * a.drop_scale : 0.f;
    }
    __syncwarp();
  }
  float dsum = 0.f;
  for (int j = lane; j < a.Kn; j += 32) dsum = fmaf(sp[j], sdp[j], dsum);
#pragma unroll
  for (int o = 16; o; o >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
  for (int j = lane, kk = 0; j < a.Kn; j += 32, ++kk) {
    const float p = sp[j];
    const float ds = p * (sdp[j] - dsum) * a.scale;
    const int64_t e = row * a.Kn + j;
    float pv = (DT == kDtBF16 && !FP32W) ? round_bf16(p) : p;  // the weight that multiplied v_j
    if (a.drop_thresh) {
      const bool keep = kk < 32 ? ((keep_bits >> kk) & 1u) != 0
                                : dropout_keep((unsigned long long)e, a.drop_seed, a.drop_offset, a.drop_thresh);
      pv = keep ? ((DT == kDtBF16 && !FP32W) ? round_bf16(pv * a.drop_scale) : pv * a.drop_scale) : 0.f;
    }
    a.ep[e] = pv;
    a.eds[e] = ds;
    sdp[j] = ds;
  }
  __syncwarp();
  float acc[EPL];
#pragma unroll
  for (int c = 0; c < EPL; ++c) acc[c] = 0.f;
  for (int it = 0; it < iters; ++it) {
    const int j = it * 4 + grp;
    if (j < a.Kn && slot_ok<IT>(a, nbr, vr, j)) {
      const int key = load_nb<IT>(nbr, j);
      const float ds = sdp[j];
      float kv[EPL];
      load_slice<DT, EPL>(row_ptr<DT>(kb, (int64_t)key * a.k_sm), e0, a.d, kv);
#pragma unroll
      for (int c = 0; c < EPL; ++c) acc[c] = fmaf(ds, kv[c], acc[c]);
    }
  }
#pragma unroll
  for (int c = 0; c < EPL; ++c) {
    acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 8);
    acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 16);
  }
  if (grp == 0) {
    void* dqr = row_ptr_mut<DT>(a.dq, orow_off);
#pragma unroll
    for (int c = 0; c < EPL; ++c)
      if (e0 + c < a.d) store1<DT>(dqr, e0 + c, acc[c]);
  }
}

// Backward, stage 1, vectorised (same conditions as k_attn_fwd_v16): the
// row's slot keys staged in shared memory, 16-byte row gathers, U rows in
// flight per 8-lane group, paired fp32 FMA.
template <int DT, int EPL, bool FP32W, typename IT>
__global__ void __launch_bounds__(256, (EPL >= 16 ? 2 : 3)) k_attn_bwd_rows_v16(AttnDev a) {
  constexpr int U = 2;
  extern __shared__ __align__(16) float s_all[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * 8 + warp;
  if (i >= (int64_t)a.B * a.H * a.N) return;
  int b, h, n, g;
  decode_row(a, i, b, h, n, g);
  const int Kp = (a.Kn + 31) & ~31;
  float* sp = s_all + warp * 3 * Kp;  // p_j
  float* sdp = sp + Kp;                // dP_j, then scale * dS_j
  int* sk = reinterpret_cast<int*>(sdp + Kp);
  const int grp = lane >> 3, li = lane & 7;
  const int64_t row = ((int64_t)b * a.H + h) * a.N + n;
  const void* nbr = static_cast<const char*>(a.nb) + row * a.Kn * (int64_t)sizeof(IT);
  const uint8_t* vr = a.valid + row * a.Kn;
  const void* kb = row_ptr<DT>(a.k, b * a.k_sb + g * a.k_sh);
  const void* vb = row_ptr<DT>(a.v, b * a.v_sb + g * a.v_sh);
  const int64_t orow_off = b * a.o_sb + h * a.o_sh + (int64_t)n * a.o_sn;

  // Slot keys padded to Kp with -1 (the loops below need no bound test); a
  // slot without a key reads key 0's rows, which its zero weight cancels.
  for (int j = lane; j < Kp; j += 32) sk[j] = (j < a.Kn && slot_ok<IT>(a, nbr, vr, j)) ? load_nb<IT>(nbr, j) : -1;
  RawSlice<DT, EPL> qr, gr;
  raw_load<DT, EPL>(row_ptr<DT>(a.q, b * a.q_sb + h * a.q_sh + (int64_t)n * a.q_sn), li, qr);
  raw_load<DT, EPL>(row_ptr<DT>(a.dO, orow_off), li, gr);
  unsigned long long q2[EPL / 2], g2[EPL / 2];
#pragma unroll
  for (int c = 0; c < EPL / 2; ++c) {
    q2[c] = raw_pair<DT, EPL>(qr, c);
    g2[c] = raw_pair<DT, EPL>(gr, c);
  }
  const float lse = a.lse_in[row];
  __syncwarp();
  // 8 slots per lane at a time (four steps of U = 2 rows in flight per
  // group), p and dP reduced over the 8-lane group with
  // group8_reduce_scatter: lane li ends with slot li of the block.
  static_assert(8 % U == 0, "slots per block");
  for (int jb = 0; jb < a.Kn; jb += 32) {
    float ps8[8], pd8[8];
#pragma unroll
    for (int st = 0; st < 8 / U; ++st) {
      RawSlice<DT, EPL> kr[U], vrw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int key = max(sk[jb + (st * U + u) * 4 + grp], 0);
        raw_load<DT, EPL>(row_ptr<DT>(kb, (int64_t)key * a.k_sm), li, kr[u]);
        raw_load<DT, EPL>(row_ptr<DT>(vb, (int64_t)key * a.v_sm), li, vrw[u]);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        unsigned long long x2 = 0ull, y2 = 0ull;
#pragma unroll
        for (int c = 0; c < EPL / 2; ++c) {
          x2 = f2_fma(q2[c], raw_pair<DT, EPL>(kr[u], c), x2);
          y2 = f2_fma(g2[c], raw_pair<DT, EPL>(vrw[u], c), y2);
        }
        float xl, xh, yl, yh;
        f2_unpack(x2, xl, xh);
        f2_unpack(y2, yl, yh);
        ps8[st * U + u] = xl + xh;
        pd8[st * U + u] = yl + yh;
      }
    }
    const float ps = group8_reduce_scatter(ps8, li);
    const float pd = group8_reduce_scatter(pd8, li);
    const int j = jb + li * 4 + grp;  // sp / sdp hold Kp entries; slots past Kn have no key
    const bool ok = sk[j] >= 0;
    sp[j] = ok ? expf(ps * a.scale - lse) : 0.f;
    sdp[j] = ok ? pd : 0.f;
  }
  __syncwarp();
  // Dropout: the gradient reaching the pre-dropout weights is dO.v_j scaled
  // by 1/(1-p) where the weight was kept, 0 where it was dropped.
  uint32_t keep_bits = 0xFFFFFFFFu;
  if (a.drop_thresh) {
    keep_bits = 0u;
    for (int j = lane, kk = 0; j < a.Kn; j += 32, ++kk) {
      const bool keep = dropout_keep((unsigned long long)row * a.Kn + j, a.drop_seed, a.drop_offset,
                                     a.drop_thresh);
      if (keep && kk < 32) keep_bits |= 1u << kk;
      sdp[j] = keep ? sdp[j] * a.drop_scale : 0.f;
    }
    __syncwarp();
  }
  float dsum = 0.f;
  for (int j = lane; j < a.Kn; j += 32) dsum = fmaf(sp[j], sdp[j], dsum);
#pragma unroll
  for (int o = 16; o; o >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
  for (int j = lane, kk = 0; j < a.Kn; j += 32, ++kk) {
    const float p = sp[j];
    const float ds = p * (sdp[j] - dsum) * a.scale;
    const int64_t e = row * a.Kn + j;
    float pv = (DT == kDtBF16 && !FP32W) ? round_bf16(p) : p;  // the weight that multiplied v_j
    if (a.drop_thresh) {
      const bool keep = kk < 32 ? ((keep_bits >> kk) & 1u) != 0
                                : dropout_keep((unsigned long long)e, a.drop_seed, a.drop_offset, a.drop_thresh);
      pv = keep ? ((DT == kDtBF16 && !FP32W) ? round_bf16(pv * a.drop_scale) : pv * a.drop_scale) : 0.f;
    }
    a.ep[e] = pv;
    a.eds[e] = ds;
    sdp[j] = ds;
  }
  __syncwarp();
  unsigned long long acc2[EPL / 2];
#pragma unroll
  for (int c = 0; c < EPL / 2; ++c) acc2[c] = 0ull;
  for (int j0 = 0; j0 < a.Kn; j0 += 4 * U) {
    RawSlice<DT, EPL> kr[U];
    float ds[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * 4 + grp;
      const int key = sk[j];
      ds[u] = key >= 0 ? sdp[j] : 0.f;
      raw_load<DT, EPL>(row_ptr<DT>(kb, (int64_t)max(key, 0) * a.k_sm), li, kr[u]);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const unsigned long long dd = f2_pack(ds[u], ds[u]);
#pragma unroll
      for (int c = 0; c < EPL / 2; ++c) acc2[c] = f2_fma(dd, raw_pair<DT, EPL>(kr[u], c), acc2[c]);
    }
  }
  float acc[EPL];
#pragma unroll
  for (int c = 0; c < EPL / 2; ++c) f2_unpack(acc2[c], acc[2 * c], acc[2 * c + 1]);
#pragma unroll
  for (int c = 0; c < EPL; ++c) {
    acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 8);
    acc[c] += __shfl_xor_sync(0xffffffffu, acc[c], 16);
  }
  if (grp == 0) {
    void* dqr = row_ptr_mut<DT>(a.dq, orow_off);
#pragma unroll
    for (int c = 0; c < EPL; ++c) store1<DT>(dqr, raw_elem<DT, EPL>(li, c), acc[c]);
  }
}

// ---------------------------------------------------------------------------
// Backward, stage 3: one warp per (kv slice, key) sums its sorted segment.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t lower_bound_u32(const uint32_t* a, int64_t n, uint32_t x) {
  int64_t lo = 0, hi = n;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (__ldg(a + mid) < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// First sorted position of every key, and seg[B*n_kv*M] = the number of
// valid edges: one thread per key, a binary search over the sorted keys.
__global__ void __launch_bounds__(256) k_seg_starts(AttnDev a, const uint32_t* n_valid) {
  const int64_t key = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)a.B * a.n_kv * a.M;
  if (key > total) return;
  a.seg[key] = (uint32_t)lower_bound_u32(a.skey, (int64_t)__ldg(n_valid), (uint32_t)key);
}

// ---------------------------------------------------------------------------
// Backward, stage 2: the inverted neighbor index (CSR). The edges (b, h, n,
// slot) of one (batch, kv-head) slice are contiguous -- rows b*H + h with
// h / rep = g, i.e. rows rep*bg .. rep*bg + rep - 1 -- so sorting each slice
// by key, least significant 8-bit digit first, sorts all edges by
// (slice, key). Invalid slots carry the key M, sorted last in every pass but
// the final one, which drops them and writes the composite key bg * M + key.
// Each pass runs over 4096-edge tiles of a slice:
//   k_esort_hist     256-bin histogram of the tile's digits;
//   k_esort_scan     per slice, an exclusive scan over (digit, tile);
//   k_esort_base     (final pass) the slices' output offsets;
//   k_esort_scatter  ranks the tile's edges digit by digit in edge order --
//                    each warp takes 512 consecutive edges 32 at a time,
//                    __match_any_sync groups equal digits, per-warp counters
//                    give the rank, a scan over warps orders the warps -- so
//                    the sort is stable, and writes them to their slots.
// ---------------------------------------------------------------------------
constexpr int kSortTile = 4096;  // edges per tile: 8 warps x 16 rounds x 32

struct SortPass {
  const uint32_t* kin;   // keys in; null in the first pass (read from nb / valid)
  const uint32_t* iin;   // edge ids in; null in the first pass (the edge's position)
  uint32_t* kout;
  uint32_t* iout;
  uint32_t* counts;      // [BG][256][tiles]: counts, then tile offsets
  uint32_t* totals;      // [BG] edges counted per slice
  uint32_t* base;        // [BG + 1] final pass: first output slot of each slice; [BG] = all
  int shift;             // digit = (key >> shift) & 255
  int final_pass;        // drop invalid edges, write bg * M + key
  int tiles;             // tiles per slice
  int64_t slice_edges;   // rep * N * Kn
};

// Key of edge e: its neighbor index if the slot takes part (valid, inside
// [0, M)), else M.
template <typename IT>
__device__ __forceinline__ uint32_t edge_key(const AttnDev& a, const SortPass& sp, int64_t e) {
  if (sp.kin) return __ldg(sp.kin + e);
  if (!__ldg(a.valid + e)) return (uint32_t)a.M;
  const int64_t x = (int64_t)__ldg(static_cast<const IT*>(a.nb) + e);
  return (x >= 0 && x < a.M) ? (uint32_t)x : (uint32_t)a.M;
}

template <typename IT>
__global__ void __launch_bounds__(256) k_esort_hist(AttnDev a, SortPass sp) {
  __shared__ uint32_t hist[256];
  const int t = blockIdx.x, bg = blockIdx.y;
  const int64_t e0 = bg * sp.slice_edges + (int64_t)t * kSortTile;
  const int64_t e1 = min(e0 + kSortTile, (bg + 1) * sp.slice_edges);
  hist[threadIdx.x] = 0;
  __syncthreads();
  for (int64_t e = e0 + threadIdx.x; e < e1; e += 256) {
    const uint32_t key = edge_key<IT>(a, sp, e);
    if (sp.final_pass && key >= (uint32_t)a.M) continue;
    atomicAdd(&hist[(key >> sp.shift) & 255u], 1u);
  }
  __syncthreads();
  sp.counts[((int64_t)bg * 256 + threadIdx.x) * sp.tiles + t] = hist[threadIdx.x];
}

// One block per slice: counts[bg][digit][tile] -> exclusive prefix in
// (digit, tile) order; totals[bg] = the slice's count.
__global__ void __launch_bounds__(1024) k_esort_scan(SortPass sp) {
  __shared__ uint32_t wsum[32];
  const int bg = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t* c = sp.counts + (int64_t)bg * 256 * sp.tiles;
  const int n = 256 * sp.tiles;
  const int per = (n + 1023) / 1024;
  const int i0 = min(threadIdx.x * per, n), i1 = min(i0 + per, n);
  uint32_t sum = 0;
  for (int i = i0; i < i1; ++i) sum += c[i];
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = wsum[lane], wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += v;
    }
    wsum[lane] = wi - w;  // exclusive prefix of the warp sums
    if (lane == 31) sp.totals[bg] = wi;
  }
  __syncthreads();
  uint32_t run = wsum[warp] + incl - sum;
  for (int i = i0; i < i1; ++i) {
    const uint32_t v = c[i];
    c[i] = run;
    run += v;
  }
}

// Final pass: base[bg] = edges kept in the slices before bg; base[BG] = all.
__global__ void __launch_bounds__(1024) k_esort_base(SortPass sp, int BG) {
  __shared__ uint32_t wsum[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int per = (BG + 1023) / 1024;
  const int i0 = min((int)threadIdx.x * per, BG), i1 = min(i0 + per, BG);
  uint32_t sum = 0;
  for (int i = i0; i < i1; ++i) sum += sp.totals[i];
  uint32_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = wsum[lane], wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += v;
    }
    wsum[lane] = wi - w;
    if (lane == 31) sp.base[BG] = wi;
  }
  __syncthreads();
  uint32_t run = wsum[warp] + incl - sum;
  for (int i = i0; i < i1; ++i) {
    sp.base[i] = run;
    run += sp.totals[i];
  }
}

template <typename IT>
__global__ void __launch_bounds__(256) k_esort_scatter(AttnDev a, SortPass sp) {
  constexpr int ROUNDS = kSortTile / 256;  // 16 rounds of 32 edges per warp
  __shared__ uint32_t wcnt[8][257];        // per-warp digit counts, then warp offsets
  __shared__ uint32_t toff[256];           // first output slot of each digit of this tile
  const int t = blockIdx.x, bg = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t e0 = bg * sp.slice_edges + (int64_t)t * kSortTile;
  const int64_t e1 = min(e0 + kSortTile, (bg + 1) * sp.slice_edges);
  for (int i = threadIdx.x; i < 8 * 257; i += 256) (&wcnt[0][0])[i] = 0;
  const uint32_t sbase = sp.final_pass ? sp.base[bg] : (uint32_t)(bg * sp.slice_edges);
  toff[threadIdx.x] = sbase + sp.counts[((int64_t)bg * 256 + threadIdx.x) * sp.tiles + t];
  __syncthreads();
  uint32_t key[ROUNDS], id[ROUNDS], rank[ROUNDS];
  int dig[ROUNDS];
#pragma unroll
  for (int r = 0; r < ROUNDS; ++r) {
    const int64_t e = e0 + warp * (32 * ROUNDS) + r * 32 + lane;
    const bool in = e < e1;
    key[r] = in ? edge_key<IT>(a, sp, e) : (uint32_t)a.M;
    id[r] = in ? (sp.iin ? __ldg(sp.iin + e) : (uint32_t)e) : 0u;
    const bool live = in && !(sp.final_pass && key[r] >= (uint32_t)a.M);
    const int d = live ? (int)((key[r] >> sp.shift) & 255u) : 256;  // 256: takes no slot
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const int leader = __ffs(peers) - 1;
    uint32_t before = 0;
    if (lane == leader) {
      before = wcnt[warp][d];
      wcnt[warp][d] = before + __popc(peers);
    }
    before = __shfl_sync(0xffffffffu, before, leader);
    rank[r] = before + __popc(peers & ((1u << lane) - 1u));
    dig[r] = live ? d : -1;
    __syncwarp();
  }
  __syncthreads();
  {  // warp order within each digit
    const int d = threadIdx.x;
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t v = wcnt[w][d];
      wcnt[w][d] = run;
      run += v;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < ROUNDS; ++r) {
    if (dig[r] < 0) continue;
    const uint32_t pos = toff[dig[r]] + wcnt[warp][dig[r]] + rank[r];
    sp.kout[pos] = sp.final_pass ? (uint32_t)bg * (uint32_t)a.M + key[r] : key[r];
    sp.iout[pos] = id[r];
  }
}

// dk / dv as a segmented sum over the edges sorted by (kv slice, key). Each
// warp takes a fixed chunk of kDkdvChunk sorted edges, so a key that many
// queries gathered (a global token) is spread over many warps. Within the
// chunk the warp walks its keys in order; a row of d elements takes d / EPW
// lanes (rounded up to a power of two) and the warp's lane groups take
// every G-th edge, two at a time, summed at the end in a fixed order. A key
// whose edges all lie in the chunk is written to dk / dv; a key that crosses
// a chunk edge leaves a partial (slot 0: it started before the chunk, slot
// 1: it started inside), which k_dkdv_fix adds up in chunk order. The
// result is deterministic.
template <int DT, int EPW, bool V16>
__global__ void __launch_bounds__(256) k_dkdv(AttnDev a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t total = (int64_t)a.B * a.n_kv * a.M;
  const int64_t ev = __ldg(a.seg + total);  // end of the valid edges
  const int64_t chunk = (int64_t)blockIdx.x * 8 + warp;
  const int64_t s0 = chunk * kDkdvChunk;
  if (s0 >= ev) return;
  const int64_t s1 = min(s0 + (int64_t)kDkdvChunk, ev);
  int lpr = 1;  // lanes per row
  while (lpr * EPW < a.d && lpr < 32) lpr <<= 1;
  const int G = 32 / lpr, grp = lane / lpr, e0 = (lane % lpr) * EPW;
  const bool in_d = e0 < a.d;
  auto rows_of = [&](uint32_t e, const void*& qr, const void*& gr) {
    const int64_t row = e / (uint32_t)a.Kn;
    const int n = (int)(row % a.N);
    const int64_t bh = row / a.N;
    const int h = (int)(bh % a.H), b = (int)(bh / a.H);
    qr = row_ptr<DT>(a.q, b * a.q_sb + h * a.q_sh + (int64_t)n * a.q_sn);
    gr = row_ptr<DT>(a.dO, b * a.o_sb + h * a.o_sh + (int64_t)n * a.o_sn);
  };
  const int64_t k_first = __ldg(a.skey + s0), k_last = __ldg(a.skey + s1 - 1);
  for (int64_t key = k_first; key <= k_last; ++key) {
    const int64_t kb = __ldg(a.seg + key), ke = __ldg(a.seg + key + 1);
    const int64_t lo = max(kb, s0), hi = min(ke, s1);
    if (lo >= hi) continue;
    float dk[EPW], dv[EPW];
#pragma unroll
    for (int c = 0; c < EPW; ++c) dk[c] = dv[c] = 0.f;
    for (int64_t s = lo + grp; s < hi; s += 2 * G) {
      const bool two = s + G < hi;
      const uint32_t ea = __ldg(a.sid + s), eb = two ? __ldg(a.sid + s + G) : ea;
      const void *qa, *ga, *qb, *gb;
      rows_of(ea, qa, ga);
      rows_of(eb, qb, gb);
      float xq[2][EPW], xg[2][EPW];
      if (in_d) {
        if constexpr (V16) {  // 16-byte aligned rows: one 16-byte load per 8 bf16
#pragma unroll
          for (int c = 0; c < EPW; c += 8) {
            load8<DT>(qa, e0 + c, xq[0] + c);
            load8<DT>(ga, e0 + c, xg[0] + c);
            load8<DT>(qb, e0 + c, xq[1] + c);
            load8<DT>(gb, e0 + c, xg[1] + c);
          }
        } else {
          load_slice<DT, EPW>(qa, e0, a.d, xq[0]);
          load_slice<DT, EPW>(ga, e0, a.d, xg[0]);
          load_slice<DT, EPW>(qb, e0, a.d, xq[1]);
          load_slice<DT, EPW>(gb, e0, a.d, xg[1]);
        }
      }
      const float pa = __ldg(a.ep + ea), da = __ldg(a.eds + ea);
      const float pb = two ? __ldg(a.ep + eb) : 0.f, db = two ? __ldg(a.eds + eb) : 0.f;
      if (in_d) {
#pragma unroll
        for (int c = 0; c < EPW; ++c) {
          dk[c] = fmaf(da, xq[0][c], dk[c]);
          dv[c] = fmaf(pa, xg[0][c], dv[c]);
        }
#pragma unroll
        for (int c = 0; c < EPW; ++c) {
          dk[c] = fmaf(db, xq[1][c], dk[c]);
          dv[c] = fmaf(pb, xg[1][c], dv[c]);
        }
      }
    }
    for (int off = lpr; off < 32; off <<= 1) {
#pragma unroll
      for (int c = 0; c < EPW; ++c) {
        dk[c] += __shfl_xor_sync(0xffffffffu, dk[c], off);
        dv[c] += __shfl_xor_sync(0xffffffffu, dv[c], off);
      }
    }
    if (grp == 0) {
      if (kb >= s0 && ke <= s1) {  // the whole segment lies in this chunk
        void* dkr = row_ptr_mut<DT>(a.dk, key * a.d);
        void* dvr = row_ptr_mut<DT>(a.dv, key * a.d);
#pragma unroll
        for (int c = 0; c < EPW; ++c) {
          if (e0 + c < a.d) {
            store1<DT>(dkr, e0 + c, dk[c]);
            store1<DT>(dvr, e0 + c, dv[c]);
          }
        }
      } else {
        float* pt = a.part + ((size_t)chunk * 2 + (kb < s0 ? 0 : 1)) * 2 * a.d;
#pragma unroll
        for (int c = 0; c < EPW; ++c) {
          if (e0 + c < a.d) {
            pt[e0 + c] = dk[c];
            pt[a.d + e0 + c] = dv[c];
          }
        }
      }
    }
  }
}

// Keys without edges get zero gradients; keys whose edges cross a chunk
// edge get their partials summed in chunk order. One warp per key.
template <int DT>
__global__ void __launch_bounds__(256) k_dkdv_fix(AttnDev a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t key = (int64_t)blockIdx.x * 8 + warp;
  const int64_t total = (int64_t)a.B * a.n_kv * a.M;
  if (key >= total) return;
  const int64_t kb = __ldg(a.seg + key), ke = __ldg(a.seg + key + 1);
  const bool empty = kb >= ke;
  const int64_t c0 = kb / kDkdvChunk, c1 = empty ? c0 : (ke - 1) / kDkdvChunk;
  if (!empty && c0 == c1) return;  // written by k_dkdv
  void* dkr = row_ptr_mut<DT>(a.dk, key * a.d);
  void* dvr = row_ptr_mut<DT>(a.dv, key * a.d);
  for (int e = lane; e < a.d; e += 32) {
    float dk = 0.f, dv = 0.f;
    if (!empty) {
      for (int64_t c = c0; c <= c1; ++c) {
        const float* pt = a.part + ((size_t)c * 2 + (c == c0 ? 1 : 0)) * 2 * a.d;
        dk += __ldg(pt + e);
        dv += __ldg(pt + a.d + e);
      }
    }
    store1<DT>(dkr, e, dk);
    store1<DT>(dvr, e, dv);
  }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
// The vectorised kernel needs the head dim to be exactly 8 * EPL and every
// row slice it loads (q, k, v) to start on a 16-byte boundary.
template <int DT, int EPL>
static bool fwd_vec16_ok(const AttnDev& a) {
  if (a.d != 8 * EPL) return false;
  const int es = DT == kDtF32 ? 4 : 2;
  auto al = [&](const void* p) { return (reinterpret_cast<uintptr_t>(p) % 16) == 0; };
  auto st = [&](int64_t x) { return (x * es) % 16 == 0; };
  return al(a.q) && al(a.k) && al(a.v) && st(a.q_sb) && st(a.q_sh) && st(a.q_sn) && st(a.k_sb) &&
         st(a.k_sh) && st(a.k_sm) && st(a.v_sb) && st(a.v_sh) && st(a.v_sm);
}

template <int DT, int EPL, bool FP32W, typename IT>
static cudaError_t fwd_t(const AttnDev& a, cudaStream_t st) {
  const int Kp = (a.Kn + 31) & ~31;
  // bf16 slices under 16 bytes, and head dims above 128: scalar kernel only
  if constexpr (!(DT == kDtBF16 && EPL < 8) && EPL <= 16) {
    // the output rows are written with 16-byte stores as well
    if (fwd_vec16_ok<DT, EPL>(a) && (reinterpret_cast<uintptr_t>(a.out) % 16) == 0 &&
        ((a.o_sb | a.o_sh | a.o_sn) * (DT == kDtF32 ? 4 : 2)) % 16 == 0) {
      const size_t smem = (size_t)8 * 2 * Kp * sizeof(float);
      auto fn = k_attn_fwd_v16<DT, EPL, FP32W, IT>;
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      const int64_t rows = (int64_t)a.B * a.H * a.N;
      fn<<<(unsigned)((rows + 7) / 8), 256, smem, st>>>(a);
      note_launch();
      return cudaGetLastError();
    }
  }
  const size_t smem = (size_t)8 * Kp * sizeof(float);
  auto fn = k_attn_fwd<DT, EPL, FP32W, IT>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t rows = (int64_t)a.B * a.H * a.N;
  fn<<<(unsigned)((rows + 7) / 8), 256, smem, st>>>(a);
  note_launch();
  return cudaGetLastError();
}

template <int DT, int EPL>
static cudaError_t fwd_e(const AttnDev& a, cudaStream_t st) {
  if (a.fp32w) return a.nb_i64 ? fwd_t<DT, EPL, true, int64_t>(a, st) : fwd_t<DT, EPL, true, int32_t>(a, st);
  return a.nb_i64 ? fwd_t<DT, EPL, false, int64_t>(a, st) : fwd_t<DT, EPL, false, int32_t>(a, st);
}

template <int DT>
static cudaError_t fwd_d(const AttnDev& a, cudaStream_t st) {
  if (a.d <= 32) return fwd_e<DT, 4>(a, st);
  if (a.d <= 64) return fwd_e<DT, 8>(a, st);
  if (a.d <= 128) return fwd_e<DT, 16>(a, st);
  return fwd_e<DT, 32>(a, st);
}

cudaError_t launch_attn_fwd(const AttnDev& a, cudaStream_t st) {
  return a.dtype == kDtF32 ? fwd_d<kDtF32>(a, st) : fwd_d<kDtBF16>(a, st);
}

// Geometry of the edge sort: E edges; a slice's rep * N * Kn edges in
// `tiles` tiles; `passes` 8-bit digits cover keys 0..M (M marks invalid).
struct SortGeom {
  int64_t E, slice_edges;
  int tiles, passes, BG;
};

static SortGeom sort_geom(const AttnDev& a) {
  SortGeom g;
  g.E = (int64_t)a.B * a.H * a.N * a.Kn;
  g.BG = a.B * a.n_kv;
  g.slice_edges = (int64_t)a.rep * a.N * a.Kn;
  g.tiles = (int)((g.slice_edges + kSortTile - 1) / kSortTile);
  const int bits = 32 - __builtin_clz((unsigned)a.M);  // M itself must fit
  g.passes = (bits + 7) / 8;
  return g;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t attn_csr_layout(const AttnDev& a, AttnDev* out, void* csr) {
  const SortGeom sg = sort_geom(a);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t o_skey = take(4 * sg.E), o_sid = take(4 * sg.E);
  const size_t o_seg = take(4 * ((size_t)sg.BG * a.M + 1));
  if (out) {
    char* base = static_cast<char*>(csr);
    out->skey = reinterpret_cast<uint32_t*>(base + o_skey);
    out->sid = reinterpret_cast<uint32_t*>(base + o_sid);
    out->seg = reinterpret_cast<uint32_t*>(base + o_seg);
  }
  return off;
}

size_t attn_bwd_workspace_layout(const AttnDev& a, AttnDev* out, void* ws) {
  const SortGeom sg = sort_geom(a);
  const int64_t E = sg.E;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t o_ep = take(4 * E), o_eds = take(4 * E);
  const size_t o_tk0 = take(4 * E), o_ti0 = take(4 * E);
  size_t o_tk1 = 0, o_ti1 = 0;
  if (sg.passes >= 3) {
    o_tk1 = take(4 * E);
    o_ti1 = take(4 * E);
  }
  const size_t o_cnt = take(4 * (size_t)sg.BG * 256 * sg.tiles);
  const size_t o_tot = take(4 * (size_t)sg.BG), o_base = take(4 * ((size_t)sg.BG + 1));
  const size_t chunks = (size_t)(E + kDkdvChunk - 1) / kDkdvChunk;
  const size_t o_part = take(sizeof(float) * chunks * 4 * (size_t)a.d);
  const size_t o_csr = off;
  off += attn_csr_layout(a, nullptr, nullptr);  // the inverted index, when the call builds its own
  if (out) {
    char* base = static_cast<char*>(ws);
    out->ep = reinterpret_cast<float*>(base + o_ep);
    out->eds = reinterpret_cast<float*>(base + o_eds);
    out->tk0 = reinterpret_cast<uint32_t*>(base + o_tk0);
    out->ti0 = reinterpret_cast<uint32_t*>(base + o_ti0);
    out->tk1 = sg.passes >= 3 ? reinterpret_cast<uint32_t*>(base + o_tk1) : nullptr;
    out->ti1 = sg.passes >= 3 ? reinterpret_cast<uint32_t*>(base + o_ti1) : nullptr;
    out->cnt = reinterpret_cast<uint32_t*>(base + o_cnt);
    out->tot = reinterpret_cast<uint32_t*>(base + o_tot);
    out->sbase = reinterpret_cast<uint32_t*>(base + o_base);
    out->part = reinterpret_cast<float*>(base + o_part);
    attn_csr_layout(a, out, base + o_csr);
  }
  return off;
}

// The inverted neighbor index into a.skey / a.sid / a.seg: the LSD passes,
// then every key's segment start.
template <typename IT>
static cudaError_t build_csr_t(const AttnDev& a, cudaStream_t st) {
  const SortGeom sg = sort_geom(a);
  const dim3 grid(sg.tiles, sg.BG);
  const uint32_t* kin = nullptr;
  const uint32_t* iin = nullptr;
  for (int pass = 0; pass < sg.passes; ++pass) {
    SortPass sp;
    sp.kin = kin;
    sp.iin = iin;
    sp.final_pass = pass == sg.passes - 1;
    sp.kout = sp.final_pass ? a.skey : (pass & 1 ? a.tk1 : a.tk0);
    sp.iout = sp.final_pass ? a.sid : (pass & 1 ? a.ti1 : a.ti0);
    sp.counts = a.cnt;
    sp.totals = a.tot;
    sp.base = a.sbase;
    sp.shift = 8 * pass;
    sp.tiles = sg.tiles;
    sp.slice_edges = sg.slice_edges;
    k_esort_hist<IT><<<grid, 256, 0, st>>>(a, sp);
    note_launch();
    k_esort_scan<<<sg.BG, 1024, 0, st>>>(sp);
    note_launch();
    if (sp.final_pass) {
      k_esort_base<<<1, 1024, 0, st>>>(sp, sg.BG);
      note_launch();
    }
    k_esort_scatter<IT><<<grid, 256, 0, st>>>(a, sp);
    note_launch();
    kin = sp.kout;
    iin = sp.iout;
  }
  const int64_t keys = (int64_t)sg.BG * a.M;
  k_seg_starts<<<(unsigned)((keys + 1 + 255) / 256), 256, 0, st>>>(a, a.sbase + sg.BG);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_build_csr(const AttnDev& a, cudaStream_t st) {
  return a.nb_i64 ? build_csr_t<int64_t>(a, st) : build_csr_t<int32_t>(a, st);
}

template <int DT, int EPL, bool FP32W, typename IT>
static cudaError_t bwd_rows_t(const AttnDev& a, cudaStream_t st) {
  const int Kp = (a.Kn + 31) & ~31;
  if constexpr (!(DT == kDtBF16 && EPL < 8) && EPL <= 16) {
    if (fwd_vec16_ok<DT, EPL>(a) && (reinterpret_cast<uintptr_t>(a.dO) % 16) == 0 &&
        ((a.o_sb | a.o_sh | a.o_sn) * (DT == kDtF32 ? 4 : 2)) % 16 == 0) {
      const size_t smem = (size_t)8 * 3 * Kp * sizeof(float);
      auto fn = k_attn_bwd_rows_v16<DT, EPL, FP32W, IT>;
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      const int64_t rows = (int64_t)a.B * a.H * a.N;
      fn<<<(unsigned)((rows + 7) / 8), 256, smem, st>>>(a);
      note_launch();
      return cudaGetLastError();
    }
  }
  const size_t smem = (size_t)8 * 2 * Kp * sizeof(float);
  auto fn = k_attn_bwd_rows<DT, EPL, FP32W, IT>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t rows = (int64_t)a.B * a.H * a.N;
  fn<<<(unsigned)((rows + 7) / 8), 256, smem, st>>>(a);
  note_launch();
  return cudaGetLastError();
}

template <int DT, int EPL>
static cudaError_t bwd_rows_e(const AttnDev& a, cudaStream_t st) {
  if (a.fp32w) return a.nb_i64 ? bwd_rows_t<DT, EPL, true, int64_t>(a, st) : bwd_rows_t<DT, EPL, true, int32_t>(a, st);
  return a.nb_i64 ? bwd_rows_t<DT, EPL, false, int64_t>(a, st) : bwd_rows_t<DT, EPL, false, int32_t>(a, st);
}

template <int DT>
static cudaError_t bwd_d(const AttnDev& a, bool build_csr, cudaStream_t st) {
  cudaError_t e;
  if (a.d <= 32) e = bwd_rows_e<DT, 4>(a, st);
  else if (a.d <= 64) e = bwd_rows_e<DT, 8>(a, st);
  else if (a.d <= 128) e = bwd_rows_e<DT, 16>(a, st);
  else e = bwd_rows_e<DT, 32>(a, st);
  if (e != cudaSuccess) return e;
  if (build_csr && (e = launch_build_csr(a, st)) != cudaSuccess) return e;
  const int64_t E = (int64_t)a.B * a.H * a.N * a.Kn;
  const int64_t keys = (int64_t)a.B * a.n_kv * a.M;
  const int64_t chunks = (E + kDkdvChunk - 1) / kDkdvChunk;
  const unsigned grid = (unsigned)((chunks + 7) / 8);
  if (chunks > 0) {
    // bf16 rows that are 16-byte aligned with d a multiple of 8: 16-byte loads
    const int es = DT == kDtF32 ? 4 : 2;
    auto al = [&](const void* p) { return (reinterpret_cast<uintptr_t>(p) % 16) == 0; };
    const bool v16 = DT == kDtBF16 && a.d % 8 == 0 && al(a.q) && al(a.dO) &&
                     ((a.q_sb | a.q_sh | a.q_sn | a.o_sb | a.o_sh | a.o_sn) * es) % 16 == 0;
    if (v16) k_dkdv<DT, 8, true><<<grid, 256, 0, st>>>(a);
    else if (a.d <= 128) k_dkdv<DT, 4, false><<<grid, 256, 0, st>>>(a);
    else k_dkdv<DT, 8, false><<<grid, 256, 0, st>>>(a);
    note_launch();
  }
  k_dkdv_fix<DT><<<(unsigned)((keys + 7) / 8), 256, 0, st>>>(a);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_attn_bwd(const AttnDev& a, bool build_csr, cudaStream_t st) {
  return a.dtype == kDtF32 ? bwd_d<kDtF32>(a, build_csr, st) : bwd_d<kDtBF16>(a, build_csr, st);
}

}  // namespace ssa
