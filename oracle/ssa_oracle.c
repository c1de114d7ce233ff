/*
 * ssa_oracle.c -- CPU restatement of SSA's sparse-attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA path
 * and the timed CPU baseline ("port") in bench.py. Nothing in the ssa_b200
 * package links, loads or calls it.
 *
 * It restates, step by step and in plain C, the algorithm of the reference's
 * `sparse_attention.py` (daedalus/SSA). Every function cites the reference
 * lines it follows. Two deliberate choices, both documented in the tests:
 *   - the bucket sort is the canonical STABLE order (ascending key index inside
 *     a bucket), the order the golden fixtures were generated with;
 *   - dot products accumulate in double, so oracle scores and hash projections
 *     are the exactly rounded values. The reference (fp32 sgemm) and the GPU
 *     (fp32 FMA) can only disagree with them where a projection is within
 *     rounding of zero or two candidate scores tie within rounding; the tests
 *     attribute every disagreement to one of those two causes.
 *
 * Layouts (all contiguous, row-major):
 *   q         (B, H, N, d)        float (bf16 inputs are passed widened)
 *   k, v      (B, n_kv, M, d)     float; head h reads kv head h / (H / n_kv)
 *   rand_proj (R, maxP, d)        float
 *   glob      (G,)                int32, already clamped to [0, M-1]
 *   lsh       (B, H, N, A)        int32
 *   nb, valid (B, H, N, Kout)     int32 / uint8
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORA_EXPORT __attribute__((visibility("default")))

static float bf16_round(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return f; /* NaN passes through */
  u += 0x7fffu + ((u >> 16) & 1u);                /* round to nearest even */
  u &= 0xffff0000u;
  memcpy(&f, &u, 4);
  return f;
}

static double dot_d(const float* a, const float* b, int d) {
  double s = 0.0;
  for (int t = 0; t < d; ++t) s += (double)a[t] * (double)b[t];
  return s;
}

/* p_eff = clamp(round(log2(M / C)), 1, max_p), Python round = half to even.
 * sparse_attention.py:552-557. */
ORA_EXPORT int ora_effective_p(int64_t M, int64_t C, int max_p) {
  if (M <= 1 || C <= 0) return 1;
  double x = log2((double)(M > 1 ? M : 1) / (double)(C > 1 ? C : 1));
  double r = nearbyint(x); /* default rounding mode: half to even */
  int p = (int)r;
  if (p > max_p) p = max_p;
  if (p < 1) p = 1;
  return p;
}

/* Bucket ids of `rows` vectors for one round: id = sum_j [x . P_j > 0] 2^j
 * (plane 0 = least significant bit). _hash / _hash_proj,
 * sparse_attention.py:559-597. `proj` (rows x p) is optional. */
static void hash_rows(const float* x, int64_t rows, int d, const float* planes,
                      int p, int32_t* ids, double* proj) {
  for (int64_t i = 0; i < rows; ++i) {
    int32_t id = 0;
    for (int j = 0; j < p; ++j) {
      double s = dot_d(x + i * d, planes + (int64_t)j * d, d);
      if (proj) proj[i * p + j] = s;
      if (s > 0.0) id |= (1 << j);
    }
    ids[i] = id;
  }
}

typedef struct {
  double s;
  int32_t key;
  int32_t pos;
} Cand;

static int cand_cmp(const void* a, const void* b) {
  const Cand* x = (const Cand*)a;
  const Cand* y = (const Cand*)b;
  if (x->s > y->s) return -1;
  if (x->s < y->s) return 1;
  return x->pos - y->pos;
}

/*
 * LSHGraphBuilder.forward for all (b, h): sparse_attention.py:814-959, with
 * _single_round (:741-812), _probe_ids (:599-646) and _gather_bucket
 * (:648-739). Output lsh (B,H,N,A) in the reference's order: eligible keys by
 * descending score, then the fallback slots. Optional k_ids (B*H,R,M) and
 * q_ids (B*H,R,N) expose the per-round bucket ids.
 */
ORA_EXPORT int ora_lsh_select(const float* q, const float* k, int B, int H,
                              int n_kv, int N, int M, int d,
                              const float* rand_proj, int R, int maxP, int p,
                              int C, int T, int A, int causal,
                              const int32_t* glob, int G, int32_t* lsh,
                              int32_t* k_ids_out, int32_t* q_ids_out) {
  if (H % n_kv || p < 1 || p > 30) return 1;
  const int rep = H / n_kv;
  const int Te = T < p ? T : p;
  const int nb = 1 << p;
  const int ntile = R * (1 + Te);
  const int BH = B * H;
  int32_t* kid = (int32_t*)malloc(sizeof(int32_t) * (size_t)BH * R * M);
  int32_t* perm = (int32_t*)malloc(sizeof(int32_t) * (size_t)BH * R * M);
  int32_t* bstart = (int32_t*)malloc(sizeof(int32_t) * (size_t)BH * R * nb);
  int32_t* bsize = (int32_t*)calloc((size_t)BH * R * nb, sizeof(int32_t));
  int32_t* qid = (int32_t*)malloc(sizeof(int32_t) * (size_t)BH * R * N);
  double* qproj = (double*)malloc(sizeof(double) * (size_t)BH * R * N * p);
  if (!kid || !perm || !bstart || !bsize || !qid || !qproj) {
    free(kid); free(perm); free(bstart); free(bsize); free(qid); free(qproj);
    return 2;
  }
  /* Phase 1, per (b, h, round): hash keys and queries, then the stable bucket
   * sort (canonical order for :781) and its tables: bstart = first sorted
   * position, M when empty (:789-791); bsize = count (:792). */
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int bh = 0; bh < BH; ++bh)
    for (int r = 0; r < R; ++r) {
      const int b = bh / H, h = bh % H;
      const float* kp = k + (((int64_t)b * n_kv + h / rep) * M) * d;
      const float* qp = q + ((int64_t)bh * N) * d;
      const float* planes = rand_proj + (int64_t)r * maxP * d;
      const int64_t sr = (int64_t)bh * R + r;
      int32_t* ki = kid + sr * M;
      hash_rows(kp, M, d, planes, p, ki, NULL);
      hash_rows(qp, N, d, planes, p, qid + sr * N, qproj + sr * N * p);
      int32_t* bs = bsize + sr * nb;
      int32_t* bst = bstart + sr * nb;
      for (int m = 0; m < M; ++m) bs[ki[m]]++;
      int acc = 0;
      for (int u = 0; u < nb; ++u) {
        bst[u] = bs[u] ? acc : M;
        acc += bs[u];
      }
      int32_t* fill = (int32_t*)calloc(nb, sizeof(int32_t));
      for (int m = 0; m < M; ++m) {
        const int u = ki[m];
        perm[sr * M + bst[u] + fill[u]++] = m;
      }
      free(fill);
      if (k_ids_out) memcpy(k_ids_out + sr * M, ki, sizeof(int32_t) * M);
      if (q_ids_out) memcpy(q_ids_out + sr * N, qid + sr * N, sizeof(int32_t) * N);
    }
  /* Phase 2, per query row. */
  int err = 0;
#pragma omp parallel
  {
    int64_t* stamp = (int64_t*)malloc(sizeof(int64_t) * (size_t)M);
    int32_t* tile_id = (int32_t*)malloc(sizeof(int32_t) * (size_t)ntile);
    Cand* cand = (Cand*)malloc(sizeof(Cand) * ((size_t)ntile * C + 1));
    const int ok = stamp && tile_id && cand;
    if (!ok) {
#pragma omp atomic write
      err = 2;
    } else {
      for (int m = 0; m < M; ++m) stamp[m] = -1;
    }
    {
#pragma omp for schedule(dynamic, 64)
      for (int64_t row = 0; row < (int64_t)BH * N; ++row) {
        if (!ok) continue;
        const int bh = (int)(row / N), n = (int)(row % N);
        const int b = bh / H, h = bh % H;
        const float* kp = k + (((int64_t)b * n_kv + h / rep) * M) * d;
        const float* qr = q + row * d;
        /* Tile bucket ids in concatenation order: round-major, then the
         * primary id followed by probes 1..Te (:843, :876-878). A probe flips
         * the bit with the t-th smallest |proj| of the ORIGINAL id
         * (:629-645); equal magnitudes keep plane order. */
        for (int r = 0; r < R; ++r) {
          const int64_t sr = (int64_t)bh * R + r;
          const double* pr = qproj + (sr * N + n) * p;
          int order[32];
          for (int j = 0; j < p; ++j) order[j] = j;
          for (int i = 1; i < p; ++i) { /* insertion sort, stable */
            const int o = order[i];
            const double mo = fabs(pr[o]);
            int j = i - 1;
            while (j >= 0 && fabs(pr[order[j]]) > mo) {
              order[j + 1] = order[j];
              --j;
            }
            order[j + 1] = o;
          }
          const int base = qid[sr * N + n];
          tile_id[r * (1 + Te)] = base;
          for (int t = 0; t < Te; ++t) tile_id[r * (1 + Te) + 1 + t] = base ^ (1 << order[t]);
        }
        /* Materialise the candidate entries exactly as _gather_bucket does,
         * then keep only the first occurrence of each key (cross-round
         * dedup, :884-890): an entry survives iff it is valid AND no earlier
         * entry, valid or not, holds the same key. */
        int ne = 0, pos = 0;
        for (int t = 0; t < ntile; ++t) {
          const int64_t sr = (int64_t)bh * R + t / (1 + Te);
          const int u = tile_id[t];
          const int s = bsize[sr * nb + u];
          const int st = bstart[sr * nb + u];
          for (int c = 0; c < C; ++c, ++pos) {
            int key, valid;
            if (s == 0) { /* empty bucket: globals then zeros, all valid (:711-737) */
              key = c < G ? glob[c] : 0;
              valid = 1;
            } else {
              if (c < s) {
                key = perm[sr * M + st + c];
                valid = 1;
              } else { /* overflow slot reads perm[M-1], invalid (:686-696) */
                key = perm[sr * M + M - 1];
                valid = 0;
              }
              if (causal && key > n) key = n; /* future -> self (:698-709) */
            }
            if (stamp[key] == row) continue; /* not the first occurrence */
            stamp[key] = row;
            if (!valid) continue;
            cand[ne].key = key;
            cand[ne].pos = pos;
            cand[ne].s = dot_d(qr, kp + (int64_t)key * d, d);
            ne++;
          }
        }
        /* Rescore + top-k (:896-922): the best A eligible keys by score. */
        qsort(cand, ne, sizeof(Cand), cand_cmp);
        int32_t* out = lsh + row * A;
        for (int j = 0; j < A; ++j) {
          if (j < ne) out[j] = cand[j].key;
          else out[j] = j < G ? glob[j] : 0; /* -inf slots -> fallback (:948-957) */
        }
      }
    }
    free(stamp); free(tile_id); free(cand);
  }
  free(kid); free(perm); free(bstart); free(bsize); free(qid); free(qproj);
  return err;
}

static int cmp_i32(const void* a, const void* b) {
  int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
  return (x > y) - (x < y);
}

/* Output width of merge_neighbors: self-attention keeps self + the first K-1
 * deduplicated slots, cross-attention the first K (:1071-1076). */
ORA_EXPORT int ora_merge_width(int K, int Kall, int is_cross) {
  if (is_cross) return K < Kall ? K : Kall;
  return (K - 1 < Kall ? K - 1 : Kall) + 1;
}

/*
 * WindowGraphBuilder.forward (:368-376), GlobalGraphBuilder (:411-415, given
 * as `glob`) and merge_neighbors (:966-1089) for all (b, h, n).
 */
ORA_EXPORT int ora_merge(const int32_t* lsh, int B, int H, int N, int M, int A,
                         int w, const int32_t* glob, int G, int causal,
                         int is_cross, int K, int32_t* nb_out, uint8_t* valid_out) {
  const int Kw = is_cross ? 0 : 2 * w + 1;
  const int Kall = Kw + G + A;
  const int Kout = ora_merge_width(K, Kall, is_cross);
  /* true_max_idx is one maximum over the whole combined tensor (:1031). */
  int64_t true_max = -1;
  for (int n = 0; n < N && Kw; ++n)
    for (int o = -w; o <= w; ++o) {
      int64_t idx = (causal && o > 0) ? n : (int64_t)n + o;
      if (idx < 0) idx = 0;
      if (idx > M - 1) idx = M - 1;
      if (idx > true_max) true_max = idx;
    }
  for (int g = 0; g < G; ++g) if (glob[g] > true_max) true_max = glob[g];
  for (int64_t i = 0; i < (int64_t)B * H * N * A; ++i) if (lsh[i] > true_max) true_max = lsh[i];
  const int64_t sentinel = true_max + 1;
#pragma omp parallel
  {
    int64_t* comb = (int64_t*)malloc(sizeof(int64_t) * (Kall + 1));
    int32_t* tmp = (int32_t*)malloc(sizeof(int32_t) * (Kall + 1));
#pragma omp for schedule(static)
    for (int64_t row = 0; row < (int64_t)B * H * N; ++row) {
      const int n = (int)(row % N);
      int c = 0;
      for (int o = -w; o <= w && Kw; ++o) {
        int64_t idx = (causal && o > 0) ? n : (int64_t)n + o;
        if (idx < 0) idx = 0;
        if (idx > M - 1) idx = M - 1;
        comb[c++] = idx;
      }
      for (int g = 0; g < G; ++g) comb[c++] = glob[g];
      for (int j = 0; j < A; ++j) comb[c++] = lsh[row * A + j];
      if (!is_cross)
        for (int j = 0; j < Kall; ++j) if (comb[j] == n) comb[j] = sentinel;
      /* sort, mark non-first duplicates as sentinel, sort again */
      for (int j = 0; j < Kall; ++j) tmp[j] = (int32_t)comb[j];
      qsort(tmp, Kall, sizeof(int32_t), cmp_i32);
      for (int j = Kall - 1; j >= 1; --j) if (tmp[j] == tmp[j - 1]) tmp[j] = (int32_t)sentinel;
      qsort(tmp, Kall, sizeof(int32_t), cmp_i32);
      int32_t* o = nb_out + row * Kout;
      uint8_t* v = valid_out + row * Kout;
      int off = 0;
      if (!is_cross) {
        o[0] = n;
        v[0] = 1;
        off = 1;
      }
      for (int j = off; j < Kout; ++j) {
        int64_t x = tmp[j - off];
        v[j] = x <= true_max;
        o[j] = x > true_max ? 0 : (int32_t)x;
      }
      for (int j = 0; j < Kout; ++j) { /* out.clamp(0, true_max) (:1089) */
        if (o[j] > true_max) o[j] = (int32_t)true_max;
        if (o[j] < 0) o[j] = 0;
      }
    }
    free(comb);
    free(tmp);
  }
  return 0;
}

/*
 * sparse_gather_attention forward (:1096-1199). `lowp` = 1 when q/k/v are
 * bf16: the default path rounds the fp32 softmax weights to bf16 before the
 * value sum and rounds the output to bf16 (:1190, :1198); with fp32_w the
 * weights stay fp32 and only the output is rounded (:1176-1181, :1199).
 * lse (B,H,N) receives max + log(sum) of the masked fp32 scores.
 */
ORA_EXPORT int ora_attn_fwd(const float* q, const float* k, const float* v,
                            const int32_t* nb, const uint8_t* valid, int B, int H,
                            int n_kv, int N, int M, int d, int Kn, float scale,
                            int lowp, int fp32_w, float* out, float* lse) {
  if (H % n_kv) return 1;
  const int rep = H / n_kv;
#pragma omp parallel
  {
    double* s = (double*)malloc(sizeof(double) * Kn);
    double* acc = (double*)malloc(sizeof(double) * d);
#pragma omp for schedule(static)
    for (int64_t row = 0; row < (int64_t)B * H * N; ++row) {
      const int64_t bh = row / N;
      const int b = (int)(bh / H), h = (int)(bh % H);
      const float* kp = k + (((int64_t)b * n_kv + h / rep) * M) * d;
      const float* vp = v + (((int64_t)b * n_kv + h / rep) * M) * d;
      const float* qr = q + row * d;
      double mx = -INFINITY;
      for (int j = 0; j < Kn; ++j) {
        if (!valid[row * Kn + j]) { s[j] = -INFINITY; continue; }
        float sc = (float)dot_d(qr, kp + (int64_t)nb[row * Kn + j] * d, d);
        s[j] = (double)(sc * scale);
        if (s[j] > mx) mx = s[j];
      }
      double z = 0.0;
      for (int j = 0; j < Kn; ++j) z += (s[j] == -INFINITY) ? 0.0 : exp(s[j] - mx);
      for (int t = 0; t < d; ++t) acc[t] = 0.0;
      for (int j = 0; j < Kn; ++j) {
        if (s[j] == -INFINITY) continue;
        float pj = (float)(exp(s[j] - mx) / z);
        if (lowp && !fp32_w) pj = bf16_round(pj);
        const float* vr = vp + (int64_t)nb[row * Kn + j] * d;
        for (int t = 0; t < d; ++t) acc[t] += (double)pj * vr[t];
      }
      for (int t = 0; t < d; ++t) out[row * d + t] = lowp ? bf16_round((float)acc[t]) : (float)acc[t];
      if (lse) lse[row] = (float)(mx + log(z));
    }
    free(s);
    free(acc);
  }
  return 0;
}

/*
 * Gradient of sum(out * dO) through sparse_gather_attention, computed in
 * double: dV[nb] += p * dO, dP = dO . V[nb], dS = p (dP - sum p dP),
 * dQ = scale sum dS K[nb], dK[nb] += scale dS q; heads of one kv group sum
 * into the same dK/dV (the repeat_interleave backward). For bf16 inputs the
 * upstream gradient and the value weights are the bf16-rounded ones the
 * reference's autograd sees.
 */
ORA_EXPORT int ora_attn_bwd(const float* q, const float* k, const float* v,
                            const int32_t* nb, const uint8_t* valid, const float* dO,
                            int B, int H, int n_kv, int N, int M, int d, int Kn,
                            float scale, int lowp, int fp32_w, float* dq,
                            float* dk, float* dv) {
  if (H % n_kv) return 1;
  const int rep = H / n_kv;
  const int64_t kv_elems = (int64_t)B * n_kv * M * d;
  double* dk_acc = (double*)calloc(kv_elems, sizeof(double));
  double* dv_acc = (double*)calloc(kv_elems, sizeof(double));
  if (!dk_acc || !dv_acc) { free(dk_acc); free(dv_acc); return 2; }
  /* rows of one kv group write the same dK/dV slice: parallelise over groups */
#pragma omp parallel
  {
    double* s = (double*)malloc(sizeof(double) * Kn);
    double* pw = (double*)malloc(sizeof(double) * Kn);
    double* dp = (double*)malloc(sizeof(double) * Kn);
    double* g = (double*)malloc(sizeof(double) * d);
#pragma omp for schedule(dynamic, 1)
    for (int bg = 0; bg < B * n_kv; ++bg) {
      const int b = bg / n_kv, gk = bg % n_kv;
      const float* kp = k + ((int64_t)bg * M) * d;
      const float* vp = v + ((int64_t)bg * M) * d;
      double* dkp = dk_acc + ((int64_t)bg * M) * d;
      double* dvp = dv_acc + ((int64_t)bg * M) * d;
      for (int h = gk * rep; h < (gk + 1) * rep; ++h)
        for (int n = 0; n < N; ++n) {
          const int64_t row = ((int64_t)b * H + h) * N + n;
          const float* qr = q + row * d;
          double mx = -INFINITY;
          for (int j = 0; j < Kn; ++j) {
            if (!valid[row * Kn + j]) { s[j] = -INFINITY; continue; }
            float sc = (float)dot_d(qr, kp + (int64_t)nb[row * Kn + j] * d, d);
            s[j] = (double)(sc * scale);
            if (s[j] > mx) mx = s[j];
          }
          double z = 0.0;
          for (int j = 0; j < Kn; ++j) z += (s[j] == -INFINITY) ? 0.0 : exp(s[j] - mx);
          for (int t = 0; t < d; ++t) g[t] = lowp ? bf16_round(dO[row * d + t]) : dO[row * d + t];
          double sum_pdp = 0.0;
          for (int j = 0; j < Kn; ++j) {
            if (s[j] == -INFINITY) { pw[j] = 0.0; dp[j] = 0.0; continue; }
            float p32 = (float)(exp(s[j] - mx) / z);
            float pv = (lowp && !fp32_w) ? bf16_round(p32) : p32;
            pw[j] = p32;
            const int64_t key = nb[row * Kn + j];
            double acc = 0.0;
            for (int t = 0; t < d; ++t) {
              acc += g[t] * (double)vp[key * d + t];
              dvp[key * d + t] += (double)pv * g[t];
            }
            dp[j] = acc;
            sum_pdp += pw[j] * acc;
          }
          for (int t = 0; t < d; ++t) dq[row * d + t] = 0.0f;
          double* dqr = (double*)calloc(d, sizeof(double));
          for (int j = 0; j < Kn; ++j) {
            if (s[j] == -INFINITY) continue;
            const double ds = pw[j] * (dp[j] - sum_pdp) * scale;
            const int64_t key = nb[row * Kn + j];
            for (int t = 0; t < d; ++t) {
              dqr[t] += ds * kp[key * d + t];
              dkp[key * d + t] += ds * qr[t];
            }
          }
          for (int t = 0; t < d; ++t) dq[row * d + t] = (float)dqr[t];
          free(dqr);
        }
    }
    free(s); free(pw); free(dp); free(g);
  }
  for (int64_t i = 0; i < kv_elems; ++i) {
    dk[i] = (float)dk_acc[i];
    dv[i] = (float)dv_acc[i];
  }
  free(dk_acc);
  free(dv_acc);
  return 0;
}

ORA_EXPORT int ora_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
