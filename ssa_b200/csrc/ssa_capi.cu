// ssa_capi.cu -- the extern "C" entry points declared in include/ssa_b200.h.
//
// Validates shapes, strides and alignment, carves the caller's workspace,
// and enqueues the kernels on the caller's stream. Nothing here allocates,
// synchronises or touches host-side tensors.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "../../include/ssa_b200.h"
#include "ssa_common.cuh"
#include "ssa_internal.h"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SSA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int elem_align(int dtype) { return dtype == SSA_F32 ? 16 : 8; }

int check_rows(const char* name, const void* ptr, int dtype, int d, int64_t s0, int64_t s1,
               int64_t s2) {
  if (!ptr) return fail(SSA_ERR_INVALID, "%s is NULL", name);
  if (!aligned(ptr, elem_align(dtype)))
    return fail(SSA_ERR_UNSUPPORTED, "%s must be %d-byte aligned", name, elem_align(dtype));
  if (d % 4) return fail(SSA_ERR_UNSUPPORTED, "head dim d=%d must be a multiple of 4", d);
  if ((s0 % 4) || (s1 % 4) || (s2 % 4))
    return fail(SSA_ERR_UNSUPPORTED, "%s strides (%lld,%lld,%lld) must be multiples of 4 elements",
                name, (long long)s0, (long long)s1, (long long)s2);
  if (s0 < 0 || s1 < 0 || s2 < 0) return fail(SSA_ERR_INVALID, "%s has a negative stride", name);
  return SSA_OK;
}

int32_t graph_width(const ssa_graph_params* p) {
  const int kw = p->is_cross ? 0 : 2 * p->window + 1;
  const int kall = kw + p->G + p->A;
  if (p->is_cross) return p->K < kall ? p->K : kall;
  return (p->K - 1 < kall ? p->K - 1 : kall) + 1;
}

int check_graph(const ssa_graph_params* p) {
  if (!p) return fail(SSA_ERR_INVALID, "params is NULL");
  if (p->B < 1 || p->H < 1 || p->n_kv < 1 || p->N < 1 || p->M < 1 || p->d < 1)
    return fail(SSA_ERR_INVALID, "B,H,n_kv,N,M,d must be >= 1");
  if (p->H % p->n_kv)
    return fail(SSA_ERR_INVALID, "num_heads (%d) must be divisible by num_kv_heads (%d)", p->H, p->n_kv);
  if (p->dtype != SSA_F32 && p->dtype != SSA_BF16) return fail(SSA_ERR_INVALID, "dtype must be F32 or BF16");
  if (p->d > 128) return fail(SSA_ERR_UNSUPPORTED, "graph build supports head dim <= 128 (got %d)", p->d);
  if (p->R < 1 || p->R > 64) return fail(SSA_ERR_INVALID, "num_hash_rounds must be in [1, 64]");
  if (p->max_p < 1 || p->max_p > 12)
    return fail(SSA_ERR_INVALID, "max_num_hashes must be in [1, 12] (reference asserts <= 12)");
  if (p->p_eff < 1 || p->p_eff > p->max_p) return fail(SSA_ERR_INVALID, "p_eff must be in [1, max_num_hashes]");
  if (p->C < 1 || p->A < 1 || p->T < 0 || p->K < 1 || p->window < 0 || p->G < 0)
    return fail(SSA_ERR_INVALID, "C, A, K >= 1 and T, window, G >= 0 required");
  if (p->M > (1 << 20)) return fail(SSA_ERR_UNSUPPORTED, "key length M=%d exceeds 2^20", p->M);
  if (p->N > (1 << 30)) return fail(SSA_ERR_UNSUPPORTED, "query length too large");
  if (p->q_row0 < 0 || (int64_t)p->q_row0 + p->N > (int64_t(1) << 30))
    return fail(SSA_ERR_INVALID, "q_row0=%d out of range", p->q_row0);
  if ((int64_t)p->B * p->H > 65535 || (int64_t)p->B * p->n_kv > 65535)
    return fail(SSA_ERR_UNSUPPORTED, "B*H must be <= 65535");
  if (p->is_cross && p->causal) return fail(SSA_ERR_INVALID, "cross-attention is never causal");
  return SSA_OK;
}

// Polls before a tensor-core scan wait gives up (ssa_debug_set_wait_limit);
// 0: the default, 2^24.
std::atomic<uint32_t> g_wait_limit{0};
// Hashing on the tensor cores where supported (ssa_debug_set_hash), the
// certification constant c (0: the default 2^-14), and the projection dump.
std::atomic<int> g_hash_tc{1};
std::atomic<float> g_hash_eps{0.f};
std::mutex g_dump_mu;
float* g_dump = nullptr;
int64_t g_dump_n = 0;

ssa::GraphDev dev_of(const ssa_graph_params* p) {
  ssa::GraphDev g;
  memset(&g, 0, sizeof(g));
  const uint32_t wl = g_wait_limit.load(std::memory_order_relaxed);
  g.wait_limit = wl ? wl : (1u << 24);
  g.B = p->B; g.H = p->H; g.n_kv = p->n_kv; g.rep = p->H / p->n_kv; g.N = p->N; g.M = p->M;
  g.d = p->d; g.dtype = p->dtype; g.R = p->R; g.max_p = p->max_p; g.p = p->p_eff; g.C = p->C;
  g.Te = p->T < p->p_eff ? p->T : p->p_eff;
  g.NT = g.R * (1 + g.Te);
  g.NB = 1 << g.p;
  g.W = (p->M + 63) / 64;
  g.Wpad = (g.W + 1) / 2 * 2;
  g.A = p->A; g.causal = p->causal; g.is_cross = p->is_cross; g.window = p->window; g.G = p->G;
  g.row0 = p->q_row0;
  g.Wout = graph_width(p);
  g.q_sb = p->q_sb; g.q_sh = p->q_sh; g.q_sn = p->q_sn;
  g.k_sb = p->k_sb; g.k_sh = p->k_sh; g.k_sm = p->k_sm;
  g.use_tc_hash = g_hash_tc.load(std::memory_order_relaxed);
  const float c = g_hash_eps.load(std::memory_order_relaxed);
  g.hash_eps = c > 0.f ? c : 1.f / 16384.f;
  {
    std::lock_guard<std::mutex> lk(g_dump_mu);
    if (g_dump && g_dump_n >= (int64_t)p->B * p->H * p->N * p->R * p->p_eff) g.hash_dump = g_dump;
  }
  return g;
}

int check_graph_inputs(const ssa_graph_params* p, const void* q, const void* k, const float* rp,
                       const int32_t* glob) {
  int rc;
  if ((rc = check_rows("q", q, p->dtype, p->d, p->q_sb, p->q_sh, p->q_sn))) return rc;
  if ((rc = check_rows("k", k, p->dtype, p->d, p->k_sb, p->k_sh, p->k_sm))) return rc;
  if (!rp || !aligned(rp, 16)) return fail(SSA_ERR_INVALID, "rand_proj must be a 16-byte aligned fp32 array");
  if (p->G > 0 && !glob) return fail(SSA_ERR_INVALID, "glob is NULL but G > 0");
  return SSA_OK;
}

int check_select_fits(const ssa::GraphDev& g) {
  int rows;
  size_t smem;
  if (ssa::choose_select_rows(g, &rows, &smem))
    return fail(SSA_ERR_UNSUPPORTED,
                "per-row top-k buffer does not fit in shared memory (A=%d, d=%d); reduce num_neighbors",
                g.A, g.d);
  return SSA_OK;
}

}  // namespace

namespace ssa {
static std::atomic<long long> g_kernel_launches{0};
void note_launch() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }

// Graph-build stage profiling: one set of events per process, recorded by
// every build while enabled (the device of the enabling call).
static std::mutex g_prof_mu;
static bool g_prof_on = false;
static cudaEvent_t g_prof_ev[kStageMarks] = {};

void stage_mark(int i, cudaStream_t st) {
  if (!g_prof_on) return;
  cudaEventRecord(g_prof_ev[i], st);
}
}  // namespace ssa

extern "C" {

const char* ssa_last_error(void) { return g_err; }

int32_t ssa_abi_version(void) { return 106; }

int32_t ssa_device_error(int32_t clear) { return ssa::read_device_error(clear); }

int ssa_debug_set_wait_limit(uint32_t polls) {
  g_wait_limit.store(polls, std::memory_order_relaxed);
  return SSA_OK;
}

int ssa_debug_set_hash(int32_t use_tc, float eps_c) {
  if (!(eps_c >= 0.f) || eps_c > 1.f) return fail(SSA_ERR_INVALID, "eps_c must be in [0, 1]");
  g_hash_tc.store(use_tc ? 1 : 0, std::memory_order_relaxed);
  g_hash_eps.store(eps_c, std::memory_order_relaxed);
  return SSA_OK;
}

int ssa_debug_hash_dump(float* buf, int64_t n_floats) {
  if (buf && n_floats < 0) return fail(SSA_ERR_INVALID, "n_floats must be >= 0");
  std::lock_guard<std::mutex> lk(g_dump_mu);
  g_dump = buf;
  g_dump_n = buf ? n_floats : 0;
  return SSA_OK;
}

int64_t ssa_debug_hash_recomputed(int32_t clear) {
  const unsigned long long v = ssa::read_hash_recomputed(clear);
  return v == ~0ull ? -1 : (int64_t)v;
}

int32_t ssa_graph_width(const ssa_graph_params* p) { return p ? graph_width(p) : -1; }

size_t ssa_graph_workspace_size(const ssa_graph_params* p) {
  if (check_graph(p)) return 0;
  ssa::GraphDev g = dev_of(p);
  return ssa::graph_workspace_layout(&g);
}

static int run_graph(const ssa_graph_params* p, const void* q, const void* k, const float* rp,
                     const int32_t* glob, int32_t* nb_out, uint8_t* valid_out, int32_t* lsh_out,
                     void* ws, size_t ws_bytes, void* stream, int mode, int prehashed = 0) {
  int rc;
  if ((rc = check_graph(p))) return rc;
  if ((rc = check_graph_inputs(p, q, k, rp, glob))) return rc;
  if (mode == 0 && (!nb_out || !valid_out)) return fail(SSA_ERR_INVALID, "nb_out/valid_out are NULL");
  if (mode == 1 && !lsh_out) return fail(SSA_ERR_INVALID, "lsh_out is NULL");
  ssa::GraphDev g = dev_of(p);
  const size_t need = ssa::graph_workspace_layout(&g);
  if (!ws || ws_bytes < need)
    return fail(SSA_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, ws_bytes);
  g.ws = ws;
  ssa::graph_workspace_layout(&g);
  g.q = q; g.k = k; g.rp = rp; g.glob = glob;
  g.lsh = lsh_out; g.nb = nb_out; g.valid = valid_out;
  if ((rc = check_select_fits(g))) return rc;  // the FMA scan is also the exact fallback
  if (prehashed) {
    if (!g.use_tc || !g.use_tc_hash || !ssa::select_tc_pointers_ok(g))
      return fail(SSA_ERR_UNSUPPORTED, "a prehashed build needs the tensor-core path (ssa_qkv_proj_hash_supported)");
    g.prehashed = 1;
  }
  cudaError_t e = ssa::launch_graph(g, mode, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "graph build launch");
  return SSA_OK;
}

int ssa_build_graph(const ssa_graph_params* p, const void* q, const void* k, const float* rand_proj,
                    const int32_t* glob, int32_t* nb_out, uint8_t* valid_out, int32_t* lsh_out,
                    void* workspace, size_t workspace_bytes, void* stream) {
  return run_graph(p, q, k, rand_proj, glob, nb_out, valid_out, lsh_out, workspace,
                   workspace_bytes, stream, 0);
}

// The q / k views of a fused projection output: (B, N, H + 2 n_kv, d) rows.
static bool proj_strides_ok(const ssa_graph_params* p) {
  const int64_t n_out = (int64_t)(p->H + 2 * p->n_kv) * p->d;
  return p->q_sb == (int64_t)p->N * n_out && p->q_sh == p->d && p->q_sn == n_out &&
         p->k_sb == (int64_t)p->N * n_out && p->k_sh == p->d && p->k_sm == n_out;
}

int32_t ssa_qkv_proj_hash_supported(const ssa_graph_params* p, int32_t d_model) {
  if (!p || check_graph(p)) return 0;
  ssa::GraphDev g = dev_of(p);
  ssa::graph_workspace_layout(&g);
  return (g.use_tc && g.use_tc_hash && ssa::proj_hash_supported(g, d_model) && proj_strides_ok(p)) ? 1 : 0;
}

int ssa_qkv_proj_hash(const ssa_graph_params* p, int32_t d_model, const void* x, const void* w_qkv,
                      void* qkv_out, const float* rand_proj, void* workspace, size_t workspace_bytes,
                      void* stream) {
  int rc;
  if ((rc = check_graph(p))) return rc;
  if (!ssa_qkv_proj_hash_supported(p, d_model))
    return fail(SSA_ERR_UNSUPPORTED,
                "fused projection + hash needs bf16 self-attention, head dim 64/128, N %% 128 == 0, "
                "d_model %% 64 == 0, (H + 2 n_kv) d %% 128 == 0 and q/k strides of the output views");
  if (!x || !w_qkv || !qkv_out || !aligned(x, 16) || !aligned(w_qkv, 16) || !aligned(qkv_out, 16))
    return fail(SSA_ERR_INVALID, "x, w_qkv and qkv_out must be non-null and 16-byte aligned");
  if (!rand_proj || !aligned(rand_proj, 16)) return fail(SSA_ERR_INVALID, "rand_proj must be a 16-byte aligned fp32 array");
  ssa::GraphDev g = dev_of(p);
  const size_t need = ssa::graph_workspace_layout(&g);
  if (!workspace || workspace_bytes < need)
    return fail(SSA_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  g.ws = workspace;
  ssa::graph_workspace_layout(&g);
  const int n_out = (p->H + 2 * p->n_kv) * p->d;
  g.q = qkv_out;
  g.k = static_cast<const uint16_t*>(qkv_out) + (int64_t)p->H * p->d;
  g.rp = rand_proj;
  ssa::ProjDev pd;
  pd.rows = p->B * p->N;
  pd.dm = d_model;
  pd.n_out = n_out;
  pd.x = x;
  pd.w = w_qkv;
  pd.out = qkv_out;
  cudaError_t e = ssa::launch_proj_hash(g, pd, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fused projection launch");
  return SSA_OK;
}

int ssa_build_graph_prehashed(const ssa_graph_params* p, const void* q, const void* k, const float* rand_proj,
                              const int32_t* glob, int32_t* nb_out, uint8_t* valid_out, void* workspace,
                              size_t workspace_bytes, void* stream) {
  return run_graph(p, q, k, rand_proj, glob, nb_out, valid_out, nullptr, workspace, workspace_bytes, stream, 0, 1);
}

int ssa_lsh_select(const ssa_graph_params* p, const void* q, const void* k, const float* rand_proj,
                   const int32_t* glob, int32_t* lsh_out, void* workspace, size_t workspace_bytes,
                   void* stream) {
  return run_graph(p, q, k, rand_proj, glob, nullptr, nullptr, lsh_out, workspace, workspace_bytes,
                   stream, 1);
}

int ssa_merge(const ssa_graph_params* p, const int32_t* lsh, const int32_t* glob,
              const int32_t* win, int32_t Kw, const int32_t* self_idx, const int32_t* true_max,
              int32_t* nb_out, uint8_t* valid_out, void* stream) {
  if (!p) return fail(SSA_ERR_INVALID, "params is NULL");
  if (p->B < 1 || p->H < 1 || p->N < 1 || p->A < 1 || p->K < 1 || p->G < 0 || Kw < 0)
    return fail(SSA_ERR_INVALID, "bad merge geometry");
  if (!lsh || !nb_out || !valid_out || !true_max || (Kw > 0 && !win))
    return fail(SSA_ERR_INVALID, "NULL lsh/win/true_max/nb_out/valid_out");
  if (p->G > 0 && !glob) return fail(SSA_ERR_INVALID, "glob is NULL but G > 0");
  ssa::MergeDev m;
  memset(&m, 0, sizeof(m));
  m.B = p->B; m.H = p->H; m.N = p->N; m.A = p->A; m.Kw = Kw; m.G = p->G;
  const int kall = Kw + p->G + p->A;
  m.Wout = self_idx ? (p->K - 1 < kall ? p->K - 1 : kall) + 1 : (p->K < kall ? p->K : kall);
  m.lsh = lsh; m.glob = glob; m.win = win; m.self_idx = self_idx; m.true_max = true_max;
  m.nb = nb_out; m.valid = valid_out;
  cudaError_t e = ssa::launch_merge(m, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorInvalidConfiguration)
    return fail(SSA_ERR_UNSUPPORTED, "window + LSH width (%d) too large for the merge kernel", Kw + p->A);
  if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  return SSA_OK;
}

int ssa_hash_ids(const void* x, int32_t dtype, int32_t B, int32_t heads, int32_t rows, int32_t d,
                 int64_t sb, int64_t sh, int64_t sn, const float* rand_proj, int32_t R,
                 int32_t max_p, int32_t p_eff, int32_t* ids_out, void* stream) {
  int rc;
  if (dtype != SSA_F32 && dtype != SSA_BF16) return fail(SSA_ERR_INVALID, "bad dtype");
  if (B < 1 || heads < 1 || rows < 1 || d < 1 || R < 1 || p_eff < 1 || p_eff > max_p || max_p > 12)
    return fail(SSA_ERR_INVALID, "bad hash geometry");
  if ((rc = check_rows("x", x, dtype, d, sb, sh, sn))) return rc;
  if (!rand_proj || !aligned(rand_proj, 16) || !ids_out) return fail(SSA_ERR_INVALID, "bad pointers");
  cudaError_t e = ssa::launch_hash_ids(x, dtype, B, heads, rows, d, sb, sh, sn, rand_proj, R, max_p,
                                       p_eff, ids_out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "hash launch");
  return SSA_OK;
}

static int check_attn(const ssa_attn_params* p, const void* q, const void* k, const void* v,
                      const void* nb, const uint8_t* valid) {
  if (p && !(p->dropout_p >= 0.f && p->dropout_p < 1.f))
    return fail(SSA_ERR_INVALID, "dropout_p=%g must be in [0, 1)", (double)p->dropout_p);
  int rc;
  if (!p) return fail(SSA_ERR_INVALID, "params is NULL");
  if (p->B < 1 || p->H < 1 || p->n_kv < 1 || p->N < 1 || p->M < 1 || p->d < 1 || p->Kn < 1)
    return fail(SSA_ERR_INVALID, "B,H,n_kv,N,M,d,Kn must be >= 1");
  if (p->H % p->n_kv)
    return fail(SSA_ERR_INVALID, "num_heads (%d) must be divisible by num_kv_heads (%d)", p->H, p->n_kv);
  if (p->dtype != SSA_F32 && p->dtype != SSA_BF16) return fail(SSA_ERR_INVALID, "dtype must be F32 or BF16");
  if (p->d > 256) return fail(SSA_ERR_UNSUPPORTED, "attention supports head dim <= 256 (got %d)", p->d);
  if (p->Kn > 8192) return fail(SSA_ERR_UNSUPPORTED, "at most 8192 neighbor slots");
  if ((rc = check_rows("q", q, p->dtype, p->d, p->q_sb, p->q_sh, p->q_sn))) return rc;
  if ((rc = check_rows("k", k, p->dtype, p->d, p->k_sb, p->k_sh, p->k_sm))) return rc;
  if ((rc = check_rows("v", v, p->dtype, p->d, p->v_sb, p->v_sh, p->v_sm))) return rc;
  if (!nb || !valid) return fail(SSA_ERR_INVALID, "neighbors/valid are NULL");
  return SSA_OK;
}

static ssa::AttnDev attn_dev(const ssa_attn_params* p) {
  ssa::AttnDev a;
  memset(&a, 0, sizeof(a));
  a.B = p->B; a.H = p->H; a.n_kv = p->n_kv; a.rep = p->H / p->n_kv; a.N = p->N; a.M = p->M;
  a.d = p->d; a.Kn = p->Kn; a.dtype = p->dtype; a.nb_i64 = p->nb_i64; a.fp32w = p->fp32_weights;
  a.scale = p->scale;
  a.q_sb = p->q_sb; a.q_sh = p->q_sh; a.q_sn = p->q_sn;
  a.k_sb = p->k_sb; a.k_sh = p->k_sh; a.k_sm = p->k_sm;
  a.v_sb = p->v_sb; a.v_sh = p->v_sh; a.v_sm = p->v_sm;
  a.o_sb = p->o_sb; a.o_sh = p->o_sh; a.o_sn = p->o_sn;
  if (p->dropout_p > 0.f) {
    const double t = (double)p->dropout_p * 4294967296.0;
    a.drop_thresh = t >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)t;
    a.drop_scale = (float)(1.0 / (1.0 - (double)p->dropout_p));
    a.drop_seed = p->dropout_seed;
    a.drop_offset = p->dropout_offset;
  }
  return a;
}

int ssa_attn_fwd(const ssa_attn_params* p, const void* q, const void* k, const void* v,
                 const void* nb, const uint8_t* valid, void* out, float* lse, void* stream) {
  int rc;
  if ((rc = check_attn(p, q, k, v, nb, valid))) return rc;
  if ((rc = check_rows("out", out, p->dtype, p->d, p->o_sb, p->o_sh, p->o_sn))) return rc;
  ssa::AttnDev a = attn_dev(p);
  a.q = q; a.k = k; a.v = v; a.nb = nb; a.valid = valid; a.out = out; a.lse = lse;
  cudaError_t e = ssa::launch_attn_fwd(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attention forward launch");
  return SSA_OK;
}

static int check_edges(const ssa_attn_params* p) {
  const int64_t E = (int64_t)p->B * p->H * p->N * p->Kn;
  if (E >= (int64_t(1) << 31)) return fail(SSA_ERR_UNSUPPORTED, "too many edges (%lld)", (long long)E);
  if ((int64_t)p->B * p->n_kv * p->M >= (int64_t(1) << 31))
    return fail(SSA_ERR_UNSUPPORTED, "B * n_kv * M too large");
  return SSA_OK;
}

size_t ssa_attn_bwd_workspace_size(const ssa_attn_params* p) {
  if (!p || p->B < 1 || p->H < 1 || p->N < 1 || p->Kn < 1) return 0;
  ssa::AttnDev a = attn_dev(p);
  return ssa::attn_bwd_workspace_layout(a, nullptr, nullptr);
}

int ssa_attn_bwd(const ssa_attn_params* p, const void* q, const void* k, const void* v,
                 const void* nb, const uint8_t* valid, const void* dO, const float* lse, void* dq,
                 void* dk, void* dv, void* workspace, size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = check_attn(p, q, k, v, nb, valid))) return rc;
  if ((rc = check_rows("dO", dO, p->dtype, p->d, p->o_sb, p->o_sh, p->o_sn))) return rc;
  if ((rc = check_rows("dq", dq, p->dtype, p->d, p->o_sb, p->o_sh, p->o_sn))) return rc;
  if (!lse || !dk || !dv) return fail(SSA_ERR_INVALID, "lse/dk/dv are NULL");
  if ((rc = check_edges(p))) return rc;
  ssa::AttnDev a = attn_dev(p);
  const size_t need = ssa::attn_bwd_workspace_layout(a, nullptr, nullptr);
  if (!workspace || workspace_bytes < need)
    return fail(SSA_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  ssa::attn_bwd_workspace_layout(a, &a, workspace);
  a.q = q; a.k = k; a.v = v; a.nb = nb; a.valid = valid; a.dO = dO; a.lse_in = lse;
  a.dq = dq; a.dk = dk; a.dv = dv;
  cudaError_t e = ssa::launch_attn_bwd(a, true, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attention backward launch");
  return SSA_OK;
}

size_t ssa_attn_csr_size(const ssa_attn_params* p) {
  if (!p || p->B < 1 || p->H < 1 || p->n_kv < 1 || p->N < 1 || p->M < 1 || p->Kn < 1 || p->H % p->n_kv)
    return 0;
  ssa::AttnDev a = attn_dev(p);
  return ssa::attn_csr_layout(a, nullptr, nullptr);
}

int ssa_attn_build_csr(const ssa_attn_params* p, const void* nb, const uint8_t* valid, void* csr,
                       size_t csr_bytes, void* workspace, size_t workspace_bytes, void* stream) {
  if (!p) return fail(SSA_ERR_INVALID, "params is NULL");
  if (p->B < 1 || p->H < 1 || p->n_kv < 1 || p->N < 1 || p->M < 1 || p->Kn < 1)
    return fail(SSA_ERR_INVALID, "B,H,n_kv,N,M,Kn must be >= 1");
  if (p->H % p->n_kv)
    return fail(SSA_ERR_INVALID, "num_heads (%d) must be divisible by num_kv_heads (%d)", p->H, p->n_kv);
  if (!nb || !valid) return fail(SSA_ERR_INVALID, "neighbors/valid are NULL");
  int rc;
  if ((rc = check_edges(p))) return rc;
  ssa::AttnDev a = attn_dev(p);
  const size_t need_csr = ssa::attn_csr_layout(a, nullptr, nullptr);
  if (!csr || csr_bytes < need_csr)
    return fail(SSA_ERR_WORKSPACE, "csr buffer of %zu bytes needed, %zu given", need_csr, csr_bytes);
  const size_t need = ssa::attn_bwd_workspace_layout(a, nullptr, nullptr);
  if (!workspace || workspace_bytes < need)
    return fail(SSA_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  ssa::attn_bwd_workspace_layout(a, &a, workspace);
  ssa::attn_csr_layout(a, &a, csr);
  a.nb = nb; a.valid = valid;
  cudaError_t e = ssa::launch_build_csr(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "inverted index launch");
  return SSA_OK;
}

int ssa_attn_bwd_csr(const ssa_attn_params* p, const void* q, const void* k, const void* v,
                     const void* nb, const uint8_t* valid, const void* dO, const float* lse, void* dq,
                     void* dk, void* dv, const void* csr, size_t csr_bytes, void* workspace,
                     size_t workspace_bytes, void* stream) {
  int rc;
  if ((rc = check_attn(p, q, k, v, nb, valid))) return rc;
  if ((rc = check_rows("dO", dO, p->dtype, p->d, p->o_sb, p->o_sh, p->o_sn))) return rc;
  if ((rc = check_rows("dq", dq, p->dtype, p->d, p->o_sb, p->o_sh, p->o_sn))) return rc;
  if (!lse || !dk || !dv) return fail(SSA_ERR_INVALID, "lse/dk/dv are NULL");
  if ((rc = check_edges(p))) return rc;
  ssa::AttnDev a = attn_dev(p);
  const size_t need_csr = ssa::attn_csr_layout(a, nullptr, nullptr);
  if (!csr || csr_bytes < need_csr)
    return fail(SSA_ERR_WORKSPACE, "csr buffer of %zu bytes needed, %zu given", need_csr, csr_bytes);
  const size_t need = ssa::attn_bwd_workspace_layout(a, nullptr, nullptr);
  if (!workspace || workspace_bytes < need)
    return fail(SSA_ERR_WORKSPACE, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  ssa::attn_bwd_workspace_layout(a, &a, workspace);
  ssa::attn_csr_layout(a, &a, const_cast<void*>(csr));
  a.q = q; a.k = k; a.v = v; a.nb = nb; a.valid = valid; a.dO = dO; a.lse_in = lse;
  a.dq = dq; a.dk = dk; a.dv = dv;
  cudaError_t e = ssa::launch_attn_bwd(a, false, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attention backward launch");
  return SSA_OK;
}

// neighbor_overlap: per-row Jaccard similarity of two neighbor sets.
int ssa_neighbor_overlap(const void* nb_a, const uint8_t* valid_a, const void* nb_b, const uint8_t* valid_b,
                         int64_t rows, int32_t K, int32_t nb_i64, float* out, void* stream) {
  if (rows < 0 || K < 1) return fail(SSA_ERR_INVALID, "rows=%lld, K=%d", (long long)rows, K);
  if (rows == 0) return SSA_OK;
  if (!nb_a || !valid_a || !nb_b || !valid_b || !out) return fail(SSA_ERR_INVALID, "NULL pointer");
  if (K > 2048) return fail(SSA_ERR_UNSUPPORTED, "neighbor_overlap supports K <= 2048 (got %d)", K);
  const size_t isz = nb_i64 ? 8 : 4;
  if (!aligned(nb_a, isz) || !aligned(nb_b, isz)) return fail(SSA_ERR_INVALID, "neighbor arrays misaligned");
  cudaError_t e = ssa::launch_neighbor_overlap(nb_a, valid_a, nb_b, valid_b, rows, K, nb_i64, out,
                                               static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "neighbor_overlap launch");
  return SSA_OK;
}

int64_t ssa_kernel_launches(void) { return ssa::g_kernel_launches.load(std::memory_order_relaxed); }

int ssa_graph_profile(int32_t enable) {
  std::lock_guard<std::mutex> lock(ssa::g_prof_mu);
  if (enable && !ssa::g_prof_on) {
    for (int i = 0; i < ssa::kStageMarks; ++i) {
      cudaError_t e = cudaEventCreate(&ssa::g_prof_ev[i]);
      if (e != cudaSuccess) {
        for (int j = 0; j < i; ++j) cudaEventDestroy(ssa::g_prof_ev[j]);
        return cuda_fail(e, "cudaEventCreate (graph profiling)");
      }
    }
    ssa::g_prof_on = true;
  } else if (!enable && ssa::g_prof_on) {
    ssa::g_prof_on = false;
    for (int i = 0; i < ssa::kStageMarks; ++i) cudaEventDestroy(ssa::g_prof_ev[i]);
  }
  return SSA_OK;
}

int ssa_graph_stage_times(float* ms_out) {
  std::lock_guard<std::mutex> lock(ssa::g_prof_mu);
  if (!ms_out) return fail(SSA_ERR_INVALID, "ms_out is NULL");
  if (!ssa::g_prof_on) return fail(SSA_ERR_INVALID, "graph profiling is off (ssa_graph_profile(1) first)");
  cudaError_t e = cudaEventSynchronize(ssa::g_prof_ev[ssa::kStageMarks - 1]);
  if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize (graph profiling)");
  for (int i = 0; i + 1 < ssa::kStageMarks; ++i) {
    e = cudaEventElapsedTime(&ms_out[i], ssa::g_prof_ev[i], ssa::g_prof_ev[i + 1]);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventElapsedTime (graph profiling): no profiled build yet?");
  }
  return SSA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Attention backward without a caller workspace: the scratch is a file-scope
// device array, one per device, whose address the host resolves once.
// ---------------------------------------------------------------------------
namespace {
// Nothing in it has to start at zero: k_attn_bwd_rows writes every edge entry
// (weight, dS, sort key, id) before the sort reads it, and the sort's
// temporaries need no initial value.
__device__ __align__(256) unsigned char g_attn_bwd_scratch[SSA_ATTN_BWD_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Address of this device's scratch array: cudaGetSymbolAddress on the first
// call per device (which may also load the module), cached afterwards.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(SSA_ERR_UNSUPPORTED, "device ordinal %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_attn_bwd_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static attention-backward scratch)");
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return SSA_OK;
}
}  // namespace

extern "C" {

int ssa_attn_bwd_noalloc(const ssa_attn_params* p, const void* q, const void* k, const void* v,
                         const void* nb, const uint8_t* valid, const void* dO, const float* lse,
                         void* dq, void* dk, void* dv, void* stream) {
  int rc;
  if ((rc = check_attn(p, q, k, v, nb, valid))) return rc;
  if ((rc = check_rows("dO", dO, p->dtype, p->d, p->o_sb, p->o_sh, p->o_sn))) return rc;
  if ((rc = check_rows("dq", dq, p->dtype, p->d, p->o_sb, p->o_sh, p->o_sn))) return rc;
  if (!lse || !dk || !dv) return fail(SSA_ERR_INVALID, "lse/dk/dv are NULL");
  const int64_t E = (int64_t)p->B * p->H * p->N * p->Kn;
  if (E >= (int64_t(1) << 31)) return fail(SSA_ERR_UNSUPPORTED, "too many edges (%lld)", (long long)E);
  if ((int64_t)p->B * p->n_kv * p->M >= (int64_t(1) << 31))
    return fail(SSA_ERR_UNSUPPORTED, "B * n_kv * M too large");
  ssa::AttnDev a = attn_dev(p);
  const size_t need = ssa::attn_bwd_workspace_layout(a, nullptr, nullptr);
  if (need > (size_t)SSA_ATTN_BWD_STATIC_SCRATCH_BYTES)
    return fail(SSA_ERR_WORKSPACE,
                "ssa_attn_bwd_noalloc: this problem needs %zu bytes of scratch but the static scratch "
                "holds %zu (B*H*N*Kn = %lld edges); call ssa_attn_bwd with a caller workspace instead",
                need, (size_t)SSA_ATTN_BWD_STATIC_SCRATCH_BYTES, (long long)E);
  void* scratch = nullptr;
  if ((rc = scratch_address(&scratch))) return rc;
  ssa::attn_bwd_workspace_layout(a, &a, scratch);
  a.q = q; a.k = k; a.v = v; a.nb = nb; a.valid = valid; a.dO = dO; a.lse_in = lse;
  a.dq = dq; a.dk = dk; a.dv = dv;
  cudaError_t e = ssa::launch_attn_bwd(a, true, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "attention backward launch (static scratch)");
  return SSA_OK;
}

}  // extern "C"
