/*
 * ssa_b200.h -- C ABI of the B200 (sm_100a) sparse-attention hot path.
 *
 * A drop-in for the hot path of daedalus/SSA's `sparse_attention.py`: the
 * LSH neighbor-graph build (hash, bucket, multi-probe, rescore + top-k,
 * window/global/self merge) and gather attention, forward and backward.
 *
 * Conventions
 *   - Every pointer argument is DEVICE memory unless stated otherwise; the
 *     caller owns every buffer (including the workspace). No entry point
 *     allocates memory or synchronises the stream.
 *   - `stream` is a cudaStream_t passed as void*. Work is enqueued on it.
 *   - Tensors are described by a base pointer and element strides; the last
 *     (head-dim) axis must be contiguous. Query-side tensors are (B, H, N, d);
 *     key/value tensors are (B, n_kv, M, d) and head h reads kv head
 *     h / (H / n_kv) -- the reference materialises that mapping with
 *     repeat_interleave (sparse_attention.py:1305-1315); here it is an index.
 *   - dtype: SSA_F32 or SSA_BF16 for q/k/v/out. Index outputs are int32.
 *   - Every function returns an ssa_status; 0 is success.
 */
#ifndef SSA_B200_H_
#define SSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SSA_API __attribute__((visibility("default")))
#else
#define SSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SSA_OK = 0,
  SSA_ERR_INVALID = 1,      /* bad shape, stride, pointer or parameter */
  SSA_ERR_UNSUPPORTED = 2,  /* valid for the reference, not built here (message says why) */
  SSA_ERR_WORKSPACE = 3,    /* workspace missing or too small */
  SSA_ERR_CUDA = 4,         /* a CUDA launch or API call failed */
  SSA_ERR_DEVICE = 5        /* a kernel raised its device error flag */
} ssa_status;

typedef enum { SSA_F32 = 0, SSA_BF16 = 1 } ssa_dtype;

/* Geometry and hyper-parameters of one graph build. The derived values
 * (C, p_eff, A) are passed in so the caller controls them exactly as the
 * reference derives them: C = 4 * lsh_k (:1294), p_eff =
 * clamp(round(log2(M / C)), 1, max_num_hashes) (:552-557), A = min(lsh_k,
 * R * C * (1 + min(T, p_eff))) (:898). */
typedef struct {
  int32_t B, H, n_kv, N, M, d;
  int32_t dtype;            /* ssa_dtype of q and k */
  int32_t R;                /* num_hash_rounds */
  int32_t max_p;            /* max_num_hashes: planes per round in rand_proj */
  int32_t p_eff;            /* planes used this call (1..12) */
  int32_t C;                /* candidates kept per bucket (lsh_candidates) */
  int32_t T;                /* lsh_num_probes (clamped to p_eff inside) */
  int32_t A;                /* LSH output width (top-k) */
  int32_t causal;           /* 1: causal LSH + window */
  int32_t is_cross;         /* 1: cross-attention (no window, no self slot) */
  int32_t K;                /* num_neighbors */
  int32_t window;           /* window_size (half width) */
  int32_t G;                /* number of global key indices */
  int64_t q_sb, q_sh, q_sn; /* element strides of q (B, H, N, d) */
  int64_t k_sb, k_sh, k_sm; /* element strides of k (B, n_kv, M, d) */
  int32_t q_row0;           /* sequence position of query row 0 (0 unless the
                             * queries are a slice of a longer sequence, e.g.
                             * one rank's rows under query-row sharding): row i
                             * is position q_row0 + i for the causal limit,
                             * the window and the self slot */
  int32_t reserved0;
} ssa_graph_params;

/* Neighbor-slot width of the merged graph: self + min(K-1, Kall) slots for
 * self-attention, min(K, Kall) for cross-attention, Kall = window slots +
 * G + A (merge_neighbors, sparse_attention.py:1071-1076). */
SSA_API int32_t ssa_graph_width(const ssa_graph_params* p);

/*
 * Fused QKV projection + LSH hash (the projections feeding the graph build,
 * sparse_attention.py:1484-1486, and _hash of their q / k, :588-597):
 *   qkv_out (B*N, (H + 2 n_kv) d) bf16 = x (B*N, d_model) bf16 times w_qkv^T,
 *   w_qkv = [Wq; Wk; Wv] ((H + 2 n_kv) d, d_model) bf16 (nn.Linear weights
 *   stacked), fp32 accumulation; and, from the bf16 q / k values, the graph
 *   build's hash state (key bucket ids and member masks, query bucket ids)
 *   written into `workspace`. Then ssa_build_graph_prehashed with the same
 *   params and workspace finishes the graph; the result equals
 *   ssa_build_graph on q / k views of qkv_out.
 * p describes the self-attention graph (M == N, bf16) with q / k strides of
 * those views: q_sb = k_sb = N (H + 2 n_kv) d, q_sh = k_sh = d,
 * q_sn = k_sm = (H + 2 n_kv) d (k starts at column H d of qkv_out).
 * ssa_qkv_proj_hash_supported returns 1 when this path serves p and d_model
 * (head dim 64 / 128, N % 128 == 0, d_model % 64 == 0, (H + 2 n_kv) d % 128
 * == 0, the tensor-core graph path), else 0.
 */
SSA_API int32_t ssa_qkv_proj_hash_supported(const ssa_graph_params* p, int32_t d_model);
SSA_API int ssa_qkv_proj_hash(const ssa_graph_params* p, int32_t d_model, const void* x, const void* w_qkv,
                              void* qkv_out, const float* rand_proj, void* workspace, size_t workspace_bytes,
                              void* stream);
SSA_API int ssa_build_graph_prehashed(const ssa_graph_params* p, const void* q, const void* k,
                                      const float* rand_proj, const int32_t* glob, int32_t* nb_out,
                                      uint8_t* valid_out, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of device workspace ssa_build_graph / ssa_lsh_select need. */
SSA_API size_t ssa_graph_workspace_size(const ssa_graph_params* p);

/*
 * SparseAttention.build_graph (sparse_attention.py:1325-1390): window +
 * global + LSH + self graph, merged and deduplicated.
 *   q          (B,H,N,d) per q_s* strides;  k (B,n_kv,M,d) per k_s* strides
 *   rand_proj  (R, max_p, d) fp32 contiguous: the LSHGraphBuilder hyperplanes
 *   glob       (G,) int32: global key indices, already clamped to [0, M-1]
 *   nb_out     (B,H,N,W) int32, valid_out (B,H,N,W) uint8, W = ssa_graph_width
 *   lsh_out    optional (B,H,N,A) int32: the LSH selection (any order)
 */
SSA_API int ssa_build_graph(const ssa_graph_params* p, const void* q, const void* k,
                    const float* rand_proj, const int32_t* glob, int32_t* nb_out,
                    uint8_t* valid_out, int32_t* lsh_out, void* workspace,
                    size_t workspace_bytes, void* stream);

/*
 * LSHGraphBuilder.forward (sparse_attention.py:814-959): per (b, h, query)
 * the top-A distinct candidate keys by q.k over the union of R rounds x
 * (1 + probes) buckets, with the reference's overflow, causal, empty-bucket
 * and fallback rules. lsh_out (B,H,N,A) int32 in descending score order,
 * fallback slots last (the reference's topk order).
 */
SSA_API int ssa_lsh_select(const ssa_graph_params* p, const void* q, const void* k,
                   const float* rand_proj, const int32_t* glob, int32_t* lsh_out,
                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * merge_neighbors (sparse_attention.py:966-1089) over explicit sources:
 *   lsh      (B,H,N,A) int32    win (N,Kw) int32 (Kw may be 0)
 *   glob     (G,) int32         self_idx (B,H,N) int32, NULL for cross-attention
 *   true_max device int32 scalar: the maximum over win, glob and lsh (the
 *            reference's true_max_idx, :1031)
 * Output (B,H,N,W): W = min(K-1, Kw+G+A) + 1 with self, min(K, Kw+G+A)
 * without. Uses p->B, H, N, A, K, G.
 */
SSA_API int ssa_merge(const ssa_graph_params* p, const int32_t* lsh, const int32_t* glob,
                      const int32_t* win, int32_t Kw, const int32_t* self_idx,
                      const int32_t* true_max, int32_t* nb_out, uint8_t* valid_out,
                      void* stream);

/*
 * Per-round bucket ids, sign(x . plane_j) packed LSB-first: the reference's
 * _hash (sparse_attention.py:559-591). x (B, heads, rows, d) with strides;
 * ids_out (B*heads, R, rows) int32.
 */
SSA_API int ssa_hash_ids(const void* x, int32_t dtype, int32_t B, int32_t heads, int32_t rows,
                 int32_t d, int64_t sb, int64_t sh, int64_t sn, const float* rand_proj,
                 int32_t R, int32_t max_p, int32_t p_eff, int32_t* ids_out, void* stream);

/* Geometry of gather attention. */
typedef struct {
  int32_t B, H, n_kv, N, M, d;
  int32_t Kn;               /* neighbor slots per query */
  int32_t dtype;            /* ssa_dtype of q, k, v, out (and dO, dq, dk, dv) */
  int32_t nb_i64;           /* 1: neighbors are int64 (reference dtype), else int32 */
  int32_t fp32_weights;     /* SSAConfig.fp32_attn_weights */
  float scale;              /* d ** -0.5 (sparse_attention.py:1249) */
  int64_t q_sb, q_sh, q_sn; /* (B,H,N,d) */
  int64_t k_sb, k_sh, k_sm; /* (B,n_kv,M,d) */
  int64_t v_sb, v_sh, v_sm; /* (B,n_kv,M,d) */
  int64_t o_sb, o_sh, o_sn; /* out / dO / dq (B,H,N,d) */
  /* Attention-weight dropout (F.dropout after the weights' cast,
   * sparse_attention.py:1193-1194): each weight is zeroed with probability
   * dropout_p, the kept ones scaled by 1 / (1 - dropout_p). 0 disables it.
   * The keep decision of slot j of row r (row = (b*H + h)*N + n) comes from
   * Philox4x32-10 keyed by dropout_seed, counter (e / 4, e >> 34,
   * dropout_offset), e = r * Kn + j, output word e % 4: kept iff that word is
   * >= dropout_p * 2^32. Forward and backward must get the same values. */
  float dropout_p;
  int32_t reserved0;
  uint64_t dropout_seed;
  uint64_t dropout_offset;
} ssa_attn_params;

/*
 * sparse_gather_attention forward (sparse_attention.py:1096-1199) as called
 * by SparseAttention.apply_graph (:1392-1418): fp32 scores q.k * scale over
 * the Kn gathered keys, invalid slots masked, fp32 softmax, weights cast to
 * the value dtype (or kept fp32 with fp32_weights), weighted sum of values.
 *   nb (B,H,N,Kn) int32/int64 contiguous, valid (B,H,N,Kn) uint8/bool
 *   out (B,H,N,d) per o_s* strides; lse (B,H,N) fp32, optional (backward)
 */
SSA_API int ssa_attn_fwd(const ssa_attn_params* p, const void* q, const void* k, const void* v,
                 const void* nb, const uint8_t* valid, void* out, float* lse,
                 void* stream);

/*
 * Backward of ssa_attn_fwd (the autograd graph of :1147-1198): dq, and dk/dv
 * accumulated per kv head over every (head, query, slot) edge that gathered
 * that key -- the index_add / repeat_interleave backward -- as a segmented
 * reduction over the inverted neighbor index (no floating-point atomics; the
 * result is deterministic). dO/dq share the o_s* strides; dk/dv are
 * (B,n_kv,M,d) contiguous. Needs ssa_attn_bwd_workspace_size bytes.
 */
SSA_API size_t ssa_attn_bwd_workspace_size(const ssa_attn_params* p);
SSA_API int ssa_attn_bwd(const ssa_attn_params* p, const void* q, const void* k, const void* v,
                 const void* nb, const uint8_t* valid, const void* dO, const float* lse,
                 void* dq, void* dk, void* dv, void* workspace, size_t workspace_bytes,
                 void* stream);

/*
 * The inverted neighbor index of a graph (nb, valid) -- every kv head's keys
 * with the edges (b, h, n, slot) that gathered them, in edge order -- built
 * once and reused by ssa_attn_bwd_csr for every layer that applies the same
 * graph: the reference's CachedGraphSparseTransformer shares one graph over
 * `reuse_every` layers (sparse_attention.py:1741-1792), and ssa_attn_bwd
 * otherwise rebuilds this index in each layer's backward (the scatter of
 * index_select's backward, :1149-1150). The index depends only on B, H,
 * n_kv, N, M, Kn, nb_i64 and the graph. ssa_attn_csr_size gives its bytes;
 * building needs a workspace of ssa_attn_bwd_workspace_size bytes.
 * ssa_attn_bwd_csr is ssa_attn_bwd with the index given (same workspace
 * size; the index is only read).
 */
SSA_API size_t ssa_attn_csr_size(const ssa_attn_params* p);
SSA_API int ssa_attn_build_csr(const ssa_attn_params* p, const void* nb, const uint8_t* valid, void* csr,
                               size_t csr_bytes, void* workspace, size_t workspace_bytes, void* stream);
SSA_API int ssa_attn_bwd_csr(const ssa_attn_params* p, const void* q, const void* k, const void* v,
                             const void* nb, const uint8_t* valid, const void* dO, const float* lse,
                             void* dq, void* dk, void* dv, const void* csr, size_t csr_bytes,
                             void* workspace, size_t workspace_bytes, void* stream);

/*
 * ssa_attn_bwd without a workspace argument -- no counterpart in the
 * reference, which allocates through PyTorch. For callers that cannot
 * allocate device memory: a host binding that only receives device buffers
 * from elsewhere and has no device allocator of its own, or a process whose
 * device memory footprint is fixed after set-up. The scratch is a file-scope
 * device array of SSA_ATTN_BWD_STATIC_SCRATCH_BYTES (64 MiB) per device, so
 * the call allocates nothing; problems whose scratch
 * (ssa_attn_bwd_workspace_size) exceeds it are rejected with
 * SSA_ERR_WORKSPACE. That is about 26 bytes per edge (B*H*N*Kn) at head dim
 * 64, 28 at 128 and 32 at 256 while M < 65536 (8 more when M >= 65536: one
 * more sort pass), so at most about 2.5, 2.3 and 2.0 million edges
 * (1.9, 1.8 and 1.6 million for M >= 65536).
 *   - The first call on each device resolves the array's address with
 *     cudaGetSymbolAddress and keeps it for the life of the process; make
 *     that first call before any stream capture, and do not use this entry
 *     point across a device reset (cudaDeviceReset or a new primary context
 *     would leave the kept address stale).
 *   - Nothing in the scratch has to start at zero.
 *   - Calls share the device's one array: two calls whose executions overlap
 *     (other streams, or host threads without ordering between them) race on
 *     it and corrupt each other's results. Serialise them on one stream.
 * Arguments and results are those of ssa_attn_bwd.
 */
#define SSA_ATTN_BWD_STATIC_SCRATCH_BYTES (64u << 20)
SSA_API int ssa_attn_bwd_noalloc(const ssa_attn_params* p, const void* q, const void* k,
                                 const void* v, const void* nb, const uint8_t* valid,
                                 const void* dO, const float* lse, void* dq, void* dk, void* dv,
                                 void* stream);

/*
 * neighbor_overlap (sparse_attention.py:1583-1615): per row, the Jaccard
 * similarity of two neighbor sets -- the number of valid A slots whose index
 * is among the valid B slots, over |valid A| + |valid B| minus that number
 * (at least 1). nb_a, nb_b (rows, K) int32 (nb_i64 = 0) or int64; valid_a,
 * valid_b (rows, K) uint8/bool; out (rows,) fp32. K <= 2048.
 */
SSA_API int ssa_neighbor_overlap(const void* nb_a, const uint8_t* valid_a, const void* nb_b,
                                 const uint8_t* valid_b, int64_t rows, int32_t K, int32_t nb_i64,
                                 float* out, void* stream);

/* Error code recorded by a kernel whose bounded wait on an on-chip barrier
 * ran out (0 = none); synchronises with the device. clear != 0 resets it. */
SSA_API int32_t ssa_device_error(int32_t clear);

/* Testing aid for that failure path (no counterpart in the reference): the
 * tensor-core candidate scan's waits on its on-chip barriers give up after
 * `polls` polls instead of 2^24 (0 restores the default), so a test can make
 * a wait run out without faulting or hanging the GPU. The kernel then stops
 * its pipeline, waits for its own copies and MMAs in flight, frees its TMEM
 * and returns; ssa_device_error reports the code and that build's output is
 * undefined. Process-wide; read when each build is launched. */
SSA_API int ssa_debug_set_wait_limit(uint32_t polls);

/* Testing aids for the tensor-core hash (no counterpart in the reference;
 * the hash ids are the same either way). Process-wide; read when each build
 * is launched.
 *   ssa_debug_set_hash: use_tc = 0 hashes keys and queries with the fp32 FMA
 *     kernels only; else bf16 inputs with head dim 64 or 128 hash on the
 *     tensor cores (the default). eps_c is the constant c of the bound
 *     eps = c * |x|_2 * max_j |P[r][j]|_2 under which a projection is
 *     recomputed in fp32 (0: the default 2^-14; larger values recompute
 *     more, up to every projection).
 *   ssa_debug_hash_dump: while buf (device, n_floats fp32) is set and holds
 *     B*H*N*R*p_eff floats, each build writes the tensor-core projection of
 *     query row i, round r, plane j to buf[(i * R + r) * p_eff + j]
 *     (rows not hashed on the tensor cores are left as they are). NULL: off.
 *   ssa_debug_hash_recomputed: (row, round) items recomputed in fp32 since
 *     the last clear (synchronises with the device); -1 on error. */
SSA_API int ssa_debug_set_hash(int32_t use_tc, float eps_c);
SSA_API int ssa_debug_hash_dump(float* buf, int64_t n_floats);
SSA_API int64_t ssa_debug_hash_recomputed(int32_t clear);

/* Human-readable text for the last error on this host thread. */
SSA_API const char* ssa_last_error(void);

/* Number of kernel launches this library has issued in this process (a
 * host-side count; library calls such as the CUB sort inside ssa_attn_bwd
 * are not included). */
SSA_API int64_t ssa_kernel_launches(void);

/*
 * Stage timing of the graph build, for profiling (no counterpart in the
 * reference). ssa_graph_profile(1) makes every later ssa_build_graph /
 * ssa_lsh_select call record CUDA events on its stream at the boundaries of
 * its kernel stages; ssa_graph_profile(0) turns that off. Events are created
 * on the current device when profiling is turned on.
 * ssa_graph_stage_times waits for the most recent profiled call to finish and
 * writes the duration in ms of each of its SSA_GRAPH_STAGES stages, in this
 * order: key hashing, bucket trim, query hashing, sample scan, threshold
 * rows, full scan, final rows, FMA scan (exact fallback, or the whole
 * selection for fp32). A stage the call's path does not run reads 0. The
 * profiling state is process-wide: profile one call at a time.
 */
#define SSA_GRAPH_STAGES 8
SSA_API int ssa_graph_profile(int32_t enable);
SSA_API int ssa_graph_stage_times(float* ms_out);

/* ABI version of this library (major * 100 + minor). */
SSA_API int32_t ssa_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* SSA_B200_H_ */
