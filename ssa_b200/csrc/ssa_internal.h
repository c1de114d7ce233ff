// ssa_internal.h -- device-side parameter blocks and launchers shared by the
// kernel files and the C ABI (ssa_capi.cu). Not part of the public ABI.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace ssa {


// Everything a graph-build kernel needs, passed by value.
struct GraphDev {
  int B, H, n_kv, rep, N, M, d, dtype;
  int R, max_p, p, C, Te, NT, NB, W, Wpad, A;
  int causal, is_cross, window, G, Wout;
  int row0;  // sequence position of query row 0 (query-row sharding)
  uint32_t wait_limit;  // polls before a tensor-core scan wait gives up (ssa_debug_set_wait_limit)
  int64_t q_sb, q_sh, q_sn, k_sb, k_sh, k_sm;
  const void* q;
  const void* k;
  const float* rp;        // (R, max_p, d)
  const int32_t* glob;    // (G,)
  // workspace
  void* ws;
  size_t zero_off, zero_bytes;
  uint16_t* kcode;                // [BG][R][M] bucket id of every key
  unsigned long long* bmap;       // [BG][Wpad/2][R][NB][2] first-C member masks (bmap_idx)
  unsigned long long* pmask;      // [BG][W] pad keys perm_r[M-1]
  uint32_t* pmax;                 // [BG][R] (bucket << 20 | key) of perm_r[M-1]
  int32_t* bsize;                 // [BG][R][NB]
  int32_t* lastc;                 // [BG][R][NB] key at rank min(size, C) - 1
  // tensor-core path (bf16): per query row
  int use_tc, capg, sample_s, fallback_only;
  uint16_t* qids;                 // [NT][B*H*N] r * NB + bucket id per (round r, probe) slot
  uint8_t* qempty;                // [B*H*N] some slot's bucket is empty
  float* tau;                     // [B*H*N] scan threshold
  int32_t* rcnt;                  // [B*H*N][2] kept candidates per scan group (> capg/2: overflow)
  float* sspec;                   // [B*H*N][R + 1] full-scan scores of the round-r pad key
                                  // (r < R) and of causal self (R) -- keys the scan skips
  unsigned long long* buf;        // [B*H*N][capg] kept (key << 32 | score bits); in the
                                  // sample pass kSampleTileBytes records per sampled tile
  uint8_t* tile_flags;            // [B*H][ceil(N/128)] tiles for the exact fallback
  uint16_t* qpc;                  // fp32 tensor-core scan: q as bf16 pieces [3*B][H][N][d]
  uint16_t* kpc;                  //                        k as bf16 pieces [3*B][n_kv][M][d]
  // tensor-core hash (bf16, head dim 64 / 128): keys always, queries with the
  // tensor-core scan
  int use_tc_hash;
  float hash_eps;                 // c of the certification bound eps = c |x|_2 max_j |P[r][j]|_2
  uint16_t* hpl;                  // hyperplane pieces in the B-operand layout (k_hash_planes)
  float* pnorm;                   // [R][p] |P[r][j]|_2, rounded up
  float* hash_dump;               // testing: tensor-core query projections [B*H*N][R][p], or null
  int prehashed;                  // the hash state is already in the workspace (ssa_qkv_proj_hash)
  unsigned int* hq_count;         // [2] fused projection: flagged items queued, keys / queries
  uint32_t* hq_keys;              // flagged (bg * M + key) << 4 | round (per-CTA segments in k_hash_tc)
  uint32_t* hq_rows;              // flagged query row << 4 | round
  // outputs
  int32_t* lsh;                   // [B][H][N][A]
  int32_t* nb;                    // [B][H][N][Wout]
  uint8_t* valid;                 // [B][H][N][Wout]
};

// Sample-pass record per sampled key tile in a row's buffer: 128 upper
// score halves (256 bytes) and the tile's 128-bit candidate mask.
constexpr int kSampleTileBytes = 272;

// The hashing kernels stage the R * p hyperplanes in shared memory when they
// take at most this many bytes, and read them through L1 otherwise.
constexpr size_t kHashPlaneSmemMax = 64 * 1024;
// Rows each group of four lanes hashes at once (a row is split over the
// four): every hyperplane element loaded serves that many rows. The
// registers of D / 4 floats per row set the count.
template <int D>
constexpr int kHashRows = D <= 64 ? 4 : 2;

// Index of the member mask of 64-key word w, round r, bucket u. The two words
// of a 128-key tile are adjacent, so one tile's masks for all (round, bucket)
// pairs form one contiguous block of R * NB * 16 bytes.
__host__ __device__ inline int64_t bmap_idx(const GraphDev& g, int bg, int w, int r, int u) {
  return ((((int64_t)bg * (g.Wpad >> 1) + (w >> 1)) * g.R + r) * g.NB + u) * 2 + (w & 1);
}

// Host-side count of kernel launches made by this library (ssa_kernel_launches).
void note_launch();

// Stage boundaries of a graph build (ssa_graph_profile / ssa_graph_stage_times):
// stage i runs between marks i and i + 1.
enum GraphStageMark {
  kStageBegin = 0,
  kStageHashKeys = 1,
  kStageBucketTrim = 2,
  kStageHashQueries = 3,
  kStageScanSample = 4,
  kStageRowsThresh = 5,
  kStageScanFull = 6,
  kStageRowsFinal = 7,
  kStageSelectFma = 8,
  kStageMarks = 9
};
// Records the profiling event of mark i on st while profiling is on.
void stage_mark(int i, cudaStream_t st);

// Fills the workspace pointers of g (g->ws may be null to only size it) and
// returns the bytes needed. Decides g->use_tc from the shapes.
size_t graph_workspace_layout(GraphDev* g);
int choose_select_rows(const GraphDev& g, int* rows_out, size_t* smem_out);
cudaError_t launch_graph(const GraphDev& g, int mode, cudaStream_t st);
bool select_tc_supported(const GraphDev& g);
bool select_tc_pointers_ok(const GraphDev& g);
cudaError_t launch_select_tc(const GraphDev& g, int mode, cudaStream_t st);
cudaError_t launch_hash_queries(const GraphDev& g, cudaStream_t st);
bool hash_tc_supported(const GraphDev& g);
size_t hash_tc_planes_bytes(const GraphDev& g);
cudaError_t launch_hash_planes(const GraphDev& g, cudaStream_t st);
cudaError_t launch_hash_tc(const GraphDev& g, bool keys, cudaStream_t st);
int read_hash_tc_error(int clear);
// Fused QKV projection + hash (self-attention, bf16): out[rows][n_out] =
// x[rows][dm] w[n_out][dm]^T, with the graph's hash state written into its
// workspace (g.q / g.k are views of out).
struct ProjDev {
  int rows, dm, n_out;
  const void* x;
  const void* w;
  void* out;
};
bool proj_hash_supported(const GraphDev& g, int dm);
cudaError_t launch_proj_hash(const GraphDev& g, const ProjDev& pd, cudaStream_t st);
cudaError_t launch_qempty(const GraphDev& g, cudaStream_t st);
unsigned long long read_hash_recomputed(int clear);
cudaError_t launch_rows(const GraphDev& g, int stage, int mode, cudaStream_t st);
size_t rows_smem_bytes(const GraphDev& g, int warps);
int read_device_error(int clear);
cudaError_t launch_neighbor_overlap(const void* nb_a, const uint8_t* va, const void* nb_b, const uint8_t* vb,
                                    int64_t rows, int K, int nb_i64, float* out, cudaStream_t st);
struct MergeDev {
  int B, H, N, A, Kw, G, Wout;
  const int32_t* lsh;       // [B][H][N][A]
  const int32_t* glob;      // [G]
  const int32_t* win;       // [N][Kw]
  const int32_t* self_idx;  // [B][H][N] or null (cross-attention)
  const int32_t* true_max;  // device scalar
  int32_t* nb;              // [B][H][N][Wout]
  uint8_t* valid;
};
cudaError_t launch_merge(const MergeDev& m, cudaStream_t st);
cudaError_t launch_hash_ids(const void* x, int dtype, int B, int heads, int rows, int d,
                            int64_t sb, int64_t sh, int64_t sn, const float* rp, int R,
                            int max_p, int p, int32_t* out, cudaStream_t st);

struct AttnDev {
  int B, H, n_kv, rep, N, M, d, Kn, dtype, nb_i64, fp32w;
  float scale;
  // attention-weight dropout: drop_thresh = dropout_p * 2^32 (0: off)
  uint32_t drop_thresh;
  float drop_scale;   // 1 / (1 - dropout_p)
  unsigned long long drop_seed, drop_offset;
  int64_t q_sb, q_sh, q_sn, k_sb, k_sh, k_sm, v_sb, v_sh, v_sm, o_sb, o_sh, o_sn;
  const void* q;
  const void* k;
  const void* v;
  const void* nb;
  const uint8_t* valid;
  void* out;
  float* lse;
  // backward
  const void* dO;
  const float* lse_in;
  void* dq;
  void* dk;
  void* dv;
  float* ep;          // [rows][Kn] value weight per edge
  float* eds;         // [rows][Kn] scale * dS per edge
  // inverted neighbor index (valid edges only, sorted by (kv slice, key))
  uint32_t* skey;     // bg * M + key of each sorted edge
  uint32_t* sid;      // edge id (row * Kn + slot) of each sorted edge
  uint32_t* seg;      // [B*n_kv*M + 1] first sorted position of each key; [B*n_kv*M] = valid edges
  // edge-sort temporaries
  uint32_t* tk0;      // [rows * Kn] keys / ids between passes (ping-pong)
  uint32_t* ti0;
  uint32_t* tk1;
  uint32_t* ti1;
  uint32_t* cnt;      // [B*n_kv][256][tiles] digit counts, then offsets
  uint32_t* tot;      // [B*n_kv] edges per slice in a pass
  uint32_t* sbase;    // [B*n_kv + 1] output offset of each slice in the last pass
  float* part;        // [chunks][2][2][d] partial dk / dv of keys that cross a chunk edge
};

cudaError_t launch_attn_fwd(const AttnDev& a, cudaStream_t st);
// Workspace of the backward (per-edge arrays, sort temporaries, partials and
// an inverted index of its own); bytes of a caller-held inverted index.
size_t attn_bwd_workspace_layout(const AttnDev& a, AttnDev* out, void* ws);
size_t attn_csr_layout(const AttnDev& a, AttnDev* out, void* csr);
cudaError_t launch_build_csr(const AttnDev& a, cudaStream_t st);
// build_csr: sort the edges first (else a.skey / sid / seg hold a built index).
cudaError_t launch_attn_bwd(const AttnDev& a, bool build_csr, cudaStream_t st);

}  // namespace ssa
