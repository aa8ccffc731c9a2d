/*
 * dforktree_b200 -- C ABI of the B200 (sm_100a) draft-tree cycle.
 *
 * Drop-in boundary for the DForkTree plugin's hot path (Perseus037/DForkTree,
 * `dforktree/`): score -> build -> GDN tree verify -> closed-form commit.
 * Every entry point takes plain device pointers, sizes and element strides,
 * launches on the given CUDA stream (`stream` is a cudaStream_t passed as
 * void*; NULL = legacy default stream), never synchronises the host and never
 * allocates, except dft_table_create.  All calls are batched over requests
 * (the reference is batch-1 only: fc1_branch64.py:13, fc1_fused.py:69) and are
 * CUDA-graph capturable.
 *
 * Return value: DFT_OK (0) or a DFT_ERR_* code for invalid arguments / CUDA
 * errors, checked on the host before launch.  Errors found by a kernel are
 * OR-ed into the optional device word `dev_status` (DFT_DEV_* bits).
 */
#ifndef DFORKTREE_B200_H
#define DFORKTREE_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define DFT_API __attribute__((visibility("default")))
#else
#define DFT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status -- */
enum {
  DFT_OK = 0,
  DFT_ERR_INVALID = 1,      /* null pointer, bad size or stride            */
  DFT_ERR_UNSUPPORTED = 2,  /* shape outside what the kernels implement    */
  DFT_ERR_CUDA = 3,         /* CUDA runtime error (launch, allocation)     */
  DFT_ERR_TABLE = 4,        /* n-gram keys unsorted, negative or too many  */
  DFT_ERR_NO_DEVICE = 5,    /* no sm_100 device current                    */
  DFT_ERR_CAPACITY = 6,     /* larger than a fixed-size static scratch     */
  DFT_ERR_IO = 7            /* table file missing, unwritable or damaged    */
};
enum {
  DFT_DEV_BAD_TOKEN = 1,    /* token id outside [-V, V)                    */
  DFT_DEV_PROBE_LIMIT = 2,  /* hash probe ran over the whole table         */
  DFT_DEV_BAD_INDEX = 4,    /* node / conv column / slot index out of range */
  DFT_DEV_TIMEOUT = 8       /* a bounded wait gave up                      */
};
typedef enum { DFT_F32 = 0, DFT_BF16 = 1, DFT_F16 = 2 } dft_dtype;

DFT_API const char* dft_status_string(int status);
DFT_API int dft_version(void);

/* ------------------------------------------------------- n-gram table -- */
/* Replaces NGramGPU.__init__ (ngram_gpu.py:8-26): the sorted-array npz table
 * becomes open-addressed hash tables in HBM with 16-byte slots:
 *   pair slot  {key u*V+v, bigram count n_uv, trigram-context count n3c(u,v)}
 *   triple slot{key (a*V+b)*V+c, count c3, rank of the key in keys3}
 *   quad slot  {key rank3*V+c, count c4}
 * so one 128-bit load answers one probe.  All arrays are device pointers;
 * the table copies what it keeps.  keys* must be strictly ascending and >= 0
 * (duplicates: the first occurrence wins, like searchsorted).              */
typedef struct dft_table dft_table;
typedef struct {
  int64_t V;
  const int64_t* keys;  const float* cab;  int64_t n_bigram;   /* 'keys','cab'   */
  const float* prev;                       /* [V] 'prev'                      */
  const float* pn;                         /* [V] fp32((nxt+1)/(N+V)), :16    */
  const int64_t* keys3; const float* c3;   int64_t n_trigram;  /* optional    */
  const int64_t* keys3c; const float* n3c; int64_t n_ctx3;     /* optional    */
  const int64_t* keys4; const float* c4;   int64_t n_quad;     /* optional    */
  const float* n4c;                        /* [n_trigram] when keys4 given    */
  float beta2, beta3, beta4, clip;         /* ngram_gpu.py:8 (Builder: beta3=60) */
  float max_load;                          /* slots per key bound; 0 -> 0.35  */
} dft_table_desc;

DFT_API int dft_table_create(const dft_table_desc* desc, dft_table** out, void* stream);
DFT_API int dft_table_destroy(dft_table* table);
/* capacities (slots) and total device bytes of the three hash tables */
DFT_API int dft_table_info(const dft_table* table, int64_t* V, int64_t* pair_slots, int64_t* trip_slots,
                   int64_t* quad_slots, int64_t* bytes);

/* Smoothing parameters of a table (e.g. after dft_table_load). */
DFT_API int dft_table_set_params(dft_table* table, float beta2, float beta3, float beta4, float clip);
/* Copy the table's prev[V] and pn[V] (fp32) to prev / pn (device or host;
 * either may be NULL), stream-ordered. */
DFT_API int dft_table_copy_marginals(const dft_table* table, float* prev, float* pn, void* stream);

/* Cached binary table.  dft_table_save writes the built hash tables (slot
 * images, prev, pn, n4c, parameters) to `path` (via a temporary file renamed
 * into place); dft_table_load maps such a file back onto the current device
 * with sequential reads and host-to-device copies -- no npz parse, no key
 * sort, no hash insert -- and the loaded slots are byte-identical to the
 * saved ones.  A missing, truncated, foreign or damaged file (64-bit checksum
 * over the payload) returns DFT_ERR_IO.  Both synchronise `stream`.
 * Replaces re-reading ngram_counts.npz in NGramGPU.__init__ (ngram_gpu.py:9). */
DFT_API int dft_table_save(const dft_table* table, const char* path, void* stream);
DFT_API int dft_table_load(const char* path, dft_table** out, void* stream);

/* Elementwise p_order / PMI over flattened, pre-broadcast id arrays.
 * Replaces NGramGPU.p2/p3/p4/pmi (ngram_gpu.py:39-70).  what: 0 = p, 1 = pmi.
 * Unused ids may be NULL (z for order<4, a for order 2). */
DFT_API int dft_ngram_eval(const dft_table* table, int order, int what, const int64_t* z, const int64_t* a,
                   const int64_t* b, const int64_t* c, int64_t n, float* out, int32_t* dev_status,
                   void* stream);

/* ------------------------------------------------------ score + build -- */
typedef struct {
  int32_t B;            /* requests                                          */
  int32_t S;            /* drafter positions (block - 1)                     */
  int32_t V;            /* vocabulary                                        */
  int32_t M;            /* candidates per position; 16 (fc1_builder.py:27)   */
  int32_t N;            /* tree nodes incl. root (FC1_TREE_N), 2..64         */
  int32_t lmax;         /* beam level cap, 99 (fc1_builder.py:37)            */
  int32_t chain_first;  /* FC1_CHAIN_FIRST (BIG = 1e4 bonus, tree_ops.py:13) */
  int32_t use_ngram;    /* 1: fork-aware PMI closure; 0: plain renormalised  */
  float lam_a, lam_p;   /* 0.3, 0.6 (fc1_builder.py:31)                      */
  int32_t pmi_order;    /* n-gram order of the closure: 2, 3 or 4 (the second
                           argument of ngram_path_fn, tree_ops.py:55); 0 = 3,
                           the Builder's (fc1_builder.py:31)                  */
} dft_build_params;

typedef struct {
  /* Builder.__call__ outputs (fc1_builder.py:49-54), all [B, ...]          */
  int64_t* tokens;      /* [B, N]    root then ids[ss, cand]                 */
  int64_t* parent;      /* [B, N]    -1 for the root                         */
  int64_t* depth;       /* [B, N]                                            */
  float* anc;           /* [B, N, N] 1.0 where column is row or its ancestor */
  int64_t* nxt;         /* [B, N]    first child or -1                       */
  int64_t* sib;         /* [B, N]    next sibling or -1                      */
  int64_t* cidx;        /* [B, N, 4] conv columns (tree_ops.py:79-88)        */
  /* optional (NULL skips); beam_tree returns (tree_ops.py:53)              */
  int64_t* ss;          /* [B, N-1] step (= depth - 1) of node 1..N-1        */
  int64_t* cand;        /* [B, N-1] candidate index of node 1..N-1           */
  uint8_t* flags;       /* [B, N-1] top-1-chain flag                          */
  float* keys;          /* [B, S, W] per-step beam keys                       */
} dft_tree_out;

/* Scoring alone: lp, ids = topk(log_softmax(logits), M); rest (fc1_builder.py:27-28).
 * logits element (b, s, v) at b*ld_b + s*ld_s + v.  ids written as int32.  */
DFT_API int dft_score(const dft_build_params* p, const void* logits, int32_t logits_dtype, int64_t ld_b, int64_t ld_s,
              float* lp, int32_t* ids, float* rest, void* stream);

/* Dense PMI tensor T of ngram_path_fn (tree_ops.py:56-65) over
 * E = [pre1; root; ids], for p->pmi_order (0 = 3):
 *   order 2: T[b, t, j, l]       = PMI2(E[t+2]_j, E[t+3]_l)      [B, S-1, M, M]
 *   order 3: T[b, t, i, j, l]    = PMI3(E[t+1]_i, .., E[t+3]_l)  [B, S-1, M, M, M]
 *   order 4: T[b, t, h, i, j, l] = PMI4(E[t]_h, .., E[t+3]_l)    [B, S-1, M, M, M, M]
 * float.  pre1 is read by order 4 only (NULL there: DFT_ERR_INVALID).       */
DFT_API int dft_pmi_dense(const dft_table* table, const dft_build_params* p, const int32_t* ids, const int64_t* root,
                  const int64_t* pre1, float* T, int32_t* dev_status, void* stream);

/* Beam search + tree structure, one CTA per request.  With use_ngram
 * the closure is the fork-aware PMI re-anchoring over T; otherwise `logc`
 * [B, S-1, M, M] (may be NULL: the no-n-gram branch of fc1_builder.py:35-36
 * is derived from lp/rest).  c0 [B, M] may be NULL (then from lp/rest). */
DFT_API int dft_beam_build(const dft_build_params* p, const float* lp, const int32_t* ids, const float* rest,
                   const float* T, const float* logc, const float* c0, const int64_t* root,
                   dft_tree_out* out, int32_t* dev_status, void* stream);

/* Whole score+build (Builder.run, fc1_builder.py:26-47) in three launches;
 * the PMI and beam launches use programmatic stream serialisation and wait
 * for the preceding kernel before their first read (stream order unchanged).
 * workspace: dft_score_build_workspace_bytes(p) bytes of device memory.    */
DFT_API int64_t dft_score_build_workspace_bytes(const dft_build_params* p);
DFT_API int dft_score_build(const dft_table* table, const dft_build_params* p, const void* logits, int32_t logits_dtype,
                    int64_t ld_b, int64_t ld_s, const int64_t* root, const int64_t* pre1, void* workspace,
                    dft_tree_out* out, int32_t* dev_status, void* stream);

/* Allocation-free score + build.  No counterpart in the reference: it exists
 * for callers that cannot allocate device memory -- a plugin inside a serving
 * engine's decode step, whose HBM belongs to the engine's static pools and to
 * torch's caching allocator (a raw cudaMalloc competes with pools sized to
 * fill the device; cudaFree synchronises it), or a C host that binds only
 * this ABI and has no device allocator.  Same inputs, outputs and kernels as
 * dft_score_build, but the scratch lives in one file-scope device array of
 * dft_score_build_static_capacity() bytes (32 MiB: 64 requests at S = 24),
 * held by every GPU that loads the library until the process exits; larger
 * shapes return DFT_ERR_CAPACITY.  The first call on a device resolves the
 * array's device address (cudaGetSymbolAddress, with that device current);
 * make that first call before any stream capture.  A device reset
 * (cudaDeviceReset) discards the array's contents and its address; the next
 * call sees the new context and resolves the address again, so after a reset
 * make one call outside any capture first.  All calls share the one
 * array: calls whose kernels overlap on the GPU (other streams, other host
 * threads) race.  Each call writes every scratch byte it reads, so nothing
 * carries over between calls.  Allocates nothing. */
DFT_API int64_t dft_score_build_static_capacity(void);
DFT_API int dft_score_build_static(const dft_table* table, const dft_build_params* p, const void* logits,
                                   int32_t logits_dtype, int64_t ld_b, int64_t ld_s, const int64_t* root,
                                   const int64_t* pre1, dft_tree_out* out, int32_t* dev_status, void* stream);

/* Tree structure for a caller-given topology (tree_ops.tree_struct,
 * tree_ops.py:68-89, plus nxt/sib of fc1_builder.py:41-47).  parent [B, N]
 * with parent[b, 0] ignored (root) and parent[b, n] < n.  Any output may be
 * NULL. */
DFT_API int dft_tree_struct(int32_t B, int32_t N, const int64_t* parent, float* anc, int64_t* depth, int64_t* cidx,
                            int64_t* nxt, int64_t* sib, int32_t* dev_status, void* stream);

/* Greedy tree acceptance: the SGLang eagle tree verification the plugin calls
 * through run_eagle_verify (fc1_branch64.py:44-46).  Starting at the root,
 * follow the first child (nxt/sib order) whose token equals target[b, cur].
 * path [B, P] accepted nodes (root first, -1 padded), accept_len [B],
 * last [B] (the next pre1 source, fc1_branch64.py:45-46), bonus [B]
 * (target token at the last node).  Outputs other than path may be NULL. */
DFT_API int dft_accept_greedy(int32_t B, int32_t N, int32_t P, const int64_t* tokens, const int64_t* nxt,
                              const int64_t* sib, const int64_t* target, int64_t* path, int64_t* accept_len,
                              int64_t* last, int64_t* bonus, int32_t* dev_status, void* stream);

/* ---------------------------------------------------------- tree conv -- */
/* Replaces fc1_conv.conv (fc1_conv.py:8-27) batched.  x element (b, n, c) at
 * b*x_sb + n*x_sn + c*x_sc; conv_state (slot, c, tap) at slot*cs_ss + c*cs_sc
 * + tap*cs_st (3 taps); weight [C, 4]; bias [C] or NULL; cidx [B, N, 4];
 * y (b, n, c) at b*y_sb + n*y_sn + c; window (dst, n, c, j) at
 * dst*iw_sd + n*iw_sn + c*iw_sc + j*iw_sj, written when iw != NULL.        */
typedef struct {
  int32_t B, N, C;
  const void* x; int32_t x_dtype; int64_t x_sb, x_sn, x_sc;
  const void* conv_state; int32_t cs_dtype; int64_t cs_ss, cs_sc, cs_st;
  const int64_t* state_slots;     /* [B] (NULL: slot b)                     */
  const void* weight; int32_t w_dtype;
  const void* bias;               /* NULL: no bias; dtype w_dtype           */
  const int64_t* cidx;            /* [B, N, 4]                              */
  void* y; int32_t y_dtype; int64_t y_sb, y_sn;
  void* iw; int32_t iw_dtype; int64_t iw_sd, iw_sn, iw_sc, iw_sj;
  const int64_t* iw_slots;        /* [B] (NULL: dst b)                      */
} dft_conv_args;
DFT_API int dft_tree_conv(const dft_conv_args* a, int32_t* dev_status, void* stream);

/* ------------------------------------------------- conv-window commit -- */
/* After acceptance, request b's conv state becomes the window of its last
 * accepted node u = last[b]: taps 1..3 of u, i.e. the inputs at conv columns
 * cidx[b, u, 1..3] (columns < 3: the old conv state, 3 + m: new token m).
 * This is what the plugin's conv hook writes into intermediate_conv_window
 * (fc1_conv.py:22-27) and SGLang's post-verify commit copies into the conv
 * state (after fc1_fused.py:87).  Batched over layers; in place. */
typedef struct {
  int32_t L, B, N, C;
  const void* x; int32_t x_dtype; int64_t x_sl, x_sb, x_sn;          /* pre-conv (l, b, n, c), c stride 1 */
  void* conv_state; int32_t cs_dtype; int64_t cs_sl, cs_ss, cs_sc, cs_st;   /* (l, slot, c, tap)  */
  const int64_t* slots;           /* [B] conv-state slot of request b; NULL: slot b */
  const int64_t* cidx;            /* [B, N, 4] conv columns                 */
  const int64_t* last;            /* [B] last accepted node; < 0: request unchanged */
} dft_conv_commit_args;
DFT_API int dft_conv_commit(const dft_conv_commit_args* a, int32_t* dev_status, void* stream);

/* ---------------------------------------------------- GDN tree verify -- */
/* Replaces tree_gdn_split (tree_kernels.py:193-208 = _tree_prepare +
 * invert32 + _tree_finish) batched.  Per request b: y (b, n, col) with
 * columns [q (Hk*Dk) | k (Hk*Dk) | v (Hv*Dv)]; a, bg (b, n, h); state pool
 * element (slot, h, v, k) -- V-major like SGLang's ssm pool; o (b, n, h, v).
 * aux (all optional): k_hat (b, head, n, k) for head = v-head (aux_k_per_v=1,
 * the reference's CTX.keys layout) or k-head; vn (b, h, n, v); G (b, h, n).
 * With `conv` set, y is not read: the tree conv of fc1_conv.py:8-27 is
 * computed from the pre-conv inputs inside the verifier (the window taps
 * are not written; dft_tree_conv does that for the drop-in hook).  The fused
 * conv runs on the tensor-core paths only (N <= 32 with Hv / Hk in {1, 2}, or
 * 32 < N <= 64 with any Hv / Hk; Dk = Dv = 128, bfloat16 x, conv state,
 * weights and o, 16-byte aligned rows); others return DFT_ERR_UNSUPPORTED and
 * take dft_tree_conv + this call on y. */
typedef struct {
  const void* x; int32_t x_dtype; int64_t x_sb, x_sn;   /* pre-conv (b, n, col), col stride 1 */
  const void* conv_state; int32_t cs_dtype; int64_t cs_ss, cs_sc, cs_st;
  const int64_t* conv_slots;      /* [B]; NULL: slot b                      */
  const void* weight; int32_t w_dtype;                  /* [C, 4]         */
  const void* bias;               /* [C] or NULL, dtype w_dtype             */
  const int64_t* cidx;            /* [B, N, 4] conv columns                 */
} dft_gdn_conv_args;

typedef struct {
  int32_t B, N, Hk, Hv, Dk, Dv;
  float scale;                    /* 0 -> Dk^-0.5                           */
  const void* y; int32_t y_dtype; int64_t y_sb, y_sn;
  const void* a; const void* bg; int32_t ab_dtype; int64_t ab_sb, ab_sn;
  const float* A_log;             /* [Hv], used when neg_exp_A == NULL      */
  const float* neg_exp_A;         /* [Hv] -exp(A_log) (fc1_fused.py:67)     */
  const void* dt_bias; int32_t dtb_dtype;
  const float* anc;               /* [B, N, N]                              */
  const float* pool; int64_t p_ss, p_sh, p_sv, p_sk;
  int64_t p_nslots;               /* slots addressable in the pool (bounds the state TMA); 0: unknown */
  const int64_t* state_slots;     /* [B]; NULL: slot b; negative -> 0       */
  void* o; int32_t o_dtype; int64_t o_sb, o_sn, o_sh;
  float* aux_k; int32_t aux_k_per_v; int64_t ak_sb, ak_sh, ak_sn;
  float* aux_vn; int64_t av_sb, av_sh, av_sn;
  float* aux_g; int64_t ag_sb, ag_sh;
  const dft_gdn_conv_args* conv;  /* NULL: read y                           */
  int32_t force_simt;             /* 1: CUDA-core path even where the tcgen05 path applies */
  /* 1: programmatic dependent launch (tcgen05 path).  The launch may start
   * while the previous kernel in the stream is still running: its set-up,
   * state / conv-state / conv-weight loads and the ancestor masks and conv
   * columns (pool, state_slots, conv_state, conv_slots, weight, bias, anc,
   * cidx) are read before it waits for that kernel; everything else (x or y,
   * a, bg, dt_bias, A_log / neg_exp_A) and every write come after.  The
   * caller guarantees that the previous kernel writes none of the former
   * (e.g. it is the previous layer's verify, or the layer's input
   * projection).  0: an ordinary launch. */
  int32_t overlap_prev;
} dft_gdn_args;
DFT_API int dft_gdn_tree_verify(const dft_gdn_args* a, int32_t* dev_status, void* stream);

/* ------------------------------------------------- closed-form commit -- */
/* Replaces fc1_fused.snapshots (fc1_fused.py:27-49) batched over layers and
 * requests: for each end u = ends[b, e] >= 0,
 *   S_u = e^{G_u} S0 + sum_{t in path[b], t anc-or-self of u} e^{G_u-G_t} vn_t k_t^T
 * S0 (l, slot, h, v, k) = state_in[l*si_sl + slot*si_ss + h*si_sh + v*si_sv + k*si_sk];
 * S_u written to state_out[l*so_sl + dst*so_ss + u*so_su + h*so_sh + v*so_sv + k*so_sk]
 * (so_su = 0 and dst = slot: in place into the pool; so_su = 0 with E > 1
 * returns DFT_ERR_INVALID, since every end would write the same tile).     */
typedef struct {
  int32_t L, B, N, Hk, Hv, Dk, Dv, P, E;
  const float* state_in; int64_t si_sl, si_ss, si_sh, si_sv, si_sk;
  float* state_out; int64_t so_sl, so_ss, so_su, so_sh, so_sv, so_sk;
  const int64_t* slots_in;        /* [B] (NULL: b)                          */
  const int64_t* slots_out;       /* [B] (NULL: b)                          */
  const float* aux_k; int32_t aux_k_per_v; int64_t ak_sl, ak_sb, ak_sh, ak_sn;
  const float* aux_vn; int64_t av_sl, av_sb, av_sh, av_sn;
  const float* aux_g; int64_t ag_sl, ag_sb, ag_sh;
  const float* anc;               /* [B, N, N]                              */
  const int64_t* path;            /* [B, P] node ids, -1 padded             */
  const int64_t* ends;            /* [B, E] end nodes, -1 = skip            */
} dft_commit_args;
DFT_API int dft_gdn_commit(const dft_commit_args* a, int32_t* dev_status, void* stream);

/* ------------------------------------------ tree-masked attention verify -- */
/* Replaces the flashinfer paged prefill the plugin plans for the gated
 * full-attention layers (fc1_plan.py:16-33, mask from fc1_branch64.py:39):
 * per request b, tree node n and q-head hq,
 *   o[b,n,hq] = softmax_j(q[b,n,hq] . k[j,hq/G] * sm_scale) . v[j,hq/G]
 * over the request's keys j = kv_indices[kv_indptr[b] .. kv_indptr[b+1]),
 * page size 1; the last N of them are the tree nodes in node order, and a
 * tree key m is visible to node n iff anc[b, n, m] > 0.5 (every prefix key
 * is visible).  bf16 q / caches / o, fp32 accumulation, P rounded to bf16
 * for the second MMA (as the reference's fa2 kernel does).  Tensor-core path:
 * D = 256, G = Hq / Hkv in {1,2,4,8}, N * G <= 128, N <= 64, 16-byte aligned
 * rows and strides; other shapes return DFT_ERR_UNSUPPORTED.
 * max_kv_len is the host-known bound on any request's key count (the plan's
 * HOST_KV_LEN); it sizes the key splits.  Splits > 1 need the workspace
 * (dft_tree_attn_workspace_bytes; 0 means none).  Keys outside
 * [0, n_slots) and lengths outside [N, max_kv_len] set DFT_DEV_BAD_INDEX. */
typedef struct {
  int32_t B, N, Hq, Hkv, D;
  const void* q; int64_t q_sb, q_sn, q_sh;      /* [B, N, Hq, D] bf16      */
  const void* k_cache; const void* v_cache;     /* [slots, Hkv, D] bf16    */
  int64_t kv_st, kv_sh;                         /* slot / head strides     */
  int64_t n_slots;
  const int32_t* kv_indptr;                     /* [B + 1]                 */
  const int32_t* kv_indices;                    /* token slots             */
  const float* anc; int64_t anc_sb;             /* [B, N, N] ancestor-or-self */
  float sm_scale;
  int32_t max_kv_len;
  void* o; int64_t o_sb, o_sn, o_sh;            /* [B, N, Hq, D] bf16      */
} dft_tree_attn_args;
DFT_API int64_t dft_tree_attn_workspace_bytes(const dft_tree_attn_args* a);
DFT_API int dft_tree_attn(const dft_tree_attn_args* a, void* workspace, int32_t* dev_status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DFORKTREE_B200_H */
