/*
 * specgrove_b200 — C ABI of the B200 (sm_100a) packed tree-verification step.
 *
 * Conventions shared by every entry point:
 *   - every pointer argument is a device pointer owned by the caller, unless
 *     its comment says "host";
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *   - the return value is an sg_status code (0 = success); nothing throws across
 *     this boundary; sg_last_error() gives a thread-local detail string;
 *   - calls are asynchronous on `stream` and re-entrant per stream.  Problems
 *     that can only be seen on the device (an out-of-range token, a negative or
 *     non-finite probability, an exhausted cache slot) are reported through the
 *     optional device word `status` (atomicMax of an sg_status code), which the
 *     caller reads with the results.
 */
#ifndef SPECGROVE_B200_H
#define SPECGROVE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SG_API __attribute__((visibility("default")))
#else
#define SG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum sg_status {
  SG_OK = 0,
  SG_ERR_INVALID_ARGUMENT = 1, /* bad sizes, strides, null pointers, alignment */
  SG_ERR_CUDA = 2,             /* a CUDA runtime call failed */
  SG_ERR_TREE = 3,             /* tree metadata out of range (device-detected) */
  SG_ERR_PROBABILITY = 4,      /* negative, non-finite or >= 2^40 probability */
  SG_ERR_CAPACITY = 5,         /* a request's KV slot would overflow */
  SG_ERR_UNSUPPORTED = 6,      /* shape or device this build does not handle */
  SG_ERR_WORKSPACE = 7         /* caller workspace too small */
};

/* Acceptance rules (sg_tree_accept_probs `rule`). */
enum sg_accept_rule {
  /* One uniform per visited depth; token = first index whose exact inclusive
   * prefix mass exceeds u * row_total (reference fused_tree_sampling.py:538-627). */
  SG_RULE_SCAN = 0,
  /* Two uniforms per depth: route among the children by exact cumulative child
   * mass (rows assumed normalised); on exit draw from the row with the children
   * removed (reference fused_tree_sampling.py:688-824). */
  SG_RULE_SPARSE_EXIT = 1
};

SG_API const char* sg_status_string(int status);
SG_API const char* sg_last_error(void);
SG_API int sg_version(void);
/* Number of kernels this library launched since load (all devices). */
SG_API uint64_t sg_launch_count(void);

/*
 * Tree-sampling acceptance over packed fp32 probability rows.
 *
 * Replaces the per-request verifier calls of the reference
 *   fused_tree_sampling.py:2172-2202  tree_verify_ancestral_fused_scan
 *   fused_tree_sampling.py:2205-2373  tree_verify_ancestral_sparse_exit_fused_scan(_batched)
 *   sampling.py:903-950               tree_verify_ancestral_batched (same law)
 * and the kernels they bind (fused.py:538-627 scan, :688-824 sparse exit).
 *
 * probs        [total_rows, vocab] fp32, row-major, 16-byte aligned rows when
 *              vocab % 4 == 0 (otherwise a scalar path is used)
 * row_offsets  [num_trees + 1] int64: tree t owns rows row_offsets[t] ..
 *              row_offsets[t+1]-1; local node j of tree t is row row_offsets[t]+j
 * parents      [total_rows] int64: local parent of each node, -1 for the root,
 *              parents[j] < j (topological order)
 * tokens       [total_rows] int64: token of each node; the root entry is ignored
 * max_depth    common output stride - 2; must be >= every tree's depth
 * uniforms     explicit uniforms [num_trees, uniform_stride] fp64 in [0,1):
 *              SG_RULE_SCAN reads u[depth], SG_RULE_SPARSE_EXIT reads
 *              u[2*depth] (route) and u[2*depth+1] (exit).  NULL selects the
 *              counter-based stream Philox4x32-10(key=seed, counter=(node,
 *              request_ids[t], purpose)).
 * request_ids  [num_trees] int64 keys for the Philox stream (ignored when
 *              uniforms != NULL; may be NULL, then t is used)
 * out          [num_trees, max_depth + 2] int64, reference layout
 *              (fused.py:149-150): slots [0, count) = accepted local nodes,
 *              out[max_depth] = count, out[max_depth+1] = bonus token; other
 *              slots are -1.
 * status       optional device int32 word, atomicMax'ed with an sg_status.
 */
SG_API int sg_tree_accept_probs(const float* probs, int64_t vocab,
                         const int64_t* row_offsets, const int64_t* parents,
                         const int64_t* tokens, int32_t num_trees,
                         int32_t max_nodes, int32_t max_depth, int32_t rule,
                         const double* uniforms, int32_t uniform_stride,
                         uint64_t seed, const int64_t* request_ids,
                         int64_t* out, int32_t* status, void* stream);

/*
 * Terminal-mass tree verifier.  Replaces
 *   sampling.py:542-735   tree_block_verify_terminal_mass (exit_mode
 *                         "internal", prefix_mode "batched"), the decoder's
 *                         default verifier (continuous_tree_block_decode.py:1328)
 * which draws the same output law as the ancestral walk as one terminal node
 * (weight P(prefix(v)) * P(exit | v)) and one bonus token from that node's
 * row with its children's tokens removed.
 *
 * probs, vocab, row_offsets, parents, tokens, num_trees, max_depth, out,
 * status: as sg_tree_accept_probs (same output layout).
 * total_rows   packed rows (row_offsets[num_trees]); one CTA per row sums
 *              the rows of internal nodes.
 * uniforms     explicit uniforms [num_trees, uniform_stride >= 2] fp64:
 *              u[0] draws the terminal node, u[1] the bonus token.  NULL
 *              selects Philox4x32-10(key=seed, counter=(0, request lo,
 *              request hi, 2)) with request_ids[t] (t when NULL).
 * workspace    device scratch of sg_tree_verify_terminal_mass_workspace_bytes
 *              (total_rows) bytes, 16-byte aligned (row masses).
 * Row masses are exact 64.64 fixed-point sums; normalisation, prefix
 * products and the terminal draw run in fp64 in node order; the bonus token
 * is the exact fixed-point inverse CDF (first token whose running mass
 * exceeds floor(u * total)).  Device-detected problems set status
 * (SG_ERR_TREE, SG_ERR_PROBABILITY) and leave the tree's output row -1.
 */
SG_API size_t sg_tree_verify_terminal_mass_workspace_bytes(int64_t total_rows);
SG_API int sg_tree_verify_terminal_mass(const float* probs, int64_t vocab,
                         const int64_t* row_offsets, const int64_t* parents,
                         const int64_t* tokens, int32_t num_trees,
                         int64_t total_rows, int32_t max_depth,
                         const double* uniforms, int32_t uniform_stride,
                         uint64_t seed, const int64_t* request_ids,
                         int64_t* out, int32_t* status, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Element types of logit rows (sg_tree_accept_logits `dtype`). */
enum sg_dtype { SG_DTYPE_F32 = 0, SG_DTYPE_BF16 = 1 };

/*
 * Tree-sampling acceptance straight from logit rows: only the visited rows
 * are normalised (reference direct-logits verifiers,
 *   fused_tree_sampling.py:2417-2465  tree_verify_ancestral_logits_fused_scan
 *   fused_tree_sampling.py:2468-2533  tree_verify_ancestral_logits_fused_scan_batched
 * and their kernels :942-1115, :1117-1236).  At a visited node the weights
 * are w_j = exp(double(logit_j) / T - max), the token is the first whose
 * exact inclusive prefix of w exceeds u[depth] * sum(w) (fallback V - 1).
 * logits       [total_rows, vocab] fp32 or bf16 (dtype), row-major
 * temperature  > 0
 * uniforms     [num_trees, uniform_stride] fp64, u[depth] read, or NULL for
 *              Philox4x32-10(seed, (node, request, purpose 0)) like
 *              sg_tree_accept_probs' scan rule
 * Other arguments and the output layout as sg_tree_accept_probs.
 */
SG_API int sg_tree_accept_logits(const void* logits, int32_t dtype, int64_t vocab, const int64_t* row_offsets,
                                 const int64_t* parents, const int64_t* tokens, int32_t num_trees,
                                 int32_t max_nodes, int32_t max_depth, double temperature, const double* uniforms,
                                 int32_t uniform_stride, uint64_t seed, const int64_t* request_ids, int64_t* out,
                                 int32_t* status, void* stream);

/*
 * Walk the trees with one pre-drawn posterior token per node
 * (reference fused_tree_sampling.py:120-151 fused_tree_follow_kernel, used by
 * tree_verify_ancestral_same_draw_fused :2376-2414; law of sampling.py:903-950).
 * posterior    [total_rows] int64 posterior token per packed node
 * other arguments as sg_tree_accept_probs.
 */
SG_API int sg_tree_follow(const int64_t* posterior, const int64_t* row_offsets,
                   const int64_t* parents, const int64_t* tokens,
                   int32_t num_trees, int32_t max_nodes, int32_t max_depth,
                   int64_t* out, int32_t* status, void* stream);

/*
 * Accepted-path KV commit: copy kept rows inside a slot-strided KV arena or
 * from a packed source into it.
 *
 * Replaces _PersistentRequestCachePool.append_packed_sequence
 * (continuous_tree_block_decode.py:215-261): for every plane (layer, K|V,
 * kv head) row dst_rows[i] of `dst` receives row src_rows[i] of `src`.
 *
 * dst, src     base pointers of [num_planes, plane_rows, row_bytes] arenas;
 *              src == dst is the in-place tail compaction
 * *_plane_rows rows per plane of each arena
 * row_bytes    bytes per row (head_dim * element size), multiple of 4
 * src_rows, dst_rows  [num_rows] int64 row indices within a plane
 * group_offsets [num_groups + 1] int64: rows of one request are
 *              group_offsets[g] .. group_offsets[g+1]-1.  Within a group, an
 *              in-place commit must satisfy dst_rows[i] <= src_rows[i] with
 *              both increasing (true for [0] + accepted nodes); groups must
 *              not share rows.
 * status       optional device word; rows out of range set SG_ERR_CAPACITY and
 *              are skipped.
 */
SG_API int sg_kv_commit(void* dst, int64_t dst_plane_rows, const void* src,
                 int64_t src_plane_rows, int64_t num_planes, int64_t row_bytes,
                 const int64_t* src_rows, const int64_t* dst_rows,
                 const int64_t* group_offsets, int32_t num_groups,
                 int32_t max_group_rows, int32_t* status, void* stream);

/*
 * Accepted-path commit driven directly by an acceptance output buffer, with no
 * host round trip: for tree t, keep rows [0] + out[t, 0:count] of the tail
 * written at slot[t] * capacity + lengths_in[t] + j are moved to
 * slot[t] * capacity + lengths_in[t] + i, for every plane; lengths_out[t] =
 * lengths_in[t] + count + 1.  Same arena layout as sg_kv_commit; this is the
 * in-place form of append_packed_sequence (continuous_tree_block_decode.py:
 * 215-261) for an engine that writes tree rows into the arena tail.
 * slots, lengths_in, lengths_out  [num_trees] int64 (lengths_out != lengths_in)
 * accept_out   [num_trees, max_depth + 2] output of sg_tree_accept_probs /
 *              sg_tree_follow; max_depth <= 63.
 * status       a count that overflows the slot sets SG_ERR_CAPACITY; a path
 *              that is not a root path inside the slot's tail (node < depth,
 *              or beyond the capacity) sets SG_ERR_TREE and that tree's rows
 *              are left unmoved.
 */
SG_API int sg_kv_commit_accepted(void* arena, int64_t plane_rows, int64_t num_planes,
                          int64_t row_bytes, int64_t capacity, const int64_t* slots,
                          const int64_t* lengths_in, int64_t* lengths_out,
                          const int64_t* accept_out, int32_t num_trees,
                          int32_t max_depth, int32_t* status, void* stream);

/*
 * Shared-budget tier allocation for the next wave (host function: every
 * pointer is a HOST pointer; no device work).  Replaces the reference's
 * exact-row allocator _allocate_global_tree_budgets
 * (continuous_tree_block_decode.py:706-795) with its wave-cost model
 * _global_wave_cost (:619-641), given the per-request weights the decoder
 * derives from progress and age (:751-760; across data-parallel ranks their
 * global terms come from the per-wave score allgather).
 *
 * weights      [num_requests] fp64 >= 0
 * options      [num_options] tier sizes in draft nodes, strictly increasing,
 *              >= 1; a tier of b nodes takes b + 1 rows
 * utilities    [num_requests, num_options] fp64 >= 1 (draft expected tokens)
 * row_budget   rows of the wave; >= num_requests * (options[0] + 1)
 * cost model   fixed_row_equivalent > 0 with curve_points == 0 (cost = fixed +
 *              rows), or fixed_row_equivalent = NaN with a piecewise-linear
 *              curve of curve_points (rows, cost) points, rows increasing,
 *              cost positive and non-decreasing
 * allocation   [num_requests] out: the chosen tier (an entry of options)
 * Returns SG_ERR_INVALID_ARGUMENT for a malformed problem.  Results are
 * bit-identical to the reference's (same fp64 evaluation order and tie rules).
 */
SG_API int sg_allocate_tiers(int32_t num_requests, const double* weights, int32_t num_options,
                             const int32_t* options, const double* utilities, int32_t row_budget,
                             double fixed_row_equivalent, const int32_t* curve_rows, const double* curve_cost,
                             int32_t curve_points, int32_t* allocation);

/*
 * sg_allocate_tiers on the device: the same knapsack, the same allocation
 * bit for bit, as one CTA reading weights and utilities that device kernels
 * produced (sg_build_draft_trees), so a wave is planned without a host round
 * trip.  weights, utilities and allocation are DEVICE pointers (8-, 8-, 4-byte
 * aligned); options and the cost curve are host arrays, checked on the host
 * like sg_allocate_tiers.  At most 8 options, row_budget <= 4096, 64 curve
 * points (SG_ERR_UNSUPPORTED otherwise).  workspace: device, 4-byte aligned,
 * sg_allocate_tiers_device_workspace_bytes(num_requests, row_budget) bytes
 * (per step and row total: the back pointer).  A weight or utility out of
 * range (device-detected) sets SG_ERR_INVALID_ARGUMENT in *status, a wave
 * that no allocation fits sets SG_ERR_CAPACITY; allocation is then -1.
 */
SG_API size_t sg_allocate_tiers_device_workspace_bytes(int32_t num_requests, int32_t row_budget);
SG_API int sg_allocate_tiers_device(int32_t num_requests, const double* weights, int32_t num_options,
                                    const int32_t* options, const double* utilities, int32_t row_budget,
                                    double fixed_row_equivalent, const int32_t* curve_rows,
                                    const double* curve_cost, int32_t curve_points, int32_t* allocation,
                                    int32_t* status, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Draft-tree construction on the device (the proposal step before a wave).
 *
 * sg_proposal_topk: per row of drafter logits (bf16 or fp32; a row = one
 * (request, draft depth); row r is element offset (r / rows_per_group) *
 * group_stride + (r % rows_per_group) * row_stride, e.g. block rows 1..L of
 * [R, block, vocab] logits), the k largest proposal masses
 * of q = softmax(logits / T) in fp64 and their token ids, sorted by mass
 * (ties to the lower token id): log_q[rows, k] fp64, ids[rows, k] int64.
 * Replaces probabilities(logits, T, float64) + torch.topk(q, k) + log
 * (sampling.py:29-36, tree.py:183-184).  1 <= k <= min(1024, vocab), T > 0.
 * Non-finite logits set SG_ERR_PROBABILITY in *status.
 */
SG_API int sg_proposal_topk(const void* logits, int32_t dtype, int64_t row_stride, int32_t rows_per_group,
                            int64_t group_stride, int32_t rows, int32_t vocab, int32_t k, double temperature,
                            double* log_q, int64_t* ids, int32_t* status, void* stream);

/*
 * sg_build_draft_trees: the best-first prefix tree of every request
 * (probability_tree, tree.py:148-212) from its ranked log masses
 * log_q/ids [num_trees, length, width] (width = the top-k kept per depth,
 * k = min(budget, vocab) in the reference), bit-equal to the reference's
 * tree for the same log masses (same fp64 operation order, same tie order).
 *   budgets      device [num_trees] per-request budgets (<= budget), or null
 *   budget       node budget (and the row stride of the outputs), <= 4096
 *   rewards      host [length] per-depth reward schedule, or null (all 0)
 *   rank_caps    host [length] per-depth rank caps (>= 1), or null
 *   adaptive_min_budget, confidence_threshold: on rounds whose mean greedy
 *                log mass over the first 4 depths is >= log(threshold) the
 *                budget becomes adaptive_min_budget (-1: off)
 *   tiers        host [num_tiers] increasing tier sizes (<= 8 tiers): the
 *                utility of tier b is the draft expected tokens of the first
 *                b nodes (_prefix_tree / _draft_tree_expected_tokens,
 *                continuous_tree_block_decode.py:560-586), NaN (and
 *                SG_ERR_TREE) when the tree has fewer nodes
 * Outputs (device): tokens [num_trees, budget] (node i >= 1 holds
 * tokens[i - 1]), parents [num_trees, budget + 1] (root -1), depths and
 * masses (prefix log mass incl. rewards) [num_trees, budget + 1],
 * node_count [num_trees], utilities [num_trees, num_tiers] fp64 (input to
 * sg_allocate_tiers_device).
 */
SG_API int sg_build_draft_trees(const double* log_q, const int64_t* ids, int32_t num_trees, int32_t length,
                                int32_t width, const int32_t* budgets, int32_t budget, const double* rewards,
                                const int32_t* rank_caps, int32_t adaptive_min_budget,
                                double confidence_threshold, const int32_t* tiers, int32_t num_tiers,
                                int64_t* tokens, int64_t* parents, int32_t* depths, double* masses,
                                int32_t* node_count, double* utilities, int32_t* status, void* stream);

/*
 * sg_pack_tree_wave: the packed verify wave of the chosen tiers: request r
 * takes rows row_offsets[r] .. row_offsets[r + 1] - 1 = its anchor token
 * (anchor_tokens[r], the last generated token; parent -1) followed by the
 * first allocation[r] nodes of its tree (parents as local row indices), the
 * inputs of sg_verify_pass.  At most 1024 trees; a tier larger than the tree
 * or a wave above max_rows sets SG_ERR_TREE (row_offsets then all 0).
 */
SG_API int sg_pack_tree_wave(const int64_t* tokens, const int64_t* parents, int32_t budget,
                             const int32_t* node_count, const int32_t* allocation, const int64_t* anchor_tokens,
                             int32_t num_trees, int64_t max_rows, int64_t* row_offsets, int64_t* wave_parents,
                             int64_t* wave_tokens, int32_t* status, void* stream);

/* Epilogues of sg_gemm_bf16. */
enum sg_gemm_epilogue {
  SG_EPI_STORE_BF16 = 0, /* C bf16 [M, ldc] = acc */
  SG_EPI_STORE_F32 = 1,  /* C fp32 [M, ldc] = acc */
  SG_EPI_RESIDUAL = 2,   /* C fp32 [M, ldc] += acc; aux bf16 [M, ld_aux] = bf16(C) if aux */
  SG_EPI_SWIGLU = 3      /* B rows interleaved in 128-row gate/up blocks:
                            C bf16 [M, N/2] = silu(gate) * up */
};

/*
 * tcgen05 GEMM: acc[M, N] = A[M, K] . B[N, K]^T, bf16 operands (row-major,
 * K contiguous, 16-byte aligned rows), fp32 accumulation in tensor memory,
 * fused epilogue.  K % 64 == 0, N % 32 == 0.  This is the projection / MLP
 * GEMM of the target pass (HF Qwen3 q/k/v/o/gate/up/down nn.Linear layers,
 * called from engine.py:499-517 through transformers' Qwen3Model).
 */
SG_API int sg_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb,
                 void* C, int64_t ldc, int32_t M, int32_t N, int32_t K,
                 int32_t epilogue, void* aux, int64_t ld_aux, int32_t* status,
                 void* stream);

/*
 * sg_gemm_bf16 with a stream-K workspace for the wave tail (no counterpart in
 * the reference): when the tiles do not fill whole waves of one CTA per SM,
 * the k-blocks of the last partial wave are split over all SMs and combined
 * through fp32 partial accumulators in `workspace` (deterministic order).
 * workspace_bytes >= sg_gemm_split_workspace_bytes(); its flag area must be
 * zero before the first call (sg_gemm_split_workspace_init), and calls sharing
 * a workspace must be ordered (one stream).  A null workspace or a smaller
 * size runs sg_gemm_bf16 unchanged.
 */
SG_API size_t sg_gemm_split_workspace_bytes(void);
SG_API int sg_gemm_split_workspace_init(void* workspace, size_t workspace_bytes, void* stream);
SG_API int sg_gemm_bf16_ws(const void* A, int64_t lda, const void* B, int64_t ldb,
                    void* C, int64_t ldc, int32_t M, int32_t N, int32_t K,
                    int32_t epilogue, void* aux, int64_t ld_aux, int32_t* status,
                    void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * The packed tree-verification pass (Qwen3 decoder shape).
 * ------------------------------------------------------------------------ */

/* Per-layer weight pointers, in this order, W_COUNT = 8 per layer:
 *   0 input RMSNorm [hidden] bf16
 *   1 fused q|k|v projection [(nq + 2 nkv) * head_dim, hidden] bf16
 *   2 q RMSNorm [head_dim] bf16      3 k RMSNorm [head_dim] bf16
 *   4 o projection [hidden, nq * head_dim] bf16
 *   5 post-attention RMSNorm [hidden] bf16
 *   6 gate|up projection, rows interleaved in 128-row blocks
 *     (gate 0..127, up 0..127, gate 128..255, ...) [2 * intermediate, hidden]
 *   7 down projection [hidden, intermediate] bf16
 * (HF Qwen3DecoderLayer: input_layernorm, self_attn.{q,k,v}_proj,
 *  self_attn.{q,k}_norm, self_attn.o_proj, post_attention_layernorm,
 *  mlp.{gate,up}_proj, mlp.down_proj.) */
#define SG_LAYER_WEIGHTS 8

typedef struct {
  int32_t num_layers, hidden, num_q_heads, num_kv_heads, head_dim, intermediate, vocab;
  float rms_eps;
  const void* embed;        /* [vocab, hidden] bf16 */
  const void* final_norm;   /* [hidden] bf16 */
  const void* lm_head;      /* [vocab, hidden] bf16 */
  const float* inv_freq;    /* [head_dim / 2] rotary inverse frequencies */
  const void* const* layers;/* host array [num_layers * SG_LAYER_WEIGHTS] of device pointers */
} sg_model_desc;

/* Persistent KV arena: bf16 [num_layers, 2 (K, V), num_kv_heads,
 * num_slots * capacity, head_dim]; request slot s owns rows
 * [s * capacity, (s + 1) * capacity) of every plane (the layout of
 * _PersistentRequestCachePool.key_storage / value_storage,
 * continuous_tree_block_decode.py:176-213, in one allocation). */
typedef struct {
  void* storage;
  int64_t num_slots, capacity;
} sg_arena_desc;

/* One wave: every request's tree rows packed back to back. */
typedef struct {
  int32_t num_requests, num_rows, max_rows_per_request, max_depth;
  const int64_t* row_offsets;    /* [R + 1] */
  const int64_t* parents;        /* [Q] local parent, -1 for the root */
  const int64_t* tokens;         /* [Q] input token (root row: last committed token) */
  const int64_t* slots;          /* [R] arena slot */
  const int64_t* cache_lengths;  /* [R] committed KV rows L_i */
  const int64_t* position_base;  /* [R] rotary position of the root row */
  const int64_t* request_ids;    /* [R] Philox key per request (NULL: index) */
  uint64_t seed;
  float temperature;             /* > 0: sample softmax(logits / T); 0: greedy,
                                    the argmax of the bf16-rounded logits
                                    (first maximum), the reference's T = 0
                                    verifier tree_verify_greedy_block,
                                    continuous_tree_block_decode.py:45-71 */
  int32_t commit;                /* 1: move accepted rows' KV to L_i.. */
  int64_t* accept_out;           /* [R, max_depth + 2] reference layout */
  int64_t* lengths_out;          /* [R] L_i + accepted + 1 (commit) */
  int64_t* posterior;            /* optional [Q] sampled token per row */
  float* lse;                    /* optional [Q] log-normaliser per row */
  float* child_logprob;          /* optional [Q] log p_parent(token), 0 at roots */
  float* hidden_out;             /* optional [Q, hidden] fp32 last residual stream */
  int32_t* status;               /* optional device status word */
  void* const* trace_events;     /* optional host array of SG_TRACE_EVENTS
                                    cudaEvent_t recorded at stage boundaries */
  /* Drafter feature hand-off (continuous_tree_block_decode.py:2144-2158: the
   * decoder concatenates output.hidden_states[l + 1] of every
   * engine.draft.target_layer_ids layer l and keeps the rows [0] + accepted
   * nodes of each request).  hidden_states[l + 1] is the residual stream after
   * layer l, and for the last layer the final-normed stream, as in HF Qwen3. */
  int32_t num_feature_layers;    /* 0: no features */
  const int32_t* feature_layers; /* HOST array [num_feature_layers], each in [0, num_layers) */
  void* features_out;            /* bf16 [Q, num_feature_layers * hidden], 16-byte aligned:
                                    layer feature_layers[f] in columns
                                    [f * hidden, (f + 1) * hidden); written by the
                                    layers' residual GEMM epilogues */
  void* features_kept;           /* optional bf16 [<= Q, num_feature_layers * hidden]:
                                    the rows [0] + accepted nodes of every
                                    request, requests in order */
  int64_t* features_kept_offsets;/* [R + 1] row offsets of each request's kept
                                    rows in features_kept (with features_kept) */
} sg_wave_desc;

/* Stage boundaries recorded into sg_wave_desc.trace_events (the stage
 * timings of the reference's StageMeter, engine.py:151-177, at kernel
 * granularity; layer-0 boundaries time each per-layer kernel once):
 *  0 start  1 tree metadata + embedding  2 L0 input norm  3 L0 QKV GEMM
 *  4 L0 q/k norm + RoPE + KV tail write  5 L0 tree attention  6 L0 O GEMM
 *  7 L0 post norm  8 L0 gate/up GEMM  9 L0 down GEMM  10 all layers
 *  11 final norm  12 LM head + sampling GEMM  13 combine (+ child log-probs)
 *  14 tree walk  15 commit (end) */
#define SG_TRACE_EVENTS 16

/* Builds TMA descriptors for every weight and allocates the activation
 * workspace for up to max_rows packed rows (cudaMalloc, freed by destroy). */
SG_API int sg_engine_create(const sg_model_desc* model, const sg_arena_desc* arena,
                     int32_t max_rows, int32_t max_requests, void** engine_out);
SG_API int sg_engine_destroy(void* engine);
SG_API size_t sg_engine_workspace_bytes(void* engine);

/*
 * One packed tree-verification step, enqueued on `stream` with no host
 * synchronisation (capturable in a CUDA graph): target forward over the
 * packed rows with request-isolated tree attention reading the arena, new
 * K/V written at each request's arena tail, LM head fused with softmax and
 * sampling (one posterior draw per row from softmax(logits / T): the law of
 * sampling.py:903-950; greedy argmax at T = 0), tree walk into accept_out,
 * optional commit.  Replaces continuous_tree_block_decode.py:1748-2129
 * (pack, target, select_commit stages).
 */
SG_API int sg_verify_pass(void* engine, const sg_wave_desc* wave, void* stream);

/* ------------------------------------------------------------------------
 * The drafter step (DFlash block drafter, the step before each wave).
 * ------------------------------------------------------------------------
 * The drafter (third_party/ddtree_official/model/dflash.py:147-200) is a
 * Qwen3 layer stack whose block rows (the request's last token, then
 * block_size - 1 mask tokens, embedded with the TARGET's embedding) attend
 * bidirectionally to each other and to the request's draft cache: the K/V
 * of every context row, projected from the target features of the rows
 * committed so far (fc, then hidden_norm; k_norm and RoPE on the keys).
 * The model descriptor is an sg_model_desc of the drafter's layers with
 * embed and lm_head pointing at the target's and final_norm the drafter's
 * norm; the draft cache is an sg_arena_desc of the drafter's layers. */
typedef struct {
  const void* fc;              /* [hidden, num_feature_layers * hidden] bf16 */
  const void* hidden_norm;     /* [hidden] bf16 */
  int32_t num_feature_layers;  /* target layers concatenated per context row */
  int32_t block_size;          /* rows per request block (16), <= 256 */
  int64_t mask_token_id;       /* token of block rows 1 .. block_size - 1 */
  int32_t max_update_rows;     /* largest number of context rows per call */
} sg_draft_desc;

/* One drafter step over R requests (the packed form of _propose_many with
 * reuse_request_draft_cache, continuous_tree_block_decode.py:889-962). */
typedef struct {
  int32_t num_requests;
  int32_t num_update_rows;        /* U = update_offsets[R] (host copy) */
  const int64_t* slots;           /* [R] draft-cache slot */
  const int64_t* cache_lengths;   /* [R] context rows already in the draft cache */
  const int64_t* update_offsets;  /* [R + 1] rows of `features` per request */
  const void* features;           /* bf16 [U, num_feature_layers * hidden], 16-byte
                                     aligned (sg_wave_desc.features_kept of the
                                     previous wave) */
  const int64_t* anchor_tokens;   /* [R] last generated token (block row 0) */
  void* logits_out;               /* bf16 [R, block_size, vocab]: the drafter's
                                     logits of every block row (row 0, the
                                     anchor's, is not a proposal) */
  int64_t* lengths_out;           /* [R] cache_lengths + update rows */
  int32_t* status;                /* optional device status word */
  int32_t context_only;           /* 1: only append the context rows' K/V
                                     (prefill of the draft cache alongside the
                                     target's prefill chunks); no block rows,
                                     logits_out and anchor_tokens unused */
} sg_draft_wave;

/* Builds the drafter engine: TMA descriptors for the drafter's weights and
 * the fc, and a workspace for max_requests * block_size block rows and
 * max_update_rows context rows (cudaMalloc, freed by sg_engine_destroy). */
SG_API int sg_draft_engine_create(const sg_model_desc* model, const sg_draft_desc* draft,
                                  const sg_arena_desc* arena, int32_t max_requests, void** engine_out);

/* One drafter step, enqueued on `stream` with no host synchronisation: the
 * context rows' K/V (fc + hidden_norm, then every layer's k/v projection,
 * k_norm, RoPE at positions cache_len ..) appended to the draft cache
 * (committed: lengths_out), the block rows' forward with bidirectional
 * attention over [cache, update, block], the drafter's final norm and the
 * target's LM head into logits_out.  The block rows' own K/V live past the
 * committed length only for this call (the reference crops them). */
SG_API int sg_draft_pass(void* engine, const sg_draft_wave* wave, void* stream);

/*
 * Final RMSNorm + LM head fused with softmax and sampling over caller-given
 * residual rows: the computation of sg_verify_pass's sampling stage, and the
 * fused form of the reference's lazy-projection verifier input (hidden states
 * plus the LM-head module instead of logits,
 * continuous_tree_block_decode.py:1795-1808, 1933-1964).
 *
 * x            fp32 [rows, hidden] residual rows (e.g. sg_wave_desc.hidden_out),
 *              16-byte aligned
 * final_norm   bf16 [hidden], 4-byte aligned;  lm_head bf16 [vocab, hidden],
 *              16-byte aligned;  hidden % 64 == 0, vocab % 32 == 0
 * row_node     int32 [rows], row_request int64 [rows]: the Philox key of each
 *              row's draw (seed, request, node), as in the pass
 * temperature  > 0 samples softmax(logits / T); 0 is greedy (argmax of the
 *              bf16-rounded logits, first maximum)
 * lse          fp32 [rows] log-normaliser of logits / T (T = 1 when greedy);
 *              posterior int64 [rows] the drawn token
 * workspace    256-byte aligned device buffer of at least
 *              sg_lm_head_sample_workspace_bytes(rows, hidden, vocab) bytes,
 *              used by this call only (calls sharing one must be ordered)
 * If the GEMM gives up a bounded wait, every row gets posterior -1 and lse
 * NaN.  Misaligned pointers return SG_ERR_INVALID_ARGUMENT before any launch.
 */
SG_API size_t sg_lm_head_sample_workspace_bytes(int32_t rows, int32_t hidden, int32_t vocab);

/*
 * sg_lm_head_sample over rows that are already final-normed, in bf16
 * ([rows, hidden], 16-byte aligned): HF's last_hidden_state, which the
 * reference's lazy-projection verifiers receive together with the LM head
 * (fused_tree_sampling.py:2758-2840, continuous_tree_block_decode.py:1933-1964).
 * Same keys, outputs and workspace size as sg_lm_head_sample.
 */
SG_API int sg_lm_head_sample_bf16(const void* xn, const void* lm_head, int32_t rows, int32_t hidden, int32_t vocab,
                                  const int32_t* row_node, const int64_t* row_request, uint64_t seed,
                                  float temperature, float* lse, int64_t* posterior, void* workspace,
                                  size_t workspace_bytes, void* stream);
SG_API int sg_lm_head_sample(const float* x, const void* final_norm, const void* lm_head, int32_t rows,
                             int32_t hidden, int32_t vocab, float rms_eps, const int32_t* row_node,
                             const int64_t* row_request, uint64_t seed, float temperature, float* lse,
                             int64_t* posterior, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Fused LM-head sampling that allocates no device memory.  No counterpart in
 * the reference: it exists for callers that cannot call cudaMalloc, such as
 * a serving process that has handed its device memory to its own pool
 * allocator, or a foreign-language caller whose FFI only passes in buffers
 * it allocated itself.
 *
 * Same arguments (minus the workspace), computation and output as
 * sg_lm_head_sample, including the alignment rules and the posterior = -1 /
 * lse = NaN answer to a GEMM that gave up a bounded wait.
 *
 * Its scratch (a status word, the normalised rows and per-vocab-tile
 * partials: sg_lm_head_sample_workspace_bytes(rows, hidden, vocab) bytes,
 * about rows * (2 * hidden + 16 * ceil(vocab / 256)) + 512) lives in one
 * library-owned device array of SG_LM_HEAD_STATIC_SCRATCH_BYTES, present on
 * every GPU that loads the library until the process exits; larger requests
 * fail with SG_ERR_WORKSPACE (e.g. 473 rows fit at hidden 4096, vocab
 * 151936).  The first call on each device looks up the array's device
 * address (cudaGetSymbolAddress) and caches it; make that first call before
 * any stream capture.  The cached address belongs to the CUDA context of
 * that first call: after cudaDeviceReset in the same process it is stale,
 * and this entry point must not be used on that device again.  All calls
 * share the array: calls whose executions overlap on the GPU (other streams,
 * other host threads) race and must be serialised by the caller.  The status
 * word is cleared at the start of every call; every other scratch value read
 * is written earlier in the same call.
 */
#define SG_LM_HEAD_STATIC_SCRATCH_BYTES (8u << 20)
SG_API int sg_lm_head_sample_static(const float* x, const void* final_norm, const void* lm_head,
                             int32_t rows, int32_t hidden, int32_t vocab, float rms_eps,
                             const int32_t* row_node, const int64_t* row_request,
                             uint64_t seed, float temperature, float* lse,
                             int64_t* posterior, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPECGROVE_B200_H */
