/* ssd_b200.h - C ABI of the B200 (sm_100a) kernels behind one SSD
 * speculative-decoding round: tree draft through a subset of the target's
 * layers plus bridges, tree attention over the shared KV cache, one-pass
 * target verification, and KV compaction.
 *
 * The reference (yotamabramson/subnetwork-speculative-decoding) is pure
 * Python/PyTorch and has no FFI. Each entry point below names the reference
 * code (path:line inside that project) whose computation it replaces; the
 * Python host package calls these through ctypes.
 *
 * Conventions
 *  - Every function returns an int status (SSD_OK == 0). On failure
 *    ssd_last_error() returns a message for the calling host thread.
 *  - Pointers are device pointers unless a parameter says otherwise. Sizes
 *    are int64. `stream` is a cudaStream_t passed as void*.
 *  - No function allocates device memory. Functions that need scratch take a
 *    caller-owned `workspace` of `workspace_bytes` bytes which must be zeroed
 *    once before its first use (its counters reset themselves afterwards);
 *    one workspace must not be shared by calls that run concurrently.
 *  - dtype SSD_F32 selects the fp32 CUDA-core path (the exact-parity tier);
 *    SSD_BF16 selects the tcgen05 tensor-core path (bf16 operands, fp32
 *    accumulation). Activations passed to a GEMM use the weights' dtype.
 *  - The residual stream is always fp32 [T, d] row-major.
 */
#ifndef SSD_B200_H
#define SSD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  SSD_OK = 0,
  SSD_ERR_INVALID = 1,     /* bad argument (maps to Python ValueError) */
  SSD_ERR_UNSUPPORTED = 2, /* shape/dtype this build does not handle */
  SSD_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  SSD_ERR_OVERFLOW = 4,    /* cache or buffer capacity exceeded (RuntimeError) */
  SSD_ERR_WORKSPACE = 5    /* workspace too small */
};

enum { SSD_F32 = 0, SSD_BF16 = 1 };
enum { SSD_ACT_NONE = 0, SSD_ACT_SILU = 1, SSD_ACT_GELU = 2, SSD_ACT_RELU = 3 };

/* Output-feature layout of a multi-segment GEMM. CONCAT: segment outputs are
 * concatenated (q|k|v). PAIRS: two segments (gate, up) of equal size
 * processed 64 features at a time so a SwiGLU epilogue sees both halves. */
enum { SSD_SEG_CONCAT = 0, SSD_SEG_PAIRS = 1 };

int ssd_version(void);
/* Kernels this library has launched (or recorded into a CUDA graph being
 * captured) in this process so far, all threads and devices together. */
int64_t ssd_launch_count(void);
const char* ssd_last_error(void);
int ssd_device_sm_count(int device);

/* Workspace bytes the GEMM / attention / head entry points need for forwards
 * of up to `max_rows` token rows whose lm_head heads (argmax / top-k) see up
 * to `max_head_rows` rows, over a vocabulary of `vocab` tokens. */
int64_t ssd_workspace_bytes(int64_t max_rows, int64_t max_head_rows, int64_t vocab);

/* RMSNorm folded into the GEMMs around it (bf16 path).
 * SsdNormOut: an epilogue that updates the fp32 residual also writes the
 * input of the next RMSNorm's consumer, out[t, n] = resid[t, n] * weight[n]
 * (bf16), and the sum of squares of resid[t, n] over each 128-feature tile i
 * of row t into ssq[t * ld_ssq + i].
 * SsdRowNorm: a GEMM whose input rows are such products scales output
 * column t (token t) by rsqrt(sum_i ssq[t * ld + i] / d + eps) before its
 * epilogue, which completes the RMSNorm (W (x_t w) s_t = W RMSNorm(x_t)).
 * Either pointer argument may be NULL (no folding). */
typedef struct SsdNormOut {
  const void* weight;
  void* out;
  int64_t ldo;
  float* ssq;
  int64_t ld_ssq;
} SsdNormOut;
typedef struct SsdRowNorm {
  const float* ssq;
  int64_t ld;
  int64_t parts;
  int64_t d;
  float eps;
} SsdRowNorm;

/* Embedding gather: resid[t, :] = table[ids[t], :] (fp32 out).
 * Replaces base.embed_tokens(input_ids), ssd/models/subnetwork_draft.py:290-291. */
int ssd_embed(const int32_t* ids, int64_t T, const void* table, int64_t vocab, int64_t d, int dtype,
              float* resid, const SsdNormOut* norm_out, uint32_t* status, void* stream);

/* RMSNorm of the fp32 residual stream into the GEMM activation dtype:
 * out = weight * (x * rsqrt(mean(x^2) + eps)).
 * Replaces LlamaRMSNorm (subnetwork_draft.py:216,245,344) and the bridge
 * RMSNorm (ssd/models/bridges.py:33-37). */
int ssd_rmsnorm(const float* x, int64_t T, int64_t d, int64_t ldx, const void* weight, float eps, void* out,
                int64_t ldo, int dtype, void* stream);

/* y = x @ W^T (+ bias) with a fused epilogue, W given as up to 3 row
 * segments w[i] of shape [rows[i], K] (row-major, K contiguous).
 *   epilogue SSD_EPI_STORE:    out[t, n] = act(acc + bias)        (dtype)
 *   epilogue SSD_EPI_RESIDUAL: resid[t, n] += acc + bias          (fp32)
 *   epilogue SSD_EPI_SWIGLU:   out[t, f] = silu(acc_g + b_g) * (acc_u + b_u)
 *                              (segments gate, up; layout SSD_SEG_PAIRS)
 *   epilogue SSD_EPI_STORE_F32: out[t, n] = acc + bias as fp32 (logits)
 * Replaces F.linear sites: o_proj + residual (subnetwork_draft.py:243), the
 * SwiGLU MLP + residual (:245), bridge MLPs (ssd/models/bridges.py:53-54,
 * 64-65, 131-135) and the lm_head (subnetwork_draft.py:347-349). */
enum { SSD_EPI_STORE = 0, SSD_EPI_RESIDUAL = 1, SSD_EPI_SWIGLU = 2, SSD_EPI_STORE_F32 = 3 };
int ssd_linear(const void* x, int64_t ldx, int64_t T, int64_t K, int n_seg, const void* const* w,
               const int64_t* rows, const void* const* bias, int seg_layout, int epilogue, int act, void* out,
               int64_t ldo, float* resid, int64_t ldr, int dtype, void* workspace, int64_t workspace_bytes,
               const SsdRowNorm* in_norm, const SsdNormOut* norm_out, uint32_t* status, void* stream);

/* ssd_linear without a workspace, for callers that cannot allocate device
 * memory (a server that reserves all memory at start-up, a plain C caller
 * with no allocator, code that must avoid the allocator's synchronisation).
 * No counterpart in the reference: it is an addition of this library.
 * Same arguments and results as ssd_linear; its split-K scratch is a fixed
 * 20 MiB array inside the library that every GPU loading the library keeps
 * until exit. Limit: T <= 64 token rows (bf16 or fp32); on a GPU of up to
 * 148 SMs every such call fits the array. Larger calls, and any shape whose
 * split-K scratch on this GPU exceeds the array, fail with
 * SSD_ERR_UNSUPPORTED before launching. Every call shares that array: calls that
 * overlap on the GPU race, so keep them ordered on one stream. The first call
 * on a device looks up the array's address and should come before any stream
 * capture. Allocates nothing. */
int ssd_linear_noalloc(const void* x, int64_t ldx, int64_t T, int64_t K, int n_seg, const void* const* w,
                       const int64_t* rows, const void* const* bias, int seg_layout, int epilogue, int act, void* out,
                       int64_t ldo, float* resid, int64_t ldr, int dtype, uint32_t* status, void* stream);

/* Fused QKV projection + rotate-half RoPE + KV-cache write:
 * q_out[t] = rope(x[t] @ Wq^T, pos[t]); k/v rows of token t are written to
 * cache slot slots[t] of this layer (k rotated). rope_cos/rope_sin are fp32
 * tables [max_pos, head_dim/2]. Cache layout per layer: [n_kv, max_slots,
 * head_dim] with head stride `cache_head_stride` elements.
 * Replaces q/k/v_proj + RoPE + KVCache.update (subnetwork_draft.py:209-222,
 * ssd/engine/kv_cache.py:32-43). */
int ssd_qkv_rope(const void* x, int64_t ldx, int64_t T, int64_t K, const void* wq, const void* wk, const void* wv,
                 int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, const float* rope_cos, const float* rope_sin,
                 int64_t max_pos, const int32_t* positions, const int32_t* slots, void* k_cache, void* v_cache,
                 int64_t cache_head_stride, int64_t max_slots, void* q_out, int64_t ldq, int dtype, void* workspace,
                 int64_t workspace_bytes, const SsdRowNorm* in_norm, uint32_t* status, void* stream);

/* One GEMM of ssd_linear_chain. With epilogue SSD_EPI_STORE, _RESIDUAL,
 * _SWIGLU or _STORE_F32 the fields mean what the arguments of ssd_linear
 * mean (in_norm.ssq / norm_out.weight NULL: no folding). With SSD_EPI_QKV it
 * is ssd_qkv_rope: w = {wq, wk, wv}, rows and seg_layout are derived from
 * the head counts, out / ldo are q_out / ldq, and the fields after norm_out
 * carry the RoPE tables, positions, cache slots and caches. */
enum { SSD_EPI_QKV = 16 };
typedef struct SsdLinearArgs {
  const void* x;
  int64_t ldx;
  int64_t K;
  int32_t n_seg;
  int32_t seg_layout;
  const void* w[3];
  int64_t rows[3];
  const void* bias[3];
  int32_t epilogue;
  int32_t act;
  void* out;
  int64_t ldo;
  float* resid;
  int64_t ldr;
  SsdRowNorm in_norm;
  SsdNormOut norm_out;
  int64_t n_heads, n_kv_heads, head_dim;
  const float* rope_cos;
  const float* rope_sin;
  int64_t max_pos;
  const int32_t* positions;
  const int32_t* slots;
  void* k_cache;
  void* v_cache;
  int64_t cache_head_stride;
  int64_t max_slots;
} SsdLinearArgs;

/* n (1..6) dependent GEMMs over the same T token rows (bf16, T <= 64) in
 * one persistent launch: link i may read what links < i wrote (its x, the
 * residual, the folded-norm sums), and every link reads only data that the
 * previous kernel in the stream or earlier links wrote. Same results as
 * calling ssd_linear / ssd_qkv_rope for each link in turn, up to the
 * summation order of the K splits (fixed by the weight shapes and the SM
 * count, never by T). For the decode-time layer sequence o_proj -> gate/up
 * -> down -> next layer's q/k/v (subnetwork_draft.py:209-246): the weights
 * of link i + 1 stream into shared memory while link i finishes, which
 * separate launches cannot do. Needs ssd_workspace_bytes(>= T, ...) of
 * workspace; after a status with the timeout bit set, zero the workspace
 * again before the next call. */
int ssd_linear_chain(int32_t n, const SsdLinearArgs* links, int64_t T, int dtype, void* workspace,
                     int64_t workspace_bytes, uint32_t* status, void* stream);

/* Tree attention over the shared cache (split-KV, GQA). Row t attends cache
 * slots [prefix_start[t], prefix_len[t]) (prefix_start NULL: from slot 0;
 * batched decoding gives each sequence its own slot range) and, if spec_mask
 * is given, slot spec_base[0] + j
 * for every set bit j of spec_mask[t * mask_words + j / 64]. Scores use
 * scale = 1/sqrt(head_dim). q: [T, n_heads*head_dim]; out the same.
 * Replaces SDPA with the bool tree mask (subnetwork_draft.py:165-191,
 * 236-242; tree_drafter.py:192-196; ssd/engine/verify.py:37-41). */
int ssd_tree_attention(const void* q, int64_t ldq, int64_t T, int64_t n_heads, int64_t n_kv_heads,
                       int64_t head_dim, const void* k_cache, const void* v_cache, int64_t cache_head_stride,
                       int64_t max_slots, const int32_t* prefix_len, const int32_t* prefix_start,
                       const int32_t* spec_base,
                       const uint64_t* spec_mask, int64_t mask_words, int64_t kv_bound, void* out, int64_t ldo,
                       int dtype, void* workspace, int64_t workspace_bytes, uint32_t* status, void* stream);

/* Verify head: full-vocab lm_head fused with a per-row argmax (first index
 * of the maximum, as torch.argmax). Also writes the top-2 gap per row.
 * Replaces lm_head + argmax (subnetwork_draft.py:349, ssd/engine/verify.py:47,
 * ssd/engine/speculative.py:81-84). */
int ssd_head_argmax(const void* x, int64_t ldx, int64_t T, int64_t K, const void* w, int64_t vocab,
                    int32_t* out_idx, float* out_max, float* out_gap, int dtype, void* workspace,
                    int64_t workspace_bytes, const SsdRowNorm* in_norm, uint32_t* status, void* stream);

/* Draft head: (sub-vocab) lm_head fused with log_softmax + per-row top-k
 * (k <= 16). Column j of W is token vocab_ids[j] (identity if NULL).
 * Outputs tokens [T, k] and fp32 log-probs [T, k], best first.
 * Replaces lm_head/_sub_head + log_softmax().topk() (subnetwork_draft.py:
 * 347-349, tree_drafter.py:128-133). */
int ssd_head_topk(const void* x, int64_t ldx, int64_t T, int64_t K, const void* w, int64_t vocab,
                  const int64_t* vocab_ids, int64_t k, int32_t* out_tok, float* out_logprob, int dtype,
                  void* workspace, int64_t workspace_bytes, const SsdRowNorm* in_norm, uint32_t* status,
                  void* stream);

/* ---------------------------------------------------------------- tree ops
 * The tree lives in device arrays: tokens[i], parents[i] (-1 = root),
 * depths[i] (1..D), ranks[i], scores[i] (fp64 cumulative log-prob) and
 * draft_pos[i]. All tree kernels are single-CTA and deterministic. */

/* One drafting level. The frontier (node indices, -1 for the root) proposes
 * k children each from topk_tok / topk_lp [n_frontier, k] (tokens < 0 or
 * -inf log-probs are missing candidates). Candidates are ordered by
 * descending cumulative score (fp64, ties keep frontier order then rank) and
 * the first `width` (all if width <= 0) are appended at index *n_nodes
 * (at index 0 for level 0, which starts a new tree), which is advanced;
 * their indices go to next_frontier. If `fed`, the level
 * is the input of the next draft forward and its ids / positions
 * (root_pos + level + 1) / cache slots (root_pos + 1 + level_slot_offset + j)
 * / prefix length (root_pos + 1) / ancestor bitmask over spec slots starting
 * at root_pos + 1 are written to the fwd_* buffers.
 * Replaces TreeDrafter.build's level step (tree_drafter.py:165-200). */
int ssd_level_prune(const int32_t* topk_tok, const float* topk_lp, int64_t n_frontier, int64_t k, int64_t width,
                    int64_t level, const int32_t* frontier, int32_t* next_frontier, int32_t* n_nodes,
                    int32_t* tokens, int32_t* parents, int32_t* depths, int32_t* ranks, double* scores,
                    int32_t* draft_pos, int64_t cap, const int32_t* root_pos, int fed, int64_t level_slot_offset,
                    int32_t* fwd_ids, int32_t* fwd_pos, int32_t* fwd_slots, int32_t* fwd_plen,
                    int32_t* fwd_spec_base, uint64_t* fwd_mask, int64_t mask_words, uint32_t* status,
                    void* stream);

/* Final max_nodes pruning: keep the best max_nodes nodes by (-score, depth),
 * close the set under ancestors and compact it in index order with parents
 * remapped (max_nodes <= 0: only drop empty slots). *n_nodes is updated.
 * Replaces tree_drafter.py:202-207 and DraftTree.subset (:80-95). */
int ssd_tree_prune(int32_t* n_nodes, int64_t max_nodes, int32_t* tokens, int32_t* parents, int32_t* depths,
                   int32_t* ranks, double* scores, int32_t* draft_pos, int64_t cap, void* stream);

/* Verify inputs for root + tree over rows_cap static rows: ids, positions
 * root_pos + depth, cache slots root_pos + row, prefix length root_pos + 1
 * and each node row's ancestor bitmask (bit i = node i at slot
 * root_pos + 1 + i); rows past the tree are inert padding.
 * Replaces verify_inputs (ssd/engine/verify.py:32-42). */
int ssd_verify_prep(const int32_t* n_nodes, int64_t rows_cap, const int32_t* root_token, const int32_t* root_pos,
                    const int32_t* tokens, const int32_t* parents, const int32_t* depths, int32_t* ids,
                    int32_t* positions, int32_t* slots, int32_t* prefix_len, int32_t* spec_base, uint64_t* mask,
                    int64_t mask_words, uint32_t* status, void* stream);

/* Greedy tree walk: from the root follow the child (lowest rank first) whose
 * token equals the row's argmax; the argmax at the last accepted node is the
 * bonus token. Writes accepted node indices, their count, the bonus and the
 * compaction source slots [root_pos, root_pos + 1 + a0, ...] (n_keep = 1 +
 * accepted). Replaces greedy_verify (ssd/engine/verify.py:45-57) and the
 * position list of ssd/engine/speculative.py:167. */
int ssd_tree_walk_greedy(const int32_t* n_nodes, int64_t max_nodes, const int32_t* argmax, const int32_t* tokens,
                         const int32_t* parents, const int32_t* ranks, const int32_t* root_pos, int32_t* accepted,
                         int32_t* n_accepted, int32_t* bonus, int32_t* keep_slots, int32_t* n_keep, void* stream);

/* In-place KV compaction over every layer: for j < *n_keep, cache slot
 * keep_slots[j] moves to slot start[0] + j. Each thread owns one 16-byte
 * group of one (layer, K/V, head) row across all kept slots and reads them
 * all before writing, so overlapping source/destination slots are safe.
 * A keep list longer than max_keep or naming a slot outside the cache copies
 * nothing and sets status bit 2 (bad index), if `status` is given.
 * Strides are in elements. Replaces KVCache.keep_positions
 * (ssd/engine/kv_cache.py:54-70). */
int ssd_kv_compact(void* cache, int64_t n_layers, int64_t layer_stride, int64_t kv_stride, int64_t n_kv_heads,
                   int64_t head_stride, int64_t head_dim, const int32_t* start, const int32_t* keep_slots,
                   const int32_t* n_keep, int64_t max_keep, int dtype, uint32_t* status, void* stream);

/* Commit one round: append the accepted tokens + bonus to out_tokens at
 * *n_out, advance *seq_len by 1 + accepted, make the bonus the new root and
 * log the committed count in round_log (round_log[0] = rounds so far).
 * Replaces the bookkeeping of ssd/engine/speculative.py:167-172. */
int ssd_round_commit(const int32_t* n_accepted, const int32_t* accepted, const int32_t* tokens,
                     const int32_t* bonus, int32_t* seq_len, int32_t* root_token, int32_t* out_tokens,
                     int32_t* n_out, int64_t out_cap, int32_t* round_log, uint32_t* status, void* stream);

/* Causal forward inputs for T rows starting at cache length *base: positions
 * and cache slots base + r, prefix length base + r + 1; ids copied from
 * src_ids if given. Replaces the default position_ids / causal mask of
 * subnetwork_draft.py:296-297,179-191. */
int ssd_causal_prep(const int32_t* base, int64_t T, const int32_t* src_ids, int32_t* ids, int32_t* positions,
                    int32_t* slots, int32_t* prefix_len, void* stream);

/* ------------------------------------------------------------- sampling
 * warp(logits) = softmax(logits / temperature) restricted to the top-p
 * nucleus (smallest prefix of the descending order with mass >= top_p),
 * renormalised, as warp_probs (ssd/engine/tree_drafter.py:34-45). A row's
 * warp is summarised by 16-byte parameters {max, 1/T, lambda, log Z}; the
 * nucleus threshold lambda is found by a deterministic radix select. Random
 * numbers are Philox4x32-10 keyed by *seed with counter (round, row, i, stream). */

/* Warp parameters of `rows` logit rows [rows, ld] (fp32) into params_out. */
int ssd_warp_params(const float* logits, int64_t ld, int64_t rows, int64_t V, float temperature, float top_p,
                    void* params_out, void* stream);

/* Warped probabilities of rows [rows, ld] into out [rows, ldo] (fp32) from
 * their warp parameters; zero outside the nucleus. */
int ssd_warp_probs(const float* logits, int64_t ld, int64_t rows, int64_t V, const void* params, float* out,
                   int64_t ldo, void* stream);

/* Per row: k tokens drawn without replacement from the warped distribution
 * (Gumbel top-k, in draw order) and their warped log-probs; fewer than k
 * kept tokens leave token -1 / log-prob -inf. Row r uses RNG row id
 * row_base + r. Replaces the sampling branch of TreeDrafter._propose
 * (tree_drafter.py:134-145). */
int ssd_gumbel_topk(const float* logits, int64_t ld, int64_t rows, int64_t V, const void* params, int64_t k,
                    const int64_t* vocab_ids, const uint64_t* seed, const int32_t* round, int64_t row_base,
                    int32_t* out_tok, float* out_logprob, void* stream);

/* Fused ssd_warp_params + ssd_gumbel_topk: each row is split over a
 * thread-block cluster of up to 8 CTAs (slices staged in shared memory,
 * reductions combined in rank order; fewer CTAs per row when that keeps all
 * rows' clusters resident at once). Writes the rows' warp parameters to
 * params_out (may be NULL when k > 0) and, for k >= 1, the same draws as
 * ssd_gumbel_topk with those parameters (RNG counters (round, row_base + r,
 * i, 0)); out_logprob may be NULL. k = 0 computes the parameters only.
 * keep_top > 0 first restricts each row to its keep_top largest logits (ties
 * at the boundary kept), then applies temperature and top_p within them, as
 * sample_next does for batched generation (ssd/data/generate_selfdistill.py:
 * 51-61, keep_top = 64); 0 = the full row. V <= 131072. Replaces the sampling
 * branch of TreeDrafter._propose (tree_drafter.py:134-145) and warp_probs
 * (:34-45) for the verify rows. */
int ssd_warp_sample_topk(const float* logits, int64_t ld, int64_t rows, int64_t V, float temperature, float top_p,
                         int64_t keep_top, int64_t k, const int64_t* vocab_ids, const uint64_t* seed,
                         const int32_t* round, int64_t row_base, void* params_out, int32_t* out_tok,
                         float* out_logprob, void* stream);

/* One token drawn from warp(logits[0..V)) into out[0]: a Gumbel-max draw on
 * one cluster (RNG counters (round, row_id, i, stream_id)); rows longer than
 * 131072 use one CTA and an inverse-CDF draw over `scratch` (V floats, may be
 * NULL otherwise). Replaces _first_token's sampling branch
 * (ssd/engine/speculative.py:81-84). */
int ssd_sample_token(const float* logits, int64_t V, float temperature, float top_p, const uint64_t* seed,
                     const int32_t* round, int64_t row_id, int64_t stream_id, float* scratch, int32_t* out,
                     void* stream);

/* Multi-candidate speculative sampling without replacement over the device
 * tree: at each node p = warp(target row), children in rank order accepted
 * with prob min(1, p(x)/q(x)); on rejection p <- norm(max(p - q, 0)) (if it
 * has mass), q(x) <- 0 renormalised; when every child is rejected the bonus
 * is drawn from p. q of a node's children = warp(draft logits row 0 for the
 * root, row draft_pos - root_pos for a fed node) over the draft vocabulary
 * (vocab_ids, NULL = the first Vd ids). target_params / draft_params are
 * ssd_warp_params of the target rows [rows, ldt] and the draft_rows draft
 * rows [draft_rows, ldd]. Runs on one cluster of up to 8 CTAs that keep
 * their vocabulary slices of p and q in shared memory; the bonus is a
 * Gumbel-max draw from p (counters (round, cur + 1, i, 2)). p_scratch /
 * q_scratch (V floats each) are used only for V > 131072 (one CTA) and may be
 * NULL otherwise. Outputs as ssd_tree_walk_greedy. Replaces sample_verify
 * (ssd/engine/verify.py:60-95). */
int ssd_tree_walk_sample(const int32_t* n_nodes, int64_t max_nodes, const int32_t* tokens, const int32_t* parents,
                         const int32_t* ranks, const int32_t* draft_pos, const int32_t* root_pos,
                         const float* target_logits, int64_t ldt, const void* target_params, int64_t V,
                         const float* draft_logits, int64_t ldd, const void* draft_params, int64_t draft_rows,
                         int64_t Vd, const int64_t* vocab_ids, const uint64_t* seed, const int32_t* round,
                         float* p_scratch, float* q_scratch, int32_t* accepted, int32_t* n_accepted, int32_t* bonus,
                         int32_t* keep_slots, int32_t* n_keep, uint32_t* status, void* stream);


/* ------------------------------------------------------- tensor parallel
 * The 70B configuration runs tensor-parallel over `world` GPUs, one process
 * per GPU: q/k/v and gate/up split by output features (heads, FFN columns),
 * o_proj and down_proj by input features, the lm_head by vocabulary rows, the
 * KV cache by KV head; embedding, norms and bridges replicated. Ranks exchange
 * data through a "region": a device buffer of ssd_tp_region_bytes bytes with
 * the same layout on every rank, zeroed once, each rank's region mapped into
 * every rank's address space (peer pointers over NVLink; the host sets the
 * mapping up, e.g. with torch symmetric memory). Kernels meet their
 * counterparts on the other ranks through flags in the regions; every wait is
 * bounded (timeout: status bit 1). Every rank must issue the same sequence of
 * these calls with the same sizes. No multicast is used. (The reference runs
 * on one device and has no tensor-parallel code.) */
#define SSD_TP_MAX_RANKS 8
typedef struct SsdTpGroup {
  int32_t rank;
  int32_t world;
  int64_t max_rows; /* token rows the region's exchange buffers hold */
  int64_t d;        /* model width (the all-reduced row length) */
  void* peer_region[SSD_TP_MAX_RANKS]; /* region of rank r as mapped in this process */
} SsdTpGroup;

int64_t ssd_tp_region_bytes(int64_t max_rows, int64_t d);
/* Polls a tensor-parallel meeting makes before it gives up, sets status bit 1
 * (timeout) and lets the kernel finish; 0 restores the default (2^22 polls,
 * about half a second). Applies to calls issued after it; returns the previous
 * limit. A lower limit lets a caller detect a rank that never arrives sooner. */
uint32_t ssd_tp_set_spin_limit(uint32_t polls);
/* Byte offset in the region of partial buffer `parity` (0 or 1), fp32
 * [max_rows, d] with row stride d: the row-parallel o_proj / down_proj GEMM
 * (ssd_linear with SSD_EPI_STORE_F32) writes this rank's partial sums there. */
int64_t ssd_tp_partial_offset(int64_t max_rows, int64_t d, int parity);

/* resid[t, :] += sum over ranks (in rank order) of the ranks' partials
 * [T, d] in buffer `parity`; with norm_out also the next RMSNorm's folded
 * input, as ssd_linear's residual epilogue (bit-identical to it when
 * world == 1). One-shot over peer memory: each rank reads the other ranks'
 * partials over NVLink after one meeting of the ranks. Consecutive calls must
 * alternate parity (a rank overwrites a partial buffer only two calls later,
 * when every rank has finished reading it). This is the all-reduce after
 * o_proj / down_proj (_layer_forward, ssd/models/subnetwork_draft.py:243,245)
 * of a tensor-parallel layer, fused with the residual add. dtype: of norm_out. */
int ssd_tp_allreduce_residual(const SsdTpGroup* group, int parity, int64_t T, float* resid, int64_t ldr,
                              const SsdNormOut* norm_out, int dtype, uint32_t* status, void* stream);

/* Vocabulary-parallel heads. w: this rank's lm_head rows [vocab_offset,
 * vocab_offset + vocab_shard) as [vocab_shard, K]. Each rank reduces its rows,
 * the per-row results of all ranks are merged through the regions, and every
 * rank receives the global outputs of ssd_head_argmax (lowest global index on
 * ties) / ssd_head_topk (log-softmax over all ranks' rows; vocab_ids maps
 * global row indices to tokens, NULL = identity). T <= max_rows. */
int ssd_tp_head_argmax(const SsdTpGroup* group, const void* x, int64_t ldx, int64_t T, int64_t K, const void* w,
                       int64_t vocab_shard, int64_t vocab_offset, int32_t* out_idx, float* out_max, float* out_gap,
                       int dtype, void* workspace, int64_t workspace_bytes, const SsdRowNorm* in_norm,
                       uint32_t* status, void* stream);
int ssd_tp_head_topk(const SsdTpGroup* group, const void* x, int64_t ldx, int64_t T, int64_t K, const void* w,
                     int64_t vocab_shard, int64_t vocab_offset, const int64_t* vocab_ids, int64_t k, int32_t* out_tok,
                     float* out_logprob, int dtype, void* workspace, int64_t workspace_bytes,
                     const SsdRowNorm* in_norm, uint32_t* status, void* stream);

/* Seeded synthetic weights: out[i, j] = scale * std * N(0, 1) for the block
 * [row0, row0 + rows) x [col0, col0 + cols) of a global matrix with full_cols
 * columns; element (gi, gj) depends only on (seed, stream_id,
 * gi * full_cols + gj) (Philox4x32-10, Box-Muller), so a tensor-parallel
 * shard of a global matrix is generated on its own rank. out: [rows, ld]. */
int ssd_fill_normal(void* out, int64_t rows, int64_t cols, int64_t ld, int64_t row0, int64_t col0, int64_t full_cols,
                    uint64_t seed, uint64_t stream_id, float std, float scale, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SSD_B200_H */
