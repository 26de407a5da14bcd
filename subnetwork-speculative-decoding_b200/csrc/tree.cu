// Device-resident draft tree and the small single-CTA kernels that build,
// prune, verify and commit it, plus the in-place KV compaction.
//
// Tree arrays (capacity `cap` nodes): tokens, parents (-1 = root, -2 = empty
// slot of a level that had fewer candidates than its static size), depths
// (1..D), ranks (proposal order among siblings), scores (fp64 cumulative
// draft log-prob, as the reference's Python floats) and draft_pos (cache slot
// the node's draft K/V went to, -1 if the node was never fed).
#include "common.cuh"
#include "host.cuh"

namespace ssd {

constexpr int kRoot = -1;
constexpr int kEmpty = -2;

// Stable descending-score order: a precedes b iff score_a > score_b, or the
// scores are equal and a was proposed first. NaN-free inputs assumed.
__device__ __forceinline__ bool cand_before(double sa, int ia, double sb, int ib) {
  return sa > sb || (sa == sb && ia < ib);
}

__global__ void level_prune_kernel(const int32_t* topk_tok, const float* topk_lp, int n_frontier, int k, int keep,
                                   int level, const int32_t* frontier, int32_t* next_frontier, int32_t* n_nodes,
                                   int32_t* tokens, int32_t* parents, int32_t* depths, int32_t* ranks, double* scores,
                                   int32_t* draft_pos, int cap, const int32_t* root_pos, int fed,
                                   int level_slot_offset, int32_t* fwd_ids, int32_t* fwd_pos, int32_t* fwd_slots,
                                   int32_t* fwd_plen, int32_t* fwd_spec_base, uint64_t* fwd_mask, int mask_words,
                                   uint32_t* status) {
  extern __shared__ uint8_t sm_raw[];
  const int n = n_frontier * k;
  double* s_score = reinterpret_cast<double*>(sm_raw);
  int* s_par = reinterpret_cast<int*>(s_score + n);
  int* s_rank = s_par + n;  // position in the sorted order
  __shared__ int s_base;
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) s_base = level == 0 ? 0 : *n_nodes;  // level 0 starts a new tree
  __syncthreads();
  const int base = s_base;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int j = i / k;
    const int par = frontier[j];
    const bool par_ok = (par == kRoot) || (par >= 0 && par < cap && parents[par] != kEmpty);
    const int tok = topk_tok[(int64_t)j * k + (i % k)];
    const float lp = topk_lp[(int64_t)j * k + (i % k)];
    const bool ok = par_ok && tok >= 0 && lp != -INFINITY;
    const double pb = (par == kRoot || !par_ok) ? 0.0 : scores[par];
    s_score[i] = ok ? pb + (double)lp : -INFINITY;
    s_par[i] = ok ? par : kEmpty;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int r = 0;
    const double si = s_score[i];
    for (int j = 0; j < n; ++j) r += cand_before(s_score[j], j, si, i) ? 1 : 0;
    s_rank[i] = r;
  }
  __syncthreads();
  const int c = root_pos[0];
  const int tree_start = c + 1;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int q = s_rank[i];
    if (q >= keep) continue;
    const int node = base + q;
    if (node >= cap) {
      report_error(status, kErrBadIndex);
      continue;
    }
    const bool ok = s_par[i] != kEmpty;
    tokens[node] = ok ? topk_tok[(int64_t)(i / k) * k + (i % k)] : -1;
    parents[node] = s_par[i];
    depths[node] = level + 1;
    ranks[node] = i % k;
    scores[node] = s_score[i];
    draft_pos[node] = fed ? tree_start + level_slot_offset + q : -1;
    next_frontier[q] = node;
  }
  __syncthreads();
  if (threadIdx.x == 0) *n_nodes = min(base + keep, cap);
  if (!fed) return;
  __threadfence_block();
  __syncthreads();
  // Inputs of the draft forward over this level.
  for (int q = threadIdx.x; q < keep; q += blockDim.x) {
    const int node = base + q;
    const bool ok = parents[node] != kEmpty;
    fwd_ids[q] = ok ? tokens[node] : 0;
    fwd_pos[q] = c + level + 1;
    fwd_slots[q] = tree_start + level_slot_offset + q;
    fwd_plen[q] = tree_start;
    for (int w = 0; w < mask_words; ++w) fwd_mask[(int64_t)q * mask_words + w] = 0ull;
    // self and ancestors (all fed), by draft slot relative to tree_start
    int a = node;
    int guard = 0;
    while (a >= 0 && guard++ < 64) {
      const int bit = draft_pos[a] - tree_start;
      if (bit >= 0 && bit < mask_words * 64) fwd_mask[(int64_t)q * mask_words + (bit >> 6)] |= 1ull << (bit & 63);
      else report_error(status, kErrBadIndex);
      a = parents[a];
    }
  }
  if (threadIdx.x == 0) fwd_spec_base[0] = tree_start;
}

// Best max_nodes by (-score, depth, index), closed under ancestors, compacted
// in index order with parents remapped.
__global__ void tree_prune_kernel(int32_t* n_nodes, int max_nodes, int32_t* tokens, int32_t* parents,
                                  int32_t* depths, int32_t* ranks, double* scores, int32_t* draft_pos, int cap) {
  extern __shared__ uint8_t sm_raw[];
  double* s_score = reinterpret_cast<double*>(sm_raw);
  int* s_tok = reinterpret_cast<int*>(s_score + cap);
  int* s_par = s_tok + cap;
  int* s_dep = s_par + cap;
  int* s_rank = s_dep + cap;
  int* s_dpos = s_rank + cap;
  int* s_keep = s_dpos + cap;
  int* s_new = s_keep + cap;
  pdl_wait();
  pdl_trigger();
  const int n = min(*n_nodes, cap);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    s_score[i] = scores[i];
    s_tok[i] = tokens[i];
    s_par[i] = parents[i];
    s_dep[i] = depths[i];
    s_rank[i] = ranks[i];
    s_dpos[i] = draft_pos[i];
  }
  __syncthreads();
  __shared__ int s_valid;
  if (threadIdx.x == 0) {
    int v = 0;
    for (int i = 0; i < n; ++i) v += (s_par[i] != kEmpty);
    s_valid = v;
  }
  __syncthreads();
  const bool prune = max_nodes > 0 && s_valid > max_nodes;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    int keep = s_par[i] != kEmpty;
    if (keep && prune) {
      int r = 0;
      for (int j = 0; j < n; ++j) {
        if (s_par[j] == kEmpty) continue;
        const bool before = s_score[j] > s_score[i] ||
                            (s_score[j] == s_score[i] && (s_dep[j] < s_dep[i] || (s_dep[j] == s_dep[i] && j < i)));
        r += before;
      }
      keep = r < max_nodes;
    }
    s_keep[i] = keep;
  }
  __syncthreads();
  // ancestor closure (parents precede children, so one pass in reverse index
  // order suffices; done serially by one thread: n is small)
  if (threadIdx.x == 0) {
    for (int i = n - 1; i >= 0; --i)
      if (s_keep[i] && s_par[i] >= 0) s_keep[s_par[i]] = 1;
    int m = 0;
    for (int i = 0; i < n; ++i) s_new[i] = s_keep[i] ? m++ : -1;
    *n_nodes = m;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (!s_keep[i]) continue;
    const int o = s_new[i];
    tokens[o] = s_tok[i];
    parents[o] = s_par[i] >= 0 ? s_new[s_par[i]] : kRoot;
    depths[o] = s_dep[i];
    ranks[o] = s_rank[i];
    scores[o] = s_score[i];
    draft_pos[o] = s_dpos[i];
  }
}

__global__ void verify_prep_kernel(const int32_t* n_nodes, int rows_cap, const int32_t* root_token,
                                   const int32_t* root_pos, const int32_t* tokens, const int32_t* parents,
                                   const int32_t* depths, int32_t* ids, int32_t* positions, int32_t* slots,
                                   int32_t* prefix_len, int32_t* spec_base, uint64_t* mask, int mask_words,
                                   uint32_t* status) {
  pdl_wait();
  pdl_trigger();
  int n = *n_nodes;
  const int c = root_pos[0];
  if (n + 1 > rows_cap) {
    if (threadIdx.x == 0) report_error(status, kErrBadIndex);
    n = rows_cap - 1;
  }
  for (int r = threadIdx.x; r < rows_cap; r += blockDim.x) {
    const int i = r - 1;
    const bool node = r > 0 && i < n;
    ids[r] = (r == 0) ? root_token[0] : (node ? max(tokens[i], 0) : 0);
    positions[r] = c + (node ? depths[i] : 0);
    slots[r] = c + r;
    prefix_len[r] = c + 1;
    for (int w = 0; w < mask_words; ++w) mask[(int64_t)r * mask_words + w] = 0ull;
    if (node) {
      int a = i, guard = 0;
      while (a >= 0 && guard++ < 256) {
        if (a < mask_words * 64) mask[(int64_t)r * mask_words + (a >> 6)] |= 1ull << (a & 63);
        else report_error(status, kErrBadIndex);
        a = parents[a];
      }
    }
  }
  if (threadIdx.x == 0) spec_base[0] = c + 1;
}

__global__ void tree_walk_greedy_kernel(const int32_t* n_nodes, int max_n, const int32_t* argmax,
                                        const int32_t* tokens, const int32_t* parents, const int32_t* ranks,
                                        const int32_t* root_pos, int32_t* accepted, int32_t* n_accepted,
                                        int32_t* bonus, int32_t* keep_slots, int32_t* n_keep) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0) return;
  const int n = min(*n_nodes, max_n);
  const int c = root_pos[0];
  int cur = kRoot, na = 0;
  keep_slots[0] = c;
  for (int step = 0; step <= n; ++step) {
    const int want = argmax[cur + 1];
    int best = -1, best_rank = INT32_MAX;
    for (int i = 0; i < n; ++i)
      if (parents[i] == cur && tokens[i] == want && ranks[i] < best_rank) {
        best = i;
        best_rank = ranks[i];
      }
    if (best < 0) {
      *bonus = want;
      break;
    }
    accepted[na] = best;
    keep_slots[1 + na] = c + 1 + best;
    ++na;
    cur = best;
  }
  *n_accepted = na;
  *n_keep = na + 1;
}

// One thread per (layer, K/V, head, 16-byte group of head_dim): read every
// kept slot first, then write, so overlapping source/destination slots of the
// same slice can never be clobbered. A keep list that does not fit (more than
// max_keep entries, or a slot outside the cache) copies nothing and sets the
// status word's bad-index bit, which the host turns into an error.
template <typename VEC>
__global__ void kv_compact_kernel(uint8_t* cache, int64_t n_layers, int64_t layer_stride_b, int64_t kv_stride_b,
                                  int64_t n_kv, int64_t head_stride_b, int64_t row_bytes, const int32_t* start,
                                  const int32_t* keep_slots, const int32_t* n_keep, int max_keep, uint32_t* status) {
  constexpr int kMaxKeep = 32;
  pdl_wait();
  pdl_trigger();
  const int64_t groups = row_bytes / (int64_t)sizeof(VEC);
  const int64_t total = n_layers * 2 * n_kv * groups;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (tid >= total) return;
  const int nk_req = *n_keep;
  const int nk = min(min(nk_req, max_keep), kMaxKeep);
  const int s0 = start[0];
  const int64_t n_slots = head_stride_b / row_bytes;
  bool bad = nk_req < 0 || nk_req > max_keep || s0 < 0 || s0 + nk > n_slots;
  for (int j = 0; j < nk && !bad; ++j) bad = keep_slots[j] < 0 || keep_slots[j] >= n_slots;
  if (bad) {
    if (tid == 0) report_error(status, kErrBadIndex);
    return;
  }
  const int64_t g = tid % groups;
  const int64_t h = (tid / groups) % n_kv;
  const int64_t kv = (tid / (groups * n_kv)) % 2;
  const int64_t l = tid / (groups * n_kv * 2);
  uint8_t* base = cache + l * layer_stride_b + kv * kv_stride_b + h * head_stride_b + g * (int64_t)sizeof(VEC);
  VEC buf[kMaxKeep];
#pragma unroll
  for (int j = 0; j < kMaxKeep; ++j)
    if (j < nk) buf[j] = *reinterpret_cast<const VEC*>(base + (int64_t)keep_slots[j] * row_bytes);
#pragma unroll
  for (int j = 0; j < kMaxKeep; ++j)
    if (j < nk && keep_slots[j] != s0 + j) *reinterpret_cast<VEC*>(base + (int64_t)(s0 + j) * row_bytes) = buf[j];
}

__global__ void round_commit_kernel(const int32_t* n_accepted, const int32_t* accepted, const int32_t* tokens,
                                    const int32_t* bonus, int32_t* seq_len, int32_t* root_token, int32_t* out_tokens,
                                    int32_t* n_out, int out_cap, int32_t* round_log, uint32_t* status) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x != 0) return;
  const int na = *n_accepted;
  int o = *n_out;
  for (int j = 0; j < na; ++j) {
    if (o < out_cap) out_tokens[o] = tokens[accepted[j]];
    else report_error(status, kErrBadIndex);
    ++o;
  }
  if (o < out_cap) out_tokens[o] = *bonus;
  else report_error(status, kErrBadIndex);
  ++o;
  if (round_log) {
    // round_log[0] = number of rounds; then one entry per round
    const int r = round_log[0];
    round_log[1 + r] = na + 1;
    round_log[0] = r + 1;
  }
  *n_out = o;
  *seq_len = *seq_len + 1 + na;
  *root_token = *bonus;
}

// positions/slots = base + r, prefix = base + r + 1 (causal rows); ids from
// `src_ids` (device) when given.
__global__ void causal_prep_kernel(const int32_t* base, int T, const int32_t* src_ids, int32_t* ids,
                                   int32_t* positions, int32_t* slots, int32_t* prefix_len) {
  pdl_wait();
  pdl_trigger();
  const int b = base[0];
  for (int r = threadIdx.x + blockIdx.x * blockDim.x; r < T; r += blockDim.x * gridDim.x) {
    if (src_ids) ids[r] = src_ids[r];
    positions[r] = b + r;
    slots[r] = b + r;
    prefix_len[r] = b + r + 1;
  }
}

}  // namespace ssd

using namespace ssd;

extern "C" {

int ssd_level_prune(const int32_t* topk_tok, const float* topk_lp, int64_t n_frontier, int64_t k, int64_t width,
                    int64_t level, const int32_t* frontier, int32_t* next_frontier, int32_t* n_nodes,
                    int32_t* tokens, int32_t* parents, int32_t* depths, int32_t* ranks, double* scores,
                    int32_t* draft_pos, int64_t cap, const int32_t* root_pos, int fed, int64_t level_slot_offset,
                    int32_t* fwd_ids, int32_t* fwd_pos, int32_t* fwd_slots, int32_t* fwd_plen,
                    int32_t* fwd_spec_base, uint64_t* fwd_mask, int64_t mask_words, uint32_t* status,
                    void* stream) {
  const int64_t n = n_frontier * k;
  if (n_frontier <= 0 || k <= 0 || n > 4096) return fail(SSD_ERR_INVALID, "ssd_level_prune: bad candidate count");
  const int64_t keep = (width > 0 && width < n) ? width : n;
  if (fed && (!fwd_ids || !fwd_pos || !fwd_slots || !fwd_plen || !fwd_spec_base || !fwd_mask || mask_words <= 0))
    return fail(SSD_ERR_INVALID, "ssd_level_prune: fed level needs forward buffers");
  if (fed && level_slot_offset + keep > mask_words * 64)
    return fail(SSD_ERR_UNSUPPORTED, "ssd_level_prune: tree slots exceed the ancestor mask");
  const size_t smem = (size_t)n * (8 + 4 + 4);
  return launch_kernel("level_prune_kernel", level_prune_kernel, dim3(1), dim3(256), smem,
      static_cast<cudaStream_t>(stream), 1, 1, topk_tok, topk_lp, (int)n_frontier, (int)k, (int)keep, (int)level, frontier, next_frontier, n_nodes, tokens,
      parents, depths, ranks, scores, draft_pos, (int)cap, root_pos, fed, (int)level_slot_offset, fwd_ids, fwd_pos,
      fwd_slots, fwd_plen, fwd_spec_base, fwd_mask, (int)mask_words, status);
}

int ssd_tree_prune(int32_t* n_nodes, int64_t max_nodes, int32_t* tokens, int32_t* parents, int32_t* depths,
                   int32_t* ranks, double* scores, int32_t* draft_pos, int64_t cap, void* stream) {
  if (cap <= 0 || cap > 4096) return fail(SSD_ERR_INVALID, "ssd_tree_prune: bad capacity");
  const size_t smem = (size_t)cap * (8 + 7 * 4);
  return launch_kernel("tree_prune_kernel", tree_prune_kernel, dim3(1), dim3(256), smem,
                       static_cast<cudaStream_t>(stream), 1, 1, n_nodes, (int)max_nodes, tokens, parents, depths,
                       ranks, scores, draft_pos, (int)cap);
}

int ssd_verify_prep(const int32_t* n_nodes, int64_t rows_cap, const int32_t* root_token, const int32_t* root_pos,
                    const int32_t* tokens, const int32_t* parents, const int32_t* depths, int32_t* ids,
                    int32_t* positions, int32_t* slots, int32_t* prefix_len, int32_t* spec_base, uint64_t* mask,
                    int64_t mask_words, uint32_t* status, void* stream) {
  if (rows_cap <= 0 || mask_words <= 0 || rows_cap - 1 > mask_words * 64)
    return fail(SSD_ERR_INVALID, "ssd_verify_prep: rows exceed the ancestor mask");
  return launch_kernel("verify_prep_kernel", verify_prep_kernel, dim3(1), dim3(256), 0,
      static_cast<cudaStream_t>(stream), 1, 1, n_nodes, (int)rows_cap, root_token, root_pos, tokens, parents, depths, ids, positions, slots, prefix_len,
      spec_base, mask, (int)mask_words, status);
}

int ssd_tree_walk_greedy(const int32_t* n_nodes, int64_t max_nodes, const int32_t* argmax, const int32_t* tokens,
                         const int32_t* parents, const int32_t* ranks, const int32_t* root_pos, int32_t* accepted,
                         int32_t* n_accepted, int32_t* bonus, int32_t* keep_slots, int32_t* n_keep, void* stream) {
  if (max_nodes < 0 || max_nodes > 4096) return fail(SSD_ERR_INVALID, "ssd_tree_walk_greedy: bad max_nodes");
  return launch_kernel("tree_walk_greedy_kernel", tree_walk_greedy_kernel, dim3(1), dim3(32), 0,
      static_cast<cudaStream_t>(stream), 1, 1, n_nodes, (int)max_nodes, argmax, tokens, parents, ranks, root_pos, accepted, n_accepted, bonus, keep_slots,
      n_keep);
}

int ssd_kv_compact(void* cache, int64_t n_layers, int64_t layer_stride, int64_t kv_stride, int64_t n_kv_heads,
                   int64_t head_stride, int64_t head_dim, const int32_t* start, const int32_t* keep_slots,
                   const int32_t* n_keep, int64_t max_keep, int dtype, uint32_t* status, void* stream) {
  if (max_keep <= 0 || max_keep > 32) return fail(SSD_ERR_UNSUPPORTED, "ssd_kv_compact: max_keep must be 1..32");
  const int64_t es = dtype == SSD_F32 ? 4 : 2;
  const int64_t row_bytes = head_dim * es;
  if (row_bytes % 16) return fail(SSD_ERR_UNSUPPORTED, "ssd_kv_compact: head_dim * elem must be a multiple of 16 B");
  const int64_t groups = row_bytes / 16;
  const int64_t total = n_layers * 2 * n_kv_heads * groups;
  const unsigned blocks = (unsigned)((total + 255) / 256);
  return launch_kernel("kv_compact_kernel", kv_compact_kernel<uint4>, dim3(blocks), dim3(256), 0,
      static_cast<cudaStream_t>(stream), 1, 1, static_cast<uint8_t*>(cache), n_layers, layer_stride * es, kv_stride * es, n_kv_heads, head_stride * es,
      row_bytes, start, keep_slots, n_keep, (int)max_keep, status);
}

int ssd_round_commit(const int32_t* n_accepted, const int32_t* accepted, const int32_t* tokens,
                     const int32_t* bonus, int32_t* seq_len, int32_t* root_token, int32_t* out_tokens,
                     int32_t* n_out, int64_t out_cap, int32_t* round_log, uint32_t* status, void* stream) {
  return launch_kernel("round_commit_kernel", round_commit_kernel, dim3(1), dim3(32), 0,
      static_cast<cudaStream_t>(stream), 1, 1, n_accepted, accepted, tokens, bonus, seq_len, root_token, out_tokens, n_out, (int)out_cap, round_log, status);
}

int ssd_causal_prep(const int32_t* base, int64_t T, const int32_t* src_ids, int32_t* ids, int32_t* positions,
                    int32_t* slots, int32_t* prefix_len, void* stream) {
  if (T <= 0) return fail(SSD_ERR_INVALID, "ssd_causal_prep: T must be positive");
  const unsigned blocks = (unsigned)((T + 255) / 256 > 64 ? 64 : (T + 255) / 256);
  return launch_kernel("causal_prep_kernel", causal_prep_kernel, dim3(blocks), dim3(256), 0,
                       static_cast<cudaStream_t>(stream), 1, 1, base, (int)T, src_ids, ids, positions, slots,
                       prefix_len);
}

}  // extern "C"
