// Sampling (temperature > 0): warped distributions, Gumbel top-k drafting and
// multi-candidate speculative sampling without replacement.
//
// warp(logits) = softmax(logits / T) restricted to the nucleus: sort the
// probabilities in descending order and keep the smallest prefix whose mass
// reaches top_p (an element is dropped when the mass strictly before it
// exceeds top_p), renormalised. Each row's warp is summarised by parameters
// {m, 1/T, lambda, log Z}: token i has log-prob (l_i - m)/T - log Z if
// l_i >= lambda, else probability 0. lambda is found without sorting by a
// 4-level radix select over the order-preserving bits of the logits, summing
// probability mass in 2^-48 fixed point with integer atomics, so the result
// does not depend on thread scheduling. All other reductions use a fixed
// per-thread partition and a fixed combine order (deterministic).
//
// Random numbers: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC 2011), keyed by the caller's seed, with
// counter (round, row, index, stream); no state is kept between launches.
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "host.cuh"

namespace ssd {

constexpr int kSampThreads = 1024;
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kMaxK = 16;

struct WarpParams {
  float m;       // row max logit
  float inv_t;   // 1 / temperature
  float lambda;  // smallest kept logit
  float log_z;   // log of the kept mass normaliser (relative to exp((l - m) / T))
};

__device__ __forceinline__ float uniform(uint64_t seed, uint32_t round, uint32_t row, uint32_t idx, uint32_t stream) {
  const uint4 r = philox4x32_10(make_uint4(round, row, idx, stream),
                                make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32)));
  return u01(r.x);
}

// ------------------------------------------------------ block reductions
// Deterministic: every thread combines its own elements in index order, then
// a fixed shuffle tree per warp, then warp results in warp order.
__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < kSampWarps; ++i) t += red[i];
  return t;
}
__device__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int i = 0; i < kSampWarps; ++i) t = fmaxf(t, red[i]);
  return t;
}

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Warp parameters of one row (all threads of the block). `red` >= 32 floats,
// `hist` 256 x u64, `sel` 4 u64 of shared memory.
// hist[bin] += v for every lane with `valid`, with one shared-memory atomic
// per distinct bin in the warp: the lanes of a bin add their values exactly
// (24-bit halves through integer warp reductions; v < 2^48) and the group's
// lowest lane adds the sum. Logit rows put most keys into a handful of bins,
// where one atomic per element would serialise. Integer sums, so the result
// does not depend on the grouping. All 32 lanes must call it together.
__device__ __forceinline__ void hist_add_warp(unsigned long long* hist, uint32_t bin, unsigned long long v,
                                              bool valid) {
  const unsigned peers = __match_any_sync(0xffffffffu, valid ? bin : 0xffffffffu);
  const unsigned lo = __reduce_add_sync(peers, static_cast<unsigned>(v & 0xffffffull));
  const unsigned hi = __reduce_add_sync(peers, static_cast<unsigned>(v >> 24));
  if (valid && (threadIdx.x & 31) == static_cast<unsigned>(__ffs(peers) - 1))
    atomicAdd(&hist[bin], (static_cast<unsigned long long>(hi) << 24) + lo);
}

__device__ WarpParams row_warp(const float* row, int V, float temperature, float top_p, float* red,
                               unsigned long long* hist, unsigned long long* sel) {
  WarpParams P;
  P.inv_t = 1.0f / temperature;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += kSampThreads) mx = fmaxf(mx, row[i]);
  P.m = block_max(mx, red);
  float z = 0.f;
  for (int i = threadIdx.x; i < V; i += kSampThreads) z += expf((row[i] - P.m) * P.inv_t);
  const float Z = block_sum(z, red);
  if (!(top_p < 1.0f)) {
    P.lambda = -INFINITY;
    P.log_z = logf(Z);
    return P;
  }
  const double scale = 281474976710656.0 / (double)Z;  // 2^48 / Z
  const unsigned long long target = static_cast<unsigned long long>((double)top_p * 281474976710656.0);
  uint32_t prefix = 0;
  unsigned long long mass_gt = 0;
  for (int level = 0; level < 4; ++level) {
    const int shift = 24 - 8 * level;
    for (int b = threadIdx.x; b < 256; b += kSampThreads) hist[b] = 0ull;
    __syncthreads();
    // Every thread runs the same number of passes (whole warps stay
    // converged for the warp-level aggregation in hist_add_warp).
    for (int base = 0; base < V; base += kSampThreads) {
      const int i = base + threadIdx.x;
      const float l = i < V ? row[i] : -INFINITY;
      const uint32_t k = order_key(l);
      const bool in = i < V && (level == 0 || (k >> (shift + 8)) == prefix);
      const unsigned long long fp =
          in ? static_cast<unsigned long long>((double)expf((l - P.m) * P.inv_t) * scale) : 0ull;
      hist_add_warp(hist, (k >> shift) & 255u, fp, in);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      // lowest non-empty bin whose mass strictly above it is <= top_p
      unsigned long long S = mass_gt, sel_S = mass_gt;
      int s = -1;
      for (int b = 255; b >= 0; --b) {
        if (hist[b] == 0ull) continue;
        if (S > target) break;
        s = b;
        sel_S = S;
        S += hist[b];
      }
      if (s < 0) s = 255;  // unreachable for a finite row
      sel[0] = (static_cast<unsigned long long>(prefix) << 8) | static_cast<unsigned>(s);
      sel[1] = sel_S;
    }
    __syncthreads();
    prefix = static_cast<uint32_t>(sel[0]);
    mass_gt = sel[1];
  }
  P.lambda = key_float(prefix);
  float zk = 0.f;
  for (int i = threadIdx.x; i < V; i += kSampThreads) {
    const float l = row[i];
    if (l >= P.lambda) zk += expf((l - P.m) * P.inv_t);
  }
  P.log_z = logf(block_sum(zk, red));
  return P;
}

__device__ __forceinline__ float warped_lp(const WarpParams& P, float l) {
  return l >= P.lambda ? (l - P.m) * P.inv_t - P.log_z : -INFINITY;
}

// One warp-parameter record per row.
__global__ void __launch_bounds__(kSampThreads) warp_params_kernel(const float* logits, int64_t ld, int V,
                                                                   float temperature, float top_p,
                                                                   WarpParams* out) {
  __shared__ float red[32];
  __shared__ unsigned long long hist[256];
  __shared__ unsigned long long sel[4];
  pdl_wait();
  pdl_trigger();
  const WarpParams P = row_warp(logits + (int64_t)blockIdx.x * ld, V, temperature, top_p, red, hist, sel);
  if (threadIdx.x == 0) out[blockIdx.x] = P;
}

// Warped probabilities of every row (grid: column blocks x rows).
__global__ void warp_probs_kernel(const float* logits, int64_t ld, int V, const WarpParams* params, float* out,
                                  int64_t ldo) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.y;
  const WarpParams P = params[r];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
    const float lp = warped_lp(P, logits[(int64_t)r * ld + i]);
    out[(int64_t)r * ldo + i] = lp == -INFINITY ? 0.f : expf(lp);
  }
}

// Gumbel top-k (sampling without replacement, in draw order) per row over
// the warped distribution; tokens through vocab_ids. Missing draws (support
// < k) get token -1 and log-prob -inf. RNG counter: (round, row_id[row], i, 0).
// Gumbel top-k of one row, split over a cluster of `gridDim.y` CTAs: CTA
// (cluster rank) s takes the vocabulary slice [s * len, (s + 1) * len), finds
// its k best keys (key desc, index asc) and pushes them into rank 0's shared
// memory; rank 0 merges the sorted slice lists. Keys and tie rules are those
// of a single pass over the whole row, so the draws do not depend on the
// split.
constexpr int kGumbelMaxSlices = 8;
__global__ void __launch_bounds__(kSampThreads) gumbel_topk_kernel(const float* logits, int64_t ld, int V,
                                                                   const WarpParams* params, int k,
                                                                   const int64_t* vocab_ids, const uint64_t* seed,
                                                                   const int32_t* round, int row_base,
                                                                   int32_t* out_tok, float* out_lp) {
  __shared__ float s_key[kSampWarps];
  __shared__ int s_idx[kSampWarps];
  __shared__ int s_own[kSampWarps];
  __shared__ float c_key[kGumbelMaxSlices * kMaxK];  // rank 0: every slice's list
  __shared__ int c_idx[kGumbelMaxSlices * kMaxK];
  pdl_wait();
  pdl_trigger();
  const int slices = gridDim.y, sl = blockIdx.y;  // cluster (1, slices): rank = sl
  const int len = (V + slices - 1) / slices;
  const int i0 = sl * len, i1 = min(V, i0 + len);
  const float* row = logits + (int64_t)blockIdx.x * ld;
  const WarpParams P = params[blockIdx.x];
  const uint64_t sd = seed[0];
  const uint32_t rnd = static_cast<uint32_t>(round ? round[0] : 0);
  const uint32_t row_id = static_cast<uint32_t>(row_base + blockIdx.x);
  // local top-k (descending key, ascending index on ties)
  float kk[kMaxK];
  int ki[kMaxK];
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    kk[j] = -INFINITY;
    ki[j] = INT32_MAX;
  }
  for (int i = i0 + threadIdx.x; i < i1; i += kSampThreads) {
    const float lp = warped_lp(P, row[i]);
    if (lp == -INFINITY) continue;
    const float g = -logf(-logf(uniform(sd, rnd, row_id, static_cast<uint32_t>(i), 0u)));
    const float key = lp + g;
    if (key > kk[k - 1] || (key == kk[k - 1] && i < ki[k - 1])) {
      int j = k - 1;
      while (j > 0 && (key > kk[j - 1] || (key == kk[j - 1] && i < ki[j - 1]))) {
        kk[j] = kk[j - 1];
        ki[j] = ki[j - 1];
        --j;
      }
      kk[j] = key;
      ki[j] = i;
    }
  }
  // this slice's k best, in order, into rank 0's candidate lists
  const uint32_t ck0 = slices > 1 ? dsmem_map(smem_u32(c_key), 0u) : 0u;
  const uint32_t ci0 = slices > 1 ? dsmem_map(smem_u32(c_idx), 0u) : 0u;
  int head = 0;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int q = 0; q < k; ++q) {
    float bk = head < k ? kk[head] : -INFINITY;
    int bi = head < k ? ki[head] : INT32_MAX;
    int own = threadIdx.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ok = __shfl_xor_sync(0xffffffffu, bk, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int oo = __shfl_xor_sync(0xffffffffu, own, o);
      if (ok > bk || (ok == bk && oi < bi)) {
        bk = ok;
        bi = oi;
        own = oo;
      }
    }
    if (lane == 0) {
      s_key[w] = bk;
      s_idx[w] = bi;
      s_own[w] = own;
    }
    __syncthreads();
    float gk = -INFINITY;
    int gi = INT32_MAX, go = -1;
    for (int j = 0; j < kSampWarps; ++j)
      if (s_key[j] > gk || (s_key[j] == gk && s_idx[j] < gi)) {
        gk = s_key[j];
        gi = s_idx[j];
        go = s_own[j];
      }
    if (threadIdx.x == go) ++head;
    if (threadIdx.x == 0) {
      if (slices > 1) {
        const uint32_t off = static_cast<uint32_t>((sl * kMaxK + q) * 4);
        dsmem_st(ck0 + off, gk);
        dsmem_st(ci0 + off, __int_as_float(gi));
      } else {
        c_key[q] = gk;
        c_idx[q] = gi;
      }
    }
    __syncthreads();
  }
  if (slices > 1) cluster_sync_all();  // every slice's list is in rank 0's shared memory
  if (sl != 0 || threadIdx.x != 0) return;
  int hd[kGumbelMaxSlices];
  for (int j = 0; j < kGumbelMaxSlices; ++j) hd[j] = 0;
  for (int q = 0; q < k; ++q) {
    float gk = -INFINITY;
    int gi = INT32_MAX, gs = -1;
    for (int j = 0; j < slices; ++j) {
      if (hd[j] >= k) continue;
      const float ck = c_key[j * kMaxK + hd[j]];
      const int cix = c_idx[j * kMaxK + hd[j]];
      if (ck > gk || (ck == gk && cix < gi)) {
        gk = ck;
        gi = cix;
        gs = j;
      }
    }
    if (gs >= 0) ++hd[gs];
    const bool ok = gk != -INFINITY;
    out_tok[(int64_t)blockIdx.x * k + q] = ok ? (vocab_ids ? (int)vocab_ids[gi] : gi) : -1;
    out_lp[(int64_t)blockIdx.x * k + q] = ok ? warped_lp(P, row[gi]) : -INFINITY;
  }
}

// Inverse-CDF draw from unnormalised non-negative weights w[0..n) with
// uniform u: contiguous per-thread chunks, exclusive scan in thread order.
__device__ int draw_from(const float* w, int n, float u, float* red, float* scan) {
  const int chunk = (n + kSampThreads - 1) / kSampThreads;
  const int b = threadIdx.x * chunk, e = min(n, b + chunk);
  float s = 0.f;
  for (int i = b; i < e; ++i) s += w[i];
  scan[threadIdx.x] = s;
  __syncthreads();
  __shared__ int s_pick;
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < kSampThreads; ++i) {
      const float v = scan[i];
      scan[i] = tot;
      tot += v;
    }
    red[0] = tot;
    s_pick = -1;
  }
  __syncthreads();
  const float target = u * red[0];
  const float lo = scan[threadIdx.x];
  if (target >= lo && target < lo + s && s > 0.f) {
    // the chunk's running sum can round below lo + s: fall back to its last
    // positive weight, never to a zero-weight index
    float c = lo;
    int pick = -1, last_pos = -1;
    for (int i = b; i < e; ++i) {
      if (!(w[i] > 0.f)) continue;
      last_pos = i;
      c += w[i];
      if (target < c) {
        pick = i;
        break;
      }
    }
    atomicMax(&s_pick, pick >= 0 ? pick : last_pos);
  }
  __syncthreads();
  int pick = s_pick;
  if (pick < 0) {  // rounding at the top end: last positive weight
    __shared__ int s_last;
    if (threadIdx.x == 0) s_last = -1;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kSampThreads)
      if (w[i] > 0.f) atomicMax(&s_last, i);
    __syncthreads();
    pick = s_last < 0 ? 0 : s_last;
  }
  __syncthreads();
  return pick;
}

// Token ~ warp(logits row): one launch, one row, one CTA; inverse-CDF draw
// with RNG counter (round[0], row_id, 0, stream). ssd_sample_token draws with
// the clustered warp_sample_kernel (Gumbel-max, counters (round[0], row_id,
// i, stream)); this kernel serves rows too long for a cluster.
__global__ void __launch_bounds__(kSampThreads) sample_token_kernel(const float* logits, int V, float temperature,
                                                                    float top_p, const uint64_t* seed,
                                                                    const int32_t* round, int row_id, int stream,
                                                                    float* scratch, int32_t* out) {
  __shared__ float red[32];
  __shared__ unsigned long long hist[256];
  __shared__ unsigned long long sel[4];
  __shared__ float scan[kSampThreads];
  pdl_wait();
  pdl_trigger();
  const WarpParams P = row_warp(logits, V, temperature, top_p, red, hist, sel);
  for (int i = threadIdx.x; i < V; i += kSampThreads) {
    const float lp = warped_lp(P, logits[i]);
    scratch[i] = lp == -INFINITY ? 0.f : expf(lp);
  }
  __syncthreads();
  const float u = uniform(seed[0], static_cast<uint32_t>(round ? round[0] : 0), static_cast<uint32_t>(row_id), 0u,
                          static_cast<uint32_t>(stream));
  const int pick = draw_from(scratch, V, u, red, scan);
  if (threadIdx.x == 0) out[0] = pick;
}

// Multi-candidate speculative sampling without replacement over the device
// tree (one CTA). Target row r of `tlogits` belongs to row r of the verify
// forward (0 = root); the draft distribution a node's children were drawn
// from is draft row 0 for the root, else draft_pos - root_pos. Warp
// parameters of every target and draft row come precomputed (tparams,
// dparams), so the walk only materialises p and q along the accepted path.
// p, q: scratch of V floats each (q is 0 outside the draft vocabulary).
// RNG counters: acceptance (round, cur + 1, child, 1), bonus (round, cur + 1, 0, 2).
__global__ void __launch_bounds__(kSampThreads) sample_verify_kernel(
    const int32_t* n_nodes, int max_nodes, const int32_t* tokens, const int32_t* parents, const int32_t* ranks,
    const int32_t* draft_pos, const int32_t* root_pos, const float* tlogits, int64_t ldt, const WarpParams* tparams,
    int V, const float* dlogits, int64_t ldd, const WarpParams* dparams, int draft_rows, int Vd,
    const int64_t* vocab_ids, const uint64_t* seed, const int32_t* round, float* p, float* q, int32_t* accepted,
    int32_t* n_accepted, int32_t* bonus, int32_t* keep_slots, int32_t* n_keep, uint32_t* status) {
  __shared__ float red[32];
  __shared__ float scan[kSampThreads];
  __shared__ int kids[64];
  __shared__ int s_nk;
  __shared__ int s_chosen;
  pdl_wait();
  pdl_trigger();
  const int n = min(*n_nodes, max_nodes);
  const int c0 = root_pos[0];
  const uint64_t sd = seed[0];
  const uint32_t rnd = static_cast<uint32_t>(round ? round[0] : 0);
  int cur = -1, na = 0;
  if (threadIdx.x == 0) keep_slots[0] = c0;
  for (int step = 0; step <= n; ++step) {
    // p = warp(target row of cur)
    const float* trow = tlogits + (int64_t)(cur + 1) * ldt;
    const WarpParams PT = tparams[cur + 1];
    for (int i = threadIdx.x; i < V; i += kSampThreads) {
      const float lp = warped_lp(PT, trow[i]);
      p[i] = lp == -INFINITY ? 0.f : expf(lp);
    }
    // children of cur in rank order (ties by index)
    if (threadIdx.x == 0) {
      int m = 0;
      for (int i = 0; i < n && m < 64; ++i)
        if (parents[i] == cur) kids[m++] = i;
      for (int a = 1; a < m; ++a) {
        const int x = kids[a];
        int b = a - 1;
        while (b >= 0 && ranks[kids[b]] > ranks[x]) {
          kids[b + 1] = kids[b];
          --b;
        }
        kids[b + 1] = x;
      }
      s_nk = m;
      s_chosen = -1;
    }
    __syncthreads();
    const int nk = s_nk;
    if (nk > 0) {
      const int drow = cur < 0 ? 0 : draft_pos[cur] - c0;
      if (drow < 0 || drow >= draft_rows) {
        if (threadIdx.x == 0) report_error(status, kErrBadIndex);
        break;
      }
      // q over the full vocabulary (0 outside the draft vocabulary)
      const float* dr = dlogits + (int64_t)drow * ldd;
      const WarpParams PD = dparams[drow];
      if (vocab_ids) {
        for (int i = threadIdx.x; i < V; i += kSampThreads) q[i] = 0.f;
        __syncthreads();
        for (int j = threadIdx.x; j < Vd; j += kSampThreads) {
          const int64_t v = vocab_ids[j];
          const float lp = warped_lp(PD, dr[j]);
          if (v >= 0 && v < V) q[v] = lp == -INFINITY ? 0.f : expf(lp);
        }
      } else {
        for (int i = threadIdx.x; i < V; i += kSampThreads) {
          const float lp = i < Vd ? warped_lp(PD, dr[i]) : -INFINITY;
          q[i] = lp == -INFINITY ? 0.f : expf(lp);
        }
      }
      __syncthreads();
      float zp = 1.f, zq = 1.f;  // p / zp and q / zq are the current distributions
      for (int ci = 0; ci < nk; ++ci) {
        const int c = kids[ci];
        const int x = tokens[c];
        const bool in = x >= 0 && x < V;
        const float qx = in ? q[x] / zq : 0.f;
        if (!(qx > 0.f)) continue;
        const float px = p[x] / zp;
        const float u = uniform(sd, rnd, static_cast<uint32_t>(cur + 1), static_cast<uint32_t>(ci), 1u);
        if (u < fminf(1.f, px / qx)) {
          if (threadIdx.x == 0) s_chosen = c;
          break;
        }
        // reject: p <- max(p - q, 0) renormalised, only if that has mass
        float rs = 0.f;
        for (int i = threadIdx.x; i < V; i += kSampThreads) rs += fmaxf(p[i] / zp - q[i] / zq, 0.f);
        const float R = block_sum(rs, red);
        if (R > 0.f) {
          for (int i = threadIdx.x; i < V; i += kSampThreads) p[i] = fmaxf(p[i] / zp - q[i] / zq, 0.f);
          zp = R;
        }
        // q <- q without x, renormalised; stop when nothing is left
        __syncthreads();
        if (threadIdx.x == 0) q[x] = 0.f;
        __syncthreads();
        float qs = 0.f;
        for (int i = threadIdx.x; i < V; i += kSampThreads) qs += q[i];
        const float Q = block_sum(qs, red);
        if (!(Q > 0.f)) break;
        zq = Q;
      }
      __syncthreads();
      if (s_chosen >= 0) {
        const int c = s_chosen;
        if (threadIdx.x == 0) {
          accepted[na] = c;
          keep_slots[1 + na] = c0 + 1 + c;
        }
        ++na;
        cur = c;
        __syncthreads();
        continue;
      }
    }
    __syncthreads();
    const float u = uniform(sd, rnd, static_cast<uint32_t>(cur + 1), 0u, 2u);
    const int pick = draw_from(p, V, u, red, scan);
    if (threadIdx.x == 0) {
      *bonus = pick;
      *n_accepted = na;
      *n_keep = na + 1;
    }
    return;
  }
  if (threadIdx.x == 0) {
    *bonus = 0;
    *n_accepted = na;
    *n_keep = na + 1;
  }
}

// ------------------------------------------------------ cluster row kernels
// One logit row split over a cluster of S CTAs (S <= 8, grid x = rank): CTA s
// stages its slice [s * len, min(V, (s + 1) * len)) of the row in shared
// memory once and every pass reads it from there. Row-wide reductions publish
// one partial per CTA in the CTA's own slot, cross one cluster barrier, and
// every CTA combines the S partials in rank order, so all CTAs hold the same
// bits and take the same decisions. Slots come in two banks used in turn
// (one counter per kernel): a bank is rewritten two exchanges later, after a
// barrier that every reader of its previous contents has passed. Each kernel
// ends with a cluster barrier, so no CTA exits while a peer may still read
// its shared memory.
constexpr int kRowMaxSlices = 8;
constexpr int kRowSliceMax = 16384;  // staged floats per CTA (64 KB)

struct RowExchange {
  float* fslot;               // [2][2] floats: (value, index bits) per bank
  unsigned long long* hslot;  // [2][256] histogram bins per bank
  float* gath;                // [2 * kRowMaxSlices] gathered partials
  unsigned long long* whist;  // [kSampWarps][256] per-warp bins (radix select)
  unsigned* cnt;              // [256] sampled key counts per top byte (radix select)
  int* slot_of;               // [256 + 8]: slot of a top byte (-1: none), then the byte of each slot
  int S;
  int n;  // exchanges so far
};

// Row-wide max (is_max) or sum of a CTA-uniform value v, in rank order.
__device__ float row_allreduce(RowExchange& x, float v, bool is_max) {
  float* slot = x.fslot + (x.n & 1) * 2;
  if (threadIdx.x == 0) slot[0] = v;
  cluster_sync_all();
  if (threadIdx.x < x.S) x.gath[threadIdx.x] = dsmem_ld(dsmem_map(smem_u32(slot), threadIdx.x));
  __syncthreads();
  float r = is_max ? -INFINITY : 0.f;
  for (int t = 0; t < x.S; ++t) r = is_max ? fmaxf(r, x.gath[t]) : r + x.gath[t];
  __syncthreads();  // gath is reused by the next exchange
  ++x.n;
  return r;
}

// Row-wide best (key desc, index asc) of CTA-uniform (key, idx) pairs.
__device__ void row_allbest(RowExchange& x, float& key, int& idx) {
  float* slot = x.fslot + (x.n & 1) * 2;
  if (threadIdx.x == 0) {
    slot[0] = key;
    slot[1] = __int_as_float(idx);
  }
  cluster_sync_all();
  if (threadIdx.x < x.S) {
    const uint32_t a = dsmem_map(smem_u32(slot), threadIdx.x);
    x.gath[2 * threadIdx.x] = dsmem_ld(a);
    x.gath[2 * threadIdx.x + 1] = dsmem_ld(a + 4);
  }
  __syncthreads();
  float bk = -INFINITY;
  int bi = INT32_MAX;
  for (int t = 0; t < x.S; ++t) {
    const float k = x.gath[2 * t];
    const int i = __float_as_int(x.gath[2 * t + 1]);
    if (k > bk || (k == bk && i < bi)) {
      bk = k;
      bi = i;
    }
  }
  __syncthreads();
  ++x.n;
  key = bk;
  idx = bi;
}

// Row max m and normaliser Z = sum exp((l - m) * inv_t) from every CTA's
// (max, sum against that max), combined in rank order.
__device__ void row_max_sum(RowExchange& x, float mc, float zc, float inv_t, float& m, float& Z) {
  float* slot = x.fslot + (x.n & 1) * 2;
  if (threadIdx.x == 0) {
    slot[0] = mc;
    slot[1] = zc;
  }
  cluster_sync_all();
  if (threadIdx.x < x.S) {
    const uint32_t a = dsmem_map(smem_u32(slot), threadIdx.x);
    x.gath[2 * threadIdx.x] = dsmem_ld(a);
    x.gath[2 * threadIdx.x + 1] = dsmem_ld(a + 4);
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int t = 0; t < x.S; ++t) mx = fmaxf(mx, x.gath[2 * t]);
  float z = 0.f;
  for (int t = 0; t < x.S; ++t) {
    const float mt = x.gath[2 * t];
    if (mt != -INFINITY) z += x.gath[2 * t + 1] * expf((mt - mx) * inv_t);
  }
  __syncthreads();
  ++x.n;
  m = mx;
  Z = z;
}

// Cluster-wide radix select over the order keys of the staged slice: four
// 8-bit levels; at each level every CTA histograms the keys >= floor_key that
// share the prefix found so far (weight(l) per key: 1 to select by count, a
// 2^48 fixed-point mass to select by probability mass), the bins are summed
// over the cluster (integers, so the sums do not depend on the split or the
// order) and the selected bin is the lowest whose weight strictly above it
// stays <= target (by mass) or, counting, the bin holding the target-th
// largest key. Returns the selected key; at_or_above (if given) receives the
// summed weight of the keys >= it.
//
// A row's keys crowd into a few top-byte bins, so the first level avoids
// shared-memory atomics on them. It first tries a window: top_bin is the top
// byte of the row maximum's key; each thread adds the weights of bins
// top_bin .. top_bin-7 into its own slots and only counts the keys of all
// lower bins (one lump, in bin top_bin-8), and the slots are summed per bin.
// The window bins are exactly the full histogram's and the rule never looks
// below the bin it selects, so when it selects a window bin the result is the
// full histogram's; when it selects the lump, the level is histogrammed again
// in full (a cluster-uniform decision): the 8 top bytes most frequent in a
// sample of the slice get per-thread slots, the others shared atomics. Deeper
// levels see few keys over spread-out bins and add to one shared histogram.
template <typename Weight>
__device__ uint32_t cluster_radix_select(const float* xs, int n, uint32_t floor_key, unsigned long long target,
                                         bool by_count, Weight weight, RowExchange& x, unsigned long long* sel,
                                         uint32_t top_bin, unsigned long long* at_or_above = nullptr) {
  uint32_t prefix = 0;
  unsigned long long above = 0;
  bool window = top_bin >= 8u && top_bin <= 255u;
  const int lane = threadIdx.x & 31;
  // Exchange banks alternate, and a bank's last remote readers finished before
  // the previous exchange's cluster barrier: the first level zeroes its bank
  // here, each level zeroes the next one after its own cluster barrier.
  for (int b = threadIdx.x; b < 256; b += kSampThreads) x.hslot[(x.n & 1) * 256 + b] = 0ull;
  for (int level = 0; level < 4; ++level) {
    const int shift = 24 - 8 * level;
    unsigned long long* hist = x.hslot + (x.n & 1) * 256;
    const bool per_warp = level == 0 && !window;
    if (level == 0) __syncthreads();  // zeroed bins before any add
    if (level == 0 && window) {
      // each thread adds into its own 8 slots (slot j of thread t at
      // whist[j * kSampThreads + t]): no other thread touches them
      unsigned long long* slot = x.whist + threadIdx.x;
#pragma unroll
      for (int j = 0; j < 8; ++j) slot[j * kSampThreads] = 0ull;
      unsigned lump = 0;
#pragma unroll 2
      for (int i = threadIdx.x; i < n; i += kSampThreads) {
        const float l = xs[i];
        const uint32_t k = order_key(l);
        if (k < floor_key) continue;
        const uint32_t d = top_bin - (k >> 24);  // keys never exceed the maximum's
        if (d >= 8u) {
          ++lump;
          continue;
        }
        slot[d * kSampThreads] += weight(l);
      }
      // The lump holds its key count: the rule only asks whether it is empty
      // (it is never above a selected bin), and selecting it means the full
      // pass.
      const unsigned lumped = __reduce_add_sync(0xffffffffu, lump);
      if (lane == 0 && lumped != 0u) atomicAdd(&hist[top_bin - 8], static_cast<unsigned long long>(lumped));
      __syncthreads();
      {
        // warp w sums slot w/4 over a quarter of the threads, exactly
        const int j = (threadIdx.x >> 5) >> 2, q = (threadIdx.x >> 5) & 3;
        const unsigned long long* src = x.whist + j * kSampThreads + q * 256 + lane;
        unsigned long long t = 0ull;
#pragma unroll
        for (int e = 0; e < 8; ++e) t += src[e * 32];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (lane == 0 && t != 0ull) atomicAdd(&hist[top_bin - j], t);
      }
    } else if (per_warp) {
      // Full first level: a sample of the slice (each thread's first key)
      // picks the 8 most populated top bytes; their weights go to per-thread
      // slots as in the window, every other byte to shared atomics. Every bin
      // is exact whichever bytes get slots.
      for (int b = threadIdx.x; b < 256; b += kSampThreads) x.cnt[b] = 0u;
      __syncthreads();
      if (threadIdx.x < n) {
        const uint32_t k = order_key(xs[threadIdx.x]);
        if (k >= floor_key) atomicAdd(&x.cnt[k >> 24], 1u);
      }
      __syncthreads();
      if (threadIdx.x < 32) {
        // warp 0: eight rounds of a (count, -byte) maximum; lane j holds bytes 8j .. 8j + 7
        unsigned c[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) c[t] = x.cnt[8 * lane + t];
        for (int b = lane; b < 256; b += 32) x.slot_of[b] = -1;
        __syncwarp();
        for (int sl = 0; sl < 8; ++sl) {
          unsigned best = 0u;
          int bb = 256;
#pragma unroll
          for (int t = 0; t < 8; ++t)
            if (c[t] > best) {
              best = c[t];
              bb = 8 * lane + t;
            }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const unsigned ob = __shfl_xor_sync(0xffffffffu, best, o);
            const int obb = __shfl_xor_sync(0xffffffffu, bb, o);
            if (ob > best || (ob == best && obb < bb)) {
              best = ob;
              bb = obb;
            }
          }
          if (lane == 0) x.slot_of[256 + sl] = best > 0u ? bb : -1;
          if (best > 0u) {
            if (lane == 0) x.slot_of[bb] = sl;
#pragma unroll
            for (int t = 0; t < 8; ++t)
              if (8 * lane + t == bb) c[t] = 0u;
          }
        }
      }
      unsigned long long* slot = x.whist + threadIdx.x;
#pragma unroll
      for (int j = 0; j < 8; ++j) slot[j * kSampThreads] = 0ull;
      __syncthreads();
      for (int i = threadIdx.x; i < n; i += kSampThreads) {
        const float l = xs[i];
        const uint32_t k = order_key(l);
        if (k < floor_key) continue;
        const int sl = x.slot_of[k >> 24];
        const unsigned long long v = weight(l);
        if (sl >= 0) {
          slot[sl * kSampThreads] += v;
        } else {
          atomicAdd(&hist[k >> 24], v);
        }
      }
      __syncthreads();
      {
        // warp w sums slot w/4 over a quarter of the threads, exactly
        const int j = (threadIdx.x >> 5) >> 2, q = (threadIdx.x >> 5) & 3;
        const int byte = x.slot_of[256 + j];
        const unsigned long long* src = x.whist + j * kSampThreads + q * 256 + lane;
        unsigned long long t = 0ull;
#pragma unroll
        for (int e = 0; e < 8; ++e) t += src[e * 32];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (lane == 0 && byte >= 0 && t != 0ull) atomicAdd(&hist[byte], t);
      }
    } else {
#pragma unroll 2
      for (int i = threadIdx.x; i < n; i += kSampThreads) {
        const float l = xs[i];
        const uint32_t k = order_key(l);
        if (k >= floor_key && (k >> (shift + 8)) == prefix) atomicAdd(&hist[(k >> shift) & 255u], weight(l));
      }
    }
    // the cluster barrier also orders this CTA's adds before the reads below
    cluster_sync_all();  // every CTA's bins are complete; whist is free again
    for (int b = threadIdx.x; b < 256; b += kSampThreads) x.hslot[((x.n + 1) & 1) * 256 + b] = 0ull;
    {
      // four quarters of the block each sum a quarter of the ranks' bins
      static_assert(kSampThreads == 4 * 256, "bin gather assumes 1024 threads");
      const int b = threadIdx.x & 255, q = threadIdx.x >> 8;
      const uint32_t a = smem_u32(hist + b);
      unsigned long long t = 0ull;
      for (int r = q; r < x.S; r += 4) t += dsmem_ld_u64(dsmem_map(a, r));
      x.whist[q * 256 + b] = t;
    }
    ++x.n;
    __syncthreads();
    if (threadIdx.x < 32) {
      // warp 0 selects the bin: lane j holds bins 255-8j down to 248-8j, a
      // shuffle scan gives the weight strictly above its first bin, and the
      // lane walks its bins downward applying the rule
      unsigned long long h[8], tot = 0ull;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int b = 255 - 8 * lane - t;
        h[t] = x.whist[b] + x.whist[256 + b] + x.whist[512 + b] + x.whist[768 + b];
        tot += h[t];
      }
      unsigned long long inc = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
      }
      unsigned long long c = above + inc - tot;
      int cand = -1, low = -1;
      unsigned long long cand_s = 0ull, low_s = 0ull, cand_h = 0ull, low_h = 0ull;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int b = 255 - 8 * lane - t;
        if (h[t] != 0ull) {
          if (by_count) {
            // counting: the first bin (from the top) that reaches the target
            if (cand < 0 && c + h[t] >= target) {
              cand = b;
              cand_s = c;
              cand_h = h[t];
            }
            low = b;
            low_s = c;
            low_h = h[t];
          } else if (c <= target) {
            // by mass: the lowest bin whose weight above stays <= target
            cand = b;
            cand_s = c;
            cand_h = h[t];
          }
          c += h[t];
        }
      }
      const unsigned has = __ballot_sync(0xffffffffu, cand >= 0);
      int src;
      int sb = 255;  // no bin qualifies: unreachable for a finite row
      unsigned long long ss = above, sh = 0ull;
      if (has != 0u) {
        src = by_count ? __ffs(has) - 1 : 31 - __clz(has);
        sb = __shfl_sync(0xffffffffu, cand, src);
        ss = __shfl_sync(0xffffffffu, cand_s, src);
        sh = __shfl_sync(0xffffffffu, cand_h, src);
      } else if (by_count) {
        // the target lies below every key: the lowest non-empty bin
        const unsigned nz = __ballot_sync(0xffffffffu, low >= 0);
        if (nz != 0u) {
          src = 31 - __clz(nz);
          sb = __shfl_sync(0xffffffffu, low, src);
          ss = __shfl_sync(0xffffffffu, low_s, src);
          sh = __shfl_sync(0xffffffffu, low_h, src);
        }
      }
      if (lane == 0) {
        sel[0] = (static_cast<unsigned long long>(prefix) << 8) | static_cast<unsigned>(sb);
        sel[1] = ss;
        sel[2] = sh;
      }
    }
    // sel is next written a level later, after the cluster barrier that every
    // thread reaches only after reading it here
    __syncthreads();
    const uint32_t got = static_cast<uint32_t>(sel[0]);
    const unsigned long long got_above = sel[1];
    if (level == 0 && window && got == top_bin - 8u) {  // the lump: histogram the level in full
      window = false;
      --level;
      continue;
    }
    prefix = got;
    above = got_above;
    if (level == 3 && at_or_above) *at_or_above = got_above + sel[2];
  }
  return prefix;
}

// Warp parameters of the row whose slice is staged in xs[0, n): max,
// kept-mass normaliser and the smallest kept logit. keep_top > 0 first keeps
// only the keep_top largest logits (ties at the boundary all kept); top_p < 1
// then keeps the nucleus of what remains, by the same radix select as
// row_warp with the bins summed over the cluster. Without keep_top each CTA
// sums against its own max and one exchange combines (max, sum) pairs. The
// kept mass of a nucleus is the radix select's integer
// mass at or above the threshold, scaled back by Z / 2^48 (each of its
// terms truncates less than 2^-48 of Z).
__device__ WarpParams cluster_row_warp(const float* xs, int n, int V, float temperature, float top_p, int keep_top,
                                       float* red, RowExchange& x, unsigned long long* sel) {
  WarpParams P;
  P.inv_t = 1.0f / temperature;
  uint32_t floor_key = 0;
  float lam_k = -INFINITY;
  float Z;
  if (keep_top > 0 && keep_top < V) {
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n; i += kSampThreads) mx = fmaxf(mx, xs[i]);
    P.m = row_allreduce(x, block_max(mx, red), true);
    floor_key = cluster_radix_select(xs, n, 0u, static_cast<unsigned long long>(keep_top), true,
                                     [](float) { return 1ull; }, x, sel, order_key(P.m) >> 24);
    lam_k = key_float(floor_key);
    float z = 0.f;
    for (int i = threadIdx.x; i < n; i += kSampThreads)
      if (xs[i] >= lam_k) z += expf((xs[i] - P.m) * P.inv_t);
    Z = row_allreduce(x, block_sum(z, red), false);
  } else {
    float mt = -INFINITY;
    for (int i = threadIdx.x; i < n; i += kSampThreads) mt = fmaxf(mt, xs[i]);
    const float mc = block_max(mt, red);
    float zt = 0.f;
    if (mc != -INFINITY)
      for (int i = threadIdx.x; i < n; i += kSampThreads) zt += expf((xs[i] - mc) * P.inv_t);
    row_max_sum(x, mc, block_sum(zt, red), P.inv_t, P.m, Z);
  }
  if (!(top_p < 1.0f)) {
    P.lambda = lam_k;
    P.log_z = logf(Z);
    return P;
  }
  const double scale = 281474976710656.0 / (double)Z;  // 2^48 / Z
  const unsigned long long target = static_cast<unsigned long long>((double)top_p * 281474976710656.0);
  const float m = P.m, inv_t = P.inv_t;
  unsigned long long kept = 0ull;
  const uint32_t key = cluster_radix_select(
      xs, n, floor_key, target, false,
      [=](float l) { return static_cast<unsigned long long>((double)expf((l - m) * inv_t) * scale); }, x, sel,
      order_key(m) >> 24, &kept);
  P.lambda = key_float(key);
  P.log_z = (float)log((double)kept * ((double)Z / 281474976710656.0));
  return P;
}

// Fused warp parameters + Gumbel top-k of each row (grid (S, rows), cluster
// (S, 1)): the parameters of row r go to params_out[r] (if given) and its k
// draws without replacement, in draw order, to out_tok / out_lp[r * k ...]
// (k = 0: parameters only). The draws equal gumbel_topk_kernel's for the same
// parameters: keys lp + Gumbel with RNG counter (round, row_base + r, i,
// stream), ties to the lower index, tokens through vocab_ids. KB >= k bounds
// the per-thread candidate list, which lives in registers.
template <int KB>
__global__ void __launch_bounds__(kSampThreads, 1) warp_sample_kernel(
    const float* logits, int64_t ld, int V, float temperature, float top_p, int keep_top, int k,
    const int64_t* vocab_ids,
    const uint64_t* seed, const int32_t* round, int row_base, int stream, WarpParams* params_out, int32_t* out_tok,
    float* out_lp) {
  extern __shared__ float xs[];
  __shared__ float red[32];
  __shared__ float fslot[4];
  __shared__ unsigned long long hslot[512];
  __shared__ float gath[2 * kRowMaxSlices];
  __shared__ unsigned long long sel[4];
  __shared__ float w_key[kSampWarps * kMaxK];  // each warp's k best
  __shared__ int w_idx[kSampWarps * kMaxK];
  __shared__ float c_key[kRowMaxSlices * kMaxK];  // rank 0: every slice's list
  __shared__ int c_idx[kRowMaxSlices * kMaxK];
  const int S = gridDim.x, s = blockIdx.x, r = blockIdx.y;
  const int len = (V + S - 1) / S;
  const int i0 = s * len, n = max(0, min(V, i0 + len) - i0);
  const float* row = logits + (int64_t)r * ld;
  pdl_wait();
  pdl_trigger();
  for (int i = threadIdx.x; i < n; i += kSampThreads) xs[i] = row[i0 + i];
  __syncthreads();
  __shared__ unsigned s_cnt[256];
  __shared__ int s_slot_of[256 + 8];
  RowExchange x{fslot, hslot, gath, nullptr, s_cnt, s_slot_of, S, 0};
  x.whist = reinterpret_cast<unsigned long long*>(xs + ((len + 1) & ~1));
  const WarpParams P = cluster_row_warp(xs, n, V, temperature, top_p, keep_top, red, x, sel);
  if (s == 0 && threadIdx.x == 0 && params_out) params_out[r] = P;
  if (k <= 0) {
    cluster_sync_all();  // peers may still read this CTA's exchange slot
    return;
  }
  const uint64_t sd = seed[0];
  const uint32_t rnd = static_cast<uint32_t>(round ? round[0] : 0);
  const uint32_t row_id = static_cast<uint32_t>(row_base + r);
  static_assert(KB >= 1 && KB <= kMaxK, "candidate list bound");
  float kk[KB];
  int ki[KB];
#pragma unroll
  for (int j = 0; j < KB; ++j) {
    kk[j] = -INFINITY;
    ki[j] = INT32_MAX;
  }
  // the thread's k best stay sorted in registers (static indices only); the
  // k-th best is mirrored in (tk, ti) for the common reject test
  float tk = -INFINITY;
  int ti = INT32_MAX;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto draw = [&](int i) {
    const int gi = i0 + i;
    const float g = -logf(-logf(uniform(sd, rnd, row_id, static_cast<uint32_t>(gi), static_cast<uint32_t>(stream))));
    float ck = warped_lp(P, xs[i]) + g;
    int ci = gi;
    if (ck > tk || (ck == tk && ci < ti)) {
      // carry the new key down the list, swapping it past every worse one
#pragma unroll
      for (int j = 0; j < KB; ++j) {
        if (j < k && (ck > kk[j] || (ck == kk[j] && ci < ki[j]))) {
          const float fk = kk[j];
          const int fi = ki[j];
          kk[j] = ck;
          ki[j] = ci;
          ck = fk;
          ci = fi;
        }
      }
#pragma unroll
      for (int j = 0; j < KB; ++j)
        if (j == k - 1) {
          tk = kk[j];
          ti = ki[j];
        }
    }
  };
  // Only nucleus members draw. Each warp queues the indices of its kept
  // logits (the radix select's histograms are free now) and draws 32 at a
  // time, so a draw pass runs with every lane busy however sparse the
  // nucleus; lanes hold different subsets than a strided loop would, but the
  // merges below order by (key, index), so the draws do not change.
  int* queue = reinterpret_cast<int*>(x.whist) + w * 64;
  int queued = 0;
  for (int base = w * 32; base < n; base += kSampThreads) {  // warp-uniform bound
    const int i = base + lane;
    const bool kept = i < n && warped_lp(P, xs[i]) != -INFINITY;
    const unsigned m = __ballot_sync(0xffffffffu, kept);
    if (kept) queue[queued + __popc(m & ((1u << lane) - 1u))] = i;
    queued += __popc(m);
    __syncwarp();
    if (queued >= 32) {
      const int mine = queue[lane];
      __syncwarp();
      if (lane < queued - 32) queue[lane] = queue[32 + lane];
      queued -= 32;
      __syncwarp();
      draw(mine);
    }
  }
  if (lane < queued) draw(queue[lane]);
  // this slice's k best, in order, into rank 0's candidate lists: each warp
  // merges its lanes' sorted lists into its own k best (the winning lane
  // shifts its list up), then warp 0 merges the warps' lists the same way
  for (int q = 0; q < k; ++q) {
    float bk = kk[0];
    int bi = ki[0], own = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ok = __shfl_xor_sync(0xffffffffu, bk, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int oo = __shfl_xor_sync(0xffffffffu, own, o);
      if (ok > bk || (ok == bk && oi < bi)) {
        bk = ok;
        bi = oi;
        own = oo;
      }
    }
    if (lane == own) {
#pragma unroll
      for (int j = 0; j + 1 < KB; ++j) {
        kk[j] = kk[j + 1];
        ki[j] = ki[j + 1];
      }
      kk[KB - 1] = -INFINITY;
      ki[KB - 1] = INT32_MAX;
    }
    if (lane == 0) {
      w_key[w * kMaxK + q] = bk;
      w_idx[w * kMaxK + q] = bi;
    }
  }
  __syncthreads();
  if (w == 0) {
    static_assert(kSampWarps == 32, "one lane per warp list");
    const uint32_t ck0 = dsmem_map(smem_u32(c_key), 0u);
    const uint32_t ci0 = dsmem_map(smem_u32(c_idx), 0u);
    int head = 0;
    for (int q = 0; q < k; ++q) {
      float bk = head < k ? w_key[lane * kMaxK + head] : -INFINITY;
      int bi = head < k ? w_idx[lane * kMaxK + head] : INT32_MAX;
      int own = lane;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ok = __shfl_xor_sync(0xffffffffu, bk, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        const int oo = __shfl_xor_sync(0xffffffffu, own, o);
        if (ok > bk || (ok == bk && oi < bi)) {
          bk = ok;
          bi = oi;
          own = oo;
        }
      }
      if (lane == own) ++head;
      if (lane == 0) {
        const uint32_t off = static_cast<uint32_t>((s * kMaxK + q) * 4);
        dsmem_st(ck0 + off, bk);
        dsmem_st(ci0 + off, __int_as_float(bi));
      }
    }
  }
  cluster_sync_all();  // every slice's list is in rank 0's shared memory
  if (s != 0 || threadIdx.x != 0) return;
  int hd[kRowMaxSlices];
  for (int j = 0; j < kRowMaxSlices; ++j) hd[j] = 0;
  for (int q = 0; q < k; ++q) {
    float gk = -INFINITY;
    int gi = INT32_MAX, gs = -1;
    for (int j = 0; j < S; ++j) {
      if (hd[j] >= k) continue;
      const float ck = c_key[j * kMaxK + hd[j]];
      const int cix = c_idx[j * kMaxK + hd[j]];
      if (ck > gk || (ck == gk && cix < gi)) {
        gk = ck;
        gi = cix;
        gs = j;
      }
    }
    if (gs >= 0) ++hd[gs];
    const bool ok = gk != -INFINITY;
    out_tok[(int64_t)r * k + q] = ok ? (vocab_ids ? (int)vocab_ids[gi] : gi) : -1;
    if (out_lp) out_lp[(int64_t)r * k + q] = ok ? warped_lp(P, row[gi]) : -INFINITY;
  }
}

// Multi-candidate speculative sampling without replacement over the device
// tree, on a cluster of S CTAs (grid (S, 1)): CTA s keeps its vocabulary
// slice of the current p and q in shared memory. Every CTA runs the walk;
// decisions use point values read from the owning CTA and sums combined in
// rank order, so all CTAs decide alike. Same inputs and RNG counters as
// sample_verify_kernel for the acceptance tests ((round, cur + 1, child, 1));
// the bonus token is a Gumbel-max draw from the current p with counters
// (round, cur + 1, i, 2) (the same distribution as an inverse-CDF draw).
__global__ void __launch_bounds__(kSampThreads, 1) sample_verify_cluster_kernel(
    const int32_t* n_nodes, int max_nodes, const int32_t* tokens, const int32_t* parents, const int32_t* ranks,
    const int32_t* draft_pos, const int32_t* root_pos, const float* tlogits, int64_t ldt, const WarpParams* tparams,
    int V, const float* dlogits, int64_t ldd, const WarpParams* dparams, int draft_rows, int Vd,
    const int64_t* vocab_ids, const uint64_t* seed, const int32_t* round, int32_t* accepted, int32_t* n_accepted,
    int32_t* bonus, int32_t* keep_slots, int32_t* n_keep, uint32_t* status) {
  extern __shared__ float dyn[];
  __shared__ float red[32];
  __shared__ float fslot[4];
  __shared__ float gath[2 * kRowMaxSlices];
  __shared__ int kids[64];
  __shared__ int s_nk;
  __shared__ float s_pt[2];
  __shared__ float s_key[kSampWarps];
  __shared__ int s_idx[kSampWarps];
  const int S = gridDim.x, s = blockIdx.x;
  const int len = (V + S - 1) / S;
  const int i0 = s * len, nl = max(0, min(V, i0 + len) - i0);
  float* ps = dyn;
  float* qs = dyn + len;
  pdl_wait();
  pdl_trigger();
  RowExchange x{fslot, nullptr, gath, nullptr, nullptr, nullptr, S, 0};
  const int n = min(*n_nodes, max_nodes);
  const int c0 = root_pos[0];
  const uint64_t sd = seed[0];
  const uint32_t rnd = static_cast<uint32_t>(round ? round[0] : 0);
  const bool lead = s == 0 && threadIdx.x == 0;
  int cur = -1, na = 0;
  if (lead) keep_slots[0] = c0;
  for (int step = 0; step <= n; ++step) {
    // p = warp(target row of cur), this CTA's slice
    const float* trow = tlogits + (int64_t)(cur + 1) * ldt;
    const WarpParams PT = tparams[cur + 1];
    for (int i = threadIdx.x; i < nl; i += kSampThreads) {
      const float lp = warped_lp(PT, trow[i0 + i]);
      ps[i] = lp == -INFINITY ? 0.f : expf(lp);
    }
    // children of cur in rank order (ties by index)
    if (threadIdx.x == 0) {
      int m = 0;
      for (int i = 0; i < n && m < 64; ++i)
        if (parents[i] == cur) kids[m++] = i;
      for (int a = 1; a < m; ++a) {
        const int c = kids[a];
        int b = a - 1;
        while (b >= 0 && ranks[kids[b]] > ranks[c]) {
          kids[b + 1] = kids[b];
          --b;
        }
        kids[b + 1] = c;
      }
      s_nk = m;
    }
    __syncthreads();
    const int nk = s_nk;
    int chosen = -1;
    if (nk > 0) {
      const int drow = cur < 0 ? 0 : draft_pos[cur] - c0;
      if (drow < 0 || drow >= draft_rows) {
        if (lead) report_error(status, kErrBadIndex);
        break;
      }
      // q over this slice of the full vocabulary (0 outside the draft vocabulary)
      const float* dr = dlogits + (int64_t)drow * ldd;
      const WarpParams PD = dparams[drow];
      if (vocab_ids) {
        for (int i = threadIdx.x; i < nl; i += kSampThreads) qs[i] = 0.f;
        __syncthreads();
        for (int j = threadIdx.x; j < Vd; j += kSampThreads) {
          const int64_t v = vocab_ids[j];
          if (v >= i0 && v < i0 + nl) {
            const float lp = warped_lp(PD, dr[j]);
            qs[v - i0] = lp == -INFINITY ? 0.f : expf(lp);
          }
        }
      } else {
        for (int i = threadIdx.x; i < nl; i += kSampThreads) {
          const float lp = i0 + i < Vd ? warped_lp(PD, dr[i0 + i]) : -INFINITY;
          qs[i] = lp == -INFINITY ? 0.f : expf(lp);
        }
      }
      cluster_sync_all();  // every slice of p and q is complete
      float zp = 1.f, zq = 1.f;  // p / zp and q / zq are the current distributions
      for (int ci = 0; ci < nk; ++ci) {
        const int c = kids[ci];
        const int tok = tokens[c];
        const bool in = tok >= 0 && tok < V;
        const int owner = in ? tok / len : 0, off = in ? tok - owner * len : 0;
        if (threadIdx.x == 0) {
          s_pt[0] = in ? dsmem_ld(dsmem_map(smem_u32(ps + off), owner)) : 0.f;
          s_pt[1] = in ? dsmem_ld(dsmem_map(smem_u32(qs + off), owner)) : 0.f;
        }
        __syncthreads();
        const float qx = s_pt[1] / zq;
        const float px = s_pt[0] / zp;
        __syncthreads();
        if (!(qx > 0.f)) continue;
        const float u = uniform(sd, rnd, static_cast<uint32_t>(cur + 1), static_cast<uint32_t>(ci), 1u);
        if (u < fminf(1.f, px / qx)) {
          chosen = c;
          break;
        }
        // reject: p <- max(p - q, 0) renormalised, only if that has mass
        float rs = 0.f;
        for (int i = threadIdx.x; i < nl; i += kSampThreads) rs += fmaxf(ps[i] / zp - qs[i] / zq, 0.f);
        const float R = row_allreduce(x, block_sum(rs, red), false);
        if (R > 0.f) {
          for (int i = threadIdx.x; i < nl; i += kSampThreads) ps[i] = fmaxf(ps[i] / zp - qs[i] / zq, 0.f);
          zp = R;
        }
        // q <- q without x, renormalised; stop when nothing is left (every
        // peer's read of q[x] came before the exchange barrier above)
        __syncthreads();
        if (in && owner == s && threadIdx.x == 0) qs[off] = 0.f;
        __syncthreads();
        float qsum = 0.f;
        for (int i = threadIdx.x; i < nl; i += kSampThreads) qsum += qs[i];
        const float Q = row_allreduce(x, block_sum(qsum, red), false);
        if (!(Q > 0.f)) break;
        zq = Q;
      }
      cluster_sync_all();  // no peer reads this step's p or q any more
      if (chosen >= 0) {
        if (lead) {
          accepted[na] = chosen;
          keep_slots[1 + na] = c0 + 1 + chosen;
        }
        ++na;
        cur = chosen;
        continue;
      }
    }
    // bonus ~ p: Gumbel-max over the slice, then over the cluster
    float bk = -INFINITY;
    int bi = INT32_MAX;
    for (int i = threadIdx.x; i < nl; i += kSampThreads) {
      const float w = ps[i];
      if (!(w > 0.f)) continue;
      const int gi = i0 + i;
      const float key =
          logf(w) - logf(-logf(uniform(sd, rnd, static_cast<uint32_t>(cur + 1), static_cast<uint32_t>(gi), 2u)));
      if (key > bk || (key == bk && gi < bi)) {
        bk = key;
        bi = gi;
      }
    }
    const int wp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ok = __shfl_xor_sync(0xffffffffu, bk, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ok > bk || (ok == bk && oi < bi)) {
        bk = ok;
        bi = oi;
      }
    }
    if (lane == 0) {
      s_key[wp] = bk;
      s_idx[wp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float gk = -INFINITY;
      int gi = INT32_MAX;
      for (int j = 0; j < kSampWarps; ++j)
        if (s_key[j] > gk || (s_key[j] == gk && s_idx[j] < gi)) {
          gk = s_key[j];
          gi = s_idx[j];
        }
      s_key[0] = gk;
      s_idx[0] = gi;
    }
    __syncthreads();
    float gk = s_key[0];
    int gi = s_idx[0];
    row_allbest(x, gk, gi);
    cluster_sync_all();  // peers may still read this CTA's exchange slot
    if (lead) {
      *bonus = gi == INT32_MAX ? 0 : gi;
      *n_accepted = na;
      *n_keep = na + 1;
    }
    return;
  }
  cluster_sync_all();
  if (lead) {
    *bonus = 0;
    *n_accepted = na;
    *n_keep = na + 1;
  }
}

// Dynamic shared memory of warp_sample_kernel: the staged slice (padded to
// 8 bytes) and the per-warp histograms of the radix select.
static size_t warp_sample_smem(int64_t V, int S) {
  const int64_t len = (V + S - 1) / S;
  return (size_t)(((len + 1) & ~int64_t(1)) * 4 + (int64_t)kSampWarps * 256 * 8);
}

// Cluster size for a row of V logits: slices of at least 2048 and at most
// kRowSliceMax floats, at most 8 CTAs. 0 = the row is too long.
static int row_slices(int64_t V) {
  int S = (int)((V + 2047) / 2048);
  if (S > kRowMaxSlices) S = kRowMaxSlices;
  if (S < 1) S = 1;
  return (V + S - 1) / S > kRowSliceMax ? 0 : S;
}

// The warp_sample_kernel instance whose candidate lists hold k draws.
using WarpSampleKernel = void (*)(const float*, int64_t, int, float, float, int, int, const int64_t*,
                                  const uint64_t*, const int32_t*, int, int, WarpParams*, int32_t*, float*);
static WarpSampleKernel warp_sample_instance(int64_t k) {
  static bool set = false;
  if (!set) {
    allow_max_dynamic_smem(warp_sample_kernel<4>);
    allow_max_dynamic_smem(warp_sample_kernel<8>);
    allow_max_dynamic_smem(warp_sample_kernel<kMaxK>);
    set = true;
  }
  return k <= 4 ? warp_sample_kernel<4> : k <= 8 ? warp_sample_kernel<8> : warp_sample_kernel<kMaxK>;
}

// Clusters of S warp_sample_kernel CTAs that can be resident at once, from
// the occupancy API; cached per instance, size, shared memory and device.
static int warp_sample_resident(WarpSampleKernel kern, int S, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<void*, int, size_t, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(reinterpret_cast<void*>(kern), S, smem, dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)S, 1);
  cfg.blockDim = dim3(kSampThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = n;
  return n;
}

// Cluster size of warp_sample_kernel for `rows` rows: the largest S up to
// row_slices(V) whose clusters for all rows are resident at once (slices of
// up to kSampSliceMax floats), else the fewest CTAs per row. 0 = the row is
// too long.
constexpr int kSampSliceMax = 32768;  // 128 KB staged + 64 KB of warp histograms
static int warp_sample_slices(int64_t V, int64_t rows, WarpSampleKernel kern) {
  const int most = row_slices(V);
  if (most == 0) return 0;
  int least = (int)((V + kSampSliceMax - 1) / kSampSliceMax);
  if (least > most) least = most;
  for (int S = most; S > least; --S)
    if (warp_sample_resident(kern, S, warp_sample_smem(V, S)) >= rows) return S;
  return least;
}

}  // namespace ssd

using namespace ssd;

extern "C" {

int ssd_warp_params(const float* logits, int64_t ld, int64_t rows, int64_t V, float temperature, float top_p,
                    void* params_out, void* stream) {
  if (rows <= 0 || V <= 0 || !(temperature > 0.f) || !(top_p > 0.f) || top_p > 1.f)
    return fail(SSD_ERR_INVALID, "ssd_warp_params: need rows, V > 0, temperature > 0, 0 < top_p <= 1");
  return launch_kernel("warp_params_kernel", warp_params_kernel, dim3((unsigned)rows), dim3(kSampThreads), 0,
                       static_cast<cudaStream_t>(stream), 1, 1, logits, ld, (int)V, temperature, top_p,
                       static_cast<WarpParams*>(params_out));
}

int ssd_warp_probs(const float* logits, int64_t ld, int64_t rows, int64_t V, const void* params, float* out,
                   int64_t ldo, void* stream) {
  if (rows <= 0 || V <= 0 || !logits || !params || !out || rows > 65535)
    return fail(SSD_ERR_INVALID, "ssd_warp_probs: bad arguments");
  const unsigned bx = (unsigned)((V + 1023) / 1024 < 64 ? (V + 1023) / 1024 : 64);
  return launch_kernel("warp_probs_kernel", warp_probs_kernel, dim3(bx, (unsigned)rows), dim3(1024), 0,
                       static_cast<cudaStream_t>(stream), 1, 1, logits, ld, (int)V,
                       static_cast<const WarpParams*>(params), out, ldo);
}

int ssd_gumbel_topk(const float* logits, int64_t ld, int64_t rows, int64_t V, const void* params, int64_t k,
                    const int64_t* vocab_ids, const uint64_t* seed, const int32_t* round, int64_t row_base,
                    int32_t* out_tok, float* out_logprob, void* stream) {
  if (k < 1 || k > kMaxK) return fail(SSD_ERR_UNSUPPORTED, "ssd_gumbel_topk: k must be 1..16");
  if (!seed) return fail(SSD_ERR_INVALID, "ssd_gumbel_topk: seed is NULL");
  if (rows <= 0 || rows > 65535 || V <= 0) return fail(SSD_ERR_INVALID, "ssd_gumbel_topk: bad shape");
  // a cluster of up to 8 CTAs per row, each over >= 4096 logits
  int slices = (int)((V + 4095) / 4096);
  if (slices > kGumbelMaxSlices) slices = kGumbelMaxSlices;
  return launch_kernel("gumbel_topk_kernel", gumbel_topk_kernel, dim3((unsigned)rows, (unsigned)slices),
                       dim3(kSampThreads), 0, static_cast<cudaStream_t>(stream), 1, (unsigned)slices, logits, ld,
                       (int)V,
                       static_cast<const WarpParams*>(params), (int)k, vocab_ids, seed, round, (int)row_base, out_tok,
                       out_logprob);
}

int ssd_warp_sample_topk(const float* logits, int64_t ld, int64_t rows, int64_t V, float temperature, float top_p,
                         int64_t keep_top, int64_t k, const int64_t* vocab_ids, const uint64_t* seed,
                         const int32_t* round, int64_t row_base, void* params_out, int32_t* out_tok,
                         float* out_logprob, void* stream) {
  if (keep_top < 0) return fail(SSD_ERR_INVALID, "ssd_warp_sample_topk: keep_top must be >= 0");
  if (rows <= 0 || rows > 65535 || V <= 0 || !logits || ld < V || !(temperature > 0.f) || !(top_p > 0.f) ||
      top_p > 1.f)
    return fail(SSD_ERR_INVALID, "ssd_warp_sample_topk: need rows, V > 0, temperature > 0, 0 < top_p <= 1");
  if (k < 0 || k > kMaxK) return fail(SSD_ERR_UNSUPPORTED, "ssd_warp_sample_topk: k must be 0..16");
  if (k > 0 && (!seed || !out_tok)) return fail(SSD_ERR_INVALID, "ssd_warp_sample_topk: NULL seed or output");
  if (k == 0 && !params_out) return fail(SSD_ERR_INVALID, "ssd_warp_sample_topk: nothing to compute");
  const WarpSampleKernel kern = warp_sample_instance(k);
  const int S = warp_sample_slices(V, rows, kern);
  if (S == 0)
    return fail(SSD_ERR_UNSUPPORTED, "ssd_warp_sample_topk: V = %lld exceeds %d", (long long)V,
                kRowMaxSlices * kRowSliceMax);
  const size_t smem = warp_sample_smem(V, S);
  return launch_kernel("warp_sample_kernel", kern, dim3((unsigned)S, (unsigned)rows),
                       dim3(kSampThreads),
                       smem, static_cast<cudaStream_t>(stream), (unsigned)S, 1u, logits, ld, (int)V, temperature,
                       top_p, (int)(keep_top < V ? keep_top : 0), (int)k, vocab_ids, seed, round, (int)row_base, 0,
                       static_cast<WarpParams*>(params_out), out_tok, out_logprob);
}

int ssd_sample_token(const float* logits, int64_t V, float temperature, float top_p, const uint64_t* seed,
                     const int32_t* round, int64_t row_id, int64_t stream_id, float* scratch, int32_t* out,
                     void* stream) {
  if (V <= 0 || !(temperature > 0.f) || !(top_p > 0.f) || top_p > 1.f || !seed || !out)
    return fail(SSD_ERR_INVALID, "ssd_sample_token: bad arguments");
  const int S = row_slices(V);
  if (S == 0) {  // rows too long for a cluster's shared memory: one CTA over global scratch
    if (!scratch) return fail(SSD_ERR_INVALID, "ssd_sample_token: scratch needed for V = %lld", (long long)V);
    return launch_kernel("sample_token_kernel", sample_token_kernel, dim3(1), dim3(kSampThreads), 0,
                         static_cast<cudaStream_t>(stream), 1, 1, logits, (int)V, temperature, top_p, seed, round,
                         (int)row_id, (int)stream_id, scratch, out);
  }
  const size_t smem = warp_sample_smem(V, S);
  return launch_kernel("warp_sample_kernel", warp_sample_instance(1), dim3((unsigned)S, 1u), dim3(kSampThreads), smem,
                       static_cast<cudaStream_t>(stream), (unsigned)S, 1u, logits, (int64_t)V, (int)V, temperature,
                       top_p, 0, 1, static_cast<const int64_t*>(nullptr), seed, round, (int)row_id, (int)stream_id,
                       static_cast<WarpParams*>(nullptr), out, static_cast<float*>(nullptr));
}

int ssd_tree_walk_sample(const int32_t* n_nodes, int64_t max_nodes, const int32_t* tokens, const int32_t* parents,
                         const int32_t* ranks, const int32_t* draft_pos, const int32_t* root_pos,
                         const float* target_logits, int64_t ldt, const void* target_params, int64_t V,
                         const float* draft_logits, int64_t ldd, const void* draft_params, int64_t draft_rows,
                         int64_t Vd, const int64_t* vocab_ids, const uint64_t* seed, const int32_t* round,
                         float* p_scratch, float* q_scratch, int32_t* accepted, int32_t* n_accepted, int32_t* bonus,
                         int32_t* keep_slots, int32_t* n_keep, uint32_t* status, void* stream) {
  if (max_nodes < 0 || max_nodes > 4096 || V <= 0 || Vd <= 0 || draft_rows <= 0 || !seed || !target_params ||
      !draft_params)
    return fail(SSD_ERR_INVALID, "ssd_tree_walk_sample: bad arguments");
  if (!vocab_ids && Vd > V) return fail(SSD_ERR_INVALID, "ssd_tree_walk_sample: draft vocabulary exceeds V");
  const int S = row_slices(V);
  if (S == 0) {  // vocabularies beyond the cluster's shared memory: one CTA over global scratch
    if (!p_scratch || !q_scratch) return fail(SSD_ERR_INVALID, "ssd_tree_walk_sample: scratch needed for this V");
    return launch_kernel("sample_verify_kernel", sample_verify_kernel, dim3(1), dim3(kSampThreads), 0,
                         static_cast<cudaStream_t>(stream), 1, 1, n_nodes, (int)max_nodes, tokens, parents, ranks,
                         draft_pos, root_pos, target_logits, ldt, static_cast<const WarpParams*>(target_params),
                         (int)V, draft_logits, ldd, static_cast<const WarpParams*>(draft_params), (int)draft_rows,
                         (int)Vd, vocab_ids, seed, round, p_scratch, q_scratch, accepted, n_accepted, bonus,
                         keep_slots, n_keep, status);
  }
  const size_t smem = (size_t)((V + S - 1) / S) * 8;  // p and q slices
  static bool set = false;
  if (!set) {
    allow_max_dynamic_smem(sample_verify_cluster_kernel);
    set = true;
  }
  return launch_kernel("sample_verify_cluster_kernel", sample_verify_cluster_kernel, dim3((unsigned)S, 1u),
                       dim3(kSampThreads), smem, static_cast<cudaStream_t>(stream), (unsigned)S, 1u, n_nodes,
                       (int)max_nodes, tokens, parents, ranks, draft_pos, root_pos, target_logits, ldt,
                       static_cast<const WarpParams*>(target_params), (int)V, draft_logits, ldd,
                       static_cast<const WarpParams*>(draft_params), (int)draft_rows, (int)Vd, vocab_ids, seed, round,
                       accepted, n_accepted, bonus, keep_slots, n_keep, status);
}

}  // extern "C"
