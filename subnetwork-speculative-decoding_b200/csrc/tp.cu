// Tensor parallelism over NVLink peer memory (one process per GPU).
//
// Tensor-parallel Llama layout: q/k/v and gate/up are split by output
// features (heads, FFN columns), o_proj and down_proj by input features, so
// each rank's o_proj / down_proj GEMM produces a partial sum of the full
// [T, d] output that the ranks must add up; the lm_head is split by
// vocabulary rows, so each rank scores a slice of the vocabulary and the
// per-row winners are merged across ranks.
//
// Exchange memory: a "region" of identical layout on every rank, mapped into
// every rank's address space (SsdTpGroup::peer_region). Layout (bytes):
//   flags   [2 channels][2 phases][kTpMaxBlocks][8 sources] u32
//   epochs  [2 channels][kTpMaxBlocks] u32   (this rank's own counters)
//   records [max_rows][kTpRecFloats] f32     (head merge input)
//   partial [2 parities][max_rows][d] f32    (row-parallel GEMM output)
//
// Synchronisation: block b of a kernel meets block b of the same kernel on
// every other rank. Each block counts its uses in its epoch counter (the same
// sequence on every rank), stores the epoch into flags[ch][phase][b][me] of
// every rank with a system-scope release and polls its own
// flags[ch][phase][b][*] with system-scope acquires until every source has
// reached the epoch (see tp_meet). Polls are bounded (ssd_tp_set_spin_limit):
// on timeout the block sets the status timeout bit and goes on (results are
// then garbage but no GPU waits forever). Flags only grow, so they never need a
// reset. Blocks wait only on blocks of other GPUs, and each kernel's blocks
// fit on the GPU together, so a wait cannot block the block it waits for.
// No multicast objects or multicast loads are used.
//
// All-reduce buffer reuse: consecutive all-reduce calls alternate the two
// partial buffers. A rank signals a call only after all its earlier kernels
// have completed (programmatic-launch wait first), so when any rank passes the
// meeting of call k + 1, every rank has finished reading the partials of call
// k; the GEMM of call k + 2, which overwrites them, comes later still.
#include <atomic>

#include "gemm.cuh"
#include "host.cuh"

namespace ssd {

constexpr int kTpMaxRanks = SSD_TP_MAX_RANKS;
constexpr int kTpMaxBlocks = 1024;
constexpr int kTpRecFloats = 2 + 2 * 16;  // largest head record: top-k with k = 16
constexpr int kTpChanAllReduce = 0, kTpChanHead = 1;
constexpr uint32_t kTpSpinLimit = 1u << 22;  // default polls of ~100 ns: ~0.4 s and more
constexpr int kTpThreads = 128;

constexpr int64_t kTpFlagBytes = 2LL * 2 * kTpMaxBlocks * kTpMaxRanks * 4;
constexpr int64_t kTpEpochBytes = 2LL * kTpMaxBlocks * 4;

__host__ __device__ inline int64_t tp_align(int64_t x) { return (x + 255) & ~int64_t(255); }
__host__ __device__ inline int64_t tp_rec_offset() { return tp_align(kTpFlagBytes + kTpEpochBytes); }
__host__ __device__ inline int64_t tp_part_offset(int64_t max_rows) {
  return tp_align(tp_rec_offset() + max_rows * kTpRecFloats * 4);
}
__host__ __device__ inline int64_t tp_region_bytes(int64_t max_rows, int64_t d) {
  return tp_align(tp_part_offset(max_rows) + 2 * max_rows * d * 4);
}

// Kernel-side view of a group.
struct TpDev {
  uint8_t* region[kTpMaxRanks];
  int rank, world;
  int64_t max_rows, d;
  uint32_t spin_limit;  // polls before a meeting gives up
};

__device__ __forceinline__ uint32_t* tp_flag(uint8_t* region, int ch, int phase, int b, int src) {
  return reinterpret_cast<uint32_t*>(region) + (((int64_t)ch * 2 + phase) * kTpMaxBlocks + b) * kTpMaxRanks + src;
}
__device__ __forceinline__ uint32_t* tp_epoch(uint8_t* region, int ch, int b) {
  return reinterpret_cast<uint32_t*>(region + kTpFlagBytes) + (int64_t)ch * kTpMaxBlocks + b;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Next epoch of block b on channel ch (thread 0 only; the same value on every
// rank because every rank runs the same sequence of calls).
__device__ __forceinline__ uint32_t tp_next_epoch(const TpDev& g, int ch, int b) {
  uint32_t* e = tp_epoch(g.region[g.rank], ch, b);
  const uint32_t v = *e + 1;
  *e = v;
  return v;
}

// Block-wide meeting of block b with its counterparts on every rank. Thread
// p (< world) signals rank p and waits for rank p's signal, so the peers are
// polled in parallel. What a meeting orders is either data written by kernels
// that completed before this one started (the programmatic-launch wait comes
// first, so those writes are visible to this thread) or loads whose values
// this block has already consumed (the __syncthreads below orders them before
// the signalling thread's store). The signal is a system-scope release store,
// which is cumulative: everything this thread has observed is ordered before
// it. The poll is a system-scope acquire load, so the peer data read after
// the meeting (with L1 bypassed, __ldcg) is at least as new as the signal.
// Returns false on timeout.
__device__ bool tp_meet(const TpDev& g, int ch, int phase, int b, uint32_t epoch, uint32_t* status) {
  __syncthreads();
  int ok = 1;
  if (threadIdx.x < g.world && threadIdx.x != g.rank) {  // (meeting oneself needs no flag)
    const int p = threadIdx.x;
    st_release_sys(tp_flag(g.region[p], ch, phase, b, g.rank), epoch);
    const uint32_t* f = tp_flag(g.region[g.rank], ch, phase, b, p);
    uint32_t it = 0;
    while ((int32_t)(ld_acquire_sys(f) - epoch) < 0) {
      if (++it > g.spin_limit) {
        report_error(status, kErrWaitTimeout);
        ok = 0;
        break;
      }
      __nanosleep(20);
    }
  }
  return __syncthreads_and(ok) != 0;
}

// ------------------------------------------------- all-reduce + residual
// One-shot: block b owns the 128-feature tile `tile` of tokens [t0, t1).
// After one meeting (every rank's partial of this parity is complete) it
// reads the tile from every rank's partial (peer loads over NVLink), sums in
// rank order (the same bits on every rank), adds the sum to the residual and
// writes the folded RMSNorm input and the tile's sums of squares,
// bit-identical to ssd_linear's residual epilogue. Four tokens per pass: their
// loads are in flight together and warp u reduces token u's squares.
template <typename T>
__global__ void __launch_bounds__(kTpThreads) tp_allreduce_kernel(TpDev g, int parity, int T_rows, int tiles, int tpb,
                                                                  float* resid, int64_t ldr, SsdNormOut no,
                                                                  uint32_t* status) {
  constexpr int kU = 4;
  __shared__ float s_sq[kU][kTpThreads];
  __shared__ uint32_t s_epoch;
  const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = b % tiles, grp = b / tiles;
  const int t0 = grp * tpb, t1 = min(T_rows, t0 + tpb);
  const int64_t d = g.d, n = (int64_t)tile * 128 + tid;
  pdl_wait();  // the partials come from the preceding GEMM
  if (tid == 0) s_epoch = tp_next_epoch(g, kTpChanAllReduce, b);
  __syncthreads();
  tp_meet(g, kTpChanAllReduce, 0, b, s_epoch, status);
  pdl_trigger();
  const int64_t po = tp_part_offset(g.max_rows) + (int64_t)parity * g.max_rows * d * 4;
  const float* part[kTpMaxRanks];
#pragma unroll
  for (int p = 0; p < kTpMaxRanks; ++p)
    part[p] = p < g.world ? reinterpret_cast<const float*>(g.region[p] + po) : nullptr;
  const T* w = static_cast<const T*>(no.weight);
  const float wn = w ? to_f32<T>(w[n]) : 0.f;
  for (int tb = t0; tb < t1; tb += kU) {
    float v[kU][kTpMaxRanks], rv[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = tb + u;
#pragma unroll
      for (int p = 0; p < kTpMaxRanks; ++p)
        v[u][p] = (t < t1 && p < g.world) ? __ldcg(part[p] + (int64_t)t * d + n) : 0.f;
      rv[u] = t < t1 ? resid[(int64_t)t * ldr + n] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = tb + u;
      float acc = 0.f;
#pragma unroll
      for (int p = 0; p < kTpMaxRanks; ++p)
        if (p < g.world) acc += v[u][p];
      const float rn = rv[u] + acc;
      if (t < t1) {
        resid[(int64_t)t * ldr + n] = rn;
        if (w) static_cast<T*>(no.out)[(int64_t)t * no.ldo + n] = from_f32<T>(rn * wn);
      }
      s_sq[u][tid] = rn * rn;
    }
    if (!w) continue;
    __syncthreads();
    if (warp < kU && tb + warp < t1) {
      const float* q = s_sq[warp];
      const float s = warp_sum((q[lane] + q[lane + 32]) + (q[lane + 64] + q[lane + 96]));
      if (lane == 0) no.ssq[(int64_t)(tb + warp) * no.ld_ssq + tile] = s;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------ head merge
// Block t merges row t's records of all ranks (this rank's were written by
// the head reducer into its region). Phase 0: all records written. Phase 1:
// all ranks done reading, so the next head call may overwrite the records.
__global__ void tp_argmax_merge_kernel(TpDev g, int32_t* out_idx, float* out_max, float* out_gap, uint32_t* status) {
  const int t = blockIdx.x;
  pdl_wait();
  __shared__ uint32_t s_epoch;
  __shared__ float s_rec[kTpMaxRanks * 3];
  if (threadIdx.x == 0) s_epoch = tp_next_epoch(g, kTpChanHead, t);
  __syncthreads();
  const uint32_t epoch = s_epoch;
  tp_meet(g, kTpChanHead, 0, t, epoch, status);
  const int64_t ro = tp_rec_offset();
  if (threadIdx.x < g.world * 3) {
    const int p = threadIdx.x / 3, j = threadIdx.x % 3;
    s_rec[threadIdx.x] = __ldcg(reinterpret_cast<const float*>(g.region[p] + ro) + (int64_t)t * 3 + j);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // ranks in order: on equal maxima the lower rank holds the lower index
    float m1 = -INFINITY, m2 = -INFINITY;
    int i1 = INT32_MAX;
    for (int p = 0; p < g.world; ++p) {
      const float a = s_rec[p * 3], b2 = s_rec[p * 3 + 2];
      const int ai = __float_as_int(s_rec[p * 3 + 1]);
      if (a > m1 || (a == m1 && ai < i1)) {
        m2 = fmaxf(m1, b2);
        m1 = a;
        i1 = ai;
      } else {
        m2 = fmaxf(m2, a);
      }
    }
    out_idx[t] = i1;
    if (out_max) out_max[t] = m1;
    if (out_gap) out_gap[t] = m1 - m2;
  }
  tp_meet(g, kTpChanHead, 1, t, epoch, status);
  pdl_trigger();
}

__global__ void tp_topk_merge_kernel(TpDev g, int k, const int64_t* vocab_ids, int32_t* out_tok, float* out_lp,
                                     uint32_t* status) {
  const int t = blockIdx.x;
  const int rec = 2 + 2 * k;
  pdl_wait();
  __shared__ uint32_t s_epoch;
  __shared__ float s_rec[kTpMaxRanks * kTpRecFloats];
  if (threadIdx.x == 0) s_epoch = tp_next_epoch(g, kTpChanHead, t);
  __syncthreads();
  const uint32_t epoch = s_epoch;
  tp_meet(g, kTpChanHead, 0, t, epoch, status);
  const int64_t ro = tp_rec_offset();
  for (int i = threadIdx.x; i < g.world * rec; i += blockDim.x) {
    const int p = i / rec, j = i % rec;
    s_rec[i] = __ldcg(reinterpret_cast<const float*>(g.region[p] + ro) + (int64_t)t * rec + j);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // global log-sum-exp from the ranks' {max, sumexp}, then a k-way merge of
    // the ranks' sorted lists (value desc, index asc)
    float M = -INFINITY;
    for (int p = 0; p < g.world; ++p) M = fmaxf(M, s_rec[p * rec]);
    float S = 0.f;
    for (int p = 0; p < g.world; ++p) {
      const float mp = s_rec[p * rec];
      if (mp != -INFINITY) S += s_rec[p * rec + 1] * expf(mp - M);
    }
    const float lse = M + logf(S);
    int head[kTpMaxRanks];
    for (int p = 0; p < kTpMaxRanks; ++p) head[p] = 0;
    for (int q = 0; q < k; ++q) {
      float bv = -INFINITY;
      int bi = INT32_MAX, bp = -1;
      for (int p = 0; p < g.world; ++p) {
        if (head[p] >= k) continue;
        const float v = s_rec[p * rec + 2 + head[p]];
        const int ix = __float_as_int(s_rec[p * rec + 2 + k + head[p]]);
        if (v > bv || (v == bv && ix < bi)) {
          bv = v;
          bi = ix;
          bp = p;
        }
      }
      if (bp >= 0) head[bp] += 1;
      const int tok = (bi == INT32_MAX) ? -1 : (vocab_ids ? (int)vocab_ids[bi] : bi);
      out_tok[(int64_t)t * k + q] = tok;
      out_lp[(int64_t)t * k + q] = (bi == INT32_MAX) ? -INFINITY : bv - lse;
    }
  }
  tp_meet(g, kTpChanHead, 1, t, epoch, status);
  pdl_trigger();
}

// ----------------------------------------------------- seeded weight fill
// out[i, j] = scale * std * N(0, 1) drawn from Philox4x32-10 with key `seed`
// and counter (global index lo, hi, stream lo, hi), Box-Muller on two of the
// four outputs. The global index is (row0 + i) * full_cols + col0 + j.
template <typename T>
__global__ void fill_normal_kernel(T* out, int64_t rows, int64_t cols, int64_t ld, int64_t row0, int64_t col0,
                                   int64_t full_cols, uint64_t seed, uint64_t stream_id, float std, float scale) {
  const int64_t n = rows * cols;
  const uint2 key = make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / cols, j = e - i * cols;
    const uint64_t gidx = static_cast<uint64_t>((row0 + i) * full_cols + col0 + j);
    const uint4 r = philox4x32_10(make_uint4(static_cast<uint32_t>(gidx), static_cast<uint32_t>(gidx >> 32),
                                             static_cast<uint32_t>(stream_id), static_cast<uint32_t>(stream_id >> 32)),
                                  key);
    const float u1 = u01(r.x), u2 = u01(r.y);
    const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    out[i * ld + j] = from_f32<T>(z * std * scale);
  }
}

namespace {
std::atomic<uint32_t> g_tp_spin_limit{kTpSpinLimit};

int tp_dev(const SsdTpGroup* g, TpDev* out, const char* who) {
  if (!g) return fail(SSD_ERR_INVALID, "%s: group is NULL", who);
  if (g->world < 1 || g->world > kTpMaxRanks || g->rank < 0 || g->rank >= g->world)
    return fail(SSD_ERR_INVALID, "%s: rank %d / world %d invalid (world <= %d)", who, g->rank, g->world, kTpMaxRanks);
  for (int p = 0; p < g->world; ++p)
    if (!g->peer_region[p]) return fail(SSD_ERR_INVALID, "%s: peer_region[%d] is NULL", who, p);
  *out = TpDev{};
  for (int p = 0; p < g->world; ++p) out->region[p] = static_cast<uint8_t*>(g->peer_region[p]);
  out->rank = g->rank;
  out->world = g->world;
  out->max_rows = g->max_rows;
  out->d = g->d;
  out->spin_limit = g_tp_spin_limit.load(std::memory_order_relaxed);
  return SSD_OK;
}
}  // namespace

// Head reducers (layer.cu), launched here in their record mode.
__global__ void argmax_reduce_kernel(const float* part, int tiles, int32_t* out_idx, float* out_max, float* out_gap,
                                     float* rec_out, int idx_offset);
__global__ void topk_reduce_kernel(const float* part, int tiles, int k, const int64_t* vocab_ids, int32_t* out_tok,
                                   float* out_lp, float* rec_out, int idx_offset);

}  // namespace ssd

using namespace ssd;

extern "C" {

int64_t ssd_tp_region_bytes(int64_t max_rows, int64_t d) {
  if (max_rows < 1 || d < 1) return -1;
  return tp_region_bytes(max_rows, d);
}

uint32_t ssd_tp_set_spin_limit(uint32_t polls) {
  return g_tp_spin_limit.exchange(polls ? polls : kTpSpinLimit);
}

int64_t ssd_tp_partial_offset(int64_t max_rows, int64_t d, int parity) {
  if (max_rows < 1 || d < 1 || parity < 0 || parity > 1) return -1;
  return tp_part_offset(max_rows) + parity * max_rows * d * 4;
}

int ssd_tp_allreduce_residual(const SsdTpGroup* grp, int parity, int64_t T, float* resid, int64_t ldr,
                              const SsdNormOut* norm_out, int dtype, uint32_t* status, void* stream) {
  TpDev g;
  if (const int rc = tp_dev(grp, &g, "ssd_tp_allreduce_residual")) return rc;
  if (T < 1 || T > g.max_rows) return fail(SSD_ERR_INVALID, "ssd_tp_allreduce_residual: T = %lld outside 1..%lld",
                                           (long long)T, (long long)g.max_rows);
  if (!resid || ldr < g.d) return fail(SSD_ERR_INVALID, "ssd_tp_allreduce_residual: bad residual");
  if (g.d % 128)
    return fail(SSD_ERR_UNSUPPORTED, "ssd_tp_allreduce_residual: d = %lld is not a multiple of 128", (long long)g.d);
  if (parity != 0 && parity != 1) return fail(SSD_ERR_INVALID, "ssd_tp_allreduce_residual: parity must be 0 or 1");
  if (dtype != SSD_BF16 && dtype != SSD_F32) return fail(SSD_ERR_INVALID, "ssd_tp_allreduce_residual: bad dtype");
  SsdNormOut no{};
  if (norm_out) {
    no = *norm_out;
    if (!no.weight || !no.out || !no.ssq) return fail(SSD_ERR_INVALID, "ssd_tp_allreduce_residual: partial norm_out");
  }
  const int tiles = (int)(g.d / 128);
  // about four blocks per SM in all, each over a run of tokens
  const int target = 4 * device_sms();
  int groups = target / tiles;
  if (groups < 1) groups = 1;
  if (groups > T) groups = (int)T;
  const int tpb = (int)((T + groups - 1) / groups);
  groups = (int)((T + tpb - 1) / tpb);
  const int blocks = tiles * groups;
  if (blocks > kTpMaxBlocks) return fail(SSD_ERR_UNSUPPORTED, "ssd_tp_allreduce_residual: too many blocks");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SSD_BF16)
    return launch_kernel("tp_allreduce_kernel", tp_allreduce_kernel<bf16>, dim3(blocks), dim3(kTpThreads), 0, s, 1, 1,
                         g, parity, (int)T, tiles, tpb, resid, ldr, no, status);
  return launch_kernel("tp_allreduce_kernel", tp_allreduce_kernel<float>, dim3(blocks), dim3(kTpThreads), 0, s, 1, 1,
                       g, parity, (int)T, tiles, tpb, resid, ldr, no, status);
}

int ssd_tp_head_argmax(const SsdTpGroup* grp, const void* x, int64_t ldx, int64_t T, int64_t K, const void* w,
                       int64_t vocab_shard, int64_t vocab_offset, int32_t* out_idx, float* out_max, float* out_gap,
                       int dtype, void* workspace, int64_t workspace_bytes, const SsdRowNorm* in_norm,
                       uint32_t* status, void* stream) {
  TpDev g;
  if (const int rc = tp_dev(grp, &g, "ssd_tp_head_argmax")) return rc;
  if (T < 1 || T > g.max_rows || T > kTpMaxBlocks)
    return fail(SSD_ERR_INVALID, "ssd_tp_head_argmax: T = %lld outside 1..%lld", (long long)T, (long long)g.max_rows);
  if (!out_idx) return fail(SSD_ERR_INVALID, "ssd_tp_head_argmax: out_idx is NULL");
  if (vocab_offset < 0 || vocab_offset + vocab_shard > INT32_MAX)
    return fail(SSD_ERR_INVALID, "ssd_tp_head_argmax: vocabulary offset out of range");
  const int64_t tiles = (vocab_shard + 127) / 128;
  const int64_t need = kCounterBytes + T * tiles * 3 * 4;
  if (!workspace || need > workspace_bytes) return fail(SSD_ERR_WORKSPACE, "ssd_tp_head_argmax: workspace too small");
  EpiArgs e{};
  e.kind = EPI_ARGMAX;
  e.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
  if (in_norm) {
    e.rn_ssq = in_norm->ssq;
    e.rn_ld = in_norm->ld;
    e.rn_parts = (int)in_norm->parts;
    e.rn_d = (int)in_norm->d;
    e.rn_eps = in_norm->eps;
    if (dtype != SSD_BF16) return fail(SSD_ERR_UNSUPPORTED, "ssd_tp_head_argmax: folded norms need bf16");
  }
  const void* ws[1] = {w};
  int64_t rows[1] = {vocab_shard};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = launch_gemm(x, ldx, T, K, 1, ws, rows, SSD_SEG_CONCAT, e, dtype, workspace, workspace_bytes, status, s,
                       T * tiles * 3 * 4);
  if (rc) return rc;
  float* rec = reinterpret_cast<float*>(g.region[g.rank] + tp_rec_offset());
  rc = launch_kernel("argmax_reduce_kernel", argmax_reduce_kernel, dim3((unsigned)T), dim3(256), 0, s, 1, 1, e.part,
                     (int)tiles, (int32_t*)nullptr, (float*)nullptr, (float*)nullptr, rec, (int)vocab_offset);
  if (rc) return rc;
  return launch_kernel("tp_argmax_merge_kernel", tp_argmax_merge_kernel, dim3((unsigned)T), dim3(32), 0, s, 1, 1, g,
                       out_idx, out_max, out_gap, status);
}

int ssd_tp_head_topk(const SsdTpGroup* grp, const void* x, int64_t ldx, int64_t T, int64_t K, const void* w,
                     int64_t vocab_shard, int64_t vocab_offset, const int64_t* vocab_ids, int64_t k, int32_t* out_tok,
                     float* out_logprob, int dtype, void* workspace, int64_t workspace_bytes,
                     const SsdRowNorm* in_norm, uint32_t* status, void* stream) {
  TpDev g;
  if (const int rc = tp_dev(grp, &g, "ssd_tp_head_topk")) return rc;
  if (T < 1 || T > g.max_rows || T > kTpMaxBlocks)
    return fail(SSD_ERR_INVALID, "ssd_tp_head_topk: T = %lld outside 1..%lld", (long long)T, (long long)g.max_rows);
  if (k < 1 || k > kMaxTopK || k > vocab_shard) return fail(SSD_ERR_UNSUPPORTED, "ssd_tp_head_topk: k must be 1..16");
  if (!out_tok || !out_logprob) return fail(SSD_ERR_INVALID, "ssd_tp_head_topk: NULL output");
  if (vocab_offset < 0 || vocab_offset + vocab_shard > INT32_MAX)
    return fail(SSD_ERR_INVALID, "ssd_tp_head_topk: vocabulary offset out of range");
  const int64_t tiles = (vocab_shard + 127) / 128;
  const int64_t rec = 2 + 2 * k;
  const int64_t need = kCounterBytes + T * tiles * rec * 4;
  if (!workspace || need > workspace_bytes) return fail(SSD_ERR_WORKSPACE, "ssd_tp_head_topk: workspace too small");
  if (tiles > 1024) return fail(SSD_ERR_UNSUPPORTED, "ssd_tp_head_topk: more than 1024 vocab tiles per rank");
  EpiArgs e{};
  e.kind = EPI_TOPK;
  e.topk = (int)k;
  e.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
  if (in_norm) {
    e.rn_ssq = in_norm->ssq;
    e.rn_ld = in_norm->ld;
    e.rn_parts = (int)in_norm->parts;
    e.rn_d = (int)in_norm->d;
    e.rn_eps = in_norm->eps;
    if (dtype != SSD_BF16) return fail(SSD_ERR_UNSUPPORTED, "ssd_tp_head_topk: folded norms need bf16");
  }
  const void* ws[1] = {w};
  int64_t rows[1] = {vocab_shard};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = launch_gemm(x, ldx, T, K, 1, ws, rows, SSD_SEG_CONCAT, e, dtype, workspace, workspace_bytes, status, s,
                       T * tiles * rec * 4);
  if (rc) return rc;
  float* recp = reinterpret_cast<float*>(g.region[g.rank] + tp_rec_offset());
  rc = launch_kernel("topk_reduce_kernel", topk_reduce_kernel, dim3((unsigned)T), dim3(256), 0, s, 1, 1, e.part,
                     (int)tiles, (int)k, (const int64_t*)nullptr, (int32_t*)nullptr, (float*)nullptr, recp,
                     (int)vocab_offset);
  if (rc) return rc;
  return launch_kernel("tp_topk_merge_kernel", tp_topk_merge_kernel, dim3((unsigned)T), dim3(64), 0, s, 1, 1, g,
                       (int)k, vocab_ids, out_tok, out_logprob, status);
}

int ssd_fill_normal(void* out, int64_t rows, int64_t cols, int64_t ld, int64_t row0, int64_t col0, int64_t full_cols,
                    uint64_t seed, uint64_t stream_id, float std, float scale, int dtype, void* stream) {
  if (!out || rows < 0 || cols < 0 || ld < cols || row0 < 0 || col0 < 0 || col0 + cols > full_cols)
    return fail(SSD_ERR_INVALID, "ssd_fill_normal: bad shape");
  if (rows == 0 || cols == 0) return SSD_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t want = (rows * cols + 255) / 256, cap = 16LL * device_sms();
  const unsigned blocks = (unsigned)(want < cap ? want : cap);
  if (dtype == SSD_BF16)
    return launch_kernel("fill_normal_kernel", fill_normal_kernel<bf16>, dim3(blocks), dim3(256), 0, s, 1, 1,
                         static_cast<bf16*>(out), rows, cols, ld, row0, col0, full_cols, seed, stream_id, std, scale);
  if (dtype == SSD_F32)
    return launch_kernel("fill_normal_kernel", fill_normal_kernel<float>, dim3(blocks), dim3(256), 0, s, 1, 1,
                         static_cast<float*>(out), rows, cols, ld, row0, col0, full_cols, seed, stream_id, std, scale);
  return fail(SSD_ERR_INVALID, "ssd_fill_normal: bad dtype");
}

}  // extern "C"
