// GEMM family for the skinny (decode-time) matrix products of one SSD round.
//
// y[t, n] = sum_k x[t, k] * W[n, k] for T <= a few hundred token rows and a
// weight matrix W streamed once from HBM. The weights are the M operand
// ("swap-AB"): a CTA owns 128 output features x BN tokens, so the token count
// only sets the MMA N dimension and every weight byte is read exactly once.
//
// Two mainloops produce the same fp32 tile:
//   * tcgen05 (bf16): TMA -> 128B-swizzled SMEM ring -> tcgen05.mma (M=128,
//     N=BN, K=16) -> TMEM accumulator -> tcgen05.ld.
//   * SIMT (fp32): CUDA-core FFMA for the exact-parity fp32 tier.
// K is split over `splits` CTAs when the tile grid alone cannot fill the
// GPU; the split partials are summed by the last CTA to finish, in split
// order, so the result does not depend on scheduling or on the token count.
#pragma once

#include "common.cuh"

namespace ssd {

enum EpiKind : int {
  EPI_STORE = SSD_EPI_STORE,
  EPI_RESIDUAL = SSD_EPI_RESIDUAL,
  EPI_SWIGLU = SSD_EPI_SWIGLU,
  EPI_STORE_F32 = SSD_EPI_STORE_F32,
  EPI_QKV = SSD_EPI_QKV,
  EPI_ARGMAX = 17,
  EPI_TOPK = 18,
};

constexpr int kTileM = 128;    // output features per CTA tile
constexpr int kChunkK = 64;    // K elements per pipeline stage (128 bytes of bf16)
constexpr int kMaxTopK = 16;
constexpr int kSimtInvariantRows = 64;  // fp32 tier: split-K fixed for T <= this

struct EpiArgs {
  int kind;
  int act;
  const void* bias[3];
  void* out;
  int64_t ldo;
  float* resid;
  int64_t ldr;
  // fused QKV + RoPE + cache write
  int head_dim, n_q, n_kv;  // n_q / n_kv are feature counts (heads * head_dim)
  const float* rope_cos;
  const float* rope_sin;
  int max_pos;
  const int32_t* positions;
  const int32_t* slots;
  void* k_cache;
  void* v_cache;
  int64_t head_stride;
  int max_slots;
  // lm_head partial reductions: [T][tiles_m][rec]
  float* part;
  int topk;
  // RMSNorm folding (SsdRowNorm / SsdNormOut of the C ABI)
  const float* rn_ssq;  // input rows are resid * w: scale column t by rsqrt(sum ssq[t] / d + eps)
  int64_t rn_ld;
  int rn_parts, rn_d;
  float rn_eps;
  const void* no_w;  // residual epilogue also writes no_out = resid * no_w and per-tile sums of squares
  void* no_out;
  int64_t no_ldo;
  float* no_ssq;
  int64_t no_ld;
};

struct GemmShape {
  int T, K, N;        // token rows, reduction length, logical output features
  int n_seg;
  int seg_start[4];   // CONCAT: feature offset of each segment, seg_start[n_seg] = N
  int layout;         // SSD_SEG_CONCAT / SSD_SEG_PAIRS
  int BN;             // tokens per tile
  int splits;         // K splits
  int kchunks;        // ceil(K / 64)
  int stages;
  int tiles_m, tiles_n;
  int a_box;          // weight rows per TMA box (stream-K kernel: 128, 64 or 32)
  int n_major;        // grid x walks the token tiles (prefill: one weight tile's CTAs run together)
  uint32_t* counters;
  float* partials;
  uint32_t* status;
};

// One link of launch_chain (host side): the operands of launch_gemm.
struct ChainLinkHost {
  const void* x;
  int64_t ldx, K;
  int n_seg, layout;
  const void* w[3];
  int64_t rows[3];
  EpiArgs e;
};
// Up to 6 dependent decode-sized bf16 GEMMs (T <= 64) in one persistent
// launch (tc_chain_kernel); workspace as for launch_gemm.
int launch_chain(int n, const ChainLinkHost* links, int64_t T, void* workspace, int64_t workspace_bytes,
                 uint32_t* status, cudaStream_t stream);
// Workspace bytes launch_chain needs for T rows on the current device.
int64_t chain_workspace_need(int64_t T);

__device__ __forceinline__ int seg_of(const GemmShape& g, int n) {
  int s = 0;
#pragma unroll
  for (int i = 1; i < 3; ++i)
    if (i < g.n_seg && n >= g.seg_start[i]) s = i;
  return s;
}

template <typename T>
__device__ __forceinline__ float load_bias(const void* b, int i) {
  return b ? to_f32<T>(static_cast<const T*>(b)[i]) : 0.0f;
}

// Record layout of one lm_head partial: argmax -> {max1, idx1, max2};
// top-k -> {max, sumexp, val[k], idx[k]}.
__host__ __device__ inline int head_rec_size(int kind, int k) { return kind == EPI_ARGMAX ? 3 : 2 + 2 * k; }

// Per-CTA table of folded-RMSNorm row scales, one per owned token column.
__device__ __forceinline__ float* epi_scale_smem() {
  __shared__ float s_scale[256];
  return s_scale;
}

// Fill epi_scale_smem()[j] = rsqrt(sum(ssq[t, :parts]) / d + eps) for the
// owned columns c = c0 + j * cstep < ncols (t = t0 + c). 128 threads; one warp
// per column, lanes over the per-tile partial sums (up to 64 of them loaded
// at once, more in a second pass), four columns per warp in flight. The sum
// order is fixed (two lanes' halves, then a butterfly), so every consumer of
// the same ssq row computes the same scale. No barrier: the caller publishes
// the table.
__device__ __forceinline__ void epi_row_scales(const EpiArgs& e, int t0, int ncols, int c0, int cstep, int tid) {
  float* s_scale = epi_scale_smem();
  const int nsub = ncols > c0 ? (ncols - c0 + cstep - 1) / cstep : 0;
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int kB = 4;
  for (int j0 = warp; j0 < nsub; j0 += 4 * kB) {
    float acc[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int j = j0 + 4 * u;
      const float* ss = e.rn_ssq + (int64_t)(t0 + c0 + j * cstep) * e.rn_ld;
      const float a = (j < nsub && lane < e.rn_parts) ? ss[lane] : 0.f;
      const float b = (j < nsub && lane + 32 < e.rn_parts) ? ss[lane + 32] : 0.f;
      acc[u] = a + b;
    }
    if (e.rn_parts > 64) {
#pragma unroll
      for (int u = 0; u < kB; ++u) {
        const int j = j0 + 4 * u;
        if (j >= nsub) continue;
        const float* ss = e.rn_ssq + (int64_t)(t0 + c0 + j * cstep) * e.rn_ld;
        for (int i = lane + 64; i < e.rn_parts; i += 32) acc[u] += ss[i];
      }
    }
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const float v = warp_sum(acc[u]);
      const int j = j0 + 4 * u;
      if (lane == 0 && j < nsub) s_scale[j] = rsqrtf(v / (float)e.rn_d + e.rn_eps);
    }
  }
}

// Columns per batch in the epilogue loops: each batch issues its global
// loads (residual rows, positions, RoPE tables) together, so a batch costs
// one memory latency instead of one per column.
constexpr int kEpiBatch = 8;

// Apply the epilogue to a finished fp32 tile stage[c * 128 + r] (c = token
// within the tile, r = row within the 128-feature tile). Runs on 128
// threads; `tid` in [0, 128). `bar_id` names a barrier over those threads.
// Columns c0, c0 + cstep, ... < ncols are processed (a cluster splits the
// columns of one tile among its CTAs). `rn_applied`: the folded-RMSNorm row
// scales (e.rn_ssq) were already multiplied into the tile by the caller.
template <typename T>
__device__ void run_epilogue(float* stage, int tile_m, int t0, int ncols, const GemmShape& g, const EpiArgs& e,
                             int tid, int bar_id, int c0 = 0, int cstep = 1, bool rn_applied = false) {
  const int r = tid;
  if (e.rn_ssq && !rn_applied) {
    // Folded RMSNorm of the input rows: scale token column c by
    // rsqrt(mean of squares + eps).
    const float* s_scale = epi_scale_smem();
    const int nsub = ncols > c0 ? (ncols - c0 + cstep - 1) / cstep : 0;
    epi_row_scales(e, t0, ncols, c0, cstep, tid);
    named_bar_sync(bar_id, kTileM);
    for (int j = 0; j < nsub; ++j) stage[(c0 + j * cstep) * kTileM + r] *= s_scale[j];
    named_bar_sync(bar_id, kTileM);
  }
  if (e.kind == EPI_RESIDUAL && e.no_w) {
    // Residual update that also produces the next RMSNorm's input
    // (resid * w, bf16) and this tile's sums of squares per token.
    const int n = tile_m * kTileM + r;
    const bool in = n < g.N;
    const int s = in ? seg_of(g, n) : 0;
    const float b = in ? load_bias<T>(e.bias[s], n - g.seg_start[s]) : 0.f;
    const float wn = in ? to_f32<T>(static_cast<const T*>(e.no_w)[n]) : 0.f;
    for (int cb = c0; cb < ncols; cb += kEpiBatch * cstep) {
      float rv[kEpiBatch];
#pragma unroll
      for (int u = 0; u < kEpiBatch; ++u) {
        const int c = cb + u * cstep;
        rv[u] = (in && c < ncols) ? e.resid[(int64_t)(t0 + c) * e.ldr + n] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kEpiBatch; ++u) {
        const int c = cb + u * cstep;
        if (c >= ncols) break;
        const int t = t0 + c;
        float rn = 0.f;
        if (in) {
          rn = rv[u] + stage[c * kTileM + r] + b;
          e.resid[(int64_t)t * e.ldr + n] = rn;
          static_cast<T*>(e.no_out)[(int64_t)t * e.no_ldo + n] = from_f32<T>(rn * wn);
        }
        stage[c * kTileM + r] = rn * rn;
      }
    }
    named_bar_sync(bar_id, kTileM);
    const int warp = tid >> 5, lane = tid & 31;
    for (int c = c0 + warp * cstep; c < ncols; c += 4 * cstep) {
      const float* col = stage + c * kTileM;
      const float v = warp_sum((col[lane] + col[lane + 32]) + (col[lane + 64] + col[lane + 96]));
      if (lane == 0) e.no_ssq[(int64_t)(t0 + c) * e.no_ld + tile_m] = v;
    }
    return;
  }
  switch (e.kind) {
    case EPI_STORE:
    case EPI_STORE_F32:
    case EPI_RESIDUAL: {
      const int n = tile_m * kTileM + r;
      if (n >= g.N) return;
      const int s = seg_of(g, n);
      const float b = load_bias<T>(e.bias[s], n - g.seg_start[s]);
      if (e.kind == EPI_RESIDUAL) {
        for (int cb = c0; cb < ncols; cb += kEpiBatch * cstep) {
          float rv[kEpiBatch];
#pragma unroll
          for (int u = 0; u < kEpiBatch; ++u) {
            const int c = cb + u * cstep;
            rv[u] = c < ncols ? e.resid[(int64_t)(t0 + c) * e.ldr + n] : 0.f;
          }
#pragma unroll
          for (int u = 0; u < kEpiBatch; ++u) {
            const int c = cb + u * cstep;
            if (c < ncols) e.resid[(int64_t)(t0 + c) * e.ldr + n] = rv[u] + (stage[c * kTileM + r] + b);
          }
        }
        return;
      }
      for (int c = c0; c < ncols; c += cstep) {
        const int t = t0 + c;
        float v = stage[c * kTileM + r] + b;
        if (e.kind == EPI_STORE_F32) {
          static_cast<float*>(e.out)[(int64_t)t * e.ldo + n] = act_f(e.act, v);
        } else {
          static_cast<T*>(e.out)[(int64_t)t * e.ldo + n] = from_f32<T>(act_f(e.act, v));
        }
      }
      return;
    }
    case EPI_SWIGLU: {
      // PAIRS layout: rows 0..63 gate, rows 64..127 up, for features tile_m*64 + r.
      if (r >= 64) return;
      const int f = tile_m * 64 + r;
      const int F = g.seg_start[1];
      if (f >= F) return;
      const float bg = load_bias<T>(e.bias[0], f), bu = load_bias<T>(e.bias[1], f);
      for (int c = c0; c < ncols; c += cstep) {
        const float gv = stage[c * kTileM + r] + bg;
        const float uv = stage[c * kTileM + r + 64] + bu;
        static_cast<T*>(e.out)[(int64_t)(t0 + c) * e.ldo + f] = from_f32<T>(silu_f(gv) * uv);
      }
      return;
    }
    case EPI_QKV: {
      const int n = tile_m * kTileM + r;
      if (n >= g.N) return;
      const int hd = e.head_dim, half = hd >> 1;
      const bool is_q = n < e.n_q, is_k = !is_q && n < e.n_q + e.n_kv;
      const bool rope = is_q || is_k;
      const int local = is_q ? n : (is_k ? n - e.n_q : n - e.n_q - e.n_kv);
      const int head = local / hd, j = local - head * hd;
      const int partner = (j < half) ? r + half : r - half;  // same head, same tile (hd divides 128)
      const int fi = j < half ? j : j - half;
      for (int cb = c0; cb < ncols; cb += kEpiBatch * cstep) {
        // Batch the index loads, then the RoPE table loads that depend on them.
        int idx[kEpiBatch];
#pragma unroll
        for (int u = 0; u < kEpiBatch; ++u) {
          const int c = cb + u * cstep;
          idx[u] = c < ncols ? (rope ? e.positions[t0 + c] : e.slots[t0 + c]) : 0;
        }
        int slot[kEpiBatch];
        float cs[kEpiBatch], sn[kEpiBatch];
#pragma unroll
        for (int u = 0; u < kEpiBatch; ++u) {
          const int c = cb + u * cstep;
          slot[u] = (is_k && c < ncols) ? e.slots[t0 + c] : idx[u];
          cs[u] = 1.f;
          sn[u] = 0.f;
          if (rope && c < ncols) {
            int p = idx[u];
            if (p < 0 || p >= e.max_pos) {
              report_error(g.status, kErrBadIndex);
              p = 0;
            }
            cs[u] = e.rope_cos[(int64_t)p * half + fi];
            sn[u] = e.rope_sin[(int64_t)p * half + fi];
          }
        }
#pragma unroll
        for (int u = 0; u < kEpiBatch; ++u) {
          const int c = cb + u * cstep;
          if (c >= ncols) break;
          const int t = t0 + c;
          float v = stage[c * kTileM + r];
          if (rope) {
            const float o = stage[c * kTileM + partner];
            v = (j < half) ? (v * cs[u] - o * sn[u]) : (v * cs[u] + o * sn[u]);
          }
          if (is_q) {
            static_cast<T*>(e.out)[(int64_t)t * e.ldo + n] = from_f32<T>(v);
          } else {
            const int sl = slot[u];
            if (sl < 0 || sl >= e.max_slots) {
              report_error(g.status, kErrBadIndex);
              continue;
            }
            T* cache = static_cast<T*>(is_k ? e.k_cache : e.v_cache);
            cache[(int64_t)head * e.head_stride + (int64_t)sl * hd + j] = from_f32<T>(v);
          }
        }
      }
      return;
    }
    case EPI_ARGMAX:
    case EPI_TOPK: {
      // One warp per token column; lanes scan the 128 rows of the tile.
      const int warp = tid >> 5, lane = tid & 31;
      const int rec = head_rec_size(e.kind, e.topk);
      for (int c = c0 + warp * cstep; c < ncols; c += 4 * cstep) {
        const int t = t0 + c;
        float v[4];
        int idx[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rr = lane + 32 * i;
          idx[i] = tile_m * kTileM + rr;
          v[i] = (idx[i] < g.N) ? stage[c * kTileM + rr] : -INFINITY;
        }
        float* out = e.part + ((int64_t)t * g.tiles_m + tile_m) * rec;
        if (e.kind == EPI_ARGMAX) {
          // top-2 with first-index tie break for the max
          float m1 = -INFINITY, m2 = -INFINITY;
          int i1 = INT32_MAX;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (v[i] > m1 || (v[i] == m1 && idx[i] < i1)) {
              m2 = fmaxf(m2, m1);
              m1 = v[i];
              i1 = idx[i];
            } else {
              m2 = fmaxf(m2, v[i]);
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float om1 = __shfl_xor_sync(0xffffffffu, m1, o);
            const int oi1 = __shfl_xor_sync(0xffffffffu, i1, o);
            const float om2 = __shfl_xor_sync(0xffffffffu, m2, o);
            if (om1 > m1 || (om1 == m1 && oi1 < i1)) {
              m2 = fmaxf(m1, om2);
              m1 = om1;
              i1 = oi1;
            } else {
              m2 = fmaxf(m2, om1);
            }
          }
          if (lane == 0) {
            out[0] = m1;
            out[1] = __int_as_float(i1);
            out[2] = m2;
          }
        } else {
          float m = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
          m = warp_max(m);
          float s = 0.f;
#pragma unroll
          for (int i = 0; i < 4; ++i) s += (v[i] == -INFINITY) ? 0.f : expf(v[i] - m);
          s = warp_sum(s);
          if (lane == 0) {
            out[0] = m;
            out[1] = s;
          }
          // k rounds of (value desc, index asc) extraction
          for (int q = 0; q < e.topk; ++q) {
            float bv = -INFINITY;
            int bi = INT32_MAX, bslot = -1;
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (v[i] > bv || (v[i] == bv && idx[i] < bi)) {
                bv = v[i];
                bi = idx[i];
                bslot = i;
              }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
              const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
              const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
              if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
              }
            }
            if (lane == 0) {
              out[2 + q] = bv;
              out[2 + e.topk + q] = __int_as_float(bi);
            }
            // remove the winner from its owner lane
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (bslot == i && idx[i] == bi) v[i] = -INFINITY, idx[i] = INT32_MAX;
          }
        }
      }
      return;
    }
    default:
      return;
  }
}

// Sum split-K partials (last CTA of a tile does it) and run the epilogue.
// stage: [BN][128] fp32 tile of this CTA's split. flag: shared int.
template <typename T>
__device__ void finish_tile(float* stage, int* flag, int tile_m, int tile_n, int split, const GemmShape& g,
                            const EpiArgs& e, int tid, int bar_id) {
  const int t0 = tile_n * g.BN;
  const int ncols = min(g.BN, g.T - t0);
  if (g.splits > 1) {
    const int64_t tile_id = (int64_t)tile_n * g.tiles_m + tile_m;
    float* mine = g.partials + ((tile_id * g.splits + split) * g.BN) * kTileM;
    for (int c = 0; c < ncols; ++c) mine[c * kTileM + tid] = stage[c * kTileM + tid];
    __threadfence();
    named_bar_sync(bar_id, 128);
    if (tid == 0) {
      const uint32_t prev = atomicAdd(&g.counters[tile_id], 1u);
      *flag = (prev == (uint32_t)(g.splits - 1)) ? 1 : 0;
    }
    named_bar_sync(bar_id, 128);
    if (*flag == 0) return;
    __threadfence();
    for (int c = 0; c < ncols; ++c) {
      float acc = 0.f;
      for (int s = 0; s < g.splits; ++s)
        acc += __ldcg(g.partials + ((tile_id * g.splits + s) * g.BN + c) * kTileM + tid);
      stage[c * kTileM + tid] = acc;
    }
    if (tid == 0) g.counters[tile_id] = 0u;  // ready for the next launch
    named_bar_sync(bar_id, 128);
  }
  run_epilogue<T>(stage, tile_m, t0, ncols, g, e, tid, bar_id);
}

}  // namespace ssd
