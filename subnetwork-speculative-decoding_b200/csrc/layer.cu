// Layer-level entry points: embedding gather, RMSNorm, the fused linear
// family (plain / residual / SwiGLU / QKV+RoPE+KV write) and the lm_head
// heads (argmax for verification, log-softmax top-k for drafting).
#include <cstring>

#include "gemm.cuh"
#include "host.cuh"

namespace ssd {

// ---------------------------------------------------------------- embedding
template <typename T>
__global__ void embed_kernel(const int32_t* ids, const T* table, int64_t vocab, int64_t d, float* out,
                             SsdNormOut no, uint32_t* status) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) report_error(status, kErrBadIndex);
    id = 0;
  }
  const T* row = table + (int64_t)id * d;
  if (!no.weight) {
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x) out[(int64_t)t * d + i] = to_f32<T>(row[i]);
    return;
  }
  // also the next RMSNorm's input (row * w) and per-128-feature sums of
  // squares, in the same tile partition as the GEMM epilogues (warp k sums
  // tiles k, k + 8, ... with a fixed shuffle order)
  const T* w = static_cast<const T*>(no.weight);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (int)((d + 127) / 128);
  for (int tl = warp; tl < tiles; tl += blockDim.x / 32) {
    float sq[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t i = (int64_t)tl * 128 + lane + 32 * k;
      float v = 0.f;
      if (i < d) {
        v = to_f32<T>(row[i]);
        out[(int64_t)t * d + i] = v;
        static_cast<T*>(no.out)[(int64_t)t * no.ldo + i] = from_f32<T>(v * to_f32<T>(w[i]));
      }
      sq[k] = v * v;
    }
    const float ssq = warp_sum((sq[0] + sq[1]) + (sq[2] + sq[3]));
    if (lane == 0) no.ssq[(int64_t)t * no.ld_ssq + tl] = ssq;
  }
}

// ------------------------------------------------------------------ RMSNorm
// out = w * (x * 1/sqrt(mean(x^2) + eps)), rounding like the reference's
// LlamaRMSNorm: the normalised value is cast to the output dtype before the
// weight multiply.
template <typename T>
__global__ void rmsnorm_kernel(const float* x, int64_t d, int64_t ldx, const T* w, float eps, T* out, int64_t ldo) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const float* row = x + (int64_t)t * ldx;
  float ss = 0.f;
  if ((d & 3) == 0 && (ldx & 3) == 0 && d <= 4LL * 4 * blockDim.x) {
    // up to 4 float4 per thread, all loads issued before use (latency-bound op)
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int n4 = (int)(d >> 2);
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = threadIdx.x + j * blockDim.x;
      v[j] = i < n4 ? r4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
  } else {
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x) ss = fmaf(row[i], row[i], ss);
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(red[0] / (float)d + eps);
  for (int64_t i = threadIdx.x; i < d; i += blockDim.x) {
    const T h = from_f32<T>(row[i] * inv);
    out[(int64_t)t * ldo + i] = from_f32<T>(to_f32<T>(w[i]) * to_f32<T>(h));
  }
}

// ------------------------------------------------------------ head reducers
// Merge the per-tile {max1, idx1, max2} records of each row.
// rec_out (tensor parallel): instead of the outputs, write this shard's
// record {max1, idx1 + idx_offset, max2} per row for the cross-rank merge.
__global__ void argmax_reduce_kernel(const float* part, int tiles, int32_t* out_idx, float* out_max, float* out_gap,
                                     float* rec_out, int idx_offset) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const float* rec = part + (int64_t)t * tiles * 3;
  float m1 = -INFINITY, m2 = -INFINITY;
  int i1 = INT32_MAX;
  for (int i = threadIdx.x; i < tiles; i += blockDim.x) {
    const float a = rec[i * 3], b = rec[i * 3 + 2];
    const int ai = __float_as_int(rec[i * 3 + 1]);
    if (a > m1 || (a == m1 && ai < i1)) {
      m2 = fmaxf(m1, b);
      m1 = a;
      i1 = ai;
    } else {
      m2 = fmaxf(m2, a);
    }
  }
  __shared__ float s1[32], s2[32];
  __shared__ int si[32];
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
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) {
    s1[warp] = m1;
    s2[warp] = m2;
    si[warp] = i1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < nw; ++w) {
      if (s1[w] > m1 || (s1[w] == m1 && si[w] < i1)) {
        m2 = fmaxf(m1, s2[w]);
        m1 = s1[w];
        i1 = si[w];
      } else {
        m2 = fmaxf(m2, s1[w]);
      }
    }
    if (rec_out) {
      rec_out[(int64_t)t * 3] = m1;
      rec_out[(int64_t)t * 3 + 1] = __int_as_float(i1 == INT32_MAX ? INT32_MAX : i1 + idx_offset);
      rec_out[(int64_t)t * 3 + 2] = m2;
      return;
    }
    out_idx[t] = i1;
    if (out_max) out_max[t] = m1;
    if (out_gap) out_gap[t] = m1 - m2;
  }
}

// Merge per-tile {max, sumexp, val[k], idx[k]} records: global log-sum-exp and
// the k best (value desc, index asc); emits tokens through vocab_ids.
// rec_out (tensor parallel): instead of the outputs, write this shard's
// merged record {max, sumexp, val[k], idx[k] + idx_offset} per row (the
// per-tile record format) for the cross-rank merge.
__global__ void topk_reduce_kernel(const float* part, int tiles, int k, const int64_t* vocab_ids, int32_t* out_tok,
                                   float* out_lp, float* rec_out, int idx_offset) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int rec = 2 + 2 * k;
  const float* base = part + (int64_t)t * tiles * rec;
  __shared__ float red[32];
  __shared__ float s_val[32];
  __shared__ int s_idx[32], s_tile[32];
  __shared__ int head[1024];  // per-tile cursor into its sorted list (tiles <= 1024 * blockDim)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  // global max
  float m = -INFINITY;
  for (int i = threadIdx.x; i < tiles; i += blockDim.x) m = fmaxf(m, base[(int64_t)i * rec]);
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = red[0];
    for (int w = 1; w < nw; ++w) v = fmaxf(v, red[w]);
    red[0] = v;
  }
  __syncthreads();
  const float M = red[0];
  __syncthreads();
  float s = 0.f;
  for (int i = threadIdx.x; i < tiles; i += blockDim.x) {
    const float mi = base[(int64_t)i * rec];
    if (mi != -INFINITY) s += base[(int64_t)i * rec + 1] * expf(mi - M);
  }
  s = warp_sum(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = 0.f;
    for (int w = 0; w < nw; ++w) v += red[w];
    red[0] = v;
  }
  __syncthreads();
  const float lse = M + logf(red[0]);
  if (rec_out && threadIdx.x == 0) {
    rec_out[(int64_t)t * rec] = M;
    rec_out[(int64_t)t * rec + 1] = red[0];
  }
  for (int i = threadIdx.x; i < tiles && i < 1024; i += blockDim.x) head[i] = 0;
  __syncthreads();
  // k rounds: every thread proposes the best head among its tiles
  for (int q = 0; q < k; ++q) {
    float bv = -INFINITY;
    int bi = INT32_MAX, bt = -1;
    for (int i = threadIdx.x; i < tiles; i += blockDim.x) {
      const int h = head[i];
      if (h >= k) continue;
      const float v = base[(int64_t)i * rec + 2 + h];
      const int ix = __float_as_int(base[(int64_t)i * rec + 2 + k + h]);
      if (v > bv || (v == bv && ix < bi)) {
        bv = v;
        bi = ix;
        bt = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      const int ot = __shfl_xor_sync(0xffffffffu, bt, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
        bt = ot;
      }
    }
    if (lane == 0) {
      s_val[warp] = bv;
      s_idx[warp] = bi;
      s_tile[warp] = bt;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < nw; ++w)
        if (s_val[w] > bv || (s_val[w] == bv && s_idx[w] < bi)) {
          bv = s_val[w];
          bi = s_idx[w];
          bt = s_tile[w];
        }
      if (bt >= 0) head[bt] += 1;
      if (rec_out) {
        rec_out[(int64_t)t * rec + 2 + q] = bv;
        rec_out[(int64_t)t * rec + 2 + k + q] = __int_as_float(bi == INT32_MAX ? INT32_MAX : bi + idx_offset);
      } else {
        const int tok = (bi == INT32_MAX) ? -1 : (vocab_ids ? (int)vocab_ids[bi] : bi);
        out_tok[(int64_t)t * k + q] = tok;
        out_lp[(int64_t)t * k + q] = (bi == INT32_MAX) ? -INFINITY : bv - lse;
      }
    }
    __syncthreads();
  }
}

}  // namespace ssd

using namespace ssd;

extern "C" {

int64_t ssd_workspace_bytes(int64_t max_rows, int64_t max_head_rows, int64_t vocab) {
  const int64_t tiles_v = (vocab + kTileM - 1) / kTileM;
  const int64_t heads = max_head_rows * tiles_v * (2 + 2 * kMaxTopK) * 4;
  // split-K partials: at most 2 CTAs per SM, each a 128 x BN fp32 tile
  int64_t bn = max_rows > 256 ? 128 : ((max_rows + 15) / 16) * 16;
  if (bn < 16) bn = 16;
  // tcgen05: <= 2 CTAs/SM, one 128 x BN tile each; SIMT (fp32): <= 4 CTAs/SM
  // per 4-token tile, up to kSimtInvariantRows / 4 token tiles.
  const int64_t simt_tiles_n = (kSimtInvariantRows + 3) / 4;
  // tcgen05: cluster split-K partials (<= 2 CTAs/SM, one tile each) or the
  // stream-K kernel's two partial slots per CTA (<= 2 CTAs/SM)
  const int64_t splitk_tc = 4LL * device_sms() * bn * kTileM * 4;
  const int64_t splitk_simt = 4LL * device_sms() * simt_tiles_n * 4 * kTileM * 4;
  const int64_t splitk = splitk_tc > splitk_simt ? splitk_tc : splitk_simt;
  // attention partials: (CTAs <= 2 * SMs + row-tile blocks) x 32 queries x
  // (head_dim <= 128 + 2) floats; row-tile blocks <= rows * n_heads / 32 with
  // n_heads <= 128.
  // (tensor-core kernel: <= 128 query rows x 132 floats per CTA-slice record set)
  const int64_t attn = (2LL * device_sms() + max_rows * 4 + 8) * 128 * 132 * 4;
  // a head GEMM keeps its partial records and the stream-K partials at once
  int64_t body = heads + splitk;
  body = body > attn ? body : attn;
  return kCounterBytes + body;
}

int ssd_embed(const int32_t* ids, int64_t T, const void* table, int64_t vocab, int64_t d, int dtype, float* resid,
              const SsdNormOut* norm_out, uint32_t* status, void* stream) {
  if (T <= 0 || d <= 0 || !ids || !table || !resid) return fail(SSD_ERR_INVALID, "ssd_embed: bad arguments");
  SsdNormOut no{};
  if (norm_out && norm_out->weight) {
    if (dtype != SSD_BF16 || !norm_out->out || !norm_out->ssq)
      return fail(SSD_ERR_INVALID, "ssd_embed: norm output needs bf16, out and ssq");
    no = *norm_out;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SSD_F32)
    return launch_kernel("embed_kernel", embed_kernel<float>, dim3((unsigned)T), dim3(256), 0, s, 1, 1, ids,
                         static_cast<const float*>(table), vocab, d, resid, no, status);
  else if (dtype == SSD_BF16)
    return launch_kernel("embed_kernel", embed_kernel<bf16>, dim3((unsigned)T), dim3(256), 0, s, 1, 1, ids,
                         static_cast<const bf16*>(table), vocab, d, resid, no, status);
  else
    return fail(SSD_ERR_UNSUPPORTED, "ssd_embed: dtype %d", dtype);
}

int ssd_rmsnorm(const float* x, int64_t T, int64_t d, int64_t ldx, const void* weight, float eps, void* out,
                int64_t ldo, int dtype, void* stream) {
  if (T <= 0 || d <= 0 || !x || !weight || !out) return fail(SSD_ERR_INVALID, "ssd_rmsnorm: bad arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == SSD_F32)
    return launch_kernel("rmsnorm_kernel", rmsnorm_kernel<float>, dim3((unsigned)T), dim3(256), 0, s, 1, 1, x, d, ldx,
                         static_cast<const float*>(weight), eps, static_cast<float*>(out), ldo);
  else if (dtype == SSD_BF16)
    return launch_kernel("rmsnorm_kernel", rmsnorm_kernel<bf16>, dim3((unsigned)T), dim3(256), 0, s, 1, 1, x, d, ldx,
                         static_cast<const bf16*>(weight), eps, static_cast<bf16*>(out), ldo);
  else
    return fail(SSD_ERR_UNSUPPORTED, "ssd_rmsnorm: dtype %d", dtype);
}

// Copies the C ABI's RMSNorm-folding arguments into the epilogue arguments.
static int set_norms(EpiArgs& e, const SsdRowNorm* in_norm, const SsdNormOut* norm_out, int dtype, const char* who) {
  if (in_norm && in_norm->ssq) {
    if (dtype != SSD_BF16 || in_norm->parts <= 0 || in_norm->d <= 0)
      return fail(SSD_ERR_INVALID, "%s: row norm needs bf16, parts > 0 and d > 0", who);
    e.rn_ssq = in_norm->ssq;
    e.rn_ld = in_norm->ld;
    e.rn_parts = (int)in_norm->parts;
    e.rn_d = (int)in_norm->d;
    e.rn_eps = in_norm->eps;
  }
  if (norm_out && norm_out->weight) {
    if (dtype != SSD_BF16 || e.kind != EPI_RESIDUAL || !norm_out->out || !norm_out->ssq)
      return fail(SSD_ERR_INVALID, "%s: norm output needs bf16, the residual epilogue, out and ssq", who);
    e.no_w = norm_out->weight;
    e.no_out = norm_out->out;
    e.no_ldo = norm_out->ldo;
    e.no_ssq = norm_out->ssq;
    e.no_ld = norm_out->ld_ssq;
  }
  return SSD_OK;
}

int ssd_linear(const void* x, int64_t ldx, int64_t T, int64_t K, int n_seg, const void* const* w,
               const int64_t* rows, const void* const* bias, int seg_layout, int epilogue, int act, void* out,
               int64_t ldo, float* resid, int64_t ldr, int dtype, void* workspace, int64_t workspace_bytes,
               const SsdRowNorm* in_norm, const SsdNormOut* norm_out, uint32_t* status, void* stream) {
  EpiArgs e{};
  e.kind = epilogue;
  e.act = act;
  for (int i = 0; i < 3; ++i) e.bias[i] = (bias && i < n_seg) ? bias[i] : nullptr;
  e.out = out;
  e.ldo = ldo;
  e.resid = resid;
  e.ldr = ldr;
  switch (epilogue) {
    case SSD_EPI_STORE:
    case SSD_EPI_STORE_F32:
      if (!out) return fail(SSD_ERR_INVALID, "ssd_linear: out is NULL");
      break;
    case SSD_EPI_RESIDUAL:
      if (!resid) return fail(SSD_ERR_INVALID, "ssd_linear: resid is NULL");
      break;
    case SSD_EPI_SWIGLU:
      if (!out || seg_layout != SSD_SEG_PAIRS) return fail(SSD_ERR_INVALID, "ssd_linear: SwiGLU needs PAIRS + out");
      break;
    default:
      return fail(SSD_ERR_INVALID, "ssd_linear: unknown epilogue %d", epilogue);
  }
  if (seg_layout == SSD_SEG_PAIRS && epilogue != SSD_EPI_SWIGLU)
    return fail(SSD_ERR_INVALID, "ssd_linear: PAIRS layout is only for SwiGLU");
  if (const int rc = set_norms(e, in_norm, norm_out, dtype, "ssd_linear")) return rc;
  return launch_gemm(x, ldx, T, K, n_seg, w, rows, seg_layout, e, dtype, workspace, workspace_bytes, status,
                     static_cast<cudaStream_t>(stream), 0);
}

int ssd_qkv_rope(const void* x, int64_t ldx, int64_t T, int64_t K, const void* wq, const void* wk, const void* wv,
                 int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, const float* rope_cos, const float* rope_sin,
                 int64_t max_pos, const int32_t* positions, const int32_t* slots, void* k_cache, void* v_cache,
                 int64_t cache_head_stride, int64_t max_slots, void* q_out, int64_t ldq, int dtype, void* workspace,
                 int64_t workspace_bytes, const SsdRowNorm* in_norm, uint32_t* status, void* stream) {
  if (head_dim <= 0 || head_dim > 128 || (128 % head_dim) || (head_dim & 1))
    return fail(SSD_ERR_UNSUPPORTED, "ssd_qkv_rope: head_dim must divide 128");
  if (!positions || !slots || !k_cache || !v_cache || !q_out || !rope_cos || !rope_sin)
    return fail(SSD_ERR_INVALID, "ssd_qkv_rope: NULL argument");
  EpiArgs e{};
  e.kind = EPI_QKV;
  e.out = q_out;
  e.ldo = ldq;
  e.head_dim = (int)head_dim;
  e.n_q = (int)(n_heads * head_dim);
  e.n_kv = (int)(n_kv_heads * head_dim);
  e.rope_cos = rope_cos;
  e.rope_sin = rope_sin;
  e.max_pos = (int)max_pos;
  e.positions = positions;
  e.slots = slots;
  e.k_cache = k_cache;
  e.v_cache = v_cache;
  e.head_stride = cache_head_stride;
  e.max_slots = (int)max_slots;
  if (const int rc = set_norms(e, in_norm, nullptr, dtype, "ssd_qkv_rope")) return rc;
  const void* w[3] = {wq, wk, wv};
  int64_t rows[3] = {n_heads * head_dim, n_kv_heads * head_dim, n_kv_heads * head_dim};
  return launch_gemm(x, ldx, T, K, 3, w, rows, SSD_SEG_CONCAT, e, dtype, workspace, workspace_bytes, status,
                     static_cast<cudaStream_t>(stream), 0);
}

int ssd_linear_chain(int32_t n, const SsdLinearArgs* links, int64_t T, int dtype, void* workspace,
                     int64_t workspace_bytes, uint32_t* status, void* stream) {
  if (dtype != SSD_BF16) return fail(SSD_ERR_UNSUPPORTED, "ssd_linear_chain: bf16 only");
  if (!links || n < 1 || n > 6) return fail(SSD_ERR_INVALID, "ssd_linear_chain: 1..6 links");
  ChainLinkHost h[6];
  for (int l = 0; l < n; ++l) {
    const SsdLinearArgs& a = links[l];
    ChainLinkHost& c = h[l];
    memset(&c, 0, sizeof(c));
    c.x = a.x;
    c.ldx = a.ldx;
    c.K = a.K;
    EpiArgs& e = c.e;
    e.kind = a.epilogue;
    e.act = a.act;
    e.out = a.out;
    e.ldo = a.ldo;
    const SsdRowNorm* rn = a.in_norm.ssq ? &a.in_norm : nullptr;
    const SsdNormOut* no = a.norm_out.weight ? &a.norm_out : nullptr;
    if (a.epilogue == SSD_EPI_QKV) {
      const int64_t hd = a.head_dim;
      if (hd <= 0 || hd > 128 || (128 % hd) || (hd & 1))
        return fail(SSD_ERR_UNSUPPORTED, "ssd_linear_chain: link %d: head_dim must divide 128", l);
      if (!a.positions || !a.slots || !a.k_cache || !a.v_cache || !a.out || !a.rope_cos || !a.rope_sin ||
          !a.w[0] || !a.w[1] || !a.w[2])
        return fail(SSD_ERR_INVALID, "ssd_linear_chain: link %d: NULL q/k/v argument", l);
      e.head_dim = (int)hd;
      e.n_q = (int)(a.n_heads * hd);
      e.n_kv = (int)(a.n_kv_heads * hd);
      e.rope_cos = a.rope_cos;
      e.rope_sin = a.rope_sin;
      e.max_pos = (int)a.max_pos;
      e.positions = a.positions;
      e.slots = a.slots;
      e.k_cache = a.k_cache;
      e.v_cache = a.v_cache;
      e.head_stride = a.cache_head_stride;
      e.max_slots = (int)a.max_slots;
      c.n_seg = 3;
      c.layout = SSD_SEG_CONCAT;
      for (int i = 0; i < 3; ++i) c.w[i] = a.w[i];
      c.rows[0] = a.n_heads * hd;
      c.rows[1] = c.rows[2] = a.n_kv_heads * hd;
      if (const int rc = set_norms(e, rn, nullptr, dtype, "ssd_linear_chain")) return rc;
      continue;
    }
    switch (a.epilogue) {
      case SSD_EPI_STORE:
      case SSD_EPI_STORE_F32:
        if (!a.out) return fail(SSD_ERR_INVALID, "ssd_linear_chain: link %d: out is NULL", l);
        break;
      case SSD_EPI_RESIDUAL:
        if (!a.resid) return fail(SSD_ERR_INVALID, "ssd_linear_chain: link %d: resid is NULL", l);
        break;
      case SSD_EPI_SWIGLU:
        if (!a.out || a.seg_layout != SSD_SEG_PAIRS)
          return fail(SSD_ERR_INVALID, "ssd_linear_chain: link %d: SwiGLU needs PAIRS + out", l);
        break;
      default:
        return fail(SSD_ERR_INVALID, "ssd_linear_chain: link %d: unknown epilogue %d", l, a.epilogue);
    }
    if (a.seg_layout == SSD_SEG_PAIRS && a.epilogue != SSD_EPI_SWIGLU)
      return fail(SSD_ERR_INVALID, "ssd_linear_chain: link %d: PAIRS layout is only for SwiGLU", l);
    if (a.n_seg < 1 || a.n_seg > 3) return fail(SSD_ERR_INVALID, "ssd_linear_chain: link %d: n_seg", l);
    c.n_seg = a.n_seg;
    c.layout = a.seg_layout;
    for (int i = 0; i < 3; ++i) {
      c.w[i] = i < a.n_seg ? a.w[i] : nullptr;
      c.rows[i] = i < a.n_seg ? a.rows[i] : 0;
      e.bias[i] = i < a.n_seg ? a.bias[i] : nullptr;
    }
    e.resid = a.resid;
    e.ldr = a.ldr;
    if (const int rc = set_norms(e, rn, no, dtype, "ssd_linear_chain")) return rc;
  }
  return launch_chain(n, h, T, workspace, workspace_bytes, status, static_cast<cudaStream_t>(stream));
}

int ssd_head_argmax(const void* x, int64_t ldx, int64_t T, int64_t K, const void* w, int64_t vocab,
                    int32_t* out_idx, float* out_max, float* out_gap, int dtype, void* workspace,
                    int64_t workspace_bytes, const SsdRowNorm* in_norm, uint32_t* status, void* stream) {
  const int64_t tiles = (vocab + kTileM - 1) / kTileM;
  const int64_t need = kCounterBytes + T * tiles * 3 * 4;
  if (!workspace || need > workspace_bytes) return fail(SSD_ERR_WORKSPACE, "ssd_head_argmax: workspace too small");
  if (!out_idx) return fail(SSD_ERR_INVALID, "ssd_head_argmax: out_idx is NULL");
  EpiArgs e{};
  e.kind = EPI_ARGMAX;
  e.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
  if (const int rc = set_norms(e, in_norm, nullptr, dtype, "ssd_head_argmax")) return rc;
  const void* ws[1] = {w};
  int64_t rows[1] = {vocab};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = launch_gemm(x, ldx, T, K, 1, ws, rows, SSD_SEG_CONCAT, e, dtype, workspace, workspace_bytes, status, s,
                       T * tiles * 3 * 4);
  if (rc) return rc;
  return launch_kernel("argmax_reduce_kernel", argmax_reduce_kernel, dim3((unsigned)T), dim3(256), 0, s, 1, 1, e.part,
                       (int)tiles, out_idx, out_max, out_gap, (float*)nullptr, 0);
}

int ssd_head_topk(const void* x, int64_t ldx, int64_t T, int64_t K, const void* w, int64_t vocab,
                  const int64_t* vocab_ids, int64_t k, int32_t* out_tok, float* out_logprob, int dtype,
                  void* workspace, int64_t workspace_bytes, const SsdRowNorm* in_norm, uint32_t* status,
                  void* stream) {
  if (k < 1 || k > kMaxTopK || k > vocab) return fail(SSD_ERR_UNSUPPORTED, "ssd_head_topk: k must be 1..16");
  const int64_t tiles = (vocab + kTileM - 1) / kTileM;
  const int64_t rec = 2 + 2 * k;
  const int64_t need = kCounterBytes + T * tiles * rec * 4;
  if (!workspace || need > workspace_bytes) return fail(SSD_ERR_WORKSPACE, "ssd_head_topk: workspace too small");
  if (!out_tok || !out_logprob) return fail(SSD_ERR_INVALID, "ssd_head_topk: NULL output");
  if (tiles > 1024) return fail(SSD_ERR_UNSUPPORTED, "ssd_head_topk: more than 1024 vocab tiles");
  EpiArgs e{};
  e.kind = EPI_TOPK;
  e.topk = (int)k;
  e.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
  if (const int rc = set_norms(e, in_norm, nullptr, dtype, "ssd_head_topk")) return rc;
  const void* ws[1] = {w};
  int64_t rows[1] = {vocab};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = launch_gemm(x, ldx, T, K, 1, ws, rows, SSD_SEG_CONCAT, e, dtype, workspace, workspace_bytes, status, s,
                       T * tiles * rec * 4);
  if (rc) return rc;
  return launch_kernel("topk_reduce_kernel", topk_reduce_kernel, dim3((unsigned)T), dim3(256), 0, s, 1, 1, e.part,
                       (int)tiles, (int)k, vocab_ids, out_tok, out_logprob, (float*)nullptr, 0);
}

}  // extern "C"
