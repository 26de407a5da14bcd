// Tree attention over the shared KV cache (split-KV "FlashDecoding" layout).
//
// Row t of the forward attends cache slots [0, prefix_len[t]) and every
// speculative slot spec_base + j whose bit j is set in its ancestor mask. A
// CTA owns one KV head, a group of token rows (times the GQA group of query
// heads that share the KV head) and one contiguous slice of the key range,
// so each K/V byte of the slice is read once for all those queries. Slices
// produce (max, sum, acc) partials; the last CTA of a (head, row-group) to
// finish merges them in slice order (deterministic).
#include "common.cuh"
#include "host.cuh"

namespace ssd {

constexpr int kAttnWarps = 8;
constexpr int kAttnQPerWarp = 4;
constexpr int kAttnQ = kAttnWarps * kAttnQPerWarp;  // queries per CTA
constexpr int kAttnBlock = 64;                        // keys per inner block
constexpr int kAttnCounterBase = 49152;               // counter slots used by attention

struct AttnArgs {
  const void* q;
  int64_t ldq;
  int T, n_heads, n_kv, hd, G;
  const void* kc;
  const void* vc;
  int64_t head_stride;
  int max_slots;
  const int32_t* prefix_len;
  const int32_t* spec_base;
  const uint64_t* mask;
  int mask_words;
  int kv_bound, split_len, n_splits, rows_per_tile, row_tiles;
  void* out;
  int64_t ldo;
  float* part;
  uint32_t* counters;
  uint32_t* status;
  float scale;
};

template <typename T>
__global__ void __launch_bounds__(256) attn_simt_kernel(const AttnArgs a) {
  extern __shared__ float sm[];
  const int hd = a.hd, hp = hd + 1;
  float* Ks = sm;                            // [64][hd+1]
  float* Vs = Ks + kAttnBlock * hp;          // [64][hd+1]
  float* Qs = Vs + kAttnBlock * hp;          // [32][hd]
  float* Ps = Qs + kAttnQ * hd;              // [8][4][64]
  int* s_plen = reinterpret_cast<int*>(Ps + kAttnWarps * kAttnQPerWarp * kAttnBlock);  // [rows_per_tile]
  int* s_misc = s_plen + kAttnQ;             // [0] need_end, [1] is_last

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x / a.row_tiles, rt = blockIdx.x % a.row_tiles;
  const int split = blockIdx.y;
  const int row0 = rt * a.rows_per_tile;
  const int nrows = min(a.rows_per_tile, a.T - row0);
  const int nq = nrows * a.G;
  const int sb = a.spec_base ? a.spec_base[0] : 0;

  if (threadIdx.x == 0) s_misc[0] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < nrows; i += blockDim.x) {
    const int t = row0 + i;
    const int pl = a.prefix_len[t];
    s_plen[i] = pl;
    int end = pl;
    if (a.mask) {
      for (int w = a.mask_words - 1; w >= 0; --w) {
        const uint64_t m = a.mask[(int64_t)t * a.mask_words + w];
        if (m) {
          end = max(end, sb + w * 64 + 64 - __clzll(m));
          break;
        }
      }
    }
    atomicMax(&s_misc[0], end);
  }
  // queries of this CTA: qi -> (row qi / G, head h*G + qi % G)
  for (int idx = threadIdx.x; idx < kAttnQ * hd; idx += blockDim.x) {
    const int qi = idx / hd, d = idx % hd;
    float v = 0.f;
    if (qi < nq) {
      const int t = row0 + qi / a.G, qh = h * a.G + qi % a.G;
      v = to_f32<T>(static_cast<const T*>(a.q)[(int64_t)t * a.ldq + (int64_t)qh * hd + d]) * a.scale;
    }
    Qs[idx] = v;
  }
  __syncthreads();
  const int need_end = min(min(s_misc[0], a.kv_bound), a.max_slots);
  const int k_lo = split * a.split_len;
  const int k_hi = min(k_lo + a.split_len, need_end);

  float m[kAttnQPerWarp], l[kAttnQPerWarp], acc[kAttnQPerWarp][4];
#pragma unroll
  for (int i = 0; i < kAttnQPerWarp; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  }
  const T* kbase = static_cast<const T*>(a.kc) + (int64_t)h * a.head_stride;
  const T* vbase = static_cast<const T*>(a.vc) + (int64_t)h * a.head_stride;

  for (int kb = k_lo; kb < k_hi; kb += kAttnBlock) {
    const int nkeys = min(kAttnBlock, k_hi - kb);
    __syncthreads();
    for (int idx = threadIdx.x; idx < kAttnBlock * hd; idx += blockDim.x) {
      const int j = idx / hd, d = idx % hd;
      float kv = 0.f, vv = 0.f;
      if (j < nkeys) {
        kv = to_f32<T>(kbase[(int64_t)(kb + j) * hd + d]);
        vv = to_f32<T>(vbase[(int64_t)(kb + j) * hd + d]);
      }
      Ks[j * hp + d] = kv;
      Vs[j * hp + d] = vv;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kAttnQPerWarp; ++i) {
      const int qi = warp * kAttnQPerWarp + i;
      if (qi >= nq) break;  // warp-uniform
      const int rl = qi / a.G;
      const int t = row0 + rl;
      const float* qv = Qs + qi * hd;
      float s[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int j = lane + 32 * u;
        const int slot = kb + j;
        bool ok = j < nkeys && slot < s_plen[rl];
        if (!ok && a.mask && j < nkeys && slot >= sb) {
          const int bit = slot - sb;
          if (bit < a.mask_words * 64) ok = (a.mask[(int64_t)t * a.mask_words + (bit >> 6)] >> (bit & 63)) & 1ull;
        }
        float dot = 0.f;
        if (ok) {
          const float* kr = Ks + j * hp;
          for (int d = 0; d < hd; ++d) dot = fmaf(qv[d], kr[d], dot);
        }
        s[u] = ok ? dot : -INFINITY;
      }
      const float mb = warp_max(fmaxf(s[0], s[1]));
      if (mb == -INFINITY) continue;  // nothing visible in this block (warp-uniform)
      const float mn = fmaxf(m[i], mb);
      const float alpha = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mn);
      const float p0 = (s[0] == -INFINITY) ? 0.f : expf(s[0] - mn);
      const float p1 = (s[1] == -INFINITY) ? 0.f : expf(s[1] - mn);
      l[i] = l[i] * alpha + warp_sum(p0 + p1);
      m[i] = mn;
      float* pb = Ps + (warp * kAttnQPerWarp + i) * kAttnBlock;
      pb[lane] = p0;
      pb[lane + 32] = p1;
      __syncwarp();
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[i][u] *= alpha;
      for (int j = 0; j < nkeys; ++j) {
        const float pj = pb[j];
        const float* vr = Vs + j * hp;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int d = lane + 32 * u;
          if (d < hd) acc[i][u] = fmaf(pj, vr[d], acc[i][u]);
        }
      }
      __syncwarp();
    }
  }

  // write this slice's partials
  const int blk = h * a.row_tiles + rt;
  const int rec = hd + 2;
#pragma unroll
  for (int i = 0; i < kAttnQPerWarp; ++i) {
    const int qi = warp * kAttnQPerWarp + i;
    if (qi >= nq) break;
    float* p = a.part + (((int64_t)blk * a.n_splits + split) * kAttnQ + qi) * rec;
    if (lane == 0) {
      p[0] = m[i];
      p[1] = l[i];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int d = lane + 32 * u;
      if (d < hd) p[2 + d] = acc[i][u];
    }
  }
  __threadfence();
  __syncthreads();
  if (a.n_splits > 1) {
    if (threadIdx.x == 0) {
      const uint32_t prev = atomicAdd(&a.counters[kAttnCounterBase + blk], 1u);
      s_misc[1] = (prev == (uint32_t)(a.n_splits - 1)) ? 1 : 0;
    }
    __syncthreads();
    if (!s_misc[1]) return;
    __threadfence();
  }
  // merge the slices in order and write the output rows
#pragma unroll
  for (int i = 0; i < kAttnQPerWarp; ++i) {
    const int qi = warp * kAttnQPerWarp + i;
    if (qi >= nq) break;
    const int t = row0 + qi / a.G, qh = h * a.G + qi % a.G;
    float M = -INFINITY;
    for (int s = 0; s < a.n_splits; ++s)
      M = fmaxf(M, __ldcg(a.part + (((int64_t)blk * a.n_splits + s) * kAttnQ + qi) * rec));
    float L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
    if (M != -INFINITY) {
      for (int s = 0; s < a.n_splits; ++s) {
        const float* p = a.part + (((int64_t)blk * a.n_splits + s) * kAttnQ + qi) * rec;
        const float ms = __ldcg(p);
        if (ms == -INFINITY) continue;
        const float w = expf(ms - M);
        L = fmaf(__ldcg(p + 1), w, L);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int d = lane + 32 * u;
          if (d < hd) o[u] = fmaf(__ldcg(p + 2 + d), w, o[u]);
        }
      }
    }
    const float inv = (L > 0.f) ? 1.0f / L : 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int d = lane + 32 * u;
      if (d < hd) static_cast<T*>(a.out)[(int64_t)t * a.ldo + (int64_t)qh * hd + d] = from_f32<T>(o[u] * inv);
    }
  }
  if (a.n_splits > 1 && threadIdx.x == 0) a.counters[kAttnCounterBase + blk] = 0u;
}

}  // namespace ssd

using namespace ssd;

extern "C" int ssd_tree_attention(const void* q, int64_t ldq, int64_t T, int64_t n_heads, int64_t n_kv_heads,
                                  int64_t head_dim, const void* k_cache, const void* v_cache,
                                  int64_t cache_head_stride, int64_t max_slots, const int32_t* prefix_len,
                                  const int32_t* spec_base, const uint64_t* spec_mask, int64_t mask_words,
                                  int64_t kv_bound, void* out, int64_t ldo, int dtype, void* workspace,
                                  int64_t workspace_bytes, uint32_t* status, void* stream) {
  if (T <= 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || head_dim <= 0 || head_dim > 128)
    return fail(SSD_ERR_INVALID, "ssd_tree_attention: bad head configuration");
  if (!q || !k_cache || !v_cache || !prefix_len || !out) return fail(SSD_ERR_INVALID, "ssd_tree_attention: NULL");
  if (spec_mask && (!spec_base || mask_words <= 0 || mask_words > 4))
    return fail(SSD_ERR_INVALID, "ssd_tree_attention: mask needs spec_base and 1..4 words");
  if (kv_bound <= 0 || kv_bound > max_slots) kv_bound = max_slots;
  AttnArgs a{};
  a.q = q;
  a.ldq = ldq;
  a.T = (int)T;
  a.n_heads = (int)n_heads;
  a.n_kv = (int)n_kv_heads;
  a.hd = (int)head_dim;
  a.G = (int)(n_heads / n_kv_heads);
  a.kc = k_cache;
  a.vc = v_cache;
  a.head_stride = cache_head_stride;
  a.max_slots = (int)max_slots;
  a.prefix_len = prefix_len;
  a.spec_base = spec_mask ? spec_base : nullptr;
  a.mask = spec_mask;
  a.mask_words = (int)mask_words;
  a.kv_bound = (int)kv_bound;
  a.out = out;
  a.ldo = ldo;
  a.status = status;
  a.scale = 1.0f / sqrtf((float)head_dim);
  if (a.G > kAttnQ) return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: GQA group > 32");
  a.rows_per_tile = kAttnQ / a.G;
  a.row_tiles = (int)((T + a.rows_per_tile - 1) / a.rows_per_tile);
  // Key slices: enough CTAs to cover the SMs twice, 64-key aligned.
  const int sms = device_sms();
  const int64_t base_ctas = (int64_t)a.n_kv * a.row_tiles;
  int64_t want = (2 * sms + base_ctas - 1) / base_ctas;
  int64_t split_len = (kv_bound + want - 1) / want;
  split_len = ((split_len + kAttnBlock - 1) / kAttnBlock) * kAttnBlock;
  if (split_len < 256) split_len = 256;
  a.split_len = (int)split_len;
  a.n_splits = (int)((kv_bound + split_len - 1) / split_len);
  const int64_t blocks = base_ctas;
  if (blocks > 16384) return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: too many row tiles");
  const int64_t need = kCounterBytes + blocks * a.n_splits * kAttnQ * (head_dim + 2) * 4;
  if (!workspace || need > workspace_bytes)
    return fail(SSD_ERR_WORKSPACE, "ssd_tree_attention: workspace too small (need %lld)", (long long)need);
  a.counters = static_cast<uint32_t*>(workspace);
  a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
  const size_t smem = (size_t)(2 * kAttnBlock * (head_dim + 1) + kAttnQ * head_dim +
                               kAttnWarps * kAttnQPerWarp * kAttnBlock) * 4 + (kAttnQ + 2) * 4;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid((unsigned)blocks, (unsigned)a.n_splits);
  if (dtype == SSD_F32) {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(attn_simt_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
      set = true;
    }
    attn_simt_kernel<float><<<grid, 256, smem, s>>>(a);
  } else if (dtype == SSD_BF16) {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(attn_simt_kernel<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
      set = true;
    }
    attn_simt_kernel<bf16><<<grid, 256, smem, s>>>(a);
  } else {
    return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: dtype %d", dtype);
  }
  return check_launch("attn_simt_kernel");
}
