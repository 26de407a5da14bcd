// Tree attention over the shared KV cache (split-KV "FlashDecoding" layout).
//
// Row t of the forward attends cache slots [prefix_start[t] (0 without the
// array), prefix_len[t]) and every
// speculative slot spec_base + j whose bit j is set in its ancestor mask. A
// CTA owns one KV head, a group of token rows (times the GQA group of query
// heads that share the KV head) and one contiguous slice of the key range,
// so each K/V byte of the slice is read once for all those queries. Slices
// produce (max, sum, acc) partials; the last CTA of a (head, row-group) to
// finish merges them in slice order (deterministic).
#include <map>
#include <mutex>
#include <tuple>

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
  const int32_t* prefix_start;  // optional first visible slot per row (NULL = 0)
  const int32_t* spec_base;
  const uint64_t* mask;
  int mask_words;
  int kv_bound, split_len, n_splits, rows_per_tile, row_tiles;
  int groups, rows_per_group;  // tensor-core kernel: query rows (token x GQA head) per CTA
  int rt, kw;                  // tensor-core kernel: 16-row tiles and key lanes per CTA
  int cluster_merge;           // key slices of a row group form a cluster and merge through DSMEM
  int two_min;                 // tensor-core kernel: key blocks from which two softmax warpgroups split them
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
  int* s_pstart = s_misc + 2;                // [rows_per_tile]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x / a.row_tiles, rt = blockIdx.x % a.row_tiles;
  const int split = blockIdx.y;
  const int row0 = rt * a.rows_per_tile;
  const int nrows = min(a.rows_per_tile, a.T - row0);
  const int nq = nrows * a.G;
  pdl_wait();
  pdl_trigger();
  const int sb = a.spec_base ? a.spec_base[0] : 0;

  if (threadIdx.x == 0) s_misc[0] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < nrows; i += blockDim.x) {
    const int t = row0 + i;
    const int pl = a.prefix_len[t];
    s_plen[i] = pl;
    s_pstart[i] = a.prefix_start ? a.prefix_start[t] : 0;
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
        bool ok = j < nkeys && slot < s_plen[rl] && slot >= s_pstart[rl];
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

// Validity of keys kb .. kb + 63 for one query row as a 64-bit word: the
// contiguous prefix [0, plen), plus the speculative slots whose bit is set in
// the row's ancestor mask (bit i = slot sb + i, mw words), clipped to the
// slice end k_hi. Built with a few integer ops instead of a per-key branch.
__device__ __forceinline__ uint64_t key_block_bits(int kb, int k_hi, int plen, const uint64_t* row_mask, int mw,
                                                   int sb, int pstart) {
  const int n_hi = min(max(k_hi - kb, 0), 64);
  const uint64_t hi = n_hi >= 64 ? ~0ull : ((1ull << n_hi) - 1ull);
  const int n_pre = min(max(plen - kb, 0), 64);
  const int n_lo = min(max(pstart - kb, 0), 64);  // keys before the row's first visible slot
  const uint64_t pre = (n_pre >= 64 ? ~0ull : ((1ull << n_pre) - 1ull)) &
                       ~(n_lo >= 64 ? ~0ull : ((1ull << n_lo) - 1ull));
  uint64_t spec = 0ull;
  const int off = kb - sb;  // mask bit of slot kb
  if (mw > 0 && off < mw * 64 && off > -64) {
    const int w0 = (off >= 0) ? (off >> 6) : -1;
    const int sh = off - w0 * 64;  // 0..63
    const uint64_t lo = (w0 >= 0 && w0 < mw) ? row_mask[w0] : 0ull;
    const uint64_t up = (w0 + 1 >= 0 && w0 + 1 < mw) ? row_mask[w0 + 1] : 0ull;
    spec = sh == 0 ? lo : ((lo >> sh) | (up << (64 - sh)));
  }
  return (pre | spec) & hi;
}

// ------------------------------------------------------ tensor-core kernel
// bf16, head_dim 64 or 128, warp-specialised. A CTA = one KV head x one group
// of query rows (row q = token * G + GQA head) x one key slice. The last warp
// produces: it streams the slice's 64-key K/V blocks into a kWsStages-deep
// shared-memory ring with cp.async (16-byte chunks XOR-swizzled by key so
// ldmatrix is conflict-free), completing each stage on an mbarrier. Consumer
// warp (ri, kw) owns 16 query rows (row tile ri, Q fragments kept in
// registers) and takes blocks kw, kw + KW, ... of the slice: S = Q K^T and
// O += P V on mma.sync m16n8k16 with fp32 accumulators, online softmax in
// base 2 on the accumulator registers, and releases the stage on its own, so
// no CTA-wide barrier sits in the key loop. With few query rows (decode,
// small tree levels) KW > 1 key lanes split the slice inside the CTA. The
// (slice, key lane) partials of a row merge in a fixed order: inside one
// cluster through DSMEM, or through a global workspace for long contexts.
constexpr int kWsMaxConsumers = 7;                   // consumer warps per CTA (+ producer: 256 threads)
constexpr int kWsStages = 4;                         // K/V blocks in flight per CTA
constexpr int kMmaMaxRows = kWsMaxConsumers * 16;    // query rows per CTA
constexpr int kMmaMaxTok = kMmaMaxRows + 1;
constexpr int kMmaMaxSplits = 32;
constexpr int kMaxAttnClusterSplits = 8;
constexpr int kMaxPartials = 32;                     // key slices x key lanes merged per row

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
// Arrive on an mbarrier once this thread's earlier cp.async copies have landed.
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Partial record of one query row of one (key slice, key lane): {m, l, pad, pad, o[hd]}.
__host__ __device__ constexpr int mma_rec(int hd) { return hd + 4; }
__host__ __device__ constexpr int ws_ring_bytes(int hd) { return kWsStages * 2 * 64 * hd * 2; }
// Partial records pushed to the CTA that merges them: [p][owned row][rec]
// with p = slice * kw + key lane and owned rows r = rank, rank + slices, ...
// (at most ceil(rows / slices) per CTA); sized for up to 8 slices.
__host__ __device__ inline int ws_recv_bytes(int hd, int kw, int rows) {
  return (rows + kMaxAttnClusterSplits) * kw * mma_rec(hd) * 4;
}
__host__ __device__ inline int ws_region_bytes(int hd, int kw, int rows) {
  return ws_ring_bytes(hd) + ws_recv_bytes(hd, kw, rows);
}
constexpr int kWsMeta = (kMmaMaxTok + 1) * 4 + kMmaMaxTok * 4 * 8 + 16 + 2 * kWsStages * 8 + 16 + (kMmaMaxTok + 1) * 4;

template <int HD>
__global__ void __launch_bounds__(32 * (kWsMaxConsumers + 1), 1) attn_ws_kernel(const AttnArgs a) {
  constexpr int CH = HD / 8;   // 16-byte chunks per K/V row
  constexpr int KS = HD / 16;  // k-steps over head_dim (QK^T)
  constexpr int NTD = HD / 8;  // n-tiles over head_dim (PV)
  constexpr int KB = 64;       // keys per block
  extern __shared__ __align__(1024) uint8_t attn_smem[];
  const int region = ws_region_bytes(HD, a.kw, a.rows_per_group);
  int* s_plen = reinterpret_cast<int*>(attn_smem + region);
  uint64_t* s_mask = reinterpret_cast<uint64_t*>(s_plen + kMmaMaxTok + 1);  // [tok][4]
  int* s_misc = reinterpret_cast<int*>(s_mask + kMmaMaxTok * 4);           // need_end, min_plen, last, pad
  uint64_t* full = reinterpret_cast<uint64_t*>(s_misc + 4);
  uint64_t* empty = full + kWsStages;
  int* s_pstart = reinterpret_cast<int*>(empty + kWsStages) + 4;  // [tok]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwc = a.rt * a.kw;  // consumer warps; warp nwc produces
  const int nwarps = nwc + 1;
  const int blk = blockIdx.x;
  const int h = blk / a.groups, gr = blk % a.groups;
  const int split = blockIdx.y;
  const int M = a.T * a.G;
  const int q0 = gr * a.rows_per_group;
  const int Mg = min(a.rows_per_group, M - q0);
  const int t_first = q0 / a.G;
  const int ntok = (q0 + Mg - 1) / a.G - t_first + 1;
  const int P = a.n_splits * a.kw;  // partials per row
  pdl_wait();
  pdl_trigger();
  const int sb = a.spec_base ? a.spec_base[0] : 0;
  const int mw = a.mask ? a.mask_words : 0;

  if (threadIdx.x == 0) {
    s_misc[0] = 0;
    s_misc[1] = INT32_MAX;
    for (int st = 0; st < kWsStages; ++st) {
      mbar_init(&full[st], 32);      // one cp.async arrival per producer lane
      mbar_init(&empty[st], a.rt);   // one arrival per consumer warp of the block's key lane
    }
    fence_mbar_init();
  }
  __syncthreads();
  for (int i = threadIdx.x; i < ntok; i += blockDim.x) {
    const int t = t_first + i;
    const int pl = a.prefix_len[t];
    s_plen[i] = pl;
    s_pstart[i] = a.prefix_start ? a.prefix_start[t] : 0;
    int end = pl;
    for (int w = 0; w < mw; ++w) {
      const uint64_t m = a.mask[(int64_t)t * mw + w];
      s_mask[i * 4 + w] = m;
      if (m) end = max(end, sb + w * 64 + 64 - __clzll(m));
    }
    atomicMax(&s_misc[0], end);
    atomicMin(&s_misc[1], pl);
  }
  __syncthreads();
  const int need_end = min(min(s_misc[0], a.kv_bound), a.max_slots);
  // Slices cut the live key range (known only on the device), not the
  // static bound the grid was sized for, so every slice gets the same work.
  const int slice = ((need_end + a.n_splits - 1) / a.n_splits + KB - 1) / KB * KB;
  const int k_lo = split * slice;
  const int k_hi = min(k_lo + slice, need_end);
  const int nblocks = k_hi > k_lo ? (k_hi - k_lo + KB - 1) / KB : 0;
  const uint32_t ring_s = smem_u32(attn_smem);
  auto stage_k = [&](int st) { return ring_s + st * 2 * KB * HD * 2; };
  auto stage_v = [&](int st) { return ring_s + st * 2 * KB * HD * 2 + KB * HD * 2; };

  const int g = lane >> 2, tq = lane & 3;
  const int ri = warp % a.rt, kw = warp / a.rt;
  const int rl0 = ri * 16 + g, rl1 = rl0 + 8;  // rows within the group
  const bool ok0 = warp < nwc && rl0 < Mg, ok1 = warp < nwc && rl1 < Mg;
  const int qr0 = q0 + rl0, qr1 = q0 + rl1;
  float o[NTD][4];
#pragma unroll
  for (int i = 0; i < NTD; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  bool failed = false;

  if (warp == nwc) {
    // ---- producer: block b -> stage b % kWsStages, in block order
    const bf16* kbase = static_cast<const bf16*>(a.kc) + (int64_t)h * a.head_stride;
    const bf16* vbase = static_cast<const bf16*>(a.vc) + (int64_t)h * a.head_stride;
    for (int b = 0; b < nblocks; ++b) {
      const int st = b % kWsStages;
      if (b >= kWsStages && !mbar_wait(&empty[st], ((b / kWsStages) - 1) & 1)) {
        if (lane == 0) report_error(a.status, kErrWaitTimeout);
        failed = true;
        break;
      }
      const int kb = k_lo + b * KB;
      for (int idx = lane; idx < KB * CH; idx += 32) {
        const int key = idx / CH, c = idx % CH;
        const int slot = kb + key;
        const bool valid = slot < k_hi;
        const int64_t off = (int64_t)(valid ? slot : 0) * HD + c * 8;
        const uint32_t dst = key * HD * 2 + ((c ^ (key & 7)) << 4);
        cp_async16(stage_k(st) + dst, kbase + off, valid);
        cp_async16(stage_v(st) + dst, vbase + off, valid);
      }
      cp_async_mbar_arrive(&full[st]);
    }
    cp_async_wait_all();  // no copy may land after the ring is reused or the CTA exits
  } else if (warp < nwc) {
    // ---- consumer (ri, kw)
    // Q fragments (A operand, rows g / g + 8 of the tile) straight from global.
    const bf16* qb = static_cast<const bf16*>(a.q);
    const bf16* qrow0 = qb + (int64_t)(qr0 / a.G) * a.ldq + (int64_t)(h * a.G + qr0 % a.G) * HD;
    const bf16* qrow1 = qb + (int64_t)(qr1 / a.G) * a.ldq + (int64_t)(h * a.G + qr1 % a.G) * HD;
    uint32_t qf[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int c0 = ks * 16 + 2 * tq;
      qf[ks][0] = ok0 ? *reinterpret_cast<const uint32_t*>(qrow0 + c0) : 0u;
      qf[ks][1] = ok1 ? *reinterpret_cast<const uint32_t*>(qrow1 + c0) : 0u;
      qf[ks][2] = ok0 ? *reinterpret_cast<const uint32_t*>(qrow0 + c0 + 8) : 0u;
      qf[ks][3] = ok1 ? *reinterpret_cast<const uint32_t*>(qrow1 + c0 + 8) : 0u;
    }
    const int tok0 = ok0 ? qr0 / a.G - t_first : 0, tok1 = ok1 ? qr1 / a.G - t_first : 0;
    const int pl0 = ok0 ? s_plen[tok0] : 0, pl1 = ok1 ? s_plen[tok1] : 0;
    const int ps0 = ok0 ? s_pstart[tok0] : 0, ps1 = ok1 ? s_pstart[tok1] : 0;
    const float sc = a.scale * 1.4426950408889634f;  // softmax in base 2
    const int mi = lane >> 3, rj = lane & 7;
    for (int b = kw; b < nblocks; b += a.kw) {
      const int st = b % kWsStages;
      if (!mbar_wait(&full[st], (b / kWsStages) & 1)) {
        if (lane == 0) report_error(a.status, kErrWaitTimeout);
        failed = true;
        break;
      }
      const int kb = k_lo + b * KB;
      float sacc[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int ntp = 0; ntp < 4; ++ntp) {
          const int key = (2 * ntp + (mi >> 1)) * 8 + rj;
          const int c = 2 * ks + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(stage_k(st) + key * HD * 2 + ((c ^ (key & 7)) << 4), b0, b1, b2, b3);
          mma_16816(sacc[2 * ntp], qf[ks], b0, b1);
          mma_16816(sacc[2 * ntp + 1], qf[ks], b2, b3);
        }
      }
      // scale + mask: rows rl0 (sacc[.][0..1]) and rl1 (sacc[.][2..3]); this
      // lane holds keys nt * 8 + 2 * tq + {0, 1} of each n-tile
      const uint64_t vb0 = ok0 ? key_block_bits(kb, k_hi, pl0, s_mask + tok0 * 4, mw, sb, ps0) >> (2 * tq) : 0ull;
      const uint64_t vb1 = ok1 ? key_block_bits(kb, k_hi, pl1, s_mask + tok1 * 4, mw, sb, ps1) >> (2 * tq) : 0ull;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint64_t vb = e >= 2 ? vb1 : vb0;
          const bool ok = ((vb >> (nt * 8 + (e & 1))) & 1ull) != 0ull;
          sacc[nt][e] = ok ? sacc[nt][e] * sc : -INFINITY;
        }
      }
      // online softmax (each row is shared by the 4 lanes of a quad)
      float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        bm0 = fmaxf(bm0, fmaxf(sacc[nt][0], sacc[nt][1]));
        bm1 = fmaxf(bm1, fmaxf(sacc[nt][2], sacc[nt][3]));
      }
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
        bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
      }
      const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
      const float al0 = (mn0 == -INFINITY || m0 == -INFINITY) ? (m0 == -INFINITY ? 0.f : 1.f) : exp2f(m0 - mn0);
      const float al1 = (mn1 == -INFINITY || m1 == -INFINITY) ? (m1 == -INFINITY ? 0.f : 1.f) : exp2f(m1 - mn1);
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        sacc[nt][0] = (sacc[nt][0] == -INFINITY) ? 0.f : exp2f(sacc[nt][0] - mn0);
        sacc[nt][1] = (sacc[nt][1] == -INFINITY) ? 0.f : exp2f(sacc[nt][1] - mn0);
        sacc[nt][2] = (sacc[nt][2] == -INFINITY) ? 0.f : exp2f(sacc[nt][2] - mn1);
        sacc[nt][3] = (sacc[nt][3] == -INFINITY) ? 0.f : exp2f(sacc[nt][3] - mn1);
        ps0 += sacc[nt][0] + sacc[nt][1];
        ps1 += sacc[nt][2] + sacc[nt][3];
      }
      l0 = l0 * al0 + ps0;
      l1 = l1 * al1 + ps1;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int dt = 0; dt < NTD; ++dt) {
        o[dt][0] *= al0;
        o[dt][1] *= al0;
        o[dt][2] *= al1;
        o[dt][3] *= al1;
      }
      // O += P V
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t pf[4];
        pf[0] = pack_bf16(sacc[2 * kk][0], sacc[2 * kk][1]);
        pf[1] = pack_bf16(sacc[2 * kk][2], sacc[2 * kk][3]);
        pf[2] = pack_bf16(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
        pf[3] = pack_bf16(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
#pragma unroll
        for (int dtp = 0; dtp < NTD / 2; ++dtp) {
          const int key = 16 * kk + (mi & 1) * 8 + rj;
          const int c = 2 * dtp + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(stage_v(st) + key * HD * 2 + ((c ^ (key & 7)) << 4), b0, b1, b2, b3);
          mma_16816(o[2 * dtp], pf, b0, b1);
          mma_16816(o[2 * dtp + 1], pf, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    // row sums across the quad
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
  }
  // Every consumer is done with the ring (and the producer's copies have
  // landed): the ring becomes the partial records. A CTA that hit a wait
  // limit still takes part in the barriers below, so its cluster peers finish.
  __syncthreads();
  bf16* outp = static_cast<bf16*>(a.out);
  if (P == 1) {
    if (warp < nwc) {
      const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
      bf16* o0 = outp + (int64_t)(qr0 / a.G) * a.ldo + (int64_t)(h * a.G + qr0 % a.G) * HD;
      bf16* o1 = outp + (int64_t)(qr1 / a.G) * a.ldo + (int64_t)(h * a.G + qr1 % a.G) * HD;
#pragma unroll
      for (int dt = 0; dt < NTD; ++dt) {
        const int d = dt * 8 + 2 * tq;
        if (ok0) *reinterpret_cast<uint32_t*>(o0 + d) = pack_bf16(o[dt][0] * i0, o[dt][1] * i0);
        if (ok1) *reinterpret_cast<uint32_t*>(o1 + d) = pack_bf16(o[dt][2] * i1, o[dt][3] * i1);
      }
    }
    return;
  }
  const int rec = mma_rec(HD);
  constexpr int DPL = HD / 32;  // dims per lane (2 or 4)
  // Merge one row over its P partials (p = slice * kw + key lane), weights
  // from the (m, l) pairs, accumulation in p order.
  auto merge_row = [&](int r, auto&& rec_at) {
    const int qr = q0 + r;
    float ms = -INFINITY, ls = 0.f;
    if (lane < P) {
      ms = rec_at(lane, 0);
      ls = rec_at(lane, 1);
    }
    const float Mx = warp_max(ms);
    const float wgt = (ms == -INFINITY || Mx == -INFINITY) ? 0.f : exp2f(ms - Mx);
    const float L = warp_sum(ls * wgt);
    float acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
    for (int p0 = 0; p0 < P; p0 += 8) {
      float v[8][DPL];
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int i = 0; i < DPL; ++i) v[u][i] = (p0 + u < P) ? rec_at(p0 + u, 4 + lane * DPL + i) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float ws = __shfl_sync(0xffffffffu, wgt, (p0 + u) & 31);
        if (p0 + u < P) {
#pragma unroll
          for (int i = 0; i < DPL; ++i) acc[i] = fmaf(ws, v[u][i], acc[i]);
        }
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    bf16* op = outp + (int64_t)(qr / a.G) * a.ldo + (int64_t)(h * a.G + qr % a.G) * HD + lane * DPL;
#pragma unroll
    for (int i = 0; i < DPL; ++i) op[i] = f2bf(acc[i] * inv);
  };
  if (a.cluster_merge || a.n_splits == 1) {
    // Push: every consumer stores its rows' partials straight into the
    // receive area of the CTA that merges the row (rank r % slices; DSMEM
    // stores, no remote loads), then one barrier, then a local merge.
    const int ns = a.n_splits;
    const int owned = (a.rows_per_group + ns - 1) / ns;
    float* recv = reinterpret_cast<float*>(attn_smem + ws_ring_bytes(HD));
    const uint32_t recv_s = smem_u32(recv);
    if (warp < nwc) {
      const int p = split * a.kw + kw;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int rl = half ? rl1 : rl0;
        if (!(half ? ok1 : ok0)) continue;
        const int owner = rl % ns, j = rl / ns;
        const uint32_t dst0 = (uint32_t)(((p * owned + j) * rec) * 4);
        const float mm = half ? m1 : m0, ll = half ? l1 : l0;
        if (a.cluster_merge) {
          const uint32_t base = dsmem_map(recv_s, static_cast<uint32_t>(owner));
          if (tq == 0) dsmem_st2(base + dst0, mm, ll);
#pragma unroll
          for (int dt = 0; dt < NTD; ++dt) {
            const int d = 4 + dt * 8 + 2 * tq;
            dsmem_st2(base + dst0 + d * 4, half ? o[dt][2] : o[dt][0], half ? o[dt][3] : o[dt][1]);
          }
        } else {
          float* dst = recv + (p * owned + j) * rec;
          if (tq == 0) {
            dst[0] = mm;
            dst[1] = ll;
          }
#pragma unroll
          for (int dt = 0; dt < NTD; ++dt) {
            const int d = 4 + dt * 8 + 2 * tq;
            *reinterpret_cast<float2*>(dst + d) =
                make_float2(half ? o[dt][2] : o[dt][0], half ? o[dt][3] : o[dt][1]);
          }
        }
      }
    }
    if (a.cluster_merge)
      cluster_sync_all();
    else
      __syncthreads();
    const int n_own = Mg > split ? (Mg - split + ns - 1) / ns : 0;
    for (int j = warp; j < n_own; j += nwarps) {
      auto at = [&](int pp, int f) { return recv[(pp * owned + j) * rec + f]; };
      merge_row(split + j * ns, at);
    }
    return;
  }
  // Long contexts: records in the global workspace slot of (row group,
  // slice); the last slice to finish merges.
  float* recs = a.part + ((int64_t)blk * a.n_splits + split) * a.kw * a.rows_per_group * rec;
  if (warp < nwc) {
    float* p0 = recs + ((int64_t)kw * a.rows_per_group + rl0) * rec;
    float* p1 = recs + ((int64_t)kw * a.rows_per_group + rl1) * rec;
    if (tq == 0) {
      if (ok0) {
        p0[0] = m0;
        p0[1] = l0;
      }
      if (ok1) {
        p1[0] = m1;
        p1[1] = l1;
      }
    }
#pragma unroll
    for (int dt = 0; dt < NTD; ++dt) {
      const int d = 4 + dt * 8 + 2 * tq;
      if (ok0) *reinterpret_cast<float2*>(p0 + d) = make_float2(o[dt][0], o[dt][1]);
      if (ok1) *reinterpret_cast<float2*>(p1 + d) = make_float2(o[dt][2], o[dt][3]);
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(&a.counters[kAttnCounterBase + blk], 1u);
    s_misc[2] = (prev == (uint32_t)(a.n_splits - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (!s_misc[2]) return;
  __threadfence();
  const float* gbase = a.part + (int64_t)blk * a.n_splits * a.kw * a.rows_per_group * rec;
  for (int r = warp; r < Mg; r += nwarps) {
    auto at = [&](int p, int f) { return __ldcg(gbase + ((int64_t)p * a.rows_per_group + r) * rec + f); };
    merge_row(r, at);
  }
  if (threadIdx.x == 0) a.counters[kAttnCounterBase + blk] = 0u;
}

// ------------------------------------------------------------ tcgen05 kernel
// KV head and row group of tcgen05-kernel CTA column blk (and of its merge):
// heads vary fastest and the row groups run from the last to the first, so
// under a causal mask (prefill) the CTAs with the most keys start in the
// first wave and the short ones fill the tail.
__device__ __forceinline__ void tc_head_group(const AttnArgs& a, int blk, int& h, int& gr) {
  h = blk % a.n_kv;
  gr = a.groups - 1 - blk / a.n_kv;
}

// bf16, head_dim 64 or 128. A CTA = one KV head x up to 128 query rows (one
// M = 128 tcgen05 tile; rows past the group are zero) x one key slice.
// Warp 0 streams the slice's 64-key K and V blocks by TMA (128-byte swizzle,
// straight from the cache rows) into a kTcAttnStages ring. Warp 1 (one
// lane) issues S = Q K^T into one of two TMEM S buffers and O += P V into
// one of two TMEM O accumulators (V read MN-major as stored). On long slices
// two softmax warpgroups split the key blocks: warps 2..5 take the even blocks
// (S, P and O buffers 0), warps 6..9 the odd ones (buffers 1), so each SM
// sub-partition runs two softmax warps; on short slices warps 2..5 take every
// block (S and P buffers alternate, one O accumulator). A softmax thread owns one query row (= TMEM lane):
// it loads S, applies the tree mask, runs the online softmax in base 2 with a
// lazy reference max (P = 2^(s - m_ref) stays below 2^8, so O is rescaled
// only when a row's max grows by more than 8) and writes P as bf16 into
// shared memory for the P V product. At the end the two warpgroups combine
// their (max, sum, O) states of each row; each writes half of the columns. Partials of the key slices merge as in the mma.sync
// kernel: pushed into the merging CTA of the cluster, or through global
// memory for long contexts.
// 2^x on the special-function unit (PTX ex2.approx.ftz.f32; 2^-inf = +0).
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr int kTcAttnStages = 4;
constexpr int kTcAttnMaxTok = 129;  // token rows spanned by 128 query rows (keeps the metadata 8-byte aligned)
constexpr int kTcAttnThreads = 352;  // K TMA warp, MMA warp, two softmax warpgroups, V TMA warp
constexpr int kTcAttnVWarp = 10;
constexpr float kLazyRescale = 8.f;  // log2 headroom of P before O is rescaled
// Key blocks per CTA from which the second softmax warpgroup takes the odd
// blocks (below it warps 2..5 take every block and accumulator 1 stays
// unused). Since S and P.V issue independently, two warpgroups pay from a few
// blocks on (measured: 3 and 6 equal 12 on long slices, 3 is 0.4 µs faster
// per launch at 1k keys).
constexpr int kTcTwoGroupsMinBlocks = 4;

struct AttnMaps {
  CUtensorMap k;  // [n_kv * max_slots, hd] bf16, box {64, 64}
  CUtensorMap v;
  CUtensorMap q;  // [T][n_heads][hd] bf16 (token stride ldq), box {64, G, 128 / G}: 128 query rows
};

template <int HD>
struct TcAttnLayout {
  static constexpr int NR = HD / 64;                 // 128-byte regions per K/V/Q row
  static constexpr int Q_BYTES = NR * 128 * 128;     // NR regions of [128 rows x 128 B]
  static constexpr int KV_REGION = 64 * 128;         // [64 keys x 128 B]
  static constexpr int STAGE = 2 * NR * KV_REGION;   // K regions, then V regions
  static constexpr int P_BYTES = 128 * 128;          // [128 rows x 64 keys] bf16
  static constexpr int OFF_RING = Q_BYTES;
  static constexpr int OFF_P = Q_BYTES + kTcAttnStages * STAGE;
  static constexpr int OFF_META = OFF_P + 2 * P_BYTES;
  static constexpr int META = (kTcAttnMaxTok + 1) * 4 + kTcAttnMaxTok * 4 * 8 + 16 + (4 * kTcAttnStages + 10) * 8 + 16 +
                              (kTcAttnMaxTok + 1) * 4;
  static constexpr int SMEM = 1024 + OFF_META + META;
};

template <int HD>
__global__ void __launch_bounds__(kTcAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ AttnMaps maps, const AttnArgs a) {
  using Lay = TcAttnLayout<HD>;
  constexpr int NR = Lay::NR;
  constexpr int KB = 64;
  extern __shared__ uint8_t attn_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(attn_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = sm;
  uint8_t* ring = sm + Lay::OFF_RING;
  uint8_t* ps = sm + Lay::OFF_P;
  int* s_plen = reinterpret_cast<int*>(sm + Lay::OFF_META);
  uint64_t* s_mask = reinterpret_cast<uint64_t*>(s_plen + kTcAttnMaxTok + 1);  // [tok][4]
  int* s_misc = reinterpret_cast<int*>(s_mask + kTcAttnMaxTok * 4);           // need_end, min_plen, last, abort
  // K and V halves of a ring stage fill and free separately: K(b) frees
  // once S(b) is computed, V(b) once P.V(b) is, so keys run ahead of values.
  uint64_t* kv_full = reinterpret_cast<uint64_t*>(s_misc + 4);  // K half of stage landed
  uint64_t* kv_empty = kv_full + kTcAttnStages;                  // K half read by S
  uint64_t* v_full = kv_empty + kTcAttnStages;
  uint64_t* v_empty = v_full + kTcAttnStages;
  uint64_t* s_full = v_empty + kTcAttnStages;  // [2]
  uint64_t* s_free = s_full + 2;                // [2]
  uint64_t* p_full = s_free + 2;                // [2]
  uint64_t* p_free = p_full + 2;                // [2]
  uint64_t* o_full = p_free + 2;
  uint64_t* q_ready = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_ready + 1);
  int* s_pstart = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(tmem_slot) + 16);  // [tok]
  volatile int* abort_flag = s_misc + 3;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = blockIdx.x;
  int h, gr;
  tc_head_group(a, blk, h, gr);
  const int split = blockIdx.y;
  const int M = a.T * a.G;
  const int q0 = gr * a.rows_per_group;
  const int Mg = min(a.rows_per_group, M - q0);
  const int t_first = q0 / a.G;
  const int ntok = (q0 + Mg - 1) / a.G - t_first + 1;
  const int P = a.n_splits;

  // Set-up that reads nothing an earlier kernel writes runs before the
  // programmatic-launch wait: barriers, TMEM, tensor-map prefetch.
  if (threadIdx.x == 0) {
    s_misc[0] = 0;
    s_misc[1] = INT32_MAX;
    s_misc[3] = 0;
    for (int st = 0; st < kTcAttnStages; ++st) {
      mbar_init(&kv_full[st], 1);
      mbar_init(&kv_empty[st], 1);
      mbar_init(&v_full[st], 1);
      mbar_init(&v_empty[st], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(q_ready, 1);  // the Q boxes landed
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.k);
    tma_prefetch_desc(&maps.v);
    tma_prefetch_desc(&maps.q);
  }
  tc_fence_before();
  __syncthreads();  // barriers, TMEM and the meta accumulators are initialised
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // Q, the new K/V rows and the row metadata come from earlier kernels
  pdl_trigger();
  if (warp == 0 && lane == 0) {
    // Q rows (A operand, K-major, 128-byte swizzle): per head g of the
    // group and 64 columns, one 3-D box of TPG = 128 / G tokens from t_first
    // lands at tile rows g * TPG.. (head-major; row groups start on a
    // token); rows past the tensor are zero, rows past the group masked.
    const int tpg = 128 / a.G;
    mbar_arrive_expect_tx(q_ready, NR * a.G * tpg * 128);
    const uint64_t pol = l2_policy_evict_first();
    for (int g = 0; g < a.G; ++g)
#pragma unroll
      for (int c = 0; c < NR; ++c)
        tma_load_3d(qs + c * (128 * 128) + g * tpg * 128, &maps.q, q_ready, c * 64, h * a.G + g, t_first, pol);
  }
  const int sb = a.spec_base ? a.spec_base[0] : 0;
  const int mw = a.mask ? a.mask_words : 0;
  for (int i = threadIdx.x; i < ntok; i += blockDim.x) {
    const int t = t_first + i;
    const int pl = a.prefix_len[t];
    s_plen[i] = pl;
    s_pstart[i] = a.prefix_start ? a.prefix_start[t] : 0;
    int end = pl;
    for (int w = 0; w < mw; ++w) {
      const uint64_t m = a.mask[(int64_t)t * mw + w];
      s_mask[i * 4 + w] = m;
      if (m) end = max(end, sb + w * 64 + 64 - __clzll(m));
    }
    atomicMax(&s_misc[0], end);
    atomicMin(&s_misc[1], pl);
  }
  __syncthreads();  // per-token metadata complete
  const int need_end = min(min(s_misc[0], a.kv_bound), a.max_slots);
  const int slice = ((need_end + a.n_splits - 1) / a.n_splits + KB - 1) / KB * KB;
  const int k_lo = split * slice;
  const int k_hi = min(k_lo + slice, need_end);
  const int nblocks = k_hi > k_lo ? (k_hi - k_lo + KB - 1) / KB : 0;
  const bool two = nblocks >= a.two_min;  // CTA-uniform
  const uint32_t qs_s = smem_u32(qs), ring_s = smem_u32(ring), ps_s = smem_u32(ps);
  // TMEM columns: S buffers [0, 64) and [64, 128), O accumulators of the
  // even and odd key blocks at [128, 128 + HD) and [256, 256 + HD)
  const uint32_t tm_o = tmem + 128;

  // softmax-side state (warps 2..9): warpgroup wg takes key blocks wg, wg + 2, ...
  const int q = warp & 3;
  const int r = q * 32 + lane;  // tile row of this thread = TMEM lane
  const int wg = warp >= 6 ? 1 : 0;
  const bool softmax_warp = warp >= 2 && warp <= 9;
  // Tile rows are head-major: rows g * TPG .. g * TPG + TPG - 1 hold head g
  // of the group for its tokens, so the valid rows of a small group spread
  // over all four TMEM lane quarters (and SM sub-partitions) instead of
  // filling the first ones. lr = the row's logical index (token * G + head),
  // which the metadata, the slice records and the output use.
  const int TPG = 128 / a.G;
  const int lr = (r % TPG) * a.G + r / TPG;
  const bool row_ok = softmax_warp && lr < Mg;
  float m_ref = -INFINITY, l = 0.f;

  if (warp == 0 || warp == kTcAttnVWarp) {
    // One thread issues a TMA stream at ~35-45 GB/s on B200, below what a
    // CTA that owns an SM needs, so K and V have a producer each (warp 0
    // lane 0: K of block b once S(b - 4) freed its half-stage; warp 10 lane
    // 0: V of block b once P.V(b - 4) freed its half).
    if (lane == 0 && nblocks > 0) {
      const bool is_v = warp == kTcAttnVWarp;
      const uint64_t pol = l2_policy_evict_first();
      constexpr int S = kTcAttnStages;
      uint64_t* fullb = is_v ? v_full : kv_full;
      uint64_t* emptyb = is_v ? v_empty : kv_empty;
      const CUtensorMap* map = is_v ? &maps.v : &maps.k;
      int issued = 0;
      for (int b = 0; b < nblocks; ++b) {
        const int st = b % S;
        if ((b >= S && !mbar_wait(&emptyb[st], ((b / S) - 1) & 1)) || *abort_flag) {
          report_error(a.status, kErrWaitTimeout);
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&fullb[st], NR * Lay::KV_REGION);
        const int row = h * a.max_slots + k_lo + b * KB;
        uint8_t* dst = ring + st * Lay::STAGE + (is_v ? NR * Lay::KV_REGION : 0);
#pragma unroll
        for (int g = 0; g < NR; ++g) tma_load_2d(dst + g * Lay::KV_REGION, map, &fullb[st], g * 64, row, pol);
        ++issued;
      }
      if (*abort_flag) {  // let every copy already issued land before the CTA moves on
        for (int b = (issued > S ? issued - S : 0); b < issued; ++b) (void)mbar_wait(&fullb[b % S], (b / S) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16_f32(128, KB);
      const uint32_t id_pv = idesc_bf16_f32_bmn(128, HD);
      bool ok = mbar_wait(q_ready, 0);
      if (!ok) {
        report_error(a.status, kErrWaitTimeout);
        *abort_flag = 1;
      }
      // S = Q K^T of block b needs its K block and a free S buffer (the
      // softmax of block b - 2 has loaded its scores); O += P V of block b
      // needs its P and its V block. Neither waits for the other: the thread polls both and
      // issues whichever is ready, so the scores of the next blocks are
      // computed while the softmax warps still work on earlier ones. (Each
      // barrier can be at most one phase ahead of the one tested: its next
      // phase needs an MMA this thread has not issued yet.)
      int nS = 0, nP = 0;
      uint32_t idle = 0;
      while (ok && nP < nblocks) {
        bool prog = false;
        if (nS < nblocks && mbar_test(&kv_full[nS % kTcAttnStages], (nS / kTcAttnStages) & 1) &&
            (nS < 2 || mbar_test(&s_free[nS & 1], ((nS >> 1) - 1) & 1))) {
          tc_fence_after();
          const uint32_t kb = ring_s + (nS % kTcAttnStages) * Lay::STAGE;
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks) {
            const uint32_t off = (ks & 3) * 32;
            umma_bf16(tmem + (nS & 1) * KB, sdesc_k_sw128(qs_s + (ks >> 2) * (128 * 128) + off),
                      sdesc_k_sw128(kb + (ks >> 2) * Lay::KV_REGION + off), id_s, ks > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[nS & 1]);
          umma_commit(&kv_empty[nS % kTcAttnStages]);  // the K half may take block nS + 4
          ++nS;
          prog = true;
        }
        if (nP < nS && mbar_test(&p_full[nP & 1], (nP >> 1) & 1) &&
            mbar_test(&v_full[nP % kTcAttnStages], (nP / kTcAttnStages) & 1)) {
          tc_fence_after();
          const int j = nP;
          const uint32_t vb = ring_s + (j % kTcAttnStages) * Lay::STAGE + NR * Lay::KV_REGION;
          const uint32_t pb = ps_s + (j & 1) * Lay::P_BYTES;
#pragma unroll
          for (int kk = 0; kk < KB / 16; ++kk)
            umma_bf16(tm_o + (two ? (j & 1) * 128 : 0), sdesc_k_sw128(pb + kk * 32),
                      sdesc_mn_sw128(vb + kk * 2048, Lay::KV_REGION, 1024), id_pv,
                      (j > (two ? 1 : 0) || kk > 0) ? 1u : 0u);
          umma_commit(&p_free[j & 1]);
          umma_commit(&v_empty[j % kTcAttnStages]);
          ++nP;
          prog = true;
        }
        idle = prog ? 0u : idle + 1u;
        if (idle > kWaitLimit || *abort_flag) {
          report_error(a.status, kErrWaitTimeout);
          *abort_flag = 1;
          ok = false;
        }
        if (!prog) __nanosleep(32);  // (see the producer)
      }
      // Arrives once every MMA above has retired (also after an abort).
      umma_commit(o_full);
    }
  } else {
    // ---- softmax warps: thread = query row r
    const int tok = row_ok ? (q0 + lr) / a.G - t_first : 0;
    const int plen = row_ok ? s_plen[tok] : 0;
    const int pstart = row_ok ? s_pstart[tok] : 0;
    const float sc = a.scale * 1.4426950408889634f;  // base 2
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    bool bad = false;
    const uint32_t tm_ow = tm_o + (two ? wg * 128 : 0);
    const int b0 = two ? wg : (wg == 0 ? 0 : nblocks), bstep = two ? 2 : 1;
    for (int b = b0; b < nblocks; b += bstep) {
      const int sbuf = b & 1;
      bad = !mbar_wait(&s_full[sbuf], (b >> 1) & 1) || *abort_flag;
      if (__any_sync(0xffffffffu, bad)) {
        if (lane == 0) {
          report_error(a.status, kErrWaitTimeout);
          *abort_flag = 1;
        }
        bad = true;
        break;
      }
      tc_fence_after();
      float sv[KB];
      tmem_ld64(tmem + lane_base + sbuf * KB, sv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[sbuf]);
      const int kb = k_lo + b * KB;
      const uint64_t vbits = row_ok ? key_block_bits(kb, k_hi, plen, s_mask + tok * 4, mw, sb, pstart) : 0ull;
      const uint32_t vlo = static_cast<uint32_t>(vbits), vhi = static_cast<uint32_t>(vbits >> 32);
      float bmx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < KB; ++j) {
        const bool ok = ((j < 32 ? vlo >> j : vhi >> (j - 32)) & 1u) != 0u;
        const float v = ok ? sv[j] * sc : -INFINITY;
        sv[j] = v;
        bmx[j & 3] = fmaxf(bmx[j & 3], v);
      }
      const float bm = fmaxf(fmaxf(bmx[0], bmx[1]), fmaxf(bmx[2], bmx[3]));
      const bool grow = bm > m_ref + kLazyRescale || (m_ref == -INFINITY && bm > -INFINITY);
      if (__any_sync(0xffffffffu, grow)) {
        const float m_new = grow ? bm : m_ref;
        const float alpha = (!grow || m_ref == -INFINITY) ? (grow ? 0.f : 1.f) : exp2f(m_ref - m_new);
        if (b >= bstep) {
          // this warpgroup's O holds earlier blocks: rescale it once P V of
          // its previous block b - bstep is done
          const int pb = b - bstep;
          const bool w_ok = mbar_wait(&p_free[pb & 1], (pb >> 1) & 1);
          if (!w_ok) report_error(a.status, kErrWaitTimeout);
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < HD; c += 16) {
            float ov[16];
            tmem_ld16(tm_ow + lane_base + c, ov);
#pragma unroll
            for (int i = 0; i < 16; ++i) ov[i] *= alpha;
            tmem_st16(tm_ow + lane_base + c, ov);
          }
          tmem_wait_st();
        }
        l *= alpha;
        m_ref = m_new;
      }
      uint32_t pk[KB / 2];
      float lsx[4] = {0.f, 0.f, 0.f, 0.f};
      const float mr = m_ref == -INFINITY ? 0.f : m_ref;  // a row with no key yet has only -inf scores
#pragma unroll
      for (int j = 0; j < KB; j += 2) {
        const float p0 = ex2_fast(sv[j] - mr);
        const float p1 = ex2_fast(sv[j + 1] - mr);
        lsx[(j >> 1) & 3] += p0 + p1;
        pk[j >> 1] = pack_bf16(p0, p1);
      }
      l += (lsx[0] + lsx[1]) + (lsx[2] + lsx[3]);
      if (b >= 2) {
        const bool w_ok = mbar_wait(&p_free[sbuf], ((b - 2) >> 1) & 1);  // P V of block b - 2 read this buffer
        if (!w_ok) report_error(a.status, kErrWaitTimeout);
      }
      uint8_t* prow = ps + sbuf * Lay::P_BYTES + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sbuf]);
    }
    (void)bad;
  }
  // ---- results: the two softmax warpgroups combine their states of each
  // row (base 2) and each reads half of the O columns of both accumulators
  constexpr int HH = HD / 2;
  float ov[HH];
#pragma unroll
  for (int i = 0; i < HH; ++i) ov[i] = 0.f;
  float Mrow = -INFINITY, Lrow = 0.f;
  const int c0 = wg * HH;
  if (softmax_warp) {
    const bool w_ok = mbar_wait(o_full, 0);
    if (!w_ok) report_error(a.status, kErrWaitTimeout);
    tc_fence_after();
    float* s_ml = reinterpret_cast<float*>(ps);  // the P buffers are free once every P V retired
    s_ml[(wg * 128 + r) * 2] = m_ref;
    s_ml[(wg * 128 + r) * 2 + 1] = l;
    named_bar_sync(3, 256);  // the eight softmax warps
    const float m0 = s_ml[r * 2], l0 = s_ml[r * 2 + 1];
    const float m1 = s_ml[(128 + r) * 2], l1 = s_ml[(128 + r) * 2 + 1];
    Mrow = fmaxf(m0, m1);
    const float a0 = m0 == -INFINITY ? 0.f : exp2f(m0 - Mrow);
    const float a1 = m1 == -INFINITY ? 0.f : exp2f(m1 - Mrow);
    Lrow = a0 * l0 + a1 * l1;
    // accumulator 0 holds data once a block ran, accumulator 1 once two did
    if (__all_sync(0xffffffffu, nblocks > 0 && w_ok && !*abort_flag)) {
      const uint32_t lb = static_cast<uint32_t>(q * 32) << 16;
#pragma unroll
      for (int i = 0; i < HH; i += 16) {
        float x[16], y[16];
        tmem_ld16(tm_o + lb + c0 + i, x);
        if (two && nblocks > 1) {
          tmem_ld16(tm_o + 128 + lb + c0 + i, y);
        } else {
#pragma unroll
          for (int k = 0; k < 16; ++k) y[k] = 0.f;
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) ov[i + k] = a0 * x[k] + a1 * y[k];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  bf16* outp = static_cast<bf16*>(a.out);
  if (P == 1) {
    if (row_ok) {
      const float inv = Lrow > 0.f ? 1.f / Lrow : 0.f;
      const int qr = q0 + lr;
      bf16* op = outp + (int64_t)(qr / a.G) * a.ldo + (int64_t)(h * a.G + qr % a.G) * HD + c0;
#pragma unroll
      for (int d = 0; d < HH; d += 2) *reinterpret_cast<uint32_t*>(op + d) = pack_bf16(ov[d] * inv, ov[d + 1] * inv);
    }
    return;
  }
  const int rec = mma_rec(HD);
  constexpr int DPL = HD / 32;
  const int nwarps = kTcAttnThreads / 32;
  auto merge_row = [&](int rr, auto&& rec_at) {
    const int qr = q0 + rr;
    float ms = -INFINITY, ls = 0.f;
    if (lane < P) {
      ms = rec_at(lane, 0);
      ls = rec_at(lane, 1);
    }
    const float Mx = warp_max(ms);
    const float wgt = (ms == -INFINITY || Mx == -INFINITY) ? 0.f : exp2f(ms - Mx);
    const float L = warp_sum(ls * wgt);
    float acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
    for (int p0 = 0; p0 < P; p0 += 8) {
      float v[8][DPL];
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int i = 0; i < DPL; ++i) v[u][i] = (p0 + u < P) ? rec_at(p0 + u, 4 + lane * DPL + i) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float ws = __shfl_sync(0xffffffffu, wgt, (p0 + u) & 31);
        if (p0 + u < P) {
#pragma unroll
          for (int i = 0; i < DPL; ++i) acc[i] = fmaf(ws, v[u][i], acc[i]);
        }
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    bf16* op = outp + (int64_t)(qr / a.G) * a.ldo + (int64_t)(h * a.G + qr % a.G) * HD + lane * DPL;
#pragma unroll
    for (int i = 0; i < DPL; ++i) op[i] = f2bf(acc[i] * inv);
  };
  if (a.cluster_merge) {
    // Every slice of the cluster is past its key loop: the rings are free and
    // become the receive areas. Push, barrier, merge locally.
    cluster_sync_all();
    const int ns = a.n_splits;
    const int owned = (a.rows_per_group + ns - 1) / ns;
    float* recv = reinterpret_cast<float*>(ring);
    if (row_ok) {
      const int owner = lr % ns, j = lr / ns;
      const uint32_t base = dsmem_map(smem_u32(recv), static_cast<uint32_t>(owner)) +
                            (uint32_t)(((split * owned + j) * rec) * 4);
      if (wg == 0) dsmem_st4(base, Mrow, Lrow, 0.f, 0.f);
#pragma unroll
      for (int d = 0; d < HH; d += 4)
        dsmem_st4(base + (uint32_t)(4 + c0 + d) * 4, ov[d], ov[d + 1], ov[d + 2], ov[d + 3]);
    }
    cluster_sync_all();
    const int n_own = Mg > split ? (Mg - split + ns - 1) / ns : 0;
    for (int j = warp; j < n_own; j += nwarps) {
      auto at = [&](int pp, int f) { return recv[(pp * owned + j) * rec + f]; };
      merge_row(split + j * ns, at);
    }
    return;
  }
  // Long contexts: records in the global workspace slot of (row group,
  // slice); attn_merge_kernel combines the slices of every row in parallel.
  float* recs = a.part + ((int64_t)blk * a.n_splits + split) * a.rows_per_group * rec;
  if (row_ok) {
    float* pr = recs + (int64_t)lr * rec;
    if (wg == 0) {
      pr[0] = Mrow;
      pr[1] = Lrow;
    }
#pragma unroll
    for (int d = 0; d < HH; d += 2) *reinterpret_cast<float2*>(pr + 4 + c0 + d) = make_float2(ov[d], ov[d + 1]);
  }
}

// Merge of the key-slice records written by attn_tc_kernel (long contexts):
// one warp per query row, all rows of all row groups in parallel. Slices
// combine in a fixed order (max, then weighted sums in slice order), lane l
// owning columns l * HD/32 ...; the same arithmetic as the in-kernel merges.
template <int HD>
__global__ void __launch_bounds__(256) attn_merge_kernel(const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int DPL = HD / 32;
  const int blk = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rr = blockIdx.y * 8 + warp;
  int h, gr;
  tc_head_group(a, blk, h, gr);
  const int M = a.T * a.G;
  const int q0 = gr * a.rows_per_group;
  const int Mg = min(a.rows_per_group, M - q0);
  if (rr >= Mg) return;
  const int P = a.n_splits, rec = mma_rec(HD);
  const float* base = a.part + (int64_t)blk * P * a.rows_per_group * rec + (int64_t)rr * rec;
  const int64_t sstride = (int64_t)a.rows_per_group * rec;
  float ms = -INFINITY, ls = 0.f;
  if (lane < P) {
    ms = base[lane * sstride];
    ls = base[lane * sstride + 1];
  }
  const float Mx = warp_max(ms);
  const float wgt = (ms == -INFINITY || Mx == -INFINITY) ? 0.f : exp2f(ms - Mx);
  const float L = warp_sum(ls * wgt);
  float acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
  for (int p0 = 0; p0 < P; p0 += 16) {
    float v[16][DPL];
#pragma unroll
    for (int u = 0; u < 16; ++u)
#pragma unroll
      for (int i = 0; i < DPL; ++i) v[u][i] = (p0 + u < P) ? base[(p0 + u) * sstride + 4 + lane * DPL + i] : 0.f;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const float ws = __shfl_sync(0xffffffffu, wgt, (p0 + u) & 31);
      if (p0 + u < P) {
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[i] = fmaf(ws, v[u][i], acc[i]);
      }
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const int qr = q0 + rr;
  bf16* op = static_cast<bf16*>(a.out) + (int64_t)(qr / a.G) * a.ldo + (int64_t)(h * a.G + qr % a.G) * HD + lane * DPL;
#pragma unroll
  for (int i = 0; i < DPL; ++i) op[i] = f2bf(acc[i] * inv);
}

// Clusters of `s` CTAs (one row group's key slices) that can be resident at
// once, from the occupancy API; cached per kernel, size and device.
int attn_resident_clusters(void (*kern)(const AttnArgs), int s, size_t smem, int threads) {
  static std::mutex mu;
  static std::map<std::tuple<void*, int, size_t, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(reinterpret_cast<void*>(kern), s, smem, dev * 4096 + threads);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, s);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = s;
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

int attn_resident_clusters_tc(void (*kern)(const AttnMaps, const AttnArgs), int s, size_t smem, int threads) {
  static std::mutex mu;
  static std::map<std::tuple<void*, int, size_t, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(reinterpret_cast<void*>(kern), s, smem, dev * 4096 + threads);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, s);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = s;
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

// bf16 tree attention with more than 16 query rows per KV head runs on the
// tcgen05 kernel; SSD_ATTN=mma keeps every size on the mma.sync kernel.
// Key blocks per CTA from which the two softmax warpgroups of the tcgen05
// kernel split the blocks (SSD_ATTN_TWO_MIN overrides).
int attn_two_groups_min_blocks() {
  static const int v = [] {
    const char* e = getenv("SSD_ATTN_TWO_MIN");
    return e ? atoi(e) : kTcTwoGroupsMinBlocks;
  }();
  return v;
}
bool attn_use_tcgen05() {
  static const bool v = [] {
    const char* e = getenv("SSD_ATTN");
    return !(e && e[0] == 'm');
  }();
  return v;
}

}  // namespace ssd

using namespace ssd;

extern "C" int ssd_tree_attention(const void* q, int64_t ldq, int64_t T, int64_t n_heads, int64_t n_kv_heads,
                                  int64_t head_dim, const void* k_cache, const void* v_cache,
                                  int64_t cache_head_stride, int64_t max_slots, const int32_t* prefix_len,
                                  const int32_t* prefix_start,
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
  a.prefix_start = prefix_start;
  a.spec_base = spec_mask ? spec_base : nullptr;
  a.mask = spec_mask;
  a.mask_words = (int)mask_words;
  a.kv_bound = (int)kv_bound;
  a.out = out;
  a.ldo = ldo;
  a.status = status;
  a.scale = 1.0f / sqrtf((float)head_dim);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int sms = device_sms();
  // More than one 16-row tile of queries per KV head: the tcgen05 kernel
  // (measured faster from 32 rows up); decode-sized row counts stay on the
  // warp-specialised mma.sync kernel, whose key lanes split the slice.
  const int64_t G_heads = n_heads / n_kv_heads;
  if (dtype == SSD_BF16 && (head_dim == 64 || head_dim == 128) && T * G_heads > 16 && 128 % G_heads == 0 &&
      128 / G_heads >= 8 &&
      attn_use_tcgen05()) {
    // tcgen05 path: up to 128 query rows of a KV head per CTA (one M = 128
    // tile), key slices merged in a cluster or through global memory.
    // Row groups start on a token (rows_per_group a multiple of G); a
    // group's Q rows land as one 3-D TMA box of 128 / G tokens per head,
    // head-major in the tile (G divides 128 and each head's rows start on
    // a 1024-byte swizzle atom: 128 / G >= 8).
    const int64_t tok_per_tile = 128 / a.G;
    a.groups = (int)((T + tok_per_tile - 1) / tok_per_tile);
    a.rows_per_group = (int)(((T + a.groups - 1) / a.groups) * a.G);
    a.rt = 8;
    a.kw = 1;
    a.two_min = attn_two_groups_min_blocks();
    const int64_t blocks = (int64_t)a.n_kv * a.groups;
    if (blocks > 16384) return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: too many row groups");
    if ((int64_t)a.n_kv * max_slots > (int64_t)1 << 31)
      return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: cache too large for a tensor map");
    AttnMaps maps;
    int rc = tma_map_bf16_2d(k_cache, (uint64_t)head_dim, (uint64_t)(a.n_kv * max_slots), (uint64_t)head_dim * 2, 64,
                             &maps.k);
    if (rc) return rc;
    rc = tma_map_bf16_2d(v_cache, (uint64_t)head_dim, (uint64_t)(a.n_kv * max_slots), (uint64_t)head_dim * 2, 64,
                         &maps.v);
    if (rc) return rc;
    if (cache_head_stride != max_slots * head_dim)
      return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: K/V heads must be contiguous [n_kv, max_slots, hd]");
    if ((reinterpret_cast<uintptr_t>(q) & 15) || (ldq * 2) % 16)
      return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: q rows must be 16-byte aligned");
    {
      TensorMapEncodeFn encode = tensor_map_encoder();
      if (!encode) return fail(SSD_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
      cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)n_heads, (cuuint64_t)T};
      cuuint64_t strides[2] = {(cuuint64_t)head_dim * 2, (cuuint64_t)ldq * 2};
      cuuint32_t box[3] = {64u, 1u, (cuuint32_t)tok_per_tile};
      cuuint32_t estr[3] = {1u, 1u, 1u};
      const CUresult r = encode(&maps.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box,
                                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) return fail(SSD_ERR_CUDA, "ssd_tree_attention: Q tensor map (%d)", (int)r);
    }
    const size_t smem = head_dim == 128 ? TcAttnLayout<128>::SMEM : TcAttnLayout<64>::SMEM;
    void (*kern)(const AttnMaps, const AttnArgs) = head_dim == 128 ? attn_tc_kernel<128> : attn_tc_kernel<64>;
    static bool tset128 = false, tset64 = false;
    bool& set = head_dim == 128 ? tset128 : tset64;
    if (!set) {
      allow_max_dynamic_smem(kern);
      set = true;
    }
    // One CTA per SM: up to 8 slices merge in a cluster for <= 8k keys;
    // beyond, one wave of slices (blocks x slices <= SMs) and a separate
    // merge kernel.
    int64_t splits = sms / blocks;
    const int64_t by_len = (kv_bound + 255) / 256;
    if (splits > by_len) splits = by_len;
    if (kv_bound <= 8 * 1024) {
      if (splits > kMaxAttnClusterSplits) splits = kMaxAttnClusterSplits;
      while (splits > 1 && attn_resident_clusters_tc(kern, (int)splits, smem, kTcAttnThreads) < blocks) --splits;
    }
    if (splits > kMaxPartials) splits = kMaxPartials;
    if (splits < 1) splits = 1;
    const int64_t split_len = ((kv_bound + splits - 1) / splits + 63) / 64 * 64;
    a.split_len = (int)split_len;
    a.n_splits = (int)((kv_bound + split_len - 1) / split_len);
    a.cluster_merge = (a.n_splits > 1 && a.n_splits <= kMaxAttnClusterSplits && kv_bound <= 8 * 1024) ? 1 : 0;
    if (a.n_splits > 1 && !a.cluster_merge) {
      const int64_t need = kCounterBytes + blocks * a.n_splits * a.rows_per_group * mma_rec((int)head_dim) * 4;
      if (!workspace || need > workspace_bytes)
        return fail(SSD_ERR_WORKSPACE, "ssd_tree_attention: workspace too small (need %lld)", (long long)need);
      a.counters = static_cast<uint32_t*>(workspace);
      a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
    }
    rc = launch_kernel("attn_tc_kernel", kern, dim3((unsigned)blocks, (unsigned)a.n_splits), dim3(kTcAttnThreads),
                       smem, s, 1u, a.cluster_merge ? (unsigned)a.n_splits : 1u, maps, a);
    if (rc || a.n_splits == 1 || a.cluster_merge) return rc;
    const dim3 mgrid((unsigned)blocks, (unsigned)((a.rows_per_group + 7) / 8));
    return head_dim == 128 ? launch_kernel("attn_merge_kernel", attn_merge_kernel<128>, mgrid, dim3(256), 0, s, 1, 1, a)
                           : launch_kernel("attn_merge_kernel", attn_merge_kernel<64>, mgrid, dim3(256), 0, s, 1, 1, a);
  }
  if (dtype == SSD_BF16 && (head_dim == 64 || head_dim == 128)) {
    // Tensor-core path: all query rows of a KV head in as few CTAs as
    // possible (<= 8 row tiles of 16 per CTA); with fewer row tiles, up to 4
    // key lanes per CTA split the key slice.
    const int64_t M = T * a.G;
    const int64_t tiles = (M + 15) / 16;
    if (tiles <= kWsMaxConsumers) {
      a.groups = 1;
      a.rt = (int)tiles;
      a.kw = kWsMaxConsumers / a.rt < 4 ? kWsMaxConsumers / a.rt : 4;
    } else {
      a.groups = (int)((tiles + kWsMaxConsumers - 1) / kWsMaxConsumers);
      a.rt = (int)((tiles + a.groups - 1) / a.groups);
      a.kw = 1;
    }
    a.rows_per_group = a.rt * 16;
    const int threads = 32 * (a.rt * a.kw + 1);
    const int64_t blocks = (int64_t)a.n_kv * a.groups;
    if (blocks > 16384) return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: too many row groups");
    const size_t smem = (size_t)ws_region_bytes((int)head_dim, a.kw, a.rows_per_group) + kWsMeta;
    void (*kern)(const AttnArgs) = head_dim == 128 ? attn_ws_kernel<128> : attn_ws_kernel<64>;
    static bool set128 = false, set64 = false;
    bool& set = head_dim == 128 ? set128 : set64;
    if (!set) {
      allow_max_dynamic_smem(kern);
      set = true;
    }
    int64_t splits = sms / blocks;
    const int64_t by_len = (kv_bound + 255) / 256;
    if (splits > by_len) splits = by_len;
    // Up to 8 slices of <= 1024 keys merge inside one cluster through DSMEM,
    // with every cluster resident at once; longer contexts use more slices
    // and a merge through global memory.
    if (kv_bound <= 8 * 1024) {
      if (splits > kMaxAttnClusterSplits) splits = kMaxAttnClusterSplits;
      while (splits > 1 && attn_resident_clusters(kern, (int)splits, smem, threads) < blocks) --splits;
    } else {
      int64_t want = (2 * sms) / blocks;
      if (want > by_len) want = by_len;
      if (want > splits) splits = want;
    }
    if (splits * a.kw > kMaxPartials) splits = kMaxPartials / a.kw;
    if (splits > kMmaMaxSplits) splits = kMmaMaxSplits;
    if (splits < 1) splits = 1;
    int64_t split_len = ((kv_bound + splits - 1) / splits + 63) / 64 * 64;
    a.split_len = (int)split_len;
    a.n_splits = (int)((kv_bound + split_len - 1) / split_len);
    a.cluster_merge = (a.n_splits > 1 && a.n_splits <= kMaxAttnClusterSplits && kv_bound <= 8 * 1024) ? 1 : 0;
    if (a.n_splits > 1 && !a.cluster_merge) {
      const int64_t need =
          kCounterBytes + blocks * a.n_splits * a.kw * a.rows_per_group * mma_rec((int)head_dim) * 4;
      if (!workspace || need > workspace_bytes)
        return fail(SSD_ERR_WORKSPACE, "ssd_tree_attention: workspace too small (need %lld)", (long long)need);
      a.counters = static_cast<uint32_t*>(workspace);
      a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
    }
    return launch_kernel("attn_ws_kernel", kern, dim3((unsigned)blocks, (unsigned)a.n_splits), dim3(threads), smem, s,
                         1u, a.cluster_merge ? (unsigned)a.n_splits : 1u, a);
  }
  if (a.G > kAttnQ) return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: GQA group > 32");
  a.rows_per_tile = kAttnQ / a.G;
  a.row_tiles = (int)((T + a.rows_per_tile - 1) / a.rows_per_tile);
  // Key slices: enough CTAs to cover the SMs twice, 64-key aligned.
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
                               kAttnWarps * kAttnQPerWarp * kAttnBlock) * 4 + (2 * kAttnQ + 2) * 4;
  dim3 grid((unsigned)blocks, (unsigned)a.n_splits);
  if (dtype == SSD_F32) {
    static bool set = false;
    if (!set) {
      allow_max_dynamic_smem(attn_simt_kernel<float>);
      set = true;
    }
    return launch_kernel("attn_simt_kernel", attn_simt_kernel<float>, grid, dim3(256), smem, s, 1u, 1u, a);
  } else if (dtype == SSD_BF16) {
    static bool set = false;
    if (!set) {
      allow_max_dynamic_smem(attn_simt_kernel<bf16>);
      set = true;
    }
    return launch_kernel("attn_simt_kernel", attn_simt_kernel<bf16>, grid, dim3(256), smem, s, 1u, 1u, a);
  }
  return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: dtype %d", dtype);
}
