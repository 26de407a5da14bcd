// Tree attention over the shared KV cache (split-KV "FlashDecoding" layout).
//
// Row t of the forward attends cache slots [0, prefix_len[t]) and every
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
  const int32_t* spec_base;
  const uint64_t* mask;
  int mask_words;
  int kv_bound, split_len, n_splits, rows_per_tile, row_tiles;
  int groups, rows_per_group;  // tensor-core kernel: query rows (token x GQA head) per CTA
  int cluster_merge;           // key slices of a row group form a cluster and merge through DSMEM
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
  pdl_wait();
  pdl_trigger();
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

// ------------------------------------------------------ tensor-core kernel
// bf16, head_dim 64 or 128. A CTA = one KV head x one group of up to 128
// query rows (row q = token * G + GQA head, 16 rows per warp) x one key
// slice. K/V blocks of 64 keys are staged by cp.async (double buffered, 16-B
// chunks XOR-swizzled by row so ldmatrix is conflict-free); S = Q K^T and
// O += P V run on mma.sync m16n8k16 with fp32 accumulators; the online
// softmax runs on the accumulator registers in the log2 domain.
constexpr int kMmaWarps = 8;
constexpr int kMmaMaxRows = kMmaWarps * 16;
constexpr int kMmaMaxTok = kMmaMaxRows + 1;
constexpr int kMmaMaxSplits = 32;
constexpr int kMaxAttnClusterSplits = 8;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
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

// Partial record of one query row of one key slice: {m, l, pad, pad, o[hd]}.
__host__ __device__ constexpr int mma_rec(int hd) { return hd + 4; }
// Shared memory before the per-token metadata: the double-buffered K/V
// stages, reused after the key loop for the partial rows (cluster merge).
constexpr int kStages = 4;  // K/V blocks in flight per CTA (memory-level parallelism)
__host__ __device__ constexpr int mma_region(int hd) {
  return (kStages * 2 * 64 * hd * 2) > (kMmaMaxRows * mma_rec(hd) * 4) ? (kStages * 2 * 64 * hd * 2)
                                                                        : (kMmaMaxRows * mma_rec(hd) * 4);
}
// Q rows of the group, bf16, 16-byte chunks XOR-swizzled by row.
__host__ __device__ constexpr int mma_qbytes(int hd) { return kMmaMaxRows * hd * 2; }
constexpr int kMmaMeta = (kMmaMaxTok + 1) * 4 + kMmaMaxTok * 4 * 8 + 16;

template <int HD>
__global__ void __launch_bounds__(256, 1) attn_mma_kernel(const AttnArgs a) {
  constexpr int CH = HD / 8;   // 16-byte chunks per K/V row
  constexpr int KS = HD / 16;  // k-steps over head_dim (QK^T)
  constexpr int NTD = HD / 8;  // n-tiles over head_dim (PV)
  constexpr int KB = 64;       // keys per block
  extern __shared__ __align__(128) uint8_t attn_smem[];
  uint8_t* kv = attn_smem;  // [kStages][K|V][64][HD] bf16, swizzled
  uint8_t* qs = attn_smem + mma_region(HD);  // [kMmaMaxRows][HD] bf16, swizzled
  int* s_plen = reinterpret_cast<int*>(qs + mma_qbytes(HD));
  uint64_t* s_mask = reinterpret_cast<uint64_t*>(s_plen + kMmaMaxTok + 1);  // [tok][mask_words]
  int* s_misc = reinterpret_cast<int*>(s_mask + kMmaMaxTok * 4);           // need_end, min_plen, last

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = blockIdx.x;
  const int h = blk / a.groups, gr = blk % a.groups;
  const int split = blockIdx.y;
  const int M = a.T * a.G;
  const int q0 = gr * a.rows_per_group;
  const int Mg = min(a.rows_per_group, M - q0);
  const int t_first = q0 / a.G;
  const int ntok = (q0 + Mg - 1) / a.G - t_first + 1;
  pdl_wait();
  pdl_trigger();
  const int sb = a.spec_base ? a.spec_base[0] : 0;
  const int mw = a.mask ? a.mask_words : 0;

  if (threadIdx.x == 0) {
    s_misc[0] = 0;
    s_misc[1] = INT32_MAX;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < ntok; i += blockDim.x) {
    const int t = t_first + i;
    const int pl = a.prefix_len[t];
    s_plen[i] = pl;
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
  const int min_plen = s_misc[1];
  const int k_lo = split * a.split_len;
  const int k_hi = min(k_lo + a.split_len, need_end);
  const int nblocks = k_hi > k_lo ? (k_hi - k_lo + KB - 1) / KB : 0;

  // Q fragments of this warp's 16 rows (A operand, row-major 16 x 16 per k-step).
  const bool active = warp * 16 < Mg;
  const int g = lane >> 2, tq = lane & 3;
  const int rl0 = warp * 16 + g, rl1 = rl0 + 8;  // rows within the group
  const bool ok0 = rl0 < Mg, ok1 = rl1 < Mg;
  const int qr0 = q0 + rl0, qr1 = q0 + rl1;
  const int tok0 = ok0 ? qr0 / a.G - t_first : 0, tok1 = ok1 ? qr1 / a.G - t_first : 0;
  // Stage the group's Q rows (A operand) in shared memory; rows past Mg are 0.
  const bf16* qb = static_cast<const bf16*>(a.q);
  for (int idx = threadIdx.x; idx < a.rows_per_group * CH; idx += blockDim.x) {
    const int r = idx / CH, c = idx % CH;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < Mg) {
      const int qr = q0 + r;
      v = *reinterpret_cast<const uint4*>(qb + (int64_t)(qr / a.G) * a.ldq + (int64_t)(h * a.G + qr % a.G) * HD +
                                          c * 8);
    }
    *reinterpret_cast<uint4*>(qs + r * HD * 2 + ((c ^ (r & 7)) << 4)) = v;
  }
  const uint32_t qs_s = smem_u32(qs);
  const int pl0 = ok0 ? s_plen[tok0] : 0, pl1 = ok1 ? s_plen[tok1] : 0;

  float o[NTD][4];
#pragma unroll
  for (int i = 0; i < NTD; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sc = a.scale * 1.4426950408889634f;  // softmax in base 2

  const bf16* kbase = static_cast<const bf16*>(a.kc) + (int64_t)h * a.head_stride;
  const bf16* vbase = static_cast<const bf16*>(a.vc) + (int64_t)h * a.head_stride;
  const uint32_t kv_s = smem_u32(kv);
  auto stage_k = [&](int st) { return kv_s + st * 2 * KB * HD * 2; };
  auto stage_v = [&](int st) { return kv_s + st * 2 * KB * HD * 2 + KB * HD * 2; };
  // kStages-deep ring: every iteration commits exactly one (possibly empty)
  // cp.async group, so waiting for all but the newest kStages-1 groups means
  // block b has landed.
  auto load_block = [&](int b) {
    if (b < nblocks) {
      const int st = b % kStages;
      const int kb = k_lo + b * KB;
      for (int idx = threadIdx.x; idx < KB * CH; idx += blockDim.x) {
        const int key = idx / CH, c = idx % CH;
        const int slot = kb + key;
        const bool valid = slot < k_hi;
        const int64_t off = (int64_t)(valid ? slot : 0) * HD + c * 8;
        const uint32_t dst = key * HD * 2 + ((c ^ (key & 7)) << 4);
        cp_async16(stage_k(st) + dst, kbase + off, valid);
        cp_async16(stage_v(st) + dst, vbase + off, valid);
      }
    }
    cp_async_commit();
  };

#pragma unroll
  for (int b = 0; b < kStages - 1; ++b) load_block(b);
  for (int b = 0; b < nblocks; ++b) {
    load_block(b + kStages - 1);
    cp_async_wait<kStages - 1>();
    __syncthreads();
    if (active) {
      const int st = b % kStages;
      const int kb = k_lo + b * KB;
      float s[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
      const int mi = lane >> 3, ri = lane & 7;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t qf[4];  // A fragment: rows warp*16 + (lane & 15), k-chunk 2*ks + (lane >> 4)
        {
          const int qrow = warp * 16 + (lane & 15);
          const int qc = 2 * ks + (lane >> 4);
          ldsm_x4(qs_s + qrow * HD * 2 + ((qc ^ (qrow & 7)) << 4), qf[0], qf[1], qf[2], qf[3]);
        }
#pragma unroll
        for (int ntp = 0; ntp < 4; ++ntp) {
          const int key = (2 * ntp + (mi >> 1)) * 8 + ri;
          const int c = 2 * ks + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(stage_k(st) + key * HD * 2 + ((c ^ (key & 7)) << 4), b0, b1, b2, b3);
          mma_16816(s[2 * ntp], qf, b0, b1);
          mma_16816(s[2 * ntp + 1], qf, b2, b3);
        }
      }
      // scale + mask: rows rl0 (s[.][0..1]) and rl1 (s[.][2..3])
      const bool full = (kb + KB <= min_plen) && (kb + KB <= k_hi);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = s[nt][e] * sc;
          if (!full) {
            const int slot = kb + nt * 8 + 2 * tq + (e & 1);
            const bool r1 = e >= 2;
            bool ok = slot < k_hi && (r1 ? ok1 : ok0);
            if (ok) {
              const int pl = r1 ? pl1 : pl0;
              if (slot >= pl) {
                const int bit = slot - sb;
                ok = false;
                if (mw && bit >= 0 && bit < mw * 64)
                  ok = (s_mask[(r1 ? tok1 : tok0) * 4 + (bit >> 6)] >> (bit & 63)) & 1ull;
              }
            }
            if (!ok) v = -INFINITY;
          }
          s[nt][e] = v;
        }
      }
      // online softmax (each row is shared by the 4 lanes of a quad)
      float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        bm0 = fmaxf(bm0, fmaxf(s[nt][0], s[nt][1]));
        bm1 = fmaxf(bm1, fmaxf(s[nt][2], s[nt][3]));
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
        s[nt][0] = (s[nt][0] == -INFINITY) ? 0.f : exp2f(s[nt][0] - mn0);
        s[nt][1] = (s[nt][1] == -INFINITY) ? 0.f : exp2f(s[nt][1] - mn0);
        s[nt][2] = (s[nt][2] == -INFINITY) ? 0.f : exp2f(s[nt][2] - mn1);
        s[nt][3] = (s[nt][3] == -INFINITY) ? 0.f : exp2f(s[nt][3] - mn1);
        ps0 += s[nt][0] + s[nt][1];
        ps1 += s[nt][2] + s[nt][3];
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
        pf[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
        pf[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
        pf[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        pf[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int dtp = 0; dtp < NTD / 2; ++dtp) {
          const int key = 16 * kk + (mi & 1) * 8 + ri;
          const int c = 2 * dtp + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(stage_v(st) + key * HD * 2 + ((c ^ (key & 7)) << 4), b0, b1, b2, b3);
          mma_16816(o[2 * dtp], pf, b0, b1);
          mma_16816(o[2 * dtp + 1], pf, b2, b3);
        }
      }
    }
    __syncthreads();  // stage b % kStages is refilled by the next iteration
  }
  cp_async_wait<0>();  // (only empty groups remain) the stages may now be reused

  // row sums across the quad
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  bf16* outp = static_cast<bf16*>(a.out);
  if (a.n_splits == 1) {
    if (active) {
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
  if (a.cluster_merge) {
    // The key slices of this (head, row group) form one cluster: each keeps
    // its partial rows in its own shared memory (the K/V stages are idle),
    // then CTA `split` merges rows split, split + n_splits, ... from every
    // peer in slice order and writes them out.
    float* sp = reinterpret_cast<float*>(attn_smem);
    if (active) {
      if (tq == 0) {
        if (ok0) {
          sp[rl0 * rec] = m0;
          sp[rl0 * rec + 1] = l0;
        }
        if (ok1) {
          sp[rl1 * rec] = m1;
          sp[rl1 * rec + 1] = l1;
        }
      }
#pragma unroll
      for (int dt = 0; dt < NTD; ++dt) {
        const int d = 4 + dt * 8 + 2 * tq;
        if (ok0) *reinterpret_cast<float2*>(sp + rl0 * rec + d) = make_float2(o[dt][0], o[dt][1]);
        if (ok1) *reinterpret_cast<float2*>(sp + rl1 * rec + d) = make_float2(o[dt][2], o[dt][3]);
      }
    }
    cluster_sync_all();
    constexpr int DPL = HD / 32;
    const uint32_t mine = smem_u32(sp);
    const uint32_t peer = lane < a.n_splits ? dsmem_map(mine, static_cast<uint32_t>(lane)) : 0u;
    for (int r = split + warp * a.n_splits; r < Mg; r += kMmaWarps * a.n_splits) {
      const int qr = q0 + r;
      float ms = -INFINITY, ls = 0.f;
      if (lane < a.n_splits) {
        ms = dsmem_ld(peer + (uint32_t)(r * rec) * 4);
        ls = dsmem_ld(peer + (uint32_t)(r * rec + 1) * 4);
      }
      const float M = warp_max(ms);
      const float wgt = (ms == -INFINITY || M == -INFINITY) ? 0.f : exp2f(ms - M);
      const float L = warp_sum(ls * wgt);
      float acc[DPL];
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
      // all peer loads in flight first, then accumulate in slice order
      float v[kMaxAttnClusterSplits][DPL];
#pragma unroll
      for (int s = 0; s < kMaxAttnClusterSplits; ++s) {
        const uint32_t ps = __shfl_sync(0xffffffffu, peer, s < a.n_splits ? s : 0);
#pragma unroll
        for (int i = 0; i < DPL; ++i)
          v[s][i] = s < a.n_splits ? dsmem_ld(ps + (uint32_t)(r * rec + 4 + lane * DPL + i) * 4) : 0.f;
      }
#pragma unroll
      for (int s = 0; s < kMaxAttnClusterSplits; ++s) {
        const float ws = __shfl_sync(0xffffffffu, wgt, s < a.n_splits ? s : 0);
        if (s < a.n_splits) {
#pragma unroll
          for (int i = 0; i < DPL; ++i) acc[i] = fmaf(ws, v[s][i], acc[i]);
        }
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      bf16* op = outp + (int64_t)(qr / a.G) * a.ldo + (int64_t)(h * a.G + qr % a.G) * HD + lane * DPL;
#pragma unroll
      for (int i = 0; i < DPL; ++i) op[i] = f2bf(acc[i] * inv);
    }
    cluster_sync_all();
    return;
  }
  float* part = a.part + ((int64_t)blk * a.n_splits + split) * a.rows_per_group * rec;
  if (active) {
    float* p0 = part + (int64_t)rl0 * rec;
    float* p1 = part + (int64_t)rl1 * rec;
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
  // Merge the slices in order: one warp per row, lanes over head_dim.
  constexpr int DPL = HD / 32;  // dims per lane (2 or 4)
  const float* base = a.part + (int64_t)blk * a.n_splits * a.rows_per_group * rec;
  for (int r = warp; r < Mg; r += kMmaWarps) {
    const int qr = q0 + r;
    float ms = -INFINITY, ls = 0.f;
    if (lane < a.n_splits) {
      const float* p = base + ((int64_t)lane * a.rows_per_group + r) * rec;
      ms = __ldcg(p);
      ls = __ldcg(p + 1);
    }
    const float M = warp_max(ms);
    const float wgt = (ms == -INFINITY || M == -INFINITY) ? 0.f : exp2f(ms - M);
    const float L = warp_sum(ls * wgt);
    float acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
    for (int s = 0; s < a.n_splits; ++s) {
      const float ws = __shfl_sync(0xffffffffu, wgt, s);
      const float* p = base + ((int64_t)s * a.rows_per_group + r) * rec + 4 + lane * DPL;
      if (ws != 0.f) {
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[i] = fmaf(ws, __ldcg(p + i), acc[i]);
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    bf16* op = outp + (int64_t)(qr / a.G) * a.ldo + (int64_t)(h * a.G + qr % a.G) * HD + lane * DPL;
#pragma unroll
    for (int i = 0; i < DPL; ++i) op[i] = f2bf(acc[i] * inv);
  }
  if (threadIdx.x == 0) a.counters[kAttnCounterBase + blk] = 0u;
}

// Clusters of `s` CTAs (one row group's key slices) that can be resident at
// once, from the occupancy API; cached per kernel, size and device.
int attn_resident_clusters(void (*kern)(const AttnArgs), int s, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<void*, int, size_t, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(reinterpret_cast<void*>(kern), s, smem, dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, s);
  cfg.blockDim = dim3(256);
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int sms = device_sms();
  if (dtype == SSD_BF16 && (head_dim == 64 || head_dim == 128)) {
    // Tensor-core path: all query rows of a KV head in as few CTAs as possible.
    const int64_t M = T * a.G;
    a.groups = (int)((M + kMmaMaxRows - 1) / kMmaMaxRows);
    a.rows_per_group = (int)(((M + a.groups - 1) / a.groups + 15) / 16 * 16);
    const int64_t blocks = (int64_t)a.n_kv * a.groups;
    if (blocks > 16384) return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: too many row groups");
    const size_t smem = (size_t)mma_region((int)head_dim) + mma_qbytes((int)head_dim) + kMmaMeta;
    void (*kern)(const AttnArgs) = head_dim == 128 ? attn_mma_kernel<128> : attn_mma_kernel<64>;
    static bool set128 = false, set64 = false;
    bool& set = head_dim == 128 ? set128 : set64;
    if (!set) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
      set = true;
    }
    int64_t splits = (2 * sms) / blocks;
    const int64_t by_len = (kv_bound + 255) / 256;
    if (splits > by_len) splits = by_len;
    // Up to 8 slices of <= 1024 keys merge inside one cluster through DSMEM,
    // with every cluster resident at once; longer contexts use more slices
    // and a merge through global memory.
    if (kv_bound <= 8 * 1024) {
      if (splits > kMaxAttnClusterSplits) splits = kMaxAttnClusterSplits;
      while (splits > 1 && attn_resident_clusters(kern, (int)splits, smem) < blocks) --splits;
    }
    if (splits > kMmaMaxSplits) splits = kMmaMaxSplits;
    if (splits < 1) splits = 1;
    int64_t split_len = ((kv_bound + splits - 1) / splits + 63) / 64 * 64;
    a.split_len = (int)split_len;
    a.n_splits = (int)((kv_bound + split_len - 1) / split_len);
    a.cluster_merge = (a.n_splits > 1 && a.n_splits <= kMaxAttnClusterSplits) ? 1 : 0;
    if (a.n_splits > 1 && !a.cluster_merge) {
      const int64_t need = kCounterBytes + blocks * a.n_splits * a.rows_per_group * mma_rec((int)head_dim) * 4;
      if (!workspace || need > workspace_bytes)
        return fail(SSD_ERR_WORKSPACE, "ssd_tree_attention: workspace too small (need %lld)", (long long)need);
      a.counters = static_cast<uint32_t*>(workspace);
      a.part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
    }
    return launch_kernel("attn_mma_kernel", kern, dim3((unsigned)blocks, (unsigned)a.n_splits), dim3(256), smem, s,
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
                               kAttnWarps * kAttnQPerWarp * kAttnBlock) * 4 + (kAttnQ + 2) * 4;
  dim3 grid((unsigned)blocks, (unsigned)a.n_splits);
  if (dtype == SSD_F32) {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(attn_simt_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
      set = true;
    }
    return launch_kernel("attn_simt_kernel", attn_simt_kernel<float>, grid, dim3(256), smem, s, 1u, 1u, a);
  } else if (dtype == SSD_BF16) {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(attn_simt_kernel<bf16>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
      set = true;
    }
    return launch_kernel("attn_simt_kernel", attn_simt_kernel<bf16>, grid, dim3(256), smem, s, 1u, 1u, a);
  }
  return fail(SSD_ERR_UNSUPPORTED, "ssd_tree_attention: dtype %d", dtype);
}
