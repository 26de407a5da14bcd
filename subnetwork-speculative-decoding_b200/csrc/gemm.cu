// Mainloops and host launcher of the skinny GEMM family (see gemm.cuh).
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "gemm.cuh"
#include "host.cuh"

namespace ssd {

// --------------------------------------------------------------- tcgen05 path
// Warp roles (192 threads): warp 0 issues TMA, warp 1 owns TMEM and issues the
// MMAs (one lane), warps 2..5 drain the accumulator and run the epilogue.
// Pipeline: full[s] = TMA bytes of stage s landed; empty[s] = the MMAs that
// read stage s retired (tcgen05.commit arrives on it).
struct TcMaps {
  CUtensorMap w[3];  // weight segments [rows, K], box {64, 32}
  CUtensorMap x;     // activations [T, K], box {64, BN}
};

constexpr int kTcThreads = 192;
constexpr int kMaxClusterSplits = 8;  // portable cluster size
constexpr int kABytes = kTileM * kChunkK * 2;  // 16 KB of weights per stage

__host__ __device__ inline int tc_stage_bytes(int BN) { return kABytes + BN * kChunkK * 2; }
__host__ __device__ inline int tc_region_bytes(int BN, int stages) {
  const int ring = stages * tc_stage_bytes(BN);
  const int epi = BN * kTileM * 4;
  return ring > epi ? ring : epi;
}
__host__ __device__ inline int tc_smem_bytes(int BN, int stages) {
  return 1024 /*alignment slack*/ + tc_region_bytes(BN, stages) + 256 /*barriers, flags*/;
}
__host__ __device__ inline uint32_t tc_tmem_cols(int BN) {
  return BN <= 32 ? 32u : (BN <= 64 ? 64u : (BN <= 128 ? 128u : 256u));
}

__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ TcMaps maps, const GemmShape g, const EpiArgs e) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stage_bytes = tc_stage_bytes(g.BN);
  uint8_t* bar_base = smem + tc_region_bytes(g.BN, g.stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_base);
  uint64_t* empty = full + g.stages;
  uint64_t* accum = empty + g.stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  int* flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_flag = flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bm = g.n_major ? blockIdx.y : blockIdx.x;
  const int tile_m = bm / g.splits, split = bm % g.splits;
  const int tile_n = g.n_major ? blockIdx.x : blockIdx.y;
  const int kc0 = (int)((int64_t)split * g.kchunks / g.splits);
  const int kc1 = (int)((int64_t)(split + 1) * g.kchunks / g.splits);
  const int nk = kc1 - kc0;
  const uint32_t ncols_alloc = tc_tmem_cols(g.BN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < g.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, ncols_alloc);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < g.n_seg; ++i) tma_prefetch_desc(&maps.w[i]);
      tma_prefetch_desc(&maps.x);
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const uint32_t tx = kABytes + g.BN * kChunkK * 2;
      // A tile = kTileM / a_box weight boxes (one 128-row box when every
      // segment starts on a tile boundary, 64 + 64 rows for gate/up pairs,
      // else four 32-row boxes); the 128-byte swizzle repeats every 8 rows,
      // so stacked boxes give the same layout as one.
      const int nA = kTileM / g.a_box;
      auto load_a = [&](int i) {
        uint8_t* a = smem + (i % g.stages) * stage_bytes;
        const int kx = (kc0 + i) * kChunkK;
        for (int grp = 0; grp < nA; ++grp) {
          int seg, row;
          if (g.layout == SSD_SEG_PAIRS) {
            if (g.a_box == 64) {
              seg = grp;
              row = tile_m * 64;
            } else {
              seg = grp >> 1;
              row = tile_m * 64 + (grp & 1) * 32;
            }
          } else {
            const int n = tile_m * kTileM + grp * g.a_box;
            seg = 0;
            for (int q = 1; q < g.n_seg; ++q)
              if (n >= g.seg_start[q]) seg = q;
            row = n - g.seg_start[seg];  // rows past the segment end are zero-filled by TMA
          }
          tma_load_2d(a + grp * g.a_box * 128, &maps.w[seg], &full[i % g.stages], kx, row, pol_w);
        }
      };
      auto load_b = [&](int i) {
        uint8_t* b = smem + (i % g.stages) * stage_bytes + kABytes;
        tma_load_2d(b, &maps.x, &full[i % g.stages], (kc0 + i) * kChunkK, tile_n * g.BN, pol_x);
      };
      // Weights are never written by any kernel: stream the first stages
      // while the predecessor kernel is still finishing (PDL).
      const int pre = nk < g.stages ? nk : g.stages;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], tx);
        load_a(i);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) load_b(i);
      int issued = pre;
      for (int i = pre; i < nk; ++i) {
        const int s = i % g.stages;
        if (!mbar_wait(&empty[s], ((i / g.stages) - 1) & 1)) {
          report_error(g.status, kErrWaitTimeout);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        mbar_arrive_expect_tx(&full[s], tx);
        load_a(i);
        load_b(i);
        ++issued;
      }
      pdl_trigger();
      // On abort, wait (bounded) for the copies already in flight to land so
      // no TMA write targets shared memory after the CTA exits.
      if (*abort_flag) {
        for (int i = (issued > g.stages ? issued - g.stages : 0); i < issued; ++i)
          (void)mbar_wait(&full[i % g.stages], (i / g.stages) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kTileM, g.BN);
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int s = i % g.stages;
        if (!mbar_wait(&full[s], (i / g.stages) & 1)) {
          report_error(g.status, kErrWaitTimeout);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a = smem_u32(smem + s * stage_bytes);
        const uint32_t b = a + kABytes;
#pragma unroll
        for (int kk = 0; kk < kChunkK / 16; ++kk)
          umma_bf16(tmem, sdesc_k_sw128(a + kk * 32), sdesc_k_sw128(b + kk * 32), idesc, (i | kk) != 0 ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      if (!ok) *abort_flag = 1;
      // Arrives once every MMA above has retired (also on abort, so the
      // epilogue never waits on MMAs still in flight). Waiting here too keeps
      // TMEM allocated until the tensor core is done with it.
      umma_commit(accum);
      if (!mbar_wait(accum, 0)) report_error(g.status, kErrWaitTimeout);
    }
  }
  // Epilogue warps 2..5 drain TMEM into this CTA's partial tile (the idle
  // ring). A warp may only touch TMEM lanes 32*(warp%4)..+31.
  const bool epi = warp >= 2;
  const int q = warp & 3;
  const int r = q * 32 + lane;
  float* stage = reinterpret_cast<float*>(smem);
  const int ncols = min(g.BN, g.T - tile_n * g.BN);
  bool ok = true;
  const float* s_scale = epi_scale_smem();
  if (epi) {
    pdl_wait();  // the epilogue writes buffers earlier kernels may still read
    // The folded-RMSNorm row scales depend only on earlier kernels' output:
    // compute them while the mainloop runs (published by the barrier below).
    if (e.rn_ssq) epi_row_scales(e, tile_n * g.BN, ncols, g.splits == 1 ? 0 : split, g.splits, r);
    if (!mbar_wait(accum, 0)) {
      report_error(g.status, kErrWaitTimeout);
      *abort_flag = 1;
    }
    tc_fence_after();
    named_bar_sync(1, 128);  // all four warps past the wait before the ring is reused
    ok = (*abort_flag == 0);  // uniform across the epilogue warps
    if (ok) {
      const bool scale = e.rn_ssq && g.splits == 1;
      for (int c0 = 0; c0 < g.BN; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (c0 + i < ncols)
            stage[(c0 + i) * kTileM + r] = (nk > 0) ? (scale ? v[i] * s_scale[c0 + i] : v[i]) : 0.f;
      }
    }
  }
  if (g.splits == 1) {
    if (epi) {
      named_bar_sync(1, 128);
      if (ok) run_epilogue<bf16>(stage, tile_m, tile_n * g.BN, ncols, g, e, r, 1, 0, 1, true);
    }
  } else {
    // The `splits` CTAs of this tile form one cluster (rank = split). After
    // the barrier every partial tile is complete; CTA `split` then owns token
    // columns split, split + splits, ...: it sums them over all ranks in rank
    // order (deterministic, independent of T) straight from the peers' shared
    // memory and runs the epilogue on them. The second barrier keeps every
    // CTA's shared memory alive until all peers have read it.
    cluster_sync_all();
    if (epi && ok) {
      uint32_t peer[kMaxClusterSplits];
#pragma unroll
      for (int s = 0; s < kMaxClusterSplits; ++s)
        peer[s] = s < g.splits ? dsmem_map(smem_u32(stage), static_cast<uint32_t>(s)) : 0u;
      // Four owned columns per batch: all their peer loads are in flight
      // together (one DSMEM round trip per batch, not per column).
      constexpr int kCols = 4;
      for (int cb = split, j0 = 0; cb < ncols; cb += kCols * g.splits, j0 += kCols) {
        float v[kCols][kMaxClusterSplits];
#pragma unroll
        for (int u = 0; u < kCols; ++u) {
          const int c = cb + u * g.splits;
          const uint32_t off = static_cast<uint32_t>((c * kTileM + r) * 4);
#pragma unroll
          for (int s = 0; s < kMaxClusterSplits; ++s)
            v[u][s] = (s < g.splits && c < ncols) ? dsmem_ld(peer[s] + off) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kCols; ++u) {
          const int c = cb + u * g.splits;
          if (c >= ncols) break;
          float acc = 0.f;
#pragma unroll
          for (int s = 0; s < kMaxClusterSplits; ++s)
            if (s < g.splits) acc += v[u][s];
          stage[c * kTileM + r] = e.rn_ssq ? acc * s_scale[j0 + u] : acc;
        }
      }
      named_bar_sync(1, 128);
      run_epilogue<bf16>(stage, tile_m, tile_n * g.BN, ncols, g, e, r, 1, split, g.splits, true);
    }
    cluster_sync_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols_alloc);
  }
}

// ------------------------------------------------------- tcgen05, stream-K
// Decode-sized GEMMs (T <= 128 token rows, one token tile) as a persistent
// stream-K kernel: the tiles_m x kchunks (weight tile, 64-wide K chunk)
// iterations are cut into gridDim.x equal contiguous ranges, one per CTA
// (two CTAs per SM), so every SM streams the same number of weight bytes
// whatever the tile count: no wave quantisation and no clusters. A range
// crosses tile boundaries; each piece of a tile it covers is a segment. The
// MMA warp accumulates a segment in one of two TMEM buffers while the
// epilogue warps drain the other. A segment covering a whole tile runs the
// epilogue directly. A tile split across P CTAs is finished by all P of
// them: each writes its partial tile (CTA c: slot 2c for its first segment,
// 2c+1 for its last), and after its own segments each sums the P partials
// of its share of the token columns in K order. The sums are deterministic
// and the cut depends only on the weight shape and the grid, so a row's
// result does not depend on how many rows are batched.
__device__ __forceinline__ int sk_cta_of(int64_t it, int64_t W, int G) {
  return (int)(((it + 1) * G - 1) / W);
}
__device__ __forceinline__ int64_t sk_begin(int c, int64_t W, int G) { return (int64_t)c * W / G; }

__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_sk_kernel(const __grid_constant__ TcMaps maps, const GemmShape g, const EpiArgs e) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stage_bytes = tc_stage_bytes(g.BN);
  float* stage = reinterpret_cast<float*>(smem + g.stages * stage_bytes);
  uint8_t* bar_base = smem + g.stages * stage_bytes + g.BN * kTileM * 4;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_base);
  uint64_t* empty = full + g.stages;
  uint64_t* accf = empty + g.stages;  // [2] accumulator buffer b holds a finished segment
  uint64_t* acce = accf + 2;          // [2] accumulator buffer b drained by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  int* flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abort_flag = flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const int64_t W = (int64_t)g.tiles_m * g.kchunks;
  const int64_t it0 = sk_begin(cta, W, G), it1 = sk_begin(cta + 1, W, G);
  const int n = (int)(it1 - it0);
  const uint32_t cols = tc_tmem_cols(g.BN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < g.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // The whole warp produces: lane 0 owns the barriers, lanes 0..nA-1 each
    // issue one A box of a stage and lane nA the B box, so the TMA
    // instructions of one stage issue in parallel.
    const int nA = kTileM / g.a_box;
    if (n > 0) {
      if (lane == 0) {
        for (int i = 0; i < g.n_seg; ++i) tma_prefetch_desc(&maps.w[i]);
        tma_prefetch_desc(&maps.x);
      }
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const uint32_t tx = kABytes + g.BN * kChunkK * 2;
      auto load_a = [&](int i, int j) {
        const int64_t it = it0 + i;
        const int tile = (int)(it / g.kchunks);
        const int kx = (int)(it - (int64_t)tile * g.kchunks) * kChunkK;
        uint8_t* a = smem + (i % g.stages) * stage_bytes + j * g.a_box * 128;
        int seg, row;
        if (g.layout == SSD_SEG_PAIRS) {
          if (g.a_box == 64) {
            seg = j;
            row = tile * 64;
          } else {
            seg = j >> 1;
            row = tile * 64 + (j & 1) * 32;
          }
        } else {
          const int nn = tile * kTileM + j * g.a_box;
          seg = 0;
          for (int q = 1; q < g.n_seg; ++q)
            if (nn >= g.seg_start[q]) seg = q;
          row = nn - g.seg_start[seg];  // rows past the segment end are zero-filled by TMA
        }
        tma_load_2d(a, &maps.w[seg], &full[i % g.stages], kx, row, pol_w);
      };
      auto load_b = [&](int i) {
        const int64_t it = it0 + i;
        const int kc = (int)(it % g.kchunks);
        uint8_t* bb = smem + (i % g.stages) * stage_bytes + kABytes;
        tma_load_2d(bb, &maps.x, &full[i % g.stages], kc * kChunkK, 0, pol_x);
      };
      // Weights are never written by any kernel: stream the first stages
      // while the predecessor kernel is still finishing (PDL).
      const int pre = n < g.stages ? n : g.stages;
      for (int i = 0; i < pre; ++i) {
        if (lane == 0) mbar_arrive_expect_tx(&full[i], tx);
        __syncwarp();
        if (lane < nA) load_a(i, lane);
      }
      pdl_wait();
      if (lane == nA)
        for (int i = 0; i < pre; ++i) load_b(i);
      int issued = pre;
      for (int i = pre; i < n; ++i) {
        const int s = i % g.stages;
        int ok = 1;
        if (lane == 0) ok = mbar_wait(&empty[s], ((i / g.stages) - 1) & 1) && !*abort_flag;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          if (lane == 0) {
            report_error(g.status, kErrWaitTimeout);
            *abort_flag = 1;
          }
          break;
        }
        if (lane == 0) mbar_arrive_expect_tx(&full[s], tx);
        __syncwarp();
        if (lane < nA) load_a(i, lane);
        if (lane == nA) load_b(i);
        ++issued;
      }
      if (lane == 0) {
        pdl_trigger();
        if (*abort_flag) {
          for (int i = (issued > g.stages ? issued - g.stages : 0); i < issued; ++i)
            (void)mbar_wait(&full[i % g.stages], (i / g.stages) & 1);
        }
      }
    } else if (lane == 0) {
      pdl_trigger();
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kTileM, g.BN);
      bool ok = true;
      int seg = 0;
      for (int64_t it = it0; it < it1 && ok; ++seg) {
        const int tile = (int)(it / g.kchunks);
        const int64_t seg_end = min(it1, (int64_t)(tile + 1) * g.kchunks);
        const int b = seg & 1;
        if (seg >= 2 && !mbar_wait(&acce[b], ((seg >> 1) - 1) & 1)) {
          report_error(g.status, kErrWaitTimeout);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + b * cols;
        const int64_t seg_begin = it;
        for (; it < seg_end; ++it) {
          const int i = (int)(it - it0);
          const int s = i % g.stages;
          if (*abort_flag || !mbar_wait(&full[s], (i / g.stages) & 1)) {
            report_error(g.status, kErrWaitTimeout);
            *abort_flag = 1;  // before the commit below, so the epilogue sees it
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * stage_bytes);
          const uint32_t bb = a + kABytes;
#pragma unroll
          for (int kk = 0; kk < kChunkK / 16; ++kk)
            umma_bf16(d, sdesc_k_sw128(a + kk * 32), sdesc_k_sw128(bb + kk * 32), idesc,
                      (it != seg_begin || kk != 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        // Arrives when every MMA issued so far has retired (also on abort, so
        // the epilogue never reads TMEM that is still being written).
        umma_commit(&accf[b]);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // Epilogue warps 2..5; warp w may only touch TMEM lanes 32*(w%4)..+31.
    // A whole tile is finished here at once. A split segment is drained
    // straight into this CTA's partial slot and counted; only after all its
    // segments does the CTA finish its (at most two) split tiles, so no CTA
    // waits while holding back a partial another CTA needs.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int ncols = min(g.BN, g.T);
    uint32_t* arrived = g.counters;
    uint32_t* finished = g.counters + kMaxCounters / 2;
    pdl_wait();  // the epilogue writes buffers earlier kernels may still read
    int split_tile[2] = {-1, -1};
    int n_split = 0;
    bool failed = false;
    int seg = 0;
    for (int64_t it = it0; it < it1; ++seg) {
      const int tile = (int)(it / g.kchunks);
      const int64_t tile_begin = (int64_t)tile * g.kchunks;
      const int64_t seg_end = min(it1, tile_begin + g.kchunks);
      const bool whole = (it == tile_begin) && (seg_end == tile_begin + g.kchunks);
      const int b = seg & 1;
      bool bad = !mbar_wait(&accf[b], (seg >> 1) & 1);
      if (bad) report_error(g.status, kErrWaitTimeout);
      tc_fence_after();
      bad = named_bar_or(1, 128, bad || *abort_flag != 0);  // one decision for all 128 threads
      if (bad) {
        if (r == 0) *abort_flag = 1;
        failed = true;
        break;
      }
      const uint32_t src = tmem + b * cols + (static_cast<uint32_t>(q * 32) << 16);
      if (whole) {
        for (int c0 = 0; c0 < g.BN; c0 += 16) {
          float v[16];
          tmem_ld16(src + c0, v);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (c0 + i < ncols) stage[(c0 + i) * kTileM + r] = v[i];
        }
        tc_fence_before();
        named_bar_sync(1, 128);
        if (r == 0) mbar_arrive(&acce[b]);  // TMEM buffer b may take segment seg + 2
        run_epilogue<bf16>(stage, tile, 0, ncols, g, e, r, 1);
        named_bar_sync(1, 128);  // the stage is reused by the next segment
      } else {
        float* mine = g.partials + (int64_t)(2 * cta + (seg == 0 ? 0 : 1)) * kTileM * g.BN + r;
        for (int c0 = 0; c0 < g.BN; c0 += 16) {
          float v[16];
          tmem_ld16(src + c0, v);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (c0 + i < ncols) __stcg(mine + (c0 + i) * kTileM, v[i]);
        }
        tc_fence_before();
        __threadfence();
        named_bar_sync(1, 128);
        if (r == 0) {
          mbar_arrive(&acce[b]);
          atomicAdd(&arrived[tile], 1u);
        }
        split_tile[n_split++] = tile;
      }
      it = seg_end;
    }
    // Finish the split tiles: participant j of P owns token columns j, j + P,
    // ...; it sums the P partials of those columns in K order and runs the
    // epilogue on them.
    for (int k = 0; k < n_split && !failed; ++k) {
      const int tile = split_tile[k];
      const int64_t tile_begin = (int64_t)tile * g.kchunks;
      const int first = sk_cta_of(tile_begin, W, G);
      const int last = sk_cta_of(tile_begin + g.kchunks - 1, W, G);
      const int P = last - first + 1;
      const int j = cta - first;
      bool ok = true;
      if (r == 0) {
        uint32_t n_in = 0;
        for (uint32_t i = 0; i < kWaitLimit; ++i) {
          n_in = ld_acquire_u32(&arrived[tile]);
          if ((int)n_in >= P) break;
        }
        ok = (int)n_in >= P;
        if (!ok) report_error(g.status, kErrWaitTimeout);
      }
      if (named_bar_or(1, 128, !ok)) {
        failed = true;
        break;
      }
      __threadfence();
      // (column, partial) pairs of this participant, partial index fastest;
      // loads go out 32 at a time and are summed into the stage in K order.
      // Slots: every participant after `first` starts its range inside the
      // tile (its first segment); `first` covers the tile start.
      const int first_slot = 2 * first + (sk_begin(first, W, G) == tile_begin ? 0 : 1);
      const int n_own = (ncols - j + P - 1) / P;
      const int total = n_own * P;
      for (int m0 = 0; m0 < total; m0 += 32) {
        float v[32];
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          const int m = m0 + u;
          v[u] = 0.f;
          if (m < total) {
            const int pi = m % P;
            const int col = j + (m / P) * P;
            const int slot = pi == 0 ? first_slot : 2 * (first + pi);
            v[u] = __ldcg(g.partials + (int64_t)slot * kTileM * g.BN + col * kTileM + r);
          }
        }
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          const int m = m0 + u;
          if (m < total) {
            const int pi = m % P;
            float* dst = stage + (j + (m / P) * P) * kTileM + r;
            *dst = (pi == 0 ? 0.f : *dst) + v[u];
          }
        }
      }
      named_bar_sync(1, 128);
      run_epilogue<bf16>(stage, tile, 0, ncols, g, e, r, 1, j, P);
      named_bar_sync(1, 128);
      if (r == 0) {
        const unsigned t = atomicAdd(&finished[tile], 1u);
        if ((int)t == P - 1) {  // every participant has read the partials: reset for the next launch
          arrived[tile] = 0u;
          finished[tile] = 0u;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * cols);
  }
}

// ------------------------------------------------------- tcgen05, GEMM chain
// Up to kChainMax dependent decode-sized GEMMs of one forward (for example
// o_proj -> gate/up -> down -> the next layer's q/k/v) in one persistent
// launch, every CTA resident. Each link is cut like the stream-K kernel: the
// link's tiles_m x kchunks iterations in G equal contiguous ranges, one per
// CTA; a CTA runs its range of link 0, then its range of link 1, and so on.
// The weight stream never waits on a dependency: when a CTA moves to the
// next link its producer fills the free ring stages with that link's weight
// boxes while the previous link's last tiles are still being reduced, and
// only the activation boxes (the previous link's output) wait until every
// CTA has finished the previous link (done[l] counts CTAs; release stores,
// acquire polls). Split tiles are summed in K order through two partial
// slots per CTA as in the stream-K kernel, so each result depends only on
// the weight shapes and the grid, never on the token count.
constexpr int kChainMax = 6;
constexpr int kChainThreads = 288;  // warps: 0, 8 activation TMA; 1 MMA; 2-5 epilogue; 6, 7 weight TMA
constexpr int kChainTiles = 1024;                // weight tiles per link (counter slots)
constexpr int64_t kChainCounterBase = 16384;     // first workspace counter of the chain block
constexpr int64_t kChainCounters = kChainMax * 2 * kChainTiles + kChainMax + 1;

struct ChainLink {
  TcMaps maps;
  GemmShape g;
  EpiArgs e;
};
struct ChainParams {
  ChainLink link[kChainMax];
  int n;
  int BN, stages;
  // [kChainMax][2][kChainTiles] arrived / finished per tile, then
  // done[kChainMax] (CTAs that finished link l), then the exit count
  uint32_t* counters;
  float* partials;  // [2 G][BN][128] partial slots, shared by the links
  uint32_t* status;
};

// A link of W iterations runs on its first min(G, W) CTAs (every one of
// them then holds at least one iteration, which the split bookkeeping
// needs); the other CTAs have an empty range for it.
__device__ __forceinline__ int chain_ctas(int64_t W, int G) { return W < G ? (int)W : G; }
__device__ __forceinline__ int64_t chain_begin(int c, int64_t W, int Gl) {
  return c >= Gl ? W : sk_begin(c, W, Gl);
}

// Bounded poll until *p >= want (acquire at GPU scope). Every CTA polls the
// same word, so after a few tight polls each one backs off 256 ns between
// polls to keep that word's L2 slice free for other traffic.
__device__ __forceinline__ bool poll_at_least(const uint32_t* p, uint32_t want) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (ld_acquire_u32(p) >= want) return true;
    if (i > 8) __nanosleep(256);
  }
  return false;
}

__global__ void __launch_bounds__(kChainThreads, 1) tc_chain_kernel(const __grid_constant__ ChainParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int BN = P.BN, stages = P.stages;
  const int stage_bytes = tc_stage_bytes(BN);
  float* stage = reinterpret_cast<float*>(smem + stages * stage_bytes);
  uint8_t* bar_base = smem + stages * stage_bytes + BN * kTileM * 4;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(bar_base);  // weight boxes of stage s landed
  uint64_t* full_b = full_a + stages;                          // activation box of stage s landed
  uint64_t* empty = full_b + stages;
  uint64_t* accf = empty + stages;  // [2] accumulator buffer b holds a finished segment
  uint64_t* acce = accf + 2;        // [2] accumulator buffer b drained by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  volatile int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  // Shapes and epilogue arguments of the links, copied out of the parameter
  // space once: indexed by a runtime link number they would otherwise be
  // read through generic loads on every use.
  __shared__ GemmShape s_g[kChainMax];
  __shared__ EpiArgs s_e[kChainMax];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;
  const uint32_t cols = tc_tmem_cols(BN);
  uint32_t* done = P.counters + kChainMax * 2 * kChainTiles;
  uint32_t* exit_count = done + kChainMax;
  if (threadIdx.x < P.n) {
    s_g[threadIdx.x] = P.link[threadIdx.x].g;
    s_e[threadIdx.x] = P.link[threadIdx.x].e;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&full_b[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // One thread issues a TMA box stream at ~40-50 GB/s on B200, under the
  // ~43 GB/s an SM needs for the HBM peak once the activation boxes are
  // added, so the weight boxes of alternate stages come from two threads
  // in two warps (6, 7) and the activation boxes of alternate stages from
  // two more (warps 0, 8); weights and activations complete on separate
  // barriers. Only the activation streams wait for dependencies: the weight
  // streams run ahead into the next link as far as the ring allows.
  if (warp >= 6 || warp == 0) {
    if (lane == 0) {
      const bool wproducer = warp == 6 || warp == 7;
      const int k = wproducer ? warp - 6 : (warp == 0 ? 0 : 1);  // positions pos with pos % 2 == k
      if (wproducer) {
        for (int l = 0; l < P.n; ++l)
          for (int i = 0; i < P.link[l].g.n_seg; ++i) tma_prefetch_desc(&P.link[l].maps.w[i]);
      } else {
        for (int l = 0; l < P.n; ++l) tma_prefetch_desc(&P.link[l].maps.x);
      }
      const uint64_t pol = wproducer ? l2_policy_evict_first() : l2_policy_evict_last();
      const uint32_t b_tx = BN * kChunkK * 2;
      int pos = 0;  // ring positions (stages) of all links so far
      int issued_to = 0;  // positions below this one this thread has issued (or skipped)
      bool ok = true;
      for (int l = 0; l < P.n && ok; ++l) {
        const TcMaps& maps = P.link[l].maps;
        const GemmShape& g = s_g[l];
        const int kchunks = g.kchunks, layout = g.layout, a_box = g.a_box, n_seg = g.n_seg;
        const int seg1 = g.seg_start[1], seg2 = g.seg_start[2];
        const int64_t W = (int64_t)g.tiles_m * kchunks;
        const int Gl = chain_ctas(W, G);
        const int64_t it0 = chain_begin(cta, W, Gl), it1 = chain_begin(cta + 1, W, Gl);
        const int n = (int)(it1 - it0);
        if (n == 0) continue;
        if (!wproducer) {
          // Activations: link 0 reads the predecessor kernel's output, link
          // l > 0 the output of link l - 1 from every CTA.
          pdl_wait();  // returns at once after the first time
          if (l > 0) {
            ok = poll_at_least(&done[l - 1], (uint32_t)G);
            fence_proxy_async_global();
            if (!ok) break;
          }
        }
        for (int j = 0; j < n; ++j, ++pos) {
          if ((pos & 1) != k) continue;
          const int s = pos % stages;
          if ((pos >= stages && !mbar_wait(&empty[s], ((pos / stages) - 1) & 1)) || *abort_flag) {
            ok = false;
            break;
          }
          const int64_t it = it0 + j;
          const int tile = (int)(it / kchunks);
          const int kc = (int)(it - (int64_t)tile * kchunks);
          uint8_t* st = smem + s * stage_bytes;
          if (wproducer) {
            mbar_arrive_expect_tx(&full_a[s], kABytes);
            for (int box = 0; box < kTileM / a_box; ++box) {
              int seg, row;
              if (layout == SSD_SEG_PAIRS) {
                if (a_box == 64) {
                  seg = box;
                  row = tile * 64;
                } else {
                  seg = box >> 1;
                  row = tile * 64 + (box & 1) * 32;
                }
              } else {
                const int nn = tile * kTileM + box * a_box;
                seg = (n_seg > 2 && nn >= seg2) ? 2 : ((n_seg > 1 && nn >= seg1) ? 1 : 0);
                row = nn - (seg == 2 ? seg2 : (seg == 1 ? seg1 : 0));  // rows past the end are zero-filled
              }
              tma_load_2d(st + box * a_box * 128, &maps.w[seg], &full_a[s], kc * kChunkK, row, pol);
            }
          } else {
            mbar_arrive_expect_tx(&full_b[s], b_tx);
            tma_load_2d(st + kABytes, &maps.x, &full_b[s], kc * kChunkK, 0, pol);
          }
          issued_to = pos + 1;
        }
      }
      if (!ok) {
        report_error(P.status, kErrWaitTimeout);
        *abort_flag = 1;
        // every copy this thread issued must land before the CTA exits
        for (int i = (issued_to > stages ? issued_to - stages : 0); i < issued_to; ++i)
          if ((i & 1) == k) (void)mbar_wait(&(wproducer ? full_a : full_b)[i % stages], (i / stages) & 1);
      }
      if (warp == 0) {
        pdl_wait();  // (a CTA without work still triggers only after its wait)
        pdl_trigger();
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kTileM, BN);
      bool ok = true;
      int i = 0, seg = 0;
      for (int l = 0; l < P.n && ok; ++l) {
        const int kchunks = s_g[l].kchunks;
        const int64_t W = (int64_t)s_g[l].tiles_m * kchunks;
        const int Gl = chain_ctas(W, G);
      const int64_t it0 = chain_begin(cta, W, Gl), it1 = chain_begin(cta + 1, W, Gl);
        for (int64_t it = it0; it < it1 && ok; ++seg) {
          const int tile = (int)(it / kchunks);
          const int64_t seg_end = min(it1, (int64_t)(tile + 1) * kchunks);
          const int b = seg & 1;
          if (seg >= 2 && !mbar_wait(&acce[b], ((seg >> 1) - 1) & 1)) {
            report_error(P.status, kErrWaitTimeout);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + b * cols;
          const int64_t seg_begin = it;
          for (; it < seg_end; ++it, ++i) {
            const int s = i % stages;
            if (*abort_flag || !mbar_wait(&full_a[s], (i / stages) & 1) || !mbar_wait(&full_b[s], (i / stages) & 1)) {
              report_error(P.status, kErrWaitTimeout);
              *abort_flag = 1;  // before the commit below, so the epilogue sees it
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a = smem_u32(smem + s * stage_bytes);
            const uint32_t bb = a + kABytes;
#pragma unroll
            for (int kk = 0; kk < kChunkK / 16; ++kk)
              umma_bf16(d, sdesc_k_sw128(a + kk * 32), sdesc_k_sw128(bb + kk * 32), idesc,
                        (it != seg_begin || kk != 0) ? 1u : 0u);
            umma_commit(&empty[s]);
          }
          // Arrives when every MMA issued so far has retired (also on abort).
          umma_commit(&accf[b]);
        }
      }
    }
  } else if (warp >= 2 && warp <= 5) {
    // Epilogue warps 2..5 (TMEM lanes 32*(w%4)..+31): a whole tile runs its
    // epilogue from TMEM; a split segment writes its fp32 partial to this
    // CTA's slot and counts itself into the tile, and the participant that
    // arrives last sums the tile's partials in K order and runs the epilogue
    // (nobody waits for a tile: no polling on the shared counters). Then one
    // count of this CTA into done[l].
    const int q = warp & 3;
    const int r = q * 32 + lane;
    volatile int* s_last = abort_flag + 1;
    pdl_wait();  // the epilogues write buffers earlier kernels may still read
    bool failed = false;
    int seg = 0;
    for (int l = 0; l < P.n && !failed; ++l) {
      const GemmShape& g = s_g[l];
      const EpiArgs& e = s_e[l];
      const int ncols = min(BN, g.T);
      const int64_t W = (int64_t)g.tiles_m * g.kchunks;
      const int Gl = chain_ctas(W, G);
      const int64_t it0 = chain_begin(cta, W, Gl), it1 = chain_begin(cta + 1, W, Gl);
      uint32_t* arrived = P.counters + (int64_t)l * 2 * kChainTiles;
      if (l > 0) {
        // The epilogue reads what link l - 1 wrote (residual rows, norm sums).
        bool ok = true;
        if (r == 0) ok = poll_at_least(&done[l - 1], (uint32_t)G);
        if (named_bar_or(1, 128, !ok)) {
          if (r == 0) {
            report_error(P.status, kErrWaitTimeout);
            *abort_flag = 1;
          }
          failed = true;
          break;
        }
      }
      int lseg = 0;
      for (int64_t it = it0; it < it1; ++seg, ++lseg) {
        const int tile = (int)(it / g.kchunks);
        const int64_t tile_begin = (int64_t)tile * g.kchunks;
        const int64_t seg_end = min(it1, tile_begin + g.kchunks);
        const bool whole = (it == tile_begin) && (seg_end == tile_begin + g.kchunks);
        const int b = seg & 1;
        bool bad = !mbar_wait(&accf[b], (seg >> 1) & 1);
        tc_fence_after();
        bad = named_bar_or(1, 128, bad || *abort_flag != 0);
        if (bad) {
          if (r == 0) {
            report_error(P.status, kErrWaitTimeout);
            *abort_flag = 1;
          }
          failed = true;
          break;
        }
        const uint32_t src = tmem + b * cols + (static_cast<uint32_t>(q * 32) << 16);
        if (whole) {
          for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
            tmem_ld16(src + c0, v);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (c0 + i < ncols) stage[(c0 + i) * kTileM + r] = v[i];
          }
          tc_fence_before();
          named_bar_sync(1, 128);
          if (r == 0) mbar_arrive(&acce[b]);  // TMEM buffer b may take segment seg + 2
          run_epilogue<bf16>(stage, tile, 0, ncols, g, e, r, 1);
          named_bar_sync(1, 128);  // the stage is reused by the next segment
        } else {
          float* mine = P.partials + (int64_t)(2 * cta + (lseg == 0 ? 0 : 1)) * kTileM * BN + r;
          for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
            tmem_ld16(src + c0, v);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (c0 + i < ncols) __stcg(mine + (c0 + i) * kTileM, v[i]);
          }
          tc_fence_before();
          __threadfence();
          named_bar_sync(1, 128);
          const int first = sk_cta_of(tile_begin, W, Gl);
          const int np = sk_cta_of(tile_begin + g.kchunks - 1, W, Gl) - first + 1;
          if (r == 0) {
            mbar_arrive(&acce[b]);
            *s_last = (atomicAdd(&arrived[tile], 1u) == (unsigned)(np - 1)) ? 1 : 0;
          }
          named_bar_sync(1, 128);
          if (*s_last) {
            // Last participant: every partial of the tile is visible. Slots:
            // the first participant's is its first or last segment (its range
            // may start before the tile), every later one's is its first.
            __threadfence();
            const int first_slot = 2 * first + (sk_begin(first, W, Gl) == tile_begin ? 0 : 1);
            constexpr int kC = 8, kP = 8;  // columns x participants per batch of loads
            for (int c0 = 0; c0 < ncols; c0 += kC) {
              float acc[kC];
#pragma unroll
              for (int u = 0; u < kC; ++u) acc[u] = 0.f;
              for (int p0 = 0; p0 < np; p0 += kP) {
                float v[kP][kC];
#pragma unroll
                for (int pi = 0; pi < kP; ++pi) {
                  const int pp = p0 + pi;
                  const int slot = pp == 0 ? first_slot : 2 * (first + pp);
                  const float* base = P.partials + (int64_t)slot * kTileM * BN + r;
#pragma unroll
                  for (int u = 0; u < kC; ++u)
                    v[pi][u] = (pp < np && c0 + u < ncols) ? __ldcg(base + (c0 + u) * kTileM) : 0.f;
                }
#pragma unroll
                for (int pi = 0; pi < kP; ++pi)
#pragma unroll
                  for (int u = 0; u < kC; ++u)
                    if (p0 + pi < np) acc[u] += v[pi][u];  // K order
              }
#pragma unroll
              for (int u = 0; u < kC; ++u)
                if (c0 + u < ncols) stage[(c0 + u) * kTileM + r] = acc[u];
            }
            named_bar_sync(1, 128);
            run_epilogue<bf16>(stage, tile, 0, ncols, g, e, r, 1);
            named_bar_sync(1, 128);
            if (r == 0) arrived[tile] = 0u;  // ready for the next launch
          }
        }
        it = seg_end;
      }
      if (failed) break;
      // This CTA's share of link l is written: publish it (generic stores
      // before later TMA reads of them on other CTAs).
      __threadfence();
      fence_proxy_async_global();
      named_bar_sync(1, 128);
      if (r == 0) atomicAdd(&done[l], 1u);
    }
    if (r == 0) {
      // The last CTA out resets the link counts for the next launch: every
      // CTA has passed all its polls of them by the time it counts here.
      __threadfence();
      const unsigned t = atomicAdd(exit_count, 1u);
      if ((int)t == G - 1 && !failed) {
        for (int l = 0; l < kChainMax; ++l) done[l] = 0u;
        __threadfence();
        *exit_count = 0u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * cols);
  }
}

// ------------------------------------------------------------------ SIMT path
// CUDA-core mainloop for the fp32 parity tier: 256 threads = 8 warps x 16
// feature rows; lanes stride K (coalesced weight rows), 4 tokens per tile.
constexpr int kSimtBN = 4;
constexpr int kSimtKC = 512;

struct SimtSegs {
  const void* p[3];
  int rows[3];
};

template <typename T>
__global__ void __launch_bounds__(256) simt_gemm_kernel(const T* __restrict__ x, int64_t ldx, const SimtSegs segs,
                                                         const GemmShape g, const EpiArgs e) {
  __shared__ float xs[kSimtBN][kSimtKC];
  __shared__ float stage[kSimtBN * kTileM];
  __shared__ int flag;
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile_m = blockIdx.x / g.splits, split = blockIdx.x % g.splits;
  const int tile_n = blockIdx.y;
  const int t0 = tile_n * kSimtBN;
  const int ncols = min(kSimtBN, g.T - t0);
  const int k_begin = (int)((int64_t)split * g.kchunks / g.splits) * kChunkK;
  const int k_end = min(g.K, (int)((int64_t)(split + 1) * g.kchunks / g.splits) * kChunkK);

  const T* wrow[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int rr = warp * 16 + i;
    int seg, row;
    if (g.layout == SSD_SEG_PAIRS) {
      seg = rr >> 6;
      row = tile_m * 64 + (rr & 63);
    } else {
      const int n = tile_m * kTileM + rr;
      seg = 0;
      for (int q = 1; q < g.n_seg; ++q)
        if (n >= g.seg_start[q]) seg = q;
      row = n - g.seg_start[seg];
    }
    wrow[i] = (row < segs.rows[seg]) ? static_cast<const T*>(segs.p[seg]) + (int64_t)row * g.K : nullptr;
  }
  float acc[16][kSimtBN];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int c = 0; c < kSimtBN; ++c) acc[i][c] = 0.f;

  for (int k0 = k_begin; k0 < k_end; k0 += kSimtKC) {
    const int kn = min(kSimtKC, k_end - k0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < kSimtBN * kSimtKC; idx += 256) {
      const int c = idx / kSimtKC, kk = idx % kSimtKC;
      xs[c][kk] = (c < ncols && kk < kn) ? to_f32<T>(x[(int64_t)(t0 + c) * ldx + k0 + kk]) : 0.f;
    }
    __syncthreads();
    for (int kk = lane; kk < kn; kk += 32) {
      float xv[kSimtBN];
#pragma unroll
      for (int c = 0; c < kSimtBN; ++c) xv[c] = xs[c][kk];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float wv = wrow[i] ? to_f32<T>(wrow[i][k0 + kk]) : 0.f;
#pragma unroll
        for (int c = 0; c < kSimtBN; ++c) acc[i][c] = fmaf(wv, xv[c], acc[i][c]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int c = 0; c < kSimtBN; ++c) {
      const float v = warp_sum(acc[i][c]);
      if (lane == 0) stage[c * kTileM + warp * 16 + i] = v;
    }
  __syncthreads();
  if (threadIdx.x < 128) finish_tile<T>(stage, &flag, tile_m, tile_n, split, g, e, threadIdx.x, 1);
}

// ------------------------------------------------------------------- host side
namespace {

struct MapKey {
  const void* p;
  uint64_t inner, outer, stride;
  uint32_t box_outer;
  bool operator==(const MapKey& o) const {
    return p == o.p && inner == o.inner && outer == o.outer && stride == o.stride && box_outer == o.box_outer;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = reinterpret_cast<uintptr_t>(k.p);
    h = h * 0x9E3779B97F4A7C15ull ^ k.inner;
    h = h * 0x9E3779B97F4A7C15ull ^ k.outer;
    h = h * 0x9E3779B97F4A7C15ull ^ k.stride;
    h = h * 0x9E3779B97F4A7C15ull ^ k.box_outer;
    return static_cast<size_t>(h);
  }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// bf16 2-D tensor map, box {64 elements (128 B), box_outer rows}, 128 B swizzle.
int get_map(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_outer,
            CUtensorMap* out) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride_bytes & 15))
    return fail(SSD_ERR_INVALID, "bf16 GEMM operands need 16-byte aligned bases and row strides");
  MapKey key{base, inner, outer, row_stride_bytes, box_outer};
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return SSD_OK;
    }
  }
  TensorMapEncodeFn encode = tensor_map_encoder();
  if (!encode) return fail(SSD_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {64u, box_outer};
  cuuint32_t estr[2] = {1u, 1u};
  CUtensorMap m;
  CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SSD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  std::lock_guard<std::mutex> lk(g_map_mu);
  if (g_maps.size() > 8192) g_maps.clear();
  g_maps.emplace(key, m);
  *out = m;
  return SSD_OK;
}

int round_bn(int64_t T) {
  if (T > 256) return 128;
  const int bn = (int)((T + 15) / 16) * 16;
  return bn < 16 ? 16 : bn;
}

// K-split count from the weight shape only (never from T), so a token's
// result is bit-identical whatever batch it is computed in.
int choose_splits(int tiles_m, int kchunks, int cta_slots) {
  if (tiles_m * 2 >= cta_slots) return 1;
  int s = cta_slots / tiles_m;
  const int max_s = kchunks / 4;
  if (s > max_s) s = max_s;
  return s < 1 ? 1 : s;
}

void set_tc_attributes() {
  static bool done = false;
  if (!done) {
    allow_max_dynamic_smem(tc_gemm_kernel);
    done = true;
  }
}

// Stream-K variant, opt-in with SSD_GEMM_SK=1 (CTAs per SM: SSD_SK_CTAS=1|2,
// default 2). Its main loop streams at the HBM peak, but finishing the split
// tiles through L2 (write, fence, count, re-read) costs ~10 us per launch on
// B200, more than the cluster kernel's DSMEM reduction, so it is not the
// default.
int sk_ctas_per_sm() {
  static const int v = [] {
    const char* s = getenv("SSD_SK_CTAS");
    return (s && atoi(s) == 1) ? 1 : 2;
  }();
  return v;
}
bool sk_enabled() {
  static const bool v = [] {
    const char* s = getenv("SSD_GEMM_SK");
    return s && s[0] == '1';
  }();
  return v;
}
constexpr int kSkBarBytes = 512;
int sk_stages(int BN) {
  const int budget = (sk_ctas_per_sm() == 2 ? 113 * 1024 : 232448) - 1024;  // static epilogue scales
  const int avail = budget - 1024 - kSkBarBytes - BN * kTileM * 4;
  const int st = avail / tc_stage_bytes(BN);
  return st > 16 ? 16 : (st < 2 ? 2 : st);
}
size_t sk_smem_bytes(int BN, int stages) {
  return 1024 + (size_t)stages * tc_stage_bytes(BN) + (size_t)BN * kTileM * 4 + kSkBarBytes;
}

// Cluster split-K kernel: CTAs resident per SM, chosen from the weight shape
// only (so the split, and with it every row's rounding, never depends on T).
// One CTA's tiled-TMA stream tops out near 34 GB/s, so an SM's bandwidth grows
// with the CTAs it holds, while each CTA's ring shrinks to fit; measured on
// the 8B shapes: two per SM suit split GEMMs that already reach 8-way splits
// and single-wave unsplit ones, more per SM pays when it buys a deeper split
// (q/k/v: 4 -> 8) or fewer waves (lm_head: 1002 tiles).
int tc_ctas_per_sm(int tiles_m, int kchunks, bool head, int sms);
int tc_stages(int BN, int per_sm) {
  // per CTA: 1 KB reserved by the system, 1 KB of static shared memory (the
  // epilogue's row-norm scales), alignment slack and barriers
  const int budget = (233472 - per_sm * 2048) / per_sm - 1024 - 256;
  const int stages = budget / tc_stage_bytes(BN);
  return stages > 8 ? 8 : (stages < 2 ? 2 : stages);
}

// Split count for a tile grid of `tiles_m` weight tiles: fill ~2 CTAs per SM,
// at most one portable cluster per tile. Depends on the weight shape only, so
// every decode-sized T uses the same split (rows are batch-invariant).
// (Requiring all clusters to be co-resident per cudaOccupancyMaxActiveClusters
// measured slower: the query is conservative and the smaller splits it
// leaves underfill HBM.)
int choose_cluster_splits(int tiles_m, int kchunks, int cta_slots) {
  int s = choose_splits(tiles_m, kchunks, cta_slots);
  if (s > kMaxClusterSplits) s = kMaxClusterSplits;
  // Power-of-two clusters pack the GPCs without leftover slots (6-CTA
  // clusters measured 2.6x slower per byte than 8-CTA ones).
  int p = 1;
  while (p * 2 <= s) p *= 2;
  return p;
}

int tc_ctas_per_sm(int tiles_m, int kchunks, bool head, int sms) {
  if (head || tiles_m * 2 >= 2 * sms) return tiles_m > 2 * sms ? 4 : 2;
  int best = 2, best_s = choose_cluster_splits(tiles_m, kchunks, 2 * sms);
  for (int per = 3; per <= 4; ++per) {
    const int s = choose_cluster_splits(tiles_m, kchunks, per * sms);
    if (s > best_s) {
      best = per;
      best_s = s;
    }
  }
  return best;
}

}  // namespace

// Weight boxes of the cluster kernel: whole-tile boxes unless SSD_GEMM_BOX=32.
static bool big_boxes() {
  static const bool v = [] {
    const char* e = getenv("SSD_GEMM_BOX");
    return !(e && e[0] == '3');
  }();
  return v;
}

int tma_map_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_outer,
                    CUtensorMap* out) {
  return get_map(base, inner, outer, row_stride_bytes, box_outer, out);
}

// Token tiling and K split of a GEMM: BN, tiles_n, splits, stages, plus the
// stream-K grid when that variant is enabled. Shared by launch_gemm and
// gemm_workspace_need so a size query always matches the launch.
struct SplitPlan {
  int BN = 0, tiles_n = 0, splits = 1, stages = 0;
  bool sk = false;
  int64_t sk_ctas = 0;
};

static SplitPlan plan_splits(int64_t T, int tiles_m, int kchunks, bool head, int dtype, int sms) {
  SplitPlan p;
  if (dtype == SSD_BF16) {
    p.BN = round_bn(T);
    p.tiles_n = (int)((T + p.BN - 1) / p.BN);
    // Several token tiles (prefill, T > 256): two or three CTAs per SM. With
    // three (two stages each) one CTA's epilogue runs under the other two's
    // main loops: the 8B gate/up pair over 2048 tokens takes 564 us against
    // 734 us at two per SM (1363 us at one), i.e. a CTA runs ~15 % longer
    // beside two others than beside one. Whichever needs fewer CTA-times in
    // whole waves wins (a small grid's last wave would run nearly empty).
    int per_sm;
    if (p.tiles_n > 1) {
      const int64_t ctas = (int64_t)tiles_m * p.tiles_n;
      const int64_t w2 = (ctas + 2 * sms - 1) / (2 * sms), w3 = (ctas + 3 * sms - 1) / (3 * sms);
      per_sm = w3 * 115 < w2 * 100 ? 3 : 2;
    } else {
      per_sm = tc_ctas_per_sm(tiles_m, kchunks, head, sms);
    }
    p.splits = (p.tiles_n == 1 && !head) ? choose_cluster_splits(tiles_m, kchunks, per_sm * sms) : 1;
    p.stages = tc_stages(p.BN, per_sm);
    p.sk = p.tiles_n == 1 && p.BN <= 128 && sk_enabled();
    if (p.sk) {
      const int64_t W = (int64_t)tiles_m * kchunks;
      p.sk_ctas = (int64_t)sms * sk_ctas_per_sm();
      if (p.sk_ctas > W) p.sk_ctas = W;
    }
  } else {
    p.BN = kSimtBN;
    p.tiles_n = (int)((T + kSimtBN - 1) / kSimtBN);
    // Same split for every decode-sized T (<= kSimtInvariantRows), so rows are
    // bit-identical whatever the batch; larger (prefill) batches do not split.
    p.splits = (T <= kSimtInvariantRows && !head) ? choose_splits(tiles_m, kchunks, 4 * sms) : 1;
  }
  return p;
}

static int64_t plan_workspace_bytes(const SplitPlan& p, int tiles_m) {
  if (p.sk) return kCounterBytes + 2 * p.sk_ctas * kTileM * p.BN * 4;
  if (p.splits <= 1) return 0;
  return kCounterBytes + (int64_t)tiles_m * p.tiles_n * p.splits * p.BN * kTileM * 4;
}

int64_t gemm_workspace_need(int64_t T, int64_t K, int n_seg, const int64_t* rows, int layout, bool head, int dtype) {
  if (T <= 0 || K <= 0 || n_seg < 1 || n_seg > 3) return -1;
  int64_t N = 0;
  for (int i = 0; i < n_seg; ++i) N += rows[i];
  const int tiles_m = (int)(layout == SSD_SEG_PAIRS ? (rows[0] + 63) / 64 : (N + kTileM - 1) / kTileM);
  const int kchunks = (int)((K + kChunkK - 1) / kChunkK);
  return plan_workspace_bytes(plan_splits(T, tiles_m, kchunks, head, dtype, device_sms()), tiles_m);
}

int launch_gemm(const void* x, int64_t ldx, int64_t T, int64_t K, int n_seg, const void* const* w,
                const int64_t* rows, int layout, const EpiArgs& e, int dtype, void* workspace,
                int64_t workspace_bytes, uint32_t* status, cudaStream_t stream, int64_t partial_offset_bytes) {
  if (T <= 0 || K <= 0 || n_seg < 1 || n_seg > 3 || !x) return fail(SSD_ERR_INVALID, "bad GEMM arguments");
  for (int i = 0; i < n_seg; ++i)
    if (!w[i] || rows[i] <= 0) return fail(SSD_ERR_INVALID, "GEMM weight segment %d is empty", i);
  if (T > (1 << 20) || K > (1 << 20)) return fail(SSD_ERR_UNSUPPORTED, "GEMM dimension too large");
  GemmShape g{};
  g.T = (int)T;
  g.K = (int)K;
  g.n_seg = n_seg;
  g.layout = layout;
  int64_t N = 0;
  for (int i = 0; i < n_seg; ++i) {
    g.seg_start[i] = (int)N;
    N += rows[i];
  }
  g.seg_start[n_seg] = (int)N;
  if (layout == SSD_SEG_PAIRS) {
    if (n_seg != 2 || rows[0] != rows[1]) return fail(SSD_ERR_INVALID, "PAIRS layout needs two equal segments");
    g.N = (int)(rows[0] * 2);
    g.tiles_m = (int)((rows[0] + 63) / 64);
  } else {
    for (int i = 0; i + 1 < n_seg; ++i)
      if (rows[i] % 32) return fail(SSD_ERR_UNSUPPORTED, "CONCAT segments must be multiples of 32 rows");
    g.N = (int)N;
    g.tiles_m = (int)((N + kTileM - 1) / kTileM);
  }
  g.kchunks = (int)((K + kChunkK - 1) / kChunkK);
  g.status = status;
  const int sms = device_sms();
  const bool head = (e.kind == EPI_ARGMAX || e.kind == EPI_TOPK);

  if (dtype != SSD_BF16 && dtype != SSD_F32) return fail(SSD_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (dtype == SSD_BF16 && K % 8) return fail(SSD_ERR_UNSUPPORTED, "bf16 GEMM needs K % 8 == 0");
  const SplitPlan plan = plan_splits(T, g.tiles_m, g.kchunks, head, dtype, sms);
  g.BN = plan.BN;
  g.tiles_n = plan.tiles_n;
  g.splits = plan.splits;
  g.stages = plan.stages;

  const int64_t tiles = (int64_t)g.tiles_m * g.tiles_n;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (g.splits > 1) {
    if (!workspace) return fail(SSD_ERR_WORKSPACE, "split-K GEMM needs a workspace");
    if (tiles > kMaxCounters) return fail(SSD_ERR_WORKSPACE, "too many split-K tiles");
    const int64_t need = kCounterBytes + partial_offset_bytes + tiles * g.splits * g.BN * kTileM * 4;
    if (need > workspace_bytes)
      return fail(SSD_ERR_WORKSPACE, "workspace too small: need %lld bytes", (long long)need);
    g.counters = reinterpret_cast<uint32_t*>(ws);
    g.partials = reinterpret_cast<float*>(ws + kCounterBytes + partial_offset_bytes);
  }
  if (g.tiles_n > 65535) return fail(SSD_ERR_UNSUPPORTED, "too many token tiles");
  dim3 grid(g.tiles_m * g.splits, g.tiles_n);
  // Several token tiles (prefill): the CTAs of one weight tile are adjacent in
  // launch order, so a wave streams each weight tile from HBM once and serves
  // its other token tiles from L2 (weight-tile-major order re-streams every
  // weight once per token tile).
  if (dtype == SSD_BF16 && g.tiles_n > 1 && g.splits == 1 && !head && !plan.sk && g.tiles_m <= 65535) {
    g.n_major = 1;
    grid = dim3(g.tiles_n, g.tiles_m);
  }

  if (dtype == SSD_BF16) {
    const bool sk = plan.sk;
    // Stream-K: one TMA box per weight segment a tile touches (128 rows when
    // every segment starts on a tile boundary, 64 + 64 for gate/up pairs),
    // else four 32-row boxes.
    g.a_box = 32;
    if (sk || big_boxes()) {
      if (layout == SSD_SEG_PAIRS) {
        g.a_box = 64;
      } else {
        bool aligned = true;
        for (int i = 1; i < n_seg; ++i) aligned = aligned && (g.seg_start[i] % kTileM == 0);
        if (aligned) g.a_box = 128;
      }
      for (int i = 0; i < n_seg; ++i)  // boxes no taller than any segment
        if (rows[i] < g.a_box) g.a_box = 32;
    }
    TcMaps maps;
    for (int i = 0; i < n_seg; ++i) {
      const int rc = get_map(w[i], (uint64_t)K, (uint64_t)rows[i], (uint64_t)K * 2, (uint32_t)g.a_box, &maps.w[i]);
      if (rc) return rc;
    }
    for (int i = n_seg; i < 3; ++i) maps.w[i] = maps.w[0];
    const int rc = get_map(x, (uint64_t)K, (uint64_t)T, (uint64_t)ldx * 2, (uint32_t)g.BN, &maps.x);
    if (rc) return rc;
    set_tc_attributes();
    if (sk) {
      const int64_t G = plan.sk_ctas;
      if (g.tiles_m > kMaxCounters / 2) return fail(SSD_ERR_WORKSPACE, "too many weight tiles");
      const int64_t need = kCounterBytes + partial_offset_bytes + 2 * G * kTileM * g.BN * 4;
      if (!workspace || need > workspace_bytes)
        return fail(SSD_ERR_WORKSPACE, "workspace too small: need %lld bytes", (long long)need);
      g.counters = reinterpret_cast<uint32_t*>(ws);
      g.partials = reinterpret_cast<float*>(ws + kCounterBytes + partial_offset_bytes);
      g.stages = sk_stages(g.BN);
      g.splits = 1;
      static bool sk_attr = false;
      if (!sk_attr) {
        allow_max_dynamic_smem(tc_gemm_sk_kernel);
        sk_attr = true;
      }
      return launch_kernel("tc_gemm_sk_kernel", tc_gemm_sk_kernel, dim3((unsigned)G), dim3(kTcThreads),
                           sk_smem_bytes(g.BN, g.stages), stream, 1u, 1u, maps, g, e);
    }
    // K-split CTAs of one tile run as one thread-block cluster (DSMEM reduction).
    return launch_kernel("tc_gemm_kernel", tc_gemm_kernel, grid, dim3(kTcThreads), tc_smem_bytes(g.BN, g.stages),
                         stream, (unsigned)g.splits, 1u, maps, g, e);
  }
  SimtSegs segs{};
  for (int i = 0; i < 3; ++i) {
    segs.p[i] = i < n_seg ? w[i] : w[0];
    segs.rows[i] = i < n_seg ? (int)rows[i] : 0;
  }
  return launch_kernel("simt_gemm_kernel", simt_gemm_kernel<float>, grid, dim3(256), 0, stream, 1u, 1u,
                       static_cast<const float*>(x), ldx, segs, g, e);
}


// ------------------------------------------------------- GEMM chain launch
// One CTA per SM: a chain CTA runs 256 threads at up to 129 registers, so
// two would not fit the register file.
static int chain_ctas_per_sm() { return 1; }
// static shared memory of tc_chain_kernel (link shapes and epilogue
// arguments, the epilogue's row-norm scales), rounded up
constexpr int kChainStaticSmem = 4096;
static_assert(kChainMax * (sizeof(GemmShape) + sizeof(EpiArgs)) + 1024 <= kChainStaticSmem, "chain static smem");
static int chain_stages(int BN, int per_sm) {
  // per CTA: 1 KB reserved by the system, 1 KB of static shared memory (the
  // epilogue's row-norm scales), alignment slack, barriers, the fp32 stage
  const int budget = (233472 - per_sm * 2048) / per_sm - kChainStaticSmem - kSkBarBytes;
  const int st = (budget - BN * kTileM * 4) / tc_stage_bytes(BN);
  return st > 16 ? 16 : st;
}
static size_t chain_smem_bytes(int BN, int stages) {
  return 1024 + (size_t)stages * tc_stage_bytes(BN) + (size_t)BN * kTileM * 4 + kSkBarBytes;
}
static_assert(sizeof(ChainParams) <= 32000, "chain parameters exceed the kernel parameter space");

// Grid of the chain kernel on this device: every CTA must be resident at
// once (CTAs wait on each other's counts), so the grid is what fits.
// The grid depends on the SM count only (not on T), so
// the K splits, and with them every row's rounding, are the same for every
// token count.
static_assert(kChainCounterBase + kChainCounters <= kMaxCounters / 2, "chain counters overlap the stream-K ones");
// Residency holds by construction: chain_stages sizes the shared memory so
// one CTA fits an SM, 256 threads x <= 255 registers fit the register file,
// and 2 x 128 TMEM columns fit TMEM. (No occupancy
// query: the first call may come during a stream capture.)
static int chain_grid(int BN, int* stages_out) {
  static bool attr = false;
  if (!attr) {
    allow_max_dynamic_smem(tc_chain_kernel);
    attr = true;
  }
  const int per_sm = chain_ctas_per_sm();
  const int stages = chain_stages(BN, per_sm);
  if (stages < 2) return 0;
  *stages_out = stages;
  return per_sm * device_sms();
}

int64_t chain_workspace_need(int64_t T) {
  if (T <= 0 || T > 64) return -1;
  const int BN = round_bn(T);
  int stages = 0;
  const int G = chain_grid(BN, &stages);
  if (G <= 0) return -1;
  return kCounterBytes + 2LL * G * kTileM * BN * 4;
}

int launch_chain(int n, const ChainLinkHost* links, int64_t T, void* workspace, int64_t workspace_bytes,
                 uint32_t* status, cudaStream_t stream) {
  if (n < 1 || n > kChainMax) return fail(SSD_ERR_INVALID, "ssd_linear_chain: 1..%d links", kChainMax);
  if (T < 1 || T > 64) return fail(SSD_ERR_UNSUPPORTED, "ssd_linear_chain: T must be 1..64");
  if (!workspace) return fail(SSD_ERR_WORKSPACE, "ssd_linear_chain needs a workspace");
  ChainParams P;
  memset(&P, 0, sizeof(P));
  P.BN = round_bn(T);
  const int G = chain_grid(P.BN, &P.stages);
  if (G <= 0) return fail(SSD_ERR_CUDA, "ssd_linear_chain: no resident grid for BN %d", P.BN);
  const int64_t need = kCounterBytes + 2LL * G * kTileM * P.BN * 4;
  if (need > workspace_bytes)
    return fail(SSD_ERR_WORKSPACE, "workspace too small: need %lld bytes", (long long)need);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  P.n = n;
  P.counters = reinterpret_cast<uint32_t*>(ws) + kChainCounterBase;
  P.partials = reinterpret_cast<float*>(ws + kCounterBytes);
  P.status = status;
  for (int l = 0; l < n; ++l) {
    const ChainLinkHost& h = links[l];
    if (!h.x || h.K <= 0 || h.K % 8 || h.n_seg < 1 || h.n_seg > 3)
      return fail(SSD_ERR_INVALID, "ssd_linear_chain: link %d: bad operands", l);
    if (h.K > (1 << 20)) return fail(SSD_ERR_UNSUPPORTED, "ssd_linear_chain: link %d: K too large", l);
    GemmShape& g = P.link[l].g;
    g.T = (int)T;
    g.K = (int)h.K;
    g.n_seg = h.n_seg;
    g.layout = h.layout;
    int64_t N = 0;
    for (int i = 0; i < h.n_seg; ++i) {
      if (!h.w[i] || h.rows[i] <= 0) return fail(SSD_ERR_INVALID, "ssd_linear_chain: link %d: empty segment", l);
      g.seg_start[i] = (int)N;
      N += h.rows[i];
    }
    g.seg_start[h.n_seg] = (int)N;
    if (h.layout == SSD_SEG_PAIRS) {
      if (h.n_seg != 2 || h.rows[0] != h.rows[1])
        return fail(SSD_ERR_INVALID, "ssd_linear_chain: link %d: PAIRS needs two equal segments", l);
      g.N = (int)(h.rows[0] * 2);
      g.tiles_m = (int)((h.rows[0] + 63) / 64);
    } else {
      for (int i = 0; i + 1 < h.n_seg; ++i)
        if (h.rows[i] % 32)
          return fail(SSD_ERR_UNSUPPORTED, "ssd_linear_chain: link %d: segments must be multiples of 32 rows", l);
      g.N = (int)N;
      g.tiles_m = (int)((N + kTileM - 1) / kTileM);
    }
    if (g.tiles_m > kChainTiles) return fail(SSD_ERR_UNSUPPORTED, "ssd_linear_chain: link %d: too many tiles", l);
    g.kchunks = (int)((h.K + kChunkK - 1) / kChunkK);
    g.BN = P.BN;
    g.tiles_n = 1;
    g.splits = 1;
    g.stages = P.stages;
    g.status = status;
    if (h.layout == SSD_SEG_PAIRS) {
      g.a_box = 64;
    } else {
      bool aligned = true;
      for (int i = 1; i < h.n_seg; ++i) aligned = aligned && (g.seg_start[i] % kTileM == 0);
      g.a_box = aligned ? 128 : 32;
    }
    for (int i = 0; i < h.n_seg; ++i)
      if (h.rows[i] < g.a_box) g.a_box = 32;
    TcMaps& maps = P.link[l].maps;
    for (int i = 0; i < h.n_seg; ++i) {
      const int rc = get_map(h.w[i], (uint64_t)h.K, (uint64_t)h.rows[i], (uint64_t)h.K * 2, (uint32_t)g.a_box,
                             &maps.w[i]);
      if (rc) return rc;
    }
    for (int i = h.n_seg; i < 3; ++i) maps.w[i] = maps.w[0];
    const int rc = get_map(h.x, (uint64_t)h.K, (uint64_t)T, (uint64_t)h.ldx * 2, (uint32_t)P.BN, &maps.x);
    if (rc) return rc;
    P.link[l].e = h.e;
  }
  return launch_kernel("tc_chain_kernel", tc_chain_kernel, dim3((unsigned)G), dim3(kChainThreads),
                       chain_smem_bytes(P.BN, P.stages), stream, 1u, 1u, P);
}

}  // namespace ssd
