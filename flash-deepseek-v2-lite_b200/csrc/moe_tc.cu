// Batch family: the whole routed + shared MoE of one layer in one persistent launch.
//
// Replaces (Flash-DeepSeeek-V2-Lite):
//   moe_batch.py:151-238   _grouped_gate_up_swiglu_kernel   (phase 1 below)
//   moe_batch.py:241-307   _grouped_down_partial_kernel     (phase 2 below)
// launched back to back by _run_batched_grouped_routed_moe_grouped_triton
// (moe_batch.py:425-557).
//
// Phase 1 item (group g, 128-row tile of the intermediate dimension, token tile):
//   h[route, i] = bf16( silu(bf16(W_gate[g] x)) * bf16(W_up[g] x) )
// Phase 2 item (group g, 256-row tile of the hidden dimension, token tile):
//   y[route_slot[route], n] = bf16(W_down[g] h[route]) * route_weight[route]
// A group is a routed expert or one half of the shared MLP (see the router's bucketing).
// All phase-1 items followed by all phase-2 items form one list, groups in order of token
// count (largest first: the shared-expert halves at large batches, whose wide epilogues
// are the longest, start early, and the list ends on the shortest items).  The first rounds are dealt round-robin;
// the rest of the list is taken from a global counter, so the two GEMMs share one
// balanced stream of weight tiles and no CTA is left with a whole extra item at the end.  A phase-2 item of group g starts once every phase-1 item of g has stored
// its h rows: the phase-1 epilogue publishes a per-group counter (release), the
// phase-2 producer polls it (acquire, bounded) before its TMA loads of h.  Each CTA
// finishes its phase-1 items before its phase-2 items, and all CTAs are resident
// (one per SM, grid <= SM count), so every wait is for work that is running.  The
// last CTA to finish returns the counters to zero for the next launch.
//
// Data path per item: TMA (128-byte swizzle) stages of W (128 gate rows and the matching
// 128 up rows, or the two 128-row halves of 256 down rows, so a token tile is read once per
// 256 weight rows) and activations (expert-ordered x, or h) through a shared-memory ring;
// tcgen05.mma with the weights as A (M = 128, two MMAs per K step) and the tokens as B
// (N = token tile);
// fp32 accumulators in TMEM, double-buffered; epilogue warps read them with
// tcgen05.ld.  Warp roles as in linear_tc.cu.
#include "linear.cuh"

namespace dsv2 {

constexpr int kMoeThreads = 192;
constexpr int kMoeQueue = 4;   // item ids the producer may run ahead of the epilogue

struct MoeParams {
  int n_groups;
  int hidden;
  int inter;
  int x_rows;
  const int* group_offsets;   // [n_groups + 1]
  int max_routes_per_group;
  const int* route_slot;      // [routes] output row of each route
  const float* route_weight;  // [routes]
  bf16* h;                    // [x_rows, inter] phase-1 output / phase-2 input
  float* y;                   // [*, hidden] fp32
  int* sync;                  // [n_groups + 2]: per-group phase-1 counters, exit ticket, item counter
  PeerTable peers;            // world > 0: y rows (route slots) live in their owner rank's part
};

struct MoeShape {
  int n_tile;
  int stages;
  int stage_bytes;   // 2 weight tiles + n_tile * 128
  int acc_cols;      // 2 * n_tile (gate + up)
  int acc_bufs;
  int tmem_cols;
  int x_box;
  int nt_count;      // token tiles per group (host bound)
  int down_rows;     // down-projection rows per item: 256 (token tiles of 128) or 128
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// orders this thread's generic-proxy global accesses with its async-proxy (TMA) ones
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void epilogue_bar() {  // the 4 epilogue warps only
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

__global__ __launch_bounds__(kMoeThreads, 1) void moe_tc_kernel(
    const MoeParams p, const __grid_constant__ CUtensorMap tm_w1,
    const __grid_constant__ CUtensorMap tm_x1, const __grid_constant__ CUtensorMap tm_x1b,
    const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_h,
    const __grid_constant__ CUtensorMap tm_hb, const MoeShape shp) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + shp.stages * shp.stage_bytes);
  uint64_t* empty_bar = full_bar + shp.stages;
  uint64_t* tfull_bar = empty_bar + shp.stages;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;            // [2]
  uint64_t* wq_full = tempty_bar + 2;              // [kMoeQueue] item id published
  uint64_t* wq_empty = wq_full + kMoeQueue;         // [kMoeQueue] item id read by MMA + 4 epilogue warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wq_empty + kMoeQueue);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ int s_r0[kTcMaxGroups], s_cnt[kTcMaxGroups], s_nts[kTcMaxGroups];
  __shared__ int s_first1[kTcMaxGroups + 1], s_first2[kTcMaxGroups + 1];
  __shared__ int s_order[kTcMaxGroups];   // list position -> group (multi-tile groups first)
  __shared__ int s_item[kMoeQueue];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < shp.stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 128);
    }
    for (int q = 0; q < kMoeQueue; ++q) {
      mbar_init(&wq_full[q], 1);
      mbar_init(&wq_empty[q], 5);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_w1);
    prefetch_tmap(&tm_x1);
    prefetch_tmap(&tm_x1b);
    prefetch_tmap(&tm_w2);
    prefetch_tmap(&tm_h);
    prefetch_tmap(&tm_hb);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, static_cast<uint32_t>(shp.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // barriers, TMEM and tensor maps are set up while the previous launch finishes; the
  // group offsets and x come from the bucketing launch just before
  pdl_enter();

  const int n_tile = shp.n_tile;
  const int G = p.n_groups;
  const int mt1 = (p.inter + kTcM - 1) / kTcM;    // phase-1 row tiles (intermediate)
  // phase-2 row tiles: 256 hidden rows (two 128-row halves sharing one h tile) when the token
  // tiles are large, so h is re-read half as often; 128 rows for small token tiles (finer items)
  const bool wide = shp.down_rows == 2 * kTcM;
  const int mt2 = (p.hidden + shp.down_rows - 1) / shp.down_rows;
  const int nkb1 = p.hidden / kTcK, nkb2 = p.inter / kTcK;
  for (int g = threadIdx.x; g < G; g += kMoeThreads) {
    const int r0 = p.group_offsets[g];
    const int cnt = p.group_offsets[g + 1] - r0;
    int nts = (max(cnt, 0) + n_tile - 1) / n_tile;
    if (nts > shp.nt_count) {
      set_device_error(kErrIndex);
      nts = shp.nt_count;
    }
    s_r0[g] = r0;
    s_cnt[g] = cnt;
    s_nts[g] = nts;
  }
  __syncthreads();
  // groups in order of token count, largest first (ties by index): the multi-tile groups
  // (the shared-expert halves at large batches) start early and the list ends on the
  // items with the shortest epilogues
  {
    for (int g = threadIdx.x; g < G; g += kMoeThreads) {
      const int cg = s_cnt[g];
      int rank = 0;   // groups with more tokens, or as many and a lower index
      for (int h = 0; h < G; ++h) {
        const int ch = s_cnt[h];
        rank += (ch > cg) || (ch == cg && h < g);
      }
      s_order[rank] = g;
    }
  }
  __syncthreads();
  if (warp == 0) {
    // item prefix over the list (exclusive scan of token tiles per position, warp-wide)
    int run = 0;
    for (int base = 0; base < G; base += 32) {
      const int i = base + lane;
      const int v = i < G ? s_nts[s_order[i]] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      if (i < G) {
        s_first1[i] = (run + incl - v) * mt1;
        s_first2[i] = (run + incl - v) * mt2;
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      s_first1[G] = run * mt1;
      s_first2[G] = run * mt2;
    }
  }
  __syncthreads();
  const int total1 = s_first1[G];
  const int total_items = total1 + s_first2[G];

  // item -> (phase, group, row tile, token tile, first route, tokens)
  auto decode = [&](int it, int& ph, int& g, int& mt, int& nt, int& r0, int& ntok) -> bool {
    const int* first = s_first1;
    int local = it;
    ph = 1;
    if (it >= total1) {
      first = s_first2;
      local = it - total1;
      ph = 2;
    }
    int lo = 0, hi = G - 1;
    while (lo < hi) {  // last list position with first[pos] <= local
      const int mid = (lo + hi + 1) >> 1;
      if (first[mid] <= local) lo = mid; else hi = mid - 1;
    }
    local -= first[lo];
    g = s_order[lo];
    const int nts = s_nts[g];
    mt = local / nts;
    nt = local - mt * nts;
    r0 = s_r0[g];
    ntok = min(n_tile, s_cnt[g] - nt * n_tile);
    return ntok > 0;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      // items of the first rounds are dealt round-robin (no atomics); the rest of the
      // list is taken from a global counter, one grab ahead so its latency overlaps
      // the current item's loads
      const int n_static = max(0, total_items / static_cast<int>(gridDim.x) - 1);
      const int dyn_base = n_static * static_cast<int>(gridDim.x);
      int next_dyn = -1;
      if (n_static == 0) next_dyn = dyn_base + atomicAdd(&p.sync[G + 1], 1);
      for (int k = 0;; ++k) {
        // next item of the list (or the end marker) into the CTA's queue
        int it;
        if (k < n_static) {
          it = blockIdx.x + k * static_cast<int>(gridDim.x);
          if (k == n_static - 1) next_dyn = dyn_base + atomicAdd(&p.sync[G + 1], 1);
        } else {
          it = next_dyn;
          if (it < total_items) next_dyn = dyn_base + atomicAdd(&p.sync[G + 1], 1);
        }
        if (it >= total_items || *abort_flag) it = -1;
        const int qs = k % kMoeQueue;
        if (k >= kMoeQueue && !mbar_wait(&wq_empty[qs], ((k / kMoeQueue) - 1) & 1)) {
          *abort_flag = 1;
          it = -1;
        }
        s_item[qs] = it;
        mbar_arrive(&wq_full[qs]);
        if (it < 0) break;
        int ph, g, mt, nt, r0, ntok;
        if (!decode(it, ph, g, mt, nt, r0, ntok)) continue;
        if (ph == 2) {
          // every phase-1 tile of this group has stored its h rows
          const int target = s_nts[g] * mt1;
          bool ready = false;
          for (uint32_t i = 0; i < kSpinLimit; ++i) {
            if (ld_acquire_gpu(&p.sync[g]) >= target) { ready = true; break; }
            if (*abort_flag) break;
            __nanosleep(32);
          }
          if (!ready) {
            set_device_error(kErrMbarTimeout);
            *abort_flag = 1;
            break;
          }
          fence_proxy_async_global();
        }
        const int npad = round_up(ntok, 16);
        const int nbig = npad / shp.x_box;
        const int nsmall = (npad - nbig * shp.x_box) / kTcBoxRows;
        const int xrow0 = r0 + nt * n_tile;
        const CUtensorMap* mx = ph == 1 ? &tm_x1 : &tm_h;
        const CUtensorMap* mxb = ph == 1 ? &tm_x1b : &tm_hb;
        // activation rows of K block kb into the token tile at sb
        auto load_x = [&](unsigned char* sb, int kb, uint64_t* bar) {
          for (int bx = 0; bx < nbig; ++bx)
            tma_load_3d(smem_u32(sb + bx * shp.x_box * 128), mxb, bar, kb * kTcK,
                        xrow0 + bx * shp.x_box, 0);
          for (int bx = 0; bx < nsmall; ++bx)
            tma_load_3d(smem_u32(sb + (nbig * shp.x_box + bx * kTcBoxRows) * 128), mx, bar, kb * kTcK,
                        xrow0 + nbig * shp.x_box + bx * kTcBoxRows, 0);
        };
        // two 128-row weight tiles per slot: phase 1 gate rows and the matching up rows of one
        // K block; phase 2 (wide) the two halves of 256 down rows of one K block, or (narrow)
        // two K blocks of 128 down rows when their token tiles fit, so the down GEMM keeps as
        // many weight bytes in flight as the gate/up GEMM
        const int per_slot = (ph == 2 && !wide && 2 * npad <= n_tile) ? 2 : 1;
        const int nkb = ph == 1 ? nkb1 : nkb2;
        for (int kb = 0; kb < nkb; kb += per_slot) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { *abort_flag = 1; break; }
          unsigned char* st = smem + stage * shp.stage_bytes;
          unsigned char* sb = st + 2 * kTcABytes;
          if (ph == 1 || wide) {
            mbar_arrive_expect_tx(&full_bar[stage], 2 * kTcABytes + npad * 128);
            if (ph == 1) {
              tma_load_3d(smem_u32(st), &tm_w1, &full_bar[stage], kb * kTcK, mt * kTcM, g);
              tma_load_3d(smem_u32(st + kTcABytes), &tm_w1, &full_bar[stage], kb * kTcK,
                          mt * kTcM + p.inter, g);  // the matching up rows
            } else {
              tma_load_3d(smem_u32(st), &tm_w2, &full_bar[stage], kb * kTcK, mt * 2 * kTcM, g);
              tma_load_3d(smem_u32(st + kTcABytes), &tm_w2, &full_bar[stage], kb * kTcK,
                          mt * 2 * kTcM + kTcM, g);
            }
            load_x(sb, kb, &full_bar[stage]);
          } else {
            const int nb = min(per_slot, nkb - kb);
            mbar_arrive_expect_tx(&full_bar[stage], nb * (kTcABytes + npad * 128));
            for (int u = 0; u < nb; ++u) {
              tma_load_3d(smem_u32(st + u * kTcABytes), &tm_w2, &full_bar[stage], (kb + u) * kTcK,
                          mt * kTcM, g);
              load_x(sb + u * npad * 128, kb + u, &full_bar[stage]);
            }
          }
          if (++stage == shp.stages) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t local = 0;
      for (int k = 0;; ++k) {
        const int qs = k % kMoeQueue;
        if (!mbar_wait(&wq_full[qs], (k / kMoeQueue) & 1)) { *abort_flag = 1; break; }
        const int it = s_item[qs];
        mbar_arrive(&wq_empty[qs]);
        if (it < 0 || *abort_flag) break;
        int ph, g, mt, nt, r0, ntok;
        if (!decode(it, ph, g, mt, nt, r0, ntok)) continue;
        const int npad = round_up(ntok, 16);
        const uint32_t idesc = make_idesc_bf16(kTcM, npad);
        const uint32_t buf = local % shp.acc_bufs;
        const uint32_t use = local / shp.acc_bufs;
        if (!mbar_wait(&tempty_bar[buf], (use & 1) ^ 1)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t dacc = tmem_base + buf * shp.acc_cols;
        const int nkb = ph == 1 ? nkb1 : nkb2;
        const int per_slot = (ph == 2 && !wide && 2 * npad <= n_tile) ? 2 : 1;
        bool ok = true;
        for (int kb = 0; kb < nkb; kb += per_slot) {
          if (!mbar_wait(&full_bar[stage], phase)) { ok = false; break; }
          tc_fence_after();
          unsigned char* st = smem + stage * shp.stage_bytes;
          unsigned char* sb = st + 2 * kTcABytes;
          if (ph == 1 || wide) {
            const uint64_t da = sw128_kmajor_desc(smem_u32(st));
            const uint64_t du = sw128_kmajor_desc(smem_u32(st + kTcABytes));
            const uint64_t db = sw128_kmajor_desc(smem_u32(sb));
#pragma unroll
            for (int k = 0; k < kTcK / 16; ++k) {
              const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
              tc_mma_bf16(dacc, da + 2 * k, db + 2 * k, idesc, acc);          // gate / down rows 0-127
              tc_mma_bf16(dacc + npad, du + 2 * k, db + 2 * k, idesc, acc);   // up / down rows 128-255
            }
          } else {
            const int nb = min(per_slot, nkb - kb);
            for (int u = 0; u < nb; ++u) {
              const uint64_t da = sw128_kmajor_desc(smem_u32(st + u * kTcABytes));
              const uint64_t db = sw128_kmajor_desc(smem_u32(sb + u * npad * 128));
#pragma unroll
              for (int k = 0; k < kTcK / 16; ++k) {
                const uint32_t acc = (kb + u > 0 || k > 0) ? 1u : 0u;
                tc_mma_bf16(dacc, da + 2 * k, db + 2 * k, idesc, acc);
              }
            }
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == shp.stages) { stage = 0; phase ^= 1; }
        }
        if (!ok) { *abort_flag = 1; break; }
        tc_commit(&tfull_bar[buf]);
        ++local;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    uint32_t local = 0;
    for (int k = 0;; ++k) {
      const int qs = k % kMoeQueue;
      if (!mbar_wait(&wq_full[qs], (k / kMoeQueue) & 1)) { *abort_flag = 1; break; }
      const int it = s_item[qs];
      __syncwarp();
      if (lane == 0) mbar_arrive(&wq_empty[qs]);
      if (it < 0) break;
      int ph, g, mt, nt, r0, ntok;
      if (!decode(it, ph, g, mt, nt, r0, ntok)) continue;
      const int npad = round_up(ntok, 16);
      const uint32_t buf = local % shp.acc_bufs;
      const uint32_t use = local / shp.acc_bufs;
      const bool ok = mbar_wait(&tfull_bar[buf], use & 1);
      if (!ok || *abort_flag) { *abort_flag = 1; break; }
      tc_fence_after();
      const int n = mt * kTcM + row_in_tile;
      const uint32_t tbase =
          tmem_base + buf * shp.acc_cols + (static_cast<uint32_t>(quad * 32) << 16);
      const int rbase = r0 + nt * n_tile;
      if (ph == 1) {
        const bool row_ok = n < p.inter;
        bf16* hp = p.h + static_cast<long long>(rbase) * p.inter + n;
        for (int c0 = 0; c0 < npad; c0 += 16) {
          float acc[16], accu[16];
          tmem_ld16(tbase + c0, acc);
          tmem_ld16(tbase + npad + c0, accu);
          tmem_ld_wait();
          if (c0 + 16 >= npad) {
            tc_fence_before();
            mbar_arrive(&tempty_bar[buf]);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float gt = bf16_round(acc[j]), up = bf16_round(accu[j]);
            if (row_ok && c0 + j < ntok)
              hp[static_cast<long long>(c0 + j) * p.inter] = __float2bfloat16_rn(silu_ref(gt) * up);
          }
        }
        // publish this tile of h: the 128 epilogue threads' stores, then one release
        epilogue_bar();
        if (warp == 2 && lane == 0) {
          fence_proxy_async_global();
          __threadfence();
          red_release_gpu_add(&p.sync[g], 1);
        }
      } else {
        // row nd (accumulator columns [0, npad)) and, wide, row nd + 128 ([npad, 2 npad))
        const int nd = mt * shp.down_rows + row_in_tile;
        const bool row_ok0 = nd < p.hidden, row_ok1 = wide && nd + kTcM < p.hidden;
        for (int c0 = 0; c0 < npad; c0 += 16) {
          float acc[16], acc1[16];
          tmem_ld16(tbase + c0, acc);
          if (wide) tmem_ld16(tbase + npad + c0, acc1);
          int my_row = 0;
          float my_scale = 1.f;
          {
            const int r = rbase + c0 + (lane & 15);
            if (c0 + (lane & 15) < ntok) {
              my_row = p.route_slot[r];
              my_scale = p.route_weight[r];
            }
          }
          tmem_ld_wait();
          if (c0 + 16 >= npad) {
            tc_fence_before();
            mbar_arrive(&tempty_bar[buf]);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int yrow = __shfl_sync(0xffffffffu, my_row, j);
            const float sc = __shfl_sync(0xffffffffu, my_scale, j);
            if (c0 + j < ntok) {
              float* dst;
              if (p.peers.world > 0) {  // slot of a row owned by rank yrow / slots_per_rank
                const int spr = 8 * p.peers.rows_per_rank;
                const int owner = yrow / spr;
                dst = reinterpret_cast<float*>(p.peers.base[owner] + p.peers.part_off) +
                      static_cast<long long>(yrow - owner * spr) * p.hidden;
              } else {
                dst = p.y + static_cast<long long>(yrow) * p.hidden;
              }
              if (row_ok0) dst[nd] = bf16_round(acc[j]) * sc;
              if (row_ok1) dst[nd + kTcM] = bf16_round(acc1[j]) * sc;
            }
          }
        }
      }
      ++local;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, static_cast<uint32_t>(shp.tmem_cols));
  }
  // the last CTA out returns the group counters and the ticket to zero (and, expert
  // parallel, tells every rank that this rank's slot outputs are in place)
  if (threadIdx.x == 0) {
    if (p.peers.world > 0) __threadfence_system(); else __threadfence();
    const int t = atomicAdd(&p.sync[G], 1);
    if (t == static_cast<int>(gridDim.x) - 1) {
      __threadfence();
      for (int g = 0; g < G; ++g) p.sync[g] = 0;
      p.sync[G] = 0;
      p.sync[G + 1] = 0;
      __threadfence();
      if (p.peers.world > 0) {
        __threadfence_system();
        for (int q = 0; q < p.peers.world; ++q) red_release_sys_add_u64(peer_ctr(p.peers, q, 1), 1ull);
      }
    }
  }
}

// Launch geometry: token tile from the largest group (<= 128 so that two gate+up
// accumulator sets fit in TMEM) unless the caller fixes it, a ring as deep as shared
// memory allows.
MoeShape moe_shape(int max_routes_per_group, int tile_tokens) {
  MoeShape s;
  s.n_tile = tile_tokens > 0 ? tile_tokens : round_up(min(max(max_routes_per_group, 1), 128), 16);
  s.stage_bytes = 2 * kTcABytes + s.n_tile * 128;
  s.stages = min(kTcMaxStages, (kTcSmemBudget - 2048) / s.stage_bytes);
  s.acc_cols = 2 * s.n_tile;
  s.acc_bufs = (2 * s.acc_cols <= kTcTmemCols) ? 2 : 1;
  int c = 32;
  while (c < s.acc_bufs * s.acc_cols) c <<= 1;
  s.tmem_cols = c;
  s.x_box = min(64, s.n_tile);
  s.nt_count = max(1, (max_routes_per_group + s.n_tile - 1) / s.n_tile);
  s.down_rows = s.n_tile >= 128 ? 2 * kTcM : kTcM;
  return s;
}

size_t moe_smem_bytes(const MoeShape& s) {
  return 1024 + static_cast<size_t>(s.stages) * s.stage_bytes +
         (2 * s.stages + 4 + 2 * kMoeQueue) * sizeof(uint64_t) + 16;
}

cudaError_t moe_tc_init() {
  return cudaFuncSetAttribute(moe_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              220 * 1024);
}

cudaError_t launch_moe_tc(const MoeParams& p, const CUtensorMap& w1, const CUtensorMap& x1,
                          const CUtensorMap& x1b, const CUtensorMap& w2, const CUtensorMap& h,
                          const CUtensorMap& hb, const MoeShape& shp, int num_sms, cudaStream_t st) {
  if (p.n_groups + 2 > kTcMaxGroups) return cudaErrorInvalidValue;
  launch_kernel(moe_tc_kernel, num_sms, kMoeThreads, moe_smem_bytes(shp), st, p, w1, x1, x1b, w2, h,
                hb, shp);
  return cudaGetLastError();
}

}  // namespace dsv2
