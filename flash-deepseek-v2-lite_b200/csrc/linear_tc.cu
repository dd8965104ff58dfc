// "Batch" kernel family: weight-streaming GEMM on the 5th-generation tensor cores.
//
// Replaces (Flash-DeepSeeek-V2-Lite):
//   attention_decode_batch.py:420-468   _batched_linear_kernel (row-batched attention linears)
//   moe_batch.py:151-307                _grouped_gate_up_swiglu_kernel / _grouped_down_partial_kernel
// and the cuBLAS GEMMs of the shared experts / dense MLP that src/run.py:340-361 leaves
// around silu_mul.
//
// Y[token, n] = sum_k W[n, k] * X[token, k].  Weights are the A operand (M = 128
// weight rows per tile, K-major), tokens are the B operand (an N tile of 16..256
// tokens chosen per launch, padded to a multiple of 16), the fp32 accumulator lives
// in TMEM.  Decode is weight-bandwidth bound, so each 128-row weight tile is streamed
// from HBM once per N tile (the CTAs sharing a weight tile run side by side, so the
// repeats are served by L2); TMA moves 64-wide K slices of W and X (128-byte swizzle)
// through a multi-stage shared-memory ring.
//
// Warp roles (192 threads, persistent CTAs, one per SM):
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocator + tcgen05.mma issuer (one elected lane)
//   warps 2..5  epilogue: tcgen05.ld of the accumulator, fused SwiGLU / route-weight
//               scaling / bf16 or fp32 store (TMEM lane quadrant = warp % 4)
// SwiGLU tiles issue two MMAs per K step (gate rows and the matching up rows) into
// two TMEM accumulators, so silu(gate) * up is computed in registers.  When two
// accumulator sets fit in TMEM's 512 columns they are double-buffered: the MMAs of
// the next work item run while the epilogue drains the previous one.
//
// Grouped (MoE) mode: group g owns rows [group_offsets[g], group_offsets[g+1]) of X
// (activations gathered in expert order), read on the device; work items of empty
// groups are skipped by every role in the same order, so the grid is fixed and
// CUDA-graph safe.  All mbarrier waits are bounded (see common.cuh).
#include <cudaTypedefs.h>

#include <type_traits>

#include "linear.cuh"

namespace dsv2 {

constexpr int kTcThreads = 192;
constexpr int kTcM = 128;
constexpr int kTcK = 64;                 // K per stage (one 128-byte swizzle row)
constexpr int kTcABytes = kTcM * 128;    // 16 KB
constexpr int kTcBoxRows = 16;           // token rows per TMA box
constexpr int kTcSmemBudget = 216 * 1024;
constexpr int kTcTmemCols = 512;
constexpr int kTcMaxGroups = 256;
constexpr int kTcMaxStages = 8;

struct TcShape {
  int stages;
  int n_tile;        // tokens per work item (multiple of 16, <= 256)
  int stage_bytes;   // A (+A_up) + n_tile * 128
  int acc_cols;      // TMEM columns of one accumulator set (n_tile or 2 * n_tile)
  int acc_bufs;      // 1 or 2 (double-buffered accumulators)
  int tmem_cols;     // power of two >= acc_bufs * acc_cols
  int x_box;         // rows of the large activation box (tmap_xb)
};

__host__ __device__ inline int round_up(int a, int b) { return (a + b - 1) / b * b; }

__device__ __forceinline__ void store_out(bf16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ void store_out(float* p, float v) { *p = v; }

// EPI: epilogue (compile time); ROUTED: output rows come from route_y_row
template <int EPI, bool ROUTED>
__global__ __launch_bounds__(kTcThreads, 1) void linear_tc_kernel(
    const LinearParams p, const __grid_constant__ CUtensorMap tmap_w,
    const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_xb,
    const TcShape shp, int mt_count, int nt_count, int up_rows, int x_grouped) {
  constexpr bool SWIGLU = (EPI == kEpiSwiglu);
  using OutT = typename std::conditional<(EPI == kEpiStoreF32 || EPI == kEpiScaleF32), float,
                                         bf16>::type;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + shp.stages * shp.stage_bytes);
  uint64_t* empty_bar = full_bar + shp.stages;
  uint64_t* tfull_bar = empty_bar + shp.stages;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ int s_r0[kTcMaxGroups], s_cnt[kTcMaxGroups], s_nts[kTcMaxGroups];
  __shared__ int s_first[kTcMaxGroups + 1];

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
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_xb);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, static_cast<uint32_t>(shp.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int nkb = p.k / kTcK;
  const int a_tiles = SWIGLU ? 2 : 1;
  const int n_tile = shp.n_tile;
  // Grouped launches whose group offsets the previous kernel wrote wait for it here.
  // Dense launches (static work list) and grouped launches whose offsets are older
  // (p.offsets_prior) wait in the producer, after requesting the weight tiles of the
  // first pass over the ring.
  const bool early = p.group_offsets == nullptr || p.offsets_prior;
  if (!early) pdl_enter();

  // Compacted work list: group g contributes mt_count * ceil(cnt_g / n_tile) items
  // (none when empty).  Every CTA builds the same prefix from the device-side group
  // offsets, then takes items blockIdx.x, blockIdx.x + gridDim.x, ... so the work is
  // spread evenly over the CTAs whatever the routing.
  // With a K split (dense mode only) every (group, split) pair is one "virtual group".
  const int S = max(p.k_splits, 1);
  const int G = p.n_groups * S;
  for (int gi = threadIdx.x; gi < G; gi += kTcThreads) {
    int r0 = 0, cnt = p.n_tokens;
    if (p.group_offsets) {
      r0 = p.group_offsets[gi];
      cnt = p.group_offsets[gi + 1] - r0;
    }
    int nts = (max(cnt, 0) + n_tile - 1) / n_tile;
    if (nts > nt_count) {  // more tokens than the host-side bound: clamp and flag
      set_device_error(kErrIndex);
      nts = nt_count;
    }
    s_r0[gi] = r0;
    s_cnt[gi] = cnt;
    s_nts[gi] = nts;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int gi = 0; gi < G; ++gi) {
      s_first[gi] = acc;
      acc += s_nts[gi] * mt_count;
    }
    s_first[G] = acc;
  }
  __syncthreads();
  const int total_items = s_first[G];

  // item -> (group, m tile, n tile, first route, tokens); n tiles vary fastest so the
  // CTAs that share a weight tile run side by side (repeat reads hit L2)
  auto decode = [&](int it, int& g, int& mt, int& nt, int& r0, int& ntok, int& kb0,
                    int& kb1, int& sp) -> bool {
    int lo = 0, hi = G - 1;
    while (lo < hi) {  // last virtual group with s_first[vg] <= it
      const int mid = (lo + hi + 1) >> 1;
      if (s_first[mid] <= it) lo = mid; else hi = mid - 1;
    }
    const int vg = lo;
    const int local = it - s_first[vg];
    const int nts = s_nts[vg];
    mt = local / nts;
    nt = local - mt * nts;
    r0 = s_r0[vg];
    ntok = min(n_tile, s_cnt[vg] - nt * n_tile);
    g = vg / S;
    sp = vg - g * S;
    kb0 = sp * nkb / S;
    kb1 = (sp + 1) * nkb / S;
    return ntok > 0;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      // activation rows of one stage: as many large boxes as fit, 16-row boxes for the
      // rest (few large TMA requests per stage instead of many 2 KB ones)
      auto load_x = [&](int stage, int kb, int xrow0, int gx, int nbig, int nsmall) {
        unsigned char* sb = smem + stage * shp.stage_bytes + a_tiles * kTcABytes;
        for (int bx = 0; bx < nbig; ++bx)
          tma_load_3d(smem_u32(sb + bx * shp.x_box * 128), &tmap_xb, &full_bar[stage], kb * kTcK,
                      xrow0 + bx * shp.x_box, gx);
        for (int bx = 0; bx < nsmall; ++bx)
          tma_load_3d(smem_u32(sb + (nbig * shp.x_box + bx * kTcBoxRows) * 128), &tmap_x,
                      &full_bar[stage], kb * kTcK, xrow0 + nbig * shp.x_box + bx * kTcBoxRows, gx);
      };
      // early launches: the stages of the first ring pass get their weight tiles before
      // pdl_wait() and their activation tiles after it
      bool waited = !early;
      int npend = 0;
      int pend_kb[kTcMaxStages], pend_row[kTcMaxStages], pend_gx[kTcMaxStages];
      int pend_big[kTcMaxStages], pend_small[kTcMaxStages];
      auto release = [&]() {
        pdl_enter();
        waited = true;
        for (int i = 0; i < npend; ++i)
          load_x(i, pend_kb[i], pend_row[i], pend_gx[i], pend_big[i], pend_small[i]);
        npend = 0;
      };
      int stage = 0;
      uint32_t phase = 0;
      for (int it = blockIdx.x; it < total_items && !*abort_flag; it += gridDim.x) {
        int g, mt, nt, r0, ntok, kb0, kb1, sp;
        if (!decode(it, g, mt, nt, r0, ntok, kb0, kb1, sp)) continue;
        const int npad = round_up(ntok, 16);
        const int nbig = npad / shp.x_box;
        const int nsmall = (npad - nbig * shp.x_box) / kTcBoxRows;
        const int xrow0 = r0 + nt * n_tile;
        const int gx = x_grouped ? g : 0;
        const uint32_t bytes = a_tiles * kTcABytes + npad * 128;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { *abort_flag = 1; break; }
          unsigned char* st = smem + stage * shp.stage_bytes;
          mbar_arrive_expect_tx(&full_bar[stage], bytes);
          tma_load_3d(smem_u32(st), &tmap_w, &full_bar[stage], kb * kTcK, mt * kTcM, g);
          if (SWIGLU)
            tma_load_3d(smem_u32(st + kTcABytes), &tmap_w, &full_bar[stage], kb * kTcK,
                        mt * kTcM + up_rows, g);
          if (waited) {
            load_x(stage, kb, xrow0, gx, nbig, nsmall);
          } else {  // first ring pass: stage == npend
            pend_kb[npend] = kb;
            pend_row[npend] = xrow0;
            pend_gx[npend] = gx;
            pend_big[npend] = nbig;
            pend_small[npend] = nsmall;
            if (++npend == shp.stages) release();
          }
          if (++stage == shp.stages) { stage = 0; phase ^= 1; }
        }
      }
      if (!waited) release();
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t local = 0;
      for (int it = blockIdx.x; it < total_items && !*abort_flag; it += gridDim.x) {
        int g, mt, nt, r0, ntok, kb0, kb1, sp;
        if (!decode(it, g, mt, nt, r0, ntok, kb0, kb1, sp)) continue;
        const int npad = round_up(ntok, 16);
        const uint32_t idesc = make_idesc_bf16(kTcM, npad);
        const uint32_t buf = local % shp.acc_bufs;
        const uint32_t use = local / shp.acc_bufs;
        if (!mbar_wait(&tempty_bar[buf], (use & 1) ^ 1)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t dacc = tmem_base + buf * shp.acc_cols;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase)) { ok = false; break; }
          tc_fence_after();
          unsigned char* st = smem + stage * shp.stage_bytes;
          const uint64_t da = sw128_kmajor_desc(smem_u32(st));
          const uint64_t du = sw128_kmajor_desc(smem_u32(st + kTcABytes));
          const uint64_t db = sw128_kmajor_desc(smem_u32(st + a_tiles * kTcABytes));
#pragma unroll
          for (int k = 0; k < kTcK / 16; ++k) {
            const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
            // advance 16 bf16 (32 bytes) along K inside the swizzle row: +2 in addr>>4 units
            tc_mma_bf16(dacc, da + 2 * k, db + 2 * k, idesc, acc);
            if (SWIGLU) tc_mma_bf16(dacc + npad, du + 2 * k, db + 2 * k, idesc, acc);
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
    for (int it = blockIdx.x; it < total_items; it += gridDim.x) {
      int g, mt, nt, r0, ntok, kb0, kb1, sp;
      if (!decode(it, g, mt, nt, r0, ntok, kb0, kb1, sp)) continue;
      const int npad = round_up(ntok, 16);
      const long long split_off = static_cast<long long>(sp) * p.y_split_stride;
      const uint32_t buf = local % shp.acc_bufs;
      const uint32_t use = local / shp.acc_bufs;
      const bool ok = mbar_wait(&tfull_bar[buf], use & 1);
      if (!ok || *abort_flag) { *abort_flag = 1; break; }
      tc_fence_after();
      const int n = mt * kTcM + row_in_tile;
      const bool row_ok = n < p.n_rows;
      const uint32_t tbase =
          tmem_base + buf * shp.acc_cols + (static_cast<uint32_t>(quad * 32) << 16);
      const int rbase = r0 + nt * n_tile;
      // output column n of group g (dense rows advance by y_row_stride per token)
      OutT* ybase = reinterpret_cast<OutT*>(p.y) + split_off + g * p.y_group_stride + n;
      for (int c0 = 0; c0 < npad; c0 += 16) {
        float acc[16], accu[16];
        tmem_ld16(tbase + c0, acc);
        if (SWIGLU) tmem_ld16(tbase + npad + c0, accu);
        // routed rows: lanes 0..15 fetch this chunk's (row, scale) once, shuffled out below
        int my_row = 0;
        float my_scale = 1.f;
        if (ROUTED) {
          const int r = rbase + c0 + (lane & 15);
          if (c0 + (lane & 15) < ntok) {
            my_row = p.route_y_row[r];
            if (EPI == kEpiScaleF32) my_scale = p.route_scale[r];
          }
        }
        tmem_ld_wait();
        if (c0 + 16 >= npad) {
          // accumulator fully read: hand the buffer back to the MMA warp before storing
          tc_fence_before();
          mbar_arrive(&tempty_bar[buf]);
        }
        if (EPI == kEpiArgmax) {
          // per token: the largest bf16 value of this warp's 32 rows, lowest row on ties;
          // lane 0 stores one key per (32-row block, token)
          unsigned long long* kp = reinterpret_cast<unsigned long long*>(p.y) +
                                   static_cast<long long>(mt * 4 + quad) * p.y_row_stride + rbase + c0;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint32_t ord = row_ok ? argmax_ord(acc[j]) : 0u;
            const uint32_t best = __reduce_max_sync(0xffffffffu, ord);
            const uint32_t cand = (row_ok && ord == best) ? (0xffffffffu - static_cast<uint32_t>(n)) : 0u;
            const uint32_t low = __reduce_max_sync(0xffffffffu, cand);
            if (lane == 0 && c0 + j < ntok) kp[j] = (static_cast<unsigned long long>(best) << 32) | low;
          }
          continue;
        }
        OutT* yp = ybase + static_cast<long long>(rbase + c0) * p.y_row_stride;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const bool ok_j = row_ok && (c0 + j < ntok);
          float v = acc[j];
          if (EPI == kEpiSwiglu) {
            const float gt = bf16_round(acc[j]), up = bf16_round(accu[j]);
            v = silu_ref(gt) * up;
          }
          if (ROUTED) {
            const int yrow = __shfl_sync(0xffffffffu, my_row, j);
            const float sc = __shfl_sync(0xffffffffu, my_scale, j);
            if (EPI == kEpiScaleF32) v = bf16_round(v) * sc;
            if (ok_j) store_out(reinterpret_cast<OutT*>(p.y) + g * p.y_group_stride +
                                    static_cast<long long>(yrow) * p.y_row_stride + n, v);
          } else {
            if (ok_j) store_out(yp + j * p.y_row_stride, v);
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
}

static int pow2_at_least(int n) {
  int c = 32;
  while (c < n) c <<= 1;
  return c;
}

// Tile shape for one launch.  n_tile: tokens per work item, shrunk (down to 32) until
// the launch has work for about two thirds of the SMs, and capped at 128 for SwiGLU so
// that two accumulator sets (gate + up) fit in TMEM.
TcShape tc_shape(bool swiglu, int n_max, long long base_items, int num_sms, bool grouped,
                 bool keep_n) {
  TcShape s;
  // grouped (MoE) launches: most groups hold a few dozen tokens, so a 128-token tile
  // leaves shared memory for a deeper ring; the rare larger group takes two tiles
  const int n_cap = (swiglu || grouped) ? 128 : 256;
  int n_tile = round_up(min(max(n_max, 1), n_cap), 16);
  if (!grouped && !keep_n) {
    while (n_tile > 16 && base_items * ((n_max + n_tile - 1) / n_tile) * 3 < 2LL * num_sms)
      n_tile = round_up(n_tile / 2, 16);
  }
  s.n_tile = n_tile;
  s.stage_bytes = (swiglu ? 2 : 1) * kTcABytes + n_tile * 128;
  s.stages = min(kTcMaxStages, (kTcSmemBudget - 2048) / s.stage_bytes);
  s.acc_cols = n_tile * (swiglu ? 2 : 1);
  s.acc_bufs = (2 * s.acc_cols <= kTcTmemCols) ? 2 : 1;
  s.tmem_cols = pow2_at_least(s.acc_bufs * s.acc_cols);
  return s;
}

size_t tc_smem_bytes(const TcShape& s) {
  return 1024 /*alignment slack*/ + static_cast<size_t>(s.stages) * s.stage_bytes +
         (2 * s.stages + 4) * sizeof(uint64_t) + 16;
}

template <int EPI, bool ROUTED>
static cudaError_t tc_set_smem() {
  return cudaFuncSetAttribute(linear_tc_kernel<EPI, ROUTED>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
}

cudaError_t linear_tc_init() {
  const cudaError_t errs[] = {
      tc_set_smem<kEpiStoreBf16, false>(), tc_set_smem<kEpiStoreBf16, true>(),
      tc_set_smem<kEpiStoreF32, false>(),  tc_set_smem<kEpiStoreF32, true>(),
      tc_set_smem<kEpiSwiglu, false>(),    tc_set_smem<kEpiSwiglu, true>(),
      tc_set_smem<kEpiScaleF32, false>(),  tc_set_smem<kEpiScaleF32, true>(),
      tc_set_smem<kEpiArgmax, false>()};
  for (cudaError_t e : errs)
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

template <int EPI, bool ROUTED>
static void tc_launch(int grid, size_t smem, cudaStream_t st, const LinearParams& p,
                      const CUtensorMap& w, const CUtensorMap& x, const CUtensorMap& xb,
                      const TcShape& shp, int mt_count, int nt_count, int up_rows, int x_grouped) {
  launch_kernel(linear_tc_kernel<EPI, ROUTED>, grid, kTcThreads, smem, st, p, w, x, xb, shp, mt_count, nt_count, up_rows, x_grouped);
}

// Launch geometry, shared with the tensor-map builder in api.cu (the large activation
// box must match the token tile).  Returns the number of work items (0 = nothing to do).
long long tc_launch_shape(const LinearParams& p, int num_sms, TcShape* shp, int* mt_count,
                          int* nt_count) {
  const bool swiglu = (p.epilogue == kEpiSwiglu);
  const bool grouped = p.group_offsets != nullptr;
  const int n_max = grouped ? p.max_routes_per_group : p.n_tokens;
  *mt_count = (p.n_rows + kTcM - 1) / kTcM;
  const int S = max(p.k_splits, 1);
  // a K split keeps every token in one tile (weights read once); without one, small
  // launches shrink the token tile to spread over more SMs
  *shp = tc_shape(swiglu, n_max, static_cast<long long>(p.n_groups) * S * *mt_count, num_sms,
                  grouped, S > 1);
  shp->x_box = grouped ? min(64, shp->n_tile) : shp->n_tile;
  *nt_count = max(1, (n_max + shp->n_tile - 1) / shp->n_tile);
  return static_cast<long long>(p.n_groups) * S * *mt_count * *nt_count;
}

// tmap_w / tmap_x / tmap_xb: tensor maps built by the caller (api.cu) for W and for X
// with 16-row and shp.x_box-row boxes
cudaError_t launch_linear_tc_impl(const LinearParams& p, const CUtensorMap& tmap_w,
                                  const CUtensorMap& tmap_x, const CUtensorMap& tmap_xb,
                                  const TcShape& shp, int mt_count, int nt_count, long long items,
                                  int up_rows, int x_grouped, int num_sms, cudaStream_t st) {
  if (items <= 0) return cudaSuccess;
  const int S = max(p.k_splits, 1);
  if (static_cast<long long>(p.n_groups) * S > kTcMaxGroups || items > 0x7fffffffLL)
    return cudaErrorInvalidValue;
  const int grid = static_cast<int>(items < num_sms ? items : static_cast<long long>(num_sms));
  const size_t smem = tc_smem_bytes(shp);
  const bool routed = p.route_y_row != nullptr;
#define DSV2_TC_LAUNCH(E)                                                                       \
  (routed ? tc_launch<E, true>(grid, smem, st, p, tmap_w, tmap_x, tmap_xb, shp, mt_count,       \
                               nt_count, up_rows, x_grouped)                                    \
          : tc_launch<E, false>(grid, smem, st, p, tmap_w, tmap_x, tmap_xb, shp, mt_count,      \
                                nt_count, up_rows, x_grouped))
  switch (p.epilogue) {
    case kEpiStoreBf16: DSV2_TC_LAUNCH(kEpiStoreBf16); break;
    case kEpiStoreF32: DSV2_TC_LAUNCH(kEpiStoreF32); break;
    case kEpiSwiglu: DSV2_TC_LAUNCH(kEpiSwiglu); break;
    case kEpiArgmax:
      tc_launch<kEpiArgmax, false>(grid, smem, st, p, tmap_w, tmap_x, tmap_xb, shp, mt_count, nt_count,
                                   up_rows, x_grouped);
      break;
    default: DSV2_TC_LAUNCH(kEpiScaleF32); break;
  }
#undef DSV2_TC_LAUNCH
  return cudaGetLastError();
}

}  // namespace dsv2
