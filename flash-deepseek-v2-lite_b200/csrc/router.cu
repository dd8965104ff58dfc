// Fused MoE router: fp32 gate GEMV + softmax + top-6, then token-to-expert bucketing.
//
// Replaces (Flash-DeepSeeek-V2-Lite):
//   moe_router.py:8-60          _router_softmax_topk6_kernel (softmax over 64 logits, six
//                                argmax rounds, weights * routed_scaling_factor; B = 1 only)
//   src/run.py:257-275          fp32 gate F.linear feeding it
//   moe_batch.py:101-148        _zero_counts / _build_route_indices (atomic bucket) /
//                                _build_route_blocks
// The gate logits follow the HF MoE gate (fp32 linear over bf16 inputs; softmax in
// fp32; greedy top-k; no renormalisation; weights scaled by routed_scaling_factor).
//
// router_topk_kernel: one CTA per 8 tokens computes all 64 logits on the tensor cores
// (mma.sync m16n8k16, experts as M, tokens as N; bf16 products are exact in fp32, so
// this is the fp32 linear up to summation order), warps split K and meet in shared
// memory (16 warps: 4 expert blocks x 4 K quarters), then one warp per token does the
// softmax and the six argmax rounds
// (lowest index first on ties).  It serves fp32 gates and the expert-parallel dispatch;
// a bf16 gate on one rank takes router_fused_kernel (experts split over a 4-CTA cluster,
// logits met in CTA 0's shared memory), which can also form its inputs (residual add +
// RMSNorm) and bucket the routes in the same launch.
//
// route_kernel: stable counting sort of the routes by local expert.  Every CTA counts
// all routes per expert (the top-k ids are a few KB) and the routes of earlier tokens,
// so it knows where its own tokens' routes go without any grid-wide synchronisation;
// inside a CTA, routes are ranked in (token, k) order.  Two extra "shared" groups
// carry the local tokens with weight 1 (slots 6 and 7), so the MoE kernels run the two
// shared experts in the same launch as the routed ones.  Optionally the same kernel
// copies each route's activation row into expert-contiguous order for the TMA path: with
// at most one token per warp, each warp loads its piece of its token's row together with
// the routing ids and stores it to all of the token's placed slots; larger CTAs copy one
// placed row per warp.
#include "params.cuh"

namespace dsv2 {

constexpr int kTopK = 6;
constexpr int kMaxExperts = 64;
constexpr int kSlots = 8;              // 6 routed + 2 shared-expert halves per token
constexpr int kRtTok = 8;              // tokens per CTA (the mma N dimension)
constexpr int kRtKParts = 4;           // K quarters per expert block
constexpr int kRtThreads = 128 * kRtKParts;  // 16 warps: 4 expert blocks of 16 x 4 K quarters
constexpr int kRtMaxHidden = 2048;
constexpr int kRouteTokMax = 32;       // tokens per route_kernel CTA (upper bound)
constexpr int kRouteThreads = 256;
constexpr int kRouteMaxRows = 4096;

// softmax + top-6 for one token with one warp; logits in shared/global memory.
// Per lane: the ranks of its two experts (lane, lane + 32) and their probabilities.
struct TopkLane {
  int r0, r1;
  float p0, p1;
};

__device__ TopkLane softmax_topk_warp(const float* lg, int n_experts, float scaling, int row,
                                      long long* ids64, int* ids32, float* tw) {
  const int lane = threadIdx.x & 31;
  float v0 = lane < n_experts ? lg[lane] : -INFINITY;
  float v1 = lane + 32 < n_experts ? lg[lane + 32] : -INFINITY;
  const float m = warp_max(fmaxf(v0, v1));
  float e0 = lane < n_experts ? expf(v0 - m) : 0.f;
  float e1 = lane + 32 < n_experts ? expf(v1 - m) : 0.f;
  const float s = warp_sum(e0 + e1);
  const float p0 = lane < n_experts ? e0 / s : -INFINITY;
  const float p1 = lane + 32 < n_experts ? e1 / s : -INFINITY;
  // top-6 by rank: expert e's rank is the number of experts with a larger probability, or
  // an equal one and a lower index (the greedy order: largest first, lowest index on ties);
  // every lane ranks its two experts against all 64 at once instead of six serial arg-max
  // rounds
  int r0 = 0, r1 = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float a = __shfl_sync(0xffffffffu, p0, j);   // expert j
    const float b = __shfl_sync(0xffffffffu, p1, j);   // expert j + 32
    r0 += (a > p0 || (a == p0 && j < lane)) + (b > p0);
    r1 += (a >= p1) + (b > p1 || (b == p1 && j < lane));
  }
  if (r0 < kTopK) {
    if (ids64) ids64[row * kTopK + r0] = lane;
    ids32[row * kTopK + r0] = lane;
    tw[row * kTopK + r0] = p0 * scaling;
  }
  if (r1 < kTopK) {
    if (ids64) ids64[row * kTopK + r1] = lane + 32;
    ids32[row * kTopK + r1] = lane + 32;
    tw[row * kTopK + r1] = p1 * scaling;
  }
  return TopkLane{r0, r1, p0, p1};
}

// Bucketing of a single row by the warp that ranked its experts (one rank, every expert
// local): the same group offsets and route arrays as route_cta gives for one token, without
// reading the ids back.  Expert e's group holds its route (slot = its rank) when e is among
// the top 6; the two shared groups follow with slots 6 and 7.
__device__ void bucket_one_row_warp(const RouterParams& p, const TopkLane& t) {
  const int lane = threadIdx.x & 31;
  const bool s0 = t.r0 < kTopK && lane < p.n_experts;
  const bool s1 = t.r1 < kTopK && lane + 32 < p.n_experts;
  const unsigned m0 = __ballot_sync(0xffffffffu, s0), m1 = __ballot_sync(0xffffffffu, s1);
  const unsigned lt = (1u << lane) - 1u;
  const int off0 = __popc(m0 & lt), off1 = __popc(m0) + __popc(m1 & lt);
  const int total = __popc(m0) + __popc(m1);
  if (lane < p.n_local) p.group_offsets[lane] = off0;
  if (lane + 32 < p.n_local) p.group_offsets[lane + 32] = off1;
  if (s0) {
    p.route_token[off0] = 0;
    p.route_slot[off0] = t.r0;
    p.route_weight[off0] = t.p0 * p.scaling;
  }
  if (s1) {
    p.route_token[off1] = 0;
    p.route_slot[off1] = t.r1;
    p.route_weight[off1] = t.p1 * p.scaling;
  }
  if (lane == 0) {
    p.group_offsets[p.n_local] = total;
    p.group_offsets[p.n_local + 1] = total + 1;
    p.group_offsets[p.n_local + 2] = total + 2;
  }
  if (lane < 2) {
    p.route_token[total + lane] = 0;
    p.route_slot[total + lane] = kTopK + lane;
    p.route_weight[total + lane] = 1.f;
  }
}

// ---------------------------------------------------------------------------------
// logits + softmax + top-6
// ---------------------------------------------------------------------------------
__global__ __launch_bounds__(kRtThreads) void router_topk_kernel(const RouterParams p) {
  pdl_enter();
  constexpr int XS = kRtMaxHidden + 8;  // padded row (bank spread for the 16-byte reads)
  __shared__ __align__(16) bf16 s_x[kRtTok][XS];
  __shared__ float s_part[kRtKParts][kMaxExperts][kRtTok];
  __shared__ float s_logits[kRtTok][kMaxExperts];
  const int row0 = blockIdx.x * kRtTok;
  const int nt = min(kRtTok, p.rows - row0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nch = p.hidden / 8;
  for (int i = tid; i < kRtTok * nch; i += kRtThreads) {
    const int t = i / nch, c = i % nch;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < nt) v = *reinterpret_cast<const uint4*>(p.x + (row0 + t) * p.x_row_stride + c * 8);
    *reinterpret_cast<uint4*>(&s_x[t][c * 8]) = v;
  }
  __syncthreads();
  // warp -> experts [16*eb, 16*eb + 16), K part kh
  const int eb = warp & 3, kh = warp >> 2;
  const int gq = lane >> 2, tq = lane & 3;
  const int eA = eb * 16 + gq, eB = eA + 8;
  const bool okA = eA < p.n_experts, okB = eB < p.n_experts;
  float c[4] = {0.f, 0.f, 0.f, 0.f};
  const int nkb = p.hidden / 32;              // 32-wide K blocks
  const int kb_beg = kh * nkb / kRtKParts, kb_end = (kh + 1) * nkb / kRtKParts;
  const bf16* xr = &s_x[gq][tq * 8];
  if (p.w_dtype == 0) {
    const bf16* wA = reinterpret_cast<const bf16*>(p.w) + static_cast<long long>(okA ? eA : 0) * p.hidden + tq * 8;
    const bf16* wB = reinterpret_cast<const bf16*>(p.w) + static_cast<long long>(okB ? eB : 0) * p.hidden + tq * 8;
    for (int kb0 = kb_beg; kb0 < kb_end; kb0 += 8) {
      uint4 a[8], b[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int kb = kb0 + u;
        a[u] = (kb < kb_end && okA) ? *reinterpret_cast<const uint4*>(wA + kb * 32) : make_uint4(0, 0, 0, 0);
        b[u] = (kb < kb_end && okB) ? *reinterpret_cast<const uint4*>(wB + kb * 32) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int kb = kb0 + u;
        if (kb >= kb_end) break;
        const uint4 xv = *reinterpret_cast<const uint4*>(xr + kb * 32);
        const uint32_t a0[4] = {a[u].x, b[u].x, a[u].y, b[u].y};
        mma_bf16_16816(c, a0, xv.x, xv.y);
        const uint32_t a1[4] = {a[u].z, b[u].z, a[u].w, b[u].w};
        mma_bf16_16816(c, a1, xv.z, xv.w);
      }
    }
  } else {
    // fp32 gate weights: CUDA-core path (exact fp32 products); thread (gq, tq) owns the
    // same (expert, token) outputs as its mma fragment would
    const float* wf = reinterpret_cast<const float*>(p.w);
    for (int k = kb_beg * 32; k < kb_end * 32; ++k) {
      const float x0 = __bfloat162float(s_x[2 * tq][k]), x1 = __bfloat162float(s_x[2 * tq + 1][k]);
      const float wa = okA ? wf[static_cast<long long>(eA) * p.hidden + k] : 0.f;
      const float wb = okB ? wf[static_cast<long long>(eB) * p.hidden + k] : 0.f;
      c[0] = fmaf(wa, x0, c[0]); c[1] = fmaf(wa, x1, c[1]);
      c[2] = fmaf(wb, x0, c[2]); c[3] = fmaf(wb, x1, c[3]);
    }
  }
  // C fragment: (expert gq, tokens 2tq, 2tq+1), (expert gq+8, ...)
  s_part[kh][eb * 16 + gq][2 * tq] = c[0];
  s_part[kh][eb * 16 + gq][2 * tq + 1] = c[1];
  s_part[kh][eb * 16 + gq + 8][2 * tq] = c[2];
  s_part[kh][eb * 16 + gq + 8][2 * tq + 1] = c[3];
  __syncthreads();
  for (int i = tid; i < kRtTok * kMaxExperts; i += kRtThreads) {
    const int t = i / kMaxExperts, e = i % kMaxExperts;
    if (e < p.n_experts && t < nt) {
      float v = s_part[0][e][t];
#pragma unroll
      for (int q = 1; q < kRtKParts; ++q) v += s_part[q][e][t];
      if (p.bias) v += p.bias[e];
      s_logits[t][e] = v;
      p.logits[(row0 + t) * p.n_experts + e] = v;
    }
  }
  __syncthreads();
  if (warp < nt)
    softmax_topk_warp(s_logits[warp], p.n_experts, p.scaling, row0 + warp, p.topk_ids, p.topk_ids32,
                      p.topk_w);
  if (p.peers.world > 0) {
    // expert-parallel dispatch: this CTA's rows (normalised x, top-6 ids and weights) go
    // to every rank's buffer at their global row, then one arrival per rank
    __syncthreads();
    const PeerTable& pt = p.peers;
    const long long g0 = static_cast<long long>(p.row_base) + row0;
    for (int q = 0; q < pt.world; ++q) {
      bf16* xg = reinterpret_cast<bf16*>(pt.base[q] + pt.xg_off) + g0 * p.hidden;
      for (int i = tid; i < nt * nch; i += kRtThreads) {
        const int t = i / nch, c = i % nch;
        *reinterpret_cast<uint4*>(xg + static_cast<long long>(t) * p.hidden + c * 8) =
            *reinterpret_cast<const uint4*>(&s_x[t][c * 8]);
      }
      int* ig = reinterpret_cast<int*>(pt.base[q] + pt.ids_off) + g0 * kTopK;
      float* wg = reinterpret_cast<float*>(pt.base[q] + pt.w_off) + g0 * kTopK;
      for (int i = tid; i < nt * kTopK; i += kRtThreads) {
        ig[i] = p.topk_ids32[row0 * kTopK + i];
        wg[i] = p.topk_w[row0 * kTopK + i];
      }
    }
    __syncthreads();
    if (tid == 0) {
      __threadfence_system();
      for (int q = 0; q < pt.world; ++q) red_release_sys_add_u64(peer_ctr(pt, q, 0), 1ull);
    }
  }
}

// ---------------------------------------------------------------------------------
// bucketing (+ optional gather of activation rows)
// ---------------------------------------------------------------------------------
struct RouteParams {
  const int* ids32;        // [rows, 6]
  const float* tw;         // [rows, 6]
  int rows;
  int expert_lo, n_local;
  int shared_lo, shared_hi;
  int* group_offsets;      // [n_local + 3]
  int* route_token;
  int* route_slot;
  float* route_weight;
  const bf16* gx;          // optional gather source [rows, cols]
  long long gx_stride;
  bf16* gout;              // optional gather destination [routes, cols]
  int cols;
  int tok_per_cta;
  PeerTable peers;         // world > 0: ids / weights / x were dispatched by every rank
  int layer;               // MoE layer index (expected dispatch arrivals)
};

// Bucketing of the tokens [cta * tok_per_cta, +tok_per_cta) by one CTA of THREADS threads
// (shared by the separate bucketing launch and the fused router).
template <int THREADS>
__device__ void route_cta(const RouteParams& p, int cta) {
  static_assert(kRouteTokMax * kTopK <= THREADS, "one thread per route of the CTA");
  constexpr int kRouteWarps = THREADS / 32;
  __shared__ int s_total[kMaxExperts];
  __shared__ int s_before[kMaxExperts];
  __shared__ int s_off[kMaxExperts + 3];
  __shared__ int s_e[kRouteTokMax * kTopK];
  __shared__ int s_pos[kRouteTokMax * kSlots];
  __shared__ int s_tok[kRouteTokMax * kSlots];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tpc = p.tok_per_cta;
  const int tok0 = cta * tpc;
  const int ntok = min(tpc, p.rows - tok0);
  const int n_routes = p.rows * kTopK;
  const int r_first = tok0 * kTopK;
  const int my_routes = ntok * kTopK;
  // Issued together with the counting loads below: this thread's own route (route tid of
  // the CTA) and, when the CTA has at most one token per warp-group, its share of its
  // token's activation row, which every placed slot of that token receives.
  int e_mine = -1;
  float w_mine = 0.f;
  if (tid < my_routes) {
    e_mine = __ldcg(p.ids32 + r_first + tid) - p.expert_lo;
    w_mine = __ldcg(p.tw + r_first + tid);
  }
  const int n16 = p.cols / 8;
  const bool reg_gather = p.gout && ntok > 0 && ntok <= kRouteWarps && n16 <= 8 * 32 * (kRouteWarps / ntok);
  const int gw_per_tok = reg_gather ? kRouteWarps / ntok : 1;
  const int g_tok = warp / gw_per_tok, g_part = warp % gw_per_tok;
  const bool g_warp = reg_gather && g_tok < ntok;
  const int c_beg = g_part * n16 / gw_per_tok, c_end = (g_part + 1) * n16 / gw_per_tok;
  uint4 xv[8];
  if (g_warp) {
    const uint4* src = reinterpret_cast<const uint4*>(p.gx + static_cast<long long>(tok0 + g_tok) * p.gx_stride);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = c_beg + u * 32 + lane;
      if (c < c_end) xv[u] = __ldcg(src + c);
    }
  }
  for (int i = tid; i < kMaxExperts; i += THREADS) { s_total[i] = 0; s_before[i] = 0; }
  __syncthreads();
  // all routes' expert ids, eight loads in flight per thread
  for (int r0 = 0; r0 < n_routes; r0 += 8 * THREADS) {
    int ev[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int r = r0 + u * THREADS + tid;
      ev[u] = r < n_routes ? __ldcg(p.ids32 + r) - p.expert_lo : -1;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int r = r0 + u * THREADS + tid;
      const int e = ev[u];
      if (r < n_routes && e >= 0 && e < p.n_local) {
        atomicAdd(&s_total[e], 1);
        if (r < r_first) atomicAdd(&s_before[e], 1);
      }
    }
  }
  __syncthreads();
  if (tid < 32) {  // exclusive scan of the expert totals (64 = 2 per lane)
    const int lane = tid;
    const int a = lane * 2 < p.n_local ? s_total[lane * 2] : 0;
    const int b = lane * 2 + 1 < p.n_local ? s_total[lane * 2 + 1] : 0;
    int incl = a + b;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int excl = incl - a - b;
    if (lane * 2 < p.n_local) s_off[lane * 2] = excl;
    if (lane * 2 + 1 < p.n_local) s_off[lane * 2 + 1] = excl + a;
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (lane == 0) {
      const int nsh = p.shared_hi - p.shared_lo;
      s_off[p.n_local] = total;
      s_off[p.n_local + 1] = total + nsh;
      s_off[p.n_local + 2] = total + 2 * nsh;
    }
  }
  // this CTA's routes, in (token, k) order
  if (tid < my_routes) s_e[tid] = (e_mine >= 0 && e_mine < p.n_local) ? e_mine : -1;
  __syncthreads();
  if (cta == 0)
    for (int g = tid; g <= p.n_local + 2; g += THREADS) p.group_offsets[g] = s_off[g];
  if (tid < my_routes) {
    const int i = tid;
    const int e = s_e[i];
    int pos = -1;
    if (e >= 0) {
      int rank = 0;
      for (int j = 0; j < i; ++j) rank += (s_e[j] == e);
      pos = s_off[e] + s_before[e] + rank;
      const int r = r_first + i;
      const int b = r / kTopK, k = r % kTopK;
      p.route_token[pos] = b;
      p.route_slot[pos] = b * kSlots + k;
      p.route_weight[pos] = w_mine;
      s_tok[i] = b;
    }
    s_pos[i] = pos;
  }
  // shared-expert routes of this CTA's tokens (slots 6 and 7)
  for (int i = tid; i < 2 * tpc; i += THREADS) {
    const int sh = i / tpc, t = i % tpc;
    const int b = tok0 + t;
    int pos = -1;
    if (t < ntok && b >= p.shared_lo && b < p.shared_hi) {
      pos = s_off[p.n_local + sh] + (b - p.shared_lo);
      p.route_token[pos] = b;
      p.route_slot[pos] = b * kSlots + kTopK + sh;
      p.route_weight[pos] = 1.f;
    }
    s_pos[tpc * kTopK + i] = pos;
    s_tok[tpc * kTopK + i] = b;
  }
  if (!p.gout) return;
  __syncthreads();
  if (reg_gather) {
    // the staged row pieces go to every placed slot of their token (6 routed, 2 shared)
    if (!g_warp) return;
    for (int sl = 0; sl < kSlots; ++sl) {
      const int pos = sl < kTopK ? s_pos[g_tok * kTopK + sl] : s_pos[tpc * kTopK + (sl - kTopK) * tpc + g_tok];
      if (pos < 0) continue;
      uint4* dst = reinterpret_cast<uint4*>(p.gout + static_cast<long long>(pos) * p.cols);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c_beg + u * 32 + lane;
        if (c < c_end) dst[c] = xv[u];
      }
    }
    return;
  }
  // gather: one warp per placed row; each lane holds up to 8 16-byte chunks in flight
  const int nslots = tpc * kSlots;
  for (int i = warp; i < nslots; i += kRouteWarps) {
    if (i < tpc * kTopK && i >= my_routes) continue;
    const int pos = s_pos[i];
    if (pos < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(p.gx + s_tok[i] * p.gx_stride);
    uint4* dst = reinterpret_cast<uint4*>(p.gout + static_cast<long long>(pos) * p.cols);
    for (int c0 = 0; c0 < n16; c0 += 8 * 32) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < n16) v[u] = __ldcg(src + c);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < n16) dst[c] = v[u];
      }
    }
  }
}

__global__ __launch_bounds__(kRouteThreads) void route_kernel(const RouteParams p) {
  pdl_enter();
  if (p.peers.world > 0) {
    // every rank's router has written its rows into this rank's buffer
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
      const unsigned long long per_rank = (p.peers.rows_per_rank + kRtTok - 1) / kRtTok;
      s_ok = wait_counter_sys(peer_ctr(p.peers, p.peers.rank, 0), peer_target(p.peers, p.layer, per_rank),
                              p.peers.wait_polls, p.peers.wait_stats);
    }
    __syncthreads();
    if (!s_ok) return;
  }
  route_cta<kRouteThreads>(p, blockIdx.x);
}

// ---------------------------------------------------------------------------------
// Fused router (bf16 gate, one rank): [residual add + RMSNorm] + gate logits + softmax +
// top-6 [+ bucketing + gather of the expert-ordered activations], one launch
// ---------------------------------------------------------------------------------
// Clusters of four CTAs share a group of 8 tokens: CTA r computes experts [16r, 16r + 16)
// (one mma M block) with its 16 warps each taking a sixteenth of K, so a CTA reads 64 KB of
// gate, and those weight fragments are loaded before the programmatic-launch wait (weights
// are never written by earlier kernels).  Every CTA stores its 16 x 8 logits into CTA 0's
// shared memory (distributed shared memory), and CTA 0 runs the softmax / top-6.  A cluster
// loops over token groups when there are more groups than clusters.
//
// With p.h set, the group's inputs are first formed here: CTA r adds the previous
// sublayer's output to the residual stream of tokens 2r and 2r + 1 and normalises them,
// one 256-thread half per token with the same per-thread chunks and reduction order as
// add_rmsnorm_kernel (so the results are bit-identical to that launch followed by the
// router), writes h and x to global memory and x into all four CTAs' shared memory.
//
// With bucketing (p.group_offsets) the CTAs then meet at a grid-wide barrier (arrival
// count + generation in p.grid_sync, bounded wait; the grid never exceeds the clusters
// that fit on the GPU at once, so every CTA is resident; a grid of one cluster uses the
// cluster barrier instead) and each CTA buckets a slice of
// the tokens and copies their activation rows into expert order (route_cta).  The
// kernel triggers its dependents only after that barrier, so the next launch cannot take
// the SMs that CTAs still waiting to start would need.
constexpr int kRcCtas = 4;                           // CTAs per cluster
constexpr int kRcExperts = kMaxExperts / kRcCtas;    // experts per CTA (16)
constexpr int kRcKParts = 16;                        // warps per CTA, one K part each
constexpr int kRcThreads = 32 * kRcKParts;
constexpr int kRcKb = kRtMaxHidden / 32 / kRcKParts;  // 32-wide K blocks per warp (4)

__device__ __forceinline__ int ld_acquire_gpu_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add_s32(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid-wide barrier of one launch: sync[0] counts arrivals, sync[1] is a generation that
// the last arrival advances (after returning the count to zero), so the pair needs no
// clearing between launches.  Bounded: returns false (device error set) if the grid does
// not gather.
__device__ bool grid_barrier(int* sync) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    const int gen = ld_acquire_gpu_s32(&sync[1]);   // read before arriving
    __threadfence();
    bool ok = true;
    if (atomicAdd(&sync[0], 1) == static_cast<int>(gridDim.x) - 1) {
      sync[0] = 0;
      red_release_gpu_add_s32(&sync[1], 1);
    } else {
      ok = false;
      for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (ld_acquire_gpu_s32(&sync[1]) != gen) { ok = true; break; }
        if ((i & 255) == 0 && *reinterpret_cast<volatile int*>(&g_device_error) != 0) break;
        __nanosleep(32);
      }
      if (!ok) set_device_error(kErrMbarTimeout);
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// Half of a 512-thread CTA (threads [256 * half, +256)): sum of v over the half, in the
// order of block_sum<256> (warp tree, then the half's eight warps in order).
__device__ __forceinline__ float half_sum(float v, float* red, int half) {
  v = warp_sum(v);
  const int warp = (threadIdx.x >> 5) & 7, lane = threadIdx.x & 31;
  if (lane == 0) red[half * 8 + warp] = v;
  asm volatile("bar.sync %0, 256;" ::"r"(1 + half) : "memory");
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += red[half * 8 + i];
  return s;
}

__global__ __cluster_dims__(kRcCtas, 1, 1) __launch_bounds__(kRcThreads) void router_fused_kernel(
    const RouterParams p) {
  // B0 of the first group: every CTA of the cluster has started (its shared memory
  // exists) before any CTA stores into it
  cluster_arrive_relaxed();
  constexpr int XS = kRtMaxHidden + 8;
  __shared__ __align__(16) bf16 s_x[kRtTok][XS];
  __shared__ float s_part[kRcKParts][kRcExperts][kRtTok];
  __shared__ float s_logits[kRtTok][kMaxExperts];
  __shared__ float s_red[16];
  const uint32_t crank = cluster_ctarank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int eA = static_cast<int>(crank) * kRcExperts + gq, eB = eA + 8;
  const bool okA = eA < p.n_experts, okB = eB < p.n_experts;
  const int nkb = p.hidden / 32;
  const int kb_beg = warp * nkb / kRcKParts, kb_end = (warp + 1) * nkb / kRcKParts;
  const bf16* w = reinterpret_cast<const bf16*>(p.w);
  const bf16* wA = w + static_cast<long long>(okA ? eA : 0) * p.hidden + tq * 8;
  const bf16* wB = w + static_cast<long long>(okB ? eB : 0) * p.hidden + tq * 8;
  uint4 a[kRcKb], b[kRcKb];
#pragma unroll
  for (int u = 0; u < kRcKb; ++u) {
    const int kb = kb_beg + u;
    a[u] = (kb < kb_end && okA) ? *reinterpret_cast<const uint4*>(wA + kb * 32) : make_uint4(0, 0, 0, 0);
    b[u] = (kb < kb_end && okB) ? *reinterpret_cast<const uint4*>(wB + kb * 32) : make_uint4(0, 0, 0, 0);
  }
  pdl_wait();
  const bool bucket = p.group_offsets != nullptr;
  if (!bucket) pdl_launch_dependents();
  // one row on one rank with every expert local and no gather: its bucketing is a few
  // ballots in the warp that ranks it (no grid barrier, no second pass over the ids)
  const bool one_row = bucket && p.rows == 1 && gridDim.x == kRcCtas && !p.gather_x && p.expert_lo == 0 &&
                       p.n_local == p.n_experts && p.shared_lo == 0 && p.shared_hi == 1;
  const int nch = p.hidden / 8;
  const int n_groups_tok = (p.rows + kRtTok - 1) / kRtTok;
  for (int grp = static_cast<int>(cluster_id_x()); grp < n_groups_tok; grp += static_cast<int>(n_clusters_x())) {
    const int row0 = grp * kRtTok;
    const int nt = min(kRtTok, p.rows - row0);
    cluster_wait_acquire();   // B0: the cluster is done with the previous group's s_x / s_logits
    if (p.h) {
      // residual add + RMSNorm of tokens 2r, 2r + 1 (one half each); x to all four CTAs
      const int half = tid >> 8, ht = tid & 255;
      const int t = 2 * static_cast<int>(crank) + half;
      if (t < nt) {
        const int row = row0 + t;
        bf16* hr = p.h + static_cast<long long>(row) * p.hidden;
        float v[8];
        float ss = 0.f;
        const int c = ht;
        if (c < nch) {
          const uint4 u = *reinterpret_cast<const uint4*>(hr + c * 8);
          const uint32_t* up = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            v[2 * j] = bf16lo(up[j]);
            v[2 * j + 1] = bf16hi(up[j]);
          }
          if (p.n_delta > 0) {
            float d[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) d[j] = 0.f;
            if (p.delta_dtype == 2) {
              const float* dp = reinterpret_cast<const float*>(p.delta) + row * p.delta_row_stride + c * 8;
              sum_parts8(dp, p.delta_part_stride, p.n_delta, d, true);
            } else {
              const bf16* dp = reinterpret_cast<const bf16*>(p.delta) + row * p.delta_row_stride + c * 8;
              for (int q = 0; q < p.n_delta; ++q) {
                const uint4 dv = *reinterpret_cast<const uint4*>(dp + q * p.delta_part_stride);
                const uint32_t* ap = reinterpret_cast<const uint32_t*>(&dv);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  d[2 * j] += bf16lo(ap[j]);
                  d[2 * j + 1] += bf16hi(ap[j]);
                }
              }
            }
            uint4 o;
            uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              op[j] = pack_bf16x2(v[2 * j] + d[2 * j], v[2 * j + 1] + d[2 * j + 1]);
              v[2 * j] = bf16lo(op[j]);
              v[2 * j + 1] = bf16hi(op[j]);
            }
            *reinterpret_cast<uint4*>(hr + c * 8) = o;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
        }
        ss = half_sum(ss, s_red, half);
        const float inv = rsqrtf(ss / static_cast<float>(p.hidden) + p.eps);
        if (c < nch) {
          uint4 o;
          uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float x0 = v[2 * j] * inv * load_w(p.norm_w, p.norm_w_dtype, c * 8 + 2 * j);
            const float x1 = v[2 * j + 1] * inv * load_w(p.norm_w, p.norm_w_dtype, c * 8 + 2 * j + 1);
            op[j] = pack_bf16x2(x0, x1);
          }
          *reinterpret_cast<uint4*>(p.x_out + static_cast<long long>(row) * p.x_row_stride + c * 8) = o;
#pragma unroll
          for (uint32_t r = 0; r < kRcCtas; ++r) st_cluster_v4(&s_x[t][c * 8], r, o);
        }
      }
    } else {
      for (int i = tid; i < kRtTok * nch; i += kRcThreads) {
        const int t = i / nch, c = i % nch;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (t < nt) v = *reinterpret_cast<const uint4*>(p.x + (row0 + t) * p.x_row_stride + c * 8);
        *reinterpret_cast<uint4*>(&s_x[t][c * 8]) = v;
      }
    }
    cluster_arrive_release();  // B1: s_x complete in every CTA
    cluster_wait_acquire();
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    const bf16* xr = &s_x[gq][tq * 8];
#pragma unroll
    for (int u = 0; u < kRcKb; ++u) {
      const int kb = kb_beg + u;
      if (kb >= kb_end) break;
      const uint4 xv = *reinterpret_cast<const uint4*>(xr + kb * 32);
      const uint32_t a0[4] = {a[u].x, b[u].x, a[u].y, b[u].y};
      mma_bf16_16816(c, a0, xv.x, xv.y);
      const uint32_t a1[4] = {a[u].z, b[u].z, a[u].w, b[u].w};
      mma_bf16_16816(c, a1, xv.z, xv.w);
    }
    s_part[warp][gq][2 * tq] = c[0];
    s_part[warp][gq][2 * tq + 1] = c[1];
    s_part[warp][gq + 8][2 * tq] = c[2];
    s_part[warp][gq + 8][2 * tq + 1] = c[3];
    __syncthreads();
    if (tid < kRcExperts * kRtTok) {
      const int el = tid / kRtTok, t = tid % kRtTok;
      const int e = static_cast<int>(crank) * kRcExperts + el;
      if (e < p.n_experts && t < nt) {
        float v = s_part[0][el][t];
#pragma unroll
        for (int q = 1; q < kRcKParts; ++q) v += s_part[q][el][t];
        if (p.bias) v += p.bias[e];
        p.logits[(row0 + t) * p.n_experts + e] = v;
        st_cluster_f32(&s_logits[t][e], 0, v);
      }
    }
    cluster_arrive_release();  // B2: CTA 0 sees every CTA's logits
    cluster_wait_acquire();
    if (crank == 0 && warp < nt) {
      const TopkLane tl = softmax_topk_warp(s_logits[warp], p.n_experts, p.scaling, row0 + warp, p.topk_ids,
                                            p.topk_ids32, p.topk_w);
      if (one_row) bucket_one_row_warp(p, tl);
    }
    cluster_arrive_release();  // B0 of the next group (or of the exit)
  }
  cluster_wait_acquire();      // no CTA leaves while another may still store into it
  if (!bucket) return;
  if (one_row) {               // bucketed above by the warp that ranked the row
    pdl_launch_dependents();
    return;
  }
  // a grid of one cluster (up to 8 tokens) meets at a cluster barrier instead of the
  // global-memory one
  bool ok = true;
  if (gridDim.x == kRcCtas) {
    cluster_arrive_release();
    cluster_wait_acquire();
  } else {
    ok = grid_barrier(p.grid_sync);
  }
  pdl_launch_dependents();
  if (!ok) return;
  RouteParams q = {};
  q.ids32 = p.topk_ids32;
  q.tw = p.topk_w;
  q.rows = p.rows;
  q.expert_lo = p.expert_lo;
  q.n_local = p.n_local;
  q.shared_lo = p.shared_lo;
  q.shared_hi = p.shared_hi;
  q.group_offsets = p.group_offsets;
  q.route_token = p.route_token;
  q.route_slot = p.route_slot;
  q.route_weight = p.route_weight;
  q.gx = p.gather_x ? (p.h ? p.x_out : p.x) : nullptr;
  q.gx_stride = p.x_row_stride;
  q.gout = p.gather_x ? reinterpret_cast<bf16*>(p.gather_out) : nullptr;
  q.cols = p.hidden;
  q.tok_per_cta = (p.rows + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
  route_cta<kRcThreads>(q, blockIdx.x);
}

// Softmax/top-6 over precomputed logits (the reference's router_softmax_topk6_triton).
__global__ void softmax_topk_kernel(const float* logits, int rows, int n_experts, float scaling,
                                    long long* ids64, int* ids32, float* tw) {
  pdl_enter();
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  softmax_topk_warp(logits + static_cast<long long>(row) * n_experts, n_experts, scaling, row,
                    ids64, ids32, tw);
}

// x_sorted[r] = x[route_token[r]] for r < group_offsets[n_groups]
__global__ void gather_rows_kernel(const bf16* __restrict__ x, long long x_row_stride,
                                   const int* __restrict__ route_token,
                                   const int* __restrict__ group_offsets, int n_groups,
                                   bf16* __restrict__ out, int cols, int max_routes) {
  pdl_enter();
  const int r = blockIdx.x;
  if (r >= max_routes || r >= group_offsets[n_groups]) return;
  const int t = route_token[r];
  const uint4* src = reinterpret_cast<const uint4*>(x + t * x_row_stride);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<long long>(r) * cols);
  for (int c = threadIdx.x; c < cols / 8; c += blockDim.x) dst[c] = src[c];
}

static cudaError_t launch_route(const int* ids32, const float* tw, int rows, int expert_lo,
                                int n_local, int shared_lo, int shared_hi, int* go, int* rt,
                                int* rs, float* rw, const bf16* gx, long long gxs, bf16* gout,
                                int cols, int num_sms, cudaStream_t st, const PeerTable* peers = nullptr,
                                int layer = 0) {
  RouteParams q = {};
  if (peers) q.peers = *peers;
  q.layer = layer;
  q.ids32 = ids32;
  q.tw = tw;
  q.rows = rows;
  q.expert_lo = expert_lo;
  q.n_local = n_local;
  q.shared_lo = shared_lo;
  q.shared_hi = shared_hi;
  q.group_offsets = go;
  q.route_token = rt;
  q.route_slot = rs;
  q.route_weight = rw;
  q.gx = gx;
  q.gx_stride = gxs;
  q.gout = gout;
  q.cols = cols;
  // about one CTA per SM (the counting pass is repeated by every CTA; the placement and
  // the row copies are split between them)
  q.tok_per_cta = min(kRouteTokMax, max(1, (rows + num_sms - 1) / max(num_sms, 1)));
  launch_kernel(route_kernel, (rows + q.tok_per_cta - 1) / q.tok_per_cta, kRouteThreads, 0, st, q);
  return cudaGetLastError();
}

// Clusters of router_fused_kernel that can be resident at once on the current device
// (the grid bound of its single-launch bucketing).
cudaError_t router_fused_max_clusters(int* n) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kRcCtas * 64);
  cfg.blockDim = dim3(kRcThreads);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kRcCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaOccupancyMaxActiveClusters(n, router_fused_kernel, &cfg);
}

// One rank, bf16 gate: router_fused_kernel, with the bucketing inside when a grid-barrier
// buffer is given and the whole grid fits (else a second launch, route_kernel).  fp32 gate
// or expert-parallel dispatch: router_topk_kernel (+ route_kernel).
cudaError_t launch_router(const RouterParams& p, int max_clusters, int num_sms, cudaStream_t st) {
  const int groups = (p.rows + kRtTok - 1) / kRtTok;
  bool second_route = p.group_offsets != nullptr;
  if (p.w_dtype == 0 && p.peers.world == 0) {
    RouterParams q = p;
    int clusters = groups;
    const int need = (p.rows + kRcCtas * kRouteTokMax - 1) / (kRcCtas * kRouteTokMax);
    if (p.group_offsets && p.grid_sync && max_clusters >= need) {
      clusters = std::min(groups, max_clusters);
      second_route = false;
    } else {
      q.group_offsets = nullptr;
    }
    launch_kernel(router_fused_kernel, clusters * kRcCtas, kRcThreads, 0, st, q);
  } else {
    launch_kernel(router_topk_kernel, groups, kRtThreads, 0, st, p);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !second_route) return e;
  return launch_route(p.topk_ids32, p.topk_w, p.rows, p.expert_lo, p.n_local, p.shared_lo,
                      p.shared_hi, p.group_offsets, p.route_token, p.route_slot, p.route_weight,
                      p.gather_x ? (p.h ? p.x_out : p.x) : nullptr, p.x_row_stride,
                      reinterpret_cast<bf16*>(p.gather_out), p.hidden, num_sms, st);
}

cudaError_t launch_bucket(const int* ids32, const float* tw, int rows, int expert_lo, int n_local,
                          int shared_lo, int shared_hi, int* go, int* rt, int* rs, float* rw,
                          const void* gx, long long gxs, void* gout, int cols, int num_sms, cudaStream_t st,
                          const PeerTable* peers, int layer) {
  return launch_route(ids32, tw, rows, expert_lo, n_local, shared_lo, shared_hi, go, rt, rs, rw,
                      reinterpret_cast<const bf16*>(gx), gxs, reinterpret_cast<bf16*>(gout), cols, num_sms,
                      st, peers, layer);
}

cudaError_t launch_softmax_topk(const float* logits, int rows, int n_experts, float scaling,
                                long long* ids64, int* ids32, float* tw, cudaStream_t st) {
  const int warps = 4;
  launch_kernel(softmax_topk_kernel, (rows + warps - 1) / warps, warps * 32, 0, st, logits, rows, n_experts, scaling, ids64, ids32, tw);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const void* x, long long xs, const int* rt, const int* go,
                               int n_groups, void* out, int cols, int max_routes, cudaStream_t st) {
  if (max_routes <= 0) return cudaSuccess;
  launch_kernel(gather_rows_kernel, max_routes, 128, 0, st, reinterpret_cast<const bf16*>(x), xs, rt, go, n_groups, reinterpret_cast<bf16*>(out), cols, max_routes);
  return cudaGetLastError();
}

}  // namespace dsv2
