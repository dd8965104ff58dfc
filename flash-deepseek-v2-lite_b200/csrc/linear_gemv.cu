// "Small" kernel family: weight-streaming GEMV for up to 8 tokens per pass.
//
// Replaces the reference's GEMV-style Triton kernels:
//   attention_decode_small.py:54-137   _gemv_contig_kernel / _gemv_2048x2048_o_kernel (B = 1)
//   attention_decode_small.py:857-901  _small_batch_gemv_kernel (B >= 2, one row per program)
//   moe_small_gemv.py:52-158, 194-307  per-route gate/up + SwiGLU and down GEMVs
// Design: each CTA owns 16 weight rows (plus the 16 matching "up" rows for SwiGLU)
// and one chunk of <= 8 tokens.  Its 8 warps split K; every lane streams 16-byte
// weight chunks straight from HBM (no L1 allocation) and feeds them to
// mma.sync.m16n8k16 with the tokens as the 8-wide N dimension.  The k order inside
// each 32-wide block is permuted identically for weights and activations, so a
// 16-byte load maps directly onto the A/B fragments without shuffles.  Partial
// sums of the 8 warps are reduced through shared memory and the epilogue (bf16 /
// fp32 store, SwiGLU, route-weight scaling) is fused.
//
// Routed (MoE) mode: group g owns routes [group_offsets[g], group_offsets[g+1]),
// read on the device, so the launch grid is fixed by host-side upper bounds and the
// kernel is CUDA-graph safe.  Unlike the reference's route-GEMV, tokens routed to
// the same expert share one pass over the expert's weights (up to 8 at a time).
#include <algorithm>

#include "linear.cuh"

namespace dsv2 {

constexpr int kGemvWarps = 8;
constexpr int kGemvRows = 16;
constexpr int kGemvTok = 8;
constexpr int kGemvMaxParts = 160;   // merged partials (one per attention CTA)

// Merge weights of the unmerged attention partials of head g (warp-wide, into wt[0, n)):
// a_c = 2^(m_c - M) / sum_c 2^(m_c - M) l_c over the partials with l_c > 0, the latent
// attention's own merge rule.  ml[i] / ll[i]: (m, l) of partial lane + 32 i, loaded by the
// caller.
constexpr int kGemvMlPerLane = (kGemvMaxParts + 31) / 32;
__device__ __forceinline__ void gemv_part_weights(int n, const float (&ml)[kGemvMlPerLane],
                                                  const float (&ll)[kGemvMlPerLane], float* wt, int lane) {
  float M = -INFINITY;
#pragma unroll
  for (int i = 0; i < kGemvMlPerLane; ++i)
    if (lane + 32 * i < n && ll[i] > 0.f) M = fmaxf(M, ml[i]);
  M = warp_max(M);
  float w[kGemvMlPerLane];
  float den = 0.f;
#pragma unroll
  for (int i = 0; i < kGemvMlPerLane; ++i) {
    w[i] = (lane + 32 * i < n && ll[i] > 0.f) ? exp2f(ml[i] - M) : 0.f;
    den += w[i] * ll[i];
  }
  den = warp_sum(den);
  const float inv = den > 0.f ? 1.f / den : 0.f;
#pragma unroll
  for (int i = 0; i < kGemvMlPerLane; ++i)
    if (lane + 32 * i < n) wt[lane + 32 * i] = w[i] * inv;
  __syncwarp();
}

// Index of the k-th group (in order) that holds at least one route, or -1.  Every warp
// of the CTA computes it from the device-side offsets (at most a few hundred groups).
__device__ __forceinline__ int kth_routed_group(const int* go, int G, int k) {
  const int lane = threadIdx.x & 31;
  int seen = 0;
  for (int base = 0; base < G; base += 32) {
    const int g = base + lane;
    const bool hit = g < G && go[g + 1] > go[g];
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    const int c = __popc(m);
    if (seen + c > k) return base + static_cast<int>(__fns(m, 0, k - seen + 1));
    seen += c;
  }
  return -1;
}

// XP: activations merged from unmerged attention partials (p.x_parts; its own instance, so
// that the registers of that path do not cut the occupancy of the others)
template <bool SWIGLU, int U, bool XP = false>
__global__ __launch_bounds__(kGemvWarps * 32) void gemv_mma_kernel(const LinearParams p,
                                                                    int rb_count, int tc_count) {
  // Dense launches, and grouped ones whose routing is older than the previous launch
  // (offsets_prior), request their first weight chunks before waiting for the previous
  // kernel; the activations are loaded after the wait.
  const bool early = p.group_offsets == nullptr || p.offsets_prior;
  bool waited = !early;
  if (!early) pdl_enter();
  __shared__ float red[kGemvWarps][32][SWIGLU ? 8 : 4];
  __shared__ unsigned long long s_key[kGemvRows * kGemvTok];  // arg-max epilogue only
  __shared__ float s_wt[kGemvWarps][XP ? kGemvMaxParts : 1];  // x_parts merge weights, per warp
  int n_parts = -1, part_c0 = 0;
  bool have_wt = false;
  int item = blockIdx.x;
  const int tc = item % tc_count;
  item /= tc_count;
  const int rb = item % rb_count;
  // grouped launches cover the groups that hold routes, in order (item / rb_count-th of them)
  const int g = p.group_offsets ? kth_routed_group(p.group_offsets, p.n_groups, item / rb_count) : item / rb_count;

  int r0, cnt;
  if (p.group_offsets) {
    if (g < 0) {
      if (!waited) pdl_enter();
      return;
    }
    r0 = p.group_offsets[g];
    cnt = p.group_offsets[g + 1] - r0;
  } else {
    r0 = 0;
    cnt = p.n_tokens;
  }
  const int tbeg = tc * kGemvTok;
  if (tbeg >= cnt) {
    if (!waited) pdl_enter();
    return;
  }
  const int tn = min(kGemvTok, cnt - tbeg);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int n0 = rb * kGemvRows;
  const int rowA = n0 + gq, rowB = n0 + gq + 8;
  const bool okA = rowA < p.n_rows, okB = rowB < p.n_rows;
  const bf16* wg = p.w + g * p.w_group_stride;
  const bf16* wA = wg + static_cast<long long>(okA ? rowA : 0) * p.w_row_stride + tq * 8;
  const bf16* wB = wg + static_cast<long long>(okB ? rowB : 0) * p.w_row_stride + tq * 8;

  // activation row for token gq of this chunk (B operand column gq)
  const bool okT = gq < tn;
  const int rtok = r0 + tbeg + (okT ? gq : 0);
  const int xrow = p.route_x_row ? p.route_x_row[rtok] : rtok;
  const bf16* xp = p.x + g * p.x_group_stride + static_cast<long long>(xrow) * p.x_row_stride + tq * 8;

  float c[4] = {0.f, 0.f, 0.f, 0.f};
  float cu[4] = {0.f, 0.f, 0.f, 0.f};
  const int nkb = p.k / 32;
  for (int kb0 = warp; kb0 < nkb; kb0 += kGemvWarps * U) {
    uint4 wa[U], wb[U], ua[U], ub[U], xv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int kb = kb0 + u * kGemvWarps;
      const uint4 z = make_uint4(0, 0, 0, 0);
      wa[u] = z; wb[u] = z; ua[u] = z; ub[u] = z; xv[u] = z;
      if (kb < nkb) {
        if (okA) wa[u] = ld_stream_v4(wA + kb * 32);
        if (okB) wb[u] = ld_stream_v4(wB + kb * 32);
        if (SWIGLU) {
          if (okA) ua[u] = ld_stream_v4(wA + p.up_offset + kb * 32);
          if (okB) ub[u] = ld_stream_v4(wB + p.up_offset + kb * 32);
        }
      }
    }
    if (!waited) {
      pdl_enter();
      waited = true;
    }
    if (XP) {
      // lane L merges element 32 kb + L of the row over the partials, then the lanes of token
      // 0 (gq == 0) gather their 8 consecutive elements as bf16 (the attention's o_lat).  The
      // first partials' values are requested together with the (m, l) pairs, before the
      // merge weights are known.
      constexpr int kPB = 4;   // partials per batch of loads
      if (n_parts < 0) {
        part_c0 = __ldcg(p.x_parts_count);
        n_parts = __ldcg(p.x_parts_count + 1);
        if (n_parts < 0 || n_parts > kGemvMaxParts || part_c0 < 0) {
          if (lane == 0) set_device_error(kErrIndex);
          n_parts = 0;
          part_c0 = 0;
        }
      }
      const long long ps = 2LL * p.n_groups * p.k;   // floats between consecutive partials
      const float* ob = p.x_parts + (static_cast<long long>(2 * part_c0) * p.n_groups + g) * p.k;
      float mv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) mv[u] = 0.f;
      for (int s0 = 0; s0 < n_parts; s0 += kPB) {
        float v[kPB][U];
#pragma unroll
        for (int q = 0; q < kPB; ++q)
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int kb = kb0 + u * kGemvWarps;
            v[q][u] = (kb < nkb && s0 + q < n_parts) ? __ldcg(ob + (s0 + q) * ps + kb * 32 + lane) : 0.f;
          }
        if (!have_wt) {
          float ml[kGemvMlPerLane], ll[kGemvMlPerLane];
#pragma unroll
          for (int i = 0; i < kGemvMlPerLane; ++i) {
            const int s = lane + 32 * i;
            const float* mp = p.x_parts_ml + (static_cast<long long>(2 * (part_c0 + s)) * p.n_groups + g) * 2;
            ml[i] = s < n_parts ? __ldcg(mp) : 0.f;
            ll[i] = s < n_parts ? __ldcg(mp + 1) : 0.f;
          }
          gemv_part_weights(n_parts, ml, ll, s_wt[warp], lane);
          have_wt = true;
        }
#pragma unroll
        for (int q = 0; q < kPB; q += 2) {
          const float w0 = s0 + q < n_parts ? s_wt[warp][s0 + q] : 0.f;
          const float w1 = s0 + q + 1 < n_parts ? s_wt[warp][s0 + q + 1] : 0.f;
#pragma unroll
          for (int u = 0; u < U; ++u) mv[u] += w0 * v[q][u] + w1 * v[q + 1][u];
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        uint32_t qv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = __shfl_sync(0xffffffffu, mv[u], tq * 8 + 2 * j);
          const float b = __shfl_sync(0xffffffffu, mv[u], tq * 8 + 2 * j + 1);
          qv[j] = pack_bf16x2(a, b);
        }
        const int kb = kb0 + u * kGemvWarps;
        if (kb < nkb && okT) xv[u] = make_uint4(qv[0], qv[1], qv[2], qv[3]);
      }
    } else {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int kb = kb0 + u * kGemvWarps;
        if (kb < nkb && okT) xv[u] = *reinterpret_cast<const uint4*>(xp + kb * 32);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      {
        const uint32_t a0[4] = {wa[u].x, wb[u].x, wa[u].y, wb[u].y};
        mma_bf16_16816(c, a0, xv[u].x, xv[u].y);
        const uint32_t a1[4] = {wa[u].z, wb[u].z, wa[u].w, wb[u].w};
        mma_bf16_16816(c, a1, xv[u].z, xv[u].w);
      }
      if (SWIGLU) {
        const uint32_t a0[4] = {ua[u].x, ub[u].x, ua[u].y, ub[u].y};
        mma_bf16_16816(cu, a0, xv[u].x, xv[u].y);
        const uint32_t a1[4] = {ua[u].z, ub[u].z, ua[u].w, ub[u].w};
        mma_bf16_16816(cu, a1, xv[u].z, xv[u].w);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    red[warp][lane][i] = c[i];
    if (SWIGLU) red[warp][lane][4 + i] = cu[i];
  }
  if (!waited) pdl_enter();  // warps without K blocks
  __syncthreads();
  // 128 output elements (16 rows x 8 tokens): thread i -> lane i/4, fragment slot i%4
  if (threadIdx.x < 128) {
    const int l = threadIdx.x >> 2, s = threadIdx.x & 3;
    float acc = 0.f, accu = 0.f;
#pragma unroll
    for (int w = 0; w < kGemvWarps; ++w) {
      acc += red[w][l][s];
      if (SWIGLU) accu += red[w][l][4 + s];
    }
    const int n = n0 + (l >> 2) + ((s & 2) ? 8 : 0);
    const int j = 2 * (l & 3) + (s & 1);
    if (p.epilogue == kEpiArgmax) {
      s_key[(n - n0) * kGemvTok + j] = (n < p.n_rows) ? argmax_key(argmax_ord(acc), n) : 0ull;
    } else if (j < tn && n < p.n_rows) {
      linear_store(p, g, r0 + tbeg + j, n, acc, accu);
    }
  }
  if (p.epilogue == kEpiArgmax) {
    // one key per (16-row block, token): the block's largest value, lowest row on ties
    __syncthreads();
    if (threadIdx.x < tn) {
      unsigned long long best = 0;
#pragma unroll
      for (int r = 0; r < kGemvRows; ++r) best = max(best, s_key[r * kGemvTok + threadIdx.x]);
      reinterpret_cast<unsigned long long*>(p.y)[static_cast<long long>(rb) * p.y_row_stride + tbeg +
                                                 threadIdx.x] = best;
    }
  }
}

// Short K (at most 8 blocks of 32, e.g. the absorbed-query GEMV, K = 128): splitting K over
// eight warps would leave most of them idle and still pay the cross-warp reduction, so here
// each warp owns 16 weight rows and the whole K (4 warps, 64 rows per CTA): all of its weight
// chunks are requested before the launch wait, its activations after it, and the mma.sync
// fragment goes straight to the epilogue.
constexpr int kShortWarps = 4;
constexpr int kShortMaxKb = 8;

__global__ __launch_bounds__(kShortWarps * 32) void gemv_short_k_kernel(const LinearParams p, int rb_count,
                                                                         int tc_count) {
  int item = blockIdx.x;
  const int tc = item % tc_count;
  item /= tc_count;
  const int rb = item % rb_count;
  const int g = item / rb_count;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int n0 = (rb * kShortWarps + warp) * kGemvRows;
  const int rowA = n0 + gq, rowB = n0 + gq + 8;
  const bool okA = rowA < p.n_rows, okB = rowB < p.n_rows;
  const bf16* wg = p.w + g * p.w_group_stride;
  const bf16* wA = wg + static_cast<long long>(okA ? rowA : 0) * p.w_row_stride + tq * 8;
  const bf16* wB = wg + static_cast<long long>(okB ? rowB : 0) * p.w_row_stride + tq * 8;
  const int nkb = p.k / 32;
  uint4 wa[kShortMaxKb], wb[kShortMaxKb], xv[kShortMaxKb];
#pragma unroll
  for (int u = 0; u < kShortMaxKb; ++u) {
    const uint4 z = make_uint4(0, 0, 0, 0);
    wa[u] = z; wb[u] = z; xv[u] = z;
    if (u < nkb) {
      if (okA) wa[u] = ld_stream_v4(wA + u * 32);
      if (okB) wb[u] = ld_stream_v4(wB + u * 32);
    }
  }
  pdl_enter();
  const int tbeg = tc * kGemvTok;
  const int tn = min(kGemvTok, p.n_tokens - tbeg);
  const bool okT = gq < tn;
  const bf16* xp = p.x + g * p.x_group_stride + static_cast<long long>(tbeg + (okT ? gq : 0)) * p.x_row_stride + tq * 8;
#pragma unroll
  for (int u = 0; u < kShortMaxKb; ++u)
    if (u < nkb && okT) xv[u] = *reinterpret_cast<const uint4*>(xp + u * 32);
  float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int u = 0; u < kShortMaxKb; ++u) {
    if (u < nkb) {
      const uint32_t a0[4] = {wa[u].x, wb[u].x, wa[u].y, wb[u].y};
      mma_bf16_16816(c, a0, xv[u].x, xv[u].y);
      const uint32_t a1[4] = {wa[u].z, wb[u].z, wa[u].w, wb[u].w};
      mma_bf16_16816(c, a1, xv[u].z, xv[u].w);
    }
  }
  // fragment element i: row gq (+8 for i >= 2), token 2 tq + (i & 1)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int n = n0 + gq + ((i & 2) ? 8 : 0);
    const int j = 2 * tq + (i & 1);
    if (j < tn && n < p.n_rows) linear_store(p, g, tbeg + j, n, c[i], 0.f);
  }
}

cudaError_t launch_linear_gemv(const LinearParams& p, cudaStream_t st) {
  if (!p.group_offsets && !p.x_parts && p.k <= 32 * kShortMaxKb && p.n_tokens > 0 &&
      (p.epilogue == kEpiStoreBf16 || p.epilogue == kEpiStoreF32)) {
    const int rb_count = (p.n_rows + kShortWarps * kGemvRows - 1) / (kShortWarps * kGemvRows);
    const int tc_count = (p.n_tokens + kGemvTok - 1) / kGemvTok;
    const long long items = static_cast<long long>(p.n_groups) * rb_count * tc_count;
    if (items <= 0) return cudaSuccess;
    if (items > 0x7fffffffLL) return cudaErrorInvalidValue;
    launch_kernel(gemv_short_k_kernel, dim3(static_cast<unsigned>(items)), kShortWarps * 32, 0, st, p, rb_count,
                  tc_count);
    return cudaGetLastError();
  }
  const int rb_count = (p.n_rows + kGemvRows - 1) / kGemvRows;
  const int max_tok = p.group_offsets ? p.max_routes_per_group : p.n_tokens;
  const int tc_count = max(1, (max_tok + kGemvTok - 1) / kGemvTok);
  const int groups = p.group_offsets ? std::max(1, std::min(p.n_groups, p.active_groups)) : p.n_groups;
  const long long items = static_cast<long long>(groups) * rb_count * tc_count;
  if (items <= 0) return cudaSuccess;
  if (items > 0x7fffffffLL) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(items));
  if (p.x_parts) {
    if (p.epilogue == kEpiSwiglu || p.n_tokens != 1) return cudaErrorInvalidValue;
    launch_kernel(gemv_mma_kernel<false, 2, true>, grid, kGemvWarps * 32, 0, st, p, rb_count, tc_count);
  } else if (p.epilogue == kEpiSwiglu) {
    launch_kernel(gemv_mma_kernel<true, 4>, grid, kGemvWarps * 32, 0, st, p, rb_count, tc_count);
  } else {
    launch_kernel(gemv_mma_kernel<false, 8>, grid, kGemvWarps * 32, 0, st, p, rb_count, tc_count);
  }
  return cudaGetLastError();
}

}  // namespace dsv2
