// Fused MoE router: fp32 gate GEMV + softmax + top-6 + token-to-expert bucketing.
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
// Bucketing is a stable counting sort: routes are ranked inside each warp with
// __match_any_sync + popc and across warps with a per-expert scan, so the route
// order inside every expert bucket is ascending in (token, k) and identical from
// run to run.  Two extra "shared" groups carry every local token with weight 1,
// which lets the MoE kernels run the two shared experts in the same launch as
// the routed ones.  The bucketing stage runs in the last CTA to finish (atomic
// ticket), so routing plus bucketing is one launch.
#include "params.cuh"

namespace dsv2 {

constexpr int kRouterThreads = 256;
constexpr int kTopK = 6;
constexpr int kMaxExperts = 64;
constexpr int kSlots = 8;  // 6 routed + 2 shared-expert halves per token


__device__ __forceinline__ float load_gate_w(const void* w, int dt, long long i) {
  return dt == 2 ? reinterpret_cast<const float*>(w)[i]
                 : __bfloat162float(reinterpret_cast<const bf16*>(w)[i]);
}

// softmax + top-6 for one token with one warp; logits in shared/global memory.
__device__ void softmax_topk_warp(const float* lg, int n_experts, float scaling, int row,
                                  long long* ids64, int* ids32, float* tw) {
  const int lane = threadIdx.x & 31;
  float v0 = lane < n_experts ? lg[lane] : -INFINITY;
  float v1 = lane + 32 < n_experts ? lg[lane + 32] : -INFINITY;
  const float m = warp_max(fmaxf(v0, v1));
  float e0 = lane < n_experts ? expf(v0 - m) : 0.f;
  float e1 = lane + 32 < n_experts ? expf(v1 - m) : 0.f;
  const float s = warp_sum(e0 + e1);
  float p0 = lane < n_experts ? e0 / s : -INFINITY;
  float p1 = lane + 32 < n_experts ? e1 / s : -INFINITY;
  for (int k = 0; k < kTopK; ++k) {
    // best value, lowest index on ties
    float bv;
    int bi;
    if (p1 > p0) { bv = p1; bi = lane + 32; } else { bv = p0; bi = lane; }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) {
      if (ids64) ids64[row * kTopK + k] = bi;
      ids32[row * kTopK + k] = bi;
      tw[row * kTopK + k] = bv * scaling;
    }
    if (bi == lane) p0 = -INFINITY;
    if (bi == lane + 32) p1 = -INFINITY;
  }
}

// Stable bucketing of all routes by local expert (+ the two shared groups).
// Must be called by every thread of one CTA (blockDim.x == kRouterThreads).
__device__ void bucket_routes(const int* ids32, const float* tw, int rows, int expert_lo,
                              int n_local, int shared_lo, int shared_hi, int* group_offsets,
                              int* route_token, int* route_slot, float* route_weight) {
  constexpr int NW = kRouterThreads / 32;
  __shared__ int s_cnt[kMaxExperts];
  __shared__ int s_off[kMaxExperts + 3];
  __shared__ int s_run[kMaxExperts];
  __shared__ int s_wh[NW][kMaxExperts];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < kMaxExperts; i += kRouterThreads) { s_cnt[i] = 0; s_run[i] = 0; }
  __syncthreads();
  const int n_routes = rows * kTopK;
  for (int r = tid; r < n_routes; r += kRouterThreads) {
    const int e = __ldcg(ids32 + r) - expert_lo;
    if (e >= 0 && e < n_local) atomicAdd(&s_cnt[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < n_local; ++e) { s_off[e] = acc; acc += s_cnt[e]; }
    const int nsh = shared_hi - shared_lo;
    s_off[n_local] = acc;
    s_off[n_local + 1] = acc + nsh;
    s_off[n_local + 2] = acc + 2 * nsh;
    for (int e = 0; e <= n_local + 2; ++e) group_offsets[e] = s_off[e];
  }
  __syncthreads();
  for (int base = 0; base < n_routes; base += kRouterThreads) {
    const int r = base + tid;
    int key = -1;
    if (r < n_routes) {
      const int e = __ldcg(ids32 + r) - expert_lo;
      if (e >= 0 && e < n_local) key = e;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    for (int i = tid; i < NW * kMaxExperts; i += kRouterThreads) (&s_wh[0][0])[i] = 0;
    __syncthreads();
    if (key >= 0 && rank == 0) s_wh[warp][key] = __popc(peers);
    __syncthreads();
    // exclusive scan over warps per expert; the chunk total goes to s_run afterwards
    if (tid < n_local) {
      int acc = 0;
      for (int w = 0; w < NW; ++w) { const int c = s_wh[w][tid]; s_wh[w][tid] = acc; acc += c; }
      s_cnt[tid] = acc;  // reuse as chunk total
    }
    __syncthreads();
    if (key >= 0) {
      const int pos = s_off[key] + s_run[key] + s_wh[warp][key] + rank;
      const int b = r / kTopK, k = r % kTopK;
      route_token[pos] = b;
      route_slot[pos] = b * kSlots + k;
      route_weight[pos] = __ldcg(tw + r);
    }
    __syncthreads();
    if (tid < n_local) s_run[tid] += s_cnt[tid];
    __syncthreads();
  }
  // shared-expert groups: every local row, weight 1
  const int nsh = shared_hi - shared_lo;
  for (int i = tid; i < 2 * nsh; i += kRouterThreads) {
    const int s = i / nsh, b = shared_lo + (i % nsh);
    const int pos = s_off[n_local + s] + (i % nsh);
    route_token[pos] = b;
    route_slot[pos] = b * kSlots + kTopK + s;
    route_weight[pos] = 1.f;
  }
}

__global__ __launch_bounds__(kRouterThreads) void router_kernel(const RouterParams p) {
  __shared__ float s_logits[kMaxExperts];
  __shared__ bool s_last;
  const int row = blockIdx.x;
  const int eg = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bf16* xr = p.x + row * p.x_row_stride;
  const int nch = p.hidden / 8;
  const int e_beg = eg * p.experts_per_cta;
  const int e_end = min(p.n_experts, e_beg + p.experts_per_cta);
  for (int e = e_beg + warp; e < e_end; e += kRouterThreads / 32) {
    float acc = 0.f;
    if (p.w_dtype == 0) {
      const bf16* wr = reinterpret_cast<const bf16*>(p.w) + static_cast<long long>(e) * p.hidden;
      for (int c = lane; c < nch; c += 32)
        acc = dot8(*reinterpret_cast<const uint4*>(xr + c * 8), *reinterpret_cast<const uint4*>(wr + c * 8), acc);
    } else {
      const float* wr = reinterpret_cast<const float*>(p.w) + static_cast<long long>(e) * p.hidden;
      for (int c = lane; c < nch; c += 32) {
        const uint4 u = *reinterpret_cast<const uint4*>(xr + c * 8);
        const uint32_t* up = reinterpret_cast<const uint32_t*>(&u);
        const float4 w0 = *reinterpret_cast<const float4*>(wr + c * 8);
        const float4 w1 = *reinterpret_cast<const float4*>(wr + c * 8 + 4);
        acc = fmaf(bf16lo(up[0]), w0.x, acc); acc = fmaf(bf16hi(up[0]), w0.y, acc);
        acc = fmaf(bf16lo(up[1]), w0.z, acc); acc = fmaf(bf16hi(up[1]), w0.w, acc);
        acc = fmaf(bf16lo(up[2]), w1.x, acc); acc = fmaf(bf16hi(up[2]), w1.y, acc);
        acc = fmaf(bf16lo(up[3]), w1.z, acc); acc = fmaf(bf16hi(up[3]), w1.w, acc);
      }
    }
    acc = warp_sum(acc);
    if (p.bias) acc += p.bias[e];
    if (lane == 0) {
      s_logits[e - e_beg] = acc;
      p.logits[row * p.n_experts + e] = acc;
    }
  }
  __syncthreads();
  const bool full = (p.experts_per_cta >= p.n_experts);
  if (full && warp == 0)
    softmax_topk_warp(s_logits, p.n_experts, p.scaling, row, p.topk_ids, p.topk_ids32, p.topk_w);
  if (full && p.group_offsets == nullptr) return;
  // ticket: the last CTA finishes top-k (when split) and bucketing
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned total = gridDim.x * gridDim.y;
    const unsigned t = atomicAdd(p.ticket, 1u);
    s_last = (t == total - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (!full) {
    for (int r = warp; r < p.rows; r += kRouterThreads / 32) {
      __shared__ float lg[kRouterThreads / 32][kMaxExperts];
      for (int e = lane; e < p.n_experts; e += 32) lg[warp][e] = __ldcg(p.logits + r * p.n_experts + e);
      __syncwarp();
      softmax_topk_warp(lg[warp], p.n_experts, p.scaling, r, p.topk_ids, p.topk_ids32, p.topk_w);
      __syncwarp();
    }
    __threadfence();
    __syncthreads();
  }
  if (p.group_offsets)
    bucket_routes(p.topk_ids32, p.topk_w, p.rows, p.expert_lo, p.n_local, p.shared_lo,
                  p.shared_hi, p.group_offsets, p.route_token, p.route_slot, p.route_weight);
  if (threadIdx.x == 0) *p.ticket = 0u;
}

// Standalone bucketing (expert parallel: runs after the all-gather of top-k results).
__global__ __launch_bounds__(kRouterThreads) void bucket_kernel(
    const int* ids32, const float* tw, int rows, int expert_lo, int n_local, int shared_lo,
    int shared_hi, int* group_offsets, int* route_token, int* route_slot, float* route_weight) {
  bucket_routes(ids32, tw, rows, expert_lo, n_local, shared_lo, shared_hi, group_offsets,
                route_token, route_slot, route_weight);
}

// Softmax/top-6 over precomputed logits (the reference's router_softmax_topk6_triton).
__global__ void softmax_topk_kernel(const float* logits, int rows, int n_experts, float scaling,
                                    long long* ids64, int* ids32, float* tw) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  softmax_topk_warp(logits + static_cast<long long>(row) * n_experts, n_experts, scaling, row,
                    ids64, ids32, tw);
}

// x_sorted[r] = x[route_token[r]] for r < group_offsets[n_groups]  (gathers the
// activations of every route into expert-contiguous rows for the TMA path)
__global__ void gather_rows_kernel(const bf16* __restrict__ x, long long x_row_stride,
                                   const int* __restrict__ route_token,
                                   const int* __restrict__ group_offsets, int n_groups,
                                   bf16* __restrict__ out, int cols, int max_routes) {
  const int r = blockIdx.x;
  if (r >= max_routes || r >= group_offsets[n_groups]) return;
  const int t = route_token[r];
  const uint4* src = reinterpret_cast<const uint4*>(x + t * x_row_stride);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<long long>(r) * cols);
  for (int c = threadIdx.x; c < cols / 8; c += blockDim.x) dst[c] = src[c];
}

cudaError_t launch_router(const RouterParams& p, cudaStream_t st) {
  const int eg = (p.n_experts + p.experts_per_cta - 1) / p.experts_per_cta;
  router_kernel<<<dim3(p.rows, eg), kRouterThreads, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_bucket(const int* ids32, const float* tw, int rows, int expert_lo, int n_local,
                          int shared_lo, int shared_hi, int* go, int* rt, int* rs, float* rw,
                          cudaStream_t st) {
  bucket_kernel<<<1, kRouterThreads, 0, st>>>(ids32, tw, rows, expert_lo, n_local, shared_lo,
                                               shared_hi, go, rt, rs, rw);
  return cudaGetLastError();
}

cudaError_t launch_softmax_topk(const float* logits, int rows, int n_experts, float scaling,
                                long long* ids64, int* ids32, float* tw, cudaStream_t st) {
  const int warps = 4;
  softmax_topk_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, st>>>(logits, rows, n_experts,
                                                                          scaling, ids64, ids32, tw);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const void* x, long long xs, const int* rt, const int* go,
                               int n_groups, void* out, int cols, int max_routes, cudaStream_t st) {
  if (max_routes <= 0) return cudaSuccess;
  gather_rows_kernel<<<max_routes, 128, 0, st>>>(reinterpret_cast<const bf16*>(x), xs, rt, go,
                                                 n_groups, reinterpret_cast<bf16*>(out), cols,
                                                 max_routes);
  return cudaGetLastError();
}

}  // namespace dsv2
