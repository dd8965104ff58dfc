// RMSNorm family, residual add, SwiGLU elementwise, decode-input preparation and
// single-token cache copies.
//
// Reference kernels these replace (Flash-DeepSeeek-V2-Lite, triton_kernels/):
//   rmsnorm.py:8-57            two-pass fp32 RMSNorm, output rounded once to the input dtype
//   attention_prepost.py:85-110 residual add in fp32 -> bf16
//   mlp_elementwise.py:8-21     silu(gate) * up in fp32 -> bf16
//   attention_prepost.py:8-36   attention_mask[b, s] = (s <= pos), position_ids[b] = pos
//   attention_prepost.py:39-82  cache[b, h, pos, :] = src[b, h, 0, :]
// The fused add_rmsnorm / embed_rmsnorm kernels merge the residual add that
// src/run.py:459-493 performs around every sublayer with the RMSNorm that follows it.
#include "params.cuh"

namespace dsv2 {

// y = bf16(x * rsqrt(mean(x^2) + eps) * w); one CTA per row, cols % 8 == 0.
// w_dtype: 0 bf16, 2 fp32.
template <int THREADS>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) s += red[i];
  __syncthreads();
  return s;
}

__device__ __forceinline__ float load_w(const void* w, int w_dtype, int i) {
  if (w_dtype == 2) return reinterpret_cast<const float*>(w)[i];
  if (w_dtype == 1) return __half2float(reinterpret_cast<const __half*>(w)[i]);
  return __bfloat162float(reinterpret_cast<const bf16*>(w)[i]);
}

// Eight consecutive 16-bit activations (bf16 or fp16) <-> fp32, for the kernels that take
// either (the reference's rmsnorm / residual add accept both, rmsnorm.py:64-65,
// attention_prepost.py:197-198).
template <typename T>
struct Act16;
template <>
struct Act16<bf16> {
  static __device__ __forceinline__ void unpack(const uint4& u, float (&v)[8]) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = bf16lo(p[j]);
      v[2 * j + 1] = bf16hi(p[j]);
    }
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) { return pack_bf16x2(a, b); }
};
template <>
struct Act16<__half> {
  static __device__ __forceinline__ void unpack(const uint4& u, float (&v)[8]) {
    const __half2* p = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __half22float2(p[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// Normalise the 8-element chunks held in v[] (fp32) and store them as T (bf16 or fp16).
template <int MAXCH, typename T = bf16>
__device__ __forceinline__ void norm_store(const float (&v)[MAXCH][8], int nch_mine, int chunk0,
                                           int chunk_step, float inv, const void* w, int w_dtype,
                                           T* y) {
#pragma unroll
  for (int i = 0; i < MAXCH; ++i) {
    if (i >= nch_mine) break;
    const int c = chunk0 + i * chunk_step;
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = v[i][2 * j] * inv * load_w(w, w_dtype, c * 8 + 2 * j);
      const float b = v[i][2 * j + 1] * inv * load_w(w, w_dtype, c * 8 + 2 * j + 1);
      op[j] = Act16<T>::pack2(a, b);
    }
    *reinterpret_cast<uint4*>(y + c * 8) = o;
  }
}

constexpr int kNormThreads = 256;
constexpr int kNormMaxCh = 2;  // up to 256 * 2 * 8 = 4096 columns

template <typename T>
__global__ __launch_bounds__(kNormThreads) void rmsnorm_kernel(const T* __restrict__ x,
                                                               long long x_stride,
                                                               const void* __restrict__ w,
                                                               int w_dtype, T* __restrict__ y,
                                                               long long y_stride, int cols,
                                                               float eps) {
  pdl_enter();
  __shared__ float red[kNormThreads / 32];
  const int row = blockIdx.x;
  const T* xr = x + row * x_stride;
  const int nch = cols / 8;
  float v[kNormMaxCh][8];
  float ss = 0.f;
  int mine = 0;
#pragma unroll
  for (int i = 0; i < kNormMaxCh; ++i) {
    const int c = threadIdx.x + i * kNormThreads;
    if (c < nch) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c * 8);
      Act16<T>::unpack(u, v[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) ss += v[i][2 * j] * v[i][2 * j] + v[i][2 * j + 1] * v[i][2 * j + 1];
      mine = i + 1;
    }
  }
  ss = block_sum<kNormThreads>(ss, red);
  const float inv = rsqrtf(ss / static_cast<float>(cols) + eps);
  norm_store<kNormMaxCh, T>(v, mine, threadIdx.x, kNormThreads, inv, w, w_dtype, y + row * y_stride);
}

// h[row] = bf16(h[row] + sum_p delta[row, p]); y[row] = rmsnorm(h[row]) * w.
// delta_dtype: 0 bf16 (row stride delta_row_stride), 2 fp32 partials laid out
// [rows][n_delta][cols] (part stride delta_part_stride).  n_delta == 0 means no add.
// When h_out != nullptr the sum is written there instead of in place.
// acc[0..7] += sum over p < n of src[p * stride + 0..7] (fp32), added in order of p.  The
// loads of eight partials are issued before their adds, so a thread keeps 16 independent
// 16-byte loads in flight instead of one round trip per partial (the MoE's eight slots
// and the split-K partials of the dense linears take one round).  l2_only: read through
// L2 only (partials written by another CTA of the previous launch).
__device__ __forceinline__ void sum_parts8(const float* src, long long stride, int n, float (&acc)[8],
                                           bool l2_only) {
  for (int p0 = 0; p0 < n; p0 += 8) {
    float4 a[8], b[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (p0 + q < n) {
        const float4* s = reinterpret_cast<const float4*>(src + (p0 + q) * stride);
        a[q] = l2_only ? __ldcg(s) : s[0];
        b[q] = l2_only ? __ldcg(s + 1) : s[1];
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (p0 + q < n) {
        acc[0] += a[q].x; acc[1] += a[q].y; acc[2] += a[q].z; acc[3] += a[q].w;
        acc[4] += b[q].x; acc[5] += b[q].y; acc[6] += b[q].z; acc[7] += b[q].w;
      }
    }
  }
}

__global__ __launch_bounds__(kNormThreads) void add_rmsnorm_kernel(
    bf16* __restrict__ h, bf16* __restrict__ h_out, const void* __restrict__ delta, int delta_dtype,
    int n_delta, long long delta_part_stride, long long delta_row_stride,
    const void* __restrict__ w, int w_dtype, bf16* __restrict__ y, int cols, float eps,
    const PeerTable peers, int layer) {
  pdl_enter();
  if (peers.world > 0) {
    // expert parallel: every rank has written its MoE slot outputs for these rows
    __shared__ int s_ok;
    if (threadIdx.x == 0)
      s_ok = wait_counter_sys(peer_ctr(peers, peers.rank, 1), peer_target(peers, layer, 1ull), peers.wait_polls,
                              peers.wait_stats ? peers.wait_stats + 2 : nullptr);
    __syncthreads();
    if (!s_ok) return;
  }
  __shared__ float red[kNormThreads / 32];
  const int row = blockIdx.x;
  bf16* hr = h + static_cast<long long>(row) * cols;
  bf16* ho = (h_out ? h_out : h) + static_cast<long long>(row) * cols;
  const int nch = cols / 8;
  float v[kNormMaxCh][8];
  float ss = 0.f;
  int mine = 0;
#pragma unroll
  for (int i = 0; i < kNormMaxCh; ++i) {
    const int c = threadIdx.x + i * kNormThreads;
    if (c < nch) {
      const uint4 u = *reinterpret_cast<const uint4*>(hr + c * 8);
      const uint32_t* up = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[i][2 * j] = bf16lo(up[j]);
        v[i][2 * j + 1] = bf16hi(up[j]);
      }
      if (n_delta > 0) {
        float d[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) d[j] = 0.f;
        if (delta_dtype == 2) {
          const float* dp = reinterpret_cast<const float*>(delta) + row * delta_row_stride + c * 8;
          sum_parts8(dp, delta_part_stride, n_delta, d, true);
        } else {
          const bf16* dp = reinterpret_cast<const bf16*>(delta) + row * delta_row_stride + c * 8;
          for (int p = 0; p < n_delta; ++p) {
            const uint4 a = *reinterpret_cast<const uint4*>(dp + p * delta_part_stride);
            const uint32_t* ap = reinterpret_cast<const uint32_t*>(&a);
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
          op[j] = pack_bf16x2(v[i][2 * j] + d[2 * j], v[i][2 * j + 1] + d[2 * j + 1]);
          v[i][2 * j] = bf16lo(op[j]);
          v[i][2 * j + 1] = bf16hi(op[j]);
        }
        *reinterpret_cast<uint4*>(ho + c * 8) = o;
      } else if (h_out) {
        *reinterpret_cast<uint4*>(ho + c * 8) = u;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
      mine = i + 1;
    }
  }
  ss = block_sum<kNormThreads>(ss, red);
  const float inv = rsqrtf(ss / static_cast<float>(cols) + eps);
  if (y) norm_store<kNormMaxCh>(v, mine, threadIdx.x, kNormThreads, inv, w, w_dtype,
                                y + static_cast<long long>(row) * cols);
}

// h[row] = table[ids[row]]; y[row] = rmsnorm(h[row]) * w   (embedding + first input norm)
__global__ __launch_bounds__(kNormThreads) void embed_rmsnorm_kernel(
    const long long* __restrict__ ids, const bf16* __restrict__ table, long long vocab,
    const void* __restrict__ w, int w_dtype, bf16* __restrict__ h, bf16* __restrict__ y, int cols,
    float eps) {
  pdl_enter();
  __shared__ float red[kNormThreads / 32];
  const int row = blockIdx.x;
  long long id = ids[row];
  if (id < 0 || id >= vocab) {
    set_device_error(kErrIndex);
    id = 0;
  }
  const bf16* src = table + id * cols;
  bf16* hr = h + static_cast<long long>(row) * cols;
  const int nch = cols / 8;
  float v[kNormMaxCh][8];
  float ss = 0.f;
  int mine = 0;
#pragma unroll
  for (int i = 0; i < kNormMaxCh; ++i) {
    const int c = threadIdx.x + i * kNormThreads;
    if (c < nch) {
      const uint4 u = *reinterpret_cast<const uint4*>(src + c * 8);
      *reinterpret_cast<uint4*>(hr + c * 8) = u;
      const uint32_t* up = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[i][2 * j] = bf16lo(up[j]);
        v[i][2 * j + 1] = bf16hi(up[j]);
        ss += v[i][2 * j] * v[i][2 * j] + v[i][2 * j + 1] * v[i][2 * j + 1];
      }
      mine = i + 1;
    }
  }
  ss = block_sum<kNormThreads>(ss, red);
  const float inv = rsqrtf(ss / static_cast<float>(cols) + eps);
  norm_store<kNormMaxCh>(v, mine, threadIdx.x, kNormThreads, inv, w, w_dtype,
                         y + static_cast<long long>(row) * cols);
}

// out = bf16(a + b), 8 elements per thread
template <typename T>
__global__ void residual_add_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                    T* __restrict__ out, long long n8) {
  pdl_enter();
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= n8) return;
  float x[8], z[8];
  Act16<T>::unpack(reinterpret_cast<const uint4*>(a)[i], x);
  Act16<T>::unpack(reinterpret_cast<const uint4*>(b)[i], z);
  uint4 o;
  uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) op[j] = Act16<T>::pack2(x[2 * j] + z[2 * j], x[2 * j + 1] + z[2 * j + 1]);
  reinterpret_cast<uint4*>(out)[i] = o;
}

// out[r, c] = sum_{p < n_parts} part[r * rs + p * ps + c], summed in part order (fp32),
// stored as bf16 (out_f32 == 0) or fp32.  8 columns per thread; grid (col chunks, rows).
__global__ void sum_partials_kernel(const float* __restrict__ part, int n_parts, long long ps,
                                    long long rs, void* __restrict__ out, int out_f32,
                                    long long ors, int cols) {
  pdl_enter();
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= cols) return;
  const long long r = blockIdx.y;
  const float* src = part + r * rs + c;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  sum_parts8(src, ps, n_parts, acc, false);
  if (out_f32) {
    float* o = reinterpret_cast<float*>(out) + r * ors + c;
    *reinterpret_cast<float4*>(o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(o + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
  } else {
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(out) + r * ors + c) = o;
  }
}

// Greedy token per row from the per-block arg-max keys [n_blocks][key_stride] (largest
// key = largest bf16 logit, lowest vocabulary index on ties): next_ids[t] = index; also
// input_ids[t] = index and positions[t] += 1 when given (the end of a decode step).
__global__ __launch_bounds__(256) void argmax_finalize_kernel(const unsigned long long* __restrict__ keys,
                                                              int n_blocks, long long key_stride,
                                                              long long* __restrict__ next_ids,
                                                              long long* __restrict__ input_ids,
                                                              long long* __restrict__ positions,
                                                              int pos_numel, long long* step_counter) {
  pdl_enter();
  if (step_counter && blockIdx.x == 0 && threadIdx.x == 0) *step_counter += 1;
  __shared__ unsigned long long s_best[8];
  const int t = blockIdx.x;
  unsigned long long best = 0;
  for (int i = threadIdx.x; i < n_blocks; i += blockDim.x) best = max(best, keys[i * key_stride + t]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) best = max(best, s_best[w]);
    best = max(best, s_best[0]);
    const long long idx = static_cast<long long>(0xffffffffu - static_cast<uint32_t>(best & 0xffffffffu));
    next_ids[t] = idx;
    if (input_ids) input_ids[t] = idx;
    if (positions && (pos_numel != 1 || t == 0)) positions[pos_numel == 1 ? 0 : t] += 1;
  }
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + expf(-g)); }

// out = bf16(silu(gate) * up)
__global__ void silu_mul_kernel(const bf16* __restrict__ gate, const bf16* __restrict__ up,
                                bf16* __restrict__ out, long long n8) {
  pdl_enter();
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= n8) return;
  const uint4 x = reinterpret_cast<const uint4*>(gate)[i];
  const uint4 z = reinterpret_cast<const uint4*>(up)[i];
  const uint32_t* xp = reinterpret_cast<const uint32_t*>(&x);
  const uint32_t* zp = reinterpret_cast<const uint32_t*>(&z);
  uint4 o;
  uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    op[j] = pack_bf16x2(silu_f(bf16lo(xp[j])) * bf16lo(zp[j]), silu_f(bf16hi(xp[j])) * bf16hi(zp[j]));
  reinterpret_cast<uint4*>(out)[i] = o;
}

// attention_mask[b, s] = (index[s] <= pos_b); position_ids[b] = pos_b.
// pos_numel == 1: one shared position (reference semantics); == batch: per-row.
__global__ void prepare_decode_inputs_kernel(const long long* __restrict__ cache_position,
                                             int pos_numel, long long* __restrict__ mask,
                                             long long mask_stride_b, long long* __restrict__ pos_ids,
                                             long long pos_ids_stride_b,
                                             const long long* __restrict__ mask_index, int max_len) {
  pdl_enter();
  const int b = blockIdx.y;
  const long long pos = cache_position[pos_numel == 1 ? 0 : b];
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (mask && s < max_len) mask[b * mask_stride_b + s] = (mask_index[s] <= pos) ? 1 : 0;
  if (s == 0 && pos_ids) pos_ids[b * pos_ids_stride_b] = pos;
}

// dst[b, h, pos_b, :] = src[b, h, 0, :]   (element size 2 or 4 bytes)
__global__ void copy_token_to_cache_kernel(const char* __restrict__ src, long long sb, long long sh,
                                           long long sd, char* __restrict__ dst, long long db,
                                           long long dh, long long ds, long long dd,
                                           const long long* __restrict__ cache_position,
                                           int pos_numel, int heads, int dim, int esize,
                                           int max_len) {
  pdl_enter();
  const int b = blockIdx.x, h = blockIdx.y;
  long long pos = cache_position[pos_numel == 1 ? 0 : b];
  if (pos < 0 || pos >= max_len) {
    set_device_error(kErrIndex);
    return;
  }
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    const char* s = src + (b * sb + h * sh + d * sd) * esize;
    char* t = dst + (b * db + h * dh + pos * ds + d * dd) * esize;
    if (esize == 2)
      *reinterpret_cast<uint16_t*>(t) = *reinterpret_cast<const uint16_t*>(s);
    else
      *reinterpret_cast<uint32_t*>(t) = *reinterpret_cast<const uint32_t*>(s);
  }
}

// Advance per-row decode state after a step: pos[b] += 1 (int64 positions).
__global__ void advance_positions_kernel(long long* __restrict__ pos, int n) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) pos[i] += 1;
}

// ---------------------------------------------------------------------------
// host launchers (called from api.cu)
// ---------------------------------------------------------------------------
cudaError_t launch_rmsnorm(const void* x, long long xs, int xd, const void* w, int wd, void* y,
                           long long ys, int rows, int cols, float eps, cudaStream_t st) {
  if (xd == 1)
    launch_kernel(rmsnorm_kernel<__half>, rows, kNormThreads, 0, st, reinterpret_cast<const __half*>(x), xs, w, wd,
                  reinterpret_cast<__half*>(y), ys, cols, eps);
  else
    launch_kernel(rmsnorm_kernel<bf16>, rows, kNormThreads, 0, st, reinterpret_cast<const bf16*>(x), xs, w, wd,
                  reinterpret_cast<bf16*>(y), ys, cols, eps);
  return cudaGetLastError();
}

cudaError_t launch_add_rmsnorm(void* h, void* h_out, const void* delta, int dd, int nd,
                               long long dps, long long drs, const void* w, int wd, void* y,
                               int rows, int cols, float eps, cudaStream_t st, const PeerTable* peers,
                               int layer) {
  PeerTable none = {};
  launch_kernel(add_rmsnorm_kernel, rows, kNormThreads, 0, st, reinterpret_cast<bf16*>(h),
                reinterpret_cast<bf16*>(h_out), delta, dd, nd, dps, drs, w, wd, reinterpret_cast<bf16*>(y),
                cols, eps, peers ? *peers : none, layer);
  return cudaGetLastError();
}

cudaError_t launch_embed_rmsnorm(const long long* ids, const void* table, long long vocab,
                                 const void* w, int wd, void* h, void* y, int rows, int cols,
                                 float eps, cudaStream_t st) {
  launch_kernel(embed_rmsnorm_kernel, rows, kNormThreads, 0, st, ids, reinterpret_cast<const bf16*>(table), vocab, w, wd, reinterpret_cast<bf16*>(h), reinterpret_cast<bf16*>(y), cols, eps);
  return cudaGetLastError();
}

cudaError_t launch_residual_add(const void* a, const void* b, void* out, long long n, int dtype,
                                cudaStream_t st) {
  const long long n8 = n / 8;
  const int thr = 256;
  const unsigned grid = static_cast<unsigned>((n8 + thr - 1) / thr);
  if (dtype == 1)
    launch_kernel(residual_add_kernel<__half>, grid, thr, 0, st, reinterpret_cast<const __half*>(a),
                  reinterpret_cast<const __half*>(b), reinterpret_cast<__half*>(out), n8);
  else
    launch_kernel(residual_add_kernel<bf16>, grid, thr, 0, st, reinterpret_cast<const bf16*>(a),
                  reinterpret_cast<const bf16*>(b), reinterpret_cast<bf16*>(out), n8);
  return cudaGetLastError();
}

cudaError_t launch_sum_partials(const float* part, int n_parts, long long ps, long long rs, void* out,
                               int out_f32, long long ors, int rows, int cols, cudaStream_t st) {
  const int thr = 128;
  dim3 grid((cols / 8 + thr - 1) / thr, rows);
  launch_kernel(sum_partials_kernel, grid, thr, 0, st, part, n_parts, ps, rs, out, out_f32, ors, cols);
  return cudaGetLastError();
}

cudaError_t launch_argmax_finalize(const unsigned long long* keys, int n_blocks, long long key_stride,
                                   int n_tokens, long long* next_ids, long long* input_ids,
                                   long long* positions, int pos_numel, long long* step_counter,
                                   cudaStream_t st) {
  launch_kernel(argmax_finalize_kernel, n_tokens, 256, 0, st, keys, n_blocks, key_stride, next_ids, input_ids,
                positions, pos_numel, step_counter);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const void* g, const void* u, void* out, long long n, cudaStream_t st) {
  const long long n8 = n / 8;
  const int thr = 256;
  launch_kernel(silu_mul_kernel, static_cast<unsigned>((n8 + thr - 1) / thr), thr, 0, st, reinterpret_cast<const bf16*>(g), reinterpret_cast<const bf16*>(u), reinterpret_cast<bf16*>(out), n8);
  return cudaGetLastError();
}

cudaError_t launch_prepare_decode_inputs(const long long* cp, int pn, long long* mask, long long msb,
                                         long long* pid, long long psb, const long long* mi,
                                         int batch, int max_len, cudaStream_t st) {
  dim3 grid((max_len + 255) / 256, batch);
  launch_kernel(prepare_decode_inputs_kernel, grid, 256, 0, st, cp, pn, mask, msb, pid, psb, mi, max_len);
  return cudaGetLastError();
}

cudaError_t launch_copy_token_to_cache(const void* src, const long long* ss, void* dst,
                                       const long long* ds, const long long* cp, int pn, int batch,
                                       int heads, int dim, int esize, int max_len,
                                       cudaStream_t st) {
  dim3 grid(batch, heads);
  launch_kernel(copy_token_to_cache_kernel, grid, 128, 0, st, reinterpret_cast<const char*>(src), ss[0], ss[1], ss[2], reinterpret_cast<char*>(dst), ds[0], ds[1], ds[2], ds[3], cp, pn, heads, dim, esize, max_len);
  return cudaGetLastError();
}

cudaError_t launch_advance_positions(long long* pos, int n, cudaStream_t st) {
  launch_kernel(advance_positions_kernel, (n + 255) / 256, 256, 0, st, pos, n);
  return cudaGetLastError();
}

}  // namespace dsv2
