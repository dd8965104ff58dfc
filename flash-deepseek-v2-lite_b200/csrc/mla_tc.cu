// Batch family: latent-attention decode on the 5th-generation tensor cores.
//
// Same computation as mla_decode_kernel (mla.cu; the reference's decode attention,
// attention_decode_batch.py:240-342, in absorbed form) with both products on tcgen05:
//   S^T = K Q^T    A = 64 cache positions x 576 dims (K-major, straight from the cache
//                  rows), B = the 16 heads' queries (K-major), D = 64 x 16 fp32 in TMEM
//                  (M = 64: rows 16q..16q+15 in lanes 0..15 of TMEM subpartition q)
//   O^T += V^T P^T A = the latent part of the same tile read MN-major (dims x positions),
//                  B = P^T (16 heads x 64 positions, written by the softmax threads),
//                  D = four 128-dim tiles x 16 heads fp32 in TMEM (lane = latent dim)
// so the softmax works on one cache position per thread and the accumulator never
// leaves TMEM.
//
// One CTA per (split, row), 6 warps:
//   warp 0      TMA producer: each 64-position tile (9 swizzle chunks of 64 dims,
//               72 KB) into one of two stages, so the next tile streams in while the
//               current one is scored and accumulated
//   warp 1      TMEM owner + MMA issuer (one thread): S^T of tile t+1 is issued before
//               P @ V of tile t, so scoring overlaps the softmax; a stage is released
//               when the P @ V products reading it complete
//   warps 2..5  load Q, then per tile: read S^T, per-head max over the tile (warp
//               transpose-reduce + shared memory), online-softmax update, P^T to shared
//               memory (two buffers), rescale O^T in TMEM when a head's maximum grew by
//               more than 2^8; at the end
//               normalise and write o_lat (or the split partials)
// All mbarrier waits are bounded (common.cuh).
//
// Measured on B200 this kernel is slower than the mma.sync kernel (one CTA per SM with a
// two-tile ring keeps too few bytes in flight, and each CTA pays its own setup), so the
// decode engine uses mla_decode_kernel for both families; this one stays selectable
// through dsv2_mla_decode_args.family = DSV2_FAMILY_BATCH and is tested for parity.
#include "params.cuh"

namespace dsv2 {

constexpr int kMtTile = 64;                          // positions per tile (M of S^T)
constexpr int kMtChunkBytes = kMtTile * 128;          // one 64-dim swizzle chunk: 8 KB
constexpr int kMtStageBytes = kChunks * kMtChunkBytes;  // 72 KB
constexpr int kMtStages = 2;
constexpr int kMtQBytes = kChunks * kHeads * 128;    // 9 chunks x 16 rows x 128 B
constexpr int kMtPBytes = kHeads * 128;              // P^T: 16 rows x 64 positions (x2 buffers)
// The running maximum used for the exponentials is only raised when a head's tile
// maximum exceeds it by more than this (log2 units): P then stays below 2^8, and the
// accumulator in TMEM is rescaled only on those (rare) tiles.  The result is the same
// softmax: numerator and denominator use the same reference value.
constexpr float kMtRescaleLog2 = 8.f;
constexpr int kMtThreads = 192;
constexpr int kMtTmemCols = 128;                     // S0, S1 (16 each), O^T 4 x 16
constexpr int kMtColO = 32;

struct MtLayout {
  static constexpr int kv = 0;
  static constexpr int q = kv + kMtStages * kMtStageBytes;
  static constexpr int pt = q + kMtQBytes;
  static constexpr int red = pt + 2 * kMtPBytes;                     // float [2][16][4]
  static constexpr int bars = red + 2 * kHeads * 4 * 4;
  static constexpr int n_bars = 2 * kMtStages + 4 + 4 + 1;
  static constexpr int tmem_slot = bars + n_bars * 8;
  static constexpr int abort_flag = tmem_slot + 4;
  static constexpr int total = tmem_slot + 16;
};

__device__ __forceinline__ void softmax_bar() {  // the 4 softmax warps only
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Bounded wait that gives up at once after any wait of the CTA has given up, so that an
// error ends the kernel quickly; every thread still takes every named barrier.
__device__ __forceinline__ bool mt_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (*abort) return false;
  if (mbar_wait(bar, parity)) return true;
  *abort = 1;
  return false;
}

// Warp-wide per-head reduction of 16 values per lane (max or sum): afterwards lane l
// holds the result for head ((l>>4)&1)*8 + ((l>>3)&1)*4 + ((l>>2)&1)*2 + ((l>>1)&1)
// (lanes 2j and 2j+1 agree).  16 shuffles instead of 16 x 5.
template <bool MAX>
__device__ __forceinline__ float warp_transpose_reduce(const float (&v)[16], int lane) {
  auto op = [](float a, float b) { return MAX ? fmaxf(a, b) : a + b; };
  float a[8];
  const bool u16 = lane & 16;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float send = u16 ? v[i] : v[i + 8];
    const float keep = u16 ? v[i + 8] : v[i];
    a[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
  float c[4];
  const bool u8 = lane & 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = u8 ? a[i] : a[i + 4];
    const float keep = u8 ? a[i + 4] : a[i];
    c[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
  float d[2];
  const bool u4 = lane & 4;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = u4 ? c[i] : c[i + 2];
    const float keep = u4 ? c[i + 2] : c[i];
    d[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  const bool u2 = lane & 2;
  float e = op(u2 ? d[1] : d[0], __shfl_xor_sync(0xffffffffu, u2 ? d[0] : d[1], 2));
  return op(e, __shfl_xor_sync(0xffffffffu, e, 1));
}
__device__ __forceinline__ int transpose_reduce_head(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

// Per-head reduction over the 128 softmax threads; every thread receives all 16 results.
// red: this round's [16][4] buffer (rounds alternate between two buffers).
template <bool MAX>
__device__ __forceinline__ void block_head_reduce(const float (&v)[16], float (&out)[16], float* red,
                                                  int sw, int lane) {
  const float r = warp_transpose_reduce<MAX>(v, lane);
  if ((lane & 1) == 0) red[transpose_reduce_head(lane) * 4 + sw] = r;
  softmax_bar();
#pragma unroll
  for (int h = 0; h < kHeads; ++h) {
    const float4 q = *reinterpret_cast<const float4*>(red + h * 4);
    out[h] = MAX ? fmaxf(fmaxf(q.x, q.y), fmaxf(q.z, q.w)) : (q.x + q.y) + (q.z + q.w);
  }
}

__global__ __launch_bounds__(kMtThreads, 1) void mla_tc_kernel(const MlaDecodeParams p,
                                                               const __grid_constant__ CUtensorMap tm_kv) {
  const bool early = p.inputs_prior != 0;
  if (!early) pdl_enter();
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + MtLayout::bars);
  uint64_t* kv_full = bars;                       // [kMtStages]
  uint64_t* kv_empty = kv_full + kMtStages;       // [kMtStages]
  uint64_t* s_full = kv_empty + kMtStages;        // [2]
  uint64_t* s_empty = s_full + 2;                 // [2]
  uint64_t* p_ready = s_empty + 2;                // [2] (by tile parity)
  uint64_t* o_done = p_ready + 2;                 // [2] (by tile parity)
  uint64_t* q_ready = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + MtLayout::tmem_slot);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + MtLayout::abort_flag);
  float* red = reinterpret_cast<float*>(smem + MtLayout::red);

  const int split = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long pos = p.positions[p.pos_numel == 1 ? 0 : b];
  const int len = static_cast<int>(min(static_cast<long long>(p.max_len), pos + 1));
  const int s_beg = split * p.split_len;
  const int s_end = min(len, s_beg + p.split_len);
  float* mlp = p.ml_part + ((static_cast<long long>(b) * p.n_splits + split) * kHeads) * 2;
  if (s_beg >= s_end) {
    if (early) pdl_enter();
    if (threadIdx.x < kHeads) {
      mlp[threadIdx.x * 2] = -INFINITY;
      mlp[threadIdx.x * 2 + 1] = 0.f;
    }
    return;
  }
  const int n_tiles = (s_end - s_beg + kMtTile - 1) / kMtTile;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kMtStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_ready[i], 128);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(q_ready, 128);
    *abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_kv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kMtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      bool waited = !early;
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int st = t % kMtStages;
        if (!mt_wait(&kv_empty[st], ((t / kMtStages) & 1) ^ 1, abort)) { ok = false; break; }
        unsigned char* dst = smem + MtLayout::kv + st * kMtStageBytes;
        mbar_arrive_expect_tx(&kv_full[st], kMtStageBytes);
        for (int c = 0; c < kChunks; ++c)
          tma_load_3d(smem_u32(dst + c * kMtChunkBytes), &tm_kv, &kv_full[st], c * 64, s_beg + t * kMtTile, b);
        if (!waited) {  // the first tile is in flight: now wait for the previous kernel
          pdl_enter();
          waited = true;
        }
      }
      if (!waited) pdl_enter();
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (early) pdl_enter();
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_bf16(kMtTile, kHeads);
      const uint32_t idesc_o = make_idesc_bf16(128, kHeads, true);
      const uint32_t q_base = smem_u32(smem + MtLayout::q);
      const uint32_t p_base = smem_u32(smem + MtLayout::pt);
      // S^T of tile t into S buffer t % 2: 9 chunks x 4 K steps
      auto issue_s = [&](int t) -> bool {
        const int st = t % kMtStages, sb = t & 1;
        if (!mt_wait(&kv_full[st], (t / kMtStages) & 1, abort)) return false;
        if (!mt_wait(&s_empty[sb], ((t >> 1) & 1) ^ 1, abort)) return false;
        tc_fence_after();
        const uint32_t kvb = smem_u32(smem + MtLayout::kv + st * kMtStageBytes);
        const uint32_t ds = tmem_base + sb * kHeads;
        for (int c = 0; c < kChunks; ++c) {
          const uint64_t da = sw128_kmajor_desc(kvb + c * kMtChunkBytes);
          const uint64_t db = sw128_kmajor_desc(q_base + c * (kHeads * 128));
#pragma unroll
          for (int k = 0; k < 4; ++k) tc_mma_bf16(ds, da + 2 * k, db + 2 * k, idesc_s, (c | k) ? 1u : 0u);
        }
        tc_commit(&s_full[sb]);
        return true;
      };
      if (!mt_wait(q_ready, 0, abort)) ok = false;
      tc_fence_after();
      if (ok && !issue_s(0)) ok = false;
      for (int t = 0; t < n_tiles && ok; ++t) {
        // scoring of the next tile overlaps this tile's softmax
        if (t + 1 < n_tiles && !issue_s(t + 1)) { ok = false; break; }
        // O^T += V^T P^T once the softmax threads have written P^T[t % 2] (and rescaled O^T)
        const int pb = t & 1;
        if (!mt_wait(&p_ready[pb], (t >> 1) & 1, abort)) { ok = false; break; }
        tc_fence_after();
        const int st = t % kMtStages;
        const uint32_t kvb = smem_u32(smem + MtLayout::kv + st * kMtStageBytes);
        for (int m = 0; m < 4; ++m) {
          const uint32_t dO = tmem_base + kMtColO + m * kHeads;
#pragma unroll
          for (int kk = 0; kk < kMtTile / 16; ++kk) {
            const uint64_t da = sw128_mnmajor_desc(kvb + (2 * m) * kMtChunkBytes + kk * 2048, kMtChunkBytes, 1024);
            const uint64_t db = sw128_kmajor_desc(p_base + pb * kMtPBytes) + 2 * kk;
            tc_mma_bf16(dO, da, db, idesc_o, (t | kk) ? 1u : 0u);
          }
        }
        tc_commit(&kv_empty[st]);
        tc_commit(&o_done[pb]);
      }
    }
  } else {
    // ---------------- Q, softmax and output (warps 2..5) ----------------
    if (early) pdl_enter();
    const int quad = warp & 3;
    const int row = quad * 32 + lane;                 // O^T: latent dim (within a 128-dim tile)
    const int prow = quad * 16 + lane;                // S^T (M = 64): position, lanes 0..15 only
    const bool plane = lane < 16;
    const int tidx = threadIdx.x - 64;               // 0..127
    // Q = [q_abs | q_pe] (16 x 576) into 9 swizzled K-major chunks of 16 rows
    unsigned char* sq = smem + MtLayout::q;
    for (int i = tidx; i < kHeads * kChunks * 8; i += 128) {
      const int h = i / (kChunks * 8), rem = i % (kChunks * 8);
      const int ch = rem / 8, c16 = rem % 8;
      const int d = ch * 64 + c16 * 8;
      const bf16* src = (d < kLatent)
                            ? p.q_abs + (static_cast<long long>(b) * kHeads + h) * kLatent + d
                            : p.q_pe + (static_cast<long long>(b) * kHeads + h) * kRope + (d - kLatent);
      *reinterpret_cast<uint4*>(sq + ch * (kHeads * 128) + swz(h, c16)) = *reinterpret_cast<const uint4*>(src);
    }
    fence_proxy_async_smem();
    mbar_arrive(q_ready);

    float m_run[kHeads], l_part[kHeads];
#pragma unroll
    for (int h = 0; h < kHeads; ++h) {
      m_run[h] = -INFINITY;
      l_part[h] = 0.f;
    }
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    bf16* spt = reinterpret_cast<bf16*>(smem + MtLayout::pt);
    for (int t = 0; t < n_tiles; ++t) {  // no early exit: every thread takes every barrier
      const int sb = t & 1;
      if (!mt_wait(&s_full[sb], (t >> 1) & 1, abort)) ok = false;
      tc_fence_after();
      float v[kHeads];
      tmem_ld16(tmem_base + lane_off + sb * kHeads, v);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);
      const bool valid = plane && s_beg + t * kMtTile + prow < s_end;
#pragma unroll
      for (int h = 0; h < kHeads; ++h) v[h] = valid ? v[h] * p.scale_log2 : -INFINITY;
      float tmax[kHeads];
      block_head_reduce<true>(v, tmax, red + (t & 1) * kHeads * 4, quad, lane);
      float alpha[kHeads];
      bool grew = false;
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        // raise the reference maximum only when this tile exceeds it by the threshold
        const bool raise = tmax[h] > m_run[h] + kMtRescaleLog2;
        const float mn = raise ? tmax[h] : m_run[h];
        alpha[h] = raise ? exp2f(m_run[h] - mn) : 1.f;
        grew |= raise;
        m_run[h] = mn;
        v[h] = exp2f(v[h] - mn);
        l_part[h] = l_part[h] * alpha[h] + v[h];
      }
      const int pb = t & 1;
      if (t > 0 && grew) {
        // O^T must hold every earlier tile before it is rescaled
        if (!mt_wait(&o_done[(t - 1) & 1], ((t - 1) >> 1) & 1, abort)) ok = false;
        tc_fence_after();
        if (ok) {
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            float o[kHeads];
            const uint32_t ta = tmem_base + lane_off + kMtColO + m * kHeads;
            tmem_ld16(ta, o);
            tmem_ld_wait();
#pragma unroll
            for (int h = 0; h < kHeads; ++h) o[h] *= alpha[h];
            tmem_st16(ta, o);
          }
          tmem_st_wait();
        }
      }
      // P^T buffer t % 2 was last read by the products of tile t - 2
      if (t > 1) {
        if (!mt_wait(&o_done[pb], ((t - 2) >> 1) & 1, abort)) ok = false;
      }
      // P^T[h, position] (K-major, 128-byte swizzle: 16 rows of 64 positions)
      if (plane) {
        const int u = prow >> 3;
        unsigned char* base = reinterpret_cast<unsigned char*>(spt) + pb * kMtPBytes + (prow & 7) * 2;
#pragma unroll
        for (int h = 0; h < kHeads; ++h)
          *reinterpret_cast<bf16*>(base + h * 128 + ((u ^ (h & 7)) << 4)) = __float2bfloat16_rn(v[h]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_ready[pb]);
    }
    if (!mt_wait(&o_done[(n_tiles - 1) & 1], ((n_tiles - 1) >> 1) & 1, abort)) ok = false;
    tc_fence_after();
    float l_tot[kHeads];
    block_head_reduce<false>(l_part, l_tot, red + (n_tiles & 1) * kHeads * 4, quad, lane);
    if (len <= p.split_len) {
      // one split holds the whole row: normalised output directly
      bf16* ob = p.o_lat + static_cast<long long>(b) * kHeads * kLatent;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        float o[kHeads];
        tmem_ld16(tmem_base + lane_off + kMtColO + m * kHeads, o);
        tmem_ld_wait();
        const int d = m * 128 + row;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) ob[h * kLatent + d] = __float2bfloat16_rn(o[h] / l_tot[h]);
      }
    } else {
      float* op = p.o_part + ((static_cast<long long>(b) * p.n_splits + split) * kHeads) * kLatent;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        float o[kHeads];
        tmem_ld16(tmem_base + lane_off + kMtColO + m * kHeads, o);
        tmem_ld_wait();
        const int d = m * 128 + row;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) op[h * kLatent + d] = o[h];
      }
      if (tidx == 0) {
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          mlp[h * 2] = m_run[h];
          mlp[h * 2 + 1] = l_tot[h];
        }
      }
    }
  }
  if (!ok) set_device_error(kErrMbarTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kMtTmemCols);
  }
}

cudaError_t mla_tc_init() {
  return cudaFuncSetAttribute(mla_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, MtLayout::total);
}

cudaError_t launch_mla_tc(const MlaDecodeParams& p, const CUtensorMap& tm_kv64, int batch, cudaStream_t st) {
  launch_kernel(mla_tc_kernel, dim3(p.n_splits, batch), kMtThreads, MtLayout::total, st, p, tm_kv64);
  return cudaGetLastError();
}

}  // namespace dsv2
