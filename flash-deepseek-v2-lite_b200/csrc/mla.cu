// Multi-head latent attention (MLA) decode over the 576-wide latent KV cache.
//
// Replaces the reference's expanded-cache attention pipeline (Flash-DeepSeeek-V2-Lite):
//   attention_decode_small.py:140-264 / :1073-1216  q/k/v build + RoPE (half-split layout)
//   attention_decode_small.py:267-339               write of expanded K (192) / V (128) per head
//   attention_decode_small.py:342-423, attention_decode_batch.py:240-342
//                                                    one-CTA-per-(b,h) online-softmax attention
// Absorbed formulation: the cache row of every position is
//   [ RMSNorm(c_kv) (512) | RoPE(k_pe) (64) ]  (bf16, shared by all 16 heads)
// and the per-head query is [ q_nope @ W_UK[h] (512) | RoPE(q_pe) (64) ], so
//   score[h, s] = scale * <q[h], row[s]>,   o_lat[h] = sum_s p[h, s] * row[s][:512],
// and the per-head value projection W_UV[h] is applied after attention.
// RoPE rotates interleaved pairs (2j, 2j+1) exactly like the HF model's
// apply_rotary_emb; q and k use the same pairing, so q.k matches the reference's
// half-split layout.
//
// mla_decode_kernel: split-KV flash-decode.  One CTA = (split, sequence), 4 warps.
// 32-position tiles of the latent cache are staged through a 2-deep cp.async ring in
// a 128-byte-swizzled layout (conflict-free ldmatrix).  Scores use mma.sync with
// the 16 heads as M: each warp owns a 144-wide slice of the 576 dims and keeps its
// query fragments in registers for the whole kernel; slices are summed through
// shared memory.  P @ V (the latent part) uses mma.sync with each warp owning 128
// latent dims.  A row that fits one split writes o_lat directly; otherwise the split
// partials (o, m, l) are merged by the last split of the row to finish (row_sync
// counters) or, without counters, by mla_combine_kernel.
#include "params.cuh"

namespace dsv2 {

constexpr int kHeads = 16;
constexpr int kLatent = 512;
constexpr int kRope = 64;
constexpr int kRow = kLatent + kRope;           // 576
constexpr int kRowBytes = kRow * 2;             // 1152
constexpr int kChunks = kRow / 64;              // 9 swizzle chunks of 64 dims
constexpr int kTile = 32;                       // positions per tile (two CTAs per SM)
constexpr int kStages = 2;
constexpr int kTileBytes = kTile * kRowBytes;   // 36864
constexpr int kQBytes = kHeads * kRowBytes;     // 18432
constexpr int kSRedStride = kTile + 4;          // fp32 row stride of the score-reduction buffer
constexpr int kPStride = kTile + 8;             // bf16 row stride of P
constexpr int kMlaPvWarps = 8;                 // warps doing P @ V (64 latent dims each)
constexpr int kMlaThreads = (kChunks) * 32;     // 9 warps: one 64-dim chunk of the scores each

// ----------------------------------------------------------------------------
// mla_prep: latent RMSNorm + RoPE + cache write for the new token, RoPE of q_pe
// ----------------------------------------------------------------------------

__global__ __launch_bounds__(256) void mla_prep_kernel(const MlaPrepParams p) {
  pdl_enter();
  __shared__ float red[8];
  __shared__ __align__(16) bf16 s_row[kHeads * 192 + kRow];  // this row of qkva, bf16
  const int b = blockIdx.x;
  // stage the row (summing fp32 split-K partials and rounding to bf16, like a bf16 linear)
  if (p.qkva_f32) {
    const float* src = reinterpret_cast<const float*>(p.qkva) + b * p.qkva_row_stride;
    for (int i = threadIdx.x; i < (kHeads * 192 + kRow) / 4; i += blockDim.x) {
      float4 acc = *reinterpret_cast<const float4*>(src + 4 * i);
      for (int s = 1; s < p.qkva_parts; ++s) {
        const float4 v = *reinterpret_cast<const float4*>(src + s * p.qkva_part_stride + 4 * i);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      uint2 o;
      o.x = pack_bf16x2(acc.x, acc.y);
      o.y = pack_bf16x2(acc.z, acc.w);
      *reinterpret_cast<uint2*>(s_row + 4 * i) = o;
    }
  } else {
    const bf16* src = reinterpret_cast<const bf16*>(p.qkva) + b * p.qkva_row_stride;
    for (int i = threadIdx.x; i < (kHeads * 192 + kRow) / 8; i += blockDim.x)
      *reinterpret_cast<uint4*>(s_row + 8 * i) = *reinterpret_cast<const uint4*>(src + 8 * i);
  }
  __syncthreads();
  const bf16* row = s_row;
  if (p.q_nope_out) {
    for (int i = threadIdx.x; i < kHeads * 16; i += blockDim.x) {
      const int h = i / 16, c = i % 16;
      *reinterpret_cast<uint4*>(p.q_nope_out + (static_cast<long long>(b) * kHeads + h) * 128 + c * 8) =
          *reinterpret_cast<const uint4*>(row + h * 192 + c * 8);
    }
  }
  long long pos = p.positions[p.pos_numel == 1 ? 0 : b];
  const bool pos_ok = (pos >= 0 && pos < p.max_len && pos < p.rope_rows);
  if (!pos_ok) {
    if (threadIdx.x == 0) set_device_error(kErrIndex);
    return;
  }
  bf16* crow = p.cache + b * p.cache_b_stride + pos * kRow;
  const float* cs = p.cos_tab + pos * p.rope_stride;
  const float* sn = p.sin_tab + pos * p.rope_stride;
  // latent RMSNorm: threads 0..63 own 8 elements each
  const int t = threadIdx.x;
  float v[8];
  float ss = 0.f;
  if (t < 64) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + kHeads * 192 + t * 8);
    const uint32_t* up = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = bf16lo(up[j]);
      v[2 * j + 1] = bf16hi(up[j]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
  }
  ss = warp_sum(ss);
  if ((t & 31) == 0) red[t >> 5] = ss;
  __syncthreads();
  if (t < 64) {
    const float inv = rsqrtf((red[0] + red[1]) / static_cast<float>(kLatent) + p.eps);
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float w0 = __bfloat162float(p.kv_norm_w[t * 8 + 2 * j]);
      const float w1 = __bfloat162float(p.kv_norm_w[t * 8 + 2 * j + 1]);
      op[j] = pack_bf16x2(v[2 * j] * inv * w0, v[2 * j + 1] * inv * w1);
    }
    *reinterpret_cast<uint4*>(crow + t * 8) = o;
  }
  // RoPE pairs: 16 heads x 32 pairs of q_pe, plus 32 pairs of k_pe
  for (int i = t; i < (kHeads + 1) * 32; i += 256) {
    const int h = i >> 5, j = i & 31;
    const bf16* src = (h < kHeads) ? (row + h * 192 + 128 + 2 * j) : (row + kHeads * 192 + kLatent + 2 * j);
    const float e = __bfloat162float(src[0]), o = __bfloat162float(src[1]);
    const float c = cs[j], s = sn[j];
    const float re = e * c - o * s, im = o * c + e * s;
    const uint32_t packed = pack_bf16x2(re, im);
    if (h < kHeads)
      *reinterpret_cast<uint32_t*>(p.q_pe_out + (static_cast<long long>(b) * kHeads + h) * kRope + 2 * j) = packed;
    else
      *reinterpret_cast<uint32_t*>(crow + kLatent + 2 * j) = packed;
  }
}

// ----------------------------------------------------------------------------
// split-KV decode
// ----------------------------------------------------------------------------

// byte offset of (row r, 16-byte column c16) inside one 64-dim swizzle chunk of R rows
__device__ __forceinline__ uint32_t swz(int r, int c16) {
  return static_cast<uint32_t>(r * 128 + ((c16 ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n));
}

// o_lat[b] = merge of the first n_active split partials of row b (the splits of a row are
// contiguous from 0): o = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s, per head.
// Partials written by other CTAs are read with L1-bypassing loads.
__device__ __forceinline__ void mla_merge_row(const float* o_part, const float* ml_part, int n_splits,
                                              int n_active, bf16* o_lat, int b, int tid, int nthreads) {
  const float* ml = ml_part + (static_cast<long long>(b) * n_splits) * kHeads * 2;
  for (int i = tid; i < kHeads * kLatent / 4; i += nthreads) {
    const int h = i / (kLatent / 4), d = (i % (kLatent / 4)) * 4;
    float M = -INFINITY;
    for (int s = 0; s < n_active; ++s) {
      const float l = __ldcg(ml + (s * kHeads + h) * 2 + 1);
      if (l > 0.f) M = fmaxf(M, __ldcg(ml + (s * kHeads + h) * 2));
    }
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, den = 0.f;
    for (int s = 0; s < n_active; ++s) {
      const float l = __ldcg(ml + (s * kHeads + h) * 2 + 1);
      if (!(l > 0.f)) continue;
      const float w = exp2f(__ldcg(ml + (s * kHeads + h) * 2) - M);
      den += w * l;
      const float4 v = __ldcg(reinterpret_cast<const float4*>(
          o_part + ((static_cast<long long>(b) * n_splits + s) * kHeads + h) * kLatent + d));
      a0 += w * v.x; a1 += w * v.y; a2 += w * v.z; a3 += w * v.w;
    }
    const float inv = den > 0.f ? 1.f / den : 0.f;
    uint2 o;
    o.x = pack_bf16x2(a0 * inv, a1 * inv);
    o.y = pack_bf16x2(a2 * inv, a3 * inv);
    *reinterpret_cast<uint2*>(o_lat + (static_cast<long long>(b) * kHeads + h) * kLatent + d) = o;
  }
}

__global__ __launch_bounds__(kMlaThreads, 2) void mla_decode_kernel(const MlaDecodeParams p,
                                                                   const __grid_constant__ CUtensorMap tm_kv) {
  // inputs_prior: positions, q_pe and the cache are older than the previous launch, so
  // the first cache tiles are requested before waiting for it (it writes q_abs)
  const bool early = p.inputs_prior != 0;
  if (!early) pdl_enter();
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* s_kv = smem;                                    // stages x 9 chunks x 32 rows x 128 B
  unsigned char* s_q = smem + kStages * kTileBytes;              // 9 chunks x 16 rows x 128 B
  float* s_red = reinterpret_cast<float*>(s_q + kQBytes);        // [9][16][kSRedStride]
  bf16* s_p = reinterpret_cast<bf16*>(s_red + kChunks * kHeads * kSRedStride);  // [16][kPStride]
  float* s_alpha = reinterpret_cast<float*>(s_p + kHeads * kPStride);           // [16]
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(s_alpha + kHeads);           // [kStages]
  uint64_t* empty_bar = full_bar + kStages;                                      // [kStages]

  const int split = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const long long pos = p.positions[p.pos_numel == 1 ? 0 : b];
  const int len = static_cast<int>(min(static_cast<long long>(p.max_len), pos + 1));
  const int s_beg = split * p.split_len;
  const int s_end = min(len, s_beg + p.split_len);
  float* mlp = p.ml_part + ((static_cast<long long>(b) * p.n_splits + split) * kHeads) * 2;
  if (s_beg >= s_end) {
    if (early) pdl_enter();
    if (tid < kHeads) {
      mlp[tid * 2] = -INFINITY;
      mlp[tid * 2 + 1] = 0.f;
    }
    return;
  }
  const int n_tiles = (s_end - s_beg + kTile - 1) / kTile;
  const bool producer = (warp == kMlaPvWarps && lane == 0);
  // tile ti -> stage ti % 2: 9 TMA boxes of 64 dims x 32 positions (128-byte swizzle);
  // positions past the split are masked below, past the cache they read as zeros
  auto load_tile = [&](int ti) {
    const int st = ti % kStages;
    mbar_arrive_expect_tx(&full_bar[st], kTileBytes);
    for (int c = 0; c < kChunks; ++c)
      tma_load_3d(smem_u32(s_kv + st * kTileBytes + c * (kTile * 128)), &tm_kv, &full_bar[st], c * 64,
                  s_beg + ti * kTile, b);
  };
  if (producer) {
    for (int st = 0; st < kStages; ++st) {
      mbar_init(&full_bar[st], 1);
      mbar_init(&empty_bar[st], kMlaPvWarps);
    }
    fence_mbar_init();
    prefetch_tmap(&tm_kv);
    load_tile(0);
    if (n_tiles > 1) load_tile(1);
  }
  if (early) pdl_enter();

  // --- stage Q = [q_abs | q_pe] (16 x 576) into swizzled smem
  for (int i = tid; i < kHeads * kChunks * 8; i += kMlaThreads) {
    const int h = i / (kChunks * 8), rem = i % (kChunks * 8);
    const int ch = rem / 8, c16 = rem % 8;
    const int d = ch * 64 + c16 * 8;
    const bf16* src = (d < kLatent)
                          ? p.q_abs + (static_cast<long long>(b) * kHeads + h) * kLatent + d
                          : p.q_pe + (static_cast<long long>(b) * kHeads + h) * kRope + (d - kLatent);
    *reinterpret_cast<uint4*>(s_q + ch * (kHeads * 128) + swz(h, c16)) = *reinterpret_cast<const uint4*>(src);
  }
  __syncthreads();  // Q and the barriers visible

  // --- query fragments of this warp's 64-dim chunk (warp w scores dims [64w, 64w + 64))
  uint32_t qa[4][4];
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int mi = lane >> 3, ri = lane & 7;
    const int row = (mi & 1) * 8 + ri;
    const int c16 = ks * 2 + (mi >> 1);
    ldmatrix_x4(smem_u32(s_q + warp * (kHeads * 128) + swz(row, c16)), qa[ks][0], qa[ks][1], qa[ks][2],
                qa[ks][3]);
  }

  // softmax state: threads 0..255, head hs = tid / 16, positions 2*js, 2*js + 1 of a tile
  const int hs = (tid >> 4) & 15, js = tid & 15;
  float m_run = -INFINITY, l_run = 0.f;
  // P @ V accumulators: warps 0..7 own latent dims [64w, 64w + 64)
  float o_acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o_acc[j][0] = o_acc[j][1] = o_acc[j][2] = o_acc[j][3] = 0.f;
  bool ok = true;

  for (int ti = 0; ti < n_tiles; ++ti) {
    const int stage = ti % kStages;
    const uint32_t par = static_cast<uint32_t>((ti / kStages) & 1);
    if (!mbar_wait(&full_bar[stage], par)) ok = false;
    const unsigned char* kv = s_kv + stage * kTileBytes;

    // --- partial scores over this warp's 64 dims for the 32 positions of the tile
    {
      float sc[kTile / 8][4];
#pragma unroll
      for (int j = 0; j < kTile / 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
      const unsigned char* kc = kv + warp * (kTile * 128);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
        for (int np = 0; np < kTile / 16; ++np) {  // pairs of n8 tiles (16 positions)
          const int mi = lane >> 3, ri = lane & 7;
          const int r = np * 16 + (mi >> 1) * 8 + ri;
          const int c16 = ks * 2 + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(smem_u32(kc + swz(r, c16)), b0, b1, b2, b3);
          mma_bf16_16816(sc[2 * np], qa[ks], b0, b1);
          mma_bf16_16816(sc[2 * np + 1], qa[ks], b2, b3);
        }
      }
      float* red_w = s_red + warp * kHeads * kSRedStride;
#pragma unroll
      for (int j = 0; j < kTile / 8; ++j) {
        const int c = j * 8 + 2 * tq;
        *reinterpret_cast<float2*>(red_w + gq * kSRedStride + c) = make_float2(sc[j][0], sc[j][1]);
        *reinterpret_cast<float2*>(red_w + (gq + 8) * kSRedStride + c) = make_float2(sc[j][2], sc[j][3]);
      }
    }
    __syncthreads();

    // --- online softmax (log2 domain) for head hs, positions 2*js, 2*js + 1
    if (tid < 256) {
      const int t0 = s_beg + ti * kTile;
      const int c = 2 * js;
      float v0 = 0.f, v1 = 0.f;
#pragma unroll
      for (int w = 0; w < kChunks; ++w) {
        const float2 r2 = *reinterpret_cast<const float2*>(s_red + (w * kHeads + hs) * kSRedStride + c);
        v0 += r2.x;
        v1 += r2.y;
      }
      v0 = (t0 + c < s_end) ? v0 * p.scale_log2 : -INFINITY;
      v1 = (t0 + c + 1 < s_end) ? v1 * p.scale_log2 : -INFINITY;
      float mx = fmaxf(v0, v1);
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m_run, mx);
      const float alpha = exp2f(m_run - m_new);
      const float p0 = exp2f(v0 - m_new), p1 = exp2f(v1 - m_new);
      float sum = p0 + p1;
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      l_run = l_run * alpha + sum;
      m_run = m_new;
      *reinterpret_cast<uint32_t*>(s_p + hs * kPStride + c) = pack_bf16x2(p0, p1);
      if (js == 0) s_alpha[hs] = alpha;
    }
    __syncthreads();

    if (warp < kMlaPvWarps) {
      // --- O[:, 64*warp .. +64] = alpha * O + P @ V
      const float a0 = s_alpha[gq], a1 = s_alpha[gq + 8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o_acc[j][0] *= a0; o_acc[j][1] *= a0;
        o_acc[j][2] *= a1; o_acc[j][3] *= a1;
      }
      const unsigned char* vc = kv + warp * (kTile * 128);
#pragma unroll
      for (int kk = 0; kk < kTile / 16; ++kk) {
        uint32_t pa[4];
        {
          const int mi = lane >> 3, ri = lane & 7;
          const int row = (mi & 1) * 8 + ri;
          const int col = kk * 16 + (mi >> 1) * 8;
          ldmatrix_x4(smem_u32(s_p + row * kPStride + col), pa[0], pa[1], pa[2], pa[3]);
        }
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          const int mi = lane >> 3, ri = lane & 7;
          const int r = kk * 16 + (mi & 1) * 8 + ri;
          const int c16 = np * 2 + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(smem_u32(vc + swz(r, c16)), b0, b1, b2, b3);
          mma_bf16_16816(o_acc[2 * np], pa, b0, b1);
          mma_bf16_16816(o_acc[2 * np + 1], pa, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[stage]);  // this warp is done with the tile
    } else if (producer && ti + kStages < n_tiles) {
      // refill this stage once the P @ V warps have released it
      if (!mbar_wait(&empty_bar[stage], par)) ok = false;
      else load_tile(ti + kStages);
    }
  }
  if (!ok) set_device_error(kErrMbarTimeout);

  if (len <= p.split_len) {
    // the whole row fitted in this one split: normalise and write o_lat directly
    // (no partials, and the merge skips the row)
    if (tid < 256 && js == 0) s_alpha[hs] = 1.f / l_run;
    __syncthreads();
    if (warp < kMlaPvWarps) {
      const float i0 = s_alpha[gq], i1 = s_alpha[gq + 8];
      bf16* ob = p.o_lat + static_cast<long long>(b) * kHeads * kLatent;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = warp * 64 + j * 8 + 2 * tq;
        *reinterpret_cast<uint32_t*>(ob + gq * kLatent + d) = pack_bf16x2(o_acc[j][0] * i0, o_acc[j][1] * i0);
        *reinterpret_cast<uint32_t*>(ob + (gq + 8) * kLatent + d) =
            pack_bf16x2(o_acc[j][2] * i1, o_acc[j][3] * i1);
      }
    }
    return;
  }
  // --- write partial results
  if (warp < kMlaPvWarps) {
    float* op = p.o_part + ((static_cast<long long>(b) * p.n_splits + split) * kHeads) * kLatent;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = warp * 64 + j * 8 + 2 * tq;
      *reinterpret_cast<float2*>(op + gq * kLatent + d) = make_float2(o_acc[j][0], o_acc[j][1]);
      *reinterpret_cast<float2*>(op + (gq + 8) * kLatent + d) = make_float2(o_acc[j][2], o_acc[j][3]);
    }
  }
  if (tid < 256 && js == 0) {
    mlp[hs * 2] = m_run;
    mlp[hs * 2 + 1] = l_run;
  }
  if (!p.row_sync) return;  // mla_combine_kernel merges the splits
  // The last split of the row to finish merges all of them (no separate launch): the
  // partial stores above are published by a fence + counter increment, the last
  // arriver reads the others' partials through L2 and returns the counter to zero.
  __syncthreads();
  int* s_flag = reinterpret_cast<int*>(s_alpha);
  if (tid == 0) {
    const int n_active = (len + p.split_len - 1) / p.split_len;
    __threadfence();
    const int t = atomicAdd(&p.row_sync[b], 1);
    const bool last = (t == n_active - 1);
    if (last) {
      p.row_sync[b] = 0;
      __threadfence();
    }
    *s_flag = last ? n_active : 0;
  }
  __syncthreads();
  const int n_active = *s_flag;
  if (n_active == 0) return;
  mla_merge_row(p.o_part, p.ml_part, p.n_splits, n_active, p.o_lat, b, tid, kMlaThreads);
}

// o_lat[b, h, :] = sum_s 2^(m_s - M) o_s / sum_s 2^(m_s - M) l_s   (bf16 out)
// (rows whose length fits one split were written directly by mla_decode_kernel)
__global__ __launch_bounds__(128) void mla_combine_kernel(const float* __restrict__ o_part,
                                                          const float* __restrict__ ml_part,
                                                          int n_splits, bf16* __restrict__ o_lat,
                                                          const long long* __restrict__ positions,
                                                          int pos_numel, int max_len, int split_len) {
  pdl_enter();
  const int b = blockIdx.x, h = blockIdx.y;
  const long long len = min(static_cast<long long>(max_len), positions[pos_numel == 1 ? 0 : b] + 1);
  if (len <= split_len) return;
  const float* ml = ml_part + (static_cast<long long>(b) * n_splits) * kHeads * 2;
  float M = -INFINITY;
  for (int s = 0; s < n_splits; ++s) {
    const float l = ml[(s * kHeads + h) * 2 + 1];
    if (l > 0.f) M = fmaxf(M, ml[(s * kHeads + h) * 2]);
  }
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float den = 0.f;
  const int d = threadIdx.x * 4;
  for (int s = 0; s < n_splits; ++s) {
    const float l = ml[(s * kHeads + h) * 2 + 1];
    if (!(l > 0.f)) continue;
    const float w = exp2f(ml[(s * kHeads + h) * 2] - M);
    den += w * l;
    const float4 v = *reinterpret_cast<const float4*>(
        o_part + ((static_cast<long long>(b) * n_splits + s) * kHeads + h) * kLatent + d);
    acc[0] += w * v.x; acc[1] += w * v.y; acc[2] += w * v.z; acc[3] += w * v.w;
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  uint2 o;
  o.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  o.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  *reinterpret_cast<uint2*>(o_lat + (static_cast<long long>(b) * kHeads + h) * kLatent + d) = o;
}

// ----------------------------------------------------------------------------
// Scratch for dsv2_mla_decode_noalloc: the split partials (o: [parts, 16, 512] then
// (m, l): [parts, 16, 2], parts = batch * n_splits <= kNoAllocMaxParts) in one
// fixed file-scope device array, so that entry point allocates nothing.  Every GPU
// that loads the library holds these 8.4 MB until the process exits.  Host code
// must not use the symbol as a pointer: its device address is looked up once per
// device with cudaGetSymbolAddress (below) and passed to the kernels.
// ----------------------------------------------------------------------------
constexpr int kNoAllocMaxParts = 256;
constexpr size_t kNoAllocFloats =
    static_cast<size_t>(kNoAllocMaxParts) * kHeads * (kLatent + 2);
static __device__ __align__(256) float g_mla_noalloc_scratch[kNoAllocFloats];
static float* g_mla_noalloc_ptr[128];

// Device address of the scratch array on the current device (looked up on first use).
cudaError_t mla_noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
  if (!g_mla_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_mla_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_mla_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_mla_noalloc_ptr[dev];
  return cudaSuccess;
}

constexpr size_t mla_decode_smem_bytes() {
  return kStages * kTileBytes + kQBytes + kChunks * kHeads * kSRedStride * sizeof(float) +
         kHeads * kPStride * sizeof(bf16) + kHeads * sizeof(float) + 2 * kStages * sizeof(uint64_t);
}

cudaError_t launch_mla_prep(const MlaPrepParams& p, int batch, cudaStream_t st) {
  launch_kernel(mla_prep_kernel, batch, 256, 0, st, p);
  return cudaGetLastError();
}

cudaError_t mla_decode_init() {
  return cudaFuncSetAttribute(mla_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(mla_decode_smem_bytes()));
}

cudaError_t launch_mla_decode(const MlaDecodeParams& p, const CUtensorMap& tm_kv, int batch,
                              cudaStream_t st) {
  launch_kernel(mla_decode_kernel, dim3(p.n_splits, batch), kMlaThreads, mla_decode_smem_bytes(), st, p,
                tm_kv);
  return cudaGetLastError();
}

cudaError_t launch_mla_combine(const MlaDecodeParams& p, int batch, cudaStream_t st) {
  // one split covers the whole cache: every row wrote its output directly; with
  // row_sync the decode kernel merged the splits itself
  if (static_cast<long long>(p.split_len) >= p.max_len || p.row_sync) return cudaSuccess;
  launch_kernel(mla_combine_kernel, dim3(batch, kHeads), 128, 0, st, p.o_part, p.ml_part, p.n_splits, p.o_lat, p.positions, p.pos_numel, p.max_len, p.split_len);
  return cudaGetLastError();
}

}  // namespace dsv2
