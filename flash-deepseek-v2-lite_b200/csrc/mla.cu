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
// mla_decode_kernel: balanced persistent flash-decode, one CTA per SM.  The 32-position
// tiles of all rows form one stream cut into equal ranges (ragged batches keep every SM
// busy); a TMA producer warp keeps 5 tiles of the latent cache (128-byte swizzle) and the
// per-row query block in flight.  Warp-specialised: 4 score warps (mma.sync, 16 heads as
// M, 8 positions each, the whole query block in registers) hand bf16 P to 4 P @ V warps
// (128 latent dims each) through a double buffer, so the scores of one tile overlap the
// P @ V of the previous one.  A row inside one CTA's range writes o_lat directly; a row
// cut by a range boundary leaves (o, m, l) partials that the last of its CTAs merges
// (row tickets), so no second launch follows.
//
// mla_combine_kernel merges the split partials of the tcgen05 kernel (mla_tc.cu).
#include <algorithm>

#include "params.cuh"

namespace dsv2 {

constexpr int kHeads = 16;
constexpr int kLatent = 512;
constexpr int kRope = 64;
constexpr int kRow = kLatent + kRope;           // 576
constexpr int kRowBytes = kRow * 2;             // 1152
constexpr int kChunks = kRow / 64;              // 9 swizzle chunks of 64 dims
constexpr int kTile = 32;                       // positions per tile
constexpr int kStages = 5;                      // cache tiles in flight per CTA (one CTA per SM)
constexpr int kSegUnits = 2;                    // per-row cost in tile units (work balance)
constexpr int kTileBytes = kTile * kRowBytes;   // 36864
constexpr int kQBytes = kHeads * kRowBytes;     // 18432
constexpr int kPStride = kTile + 8;             // bf16 row stride of P
constexpr int kScoreWarps = 4;                  // per half of the 576 dims: 8 positions of a tile each
constexpr int kPvWarps = 4;                     // 128 latent dims each
constexpr int kProducerWarp = 2 * kScoreWarps + kPvWarps;      // warp 12
constexpr int kTicketWarp = kProducerWarp + 1;                 // warp 13
constexpr int kMergeThreads = kProducerWarp * 32;              // 384 compute threads
constexpr int kMlaThreads = kMergeThreads + 64;                // + the TMA producer and ticket warps
constexpr int kQSteps = kRow / 16 / 2;          // 18 mma k-steps of 16 dims per score half
static_assert(kMlaThreads / 32 <= 16, "per-warp prefix sums hold 16 warps");
constexpr int kMlaMaxCtas = 160;                // merge scratch: 2 x 16 x CTAs floats (in the drained ring)

// ----------------------------------------------------------------------------
// mla_prep: latent RMSNorm + RoPE + cache write for the new token, RoPE of q_pe
// ----------------------------------------------------------------------------

__global__ __launch_bounds__(256) void mla_prep_kernel(const MlaPrepParams p) {
  const int t = threadIdx.x;
  // the latent norm weights are never written by earlier kernels: load them before the wait
  float kw[8];
  if (t < 64) {
#pragma unroll
    for (int j = 0; j < 8; ++j) kw[j] = __bfloat162float(p.kv_norm_w[t * 8 + j]);
  }
  pdl_enter();
  __shared__ float red[8];
  __shared__ __align__(16) bf16 s_row[kHeads * 192 + kRow];  // this row of qkva, bf16
  const int b = blockIdx.x;
  // position, cache row and this thread's RoPE coefficients (every RoPE pair of thread t
  // has pair index t % 32) are fetched while the split-K partials are in flight
  const long long pos = p.positions[p.pos_numel == 1 ? 0 : b];
  const bool pos_ok = (pos >= 0 && pos < p.max_len && pos < p.rope_rows);
  const int cr = p.cache_rows ? p.cache_rows[b] : b;
  float rc = 0.f, rs = 0.f;
  if (pos_ok) {
    rc = p.cos_tab[pos * p.rope_stride + (t & 31)];
    rs = p.sin_tab[pos * p.rope_stride + (t & 31)];
  }
  // stage the row (summing fp32 split-K partials and rounding to bf16, like a bf16 linear)
  if (p.qkva_f32) {
    // 912 float4 per row over 256 threads: each thread sums its (up to 4) float4 columns,
    // four partials at a time with all their loads in flight, in order of the partial
    const float* src = reinterpret_cast<const float*>(p.qkva) + b * p.qkva_row_stride;
    constexpr int kN4 = (kHeads * 192 + kRow) / 4;
    constexpr int kPer = (kN4 + 255) / 256;
    float4 acc[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < p.qkva_parts; s0 += 4) {
      float4 v[4][kPer];
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          const int i = threadIdx.x + k * 256;
          if (s0 + q < p.qkva_parts && i < kN4)
            v[q][k] = __ldcg(reinterpret_cast<const float4*>(src + (s0 + q) * p.qkva_part_stride + 4 * i));
        }
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
          const int i = threadIdx.x + k * 256;
          if (s0 + q < p.qkva_parts && i < kN4) {
            acc[k].x += v[q][k].x; acc[k].y += v[q][k].y; acc[k].z += v[q][k].z; acc[k].w += v[q][k].w;
          }
        }
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = threadIdx.x + k * 256;
      if (i < kN4) {
        uint2 o;
        o.x = pack_bf16x2(acc[k].x, acc[k].y);
        o.y = pack_bf16x2(acc[k].z, acc[k].w);
        *reinterpret_cast<uint2*>(s_row + 4 * i) = o;
      }
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
  if (!pos_ok) {
    if (threadIdx.x == 0) set_device_error(kErrIndex);
    return;
  }
  if (cr < 0 || cr >= p.cache_batch) {
    if (threadIdx.x == 0) set_device_error(kErrIndex);
    return;
  }
  bf16* crow = p.cache + static_cast<long long>(cr) * p.cache_b_stride + pos * kRow;
  // latent RMSNorm: threads 0..63 own 8 elements each
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
    for (int j = 0; j < 4; ++j) op[j] = pack_bf16x2(v[2 * j] * inv * kw[2 * j], v[2 * j + 1] * inv * kw[2 * j + 1]);
    *reinterpret_cast<uint4*>(crow + t * 8) = o;
  }
  // RoPE pairs: 16 heads x 32 pairs of q_pe, plus 32 pairs of k_pe
  for (int i = t; i < (kHeads + 1) * 32; i += 256) {
    const int h = i >> 5, j = i & 31;
    const bf16* src = (h < kHeads) ? (row + h * 192 + 128 + 2 * j) : (row + kHeads * 192 + kLatent + 2 * j);
    const float e = __bfloat162float(src[0]), o = __bfloat162float(src[1]);
    const float re = e * rc - o * rs, im = o * rc + e * rs;
    const uint32_t packed = pack_bf16x2(re, im);
    if (h < kHeads)
      *reinterpret_cast<uint32_t*>(p.q_pe_out + (static_cast<long long>(b) * kHeads + h) * kRope + 2 * j) = packed;
    else
      *reinterpret_cast<uint32_t*>(crow + kLatent + 2 * j) = packed;
  }
}

// ----------------------------------------------------------------------------
// balanced persistent decode
// ----------------------------------------------------------------------------

// byte offset of (row r, 16-byte column c16) inside one 64-dim swizzle chunk of R rows
__device__ __forceinline__ uint32_t swz(int r, int c16) {
  return static_cast<uint32_t>(r * 128 + ((c16 ^ (r & 7)) << 4));
}

__device__ __forceinline__ void bar_half0() {   // the 4 softmax (first-half score) warps
  asm volatile("bar.sync 1, %0;" ::"n"(kScoreWarps * 32) : "memory");
}
__device__ __forceinline__ void bar_score() {   // all 8 score warps
  asm volatile("bar.sync 2, %0;" ::"n"(2 * kScoreWarps * 32) : "memory");
}
__device__ __forceinline__ void bar_all() {     // score + P @ V warps
  asm volatile("bar.sync 3, %0;" ::"n"(kMergeThreads) : "memory");
}

// Attended length of row b (0 .. max_len) and its number of 32-position tiles; a row
// with nothing to attend still owns one fully masked tile (its output is zero).
__device__ __forceinline__ int mla_row_len(const MlaDecodeParams& p, int b) {
  const long long pos = p.positions[p.pos_numel == 1 ? 0 : b];
  return static_cast<int>(max(0LL, min(static_cast<long long>(p.max_len), pos + 1)));
}
__device__ __forceinline__ int mla_tiles_of(int len) { return len > 0 ? (len + kTile - 1) / kTile : 1; }
// Units of row b in the work stream that is cut between the CTAs: its tiles plus kSegUnits
// units of fixed per-row cost (query block, softmax finish, output store), which come
// before the row's first tile, so that a CTA's share of rows counts in its share of work.
__device__ __forceinline__ int mla_units_of(int len) { return mla_tiles_of(len) + kSegUnits; }

// Bounded mbarrier wait that gives up at once when this CTA (or any kernel) has already
// recorded a failure, so that one lost wait cannot turn into a long chain of timeouts.
__device__ __forceinline__ bool mla_wait(uint64_t* bar, uint32_t parity, volatile int* s_abort) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023) == 1023 &&
        (*s_abort != 0 || *reinterpret_cast<volatile int*>(&g_device_error) != 0))
      break;
  }
  *s_abort = 1;
  set_device_error(kErrMbarTimeout);
  return false;
}

// Slot of the partial that CTA c holds for a row starting at tile S_b of the stream:
// 0 when the row is the CTA's first segment, 1 when it is its last one.
__device__ __forceinline__ int mla_slot(long long S_b, long long cta_start) { return S_b <= cta_start ? 0 : 1; }

// First tile of CTA c's range when T tiles are spread over n CTAs, and the CTA that owns tile t.
__device__ __forceinline__ long long mla_range_start(long long c, long long T, long long n) { return c * T / n; }
__device__ __forceinline__ long long mla_owner(long long t, long long T, long long n) {
  return ((t + 1) * n - 1) / T;
}

// The whole decode in one launch: the rows form one stream of T = sum_b (ceil(len_b / 32)
// + kSegUnits) units (each row's per-row cost, then its 32-position tiles), cut into equal
// contiguous ranges, one per CTA (one CTA per SM, so ragged batches keep every SM busy to
// the end, and a CTA that takes more rows takes fewer tiles).  Each CTA walks its
// range row by row ("segments"): a row that lies wholly inside the range is normalised
// and written to o_lat; a row cut by a range boundary leaves (o, m, l) partials in the
// CTA's slot 0 (first segment) or 1 (last segment), and the last of the row's CTAs to
// publish merges them (row_sync ticket) after its own range — no second launch.
//
// Warp roles (warp-specialised; the scores of tile t + 1 overlap P @ V of tile t):
//  - warps 0-7, scores: half h = warp / 4 covers k-steps [18h, 18h + 18) of the 36
//    (16 dims each) with its query slice in registers; warp w = warp % 4 owns positions
//    [8w, 8w + 8) of a tile.  Half 1 hands its partial scores to half 0 through shared
//    memory; half 0 exchanges the tile max per head (one 128-thread barrier), runs the
//    online softmax and hands bf16 P and the rescale factors to the P @ V warps through a
//    double buffer (mbarriers);
//  - warps 8-11, P @ V: warp v owns latent dims [128v, 128v + 128);
//  - warp 12, producer: TMA ring of 5 cache tiles and the per-segment query block;
//  - warp 13, tickets: publishes the CTA's (at most two) partial rows and records which
//    of them this CTA has to merge, off the compute warps' path.
__global__ __launch_bounds__(kMlaThreads, 1) void mla_decode_kernel(const MlaDecodeParams p,
                                                                   const __grid_constant__ CUtensorMap tm_kv,
                                                                   const __grid_constant__ CUtensorMap tm_qa,
                                                                   const __grid_constant__ CUtensorMap tm_qp) {
  extern __shared__ __align__(1024) unsigned char smem[];
  unsigned char* s_kv = smem;                                    // stages x 32 positions x 9 chunks x 128 B
  unsigned char* s_q = smem + kStages * kTileBytes;              // [2] x 9 chunks x 16 rows x 128 B
  bf16* s_p = reinterpret_cast<bf16*>(s_q + 2 * kQBytes);        // [2][16][kPStride]
  float* s_max = reinterpret_cast<float*>(s_p + 2 * kHeads * kPStride);  // [2][4][16]
  float* s_alpha = s_max + 2 * kScoreWarps * kHeads;             // [2][16]
  float* s_lsum = s_alpha + 2 * kHeads;                          // [4][16]
  float* s_fin = s_lsum + kScoreWarps * kHeads;                  // [2][16] 1/l of a finished segment
  float* s_part = s_fin + 2 * kHeads;                            // [2][4][32 lanes][4] second-half scores
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_part + 2 * kScoreWarps * 32 * 4);
  uint64_t* full_bar = bars;                                     // [kStages] cache tile landed
  uint64_t* empty_bar = full_bar + kStages;                      // [kStages] tile consumed
  uint64_t* p_full = empty_bar + kStages;                        // [2] P handed over
  uint64_t* p_empty = p_full + 2;                                // [2] P consumed
  uint64_t* q_full = p_empty + 2;                                // [2] query block landed
  uint64_t* q_empty = q_full + 2;                                // [2] query block in registers
  uint64_t* fin_full = q_empty + 2;                              // [2] 1/l of a segment published
  uint64_t* fin_empty = fin_full + 2;                            // [2] 1/l read
  uint64_t* tk_full = fin_empty + 2;                             // [2] partial of slot 0 / 1 written
  uint64_t* tk_done = tk_full + 2;                               // tickets taken, merge list final
  int* s_misc = reinterpret_cast<int*>(tk_done + 1);             // [16] named slots (below)
  int* s_wsum = s_misc + 16;                                     // [16] per-warp tile sums of the prefix
  long long* s_ll = reinterpret_cast<long long*>(s_misc + 32);   // [4]: S of the first row, pending S
  volatile int* s_abort = s_misc + 12;
  float* s_mrg = reinterpret_cast<float*>(s_kv);                 // merge scratch, once the ring is drained

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int B = p.batch;
  const bool early = p.inputs_prior != 0;
  // one row whose partials are left for the consumer to merge: no tickets, no o_lat
  const bool defer = p.part_count != nullptr;

  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&tm_kv);
    prefetch_tmap(&tm_qa);
    prefetch_tmap(&tm_qp);
  }
  // positions may come from the previous launch unless inputs_prior
  if (!early) pdl_enter();
  if (tid == 0) {
    for (int st = 0; st < kStages; ++st) {
      mbar_init(&full_bar[st], 1);
      mbar_init(&empty_bar[st], 2 * kScoreWarps + kPvWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], kScoreWarps);
      mbar_init(&p_empty[i], kPvWarps);
      mbar_init(&fin_full[i], 1);
      mbar_init(&fin_empty[i], kPvWarps);
      mbar_init(&tk_full[i], 1 + kPvWarps);
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 2 * kScoreWarps);
    }
    mbar_init(tk_done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }

  // --- unit prefix over the rows (every CTA computes the same one): T = all units, then
  // this CTA's range [start, end) and its first row b0 (S_b0 <= start < S_b0 + units_b0).
  // One pass when the batch fits the block (the usual case), else two.
  long long T = 0, start = 0, end = 0, c = blockIdx.x, n_cta = 0;
  const long long min_tpc = max(1, p.split_len / kTile);
  int nt_mine = 0, incl = 0;
  for (int base = 0; base < B; base += kMlaThreads) {
    const int b = base + tid;
    const int nt = b < B ? mla_units_of(mla_row_len(p, b)) : 0;
    int v = nt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    if (lane == 31) s_wsum[warp] = v;
    if (base == 0) {
      nt_mine = nt;
      incl = v;
    }
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kMlaThreads / 32; ++w) T += s_wsum[w];
    __syncthreads();
  }
  n_cta = min(static_cast<long long>(gridDim.x), (T + min_tpc - 1) / min_tpc);
  if (c >= n_cta) {
    if (early) pdl_enter();
    return;
  }
  start = mla_range_start(c, T, n_cta);
  end = mla_range_start(c + 1, T, n_cta);
  if (B <= kMlaThreads) {
    // s_wsum still holds the warp totals of the only chunk
    long long off = 0;
#pragma unroll
    for (int w = 0; w < kMlaThreads / 32; ++w)
      if (w < warp) off += s_wsum[w];
    const long long S = off + incl - nt_mine;
    if (tid < B && S <= start && start < S + nt_mine) {
      s_ll[0] = S;
      s_misc[10] = tid;
    }
  } else {
    long long run = 0;
    for (int base = 0; base < B; base += kMlaThreads) {
      const int b = base + tid;
      const int nt = b < B ? mla_units_of(mla_row_len(p, b)) : 0;
      int v = nt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (lane == 31) s_wsum[warp] = v;
      __syncthreads();
      long long off = run, total = 0;
#pragma unroll
      for (int w = 0; w < kMlaThreads / 32; ++w) {
        if (w < warp) off += s_wsum[w];
        total += s_wsum[w];
      }
      const long long S = off + v - nt;
      if (b < B && S <= start && start < S + nt) {
        s_ll[0] = S;
        s_misc[10] = b;
      }
      __syncthreads();
      run += total;
      if (run > start) break;  // uniform across the block
    }
  }
  __syncthreads();
  const long long S0 = s_ll[0];
  const int b0 = s_misc[10];

  if (warp == kProducerWarp) {
    // ================= producer warp: cache tiles and query blocks
    if (lane == 0) {
      bool waited = !early, ok = true;
      int early_rows[kStages];
      int q_issued = 0, seg = 0;
      long long g = 0;
      auto issue_q = [&](int k, int row) {
        // query buffer k & 1 (two segments in flight)
        const int qb = k & 1;
        if (k >= 2 && ok) ok = mla_wait(&q_empty[qb], static_cast<uint32_t>(((k >> 1) - 1) & 1), s_abort);
        if (!ok) return;
        unsigned char* dq = s_q + qb * kQBytes;
        mbar_arrive_expect_tx(&q_full[qb], kQBytes);
        for (int ch = 0; ch < kLatent / 64; ++ch)
          tma_load_3d(smem_u32(dq + ch * (kHeads * 128)), &tm_qa, &q_full[qb], ch * 64, 0, row);
        tma_load_3d(smem_u32(dq + (kLatent / 64) * (kHeads * 128)), &tm_qp, &q_full[qb], 0, 0, row);
      };
      long long S = S0;
      for (int b = b0; S + kSegUnits < end && b < B; ++b, ++seg) {
        const int len = mla_row_len(p, b), nt = mla_tiles_of(len);
        const long long St = S + kSegUnits;   // stream position of the row's first tile
        const int j0 = static_cast<int>(max(0LL, start - St)), j1 = static_cast<int>(min(static_cast<long long>(nt), end - St));
        // cache row read by query row b (prefill: many query rows share one sequence)
        int crow_b = p.cache_rows ? p.cache_rows[b] : b;
        if (crow_b < 0 || crow_b >= p.cache_batch) {
          set_device_error(kErrIndex);
          crow_b = 0;
        }
        if (seg < kStages) early_rows[seg] = b;
        for (int j = j0; j < j1; ++j, ++g) {
          if (!waited && g >= kStages) {
            pdl_enter();
            waited = true;
          }
          if (waited) {
            for (; q_issued <= seg; ++q_issued) issue_q(q_issued, q_issued < kStages ? early_rows[q_issued] : b);
          }
          const int st = static_cast<int>(g % kStages);
          if (g >= kStages && ok) ok = mla_wait(&empty_bar[st], static_cast<uint32_t>(((g / kStages) - 1) & 1), s_abort);
          if (!ok) continue;
          mbar_arrive_expect_tx(&full_bar[st], kTileBytes);
          for (int ch = 0; ch < kChunks; ++ch)
            tma_load_3d(smem_u32(s_kv + st * kTileBytes + ch * (kTile * 128)), &tm_kv, &full_bar[st], ch * 64,
                        j * kTile, crow_b);
        }
        S += nt + kSegUnits;
      }
      if (!waited) pdl_enter();
      for (; q_issued < seg; ++q_issued) issue_q(q_issued, early_rows[q_issued]);
      // every issued copy has landed before the CTA may exit (consumed ones at once; after
      // a failed wait, the ones nobody consumed)
      for (int st = 0; st < kStages && st < g; ++st) {
        const long long last = g - 1 - ((g - 1 - st) % kStages);
        for (uint32_t i = 0; i < (1u << 20) && !mbar_try_wait(&full_bar[st], static_cast<uint32_t>((last / kStages) & 1)); ++i) {
        }
      }
      for (int k = max(0, seg - 2); k < seg; ++k)
        for (uint32_t i = 0; i < (1u << 20) && !mbar_try_wait(&q_full[k & 1], static_cast<uint32_t>((k >> 1) & 1)); ++i) {
        }
    } else if (early) {
      pdl_enter();
    }
    return;
  }

  if (warp == kTicketWarp) {
    // ================= ticket warp: publish the CTA's partial rows (slot 0: a row that
    // began before this range, slot 1: a row that ends after it)
    if (early) pdl_enter();
    if (lane == 0) {
      int n_pend = 0;
      long long S = S0;
      for (int b = b0; !defer && S + kSegUnits < end && b < B; ++b) {
        const int nt = mla_tiles_of(mla_row_len(p, b));
        const long long St = S + kSegUnits;
        if (!((St >= start) && (St + nt <= end))) {
          const int slot = mla_slot(S, start);
          if (mla_wait(&tk_full[slot], 0, s_abort)) {
            const int n_seg = static_cast<int>(mla_owner(St + nt - 1, T, n_cta) - mla_owner(St, T, n_cta) + 1);
            __threadfence();   // the partial (written by other warps, ordered by the mbarrier) first
            const int t = atomicAdd(&p.row_sync[b], 1);
            if (t == n_seg - 1) {
              p.row_sync[b] = 0;
              __threadfence();
              s_misc[13 + n_pend] = b;
              s_misc[5 + n_pend] = nt;
              s_ll[2 + n_pend] = S;
              ++n_pend;
            }
          }
        }
        S += nt + kSegUnits;
      }
      s_misc[15] = n_pend;
      mbar_arrive(tk_done);
    }
    return;
  }

  // ================= compute warps
  if (early) pdl_enter();
  // deferred merge (one row): the consumer merges slot 0 of CTAs [first, first + count),
  // the CTAs that hold tiles of the row (a first range of per-row units alone holds none)
  if (defer && c == 0 && tid == 0) {
    const long long c_first = mla_owner(kSegUnits, T, n_cta), c_last = mla_owner(T - 1, T, n_cta);
    p.part_count[0] = static_cast<int>(c_first);
    p.part_count[1] = static_cast<int>(c_last - c_first + 1);
  }
  const int gq = lane >> 2, tq = lane & 3;
  const int mi = lane >> 3, ri = lane & 7;
  long long g = 0;   // tiles of this CTA so far (ring slot, P buffer)
  int seg = 0;
  long long S = S0;

  if (warp < 2 * kScoreWarps) {
    // ============ score warps
    const int half = warp / kScoreWarps, sw = warp % kScoreWarps;
    for (int b = b0; S + kSegUnits < end && b < B; ++b, ++seg) {
      const int len = mla_row_len(p, b), nt = mla_tiles_of(len);
      const long long St = S + kSegUnits;
      const int j0 = static_cast<int>(max(0LL, start - St)), j1 = static_cast<int>(min(static_cast<long long>(nt), end - St));
      const bool complete = !defer && (St >= start) && (St + nt <= end);
      // this half's 16 x 288 query slice as 18 A fragments (k-steps of 16 dims)
      const int qb = seg & 1;
      mla_wait(&q_full[qb], static_cast<uint32_t>((seg >> 1) & 1), s_abort);
      uint32_t qa[kQSteps][4];
#pragma unroll
      for (int i = 0; i < kQSteps; ++i) {
        const int ks = half * kQSteps + i;
        const int row = (mi & 1) * 8 + ri;
        const int c16 = (ks & 3) * 2 + (mi >> 1);
        ldmatrix_x4(smem_u32(s_q + qb * kQBytes + (ks >> 2) * (kHeads * 128) + swz(row, c16)), qa[i][0], qa[i][1],
                    qa[i][2], qa[i][3]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&q_empty[qb]);
      float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;   // heads gq, gq + 8 (half 0)

      for (int j = j0; j < j1; ++j, ++g) {
        const int st = static_cast<int>(g % kStages);
        const int buf = static_cast<int>(g & 1);
        mla_wait(&full_bar[st], static_cast<uint32_t>((g / kStages) & 1), s_abort);
        const unsigned char* kv = s_kv + st * kTileBytes;
        // S[16 heads, 8 positions] over this half's dims; B fragments of two k-steps per ldmatrix
        float acc[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
        for (int kp = 0; kp < kQSteps / 2; ++kp) {
          const int i = 2 * kp, ks = half * kQSteps + i;
          uint32_t b0r, b1r, b2r, b3r;
          ldmatrix_x4(smem_u32(kv + (ks >> 2) * (kTile * 128) + swz(8 * sw + ri, (ks & 3) * 2 + mi)), b0r, b1r,
                      b2r, b3r);
          mma_bf16_16816(acc[0], qa[i], b0r, b1r);
          mma_bf16_16816(acc[1], qa[i + 1], b2r, b3r);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[st]);  // this warp is done with K
        float s00 = acc[0][0] + acc[1][0];
        float s01 = acc[0][1] + acc[1][1];
        float s10 = acc[0][2] + acc[1][2];
        float s11 = acc[0][3] + acc[1][3];
        float4* sp = reinterpret_cast<float4*>(s_part) + (buf * kScoreWarps + sw) * 32 + lane;
        if (half == 1) *sp = make_float4(s00, s01, s10, s11);
        bar_score();
        if (half == 1) continue;
        {
          const float4 o = *sp;
          s00 += o.x; s01 += o.y; s10 += o.z; s11 += o.w;
        }
        const int t0 = j * kTile + 8 * sw + 2 * tq;
        const bool v0 = t0 < len, v1 = t0 + 1 < len;
        s00 = v0 ? s00 * p.scale_log2 : -INFINITY;
        s01 = v1 ? s01 * p.scale_log2 : -INFINITY;
        s10 = v0 ? s10 * p.scale_log2 : -INFINITY;
        s11 = v1 ? s11 * p.scale_log2 : -INFINITY;
        float x0 = fmaxf(s00, s01), x1 = fmaxf(s10, s11);
        x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, 1));
        x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, 1));
        x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, 2));
        x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, 2));
        float* smx = s_max + buf * (kScoreWarps * kHeads);
        if (tq == 0) {
          smx[sw * kHeads + gq] = x0;
          smx[sw * kHeads + gq + 8] = x1;
        }
        bar_half0();
#pragma unroll
        for (int w = 0; w < kScoreWarps; ++w) {
          x0 = fmaxf(x0, smx[w * kHeads + gq]);
          x1 = fmaxf(x1, smx[w * kHeads + gq + 8]);
        }
        const float n0 = fmaxf(m0, x0), n1 = fmaxf(m1, x1);
        const float u0 = (n0 == -INFINITY) ? 0.f : n0, u1 = (n1 == -INFINITY) ? 0.f : n1;
        const float a0 = exp2f(m0 - u0), a1 = exp2f(m1 - u1);
        const float p00 = exp2f(s00 - u0), p01 = exp2f(s01 - u0);
        const float p10 = exp2f(s10 - u1), p11 = exp2f(s11 - u1);
        l0 = l0 * a0 + p00 + p01;
        l1 = l1 * a1 + p10 + p11;
        m0 = n0;
        m1 = n1;
        // hand P (bf16) and the rescale factors to the P @ V warps
        if (g >= 2) mla_wait(&p_empty[buf], static_cast<uint32_t>(((g >> 1) - 1) & 1), s_abort);
        bf16* pb = s_p + buf * (kHeads * kPStride);
        *reinterpret_cast<uint32_t*>(pb + gq * kPStride + 8 * sw + 2 * tq) = pack_bf16x2(p00, p01);
        *reinterpret_cast<uint32_t*>(pb + (gq + 8) * kPStride + 8 * sw + 2 * tq) = pack_bf16x2(p10, p11);
        if (sw == 0 && tq == 0) {
          s_alpha[buf * kHeads + gq] = a0;
          s_alpha[buf * kHeads + gq + 8] = a1;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[buf]);
      }

      if (half == 0) {
        // --- segment end: l per head (this thread's quad, then the 4 warps); warp 0
        // publishes 1/l (and m, l of a partial row) without waiting for the other roles
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
        if (tq == 0) {
          s_lsum[sw * kHeads + gq] = l0;
          s_lsum[sw * kHeads + gq + 8] = l1;
        }
        bar_half0();
        if (sw == 0) {
          const int fb = seg & 1;
          if (tq == 0) {
            float L0 = 0.f, L1 = 0.f;
#pragma unroll
            for (int w = 0; w < kScoreWarps; ++w) {
              L0 += s_lsum[w * kHeads + gq];
              L1 += s_lsum[w * kHeads + gq + 8];
            }
            if (seg >= 2) mla_wait(&fin_empty[fb], static_cast<uint32_t>(((seg >> 1) - 1) & 1), s_abort);
            s_fin[fb * kHeads + gq] = L0 > 0.f ? 1.f / L0 : 0.f;
            s_fin[fb * kHeads + gq + 8] = L1 > 0.f ? 1.f / L1 : 0.f;
            if (!complete) {
              float* ml = p.ml_part + (c * 2 + mla_slot(S, start)) * kHeads * 2;
              ml[gq * 2] = m0;
              ml[gq * 2 + 1] = L0;
              ml[(gq + 8) * 2] = m1;
              ml[(gq + 8) * 2 + 1] = L1;
            }
          }
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&fin_full[fb]);
            if (!complete) mbar_arrive(&tk_full[mla_slot(S, start)]);
          }
        }
        // s_lsum is rewritten at the next segment end, after that segment's tile barriers
      }
      S += nt + kSegUnits;
    }
  } else {
    // ============ P @ V warps
    const int pv = warp - 2 * kScoreWarps;   // latent dims [128 pv, 128 pv + 128)
    for (int b = b0; S + kSegUnits < end && b < B; ++b, ++seg) {
      const int len = mla_row_len(p, b), nt = mla_tiles_of(len);
      const long long St = S + kSegUnits;
      const int j0 = static_cast<int>(max(0LL, start - St)), j1 = static_cast<int>(min(static_cast<long long>(nt), end - St));
      const bool complete = !defer && (St >= start) && (St + nt <= end);
      float o_acc[16][4];
#pragma unroll
      for (int i = 0; i < 16; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;
      for (int j = j0; j < j1; ++j, ++g) {
        const int st = static_cast<int>(g % kStages);
        const int buf = static_cast<int>(g & 1);
        mla_wait(&p_full[buf], static_cast<uint32_t>((g >> 1) & 1), s_abort);
        mla_wait(&full_bar[st], static_cast<uint32_t>((g / kStages) & 1), s_abort);
        const unsigned char* kv = s_kv + st * kTileBytes;
        const float a0 = s_alpha[buf * kHeads + gq], a1 = s_alpha[buf * kHeads + gq + 8];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          o_acc[i][0] *= a0; o_acc[i][1] *= a0;
          o_acc[i][2] *= a1; o_acc[i][3] *= a1;
        }
        const bf16* pb = s_p + buf * (kHeads * kPStride);
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          uint32_t pa[4];
          ldmatrix_x4(smem_u32(pb + ((mi & 1) * 8 + ri) * kPStride + kk * 16 + (mi >> 1) * 8), pa[0], pa[1], pa[2],
                      pa[3]);
#pragma unroll
          for (int np = 0; np < 8; ++np) {
            const int r = kk * 16 + (mi & 1) * 8 + ri;
            const int c16 = (np & 3) * 2 + (mi >> 1);
            uint32_t b0r, b1r, b2r, b3r;
            ldmatrix_x4_trans(smem_u32(kv + (2 * pv + (np >> 2)) * (kTile * 128) + swz(r, c16)), b0r, b1r, b2r,
                              b3r);
            mma_bf16_16816(o_acc[2 * np], pa, b0r, b1r);
            mma_bf16_16816(o_acc[2 * np + 1], pa, b2r, b3r);
          }
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&empty_bar[st]);
          mbar_arrive(&p_empty[buf]);
        }
      }
      const int fb = seg & 1;
      mla_wait(&fin_full[fb], static_cast<uint32_t>((seg >> 1) & 1), s_abort);
      if (complete) {
        const float i0 = s_fin[fb * kHeads + gq], i1 = s_fin[fb * kHeads + gq + 8];
        bf16* ob = p.o_lat + static_cast<long long>(b) * kHeads * kLatent;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int d = pv * 128 + i * 8 + 2 * tq;
          *reinterpret_cast<uint32_t*>(ob + gq * kLatent + d) = pack_bf16x2(o_acc[i][0] * i0, o_acc[i][1] * i0);
          *reinterpret_cast<uint32_t*>(ob + (gq + 8) * kLatent + d) =
              pack_bf16x2(o_acc[i][2] * i1, o_acc[i][3] * i1);
        }
      } else {
        float* op = p.o_part + (c * 2 + mla_slot(S, start)) * kHeads * kLatent;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int d = pv * 128 + i * 8 + 2 * tq;
          *reinterpret_cast<float2*>(op + gq * kLatent + d) = make_float2(o_acc[i][0], o_acc[i][1]);
          *reinterpret_cast<float2*>(op + (gq + 8) * kLatent + d) = make_float2(o_acc[i][2], o_acc[i][3]);
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&fin_empty[fb]);
        if (!complete) mbar_arrive(&tk_full[mla_slot(S, start)]);
      }
      S += nt + kSegUnits;
    }
  }

  // ================= merges of the rows this CTA published last (all compute warps)
  mla_wait(tk_done, 0, s_abort);
  const int n_pend = min(s_misc[15], 2);
  for (int pi = 0; pi < n_pend; ++pi) {
    const int b = s_misc[13 + pi], nt = s_misc[5 + pi];
    const long long Sb = s_ll[2 + pi];
    const long long c_first = mla_owner(Sb + kSegUnits, T, n_cta), c_last = mla_owner(Sb + kSegUnits + nt - 1, T, n_cta);
    const int n_seg = static_cast<int>(c_last - c_first + 1);
    float* s_m = s_mrg;
    float* s_l = s_mrg + kHeads * n_seg;
    auto part_index = [&](int k) -> long long {
      const long long cc = c_first + k;
      return cc * 2 + ((k == 0) ? mla_slot(Sb, mla_range_start(cc, T, n_cta)) : 0);
    };
    bar_all();   // s_mrg (the drained ring) is free; the previous merge is done with it
    for (int i = tid; i < kHeads * n_seg; i += kMergeThreads) {
      const int h = i / n_seg, k = i % n_seg;
      const long long pk = part_index(k);
      s_m[i] = __ldcg(p.ml_part + (pk * kHeads + h) * 2);
      s_l[i] = __ldcg(p.ml_part + (pk * kHeads + h) * 2 + 1);
    }
    bar_all();
    if (tid < kHeads) {
      // w_k = 2^(m_k - M) / sum_k 2^(m_k - M) l_k
      float M = -INFINITY;
      for (int k = 0; k < n_seg; ++k)
        if (s_l[tid * n_seg + k] > 0.f) M = fmaxf(M, s_m[tid * n_seg + k]);
      float den = 0.f;
      for (int k = 0; k < n_seg; ++k) {
        const float l = s_l[tid * n_seg + k];
        const float w = l > 0.f ? exp2f(s_m[tid * n_seg + k] - M) : 0.f;
        s_m[tid * n_seg + k] = w;
        den += w * l;
      }
      const float inv = den > 0.f ? 1.f / den : 0.f;
      for (int k = 0; k < n_seg; ++k) s_m[tid * n_seg + k] *= inv;
    }
    bar_all();
    constexpr int kItems = kHeads * kLatent / 4;
    constexpr int kPer = (kItems + kMergeThreads - 1) / kMergeThreads;   // 6
    float4 acc[kPer];
#pragma unroll
    for (int r = 0; r < kPer; ++r) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    // two partials per round: 2 x 6 independent 16-byte loads in flight per thread
    for (int k = 0; k < n_seg; k += 2) {
      const bool two = k + 1 < n_seg;
      const float4* o0 = reinterpret_cast<const float4*>(p.o_part + part_index(k) * kHeads * kLatent);
      const float4* o1 = two ? reinterpret_cast<const float4*>(p.o_part + part_index(k + 1) * kHeads * kLatent) : o0;
      float4 v0[kPer], v1[kPer];
#pragma unroll
      for (int r = 0; r < kPer; ++r) {
        const int i = tid + r * kMergeThreads;
        const bool in = i < kItems;
        v0[r] = in ? __ldcg(o0 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        v1[r] = (in && two) ? __ldcg(o1 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int r = 0; r < kPer; ++r) {
        const int i = tid + r * kMergeThreads;
        const int h = (i < kItems ? i : 0) / (kLatent / 4);
        const float w0 = i < kItems ? s_m[h * n_seg + k] : 0.f;
        const float w1 = (i < kItems && two) ? s_m[h * n_seg + k + 1] : 0.f;
        acc[r].x += w0 * v0[r].x + w1 * v1[r].x;
        acc[r].y += w0 * v0[r].y + w1 * v1[r].y;
        acc[r].z += w0 * v0[r].z + w1 * v1[r].z;
        acc[r].w += w0 * v0[r].w + w1 * v1[r].w;
      }
    }
    bf16* ob = p.o_lat + static_cast<long long>(b) * kHeads * kLatent;
#pragma unroll
    for (int r = 0; r < kPer; ++r) {
      const int i = tid + r * kMergeThreads;
      if (i < kItems) {
        uint2 o;
        o.x = pack_bf16x2(acc[r].x, acc[r].y);
        o.y = pack_bf16x2(acc[r].z, acc[r].w);
        *reinterpret_cast<uint2*>(ob + 4 * i) = o;
      }
    }
  }
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
// Scratch for dsv2_mla_decode_noalloc: the partials (o: [parts, 16, 512] then
// (m, l): [parts, 16, 2], two parts per CTA, kNoAllocMaxParts parts) and the row
// tickets (int32[kNoAllocMaxRows], zero from load time; every call that completes leaves
// them zero, and clearing a nonzero device error word zeroes them after one that gave up)
// in one fixed file-scope device array, so that entry point allocates nothing.  Every
// GPU that loads the library holds these 8.4 MB until the process exits.  Host code
// must not use the symbol as a pointer: its device address is looked up once per
// device with cudaGetSymbolAddress (below) and passed to the kernels.
// ----------------------------------------------------------------------------
constexpr int kNoAllocMaxParts = 256;
constexpr int kNoAllocMaxRows = 4096;
constexpr size_t kNoAllocFloats =
    static_cast<size_t>(kNoAllocMaxParts) * kHeads * (kLatent + 2) + kNoAllocMaxRows;
constexpr size_t kNoAllocTicketOffset = static_cast<size_t>(kNoAllocMaxParts) * kHeads * (kLatent + 2);
static __device__ __align__(256) float g_mla_noalloc_scratch[kNoAllocFloats];

// Device address of the scratch array on the current device.  Called once per device by
// the library's per-device set-up (under its lock); the result is cached there.
cudaError_t mla_noalloc_lookup(float** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_mla_noalloc_scratch);
  if (e != cudaSuccess) return e;
  *out = static_cast<float*>(p);
  return cudaSuccess;
}

constexpr size_t mla_decode_smem_bytes() {
  return kStages * kTileBytes + 2 * kQBytes + 2 * kHeads * kPStride * sizeof(bf16) +
         (2 * kScoreWarps * kHeads + 2 * kHeads + kScoreWarps * kHeads + 2 * kHeads + 2 * kScoreWarps * 32 * 4) *
             sizeof(float) +
         (2 * kStages + 15) * sizeof(uint64_t) + 32 * sizeof(int) + 4 * sizeof(long long);
}
static_assert(mla_decode_smem_bytes() <= 232448, "latent-attention shared memory exceeds 227 KB");
static_assert(2 * kHeads * kMlaMaxCtas * sizeof(float) <= kStages * kTileBytes, "merge scratch exceeds the ring");

cudaError_t launch_mla_prep(const MlaPrepParams& p, int batch, cudaStream_t st) {
  launch_kernel(mla_prep_kernel, batch, 256, 0, st, p);
  return cudaGetLastError();
}

cudaError_t mla_decode_init() {
  return cudaFuncSetAttribute(mla_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(mla_decode_smem_bytes()));
}

// CTAs of the balanced decode: one per SM, at most one per tile of the largest possible
// stream, and two partial slots each within the caller's batch * n_splits slots.
int mla_decode_grid(const MlaDecodeParams& p, int num_sms, long long part_slots) {
  const long long tiles = static_cast<long long>(p.batch) * ((p.max_len + kTile - 1) / kTile);
  const long long slots = part_slots / 2;
  long long g = num_sms;
  g = std::min<long long>(g, kMlaMaxCtas);
  g = std::min<long long>(g, tiles);
  g = std::min<long long>(g, slots);
  return static_cast<int>(std::max<long long>(g, 0));
}

cudaError_t launch_mla_decode(const MlaDecodeParams& p, const CUtensorMap& tm_kv, const CUtensorMap& tm_qa,
                              const CUtensorMap& tm_qp, int grid, cudaStream_t st) {
  launch_kernel(mla_decode_kernel, grid, kMlaThreads, mla_decode_smem_bytes(), st, p, tm_kv, tm_qa, tm_qp);
  return cudaGetLastError();
}

cudaError_t launch_mla_combine(const MlaDecodeParams& p, int batch, cudaStream_t st) {
  // one split covers the whole cache: every row wrote its output directly; with
  // row_sync the decode kernel merged the splits itself
  if (static_cast<long long>(p.split_len) >= p.max_len) return cudaSuccess;
  launch_kernel(mla_combine_kernel, dim3(batch, kHeads), 128, 0, st, p.o_part, p.ml_part, p.n_splits, p.o_lat, p.positions, p.pos_numel, p.max_len, p.split_len);
  return cudaGetLastError();
}

}  // namespace dsv2
