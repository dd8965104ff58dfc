// Batch family: dense split-K linear for decode batches (<= 256 tokens), weights resident.
//
// Replaces (Flash-DeepSeeek-V2-Lite):
//   attention_decode_batch.py:420-468   _batched_linear_kernel, for the q + kv-a
//                                        projection and o_proj of the batched decode step
//
// Y_s[token, n] = sum over the K blocks of split s of W[n, k] * X[token, k]  (fp32 partials,
// the consumer sums the S splits: mla_prep, the fused add + RMSNorm / router).
// At decode batch sizes these launches are short (the q + kv-a weights are 15 MB, o_proj 8
// MB) and their cost is latency: the time from the previous kernel's end to this one's
// last store.  So every CTA takes one (128-row tile, K split) item, and its whole weight
// slice (up to kSkWSlots 64-wide K blocks of 16 KB) is requested into
// shared memory before the programmatic-launch wait: weights are never written by earlier
// kernels, so their HBM reads overlap the previous kernel.  After the wait only the
// activation K blocks (L2-resident, written by the previous kernel) stream through a
// separate ring into tcgen05.mma (M = 128 weight rows, N = all tokens, fp32 accumulator in
// TMEM), and the epilogue stores the partial tile.  The grid covers about every SM (K
// splits = SMs / row tiles), so the activation re-reads of the row tiles are spread wide.
// Longer K than the weight slots hold (the dense MLP's down projection) streams the rest of
// the weights through the same slots.
//
// Warp roles (192 threads, one CTA per SM): warp 0 TMA producer, warp 1 TMEM allocator and
// MMA issuer, warps 2-5 epilogue (TMEM lane quadrant = warp % 4).  Every mbarrier wait is
// bounded (common.cuh).
#include "linear.cuh"

namespace dsv2 {

constexpr int kSkThreads = 192;
constexpr int kSkWSlots = 8;        // weight K blocks resident per CTA (8 x 16 KB)
constexpr int kSkMaxXStages = 8;
constexpr int kSkMaxTokens = 256;
constexpr int kSkStoreTokens = 32;   // tokens per TMA store box (32 x 128 fp32 = 16 KB)

struct SkShape {
  int w_slots;       // resident weight K blocks (<= kSkWSlots)
  int npad;          // tokens padded to 16
  int x_stages;      // activation ring depth
  int x_bytes;       // npad x 128 B per activation K block
  int tmem_cols;
};

__device__ __forceinline__ void epilogue_bar_sk() {  // the 4 epilogue warps only
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

__global__ __launch_bounds__(kSkThreads, 1) void linear_splitk_kernel(
    const LinearParams p, const __grid_constant__ CUtensorMap tmap_w,
    const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_y,
    const SkShape shp) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int WS = shp.w_slots;
  unsigned char* s_w = smem;                                   // WS x 16 KB
  unsigned char* s_x = smem + WS * kTcABytes;                  // x_stages x x_bytes
  uint64_t* w_full = reinterpret_cast<uint64_t*>(s_x + shp.x_stages * shp.x_bytes);
  uint64_t* w_empty = w_full + kSkWSlots;
  uint64_t* x_full = w_empty + kSkWSlots;
  uint64_t* x_empty = x_full + kSkMaxXStages;
  uint64_t* acc_bar = x_empty + kSkMaxXStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = gridDim.x;
  const int s = blockIdx.x;
  const int m0 = blockIdx.y * kTcM;
  const int nkb = p.k / kTcK;
  const int kb0 = s * nkb / S, kb1 = (s + 1) * nkb / S;
  const int nk = kb1 - kb0;
  const int npad = shp.npad;
  const int XS = shp.x_stages;

  if (threadIdx.x == 0) {
    for (int i = 0; i < WS; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], 1);
    }
    for (int i = 0; i < XS; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    mbar_init(acc_bar, 1);
    fence_mbar_init();
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, static_cast<uint32_t>(shp.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // the weight slice (or the first kSkWSlots K blocks of it) before the wait
      const int w_first = min(nk, WS);
      for (int i = 0; i < w_first; ++i) {
        mbar_arrive_expect_tx(&w_full[i], kTcABytes);
        tma_load_3d(smem_u32(s_w + i * kTcABytes), &tmap_w, &w_full[i], (kb0 + i) * kTcK, m0, 0);
      }
      pdl_enter();
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        // activation block i into ring slot i % XS (first pass: free)
        const int xs = i % XS;
        if (i >= XS && !mbar_wait(&x_empty[xs], ((i / XS) - 1) & 1)) ok = false;
        if (ok) {
          mbar_arrive_expect_tx(&x_full[xs], shp.x_bytes);
          tma_load_3d(smem_u32(s_x + xs * shp.x_bytes), &tmap_x, &x_full[xs], (kb0 + i) * kTcK, 0, 0);
        }
        // weight block i + WS into the slot block i frees (long K only)
        const int j = i + WS;
        if (ok && j < nk) {
          const int ws = j % WS;
          if (!mbar_wait(&w_empty[ws], ((j / WS) - 1) & 1)) ok = false;
          if (ok) {
            mbar_arrive_expect_tx(&w_full[ws], kTcABytes);
            tma_load_3d(smem_u32(s_w + ws * kTcABytes), &tmap_w, &w_full[ws], (kb0 + j) * kTcK, m0, 0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_bf16(kTcM, npad);
      for (int i = 0; i < nk; ++i) {
        const int ws = i % WS, xs = i % XS;
        if (!mbar_wait(&w_full[ws], (i / WS) & 1)) break;
        if (!mbar_wait(&x_full[xs], (i / XS) & 1)) break;
        tc_fence_after();
        const uint64_t da = sw128_kmajor_desc(smem_u32(s_w + ws * kTcABytes));
        const uint64_t db = sw128_kmajor_desc(smem_u32(s_x + xs * shp.x_bytes));
#pragma unroll
        for (int k = 0; k < kTcK / 16; ++k)
          tc_mma_bf16(tmem_base, da + 2 * k, db + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
        tc_commit(&x_empty[xs]);
        tc_commit(&w_empty[ws]);
      }
      // arrives once every MMA above has completed
      tc_commit(acc_bar);
    }
  } else {
    // epilogue: the partial tile of split s (fp32, token t, row n at y + s * y_split_stride +
    // t * y_row_stride + n) is staged in the drained shared memory, 32 tokens x 128 rows per
    // box, and written by TMA stores (rows past n_rows and tokens past n_tokens are clipped)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int ntok = p.n_tokens;
    float* stage = reinterpret_cast<float*>(smem);
    if (mbar_wait(acc_bar, 0)) {
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
      for (int c0 = 0; c0 < npad && c0 < ntok; c0 += kSkStoreTokens) {
        float a[16], b[16];
        tmem_ld16(tbase + c0, a);
        if (c0 + 16 < npad) tmem_ld16(tbase + c0 + 16, b);
        tmem_ld_wait();
        float* box = stage + c0 * kTcM;   // [32 tokens][128 rows]
#pragma unroll
        for (int j = 0; j < 16; ++j) box[j * kTcM + r] = a[j];
        if (c0 + 16 < npad) {
#pragma unroll
          for (int j = 0; j < 16; ++j) box[(16 + j) * kTcM + r] = b[j];
        }
        fence_proxy_async_smem();
        epilogue_bar_sk();
        if (warp == 2 && lane == 0) tma_store_3d(&tmap_y, smem_u32(box), m0, c0, s);
      }
      if (warp == 2 && lane == 0) {
        bulk_commit_group();
        bulk_wait_all();   // the stores are done (and shared memory read) before the CTA exits
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, static_cast<uint32_t>(shp.tmem_cols));
  }
}

// Weight slots for the longest split (all of it when it fits), activation stages in the rest
// of shared memory.
static SkShape sk_shape(int n_tokens, int max_kb_per_split) {
  SkShape s;
  s.w_slots = std::max(1, std::min(kSkWSlots, max_kb_per_split));
  s.npad = round_up(std::max(n_tokens, 1), 16);
  s.x_bytes = s.npad * 128;
  s.x_stages = std::min(kSkMaxXStages, (kTcSmemBudget - 2048 - s.w_slots * kTcABytes) / s.x_bytes);
  int c = 32;
  while (c < s.npad) c <<= 1;
  s.tmem_cols = c;
  return s;
}

static size_t sk_smem_bytes(const SkShape& s) {
  return 1024 + static_cast<size_t>(s.w_slots) * kTcABytes + static_cast<size_t>(s.x_stages) * s.x_bytes +
         (2 * kSkWSlots + 2 * kSkMaxXStages + 1) * sizeof(uint64_t) + 16;
}

cudaError_t linear_splitk_init() {
  return cudaFuncSetAttribute(linear_splitk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
}

// Dense launch of up to 256 tokens: grid (k_splits, row tiles), one item per CTA; fp32
// output, split s at y + s * y_split_stride (tmap_y: that output as {rows, tokens, splits}).
cudaError_t launch_linear_splitk(const LinearParams& p, const CUtensorMap& tmap_w, const CUtensorMap& tmap_x,
                                 const CUtensorMap& tmap_y, cudaStream_t st) {
  const int S = std::max(p.k_splits, 1);
  if (p.n_tokens < 1 || p.n_tokens > kSkMaxTokens || p.epilogue != kEpiStoreF32) return cudaErrorInvalidValue;
  const int nkb = p.k / kTcK;
  if (S > nkb) return cudaErrorInvalidValue;
  const SkShape shp = sk_shape(p.n_tokens, (nkb + S - 1) / S);
  if (shp.x_stages < 2) return cudaErrorInvalidValue;
  // the store boxes are staged in the drained weight slots and activation ring
  if ((shp.npad + kSkStoreTokens - 1) / kSkStoreTokens * kSkStoreTokens * kTcM * 4 >
      shp.w_slots * kTcABytes + shp.x_stages * shp.x_bytes)
    return cudaErrorInvalidValue;
  const dim3 grid(S, (p.n_rows + kTcM - 1) / kTcM);
  launch_kernel(linear_splitk_kernel, grid, kSkThreads, sk_smem_bytes(shp), st, p, tmap_w, tmap_x, tmap_y, shp);
  return cudaGetLastError();
}

}  // namespace dsv2
