// "Batch" kernel family: weight-streaming GEMM on the 5th-generation tensor cores.
//
// Replaces (Flash-DeepSeeek-V2-Lite):
//   attention_decode_batch.py:420-468   _batched_linear_kernel (row-batched attention linears)
//   moe_batch.py:151-307                _grouped_gate_up_swiglu_kernel / _grouped_down_partial_kernel
// and the cuBLAS GEMMs of the shared experts / dense MLP that src/run.py:340-361 leaves
// around silu_mul.
//
// Y[token, n] = sum_k W[n, k] * X[token, k].  Weights are the A operand (M = 128
// weight rows per tile, K-major), tokens are the B operand (N = up to 256 tokens,
// padded to a multiple of 16), the fp32 accumulator lives in TMEM.  Decode is
// weight-bandwidth bound, so each 128-row weight tile is streamed from HBM exactly
// once per 256 tokens; TMA moves 64-wide K slices of W and X (128-byte swizzle)
// through a multi-stage shared-memory ring.
//
// Warp roles (192 threads, persistent CTAs, one per SM):
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocator + tcgen05.mma issuer (one elected lane)
//   warps 2..5  epilogue: tcgen05.ld of the accumulator, fused SwiGLU / route-weight
//               scaling / bf16 or fp32 store (TMEM lane quadrant = warp % 4)
// SwiGLU tiles issue two MMAs per K step (gate rows and the matching up rows) into
// two TMEM accumulators, so silu(gate) * up is computed in registers.
//
// Grouped (MoE) mode: group g owns rows [group_offsets[g], group_offsets[g+1]) of X
// (activations gathered in expert order), read on the device; work items of empty
// groups are skipped by every role in the same order, so the grid is fixed and
// CUDA-graph safe.  All mbarrier waits are bounded (see common.cuh).
#include <cudaTypedefs.h>

#include "linear.cuh"

namespace dsv2 {

constexpr int kTcThreads = 192;
constexpr int kTcM = 128;
constexpr int kTcK = 64;                 // K per stage (one 128-byte swizzle row)
constexpr int kTcNMax = 256;
constexpr int kTcABytes = kTcM * 128;    // 16 KB
constexpr int kTcBoxRows = 16;           // token rows per TMA box
constexpr int kTcSmemBudget = 200 * 1024;

struct TcShape {
  int stages;
  int b_bytes;       // B region per stage (n_max_pad * 128)
  int stage_bytes;   // A (+A_up) + B
  int tmem_cols;
};

__host__ __device__ inline int round_up(int a, int b) { return (a + b - 1) / b * b; }

template <bool SWIGLU>
__global__ __launch_bounds__(kTcThreads, 1) void linear_tc_kernel(
    const LinearParams p, const __grid_constant__ CUtensorMap tmap_w,
    const __grid_constant__ CUtensorMap tmap_x, const TcShape shp, int mt_count, int nt_count,
    int up_rows, int x_grouped) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + shp.stages * shp.stage_bytes);
  uint64_t* empty_bar = full_bar + shp.stages;
  uint64_t* tfull_bar = empty_bar + shp.stages;
  uint64_t* tempty_bar = tfull_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < shp.stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, 128);
    *abort_flag = 0;
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

  const int n_groups = p.n_groups;
  const long long total_items = static_cast<long long>(n_groups) * mt_count * nt_count;
  const int nkb = p.k / kTcK;
  const int a_tiles = SWIGLU ? 2 : 1;

  // decode an item into (group, m tile, n tile, first route, tokens); false if empty
  auto decode = [&](long long it, int& g, int& mt, int& nt, int& r0, int& ntok) -> bool {
    nt = static_cast<int>(it % nt_count);
    long long rest = it / nt_count;
    mt = static_cast<int>(rest % mt_count);
    g = static_cast<int>(rest / mt_count);
    int cnt;
    if (p.group_offsets) {
      r0 = p.group_offsets[g];
      cnt = p.group_offsets[g + 1] - r0;
    } else {
      r0 = 0;
      cnt = p.n_tokens;
    }
    ntok = min(kTcNMax, cnt - nt * kTcNMax);
    const int cap = shp.b_bytes / 128;
    if (ntok > cap) {  // more tokens than the host-side bound: clamp and flag
      set_device_error(kErrIndex);
      ntok = cap;
    }
    return ntok > 0;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (long long it = blockIdx.x; it < total_items && !*abort_flag; it += gridDim.x) {
        int g, mt, nt, r0, ntok;
        if (!decode(it, g, mt, nt, r0, ntok)) continue;
        const int npad = round_up(ntok, 16);
        const int nbox = npad / kTcBoxRows;
        const int xrow0 = r0 + nt * kTcNMax;
        const int gx = x_grouped ? g : 0;
        const uint32_t bytes = a_tiles * kTcABytes + nbox * kTcBoxRows * 128;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { *abort_flag = 1; break; }
          unsigned char* st = smem + stage * shp.stage_bytes;
          mbar_arrive_expect_tx(&full_bar[stage], bytes);
          tma_load_3d(smem_u32(st), &tmap_w, &full_bar[stage], kb * kTcK, mt * kTcM, g);
          if (SWIGLU)
            tma_load_3d(smem_u32(st + kTcABytes), &tmap_w, &full_bar[stage], kb * kTcK,
                        mt * kTcM + up_rows, g);
          unsigned char* sb = st + a_tiles * kTcABytes;
          for (int bx = 0; bx < nbox; ++bx)
            tma_load_3d(smem_u32(sb + bx * kTcBoxRows * 128), &tmap_x, &full_bar[stage], kb * kTcK,
                        xrow0 + bx * kTcBoxRows, gx);
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
      for (long long it = blockIdx.x; it < total_items && !*abort_flag; it += gridDim.x) {
        int g, mt, nt, r0, ntok;
        if (!decode(it, g, mt, nt, r0, ntok)) continue;
        const int npad = round_up(ntok, 16);
        const uint32_t idesc = make_idesc_bf16(kTcM, npad);
        if (!mbar_wait(tempty_bar, (local & 1) ^ 1)) { *abort_flag = 1; break; }
        tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase)) { ok = false; break; }
          tc_fence_after();
          unsigned char* st = smem + stage * shp.stage_bytes;
          const uint64_t da = sw128_kmajor_desc(smem_u32(st));
          const uint64_t du = sw128_kmajor_desc(smem_u32(st + kTcABytes));
          const uint64_t db = sw128_kmajor_desc(smem_u32(st + a_tiles * kTcABytes));
#pragma unroll
          for (int k = 0; k < kTcK / 16; ++k) {
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
            // advance 16 bf16 (32 bytes) along K inside the swizzle row: +2 in addr>>4 units
            tc_mma_bf16(tmem_base, da + 2 * k, db + 2 * k, idesc, acc);
            if (SWIGLU) tc_mma_bf16(tmem_base + npad, du + 2 * k, db + 2 * k, idesc, acc);
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == shp.stages) { stage = 0; phase ^= 1; }
        }
        if (!ok) { *abort_flag = 1; break; }
        tc_commit(tfull_bar);
        ++local;
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    uint32_t local = 0;
    for (long long it = blockIdx.x; it < total_items; it += gridDim.x) {
      int g, mt, nt, r0, ntok;
      if (!decode(it, g, mt, nt, r0, ntok)) continue;
      const int npad = round_up(ntok, 16);
      const bool ok = mbar_wait(tfull_bar, local & 1);
      if (!ok || *abort_flag) { *abort_flag = 1; break; }
      tc_fence_after();
      const int n = mt * kTcM + row_in_tile;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
      for (int c0 = 0; c0 < npad; c0 += 16) {
        float acc[16], accu[16];
        tmem_ld16(tbase + c0, acc);
        if (SWIGLU) tmem_ld16(tbase + npad + c0, accu);
        tmem_ld_wait();
        if (n < p.n_rows) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int tok = c0 + j;
            if (tok < ntok) linear_store(p, g, r0 + nt * kTcNMax + tok, n, acc[j], SWIGLU ? accu[j] : 0.f);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(tempty_bar);
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

static int tmem_cols_for(int n) {
  int c = 32;
  while (c < n) c <<= 1;
  return c;
}

TcShape tc_shape(bool swiglu, int n_max) {
  TcShape s;
  const int npad = round_up(min(max(n_max, 1), kTcNMax), 16);
  s.b_bytes = npad * 128;
  s.stage_bytes = (swiglu ? 2 : 1) * kTcABytes + s.b_bytes;
  s.stages = min(8, (kTcSmemBudget - 2048) / s.stage_bytes);
  s.tmem_cols = tmem_cols_for(npad * (swiglu ? 2 : 1));
  return s;
}

size_t tc_smem_bytes(const TcShape& s) {
  return 1024 /*alignment slack*/ + static_cast<size_t>(s.stages) * s.stage_bytes +
         (2 * s.stages + 2) * sizeof(uint64_t) + 16;
}

cudaError_t linear_tc_init() {
  cudaError_t e = cudaFuncSetAttribute(linear_tc_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(linear_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              227 * 1024);
}

// tmap_w / tmap_x: CUtensorMap built by the caller (api.cu) for W and X
cudaError_t launch_linear_tc_impl(const LinearParams& p, const CUtensorMap& tmap_w,
                                  const CUtensorMap& tmap_x, int up_rows, int x_grouped,
                                  int num_sms, cudaStream_t st) {
  const bool swiglu = (p.epilogue == kEpiSwiglu);
  const int n_max = p.group_offsets ? p.max_routes_per_group : p.n_tokens;
  const TcShape shp = tc_shape(swiglu, n_max);
  const int mt_count = (p.n_rows + kTcM - 1) / kTcM;
  const int nt_count = max(1, (n_max + kTcNMax - 1) / kTcNMax);
  const long long items = static_cast<long long>(p.n_groups) * mt_count * nt_count;
  if (items <= 0) return cudaSuccess;
  const int grid = static_cast<int>(items < num_sms ? items : static_cast<long long>(num_sms));
  const size_t smem = tc_smem_bytes(shp);
  if (swiglu)
    linear_tc_kernel<true><<<grid, kTcThreads, smem, st>>>(p, tmap_w, tmap_x, shp, mt_count,
                                                           nt_count, up_rows, x_grouped);
  else
    linear_tc_kernel<false><<<grid, kTcThreads, smem, st>>>(p, tmap_w, tmap_x, shp, mt_count,
                                                            nt_count, up_rows, x_grouped);
  return cudaGetLastError();
}

}  // namespace dsv2
