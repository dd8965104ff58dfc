// Parameters shared by the two linear kernels (CUDA-core/mma.sync "small" family and
// the tcgen05 "batch" family).  Mirrors dsv2_linear_args of the public header.
#pragma once
#include "common.cuh"

namespace dsv2 {

enum Epilogue : int {
  kEpiStoreBf16 = 0,   // y = bf16(acc)
  kEpiStoreF32 = 1,    // y = acc
  kEpiSwiglu = 2,      // y = bf16(silu(bf16(acc_gate)) * bf16(acc_up)) computed in fp32
  kEpiScaleF32 = 3,    // y = bf16(acc) * route_scale[route]   (fp32 store)
  kEpiArgmax = 4,      // y = per-row-block arg-max keys of bf16(acc) (uint64, see argmax_key)
};

// Arg-max key of output row n with value v (rounded to bf16 first, like bf16 logits):
// the value's bits in an order-preserving form above, and ~n below, so the largest key
// is the largest value and, among equal values, the lowest row.
__device__ __forceinline__ uint32_t argmax_ord(float v) {
  const uint32_t u = __float_as_uint(bf16_round(v));
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ unsigned long long argmax_key(uint32_t ord, uint32_t row) {
  return (static_cast<unsigned long long>(ord) << 32) | (0xffffffffu - row);
}

struct LinearParams {
  const bf16* w;
  long long w_row_stride;
  long long w_group_stride;
  long long up_offset;
  int n_rows;
  int k;
  const bf16* x;
  long long x_row_stride;
  long long x_group_stride;
  void* y;
  long long y_row_stride;
  long long y_group_stride;
  int epilogue;
  int n_groups;
  int n_tokens;
  const int* group_offsets;
  const int* route_x_row;
  const int* route_y_row;
  const float* route_scale;
  int max_routes_per_group;
  int k_splits;                 // batch family, dense fp32 output: K split across CTAs
  long long y_split_stride;     // elements between the fp32 partial outputs of the splits
  int offsets_prior;            // group_offsets were written at least two launches earlier
  int active_groups;            // grouped small family: launch work for this many non-empty groups
  // small family, one token, dense: the token's activation row of group g is the merge of a
  // one-row latent attention's unmerged partials instead of x: partial c holds o at
  // x_parts + (2c * n_groups + g) * k and (m, l) at x_parts_ml + (2c * n_groups + g) * 2,
  // for c in [x_parts_count[0], x_parts_count[0] + x_parts_count[1])
  const float* x_parts;
  const float* x_parts_ml;
  const int* x_parts_count;
};

__device__ __forceinline__ float silu_ref(float g) { return g / (1.f + expf(-g)); }

// Epilogue for one output element (row n, route r, accumulators acc/acc_up).
__device__ __forceinline__ void linear_store(const LinearParams& p, int g, int r, int n, float acc,
                                             float acc_up, long long split_off = 0) {
  const int yrow = p.route_y_row ? p.route_y_row[r] : r;
  const long long off =
      split_off + g * p.y_group_stride + static_cast<long long>(yrow) * p.y_row_stride + n;
  switch (p.epilogue) {
    case kEpiStoreBf16:
      reinterpret_cast<bf16*>(p.y)[off] = __float2bfloat16_rn(acc);
      break;
    case kEpiStoreF32:
      reinterpret_cast<float*>(p.y)[off] = acc;
      break;
    case kEpiSwiglu: {
      const float gt = bf16_round(acc), up = bf16_round(acc_up);
      reinterpret_cast<bf16*>(p.y)[off] = __float2bfloat16_rn(silu_ref(gt) * up);
      break;
    }
    default: {
      reinterpret_cast<float*>(p.y)[off] = bf16_round(acc) * p.route_scale[r];
      break;
    }
  }
}

cudaError_t launch_linear_gemv(const LinearParams& p, cudaStream_t st);

}  // namespace dsv2
