// Kernel parameter blocks and launcher declarations shared between the kernel
// translation units and the C-ABI layer (api.cu).
#pragma once
#include "linear.cuh"

namespace dsv2 {

// Expert-parallel peer table: every rank's peer-visible buffer as mapped in this process
// (base[rank] is local), with the same layout in every buffer:
//   xg   [world * rows_per_rank, hidden] bf16   normalised MoE inputs of all rows
//   ids  [world * rows_per_rank, 6] int32, w [...] fp32   their top-6 routing
//   part [rows_per_rank, 8, hidden] fp32         slot outputs of this rank's rows
//   ctr  two uint64 counters (128 B apart): dispatch arrivals, combine arrivals
// world == 0: single GPU (no peers).
constexpr int kMaxPeers = 8;
struct PeerTable {
  int world;
  int rank;
  char* base[kMaxPeers];
  long long xg_off, ids_off, w_off, part_off, ctr_off;
  int rows_per_rank;
  int n_moe;                  // MoE layers per step
  const long long* epoch;     // completed steps of this rank
  unsigned int wait_polls;    // poll limit of the cross-GPU waits (0 = kPeerWaitPolls)
  unsigned long long* wait_stats;  // optional [4]: dispatch waits (ns, count), combine waits (ns, count)
};

__device__ __forceinline__ unsigned long long* peer_ctr(const PeerTable& t, int rank, int which) {
  return reinterpret_cast<unsigned long long*>(t.base[rank] + t.ctr_off + which * 128);
}
// value of a counter once every rank has signalled layer `layer` of the current step
__device__ __forceinline__ unsigned long long peer_target(const PeerTable& t, int layer,
                                                          unsigned long long per_rank) {
  const unsigned long long e = static_cast<unsigned long long>(*t.epoch);
  return (e * t.n_moe + layer + 1) * static_cast<unsigned long long>(t.world) * per_rank;
}

struct RouterParams {
  const bf16* x;           // [rows, hidden] normalised activations
  long long x_row_stride;
  const void* w;           // [n_experts, hidden] gate weight, bf16 or fp32
  int w_dtype;             // 0 bf16, 2 fp32
  const float* bias;       // optional per-expert logit offset (nullptr = none)
  int rows;
  int hidden;
  int n_experts;
  float scaling;
  float* logits;           // [rows, n_experts] workspace (fp32)
  long long* topk_ids;     // [rows, 6] int64 (may be nullptr)
  int* topk_ids32;         // [rows, 6] int32 (bucketing input)
  float* topk_w;           // [rows, 6]
  // bucketing (skipped when group_offsets == nullptr)
  int expert_lo;           // first local expert
  int n_local;             // local routed experts
  int shared_lo, shared_hi;  // rows whose shared-expert routes are local
  int* group_offsets;      // [n_local + 3]
  int* route_token;        // [rows*6 + 2*(shared_hi-shared_lo)]
  int* route_slot;
  float* route_weight;
  int gather_x;            // copy each route's x row into gather_out (expert order)
  void* gather_out;
  PeerTable peers;         // world > 0: write x / ids / weights of these rows to every rank
  int row_base;            // global index of this rank's first row
  // fused residual add + RMSNorm ahead of the gate (h != nullptr; router_fused_kernel):
  // h[r] = bf16(h[r] + sum_p delta[r, p]), x_out[r] = rmsnorm(h[r]) * norm_w
  bf16* h;
  const void* delta;
  int delta_dtype;         // 0 bf16, 2 fp32 partials
  int n_delta;
  long long delta_part_stride, delta_row_stride;
  const void* norm_w;
  int norm_w_dtype;
  float eps;
  bf16* x_out;             // normalised rows (row stride x_row_stride); x == x_out then
  int* grid_sync;          // [2] grid barrier of the single-launch bucketing (nullptr: two launches)
};

struct MlaPrepParams {
  const void* qkva;            // [B, 3072 + 576]: q (16 x 192) | c_kv (512) | k_pe (64)
  int qkva_f32;                // 1: fp32 split-K partials (qkva_parts of them), 0: bf16
  int qkva_parts;
  long long qkva_part_stride;  // elements
  bf16* q_nope_out;            // optional [B, 16, 128]
  long long qkva_row_stride;
  const bf16* kv_norm_w;       // [512]
  float eps;
  const float* cos_tab;        // [positions, rope_stride] (first 32 entries used)
  const float* sin_tab;
  long long rope_stride;
  int rope_rows;
  const long long* positions;  // [1] or [B]: write position of the new token
  int pos_numel;
  bf16* cache;                 // [B, max_len, 576] (this layer)
  long long cache_b_stride;    // elements
  int max_len;
  bf16* q_pe_out;              // [B, 16, 64]
  const int* cache_rows;       // optional [B]: cache row of input row b (else b)
  int cache_batch;             // rows of the cache
};

struct MlaDecodeParams {
  const bf16* q_abs;           // [B, 16, 512]
  const bf16* q_pe;            // [B, 16, 64]
  const bf16* cache;           // [B, max_len, 576]
  long long cache_b_stride;
  int max_len;
  const long long* positions;  // [1] or [B]; attended length = position + 1
  int pos_numel;
  float scale_log2;            // softmax_scale * log2(e)
  // mma.sync kernel: split_len = fewest positions per CTA, o_part / ml_part hold
  // batch * n_splits partial slots (two per CTA), row_sync = per-row merge tickets.
  // tcgen05 kernel: split_len = positions per split, o_part [B, n_splits, 16, 512].
  int split_len;
  int n_splits;
  float* o_part;
  float* ml_part;              // (m in log2 domain, l) per head and partial
  bf16* o_lat;                 // [B, 16, 512] output
  int inputs_prior;            // q_pe / positions / cache written >= 2 launches earlier
  int* row_sync;               // [B] zero-initialised, left zero
  int batch;
  const int* cache_rows;       // optional [B]: cache row read by query row b (else b)
  int cache_batch;             // rows of the cache
  int* part_count;             // optional (B = 1): partials left unmerged; [first CTA, count]
};

// norm.cu
cudaError_t launch_rmsnorm(const void*, long long, int, const void*, int, void*, long long, int, int,
                           float, cudaStream_t);
cudaError_t launch_add_rmsnorm(void*, void*, const void*, int, int, long long, long long,
                               const void*, int, void*, int, int, float, cudaStream_t,
                               const PeerTable* peers = nullptr, int layer = 0);
cudaError_t launch_embed_rmsnorm(const long long*, const void*, long long, const void*, int, void*,
                                 void*, int, int, float, cudaStream_t);
cudaError_t launch_residual_add(const void*, const void*, void*, long long, int, cudaStream_t);
cudaError_t launch_silu_mul(const void*, const void*, void*, long long, cudaStream_t);
cudaError_t launch_sum_partials(const float* part, int n_parts, long long ps, long long rs, void* out,
                               int out_f32, long long ors, int rows, int cols, cudaStream_t st);
cudaError_t launch_prepare_decode_inputs(const long long*, int, long long*, long long, long long*,
                                         long long, const long long*, int, int, cudaStream_t);
cudaError_t launch_copy_token_to_cache(const void*, const long long*, void*, const long long*,
                                       const long long*, int, int, int, int, int, int,
                                       cudaStream_t);
cudaError_t launch_advance_positions(long long*, int, cudaStream_t);
cudaError_t launch_argmax_finalize(const unsigned long long* keys, int n_blocks, long long key_stride,
                                   int n_tokens, long long* next_ids, long long* input_ids,
                                   long long* positions, int pos_numel, long long* step_counter,
                                   cudaStream_t st);
// router.cu
cudaError_t launch_router(const RouterParams&, int max_clusters, int num_sms, cudaStream_t);
cudaError_t router_fused_max_clusters(int* n);
cudaError_t launch_bucket(const int*, const float*, int, int, int, int, int, int*, int*, int*,
                          float*, const void*, long long, void*, int, int, cudaStream_t,
                          const PeerTable* peers, int layer);
cudaError_t launch_softmax_topk(const float*, int, int, float, long long*, int*, float*,
                                cudaStream_t);
cudaError_t launch_gather_rows(const void*, long long, const int*, const int*, int, void*, int,
                               int, cudaStream_t);
// mla.cu
cudaError_t launch_mla_prep(const MlaPrepParams&, int, cudaStream_t);
cudaError_t mla_decode_init();
int mla_decode_grid(const MlaDecodeParams&, int num_sms, long long part_slots);
cudaError_t launch_mla_decode(const MlaDecodeParams&, const CUtensorMap& tm_kv, const CUtensorMap& tm_qa,
                              const CUtensorMap& tm_qp, int grid, cudaStream_t);
cudaError_t launch_mla_combine(const MlaDecodeParams&, int, cudaStream_t);
// linear_tc.cu (TcShape, tc_launch_shape and launch_linear_tc_impl are defined there; the
// unity build includes it before api.cu)
cudaError_t linear_tc_init();

}  // namespace dsv2
