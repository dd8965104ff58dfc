// extern "C" entry points of libdsv2.so (declared in include/dsv2.h).
//
// Argument validation, per-device one-time setup, TMA tensor-map construction (cached
// by shape and address), and dispatch to the kernel launchers.  No entry point
// allocates device memory or synchronises the stream.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "../../include/dsv2.h"
#include "params.cuh"


using namespace dsv2;

namespace {

thread_local std::string g_last_error;
std::mutex g_mu;
bool g_dev_init[128];
int g_dev_sms[128];
float* g_noalloc_scratch[128];  // device address of the allocation-free entry point's array
int g_router_clusters[128];     // router_fused_kernel clusters resident at once

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(DSV2_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return DSV2_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int ensure_init(int* sms_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(DSV2_ERR_LAUNCH, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 128) return fail(DSV2_ERR_INVALID, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  static bool env_read = false;
  if (!env_read) {  // DSV2_PDL=0 turns programmatic dependent launch off
    const char* v = getenv("DSV2_PDL");
    if (v && v[0] == '0') g_pdl_enabled = false;
    env_read = true;
  }
  if (!g_dev_init[dev]) {
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (major != 10)
      return fail(DSV2_ERR_UNSUPPORTED, "libdsv2 is built for sm_100a; device %d is sm_%d%d", dev,
                  major, minor);
    if ((e = mla_decode_init()) != cudaSuccess)
      return fail(DSV2_ERR_LAUNCH, "mla_decode_init: %s", cudaGetErrorString(e));
    if ((e = linear_tc_init()) != cudaSuccess)
      return fail(DSV2_ERR_LAUNCH, "linear_tc_init: %s", cudaGetErrorString(e));
    if ((e = moe_tc_init()) != cudaSuccess)
      return fail(DSV2_ERR_LAUNCH, "moe_tc_init: %s", cudaGetErrorString(e));
    if ((e = mla_tc_init()) != cudaSuccess)
      return fail(DSV2_ERR_LAUNCH, "mla_tc_init: %s", cudaGetErrorString(e));
    if ((e = mla_noalloc_lookup(&g_noalloc_scratch[dev])) != cudaSuccess)
      return fail(DSV2_ERR_LAUNCH, "scratch address of the allocation-free entry point: %s", cudaGetErrorString(e));
    if ((e = router_fused_max_clusters(&g_router_clusters[dev])) != cudaSuccess)
      return fail(DSV2_ERR_LAUNCH, "router occupancy: %s", cudaGetErrorString(e));
    if ((e = linear_splitk_init()) != cudaSuccess)
      return fail(DSV2_ERR_LAUNCH, "linear_splitk_init: %s", cudaGetErrorString(e));
    g_dev_sms[dev] = sms;
    g_dev_init[dev] = true;
  }
  if (sms_out) *sms_out = g_dev_sms[dev];
  return DSV2_OK;
}

// router_fused_kernel clusters resident at once on the current device (after ensure_init)
int router_clusters() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 0;
  std::lock_guard<std::mutex> lk(g_mu);
  return g_router_clusters[dev];
}

// ---- TMA tensor maps ---------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encode() {
  if (g_encode) return DSV2_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return fail(DSV2_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return DSV2_OK;
}

typedef std::tuple<int, uintptr_t, uint64_t, uint64_t, uint64_t, uint64_t, uint64_t, uint32_t,
                   uint32_t>
    MapKey;
std::map<MapKey, CUtensorMap> g_maps;

// 3-D bf16 tensor map {inner, rows, groups} with a {64, box_rows, 1} box, 128-byte swizzle.
int tensor_map_3d(const void* base, uint64_t inner, uint64_t rows, uint64_t groups,
                  uint64_t row_stride_b, uint64_t group_stride_b, uint32_t box_rows,
                  CUtensorMap* out) {
  int dev = 0;
  cudaGetDevice(&dev);
  const MapKey key(dev, reinterpret_cast<uintptr_t>(base), inner, rows, groups, row_stride_b,
                   group_stride_b, box_rows, 0);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return DSV2_OK;
    }
  }
  int rc = get_encode();
  if (rc) return rc;
  if (!aligned16(base) || (row_stride_b & 15) || (group_stride_b & 15))
    return fail(DSV2_ERR_INVALID, "TMA operand not 16-byte aligned (base %p, strides %llu/%llu)",
                base, (unsigned long long)row_stride_b, (unsigned long long)group_stride_b);
  cuuint64_t dims[3] = {inner, rows, groups};
  cuuint64_t strides[2] = {row_stride_b, group_stride_b};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap m;
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DSV2_ERR_INVALID,
                "cuTensorMapEncodeTiled failed (%d): dims %llu x %llu x %llu strides %llu %llu",
                static_cast<int>(r), (unsigned long long)inner, (unsigned long long)rows,
                (unsigned long long)groups, (unsigned long long)row_stride_b,
                (unsigned long long)group_stride_b);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps[key] = m;
  *out = m;
  return DSV2_OK;
}

// 3-D fp32 tensor map {inner, rows, groups} with a {128, box_rows, 1} box, no swizzle: the
// partial-tile stores of the split-K linear.
int tensor_map_f32_store(void* base, uint64_t inner, uint64_t rows, uint64_t groups, uint64_t row_stride_b,
                         uint64_t group_stride_b, uint32_t box_rows, CUtensorMap* out) {
  int dev = 0;
  cudaGetDevice(&dev);
  const MapKey key(dev, reinterpret_cast<uintptr_t>(base), inner, rows, groups, row_stride_b, group_stride_b,
                   box_rows, 1);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return DSV2_OK;
    }
  }
  int rc = get_encode();
  if (rc) return rc;
  if (!aligned16(base) || (row_stride_b & 15) || (group_stride_b & 15))
    return fail(DSV2_ERR_INVALID, "TMA output not 16-byte aligned (base %p, strides %llu/%llu)", base,
                (unsigned long long)row_stride_b, (unsigned long long)group_stride_b);
  cuuint64_t dims[3] = {inner, rows, groups};
  cuuint64_t strides[2] = {row_stride_b, group_stride_b};
  cuuint32_t box[3] = {128, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap m;
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DSV2_ERR_INVALID, "cuTensorMapEncodeTiled (fp32 store) failed (%d)", static_cast<int>(r));
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps[key] = m;
  *out = m;
  return DSV2_OK;
}

// Latent cache [batch][max_len][576] bf16 as a TMA map: boxes of 64 dims x box_rows positions.
int mla_cache_map(const void* cache, int64_t cache_b_stride, int max_len, int batch, uint32_t box_rows,
                  CUtensorMap* out) {
  return tensor_map_3d(cache, 576, static_cast<uint64_t>(max_len), static_cast<uint64_t>(batch), 576 * 2,
                       static_cast<uint64_t>(cache_b_stride) * 2, box_rows, out);
}

// Balanced mma.sync latent attention: cache / query tensor maps, grid, launch.
int mla_decode_balanced(const MlaDecodeParams& p, int sms, long long part_slots, cudaStream_t st,
                        const char* what) {
  CUtensorMap tm_kv, tm_qa, tm_qp;
  int rc = mla_cache_map(p.cache, p.cache_b_stride, p.max_len, p.cache_batch, 32, &tm_kv);
  if (rc) return rc;
  // q_abs [B][16][512] and q_pe [B][16][64] as {dims, heads, rows} maps with 64 x 16 boxes
  if ((rc = tensor_map_3d(p.q_abs, 512, 16, static_cast<uint64_t>(p.batch), 1024, 16384, 16, &tm_qa))) return rc;
  if ((rc = tensor_map_3d(p.q_pe, 64, 16, static_cast<uint64_t>(p.batch), 128, 2048, 16, &tm_qp))) return rc;
  const int grid = mla_decode_grid(p, sms, part_slots);
  if (grid <= 0) return fail(DSV2_ERR_INVALID, "%s: no partial slots", what);
  return check_launch(launch_mla_decode(p, tm_kv, tm_qa, tm_qp, grid, st), what);
}

// dsv2_peer_table -> kernel-side PeerTable (world 0 when NULL or single GPU)
int to_peers(const dsv2_peer_table* t, PeerTable* out) {
  *out = PeerTable{};
  if (!t || t->world <= 1) return DSV2_OK;
  if (t->world > kMaxPeers || t->rank < 0 || t->rank >= t->world || !t->epoch || t->rows_per_rank <= 0 ||
      t->n_moe_layers <= 0)
    return fail(DSV2_ERR_INVALID, "peer table: world %d rank %d", t->world, t->rank);
  for (int q = 0; q < t->world; ++q) {
    if (!t->base[q]) return fail(DSV2_ERR_INVALID, "peer table: buffer of rank %d missing", q);
    out->base[q] = static_cast<char*>(t->base[q]);
  }
  out->world = t->world;
  out->rank = t->rank;
  out->xg_off = t->xg_offset;
  out->ids_off = t->ids_offset;
  out->w_off = t->w_offset;
  out->part_off = t->part_offset;
  out->ctr_off = t->ctr_offset;
  out->rows_per_rank = t->rows_per_rank;
  out->n_moe = t->n_moe_layers;
  out->epoch = reinterpret_cast<const long long*>(t->epoch);
  if (t->wait_polls < 0) return fail(DSV2_ERR_INVALID, "peer table: wait_polls %d", t->wait_polls);
  out->wait_polls = static_cast<unsigned int>(t->wait_polls);
  out->wait_stats = reinterpret_cast<unsigned long long*>(t->wait_stats);
  return DSV2_OK;
}

}  // namespace

extern "C" {

int dsv2_peer_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(DSV2_ERR_INVALID, "peer_alloc: bad arguments");
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return check_launch(e, "peer_alloc");
  e = cudaMemset(*ptr, 0, bytes);
  return check_launch(e, "peer_alloc: clear");
}

int dsv2_peer_free(void* ptr) { return check_launch(cudaFree(ptr), "peer_free"); }

int dsv2_peer_export(const void* ptr, void* handle) {
  if (!ptr || !handle) return fail(DSV2_ERR_INVALID, "peer_export: null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return check_launch(e, "peer_export");
  memcpy(handle, &h, sizeof(h));
  return DSV2_OK;
}

int dsv2_peer_import(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(DSV2_ERR_INVALID, "peer_import: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return check_launch(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "peer_import");
}

int dsv2_peer_close(void* ptr) { return check_launch(cudaIpcCloseMemHandle(ptr), "peer_close"); }

int dsv2_version(void) { return 100; }

const char* dsv2_last_error(void) { return g_last_error.c_str(); }

int dsv2_init(void) { return ensure_init(nullptr); }

int dsv2_set_programmatic_launch(int enable) {
  const int prev = g_pdl_enabled ? 1 : 0;
  g_pdl_enabled = enable != 0;
  return prev;
}

int64_t dsv2_kernel_launches(void) { return g_kernel_launches.load(std::memory_order_relaxed); }

int dsv2_get_device_error(int* code, int clear) {
  if (!code) return fail(DSV2_ERR_INVALID, "code is NULL");
  cudaError_t e = cudaMemcpyFromSymbol(code, g_device_error, sizeof(int));
  if (e != cudaSuccess) return check_launch(e, "read device error");
  if (clear && *code != 0) {
    // a launch that gave up may have left row tickets of the allocation-free attention
    // entry point's array nonzero: wait for the device, then zero them with the word
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) return check_launch(e, "clear device error: sync");
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return check_launch(e, "clear device error: device");
    float* scratch = nullptr;
    if (dev >= 0 && dev < 128) {
      std::lock_guard<std::mutex> lk(g_mu);
      scratch = g_noalloc_scratch[dev];
    }
    if (scratch && (e = cudaMemset(scratch + kNoAllocTicketOffset, 0, kNoAllocMaxRows * sizeof(int))) != cudaSuccess)
      return check_launch(e, "clear device error: row tickets");
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return check_launch(e, "clear device error");
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) return check_launch(e, "clear device error: sync");
  }
  return DSV2_OK;
}

int dsv2_stream_check(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return check_launch(e, "stream_check: synchronize");
  int code = 0;
  if ((e = cudaMemcpyFromSymbol(&code, g_device_error, sizeof(int))) != cudaSuccess)
    return check_launch(e, "stream_check: read device error");
  if (code == 0) return DSV2_OK;
  static const char* what[] = {"none", "a bounded wait gave up", "an index was out of range",
                               "tensor memory allocation failed"};
  return fail(DSV2_ERR_DEVICE, "device error word %d (%s); read and clear it with dsv2_get_device_error",
              code, code >= 0 && code <= 3 ? what[code] : "unknown");
}

int dsv2_reset_progress(void* counters, int64_t count, void* stream) {
  if (count < 0 || (count > 0 && !counters)) return fail(DSV2_ERR_INVALID, "reset_progress: bad arguments");
  if (count == 0) return DSV2_OK;
  return check_launch(cudaMemsetAsync(counters, 0, static_cast<size_t>(count) * sizeof(int32_t),
                                      static_cast<cudaStream_t>(stream)),
                      "reset_progress");
}

int dsv2_rmsnorm(const void* x, int64_t x_row_stride, int x_dtype, const void* w, int w_dtype, void* y,
                 int64_t y_row_stride, int rows, int cols, float eps, void* stream) {
  if (!x || !w || !y) return fail(DSV2_ERR_INVALID, "rmsnorm: null pointer");
  if (cols <= 0 || cols % 8 || cols > 4096)
    return fail(DSV2_ERR_UNSUPPORTED, "rmsnorm: cols=%d (need multiple of 8, <= 4096)", cols);
  if (x_dtype != DSV2_BF16 && x_dtype != DSV2_F16)
    return fail(DSV2_ERR_UNSUPPORTED, "rmsnorm: activation dtype %d", x_dtype);
  if (w_dtype != DSV2_BF16 && w_dtype != DSV2_F16 && w_dtype != DSV2_F32)
    return fail(DSV2_ERR_UNSUPPORTED, "rmsnorm: weight dtype %d", w_dtype);
  if (!aligned16(x) || !aligned16(y) || (x_row_stride % 8) || (y_row_stride % 8))
    return fail(DSV2_ERR_INVALID, "rmsnorm: rows must be 16-byte aligned");
  if (rows <= 0) return DSV2_OK;
  return check_launch(launch_rmsnorm(x, x_row_stride, x_dtype, w, w_dtype, y, y_row_stride, rows, cols, eps,
                                     static_cast<cudaStream_t>(stream)),
                      "rmsnorm");
}

int dsv2_add_rmsnorm(void* h, void* h_out, const void* delta, int delta_dtype, int n_delta,
                     int64_t delta_part_stride, int64_t delta_row_stride, const void* w,
                     int w_dtype, void* y, int rows, int cols, float eps,
                     const dsv2_peer_table* peers, int moe_layer, void* stream) {
  PeerTable pt;
  if (int rc = to_peers(peers, &pt)) return rc;
  if (!h || (n_delta > 0 && !delta) || (y && !w))
    return fail(DSV2_ERR_INVALID, "add_rmsnorm: null pointer");
  if (cols <= 0 || cols % 8 || cols > 4096)
    return fail(DSV2_ERR_UNSUPPORTED, "add_rmsnorm: cols=%d", cols);
  if (delta_dtype != DSV2_BF16 && delta_dtype != DSV2_F32)
    return fail(DSV2_ERR_UNSUPPORTED, "add_rmsnorm: delta dtype %d", delta_dtype);
  if (!aligned16(h) || (h_out && !aligned16(h_out)) || (y && !aligned16(y)) ||
      (n_delta > 0 && (!aligned16(delta) || delta_part_stride % 8 || delta_row_stride % 8)))
    return fail(DSV2_ERR_INVALID, "add_rmsnorm: operands must be 16-byte aligned");
  if (rows <= 0) return DSV2_OK;
  return check_launch(launch_add_rmsnorm(h, h_out, delta, delta_dtype, n_delta, delta_part_stride,
                                         delta_row_stride, w, w_dtype, y, rows, cols, eps,
                                         static_cast<cudaStream_t>(stream), &pt, moe_layer),
                      "add_rmsnorm");
}

int dsv2_embed_rmsnorm(const int64_t* ids, const void* table, int64_t vocab, const void* w,
                       int w_dtype, void* h, void* y, int rows, int cols, float eps,
                       void* stream) {
  if (!ids || !table || !w || !h || !y) return fail(DSV2_ERR_INVALID, "embed_rmsnorm: null pointer");
  if (cols <= 0 || cols % 8 || cols > 4096)
    return fail(DSV2_ERR_UNSUPPORTED, "embed_rmsnorm: cols=%d", cols);
  if (!aligned16(table) || !aligned16(h) || !aligned16(y))
    return fail(DSV2_ERR_INVALID, "embed_rmsnorm: operands must be 16-byte aligned");
  if (rows <= 0) return DSV2_OK;
  return check_launch(
      launch_embed_rmsnorm(reinterpret_cast<const long long*>(ids), table, vocab, w, w_dtype, h, y,
                           rows, cols, eps, static_cast<cudaStream_t>(stream)),
      "embed_rmsnorm");
}

int dsv2_residual_add(const void* a, const void* b, void* out, int64_t n, int dtype, void* stream) {
  if (!a || !b || !out) return fail(DSV2_ERR_INVALID, "residual_add: null pointer");
  if (dtype != DSV2_BF16 && dtype != DSV2_F16)
    return fail(DSV2_ERR_UNSUPPORTED, "residual_add: dtype %d", dtype);
  if (n % 8) return fail(DSV2_ERR_UNSUPPORTED, "residual_add: n=%lld not a multiple of 8", (long long)n);
  if (!aligned16(a) || !aligned16(b) || !aligned16(out))
    return fail(DSV2_ERR_INVALID, "residual_add: operands must be 16-byte aligned");
  if (n <= 0) return DSV2_OK;
  return check_launch(launch_residual_add(a, b, out, n, dtype, static_cast<cudaStream_t>(stream)),
                      "residual_add");
}

int dsv2_silu_mul(const void* gate, const void* up, void* out, int64_t n, void* stream) {
  if (!gate || !up || !out) return fail(DSV2_ERR_INVALID, "silu_mul: null pointer");
  if (n % 8) return fail(DSV2_ERR_UNSUPPORTED, "silu_mul: n=%lld not a multiple of 8", (long long)n);
  if (!aligned16(gate) || !aligned16(up) || !aligned16(out))
    return fail(DSV2_ERR_INVALID, "silu_mul: operands must be 16-byte aligned");
  if (n <= 0) return DSV2_OK;
  return check_launch(launch_silu_mul(gate, up, out, n, static_cast<cudaStream_t>(stream)),
                      "silu_mul");
}

int dsv2_sum_partials(const float* part, int n_parts, int64_t part_stride, int64_t row_stride, void* out,
                      int out_dtype, int64_t out_row_stride, int rows, int cols, void* stream) {
  if (!part || !out) return fail(DSV2_ERR_INVALID, "sum_partials: null pointer");
  if (out_dtype != DSV2_BF16 && out_dtype != DSV2_F32)
    return fail(DSV2_ERR_UNSUPPORTED, "sum_partials: output dtype %d", out_dtype);
  if (cols < 0 || cols % 8 || n_parts < 0 || rows < 0 || rows > 65535)
    return fail(DSV2_ERR_UNSUPPORTED, "sum_partials: rows=%d cols=%d parts=%d", rows, cols, n_parts);
  if (!aligned16(part) || !aligned16(out) || part_stride % 4 || row_stride % 4 ||
      out_row_stride % (out_dtype == DSV2_F32 ? 4 : 8))
    return fail(DSV2_ERR_INVALID, "sum_partials: operands and strides must be 16-byte aligned");
  if (rows == 0 || cols == 0) return DSV2_OK;
  return check_launch(launch_sum_partials(part, n_parts, part_stride, row_stride, out,
                                          out_dtype == DSV2_F32, out_row_stride, rows, cols,
                                          static_cast<cudaStream_t>(stream)),
                      "sum_partials");
}

int dsv2_prepare_decode_inputs(const int64_t* cache_position, int pos_numel,
                               int64_t* attention_mask, int64_t mask_stride_b,
                               int64_t* position_ids, int64_t position_ids_stride_b,
                               const int64_t* attention_mask_index, int batch, int max_len,
                               void* stream) {
  if (!cache_position || (attention_mask && !attention_mask_index))
    return fail(DSV2_ERR_INVALID, "prepare_decode_inputs: null pointer");
  if (pos_numel != 1 && pos_numel != batch)
    return fail(DSV2_ERR_INVALID, "prepare_decode_inputs: cache_position has %d elements for batch %d",
                pos_numel, batch);
  if (batch <= 0 || max_len <= 0) return DSV2_OK;
  return check_launch(
      launch_prepare_decode_inputs(reinterpret_cast<const long long*>(cache_position), pos_numel,
                                   reinterpret_cast<long long*>(attention_mask), mask_stride_b,
                                   reinterpret_cast<long long*>(position_ids), position_ids_stride_b,
                                   reinterpret_cast<const long long*>(attention_mask_index), batch,
                                   max_len, static_cast<cudaStream_t>(stream)),
      "prepare_decode_inputs");
}

int dsv2_copy_token_to_cache(const void* src, const int64_t* src_strides, void* dst,
                             const int64_t* dst_strides, const int64_t* cache_position,
                             int pos_numel, int batch, int heads, int dim, int elem_size,
                             int max_len, void* stream) {
  if (!src || !dst || !src_strides || !dst_strides || !cache_position)
    return fail(DSV2_ERR_INVALID, "copy_token_to_cache: null pointer");
  if (elem_size != 2 && elem_size != 4)
    return fail(DSV2_ERR_UNSUPPORTED, "copy_token_to_cache: element size %d", elem_size);
  if (pos_numel != 1 && pos_numel != batch)
    return fail(DSV2_ERR_INVALID, "copy_token_to_cache: cache_position numel %d", pos_numel);
  if (batch <= 0 || heads <= 0 || dim <= 0) return DSV2_OK;
  long long ss[3] = {src_strides[0], src_strides[1], src_strides[2]};
  long long ds[4] = {dst_strides[0], dst_strides[1], dst_strides[2], dst_strides[3]};
  return check_launch(launch_copy_token_to_cache(src, ss, dst, ds,
                                                 reinterpret_cast<const long long*>(cache_position),
                                                 pos_numel, batch, heads, dim, elem_size, max_len,
                                                 static_cast<cudaStream_t>(stream)),
                      "copy_token_to_cache");
}

int dsv2_advance_positions(int64_t* pos, int n, void* stream) {
  if (!pos) return fail(DSV2_ERR_INVALID, "advance_positions: null pointer");
  if (n <= 0) return DSV2_OK;
  return check_launch(launch_advance_positions(reinterpret_cast<long long*>(pos), n,
                                               static_cast<cudaStream_t>(stream)),
                      "advance_positions");
}

static int linear_impl(const dsv2_linear_args* a, int family, void* stream, bool argmax);

int dsv2_linear(const dsv2_linear_args* a, int family, void* stream) {
  return linear_impl(a, family, stream, false);
}

int dsv2_lm_head_argmax(const void* w, int vocab, int hidden, const void* x, int64_t x_row_stride,
                        int n_tokens, uint64_t* keys, int64_t keys_capacity, int64_t* next_ids,
                        int64_t* input_ids, int64_t* positions, int pos_numel, int64_t* step_counter,
                        int family, void* stream) {
  if (!w || !x || !keys || !next_ids) return fail(DSV2_ERR_INVALID, "lm_head_argmax: null pointer");
  if (vocab <= 0 || hidden <= 0 || n_tokens < 0)
    return fail(DSV2_ERR_INVALID, "lm_head_argmax: vocab %d hidden %d tokens %d", vocab, hidden, n_tokens);
  if (positions && pos_numel != 1 && pos_numel != n_tokens)
    return fail(DSV2_ERR_INVALID, "lm_head_argmax: positions numel %d for %d tokens", pos_numel, n_tokens);
  if (n_tokens == 0) return DSV2_OK;
  const long long n_blocks = family == DSV2_FAMILY_BATCH ? (static_cast<long long>(vocab) + 127) / 128 * 4
                                                         : (static_cast<long long>(vocab) + 15) / 16;
  if (keys_capacity < n_blocks * n_tokens)
    return fail(DSV2_ERR_INVALID, "lm_head_argmax: keys hold %lld entries, %lld needed",
                static_cast<long long>(keys_capacity), n_blocks * n_tokens);
  dsv2_linear_args a = {};
  a.w = w;
  a.w_row_stride = hidden;
  a.n_rows = vocab;
  a.k = hidden;
  a.x = x;
  a.x_row_stride = x_row_stride;
  a.y = keys;
  a.y_row_stride = n_tokens;
  a.epilogue = DSV2_EPI_ARGMAX;
  a.n_groups = 1;
  a.n_tokens = n_tokens;
  a.w_group_rows = vocab;
  a.x_group_rows = n_tokens;
  int rc = linear_impl(&a, family, stream, true);
  if (rc) return rc;
  return check_launch(launch_argmax_finalize(reinterpret_cast<const unsigned long long*>(keys),
                                             static_cast<int>(n_blocks), n_tokens, n_tokens,
                                             reinterpret_cast<long long*>(next_ids),
                                             reinterpret_cast<long long*>(input_ids),
                                             reinterpret_cast<long long*>(positions), pos_numel,
                                             reinterpret_cast<long long*>(step_counter),
                                             static_cast<cudaStream_t>(stream)),
                      "lm_head_argmax: finalize");
}

static int linear_impl(const dsv2_linear_args* a, int family, void* stream, bool argmax) {
  if (!a || !a->w || (!a->x && !a->x_parts) || !a->y) return fail(DSV2_ERR_INVALID, "linear: null pointer");
  if (a->x_parts && (family != DSV2_FAMILY_SMALL || a->n_tokens != 1 || a->group_offsets || argmax ||
                     !a->x_parts_ml || !a->x_parts_count))
    return fail(DSV2_ERR_UNSUPPORTED,
                "linear: x_parts needs the small family, one token, dense mode, x_parts_ml and x_parts_count");
  if (a->n_rows <= 0 || a->k <= 0 || a->n_groups <= 0)
    return fail(DSV2_ERR_INVALID, "linear: n_rows=%d k=%d n_groups=%d", a->n_rows, a->k, a->n_groups);
  if (a->epilogue < DSV2_EPI_STORE_BF16 || a->epilogue > (argmax ? DSV2_EPI_ARGMAX : DSV2_EPI_SCALE_F32))
    return fail(DSV2_ERR_INVALID, "linear: epilogue %d", a->epilogue);
  if (a->epilogue == DSV2_EPI_SCALE_F32 && !a->route_scale)
    return fail(DSV2_ERR_INVALID, "linear: SCALE epilogue needs route_scale");
  if (a->epilogue == DSV2_EPI_SCALE_F32 && !a->group_offsets)
    return fail(DSV2_ERR_INVALID, "linear: SCALE epilogue needs grouped mode");
  if (!aligned16(a->w) || !aligned16(a->x) || a->w_row_stride % 8 || a->x_row_stride % 8 ||
      a->w_group_stride % 8 || a->x_group_stride % 8 || a->up_offset % 8)
    return fail(DSV2_ERR_INVALID, "linear: W/X rows must be 16-byte aligned");
  const int n_tok = a->group_offsets ? a->max_routes_per_group : a->n_tokens;
  if (n_tok <= 0) return DSV2_OK;
  LinearParams p = {};
  p.w = reinterpret_cast<const bf16*>(a->w);
  p.w_row_stride = a->w_row_stride;
  p.w_group_stride = a->w_group_stride;
  p.up_offset = a->up_offset;
  p.n_rows = a->n_rows;
  p.k = a->k;
  p.x = reinterpret_cast<const bf16*>(a->x);
  p.x_row_stride = a->x_row_stride;
  p.x_group_stride = a->x_group_stride;
  p.y = a->y;
  p.y_row_stride = a->y_row_stride;
  p.y_group_stride = a->y_group_stride;
  p.epilogue = a->epilogue;
  p.n_groups = a->n_groups;
  p.n_tokens = a->n_tokens;
  p.group_offsets = a->group_offsets;
  p.route_x_row = a->route_x_row;
  p.route_y_row = a->route_y_row;
  p.route_scale = a->route_scale;
  p.max_routes_per_group = a->max_routes_per_group;
  p.k_splits = a->k_splits > 1 ? a->k_splits : 1;
  p.y_split_stride = a->y_split_stride;
  p.offsets_prior = a->offsets_prior != 0;
  p.active_groups = (a->group_offsets && a->max_routes > 0) ? std::min(a->n_groups, a->max_routes) : a->n_groups;
  p.x_parts = a->x_parts;
  p.x_parts_ml = a->x_parts_ml;
  p.x_parts_count = a->x_parts_count;
  if (p.k_splits > 1) {
    if (family != DSV2_FAMILY_BATCH || a->group_offsets || a->epilogue != DSV2_EPI_STORE_F32)
      return fail(DSV2_ERR_UNSUPPORTED, "linear: a K split needs the batch family, dense mode and fp32 output");
    if (p.k_splits > a->k / 64)
      return fail(DSV2_ERR_INVALID, "linear: k_splits %d exceeds k/64 = %d", p.k_splits, a->k / 64);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (family == DSV2_FAMILY_SMALL) {
    if (a->k % 32) return fail(DSV2_ERR_UNSUPPORTED, "linear(small): k=%d not a multiple of 32", a->k);
    return check_launch(launch_linear_gemv(p, st), "linear(small)");
  }
  if (family != DSV2_FAMILY_BATCH) return fail(DSV2_ERR_INVALID, "linear: family %d", family);
  if (a->k % 64) return fail(DSV2_ERR_UNSUPPORTED, "linear(batch): k=%d not a multiple of 64", a->k);
  if (a->route_x_row)
    return fail(DSV2_ERR_UNSUPPORTED, "linear(batch): gathered X rows are not supported (gather first)");
  if (a->w_group_rows <= 0 || a->x_group_rows <= 0)
    return fail(DSV2_ERR_INVALID, "linear(batch): w_group_rows / x_group_rows required");
  if (a->n_groups > 1 && a->w_group_stride == 0)
    return fail(DSV2_ERR_INVALID, "linear(batch): groups need a weight group stride");
  int up_rows = 0;
  if (a->epilogue == DSV2_EPI_SWIGLU) {
    if (a->up_offset % a->w_row_stride)
      return fail(DSV2_ERR_INVALID, "linear(batch): up_offset must be whole rows");
    up_rows = static_cast<int>(a->up_offset / a->w_row_stride);
  }
  int sms = 0;
  int rc = ensure_init(&sms);
  if (rc) return rc;
  CUtensorMap mw, mx;
  const uint64_t wrs = static_cast<uint64_t>(a->w_row_stride) * 2;
  const uint64_t wgs = a->n_groups > 1 ? static_cast<uint64_t>(a->w_group_stride) * 2
                                       : wrs * static_cast<uint64_t>(a->w_group_rows);
  rc = tensor_map_3d(a->w, a->k, a->w_group_rows, a->n_groups, wrs, wgs, 128, &mw);
  if (rc) return rc;
  const bool xg = a->x_group_stride != 0 && a->n_groups > 1;
  const uint64_t xrs = static_cast<uint64_t>(a->x_row_stride) * 2;
  const uint64_t xgs = xg ? static_cast<uint64_t>(a->x_group_stride) * 2
                          : xrs * static_cast<uint64_t>(a->x_group_rows);
  rc = tensor_map_3d(a->x, a->k, a->x_group_rows, xg ? a->n_groups : 1, xrs, xgs, 16, &mx);
  if (rc) return rc;
  if (p.k_splits > 1 && a->n_groups == 1 && a->n_tokens <= 256 && !a->route_y_row) {
    // decode-sized dense split: one (row tile, split) per CTA, weights requested before the
    // programmatic-launch wait
    CUtensorMap mxs, mys;
    rc = tensor_map_3d(a->x, a->k, a->x_group_rows, 1, xrs, xgs, static_cast<uint32_t>(round_up(a->n_tokens, 16)),
                       &mxs);
    if (rc) return rc;
    // partial tiles leave through TMA stores of 128 rows x 32 tokens
    rc = tensor_map_f32_store(a->y, static_cast<uint64_t>(a->n_rows), static_cast<uint64_t>(a->n_tokens),
                              static_cast<uint64_t>(p.k_splits), static_cast<uint64_t>(a->y_row_stride) * 4,
                              static_cast<uint64_t>(a->y_split_stride) * 4, kSkStoreTokens, &mys);
    if (rc) return rc;
    return check_launch(launch_linear_splitk(p, mw, mxs, mys, st), "linear(batch, split K)");
  }
  TcShape shp;
  int mt_count = 0, nt_count = 0;
  const long long items = tc_launch_shape(p, sms, &shp, &mt_count, &nt_count);
  CUtensorMap mxb;
  rc = tensor_map_3d(a->x, a->k, a->x_group_rows, xg ? a->n_groups : 1, xrs, xgs,
                     static_cast<uint32_t>(shp.x_box), &mxb);
  if (rc) return rc;
  return check_launch(launch_linear_tc_impl(p, mw, mx, mxb, shp, mt_count, nt_count, items, up_rows,
                                            xg ? 1 : 0, sms, st),
                      "linear(batch)");
}

int dsv2_moe(const dsv2_moe_args* a, void* stream) {
  if (!a || !a->gate_up || !a->down || !a->x_sorted || !a->h || !a->group_offsets || !a->route_slot ||
      !a->route_weight || !a->y || !a->sync)
    return fail(DSV2_ERR_INVALID, "moe: null pointer");
  if (a->n_groups <= 0 || a->n_groups + 2 > kTcMaxGroups)
    return fail(DSV2_ERR_UNSUPPORTED, "moe: n_groups=%d (max %d)", a->n_groups, kTcMaxGroups - 2);
  if (a->hidden <= 0 || a->inter <= 0 || a->hidden % 64 || a->inter % 64)
    return fail(DSV2_ERR_UNSUPPORTED, "moe: hidden %d / inter %d must be multiples of 64", a->hidden,
                a->inter);
  if (a->x_rows <= 0 || a->max_routes_per_group <= 0) return DSV2_OK;
  if (!aligned16(a->gate_up) || !aligned16(a->down) || !aligned16(a->x_sorted) || !aligned16(a->h) ||
      !aligned16(a->y))
    return fail(DSV2_ERR_INVALID, "moe: operands must be 16-byte aligned");
  int sms = 0;
  int rc = ensure_init(&sms);
  if (rc) return rc;
  const uint64_t H = static_cast<uint64_t>(a->hidden), I = static_cast<uint64_t>(a->inter);
  const uint64_t G = static_cast<uint64_t>(a->n_groups), R = static_cast<uint64_t>(a->x_rows);
  if (a->tile_tokens < 0 || a->tile_tokens > 128 || a->tile_tokens % 16)
    return fail(DSV2_ERR_INVALID, "moe: tile_tokens %d (0, or a multiple of 16 up to 128)", a->tile_tokens);
  const MoeShape shp = moe_shape(a->max_routes_per_group, a->tile_tokens);
  CUtensorMap w1, x1, x1b, w2, hm, hb;
  if ((rc = tensor_map_3d(a->gate_up, H, 2 * I, G, H * 2, 2 * I * H * 2, 128, &w1))) return rc;
  if ((rc = tensor_map_3d(a->x_sorted, H, R, 1, H * 2, R * H * 2, 16, &x1))) return rc;
  if ((rc = tensor_map_3d(a->x_sorted, H, R, 1, H * 2, R * H * 2, shp.x_box, &x1b))) return rc;
  if ((rc = tensor_map_3d(a->down, I, H, G, I * 2, H * I * 2, 128, &w2))) return rc;
  if ((rc = tensor_map_3d(a->h, I, R, 1, I * 2, R * I * 2, 16, &hm))) return rc;
  if ((rc = tensor_map_3d(a->h, I, R, 1, I * 2, R * I * 2, shp.x_box, &hb))) return rc;
  MoeParams p = {};
  if ((rc = to_peers(a->peers, &p.peers))) return rc;
  p.n_groups = a->n_groups;
  p.hidden = a->hidden;
  p.inter = a->inter;
  p.x_rows = a->x_rows;
  p.group_offsets = a->group_offsets;
  p.max_routes_per_group = a->max_routes_per_group;
  p.route_slot = a->route_slot;
  p.route_weight = a->route_weight;
  p.h = reinterpret_cast<bf16*>(a->h);
  p.y = a->y;
  p.sync = a->sync;
  return check_launch(launch_moe_tc(p, w1, x1, x1b, w2, hm, hb, shp, sms,
                                    static_cast<cudaStream_t>(stream)),
                      "moe");
}

int dsv2_router(const dsv2_router_args* a, void* stream) {
  if (!a || !a->x || !a->w || !a->logits || !a->topk_ids32 || !a->topk_weights)
    return fail(DSV2_ERR_INVALID, "router: null pointer");
  if (a->n_experts <= 0 || a->n_experts > 64)
    return fail(DSV2_ERR_UNSUPPORTED, "router: n_experts=%d (max 64)", a->n_experts);
  if (a->hidden > 2048 || a->hidden % 64)
    return fail(DSV2_ERR_UNSUPPORTED, "router: hidden %d (need a multiple of 64, <= 2048)", a->hidden);
  if (a->rows > 4096) return fail(DSV2_ERR_UNSUPPORTED, "router: at most 4096 rows (got %d)", a->rows);
  if (!aligned16(a->x) || a->x_row_stride % 8)
    return fail(DSV2_ERR_INVALID, "router: activations must be 16-byte aligned rows");
  if (a->w_dtype != DSV2_BF16 && a->w_dtype != DSV2_F32)
    return fail(DSV2_ERR_UNSUPPORTED, "router: gate dtype %d", a->w_dtype);
  if (a->gather_out && (!a->group_offsets || !aligned16(a->gather_out)))
    return fail(DSV2_ERR_INVALID, "router: gather_out needs bucketing and 16-byte alignment");
  if (a->h) {
    if (a->w_dtype != DSV2_BF16 || (a->peers && a->peers->world > 1))
      return fail(DSV2_ERR_UNSUPPORTED, "router: the fused residual add + RMSNorm needs a bf16 gate on one rank");
    if (!a->norm_w || (a->n_delta > 0 && !a->delta) || a->n_delta < 0)
      return fail(DSV2_ERR_INVALID, "router: fused RMSNorm needs norm_w (and delta when n_delta > 0)");
    if (a->delta_dtype != DSV2_BF16 && a->delta_dtype != DSV2_F32)
      return fail(DSV2_ERR_UNSUPPORTED, "router: delta dtype %d", a->delta_dtype);
    if (a->norm_w_dtype != DSV2_BF16 && a->norm_w_dtype != DSV2_F32)
      return fail(DSV2_ERR_UNSUPPORTED, "router: norm weight dtype %d", a->norm_w_dtype);
    if (!aligned16(a->h) || (a->delta && !aligned16(a->delta)) || a->delta_row_stride % 8 ||
        a->delta_part_stride % 8)
      return fail(DSV2_ERR_INVALID, "router: h / delta must be 16-byte aligned rows");
  }
  if (a->rows <= 0) return DSV2_OK;
  if (a->group_offsets) {
    if (!a->route_token || !a->route_slot || !a->route_weight)
      return fail(DSV2_ERR_INVALID, "router: bucketing outputs missing");
    if (a->expert_lo < 0 || a->n_local < 0 || a->expert_lo + a->n_local > a->n_experts ||
        a->shared_lo < 0 || a->shared_hi < a->shared_lo || a->shared_hi > a->rows)
      return fail(DSV2_ERR_INVALID, "router: bad expert/shared ranges");
  }
  RouterParams p = {};
  if (int rc = to_peers(a->peers, &p.peers)) return rc;
  p.row_base = a->row_base;
  p.x = reinterpret_cast<const bf16*>(a->x);
  p.x_row_stride = a->x_row_stride;
  p.w = a->w;
  p.w_dtype = a->w_dtype;
  p.bias = a->bias;
  p.rows = a->rows;
  p.hidden = a->hidden;
  p.n_experts = a->n_experts;
  p.scaling = a->scaling;
  p.logits = a->logits;
  p.topk_ids = reinterpret_cast<long long*>(a->topk_ids64);
  p.topk_ids32 = a->topk_ids32;
  p.topk_w = a->topk_weights;
  p.gather_x = a->gather_out ? 1 : 0;
  p.gather_out = a->gather_out;
  p.expert_lo = a->expert_lo;
  p.n_local = a->n_local;
  p.shared_lo = a->shared_lo;
  p.shared_hi = a->shared_hi;
  p.group_offsets = a->group_offsets;
  p.route_token = a->route_token;
  p.route_slot = a->route_slot;
  p.route_weight = a->route_weight;
  p.h = reinterpret_cast<bf16*>(a->h);
  p.delta = a->delta;
  p.delta_dtype = a->delta_dtype;
  p.n_delta = a->delta ? a->n_delta : 0;
  p.delta_part_stride = a->delta_part_stride;
  p.delta_row_stride = a->delta_row_stride;
  p.norm_w = a->norm_w;
  p.norm_w_dtype = a->norm_w_dtype;
  p.eps = a->eps;
  p.x_out = a->h ? reinterpret_cast<bf16*>(const_cast<void*>(a->x)) : nullptr;
  p.grid_sync = a->sync;
  int sms = 0;
  if (int rc = ensure_init(&sms)) return rc;
  return check_launch(launch_router(p, router_clusters(), sms, static_cast<cudaStream_t>(stream)), "router");
}

int dsv2_softmax_topk(const float* logits, int rows, int n_experts, float scaling,
                      int64_t* topk_ids64, int32_t* topk_ids32, float* topk_weights,
                      void* stream) {
  if (!logits || !topk_ids32 || !topk_weights) return fail(DSV2_ERR_INVALID, "softmax_topk: null pointer");
  if (n_experts < 6 || n_experts > 64)
    return fail(DSV2_ERR_UNSUPPORTED, "softmax_topk: n_experts=%d", n_experts);
  if (rows <= 0) return DSV2_OK;
  return check_launch(launch_softmax_topk(logits, rows, n_experts, scaling,
                                          reinterpret_cast<long long*>(topk_ids64), topk_ids32,
                                          topk_weights, static_cast<cudaStream_t>(stream)),
                      "softmax_topk");
}

int dsv2_moe_bucket(const int32_t* topk_ids32, const float* topk_weights, int rows,
                    int expert_lo, int n_local, int shared_lo, int shared_hi,
                    int32_t* group_offsets, int32_t* route_token, int32_t* route_slot,
                    float* route_weight, const void* gather_src, int64_t gather_src_stride,
                    void* gather_out, int cols, const dsv2_peer_table* peers, int moe_layer,
                    void* stream) {
  if (!topk_ids32 || !topk_weights || !group_offsets || !route_token || !route_slot || !route_weight)
    return fail(DSV2_ERR_INVALID, "moe_bucket: null pointer");
  PeerTable pt;
  if (int rc = to_peers(peers, &pt)) return rc;
  if (rows > 4096) return fail(DSV2_ERR_UNSUPPORTED, "moe_bucket: at most 4096 rows (got %d)", rows);
  if (n_local < 0 || n_local > 64 || shared_lo < 0 || shared_hi < shared_lo || shared_hi > rows)
    return fail(DSV2_ERR_INVALID, "moe_bucket: bad ranges");
  if (gather_out && (!gather_src || cols % 8 || gather_src_stride % 8 || !aligned16(gather_src) ||
                     !aligned16(gather_out)))
    return fail(DSV2_ERR_INVALID, "moe_bucket: gather rows must be 16-byte aligned");
  if (rows <= 0) return DSV2_OK;
  int sms = 0;
  if (int rc = ensure_init(&sms)) return rc;
  return check_launch(launch_bucket(topk_ids32, topk_weights, rows, expert_lo, n_local, shared_lo,
                                    shared_hi, group_offsets, route_token, route_slot, route_weight,
                                    gather_out ? gather_src : nullptr, gather_src_stride, gather_out,
                                    cols, sms, static_cast<cudaStream_t>(stream), &pt, moe_layer),
                      "moe_bucket");
}

int dsv2_gather_rows(const void* x, int64_t x_row_stride, const int32_t* route_token,
                     const int32_t* group_offsets, int n_groups, void* out, int cols,
                     int max_routes, void* stream) {
  if (!x || !route_token || !group_offsets || !out) return fail(DSV2_ERR_INVALID, "gather_rows: null pointer");
  if (cols % 8 || !aligned16(x) || !aligned16(out) || x_row_stride % 8)
    return fail(DSV2_ERR_INVALID, "gather_rows: rows must be 16-byte aligned");
  return check_launch(launch_gather_rows(x, x_row_stride, route_token, group_offsets, n_groups,
                                         out, cols, max_routes, static_cast<cudaStream_t>(stream)),
                      "gather_rows");
}

int dsv2_mla_prep(const dsv2_mla_prep_args* a, void* stream) {
  if (!a || !a->qkva || !a->kv_norm_w || !a->cos_tab || !a->sin_tab || !a->positions || !a->cache ||
      !a->q_pe_out)
    return fail(DSV2_ERR_INVALID, "mla_prep: null pointer");
  if (a->pos_numel != 1 && a->pos_numel != a->batch)
    return fail(DSV2_ERR_INVALID, "mla_prep: positions numel %d for batch %d", a->pos_numel, a->batch);
  if (!aligned16(a->qkva) || a->qkva_row_stride % 8 || !aligned16(a->cache) || a->cache_b_stride % 8)
    return fail(DSV2_ERR_INVALID, "mla_prep: operands must be 16-byte aligned");
  if (a->rope_stride < 32) return fail(DSV2_ERR_INVALID, "mla_prep: rope table stride %lld < 32", (long long)a->rope_stride);
  if (a->batch <= 0) return DSV2_OK;
  if (a->cache_batch < 0) return fail(DSV2_ERR_INVALID, "mla_prep: cache_batch %d", a->cache_batch);
  MlaPrepParams p = {};
  p.cache_rows = a->cache_rows;
  p.cache_batch = a->cache_batch > 0 ? a->cache_batch : a->batch;
  if (a->qkva_dtype != DSV2_BF16 && a->qkva_dtype != DSV2_F32)
    return fail(DSV2_ERR_UNSUPPORTED, "mla_prep: qkva dtype %d", a->qkva_dtype);
  if (a->qkva_dtype == DSV2_F32 && (a->qkva_parts < 1 || a->qkva_part_stride % 4))
    return fail(DSV2_ERR_INVALID, "mla_prep: fp32 qkva needs >= 1 part and 16-byte part stride");
  if (a->q_nope_out && !aligned16(a->q_nope_out))
    return fail(DSV2_ERR_INVALID, "mla_prep: q_nope_out must be 16-byte aligned");
  p.qkva = a->qkva;
  p.qkva_f32 = a->qkva_dtype == DSV2_F32 ? 1 : 0;
  p.qkva_parts = a->qkva_dtype == DSV2_F32 ? a->qkva_parts : 1;
  p.qkva_part_stride = a->qkva_part_stride;
  p.q_nope_out = reinterpret_cast<bf16*>(a->q_nope_out);
  p.qkva_row_stride = a->qkva_row_stride;
  p.kv_norm_w = reinterpret_cast<const bf16*>(a->kv_norm_w);
  p.eps = a->eps;
  p.cos_tab = a->cos_tab;
  p.sin_tab = a->sin_tab;
  p.rope_stride = a->rope_stride;
  p.rope_rows = a->rope_rows;
  p.positions = reinterpret_cast<const long long*>(a->positions);
  p.pos_numel = a->pos_numel;
  p.cache = reinterpret_cast<bf16*>(a->cache);
  p.cache_b_stride = a->cache_b_stride;
  p.max_len = a->max_len;
  p.q_pe_out = reinterpret_cast<bf16*>(a->q_pe_out);
  return check_launch(launch_mla_prep(p, a->batch, static_cast<cudaStream_t>(stream)), "mla_prep");
}

int dsv2_mla_decode(const dsv2_mla_decode_args* a, void* stream) {
  if (!a || !a->q_abs || !a->q_pe || !a->cache || !a->positions || !a->o_part || !a->ml_part || !a->o_lat)
    return fail(DSV2_ERR_INVALID, "mla_decode: null pointer");
  const bool tc = a->family == DSV2_FAMILY_BATCH;
  if (!tc && a->family != DSV2_FAMILY_SMALL) return fail(DSV2_ERR_INVALID, "mla_decode: family %d", a->family);
  if (a->split_len <= 0 || a->split_len % (tc ? 64 : 32))
    return fail(DSV2_ERR_INVALID, "mla_decode: split_len %d must be a positive multiple of %d", a->split_len,
                tc ? 64 : 32);
  if (a->max_len <= 0 || a->n_splits <= 0) return fail(DSV2_ERR_INVALID, "mla_decode: max_len / n_splits");
  if (tc && static_cast<long long>(a->n_splits) * a->split_len < a->max_len)
    return fail(DSV2_ERR_INVALID, "mla_decode(batch): n_splits * split_len < max_len");
  if (!tc && !a->row_sync) return fail(DSV2_ERR_INVALID, "mla_decode: row_sync (int32[batch], zeroed) is required");
  if (tc && a->row_sync) return fail(DSV2_ERR_UNSUPPORTED, "mla_decode(batch): row_sync is not supported");
  if (tc && a->cache_rows) return fail(DSV2_ERR_UNSUPPORTED, "mla_decode(batch): cache_rows is not supported");
  if (a->cache_batch < 0) return fail(DSV2_ERR_INVALID, "mla_decode: cache_batch %d", a->cache_batch);
  if (!tc && static_cast<long long>(a->batch) * a->n_splits < 2)
    return fail(DSV2_ERR_INVALID, "mla_decode: batch * n_splits must give at least 2 partial slots");
  if (a->pos_numel != 1 && a->pos_numel != a->batch)
    return fail(DSV2_ERR_INVALID, "mla_decode: positions numel %d for batch %d", a->pos_numel, a->batch);
  if (!aligned16(a->q_abs) || !aligned16(a->q_pe) || !aligned16(a->cache) || a->cache_b_stride % 8 ||
      !aligned16(a->o_part))
    return fail(DSV2_ERR_INVALID, "mla_decode: operands must be 16-byte aligned");
  if (a->batch <= 0) return DSV2_OK;
  int sms = 0;
  int rc = ensure_init(&sms);
  if (rc) return rc;
  MlaDecodeParams p = {};
  p.q_abs = reinterpret_cast<const bf16*>(a->q_abs);
  p.q_pe = reinterpret_cast<const bf16*>(a->q_pe);
  p.cache = reinterpret_cast<const bf16*>(a->cache);
  p.cache_b_stride = a->cache_b_stride;
  p.max_len = a->max_len;
  p.positions = reinterpret_cast<const long long*>(a->positions);
  p.pos_numel = a->pos_numel;
  p.scale_log2 = a->softmax_scale * 1.4426950408889634f;
  p.split_len = a->split_len;
  p.n_splits = a->n_splits;
  p.o_part = a->o_part;
  p.ml_part = a->ml_part;
  p.o_lat = reinterpret_cast<bf16*>(a->o_lat);
  p.inputs_prior = a->inputs_prior != 0;
  p.row_sync = a->row_sync;
  p.batch = a->batch;
  p.cache_rows = a->cache_rows;
  p.cache_batch = a->cache_batch > 0 ? a->cache_batch : a->batch;
  if (a->part_count) {
    if (tc || a->batch != 1 || a->cache_rows)
      return fail(DSV2_ERR_UNSUPPORTED, "mla_decode: part_count (unmerged partials) needs the small family and batch 1");
    p.part_count = a->part_count;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap tm_kv;
  if (tc) {
    if ((rc = mla_cache_map(a->cache, a->cache_b_stride, a->max_len, a->batch, 64, &tm_kv))) return rc;
    rc = check_launch(launch_mla_tc(p, tm_kv, a->batch, st), "mla_decode(batch)");
    if (rc) return rc;
    return check_launch(launch_mla_combine(p, a->batch, st), "mla_combine");
  }
  return mla_decode_balanced(p, sms, static_cast<long long>(a->batch) * a->n_splits, st, "mla_decode");
}

// Same computation as dsv2_mla_decode (mma.sync kernel), with the partials and the row
// tickets kept in the library's fixed device array instead of caller buffers (no
// allocation of any kind here).
int dsv2_mla_decode_noalloc(const void* q_abs, const void* q_pe, const void* cache,
                            int64_t cache_b_stride, int max_len, const int64_t* positions,
                            int pos_numel, float softmax_scale, int split_len, void* o_lat,
                            int batch, void* stream) {
  if (!q_abs || !q_pe || !cache || !positions || !o_lat)
    return fail(DSV2_ERR_INVALID, "mla_decode_noalloc: null pointer");
  if (split_len <= 0 || split_len % 32 || max_len <= 0)
    return fail(DSV2_ERR_INVALID, "mla_decode_noalloc: split_len %d must be a positive multiple of 32",
                split_len);
  if (pos_numel != 1 && pos_numel != batch)
    return fail(DSV2_ERR_INVALID, "mla_decode_noalloc: positions numel %d for batch %d", pos_numel, batch);
  if (!aligned16(q_abs) || !aligned16(q_pe) || !aligned16(cache) || cache_b_stride % 8)
    return fail(DSV2_ERR_INVALID, "mla_decode_noalloc: operands must be 16-byte aligned");
  if (batch <= 0) return DSV2_OK;
  if (batch > kNoAllocMaxRows)
    return fail(DSV2_ERR_INVALID, "mla_decode_noalloc: batch %d exceeds the %d row tickets of the built-in "
                "scratch; use dsv2_mla_decode", batch, kNoAllocMaxRows);
  int sms = 0;
  int rc = ensure_init(&sms);
  if (rc) return rc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(DSV2_ERR_LAUNCH, "mla_decode_noalloc: cudaGetDevice");
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    scratch = g_noalloc_scratch[dev];
  }
  MlaDecodeParams p = {};
  p.q_abs = reinterpret_cast<const bf16*>(q_abs);
  p.q_pe = reinterpret_cast<const bf16*>(q_pe);
  p.cache = reinterpret_cast<const bf16*>(cache);
  p.cache_b_stride = cache_b_stride;
  p.max_len = max_len;
  p.positions = reinterpret_cast<const long long*>(positions);
  p.pos_numel = pos_numel;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.split_len = split_len;
  p.n_splits = 1;
  p.o_part = scratch;
  p.ml_part = scratch + static_cast<size_t>(kNoAllocMaxParts) * kHeads * kLatent;
  p.row_sync = reinterpret_cast<int*>(scratch + kNoAllocTicketOffset);
  p.o_lat = reinterpret_cast<bf16*>(o_lat);
  p.batch = batch;
  p.cache_batch = batch;
  return mla_decode_balanced(p, sms, kNoAllocMaxParts, static_cast<cudaStream_t>(stream), "mla_decode_noalloc");
}

}  // extern "C"
