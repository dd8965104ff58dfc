// Shared device helpers for the DeepSeek-V2-Lite decode kernels (sm_100a only).
//
// bf16 packing helpers, warp reductions, cp.async / ldmatrix / mma.sync wrappers
// for the latent-attention kernel, and the mbarrier / TMA / tcgen05 wrappers used
// by the tensor-core linear kernel.  Every spin-wait here is bounded: a wait that
// runs out of iterations returns false and the caller records an error status
// instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "this library targets sm_100a only"
#endif

namespace dsv2 {

typedef __nv_bfloat16 bf16;

// Device-side error word shared by every kernel of the library.  A nonzero value
// means a bounded wait gave up or an index check failed; the host reads it back
// through dsv2_get_device_error().
enum DeviceError : int {
  kErrNone = 0,
  kErrMbarTimeout = 1,
  kErrIndex = 2,
  kErrTmemAlloc = 3,
};

// Defined here: the library is one translation unit (dsv2_all.cu).
__device__ int g_device_error = 0;

__device__ __forceinline__ void set_device_error(int code) {
  atomicCAS(&g_device_error, 0, code);
}

// ----------------------------------------------------------------------------
// Programmatic dependent launch
// ----------------------------------------------------------------------------
// Every kernel of the library is launched with programmatic stream serialization
// (launch_kernel below): the next kernel of the stream may be scheduled before this
// one completes.  Protocol, followed by every kernel:
//   1. work that touches no data written by the last two kernels of the stream
//      (weights, tensor maps, shared memory / TMEM setup, and inputs the caller
//      states were written earlier) may run first;
//   2. pdl_wait() before reading anything the previous kernel wrote or writing
//      anything it may still read (griddepcontrol.wait: the previous grid has
//      completed and its writes are visible);
//   3. pdl_launch_dependents() only after that wait, so the next kernel starts once
//      every CTA of this one is past its wait, i.e. once the kernel before this one
//      has completed.  That is what makes inputs written two launches back safe to
//      read in step 1, and it keeps at most one early grid waiting per kernel.
// Every CTA reaches pdl_wait() on every path, early exits included, so a grid never
// completes before its predecessor and completion stays ordered along the stream.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// steps 2 and 3, at the top of a kernel that has nothing to do before its inputs are ready
__device__ __forceinline__ void pdl_enter() {
  pdl_wait();
  pdl_launch_dependents();
}

// ----------------------------------------------------------------------------
// Cross-GPU signals (expert parallelism over NVLink peer memory)
// ----------------------------------------------------------------------------
// A writer stores its data into a peer's buffer, fences at system scope and adds to the
// peer's counter with release semantics; the reader polls its own counter with acquire
// semantics (bounded) and then reads the data with L1-bypassing loads.  Counters only
// grow; the expected value of a wait is derived from the step counter.
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Returns false (and records kErrMbarTimeout) when the counter does not reach target
// within `polls` polls (0: 2^24, several seconds); gives up at once when an earlier wait
// of any kernel already failed (so that a broken exchange ends quickly instead of timing
// out at every layer).
constexpr uint32_t kPeerWaitPolls = 1u << 24;
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// stat (optional): [0] += nanoseconds spent in this wait, [1] += 1
__device__ __forceinline__ bool wait_counter_sys(const unsigned long long* ctr, unsigned long long target,
                                                 uint32_t polls, unsigned long long* stat = nullptr) {
  const uint32_t limit = polls ? polls : kPeerWaitPolls;
  const unsigned long long t0 = stat ? globaltimer_ns() : 0ull;
  bool ok = false;
  for (uint32_t i = 0; i < limit; ++i) {
    if (ld_acquire_sys_u64(ctr) >= target) { ok = true; break; }
    if ((i & 255) == 0 && *reinterpret_cast<volatile int*>(&g_device_error) != 0) return false;
    __nanosleep(64);
  }
  if (stat) {
    atomicAdd(&stat[0], globaltimer_ns() - t0);
    atomicAdd(&stat[1], 1ull);
  }
  if (!ok) set_device_error(kErrMbarTimeout);
  return ok;
}

// ----------------------------------------------------------------------------
// bf16 <-> fp32
// ----------------------------------------------------------------------------
__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// dot of 8 bf16 pairs packed in two uint4 words, accumulated in fp32
__device__ __forceinline__ float dot8(const uint4& a, const uint4& b, float acc) {
  acc = fmaf(bf16lo(a.x), bf16lo(b.x), acc);
  acc = fmaf(bf16hi(a.x), bf16hi(b.x), acc);
  acc = fmaf(bf16lo(a.y), bf16lo(b.y), acc);
  acc = fmaf(bf16hi(a.y), bf16hi(b.y), acc);
  acc = fmaf(bf16lo(a.z), bf16lo(b.z), acc);
  acc = fmaf(bf16hi(a.z), bf16hi(b.z), acc);
  acc = fmaf(bf16lo(a.w), bf16lo(b.w), acc);
  acc = fmaf(bf16hi(a.w), bf16hi(b.w), acc);
  return acc;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Streaming 16-byte load that bypasses L1 allocation (weights are read once).
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------------------
// cp.async (16 B) + ldmatrix + mma.sync.m16n8k16 (bf16 -> fp32)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ----------------------------------------------------------------------------
// mbarrier (bounded waits)
// ----------------------------------------------------------------------------
// Iteration cap for every mbarrier wait: ~2^27 polls is several seconds on a
// B200, far above any legitimate wait in these kernels.
constexpr uint32_t kSpinLimit = 1u << 27;

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Returns false (and records kErrMbarTimeout) when the wait gives up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  set_device_error(kErrMbarTimeout);
  return false;
}

// ----------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(dst),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4, %5}], [%2];" ::"r"(dst),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// TMA store of a box from shared memory (bulk-group completion)
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// every committed bulk store of this thread has completed (its global writes are done)
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ----------------------------------------------------------------------------
// Thread-block clusters and distributed shared memory
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t n_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_addr(const void* local, uint32_t rank) {
  const uint32_t la = static_cast<uint32_t>(__cvta_generic_to_shared(local));
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(rank));
  return ra;
}
// store v at the address of `local` in the shared memory of cluster CTA `rank`
__device__ __forceinline__ void st_cluster_f32(const float* local, uint32_t rank, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr(local, rank)), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_v4(const void* local, uint32_t rank, uint4 v) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr(local, rank)),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
// ----------------------------------------------------------------------------
// tcgen05 (5th-gen tensor cores, accumulators in TMEM), cta_group::1 only
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc)^T, bf16 inputs, fp32 accumulate
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// 32 lanes x 16 columns of 32-bit: thread i of the warp gets lane (quadrant base + i)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%"
      "15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 16 columns of 32-bit from registers (the inverse of tmem_ld16)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%"
      "16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// make this thread's generic-proxy shared-memory writes visible to the async proxy
// (tensor-core operand reads)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor for an MN-major operand stored with the 128-byte
// swizzle: rows of 64 MN-contiguous bf16 (one K index each), 8-row atoms of 1024 B along
// K (stride sbo between atoms), the next 64 MN elements lbo bytes further.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3fffu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;             // descriptor version for sm_100
  d |= static_cast<uint64_t>(2u) << 61;             // SWIZZLE_128B
  return d;
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 64 bf16, 8-row atoms of 1024 B).  Field layout:
// start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46), version=1 [46,48),
// base offset [49,52), layout type [61,64) (2 = SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3fffu);
  d |= static_cast<uint64_t>(1u) << 16;             // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;     // SBO: 8 rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;             // descriptor version for sm_100
  d |= static_cast<uint64_t>(2u) << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B, fp32 D, both K-major
// (a_mn_major: A is MN-major instead, bit 15).
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, bool a_mn_major = false) {
  return (1u << 4)                                  // D format: f32
         | (1u << 7)                                // A format: bf16
         | (1u << 10)                               // B format: bf16
         | (a_mn_major ? (1u << 15) : 0u)           // A major-ness
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

}  // namespace dsv2

// ----------------------------------------------------------------------------
// Host-side launch helper
// ----------------------------------------------------------------------------
#include <atomic>

namespace dsv2 {

// Programmatic stream serialization for every launch (on unless DSV2_PDL=0 in the
// environment when the library initialises) and a count of the kernels enqueued.
inline bool g_pdl_enabled = true;
inline std::atomic<long long> g_kernel_launches{0};

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = g_pdl_enabled ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace dsv2
