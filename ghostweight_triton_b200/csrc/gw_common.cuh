// Shared device helpers for the ghostweight B200 kernels (sm_100a only).
//
// Everything here is hand-written inline PTX for the Blackwell async machinery:
// mbarriers, TMA tile loads, and the tcgen05 (5th-gen tensor core + TMEM) ops.
// Each wait on an mbarrier is bounded: after GW_WAIT_LIMIT_NS of wall time the
// wait gives up, raises a bit in the module error word and tells the caller to
// abandon its loop, so a logic error can never wedge the GPU.
#pragma once

#include <cstdint>
#include <mutex>
#include <unordered_map>
#include <utility>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "../../include/ghostweight_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "ghostweight_b200 kernels are written for sm_100a (B200) only"
#endif

namespace gw {

// Wall-clock limit for any single mbarrier wait (2 s). A correct kernel never
// comes close: the longest legitimate wait is one output tile's main loop.
constexpr unsigned long long GW_WAIT_LIMIT_NS = 2000000000ull;

// Bits of the module-wide device error word (read back by gw_get_device_error).
enum : unsigned int {
  GW_DERR_WAIT_TIMEOUT = 1u << 0,   // an mbarrier wait ran out of time
  GW_DERR_BAD_INDEX    = 1u << 1,   // an alive index was outside [0, K)
};

// The error word lives in gw_api.cu; kernels in other translation units get
// its device address as a parameter (no relocatable device code).
__device__ __forceinline__ void raise_error(unsigned int* err, unsigned int bits) {
  if (err) atomicOr(err, bits);
}

// First x column of k-block j when the alive columns form 64-column runs:
// cols[64 j]. Producers load it one stage ahead (run_start_load) so that the
// load's latency hides behind the wait for a free stage, then validate it
// (run_start_check): a TMA box may only start at a column whose byte offset is
// a multiple of 16 (8 columns of 16 bits), so a start outside [0, width) or not
// a multiple of 8 raises GW_DERR_BAD_INDEX and column 0 is loaded instead.
__device__ __forceinline__ int64_t run_start_load(const int64_t* cols, int j) {
  return __ldg(cols + static_cast<int64_t>(j) * 64);
}
__device__ __forceinline__ int run_start_check(int64_t c, int64_t width, unsigned int* err) {
  if (c < 0 || c >= width || (c & 7) != 0) {
    raise_error(err, GW_DERR_BAD_INDEX);
    return 0;
  }
  return static_cast<int>(c);
}

// k-blocks of a GEMM whose alive count lives on the device (written by an
// earlier kernel; read after griddepcontrol.wait): ceil(count / 64), at least
// one (a zero-filled k-block when the count is 0), at most the launch's bound.
__device__ __forceinline__ int device_num_kb(const int32_t* k_dev, int max_kb) {
  const int n = *reinterpret_cast<const volatile int32_t*>(k_dev);
  const int kb = (max(n, 0) + 63) / 64;
  return min(max(kb, 1), max_kb);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ----------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :: "r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity. Returns false when the
// CTA-wide abort flag is (or becomes) set, or the wall-clock limit is hit; in
// the latter case the abort flag and the module error word are raised.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          volatile int* abort_flag,
                                          unsigned int* err,
                                          unsigned long long limit_ns = GW_WAIT_LIMIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0u) {
      if (abort_flag && *abort_flag) return false;
      if (global_timer_ns() - t0 > limit_ns) {
        if (abort_flag) *abort_flag = 1;
        raise_error(err, GW_DERR_WAIT_TIMEOUT);
        return false;
      }
    }
  }
}

// ----------------------------------------------------------------------------
// TMA (non-multicast tile loads only)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// Brings a 2-D tile of the tensor into L2 (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_l2_2d(const void* tmap, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];"
               :: "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y) : "memory");
}

// 2-D tile load global -> shared, completion signalled on `bar` as tx bytes.
// x is the innermost (contiguous) coordinate in elements; callers keep
// x * sizeof(elem) a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int32_t x, int32_t y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];"
      :: "r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2-D tile store shared -> global through the TMA unit, tracked by the
// thread's bulk async-group. x * sizeof(elem) must be a multiple of 16 bytes
// and x, y non-negative; elements outside the tensor map's extent are not
// written.
__device__ __forceinline__ void tma_store_2d(const void* tmap, uint32_t src, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];"
      :: "l"(reinterpret_cast<uint64_t>(tmap)), "r"(src), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N of this thread's bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" :: "n"(N) : "memory");
}
// Wait until all of this thread's bulk groups have completed.
__device__ __forceinline__ void bulk_wait_group_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Orders generic-proxy global accesses against async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Streaming 16-bit global load that does not allocate in L1.
__device__ __forceinline__ uint32_t ld_stream_u16(const uint16_t* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const unsigned int* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(unsigned int* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

// Barrier over `nthreads` threads (a multiple of 32) of the CTA, id 1..15.
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

// Bounded wait until *counter >= target (acquire). Same abort/timeout contract
// as mbar_wait.
__device__ __forceinline__ bool wait_counter_geq(const unsigned int* counter, uint32_t target,
                                                 volatile int* abort_flag, unsigned int* err,
                                                 unsigned long long limit_ns = GW_WAIT_LIMIT_NS) {
  if (ld_acquire_gpu(counter) >= target) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(64);
    if (ld_acquire_gpu(counter) >= target) return true;
    if ((i & 63u) == 0u) {
      if (abort_flag && *abort_flag) return false;
      if (global_timer_ns() - t0 > limit_ns) {
        if (abort_flag) *abort_flag = 1;
        raise_error(err, GW_DERR_WAIT_TIMEOUT);
        return false;
      }
    }
  }
}

// ----------------------------------------------------------------------------
// tcgen05 / TMEM
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(dst_smem), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
               :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16 or bf16 in, fp32 accumulate).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every previously issued tcgen05 op of this thread completes.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(bar) : "memory");
}

__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Each lane reads 32 consecutive 32-bit TMEM columns of its own lane (row).
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Each lane reads 16 consecutive 32-bit TMEM columns of its own lane (row).
__device__ __forceinline__ void tc_ld_32x32b_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored in the
// 128-byte-swizzled canonical layout: rows of 128 B (64 16-bit elements),
// 16-byte chunk c of row r stored at chunk position c ^ (r % 8), groups of 8
// rows 1024 B apart. Tile base must be 1024-byte aligned.
__device__ __forceinline__ uint64_t smem_desc_kmajor_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);      // start address
  d |= static_cast<uint64_t>(1u) << 16;                     // leading byte offset (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;             // stride byte offset: 8 rows * 128 B
  d |= static_cast<uint64_t>(1u) << 46;                     // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;                     // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor, kind::f16, fp32 accumulate, A and B both K-major.
// ab_format: 0 = fp16, 1 = bf16 (A and B always share one type).
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t ab_format, uint32_t m, uint32_t n) {
  return (1u << 4)                 // D format: f32
       | (ab_format << 7)          // A format
       | (ab_format << 10)         // B format
       | ((n >> 3) << 17)          // N / 8
       | ((m >> 4) << 24);         // M / 16
}

// ----------------------------------------------------------------------------
// Clusters of two CTAs (2-SM tcgen05 MMA). No TMA multicast anywhere: each CTA
// loads its own operand halves; only MMA completion is multicast (commit).
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(saddr), "r"(rank));
  return out;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// The two halves of cluster_sync, for barriers whose wait can come much later
// than the arrive (every thread of the CTA executes each, in order).
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive without ordering this thread's earlier memory operations (a release
// arrive waits for them, remote stores included).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// this CTA's shared memory into another CTA's (cluster-window address of the
// destination and of its mbarrier), counted as transaction bytes on that
// mbarrier. The source must stay untouched until the data has landed.
__device__ __forceinline__ void bulk_copy_to_cta(uint32_t cluster_dst, uint32_t src, uint32_t bytes,
                                                 uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      :: "r"(cluster_dst), "r"(src), "r"(bytes), "r"(cluster_bar) : "memory");
}

// 16-byte store into another CTA's shared memory (cluster-window addresses of
// the destination and of its mbarrier), counted as 16 transaction bytes on
// that mbarrier when it lands.
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, float a, float b, float c,
                                            float d, uint32_t cluster_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
      :: "r"(cluster_addr), "f"(a), "f"(b), "f"(c), "f"(d), "r"(cluster_bar) : "memory");
}

// Arrive on an mbarrier of another CTA of the cluster (cluster-window address).
// Default semantics (release at CTA scope): the arrivals this is used for only
// publish "my tensor-memory reads are complete" (ordered by tcgen05.wait::ld
// and tcgen05.fence::before_thread_sync), so they need not wait for the
// thread's outstanding global stores as a cluster-scope release would.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];"
               :: "r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}

// Bounded wait with cluster-scope acquire, for barriers that other CTAs (or
// their TMA/MMA completions) arrive on. Same contract as mbar_wait.
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity,
                                                  volatile int* abort_flag, unsigned int* err,
                                                  unsigned long long limit_ns = GW_WAIT_LIMIT_NS) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 255u) == 0u) {
      if (abort_flag && *abort_flag) return false;
      if (global_timer_ns() - t0 > limit_ns) {
        if (abort_flag) *abort_flag = 1;
        raise_error(err, GW_DERR_WAIT_TIMEOUT);
        return false;
      }
    }
  }
}

// 2-D TMA tile load into this CTA's shared memory whose completion bytes are
// counted on `cluster_bar` (the pair leader's barrier). Not multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* tmap, int32_t x,
                                                 int32_t y, uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];"
      :: "r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(cluster_bar)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(dst_smem), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;"
               :: "r"(taddr), "r"(ncols) : "memory");
}

// D (both CTAs' TMEM) (+)= A (both CTAs' smem) * B (both CTAs' smem)^T, M = 256.
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the barrier at this shared offset in every CTA of `mask` when
// this thread's prior pair MMAs complete.
__device__ __forceinline__ void tc_commit_pair_mc(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;"
      :: "r"(bar), "h"(mask) : "memory");
}

// Host: raise `kern`'s dynamic shared-memory limit to `bytes` once per device
// (the attribute sticks to the function; re-setting it on every launch costs a
// driver call).
inline cudaError_t ensure_smem_attr(const void* kern, int bytes) {
  static std::mutex mu;
  static std::unordered_map<const void*, uint64_t> done;   // bit d: set on device d
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (uint64_t{1} << dev) : 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = done.find(kern);
    if (bit && it != done.end() && (it->second & bit)) return cudaSuccess;
  }
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  done[kern] |= bit;
  return cudaSuccess;
}

// Host: launch `kern` as a programmatic dependent of the previous work of the
// stream (it may start before that work completes and must execute
// griddepcontrol.wait before touching its results).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ----------------------------------------------------------------------------
// Scalar conversions
// ----------------------------------------------------------------------------
template <int DT> struct Elem;
template <> struct Elem<GW_DTYPE_F16> {
  using raw = uint16_t;
  static __device__ __forceinline__ float to_f(raw v) { return __half2float(__ushort_as_half(v)); }
  static __device__ __forceinline__ raw from_f(float f) { return __half_as_ushort(__float2half_rn(f)); }
  // Two values rounded in one packed conversion: lo in bits 0-15, hi in 16-31.
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};
template <> struct Elem<GW_DTYPE_BF16> {
  using raw = uint16_t;
  static __device__ __forceinline__ float to_f(raw v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }
  static __device__ __forceinline__ raw from_f(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};
template <> struct Elem<GW_DTYPE_F32> {
  using raw = uint32_t;
  static __device__ __forceinline__ float to_f(raw v) { return __uint_as_float(v); }
  static __device__ __forceinline__ raw from_f(float f) { return __float_as_uint(f); }
};

// Output activation applied in GEMM epilogues, from the GELU definitions
// (Hendrycks & Gimpel): exact erf form and the tanh approximation. erff / tanhf
// are CUDA's own functions.
__device__ __forceinline__ float apply_epilogue(float v, int epi) {
  if (epi == GW_EPI_GELU_ERF) {
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
  } else if (epi == GW_EPI_GELU_TANH) {
    const float u = 0.79788456080286535588f * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.0f + tanhf(u));
  }
  return v;
}

// The same for epilogues that round to fp16/bf16: the tanh form uses the
// identity 0.5 v (1 + tanh(u)) = v * sigmoid(2 u) = v / (1 + exp(-2 u)) with
// CUDA's fast exponential and division intrinsics (a few ulp of fp32, far below
// the 16-bit rounding), a third of tanhf's instructions; the erf form is
// unchanged.
__device__ __forceinline__ float apply_epilogue16(float v, int epi) {
  if (epi == GW_EPI_GELU_TANH) {
    const float u = 0.79788456080286535588f * (v + 0.044715f * v * v * v);
    return __fdividef(v, 1.0f + __expf(-2.0f * u));
  }
  return apply_epilogue(v, epi);
}

// Epilogue arithmetic for 32 consecutive output columns [n0, n0 + 32) of one
// row (the 32 values a lane holds after one 32-column TMEM load).
// Bias: four 16-byte loads when the 32 values lie inside [0, N) and are
// 16-byte aligned (every lane of the warp reads the same addresses), else one
// load per element.
template <int DT>
__device__ __forceinline__ void add_bias32(float (&f)[32], const uint16_t* bias, int64_t n0,
                                           int64_t N) {
  const uint16_t* b = bias + n0;
  if (n0 + 32 <= N && (reinterpret_cast<uintptr_t>(b) & 15u) == 0) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(b) + v);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        f[8 * v + 2 * k] += Elem<DT>::to_f(static_cast<uint16_t>(w[k] & 0xFFFFu));
        f[8 * v + 2 * k + 1] += Elem<DT>::to_f(static_cast<uint16_t>(w[k] >> 16));
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < N) f[j] += Elem<DT>::to_f(__ldg(bias + n0 + j));
  }
}
// The same for four consecutive columns [n0, n0 + 4): one 8-byte load when
// they lie inside [0, N) and are 8-byte aligned.
template <int DT>
__device__ __forceinline__ void add_bias4(float (&f)[4], const uint16_t* bias, int64_t n0,
                                          int64_t N) {
  const uint16_t* b = bias + n0;
  if (n0 + 4 <= N && (reinterpret_cast<uintptr_t>(b) & 7u) == 0) {
    const uint2 q = __ldg(reinterpret_cast<const uint2*>(b));
    f[0] += Elem<DT>::to_f(static_cast<uint16_t>(q.x & 0xFFFFu));
    f[1] += Elem<DT>::to_f(static_cast<uint16_t>(q.x >> 16));
    f[2] += Elem<DT>::to_f(static_cast<uint16_t>(q.y & 0xFFFFu));
    f[3] += Elem<DT>::to_f(static_cast<uint16_t>(q.y >> 16));
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (n0 + j < N) f[j] += Elem<DT>::to_f(__ldg(bias + n0 + j));
  }
}
// Activation chosen at compile time, so a kernel instantiation carries the
// code of one activation only.
template <int EPI>
__device__ __forceinline__ void activate32(float (&f)[32]) {
  if constexpr (EPI != GW_EPI_NONE) {
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = apply_epilogue16(f[j], EPI);
  }
}
template <int EPI>
__device__ __forceinline__ void activate4(float (&f)[4]) {
  if constexpr (EPI != GW_EPI_NONE) {
#pragma unroll
    for (int j = 0; j < 4; ++j) f[j] = apply_epilogue16(f[j], EPI);
  }
}

}  // namespace gw
