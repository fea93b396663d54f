// fqkv_device.cuh -- sm_100a device primitives used by the fused RMSNorm+QKV kernels:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM alloc / MMA / commit /
// load), UMMA shared-memory descriptors, cluster (DSMEM) helpers and programmatic
// dependent launch.  Every wait in this file gives up after a time limit, records
// FQKV_STATUS_WAIT_TIMEOUT in the device status word and returns false, so no kernel
// built on it can spin forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/fused_rmsnorm_qkv.h"

namespace fqkv {

// Device status word (one per device that loaded the library).  Written only on
// failure; read and cleared by fqkv_device_status().
extern __device__ int g_status;

// A bounded wait gives up after g_wait_limit_ns nanoseconds of %globaltimer: 1 s unless a
// test shortens it (fqkv_test_set_wait_limit_ns).
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s
extern __device__ unsigned long long g_wait_limit_ns;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_status(int bits) { atomicOr(&g_status, bits); }

// ------------------------------------------------------------------ timeline trace
// Profiling builds only (-DFQKV_TRACE): a kernel takes one record per CTA from a buffer
// installed with fqkv_trace_attach and writes %clock64 at its phase boundaries, plus its
// block index, SM and %globaltimer at entry and exit, so that CTAs of consecutive launches
// can be laid out on one time axis.  In the normal build the macros expand to nothing.
#ifdef FQKV_TRACE
constexpr int kTraceSlots = 24;
extern __device__ unsigned long long* g_trace_buf;
extern __device__ unsigned int g_trace_cap;
extern __device__ unsigned int g_trace_ctr;
__device__ __forceinline__ unsigned long long clock64_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
  return t;
}
// The stamps are kept in shared memory while the kernel runs and written out by
// FQKV_TRACE_END; the record index (a global atomic) is requested at entry but first used at
// the end, so its latency stays off the traced path.
#define FQKV_TRACE_DECL                                                                                  \
  __shared__ unsigned long long fqkv_trace_s_[::fqkv::kTraceSlots];                                      \
  unsigned int fqkv_trace_i_ = 0xFFFFFFFFu;
// Thread 0, first thing in the kernel.
#define FQKV_TRACE_BEGIN()                                                                               \
  do {                                                                                                   \
    if (threadIdx.x == 0) {                                                                              \
      unsigned long long g0;                                                                             \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g0));                                             \
      const unsigned long long c0 = ::fqkv::clock64_now();                                               \
      unsigned int smid;                                                                                 \
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));                                                  \
      if (::fqkv::g_trace_buf) fqkv_trace_i_ = atomicAdd(&::fqkv::g_trace_ctr, 1u);                      \
      fqkv_trace_s_[0] = (unsigned long long)blockIdx.x | ((unsigned long long)blockIdx.y << 16) |       \
                         ((unsigned long long)smid << 32) | ((unsigned long long)gridDim.x << 40) |      \
                         ((unsigned long long)gridDim.y << 48);                                          \
      fqkv_trace_s_[1] = g0;                                                                             \
      fqkv_trace_s_[2] = c0;                                                                             \
    }                                                                                                    \
  } while (0)
// Slots a CTA does not stamp hold whatever shared memory held; readers keep only stamps
// between the entry and exit clocks.
#define FQKV_TRACE_POINT(slot) (fqkv_trace_s_[(slot)] = ::fqkv::clock64_now())
// Every thread of the block, once all of them have made their last stamp.
#define FQKV_TRACE_END()                                                                                 \
  do {                                                                                                   \
    __syncthreads();                                                                                     \
    if (threadIdx.x == 0 && fqkv_trace_i_ < ::fqkv::g_trace_cap) {                                       \
      unsigned long long g1;                                                                             \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(g1));                                             \
      fqkv_trace_s_[::fqkv::kTraceSlots - 2] = ::fqkv::clock64_now();                                    \
      fqkv_trace_s_[::fqkv::kTraceSlots - 1] = g1;                                                       \
      for (int s_ = 0; s_ < ::fqkv::kTraceSlots; ++s_)                                                   \
        ::fqkv::g_trace_buf[(size_t)fqkv_trace_i_ * ::fqkv::kTraceSlots + s_] = fqkv_trace_s_[s_];       \
    }                                                                                                    \
  } while (0)
#else
#define FQKV_TRACE_DECL
#define FQKV_TRACE_BEGIN() ((void)0)
#define FQKV_TRACE_POINT(slot) ((void)0)
#define FQKV_TRACE_END() ((void)0)
#endif

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init_cluster() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Arrive on an mbarrier of another CTA of the cluster (address from mapa_shared).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// Relaxed remote arrive: pair with one fence_acq_rel_cluster() before a batch of them.
__device__ __forceinline__ void mbar_arrive_remote_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }

// Local arrive that also announces `bytes` of incoming transactions (cluster scope: the
// bytes come from st.async writes of other CTAs).
__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.relaxed.cluster.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Store 4 bytes into another CTA's shared memory and count them on that CTA's mbarrier
// (complete_tx); the data is visible to whoever observes the barrier phase complete.
__device__ __forceinline__ void st_async_f32(uint32_t cluster_addr, float v, uint32_t cluster_bar) {
  asm volatile("st.async.weak.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(cluster_addr),
               "r"(__float_as_uint(v)), "r"(cluster_bar)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false (and records
// a timeout) if it has not completed within g_wait_limit_ns.
template <bool kClusterScope = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (kClusterScope ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns(), limit = *(volatile unsigned long long*)&g_wait_limit_ns;
  for (uint32_t it = 1;; ++it) {
    if (kClusterScope ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u && globaltimer_ns() - t0 > limit) {
      record_status(FQKV_STATUS_WAIT_TIMEOUT);
      return false;
    }
  }
}

// AND of `v` over the `count` threads meeting at named barrier `id` (uniform result).
__device__ __forceinline__ bool bar_and(int id, int count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// ------------------------------------------------------------------ fences
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bring the 128-byte line that holds `p` (a global-memory address) into L2; nothing is
// loaded into registers.
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p) : "memory");
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of box {x = inner (K), y = rows} into CTA-local shared memory,
// completing `bytes` on `bar`.  x must be a multiple of 8 elements (16 bytes).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Same, with an L2 eviction-priority hint (createpolicy result).
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                                 int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// Bulk copy from this CTA's shared memory into another CTA's shared memory (cluster
// addresses for the destination and its mbarrier), counted there by complete_tx.  Both
// addresses 16-byte aligned, `bytes` a multiple of 16; one destination, no multicast.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src_smem, uint32_t bytes,
                                                  uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst_cluster),
               "r"(src_smem), "r"(bytes), "r"(bar_cluster)
               : "memory");
}

// 2-D tiled store of box {x, y} from this CTA's shared memory to global memory, tracked
// by the issuing thread's bulk async-groups.  x must be a multiple of 8 elements and
// x, y >= 0; the parts of the box outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N of this thread's bulk async-groups are still reading shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until at most N of this thread's bulk async-groups are incomplete (writes performed).
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ------------------------------------------------------------------ PDL
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------ cluster
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Named CTA barriers: `count` threads (a multiple of 32) in all; arriving threads do not wait.
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync() {
  cluster_arrive_release();
  cluster_wait_acquire();
}
// Per-thread (not warp-aligned) halves of the cluster barrier, for warps whose lanes
// reach them at different points.
__device__ __forceinline__ void cluster_arrive_release_thread() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
// Arrival that orders nothing: for barriers that only have to synchronise execution.
__device__ __forceinline__ void cluster_arrive_relaxed_thread() {
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire_thread() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}

// Shared::cluster address of the variable at `local_addr` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16 or bf16 in, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f8f6f4 (here e4m3 x e4m3, fp32 accumulate):
// 32 one-byte K elements per instruction, the same 32-byte descriptor step as kind::f16.
__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
// ---- CTA pairs (cta_group::2): one MMA spans the tensor cores of both CTAs of a
// 2-CTA cluster.  Each CTA holds half of A (its 128 rows) and half of B (BN/2 rows) at
// the same shared-memory offsets; the even CTA issues the MMA, and D's 256 rows land 128
// per CTA at the same TMEM address.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at this offset in every CTA of `cta_mask` once this thread's
// earlier tcgen05 operations have completed (a commit, not a data load).
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on an mbarrier that
// may be the peer CTA's (cluster address); a single destination, no multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.cta_group::2 [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bits, 16 consecutive columns: thread i of the warp receives
// TMEM[lane_base + i][col .. col+15].
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Instruction descriptor for kind::f16 with fp32 accumulation, both operands K-major.
//   bits [4,6) D format (1 = f32), [7,10) A format, [10,13) B format (0 = f16, 1 = bf16),
//   bit 15/16 A/B major (0 = K), [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t make_idesc_f16(int m, int n, bool bf16) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// Instruction descriptor for kind::f8f6f4 with e4m3 A and B (format code 0 in bits [7,10) and
// [10,13)), both K-major, fp32 accumulation; other fields as make_idesc_f16.
__host__ __device__ constexpr uint32_t make_idesc_f8(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major operand stored in the canonical
// 128-byte-swizzled layout: rows of 128 bytes (64 x 16-bit elements), 8-row atoms of
// 1024 bytes stacked contiguously (stride byte offset 1024), atom base 1024-aligned.
//   bits [0,14) start >> 4, [16,30) leading byte offset >> 4 (unused for swizzled
//   K-major, set to 1), [32,46) stride byte offset >> 4, [46,48) version = 1,
//   [61,64) layout = 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a 128B-swizzled,
// K-major tile whose rows are 128 bytes (the pattern TMA SWIZZLE_128B writes).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// ------------------------------------------------------------------ numerics
template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
  static __device__ __forceinline__ uint16_t from_f(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
  // Two values rounded to nearest-even and packed (low half = a): one cvt instruction.
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
};
template <>
struct Elem<__half> {
  static __device__ __forceinline__ float to_f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
  static __device__ __forceinline__ uint16_t from_f(float f) { return __half_as_ushort(__float2half_rn(f)); }
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
};

// Gain element k as fp32 (the gain may be fp32, fp16 or bf16, kernel.py:203).
__device__ __forceinline__ float load_gain(const void* g, int gdt, int64_t k) {
  if (gdt == FQKV_F32) return reinterpret_cast<const float*>(g)[k];
  const uint16_t b = reinterpret_cast<const uint16_t*>(g)[k];
  return gdt == FQKV_BF16 ? Elem<__nv_bfloat16>::to_f(b) : Elem<__half>::to_f(b);
}

// rstd = 1 / sqrt(sum_sq / H + eps): the mean square is the row sum divided by H
// (baseline.py:59-61, kernel.py:181); IEEE division and square root.
__device__ __forceinline__ float row_rstd(float sum_sq, int64_t H, float eps) {
  const float mean = __fdiv_rn(sum_sq, (float)H);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

}  // namespace fqkv
