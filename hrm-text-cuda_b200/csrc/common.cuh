// Shared device helpers for the sm_100a layer-op kernels.
//
// bf16 values travel as raw 16-bit patterns packed two per 32-bit word; a
// 16-byte vector (uint4) carries 8 of them.  Conversions:
//   bf16 -> f32 : exact, the pattern shifted into the high half of a binary32;
//   f32  -> bf16: round-to-nearest-even via the cvt.rn.bf16x2.f32 instruction
//                 (__float22bfloat162_rn), the rounding used by
//                 __float2bfloat16 / __float22bfloat162_rn in the reference
//                 kernels (e.g. src/kernels/additive_inject.cu:31).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hrm {

// ---------------------------------------------------------------- bf16 <-> f32
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float bf16_to_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

// Packs (lo, hi) into one word, each rounded to nearest even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __float22bfloat162_rn(make_float2(lo, hi));
  return *reinterpret_cast<uint32_t*>(&p);
}
__device__ __forceinline__ uint16_t f32_to_bf16(float x) {
  __nv_bfloat16 b = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&b);
}

__device__ __forceinline__ uint32_t vget(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
__device__ __forceinline__ void vset(uint4& v, int i, uint32_t w) {
  if (i == 0) v.x = w; else if (i == 1) v.y = w; else if (i == 2) v.z = w; else v.w = w;
}

// ------------------------------------------------------------- memory access
// Streaming (read-once / write-once) accesses: evict-first in L1 and L2 so
// that reused data (weights, rope tables, embedding rows) keeps its L2 lines.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(uint4* p, const uint4& v) { __stcs(p, v); }
// Streamed data with the default L2 priority (ld.global.cg / st.global.cg:
// L2 only, normal eviction).  Measured on B200 against the evict-first forms
// above, same bits: RMSNorm bf16 [4096 x 2048] 6.40 -> 5.80 us (loads and
// stores), add + RMSNorm [16384 x 2048] 6.50 -> 6.71 TB/s (loads and stores),
// RMSNorm fp32 [4096 x 2048] 5.84 -> 5.98 TB/s (loads and stores), SwiGLU
// 6.90 -> 7.00 and the attention gate 6.84 -> 6.95 TB/s (loads); RoPE
// unchanged.  Evict-first stores stay where an output must not displace
// reused lines: the embedding gather (its table rows repeat) measured 3.7%
// slower with default-priority stores.
__device__ __forceinline__ uint4 ld_l2(const uint4* p) { return __ldcg(p); }
__device__ __forceinline__ void st_l2(uint4* p, const uint4& v) { __stcg(p, v); }
__device__ __forceinline__ float4 ld_l2(const float4* p) { return __ldcg(p); }
__device__ __forceinline__ void st_l2(float4* p, const float4& v) { __stcg(p, v); }
// Reused read-only data (weights, tables): normal caching.
__device__ __forceinline__ uint4 ld_keep(const uint4* p) { return __ldg(p); }
__device__ __forceinline__ float4 ld_keep(const float4* p) { return __ldg(p); }
// Reused read-only data marked evict-last in L2 (an L2 access policy made by
// createpolicy), so that streaming traffic is evicted before it.
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint4 ld_keep_last(const uint4* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

// ------------------------------------------- programmatic dependent launch
// Every kernel calls this before its first global-memory access.  The wait
// (griddepcontrol.wait) returns once the grid this launch depends on has
// completed and its writes are visible; for a launch that was not
// programmatic it returns at once.  The trigger (griddepcontrol.launch_
// dependents) then lets the next programmatic launch in the stream be
// scheduled while this grid still runs: its CTAs start once every CTA here has
// passed this point and park in their own wait, so the launch latency of the
// next kernel overlaps this one's execution instead of following it.
__device__ __forceinline__ void grid_dependency_begin() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// L2 prefetch of `bytes` (a multiple of 16) at the 16-byte aligned address p,
// by the bulk-copy engine.  A kernel may issue it BEFORE grid_dependency_begin
// for inputs the previous grid may still be writing: L2 is the point of
// coherence for global memory, so the prefetch can only warm lines -- the
// loads issued after the wait still see the previous grid's writes -- while
// the DRAM reads start during the previous grid's drain instead of after it.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

// ---------------------------------------------------------- async staging
// cp.async (LDGSTS) of one 16-byte chunk global -> shared, L2-cached only.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// ------------------------------------------- bulk copies (TMA engine), mbarriers
// One-dimensional bulk copies global -> shared (cp.async.bulk, no tensor map,
// no multicast) completing on an mbarrier's transaction count.  Source and
// destination 16-byte aligned, size a multiple of 16 bytes.
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
// Makes initialised mbarriers visible to the bulk-copy (async) proxy.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
// One arrival plus `bytes` of expected transactions for the current phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Orders this thread's earlier generic-proxy shared-memory accesses before its
// later bulk copies into the same shared memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s_hint(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;\n" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

// Deadline of every mbarrier wait (nanoseconds of %globaltimer).  A wait that
// runs out counts itself in g_wait_timeouts and returns false; a bulk copy of
// valid, host-checked addresses completes in microseconds, so a timeout means
// a defect, reported instead of hung on.
#ifndef HRM_WAIT_LIMIT_NS
#define HRM_WAIT_LIMIT_NS 1000000000ull
#endif
// Per translation unit; the host reads it with cudaMemcpyFromSymbol.
static __device__ unsigned int g_wait_timeouts;

// Whole-warp bounded wait for phase `parity` of the mbarrier at `bar`: true
// once every lane has observed the completed phase, false (in every lane)
// when the deadline passes first.
__device__ __forceinline__ bool warp_wait_bounded(uint32_t bar, uint32_t parity,
                                                  uint64_t limit_ns = HRM_WAIT_LIMIT_NS) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
    if (__any_sync(0xffffffffu, globaltimer_ns() - t0 > limit_ns)) return false;
  }
}

}  // namespace hrm
