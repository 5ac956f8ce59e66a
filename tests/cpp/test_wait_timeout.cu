// Self-test of the bounded mbarrier wait used by the bulk-copy kernels
// (warp_wait_bounded in csrc/common.cuh).  Needs a GPU; exits non-zero on a
// failure.  Nothing here faults, traps or hangs: every wait has a deadline.
//   1. a barrier that completes (one arrival) -> the wait returns true;
//   2. a barrier whose bulk copy delivers all expected bytes -> true, data intact;
//   3. a barrier that nothing completes -> false after the deadline (50 ms);
//   4. a barrier expecting transaction bytes that no copy delivers (a wrong
//      byte count, the defect the deadline guards against) -> false after the
//      deadline; no copy was issued, so nothing is left in flight;
//   5. the context still works afterwards, and the timeout counter reads 2.
#include <chrono>
#include <cstdio>
#include <cstring>

#include "common.cuh"

using namespace hrm;

namespace {

constexpr unsigned long long kLimitNs = 50ull * 1000 * 1000;

__global__ void wait_kernel(int mode, const uint4* src, uint4* dst, int* result) {
  __shared__ uint64_t bar;
  __shared__ __align__(16) uint4 buf[64];
  const uint32_t b = smem_addr(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    mbar_init_fence();
    if (mode == 1) {
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(b) : "memory");
    } else if (mode == 2) {
      mbar_arrive_expect_tx(b, 1024u);
      bulk_g2s(smem_addr(buf), src, 1024u, b);
    } else if (mode == 4) {
      mbar_arrive_expect_tx(b, 1024u);
    }
  }
  __syncwarp();
  const bool ok = warp_wait_bounded(b, 0, kLimitNs);
  if (!ok && threadIdx.x == 0) atomicAdd(&g_wait_timeouts, 1u);
  if (ok && mode == 2) {
    dst[threadIdx.x] = buf[threadIdx.x];
    dst[threadIdx.x + 32] = buf[threadIdx.x + 32];
  }
  if (threadIdx.x == 0) *result = ok ? 1 : 0;
}

bool run(int mode, const uint4* src, uint4* dst, int* d_result, int expect, double* ms) {
  const auto t0 = std::chrono::steady_clock::now();
  wait_kernel<<<1, 32>>>(mode, src, dst, d_result);
  cudaError_t e = cudaDeviceSynchronize();
  *ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  int r = -1;
  if (e == cudaSuccess) e = cudaMemcpy(&r, d_result, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    std::printf("FAIL mode %d: %s\n", mode, cudaGetErrorString(e));
    return false;
  }
  if (r != expect) {
    std::printf("FAIL mode %d: wait returned %d, expected %d\n", mode, r, expect);
    return false;
  }
  std::printf("ok   mode %d: wait returned %d after %.1f ms\n", mode, r, *ms);
  return true;
}

}  // namespace

int main() {
  uint4 *src = nullptr, *dst = nullptr;
  int* d_result = nullptr;
  if (cudaMalloc(&src, 1024) != cudaSuccess || cudaMalloc(&dst, 1024) != cudaSuccess ||
      cudaMalloc(&d_result, sizeof(int)) != cudaSuccess) {
    std::printf("FAIL cudaMalloc\n");
    return 1;
  }
  unsigned char host[1024], back[1024];
  for (int i = 0; i < 1024; ++i) host[i] = (unsigned char)(i * 37 + 11);
  cudaMemcpy(src, host, 1024, cudaMemcpyHostToDevice);
  double ms = 0;
  if (!run(1, src, dst, d_result, 1, &ms)) return 1;
  if (!run(2, src, dst, d_result, 1, &ms)) return 1;
  cudaMemcpy(back, dst, 1024, cudaMemcpyDeviceToHost);
  if (std::memcmp(host, back, 1024) != 0) {
    std::printf("FAIL mode 2: bulk-copied data differs\n");
    return 1;
  }
  if (!run(3, src, dst, d_result, 0, &ms)) return 1;
  if (ms < 45.0 || ms > 5000.0) {
    std::printf("FAIL mode 3: returned after %.1f ms, deadline 50 ms\n", ms);
    return 1;
  }
  if (!run(4, src, dst, d_result, 0, &ms)) return 1;
  unsigned int timeouts = 0;
  if (cudaMemcpyFromSymbol(&timeouts, g_wait_timeouts, sizeof(timeouts)) != cudaSuccess || timeouts != 2) {
    std::printf("FAIL timeout counter reads %u, expected 2\n", timeouts);
    return 1;
  }
  // the context is still usable
  if (cudaMemset(dst, 0, 1024) != cudaSuccess || !run(1, src, dst, d_result, 1, &ms)) return 1;
  cudaFree(src);
  cudaFree(dst);
  cudaFree(d_result);
  std::printf("all wait tests passed\n");
  return 0;
}
