// Self-test of the bounded waits that keep the tensor-core kernels from
// hanging a GPU: a kernel whose every thread waits on an mbarrier phase that
// nothing completes, with a short limit chosen by the host. The wait must give
// up, record TAU_DXB_DEVERR_SELFTEST in the device error word, raise the CTA's
// abort flag (so that the other waiters leave too), and the CTA must free the
// tensor memory it holds and return -- the same teardown the attention kernels
// run when one of their waits runs out. No fault and no trap is involved: the
// wait is on a flag that nothing sets.

#include "attn.h"
#include "tc_common.cuh"

namespace taudxb {
namespace {

constexpr int kSelftestThreads = 128;

__device__ int g_selftest_status;   // bit 0: a wait completed, bit 1: abort flag raised

__global__ void __launch_bounds__(kSelftestThreads, 1)
wait_selftest_kernel(uint64_t limit_ns, int* err, int* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);      // one arrival completes phase 0; none comes
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) { tc::tmem_alloc(&tmem_base, 32); tc::tmem_relinquish(); }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const bool completed = tc::mbar_wait(&bar, 0, &abort_flag, err, TAU_DXB_DEVERR_SELFTEST, limit_ns);
  if (completed) atomicOr(status, 1);          // a phase nothing completes cannot complete
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem_base, 32);
  }
  if (threadIdx.x == 0) atomicOr(status, abort_flag ? 2 : 0);
}

}  // namespace

int wait_selftest(uint64_t limit_ns, int32_t* status_out, cudaStream_t st) {
  int* err = device_error_word();
  if (!err) return fail(TAU_DXB_ERR_CUDA, "cannot resolve the device error word");
  int* status = nullptr;
  TDX_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&status), g_selftest_status));
  TDX_CUDA(cudaMemsetAsync(status, 0, sizeof(int), st));
  wait_selftest_kernel<<<1, kSelftestThreads, 0, st>>>(limit_ns, err, status);
  const int rc = check_launch("wait_selftest_kernel");
  if (rc) return rc;
  int host = 0;
  TDX_CUDA(cudaMemcpyAsync(&host, status, sizeof(int), cudaMemcpyDeviceToHost, st));
  TDX_CUDA(cudaStreamSynchronize(st));
  *status_out = host;
  return TAU_DXB_OK;
}

}  // namespace taudxb
