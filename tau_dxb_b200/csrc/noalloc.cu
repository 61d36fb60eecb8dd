// tau_attn_bwd_noalloc: the attention backward with its scratch memory in a
// fixed, library-owned device array instead of a caller-provided workspace.
//
// Who needs it: hosts that own every byte of device memory through their own
// pool or run under a fixed memory budget, and C/FFI callers with no device
// allocator of their own. Such callers cannot let a library call cudaMalloc
// behind their back -- it bypasses their accounting and can synchronise the
// whole device -- and may have no way to hand over a workspace either. This
// entry point calls no cudaMalloc, cudaFree or allocating library routine.
//
// Cost and limits:
//   * every GPU that loads the library holds kNoAllocScratchBytes (16 MiB) of
//     scratch in the static array below until the process exits;
//   * problems whose backward workspace (tau_attn_bwd_workspace_bytes) exceeds
//     16 MiB are rejected with TAU_DXB_ERR_WORKSPACE;
//   * all calls on one device share the array, which keeps the last call's
//     contents: the regions that must start at zero are cleared on the stream
//     by each call, and calls whose GPU work overlaps (two streams, or two
//     host threads) race on the array -- serialise them;
//   * each call resolves the array's device address on the current device
//     (cudaGetSymbolAddress; the first call on a device also loads the
//     library's device code there, so make it before any stream capture);
//   * the results are valid only if tau_dxb_device_error() reads 0 after the
//     call's work is done: a tensor-core wait that gave up skips its stores,
//     and the epilogue would then read what the array held from an earlier call.

#include "attn.h"

namespace taudxb {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;   // 16 MiB

// In host code the name below is only a host-side stand-in for the symbol;
// kernels get the device address resolved by scratch_address().
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch array on the current device. Resolved on
// every call: a cached address would go stale if the caller reset the device
// (cudaDeviceReset) and the module were loaded again elsewhere.
int scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || !p)
    return fail(TAU_DXB_ERR_CUDA, "tau_attn_bwd_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
  *out = p;
  return TAU_DXB_OK;
}

}  // namespace
}  // namespace taudxb

using namespace taudxb;

extern "C" int tau_attn_bwd_noalloc(
    const void* q, const int64_t q_stride[4], const void* k, const int64_t k_stride[4],
    const void* v, const int64_t v_stride[4], const void* out, const int64_t out_stride[4],
    const void* dout, const int64_t dout_stride[4], int32_t dtype, int64_t B, int64_t H, int64_t Lq,
    int64_t Lk, int64_t D, const float* tau, const float* alpha, int32_t sigma_id, float scale,
    const void* mask, int32_t mask_dtype, const int64_t mask_stride[4], int32_t causal,
    const float* row_max, const float* row_z, const int32_t* row_argmax, void* dq,
    const int64_t dq_stride[4], void* dk, const int64_t dk_stride[4], void* dv,
    const int64_t dv_stride[4], float* dtau, float* dalpha, int32_t path, void* stream) {
  // tau_attn_bwd_workspace_bytes saturates instead of wrapping, so shapes too
  // large for any workspace land here as well
  const size_t need = tau_attn_bwd_workspace_bytes(B, H, Lq, Lk, D);
  if (need > kNoAllocScratchBytes)
    return fail(TAU_DXB_ERR_WORKSPACE,
                "tau_attn_bwd_noalloc: this problem needs %zu bytes of scratch; the fixed array "
                "holds %zu (16 MiB) -- use tau_attn_bwd with a caller workspace",
                need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc) return rc;
  return tau_attn_bwd(q, q_stride, k, k_stride, v, v_stride, out, out_stride, dout, dout_stride,
                      dtype, B, H, Lq, Lk, D, tau, alpha, sigma_id, scale, mask, mask_dtype,
                      mask_stride, causal, row_max, row_z, row_argmax, dq, dq_stride, dk,
                      dk_stride, dv, dv_stride, dtau, dalpha, scratch, kNoAllocScratchBytes, path,
                      stream);
}
