// Cross-entropy over bf16 logits, as autocast runs F.cross_entropy (fp32
// math over the bf16 logits, mean over the rows whose label is not ignored),
// without the fp32 copy of the logits: the train step's loss over
// [rows = batch x label tokens, vocab ~ 52k].
//
//   forward : one CTA per row; each thread keeps a running max and a sum of
//             exp(x - max) over its 8-element chunks (16-byte loads), the CTA
//             combines them; lse = max + log(sum), loss_row = lse - x[label]
//             (0 for an ignored row), lse saved for the backward.
//   backward: dx = (exp(x - lse) - [j == label]) * g[0], written in bf16, with
//             g on the device (dloss / number of counted rows): no host read.

#include "common.cuh"

namespace taudxb {
namespace {

constexpr int kXeThreads = 256;

__device__ __forceinline__ void xe_load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// (m, s) pairs: s = sum exp(x - m)
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;   // both empty (all -inf so far)
  s = s * expf(m - mm) + s2 * expf(m2 - mm);
  m = mm;
}

__global__ void __launch_bounds__(kXeThreads)
xent_fwd_kernel(const __nv_bfloat16* __restrict__ x, const int64_t* __restrict__ labels, int64_t V,
                int64_t ignore_index, float* __restrict__ loss_row, float* __restrict__ lse_out) {
  __shared__ float sm_m[kXeThreads / 32], sm_s[kXeThreads / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * V;
  float m = -INFINITY, s = 0.f;
  for (int64_t j = static_cast<int64_t>(threadIdx.x) * 8; j < V; j += kXeThreads * 8) {
    float v[8];
    xe_load8(xr + j, v);
    float cm = v[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) cm = fmaxf(cm, v[i]);
    if (cm == -INFINITY) continue;
    float cs = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) cs += expf(v[i] - cm);
    lse_merge(m, s, cm, cs);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, m2, s2);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm_m[warp] = m;
    sm_s[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = sm_m[0], S = sm_s[0];
    for (int w = 1; w < kXeThreads / 32; ++w) lse_merge(M, S, sm_m[w], sm_s[w]);
    const float lse = M + logf(S);
    lse_out[row] = lse;
    const int64_t lab = labels[row];
    float l = 0.f;
    if (lab != ignore_index) {
      // labels outside [0, V) other than ignore_index give NaN (the host
      // checks them before the call)
      l = (lab >= 0 && lab < V) ? lse - __bfloat162float(xr[lab]) : __int_as_float(0x7fc00000);
    }
    loss_row[row] = l;
  }
}

__global__ void __launch_bounds__(kXeThreads)
xent_bwd_kernel(const __nv_bfloat16* __restrict__ x, const int64_t* __restrict__ labels, int64_t V,
                int64_t ignore_index, const float* __restrict__ lse_in, const float* __restrict__ g,
                __nv_bfloat16* __restrict__ dx) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * V;
  __nv_bfloat16* dr = dx + row * V;
  const int64_t lab = labels[row];
  const bool counted = lab != ignore_index;
  const float lse = lse_in[row], scale = counted ? __ldg(g) : 0.f;
  for (int64_t j = static_cast<int64_t>(threadIdx.x) * 8; j < V; j += kXeThreads * 8) {
    float v[8];
    xe_load8(xr + j, v);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = expf(v[2 * i] - lse), b = expf(v[2 * i + 1] - lse);
      if (j + 2 * i == lab) a -= 1.f;
      if (j + 2 * i + 1 == lab) b -= 1.f;
      const __nv_bfloat162 h = __floats2bfloat162_rn(a * scale, b * scale);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(dr + j) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace

int cross_entropy_fwd_impl(const void* logits, int64_t M, int64_t V, const int64_t* labels, int64_t ignore_index,
                           float* loss_row, float* lse, cudaStream_t st) {
  TDX_CHECK_ARG(M >= 0 && V > 0 && V % 8 == 0, "cross entropy: need V a multiple of 8 (got %lld)", (long long)V);
  if (M == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(logits && labels && loss_row && lse, "cross entropy: null pointer");
  TDX_CHECK_ARG((reinterpret_cast<uintptr_t>(logits) & 15) == 0, "cross entropy: logits must be 16-byte aligned");
  TDX_CHECK_ARG(M < (1ll << 31), "cross entropy: too many rows");
  xent_fwd_kernel<<<static_cast<unsigned>(M), kXeThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(logits), labels,
                                                                    V, ignore_index, loss_row, lse);
  return check_launch("xent_fwd_kernel");
}

int cross_entropy_bwd_impl(const void* logits, int64_t M, int64_t V, const int64_t* labels, int64_t ignore_index,
                           const float* lse, const float* grad_scale, void* dlogits, cudaStream_t st) {
  TDX_CHECK_ARG(M >= 0 && V > 0 && V % 8 == 0, "cross entropy: need V a multiple of 8 (got %lld)", (long long)V);
  if (M == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(logits && labels && lse && grad_scale && dlogits, "cross entropy: null pointer");
  TDX_CHECK_ARG((reinterpret_cast<uintptr_t>(logits) & 15) == 0 && (reinterpret_cast<uintptr_t>(dlogits) & 15) == 0,
                "cross entropy: logits and dlogits must be 16-byte aligned");
  TDX_CHECK_ARG(M < (1ll << 31), "cross entropy: too many rows");
  xent_bwd_kernel<<<static_cast<unsigned>(M), kXeThreads, 0, st>>>(
      static_cast<const __nv_bfloat16*>(logits), labels, V, ignore_index, lse, grad_scale,
      static_cast<__nv_bfloat16*>(dlogits));
  return check_launch("xent_bwd_kernel");
}

}  // namespace taudxb
