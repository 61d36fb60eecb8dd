// Fixed-tau attention weights from materialised scores: the forward and the
// score gradient of STauOpusMaxStableFn (echo/patch_whisper_stau.py:74-112),
// the operator of the fixed-tau patch (apply_fixed_stau). One warp per score
// row, three passes over the row (it stays in L1 between them), fp32 with
// CUDA's accurate math functions throughout.
//
// Per row, with x = s - max(s) and every sigma clamped at 1e-8:
//   forward : q = max(sigma(x), 1e-8)^tau (no clamp on q), S = max(sum q, 1e-8),
//             attn = q / S
//   backward: A = tau max(sigma, 1e-8)^(tau - 1) sigma'(x)  (sigma' unclamped),
//             ds = A (g / S - sum(g q) / S^2); the row's first argmax also
//             gets - (sum(g A) / S - sum(g q) sum(A) / S^2)
// HBM-bound: the row is read once per call from DRAM, written once.

#include <cmath>

#include "common.cuh"

namespace taudxb {
namespace {

constexpr int kFixWarps = 8;

__device__ __forceinline__ float fixed_sigma(int sid, float x) {
  float v;
  switch (sid) {
    case TAU_DXB_SIGMA_SOFTPLUS: v = x > 20.f ? x : log1pf(expf(x)); break;
    case TAU_DXB_SIGMA_SIGMOID: v = 1.f / (1.f + expf(-x)); break;
    case TAU_DXB_SIGMA_EXP: v = expf(fminf(x, 20.f)); break;
    case TAU_DXB_SIGMA_RELU: v = fmaxf(x, 0.f); break;
    default: v = tanhf(x) + 1.f; break;   // tanh_shift
  }
  return fmaxf(v, kClampMin);
}

__device__ __forceinline__ float fixed_sigma_prime(int sid, float x) {
  switch (sid) {
    case TAU_DXB_SIGMA_SOFTPLUS: return 1.f / (1.f + expf(-x));
    case TAU_DXB_SIGMA_SIGMOID: { const float s = 1.f / (1.f + expf(-x)); return s * (1.f - s); }
    case TAU_DXB_SIGMA_EXP: return expf(fminf(x, 15.f));
    case TAU_DXB_SIGMA_RELU: return x > 0.f ? 1.f : 0.f;
    default: { const float t = tanhf(x); return 1.f - t * t; }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// row max and its first index (NaN rows give NaN, as torch.max does)
__device__ __forceinline__ void row_max_first(const float* s, int64_t L, int lane, float& m, int64_t& idx) {
  m = -INFINITY;
  idx = INT64_MAX;
  bool nan = false;
  for (int64_t c = lane; c < L; c += 32) {
    const float v = s[c];
    if (v != v) nan = true;
    if (v > m) { m = v; idx = c; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (om > m || (om == m && oi < idx)) { m = om; idx = oi; }
  }
  if (__any_sync(0xffffffffu, nan)) m = NAN;
  if (idx == INT64_MAX) idx = 0;
}

__global__ void __launch_bounds__(kFixWarps * 32)
fixed_fwd_kernel(const float* __restrict__ scores, int64_t rows, int64_t L, int64_t stride,
                 const float* __restrict__ tau, int64_t n_tau, int64_t rows_per_tau, int sid,
                 float* __restrict__ attn) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kFixWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* s = scores + row * stride;
  float* out = attn + row * L;
  const float t = tau[(row / rows_per_tau) % n_tau];
  float m;
  int64_t amax;
  row_max_first(s, L, lane, m, amax);
  float acc = 0.f;
  for (int64_t c = lane; c < L; c += 32) {
    const float q = powf(fixed_sigma(sid, s[c] - m), t);
    out[c] = q;
    acc += q;
  }
  const float S = fmaxf(warp_sum(acc), kClampMin);
  __syncwarp();
  for (int64_t c = lane; c < L; c += 32) out[c] = __fdiv_rn(out[c], S);
}

__global__ void __launch_bounds__(kFixWarps * 32)
fixed_bwd_kernel(const float* __restrict__ scores, const float* __restrict__ g, int64_t rows, int64_t L,
                 int64_t stride, const float* __restrict__ tau, int64_t n_tau, int64_t rows_per_tau, int sid,
                 float* __restrict__ ds) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kFixWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* s = scores + row * stride;
  const float* gr = g + row * L;
  float* out = ds + row * L;
  const float t = tau[(row / rows_per_tau) % n_tau];
  float m;
  int64_t amax;
  row_max_first(s, L, lane, m, amax);
  float sq = 0.f, wda = 0.f, da = 0.f, sa = 0.f;
  for (int64_t c = lane; c < L; c += 32) {
    const float x = s[c] - m;
    const float sg = fixed_sigma(sid, x);
    const float q = powf(sg, t);
    const float A = t * powf(sg, t - 1.f) * fixed_sigma_prime(sid, x);
    const float gv = gr[c];
    sq += q;
    wda += gv * q;
    da += gv * A;
    sa += A;
  }
  const float S = fmaxf(warp_sum(sq), kClampMin);
  wda = warp_sum(wda);
  da = warp_sum(da);
  sa = warp_sum(sa);
  const float S2 = S * S;
  const float wS2 = __fdiv_rn(wda, S2);
  const float t2 = __fdiv_rn(da, S) - __fdiv_rn(wda * sa, S2);
  for (int64_t c = lane; c < L; c += 32) {
    const float x = s[c] - m;
    const float sg = fixed_sigma(sid, x);
    const float A = t * powf(sg, t - 1.f) * fixed_sigma_prime(sid, x);
    float v = A * (__fdiv_rn(gr[c], S) - wS2);
    if (c == amax) v -= t2;
    out[c] = v;
  }
}

int fixed_grid(int64_t rows) { return static_cast<int>((rows + kFixWarps - 1) / kFixWarps); }

}  // namespace

int fixed_fwd_impl(const float* scores, int64_t rows, int64_t L, int64_t stride, const float* tau, int64_t n_tau,
                   int64_t rows_per_tau, int32_t sid, float* attn, cudaStream_t st) {
  TDX_CHECK_ARG(rows >= 0 && L >= 0 && stride >= L, "tau_opus_fixed_fwd: bad shape");
  TDX_CHECK_ARG(sid >= TAU_DXB_SIGMA_SOFTPLUS && sid <= TAU_DXB_SIGMA_TANH_SHIFT, "tau_opus_fixed_fwd: bad sigma id %d", sid);
  TDX_CHECK_ARG(n_tau >= 1 && rows_per_tau >= 1, "tau_opus_fixed_fwd: n_tau and rows_per_tau must be >= 1");
  if (rows == 0 || L == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(scores && tau && attn, "tau_opus_fixed_fwd: null pointer");
  TDX_CHECK_ARG(rows / kFixWarps < (1ll << 31), "tau_opus_fixed_fwd: too many rows");
  fixed_fwd_kernel<<<fixed_grid(rows), kFixWarps * 32, 0, st>>>(scores, rows, L, stride, tau, n_tau, rows_per_tau,
                                                                  sid, attn);
  return check_launch("fixed_fwd_kernel");
}

int fixed_bwd_impl(const float* scores, const float* g, int64_t rows, int64_t L, int64_t stride, const float* tau,
                   int64_t n_tau, int64_t rows_per_tau, int32_t sid, float* ds, cudaStream_t st) {
  TDX_CHECK_ARG(rows >= 0 && L >= 0 && stride >= L, "tau_opus_fixed_bwd: bad shape");
  TDX_CHECK_ARG(sid >= TAU_DXB_SIGMA_SOFTPLUS && sid <= TAU_DXB_SIGMA_TANH_SHIFT, "tau_opus_fixed_bwd: bad sigma id %d", sid);
  TDX_CHECK_ARG(n_tau >= 1 && rows_per_tau >= 1, "tau_opus_fixed_bwd: n_tau and rows_per_tau must be >= 1");
  if (rows == 0 || L == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(scores && g && tau && ds, "tau_opus_fixed_bwd: null pointer");
  TDX_CHECK_ARG(rows / kFixWarps < (1ll << 31), "tau_opus_fixed_bwd: too many rows");
  fixed_bwd_kernel<<<fixed_grid(rows), kFixWarps * 32, 0, st>>>(scores, g, rows, L, stride, tau, n_tau, rows_per_tau,
                                                                  sid, ds);
  return check_launch("fixed_bwd_kernel");
}

}  // namespace taudxb
