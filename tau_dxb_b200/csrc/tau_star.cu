// tau* solver on the GPU: the batched Newton iteration of
// tau_star/tau_star_solver.py:60-128,
//
//   tau* = argmin_tau KL(softmax(s) || softmax(tau * log sigma(s)))   per score row s,
//
// fused into one kernel. The reference runs each Newton step as ~8 full tensor
// passes over the [rows, T] scores (n_iter = 100 in
// tau_star/compute_tau_star_echo.py:127, on host copies of the scores); here one
// warp owns a row, reads it once, and runs every step on chip:
//
//   * rows of T <= 2048 keys: log sigma(s) and the step's weights live in
//     registers (NPL = ceil(T / 32) per lane, element j on lane j % 32);
//   * longer rows: log sigma(s) and softmax(s) in shared memory.
//
// Per step: logits x_j = tau log sigma_j rounded to fp32 as the reference forms
// them (no fused multiply-add, so that exp(x_j - m) rounds alike);
// m = max_j x_j, taken as tau * max (or min, for tau < 0) of log sigma, which
// rounds exactly like the max of the rounded products; w_j = exp(x_j - m); E_p = sum w ls / sum w; Var_p =
// sum w (ls - E_p)^2 / sum w (the reference's two-pass form); tau <- clamp(tau
// - (E_p - e_ref) / (Var_p + eps)). fp32 with CUDA's accurate expf / logf /
// log1pf. A NaN tau stays NaN through the clamp, as torch.clamp keeps it, and
// is replaced by tau_init at the end (non-finite KL by 0), as the reference
// sanitises.

#include "tc_common.cuh"

namespace taudxb {
namespace {

constexpr int kTsRegWarps = 4;   // rows per CTA, register kernel
constexpr int kTsRegMaxNpl = 64; // register kernel up to 2048 keys
constexpr uint32_t kAll = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kAll, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kAll, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(kAll, v, o));
  return v;
}

// torch.clamp / F.relu keep a NaN (fmaxf / fminf would drop it). The KL of a
// row whose padded keys have ref = p = 0 is NaN through 0 / 0, and the
// reference then reports 0 for it.
__device__ __forceinline__ float max_keep_nan(float x, float lo) { return x != x ? x : fmaxf(x, lo); }
__device__ __forceinline__ float min_keep_nan(float x, float hi) { return x != x ? x : fminf(x, hi); }
__device__ __forceinline__ float clamp_keep_nan(float x, float lo, float hi) {
  return x != x ? x : fminf(fmaxf(x, lo), hi);
}

// log sigma(s) of tau_star/tau_star_solver.py:25-43 (F.softplus thresholds at 20)
__device__ __forceinline__ float ts_log_sigma(int sid, float s) {
  switch (sid) {
    case TAU_DXB_SIGMA_SOFTPLUS: return logf(max_keep_nan(s > 20.f ? s : log1pf(expf(s)), 1e-30f));
    case TAU_DXB_SIGMA_SIGMOID: return -(-s > 20.f ? -s : log1pf(expf(-s)));
    case TAU_DXB_SIGMA_EXP: return min_keep_nan(s, 20.f);
    default: return logf(max_keep_nan(max_keep_nan(s, 0.f), 1e-30f));
  }
}

__device__ __forceinline__ float newton_step(float tau, float e_p, float e_ref, float var, float eps, float lo,
                                             float hi) {
  return clamp_keep_nan(tau - (e_p - e_ref) / (var + eps), lo, hi);
}

__device__ __forceinline__ void write_result(float* tau_out, float* kl_out, int64_t row, float tau, float kl,
                                             float tau_init) {
  tau_out[row] = isfinite(tau) ? tau : tau_init;
  kl_out[row] = isfinite(kl) ? kl : 0.f;
}

// One warp per row, the row in registers as packed pairs: ls2[q].x is key
// lane + 64 q, ls2[q].y key lane + 64 q + 32. A size bucket NPL covers
// 32 NLO < T <= 32 NPL, so chunks below NLO are full for every lane and only
// the last NPL - NLO chunks test j < T; keys past T hold ls = 0, weight 0.
//
// Inside the Newton steps the weights are w_j = 2^(ls_j tau log2(e) - m') on
// the special-function unit (one ex2 per key, packed fp32x2 arithmetic around
// it, independent accumulation chains); they only enter sums. The
// reported KL is formed again with accurate expf and the reference's rounding
// of tau * ls, since whether p underflows to zero decides its NaN -> 0 rows.
// CTAs per SM to ask of the register allocator: the row (NPL registers) plus
// about 40 for the rest of the state
constexpr int ts_min_blocks(int npl) {
  return 65536 / (kTsRegWarps * 32 * (npl + 40)) > 16 ? 16 : 65536 / (kTsRegWarps * 32 * (npl + 40));
}

template <int NPL, int NLO>
__global__ void __launch_bounds__(kTsRegWarps * 32, ts_min_blocks(NPL))
tau_star_reg_kernel(const float* __restrict__ scores, int64_t n_rows, int T, int64_t row_stride, int sid,
                    int n_iter, float tau_init, float tau_min, float tau_max, float eps,
                    float* __restrict__ tau_out, float* __restrict__ kl_out) {
  static_assert(NPL % 2 == 0 && NLO % 2 == 0 && NLO < NPL, "even chunk counts");
  constexpr int NP = NPL / 2;
  constexpr float kLog2e = 1.4426950408889634f;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kTsRegWarps + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const float* s = scores + row * row_stride;
  const int cnt = T > lane ? (T - lane + 31) / 32 : 0;   // valid chunks of this lane
  auto valid = [&](int i) { return i < NLO || i < cnt; };
  float2 ls2[NP];
  float smax = -INFINITY, lsmax = -INFINITY, lsmin = INFINITY;
#pragma unroll
  for (int q = 0; q < NP; ++q) {
    float l[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = 2 * q + h;
      l[h] = 0.f;
      if (valid(i)) {
        const float v = __ldg(s + lane + 32 * i);
        l[h] = ts_log_sigma(sid, v);
        smax = fmaxf(smax, v);
        lsmax = fmaxf(lsmax, l[h]);
        lsmin = fminf(lsmin, l[h]);
      }
    }
    ls2[q] = make_float2(l[0], l[1]);
  }
  smax = warp_max(smax);
  lsmax = warp_max(lsmax);
  lsmin = warp_min(lsmin);
  // reference distribution softmax(s) (accurate expf, the row read again from
  // L1) and e_ref = E_ref[log sigma] = sum e ls / sum e
  float z = 0.f, ez = 0.f;
#pragma unroll
  for (int q = 0; q < NP; ++q) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = 2 * q + h;
      if (valid(i)) {
        const float e = expf(__ldg(s + lane + 32 * i) - smax);
        z += e;
        ez = fmaf(e, h ? ls2[q].y : ls2[q].x, ez);
      }
    }
  }
  z = warp_sum(z);
  const float e_ref = warp_sum(ez) / z;

  // Each step is one pass: with c = the previous step's E_p (e_ref at first),
  // d = ls - c, E_p = c + sum w d / sum w and Var_p = sum w d^2 / sum w
  // - (E_p - c)^2, the reference's two-pass variance rewritten about a centre
  // that tracks E_p, so that the subtraction loses almost nothing.
  float tau = tau_init, c = e_ref;
  for (int it = 0; it < n_iter; ++it) {
    const float tl = tau * kLog2e;
    const float m = tl * (tl >= 0.f ? lsmax : lsmin);
    const float2 tl2 = make_float2(tl, tl), nm2 = make_float2(-m, -m), nc2 = make_float2(-c, -c);
    float2 a[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    float2 b[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    float2 v[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      const float2 arg = tc::fma2(ls2[q], tl2, nm2);
      float2 w = make_float2(tc::ex2(arg.x), tc::ex2(arg.y));
      if (2 * q + 1 >= NLO) {
        w.x = valid(2 * q) ? w.x : 0.f;
        w.y = valid(2 * q + 1) ? w.y : 0.f;
      }
      const float2 d = tc::add2(ls2[q], nc2);
      const float2 wd = tc::mul2(w, d);
      a[q & 1] = tc::add2(a[q & 1], w);
      b[q & 1] = tc::add2(b[q & 1], wd);
      v[q & 1] = tc::fma2(wd, d, v[q & 1]);
    }
    float sa = (a[0].x + a[0].y) + (a[1].x + a[1].y);
    float sb = (b[0].x + b[0].y) + (b[1].x + b[1].y);
    float sv = (v[0].x + v[0].y) + (v[1].x + v[1].y);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sa += __shfl_xor_sync(kAll, sa, o);
      sb += __shfl_xor_sync(kAll, sb, o);
      sv += __shfl_xor_sync(kAll, sv, o);
    }
    const float mu = sb / sa;
    const float e_p = c + mu;
    const float var = fmaxf(sv / sa - mu * mu, 0.f);
    tau = newton_step(tau, e_p, e_ref, var, eps, tau_min, tau_max);
    c = e_p;
  }
  // KL(ref || p_tau) = sum ref log(max(ref / p, 1e-30)): log_norm, p and ref
  // (from the row) with accurate expf and x = tau * ls rounded as the reference
  const float m = __fmul_rn(tau, tau >= 0.f ? lsmax : lsmin);
  float s0 = 0.f;
#pragma unroll
  for (int q = 0; q < NP; ++q) {
    if (valid(2 * q)) s0 += expf(__fmul_rn(tau, ls2[q].x) - m);
    if (valid(2 * q + 1)) s0 += expf(__fmul_rn(tau, ls2[q].y) - m);
  }
  const float ln = m + logf(warp_sum(s0));
  float kl = 0.f;
#pragma unroll
  for (int q = 0; q < NP; ++q) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = 2 * q + h;
      if (valid(i)) {
        const float l = h ? ls2[q].y : ls2[q].x;
        const float r = expf(__ldg(s + lane + 32 * i) - smax) / z;
        const float p = expf(__fmul_rn(tau, l) - ln);
        kl = fmaf(r, logf(max_keep_nan(r / p, 1e-30f)), kl);
      }
    }
  }
  kl = warp_sum(kl);
  if (lane == 0) write_result(tau_out, kl_out, row, tau, kl, tau_init);
}

// One warp per row, log sigma(s) and softmax(s) in shared memory (2 T floats
// per warp); rows of any length up to TAU_DXB_TAU_STAR_MAX_KEYS.
__global__ void __launch_bounds__(128)
tau_star_smem_kernel(const float* __restrict__ scores, int64_t n_rows, int T, int64_t row_stride, int sid,
                     int n_iter, float tau_init, float tau_min, float tau_max, float eps,
                     float* __restrict__ tau_out, float* __restrict__ kl_out) {
  extern __shared__ float tsm[];
  const int warps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * warps + warp;
  if (row >= n_rows) return;
  float* ls = tsm + static_cast<size_t>(warp) * 2 * T;
  float* ref = ls + T;
  const float* s = scores + row * row_stride;
  float smax = -INFINITY, lsmax = -INFINITY, lsmin = INFINITY;
  for (int j = lane; j < T; j += 32) {
    const float v = __ldg(s + j);
    const float l = ts_log_sigma(sid, v);
    ref[j] = v;
    ls[j] = l;
    smax = fmaxf(smax, v);
    lsmax = fmaxf(lsmax, l);
    lsmin = fminf(lsmin, l);
  }
  smax = warp_max(smax);
  lsmax = warp_max(lsmax);
  lsmin = warp_min(lsmin);
  float z = 0.f;
  for (int j = lane; j < T; j += 32) {
    const float e = expf(ref[j] - smax);
    ref[j] = e;
    z += e;
  }
  z = warp_sum(z);
  float e_ref = 0.f;
  for (int j = lane; j < T; j += 32) {
    const float r = ref[j] / z;
    ref[j] = r;
    e_ref = fmaf(r, ls[j], e_ref);
  }
  e_ref = warp_sum(e_ref);

  float tau = tau_init;
  float m = 0.f, s0 = 1.f;
  auto weights = [&](float t) -> float {
    m = __fmul_rn(t, t >= 0.f ? lsmax : lsmin);
    float a = 0.f, b = 0.f;
    for (int j = lane; j < T; j += 32) {
      const float wj = expf(__fmul_rn(t, ls[j]) - m);
      a += wj;
      b = fmaf(wj, ls[j], b);
    }
    s0 = warp_sum(a);
    return warp_sum(b) / s0;
  };
  for (int it = 0; it < n_iter; ++it) {
    const float e_p = weights(tau);
    float v = 0.f;
    for (int j = lane; j < T; j += 32) {
      const float d = ls[j] - e_p;
      v = fmaf(expf(__fmul_rn(tau, ls[j]) - m), d * d, v);
    }
    const float var = warp_sum(v) / s0;
    tau = newton_step(tau, e_p, e_ref, var, eps, tau_min, tau_max);
  }
  weights(tau);
  const float ln = m + logf(s0);
  float kl = 0.f;
  for (int j = lane; j < T; j += 32) {
    const float p = expf(__fmul_rn(tau, ls[j]) - ln);
    kl = fmaf(ref[j], logf(max_keep_nan(ref[j] / p, 1e-30f)), kl);
  }
  kl = warp_sum(kl);
  if (lane == 0) write_result(tau_out, kl_out, row, tau, kl, tau_init);
}

// One-shot estimate of solve_tau_star_analytic (tau_star/tau_star_solver.py:
// 131-151): tau = clamp(cov_ref(s, ls) / (var_ref(ls) + 1e-6), 0.1, 10) under
// ref = softmax(s), one warp per row, three passes over the row (L1-resident
// after the first). The reference does not sanitise this one: a NaN stays.
__global__ void __launch_bounds__(128)
tau_star_analytic_kernel(const float* __restrict__ scores, int64_t n_rows, int T, int64_t row_stride, int sid,
                         float* __restrict__ tau_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 4 + (threadIdx.x >> 5);
  if (row >= n_rows) return;
  const float* s = scores + row * row_stride;
  float smax = -INFINITY;
  for (int j = lane; j < T; j += 32) smax = fmaxf(smax, __ldg(s + j));
  smax = warp_max(smax);
  float z = 0.f, zs = 0.f, zl = 0.f;
  for (int j = lane; j < T; j += 32) {
    const float v = __ldg(s + j);
    const float e = expf(v - smax);
    z += e;
    zs = fmaf(e, v, zs);
    zl = fmaf(e, ts_log_sigma(sid, v), zl);
  }
  z = warp_sum(z);
  const float mu_s = warp_sum(zs) / z, mu_l = warp_sum(zl) / z;
  float cv = 0.f, vr = 0.f;
  for (int j = lane; j < T; j += 32) {
    const float v = __ldg(s + j);
    const float e = expf(v - smax);
    const float dl = ts_log_sigma(sid, v) - mu_l;
    cv = fmaf(e * (v - mu_s), dl, cv);
    vr = fmaf(e * dl, dl, vr);
  }
  const float cov = warp_sum(cv) / z, var = warp_sum(vr) / z;
  if (lane == 0) tau_out[row] = clamp_keep_nan(cov / (var + 1e-6f), 0.1f, 10.f);
}

__global__ void tau_star_trivial_kernel(int64_t n_rows, float tau_init, float* tau_out, float* kl_out) {
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < n_rows;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    tau_out[r] = tau_init;
    kl_out[r] = 0.f;
  }
}

using RegKernel = void (*)(const float*, int64_t, int, int64_t, int, int, float, float, float, float, float*,
                           float*);

RegKernel reg_kernel_for(int npl) {
  // buckets of 32-key chunks: NPL with the previous bucket as NLO
  static const int kNpl[] = {2, 4, 8, 12, 16, 24, 32, 40, 48, 56, 64};
  static const RegKernel kFn[] = {
      tau_star_reg_kernel<2, 0>,   tau_star_reg_kernel<4, 2>,   tau_star_reg_kernel<8, 4>,
      tau_star_reg_kernel<12, 8>,  tau_star_reg_kernel<16, 12>, tau_star_reg_kernel<24, 16>,
      tau_star_reg_kernel<32, 24>, tau_star_reg_kernel<40, 32>, tau_star_reg_kernel<48, 40>,
      tau_star_reg_kernel<56, 48>, tau_star_reg_kernel<64, 56>};
  static_assert(kTsRegMaxNpl == 64, "last bucket");
  for (size_t i = 0; i < sizeof(kNpl) / sizeof(kNpl[0]); ++i)
    if (npl <= kNpl[i]) return kFn[i];
  return nullptr;
}

}  // namespace

int tau_star_solve_impl(const float* scores, int64_t n_rows, int64_t T, int64_t row_stride, int32_t sigma_id,
                        int32_t n_iter, float tau_init, float tau_min, float tau_max, float eps, float* tau_out,
                        float* kl_out, cudaStream_t st) {
  TDX_CHECK_ARG(n_rows >= 0 && T >= 1 && T <= TAU_DXB_TAU_STAR_MAX_KEYS,
                "tau_star_solve: need 1 <= T <= %d (got %lld)", TAU_DXB_TAU_STAR_MAX_KEYS, (long long)T);
  TDX_CHECK_ARG(sigma_id >= TAU_DXB_SIGMA_SOFTPLUS && sigma_id <= TAU_DXB_SIGMA_RELU,
                "tau_star_solve: bad sigma id %d", sigma_id);
  TDX_CHECK_ARG(n_iter >= 0, "tau_star_solve: n_iter < 0");
  TDX_CHECK_ARG(row_stride >= T || n_rows <= 1, "tau_star_solve: row stride %lld < T %lld", (long long)row_stride,
                (long long)T);
  if (n_rows == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(tau_out && kl_out && (scores || T <= 1), "tau_star_solve: null pointer");
  if (T <= 1) {   // one key: tau undefined, (tau_init, 0) as the reference returns
    const int64_t blocks = (n_rows + 255) / 256;
    tau_star_trivial_kernel<<<static_cast<unsigned>(blocks < 4096 ? blocks : 4096), 256, 0, st>>>(
        n_rows, tau_init, tau_out, kl_out);
    return check_launch("tau_star_trivial_kernel");
  }
  const int Ti = static_cast<int>(T);
  if (RegKernel fn = reg_kernel_for((Ti + 31) / 32)) {
    const int64_t blocks = (n_rows + kTsRegWarps - 1) / kTsRegWarps;
    TDX_CHECK_ARG(blocks < (1ll << 31), "tau_star_solve: too many rows");
    fn<<<static_cast<unsigned>(blocks), kTsRegWarps * 32, 0, st>>>(scores, n_rows, Ti, row_stride, sigma_id, n_iter,
                                                                   tau_init, tau_min, tau_max, eps, tau_out, kl_out);
    return check_launch("tau_star_reg_kernel");
  }
  constexpr size_t kSmemMax = 227 * 1024;
  const size_t per_warp = static_cast<size_t>(2) * Ti * sizeof(float);
  int warps = static_cast<int>(kSmemMax / per_warp);
  warps = warps < 1 ? 1 : (warps > 4 ? 4 : warps);
  const size_t smem = per_warp * warps;
  TDX_CUDA(cudaFuncSetAttribute(tau_star_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem)));
  const int64_t blocks = (n_rows + warps - 1) / warps;
  TDX_CHECK_ARG(blocks < (1ll << 31), "tau_star_solve: too many rows");
  tau_star_smem_kernel<<<static_cast<unsigned>(blocks), warps * 32, smem, st>>>(
      scores, n_rows, Ti, row_stride, sigma_id, n_iter, tau_init, tau_min, tau_max, eps, tau_out, kl_out);
  return check_launch("tau_star_smem_kernel");
}

int tau_star_analytic_impl(const float* scores, int64_t n_rows, int64_t T, int64_t row_stride, int32_t sigma_id,
                           float* tau_out, cudaStream_t st) {
  TDX_CHECK_ARG(n_rows >= 0 && T >= 1 && T < (1ll << 31), "tau_star_analytic: bad T %lld", (long long)T);
  TDX_CHECK_ARG(sigma_id >= TAU_DXB_SIGMA_SOFTPLUS && sigma_id <= TAU_DXB_SIGMA_RELU,
                "tau_star_analytic: bad sigma id %d", sigma_id);
  TDX_CHECK_ARG(row_stride >= T || n_rows <= 1, "tau_star_analytic: row stride < T");
  if (n_rows == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(scores && tau_out, "tau_star_analytic: null pointer");
  const int64_t blocks = (n_rows + 3) / 4;
  TDX_CHECK_ARG(blocks < (1ll << 31), "tau_star_analytic: too many rows");
  tau_star_analytic_kernel<<<static_cast<unsigned>(blocks), 128, 0, st>>>(scores, n_rows, static_cast<int>(T),
                                                                          row_stride, sigma_id, tau_out);
  return check_launch("tau_star_analytic_kernel");
}

}  // namespace taudxb
