// fp32 LayerNorm forward and backward for the Whisper train step's 62 layer
// norms (d = 768; rows = batch x frames), as autocast runs them: fp32 input,
// weight and bias, fp32 output. Both kernels are HBM-bound row sweeps:
//
//   forward : one warp per row, the row in registers (d / 128 float4 chunks per
//             lane); mean, then the variance about it (no E[x^2] - mean^2
//             cancellation), y = (x - mean) rstd gamma + beta; writes y (fp32,
//             or bf16 rounded to nearest even for a norm whose one consumer is
//             a bf16 GEMM under autocast), mean, rstd. 8 (6) bytes per element.
//   backward: one warp per row, persistent CTAs; per row xhat = (x - mean) rstd,
//             g = gamma dy, dx = rstd (g - mean(g) - xhat mean(g xhat)), and
//             per-column dgamma += dy xhat, dbeta += dy kept in registers over
//             all of a warp's rows; the warps of a CTA add theirs in shared
//             memory into one partial row per CTA, and a second kernel sums the
//             partial rows column by column in a fixed order (deterministic).
//             dy is fp32 or bf16 (the gradient of a bf16 y). 12 (10) bytes per
//             element plus 2 x 4 x d per CTA.

#include <type_traits>

#include "common.cuh"

namespace taudxb {
namespace {

constexpr int kLnWarps = 8;            // rows in flight per CTA
constexpr uint32_t kFull = 0xffffffffu;

__device__ __forceinline__ float ln_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// four fp32 values to memory as fp32 (16 B) or bf16 (8 B, round to nearest even)
__device__ __forceinline__ void store4(float* p, int64_t i4, float4 v) { reinterpret_cast<float4*>(p)[i4] = v; }
__device__ __forceinline__ void store4(__nv_bfloat16* p, int64_t i4, float4 v) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&lo);
  u.y = *reinterpret_cast<const uint32_t*>(&hi);
  reinterpret_cast<uint2*>(p)[i4] = u;
}
__device__ __forceinline__ float4 load4(const float* p, int64_t i4) {
  return __ldcs(reinterpret_cast<const float4*>(p) + i4);
}
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p, int64_t i4) {
  const uint2 u = __ldcs(reinterpret_cast<const uint2*>(p) + i4);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}

template <int NCH, typename TY>
__global__ void __launch_bounds__(kLnWarps * 32)
ln_fwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
              float eps, int64_t M, TY* __restrict__ y, float* __restrict__ mean_out,
              float* __restrict__ rstd_out) {
  constexpr int N = NCH * 128;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kLnWarps;
  float4 g[NCH], b[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    g[c] = __ldg(reinterpret_cast<const float4*>(gamma) + c * 32 + lane);
    b[c] = __ldg(reinterpret_cast<const float4*>(beta) + c * 32 + lane);
  }
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kLnWarps + (threadIdx.x >> 5); row < M; row += warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + row * N);
    float4 v[NCH];
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      v[c] = __ldcs(xr + c * 32 + lane);
      s += (v[c].x + v[c].y) + (v[c].z + v[c].w);
    }
    const float mean = ln_warp_sum(s) * (1.f / N);
    float q = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const float a = v[c].x - mean, bb = v[c].y - mean, cc = v[c].z - mean, d = v[c].w - mean;
      q = fmaf(a, a, fmaf(bb, bb, fmaf(cc, cc, fmaf(d, d, q))));
    }
    const float rstd = rsqrtf(ln_warp_sum(q) * (1.f / N) + eps);
    TY* yr = y + row * N;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      float4 o;
      o.x = fmaf((v[c].x - mean) * rstd, g[c].x, b[c].x);
      o.y = fmaf((v[c].y - mean) * rstd, g[c].y, b[c].y);
      o.z = fmaf((v[c].z - mean) * rstd, g[c].z, b[c].z);
      o.w = fmaf((v[c].w - mean) * rstd, g[c].w, b[c].w);
      store4(yr, c * 32 + lane, o);
    }
    if (lane == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
}

// Backward CTA shape: 8 warps; 4 warps for rows of 768 and more, whose ~150
// registers per thread would otherwise leave one 8-warp CTA per SM (4-warp
// CTAs fit three: 12 warps of loads in flight instead of 8).
constexpr int ln_bwd_warps(int nch) { return nch >= 6 ? 4 : 8; }
constexpr int ln_bwd_ctas_per_sm(int nch) { return nch >= 6 ? 3 : 2; }

template <int NCH, typename TD, int WARPS = ln_bwd_warps(NCH)>
__global__ void __launch_bounds__(WARPS * 32)
ln_bwd_kernel(const TD* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ mean_in,
              const float* __restrict__ rstd_in, const float* __restrict__ gamma, int64_t M,
              float* __restrict__ dx, float* __restrict__ part_dg, float* __restrict__ part_db) {
  constexpr int N = NCH * 128;
  __shared__ float4 red[WARPS][NCH * 32];
  __shared__ float4 sg[NCH * 32];          // gamma, read per row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * WARPS;
  for (int i = threadIdx.x; i < NCH * 32; i += WARPS * 32) sg[i] = __ldg(reinterpret_cast<const float4*>(gamma) + i);
  __syncthreads();
  float4 adg[NCH], adb[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    adg[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    adb[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // the next row's dy and x are loaded while this one is processed
  using DV = typename std::conditional<sizeof(TD) == 2, uint2, float4>::type;
  auto ld_dy = [&](int64_t r, int c) -> DV { return __ldcs(reinterpret_cast<const DV*>(dy + r * N) + c * 32 + lane); };
  auto to4 = [](DV v) -> float4 {
    if constexpr (sizeof(TD) == 2)
      return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                         __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
    else
      return v;
  };
  int64_t row = static_cast<int64_t>(blockIdx.x) * WARPS + warp;
  DV nd[NCH];
  float4 nx[NCH];
  if (row < M) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      nd[c] = ld_dy(row, c);
      nx[c] = __ldcs(reinterpret_cast<const float4*>(x + row * N) + c * 32 + lane);
    }
  }
  for (; row < M; row += warps) {
    float4 d[NCH], xh[NCH];
    const float mean = __ldg(mean_in + row), rstd = __ldg(rstd_in + row);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      d[c] = to4(nd[c]);
      xh[c] = nx[c];
    }
    const int64_t nrow = row + warps;
    if (nrow < M) {
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        nd[c] = ld_dy(nrow, c);
        nx[c] = __ldcs(reinterpret_cast<const float4*>(x + nrow * N) + c * 32 + lane);
      }
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const float4 xv = xh[c];
      xh[c] = make_float4((xv.x - mean) * rstd, (xv.y - mean) * rstd, (xv.z - mean) * rstd, (xv.w - mean) * rstd);
      const float4 gm = sg[c * 32 + lane];
      const float gx = gm.x * d[c].x, gy = gm.y * d[c].y, gz = gm.z * d[c].z, gw = gm.w * d[c].w;
      s1 += (gx + gy) + (gz + gw);
      s2 = fmaf(gx, xh[c].x, fmaf(gy, xh[c].y, fmaf(gz, xh[c].z, fmaf(gw, xh[c].w, s2))));
      adg[c].x = fmaf(d[c].x, xh[c].x, adg[c].x);
      adg[c].y = fmaf(d[c].y, xh[c].y, adg[c].y);
      adg[c].z = fmaf(d[c].z, xh[c].z, adg[c].z);
      adg[c].w = fmaf(d[c].w, xh[c].w, adg[c].w);
      adb[c].x += d[c].x;
      adb[c].y += d[c].y;
      adb[c].z += d[c].z;
      adb[c].w += d[c].w;
    }
    const float m1 = ln_warp_sum(s1) * (1.f / N), m2 = ln_warp_sum(s2) * (1.f / N);
    float4* dxr = reinterpret_cast<float4*>(dx + row * N);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      float4 o;
      const float4 gm = sg[c * 32 + lane];
      o.x = rstd * (gm.x * d[c].x - m1 - xh[c].x * m2);
      o.y = rstd * (gm.y * d[c].y - m1 - xh[c].y * m2);
      o.z = rstd * (gm.z * d[c].z - m1 - xh[c].z * m2);
      o.w = rstd * (gm.w * d[c].w - m1 - xh[c].w * m2);
      dxr[c * 32 + lane] = o;
    }
  }
  // this CTA's column partials: warps in a fixed order through shared memory,
  // dgamma then dbeta through the same buffer
#pragma unroll
  for (int which = 0; which < 2; ++which) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) red[warp][c * 32 + lane] = which ? adb[c] : adg[c];
    __syncthreads();
    for (int col4 = threadIdx.x; col4 < NCH * 32; col4 += WARPS * 32) {
      float4 acc = red[0][col4];
#pragma unroll
      for (int w = 1; w < WARPS; ++w) {
        const float4 v = red[w][col4];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      float* dst = (which ? part_db : part_dg) + static_cast<int64_t>(blockIdx.x) * N;
      reinterpret_cast<float4*>(dst)[col4] = acc;
    }
    __syncthreads();
  }
}

// dgamma[c] = sum_b part_dg[b][c], dbeta likewise. A CTA takes 32 columns of
// the [2, parts, N] partials; its 8 warps each sum a contiguous range of the
// partial rows (lane = column, coalesced), then warp 0 adds the 8 sums in
// warp order: a fixed order, and 8 independent add chains per column instead
// of one.
constexpr int kLnRedWarps = 8;
__global__ void __launch_bounds__(kLnRedWarps * 32)
ln_bwd_reduce_kernel(const float* __restrict__ part_dg, const float* __restrict__ part_db, int parts, int N,
                     float* __restrict__ dgamma, float* __restrict__ dbeta) {
  __shared__ float red[kLnRedWarps][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;          // over 2 N: dgamma columns, then dbeta
  const bool ok = col < 2 * N;
  const float* src = col < N ? part_dg + col : part_db + (col - N);
  const int per = (parts + kLnRedWarps - 1) / kLnRedWarps;
  const int b0 = warp * per, b1 = b0 + per < parts ? b0 + per : parts;
  // four independent chains (loads in flight), added in a fixed order
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  if (ok) {
    int b = b0;
    for (; b + 3 < b1; b += 4) {
      a0 += src[static_cast<int64_t>(b) * N];
      a1 += src[static_cast<int64_t>(b + 1) * N];
      a2 += src[static_cast<int64_t>(b + 2) * N];
      a3 += src[static_cast<int64_t>(b + 3) * N];
    }
    for (; b < b1; ++b) a0 += src[static_cast<int64_t>(b) * N];
  }
  red[warp][lane] = (a0 + a1) + (a2 + a3);
  __syncthreads();
  if (warp == 0 && ok) {
    float t = red[0][lane];
#pragma unroll
    for (int w = 1; w < kLnRedWarps; ++w) t += red[w][lane];
    if (col < N) dgamma[col] = t;
    else dbeta[col - N] = t;
  }
}

// backward CTAs (= partial rows): one wave of the CTAs that fit
int ln_parts(int64_t M, int64_t N) {
  const int nch = static_cast<int>(N / 128);
  const int64_t warps = ln_bwd_warps(nch);
  const int64_t want = (M + 8 * warps - 1) / (8 * warps);     // at least 8 rows per warp
  const int64_t cap = static_cast<int64_t>(sm_count()) * ln_bwd_ctas_per_sm(nch);
  return static_cast<int>(want < cap ? (want < 1 ? 1 : want) : cap);
}

template <template <int> class Launch, typename... A>
int dispatch_nch(int N, A... args) {
  switch (N / 128) {
    case 1: return Launch<1>::run(args...);
    case 2: return Launch<2>::run(args...);
    case 3: return Launch<3>::run(args...);
    case 4: return Launch<4>::run(args...);
    case 5: return Launch<5>::run(args...);
    case 6: return Launch<6>::run(args...);
    case 7: return Launch<7>::run(args...);
    case 8: return Launch<8>::run(args...);
    default: return fail(TAU_DXB_ERR_UNSUPPORTED, "layer norm: d = %d unsupported", N);
  }
}

template <int NCH>
struct FwdLaunch {
  static int run(const float* x, const float* g, const float* b, float eps, int64_t M, void* y, int y_bf16,
                 float* mean, float* rstd, cudaStream_t st) {
    const int grid = static_cast<int>((M + kLnWarps - 1) / kLnWarps < 8ll * sm_count()
                                          ? (M + kLnWarps - 1) / kLnWarps : 8ll * sm_count());
    if (y_bf16)
      ln_fwd_kernel<NCH, __nv_bfloat16><<<grid, kLnWarps * 32, 0, st>>>(
          x, g, b, eps, M, static_cast<__nv_bfloat16*>(y), mean, rstd);
    else
      ln_fwd_kernel<NCH, float><<<grid, kLnWarps * 32, 0, st>>>(x, g, b, eps, M, static_cast<float*>(y), mean, rstd);
    return check_launch("ln_fwd_kernel");
  }
};

template <int NCH>
struct BwdLaunch {
  static int run(const void* dy, int dy_bf16, const float* x, const float* mean, const float* rstd, const float* g,
                 int64_t M, float* dx, float* pdg, float* pdb, int parts, cudaStream_t st) {
    if (dy_bf16)
      ln_bwd_kernel<NCH, __nv_bfloat16><<<parts, ln_bwd_warps(NCH) * 32, 0, st>>>(
          static_cast<const __nv_bfloat16*>(dy), x, mean, rstd, g, M, dx, pdg, pdb);
    else
      ln_bwd_kernel<NCH, float><<<parts, ln_bwd_warps(NCH) * 32, 0, st>>>(static_cast<const float*>(dy), x, mean, rstd, g,
                                                                 M, dx, pdg, pdb);
    return check_launch("ln_bwd_kernel");
  }
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

size_t layer_norm_bwd_workspace(int64_t M, int64_t N) {
  if (M <= 0 || N <= 0) return 0;
  return static_cast<size_t>(ln_parts(M, N)) * static_cast<size_t>(N) * 2 * sizeof(float);
}

int layer_norm_fwd_impl(const float* x, int64_t M, int64_t N, const float* gamma, const float* beta, float eps,
                        void* y, int32_t y_dtype, float* mean, float* rstd, cudaStream_t st) {
  TDX_CHECK_ARG(y_dtype == TAU_DXB_F32 || y_dtype == TAU_DXB_BF16, "layer norm: y must be fp32 or bf16");
  TDX_CHECK_ARG(M >= 0 && N > 0 && N % 128 == 0 && N <= 1024,
                "layer norm: need d a multiple of 128 up to 1024 (got %lld)", (long long)N);
  if (M == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(x && gamma && beta && y && mean && rstd, "layer norm: null pointer");
  TDX_CHECK_ARG(aligned16(x) && aligned16(gamma) && aligned16(beta) && aligned16(y),
                "layer norm: x, gamma, beta and y must be 16-byte aligned");
  return dispatch_nch<FwdLaunch>(static_cast<int>(N), x, gamma, beta, eps, M, y,
                                 static_cast<int>(y_dtype == TAU_DXB_BF16), mean, rstd, st);
}

int layer_norm_bwd_impl(const void* dy, int32_t dy_dtype, const float* x, const float* mean, const float* rstd,
                        const float* gamma, int64_t M, int64_t N, float* dx, float* dgamma, float* dbeta,
                        void* workspace, size_t workspace_bytes, cudaStream_t st) {
  TDX_CHECK_ARG(dy_dtype == TAU_DXB_F32 || dy_dtype == TAU_DXB_BF16, "layer norm: dy must be fp32 or bf16");
  TDX_CHECK_ARG(M >= 0 && N > 0 && N % 128 == 0 && N <= 1024,
                "layer norm: need d a multiple of 128 up to 1024 (got %lld)", (long long)N);
  TDX_CHECK_ARG(dgamma && dbeta, "layer norm: null pointer");
  if (M == 0) {
    TDX_CUDA(cudaMemsetAsync(dgamma, 0, N * sizeof(float), st));
    TDX_CUDA(cudaMemsetAsync(dbeta, 0, N * sizeof(float), st));
    return TAU_DXB_OK;
  }
  TDX_CHECK_ARG(dy && x && mean && rstd && gamma && dx && workspace, "layer norm: null pointer");
  TDX_CHECK_ARG(aligned16(dy) && aligned16(x) && aligned16(gamma) && aligned16(dx) && aligned16(workspace),
                "layer norm: dy, x, gamma, dx and the workspace must be 16-byte aligned");
  const size_t need = layer_norm_bwd_workspace(M, N);
  if (workspace_bytes < need)
    return fail(TAU_DXB_ERR_WORKSPACE, "layer norm: workspace of %zu bytes, need %zu", workspace_bytes, need);
  const int parts = ln_parts(M, N);
  float* pdg = static_cast<float*>(workspace);
  float* pdb = pdg + static_cast<size_t>(parts) * N;
  int rc = dispatch_nch<BwdLaunch>(static_cast<int>(N), dy, static_cast<int>(dy_dtype == TAU_DXB_BF16), x, mean,
                                   rstd, gamma, M, dx, pdg, pdb, parts, st);
  if (rc) return rc;
  const int blocks = static_cast<int>((2 * N + 31) / 32);
  ln_bwd_reduce_kernel<<<blocks, kLnRedWarps * 32, 0, st>>>(pdg, pdb, parts, static_cast<int>(N), dgamma, dbeta);
  return check_launch("ln_bwd_reduce_kernel");
}

}  // namespace taudxb
