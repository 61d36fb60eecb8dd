// tau-opus attention, precise path: fp32 CUDA-core math and accumulation.
//
// This is the fp32-checked path (inputs of any dtype are widened to fp32 on
// load; every product, sum and transcendental is fp32 with CUDA's accurate
// math functions). It follows the reference eager operator
// (echo/stau_opus_operator.py:66-166) operation by operation and is held to
// 1e-4 relative error against it.
//
// Forward  (one CTA = 64 query rows of one (b,h); 256 threads, 4x4 micro-tiles):
//   pass 1 sweeps all key tiles for the row max and first argmax (the sigma of
//   the reference is applied to s - max(s) and is not shift invariant, so the
//   exact max is needed before any sigma); pass 2 recomputes the identical
//   scores and accumulates sum(q) and q V.
// Backward main (one CTA = 64 keys of one (b,h)): sweeps all query tiles,
//   recomputes S and dP = dO V^T, forms P and F, accumulates dV and dK in
//   registers, adds dQ partials and rowsum(F) with fp32 atomics, and reduces
//   the dtau / dalpha sums per CTA.

#include "attn.h"

namespace taudxb {
namespace {

constexpr int BM = 64, BN = 64, DM = 64, LDT = 68, NT = 256;

template <typename T>
__device__ __forceinline__ float ld(const void* base, int64_t off) {
  return Elem<T>::to_f(static_cast<const T*>(base)[off]);
}

__device__ __forceinline__ int64_t off4(const int64_t* s, int64_t b, int64_t h, int64_t l, int64_t d) {
  return b * s[0] + h * s[1] + l * s[2] + d * s[3];
}

// Loads a [64 rows][D] tile into smem transposed (dst[d*LDT + r]) and/or
// row-major (dst2[r*LDT + d]); rows beyond `rows` and columns beyond D are 0.
template <typename T>
__device__ __forceinline__ void load_tile(const void* src, const int64_t* s, int b, int h, int row0,
                                          int rows, int D, float* tr, float* rm) {
  for (int idx = threadIdx.x; idx < 64 * DM; idx += NT) {
    const int r = idx / DM, d = idx % DM;
    float v = 0.f;
    if (r < rows && d < D) v = ld<T>(src, off4(s, b, h, row0 + r, d));
    if (tr) tr[d * LDT + r] = v;
    if (rm) rm[r * LDT + d] = v;
  }
}

// acc[i][j] += sum_d A[d][ra+i] * B[d][cb+j] over d < n; A, B stored [d][LDT].
__device__ __forceinline__ void mma_tt(const float* A, const float* Bm, int n, int ra, int cb,
                                       float acc[4][4]) {
  for (int d = 0; d < n; ++d) {
    const float4 a = *reinterpret_cast<const float4*>(A + d * LDT + ra);
    const float4 b = *reinterpret_cast<const float4*>(Bm + d * LDT + cb);
    const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
  }
}

__device__ __forceinline__ float mask_value(const AttnProblem& p, int b, int h, int r, int c) {
  float mv = 0.f;
  if (p.mask) mv = load_as_float(p.mask, p.mask_dtype, off4(p.ms, b, h, r, c));
  if (p.causal && c > r + (p.Lk - p.Lq)) mv += kMaskMin;
  return mv;
}

template <typename T>
__global__ void __launch_bounds__(NT) attn_fwd_precise_kernel(const AttnProblem p) {
  extern __shared__ __align__(16) float sm[];
  float* Qt = sm;                 // [DM][LDT]
  float* Kt = Qt + DM * LDT;      // [DM][LDT]
  float* Vs = Kt + DM * LDT;      // [BN][LDT] row-major
  float* Pt = Vs + BN * LDT;      // [BN][LDT]  Pt[c][r]
  const int b = blockIdx.z, h = blockIdx.y, r0 = blockIdx.x * BM;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int rows = min(BM, p.Lq - r0);
  const float tau = p.tau[h];
  const float alpha = p.alpha[h];
  const bool has_mask = p.mask != nullptr || p.causal;

  load_tile<T>(p.q, p.qs, b, h, r0, rows, p.D, Qt, nullptr);

  // ---- pass 1: row max and first argmax ----
  float best[4];
  int bidx[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) { best[i] = -INFINITY; bidx[i] = 0x7fffffff; }
  for (int c0 = 0; c0 < p.Lk; c0 += BN) {
    __syncthreads();
    load_tile<T>(p.k, p.ks, b, h, c0, min(BN, p.Lk - c0), p.D, Kt, nullptr);
    __syncthreads();
    float s[4][4] = {};
    mma_tt(Qt, Kt, p.D, ty * 4, tx * 4, s);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = r0 + ty * 4 + i, c = c0 + tx * 4 + j;
        if (c < p.Lk && r < p.Lq) {
          float v = s[i][j] * p.scale;
          if (has_mask) v += mask_value(p, b, h, r, c);
          if (v > best[i]) { best[i] = v; bidx[i] = c; }
        }
      }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best[i], off);
      const int oi = __shfl_xor_sync(0xffffffffu, bidx[i], off);
      if (ov > best[i] || (ov == best[i] && oi < bidx[i])) { best[i] = ov; bidx[i] = oi; }
    }

  // ---- pass 2: q = max(sigma(alpha (s - m))^tau, 1e-8), l = sum q, O = q V ----
  float l[4] = {0.f, 0.f, 0.f, 0.f};
  float o[4][4] = {};
  for (int c0 = 0; c0 < p.Lk; c0 += BN) {
    __syncthreads();
    const int cols = min(BN, p.Lk - c0);
    load_tile<T>(p.k, p.ks, b, h, c0, cols, p.D, Kt, nullptr);
    load_tile<T>(p.v, p.vs, b, h, c0, cols, p.D, nullptr, Vs);
    __syncthreads();
    float s[4][4] = {};
    mma_tt(Qt, Kt, p.D, ty * 4, tx * 4, s);
    float qv[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = r0 + ty * 4 + i, c = c0 + tx * 4 + j;
        float qq = 0.f;
        if (c < p.Lk && r < p.Lq) {
          float v = s[i][j] * p.scale;
          if (has_mask) v += mask_value(p, b, h, r, c);
          const float x = v - best[i];
          const float sg = sigma_precise(p.sigma, alpha * x);
          qq = fmaxf(powf(sg, tau), kClampMin);
        }
        qv[i][j] = qq;
        l[i] += qq;
      }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(Pt + (tx * 4 + j) * LDT + ty * 4) =
          make_float4(qv[0][j], qv[1][j], qv[2][j], qv[3][j]);
    __syncthreads();
    mma_tt(Pt, Vs, BN, ty * 4, tx * 4, o);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) l[i] += __shfl_xor_sync(0xffffffffu, l[i], off);

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + ty * 4 + i;
    if (r >= p.Lq) continue;
    const float Z = fmaxf(l[i], kClampMin);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int d = tx * 4 + j;
      if (d < p.D)
        static_cast<T*>(p.out)[off4(p.outs, b, h, r, d)] = Elem<T>::from_f(o[i][j] / Z);
    }
    if (tx == 0) {
      const int64_t ri = (static_cast<int64_t>(b) * p.H + h) * p.Lq + r;
      p.row_max[ri] = best[i];
      p.row_z[ri] = Z;
      p.row_argmax[ri] = bidx[i];
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(NT) attn_bwd_precise_kernel(const AttnProblem p) {
  extern __shared__ __align__(16) float sm[];
  float* Kt = sm;                  // [DM][LDT] K^T
  float* Ks = Kt + DM * LDT;       // [BN][LDT] K
  float* Vt = Ks + BN * LDT;       // [DM][LDT] V^T
  float* Qt = Vt + DM * LDT;       // [DM][LDT] Q^T
  float* Qs = Qt + DM * LDT;       // [BM][LDT] Q
  float* dOt = Qs + BM * LDT;      // [DM][LDT] dO^T
  float* dOs = dOt + DM * LDT;     // [BM][LDT] dO
  float* Ps = dOs + BM * LDT;      // [BM][LDT] P[r][c]
  float* Fs = Ps + BM * LDT;       // [BM][LDT] F[r][c]
  float* Ft = Fs + BM * LDT;       // [BN][LDT] F[c][r]
  float* rstat = Ft + BN * LDT;    // m[64], Z[64], Drow[64]
  float* red = rstat + 3 * BM;     // [2][8] block reduction
  const int b = blockIdx.z, h = blockIdx.y, c0 = blockIdx.x * BN;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int cols = min(BN, p.Lk - c0);
  const float tau = p.tau[h];
  const float alpha = p.alpha[h];
  const bool has_mask = p.mask != nullptr || p.causal;
  const int64_t bh = static_cast<int64_t>(b) * p.H + h;

  load_tile<T>(p.k, p.ks, b, h, c0, cols, p.D, Kt, Ks);
  load_tile<T>(p.v, p.vs, b, h, c0, cols, p.D, Vt, nullptr);

  float dv[4][4] = {}, dk[4][4] = {};
  float dtau = 0.f, dalpha = 0.f;
  for (int r0 = 0; r0 < p.Lq; r0 += BM) {
    const int rows = min(BM, p.Lq - r0);
    __syncthreads();
    load_tile<T>(p.q, p.qs, b, h, r0, rows, p.D, Qt, Qs);
    load_tile<T>(p.dout, p.dos, b, h, r0, rows, p.D, dOt, dOs);
    for (int r = tid; r < BM; r += NT) {
      const bool ok = r < rows;
      rstat[r] = ok ? p.row_max[bh * p.Lq + r0 + r] : 0.f;
      rstat[BM + r] = ok ? p.row_z[bh * p.Lq + r0 + r] : 1.f;
      rstat[2 * BM + r] = ok ? p.ws_drow[bh * p.Lq + r0 + r] : 0.f;
    }
    __syncthreads();
    float s[4][4] = {}, dp[4][4] = {};
    mma_tt(Qt, Kt, p.D, ty * 4, tx * 4, s);
    mma_tt(dOt, Vt, p.D, ty * 4, tx * 4, dp);
    float P[4][4], F[4][4], rowf[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      rowf[i] = 0.f;
      const int rl = ty * 4 + i, r = r0 + rl;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = c0 + tx * 4 + j;
        float pv = 0.f, fv = 0.f;
        if (rl < rows && c < p.Lk) {
          float v = s[i][j] * p.scale;
          if (has_mask) v += mask_value(p, b, h, r, c);
          const float x = v - rstat[rl];
          const float ax = alpha * x;
          const float sg = sigma_precise(p.sigma, ax);
          const float qq = fmaxf(powf(sg, tau), kClampMin);
          pv = qq / rstat[BM + rl];
          const float sgp = sigma_prime_precise(p.sigma, ax);
          const float ratio = sgp / sg;
          const float t = pv * (dp[i][j] - rstat[2 * BM + rl]);
          fv = tau * t * ratio * alpha;
          dtau += t * fmaxf(logf(sg), -30.f);
          dalpha += tau * t * fminf(fmaxf(ratio * x, -30.f), 30.f);
        }
        P[i][j] = pv;
        F[i][j] = fv;
        rowf[i] += fv;
      }
      *reinterpret_cast<float4*>(Ps + rl * LDT + tx * 4) = make_float4(P[i][0], P[i][1], P[i][2], P[i][3]);
      *reinterpret_cast<float4*>(Fs + rl * LDT + tx * 4) = make_float4(F[i][0], F[i][1], F[i][2], F[i][3]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(Ft + (tx * 4 + j) * LDT + ty * 4) =
          make_float4(F[0][j], F[1][j], F[2][j], F[3][j]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) rowf[i] += __shfl_xor_sync(0xffffffffu, rowf[i], off);
      const int rl = ty * 4 + i;
      if (tx == 0 && rl < rows) atomicAdd(p.ws_rowf + bh * p.Lq + r0 + rl, rowf[i]);
    }
    __syncthreads();
    // dV[c][d] += sum_r P[r][c] dO[r][d];  dK[c][d] += sum_r F[r][c] Q[r][d]
    mma_tt(Ps, dOs, rows, ty * 4, tx * 4, dv);
    mma_tt(Fs, Qs, rows, ty * 4, tx * 4, dk);
    // dQ[r][d] += sum_c F[r][c] K[c][d]
    float dq[4][4] = {};
    mma_tt(Ft, Ks, cols, ty * 4, tx * 4, dq);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rl = ty * 4 + i;
      if (rl >= rows) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d = tx * 4 + j;
        if (d < p.D) atomicAdd(p.ws_dq + (bh * p.Lq + r0 + rl) * p.D + d, dq[i][j]);
      }
    }
  }
  // write dV (final) and the unscaled dK accumulator
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int cl = ty * 4 + i;
    if (cl >= cols) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int d = tx * 4 + j;
      if (d >= p.D) continue;
      static_cast<T*>(p.dv)[off4(p.dvs, b, h, c0 + cl, d)] = Elem<T>::from_f(dv[i][j]);
      p.ws_dk[(bh * p.Lk + c0 + cl) * p.D + d] = dk[i][j];
    }
  }
  // per-CTA dtau / dalpha
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    dtau += __shfl_xor_sync(0xffffffffu, dtau, off);
    dalpha += __shfl_xor_sync(0xffffffffu, dalpha, off);
  }
  if ((tid & 31) == 0) { red[tid >> 5] = dtau; red[8 + (tid >> 5)] = dalpha; }
  __syncthreads();
  if (tid == 0) {
    float a = 0.f, c = 0.f;
    for (int w = 0; w < NT / 32; ++w) { a += red[w]; c += red[8 + w]; }
    atomicAdd(p.dtau + h, a);
    atomicAdd(p.dalpha + h, c);
  }
}

template <typename T>
int launch_fwd(const AttnProblem& p, cudaStream_t st) {
  const size_t smem = (2 * DM * LDT + 2 * BN * LDT) * sizeof(float);
  auto kern = attn_fwd_precise_kernel<T>;
  TDX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.Lq + BM - 1) / BM, p.H, p.B);
  kern<<<grid, NT, smem, st>>>(p);
  return check_launch("attn_fwd_precise_kernel");
}

template <typename T>
int launch_bwd(const AttnProblem& p, cudaStream_t st) {
  const size_t smem = (4 * DM * LDT + 6 * BN * LDT + 3 * BM + 16) * sizeof(float);
  auto kern = attn_bwd_precise_kernel<T>;
  TDX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.Lk + BN - 1) / BN, p.H, p.B);
  kern<<<grid, NT, smem, st>>>(p);
  return check_launch("attn_bwd_precise_kernel");
}

}  // namespace

int attn_fwd_precise(const AttnProblem& p, cudaStream_t st) {
  if (p.D > DM) return fail(TAU_DXB_ERR_UNSUPPORTED, "precise attention path supports D <= %d (got %d)", DM, p.D);
  switch (p.dtype) {
    case TAU_DXB_F32: return launch_fwd<float>(p, st);
    case TAU_DXB_BF16: return launch_fwd<__nv_bfloat16>(p, st);
    default: return launch_fwd<__half>(p, st);
  }
}

int attn_bwd_precise_main(const AttnProblem& p, cudaStream_t st) {
  if (p.D > DM) return fail(TAU_DXB_ERR_UNSUPPORTED, "precise attention path supports D <= %d (got %d)", DM, p.D);
  switch (p.dtype) {
    case TAU_DXB_F32: return launch_bwd<float>(p, st);
    case TAU_DXB_BF16: return launch_bwd<__nv_bfloat16>(p, st);
    default: return launch_bwd<__half>(p, st);
  }
}

}  // namespace taudxb
