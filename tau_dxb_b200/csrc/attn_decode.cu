// tau-opus attention forward for a few query rows (KV-cached decoding).
//
// Autoregressive decoding with a KV cache (predict.py's generate loop over the
// patched Whisper, echo/patch_whisper_stau.py:217-260) calls the operator with
// Lq = 1 against every cached key: decoder self-attention over the tokens so
// far, cross-attention over the 1500 encoder frames. The tiled kernels would
// spend a 64- or 256-row tile on that single row; here one CTA serves one
// query row, so the work is one pass over the row's K and V -- memory bound.
//
// Per row (echo/stau_opus_operator.py:82-101, with the precise path's fp32
// math, so it is held to the same 1e-4):
//   1. s_j = scale * q.k_j (+ mask) for every key into shared memory: eight
//      lanes per key row (16-byte loads of 8 dims each, four rows per warp
//      instruction), with the running max and first argmax;
//   2. block max / first argmax;
//   3. q_j = max(sigma(alpha (s_j - m))^tau, 1e-8) in place, Z = sum q_j;
//   4. O = sum_j q_j V_j / max(Z, 1e-8): each thread owns 8 dims of every 64th
//      V row (16-byte loads), partial sums reduced by shuffles and shared memory.
// Row state (max, Z, argmax) is written as by the other forward kernels, so
// the backward kernels accept it. Layout: bf16 / f16, D = 64, unit d-stride,
// 16-byte aligned rows (the tiled precise kernel serves everything else).

#include "attn.h"

namespace taudxb {
namespace {

constexpr int kDecThreads = 512, kDecWarps = kDecThreads / 32, kDecD = 64;

__device__ __forceinline__ int64_t doff(const int64_t* s, int64_t b, int64_t h, int64_t l, int64_t d) {
  return b * s[0] + h * s[1] + l * s[2] + d * s[3];
}

__device__ __forceinline__ float dec_mask(const AttnProblem& p, int b, int h, int r, int c) {
  float mv = 0.f;
  if (p.mask) mv = load_as_float(p.mask, p.mask_dtype, doff(p.ms, b, h, r, c));
  if (p.causal && c > r + (p.Lk - p.Lq)) mv += kMaskMin;
  return mv;
}

// 8 consecutive 16-bit floats (one 16-byte word) widened to fp32
template <typename T>
__device__ __forceinline__ void widen8(const uint4 w, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = Elem<T>::to_f(e[i]);
}

template <typename T>
__global__ void __launch_bounds__(kDecThreads) attn_fwd_decode_kernel(const AttnProblem p) {
  extern __shared__ __align__(16) float dsm[];
  float* red = dsm;                                  // [warps][64] partial O
  float* wmax = red + kDecWarps * kDecD;             // [warps]
  int* widx = reinterpret_cast<int*>(wmax + kDecWarps);
  float* s = reinterpret_cast<float*>(widx + kDecWarps);   // [Lk] scores, then q
  const int r = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Lk = p.Lk;
  const float tau = p.tau[h], alpha = p.alpha[h];
  const bool has_mask = p.mask != nullptr || p.causal;
  const T* kb = static_cast<const T*>(p.k) + b * p.ks[0] + h * p.ks[1];
  const T* vb = static_cast<const T*>(p.v) + b * p.vs[0] + h * p.vs[1];

  // 1. scores: lane group kg (4 per warp) takes a key row, lane part its 8 dims
  const int kg = lane >> 3, part = lane & 7;
  float qv[8];
  widen8<T>(*reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) + doff(p.qs, b, h, r, 8 * part)), qv);
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  for (int j0 = 4 * warp; j0 < Lk; j0 += 4 * kDecWarps) {
    const int j = j0 + kg;
    float dot = 0.f;
    if (j < Lk) {
      float kf[8];
      widen8<T>(__ldg(reinterpret_cast<const uint4*>(kb + static_cast<int64_t>(j) * p.ks[2] + 8 * part)), kf);
#pragma unroll
      for (int i = 0; i < 8; ++i) dot = fmaf(qv[i], kf[i], dot);
    }
    dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    dot += __shfl_xor_sync(0xffffffffu, dot, 2);
    dot += __shfl_xor_sync(0xffffffffu, dot, 4);
    if (j < Lk) {
      float v = dot * p.scale;
      if (has_mask) v += dec_mask(p, b, h, r, j);
      if (part == 0) s[j] = v;
      if (v > best) { best = v; bidx = j; }   // keys in increasing order per lane
    }
  }
  // warp: the largest value, the smallest key holding it
#pragma unroll
  for (int off = 8; off < 32; off <<= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bidx, off);
    if (ov > best || (ov == best && oi < bidx)) { best = ov; bidx = oi; }
  }
  if (lane == 0) { wmax[warp] = best; widx[warp] = bidx; }
  __syncthreads();
  // 2. block max and first argmax
  float m = wmax[0];
  int amax = widx[0];
#pragma unroll
  for (int w = 1; w < kDecWarps; ++w) {
    const float ov = wmax[w];
    const int oi = widx[w];
    if (ov > m || (ov == m && oi < amax)) { m = ov; amax = oi; }
  }
  if (amax == 0x7fffffff) amax = 0;

  // 3. q_j in place and Z
  float l = 0.f;
  for (int j = tid; j < Lk; j += kDecThreads) {
    const float sg = sigma_precise(p.sigma, alpha * (s[j] - m));
    const float qq = fmaxf(powf(sg, tau), kClampMin);
    s[j] = qq;
    l += qq;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
  __syncthreads();                 // every q_j written, every wmax read
  if (lane == 0) wmax[warp] = l;

  // 4. O: thread (row slot rs, dim block db) sums q_j V_j[8 db .. 8 db + 8) over j = rs mod 64
  const int rs = tid >> 3, db = tid & 7;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int j = rs; j < Lk; j += kDecThreads / 8) {
    float vf[8];
    widen8<T>(__ldg(reinterpret_cast<const uint4*>(vb + static_cast<int64_t>(j) * p.vs[2] + 8 * db)), vf);
    const float qj = s[j];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = fmaf(qj, vf[i], acc[i]);
  }
  // the four row slots of a warp hold the same dims: lanes db, db+8, db+16, db+24
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 8);
    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 16);
  }
  if (lane < 8) {
#pragma unroll
    for (int i = 0; i < 8; ++i) red[warp * kDecD + 8 * db + i] = acc[i];
  }
  __syncthreads();
  if (tid < kDecD) {
    float Z = 0.f, o = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
      Z += wmax[w];
      o += red[w * kDecD + tid];
    }
    Z = fmaxf(Z, kClampMin);
    static_cast<T*>(p.out)[doff(p.outs, b, h, r, tid)] = Elem<T>::from_f(o / Z);
    if (tid == 0) {
      const int64_t ri = (static_cast<int64_t>(b) * p.H + h) * p.Lq + r;
      p.row_max[ri] = m;
      p.row_z[ri] = Z;
      p.row_argmax[ri] = amax;
    }
  }
}

template <typename T>
int launch_decode(const AttnProblem& p, cudaStream_t st) {
  const size_t smem = (kDecWarps * kDecD + 2 * kDecWarps) * sizeof(float) + static_cast<size_t>(p.Lk) * sizeof(float);
  auto kern = attn_fwd_decode_kernel<T>;
  TDX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(p.Lq, p.H, p.B);
  kern<<<grid, kDecThreads, smem, st>>>(p);
  return check_launch("attn_fwd_decode_kernel");
}

bool rows16(const void* ptr, const int64_t s[4]) {
  return s[3] == 1 && reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && s[0] % 8 == 0 && s[1] % 8 == 0 &&
         s[2] % 8 == 0 && s[0] >= 0 && s[1] >= 0 && s[2] > 0;
}

}  // namespace

bool attn_decode_supported(const AttnProblem& p) {
  return p.Lq >= 1 && p.Lq <= kDecodeMaxRows && p.D == kDecD && p.Lk >= 1 && p.Lk <= kDecodeMaxKeys &&
         (p.dtype == TAU_DXB_BF16 || p.dtype == TAU_DXB_F16) && rows16(p.q, p.qs) && rows16(p.k, p.ks) &&
         rows16(p.v, p.vs);
}

int attn_fwd_decode(const AttnProblem& p, cudaStream_t st) {
  if (!attn_decode_supported(p))
    return fail(TAU_DXB_ERR_UNSUPPORTED, "decode forward needs Lq <= %d, D == 64, Lk <= %d, bf16/f16 "
                "with 16-byte aligned rows", kDecodeMaxRows, kDecodeMaxKeys);
  return p.dtype == TAU_DXB_BF16 ? launch_decode<__nv_bfloat16>(p, st) : launch_decode<__half>(p, st);
}

}  // namespace taudxb
