// tau-opus attention backward: stages shared by the precise and tensor paths.
//
//   prologue (K0): zero the accumulators; Drow[i] = sum_d dO[i,d] * O[i,d]
//                  (= sum_j P_ij dP_ij, the reference's `weighted`,
//                  echo/stau_opus_operator.py:135).
//   epilogue (K3): the max-shift correction of echo/stau_opus_operator.py:139-141,
//                  F[i, amax_i] -= rowsum(F)_i, applied to the products instead
//                  of to F:  dQ_i -= rowsumF_i * K[amax_i],
//                            dK[amax_i] -= rowsumF_i * Q_i  (scatter-add),
//                  then the scale and the dtype cast of dQ / dK.

#include "attn.h"

namespace taudxb {
namespace {

__device__ __forceinline__ int64_t off4(const int64_t* s, int64_t b, int64_t h, int64_t l, int64_t d) {
  return b * s[0] + h * s[1] + l * s[2] + d * s[3];
}

template <typename T>
__global__ void drow_kernel(const AttnProblem p) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t nrows = static_cast<int64_t>(p.B) * p.H * p.Lq;
  if (row >= nrows) return;
  const int64_t bh = row / p.Lq, i = row % p.Lq, b = bh / p.H, h = bh % p.H;
  float acc = 0.f;
  for (int d = lane; d < p.D; d += 32) {
    const float g = Elem<T>::to_f(static_cast<const T*>(p.dout)[off4(p.dos, b, h, i, d)]);
    const float o = Elem<T>::to_f(static_cast<const T*>(p.o)[off4(p.os, b, h, i, d)]);
    acc = fmaf(g, o, acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) p.ws_drow[row] = acc;
}

// One warp per query row: dQ = scale * (acc - rowF * K[amax]); scatter into dK acc.
template <typename T>
__global__ void fix_dq_kernel(const AttnProblem p) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t nrows = static_cast<int64_t>(p.B) * p.H * p.Lq;
  if (row >= nrows) return;
  const int64_t bh = row / p.Lq, i = row % p.Lq, b = bh / p.H, h = bh % p.H;
  const float f = p.ws_rowf[row];
  const int a = p.row_argmax[row];
  const bool amax_ok = a >= 0 && a < p.Lk;
  for (int d = lane; d < p.D; d += 32) {
    float kv = 0.f, qv = 0.f;
    if (amax_ok) {
      kv = Elem<T>::to_f(static_cast<const T*>(p.k)[off4(p.ks, b, h, a, d)]);
      qv = Elem<T>::to_f(static_cast<const T*>(p.q)[off4(p.qs, b, h, i, d)]);
      atomicAdd(p.ws_dk + (bh * p.Lk + a) * p.D + d, -f * qv);
    }
    const float g = p.ws_dq[row * p.D + d] - f * kv;
    static_cast<T*>(p.dq)[off4(p.dqs, b, h, i, d)] = Elem<T>::from_f(g * p.scale);
  }
}

template <typename T>
__global__ void write_dk_kernel(const AttnProblem p) {
  const int64_t total = static_cast<int64_t>(p.B) * p.H * p.Lk * p.D;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t d = e % p.D, rest = e / p.D, j = rest % p.Lk, bh = rest / p.Lk;
    const int64_t b = bh / p.H, h = bh % p.H;
    static_cast<T*>(p.dk)[off4(p.dks, b, h, j, d)] = Elem<T>::from_f(p.ws_dk[e] * p.scale);
  }
}

template <typename T>
int prologue(const AttnProblem& p, cudaStream_t st) {
  const int64_t nrows = static_cast<int64_t>(p.B) * p.H * p.Lq;
  drow_kernel<T><<<static_cast<unsigned>((nrows + 7) / 8), 256, 0, st>>>(p);
  return check_launch("drow_kernel");
}

template <typename T>
int epilogue(const AttnProblem& p, cudaStream_t st) {
  const int64_t nrows = static_cast<int64_t>(p.B) * p.H * p.Lq;
  if (nrows > 0) {
    fix_dq_kernel<T><<<static_cast<unsigned>((nrows + 7) / 8), 256, 0, st>>>(p);
    int rc = check_launch("fix_dq_kernel");
    if (rc) return rc;
  }
  const int64_t total = static_cast<int64_t>(p.B) * p.H * p.Lk * p.D;
  if (total > 0) {
    int64_t blocks = (total + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    write_dk_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, st>>>(p);
    return check_launch("write_dk_kernel");
  }
  return TAU_DXB_OK;
}

size_t align_up(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

}  // namespace

WorkspaceLayout workspace_layout(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D) {
  WorkspaceLayout w;
  size_t o = 0;
  w.dq = o;   o += align_up(static_cast<size_t>(B * H * Lq * D) * 4);
  w.dk = o;   o += align_up(static_cast<size_t>(B * H * Lk * D) * 4);
  w.drow = o; o += align_up(static_cast<size_t>(B * H * Lq) * 4);
  w.rowf = o; o += align_up(static_cast<size_t>(B * H * Lq) * 4);
  w.total = o;
  return w;
}

int attn_bwd_prologue(const AttnProblem& p, cudaStream_t st) {
  const WorkspaceLayout w = workspace_layout(p.B, p.H, p.Lq, p.Lk, p.D);
  // dQ accumulator, rowsum(F) and the per-head sums start at zero.
  TDX_CUDA(cudaMemsetAsync(p.ws_dq, 0, w.dk - w.dq, st));
  TDX_CUDA(cudaMemsetAsync(p.ws_rowf, 0, w.total - w.rowf, st));
  TDX_CUDA(cudaMemsetAsync(p.dtau, 0, p.H * sizeof(float), st));
  TDX_CUDA(cudaMemsetAsync(p.dalpha, 0, p.H * sizeof(float), st));
  switch (p.dtype) {
    case TAU_DXB_F32: return prologue<float>(p, st);
    case TAU_DXB_BF16: return prologue<__nv_bfloat16>(p, st);
    default: return prologue<__half>(p, st);
  }
}

int attn_bwd_epilogue(const AttnProblem& p, cudaStream_t st) {
  switch (p.dtype) {
    case TAU_DXB_F32: return epilogue<float>(p, st);
    case TAU_DXB_BF16: return epilogue<__nv_bfloat16>(p, st);
    default: return epilogue<__half>(p, st);
  }
}

}  // namespace taudxb
