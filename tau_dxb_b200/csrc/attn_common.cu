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

// ---- vectorized forms for bf16, D = 64, unit d-stride, 16-byte aligned rows
// (the tensor-core path's layouts). Eight threads cover one 64-element row,
// 16 bytes of bf16 (32 bytes of fp32) each.
constexpr int kVecD = 64;

__device__ __forceinline__ void bf16x8_to_f32(uint4 w, float (&f)[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    f[2 * k] = __uint_as_float(u[k] << 16);
    f[2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint4 f32x8_to_bf16(const float (&f)[8]) {
  uint4 w;
  uint32_t* u = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __nv_bfloat162 b2 = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
    u[k] = *reinterpret_cast<const uint32_t*>(&b2);
  }
  return w;
}
__device__ __forceinline__ const uint4* row_ptr(const void* base, const int64_t* s, int b, int h, int l,
                                                int part) {
  return reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(base) + b * s[0] + h * s[1] +
                                        static_cast<int64_t>(l) * s[2]) + part;
}

// Drow = rowsum(dO * O); also zeroes the dQ accumulator row and rowsum(F).
__global__ void prep_vec_kernel(const AttnProblem p) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t row = t >> 3;
  const int part = static_cast<int>(t & 7);
  const int64_t nrows = static_cast<int64_t>(p.B) * p.H * p.Lq;
  if (row >= nrows) return;     // whole groups of 8 lanes leave together
  const int bh = static_cast<int>(row / p.Lq), i = static_cast<int>(row - static_cast<int64_t>(bh) * p.Lq);
  const int b = bh / p.H, h = bh - b * p.H;
  float g[8], o[8];
  bf16x8_to_f32(__ldg(row_ptr(p.dout, p.dos, b, h, i, part)), g);
  bf16x8_to_f32(__ldg(row_ptr(p.o, p.os, b, h, i, part)), o);
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) acc = fmaf(g[k], o[k], acc);
  const unsigned grp = 0xffu << (threadIdx.x & 24);   // this row's 8 lanes
  acc += __shfl_xor_sync(grp, acc, 4);
  acc += __shfl_xor_sync(grp, acc, 2);
  acc += __shfl_xor_sync(grp, acc, 1);
  float4* dq = reinterpret_cast<float4*>(p.ws_dq + row * kVecD) + 2 * part;
  dq[0] = make_float4(0.f, 0.f, 0.f, 0.f);
  dq[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (part == 0) {
    p.ws_drow[row] = acc;
    p.ws_rowf[row] = 0.f;
  }
  if (t < p.H) {
    p.dtau[t] = 0.f;
    p.dalpha[t] = 0.f;
  }
}

// dQ_i = scale (acc_i - rowF_i K[amax_i]) as bf16; dK_acc[amax_i] -= rowF_i Q_i.
__global__ void fix_dq_vec_kernel(const AttnProblem p) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t row = t >> 3;
  const int part = static_cast<int>(t & 7);
  const int64_t nrows = static_cast<int64_t>(p.B) * p.H * p.Lq;
  if (row >= nrows) return;
  const int bh = static_cast<int>(row / p.Lq), i = static_cast<int>(row - static_cast<int64_t>(bh) * p.Lq);
  const int b = bh / p.H, h = bh - b * p.H;
  const float f = p.ws_rowf[row];
  const int a = p.row_argmax[row];
  const float4* acc = reinterpret_cast<const float4*>(p.ws_dq + row * kVecD) + 2 * part;
  const float4 a0 = acc[0], a1 = acc[1];
  float g[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  if (a >= 0 && a < p.Lk) {
    float kv[8], qv[8];
    bf16x8_to_f32(__ldg(row_ptr(p.k, p.ks, b, h, a, part)), kv);
    bf16x8_to_f32(__ldg(row_ptr(p.q, p.qs, b, h, i, part)), qv);
#pragma unroll
    for (int k = 0; k < 8; ++k) g[k] = fmaf(-f, kv[k], g[k]);
    float4* dk = reinterpret_cast<float4*>(p.ws_dk + (static_cast<int64_t>(bh) * p.Lk + a) * kVecD) + 2 * part;
    atomicAdd(dk, make_float4(-f * qv[0], -f * qv[1], -f * qv[2], -f * qv[3]));
    atomicAdd(dk + 1, make_float4(-f * qv[4], -f * qv[5], -f * qv[6], -f * qv[7]));
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) g[k] *= p.scale;
  *reinterpret_cast<uint4*>(const_cast<uint4*>(row_ptr(p.dq, p.dqs, b, h, i, part))) = f32x8_to_bf16(g);
}

__global__ void write_dk_vec_kernel(const AttnProblem p) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t row = t >> 3;
  const int part = static_cast<int>(t & 7);
  const int64_t nrows = static_cast<int64_t>(p.B) * p.H * p.Lk;
  if (row >= nrows) return;
  const int bh = static_cast<int>(row / p.Lk), j = static_cast<int>(row - static_cast<int64_t>(bh) * p.Lk);
  const int b = bh / p.H, h = bh - b * p.H;
  const float4* acc = reinterpret_cast<const float4*>(p.ws_dk + row * kVecD) + 2 * part;
  const float4 a0 = acc[0], a1 = acc[1];
  const float g[8] = {a0.x * p.scale, a0.y * p.scale, a0.z * p.scale, a0.w * p.scale,
                      a1.x * p.scale, a1.y * p.scale, a1.z * p.scale, a1.w * p.scale};
  *reinterpret_cast<uint4*>(const_cast<uint4*>(row_ptr(p.dk, p.dks, b, h, j, part))) = f32x8_to_bf16(g);
}

bool vec_layout_ok(const void* ptr, const int64_t s[4]) {
  return s[3] == 1 && reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && s[0] % 8 == 0 && s[1] % 8 == 0 &&
         s[2] % 8 == 0;
}
bool vec_ok(const AttnProblem& p) {
  return p.dtype == TAU_DXB_BF16 && p.D == kVecD && vec_layout_ok(p.q, p.qs) && vec_layout_ok(p.k, p.ks) &&
         vec_layout_ok(p.o, p.os) && vec_layout_ok(p.dout, p.dos) && vec_layout_ok(p.dq, p.dqs) &&
         vec_layout_ok(p.dk, p.dks) && static_cast<int64_t>(p.B) * p.H * (p.Lq > p.Lk ? p.Lq : p.Lk) < (1ll << 31);
}
unsigned vec_blocks(int64_t rows) { return static_cast<unsigned>((rows * 8 + 255) / 256); }

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

// Products and sums that saturate at SIZE_MAX instead of wrapping, so that
// no shape can make the required workspace look small.
static size_t mul_sat(size_t a, size_t b) {
  size_t r;
  return __builtin_mul_overflow(a, b, &r) ? SIZE_MAX : r;
}
static size_t add_sat(size_t a, size_t b) {
  size_t r;
  return __builtin_add_overflow(a, b, &r) ? SIZE_MAX : r;
}

WorkspaceLayout workspace_layout(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D) {
  WorkspaceLayout w;
  const size_t bh = mul_sat(static_cast<size_t>(B), static_cast<size_t>(H));
  auto region = [&](int64_t L, int64_t d) {
    const size_t bytes = mul_sat(mul_sat(mul_sat(bh, static_cast<size_t>(L)), static_cast<size_t>(d)), 4);
    return bytes > SIZE_MAX - 255 ? SIZE_MAX : align_up(bytes);
  };
  size_t o = 0;
  w.dq = o;   o = add_sat(o, region(Lq, D));
  w.dk = o;   o = add_sat(o, region(Lk, D));
  w.drow = o; o = add_sat(o, region(Lq, 1));
  w.rowf = o; o = add_sat(o, region(Lq, 1));
  w.total = o;
  return w;
}

int attn_bwd_prologue(const AttnProblem& p, cudaStream_t st) {
  const int64_t nrows = static_cast<int64_t>(p.B) * p.H * p.Lq;
  if (vec_ok(p) && nrows >= p.H) {
    prep_vec_kernel<<<vec_blocks(nrows), 256, 0, st>>>(p);
    return check_launch("prep_vec_kernel");
  }
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
  if (vec_ok(p)) {
    const int64_t nq = static_cast<int64_t>(p.B) * p.H * p.Lq, nk = static_cast<int64_t>(p.B) * p.H * p.Lk;
    if (nq > 0) {
      fix_dq_vec_kernel<<<vec_blocks(nq), 256, 0, st>>>(p);
      const int rc = check_launch("fix_dq_vec_kernel");
      if (rc) return rc;
    }
    if (nk > 0) {
      write_dk_vec_kernel<<<vec_blocks(nk), 256, 0, st>>>(p);
      return check_launch("write_dk_vec_kernel");
    }
    return TAU_DXB_OK;
  }
  switch (p.dtype) {
    case TAU_DXB_F32: return epilogue<float>(p, st);
    case TAU_DXB_BF16: return epilogue<__nv_bfloat16>(p, st);
    default: return epilogue<__half>(p, st);
  }
}

}  // namespace taudxb
