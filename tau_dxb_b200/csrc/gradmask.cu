// Soft-prune gradient masks of the FFN weights: out = grad * keep, with keep a
// 0/1 byte per FFN neuron applied along the rows (fc1.weight [d_ff, d_model],
// fc1.bias [d_ff]) or along the columns (fc2.weight [d_model, d_ff]) -- the
// gradient hooks of echo/patch_whisper_sparse_grad.py:167-194 in one pass over
// the gradient, reading the keep bytes directly (no float copy of the mask).
// The product is a multiply by 1.0 / 0.0 in the gradient's type, as in the
// reference, so a non-finite gradient under a 0 stays NaN. HBM-bound: the
// gradient is read and written once with 16-byte accesses where aligned.

#include "common.cuh"

namespace taudxb {
namespace {

template <typename T> struct Vec;
template <> struct Vec<float> { static constexpr int N = 4; };
template <> struct Vec<__nv_bfloat16> { static constexpr int N = 8; };
template <> struct Vec<__half> { static constexpr int N = 8; };

// rows x cols row-major, cols % Vec<T>::N == 0 and 16-byte aligned pointers:
// one 16-byte vector per thread and grid-stride loop
template <typename T, bool COLS>
__global__ void __launch_bounds__(256) grad_mask_vec_kernel(const T* __restrict__ g, int64_t rows, int64_t cols,
                                                            const uint8_t* __restrict__ keep, T* __restrict__ out) {
  constexpr int V = Vec<T>::N;
  const int64_t vcols = cols / V;
  const int64_t n = rows * vcols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vcols, c0 = (i - r * vcols) * V;
    uint4 w = __ldcs(reinterpret_cast<const uint4*>(g) + i);
    T* e = reinterpret_cast<T*>(&w);
    if (COLS) {
#pragma unroll
      for (int u = 0; u < V; ++u) {
        const float kf = keep[c0 + u] ? 1.f : 0.f;
        e[u] = Elem<T>::from_f(Elem<T>::to_f(e[u]) * kf);
      }
    } else {
      const float kf = keep[r] ? 1.f : 0.f;
#pragma unroll
      for (int u = 0; u < V; ++u) e[u] = Elem<T>::from_f(Elem<T>::to_f(e[u]) * kf);
    }
    __stcs(reinterpret_cast<uint4*>(out) + i, w);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) grad_mask_kernel(const T* __restrict__ g, int64_t rows, int64_t cols, int axis,
                                                        const uint8_t* __restrict__ keep, T* __restrict__ out) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const float kf = keep[axis ? c : r] ? 1.f : 0.f;
    out[i] = Elem<T>::from_f(Elem<T>::to_f(g[i]) * kf);
  }
}

template <typename T>
int launch_grad_mask(const void* g, int64_t rows, int64_t cols, const uint8_t* keep, int axis, void* out,
                     cudaStream_t st) {
  constexpr int V = Vec<T>::N;
  const bool vec = cols % V == 0 && reinterpret_cast<uintptr_t>(g) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out) % 16 == 0;
  const int64_t work = vec ? rows * (cols / V) : rows * cols;
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const T* gp = static_cast<const T*>(g);
  T* op = static_cast<T*>(out);
  if (vec) {
    if (axis) grad_mask_vec_kernel<T, true><<<static_cast<unsigned>(blocks), 256, 0, st>>>(gp, rows, cols, keep, op);
    else grad_mask_vec_kernel<T, false><<<static_cast<unsigned>(blocks), 256, 0, st>>>(gp, rows, cols, keep, op);
    return check_launch("grad_mask_vec_kernel");
  }
  grad_mask_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, st>>>(gp, rows, cols, axis, keep, op);
  return check_launch("grad_mask_kernel");
}

}  // namespace

int grad_mask_impl(const void* g, int32_t dtype, int64_t rows, int64_t cols, const uint8_t* keep, int32_t axis,
                   void* out, cudaStream_t st) {
  TDX_CHECK_ARG(rows >= 0 && cols >= 0, "tau_grad_mask: negative shape");
  TDX_CHECK_ARG(axis == 0 || axis == 1, "tau_grad_mask: axis must be 0 (rows) or 1 (columns)");
  TDX_CHECK_ARG(dtype == TAU_DXB_F32 || dtype == TAU_DXB_BF16 || dtype == TAU_DXB_F16, "tau_grad_mask: bad dtype %d",
                dtype);
  if (rows == 0 || cols == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(g && keep && out, "tau_grad_mask: null pointer");
  switch (dtype) {
    case TAU_DXB_F32: return launch_grad_mask<float>(g, rows, cols, keep, axis, out, st);
    case TAU_DXB_BF16: return launch_grad_mask<__nv_bfloat16>(g, rows, cols, keep, axis, out, st);
    default: return launch_grad_mask<__half>(g, rows, cols, keep, axis, out, st);
  }
}

}  // namespace taudxb
