// Column sums of a row-major [M, N] bf16 / fp32 matrix: the bias gradient of a
// linear layer, db[n] = sum_m dy[m, n]. HBM-bound: every element is read once
// with 16-byte loads, fp32 accumulation.
//
// Stage 1: CTA (column tile of 256 columns, row split) of 8 warps; each lane
// owns 8 columns of the tile (bf16) and walks rows r = split_lo + warp,
// + 8, ...; the 8 warps add theirs through shared memory in a fixed order into
// one fp32 partial row per split. Stage 2 adds the partial rows of each
// column in a fixed order. Same bits on every call.

#include "common.cuh"

namespace taudxb {
namespace {

constexpr int kCsWarps = 8;
constexpr int kCsCols = 256;           // columns per CTA (8 per lane)

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldcs(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
  const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
  const float4 b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <typename T>
__global__ void __launch_bounds__(kCsWarps * 32)
colsum_partial_kernel(const T* __restrict__ x, int64_t M, int N, int64_t rows_per_split,
                      float* __restrict__ part) {
  __shared__ float red[kCsWarps][kCsCols];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col0 = blockIdx.x * kCsCols + lane * 8;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * rows_per_split;
  const int64_t r1 = r0 + rows_per_split < M ? r0 + rows_per_split : M;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (col0 < N) {
    int64_t r = r0 + warp;
    // two rows in flight per warp
    for (; r + kCsWarps < r1; r += 2 * kCsWarps) {
      float a[8], b[8];
      load8<T>(x + r * N + col0, a);
      load8<T>(x + (r + kCsWarps) * N + col0, b);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += a[i] + b[i];
    }
    if (r < r1) {
      float a[8];
      load8<T>(x + r * N + col0, a);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += a[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) red[warp][lane * 8 + i] = acc[i];
  __syncthreads();
  for (int c = threadIdx.x; c < kCsCols; c += kCsWarps * 32) {
    const int col = blockIdx.x * kCsCols + c;
    if (col >= N) continue;
    float s = red[0][c];
#pragma unroll
    for (int w = 1; w < kCsWarps; ++w) s += red[w][c];
    part[static_cast<int64_t>(blockIdx.y) * N + col] = s;
  }
}

// Stage 2: a CTA takes 32 columns; its 8 warps each sum a contiguous range of
// the partial rows (lane = column, coalesced loads, four add chains), then
// warp 0 adds the 8 sums in warp order -- a fixed order.
constexpr int kCsRedWarps = 8;
template <typename T>
__global__ void __launch_bounds__(kCsRedWarps * 32)
colsum_final_kernel(const float* __restrict__ part, int splits, int N, T* __restrict__ out) {
  __shared__ float red[kCsRedWarps][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  const int per = (splits + kCsRedWarps - 1) / kCsRedWarps;
  const int k0 = warp * per, k1 = k0 + per < splits ? k0 + per : splits;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (col < N) {
    int k = k0;
    for (; k + 3 < k1; k += 4) {
      s0 += part[static_cast<int64_t>(k) * N + col];
      s1 += part[static_cast<int64_t>(k + 1) * N + col];
      s2 += part[static_cast<int64_t>(k + 2) * N + col];
      s3 += part[static_cast<int64_t>(k + 3) * N + col];
    }
    for (; k < k1; ++k) s0 += part[static_cast<int64_t>(k) * N + col];
  }
  red[warp][lane] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (warp == 0 && col < N) {
    float t = red[0][lane];
#pragma unroll
    for (int w = 1; w < kCsRedWarps; ++w) t += red[w][lane];
    out[col] = Elem<T>::from_f(t);
  }
}

void colsum_shape(int64_t M, int64_t N, int* splits, int64_t* rows_per_split) {
  const int64_t tiles = (N + kCsCols - 1) / kCsCols;
  int64_t want = (4ll * sm_count() + tiles - 1) / tiles;      // ~4 CTAs per SM
  const int64_t max_by_rows = (M + 4 * kCsWarps - 1) / (4 * kCsWarps);   // >= 4 rows per warp
  if (want > max_by_rows) want = max_by_rows;
  if (want < 1) want = 1;
  if (want > 65535) want = 65535;
  *rows_per_split = (M + want - 1) / want;
  *splits = static_cast<int>((M + *rows_per_split - 1) / *rows_per_split);
}

}  // namespace

size_t column_sum_workspace(int64_t M, int64_t N) {
  if (M <= 0 || N <= 0) return 0;
  int splits = 0;
  int64_t rps = 0;
  colsum_shape(M, N, &splits, &rps);
  return static_cast<size_t>(splits) * static_cast<size_t>(N) * sizeof(float);
}

int column_sum_impl(const void* x, int32_t dtype, int64_t M, int64_t N, void* out, int32_t out_dtype,
                    void* workspace, size_t workspace_bytes, cudaStream_t st) {
  TDX_CHECK_ARG(dtype == TAU_DXB_BF16 || dtype == TAU_DXB_F32, "column sum: x must be bf16 or fp32");
  TDX_CHECK_ARG(out_dtype == TAU_DXB_BF16 || out_dtype == TAU_DXB_F32, "column sum: out must be bf16 or fp32");
  TDX_CHECK_ARG(M >= 0 && N > 0 && N % 8 == 0 && N < (1ll << 31), "column sum: need N a multiple of 8 (got %lld)",
                (long long)N);
  TDX_CHECK_ARG(out, "column sum: null pointer");
  if (M == 0) {
    TDX_CUDA(cudaMemsetAsync(out, 0, N * (out_dtype == TAU_DXB_F32 ? 4 : 2), st));
    return TAU_DXB_OK;
  }
  TDX_CHECK_ARG(x && workspace, "column sum: null pointer");
  TDX_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(workspace) & 3) == 0,
                "column sum: x must be 16-byte aligned");
  const size_t need = column_sum_workspace(M, N);
  if (workspace_bytes < need)
    return fail(TAU_DXB_ERR_WORKSPACE, "column sum: workspace of %zu bytes, need %zu", workspace_bytes, need);
  int splits = 0;
  int64_t rps = 0;
  colsum_shape(M, N, &splits, &rps);
  float* part = static_cast<float*>(workspace);
  const dim3 grid(static_cast<unsigned>((N + kCsCols - 1) / kCsCols), static_cast<unsigned>(splits));
  if (dtype == TAU_DXB_BF16)
    colsum_partial_kernel<__nv_bfloat16><<<grid, kCsWarps * 32, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), M, static_cast<int>(N), rps, part);
  else
    colsum_partial_kernel<float><<<grid, kCsWarps * 32, 0, st>>>(static_cast<const float*>(x), M,
                                                                  static_cast<int>(N), rps, part);
  int rc = check_launch("colsum_partial_kernel");
  if (rc) return rc;
  const int blocks = static_cast<int>((N + 31) / 32);
  if (out_dtype == TAU_DXB_BF16)
    colsum_final_kernel<__nv_bfloat16><<<blocks, kCsRedWarps * 32, 0, st>>>(part, splits, static_cast<int>(N),
                                                                             static_cast<__nv_bfloat16*>(out));
  else
    colsum_final_kernel<float><<<blocks, kCsRedWarps * 32, 0, st>>>(part, splits, static_cast<int>(N),
                                                                     static_cast<float*>(out));
  return check_launch("colsum_final_kernel");
}

}  // namespace taudxb
