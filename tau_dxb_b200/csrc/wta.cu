// WTA top-k sparsity kernels (K4 forward / K5 backward) for sm_100a.
//
// Forward: one warp per row. A bf16/f16 row of d = 256*CH elements is read
// once with 128-bit loads into registers (CH*4 words per lane), turned into
// order-preserving 16-bit keys, and the k-th largest key is found by a
// two-pass MSB radix select (8-bit digits). Every lane counts its own keys in
// a private column of a [257 bins][32 lanes] u8 histogram in shared memory
// (no atomics, no cross-lane contention); a digit pass ends with one warp
// reduction that locates the digit holding the k-th largest key. The mask is
// then written as bits (1/8 byte per element), y = keep ? x : 0 as bf16, and
// optionally per-column win counts. HBM traffic per element: 2 B read, 2 B
// written (y), 1/8 B mask -- nothing else touches DRAM.
//
// Semantics (reference):
//   threshold -- keep = x >= k-th largest value (echo/triton_wta.py:81-83,46-47;
//                echo/patch_whisper_sparse_grad.py:52-53); ties keep more than k.
//   exact_k   -- exactly k kept (echo/triton_wta.py:117-123); among values equal
//                to the threshold the lowest indices win. y = x * keep as the
//                reference computes it, so a dropped negative value is -0
//                (threshold mode writes +0, like the reference's tl.where).
//   backward  -- dx = dy * keep (echo/triton_wta.py:66-67;
//                echo/patch_whisper_sparse_grad.py:58-60).
// Float comparisons are reproduced on keys: +0 and -0 compare equal.

#include "common.cuh"

namespace taudxb {
namespace {

constexpr int kBins = 257;                   // 256 digit bins + 1 discard bin
constexpr int kHist16Bytes = kBins * 64;     // u16 counters, [bin][lane]
constexpr uint32_t kFull = 0xffffffffu;

__device__ __forceinline__ uint32_t keys16(uint32_t w) {
  const uint32_t s = (w >> 15) & 0x00010001u;          // sign of each half
  return w ^ ((s * 0x7FFFu) | 0x80008000u);
}
__device__ __forceinline__ uint32_t unkeys16(uint32_t kw) {
  const uint32_t s = ((~kw) >> 15) & 0x00010001u;      // 1 where x was negative
  return kw ^ ((s * 0x7FFFu) | 0x80008000u);
}
__device__ __forceinline__ uint32_t key32(uint32_t w) {
  return w ^ ((w & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
}

// Locate the digit bin that holds the k-th largest key, given per-lane
// counters (CT = uint8_t or uint16_t) laid out [bin][lane]. Lane l owns bins
// l + 32*j. Returns the bin and the number of keys in higher bins; clears the
// counters of bins 0..255 it read.
template <typename CT>
__device__ __forceinline__ void select_bin(CT* hist, int lane, int k, int& bstar, int& above_out) {
  uint32_t cnt[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4* p = reinterpret_cast<uint4*>(hist + (lane + 32 * j) * 32);
    uint32_t s = 0;
    if (sizeof(CT) == 1) {
      const uint4 a = p[0], b = p[1];
      s = __dp4a(a.x, 0x01010101u, s); s = __dp4a(a.y, 0x01010101u, s);
      s = __dp4a(a.z, 0x01010101u, s); s = __dp4a(a.w, 0x01010101u, s);
      s = __dp4a(b.x, 0x01010101u, s); s = __dp4a(b.y, 0x01010101u, s);
      s = __dp4a(b.z, 0x01010101u, s); s = __dp4a(b.w, 0x01010101u, s);
      p[0] = make_uint4(0, 0, 0, 0); p[1] = make_uint4(0, 0, 0, 0);
    } else {
      uint32_t acc = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 a = p[q];
        acc += a.x + a.y + a.z + a.w;   // two 16-bit fields, each < 65536
        p[q] = make_uint4(0, 0, 0, 0);
      }
      s = (acc & 0xFFFFu) + (acc >> 16);
    }
    cnt[j] = s;
  }
  int above = 0, jstar = 0;
  bool found = false;
#pragma unroll
  for (int j = 7; j >= 0; --j) {
    const int g = static_cast<int>(__reduce_add_sync(kFull, cnt[j]));
    if (!found) {
      if (above + g >= k) { jstar = j; found = true; }
      else above += g;
    }
  }
  uint32_t c = cnt[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) if (j == jstar) c = cnt[j];
  uint32_t s = c;                                // inclusive suffix sum over lanes
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t t = __shfl_down_sync(kFull, s, off);
    if (lane + off < 32) s += t;
  }
  const uint32_t S = s + static_cast<uint32_t>(above);
  const uint32_t ge = __ballot_sync(kFull, S >= static_cast<uint32_t>(k));
  const int lstar = 31 - __clz(ge);
  const uint32_t S_l = __shfl_sync(kFull, S, lstar);
  const uint32_t c_l = __shfl_sync(kFull, c, lstar);
  bstar = 32 * jstar + lstar;
  above_out = static_cast<int>(S_l - c_l);
}

__device__ __forceinline__ int warp_excl_scan(int v, int lane, int& total) {
  int s = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int t = __shfl_up_sync(kFull, s, off);
    if (lane >= off) s += t;
  }
  total = __shfl_sync(kFull, s, 31);
  return s - v;
}

// ---------------------------------------------------------------------------
// Fast path: 16-bit elements, d = 256 * CH, rows 16-byte aligned.
//
// Counters: per warp a [257 bins][16 words] u32 array; lane l owns the 16-bit
// half (l & 1) of word (l >> 1) in every bin row. Updates are fire-and-forget
// `red.shared.add` (no load-add-store dependency chain through shared memory);
// only the two lanes sharing a word can collide on one address.

__device__ __forceinline__ void red_shared_add(uint32_t addr, uint32_t v) {
  asm volatile("red.shared.add.u32 [%0], %1;" :: "r"(addr), "r"(v) : "memory");
}

// Find the digit bin holding the k-th largest key from u16-pair counters.
// Lane l owns bins l + 32*j; it sums the 16 words of each of its bins (4
// staggered 16-byte loads, conflict-free) and zeroes them.
__device__ __forceinline__ void select_bin_pairs(uint32_t* hist, int lane, int k, int& bstar,
                                                 int& above_out) {
  uint32_t cnt[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4* row = reinterpret_cast<uint4*>(hist + (lane + 32 * j) * 16);
    uint32_t acc = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = (q + (lane >> 1)) & 3;
      const uint4 a = row[c];
      acc += a.x + a.y + a.z + a.w;          // two 16-bit fields, each <= d
      row[c] = make_uint4(0, 0, 0, 0);
    }
    cnt[j] = (acc & 0xFFFFu) + (acc >> 16);
  }
  int above = 0, jstar = 0;
  bool found = false;
#pragma unroll
  for (int j = 7; j >= 0; --j) {
    const int g = static_cast<int>(__reduce_add_sync(kFull, cnt[j]));
    if (!found) {
      if (above + g >= k) { jstar = j; found = true; }
      else above += g;
    }
  }
  uint32_t c = cnt[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) if (j == jstar) c = cnt[j];
  uint32_t s = c;                                // inclusive suffix sum over lanes
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t t = __shfl_down_sync(kFull, s, off);
    if (lane + off < 32) s += t;
  }
  const uint32_t S = s + static_cast<uint32_t>(above);
  const uint32_t ge = __ballot_sync(kFull, S >= static_cast<uint32_t>(k));
  const int lstar = 31 - __clz(ge);
  const uint32_t S_l = __shfl_sync(kFull, S, lstar);
  const uint32_t c_l = __shfl_sync(kFull, c, lstar);
  bstar = 32 * jstar + lstar;
  above_out = static_cast<int>(S_l - c_l);
}

constexpr int kFastWarps = 4;                    // rows in flight per block
constexpr int kPairHistBytes = kBins * 64;       // [257][16] u32 per warp

template <int CH, bool EXACT, bool WRITE_Y, bool HIST>
__global__ void __launch_bounds__(kFastWarps * 32, 3)
wta_fwd16_kernel(const uint16_t* __restrict__ x, int64_t n_rows, int64_t row_stride,
                 int k_host, const int32_t* __restrict__ k_dev,
                 uint16_t* __restrict__ y, uint8_t* __restrict__ bitmask,
                 int32_t* __restrict__ win) {
  constexpr int D = 256 * CH;
  extern __shared__ __align__(16) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + warp * kPairHistBytes);
  int32_t* shist = reinterpret_cast<int32_t*>(smem + kFastWarps * kPairHistBytes);
  for (int i = lane; i < kPairHistBytes / 16; i += 32)
    reinterpret_cast<uint4*>(hist)[i] = make_uint4(0, 0, 0, 0);
  if (HIST)
    for (int i = threadIdx.x; i < D; i += blockDim.x) shist[i] = 0;
  __syncthreads();
  int k = k_dev ? *k_dev : k_host;
  k = max(1, min(D, k));
  // this lane's counter: word (lane >> 1) of a bin row, 16-bit half (lane & 1)
  const uint32_t hbase = static_cast<uint32_t>(__cvta_generic_to_shared(hist)) + (lane >> 1) * 4;
  const uint32_t inc = 1u << ((lane & 1) * 16);

  const int64_t stride_rows = static_cast<int64_t>(gridDim.x) * kFastWarps;
  int64_t row = static_cast<int64_t>(blockIdx.x) * kFastWarps + warp;
  uint4 nxt[CH];
  if (row < n_rows) {
    const uint4* src = reinterpret_cast<const uint4*>(x + row * row_stride);
#pragma unroll
    for (int c = 0; c < CH; ++c) nxt[c] = __ldcs(src + c * 32 + lane);
  }
  for (; row < n_rows; row += stride_rows) {
    uint32_t kw[CH][4];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      kw[c][0] = keys16(nxt[c].x); kw[c][1] = keys16(nxt[c].y);
      kw[c][2] = keys16(nxt[c].z); kw[c][3] = keys16(nxt[c].w);
    }
    // prefetch the next row while this one is selected
    const int64_t nrow = row + stride_rows;
    if (nrow < n_rows) {
      const uint4* src = reinterpret_cast<const uint4*>(x + nrow * row_stride);
#pragma unroll
      for (int c = 0; c < CH; ++c) nxt[c] = __ldcs(src + c * 32 + lane);
    }
    // pass 1: high byte of every key
#pragma unroll
    for (int c = 0; c < CH; ++c)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t w = kw[c][i];
        red_shared_add(hbase + __byte_perm(w, 0, 0x4441) * 64, inc);
        red_shared_add(hbase + (w >> 24) * 64, inc);
      }
    __syncwarp();
    int b1, above1;
    select_bin_pairs(hist, lane, k, b1, above1);
    __syncwarp();
    // pass 2: low byte of keys whose high byte is b1; others go to bin 256
    const uint32_t hb2 = (static_cast<uint32_t>(b1) << 8) | (static_cast<uint32_t>(b1) << 24);
#pragma unroll
    for (int c = 0; c < CH; ++c)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t xw = kw[c][i] ^ hb2;            // matching keys -> high byte 0
        red_shared_add(hbase + min(xw & 0xFFFFu, 256u) * 64, inc);
        red_shared_add(hbase + min(xw >> 16, 256u) * 64, inc);
      }
    __syncwarp();
    int b2, above2;
    select_bin_pairs(hist, lane, k - above1, b2, above2);
    __syncwarp();
    const uint32_t t = (static_cast<uint32_t>(b1) << 8) | static_cast<uint32_t>(b2);
    uint32_t tlo = t, thi = t;
    if (t == 0x8000u || t == 0x7FFFu) { tlo = 0x7FFFu; thi = 0x8000u; }   // +0 == -0

    int need = 0, rank_base = 0;
    if (EXACT) {
      int gt = 0;
#pragma unroll
      for (int c = 0; c < CH; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          gt += ((kw[c][i] & 0xFFFFu) > thi) + ((kw[c][i] >> 16) > thi);
      need = k - static_cast<int>(__reduce_add_sync(kFull, static_cast<uint32_t>(gt)));
    }
    uint8_t* mrow = bitmask + row * (D / 8);
    uint4* yrow = WRITE_Y ? reinterpret_cast<uint4*>(y + row * static_cast<int64_t>(D)) : nullptr;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      uint32_t bits = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = kw[c][i] & 0xFFFFu, hi = kw[c][i] >> 16;
        if (EXACT) {
          bits |= static_cast<uint32_t>(lo > thi) << (2 * i);
          bits |= static_cast<uint32_t>(hi > thi) << (2 * i + 1);
        } else {
          bits |= static_cast<uint32_t>(lo >= tlo) << (2 * i);
          bits |= static_cast<uint32_t>(hi >= tlo) << (2 * i + 1);
        }
      }
      if (EXACT) {
        uint32_t tie = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t lo = kw[c][i] & 0xFFFFu, hi = kw[c][i] >> 16;
          tie |= static_cast<uint32_t>(lo >= tlo && lo <= thi) << (2 * i);
          tie |= static_cast<uint32_t>(hi >= tlo && hi <= thi) << (2 * i + 1);
        }
        int total;
        int r = rank_base + warp_excl_scan(__popc(tie), lane, total);
        rank_base += total;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if ((tie >> e) & 1u) { if (r < need) bits |= 1u << e; ++r; }
      }
      mrow[c * 32 + lane] = static_cast<uint8_t>(bits);
      if (WRITE_Y) {
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint32_t sel = (((bits >> (2 * i)) & 1u) ? 0x0000FFFFu : 0u) |
                         (((bits >> (2 * i + 1)) & 1u) ? 0xFFFF0000u : 0u);
          if (EXACT) sel |= 0x80008000u;   // x * 0 keeps the sign
          o[i] = unkeys16(kw[c][i]) & sel;
        }
        __stcs(yrow + c * 32 + lane, make_uint4(o[0], o[1], o[2], o[3]));
      }
      if (HIST) {
        const int col0 = (c * 32 + lane) * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if ((bits >> e) & 1u) atomicAdd(&shist[col0 + e], 1);
      }
    }
  }
  if (HIST) {
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x)
      if (shist[i]) atomicAdd(&win[i], shist[i]);
  }
}

// ---------------------------------------------------------------------------
// Generic path: any d < 65536, any supported dtype, any row stride. One warp
// per row; the row is re-read (L1/L2) for every digit pass.
template <typename T>
__device__ __forceinline__ uint32_t load_key(const T* p);
template <> __device__ __forceinline__ uint32_t load_key<uint16_t>(const uint16_t* p) {
  return keys16(static_cast<uint32_t>(*p)) & 0xFFFFu;
}
template <> __device__ __forceinline__ uint32_t load_key<uint32_t>(const uint32_t* p) {
  return key32(*p);
}

template <typename T>
__global__ void __launch_bounds__(4 * 32)
wta_fwd_generic_kernel(const T* __restrict__ x, int64_t n_rows, int d, int64_t row_stride,
                       int k_host, const int32_t* __restrict__ k_dev, int exact,
                       T* __restrict__ y, uint8_t* __restrict__ bitmask,
                       int32_t* __restrict__ win) {
  constexpr int KB = sizeof(T) * 8;  // key bits
  extern __shared__ __align__(16) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint16_t* hist = reinterpret_cast<uint16_t*>(smem + warp * kHist16Bytes);
  for (int i = lane; i < kHist16Bytes / 16; i += 32)
    reinterpret_cast<uint4*>(hist)[i] = make_uint4(0, 0, 0, 0);
  __syncwarp();
  int k = k_dev ? *k_dev : k_host;
  k = max(1, min(d, k));
  const int64_t mbytes = (d + 7) / 8;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * 4 + warp; row < n_rows;
       row += static_cast<int64_t>(gridDim.x) * 4) {
    const T* xr = x + row * row_stride;
    uint32_t prefix = 0;
    int kk = k;
    for (int p = 0; p < KB / 8; ++p) {
      const int shift = KB - 8 * (p + 1);
      for (int j = lane; j < d; j += 32) {
        const uint32_t key = load_key(xr + j);
        const bool match = (p == 0) || ((key >> (shift + 8)) == prefix);
        const uint32_t bin = match ? ((key >> shift) & 0xFFu) : 256u;
        hist[bin * 32 + lane] += 1;
      }
      __syncwarp();
      int b, above;
      select_bin(hist, lane, kk, b, above);
      __syncwarp();
      prefix = (prefix << 8) | static_cast<uint32_t>(b);
      kk -= above;
    }
    const uint32_t t = prefix;
    uint32_t tlo = t, thi = t;
    const uint32_t pz = (KB == 16) ? 0x8000u : 0x80000000u, nz = pz - 1u;
    if (t == pz || t == nz) { tlo = nz; thi = pz; }
    int need = 0;
    if (exact) {
      int gt = 0;
      for (int j = lane; j < d; j += 32) gt += load_key(xr + j) > thi;
      need = k - static_cast<int>(__reduce_add_sync(kFull, static_cast<uint32_t>(gt)));
    }
    int rank = 0;
    uint8_t* mrow = bitmask + row * mbytes;
    for (int j0 = 0; j0 < d; j0 += 32) {
      const int j = j0 + lane;
      bool keep = false;
      if (j < d) {
        const uint32_t key = load_key(xr + j);
        keep = exact ? (key > thi) : (key >= tlo);
        const bool tie = exact && key >= tlo && key <= thi;
        const uint32_t tb = __ballot_sync(__activemask(), tie);
        if (tie) keep = (rank + __popc(tb & ((1u << lane) - 1u))) < need;
        rank += __popc(tb);
        if (y) {
          const T sign_only = static_cast<T>(xr[j] & (T(1) << (KB - 1)));
          y[row * static_cast<int64_t>(d) + j] = keep ? xr[j] : (exact ? sign_only : T(0));
        }
        if (win && keep) atomicAdd(&win[j], 1);
      }
      const uint32_t kb = __ballot_sync(kFull, keep);
      // lanes 0..3 write the 4 mask bytes of this 32-element group
      if (lane < 4 && j0 / 8 + lane < mbytes) mrow[j0 / 8 + lane] = static_cast<uint8_t>(kb >> (8 * lane));
    }
  }
}

// ---------------------------------------------------------------------------
// Backward: dx = dy * keep, 8 elements per mask byte.
template <typename T>
__global__ void __launch_bounds__(256)
wta_bwd_vec_kernel(const T* __restrict__ dy, const uint8_t* __restrict__ mask,
                   T* __restrict__ dx, int64_t n_bytes) {
  constexpr int V = 16 / sizeof(T);          // elements per 16-byte vector
  constexpr int NV = 8 / V;                  // vectors per mask byte
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_bytes;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t m = mask[i];
    const uint4* src = reinterpret_cast<const uint4*>(dy) + i * NV;
    uint4* dst = reinterpret_cast<uint4*>(dx) + i * NV;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      uint4 raw = __ldcs(src + v);
      T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float f = Elem<T>::to_f(e[j]) * (((m >> (v * V + j)) & 1u) ? 1.f : 0.f);
        e[j] = Elem<T>::from_f(f);
      }
      __stcs(dst + v, raw);
    }
  }
}

template <typename T>
__global__ void wta_bwd_generic_kernel(const T* __restrict__ dy, const uint8_t* __restrict__ mask,
                                       T* __restrict__ dx, int64_t n_rows, int64_t d) {
  const int64_t total = n_rows * d, mbytes = (d + 7) / 8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / d, c = i - r * d;
    const uint32_t bit = (mask[r * mbytes + c / 8] >> (c % 8)) & 1u;
    dx[i] = Elem<T>::from_f(Elem<T>::to_f(dy[i]) * (bit ? 1.f : 0.f));
  }
}

__global__ void k_from_logits_kernel(const float* __restrict__ logits, int64_t n, int64_t d_ff,
                                     int32_t* __restrict__ k_out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float s = 1.f / (1.f + expf(-logits[i]));
  const double v = rint(static_cast<double>(s) * static_cast<double>(d_ff));  // half-even
  int64_t k = static_cast<int64_t>(v);
  k = k < 1 ? 1 : (k > d_ff ? d_ff : k);
  k_out[i] = static_cast<int32_t>(k);
}

template <int CH, bool EXACT, bool WRITE_Y, bool HIST>
int launch_fwd16(const void* x, int64_t n_rows, int64_t row_stride, int k, const int32_t* k_dev,
                 void* y, uint8_t* bitmask, int32_t* win, cudaStream_t st) {
  auto kern = wta_fwd16_kernel<CH, EXACT, WRITE_Y, HIST>;
  const size_t smem = kFastWarps * kPairHistBytes + (HIST ? 256 * CH * 4 : 0);
  TDX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  TDX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kFastWarps * 32, smem));
  per_sm = per_sm < 1 ? 1 : per_sm;
  int64_t blocks = (n_rows + kFastWarps - 1) / kFastWarps;
  const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
  if (blocks > cap) blocks = cap;
  kern<<<static_cast<unsigned>(blocks), kFastWarps * 32, smem, st>>>(
      static_cast<const uint16_t*>(x), n_rows, row_stride, k, k_dev,
      static_cast<uint16_t*>(y), bitmask, win);
  return check_launch("wta_fwd16_kernel");
}

template <int CH>
int dispatch_fwd16(const void* x, int64_t n_rows, int64_t row_stride, int k, const int32_t* k_dev,
                   int mode, void* y, uint8_t* bitmask, int32_t* win, cudaStream_t st) {
  const bool exact = mode == TAU_DXB_WTA_EXACT_K, wy = y != nullptr, h = win != nullptr;
#define TDX_WTA_CASE(E, W, H)                                                        \
  if (exact == E && wy == W && h == H)                                               \
    return launch_fwd16<CH, E, W, H>(x, n_rows, row_stride, k, k_dev, y, bitmask, win, st);
  TDX_WTA_CASE(false, true, false) TDX_WTA_CASE(false, false, false)
  TDX_WTA_CASE(false, true, true)  TDX_WTA_CASE(false, false, true)
  TDX_WTA_CASE(true, true, false)  TDX_WTA_CASE(true, false, false)
  TDX_WTA_CASE(true, true, true)   TDX_WTA_CASE(true, false, true)
#undef TDX_WTA_CASE
  return fail(TAU_DXB_ERR_UNSUPPORTED, "wta_fwd: no kernel for this mode");
}

}  // namespace

int wta_fwd_impl(const void* x, int32_t dtype, int64_t n_rows, int64_t d, int64_t row_stride,
                 int64_t k, const int32_t* k_dev, int32_t mode, void* y, uint8_t* bitmask,
                 int32_t* win, cudaStream_t st) {
  TDX_CHECK_ARG(n_rows >= 0 && d >= 1 && d < 65536, "wta_fwd: need 0 <= n_rows, 1 <= d < 65536 (d=%lld)", (long long)d);
  if (n_rows == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(x && bitmask, "wta_fwd: x and bitmask are required");
  TDX_CHECK_ARG(row_stride >= d, "wta_fwd: row_stride (%lld) < d (%lld)", (long long)row_stride, (long long)d);
  TDX_CHECK_ARG(mode == TAU_DXB_WTA_THRESHOLD || mode == TAU_DXB_WTA_EXACT_K, "wta_fwd: bad mode %d", mode);
  TDX_CHECK_ARG(dtype == TAU_DXB_F32 || dtype == TAU_DXB_BF16 || dtype == TAU_DXB_F16, "wta_fwd: bad dtype %d", dtype);
  const int kk = static_cast<int>(k < 1 ? 1 : (k > d ? d : k));
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (row_stride % 8 == 0) &&
                       (!y || reinterpret_cast<uintptr_t>(y) % 16 == 0);
  if (dtype != TAU_DXB_F32 && aligned && d % 256 == 0) {
    switch (d / 256) {
      case 3:  return dispatch_fwd16<3>(x, n_rows, row_stride, kk, k_dev, mode, y, bitmask, win, st);
      case 4:  return dispatch_fwd16<4>(x, n_rows, row_stride, kk, k_dev, mode, y, bitmask, win, st);
      case 6:  return dispatch_fwd16<6>(x, n_rows, row_stride, kk, k_dev, mode, y, bitmask, win, st);
      case 8:  return dispatch_fwd16<8>(x, n_rows, row_stride, kk, k_dev, mode, y, bitmask, win, st);
      case 12: return dispatch_fwd16<12>(x, n_rows, row_stride, kk, k_dev, mode, y, bitmask, win, st);
      case 16: return dispatch_fwd16<16>(x, n_rows, row_stride, kk, k_dev, mode, y, bitmask, win, st);
      default: break;
    }
  }
  const size_t smem = 4 * kHist16Bytes;
  int64_t blocks = (n_rows + 3) / 4;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  const int exact = mode == TAU_DXB_WTA_EXACT_K;
  if (dtype == TAU_DXB_F32) {
    auto kern = wta_fwd_generic_kernel<uint32_t>;
    TDX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<static_cast<unsigned>(blocks), 128, smem, st>>>(
        static_cast<const uint32_t*>(x), n_rows, static_cast<int>(d), row_stride, kk, k_dev, exact,
        static_cast<uint32_t*>(y), bitmask, win);
  } else {
    auto kern = wta_fwd_generic_kernel<uint16_t>;
    TDX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<static_cast<unsigned>(blocks), 128, smem, st>>>(
        static_cast<const uint16_t*>(x), n_rows, static_cast<int>(d), row_stride, kk, k_dev, exact,
        static_cast<uint16_t*>(y), bitmask, win);
  }
  return check_launch("wta_fwd_generic_kernel");
}

int wta_bwd_impl(const void* dy, int32_t dtype, const uint8_t* bitmask, int64_t n_rows, int64_t d,
                 void* dx, cudaStream_t st) {
  TDX_CHECK_ARG(n_rows >= 0 && d >= 1, "wta_bwd: bad shape");
  if (n_rows == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(dy && bitmask && dx, "wta_bwd: dy, bitmask and dx are required");
  TDX_CHECK_ARG(dtype == TAU_DXB_F32 || dtype == TAU_DXB_BF16 || dtype == TAU_DXB_F16, "wta_bwd: bad dtype %d", dtype);
  const bool aligned = reinterpret_cast<uintptr_t>(dy) % 16 == 0 && reinterpret_cast<uintptr_t>(dx) % 16 == 0;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (d % 8 == 0 && aligned) {
    const int64_t n_bytes = n_rows * d / 8;
    int64_t blocks = (n_bytes + 255) / 256;
    if (blocks > cap) blocks = cap;
    if (dtype == TAU_DXB_F32)
      wta_bwd_vec_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const float*>(dy), bitmask, static_cast<float*>(dx), n_bytes);
    else if (dtype == TAU_DXB_BF16)
      wta_bwd_vec_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(dy), bitmask, static_cast<__nv_bfloat16*>(dx), n_bytes);
    else
      wta_bwd_vec_kernel<__half><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const __half*>(dy), bitmask, static_cast<__half*>(dx), n_bytes);
    return check_launch("wta_bwd_vec_kernel");
  }
  int64_t blocks = (n_rows * d + 255) / 256;
  if (blocks > cap) blocks = cap;
  if (dtype == TAU_DXB_F32)
    wta_bwd_generic_kernel<float><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const float*>(dy), bitmask, static_cast<float*>(dx), n_rows, d);
  else if (dtype == TAU_DXB_BF16)
    wta_bwd_generic_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(dy), bitmask, static_cast<__nv_bfloat16*>(dx), n_rows, d);
  else
    wta_bwd_generic_kernel<__half><<<(unsigned)blocks, 256, 0, st>>>(static_cast<const __half*>(dy), bitmask, static_cast<__half*>(dx), n_rows, d);
  return check_launch("wta_bwd_generic_kernel");
}

int wta_k_from_logits_impl(const float* logits, int64_t n, int64_t d_ff, int32_t* k_out,
                           cudaStream_t st) {
  TDX_CHECK_ARG(logits && k_out && n >= 0 && d_ff >= 1, "wta_k_from_logits: bad arguments");
  if (n == 0) return TAU_DXB_OK;
  k_from_logits_kernel<<<static_cast<unsigned>((n + 127) / 128), 128, 0, st>>>(logits, n, d_ff, k_out);
  return check_launch("k_from_logits_kernel");
}

}  // namespace taudxb
