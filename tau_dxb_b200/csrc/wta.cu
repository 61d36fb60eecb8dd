// WTA top-k sparsity kernels (K4 forward / K5 backward) for sm_100a.
//
// Forward, fast path (bf16/f16 rows of d = 256*CH, 16-byte aligned): one warp
// per row, read once with 128-bit loads into registers (CH*4 words per lane).
// The k-th largest value is found by a search over the ordered 16-bit value
// space whose probe, count(x >= v), is one packed bf16x2/f16x2 compare per two
// elements plus a warp reduction -- registers only, no shared memory. Each
// warp starts its search at the threshold of the row it did before. The mask
// is written as bits (1/8 byte per element), y = keep ? x : 0 as bf16, and
// optionally per-column win counts. HBM traffic per element: 2 B read, 2 B
// written (y), 1/8 B mask -- nothing else touches DRAM.
// Generic path (fp32, other widths, unaligned rows): two-pass MSB radix
// select (8-bit digits) over order-preserving keys with per-lane shared-memory
// counters.
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
// Fast path: 16-bit floats (bf16 / f16), d = 256 * CH, rows 16-byte aligned.
//
// One warp per row, the row held in registers (CH x 16 bytes per lane). The
// k-th largest value t is found by a search over the ordered 16-bit value
// space, with no shared memory: count_ge(v) = #{x >= v} costs one packed
// compare per two elements (set.ge.u32.{bf16x2,f16x2} gives 0xFFFF per true
// half) and one subtraction into a register accumulator, then one warp
// reduction. The search starts at the threshold of the row this warp did
// before (rows of one activation tensor are alike) -- for a warp's first row,
// the threshold its slot ended on in the previous launch -- probes once at the
// distance the count there suggests (the count difference times the keys per
// unit of count seen on earlier rows), gallops away from the bracket edge that
// probe set, then bisects; without a start it bisects the whole range.
//
// The compares are float compares, as in the reference: +0 == -0. The search
// counts NaN as larger than everything (set.geu), as torch.topk / kthvalue
// order it, so with n NaN in a row t is the (k - n)-th largest non-NaN value;
// the mask compare x >= t is ordered, so NaN is never kept, and a row with
// n >= k keeps nothing (the reference's threshold is then NaN).

// Bit pattern of the 16-bit float whose order-preserving key (keys16) is `key`.
__device__ __forceinline__ uint32_t key_to_bits16(uint32_t key) {
  return key ^ ((key & 0x8000u) ? 0x8000u : 0xFFFFu);
}

template <bool BF>
__device__ __forceinline__ uint32_t cmp_ge2(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (BF) asm("set.ge.u32.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("set.ge.u32.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// x >= v or unordered: NaN counts as larger than every value (torch's order)
template <bool BF>
__device__ __forceinline__ uint32_t cmp_geu2(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (BF) asm("set.geu.u32.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("set.geu.u32.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <bool BF>
__device__ __forceinline__ uint32_t cmp_gt2(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (BF) asm("set.gt.u32.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("set.gt.u32.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <bool BF>
__device__ __forceinline__ uint32_t cmp_eq2(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (BF) asm("set.eq.u32.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else asm("set.eq.u32.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// acc - m as an integer multiply-add by a register holding -1 (neg1, not a
// compile-time constant, so it stays a multiply-add): the packed compares
// occupy the ALU pipe, the accumulation goes to the FMA pipe.
__device__ __forceinline__ uint32_t sub_mad(uint32_t acc, uint32_t m, uint32_t neg1) {
  uint32_t r;
  asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(m), "r"(neg1), "r"(acc));
  return r;
}

// Sum of packed compare masks: subtracting a mask m = 0xFFFF*l + 0xFFFF0000*h
// adds l - 65536*(l - h) (mod 2^32), so a sum S over words (and lanes) holds
// L = S mod 65536 true low halves and (S - L) / 65536 = H - L; exact while
// L < 65536 and |H - L| < 32768 (d <= 4096 here).
__device__ __forceinline__ int decode_mask_sum(uint32_t s) {
  const uint32_t lo = s & 0xFFFFu;
  return static_cast<int>(2u * lo) + (static_cast<int>(s - lo) >> 16);
}

// Mask byte of 8 consecutive elements from the 4 packed masks of one lane's
// 16-byte chunk: bit 2i <- low half of m_i, bit 2i+1 <- high half.
__device__ __forceinline__ uint32_t mask_byte(uint32_t m0, uint32_t m1, uint32_t m2, uint32_t m3) {
  const uint32_t t = (m0 & 0x00010001u) | ((m1 & 0x00010001u) << 2) | ((m2 & 0x00010001u) << 4) |
                     ((m3 & 0x00010001u) << 6);
  return (t | (t >> 15)) & 0xFFu;
}

constexpr int kFastWarps = 4;                    // rows in flight per block
constexpr uint32_t kGallopMax = 64;

// Search warm start across launches: the threshold key each warp of the fast
// kernel ended on, and its estimate of keys per unit of count near the
// threshold, kept per (block, warp) slot. The next launch starts each warp's
// first row from its slot instead of bisecting the whole key range. A slot
// only says where a search begins -- the bracket search below is exact from
// any start -- so launches that race on a slot (two streams) still give exact
// results. The tag in bits 16+ keeps bf16 and f16 key spaces apart.
constexpr int kHintSlots = 8192;
__device__ uint32_t g_wta_hint_key[kHintSlots];
__device__ float g_wta_hint_ipc[kHintSlots];

template <bool B> struct BoolC { static constexpr bool value = B; };

// GELU (erf form) as PyTorch's CUDA kernels evaluate it for bf16 tensors: fp32
// math, y = (x * 0.5) * (1 + erf(x / sqrt(2))); gradient dy * (cdf + x * pdf)
// with cdf = 0.5 (1 + erf(x / sqrt(2))), pdf = exp(-x^2 / 2) / sqrt(2 pi)
__device__ __forceinline__ float gelu_erf(float x) {
  constexpr float kAlpha = static_cast<float>(0.70710678118654752440);
  return x * 0.5f * (1.f + erff(x * kAlpha));
}
__device__ __forceinline__ float gelu_erf_grad(float dy, float x) {
  constexpr float kAlpha = static_cast<float>(0.70710678118654752440);
  constexpr float kBeta = static_cast<float>(1.12837916709551257390 * 0.70710678118654752440 * 0.5);
  const float cdf = 0.5f * (1.f + erff(x * kAlpha));
  const float pdf = expf(-0.5f * x * x) * kBeta;
  return dy * (cdf + x * pdf);
}
// two bf16 in a word -> gelu of each, rounded to nearest even
__device__ __forceinline__ uint32_t gelu_bf16x2(uint32_t w) {
  const __nv_bfloat162 r = __floats2bfloat162_rn(gelu_erf(__uint_as_float(w << 16)),
                                                 gelu_erf(__uint_as_float(w & 0xffff0000u)));
  return *reinterpret_cast<const uint32_t*>(&r);
}

// Blocks per SM the register budget is sized for: two rows (this one and the
// prefetched next) take 8*CH registers per thread.
// Without the prefetch (PF = false: launches with few rows per warp, where a
// prefetch has little to overlap) one row takes 4*CH registers, so more warps
// fit per SM to hide the search's dependent probes.
template <int CH, bool HIST, bool GELU = false, bool PF = true>
constexpr int fwd16_min_blocks() {
  return !PF ? (CH > 12 ? 3 : 6) : (CH > 12 ? 2 : (CH == 12 && (HIST || GELU) ? 3 : 4));
}

template <int CH, bool BF, bool EXACT, bool WRITE_Y, bool HIST, bool GELU = false, bool PF = true>
__global__ void __launch_bounds__(kFastWarps * 32, fwd16_min_blocks<CH, HIST, GELU, PF>())
wta_fwd16_kernel(const uint16_t* __restrict__ x, int64_t n_rows, int64_t row_stride,
                 int k_host, const int32_t* __restrict__ k_dev,
                 uint16_t* __restrict__ y, uint8_t* __restrict__ bitmask,
                 int32_t* __restrict__ win) {
  constexpr int D = 256 * CH;
  // key range of the non-NaN values: [-inf, +inf]
  constexpr uint32_t kNeg = BF ? 0x007Fu : 0x03FFu, kPos = BF ? 0xFF80u : 0xFC00u;
  extern __shared__ __align__(16) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t* shist = reinterpret_cast<int32_t*>(smem);
  if (HIST) {
    for (int i = threadIdx.x; i < D; i += blockDim.x) shist[i] = 0;
    __syncthreads();
  }
  int k = k_dev ? *k_dev : k_host;
  k = max(1, min(D, k));
  // -1 for every valid launch (row_stride >= 0), unknown to the compiler
  const uint32_t neg1 = ~static_cast<uint32_t>(row_stride >> 63);

  const int64_t stride_rows = static_cast<int64_t>(gridDim.x) * kFastWarps;
  int64_t row = static_cast<int64_t>(blockIdx.x) * kFastWarps + warp;
  uint4 nxt[PF ? CH : 1];
  if (PF && row < n_rows) {
    const uint4* src = reinterpret_cast<const uint4*>(x + row * row_stride);
#pragma unroll
    for (int c = 0; c < CH; ++c) nxt[c] = __ldcs(src + c * 32 + lane);
  }
  // warp-uniform search state: the previous row's threshold key and how far
  // it moved from the row before; galloping pays while that distance is small
  // (about 2 log2(distance) + 2 probes against 16 for a full bisection).
  // ipc: keys per unit of count near the threshold (from the rows searched so
  // far), which turns the first probe's count into a jump estimate.
  constexpr uint32_t kTag = BF ? 0x10000u : 0x20000u;
  const int slot = blockIdx.x * kFastWarps + warp;
  bool have_prev = false;
  uint32_t t_prev = 0, dist_prev = 0;
  float ipc = 0.25f;
  if (slot < kHintSlots) {
    const uint32_t h = g_wta_hint_key[slot];
    if ((h & 0xFFFF0000u) == kTag) {
      const uint32_t hk = h & 0xFFFFu;
      if (hk >= kNeg && hk <= kPos) {
        have_prev = true;
        t_prev = hk;
        const float hi_pc = g_wta_hint_ipc[slot];
        if (hi_pc > 0.f && hi_pc < 64.f) ipc = hi_pc;
      }
    }
  }
  for (; row < n_rows; row += stride_rows) {
    uint4 w[CH];
    if constexpr (PF) {
#pragma unroll
      for (int c = 0; c < CH; ++c) w[c] = nxt[c];
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(x + row * row_stride);
#pragma unroll
      for (int c = 0; c < CH; ++c) w[c] = __ldcs(src + c * 32 + lane);
    }
    if constexpr (GELU) {     // the row is the pre-activation: select on gelu(x)
      static_assert(BF, "GELU input is bf16 only");
#pragma unroll
      for (int c = 0; c < CH; ++c)
        w[c] = make_uint4(gelu_bf16x2(w[c].x), gelu_bf16x2(w[c].y), gelu_bf16x2(w[c].z), gelu_bf16x2(w[c].w));
    }
    // prefetch the next row while this one is selected
    const int64_t nrow = row + stride_rows;
    if (PF && nrow < n_rows) {
      const uint4* src = reinterpret_cast<const uint4*>(x + nrow * row_stride);
#pragma unroll
      for (int c = 0; c < CH; ++c) nxt[c] = __ldcs(src + c * 32 + lane);
    }
    // #{x >= v}, NaN included when UNORD (NaN sorts above +inf)
    auto count_ge = [&](uint32_t key, auto unord) -> int {
      const uint32_t b = key_to_bits16(key);
      const uint32_t v2 = b | (b << 16);
      uint32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        if constexpr (decltype(unord)::value) {
          a0 = sub_mad(a0, cmp_geu2<BF>(w[c].x, v2), neg1);
          a1 = sub_mad(a1, cmp_geu2<BF>(w[c].y, v2), neg1);
          a2 = sub_mad(a2, cmp_geu2<BF>(w[c].z, v2), neg1);
          a3 = sub_mad(a3, cmp_geu2<BF>(w[c].w, v2), neg1);
        } else {
          a0 = sub_mad(a0, cmp_ge2<BF>(w[c].x, v2), neg1);
          a1 = sub_mad(a1, cmp_ge2<BF>(w[c].y, v2), neg1);
          a2 = sub_mad(a2, cmp_ge2<BF>(w[c].z, v2), neg1);
          a3 = sub_mad(a3, cmp_ge2<BF>(w[c].w, v2), neg1);
        }
      }
      return decode_mask_sum(__reduce_add_sync(kFull, (a0 + a1) + (a2 + a3)));
    };
    // The largest t with #{x >= t} + #NaN >= k is the (k - #NaN)-th largest
    // non-NaN value. Invariant: count(lo) >= k > count(hi) = c_hi, with the
    // sentinel hi = kPos + 1 ("above +inf"); count(kNeg) = d >= k.
    uint32_t lo = kNeg, hi = kPos + 1;
    const bool gallop = have_prev && dist_prev <= kGallopMax;
    int c0 = 0;
    uint32_t t_start = t_prev;
    if (gallop) {
      // count at the previous threshold; then one probe at the estimate
      // t_prev +- |c0 - k| * ipc, which usually lands on or next to the
      // answer; then gallop from the bracket edge it set, and bisect
      c0 = count_ge(t_prev, BoolC<true>{});
      // the linear estimate only where keys near the threshold are dense in
      // count (a few keys per count at most); elsewhere (thresholds near 0,
      // where keys spread over many exponents) step 1 and gallop
      // (d = 0: no estimate probe, gallop from t_prev at once)
      const uint32_t d = ipc <= 2.f
          ? max(1u, static_cast<uint32_t>(fminf(static_cast<float>(abs(c0 - k)) * ipc + 0.5f, 64.f))) : 0u;
      bool up;
      if (c0 >= k) {
        lo = t_prev;
        up = true;
        const uint32_t p = lo + d < hi ? lo + d : hi - 1;
        if (d > 0 && p > lo) {
          if (count_ge(p, BoolC<true>{}) >= k) lo = p;
          else { hi = p; up = false; }
        }
      } else {
        hi = t_prev;
        up = false;
        const uint32_t p = hi - kNeg > d ? hi - d : kNeg;
        if (d > 0 && p < hi && p > kNeg) {
          if (count_ge(p, BoolC<true>{}) >= k) { lo = p; up = true; }
          else hi = p;
        }
      }
      if (up) {            // the answer is at lo or above: walk up
        for (uint32_t step = 1; lo + step < hi; step <<= 1) {
          const uint32_t p = lo + step;
          if (count_ge(p, BoolC<true>{}) >= k) {
            lo = p;
          } else {
            hi = p;
            break;
          }
        }
      } else {             // the answer is below hi: walk down
        for (uint32_t step = 1; hi - lo > step; step <<= 1) {
          const uint32_t p = hi - step;
          if (count_ge(p, BoolC<true>{}) >= k) {
            lo = p;
            break;
          }
          hi = p;
        }
      }
    }
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      if (count_ge(mid, BoolC<true>{}) >= k) lo = mid;
      else hi = mid;
    }
    uint32_t t = lo;
    bool none = false;
    int c_gt = 0;                  // #{non-NaN x > t}
    if (t == kPos) {
      // threshold +inf, or #NaN >= k: then the reference's threshold is NaN
      // and nothing is kept
      const int n_nan = count_ge(kPos, BoolC<true>{}) - count_ge(kPos, BoolC<false>{});
      none = n_nan >= k;
    } else if (EXACT) {
      c_gt = count_ge(t + 1, BoolC<false>{});
    }
    dist_prev = have_prev ? (t > t_prev ? t - t_prev : t_prev - t) : 0u;
    if (gallop && t != t_start && c0 != k) {
      // keys per unit of count between the previous threshold and this one
      const float r = static_cast<float>(dist_prev) / static_cast<float>(abs(c0 - k));
      ipc = 0.5f * (ipc + fminf(r, 64.f));
    }
    t_prev = t;
    have_prev = true;
    const uint32_t tb = key_to_bits16(t);
    const uint32_t t2 = tb | (tb << 16);
    const int need = k - c_gt;     // exact_k: ties at t kept in index order
    int rank_base = 0;
    uint8_t* mrow = bitmask + row * (D / 8);
    uint4* yrow = WRITE_Y ? reinterpret_cast<uint4*>(y + row * static_cast<int64_t>(D)) : nullptr;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const uint32_t wv[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
      uint32_t m[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) m[i] = none ? 0u : (EXACT ? cmp_gt2<BF>(wv[i], t2) : cmp_ge2<BF>(wv[i], t2));
      uint32_t bits = mask_byte(m[0], m[1], m[2], m[3]);
      if (EXACT) {
        uint32_t e[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) e[i] = none ? 0u : cmp_eq2<BF>(wv[i], t2);
        const uint32_t tie = mask_byte(e[0], e[1], e[2], e[3]);
        int total;
        int r = rank_base + warp_excl_scan(__popc(tie), lane, total);
        rank_base += total;
#pragma unroll
        for (int b = 0; b < 8; ++b)
          if ((tie >> b) & 1u) { if (r < need) bits |= 1u << b; ++r; }
      }
      mrow[c * 32 + lane] = static_cast<uint8_t>(bits);
      if (WRITE_Y) {
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (EXACT) {
            // y = x * keep: a dropped value keeps only its sign
            const uint32_t sel = (((bits >> (2 * i)) & 1u) ? 0x0000FFFFu : 0u) |
                                 (((bits >> (2 * i + 1)) & 1u) ? 0xFFFF0000u : 0u) | 0x80008000u;
            o[i] = wv[i] & sel;
          } else {
            o[i] = wv[i] & m[i];    // y = where(keep, x, +0)
          }
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
  if (have_prev && lane == 0 && slot < kHintSlots) {     // warm start for the next launch
    g_wta_hint_key[slot] = kTag | t_prev;
    g_wta_hint_ipc[slot] = ipc;
  }
  if (HIST) {
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x)
      if (shist[i]) atomicAdd(&win[i], shist[i]);
  }
}

// ---------------------------------------------------------------------------
// Generic path: any d < 65536, any supported dtype, any row stride. One warp
// per row; the row is re-read (L1/L2) for every digit pass. NaN gets key 0,
// below every other key, and the select runs on k - #NaN, so NaN is handled as
// on the fast path (never kept; t is the (k - #NaN)-th largest non-NaN value).
// FMT: 0 fp32, 1 bf16, 2 f16.
template <int FMT>
__device__ __forceinline__ bool is_nan_bits(uint32_t b) {
  if (FMT == 0) return (b & 0x7FFFFFFFu) > 0x7F800000u;
  if (FMT == 1) return (b & 0x7FFFu) > 0x7F80u;
  return (b & 0x7FFFu) > 0x7C00u;
}
template <int FMT, typename T>
__device__ __forceinline__ uint32_t load_key(const T* p) {
  const uint32_t b = static_cast<uint32_t>(*p);
  if (is_nan_bits<FMT>(b)) return 0u;
  return FMT == 0 ? key32(b) : (keys16(b) & 0xFFFFu);
}

template <typename T, int FMT>
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
    int nan_count = 0;
    for (int j = lane; j < d; j += 32) nan_count += is_nan_bits<FMT>(static_cast<uint32_t>(xr[j]));
    int kk = k - static_cast<int>(__reduce_add_sync(kFull, static_cast<uint32_t>(nan_count)));
    const bool none = kk <= 0;
    uint32_t prefix = 0;
    for (int p = 0; p < KB / 8 && !none; ++p) {
      const int shift = KB - 8 * (p + 1);
      for (int j = lane; j < d; j += 32) {
        const uint32_t key = load_key<FMT>(xr + j);
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
    // with no winners the threshold is above every key
    const uint32_t t = none ? (KB == 16 ? 0x10000u : 0xFFFFFFFFu) : prefix;
    uint32_t tlo = t, thi = t;
    const uint32_t pz = (KB == 16) ? 0x8000u : 0x80000000u, nz = pz - 1u;
    if (t == pz || t == nz) { tlo = nz; thi = pz; }
    int need = 0;
    if (exact) {
      int gt = 0;
      for (int j = lane; j < d; j += 32) gt += load_key<FMT>(xr + j) > thi;
      need = none ? 0 : k - static_cast<int>(__reduce_add_sync(kFull, static_cast<uint32_t>(gt)));
    }
    int rank = 0;
    uint8_t* mrow = bitmask + row * mbytes;
    for (int j0 = 0; j0 < d; j0 += 32) {
      const int j = j0 + lane;
      bool keep = false;
      if (j < d) {
        const uint32_t key = load_key<FMT>(xr + j);
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

// Backward through GELU then WTA (bf16): dx = gelu'(x) * (dy * keep), each
// factor as PyTorch forms it (dy * keep in bf16, then the GELU gradient in fp32).
__global__ void __launch_bounds__(256)
wta_bwd_gelu_vec_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                        const uint8_t* __restrict__ mask, __nv_bfloat16* __restrict__ dx, int64_t n_bytes) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_bytes;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t m = mask[i];
    const uint4 gv = __ldcs(reinterpret_cast<const uint4*>(dy) + i);
    const uint4 xv = __ldcs(reinterpret_cast<const uint4*>(x) + i);
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, xw[4] = {xv.x, xv.y, xv.z, xv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float g0 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(gw[j] << 16) *
                                                            (((m >> (2 * j)) & 1u) ? 1.f : 0.f)));
      const float g1 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(gw[j] & 0xffff0000u) *
                                                            (((m >> (2 * j + 1)) & 1u) ? 1.f : 0.f)));
      const __nv_bfloat162 r = __floats2bfloat162_rn(gelu_erf_grad(g0, __uint_as_float(xw[j] << 16)),
                                                     gelu_erf_grad(g1, __uint_as_float(xw[j] & 0xffff0000u)));
      o[j] = *reinterpret_cast<const uint32_t*>(&r);
    }
    __stcs(reinterpret_cast<uint4*>(dx) + i, make_uint4(o[0], o[1], o[2], o[3]));
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

template <int CH, bool BF, bool EXACT, bool WRITE_Y, bool HIST, bool GELU = false>
int launch_fwd16(const void* x, int64_t n_rows, int64_t row_stride, int k, const int32_t* k_dev,
                 void* y, uint8_t* bitmask, int32_t* win, cudaStream_t st) {
  auto kern = wta_fwd16_kernel<CH, BF, EXACT, WRITE_Y, HIST, GELU>;
  if constexpr (!HIST && !GELU) {
    // few rows per warp at the prefetching kernel's occupancy (4 blocks per
    // SM): the variant without prefetch runs more warps instead
    if (n_rows < static_cast<int64_t>(sm_count()) * 4 * kFastWarps * 4)
      kern = wta_fwd16_kernel<CH, BF, EXACT, WRITE_Y, HIST, GELU, false>;
  }
  const size_t smem = HIST ? 256 * CH * 4 : 0;
  if (smem) TDX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
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

template <int CH, bool BF>
int dispatch_fwd16(const void* x, int64_t n_rows, int64_t row_stride, int k, const int32_t* k_dev,
                   int mode, void* y, uint8_t* bitmask, int32_t* win, cudaStream_t st, bool gelu = false) {
  const bool exact = mode == TAU_DXB_WTA_EXACT_K, wy = y != nullptr, h = win != nullptr;
  if (gelu) {
    if constexpr (BF) {
      if (!exact && wy && h) return launch_fwd16<CH, true, false, true, true, true>(x, n_rows, row_stride, k, k_dev,
                                                                                   y, bitmask, win, st);
      if (!exact && wy && !h) return launch_fwd16<CH, true, false, true, false, true>(x, n_rows, row_stride, k,
                                                                                     k_dev, y, bitmask, win, st);
    }
    return fail(TAU_DXB_ERR_UNSUPPORTED, "wta_fwd: GELU input needs bf16, threshold mode and y");
  }
#define TDX_WTA_CASE(E, W, H)                                                        \
  if (exact == E && wy == W && h == H)                                               \
    return launch_fwd16<CH, BF, E, W, H>(x, n_rows, row_stride, k, k_dev, y, bitmask, win, st);
  TDX_WTA_CASE(false, true, false) TDX_WTA_CASE(false, false, false)
  TDX_WTA_CASE(false, true, true)  TDX_WTA_CASE(false, false, true)
  TDX_WTA_CASE(true, true, false)  TDX_WTA_CASE(true, false, false)
  TDX_WTA_CASE(true, true, true)   TDX_WTA_CASE(true, false, true)
#undef TDX_WTA_CASE
  return fail(TAU_DXB_ERR_UNSUPPORTED, "wta_fwd: no kernel for this mode");
}

template <bool BF>
int dispatch_fwd16_width(int64_t d, const void* x, int64_t n_rows, int64_t row_stride, int k,
                         const int32_t* k_dev, int mode, void* y, uint8_t* bitmask, int32_t* win,
                         cudaStream_t st, bool gelu = false) {
  switch (d / 256) {
    case 3:  return dispatch_fwd16<3, BF>(x, n_rows, row_stride, k, k_dev, mode, y, bitmask, win, st, gelu);
    case 4:  return dispatch_fwd16<4, BF>(x, n_rows, row_stride, k, k_dev, mode, y, bitmask, win, st, gelu);
    case 6:  return dispatch_fwd16<6, BF>(x, n_rows, row_stride, k, k_dev, mode, y, bitmask, win, st, gelu);
    case 8:  return dispatch_fwd16<8, BF>(x, n_rows, row_stride, k, k_dev, mode, y, bitmask, win, st, gelu);
    case 12: return dispatch_fwd16<12, BF>(x, n_rows, row_stride, k, k_dev, mode, y, bitmask, win, st, gelu);
    case 16: return dispatch_fwd16<16, BF>(x, n_rows, row_stride, k, k_dev, mode, y, bitmask, win, st, gelu);
    default: return 1;   // no fast kernel for this width
  }
}

}  // namespace

int wta_fwd_impl(const void* x, int32_t dtype, int64_t n_rows, int64_t d, int64_t row_stride,
                 int64_t k, const int32_t* k_dev, int32_t mode, void* y, uint8_t* bitmask,
                 int32_t* win, cudaStream_t st) {
  TDX_CHECK_ARG(n_rows >= 0 && d >= 1 && d < 65536, "wta_fwd: need 0 <= n_rows, 1 <= d < 65536 (d=%lld)", (long long)d);
  if (n_rows == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(x && bitmask, "wta_fwd: x and bitmask are required");
  TDX_CHECK_ARG(row_stride >= d, "wta_fwd: row_stride (%lld) < d (%lld)", (long long)row_stride, (long long)d);
  const bool gelu = (mode & TAU_DXB_WTA_GELU_INPUT) != 0;
  mode &= ~TAU_DXB_WTA_GELU_INPUT;
  TDX_CHECK_ARG(mode == TAU_DXB_WTA_THRESHOLD || mode == TAU_DXB_WTA_EXACT_K, "wta_fwd: bad mode %d", mode);
  TDX_CHECK_ARG(dtype == TAU_DXB_F32 || dtype == TAU_DXB_BF16 || dtype == TAU_DXB_F16, "wta_fwd: bad dtype %d", dtype);
  const int kk = static_cast<int>(k < 1 ? 1 : (k > d ? d : k));
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (row_stride % 8 == 0) &&
                       (!y || reinterpret_cast<uintptr_t>(y) % 16 == 0);
  if (gelu) {
    TDX_CHECK_ARG(dtype == TAU_DXB_BF16 && aligned && d % 256 == 0 && y,
                  "wta_fwd: GELU input needs bf16 rows of d a multiple of 256, 16-byte aligned, and y");
    const int rc = dispatch_fwd16_width<true>(d, x, n_rows, row_stride, kk, k_dev, mode, y, bitmask, win, st, true);
    if (rc == 1) return fail(TAU_DXB_ERR_UNSUPPORTED, "wta_fwd: no GELU-input kernel for d = %lld", (long long)d);
    return rc;
  }
  if (dtype != TAU_DXB_F32 && aligned && d % 256 == 0) {
    const int rc = dtype == TAU_DXB_BF16
        ? dispatch_fwd16_width<true>(d, x, n_rows, row_stride, kk, k_dev, mode, y, bitmask, win, st)
        : dispatch_fwd16_width<false>(d, x, n_rows, row_stride, kk, k_dev, mode, y, bitmask, win, st);
    if (rc <= 0) return rc;        // launched (or failed); 1 = width without a fast kernel
  }
  const size_t smem = 4 * kHist16Bytes;
  int64_t blocks = (n_rows + 3) / 4;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  const int exact = mode == TAU_DXB_WTA_EXACT_K;
  if (dtype == TAU_DXB_F32) {
    auto kern = wta_fwd_generic_kernel<uint32_t, 0>;
    TDX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<static_cast<unsigned>(blocks), 128, smem, st>>>(
        static_cast<const uint32_t*>(x), n_rows, static_cast<int>(d), row_stride, kk, k_dev, exact,
        static_cast<uint32_t*>(y), bitmask, win);
  } else {
    auto kern = dtype == TAU_DXB_BF16 ? wta_fwd_generic_kernel<uint16_t, 1> : wta_fwd_generic_kernel<uint16_t, 2>;
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

int wta_bwd_gelu_impl(const void* dy, const void* x, const uint8_t* bitmask, int64_t n_rows, int64_t d, void* dx,
                      cudaStream_t st) {
  TDX_CHECK_ARG(n_rows >= 0 && d >= 1 && d % 8 == 0, "wta_bwd_gelu: need d a multiple of 8");
  if (n_rows == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(dy && x && bitmask && dx, "wta_bwd_gelu: dy, x, bitmask and dx are required");
  TDX_CHECK_ARG(reinterpret_cast<uintptr_t>(dy) % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(dx) % 16 == 0, "wta_bwd_gelu: dy, x and dx must be 16-byte aligned");
  const int64_t n_bytes = n_rows * d / 8;
  int64_t blocks = (n_bytes + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  wta_bwd_gelu_vec_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x), bitmask,
      static_cast<__nv_bfloat16*>(dx), n_bytes);
  return check_launch("wta_bwd_gelu_vec_kernel");
}

int wta_k_from_logits_impl(const float* logits, int64_t n, int64_t d_ff, int32_t* k_out,
                           cudaStream_t st) {
  TDX_CHECK_ARG(logits && k_out && n >= 0 && d_ff >= 1, "wta_k_from_logits: bad arguments");
  if (n == 0) return TAU_DXB_OK;
  k_from_logits_kernel<<<static_cast<unsigned>((n + 127) / 128), 128, 0, st>>>(logits, n, d_ff, k_out);
  return check_launch("k_from_logits_kernel");
}

}  // namespace taudxb
