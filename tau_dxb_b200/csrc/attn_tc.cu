// tau-opus attention, tensor-core path for sm_100a (bf16 in, fp32 accumulate).
//
// Forward kernel (one CTA = two 128-row query tiles of one (b, h)):
//   warp 0      TMA producer: Q tiles once, then K tiles (pass 1) and K,V
//               tiles (pass 2) through a 3-stage shared-memory ring.
//   warp 1      TMEM owner; lane 0 issues every tcgen05.mma:
//                 S_t = Q_t K_j^T  (M=128, N=128, K=64) into TMEM columns [128t, 128t+128)
//                 O_t += P_t V_j   (M=128, N=64,  K=128) into TMEM columns [256+64t, ...)
//   warps 4-7   softmax group for query tile 0, warps 8-11 for tile 1: each
//               thread owns one query row (= one TMEM lane). The two groups
//               alternate with the tensor core: while group 0 turns S_0 into
//               P_0, the MMA warp computes S_1, and vice versa.
// Pass 1 sweeps every key tile for the exact row max and first argmax of
// s = scale*QK^T (+mask): the reference applies sigma to s - max(s), which is
// not shift invariant for softplus/sigmoid, so no online rescaling is possible.
// Pass 2 recomputes S, forms q = max(sigma(alpha (s - m))^tau, 1e-8) in fp32,
// stores it as bf16 P (128B-swizzled K-major, the A operand of the PV MMA),
// accumulates l = sum q, and finally writes O / max(l, 1e-8).
//
// Per score element the forward spends two special-function ops (exp2) for
// softplus/sigmoid and one for exp: log2 sigma(x) is evaluated as
// x log2(e) + G(exp(x)) with G a polynomial on [0, 1] (poly_coeffs.h), tau
// is folded into the polynomial's coefficients and the two clamps of the
// reference collapse into one. TMEM loads are double-buffered: the next
// 32-column chunk is in flight while the current one is processed.

#include <cmath>

#include "attn.h"
#include "poly_coeffs.h"
#include "tc_common.cuh"

namespace taudxb {

bool make_tmap_bhld(CUtensorMap* map, const void* base, int64_t D, int64_t L, int64_t H, int64_t B,
                    const int64_t s[4], int box_rows) {
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p) {
      set_last_error("cuTensorMapEncodeTiled is not available from the driver");
      return false;
    }
    fn = reinterpret_cast<EncodeFn>(p);
  }
  const cuuint64_t gdim[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(L),
                              static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(B)};
  const cuuint64_t gstride[3] = {static_cast<cuuint64_t>(s[2] * 2), static_cast<cuuint64_t>(s[1] * 2),
                                 static_cast<cuuint64_t>(s[0] * 2)};
  const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(box_rows), 1, 1};
  const cuuint32_t estride[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), gdim,
                        gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return false;
  }
  return true;
}

namespace {

constexpr int kBM = 128, kBN = 128, kD = 64, kStages = 3;
constexpr int kFwdThreads = 384;
constexpr uint32_t kTileBytes = kBN * kD * 2;            // 16 KB bf16 tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLog2Clamp = -26.575424759098897f;      // log2(1e-8)

// error codes recorded in the device error word
constexpr int kErrTimeoutTma = 1, kErrTimeoutMma = 2, kErrTimeoutSoftmax = 4;

__device__ int g_error_word;

struct FwdParams {
  CUtensorMap tq, tk, tv;
  int B, H, Lq, Lk;
  const float* tau;
  const float* alpha;
  float scale;
  int causal;
  const void* mask; int mask_dtype; int64_t ms[4];
  void* out; int64_t os[4];
  float* row_max; float* row_z; int32_t* row_argmax;
  int* err;
};

struct __align__(8) FwdBarriers {
  uint64_t q_full;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];     // S_t in TMEM (and, in pass 2, the previous PV_t done with P_t)
  uint64_t s_free[2];     // S_t read out of TMEM by its softmax group
  uint64_t sp_ready[2];   // P_t written to shared memory (pass 2)
  uint64_t o_full[2];
  uint32_t tmem_base;
  int abort_flag;
};

constexpr uint32_t kSmemQ = 0;                                   // 2 x 16 KB
constexpr uint32_t kSmemK = kSmemQ + 2 * kTileBytes;             // stages x 16 KB
constexpr uint32_t kSmemV = kSmemK + kStages * kTileBytes;       // stages x 16 KB
constexpr uint32_t kSmemP = kSmemV + kStages * kTileBytes;       // 2 x 32 KB
constexpr uint32_t kSmemBar = kSmemP + 2 * 2 * kTileBytes;
constexpr uint32_t kFwdSmemBytes = kSmemBar + sizeof(FwdBarriers) + 1024;  // + alignment slack

__device__ __forceinline__ float fwd_mask_value(const FwdParams& p, int b, int h, int r, int c) {
  float mv = 0.f;
  if (p.mask) {
    const int64_t off = b * p.ms[0] + h * p.ms[1] + static_cast<int64_t>(r) * p.ms[2] +
                        static_cast<int64_t>(c) * p.ms[3];
    mv = load_as_float(p.mask, p.mask_dtype, off);
  }
  if (p.causal && c > r + (p.Lk - p.Lq)) mv += kMaskMin;
  return mv;
}

template <int V> struct IntC { static constexpr int value = V; };

template <int SIG>
__global__ void __launch_bounds__(kFwdThreads, 1) attn_fwd_tc_kernel(const __grid_constant__ FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base by pointer arithmetic on the __shared__ array, so the
  // compiler keeps every derived pointer in the shared address space
  uint8_t* smem = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  FwdBarriers* bars = reinterpret_cast<FwdBarriers*>(smem + kSmemBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * 2 * kBM;
  const int nK = (p.Lk + kBN - 1) / kBN;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    tc::mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) { tc::mbar_init(&bars->kv_full[s], 1); tc::mbar_init(&bars->kv_empty[s], 1); }
    for (int t = 0; t < 2; ++t) {
      tc::mbar_init(&bars->s_full[t], 1);
      tc::mbar_init(&bars->s_free[t], 4);
      tc::mbar_init(&bars->sp_ready[t], 4);
      tc::mbar_init(&bars->o_full[t], 1);
    }
    bars->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) { tc::tmem_alloc(&bars->tmem_base, 512); tc::tmem_relinquish(); }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tc::mbar_arrive_expect_tx(&bars->q_full, 2 * kTileBytes);
      tc::tma_load_4d(smem + kSmemQ, &p.tq, &bars->q_full, 0, q0, h, b);
      tc::tma_load_4d(smem + kSmemQ + kTileBytes, &p.tq, &bars->q_full, 0, q0 + kBM, h, b);
      int it = 0;
      bool ok = true;
      for (int pass = 0; pass < 2 && ok; ++pass) {
        for (int j = 0; j < nK; ++j, ++it) {
          const int s = it % kStages;
          if (it >= kStages &&
              !tc::mbar_wait(&bars->kv_empty[s], ((it / kStages) - 1) & 1, abort_flag, p.err, kErrTimeoutTma)) {
            ok = false;
            break;
          }
          tc::mbar_arrive_expect_tx(&bars->kv_full[s], pass == 0 ? kTileBytes : 2 * kTileBytes);
          tc::tma_load_4d(smem + kSmemK + s * kTileBytes, &p.tk, &bars->kv_full[s], 0, j * kBN, h, b);
          if (pass == 1)
            tc::tma_load_4d(smem + kSmemV + s * kTileBytes, &p.tv, &bars->kv_full[s], 0, j * kBN, h, b);
        }
      }
      if (*abort_flag) {
        // drain: let the copies this thread started land before the CTA exits
        const uint64_t t0 = tc::globaltimer_ns();
        for (int s = 0; s < kStages && s < it; ++s) {
          const int fills = (it - s + kStages - 1) / kStages;
          const uint32_t a = tc::smem_u32(&bars->kv_full[s]);
          while (!tc::mbar_try_wait(a, (fills - 1) & 1) && tc::globaltimer_ns() - t0 < tc::kWaitLimitNs) {
          }
        }
        const uint32_t qa = tc::smem_u32(&bars->q_full);
        while (!tc::mbar_try_wait(qa, 0) && tc::globaltimer_ns() - t0 < tc::kWaitLimitNs) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = tc::idesc_bf16(kBM, kBN, 0, 0);
      constexpr uint32_t idO = tc::idesc_bf16(kBM, kD, 0, 1);
      const uint32_t sQ = tc::smem_u32(smem + kSmemQ);
      const uint32_t sK = tc::smem_u32(smem + kSmemK);
      const uint32_t sV = tc::smem_u32(smem + kSmemV);
      const uint32_t sP = tc::smem_u32(smem + kSmemP);
      bool ok = tc::mbar_wait(&bars->q_full, 0, abort_flag, p.err, kErrTimeoutMma);
      tc::tc_fence_after();
      int s_prev = 0;
      // descriptors as 32-bit halves: K-slices of 16 step 32 B (2) in K-major
      // tiles and 2048 B (128) in the MN-major V tile; the high half is shared
      constexpr uint32_t hi = tc::sdesc_hi_sw128(1024);
      constexpr uint32_t tileStep = kTileBytes >> 4;
      const uint32_t kQ = tc::sdesc_lo(sQ, 16), kK = tc::sdesc_lo(sK, 16);
      const uint32_t kP = tc::sdesc_lo(sP, 16), mV = tc::sdesc_lo(sV, 16384);
      auto issue_S = [&](int t, int s) {
        const uint32_t d = tmem + t * kBN;
        const uint32_t qa = kQ + t * tileStep, kb = kK + s * tileStep;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) tc::umma_f16_ss2(d, qa + 2 * kk, hi, kb + 2 * kk, hi, idS, kk > 0);
      };
      auto issue_PV = [&](int t, int s, bool first) {
        const uint32_t d = tmem + 256 + t * kD;
        const uint32_t pa = kP + t * 2 * tileStep, vb = mV + s * tileStep;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          tc::umma_f16_ss2(d, pa + (kk >> 2) * tileStep + (kk & 3) * 2, hi, vb + 128 * kk, hi, idO,
                           !first || kk > 0);
      };
      // Step i (pass 1: key tile i; pass 2: key tile i - nK): S_t into TMEM
      // once group t has read the previous S_t out; in pass 2 then PV_t of the
      // previous key tile once P_t is written, and s_full_t covers both (the
      // group overwrites P_t only after that PV is done).
      for (int i = 0; i < 2 * nK && ok; ++i) {
        const bool pass2 = i >= nK;
        const int j = pass2 ? i - nK : i;
        const int s = i % kStages;
        ok = tc::mbar_wait(&bars->kv_full[s], (i / kStages) & 1, abort_flag, p.err, kErrTimeoutMma);
        if (!ok) break;
        tc::tc_fence_after();
        for (int t = 0; t < 2 && ok; ++t) {      // group 0 runs ahead of group 1
          if (i > 0) {
            ok = tc::mbar_wait(&bars->s_free[t], (i - 1) & 1, abort_flag, p.err, kErrTimeoutMma);
            if (!ok) break;
            tc::tc_fence_after();
          }
          issue_S(t, s);
          if (pass2 && j > 0) {
            ok = tc::mbar_wait(&bars->sp_ready[t], (j - 1) & 1, abort_flag, p.err, kErrTimeoutMma);
            if (!ok) break;
            tc::tc_fence_after();
            issue_PV(t, s_prev, j == 1);
          }
          tc::umma_commit(&bars->s_full[t]);
        }
        if (!ok) break;
        if (pass2 && j > 0) tc::umma_commit(&bars->kv_empty[s_prev]);
        if (!pass2) tc::umma_commit(&bars->kv_empty[s]);
        else s_prev = s;
      }
      for (int t = 0; t < 2 && ok; ++t) {
        ok = tc::mbar_wait(&bars->sp_ready[t], (nK - 1) & 1, abort_flag, p.err, kErrTimeoutMma);
        if (!ok) break;
        tc::tc_fence_after();
        issue_PV(t, s_prev, nK == 1);
        tc::umma_commit(&bars->o_full[t]);
      }
      // every MMA issued so far must finish before TMEM is released
      tc::umma_commit(&bars->q_full);
      {
        const uint64_t t0 = tc::globaltimer_ns();
        const uint32_t qa = tc::smem_u32(&bars->q_full);
        while (!tc::mbar_try_wait(qa, 1) && tc::globaltimer_ns() - t0 < tc::kWaitLimitNs) {
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax groups
    const int t = (warp - 4) >> 2;                 // query tile of this group
    const int r = ((warp & 3) << 5) + lane;        // row within the tile = TMEM lane
    const int grow = q0 + t * kBM + r;
    const bool row_ok = grow < p.Lq;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const uint32_t tS = tmem + lane_base + t * kBN;
    const uint32_t tO = tmem + lane_base + 256 + t * kD;
    const float tau = p.tau[h], alpha = p.alpha[h];
    const bool explicit_mask = p.mask != nullptr;
    // keys >= lim_c of this row are causally masked (score + finfo.min), keys
    // >= Lk are padding (no contribution at all)
    const int lim_c = p.causal ? min(p.Lk, grow + (p.Lk - p.Lq) + 1) : p.Lk;
    uint8_t* Pt = smem + kSmemP + t * 2 * kTileBytes;
    bool ok = true;
    int i = 0;
    float m = -INFINITY;
    int amax = 0;
    // Per key tile the warp takes one of three branch-free element paths:
    // kFast (every key valid and unmasked for all 32 rows, no mask tensor,
    // scale > 0), kLimited (causal limit / padding per row, no mask tensor),
    // kGeneral (mask tensor).
    constexpr int kFast = 0, kLimited = 1, kGeneral = 2;
    auto tile_mode = [&](int j) -> int {
      if (explicit_mask) return kGeneral;
      const bool full = (j + 1) * kBN <= lim_c && p.scale > 0.f;
      return __all_sync(0xffffffffu, full) ? kFast : kLimited;
    };
    // pass 1: exact row max and first argmax of s = scale * QK^T (+ mask) in
    // increasing key order. The chunk max comes from four independent fmax
    // chains; only when it beats the running max is the first index found.
    // Pass 1: per 32-key chunk, four interleaved chains (keys e = a mod 4) keep
    // their max and its first key (strictly larger replaces), so the first
    // argmax costs no data-dependent branch. The fast path compares the raw
    // QK^T values (scale > 0 keeps their order).
    auto pass1_chunk = [&](auto mode_c, const uint32_t (&v)[32], int key0) {
      constexpr int kMode = decltype(mode_c)::value;
      float x[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float raw = __uint_as_float(v[e]);
        if constexpr (kMode == kFast) {
          x[e] = raw;
        } else {
          float sv = raw * p.scale;
          if constexpr (kMode == kLimited) {
            if (key0 + e >= lim_c) sv += kMaskMin;
          } else {
            if (row_ok) sv += fwd_mask_value(p, b, h, grow, key0 + e);
          }
          x[e] = key0 + e < p.Lk ? sv : -INFINITY;
        }
      }
      float c4[4] = {x[0], x[1], x[2], x[3]};
      int i4[4] = {0, 1, 2, 3};
#pragma unroll
      for (int e = 4; e < 32; ++e) {
        const bool gt = x[e] > c4[e & 3];
        c4[e & 3] = gt ? x[e] : c4[e & 3];
        i4[e & 3] = gt ? e : i4[e & 3];
      }
      // combine: the largest value, the smallest key among the chains holding it
      float cx = fmaxf(fmaxf(c4[0], c4[1]), fmaxf(c4[2], c4[3]));
      int first = 32;
#pragma unroll
      for (int a4 = 0; a4 < 4; ++a4) first = min(first, c4[a4] == cx ? i4[a4] : 32);
      const float cm = kMode == kFast ? cx * p.scale : cx;
      if (cm > m && first < 32) {           // strictly larger: earlier chunks win ties
        m = cm;
        amax = key0 + first;
      }
    };
    auto release_s = [&]() {      // every TMEM read of S for this step is done
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars->s_free[t]);
    };
    for (int j = 0; j < nK && ok; ++j, ++i) {
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars->s_full[t], i & 1, abort_flag, p.err, kErrTimeoutSoftmax));
      if (!ok) break;
      tc::tc_fence_after();
      const int mode = tile_mode(j);
      auto run = [&](auto mode_c) {
        uint32_t va[32], vb[32];
        tc::tmem_ld32(tS, va);
        tc::tmem_wait_ld_regs(va);
#pragma unroll 1
        for (int c = 0; c < kBN / 32; c += 2) {
          tc::tmem_ld32(tS + (c + 1) * 32, vb);           // next chunk in flight
          pass1_chunk(mode_c, va, j * kBN + c * 32);
          tc::tmem_wait_ld_regs(vb);
          if (c + 2 < kBN / 32) tc::tmem_ld32(tS + (c + 2) * 32, va);
          else release_s();
          pass1_chunk(mode_c, vb, j * kBN + (c + 1) * 32);
          if (c + 2 < kBN / 32) tc::tmem_wait_ld_regs(va);
        }
      };
      if (mode == kFast) run(IntC<kFast>{});
      else if (mode == kLimited) run(IntC<kLimited>{});
      else run(IntC<kGeneral>{});
    }
    if (!row_ok) m = 0.f;
    // pass 2: q = max(sigma(alpha (s - m))^tau, 1e-8) = 2^max(tau log2 sigma, ylo)
    // with ylo = max(tau, 1) * log2(1e-8), the two clamps of the reference folded
    // into one (tau log2 sigma_clamped >= tau log2(1e-8)).
    const float al2 = alpha * kLog2e;
    const float sa2 = p.scale * al2, ma2 = m * al2;
    const float ylo = fmaxf(tau * kLog2Clamp, kLog2Clamp);
    float l0 = 0.f, l1 = 0.f;
    auto qval = [&](float a2) -> float {
      float y;
      if (SIG == TAU_DXB_SIGMA_SOFTPLUS) {
        y = fmaf(tau, a2, poly::G_scaled(tc::ex2(a2), tau));
      } else if (SIG == TAU_DXB_SIGMA_SIGMOID) {
        y = fmaf(tau, a2, -poly::H_scaled(tc::ex2(a2), tau));
      } else if (SIG == TAU_DXB_SIGMA_EXP) {
        y = tau * a2;
      } else {
        y = ylo;   // relu(x <= 0) = 0 -> clamped sigma 1e-8
      }
      return tc::ex2(fmaxf(y, ylo));
    };
    auto pass2_chunk = [&](auto mode_c, const uint32_t (&v)[32], int c, int key0) {
      constexpr int kMode = decltype(mode_c)::value;
      uint32_t pk[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float qq[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const float raw = __uint_as_float(v[e + u]);
          const int key = key0 + e + u;
          if constexpr (kMode == kFast) {
            qq[u] = qval(fmaf(raw, sa2, -ma2));
          } else if constexpr (kMode == kLimited) {
            // masked: ((s + finfo.min) - m) alpha log2(e), rounded as the reference
            const float a2 = key < lim_c ? fmaf(raw, sa2, -ma2) : (raw * p.scale + kMaskMin - m) * al2;
            const float qv = qval(a2);
            qq[u] = key < p.Lk ? qv : 0.f;
          } else {
            // unmasked scores as in the fast path, masked ones as in the limited path
            const float mv = row_ok ? fwd_mask_value(p, b, h, grow, key) : 0.f;
            const float a2 = mv == 0.f ? fmaf(raw, sa2, -ma2) : (raw * p.scale + mv - m) * al2;
            const float qv = qval(a2);
            qq[u] = key < p.Lk ? qv : 0.f;
          }
        }
        l0 += qq[0];
        l1 += qq[1];
        pk[e >> 1] = tc::pack_bf16(qq[0], qq[1]);
      }
      // 32 keys -> 4 x 16-byte chunks of the 128B-swizzled K-major P tile
      uint8_t* rowp = Pt + (c >> 1) * kTileBytes + r * 128;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int chunk = ((c & 1) * 4 + u) ^ (r & 7);
        *reinterpret_cast<uint4*>(rowp + chunk * 16) =
            make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
      }
    };
    for (int j = 0; j < nK && ok; ++j, ++i) {
      // s_full also means the PV MMA of the previous step is done with P
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars->s_full[t], i & 1, abort_flag, p.err, kErrTimeoutSoftmax));
      if (!ok) break;
      tc::tc_fence_after();
      const int mode = tile_mode(j);
      auto run = [&](auto mode_c) {
        uint32_t va[32], vb[32];
        tc::tmem_ld32(tS, va);
        tc::tmem_wait_ld_regs(va);
#pragma unroll 1
        for (int c = 0; c < kBN / 32; c += 2) {
          tc::tmem_ld32(tS + (c + 1) * 32, vb);           // next chunk in flight
          pass2_chunk(mode_c, va, c, j * kBN + c * 32);
          tc::tmem_wait_ld_regs(vb);
          if (c + 2 < kBN / 32) tc::tmem_ld32(tS + (c + 2) * 32, va);
          else release_s();
          pass2_chunk(mode_c, vb, c + 1, j * kBN + (c + 1) * 32);
          if (c + 2 < kBN / 32) tc::tmem_wait_ld_regs(va);
        }
      };
      if (mode == kFast) run(IntC<kFast>{});
      else if (mode == kLimited) run(IntC<kLimited>{});
      else run(IntC<kGeneral>{});
      tc::fence_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars->sp_ready[t]);
    }
    const float l = l0 + l1;
    // epilogue: O / Z
    if (ok) ok = tc::mbar_wait(&bars->o_full[t], 0, abort_flag, p.err, kErrTimeoutSoftmax);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc::tc_fence_after();
      uint32_t o0[32], o1[32];
      tc::tmem_ld32(tO, o0);
      tc::tmem_ld32(tO + 32, o1);
      tc::tmem_wait_ld();
      const float Z = fmaxf(l, kClampMin);
      const float rz = 1.f / Z;
      if (row_ok) {
        __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + b * p.os[0] + h * p.os[1] +
                              static_cast<int64_t>(grow) * p.os[2];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 w;
          w.x = tc::pack_bf16(__uint_as_float(o0[8 * u + 0]) * rz, __uint_as_float(o0[8 * u + 1]) * rz);
          w.y = tc::pack_bf16(__uint_as_float(o0[8 * u + 2]) * rz, __uint_as_float(o0[8 * u + 3]) * rz);
          w.z = tc::pack_bf16(__uint_as_float(o0[8 * u + 4]) * rz, __uint_as_float(o0[8 * u + 5]) * rz);
          w.w = tc::pack_bf16(__uint_as_float(o0[8 * u + 6]) * rz, __uint_as_float(o0[8 * u + 7]) * rz);
          reinterpret_cast<uint4*>(orow)[u] = w;
          w.x = tc::pack_bf16(__uint_as_float(o1[8 * u + 0]) * rz, __uint_as_float(o1[8 * u + 1]) * rz);
          w.y = tc::pack_bf16(__uint_as_float(o1[8 * u + 2]) * rz, __uint_as_float(o1[8 * u + 3]) * rz);
          w.z = tc::pack_bf16(__uint_as_float(o1[8 * u + 4]) * rz, __uint_as_float(o1[8 * u + 5]) * rz);
          w.w = tc::pack_bf16(__uint_as_float(o1[8 * u + 6]) * rz, __uint_as_float(o1[8 * u + 7]) * rz);
          reinterpret_cast<uint4*>(orow)[4 + u] = w;
        }
        const int64_t ri = (static_cast<int64_t>(b) * p.H + h) * p.Lq + grow;
        p.row_max[ri] = m;
        p.row_z[ri] = Z;
        p.row_argmax[ri] = amax;
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

}  // namespace

// TMA needs 16-byte aligned rows and strides; the kernels need unit d-stride.
static bool tensor_layout_ok(const void* ptr, const int64_t s[4]) {
  return s[3] == 1 && (reinterpret_cast<uintptr_t>(ptr) % 16 == 0) && s[0] % 8 == 0 &&
         s[1] % 8 == 0 && s[2] % 8 == 0 && s[0] >= 0 && s[1] >= 0 && s[2] > 0;
}

bool attn_tensor_supported(const AttnProblem& p) {
  if (p.dtype != TAU_DXB_BF16 || p.D != kD) return false;
  if (!tensor_layout_ok(p.q, p.qs) || !tensor_layout_ok(p.k, p.ks) || !tensor_layout_ok(p.v, p.vs))
    return false;
  if (p.out && !tensor_layout_ok(p.out, p.outs)) return false;
  return true;
}


int attn_fwd_tensor(const AttnProblem& p, cudaStream_t st) {
  FwdParams fp;
  memset(&fp, 0, sizeof(fp));
  if (!make_tmap_bhld(&fp.tq, p.q, p.D, p.Lq, p.H, p.B, p.qs, kBM) ||
      !make_tmap_bhld(&fp.tk, p.k, p.D, p.Lk, p.H, p.B, p.ks, kBN) ||
      !make_tmap_bhld(&fp.tv, p.v, p.D, p.Lk, p.H, p.B, p.vs, kBN))
    return TAU_DXB_ERR_CUDA;
  fp.B = p.B; fp.H = p.H; fp.Lq = p.Lq; fp.Lk = p.Lk;
  fp.tau = p.tau; fp.alpha = p.alpha; fp.scale = p.scale; fp.causal = p.causal;
  fp.mask = p.mask; fp.mask_dtype = p.mask_dtype;
  for (int i = 0; i < 4; ++i) { fp.ms[i] = p.ms[i]; fp.os[i] = p.outs[i]; }
  fp.out = p.out; fp.row_max = p.row_max; fp.row_z = p.row_z; fp.row_argmax = p.row_argmax;
  int* err = device_error_word();
  if (!err) return fail(TAU_DXB_ERR_CUDA, "cannot resolve the device error word");
  fp.err = err;
  dim3 grid((p.Lq + 2 * kBM - 1) / (2 * kBM), p.H, p.B);
  auto launch = [&](auto kern) -> int {
    TDX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFwdSmemBytes));
    kern<<<grid, kFwdThreads, kFwdSmemBytes, st>>>(fp);
    return check_launch("attn_fwd_tc_kernel");
  };
  switch (p.sigma) {
    case TAU_DXB_SIGMA_SOFTPLUS: return launch(attn_fwd_tc_kernel<TAU_DXB_SIGMA_SOFTPLUS>);
    case TAU_DXB_SIGMA_SIGMOID: return launch(attn_fwd_tc_kernel<TAU_DXB_SIGMA_SIGMOID>);
    case TAU_DXB_SIGMA_EXP: return launch(attn_fwd_tc_kernel<TAU_DXB_SIGMA_EXP>);
    default: return launch(attn_fwd_tc_kernel<TAU_DXB_SIGMA_RELU>);
  }
}

int* device_error_word() {
  int* err = nullptr;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_error_word) != cudaSuccess) return nullptr;
  return err;
}

int read_device_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_error_word, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int z = 0;
    cudaMemcpyToSymbol(g_error_word, &z, sizeof(int));
  }
  return v;
}

}  // namespace taudxb
