// tau-opus attention, tensor-core path for sm_100a (bf16 in, fp32 accumulate).
//
// Forward kernel (one CTA = two 128-row query tiles of one (b, h)):
//   warp 0      TMA producer: Q tiles once, then K tiles (pass 1) and K,V
//               tiles (pass 2) through a 3-stage shared-memory ring.
//   warp 1      TMEM owner; lane 0 issues every tcgen05.mma:
//                 S_t = Q_t K_j^T  (M=128, N=128, K=64) into TMEM columns [128t, 128t+128)
//                 O_t += P_t V_j   (M=128, N=64,  K=128) into TMEM columns [256+64t, ...)
//   warps 4-19  four softmax warpgroups: warpgroup g serves query tile g >> 1
//               and key half g & 1 (keys [64 h, 64 h + 64) of every key tile).
//               Each thread owns one query row (= one TMEM lane) for that half;
//               the two halves of a row combine max / argmax and the row sum
//               through shared memory. The tiles alternate with the tensor
//               core: while tile 0's warpgroups turn S_0 into P_0, the MMA warp
//               computes S_1, and vice versa.
// Pass 1 sweeps every key tile for the exact row max of s = scale*QK^T (+mask):
// the reference applies sigma to s - max(s), which is not shift invariant for
// softplus/sigmoid, so no online rescaling is possible. Pass 2 recomputes S
// (the same MMAs on the same tiles, so the same bits), finds the first key
// whose score equals the max (the argmax the backward needs), forms
// q = max(sigma(alpha (s - m))^tau, 1e-8) in fp32, stores it as bf16 P
// (128B-swizzled K-major, the A operand of the PV MMA), accumulates l = sum q,
// and finally writes O / max(l, 1e-8).
//
// Per score element the forward spends two special-function ops (exp2) for
// softplus/sigmoid and one for exp: log2 sigma(x) is evaluated as
// x log2(e) + G(exp(x)) with G a polynomial on [0, 1] (poly_coeffs.h), tau
// is folded into the polynomial's coefficients and the two clamps of the
// reference collapse into one. TMEM loads are double-buffered: the next
// 32-column chunk is in flight while the current one is processed.

#include <climits>
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
constexpr int kFwdThreads = 640;     // 20 warps: TMA, MMA, 2 idle, 4 softmax warpgroups
constexpr int kFwdLaunchRegs = (65536 / kFwdThreads) & ~7;   // registers per thread at launch
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
  uint64_t s_full[2];     // S_t in TMEM
  uint64_t s_free[2];     // S_t read out of TMEM by its softmax warpgroups
  uint64_t sp_ready[2];   // P_t written to shared memory (pass 2)
  uint64_t pv_done[2];    // the PV_t MMA of the previous key tile is done with P_t
  uint64_t o_full[2];
  uint32_t tmem_base;
  int abort_flag;
};

constexpr uint32_t kSmemQ = 0;                                   // 2 x 16 KB
constexpr uint32_t kSmemK = kSmemQ + 2 * kTileBytes;             // stages x 16 KB
constexpr uint32_t kSmemV = kSmemK + kStages * kTileBytes;       // stages x 16 KB
constexpr uint32_t kSmemP = kSmemV + kStages * kTileBytes;       // 2 x 32 KB
constexpr uint32_t kSmemX = kSmemP + 2 * 2 * kTileBytes;        // row-state exchange: [tile][half][128] x {m, argmax, l}
constexpr uint32_t kSmemBar = kSmemX + 2 * 2 * kBM * 3 * 4;
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
  // Built-in causal mask (no mask tensor, Lq <= Lk): key tiles that every row
  // of this CTA has masked are skipped. The reference gives each masked key
  // the floor q = 1e-8; the row sums get that exactly (n_skip keys below), the
  // output's share of it (1e-8 of the row weight per key) is dropped.
  int nK = (p.Lk + kBN - 1) / kBN;
  if (p.causal && !p.mask && p.Lq <= p.Lk) {
    const int last_row = min(q0 + 2 * kBM, p.Lq) - 1;
    const int lim = last_row + (p.Lk - p.Lq) + 1;      // keys >= lim are masked for every row here
    nK = min(nK, max(1, (lim + kBN - 1) / kBN));
  }
  const int n_skip = max(0, p.Lk - nK * kBN);          // masked keys not visited
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    tc::mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) { tc::mbar_init(&bars->kv_full[s], 1); tc::mbar_init(&bars->kv_empty[s], 1); }
    for (int t = 0; t < 2; ++t) {
      tc::mbar_init(&bars->s_full[t], 1);
      tc::mbar_init(&bars->s_free[t], 8);
      tc::mbar_init(&bars->sp_ready[t], 8);
      tc::mbar_init(&bars->o_full[t], 1);
      tc::mbar_init(&bars->pv_done[t], 1);
    }
    bars->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) { tc::tmem_alloc(&bars->tmem_base, 512); tc::tmem_relinquish(); }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  // Register split of the 96 x 640 the block is launched with (65536 / 640
  // rounded down to a multiple of 8): warpgroup 0 (TMA, MMA) 64 per thread,
  // the four softmax warpgroups 104 (64*128 + 104*512 = 61440). setmaxnreg.inc
  // can only take what the block's own decs release.
  static_assert(64 * 128 + 104 * 512 <= kFwdLaunchRegs * kFwdThreads, "register split");
  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 64;" ::: "memory");
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
        // once tile t's warpgroups have read the previous S_t out (s_full_t);
        // in pass 2 then PV_t of the previous key tile once P_t is written
        // (pv_done_t: the warpgroups overwrite P_t only after that PV is done,
        // and start on the next S_t before it).
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
            tc::umma_commit(&bars->s_full[t]);
            if (pass2 && j > 0) {
              ok = tc::mbar_wait(&bars->sp_ready[t], (j - 1) & 1, abort_flag, p.err, kErrTimeoutMma);
              if (!ok) break;
              tc::tc_fence_after();
              issue_PV(t, s_prev, j == 1);
              tc::umma_commit(&bars->pv_done[t]);
            }
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
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 104;" ::: "memory");
    // ------------------------------------------------------------ softmax warpgroups
    const int g = (warp - 4) >> 2;                 // warpgroup 0..3
    const int t = g >> 1;                          // query tile of this warpgroup
    const int hc = g & 1;                          // key half: keys [64 hc, 64 hc + 64) of each tile
    const int kh = hc * 64;
    const int r = ((warp & 3) << 5) + lane;        // row within the tile = TMEM lane
    const int grow = q0 + t * kBM + r;
    const bool row_ok = grow < p.Lq;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const uint32_t tS = tmem + lane_base + t * kBN + kh;
    const uint32_t tO = tmem + lane_base + 256 + t * kD + hc * 32;
    const float tau = p.tau[h], alpha = p.alpha[h];
    const bool explicit_mask = p.mask != nullptr;
    // keys >= lim_c of this row are causally masked (score + finfo.min), keys
    // >= Lk are padding (no contribution at all)
    const int lim_c = p.causal ? min(p.Lk, grow + (p.Lk - p.Lq) + 1) : p.Lk;
    uint8_t* Pt = smem + kSmemP + t * 2 * kTileBytes + hc * kTileBytes;   // this half's 64-key atom
    // row-state exchange between the two halves of a row (named barrier 1 + t)
    float* xm = reinterpret_cast<float*>(smem + kSmemX) + (t * 2) * kBM;   // [half][128]
    int* xa = reinterpret_cast<int*>(xm + 2 * 2 * kBM);
    float* xl = xm + 2 * 2 * 2 * kBM;
    bool ok = true;
    int i = 0;
    // pass 1 maxima: mraw over fast chunks (raw QK^T, scale > 0 keeps the
    // order), mlim over the others (scaled, masked scores); mchunk is the
    // first fast 16-key chunk (4 key tile + chunk) that reached mraw
    float mraw = -INFINITY, mlim = -INFINITY;
    int mchunk = -1;
    // Per key tile the warp takes one of three branch-free element paths:
    // kFast (every key of its half valid and unmasked for all 32 rows, no mask
    // tensor, scale > 0), kLimited (causal limit / padding per row, no mask
    // tensor), kGeneral (mask tensor).
    constexpr int kFast = 0, kLimited = 1, kGeneral = 2;
    auto tile_mode = [&](int j) -> int {
      if (explicit_mask) return kGeneral;
      const bool full = j * kBN + kh + 64 <= lim_c && p.scale > 0.f;
      return __all_sync(0xffffffffu, full) ? kFast : kLimited;
    };
    // Pass 1: exact row max of s = scale * QK^T (+ mask), three-input max
    // trees. The first argmax is found in pass 2, which recomputes S with the
    // same MMA on the same tiles (bit-identical scores): the first key whose
    // score equals the max. For fast chunks only the chunk pass 1 recorded is
    // searched.
    auto score_x = [&](auto mode_c, float raw, int key) -> float {
      constexpr int kMode = decltype(mode_c)::value;
      if constexpr (kMode == kFast) {
        return raw;
      } else {
        float sv = raw * p.scale;
        if constexpr (kMode == kLimited) {
          if (key >= lim_c) sv += kMaskMin;
        } else {
          if (row_ok) sv += fwd_mask_value(p, b, h, grow, key);
        }
        return key < p.Lk ? sv : -INFINITY;
      }
    };
    auto pass1_chunk = [&](auto mode_c, const uint32_t (&v)[16], int key0, int cid) {
      constexpr int kMode = decltype(mode_c)::value;
      float x[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) x[e] = score_x(mode_c, __uint_as_float(v[e]), key0 + e);
      const float c0 = tc::max3(x[0], x[1], x[2]), c1 = tc::max3(x[3], x[4], x[5]);
      const float c2 = tc::max3(x[6], x[7], x[8]), c3 = tc::max3(x[9], x[10], x[11]);
      const float c4 = tc::max3(x[12], x[13], x[14]);
      const float cx = tc::max3(tc::max3(c0, c1, c2), c3, c4);
      if constexpr (kMode == kFast) {
        const float cm = fmaxf(cx, x[15]);
        if (cm > mraw) {                 // strictly larger: the first chunk holding the max
          mraw = cm;
          mchunk = cid;
        }
      } else {
        mlim = tc::max3(mlim, cx, x[15]);
      }
    };
    auto release_s = [&]() {      // every TMEM read of S for this step is done
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars->s_free[t]);
    };
    // the 64 keys of this half as four 16-column TMEM chunks, the next one in
    // flight while the current one is processed; S is released after the last load
    auto sweep = [&](auto&& chunk_fn) {
      uint32_t va[16], vb[16];
      tc::tmem_ld16(tS, va);
      tc::tmem_wait_ld_regs16(va);
#pragma unroll 1
      for (int c = 0; c < 4; c += 2) {
        tc::tmem_ld16(tS + (c + 1) * 16, vb);
        chunk_fn(va, c);
        tc::tmem_wait_ld_regs16(vb);
        if (c + 2 < 4) tc::tmem_ld16(tS + (c + 2) * 16, va);
        else release_s();
        chunk_fn(vb, c + 1);
        if (c + 2 < 4) tc::tmem_wait_ld_regs16(va);
      }
    };
    for (int j = 0; j < nK && ok; ++j, ++i) {
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars->s_full[t], i & 1, abort_flag, p.err, kErrTimeoutSoftmax));
      if (!ok) break;
      tc::tc_fence_after();
      const int mode = tile_mode(j);
      auto run = [&](auto mode_c) {
        sweep([&](const uint32_t (&v)[16], int c) { pass1_chunk(mode_c, v, j * kBN + kh + 16 * c, 4 * j + c); });
      };
      if (mode == kFast) run(IntC<kFast>{});
      else if (mode == kLimited) run(IntC<kLimited>{});
      else run(IntC<kGeneral>{});
    }
    // row max over both halves
    float m = fmaxf(mraw * p.scale, mlim);
    xm[hc * kBM + r] = m;
    tc::named_barrier_sync(1 + t, 256);
    m = fmaxf(m, xm[(hc ^ 1) * kBM + r]);
    if (!row_ok) m = 0.f;
    // the value a fast chunk's raw score must equal to be the max (NaN: none)
    const float traw = mraw * p.scale == m ? mraw : __int_as_float(0x7fc00000);
    int amax = INT_MAX;            // first key of this half whose score is the max
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
    // q for a pair of scores on packed fp32 pairs (fast chunks)
    float2 cyp[TAU_POLY_DEG + 1];
    {
      const float g0[] = TAU_POLY_G_COEFFS, h0[] = TAU_POLY_H_COEFFS;
#pragma unroll
      for (int u = 0; u <= TAU_POLY_DEG; ++u) {
        const float yc = SIG == TAU_DXB_SIGMA_SIGMOID ? -tau * h0[u] : tau * g0[u];
        cyp[u] = make_float2(yc, yc);
      }
    }
    const float2 tau2 = make_float2(tau, tau), sa22 = make_float2(sa2, sa2), nma22 = make_float2(-ma2, -ma2);
    auto qval2 = [&](float2 raw2) -> float2 {
      const float2 a2 = tc::fma2(raw2, sa22, nma22);
      float2 y;
      if (SIG == TAU_DXB_SIGMA_SOFTPLUS || SIG == TAU_DXB_SIGMA_SIGMOID) {
        const float2 ex = make_float2(tc::ex2(a2.x), tc::ex2(a2.y));
        float2 acc = cyp[TAU_POLY_DEG];
#pragma unroll
        for (int u = TAU_POLY_DEG - 1; u >= 0; --u) acc = tc::fma2(acc, ex, cyp[u]);
        y = tc::fma2(tau2, a2, acc);
      } else if (SIG == TAU_DXB_SIGMA_EXP) {
        y = tc::mul2(tau2, a2);
      } else {
        y = make_float2(ylo, ylo);
      }
      return make_float2(tc::ex2(fmaxf(y.x, ylo)), tc::ex2(fmaxf(y.y, ylo)));
    };
    int j2 = 0;                    // key tile of the current pass-2 step
    auto pass2_chunk = [&](auto mode_c, const uint32_t (&v)[16], int c, int key0, int cid) {
      constexpr int kMode = decltype(mode_c)::value;
      uint32_t pk[8];
      uint32_t eq = 0;             // keys of this chunk whose score equals the max
      float2 l2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        if constexpr (kMode == kFast) {
          const float2 q2 = qval2(make_float2(__uint_as_float(v[e]), __uint_as_float(v[e + 1])));
          l2 = tc::add2(l2, q2);
          pk[e >> 1] = tc::pack_bf16(q2.x, q2.y);
          continue;
        }
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
            eq |= tc::eq_mask(score_x(mode_c, raw, key), m) & (1u << (e + u));
          } else {
            // unmasked scores as in the fast path, masked ones as in the limited path
            const float mv = row_ok ? fwd_mask_value(p, b, h, grow, key) : 0.f;
            const float a2 = mv == 0.f ? fmaf(raw, sa2, -ma2) : (raw * p.scale + mv - m) * al2;
            const float qv = qval(a2);
            qq[u] = key < p.Lk ? qv : 0.f;
            eq |= tc::eq_mask(key < p.Lk ? raw * p.scale + mv : -INFINITY, m) & (1u << (e + u));
          }
        }
        l0 += qq[0];
        l1 += qq[1];
        pk[e >> 1] = tc::pack_bf16(qq[0], qq[1]);
      }
      l0 += l2.x;
      l1 += l2.y;
      if constexpr (kMode == kFast) {
        if (cid == mchunk) {             // the chunk that holds this half's first fast max
          // bit e of the sum = (raw_e == traw); 1.0 / 0.0 flags, FMA-pipe accumulation
          float acc = 0.f;
#pragma unroll
          for (int e = 0; e < 16; ++e) acc = fmaf(tc::eq_flag(__uint_as_float(v[e]), traw), float(1 << e), acc);
          eq = __float_as_uint(acc + 8388608.f) & 0xFFFFu;
        }
      }
      if (eq != 0 && amax == INT_MAX) amax = key0 + __ffs(eq) - 1;
      if (c == 0 && j2 > 0) {
        // the PV MMA of the previous key tile must be done reading P
        ok = __all_sync(0xffffffffu, ok && tc::mbar_wait(&bars->pv_done[t], (j2 - 1) & 1, abort_flag,
                                                          p.err, kErrTimeoutSoftmax));
        tc::tc_fence_after();
      }
      // 16 keys -> 2 x 16-byte chunks of this half's 128B-swizzled K-major atom
      uint8_t* rowp = Pt + r * 128;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int chunk = (c * 2 + u) ^ (r & 7);
        *reinterpret_cast<uint4*>(rowp + chunk * 16) =
            make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
      }
    };
    for (int j = 0; j < nK && ok; ++j, ++i) {
      ok = __all_sync(0xffffffffu, tc::mbar_wait(&bars->s_full[t], i & 1, abort_flag, p.err, kErrTimeoutSoftmax));
      if (!ok) break;
      tc::tc_fence_after();
      const int mode = tile_mode(j);
      j2 = j;
      auto run = [&](auto mode_c) {
        sweep([&](const uint32_t (&v)[16], int c) { pass2_chunk(mode_c, v, c, j * kBN + kh + 16 * c, 4 * j + c); });
      };
      if (mode == kFast) run(IntC<kFast>{});
      else if (mode == kLimited) run(IntC<kLimited>{});
      else run(IntC<kGeneral>{});
      tc::fence_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars->sp_ready[t]);
    }
    // row sum and first argmax over both halves
    xl[hc * kBM + r] = l0 + l1;
    xa[hc * kBM + r] = amax;
    tc::named_barrier_sync(1 + t, 256);
    const float l = xl[hc * kBM + r] + xl[(hc ^ 1) * kBM + r] +
                    (n_skip ? static_cast<float>(n_skip) * tc::ex2(ylo) : 0.f);
    amax = min(amax, xa[(hc ^ 1) * kBM + r]);
    if (amax == INT_MAX) amax = 0;
    // epilogue: O / Z, this half's 32 output columns
    if (ok) ok = tc::mbar_wait(&bars->o_full[t], 0, abort_flag, p.err, kErrTimeoutSoftmax);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc::tc_fence_after();
      uint32_t o0[32];
      tc::tmem_ld32(tO, o0);
      tc::tmem_wait_ld_regs(o0);
      const float Z = fmaxf(l, kClampMin);
      const float rz = 1.f / Z;
      if (row_ok) {
        __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(p.out) + b * p.os[0] + h * p.os[1] +
                              static_cast<int64_t>(grow) * p.os[2] + hc * 32;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 w;
          w.x = tc::pack_bf16(__uint_as_float(o0[8 * u + 0]) * rz, __uint_as_float(o0[8 * u + 1]) * rz);
          w.y = tc::pack_bf16(__uint_as_float(o0[8 * u + 2]) * rz, __uint_as_float(o0[8 * u + 3]) * rz);
          w.z = tc::pack_bf16(__uint_as_float(o0[8 * u + 4]) * rz, __uint_as_float(o0[8 * u + 5]) * rz);
          w.w = tc::pack_bf16(__uint_as_float(o0[8 * u + 6]) * rz, __uint_as_float(o0[8 * u + 7]) * rz);
          reinterpret_cast<uint4*>(orow)[u] = w;
        }
        if (hc == 0) {
          const int64_t ri = (static_cast<int64_t>(b) * p.H + h) * p.Lq + grow;
          p.row_max[ri] = m;
          p.row_z[ri] = Z;
          p.row_argmax[ri] = amax;
        }
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
