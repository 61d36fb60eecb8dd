// tau-opus attention backward, tensor-core path for sm_100a (bf16, D = 64).
//
// A CTA owns a 128-key tile of one (b, h) at a time and streams every 128-row
// query tile through it (K, V loaded once; Q_i, dO_i and the row statistics in a
// three-stage TMA ring, so the loads for tile i+2 are in flight while tile i
// is processed):
//   S^T  = K Q_i^T          (M=128 keys, N=128 queries, K=64)   -> TMEM [0,128)
//   dP^T = V dO_i^T         (M=128,      N=128,         K=64)   -> TMEM [128,256)
//   elementwise, one thread per key row: P = q / Z and
//     F = tau alpha P (dP - D) sigma'/sigma   (the reference's d_s_stable before
//     the argmax shift, echo/stau_opus_operator.py:134-137); P^T goes to TMEM
//     [448,512) as packed bf16, dS^T = F^T / (tau alpha) to a double-buffered
//     128B-swizzled shared-memory tile; dtau / dalpha stay in registers.
//     The per-head factor tau alpha is applied once, to dQ, dK and rowsum(F),
//     by the epilogue warps, which also reduce rowsum_keys(F) from the dS^T tile.
//   dV  += P^T dO_i         (M=128 keys, N=64, K=128 queries; A from TMEM) -> [256,320)
//   dK  += dS^T Q_i         (A = dS^T K-major in shared memory)            -> [320,384)
//   dQ_i = dS K             (M=128 queries; the same dS^T tile as MN-major A) -> [384,448)
//   dQ_i leaves through TMA bulk reduce-adds into the fp32 dQ accumulator,
//   32 columns at a time through one 16 KB staging box.
// Warp roles (24 warps): 0 TMA, 1 MMA + TMEM owner, 2 row statistics of each
// query tile, 4-7 dQ epilogue (and each item's dK / dV store), 8-23 elementwise
// (four groups of 4 warps, 32 query columns each).
// The grid is persistent: one CTA per SM loops over (b, h, key tile) items.
// The next item's K / V (second buffer) and first query tiles load, and its
// first S / dP tiles are computed, while the previous item's dK / dV leave TMEM.
// The argmax correction, dK scaling and dtype casts run afterwards in the
// shared epilogue kernels (attn_common.cu).

#include "attn.h"
#include "poly_coeffs.h"
#include "tc_common.cuh"

namespace taudxb {

bool make_tmap_f32_rows64(CUtensorMap* map, void* base, int64_t rows, int64_t planes, int box_rows) {
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
  const cuuint64_t gdim[3] = {64, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(planes)};
  const cuuint64_t gstride[2] = {64 * 4, static_cast<cuuint64_t>(rows) * 64 * 4};
  const cuuint32_t box[3] = {32, static_cast<cuuint32_t>(box_rows), 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled (fp32) failed (%d)", static_cast<int>(r));
    return false;
  }
  return true;
}

namespace {

constexpr int kT = 128, kD = 64, kThreads = 768;   // 24 warps
constexpr int kComputeWarps = 16;
constexpr uint32_t kTile = kT * kD * 2;       // 16 KB bf16 tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLog2Clamp = -26.575424759098897f;   // log2(1e-8)
constexpr int kErrTimeoutTma = 1, kErrTimeoutMma = 2, kErrTimeoutCompute = 4;
constexpr int kQStages = 3;      // Q / dO / row-statistics ring
constexpr int kKVBufs = 2;       // K / V of consecutive items
constexpr int kDSBufs = 1;       // dS^T tiles (2 atoms of 64 queries each)
// registers per thread after setmaxnreg: producer warpgroup (TMA, MMA, row
// statistics), epilogue warpgroup, elementwise warps
constexpr int kRegProducer = 64, kRegEpilogue = 64, kRegCompute = 88;

struct BwdParams {
  CUtensorMap tq, tk, tv, tdo, tdq;
  int B, H, Lq, Lk;
  const float* tau;
  const float* alpha;
  float scale;
  int causal;
  const void* mask; int mask_dtype; int64_t ms[4];
  const float* row_max; const float* row_z; const float* drow;
  float* ws_rowf; float* ws_dk;
  void* dv; int64_t dvs[4];
  float* dtau; float* dalpha;
  int* err;
  int n_items;              // (b, h, key tile) work items
};

struct __align__(8) BwdBarriers {
  uint64_t kv_full[kKVBufs];
  uint64_t qd_full[kQStages];
  uint64_t qd_empty[kQStages];
  uint64_t s_full;
  uint64_t s_free;
  uint64_t ds_ready;
  uint64_t p_free;        // dV MMA done with P^T in TMEM
  uint64_t ds_free[kDSBufs];      // dK / dQ MMAs and the rowsum readers done with dS^T buffer b
  uint64_t ds_full_epi[kDSBufs];  // dS^T buffer b written (for the epilogue's rowsum)
  uint64_t dq_full;
  uint64_t dq_free;
  uint64_t fin[kKVBufs];  // an item's MMAs are done (its K / V buffer free; dK, dV complete)
  uint64_t acc_free;      // the epilogue has read an item's dK, dV out of TMEM
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  float red_tau[2], red_alpha[2];   // per-item sums of the elementwise warps (by item parity)
};

constexpr uint32_t kOffK = 0;                             // kKVBufs buffers
constexpr uint32_t kOffV = kOffK + kKVBufs * kTile;       // kKVBufs buffers
constexpr uint32_t kOffQ = kOffV + kKVBufs * kTile;       // kQStages stages
constexpr uint32_t kOffDO = kOffQ + kQStages * kTile;     // kQStages stages
constexpr uint32_t kOffDS = kOffDO + kQStages * kTile;    // dS^T, kDSBufs buffers x 2 atoms of 64 queries
constexpr uint32_t kOffStage = kOffDS + kDSBufs * 2 * kTile;   // dQ staging, one box [128][32] fp32
constexpr uint32_t kOffStats = kOffStage + kTile;         // kQStages x {mc, rz, dq} x 128 fp32
constexpr uint32_t kOffBar = kOffStats + kQStages * 3 * kT * 4;
constexpr uint32_t kBwdSmem = kOffBar + sizeof(BwdBarriers) + 1024;
static_assert(kBwdSmem <= 227 * 1024, "backward shared memory above the 227 KB a CTA may use");

constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 320, kColDQ = 384, kColP = 448;

__device__ __forceinline__ float bwd_mask_value(const BwdParams& p, int b, int h, int r, int c) {
  float mv = 0.f;
  if (p.mask) {
    const int64_t off = b * p.ms[0] + h * p.ms[1] + static_cast<int64_t>(r) * p.ms[2] +
                        static_cast<int64_t>(c) * p.ms[3];
    mv = load_as_float(p.mask, p.mask_dtype, off);
  }
  if (p.causal && c > r + (p.Lk - p.Lq)) mv += kMaskMin;
  return mv;
}

template <bool B> struct BoolC { static constexpr bool value = B; };

// Horner's rule on packed pairs, coefficients in increasing degree
template <int N>
__device__ __forceinline__ float2 horner2(const float2 (&c)[N], float2 x) {
  float2 acc = c[N - 1];
#pragma unroll
  for (int i = N - 2; i >= 0; --i) acc = tc::fma2(acc, x, c[i]);
  return acc;
}

// One work item: the 128-key tile k0 of (b, h), with the query tiles
// qt0 .. qt0 + nQ - 1 streamed past it.
struct BwdItem {
  int b, h, k0, qt0, nQ;
  int64_t bh;
};

__device__ __forceinline__ BwdItem bwd_item(const BwdParams& p, int it) {
  BwdItem t;
  const bool causal_only = p.causal && !p.mask && p.Lq <= p.Lk;
  int bhi, kt;
  if (causal_only) {
    // longest items first (key tile 0 of every (b, h), then key tile 1, ...):
    // CTAs that take items round-robin end up with near-equal work
    const int nbh = p.B * p.H;
    kt = it / nbh;
    bhi = it - kt * nbh;
  } else {
    // the key tiles of one (b, h) together: they read the same Q and dO
    const int nkt = (p.Lk + kT - 1) / kT;
    bhi = it / nkt;
    kt = it - bhi * nkt;
  }
  t.k0 = kt * kT;
  t.b = bhi / p.H;
  t.h = bhi - t.b * p.H;
  t.bh = bhi;
  // Built-in causal mask (no mask tensor): query tiles whose every row sees
  // none of this item's keys are skipped. Their masked scores carry only the
  // reference's floor q = 1e-8 per key, so their share of every gradient is
  // below 1e-8 of the row's weight (under the bf16 rounding of P).
  // (Lq <= Lk only: with Lq > Lk the first rows see no key at all, and the
  // reference gives such rows uniform weights that are not negligible.)
  t.qt0 = 0;
  if (p.causal && !p.mask && p.Lq <= p.Lk) {
    const int lim = t.k0 - (p.Lk - p.Lq);      // rows >= lim see key k0
    t.qt0 = lim > 0 ? lim / kT : 0;
  }
  t.nQ = (p.Lq + kT - 1) / kT - t.qt0;
  return t;
}

// tau and alpha of item it (zeros past the last item): loaded one item ahead,
// so the loads are not on the path into the next item
__device__ __forceinline__ float2 bwd_item_tau_alpha(const BwdParams& p, int it) {
  if (it >= p.n_items) return make_float2(0.f, 0.f);
  const int h = bwd_item(p, it).h;
  return make_float2(p.tau[h], p.alpha[h]);
}

// Each CTA takes the items blockIdx.x, blockIdx.x + gridDim.x, ... (one per
// CTA when the grid covers them all; one CTA per SM otherwise). Every role
// counts the query tiles it has passed over all of its items (g), and the
// per-tile barriers' phases follow that count, so the next item's loads,
// S / dP MMAs and elementwise work start while the previous item's dK / dV
// are still being stored.
template <int SIG>
__global__ void __launch_bounds__(kThreads, 1) attn_bwd_tc_kernel(const __grid_constant__ BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base by pointer arithmetic on the __shared__ array, so the
  // compiler keeps every derived pointer in the shared address space
  uint8_t* smem = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  BwdBarriers* bars = reinterpret_cast<BwdBarriers*>(smem + kOffBar);
  float* stats = reinterpret_cast<float*>(smem + kOffStats);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool causal_only = p.causal && !p.mask && p.Lq <= p.Lk;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kKVBufs; ++s) {
      tc::mbar_init(&bars->kv_full[s], 1);
      tc::mbar_init(&bars->fin[s], 1);
    }
    for (int s = 0; s < kQStages; ++s) {
      tc::mbar_init(&bars->qd_full[s], 2);               // TMA bytes + row-statistics warp
      tc::mbar_init(&bars->qd_empty[s], 1);
    }
    for (int s = 0; s < kDSBufs; ++s) {
      tc::mbar_init(&bars->ds_free[s], 1 + 4);          // MMA commit + 4 epilogue warps
      tc::mbar_init(&bars->ds_full_epi[s], kComputeWarps);
    }
    tc::mbar_init(&bars->s_full, 1);
    tc::mbar_init(&bars->s_free, kComputeWarps);
    tc::mbar_init(&bars->ds_ready, kComputeWarps);
    tc::mbar_init(&bars->p_free, 1);
    tc::mbar_init(&bars->dq_full, 1);
    tc::mbar_init(&bars->dq_free, 4);
    tc::mbar_init(&bars->acc_free, 4);
    tc::mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    bars->red_tau[0] = bars->red_tau[1] = bars->red_alpha[0] = bars->red_alpha[1] = 0.f;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) { tc::tmem_alloc(&bars->tmem_base, 512); tc::tmem_relinquish(); }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  // Register split of the 80 x 768 launched: producer warpgroup (warps 0-3)
  // and epilogue warpgroup 64 per thread, elementwise warps 88
  // (64*128 + 64*128 + 88*512 = 61440; 48 / 48 / 96 spilled in the producer
  // and epilogue warps). Each warpgroup's code is reached only through its own
  // setmaxnreg, so the compiler allocates each to its limit.
  static_assert(kRegProducer * 128 + kRegEpilogue * 128 + kRegCompute * 512 <= 80 * kThreads, "register split");
  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" :: "n"(kRegProducer) : "memory");
  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      int issued = 0, kv_items = 0;      // query tiles / K-V pairs whose loads were issued
      bool ok = true;
      for (int it = blockIdx.x, n = 0, g = 0; it < p.n_items && ok; it += gridDim.x, ++n) {
        const BwdItem t = bwd_item(p, it);
        const int kvb = n % kKVBufs;
        // buffer kvb held the K and V of item n - kKVBufs until its last MMAs (fin)
        if (n >= kKVBufs &&
            !tc::mbar_wait(&bars->fin[kvb], (n / kKVBufs - 1) & 1, abort_flag, p.err, kErrTimeoutTma))
          break;
        tc::mbar_arrive_expect_tx(&bars->kv_full[kvb], 2 * kTile);
        tc::tma_load_4d(smem + kOffK + kvb * kTile, &p.tk, &bars->kv_full[kvb], 0, t.k0, t.h, t.b);
        tc::tma_load_4d(smem + kOffV + kvb * kTile, &p.tv, &bars->kv_full[kvb], 0, t.k0, t.h, t.b);
        kv_items = n + 1;
        for (int i = 0; i < t.nQ; ++i, ++g) {   // stage s of tile g, ph = (g / kQStages) & 1
          const int s = g % kQStages, ph = (g / kQStages) & 1;
          if (g >= kQStages && !tc::mbar_wait(&bars->qd_empty[s], ph ^ 1, abort_flag, p.err, kErrTimeoutTma)) {
            ok = false;
            break;
          }
          tc::mbar_arrive_expect_tx(&bars->qd_full[s], 2 * kTile);
          tc::tma_load_4d(smem + kOffQ + s * kTile, &p.tq, &bars->qd_full[s], 0, (t.qt0 + i) * kT, t.h, t.b);
          tc::tma_load_4d(smem + kOffDO + s * kTile, &p.tdo, &bars->qd_full[s], 0, (t.qt0 + i) * kT, t.h, t.b);
          issued = g + 1;
        }
      }
      if (*abort_flag) {   // let started copies land before the CTA exits
        const uint64_t t0 = tc::globaltimer_ns();
        for (int i = (issued > kQStages ? issued - kQStages : 0); i < issued; ++i) {
          const uint32_t a = tc::smem_u32(&bars->qd_full[i % kQStages]);
          while (!tc::mbar_try_wait(a, (i / kQStages) & 1) && tc::globaltimer_ns() - t0 < tc::kWaitLimitNs) {
          }
        }
        for (int n = (kv_items > kKVBufs ? kv_items - kKVBufs : 0); n < kv_items; ++n) {
          const uint32_t a = tc::smem_u32(&bars->kv_full[n % kKVBufs]);
          while (!tc::mbar_try_wait(a, (n / kKVBufs) & 1) && tc::globaltimer_ns() - t0 < tc::kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idS = tc::idesc_bf16(kT, kT, 0, 0);
      constexpr uint32_t idG = tc::idesc_bf16(kT, kD, 0, 1);
      constexpr uint32_t idQ = tc::idesc_bf16(kT, kD, 1, 1);
      // descriptor low halves; K-major operands step 32 B (2) per K slice of 16,
      // MN-major ones 2048 B (128), the high half is the same for both layouts
      constexpr uint32_t hi = tc::sdesc_hi_sw128(1024);
      const uint32_t sK = tc::smem_u32(smem + kOffK), sV = tc::smem_u32(smem + kOffV);
      const uint32_t sQ = tc::smem_u32(smem + kOffQ), sDO = tc::smem_u32(smem + kOffDO);
      const uint32_t sDS = tc::smem_u32(smem + kOffDS);
      const uint32_t kK = tc::sdesc_lo(sK, 16), kV = tc::sdesc_lo(sV, 16), mK = tc::sdesc_lo(sK, 16384);
      constexpr uint32_t tileStep = kTile >> 4;
      // One stream of query tiles over all items: S / dP of tile g, then the
      // dV / dK / dQ of tile g - 1 (possibly the previous item's last), so the
      // tensor pipe runs on across item boundaries.
      struct Prev { int g, kvb, item; bool first, last; };
      Prev pv = {-1, 0, 0, false, false};
      bool ok = true;
      auto tail = [&](const Prev& q) -> bool {      // dV / dK / dQ of tile q.g
        const int gj = q.g, sj = gj % kDSBufs, qj = gj % kQStages;
        bool w = tc::mbar_wait(&bars->ds_ready, gj & 1, abort_flag, p.err, kErrTimeoutMma);
        if (w && gj > 0) w = tc::mbar_wait(&bars->dq_free, (gj - 1) & 1, abort_flag, p.err, kErrTimeoutMma);
        // an item's first dV / dK MMA overwrites the accumulators: the
        // epilogue must have read the previous item's out of TMEM
        if (w && q.first && q.item > 0)
          w = tc::mbar_wait(&bars->acc_free, (q.item - 1) & 1, abort_flag, p.err, kErrTimeoutMma);
        if (!w) return false;
        tc::tc_fence_after();
        const uint32_t mDO = tc::sdesc_lo(sDO, 16384) + qj * tileStep;
        const uint32_t mQ = tc::sdesc_lo(sQ, 16384) + qj * tileStep;
        const uint32_t kDS = tc::sdesc_lo(sDS, 16) + sj * 2 * tileStep;
        const uint32_t mDS = tc::sdesc_lo(sDS, 16384) + sj * 2 * tileStep;
        const uint32_t mKb = mK + q.kvb * tileStep;
        const bool acc0 = !q.first;
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk)      // dV += P^T dO_j, P^T from TMEM
          tc::umma_f16_ts2(tmem + kColDV, tmem + kColP + kk * 8, mDO + 128 * kk, hi, idG, acc0 || kk > 0);
        tc::umma_commit(&bars->p_free);
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk)      // dK += dS^T Q_j
          tc::umma_f16_ss2(tmem + kColDK, kDS + (kk >> 2) * tileStep + (kk & 3) * 2, hi, mQ + 128 * kk, hi,
                           idG, acc0 || kk > 0);
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk)      // dQ_j = dS K
          tc::umma_f16_ss2(tmem + kColDQ, mDS + 128 * kk, hi, mKb + 128 * kk, hi, idQ, kk > 0);
        tc::umma_commit(&bars->ds_free[sj]);
        tc::umma_commit(&bars->qd_empty[qj]);
        tc::umma_commit(&bars->dq_full);
        if (q.last) tc::umma_commit(&bars->fin[q.kvb]);   // the item's K / V buffer, dK and dV are done
        return true;
      };
      for (int it = blockIdx.x, n = 0, g = 0; it < p.n_items && ok; it += gridDim.x, ++n) {
        const int nQ = bwd_item(p, it).nQ, kvb = n % kKVBufs;
        // with one K / V buffer, the previous item's last MMAs must free it first
        if (kKVBufs == 1 && pv.g >= 0) {
          ok = tail(pv);
          pv.g = -1;
          if (!ok) break;
        }
        ok = tc::mbar_wait(&bars->kv_full[kvb], (n / kKVBufs) & 1, abort_flag, p.err, kErrTimeoutMma);
        const uint32_t kKb = kK + kvb * tileStep, kVb = kV + kvb * tileStep;
        for (int i = 0; i < nQ && ok; ++i, ++g) {
          const int s = g % kQStages, ph = (g / kQStages) & 1;
          ok = tc::mbar_wait(&bars->qd_full[s], ph, abort_flag, p.err, kErrTimeoutMma);
          if (ok && g > 0) ok = tc::mbar_wait(&bars->s_free, (g - 1) & 1, abort_flag, p.err, kErrTimeoutMma);
          if (!ok) break;
          tc::tc_fence_after();
          const uint32_t kQ = tc::sdesc_lo(sQ, 16) + s * tileStep, kDO = tc::sdesc_lo(sDO, 16) + s * tileStep;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            tc::umma_f16_ss2(tmem + kColS, kKb + 2 * kk, hi, kQ + 2 * kk, hi, idS, kk > 0);
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            tc::umma_f16_ss2(tmem + kColDP, kVb + 2 * kk, hi, kDO + 2 * kk, hi, idS, kk > 0);
          tc::umma_commit(&bars->s_full);
          if (pv.g >= 0) ok = tail(pv);
          pv = {g, kvb, n, i == 0, i == nQ - 1};
        }
      }
      if (ok && pv.g >= 0) tail(pv);
      tc::umma_commit(&bars->drain);
      const uint64_t t0 = tc::globaltimer_ns();
      const uint32_t a = tc::smem_u32(&bars->drain);
      while (!tc::mbar_try_wait(a, 0) && tc::globaltimer_ns() - t0 < tc::kWaitLimitNs) {
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- row statistics
    bool ok = true;
    for (int it = blockIdx.x, n = 0, g = 0; it < p.n_items && ok; it += gridDim.x, ++n) {
      const BwdItem t = bwd_item(p, it);
      for (int i = 0; i < t.nQ; ++i, ++g) {
        const int s = g % kQStages, ph = (g / kQStages) & 1;
        if (g >= kQStages && !__all_sync(0xffffffffu, tc::mbar_wait(&bars->qd_empty[s], ph ^ 1,
                                                                     abort_flag, p.err, kErrTimeoutTma))) {
          ok = false;
          break;
        }
        float* st = stats + s * 3 * kT;
        // all 12 loads of this lane in flight at once (one round of global latency)
        float m4[4], z4[4], d4[4];
        const float al2 = p.alpha[t.h] * kLog2e;     // (in flight with the row loads)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int q = (t.qt0 + i) * kT + lane + 32 * u;
          const int64_t ri = t.bh * p.Lq + (q < p.Lq ? q : 0);
          m4[u] = p.row_max[ri];
          z4[u] = p.row_z[ri];
          d4[u] = p.drow[ri];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int r = lane + 32 * u;
          const bool q_ok = (t.qt0 + i) * kT + r < p.Lq;
          st[r] = q_ok ? -m4[u] * al2 : 0.f;
          st[kT + r] = q_ok ? 1.f / z4[u] : 0.f;
          st[2 * kT + r] = q_ok ? -d4[u] : 0.f;       // -D: t = P (dP + (-D)), no negation per score
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars->qd_full[s]);
      }
    }
  }
  } else if (warp < 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" :: "n"(kRegEpilogue) : "memory");
    // ---------------------------------------------------------------- dQ epilogue
    // One thread per query row; dQ_j's 64 TMEM columns in two halves of 32,
    // each scaled by tau*alpha, staged in one 128B-swizzled box and sent with
    // a TMA bulk reduce-add (thread 128 issues it and waits for the box to be
    // read before it is refilled). After an item's last tile: its dK / dV.
    const int r = ((warp & 3) << 5) + lane;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) << 5) << 16;
    uint8_t* stage = smem + kOffStage;
    bool ok = true;
    float2 nx = bwd_item_tau_alpha(p, blockIdx.x);
    for (int it = blockIdx.x, n = 0, g = 0; it < p.n_items && ok; it += gridDim.x, ++n) {
      const BwdItem t = bwd_item(p, it);
      const float ta = nx.x * nx.y;
      nx = bwd_item_tau_alpha(p, it + gridDim.x);
      for (int j = 0; j < t.nQ && ok; ++j) {
        const int gj = g + j;
        // rowsum_keys(F) of query r from the bf16 dS^T tile (key rows, 128B-swizzled)
        // (first, so the dS^T buffer is released early; one decision for the
        // whole group, which meets again at named barriers below)
        ok = tc::named_barrier_and(1, 128, tc::mbar_wait(&bars->ds_full_epi[gj % kDSBufs], (gj / kDSBufs) & 1,
                                                          abort_flag, p.err, kErrTimeoutCompute));
        if (!ok) break;
        // thread r: 8 queries (16-byte chunk c8 of 64-query atom r>>6) over the
        // 16 key rows kp, kp+8, ...; in a 128B-swizzled row k the chunk sits at
        // c8 ^ (k & 7) = c8 ^ kp, the same for all 16 rows
        const int c8 = (r >> 3) & 7, kp = r & 7;
        const uint8_t* dsb = smem + kOffDS + (gj % kDSBufs) * 2 * kTile + (r >> 6) * kTile + kp * 128 + ((c8 ^ kp) << 4);
        float2 cs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int m = 0; m < kT / 8; ++m) {
          const uint4 w = *reinterpret_cast<const uint4*>(dsb + m * 1024);
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int u = 0; u < 4; ++u)
            cs[u] = tc::add2(cs[u], make_float2(__uint_as_float(ws[u] << 16), __uint_as_float(ws[u] & 0xffff0000u)));
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars->ds_free[gj % kDSBufs]);
        // reduce over the 8 lanes kp = 0..7 of this chunk; lane kp ends with query 8 c8 + kp
        float v[8] = {cs[0].x, cs[0].y, cs[1].x, cs[1].y, cs[2].x, cs[2].y, cs[3].x, cs[3].y};
#pragma unroll
        for (int lvl = 4; lvl >= 1; lvl >>= 1) {
          const bool upper = (kp & lvl) != 0;
#pragma unroll
          for (int u = 0; u < lvl; ++u) {
            const float send = upper ? v[u] : v[u + lvl];
            const float keep = upper ? v[u + lvl] : v[u];
            v[u] = keep + __shfl_xor_sync(0xffffffffu, send, lvl);
          }
        }
        {
          const int q = (t.qt0 + j) * kT + (r >> 6) * 64 + c8 * 8 + kp;
          if (q < p.Lq) atomicAdd(p.ws_rowf + t.bh * p.Lq + q, v[0] * ta);
        }
        // dQ_j
        ok = tc::named_barrier_and(1, 128, tc::mbar_wait(&bars->dq_full, gj & 1, abort_flag, p.err,
                                                         kErrTimeoutCompute));
        if (!ok) break;
        tc::tc_fence_after();
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t a[32];
          tc::tmem_ld32(tmem + lane_base + kColDQ + 32 * half, a);
          tc::tmem_wait_ld_regs(a);
          if (half == 1) {         // every TMEM read of dQ_j is done
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bars->dq_free);
          }
          // the previous reduce must have finished reading the box
          if (threadIdx.x == 128) tc::bulk_wait_group_read0();
          tc::named_barrier_sync(1, 128);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int pc = (u ^ (r & 7)) << 4;
            *reinterpret_cast<float4*>(stage + r * 128 + pc) =
                make_float4(__uint_as_float(a[4 * u]) * ta, __uint_as_float(a[4 * u + 1]) * ta,
                            __uint_as_float(a[4 * u + 2]) * ta, __uint_as_float(a[4 * u + 3]) * ta);
          }
          tc::fence_async_smem();
          tc::named_barrier_sync(1, 128);
          if (threadIdx.x == 128) {
            tc::tma_reduce_add_3d(&p.tdq, stage, 32 * half, (t.qt0 + j) * kT, static_cast<int>(t.bh));
            tc::bulk_commit_group();
          }
        }
      }
      g += t.nQ;
      // this item's dK / dV (one thread per key row)
      // (all four warps decide together: each of them meets the others at named barriers again)
      ok = tc::named_barrier_and(1, 128, ok && tc::mbar_wait(&bars->fin[n % kKVBufs], (n / kKVBufs) & 1, abort_flag, p.err,
                                                             kErrTimeoutCompute));
      if (!ok) break;
      tc::tc_fence_after();
      const BwdItem u = bwd_item(p, it);        // recomputed: not held over the tile loop
      const int key = u.k0 + r;
      __nv_bfloat16* dvrow = static_cast<__nv_bfloat16*>(p.dv) + u.b * p.dvs[0] + u.h * p.dvs[1] +
                             static_cast<int64_t>(key) * p.dvs[2];
      float4* dkrow = reinterpret_cast<float4*>(p.ws_dk + (u.bh * p.Lk + key) * kD);
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t v[32];
        tc::tmem_ld32(tmem + lane_base + kColDV + 32 * half, v);
        tc::tmem_wait_ld_regs(v);
        if (key < p.Lk) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint4 w;
            w.x = tc::pack_bf16(__uint_as_float(v[8 * u]), __uint_as_float(v[8 * u + 1]));
            w.y = tc::pack_bf16(__uint_as_float(v[8 * u + 2]), __uint_as_float(v[8 * u + 3]));
            w.z = tc::pack_bf16(__uint_as_float(v[8 * u + 4]), __uint_as_float(v[8 * u + 5]));
            w.w = tc::pack_bf16(__uint_as_float(v[8 * u + 6]), __uint_as_float(v[8 * u + 7]));
            reinterpret_cast<uint4*>(dvrow)[4 * half + u] = w;
          }
        }
        tc::tmem_ld32(tmem + lane_base + kColDK + 32 * half, v);
        tc::tmem_wait_ld_regs(v);
        if (half == 1) {         // every TMEM read of this item's dK / dV is done
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&bars->acc_free);
        }
        if (key < p.Lk) {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            dkrow[8 * half + u] = make_float4(__uint_as_float(v[4 * u]) * ta, __uint_as_float(v[4 * u + 1]) * ta,
                                              __uint_as_float(v[4 * u + 2]) * ta, __uint_as_float(v[4 * u + 3]) * ta);
        }
      }
    }
    if (threadIdx.x == 128) tc::bulk_wait_group0();
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" :: "n"(kRegCompute) : "memory");
    // ---------------------------------------------------------------- elementwise
    // Per score: a2 = log2(e) alpha (s scale - m), y = tau log2 sigma,
    // q = 2^max(y, ylo) (both clamps of the reference in one), P = q / Z,
    // t = P (dP - D) (the statistics hold -D), F / (tau alpha) = t sigma'/sigma.
    // Sums kept scaled: acc_tau = sum t tau log2 sigma_clamped and
    // acc_alpha = sum t clip(ratio a2, +-30 log2(e) alpha); the constants are
    // divided out once per item, when each warp adds its sums to dtau / dalpha.
    const int grp = (warp - 8) >> 2;                 // query columns [32 grp, 32 grp + 32)
    const int r = ((warp & 3) << 5) + lane;          // key row = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) << 5) << 16;
    bool ok = true;
    float2 nx = bwd_item_tau_alpha(p, blockIdx.x);
    for (int it = blockIdx.x, n = 0, g = 0; it < p.n_items && ok; it += gridDim.x, ++n) {
      const BwdItem t = bwd_item(p, it);
      const int b = t.b, h = t.h, k0 = t.k0, qt0 = t.qt0, nQ = t.nQ;
      const float tau = nx.x, alpha = nx.y;
      nx = bwd_item_tau_alpha(p, it + gridDim.x);
      const int key = k0 + r;
      const bool key_ok = key < p.Lk;
      const float al2 = alpha * kLog2e;
      const float sa2 = p.scale * al2;
      const float ylo = fmaxf(tau * kLog2Clamp, kLog2Clamp);
      const float ytau = tau * kLog2Clamp;
      const float glim = 30.f * al2;
      const float kmask = key_ok ? 1.f : 0.f;
      const float2 kmask2 = make_float2(kmask, kmask), sa2x2 = make_float2(sa2, sa2);
      const float2 taux2 = make_float2(tau, tau);
      // polynomial coefficients as broadcast pairs: tau log2 sigma = tau a2 + cy(e)
      // (tau folded in; minus for sigmoid's -H) and sigma'/sigma = cr(e)
      float2 cy[TAU_POLY_DEG + 1], cr[TAU_POLY_DEG + 1];
      {
        const bool sg = SIG == TAU_DXB_SIGMA_SIGMOID;
        const float g0[] = TAU_POLY_G_COEFFS, h0[] = TAU_POLY_H_COEFFS;
        const float r0[] = TAU_POLY_R_COEFFS, s0[] = TAU_POLY_S_COEFFS;
#pragma unroll
        for (int u = 0; u <= TAU_POLY_DEG; ++u) {
          const float yc = sg ? -tau * h0[u] : tau * g0[u], rc = sg ? s0[u] : r0[u];
          cy[u] = make_float2(yc, yc);
          cr[u] = make_float2(rc, rc);
        }
      }
      const bool tile_full = k0 + kT <= p.Lk;
      float2 acc_tau = make_float2(0.f, 0.f), acc_alpha = make_float2(0.f, 0.f);
      int qs = g % kQStages, qph = (g / kQStages) & 1;   // stage and phase of tile g in the Q / dO / statistics ring
      // Clean chunks: where every x = alpha (s - m) of the chunk is above
      // a2_clean / log2(e), none of the reference's clamps can act -- sigma and
      // sigma^tau stay >= 1e-8 and sigma'/sigma (s - m) >= -30 (sigma'/sigma <= 1)
      // -- so those chunks skip the three clamps. x_thr solves
      // sigma(x_thr) = max(1e-8^(1/tau), 1e-8); the margin of 0.01 covers the
      // polynomial and ex2 approximation errors.
      float a2_clean = INFINITY;
      if (SIG != TAU_DXB_SIGMA_RELU) {
        const float pth = fmaxf(exp2f(kLog2Clamp / tau), 1e-8f);
        const float x_thr = SIG == TAU_DXB_SIGMA_SOFTPLUS ? logf(expm1f(pth))
                            : SIG == TAU_DXB_SIGMA_SIGMOID ? logf(pth / (1.f - pth)) : logf(pth);
        a2_clean = kLog2e * fmaxf(x_thr + 0.01f, -29.9f * alpha);
      }
      // a2 = log2(e) alpha (s scale - m) of a 16-column chunk; true if the chunk is clean
      auto chunk_a2 = [&](const uint32_t (&rr)[32], int col0, float2 (&a2v)[8]) -> bool {
        const float* stc = stats + qs * 3 * kT;
  #pragma unroll
        for (int e4 = 0; e4 < 16; e4 += 4) {
          const float4 mc4 = *reinterpret_cast<const float4*>(stc + col0 + e4);
          a2v[e4 >> 1] = tc::fma2(make_float2(__uint_as_float(rr[e4]), __uint_as_float(rr[e4 + 1])), sa2x2,
                                  make_float2(mc4.x, mc4.y));
          a2v[(e4 >> 1) + 1] = tc::fma2(make_float2(__uint_as_float(rr[e4 + 2]), __uint_as_float(rr[e4 + 3])),
                                        sa2x2, make_float2(mc4.z, mc4.w));
        }
        // key rows past Lk (zero-filled by TMA, so s = 0 and a2 = -m alpha log2 e)
        // take a2 = 0: their P is zeroed later, and a row max far below 0 would
        // otherwise send the sigma polynomials out of range (inf * 0 = NaN)
        if (!key_ok) {
  #pragma unroll
          for (int u = 0; u < 8; ++u) a2v[u] = make_float2(0.f, 0.f);
        }
        const float m0 = tc::min3(a2v[0].x, a2v[0].y, a2v[1].x), m1 = tc::min3(a2v[1].y, a2v[2].x, a2v[2].y);
        const float m2 = tc::min3(a2v[3].x, a2v[3].y, a2v[4].x), m3 = tc::min3(a2v[4].y, a2v[5].x, a2v[5].y);
        const float m4 = tc::min3(a2v[6].x, a2v[6].y, a2v[7].x);
        const float amin = tc::min3(tc::min3(m0, m1, m2), tc::min3(m3, m4, a2v[7].y), INFINITY);
        return __all_sync(0xffffffffu, amin >= a2_clean);
      };
      auto chunk_math = [&](auto masked_c, auto full_c, auto clean_c, const uint32_t (&rr)[32], int i, int col0,
                            const float2 (&a2v)[8], uint32_t (&pp)[8], uint32_t (&pf)[8]) {
        constexpr bool kMasked = decltype(masked_c)::value, kFull = decltype(full_c)::value;
        constexpr bool kClean = decltype(clean_c)::value;
        const float* stc = stats + qs * 3 * kT;
        float mv[kMasked ? 16 : 1];
        if constexpr (kMasked) {
  #pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int q = (qt0 + i) * kT + col0 + e;
            mv[e] = (key_ok && q < p.Lq) ? bwd_mask_value(p, b, h, q, key) : 0.f;
          }
        }
  #pragma unroll
          for (int e4 = 0; e4 < 16; e4 += 4) {
            const float4 mc4 = kMasked ? *reinterpret_cast<const float4*>(stc + col0 + e4) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 rz4 = *reinterpret_cast<const float4*>(stc + kT + col0 + e4);
            const float4 dq4 = *reinterpret_cast<const float4*>(stc + 2 * kT + col0 + e4);
  #pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {      // a pair of query columns per f32x2 lane pair
              const int e = e4 + 2 * h2;
              const float2 mc = h2 ? make_float2(mc4.z, mc4.w) : make_float2(mc4.x, mc4.y);
              const float2 rz = h2 ? make_float2(rz4.z, rz4.w) : make_float2(rz4.x, rz4.y);
              const float2 dq = h2 ? make_float2(dq4.z, dq4.w) : make_float2(dq4.x, dq4.y);
              float2 a2;
              if constexpr (kMasked) {
                a2 = tc::fma2(make_float2(__uint_as_float(rr[e]), __uint_as_float(rr[e + 1])), sa2x2, mc);
                a2.x = fmaf(mv[e], al2, a2.x);
                a2.y = fmaf(mv[e + 1], al2, a2.y);
                if constexpr (!kFull) {
                  if (!key_ok) a2 = make_float2(0.f, 0.f);   // key rows past Lk, as in chunk_a2
                }
              } else {
                a2 = a2v[e >> 1];
              }
              float2 y, ratio;
              if (SIG == TAU_DXB_SIGMA_SOFTPLUS || SIG == TAU_DXB_SIGMA_SIGMOID) {
                const float2 ex = make_float2(tc::ex2(a2.x), tc::ex2(a2.y));
                y = tc::fma2(taux2, a2, horner2(cy, ex));
                ratio = horner2(cr, ex);
              } else if (SIG == TAU_DXB_SIGMA_EXP) {
                y = tc::mul2(taux2, a2);
                ratio = make_float2(1.f, 1.f);
              } else {
                y = make_float2(ytau, ytau);
                ratio = make_float2(1.f, 1.f);
              }
              float2 P;
              if constexpr (kClean) P = tc::mul2(make_float2(tc::ex2(y.x), tc::ex2(y.y)), rz);
              else P = tc::mul2(make_float2(tc::ex2(fmaxf(y.x, ylo)), tc::ex2(fmaxf(y.y, ylo))), rz);
              if constexpr (!kFull) P = tc::mul2(P, kmask2);
              const float2 t = tc::mul2(P, tc::add2(make_float2(__uint_as_float(rr[16 + e]),
                                                                __uint_as_float(rr[17 + e])), dq));
              const float2 F = tc::mul2(t, ratio);
              if constexpr (kClean) {
                // no clip can act: t ratio a2 = F a2
                acc_tau = tc::fma2(t, y, acc_tau);
                acc_alpha = tc::fma2(F, a2, acc_alpha);
              } else {
                // x = s - rowmax <= 0, so ratio * a2 <= 0: only the lower clip can act
                const float2 ra = tc::mul2(ratio, a2);
                acc_tau = tc::fma2(t, make_float2(fmaxf(y.x, ytau), fmaxf(y.y, ytau)), acc_tau);
                acc_alpha = tc::fma2(t, make_float2(fmaxf(ra.x, -glim), fmaxf(ra.y, -glim)), acc_alpha);
              }
              pp[e >> 1] = tc::pack_bf16(P.x, P.y);
              pf[e >> 1] = tc::pack_bf16(F.x, F.y);
            }
          }
      };
      for (int i = 0; i < nQ && ok; ++i) {
        const int gi = g + i, sb = gi % kDSBufs;
        ok = tc::mbar_wait(&bars->qd_full[qs], qph, abort_flag, p.err, kErrTimeoutCompute);
        ok = ok && tc::mbar_wait(&bars->s_full, gi & 1, abort_flag, p.err, kErrTimeoutCompute);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc::tc_fence_after();
        uint8_t* DSt = smem + kOffDS + sb * 2 * kTile + (grp >> 1) * kTile;   // this group's 64-query atom
        // chunk c = 16 query columns: S^T and dP^T from TMEM, the elementwise math,
        // P^T back to TMEM and dS^T to shared memory. Chunk 1's TMEM loads are
        // issued right after chunk 0's math, so their latency overlaps chunk 0's
        // stores and the wait for the previous tile's MMAs.
        uint32_t rr[32];       // [0,16) scores, [16,32) dP of 16 query columns
        auto chunk = [&](int c) {
          const int col0 = grp * 32 + c * 16;
          uint32_t pp[8], pf[8];
          // branch-free bodies (mask / partial key tile decided per chunk) so the
          // scheduler can interleave the eight column pairs
          float2 a2v[8];
          // with the built-in causal mask only, a chunk none of whose (key,
          // query) pairs of this warp is masked takes the unmasked path
          const bool masked = p.mask != nullptr ||
                              (p.causal && (!causal_only ||
                                            k0 + ((warp & 3) << 5) + 31 > (qt0 + i) * kT + col0 + (p.Lk - p.Lq)));
          if (masked) {
            if (tile_full) chunk_math(BoolC<true>{}, BoolC<true>{}, BoolC<false>{}, rr, i, col0, a2v, pp, pf);
            else chunk_math(BoolC<true>{}, BoolC<false>{}, BoolC<false>{}, rr, i, col0, a2v, pp, pf);
          } else if (chunk_a2(rr, col0, a2v)) {
            if (tile_full) chunk_math(BoolC<false>{}, BoolC<true>{}, BoolC<true>{}, rr, i, col0, a2v, pp, pf);
            else chunk_math(BoolC<false>{}, BoolC<false>{}, BoolC<true>{}, rr, i, col0, a2v, pp, pf);
          } else {
            if (tile_full) chunk_math(BoolC<false>{}, BoolC<true>{}, BoolC<false>{}, rr, i, col0, a2v, pp, pf);
            else chunk_math(BoolC<false>{}, BoolC<false>{}, BoolC<false>{}, rr, i, col0, a2v, pp, pf);
          }
          if (c == 0) {
            // chunk 1's columns in flight while chunk 0 is stored
            tc::tmem_ld16(tmem + lane_base + kColS + col0 + 16, rr);
            tc::tmem_ld16(tmem + lane_base + kColDP + col0 + 16, rr + 16);
            // P^T in TMEM is free once the previous tile's dV MMA is done, the dS^T
            // buffer once the MMAs of the tile two back are done with it
            bool fr = gi == 0 || tc::mbar_wait(&bars->p_free, (gi - 1) & 1, abort_flag, p.err, kErrTimeoutCompute);
            if (fr && gi >= kDSBufs) fr = tc::mbar_wait(&bars->ds_free[sb], (gi / kDSBufs - 1) & 1, abort_flag, p.err,
                                                 kErrTimeoutCompute);
            ok = __all_sync(0xffffffffu, fr);
            tc::tc_fence_after();
          }
          // P^T: 16 queries = 8 packed columns of this lane's TMEM row
          tc::tmem_st8(tmem + lane_base + kColP + (col0 >> 1), pp);
          // dS^T row: key r, 16 queries = two 16-byte chunks of the 64-query atom
  #pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int ch = (((grp & 1) * 4 + c * 2 + u) ^ (r & 7)) << 4;
            *reinterpret_cast<uint4*>(DSt + r * 128 + ch) =
                make_uint4(pf[4 * u], pf[4 * u + 1], pf[4 * u + 2], pf[4 * u + 3]);
          }
        };
        tc::tmem_ld16(tmem + lane_base + kColS + grp * 32, rr);
        tc::tmem_ld16(tmem + lane_base + kColDP + grp * 32, rr + 16);
        tc::tmem_wait_ld_regs(rr);
        chunk(0);
        tc::tmem_wait_ld_regs(rr);
        // every TMEM read of this tile's S^T / dP^T is done
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bars->s_free);
        if (ok) chunk(1);
        if (!ok) break;
        tc::tmem_wait_st();
        tc::fence_async_smem();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          tc::mbar_arrive(&bars->ds_ready);
          tc::mbar_arrive(&bars->ds_full_epi[sb]);
        }
        if (++qs == kQStages) { qs = 0; qph ^= 1; }
      }
      g += nQ;
      float sum_tau = acc_tau.x + acc_tau.y, sum_alpha = acc_alpha.x + acc_alpha.y;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        sum_tau += __shfl_xor_sync(0xffffffffu, sum_tau, off);
        sum_alpha += __shfl_xor_sync(0xffffffffu, sum_alpha, off);
      }
      const int rs = n & 1;
      if (lane == 0) {
        atomicAdd(&bars->red_tau[rs], sum_tau);
        atomicAdd(&bars->red_alpha[rs], sum_alpha);
      }
      // Every elementwise warp reaches this barrier once per item, also after
      // leaving the tile loop early (its waits return at once when another
      // role gave up), and all of them take the same decision from it.
      ok = tc::named_barrier_and(2, kComputeWarps * 32, ok);
      if (warp == 8 && lane == 0) {
        // dtau = sum t ln(sigma_clamped), dalpha = tau sum t clip(sigma'/sigma (s - m), +-30)
        if (ok) {
          atomicAdd(p.dtau + h, bars->red_tau[rs] * (kLn2 / tau));
          atomicAdd(p.dalpha + h, bars->red_alpha[rs] * (tau / (alpha * kLog2e)));
        }
        bars->red_tau[rs] = 0.f;        // for item n + 2; no warp adds to it before the next barrier
        bars->red_alpha[rs] = 0.f;
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

static bool layout16(const void* ptr, const int64_t s[4]) {
  return s[3] == 1 && (reinterpret_cast<uintptr_t>(ptr) % 16 == 0) && s[0] % 8 == 0 &&
         s[1] % 8 == 0 && s[2] % 8 == 0 && s[0] >= 0 && s[1] >= 0 && s[2] > 0;
}

bool attn_tensor_bwd_supported(const AttnProblem& p) {
  if (!attn_tensor_supported(p)) return false;
  return layout16(p.dout, p.dos) && layout16(p.dv, p.dvs);
}

int attn_bwd_tensor_main(const AttnProblem& p, cudaStream_t st) {
  BwdParams bp;
  memset(&bp, 0, sizeof(bp));
  if (!make_tmap_bhld(&bp.tq, p.q, p.D, p.Lq, p.H, p.B, p.qs, kT) ||
      !make_tmap_bhld(&bp.tk, p.k, p.D, p.Lk, p.H, p.B, p.ks, kT) ||
      !make_tmap_bhld(&bp.tv, p.v, p.D, p.Lk, p.H, p.B, p.vs, kT) ||
      !make_tmap_bhld(&bp.tdo, p.dout, p.D, p.Lq, p.H, p.B, p.dos, kT) ||
      !make_tmap_f32_rows64(&bp.tdq, p.ws_dq, p.Lq, static_cast<int64_t>(p.B) * p.H, kT))
    return TAU_DXB_ERR_CUDA;
  bp.B = p.B; bp.H = p.H; bp.Lq = p.Lq; bp.Lk = p.Lk;
  bp.tau = p.tau; bp.alpha = p.alpha; bp.scale = p.scale; bp.causal = p.causal;
  bp.mask = p.mask; bp.mask_dtype = p.mask_dtype;
  for (int i = 0; i < 4; ++i) { bp.ms[i] = p.ms[i]; bp.dvs[i] = p.dvs[i]; }
  bp.row_max = p.row_max; bp.row_z = p.row_z; bp.drow = p.ws_drow;
  bp.ws_rowf = p.ws_rowf; bp.ws_dk = p.ws_dk;
  bp.dv = p.dv; bp.dtau = p.dtau; bp.dalpha = p.dalpha;
  bp.err = device_error_word();
  if (!bp.err) return fail(TAU_DXB_ERR_CUDA, "cannot resolve the device error word");
  const int64_t items = static_cast<int64_t>((p.Lk + kT - 1) / kT) * p.H * p.B;
  if (items > INT32_MAX) return fail(TAU_DXB_ERR_INVALID_ARGUMENT, "too many key tiles for the backward (%lld)",
                                     static_cast<long long>(items));
  bp.n_items = static_cast<int>(items);
  // one CTA per SM, each looping over its items
  dim3 grid(static_cast<unsigned>(std::min<int64_t>(items, sm_count())));
  auto launch = [&](auto kern) -> int {
    TDX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBwdSmem));
    kern<<<grid, kThreads, kBwdSmem, st>>>(bp);
    return check_launch("attn_bwd_tc_kernel");
  };
  switch (p.sigma) {
    case TAU_DXB_SIGMA_SOFTPLUS: return launch(attn_bwd_tc_kernel<TAU_DXB_SIGMA_SOFTPLUS>);
    case TAU_DXB_SIGMA_SIGMOID: return launch(attn_bwd_tc_kernel<TAU_DXB_SIGMA_SIGMOID>);
    case TAU_DXB_SIGMA_EXP: return launch(attn_bwd_tc_kernel<TAU_DXB_SIGMA_EXP>);
    default: return launch(attn_bwd_tc_kernel<TAU_DXB_SIGMA_RELU>);
  }
}

}  // namespace taudxb
