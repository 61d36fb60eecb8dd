// Whisper log-mel features on the GPU (the reference computes them per sample
// on the host: WhisperFeatureExtractor, echo/train_echo_opus1.py:126).
//
// Kernel 1 (one CTA per 16 frames of one sample, 256 threads): the frames'
// samples -- reflect-padded by 200 at both ends of the waveform -- go to
// shared memory; the 400-point DFT of each Hann-windowed frame is a 16 x 25
// Cooley-Tukey split (n = 25 n1 + n2, k = k1 + 16 k2):
//   Y[n2][k1] = W400^(n2 k1) sum_n1 w x[25 n1 + n2] W16^(n1 k1)   (16-point DFTs)
//   X[k]      = sum_n2 Y[n2][k mod 16] W25^(n2 floor(k / 16))     (25-point DFTs)
// for the 201 bins k = 0..200 (35k multiply-adds per frame instead of 160k
// for the direct DFT); then |X|^2, the 80 sparse triangular mel filters,
// log10(max(mel, 1e-10)), and an order-preserving atomicMax of the sample's
// largest value. fp32 throughout; trigonometric tables from sincospif.
// Kernel 2: x = (max(x, max_sample - 8) + 4) / 4 over the whole output.
// A one-CTA pre-kernel packs the dense [201][80] filter bank (the extractor's
// mel_filters) into per-band [first bin, bin count] and the band's weights,
// in the caller's workspace.

#include "common.cuh"

namespace taudxb {
namespace {

constexpr int kNfft = 400, kHop = 160, kBins = 201, kMels = 80;
constexpr int kN1 = 16, kN2 = 25;        // 400 = 16 * 25
constexpr int kFR = 16;                  // frames per CTA
constexpr int kLmThreads = 256;
constexpr int kSeg = kFR * kHop + (kNfft - kHop);   // samples of a CTA's frames

__device__ __forceinline__ uint32_t f2ord(float f) {
  const uint32_t u = __float_as_uint(f);
  return u ^ ((u & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint32_t o) {
  return __uint_as_float(o ^ ((o & 0x80000000u) ? 0x80000000u : 0xFFFFFFFFu));
}

__global__ void __launch_bounds__(kLmThreads) log_mel_kernel(const float* __restrict__ audio, int64_t n_samples,
                                                            int n_frames, const int32_t* __restrict__ meta,
                                                            const float* __restrict__ weights,
                                                            float* __restrict__ out, uint32_t* __restrict__ smax) {
  extern __shared__ __align__(16) float2 lsm[];
  float2* Y = lsm;                            // [f][n2][k1]
  float2* w16 = Y + kFR * kN2 * kN1;          // [n1][k1] (cos, -sin)(2 pi n1 k1 / 16)
  float2* tw = w16 + kN1 * kN1;               // [n2][k1] W400^(n2 k1)
  float2* w25 = tw + kN2 * kN1;               // [n2][k2] W25^(n2 k2), k2 < 13
  float* xs = reinterpret_cast<float*>(w25 + kN2 * 13);   // [kSeg]
  float* win = xs + kSeg;                     // [400]
  float* P = win + kNfft;                     // [f][k]
  float* cmax = P + kFR * kBins;              // [warps]
  const int b = blockIdx.y, t0 = blockIdx.x * kFR, tid = threadIdx.x;
  const float* x = audio + static_cast<int64_t>(b) * n_samples;

  // tables
  for (int i = tid; i < kNfft; i += kLmThreads) win[i] = 0.5f - 0.5f * cospif(2.f * i / kNfft);
  for (int i = tid; i < kN1 * kN1; i += kLmThreads) {
    float s, c;
    sincospif(2.f * ((i / kN1) * (i % kN1) % kN1) / kN1, &s, &c);
    w16[i] = make_float2(c, -s);
  }
  for (int i = tid; i < kN2 * kN1; i += kLmThreads) {
    float s, c;
    sincospif(2.f * ((i / kN1) * (i % kN1) % kNfft) / kNfft, &s, &c);
    tw[i] = make_float2(c, -s);
  }
  for (int i = tid; i < kN2 * 13; i += kLmThreads) {
    float s, c;
    sincospif(2.f * ((i / 13) * (i % 13) % kN2) / kN2, &s, &c);
    w25[i] = make_float2(c, -s);
  }
  // samples of padded positions [t0 hop, t0 hop + kSeg); padded position i is
  // waveform sample i - 200, reflected at both ends
  for (int i = tid; i < kSeg; i += kLmThreads) {
    int64_t s = static_cast<int64_t>(t0) * kHop + i - kNfft / 2;
    if (s < 0) s = -s;
    if (s >= n_samples) s = 2 * (n_samples - 1) - s;
    // the frames that are written (t < n_frames) reach at most sample
    // n_samples + 40 before reflection; the clamp only keeps the frames past
    // the end of the last CTA (never written) inside the waveform
    s = s < 0 ? 0 : (s >= n_samples ? n_samples - 1 : s);
    xs[i] = x[s];
  }
  __syncthreads();

  // 16-point DFTs of the decimated, windowed sequences, twiddled
  for (int o = tid; o < kFR * kN2 * kN1; o += kLmThreads) {
    const int f = o / (kN2 * kN1), rem = o % (kN2 * kN1), n2 = rem / kN1, k1 = rem % kN1;
    const float* xf = xs + f * kHop + n2;
    float re = 0.f, im = 0.f;
#pragma unroll
    for (int n1 = 0; n1 < kN1; ++n1) {
      const float a = win[kN2 * n1 + n2] * xf[kN2 * n1];
      const float2 w = w16[n1 * kN1 + k1];
      re = fmaf(a, w.x, re);
      im = fmaf(a, w.y, im);
    }
    const float2 t = tw[n2 * kN1 + k1];
    Y[o] = make_float2(re * t.x - im * t.y, re * t.y + im * t.x);
  }
  __syncthreads();

  // 25-point DFTs for bins 0..200, power
  for (int o = tid; o < kFR * kBins; o += kLmThreads) {
    const int f = o / kBins, k = o % kBins, k1 = k % kN1, k2 = k / kN1;
    const float2* yf = Y + f * kN2 * kN1 + k1;
    float re = 0.f, im = 0.f;
#pragma unroll 5
    for (int n2 = 0; n2 < kN2; ++n2) {
      const float2 y = yf[n2 * kN1];
      const float2 w = w25[n2 * 13 + k2];
      re = fmaf(y.x, w.x, fmaf(-y.y, w.y, re));
      im = fmaf(y.x, w.y, fmaf(y.y, w.x, im));
    }
    P[o] = fmaf(re, re, im * im);
  }
  __syncthreads();

  // mel filters, log10; 16 consecutive lanes write 16 consecutive frames of one mel band
  float lmax = -INFINITY;
  for (int o = tid; o < kFR * kMels; o += kLmThreads) {
    const int f = o % kFR, m = o / kFR, t = t0 + f;
    const int lo = meta[2 * m], cnt = meta[2 * m + 1];
    const float* wv = weights + m * kBins;
    const float* pf = P + f * kBins + lo;
    float acc = 0.f;
    for (int j = 0; j < cnt; ++j) acc = fmaf(__ldg(wv + j), pf[j], acc);
    const float v = log10f(fmaxf(acc, 1e-10f));
    if (t < n_frames) {
      out[(static_cast<int64_t>(b) * kMels + m) * n_frames + t] = v;
      lmax = fmaxf(lmax, v);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, off));
  if ((tid & 31) == 0) cmax[tid >> 5] = lmax;
  __syncthreads();
  if (tid == 0) {
    float m = cmax[0];
    for (int w = 1; w < kLmThreads / 32; ++w) m = fmaxf(m, cmax[w]);
    atomicMax(smax + b, f2ord(m));
  }
}

// thread m: the nonzero bin range of band m and its weights
__global__ void mel_pack_kernel(const float* __restrict__ filters, int32_t* __restrict__ meta,
                                float* __restrict__ weights) {
  const int m = threadIdx.x;
  if (m >= kMels) return;
  int lo = kBins, hi = 0;
  for (int k = 0; k < kBins; ++k) {
    if (filters[k * kMels + m] != 0.f) {
      lo = min(lo, k);
      hi = k + 1;
    }
  }
  if (hi == 0) lo = 0;
  meta[2 * m] = lo;
  meta[2 * m + 1] = hi - lo;
  for (int k = lo; k < hi; ++k) weights[m * kBins + k - lo] = filters[k * kMels + m];
}

__global__ void log_mel_normalize_kernel(float* __restrict__ out, int64_t per_sample, int64_t total,
                                         const uint32_t* __restrict__ smax) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float lo = ord2f(smax[i / per_sample]) - 8.f;
    out[i] = (fmaxf(out[i], lo) + 4.f) * 0.25f;
  }
}

}  // namespace

size_t whisper_log_mel_workspace(int64_t batch) {
  return 256 + static_cast<size_t>(batch) * sizeof(uint32_t) + 256 + 2 * kMels * sizeof(int32_t) +
         static_cast<size_t>(kMels) * kBins * sizeof(float) + 256;
}

int whisper_log_mel_impl(const float* audio, int64_t batch, int64_t n_samples, const float* mel_filters,
                         float* out, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  TDX_CHECK_ARG(batch >= 0 && n_samples >= kNfft && n_samples % kHop == 0 && n_samples < (1ll << 31),
                "whisper_log_mel: need n_samples >= 400 and a multiple of 160 (got %lld)", (long long)n_samples);
  if (batch == 0) return TAU_DXB_OK;
  TDX_CHECK_ARG(audio && mel_filters && out && workspace, "whisper_log_mel: null pointer");
  TDX_CHECK_ARG(batch <= 65535, "whisper_log_mel: batch > 65535");
  if (workspace_bytes < whisper_log_mel_workspace(batch))
    return fail(TAU_DXB_ERR_WORKSPACE, "whisper_log_mel: workspace of %zu bytes, need %zu", workspace_bytes,
                whisper_log_mel_workspace(batch));
  auto align = [](uintptr_t v) { return (v + 255) & ~static_cast<uintptr_t>(255); };
  const uintptr_t base = align(reinterpret_cast<uintptr_t>(workspace));
  uint32_t* sample_max = reinterpret_cast<uint32_t*>(base);
  int32_t* meta = reinterpret_cast<int32_t*>(align(base + static_cast<size_t>(batch) * sizeof(uint32_t)));
  float* weights = reinterpret_cast<float*>(align(reinterpret_cast<uintptr_t>(meta + 2 * kMels)));
  const int n_frames = static_cast<int>(n_samples / kHop);
  mel_pack_kernel<<<1, 128, 0, st>>>(mel_filters, meta, weights);
  int rc = check_launch("mel_pack_kernel");
  if (rc) return rc;
  TDX_CUDA(cudaMemsetAsync(sample_max, 0, static_cast<size_t>(batch) * sizeof(uint32_t), st));
  dim3 grid((n_frames + kFR - 1) / kFR, static_cast<unsigned>(batch));
  const size_t smem = (kFR * kN2 * kN1 + kN1 * kN1 + kN2 * kN1 + kN2 * 13) * sizeof(float2) +
                      (kSeg + kNfft + kFR * kBins + kLmThreads / 32) * sizeof(float);
  TDX_CUDA(cudaFuncSetAttribute(log_mel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  log_mel_kernel<<<grid, kLmThreads, smem, st>>>(audio, n_samples, n_frames, meta, weights, out, sample_max);
  rc = check_launch("log_mel_kernel");
  if (rc) return rc;
  const int64_t per = static_cast<int64_t>(kMels) * n_frames, total = per * batch;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  log_mel_normalize_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(out, per, total, sample_max);
  return check_launch("log_mel_normalize_kernel");
}

}  // namespace taudxb
