// C ABI entry points (include/tau_dxb.h): argument validation, dispatch, errors.

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "attn.h"

namespace taudxb {

namespace {
thread_local char g_last_error[512] = "";
}

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(TAU_DXB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return TAU_DXB_OK;
}

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

int wta_fwd_impl(const void*, int32_t, int64_t, int64_t, int64_t, int64_t, const int32_t*, int32_t,
                 void*, uint8_t*, int32_t*, cudaStream_t);
int wta_bwd_impl(const void*, int32_t, const uint8_t*, int64_t, int64_t, void*, cudaStream_t);
int wta_bwd_gelu_impl(const void*, const void*, const uint8_t*, int64_t, int64_t, void*, cudaStream_t);
int wta_k_from_logits_impl(const float*, int64_t, int64_t, int32_t*, cudaStream_t);
size_t whisper_log_mel_workspace(int64_t batch);
int whisper_log_mel_impl(const float*, int64_t, int64_t, const float*, float*, void*, size_t, cudaStream_t);
int tau_star_solve_impl(const float*, int64_t, int64_t, int64_t, int32_t, int32_t, float, float, float, float,
                        float*, float*, cudaStream_t);
int tau_star_analytic_impl(const float*, int64_t, int64_t, int64_t, int32_t, float*, cudaStream_t);
size_t layer_norm_bwd_workspace(int64_t M, int64_t N);
size_t column_sum_workspace(int64_t M, int64_t N);
int grad_mask_impl(const void*, int32_t, int64_t, int64_t, const uint8_t*, int32_t, void*, cudaStream_t);
int fixed_fwd_impl(const float*, int64_t, int64_t, int64_t, const float*, int64_t, int64_t, int32_t, float*,
                   cudaStream_t);
int fixed_bwd_impl(const float*, const float*, int64_t, int64_t, int64_t, const float*, int64_t, int64_t, int32_t,
                   float*, cudaStream_t);
int column_sum_impl(const void*, int32_t, int64_t, int64_t, void*, int32_t, void*, size_t, cudaStream_t);
int cross_entropy_fwd_impl(const void*, int64_t, int64_t, const int64_t*, int64_t, float*, float*, cudaStream_t);
int cross_entropy_bwd_impl(const void*, int64_t, int64_t, const int64_t*, int64_t, const float*, const float*, void*,
                           cudaStream_t);
int layer_norm_fwd_impl(const float*, int64_t, int64_t, const float*, const float*, float, void*, int32_t, float*,
                        float*, cudaStream_t);
int layer_norm_bwd_impl(const void*, int32_t, const float*, const float*, const float*, const float*, int64_t,
                        int64_t, float*, float*, float*, void*, size_t, cudaStream_t);

namespace {

bool valid_dtype(int32_t d) { return d == TAU_DXB_F32 || d == TAU_DXB_BF16 || d == TAU_DXB_F16; }

int fill_common(AttnProblem& p, const void* q, const int64_t* qs, const void* k, const int64_t* ks,
                const void* v, const int64_t* vs, int32_t dtype, int64_t B, int64_t H, int64_t Lq,
                int64_t Lk, int64_t D, const float* tau, const float* alpha, int32_t sigma,
                float scale, const void* mask, int32_t mask_dtype, const int64_t* ms, int32_t causal) {
  memset(&p, 0, sizeof(p));
  TDX_CHECK_ARG(q && k && v && qs && ks && vs, "attention: q, k, v and their strides are required");
  TDX_CHECK_ARG(tau && alpha, "attention: tau and alpha are required");
  TDX_CHECK_ARG(valid_dtype(dtype), "attention: bad dtype %d", dtype);
  TDX_CHECK_ARG(B >= 0 && H >= 1 && Lq >= 0 && Lk >= 1 && D >= 1,
                "attention: bad shape B=%lld H=%lld Lq=%lld Lk=%lld D=%lld",
                (long long)B, (long long)H, (long long)Lq, (long long)Lk, (long long)D);
  TDX_CHECK_ARG(B < (1 << 16) && H < (1 << 16) && Lq < (1 << 24) && Lk < (1 << 24) && D <= 128,
                "attention: shape too large (need B,H < 65536, L < 2^24, D <= 128)");
  TDX_CHECK_ARG(sigma >= TAU_DXB_SIGMA_SOFTPLUS && sigma <= TAU_DXB_SIGMA_RELU, "attention: bad sigma id %d", sigma);
  TDX_CHECK_ARG(!mask || (ms && valid_dtype(mask_dtype)), "attention: mask needs strides and a valid dtype");
  p.q = q; p.k = k; p.v = v;
  memcpy(p.qs, qs, sizeof(p.qs)); memcpy(p.ks, ks, sizeof(p.ks)); memcpy(p.vs, vs, sizeof(p.vs));
  p.dtype = dtype;
  p.B = (int)B; p.H = (int)H; p.Lq = (int)Lq; p.Lk = (int)Lk; p.D = (int)D;
  p.tau = tau; p.alpha = alpha;
  p.sigma = sigma; p.scale = scale;
  p.mask = mask; p.mask_dtype = mask_dtype;
  if (mask) memcpy(p.ms, ms, sizeof(p.ms));
  p.causal = causal ? 1 : 0;
  return TAU_DXB_OK;
}

bool use_tensor(const AttnProblem& p, int32_t path, int* rc, bool bwd) {
  *rc = TAU_DXB_OK;
  if (path == TAU_DXB_PATH_PRECISE) return false;
  const bool ok = bwd ? attn_tensor_bwd_supported(p) : attn_tensor_supported(p);
  if (path == TAU_DXB_PATH_TENSOR && !ok)
    *rc = fail(TAU_DXB_ERR_UNSUPPORTED, "tensor-core attention path needs bf16/f16, D == 64 and 16-byte aligned rows with unit d-stride");
  return ok;
}

}  // namespace
}  // namespace taudxb

using namespace taudxb;

extern "C" {

int tau_dxb_version(void) { return 100; }

const char* tau_dxb_strerror(int status) {
  switch (status) {
    case TAU_DXB_OK: return "ok";
    case TAU_DXB_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TAU_DXB_ERR_UNSUPPORTED: return "unsupported problem";
    case TAU_DXB_ERR_CUDA: return "CUDA error";
    case TAU_DXB_ERR_WORKSPACE: return "workspace too small";
    case TAU_DXB_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

const char* tau_dxb_last_error(void) { return g_last_error; }

int tau_attn_fwd(const void* q, const int64_t q_stride[4], const void* k, const int64_t k_stride[4],
                 const void* v, const int64_t v_stride[4], int32_t dtype, int64_t B, int64_t H,
                 int64_t Lq, int64_t Lk, int64_t D, const float* tau, const float* alpha,
                 int32_t sigma_id, float scale, const void* mask, int32_t mask_dtype,
                 const int64_t mask_stride[4], int32_t causal, void* out, const int64_t out_stride[4],
                 float* row_max, float* row_z, int32_t* row_argmax, int32_t path, void* stream) {
  g_last_error[0] = 0;
  AttnProblem p;
  int rc = fill_common(p, q, q_stride, k, k_stride, v, v_stride, dtype, B, H, Lq, Lk, D, tau,
                       alpha, sigma_id, scale, mask, mask_dtype, mask_stride, causal);
  if (rc) return rc;
  TDX_CHECK_ARG(out && out_stride && row_max && row_z && row_argmax, "tau_attn_fwd: outputs are required");
  TDX_CHECK_ARG(path >= TAU_DXB_PATH_AUTO && path <= TAU_DXB_PATH_TENSOR, "tau_attn_fwd: bad path %d", path);
  p.out = out; memcpy(p.outs, out_stride, sizeof(p.outs));
  p.row_max = row_max; p.row_z = row_z; p.row_argmax = row_argmax;
  if (B == 0 || Lq == 0) return TAU_DXB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // a few query rows (KV-cached decoding): one pass over K and V per row
  if (path == TAU_DXB_PATH_AUTO && attn_decode_supported(p)) return attn_fwd_decode(p, st);
  const bool tc = use_tensor(p, path, &rc, false);
  if (rc) return rc;
  return tc ? attn_fwd_tensor(p, st) : attn_fwd_precise(p, st);
}

size_t tau_attn_bwd_workspace_bytes(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D) {
  if (B < 0 || H < 0 || Lq < 0 || Lk < 0 || D < 0) return 0;
  return workspace_layout(B, H, Lq, Lk, D).total;
}

int tau_attn_bwd(const void* q, const int64_t q_stride[4], const void* k, const int64_t k_stride[4],
                 const void* v, const int64_t v_stride[4], const void* out, const int64_t out_stride[4],
                 const void* dout, const int64_t dout_stride[4], int32_t dtype, int64_t B, int64_t H,
                 int64_t Lq, int64_t Lk, int64_t D, const float* tau, const float* alpha,
                 int32_t sigma_id, float scale, const void* mask, int32_t mask_dtype,
                 const int64_t mask_stride[4], int32_t causal, const float* row_max,
                 const float* row_z, const int32_t* row_argmax, void* dq, const int64_t dq_stride[4],
                 void* dk, const int64_t dk_stride[4], void* dv, const int64_t dv_stride[4],
                 float* dtau, float* dalpha, void* workspace, size_t workspace_bytes,
                 int32_t path, void* stream) {
  g_last_error[0] = 0;
  AttnProblem p;
  int rc = fill_common(p, q, q_stride, k, k_stride, v, v_stride, dtype, B, H, Lq, Lk, D, tau,
                       alpha, sigma_id, scale, mask, mask_dtype, mask_stride, causal);
  if (rc) return rc;
  TDX_CHECK_ARG(out && out_stride && dout && dout_stride, "tau_attn_bwd: out and dout are required");
  TDX_CHECK_ARG(row_max && row_z && row_argmax, "tau_attn_bwd: forward row state is required");
  TDX_CHECK_ARG(dq && dq_stride && dk && dk_stride && dv && dv_stride && dtau && dalpha,
                "tau_attn_bwd: gradient outputs are required");
  TDX_CHECK_ARG(path >= TAU_DXB_PATH_AUTO && path <= TAU_DXB_PATH_TENSOR, "tau_attn_bwd: bad path %d", path);
  const WorkspaceLayout w = workspace_layout(B, H, Lq, Lk, D);
  if (!workspace || workspace_bytes < w.total)
    return fail(TAU_DXB_ERR_WORKSPACE, "tau_attn_bwd: workspace needs %zu bytes, got %zu", w.total, workspace_bytes);
  TDX_CHECK_ARG(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, "tau_attn_bwd: workspace must be 256-byte aligned");
  p.o = out; memcpy(p.os, out_stride, sizeof(p.os));
  p.dout = dout; memcpy(p.dos, dout_stride, sizeof(p.dos));
  p.row_max = const_cast<float*>(row_max); p.row_z = const_cast<float*>(row_z);
  p.row_argmax = const_cast<int32_t*>(row_argmax);
  p.dq = dq; memcpy(p.dqs, dq_stride, sizeof(p.dqs));
  p.dk = dk; memcpy(p.dks, dk_stride, sizeof(p.dks));
  p.dv = dv; memcpy(p.dvs, dv_stride, sizeof(p.dvs));
  p.dtau = dtau; p.dalpha = dalpha;
  char* ws = static_cast<char*>(workspace);
  p.ws_dq = reinterpret_cast<float*>(ws + w.dq);
  p.ws_dk = reinterpret_cast<float*>(ws + w.dk);
  p.ws_drow = reinterpret_cast<float*>(ws + w.drow);
  p.ws_rowf = reinterpret_cast<float*>(ws + w.rowf);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0 || Lq == 0) {
    // no query rows: every gradient is zero
    TDX_CUDA(cudaMemsetAsync(p.dtau, 0, H * sizeof(float), st));
    TDX_CUDA(cudaMemsetAsync(p.dalpha, 0, H * sizeof(float), st));
    TDX_CUDA(cudaMemsetAsync(p.ws_dk, 0, w.drow - w.dk, st));
    p.Lq = 0;
    return attn_bwd_epilogue(p, st);
  }
  const bool tc = use_tensor(p, path, &rc, true);
  if (rc) return rc;
  rc = attn_bwd_prologue(p, st);
  if (rc) return rc;
  rc = tc ? attn_bwd_tensor_main(p, st) : attn_bwd_precise_main(p, st);
  if (rc) return rc;
  return attn_bwd_epilogue(p, st);
}

int tau_dxb_device_error(int32_t reset) { return read_device_error(reset); }

int tau_dxb_selftest_wait_timeout(uint64_t limit_ns, int32_t* status, void* stream) {
  g_last_error[0] = 0;
  TDX_CHECK_ARG(status, "tau_dxb_selftest_wait_timeout: status is required");
  TDX_CHECK_ARG(limit_ns > 0 && limit_ns <= 10000000000ull,
                "tau_dxb_selftest_wait_timeout: limit_ns must be in (0, 10 s]");
  return wait_selftest(limit_ns, status, static_cast<cudaStream_t>(stream));
}

int wta_fwd(const void* x, int32_t dtype, int64_t n_rows, int64_t d, int64_t row_stride, int64_t k,
            const int32_t* k_dev, int32_t mode, void* y, uint8_t* bitmask, int32_t* win_counts,
            void* stream) {
  g_last_error[0] = 0;
  return wta_fwd_impl(x, dtype, n_rows, d, row_stride, k, k_dev, mode, y, bitmask, win_counts,
                      static_cast<cudaStream_t>(stream));
}

int wta_bwd(const void* dy, int32_t dtype, const uint8_t* bitmask, int64_t n_rows, int64_t d,
            void* dx, void* stream) {
  g_last_error[0] = 0;
  return wta_bwd_impl(dy, dtype, bitmask, n_rows, d, dx, static_cast<cudaStream_t>(stream));
}

int wta_bwd_gelu(const void* dy, const void* x, const uint8_t* bitmask, int64_t n_rows, int64_t d, void* dx,
                 void* stream) {
  g_last_error[0] = 0;
  return wta_bwd_gelu_impl(dy, x, bitmask, n_rows, d, dx, static_cast<cudaStream_t>(stream));
}

int wta_k_from_logits(const float* logits, int64_t n, int64_t d_ff, int32_t* k_out, void* stream) {
  g_last_error[0] = 0;
  return wta_k_from_logits_impl(logits, n, d_ff, k_out, static_cast<cudaStream_t>(stream));
}

size_t whisper_log_mel_workspace_bytes(int64_t batch) {
  return batch < 0 ? 0 : whisper_log_mel_workspace(batch);
}

int whisper_log_mel(const float* audio, int64_t batch, int64_t n_samples, const float* mel_filters,
                    float* out, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error[0] = 0;
  return whisper_log_mel_impl(audio, batch, n_samples, mel_filters, out, workspace, workspace_bytes,
                              static_cast<cudaStream_t>(stream));
}

int tau_star_solve(const float* scores, int64_t n_rows, int64_t T, int64_t row_stride, int32_t sigma,
                   int32_t n_iter, float tau_init, float tau_min, float tau_max, float eps, float* tau_out,
                   float* kl_out, void* stream) {
  g_last_error[0] = 0;
  return tau_star_solve_impl(scores, n_rows, T, row_stride, sigma, n_iter, tau_init, tau_min, tau_max, eps,
                             tau_out, kl_out, static_cast<cudaStream_t>(stream));
}

int tau_star_analytic(const float* scores, int64_t n_rows, int64_t T, int64_t row_stride, int32_t sigma,
                      float* tau_out, void* stream) {
  g_last_error[0] = 0;
  return tau_star_analytic_impl(scores, n_rows, T, row_stride, sigma, tau_out, static_cast<cudaStream_t>(stream));
}

int tau_layer_norm_fwd(const float* x, int64_t M, int64_t d, const float* gamma, const float* beta, float eps,
                       void* y, int32_t y_dtype, float* mean, float* rstd, void* stream) {
  g_last_error[0] = 0;
  return layer_norm_fwd_impl(x, M, d, gamma, beta, eps, y, y_dtype, mean, rstd, static_cast<cudaStream_t>(stream));
}

size_t tau_layer_norm_bwd_workspace_bytes(int64_t M, int64_t d) { return layer_norm_bwd_workspace(M, d); }

int tau_layer_norm_bwd(const void* dy, int32_t dy_dtype, const float* x, const float* mean, const float* rstd,
                       const float* gamma, int64_t M, int64_t d, float* dx, float* dgamma, float* dbeta,
                       void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error[0] = 0;
  return layer_norm_bwd_impl(dy, dy_dtype, x, mean, rstd, gamma, M, d, dx, dgamma, dbeta, workspace,
                             workspace_bytes, static_cast<cudaStream_t>(stream));
}

int tau_opus_fixed_fwd(const float* scores, int64_t rows, int64_t L, int64_t row_stride, const float* tau,
                       int64_t n_tau, int64_t rows_per_tau, int32_t sigma_id, float* attn, void* stream) {
  g_last_error[0] = 0;
  return fixed_fwd_impl(scores, rows, L, row_stride, tau, n_tau, rows_per_tau, sigma_id, attn,
                        static_cast<cudaStream_t>(stream));
}

int tau_opus_fixed_bwd(const float* scores, const float* grad_attn, int64_t rows, int64_t L, int64_t row_stride,
                       const float* tau, int64_t n_tau, int64_t rows_per_tau, int32_t sigma_id, float* grad_scores,
                       void* stream) {
  g_last_error[0] = 0;
  return fixed_bwd_impl(scores, grad_attn, rows, L, row_stride, tau, n_tau, rows_per_tau, sigma_id, grad_scores,
                        static_cast<cudaStream_t>(stream));
}

int tau_grad_mask(const void* grad, int32_t dtype, int64_t rows, int64_t cols, const uint8_t* keep, int32_t axis,
                  void* out, void* stream) {
  g_last_error[0] = 0;
  return grad_mask_impl(grad, dtype, rows, cols, keep, axis, out, static_cast<cudaStream_t>(stream));
}

size_t tau_column_sum_workspace_bytes(int64_t M, int64_t N) { return column_sum_workspace(M, N); }

int tau_column_sum(const void* x, int32_t dtype, int64_t M, int64_t N, void* out, int32_t out_dtype,
                   void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error[0] = 0;
  return column_sum_impl(x, dtype, M, N, out, out_dtype, workspace, workspace_bytes,
                         static_cast<cudaStream_t>(stream));
}

int tau_cross_entropy_fwd(const void* logits, int64_t M, int64_t V, const int64_t* labels, int64_t ignore_index,
                          float* loss_row, float* lse, void* stream) {
  g_last_error[0] = 0;
  return cross_entropy_fwd_impl(logits, M, V, labels, ignore_index, loss_row, lse, static_cast<cudaStream_t>(stream));
}

int tau_cross_entropy_bwd(const void* logits, int64_t M, int64_t V, const int64_t* labels, int64_t ignore_index,
                          const float* lse, const float* grad_scale, void* dlogits, void* stream) {
  g_last_error[0] = 0;
  return cross_entropy_bwd_impl(logits, M, V, labels, ignore_index, lse, grad_scale, dlogits,
                                static_cast<cudaStream_t>(stream));
}

}  // extern "C"
