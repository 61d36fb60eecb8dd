/*
 * tau_dxb.h -- C ABI of the B200 (sm_100a) kernels behind tau-dxb's two
 * training hot paths: tau-opus attention and WTA top-k sparsity.
 *
 * Conventions
 *   - Every tensor pointer is a DEVICE pointer owned by the caller; the
 *     library never allocates device memory except where a function says so.
 *   - Strides are in ELEMENTS, ordered (B, H, L, D) for attention tensors.
 *     A broadcast mask dimension has stride 0.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default).
 *   - Functions return 0 (TAU_DXB_OK) or a negative status; they never throw.
 *     tau_dxb_last_error() gives a message for the calling thread's last error.
 *   - All work is asynchronous on `stream`; nothing synchronises the host.
 *
 * The reference (inkamrais-hub/tau-dxb) is pure Python; each entry point names
 * the reference function it replaces (path:line inside that project).
 */
#ifndef TAU_DXB_H
#define TAU_DXB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TAU_DXB_API __attribute__((visibility("default")))
#else
#define TAU_DXB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define TAU_DXB_OK                    0
#define TAU_DXB_ERR_INVALID_ARGUMENT (-1)
#define TAU_DXB_ERR_UNSUPPORTED      (-2)
#define TAU_DXB_ERR_CUDA             (-3)
#define TAU_DXB_ERR_WORKSPACE        (-4)
#define TAU_DXB_ERR_NO_DEVICE        (-5)

/* ---- element types ----------------------------------------------------- */
#define TAU_DXB_F32  0
#define TAU_DXB_BF16 1
#define TAU_DXB_F16  2

/* ---- sigma ids: same numbering as the reference's _SIGMA_NAME_TO_ID
 *      (echo/stau_opus_flash_v2.py:400) ---------------------------------- */
#define TAU_DXB_SIGMA_SOFTPLUS 0
#define TAU_DXB_SIGMA_SIGMOID  1
#define TAU_DXB_SIGMA_EXP      2
#define TAU_DXB_SIGMA_RELU     3
#define TAU_DXB_SIGMA_TANH_SHIFT 4  /* tanh(x) + 1; fixed-tau weights (tau_opus_fixed_*) only */

/* ---- longest score row tau_star_solve accepts --------------------------- */
#define TAU_DXB_TAU_STAR_MAX_KEYS 28672

/* ---- attention kernel path ---------------------------------------------- */
#define TAU_DXB_PATH_AUTO    0  /* forward with Lq <= 8 (KV-cached decoding):
                                   one pass over K and V per query row, fp32
                                   math; otherwise tensor cores when supported,
                                   else precise */
#define TAU_DXB_PATH_PRECISE 1  /* fp32 CUDA-core math and accumulation */
#define TAU_DXB_PATH_TENSOR  2  /* tcgen05/TMEM + TMA; error if unsupported */

/* ---- WTA modes ------------------------------------------------------------ */
#define TAU_DXB_WTA_THRESHOLD 0 /* keep x >= k-th largest (ties keep more) */
#define TAU_DXB_WTA_EXACT_K   1 /* keep exactly k; ties by lowest index    */
#define TAU_DXB_WTA_GELU_INPUT 0x100 /* or'ed into the mode of wta_fwd: x is the
                                        pre-activation, the select runs on
                                        gelu(x) (erf form, bf16-rounded) and y
                                        is gelu(x) where kept; bf16 rows of d a
                                        multiple of 256, threshold mode, y given */

/* Library version (major*10000 + minor*100 + patch). */
TAU_DXB_API int tau_dxb_version(void);

/* Static message for a status code. */
TAU_DXB_API const char* tau_dxb_strerror(int status);

/* Message describing the calling thread's most recent failure ("" if none). */
TAU_DXB_API const char* tau_dxb_last_error(void);

/* Device-side error word of the current device (0 = none): bit 1/2/4 = a
 * tensor-core kernel gave up waiting (TMA / MMA / softmax role) after its
 * time limit instead of hanging; TAU_DXB_DEVERR_SELFTEST = the wait of
 * tau_dxb_selftest_wait_timeout gave up. Synchronises the device; reset != 0
 * clears it. Returns -1 if it cannot be read. No reference counterpart
 * (diagnostic). */
#define TAU_DXB_DEVERR_SELFTEST 0x100
TAU_DXB_API int tau_dxb_device_error(int32_t reset);

/* Self-test of the bounded waits (no reference counterpart; diagnostic).
 * Launches one CTA whose threads wait on an mbarrier phase that nothing
 * completes, with a limit of `limit_ns` nanoseconds (0 < limit_ns <= 10 s)
 * instead of the kernels' 2 s. The wait gives up, sets
 * TAU_DXB_DEVERR_SELFTEST in the device error word and raises the CTA's abort
 * flag; the CTA frees its tensor memory and returns. Synchronises `stream`.
 * *status: bit 0 = a wait reported completion (a failure), bit 1 = the abort
 * flag was raised (expected). No fault and no trap is involved. */
TAU_DXB_API int tau_dxb_selftest_wait_timeout(uint64_t limit_ns, int32_t* status, void* stream);

/*
 * tau-opus attention forward.
 * Replaces STauOpusAttentionFunction.forward (echo/stau_opus_operator.py:66-111)
 * and STauOpusFlashV2Function.forward (echo/stau_opus_flash_v2.py:406-463).
 *
 *   s = scale * Q K^T (+ mask) (+ causal: finfo(float).min where j > i + Lk - Lq)
 *   m = rowmax s, amax = first argmax,  sig = max(sigma(alpha (s - m)), 1e-8)
 *   q = max(sig^tau, 1e-8),  Z = max(sum q, 1e-8),  out = (q V) / Z
 *
 * tau, alpha: fp32 [H], the per-head VALUES. The reference parametrises them
 *       as tau = softplus(log_tau) + 1 and alpha = exp(log_alpha), computed in
 *       the parameter's dtype (echo/stau_opus_operator.py:90-91); the caller
 *       evaluates that and passes the results.
 * q/k/v/out: `dtype` elements, [B,H,Lq|Lk,D] addressed through the strides.
 * mask: optional additive mask of `mask_dtype`, indexed (b,h,i,j) through
 *       mask_stride (0 strides broadcast). May be combined with `causal`.
 * row_max, row_z: fp32 [B*H*Lq]; row_argmax: int32 [B*H*Lq] (contiguous,
 *       index (b*H + h)*Lq + i) -- the state the backward needs.
 * D must be <= 64 (the tensor path needs D == 64 and bf16/f16).
 */
TAU_DXB_API int tau_attn_fwd(const void* q, const int64_t q_stride[4],
                 const void* k, const int64_t k_stride[4],
                 const void* v, const int64_t v_stride[4],
                 int32_t dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D,
                 const float* tau, const float* alpha,
                 int32_t sigma_id, float scale,
                 const void* mask, int32_t mask_dtype, const int64_t mask_stride[4],
                 int32_t causal,
                 void* out, const int64_t out_stride[4],
                 float* row_max, float* row_z, int32_t* row_argmax,
                 int32_t path, void* stream);

/* Bytes of device workspace tau_attn_bwd needs for this problem (SIZE_MAX
 * when the size does not fit a size_t: such a problem cannot run). */
TAU_DXB_API size_t tau_attn_bwd_workspace_bytes(int64_t B, int64_t H, int64_t Lq, int64_t Lk,
                                    int64_t D);

/*
 * tau-opus attention backward.
 * Replaces STauOpusAttentionFunction.backward (echo/stau_opus_operator.py:113-166)
 * and STauOpusFlashV2Function.backward (echo/stau_opus_flash_v2.py:466-551).
 *
 * Takes the forward's inputs, its output `out` and the upstream gradient
 * `dout`, plus row_max/row_z/row_argmax from tau_attn_fwd. Writes dq, dk, dv
 * (`dtype`, strided) and the per-head sums dtau, dalpha (fp32 [H],
 * overwritten):
 *   dtau[h]   = sum P (dP - D) max(log sig, -30)
 *   dalpha[h] = sum tau P (dP - D) clip(sig'/sig * (s - m), -30, 30)
 * The caller applies the parametrisation's chain rule
 * (dlog_tau = dtau * sigmoid(log_tau), dlog_alpha = dalpha * exp(log_alpha),
 * echo/stau_opus_operator.py:154-161).
 * `workspace` must hold tau_attn_bwd_workspace_bytes(...) bytes of device
 * memory (256-byte aligned); its contents on entry do not matter.
 */
TAU_DXB_API int tau_attn_bwd(const void* q, const int64_t q_stride[4],
                 const void* k, const int64_t k_stride[4],
                 const void* v, const int64_t v_stride[4],
                 const void* out, const int64_t out_stride[4],
                 const void* dout, const int64_t dout_stride[4],
                 int32_t dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D,
                 const float* tau, const float* alpha,
                 int32_t sigma_id, float scale,
                 const void* mask, int32_t mask_dtype, const int64_t mask_stride[4],
                 int32_t causal,
                 const float* row_max, const float* row_z, const int32_t* row_argmax,
                 void* dq, const int64_t dq_stride[4],
                 void* dk, const int64_t dk_stride[4],
                 void* dv, const int64_t dv_stride[4],
                 float* dtau, float* dalpha,
                 void* workspace, size_t workspace_bytes,
                 int32_t path, void* stream);

/*
 * tau-opus attention backward that allocates nothing (no counterpart in the
 * reference). For hosts that manage all device memory through their own pool
 * or a fixed budget, and FFI callers without a device allocator: they cannot
 * have the library call cudaMalloc (it bypasses their accounting and can
 * synchronise the device) and may have no workspace to pass in.
 * Same arguments and results as tau_attn_bwd without the workspace; the scratch
 * lives in a fixed 16 MiB device array of the library (held on every GPU that
 * loads the library until exit). Problems needing more than 16 MiB of
 * workspace (tau_attn_bwd_workspace_bytes) return TAU_DXB_ERR_WORKSPACE. Each
 * call resolves the array's address on the current device; the first call on
 * a device also loads the library's device code there, so make it before any
 * stream capture. All calls on a device share the array, which keeps the last
 * call's contents (each call clears what must start at zero): calls whose GPU
 * work overlaps race and must be serialised by the caller. The results are
 * valid only if tau_dxb_device_error() reads 0 once the call's work is done.
 */
TAU_DXB_API int tau_attn_bwd_noalloc(const void* q, const int64_t q_stride[4],
                 const void* k, const int64_t k_stride[4],
                 const void* v, const int64_t v_stride[4],
                 const void* out, const int64_t out_stride[4],
                 const void* dout, const int64_t dout_stride[4],
                 int32_t dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D,
                 const float* tau, const float* alpha,
                 int32_t sigma_id, float scale,
                 const void* mask, int32_t mask_dtype, const int64_t mask_stride[4],
                 int32_t causal,
                 const float* row_max, const float* row_z, const int32_t* row_argmax,
                 void* dq, const int64_t dq_stride[4],
                 void* dk, const int64_t dk_stride[4],
                 void* dv, const int64_t dv_stride[4],
                 float* dtau, float* dalpha,
                 int32_t path, void* stream);

/*
 * WTA forward: per-row top-k selection over the last dimension.
 * Replaces _triton_wta_forward / _WTAFusedSTE.forward (echo/triton_wta.py:71-100),
 * _torch_wta_forward (echo/triton_wta.py:117-123) and the mask of
 * SparseGradWTA_Function.forward (echo/patch_whisper_sparse_grad.py:45-55).
 *
 * x: [n_rows, d] of `dtype`, rows `row_stride` elements apart.
 * k: number of winners; if k_dev is non-NULL the kernel reads k from that
 *    device int32 instead (no host round trip). k is clamped to [1, d].
 * mode: TAU_DXB_WTA_THRESHOLD or TAU_DXB_WTA_EXACT_K.
 * y: optional [n_rows, d] contiguous output y = keep ? x : 0 (NULL: mask only,
 *    the sparse_grad identity forward).
 * bitmask: [n_rows, (d+7)/8] bytes, bit (j%8) of byte j/8 = keep[j].
 * win_counts: optional int32 [d]; each kept element adds 1 to its column.
 */
TAU_DXB_API int wta_fwd(const void* x, int32_t dtype, int64_t n_rows, int64_t d, int64_t row_stride,
            int64_t k, const int32_t* k_dev, int32_t mode,
            void* y, uint8_t* bitmask, int32_t* win_counts, void* stream);

/*
 * WTA backward (straight-through): dx = dy * keep.
 * Replaces _wta_backward_kernel / _WTAFusedSTE.backward (echo/triton_wta.py:53-68,
 * 102-114) and SparseGradWTA_Function.backward
 * (echo/patch_whisper_sparse_grad.py:57-60).
 * dy, dx: contiguous [n_rows, d] of `dtype` (may alias); bitmask as wta_fwd.
 */
TAU_DXB_API int wta_bwd(const void* dy, int32_t dtype, const uint8_t* bitmask,
            int64_t n_rows, int64_t d, void* dx, void* stream);

/*
 * Backward through GELU and WTA together, for a forward run with
 * TAU_DXB_WTA_GELU_INPUT: dx = gelu'(x) * (dy * keep), with dy * keep rounded to
 * bf16 and the GELU gradient in fp32 as PyTorch's bf16 GELU backward forms it.
 * Replaces the WTA backward (echo/triton_wta.py:53-68) followed by the MLP's
 * GELU backward in the encoder layers of echo/patch_whisper_sparse_grad.py.
 * dy, x (the pre-activation), dx: bf16 [n_rows, d] contiguous, 16-byte
 * aligned, d a multiple of 8; bitmask as wta_fwd.
 */
TAU_DXB_API int wta_bwd_gelu(const void* dy, const void* x, const uint8_t* bitmask, int64_t n_rows,
                             int64_t d, void* dx, void* stream);

/*
 * k for every learnable-k layer at once, on the device:
 *   k[i] = clamp(round_half_even(sigmoid(logit[i]) * d_ff), 1, d_ff)
 * Replaces LearnableKRatio.get_k (echo/patch_whisper_sparse_grad.py:159-161)
 * without its per-layer .item() host sync. logits: fp32 [n]; k_out: int32 [n].
 */
TAU_DXB_API int wta_k_from_logits(const float* logits, int64_t n, int64_t d_ff, int32_t* k_out,
                      void* stream);

/*
 * Whisper log-mel features of a batch of waveforms on the GPU.
 * Replaces the per-sample host call processor.feature_extractor(audio,
 * sampling_rate=16000) of the reference's dataset (echo/train_echo_opus1.py:126),
 * i.e. WhisperFeatureExtractor: centred 400-sample frames every 160 samples
 * (reflect padding), periodic Hann window, power spectrum, mel filter bank,
 * log10(max(mel, 1e-10)), then per sample max(x, max - 8) and (x + 4) / 4.
 *
 * audio: fp32 [batch, n_samples], 16 kHz, n_samples a multiple of 160 and
 *        >= 400 (480000 = 30 s for Whisper; pad or truncate before the call).
 * mel_filters: fp32 [201][80] (row = frequency bin), the extractor's mel_filters.
 * out: fp32 [batch, 80, n_samples / 160].
 * workspace: device memory of whisper_log_mel_workspace_bytes(batch) bytes.
 */
TAU_DXB_API size_t whisper_log_mel_workspace_bytes(int64_t batch);
TAU_DXB_API int whisper_log_mel(const float* audio, int64_t batch, int64_t n_samples,
                                const float* mel_filters, float* out, void* workspace,
                                size_t workspace_bytes, void* stream);

/*
 * tau* per score row: the batched Newton solver for
 *   tau* = argmin_tau KL(softmax(s) || softmax(tau * log sigma(s))).
 * Replaces solve_tau_star (tau_star/tau_star_solver.py:60-128), as
 * estimate_tau_per_head calls it (tau_star/compute_tau_star_echo.py:116-136,
 * n_iter = 100), with every Newton step of a row fused on chip.
 *
 * scores: fp32 [n_rows, T] with row stride row_stride (elements), T in
 *         [1, TAU_DXB_TAU_STAR_MAX_KEYS]; masked keys may hold any finite
 *         value or -inf, as in the reference.
 * sigma: TAU_DXB_SIGMA_*; n_iter >= 0 Newton steps from tau_init, each
 *        clamped to [tau_min, tau_max]; eps damps zero variance.
 * tau_out, kl_out: fp32 [n_rows]; T == 1 gives (tau_init, 0); non-finite
 *        results become tau_init and 0, as in the reference.
 */
TAU_DXB_API int tau_star_solve(const float* scores, int64_t n_rows, int64_t T, int64_t row_stride,
                               int32_t sigma, int32_t n_iter, float tau_init, float tau_min,
                               float tau_max, float eps, float* tau_out, float* kl_out,
                               void* stream);

/*
 * One-shot tau estimate per score row, the Newton solver's warm start:
 *   tau = clamp(Cov_ref(s, log sigma(s)) / (Var_ref(log sigma(s)) + 1e-6), 0.1, 10)
 * under ref = softmax(s). Replaces solve_tau_star_analytic
 * (tau_star/tau_star_solver.py:131-151). scores as tau_star_solve (any T >= 1);
 * tau_out: fp32 [n_rows]. A NaN result is kept, as in the reference.
 */
TAU_DXB_API int tau_star_analytic(const float* scores, int64_t n_rows, int64_t T, int64_t row_stride,
                                  int32_t sigma, float* tau_out, void* stream);

/*
 * fp32 LayerNorm over the last dimension, as autocast runs the nn.LayerNorm
 * layers of the Whisper model trained by echo/train_echo_opus1.py:405-434
 * (transformers' WhisperEncoderLayer / WhisperDecoderLayer norms and the two
 * final norms): y = (x - mean) * rstd * gamma + beta with
 * rstd = 1 / sqrt(var + eps), var the biased variance.
 * x: fp32 [M, d] contiguous; y: [M, d] of y_dtype (TAU_DXB_F32, or TAU_DXB_BF16
 * rounded to nearest even -- what autocast would cast the fp32 output to for a
 * bf16 GEMM that is its only consumer); gamma, beta: fp32 [d]; mean, rstd:
 * fp32 [M] (saved for the backward). d a multiple of 128 up to 1024; x, y,
 * gamma and beta 16-byte aligned.
 */
TAU_DXB_API int tau_layer_norm_fwd(const float* x, int64_t M, int64_t d, const float* gamma,
                                   const float* beta, float eps, void* y, int32_t y_dtype,
                                   float* mean, float* rstd, void* stream);

/*
 * Its backward: dy [M, d] of dy_dtype (fp32 or bf16), dx fp32 [M, d], and
 * dgamma, dbeta [d] summed over the rows in a fixed order (the same bits on
 * every call). workspace: device memory of
 * tau_layer_norm_bwd_workspace_bytes(M, d) bytes, 16-byte aligned.
 */
TAU_DXB_API size_t tau_layer_norm_bwd_workspace_bytes(int64_t M, int64_t d);
TAU_DXB_API int tau_layer_norm_bwd(const void* dy, int32_t dy_dtype, const float* x,
                                   const float* mean, const float* rstd, const float* gamma,
                                   int64_t M, int64_t d, float* dx, float* dgamma, float* dbeta,
                                   void* workspace, size_t workspace_bytes, void* stream);

/*
 * Column sums of a row-major [M, N] matrix, out[n] = sum_m x[m, n], fp32
 * accumulation in a fixed order (the same bits on every call): the bias
 * gradient of the linear layers of the Whisper model that
 * echo/train_echo_opus1.py:405-434 trains (autograd's grad_output.sum(0)).
 * x: bf16 or fp32 (dtype), 16-byte aligned, N a multiple of 8; out: N
 * values of out_dtype (bf16 or fp32). workspace: device memory of
 * tau_column_sum_workspace_bytes(M, N) bytes, 4-byte aligned.
 */
TAU_DXB_API size_t tau_column_sum_workspace_bytes(int64_t M, int64_t N);
TAU_DXB_API int tau_column_sum(const void* x, int32_t dtype, int64_t M, int64_t N, void* out,
                               int32_t out_dtype, void* workspace, size_t workspace_bytes,
                               void* stream);

/*
 * Fixed-tau attention weights from materialised scores: the forward of
 * STauOpusMaxStableFn (echo/patch_whisper_stau.py:74-87), the operator of the
 * fixed-tau patch (apply_fixed_stau, echo/patch_whisper_stau.py:279-322).
 * scores: fp32 rows of length L, `row_stride` elements apart; attn: fp32
 * [rows, L] contiguous. Per row: x = s - max(s), q = max(sigma(x), 1e-8)^tau,
 * attn = q / max(sum q, 1e-8). tau: fp32 device array of n_tau values; row r
 * uses tau[(r / rows_per_tau) % n_tau] (n_tau = H and rows_per_tau = Lq for
 * [B, H, Lq, Lk] scores and a per-head tau; n_tau = 1 for one tau).
 * sigma: TAU_DXB_SIGMA_SOFTPLUS .. TAU_DXB_SIGMA_TANH_SHIFT.
 */
TAU_DXB_API int tau_opus_fixed_fwd(const float* scores, int64_t rows, int64_t L, int64_t row_stride,
                                   const float* tau, int64_t n_tau, int64_t rows_per_tau,
                                   int32_t sigma_id, float* attn, void* stream);

/*
 * Its backward (echo/patch_whisper_stau.py:89-112): grad_scores from the
 * upstream gradient of attn (fp32 [rows, L] contiguous), the same scores, tau
 * and sigma; grad_scores is fp32 [rows, L] contiguous.
 */
TAU_DXB_API int tau_opus_fixed_bwd(const float* scores, const float* grad_attn, int64_t rows, int64_t L,
                                   int64_t row_stride, const float* tau, int64_t n_tau,
                                   int64_t rows_per_tau, int32_t sigma_id, float* grad_scores,
                                   void* stream);

/*
 * Soft-prune gradient mask: out = grad * keep along one axis.
 * Replaces the gradient hooks of echo/patch_whisper_sparse_grad.py:167-194
 * (fc1.weight rows, fc1.bias, fc2.weight columns) that prune_low_winners
 * (echo/patch_whisper_sparse_grad.py:352-395) activates.
 * grad, out: [rows, cols] row-major of `dtype` (may alias); keep: uint8 [rows]
 * (axis 0) or [cols] (axis 1), nonzero = keep. The product is a multiply by
 * 1.0 / 0.0 in the gradient's type, so a non-finite gradient under a 0 stays
 * NaN, as in the reference.
 */
TAU_DXB_API int tau_grad_mask(const void* grad, int32_t dtype, int64_t rows, int64_t cols,
                              const uint8_t* keep, int32_t axis, void* out, void* stream);

/*
 * Cross-entropy over bf16 logits with fp32 math, the loss of
 * echo/train_echo_opus1.py:405-420 (F.cross_entropy of the LM-head logits,
 * labels == ignore_index not counted), without an fp32 copy of the logits.
 * logits: bf16 [M, V] row-major, 16-byte aligned, V a multiple of 8;
 * labels: int64 [M]. Forward writes loss_row[m] = logsumexp(x_m) - x_m[label]
 * (0 for an ignored row, NaN for a label outside [0, V)) and lse[m]; the mean
 * is loss_row summed / the number of counted rows. Backward writes
 * dlogits = (softmax(x_m) - onehot(label)) * grad_scale[0] in bf16, 0 for
 * ignored rows; grad_scale is a device fp32 scalar (dloss / counted rows).
 */
TAU_DXB_API int tau_cross_entropy_fwd(const void* logits, int64_t M, int64_t V, const int64_t* labels,
                                      int64_t ignore_index, float* loss_row, float* lse, void* stream);
TAU_DXB_API int tau_cross_entropy_bwd(const void* logits, int64_t M, int64_t V, const int64_t* labels,
                                      int64_t ignore_index, const float* lse, const float* grad_scale,
                                      void* dlogits, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TAU_DXB_H */
