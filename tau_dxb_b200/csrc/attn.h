// Internal interface shared by the tau-opus attention kernels.
#pragma once

#include "common.cuh"

namespace taudxb {

struct AttnProblem {
  // inputs (element strides, order b, h, l, d)
  const void* q; int64_t qs[4];
  const void* k; int64_t ks[4];
  const void* v; int64_t vs[4];
  const void* o; int64_t os[4];       // forward output (backward input)
  const void* dout; int64_t dos[4];   // upstream gradient (backward)
  int dtype;
  int B, H, Lq, Lk, D;
  const float* tau;      // [H] per-head tau values
  const float* alpha;    // [H] per-head alpha values
  int sigma;
  float scale;
  const void* mask; int mask_dtype; int64_t ms[4];
  int causal;
  // forward outputs
  void* out; int64_t outs[4];
  float* row_max; float* row_z; int32_t* row_argmax;
  // backward outputs
  void* dq; int64_t dqs[4];
  void* dk; int64_t dks[4];
  void* dv; int64_t dvs[4];
  float* dtau; float* dalpha;   // [H] sums, zeroed by the prologue
  // backward workspace slices (fp32)
  float* ws_dq;    // [B*H, Lq, D] dQ accumulator (unscaled)
  float* ws_dk;    // [B*H, Lk, D] dK accumulator (unscaled)
  float* ws_drow;  // [B*H, Lq]   rowsum(dO * O)
  float* ws_rowf;  // [B*H, Lq]   rowsum(F) for the argmax correction
};

struct WorkspaceLayout {
  size_t dq, dk, drow, rowf, total;
};
WorkspaceLayout workspace_layout(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D);

// precise (fp32 CUDA-core) kernels
int attn_fwd_precise(const AttnProblem& p, cudaStream_t st);
int attn_bwd_precise_main(const AttnProblem& p, cudaStream_t st);

// tensor-core (tcgen05) kernels; return TAU_DXB_ERR_UNSUPPORTED when the
// problem is outside what they handle.
bool attn_tensor_supported(const AttnProblem& p);
bool attn_tensor_bwd_supported(const AttnProblem& p);
int read_device_error(int reset);
int* device_error_word();   // device address of the kernels' error word
int wait_selftest(uint64_t limit_ns, int32_t* status, cudaStream_t st);   // selftest.cu
int attn_fwd_tensor(const AttnProblem& p, cudaStream_t st);
int attn_bwd_tensor_main(const AttnProblem& p, cudaStream_t st);

// decode forward for a few query rows (KV-cached decoding): one CTA per row,
// one pass over K and V
constexpr int kDecodeMaxRows = 8, kDecodeMaxKeys = 32768;
bool attn_decode_supported(const AttnProblem& p);
int attn_fwd_decode(const AttnProblem& p, cudaStream_t st);

// shared backward stages
int attn_bwd_prologue(const AttnProblem& p, cudaStream_t st);   // zero + rowsum(dO*O)
int attn_bwd_epilogue(const AttnProblem& p, cudaStream_t st);   // argmax fix, scaled dQ/dK

}  // namespace taudxb
