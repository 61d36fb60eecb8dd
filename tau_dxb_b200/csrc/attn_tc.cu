// tau-opus attention, tensor-core path (tcgen05 + TMEM + TMA) -- placeholder
// until the sm_100a kernels land; reports the problem as unsupported.
#include "attn.h"

namespace taudxb {

bool attn_tensor_supported(const AttnProblem&) { return false; }

int attn_fwd_tensor(const AttnProblem&, cudaStream_t) {
  return fail(TAU_DXB_ERR_UNSUPPORTED, "tensor-core attention path not built");
}

int attn_bwd_tensor_main(const AttnProblem&, cudaStream_t) {
  return fail(TAU_DXB_ERR_UNSUPPORTED, "tensor-core attention path not built");
}

}  // namespace taudxb
