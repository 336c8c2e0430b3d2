// Tensor-core (tcgen05) tree attention.  Not wired in yet: every shape takes
// the CUDA-core kernel until this path lands.
#include "attn.cuh"

namespace gorgon {

bool attn_tc_supported(const AttnArgs&, int) { return false; }

size_t attn_tc_workspace(const AttnArgs&) { return 0; }

void attn_tc_plan(const AttnArgs&, int32_t* splits, int32_t* launches) {
  *splits = 1;
  *launches = 1;
}

int launch_attn_tc(const AttnArgs&, int, void*, size_t, cudaStream_t) {
  return set_error(GORGON_ERR_UNSUPPORTED, "tcgen05 tree attention is not built");
}

}  // namespace gorgon
