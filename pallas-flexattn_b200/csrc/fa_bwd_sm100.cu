// FlexAttention backward for B200 (sm_100a): not built yet; fa_bwd falls back to the
// generic kernels while bwd_tc_max_stages reports 0.
#include "fa_internal.h"

namespace fa {

int bwd_tc_max_stages(int, int) { return 0; }

cudaError_t launch_bwd_tc(const AttnArgs&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                          const CUtensorMap&, cudaStream_t) {
  return cudaErrorNotSupported;
}

}  // namespace fa
