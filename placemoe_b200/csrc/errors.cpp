// Aggregates the error words of every kernel translation unit.
#include "ops.h"

namespace pm {
int device_error(bool reset) {
  const int codes[] = {pm_error_gemm_dense(reset), pm_error_gemm_moe_fwd(reset), pm_error_gemm_moe_bwd(reset), pm_error_norm(reset), pm_error_route(reset), pm_error_optim(reset),
                       pm_error_loss(reset), pm_error_attn(reset), pm_error_p2p(reset)};
  for (int c : codes)
    if (c) return c;
  return 0;
}
}  // namespace pm
