// tc.cu - the prefill GEMM route (tcgen05).  Not built yet: the route reports that it
// cannot run any shape, so AUTO never selects it.
#include "kernels.h"

namespace bybycu {

bool tc_supports(const GemmArgs&) { return false; }

int launch_tc(const GemmArgs&) {
    return set_error(BYBYCU_ERR_SHAPE, "tensor-core route is not available in this build");
}

}  // namespace bybycu
