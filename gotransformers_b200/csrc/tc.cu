// tc.cu -- tcgen05 grouped SwiGLU (placeholder until the kernel lands).
#include "handle.h"

namespace gtmoe {

bool tc_supported(const gtmoe_handle *, int64_t) { return false; }
int tc_prepare(gtmoe_handle *, TcWeights &) { return 0; }
int launch_grouped_tc(gtmoe_handle *, TcWeights &, const TcArgs &, cudaStream_t) {
    return fail(GTMOE_EINVAL, "tensor-core path not available");
}
void tc_release(TcWeights &) {}

}  // namespace gtmoe
