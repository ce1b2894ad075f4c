// ep.cu -- expert parallelism across GPUs (placeholder until NCCL lands).
#include "handle.h"

namespace gtmoe {

void ep_destroy(gtmoe_handle *) {}

int ep_forward(gtmoe_handle *, const void *, int, int64_t, const int64_t *, const void *, void *, int, int32_t *,
               double *, int32_t *, int64_t *) {
    return fail(GTMOE_EINVAL, "expert parallelism is not available");
}

int ep_global_load(gtmoe_handle *h, int64_t *load) {
    GT_CUDA(cudaMemcpyAsync(load, h->load.p, sizeof(int64_t) * h->cfg.n_routed, cudaMemcpyDeviceToHost, h->stream));
    GT_CUDA(cudaStreamSynchronize(h->stream));
    return 0;
}

}  // namespace gtmoe

extern "C" {
int gtmoe_ep_unique_id(void *) { return gtmoe::fail(GTMOE_EINVAL, "expert parallelism is not available"); }
int gtmoe_create_ep(const gtmoe_config *, int, int, int, const void *, gtmoe_t *) {
    return gtmoe::fail(GTMOE_EINVAL, "expert parallelism is not available");
}
}
