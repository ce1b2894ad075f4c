// selftest.cu -- the library's failure path on a device, without a fault.
//
// Every device-side wait of the library is bounded (kWaitLimitNs of
// %globaltimer): on expiry the waiting kernel records an error code, raises
// its abort flag, lets its other roles leave their loops and returns, and the
// host reports GTMOE_ETIMEOUT with the context still usable.  This entry
// point runs that wait (mbar_wait, the primitive of the router, tensor-core
// and decode kernels) on an mbarrier that nothing ever completes, so that a
// caller -- or a test -- can see the timeout reported on a real device
// instead of waiting for a genuine failure.
#include "handle.h"
#include "sm100.cuh"

namespace gtmoe {
namespace {

constexpr int kSelftestCode = 99;

__global__ void wait_selftest_kernel(int *err) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);  // one arrival would complete phase 0; none comes
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(&bar, 0, (volatile int *)&abort_flag, err, kSelftestCode);
}

}  // namespace
}  // namespace gtmoe

using namespace gtmoe;

extern "C" GTMOE_API int gtmoe_bounded_wait_selftest(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return fail(GTMOE_ENODEVICE, "device %d does not exist", device);
    }
    GT_CUDA(cudaSetDevice(device));
    int *err = nullptr;
    GT_CUDA(cudaMalloc(&err, sizeof(int)));
    int rc = 0, v = 0;
    if (cudaMemset(err, 0, sizeof(int)) != cudaSuccess) rc = GTMOE_ECUDA;
    if (!rc) {
        wait_selftest_kernel<<<1, 32>>>(err);
        note_launches(1);
        if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
            cudaMemcpy(&v, err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = GTMOE_ECUDA;
    }
    cudaFree(err);
    if (rc) return fail(rc, "bounded-wait self-test: CUDA error");
    if (v == kSelftestCode)
        return fail(GTMOE_ETIMEOUT, "bounded-wait self-test: the wait gave up after %.1f s and reported it (expected)",
                    kWaitLimitNs * 1e-9);
    return fail(GTMOE_ECUDA, "bounded-wait self-test: the wait did not report a timeout (code %d)", v);
}
