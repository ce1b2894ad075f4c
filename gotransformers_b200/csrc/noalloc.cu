// noalloc.cu -- routing without any device allocation (gtmoe_route_noalloc).
//
// Some callers cannot allocate device memory while they run: a token-by-token
// generation loop (the reference's transformer.Block.ForwardOneToken calls the
// mixture once per generated token, transformer/block.go:111-128) where a
// cudaMalloc would synchronise the whole device between tokens, or a server
// that plans all of its device memory up front and must not grow it.  This
// entry point runs the router of gtmoe_forward (logits, sqrt-softplus
// affinities, exact top-k with the float64 near-tie fix-up, gates) with its
// scratch -- the logits, the float32 gates and the fix-up list -- in one
// file-scope __device__ array instead of the handle's workspace.
//
// The array is kScratchBytes (about 4.3 MB) and exists on every GPU that loads
// the library until the process exits.  Its device address is looked up once
// per device, with that device current, by the first call on that device (so
// that first call should come before any stream capture).  Every call shares
// the array and it keeps the last call's contents; the parts that must start
// at zero are cleared by each call.  Calls that overlap on the GPU (different
// streams or handles on one device) race on the array.
//
// Failures inside a call's kernels -- a bounded wait of the tensor-core router
// that ran out, or (hash routing) a negative token ID, which the reference
// panics on (mixtureofexperts.go:141-143) -- cannot be seen when the call
// returns, since the call does not wait for its kernels.  The kernels record
// them in an error word of the array that only a report clears; each call
// first waits for the work already queued on its stream and, if that word is
// set, clears it and returns the error (GTMOE_ETIMEOUT or GTMOE_EINVAL)
// without routing, so the previous call's chosen/gates are known to be invalid.
#include <mutex>

#include "handle.h"

namespace gtmoe {
namespace {

constexpr int64_t kMaxLogits = 262144;   // T * n_routed doubles
constexpr int64_t kMaxTokens = 65536;    // T
constexpr int64_t kMaxChoices = 524288;  // T * experts_per_token
constexpr size_t kOffLogits = 0;
constexpr size_t kOffGates32 = kOffLogits + kMaxLogits * sizeof(double);
constexpr size_t kOffFlagged = kOffGates32 + kMaxChoices * sizeof(float);
constexpr size_t kOffXnorm = kOffFlagged + kMaxTokens * sizeof(int);  // ||x_t|| of a few-token batch
constexpr size_t kOffCounters = kOffXnorm + kRouterSmallMaxT * sizeof(double);  // [0] fix-up count, [1] error word
constexpr size_t kScratchBytes = kOffCounters + 256;

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
unsigned char *g_scratch_ptr[kMaxDevices];

}  // namespace

static __device__ __align__(256) unsigned char g_route_scratch[kScratchBytes];

// Device address of g_route_scratch on the current device (looked up once).
static int scratch_on_device(int device, unsigned char **out) {
    if (device < 0 || device >= kMaxDevices) return fail(GTMOE_ENODEVICE, "device %d out of range", device);
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[device]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
        if (e != cudaSuccess || !p)
            return fail(GTMOE_ECUDA, "cudaGetSymbolAddress of the routing scratch failed: %s", cudaGetErrorString(e));
        g_scratch_ptr[device] = (unsigned char *)p;
    }
    *out = g_scratch_ptr[device];
    return 0;
}

static bool on_device(const void *p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

}  // namespace gtmoe

using namespace gtmoe;

extern "C" GTMOE_API int gtmoe_route_noalloc(gtmoe_t h, const void *x, int x_dtype, int64_t T,
                                             const int64_t *token_ids, int32_t *chosen, double *gates) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    const gtmoe_config &c = h->cfg;
    const int E = c.n_routed, k = c.experts_per_token, d = c.d_model;
    if (T < 0) return fail(GTMOE_EINVAL, "negative number of rows %lld", (long long)T);
    if (T > kMaxTokens || T * E > kMaxLogits || T * k > kMaxChoices)
        return fail(GTMOE_EINVAL,
                    "gtmoe_route_noalloc: %lld tokens x %d experts (top-%d) exceed its fixed scratch "
                    "(at most %lld tokens, tokens*experts <= %lld, tokens*top-k <= %lld)",
                    (long long)T, E, k, (long long)kMaxTokens, (long long)kMaxLogits, (long long)kMaxChoices);
    if (x_dtype < GTMOE_DTYPE_F64 || x_dtype > GTMOE_DTYPE_BF16) return fail(GTMOE_EINVAL, "unknown dtype");
    if (T == 0) return 0;
    GT_CUDA(cudaSetDevice(h->device));
    if (!x || !chosen || !gates || !on_device(x) || !on_device(chosen) || !on_device(gates))
        return fail(GTMOE_EINVAL, "gtmoe_route_noalloc takes device pointers for x, chosen and gates");
    if (c.hash_routing && (!token_ids || !on_device(token_ids)))
        return fail(GTMOE_EINVAL, "hash routing needs device token IDs");
    if (!c.hash_routing && !h->router_set) return fail(GTMOE_ENOTREADY, "router weights are not set");
    unsigned char *scratch = nullptr;
    GT_CHECK(scratch_on_device(h->device, &scratch));
    int sms = 148;
    GT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, h->device));
    int *counters = (int *)(scratch + kOffCounters);
    // an error an earlier call's kernels recorded (the word is sticky until reported)
    int prev_err = 0;
    GT_CUDA(cudaMemcpyAsync(&prev_err, counters + 1, sizeof(int), cudaMemcpyDeviceToHost, h->stream));
    GT_CUDA(cudaStreamSynchronize(h->stream));
    if (prev_err != 0) {
        GT_CUDA(cudaMemsetAsync(counters + 1, 0, sizeof(int), h->stream));
        GT_CUDA(cudaStreamSynchronize(h->stream));
        if (prev_err == kErrNegativeTokenId)
            return fail(GTMOE_EINVAL,
                        "gtmoe_route_noalloc: an earlier call was given a negative token ID (its chosen and gates "
                        "are invalid); this call did not run");
        return fail(GTMOE_ETIMEOUT,
                    "gtmoe_route_noalloc: an earlier call's router gave up waiting (barrier %d; its chosen and "
                    "gates are invalid); this call did not run",
                    prev_err);
    }
    GT_CUDA(cudaMemsetAsync(counters, 0, sizeof(int), h->stream));

    RouterArgs ra;
    ra.hash = c.hash_routing;
    ra.x = x;
    ra.x_dtype = x_dtype;
    ra.T = T;
    ra.E = E;
    ra.k = k;
    ra.d = d;
    ra.token_ids = token_ids;
    ra.w32 = h->wr32.as<float>();
    ra.w64 = h->wr64.as<double>();
    ra.bias = h->br.as<double>();
    ra.balance = h->bal.as<double>();
    ra.use_tc = !c.hash_routing && h->wr3.p && !h->no_tc && router_tc_usable(x, x_dtype, T, d);
    ra.thresh_scale = (ra.use_tc ? kRouterTcErr : kRouterSimtErr) * h->wmax;
    ra.w3 = h->wr3.p;
    ra.e_pad = h->e_pad;
    ra.err = counters + 1;
    ra.sms = sms;
    ra.logits = (double *)(scratch + kOffLogits);
    ra.xnorm = (double *)(scratch + kOffXnorm);
    ra.chosen = chosen;
    ra.gates64 = gates;
    ra.gates32 = (float *)(scratch + kOffGates32);
    ra.n_fixups = counters;
    ra.flagged = (int *)(scratch + kOffFlagged);
    return launch_router(ra, h->stream);
}
