// block.cu -- the mixture-of-experts half of a transformer block on the GPU:
// out = x + MoE(RMSNorm(x)) (transformer.Block.Forward without hyper-
// connections, transformer/block.go:72-77; dropout is the identity at
// inference), so that a block's feed-forward step needs one call and no host
// round trip between the norm, the mixture and the residual.
//
// RMSNorm.Forward (normalization/rmsnorm.go:33-53) is restated operation for
// operation in float64: the sum of squares is one sequential DotProduct
// (vectormath/vector.go:67-74, each product and partial sum rounded), then
// / d, + epsilon, a correctly rounded square root, and value / rms * weight
// per element.  The normalized rows are the reference's bits, so routing on
// them is exact as in gtmoe_forward.
#include "handle.h"

namespace gtmoe {
namespace {

// One warp per row: lanes square 32 inputs at a time (products rounded as in
// the reference), lane 0 adds them in order from shared memory; then every
// lane writes its share of the normalized row.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const void *__restrict__ x, int x_dtype, int64_t T, int d,
                                                      const double *__restrict__ w, double eps,
                                                      double *__restrict__ y, __nv_bfloat16 *__restrict__ y16,
                                                      __nv_bfloat16 *__restrict__ y16mid,
                                                      __nv_bfloat16 *__restrict__ y16lo) {
    __shared__ double buf[8][32];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    const int64_t warps = (int64_t)gridDim.x * 8;
    for (int64_t t = (int64_t)blockIdx.x * 8 + wib; t < T; t += warps) {
        const int64_t x0 = t * d;
        double s = 0;
        for (int i0 = 0; i0 < d; i0 += 32) {
            const int i = i0 + lane;
            double v = 0;
            if (i < d) v = load_as_double(x, x_dtype, x0 + i);
            buf[wib][lane] = __dmul_rn(v, v);
            __syncwarp();
            if (lane == 0) {
                const int n = d - i0 < 32 ? d - i0 : 32;
                for (int j = 0; j < n; j++) s = __dadd_rn(s, buf[wib][j]);
            }
            __syncwarp();
        }
        s = __shfl_sync(0xffffffffu, s, 0);
        const double rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(s, (double)d), eps));
        for (int i = lane; i < d; i += 32) {
            const double v = __dmul_rn(__ddiv_rn(load_as_double(x, x_dtype, x0 + i), rms), w[i]);
            y[x0 + i] = v;
            const __nv_bfloat16 hi = __double2bfloat16(v);  // what the gather would make of v
            y16[x0 + i] = hi;
            // the router's second and third terms (v - hi - mid - lo within 2^-24 |v|)
            const double r1 = v - (double)__bfloat162float(hi);
            const __nv_bfloat16 mid = __double2bfloat16(r1);
            y16mid[x0 + i] = mid;
            y16lo[x0 + i] = __double2bfloat16(r1 - (double)__bfloat162float(mid));
        }
    }
}

}  // namespace
}  // namespace gtmoe

using namespace gtmoe;

extern "C" {

int gtmoe_set_norm(gtmoe_t h, const double *weights, double epsilon) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    if (!weights) return fail(GTMOE_EINVAL, "RMSNorm weights are NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    GT_CUDA(cudaSetDevice(h->device));
    GT_CHECK(h->norm_w.ensure(sizeof(double) * h->cfg.d_model));
    GT_CUDA(cudaMemcpyAsync(h->norm_w.p, weights, sizeof(double) * h->cfg.d_model, cudaMemcpyDefault, h->stream));
    GT_CUDA(cudaStreamSynchronize(h->stream));
    h->norm_eps = epsilon;
    h->norm_set = 1;
    return 0;
}

int gtmoe_forward_block(gtmoe_t h, const void *x, int x_dtype, int64_t T, const int64_t *token_ids, void *out,
                        int out_dtype, int32_t *chosen, double *gates, int32_t *perm, int64_t *load) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    {
        std::lock_guard<std::mutex> lock(h->mu);
        if (!h->norm_set) return fail(GTMOE_ENOTREADY, "the block's RMSNorm weights are not set (gtmoe_set_norm)");
        if (h->n_ranks > 1) return fail(GTMOE_EINVAL, "gtmoe_forward_block runs on one GPU");
        if (T < 0) return fail(GTMOE_EINVAL, "mixture of experts: negative number of rows %lld", (long long)T);
        if (T > 0 && (!x || !out)) return fail(GTMOE_EINVAL, "mixture of experts: x and out must be given");
        if (x_dtype < GTMOE_DTYPE_F64 || x_dtype > GTMOE_DTYPE_BF16 || out_dtype != x_dtype)
            return fail(GTMOE_EINVAL, "the block's output has the input's dtype (the residual is the input)");
        if (T == 0) return forward_locked(h, x, x_dtype, 0, token_ids, nullptr, out, out_dtype, chosen, gates, perm, load);
        GT_CUDA(cudaSetDevice(h->device));
        const int d = h->cfg.d_model;
        const size_t xbytes = dtype_size(x_dtype) * (size_t)T * d;
        cudaPointerAttributes at;
        const bool x_dev = cudaPointerGetAttributes(&at, x) == cudaSuccess &&
                           (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged);
        cudaGetLastError();
        const void *xd = x;
        if (!x_dev) {
            GT_CHECK(h->block_x.ensure(xbytes));
            GT_CUDA(cudaMemcpyAsync(h->block_x.p, x, xbytes, cudaMemcpyHostToDevice, h->stream));
            xd = h->block_x.p;
        }
        GT_CHECK(h->block_xn.ensure(sizeof(double) * (size_t)T * d));
        GT_CHECK(h->block_xn16.ensure(sizeof(__nv_bfloat16) * (size_t)T * d));
        GT_CHECK(h->block_xn16mid.ensure(sizeof(__nv_bfloat16) * (size_t)T * d));
        GT_CHECK(h->block_xn16lo.ensure(sizeof(__nv_bfloat16) * (size_t)T * d));
        const int64_t blocks = (T + 7) / 8;
        rmsnorm_kernel<<<(unsigned)(blocks < 65535 ? blocks : 65535), 256, 0, h->stream>>>(
            xd, x_dtype, T, d, h->norm_w.as<double>(), h->norm_eps, h->block_xn.as<double>(),
            h->block_xn16.as<__nv_bfloat16>(), h->block_xn16mid.as<__nv_bfloat16>(),
            h->block_xn16lo.as<__nv_bfloat16>());
        GT_CUDA(cudaGetLastError());
        note_launches(1);
        // the mixture on the normalized rows (device, float64; the experts'
        // bf16 rows gathered from their bf16 rounding), the input as the residual
        h->gather_bf16 = h->block_xn16.p;
        h->router_bf16_mid = h->block_xn16mid.p;
        h->router_bf16_lo = h->block_xn16lo.p;
        const int rc = forward_locked(h, h->block_xn.p, GTMOE_DTYPE_F64, T, token_ids, xd, out, out_dtype, chosen,
                                      gates, perm, load);
        h->gather_bf16 = nullptr;
        h->router_bf16_mid = nullptr;
        h->router_bf16_lo = nullptr;
        return rc;
    }
}

}  // extern "C"
