// combine.cu -- gate-weighted combine (mixtureofexperts.go:182-205) with an
// optional residual (transformer/block.go:77).
//
// Per output element, in the reference's order: start from zero, add each
// shared expert's output (AddMatrices, :183-185), then for each chosen expert
// in the token's chosen order add gate * expert output (:197-205), then add the
// residual if one is given.  Float accumulation for float/bf16 expert outputs,
// double for double.
#include "common.cuh"
#include "internal.h"

namespace gtmoe {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// The token's output rows and gates, read once into shared memory, so that
// each thread's loads of the k expert outputs do not wait on them one by one.
template <typename G>
__device__ __forceinline__ void stage_slots(const CombineArgs &a, int64_t t, int64_t *srow, G *sgate) {
    if (threadIdx.x < a.k) {
        srow[threadIdx.x] = a.routed_row0 + a.slot_row[t * a.k + threadIdx.x];
        if constexpr (sizeof(G) == 8) sgate[threadIdx.x] = a.gates64[t * a.k + threadIdx.x];
        else sgate[threadIdx.x] = a.gates32[t * a.k + threadIdx.x];
    }
    __syncthreads();
}

template <typename YT, typename ACC>
__global__ void __launch_bounds__(256) combine_kernel(CombineArgs a) {
    const int64_t t = blockIdx.x;
    const YT *__restrict__ y = (const YT *)a.y;
    const YT *__restrict__ yr = (const YT *)(a.y_routed ? a.y_routed : a.y);
    const int d = a.d;
    __shared__ int64_t srow[kMaxTopK];
    __shared__ ACC sgate[kMaxTopK];
    stage_slots(a, t, srow, sgate);
    for (int col = threadIdx.x; col < d; col += blockDim.x) {
        ACC acc = ACC(0);
        for (int s = 0; s < a.S; s++) {
            ACC v;
            if constexpr (sizeof(YT) == 8) v = y[(a.shared_row0 + (int64_t)s * a.T + t) * d + col];
            else v = (ACC)to_f<YT>(y[(a.shared_row0 + (int64_t)s * a.T + t) * d + col]);
            acc = acc + v;
        }
#pragma unroll 4
        for (int j = 0; j < a.k; j++) {
            ACC v;
            if constexpr (sizeof(YT) == 8) v = yr[srow[j] * d + col];
            else v = (ACC)to_f<YT>(yr[srow[j] * d + col]);
            acc += sgate[j] * v;
        }
        const int64_t o = t * d + col;
        if (a.residual) acc = (ACC)load_as_double(a.residual, a.out_dtype, o) + acc;
        if (a.out_dtype == GTMOE_DTYPE_F64) ((double *)a.out)[o] = (double)acc;
        else if (a.out_dtype == GTMOE_DTYPE_F32) ((float *)a.out)[o] = (float)acc;
        else ((__nv_bfloat16 *)a.out)[o] = __float2bfloat16((float)acc);
    }
}

// bf16 expert outputs, d % 8 == 0: each thread combines 8 consecutive
// columns with 16-byte loads (same per-element order as combine_kernel).
template <typename OT>
__global__ void __launch_bounds__(256) combine_bf16x8_kernel(CombineArgs a) {
    const int64_t t = blockIdx.x;
    const uint4 *__restrict__ y = (const uint4 *)a.y;
    const uint4 *__restrict__ yr = (const uint4 *)(a.y_routed ? a.y_routed : a.y);
    const int dv = a.d / 8;
    __shared__ int64_t srow[kMaxTopK];
    __shared__ float sgate[kMaxTopK];
    stage_slots(a, t, srow, sgate);
    for (int v = threadIdx.x; v < dv; v += blockDim.x) {
        float acc[8];
#pragma unroll
        for (int q = 0; q < 8; q++) acc[q] = 0.f;
        for (int s = 0; s < a.S; s++) {
            const uint4 p = y[(a.shared_row0 + (int64_t)s * a.T + t) * dv + v];
            const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&p);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float2 f = __bfloat1622float2(h[q]);
                acc[2 * q] = acc[2 * q] + f.x;
                acc[2 * q + 1] = acc[2 * q + 1] + f.y;
            }
        }
#pragma unroll 4
        for (int j = 0; j < a.k; j++) {
            const float g = sgate[j];
            const uint4 p = yr[srow[j] * dv + v];
            const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&p);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float2 f = __bfloat1622float2(h[q]);
                acc[2 * q] += g * f.x;
                acc[2 * q + 1] += g * f.y;
            }
        }
        const int64_t o = t * a.d + (int64_t)v * 8;
        if (a.residual) {
#pragma unroll
            for (int q = 0; q < 8; q++) acc[q] = (float)load_as_double(a.residual, a.out_dtype, o + q) + acc[q];
        }
        if constexpr (sizeof(OT) == 2) {
            uint4 r;
            uint32_t *rw = reinterpret_cast<uint32_t *>(&r);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
                rw[q] = *reinterpret_cast<uint32_t *>(&b);
            }
            *reinterpret_cast<uint4 *>((__nv_bfloat16 *)a.out + o) = r;
        } else if constexpr (sizeof(OT) == 4) {
            float4 *dst = reinterpret_cast<float4 *>((float *)a.out + o);
            dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
        } else {
            double2 *dst = reinterpret_cast<double2 *>((double *)a.out + o);
#pragma unroll
            for (int q = 0; q < 4; q++) dst[q] = make_double2(acc[2 * q], acc[2 * q + 1]);
        }
    }
}

int launch_combine(const CombineArgs &a, cudaStream_t st) {
    if (a.T == 0) return 0;
    if (a.y_dtype == GTMOE_DTYPE_BF16 && a.d % 8 == 0 && ((uintptr_t)a.out & 15) == 0) {
        const int dv = a.d / 8;
        const int threads = dv >= 256 ? 256 : ((dv + 31) / 32) * 32;
        if (a.out_dtype == GTMOE_DTYPE_BF16) combine_bf16x8_kernel<__nv_bfloat16><<<(unsigned)a.T, threads, 0, st>>>(a);
        else if (a.out_dtype == GTMOE_DTYPE_F32) combine_bf16x8_kernel<float><<<(unsigned)a.T, threads, 0, st>>>(a);
        else combine_bf16x8_kernel<double><<<(unsigned)a.T, threads, 0, st>>>(a);
        GT_CUDA(cudaGetLastError());
        note_launches(1);
        return 0;
    }
    int threads = a.d >= 256 ? 256 : ((a.d + 31) / 32) * 32;
    if (a.y_dtype == GTMOE_DTYPE_F64) combine_kernel<double, double><<<(unsigned)a.T, threads, 0, st>>>(a);
    else if (a.y_dtype == GTMOE_DTYPE_F32) combine_kernel<float, float><<<(unsigned)a.T, threads, 0, st>>>(a);
    else combine_kernel<__nv_bfloat16, float><<<(unsigned)a.T, threads, 0, st>>>(a);
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    return 0;
}

}  // namespace gtmoe
