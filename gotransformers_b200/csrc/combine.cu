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

template <typename YT, typename ACC>
__global__ void __launch_bounds__(256) combine_kernel(CombineArgs a) {
    const int64_t t = blockIdx.x;
    const YT *__restrict__ y = (const YT *)a.y;
    const int d = a.d;
    for (int col = threadIdx.x; col < d; col += blockDim.x) {
        ACC acc = ACC(0);
        for (int s = 0; s < a.S; s++) {
            ACC v;
            if constexpr (sizeof(YT) == 8) v = y[(a.shared_row0 + (int64_t)s * a.T + t) * d + col];
            else v = (ACC)to_f<YT>(y[(a.shared_row0 + (int64_t)s * a.T + t) * d + col]);
            acc = acc + v;
        }
        for (int j = 0; j < a.k; j++) {
            const int64_t row = a.routed_row0 + a.slot_row[t * a.k + j];
            ACC g, v;
            if constexpr (sizeof(ACC) == 8) {
                g = a.gates64[t * a.k + j];
            } else {
                g = a.gates32[t * a.k + j];
            }
            if constexpr (sizeof(YT) == 8) v = y[row * d + col];
            else v = (ACC)to_f<YT>(y[row * d + col]);
            acc += g * v;
        }
        const int64_t o = t * d + col;
        if (a.residual) acc = (ACC)load_as_double(a.residual, a.out_dtype, o) + acc;
        if (a.out_dtype == GTMOE_DTYPE_F64) ((double *)a.out)[o] = (double)acc;
        else if (a.out_dtype == GTMOE_DTYPE_F32) ((float *)a.out)[o] = (float)acc;
        else ((__nv_bfloat16 *)a.out)[o] = __float2bfloat16((float)acc);
    }
}

int launch_combine(const CombineArgs &a, cudaStream_t st) {
    if (a.T == 0) return 0;
    int threads = a.d >= 256 ? 256 : ((a.d + 31) / 32) * 32;
    if (a.y_dtype == GTMOE_DTYPE_F64) combine_kernel<double, double><<<(unsigned)a.T, threads, 0, st>>>(a);
    else if (a.y_dtype == GTMOE_DTYPE_F32) combine_kernel<float, float><<<(unsigned)a.T, threads, 0, st>>>(a);
    else combine_kernel<__nv_bfloat16, float><<<(unsigned)a.T, threads, 0, st>>>(a);
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    return 0;
}

}  // namespace gtmoe
