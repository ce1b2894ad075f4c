// common.cuh -- shared definitions of libgtmoe.so (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/gtmoe.h"

namespace gtmoe {

// Error reporting: thread-local message + code (api.cu).
void set_error(const char *fmt, ...);
int fail(int code, const char *fmt, ...);

#define GT_CUDA(call)                                                                                   \
    do {                                                                                                \
        cudaError_t e_ = (call);                                                                        \
        if (e_ != cudaSuccess)                                                                          \
            return ::gtmoe::fail(GTMOE_ECUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                 __FILE__, __LINE__);                                                   \
    } while (0)

#define GT_CHECK(call)             \
    do {                           \
        int rc_ = (call);          \
        if (rc_ != 0) return rc_;  \
    } while (0)

// Values per float32 scale in Int8/FP4 rows (lowprecision/lowprecision.go:46).
constexpr int kValuesPerScale = 16;

__host__ __device__ inline int scale_blocks(int width) { return (width + kValuesPerScale - 1) / kValuesPerScale; }
__host__ __device__ inline int fp4_row_bytes(int width) { return (width + 1) / 2; }

// E2M1 magnitudes with the sign in bit 3 (lowprecision/rows.go:205).
// Built from the bits: magnitude code c = 2e + m is m/2 for e = 0, else
// (1 + m/2) * 2^(e-1); code 8 is +0 as in the reference table.
__device__ __forceinline__ float fp4_value(uint32_t code) {
    uint32_t e = (code >> 1) & 3u, m = code & 1u;
    uint32_t bits = e ? (((e + 126u) << 23) | (m << 22)) : (m ? 0x3f000000u : 0u);
    if (code & 7u) bits |= (code & 8u) << 28;
    return __uint_as_float(bits);
}

// Activations in float32/float64 (activationfunction.go:35-37, :102-105;
// moreactivationfunctions.go:207-243).
template <typename T>
__device__ __forceinline__ T sigmoid_t(T x) {
    return T(1) / (T(1) + exp(-x));
}
template <>
__device__ __forceinline__ float sigmoid_t<float>(float x) {
    return 1.f / (1.f + __expf(-x));
}

template <typename T>
__device__ __forceinline__ T gate_act(T x, int clamped, T limit) {
    if (clamped && x > limit) x = limit;
    return x * sigmoid_t<T>(x);
}
// float SiLU as x / (1 + e^-x) with the fast reciprocal (<= 2 ulp)
template <>
__device__ __forceinline__ float gate_act<float>(float x, int clamped, float limit) {
    if (clamped && x > limit) x = limit;
    return __fdividef(x, 1.f + __expf(-x));
}
template <typename T>
__device__ __forceinline__ T up_act(T x, int clamped, T limit) {
    if (clamped) {
        if (x > limit) return limit;
        if (x < -limit) return -limit;
    }
    return x;
}

// dtype helpers
template <typename T>
__device__ __forceinline__ T from_double(double v);
template <>
__device__ __forceinline__ double from_double<double>(double v) { return v; }
template <>
__device__ __forceinline__ float from_double<float>(double v) { return (float)v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_double<__nv_bfloat16>(double v) { return __double2bfloat16(v); }

__device__ __forceinline__ double load_as_double(const void *p, int dtype, int64_t i) {
    switch (dtype) {
    case GTMOE_DTYPE_F64: return ((const double *)p)[i];
    case GTMOE_DTYPE_F32: return (double)((const float *)p)[i];
    default: return (double)__bfloat162float(((const __nv_bfloat16 *)p)[i]);
    }
}

inline size_t dtype_size(int dtype) {
    return dtype == GTMOE_DTYPE_F64 ? 8 : dtype == GTMOE_DTYPE_F32 ? 4 : 2;
}

// One expert's three layers as the grouped kernels read them.
struct ExpertLayers {
    const void *w[3];       // codes: f64 / f32 / int8 / packed fp4
    const float *s[3];      // Int8/FP4 scales, rows*ceil(width/16)
    const float *b32[3];    // biases as float
    const double *b64[3];   // biases as double
    const uint8_t *tiled[3];  // Int8/FP4 codes+scales re-laid in tile chunks (tensor-core path) or NULL
};

// One group of rows that run through one expert (shared or routed).
struct Group {
    int64_t x_row0;   // first row in the activation buffer
    int64_t h_row0;   // first row in the hidden / expert-output buffers
    int64_t m;        // rows
    int32_t expert;   // index into the ExpertLayers table
    int32_t pad;
};

// Bounded spin limit of every device-side wait, in nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

}  // namespace gtmoe
