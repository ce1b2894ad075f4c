// quantize.cu -- the reference quantiser on the GPU (lowprecision.Rows.Append,
// lowprecision/rows.go:38-79 with encodeInt8 / encodeFP4,
// lowprecision/lowprecision.go:56-94) and the benchmark input generator.
//
// The quantiser is bit-identical to the reference: block maxima, the float64
// division by 127 or 6, the float32 rounding of the scale, the float64
// division value/scale (IEEE correctly rounded on the GPU as on the CPU),
// round-half-away-from-zero and the strict '>' comparisons against the FP4
// half-way points.
#include "common.cuh"
#include "internal.h"

namespace gtmoe {

__global__ void quantize_rows_kernel(int precision, const double *__restrict__ values, int64_t rows, int width,
                                     void *__restrict__ codes, float *__restrict__ scales) {
    const int blocks = scale_blocks(width);
    const int64_t item = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (precision == GTMOE_FLOAT64 || precision == GTMOE_FLOAT32) {
        if (item >= rows * (int64_t)width) return;
        if (precision == GTMOE_FLOAT64) ((double *)codes)[item] = values[item];
        else ((float *)codes)[item] = (float)values[item];
        return;
    }
    if (item >= rows * (int64_t)blocks) return;
    const int64_t r = item / blocks;
    const int b = (int)(item % blocks);
    const int start = b * kValuesPerScale;
    const int end = min(start + kValuesPerScale, width);
    const double *v = values + r * width;
    double largest = 0.0;
    for (int i = start; i < end; i++)
        if (fabs(v[i]) > largest) largest = fabs(v[i]);
    if (precision == GTMOE_INT8) {
        float s32 = (float)(largest / 127);
        scales[r * blocks + b] = s32;
        double scale = (double)s32;
        int8_t *out = (int8_t *)codes + r * width;
        for (int i = start; i < end; i++) {
            int8_t q = 0;
            if (scale != 0) {
                double rounded = round(v[i] / scale);
                if (rounded > 127) rounded = 127;
                if (rounded < -127) rounded = -127;
                q = (int8_t)rounded;
            }
            out[i] = q;
        }
    } else {
        float s32 = (float)(largest / 6);
        scales[r * blocks + b] = s32;
        double scale = (double)s32;
        const double halfway[7] = {0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5};
        uint8_t *out = (uint8_t *)codes + r * fp4_row_bytes(width);
        for (int i = start; i < end; i += 2) {
            uint8_t pair = 0;
            for (int q = 0; q < 2 && i + q < end; q++) {
                double value = v[i + q];
                uint8_t code = 0;
                if (scale != 0) {
                    uint8_t sign = value < 0 ? 8 : 0;
                    double scaled = fabs(value) / scale;
                    int idx = 0;
                    while (idx < 7 && scaled > halfway[idx]) idx++;
                    code = (uint8_t)(sign | idx);
                }
                pair |= (uint8_t)(code << (4 * q));
            }
            out[i / 2] = pair;
        }
    }
}

int launch_quantize_rows(int precision, const double *values, int64_t rows, int width, void *codes, float *scales,
                         cudaStream_t st) {
    int64_t items = (precision == GTMOE_FLOAT64 || precision == GTMOE_FLOAT32) ? rows * (int64_t)width
                                                                               : rows * (int64_t)scale_blocks(width);
    if (items == 0) return 0;
    quantize_rows_kernel<<<(unsigned)((items + 255) / 256), 256, 0, st>>>(precision, values, rows, width, codes,
                                                                          scales);
    GT_CUDA(cudaGetLastError());
    return 0;
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    uint64_t z = x;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void fill_normal_kernel(void *__restrict__ dev, int dtype, int64_t n, uint64_t key, int64_t offset,
                                   double stddev) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    const uint64_t i = (uint64_t)(offset + j);
    const uint64_t a = splitmix64(key + 2 * i), b = splitmix64(key + 2 * i + 1);
    const double u1 = ((double)(a >> 11) + 1.0) * 0x1.0p-53;
    const double u2 = (double)(b >> 11) * 0x1.0p-53;
    const double z = sqrt(-2.0 * log(u1)) * cospi(2.0 * u2) * stddev;
    if (dtype == GTMOE_DTYPE_F64) ((double *)dev)[j] = z;
    else if (dtype == GTMOE_DTYPE_F32) ((float *)dev)[j] = (float)z;
    else ((__nv_bfloat16 *)dev)[j] = __double2bfloat16(z);
}

int launch_fill_normal(void *dev, int dtype, int64_t n, uint64_t seed, uint64_t stream, int64_t offset, double stddev,
                       cudaStream_t st) {
    if (n == 0) return 0;
    // stream key, as synthetic.stream_key
    uint64_t x = seed ^ (stream * 0xD1B54A32D192ED03ull);
    x += 0x9E3779B97F4A7C15ull;
    uint64_t z = x;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    uint64_t key = z ^ (z >> 31);
    fill_normal_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(dev, dtype, n, key, offset, stddev);
    GT_CUDA(cudaGetLastError());
    return 0;
}

}  // namespace gtmoe
