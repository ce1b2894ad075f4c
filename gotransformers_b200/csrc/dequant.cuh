// dequant.cuh -- decoding of the reference's Int8 / FP4 rows to bf16 in
// registers (shared by the tensor-core kernels and the decode kernels).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "sm100.cuh"

namespace gtmoe {

// Tile-chunk layout of Int8/FP4 weights (tc.cu, decode.cu): per 128-row block
// and 64-input step one chunk of two 64-row halves, each codes
// [64][code_bytes] then block scales [64][4 floats], so that a half is one
// contiguous bulk copy.  Int8 codes are stored biased, as the bytes q + 128
// (the decoders place them straight into a float or half mantissa).
// Tile-chunk layout of an Int8/FP4 layer for the tensor-core and decode
// kernels (built at set time by tc.cu's relayout): the rows in blocks of 64
// ("halves"), each half's k-blocks (64 inputs) consecutive, so that the
// records of one half over consecutive k-blocks are one contiguous copy.  A
// (half, k-block) record holds the codes column-group major -- 16-byte group
// j of all 64 rows, then group j+1 -- followed by the scales [64 rows][4].
// A lane that reads "its" row's group then touches consecutive 16-byte words
// across the warp (no bank conflicts).  Int8 codes are stored biased (q + 128)
// for the decoders' float/half magic-number conversions.
constexpr int kHalfRows = 64;
__host__ __device__ __forceinline__ constexpr int half_bytes(int code_bytes) { return kHalfRows * (code_bytes + 16); }
// byte `byte` of row r's codes within a record
__host__ __device__ __forceinline__ constexpr int half_code_off(int r, int byte) {
    return (byte >> 4) * (kHalfRows * 16) + r * 16 + (byte & 15);
}
// row r's four block scales (float4) within a record
__host__ __device__ __forceinline__ constexpr int half_scale_off(int r, int code_bytes) {
    return kHalfRows * code_bytes + r * 16;
}

// prmt with the sign-replicating selector mode (msb of a selector nibble set)
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// FP4 (E2M1 magnitudes {0,.5,1,1.5,2,3,4,6}, sign in bit 3; lowprecision.go:48,
// rows.go:205) -> bf16(code * scale).  The eight scaled magnitudes of one
// 16-value block, rounded once to bf16, are split into a high-byte and a
// low-byte table of 8 bytes each; prmt then looks up four codes at a time.
struct Fp4Tables {
    uint32_t hlo, hhi, llo, lhi;
};
__device__ __forceinline__ Fp4Tables fp4_tables(float s) {
    const uint32_t p0 = pack_bf16(0.f, 0.5f * s);
    const uint32_t p1 = pack_bf16(s, 1.5f * s);
    const uint32_t p2 = pack_bf16(2.f * s, 3.f * s);
    const uint32_t p3 = pack_bf16(4.f * s, 6.f * s);
    Fp4Tables t;
    t.hlo = prmt(p0, p1, 0x7531);
    t.hhi = prmt(p2, p3, 0x7531);
    t.llo = prmt(p0, p1, 0x6420);
    t.lhi = prmt(p2, p3, 0x6420);
    return t;
}
// Eight codes (low nibble = even element, rows.go:68-74) -> four bf16x2.
__device__ __forceinline__ void fp4_decode8(uint32_t w, const Fp4Tables &t, uint32_t *o) {
    const uint32_t mag = w & 0x77777777u;
    const uint32_t magh = mag >> 16;
    uint32_t h0 = prmt(t.hlo, t.hhi, mag);
    uint32_t h1 = prmt(t.hlo, t.hhi, magh);
    const uint32_t l0 = prmt(t.llo, t.lhi, mag);
    const uint32_t l1 = prmt(t.llo, t.lhi, magh);
    // sign of code i is bit 4i+3: replicate it into the msb of high byte i
    const uint32_t w4 = w << 4;
    h0 |= prmt(w, w4, 0x9D8C) & 0x80808080u;
    h1 |= prmt(w, w4, 0xBFAE) & 0x80808080u;
    o[0] = prmt(l0, h0, 0x5140);
    o[1] = prmt(l0, h0, 0x7362);
    o[2] = prmt(l1, h1, 0x5140);
    o[3] = prmt(l1, h1, 0x7362);
}

// Four biased Int8 codes (bytes q + 128) -> two bf16x2 of bf16(q * scale):
// the byte becomes the low byte of the float 2^23 + q + 128, from which q is
// recovered exactly.
__device__ __forceinline__ void int8_decode4(uint32_t u, float s, uint32_t *o) {
    const float magic = 8388736.f;  // 2^23 + 128
    const float f0 = __uint_as_float(prmt(u, 0x4B000000u, 0x7650)) - magic;
    const float f1 = __uint_as_float(prmt(u, 0x4B000000u, 0x7651)) - magic;
    const float f2 = __uint_as_float(prmt(u, 0x4B000000u, 0x7652)) - magic;
    const float f3 = __uint_as_float(prmt(u, 0x4B000000u, 0x7653)) - magic;
    o[0] = pack_bf16(f0 * s, f1 * s);
    o[1] = pack_bf16(f2 * s, f3 * s);
}


// ---- f16 variants (decode kernels): the same codes to f16(code * scale)

__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
}

// FP4 tables as in fp4_tables, with the eight scaled magnitudes rounded to f16.
__device__ __forceinline__ Fp4Tables fp4_tables_f16(float s) {
    const uint32_t p0 = pack_f16(0.f, 0.5f * s);
    const uint32_t p1 = pack_f16(s, 1.5f * s);
    const uint32_t p2 = pack_f16(2.f * s, 3.f * s);
    const uint32_t p3 = pack_f16(4.f * s, 6.f * s);
    Fp4Tables t;
    t.hlo = prmt(p0, p1, 0x7531);
    t.hhi = prmt(p2, p3, 0x7531);
    t.llo = prmt(p0, p1, 0x6420);
    t.lhi = prmt(p2, p3, 0x6420);
    return t;
}

// Four biased Int8 codes (bytes q + 128) -> two f16x2 of f16(q * scale): the
// byte becomes the low byte of the f16 1024 + (q + 128); subtracting 1152
// leaves q exactly, and one multiplication by the f16 scale rounds once.
__device__ __forceinline__ void int8_decode4_f16(uint32_t u, uint32_t s2, uint32_t *o) {
    const uint32_t h01 = prmt(u, 0x64646464u, 0x5140);
    const uint32_t h23 = prmt(u, 0x64646464u, 0x7362);
    const __half2 bias = __floats2half2_rn(1152.f, 1152.f);
    const __half2 sc = *reinterpret_cast<const __half2 *>(&s2);
    __half2 v01 = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&h01), bias), sc);
    __half2 v23 = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&h23), bias), sc);
    o[0] = *reinterpret_cast<uint32_t *>(&v01);
    o[1] = *reinterpret_cast<uint32_t *>(&v23);
}

}  // namespace gtmoe
