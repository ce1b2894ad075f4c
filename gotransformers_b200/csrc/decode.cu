// decode.cu -- grouped SwiGLU expert products for few rows per expert
// (decode-shaped batches, every group <= kDecodeMaxRows rows, run in tiles
// of 16 rows).
//
// With a handful of tokens per expert the expert products are bound by the
// bytes of the expert weights (feedforward/gatedfeedforward.go:49-57 over
// lowprecision rows, rows.go:207-257), not by tensor throughput.  These
// kernels stream each touched expert's Int8/FP4 weight rows once, in the
// record layout the tensor-core kernels use (dequant.cuh: 64 rows x 64
// inputs, codes then block scales), dequantise them in registers straight into mma.sync
// B fragments (no shared-memory round trip for the decoded weights) and run
// them against the few token rows (16 per m-tile).
//
// Arithmetic: the token rows (bf16) are converted once per unit to f16,
// each row scaled by a power of two that puts its largest magnitude in
// [2^14, 2^15) (exact for every value above 2^-28 of the row's largest,
// since bf16 significands fit f16's), and the weight codes are decoded to
// their unscaled values, exact in f16 (Int8: two byte permutes and a packed
// subtraction per four codes).  One MMA k-step is one 16-input block, which
// shares one float32 scale per weight row, so each MMA runs from a zero
// accumulator and its float32 result is scaled and added to the row's sum
// (fmaf): the products are exact, the scale is applied at full float32
// precision, and the MMAs of a step do not wait on one another.  Int8 16-row
// tiles instead decode f16(code * scale) and accumulate in the MMA
// (decode_scale_after).  The epilogue takes the token rows' power-of-two
// scales back out.
//
// Work unit: (tile of TR = 16 rows of a group, or 8 for batches of at most 8
// tokens, block of 64 output features = one 64-row half of a weight chunk).
// A CTA of eight compute warps and one producer warp runs a contiguous range
// of units, tile-major, so consecutive units share their token tile: the
// producer copies a tile's token rows once per run (one bulk copy per row,
// all inputs; padded rows: conflict-free fragment loads), the compute warps
// convert them once.  The producer keeps a ring of weight steps, one
// contiguous bulk copy per layer per 128-input step (gate and up for kernel
// 1; the records of consecutive k-blocks of a 64-row half are adjacent): the
// TMA engine's rate per CTA grows with the size of each copy, so few large
// copies replace many small ones.  At a tile change it issues the new unit's
// first weight steps before it waits for the previous tile to be released,
// so the ring refills while the last steps of the previous tile are
// computed.  The ring has 2 stages when the batch has units for every CTA
// that fits; a few-token batch runs one or two CTAs per SM with the deepest
// ring that fits.  "full" mbarriers carry the transaction counts,
// "empty" ones are released by each compute warp; no CTA-wide barrier.  The
// tokens are the MMA's M side (16 per m-tile) and the weights its N side:
// warp w owns features 8w..8w+7, so each lane decodes one weight row per
// 16-input block.  Inside a block the MMA's k-slots are mapped to the
// physical inputs {4q..4q+3} of lane q, identically for weights and tokens,
// so a lane decodes one 32-bit word of Int8 codes (or one 16-bit pair of FP4
// codes) per row and block.
#include "common.cuh"
#include "dequant.cuh"
#include "internal.h"

namespace gtmoe {

namespace {

constexpr int kComputeWarps = 8;                          // 8 features each
constexpr int kDecodeThreads = (kComputeWarps + 1) * 32;  // + one producer warp
constexpr int kDecodeFeatures = kHalfRows;               // output features per unit
constexpr int kDecodeStepKB = 2;                          // 64-input k-blocks per weight step
constexpr int kDecodeStages = 2;       // ring depth with as many CTAs per SM as fit
constexpr int kDecodeMaxStages = 12;   // deepest ring (few-unit batches)
#ifndef GTMOE_DECODE_DEEP_RINGS
#define GTMOE_DECODE_DEEP_RINGS 1
#endif
constexpr bool kDecodeDeepRings = GTMOE_DECODE_DEEP_RINGS;
constexpr int kDecodeSmemPerSm = 228 * 1024;   // B200 shared memory per SM
constexpr int kDecodeSmemPerCta = 227 * 1024;  // largest dynamic allocation of one CTA
constexpr int kDecodeStaticSmem = 512;         // the kernel's barriers, row scales, flag (rounded up)

template <int PREC>
struct DecodeLayout {
    static constexpr int kCodeBytes = PREC == GTMOE_INT8 ? 64 : 32;  // per row and 64 inputs
    static constexpr int kChunkRowBytes = kCodeBytes + 16;           // codes + 4 float scales
    static constexpr int kHalf = half_bytes(kCodeBytes);             // codes + scales: one bulk copy
    static_assert(kHalf == kDecodeFeatures * kChunkRowBytes, "one record per 64-row half");
};

// One weight step: per layer the half's records of kDecodeStepKB consecutive
// k-blocks, contiguous in the layer's buffer, so one bulk copy per layer.
template <int PREC, bool GATED>
struct DecodeStage {
    static constexpr int kLayers = GATED ? 2 : 1;
    static constexpr int kLayerBytes = kDecodeStepKB * DecodeLayout<PREC>::kHalf;
    static constexpr int kBytes = kLayers * kLayerBytes;
};

// Token-row pitch in shared memory for K inputs: 32 bytes of padding make
// the 8-byte fragment loads of one warp conflict-free.
__host__ __device__ __forceinline__ int decode_x_pitch(int K) { return 2 * K + 32; }

__device__ __forceinline__ void bulk_copy(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Not volatile: a pure function of its operands, so the compiler may overlap
// the next block's loads and decoding with it.  d = A B (no accumulator
// input): one 16-input block's products, scaled by the caller.
__device__ __forceinline__ void mma_f16_16816_zero(float *d, const uint32_t *a, uint32_t b0, uint32_t b1) {
    const float z = 0.f;
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(z));
}

// B fragment of one weight row (16 inputs of block s): two f16x2, k-slots
// (2q, 2q+1) and (2q+8, 2q+9) = physical inputs 4q..4q+3.  The codes' values
// without their block scale (Int8 -127..127, FP4 +-{0, 0.5, .., 6}), exact in
// f16: the block of 16 inputs is exactly one MMA k-step, so the scale is
// applied to the MMA's float32 result instead (decode_scale below).
template <int PREC>
__device__ __forceinline__ void decode_row_block(const uint8_t *codes, int row, int s, int q, const Fp4Tables &t1,
                                                 uint32_t *o) {
    if (PREC == GTMOE_INT8) {
        // stored codes are code + 128: f16 1024 + byte, minus 1152
        const uint32_t w = *reinterpret_cast<const uint32_t *>(codes + half_code_off(row, 16 * s + 4 * q));
        const uint32_t h01 = prmt(w, 0x64646464u, 0x5140), h23 = prmt(w, 0x64646464u, 0x7362);
        const __half2 bias = __floats2half2_rn(1152.f, 1152.f);
        const __half2 v01 = __hsub2(*reinterpret_cast<const __half2 *>(&h01), bias);
        const __half2 v23 = __hsub2(*reinterpret_cast<const __half2 *>(&h23), bias);
        o[0] = *reinterpret_cast<const uint32_t *>(&v01);
        o[1] = *reinterpret_cast<const uint32_t *>(&v23);
    } else {
        const uint32_t w = *reinterpret_cast<const uint16_t *>(codes + half_code_off(row, 8 * s + 2 * q));
        uint32_t v[4];
        fp4_decode8(w, t1, v);
        o[0] = v[0];
        o[1] = v[1];
    }
}

// Int8 with the block scale folded into the weights: f16(code * scale) (one
// more packed multiplication per four codes), for the kernels that
// accumulate in the MMA (decode_scale_after below).
__device__ __forceinline__ void decode_row_block_scaled(const uint8_t *codes, float sc, int row, int s, int q,
                                                        uint32_t *o) {
    const uint32_t w = *reinterpret_cast<const uint32_t *>(codes + half_code_off(row, 16 * s + 4 * q));
    int8_decode4_f16(w, pack_f16(sc, sc), o);
}

// Where the block scale is applied.  After the MMA (zero-accumulator MMA per
// 16-input block, scaled float32 result added by fmaf): FP4, whose scaled
// decode would rebuild its lookup table for every block, and 8-row tiles.
// Before it (f16(code * scale) weights accumulated by the MMA itself): Int8
// 16-row tiles, where the extra fmaf and registers cost more than the
// multiplication saves (c4 T=64: gate/up 112 vs 117 us).
template <int PREC, int TR>
constexpr bool decode_scale_after() { return PREC == GTMOE_FP4 || TR == 8; }

__device__ __forceinline__ void mma_f16_16816(float *c, const uint32_t *a, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float pick4(const float4 &v, int s) {
    return s == 0 ? v.x : s == 1 ? v.y : s == 2 ? v.z : v.w;
}

// Unit u -> (group, tile, feature block): the m-tile prefix counts tiles of
// TR rows per group.  The CTA keeps the prefix in shared memory (a search
// through global memory would cost a dependent load per step, at every unit).
__device__ __forceinline__ int unit_group(const int *prefix, int n_groups, int tile) {
    int lo = 0, hi = n_groups;  // last g with prefix[g] <= tile
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (prefix[mid] <= tile) lo = mid;
        else hi = mid;
    }
    return lo;
}

// Shared memory of a CTA: the token tile, the weight ring, the tile prefix.
__host__ __device__ __forceinline__ int decode_prefix_bytes(int n_groups) { return ((n_groups + 1) * 4 + 15) & ~15; }

template <int PREC, bool GATED, int TR>
__global__ void __launch_bounds__(kDecodeThreads) decode_kernel(const DecodeArgs a, const int stages) {
    static_assert(TR == 8 || TR == 16, "one m16 MMA tile; 8-row tiles leave its rows 8-15 zero");
    using DL = DecodeLayout<PREC>;
    using ST = DecodeStage<PREC, GATED>;
    extern __shared__ __align__(128) uint8_t dsmem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g8 = lane >> 2, q = lane & 3;
    const int K = GATED ? a.d : a.h;
    const int n_out = GATED ? a.h : a.d;
    const int KB = K / 64;
    const int steps = KB / kDecodeStepKB;  // weight steps per unit
    const int blocks = n_out / kDecodeFeatures;
    const int which = GATED ? 0 : 2;
    const int xpitch = decode_x_pitch(K);
    const __nv_bfloat16 *xin = (const __nv_bfloat16 *)(GATED ? a.xp : a.hp);
    __nv_bfloat16 *out = (__nv_bfloat16 *)(GATED ? a.hp : a.yp);
    uint8_t *xs = dsmem;                                  // TR x xpitch
    uint8_t *ring = dsmem + TR * xpitch;                  // stages x ST::kBytes
    int *sprefix = (int *)(ring + stages * ST::kBytes);   // n_groups + 1 tile counts

    __shared__ uint64_t full[kDecodeMaxStages];   // weight step landed (expect_tx by the producer)
    __shared__ uint64_t empty[kDecodeMaxStages];  // every compute warp is done with the step
    __shared__ uint64_t xfull, xempty;            // token rows of a tile landed / released
    __shared__ float rscale[TR];  // 2^-e of each token row (f16 tile = bf16 row * 2^e)
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kComputeWarps);
        }
        mbar_init(&xfull, 1);
        mbar_init(&xempty, kComputeWarps);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int g = threadIdx.x; g <= a.n_groups; g += blockDim.x) sprefix[g] = (int)__ldg(a.tile_prefix + g);
    __syncthreads();
    const int units = sprefix[a.n_groups] * blocks;  // at most a few hundred thousand
    // a contiguous range of units per CTA, tile-major: consecutive units of a
    // run share their token tile, which is loaded and converted once per run
    const int per_cta = units / (int)gridDim.x, extra = units % (int)gridDim.x;
    const int u_begin = (int)blockIdx.x * per_cta + ((int)blockIdx.x < extra ? (int)blockIdx.x : extra);
    const int u_end = u_begin + per_cta + ((int)blockIdx.x < extra ? 1 : 0);
    volatile int *abort_p = (volatile int *)&abort_flag;
    // ring position of the next weight step (the same sequence for the
    // producer and the compute warps): slot, the parity of its barriers'
    // current phase, and whether the ring has wrapped once (the producer
    // then waits for the slot to be released)
    int slot = 0;
    uint32_t phase = 0;
    bool wrapped = false;
    uint32_t nx = 0;  // token tiles of this CTA so far (xfull / xempty parity)

    // Every warp walks all of this CTA's units, also after an abort (its
    // waits then return at once): the compute warps' named barrier is
    // reached by all eight of them, whatever each one saw of the flag.
    for (int u = u_begin; u < u_end; u++) {
        const int tile = u / blocks;
        const int fb = u - tile * blocks;
        const bool new_tile = u == u_begin || fb == 0;
        const bool last_of_tile = u + 1 == u_end || fb == blocks - 1;
        const int gi = unit_group(sprefix, a.n_groups, tile);
        const Group grp = a.groups[gi];
        const ExpertLayers &L = a.experts[grp.expert];
        const int64_t r0 = (int64_t)(tile - sprefix[gi]) * TR;  // first row of this tile
        const int m = grp.m - r0 < TR ? (int)(grp.m - r0) : TR;

        if (warp == kComputeWarps) {
            // ---- producer: the unit's weight steps into the ring and, for a
            // new tile, its token rows.  The rows wait until the compute
            // warps release the previous tile, so the first weight steps
            // (as many as the ring holds) go out before that wait: the ring
            // refills while the previous unit's last steps are computed.
            const int nt = fb >> 1, half = fb & 1;
            // the 64-row block (2 nt + half) of each layer, its k-block records consecutive
            const uint8_t *w0 = L.tiled[which] + (int64_t)(2 * nt + half) * KB * DL::kHalf;
            const uint8_t *w1 = GATED ? L.tiled[1] + (int64_t)(2 * nt + half) * KB * DL::kHalf : nullptr;
            const uint8_t *xrow0 = (const uint8_t *)(xin + ((GATED ? grp.x_row0 : grp.h_row0) + r0) * (int64_t)K);
            const int x_at = !new_tile ? -1 : nx == 0 ? 0 : (steps < stages ? steps : stages);
            for (int i = 0; i <= steps && !*abort_p; i++) {
                if (i == x_at) {
                    if (nx > 0) mbar_wait(&xempty, (nx - 1) & 1, abort_p, a.err, 13);
                    if (*abort_p) break;  // no new copies once a wait has given up
                    if (lane == 0) mbar_arrive_expect_tx(&xfull, (uint32_t)m * K * 2);
                    __syncwarp();
                    for (int r = lane; r < m; r += 32)
                        bulk_copy(xs + r * xpitch, xrow0 + (int64_t)r * K * 2, K * 2, &xfull);
                }
                if (i == steps) break;
                if (wrapped) mbar_wait(&empty[slot], phase ^ 1, abort_p, a.err, 10);
                if (*abort_p) break;
                if (lane == 0) {
                    uint8_t *st = ring + slot * ST::kBytes;
                    const int kb = i * kDecodeStepKB;
                    mbar_arrive_expect_tx(&full[slot], ST::kBytes);
                    bulk_copy(st, w0 + (int64_t)kb * DL::kHalf, ST::kLayerBytes, &full[slot]);
                    if (GATED)
                        bulk_copy(st + ST::kLayerBytes, w1 + (int64_t)kb * DL::kHalf, ST::kLayerBytes, &full[slot]);
                }
                __syncwarp();
                if (++slot == stages) {
                    slot = 0;
                    phase ^= 1;
                    wrapped = true;
                }
            }
            if (new_tile) nx++;
            continue;
        }

        // ---- compute warps: acc[l] = this tile's 16 tokens x the warp's 8 features
        float acc[2][4];
#pragma unroll
        for (int l = 0; l < 2; l++)
#pragma unroll
            for (int c = 0; c < 4; c++) acc[l][c] = 0.f;
        const int row = warp * 8 + g8;  // this lane's weight row (feature) in the half
        // the epilogue's biases, loaded now so that their latency hides behind the unit
        const int f = fb * kDecodeFeatures + warp * 8 + 2 * q;
        const float *bias0 = L.b32[which];
        const float *bias1 = GATED ? L.b32[1] : nullptr;
        const float b00 = bias0 ? __ldg(bias0 + f) : 0.f, b01 = bias0 ? __ldg(bias0 + f + 1) : 0.f;
        const float b10 = bias1 ? __ldg(bias1 + f) : 0.f, b11 = bias1 ? __ldg(bias1 + f + 1) : 0.f;
        if (new_tile) {
            if (!*abort_p) mbar_wait(&xfull, nx & 1, abort_p, a.err, 14);
            // bf16 token rows -> f16 in place, each row scaled by the power of two
            // that puts its largest magnitude in [2^14, 2^15): exact, no overflow
#pragma unroll
            for (int rr = 0; rr < TR / kComputeWarps; rr++) {
                const int r = warp + kComputeWarps * rr;
                if (r >= m) continue;
                uint32_t *p = reinterpret_cast<uint32_t *>(xs + r * xpitch);
                float mx = 0.f;
                for (int i = lane; i < K / 2; i += 32) {
                    const uint32_t v = p[i];
                    mx = fmaxf(mx,
                               fmaxf(fabsf(__uint_as_float(v << 16)), fabsf(__uint_as_float(v & 0xFFFF0000u))));
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                int e = mx > 0.f ? 14 - ((int)((__float_as_uint(mx) >> 23) & 0xFF) - 127) : 0;
                e = e < -100 ? -100 : e > 100 ? 100 : e;
                const float up = __uint_as_float((uint32_t)(e + 127) << 23);
                for (int i = lane; i < K / 2; i += 32) {
                    const uint32_t v = p[i];
                    p[i] = pack_f16(__uint_as_float(v << 16) * up, __uint_as_float(v & 0xFFFF0000u) * up);
                }
                if (lane == 0) rscale[r] = __uint_as_float((uint32_t)(127 - e) << 23);
            }
            // the producer's next copies into the tile come after these writes
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("bar.sync 1, %0;" ::"n"(kComputeWarps * 32) : "memory");
            nx++;
        }
        const uint8_t *xrow = xs + g8 * xpitch + 8 * q;
        constexpr bool kAfter = decode_scale_after<PREC, TR>();
        const int fcol = warp * 8 + 2 * q;  // this lane's two accumulator features in the half
        const Fp4Tables t1 = fp4_tables_f16(1.f);
        for (int kb0 = 0; kb0 < KB; kb0 += kDecodeStepKB) {
            if (!*abort_p) mbar_wait(&full[slot], phase, abort_p, a.err, 9);
            if (*abort_p) break;  // every later wait returns at once: the ring position no longer matters
            const uint8_t *st = ring + slot * ST::kBytes;
#pragma unroll
            for (int sub = 0; sub < kDecodeStepKB; sub++) {
                const int kb = kb0 + sub;
                // block scales: after the MMA those of the accumulator features
                // fcol and fcol + 1, before it those of this lane's decode row
                float4 sa[2], sb[2];
#pragma unroll
                for (int l = 0; l < ST::kLayers; l++) {
                    const uint8_t *rec = st + l * ST::kLayerBytes + sub * DL::kHalf;
                    if constexpr (kAfter) {
                        const uint8_t *sp = rec + half_scale_off(fcol, DL::kCodeBytes);
                        sa[l] = *reinterpret_cast<const float4 *>(sp);
                        sb[l] = *reinterpret_cast<const float4 *>(sp + 16);
                    } else {
                        sa[l] = *reinterpret_cast<const float4 *>(rec + half_scale_off(row, DL::kCodeBytes));
                    }
                }
#pragma unroll
                for (int s = 0; s < 4; s++) {
                    const uint8_t *xa = xrow + kb * 128 + 32 * s;
                    const uint2 lo = *reinterpret_cast<const uint2 *>(xa);
                    const uint2 hi = TR > 8 ? *reinterpret_cast<const uint2 *>(xa + 8 * xpitch) : make_uint2(0u, 0u);
                    const uint32_t af[4] = {lo.x, hi.x, lo.y, hi.y};
#pragma unroll
                    for (int l = 0; l < ST::kLayers; l++) {
                        const uint8_t *rec = st + l * ST::kLayerBytes + sub * DL::kHalf;
                        uint32_t bw[2];
                        if constexpr (kAfter) {
                            decode_row_block<PREC>(rec, row, s, q, t1, bw);
                            float dd[4];
                            mma_f16_16816_zero(dd, af, bw[0], bw[1]);
                            const float ka = pick4(sa[l], s), kbs = pick4(sb[l], s);
                            acc[l][0] = fmaf(ka, dd[0], acc[l][0]);
                            acc[l][1] = fmaf(kbs, dd[1], acc[l][1]);
                            acc[l][2] = fmaf(ka, dd[2], acc[l][2]);
                            acc[l][3] = fmaf(kbs, dd[3], acc[l][3]);
                        } else {
                            decode_row_block_scaled(rec, pick4(sa[l], s), row, s, q, bw);
                            mma_f16_16816(acc[l], af, bw[0], bw[1]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == stages) {
                slot = 0;
                phase ^= 1;
            }
        }
        // the rows' scales are read before the tile is released: the next
        // tile's conversion rewrites them
        const float rs0 = rscale[g8], rs1 = TR > 8 ? rscale[(g8 + 8) % TR] : 0.f;
        __syncwarp();
        if (last_of_tile && lane == 0) mbar_arrive(&xempty);

        // epilogue: acc[l] = tokens (r0 + g8, r0 + g8 + 8) x features (f, f + 1),
        // in units of the rows' scales
#pragma unroll
        for (int l = 0; l < 2; l++) {
            acc[l][0] *= rs0;
            acc[l][1] *= rs0;
            acc[l][2] *= rs1;
            acc[l][3] *= rs1;
        }
        const float lim = (float)a.clamp_limit;
#pragma unroll
        for (int hf = 0; hf < TR / 8; hf++) {
            const int t = g8 + 8 * hf;
            if (t >= m) continue;
            float v0 = acc[0][2 * hf] + b00, v1 = acc[0][2 * hf + 1] + b01;
            if (GATED) {
                const float u0 = acc[1][2 * hf] + b10, u1 = acc[1][2 * hf + 1] + b11;
                v0 = gate_act<float>(v0, a.clamped, lim) * up_act<float>(u0, a.clamped, lim);
                v1 = gate_act<float>(v1, a.clamped, lim) * up_act<float>(u1, a.clamped, lim);
            }
            *reinterpret_cast<uint32_t *>(out + (grp.h_row0 + r0 + t) * (int64_t)n_out + f) = pack_bf16(v0, v1);
        }
    }
    // every copy the producer issued was waited for by the compute warps;
    // after an abort some may not have been: let them land before the CTA exits
    if (warp == kComputeWarps && *abort_p) {
        const uint64_t t0 = global_timer_ns();
        while (global_timer_ns() - t0 < 1000000ull) {
        }
    }
}

template <int PREC, bool GATED, int TR>
int decode_smem_bytes(const DecodeArgs &a, int stages) {
    return TR * decode_x_pitch(GATED ? a.d : a.h) + stages * DecodeStage<PREC, GATED>::kBytes +
           decode_prefix_bytes(a.n_groups);
}

// Launch shape.  A batch with work units for at least two CTAs per SM runs
// as many CTAs per SM as fit with a 2-stage ring (compute warps per SM hide
// the decode -> MMA latency chains), each with the deepest ring that still
// lets that many fit (c4 T = 8 down kernel: 4 CTAs with 3 stages, 37.5 ->
// 35.9 us).  A batch with fewer units (few tokens: T = 1 makes 154 gate/up
// units) would leave most CTAs idle; it runs one or two CTAs per SM, each
// with the deepest ring that fits.
template <int PREC, bool GATED, int TR>
int decode_ring_for(const DecodeArgs &a, int per_sm) {
    const int budget = (per_sm == 1 ? kDecodeSmemPerCta : kDecodeSmemPerSm / per_sm - 1024) - kDecodeStaticSmem;
    const int room = (budget - decode_smem_bytes<PREC, GATED, TR>(a, 0)) / DecodeStage<PREC, GATED>::kBytes;
    return room < kDecodeStages ? kDecodeStages : room > kDecodeMaxStages ? kDecodeMaxStages : room;
}

template <int PREC, bool GATED, int TR>
int launch_decode_one(const DecodeArgs &a, cudaStream_t st) {
    auto kern = decode_kernel<PREC, GATED, TR>;
    const int n_out = GATED ? a.h : a.d;
    const int64_t units_max = a.max_tiles * (n_out / kDecodeFeatures);
    static int attr = 0;
    auto set_attr = [&](int bytes) -> int {
        if (bytes > attr) {
            GT_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
            attr = bytes;
        }
        return 0;
    };
    int per_sm = 0;
    if (kDecodeDeepRings && units_max <= 2 * (int64_t)a.sms) {
        per_sm = units_max <= a.sms ? 1 : 2;
    } else {
        const int smem2 = decode_smem_bytes<PREC, GATED, TR>(a, kDecodeStages);
        GT_CHECK(set_attr(smem2));
        GT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kDecodeThreads, smem2));
        per_sm = per_sm < 1 ? 1 : per_sm;
    }
    const int stages = decode_ring_for<PREC, GATED, TR>(a, per_sm);
    const int smem = decode_smem_bytes<PREC, GATED, TR>(a, stages);
    GT_CHECK(set_attr(smem));
    // at most per_sm CTAs per SM, as many as fit with this ring
    int fit = 0;
    GT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&fit, kern, kDecodeThreads, smem));
    fit = fit < 1 ? 1 : fit;
    per_sm = per_sm > fit ? fit : per_sm;
    kern<<<per_sm * a.sms, kDecodeThreads, smem, st>>>(a, stages);
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    return 0;
}
}  // namespace

bool decode_usable(int precision, int d, int h, int64_t T, int n_groups) {
    // the token tile of a unit (16 rows x all inputs), the weight ring and the
    // tile prefix fit in shared memory
    const int kmax = d > h ? d : h;
    const int smem = kDecodeTileRows * decode_x_pitch(kmax) + kDecodeStages * DecodeStage<GTMOE_INT8, true>::kBytes +
                     decode_prefix_bytes(n_groups);
    return (precision == GTMOE_INT8 || precision == GTMOE_FP4) && T <= kDecodeMaxRows &&
           d % (64 * kDecodeStepKB) == 0 && h % (64 * kDecodeStepKB) == 0 && d % 128 == 0 && h % 128 == 0 &&
           smem <= 200 * 1024;
}

template <int TR>
static int launch_decode_rows(const DecodeArgs &a, int which, cudaStream_t st) {
    if (a.precision == GTMOE_INT8)
        return which == 1 ? launch_decode_one<GTMOE_INT8, true, TR>(a, st)
                          : launch_decode_one<GTMOE_INT8, false, TR>(a, st);
    return which == 1 ? launch_decode_one<GTMOE_FP4, true, TR>(a, st) : launch_decode_one<GTMOE_FP4, false, TR>(a, st);
}

int launch_decode(const DecodeArgs &a, int which, cudaStream_t st) {
    if (a.tile_rows != 8 && a.tile_rows != kDecodeTileRows)
        return fail(GTMOE_EINVAL, "decode tiles of %d rows (8 or 16 supported)", a.tile_rows);
    return a.tile_rows == 8 ? launch_decode_rows<8>(a, which, st) : launch_decode_rows<kDecodeTileRows>(a, which, st);
}

}  // namespace gtmoe
