// router_tc.cu -- router logits on the tcgen05 tensor cores for bf16
// activations (RouterLayer.Forward, mixtureofexperts.go:154 ->
// perceptron/layer.go:133-162: logits = x W_r^T, W_r float64 E x d).
//
// The float64 router weights are split once (at set time) into three bf16
// terms, w = w_hi + w_mid + w_lo + r with |r| <= 2^-24 |w|.  bf16 activations
// are exact, so every product x*w_t is exact in the tensor core; the
// accumulator is reset every 64-element k-block and each block's float32 sum
// is added into float64 registers by the epilogue warps.  Assuming at most one
// float32 rounding per accumulated element, a k-block contributes at most
// 64 * 2^-23 * sum_block |x w| of error, so a logit is within
// 70 * 2^-23 * ||x_t|| * max_e ||w_e|| of the float64 value (Cauchy-Schwarz),
// which is the margin the selection kernel uses to decide when to recompute a
// token's logits in float64 (router.cu).
//
// Float64 rows (the block step's RMSNorm output) are split once into three
// bf16 terms, x = x_hi + x_mid + x_lo + r with |r| <= 2^-24 |x|, and the MMAs
// add x_hi w_t (t = hi, mid, lo), x_mid w_t (t = hi, mid) and x_lo w_hi: the
// dropped r w, x_mid w_lo, x_lo w_mid and the weight residual (2^-24 each) and
// twice the accumulation allowance give 136 * 2^-23 * ||x_t|| * max_e ||w_e||
// (kRouterTc3Err); tokens inside that margin are settled in float64 as
// before.
//
// Persistent kernel, one CTA per SM: warp 0 TMA producer (x tile + the three
// weight tiles), warp 1 TMEM allocator + MMA issuer, warps 2-9 epilogue
// (4 TMEM lane quadrants x 2 column halves).  Tile 128 tokens x 128 experts,
// 3-stage ring of 64 KB, two TMEM accumulators so the float64 accumulation of
// block k overlaps the MMAs of block k+1.  All waits are bounded.
#include "handle.h"
#include "sm100.cuh"

namespace gtmoe {

namespace {

constexpr int kRBM = 128;
constexpr int kRBN = 128;
constexpr int kRBK = 64;
constexpr int kRATile = kRBM * kRBK * 2;      // 16 KB per activation term
constexpr int kRBSub = kRBN * kRBK * 2;       // 16 KB per weight term
constexpr int kRBTile = 3 * kRBSub;           // 48 KB
constexpr int kREpiWarps = 8;
constexpr int kRThreads = (2 + kREpiWarps) * 32;
constexpr int kRTmemCols = 256;
// NX activation terms per row: 1 (bf16 rows, exact) or 3 (float64 rows split
// into three bf16 terms: the block step's normalized rows).  Ring depth as
// shared memory allows.
template <int NX>
struct RouterTcShape {
    static constexpr int kStages = NX == 1 ? 3 : 2;
    static constexpr int kATile = NX * kRATile;
    static constexpr int kSmem = kStages * (kATile + kRBTile) + 1024 + 256;
};
static_assert(RouterTcShape<3>::kSmem <= 232448, "shared memory per CTA");
constexpr uint32_t kRIdesc =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kRBN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

struct RouterTcArgs {
    int64_t T;
    int E, E_pad, d;
    double *logits;
    int *err;
};

template <int NX>
__global__ void __launch_bounds__(kRThreads, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap xmmap,
                     const __grid_constant__ CUtensorMap xlmap, const __grid_constant__ CUtensorMap wmap,
                     const RouterTcArgs a) {
    using SH = RouterTcShape<NX>;
    constexpr int kRStages = SH::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *a_tiles = smem;  // per stage: the x_hi tile (then x_mid, x_lo when NX = 3)
    uint8_t *b_tiles = smem + kRStages * SH::kATile;
    uint64_t *bars = (uint64_t *)(smem + kRStages * (SH::kATile + kRBTile));
    uint64_t *full = bars;
    uint64_t *empty = bars + kRStages;
    uint64_t *tfull = bars + 2 * kRStages;
    uint64_t *tempty = bars + 2 * kRStages + 2;
    uint32_t *tmem_slot = (uint32_t *)(bars + 2 * kRStages + 4);
    volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_nt = a.E_pad / kRBN;
    const int64_t n_mt = (a.T + kRBM - 1) / kRBM;
    const int64_t total = n_mt * n_nt;
    const int KB = a.d / kRBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kRStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kREpiWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kRTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&xmap) : "memory");
            if (NX == 3) {
                asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&xmmap) : "memory");
                asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&xlmap) : "memory");
            }
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&wmap) : "memory");
            int stage = 0;
            uint32_t phase = 0;
            for (int64_t u = blockIdx.x; u < total && !*abort_flag; u += gridDim.x) {
                const int mt = (int)(u / n_nt), nt = (int)(u % n_nt);
                for (int kb = 0; kb < KB; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, a.err, 11)) break;
                    mbar_arrive_expect_tx(&full[stage], SH::kATile + kRBTile);
                    tma_load_2d(a_tiles + stage * SH::kATile, &xmap, kb * kRBK, mt * kRBM, &full[stage]);
                    if (NX == 3) {
                        tma_load_2d(a_tiles + stage * SH::kATile + kRATile, &xmmap, kb * kRBK, mt * kRBM,
                                    &full[stage]);
                        tma_load_2d(a_tiles + stage * SH::kATile + 2 * kRATile, &xlmap, kb * kRBK, mt * kRBM,
                                    &full[stage]);
                    }
                    uint8_t *bt = b_tiles + stage * kRBTile;
#pragma unroll
                    for (int t = 0; t < 3; t++)
                        tma_load_2d(bt + t * kRBSub, &wmap, kb * kRBK, t * a.E_pad + nt * kRBN, &full[stage]);
                    if (++stage == kRStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (*abort_flag) {
                const uint64_t t0 = global_timer_ns();
                while (global_timer_ns() - t0 < 1000000ull) {
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t j = 0;  // k-blocks issued
            bool ok = true;
            for (int64_t u = blockIdx.x; u < total && ok && !*abort_flag; u += gridDim.x) {
                for (int kb = 0; kb < KB; kb++, j++) {
                    const int acc = j & 1;
                    if (!mbar_wait(&tempty[acc], ((j >> 1) & 1) ^ 1, abort_flag, a.err, 12) ||
                        !mbar_wait(&full[stage], phase, abort_flag, a.err, 13)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = sw128_desc(smem_u32(a_tiles + stage * SH::kATile));
                    const uint64_t bdesc = sw128_desc(smem_u32(b_tiles + stage * kRBTile));
                    const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kRBN);
                    // x_hi against the three weight terms; for split rows also
                    // x_mid against w_hi and w_mid, x_lo against w_hi
#pragma unroll
                    for (int k = 0; k < kRBK / 16; k++)
#pragma unroll
                        for (int xi = 0; xi < NX; xi++)
#pragma unroll
                            for (int t = 0; t < 3 - xi; t++)
                                umma_bf16(d_tmem, adesc + (uint64_t)((xi * kRATile) >> 4) + (uint64_t)(2 * k),
                                          bdesc + (uint64_t)((t * kRBSub) >> 4) + (uint64_t)(2 * k), kRIdesc,
                                          (k | t | xi) != 0);
                    umma_commit(&empty[stage]);
                    umma_commit(&tfull[acc]);
                    if (++stage == kRStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else {
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;  // column half: 0 or 1
        uint32_t j = 0;
        bool ok = true;
        for (int64_t u = blockIdx.x; u < total && ok && !*abort_flag; u += gridDim.x) {
            const int mt = (int)(u / n_nt), nt = (int)(u % n_nt);
            double acc64[64];
#pragma unroll
            for (int c = 0; c < 64; c++) acc64[c] = 0.0;
            for (int kb = 0; kb < KB; kb++, j++) {
                const int acc = j & 1;
                if (!mbar_wait(&tfull[acc], (j >> 1) & 1, abort_flag, a.err, 14)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * kRBN + half * 64);
#pragma unroll
                for (int c = 0; c < 64; c += 16) {
                    uint32_t v[16];
                    tmem_ld16(taddr + c, v);
                    tmem_ld_wait();
#pragma unroll
                    for (int q = 0; q < 16; q++) acc64[c + q] += (double)__uint_as_float(v[q]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[acc]);
            }
            if (!ok) break;
            const int64_t t = (int64_t)mt * kRBM + quad * 32 + lane;
            if (t < a.T) {
                double *dst = a.logits + t * a.E;
                const int e0 = nt * kRBN + half * 64;
#pragma unroll
                for (int c = 0; c < 64; c++)
                    if (e0 + c < a.E) dst[e0 + c] = acc64[c];
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kRTmemCols));
    }
}

}  // namespace

bool router_tc_usable(const void *x, int x_dtype, int64_t T, int d) {
    if (x_dtype != GTMOE_DTYPE_BF16 || T < 256 || d % kRBK != 0) return false;
    if (((uintptr_t)x & 15) != 0) return false;
    return true;
}

int launch_router_logits_tc(const void *x, const void *x_mid, const void *x_lo, int64_t T, int d, int E, int E_pad,
                            const void *w3, double *logits, int *err, int sms, cudaStream_t st) {
    CUtensorMap xmap, xmmap, xlmap, wmap;
    const bool split = x_mid && x_lo;
    GT_CHECK(encode_bf16_2d(&xmap, x, d, T, kRBK, kRBM));
    GT_CHECK(encode_bf16_2d(&xmmap, split ? x_mid : x, d, T, kRBK, kRBM));
    GT_CHECK(encode_bf16_2d(&xlmap, split ? x_lo : x, d, T, kRBK, kRBM));
    GT_CHECK(encode_bf16_2d(&wmap, w3, d, (int64_t)3 * E_pad, kRBK, kRBN));
    RouterTcArgs a;
    a.T = T;
    a.E = E;
    a.E_pad = E_pad;
    a.d = d;
    a.logits = logits;
    a.err = err;
    static bool attr_set = false;
    if (!attr_set) {
        GT_CUDA(cudaFuncSetAttribute(router_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     RouterTcShape<1>::kSmem));
        GT_CUDA(cudaFuncSetAttribute(router_tc_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     RouterTcShape<3>::kSmem));
        attr_set = true;
    }
    const int64_t tiles = ((T + kRBM - 1) / kRBM) * (E_pad / kRBN);
    const int grid = (int)(tiles < sms ? tiles : sms);
    if (split)
        router_tc_kernel<3><<<grid, kRThreads, RouterTcShape<3>::kSmem, st>>>(xmap, xmmap, xlmap, wmap, a);
    else
        router_tc_kernel<1><<<grid, kRThreads, RouterTcShape<1>::kSmem, st>>>(xmap, xmmap, xlmap, wmap, a);
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    return 0;
}

}  // namespace gtmoe
