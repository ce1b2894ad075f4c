// tc.cu -- grouped SwiGLU expert products on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), for Int8 and FP4 expert weights.
//
// Per expert (GatedFeedForward.Forward, feedforward/gatedfeedforward.go:49-57):
//   kernel 1 (GATED):  H = act_g(X Wg^T + bg) * act_u(X Wu^T + bu)  -> bf16
//   kernel 2 (DOWN):   Y = H Wd^T + bd                               -> bf16
// X / H rows of every expert are contiguous (the dispatch's expert-sorted
// buffer).  Tiles are 128 rows x 256 columns; for kernel 1 the 256 columns are
// 128 gate features and the same 128 up features, so each epilogue thread holds
// both operands of its SwiGLU products in registers.
//
// The Int8/FP4 weights stay compressed in HBM exactly as lowprecision.Rows
// stores them (codes row-major, one float32 scale per 16 values of a row,
// lowprecision/rows.go:38-79).  Dequantisation warps read them (L2-resident:
// every weight tile is reused by all m-tiles of its expert), multiply code by
// scale in float32 and round once to bf16 straight into the shared-memory
// operand in the UMMA canonical K-major SWIZZLE_128B layout (Rows.Row
// semantics, rows.go:87-119).  Activations arrive by TMA in the same layout.
// One elected thread issues tcgen05.mma kind::f16 (bf16 x bf16 -> f32 in
// TMEM); four epilogue warps read TMEM with tcgen05.ld.
//
// Persistent kernel, one CTA per SM, warp roles:
//   warp 0      TMA producer of the activation tile
//   warp 1      TMEM allocator and MMA issuer
//   warps 2-5   epilogue (TMEM -> bias, SwiGLU -> bf16 -> global)
//   warps 6-13  dequantisation of the weight tile
// 4-stage shared-memory ring (48 KB per stage), 2 TMEM accumulators of 256
// columns (the epilogue of one tile overlaps the main loop of the next).
//
// Every mbarrier wait is bounded (kWaitLimitNs of %globaltimer).  On expiry
// the kernel records an error code in *err, raises a CTA-wide abort flag so
// every role leaves its loop, lets in-flight copies land, frees TMEM and
// returns; the host reports GTMOE_ETIMEOUT.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include "handle.h"
#include "sm100.cuh"

namespace gtmoe {

namespace {

constexpr int kStages = 4;
constexpr int kBK = 64;                 // K elements per stage (128 bytes of bf16)
constexpr int kNumDequantWarps = 8;
constexpr int kDequantThreads = kNumDequantWarps * 32;
constexpr int kNumThreads = (6 + kNumDequantWarps) * 32;  // 448
constexpr int kTmemCols = 512;

// Tile shape: MH halves of 128 rows (one UMMA of M=128 each, sharing the
// weight tile) x BN columns; two accumulators of MH*BN columns fit TMEM.
template <int MH, int BN>
struct Shape {
    static_assert(MH * BN * 2 <= kTmemCols, "accumulators exceed TMEM");
    static constexpr int kBM = 128 * MH;
    static constexpr int kATileBytes = kBM * kBK * 2;
    static constexpr int kBTileBytes = BN * kBK * 2;
    static constexpr int kSmemBytes = kStages * (kATileBytes + kBTileBytes) + 1024 /*align*/ + 256 /*barriers*/;
    static constexpr int kItems = BN * 4 / kDequantThreads;  // (row, 16-value block) items per dequant thread
    // instruction descriptor: D f32, A bf16, B bf16, both K-major, N=BN, M=128
    static constexpr uint32_t kIdesc =
        (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
};

struct TcKernelArgs {
    const Group *groups;
    const int64_t *tile_prefix;
    const ExpertLayers *experts;
    int n_groups;
    int K;          // reduction length (d for GATED, h for DOWN)
    int n_out;      // output features (h for GATED, d for DOWN)
    int clamped;
    float clamp_limit;
    __nv_bfloat16 *out;  // hp (GATED) or yp (DOWN)
    int *err;
};

// Work unit u -> (group, n-tile, m-tile); m-tiles innermost so that
// neighbouring CTAs share one weight tile in L2.
struct Unit {
    int g;
    int nt;
    int64_t mt;
};
__device__ __forceinline__ Unit decode_unit(int64_t u, const int64_t *__restrict__ prefix, int n_groups, int n_tiles) {
    int lo = 0, hi = n_groups - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (__ldg(prefix + mid) * n_tiles <= u) lo = mid;
        else hi = mid - 1;
    }
    Unit w;
    w.g = lo;
    const int64_t mt_g = __ldg(prefix + lo + 1) - __ldg(prefix + lo);
    const int64_t r = u - __ldg(prefix + lo) * n_tiles;
    w.nt = (int)(r / mt_g);
    w.mt = r % mt_g;
    return w;
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

// Four Int8 codes -> two bf16x2 of bf16(code * scale): q + 128 becomes the
// low byte of the float 2^23 + q + 128, from which q is recovered exactly.
__device__ __forceinline__ void int8_decode4(uint32_t w, float s, uint32_t *o) {
    const uint32_t u = w ^ 0x80808080u;
    const float magic = 8388736.f;  // 2^23 + 128
    const float f0 = __uint_as_float(prmt(u, 0x4B000000u, 0x7650)) - magic;
    const float f1 = __uint_as_float(prmt(u, 0x4B000000u, 0x7651)) - magic;
    const float f2 = __uint_as_float(prmt(u, 0x4B000000u, 0x7652)) - magic;
    const float f3 = __uint_as_float(prmt(u, 0x4B000000u, 0x7653)) - magic;
    o[0] = pack_bf16(f0 * s, f1 * s);
    o[1] = pack_bf16(f2 * s, f3 * s);
}

// Raw compressed weights of one dequantisation step for one thread: kItems
// items of (row, 16-value block).
template <int NI>
struct Raw {
    uint4 c[NI];  // Int8: 16 codes; FP4: .x/.y hold 16 codes
    float s[NI];
};

template <int PREC, bool GATED, int BN, int NI>
__device__ __forceinline__ void load_raw(Raw<NI> &raw, const ExpertLayers &L, int n0, int kb, int K, int tid) {
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int item = tid + i * kDequantThreads;
        const int r = item >> 2;    // row of the B tile
        const int b = item & 3;     // 16-value block within the 64-wide k-step
        int which, row;
        if (GATED) {
            which = r < BN / 2 ? 0 : 1;
            row = n0 + (r & (BN / 2 - 1));
        } else {
            which = 2;
            row = n0 + r;
        }
        const int k = kb * kBK + b * 16;
        raw.s[i] = __ldg(L.s[which] + (int64_t)row * (K / 16) + (k >> 4));
        if (PREC == GTMOE_INT8) {
            raw.c[i] = __ldg((const uint4 *)((const int8_t *)L.w[which] + (int64_t)row * K + k));
        } else {
            const uint2 v = __ldg((const uint2 *)((const uint8_t *)L.w[which] + (int64_t)row * (K / 2) + (k >> 1)));
            raw.c[i] = make_uint4(v.x, v.y, 0, 0);
        }
    }
}

template <int PREC, int NI>
__device__ __forceinline__ void store_dequant(const Raw<NI> &raw, uint8_t *btile, int tid) {
#pragma unroll
    for (int i = 0; i < NI; i++) {
        const int item = tid + i * kDequantThreads;
        const int r = item >> 2;
        const int b = item & 3;
        uint32_t w[8];
        if (PREC == GTMOE_INT8) {
            int8_decode4(raw.c[i].x, raw.s[i], w);
            int8_decode4(raw.c[i].y, raw.s[i], w + 2);
            int8_decode4(raw.c[i].z, raw.s[i], w + 4);
            int8_decode4(raw.c[i].w, raw.s[i], w + 6);
        } else {
            const Fp4Tables t = fp4_tables(raw.s[i]);
            fp4_decode8(raw.c[i].x, t, w);
            fp4_decode8(raw.c[i].y, t, w + 4);
        }
        // 16 values = logical 16-byte chunks 2b, 2b+1 of row r, placed at
        // chunk ^ (r & 7) (SWIZZLE_128B)
        uint8_t *row = btile + r * 128;
        const int c0 = (2 * b) ^ (r & 7), c1 = (2 * b + 1) ^ (r & 7);
        *reinterpret_cast<uint4 *>(row + c0 * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4 *>(row + c1 * 16) = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

template <int PREC, bool GATED, int MH, int BN>
__global__ void __launch_bounds__(kNumThreads, 1)
    grouped_tc_kernel(const __grid_constant__ CUtensorMap amap, const TcKernelArgs a) {
    using Sh = Shape<MH, BN>;
    constexpr int kBM = Sh::kBM;
    constexpr int NI = Sh::kItems;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *a_tiles = smem;
    uint8_t *b_tiles = smem + kStages * Sh::kATileBytes;
    uint64_t *bars = (uint64_t *)(smem + kStages * (Sh::kATileBytes + Sh::kBTileBytes));
    uint64_t *full_a = bars;                        // [kStages]
    uint64_t *full_b = bars + kStages;              // [kStages]
    uint64_t *empty = bars + 2 * kStages;           // [kStages]
    uint64_t *tmem_full = bars + 3 * kStages;       // [2]
    uint64_t *tmem_empty = bars + 3 * kStages + 2;  // [2]
    uint32_t *tmem_slot = (uint32_t *)(bars + 3 * kStages + 4);
    volatile int *abort_flag = (volatile int *)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // GATED: BN/2 gate + the same BN/2 up features per tile
    const int n_tiles = GATED ? a.n_out / (BN / 2) : a.n_out / BN;
    const int64_t total = __ldg(a.tile_prefix + a.n_groups) * n_tiles;
    const int KB = a.K / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full_a[s], 1);
            mbar_init(&full_b[s], kNumDequantWarps);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 4);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer of the activation tiles
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&amap) : "memory");
            int stage = 0;
            uint32_t phase = 0;
            for (int64_t u = blockIdx.x; u < total && !*abort_flag; u += gridDim.x) {
                const Unit w = decode_unit(u, a.tile_prefix, a.n_groups, n_tiles);
                const Group grp = a.groups[w.g];
                const int row0 = (int)((GATED ? grp.x_row0 : grp.h_row0) + w.mt * kBM);
                for (int kb = 0; kb < KB; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, a.err, 1)) break;
                    mbar_arrive_expect_tx(&full_a[stage], Sh::kATileBytes);
                    tma_load_2d(a_tiles + stage * Sh::kATileBytes, &amap, kb * kBK, row0, &full_a[stage]);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (*abort_flag) {
                // let copies already issued land before the CTA can exit
                const uint64_t t0 = global_timer_ns();
                while (global_timer_ns() - t0 < 1000000ull) {
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int64_t u = blockIdx.x; u < total && !*abort_flag; u += gridDim.x) {
                int halves = MH;
                if (MH > 1) {
                    // skip the second half when it holds no row of the group
                    const Unit w = decode_unit(u, a.tile_prefix, a.n_groups, n_tiles);
                    const int64_t m_left = a.groups[w.g].m - w.mt * kBM;
                    halves = m_left > 128 ? MH : 1;
                }
                if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1, abort_flag, a.err, 2)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * MH * BN);
                bool ok = true;
                for (int kb = 0; kb < KB; kb++) {
                    if (!mbar_wait(&full_a[stage], phase, abort_flag, a.err, 3) ||
                        !mbar_wait(&full_b[stage], phase, abort_flag, a.err, 4)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = sw128_desc(smem_u32(a_tiles + stage * Sh::kATileBytes));
                    const uint64_t bdesc = sw128_desc(smem_u32(b_tiles + stage * Sh::kBTileBytes));
#pragma unroll
                    for (int k = 0; k < kBK / 16; k++) {
                        umma_bf16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), Sh::kIdesc,
                                  (kb | k) != 0);
                        if (MH > 1 && halves > 1)
                            umma_bf16(d_tmem + BN, adesc + (uint64_t)((128 * 128) >> 4) + (uint64_t)(2 * k),
                                      bdesc + (uint64_t)(2 * k), Sh::kIdesc, (kb | k) != 0);
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit(&tmem_full[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
        }
    } else if (warp < 6) {
        // ---------------- epilogue: TMEM -> registers -> global
        const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int64_t u = blockIdx.x; u < total && !*abort_flag; u += gridDim.x) {
            const Unit w = decode_unit(u, a.tile_prefix, a.n_groups, n_tiles);
            const Group grp = a.groups[w.g];
            const ExpertLayers L = a.experts[grp.expert];
            if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, a.err, 5)) break;
            tc_fence_after();
            const int64_t m_left = grp.m - w.mt * kBM;
#pragma unroll 1
            for (int hh = 0; hh < MH; hh++) {
                if (hh > 0 && m_left <= 128) break;  // the MMA skipped this half
                const int row_in_tile = hh * 128 + quad * 32 + lane;
                const bool valid = row_in_tile < m_left;
                const uint32_t t_row =
                    tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * MH * BN + hh * BN);
                __nv_bfloat16 *dst = a.out + (grp.h_row0 + w.mt * kBM + row_in_tile) * (int64_t)a.n_out;
                if (GATED) {
                    constexpr int HW = BN / 2;
                    const int f0 = w.nt * HW;
                    const float *bg = L.b32[0];
                    const float *bu = L.b32[1];
#pragma unroll 1
                    for (int c = 0; c < HW; c += 16) {
                        uint32_t g[16], up[16];
                        tmem_ld16(t_row + c, g);
                        tmem_ld16(t_row + HW + c, up);
                        tmem_ld_wait();
                        uint32_t o[8];
#pragma unroll
                        for (int j = 0; j < 16; j += 2) {
                            float hv[2];
#pragma unroll
                            for (int q = 0; q < 2; q++) {
                                float gv = __uint_as_float(g[j + q]) + (bg ? __ldg(bg + f0 + c + j + q) : 0.f);
                                float uv = __uint_as_float(up[j + q]) + (bu ? __ldg(bu + f0 + c + j + q) : 0.f);
                                hv[q] = gate_act<float>(gv, a.clamped, a.clamp_limit) *
                                        up_act<float>(uv, a.clamped, a.clamp_limit);
                            }
                            o[j / 2] = pack_bf16(hv[0], hv[1]);
                        }
                        if (valid) {
                            uint4 *p = reinterpret_cast<uint4 *>(dst + f0 + c);
                            p[0] = make_uint4(o[0], o[1], o[2], o[3]);
                            p[1] = make_uint4(o[4], o[5], o[6], o[7]);
                        }
                    }
                } else {
                    const int f0 = w.nt * BN;
                    const float *bd = L.b32[2];
#pragma unroll 1
                    for (int c = 0; c < BN; c += 16) {
                        uint32_t y[16];
                        tmem_ld16(t_row + c, y);
                        tmem_ld_wait();
                        uint32_t o[8];
#pragma unroll
                        for (int j = 0; j < 16; j += 2) {
                            float y0 = __uint_as_float(y[j]) + (bd ? __ldg(bd + f0 + c + j) : 0.f);
                            float y1 = __uint_as_float(y[j + 1]) + (bd ? __ldg(bd + f0 + c + j + 1) : 0.f);
                            o[j / 2] = pack_bf16(y0, y1);
                        }
                        if (valid) {
                            uint4 *p = reinterpret_cast<uint4 *>(dst + f0 + c);
                            p[0] = make_uint4(o[0], o[1], o[2], o[3]);
                            p[1] = make_uint4(o[4], o[5], o[6], o[7]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[acc]);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
    } else {
        // ---------------- dequantisation of the weight tiles
        const int tid = threadIdx.x - 6 * 32;
        int stage = 0;
        uint32_t phase = 0;
        int64_t u = blockIdx.x;
        int kb = 0;
        Raw<NI> cur, nxt;
        ExpertLayers L{};
        int n0 = 0;
        auto setup_unit = [&](int64_t uu, ExpertLayers &LL, int &nn0) {
            const Unit w = decode_unit(uu, a.tile_prefix, a.n_groups, n_tiles);
            const Group grp = a.groups[w.g];
            LL = a.experts[grp.expert];
            nn0 = GATED ? w.nt * (BN / 2) : w.nt * BN;
        };
        if (u < total) {
            setup_unit(u, L, n0);
            load_raw<PREC, GATED, BN, NI>(cur, L, n0, 0, a.K, tid);
        }
        while (u < total && !*abort_flag) {
            // prefetch the next step's raw weights
            int64_t un = u;
            int kbn = kb + 1;
            ExpertLayers Ln = L;
            int n0n = n0;
            if (kbn == KB) {
                kbn = 0;
                un = u + gridDim.x;
                if (un < total) setup_unit(un, Ln, n0n);
            }
            if (un < total) load_raw<PREC, GATED, BN, NI>(nxt, Ln, n0n, kbn, a.K, tid);
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, a.err, 6)) break;
            store_dequant<PREC, NI>(cur, b_tiles + stage * Sh::kBTileBytes, tid);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_b[stage]);
            if (++stage == kStages) {
                stage = 0;
                phase ^= 1;
            }
            u = un;
            kb = kbn;
            L = Ln;
            n0 = n0n;
            cur = nxt;
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols));
    }
}

int make_act_map(CUtensorMap *map, const void *base, int64_t rows, int K, int box_rows) {
    return encode_bf16_2d(map, base, K, rows, kBK, box_rows);
}

template <int PREC, bool GATED, int MH, int BN>
int launch_one(const CUtensorMap &map, const TcKernelArgs &ka, int sms, cudaStream_t st) {
    using Sh = Shape<MH, BN>;
    auto kern = grouped_tc_kernel<PREC, GATED, MH, BN>;
    static bool attr_set = false;
    if (!attr_set) {
        GT_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Sh::kSmemBytes));
        attr_set = true;
    }
    kern<<<sms, kNumThreads, Sh::kSmemBytes, st>>>(map, ka);
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    return 0;
}

template <int MH, int BN>
int launch_pair(gtmoe_handle *h, TcWeights &w, const TcArgs &ta, TcKernelArgs ka, cudaStream_t st) {
    const gtmoe_config &c = h->cfg;
    CUtensorMap xmap, hmap;
    GT_CHECK(make_act_map(&xmap, ta.xp, ta.rows_x, c.d_model, 128 * MH));
    GT_CHECK(make_act_map(&hmap, ta.hp, ta.rows_h, c.hidden, 128 * MH));
    const int prec = c.weight_precision;
    GT_CHECK(h->phase_begin(3));
    ka.K = c.d_model;
    ka.n_out = c.hidden;
    ka.out = (__nv_bfloat16 *)ta.hp;
    if (prec == GTMOE_INT8) GT_CHECK((launch_one<GTMOE_INT8, true, MH, BN>(xmap, ka, w.sms, st)));
    else GT_CHECK((launch_one<GTMOE_FP4, true, MH, BN>(xmap, ka, w.sms, st)));
    GT_CHECK(h->phase_end(3));

    GT_CHECK(h->phase_begin(4));
    ka.K = c.hidden;
    ka.n_out = c.d_model;
    ka.out = (__nv_bfloat16 *)ta.yp;
    if (prec == GTMOE_INT8) GT_CHECK((launch_one<GTMOE_INT8, false, MH, BN>(hmap, ka, w.sms, st)));
    else GT_CHECK((launch_one<GTMOE_FP4, false, MH, BN>(hmap, ka, w.sms, st)));
    GT_CHECK(h->phase_end(4));
    return 0;
}

}  // namespace

// Tile shapes: 256 rows x 128 columns (two M=128 UMMAs share each dequantised
// weight tile: half the dequantisation per MMA) by default; GTMOE_TC_SHAPE=
// 128x256 selects one M=128 x N=256 UMMA per k-slice.
static void choose_shape(TcWeights &w) {
    const char *e = getenv("GTMOE_TC_SHAPE");
    if (e && strcmp(e, "128x256") == 0) {
        w.mh = 1;
        w.bn = 256;
    } else {
        w.mh = 2;
        w.bn = 128;
    }
    w.bm = 128 * w.mh;
}

bool tc_supported(const gtmoe_handle *h, int64_t T) {
    const gtmoe_config &c = h->cfg;
    if (c.weight_precision != GTMOE_INT8 && c.weight_precision != GTMOE_FP4) return false;
    if (T <= 0) return false;
    if (getenv("GTMOE_DISABLE_TC")) return false;
    TcWeights w;
    choose_shape(w);
    // gate/up tiles hold bn/2 features of each; down tiles bn features; K in
    // steps of 64
    if (c.hidden % (w.bn / 2) != 0 || c.d_model % w.bn != 0) return false;
    if (c.d_model % kBK != 0 || c.hidden % kBK != 0) return false;
    return true;
}

int tc_prepare(gtmoe_handle *h, TcWeights &w) {
    if (!w.err) {
        GT_CUDA(cudaMalloc(&w.err, sizeof(int)));
        GT_CUDA(cudaMemset(w.err, 0, sizeof(int)));
    }
    int dev = 0;
    GT_CUDA(cudaGetDevice(&dev));
    GT_CUDA(cudaDeviceGetAttribute(&w.sms, cudaDevAttrMultiProcessorCount, dev));
    choose_shape(w);
    w.ready = 1;
    (void)h;
    return 0;
}

int tc_tile_rows(TcWeights &w) {
    choose_shape(w);
    return w.bm;
}

int launch_grouped_tc(gtmoe_handle *h, TcWeights &w, const TcArgs &ta, cudaStream_t st) {
    const gtmoe_config &c = h->cfg;
    TcKernelArgs ka;
    ka.groups = ta.groups;
    ka.tile_prefix = ta.tile_prefix;
    ka.experts = h->table.as<ExpertLayers>();
    ka.n_groups = ta.n_groups;
    ka.clamped = c.clamped;
    ka.clamp_limit = (float)c.clamp_limit;
    ka.err = w.err;
    if (w.mh == 1) return launch_pair<1, 256>(h, w, ta, ka, st);
    return launch_pair<2, 128>(h, w, ta, ka, st);
}

int tc_check_error(TcWeights &w) {
    if (!w.err) return 0;
    int v = 0;
    GT_CUDA(cudaMemcpy(&v, w.err, sizeof(int), cudaMemcpyDeviceToHost));
    if (v != 0) {
        cudaMemset(w.err, 0, sizeof(int));
        return fail(GTMOE_ETIMEOUT, "tensor-core expert kernel gave up waiting (barrier %d); results are invalid", v);
    }
    return 0;
}

void tc_release(TcWeights &w) {
    if (w.err) cudaFree(w.err);
    w.err = nullptr;
}

}  // namespace gtmoe
