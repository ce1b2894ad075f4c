// tc.cu -- grouped SwiGLU expert products on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), for Int8 and FP4 expert weights.
//
// Per expert (GatedFeedForward.Forward, feedforward/gatedfeedforward.go:49-57):
//   kernel 1 (GATED):  H = act_g(X Wg^T + bg) * act_u(X Wu^T + bu)  -> bf16
//   kernel 2 (DOWN):   Y = H Wd^T + bd                               -> bf16
// X / H rows of every expert are contiguous (the dispatch's expert-sorted
// buffer).  A tile is 256 rows x 128 columns computed by two M=128 UMMAs that
// share one weight tile, so every dequantised weight feeds 256 rows of MMA
// work.  For kernel 1 the 128 columns are 64 gate features and the same 64
// up features, so each epilogue thread holds both operands of its SwiGLU
// products in registers.
//
// The Int8/FP4 weights stay compressed in HBM: the bytes of the
// lowprecision.Rows snapshot (codes, one float32 scale per 16 values of a
// row; lowprecision/rows.go:38-79) are only permuted at set time into chunks
// of (row tile, 64-wide k-block), codes then scales, so that one bulk async
// copy moves the raw weights of one pipeline stage into shared memory.
// Dequantisation warps turn them into bf16(code * scale) (Rows.Row semantics,
// rows.go:87-119) straight in the UMMA canonical K-major SWIZZLE_128B layout;
// activations arrive by TMA in the same layout.  One elected thread issues
// tcgen05.mma kind::f16 (bf16 x bf16 -> f32 in TMEM); four epilogue warps read
// TMEM with tcgen05.ld.
//
// Persistent kernel, one CTA per SM, warp roles:
//   warp 0      TMA / bulk-copy producer (activation tile + raw weight chunks)
//   warp 1      TMEM allocator and MMA issuer
//   warps 2-5   epilogue (TMEM -> bias, SwiGLU -> bf16 -> global)
//   warps 6-13  dequantisation of the weight tile
// A ring of shared-memory stages (activations 32 KB, bf16 weights 16 KB, raw
// weights 6 KB FP4 / 10 KB Int8 each) and two TMEM accumulators of 256
// columns (the epilogue of one tile overlaps the main loop of the next).
//
// Every mbarrier wait is bounded (kWaitLimitNs of %globaltimer).  On expiry
// the kernel records an error code in *err, raises a CTA-wide abort flag so
// every role leaves its loop, lets in-flight copies land, frees TMEM and
// returns; the host reports GTMOE_ETIMEOUT.
#include <stdlib.h>
#include <string.h>

#include "dequant.cuh"
#include "handle.h"
#include "sm100.cuh"

namespace gtmoe {


namespace {

constexpr int kBK = 64;              // K elements per stage (128 bytes of bf16)
constexpr int kCtaRows = 128;        // token rows per CTA (UMMA M=256 over the pair)
constexpr int kTileM = 2 * kCtaRows; // rows per cluster tile
constexpr int kTileN = 256;          // B rows (output columns) per cluster tile, 128 per CTA
constexpr int kChunkRows = 128;      // weight rows per raw chunk = one CTA's half of B
static_assert(kChunkRows == 2 * kChunkHalfRows, "a chunk is two halves");
constexpr int kNumDequantWarps = 8;
constexpr int kDequantThreads = kNumDequantWarps * 32;
constexpr int kNumThreads = (6 + kNumDequantWarps) * 32;  // 448
// Expert parallel: two more warps in the down kernel copy finished output
// rows to their tokens' ranks (coalesced 512-byte row segments).
constexpr int kReturnWarps = 4;
constexpr int kMaxThreads = kNumThreads + kReturnWarps * 32;
constexpr int kTmemCols = 512;
constexpr int kATileBytes = kCtaRows * kBK * 2;    // 16 KB per CTA
constexpr int kBTileBytes = kChunkRows * kBK * 2;  // 16 KB per CTA
constexpr int kItems = kChunkRows * 4 / kDequantThreads;  // (row, 16-value block) items per dequant thread
constexpr int kPrefixCache = 2048;  // m-tile prefix entries cached in shared memory
// instruction descriptor: D f32, A bf16, B bf16, both K-major, N=256, M=256 (2-SM)
constexpr uint32_t kIdesc =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTileN >> 3) << 17) | ((uint32_t)(kTileM >> 4) << 24);

// Raw chunk geometry: code bytes per row per k-block, stage bytes.
template <int PREC>
struct Raw {
    static constexpr int kCodeBytes = PREC == GTMOE_INT8 ? 64 : 32;
    static constexpr int kRowBytes = kCodeBytes + 16;  // codes + 4 float scales
    static constexpr int kStageBytes = kChunkRows * kRowBytes;
    static constexpr int kStages = 5;
    static constexpr int kSmemBytes =
        kStages * (kATileBytes + kBTileBytes + kStageBytes) + 1024 + 256 + kPrefixCache * 4;
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
    // expert-parallel return of the down kernel (TcArgs)
    int ret_ranks;
    int64_t ret_row0;
    const int64_t *ret_route;
    unsigned char *const *ret_peers;
    unsigned long long *const *ret_sigs;
    unsigned int *ret_done;
};

__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Bounded wait of the 2-SM kernel: on expiry it records `code`, raises the
// abort flag of this CTA and of its peer, and returns false.
template <bool CLUSTER_ACQUIRE>
__device__ __forceinline__ bool pair_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                          uint32_t peer_abort, int *err, int code) {
    auto probe = [&]() { return CLUSTER_ACQUIRE ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity); };
    if (probe()) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        for (int i = 0; i < 32; i++)
            if (probe()) return true;
        if (*abort_flag) return false;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicCAS(err, 0, code);
            *abort_flag = 1;
            asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1) : "memory");
            return false;
        }
    }
}

// Work unit u -> (group, n-tile, m-tile); m-tiles innermost so that
// neighbouring clusters share one weight tile in L2.  Each role walks its
// units in increasing order, so the group index only moves forward: the
// decoder keeps it and the group's record, and reads the m-tile prefix from
// shared memory.
struct Unit {
    int g;
    int nt;
    int64_t mt;
};
struct UnitDecoder {
    const int *prefix;  // shared-memory copy (n_groups + 1 entries)
    const Group *groups;
    int n_groups, n_tiles;
    int g = -1;
    Group grp;
    __device__ __forceinline__ bool advance(int64_t u, Unit &w) {
        bool changed = false;
        if (g < 0) {
            g = 0;
            changed = true;
        }
        while (g + 1 < n_groups && (int64_t)prefix[g + 1] * n_tiles <= u) {
            g++;
            changed = true;
        }
        if (changed) grp = groups[g];
        const int64_t mt_g = prefix[g + 1] - prefix[g];
        const int64_t r = u - (int64_t)prefix[g] * n_tiles;
        w.g = g;
        w.nt = (int)(r / mt_g);
        w.mt = r % mt_g;
        return changed;
    }
};

// Dequantises one stage of this CTA's 128 B rows: item (r, b) = 16 values of
// row r, k-block quarter b.  The raw stage is one chunk (two 64-row halves of
// codes then scales, chunk_code_off / chunk_scale_off).
template <int PREC>
__device__ __forceinline__ void dequant_stage(const uint8_t *raw, uint8_t *btile, int tid) {
    using R = Raw<PREC>;
#pragma unroll
    for (int i = 0; i < kItems; i++) {
        const int item = tid + i * kDequantThreads;
        const int r = item >> 2;
        const int b = item & 3;
        const float s = *reinterpret_cast<const float *>(raw + chunk_scale_off(r, R::kCodeBytes) + b * 4);
        uint32_t w[8];
        if (PREC == GTMOE_INT8) {
            const uint4 c = *reinterpret_cast<const uint4 *>(raw + chunk_code_off(r, R::kCodeBytes) + b * 16);
            int8_decode4(c.x, s, w);
            int8_decode4(c.y, s, w + 2);
            int8_decode4(c.z, s, w + 4);
            int8_decode4(c.w, s, w + 6);
        } else {
            const uint2 c = *reinterpret_cast<const uint2 *>(raw + chunk_code_off(r, R::kCodeBytes) + b * 8);
            const Fp4Tables t = fp4_tables(s);
            fp4_decode8(c.x, t, w);
            fp4_decode8(c.y, t, w + 4);
        }
        // 16 values = logical 16-byte chunks 2b, 2b+1 of row r, placed at
        // chunk ^ (r & 7) (SWIZZLE_128B)
        uint8_t *row = btile + r * 128;
        const int c0 = (2 * b) ^ (r & 7), c1 = (2 * b + 1) ^ (r & 7);
        *reinterpret_cast<uint4 *>(row + c0 * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4 *>(row + c1 * 16) = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// Grouped SwiGLU GEMM on a CTA pair (cluster of 2, tcgen05.mma.cta_group::2):
// the pair computes a 256-row x 256-column tile, CTA rank r holding A rows
// r*128..r*128+127 and B rows r*128..r*128+127 in its own shared memory and
// D rows r*128.. in its own TMEM.  For kernel 1 the pair's B rows are 128
// gate features (rank 0) and the same 128 up features (rank 1), so D columns
// 0..127 / 128..255 of each TMEM lane are the gate / up values of one
// (token, feature).  Rank 0 (the leader) issues the MMAs.
template <int PREC, bool GATED>
__global__ void __launch_bounds__(kMaxThreads, 1)
    grouped_tc_kernel(const __grid_constant__ CUtensorMap amap, const TcKernelArgs a) {
    using R = Raw<PREC>;
    constexpr int S = R::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *a_tiles = smem;
    uint8_t *b_tiles = smem + S * kATileBytes;
    uint8_t *raw_tiles = b_tiles + S * kBTileBytes;
    uint64_t *bars = (uint64_t *)(raw_tiles + S * R::kStageBytes);
    uint64_t *full_a = bars;                  // [S] both activation tiles landed (leader)
    uint64_t *full_raw = bars + S;            // [S] this CTA's raw weights landed
    uint64_t *full_b = bars + 2 * S;          // [S] both bf16 weight halves written (leader)
    uint64_t *empty = bars + 3 * S;           // [S] MMAs of the stage done (both CTAs)
    uint64_t *tmem_full = bars + 4 * S;       // [2] accumulator ready (both CTAs)
    uint64_t *tmem_empty = bars + 4 * S + 2;  // [2] both epilogues done (leader)
    uint32_t *tmem_slot = (uint32_t *)(bars + 4 * S + 4);
    volatile int *abort_flag = (volatile int *)(tmem_slot + 1);
    volatile int *tiles_out = (volatile int *)(tmem_slot + 2);  // epilogue warps' finished tiles (x4)
    int *prefix_s = (int *)(smem + S * (kATileBytes + kBTileBytes + R::kStageBytes) + 256);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
    const uint32_t peer_abort = mapa_shared(smem_u32((const void *)abort_flag), rank ^ 1u);
    // kernel 1: 128 gate + the same 128 up features per tile; kernel 2: 256 features
    const int n_tiles = GATED ? a.n_out / kChunkRows : a.n_out / kTileN;
    const int64_t total = __ldg(a.tile_prefix + a.n_groups) * n_tiles;
    const int KB = a.K / kBK;
    for (int i = threadIdx.x; i <= a.n_groups; i += blockDim.x) prefix_s[i] = (int)__ldg(a.tile_prefix + i);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full_a[s], 1);
            mbar_init(&full_raw[s], 1);
            mbar_init(&full_b[s], 2 * kNumDequantWarps);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 2 * 4);
        }
        *abort_flag = 0;
        *tiles_out = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer's barriers are initialised before any remote operation
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- producer: activation tile (TMA, counted on the leader) + raw weight chunk (bulk)
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&amap) : "memory");
            int stage = 0;
            uint32_t phase = 0;
            constexpr uint32_t chunk_bytes = R::kStageBytes;
            UnitDecoder dec{prefix_s, a.groups, a.n_groups, n_tiles};
            const uint8_t *src = nullptr;
            for (int64_t u = cluster; u < total && !*abort_flag; u += n_clusters) {
                Unit w;
                if (dec.advance(u, w)) {
                    const ExpertLayers &L = a.experts[dec.grp.expert];
                    src = GATED ? L.tiled[rank] : L.tiled[2];
                }
                const Group &grp = dec.grp;
                const int row0 = (int)((GATED ? grp.x_row0 : grp.h_row0) + w.mt * kTileM + rank * kCtaRows);
                // chunk (t, k-block) of a layer sits at (t * KB + kb) * chunk_bytes
                const int64_t chunk = GATED ? w.nt : 2 * w.nt + rank;
                for (int kb = 0; kb < KB; kb++) {
                    if (!pair_wait<false>(&empty[stage], phase ^ 1, abort_flag, peer_abort, a.err, 1)) break;
                    if (leader) mbar_arrive_expect_tx(&full_a[stage], 2 * kATileBytes);
                    tma_load_2d_pair(a_tiles + stage * kATileBytes, &amap, kb * kBK, row0,
                                     mapa_shared(smem_u32(&full_a[stage]), 0));
                    mbar_arrive_expect_tx(&full_raw[stage], chunk_bytes);
                    bulk_load(raw_tiles + stage * R::kStageBytes, src + ((size_t)chunk * KB + kb) * chunk_bytes,
                              chunk_bytes, &full_raw[stage]);
                    if (++stage == S) {
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
        // ---------------- MMA issuer (leader CTA)
        if (leader && lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int64_t u = cluster; u < total && !*abort_flag; u += n_clusters) {
                if (!pair_wait<false>(&tmem_empty[acc], acc_phase ^ 1, abort_flag, peer_abort, a.err, 2)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kTileN);
                bool ok = true;
                for (int kb = 0; kb < KB; kb++) {
                    if (!pair_wait<false>(&full_a[stage], phase, abort_flag, peer_abort, a.err, 3) ||
                        !pair_wait<false>(&full_b[stage], phase, abort_flag, peer_abort, a.err, 4)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = sw128_desc(smem_u32(a_tiles + stage * kATileBytes));
                    const uint64_t bdesc = sw128_desc(smem_u32(b_tiles + stage * kBTileBytes));
#pragma unroll
                    for (int k = 0; k < kBK / 16; k++)
                        umma2_bf16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), kIdesc,
                                   (kb | k) != 0);
                    umma2_commit_mc(&empty[stage], 0x3);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                umma2_commit_mc(&tmem_full[acc], 0x3);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
        }
    } else if (warp < 6) {
        // ---------------- epilogue: TMEM -> registers -> global (both CTAs)
        const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
        const uint32_t tmem_empty_leader0 = mapa_shared(smem_u32(&tmem_empty[0]), 0);
        int acc = 0;
        uint32_t acc_phase = 0;
        UnitDecoder dec{prefix_s, a.groups, a.n_groups, n_tiles};
        const float *b0 = nullptr, *b1 = nullptr;
        for (int64_t u = cluster; u < total && !*abort_flag; u += n_clusters) {
            Unit w;
            if (dec.advance(u, w)) {
                const ExpertLayers &L = a.experts[dec.grp.expert];
                b0 = GATED ? L.b32[0] : L.b32[2];
                b1 = L.b32[1];
            }
            const Group &grp = dec.grp;
            if (!pair_wait<false>(&tmem_full[acc], acc_phase, abort_flag, peer_abort, a.err, 5)) break;
            tc_fence_after();
            const int row_in_tile = (int)rank * kCtaRows + quad * 32 + lane;
            const bool valid = row_in_tile < grp.m - w.mt * kTileM;
            const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * kTileN);
            __nv_bfloat16 *dst = a.out + (grp.h_row0 + w.mt * kTileM + row_in_tile) * (int64_t)a.n_out;
            if (GATED) {
                const int f0 = w.nt * kChunkRows;
                const float *bg = b0;
                const float *bu = b1;
#pragma unroll 1
                for (int c = 0; c < kChunkRows; c += 16) {
                    uint32_t g[16], up[16];
                    tmem_ld16(t_row + c, g);
                    tmem_ld16(t_row + kChunkRows + c, up);
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
                const int f0 = w.nt * kTileN;
                const float *bd = b0;
#pragma unroll 1
                for (int c = 0; c < kTileN; c += 16) {
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
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(tmem_empty_leader0 + (uint32_t)(acc * sizeof(uint64_t)));
            if (!GATED && a.ret_ranks > 0 && lane == 0) {
                // the tile's rows are in global memory: hand them to the return warps
                __threadfence_block();
                atomicAdd((int *)tiles_out, 1);
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
    } else if (warp >= 6 + kNumDequantWarps) {
        // ---------------- expert parallel (down kernel): finished output rows
        // of routed experts to their tokens' ranks, one tile behind the epilogue
        const int rw = warp - (6 + kNumDequantWarps);
        UnitDecoder dec{prefix_s, a.groups, a.n_groups, n_tiles};
        int done = 0;
        for (int64_t u = cluster; u < total && !*abort_flag; u += n_clusters) {
            Unit w;
            dec.advance(u, w);
            const Group &grp = dec.grp;
            done += 4;
            if (*tiles_out < done) {
                const uint64_t t0 = global_timer_ns();
                bool ok = true;
                while (*tiles_out < done) {
                    if (*abort_flag) {
                        ok = false;
                        break;
                    }
                    if (global_timer_ns() - t0 > kWaitLimitNs) {
                        atomicCAS(a.err, 0, 8);
                        *abort_flag = 1;
                        asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1) : "memory");
                        ok = false;
                        break;
                    }
                }
                if (!ok) break;
            }
            __threadfence_block();
            const int f0 = w.nt * kTileN;  // this tile's 256 output features: 512 bytes per row
            const int64_t row_base = grp.h_row0 + w.mt * kTileM + (int64_t)rank * kCtaRows;
            const int64_t left = grp.m - w.mt * kTileM - (int64_t)rank * kCtaRows;
            const int n_valid = left < kCtaRows ? (int)left : kCtaRows;
            const int r0 = rw * (kCtaRows / kReturnWarps);
            const int r1 = min(n_valid, r0 + kCtaRows / kReturnWarps);
            for (int r = r0; r < r1; r += 8) {
                uint4 v[8];
                uint4 *dst[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int64_t out_row = row_base + r + j;
                    dst[j] = nullptr;
                    if (r + j < r1 && out_row >= a.ret_row0) {
                        const int64_t route = __ldg(a.ret_route + (out_row - a.ret_row0));
                        dst[j] = reinterpret_cast<uint4 *>((__nv_bfloat16 *)a.ret_peers[route >> 48] +
                                                           (route & 0xFFFFFFFFFFFFll) * (int64_t)a.n_out + f0) +
                                 lane;
                        v[j] = __ldcg(reinterpret_cast<const uint4 *>(a.out + out_row * (int64_t)a.n_out + f0) + lane);
                    }
                }
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (dst[j]) *dst[j] = v[j];
            }
        }
        __threadfence_system();  // rows on other GPUs visible before the arrival below
    } else {
        // ---------------- dequantisation of this CTA's half of the weight tile
        const int tid = threadIdx.x - 6 * 32;
        const uint32_t full_b_leader0 = mapa_shared(smem_u32(&full_b[0]), 0);
        int stage = 0;
        uint32_t phase = 0;
        const int64_t units = cluster < total ? (total - cluster + n_clusters - 1) / n_clusters : 0;
        const int64_t steps = units * KB;  // stages this CTA runs
        for (int64_t j = 0; j < steps && !*abort_flag; j++) {
            if (!pair_wait<false>(&full_raw[stage], phase, abort_flag, peer_abort, a.err, 6)) break;
            dequant_stage<PREC>(raw_tiles + stage * R::kStageBytes, b_tiles + stage * kBTileBytes, tid);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(full_b_leader0 + (uint32_t)(stage * sizeof(uint64_t)));
            if (++stage == S) {
                stage = 0;
                phase ^= 1;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while its peer may still signal it
    tc_fence_after();
    if (warp == 1) {
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols));
    }
    // expert parallel: the last CTA to finish tells every rank that this
    // rank's output rows have landed (an aborted CTA never counts, so the
    // other ranks' waits run out instead of reading partial rows)
    if (!GATED && a.ret_ranks > 0 && threadIdx.x == 0 && !*abort_flag) {
        const unsigned int done = atomicAdd(a.ret_done, 1u);
        if (done == gridDim.x - 1) {
            *a.ret_done = 0;
            __threadfence_system();
            for (int q = 0; q < a.ret_ranks; q++) atomicAdd_system(a.ret_sigs[q], 1ull);
        }
    }
}

// Re-lays one Int8/FP4 layer (rows x K, reference snapshot layout) into
// chunks of (chunk_rows rows, 64-wide k-block), each two 64-row halves of
// codes [64][code bytes] then scales [64][4].  One thread per (row, k-block).
__global__ void relayout_kernel(const uint8_t *__restrict__ codes, const float *__restrict__ scales, int rows, int K,
                                int code_bytes, int chunk_rows, uint8_t *__restrict__ out) {
    const int KB = K / kBK;
    const int64_t item = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (item >= (int64_t)rows * KB) return;
    const int row = (int)(item / KB), kb = (int)(item % KB);
    const int nt = row / chunk_rows, lr = row % chunk_rows;
    const int row_bytes = code_bytes + 16;
    uint8_t *chunk = out + ((int64_t)nt * KB + kb) * chunk_rows * row_bytes;
    const int64_t src_row = (int64_t)row * KB * code_bytes + (int64_t)kb * code_bytes;
    // Int8 codes biased to q + 128 (see chunk_code_off)
    const uint32_t bias = code_bytes == 64 ? 0x80808080u : 0u;
    for (int i = 0; i < code_bytes; i += 16) {
        uint4 c = *reinterpret_cast<const uint4 *>(codes + src_row + i);
        c.x ^= bias;
        c.y ^= bias;
        c.z ^= bias;
        c.w ^= bias;
        *reinterpret_cast<uint4 *>(chunk + chunk_code_off(lr, code_bytes) + i) = c;
    }
    const float4 s = *reinterpret_cast<const float4 *>(scales + (int64_t)row * (K / 16) + kb * 4);
    *reinterpret_cast<float4 *>(chunk + chunk_scale_off(lr, code_bytes)) = s;
}

template <int PREC, bool GATED>
int launch_one(const CUtensorMap &map, const TcKernelArgs &ka, int sms, cudaStream_t st) {
    const int threads = (!GATED && ka.ret_ranks > 0) ? kMaxThreads : kNumThreads;
    auto kern = grouped_tc_kernel<PREC, GATED>;
    static int grid = 0;
    if (!grid) {
        GT_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Raw<PREC>::kSmemBytes));
        // one CTA pair per two SMs, as many pairs as can be resident at once
        cudaLaunchConfig_t q = {};
        q.gridDim = dim3(2 * ((sms + 1) / 2));
        q.blockDim = dim3(kMaxThreads);
        q.dynamicSmemBytes = Raw<PREC>::kSmemBytes;
        cudaLaunchAttribute qa;
        qa.id = cudaLaunchAttributeClusterDimension;
        qa.val.clusterDim.x = 2;
        qa.val.clusterDim.y = 1;
        qa.val.clusterDim.z = 1;
        q.attrs = &qa;
        q.numAttrs = 1;
        int clusters = 0;
        GT_CUDA(cudaOccupancyMaxActiveClusters(&clusters, kern, &q));
        if (clusters < 1) return fail(GTMOE_ECUDA, "no CTA pair of the tensor-core kernel fits on this device");
        grid = 2 * (clusters < sms / 2 ? clusters : sms / 2);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = Raw<PREC>::kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    GT_CUDA(cudaLaunchKernelEx(&cfg, kern, map, ka));
    note_launches(1);
    return 0;
}

bool shapes_ok(const gtmoe_config &c) {
    // gate/up tiles hold 128 features of each, down tiles 256; K in steps of
    // 64; the group prefix fits the shared-memory cache
    return c.hidden % kChunkRows == 0 && c.d_model % kTileN == 0 && c.d_model % kBK == 0 && c.hidden % kBK == 0 &&
           c.n_shared + c.n_routed + 1 <= kPrefixCache;
}

}  // namespace

bool tc_supported(const gtmoe_handle *h, int64_t T) {
    const gtmoe_config &c = h->cfg;
    if (c.weight_precision != GTMOE_INT8 && c.weight_precision != GTMOE_FP4) return false;
    if (T <= 0) return false;
    if (getenv("GTMOE_DISABLE_TC")) return false;
    return shapes_ok(c);
}

int tc_relayout_layer(gtmoe_handle *h, LayerDev &L, int which) {
    const gtmoe_config &c = h->cfg;
    L.tiled.release();
    if (c.weight_precision != GTMOE_INT8 && c.weight_precision != GTMOE_FP4) return 0;
    if (!shapes_ok(c)) return 0;
    const int code_bytes = c.weight_precision == GTMOE_INT8 ? 64 : 32;
    const int chunk_rows = kChunkRows;
    (void)which;
    const int64_t items = (int64_t)L.rows * (L.width / kBK);
    GT_CHECK(L.tiled.ensure((size_t)items * (code_bytes + 16)));
    relayout_kernel<<<(unsigned)((items + 255) / 256), 256, 0, h->stream>>>(
        (const uint8_t *)L.w.p, L.s.as<float>(), L.rows, L.width, code_bytes, chunk_rows, L.tiled.as<uint8_t>());
    GT_CUDA(cudaGetLastError());
    return 0;
}

int tc_prepare(gtmoe_handle *h, TcWeights &w) {
    if (!w.err) {
        GT_CUDA(cudaMalloc(&w.err, sizeof(int)));
        GT_CUDA(cudaMemset(w.err, 0, sizeof(int)));
    }
    int dev = 0;
    GT_CUDA(cudaGetDevice(&dev));
    GT_CUDA(cudaDeviceGetAttribute(&w.sms, cudaDevAttrMultiProcessorCount, dev));
    w.ready = 1;
    (void)h;
    return 0;
}

int tc_tile_rows(TcWeights &) { return kTileM; }

int launch_grouped_tc(gtmoe_handle *h, TcWeights &w, const TcArgs &ta, cudaStream_t st) {
    const gtmoe_config &c = h->cfg;
    TcKernelArgs ka;
    ka.groups = ta.groups;
    ka.tile_prefix = ta.tile_prefix;
    ka.experts = h->table.as<ExpertLayers>();
    ka.n_groups = ta.n_groups;
    ka.ret_ranks = 0;
    ka.ret_row0 = 0;
    ka.ret_route = nullptr;
    ka.ret_peers = nullptr;
    ka.ret_sigs = nullptr;
    ka.ret_done = nullptr;
    ka.clamped = c.clamped;
    ka.clamp_limit = (float)c.clamp_limit;
    ka.err = w.err;
    CUtensorMap xmap, hmap;
    GT_CHECK(encode_bf16_2d(&xmap, ta.xp, c.d_model, ta.rows_x, kBK, kCtaRows));
    GT_CHECK(encode_bf16_2d(&hmap, ta.hp, c.hidden, ta.rows_h, kBK, kCtaRows));
    const int prec = c.weight_precision;

    GT_CHECK(h->phase_begin(3));
    ka.K = c.d_model;
    ka.n_out = c.hidden;
    ka.out = (__nv_bfloat16 *)ta.hp;
    if (prec == GTMOE_INT8) GT_CHECK((launch_one<GTMOE_INT8, true>(xmap, ka, w.sms, st)));
    else GT_CHECK((launch_one<GTMOE_FP4, true>(xmap, ka, w.sms, st)));
    GT_CHECK(h->phase_end(3));

    GT_CHECK(h->phase_begin(4));
    ka.K = c.hidden;
    ka.n_out = c.d_model;
    ka.out = (__nv_bfloat16 *)ta.yp;
    ka.ret_ranks = ta.ret_ranks;
    ka.ret_row0 = ta.ret_row0;
    ka.ret_route = ta.ret_route;
    ka.ret_peers = ta.ret_peers;
    ka.ret_sigs = ta.ret_sigs;
    ka.ret_done = ta.ret_done;
    if (prec == GTMOE_INT8) GT_CHECK((launch_one<GTMOE_INT8, false>(hmap, ka, w.sms, st)));
    else GT_CHECK((launch_one<GTMOE_FP4, false>(hmap, ka, w.sms, st)));
    GT_CHECK(h->phase_end(4));
    return 0;
}

int tc_check_error(TcWeights &w) {
    if (!w.err) return 0;
    int v = 0;
    GT_CUDA(cudaMemcpy(&v, w.err, sizeof(int), cudaMemcpyDeviceToHost));
    if (v != 0) {
        cudaMemset(w.err, 0, sizeof(int));
        return fail(GTMOE_ETIMEOUT, "tensor-core kernel gave up waiting (barrier %d); results are invalid", v);
    }
    return 0;
}


void tc_release(TcWeights &w) {
    if (w.err) cudaFree(w.err);
    w.err = nullptr;
}

}  // namespace gtmoe
