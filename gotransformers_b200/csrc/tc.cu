// tc.cu -- grouped SwiGLU expert products on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), for Int8 and FP4 expert weights.
//
// Per expert (GatedFeedForward.Forward, feedforward/gatedfeedforward.go:49-57):
//   kernel 1 (GATED):  H = act_g(X Wg^T + bg) * act_u(X Wu^T + bu)  -> bf16
//   kernel 2 (DOWN):   Y = H Wd^T + bd                               -> bf16
// X / H rows of every expert are contiguous (the dispatch's expert-sorted
// buffer).
//
// The products are computed transposed, D = W X^T.  The dequantised weights
// are the MMA's A operand and go from the dequantisation warps' registers
// straight into tensor memory (tcgen05.st); the token rows are the B operand,
// staged in shared memory by TMA.  The bf16 weight tile therefore never
// passes through shared memory: writing it there and reading it back for the
// MMA was the shared-memory traffic that bounded the previous form of this
// kernel.  The Int8/FP4 weights stay compressed in HBM: the bytes of the
// lowprecision.Rows snapshot (codes, one float32 scale per 16 values of a
// row; lowprecision/rows.go:38-79) are only permuted at set time into
// 64-row records (dequant.cuh), and the dequantisation is Rows.Row's
// bf16(code * scale) (rows.go:87-119).
//
// A CTA pair (cluster of 2, tcgen05.mma.cta_group::2, M = 256, N = 192)
// computes 256 weight rows x 192 tokens: each CTA holds 128 weight rows in
// its TMEM lanes and 96 of the tokens in shared memory, and accumulates its
// 128 rows x 192 tokens in its own TMEM.  In kernel 1 a CTA's 128 weight rows
// are 64 gate features and the same 64 up features, so one pair tile yields
// 128 hidden features; in kernel 2 they are 128 consecutive output features.
// One pipeline step covers 128 inputs: 8 MMAs between one pair of barrier
// waits and one commit, which keeps the single issuing thread ahead of the
// tensor pipe.
//
// Persistent kernel, one CTA per SM, warp roles:
//   warp 0      TMA / bulk-copy producer (token tiles + raw weight records)
//   warp 1      TMEM allocator and MMA issuer
//   warps 2-5   epilogue (TMEM -> bias, SwiGLU -> bf16 -> shared-memory
//               transpose -> coalesced global rows)
//   warps 6-13  dequantisation, two groups of four (one per TMEM lane
//               quadrant) taking alternate steps
//   warps 14-17 expert parallel only (kernel 2): finished rows to their
//               tokens' ranks
// TMEM: two accumulators of 192 columns (the epilogue of one tile overlaps
// the main loop of the next) and a two-stage ring of 64-column A stages.
//
// Every mbarrier wait is bounded (kWaitLimitNs of %globaltimer).  On expiry
// the kernel records an error code in *err, raises a CTA-wide abort flag so
// every role leaves its loop, lets in-flight copies and MMAs finish, frees
// TMEM and returns; the host reports GTMOE_ETIMEOUT.
#include <stdlib.h>
#include <string.h>

#include "dequant.cuh"
#include "handle.h"
#include "sm100.cuh"

namespace gtmoe {


namespace {

constexpr int kBK = 64;                 // inputs per k-block (one raw record)
constexpr int kStepK = 128;             // inputs per pipeline step
constexpr int kStepKB = kStepK / kBK;   // k-blocks per step
constexpr int kCtaTok = 96;             // token rows per CTA (its half of B)
constexpr int kTileTok = 2 * kCtaTok;   // tokens per pair tile (UMMA N)
constexpr int kCtaW = 2 * kHalfRows;    // weight rows per CTA (TMEM lanes; UMMA M = 256 over the pair)
constexpr int kGatedFeat = 2 * kHalfRows;  // kernel 1: hidden features per pair tile
constexpr int kDownFeat = 2 * kCtaW;       // kernel 2: output features per pair tile
constexpr int kNumWriterWarps = 8;      // dequantisation: 2 groups x 4 lane quadrants
constexpr int kEpiWarps = 4;
constexpr int kNumThreads = (2 + kEpiWarps + kNumWriterWarps) * 32;  // 448
// Expert parallel: four more warps in the down kernel copy finished output
// rows to their tokens' ranks.
constexpr int kReturnWarps = 4;
constexpr int kMaxThreads = kNumThreads + kReturnWarps * 32;  // 576
constexpr int kTmemCols = 512;
constexpr int kAccCols = kTileTok;          // f32 accumulator columns
constexpr int kRingCol = 2 * kAccCols;      // first column of the A ring
constexpr int kAStageCols = kStepK / 2;     // bf16 pairs per lane per step
static_assert(kRingCol + 2 * kAStageCols <= kTmemCols, "tensor memory");
constexpr int kBSubBytes = kCtaTok * 128;   // one k-block of this CTA's tokens (SWIZZLE_128B rows)
constexpr int kBStageBytes = kStepKB * kBSubBytes;
static_assert(kBSubBytes % 1024 == 0, "swizzle atoms stay 1024-byte aligned");
constexpr int kEpiChunk = 32;               // tokens per epilogue round
// Epilogue staging, f32 [32 tokens][pitch]: kernel 1 the gate and the up
// values of the CTA's 64 features (pitch 68 each), kernel 2 its 128 output
// features (pitch 132).  Pitches of 4 mod 32 words keep both the column
// writes (lanes = features) and the row reads (lanes = tokens) free of bank
// conflicts.
constexpr int kGatePitch = 68;
constexpr int kDownPitch = 132;
constexpr int kEpiBytes = 2 * kEpiChunk * kGatePitch * 4;  // 17408
static_assert(kEpiChunk * kDownPitch * 4 <= kEpiBytes, "epilogue staging");
constexpr int kPrefixCache = 2048;          // m-tile prefix entries cached in shared memory
constexpr int kBandTiles = 16;              // m-tiles per band of the unit order (UnitDecoder)
// instruction descriptor: D f32, A bf16, B bf16, both K-major, N = 192, M = 256 (2-SM)
constexpr uint32_t kIdesc =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTileTok >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
static_assert(kTileTok % 16 == 0 && kTileTok <= 256, "UMMA N for M = 256");

// Raw record geometry and the shared-memory plan of one precision: a ring of
// token tiles (released when the step's MMAs complete) and a separate ring of
// raw weight records (released as soon as the dequantisation warps have
// decoded them, so that weight loads run further ahead).
constexpr int kBStages = 5;
template <int PREC>
struct Raw {
    static constexpr int kCodeBytes = PREC == GTMOE_INT8 ? 64 : 32;  // per row and k-block
    static constexpr int kHalfBytes = half_bytes(kCodeBytes);        // one (64-row, k-block) record
    static constexpr int kStageBytes = 2 * kStepKB * kHalfBytes;     // two halves x the step's k-blocks
    static constexpr int kStages = 4;
    static constexpr int kBarBytes = 256;
    static constexpr int kSmemBytes = 1024 + kBStages * kBStageBytes + kStages * kStageBytes + kEpiBytes +
                                      kBarBytes + kPrefixCache * 4;
};
static_assert(Raw<GTMOE_INT8>::kSmemBytes <= 232448, "shared memory per CTA");

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

// Half of the MMAs of one step (K = 128; half 0: inputs 0-63, half 1:
// 64-127): A columns a_tmem + 8k, B k-blocks at bdesc (inputs 0-63) and
// bdesc + kBSubBytes (64-127), 32 bytes of K per MMA (+2 in the descriptor's
// 16-byte address units).  Only the step's first MMA may start a fresh
// accumulation.
template <int HALF>
__device__ __forceinline__ void umma2_ts_half(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, bool accumulate) {
    constexpr uint64_t kSub = HALF ? (kBSubBytes >> 4) : 0;
    const uint32_t a0 = a_tmem + HALF * 32;
    asm volatile(
        "{\n\t.reg .pred p, t;\n\t"
        "setp.ne.b32 p, %10, 0;\n\t"
        "setp.eq.b32 t, 0, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %9, p;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%3], %4, %9, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%5], %6, %9, t;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%7], %8, %9, t;\n\t}\n" ::"r"(d_tmem),
        "r"(a0), "l"(bdesc + kSub), "r"(a0 + 8), "l"(bdesc + kSub + 2), "r"(a0 + 16), "l"(bdesc + kSub + 4),
        "r"(a0 + 24), "l"(bdesc + kSub + 6), "r"(kIdesc), "r"((uint32_t)(HALF || accumulate)));
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory"); }
// Barrier of the epilogue warps that also ANDs their verdicts, so that all
// of them take a tile (and its named barriers) or all of them stop.
__device__ __forceinline__ bool epi_vote(bool ok) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(r)
        : "r"((uint32_t)ok), "n"(kEpiWarps * 32)
        : "memory");
    return r != 0;
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

// Work unit u -> (group, n-tile, m-tile).  Within a group the m-tiles run
// in bands of kBandTiles: a band's units are n-tile major, m-tiles innermost,
// so the clusters working at one time share each weight tile and, for a
// large group (the shared expert sees every token), re-read each token tile
// for the next n-tiles from L2 instead of HBM.  A group of at most
// kBandTiles m-tiles is one band.  Each role walks its units in increasing
// order, so the group index only moves forward: the decoder keeps it and the
// group's record, and reads the m-tile prefix from shared memory.
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
        const int64_t full = mt_g / kBandTiles;  // complete bands
        const int64_t band_units = (int64_t)kBandTiles * n_tiles;
        w.g = g;
        if (r < full * band_units) {
            const int64_t q = r % band_units;
            w.nt = (int)(q / kBandTiles);
            w.mt = (r / band_units) * kBandTiles + q % kBandTiles;
        } else {
            const int64_t rest = mt_g - full * kBandTiles, q = r - full * band_units;
            w.nt = (int)(q / rest);
            w.mt = full * kBandTiles + q % rest;
        }
        return changed;
    }
};

// One weight row of one step (128 inputs = two k-block records of the row's
// half) -> 64 bf16 pairs in K order: the A columns of this lane.
template <int PREC>
__device__ __forceinline__ void dequant_row(const uint8_t *half_rec, int hr, uint32_t (&v)[64]) {
    using R = Raw<PREC>;
#pragma unroll
    for (int kb = 0; kb < kStepKB; kb++) {
        const uint8_t *rec = half_rec + kb * R::kHalfBytes;
        const float4 sc = *reinterpret_cast<const float4 *>(rec + half_scale_off(hr, R::kCodeBytes));
        const float s4[4] = {sc.x, sc.y, sc.z, sc.w};
        uint32_t *o = v + kb * 32;
        if (PREC == GTMOE_INT8) {
#pragma unroll
            for (int b = 0; b < 4; b++) {  // 16-byte group b = block b (16 codes)
                const uint4 c = *reinterpret_cast<const uint4 *>(rec + half_code_off(hr, 16 * b));
                int8_decode4(c.x, s4[b], o + 8 * b);
                int8_decode4(c.y, s4[b], o + 8 * b + 2);
                int8_decode4(c.z, s4[b], o + 8 * b + 4);
                int8_decode4(c.w, s4[b], o + 8 * b + 6);
            }
        } else {
#pragma unroll
            for (int gi = 0; gi < 2; gi++) {  // 16-byte group gi = blocks 2gi, 2gi+1
                const uint4 c = *reinterpret_cast<const uint4 *>(rec + half_code_off(hr, 16 * gi));
                const Fp4Tables t0 = fp4_tables(s4[2 * gi]);
                fp4_decode8(c.x, t0, o + 16 * gi);
                fp4_decode8(c.y, t0, o + 16 * gi + 4);
                const Fp4Tables t1 = fp4_tables(s4[2 * gi + 1]);
                fp4_decode8(c.z, t1, o + 16 * gi + 8);
                fp4_decode8(c.w, t1, o + 16 * gi + 12);
            }
        }
    }
}

// Grouped SwiGLU GEMM on a CTA pair; see the file comment for the roles.
// Rank 0 (the leader) issues the MMAs.
template <int PREC, bool GATED>
__global__ void __launch_bounds__(kMaxThreads, 1)
    grouped_tc_kernel(const __grid_constant__ CUtensorMap amap, const TcKernelArgs a) {
    using R = Raw<PREC>;
    constexpr int SB = kBStages, SR = R::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *b_tiles = smem;                               // [SB] this CTA's tokens, 2 SW128 k-blocks
    uint8_t *raw_tiles = b_tiles + SB * kBStageBytes;      // [SR] this CTA's raw weight records
    uint8_t *epi = raw_tiles + SR * R::kStageBytes;        // epilogue staging
    uint64_t *bars = (uint64_t *)(epi + kEpiBytes);
    // step j uses token stage j % SB, raw stage j % SR and A stage j & 1; its
    // MMAs wait for one barrier, full[j % SB] on the leader, which counts the
    // leader producer's arrival (with both CTAs' token bytes) and the eight
    // dequantisation warps of the pair that wrote the A stage
    uint64_t *full = bars;                            // [SB] step ready (leader)
    uint64_t *b_empty = bars + SB;                    // [SB] MMAs of the step done (both CTAs)
    uint64_t *full_raw = bars + 2 * SB;               // [SR] this CTA's raw weights landed
    uint64_t *raw_empty = bars + 2 * SB + SR;         // [SR] raw records decoded (this CTA)
    uint64_t *tmem_full = bars + 2 * SB + 2 * SR;     // [2] accumulator ready (both CTAs)
    uint64_t *tmem_empty = tmem_full + 2;             // [2] both epilogues done (leader)
    uint32_t *tmem_slot = (uint32_t *)(tmem_full + 4);
    volatile int *abort_flag = (volatile int *)(tmem_slot + 1);
    volatile int *tiles_out = (volatile int *)(tmem_slot + 2);  // epilogue warps' finished tiles (x4)
    int *prefix_s = (int *)((uint8_t *)bars + R::kBarBytes);
    static_assert((2 * SB + 2 * SR + 4) * 8 + 12 <= R::kBarBytes, "barrier area");

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
    const uint32_t peer_abort = mapa_shared(smem_u32((const void *)abort_flag), rank ^ 1u);
    const int n_tiles = GATED ? a.n_out / kGatedFeat : a.n_out / kDownFeat;
    const int64_t total = __ldg(a.tile_prefix + a.n_groups) * n_tiles;
    const int KB = a.K / kBK;
    const int KS = a.K / kStepK;
    for (int i = threadIdx.x; i <= a.n_groups; i += blockDim.x) prefix_s[i] = (int)__ldg(a.tile_prefix + i);

    if (threadIdx.x == 0) {
        for (int s = 0; s < SB; s++) {
            mbar_init(&full[s], 1 + 2 * 4);
            mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < SR; s++) {
            mbar_init(&full_raw[s], 1);
            mbar_init(&raw_empty[s], 4);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&tmem_full[b], 1);
            mbar_init(&tmem_empty[b], 2 * kEpiWarps);
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
        // ---------------- producer: token tiles (TMA, counted on the leader) + raw weight records (bulk)
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&amap) : "memory");
            int64_t j = 0;  // steps issued by this CTA
            UnitDecoder dec{prefix_s, a.groups, a.n_groups, n_tiles};
            const uint8_t *src0 = nullptr, *src1 = nullptr;
            for (int64_t u = cluster; u < total && !*abort_flag; u += n_clusters) {
                Unit w;
                if (dec.advance(u, w)) {
                    const ExpertLayers &L = a.experts[dec.grp.expert];
                    src0 = GATED ? L.tiled[0] : L.tiled[2];
                    src1 = GATED ? L.tiled[1] : L.tiled[2];
                }
                const Group &grp = dec.grp;
                const int row0 = (int)((GATED ? grp.x_row0 : grp.h_row0) + w.mt * kTileTok + rank * kCtaTok);
                // this CTA's two 64-row weight blocks: kernel 1 the gate and the up
                // block of its 64 features, kernel 2 two consecutive blocks
                const int64_t hb0 = GATED ? 2 * w.nt + rank : 4 * w.nt + 2 * rank;
                const int64_t hb1 = GATED ? hb0 : hb0 + 1;
                const uint8_t *p0 = src0 + hb0 * KB * R::kHalfBytes;
                const uint8_t *p1 = src1 + hb1 * KB * R::kHalfBytes;
                for (int s = 0; s < KS; s++, j++) {
                    // raw weights first: the dequantisation needs them two steps before the MMAs
                    const int sr = (int)(j % SR), sb = (int)(j % SB);
                    if (!pair_wait<false>(&raw_empty[sr], ((uint32_t)(j / SR) & 1) ^ 1, abort_flag, peer_abort, a.err,
                                          1))
                        break;
                    uint8_t *rs = raw_tiles + sr * R::kStageBytes;
                    const int64_t off = (int64_t)s * kStepKB * R::kHalfBytes;
                    mbar_arrive_expect_tx(&full_raw[sr], R::kStageBytes);
                    bulk_load(rs, p0 + off, kStepKB * R::kHalfBytes, &full_raw[sr]);
                    bulk_load(rs + kStepKB * R::kHalfBytes, p1 + off, kStepKB * R::kHalfBytes, &full_raw[sr]);
                    if (!pair_wait<false>(&b_empty[sb], ((uint32_t)(j / SB) & 1) ^ 1, abort_flag, peer_abort, a.err,
                                          1))
                        break;
                    if (leader) mbar_arrive_expect_tx(&full[sb], 2 * kBStageBytes);
                    uint8_t *bt = b_tiles + sb * kBStageBytes;
#pragma unroll
                    for (int i = 0; i < kStepKB; i++)
                        tma_load_2d_pair(bt + i * kBSubBytes, &amap, (s * kStepKB + i) * kBK, row0,
                                         mapa_shared(smem_u32(&full[sb]), 0));
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
            uint32_t j = 0;  // steps issued (A ring stage j & 1, use j >> 1; token stage j % SB)
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int64_t u = cluster; u < total && !*abort_flag; u += n_clusters) {
                if (!pair_wait<false>(&tmem_empty[acc], acc_phase ^ 1, abort_flag, peer_abort, a.err, 2)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kAccCols);
                bool ok = true;
                bool seen = false;  // this step's barrier was already seen complete by the probe below
                for (int s = 0; s < KS; s++, j++) {
                    const int sb = (int)(j % SB);
                    if (!seen && !pair_wait<false>(&full[sb], (j / SB) & 1, abort_flag, peer_abort, a.err, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_tmem = tmem_base + (uint32_t)(kRingCol + (j & 1) * kAStageCols);
                    const uint64_t bdesc = sw128_desc(smem_u32(b_tiles + sb * kBStageBytes));
                    umma2_ts_half<0>(d_tmem, a_tmem, bdesc, s != 0);
                    // probe the next step's barrier between the two halves, so that its
                    // latency overlaps the MMA issue (that phase cannot complete twice
                    // before the next step's MMAs are issued)
                    seen = s + 1 < KS && mbar_try_wait(&full[(j + 1) % SB], ((j + 1) / SB) & 1);
                    umma2_ts_half<1>(d_tmem, a_tmem, bdesc, true);
                    umma2_commit_mc(&b_empty[sb], 0x3);
                }
                if (!ok) break;
                umma2_commit_mc(&tmem_full[acc], 0x3);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
            if (*abort_flag) {
                // let MMAs already issued finish before TMEM is freed
                const uint64_t t0 = global_timer_ns();
                while (global_timer_ns() - t0 < 1000000ull) {
                }
            }
        }
    } else if (warp < 2 + kEpiWarps) {
        // ---------------- epilogue: TMEM -> registers -> shared memory -> global rows (both CTAs)
        // Per 32-token chunk every warp first parks its lanes' bias-added
        // values in shared memory (lanes = features); after a barrier the
        // four warps take 32 tokens each (lanes = tokens), do the activation
        // work evenly and write 16-byte pieces of the output rows.
        const int quad = warp & 3;         // TMEM lanes 32*quad .. 32*quad+31
        const int ew = warp - 2;           // 0..3: this warp's feature slice in the second phase
        const uint32_t tmem_empty_leader0 = mapa_shared(smem_u32(&tmem_empty[0]), 0);
        float *stage_f = reinterpret_cast<float *>(epi);
        int acc = 0;
        uint32_t acc_phase = 0;
        UnitDecoder dec{prefix_s, a.groups, a.n_groups, n_tiles};
        const float *b0 = nullptr, *b1 = nullptr;
        // (no abort test in the loop condition: the vote below is the one place
        // where the four warps decide together to stop)
        for (int64_t u = cluster; u < total; u += n_clusters) {
            Unit w;
            if (dec.advance(u, w)) {
                const ExpertLayers &L = a.experts[dec.grp.expert];
                b0 = GATED ? L.b32[0] : L.b32[2];
                b1 = L.b32[1];
            }
            const Group &grp = dec.grp;
            const bool ready = pair_wait<false>(&tmem_full[acc], acc_phase, abort_flag, peer_abort, a.err, 5);
            if (!epi_vote(ready)) break;
            tc_fence_after();
            const int64_t left = grp.m - w.mt * kTileTok;
            const int n_valid = left < kTileTok ? (int)left : kTileTok;
            const int n_chunks = (n_valid + kEpiChunk - 1) / kEpiChunk;
            const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * kAccCols);
            const int64_t row0 = grp.h_row0 + w.mt * kTileTok;
            if (GATED) {
                // TMEM lanes 0-63 gate, 64-127 up of the CTA's 64 features
                const int f0 = w.nt * kGatedFeat + (int)rank * kHalfRows;
                const int fl = (quad & 1) * 32 + lane;
                const float *bp = quad < 2 ? b0 : b1;
                const float bias = bp ? __ldg(bp + f0 + fl) : 0.f;
                float *col = stage_f + (quad < 2 ? 0 : kEpiChunk * kGatePitch) + fl;
                const float *gate_row = stage_f + lane * kGatePitch + ew * 16;
                const float *up_row = gate_row + kEpiChunk * kGatePitch;
                __nv_bfloat16 *dst = a.out + (row0 + lane) * (int64_t)a.n_out + f0 + ew * 16;
#pragma unroll 1
                for (int c = 0; c < n_chunks; c++) {
                    uint32_t v[32];
                    tmem_ld16(t_row + c * kEpiChunk, *reinterpret_cast<uint32_t(*)[16]>(v));
                    tmem_ld16(t_row + c * kEpiChunk + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < kEpiChunk; i++) col[i * kGatePitch] = __uint_as_float(v[i]) + bias;
                    epi_bar();
                    if (c * kEpiChunk + lane < n_valid) {
                        uint32_t o[8];
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            const float4 gv = *reinterpret_cast<const float4 *>(gate_row + 4 * q);
                            const float4 uv = *reinterpret_cast<const float4 *>(up_row + 4 * q);
                            const float h0 = gate_act<float>(gv.x, a.clamped, a.clamp_limit) *
                                             up_act<float>(uv.x, a.clamped, a.clamp_limit);
                            const float h1 = gate_act<float>(gv.y, a.clamped, a.clamp_limit) *
                                             up_act<float>(uv.y, a.clamped, a.clamp_limit);
                            const float h2 = gate_act<float>(gv.z, a.clamped, a.clamp_limit) *
                                             up_act<float>(uv.z, a.clamped, a.clamp_limit);
                            const float h3 = gate_act<float>(gv.w, a.clamped, a.clamp_limit) *
                                             up_act<float>(uv.w, a.clamped, a.clamp_limit);
                            o[2 * q] = pack_bf16(h0, h1);
                            o[2 * q + 1] = pack_bf16(h2, h3);
                        }
                        uint4 *p = reinterpret_cast<uint4 *>(dst + (int64_t)(c * kEpiChunk) * a.n_out);
                        p[0] = make_uint4(o[0], o[1], o[2], o[3]);
                        p[1] = make_uint4(o[4], o[5], o[6], o[7]);
                    }
                    epi_bar();
                }
            } else {
                const int f0 = w.nt * kDownFeat + (int)rank * kCtaW;
                const int fl = quad * 32 + lane;
                const float bias = b0 ? __ldg(b0 + f0 + fl) : 0.f;
                float *col = stage_f + fl;
                const float *row = stage_f + lane * kDownPitch + ew * 32;
                __nv_bfloat16 *dst = a.out + (row0 + lane) * (int64_t)a.n_out + f0 + ew * 32;
#pragma unroll 1
                for (int c = 0; c < n_chunks; c++) {
                    uint32_t v[32];
                    tmem_ld16(t_row + c * kEpiChunk, *reinterpret_cast<uint32_t(*)[16]>(v));
                    tmem_ld16(t_row + c * kEpiChunk + 16, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < kEpiChunk; i++) col[i * kDownPitch] = __uint_as_float(v[i]) + bias;
                    epi_bar();
                    if (c * kEpiChunk + lane < n_valid) {
                        uint4 *p = reinterpret_cast<uint4 *>(dst + (int64_t)(c * kEpiChunk) * a.n_out);
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            const float4 y0 = *reinterpret_cast<const float4 *>(row + 8 * q);
                            const float4 y1 = *reinterpret_cast<const float4 *>(row + 8 * q + 4);
                            p[q] = make_uint4(pack_bf16(y0.x, y0.y), pack_bf16(y0.z, y0.w), pack_bf16(y1.x, y1.y),
                                              pack_bf16(y1.z, y1.w));
                        }
                    }
                    epi_bar();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(tmem_empty_leader0 + (uint32_t)(acc * sizeof(uint64_t)));
            if (!GATED && a.ret_ranks > 0) {
                // the tile's rows are in global memory: hand them to the return warps
                __threadfence_block();
                __syncwarp();
                if (lane == 0) atomicAdd((int *)tiles_out, 1);
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
    } else if (warp >= 2 + kEpiWarps + kNumWriterWarps) {
        // ---------------- expert parallel (down kernel): finished output rows
        // of routed experts to their tokens' ranks, one tile behind the epilogue
        const int rw = warp - (2 + kEpiWarps + kNumWriterWarps);
        UnitDecoder dec{prefix_s, a.groups, a.n_groups, n_tiles};
        int done = 0;
        for (int64_t u = cluster; u < total && !*abort_flag; u += n_clusters) {
            Unit w;
            dec.advance(u, w);
            const Group &grp = dec.grp;
            done += kEpiWarps;
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
            // this CTA's 128 output features of the tile: 256 bytes per token row
            const int f0 = w.nt * kDownFeat + (int)rank * kCtaW;
            const int64_t row_base = grp.h_row0 + w.mt * kTileTok;
            const int64_t left = grp.m - w.mt * kTileTok;
            const int n_valid = left < kTileTok ? (int)left : kTileTok;
            const int per = kTileTok / kReturnWarps;
            const int r0 = rw * per;
            const int r1 = min(n_valid, r0 + per);
            const int sg = lane & 15;
            for (int r = r0; r < r1; r += 8) {
                uint4 v[4];
                uint4 *dst[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int rr = r + 2 * q + (lane >> 4);
                    const int64_t out_row = row_base + rr;
                    dst[q] = nullptr;
                    if (rr < r1 && out_row >= a.ret_row0) {
                        const int64_t route = __ldg(a.ret_route + (out_row - a.ret_row0));
                        dst[q] = reinterpret_cast<uint4 *>((__nv_bfloat16 *)a.ret_peers[route >> 48] +
                                                           (route & 0xFFFFFFFFFFFFll) * (int64_t)a.n_out + f0) +
                                 sg;
                        v[q] = __ldcg(reinterpret_cast<const uint4 *>(a.out + out_row * (int64_t)a.n_out + f0) + sg);
                    }
                }
#pragma unroll
                for (int q = 0; q < 4; q++)
                    if (dst[q]) *dst[q] = v[q];
            }
        }
        __threadfence_system();  // rows on other GPUs visible before the arrival below
    } else {
        // ---------------- dequantisation: group g fills the A stage g of steps g, g+2, ...
        const int g = (warp - (2 + kEpiWarps)) >> 2;
        const int quad = warp & 3;              // TMEM lanes 32*quad .. 32*quad+31
        const int lr = quad * 32 + lane;        // this lane's weight row in the CTA
        const int half = lr / kHalfRows, hr = lr % kHalfRows;
        const uint32_t full_leader0 = mapa_shared(smem_u32(&full[0]), 0);
        const uint32_t t_dst = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(kRingCol + g * kAStageCols);
        const int64_t units = cluster < total ? (total - cluster + n_clusters - 1) / n_clusters : 0;
        const int64_t steps = units * KS;  // steps this CTA runs
        // every decision to stop is taken by the whole warp (__all_sync): the
        // tensor-memory stores below are warp-collective
        for (int64_t j = g; j < steps; j += 2) {
            const int sr = (int)(j % SR);
            bool ok = pair_wait<false>(&full_raw[sr], (uint32_t)(j / SR) & 1, abort_flag, peer_abort, a.err, 6);
            if (!__all_sync(0xffffffffu, ok)) break;
            uint32_t v[64];
            dequant_row<PREC>(raw_tiles + sr * R::kStageBytes + half * kStepKB * R::kHalfBytes, hr, v);
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[sr]);
            // the A stage is free once the MMAs of step j - 2 are done (this
            // group's previous wait saw step j - 4's, so the parity is not stale)
            if (j >= 2) {
                ok = pair_wait<false>(&b_empty[(j - 2) % SB], (uint32_t)((j - 2) / SB) & 1, abort_flag, peer_abort,
                                      a.err, 7);
                if (!__all_sync(0xffffffffu, ok)) break;
            }
            tc_fence_after();
#pragma unroll
            for (int i = 0; i < 4; i++) tmem_st16(t_dst + 16 * i, v + 16 * i);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(full_leader0 + (uint32_t)((j % SB) * sizeof(uint64_t)));
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

// Re-lays one Int8/FP4 layer (rows x K, reference snapshot layout) into the
// records of dequant.cuh: record (row / 64) * KB + kb holds the row's codes
// of k-block kb column-group major and its four block scales.  One thread
// per (row, k-block).
__global__ void relayout_kernel(const uint8_t *__restrict__ codes, const float *__restrict__ scales, int rows, int K,
                                int code_bytes, uint8_t *__restrict__ out) {
    const int KB = K / kBK;
    const int64_t item = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (item >= (int64_t)rows * KB) return;
    const int row = (int)(item / KB), kb = (int)(item % KB);
    const int hr = row % kHalfRows;
    uint8_t *rec = out + ((int64_t)(row / kHalfRows) * KB + kb) * half_bytes(code_bytes);
    const int64_t src_row = (int64_t)row * KB * code_bytes + (int64_t)kb * code_bytes;
    // Int8 codes biased to q + 128
    const uint32_t bias = code_bytes == 64 ? 0x80808080u : 0u;
    for (int i = 0; i < code_bytes; i += 16) {
        uint4 c = *reinterpret_cast<const uint4 *>(codes + src_row + i);
        c.x ^= bias;
        c.y ^= bias;
        c.z ^= bias;
        c.w ^= bias;
        *reinterpret_cast<uint4 *>(rec + half_code_off(hr, i)) = c;
    }
    const float4 s = *reinterpret_cast<const float4 *>(scales + (int64_t)row * (K / 16) + kb * 4);
    *reinterpret_cast<float4 *>(rec + half_scale_off(hr, code_bytes)) = s;
}

// The inverse of relayout_kernel: a record back to the row's codes (Int8
// bias removed) and its four block scales in the RowsSnapshot layout.
__global__ void unrelayout_kernel(const uint8_t *__restrict__ tiled, int rows, int K, int code_bytes,
                                  uint8_t *__restrict__ codes, float *__restrict__ scales) {
    const int KB = K / kBK;
    const int64_t item = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (item >= (int64_t)rows * KB) return;
    const int row = (int)(item / KB), kb = (int)(item % KB);
    const int hr = row % kHalfRows;
    const uint8_t *rec = tiled + ((int64_t)(row / kHalfRows) * KB + kb) * half_bytes(code_bytes);
    const int64_t dst_row = (int64_t)row * KB * code_bytes + (int64_t)kb * code_bytes;
    const uint32_t bias = code_bytes == 64 ? 0x80808080u : 0u;
    for (int i = 0; i < code_bytes; i += 16) {
        uint4 c = *reinterpret_cast<const uint4 *>(rec + half_code_off(hr, i));
        c.x ^= bias;
        c.y ^= bias;
        c.z ^= bias;
        c.w ^= bias;
        *reinterpret_cast<uint4 *>(codes + dst_row + i) = c;
    }
    *reinterpret_cast<float4 *>(scales + (int64_t)row * (K / 16) + kb * 4) =
        *reinterpret_cast<const float4 *>(rec + half_scale_off(hr, code_bytes));
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
    // kernel 1 tiles 128 hidden features, kernel 2 256 output features; K in
    // steps of 128; the group prefix fits the shared-memory cache
    return c.hidden % kGatedFeat == 0 && c.d_model % kDownFeat == 0 && c.d_model % kStepK == 0 &&
           c.hidden % kStepK == 0 && c.n_shared + c.n_routed + 1 <= kPrefixCache;
}

}  // namespace

bool tc_supported(const gtmoe_handle *h, int64_t T) {
    const gtmoe_config &c = h->cfg;
    if (c.weight_precision != GTMOE_INT8 && c.weight_precision != GTMOE_FP4) return false;
    if (T <= 0) return false;
    if (h->no_tc) return false;
    return shapes_ok(c);
}

int tc_relayout_layer(gtmoe_handle *h, LayerDev &L, int which) {
    const gtmoe_config &c = h->cfg;
    L.tiled.release();
    if (c.weight_precision != GTMOE_INT8 && c.weight_precision != GTMOE_FP4) return 0;
    if (!shapes_ok(c)) return 0;
    const int code_bytes = c.weight_precision == GTMOE_INT8 ? 64 : 32;
    (void)which;
    if (L.rows % kHalfRows != 0 || L.width % kBK != 0) return fail(GTMOE_EINVAL, "layer shape does not tile");
    const int64_t items = (int64_t)L.rows * (L.width / kBK);
    GT_CHECK(L.tiled.ensure((size_t)items * (code_bytes + 16)));
    relayout_kernel<<<(unsigned)((items + 255) / 256), 256, 0, h->stream>>>(
        (const uint8_t *)L.w.p, L.s.as<float>(), L.rows, L.width, code_bytes, L.tiled.as<uint8_t>());
    GT_CUDA(cudaGetLastError());
    return 0;
}

int tc_restore_raw(gtmoe_handle *h, LayerDev &L) {
    if (!L.raw_dropped) return 0;
    const int code_bytes = L.precision == GTMOE_INT8 ? 64 : 32;
    const int64_t items = (int64_t)L.rows * (L.width / kBK);
    GT_CHECK(L.w.ensure((size_t)L.rows * (L.width / kBK) * code_bytes));
    GT_CHECK(L.s.ensure(sizeof(float) * (size_t)L.rows * (L.width / 16)));
    unrelayout_kernel<<<(unsigned)((items + 255) / 256), 256, 0, h->stream>>>(
        L.tiled.as<uint8_t>(), L.rows, L.width, code_bytes, L.w.as<uint8_t>(), L.s.as<float>());
    GT_CUDA(cudaGetLastError());
    L.raw_dropped = 0;
    h->table_dirty = 1;
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

int tc_tile_rows(TcWeights &) { return kTileTok; }

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
    GT_CHECK(encode_bf16_2d(&xmap, ta.xp, c.d_model, ta.rows_x, kBK, kCtaTok));
    GT_CHECK(encode_bf16_2d(&hmap, ta.hp, c.hidden, ta.rows_h, kBK, kCtaTok));
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
