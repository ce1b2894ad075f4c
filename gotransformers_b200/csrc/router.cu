// router.cu -- router logits, sqrt-softplus affinities, top-k selection and
// gates (mixtureofexperts.go:80-82, :98-112, :154-172), and hash routing
// (:88-96, :142-152).
//
// Selection must reproduce the reference's float64 choice exactly.  The
// logits are first computed either here from float32 operands (float32
// products summed per 16-element block, block sums accumulated in float64;
// error below eps_t = 32 * 2^-24 * ||x_t|| * max_e ||w_e||, Cauchy-Schwarz
// bounding sum |x_i w_i|) or, for bf16 activations, on the tensor cores
// (router_tc.cu; eps_t = 70 * 2^-23 * ||x_t|| * max_e ||w_e||).  As
// |d affinity / d logit| < 0.5, a score moves by less than 0.5 * eps_t.  If
// the gap between the k-th and the (k+1)-th score exceeds 2 * 0.5 * eps_t the
// chosen set is the reference's;
// otherwise the warp recomputes that token's logits in float64 in the
// reference's summation order, with separately rounded multiplies and adds
// (one sequential sum per expert, as vectormath.DotProduct, vector.go:67-74),
// and selects again.
#include <cuda_bf16.h>

#include "common.cuh"
#include "internal.h"
#include "dispatch_small.cuh"

namespace gtmoe {

constexpr int kRouterTile = 64;
constexpr int kRouterK = 16;

template <int XDT>
__device__ __forceinline__ float load_x_f32(const void *x, int64_t i) {
    if (XDT == GTMOE_DTYPE_F64) return (float)((const double *)x)[i];
    if (XDT == GTMOE_DTYPE_F32) return ((const float *)x)[i];
    return __bfloat162float(((const __nv_bfloat16 *)x)[i]);
}

// logits[t, e] = sum_i x[t, i] * w[e, i]   (no bias; added in float64 later)
template <int XDT>
__global__ void __launch_bounds__(256) router_logits_kernel(const void *__restrict__ x, const float *__restrict__ w,
                                                            int64_t T, int E, int d, double *__restrict__ logits) {
    __shared__ float xs[kRouterK][kRouterTile + 4];
    __shared__ float ws[kRouterK][kRouterTile + 4];
    const int64_t t0 = (int64_t)blockIdx.x * kRouterTile;
    const int e0 = blockIdx.y * kRouterTile;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    double acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0;

    // each thread's share of a 16-input chunk, the next chunk's loaded into
    // registers while this one is multiplied (the loop is otherwise bound by
    // one global-load latency per chunk)
    constexpr int kPer = kRouterTile * kRouterK / 256;
    float rx[kPer], rw[kPer];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int j = 0; j < kPer; j++) {
            const int i = threadIdx.x + 256 * j;
            const int r = i / kRouterK, c = i % kRouterK;
            const int64_t t = t0 + r;
            const int kk = k0 + c;
            rx[j] = (t < T && kk < d) ? load_x_f32<XDT>(x, t * d + kk) : 0.f;
            const int e = e0 + r;
            rw[j] = (e < E && kk < d) ? w[(int64_t)e * d + kk] : 0.f;
        }
    };
    fetch(0);
    for (int k0 = 0; k0 < d; k0 += kRouterK) {
#pragma unroll
        for (int j = 0; j < kPer; j++) {
            const int i = threadIdx.x + 256 * j;
            xs[i % kRouterK][i / kRouterK] = rx[j];
            ws[i % kRouterK][i / kRouterK] = rw[j];
        }
        __syncthreads();
        if (k0 + kRouterK < d) fetch(k0 + kRouterK);
        float part[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) part[i][j] = 0.f;
#pragma unroll
        for (int c = 0; c < kRouterK; c++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = xs[c][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; j++) b[j] = ws[c][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) part[i][j] = fmaf(a[i], b[j], part[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] += (double)part[i][j];
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        int64_t t = t0 + ty * 4 + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int e = e0 + tx * 4 + j;
            if (e < E) logits[t * E + e] = acc[i][j];
        }
    }
}

// Few tokens (decode-shaped batches): one warp per (token, expert) instead of
// 64 x 64 tiles, so that the whole GPU works on a handful of tokens.  The
// arithmetic is router_logits_kernel's, operation for operation: float32
// sums of each 16-input block by sequential fmaf from zero, then the blocks
// added in float64 in input order -- both kernels give the same bits.
constexpr int kRouterSmallWarps = 8;

// The warp stages 512-input chunks of the token row and the expert's weight
// row in shared memory (element j at j + j/16, so that lane l reading block
// l's 16 values hits 32 different banks); lane l then forms block l's sum,
// and the warp adds the chunk's 32 block sums in order.  A chunk's 32 loads
// per lane are issued together into registers, and the next chunk's while
// the current one is summed, so a row costs about one memory latency rather
// than one per load.  Warp 0 of the first expert block also sums the
// token's squares in float64 (||x_t|| for the selection's error margin;
// squares of float32/bf16 values are exact, float64 rows as loaded), which
// spares the selection kernel a second pass over the row.
constexpr int kSmallChunk = 512;
constexpr int kSmallPitch = kSmallChunk + kSmallChunk / kRouterK;  // 544
constexpr int kSmallPer = kSmallChunk / 32;                       // loads per lane and chunk

template <int XDT>
__global__ void __launch_bounds__(kRouterSmallWarps * 32)
    router_logits_small_kernel(const void *__restrict__ x, const float *__restrict__ w, int64_t T, int E, int d,
                               double *__restrict__ logits, double *__restrict__ xnorm) {
    __shared__ float xs[kRouterSmallWarps][kSmallPitch];
    __shared__ float ws[kRouterSmallWarps][kSmallPitch];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * kRouterSmallWarps + warp;
    const int64_t t = blockIdx.y;
    if (e >= E) return;
    const bool norm_warp = xnorm && blockIdx.x == 0 && warp == 0;
    const float *we = w + (int64_t)e * d;
    float *xw = xs[warp], *ww = ws[warp];
    float rx[kSmallPer], rw[kSmallPer];
    double sq = 0.0;
    auto fetch = [&](int c0) {
#pragma unroll
        for (int i = 0; i < kSmallPer; i++) {
            const int kk = c0 + 32 * i + lane;
            if (XDT == GTMOE_DTYPE_F64) {
                const double v = kk < d ? ((const double *)x)[t * d + kk] : 0.0;
                rx[i] = (float)v;
                if (norm_warp) sq += v * v;
            } else {
                rx[i] = kk < d ? load_x_f32<XDT>(x, t * d + kk) : 0.f;
                if (norm_warp) sq += (double)rx[i] * (double)rx[i];
            }
            rw[i] = kk < d ? __ldg(we + kk) : 0.f;
        }
    };
    double acc = 0.0;
    fetch(0);
    for (int c0 = 0; c0 < d; c0 += kSmallChunk) {
#pragma unroll
        for (int i = 0; i < kSmallPer; i++) {
            const int j = 32 * i + lane;
            xw[j + j / kRouterK] = rx[i];
            ww[j + j / kRouterK] = rw[i];
        }
        __syncwarp();
        if (c0 + kSmallChunk < d) fetch(c0 + kSmallChunk);
        float p = 0.f;  // block (c0 / 16 + lane): inputs past d are zero products
#pragma unroll
        for (int c = 0; c < kRouterK; c++) p = fmaf(xw[lane * (kRouterK + 1) + c], ww[lane * (kRouterK + 1) + c], p);
        const int nblk = min(32, (d - c0 + kRouterK - 1) / kRouterK);  // blocks of this chunk inside d
        for (int b = 0; b < nblk; b++) acc += (double)__shfl_sync(0xffffffffu, p, b);
        __syncwarp();
    }
    if (lane == 0) logits[t * E + e] = acc;
    if (norm_warp) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
        if (lane == 0) xnorm[t] = sqrt(sq);
    }
}

// activationfunction/moreactivationfunctions.go:8-16, mixtureofexperts.go:80-82
__device__ __forceinline__ double affinity_d(double logit) {
    double sp;
    if (logit > 20) sp = logit;
    else if (logit < -20) sp = exp(logit);
    else sp = log1p(exp(logit));
    return sqrt(sp);
}

// Picks `count` experts by descending score among those not masked, ties to
// the lower index (the first k of sort.SliceStable, mixtureofexperts.go:106-109).
template <int MAXJ>
__device__ __forceinline__ void warp_top(const double (&score)[MAXJ], const double (&aff)[MAXJ], uint32_t masked,
                                         int E, int count, int *pick, double *pick_score, double *pick_aff) {
    const int lane = threadIdx.x & 31;
    uint32_t taken = masked;
    for (int i = 0; i < count; i++) {
        double best = 0;
        int best_e = 0x7fffffff;
        double best_a = 0;
#pragma unroll
        for (int j = 0; j < MAXJ; j++) {
            int e = lane + 32 * j;
            if (e >= E || (taken >> j) & 1u) continue;
            if (best_e == 0x7fffffff || score[j] > best) {
                best = score[j];
                best_e = e;
                best_a = aff[j];
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            double ob = __shfl_xor_sync(0xffffffffu, best, off);
            int oe = __shfl_xor_sync(0xffffffffu, best_e, off);
            double oa = __shfl_xor_sync(0xffffffffu, best_a, off);
            bool better = oe != 0x7fffffff && (best_e == 0x7fffffff || ob > best || (ob == best && oe < best_e));
            if (better) {
                best = ob;
                best_e = oe;
                best_a = oa;
            }
        }
        pick[i] = best_e;
        pick_score[i] = best;
        pick_aff[i] = best_a;
        if (best_e != 0x7fffffff && (best_e & 31) == lane) taken |= 1u << (best_e >> 5);
    }
}

template <int XDT, int MAXJ>
__device__ __forceinline__ void load_scores(const double *__restrict__ logits, const double *__restrict__ bias,
                                            const double *__restrict__ balance, int64_t t, int E, double (&score)[MAXJ],
                                            double (&aff)[MAXJ]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < MAXJ; j++) {
        int e = lane + 32 * j;
        score[j] = 0;
        aff[j] = 0;
        if (e < E) {
            double l = logits[t * E + e] + bias[e];  // perceptron/layer.go:150-153
            aff[j] = affinity_d(l);
            score[j] = aff[j] + balance[e];  // mixtureofexperts.go:103-105
        }
    }
}

// ||x_t|| for the error margin.  bf16 rows (16-byte aligned, d a multiple of
// 8) are read 16 bytes per lane with four loads in flight; other rows by
// element, unrolled by four.  Squares of bf16/float32 values are exact in
// float64; only the sum rounds (far below the margin's slack).
template <int XDT>
__device__ __forceinline__ double warp_x_norm(const void *__restrict__ x, int64_t t, int d) {
    const int lane = threadIdx.x & 31;
    double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    if (XDT == GTMOE_DTYPE_BF16 && (d & 7) == 0 && (((uintptr_t)x) & 15) == 0) {
        const uint4 *row = reinterpret_cast<const uint4 *>((const __nv_bfloat16 *)x + t * d);
        const int nv = d >> 3;
        auto sq8 = [](const uint4 v) {
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
            double a = 0;
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const double lo = (double)__uint_as_float(w[q] << 16), hi = (double)__uint_as_float(w[q] & 0xFFFF0000u);
                a += lo * lo + hi * hi;
            }
            return a;
        };
        int i = lane;
        for (; i + 96 < nv; i += 128) {
            const uint4 v0 = __ldg(row + i), v1 = __ldg(row + i + 32), v2 = __ldg(row + i + 64), v3 = __ldg(row + i + 96);
            s0 += sq8(v0);
            s1 += sq8(v1);
            s2 += sq8(v2);
            s3 += sq8(v3);
        }
        for (; i < nv; i += 32) s0 += sq8(__ldg(row + i));
    } else {
        int i = lane;
        for (; i + 96 < d; i += 128) {
            const double v0 = load_as_double(x, XDT, t * d + i), v1 = load_as_double(x, XDT, t * d + i + 32);
            const double v2 = load_as_double(x, XDT, t * d + i + 64), v3 = load_as_double(x, XDT, t * d + i + 96);
            s0 += v0 * v0;
            s1 += v1 * v1;
            s2 += v2 * v2;
            s3 += v3 * v3;
        }
        for (; i < d; i += 32) {
            const double v = load_as_double(x, XDT, t * d + i);
            s0 += v * v;
        }
    }
    double ss = (s0 + s1) + (s2 + s3);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    return sqrt(ss);
}

// sort.Ints(chosen) (mixtureofexperts.go:110) and the gates (:162-169).
__device__ __forceinline__ void write_choice(int64_t t, int k, int *pick, double *paff, int32_t *__restrict__ chosen,
                                             double *__restrict__ gates64, float *__restrict__ gates32) {
    const int lane = threadIdx.x & 31;
    for (int i = 1; i < k; i++) {
        int v = pick[i];
        double a = paff[i];
        int j = i - 1;
        while (j >= 0 && pick[j] > v) {
            pick[j + 1] = pick[j];
            paff[j + 1] = paff[j];
            j--;
        }
        pick[j + 1] = v;
        paff[j + 1] = a;
    }
    double total = 0;
    for (int i = 0; i < k; i++) total += paff[i];
    if (lane < k) {
        int e = pick[0];
        double a = paff[0];
        for (int q = 1; q < k; q++)
            if (q == lane) {
                e = pick[q];
                a = paff[q];
            }
        double g = a / total;
        chosen[t * k + lane] = e;
        gates64[t * k + lane] = g;
        gates32[t * k + lane] = (float)g;
    }
}

// x[x0 .. x0+d) . w[0 .. d) as one sequential float64 sum, each product and
// each partial sum rounded separately, in input order (vectormath.DotProduct,
// vector.go:67-74), by the whole warp: lane l fetches inputs 32b+l of every
// batch b (four batches ahead) and forms the products, lane 0 adds each
// batch's 32 products in order from shared memory.  Only the additions are
// serial.  Every lane calls it with the same arguments; all get the result.
template <int XDT>
__device__ double exact_dot_warp(const void *x, int64_t x0, const double *__restrict__ w, int d, double *buf,
                                 int lane) {
    constexpr int R = 4;
    const int nb = (d + 31) / 32;
    double xr[R], wr[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        const int i = 32 * r + lane;
        xr[r] = i < d ? load_as_double(x, XDT, x0 + i) : 0.0;
        wr[r] = i < d ? __ldg(w + i) : 0.0;
    }
    double s = 0;
    for (int b = 0; b < nb; b++) {
        const double p = __dmul_rn(xr[0], wr[0]);
#pragma unroll
        for (int r = 0; r < R - 1; r++) {
            xr[r] = xr[r + 1];
            wr[r] = wr[r + 1];
        }
        const int i = 32 * (b + R) + lane;
        xr[R - 1] = i < d ? load_as_double(x, XDT, x0 + i) : 0.0;
        wr[R - 1] = i < d ? __ldg(w + i) : 0.0;
        buf[lane] = p;
        __syncwarp();
        if (lane == 0) {
            const int n = d - 32 * b < 32 ? d - 32 * b : 32;
            for (int j = 0; j < n; j++) s = __dadd_rn(s, buf[j]);
        }
        __syncwarp();
    }
    return __shfl_sync(0xffffffffu, s, 0);
}

// One warp per flagged token.  With fast scores s^ within eps of the exact
// ones (thresh = 2 eps), L = s^_(k) and U = s^_(k+1): an expert with
// s^ > U + thresh is certainly chosen (only the other computed top-k experts
// can beat it), one with s^ < L - thresh certainly not (the k computed top-k
// experts beat it).  Only the experts in between get float64 logits, in the
// reference's order with separately rounded products and sums (one sequential
// sum, vectormath.DotProduct, vector.go:67-74), and fill the remaining places
// by exact score, ties to the lower index.
template <int XDT, int MAXJ>
__device__ void fixup_token(int64_t t, const double *__restrict__ logits, const double *__restrict__ bias,
                            const double *__restrict__ balance, int E, int k, const void *__restrict__ x, int d,
                            const double *__restrict__ w64, double thresh_scale, const double *__restrict__ xnorm,
                            int32_t *__restrict__ chosen, double *__restrict__ gates64, float *__restrict__ gates32,
                            double *wbuf) {
    const int lane = threadIdx.x & 31;
    double score[MAXJ], aff[MAXJ];
    load_scores<XDT, MAXJ>(logits, bias, balance, t, E, score, aff);
    int pick[kMaxTopK + 1];
    double pscore[kMaxTopK + 1], paff[kMaxTopK + 1];
    warp_top<MAXJ>(score, aff, 0u, E, k + 1, pick, pscore, paff);
    const double thresh = thresh_scale * (xnorm ? xnorm[t] : warp_x_norm<XDT>(x, t, d));
    const double L = pscore[k - 1], U = pscore[k];
    uint32_t sure = 0, unsure = 0;
#pragma unroll
    for (int j = 0; j < MAXJ; j++) {
        const int e = lane + 32 * j;
        if (e >= E) continue;
        if (score[j] > U + thresh) sure |= 1u << j;
        else if (!(score[j] < L - thresh)) unsure |= 1u << j;
    }
#pragma unroll
    for (int j = 0; j < MAXJ; j++) {
        uint32_t todo = __ballot_sync(0xffffffffu, (unsure >> j) & 1u);
        while (todo) {
            const int src = __ffs(todo) - 1;
            todo &= todo - 1;
            const int e = src + 32 * j;
            double s = exact_dot_warp<XDT>(x, t * d, w64 + (int64_t)e * d, d, wbuf, lane);
            if (lane == src) {
                s = __dadd_rn(s, bias[e]);
                aff[j] = affinity_d(s);
                score[j] = aff[j] + balance[e];
            }
        }
    }
    int n_sure = 0;
#pragma unroll
    for (int j = 0; j < MAXJ; j++) n_sure += __popc(__ballot_sync(0xffffffffu, (sure >> j) & 1u));
    // the sure experts first (any order), then the best unsure ones
    int npick = 0;
#pragma unroll
    for (int j = 0; j < MAXJ; j++) {
        uint32_t bal = __ballot_sync(0xffffffffu, (sure >> j) & 1u);
        while (bal) {
            const int src = __ffs(bal) - 1;
            bal &= bal - 1;
            const double a = __shfl_sync(0xffffffffu, aff[j], src);
            if (npick < kMaxTopK) {
                pick[npick] = src + 32 * j;
                paff[npick] = a;
            }
            npick++;
        }
    }
    warp_top<MAXJ>(score, aff, ~unsure, E, k - n_sure, pick + n_sure, pscore, paff + n_sure);
    write_choice(t, k, pick, paff, chosen, gates64, gates32);
}

template <int XDT, int MAXJ>
__global__ void __launch_bounds__(256)
    router_fixup_kernel(const double *__restrict__ logits, const double *__restrict__ bias,
                        const double *__restrict__ balance, int E, int k, const void *__restrict__ x, int d,
                        const double *__restrict__ w64, double thresh_scale, const double *__restrict__ xnorm,
                        int32_t *__restrict__ chosen, double *__restrict__ gates64, float *__restrict__ gates32,
                        const int *__restrict__ flagged, const int *__restrict__ n_flagged) {
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int n = *n_flagged;
    __shared__ double wsum[8][32];  // per warp: one batch of products (exact_dot_warp)
    double *wbuf = wsum[threadIdx.x >> 5];
    for (int wi = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); wi < n; wi += warps)
        fixup_token<XDT, MAXJ>(flagged[wi], logits, bias, balance, E, k, x, d, w64, thresh_scale, xnorm, chosen,
                               gates64, gates32, wbuf);
}

// One warp per token: scores from the fast logits, top-(k+1), and either the
// final choice or, when the k-th and (k+1)-th scores are within the error
// margin, the token's index on the fix-up list -- or, for a small batch
// (inline_fixup), the fix-up itself in this warp.
template <int XDT, int MAXJ, bool INLINE_FIXUP>
__device__ __forceinline__ void select_token(int64_t t, const double *__restrict__ logits,
                                             const double *__restrict__ bias, const double *__restrict__ balance,
                                             int E, int k, const void *__restrict__ x, int d, double thresh_scale,
                                             const double *__restrict__ xnorm, int32_t *__restrict__ chosen,
                                             double *__restrict__ gates64, float *__restrict__ gates32,
                                             int *__restrict__ flagged, int *__restrict__ n_flagged,
                                             const double *__restrict__ w64, double *wbuf) {
    const int lane = threadIdx.x & 31;
    double score[MAXJ], aff[MAXJ];
    load_scores<XDT, MAXJ>(logits, bias, balance, t, E, score, aff);
    int pick[kMaxTopK + 1];
    double pscore[kMaxTopK + 1], paff[kMaxTopK + 1];
    const int count = k < E ? k + 1 : k;
    warp_top<MAXJ>(score, aff, 0u, E, count, pick, pscore, paff);
    if (k < E) {
        const double thresh = thresh_scale * (xnorm ? xnorm[t] : warp_x_norm<XDT>(x, t, d));
        if (!(pscore[k - 1] - pscore[k] > thresh)) {
            if (INLINE_FIXUP) {
                // small batches: this warp settles the token itself (one launch fewer)
                fixup_token<XDT, MAXJ>(t, logits, bias, balance, E, k, x, d, w64, thresh_scale, xnorm, chosen,
                                       gates64, gates32, wbuf);
            } else if (lane == 0) {
                flagged[atomicAdd(n_flagged, 1)] = (int)t;
            }
            return;
        }
    }
    write_choice(t, k, pick, paff, chosen, gates64, gates32);
}

template <int XDT, int MAXJ, bool INLINE_FIXUP>
__global__ void __launch_bounds__(256)
    router_select_kernel(const double *__restrict__ logits, const double *__restrict__ bias,
                         const double *__restrict__ balance, int64_t T, int E, int k, const void *__restrict__ x, int d,
                         double thresh_scale, const double *__restrict__ xnorm, int32_t *__restrict__ chosen,
                         double *__restrict__ gates64, float *__restrict__ gates32, int *__restrict__ flagged,
                         int *__restrict__ n_flagged, const double *__restrict__ w64) {
    __shared__ double wsum[INLINE_FIXUP ? 8 : 1][32];  // inline fix-up: per warp one batch of products
    const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (t >= T) return;
    select_token<XDT, MAXJ, INLINE_FIXUP>(t, logits, bias, balance, E, k, x, d, thresh_scale, xnorm, chosen, gates64,
                                          gates32, flagged, n_flagged, w64,
                                          wsum[INLINE_FIXUP ? (threadIdx.x >> 5) : 0]);
}

// A batch of at most kFusedDispatchT tokens: one CTA selects every token's
// experts (a warp per token, fix-ups inline) and then runs the dispatch on
// the choices it just wrote (dispatch_small_body), one launch for both.
constexpr int64_t kFusedDispatchT = 32;
// ... and at most 128 experts: a warp's scores then fit the registers that
// 1024 threads leave each thread (64)
constexpr int kFusedDispatchMaxJ = 4;
constexpr int kFusedDispatchMaxE = 32 * kFusedDispatchMaxJ;

template <int XDT, int MAXJ>
__global__ void __launch_bounds__(kSmallDispatchThreads)
    router_select_dispatch_kernel(const double *__restrict__ logits, const double *__restrict__ bias,
                                  const double *__restrict__ balance, int64_t T, int E, int k,
                                  const void *__restrict__ x, int d, double thresh_scale,
                                  const double *__restrict__ xnorm, int32_t *__restrict__ chosen,
                                  double *__restrict__ gates64, float *__restrict__ gates32,
                                  const double *__restrict__ w64, const DispatchArgs da) {
    extern __shared__ int64_t dsm[];  // dispatch: E int64 positions, E int32 counts
    __shared__ double wsum[kFusedDispatchT][32];
    const int64_t t = threadIdx.x >> 5;
    if (t < T)
        select_token<XDT, MAXJ, true>(t, logits, bias, balance, E, k, x, d, thresh_scale, xnorm, chosen, gates64,
                                      gates32, nullptr, nullptr, w64, wsum[t]);
    __syncthreads();  // every token's choice is in `chosen`, visible to the whole CTA
    dispatch_small_body(chosen, T, E, k, da.S, da.bm, da.load, da.offsets, da.groups, da.tile_prefix, da.perm,
                        da.slot_row, dsm, reinterpret_cast<int32_t *>(dsm + E));
}

// hashedExperts (mixtureofexperts.go:88-96); gates 1/k (:148-151)
// A negative token ID is misuse that the reference panics on
// (mixtureofexperts.go:141-143); callers that pass device IDs the host has not
// checked see it as kErrNegativeTokenId in *err (the experts computed from the
// wrapped ID stay in range, so later kernels read valid indices).
__global__ void hash_route_kernel(const int64_t *__restrict__ ids, int64_t T, int E, int k, int32_t *__restrict__ chosen,
                                  double *__restrict__ gates64, float *__restrict__ gates32, int *err) {
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    if (ids[t] < 0 && err) atomicCAS(err, 0, kErrNegativeTokenId);
    uint64_t first = ((uint64_t)ids[t] * 2654435761ull + 12345ull) % (uint64_t)E;
    double g = 1.0 / (double)k;
    for (int i = 0; i < k; i++) {
        chosen[t * k + i] = (int32_t)((first + (uint64_t)i) % (uint64_t)E);
        gates64[t * k + i] = g;
        gates32[t * k + i] = (float)g;
    }
}

constexpr int64_t kInlineFixupT = 256;

template <int XDT, int MAXJ>
static int launch_select(const RouterArgs &a, const double *xnorm, cudaStream_t st) {
    if constexpr (MAXJ <= kFusedDispatchMaxJ) {
        if (router_fuses_dispatch(a)) {
            const unsigned threads = (unsigned)(a.T * 32 < 256 ? 256 : a.T * 32);
            router_select_dispatch_kernel<XDT, MAXJ><<<1, threads, a.E * (sizeof(int64_t) + sizeof(int32_t)), st>>>(
                a.logits, a.bias, a.balance, a.T, a.E, a.k, a.x, a.d, a.thresh_scale, xnorm, a.chosen, a.gates64,
                a.gates32, a.w64, *a.dispatch);
            GT_CUDA(cudaGetLastError());
            note_launches(1);
            return 0;
        }
    }
    unsigned sel_blocks = (unsigned)((a.T * 32 + 255) / 256);
    // a small batch has few tokens to settle: the select kernel's warps do it
    // (and the fix-up list, with its counter, is not used)
    const bool inline_fixup = a.T <= kInlineFixupT;
    if (!inline_fixup) GT_CUDA(cudaMemsetAsync(a.n_fixups, 0, sizeof(int), st));
    if (inline_fixup)
        router_select_kernel<XDT, MAXJ, true><<<sel_blocks, 256, 0, st>>>(
            a.logits, a.bias, a.balance, a.T, a.E, a.k, a.x, a.d, a.thresh_scale, xnorm, a.chosen, a.gates64,
            a.gates32, a.flagged, a.n_fixups, a.w64);
    else
        router_select_kernel<XDT, MAXJ, false><<<sel_blocks, 256, 0, st>>>(
            a.logits, a.bias, a.balance, a.T, a.E, a.k, a.x, a.d, a.thresh_scale, xnorm, a.chosen, a.gates64,
            a.gates32, a.flagged, a.n_fixups, a.w64);
    GT_CUDA(cudaGetLastError());
    if (a.k < a.E && !inline_fixup) {
        int64_t want = (a.T * 32 + 255) / 256;
        unsigned fix_blocks = (unsigned)(want < (int64_t)a.sms * 8 ? want : (int64_t)a.sms * 8);
        router_fixup_kernel<XDT, MAXJ><<<fix_blocks, 256, 0, st>>>(a.logits, a.bias, a.balance, a.E, a.k, a.x, a.d,
                                                                   a.w64, a.thresh_scale, xnorm, a.chosen,
                                                                   a.gates64, a.gates32, a.flagged, a.n_fixups);
        GT_CUDA(cudaGetLastError());
        note_launches(1);
    }
    note_launches(1);
    return 0;
}

template <int XDT>
static int launch_select_e(const RouterArgs &a, const double *xnorm, cudaStream_t st) {
    if (a.E <= 32) return launch_select<XDT, 1>(a, xnorm, st);
    if (a.E <= 64) return launch_select<XDT, 2>(a, xnorm, st);
    if (a.E <= 128) return launch_select<XDT, 4>(a, xnorm, st);
    if (a.E <= 256) return launch_select<XDT, 8>(a, xnorm, st);
    if (a.E <= 512) return launch_select<XDT, 16>(a, xnorm, st);
    return launch_select<XDT, 32>(a, xnorm, st);
}

bool router_fuses_dispatch(const RouterArgs &a) {
    return a.dispatch && !a.hash && a.T > 0 && a.T <= kFusedDispatchT && a.E <= kFusedDispatchMaxE && a.k < a.E &&
           a.dispatch->T == a.T && a.dispatch->chosen == a.chosen;
}

int launch_router(const RouterArgs &a, cudaStream_t st) {
    if (a.T == 0) return 0;
    if (a.hash) {
        hash_route_kernel<<<(unsigned)((a.T + 255) / 256), 256, 0, st>>>(a.token_ids, a.T, a.E, a.k, a.chosen,
                                                                         a.gates64, a.gates32, a.err);
        GT_CUDA(cudaGetLastError());
        note_launches(1);
        return 0;
    }
    const double *xnorm = nullptr;  // ||x_t|| per token, when the logits kernel left it
    if (a.use_tc) {
        GT_CHECK(launch_router_logits_tc(a.x_tc ? a.x_tc : a.x, a.x_tc_mid, a.x_tc_lo, a.T, a.d, a.E, a.e_pad, a.w3,
                                         a.logits, a.err, a.sms, st));
    } else if (a.T <= kRouterSmallMaxT) {
        dim3 grid((unsigned)((a.E + kRouterSmallWarps - 1) / kRouterSmallWarps), (unsigned)a.T);
        if (a.x_dtype == GTMOE_DTYPE_F64)
            router_logits_small_kernel<GTMOE_DTYPE_F64><<<grid, kRouterSmallWarps * 32, 0, st>>>(
                a.x, a.w32, a.T, a.E, a.d, a.logits, a.xnorm);
        else if (a.x_dtype == GTMOE_DTYPE_F32)
            router_logits_small_kernel<GTMOE_DTYPE_F32><<<grid, kRouterSmallWarps * 32, 0, st>>>(
                a.x, a.w32, a.T, a.E, a.d, a.logits, a.xnorm);
        else
            router_logits_small_kernel<GTMOE_DTYPE_BF16><<<grid, kRouterSmallWarps * 32, 0, st>>>(
                a.x, a.w32, a.T, a.E, a.d, a.logits, a.xnorm);
        GT_CUDA(cudaGetLastError());
        note_launches(1);
        xnorm = a.xnorm;
    } else {
        dim3 grid((unsigned)((a.T + kRouterTile - 1) / kRouterTile),
                  (unsigned)((a.E + kRouterTile - 1) / kRouterTile));
        if (a.x_dtype == GTMOE_DTYPE_F64)
            router_logits_kernel<GTMOE_DTYPE_F64><<<grid, 256, 0, st>>>(a.x, a.w32, a.T, a.E, a.d, a.logits);
        else if (a.x_dtype == GTMOE_DTYPE_F32)
            router_logits_kernel<GTMOE_DTYPE_F32><<<grid, 256, 0, st>>>(a.x, a.w32, a.T, a.E, a.d, a.logits);
        else
            router_logits_kernel<GTMOE_DTYPE_BF16><<<grid, 256, 0, st>>>(a.x, a.w32, a.T, a.E, a.d, a.logits);
        GT_CUDA(cudaGetLastError());
        note_launches(1);
    }
    if (a.x_dtype == GTMOE_DTYPE_F64) return launch_select_e<GTMOE_DTYPE_F64>(a, xnorm, st);
    if (a.x_dtype == GTMOE_DTYPE_F32) return launch_select_e<GTMOE_DTYPE_F32>(a, xnorm, st);
    return launch_select_e<GTMOE_DTYPE_BF16>(a, xnorm, st);
}

}  // namespace gtmoe
