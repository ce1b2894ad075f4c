// dispatch.cu -- expert-sorted token permutation (rowsForExpert,
// mixtureofexperts.go:175-180), per-expert load (:188-190), the group table
// of the grouped GEMMs, and the row gather (gatherRows, :114-120).
//
// rowsForExpert lists, for each expert, the tokens that chose it in
// ascending token order.  The scatter is therefore stable: (token, slot)
// pairs are ranked in token-major order, chunk by chunk, and within a chunk
// by warp match over 32 consecutive pairs; a token never lists an expert
// twice, so token-major pair order is token order per expert.  No atomics
// decide a position.
#include "common.cuh"
#include "internal.h"
#include "dispatch_small.cuh"

namespace gtmoe {

__global__ void dispatch_count_kernel(const int32_t *__restrict__ chosen, int64_t T, int E, int k,
                                      int32_t *__restrict__ counts) {
    extern __shared__ int32_t c_smem[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) c_smem[e] = 0;
    __syncthreads();
    int64_t t0 = (int64_t)blockIdx.x * kDispatchChunk;
    int64_t t1 = min(T, t0 + kDispatchChunk);
    for (int64_t p = t0 * k + threadIdx.x; p < t1 * k; p += blockDim.x) atomicAdd(&c_smem[chosen[p]], 1);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) counts[(int64_t)blockIdx.x * E + e] = c_smem[e];
}

__global__ void dispatch_scan_kernel(int32_t *__restrict__ counts, int n_chunks, int64_t T, int E, int S, int bm,
                                     int64_t *__restrict__ load, int64_t *__restrict__ offsets, Group *__restrict__ groups,
                                     int64_t *__restrict__ tile_prefix) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int32_t run = 0;
        for (int c = 0; c < n_chunks; c++) {
            int32_t v = counts[(int64_t)c * E + e];
            counts[(int64_t)c * E + e] = run;
            run += v;
        }
        load[e] = run;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int64_t xbase = S > 0 ? T : 0;
        int64_t off = 0, tiles = 0;
        for (int s = 0; s < S; s++) {
            Group g;
            g.x_row0 = 0;
            g.h_row0 = (int64_t)s * T;
            g.m = T;
            g.expert = s;
            g.pad = 0;
            groups[s] = g;
            tile_prefix[s] = tiles;
            tiles += (T + bm - 1) / bm;
        }
        for (int e = 0; e < E; e++) {
            offsets[e] = off;
            Group g;
            g.x_row0 = xbase + off;
            g.h_row0 = (int64_t)S * T + off;
            g.m = load[e];
            g.expert = S + e;
            g.pad = 0;
            groups[S + e] = g;
            tile_prefix[S + e] = tiles;
            tiles += (load[e] + bm - 1) / bm;
            off += load[e];
        }
        offsets[E] = off;
        tile_prefix[S + E] = tiles;
    }
}

__global__ void dispatch_scatter_kernel(const int32_t *__restrict__ chosen, const int32_t *__restrict__ counts,
                                        const int64_t *__restrict__ offsets, int64_t T, int E, int k,
                                        int32_t *__restrict__ perm, int64_t *__restrict__ slot_row) {
    extern __shared__ int64_t base[];
    const int lane = threadIdx.x;
    for (int e = lane; e < E; e += 32) base[e] = offsets[e] + counts[(int64_t)blockIdx.x * E + e];
    __syncwarp();
    int64_t t0 = (int64_t)blockIdx.x * kDispatchChunk;
    int64_t t1 = min(T, t0 + kDispatchChunk);
    const uint32_t lt = (1u << lane) - 1u;
    for (int64_t p0 = t0 * k; p0 < t1 * k; p0 += 32) {
        int64_t p = p0 + lane;
        bool valid = p < t1 * k;
        int e = valid ? chosen[p] : -1;
        uint32_t peers = __match_any_sync(0xffffffffu, e);
        int rank = __popc(peers & lt);
        int64_t pos = 0;
        if (valid) pos = base[e] + rank;
        __syncwarp();
        if (valid) {
            perm[pos] = (int32_t)(p / k);
            slot_row[p] = pos;
            if (rank == 0) base[e] += __popc(peers);
        }
        __syncwarp();
    }
}

// A batch of at most one chunk (decode-shaped): count, scan and scatter of
// the three kernels above in one CTA (dispatch_small.cuh), so that a small
// forward pays one launch for its dispatch.
__global__ void __launch_bounds__(kSmallDispatchThreads)
    dispatch_small_kernel(const int32_t *__restrict__ chosen, int64_t T, int E, int k, int S, int bm,
                          int64_t *__restrict__ load, int64_t *__restrict__ offsets, Group *__restrict__ groups,
                          int64_t *__restrict__ tile_prefix, int32_t *__restrict__ perm,
                          int64_t *__restrict__ slot_row) {
    extern __shared__ int64_t base[];  // E: next position of each expert's rows, then E int32 counts
    dispatch_small_body(chosen, T, E, k, S, bm, load, offsets, groups, tile_prefix, perm, slot_row, base,
                        reinterpret_cast<int32_t *>(base + E));
}

int launch_dispatch(const DispatchArgs &a, cudaStream_t st) {
    int n_chunks = (int)((a.T + kDispatchChunk - 1) / kDispatchChunk);
    if (a.T > 0 && a.T <= kDispatchChunk) {
        dispatch_small_kernel<<<1, kSmallDispatchThreads, a.E * (sizeof(int64_t) + sizeof(int32_t)), st>>>(
            a.chosen, a.T, a.E, a.k, a.S, a.bm, a.load, a.offsets, a.groups, a.tile_prefix, a.perm, a.slot_row);
        GT_CUDA(cudaGetLastError());
        note_launches(1);
        return 0;
    }
    if (a.T > 0) {
        dispatch_count_kernel<<<n_chunks, 256, a.E * sizeof(int32_t), st>>>(a.chosen, a.T, a.E, a.k, a.chunk_counts);
        GT_CUDA(cudaGetLastError());
        note_launches(1);
    }
    dispatch_scan_kernel<<<1, 1024, 0, st>>>(a.chunk_counts, n_chunks, a.T, a.E, a.S, a.bm, a.load, a.offsets,
                                             a.groups, a.tile_prefix);
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    if (a.T > 0) {
        dispatch_scatter_kernel<<<n_chunks, 32, a.E * sizeof(int64_t), st>>>(a.chosen, a.chunk_counts, a.offsets,
                                                                             a.T, a.E, a.k, a.perm, a.slot_row);
        GT_CUDA(cudaGetLastError());
        note_launches(1);
    }
    return 0;
}

// The gather is token-major: each token row of x is read once and written
// to its shared-expert row (row t) and to its k routed rows (the dispatch's
// slot_row), so x is read from memory once instead of once per copy (the
// routed order visits the tokens in expert order, which at c5-like sizes does
// not stay in L2 between an expert and the next).

// Conversions: one CTA of kGatherThreads per token; each thread's loads of a
// row are issued kGatherUnroll at a time, so a row of a few-token batch costs
// about one memory latency.  A batch too small to fill the GPU this way
// (fewer than kGatherSplitCtas tokens x copies) takes one CTA per (token,
// copy) instead (gridDim.y = copies): its rows are in L2 anyway.
constexpr int kGatherThreads = 256;
constexpr int kGatherUnroll = 8;
constexpr int64_t kGatherSplitCtas = 296;

template <typename IN>
__device__ __forceinline__ double in_as_double(IN v) {
    if constexpr (sizeof(IN) == 2) return (double)__bfloat162float(v);
    else return (double)v;
}

template <typename IN, typename OUT>
__global__ void __launch_bounds__(kGatherThreads)
    gather_kernel(const IN *__restrict__ x, int d, const int64_t *__restrict__ slot_row, int k, int64_t xbase,
                  int copy_shared, OUT *__restrict__ xp) {
    const int64_t t = blockIdx.x;
    __shared__ int64_t dst[kMaxTopK + 1];
    const int n_dst = (copy_shared ? 1 : 0) + k;
    if (threadIdx.x < n_dst) {
        const int j = (int)threadIdx.x - (copy_shared ? 1 : 0);
        dst[threadIdx.x] = (j < 0 ? t : xbase + slot_row[t * k + j]) * d;
    }
    __syncthreads();
    const int c0 = gridDim.y > 1 ? (int)blockIdx.y : 0, c1 = gridDim.y > 1 ? c0 + 1 : n_dst;  // copies of this CTA
    const IN *row = x + t * d;
    constexpr int kStride = kGatherThreads * kGatherUnroll;
    int i = threadIdx.x;
    for (; i + kGatherThreads * (kGatherUnroll - 1) < d; i += kStride) {
        IN v[kGatherUnroll];
#pragma unroll
        for (int u = 0; u < kGatherUnroll; u++) v[u] = row[i + kGatherThreads * u];
#pragma unroll
        for (int u = 0; u < kGatherUnroll; u++) {
            const OUT o = from_double<OUT>(in_as_double(v[u]));
            for (int c = c0; c < c1; c++) xp[dst[c] + i + kGatherThreads * u] = o;
        }
    }
    for (; i < d; i += kGatherThreads) {
        const OUT o = from_double<OUT>(in_as_double(row[i]));
        for (int c = c0; c < c1; c++) xp[dst[c] + i] = o;
    }
}

template <typename OUT>
static void launch_gather_rows(const void *x, int x_dtype, int64_t T, int d, const int64_t *slot_row, int k,
                               int64_t xbase, int copy_shared, OUT *xp, cudaStream_t st) {
    const int n_dst = (copy_shared ? 1 : 0) + k;
    const dim3 grid((unsigned)T, T * n_dst < kGatherSplitCtas ? (unsigned)n_dst : 1u);
    if (x_dtype == GTMOE_DTYPE_F64)
        gather_kernel<double, OUT><<<grid, kGatherThreads, 0, st>>>((const double *)x, d, slot_row, k, xbase,
                                                                   copy_shared, xp);
    else if (x_dtype == GTMOE_DTYPE_F32)
        gather_kernel<float, OUT><<<grid, kGatherThreads, 0, st>>>((const float *)x, d, slot_row, k, xbase,
                                                                  copy_shared, xp);
    else
        gather_kernel<__nv_bfloat16, OUT><<<grid, kGatherThreads, 0, st>>>((const __nv_bfloat16 *)x, d, slot_row, k,
                                                                          xbase, copy_shared, xp);
}

// Same-type bf16 rows: one warp per token, 16-byte pieces, four loads in
// flight per lane, each piece stored to every copy of the row.
constexpr int kGatherVecUnroll = 4;

__global__ void __launch_bounds__(256)
    gather_bf16_vec_kernel(const uint4 *__restrict__ x, int64_t T, int dv, const int64_t *__restrict__ slot_row,
                           int k, int64_t xbase, int copy_shared, uint4 *__restrict__ xp) {
    const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    // lane j < k holds the first 16-byte piece of routed copy j
    const int64_t my_dst = lane < k ? (xbase + slot_row[t * k + lane]) * dv : 0;
    const uint4 *row = x + t * dv;
    uint4 *shared_row = copy_shared ? xp + t * dv : nullptr;
    constexpr int kStride = 32 * kGatherVecUnroll;
    for (int i0 = 0; i0 < dv; i0 += kStride) {
        uint4 v[kGatherVecUnroll];
#pragma unroll
        for (int u = 0; u < kGatherVecUnroll; u++) {
            const int i = i0 + 32 * u + lane;
            if (i < dv) v[u] = row[i];
        }
#pragma unroll
        for (int u = 0; u < kGatherVecUnroll; u++) {
            const int i = i0 + 32 * u + lane;
            if (shared_row && i < dv) shared_row[i] = v[u];
        }
        for (int j = 0; j < k; j++) {
            const int64_t o = __shfl_sync(0xffffffffu, my_dst, j);
#pragma unroll
            for (int u = 0; u < kGatherVecUnroll; u++) {
                const int i = i0 + 32 * u + lane;
                if (i < dv) xp[o + i] = v[u];
            }
        }
    }
}

int launch_gather(const void *x, int x_dtype, int64_t T, int d, const int64_t *slot_row, int k, int64_t xbase,
                  int copy_shared, void *xp, int xp_dtype, cudaStream_t st) {
    if (T == 0 || (k == 0 && !copy_shared)) return 0;
    if (k > kMaxTopK) return fail(GTMOE_EINVAL, "gather: %d copies per token (at most %d)", k, kMaxTopK);
    if (x_dtype == GTMOE_DTYPE_BF16 && xp_dtype == GTMOE_DTYPE_BF16 && d % 8 == 0) {
        const unsigned blocks = (unsigned)((T * 32 + 255) / 256);
        gather_bf16_vec_kernel<<<blocks, 256, 0, st>>>((const uint4 *)x, T, d / 8, slot_row, k, xbase, copy_shared,
                                                       (uint4 *)xp);
    } else if (xp_dtype == GTMOE_DTYPE_F64) {
        launch_gather_rows<double>(x, x_dtype, T, d, slot_row, k, xbase, copy_shared, (double *)xp, st);
    } else if (xp_dtype == GTMOE_DTYPE_F32) {
        launch_gather_rows<float>(x, x_dtype, T, d, slot_row, k, xbase, copy_shared, (float *)xp, st);
    } else {
        launch_gather_rows<__nv_bfloat16>(x, x_dtype, T, d, slot_row, k, xbase, copy_shared, (__nv_bfloat16 *)xp,
                                          st);
    }
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    return 0;
}

}  // namespace gtmoe
