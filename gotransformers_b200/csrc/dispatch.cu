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
// the three kernels above in one CTA, with the same arithmetic and the same
// outputs, so that a small forward pays one launch for its dispatch.  The
// scan over experts runs on all threads (each a run of consecutive experts,
// then a block-wide exclusive scan of the runs' row and tile counts), so the
// group table is written in parallel instead of by one thread.
constexpr int kSmallDispatchThreads = 1024;

__global__ void __launch_bounds__(kSmallDispatchThreads)
    dispatch_small_kernel(const int32_t *__restrict__ chosen, int64_t T, int E, int k, int S, int bm,
                          int64_t *__restrict__ load, int64_t *__restrict__ offsets, Group *__restrict__ groups,
                          int64_t *__restrict__ tile_prefix, int32_t *__restrict__ perm,
                          int64_t *__restrict__ slot_row) {
    extern __shared__ int64_t base[];  // E: next position of each expert's rows
    int32_t *cnt = reinterpret_cast<int32_t *>(base + E);
    __shared__ int64_t wrows[kSmallDispatchThreads / 32], wtiles[kSmallDispatchThreads / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int64_t p = tid; p < T * k; p += blockDim.x) atomicAdd(&cnt[chosen[p]], 1);
    __syncthreads();
    // this thread's run of experts [e0, e1)
    const int per = (E + blockDim.x - 1) / blockDim.x;
    const int e0 = min(E, tid * per), e1 = min(E, e0 + per);
    int64_t rows = 0, tiles = 0;
    for (int e = e0; e < e1; e++) {
        rows += cnt[e];
        tiles += (cnt[e] + bm - 1) / bm;
    }
    // exclusive scan of (rows, tiles) over the threads
    int64_t ir = rows, it = tiles;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int64_t r = __shfl_up_sync(0xffffffffu, ir, off), q = __shfl_up_sync(0xffffffffu, it, off);
        if (lane >= off) {
            ir += r;
            it += q;
        }
    }
    if (lane == 31) {
        wrows[warp] = ir;
        wtiles[warp] = it;
    }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        int64_t r = lane < nw ? wrows[lane] : 0, q = lane < nw ? wtiles[lane] : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int64_t r2 = __shfl_up_sync(0xffffffffu, r, off), q2 = __shfl_up_sync(0xffffffffu, q, off);
            if (lane >= off) {
                r += r2;
                q += q2;
            }
        }
        if (lane < nw) {
            wrows[lane] = r;  // inclusive over warps
            wtiles[lane] = q;
        }
    }
    __syncthreads();
    const int64_t shared_tiles = (int64_t)S * ((T + bm - 1) / bm);
    int64_t off = ir - rows + (warp > 0 ? wrows[warp - 1] : 0);
    int64_t tl = shared_tiles + it - tiles + (warp > 0 ? wtiles[warp - 1] : 0);
    const int64_t xbase = S > 0 ? T : 0;
    for (int e = e0; e < e1; e++) {
        const int64_t n = cnt[e];
        load[e] = n;
        offsets[e] = off;
        base[e] = off;
        groups[S + e] = Group{xbase + off, (int64_t)S * T + off, n, S + e, 0};
        tile_prefix[S + e] = tl;
        tl += (n + bm - 1) / bm;
        off += n;
    }
    if (tid < S) {
        groups[tid] = Group{0, (int64_t)tid * T, T, tid, 0};
        tile_prefix[tid] = (int64_t)tid * ((T + bm - 1) / bm);
    }
    if (tid == blockDim.x - 1) {  // the last run ends at the totals
        offsets[E] = off;
        tile_prefix[S + E] = tl;
    }
    __syncthreads();
    if (warp == 0) {  // the scatter of dispatch_scatter_kernel, one warp over the chunk
        const uint32_t lt = (1u << lane) - 1u;
        for (int64_t p0 = 0; p0 < T * k; p0 += 32) {
            const int64_t p = p0 + lane;
            const bool valid = p < T * k;
            const int e = valid ? chosen[p] : -1;
            const uint32_t peers = __match_any_sync(0xffffffffu, e);
            const int rank = __popc(peers & lt);
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

// One CTA of kGatherThreads per row; each thread's loads of a row are issued
// kGatherUnroll at a time, so a row of a few-token batch costs about one memory
// latency.
constexpr int kGatherThreads = 256;
constexpr int kGatherUnroll = 8;

template <typename IN>
__device__ __forceinline__ double in_as_double(IN v) {
    if constexpr (sizeof(IN) == 2) return (double)__bfloat162float(v);
    else return (double)v;
}

template <typename IN, typename OUT>
__global__ void __launch_bounds__(kGatherThreads)
    gather_kernel(const IN *__restrict__ x, int64_t T, int d, const int32_t *__restrict__ perm, int64_t n_routed,
                  int64_t xbase, int copy_shared, OUT *__restrict__ xp) {
    const int64_t w = blockIdx.x;
    const int64_t n_shared_rows = copy_shared ? T : 0;
    int64_t src, dst;
    if (w < n_shared_rows) {
        src = w;
        dst = w;
    } else {
        const int64_t r = w - n_shared_rows;
        src = perm[r];
        dst = xbase + r;
    }
    const IN *row = x + src * d;
    OUT *out = xp + dst * d;
    constexpr int kStride = kGatherThreads * kGatherUnroll;
    int i = threadIdx.x;
    for (; i + kGatherThreads * (kGatherUnroll - 1) < d; i += kStride) {
        IN v[kGatherUnroll];
#pragma unroll
        for (int u = 0; u < kGatherUnroll; u++) v[u] = row[i + kGatherThreads * u];
#pragma unroll
        for (int u = 0; u < kGatherUnroll; u++) out[i + kGatherThreads * u] = from_double<OUT>(in_as_double(v[u]));
    }
    for (; i < d; i += kGatherThreads) out[i] = from_double<OUT>(in_as_double(row[i]));
}

template <typename OUT>
static void launch_gather_rows(const void *x, int x_dtype, int64_t T, int d, const int32_t *perm, int64_t n_routed,
                               int64_t xbase, int copy_shared, OUT *xp, int64_t rows, cudaStream_t st) {
    if (x_dtype == GTMOE_DTYPE_F64)
        gather_kernel<double, OUT><<<(unsigned)rows, kGatherThreads, 0, st>>>((const double *)x, T, d, perm, n_routed,
                                                                             xbase, copy_shared, xp);
    else if (x_dtype == GTMOE_DTYPE_F32)
        gather_kernel<float, OUT><<<(unsigned)rows, kGatherThreads, 0, st>>>((const float *)x, T, d, perm, n_routed,
                                                                            xbase, copy_shared, xp);
    else
        gather_kernel<__nv_bfloat16, OUT><<<(unsigned)rows, kGatherThreads, 0, st>>>(
            (const __nv_bfloat16 *)x, T, d, perm, n_routed, xbase, copy_shared, xp);
}

// Same-type bf16 rows: 16-byte vector copies.
__global__ void gather_bf16_vec_kernel(const uint4 *__restrict__ x, int64_t T, int vec_per_row,
                                       const int32_t *__restrict__ perm, int64_t n_routed, int64_t xbase,
                                       int copy_shared, uint4 *__restrict__ xp) {
    int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    int64_t n_shared_rows = copy_shared ? T : 0;
    if (w >= n_shared_rows + n_routed) return;
    int64_t src, dst;
    if (w < n_shared_rows) {
        src = w;
        dst = w;
    } else {
        int64_t r = w - n_shared_rows;
        src = perm[r];
        dst = xbase + r;
    }
    for (int i = lane; i < vec_per_row; i += 32) xp[dst * vec_per_row + i] = x[src * vec_per_row + i];
}

int launch_gather(const void *x, int x_dtype, int64_t T, int d, const int32_t *perm, int64_t n_routed_rows,
                  int64_t xbase, int copy_shared, void *xp, int xp_dtype, cudaStream_t st) {
    int64_t rows = (copy_shared ? T : 0) + n_routed_rows;
    if (rows == 0) return 0;
    unsigned blocks = (unsigned)((rows * 32 + 255) / 256);
    if (x_dtype == GTMOE_DTYPE_BF16 && xp_dtype == GTMOE_DTYPE_BF16 && d % 8 == 0) {
        gather_bf16_vec_kernel<<<blocks, 256, 0, st>>>((const uint4 *)x, T, d / 8, perm, n_routed_rows, xbase,
                                                       copy_shared, (uint4 *)xp);
    } else if (xp_dtype == GTMOE_DTYPE_F64) {
        launch_gather_rows<double>(x, x_dtype, T, d, perm, n_routed_rows, xbase, copy_shared, (double *)xp, rows, st);
    } else if (xp_dtype == GTMOE_DTYPE_F32) {
        launch_gather_rows<float>(x, x_dtype, T, d, perm, n_routed_rows, xbase, copy_shared, (float *)xp, rows, st);
    } else {
        launch_gather_rows<__nv_bfloat16>(x, x_dtype, T, d, perm, n_routed_rows, xbase, copy_shared,
                                          (__nv_bfloat16 *)xp, rows, st);
    }
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    return 0;
}

}  // namespace gtmoe
