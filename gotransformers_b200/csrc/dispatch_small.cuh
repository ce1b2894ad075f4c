// dispatch_small.cuh -- the dispatch of a decode-sized batch inside one CTA
// (rowsForExpert, mixtureofexperts.go:175-180; per-expert load, :188-190),
// shared by the small dispatch kernel and the router's fused select+dispatch.
#pragma once
#include "common.cuh"
#include "internal.h"

namespace gtmoe {

// Dispatch of a batch of at most one chunk inside one CTA of any size up to
// kSmallDispatchThreads: the count, scan and scatter of the chunked dispatch
// kernels (dispatch.cu) with the same arithmetic and the same outputs.  The
// scan over experts runs on all threads (each a run of consecutive experts,
// then a block-wide exclusive scan of the runs' row and tile counts), so the
// group table is written in parallel instead of by one thread.  base and cnt
// are E int64 / E int32 of shared memory.  All threads of the CTA call it.
constexpr int kSmallDispatchThreads = 1024;

__device__ __forceinline__ void dispatch_small_body(const int32_t *__restrict__ chosen, int64_t T, int E, int k,
                                                    int S, int bm, int64_t *__restrict__ load,
                                                    int64_t *__restrict__ offsets, Group *__restrict__ groups,
                                                    int64_t *__restrict__ tile_prefix, int32_t *__restrict__ perm,
                                                    int64_t *__restrict__ slot_row, int64_t *base, int32_t *cnt) {
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

}  // namespace gtmoe
