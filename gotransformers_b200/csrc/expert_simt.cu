// expert_simt.cu -- grouped SwiGLU expert products on the SIMT cores
// (GatedFeedForward.Forward, feedforward/gatedfeedforward.go:49-57, over the
// rows of each expert; perceptron/layer.go:121-162 for each layer).
//
// Used for Float64 and Float32 experts (computed in float64 / float32: the
// north star's 1e-5 bound for Float32 rules out a single bf16 tensor-core
// pass) and for shapes the tensor-core kernels do not tile.  Int8 and FP4
// weights are decoded in the operand load exactly as Rows.Row does
// (lowprecision/rows.go:87-119).
//
// Persistent grid: each block walks work units u = (group, n-tile, m-tile)
// from a device-side prefix of m-tiles, so the launch needs no host copy of
// the per-expert loads.
#include "common.cuh"
#include "internal.h"

namespace gtmoe {

constexpr int kBN = 64;
constexpr int kBK = 16;

template <int PREC, typename CT>
__device__ __forceinline__ void load_w4(const void *__restrict__ w, const float *__restrict__ s, int rows, int width,
                                        int row, int k, CT (&out)[4]) {
    // four consecutive values of one row; k is a multiple of 4, so all four
    // share one 16-value scale block
#pragma unroll
    for (int i = 0; i < 4; i++) out[i] = CT(0);
    if (row >= rows) return;
    const int64_t base = (int64_t)row * width;
    if (PREC == GTMOE_FLOAT64) {
#pragma unroll
        for (int i = 0; i < 4; i++)
            if (k + i < width) out[i] = (CT)((const double *)w)[base + k + i];
    } else if (PREC == GTMOE_FLOAT32) {
#pragma unroll
        for (int i = 0; i < 4; i++)
            if (k + i < width) out[i] = (CT)((const float *)w)[base + k + i];
    } else if (PREC == GTMOE_INT8) {
        if (k >= width) return;
        CT sc = (CT)s[(int64_t)row * scale_blocks(width) + k / kValuesPerScale];
#pragma unroll
        for (int i = 0; i < 4; i++)
            if (k + i < width) out[i] = (CT)((const int8_t *)w)[base + k + i] * sc;
    } else {
        if (k >= width) return;
        CT sc = (CT)s[(int64_t)row * scale_blocks(width) + k / kValuesPerScale];
        const uint8_t *p = (const uint8_t *)w + (int64_t)row * fp4_row_bytes(width);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int kk = k + i;
            if (kk < width) {
                uint8_t b = p[kk / 2];
                uint32_t code = (kk & 1) ? (b >> 4) : (b & 15u);
                out[i] = (CT)fp4_value(code) * sc;
            }
        }
    }
}

template <int PREC, typename CT, bool GATED>
__global__ void __launch_bounds__(256) grouped_simt_kernel(GroupedArgs a) {
    __shared__ CT As[kBK][kSimtBM + 4];
    __shared__ CT Bg[kBK][kBN + 4];
    __shared__ CT Bu[GATED ? kBK : 1][kBN + 4];

    const int n_out = GATED ? a.h : a.d;
    const int K = GATED ? a.d : a.h;
    const int n_tiles = (n_out + kBN - 1) / kBN;
    const int64_t total = a.tile_prefix[a.n_groups] * n_tiles;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const CT limit = (CT)a.clamp_limit;
    const CT *__restrict__ in = (const CT *)(GATED ? a.xp : a.hp);
    CT *__restrict__ outp = (CT *)(GATED ? a.hp : a.yp);

    for (int64_t u = blockIdx.x; u < total; u += gridDim.x) {
        // group of work unit u
        int lo = 0, hi = a.n_groups - 1;
        while (lo < hi) {
            int mid = (lo + hi + 1) >> 1;
            if (a.tile_prefix[mid] * n_tiles <= u) lo = mid;
            else hi = mid - 1;
        }
        const int g = lo;
        const Group grp = a.groups[g];
        const int64_t mt_g = a.tile_prefix[g + 1] - a.tile_prefix[g];
        const int64_t r = u - a.tile_prefix[g] * n_tiles;
        const int nt = (int)(r / mt_g);
        const int64_t mt = r % mt_g;
        const int64_t in_row0 = (GATED ? grp.x_row0 : grp.h_row0) + mt * kSimtBM;
        const int64_t m_left = grp.m - mt * kSimtBM;
        const ExpertLayers L = a.experts[grp.expert];
        const int n0 = nt * kBN;

        CT accG[4][4], accU[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                accG[i][j] = CT(0);
                accU[i][j] = CT(0);
            }

        const int lr = threadIdx.x / 4;       // 0..63 row of the tile being loaded
        const int lk = (threadIdx.x % 4) * 4;  // 0,4,8,12
        for (int k0 = 0; k0 < K; k0 += kBK) {
            {
                CT v[4];
#pragma unroll
                for (int i = 0; i < 4; i++) v[i] = CT(0);
                if (lr < m_left) {
                    const CT *src = in + (in_row0 + lr) * (int64_t)K;
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        if (k0 + lk + i < K) v[i] = src[k0 + lk + i];
                }
#pragma unroll
                for (int i = 0; i < 4; i++) As[lk + i][lr] = v[i];
            }
            {
                CT v[4];
                load_w4<PREC, CT>(L.w[GATED ? 0 : 2], L.s[GATED ? 0 : 2], n_out, K, n0 + lr, k0 + lk, v);
#pragma unroll
                for (int i = 0; i < 4; i++) Bg[lk + i][lr] = v[i];
                if (GATED) {
                    load_w4<PREC, CT>(L.w[1], L.s[1], n_out, K, n0 + lr, k0 + lk, v);
#pragma unroll
                    for (int i = 0; i < 4; i++) Bu[lk + i][lr] = v[i];
                }
            }
            __syncthreads();
#pragma unroll
            for (int c = 0; c < kBK; c++) {
                CT av[4], bg[4], bu[4];
#pragma unroll
                for (int i = 0; i < 4; i++) av[i] = As[c][ty * 4 + i];
#pragma unroll
                for (int j = 0; j < 4; j++) bg[j] = Bg[c][tx * 4 + j];
                if (GATED) {
#pragma unroll
                    for (int j = 0; j < 4; j++) bu[j] = Bu[c][tx * 4 + j];
                }
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        accG[i][j] = fma(av[i], bg[j], accG[i][j]);
                        if (GATED) accU[i][j] = fma(av[i], bu[j], accU[i][j]);
                    }
            }
            __syncthreads();
        }

        const int64_t out_row0 = grp.h_row0 + mt * kSimtBM;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int rr = ty * 4 + i;
            if (rr >= m_left) continue;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                int col = n0 + tx * 4 + j;
                if (col >= n_out) continue;
                CT v;
                if (GATED) {
                    CT bg = L.b64[0] ? (sizeof(CT) == 8 ? (CT)L.b64[0][col] : (CT)L.b32[0][col]) : CT(0);
                    CT bu = L.b64[1] ? (sizeof(CT) == 8 ? (CT)L.b64[1][col] : (CT)L.b32[1][col]) : CT(0);
                    v = gate_act<CT>(accG[i][j] + bg, a.clamped, limit) * up_act<CT>(accU[i][j] + bu, a.clamped, limit);
                } else {
                    CT bd = L.b64[2] ? (sizeof(CT) == 8 ? (CT)L.b64[2][col] : (CT)L.b32[2][col]) : CT(0);
                    v = accG[i][j] + bd;
                }
                outp[(out_row0 + rr) * (int64_t)n_out + col] = v;
            }
        }
    }
}

template <int PREC, typename CT>
static int launch_one(const GroupedArgs &a, int which, cudaStream_t st) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    unsigned grid = (unsigned)(sms * 4);
    if (which == 1) grouped_simt_kernel<PREC, CT, true><<<grid, 256, 0, st>>>(a);
    else grouped_simt_kernel<PREC, CT, false><<<grid, 256, 0, st>>>(a);
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    return 0;
}

int launch_grouped_simt(const GroupedArgs &a, int which, cudaStream_t st) {
    if (a.compute == GTMOE_DTYPE_F64) {
        switch (a.precision) {
        case GTMOE_FLOAT64: return launch_one<GTMOE_FLOAT64, double>(a, which, st);
        case GTMOE_FLOAT32: return launch_one<GTMOE_FLOAT32, double>(a, which, st);
        case GTMOE_INT8: return launch_one<GTMOE_INT8, double>(a, which, st);
        default: return launch_one<GTMOE_FP4, double>(a, which, st);
        }
    }
    switch (a.precision) {
    case GTMOE_FLOAT64: return launch_one<GTMOE_FLOAT64, float>(a, which, st);
    case GTMOE_FLOAT32: return launch_one<GTMOE_FLOAT32, float>(a, which, st);
    case GTMOE_INT8: return launch_one<GTMOE_INT8, float>(a, which, st);
    default: return launch_one<GTMOE_FP4, float>(a, which, st);
    }
}

}  // namespace gtmoe
