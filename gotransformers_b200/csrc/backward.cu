// backward.cu -- MixtureOfExperts.Backward (mixtureofexperts.go:227-285) on
// the GPU, in float64, for the last Forward of a handle in training mode.
//
// The reference's pieces, restated:
// * every shared expert's GatedFeedForward.Backward on the output gradients,
//   summed (AddMatrices) in expert order; then for each routed expert in
//   ascending order the backward of its rows with the output gradient rows
//   scaled by the token's gate, added into the token's row (:235-257);
// * GatedFeedForward.Backward (feedforward/gatedfeedforward.go:59-66):
//   dH = Down.Backward(dY); gate' = dH * up outputs; up' = dH * gate outputs;
//   dX = Gate.Backward(gate') + Up.Backward(up');
// * perceptron.Layer.Backward for compressed rows (layer.go:164-207): the
//   pre-activation gradient g * act'(pre) per (example, neuron); the expert
//   layers are compressed, so frozen (no weight gradients, :165-167, 184);
//   the input gradients add every neuron's scaled row in ascending neuron
//   order, skipping zero gradients (adapter.go:108-120 ->
//   Rows.AddScaledRowTo, lowprecision/rows.go:285-324: Float64 g * w,
//   Float32 g * float64(w), Int8 (g * scale) * q, FP4 (g * scale) * value);
// * the router term (:262-284): per token, gate gradient i = dout . y_i (the
//   expert's output row), then (gate gradient i - sum_j gate gradient j *
//   gate j) / sum of the chosen affinities, times affinityDerivative
//   (softplus'(logit) / (2 affinity), :84-86), as the gradient of logit i;
//   RouterLayer.Backward on these logit gradients: bias gradients added per
//   example, weight gradients as TransposedTimesMatrix (tokens ascending,
//   vectormath/backend.go:139-158) added after, input gradients through the
//   dense weights (MatrixTimesWeights, backend.go:84-112: experts ascending,
//   zeros skipped); dx = expert input gradients + router input gradients.
//
// The gate/up pre-activations, hidden values and expert outputs the reference
// keeps from Forward are recomputed here from the saved float64 input rows.
// Work rows: r < S*T are (shared expert r / T, token r % T); after them
// (token t, slot i) for t*k + i.  The experts' part runs as four grouped
// float64 GEMM stages over tiles of one expert's rows (bwd_gemm_kernel), each
// output one float64 sum over its inputs in ascending order: the reference's
// values up to summation rounding (per-16-value partial sums times the scale,
// rows.go:207-257, and zero gradients skipped there, not here).
#include "handle.h"

namespace gtmoe {
namespace {

__device__ __forceinline__ double sigmoid_d(double x) { return 1.0 / (1.0 + exp(-x)); }

// Derivatives of the expert activations, taking the pre-activation: SiLU
// s + x s (1 - s) (activationfunction.go:106-109), Linear 1 (:162-164), and
// the clamped variants, 0 where the forward clamps
// (moreactivationfunctions.go:207-243).
__device__ __forceinline__ double gate_deriv(double x, int clamped, double limit) {
    if (clamped && x > limit) return 0.0;
    const double s = sigmoid_d(x);
    return s + x * s * (1 - s);
}
__device__ __forceinline__ double up_deriv(double x, int clamped, double limit) {
    if (clamped && (x > limit || x < -limit)) return 0.0;
    return 1.0;
}

// The router's softplus (moreactivationfunctions.go:8-16).
__device__ __forceinline__ double softplus_d(double x) {
    if (x > 20) return x;
    if (x < -20) return exp(x);
    return log1p(exp(x));
}

struct BwdArgs {
    const ExpertLayers *experts;
    int prec;
    int S, k, d, h;
    int clamped;
    double limit;
    int64_t T;
    const double *x;        // T x d, the Forward's input rows
    const int32_t *chosen;  // T x k, ascending per token
    const double *gates;    // T x k
    const double *dout;     // T x d
    double *rows_dx;        // (S*T + T*k) x d: input gradients of each work row
    double *rows_y;         // T*k x d: routed experts' output rows
};

// ---- Grouped float64 GEMM stages (the expert part of the backward).
//
// The work rows are taken expert by expert (shared experts' rows s*T + t,
// then each routed expert's (token, slot) rows in the forward's token order),
// in tiles of kBgRows rows of one expert, so that every dequantised weight
// tile serves kBgRows rows instead of one:
//   stage 0: PG, PU = X Wg^T + bg, X Wu^T + bu          (K = d, N = h)
//   stage 1: Y = H Wd^T + bd, H = act_g(PG) act_u(PU)     (routed rows; K = h, N = d)
//   stage 2: dH = dY' Wd (dY' = dout, gate-scaled for routed rows), then in
//            place PG <- dH act_u(PU) act_g'(PG), PU <- dH act_g(PG) act_u'(PU)
//                                                        (K = d, N = h)
//   stage 3: dX = dG Wg + dU Wu                          (K = h, N = d)
// Each output is one float64 sum over K in ascending order; against the
// reference's sequence (per-block partial sums times the scale, zeros
// skipped) it differs by rounding only.
constexpr int kBgRows = 64;   // rows per tile (one expert)
constexpr int kBgCols = 64;   // output columns per tile
constexpr int kBgK = 16;      // inputs per shared-memory step
constexpr int kBgThreads = 256;

// Work rows in expert-major order (wrow) and each group's first entry (goff):
// group s < S is shared expert s (rows s*T + t), group S + e routed expert e.
__global__ void bwd_worklist_kernel(const int32_t *__restrict__ chosen, const int32_t *__restrict__ perm,
                                    const int64_t *__restrict__ offsets, int64_t T, int k, int S, int E,
                                    int64_t *__restrict__ wrow, int64_t *__restrict__ goff) {
    const int64_t n_shared = (int64_t)S * T;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i <= S + E) goff[i] = i <= S ? i * T : n_shared + offsets[i - S];
    if (i < n_shared) wrow[i] = i;
    if (i < T * k) {
        // the (token, slot) pair i: its position in its expert's token list
        const int64_t t = i / k;
        const int e = chosen[i];
        int64_t lo = offsets[e], hi = offsets[e + 1];  // perm[lo..hi) ascending tokens
        while (hi - lo > 1) {
            const int64_t mid = (lo + hi) >> 1;
            if (perm[mid] <= t) lo = mid;
            else hi = mid;
        }
        wrow[n_shared + lo] = n_shared + i;
    }
}

// Tiles of kBgRows rows per group: tprefix[g] = tiles before group g.
__global__ void bwd_tiles_kernel(const int64_t *__restrict__ goff, int G, int64_t *__restrict__ tprefix) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int64_t n = 0;
    for (int g = 0; g < G; g++) {
        tprefix[g] = n;
        n += (goff[g + 1] - goff[g] + kBgRows - 1) / kBgRows;
    }
    tprefix[G] = n;
}

// Weight (row, col) of a layer as float64 (code times its block scale).
__device__ __forceinline__ double layer_value(const void *w, const float *s, int prec, int width, int row, int col) {
    if (prec == GTMOE_FLOAT64) return ((const double *)w)[(int64_t)row * width + col];
    if (prec == GTMOE_FLOAT32) return (double)((const float *)w)[(int64_t)row * width + col];
    const double sc = (double)s[(int64_t)row * scale_blocks(width) + col / kValuesPerScale];
    if (prec == GTMOE_INT8) return sc * (double)((const int8_t *)w)[(int64_t)row * width + col];
    const uint8_t byte = ((const uint8_t *)w)[(int64_t)row * fp4_row_bytes(width) + col / 2];
    return sc * (double)fp4_value((col & 1) ? (byte >> 4) : (byte & 15u));
}

struct BgArgs {
    const ExpertLayers *experts;  // shared experts first, then routed
    int prec, S, k, d, h, clamped;
    double limit;
    int64_t T;
    const int64_t *wrow, *goff, *tprefix;
    int G;                 // groups: S + E
    const double *x;       // T x d, the Forward's input rows
    const double *dout;    // T x d
    const double *gates;   // T x k
    double *pg, *pu;       // n_rows x h, by work row
    double *rows_y;        // T*k x d
    double *rows_dx;       // n_rows x d
};

// One tile of kBgRows rows (one group) x kBgCols outputs of stage MODE.
template <int MODE>
__global__ void __launch_bounds__(kBgThreads) bwd_gemm_kernel(const BgArgs a) {
    constexpr bool kDual = MODE == 0 || MODE == 3;  // two weight layers (gate and up)
    constexpr bool kNT = MODE == 0 || MODE == 1;    // W indexed [output][input]
    const int K = (MODE == 0 || MODE == 2) ? a.d : a.h;
    const int N = (MODE == 0 || MODE == 2) ? a.h : a.d;
    __shared__ double sa[kDual && MODE == 3 ? 2 : 1][kBgRows][kBgK + 1];
    __shared__ double sb[kDual ? 2 : 1][kBgK][kBgCols + 1];
    __shared__ int64_t srow[kBgRows];
    const int64_t tile = blockIdx.x;
    if (tile >= a.tprefix[a.G]) return;
    int lo = 0, hi = a.G;  // the group of this tile: last g with tprefix[g] <= tile
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (a.tprefix[mid] <= tile) lo = mid;
        else hi = mid;
    }
    const int g = lo;
    if (MODE == 1 && g < a.S) return;  // the expert outputs are needed for routed rows only
    const int64_t n_shared = (int64_t)a.S * a.T;
    const int64_t r0 = (tile - a.tprefix[g]) * kBgRows;
    const int64_t n_g = a.goff[g + 1] - a.goff[g];
    const int n0 = blockIdx.y * kBgCols;
    if (threadIdx.x < kBgRows) {
        const int64_t i = r0 + threadIdx.x;
        srow[threadIdx.x] = i < n_g ? a.wrow[a.goff[g] + i] : -1;
    }
    const ExpertLayers &L = a.experts[g];
    __syncthreads();
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // outputs 4 tx .. 4 tx + 3, rows 4 ty .. 4 ty + 3
    double acc[kDual ? 2 : 1][4][4];
#pragma unroll
    for (int l = 0; l < (kDual ? 2 : 1); l++)
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[l][i][j] = 0.0;
    for (int k0 = 0; k0 < K; k0 += kBgK) {
        for (int e = threadIdx.x; e < kBgRows * kBgK; e += kBgThreads) {
            const int rr = e / kBgK, kk = e % kBgK;
            const int64_t r = srow[rr];
            const int kc = k0 + kk;
            double v0 = 0.0, v1 = 0.0;
            if (r >= 0 && kc < K) {
                const int64_t t = r < n_shared ? r % a.T : (r - n_shared) / a.k;
                if (MODE == 0) {
                    v0 = a.x[t * a.d + kc];
                } else if (MODE == 1) {
                    v0 = gate_act<double>(a.pg[r * a.h + kc], a.clamped, a.limit) *
                         up_act<double>(a.pu[r * a.h + kc], a.clamped, a.limit);
                } else if (MODE == 2) {
                    const double g0 = a.dout[t * a.d + kc];
                    v0 = r < n_shared ? g0 : g0 * a.gates[r - n_shared];  // vectormath.Scale for routed rows
                } else {
                    v0 = a.pg[r * a.h + kc];
                    v1 = a.pu[r * a.h + kc];
                }
            }
            sa[0][rr][kk] = v0;
            if (MODE == 3) sa[MODE == 3 ? 1 : 0][rr][kk] = v1;
        }
        for (int e = threadIdx.x; e < kBgK * kBgCols; e += kBgThreads) {
            // coalesced along the layer rows: inputs fastest for [output][input], outputs fastest otherwise
            const int kk = kNT ? e % kBgK : e / kBgCols, nn = kNT ? e / kBgK : e % kBgCols;
            const int kc = k0 + kk, nc = n0 + nn;
            double w0 = 0.0, w1 = 0.0;
            if (kc < K && nc < N) {
                if (MODE == 0) {
                    w0 = layer_value(L.w[0], L.s[0], a.prec, a.d, nc, kc);
                    w1 = layer_value(L.w[1], L.s[1], a.prec, a.d, nc, kc);
                } else if (MODE == 1) {
                    w0 = layer_value(L.w[2], L.s[2], a.prec, a.h, nc, kc);
                } else if (MODE == 2) {
                    w0 = layer_value(L.w[2], L.s[2], a.prec, a.h, kc, nc);
                } else {
                    w0 = layer_value(L.w[0], L.s[0], a.prec, a.d, kc, nc);
                    w1 = layer_value(L.w[1], L.s[1], a.prec, a.d, kc, nc);
                }
            }
            sb[0][kk][nn] = w0;
            if (kDual) sb[kDual ? 1 : 0][kk][nn] = w1;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kBgK; kk++) {
            double av[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) av[i] = sa[0][4 * ty + i][kk];
#pragma unroll
            for (int j = 0; j < 4; j++) b[j] = sb[0][kk][4 * tx + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[0][i][j] = fma(av[i], b[j], acc[0][i][j]);
            if (kDual) {
                if (MODE == 3)
#pragma unroll
                    for (int i = 0; i < 4; i++) av[i] = sa[MODE == 3 ? 1 : 0][4 * ty + i][kk];
#pragma unroll
                for (int j = 0; j < 4; j++) b[j] = sb[kDual ? 1 : 0][kk][4 * tx + j];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 4; j++) acc[kDual ? 1 : 0][i][j] = fma(av[i], b[j], acc[kDual ? 1 : 0][i][j]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int64_t r = srow[4 * ty + i];
        if (r < 0) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int n = n0 + 4 * tx + j;
            if (n >= N) continue;
            if (MODE == 0) {
                a.pg[r * a.h + n] = acc[0][i][j] + (L.b64[0] ? L.b64[0][n] : 0.0);
                a.pu[r * a.h + n] = acc[kDual ? 1 : 0][i][j] + (L.b64[1] ? L.b64[1][n] : 0.0);
            } else if (MODE == 1) {
                a.rows_y[(r - n_shared) * a.d + n] = acc[0][i][j] + (L.b64[2] ? L.b64[2][n] : 0.0);
            } else if (MODE == 2) {
                // the linear down layer's derivative is 1; then the gate / up
                // pre-activation gradients, in place of the pre-activations
                const double dh = acc[0][i][j];
                const double pg = a.pg[r * a.h + n], pu = a.pu[r * a.h + n];
                const double go = gate_act<double>(pg, a.clamped, a.limit);
                const double uo = up_act<double>(pu, a.clamped, a.limit);
                a.pg[r * a.h + n] = (dh * uo) * gate_deriv(pg, a.clamped, a.limit);
                a.pu[r * a.h + n] = (dh * go) * up_deriv(pu, a.clamped, a.limit);
            } else {
                a.rows_dx[r * a.d + n] = acc[0][i][j] + acc[kDual ? 1 : 0][i][j];
            }
        }
    }
}

// Per token, the chosen experts' router logits in float64 (DotProduct,
// inputs ascending, then the bias), their affinities and the gates as
// Forward forms them (mixtureofexperts.go:154-169): the affinity total over
// the chosen experts in order, gate i = affinity i / total.  (The forward's
// gates come from tensor-core logits, exact only where the selection needed
// it; the backward uses the reference's values.)
__global__ void bwd_gates_kernel(const double *__restrict__ x, const double *__restrict__ wr,
                                 const double *__restrict__ br, const int32_t *__restrict__ chosen, int64_t T, int d,
                                 int k, double *__restrict__ logit, double *__restrict__ aff,
                                 double *__restrict__ gate) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    const double *xr = x + t * d;
    double total = 0;
    for (int i = 0; i < k; i++) {
        const int e = chosen[t * k + i];
        double z = 0;
        for (int c = 0; c < d; c++) z += xr[c] * wr[(int64_t)e * d + c];
        z += br[e];
        const double a = sqrt(softplus_d(z));
        logit[t * k + i] = z;
        aff[t * k + i] = a;
        total += a;
    }
    for (int i = 0; i < k; i++) gate[t * k + i] = aff[t * k + i] / total;
}

// Router term per token: the gate gradients and the logit gradients (T x k).
__global__ void bwd_router_kernel(const double *__restrict__ logit, const double *__restrict__ aff,
                                  const double *__restrict__ gates, const double *__restrict__ dout,
                                  const double *__restrict__ rows_y, int64_t T, int d, int k,
                                  double *__restrict__ lg) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    const double *gr = dout + t * d;
    double gate_grad[kMaxTopK];
    double weighted = 0, total = 0;
    for (int i = 0; i < k; i++) {
        const double *yr = rows_y + (t * k + i) * d;
        double gg = 0;
        for (int c = 0; c < d; c++) gg += gr[c] * yr[c];
        gate_grad[i] = gg;
        weighted += gg * gates[t * k + i];
        total += aff[t * k + i];
    }
    for (int i = 0; i < k; i++) {
        const double ag = (gate_grad[i] - weighted) / total;
        lg[t * k + i] = ag * (sigmoid_d(logit[t * k + i]) / (2 * aff[t * k + i]));
    }
}

// dx per (token, input): shared experts' rows summed in order from zero, the
// routed rows added in ascending expert order, then the router's input
// gradient (experts ascending; only chosen experts have nonzero logit
// gradients) added to the total.
template <typename OT>
__global__ void bwd_dx_kernel(const double *__restrict__ rows_dx, const double *__restrict__ lg,
                              const int32_t *__restrict__ chosen, const double *__restrict__ wr, int64_t T, int d,
                              int S, int k, int router, OT *__restrict__ dx) {
    const int64_t n = T * d;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = p / d;
        const int c = (int)(p % d);
        double v = 0;
        for (int s = 0; s < S; s++) v = v + rows_dx[((int64_t)s * T + t) * d + c];
        for (int i = 0; i < k; i++) v += rows_dx[((int64_t)S * T + t * k + i) * d + c];
        if (router) {
            double rg = 0;
            for (int i = 0; i < k; i++) {
                const double g = lg[t * k + i];
                if (g != 0) rg += g * wr[(int64_t)chosen[t * k + i] * d + c];
            }
            v = v + rg;
        }
        dx[p] = from_double<OT>(v);
    }
}

// RouterLayer.Backward parameter gradients: bias[e] += each token's logit
// gradient in token order; weight[e][c] += (sum over tokens ascending of
// logit gradient * x[t][c]), the tokens of expert e from the Forward's
// expert-sorted lists (token-ascending).
__global__ void bwd_router_params_kernel(const double *__restrict__ lg, const double *__restrict__ x,
                                         const int32_t *__restrict__ chosen, const int32_t *__restrict__ perm,
                                         const int64_t *__restrict__ offsets, int E, int d, int k,
                                         double *__restrict__ wgrad, double *__restrict__ bgrad) {
    const int64_t n = (int64_t)E * d;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n; p += (int64_t)gridDim.x * blockDim.x) {
        const int e = (int)(p / d);
        const int c = (int)(p % d);
        double acc = 0, bacc = bgrad ? bgrad[e] : 0.0;
        for (int64_t q = offsets[e]; q < offsets[e + 1]; q++) {
            const int64_t t = perm[q];
            int i = 0;
            while (i < k && chosen[t * k + i] != e) i++;
            const double g = lg[t * k + i];
            if (c == 0) bacc += g;
            if (g != 0) acc += g * x[t * d + c];
        }
        if (wgrad) wgrad[p] += acc;
        if (c == 0 && bgrad) bgrad[e] = bacc;
    }
}

__global__ void to_f64_kernel(const void *__restrict__ src, int dtype, int64_t n, double *__restrict__ dst) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = load_as_double(src, dtype, i);
}

unsigned grid_for(int64_t n, int threads) {
    const int64_t b = (n + threads - 1) / threads;
    return (unsigned)(b < 1 ? 1 : b > 65535 ? 65535 : b);
}

}  // namespace

int save_training_state(gtmoe_handle *h, const void *x_dev, int x_dtype, int64_t T) {
    const gtmoe_config &c = h->cfg;
    cudaStream_t st = h->stream;
    const int d = c.d_model, k = c.experts_per_token, E = c.n_routed;
    h->tr_valid = 0;
    h->tr_T = T;
    if (T > 0) {
        GT_CHECK(h->tr_x.ensure(sizeof(double) * (size_t)T * d));
        GT_CHECK(h->tr_chosen.ensure(sizeof(int32_t) * (size_t)T * k));
        GT_CHECK(h->tr_gates.ensure(sizeof(double) * (size_t)T * k));
        GT_CHECK(h->tr_perm.ensure(sizeof(int32_t) * (size_t)T * k));
        GT_CHECK(h->tr_offsets.ensure(sizeof(int64_t) * (E + 1)));
        to_f64_kernel<<<grid_for(T * d, 256), 256, 0, st>>>(x_dev, x_dtype, T * d, h->tr_x.as<double>());
        GT_CUDA(cudaGetLastError());
        note_launches(1);
        GT_CUDA(cudaMemcpyAsync(h->tr_chosen.p, h->chosen.p, sizeof(int32_t) * T * k, cudaMemcpyDeviceToDevice, st));
        GT_CUDA(cudaMemcpyAsync(h->tr_gates.p, h->gates64.p, sizeof(double) * T * k, cudaMemcpyDeviceToDevice, st));
        GT_CUDA(cudaMemcpyAsync(h->tr_perm.p, h->perm.p, sizeof(int32_t) * T * k, cudaMemcpyDeviceToDevice, st));
        GT_CUDA(cudaMemcpyAsync(h->tr_offsets.p, h->offsets.p, sizeof(int64_t) * (E + 1), cudaMemcpyDeviceToDevice,
                                st));
    }
    h->tr_valid = 1;
    return 0;
}

void release_training_state(gtmoe_handle *h) {
    DevBuf *bufs[] = {&h->tr_x,    &h->tr_chosen, &h->tr_gates, &h->tr_perm, &h->tr_offsets, &h->bw_in,
                      &h->bw_dout, &h->bw_dx,     &h->bw_rows,  &h->bw_y,    &h->bw_lg,      &h->bw_zag,
                      &h->bw_rw,   &h->bw_rb,     &h->bw_work,  &h->bw_pgpu};
    for (DevBuf *b : bufs) b->release();
    h->tr_valid = 0;
}

}  // namespace gtmoe

using namespace gtmoe;

extern "C" {

int gtmoe_set_training(gtmoe_t h, int on) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    if (on && h->n_ranks > 1) return fail(GTMOE_EINVAL, "training state is kept on one GPU (not expert parallel)");
    if (on) {
        // the backward reads the layers in the RowsSnapshot layout
        GT_CUDA(cudaSetDevice(h->device));
        for (auto &L : h->layers) GT_CHECK(tc_restore_raw(h, L));
        GT_CUDA(cudaStreamSynchronize(h->stream));
    }
    h->training = on ? 1 : 0;
    if (!on) h->tr_valid = 0;
    return 0;
}

int gtmoe_backward(gtmoe_t h, const void *dout, int dout_dtype, void *dx, int dx_dtype, double *router_weight_grad,
                   double *router_bias_grad) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    if (h->n_ranks > 1) return fail(GTMOE_EINVAL, "gtmoe_backward runs on one GPU");
    if (!h->training || !h->tr_valid)
        return fail(GTMOE_ENOTREADY, "mixture of experts: call Forward (with training on) before Backward");
    if (dout_dtype < GTMOE_DTYPE_F64 || dout_dtype > GTMOE_DTYPE_BF16 || dx_dtype < GTMOE_DTYPE_F64 ||
        dx_dtype > GTMOE_DTYPE_BF16)
        return fail(GTMOE_EINVAL, "unknown dtype");
    const gtmoe_config &c = h->cfg;
    const int64_t T = h->tr_T;
    const int d = c.d_model, hd = c.hidden, k = c.experts_per_token, E = c.n_routed, S = c.n_shared;
    if (T > 0 && (!dout || !dx)) return fail(GTMOE_EINVAL, "mixture of experts: dout and dx must be given");
    if (T == 0) return 0;
    GT_CUDA(cudaSetDevice(h->device));
    GT_CHECK(refresh_table(h));
    cudaStream_t st = h->stream;
    const bool router = !c.hash_routing;

    // output gradients as float64 on the device
    const size_t in_bytes = dtype_size(dout_dtype) * (size_t)T * d;
    const void *dout_dev = dout;
    if (!is_device_ptr(dout)) {
        GT_CHECK(upload(h->bw_in, dout, in_bytes, st));
        dout_dev = h->bw_in.p;
    }
    GT_CHECK(h->bw_dout.ensure(sizeof(double) * (size_t)T * d));
    to_f64_kernel<<<grid_for(T * d, 256), 256, 0, st>>>(dout_dev, dout_dtype, T * d, h->bw_dout.as<double>());
    GT_CUDA(cudaGetLastError());

    const int64_t n_rows = (int64_t)S * T + T * k;
    GT_CHECK(h->bw_rows.ensure(sizeof(double) * (size_t)n_rows * d));
    GT_CHECK(h->bw_y.ensure(sizeof(double) * (size_t)T * k * d));
    GT_CHECK(h->bw_lg.ensure(sizeof(double) * (size_t)T * k));
    GT_CHECK(h->bw_zag.ensure(3 * sizeof(double) * (size_t)T * k));
    double *zl = h->bw_zag.as<double>(), *za = zl + T * k, *zg = za + T * k;
    if (router) {
        bwd_gates_kernel<<<grid_for(T, 128), 128, 0, st>>>(h->tr_x.as<double>(), h->wr64.as<double>(),
                                                            h->br.as<double>(), h->tr_chosen.as<int32_t>(), T, d, k,
                                                            zl, za, zg);
        GT_CUDA(cudaGetLastError());
    }

    BwdArgs a;
    a.experts = h->table.as<ExpertLayers>();
    a.prec = c.weight_precision;
    a.S = S;
    a.k = k;
    a.d = d;
    a.h = hd;
    a.clamped = c.clamped;
    a.limit = c.clamp_limit;
    a.T = T;
    a.x = h->tr_x.as<double>();
    a.chosen = h->tr_chosen.as<int32_t>();
    a.gates = router ? zg : h->tr_gates.as<double>();  // hash routing: 1/k from Forward
    a.dout = h->bw_dout.as<double>();
    a.rows_dx = h->bw_rows.as<double>();
    a.rows_y = h->bw_y.as<double>();
    // the experts' part as four grouped float64 GEMM stages over the work
    // rows taken expert by expert (see bwd_gemm_kernel)
    const int G = S + E;
    GT_CHECK(h->bw_work.ensure(sizeof(int64_t) * ((size_t)n_rows + 2 * (size_t)(G + 1))));
    GT_CHECK(h->bw_pgpu.ensure(2 * sizeof(double) * (size_t)n_rows * hd));
    int64_t *wrow = h->bw_work.as<int64_t>(), *goff = wrow + n_rows, *tprefix = goff + G + 1;
    {
        int64_t n = (int64_t)S * T > T * k ? (int64_t)S * T : T * k;
        n = n > G + 1 ? n : G + 1;
        bwd_worklist_kernel<<<grid_for(n, 256), 256, 0, st>>>(a.chosen, h->tr_perm.as<int32_t>(),
                                                               h->tr_offsets.as<int64_t>(), T, k, S, E, wrow, goff);
        GT_CUDA(cudaGetLastError());
        bwd_tiles_kernel<<<1, 32, 0, st>>>(goff, G, tprefix);
        GT_CUDA(cudaGetLastError());
    }
    BgArgs b;
    b.experts = a.experts;
    b.prec = a.prec;
    b.S = S;
    b.k = k;
    b.d = d;
    b.h = hd;
    b.clamped = a.clamped;
    b.limit = a.limit;
    b.T = T;
    b.wrow = wrow;
    b.goff = goff;
    b.tprefix = tprefix;
    b.G = G;
    b.x = a.x;
    b.dout = a.dout;
    b.gates = a.gates;
    b.pg = h->bw_pgpu.as<double>();
    b.pu = b.pg + (size_t)n_rows * hd;
    b.rows_y = a.rows_y;
    b.rows_dx = a.rows_dx;
    const unsigned tiles_ub = (unsigned)(n_rows / kBgRows + G);
    const dim3 grid_h(tiles_ub, (unsigned)((hd + kBgCols - 1) / kBgCols));
    const dim3 grid_d(tiles_ub, (unsigned)((d + kBgCols - 1) / kBgCols));
    bwd_gemm_kernel<0><<<grid_h, kBgThreads, 0, st>>>(b);
    GT_CUDA(cudaGetLastError());
    if (router) {
        bwd_gemm_kernel<1><<<grid_d, kBgThreads, 0, st>>>(b);
        GT_CUDA(cudaGetLastError());
    }
    bwd_gemm_kernel<2><<<grid_h, kBgThreads, 0, st>>>(b);
    GT_CUDA(cudaGetLastError());
    bwd_gemm_kernel<3><<<grid_d, kBgThreads, 0, st>>>(b);
    GT_CUDA(cudaGetLastError());
    note_launches(router ? 6 : 5);
    if (router) {
        bwd_router_kernel<<<grid_for(T, 128), 128, 0, st>>>(zl, za, zg, a.dout, a.rows_y, T, d, k,
                                                             h->bw_lg.as<double>());
        GT_CUDA(cudaGetLastError());
    }

    // dx (device, in dx_dtype)
    const size_t out_bytes = dtype_size(dx_dtype) * (size_t)T * d;
    void *dx_dev = dx;
    const bool dx_host = !is_device_ptr(dx);
    if (dx_host) {
        GT_CHECK(h->bw_dx.ensure(out_bytes));
        dx_dev = h->bw_dx.p;
    }
    const unsigned gdx = grid_for(T * d, 256);
    const double *lg = h->bw_lg.as<double>();
    const double *wr = h->wr64.as<double>();
    if (dx_dtype == GTMOE_DTYPE_F64)
        bwd_dx_kernel<double><<<gdx, 256, 0, st>>>(a.rows_dx, lg, a.chosen, wr, T, d, S, k, router, (double *)dx_dev);
    else if (dx_dtype == GTMOE_DTYPE_F32)
        bwd_dx_kernel<float><<<gdx, 256, 0, st>>>(a.rows_dx, lg, a.chosen, wr, T, d, S, k, router, (float *)dx_dev);
    else
        bwd_dx_kernel<__nv_bfloat16><<<gdx, 256, 0, st>>>(a.rows_dx, lg, a.chosen, wr, T, d, S, k, router,
                                                           (__nv_bfloat16 *)dx_dev);
    GT_CUDA(cudaGetLastError());
    note_launches(router ? 5 : 3);

    // router parameter gradients, added to the caller's
    if (router && (router_weight_grad || router_bias_grad)) {
        double *wg = router_weight_grad, *bg = router_bias_grad;
        const bool wg_host = wg && !is_device_ptr(wg), bg_host = bg && !is_device_ptr(bg);
        if (wg_host) {
            GT_CHECK(upload(h->bw_rw, wg, sizeof(double) * (size_t)E * d, st));
            wg = h->bw_rw.as<double>();
        }
        if (bg_host) {
            GT_CHECK(upload(h->bw_rb, bg, sizeof(double) * E, st));
            bg = h->bw_rb.as<double>();
        }
        bwd_router_params_kernel<<<grid_for((int64_t)E * d, 256), 256, 0, st>>>(
            lg, a.x, a.chosen, h->tr_perm.as<int32_t>(), h->tr_offsets.as<int64_t>(), E, d, k, wg, bg);
        GT_CUDA(cudaGetLastError());
        note_launches(1);
        if (wg_host)
            GT_CUDA(cudaMemcpyAsync(router_weight_grad, wg, sizeof(double) * (size_t)E * d, cudaMemcpyDeviceToHost,
                                    st));
        if (bg_host) GT_CUDA(cudaMemcpyAsync(router_bias_grad, bg, sizeof(double) * E, cudaMemcpyDeviceToHost, st));
    }
    if (dx_host) GT_CUDA(cudaMemcpyAsync(dx, dx_dev, out_bytes, cudaMemcpyDeviceToHost, st));
    GT_CUDA(cudaStreamSynchronize(st));
    return 0;
}

}  // extern "C"
