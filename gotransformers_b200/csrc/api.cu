// api.cu -- the C ABI of libgtmoe.so (include/gtmoe.h): handles, weight
// upload, and the Forward orchestration
//   router -> dispatch -> gather -> grouped SwiGLU -> combine
// of MixtureOfExperts.Forward (mixtureofexperts/mixtureofexperts.go:122-216).
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "handle.h"

namespace gtmoe {

static thread_local char g_error[2048];

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
    return code;
}

static std::atomic<int64_t> g_launches{0};
void note_launches(int n) { g_launches += n; }
int64_t launches_so_far() { return g_launches.load(); }

bool is_device_ptr(const void *p) {
    if (!p) return false;
    cudaPointerAttributes at;
    cudaError_t e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

static size_t precision_bytes(int precision, int64_t rows, int width) {
    switch (precision) {
    case GTMOE_FLOAT64: return (size_t)rows * width * 8;
    case GTMOE_FLOAT32: return (size_t)rows * width * 4;
    case GTMOE_INT8: return (size_t)rows * width;
    default: return (size_t)rows * fp4_row_bytes(width);
    }
}

}  // namespace gtmoe

using namespace gtmoe;

int gtmoe_handle::phase_begin(int p) {
    if (!timing) return 0;
    if (tev_used == tev.size()) {
        PhaseEvents pe;
        for (int i = 0; i < GTMOE_N_PHASES; i++) {
            GT_CUDA(cudaEventCreate(&pe.start[i]));
            GT_CUDA(cudaEventCreate(&pe.stop[i]));
        }
        tev.push_back(pe);
    }
    GT_CUDA(cudaEventRecord(tev[tev_used].start[p], stream));
    return 0;
}

int gtmoe_handle::phase_end(int p) {
    if (!timing) return 0;
    GT_CUDA(cudaEventRecord(tev[tev_used].stop[p], stream));
    return 0;
}

namespace gtmoe {

int layer_index(const gtmoe_handle *h, int kind, int index, int which) {
    if (kind == GTMOE_SHARED) return 3 * index + which;
    return 3 * h->slot_of[index] + which;
}

static int validate_config(const gtmoe_config *c) {
    if (!c) return fail(GTMOE_EINVAL, "config is NULL");
    if (c->d_model < 1 || c->hidden < 1)
        return fail(GTMOE_EINVAL, "NewMixtureOfExperts: needs d_model >= 1 and hidden >= 1, got %d and %d",
                    c->d_model, c->hidden);
    if (c->n_shared < 0)
        return fail(GTMOE_EINVAL, "NewMixtureOfExperts: number of shared experts can't be negative, got %d",
                    c->n_shared);
    if (c->n_routed < 1)
        return fail(GTMOE_EINVAL, "NewMixtureOfExperts: needs at least 1 routed expert, got %d", c->n_routed);
    if (c->experts_per_token < 1 || c->experts_per_token > c->n_routed)
        return fail(GTMOE_EINVAL, "NewMixtureOfExperts: experts per token must be between 1 and %d, got %d",
                    c->n_routed, c->experts_per_token);
    if (c->clamped && !(c->clamp_limit > 0))
        return fail(GTMOE_EINVAL, "NewClampedSwiGLU: limit must be above 0, got %g", c->clamp_limit);
    if (c->weight_precision < GTMOE_FLOAT64 || c->weight_precision > GTMOE_FP4)
        return fail(GTMOE_EINVAL, "unknown precision %d", c->weight_precision);
    if (c->n_routed > kMaxRoutedExperts)
        return fail(GTMOE_EINVAL, "this build supports at most %d routed experts, got %d", kMaxRoutedExperts,
                    c->n_routed);
    if (c->experts_per_token > kMaxTopK)
        return fail(GTMOE_EINVAL, "this build supports at most %d experts per token, got %d", kMaxTopK,
                    c->experts_per_token);
    return 0;
}

static int open_device(int device) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(GTMOE_ENODEVICE, "no CUDA device: %s", e == cudaSuccess ? "count is 0" : cudaGetErrorString(e));
    }
    if (device < 0 || device >= n) return fail(GTMOE_ENODEVICE, "device %d does not exist (%d devices)", device, n);
    cudaDeviceProp p;
    GT_CUDA(cudaGetDeviceProperties(&p, device));
    if (p.major != 10)
        return fail(GTMOE_ENODEVICE, "device %d is sm_%d%d; libgtmoe.so is built for sm_100a only", device, p.major,
                    p.minor);
    GT_CUDA(cudaSetDevice(device));
    return 0;
}

int create_handle(const gtmoe_config *cfg, int device, int n_ranks, int rank, gtmoe_t *out) {
    if (!out) return fail(GTMOE_EINVAL, "out is NULL");
    *out = nullptr;
    GT_CHECK(validate_config(cfg));
    GT_CHECK(open_device(device));
    if (n_ranks < 1 || rank < 0 || rank >= n_ranks || cfg->n_routed % n_ranks != 0)
        return fail(GTMOE_EINVAL, "%d routed experts cannot be split evenly over %d ranks (rank %d)", cfg->n_routed,
                    n_ranks, rank);
    gtmoe_handle *h = new gtmoe_handle();
    h->cfg = *cfg;
    h->device = device;
    h->n_ranks = n_ranks;
    h->rank = rank;
    h->e_local = cfg->n_routed / n_ranks;
    h->e_begin = rank * h->e_local;
    h->layers.resize((size_t)3 * (cfg->n_shared + h->e_local));
    h->slot_of.assign(cfg->n_routed, -1);
    h->routed_of_slot.assign(cfg->n_shared + h->e_local, -1);
    h->replicated.assign(cfg->n_routed, 0);
    for (int i = 0; i < h->e_local; i++) {
        h->slot_of[h->e_begin + i] = cfg->n_shared + i;
        h->routed_of_slot[cfg->n_shared + i] = h->e_begin + i;
    }
    // test switches, read once per handle: GTMOE_DISABLE_TC sends every batch
    // to the SIMT kernels and the float32 router, GTMOE_DISABLE_DECODE sends
    // small batches to the prefill kernels (the parity tests compare paths)
    h->no_tc = getenv("GTMOE_DISABLE_TC") != nullptr;
    h->no_decode = getenv("GTMOE_DISABLE_DECODE") != nullptr;
    h->h_bal.assign(cfg->n_routed, 0.0);
    cudaError_t e = cudaStreamCreateWithFlags(&h->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete h;
        return fail(GTMOE_ECUDA, "cudaStreamCreate failed: %s", cudaGetErrorString(e));
    }
    h->stream = h->own_stream;
    int rc = h->bal.ensure(sizeof(double) * cfg->n_routed);
    if (rc == 0) rc = cudaMemset(h->bal.p, 0, sizeof(double) * cfg->n_routed) == cudaSuccess ? 0 : GTMOE_ECUDA;
    if (rc != 0) {
        gtmoe_destroy(h);
        return rc;
    }
    *out = h;
    return 0;
}

int upload(DevBuf &dst, const void *src, size_t bytes, cudaStream_t st) {
    GT_CHECK(dst.ensure(bytes));
    if (bytes) GT_CUDA(cudaMemcpyAsync(dst.p, src, bytes, cudaMemcpyDefault, st));
    return 0;
}

static int to_host(std::vector<char> &buf, const void *src, size_t bytes) {
    buf.resize(bytes);
    if (bytes) GT_CUDA(cudaMemcpy(buf.data(), src, bytes, cudaMemcpyDefault));
    return 0;
}

// Decodes RowsSnapshot arrays to float64 exactly as Rows.Row does
// (lowprecision/rows.go:87-119).
static void decode_rows_host(int precision, int rows, int width, const void *values, const float *scales,
                             double *out) {
    int blocks = scale_blocks(width);
    for (int r = 0; r < rows; r++)
        for (int i = 0; i < width; i++) {
            double v;
            size_t o = (size_t)r * width + i;
            switch (precision) {
            case GTMOE_FLOAT64: v = ((const double *)values)[o]; break;
            case GTMOE_FLOAT32: v = (double)((const float *)values)[o]; break;
            case GTMOE_INT8: v = (double)((const int8_t *)values)[o] * (double)scales[(size_t)r * blocks + i / 16]; break;
            default: {
                uint8_t b = ((const uint8_t *)values)[(size_t)r * fp4_row_bytes(width) + i / 2];
                int c = (i & 1) ? (b >> 4) : (b & 15);
                static const double mag[8] = {0, 0.5, 1, 1.5, 2, 3, 4, 6};
                double m = mag[c & 7] * (double)scales[(size_t)r * blocks + i / 16];
                v = (c & 8) ? -m : m;
            }
            }
            out[o] = v;
        }
}

// bf16 round-to-nearest-even of a float, and back.
static uint16_t bf16_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static double bf16_value(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return (double)f;
}

static int all_layers_set(const gtmoe_handle *h) {
    for (size_t i = 0; i < h->layers.size(); i++)
        if (!h->layers[i].set) {
            int S = h->cfg.n_shared;
            int e = (int)(i / 3);
            const char *which = (i % 3 == 0) ? "gate" : (i % 3 == 1) ? "up" : "down";
            if (e < S) return fail(GTMOE_ENOTREADY, "shared expert %d %s layer is not set", e, which);
            return fail(GTMOE_ENOTREADY, "routed expert %d %s layer is not set", h->routed_of_slot[e], which);
        }
    if (!h->cfg.hash_routing && !h->router_set) return fail(GTMOE_ENOTREADY, "router weights are not set");
    return 0;
}

int refresh_table(gtmoe_handle *h) {
    if (!h->table_dirty) return 0;
    int n = (int)(h->layers.size() / 3);
    std::vector<ExpertLayers> t(n);
    for (int e = 0; e < n; e++)
        for (int w = 0; w < 3; w++) {
            LayerDev &L = h->layers[3 * e + w];
            t[e].w[w] = L.w.p;
            t[e].s[w] = L.s.as<float>();
            t[e].b32[w] = L.has_bias ? L.b32.as<float>() : nullptr;
            t[e].b64[w] = L.has_bias ? L.b64.as<double>() : nullptr;
            t[e].tiled[w] = L.tiled.as<uint8_t>();
        }
    GT_CHECK(h->table.ensure(sizeof(ExpertLayers) * n));
    GT_CUDA(cudaMemcpy(h->table.p, t.data(), sizeof(ExpertLayers) * n, cudaMemcpyHostToDevice));
    GT_CHECK(tc_prepare(h, h->tc));
    h->table_dirty = 0;
    return 0;
}

// Single-GPU forward on device-resident x (x_dev) producing device out.
static int forward_prepare(gtmoe_handle *h, int64_t T);
// Host-buffer batches from this many rows on are pipelined in chunks.
constexpr int64_t kPipelineMinRows = 16384;
constexpr int kMaxPipeChunks = 4;

__global__ void add_load_kernel(int64_t *__restrict__ acc, const int64_t *__restrict__ load, int E) {
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < E; e += gridDim.x * blockDim.x) acc[e] += load[e];
}

// A large batch in host memory, as chunks: chunk c+1's input copy and chunk
// c-1's output copy (their own streams) run while chunk c computes.  Rows are
// independent, so the outputs equal one whole-batch forward's; the per-expert
// load is summed over the chunks (LastExpertLoad sees the whole batch).
static int forward_pipelined(gtmoe_handle *h, const void *x, int x_dtype, int64_t T, const int64_t *ids_dev,
                             const void *res_dev, void *out, int out_dtype, int32_t *chosen, double *gates,
                             int64_t *load, int nc) {
    const gtmoe_config &c = h->cfg;
    const int d = c.d_model, k = c.experts_per_token, E = c.n_routed;
    cudaStream_t st = h->stream;
    const size_t xrow = dtype_size(x_dtype) * d, orow = dtype_size(out_dtype) * d;
    // chunk bounds: the first and the last chunk are the smaller ones (a
    // quarter of the batch each for 3 chunks, an eighth for 4), since only
    // their copies are not hidden behind another chunk's compute
    int64_t bound[kMaxPipeChunks + 1];
    nc = nc < 2 ? 2 : nc > kMaxPipeChunks ? kMaxPipeChunks : nc;
    const int64_t edge = nc == 2 ? (T + 1) / 2 : T / (nc == 3 ? 4 : 8);
    bound[0] = 0;
    bound[nc] = T;
    for (int ci = 1; ci < nc; ci++)
        bound[ci] = ci == 1 ? edge : ci == nc - 1 ? T - edge : edge + (T - 2 * edge) * (ci - 1) / (nc - 2);
    int64_t Tc = 0;
    for (int ci = 0; ci < nc; ci++) Tc = bound[ci + 1] - bound[ci] > Tc ? bound[ci + 1] - bound[ci] : Tc;
    if (!h->h2d_stream) GT_CUDA(cudaStreamCreateWithFlags(&h->h2d_stream, cudaStreamNonBlocking));
    if (!h->d2h_stream) GT_CUDA(cudaStreamCreateWithFlags(&h->d2h_stream, cudaStreamNonBlocking));
    for (cudaEvent_t &e : h->pipe_ev)
        if (!e) GT_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    for (int s = 0; s < 2; s++) {
        GT_CHECK(h->x_pipe[s].ensure(xrow * (size_t)Tc));
        GT_CHECK(h->out_pipe[s].ensure(orow * (size_t)Tc));
    }
    GT_CHECK(h->load_acc.ensure(sizeof(int64_t) * E));
    GT_CHECK(forward_prepare(h, Tc));
    GT_CUDA(cudaMemsetAsync(h->load_acc.p, 0, sizeof(int64_t) * E, st));
    // the side streams start after everything already queued on the handle's stream
    cudaEvent_t *x_ready = h->pipe_ev, *x_free = h->pipe_ev + 2, *out_ready = h->pipe_ev + 4,
                *out_free = h->pipe_ev + 6;
    GT_CUDA(cudaEventRecord(x_free[0], st));
    GT_CUDA(cudaStreamWaitEvent(h->h2d_stream, x_free[0], 0));
    GT_CUDA(cudaStreamWaitEvent(h->d2h_stream, x_free[0], 0));
    for (int ci = 0; ci < nc; ci++) {
        const int64_t t0 = bound[ci];
        const int64_t n = bound[ci + 1] - t0;
        if (n <= 0) continue;
        const int s = ci & 1;
        if (ci >= 2) GT_CUDA(cudaStreamWaitEvent(h->h2d_stream, x_free[s], 0));
        GT_CUDA(cudaMemcpyAsync(h->x_pipe[s].p, (const char *)x + t0 * xrow, n * xrow, cudaMemcpyHostToDevice,
                                h->h2d_stream));
        GT_CUDA(cudaEventRecord(x_ready[s], h->h2d_stream));
        GT_CUDA(cudaStreamWaitEvent(st, x_ready[s], 0));
        if (ci >= 2) GT_CUDA(cudaStreamWaitEvent(st, out_free[s], 0));
        GT_CHECK(forward_device(h, h->x_pipe[s].p, x_dtype, n, ids_dev ? ids_dev + t0 : nullptr,
                                res_dev ? (const char *)res_dev + t0 * orow : nullptr, h->out_pipe[s].p, out_dtype));
        GT_CUDA(cudaEventRecord(x_free[s], st));
        add_load_kernel<<<1, 256, 0, st>>>(h->load_acc.as<int64_t>(), h->load.as<int64_t>(), E);
        GT_CUDA(cudaGetLastError());
        note_launches(1);
        // the next chunk overwrites the routing workspace: copy this chunk's now
        if (chosen) GT_CUDA(cudaMemcpyAsync(chosen + t0 * k, h->chosen.p, sizeof(int32_t) * n * k, cudaMemcpyDefault, st));
        if (gates) GT_CUDA(cudaMemcpyAsync(gates + t0 * k, h->gates64.p, sizeof(double) * n * k, cudaMemcpyDefault, st));
        GT_CUDA(cudaEventRecord(out_ready[s], st));
        GT_CUDA(cudaStreamWaitEvent(h->d2h_stream, out_ready[s], 0));
        GT_CUDA(cudaMemcpyAsync((char *)out + t0 * orow, h->out_pipe[s].p, n * orow, cudaMemcpyDeviceToHost,
                                h->d2h_stream));
        GT_CUDA(cudaEventRecord(out_free[s], h->d2h_stream));
    }
    // the whole batch's load where LastExpertLoad and UpdateBalance read it
    GT_CUDA(cudaMemcpyAsync(h->load.p, h->load_acc.p, sizeof(int64_t) * E, cudaMemcpyDeviceToDevice, st));
    if (load) GT_CUDA(cudaMemcpyAsync(load, h->load.p, sizeof(int64_t) * E, cudaMemcpyDefault, st));
    GT_CUDA(cudaStreamSynchronize(h->d2h_stream));
    GT_CUDA(cudaStreamSynchronize(st));
    GT_CHECK(tc_check_error(h->tc));
    h->last_T = T;
    h->have_load = 1;
    return 0;
}

// Workspace of a T-row forward on one GPU (grow-only; no-op when it fits).
static int forward_prepare(gtmoe_handle *h, int64_t T) {
    const gtmoe_config &c = h->cfg;
    const int E = c.n_routed, k = c.experts_per_token, S = c.n_shared, d = c.d_model, hd = c.hidden;
    const bool use_tc = tc_supported(h, T);
    const int compute = c.weight_precision == GTMOE_FLOAT64 ? GTMOE_DTYPE_F64
                        : use_tc                            ? GTMOE_DTYPE_BF16
                                                            : GTMOE_DTYPE_F32;
    const size_t cs = dtype_size(compute);
    const int64_t TK = T * k;
    const int64_t rows_x = (S > 0 ? T : 0) + TK;
    const int64_t rows_h = (int64_t)S * T + TK;
    const int n_chunks = (int)((T + kDispatchChunk - 1) / kDispatchChunk);
    // the logits, then ||x_t|| of a few-token batch
    GT_CHECK(h->logits.ensure(sizeof(double) * ((size_t)T * E + (size_t)std::min<int64_t>(T, kRouterSmallMaxT))));
    GT_CHECK(h->chosen.ensure(sizeof(int32_t) * (size_t)TK));
    GT_CHECK(h->gates64.ensure(sizeof(double) * (size_t)TK));
    GT_CHECK(h->gates32.ensure(sizeof(float) * (size_t)TK));
    GT_CHECK(h->counts.ensure(sizeof(int32_t) * (size_t)(n_chunks > 0 ? n_chunks : 1) * E));
    GT_CHECK(h->load.ensure(sizeof(int64_t) * E));
    GT_CHECK(h->offsets.ensure(sizeof(int64_t) * (E + 1)));
    GT_CHECK(h->perm.ensure(sizeof(int32_t) * (size_t)TK));
    GT_CHECK(h->slot_row.ensure(sizeof(int64_t) * (size_t)TK));
    GT_CHECK(h->groups.ensure(sizeof(Group) * (S + E)));
    GT_CHECK(h->tile_prefix.ensure(sizeof(int64_t) * (S + E + 1)));
    GT_CHECK(h->xp.ensure(cs * (size_t)rows_x * d));
    GT_CHECK(h->hp.ensure(cs * (size_t)rows_h * hd));
    GT_CHECK(h->yp.ensure(cs * (size_t)rows_h * d));
    GT_CHECK(h->fixups.ensure(sizeof(int)));
    GT_CHECK(h->flagged.ensure(sizeof(int) * (size_t)(T > 0 ? T : 1)));
    GT_CHECK(refresh_table(h));
    return 0;
}

// Arguments and every device address a captured forward bakes in.
static std::vector<uint64_t> graph_key(gtmoe_handle *h, const void *x, int x_dtype, int64_t T, const void *res,
                                       void *out, int out_dtype) {
    uint64_t wbits;
    memcpy(&wbits, &h->wmax, sizeof(wbits));
    const bool use_tc = tc_supported(h, T);
    const bool use_decode = use_tc && decode_usable(h->cfg.weight_precision, h->cfg.d_model, h->cfg.hidden, T,
                                                      h->cfg.n_shared + h->cfg.n_routed) &&
                            !h->no_decode;
    std::vector<uint64_t> k = {(uint64_t)(uintptr_t)x, (uint64_t)x_dtype, (uint64_t)T, (uint64_t)(uintptr_t)res,
                               (uint64_t)(uintptr_t)out, (uint64_t)out_dtype, (uint64_t)(uintptr_t)h->stream, wbits,
                               (uint64_t)h->e_pad, (uint64_t)use_tc, (uint64_t)use_decode,
                               (uint64_t)(uintptr_t)h->tc.err, (uint64_t)(uintptr_t)h->gather_bf16,
                               (uint64_t)(uintptr_t)h->router_bf16_mid, (uint64_t)(uintptr_t)h->router_bf16_lo};
    const gtmoe::DevBuf *bufs[] = {&h->wr64,   &h->wr32,   &h->br,     &h->bal,    &h->wr3,   &h->table,
                                   &h->logits, &h->chosen, &h->gates64, &h->gates32, &h->counts, &h->load,
                                   &h->offsets, &h->perm,  &h->slot_row, &h->groups, &h->tile_prefix, &h->xp,
                                   &h->hp,     &h->yp,     &h->fixups, &h->flagged};
    for (const gtmoe::DevBuf *b : bufs) k.push_back((uint64_t)(uintptr_t)b->p);
    return k;
}

// forward_device, or its CUDA-graph replay when this call repeats the last
// one exactly (same arguments and workspace): a decode loop calls the mixture
// once per token with the same buffers, and replaying the dozen small launches
// as one graph takes the host's launch cost off the GPU's timeline.
static int run_forward(gtmoe_handle *h, bool graphable, const void *x_dev, int x_dtype, int64_t T,
                       const int64_t *ids_dev, const void *res_dev, void *out_dev, int out_dtype) {
    if (!graphable || !h->graphs || h->timing || T == 0) {
        h->drop_graph();
        return forward_device(h, x_dev, x_dtype, T, ids_dev, res_dev, out_dev, out_dtype);
    }
    GT_CHECK(forward_prepare(h, T));  // every allocation happens outside a capture
    std::vector<uint64_t> key = graph_key(h, x_dev, x_dtype, T, res_dev, out_dev, out_dtype);
    if (key != h->gkey) {
        h->drop_graph();
        h->gkey = key;
        return forward_device(h, x_dev, x_dtype, T, ids_dev, res_dev, out_dev, out_dtype);
    }
    if (!h->gexec) {
        // second identical call: capture it, then replay from now on
        const int64_t before = launches_so_far();
        GT_CUDA(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
        int rc = forward_device(h, x_dev, x_dtype, T, ids_dev, res_dev, out_dev, out_dtype);
        cudaGraph_t graph = nullptr;
        cudaError_t e = cudaStreamEndCapture(h->stream, &graph);
        if (rc != 0 || e != cudaSuccess) {
            if (graph) cudaGraphDestroy(graph);
            cudaGetLastError();
            h->drop_graph();
            if (rc != 0) return rc;
            return fail(GTMOE_ECUDA, "stream capture of the forward failed: %s", cudaGetErrorString(e));
        }
        h->glaunches = launches_so_far() - before;
        e = cudaGraphInstantiate(&h->gexec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) {
            h->gexec = nullptr;
            h->drop_graph();
            return fail(GTMOE_ECUDA, "cudaGraphInstantiate failed: %s", cudaGetErrorString(e));
        }
    } else {
        note_launches((int)h->glaunches);
    }
    GT_CUDA(cudaGraphLaunch(h->gexec, h->stream));
    h->last_T = T;
    h->have_load = 1;
    return 0;
}

int forward_device(gtmoe_handle *h, const void *x_dev, int x_dtype, int64_t T, const int64_t *ids_dev,
                   const void *res_dev, void *out_dev, int out_dtype) {
    const gtmoe_config &c = h->cfg;
    const int E = c.n_routed, k = c.experts_per_token, S = c.n_shared, d = c.d_model, hd = c.hidden;
    cudaStream_t st = h->stream;
    const bool use_tc = tc_supported(h, T);
    // few rows per expert: stream the weights (decode.cu) instead of 256-row tiles
    const bool use_decode =
        use_tc && decode_usable(c.weight_precision, d, hd, T, S + E) && !h->no_decode;
    const int compute = c.weight_precision == GTMOE_FLOAT64 ? GTMOE_DTYPE_F64
                        : use_tc                            ? GTMOE_DTYPE_BF16
                                                            : GTMOE_DTYPE_F32;
    const size_t cs = dtype_size(compute);
    const int64_t TK = T * k;
    const int64_t rows_x = (S > 0 ? T : 0) + TK;
    const int64_t rows_h = (int64_t)S * T + TK;

    GT_CHECK(forward_prepare(h, T));

    RouterArgs ra;
    ra.hash = c.hash_routing;
    ra.x = x_dev;
    ra.x_dtype = x_dtype;
    ra.T = T;
    ra.E = E;
    ra.k = k;
    ra.d = d;
    ra.token_ids = ids_dev;
    ra.w32 = h->wr32.as<float>();
    ra.w64 = h->wr64.as<double>();
    ra.bias = h->br.as<double>();
    ra.balance = h->bal.as<double>();
    ra.use_tc = !c.hash_routing && h->wr3.p && !h->no_tc && router_tc_usable(x_dev, x_dtype, T, d);
    double router_err = ra.use_tc ? kRouterTcErr : kRouterSimtErr;
    // float64 rows that come with their three-term bf16 split (the block
    // step): logits on the tensor cores from the terms, with the split's margin
    if (!ra.use_tc && !c.hash_routing && h->wr3.p && !h->no_tc && x_dtype == GTMOE_DTYPE_F64 && h->gather_bf16 &&
        h->router_bf16_mid && h->router_bf16_lo && router_tc_usable(h->gather_bf16, GTMOE_DTYPE_BF16, T, d) &&
        router_tc_usable(h->router_bf16_mid, GTMOE_DTYPE_BF16, T, d) &&
        router_tc_usable(h->router_bf16_lo, GTMOE_DTYPE_BF16, T, d)) {
        ra.use_tc = 1;
        ra.x_tc = h->gather_bf16;
        ra.x_tc_mid = h->router_bf16_mid;
        ra.x_tc_lo = h->router_bf16_lo;
        router_err = kRouterTc3Err;
    }
    ra.thresh_scale = router_err * h->wmax;
    ra.w3 = h->wr3.p;
    ra.e_pad = h->e_pad;
    ra.err = h->tc.err;
    ra.sms = h->tc.sms;
    ra.logits = h->logits.as<double>();
    ra.xnorm = ra.logits + (size_t)T * E;
    ra.chosen = h->chosen.as<int32_t>();
    ra.gates64 = h->gates64.as<double>();
    ra.gates32 = h->gates32.as<float>();
    ra.n_fixups = h->fixups.as<int>();
    ra.flagged = h->flagged.as<int>();

    DispatchArgs da;
    da.T = T;
    da.E = E;
    da.k = k;
    da.S = S;
    da.chosen = ra.chosen;
    da.chunk_counts = h->counts.as<int32_t>();
    da.load = h->load.as<int64_t>();
    da.offsets = h->offsets.as<int64_t>();
    da.perm = h->perm.as<int32_t>();
    da.slot_row = h->slot_row.as<int64_t>();
    da.groups = h->groups.as<Group>();
    da.tile_prefix = h->tile_prefix.as<int64_t>();
    da.bm = use_decode ? decode_tile_rows(T) : use_tc ? tc_tile_rows(h->tc) : kSimtBM;
    ra.dispatch = &da;  // a small batch's router runs the dispatch too (its phase then holds both)

    GT_CHECK(h->phase_begin(0));
    GT_CHECK(launch_router(ra, st));
    GT_CHECK(h->phase_end(0));
    if (!router_fuses_dispatch(ra)) {
        GT_CHECK(h->phase_begin(1));
        GT_CHECK(launch_dispatch(da, st));
        GT_CHECK(h->phase_end(1));
    }

    GT_CHECK(h->phase_begin(2));
    const bool bf16_rows = h->gather_bf16 && compute == GTMOE_DTYPE_BF16;
    GT_CHECK(launch_gather(bf16_rows ? h->gather_bf16 : x_dev, bf16_rows ? GTMOE_DTYPE_BF16 : x_dtype, T, d,
                           da.slot_row, k, S > 0 ? T : 0, S > 0, h->xp.p, compute, st));
    GT_CHECK(h->phase_end(2));

    if (use_decode) {
        DecodeArgs dc;
        dc.groups = da.groups;
        dc.tile_prefix = da.tile_prefix;
        dc.n_groups = S + E;
        dc.experts = h->table.as<ExpertLayers>();
        dc.d = d;
        dc.h = hd;
        dc.precision = c.weight_precision;
        dc.clamped = c.clamped;
        dc.clamp_limit = c.clamp_limit;
        dc.xp = h->xp.p;
        dc.hp = h->hp.p;
        dc.yp = h->yp.p;
        dc.sms = h->tc.sms;
        dc.tile_rows = decode_tile_rows(T);
        dc.max_tiles = decode_max_tiles(T, E, k, S, dc.tile_rows);
        dc.err = h->tc.err;
        GT_CHECK(h->phase_begin(3));
        GT_CHECK(launch_decode(dc, 1, st));
        GT_CHECK(h->phase_end(3));
        GT_CHECK(h->phase_begin(4));
        GT_CHECK(launch_decode(dc, 2, st));
        GT_CHECK(h->phase_end(4));
    } else if (use_tc) {
        TcArgs ta;
        ta.n_groups = S + E;
        ta.groups = da.groups;
        ta.tile_prefix = da.tile_prefix;
        ta.rows_x = rows_x;
        ta.rows_h = rows_h;
        ta.xp = h->xp.p;
        ta.hp = h->hp.p;
        ta.yp = h->yp.p;
        GT_CHECK(launch_grouped_tc(h, h->tc, ta, st));  // records phases 3 and 4
    } else {
        GroupedArgs ga;
        ga.precision = c.weight_precision;
        ga.compute = compute;
        ga.n_groups = S + E;
        ga.groups = da.groups;
        ga.tile_prefix = da.tile_prefix;
        ga.experts = h->table.as<ExpertLayers>();
        ga.d = d;
        ga.h = hd;
        ga.clamped = c.clamped;
        ga.clamp_limit = c.clamp_limit;
        ga.xp = h->xp.p;
        ga.hp = h->hp.p;
        ga.yp = h->yp.p;
        GT_CHECK(h->phase_begin(3));
        if (T > 0) GT_CHECK(launch_grouped_simt(ga, 1, st));
        GT_CHECK(h->phase_end(3));
        GT_CHECK(h->phase_begin(4));
        if (T > 0) GT_CHECK(launch_grouped_simt(ga, 2, st));
        GT_CHECK(h->phase_end(4));
    }

    CombineArgs ca;
    ca.T = T;
    ca.d = d;
    ca.k = k;
    ca.S = S;
    ca.y = h->yp.p;
    ca.y_dtype = compute;
    ca.shared_row0 = 0;
    ca.routed_row0 = (int64_t)S * T;
    ca.slot_row = da.slot_row;
    ca.gates32 = ra.gates32;
    ca.gates64 = ra.gates64;
    ca.residual = res_dev;
    ca.out = out_dev;
    ca.out_dtype = out_dtype;
    GT_CHECK(h->phase_begin(5));
    GT_CHECK(launch_combine(ca, st));
    GT_CHECK(h->phase_end(5));
    if (h->timing) h->tev_used++;
    h->last_T = T;
    h->have_load = 1;
    return 0;
}

}  // namespace gtmoe

extern "C" {

int gtmoe_version(void) { return GTMOE_VERSION; }

const char *gtmoe_last_error(void) { return g_error; }

int gtmoe_create(const gtmoe_config *cfg, int device, gtmoe_t *out) {
    g_error[0] = 0;
    return create_handle(cfg, device, 1, 0, out);
}

void gtmoe_destroy(gtmoe_t h) {
    if (!h) return;
    {
        std::lock_guard<std::mutex> lock(h->mu);
        cudaSetDevice(h->device);
        if (h->stream) cudaStreamSynchronize(h->stream);
        h->drop_graph();
        ep_destroy(h);
        tc_release(h->tc);
        for (auto &L : h->layers) {
            L.tiled.release();
            L.w.release();
            L.s.release();
            L.b32.release();
            L.b64.release();
        }
        DevBuf *bufs[] = {&h->wr64, &h->wr32, &h->wr3, &h->br, &h->bal, &h->table, &h->x_in, &h->ids, &h->logits,
                          &h->chosen, &h->gates64, &h->gates32, &h->counts, &h->load, &h->offsets, &h->perm,
                          &h->slot_row, &h->groups, &h->tile_prefix, &h->xp, &h->hp, &h->yp, &h->out_dev,
                          &h->res_dev, &h->fixups, &h->flagged, &h->x_pipe[0], &h->x_pipe[1], &h->out_pipe[0],
                          &h->out_pipe[1], &h->load_acc, &h->norm_w, &h->block_x, &h->block_xn,
                          &h->block_xn16};
        for (DevBuf *b : bufs) b->release();
        release_training_state(h);
        for (cudaEvent_t e : h->pipe_ev)
            if (e) cudaEventDestroy(e);
        if (h->h2d_stream) cudaStreamDestroy(h->h2d_stream);
        if (h->d2h_stream) cudaStreamDestroy(h->d2h_stream);
        for (auto &pe : h->tev)
            for (int i = 0; i < GTMOE_N_PHASES; i++) {
                cudaEventDestroy(pe.start[i]);
                cudaEventDestroy(pe.stop[i]);
            }
        if (h->own_stream) cudaStreamDestroy(h->own_stream);
    }
    delete h;
}

int gtmoe_set_stream(gtmoe_t h, void *stream) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    h->stream = stream ? (cudaStream_t)stream : h->own_stream;
    return 0;
}

int gtmoe_set_graphs(gtmoe_t h, int on) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    GT_CUDA(cudaSetDevice(h->device));
    h->graphs = on ? 1 : 0;
    if (!on) h->drop_graph();
    return 0;
}

int gtmoe_set_router(gtmoe_t h, int precision, const void *values, const float *scales, const double *bias) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    GT_CUDA(cudaSetDevice(h->device));
    const int E = h->cfg.n_routed, d = h->cfg.d_model;
    if (precision < GTMOE_FLOAT64 || precision > GTMOE_FP4) return fail(GTMOE_EINVAL, "unknown precision %d", precision);
    if (!values) return fail(GTMOE_EINVAL, "router values are NULL");
    if ((precision == GTMOE_INT8 || precision == GTMOE_FP4) && !scales)
        return fail(GTMOE_EINVAL, "compressed router needs scales");
    std::vector<char> hv, hs, hb;
    GT_CHECK(to_host(hv, values, precision_bytes(precision, E, d)));
    if (scales) GT_CHECK(to_host(hs, scales, sizeof(float) * (size_t)E * scale_blocks(d)));
    std::vector<double> w64((size_t)E * d);
    decode_rows_host(precision, E, d, hv.data(), (const float *)hs.data(), w64.data());
    std::vector<float> w32(w64.size());
    double wmax = 0;
    for (int e = 0; e < E; e++) {
        double ss = 0;
        for (int i = 0; i < d; i++) {
            double v = w64[(size_t)e * d + i];
            ss += v * v;
            w32[(size_t)e * d + i] = (float)v;
        }
        wmax = fmax(wmax, sqrt(ss));
    }
    std::vector<double> b(E, 0.0);
    if (bias) {
        GT_CHECK(to_host(hb, bias, sizeof(double) * E));
        memcpy(b.data(), hb.data(), sizeof(double) * E);
    }
    // bf16 split w = hi + mid + lo (+ residual below 2^-24 |w|) for the
    // tensor-core router, rows padded with zeros to a multiple of 128
    const int e_pad = (E + 127) / 128 * 128;
    std::vector<uint16_t> w3((size_t)3 * e_pad * d, 0);
    for (int e = 0; e < E; e++)
        for (int i = 0; i < d; i++) {
            double r = w64[(size_t)e * d + i];
            for (int t = 0; t < 3; t++) {
                uint16_t b = bf16_bits((float)r);
                w3[((size_t)t * e_pad + e) * d + i] = b;
                r -= bf16_value(b);
            }
        }
    GT_CHECK(upload(h->wr3, w3.data(), sizeof(uint16_t) * w3.size(), h->stream));
    h->e_pad = e_pad;
    GT_CHECK(upload(h->wr64, w64.data(), sizeof(double) * w64.size(), h->stream));
    GT_CHECK(upload(h->wr32, w32.data(), sizeof(float) * w32.size(), h->stream));
    GT_CHECK(upload(h->br, b.data(), sizeof(double) * E, h->stream));
    GT_CUDA(cudaStreamSynchronize(h->stream));
    h->wmax = wmax * (1 + 1e-6);
    h->router_set = 1;
    return 0;
}

int gtmoe_set_balance(gtmoe_t h, const double *balance) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    if (!balance) return fail(GTMOE_EINVAL, "balance is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    GT_CUDA(cudaSetDevice(h->device));
    std::vector<char> hb;
    GT_CHECK(to_host(hb, balance, sizeof(double) * h->cfg.n_routed));
    memcpy(h->h_bal.data(), hb.data(), sizeof(double) * h->cfg.n_routed);
    GT_CHECK(upload(h->bal, h->h_bal.data(), sizeof(double) * h->cfg.n_routed, h->stream));
    GT_CUDA(cudaStreamSynchronize(h->stream));
    return 0;
}

int gtmoe_get_balance(gtmoe_t h, double *balance) {
    if (!h || !balance) return fail(GTMOE_EINVAL, "handle or balance is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    GT_CUDA(cudaSetDevice(h->device));
    GT_CUDA(cudaMemcpy(balance, h->h_bal.data(), sizeof(double) * h->cfg.n_routed, cudaMemcpyDefault));
    return 0;
}

int gtmoe_set_expert_layer(gtmoe_t h, int kind, int index, int which, int precision, const void *values,
                           const float *scales, int rows, int width, const double *bias) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    GT_CUDA(cudaSetDevice(h->device));
    const gtmoe_config &c = h->cfg;
    if (kind == GTMOE_SHARED) {
        if (index < 0 || index >= c.n_shared)
            return fail(GTMOE_EINVAL, "shared expert %d does not exist (%d shared)", index, c.n_shared);
    } else if (kind == GTMOE_ROUTED) {
        if (index < 0 || index >= c.n_routed)
            return fail(GTMOE_EINVAL, "routed expert %d does not exist (%d routed)", index, c.n_routed);
        if (h->slot_of[index] < 0)
            return fail(GTMOE_EINVAL, "routed expert %d is not owned by rank %d (owns %d..%d) nor replicated on it",
                        index, h->rank, h->e_begin, h->e_begin + h->e_local - 1);
    } else {
        return fail(GTMOE_EINVAL, "kind must be GTMOE_SHARED or GTMOE_ROUTED, got %d", kind);
    }
    if (which < GTMOE_GATE || which > GTMOE_DOWN) return fail(GTMOE_EINVAL, "which must be gate, up or down");
    if (precision != c.weight_precision)
        return fail(GTMOE_EINVAL, "layer precision %d differs from the handle's weight precision %d", precision,
                    c.weight_precision);
    int want_rows = which == GTMOE_DOWN ? c.d_model : c.hidden;
    int want_width = which == GTMOE_DOWN ? c.hidden : c.d_model;
    if (rows != want_rows || width != want_width)
        return fail(GTMOE_EINVAL, "layer: got %dx%d compressed weights but it holds %dx%d", rows, width, want_rows,
                    want_width);
    if (!values) return fail(GTMOE_EINVAL, "values are NULL");
    if ((precision == GTMOE_INT8 || precision == GTMOE_FP4) && !scales)
        return fail(GTMOE_EINVAL, "Int8/FP4 layers need scales");
    LayerDev &L = h->layers[layer_index(h, kind, index, which)];
    GT_CHECK(upload(L.w, values, precision_bytes(precision, rows, width), h->stream));
    if (precision == GTMOE_INT8 || precision == GTMOE_FP4)
        GT_CHECK(upload(L.s, scales, sizeof(float) * (size_t)rows * scale_blocks(width), h->stream));
    L.has_bias = 0;
    if (bias) {
        std::vector<char> hb;
        GT_CHECK(to_host(hb, bias, sizeof(double) * rows));
        std::vector<float> b32(rows);
        const double *b = (const double *)hb.data();
        int nonzero = 0;
        for (int i = 0; i < rows; i++) {
            b32[i] = (float)b[i];
            nonzero |= b[i] != 0;
        }
        if (nonzero) {
            GT_CHECK(upload(L.b64, b, sizeof(double) * rows, h->stream));
            GT_CHECK(upload(L.b32, b32.data(), sizeof(float) * rows, h->stream));
            L.has_bias = 1;
        }
    }
    L.precision = precision;
    L.rows = rows;
    L.width = width;
    GT_CHECK(tc_relayout_layer(h, L, which));
    GT_CUDA(cudaStreamSynchronize(h->stream));
    // With the record copy built, the snapshot-layout copy is read only by the
    // SIMT kernels (which such a shape never runs unless the tensor cores are
    // switched off) and by the backward: drop it, halving the resident
    // weights; gtmoe_set_training rebuilds it from the records.
    L.raw_dropped = 0;
    if (L.tiled.p && !h->no_tc && !h->training) {
        L.w.release();
        L.s.release();
        L.raw_dropped = 1;
    }
    L.set = 1;
    h->table_dirty = 1;
    return 0;
}

int gtmoe_forward(gtmoe_t h, const void *x, int x_dtype, int64_t T, const int64_t *token_ids, const void *residual,
                  void *out, int out_dtype, int32_t *chosen, double *gates, int32_t *perm, int64_t *load) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    return forward_locked(h, x, x_dtype, T, token_ids, residual, out, out_dtype, chosen, gates, perm, load);
}

}  // extern "C"

namespace gtmoe {

int forward_locked(gtmoe_t h, const void *x, int x_dtype, int64_t T, const int64_t *token_ids, const void *residual,
                   void *out, int out_dtype, int32_t *chosen, double *gates, int32_t *perm, int64_t *load) {
    GT_CUDA(cudaSetDevice(h->device));
    const gtmoe_config &c = h->cfg;
    auto check_args = [&]() -> int {
        if (T < 0) return fail(GTMOE_EINVAL, "mixture of experts: negative number of rows %lld", (long long)T);
        if (T > 0 && (!x || !out)) return fail(GTMOE_EINVAL, "mixture of experts: x and out must be given");
        if (x_dtype < GTMOE_DTYPE_F64 || x_dtype > GTMOE_DTYPE_BF16 || out_dtype < GTMOE_DTYPE_F64 ||
            out_dtype > GTMOE_DTYPE_BF16)
            return fail(GTMOE_EINVAL, "unknown dtype");
        if (c.hash_routing && T > 0 && !token_ids)
            return fail(GTMOE_EINVAL,
                        "mixture of experts: hash routing needs one token ID per row, got none for %lld rows",
                        (long long)T);
        return all_layers_set(h);
    };
    const int arg_rc = check_args();
    // expert parallel: a rank whose arguments are wrong still joins the
    // step's count exchange, so that every rank fails instead of waiting
    if (h->n_ranks > 1)
        return ep_forward(h, x, x_dtype, T, token_ids, residual, out, out_dtype, chosen, gates, perm, load, arg_rc);
    if (arg_rc != 0) return arg_rc;

    cudaStream_t st = h->stream;
    const int d = c.d_model, k = c.experts_per_token, E = c.n_routed;
    const size_t xbytes = dtype_size(x_dtype) * (size_t)T * d;
    const size_t obytes = dtype_size(out_dtype) * (size_t)T * d;

    // a large batch in host memory runs as chunks whose copies overlap compute
    // (not with timing, a host residual, or the whole-batch permutation asked for)
    const bool pipelined = T >= kPipelineMinRows && !h->timing && !perm && !h->training && !is_device_ptr(x) &&
                           !is_device_ptr(out) && (!residual || is_device_ptr(residual));
    h->tr_valid = 0;  // a backward refers to the last Forward only

    const void *x_dev = x;
    if (T > 0 && !pipelined && !is_device_ptr(x)) {
        GT_CHECK(upload(h->x_in, x, xbytes, st));
        x_dev = h->x_in.p;
    }
    const int64_t *ids_dev = nullptr;
    if (c.hash_routing && T > 0) {
        std::vector<char> hid;
        GT_CHECK(to_host(hid, token_ids, sizeof(int64_t) * T));
        const int64_t *ids = (const int64_t *)hid.data();
        for (int64_t t = 0; t < T; t++)
            if (ids[t] < 0)
                return fail(GTMOE_EINVAL, "mixture of experts: token ID %lld at row %lld is negative",
                            (long long)ids[t], (long long)t);
        GT_CHECK(upload(h->ids, hid.data(), sizeof(int64_t) * T, st));
        ids_dev = h->ids.as<int64_t>();
    }
    const void *res_dev = residual;
    if (residual && T > 0 && !is_device_ptr(residual)) {
        GT_CHECK(upload(h->res_dev, residual, obytes, st));
        res_dev = h->res_dev.p;
    }
    void *out_dev = out;
    const bool out_host = T > 0 && !pipelined && !is_device_ptr(out);
    if (out_host) {
        GT_CHECK(h->out_dev.ensure(obytes));
        out_dev = h->out_dev.p;
    }
    if (pipelined) {
        h->drop_graph();
        return forward_pipelined(h, x, x_dtype, T, ids_dev, res_dev, out, out_dtype, chosen, gates, load,
                                 T >= 4 * kPipelineMinRows ? 4 : 3);
    }
    // device pointers only, no host round trip inside: the forward may be replayed as a CUDA graph
    const bool graphable = !c.hash_routing && x_dev == x && out_dev == out && res_dev == residual;
    GT_CHECK(run_forward(h, graphable, x_dev, x_dtype, T, ids_dev, res_dev, out_dev, out_dtype));
    if (h->training) GT_CHECK(save_training_state(h, x_dev, x_dtype, T));

    bool sync = out_host;
    const int64_t TK = T * k;
    if (out_host) GT_CUDA(cudaMemcpyAsync(out, out_dev, obytes, cudaMemcpyDeviceToHost, st));
    if (chosen && TK) {
        GT_CUDA(cudaMemcpyAsync(chosen, h->chosen.p, sizeof(int32_t) * TK, cudaMemcpyDefault, st));
        sync |= !is_device_ptr(chosen);
    }
    if (gates && TK) {
        GT_CUDA(cudaMemcpyAsync(gates, h->gates64.p, sizeof(double) * TK, cudaMemcpyDefault, st));
        sync |= !is_device_ptr(gates);
    }
    if (perm && TK) {
        GT_CUDA(cudaMemcpyAsync(perm, h->perm.p, sizeof(int32_t) * TK, cudaMemcpyDefault, st));
        sync |= !is_device_ptr(perm);
    }
    if (load) {
        GT_CUDA(cudaMemcpyAsync(load, h->load.p, sizeof(int64_t) * E, cudaMemcpyDefault, st));
        sync |= !is_device_ptr(load);
    }
    if (sync) {
        GT_CUDA(cudaStreamSynchronize(st));
        GT_CHECK(tc_check_error(h->tc));
    }
    return 0;
}

}  // namespace gtmoe

extern "C" {

int gtmoe_last_expert_load(gtmoe_t h, int64_t *load) {
    if (!h || !load) return fail(GTMOE_EINVAL, "handle or load is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    if (!h->have_load) return fail(GTMOE_ENOTREADY, "LastExpertLoad before the first Forward");
    GT_CUDA(cudaSetDevice(h->device));
    GT_CUDA(cudaMemcpyAsync(load, h->load.p, sizeof(int64_t) * h->cfg.n_routed, cudaMemcpyDefault, h->stream));
    GT_CUDA(cudaStreamSynchronize(h->stream));
    return 0;
}

int gtmoe_update_balance(gtmoe_t h, double rate) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    if (!h->have_load || h->cfg.hash_routing) return 0;
    GT_CUDA(cudaSetDevice(h->device));
    const int E = h->cfg.n_routed;
    std::vector<int64_t> load(E);
    GT_CHECK(ep_global_load(h, load.data()));
    int64_t total = 0;
    for (int e = 0; e < E; e++) total += load[e];
    double average = (double)total / (double)E;
    for (int e = 0; e < E; e++) {
        if ((double)load[e] < average) h->h_bal[e] += rate;
        if ((double)load[e] > average) h->h_bal[e] -= rate;
    }
    GT_CHECK(upload(h->bal, h->h_bal.data(), sizeof(double) * E, h->stream));
    GT_CUDA(cudaStreamSynchronize(h->stream));
    return 0;
}

int gtmoe_set_timing(gtmoe_t h, int enable) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    h->timing = enable != 0;
    h->tev_used = 0;
    h->launches_at_read = launches_so_far();
    return 0;
}

int gtmoe_read_timing(gtmoe_t h, double *ms, int n_phases, int64_t *calls, int64_t *kernel_launches) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    GT_CUDA(cudaSetDevice(h->device));
    GT_CUDA(cudaStreamSynchronize(h->stream));
    GT_CHECK(tc_check_error(h->tc));
    for (int p = 0; p < n_phases && p < GTMOE_N_PHASES; p++) {
        double total = 0;
        for (size_t i = 0; i < h->tev_used; i++) {
            float t = 0;
            cudaError_t e = cudaEventElapsedTime(&t, h->tev[i].start[p], h->tev[i].stop[p]);
            if (e == cudaSuccess) total += t;
            else cudaGetLastError();  // phase not recorded in this call
        }
        if (ms) ms[p] += total;
    }
    if (calls) *calls = (int64_t)h->tev_used;
    int64_t now = launches_so_far();
    if (kernel_launches) *kernel_launches = now - h->launches_at_read;
    h->launches_at_read = now;
    h->tev_used = 0;
    return 0;
}

int gtmoe_quantize_rows(int precision, const double *values, int64_t rows, int width, void *codes, float *scales) {
    if (precision < GTMOE_FLOAT64 || precision > GTMOE_FP4) return fail(GTMOE_EINVAL, "unknown precision %d", precision);
    if (width <= 0 || rows < 0) return fail(GTMOE_EINVAL, "NewRows: width must be at least 1, got %d", width);
    if (rows == 0) return 0;
    if (!values || !codes || ((precision == GTMOE_INT8 || precision == GTMOE_FP4) && !scales))
        return fail(GTMOE_EINVAL, "NULL pointer");
    int dev = 0;
    GT_CUDA(cudaGetDevice(&dev));
    GT_CHECK(open_device(dev));
    const size_t vbytes = sizeof(double) * (size_t)rows * width;
    const size_t cbytes = precision_bytes(precision, rows, width);
    const size_t sbytes = sizeof(float) * (size_t)rows * scale_blocks(width);
    DevBuf dv, dc, ds;
    const double *v = values;
    void *cd = codes;
    float *sd = scales;
    int rc = 0;
    if (!is_device_ptr(values)) {
        if ((rc = upload(dv, values, vbytes, 0))) goto done;
        v = dv.as<double>();
    }
    if (!is_device_ptr(codes)) {
        if ((rc = dc.ensure(cbytes))) goto done;
        cd = dc.p;
    }
    if (scales && !is_device_ptr(scales)) {
        if ((rc = ds.ensure(sbytes))) goto done;
        sd = ds.as<float>();
    }
    if ((rc = launch_quantize_rows(precision, v, rows, width, cd, sd, 0))) goto done;
    if (cd != codes && cudaMemcpy(codes, cd, cbytes, cudaMemcpyDeviceToHost) != cudaSuccess) rc = GTMOE_ECUDA;
    if (!rc && scales && sd != scales && (precision == GTMOE_INT8 || precision == GTMOE_FP4) &&
        cudaMemcpy(scales, sd, sbytes, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = GTMOE_ECUDA;
    if (!rc && cudaDeviceSynchronize() != cudaSuccess) rc = fail(GTMOE_ECUDA, "quantiser failed");
done:
    dv.release();
    dc.release();
    ds.release();
    return rc;
}

int gtmoe_fill_normal(void *dev, int dtype, int64_t n, uint64_t seed, uint64_t stream, int64_t offset,
                      double stddev) {
    if (n < 0 || (n > 0 && !dev)) return fail(GTMOE_EINVAL, "bad arguments");
    if (n > 0 && !is_device_ptr(dev)) return fail(GTMOE_EINVAL, "gtmoe_fill_normal writes device memory only");
    GT_CHECK(launch_fill_normal(dev, dtype, n, seed, stream, offset, stddev, 0));
    GT_CUDA(cudaDeviceSynchronize());
    return 0;
}

}  // extern "C"
