// ep.cu -- expert parallelism across GPUs (one process per GPU, NCCL).
//
// The reference runs MixtureOfExperts.Forward in one process
// (mixtureofexperts.go:122-216); BASELINE's config 5 shards its routed
// experts over 1-8 GPUs.  Per rank r of G (routed experts r*E/G .. (r+1)*E/G-1
// owned, router and shared experts replicated, tokens split by the caller):
//   1. route this rank's tokens (router.cu) and dispatch them over all E
//      experts (dispatch.cu): the stable permutation orders (token, slot)
//      rows by global expert, i.e. by destination rank, token-ascending;
//   2. gather those rows (send buffer), all-gather every rank's per-expert
//      counts (one G x E int64 exchange, one host synchronisation: message
//      sizes must be known on the host);
//   3. grouped ncclSend/ncclRecv of the rows; a segment copy regroups the
//      received rows expert-major (source-ascending inside an expert, so an
//      expert's rows are the reference's token order over the whole batch);
//   4. the grouped SwiGLU kernels (shared experts on this rank's tokens,
//      owned routed experts on the received rows);
//   5. the inverse segment copy and the reverse exchange bring every output
//      row back to its token's rank, where combine.cu adds them in the
//      reference's order.
// Remote rows always land in local buffers before any kernel reads them.
// NCCL is loaded at run time (dlopen), only when an expert-parallel handle is
// created.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <vector>

#include "handle.h"

namespace gtmoe {

namespace {

struct NcclApi {
    bool loaded = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *);
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*CommDestroy)(ncclComm_t);
    const char *(*GetErrorString)(ncclResult_t);
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
    ncclResult_t (*GroupStart)();
    ncclResult_t (*GroupEnd)();
};
NcclApi g_nccl;
std::mutex g_nccl_mu;

int load_nccl() {
    std::lock_guard<std::mutex> lock(g_nccl_mu);
    if (g_nccl.loaded) return 0;
    void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) return fail(GTMOE_ENCCL, "could not load libnccl.so.2: %s", dlerror());
    struct {
        const char *name;
        void **slot;
    } syms[] = {
        {"ncclGetUniqueId", (void **)&g_nccl.GetUniqueId},   {"ncclCommInitRank", (void **)&g_nccl.CommInitRank},
        {"ncclCommDestroy", (void **)&g_nccl.CommDestroy},   {"ncclGetErrorString", (void **)&g_nccl.GetErrorString},
        {"ncclAllGather", (void **)&g_nccl.AllGather},       {"ncclSend", (void **)&g_nccl.Send},
        {"ncclRecv", (void **)&g_nccl.Recv},                 {"ncclGroupStart", (void **)&g_nccl.GroupStart},
        {"ncclGroupEnd", (void **)&g_nccl.GroupEnd},
    };
    for (auto &s : syms) {
        *s.slot = dlsym(lib, s.name);
        if (!*s.slot) return fail(GTMOE_ENCCL, "libnccl.so.2 is missing %s", s.name);
    }
    g_nccl.loaded = true;
    return 0;
}

#define GT_NCCL(call)                                                                                      \
    do {                                                                                                   \
        ncclResult_t r_ = (call);                                                                          \
        if (r_ != ncclSuccess)                                                                             \
            return ::gtmoe::fail(GTMOE_ENCCL, "%s failed: %s", #call, g_nccl.GetErrorString(r_));          \
    } while (0)

// One contiguous block of rows moved between two buffers.
struct Segment {
    int64_t src_row, dst_row, rows;
};

__global__ void segment_copy_kernel(const uint4 *__restrict__ src, uint4 *__restrict__ dst,
                                    const Segment *__restrict__ segs, int n_segs, int vec_per_row) {
    for (int s = blockIdx.y; s < n_segs; s += gridDim.y) {
        const Segment g = segs[s];
        const int64_t n = g.rows * vec_per_row;
        const uint4 *a = src + g.src_row * vec_per_row;
        uint4 *b = dst + g.dst_row * vec_per_row;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
            b[i] = a[i];
    }
}

}  // namespace

struct EpState {
    ncclComm_t comm = nullptr;
    DevBuf gathered_load;  // G x E int64 (device)
    std::vector<int64_t> h_gathered;
    int have_gathered = 0;
    DevBuf sendbuf, recvbuf, yback, yret, segs_fwd, segs_back;
};

static EpState *ep_of(gtmoe_handle *h) { return (EpState *)h->ep; }

void ep_destroy(gtmoe_handle *h) {
    EpState *ep = ep_of(h);
    if (!ep) return;
    if (ep->comm && g_nccl.loaded) g_nccl.CommDestroy(ep->comm);
    DevBuf *bufs[] = {&ep->gathered_load, &ep->sendbuf, &ep->recvbuf, &ep->yback, &ep->yret, &ep->segs_fwd,
                      &ep->segs_back};
    for (DevBuf *b : bufs) b->release();
    delete ep;
    h->ep = nullptr;
}

static int segment_copy(const void *src, void *dst, const std::vector<Segment> &segs, DevBuf &table,
                        size_t row_bytes, cudaStream_t st) {
    if (segs.empty()) return 0;
    if (row_bytes % 16 != 0) return fail(GTMOE_EINVAL, "expert-parallel rows must be a multiple of 16 bytes");
    GT_CHECK(table.ensure(sizeof(Segment) * segs.size()));
    GT_CUDA(cudaMemcpyAsync(table.p, segs.data(), sizeof(Segment) * segs.size(), cudaMemcpyHostToDevice, st));
    dim3 grid(8, (unsigned)(segs.size() < 65535 ? segs.size() : 65535));
    segment_copy_kernel<<<grid, 256, 0, st>>>((const uint4 *)src, (uint4 *)dst, table.as<Segment>(), (int)segs.size(),
                                              (int)(row_bytes / 16));
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    // the host table must outlive the copy: wait for it before returning
    GT_CUDA(cudaStreamSynchronize(st));
    return 0;
}

int ep_global_load(gtmoe_handle *h, int64_t *load) {
    EpState *ep = ep_of(h);
    const int E = h->cfg.n_routed;
    if (!ep) {
        GT_CUDA(cudaMemcpyAsync(load, h->load.p, sizeof(int64_t) * E, cudaMemcpyDeviceToHost, h->stream));
        GT_CUDA(cudaStreamSynchronize(h->stream));
        return 0;
    }
    if (!ep->have_gathered) return fail(GTMOE_ENOTREADY, "no Forward yet");
    for (int e = 0; e < E; e++) {
        int64_t s = 0;
        for (int r = 0; r < h->n_ranks; r++) s += ep->h_gathered[(size_t)r * E + e];
        load[e] = s;
    }
    return 0;
}

int ep_forward(gtmoe_handle *h, const void *x, int x_dtype, int64_t T, const int64_t *token_ids, const void *residual,
               void *out, int out_dtype, int32_t *chosen_out, double *gates_out, int32_t *perm_out,
               int64_t *load_out) {
    EpState *ep = ep_of(h);
    const gtmoe_config &c = h->cfg;
    const int E = c.n_routed, k = c.experts_per_token, S = c.n_shared, d = c.d_model, hd = c.hidden;
    const int G = h->n_ranks, r = h->rank, El = h->e_local;
    cudaStream_t st = h->stream;
    const bool use_tc = tc_supported(h, 1);
    const int compute = c.weight_precision == GTMOE_FLOAT64 ? GTMOE_DTYPE_F64
                        : use_tc                            ? GTMOE_DTYPE_BF16
                                                            : GTMOE_DTYPE_F32;
    const size_t cs = dtype_size(compute);
    const size_t row_bytes = cs * d;
    const int64_t TK = T * k;
    const int n_chunks = (int)((T + kDispatchChunk - 1) / kDispatchChunk);

    // ---- inputs on the device
    const size_t xbytes = dtype_size(x_dtype) * (size_t)T * d;
    const size_t obytes = dtype_size(out_dtype) * (size_t)T * d;
    auto is_dev = [](const void *p) {
        cudaPointerAttributes at;
        if (!p || cudaPointerGetAttributes(&at, p) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
    };
    const void *x_dev = x;
    if (T > 0 && !is_dev(x)) {
        GT_CHECK(h->x_in.ensure(xbytes));
        GT_CUDA(cudaMemcpyAsync(h->x_in.p, x, xbytes, cudaMemcpyDefault, st));
        x_dev = h->x_in.p;
    }
    const int64_t *ids_dev = nullptr;
    if (c.hash_routing && T > 0) {
        std::vector<int64_t> hid(T);
        GT_CUDA(cudaMemcpy(hid.data(), token_ids, sizeof(int64_t) * T, cudaMemcpyDefault));
        for (int64_t t = 0; t < T; t++)
            if (hid[t] < 0)
                return fail(GTMOE_EINVAL, "mixture of experts: token ID %lld at row %lld is negative",
                            (long long)hid[t], (long long)t);
        GT_CHECK(h->ids.ensure(sizeof(int64_t) * T));
        GT_CUDA(cudaMemcpyAsync(h->ids.p, hid.data(), sizeof(int64_t) * T, cudaMemcpyHostToDevice, st));
        ids_dev = h->ids.as<int64_t>();
    }
    const void *res_dev = residual;
    if (residual && T > 0 && !is_dev(residual)) {
        GT_CHECK(h->res_dev.ensure(obytes));
        GT_CUDA(cudaMemcpyAsync(h->res_dev.p, residual, obytes, cudaMemcpyDefault, st));
        res_dev = h->res_dev.p;
    }
    void *out_dev = out;
    const bool out_host = T > 0 && !is_dev(out);
    if (out_host) {
        GT_CHECK(h->out_dev.ensure(obytes));
        out_dev = h->out_dev.p;
    }

    // ---- routing and dispatch over all E experts (this rank's tokens)
    GT_CHECK(h->logits.ensure(sizeof(double) * (size_t)(T > 0 ? T : 1) * E));
    GT_CHECK(h->chosen.ensure(sizeof(int32_t) * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(h->gates64.ensure(sizeof(double) * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(h->gates32.ensure(sizeof(float) * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(h->counts.ensure(sizeof(int32_t) * (size_t)(n_chunks > 0 ? n_chunks : 1) * E));
    GT_CHECK(h->load.ensure(sizeof(int64_t) * E));
    GT_CHECK(h->offsets.ensure(sizeof(int64_t) * (E + 1)));
    GT_CHECK(h->perm.ensure(sizeof(int32_t) * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(h->slot_row.ensure(sizeof(int64_t) * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(h->groups.ensure(sizeof(Group) * (S + E)));
    GT_CHECK(h->tile_prefix.ensure(sizeof(int64_t) * (S + E + 1)));
    GT_CHECK(h->fixups.ensure(sizeof(int)));
    GT_CHECK(h->flagged.ensure(sizeof(int) * (size_t)(T > 0 ? T : 1)));
    GT_CHECK(ep->gathered_load.ensure(sizeof(int64_t) * (size_t)G * E));
    GT_CHECK(ep->sendbuf.ensure(row_bytes * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(ep->yret.ensure(row_bytes * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(refresh_table(h));

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
    ra.use_tc = !c.hash_routing && h->wr3.p && router_tc_usable(x_dev, x_dtype, T, d);
    ra.thresh_scale = (ra.use_tc ? kRouterTcErr : kRouterSimtErr) * h->wmax;
    ra.w3 = h->wr3.p;
    ra.e_pad = h->e_pad;
    ra.err = h->tc.err;
    ra.sms = h->tc.sms;
    ra.logits = h->logits.as<double>();
    ra.chosen = h->chosen.as<int32_t>();
    ra.gates64 = h->gates64.as<double>();
    ra.gates32 = h->gates32.as<float>();
    ra.n_fixups = h->fixups.as<int>();
    ra.flagged = h->flagged.as<int>();
    GT_CHECK(h->phase_begin(0));
    GT_CHECK(launch_router(ra, st));
    GT_CHECK(h->phase_end(0));

    DispatchArgs da;
    da.T = T;
    da.E = E;
    da.k = k;
    da.S = 0;
    da.chosen = ra.chosen;
    da.chunk_counts = h->counts.as<int32_t>();
    da.load = h->load.as<int64_t>();
    da.offsets = h->offsets.as<int64_t>();
    da.perm = h->perm.as<int32_t>();
    da.slot_row = h->slot_row.as<int64_t>();
    da.groups = h->groups.as<Group>();
    da.tile_prefix = h->tile_prefix.as<int64_t>();
    da.bm = use_tc ? tc_tile_rows(h->tc) : kSimtBM;
    GT_CHECK(h->phase_begin(1));
    GT_CHECK(launch_dispatch(da, st));
    GT_CHECK(h->phase_end(1));

    // ---- send rows in global-expert order, and everybody's per-expert counts
    GT_CHECK(h->phase_begin(6));
    GT_CHECK(launch_gather(x_dev, x_dtype, T, d, da.perm, TK, 0, 0, ep->sendbuf.p, compute, st));
    GT_NCCL(g_nccl.AllGather(h->load.p, ep->gathered_load.p, (size_t)E, ncclInt64, ep->comm, st));
    ep->h_gathered.resize((size_t)G * E);
    GT_CUDA(cudaMemcpyAsync(ep->h_gathered.data(), ep->gathered_load.p, sizeof(int64_t) * G * E,
                            cudaMemcpyDeviceToHost, st));
    GT_CUDA(cudaStreamSynchronize(st));
    ep->have_gathered = 1;
    const int64_t *Lg = ep->h_gathered.data();  // Lg[s * E + e]: rows of rank s for expert e
    std::vector<int64_t> send_cnt(G, 0), send_off(G + 1, 0), recv_cnt(G, 0), recv_off(G + 1, 0), tot(El, 0),
        eoff(El + 1, 0);
    for (int q = 0; q < G; q++)
        for (int e = q * El; e < (q + 1) * El; e++) send_cnt[q] += Lg[(size_t)r * E + e];
    for (int s = 0; s < G; s++)
        for (int el = 0; el < El; el++) {
            const int64_t n = Lg[(size_t)s * E + r * El + el];
            recv_cnt[s] += n;
            tot[el] += n;
        }
    for (int q = 0; q < G; q++) send_off[q + 1] = send_off[q] + send_cnt[q];
    for (int s = 0; s < G; s++) recv_off[s + 1] = recv_off[s] + recv_cnt[s];
    for (int el = 0; el < El; el++) eoff[el + 1] = eoff[el] + tot[el];
    const int64_t n_recv = recv_off[G];
    const int64_t xbase = S > 0 ? T : 0;
    const int64_t rows_x = xbase + n_recv;
    const int64_t rows_h = (int64_t)S * T + n_recv;
    GT_CHECK(ep->recvbuf.ensure(row_bytes * (size_t)(n_recv > 0 ? n_recv : 1)));
    GT_CHECK(ep->yback.ensure(row_bytes * (size_t)(n_recv > 0 ? n_recv : 1)));
    GT_CHECK(h->xp.ensure(row_bytes * (size_t)(rows_x > 0 ? rows_x : 1)));
    GT_CHECK(h->hp.ensure(cs * (size_t)hd * (rows_h > 0 ? rows_h : 1)));
    GT_CHECK(h->yp.ensure(row_bytes * (size_t)(rows_h > 0 ? rows_h : 1)));

    GT_NCCL(g_nccl.GroupStart());
    for (int q = 0; q < G; q++)
        if (send_cnt[q] > 0)
            GT_NCCL(g_nccl.Send((const char *)ep->sendbuf.p + send_off[q] * row_bytes, send_cnt[q] * row_bytes,
                                ncclUint8, q, ep->comm, st));
    for (int s = 0; s < G; s++)
        if (recv_cnt[s] > 0)
            GT_NCCL(g_nccl.Recv((char *)ep->recvbuf.p + recv_off[s] * row_bytes, recv_cnt[s] * row_bytes, ncclUint8,
                                s, ep->comm, st));
    GT_NCCL(g_nccl.GroupEnd());

    // received [source][expert] -> expert-major, source-ascending
    std::vector<Segment> fwd, back;
    for (int el = 0; el < El; el++) {
        int64_t dst = eoff[el];
        for (int s = 0; s < G; s++) {
            int64_t src = recv_off[s];
            for (int e2 = 0; e2 < el; e2++) src += Lg[(size_t)s * E + r * El + e2];
            const int64_t n = Lg[(size_t)s * E + r * El + el];
            if (n > 0) {
                fwd.push_back({src, xbase + dst, n});
                back.push_back({(int64_t)S * T + dst, src, n});
            }
            dst += n;
        }
    }
    if (S > 0) GT_CHECK(launch_gather(x_dev, x_dtype, T, d, nullptr, 0, 0, 1, h->xp.p, compute, st));
    GT_CHECK(segment_copy(ep->recvbuf.p, h->xp.p, fwd, ep->segs_fwd, row_bytes, st));
    GT_CHECK(h->phase_end(6));

    // ---- group table of this rank: shared experts on its tokens, owned experts on received rows
    std::vector<Group> groups(S + El);
    std::vector<int64_t> prefix(S + El + 1, 0);
    const int bm = use_tc ? tc_tile_rows(h->tc) : kSimtBM;
    for (int s = 0; s < S; s++) groups[s] = Group{0, (int64_t)s * T, T, s, 0};
    for (int el = 0; el < El; el++) groups[S + el] = Group{xbase + eoff[el], (int64_t)S * T + eoff[el], tot[el], S + el, 0};
    for (int g = 0; g < S + El; g++) prefix[g + 1] = prefix[g] + (groups[g].m + bm - 1) / bm;
    GT_CUDA(cudaMemcpyAsync(h->groups.p, groups.data(), sizeof(Group) * (S + El), cudaMemcpyHostToDevice, st));
    GT_CUDA(cudaMemcpyAsync(h->tile_prefix.p, prefix.data(), sizeof(int64_t) * (S + El + 1), cudaMemcpyHostToDevice,
                            st));

    if (rows_h > 0) {
        if (use_tc) {
            TcArgs ta;
            ta.n_groups = S + El;
            ta.groups = h->groups.as<Group>();
            ta.tile_prefix = h->tile_prefix.as<int64_t>();
            ta.rows_x = rows_x;
            ta.rows_h = rows_h;
            ta.xp = h->xp.p;
            ta.hp = h->hp.p;
            ta.yp = h->yp.p;
            GT_CHECK(launch_grouped_tc(h, h->tc, ta, st));
        } else {
            GroupedArgs ga;
            ga.precision = c.weight_precision;
            ga.compute = compute;
            ga.n_groups = S + El;
            ga.groups = h->groups.as<Group>();
            ga.tile_prefix = h->tile_prefix.as<int64_t>();
            ga.experts = h->table.as<ExpertLayers>();
            ga.d = d;
            ga.h = hd;
            ga.clamped = c.clamped;
            ga.clamp_limit = c.clamp_limit;
            ga.xp = h->xp.p;
            ga.hp = h->hp.p;
            ga.yp = h->yp.p;
            GT_CHECK(h->phase_begin(3));
            GT_CHECK(launch_grouped_simt(ga, 1, st));
            GT_CHECK(h->phase_end(3));
            GT_CHECK(h->phase_begin(4));
            GT_CHECK(launch_grouped_simt(ga, 2, st));
            GT_CHECK(h->phase_end(4));
        }
    }
    // keep the host tables alive until their copies ran
    GT_CUDA(cudaStreamSynchronize(st));

    // ---- outputs back to the tokens' ranks
    GT_CHECK(h->phase_begin(7));
    GT_CHECK(segment_copy(h->yp.p, ep->yback.p, back, ep->segs_back, row_bytes, st));
    GT_NCCL(g_nccl.GroupStart());
    for (int s = 0; s < G; s++)
        if (recv_cnt[s] > 0)
            GT_NCCL(g_nccl.Send((const char *)ep->yback.p + recv_off[s] * row_bytes, recv_cnt[s] * row_bytes,
                                ncclUint8, s, ep->comm, st));
    for (int q = 0; q < G; q++)
        if (send_cnt[q] > 0)
            GT_NCCL(g_nccl.Recv((char *)ep->yret.p + send_off[q] * row_bytes, send_cnt[q] * row_bytes, ncclUint8, q,
                                ep->comm, st));
    GT_NCCL(g_nccl.GroupEnd());
    GT_CHECK(h->phase_end(7));

    CombineArgs ca;
    ca.T = T;
    ca.d = d;
    ca.k = k;
    ca.S = S;
    ca.y = h->yp.p;
    ca.y_routed = ep->yret.p;
    ca.y_dtype = compute;
    ca.shared_row0 = 0;
    ca.routed_row0 = 0;
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

    if (out_host) GT_CUDA(cudaMemcpyAsync(out, out_dev, obytes, cudaMemcpyDeviceToHost, st));
    if (chosen_out && TK) GT_CUDA(cudaMemcpyAsync(chosen_out, h->chosen.p, sizeof(int32_t) * TK, cudaMemcpyDefault, st));
    if (gates_out && TK) GT_CUDA(cudaMemcpyAsync(gates_out, h->gates64.p, sizeof(double) * TK, cudaMemcpyDefault, st));
    if (perm_out && TK) GT_CUDA(cudaMemcpyAsync(perm_out, h->perm.p, sizeof(int32_t) * TK, cudaMemcpyDefault, st));
    if (load_out) GT_CUDA(cudaMemcpyAsync(load_out, h->load.p, sizeof(int64_t) * E, cudaMemcpyDefault, st));
    GT_CUDA(cudaStreamSynchronize(st));
    GT_CHECK(tc_check_error(h->tc));
    return 0;
}

}  // namespace gtmoe

using namespace gtmoe;

extern "C" {

int gtmoe_ep_unique_id(void *nccl_id_128) {
    if (!nccl_id_128) return fail(GTMOE_EINVAL, "nccl_id is NULL");
    GT_CHECK(load_nccl());
    ncclUniqueId id;
    GT_NCCL(g_nccl.GetUniqueId(&id));
    memcpy(nccl_id_128, &id, sizeof(id));
    return 0;
}

int gtmoe_create_ep(const gtmoe_config *cfg, int device, int n_ranks, int rank, const void *nccl_id_128,
                    gtmoe_t *out) {
    if (!nccl_id_128) return fail(GTMOE_EINVAL, "nccl_id is NULL");
    GT_CHECK(load_nccl());
    gtmoe_t h = nullptr;
    GT_CHECK(create_handle(cfg, device, n_ranks, rank, &h));
    EpState *ep = new EpState();
    h->ep = ep;
    ncclUniqueId id;
    memcpy(&id, nccl_id_128, sizeof(id));
    ncclResult_t r = g_nccl.CommInitRank(&ep->comm, n_ranks, id, rank);
    if (r != ncclSuccess) {
        ep->comm = nullptr;
        gtmoe_destroy(h);
        return fail(GTMOE_ENCCL, "ncclCommInitRank failed: %s", g_nccl.GetErrorString(r));
    }
    *out = h;
    return 0;
}

}  // extern "C"
