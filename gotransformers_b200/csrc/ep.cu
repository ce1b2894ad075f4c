// ep.cu -- expert parallelism across GPUs (one process per GPU).
//
// The reference runs MixtureOfExperts.Forward in one process
// (mixtureofexperts.go:122-216); the benchmark's config c5 shards its routed
// experts over 1-8 GPUs.  Per rank r of G (routed experts r*E/G .. (r+1)*E/G-1
// owned, router and shared experts replicated, tokens split by the caller):
//   1. route this rank's tokens (router.cu) and dispatch them over all E
//      experts (dispatch.cu): the stable permutation orders (token, slot)
//      rows by global expert, i.e. by destination rank, token-ascending;
//   2. exchange every rank's per-expert counts and token count (each rank
//      stores its E+1 int64 into every rank's mailbox over the IPC mappings
//      and signals; a bounded wait for all G arrivals; one host
//      synchronisation: the host needs the sizes for the group table and the
//      buffers).  A rank that stops calling Forward makes the others' wait run
//      out (GTMOE_ETIMEOUT) instead of hanging them; NCCL is used only at set
//      up and when the peer buffers grow;
//   3. the push kernel copies each (token, slot) row straight into the owning
//      GPU's GEMM input over NVLink (CUDA IPC mappings of every rank's
//      buffers): expert-major, source-ascending inside an expert, so an
//      expert's rows are the reference's token order over the whole batch;
//   4. the grouped SwiGLU kernels (shared experts on this rank's tokens,
//      owned routed experts on the received rows);
//   5. the return kernel copies every output row straight into its token's
//      rank, at the (token, slot) position, where combine.cu adds them in the
//      reference's order.
// Hot-expert replicas (gtmoe_ep_set_replicas, opt-in): a routed expert that
// every rank holds is computed on each token's own rank, like the shared
// experts -- its rows are copied into this rank's own GEMM input and its
// outputs stored into this rank's own return buffer, and never cross NVLink.
// Under a skewed router (a few experts chosen by nearly every token) this
// takes the hottest experts' rows off the ranks that own them.  Every other
// routed expert stays owned by index.
// A kernel that pushed rows fences them (system scope) and then increments
// an arrival counter on every rank, once per CTA; the receiver's wait kernel
// spins (bounded) until all G sources' CTAs of this step have arrived.
// Buffers are reused across steps without a race: a rank pushes step n+1 only
// after the step n+1 count all-gather, which no rank joins before its stream
// has finished step n.  NCCL is loaded at run time (dlopen), only when an
// expert-parallel handle is created.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <string>
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
        {"ncclAllGather", (void **)&g_nccl.AllGather},
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

constexpr int kMaxEpRanks = 16;
// Fixed grids of the push and return kernels: every rank knows how many
// arrivals a step brings (G sources x this many CTAs).
constexpr int kPushCtas = 1184;
constexpr int kPushThreads = 256;
constexpr int kSigForward = 0, kSigReturn = 1, kSigCounts = 2;
// Each rank's IPC-shared signal block: 32 arrival counters, then the count
// mailboxes [2 step parities][G ranks][E + 1] int64.
constexpr size_t kSigCounterBytes = 256;

struct PeerRows {
    unsigned char *p[kMaxEpRanks];
};
struct PeerSigs {
    unsigned long long *p[kMaxEpRanks];
};

// One run of consecutive output rows that returns to one rank.
struct RetSeg {
    int64_t src_row;  // first row in this rank's expert output buffer
    int64_t dst_row;  // first (token, slot) position on the token's rank
    int64_t rows;
    int64_t rank;
};

__device__ __forceinline__ void copy_row(uint4 *__restrict__ dst, const uint4 *__restrict__ src, int nvec, int lane) {
    int i = lane;
    for (; i + 96 < nvec; i += 128) {
        const uint4 a = __ldg(src + i), b = __ldg(src + i + 32), c = __ldg(src + i + 64), e = __ldg(src + i + 96);
        dst[i] = a;
        dst[i + 32] = b;
        dst[i + 64] = c;
        dst[i + 96] = e;
    }
    for (; i < nvec; i += 32) dst[i] = __ldg(src + i);
}

// Every thread fences its own stores at system scope; the last CTA of the
// launch to get here then adds one arrival to every rank's counter `which`
// (`done` counts the launch's finished CTAs and is reset for the next launch).
__device__ __forceinline__ void signal_ranks(const PeerSigs &sig, int G, int which, unsigned int *done) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int n = atomicAdd(done, 1u);
        if (n == gridDim.x - 1) {
            *done = 0;
            __threadfence_system();
            for (int q = 0; q < G; q++) atomicAdd_system(sig.p[q] + which, 1ull);
        }
    }
}

// Rows of this rank's (token, slot) pairs, in dispatch order, to the ranks
// that compute them (dst_base[e] = (rank << 48) | first row of this rank's
// rows of expert e there); then (copy_shared) all T token rows to this rank's
// own buffer after its received rows, for the shared experts.
__global__ void __launch_bounds__(kPushThreads) ep_push_kernel(
    const uint4 *__restrict__ x, int vec_per_row, const int32_t *__restrict__ perm, int64_t TK,
    const int64_t *__restrict__ offsets, int E, const int64_t *__restrict__ dst_base, int64_t T,
    int copy_shared, int64_t shared_row0, int rank, const __grid_constant__ PeerRows rows,
    const __grid_constant__ PeerSigs sig, int G, unsigned int *done) {
    extern __shared__ int64_t off_s[];  // E + 1 exclusive prefix of this rank's per-expert counts
    for (int e = threadIdx.x; e <= E; e += blockDim.x) off_s[e] = offsets[e];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t n = TK + (copy_shared ? T : 0);
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < n; w += warps) {
        if (w < TK) {
            int lo = 0, hi = E;  // last e with off_s[e] <= w
            while (hi - lo > 1) {
                const int mid = (lo + hi) >> 1;
                if (off_s[mid] <= w) lo = mid;
                else hi = mid;
            }
            const int64_t code = dst_base[lo];
            const int q = (int)(code >> 48);
            const int64_t dst = (code & 0xFFFFFFFFFFFFll) + (w - off_s[lo]);
            copy_row((uint4 *)rows.p[q] + dst * vec_per_row, x + (int64_t)perm[w] * vec_per_row, vec_per_row, lane);
        } else {
            const int64_t t = w - TK;
            copy_row((uint4 *)rows.p[rank] + (shared_row0 + t) * vec_per_row, x + t * vec_per_row, vec_per_row,
                     lane);
        }
    }
    signal_ranks(sig, G, kSigForward, done);
}

// Expert output rows back to their tokens' ranks.
__global__ void __launch_bounds__(kPushThreads) ep_return_kernel(
    const uint4 *__restrict__ y, int vec_per_row, const RetSeg *__restrict__ segs, int n_segs, int64_t row0,
    int64_t n_rows, const __grid_constant__ PeerRows rows, const __grid_constant__ PeerSigs sig, int G,
    unsigned int *done) {
    extern __shared__ int64_t start_s[];  // first row (relative to row0) of each segment
    for (int i = threadIdx.x; i < n_segs; i += blockDim.x) start_s[i] = segs[i].src_row - row0;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < n_rows; w += warps) {
        int lo = 0, hi = n_segs;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (start_s[mid] <= w) lo = mid;
            else hi = mid;
        }
        const RetSeg g = segs[lo];
        const int64_t dst = g.dst_row + (w - start_s[lo]);
        copy_row((uint4 *)rows.p[g.rank] + dst * vec_per_row, y + (row0 + w) * vec_per_row, vec_per_row, lane);
    }
    signal_ranks(sig, G, kSigReturn, done);
}

// Destination of every output row the down kernel returns: (rank << 48) | row.
__global__ void ep_route_kernel(const RetSeg *__restrict__ segs, int n_segs, int64_t row0, int64_t n_rows,
                                int64_t *__restrict__ route) {
    extern __shared__ int64_t start_s[];
    for (int i = threadIdx.x; i < n_segs; i += blockDim.x) start_s[i] = segs[i].src_row - row0;
    __syncthreads();
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n_rows; j += (int64_t)gridDim.x * blockDim.x) {
        int lo = 0, hi = n_segs;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (start_s[mid] <= j) lo = mid;
            else hi = mid;
        }
        route[j] = (segs[lo].rank << 48) | (segs[lo].dst_row + (j - start_s[lo]));
    }
}

// The step's count exchange: this rank's E + 1 values (per-expert rows, then
// its token count) into mailbox row `rank` of parity `slot` on every rank,
// one arrival on every rank's count counter, then a bounded wait until all G
// ranks' arrivals of this exchange are in.  The mailboxes alternate between
// two parities: a rank writes exchange n + 2 only after exchange n + 1, which
// no rank joins before it has read exchange n.
__global__ void ep_counts_kernel(const int64_t *__restrict__ mine, int n, int rank, int G, int slot,
                                 const __grid_constant__ PeerSigs sig, unsigned long long target, int *err) {
    for (int q = 0; q < G; q++) {
        int64_t *box = reinterpret_cast<int64_t *>(reinterpret_cast<unsigned char *>(sig.p[q]) + kSigCounterBytes) +
                       ((int64_t)slot * G + rank) * n;
        for (int i = threadIdx.x; i < n; i += blockDim.x) box[i] = mine[i];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int q = 0; q < G; q++) atomicAdd_system(sig.p[q] + kSigCounts, 1ull);
    const unsigned long long *counter = sig.p[rank] + kSigCounts;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(counter) : "memory");
        if (v >= target) break;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicCAS(err, 0, 3);
            return;
        }
        __nanosleep(256);
    }
}

// Bounded wait until this rank's arrival counter reaches `target`.
__global__ void ep_wait_kernel(const unsigned long long *counter, unsigned long long target, int *err, int code) {
    if (threadIdx.x != 0) return;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(counter) : "memory");
        if (v >= target) break;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicCAS(err, 0, code);
            return;
        }
        __nanosleep(256);
    }
    // the next kernels read the rows with TMA (async proxy)
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

}  // namespace

struct EpState {
    ncclComm_t comm = nullptr;
    int G = 1, r = 0;
    std::vector<int64_t> h_gathered;  // G x (E + 1): per-expert counts, then the token count
    int have_gathered = 0;
    unsigned long long epoch = 0;         // completed row exchanges (same on every rank)
    unsigned long long count_epoch = 0;   // completed count exchanges (same on every rank)
    // IPC-shared buffers: the GEMM input (received rows, then own token rows)
    // and the returned expert outputs ((token, slot) order); capacities in
    // bytes, tracked identically on every rank
    void *x_local = nullptr, *y_local = nullptr, *sig_local = nullptr;
    std::vector<void *> peer_x, peer_y, peer_sig;
    std::vector<size_t> cap_x, cap_y;
    int *err = nullptr;
    unsigned int *done = nullptr;  // [0] push, [1] return, [2] fused down kernel: finished CTAs
    DevBuf staging, xconv, dst_base, ret_segs, route, peer_tab;
};

static EpState *ep_of(gtmoe_handle *h) { return (EpState *)h->ep; }

// NCCL all-gather of `n` bytes per rank through device staging (host in, host out).
static int allgather_bytes(EpState *ep, const void *mine, size_t n, void *all, cudaStream_t st) {
    GT_CHECK(ep->staging.ensure(n * ep->G));
    unsigned char *base = (unsigned char *)ep->staging.p;
    GT_CUDA(cudaMemcpyAsync(base + n * ep->r, mine, n, cudaMemcpyHostToDevice, st));
    GT_NCCL(g_nccl.AllGather(base + n * ep->r, base, n, ncclUint8, ep->comm, st));
    GT_CUDA(cudaMemcpyAsync(all, base, n * ep->G, cudaMemcpyDeviceToHost, st));
    GT_CUDA(cudaStreamSynchronize(st));
    return 0;
}

static void close_peer(void *&p) {
    if (p) cudaIpcCloseMemHandle(p);
    p = nullptr;
}

void ep_destroy(gtmoe_handle *h) {
    EpState *ep = ep_of(h);
    if (!ep) return;
    cudaSetDevice(h->device);
    cudaStreamSynchronize(h->stream);
    for (int q = 0; q < ep->G; q++) {
        if (q == ep->r) continue;
        if (q < (int)ep->peer_x.size()) close_peer(ep->peer_x[q]);
        if (q < (int)ep->peer_y.size()) close_peer(ep->peer_y[q]);
        if (q < (int)ep->peer_sig.size()) close_peer(ep->peer_sig[q]);
    }
    if (ep->comm && g_nccl.loaded) g_nccl.CommDestroy(ep->comm);
    for (void *p : {ep->x_local, ep->y_local, ep->sig_local, (void *)ep->err, (void *)ep->done})
        if (p) cudaFree(p);
    DevBuf *bufs[] = {&ep->staging, &ep->xconv, &ep->dst_base, &ep->ret_segs, &ep->route, &ep->peer_tab};
    for (DevBuf *b : bufs) b->release();
    delete ep;
    h->ep = nullptr;
}

static size_t sig_bytes(int G, int E) { return kSigCounterBytes + 2 * (size_t)G * (E + 1) * sizeof(int64_t); }

// Maps every rank's signal block -- arrival counters and count mailboxes --
// (once, at creation).
static int ep_map_signals(gtmoe_handle *h, EpState *ep) {
    const int G = ep->G;
    const size_t sb = sig_bytes(G, h->cfg.n_routed);
    GT_CUDA(cudaMalloc(&ep->sig_local, sb));
    GT_CUDA(cudaMemset(ep->sig_local, 0, sb));
    GT_CUDA(cudaMalloc(&ep->err, sizeof(int)));
    GT_CUDA(cudaMemset(ep->err, 0, sizeof(int)));
    GT_CUDA(cudaMalloc(&ep->done, 4 * sizeof(unsigned int)));
    GT_CUDA(cudaMemset(ep->done, 0, 4 * sizeof(unsigned int)));
    GT_CUDA(cudaDeviceSynchronize());
    cudaIpcMemHandle_t mine;
    GT_CUDA(cudaIpcGetMemHandle(&mine, ep->sig_local));
    std::vector<cudaIpcMemHandle_t> all(G);
    GT_CHECK(allgather_bytes(ep, &mine, sizeof(mine), all.data(), h->stream));
    ep->peer_sig.assign(G, nullptr);
    ep->peer_x.assign(G, nullptr);
    ep->peer_y.assign(G, nullptr);
    ep->cap_x.assign(G, 0);
    ep->cap_y.assign(G, 0);
    for (int q = 0; q < G; q++) {
        if (q == ep->r) {
            ep->peer_sig[q] = ep->sig_local;
            continue;
        }
        GT_CUDA(cudaIpcOpenMemHandle(&ep->peer_sig[q], all[q], cudaIpcMemLazyEnablePeerAccess));
    }
    return 0;
}

// Grows the IPC-shared row buffers of every rank that needs more than it has
// (a collective step: every rank takes it with the same sizes).
static int ep_ensure_buffers(gtmoe_handle *h, EpState *ep, const std::vector<size_t> &need_x,
                             const std::vector<size_t> &need_y) {
    const int G = ep->G, r = ep->r;
    std::vector<char> grow(G, 0);
    bool any = false;
    for (int q = 0; q < G; q++)
        if (need_x[q] > ep->cap_x[q] || need_y[q] > ep->cap_y[q]) grow[q] = 1, any = true;
    if (!any) return 0;
    cudaStream_t st = h->stream;
    // 1. drop the mappings of buffers about to be replaced; 2. wait until
    // every rank has (nobody frees a buffer a peer still maps)
    for (int q = 0; q < G; q++)
        if (grow[q] && q != r) close_peer(ep->peer_x[q]), close_peer(ep->peer_y[q]);
    GT_CUDA(cudaStreamSynchronize(st));
    int token = 1;
    std::vector<int> tokens(G);
    GT_CHECK(allgather_bytes(ep, &token, sizeof(int), tokens.data(), st));
    // 3. new capacities (a quarter of headroom), the same on every rank
    auto grown = [](size_t cap, size_t need) {
        size_t c = need <= cap ? cap : need + need / 4;
        if (c < 4096) c = 4096;
        return (c + 255) / 256 * 256;
    };
    for (int q = 0; q < G; q++)
        if (grow[q]) {
            ep->cap_x[q] = grown(ep->cap_x[q], need_x[q]);
            ep->cap_y[q] = grown(ep->cap_y[q], need_y[q]);
        }
    struct {
        cudaIpcMemHandle_t x, y;
    } mine, zero;
    memset(&mine, 0, sizeof(mine));
    memset(&zero, 0, sizeof(zero));
    if (grow[r]) {
        if (ep->x_local) cudaFree(ep->x_local);
        if (ep->y_local) cudaFree(ep->y_local);
        ep->x_local = ep->y_local = nullptr;
        cudaError_t e1 = cudaMalloc(&ep->x_local, ep->cap_x[r]);
        cudaError_t e2 = e1 == cudaSuccess ? cudaMalloc(&ep->y_local, ep->cap_y[r]) : e1;
        if (e1 != cudaSuccess || e2 != cudaSuccess) {
            cudaGetLastError();
            return fail(GTMOE_ENOMEM, "expert-parallel buffers of %zu + %zu bytes: %s", ep->cap_x[r], ep->cap_y[r],
                        cudaGetErrorString(e1 != cudaSuccess ? e1 : e2));
        }
        GT_CUDA(cudaIpcGetMemHandle(&mine.x, ep->x_local));
        GT_CUDA(cudaIpcGetMemHandle(&mine.y, ep->y_local));
        ep->peer_x[r] = ep->x_local;
        ep->peer_y[r] = ep->y_local;
    }
    // 4. everybody's handles; open the new ones
    std::vector<decltype(mine)> all(G);
    GT_CHECK(allgather_bytes(ep, &mine, sizeof(mine), all.data(), st));
    for (int q = 0; q < G; q++) {
        if (!grow[q] || q == r) continue;
        GT_CUDA(cudaIpcOpenMemHandle(&ep->peer_x[q], all[q].x, cudaIpcMemLazyEnablePeerAccess));
        GT_CUDA(cudaIpcOpenMemHandle(&ep->peer_y[q], all[q].y, cudaIpcMemLazyEnablePeerAccess));
    }
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
        for (int r = 0; r < h->n_ranks; r++) s += ep->h_gathered[(size_t)r * (E + 1) + e];
        load[e] = s;
    }
    return 0;
}

// The step's count exchange: h->load holds this rank's per-expert rows and,
// at [E], its token count; afterwards ep->h_gathered holds every rank's.
static int ep_exchange_counts(gtmoe_handle *h, EpState *ep, cudaStream_t st) {
    const int E = h->cfg.n_routed, G = ep->G, n = E + 1;
    const int slot = (int)(ep->count_epoch & 1);
    ep->count_epoch++;
    PeerSigs sg;
    for (int q = 0; q < kMaxEpRanks; q++) sg.p[q] = q < G ? (unsigned long long *)ep->peer_sig[q] : nullptr;
    ep_counts_kernel<<<1, 256, 0, st>>>(h->load.as<int64_t>(), n, ep->r, G, slot, sg,
                                        ep->count_epoch * (unsigned long long)G, ep->err);
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    ep->h_gathered.resize((size_t)G * n);
    const int64_t *box = reinterpret_cast<const int64_t *>((const unsigned char *)ep->sig_local + kSigCounterBytes) +
                         (size_t)slot * G * n;
    GT_CUDA(cudaMemcpyAsync(ep->h_gathered.data(), box, sizeof(int64_t) * G * n, cudaMemcpyDeviceToHost, st));
    GT_CUDA(cudaStreamSynchronize(st));
    int werr = 0;
    GT_CUDA(cudaMemcpy(&werr, ep->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (werr)
        return fail(GTMOE_ETIMEOUT,
                    "expert-parallel count exchange gave up waiting for the other ranks (a rank did not call "
                    "Forward for this step); the handle is unusable");
    return 0;
}

// The step's count exchange with this rank's counts replaced by a refusal
// marker (token count -1): every rank then fails the step together.
static int ep_refuse_step(gtmoe_handle *h, EpState *ep, int rc) {
    const std::string msg = gtmoe_last_error();
    const int E = h->cfg.n_routed;
    cudaStream_t st = h->stream;
    GT_CHECK(h->load.ensure(sizeof(int64_t) * (E + 1)));
    std::vector<int64_t> mine(E + 1, 0);
    mine[E] = -1;
    GT_CUDA(cudaMemcpyAsync(h->load.p, mine.data(), sizeof(int64_t) * (E + 1), cudaMemcpyHostToDevice, st));
    GT_CHECK(ep_exchange_counts(h, ep, st));
    return fail(rc, "%s", msg.c_str());
}

int ep_forward(gtmoe_handle *h, const void *x, int x_dtype, int64_t T, const int64_t *token_ids, const void *residual,
               void *out, int out_dtype, int32_t *chosen_out, double *gates_out, int32_t *perm_out,
               int64_t *load_out, int arg_rc) {
    EpState *ep = ep_of(h);
    if (arg_rc != 0) return ep_refuse_step(h, ep, arg_rc);
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
    if (row_bytes % 16 != 0)
        return ep_refuse_step(h, ep, fail(GTMOE_EINVAL, "expert-parallel rows must be a multiple of 16 bytes"));
    const int vec = (int)(row_bytes / 16);
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
                return ep_refuse_step(h, ep,
                                      fail(GTMOE_EINVAL, "mixture of experts: token ID %lld at row %lld is negative",
                                           (long long)hid[t], (long long)t));
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
    GT_CHECK(h->logits.ensure(sizeof(double) *
                              ((size_t)(T > 0 ? T : 1) * E + (size_t)std::min<int64_t>(T, kRouterSmallMaxT))));
    GT_CHECK(h->chosen.ensure(sizeof(int32_t) * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(h->gates64.ensure(sizeof(double) * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(h->gates32.ensure(sizeof(float) * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(h->counts.ensure(sizeof(int32_t) * (size_t)(n_chunks > 0 ? n_chunks : 1) * E));
    GT_CHECK(h->load.ensure(sizeof(int64_t) * (E + 1)));
    GT_CHECK(h->offsets.ensure(sizeof(int64_t) * (E + 1)));
    GT_CHECK(h->perm.ensure(sizeof(int32_t) * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(h->slot_row.ensure(sizeof(int64_t) * (size_t)(TK > 0 ? TK : 1)));
    GT_CHECK(h->groups.ensure(sizeof(Group) * (S + E)));
    GT_CHECK(h->tile_prefix.ensure(sizeof(int64_t) * (S + E + 1)));
    GT_CHECK(h->fixups.ensure(sizeof(int)));
    GT_CHECK(h->flagged.ensure(sizeof(int) * (size_t)(T > 0 ? T : 1)));
    GT_CHECK(ep->dst_base.ensure(sizeof(int64_t) * E));
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
    ra.use_tc = !c.hash_routing && h->wr3.p && !h->no_tc && router_tc_usable(x_dev, x_dtype, T, d);
    ra.thresh_scale = (ra.use_tc ? kRouterTcErr : kRouterSimtErr) * h->wmax;
    ra.w3 = h->wr3.p;
    ra.e_pad = h->e_pad;
    ra.err = h->tc.err;
    ra.sms = h->tc.sms;
    ra.logits = h->logits.as<double>();
    ra.xnorm = ra.logits + (size_t)(T > 0 ? T : 1) * E;
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

    // ---- everybody's per-expert counts and token counts
    GT_CHECK(h->phase_begin(6));
    const int64_t T_mine = T;
    GT_CUDA(cudaMemcpyAsync(h->load.as<int64_t>() + E, &T_mine, sizeof(int64_t), cudaMemcpyHostToDevice, st));
    GT_CHECK(ep_exchange_counts(h, ep, st));
    ep->have_gathered = 1;
    const int64_t *hg = ep->h_gathered.data();
    auto L = [&](int s, int e) { return hg[(size_t)s * (E + 1) + e]; };  // rows of rank s for expert e
    auto Tof = [&](int s) { return hg[(size_t)s * (E + 1) + E]; };
    for (int s = 0; s < G; s++)
        if (Tof(s) < 0)
            return fail(GTMOE_EINVAL, "expert-parallel rank %d refused its Forward arguments; no rank ran this step", s);
    // Rows of expert e that rank q computes: a replicated expert's rows of
    // q's own tokens, an owned expert's rows from every rank, else none.
    const std::vector<char> &rep = h->replicated;
    auto held_rows = [&](int q, int e) -> int64_t {
        if (rep[e]) return L(q, e);
        if (e / El != q) return 0;
        int64_t n = 0;
        for (int s = 0; s < G; s++) n += L(s, e);
        return n;
    };
    auto held = [&](int q, int e) { return rep[e] || e / El == q; };
    // eoff[q*E + e]: first row of expert e in rank q's GEMM input (expert-major,
    // experts ascending, sources ascending inside an expert)
    std::vector<int64_t> eoff((size_t)G * E, 0), n_recv(G, 0);
    for (int q = 0; q < G; q++) {
        int64_t run = 0;
        for (int e = 0; e < E; e++) {
            eoff[(size_t)q * E + e] = run;
            run += held_rows(q, e);
        }
        n_recv[q] = run;
    }
    std::vector<size_t> need_x(G), need_y(G);
    for (int q = 0; q < G; q++) {
        need_x[q] = row_bytes * (size_t)(n_recv[q] + (S > 0 ? Tof(q) : 0));
        need_y[q] = row_bytes * (size_t)(Tof(q) * k);
    }
    GT_CHECK(ep_ensure_buffers(h, ep, need_x, need_y));

    // where this rank's rows for expert e go: (rank << 48) | first row there
    std::vector<int64_t> dst_base(E);
    for (int e = 0; e < E; e++) {
        const int q = rep[e] ? r : e / El;
        int64_t b = eoff[(size_t)q * E + e];
        if (!rep[e])
            for (int s = 0; s < r; s++) b += L(s, e);
        dst_base[e] = ((int64_t)q << 48) | b;
    }
    // this rank's group table: shared experts on its own tokens (after the
    // received rows), then every expert it holds, ascending
    const int64_t nr = n_recv[r];
    const int64_t rows_x = nr + (S > 0 ? T : 0);
    const int64_t rows_h = (int64_t)S * T + nr;
    std::vector<Group> groups;
    const int bm = use_tc ? tc_tile_rows(h->tc) : kSimtBM;
    for (int s = 0; s < S; s++) groups.push_back(Group{nr, (int64_t)s * T, T, s, 0});
    for (int e = 0; e < E; e++)
        if (held(r, e)) {
            const int64_t o = eoff[(size_t)r * E + e];
            groups.push_back(Group{o, (int64_t)S * T + o, held_rows(r, e), h->slot_of[e], 0});
        }
    const int n_groups = (int)groups.size();
    std::vector<int64_t> prefix(n_groups + 1, 0);
    for (int g = 0; g < n_groups; g++) prefix[g + 1] = prefix[g] + (groups[g].m + bm - 1) / bm;
    // output rows back: (held expert, source) runs to the source's (token,
    // slot) positions, which follow the source's dispatch order
    std::vector<int64_t> slot0((size_t)G * E, 0);  // exclusive prefix of each rank's counts
    for (int s = 0; s < G; s++)
        for (int e = 1; e < E; e++) slot0[(size_t)s * E + e] = slot0[(size_t)s * E + e - 1] + L(s, e - 1);
    std::vector<RetSeg> back;
    for (int e = 0; e < E; e++) {
        if (!held(r, e)) continue;
        int64_t src = (int64_t)S * T + eoff[(size_t)r * E + e];
        for (int s = 0; s < G; s++) {
            if (rep[e] && s != r) continue;
            const int64_t n = L(s, e);
            if (n > 0) back.push_back(RetSeg{src, slot0[(size_t)s * E + e], n, s});
            src += n;
        }
    }
    GT_CUDA(cudaMemcpyAsync(ep->dst_base.p, dst_base.data(), sizeof(int64_t) * E, cudaMemcpyHostToDevice, st));
    GT_CUDA(cudaMemcpyAsync(h->groups.p, groups.data(), sizeof(Group) * n_groups, cudaMemcpyHostToDevice, st));
    GT_CUDA(cudaMemcpyAsync(h->tile_prefix.p, prefix.data(), sizeof(int64_t) * (n_groups + 1), cudaMemcpyHostToDevice,
                            st));
    if (!back.empty()) {
        GT_CHECK(ep->ret_segs.ensure(sizeof(RetSeg) * back.size()));
        GT_CUDA(cudaMemcpyAsync(ep->ret_segs.p, back.data(), sizeof(RetSeg) * back.size(), cudaMemcpyHostToDevice,
                                st));
    }
    PeerRows px, py;
    PeerSigs sg;
    for (int q = 0; q < kMaxEpRanks; q++) {
        px.p[q] = q < G ? (unsigned char *)ep->peer_x[q] : nullptr;
        py.p[q] = q < G ? (unsigned char *)ep->peer_y[q] : nullptr;
        sg.p[q] = q < G ? (unsigned long long *)ep->peer_sig[q] : nullptr;
    }
    // rows in the compute type, token order
    const void *xrows = x_dev;
    if (T > 0 && x_dtype != compute) {
        GT_CHECK(ep->xconv.ensure(row_bytes * (size_t)T));
        GT_CHECK(launch_gather(x_dev, x_dtype, T, d, nullptr, 0, 0, 1, ep->xconv.p, compute, st));
        xrows = ep->xconv.p;
    }
    ep->epoch++;
    const unsigned long long arrivals = ep->epoch * (unsigned long long)G;  // one per source rank and step
    ep_push_kernel<<<kPushCtas, kPushThreads, sizeof(int64_t) * (E + 1), st>>>(
        (const uint4 *)xrows, vec, da.perm, TK, da.offsets, E, ep->dst_base.as<int64_t>(), T, S > 0 ? 1 : 0, nr, r,
        px, sg, G, ep->done + 0);
    GT_CUDA(cudaGetLastError());
    ep_wait_kernel<<<1, 32, 0, st>>>((unsigned long long *)ep->sig_local + kSigForward, arrivals, ep->err, 1);
    GT_CUDA(cudaGetLastError());
    note_launches(2);
    GT_CHECK(h->phase_end(6));

    GT_CHECK(h->hp.ensure(cs * (size_t)hd * (rows_h > 0 ? rows_h : 1)));
    GT_CHECK(h->yp.ensure(row_bytes * (size_t)(rows_h > 0 ? rows_h : 1)));
    // the tensor-core down kernel returns the routed rows itself
    const bool fused_return = use_tc && rows_h > 0;
    if (fused_return) {
        GT_CHECK(ep->route.ensure(sizeof(int64_t) * (size_t)(nr > 0 ? nr : 1)));
        GT_CHECK(ep->peer_tab.ensure(2 * sizeof(void *) * G));
        std::vector<void *> tab(2 * G);
        for (int q = 0; q < G; q++)
            tab[q] = ep->peer_y[q], tab[G + q] = (unsigned long long *)ep->peer_sig[q] + kSigReturn;
        GT_CUDA(cudaMemcpyAsync(ep->peer_tab.p, tab.data(), sizeof(void *) * 2 * G, cudaMemcpyHostToDevice, st));
        if (nr > 0) {
            ep_route_kernel<<<296, 256, sizeof(int64_t) * back.size(), st>>>(
                ep->ret_segs.as<RetSeg>(), (int)back.size(), (int64_t)S * T, nr, ep->route.as<int64_t>());
            GT_CUDA(cudaGetLastError());
            note_launches(1);
        }
    }
    if (rows_h > 0) {
        if (use_tc) {
            TcArgs ta;
            ta.n_groups = n_groups;
            ta.groups = h->groups.as<Group>();
            ta.tile_prefix = h->tile_prefix.as<int64_t>();
            ta.rows_x = rows_x;
            ta.rows_h = rows_h;
            ta.xp = ep->x_local;
            ta.hp = h->hp.p;
            ta.yp = h->yp.p;
            ta.ret_ranks = G;
            ta.ret_row0 = (int64_t)S * T;
            ta.ret_route = ep->route.as<int64_t>();
            ta.ret_peers = ep->peer_tab.as<unsigned char *const>();
            ta.ret_sigs = (unsigned long long *const *)(ep->peer_tab.as<void *>() + G);
            ta.ret_done = ep->done + 2;
            GT_CHECK(launch_grouped_tc(h, h->tc, ta, st));
        } else {
            GroupedArgs ga;
            ga.precision = c.weight_precision;
            ga.compute = compute;
            ga.n_groups = n_groups;
            ga.groups = h->groups.as<Group>();
            ga.tile_prefix = h->tile_prefix.as<int64_t>();
            ga.experts = h->table.as<ExpertLayers>();
            ga.d = d;
            ga.h = hd;
            ga.clamped = c.clamped;
            ga.clamp_limit = c.clamp_limit;
            ga.xp = ep->x_local;
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
    // ---- outputs back to the tokens' ranks
    GT_CHECK(h->phase_begin(7));
    if (!fused_return) {
        ep_return_kernel<<<kPushCtas, kPushThreads, sizeof(int64_t) * (back.empty() ? 1 : back.size()), st>>>(
            (const uint4 *)h->yp.p, vec, ep->ret_segs.as<RetSeg>(), (int)back.size(), (int64_t)S * T,
            back.empty() ? 0 : nr, py, sg, G, ep->done + 1);
        GT_CUDA(cudaGetLastError());
        note_launches(1);
    }
    ep_wait_kernel<<<1, 32, 0, st>>>((unsigned long long *)ep->sig_local + kSigReturn, arrivals, ep->err, 2);
    GT_CUDA(cudaGetLastError());
    note_launches(1);
    GT_CHECK(h->phase_end(7));

    CombineArgs ca;
    ca.T = T;
    ca.d = d;
    ca.k = k;
    ca.S = S;
    ca.y = h->yp.p;
    ca.y_routed = ep->y_local;
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
    int werr = 0;
    GT_CUDA(cudaMemcpy(&werr, ep->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (werr)
        return fail(GTMOE_ETIMEOUT,
                    "expert-parallel exchange gave up waiting for the other ranks' %s; the handle is unusable",
                    werr == 1 ? "token rows" : "expert outputs");
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

int gtmoe_ep_set_replicas(gtmoe_t h, int n, const int32_t *experts) {
    if (!h) return fail(GTMOE_EINVAL, "handle is NULL");
    std::lock_guard<std::mutex> lock(h->mu);
    EpState *ep = ep_of(h);
    if (!ep) return fail(GTMOE_EINVAL, "hot-expert replicas are for expert-parallel handles");
    if (ep->have_gathered || ep->epoch > 0)
        return fail(GTMOE_EINVAL, "hot-expert replicas must be set before the first Forward");
    const int E = h->cfg.n_routed, S = h->cfg.n_shared, El = h->e_local;
    if (n < 0 || n > E || (n > 0 && !experts))
        return fail(GTMOE_EINVAL, "gtmoe_ep_set_replicas: %d experts of %d", n, E);
    std::vector<char> rep(E, 0);
    for (int i = 0; i < n; i++) {
        const int e = experts[i];
        if (e < 0 || e >= E) return fail(GTMOE_EINVAL, "routed expert %d does not exist (%d routed)", e, E);
        if (rep[e]) return fail(GTMOE_EINVAL, "routed expert %d is listed twice", e);
        rep[e] = 1;
    }
    // the owned experts keep their slots; replicas owned by other ranks get
    // new, unset slots after them (slots of an earlier list are dropped)
    const size_t kept = (size_t)3 * (S + El);
    cudaSetDevice(h->device);
    for (size_t i = kept; i < h->layers.size(); i++) {
        LayerDev &L = h->layers[i];
        L.tiled.release();
        L.w.release();
        L.s.release();
        L.b32.release();
        L.b64.release();
    }
    h->layers.resize(kept);
    h->routed_of_slot.resize(S + El);
    for (int e = 0; e < E; e++)
        if (h->slot_of[e] >= S + El) h->slot_of[e] = -1;
    for (int e = 0; e < E; e++)
        if (rep[e] && h->slot_of[e] < 0) {
            h->slot_of[e] = (int)h->routed_of_slot.size();
            h->routed_of_slot.push_back(e);
            h->layers.resize(h->layers.size() + 3);
        }
    h->replicated = rep;
    h->n_replicas = n;
    h->table_dirty = 1;
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
    if (n_ranks > kMaxEpRanks) {
        gtmoe_destroy(h);
        return fail(GTMOE_EINVAL, "at most %d expert-parallel ranks, got %d", kMaxEpRanks, n_ranks);
    }
    ep->G = n_ranks;
    ep->r = rank;
    ncclResult_t r = g_nccl.CommInitRank(&ep->comm, n_ranks, id, rank);
    if (r != ncclSuccess) {
        ep->comm = nullptr;
        gtmoe_destroy(h);
        return fail(GTMOE_ENCCL, "ncclCommInitRank failed: %s", g_nccl.GetErrorString(r));
    }
    int rc = ep_map_signals(h, ep);
    if (rc != 0) {
        std::string msg = gtmoe_last_error();
        gtmoe_destroy(h);
        return fail(rc, "%s", msg.c_str());
    }
    *out = h;
    return 0;
}

}  // extern "C"
