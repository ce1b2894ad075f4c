// handle.h -- the state behind a gtmoe_t (shared by api.cu, tc.cu, ep.cu).
#pragma once

#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"

namespace gtmoe {

// Grow-only device buffer.
struct DevBuf {
    void *p = nullptr;
    size_t n = 0;
    int ensure(size_t bytes) {
        if (bytes <= n) return 0;
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
        size_t want = bytes < 256 ? 256 : bytes;
        cudaError_t e = cudaMalloc(&p, want);
        if (e != cudaSuccess) {
            p = nullptr;
            cudaGetLastError();
            return fail(GTMOE_ENOMEM, "cudaMalloc of %zu bytes failed: %s", want, cudaGetErrorString(e));
        }
        n = want;
        return 0;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    template <typename T>
    T *as() const {
        return (T *)p;
    }
};

struct LayerDev {
    int set = 0;
    int precision = 0, rows = 0, width = 0;
    DevBuf w, s, b32, b64;
    DevBuf tiled;  // tile-chunk layout of w + s for the tensor-core kernels (tc.cu)
    int has_bias = 0;
    // w and s (the RowsSnapshot layout, read only by the SIMT kernels and the
    // backward) are released once `tiled` holds the same bytes, and rebuilt
    // from it when training is switched on (tc_restore_raw)
    int raw_dropped = 0;
};

}  // namespace gtmoe

#include "tc.h"

struct gtmoe_handle {
    using DevBuf = gtmoe::DevBuf;
    using LayerDev = gtmoe::LayerDev;
    gtmoe_config cfg;
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaStream_t own_stream = nullptr;
    std::mutex mu;
    int no_tc = 0, no_decode = 0;  // kernel-path test switches (read at creation)

    // expert parallelism
    int n_ranks = 1, rank = 0;
    int e_begin = 0, e_local = 0;
    void *ep = nullptr;  // EpState (ep.cu)
    // Expert table: slot of each routed expert this handle holds (-1 if it
    // does not), and the routed expert of each slot from n_shared on.  The
    // owned experts take slots n_shared .. n_shared + e_local - 1; hot-expert
    // replicas that another rank owns (gtmoe_ep_set_replicas) follow.
    std::vector<int> slot_of, routed_of_slot;
    std::vector<char> replicated;  // per routed expert (expert parallel)
    int n_replicas = 0;

    // router
    int router_set = 0;
    DevBuf wr64, wr32, br, bal, wr3;  // wr3: bf16 hi/mid/lo split, 3 x e_pad x d
    int e_pad = 0;
    std::vector<double> h_bal;
    double wmax = 0;

    std::vector<LayerDev> layers;  // (number of slots) * 3
    DevBuf table;
    int table_dirty = 1;
    gtmoe::TcWeights tc;  // tensor-core layouts (tc.h)

    // per-call workspace
    DevBuf x_in, ids, logits, chosen, gates64, gates32, counts, load, offsets, perm, slot_row, groups, tile_prefix, xp,
        hp, yp, out_dev, res_dev, fixups, flagged;
    int have_load = 0;
    int64_t last_T = 0;
    int last_fixups = 0;

    // per-phase timing (gtmoe_set_timing / gtmoe_read_timing)
    struct PhaseEvents {
        cudaEvent_t start[GTMOE_N_PHASES];
        cudaEvent_t stop[GTMOE_N_PHASES];
    };
    int timing = 0;
    std::vector<PhaseEvents> tev;
    size_t tev_used = 0;
    int64_t launches_at_read = 0;

    // the block's RMSNorm (block.cu): weights (d, float64), epsilon, and the
    // input / normalized rows of gtmoe_forward_block
    DevBuf norm_w, block_x, block_xn, block_xn16, block_xn16mid, block_xn16lo;
    // set by gtmoe_forward_block for its inner Forward: the bf16 rounding of
    // the normalized rows, which the gather copies instead of converting the
    // float64 rows (the same bits: both round the same double once)
    const void *gather_bf16 = nullptr;
    // ... and the second and third bf16 terms of those rows, with which the
    // router computes their logits on the tensor cores (router_tc.cu)
    const void *router_bf16_mid = nullptr;
    const void *router_bf16_lo = nullptr;
    double norm_eps = 0;
    int norm_set = 0;

    // training (backward.cu): what gtmoe_backward needs from the last Forward
    // (its input rows as float64, chosen experts, gates, the expert-sorted
    // token lists) and the backward's workspace
    int training = 0;
    int tr_valid = 0;
    int64_t tr_T = 0;
    DevBuf tr_x, tr_chosen, tr_gates, tr_perm, tr_offsets;
    DevBuf bw_in, bw_dout, bw_dx, bw_rows, bw_y, bw_lg, bw_zag, bw_rw, bw_rb;
    DevBuf bw_work;  // work rows expert by expert, group offsets, tile prefix
    DevBuf bw_pgpu;  // gate / up pre-activations, then their gradients (work rows x hidden, twice)

    // host-buffer forwards of large batches: chunks whose copies overlap the
    // compute of their neighbours (api.cu, forward_pipelined)
    DevBuf x_pipe[2], out_pipe[2], load_acc;
    cudaStream_t h2d_stream = nullptr, d2h_stream = nullptr;
    cudaEvent_t pipe_ev[8] = {};  // x ready / x free / out ready / out free, per slot

    // CUDA-graph replay of the device forward (gtmoe_set_graphs): a call
    // whose arguments and workspace equal the previous call's replays the
    // graph captured on the second such call
    int graphs = 1;
    std::vector<uint64_t> gkey;  // arguments and workspace of the last call
    int gkey_hits = 0;
    cudaGraphExec_t gexec = nullptr;
    int64_t glaunches = 0;  // kernel launches inside the graph
    void drop_graph() {
        if (gexec) cudaGraphExecDestroy(gexec);
        gexec = nullptr;
        gkey.clear();
        gkey_hits = 0;
    }

    int phase_begin(int p);
    int phase_end(int p);
};


namespace gtmoe {
int layer_index(const gtmoe_handle *h, int kind, int index, int which);
int refresh_table(gtmoe_handle *h);  // device table of expert layers (+ tensor-core set-up)
int forward_device(gtmoe_handle *h, const void *x_dev, int x_dtype, int64_t T, const int64_t *ids_dev,
                   const void *res_dev, void *out_dev, int out_dtype);
int create_handle(const gtmoe_config *cfg, int device, int n_ranks, int rank, gtmoe_t *out);

// expert parallelism (ep.cu)
void ep_destroy(gtmoe_handle *h);
// gtmoe_forward with the handle's lock already held
bool is_device_ptr(const void *p);  // device or managed memory
int upload(DevBuf &dst, const void *src, size_t bytes, cudaStream_t st);  // ensure + async copy
// After a successful single-GPU Forward with training on: keep its state (backward.cu).
int save_training_state(gtmoe_handle *h, const void *x_dev, int x_dtype, int64_t T);
void release_training_state(gtmoe_handle *h);
int forward_locked(gtmoe_t h, const void *x, int x_dtype, int64_t T, const int64_t *token_ids, const void *residual,
                   void *out, int out_dtype, int32_t *chosen, double *gates, int32_t *perm, int64_t *load);
int ep_forward(gtmoe_handle *h, const void *x, int x_dtype, int64_t T, const int64_t *token_ids, const void *residual,
               void *out, int out_dtype, int32_t *chosen, double *gates, int32_t *perm, int64_t *load, int arg_rc);
int ep_global_load(gtmoe_handle *h, int64_t *load);

// kernel launches made by the library (all handles)
int64_t launches_so_far();
}  // namespace gtmoe
