// tc.h -- grouped SwiGLU expert products on the tcgen05 tensor cores.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

struct gtmoe_handle;

namespace gtmoe {

struct LayerDev;

struct TcWeights {
    int ready = 0;
    int sms = 148;
    int *err = nullptr;  // device flag: nonzero when a bounded wait expired
};

struct TcArgs {
    int n_groups;
    const Group *groups;
    const int64_t *tile_prefix;
    int64_t rows_x, rows_h;
    void *xp;  // rows_x x d bf16
    void *hp;  // rows_h x h bf16
    void *yp;  // rows_h x d bf16
    // Expert parallel: the down kernel writes output rows at or after
    // ret_row0 straight to their token's rank instead of yp, and its last CTA
    // then adds one arrival to every rank's counter (ret_ranks = 0: off).
    int ret_ranks = 0;
    int64_t ret_row0 = 0;
    const int64_t *ret_route = nullptr;             // per row: (rank << 48) | row on that rank
    unsigned char *const *ret_peers = nullptr;      // per rank: its returned-output buffer (device array)
    unsigned long long *const *ret_sigs = nullptr;  // per rank: its return arrival counter (device array)
    unsigned int *ret_done = nullptr;               // CTAs of this launch that finished (device, starts at 0)
};

bool tc_supported(const gtmoe_handle *h, int64_t T);
// Builds L.tiled (the chunk layout the tensor-core kernels stream) when the
// handle's shapes and precision use the tensor-core path; no-op otherwise.
int tc_relayout_layer(gtmoe_handle *h, LayerDev &L, int which);
// The RowsSnapshot arrays (L.w, L.s) rebuilt from L.tiled, after the layer
// dropped them (an exact inverse of the set-time permutation).
int tc_restore_raw(gtmoe_handle *h, LayerDev &L);
int tc_tile_rows(TcWeights &w);  // m-tile height of the current shape
int tc_prepare(gtmoe_handle *h, TcWeights &w);
int launch_grouped_tc(gtmoe_handle *h, TcWeights &w, const TcArgs &a, cudaStream_t st);
void tc_release(TcWeights &w);
// GTMOE_ETIMEOUT (and clears the flag) if a kernel recorded an expired wait.
int tc_check_error(TcWeights &w);

}  // namespace gtmoe
