// internal.h -- launchers shared between the .cu files of libgtmoe.so.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace gtmoe {

// Counts kernel launches made by the library (gtmoe_read_timing).
void note_launches(int n);



// Limits of this build (checked by gtmoe_create).
constexpr int kMaxRoutedExperts = 1024;
constexpr int kMaxTopK = 32;

struct DispatchArgs;
struct RouterArgs {
    int hash;
    const void *x;
    int x_dtype;
    int64_t T;
    int E, k, d;
    const int64_t *token_ids;   // hash routing (device)
    const float *w32;           // E x d
    const double *w64;          // E x d
    const double *bias;         // E
    const double *balance;      // E
    double thresh_scale;        // score margin per unit ||x_t||: 2 * 0.5 * (logit error bound) / ||x_t||
    int use_tc;                 // logits on the tensor cores (router_tc.cu)
    const void *x_tc = nullptr;      // their bf16 rows when x is not bf16: x_hi of a float64 split ...
    const void *x_tc_mid = nullptr;  // ... x_mid ...
    const void *x_tc_lo = nullptr;   // ... and x_lo (router_tc.cu)
    const void *w3;             // 3 x E_pad x d bf16 split of w64 (tensor-core path)
    int e_pad;
    int *err;                   // error flag: a bounded wait's code, or kErrNegativeTokenId
    int sms;
    double *logits;             // T x E scratch
    int32_t *chosen;            // T x k
    double *gates64;            // T x k
    float *gates32;             // T x k
    int *n_fixups;              // counter of tokens re-selected in float64
    int *flagged;               // T: tokens whose choice the fix-up kernel settles
    double *xnorm = nullptr;    // min(T, kRouterSmallMaxT): ||x_t||, left by the few-token logits kernel
    // the dispatch of this batch, for a router that runs it itself (router_fuses_dispatch)
    const DispatchArgs *dispatch = nullptr;
};
// Batches of at most this many tokens take the one-warp-per-(token, expert)
// logits kernel (when not on the tensor cores).
constexpr int64_t kRouterSmallMaxT = 256;
int launch_router(const RouterArgs &a, cudaStream_t st);
// True when launch_router also runs the dispatch of a.dispatch (a batch of at
// most 32 tokens over at most 128 experts: one CTA selects and dispatches);
// the caller then skips launch_dispatch.
bool router_fuses_dispatch(const RouterArgs &a);
// Error code the hash router records for a negative device token ID.
constexpr int kErrNegativeTokenId = 100;
bool router_tc_usable(const void *x, int x_dtype, int64_t T, int d);
// x_mid, x_lo: NULL for bf16 rows x, else the second and third bf16 terms of
// split float64 rows (x = x + x_mid + x_lo to 2^-24)
int launch_router_logits_tc(const void *x, const void *x_mid, const void *x_lo, int64_t T, int d, int E, int E_pad,
                            const void *w3, double *logits, int *err, int sms, cudaStream_t st);
// Logit error bounds (relative to ||x_t|| * max_e ||w_e||) of the paths.
constexpr double kRouterSimtErr = 32.0 / 16777216.0;  // 32 * 2^-24
constexpr double kRouterTcErr = 70.0 / 8388608.0;     // 70 * 2^-23
constexpr double kRouterTc3Err = 136.0 / 8388608.0;   // 136 * 2^-23: float64 rows as three bf16 terms

// Dispatch: builds the token-ascending permutation of (token, slot) pairs by
// expert (rowsForExpert, mixtureofexperts.go:175-180) and the group table.
constexpr int kDispatchChunk = 256;
struct DispatchArgs {
    int64_t T;
    int E, k, S;
    const int32_t *chosen;     // T x k
    int32_t *chunk_counts;     // n_chunks x E scratch
    int64_t *load;             // E
    int64_t *offsets;          // E + 1
    int32_t *perm;             // T*k : token of each routed row
    int64_t *slot_row;         // T*k : routed row of (token, slot)
    Group *groups;             // S + E
    int64_t *tile_prefix;      // S + E + 1 : prefix of m-tiles per group
    int bm;                    // m-tile height for the prefix
};
int launch_dispatch(const DispatchArgs &a, cudaStream_t st);

// Gathers activation rows into the expert-sorted buffer, converting dtype.
// Rows [0, T) are x itself when there are shared experts (copy_shared); the
// routed copy j of token t is row xbase + slot_row[t * k + j] (k may be 0:
// a plain conversion of x).
int launch_gather(const void *x, int x_dtype, int64_t T, int d, const int64_t *slot_row, int k, int64_t xbase,
                  int copy_shared, void *xp, int xp_dtype, cudaStream_t st);

// Grouped SwiGLU on SIMT cores, any precision and shape.
struct GroupedArgs {
    int precision;             // weight precision
    int compute;               // GTMOE_DTYPE_F32 or GTMOE_DTYPE_F64
    int n_groups;
    const Group *groups;
    const int64_t *tile_prefix;
    const ExpertLayers *experts;
    int d, h;
    int clamped;
    double clamp_limit;
    const void *xp;            // rows x d   (compute dtype)
    void *hp;                  // rows x h   (compute dtype)
    void *yp;                  // rows x d   (compute dtype)
};
constexpr int kSimtBM = 64;

// Weight-streaming expert products for decode-shaped batches (decode.cu):
// every group has at most kDecodeMaxRows rows; weights in the tile-chunk
// layout of the tensor-core path (ExpertLayers::tiled).
constexpr int kDecodeMaxRows = 64;
constexpr int kDecodeTileRows = 16;  // most rows per decode work unit (dispatch tile height)
// rows per decode work unit for a batch of T tokens: no group has more than
// T rows, so batches of up to 8 tokens use 8-row tiles (half the token tile's
// shared memory, more CTAs per SM)
inline int decode_tile_rows(int64_t T) { return T <= 8 ? 8 : kDecodeTileRows; }
struct DecodeArgs {
    const Group *groups;
    const int64_t *tile_prefix;  // one tile per non-empty group
    int n_groups;
    const ExpertLayers *experts;
    int d, h, precision, clamped;
    double clamp_limit;
    const void *xp;  // bf16 rows x d
    void *hp;        // bf16 rows x h
    void *yp;        // bf16 rows x d
    int sms;
    int tile_rows;  // decode_tile_rows(T): 8 or 16
    int64_t max_tiles;  // upper bound on the batch's tiles (decode_max_tiles), sizes the launch
    int *err;  // device flag: nonzero when a bounded wait expired
};
// Most tiles of tile_rows rows a batch of T tokens can make: S shared groups
// of T rows, and at most min(E, T k) routed groups of at most T rows each
// (a token picks an expert once) holding T k rows in all.
inline int64_t decode_max_tiles(int64_t T, int E, int k, int S, int tile_rows) {
    const int64_t per_group = (T + tile_rows - 1) / tile_rows;
    const int64_t routed_groups = (int64_t)E < T * k ? (int64_t)E : T * k;
    const int64_t by_rows = (T * k + tile_rows - 1) / tile_rows + routed_groups;
    const int64_t by_groups = routed_groups * per_group;
    return (int64_t)S * per_group + (by_rows < by_groups ? by_rows : by_groups);
}
bool decode_usable(int precision, int d, int h, int64_t T, int n_groups);  // n_groups = shared + routed
int launch_decode(const DecodeArgs &a, int which, cudaStream_t st);  // which: 1 gate/up, 2 down
// which: 1 = gate/up + SwiGLU into hp, 2 = down into yp
int launch_grouped_simt(const GroupedArgs &a, int which, cudaStream_t st);

// Combine (mixtureofexperts.go:182-205): out = residual + sum_s shared_s +
// sum_j gate_j * y[slot_row], in the reference's order.
struct CombineArgs {
    int64_t T;
    int d, k, S;
    const void *y;             // rows x d, y_dtype
    const void *y_routed = nullptr;  // routed rows if not in y (expert parallelism)
    int y_dtype;
    int64_t shared_row0;       // row of shared expert 0 (rows s*T + t)
    int64_t routed_row0;       // row of routed row 0
    const int64_t *slot_row;   // T x k
    const float *gates32;      // T x k
    const double *gates64;     // T x k
    const void *residual;      // NULL or T x d in out_dtype
    void *out;
    int out_dtype;
};
int launch_combine(const CombineArgs &a, cudaStream_t st);

// Quantiser (lowprecision/rows.go:38-79) and the benchmark input generator.
int launch_quantize_rows(int precision, const double *values, int64_t rows, int width, void *codes, float *scales,
                         cudaStream_t st);
int launch_fill_normal(void *dev, int dtype, int64_t n, uint64_t seed, uint64_t stream, int64_t offset, double stddev,
                       cudaStream_t st);

}  // namespace gtmoe
