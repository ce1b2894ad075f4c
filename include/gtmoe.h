/*
 * gtmoe.h -- C ABI of libgtmoe.so, a B200 (sm_100a) implementation of the
 * forward path of GoTransformers' mixtureofexperts package.
 *
 * The Go reference has no FFI for this path; its seam is the
 * transformer.FeedForwardLayer interface (transformer/block.go:24-29) that
 * *mixtureofexperts.MixtureOfExperts implements.  A Go wrapper type loads this
 * library at run time with purego, the way gpu/library_unix.go:19-33 and
 * gpu/vulkan.go:443-518 load Vulkan, so CGO_ENABLED=0 builds keep working.
 * Every entry point below names the reference function it replaces.
 *
 * Conventions
 *  - Every function returning int returns 0 on success or a negative
 *    GTMOE_E* code; gtmoe_last_error() then holds a message for the calling
 *    thread.  Argument errors are the misuse the reference panics on.
 *  - Pointers may be host memory (Go slices) or CUDA device memory; the
 *    library detects which.  Host pointers are only read or written during
 *    the call.  Weights are copied to the device at set time.
 *  - A handle serialises its own calls with a mutex; separate handles may be
 *    used from separate threads.
 *  - There is no CPU fallback: without a usable sm_100 GPU gtmoe_create
 *    fails with GTMOE_ENODEVICE.
 */
#ifndef GTMOE_H
#define GTMOE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define GTMOE_API __attribute__((visibility("default")))
#else
#define GTMOE_API
#endif

#define GTMOE_VERSION 100

/* lowprecision.Precision (lowprecision/lowprecision.go:9-16). */
#define GTMOE_FLOAT64 0
#define GTMOE_FLOAT32 1
#define GTMOE_INT8 2
#define GTMOE_FP4 3

/* Element types of activations passed across the boundary. */
#define GTMOE_DTYPE_F64 0
#define GTMOE_DTYPE_F32 1
#define GTMOE_DTYPE_BF16 2

/* Which experts / which layer of a GatedFeedForward
 * (feedforward/gatedfeedforward.go:11-16). */
#define GTMOE_SHARED 0
#define GTMOE_ROUTED 1
#define GTMOE_GATE 0
#define GTMOE_UP 1
#define GTMOE_DOWN 2

/* Error codes. */
#define GTMOE_OK 0
#define GTMOE_EINVAL (-1)    /* bad argument (the reference panics)        */
#define GTMOE_ENODEVICE (-2) /* no usable sm_100 device                    */
#define GTMOE_ECUDA (-3)     /* CUDA runtime error                         */
#define GTMOE_ENOTREADY (-4) /* weights missing, or Forward not yet called */
#define GTMOE_ENOMEM (-5)    /* device allocation failed                   */
#define GTMOE_ETIMEOUT (-6)  /* a bounded device-side wait gave up         */
#define GTMOE_ENCCL (-7)     /* NCCL error (expert parallel only)          */

/* Constructor arguments of NewMixtureOfExperts / NewClampedMixtureOfExperts
 * (mixtureofexperts/mixtureofexperts.go:33-70) plus the precision that
 * Layer.CompressWeights gave the expert layers (perceptron/layer.go:52-61). */
typedef struct gtmoe_config {
    int32_t d_model;           /* vectorSize                                */
    int32_t hidden;            /* expertHiddenSize                          */
    int32_t n_shared;          /* numberOfSharedExperts  (>= 0)             */
    int32_t n_routed;          /* numberOfRoutedExperts  (>= 1)             */
    int32_t experts_per_token; /* expertsPerToken, 1..n_routed              */
    int32_t hash_routing;      /* MixtureOfExperts.UseHashRouting           */
    int32_t clamped;           /* 1 = NewClampedMixtureOfExperts            */
    int32_t weight_precision;  /* GTMOE_FLOAT64/FLOAT32/INT8/FP4 of experts */
    double clamp_limit;        /* clampLimit (> 0 when clamped)             */
} gtmoe_config;

typedef struct gtmoe_handle *gtmoe_t;

/* GTMOE_VERSION of the loaded library. */
GTMOE_API int gtmoe_version(void);

/* Message for the last failed call on this thread ("" if none). */
GTMOE_API const char *gtmoe_last_error(void);

/* buildMixtureOfExperts (mixtureofexperts.go:47-70): validates the same
 * arguments and creates a handle on CUDA device `device`.  Weights start
 * unset; Forward fails with GTMOE_ENOTREADY until every layer is set. */
GTMOE_API int gtmoe_create(const gtmoe_config *cfg, int device, gtmoe_t *out);

/* Expert-parallel variant: this process is rank `rank` of `n_ranks`, one per
 * GPU.  Routed experts are owned contiguously by index, E/n_ranks per rank
 * (E must divide evenly).  Router and shared experts are replicated.
 * nccl_id is the 128-byte ncclUniqueId from gtmoe_ep_unique_id() on rank 0,
 * distributed by the caller.  No counterpart in the reference (it has no
 * multi-GPU MoE); Forward keeps the reference's per-token semantics. */
GTMOE_API int gtmoe_ep_unique_id(void *nccl_id_128);
GTMOE_API int gtmoe_create_ep(const gtmoe_config *cfg, int device, int n_ranks, int rank, const void *nccl_id_128,
                    gtmoe_t *out);

/* Hot-expert replicas of an expert-parallel handle (opt-in; no counterpart in
 * the reference, which has no multi-GPU MoE).  The n routed experts listed in
 * `experts` (host int32, distinct) are held by EVERY rank: each rank computes
 * their rows for its own tokens, the way it computes the shared experts, so
 * those rows never cross NVLink and never queue on the owning rank.  Every
 * other routed expert stays owned by index.  Under a skewed router (a few
 * experts that nearly every token picks) this evens out the ranks' work.
 * Results are those of the plain layout (a row's arithmetic does not depend on
 * where it runs).  Call it identically on every rank, before the first
 * Forward; then set the listed experts' layers on every rank too
 * (gtmoe_set_expert_layer accepts owned and replicated experts).  A later call
 * replaces the list; n = 0 drops it.  GTMOE_EINVAL on a single-GPU handle. */
GTMOE_API int gtmoe_ep_set_replicas(gtmoe_t h, int n, const int32_t *experts);

/* The mixture-of-experts half of transformer.Block.Forward (block.go:72-77,
 * no hyper-connections, dropout off): out = x + Forward(RMSNorm(x)), in one
 * call.  gtmoe_set_norm sets the block's FeedForwardNorm (RMSNorm weights,
 * d_model float64, and epsilon; normalization/rmsnorm.go:10-31);
 * gtmoe_forward_block normalizes on the GPU in float64 exactly as
 * RMSNorm.Forward (:33-53) does, routes and runs the experts on the
 * normalized rows and adds x.  out_dtype must equal x_dtype.  The optional
 * routing outputs are gtmoe_forward's.  One GPU (not expert parallel).  No
 * counterpart in the reference's MoE API. */
GTMOE_API int gtmoe_set_norm(gtmoe_t h, const double *weights, double epsilon);
GTMOE_API int gtmoe_forward_block(gtmoe_t h, const void *x, int x_dtype, int64_t T, const int64_t *token_ids,
                                  void *out, int out_dtype, int32_t *chosen, double *gates, int32_t *perm,
                                  int64_t *load);

/* MixtureOfExperts.Backward (mixtureofexperts.go:227-285) for the last
 * Forward.  gtmoe_set_training(h, 1) makes every later Forward keep what the
 * backward needs (its input rows as float64, the chosen experts, the gates
 * and the expert-sorted token lists; a host-buffer batch then runs unchunked).
 * gtmoe_backward takes the output gradients dout (T x d_model, the last
 * Forward's T) and writes the input gradients dx (T x d_model); when
 * router_weight_grad (n_routed x d_model) / router_bias_grad (n_routed) are
 * given, the router's gradients are ADDED to them, as the reference's
 * RouterLayer.Backward accumulates into its gradient storage
 * (perceptron/layer.go:184-195).  The expert layers are compressed rows and
 * take part as frozen layers (layer.go:165-167, 184: no weight gradients;
 * input gradients through the rows, adapter.go:108-120).  Computed in float64
 * on the GPU; the gate/up/down values are recomputed from the saved input.
 * Hash routing: no router term (:258-260).  GTMOE_ENOTREADY without a
 * Forward since training was switched on; one GPU (not expert parallel). */
GTMOE_API int gtmoe_set_training(gtmoe_t h, int on);
GTMOE_API int gtmoe_backward(gtmoe_t h, const void *dout, int dout_dtype, void *dx, int dx_dtype,
                             double *router_weight_grad, double *router_bias_grad);

/* GoTransformers binary weights files (weightfile/binaryfile.go): a saved
 * model's parameters read straight into a handle.  gtmoe_weightfile_open maps
 * the file, checks its marker (GOTRANSFORMERS-WEIGHTS-1 or -2,
 * binaryfile.go:13-14) and indexes every parameter record the way
 * ReadBinaryKeepingCompressed walks them (:157-230), with the same checks on
 * names, counts and sizes (and RowsFromSnapshot's, lowprecision/rows.go:
 * 172-203); errors are GTMOE_EINVAL with the reference's message.  Host only:
 * needs no GPU.  No counterpart in the reference's MoE API (it loads through
 * weightfile.ReadBinaryKeepingCompressed into Go memory). */
typedef struct gtmoe_weightfile *gtmoe_wf_t;
GTMOE_API int gtmoe_weightfile_open(const char *path, gtmoe_wf_t *out);
GTMOE_API void gtmoe_weightfile_close(gtmoe_wf_t wf);
GTMOE_API int gtmoe_weightfile_count(gtmoe_wf_t wf);
/* Parameter i: its name (valid until close), how it is stored (1 float64,
 * 2 float32, 3 bfloat16, 4 compressed rows, binaryfile.go:16-21); for
 * compressed rows its precision (GTMOE_FLOAT64..GTMOE_FP4), rows and width
 * (-1, 0, 0 otherwise); values = rows*width or the dense value count. */
GTMOE_API int gtmoe_weightfile_info(gtmoe_wf_t wf, int i, const char **name, int *stored_as, int *precision,
                                    int64_t *rows, int64_t *width, int64_t *values);
/* gtmoe_set_expert_layer from the file: `weights` names a compressed-rows
 * parameter (its RowsSnapshot lists go to the device as they are in the file)
 * or a dense one (float64 layer; float32/bfloat16 values widened as
 * ReadBinary does); `bias` a dense parameter of `rows` values or NULL. */
GTMOE_API int gtmoe_weightfile_set_expert_layer(gtmoe_wf_t wf, gtmoe_t h, int kind, int index, int which,
                                                const char *weights, const char *bias);
/* gtmoe_set_router from the file (E x d weights, E-value bias or NULL). */
GTMOE_API int gtmoe_weightfile_set_router(gtmoe_wf_t wf, gtmoe_t h, const char *weights, const char *bias);

/* Frees every device allocation of the handle.  NULL is ignored. */
GTMOE_API void gtmoe_destroy(gtmoe_t h);

/* Runs the handle's work on `stream` (a cudaStream_t; NULL = the handle's
 * own stream). */
GTMOE_API int gtmoe_set_stream(gtmoe_t h, void *stream);

/* CUDA-graph replay (default on).  A Forward with device pointers for x, out
 * and residual (no hash routing) that repeats the previous call exactly --
 * same T, pointers and dtypes, and no weight buffer reallocated since -- is
 * captured on its second occurrence and replayed as one CUDA graph from then
 * on, the way a generation loop calls the mixture once per token
 * (transformer/block.go:111-128).  No counterpart in the reference.  Timing
 * (gtmoe_set_timing) runs the forward without graphs. */
GTMOE_API int gtmoe_set_graphs(gtmoe_t h, int on);

/* RouterLayer weights and biases (perceptron.Layer d -> E, Linear;
 * mixtureofexperts.go:60; Layer.SetWeights/SetBiases layer.go:234-254).
 * precision GTMOE_FLOAT64 takes values = double[E*d] and scales = NULL;
 * a compressed router (transformer/memory.go:25-34 compresses it too) takes
 * the RowsSnapshot arrays as in gtmoe_set_expert_layer.  bias = double[E] or
 * NULL for zeros. */
GTMOE_API int gtmoe_set_router(gtmoe_t h, int precision, const void *values, const float *scales, const double *bias);

/* MixtureOfExperts.BalanceBiases (mixtureofexperts.go:21), double[E]. */
GTMOE_API int gtmoe_set_balance(gtmoe_t h, const double *balance);
GTMOE_API int gtmoe_get_balance(gtmoe_t h, double *balance);

/* One perceptron.Layer of one expert, as lowprecision.Rows.Snapshot()
 * returns it (lowprecision/rows.go:148-170; Layer.SetCompressedWeights
 * layer.go:63-73):
 *   GTMOE_FLOAT64: values = double[rows*width],  scales = NULL
 *   GTMOE_FLOAT32: values = float[rows*width],   scales = NULL
 *   GTMOE_INT8:    values = int8[rows*width],    scales = float[rows*ceil(width/16)]
 *   GTMOE_FP4:     values = uint8[rows*((width+1)/2)] (low nibble = even
 *                  element), scales = float[rows*ceil(width/16)]
 * gate/up are hidden x d_model, down is d_model x hidden (outputs x inputs,
 * row-major, layer.go:34).  bias = double[rows] or NULL for zeros.
 * precision must equal cfg.weight_precision. */
GTMOE_API int gtmoe_set_expert_layer(gtmoe_t h, int kind, int index, int which, int precision, const void *values,
                           const float *scales, int rows, int width, const double *bias);

/* MixtureOfExperts.Forward (mixtureofexperts.go:122-216).
 *   x         T x d_model, x_dtype GTMOE_DTYPE_*
 *   token_ids T int64 ids; required with hash routing, else may be NULL
 *   residual  NULL, or T x d_model in out_dtype: added to the output (the
 *             residual of transformer.Block.Forward, block.go:77; the
 *             reference's Forward itself returns no residual)
 *   out       T x d_model in out_dtype
 * Optional (NULL to skip), all in the reference's order:
 *   chosen    int32[T*k]  lastChosenExperts
 *   gates     double[T*k] lastGates
 *   perm      int32[T*k]  lastRowsForExpert concatenated, e = 0..E-1
 *   load      int64[E]    lastExpertLoad
 * In expert-parallel handles T, x, out and the optional outputs are this
 * rank's tokens: perm lists their rows in expert order and load counts them
 * per expert (all n_routed experts).  Forward is then a collective step:
 * every rank calls it once per step, in the same order.  A rank that cannot
 * run a step calls it with T = -1 (any argument error does the same): the
 * step then fails on every rank with GTMOE_EINVAL and the handles stay
 * usable.  A device wait for the other ranks' counts or rows that runs out
 * (about 2 s; e.g. a rank that does not call Forward for the step) fails the
 * step with GTMOE_ETIMEOUT and leaves the handle unusable.
 * With host output pointers the call returns after the results are there;
 * with device pointers it is asynchronous on the handle's stream. */
GTMOE_API int gtmoe_forward(gtmoe_t h, const void *x, int x_dtype, int64_t T, const int64_t *token_ids, const void *residual,
                  void *out, int out_dtype, int32_t *chosen, double *gates, int32_t *perm, int64_t *load);

/* MixtureOfExperts.LastExpertLoad (mixtureofexperts.go:287-291), int64[E]
 * (this rank's tokens under expert parallelism; gtmoe_update_balance uses the
 * sum over ranks).  GTMOE_ENOTREADY before the first Forward. */
GTMOE_API int gtmoe_last_expert_load(gtmoe_t h, int64_t *load);

/* MixtureOfExperts.UpdateBalance (mixtureofexperts.go:293-310) from the last
 * Forward's load.  No-op with hash routing or before the first Forward. */
GTMOE_API int gtmoe_update_balance(gtmoe_t h, double rate);

/* Per-phase device timing, the counterpart of the reference's
 * gpu.Recorder.MeasureTime (gpu/compute.go:653-693).  While enabled, each
 * Forward records CUDA events on its stream between its phases:
 *   0 router, 1 dispatch, 2 gather, 3 expert gate/up, 4 expert down,
 *   5 combine, 6 expert-parallel send, 7 expert-parallel return.
 * gtmoe_read_timing waits for the stream, adds the milliseconds of each phase
 * over all Forward calls since the last read into ms[0..n_phases-1], stores
 * the number of calls and of kernels the library launched in them, and
 * resets the record. */
#define GTMOE_N_PHASES 8
GTMOE_API int gtmoe_set_timing(gtmoe_t h, int enable);
GTMOE_API int gtmoe_read_timing(gtmoe_t h, double *ms, int n_phases, int64_t *calls, int64_t *kernel_launches);

/* Routing only, allocating nothing.  No counterpart in the reference.  For
 * callers that cannot allocate device memory while they run -- a
 * token-by-token generation loop, where a cudaMalloc would synchronise the
 * device between tokens, or a server that plans its device memory up front --
 * this runs the router of gtmoe_forward (logits, exact top-k, gates) with its
 * scratch in a fixed array of about 4.3 MB that the library holds on every
 * GPU it is loaded on until exit.  Limits: T <= 65536, T * n_routed <= 262144,
 * T * experts_per_token <= 524288; larger calls fail with GTMOE_EINVAL.  x,
 * chosen (int32[T*k]), gates (double[T*k]) and, with hash routing, token_ids
 * are device pointers; the results equal gtmoe_forward's chosen and gates.
 * Asynchronous on the handle's stream.  The first call on a device looks the
 * array up and should come before any stream capture.  Calls share the array:
 * calls that overlap on the GPU race.
 * Errors of the kernels themselves are reported by the NEXT call: a call
 * first waits for the work already queued on the handle's stream, and if an
 * earlier call recorded a failure -- a bounded device wait of the router that
 * ran out, or, with hash routing, a negative token ID (the reference panics,
 * mixtureofexperts.go:141-143; token_ids are device memory here and are not
 * checked on the host) -- it returns GTMOE_ETIMEOUT or GTMOE_EINVAL without
 * routing: that earlier call's chosen and gates are invalid. */
GTMOE_API int gtmoe_route_noalloc(gtmoe_t h, const void *x, int x_dtype, int64_t T, const int64_t *token_ids,
                                  int32_t *chosen, double *gates);

/* The library's failure path on a device, without a fault; no counterpart in
 * the reference.  Every device-side wait of this library is bounded (2 s of
 * %globaltimer): on expiry the kernel records an error code, stops and
 * returns, the call reports GTMOE_ETIMEOUT and the CUDA context stays
 * usable.  This runs that bounded wait on an mbarrier nothing completes and
 * returns GTMOE_ETIMEOUT once the wait has given up and been reported -- the
 * expected result; any other code means the failure path does not work on
 * this device.  Takes about two seconds; allocates 4 bytes. */
GTMOE_API int gtmoe_bounded_wait_selftest(int device);

/* lowprecision.RowsFromMatrix (lowprecision/rows.go:276-283, Rows.Append
 * rows.go:38-79) on the GPU: quantises rows x width float64 values into the
 * RowsSnapshot arrays described above.  Bit-identical to the reference
 * quantiser.  Any mix of host and device pointers. */
GTMOE_API int gtmoe_quantize_rows(int precision, const double *values, int64_t rows, int width, void *codes, float *scales);

/* Benchmark input generator, no counterpart in the reference: fills n values
 * of dtype on device memory `dev` with stddev * N(0,1) samples; value j is
 * sample offset+j of stream (seed, stream), derived only from those numbers
 * by SplitMix64 + Box-Muller (the definition in synthetic.py). */
GTMOE_API int gtmoe_fill_normal(void *dev, int dtype, int64_t n, uint64_t seed, uint64_t stream, int64_t offset,
                      double stddev);

#ifdef __cplusplus
}
#endif
#endif
