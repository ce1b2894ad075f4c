/*
 * wrapper_sequence.c -- the Go drop-in's call sequence, replayed in C through
 * include/gtmoe.h.
 *
 * The reference's seam for the mixture of experts is
 * transformer.FeedForwardLayer (transformer/block.go:24-29).  A Go wrapper
 * type that satisfies it loads libgtmoe.so with purego and makes, call for
 * call, the calls below (INTEGRATION.md holds that Go code).  No Go toolchain
 * exists on this image, so this program stands in for it: it reads a
 * mixture described the way the Go structs hold it (mixtureofexperts.go:14-31,
 * perceptron/layer.go:12-25, lowprecision/rows.go:148-157), makes the same
 * decisions the Go wrapper makes and checks every return code the same way.
 *
 *   wrap():   refuse layers with a low-rank adapter (perceptron/layer.go:
 *             145-148 applies it inside Forward; the library does not), read
 *             the clamp limit from the gate activation's name
 *             ("ClampedSiLU(%g)", activationfunction/moreactivationfunctions.go:
 *             207-223), check that every expert layer is stored the same way
 *             (compressed rows of one precision, or plain float64 weights),
 *             gtmoe_create, the router (its RowsSnapshot when
 *             Model.CompressWeights compressed it too, transformer/memory.go:
 *             25-34, else its float64 weights), the balance biases, and every
 *             expert layer with its biases.
 *   then:     gtmoe_set_training, gtmoe_forward (host float64 matrices, as Go
 *             passes them), gtmoe_backward (router gradients added to the
 *             router's gradient storage), gtmoe_last_expert_load,
 *             gtmoe_update_balance, gtmoe_get_balance.  Before the backward it
 *             checks what Layer.Backward checks (perceptron/layer.go:164-167):
 *             a compressed layer must be frozen (FreezeBase); the library
 *             computes no expert weight gradients, so every expert layer must
 *             be frozen; a frozen router gets no gradients.
 *
 * Usage: wrapper_sequence <model file> <output file>
 * Exit status: 0 on success; 2 when gtmoe_create finds no usable GPU (the
 * message is printed: "gtmoe: no device: ..."); 1 on any other failure.
 *
 * Model file (little endian): "GTMW", int32 d, h, n_shared, n_routed, k,
 * hash_routing; the router layer; n_routed float64 balance biases;
 * (n_shared + n_routed) x {gate, up, down} layers; int64 T; T*d float64
 * inputs; T int64 token IDs; T*d float64 output gradients; float64 balance
 * rate.  A layer: int32 name length + name, int32 activation-name length +
 * name, int32 has_adapter, int32 freeze_base, int32 compressed, int32
 * precision, int32 rows,
 * int32 width, int64 value bytes + values (float64 weights when not
 * compressed, else the snapshot's list of that precision), int64 scale count +
 * float32 scales, rows float64 biases.
 * Output file: out (T*d float64), input gradients (T*d float64), router
 * weight gradients (n_routed*d float64), router bias gradients (n_routed
 * float64), the expert load (n_routed int64), the balance biases after the
 * update (n_routed float64).
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "gtmoe.h"

typedef struct {
    char name[128];
    char activation[64];
    int has_adapter, freeze_base, compressed, precision, rows, width;
    void *values;
    int64_t value_bytes;
    float *scales;
    int64_t n_scales;
    double *biases;
} Layer;

typedef struct {
    int d, h, n_shared, n_routed, k, hash_routing;
    Layer router;
    double *balance;
    Layer *experts; /* (n_shared + n_routed) * 3: gate, up, down */
} Mixture;

static FILE *g_in;

static void read_or_die(void *p, size_t n) {
    if (n && fread(p, 1, n, g_in) != n) {
        fprintf(stderr, "model file is short\n");
        exit(1);
    }
}
static int32_t read_i32(void) {
    int32_t v;
    read_or_die(&v, 4);
    return v;
}
static int64_t read_i64(void) {
    int64_t v;
    read_or_die(&v, 8);
    return v;
}
static void *read_block(size_t n) {
    void *p = malloc(n ? n : 1);
    if (!p) exit(1);
    read_or_die(p, n);
    return p;
}
static void read_string(char *dst, size_t cap) {
    int32_t n = read_i32();
    if (n < 0 || (size_t)n >= cap) exit(1);
    read_or_die(dst, (size_t)n);
    dst[n] = 0;
}
static void read_layer(Layer *L) {
    read_string(L->name, sizeof(L->name));
    read_string(L->activation, sizeof(L->activation));
    L->has_adapter = read_i32();
    L->freeze_base = read_i32();
    L->compressed = read_i32();
    L->precision = read_i32();
    L->rows = read_i32();
    L->width = read_i32();
    L->value_bytes = read_i64();
    L->values = read_block((size_t)L->value_bytes);
    L->n_scales = read_i64();
    L->scales = (float *)read_block((size_t)L->n_scales * 4);
    L->biases = (double *)read_block((size_t)L->rows * 8);
}

/* The Go wrapper turns a failed call into an error carrying the library's
 * message (lastError); here it is printed and the program stops. */
static void check(int rc, const char *what) {
    if (rc == 0) return;
    fprintf(stderr, "gtmoe: %s failed (%d): %s\n", what, rc, gtmoe_last_error());
    exit(rc == GTMOE_ENODEVICE ? 2 : 1);
}

/* Activation name -> (clamped, limit): "SiLU"/"Linear" or
 * "ClampedSiLU(<%g>)"/"ClampedLinear(<%g>)". */
static int parse_activation(const char *name, const char *plain, const char *clamped_prefix, int *clamped,
                            double *limit) {
    size_t n = strlen(clamped_prefix);
    if (strcmp(name, plain) == 0) {
        *clamped = 0;
        *limit = 0;
        return 0;
    }
    if (strncmp(name, clamped_prefix, n) == 0) {
        char *end = NULL;
        *limit = strtod(name + n, &end);
        if (end && strcmp(end, ")") == 0 && *limit > 0) {
            *clamped = 1;
            return 0;
        }
    }
    return -1;
}

/* precision and value pointer of a layer's weights, as the Go wrapper's
 * weightsOf(): the snapshot's list of its precision, or Weights.Values */
static int layer_precision(const Layer *L) { return L->compressed ? L->precision : GTMOE_FLOAT64; }

static gtmoe_t wrap(const Mixture *m, int device) {
    const int S = m->n_shared, E = m->n_routed;
    /* 1. layers this library cannot run */
    if (m->router.has_adapter) {
        fprintf(stderr, "layer %s has a low-rank adapter, which the GPU mixture does not apply\n", m->router.name);
        exit(1);
    }
    for (int i = 0; i < 3 * (S + E); i++)
        if (m->experts[i].has_adapter) {
            fprintf(stderr, "layer %s has a low-rank adapter, which the GPU mixture does not apply\n",
                    m->experts[i].name);
            exit(1);
        }
    /* 2. SwiGLU or clamped SwiGLU experts, all alike */
    const Layer *first = &m->experts[0];
    int clamped = 0, clamped_up = 0;
    double limit = 0, limit_up = 0;
    if (parse_activation(first[0].activation, "SiLU", "ClampedSiLU(", &clamped, &limit) ||
        parse_activation(first[1].activation, "Linear", "ClampedLinear(", &clamped_up, &limit_up) ||
        clamped != clamped_up || limit != limit_up || strcmp(first[2].activation, "Linear") != 0) {
        fprintf(stderr, "expert %s is not a SwiGLU / clamped SwiGLU feed-forward\n", first[0].name);
        exit(1);
    }
    const int precision = layer_precision(first);
    for (int i = 0; i < 3 * (S + E); i++) {
        const Layer *L = &m->experts[i];
        if (strcmp(L->activation, first[i % 3].activation) != 0 || layer_precision(L) != precision) {
            fprintf(stderr, "expert layer %s differs from %s in activation or storage\n", L->name, first[i % 3].name);
            exit(1);
        }
    }
    /* 3. the handle */
    gtmoe_config cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.d_model = m->d;
    cfg.hidden = m->h;
    cfg.n_shared = S;
    cfg.n_routed = E;
    cfg.experts_per_token = m->k;
    cfg.hash_routing = m->hash_routing;
    cfg.clamped = clamped;
    cfg.clamp_limit = limit;
    cfg.weight_precision = precision;
    gtmoe_t h = NULL;
    check(gtmoe_create(&cfg, device, &h), "gtmoe_create");
    /* 4. router (compressed or float64), balance, expert layers */
    if (!m->hash_routing) {
        const Layer *r = &m->router;
        check(gtmoe_set_router(h, layer_precision(r), r->values, r->n_scales ? r->scales : NULL, r->biases),
              "gtmoe_set_router");
    }
    check(gtmoe_set_balance(h, m->balance), "gtmoe_set_balance");
    for (int e = 0; e < S + E; e++)
        for (int which = 0; which < 3; which++) {
            const Layer *L = &m->experts[3 * e + which];
            const int kind = e < S ? GTMOE_SHARED : GTMOE_ROUTED, index = e < S ? e : e - S;
            check(gtmoe_set_expert_layer(h, kind, index, which, layer_precision(L), L->values,
                                         L->n_scales ? L->scales : NULL, L->rows, L->width, L->biases),
                  "gtmoe_set_expert_layer");
        }
    return h;
}

int main(int argc, char **argv) {
    if (argc != 3) {
        fprintf(stderr, "usage: %s <model file> <output file>\n", argv[0]);
        return 1;
    }
    g_in = fopen(argv[1], "rb");
    if (!g_in) return 1;
    char magic[4];
    read_or_die(magic, 4);
    if (memcmp(magic, "GTMW", 4) != 0) return 1;
    Mixture m;
    m.d = read_i32();
    m.h = read_i32();
    m.n_shared = read_i32();
    m.n_routed = read_i32();
    m.k = read_i32();
    m.hash_routing = read_i32();
    const int S = m.n_shared, E = m.n_routed, d = m.d;
    read_layer(&m.router);
    m.balance = (double *)read_block(8 * (size_t)E);
    m.experts = (Layer *)calloc((size_t)3 * (S + E), sizeof(Layer));
    for (int i = 0; i < 3 * (S + E); i++) read_layer(&m.experts[i]);
    const int64_t T = read_i64();
    double *x = (double *)read_block(8 * (size_t)T * d);
    int64_t *ids = (int64_t *)read_block(8 * (size_t)T);
    double *dout = (double *)read_block(8 * (size_t)T * d);
    double rate;
    read_or_die(&rate, 8);
    fclose(g_in);

    gtmoe_t h = wrap(&m, 0);
    double *out = (double *)calloc((size_t)T * d, 8), *dx = (double *)calloc((size_t)T * d, 8);
    double *wg = (double *)calloc((size_t)E * d, 8), *bg = (double *)calloc((size_t)E, 8);
    int64_t *load = (int64_t *)calloc((size_t)E, 8);
    double *balance = (double *)calloc((size_t)E, 8);
    /* Layer.SetTraining, Forward, Backward, LastExpertLoad, UpdateBalance */
    check(gtmoe_set_training(h, 1), "gtmoe_set_training");
    check(gtmoe_forward(h, x, GTMOE_DTYPE_F64, T, m.hash_routing ? ids : NULL, NULL, out, GTMOE_DTYPE_F64, NULL, NULL,
                        NULL, NULL),
          "gtmoe_forward");
    /* Layer.Backward's preconditions, before any gradient is written */
    for (int i = 0; i < 3 * (S + E); i++) {
        const Layer *L = &m.experts[i];
        if (L->compressed && !L->freeze_base) {
            fprintf(stderr,
                    "layer \"%s\": weights are compressed for running the model, call DecompressWeights before "
                    "training, or add a low-rank adapter to train around them\n",
                    L->name);
            return 1;
        }
        if (!L->freeze_base) {
            fprintf(stderr, "layer \"%s\": the GPU mixture trains around frozen experts only (FreezeBase)\n", L->name);
            return 1;
        }
    }
    const int router_grads = !m.hash_routing && !m.router.freeze_base;
    if (!m.hash_routing && m.router.compressed && !m.router.freeze_base) {
        fprintf(stderr,
                "layer \"%s\": weights are compressed for running the model, call DecompressWeights before "
                "training, or add a low-rank adapter to train around them\n",
                m.router.name);
        return 1;
    }
    check(gtmoe_backward(h, dout, GTMOE_DTYPE_F64, dx, GTMOE_DTYPE_F64, router_grads ? wg : NULL,
                         router_grads ? bg : NULL),
          "gtmoe_backward");
    check(gtmoe_last_expert_load(h, load), "gtmoe_last_expert_load");
    check(gtmoe_update_balance(h, rate), "gtmoe_update_balance");
    check(gtmoe_get_balance(h, balance), "gtmoe_get_balance");
    gtmoe_destroy(h);

    FILE *o = fopen(argv[2], "wb");
    if (!o) return 1;
    fwrite(out, 8, (size_t)T * d, o);
    fwrite(dx, 8, (size_t)T * d, o);
    fwrite(wg, 8, (size_t)E * d, o);
    fwrite(bg, 8, (size_t)E, o);
    fwrite(load, 8, (size_t)E, o);
    fwrite(balance, 8, (size_t)E, o);
    fclose(o);
    return 0;
}
