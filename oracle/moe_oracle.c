/*
 * moe_oracle.c -- CPU float64 restatement of GoTransformers' mixture-of-experts
 * forward path.  TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check
 * and the benchmark's CPU-baseline leg call this library as the checker.  The
 * product (libgtmoe.so) never links, loads or calls it.
 *
 * Every function restates one reference function; the citation is the file
 * and line in javanhut/GoTransformers.  Arithmetic follows the reference
 * exactly: float64 everywhere, sums accumulated sequentially in ascending
 * index order, block partial sums multiplied by float64(scale) for Int8/FP4
 * rows, and the same branch structure in the activations.  Go and C agree on
 * the primitive operations used here: float64 +,-,*,/ and sqrt are IEEE
 * correctly rounded in both; Go's math.Round is C round() (half away from
 * zero); float32(x) is the C cast (round to nearest even).  Go's exp/log1p
 * may differ from glibc by an ulp, which no tolerance here depends on.
 *
 * Parity pinning: the reference publishes no value-level golden vectors for
 * the MoE forward.  The oracle is pinned against the reference's own
 * known-answer tests (lowprecision_test.go:39-47 FP4 exact values,
 * lowprecision_test.go:49-64 exact byte counts) and against every property the
 * reference's mixtureofexperts_test.go checks; see tests/test_oracle.py.
 *
 * Threading: dense and compressed layer products split output neurons across
 * worker threads the way vectormath.SplitAcrossThreads does
 * (vectormath/backend.go:58-78, perceptron/layer.go:121-131); the per-element
 * arithmetic does not depend on the split, so results are identical for any
 * thread count.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define GTO_FLOAT64 0
#define GTO_FLOAT32 1
#define GTO_INT8 2
#define GTO_FP4 3

#define GTO_ACT_LINEAR 0
#define GTO_ACT_SILU 1
#define GTO_ACT_CLAMPED_SILU 2
#define GTO_ACT_CLAMPED_LINEAR 3

/* lowprecision/lowprecision.go:46 */
#define VALUES_PER_SCALE 16

/* lowprecision/lowprecision.go:48 */
static const double fp4_magnitudes[8] = {0, 0.5, 1, 1.5, 2, 3, 4, 6};
/* lowprecision/lowprecision.go:96 */
static const double fp4_halfway[7] = {0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5};
/* lowprecision/rows.go:205 */
static const double fp4_signed[16] = {0, 0.5, 1, 1.5, 2, 3, 4, 6, 0, -0.5, -1, -1.5, -2, -3, -4, -6};

/* One perceptron.Layer (perceptron/layer.go:12-25): weights rows x width as
 * stored by lowprecision.Rows (rows.go:8-18), plus float64 biases. */
typedef struct {
    int precision;
    int rows;
    int width;
    const double *f64;     /* rows*width                      */
    const float *f32;      /* rows*width                      */
    const int8_t *i8;      /* rows*width                      */
    const uint8_t *fp4;    /* rows*((width+1)/2)              */
    const float *scales;   /* rows*ceil(width/16)             */
    const double *bias;    /* rows, may be NULL (all zero)    */
} gto_layer;

/* mixtureofexperts.go:14-31 -- the parts Forward reads. layers holds
 * (n_shared + n_routed) experts x {gate, up, down}. */
typedef struct {
    int d, h, n_shared, n_routed, k;
    int hash_routing;
    int clamped;
    double clamp_limit;
    gto_layer router;          /* n_routed x d, Linear activation */
    const double *balance;     /* n_routed, may be NULL           */
    const gto_layer *layers;   /* (n_shared+n_routed)*3           */
} gto_moe;

/* ---------------------------------------------------------------- helpers */

/* lowprecision/lowprecision.go:52-54 */
int gto_scale_blocks(int width) { return (width + VALUES_PER_SCALE - 1) / VALUES_PER_SCALE; }

/* lowprecision/rows.go:34-36 */
int gto_fp4_row_bytes(int width) { return (width + 1) / 2; }

/* activationfunction/activationfunction.go:35-37 */
static double sigmoid(double x) { return 1 / (1 + exp(-x)); }

/* activationfunction/activationfunction.go:102-105 */
static double silu(double x) { return x * sigmoid(x); }

/* activationfunction/moreactivationfunctions.go:8-16 */
double gto_softplus(double x) {
    if (x > 20) return x;
    if (x < -20) return exp(x);
    return log1p(exp(x));
}

/* activationfunction/activationfunction.go:158-160 (Linear),
 * :102-105 (SiLU), moreactivationfunctions.go:207-223 (ClampedSiLU),
 * :225-243 (ClampedLinear). */
double gto_activate(int act, double limit, double x) {
    switch (act) {
    case GTO_ACT_SILU:
        return silu(x);
    case GTO_ACT_CLAMPED_SILU:
        if (x > limit) return silu(limit);
        return silu(x);
    case GTO_ACT_CLAMPED_LINEAR:
        if (x > limit) return limit;
        if (x < -limit) return -limit;
        return x;
    default:
        return x;
    }
}

/* mixtureofexperts.go:80-82 */
double gto_affinity(double logit) { return sqrt(gto_softplus(logit)); }

/* ------------------------------------------------------------ quantiser */

/* lowprecision/lowprecision.go:56-64 */
static double largest_magnitude(const double *v, int n) {
    double largest = 0.0;
    for (int i = 0; i < n; i++)
        if (fabs(v[i]) > largest) largest = fabs(v[i]);
    return largest;
}

/* lowprecision/lowprecision.go:66-78 */
static int8_t encode_int8(double value, double scale) {
    if (scale == 0) return 0;
    double rounded = round(value / scale);
    if (rounded > 127) rounded = 127;
    if (rounded < -127) rounded = -127;
    return (int8_t)rounded;
}

/* lowprecision/lowprecision.go:80-94 */
static uint8_t encode_fp4(double value, double scale) {
    if (scale == 0) return 0;
    uint8_t sign = value < 0 ? 8 : 0;
    double scaled = fabs(value) / scale;
    int idx = 0;
    while (idx < 7 && scaled > fp4_halfway[idx]) idx++;
    return (uint8_t)(sign | idx);
}

/* lowprecision/lowprecision.go:98-104 */
double gto_decode_fp4(int code, double scale) {
    double value = fp4_magnitudes[code & 7] * scale;
    return (code & 8) ? -value : value;
}

/* Rows.Append for `rows` consecutive rows (lowprecision/rows.go:38-79;
 * RowsFromMatrix rows.go:276-283).  Output arrays follow RowsSnapshot
 * (rows.go:148-157): Float64 -> double[rows*width], Float32 ->
 * float[rows*width], Int8 -> int8[rows*width] + float scales
 * [rows*blocks], FP4 -> uint8[rows*((width+1)/2)] + float scales.
 * Returns 0, or -1 for bad arguments (NewRows panics, rows.go:20-28). */
int gto_quantize_rows(int precision, int rows, int width, const double *values, void *codes, float *scales) {
    if (width <= 0 || rows < 0 || precision < GTO_FLOAT64 || precision > GTO_FP4) return -1;
    int blocks = gto_scale_blocks(width);
    for (int r = 0; r < rows; r++) {
        const double *v = values + (size_t)r * width;
        switch (precision) {
        case GTO_FLOAT64:
            memcpy((double *)codes + (size_t)r * width, v, sizeof(double) * width);
            break;
        case GTO_FLOAT32:
            for (int i = 0; i < width; i++) ((float *)codes)[(size_t)r * width + i] = (float)v[i];
            break;
        case GTO_INT8:
            for (int b = 0; b < blocks; b++) {
                int start = b * VALUES_PER_SCALE;
                int end = start + VALUES_PER_SCALE < width ? start + VALUES_PER_SCALE : width;
                double scale = largest_magnitude(v + start, end - start) / 127;
                float s32 = (float)scale;
                scales[(size_t)r * blocks + b] = s32;
                for (int i = start; i < end; i++)
                    ((int8_t *)codes)[(size_t)r * width + i] = encode_int8(v[i], (double)s32);
            }
            break;
        case GTO_FP4: {
            int row_bytes = gto_fp4_row_bytes(width);
            uint8_t *packed = (uint8_t *)codes + (size_t)r * row_bytes;
            memset(packed, 0, row_bytes);
            for (int b = 0; b < blocks; b++) {
                int start = b * VALUES_PER_SCALE;
                int end = start + VALUES_PER_SCALE < width ? start + VALUES_PER_SCALE : width;
                double scale = largest_magnitude(v + start, end - start) / 6;
                float s32 = (float)scale;
                scales[(size_t)r * blocks + b] = s32;
                for (int i = start; i < end; i++) {
                    uint8_t code = encode_fp4(v[i], (double)s32);
                    /* rows.go:68-74: low nibble holds the even element */
                    if (i % 2 == 0) packed[i / 2] = code;
                    else packed[i / 2] |= (uint8_t)(code << 4);
                }
            }
            break;
        }
        }
    }
    return 0;
}

/* Rows.Row (lowprecision/rows.go:87-119) for every row: decoded float64. */
int gto_decode_rows(const gto_layer *L, double *out) {
    int blocks = gto_scale_blocks(L->width), w = L->width;
    for (int r = 0; r < L->rows; r++) {
        for (int i = 0; i < w; i++) {
            double v = 0;
            switch (L->precision) {
            case GTO_FLOAT64: v = L->f64[(size_t)r * w + i]; break;
            case GTO_FLOAT32: v = (double)L->f32[(size_t)r * w + i]; break;
            case GTO_INT8:
                v = (double)L->i8[(size_t)r * w + i] * (double)L->scales[(size_t)r * blocks + i / VALUES_PER_SCALE];
                break;
            case GTO_FP4: {
                uint8_t packed = L->fp4[(size_t)r * gto_fp4_row_bytes(w) + i / 2];
                int code = (i % 2 == 1) ? (packed >> 4) : (packed & 15);
                v = gto_decode_fp4(code, (double)L->scales[(size_t)r * blocks + i / VALUES_PER_SCALE]);
                break;
            }
            }
            out[(size_t)r * w + i] = v;
        }
    }
    return 0;
}

/* Rows.DotRow (lowprecision/rows.go:207-257); Float64 rows and dense
 * layers use vectormath.DotProduct (vector.go:67-74): one sequential sum. */
double gto_dot_row(const gto_layer *L, int row, const double *x) {
    int w = L->width, blocks = gto_scale_blocks(w);
    double sum = 0.0;
    switch (L->precision) {
    case GTO_FLOAT64: {
        const double *v = L->f64 + (size_t)row * w;
        for (int i = 0; i < w; i++) sum += x[i] * v[i];
        break;
    }
    case GTO_FLOAT32: {
        const float *v = L->f32 + (size_t)row * w;
        for (int i = 0; i < w; i++) sum += x[i] * (double)v[i];
        break;
    }
    case GTO_INT8: {
        const int8_t *v = L->i8 + (size_t)row * w;
        for (int b = 0; b < blocks; b++) {
            int start = b * VALUES_PER_SCALE;
            int end = start + VALUES_PER_SCALE < w ? start + VALUES_PER_SCALE : w;
            double block_sum = 0.0;
            for (int i = start; i < end; i++) block_sum += x[i] * (double)v[i];
            sum += block_sum * (double)L->scales[(size_t)row * blocks + b];
        }
        break;
    }
    case GTO_FP4: {
        const uint8_t *packed = L->fp4 + (size_t)row * gto_fp4_row_bytes(w);
        for (int b = 0; b < blocks; b++) {
            int start = b * VALUES_PER_SCALE;
            int end = start + VALUES_PER_SCALE < w ? start + VALUES_PER_SCALE : w;
            double block_sum = 0.0;
            for (int i = start; i < end; i++) {
                uint8_t p = packed[i / 2];
                int code = (i % 2 == 1) ? (p >> 4) : (p & 15);
                block_sum += x[i] * fp4_signed[code];
            }
            sum += block_sum * (double)L->scales[(size_t)row * blocks + b];
        }
        break;
    }
    }
    return sum;
}

/* ------------------------------------------------------ threaded layers */

typedef struct {
    const gto_layer *L;
    int act;
    double limit;
    int n;
    const double *x;
    double *out;
    int first, last;
} layer_job;

static void *layer_worker(void *arg) {
    layer_job *j = (layer_job *)arg;
    const gto_layer *L = j->L;
    for (int neuron = j->first; neuron < j->last; neuron++) {
        double b = L->bias ? L->bias[neuron] : 0.0;
        for (int ex = 0; ex < j->n; ex++) {
            /* perceptron/layer.go:141-157: pre = x.W^T, pre += bias, act(pre) */
            double pre = gto_dot_row(L, neuron, j->x + (size_t)ex * L->width);
            pre += b;
            j->out[(size_t)ex * L->rows + neuron] = gto_activate(j->act, j->limit, pre);
        }
    }
    return NULL;
}

static int g_threads = 1;

/* Thread count for every threaded product (vectormath/backend.go:58-78 uses
 * GOMAXPROCS). */
void gto_set_threads(int n) { g_threads = n < 1 ? 1 : n; }

/* SplitAcrossThreads' threshold (vectormath/backend.go:56). */
#define WORK_BEFORE_MORE_THREADS (64 * 64 * 64)

/* perceptron.Layer.Forward (perceptron/layer.go:133-162) over n rows.
 * out is n x L->rows. */
int gto_layer_forward(const gto_layer *L, int act, double limit, int n, const double *x, double *out) {
    int items = L->rows;
    long work = (long)n * L->width;
    int nt = g_threads;
    if ((long)items * work < WORK_BEFORE_MORE_THREADS || nt == 1 || items < 2) nt = 1;
    if (nt > items) nt = items;
    int per = (items + nt - 1) / nt;
    layer_job jobs[256];
    pthread_t tids[256];
    if (nt > 256) nt = 256;
    int started = 0;
    for (int first = 0; first < items && started < nt; first += per) {
        layer_job *j = &jobs[started];
        j->L = L; j->act = act; j->limit = limit; j->n = n; j->x = x; j->out = out;
        j->first = first;
        j->last = first + per < items ? first + per : items;
        started++;
    }
    if (started == 1) {
        layer_worker(&jobs[0]);
        return 0;
    }
    for (int i = 0; i < started; i++) pthread_create(&tids[i], NULL, layer_worker, &jobs[i]);
    for (int i = 0; i < started; i++) pthread_join(tids[i], NULL);
    return 0;
}

/* GatedFeedForward.Forward (feedforward/gatedfeedforward.go:49-57) with the
 * SwiGLU activations (:30-39).  out is n x d. */
int gto_gated_forward(const gto_layer *gate, const gto_layer *up, const gto_layer *down, int clamped, double limit,
                      int n, const double *x, double *out) {
    int h = gate->rows;
    double *g = (double *)malloc(sizeof(double) * (size_t)n * h);
    double *u = (double *)malloc(sizeof(double) * (size_t)n * h);
    if (!g || !u) { free(g); free(u); return -1; }
    gto_layer_forward(gate, clamped ? GTO_ACT_CLAMPED_SILU : GTO_ACT_SILU, limit, n, x, g);
    gto_layer_forward(up, clamped ? GTO_ACT_CLAMPED_LINEAR : GTO_ACT_LINEAR, limit, n, x, u);
    /* vectormath.MultiplyMatricesEach (matrix.go:121-128) */
    for (size_t i = 0; i < (size_t)n * h; i++) g[i] = g[i] * u[i];
    gto_layer_forward(down, GTO_ACT_LINEAR, 0, n, g, out);
    free(g);
    free(u);
    return 0;
}

/* ------------------------------------------------------------- routing */

/* mixtureofexperts.go:88-96 */
void gto_hashed_experts(int64_t token_id, int E, int k, int32_t *chosen) {
    uint64_t first = ((uint64_t)token_id * 2654435761ULL + 12345ULL) % (uint64_t)E;
    for (int i = 0; i < k; i++) chosen[i] = (int32_t)((first + (uint64_t)i) % (uint64_t)E);
}

/* mixtureofexperts.go:98-112: stable descending sort by
 * affinity+balance, keep k, sort ascending.  Repeated first-maximum
 * selection is the same as the first k of a stable descending sort. */
void gto_routed_experts(const double *aff, const double *balance, int E, int k, int32_t *chosen) {
    char *taken = (char *)calloc((size_t)E, 1);
    for (int i = 0; i < k; i++) {
        int best = -1;
        double best_score = 0;
        for (int e = 0; e < E; e++) {
            if (taken[e]) continue;
            double s = aff[e] + (balance ? balance[e] : 0.0);
            if (best < 0 || s > best_score) { best = e; best_score = s; }
        }
        taken[best] = 1;
        chosen[i] = best;
    }
    free(taken);
    /* sort.Ints */
    for (int i = 1; i < k; i++) {
        int32_t v = chosen[i];
        int j = i - 1;
        while (j >= 0 && chosen[j] > v) { chosen[j + 1] = chosen[j]; j--; }
        chosen[j + 1] = v;
    }
}

/* The routing half of Forward (mixtureofexperts.go:137-173): chosen experts
 * and gates for every token, optionally the router logits. */
int gto_moe_route(const gto_moe *m, int T, const double *x, const int64_t *token_ids, int32_t *chosen,
                  double *gates, double *logits_out) {
    int E = m->n_routed, k = m->k;
    if (E < 1 || k < 1 || k > E || m->n_shared < 0) return -2;
    if (m->hash_routing && !token_ids && T > 0) return -3;
    if (m->hash_routing) {
        for (int t = 0; t < T; t++) {
            if (token_ids[t] < 0) return -4;
            gto_hashed_experts(token_ids[t], E, k, chosen + (size_t)t * k);
            for (int i = 0; i < k; i++) gates[(size_t)t * k + i] = 1 / (double)k;
        }
        return 0;
    }
    double *logits = (double *)malloc(sizeof(double) * (size_t)(T > 0 ? T : 1) * E);
    double *aff = (double *)malloc(sizeof(double) * (size_t)E);
    gto_layer_forward(&m->router, GTO_ACT_LINEAR, 0, T, x, logits);
    for (int t = 0; t < T; t++) {
        const double *lt = logits + (size_t)t * E;
        for (int e = 0; e < E; e++) aff[e] = gto_affinity(lt[e]);
        int32_t *c = chosen + (size_t)t * k;
        gto_routed_experts(aff, m->balance, E, k, c);
        double total = 0.0;
        for (int i = 0; i < k; i++) total += aff[c[i]];
        for (int i = 0; i < k; i++) gates[(size_t)t * k + i] = aff[c[i]] / total;
    }
    if (logits_out) memcpy(logits_out, logits, sizeof(double) * (size_t)T * E);
    free(aff);
    free(logits);
    return 0;
}

/* MixtureOfExperts.Forward (mixtureofexperts.go:122-216).
 *   x: T x d;  token_ids: T (needed for hash routing, else may be NULL)
 *   out: T x d (the MoE output, no residual)
 * Optional outputs (NULL to skip):
 *   chosen T x k, gates T x k (in the reference's chosen order),
 *   perm T*k (rowsForExpert concatenated for e = 0..E-1),
 *   load E (lastExpertLoad), logits T x E (router logits, routed only).
 * Returns 0, or a negative value for the misuse the reference panics on. */
int gto_moe_forward(const gto_moe *m, int T, const double *x, const int64_t *token_ids, double *out,
                    int32_t *chosen_out, double *gates_out, int32_t *perm_out, int64_t *load_out,
                    double *logits_out) {
    int d = m->d, E = m->n_routed, k = m->k;
    if (E < 1 || k < 1 || k > E || m->n_shared < 0) return -2;
    if (m->hash_routing && !token_ids && T > 0) return -3;
    int32_t *chosen = (int32_t *)malloc(sizeof(int32_t) * (size_t)(T > 0 ? T : 1) * k);
    double *gates = (double *)malloc(sizeof(double) * (size_t)(T > 0 ? T : 1) * k);
    int rc = gto_moe_route(m, T, x, token_ids, chosen, gates, logits_out);
    if (rc != 0) {
        free(chosen);
        free(gates);
        return rc;
    }

    /* rowsForExpert (:175-180): token-ascending per expert */
    int64_t *load = (int64_t *)calloc((size_t)E, sizeof(int64_t));
    for (size_t i = 0; i < (size_t)T * k; i++) load[chosen[i]]++;
    int64_t *start = (int64_t *)calloc((size_t)E + 1, sizeof(int64_t));
    for (int e = 0; e < E; e++) start[e + 1] = start[e] + load[e];
    int32_t *rows_for = (int32_t *)malloc(sizeof(int32_t) * (size_t)(T > 0 ? T : 1) * k);
    int64_t *pos_of = (int64_t *)malloc(sizeof(int64_t) * (size_t)(T > 0 ? T : 1) * k);
    int64_t *fill = (int64_t *)calloc((size_t)E, sizeof(int64_t));
    for (int t = 0; t < T; t++)
        for (int i = 0; i < k; i++) {
            int e = chosen[(size_t)t * k + i];
            int64_t p = start[e] + fill[e]++;
            rows_for[p] = t;
            pos_of[(size_t)t * k + i] = p - start[e]; /* indexOf(rowsForExpert[e], t) */
        }

    /* shared experts (:182-185): outputs = 0 + s_0 + s_1 ... */
    memset(out, 0, sizeof(double) * (size_t)T * d);
    double *tmp = (double *)malloc(sizeof(double) * (size_t)(T > 0 ? T : 1) * d);
    for (int s = 0; s < m->n_shared; s++) {
        const gto_layer *L = m->layers + 3 * s;
        gto_gated_forward(&L[0], &L[1], &L[2], m->clamped, m->clamp_limit, T, x, tmp);
        for (size_t i = 0; i < (size_t)T * d; i++) out[i] = out[i] + tmp[i];
    }
    free(tmp);

    /* routed experts (:187-195) over gathered rows */
    double **yexp = (double **)calloc((size_t)E, sizeof(double *));
    for (int e = 0; e < E; e++) {
        int64_t n = load[e];
        if (n == 0) continue;
        double *gathered = (double *)malloc(sizeof(double) * (size_t)n * d);
        for (int64_t i = 0; i < n; i++)
            memcpy(gathered + (size_t)i * d, x + (size_t)rows_for[start[e] + i] * d, sizeof(double) * d);
        yexp[e] = (double *)malloc(sizeof(double) * (size_t)n * d);
        const gto_layer *L = m->layers + 3 * (m->n_shared + e);
        gto_gated_forward(&L[0], &L[1], &L[2], m->clamped, m->clamp_limit, (int)n, gathered, yexp[e]);
        free(gathered);
    }

    /* combine (:197-205): chosen order, out += gate * y */
    for (int t = 0; t < T; t++) {
        double *orow = out + (size_t)t * d;
        for (int i = 0; i < k; i++) {
            int e = chosen[(size_t)t * k + i];
            const double *yrow = yexp[e] + (size_t)pos_of[(size_t)t * k + i] * d;
            double g = gates[(size_t)t * k + i];
            for (int j = 0; j < d; j++) orow[j] += g * yrow[j];
        }
    }

    if (chosen_out) memcpy(chosen_out, chosen, sizeof(int32_t) * (size_t)T * k);
    if (gates_out) memcpy(gates_out, gates, sizeof(double) * (size_t)T * k);
    if (perm_out) memcpy(perm_out, rows_for, sizeof(int32_t) * (size_t)T * k);
    if (load_out) memcpy(load_out, load, sizeof(int64_t) * E);
    for (int e = 0; e < E; e++) free(yexp[e]);
    free(yexp);
    free(fill);
    free(pos_of);
    free(rows_for);
    free(start);
    free(load);
    free(gates);
    free(chosen);
    return 0;
}

/* MixtureOfExperts.UpdateBalance (mixtureofexperts.go:293-310). */
void gto_update_balance(double *balance, const int64_t *load, int E, double rate) {
    int64_t total = 0;
    for (int e = 0; e < E; e++) total += load[e];
    double average = (double)total / (double)E;
    for (int e = 0; e < E; e++) {
        if ((double)load[e] < average) balance[e] += rate;
        if ((double)load[e] > average) balance[e] -= rate;
    }
}

/* ------------------------------------------- seeded benchmark inputs */

/* Not a reference function: the benchmark's synthetic inputs, so that the
 * CPU reference arm of bench.py can make its weights without the GPU library.
 * Value j of stream (seed, stream) is a pure function of those numbers --
 * SplitMix64 + Box-Muller, the definition written out in
 * gotransformers_b200/synthetic.py (which the library's GPU generator follows
 * too; libm and CUDA's log/cos may differ in the last bit of a value):
 *   key = splitmix64(seed ^ (stream * 0xD1B54A32D192ED03))
 *   a, b = splitmix64(key + 2j), splitmix64(key + 2j + 1)
 *   u1 = ((a >> 11) + 1) * 2^-53, u2 = (b >> 11) * 2^-53
 *   z = sqrt(-2 ln u1) * cos(2 pi u2)                                     */
static uint64_t splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static double synth_normal(uint64_t key, uint64_t j) {
    const uint64_t a = splitmix64(key + 2 * j), b = splitmix64(key + 2 * j + 1);
    const double u1 = ((double)(a >> 11) + 1.0) * 0x1p-53;
    const double u2 = (double)(b >> 11) * 0x1p-53;
    return sqrt(-2.0 * log(u1)) * cos(2.0 * M_PI * u2);
}

typedef struct {
    int precision, width;
    uint64_t key;
    double stddev;
    int first, last;
    unsigned char *codes;
    float *scales;
    size_t row_bytes;
    int blocks;
    int rc;
} synth_job;

static void *synth_worker(void *arg) {
    synth_job *j = (synth_job *)arg;
    double *row = (double *)malloc(sizeof(double) * (size_t)j->width);
    if (!row) {
        j->rc = -1;
        return NULL;
    }
    for (int r = j->first; r < j->last; r++) {
        for (int i = 0; i < j->width; i++)
            row[i] = j->stddev * synth_normal(j->key, (uint64_t)r * (uint64_t)j->width + (uint64_t)i);
        /* lowprecision.Rows.Append, one row at a time (rows.go:38-79) */
        int rc = gto_quantize_rows(j->precision, 1, j->width, row, j->codes + (size_t)r * j->row_bytes,
                                   j->scales ? j->scales + (size_t)r * j->blocks : NULL);
        if (rc) j->rc = rc;
    }
    free(row);
    return NULL;
}

/* rows x width values stddev * z (value index r*width + i of the stream),
 * quantised row by row into the RowsSnapshot arrays of `precision`. */
int gto_synth_rows(int precision, int rows, int width, uint64_t seed, uint64_t stream, double stddev, void *codes,
                   float *scales, int threads) {
    if (rows < 0 || width < 1) return -1;
    const uint64_t key = splitmix64(seed ^ (stream * 0xD1B54A32D192ED03ull));
    size_t row_bytes = precision == GTO_FLOAT64   ? 8 * (size_t)width
                       : precision == GTO_FLOAT32 ? 4 * (size_t)width
                       : precision == GTO_INT8    ? (size_t)width
                                                  : (size_t)gto_fp4_row_bytes(width);
    int nt = threads < 1 ? 1 : threads > 256 ? 256 : threads;
    if (nt > rows) nt = rows < 1 ? 1 : rows;
    synth_job jobs[256];
    pthread_t tids[256];
    int per = (rows + nt - 1) / nt, rc = 0;
    for (int t = 0; t < nt; t++) {
        int first = t * per, last = first + per < rows ? first + per : rows;
        jobs[t] = (synth_job){precision, width, key, stddev, first, last, (unsigned char *)codes,
                              (precision == GTO_INT8 || precision == GTO_FP4) ? scales : NULL, row_bytes,
                              gto_scale_blocks(width), 0};
        if (nt > 1) pthread_create(&tids[t], NULL, synth_worker, &jobs[t]);
        else synth_worker(&jobs[t]);
    }
    for (int t = 0; t < nt; t++) {
        if (nt > 1) pthread_join(tids[t], NULL);
        if (jobs[t].rc) rc = jobs[t].rc;
    }
    return rc;
}
