/*
 * oracle.c - CPU restatement of the reference's f64 oracles.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Compiled with -ffp-contract=off
 * so that f32 expressions round exactly as written.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ threading */

typedef void (*range_fn)(void* ctx, uint64_t begin, uint64_t end);
typedef struct {
    range_fn fn;
    void* ctx;
    uint64_t begin, end;
} range_job;

static void* run_range(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->ctx, j->begin, j->end);
    return NULL;
}

/* Runs fn over [0, n) split into `threads` contiguous ranges. */
static void parallel_for(uint64_t n, int threads, range_fn fn, void* ctx) {
    if (threads <= 1 || n < 2) {
        fn(ctx, 0, n);
        return;
    }
    if ((uint64_t)threads > n) threads = (int)n;
    pthread_t* tid = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    range_job* jobs = (range_job*)calloc((size_t)threads, sizeof(range_job));
    for (int t = 0; t < threads; ++t) {
        jobs[t].fn = fn;
        jobs[t].ctx = ctx;
        jobs[t].begin = n * (uint64_t)t / (uint64_t)threads;
        jobs[t].end = n * (uint64_t)(t + 1) / (uint64_t)threads;
        pthread_create(&tid[t], NULL, run_range, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(tid);
    free(jobs);
}

static uint64_t product(const uint64_t* d, int n) {
    uint64_t p = 1;
    for (int i = 0; i < n; ++i) p *= d[i];
    return p;
}

/* coordinates() (conformance/convolution.rs:11-18). */
static void coords_of(uint64_t flat, const uint64_t* dims, int rank, uint64_t* out) {
    for (int a = rank - 1; a >= 0; --a) {
        out[a] = flat % dims[a];
        flat /= dims[a];
    }
}

/* address() with unit-dim broadcasting (conformance/convolution.rs:19-23). */
static uint64_t address(const uint64_t* dims, const uint64_t* coords, int rank) {
    uint64_t off = 0;
    for (int a = 0; a < rank; ++a) off = off * dims[a] + (dims[a] == 1 ? 0 : coords[a]);
    return off;
}

/* ----------------------------------------------------------------- data */

void oracle_data(uint64_t n, uint64_t seed, float* out) {
    for (uint64_t i = 0; i < n; ++i) out[i] = (float)((i * 17 + i / 19 + seed * 7) % 43) / 16.0f - 1.25f;
}

/* ----------------------------------------------------------------- conv */

int oracle_conv_dims(const uint64_t* in_dims, const uint64_t* w_dims, int rank, const uint64_t* strides,
                     const uint64_t* dilations, const uint64_t* pad_before, const uint64_t* pad_after,
                     uint64_t* out_dims) {
    int spatial = rank - 2;
    out_dims[0] = in_dims[0];
    out_dims[1] = w_dims[0];
    for (int a = 0; a < spatial; ++a) {
        __int128 length = (__int128)in_dims[a + 2] + pad_before[a] + pad_after[a];
        __int128 window = ((__int128)w_dims[a + 2] - 1) * dilations[a] + 1;
        out_dims[a + 2] = length < window ? 0 : (uint64_t)((length - window) / strides[a] + 1);
    }
    return rank;
}

typedef struct {
    const uint64_t *in_dims, *w_dims, *strides, *dilations, *pad_before, *pad_after;
    const float *in, *w;
    int rank;
    uint64_t groups;
    uint64_t out_dims[5];
    double* out64;
    float* out32;
} conv_ctx;

static void conv_range(void* p, uint64_t begin, uint64_t end) {
    conv_ctx* c = (conv_ctx*)p;
    const int spatial = c->rank - 2;
    const uint64_t kvol = product(c->w_dims + 2, spatial);
    uint64_t out[5], k[3], src[5], filt[5];
    for (uint64_t flat = begin; flat < end; ++flat) {
        coords_of(flat, c->out_dims, c->rank, out);
        const uint64_t group = out[1] / (c->w_dims[0] / c->groups);
        double sum = 0.0;
        float total = 0.0f;
        for (uint64_t ch = 0; ch < c->w_dims[1]; ++ch) {
            for (uint64_t kernel = 0; kernel < kvol; ++kernel) {
                coords_of(kernel, c->w_dims + 2, spatial, k);
                src[0] = out[0];
                src[1] = group * c->w_dims[1] + ch;
                int inside = 1;
                for (int a = 0; a < spatial; ++a) {
                    __int128 x = (__int128)out[a + 2] * c->strides[a] + (__int128)k[a] * c->dilations[a] -
                                 (__int128)c->pad_before[a];
                    if (x < 0 || x >= (__int128)c->in_dims[a + 2]) {
                        inside = 0;
                        break;
                    }
                    src[a + 2] = (uint64_t)x;
                }
                if (!inside) continue;
                filt[0] = out[1];
                filt[1] = ch;
                for (int a = 0; a < spatial; ++a) filt[a + 2] = k[a];
                const float a = c->in[address(c->in_dims, src, c->rank)];
                const float b = c->w[address(c->w_dims, filt, c->rank)];
                if (c->out64) sum += (double)a * (double)b;
                if (c->out32) {
                    const float prod = a * b; /* rounded product, then rounded sum */
                    total = total + prod;
                }
            }
        }
        if (c->out64) c->out64[flat] = sum;
        if (c->out32) c->out32[flat] = total;
    }
}

static void conv_common(const uint64_t* in_dims, const float* in, const uint64_t* w_dims, const float* w, int rank,
                        const uint64_t* strides, const uint64_t* dilations, const uint64_t* pad_before,
                        const uint64_t* pad_after, uint64_t groups, double* out64, float* out32, int threads) {
    conv_ctx c = {in_dims, w_dims, strides, dilations, pad_before, pad_after, in, w, rank, groups, {0}, out64, out32};
    oracle_conv_dims(in_dims, w_dims, rank, strides, dilations, pad_before, pad_after, c.out_dims);
    parallel_for(product(c.out_dims, rank), threads, conv_range, &c);
}

void oracle_conv(const uint64_t* in_dims, const float* in, const uint64_t* w_dims, const float* w, int rank,
                 const uint64_t* strides, const uint64_t* dilations, const uint64_t* pad_before,
                 const uint64_t* pad_after, uint64_t groups, double* out, int threads) {
    conv_common(in_dims, in, w_dims, w, rank, strides, dilations, pad_before, pad_after, groups, out, NULL, threads);
}

void oracle_conv_f32_seq(const uint64_t* in_dims, const float* in, const uint64_t* w_dims, const float* w, int rank,
                         const uint64_t* strides, const uint64_t* dilations, const uint64_t* pad_before,
                         const uint64_t* pad_after, uint64_t groups, float* out, int threads) {
    conv_common(in_dims, in, w_dims, w, rank, strides, dilations, pad_before, pad_after, groups, NULL, out, threads);
}

/* ------------------------------------------------------------ attention */

typedef struct {
    const uint64_t *q, *k, *v;
    int qr, kr, vr;
    const float *qd, *kd, *vd;
    const uint64_t* mdims;
    int mrank;
    const double* mask;
    double scale;
    int has_causal;
    int32_t causal;
    uint64_t batches[8];
    int batch_rank;
    uint64_t n, keys, d, dv, heads, group;
    double* out;
} attn_ctx;

/* address() of conformance/attention.rs:140-147: dims align to the trailing
 * coordinates. */
static uint64_t attn_address(const uint64_t* dims, int rank, const uint64_t* coords, int ncoords) {
    int start = ncoords - rank;
    uint64_t idx = 0;
    for (int i = 0; i < rank; ++i) idx = idx * dims[i] + (dims[i] == 1 ? 0 : coords[start + i]);
    return idx;
}

static void attn_range(void* p, uint64_t begin, uint64_t end) {
    attn_ctx* c = (attn_ctx*)p;
    const int br = c->batch_rank;
    uint64_t cb[11];
    double* logits = (double*)malloc(sizeof(double) * (c->keys ? c->keys : 1));
    double* weights = (double*)malloc(sizeof(double) * (c->keys ? c->keys : 1));
    /* Work unit = (batch, head). */
    for (uint64_t unit = begin; unit < end; ++unit) {
        const uint64_t batch = unit / c->heads, head = unit % c->heads;
        coords_of(batch, c->batches, br, cb);
        const uint64_t kv_head = head / c->group;
        for (uint64_t row = 0; row < c->n; ++row) {
            double* o = c->out + ((unit * c->n) + row) * c->dv;
            for (uint64_t col = 0; col < c->keys; ++col) {
                logits[col] = -INFINITY;
                if (c->has_causal && (__int128)col > (__int128)row + (__int128)c->causal) continue;
                cb[br] = head;
                cb[br + 1] = row;
                cb[br + 2] = col;
                double bias = c->mask ? c->mask[attn_address(c->mdims, c->mrank, cb, br + 3)] : 0.0;
                if (bias == -INFINITY) continue;
                cb[br] = head;
                cb[br + 1] = row;
                cb[br + 2] = 0;
                uint64_t qb = attn_address(c->q, c->qr, cb, br + 3);
                cb[br] = kv_head;
                cb[br + 1] = col;
                cb[br + 2] = 0;
                uint64_t kb = attn_address(c->k, c->kr, cb, br + 3);
                double dot = 0.0;
                for (uint64_t i = 0; i < c->d; ++i) dot += (double)c->qd[qb + i] * (double)c->kd[kb + i];
                logits[col] = dot * c->scale + bias;
            }
            double mx = -INFINITY;
            for (uint64_t col = 0; col < c->keys; ++col) mx = fmax(mx, logits[col]);
            if (mx == -INFINITY) {
                for (uint64_t ch = 0; ch < c->dv; ++ch) o[ch] = 0.0;
                continue;
            }
            double sum = 0.0;
            for (uint64_t col = 0; col < c->keys; ++col) {
                weights[col] = exp(logits[col] - mx);
                sum += weights[col];
            }
            cb[br] = kv_head;
            cb[br + 1] = 0;
            cb[br + 2] = 0;
            uint64_t vbase = attn_address(c->v, c->vr, cb, br + 3);
            uint64_t col_stride = c->v[c->vr - 2] == 1 ? 0 : c->dv;
            uint64_t ch_stride = c->dv != 1 ? 1 : 0;
            for (uint64_t ch = 0; ch < c->dv; ++ch) {
                double r = 0.0;
                for (uint64_t col = 0; col < c->keys; ++col)
                    r += weights[col] / sum * (double)c->vd[vbase + ch * ch_stride + col * col_stride];
                o[ch] = r;
            }
        }
    }
    free(logits);
    free(weights);
}

uint64_t oracle_attention(const uint64_t* q_dims, int q_rank, const float* q, const uint64_t* k_dims, int k_rank,
                          const float* k, const uint64_t* v_dims, int v_rank, const float* v,
                          const uint64_t* mask_dims, int mask_rank, const double* mask, int has_scale, float scale,
                          int has_causal, int32_t causal, double* out, int threads) {
    /* canonical(): rank-2 operands gain a unit head axis. */
    uint64_t qc[8], kc[8], vc[8];
    int qr = q_rank, kr = k_rank, vr = v_rank;
    if (q_rank == 2) { qc[0] = 1; qc[1] = q_dims[0]; qc[2] = q_dims[1]; qr = 3; } else memcpy(qc, q_dims, 8 * (size_t)q_rank);
    if (k_rank == 2) { kc[0] = 1; kc[1] = k_dims[0]; kc[2] = k_dims[1]; kr = 3; } else memcpy(kc, k_dims, 8 * (size_t)k_rank);
    if (v_rank == 2) { vc[0] = 1; vc[1] = v_dims[0]; vc[2] = v_dims[1]; vr = 3; } else memcpy(vc, v_dims, 8 * (size_t)v_rank);
    attn_ctx c;
    memset(&c, 0, sizeof(c));
    c.q = qc; c.k = kc; c.v = vc; c.qr = qr; c.kr = kr; c.vr = vr;
    c.qd = q; c.kd = k; c.vd = v;
    c.mdims = mask_dims; c.mrank = mask_rank; c.mask = mask;
    c.n = qc[qr - 2]; c.keys = kc[kr - 2]; c.d = qc[qr - 1]; c.dv = vc[vr - 1];
    c.heads = qc[qr - 3]; c.group = c.heads / kc[kr - 3];
    int br = qr > kr ? qr : kr;
    br = (br > vr ? br : vr) - 3;
    c.batch_rank = br;
    for (int i = 0; i < br; ++i) c.batches[i] = 1;
    const uint64_t* ops[3] = {qc, kc, vc};
    int ranks[3] = {qr, kr, vr};
    for (int t = 0; t < 3; ++t) {
        int plen = ranks[t] - 3;
        for (int a = 0; a < plen; ++a)
            if (ops[t][a] != 1) c.batches[br - plen + a] = ops[t][a];
    }
    uint64_t batch_count = product(c.batches, br);
    uint64_t total = batch_count * c.heads * c.n * c.dv;
    if (total == 0) return 0;
    /* scale.unwrap_or((d as f32).sqrt().recip()) in f32, then widened. */
    c.scale = has_scale ? (double)scale : (double)(1.0f / sqrtf((float)c.d));
    c.has_causal = has_causal;
    c.causal = causal;
    c.out = out;
    parallel_for(batch_count * c.heads, threads, attn_range, &c);
    return total;
}

/* ------------------------------------------------------------ reductions */

static uint64_t output_index(uint64_t flat, const uint64_t* dims, int rank, const uint32_t* axes, int n_axes) {
    uint64_t coords[16];
    coords_of(flat, dims, rank, coords);
    uint64_t idx = 0;
    for (int a = 0; a < rank; ++a) {
        int reduced = 0;
        for (int j = 0; j < n_axes; ++j) reduced |= (int)axes[j] == a;
        if (!reduced) idx = idx * dims[a] + coords[a];
    }
    return idx;
}

static uint64_t kept_size(const uint64_t* dims, int rank, const uint32_t* axes, int n_axes) {
    uint64_t s = 1;
    for (int a = 0; a < rank; ++a) {
        int reduced = 0;
        for (int j = 0; j < n_axes; ++j) reduced |= (int)axes[j] == a;
        if (!reduced) s *= dims[a];
    }
    return s;
}

void oracle_reduce_f32(const float* x, const uint64_t* dims, int rank, const uint32_t* axes, int n_axes, int op,
                       float* out) {
    uint64_t size = kept_size(dims, rank, axes, n_axes), n = product(dims, rank);
    double init = op == 0 ? 0.0 : op == 1 ? 1.0 : op == 2 ? INFINITY : -INFINITY;
    double* r = (double*)malloc(sizeof(double) * (size ? size : 1));
    for (uint64_t i = 0; i < size; ++i) r[i] = init;
    for (uint64_t i = 0; i < n; ++i) {
        double* e = &r[output_index(i, dims, rank, axes, n_axes)];
        double v = (double)x[i];
        *e = op == 0 ? *e + v : op == 1 ? *e * v : op == 2 ? fmin(*e, v) : fmax(*e, v);
    }
    for (uint64_t i = 0; i < size; ++i) out[i] = (float)r[i];
    free(r);
}

void oracle_reduce_u32(const uint32_t* x, const uint64_t* dims, int rank, const uint32_t* axes, int n_axes, int op,
                       uint32_t* out) {
    uint64_t size = kept_size(dims, rank, axes, n_axes), n = product(dims, rank);
    uint32_t init = op == 1 ? 1u : op == 2 ? 0xffffffffu : 0u;
    for (uint64_t i = 0; i < size; ++i) out[i] = init;
    for (uint64_t i = 0; i < n; ++i) {
        uint32_t* e = &out[output_index(i, dims, rank, axes, n_axes)];
        uint32_t v = x[i];
        *e = op == 0 ? *e + v : op == 1 ? *e * v : op == 2 ? (*e < v ? *e : v) : (*e > v ? *e : v);
    }
}

/* ------------------------------------------------------------ statistics */

/* One group of the statistics reference: values gathered in flat order. */
static void stats_group(const double* xs, const uint64_t* flat, uint64_t n, float eps, float* mean, float* variance,
                        float* softmax, float* log_softmax, float* lse, float* norm, uint64_t row) {
    const int want_moments = mean || variance || norm;
    const int want_exp = softmax || log_softmax || lse;
    const double origin = xs[0];
    double delta = 0.0, var = 0.0;
    if (want_moments) {
        for (uint64_t i = 0; i < n; ++i) delta += xs[i] - origin;
        delta /= (double)n;
        for (uint64_t i = 0; i < n; ++i) {
            double d = xs[i] - origin - delta;
            var += d * d;
        }
        var /= (double)n;
    }
    double mx = -INFINITY, es = 0.0, ls = 0.0;
    if (want_exp) {
        for (uint64_t i = 0; i < n; ++i) mx = fmax(mx, xs[i]);
        for (uint64_t i = 0; i < n; ++i) es += exp(xs[i] - mx);
        ls = log(es);
    }
    if (mean) mean[row] = (float)(origin + delta);
    if (variance) variance[row] = (float)var;
    if (lse) lse[row] = (float)(mx + ls);
    if (!softmax && !log_softmax && !norm) return;
    for (uint64_t i = 0; i < n; ++i) {
        uint64_t f = flat ? flat[i] : row * n + i;
        if (softmax) softmax[f] = (float)(exp(xs[i] - mx) / es);
        if (log_softmax) log_softmax[f] = (float)(xs[i] - mx - ls);
        if (norm) norm[f] = (float)((xs[i] - origin - delta) / sqrt(var + (double)eps));
    }
}

void oracle_stats(const float* x, const uint64_t* dims, int rank, const uint32_t* axes, int n_axes, float eps,
                  float* mean, float* variance, float* softmax, float* log_softmax, float* logsumexp, float* norm) {
    uint64_t rows = kept_size(dims, rank, axes, n_axes), n = product(dims, rank);
    if (rows == 0 || n == 0) return;
    uint64_t per = n / rows;
    double* xs = (double*)malloc(sizeof(double) * n);
    uint64_t* flat = (uint64_t*)malloc(sizeof(uint64_t) * n);
    uint64_t* fill = (uint64_t*)calloc(rows, sizeof(uint64_t));
    /* rows[row].push((flat, x)) in flat order (conformance/statistics.rs:269-283). */
    for (uint64_t i = 0; i < n; ++i) {
        uint64_t r = output_index(i, dims, rank, axes, n_axes);
        xs[r * per + fill[r]] = (double)x[i];
        flat[r * per + fill[r]] = i;
        fill[r]++;
    }
    for (uint64_t r = 0; r < rows; ++r)
        stats_group(xs + r * per, flat + r * per, per, eps, mean, variance, softmax, log_softmax, logsumexp, norm, r);
    free(xs);
    free(flat);
    free(fill);
}

typedef struct {
    const float* x;
    uint64_t cols;
    float eps;
    float *mean, *var, *sm, *lsm, *lse, *norm;
    int op;
    float* out;
    uint32_t* idx;
} rows_ctx;

static void row_stats_range(void* p, uint64_t begin, uint64_t end) {
    rows_ctx* c = (rows_ctx*)p;
    double* xs = (double*)malloc(sizeof(double) * (c->cols ? c->cols : 1));
    for (uint64_t r = begin; r < end; ++r) {
        for (uint64_t i = 0; i < c->cols; ++i) xs[i] = (double)c->x[r * c->cols + i];
        stats_group(xs, NULL, c->cols, c->eps, c->mean, c->var, c->sm, c->lsm, c->lse, c->norm, r);
    }
    free(xs);
}

void oracle_row_stats(const float* x, uint64_t rows, uint64_t cols, float eps, float* mean, float* variance,
                      float* softmax, float* log_softmax, float* logsumexp, float* norm, int threads) {
    rows_ctx c = {x, cols, eps, mean, variance, softmax, log_softmax, logsumexp, norm, 0, NULL, NULL};
    parallel_for(rows, threads, row_stats_range, &c);
}

static void row_reduce_range(void* p, uint64_t begin, uint64_t end) {
    rows_ctx* c = (rows_ctx*)p;
    for (uint64_t r = begin; r < end; ++r) {
        const float* row = c->x + r * c->cols;
        double acc = c->op == 0 ? 0.0 : c->op == 1 ? 1.0 : c->op == 2 ? INFINITY : -INFINITY;
        for (uint64_t i = 0; i < c->cols; ++i) {
            double v = (double)row[i];
            acc = c->op == 0 ? acc + v : c->op == 1 ? acc * v : c->op == 2 ? fmin(acc, v) : fmax(acc, v);
        }
        c->out[r] = (float)acc;
    }
}

void oracle_row_reduce(const float* x, uint64_t rows, uint64_t cols, int op, float* out, int threads) {
    rows_ctx c;
    memset(&c, 0, sizeof(c));
    c.x = x;
    c.cols = cols;
    c.op = op;
    c.out = out;
    parallel_for(rows, threads, row_reduce_range, &c);
}

/* f32::total_cmp key: flips the magnitude bits of negatives so that signed
 * integer order equals the IEEE total order. */
static int32_t total_key(float f) {
    int32_t b;
    memcpy(&b, &f, 4);
    return b ^ (int32_t)((uint32_t)(b >> 31) >> 1);
}

static void argmax_range(void* p, uint64_t begin, uint64_t end) {
    rows_ctx* c = (rows_ctx*)p;
    for (uint64_t r = begin; r < end; ++r) {
        const float* row = c->x + r * c->cols;
        uint64_t best = 0;
        for (uint64_t i = 1; i < c->cols; ++i)
            if (total_key(row[i]) > total_key(row[best])) best = i; /* ties keep the lowest index */
        c->idx[r] = (uint32_t)best;
    }
}

void oracle_argmax_rows(const float* x, uint64_t rows, uint64_t cols, uint32_t* out, int threads) {
    rows_ctx c;
    memset(&c, 0, sizeof(c));
    c.x = x;
    c.cols = cols;
    c.idx = out;
    parallel_for(rows, threads, argmax_range, &c);
}

typedef struct {
    const float* x;
    uint64_t n;
    int threads;
    double partial[256];
} sum_ctx;

static void sum_range(void* p, uint64_t begin, uint64_t end) {
    sum_ctx* c = (sum_ctx*)p;
    for (uint64_t t = begin; t < end; ++t) {
        uint64_t lo = c->n * t / (uint64_t)c->threads, hi = c->n * (t + 1) / (uint64_t)c->threads;
        double s = 0.0;
        for (uint64_t i = lo; i < hi; ++i) s += (double)c->x[i];
        c->partial[t] = s;
    }
}

double oracle_sum_f64(const float* x, uint64_t n, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    sum_ctx c;
    c.x = x;
    c.n = n;
    c.threads = threads;
    parallel_for((uint64_t)threads, threads, sum_range, &c);
    double s = 0.0;
    for (int t = 0; t < threads; ++t) s += c.partial[t];
    return s;
}

/* ------------------------------------------------------------ low codec */

/* decode() (conformance/low_precision.rs:7-27), in f64 then narrowed. */
static double decode_low(int bf16, uint16_t bits) {
    int fraction_bits = bf16 ? 7 : 10, exponent_bits = bf16 ? 8 : 5, bias = bf16 ? 127 : 15;
    uint32_t fraction = bits & ((1u << fraction_bits) - 1);
    uint32_t exponent = (bits >> fraction_bits) & ((1u << exponent_bits) - 1);
    double value;
    if (exponent == (1u << exponent_bits) - 1)
        value = fraction == 0 ? INFINITY : NAN;
    else if (exponent == 0)
        value = ldexp((double)fraction, 1 - bias - fraction_bits);
    else
        value = ldexp(1.0 + ldexp((double)fraction, -fraction_bits), (int)exponent - bias);
    return (bits & 0x8000) ? -value : value;
}

/* round() (conformance/low_ops.rs:20-51): nearest-even by value search. */
static uint16_t round_low(int bf16, float x) {
    uint16_t sign = signbit(x) ? 0x8000 : 0;
    double value = fabs((double)x);
    uint16_t max = bf16 ? 0x7f7f : 0x7bff;
    if (isnan(value)) return sign | (uint16_t)(max + 2);
    double last = decode_low(bf16, max);
    double overflow = last + (last - decode_low(bf16, max - 1)) * 0.5;
    if (value >= overflow) return sign | (uint16_t)(max + 1);
    uint16_t lo = 0, hi = max;
    while (lo < hi) {
        uint16_t mid = (uint16_t)(lo + (hi - lo + 1) / 2);
        if (decode_low(bf16, mid) <= value)
            lo = mid;
        else
            hi = (uint16_t)(mid - 1);
    }
    if (lo == max) return sign | lo;
    double below = value - decode_low(bf16, lo), above = decode_low(bf16, lo + 1) - value;
    return sign | ((below < above || (below == above && (lo & 1) == 0)) ? lo : (uint16_t)(lo + 1));
}

uint16_t oracle_round_bf16(float x) { return round_low(1, x); }
uint16_t oracle_round_f16(float x) { return round_low(0, x); }
float oracle_decode_bf16(uint16_t b) { return (float)decode_low(1, b); }
float oracle_decode_f16(uint16_t b) { return (float)decode_low(0, b); }
