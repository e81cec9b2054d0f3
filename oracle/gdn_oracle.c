/* gdn_oracle.c -- CPU restatement of the reference decode step.
 *
 * TEST INFRASTRUCTURE ONLY (see gdn_oracle.h). Build with
 * -ffp-contract=off and without -ffast-math: every expression below is
 * evaluated left to right with one rounding per operation, as the
 * reference's native build (c_impl/Makefile:26-31) does.
 *
 * Each function cites the reference lines (c_impl/gdn_model.cpp) it restates.
 */
#include "gdn_oracle.h"
#include "../gateddeltanet_b200/csrc/gdn_synth.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- BF16 ---- */

static inline uint32_t f2u(float v) { uint32_t b; memcpy(&b, &v, 4); return b; }
static inline float u2f(uint32_t b) { float v; memcpy(&v, &b, 4); return v; }

/* fp32_to_bf16_rne, c_impl/gdn_model.cpp:314-325 */
uint16_t gdn_oracle_bf16_rne_bits(uint32_t bits) {
    const uint32_t mag = bits & 0x7fffffffu;
    if (mag >= 0x7f800000u) {
        if (mag == 0x7f800000u) return (uint16_t)(bits >> 16);
        return (uint16_t)((bits & 0x80000000u) ? 0xffc0u : 0x7fc0u);
    }
    return (uint16_t)((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}

static inline float bf16r(float v) { return u2f((uint32_t)gdn_oracle_bf16_rne_bits(f2u(v)) << 16); }

/* Rounds at an operator boundary in BF16-boundary mode, identity otherwise. */
static inline float bnd(float v, int bf16_boundary) { return bf16_boundary ? bf16r(v) : v; }

/* gdn_native_bf16_product_bits (native branch), c_impl/gdn_model.cpp:392-462:
 * specials first (NaN -> 0x7fc0, Inf*0 -> 0x7fc0, Inf -> signed Inf,
 * zero/subnormal operand -> signed zero), then the exact FP32 product, flushed
 * when its magnitude is below 0x007fc000, else RNE to BF16 and flushed when the
 * rounded exponent field is zero. Returned as FP32 bits. */
uint32_t gdn_oracle_native_product_bits(uint16_t lhs, uint16_t rhs) {
    const uint32_t le = (lhs >> 7) & 0xffu, re = (rhs >> 7) & 0xffu;
    const uint32_t lf = lhs & 0x7fu, rf = rhs & 0x7fu;
    const int lnan = le == 0xffu && lf != 0, rnan = re == 0xffu && rf != 0;
    const int linf = le == 0xffu && lf == 0, rinf = re == 0xffu && rf == 0;
    const int lzero = le == 0, rzero = re == 0;
    const uint32_t sign = (uint32_t)((lhs ^ rhs) & 0x8000u);
    if (lnan || rnan || (linf && rzero) || (rinf && lzero)) return 0x7fc00000u;
    if (linf || rinf) return (sign | 0x7f80u) << 16;
    if (lzero || rzero) return sign << 16;
    volatile float prod = u2f((uint32_t)lhs << 16) * u2f((uint32_t)rhs << 16);
    const uint32_t pb = f2u(prod);
    const uint32_t mag = pb & 0x7fffffffu;
    if (mag == 0x7f800000u) return pb & 0xffff0000u;
    if (mag < 0x007fc000u) return pb & 0x80000000u;
    const uint32_t rounded = pb + 0x7fffu + ((pb >> 16) & 1u);
    const uint32_t res = (rounded >> 16) & 0xffffu;
    if ((res & 0x7f80u) == 0) return (res & 0x8000u) << 16;
    return res << 16;
}

/* Same as above for operands that are already BF16-exact floats; the common
 * path (both operands normal, product normal) without the bit juggling of the
 * special cases. */
static inline float native_mul(float w, float x) {
    const uint32_t wb = f2u(w), xb = f2u(x);
    const uint32_t we = (wb >> 23) & 0xffu, xe = (xb >> 23) & 0xffu;
    if (we == 0 || xe == 0 || we == 0xffu || xe == 0xffu)
        return u2f(gdn_oracle_native_product_bits((uint16_t)(wb >> 16), (uint16_t)(xb >> 16)));
    const float prod = w * x;
    const uint32_t pb = f2u(prod);
    const uint32_t mag = pb & 0x7fffffffu;
    if (mag == 0x7f800000u) return u2f(pb & 0xffff0000u);
    if (mag < 0x007fc000u) return u2f(pb & 0x80000000u);
    const uint32_t res = ((pb + 0x7fffu + ((pb >> 16) & 1u)) >> 16) & 0xffffu;
    if ((res & 0x7f80u) == 0) return u2f((res & 0x8000u) << 16);
    return u2f(res << 16);
}

/* ------------------------------------------------------- scalar helpers ---- */

/* gdn_sigmoid / gdn_silu / gdn_softplus, c_impl/gdn_model.cpp:1307-1330 */
static float sigmoid_ref(float x) {
    if (x >= 0.0f) {
        float z = expf(-x);
        return 1.0f / (1.0f + z);
    }
    {
        float z = expf(x);
        return z / (1.0f + z);
    }
}
static float silu_ref(float x) { return x * sigmoid_ref(x); }
static float softplus_ref(float x) {
    if (x > 20.0f) return x;
    if (x < -20.0f) return expf(x);
    return log1pf(expf(x));
}

/* gdn_tree_reduce_256, c_impl/gdn_model.cpp:1336-1375: pairwise levels. */
static float tree256(const float *a) {
    float l[128];
    for (int i = 0; i < 128; ++i) l[i] = a[2 * i] + a[2 * i + 1];
    for (int n = 64; n >= 1; n >>= 1)
        for (int i = 0; i < n; ++i) l[i] = l[2 * i] + l[2 * i + 1];
    return l[0];
}

/* gemv32_tree16 / gdn_tree16, c_impl/gdn_model.cpp:4004-4035, 1479-1489 */
static inline float tree16(const float *p) {
    const float s0 = p[0] + p[1], s1 = p[2] + p[3], s2 = p[4] + p[5], s3 = p[6] + p[7];
    const float s4 = p[8] + p[9], s5 = p[10] + p[11], s6 = p[12] + p[13], s7 = p[14] + p[15];
    const float a0 = s0 + s1, a1 = s2 + s3, a2 = s4 + s5, a3 = s6 + s7;
    const float b0 = a0 + a1, b1 = a2 + a3;
    return b0 + b1;
}

/* One GEMV row (c_impl/gdn_model.cpp:4444-4586, 4037-4127): per 32-column
 * beat wb the two 16-lane halves go through tree16; four banks accumulate
 * them (lo/hi half x even/odd beat), each starting from 0.0f at its first
 * beat; the row result is (lo_even + hi_even) + (lo_odd + hi_odd). */
static float row_dot(const float *w, const float *x, uint32_t k, int native) {
    float bank[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float p[32];
    for (uint32_t wb = 0; wb < k / 32; ++wb) {
        const float *ww = w + (size_t)wb * 32, *xx = x + (size_t)wb * 32;
        if (native)
            for (int i = 0; i < 32; ++i) p[i] = native_mul(ww[i], xx[i]);
        else
            for (int i = 0; i < 32; ++i) p[i] = ww[i] * xx[i];
        const float dlo = tree16(p), dhi = tree16(p + 16);
        const int odd = (int)(wb & 1u);
        const int first = wb < 2;
        bank[2 * odd] = (first ? 0.0f : bank[2 * odd]) + dlo;
        bank[2 * odd + 1] = (first ? 0.0f : bank[2 * odd + 1]) + dhi;
    }
    const float s0 = bank[0] + bank[1];
    const float s1 = bank[2] + bank[3];
    return s0 + s1;
}

float gdn_oracle_row_dot(const float *w_row, const float *x, uint32_t k, int native_product) {
    return row_dot(w_row, x, k, native_product);
}

/* RMSNorm of a hidden vector, c_impl/gdn_model.cpp:1394-1476 (and the norm
 * half of 3379-3452): per 32-lane beat, each 16-lane half sums its squares
 * sequentially from 0, then `sum += s`; scale = 1/sqrtf(sum/n + eps);
 * out = round((v * scale) * w). */
static void rmsnorm(float *out, const float *in, const float *w, uint32_t n, float eps, int bb) {
    float sum = 0.0f;
    for (uint32_t cp = 0; cp < n / 32; ++cp) {
        for (int half = 0; half < 2; ++half) {
            float s = 0.0f;
            for (int kk = 0; kk < 16; ++kk) {
                const float v = in[cp * 32 + half * 16 + kk];
                s += v * v;
            }
            sum += s;
        }
    }
    const float scale = 1.0f / sqrtf((float)(sum / (float)n) + eps);
    for (uint32_t i = 0; i < n; ++i) out[i] = bnd(in[i] * scale * w[i], bb);
}

/* ------------------------------------------------------- thread helper ---- */

typedef void (*range_fn)(void *ctx, size_t begin, size_t end);
typedef struct { range_fn fn; void *ctx; size_t begin, end; } range_job;

static void *range_thread(void *arg) {
    range_job *j = (range_job *)arg;
    j->fn(j->ctx, j->begin, j->end);
    return NULL;
}

static void parallel_for(size_t n, int threads, range_fn fn, void *ctx) {
    if (threads < 1) threads = 1;
    if ((size_t)threads > n) threads = (int)(n ? n : 1);
    if (threads == 1) { fn(ctx, 0, n); return; }
    pthread_t tid[256];
    range_job job[256];
    if (threads > 256) threads = 256;
    for (int t = 0; t < threads; ++t) {
        job[t].fn = fn; job[t].ctx = ctx;
        job[t].begin = n * (size_t)t / (size_t)threads;
        job[t].end = n * (size_t)(t + 1) / (size_t)threads;
    }
    for (int t = 1; t < threads; ++t) {
        if (pthread_create(&tid[t], NULL, range_thread, &job[t]) != 0) {
            /* no thread available: run the slice here */
            job[t].fn(job[t].ctx, job[t].begin, job[t].end);
            job[t].fn = NULL;
        }
    }
    fn(ctx, job[0].begin, job[0].end);
    for (int t = 1; t < threads; ++t)
        if (job[t].fn != NULL) pthread_join(tid[t], NULL);
}

typedef struct {
    const float *w;    /* rows x k */
    const float *x;
    float *out;
    uint32_t k;
    int native;
} gemv_ctx;

static void gemv_range(void *c, size_t b, size_t e) {
    gemv_ctx *g = (gemv_ctx *)c;
    for (size_t r = b; r < e; ++r) g->out[r] = row_dot(g->w + r * g->k, g->x, g->k, g->native);
}

static void gemv(const float *w, const float *x, float *out, uint32_t rows, uint32_t k,
                 int native, int threads) {
    gemv_ctx c = {w, x, out, k, native};
    parallel_for(rows, threads, gemv_range, &c);
}

/* ------------------------------------------------------ blob geometry ---- */

size_t gdn_oracle_weight_floats(const GdnOracleDims *d) {
    const size_t H = d->hidden, nh = d->heads, hd = d->head_dim, I = d->inter, cs = d->conv;
    const size_t per_layer = H + 2 * nh + 3 * H * H + 2 * nh * H + 3 * H * cs + H * H + hd +
                             H * H + H + 2 * I * H + H * I;
    return (size_t)d->vocab * H + d->layers * per_layer + H + (size_t)d->vocab * H;
}
size_t gdn_oracle_rec_floats(const GdnOracleDims *d) {
    return (size_t)d->layers * d->heads * d->head_dim * d->head_dim;
}
size_t gdn_oracle_conv_floats(const GdnOracleDims *d) {
    return (size_t)d->layers * 3 * (d->conv - 1) * d->hidden;
}

typedef struct {
    const float *attn_norm, *a_log, *dt_bias, *q, *k, *v, *a, *b, *qc, *kc, *vc, *g, *o_norm, *o,
        *mlp_norm, *gate, *up, *down;
} layer_views;

/* gdn_assign_weight_views, c_impl/gdn_model.cpp:1102-1159 */
static void views(const GdnOracleDims *d, const float *blob, uint32_t l, layer_views *v,
                  const float **final_norm, const float **lm_head) {
    const size_t H = d->hidden, nh = d->heads, hd = d->head_dim, I = d->inter, cs = d->conv;
    const size_t per_layer = H + 2 * nh + 3 * H * H + 2 * nh * H + 3 * H * cs + H * H + hd +
                             H * H + H + 2 * I * H + H * I;
    const float *p = blob + (size_t)d->vocab * H + (size_t)l * per_layer;
    if (v != NULL) {
        v->attn_norm = p; p += H;
        v->a_log = p; p += nh;
        v->dt_bias = p; p += nh;
        v->q = p; p += H * H;
        v->k = p; p += H * H;
        v->v = p; p += H * H;
        v->a = p; p += nh * H;
        v->b = p; p += nh * H;
        v->qc = p; p += H * cs;
        v->kc = p; p += H * cs;
        v->vc = p; p += H * cs;
        v->g = p; p += H * H;
        v->o_norm = p; p += hd;
        v->o = p; p += H * H;
        v->mlp_norm = p; p += H;
        v->gate = p; p += I * H;
        v->up = p; p += I * H;
        v->down = p;
    }
    if (final_norm != NULL) {
        const float *f = blob + (size_t)d->vocab * H + (size_t)d->layers * per_layer;
        *final_norm = f;
        *lm_head = f + H;
    }
}

typedef struct {
    const GdnOracleDims *d;
    uint64_t seed;
    float *blob;
} synth_ctx;

/* Walk the blob in fixed 1M-float pieces; each piece knows its tensor(s). */
static void synth_range(void *c, size_t b, size_t e) {
    synth_ctx *s = (synth_ctx *)c;
    const GdnOracleDims *d = s->d;
    const size_t H = d->hidden, nh = d->heads, hd = d->head_dim, I = d->inter, cs = d->conv;
    const size_t sizes[GDN_SYNTH_TENSORS_PER_LAYER] = {H, nh, nh, H * H, H * H, H * H, nh * H, nh * H,
                                                       H * cs, H * cs, H * cs, H * H, hd, H * H, H,
                                                       I * H, I * H, H * I};
    const size_t piece = (size_t)1 << 20;
    for (size_t pc = b; pc < e; ++pc) {
        const size_t lo = pc * piece, hi = lo + piece;
        /* enumerate tensors overlapping [lo, hi) */
        size_t off = 0;
        const uint32_t ntensors = 3 + GDN_SYNTH_TENSORS_PER_LAYER * d->layers;
        for (uint32_t t = 0; t < ntensors; ++t) {
            size_t sz;
            if (t == 0 || t == ntensors - 1) sz = (size_t)d->vocab * H;
            else if (t == ntensors - 2) sz = H;
            else sz = sizes[(t - 1) % GDN_SYNTH_TENSORS_PER_LAYER];
            const size_t tb = off, te = off + sz;
            off = te;
            if (te <= lo) continue;
            if (tb >= hi) break;
            const size_t b0 = tb > lo ? tb : lo, e0 = te < hi ? te : hi;
            gdn_synth_fill(s->blob + b0, s->seed, t, gdn_synth_tensor_dist(t, d->layers),
                           b0 - tb, e0 - tb);
        }
    }
}

void gdn_oracle_synth_weights(const GdnOracleDims *d, uint64_t seed, float *blob, int threads) {
    const size_t total = gdn_oracle_weight_floats(d);
    const size_t piece = (size_t)1 << 20;
    synth_ctx c = {d, seed, blob};
    parallel_for((total + piece - 1) / piece, threads, synth_range, &c);
}

void gdn_oracle_bf16_rne_batch(const uint32_t *in, size_t n, uint16_t *out) {
    for (size_t i = 0; i < n; ++i) out[i] = gdn_oracle_bf16_rne_bits(in[i]);
}

void gdn_oracle_native_product_grid(const uint16_t *w, size_t n_w, const uint16_t *a, size_t n_a, uint32_t *out) {
    for (size_t j = 0; j < n_a; ++j)
        for (size_t i = 0; i < n_w; ++i) out[j * n_w + i] = gdn_oracle_native_product_bits(w[i], a[j]);
}

typedef struct {
    const float *lm;
    const uint16_t *act;
    float *out;
    uint32_t H;
} logits_ctx;

static void logits_range(void *c, size_t b, size_t e) {
    logits_ctx *g = (logits_ctx *)c;
    for (size_t v = b; v < e; ++v) {
        const float *row = g->lm + v * g->H;
        float sum = 0.0f;
        for (uint32_t i = 0; i < g->H; ++i)
            sum += u2f(gdn_oracle_native_product_bits((uint16_t)(f2u(row[i]) >> 16), g->act[i]));
        g->out[v] = sum;
    }
}

void gdn_oracle_compute_logits(const GdnOracleDims *d, const float *blob, const float *hidden, float *logits,
                               int threads) {
    const float *final_norm, *lm_head;
    views(d, blob, 0, NULL, &final_norm, &lm_head);
    uint16_t *act = (uint16_t *)malloc(sizeof(uint16_t) * d->hidden);
    if (act == NULL) return;
    for (uint32_t i = 0; i < d->hidden; ++i) act[i] = gdn_oracle_bf16_rne_bits(f2u(hidden[i]));
    logits_ctx c = {lm_head, act, logits, d->hidden};
    parallel_for(d->vocab, threads, logits_range, &c);
    free(act);
}

int32_t gdn_oracle_synth_token(uint64_t seed, uint32_t stream, uint64_t i, uint32_t vocab) {
    return gdn_synth_token(seed, stream, i, vocab);
}

void gdn_oracle_synth_state(const GdnOracleDims *d, uint64_t state_seed, float *rec, float *conv) {
    const size_t nr = gdn_oracle_rec_floats(d), nc = gdn_oracle_conv_floats(d);
    for (size_t i = 0; i < nr; ++i)
        rec[i] = state_seed ? gdn_synth_round_bf16(gdn_synth_normal(state_seed, GDN_SYNTH_STREAM_STATE, i, 0.05)) : 0.0f;
    for (size_t i = 0; i < nc; ++i)
        conv[i] = state_seed ? gdn_synth_round_bf16(gdn_synth_normal(state_seed, GDN_SYNTH_STREAM_STATE + 1, i, 0.5)) : 0.0f;
}

/* --------------------------------------------------- gated delta rule ---- */

/* Read pass, delta/output and update of gdn_recurrent_attention_island,
 * c_impl/gdn_model.cpp:2119-2300 (alpha :2119-2124, read :2184-2210,
 * delta/output :2214-2243 with q_scale = 1/sqrtf(256), update :2268-2300).
 * S is [K][V]; qn/kn are normalised; o is unrounded. */
void gdn_oracle_delta_rule_head(float *S, const float *qn, const float *kn, const float *v,
                                float decay, float beta, int bf16_state, float *o) {
    enum { DK = 256, DV = 256 };
    const float q_scale = 1.0f / sqrtf((float)DK);
    float prod[DK];
    for (int j = 0; j < DK; ++j) prod[j] = qn[j] * kn[j];
    const float alpha = tree256(prod);
    float r[DV], p[DV], delta[DV];
    for (int c = 0; c < DV; ++c) { r[c] = 0.0f; p[c] = 0.0f; }
    for (int row = 0; row < DK; ++row) {
        const float kj = kn[row], qj = qn[row];
        const float *Sr = S + (size_t)row * DV;
        for (int c = 0; c < DV; ++c) {
            r[c] = r[c] + Sr[c] * kj;
            p[c] = p[c] + Sr[c] * qj;
        }
    }
    for (int c = 0; c < DV; ++c) {
        delta[c] = beta * (v[c] - decay * r[c]);
        o[c] = q_scale * (decay * p[c] + alpha * delta[c]);
    }
    for (int row = 0; row < DK; ++row) {
        const float kj = kn[row];
        float *Sr = S + (size_t)row * DV;
        for (int c = 0; c < DV; ++c) {
            const float upd = decay * Sr[c] + kj * delta[c];
            Sr[c] = bf16_state ? bf16r(upd) : upd;
        }
    }
}

/* ------------------------------------------------------------ the step ---- */

typedef struct {
    const GdnOracleDims *d;
    const layer_views *lv;
    GdnOracleMode mode;
    float *rec_layer;          /* [H][K][V] */
    const float *convq, *convk, *convv, *a, *b;
    float *attn;
} recur_ctx;

static void recur_range(void *c, size_t hb, size_t he) {
    recur_ctx *r = (recur_ctx *)c;
    enum { DK = 256 };
    for (size_t h = hb; h < he; ++h) {
        const float *q = r->convq + h * DK, *k = r->convk + h * DK, *v = r->convv + h * DK;
        float qn[DK], kn[DK], qsq[DK], ksq[DK], o[DK];
        /* c_impl/gdn_model.cpp:2059-2092 */
        for (int j = 0; j < DK; ++j) { qsq[j] = q[j] * q[j]; ksq[j] = k[j] * k[j]; }
        const float q_inv = 1.0f / sqrtf(tree256(qsq) + 1e-6f);
        const float k_inv = 1.0f / sqrtf(tree256(ksq) + 1e-6f);
        for (int j = 0; j < DK; ++j) { qn[j] = q[j] * q_inv; kn[j] = k[j] * k_inv; }
        /* c_impl/gdn_model.cpp:2101-2105 */
        const float beta = sigmoid_ref(r->b[h]);
        const float decay_in = r->a[h] + r->lv->dt_bias[h];
        const float decay_val = -expf(r->lv->a_log[h]) * softplus_ref(decay_in);
        const float decay = expf(decay_val);
        gdn_oracle_delta_rule_head(r->rec_layer + h * DK * DK, qn, kn, v, decay, beta,
                                   r->mode.bf16_state, o);
        /* merge, c_impl/gdn_model.cpp:2904-2933: output rounded to BF16 */
        for (int c2 = 0; c2 < DK; ++c2) r->attn[h * DK + c2] = bnd(o[c2], r->mode.bf16_boundary);
    }
}

int gdn_oracle_step(const GdnOracleDims *d, const float *blob, GdnOracleMode mode,
                    float *rec, float *conv, int32_t token,
                    float *logits, float *final_hidden, int32_t *argmax, int threads) {
    const uint32_t H = d->hidden, nh = d->heads, hd = d->head_dim, I = d->inter, V = d->vocab;
    const uint32_t W = d->conv;
    const int bb = mode.bf16_boundary;
    const int native = mode.native_product;
    if (token < 0 || (uint32_t)token >= V || hd != 256 || H != nh * hd || W != 4 || H % 32 || I % 32)
        return -1;
    if (native && !bb) return -1; /* the BF16 product needs BF16 operands */

    float *x = (float *)malloc(sizeof(float) * H);
    float *x_alt = (float *)malloc(sizeof(float) * H);
    float *xn = (float *)malloc(sizeof(float) * H);
    float *raw = (float *)malloc(sizeof(float) * 4 * H);
    float *cq = (float *)malloc(sizeof(float) * 3 * H);
    float *attn = (float *)malloc(sizeof(float) * H);
    float *gated = (float *)malloc(sizeof(float) * H);
    float *y = (float *)malloc(sizeof(float) * H);
    float *gu = (float *)malloc(sizeof(float) * 2 * I);
    float *m = (float *)malloc(sizeof(float) * I);
    float *lg = (float *)malloc(sizeof(float) * V);
    float ab[64];
    if (!x || !x_alt || !xn || !raw || !cq || !attn || !gated || !y || !gu || !m || !lg || nh > 32) {
        free(x); free(x_alt); free(xn); free(raw); free(cq); free(attn); free(gated); free(y);
        free(gu); free(m); free(lg);
        return -1;
    }
    const float *final_norm, *lm_head;
    views(d, blob, 0, NULL, &final_norm, &lm_head);

    /* embedding import, c_impl/gdn_model.cpp:3719-3731 */
    const float *erow = blob + (size_t)token * H;
    for (uint32_t i = 0; i < H; ++i) x[i] = bnd(erow[i], bb);
    {
        layer_views l0;
        views(d, blob, 0, &l0, NULL, NULL);
        rmsnorm(xn, x, l0.attn_norm, H, d->eps, bb); /* :3738-3740 */
    }

    for (uint32_t l = 0; l < d->layers; ++l) {
        layer_views lv;
        views(d, blob, l, &lv, NULL, NULL);

        /* a/b tiny GEMV, :1501-1535: exact products, acc = (acc + T(lo)) + T(hi) */
        for (uint32_t c = 0; c < 2 * nh; ++c) {
            const float *wrow = (c < nh ? lv.a + (size_t)c * H : lv.b + (size_t)(c - nh) * H);
            float acc = 0.0f, p[32];
            for (uint32_t j = 0; j < H / 32; ++j) {
                for (int i = 0; i < 32; ++i) p[i] = xn[j * 32 + i] * wrow[j * 32 + i];
                const float t0 = tree16(p), t1 = tree16(p + 16);
                acc = (acc + t0) + t1;
            }
            ab[c] = bnd(acc, bb);
        }

        /* QKVG GEMV, :3789-3796 (rows q | k | v | g) */
        gemv(lv.q, xn, raw, H, H, native, threads);
        gemv(lv.k, xn, raw + H, H, H, native, threads);
        gemv(lv.v, xn, raw + 2 * H, H, H, native, threads);
        gemv(lv.g, xn, raw + 3 * H, H, H, native, threads);
        for (uint32_t i = 0; i < 4 * H; ++i) raw[i] = bnd(raw[i], bb);

        /* depthwise conv + SiLU and tail update, :1543-1660, :5113-5127.
         * window = [tail0, tail1, tail2, new]; sum left to right. */
        for (uint32_t kind = 0; kind < 3; ++kind) {
            const float *cw = kind == 0 ? lv.qc : kind == 1 ? lv.kc : lv.vc;
            float *tails = conv + ((size_t)l * 3 + kind) * (W - 1) * H; /* [3][H] */
            for (uint32_t dch = 0; dch < H; ++dch) {
                const float t0 = tails[dch], t1 = tails[H + dch], t2 = tails[2 * H + dch];
                const float nv = raw[kind * H + dch];
                const float *w4 = cw + (size_t)dch * 4;
                const float sum = t0 * w4[0] + t1 * w4[1] + t2 * w4[2] + nv * w4[3];
                cq[kind * H + dch] = bnd(silu_ref(sum), bb);
                tails[dch] = t1;
                tails[H + dch] = t2;
                tails[2 * H + dch] = nv;
            }
        }

        /* gated delta rule per head, :1932-2340 */
        {
            recur_ctx rc = {d, &lv, mode, rec + (size_t)l * nh * hd * hd, cq, cq + H, cq + 2 * H,
                            ab, ab + nh, attn};
            parallel_for(nh, threads, recur_range, &rc);
        }

        /* output RMSNorm x swish gate, :3226-3349 */
        for (uint32_t h = 0; h < nh; ++h) {
            const float *a = attn + (size_t)h * hd;
            const float *g = raw + 3 * H + (size_t)h * hd;
            float sum = 0.0f;
            for (uint32_t ip = 0; ip < hd / 32; ++ip)
                for (int half = 0; half < 2; ++half) {
                    float s = 0.0f;
                    for (int kk = 0; kk < 16; ++kk) {
                        const float av = a[ip * 32 + half * 16 + kk];
                        s += av * av;
                    }
                    sum += s;
                }
            const float scale = 1.0f / sqrtf(sum / (float)hd + d->eps);
            for (uint32_t i = 0; i < hd; ++i) {
                const float normalized = a[i] * scale * lv.o_norm[i];
                const float gv = g[i];
                gated[h * hd + i] = bnd(normalized * gv * sigmoid_ref(gv), bb);
            }
        }

        /* o_proj, :3803-3810 */
        gemv(lv.o, gated, y, H, H, native, threads);
        for (uint32_t i = 0; i < H; ++i) y[i] = bnd(y[i], bb);

        /* residual + MLP norm, :3351-3452 */
        for (uint32_t i = 0; i < H; ++i) x_alt[i] = bnd(x[i] + y[i], bb);
        rmsnorm(xn, x_alt, lv.mlp_norm, H, d->eps, bb);

        /* gate/up + SwiGLU, :3815-3822, :4751-4770 */
        gemv(lv.gate, xn, gu, I, H, native, threads);
        gemv(lv.up, xn, gu + I, I, H, native, threads);
        for (uint32_t i = 0; i < I; ++i) {
            const float gv = bnd(gu[i], bb), uv = bnd(gu[I + i], bb);
            m[i] = bnd(silu_ref(gv) * uv, bb);
        }

        /* down, :3827-3834, then residual + next norm, :3836-3842 */
        gemv(lv.down, m, y, H, I, native, threads);
        for (uint32_t i = 0; i < H; ++i) y[i] = bnd(y[i], bb);
        for (uint32_t i = 0; i < H; ++i) x[i] = bnd(x_alt[i] + y[i], bb);
        if (l + 1 < d->layers) {
            layer_views nx;
            views(d, blob, l + 1, &nx, NULL, NULL);
            rmsnorm(xn, x, nx.attn_norm, H, d->eps, bb);
        } else {
            rmsnorm(xn, x, final_norm, H, d->eps, bb);
        }
    }

    /* LM head (FP32 logits, not rounded) + strict first-index argmax, :3859-3888, :4775-4925 */
    gemv(lm_head, xn, lg, V, H, native, threads);
    float best = -3.402823466e38f;
    int32_t best_i = 0;
    for (uint32_t v = 0; v < V; ++v)
        if (lg[v] > best) { best = lg[v]; best_i = (int32_t)v; }
    if (logits) memcpy(logits, lg, sizeof(float) * V);
    if (final_hidden) memcpy(final_hidden, xn, sizeof(float) * H);
    if (argmax) *argmax = best_i;

    free(x); free(x_alt); free(xn); free(raw); free(cq); free(attn); free(gated); free(y);
    free(gu); free(m); free(lg);
    return 0;
}
