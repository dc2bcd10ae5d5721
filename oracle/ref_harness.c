/* ref_harness.c - drives the reference sample.c, compiled unmodified.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h). Built by oracle/Makefile into
 * oracle/_ref/libsample_ref.so with -I<reference tree>; the reference source is
 * #included from where it lies, never copied. Including it (instead of linking
 * sample.o) gives this file access to struct quasar_sampler (sample.c:17-29),
 * which is how per-row history is injected: sample.h has no history setter.
 *
 * Each row gets its own sampler object, configured through the reference's
 * quasar_sampler_config (so its clamps and seeding apply), then picked once with
 * quasar_sampler_pick. The pick's id is the result; the diagnostics (window
 * size, kept count, margins) are read off the sampler's own sorted candidate
 * array and cross-checked against that id. */
#include "sample.c"

#include "oracle.h"
#include "diag.h"

#include <math.h>
#include <string.h>

_Static_assert(sizeof(cand_t) == sizeof(qs_cand), "cand_t layout");

typedef struct {
    const float *logits; int64_t ld; int V;
    const qs_params *params; int per_row;
    const int32_t *hist; int cap; const int32_t *len; const int32_t *head;
    uint64_t *rng; qs_result *res; int err;
    int ld_rows;   /* decode loop: results are [step][ld_rows] */
} ref_ctx;

/* One quasar_sampler_pick on s over row[V], with the diagnostics read off the
 * sampler's own sorted candidate array and cross-checked against the id. */
static int ref_pick_diag(quasar_sampler *s, const float *row, int V, qs_result *res) {
    memset(res, 0, sizeof *res);
    uint64_t st = s->rng;
    int id = quasar_sampler_pick(s, row, V);
    res->id = id;
    res->rng_out = s->rng;
    if (V > 0 && s->temperature <= 0.0f) {
        res->greedy = 1;
        res->margin = INFINITY;
    } else if (V > 0) {
        /* s->work still holds the penalized logits of this pick */
        float maxl = -INFINITY;
        for (int i = 0; i < V; i++) if (s->work[i] > maxl) maxl = s->work[i];
        const float inv_t = 1.0f / s->temperature;
        const float thr = maxl * inv_t - 30.0f;
        int nw = 0;
        for (int i = 0; i < V; i++) if (s->work[i] * inv_t >= thr) nw++;
        double u = qs_rng_unit(&st);
        qs_diag((const qs_cand *)s->cand, nw, s->top_p, s->top_k, s->min_p, u, res);
        res->inv_sum = s->cand[0].p;
        res->rng_out = s->rng;
        if (res->id != id) { res->id = id; return -3; }
    }
    return 0;
}

/* A reference object for row r: configured through quasar_sampler_config
 * (clamps and seeding of sample.c:47-68), history injected into its ring. */
static quasar_sampler *ref_object(const ref_ctx *c, int r, int *err) {
    const qs_params *p = c->per_row ? &c->params[r] : &c->params[0];
    quasar_sampler *s = quasar_sampler_new();
    if (!s) { *err = -1; return NULL; }
    uint64_t seed = c->rng[r];
    if (seed == 0) { *err = -2; quasar_sampler_free(s); return NULL; }   /* 0 = time-seeded */
    quasar_sampler_config(s, p->temperature, p->top_p, p->top_k, p->min_p,
                          p->repeat_penalty, c->cap, seed);
    if (c->cap > 0 && s->hist_cap == c->cap) {
        memcpy(s->hist, c->hist + (int64_t)r * c->cap, (size_t)c->cap * sizeof(int32_t));
        s->hist_len = c->len ? c->len[r] : c->cap;
        s->hist_head = c->head ? c->head[r] : 0;
    }
    return s;
}

static void ref_row(void *vctx, int r) {
    ref_ctx *c = (ref_ctx *)vctx;
    qs_result *res = &c->res[r];
    memset(res, 0, sizeof *res);
    quasar_sampler *s = ref_object(c, r, &c->err);
    if (!s) return;
    if (ref_pick_diag(s, c->logits + (int64_t)r * c->ld, c->V, res) != 0) c->err = -3;
    c->rng[r] = s->rng;
    quasar_sampler_free(s);
}

typedef struct {
    ref_ctx base;
    int n_steps;
    int32_t *hist_out, *len_out, *head_out;
} decode_ctx;

/* Row r of a decode loop: one object, n_steps picks of the same logits row,
 * each choice recorded in its ring (sample.c:83-92). */
static void decode_row(void *vctx, int r) {
    decode_ctx *d = (decode_ctx *)vctx;
    ref_ctx *c = &d->base;
    quasar_sampler *s = ref_object(c, r, &c->err);
    if (!s) return;
    const float *row = c->logits + (int64_t)r * c->ld;
    for (int t = 0; t < d->n_steps; t++)
        if (ref_pick_diag(s, row, c->V, &c->res[(int64_t)t * d->base.ld_rows + r]) != 0) c->err = -3;
    c->rng[r] = s->rng;
    if (d->hist_out && c->cap > 0 && s->hist_cap == c->cap) {
        memcpy(d->hist_out + (int64_t)r * c->cap, s->hist, (size_t)c->cap * sizeof(int32_t));
        d->len_out[r] = s->hist_len;
        d->head_out[r] = s->hist_head;
    }
    quasar_sampler_free(s);
}

int qs_ref_pick_rows(const float *logits, int64_t ld, int B, int V,
                     const qs_params *params, int per_row_params,
                     const int32_t *hist, int hist_cap,
                     const int32_t *hist_len, const int32_t *hist_head,
                     uint64_t *rng, qs_result *res, int nthreads) {
    ref_ctx c = { logits, ld, V, params, per_row_params, hist, hist_cap,
                  hist_len, hist_head, rng, res, 0, B };
    if (qs_run_rows(ref_row, &c, B, nthreads) != 0) return -1;
    return c.err;
}

int qs_ref_sequence(const float *logits, int64_t ld, int n_steps, int V,
                    const qs_params *prm, int repeat_last_n, uint64_t seed,
                    int32_t *ids_out) {
    if (seed == 0) return -2;
    quasar_sampler *s = quasar_sampler_new();
    if (!s) return -1;
    quasar_sampler_config(s, prm->temperature, prm->top_p, prm->top_k, prm->min_p,
                          prm->repeat_penalty, repeat_last_n, seed);
    for (int t = 0; t < n_steps; t++)
        ids_out[t] = quasar_sampler_pick(s, logits + (int64_t)t * ld, V);
    quasar_sampler_free(s);
    return 0;
}

int qs_ref_decode(const float *logits, int64_t ld, int B, int V,
                  const qs_params *params, int per_row_params,
                  const int32_t *hist, int hist_cap,
                  const int32_t *hist_len, const int32_t *hist_head,
                  uint64_t *rng, int n_steps, qs_result *res,
                  int32_t *hist_out, int32_t *len_out, int32_t *head_out, int nthreads) {
    decode_ctx d;
    memset(&d, 0, sizeof d);
    ref_ctx c = { logits, ld, V, params, per_row_params, hist, hist_cap,
                  hist_len, hist_head, rng, res, 0, B };
    d.base = c;
    d.n_steps = n_steps;
    d.hist_out = hist_out;
    d.len_out = len_out;
    d.head_out = head_out;
    if (qs_run_rows(decode_row, &d, B, nthreads) != 0) return -1;
    return d.base.err;
}

int qs_ref_sequence_diag(const float *logits, int64_t ld, int n_steps, int V,
                         const qs_params *prm, int repeat_last_n, uint64_t seed,
                         qs_result *res) {
    if (seed == 0) return -2;
    quasar_sampler *s = quasar_sampler_new();
    if (!s) return -1;
    quasar_sampler_config(s, prm->temperature, prm->top_p, prm->top_k, prm->min_p,
                          prm->repeat_penalty, repeat_last_n, seed);
    int err = 0;
    for (int t = 0; t < n_steps; t++)
        if (ref_pick_diag(s, logits + (int64_t)t * ld, V, &res[t]) != 0) err = -3;
    quasar_sampler_free(s);
    return err;
}
