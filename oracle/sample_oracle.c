/* sample_oracle.c - plain-C restatement of the reference token sampler.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h): the checker for the CUDA sampler and
 * the CPU baseline when the reference build (oracle/_ref) is absent. Parity of
 * this file with the reference is pinned by tests/test_oracle.py (same inputs
 * through the compiled reference sample.c) and tests/golden/.
 *
 * Follows franzvill/quasar sample.c step by step:
 *   clamps                 sample.c:51-56
 *   penalty + running max  sample.c:118-128
 *   greedy argmax          sample.c:130-134 (strict >, first index wins, no draw)
 *   30-nat window          sample.c:136-144 (inv_t = 1.0f/T, msc = maxl*inv_t)
 *   softmax                sample.c:146-150 (float expf, double sum, float inv)
 *   sort                   sample.c:151 (p descending; glibc's stable merge sort
 *                          keeps ties in id order, restated as an id tie-break)
 *   cuts + draw            sample.c:153-177 via qs_diag (diag.c)
 * History ids outside [0, V) are ignored (the reference only ever records ids
 * it produced itself, so it never meets one). */
#include "oracle.h"
#include "diag.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static int cmp_p_desc_id_asc(const void *a, const void *b) {
    const qs_cand *x = (const qs_cand *)a, *y = (const qs_cand *)b;
    if (x->p > y->p) return -1;
    if (x->p < y->p) return 1;
    return (x->id > y->id) - (x->id < y->id);
}

int qs_oracle_pick(const float *logits, int V, const qs_params *prm,
                   const int32_t *hist, int hist_cap, int hist_len, int hist_head,
                   uint64_t *rng, qs_result *res) {
    memset(res, 0, sizeof *res);
    res->rng_out = *rng;
    if (V <= 0) return 0;                                   /* sample.c:112 */

    const float T = prm->temperature;
    const float top_p = (prm->top_p > 0.0f && prm->top_p < 1.0f) ? prm->top_p : 1.0f;
    const int top_k = prm->top_k > 0 ? prm->top_k : 0;
    const float min_p = prm->min_p > 0.0f ? prm->min_p : 0.0f;
    const float rp = prm->repeat_penalty > 1.0f ? prm->repeat_penalty : 1.0f;

    float *work = (float *)malloc((size_t)V * sizeof *work);
    uint8_t *flag = (uint8_t *)calloc((size_t)V, 1);
    qs_cand *cand = (qs_cand *)malloc((size_t)V * sizeof *cand);
    if (!work || !flag || !cand) { free(work); free(flag); free(cand); return -1; }

    if (rp > 1.0f && hist && hist_cap > 0) {
        for (int i = 0; i < hist_len; i++) {
            int32_t id = hist[(hist_head + i) % hist_cap];
            if (id >= 0 && id < V) flag[id] = 1;
        }
    }
    float maxl = -INFINITY;
    for (int i = 0; i < V; i++) {
        float l = logits[i];
        if (flag[i]) l = (l > 0.0f) ? l / rp : l * rp;
        work[i] = l;
        if (l > maxl) maxl = l;
    }

    if (T <= 0.0f) {
        int bi = 0;
        for (int i = 1; i < V; i++) if (work[i] > work[bi]) bi = i;
        res->id = bi;
        res->greedy = 1;
        res->margin = INFINITY;
        free(work); free(flag); free(cand);
        return 0;
    }

    const float inv_t = 1.0f / T;
    const float msc = maxl * inv_t;
    const float thr = msc - 30.0f;
    int nc = 0;
    for (int i = 0; i < V; i++) {
        float sc = work[i] * inv_t;
        if (sc >= thr) { cand[nc].id = i; cand[nc].logit = sc; nc++; }
    }
    double sum = 0.0;
    for (int i = 0; i < nc; i++) { float e = expf(cand[i].logit - msc); cand[i].p = e; sum += e; }
    const float inv = (float)(1.0 / sum);
    for (int i = 0; i < nc; i++) cand[i].p *= inv;
    qsort(cand, (size_t)nc, sizeof *cand, cmp_p_desc_id_asc);

    uint64_t st = *rng;
    double u = qs_rng_unit(&st);
    *rng = st;
    qs_diag(cand, nc, top_p, top_k, min_p, u, res);
    res->inv_sum = inv;
    res->rng_out = st;
    free(work); free(flag); free(cand);
    return 0;
}

typedef struct {
    const float *logits; int64_t ld; int V;
    const qs_params *params; int per_row;
    const int32_t *hist; int cap; const int32_t *len; const int32_t *head;
    uint64_t *rng; qs_result *res; int err;
} rows_ctx;

static void one_row(void *vctx, int r) {
    rows_ctx *c = (rows_ctx *)vctx;
    const qs_params *p = c->per_row ? &c->params[r] : &c->params[0];
    int len = c->cap > 0 ? (c->len ? c->len[r] : c->cap) : 0;
    int head = c->head ? c->head[r] : 0;
    const int32_t *h = c->cap > 0 ? c->hist + (int64_t)r * c->cap : NULL;
    if (qs_oracle_pick(c->logits + (int64_t)r * c->ld, c->V, p, h, c->cap, len, head,
                       &c->rng[r], &c->res[r]) != 0)
        c->err = -1;
}

int qs_oracle_pick_rows(const float *logits, int64_t ld, int B, int V,
                        const qs_params *params, int per_row_params,
                        const int32_t *hist, int hist_cap,
                        const int32_t *hist_len, const int32_t *hist_head,
                        uint64_t *rng, qs_result *res, int nthreads) {
    rows_ctx c = { logits, ld, V, params, per_row_params, hist, hist_cap,
                   hist_len, hist_head, rng, res, 0 };
    if (qs_run_rows(one_row, &c, B, nthreads) != 0) return -1;
    return c.err;
}
