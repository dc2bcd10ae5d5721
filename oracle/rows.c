/* rows.c - pthread row splitter shared by both oracle builds.
 * TEST INFRASTRUCTURE ONLY (see oracle.h). */
#include "diag.h"

#include <pthread.h>
#include <stdlib.h>

typedef struct {
    qs_row_fn fn;
    void *ctx;
    int begin, end;
} qs_span;

static void *run_span(void *arg) {
    qs_span *s = (qs_span *)arg;
    for (int r = s->begin; r < s->end; r++) s->fn(s->ctx, r);
    return NULL;
}

int qs_run_rows(qs_row_fn fn, void *ctx, int B, int nthreads) {
    if (B <= 0) return 0;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > B) nthreads = B;
    if (nthreads == 1) {
        for (int r = 0; r < B; r++) fn(ctx, r);
        return 0;
    }
    pthread_t *th = (pthread_t *)calloc((size_t)nthreads, sizeof *th);
    qs_span *sp = (qs_span *)calloc((size_t)nthreads, sizeof *sp);
    if (!th || !sp) { free(th); free(sp); return -1; }
    int started = 0;
    for (int t = 0; t < nthreads; t++) {
        sp[t].fn = fn; sp[t].ctx = ctx;
        sp[t].begin = (int)((int64_t)B * t / nthreads);
        sp[t].end = (int)((int64_t)B * (t + 1) / nthreads);
        if (pthread_create(&th[t], NULL, run_span, &sp[t]) != 0) break;
        started++;
    }
    for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
    /* spans whose thread could not start run here */
    for (int t = started; t < nthreads; t++) run_span(&sp[t]);
    free(th); free(sp);
    return 0;
}
