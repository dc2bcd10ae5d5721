/* diag.h - shared helpers of the two oracle builds. TEST INFRASTRUCTURE ONLY. */
#ifndef QUASAR_ORACLE_DIAG_H
#define QUASAR_ORACLE_DIAG_H

#include "oracle.h"

/* Layout of sample.c:15's cand_t. */
typedef struct { int id; float logit; float p; } qs_cand;

void qs_diag(const qs_cand *c, int n_window, float top_p, int top_k, float min_p,
             double u, qs_result *res);

/* xorshift64* step and the [0,1) draw of sample.c:72-81, restated. */
static inline uint64_t qs_xorshift64(uint64_t *st) {
    uint64_t x = *st;
    x ^= x << 13; x ^= x >> 7; x ^= x << 17;
    *st = x;
    return x * 0x2545F4914F6CDD1Dull;
}
static inline double qs_rng_unit(uint64_t *st) {
    return (double)(qs_xorshift64(st) >> 11) * (1.0 / 9007199254740992.0);
}

/* Split rows [0, B) over nthreads pthreads; fn(ctx, row) does one row. */
typedef void (*qs_row_fn)(void *ctx, int row);
int qs_run_rows(qs_row_fn fn, void *ctx, int B, int nthreads);

#endif
