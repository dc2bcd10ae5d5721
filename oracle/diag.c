/* diag.c - cut / draw bookkeeping and boundary margins over a sorted candidate
 * list. TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Input is the candidate list of one non-greedy pick after the softmax and the
 * sort (sample.c:146-151): qs_cand has the layout of sample.c:15's cand_t
 * {int id; float logit; float p} and is ordered by p descending, ties by id
 * ascending (glibc's qsort is a stable merge sort, so equal p keep id order).
 * qs_diag replays the cuts and the draw (sample.c:153-177) and records how far
 * each decision sits from the boundary where it would flip. */
#include "oracle.h"
#include "diag.h"

#include <math.h>

static double rel_gap(float a, float b) {
    double hi = fabs((double)a) > fabs((double)b) ? fabs((double)a) : fabs((double)b);
    if (hi == 0.0) return 0.0;
    return fabs((double)a - (double)b) / hi;
}

static void keep_min(double *m, double v) { if (v < *m) *m = v; }

void qs_diag(const qs_cand *c, int n_window, float top_p, int top_k, float min_p,
             double u, qs_result *res) {
    double margin = INFINITY;
    int nc = n_window;

    /* top-k (sample.c:154) */
    if (top_k > 0 && top_k < nc) {
        keep_min(&margin, rel_gap(c[top_k - 1].p, c[top_k].p));
        nc = top_k;
    }
    /* top-p (sample.c:156-160): first prefix whose double cumsum reaches top_p */
    if (top_p < 1.0f) {
        double cum = 0.0, prev = 0.0;
        int keep = nc;
        for (int i = 0; i < nc; i++) {
            prev = cum;
            cum += c[i].p;
            if (cum >= top_p) {
                keep = i + 1;
                keep_min(&margin, cum - (double)top_p);
                keep_min(&margin, (double)top_p - prev);
                break;
            }
        }
        nc = keep;
    }
    /* min-p (sample.c:162-167): floor against the top candidate */
    if (min_p > 0.0f) {
        float floor_p = min_p * c[0].p;
        int keep = nc;
        for (int i = 1; i < nc; i++)
            if (c[i].p < floor_p) { keep = i; break; }
        if (floor_p > 0.0f) {
            if (keep < nc) keep_min(&margin, ((double)floor_p - c[keep].p) / floor_p);
            if (keep - 1 >= 1) keep_min(&margin, ((double)c[keep - 1].p - floor_p) / floor_p);
        }
        nc = keep;
    }
    if (nc < 1) nc = 1;

    /* draw (sample.c:171-175) */
    double rsum = 0.0;
    for (int i = 0; i < nc; i++) rsum += c[i].p;
    double r = u * rsum, acc = 0.0, prev = 0.0;
    int chosen = nc - 1, hit = 0;
    for (int i = 0; i < nc; i++) {
        prev = acc;
        acc += c[i].p;
        if (r <= acc) { chosen = i; hit = 1; break; }
    }
    if (hit) {
        keep_min(&margin, acc - r);
        if (chosen > 0) keep_min(&margin, r - prev);
    } else {
        margin = 0.0;
    }
    /* order near-ties around the chosen index */
    if (chosen > 0) keep_min(&margin, rel_gap(c[chosen].p, c[chosen - 1].p));
    if (chosen + 1 < n_window) keep_min(&margin, rel_gap(c[chosen].p, c[chosen + 1].p));

    res->id = c[chosen].id;
    res->n_window = n_window;
    res->n_kept = nc;
    res->greedy = 0;
    res->p_chosen = c[chosen].p;
    res->margin = margin;
}
