/* oracle.h - CPU checker for the batched token sampler.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the shipped library links, loads or calls
 * this code; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference arm use it, and only as the checker or the timed CPU baseline.
 *
 * Two builds share this header:
 *   oracle/_lib/liboracle.so      - qs_oracle_*: a plain-C restatement of the
 *                                   reference sampler (franzvill/quasar sample.c).
 *   oracle/_ref/libsample_ref.so  - qs_ref_*: the reference sample.c itself,
 *                                   compiled unmodified from the reference tree and
 *                                   driven through its own sample.h API.
 * Both export qs_synth_* (the deterministic synthetic-input recipe, synth.c).
 *
 * Parity is pinned by running both builds on the same seeded inputs
 * (tests/test_oracle.py) and by the committed fixtures in tests/golden/, which
 * were produced by the reference build. */
#ifndef QUASAR_ORACLE_H
#define QUASAR_ORACLE_H

#include <stdint.h>

/* Only the qs_* API is exported; the reference build compiles with
 * -fvisibility=hidden so its quasar_sampler_* symbols stay private. */
#define QS_API __attribute__((visibility("default")))

#ifdef __cplusplus
extern "C" {
#endif

/* Per-row sampling parameters. Same layout as quasar_sample_params in
 * include/quasar_sampler.h (24 bytes); raw values, clamped the way
 * sample.c:51-56 clamps them. */
typedef struct {
    float   temperature;
    float   top_p;
    float   min_p;
    float   repeat_penalty;
    int32_t top_k;
    int32_t reserved;
} qs_params;

/* What one pick produced, plus the boundary distances the parity checker needs.
 * `margin` is the smallest distance from any decision the pick made to the
 * boundary where it would flip, measured on the oracle's own sorted order:
 *   - draw:   |r - acc| to the two cumulative sums around the chosen index (abs);
 *   - top_p:  |cum - top_p| at the crossing index and the one before (abs);
 *   - top_k:  relative gap p[k-1] vs p[k] at the cut (0 on an exact tie);
 *   - min_p:  relative gap of the last kept / first dropped p to the floor;
 *   - order:  relative gap of the chosen p to its sorted neighbours.
 * Greedy rows report margin = +inf (they must match bit for bit). */
typedef struct {
    int32_t  id;          /* chosen token id */
    int32_t  n_window;    /* candidates inside the 30-nat window (0 when greedy) */
    int32_t  n_kept;      /* survivors after top-k / top-p / min-p (0 when greedy) */
    int32_t  greedy;      /* 1 when temperature <= 0 */
    float    p_chosen;    /* normalised probability of the chosen token */
    float    inv_sum;     /* (float)(1 / sum of window exps) */
    double   margin;      /* see above */
    uint64_t rng_out;     /* PRNG state after the pick */
} qs_result;

/* ---- restatement (liboracle.so) ------------------------------------------ */

/* One pick over logits[V]. hist is a ring of capacity hist_cap holding hist_len
 * ids starting at hist_head (sample.c:22-23); *rng is advanced in place. */
QS_API int qs_oracle_pick(const float *logits, int V, const qs_params *prm,
                   const int32_t *hist, int hist_cap, int hist_len, int hist_head,
                   uint64_t *rng, qs_result *res);

/* B independent rows (row r: logits + r*ld, params[r] or params[0] when
 * per_row_params == 0, hist + r*hist_cap, rng[r]); nthreads pthreads. */
QS_API int qs_oracle_pick_rows(const float *logits, int64_t ld, int B, int V,
                        const qs_params *params, int per_row_params,
                        const int32_t *hist, int hist_cap,
                        const int32_t *hist_len, const int32_t *hist_head,
                        uint64_t *rng, qs_result *res, int nthreads);

/* ---- reference build (libsample_ref.so) ----------------------------------- */

/* Same contract as qs_oracle_pick_rows, computed by the reference sample.c:
 * one quasar_sampler per row, configured through quasar_sampler_config with
 * seed = rng[r] and repeat_last_n = hist_cap, history injected into the ring,
 * then quasar_sampler_pick. */
QS_API int qs_ref_pick_rows(const float *logits, int64_t ld, int B, int V,
                     const qs_params *params, int per_row_params,
                     const int32_t *hist, int hist_cap,
                     const int32_t *hist_len, const int32_t *hist_head,
                     uint64_t *rng, qs_result *res, int nthreads);

/* A sequence of picks through one reference sampler object, the way the
 * server's generation loop drives it (server.c:258-298): config once, then
 * pick(step_logits) n_steps times, recording each choice. Writes the ids. */
QS_API int qs_ref_sequence(const float *logits, int64_t ld, int n_steps, int V,
                    const qs_params *prm, int repeat_last_n, uint64_t seed,
                    int32_t *ids_out);

/* qs_ref_sequence with each pick's full result (id, kept count, p, margin). */
QS_API int qs_ref_sequence_diag(const float *logits, int64_t ld, int n_steps, int V,
                         const qs_params *prm, int repeat_last_n, uint64_t seed,
                         qs_result *res);

/* The decode loop of a batch: row r gets its own reference object (set up as
 * qs_ref_pick_rows sets it up) and is picked n_steps times on the same logits
 * row, each choice recorded in its ring (sample.c:83-92), as a server that
 * keeps re-sampling would drive it. res is [n_steps][B]; rng[] ends at the
 * final states; hist_out [B][hist_cap], len_out [B] and head_out [B] (may be
 * NULL) get the final rings. */
QS_API int qs_ref_decode(const float *logits, int64_t ld, int B, int V,
                  const qs_params *params, int per_row_params,
                  const int32_t *hist, int hist_cap,
                  const int32_t *hist_len, const int32_t *hist_head,
                  uint64_t *rng, int n_steps, qs_result *res,
                  int32_t *hist_out, int32_t *len_out, int32_t *head_out, int nthreads);

/* ---- synthetic inputs (both builds; synth.c) ------------------------------ */

enum { QS_SYNTH_NORMAL = 0, QS_SYNTH_GUMBEL_PEAK = 1, QS_SYNTH_ZIPF = 2 };

QS_API uint64_t qs_mix64(uint64_t z);
QS_API uint64_t qs_hash3(uint64_t seed, uint64_t a, uint64_t b);
QS_API double   qs_det_log(double x);
QS_API void     qs_synth_logits(int kind, uint64_t seed, int64_t row0, int B, int V,
                         int64_t ld, float scale, float *out);
QS_API void     qs_synth_hist(uint64_t seed, int64_t row0, int B, int H, int V, int32_t *out);
QS_API void     qs_synth_uniform(uint64_t seed, int64_t row0, int B, float lo, float hi,
                          float *out);

#ifdef __cplusplus
}
#endif

#endif /* QUASAR_ORACLE_H */
