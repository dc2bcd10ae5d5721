/* synth.c - deterministic synthetic sampler inputs (CPU side).
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h). The same recipe is implemented for
 * the device in quasar_b200/csrc/synth.cu; both use only integer hashing and
 * IEEE-754 +, -, *, / with floating-point contraction disabled, so a logit
 * generated on the CPU and on the GPU has identical bits (checked by
 * tests/test_gpu_parity.py::test_synth_bits_match).
 *
 * Recipes (the reference publishes no dataset; these stand in for the shapes
 * that BASELINE.json names):
 *   NORMAL       z = (sum of twelve 16-bit uniforms, centred) / 2^16  ~ N(0,1)
 *                (Irwin-Hall, exact in float), logit = z * scale.
 *   GUMBEL_PEAK  u = (53-bit hash + 0.5) * 2^-53, logit = -log(-log(u)) with a
 *                planted +8 at one column per row (column = hash % V).
 *   ZIPF         rank = (a*col + b) mod V + 1 with a per-row a coprime to V
 *                (a permutation of 1..V), logit = -scale * log(rank).
 * log is qs_det_log: frexp-style split plus the atanh series, in double. */
#include "oracle.h"

#include <string.h>

uint64_t qs_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t qs_hash3(uint64_t seed, uint64_t a, uint64_t b) {
    return qs_mix64(qs_mix64(seed ^ (a * 0xD1B54A32D192ED03ull)) ^ (b * 0xABC98388FB8FAC03ull));
}

/* log(x) for finite x > 0 (normal range): x = m * 2^e with m in [1/sqrt2, sqrt2],
 * log(m) = 2*atanh(t), t = (m-1)/(m+1), |t| <= 0.1716, series to t^23. */
double qs_det_log(double x) {
    uint64_t bits;
    memcpy(&bits, &x, sizeof bits);
    int e = (int)((bits >> 52) & 0x7FF) - 1023;
    bits = (bits & 0x000FFFFFFFFFFFFFull) | 0x3FF0000000000000ull;
    double m;
    memcpy(&m, &bits, sizeof m);
    if (m > 1.4142135623730951) { m = m * 0.5; e = e + 1; }
    double t = (m - 1.0) / (m + 1.0);
    double t2 = t * t;
    double s = 0.043478260869565216;          /* 1/23 */
    s = s * t2 + 0.047619047619047616;        /* 1/21 */
    s = s * t2 + 0.05263157894736842;         /* 1/19 */
    s = s * t2 + 0.058823529411764705;        /* 1/17 */
    s = s * t2 + 0.06666666666666667;         /* 1/15 */
    s = s * t2 + 0.07692307692307693;         /* 1/13 */
    s = s * t2 + 0.09090909090909091;         /* 1/11 */
    s = s * t2 + 0.1111111111111111;          /* 1/9  */
    s = s * t2 + 0.14285714285714285;         /* 1/7  */
    s = s * t2 + 0.2;                         /* 1/5  */
    s = s * t2 + 0.3333333333333333;          /* 1/3  */
    s = s * t2 + 1.0;
    return (double)e * 0.6931471805599453 + 2.0 * t * s;
}

static uint64_t gcd_u64(uint64_t a, uint64_t b) {
    while (b) { uint64_t t = a % b; a = b; b = t; }
    return a;
}

static float synth_one(int kind, uint64_t seed, uint64_t row, uint64_t col, int V,
                       float scale, uint64_t zipf_a, uint64_t zipf_b, uint64_t peak) {
    if (kind == QS_SYNTH_NORMAL) {
        int64_t s = 0;
        for (uint64_t k = 0; k < 3; k++) {
            uint64_t h = qs_hash3(seed, row, (col << 2) | k);
            s += (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF)
               + (int64_t)((h >> 32) & 0xFFFF) + (int64_t)(h >> 48);
        }
        float z = (float)(2 * s - 786420) * (1.0f / 131072.0f);
        return z * scale;
    }
    if (kind == QS_SYNTH_GUMBEL_PEAK) {
        uint64_t h = qs_hash3(seed, row, col << 2);
        double u = ((double)(h >> 11) + 0.5) * (1.0 / 9007199254740992.0);
        float g = (float)(-qs_det_log(-qs_det_log(u)));
        if (col == peak) g = g + 8.0f;
        return g;
    }
    /* QS_SYNTH_ZIPF */
    uint64_t rank = (zipf_a * col + zipf_b) % (uint64_t)V + 1;
    return (float)(-(double)scale * qs_det_log((double)rank));
}

static void row_consts(uint64_t seed, uint64_t row, int V,
                       uint64_t *a, uint64_t *b, uint64_t *peak) {
    uint64_t va = qs_hash3(seed, row, 1ull << 62) % (uint64_t)V;
    if (va == 0) va = 1;
    while (gcd_u64(va, (uint64_t)V) != 1) va = va + 1 < (uint64_t)V ? va + 1 : 1;
    *a = va;
    *b = qs_hash3(seed, row, (1ull << 62) + 1) % (uint64_t)V;
    *peak = qs_hash3(seed, row, 0xFFFFFFFFFFFFull) % (uint64_t)V;
}

void qs_synth_logits(int kind, uint64_t seed, int64_t row0, int B, int V,
                     int64_t ld, float scale, float *out) {
    for (int r = 0; r < B; r++) {
        uint64_t row = (uint64_t)(row0 + r), a, b, peak;
        row_consts(seed, row, V, &a, &b, &peak);
        float *o = out + (int64_t)r * ld;
        for (int c = 0; c < V; c++)
            o[c] = synth_one(kind, seed, row, (uint64_t)c, V, scale, a, b, peak);
    }
}

void qs_synth_hist(uint64_t seed, int64_t row0, int B, int H, int V, int32_t *out) {
    for (int r = 0; r < B; r++)
        for (int j = 0; j < H; j++)
            out[(int64_t)r * H + j] =
                (int32_t)(qs_hash3(seed ^ 0x5DEECE66Dull, (uint64_t)(row0 + r), (uint64_t)j) % (uint64_t)V);
}

void qs_synth_uniform(uint64_t seed, int64_t row0, int B, float lo, float hi, float *out) {
    for (int r = 0; r < B; r++) {
        uint64_t h = qs_hash3(seed ^ 0x7F4A7C15ull, (uint64_t)(row0 + r), 0);
        float u = (float)(h >> 40) * (1.0f / 16777216.0f);
        out[r] = lo + (hi - lo) * u;
    }
}
