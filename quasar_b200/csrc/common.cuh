// common.cuh - shared device helpers for the sm_100a sampler kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/quasar_sampler.h"

namespace qs {

constexpr unsigned FULL = 0xFFFFFFFFu;

// Order-preserving map float -> uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t ord_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord_key_inv(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
}

// Repeat penalty of sample.c:124, with IEEE division / multiplication.
__device__ __forceinline__ float penalize(float l, float rp) {
    return (l > 0.0f) ? __fdiv_rn(l, rp) : __fmul_rn(l, rp);
}

// xorshift64* step and its [0,1) double (sample.c:72-81).
__device__ __forceinline__ double rng_unit(uint64_t* st) {
    uint64_t x = *st;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *st = x;
    return (double)((x * 0x2545F4914F6CDD1Dull) >> 11) * (1.0 / 9007199254740992.0);
}

// Parameters of one row after the clamps of sample.c:51-56.
struct RowParams {
    float T, top_p, min_p, rp;
    int top_k;
};

__device__ __forceinline__ RowParams clamp_params(const quasar_sample_params& p) {
    RowParams r;
    r.T = p.temperature;
    r.top_p = (p.top_p > 0.0f && p.top_p < 1.0f) ? p.top_p : 1.0f;
    r.top_k = p.top_k > 0 ? p.top_k : 0;
    r.min_p = p.min_p > 0.0f ? p.min_p : 0.0f;
    r.rp = p.repeat_penalty > 1.0f ? p.repeat_penalty : 1.0f;
    return r;
}

// e^x for x <= 0, used for the terms of the window sum only (the reported
// probabilities use a correctly rounded exp). exp(x) = 2^(x*log2e): the product
// x*log2e is split into t + tl exactly (FMA remainder, plus the rounding error
// of the float log2e), 2^t comes from ex2.approx and the remainder is applied
// as 2^t * (1 + tl*ln2). The error is that of ex2.approx alone (~2 ulp, checked
// for size and bias against a double-precision exp by the GPU self-test).
// x < -126 returns 0 (flushed), so x = -inf is safe.
__device__ __forceinline__ float exp_term(float x) {
    const float kLog2e = 1.44269502162933349609375f;    // float(log2 e)
    const float kLog2eLo = 1.925963033500011e-08f;       // log2 e - kLog2e
    x = fmaxf(x, -126.0f);
    const float t = __fmul_rn(x, kLog2e);
    float tl = __fmaf_rn(x, kLog2e, -t);
    tl = __fmaf_rn(x, kLog2eLo, tl);
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t));
    return __fmaf_rn(e, __fmul_rn(tl, 0.693147182464599609375f), e);
}

// e^x for x <= 0 with FMA-pipe arithmetic only: Cody-Waite reduction
// x = k*ln2 + r (|r| <= ln2/2; ln2 split in an 11-bit head, so k*head is
// exact, and a float tail), e^r from a degree-6 polynomial fitted to e^r on
// [-ln2/2, ln2/2] by least squares at Chebyshev nodes (relative error 1.8e-8
// with these float coefficients), 2^k added to the exponent field. Rounding is
// to nearest throughout, so the error (~1 ulp) has no systematic sign.
// x < -86 is clamped to -86 (4e-38, keeps 2^k normal).
__device__ __forceinline__ float exp_poly(float x) {
    const float kMagic = 12582912.0f;  // 1.5 * 2^23: adding it rounds to an integer
    x = fmaxf(x, -86.0f);
    const float t = __fmaf_rn(x, 1.44269502162933349609375f, kMagic);
    const float kf = __fsub_rn(t, kMagic);
    float r = __fmaf_rn(kf, -0.693359375f, x);               // exact
    r = __fmaf_rn(kf, 2.1219444170128554e-04f, r);             // ln2 = head - (-tail)
    float p = 0.0013829420786350965f;
    p = __fmaf_rn(p, r, 0.008374771103262901f);
    p = __fmaf_rn(p, r, 0.0416683591902256f);
    p = __fmaf_rn(p, r, 0.1666642129421234f);
    p = __fmaf_rn(p, r, 0.49999991059303284f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    // bits(t) = bits(kMagic) + k and bits(kMagic) << 23 == 0 (mod 2^32)
    return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// ---- packed fp32x2 arithmetic (sm_100: one instruction for two lanes, each
// lane an IEEE round-to-nearest operation, so results equal the scalar ops) ----
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pack2(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack2(f32x2 v, float& lo, float& hi) {
    asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// max of three (sm_100 three-input max.f32; NaN inputs are ignored like fmaxf)
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// exp_poly on two lanes at once: the same operations in the same order, so
// each lane's result equals exp_poly of that lane.
__device__ __forceinline__ f32x2 exp_poly2(float a, float b) {
    const f32x2 kLog2e = 0x3fb8aa3b3fb8aa3bull, kMagic = 0x4b4000004b400000ull,
                kNegMagic = 0xcb400000cb400000ull, kNegHi = 0xbf318000bf318000ull,
                kLo = 0x395e8083395e8083ull, kC6 = 0x3ab543d63ab543d6ull, kC5 = 0x3c0936563c093656ull,
                kC4 = 0x3d2aac713d2aac71ull, kC3 = 0x3e2aaa063e2aaa06ull, kC2 = 0x3efffffd3efffffdull,
                kOne = 0x3f8000003f800000ull;
    const f32x2 x = pack2(fmaxf(a, -86.0f), fmaxf(b, -86.0f));
    const f32x2 t = fma2(x, kLog2e, kMagic);
    const f32x2 kf = add2(t, kNegMagic);
    f32x2 r = fma2(kf, kNegHi, x);
    r = fma2(kf, kLo, r);
    f32x2 p = fma2(kC6, r, kC5);
    p = fma2(p, r, kC4);
    p = fma2(p, r, kC3);
    p = fma2(p, r, kC2);
    p = fma2(p, r, kOne);
    p = fma2(p, r, kOne);
    float pa, pb, ta, tb;
    unpack2(p, pa, pb);
    unpack2(t, ta, tb);
    // bits(t) = 0x4b400000 + k and 0x4b400000 << 23 == 0 (mod 2^32), so
    // bits(t) << 23 == k << 23: the exponent step of 2^k in one shift
    return pack2(__int_as_float(__float_as_int(pa) + (__float_as_int(ta) << 23)),
                 __int_as_float(__float_as_int(pb) + (__float_as_int(tb) << 23)));
}

// 2^t from the MUFU unit (PTX ex2.approx.ftz.f32: ~2 ulp; -inf gives +0).
__device__ __forceinline__ float ex2_approx(float t) {
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t));
    return e;
}

// e^x = 2^(x * float(log2 e)) for x <= 0: one multiply and one MUFU op, no
// clamp needed (x = -inf gives 0). Error: ex2.approx (~2 ulp) plus the
// rounding of the product (|x*log2e| * 2^-24 absolute in the exponent); both
// are small for the terms that carry the window sum (x near 0).
__device__ __forceinline__ float exp_fast(float x) {
    return ex2_approx(__fmul_rn(x, 1.44269502162933349609375f));
}
// Two lanes: one packed multiply, two MUFU ops.
__device__ __forceinline__ f32x2 exp_fast2(f32x2 x) {
    const f32x2 kLog2e = 0x3fb8aa3b3fb8aa3bull;
    float t0, t1;
    unpack2(mul2(x, kLog2e), t0, t1);
    return pack2(ex2_approx(t0), ex2_approx(t1));
}

// The exp used for the terms of the window sum (compile-time choice):
// 0 expf, 1 exp_term, 2 exp_poly, 3 exp_fast (MUFU), 4 half of the pairs of
// a tile on MUFU and half on the FMA pipe (exp_poly), balancing the two units.
#ifndef QS_SUM_EXP
#define QS_SUM_EXP 3
#endif
__device__ __forceinline__ float sum_term_exp(float x) {
#if QS_SUM_EXP == 0
    return expf(x);
#elif QS_SUM_EXP == 1
    return exp_term(x);
#elif QS_SUM_EXP == 2 || QS_SUM_EXP == 4
    return exp_poly(x);
#else
    return exp_fast(x);
#endif
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(FULL, v, o));
    return v;
}
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}
template <typename T>
__device__ __forceinline__ T warp_incl_scan(T v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T n = __shfl_up_sync(FULL, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// exp(x) rounded once to float (through double). Kept out of line: the
// whole-row passes of the select path call it from unrolled loops, where an
// inlined copy per element made the kernel's code too large for the
// instruction cache.
#ifndef QS_EXP_NOINLINE
#define QS_EXP_NOINLINE 1
#endif
#if QS_EXP_NOINLINE
static __device__ __noinline__
#else
static __device__ __forceinline__
#endif
float exp_rounded(float x) {
    return __double2float_rn(exp((double)x));
}
// p key of one penalized, scaled logit: bits of p = (float)exp(sc - M) * inv,
// 0 outside the window. Every path uses it, so they agree bit for bit. For
// finite logits p <= 1; the clamp keeps every key that non-finite logits
// could produce (inf, NaN, negative NaN bits) at or below the key of 1.0f,
// so keys always index the histograms and buckets in range.
__device__ __forceinline__ uint32_t p_key(float sc, float M, float thr, float inv) {
    if (!(sc >= thr)) return 0u;
    const float e = exp_rounded(__fsub_rn(sc, M));
    return min(__float_as_uint(__fmul_rn(e, inv)), 0x3F800000u);
}

}  // namespace qs
