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

}  // namespace qs
