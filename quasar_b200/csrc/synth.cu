// synth.cu - deterministic synthetic sampler inputs on the device.
//
// Benchmark / test utility (the reference has no counterpart). The recipe uses
// only integer hashing and IEEE +, -, *, / and this file is compiled with
// -fmad=false, so every value is bit-identical to the CPU recipe the tests use:
//   NORMAL       Irwin-Hall: twelve 16-bit uniforms from three 64-bit hashes,
//                z = (2*sum - 786420) / 2^17 (exact in float), logit = z * scale
//   GUMBEL_PEAK  u = (53-bit hash + 0.5) * 2^-53, logit = -log(-log(u)), and +8
//                at one column per row (column = hash % V)
//   ZIPF         rank = (a*col + b) mod V + 1 (a coprime to V: a permutation),
//                logit = -scale * log(rank)
// log() is det_log: exponent split plus the atanh series, in double.
#include <stdint.h>

#include "../../include/quasar_sampler.h"

namespace qs {
namespace synth {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t hash3(uint64_t seed, uint64_t a, uint64_t b) {
    return mix64(mix64(seed ^ (a * 0xD1B54A32D192ED03ull)) ^ (b * 0xABC98388FB8FAC03ull));
}

__device__ double det_log(double x) {
    uint64_t bits = (uint64_t)__double_as_longlong(x);
    int e = (int)((bits >> 52) & 0x7FF) - 1023;
    bits = (bits & 0x000FFFFFFFFFFFFFull) | 0x3FF0000000000000ull;
    double m = __longlong_as_double((long long)bits);
    if (m > 1.4142135623730951) {
        m = m * 0.5;
        e = e + 1;
    }
    const double t = (m - 1.0) / (m + 1.0);
    const double t2 = t * t;
    double s = 0.043478260869565216;
    s = s * t2 + 0.047619047619047616;
    s = s * t2 + 0.05263157894736842;
    s = s * t2 + 0.058823529411764705;
    s = s * t2 + 0.06666666666666667;
    s = s * t2 + 0.07692307692307693;
    s = s * t2 + 0.09090909090909091;
    s = s * t2 + 0.1111111111111111;
    s = s * t2 + 0.14285714285714285;
    s = s * t2 + 0.2;
    s = s * t2 + 0.3333333333333333;
    s = s * t2 + 1.0;
    return (double)e * 0.6931471805599453 + 2.0 * t * s;
}

__device__ uint64_t gcd_u64(uint64_t a, uint64_t b) {
    while (b) {
        const uint64_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

constexpr int CHUNK = 4096;  // columns per CTA

__global__ void synth_logits_kernel(int kind, uint64_t seed, int64_t row0, int V, int64_t ld,
                                    float scale, float* out) {
    __shared__ uint64_t c_a, c_b, c_peak;
    const uint64_t row = (uint64_t)(row0 + blockIdx.y);
    if (threadIdx.x == 0) {
        uint64_t va = hash3(seed, row, 1ull << 62) % (uint64_t)V;
        if (va == 0) va = 1;
        while (gcd_u64(va, (uint64_t)V) != 1) va = va + 1 < (uint64_t)V ? va + 1 : 1;
        c_a = va;
        c_b = hash3(seed, row, (1ull << 62) + 1) % (uint64_t)V;
        c_peak = hash3(seed, row, 0xFFFFFFFFFFFFull) % (uint64_t)V;
    }
    __syncthreads();
    float* o = out + (int64_t)blockIdx.y * ld;
    const int c0 = blockIdx.x * CHUNK;
    const int c1 = min(c0 + CHUNK, V);
    for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
        const uint64_t col = (uint64_t)c;
        float v;
        if (kind == QUASAR_SYNTH_NORMAL) {
            int64_t s = 0;
            for (uint64_t k = 0; k < 3; k++) {
                const uint64_t h = hash3(seed, row, (col << 2) | k);
                s += (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) +
                     (int64_t)((h >> 32) & 0xFFFF) + (int64_t)(h >> 48);
            }
            const float z = (float)(2 * s - 786420) * (1.0f / 131072.0f);
            v = z * scale;
        } else if (kind == QUASAR_SYNTH_GUMBEL_PEAK) {
            const uint64_t h = hash3(seed, row, col << 2);
            const double u = ((double)(h >> 11) + 0.5) * (1.0 / 9007199254740992.0);
            float g = (float)(-det_log(-det_log(u)));
            if (col == c_peak) g = g + 8.0f;
            v = g;
        } else {
            const uint64_t rank = (c_a * col + c_b) % (uint64_t)V + 1;
            v = (float)(-(double)scale * det_log((double)rank));
        }
        o[c] = v;
    }
}

__global__ void synth_hist_kernel(uint64_t seed, int64_t row0, int B, int H, int V, int32_t* out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)B * H) return;
    const int64_t r = i / H, j = i % H;
    out[i] = (int32_t)(hash3(seed ^ 0x5DEECE66Dull, (uint64_t)(row0 + r), (uint64_t)j) % (uint64_t)V);
}

__global__ void synth_uniform_kernel(uint64_t seed, int64_t row0, int B, float lo, float hi,
                                     float* out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= B) return;
    const uint64_t h = hash3(seed ^ 0x7F4A7C15ull, (uint64_t)(row0 + r), 0);
    const float u = (float)(h >> 40) * (1.0f / 16777216.0f);
    out[r] = lo + (hi - lo) * u;
}

}  // namespace synth
}  // namespace qs

extern "C" int quasar_synth_logits(int kind, uint64_t seed, int64_t row0, int B, int V,
                                   int64_t ld, float scale, float* d_out, void* stream) {
    if (B < 0 || V < 1 || ld < V || !d_out || kind < 0 || kind > 2) return QUASAR_EINVAL;
    if (B == 0) return QUASAR_OK;
    if (B > 65535) {
        for (int64_t r = 0; r < B; r += 65535) {
            const int n = (int)(B - r < 65535 ? B - r : 65535);
            const int rc = quasar_synth_logits(kind, seed, row0 + r, n, V, ld, scale,
                                               d_out + r * ld, stream);
            if (rc != QUASAR_OK) return rc;
        }
        return QUASAR_OK;
    }
    dim3 grid((V + qs::synth::CHUNK - 1) / qs::synth::CHUNK, B);
    qs::synth::synth_logits_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(kind, seed, row0, V,
                                                                           ld, scale, d_out);
    return cudaGetLastError() == cudaSuccess ? QUASAR_OK : QUASAR_ECUDA;
}

extern "C" int quasar_synth_hist(uint64_t seed, int64_t row0, int B, int H, int V,
                                 int32_t* d_out, void* stream) {
    if (B < 0 || H < 0 || V < 1 || (!d_out && (int64_t)B * H > 0)) return QUASAR_EINVAL;
    const int64_t n = (int64_t)B * H;
    if (n == 0) return QUASAR_OK;
    const int64_t blocks = (n + 255) / 256;
    qs::synth::synth_hist_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(seed, row0, B,
                                                                                    H, V, d_out);
    return cudaGetLastError() == cudaSuccess ? QUASAR_OK : QUASAR_ECUDA;
}

extern "C" int quasar_synth_uniform(uint64_t seed, int64_t row0, int B, float lo, float hi,
                                    float* d_out, void* stream) {
    if (B < 0 || (!d_out && B > 0)) return QUASAR_EINVAL;
    if (B == 0) return QUASAR_OK;
    qs::synth::synth_uniform_kernel<<<(B + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
        seed, row0, B, lo, hi, d_out);
    return cudaGetLastError() == cudaSuccess ? QUASAR_OK : QUASAR_ECUDA;
}
