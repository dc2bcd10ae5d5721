// selftest.cu - device self-test entry of libquasar_cuda (no reference
// counterpart): evaluates the exp variants the sampler uses on caller data so
// the GPU tests can bound their error and bias against a double-precision exp.
#include <math.h>

#include "common.cuh"

namespace qs {
namespace selftest {

__global__ void exp_kernel(const float* x, float* out, int n, int which) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = x[i];
        float r;
        if (which == 0) r = exp_term(v);
        else if (which == 1) r = expf(v);
        else if (which == 2) r = __double2float_rn(exp((double)v));
        else if (which == 3) r = exp_poly(v);
        else r = exp_fast(v);
        out[i] = r;
    }
}

}  // namespace selftest
}  // namespace qs

extern "C" int quasar_selftest_exp(const float* d_x, float* d_out, int n, int which, void* stream) {
    if (n < 0 || which < 0 || which > 4 || (n > 0 && (!d_x || !d_out))) return QUASAR_EINVAL;
    if (n == 0) return QUASAR_OK;
    const int blocks = (n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096;
    qs::selftest::exp_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(d_x, d_out, n, which);
    return cudaGetLastError() == cudaSuccess ? QUASAR_OK : QUASAR_ECUDA;
}
