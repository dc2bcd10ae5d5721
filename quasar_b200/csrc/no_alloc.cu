// no_alloc.cu - quasar_sampler_pick_batch_noalloc: the batched sampler with its
// workspace in a fixed device array, so the call itself allocates nothing.
//
// Who needs it: a serving engine that reserves nearly all free device memory
// up front (KV cache pools sized to fill HBM) has nothing left for a
// cudaMalloc at sampling time, and a caller on a latency-critical decode loop
// cannot take the implicit device-wide synchronisation that cudaMalloc /
// cudaFree may bring. quasar_sampler_pick_batch either takes caller memory or
// allocates (and grows) a library-owned workspace; this entry point does
// neither: its workspace is the file-scope array below, created with the
// module, so no allocation happens on the call path.
//
// Limits: the array holds QUASAR_NOALLOC_WORKSPACE_BYTES; a call that needs
// more (quasar_sampler_workspace_bytes(B, hist_cap)) fails with
// QUASAR_EOVERFLOW before touching the GPU. There is one array per device and
// process, so two calls that overlap on one device (different streams or
// threads) would share it and corrupt each other's summaries: callers
// serialise them. The first call on a device looks the array's address up
// (cudaGetSymbolAddress) and sets the kernels' shared-memory attributes; that
// set-up belongs before any stream capture. The address is kept for the life
// of the process: after a cudaDeviceReset the module (and the array) may be
// loaded elsewhere, so this entry point must not be used across a device
// reset. Arguments are checked exactly as quasar_sampler_pick_batch checks
// them (QUASAR_EINVAL / QUASAR_EUNSUPPORTED) before the size check. The one workspace word that must
// be zero when the kernels start, the abort flag, is cleared by every call
// with a cudaMemsetAsync on the caller's stream (a memset, not an allocation);
// every other byte is written by the streaming kernel before the finishing
// kernel reads it.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/quasar_sampler.h"
#include "sample_rows.cuh"

namespace {

__device__ __align__(256) unsigned char g_noalloc_ws[QUASAR_NOALLOC_WORKSPACE_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_ws_addr[kMaxDevices];  // device address of g_noalloc_ws, per device

}  // namespace

extern "C" int quasar_sampler_pick_batch_noalloc(const float* d_logits, int64_t ld, int B, int V,
                                                 const quasar_sample_params* d_params,
                                                 const quasar_sample_params* h_params, uint64_t* d_rng,
                                                 int32_t* d_hist, int hist_cap, int32_t* d_hist_len,
                                                 int32_t* d_hist_head, int record, int32_t* d_out,
                                                 quasar_pick_diag* d_diag, int flags, void* stream) {
    // the same argument checks as quasar_sampler_pick_batch, before the size check
    const int rc = qs::check_pick_batch_args(d_logits, ld, B, V, d_params, h_params, d_rng, d_hist, hist_cap,
                                             d_hist_len, d_hist_head, record, d_out);
    if (rc != QUASAR_OK || B == 0) return rc;
    if (quasar_sampler_workspace_bytes(B, hist_cap) > (size_t)QUASAR_NOALLOC_WORKSPACE_BYTES)
        return QUASAR_EOVERFLOW;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return QUASAR_ECUDA;
    if (dev < 0 || dev >= kMaxDevices) return QUASAR_EUNSUPPORTED;
    void* ws = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (!g_ws_addr[dev]) {
            void* p = nullptr;
            if (cudaGetSymbolAddress(&p, g_noalloc_ws) != cudaSuccess || !p) return QUASAR_ECUDA;
            g_ws_addr[dev] = p;
        }
        ws = g_ws_addr[dev];
    }
    return quasar_sampler_pick_batch(d_logits, ld, B, V, d_params, h_params, d_rng, d_hist, hist_cap,
                                     d_hist_len, d_hist_head, record, d_out, d_diag, ws,
                                     (size_t)QUASAR_NOALLOC_WORKSPACE_BYTES, flags, stream);
}
