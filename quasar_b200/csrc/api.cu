// api.cu - C ABI of libquasar_cuda: the sample.h drop-in and the batched entry.
//
// Reference interface replaced: franzvill/quasar sample.h:12-29 (sample.c:31-178).
// The sampler object keeps the reference's host-side fields (params, clamps,
// seeding) and moves the state that a pick touches - the PRNG word and the
// history ring - into device memory, so a pick is one kernel launch.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <map>
#include <mutex>
#include <utility>

#include "../../include/quasar_sampler.h"
#include "sample_rows.cuh"

struct quasar_sampler {
    // configuration after the clamps of sample.c:51-56
    float temperature, top_p, min_p, repeat_penalty;
    int top_k, repeat_last_n;
    uint64_t seed_state;  // PRNG word to upload when `rng_dirty`
    int rng_dirty;

    // device state, allocated lazily on `device`
    int device;
    cudaStream_t stream;
    uint64_t* d_rng;
    int32_t* d_meta;  // [0] ring length, [1] ring head, [2] chosen id
    int32_t* d_hist;
    int hist_cap;
    float* d_logits;
    int logits_cap;
    int32_t* h_id;  // pinned
    void* d_ws;     // this object's kernel workspace (stream-ordered allocation)
    size_t ws_bytes;
    int last_error;
};

namespace {

// Workspaces the library keeps for quasar_sampler_pick_batch callers that pass
// none: one per (device, stream), so calls on different streams never share
// one, and calls on one stream are ordered by the stream. Growth frees the old
// buffer stream-ordered (cudaFreeAsync after the work already queued on that
// stream) and allocates the new one the same way, so it never waits for the
// device. The mutex is held until the launch is queued, so a concurrent grow
// on the same stream cannot free a buffer another thread is about to use.
struct ManagedWs {
    void* ptr;     // allocation
    size_t bytes;  // usable bytes from align256(ptr)
};

// Workspaces must start on a 256-byte boundary; allocations get 256 bytes of
// slack and are used from the first aligned address.
void* align256(void* p) { return (void*)(((uintptr_t)p + 255) & ~(uintptr_t)255); }
std::mutex g_ws_mu;
std::map<std::pair<int, uintptr_t>, ManagedWs> g_ws;

int managed_workspace(size_t bytes, cudaStream_t stream, void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return QUASAR_ECUDA;
    ManagedWs& w = g_ws[std::make_pair(dev, (uintptr_t)stream)];
    if (w.bytes < bytes) {
        if (w.ptr && cudaFreeAsync(w.ptr, stream) != cudaSuccess) return QUASAR_ECUDA;
        w.ptr = nullptr;
        w.bytes = 0;
        const size_t grow = bytes < ((size_t)1 << 16) ? ((size_t)1 << 16) : bytes;
        if (cudaMallocAsync(&w.ptr, grow + 256, stream) != cudaSuccess) {
            w.ptr = nullptr;
            return QUASAR_ENOMEM;
        }
        w.bytes = grow;
    }
    *out = align256(w.ptr);
    return QUASAR_OK;
}

// Grows a sampler object's own workspace on its own stream (sample.c:94-104
// keeps scratch per object the same way).
int object_workspace(quasar_sampler* s, size_t bytes) {
    if (s->ws_bytes >= bytes) return QUASAR_OK;
    if (s->d_ws && cudaFreeAsync(s->d_ws, s->stream) != cudaSuccess) return QUASAR_ECUDA;
    s->d_ws = nullptr;
    s->ws_bytes = 0;
    if (cudaMallocAsync(&s->d_ws, bytes + 256, s->stream) != cudaSuccess) {
        s->d_ws = nullptr;
        return QUASAR_ENOMEM;
    }
    s->ws_bytes = bytes;
    return QUASAR_OK;
}

int set_err(quasar_sampler* s, int rc) {
    if (s) s->last_error = rc;
    return rc;
}

int ensure_device(quasar_sampler* s) {
    if (s->stream) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return QUASAR_ECUDA;
        if (dev != s->device && cudaSetDevice(s->device) != cudaSuccess) return QUASAR_ECUDA;
        return QUASAR_OK;
    }
    if (cudaGetDevice(&s->device) != cudaSuccess) return QUASAR_ECUDA;
    if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess) {
        s->stream = nullptr;
        return QUASAR_ECUDA;
    }
    if (cudaMalloc(&s->d_rng, sizeof(uint64_t)) != cudaSuccess) return QUASAR_ENOMEM;
    if (cudaMalloc(&s->d_meta, 4 * sizeof(int32_t)) != cudaSuccess) return QUASAR_ENOMEM;
    if (cudaMallocHost(&s->h_id, sizeof(int32_t)) != cudaSuccess) return QUASAR_ENOMEM;
    if (cudaMemsetAsync(s->d_meta, 0, 4 * sizeof(int32_t), s->stream) != cudaSuccess)
        return QUASAR_ECUDA;
    s->rng_dirty = 1;
    return QUASAR_OK;
}

int sync_config(quasar_sampler* s) {
    int rc = ensure_device(s);
    if (rc != QUASAR_OK) return rc;
    // sample.c:61-66: the ring is reallocated only for a new nonzero capacity;
    // repeat_last_n = 0 keeps an existing ring (and its recording) in place.
    if (s->repeat_last_n > 0 && s->repeat_last_n != s->hist_cap) {
        if (s->d_hist && cudaFreeAsync(s->d_hist, s->stream) != cudaSuccess) return QUASAR_ECUDA;
        s->d_hist = nullptr;
        s->hist_cap = 0;
        if (cudaMallocAsync((void**)&s->d_hist, (size_t)s->repeat_last_n * sizeof(int32_t), s->stream) !=
            cudaSuccess) {
            s->d_hist = nullptr;
            return QUASAR_ENOMEM;
        }
        if (cudaMemsetAsync(s->d_hist, 0, (size_t)s->repeat_last_n * sizeof(int32_t),
                            s->stream) != cudaSuccess)
            return QUASAR_ECUDA;
        s->hist_cap = s->repeat_last_n;
    }
    // this object's own workspace for a one-row pick with its ring
    rc = object_workspace(s, qs::rows_workspace_bytes(1, s->hist_cap));
    if (rc != QUASAR_OK) return rc;
    if (s->rng_dirty) {
        if (cudaMemcpyAsync(s->d_rng, &s->seed_state, sizeof(uint64_t), cudaMemcpyHostToDevice,
                            s->stream) != cudaSuccess)
            return QUASAR_ECUDA;
        // the host word must outlive the async copy
        if (cudaStreamSynchronize(s->stream) != cudaSuccess) return QUASAR_ECUDA;
        s->rng_dirty = 0;
    }
    return QUASAR_OK;
}

}  // namespace

namespace qs {

bool rows_tma_ok(const float* d_logits, int64_t ld, int V) {
    return ((uintptr_t)d_logits % 16 == 0) && (ld % 4 == 0) && (V % 4 == 0) &&
           rows_tma_smem_bytes(V) <= 220 * 1024;
}

int check_pick_batch_args(const float* d_logits, int64_t ld, int B, int V, const quasar_sample_params* d_params,
                          const quasar_sample_params* h_params, const uint64_t* d_rng, const int32_t* d_hist,
                          int hist_cap, const int32_t* d_hist_len, const int32_t* d_hist_head, int record,
                          const int32_t* d_out) {
    if (B < 0 || V < 1 || V > QUASAR_MAX_VOCAB || ld < V) return QUASAR_EINVAL;
    if (B == 0) return QUASAR_OK;
    if (!d_logits || !d_rng || !d_out || (!d_params && !h_params)) return QUASAR_EINVAL;
    if (hist_cap < 0 || (hist_cap > 0 && !d_hist)) return QUASAR_EINVAL;
    if (record && hist_cap > 0 && (!d_hist_len || !d_hist_head)) return QUASAR_EINVAL;
    if (!rows_tma_ok(d_logits, ld, V) && rows_smem_bytes(V) > 220 * 1024) return QUASAR_EUNSUPPORTED;
    return QUASAR_OK;
}

}  // namespace qs

extern "C" {

const char* quasar_status_string(int status) {
    switch (status) {
        case QUASAR_OK: return "ok";
        case QUASAR_EINVAL: return "invalid argument";
        case QUASAR_EUNSUPPORTED: return "unsupported shape";
        case QUASAR_ECUDA: return "CUDA error";
        case QUASAR_ENOMEM: return "out of memory";
        case QUASAR_ENCCL: return "NCCL error";
        case QUASAR_EOVERFLOW: return "buffer overflow";
        default: return "unknown status";
    }
}

int quasar_sampler_pick_batch_launches(void) { return 2; }

int quasar_sampler_split_shards(const float* d_logits, int64_t ld, int B, int V,
                                const quasar_sample_params* d_params, const quasar_sample_params* h_params,
                                int hist_cap, int flags) {
    if (B < 1 || V < 1 || V > QUASAR_MAX_VOCAB || ld < V || (!d_params && !h_params) || hist_cap < 0) return 0;
    qs::RowsArgs a;
    memset(&a, 0, sizeof a);
    a.B = B;
    a.V = V;
    a.d_params = d_params;
    if (h_params) a.h_params = *h_params;
    a.hist = hist_cap > 0 ? reinterpret_cast<int32_t*>(1) : nullptr;  // only its presence is read
    a.hist_cap = hist_cap;
    a.flags = flags;
    a.tma = qs::rows_tma_ok(d_logits, ld, V) && !(flags & QUASAR_FLAG_NO_TMA);
    return qs::small_batch_shards(a);
}

size_t quasar_sampler_workspace_bytes(int B, int hist_cap) {
    return B > 0 ? qs::rows_workspace_bytes(B, hist_cap) : 0;
}

int quasar_sampler_pick_batch(const float* d_logits, int64_t ld, int B, int V,
                              const quasar_sample_params* d_params,
                              const quasar_sample_params* h_params, uint64_t* d_rng,
                              int32_t* d_hist, int hist_cap, int32_t* d_hist_len,
                              int32_t* d_hist_head, int record, int32_t* d_out,
                              quasar_pick_diag* d_diag, void* d_workspace, size_t workspace_bytes,
                              int flags, void* stream) {
    const int rc = qs::check_pick_batch_args(d_logits, ld, B, V, d_params, h_params, d_rng, d_hist, hist_cap,
                                             d_hist_len, d_hist_head, record, d_out);
    if (rc != QUASAR_OK || B == 0) return rc;
    qs::RowsArgs a;
    memset(&a, 0, sizeof a);
    a.logits = d_logits;
    a.ld = ld;
    a.B = B;
    a.V = V;
    a.d_params = d_params;
    if (h_params) a.h_params = *h_params;
    a.rng = d_rng;
    a.hist = hist_cap > 0 ? d_hist : nullptr;
    a.hist_cap = hist_cap;
    a.hist_len = d_hist_len;
    a.hist_head = d_hist_head;
    a.record = record;
    a.out = d_out;
    a.diag = d_diag;
    a.flags = flags;
    a.vec = ((uintptr_t)d_logits % 32 == 0) && (ld % 8 == 0);
    a.tma = qs::rows_tma_ok(d_logits, ld, V) && !(flags & QUASAR_FLAG_NO_TMA);
    const cudaStream_t st = (cudaStream_t)stream;
    if (d_workspace && (workspace_bytes < qs::rows_workspace_bytes(B, hist_cap) || (uintptr_t)d_workspace % 256 != 0))
        return QUASAR_EINVAL;
    // a small batch with host parameters: one fused kernel, a cluster of G
    // CTAs per row (no workspace)
    const int G = qs::small_batch_shards(a);
    if (G > 0) return qs::launch_small_batch(a, G, st) == cudaSuccess ? QUASAR_OK : QUASAR_ECUDA;
    if (d_workspace) return qs::launch_sample_rows(a, d_workspace, st) == cudaSuccess ? QUASAR_OK : QUASAR_ECUDA;
    std::lock_guard<std::mutex> lock(g_ws_mu);  // held until the launch is queued
    void* ws = nullptr;
    const int wrc = managed_workspace(qs::rows_workspace_bytes(B, hist_cap), st, &ws);
    if (wrc != QUASAR_OK) return wrc;
    return qs::launch_sample_rows(a, ws, st) == cudaSuccess ? QUASAR_OK : QUASAR_ECUDA;
}

quasar_sampler* quasar_sampler_new(void) {
    quasar_sampler* s = (quasar_sampler*)calloc(1, sizeof *s);
    if (!s) return nullptr;
    s->temperature = 0.0f;  // greedy by default (sample.c:34)
    s->top_p = 1.0f;
    s->top_k = 0;
    s->min_p = 0.0f;
    s->repeat_penalty = 1.0f;
    s->repeat_last_n = 0;
    s->seed_state = 0x9E3779B97F4A7C15ull;  // sample.c:37
    s->rng_dirty = 1;
    return s;
}

void quasar_sampler_free(quasar_sampler* s) {
    if (!s) return;
    if (s->stream) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev != s->device) cudaSetDevice(s->device);
        if (s->d_ws) cudaFreeAsync(s->d_ws, s->stream);
        if (s->d_hist) cudaFreeAsync(s->d_hist, s->stream);
        if (s->d_logits) cudaFreeAsync(s->d_logits, s->stream);
        cudaStreamSynchronize(s->stream);
        cudaFree(s->d_rng);
        cudaFree(s->d_meta);
        cudaFreeHost(s->h_id);
        cudaStreamDestroy(s->stream);
        if (dev != s->device) cudaSetDevice(dev);
    }
    free(s);
}

void quasar_sampler_config(quasar_sampler* s, float temperature, float top_p, int top_k,
                           float min_p, float repeat_penalty, int repeat_last_n, uint64_t seed) {
    if (!s) return;
    s->temperature = temperature;
    s->top_p = (top_p > 0.0f && top_p < 1.0f) ? top_p : 1.0f;
    s->top_k = top_k > 0 ? top_k : 0;
    s->min_p = min_p > 0.0f ? min_p : 0.0f;
    s->repeat_penalty = repeat_penalty > 1.0f ? repeat_penalty : 1.0f;
    s->repeat_last_n = repeat_last_n > 0 ? repeat_last_n : 0;
    if (seed == 0) seed = (uint64_t)time(NULL) * 2654435761u + 0x1234567u;  // sample.c:58
    s->seed_state = seed ? seed : 0x9E3779B97F4A7C15ull;
    s->rng_dirty = 1;
    int rc = sync_config(s);
    if (rc == QUASAR_OK && s->d_meta &&
        cudaMemsetAsync(s->d_meta, 0, 2 * sizeof(int32_t), s->stream) != cudaSuccess)
        rc = QUASAR_ECUDA;
    set_err(s, rc);
}

void quasar_sampler_reset(quasar_sampler* s) {
    if (!s) return;
    int rc = ensure_device(s);
    if (rc == QUASAR_OK &&
        cudaMemsetAsync(s->d_meta, 0, 2 * sizeof(int32_t), s->stream) != cudaSuccess)
        rc = QUASAR_ECUDA;
    set_err(s, rc);
}

int quasar_sampler_last_error(const quasar_sampler* s) { return s ? s->last_error : QUASAR_EINVAL; }

int quasar_sampler_pick(quasar_sampler* s, const float* logits, int n_vocab) {
    if (!s) return -1;
    if (n_vocab <= 0) return 0;  // sample.c:112
    if (!logits || n_vocab > QUASAR_MAX_VOCAB) {
        set_err(s, QUASAR_EINVAL);
        return -1;
    }
    int rc = sync_config(s);
    if (rc != QUASAR_OK) return set_err(s, rc), -1;

    const float* d_in = logits;
    cudaPointerAttributes attr;
    const bool on_device = cudaPointerGetAttributes(&attr, logits) == cudaSuccess &&
                           (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged);
    cudaGetLastError();  // clear a benign error from the attribute query
    if (!on_device) {
        if (s->logits_cap < n_vocab) {
            if (s->d_logits && cudaFreeAsync(s->d_logits, s->stream) != cudaSuccess)
                return set_err(s, QUASAR_ECUDA), -1;
            s->d_logits = nullptr;
            s->logits_cap = 0;
            if (cudaMallocAsync((void**)&s->d_logits, (size_t)n_vocab * sizeof(float), s->stream) != cudaSuccess) {
                s->d_logits = nullptr;
                return set_err(s, QUASAR_ENOMEM), -1;
            }
            s->logits_cap = n_vocab;
        }
        if (cudaMemcpyAsync(s->d_logits, logits, (size_t)n_vocab * sizeof(float),
                            cudaMemcpyHostToDevice, s->stream) != cudaSuccess)
            return set_err(s, QUASAR_ECUDA), -1;
        d_in = s->d_logits;
    }
    quasar_sample_params p;
    p.temperature = s->temperature;
    p.top_p = s->top_p;
    p.min_p = s->min_p;
    p.repeat_penalty = s->repeat_penalty;
    p.top_k = s->top_k;
    p.reserved = 0;
    rc = quasar_sampler_pick_batch(d_in, n_vocab, 1, n_vocab, nullptr, &p, s->d_rng, s->d_hist,
                                   s->hist_cap, s->d_meta, s->d_meta + 1, 1, s->d_meta + 2,
                                   nullptr, align256(s->d_ws), s->ws_bytes, 0, s->stream);
    if (rc != QUASAR_OK) return set_err(s, rc), -1;
    if (cudaMemcpyAsync(s->h_id, s->d_meta + 2, sizeof(int32_t), cudaMemcpyDeviceToHost,
                        s->stream) != cudaSuccess ||
        cudaStreamSynchronize(s->stream) != cudaSuccess)
        return set_err(s, QUASAR_ECUDA), -1;
    set_err(s, QUASAR_OK);
    return *s->h_id;
}

}  // extern "C"
