// nccl_shard.cu - vocab-sharded sampling over NCCL, in C: a communicator
// wrapper with bounded waits and abort, and quasar_shard_pick, which runs the
// three phases of sample_rows.cu in shard mode with the two exchanges between
// them on the caller's stream.
//
// No counterpart in franzvill/quasar (its sampler, sample.c:111-178, is one
// CPU row at a time). The exchanges are NCCL all-gathers, in place: phase 1
// writes this rank's per-row stats straight into its slot of the gathered
// array, phase 2 its candidate keys likewise, so no copies are needed.
//
// NCCL is loaded at run time (dlopen), not linked: the library the process
// already uses (a framework's libnccl.so.2) is picked first, so a caller's
// own communicator (quasar_nccl_wrap) and ours come from the same library;
// QUASAR_NCCL_LIBRARY names another one; libnccl.so.2 on the loader path
// is the fallback. Communicators made here are non-blocking
// (ncclConfig_t.blocking = 0): every NCCL call that reports ncclInProgress
// is polled with ncclCommGetAsyncError under the communicator's time limit,
// and on expiry the communicator is aborted (ncclCommAbort) and the call
// returns QUASAR_ENCCL.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <mutex>

#include "../../include/quasar_sampler.h"
#include "sample_rows.cuh"

static_assert(sizeof(ncclUniqueId) == QUASAR_NCCL_ID_BYTES, "unique id size");
static_assert(sizeof(quasar_shard_stat) == 16, "shard stat layout");

namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id;
    decltype(&ncclCommInitRankConfig) init_rank_config;
    decltype(&ncclCommGetAsyncError) get_async_error;
    decltype(&ncclCommAbort) abort;
    decltype(&ncclCommFinalize) finalize;
    decltype(&ncclCommDestroy) destroy;
    decltype(&ncclAllGather) all_gather;
    decltype(&ncclGetVersion) get_version;
};

std::once_flag g_once;
NcclApi g_api;
int g_api_status = QUASAR_ENCCL;

void load_api() {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // already in the process
    if (!h) {
        const char* path = getenv("QUASAR_NCCL_LIBRARY");
        if (path && *path) h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
    }
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    NcclApi api;
    api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
    api.init_rank_config = (decltype(api.init_rank_config))dlsym(h, "ncclCommInitRankConfig");
    api.get_async_error = (decltype(api.get_async_error))dlsym(h, "ncclCommGetAsyncError");
    api.abort = (decltype(api.abort))dlsym(h, "ncclCommAbort");
    api.finalize = (decltype(api.finalize))dlsym(h, "ncclCommFinalize");
    api.destroy = (decltype(api.destroy))dlsym(h, "ncclCommDestroy");
    api.all_gather = (decltype(api.all_gather))dlsym(h, "ncclAllGather");
    api.get_version = (decltype(api.get_version))dlsym(h, "ncclGetVersion");
    if (!api.get_unique_id || !api.init_rank_config || !api.get_async_error || !api.abort || !api.finalize ||
        !api.destroy || !api.all_gather || !api.get_version)
        return;
    g_api = api;
    g_api_status = QUASAR_OK;
}

int api() {
    std::call_once(g_once, load_api);
    return g_api_status;
}

double now_ms() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

void sleep_us(long us) {
    timespec ts = {us / 1000000, (us % 1000000) * 1000};
    nanosleep(&ts, nullptr);
}

}  // namespace

struct quasar_nccl {
    ncclComm_t comm;
    int nranks, rank, device;
    int timeout_ms;
    int owned;   // made by quasar_nccl_init (destroyed by quasar_nccl_free)
    int failed;  // aborted after an error or a timeout: unusable
};

namespace {

// Waits (bounded) until the communicator has no operation in progress on the
// host side. On an error or the time limit: abort, mark failed, QUASAR_ENCCL.
int settle(quasar_nccl* c, ncclResult_t rc) {
    if (rc == ncclSuccess) return QUASAR_OK;
    if (rc != ncclInProgress) {
        g_api.abort(c->comm);
        c->failed = 1;
        return QUASAR_ENCCL;
    }
    const double t0 = now_ms();
    for (;;) {
        ncclResult_t st = ncclInProgress;
        if (g_api.get_async_error(c->comm, &st) != ncclSuccess) st = ncclInternalError;
        if (st == ncclSuccess) return QUASAR_OK;
        if (st != ncclInProgress || (c->timeout_ms > 0 && now_ms() - t0 > c->timeout_ms)) {
            g_api.abort(c->comm);
            c->failed = 1;
            return QUASAR_ENCCL;
        }
        sleep_us(200);
    }
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

extern "C" {

int quasar_nccl_available(void) { return api(); }

int quasar_nccl_unique_id(void* id_out) {
    if (!id_out) return QUASAR_EINVAL;
    if (api() != QUASAR_OK) return QUASAR_ENCCL;
    ncclUniqueId id;
    if (g_api.get_unique_id(&id) != ncclSuccess) return QUASAR_ENCCL;
    memcpy(id_out, &id, sizeof id);
    return QUASAR_OK;
}

int quasar_nccl_init(quasar_nccl** out, int nranks, int rank, const void* unique_id, int timeout_ms) {
    if (!out || !unique_id || nranks < 1 || nranks > 64 || rank < 0 || rank >= nranks || timeout_ms < 0)
        return QUASAR_EINVAL;
    *out = nullptr;
    if (api() != QUASAR_OK) return QUASAR_ENCCL;
    quasar_nccl* c = (quasar_nccl*)calloc(1, sizeof *c);
    if (!c) return QUASAR_ENOMEM;
    if (cudaGetDevice(&c->device) != cudaSuccess) {
        free(c);
        return QUASAR_ECUDA;
    }
    c->nranks = nranks;
    c->rank = rank;
    c->timeout_ms = timeout_ms;
    c->owned = 1;
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof id);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // every call returns at once; completion is polled (settle)
    const ncclResult_t rc = g_api.init_rank_config(&c->comm, nranks, id, rank, &cfg);
    if (rc != ncclSuccess && rc != ncclInProgress) {
        if (c->comm) g_api.abort(c->comm);
        free(c);
        return QUASAR_ENCCL;
    }
    // a rank that never joins leaves the bootstrap waiting: the time limit ends it
    if (settle(c, rc) != QUASAR_OK) {
        free(c);
        return QUASAR_ENCCL;
    }
    *out = c;
    return QUASAR_OK;
}

int quasar_nccl_wrap(quasar_nccl** out, void* nccl_comm, int nranks, int rank, int timeout_ms) {
    if (!out || !nccl_comm || nranks < 1 || nranks > 64 || rank < 0 || rank >= nranks || timeout_ms < 0)
        return QUASAR_EINVAL;
    *out = nullptr;
    if (api() != QUASAR_OK) return QUASAR_ENCCL;
    quasar_nccl* c = (quasar_nccl*)calloc(1, sizeof *c);
    if (!c) return QUASAR_ENOMEM;
    if (cudaGetDevice(&c->device) != cudaSuccess) {
        free(c);
        return QUASAR_ECUDA;
    }
    c->comm = (ncclComm_t)nccl_comm;
    c->nranks = nranks;
    c->rank = rank;
    c->timeout_ms = timeout_ms;
    *out = c;
    return QUASAR_OK;
}

int quasar_nccl_abort(quasar_nccl* c) {
    if (!c) return QUASAR_EINVAL;
    if (!c->failed && c->comm) g_api.abort(c->comm);
    c->failed = 1;
    return QUASAR_OK;
}

int quasar_nccl_free(quasar_nccl* c) {
    if (!c) return QUASAR_OK;
    int rc = QUASAR_OK;
    if (c->owned && !c->failed && c->comm) {
        // flush what is queued, then release; an error or the time limit aborts
        rc = settle(c, g_api.finalize(c->comm));
        if (rc == QUASAR_OK && g_api.destroy(c->comm) != ncclSuccess) rc = QUASAR_ENCCL;
    }
    free(c);
    return rc;
}

int quasar_nccl_wait(quasar_nccl* c, void* stream, int timeout_ms) {
    if (!c) return QUASAR_EINVAL;
    if (c->failed) return QUASAR_ENCCL;
    cudaEvent_t ev;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return QUASAR_ECUDA;
    if (cudaEventRecord(ev, (cudaStream_t)stream) != cudaSuccess) {
        cudaEventDestroy(ev);
        return QUASAR_ECUDA;
    }
    const double t0 = now_ms();
    int rc = QUASAR_OK;
    for (;;) {
        const cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) {
            rc = QUASAR_ECUDA;
            break;
        }
        ncclResult_t st = ncclSuccess;
        if (g_api.get_async_error(c->comm, &st) != ncclSuccess || (st != ncclSuccess && st != ncclInProgress) ||
            (timeout_ms > 0 && now_ms() - t0 > timeout_ms)) {
            // a peer that stopped answering: abort, which also ends this
            // communicator's kernels still waiting on the device
            g_api.abort(c->comm);
            c->failed = 1;
            rc = QUASAR_ENCCL;
            break;
        }
        sleep_us(100);
    }
    if (rc == QUASAR_ENCCL) {
        // the aborted kernels finish; the event completes after them (bounded)
        const double t1 = now_ms();
        while (cudaEventQuery(ev) == cudaErrorNotReady && now_ms() - t1 < 10000.0) sleep_us(1000);
    }
    cudaEventDestroy(ev);
    return rc;
}

size_t quasar_shard_workspace_bytes(int B, int hist_cap, int G, int k) {
    if (B <= 0 || G < 1 || k < 1) return 0;
    return align256(qs::rows_workspace_bytes(B, hist_cap)) + align256((size_t)G * B * sizeof(quasar_shard_stat)) +
           align256((size_t)G * B * k * sizeof(uint64_t));
}

int quasar_shard_pick(quasar_nccl* c, const float* d_logits, int64_t ld, int B, int Vs, int64_t col0,
                      const quasar_sample_params* d_params, const quasar_sample_params* h_params, uint64_t* d_rng,
                      int32_t* d_hist, int hist_cap, int32_t* d_hist_len, int32_t* d_hist_head, int record,
                      int32_t* d_out, quasar_pick_diag* d_diag, int k, void* d_workspace, size_t workspace_bytes,
                      int flags, void* stream) {
    if (!c) return QUASAR_EINVAL;
    if (c->failed) return QUASAR_ENCCL;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return QUASAR_ECUDA;
    if (dev != c->device) return QUASAR_EINVAL;  // the communicator's device must be current
    const int G = c->nranks, rank = c->rank;
    if (B < 0 || k < 1 || k > 256) return QUASAR_EINVAL;
    if (B == 0) return QUASAR_OK;
    if (!d_workspace || (uintptr_t)d_workspace % 256 != 0 || workspace_bytes < quasar_shard_workspace_bytes(B, hist_cap, G, k))
        return QUASAR_EINVAL;
    char* ws = (char*)d_workspace;
    void* rows_ws = ws;
    const size_t rows_bytes = align256(qs::rows_workspace_bytes(B, hist_cap));
    quasar_shard_stat* all_stats = (quasar_shard_stat*)(ws + rows_bytes);
    uint64_t* all_cand = (uint64_t*)(ws + rows_bytes + align256((size_t)G * B * sizeof(quasar_shard_stat)));
    const size_t stat_bytes = (size_t)B * sizeof(quasar_shard_stat);
    const size_t cand_bytes = (size_t)B * k * sizeof(uint64_t);
    const cudaStream_t st = (cudaStream_t)stream;
    // phase 1: this rank's stats, in its slot of the gathered array
    int rc = quasar_shard_stats(d_logits, ld, B, Vs, col0, d_params, h_params, d_hist, hist_cap, d_hist_len,
                                d_hist_head, all_stats + (size_t)rank * B, rows_ws,
                                qs::rows_workspace_bytes(B, hist_cap), flags, stream);
    if (rc != QUASAR_OK) return rc;
    rc = settle(c, g_api.all_gather((const char*)(all_stats + (size_t)rank * B), all_stats, stat_bytes, ncclUint8,
                                    c->comm, st));
    if (rc != QUASAR_OK) return rc;
    // phase 2: this rank's k best candidates per row under the global max and sum
    rc = quasar_shard_candidates(d_logits, ld, B, Vs, col0, d_params, h_params, d_hist, hist_cap, d_hist_len,
                                 d_hist_head, all_stats, G, rank, k, all_cand + (size_t)rank * B * k, rows_ws,
                                 qs::rows_workspace_bytes(B, hist_cap), flags, stream);
    if (rc != QUASAR_OK) return rc;
    rc = settle(c, g_api.all_gather((const char*)(all_cand + (size_t)rank * B * k), all_cand, cand_bytes, ncclUint8,
                                    c->comm, st));
    if (rc != QUASAR_OK) return rc;
    // phase 3: merge, cuts, draw, PRNG step and ring append - the same on every rank
    return quasar_shard_finish(all_cand, all_stats, G, k, B, d_params, h_params, d_rng, d_hist, hist_cap, d_hist_len,
                               d_hist_head, record, d_out, d_diag, stream);
}

}  // extern "C"
