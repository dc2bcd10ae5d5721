// shard.cu - C ABI of the vocab-sharded sampler (quasar_shard_*): argument
// checks and launches of the kernels in sample_rows.cu in shard mode.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/quasar_sampler.h"
#include "sample_rows.cuh"

namespace {

int common_args(qs::RowsArgs& a, const float* d_logits, int64_t ld, int B, int Vs, int64_t col0,
                const quasar_sample_params* d_params, const quasar_sample_params* h_params, const int32_t* d_hist,
                int hist_cap, const int32_t* d_hist_len, const int32_t* d_hist_head, int flags) {
    if (B < 0 || Vs < 1 || Vs > QUASAR_MAX_VOCAB || ld < Vs || col0 < 0) return QUASAR_EINVAL;
    if (B > 0 && (!d_logits || (!d_params && !h_params))) return QUASAR_EINVAL;
    if (hist_cap < 0 || (hist_cap > 0 && !d_hist)) return QUASAR_EINVAL;
    const bool tma = ((uintptr_t)d_logits % 16 == 0) && (ld % 4 == 0) && (Vs % 4 == 0) &&
                     qs::rows_tma_smem_bytes(Vs) <= 220 * 1024;
    if (!tma && qs::rows_smem_bytes(Vs) > 220 * 1024) return QUASAR_EUNSUPPORTED;
    memset(&a, 0, sizeof a);
    a.logits = d_logits;
    a.ld = ld;
    a.B = B;
    a.V = Vs;
    a.d_params = d_params;
    if (h_params) a.h_params = *h_params;
    a.hist = hist_cap > 0 ? const_cast<int32_t*>(d_hist) : nullptr;
    a.hist_cap = hist_cap;
    a.hist_len = const_cast<int32_t*>(d_hist_len);
    a.hist_head = const_cast<int32_t*>(d_hist_head);
    a.flags = flags;
    a.vec = ((uintptr_t)d_logits % 32 == 0) && (ld % 8 == 0);
    a.tma = tma && !(flags & QUASAR_FLAG_NO_TMA);
    a.col0 = col0;
    return QUASAR_OK;
}

int workspace_ok(const void* ws, size_t bytes, int B, int hist_cap) {
    return ws && bytes >= qs::rows_workspace_bytes(B, hist_cap) && (uintptr_t)ws % 256 == 0;
}

}  // namespace

extern "C" int quasar_shard_stats(const float* d_logits, int64_t ld, int B, int Vs, int64_t col0,
                                  const quasar_sample_params* d_params, const quasar_sample_params* h_params,
                                  const int32_t* d_hist, int hist_cap, const int32_t* d_hist_len,
                                  const int32_t* d_hist_head, quasar_shard_stat* d_stats, void* d_workspace,
                                  size_t workspace_bytes, int flags, void* stream) {
    qs::RowsArgs a;
    int rc = common_args(a, d_logits, ld, B, Vs, col0, d_params, h_params, d_hist, hist_cap, d_hist_len,
                         d_hist_head, flags);
    if (rc != QUASAR_OK) return rc;
    if (B == 0) return QUASAR_OK;
    if (!d_stats || !workspace_ok(d_workspace, workspace_bytes, B, hist_cap)) return QUASAR_EINVAL;
    a.shard_stats = d_stats;
    return qs::launch_shard_stats(a, d_workspace, (cudaStream_t)stream) == cudaSuccess ? QUASAR_OK : QUASAR_ECUDA;
}

extern "C" int quasar_shard_candidates(const float* d_logits, int64_t ld, int B, int Vs, int64_t col0,
                                       const quasar_sample_params* d_params,
                                       const quasar_sample_params* h_params, const int32_t* d_hist,
                                       int hist_cap, const int32_t* d_hist_len, const int32_t* d_hist_head,
                                       const quasar_shard_stat* d_all_stats, int G, int rank, int k,
                                       uint64_t* d_cand, void* d_workspace, size_t workspace_bytes, int flags,
                                       void* stream) {
    qs::RowsArgs a;
    int rc = common_args(a, d_logits, ld, B, Vs, col0, d_params, h_params, d_hist, hist_cap, d_hist_len,
                         d_hist_head, flags);
    if (rc != QUASAR_OK) return rc;
    if (G < 1 || G > 64 || rank < 0 || rank >= G || k < 1 || k > 256) return QUASAR_EINVAL;
    if (B == 0) return QUASAR_OK;
    if (!d_all_stats || !d_cand || !workspace_ok(d_workspace, workspace_bytes, B, hist_cap)) return QUASAR_EINVAL;
    a.all_stats = d_all_stats;
    a.shard_G = G;
    a.shard_rank = rank;
    a.shard_k = k;
    a.shard_cand = d_cand;
    a.flags &= ~QUASAR_FLAG_EXACT_SELECT;  // shards always use the candidate path
    return qs::launch_shard_candidates(a, d_workspace, (cudaStream_t)stream) == cudaSuccess ? QUASAR_OK
                                                                                            : QUASAR_ECUDA;
}

extern "C" int quasar_shard_finish(const uint64_t* d_all_cand, const quasar_shard_stat* d_all_stats, int G, int k,
                                   int B, const quasar_sample_params* d_params,
                                   const quasar_sample_params* h_params, uint64_t* d_rng, int32_t* d_hist,
                                   int hist_cap, int32_t* d_hist_len, int32_t* d_hist_head, int record,
                                   int32_t* d_out, quasar_pick_diag* d_diag, void* stream) {
    if (B < 0 || G < 1 || G > 64 || k < 1 || k > 256) return QUASAR_EINVAL;
    if (B == 0) return QUASAR_OK;
    if (!d_all_cand || !d_all_stats || !d_rng || !d_out || (!d_params && !h_params)) return QUASAR_EINVAL;
    if (hist_cap < 0 || (hist_cap > 0 && !d_hist)) return QUASAR_EINVAL;
    if (record && hist_cap > 0 && (!d_hist_len || !d_hist_head)) return QUASAR_EINVAL;
    qs::RowsArgs a;
    memset(&a, 0, sizeof a);
    a.B = B;
    a.V = 1;
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
    a.all_stats = d_all_stats;
    a.shard_G = G;
    a.shard_k = k;
    a.shard_cand = const_cast<uint64_t*>(d_all_cand);
    return qs::launch_shard_merge(a, (cudaStream_t)stream) == cudaSuccess ? QUASAR_OK : QUASAR_ECUDA;
}
