// sample_rows.cuh - launcher of the batched row sampler (sample_rows.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/quasar_sampler.h"

namespace qs {

struct RowsArgs {
    const float* logits;
    int64_t ld;
    int B, V;
    const quasar_sample_params* d_params;
    quasar_sample_params h_params;
    uint64_t* rng;
    int32_t* hist;
    int hist_cap;
    int32_t* hist_len;
    int32_t* hist_head;
    int record;
    int32_t* out;
    quasar_pick_diag* diag;
    int flags;
    int vec;     // rows 32-byte aligned with ld % 8 == 0 (256-bit global loads)
    int tma;     // rows 16-byte aligned, ld % 4 == 0, V % 4 == 0 (bulk-copy ring kernel)
    int nwords;  // bitset words (set by the launcher)
    // per-row summaries kernel A leaves for kernel B (workspace; set by the launcher)
    int* work_abort;
    float4* work_info;      // (max scaled logit, 1/sum, penalized count as int bits, 0)
    float* work_tfmax;      // [B][256] per-thread final maxima
    int2* work_pen;         // [B][hist_cap] (id, scaled penalized logit as int bits)
    uint8_t* work_tmax;     // [B][TMAX] tile-max deficits
    uint8_t* work_anc;      // [B][NCK][256] checkpoint deficits below the thread's final max
    // vocab shards (quasar_shard_*): this matrix holds global columns
    // [col0, col0 + V); kernel A publishes per-row stats instead of finishing
    // greedy rows, and the finishing kernel emits candidate keys
    int64_t col0;
    quasar_shard_stat* shard_stats;        // [B] out (kernel A), or NULL
    const quasar_shard_stat* all_stats;    // [G][B] in (candidate and merge kernels)
    int shard_G, shard_k, shard_rank;
    uint64_t* shard_cand;                  // candidate kernel: [B][k] out; merge: [G][B][k] in
};

size_t rows_smem_bytes(int V);      // one-CTA-per-row kernel
size_t rows_tma_smem_bytes(int V);  // persistent bulk-copy ring kernel
size_t rows_finish_smem_bytes(int V);
size_t rows_workspace_bytes(int B, int hist_cap);  // device workspace of one launch
int rows_threads();
// Rows that the bulk-copy ring kernel can stream (16-byte aligned, ld % 4 == 0,
// V % 4 == 0, ring + bitset within shared memory).
bool rows_tma_ok(const float* d_logits, int64_t ld, int V);
// Argument checks of quasar_sampler_pick_batch (QUASAR_OK, QUASAR_EINVAL or
// QUASAR_EUNSUPPORTED); B == 0 passes.
int check_pick_batch_args(const float* d_logits, int64_t ld, int B, int V, const quasar_sample_params* d_params,
                          const quasar_sample_params* h_params, const uint64_t* d_rng, const int32_t* d_hist,
                          int hist_cap, const int32_t* d_hist_len, const int32_t* d_hist_head, int record,
                          const int32_t* d_out);
// Launches kernel A (one streaming pass per row) and kernel B (cuts and draw).
cudaError_t launch_sample_rows(const RowsArgs& args, void* workspace, cudaStream_t stream);
// Vocab shards: kernel A alone (per-row stats into args.shard_stats), kernel
// B in candidate mode (needs the same workspace), and the merge kernel.
cudaError_t launch_shard_stats(const RowsArgs& args, void* workspace, cudaStream_t stream);
cudaError_t launch_shard_candidates(const RowsArgs& args, void* workspace, cudaStream_t stream);
size_t rows_merge_smem_bytes(int G, int k);
cudaError_t launch_shard_merge(const RowsArgs& args, cudaStream_t stream);
// Small batches (small_batch.cu): at most SPLIT_MAX_B rows whose parameters
// are on the host (args.d_params NULL), each greedy or with 1 <= top_k <= 256,
// are sampled by one fused kernel in which a cluster of G CTAs holds each row
// in shared memory. small_batch_shards returns G (0: the batch does not
// qualify); launch_small_batch needs no workspace.
constexpr int SPLIT_MAX_B = 16;
int small_batch_shards(const RowsArgs& args);
cudaError_t launch_small_batch(const RowsArgs& args, int G, cudaStream_t stream);

}  // namespace qs
