/* quasar_sampler.h - C ABI of libquasar_cuda, the B200 token sampler.
 *
 * A drop-in for franzvill/quasar's sampler (sample.h / sample.c): the five
 * sample.h entry points keep their names, signatures and meaning, and a batched
 * entry point samples B rows of device-resident logits per call on sm_100a.
 * All pointers named d_* are device pointers; `stream` is a cudaStream_t
 * (NULL = the legacy default stream). Status codes are QUASAR_OK (0) or one of
 * the negative QUASAR_E* values; nothing aborts and nothing falls back to the
 * CPU.
 *
 * Sampling semantics are those of sample.c:111-178, row by row:
 *   repeat penalty over the row's history ring (ids marked once, l>0 ? l/rp : l*rp)
 *   -> temperature <= 0: argmax, first index on ties, no PRNG draw
 *   -> inv_t = 1.0f/T, window sc >= max*inv_t - 30, softmax (double sum)
 *   -> order by p descending, ties by id ascending
 *   -> top-k, top-p (double cumsum >= top_p), min-p (p < min_p * p_max cuts)
 *   -> one xorshift64* draw u in [0,1), first kept index with u*rsum <= cumsum
 *   -> optional append of the chosen id to the history ring. */
#ifndef QUASAR_SAMPLER_H
#define QUASAR_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QUASAR_OK               0
#define QUASAR_EINVAL          -1  /* bad argument (size, pointer, alignment) */
#define QUASAR_EUNSUPPORTED    -2  /* shape outside what the kernels support */
#define QUASAR_ECUDA           -3  /* a CUDA runtime call failed */
#define QUASAR_ENOMEM          -4  /* device or host allocation failed */
#define QUASAR_ENCCL           -5  /* an NCCL call failed or timed out */
#define QUASAR_EOVERFLOW       -6  /* a fixed-capacity buffer was too small */

/* ---- sample.h drop-in --------------------------------------------------- */

typedef struct quasar_sampler quasar_sampler;

/* Replaces sample.h:14 / sample.c:31-39. Defaults: greedy (temperature 0),
 * top_p 1, top_k 0, min_p 0, repeat_penalty 1, repeat_last_n 0, PRNG state
 * 0x9E3779B97F4A7C15. Device buffers - PRNG word, history ring and the
 * object's own kernel workspace, like the per-object scratch of
 * sample.c:94-104 - are allocated lazily on the current CUDA device and used
 * on the object's own stream, so distinct objects can pick concurrently from
 * different host threads. Returns NULL when the host allocation fails. */
quasar_sampler *quasar_sampler_new(void);

/* Replaces sample.h:15 / sample.c:41-45. NULL-safe. */
void quasar_sampler_free(quasar_sampler *s);

/* Replaces sample.h:19-22 / sample.c:47-68, same clamps: top_p outside (0,1)
 * -> 1, top_k <= 0 -> 0, min_p <= 0 -> 0, repeat_penalty <= 1 -> 1,
 * repeat_last_n <= 0 -> 0; seed 0 -> time-seeded; history cleared. */
void quasar_sampler_config(quasar_sampler *s,
                           float temperature, float top_p, int top_k,
                           float min_p, float repeat_penalty, int repeat_last_n,
                           uint64_t seed);

/* Replaces sample.h:25 / sample.c:70: clears history, keeps the PRNG state. */
void quasar_sampler_reset(quasar_sampler *s);

/* Replaces sample.h:29 / sample.c:111-178. logits[n_vocab] may be a host
 * pointer (copied to the device) or a device pointer (read in place); it is
 * not modified. Records the choice in history. n_vocab <= 0 returns 0, as in
 * the reference. On a CUDA failure returns -1 and quasar_sampler_last_error()
 * gives the status (the reference has no error path here; -1 is never a valid
 * token id). Blocks until the id is on the host. */
int quasar_sampler_pick(quasar_sampler *s, const float *logits, int n_vocab);

/* Extension: status of the last call on s (QUASAR_OK or QUASAR_E*). */
int quasar_sampler_last_error(const quasar_sampler *s);

/* Extension: human-readable name of a status code. */
const char *quasar_status_string(int status);

/* ---- batched sampler ------------------------------------------------------ */

/* Per-row parameters, raw (clamped inside, as quasar_sampler_config does). */
typedef struct {
    float   temperature;
    float   top_p;
    float   min_p;
    float   repeat_penalty;
    int32_t top_k;
    int32_t reserved;        /* set to 0 */
} quasar_sample_params;

/* Optional per-row report. */
typedef struct {
    int32_t n_kept;          /* survivors of top-k/top-p/min-p (0 when greedy) */
    float   p_chosen;        /* normalised probability of the chosen id (greedy: 1) */
    float   inv_sum;         /* (float)(1 / window sum) (greedy: 0) */
    int32_t path;            /* QUASAR_PATH_* that produced the row */
} quasar_pick_diag;

#define QUASAR_PATH_GREEDY     0   /* temperature <= 0: penalized argmax */
#define QUASAR_PATH_CANDIDATE  1   /* candidates collected in one HBM pass, exact cuts */
#define QUASAR_PATH_SELECT     2   /* exact radix select over the row (any params),
                                      in a second kernel */

/* Flags for quasar_sampler_pick_batch. */
#define QUASAR_FLAG_EXACT_SELECT  1  /* route every stochastic row through the
                                        radix-select path (same results; slower) */
#define QUASAR_FLAG_NO_TMA        2  /* stream with 256-bit register loads even
                                        where the bulk-copy ring applies (same
                                        results) */
#define QUASAR_FLAG_NO_SPLIT      4  /* stream every row on one CTA, also for
                                        the small batches that are otherwise
                                        sampled by a cluster of CTAs per row
                                        (same ids within the stochastic
                                        tolerance) */

/* Sample B rows of d_logits (row r at d_logits + r*ld, V columns, fp32).
 *   d_params    [B] per-row parameters on the device, or NULL to use *h_params
 *               for every row (h_params must then be non-NULL).
 *   d_rng       [B] xorshift64* states, advanced in place: one step per
 *               stochastic row, none for a greedy row (sample.c:72-81, 130-134).
 *   d_hist      [B, hist_cap] history rings (sample.c:22-23); row r holds
 *               d_hist_len[r] ids starting at d_hist_head[r]. hist_cap == 0
 *               disables history (d_hist may then be NULL). d_hist_len NULL
 *               means every ring is full; d_hist_head NULL means head 0.
 *   record      nonzero: append each chosen id to its ring the way sample.c:83-92
 *               does (needs d_hist_len and d_hist_head).
 *   d_out       [B] chosen ids.
 *   d_diag      [B] optional report, or NULL.
 * Requirements: 1 <= V <= QUASAR_MAX_VOCAB, ld >= V. When the rows start
 * 16-byte aligned with ld % 4 == 0 and V % 4 == 0, persistent CTAs stream them
 * through a shared-memory ring filled by bulk copies (TMA); otherwise the same
 * persistent CTAs read them with 256-bit (32-byte aligned rows) or scalar
 * loads. A second kernel finishes the stochastic rows. Small batches
 * (B <= 16) with host parameters (d_params NULL) whose rows are greedy or have
 * 1 <= top_k <= 256 take one fused kernel instead (the latency case of one
 * row, as quasar_sampler_pick makes it): a cluster of 8 CTAs per row, each
 * holding V/8 columns in shared memory, exchanging the row's max and sum and
 * its top-k candidates through distributed shared memory; it needs the
 * bulk-copy conditions above, V % 32 == 0 and V >= 8192 (no workspace is
 * used). Finite logits
 * only (as in the reference, NaN/inf give unspecified picks). Asynchronous on
 * `stream`; returns after the launch. Replaces, batched, sample.h:29. */
#define QUASAR_MAX_VOCAB (1 << 20)
int quasar_sampler_pick_batch(const float *d_logits, int64_t ld, int B, int V,
                              const quasar_sample_params *d_params,
                              const quasar_sample_params *h_params,
                              uint64_t *d_rng,
                              int32_t *d_hist, int hist_cap,
                              int32_t *d_hist_len, int32_t *d_hist_head,
                              int record,
                              int32_t *d_out, quasar_pick_diag *d_diag,
                              void *d_workspace, size_t workspace_bytes,
                              int flags, void *stream);

/* Device workspace one quasar_sampler_pick_batch call of B rows with history
 * capacity hist_cap needs: the per-row summaries the streaming kernel leaves
 * for the finishing kernel (row max and 1/sum, per-thread maxima, tile-max
 * table, penalized-id list; ~15 KB per row at hist_cap 256). Pass
 * d_workspace = NULL to use a workspace the library allocates and keeps per
 * (device, stream): calls on different streams never share one, and calls on
 * one stream are ordered by it. It grows with stream-ordered allocations
 * (cudaMallocAsync / cudaFreeAsync on that stream), never a device-wide
 * synchronisation. */
size_t quasar_sampler_workspace_bytes(int B, int hist_cap);

/* CTAs per row (the cluster size) of the fused small-batch kernel that
 * quasar_sampler_pick_batch uses for these arguments (0: the batch takes the
 * streaming and finishing kernels, one CTA per row). Host-side arithmetic
 * only: no GPU call, pointers are not dereferenced. */
int quasar_sampler_split_shards(const float *d_logits, int64_t ld, int B, int V,
                                const quasar_sample_params *d_params,
                                const quasar_sample_params *h_params, int hist_cap, int flags);

/* Kernel launches one quasar_sampler_pick_batch call makes (2: the streaming
 * kernel, which also finishes greedy rows, and the finishing kernel of the
 * stochastic rows: cuts, exact select where needed, draw), plus one 4-byte
 * memset of the workspace abort word. A small batch that takes the fused
 * cluster kernel makes 1 launch and no memset. A row whose id comes
 * back -1 hit the bounded-wait timeout of the bulk-copy ring (a device fault,
 * not a sampling result). */
int quasar_sampler_pick_batch_launches(void);

/* ---- batched sampler without allocation (no counterpart in the reference) -- */

/* Size of the fixed device array that serves as the workspace of
 * quasar_sampler_pick_batch_noalloc (about 2,180 rows at hist_cap 256). */
#define QUASAR_NOALLOC_WORKSPACE_BYTES (32u << 20)

/* quasar_sampler_pick_batch with the same arguments and results, but its
 * workspace is a file-scope device array of QUASAR_NOALLOC_WORKSPACE_BYTES, so
 * the call allocates nothing: for callers that have no device memory to spare
 * at sampling time (engines that reserve free HBM for their KV cache) or must
 * not take the synchronisation an allocation can bring. A call whose
 * quasar_sampler_workspace_bytes(B, hist_cap) exceeds the array returns
 * QUASAR_EOVERFLOW without touching the GPU. The array is shared by all calls
 * on one device in the process: calls that overlap (two streams or threads)
 * race on it and must be serialised by the caller. The first call on each
 * device sets up (array address lookup, kernel attributes); make it before any
 * stream capture. The array's address is looked up once per device and kept,
 * so do not use this entry point across a cudaDeviceReset. Arguments are
 * checked as quasar_sampler_pick_batch checks them, before the size check.
 * Every call clears the one word that must start at zero (the abort flag)
 * with a memset on `stream`. */
int quasar_sampler_pick_batch_noalloc(const float *d_logits, int64_t ld, int B, int V,
                                      const quasar_sample_params *d_params,
                                      const quasar_sample_params *h_params,
                                      uint64_t *d_rng,
                                      int32_t *d_hist, int hist_cap,
                                      int32_t *d_hist_len, int32_t *d_hist_head,
                                      int record,
                                      int32_t *d_out, quasar_pick_diag *d_diag,
                                      int flags, void *stream);

/* ---- vocab-sharded sampling (tensor-parallel LM heads; new, no counterpart
 * in the reference) ----------------------------------------------------------
 * Rank g of G holds global columns [col0, col0 + Vs) of every row; history
 * ids stay global. A batch is sampled in three phases with two all-gathers
 * between them (done by the caller, e.g. NCCL), and every rank ends with the
 * same ids, PRNG states and rings as an unsharded quasar_sampler_pick_batch
 * over the full rows (within the stochastic tolerance of the candidate path):
 *   1. quasar_shard_stats      -> d_stats[B] per rank; all-gather -> [G][B]
 *   2. quasar_shard_candidates -> d_cand[B][k] per rank; all-gather -> [G][B][k]
 *   3. quasar_shard_finish     -> ids, PRNG steps, ring appends (every rank)
 * Stochastic rows need 1 <= top_k <= k <= 256 (the merge is exact because
 * the global top-k lies in the union of the shards' top-k), or min_p > 0
 * with at most k keys per shard at or above the min-p threshold of the
 * global max (every survivor of the floor is sent, so the top-p and min-p
 * cuts over the merged keys are exact); other stochastic rows (top-p alone,
 * pure multinomial), and rows whose candidates a shard cannot bound or send,
 * come back as -1. Greedy rows merge the shards' penalized argmax (lowest
 * global id on ties). */
typedef struct {
    float   max;   /* stochastic row: max scaled logit of the shard;
                      greedy row: its largest penalized logit */
    int32_t best;  /* greedy row: that logit's column in the shard (-1: none) */
    double  sum;   /* stochastic row: sum of exp(sc - max) over the shard */
} quasar_shard_stat;

/* Phase 1. d_workspace (quasar_sampler_workspace_bytes(B, hist_cap) bytes)
 * keeps per-row summaries for phase 2 of the same batch. */
int quasar_shard_stats(const float *d_logits, int64_t ld, int B, int Vs, int64_t col0,
                       const quasar_sample_params *d_params,
                       const quasar_sample_params *h_params,
                       const int32_t *d_hist, int hist_cap,
                       const int32_t *d_hist_len, const int32_t *d_hist_head,
                       quasar_shard_stat *d_stats,
                       void *d_workspace, size_t workspace_bytes, int flags, void *stream);

/* Phase 2, with every rank's stats gathered in rank order (d_all_stats
 * [G][B]) and the workspace of phase 1: this rank's k best candidates per row
 * by (p desc, global id asc), as keys (p bits << 32 | ~global id), 0-padded. */
int quasar_shard_candidates(const float *d_logits, int64_t ld, int B, int Vs, int64_t col0,
                            const quasar_sample_params *d_params,
                            const quasar_sample_params *h_params,
                            const int32_t *d_hist, int hist_cap,
                            const int32_t *d_hist_len, const int32_t *d_hist_head,
                            const quasar_shard_stat *d_all_stats, int G, int rank, int k,
                            uint64_t *d_cand,
                            void *d_workspace, size_t workspace_bytes, int flags, void *stream);

/* Phase 3, with every rank's candidates gathered in rank order (d_all_cand
 * [G][B][k]): merge, cuts and draw (sample.c:151-177), one PRNG step per
 * stochastic row, optional ring append; d_out gets global ids. */
int quasar_shard_finish(const uint64_t *d_all_cand, const quasar_shard_stat *d_all_stats,
                        int G, int k, int B,
                        const quasar_sample_params *d_params,
                        const quasar_sample_params *h_params,
                        uint64_t *d_rng,
                        int32_t *d_hist, int hist_cap,
                        int32_t *d_hist_len, int32_t *d_hist_head,
                        int record,
                        int32_t *d_out, quasar_pick_diag *d_diag, void *stream);

/* ---- vocab-sharded sampling over NCCL (no counterpart in the reference) ----
 * The three phases above with their two exchanges, in one call on the
 * caller's stream, for callers in C. NCCL is loaded at run time: the
 * libnccl.so.2 the process already has, else the file QUASAR_NCCL_LIBRARY
 * names, else libnccl.so.2 from the loader path (QUASAR_ENCCL when none
 * loads). Communicators made by quasar_nccl_init are non-blocking: every
 * NCCL call is followed until it has left the host, under the communicator's
 * time limit; on an error or on expiry the communicator is aborted
 * (ncclCommAbort) and the call returns QUASAR_ENCCL - a rank that never joins
 * or stops answering ends the others' calls instead of hanging them. An
 * aborted communicator stays unusable (every later call: QUASAR_ENCCL). */
#define QUASAR_NCCL_ID_BYTES 128   /* sizeof(ncclUniqueId) */
typedef struct quasar_nccl quasar_nccl;

/* QUASAR_OK when an NCCL library could be loaded, else QUASAR_ENCCL. */
int quasar_nccl_available(void);

/* A new communicator id (rank 0 makes it; every rank passes it to _init). */
int quasar_nccl_unique_id(void *id_out /* QUASAR_NCCL_ID_BYTES */);

/* Rank `rank` of `nranks` joins the communicator of unique_id on the current
 * CUDA device. timeout_ms bounds the join and every later NCCL call of this
 * communicator (0: no limit). */
int quasar_nccl_init(quasar_nccl **comm, int nranks, int rank, const void *unique_id, int timeout_ms);

/* Wraps a communicator the caller made (an ncclComm_t of the same NCCL
 * library, on the current device); quasar_nccl_free does not destroy it. */
int quasar_nccl_wrap(quasar_nccl **comm, void *nccl_comm, int nranks, int rank, int timeout_ms);

/* Aborts the communicator (ncclCommAbort): its operations still queued or
 * running end; it cannot be used again. */
int quasar_nccl_abort(quasar_nccl *comm);

/* Finalizes and destroys a communicator made by quasar_nccl_init (bounded by
 * its time limit), and frees the handle. NULL-safe. */
int quasar_nccl_free(quasar_nccl *comm);

/* Blocks until the work queued on `stream` so far has completed, while
 * watching the communicator: an NCCL error, or timeout_ms (> 0) passing
 * first, aborts it and returns QUASAR_ENCCL (its kernels still waiting for a
 * peer then end). */
int quasar_nccl_wait(quasar_nccl *comm, void *stream, int timeout_ms);

/* Workspace of quasar_shard_pick: the row summaries of
 * quasar_sampler_workspace_bytes(B, hist_cap) plus the gathered stats
 * [G][B] and candidate keys [G][B][k]. */
size_t quasar_shard_workspace_bytes(int B, int hist_cap, int G, int k);

/* Samples B rows split by vocab over the communicator's ranks: this rank
 * holds global columns [col0, col0 + Vs) of each row (d_logits, row stride
 * ld); every rank passes its replica of the per-row parameters, PRNG states
 * and history rings, and every rank ends with the same ids, states and rings
 * (quasar_shard_stats -> all-gather -> quasar_shard_candidates ->
 * all-gather -> quasar_shard_finish, the gathers in place in d_workspace,
 * 256-byte aligned, quasar_shard_workspace_bytes(B, hist_cap, G, k) bytes).
 * Row requirements as for the phases (stochastic rows: 1 <= top_k <= k, or
 * min_p > 0 with at most k survivors of the min-p floor per shard; other rows
 * come back as -1). Asynchronous on `stream`; pair with quasar_nccl_wait to
 * bound the wait for the peers. */
int quasar_shard_pick(quasar_nccl *comm, const float *d_logits, int64_t ld, int B, int Vs, int64_t col0,
                      const quasar_sample_params *d_params,
                      const quasar_sample_params *h_params,
                      uint64_t *d_rng,
                      int32_t *d_hist, int hist_cap,
                      int32_t *d_hist_len, int32_t *d_hist_head,
                      int record,
                      int32_t *d_out, quasar_pick_diag *d_diag,
                      int k, void *d_workspace, size_t workspace_bytes,
                      int flags, void *stream);

/* ---- synthetic inputs (benchmark / test utility, not in the reference) ---- */

#define QUASAR_SYNTH_NORMAL       0  /* Irwin-Hall N(0,1) * scale */
#define QUASAR_SYNTH_GUMBEL_PEAK  1  /* Gumbel(0,1), +8 at one column per row */
#define QUASAR_SYNTH_ZIPF         2  /* -scale * log(rank), rank a row permutation */

/* Fill rows [row0, row0+B) of a deterministic synthetic logits matrix into
 * d_out (row stride ld). Bit-identical to the CPU recipe used by the tests. */
int quasar_synth_logits(int kind, uint64_t seed, int64_t row0, int B, int V,
                        int64_t ld, float scale, float *d_out, void *stream);
/* History ids uniform in [0, V): d_out[B, H]. */
int quasar_synth_hist(uint64_t seed, int64_t row0, int B, int H, int V,
                      int32_t *d_out, void *stream);
/* Per-row uniform values lo + (hi-lo)*u24: d_out[B]. */
int quasar_synth_uniform(uint64_t seed, int64_t row0, int B, float lo, float hi,
                         float *d_out, void *stream);

/* ---- self-test (no reference counterpart) -------------------------------- */

/* Evaluates one of the sampler's exp variants on d_x[n] into d_out[n]:
 * which = 0 ex2.approx with a split argument, 1 CUDA expf, 2 a correctly
 * rounded (float)exp((double)x), 3 an FMA-pipe polynomial exp, 4 the MUFU
 * exp (ex2.approx of x*log2e) the window sum uses by default.
 * Used by the GPU tests to bound the sum term's error and bias. */
int quasar_selftest_exp(const float *d_x, float *d_out, int n, int which, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* QUASAR_SAMPLER_H */
