/* batched_decode.c - a batched decode loop in C over libquasar_cuda.
 *
 * The reference server generates one sequence at a time: run_generation
 * (franzvill/quasar server.c:225-309) runs the forward pass, calls
 * quasar_sampler_pick on the host logits row (server.c:259), decodes the
 * token and checks stop conditions, token after token. This program is the
 * batched form of that loop: B sequences, each with its own sampling
 * parameters, seed and repeat-penalty ring (server.c:313-322 configures them
 * per request), whose sampler state stays on the device; every step is one
 * quasar_sampler_pick_batch call over all B rows, and only the B chosen ids
 * come back to the host, where stop tokens end sequences (as the server's
 * stop checks would; stop strings and streaming stay host-side).
 *
 * The forward pass is out of scope: step t's logits come from the library's
 * deterministic synthetic generator (quasar_synth_logits, seed base + t),
 * which the tests regenerate on the CPU to drive one reference sampler
 * object per sequence over the same rows.
 *
 *   batched_decode --rows B --steps N [--vocab V] [--seed S] [--hist H]
 *                  [--stop ID] --out FILE
 *
 * Row r's parameters (the test restates these formulas):
 *   temperature 0 when r % 5 == 0, else 0.6 + 0.1 * (r % 7)
 *   top_k 40 when r % 3 == 1, else 0;  top_p 0.9;  min_p 0.05 when r is odd
 *   repeat_penalty 1.1 over the last H ids;  seed 1000 + r
 * FILE gets B int32 sequence lengths, then B x N int32 ids (row-major; ids
 * past a sequence's length are -1). Exit status 0 on success. */
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "quasar_sampler.h"

#define CHECK_CUDA(x)                                                                   \
    do {                                                                                \
        cudaError_t e_ = (x);                                                           \
        if (e_ != cudaSuccess) {                                                        \
            fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_)); \
            return 2;                                                                   \
        }                                                                               \
    } while (0)

static void row_params(int r, quasar_sample_params *p) {
    p->temperature = (r % 5 == 0) ? 0.0f : 0.6f + 0.1f * (float)(r % 7);
    p->top_p = 0.9f;
    p->min_p = (r % 2) ? 0.05f : 0.0f;
    p->repeat_penalty = 1.1f;
    p->top_k = (r % 3 == 1) ? 40 : 0;
    p->reserved = 0;
}

int main(int argc, char **argv) {
    int B = 64, N = 32, V = 151936, H = 64;
    long long stop = -1;
    uint64_t seed = 7;
    const char *out_path = NULL;
    for (int i = 1; i + 1 < argc; i += 2) {
        if (!strcmp(argv[i], "--rows")) B = atoi(argv[i + 1]);
        else if (!strcmp(argv[i], "--steps")) N = atoi(argv[i + 1]);
        else if (!strcmp(argv[i], "--vocab")) V = atoi(argv[i + 1]);
        else if (!strcmp(argv[i], "--hist")) H = atoi(argv[i + 1]);
        else if (!strcmp(argv[i], "--seed")) seed = strtoull(argv[i + 1], NULL, 10);
        else if (!strcmp(argv[i], "--stop")) stop = atoll(argv[i + 1]);
        else if (!strcmp(argv[i], "--out")) out_path = argv[i + 1];
        else {
            fprintf(stderr, "unknown argument %s\n", argv[i]);
            return 1;
        }
    }
    if (!out_path || B < 1 || N < 1 || V < 1 || H < 1) {
        fprintf(stderr, "usage: %s --rows B --steps N [--vocab V] [--seed S] [--hist H] [--stop ID] --out FILE\n",
                argv[0]);
        return 1;
    }

    /* per-sequence state on the device: params, PRNG words, history rings */
    quasar_sample_params *h_params = (quasar_sample_params *)calloc((size_t)B, sizeof *h_params);
    uint64_t *h_rng = (uint64_t *)calloc((size_t)B, sizeof *h_rng);
    int32_t *ids = (int32_t *)malloc((size_t)B * N * sizeof *ids);
    int32_t *len = (int32_t *)calloc((size_t)B, sizeof *len);
    char *done = (char *)calloc((size_t)B, 1);
    if (!h_params || !h_rng || !ids || !len || !done) return 2;
    for (int r = 0; r < B; r++) {
        row_params(r, &h_params[r]);
        h_rng[r] = 1000u + (uint64_t)r;  /* the seed, as quasar_sampler_config takes it */
    }
    for (size_t i = 0; i < (size_t)B * N; i++) ids[i] = -1;

    cudaStream_t st;
    CHECK_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    float *d_logits;
    quasar_sample_params *d_params;
    uint64_t *d_rng;
    int32_t *d_hist, *d_len, *d_head, *d_out, *h_out;
    CHECK_CUDA(cudaMalloc((void **)&d_logits, (size_t)B * V * sizeof(float)));
    CHECK_CUDA(cudaMalloc((void **)&d_params, (size_t)B * sizeof *d_params));
    CHECK_CUDA(cudaMalloc((void **)&d_rng, (size_t)B * sizeof *d_rng));
    CHECK_CUDA(cudaMalloc((void **)&d_hist, (size_t)B * H * sizeof(int32_t)));
    CHECK_CUDA(cudaMalloc((void **)&d_len, (size_t)B * sizeof(int32_t)));
    CHECK_CUDA(cudaMalloc((void **)&d_head, (size_t)B * sizeof(int32_t)));
    CHECK_CUDA(cudaMalloc((void **)&d_out, (size_t)B * sizeof(int32_t)));
    CHECK_CUDA(cudaMallocHost((void **)&h_out, (size_t)B * sizeof(int32_t)));
    const size_t ws_bytes = quasar_sampler_workspace_bytes(B, H);
    void *d_ws;
    CHECK_CUDA(cudaMalloc(&d_ws, ws_bytes));
    CHECK_CUDA(cudaMemcpyAsync(d_params, h_params, (size_t)B * sizeof *d_params, cudaMemcpyHostToDevice, st));
    CHECK_CUDA(cudaMemcpyAsync(d_rng, h_rng, (size_t)B * sizeof *d_rng, cudaMemcpyHostToDevice, st));
    /* empty rings (a fresh request: quasar_sampler_config clears history) */
    CHECK_CUDA(cudaMemsetAsync(d_hist, 0, (size_t)B * H * sizeof(int32_t), st));
    CHECK_CUDA(cudaMemsetAsync(d_len, 0, (size_t)B * sizeof(int32_t), st));
    CHECK_CUDA(cudaMemsetAsync(d_head, 0, (size_t)B * sizeof(int32_t), st));

    int live = B;
    for (int t = 0; t < N && live > 0; t++) {
        /* the "forward pass": step t's logits for every sequence */
        int rc = quasar_synth_logits(QUASAR_SYNTH_NORMAL, seed + (uint64_t)t, 0, B, V, V, 3.0f, d_logits, st);
        if (rc == QUASAR_OK)
            rc = quasar_sampler_pick_batch(d_logits, V, B, V, d_params, NULL, d_rng, d_hist, H, d_len, d_head, 1,
                                           d_out, NULL, d_ws, ws_bytes, 0, st);
        if (rc != QUASAR_OK) {
            fprintf(stderr, "step %d: %s\n", t, quasar_status_string(rc));
            return 3;
        }
        CHECK_CUDA(cudaMemcpyAsync(h_out, d_out, (size_t)B * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
        CHECK_CUDA(cudaStreamSynchronize(st));
        /* host side of the step: append, stop tokens end sequences (a
           finished row is still sampled with the batch; its ids are dropped) */
        for (int r = 0; r < B; r++) {
            if (done[r]) continue;
            if (h_out[r] < 0) {
                fprintf(stderr, "row %d step %d: sampler failure\n", r, t);
                return 3;
            }
            ids[(size_t)r * N + t] = h_out[r];
            len[r] = t + 1;
            if (stop >= 0 && h_out[r] == stop) {
                done[r] = 1;
                live--;
            }
        }
    }
    FILE *f = fopen(out_path, "wb");
    if (!f) return 4;
    if (fwrite(len, sizeof(int32_t), (size_t)B, f) != (size_t)B ||
        fwrite(ids, sizeof(int32_t), (size_t)B * N, f) != (size_t)B * N) {
        fclose(f);
        return 4;
    }
    fclose(f);
    printf("batched_decode: %d sequences x %d steps, %d still running\n", B, N, live);
    cudaFree(d_logits);
    cudaFree(d_params);
    cudaFree(d_rng);
    cudaFree(d_hist);
    cudaFree(d_len);
    cudaFree(d_head);
    cudaFree(d_out);
    cudaFree(d_ws);
    cudaFreeHost(h_out);
    cudaStreamDestroy(st);
    free(h_params);
    free(h_rng);
    free(ids);
    free(len);
    free(done);
    return 0;
}
