// small_batch.cu - one fused kernel for small batches: every row is sampled
// by a thread-block cluster of G CTAs on one GPU.
//
// With B rows the streaming kernel runs B CTAs, so a batch of a few rows
// keeps a few of the 148 SMs busy and one row's latency is one SM's
// bandwidth over 608 KB (sample.c:111-178 on a single row is the reference
// server's latency case). Here CTA g of row b's cluster copies columns
// [g*V/G, (g+1)*V/G) of the row into its shared memory with bulk copies (no
// multicast), penalizes and scales them there (sample.c:118-142), and
// reduces its max, its sum of exp against that max and its penalized argmax;
// the cluster exchanges these through distributed shared memory, so every
// CTA knows the row's max M and 1/sum. Each CTA then selects its shard's
// top-k keys (p desc, id asc; sample.c:151-154) from the values in shared
// memory and writes them into CTA 0's shared memory, which merges the G
// sorted lists and applies the top-k, top-p and min-p cuts and the draw
// (sample.c:154-177) with the row's PRNG state, then appends to the ring
// (sample.c:83-92). One launch, no workspace, no second pass over HBM.
//
// Rows handled: greedy, and stochastic rows with 1 <= top_k <= 256 (every
// kept element is among some shard's top_k). The host sends other rows to
// the streaming/finishing kernels (sample_rows.cu).
#include <cooperative_groups.h>
#include <float.h>
#include <math.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "ptx.cuh"
#include "sample_rows.cuh"

namespace cg = cooperative_groups;

namespace qs {
namespace small {

constexpr int T = 256;        // threads per CTA
constexpr int NW = T / 32;
constexpr int KMAX = 256;     // top_k at most: the keys a CTA sends
constexpr int LCAP = 1024;    // a CTA's listed candidates at most (more: the exact select)

struct Stat {
    double S;      // sum of exp(v - m) over the shard
    float m;       // shard max of the scaled, penalized values
    float best_v;  // greedy: largest penalized logit
    int best_i;    // ... its lowest global column (INT_MAX: none)
    int abort;     // the bulk copy did not land in time
};

struct Smem {
    Stat st;            // this CTA's shard statistics (read by the cluster)
    uint64_t bar;       // mbarrier of the bulk copy
    double rd[NW];
    float rf[NW];
    int ri[NW];
    float M, inv;       // the row's max and 1/sum
    int nk;             // real keys in the merged lists (CTA 0)
    int nlist;          // candidates listed by this CTA
    int abort;
    uint32_t hist[256]; // radix-select bins
    uint32_t pick_bin, pick_above;
    float wk[NW];       // each warp's ceil(k/8)-th largest thread max
    uint64_t rng;       // the row's PRNG word (CTA 0)
};

// Dynamic shared memory: [shard values, Vs floats][penalty bits][merge keys,
// G*KMAX (CTA 0)][listed candidates, LCAP].
__host__ __device__ inline size_t off_bits(int Vs) { return ((size_t)Vs * 4 + 15) & ~(size_t)15; }
__host__ __device__ inline size_t off_keys(int Vs) {
    return (off_bits(Vs) + (((size_t)Vs + 31) / 32) * 4 + 15) & ~(size_t)15;
}
__host__ __device__ inline size_t off_list(int Vs, int G) { return off_keys(Vs) + (size_t)G * KMAX * 8; }
__host__ __device__ inline size_t smem_bytes(int Vs, int G) { return off_list(Vs, G) + (size_t)LCAP * 8; }

__device__ __forceinline__ void bsync() { __syncthreads(); }

// Block-wide radix select: the need-th largest key (1-based) among the keys
// key_of(e) that `take` admits, e over [0, n), `passes` digits of 8 bits from
// the top of a `bits`-bit key. Returns the key; *total gets the number of
// admitted keys (the select is skipped, and 0 returned, when total <= need).
template <typename K, typename Take, typename KeyOf>
__device__ K cta_select(int n, int bits, int need, Take take, KeyOf key_of, Smem& s, int* total) {
    const int tid = threadIdx.x, lane = tid & 31;
    K prefix = 0;
    for (int shift = bits - 8; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += T) s.hist[i] = 0u;
        bsync();
        const K hi = shift + 8 >= bits ? (K)0 : (K)(~(K)0) << (shift + 8);
        for (int e = tid; e < n; e += T) {
            if (!take(e)) continue;
            const K key = key_of(e);
            if ((key & hi) == prefix) atomicAdd(&s.hist[(uint32_t)(key >> shift) & 255u], 1u);
        }
        bsync();
        if (tid < 32) {
            // bins in descending order, eight per lane
            uint32_t c[8], t = 0u;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                c[j] = s.hist[255 - 8 * lane - j];
                t += c[j];
            }
            const uint32_t incl = warp_incl_scan(t, lane), excl = incl - t;
            if (shift + 8 >= bits && lane == 31) *total = (int)incl;
            const uint32_t want = (uint32_t)need;
            if (excl < want && incl >= want) {
                uint32_t acc = excl;
                for (int j = 0; j < 8; j++) {
                    if (acc + c[j] >= want) {
                        s.pick_bin = 255u - 8u * lane - j;
                        s.pick_above = acc;
                        break;
                    }
                    acc += c[j];
                }
            }
        }
        bsync();
        if (shift + 8 >= bits && *total <= need) return (K)0;
        prefix |= (K)s.pick_bin << shift;
        need -= (int)s.pick_above;
        bsync();
    }
    return prefix;
}

__global__ void __launch_bounds__(T) sample_rows_small(RowsArgs a, int G) {
    extern __shared__ __align__(128) unsigned char dyn[];
    __shared__ Smem s;
    __shared__ int total_s;
    cg::cluster_group cl = cg::this_cluster();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = (int)cl.block_rank();
    const int b = blockIdx.x / G;
    const int Vs = a.V / G;
    const int64_t col0 = (int64_t)g * Vs;
    float* data = reinterpret_cast<float*>(dyn);
    uint32_t* bits = reinterpret_cast<uint32_t*>(dyn + off_bits(Vs));
    uint64_t* keys = reinterpret_cast<uint64_t*>(dyn + off_keys(Vs));
    uint64_t* list = reinterpret_cast<uint64_t*>(dyn + off_list(Vs, G));
    const uint32_t bar = smem_u32(&s.bar);

    // ---- the shard into shared memory; meanwhile parameters and penalty bits ----
    if (tid == 0) {
        mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const uint32_t bytes = (uint32_t)Vs * 4u;
        mbar_arrive_tx(bar, bytes);
        const char* src = reinterpret_cast<const char*>(a.logits + (int64_t)b * a.ld + col0);
        for (uint32_t off = 0; off < bytes; off += 16384u)
            bulk_g2s(smem_u32(data) + off, src + off, min(16384u, bytes - off), bar);
        s.nlist = 0;
        s.abort = 0;
    }
    const int nwords = (Vs + 31) / 32;
    for (int i = tid; i < nwords; i += T) bits[i] = 0u;
    const quasar_sample_params pr = a.d_params ? a.d_params[b] : a.h_params;
    const RowParams P = clamp_params(pr);
    const bool greedy = !(P.T > 0.0f);
    const int cap = a.hist ? a.hist_cap : 0;
    int len = 0, head = 0;
    if (cap > 0) {
        len = a.hist_len ? min(max(a.hist_len[b], 0), cap) : cap;
        head = a.hist_head ? ((a.hist_head[b] % cap) + cap) % cap : 0;
    }
    const int32_t* ring = cap > 0 ? a.hist + (int64_t)b * cap : nullptr;
    const bool use_pen = P.rp > 1.0f && len > 0;
    const uint64_t rng0 = (g == 0 && !greedy && tid == 0) ? a.rng[b] : 0ull;  // read early: CTA 0 draws
    bsync();  // bits cleared
    if (use_pen)
        for (int i = tid; i < len; i += T) {  // the ring's len entries from head (sample.c:118-128)
            const int64_t id = (int64_t)ring[(head + i) % cap] - col0;
            if (id >= 0 && id < Vs) atomicOr(&bits[(int)id >> 5], 1u << ((int)id & 31));
        }
    const bool landed = mbar_wait(bar, 0);
    if (!landed) s.abort = 1;  // (benign race: every writer stores 1)
    bsync();

    // ---- penalize and scale in place; shard max (or penalized argmax) ----
    const float inv_t = greedy ? 0.0f : __fdiv_rn(1.0f, P.T);  // sample.c:137
    // four consecutive columns per thread and step (16-byte shared loads)
    const int Vs4 = Vs >> 2;
    float4* d4 = reinterpret_cast<float4*>(data);
    float m = -INFINITY;
    int mi = 0x7FFFFFFF;
#pragma unroll 2
    for (int q = tid; q < Vs4; q += T) {
        const float4 v4 = d4[q];
        float x[4] = {v4.x, v4.y, v4.z, v4.w};
        const int e0 = 4 * q;
        if (use_pen) {
            const uint32_t pb = (bits[e0 >> 5] >> (e0 & 31)) & 15u;  // e0 % 4 == 0: one word
            if (pb)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if ((pb >> j) & 1u) x[j] = penalize(x[j], P.rp);  // sample.c:124
        }
        if (greedy) {
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (x[j] > m) {  // strictly larger: each thread sees ascending columns
                    m = x[j];
                    mi = e0 + j;
                }
        } else {
#pragma unroll
            for (int j = 0; j < 4; j++) {
                x[j] = __fmul_rn(x[j], inv_t);  // sample.c:142
                m = fmaxf(m, x[j]);
            }
            d4[q] = make_float4(x[0], x[1], x[2], x[3]);
        }
    }
    const int k = greedy ? 1 : min(max(P.top_k, 1), KMAX);
    if (!greedy) {
        // A bound for the shard's top k: each warp sorts its 32 thread maxima
        // (a shuffle bitonic network, descending) and keeps its c-th largest,
        // c = ceil(k/8); the smallest of the 8 has at least 8c >= k thread
        // maxima - k distinct elements - at or above it, so it is at most the
        // shard's k-th largest value.
        float v = m;
#pragma unroll
        for (int size = 2; size <= 32; size <<= 1)
#pragma unroll
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                const float o = __shfl_xor_sync(FULL, v, stride);
                const bool desc = (lane & size) == 0;  // this segment's direction
                v = (((lane & stride) == 0) == desc) ? fmaxf(v, o) : fminf(v, o);
            }
        const float vc = __shfl_sync(FULL, v, (k + NW - 1) / NW - 1);
        if (lane == 0) s.wk[warp] = vc;
    }
    // block max (greedy: value desc, column asc)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(FULL, m, o);
        const int oi = __shfl_xor_sync(FULL, mi, o);
        if (ov > m || (ov == m && oi < mi)) {
            m = ov;
            mi = oi;
        }
    }
    if (lane == 0) {
        s.rf[warp] = m;
        s.ri[warp] = mi;
    }
    bsync();
    m = s.rf[0];
    mi = s.ri[0];
    for (int w = 1; w < NW; w++)
        if (s.rf[w] > m || (s.rf[w] == m && s.ri[w] < mi)) {
            m = s.rf[w];
            mi = s.ri[w];
        }
    double S = 0.0;
    if (!greedy && m > -INFINITY) {
        // sum of exp(v - m), fp32 over 16 terms at a time, double across
        float part = 0.0f;
        int n4 = 0;
#pragma unroll 2
        for (int q = tid; q < Vs4; q += T) {
            const float4 v4 = d4[q];
            part += (exp_fast(__fsub_rn(v4.x, m)) + exp_fast(__fsub_rn(v4.y, m))) +
                    (exp_fast(__fsub_rn(v4.z, m)) + exp_fast(__fsub_rn(v4.w, m)));
            if (++n4 == 4) {
                S += (double)part;
                part = 0.0f;
                n4 = 0;
            }
        }
        S += (double)part;
    }
    S = warp_sum(S);
    bsync();  // s.rf / s.ri reads done
    if (lane == 0) s.rd[warp] = S;
    bsync();
    if (tid == 0) {
        double St = 0.0;
        for (int w = 0; w < NW; w++) St += s.rd[w];
        s.st.S = St;
        s.st.m = m;
        s.st.best_v = m;
        s.st.best_i = mi == 0x7FFFFFFF ? 0x7FFFFFFF : (int)col0 + mi;
        s.st.abort = s.abort;
    }
    cl.sync();  // #1: every shard's statistics are published

    // ---- the row's max, 1/sum and penalized argmax, the same bits in every CTA ----
    if (warp == 0) {
        Stat st;
        st.S = 0.0;
        st.m = -INFINITY;
        st.best_v = -INFINITY;
        st.best_i = 0x7FFFFFFF;
        st.abort = 0;
        if (lane < G) st = *cl.map_shared_rank(&s.st, lane);
        const float M = warp_max(st.m);
        double Sg = st.m > -INFINITY ? st.S * exp((double)st.m - (double)M) : 0.0;
        Sg = warp_sum(Sg);
        float bv = st.best_v;
        int bi = st.best_i;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(FULL, bv, o);
            const int oi = __shfl_xor_sync(FULL, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        const int ab = __any_sync(FULL, st.abort != 0);
        if (lane == 0) {
            s.M = M;
            s.inv = __double2float_rn(1.0 / Sg);
            s.abort = ab;
            s.ri[0] = bi;
        }
    }
    bsync();
    const float M = s.M, inv = s.inv;
    const bool abort = s.abort != 0 || (!greedy && !(P.top_k >= 1 && P.top_k <= KMAX));
    uint64_t st_rng = 0ull;

    if (!greedy) {
        // ---- this shard's top k keys, ranked, into CTA 0's merge buffer ----
        const float thr = __fsub_rn(M, 30.0f);
        float lo0 = thr;
        if (P.min_p > 0.0f) lo0 = fmaxf(lo0, __fadd_rn(M, logf(fminf(P.min_p, 1.0f)) - 0.01f));
        // Only elements at or above the warps' bound (s.wk) are listed, less a
        // tie margin that keeps every element whose p could equal the k-th
        // one's; as raw (value, column) entries, their keys computed below.
        float fk = s.wk[0];
#pragma unroll
        for (int w = 1; w < NW; w++) fk = fminf(fk, s.wk[w]);
        const float lo = fk > -INFINITY ? fmaxf(lo0, fk - (1e-5f + 1e-5f * fabsf(fk))) : lo0;
#pragma unroll 2
        for (int q = tid; q < Vs4; q += T) {
            const float4 v4 = d4[q];
            const float x[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (x[j] >= lo) {
                    const int pos = atomicAdd(&s.nlist, 1);
                    if (pos < LCAP) list[pos] = ((uint64_t)__float_as_uint(x[j]) << 32) | (uint32_t)(4 * q + j);
                }
        }
        bsync();
        int nl = s.nlist;
        if (nl <= LCAP) {
            // the listed entries' keys (p desc, global id asc), one per thread
            for (int i = tid; i < nl; i += T) {
                const uint64_t en = list[i];
                list[i] = ((uint64_t)p_key(__uint_as_float((uint32_t)(en >> 32)), M, thr, inv) << 32) |
                          (uint32_t)(~(uint32_t)(col0 + (uint32_t)en));
            }
            bsync();
        }
        if (nl > LCAP) {
            // more elements tie at the k-th value than the list holds: the
            // exact k-th key (p desc, id asc) over them, then exactly k keys
            auto at_lo = [&](int e) { return data[e] >= lo; };
            auto pkey = [&](int e) {
                return ((uint64_t)p_key(data[e], M, thr, inv) << 32) | (uint32_t)(~(uint32_t)(col0 + e));
            };
            const uint64_t kk = cta_select<uint64_t>(Vs, 64, k, at_lo, pkey, s, &total_s);
            if (tid == 0) s.nlist = 0;
            bsync();
            for (int e = tid; e < Vs; e += T) {
                if (data[e] < lo) continue;
                const uint64_t key = pkey(e);
                if (key >= kk) {
                    const int pos = atomicAdd(&s.nlist, 1);
                    if (pos < LCAP) list[pos] = key;
                }
            }
            bsync();
            nl = min(s.nlist, k);
        }
        // each listed key's rank (keys are distinct), the first k to CTA 0
        uint64_t* dst = cl.map_shared_rank(keys, 0) + (size_t)g * k;
        for (int i = tid; i < nl; i += T) {
            const uint64_t key = list[i];
            int rank = 0;
            for (int j = 0; j < nl; j++) rank += list[j] > key ? 1 : 0;
            if (rank < k) dst[rank] = key;
        }
        for (int i = nl + tid; i < k; i += T) dst[i] = 0ull;
    }
    cl.sync();  // #2: every shard's keys are in CTA 0 (no remote access after this)
    if (g != 0) return;

    int chosen = 0, nkept = 0;
    float pch = 1.0f;
    if (greedy) {
        // the largest penalized logit over the shards, lowest id on ties;
        // an all -inf row gives id 0 (sample.c:130-134)
        chosen = s.ri[0] == 0x7FFFFFFF ? 0 : s.ri[0];
    } else {
        if (tid == 0) s.rng = rng0;
        bsync();
        st_rng = s.rng;
        const double u = rng_unit(&st_rng);  // sample.c:173: one step per stochastic row
        // the merged order: each key's place in its own list plus, per other
        // list, the keys greater than it (binary searches)
        const int n = G * k;
        int cnt = 0;
        for (int i = tid; i < n; i += T) cnt += (keys[i] >> 32) != 0ull ? 1 : 0;
        cnt = warp_sum(cnt);
        if (lane == 0) s.ri[warp] = cnt;
        bsync();
        int nk = 0;
        for (int w = 0; w < NW; w++) nk += s.ri[w];
        const int L = (P.top_k > 0 && P.top_k < nk) ? P.top_k : nk;
        uint64_t* sorted = list;  // the merged prefix, L <= KMAX keys
        for (int i = tid; i < n; i += T) {
            const uint64_t key = keys[i];
            if ((key >> 32) == 0ull) continue;
            int rank = 0;
            if (n <= 512) {
                // every key against every key, all threads reading the same one
                for (int j = 0; j < n; j++) rank += keys[j] > key ? 1 : 0;
            } else {
                const int gi = i / k;
                rank = i - gi * k;  // its place in its own list, plus per other list
                for (int h = 0; h < G; h++) {
                    if (h == gi) continue;
                    const uint64_t* lst = keys + h * k;
                    int l0 = 0, l1 = k;  // first position whose key is not greater
                    while (l0 < l1) {
                        const int mid = (l0 + l1) >> 1;
                        if (lst[mid] > key) l0 = mid + 1;
                        else l1 = mid;
                    }
                    rank += l0;
                }
            }
            if (rank < L) sorted[rank] = key;
        }
        bsync();
        // cuts and draw over the merged prefix (one warp): top-k (sample.c:154),
        // top-p (sample.c:156-160), min-p (sample.c:162-167), inverse CDF
        // (sample.c:171-177); cumulative sums per lane in double, joined by a
        // warp scan
        if (warp == 0 && nk > 0 && !abort) {
            const int BEYOND = 0x7FFFFFFF;
            auto pval = [&](int i) { return __uint_as_float((uint32_t)(sorted[i] >> 32)); };
            const int SEG = (L + 31) / 32;
            const int i0 = min(lane * SEG, L), i1 = min(i0 + SEG, L);
            double seg = 0.0;
            for (int i = i0; i < i1; i++) seg += (double)pval(i);
            const double incl = warp_incl_scan(seg, lane), excl = incl - seg;
            const int nc1 = (P.top_k > 0 && P.top_k < nk) ? P.top_k : BEYOND;
            const int lim = min(nc1, nk);
            const float floor_p = P.min_p > 0.0f ? __fmul_rn(P.min_p, inv) : 0.0f;
            int cut_p = BEYOND, cut_m = L;
            double cum = excl;
            for (int i = i0; i < i1; i++) {
                cum += (double)pval(i);
                if (P.top_p < 1.0f && i < lim && cut_p == BEYOND && cum >= (double)P.top_p) cut_p = i + 1;
                if (i >= 1 && cut_m == L && pval(i) < floor_p) cut_m = i;
            }
            cut_p = __reduce_min_sync(FULL, cut_p);
            cut_m = __reduce_min_sync(FULL, cut_m);
            const int nc2 = cut_p != BEYOND ? cut_p : nc1;
            const int nc = max(1, min(nc2, cut_m));
            double rs = 0.0;
            if (nc - 1 >= i0 && nc - 1 < i1) {
                rs = excl;
                for (int i = i0; i < nc; i++) rs += (double)pval(i);
            }
            const int owner = max(__ffs(__ballot_sync(FULL, nc - 1 >= i0 && nc - 1 < i1)) - 1, 0);
            const double r = u * __shfl_sync(FULL, rs, owner);
            int cut_d = BEYOND;
            cum = excl;
            for (int i = i0; i < min(i1, nc); i++) {
                cum += (double)pval(i);
                if (cum >= r) {
                    cut_d = i;
                    break;
                }
            }
            cut_d = __reduce_min_sync(FULL, cut_d);
            const int c = cut_d != BEYOND ? cut_d : nc - 1;
            if (lane == 0) {
                s.ri[0] = (int)(~(uint32_t)sorted[c]);
                s.ri[1] = nc;
                s.rf[0] = pval(c);
            }
        }
        bsync();
        if (nk > 0 && !abort) {
            chosen = s.ri[0];
            nkept = s.ri[1];
            pch = s.rf[0];
        } else {
            chosen = -1;
            pch = 0.0f;
        }
    }
    if (tid == 0) {
        if (abort) chosen = -1;
        if (!greedy) a.rng[b] = st_rng;
        a.out[b] = chosen;
        if (a.diag) {
            quasar_pick_diag d;
            d.n_kept = nkept;
            d.p_chosen = pch;
            d.inv_sum = greedy ? 0.0f : inv;
            d.path = greedy ? QUASAR_PATH_GREEDY : QUASAR_PATH_CANDIDATE;
            a.diag[b] = d;
        }
        if (a.record && cap > 0 && a.hist_len && a.hist_head && chosen >= 0) {
            int32_t* wring = a.hist + (int64_t)b * cap;
            if (len < cap) {  // sample.c:85-87
                wring[(head + len) % cap] = chosen;
                a.hist_len[b] = len + 1;
            } else {          // sample.c:88-90
                wring[head] = chosen;
                a.hist_head[b] = (head + 1) % cap;
            }
        }
    }
}

}  // namespace small

namespace {
std::mutex g_small_mu;
std::atomic<size_t> g_small_smem[64];
}  // namespace

#ifndef QS_CLUSTER_G
#define QS_CLUSTER_G 8  // CTAs per row (a portable cluster size)
#endif

int small_batch_shards(const RowsArgs& a) {
    if (a.B < 1 || a.B > SPLIT_MAX_B || a.d_params || !a.tma) return 0;
    if (a.flags & (QUASAR_FLAG_EXACT_SELECT | QUASAR_FLAG_NO_SPLIT)) return 0;
    const quasar_sample_params& p = a.h_params;
    if (p.temperature > 0.0f && !(p.top_k >= 1 && p.top_k <= small::KMAX)) return 0;
    const int G = QS_CLUSTER_G;
    if (a.V % G != 0 || (a.V / G) % 4 != 0 || a.V / G < 1024) return 0;
    if (small::smem_bytes(a.V / G, G) > (size_t)200 * 1024) return 0;
    return G;
}

cudaError_t launch_small_batch(const RowsArgs& a, int G, cudaStream_t stream) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const size_t smem = small::smem_bytes(a.V / G, G);
    if (g_small_smem[dev].load(std::memory_order_acquire) < smem) {
        std::lock_guard<std::mutex> lock(g_small_mu);
        if (g_small_smem[dev].load() < smem) {
            err = cudaFuncSetAttribute((const void*)small::sample_rows_small,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (err != cudaSuccess) return err;
            g_small_smem[dev].store(smem, std::memory_order_release);
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(a.B * G));
    cfg.blockDim = dim3(small::T);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)G;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    err = cudaLaunchKernelEx(&cfg, small::sample_rows_small, a, G);
    if (err != cudaSuccess) return err;
    return cudaGetLastError();
}

}  // namespace qs
