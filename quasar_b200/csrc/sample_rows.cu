// sample_rows.cu - batched token sampler for sm_100a: one CTA per logits row.
//
// Replaces franzvill/quasar sample.c:111-178 (quasar_sampler_pick), batched.
// Per row, in sample.c's order:
//   1. history ring -> shared-memory bitset of penalized ids (sample.c:120)
//   2. ONE streaming pass over the row in HBM (128-bit loads): penalty
//      (sample.c:124), temperature scale (sample.c:137,142), running max, online
//      window sum of exp(sc - running max) in double (sample.c:147), and - when
//      min_p > 0 - collection of every element that can survive the min-p cut
//      into a shared-memory candidate list.
//   3. candidate path: exact p = (float)exp(sc - max) * (float)(1/sum) for the
//      candidates, bitonic sort by (p desc, id asc) (= glibc's stable qsort of
//      sample.c:151), top-k / top-p / min-p cuts and the inverse-CDF draw with
//      the row's xorshift64* state (sample.c:153-177).
//   4. select path (any parameters, or when the candidate list overflows):
//      exact radix select over the p keys of the whole row, re-reading it.
// Greedy rows (temperature <= 0) take one pass: penalized argmax, first index
// on ties, no PRNG step (sample.c:130-134).
#include <math.h>

#include "common.cuh"
#include "sample_rows.cuh"

namespace qs {
namespace rows {

constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;
constexpr int UNROLL = 4;                  // float4 loads in flight per thread per tile
constexpr int TILE_Q = THREADS * UNROLL;   // float4 groups per tile
constexpr int CAP = 4096;                  // candidate list capacity (entries)
constexpr int NB = 1024;                   // radix bins per level (10 bits)

// The select path reuses the candidate list storage as histograms.
struct Hist {
    uint32_t cnt1[NB];
    unsigned long long mass1[NB];
    uint32_t cnt2[NB];
    unsigned long long mass2[NB];
    int32_t minid2[NB];
};
static_assert(sizeof(Hist) <= CAP * sizeof(uint64_t), "histograms fit the candidate list");

struct Shared {
    unsigned int maxkey;  // ord_key of the largest scaled logit published so far
    int cnt;              // candidates appended
    float rf[WARPS];
    double rd[WARPS];
    int ri[WARPS];
    unsigned long long ru[WARPS];
    // broadcast slots
    int bin_found, bin;
    unsigned long long bin_mass_above;
    unsigned int bin_cnt_above;
    float pf_lo, pf_hi;
    int res_id, res_nc, res_pos;
    float res_p;
};

// Mass fixed point: p * 2^62 truncated (p <= 1, row sums stay below 2^64).
__device__ __forceinline__ unsigned long long fixp(uint32_t pkey) {
    return __float2ull_rz(__fmul_rn(__uint_as_float(pkey), 4611686018427387904.0f));
}

__device__ __forceinline__ float4 load4(const float* row, int q, int V, bool vec) {
    const int e = q * 4;
    if (vec && e + 3 < V) return __ldcs(reinterpret_cast<const float4*>(row) + q);
    float4 v;
    v.x = (e + 0 < V) ? __ldcs(row + e + 0) : -INFINITY;
    v.y = (e + 1 < V) ? __ldcs(row + e + 1) : -INFINITY;
    v.z = (e + 2 < V) ? __ldcs(row + e + 2) : -INFINITY;
    v.w = (e + 3 < V) ? __ldcs(row + e + 3) : -INFINITY;
    return v;
}

__device__ __forceinline__ void apply_pen(float4& v, const uint32_t* bits, int q, float rp) {
    const uint32_t nib = (bits[q >> 3] >> ((q & 7) << 2)) & 0xFu;
    if (nib) {
        if (nib & 1u) v.x = penalize(v.x, rp);
        if (nib & 2u) v.y = penalize(v.y, rp);
        if (nib & 4u) v.z = penalize(v.z, rp);
        if (nib & 8u) v.w = penalize(v.w, rp);
    }
}

// p key of one penalized logit: bits of p = (float)exp(sc - M) * inv, 0 outside
// the window. The same function serves both paths, so they agree bit for bit.
__device__ __forceinline__ uint32_t p_key(float sc, float M, float thr, float inv) {
    if (!(sc >= thr)) return 0u;
    const float e = __double2float_rn(exp((double)__fsub_rn(sc, M)));
    return __float_as_uint(__fmul_rn(e, inv));
}

__device__ float block_max_f(float v, Shared& s) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) s.rf[threadIdx.x >> 5] = v;
    __syncthreads();
    float r = s.rf[0];
#pragma unroll
    for (int i = 1; i < WARPS; i++) r = fmaxf(r, s.rf[i]);
    __syncthreads();
    return r;
}

__device__ double block_sum_d(double v, Shared& s) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) s.rd[threadIdx.x >> 5] = v;
    __syncthreads();
    double r = 0.0;
#pragma unroll
    for (int i = 0; i < WARPS; i++) r += s.rd[i];
    __syncthreads();
    return r;
}

__device__ int block_sum_i(int v, Shared& s) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) s.ri[threadIdx.x >> 5] = v;
    __syncthreads();
    int r = 0;
#pragma unroll
    for (int i = 0; i < WARPS; i++) r += s.ri[i];
    __syncthreads();
    return r;
}

// Descending bitonic sort of n (power of two) 64-bit keys in shared memory.
__device__ void bitonic_desc(uint64_t* a, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += THREADS) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t x = a[i], y = a[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (x < y) : (x > y)) { a[i] = y; a[ixj] = x; }
                }
            }
            __syncthreads();
        }
    }
}

// ---------------------------------------------------------------------------
// Row context shared by the passes.
struct Row {
    const float* ptr;
    int V, nq;
    bool vec, use_pen;
    float rp, inv_t, M, thr, inv;
};

// Calls f(sc, idx) for every in-range element whose scaled logit lies in
// [s_lo, s_hi], in coalesced order (thread-interleaved float4 groups).
template <class F>
__device__ __forceinline__ void scan_row(const Row& R, const uint32_t* bits, float s_lo,
                                         float s_hi, F&& f) {
    for (int q = threadIdx.x; q < R.nq; q += THREADS) {
        float4 v = load4(R.ptr, q, R.V, R.vec);
        if (R.use_pen) apply_pen(v, bits, q, R.rp);
        const float sc[4] = {__fmul_rn(v.x, R.inv_t), __fmul_rn(v.y, R.inv_t),
                             __fmul_rn(v.z, R.inv_t), __fmul_rn(v.w, R.inv_t)};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int idx = 4 * q + k;
            if (idx < R.V && sc[k] >= s_lo && sc[k] <= s_hi) f(sc[k], idx);
        }
    }
}

// Scaled-logit interval that can hold p keys in [klo, khi) (khi exclusive).
// Computed once by thread 0 in double with a slack far above every rounding
// step between sc and p (float subtraction, exp, product with inv).
__device__ void key_range_to_sc(const Row& R, uint32_t klo, uint64_t khi, Shared& s) {
    __syncthreads();  // earlier readers of pf_lo / pf_hi are done
    if (threadIdx.x == 0) {
        const double slack = 1e-4 + 1e-6 * fabs((double)R.M);
        const double M = (double)R.M, inv = (double)R.inv;
        float lo = -INFINITY, hi = INFINITY;
        if (klo > 0u) lo = (float)(M + log((double)__uint_as_float(klo) / inv) - slack);
        if (khi < 0x7F800000ull)
            hi = (float)(M + log((double)__uint_as_float((uint32_t)khi) / inv) + slack);
        s.pf_lo = lo;
        s.pf_hi = hi;
    }
    __syncthreads();
}

// Warp 0: first bin, scanning from the top bin down, where the running total
// (mass or count) reaches `target`. Publishes the bin and the mass / count of
// all higher bins. bin_found = 0 when the total stays below target.
__device__ void find_bin(const uint32_t* cnt, const unsigned long long* mass, bool by_mass,
                         unsigned long long target, Shared& s) {
    __syncthreads();  // earlier readers of the bin_* slots are done
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const int hi = NB - 1 - 32 * lane;  // this lane owns bins hi, hi-1, ..., hi-31
        unsigned long long tv = 0, tm = 0;
        unsigned int tc = 0;
        for (int b = hi; b > hi - 32; b--) {
            tm += mass[b];
            tc += cnt[b];
        }
        tv = by_mass ? tm : (unsigned long long)tc;
        unsigned long long incl_v = warp_incl_scan(tv, lane);
        unsigned long long incl_m = warp_incl_scan(tm, lane);
        unsigned int incl_c = warp_incl_scan(tc, lane);
        const unsigned bal = __ballot_sync(FULL, incl_v >= target);
        if (bal == 0u) {
            if (lane == 0) s.bin_found = 0;
        } else {
            const int L = __ffs(bal) - 1;
            if (lane == L) {
                unsigned long long av = incl_v - tv, am = incl_m - tm;
                unsigned int ac = incl_c - tc;
                int found = hi - 31;
                for (int b = hi; b > hi - 32; b--) {
                    const unsigned long long v = by_mass ? mass[b] : (unsigned long long)cnt[b];
                    if (av + v >= target) { found = b; break; }
                    av += v;
                    am += mass[b];
                    ac += cnt[b];
                }
                s.bin_found = 1;
                s.bin = found;
                s.bin_mass_above = am;
                s.bin_cnt_above = ac;
            }
        }
    }
    __syncthreads();
}

__device__ void zero_level2(Hist* H) {
    for (int i = threadIdx.x; i < NB; i += THREADS) {
        H->cnt2[i] = 0u;
        H->mass2[i] = 0ull;
        H->minid2[i] = 0x7FFFFFFF;
    }
    __syncthreads();
}

// Histogram of key bits [shift, shift+10) over the elements whose key has
// prefix `prefix` above bit shift+10.
__device__ void refine(const Row& R, const uint32_t* bits, Hist* H, uint32_t prefix, int shift,
                       Shared& s) {
    zero_level2(H);
    const uint32_t klo = prefix << (shift + 10);
    const uint64_t khi = (uint64_t)(prefix + 1) << (shift + 10);
    key_range_to_sc(R, klo, khi, s);
    const float s_lo = s.pf_lo, s_hi = s.pf_hi;
    scan_row(R, bits, s_lo, s_hi, [&](float sc, int idx) {
        const uint32_t key = p_key(sc, R.M, R.thr, R.inv);
        if (key != 0u && (key >> (shift + 10)) == prefix) {
            const int b = (key >> shift) & (NB - 1);
            atomicAdd(&H->cnt2[b], 1u);
            atomicAdd(&H->mass2[b], fixp(key));
            atomicMin(&H->minid2[b], idx);
        }
    });
    __syncthreads();
}

struct Sel {
    int found;
    int rank;            // position in (p desc, id asc) order
    uint32_t key;        // p key of that position
    int t;               // index inside the group of equal keys (id order)
    int minid;           // smallest id with this key
    unsigned long long m_above;  // mass of strictly larger keys
    unsigned int c_above;        // count of strictly larger keys
};

// Exact select over the row: by_mass -> smallest rank whose cumulative mass
// reaches target; otherwise the element of rank target-1 (target = rank + 1).
__device__ Sel select_row(const Row& R, const uint32_t* bits, Hist* H, bool by_mass,
                          unsigned long long target, Shared& s) {
    Sel out = {};
    if (by_mass && target == 0ull) target = 1ull;  // every window element carries mass >= 1
    find_bin(H->cnt1, H->mass1, by_mass, target, s);
    if (!s.bin_found) return out;
    uint32_t prefix = (uint32_t)s.bin;
    unsigned long long m_above = s.bin_mass_above;
    unsigned int c_above = s.bin_cnt_above;
    int n_eq = 0, minid = 0;
    for (int level = 0; level < 2; level++) {
        const int shift = level == 0 ? 10 : 0;
        refine(R, bits, H, prefix, shift, s);
        const unsigned long long rem = target - (by_mass ? m_above : (unsigned long long)c_above);
        find_bin(H->cnt2, H->mass2, by_mass, rem, s);
        if (!s.bin_found) return out;  // unreachable for consistent histograms
        prefix = (prefix << 10) | (uint32_t)s.bin;
        m_above += s.bin_mass_above;
        c_above += s.bin_cnt_above;
        n_eq = (int)H->cnt2[s.bin];
        minid = H->minid2[s.bin];
        __syncthreads();
    }
    out.found = 1;
    out.key = prefix;
    out.m_above = m_above;
    out.c_above = c_above;
    out.minid = minid;
    if (by_mass) {
        const unsigned long long pf = fixp(prefix);
        const unsigned long long rem = target - m_above;
        long long t = pf ? (long long)((rem + pf - 1) / pf) - 1 : 0;
        out.t = (int)min(max(t, 0ll), (long long)(n_eq - 1));
    } else {
        out.t = (int)(target - 1 - c_above);
    }
    out.rank = (int)c_above + out.t;
    return out;
}

// Id of the t-th element (ascending id) whose key equals `key`.
__device__ int resolve_id(const Row& R, const uint32_t* bits, const Sel& sel, Shared& s) {
    if (sel.t == 0) return sel.minid;
    key_range_to_sc(R, sel.key, (uint64_t)sel.key + 1, s);
    const float s_lo = s.pf_lo, s_hi = s.pf_hi;
    // each thread owns a contiguous run of float4 groups
    const int per = (R.nq + THREADS - 1) / THREADS;
    const int q0 = threadIdx.x * per, q1 = min(q0 + per, R.nq);
    int mine = 0;
    for (int q = q0; q < q1; q++) {
        float4 v = load4(R.ptr, q, R.V, R.vec);
        if (R.use_pen) apply_pen(v, bits, q, R.rp);
        const float l[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float sc = __fmul_rn(l[k], R.inv_t);
            if (4 * q + k < R.V && sc >= s_lo && sc <= s_hi && p_key(sc, R.M, R.thr, R.inv) == sel.key)
                mine++;
        }
    }
    // exclusive block scan of `mine`
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int incl = warp_incl_scan(mine, lane);
    if (lane == 31) s.ri[w] = incl;
    __syncthreads();
    int before = incl - mine;
    for (int i = 0; i < w; i++) before += s.ri[i];
    if (sel.t >= before && sel.t < before + mine) {
        int want = sel.t - before;
        for (int q = q0; q < q1 && want >= 0; q++) {
            float4 v = load4(R.ptr, q, R.V, R.vec);
            if (R.use_pen) apply_pen(v, bits, q, R.rp);
            const float l[4] = {v.x, v.y, v.z, v.w};
            for (int k = 0; k < 4; k++) {
                const float sc = __fmul_rn(l[k], R.inv_t);
                if (4 * q + k < R.V && sc >= s_lo && sc <= s_hi &&
                    p_key(sc, R.M, R.thr, R.inv) == sel.key) {
                    if (want == 0) s.res_pos = 4 * q + k;
                    want--;
                    if (want < 0) break;
                }
            }
        }
    }
    __syncthreads();
    const int id = s.res_pos;
    __syncthreads();
    return id;
}

// Select path: exact cuts and draw over the whole row. Publishes res_id,
// res_nc, res_p.
__device__ void select_path(const Row& R, const uint32_t* bits, Hist* H, const RowParams& P,
                            double u, Shared& s) {
    // level-1 histogram over all window elements
    for (int i = threadIdx.x; i < NB; i += THREADS) {
        H->cnt1[i] = 0u;
        H->mass1[i] = 0ull;
    }
    __syncthreads();
    int nw_local = 0;
    scan_row(R, bits, R.thr, INFINITY, [&](float sc, int idx) {
        const uint32_t key = p_key(sc, R.M, R.thr, R.inv);
        if (key != 0u) {
            atomicAdd(&H->cnt1[key >> 20], 1u);
            atomicAdd(&H->mass1[key >> 20], fixp(key));
            nw_local++;
        }
    });
    const int n_window = block_sum_i(nw_local, s);  // includes the barrier after the pass

    // top-k (sample.c:154)
    const int nc1 = (P.top_k > 0 && P.top_k < n_window) ? P.top_k : n_window;
    // top-p (sample.c:156-160)
    int nc2 = nc1;
    if (P.top_p < 1.0f) {
        const unsigned long long tgt =
            (unsigned long long)ceil((double)P.top_p * 4611686018427387904.0);
        const Sel sp = select_row(R, bits, H, true, tgt, s);
        if (sp.found && sp.rank < nc1) nc2 = sp.rank + 1;
    }
    // min-p (sample.c:162-167): keep = min(nc, max(1, #{p >= min_p * p_max}))
    int nc = nc2;
    if (P.min_p > 0.0f) {
        const float floor_p = __fmul_rn(P.min_p, R.inv);  // p_max = 1 * inv
        const uint32_t fk = __float_as_uint(floor_p);
        const uint32_t fb = fk >> 20;
        int above = 0;
        for (int b = threadIdx.x; b < NB; b += THREADS)
            if ((uint32_t)b > fb) above += (int)H->cnt1[b];
        int in_bin = 0;
        if (fb < (uint32_t)NB) {
            key_range_to_sc(R, fk, (uint64_t)(fb + 1) << 20, s);
            const float s_lo = s.pf_lo, s_hi = s.pf_hi;
            scan_row(R, bits, s_lo, s_hi, [&](float sc, int) {
                const uint32_t key = p_key(sc, R.M, R.thr, R.inv);
                if (key >= fk && (key >> 20) == fb) in_bin++;
            });
        }
        const int ge = block_sum_i(above + in_bin, s);
        nc = min(nc2, max(1, ge));
    }
    if (nc < 1) nc = 1;

    // the last kept element and the kept mass
    const Sel last = select_row(R, bits, H, false, (unsigned long long)nc, s);
    const unsigned long long rsum_fix =
        last.m_above + (unsigned long long)(last.t + 1) * fixp(last.key);
    const double rsum = (double)rsum_fix * (1.0 / 4611686018427387904.0);
    const double r = u * rsum;
    const unsigned long long tgt = (unsigned long long)ceil(r * 4611686018427387904.0);
    Sel d = select_row(R, bits, H, true, tgt, s);
    if (!d.found || d.rank >= nc) d = last;
    const int id = resolve_id(R, bits, d, s);
    if (threadIdx.x == 0) {
        s.res_id = id;
        s.res_nc = nc;
        s.res_p = __uint_as_float(d.key);
    }
    __syncthreads();
}

// Candidate path over the sorted list keys[0, nk): cuts, draw. Warp 0 only.
__device__ void candidate_cuts(const uint64_t* keys, int nk, const RowParams& P, float floor_p,
                               double u, Shared& s) {
    const int lane = threadIdx.x & 31;
    auto pval = [&](int i) { return __uint_as_float((uint32_t)(keys[i] >> 32)); };
    const int BEYOND = 0x7FFFFFFF;
    // top-k: a cut inside the list is exact; a larger k is beyond the min-p cut
    const int nc1 = (P.top_k > 0 && P.top_k < nk) ? P.top_k : BEYOND;
    const int lim = min(nc1, nk);
    int nc2 = nc1;
    if (P.top_p < 1.0f) {
        double carry = 0.0;
        for (int base = 0; base < lim; base += 32) {
            const int i = base + lane;
            const double p = i < lim ? (double)pval(i) : 0.0;
            const double c = warp_incl_scan(p, lane) + carry;
            const unsigned bal = __ballot_sync(FULL, i < lim && c >= (double)P.top_p);
            if (bal) { nc2 = base + __ffs(bal); break; }
            carry = __shfl_sync(FULL, c, 31);
        }
    }
    // min-p: first i >= 1 below the floor; every element outside the list is
    // below the floor, so "not found" means nk
    int fb = nk;
    for (int base = 0; base < nk; base += 32) {
        const int i = base + lane;
        const unsigned bal = __ballot_sync(FULL, i >= 1 && i < nk && pval(i) < floor_p);
        if (bal) { fb = base + __ffs(bal) - 1; break; }
    }
    int nc = min(nc2, fb);
    if (nc < 1) nc = 1;
    // draw
    double part = 0.0;
    for (int i = lane; i < nc; i += 32) part += (double)pval(i);
    const double rsum = warp_sum(part);
    const double r = u * rsum;
    int chosen = nc - 1;
    double carry = 0.0;
    for (int base = 0; base < nc; base += 32) {
        const int i = base + lane;
        const double p = i < nc ? (double)pval(i) : 0.0;
        const double c = warp_incl_scan(p, lane) + carry;
        const unsigned bal = __ballot_sync(FULL, i < nc && c >= r);
        if (bal) { chosen = base + __ffs(bal) - 1; break; }
        carry = __shfl_sync(FULL, c, 31);
    }
    if (lane == 0) {
        s.res_id = (int)(~(uint32_t)keys[chosen]);
        s.res_nc = nc;
        s.res_p = pval(chosen);
    }
}

__global__ void __launch_bounds__(THREADS, 4) sample_rows_kernel(RowsArgs a) {
    extern __shared__ __align__(16) unsigned char dyn[];
    uint64_t* buf = reinterpret_cast<uint64_t*>(dyn);
    uint32_t* bits = reinterpret_cast<uint32_t*>(dyn + CAP * sizeof(uint64_t));
    Hist* H = reinterpret_cast<Hist*>(dyn);
    __shared__ Shared s;
    const int tid = threadIdx.x;

    for (int i = tid; i < a.nwords; i += THREADS) bits[i] = 0u;
    __syncthreads();

    for (int row = blockIdx.x; row < a.B; row += gridDim.x) {
        const RowParams P = clamp_params(a.d_params ? a.d_params[row] : a.h_params);
        const int cap = a.hist ? a.hist_cap : 0;
        int len = 0, head = 0;
        const int32_t* ring = nullptr;
        if (cap > 0) {
            ring = a.hist + (int64_t)row * cap;
            len = a.hist_len ? min(max(a.hist_len[row], 0), cap) : cap;
            head = a.hist_head ? ((a.hist_head[row] % cap) + cap) % cap : 0;
        }
        Row R;
        R.ptr = a.logits + (int64_t)row * a.ld;
        R.V = a.V;
        R.nq = (a.V + 3) >> 2;
        R.vec = a.vec != 0;
        R.use_pen = P.rp > 1.0f && len > 0;
        R.rp = P.rp;
        if (R.use_pen) {
            for (int i = tid; i < len; i += THREADS) {
                const int id = ring[(head + i) % cap];
                if (id >= 0 && id < a.V) atomicOr(&bits[id >> 5], 1u << (id & 31));
            }
        }
        if (tid == 0) {
            s.maxkey = 0u;
            s.cnt = 0;
        }
        __syncthreads();

        int path;
        if (P.T <= 0.0f) {
            // ---- greedy: penalized argmax, first index on ties ----
            float bv = -INFINITY;
            int bi = 0x7FFFFFFF;
            for (int base = 0; base < R.nq; base += TILE_Q) {
                float4 v[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; u++) {
                    const int q = base + u * THREADS + tid;
                    v[u] = q < R.nq ? load4(R.ptr, q, R.V, R.vec)
                                    : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
                }
#pragma unroll
                for (int u = 0; u < UNROLL; u++) {
                    const int q = base + u * THREADS + tid;
                    if (q >= R.nq) continue;
                    if (R.use_pen) apply_pen(v[u], bits, q, R.rp);
                    if (v[u].x > bv) { bv = v[u].x; bi = 4 * q; }
                    if (v[u].y > bv) { bv = v[u].y; bi = 4 * q + 1; }
                    if (v[u].z > bv) { bv = v[u].z; bi = 4 * q + 2; }
                    if (v[u].w > bv) { bv = v[u].w; bi = 4 * q + 3; }
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(FULL, bv, o);
                const int oi = __shfl_xor_sync(FULL, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if ((tid & 31) == 0) {
                s.rf[tid >> 5] = bv;
                s.ri[tid >> 5] = bi;
            }
            __syncthreads();
            if (tid == 0) {
                float best = s.rf[0];
                int besti = s.ri[0];
                for (int w = 1; w < WARPS; w++)
                    if (s.rf[w] > best || (s.rf[w] == best && s.ri[w] < besti)) {
                        best = s.rf[w];
                        besti = s.ri[w];
                    }
                s.res_id = (besti == 0x7FFFFFFF || besti >= a.V) ? 0 : besti;
                s.res_nc = 0;
                s.res_p = 1.0f;
            }
            path = QUASAR_PATH_GREEDY;
            R.inv = 0.0f;
            __syncthreads();
        } else {
            // ---- one streaming pass: max, online window sum, candidates ----
            R.inv_t = __fdiv_rn(1.0f, P.T);
            const bool collect = !(a.flags & QUASAR_FLAG_EXACT_SELECT) && P.min_p > 0.0f;
            // every element with p >= min_p * p_max has sc >= max + cmargin (1% slack)
            const float cmargin =
                collect ? (float)(log((double)fminf(P.min_p, 1.0f)) - 0.01) : 0.0f;
            float m = -INFINITY;
            double S = 0.0;
            const int ntiles = (R.nq + TILE_Q - 1) / TILE_Q;
            for (int it = 0; it < ntiles; it++) {
                const int base = it * TILE_Q;
                float4 v[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; u++) {
                    const int q = base + u * THREADS + tid;
                    v[u] = q < R.nq ? load4(R.ptr, q, R.V, R.vec)
                                    : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
                }
                float sc[4 * UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; u++) {
                    const int q = base + u * THREADS + tid;
                    if (R.use_pen && q < R.nq) apply_pen(v[u], bits, q, R.rp);
                    sc[4 * u + 0] = __fmul_rn(v[u].x, R.inv_t);
                    sc[4 * u + 1] = __fmul_rn(v[u].y, R.inv_t);
                    sc[4 * u + 2] = __fmul_rn(v[u].z, R.inv_t);
                    sc[4 * u + 3] = __fmul_rn(v[u].w, R.inv_t);
                }
                float mt = sc[0];
#pragma unroll
                for (int j = 1; j < 4 * UNROLL; j++) mt = fmaxf(mt, sc[j]);
                if (mt > m) {
                    S *= exp((double)m - (double)mt);
                    m = mt;
                    if (collect) atomicMax(&s.maxkey, ord_key(m));
                }
                if (it == 0) __syncthreads();  // first-tile maxima are published
                if (m > -INFINITY) {
                    const float lo = __fsub_rn(m, 30.0f);
                    float part = 0.0f;
#pragma unroll
                    for (int j = 0; j < 4 * UNROLL; j++)
                        part += (sc[j] >= lo) ? expf(__fsub_rn(sc[j], m)) : 0.0f;
                    S += (double)part;
                }
                if (collect) {
                    const unsigned int mk = *reinterpret_cast<volatile unsigned int*>(&s.maxkey);
                    const float ref = mk ? fmaxf(m, ord_key_inv(mk)) : m;
                    const float tau = __fadd_rn(ref, cmargin);
#pragma unroll
                    for (int j = 0; j < 4 * UNROLL; j++) {
                        if (sc[j] >= tau) {
                            const int idx = 4 * (base + (j >> 2) * THREADS + tid) + (j & 3);
                            if (idx < R.V) {
                                const int pos = atomicAdd(&s.cnt, 1);
                                if (pos < CAP)
                                    buf[pos] = ((uint64_t)__float_as_uint(sc[j]) << 32) | (uint32_t)idx;
                            }
                        }
                    }
                }
            }
            __syncthreads();
            R.M = block_max_f(m, s);
            const double contrib = (m > -INFINITY) ? S * exp((double)m - (double)R.M) : 0.0;
            const double Stot = block_sum_d(contrib, s);
            R.inv = __double2float_rn(1.0 / Stot);
            R.thr = __fsub_rn(R.M, 30.0f);

            // PRNG draw (sample.c:173): one step per stochastic row
            uint64_t st = a.rng[row];
            const double u = rng_unit(&st);

            bool done = false;
            const int n = s.cnt;
            if (collect && n <= CAP && n > 0) {
                const float lo = fmaxf(__fadd_rn(R.M, cmargin), R.thr);
                int mine = 0;
                for (int i = tid; i < n; i += THREADS) {
                    const uint64_t e = buf[i];
                    const float sc = __uint_as_float((uint32_t)(e >> 32));
                    const uint32_t idx = (uint32_t)e;
                    uint64_t key = 0;
                    if (sc >= lo) {
                        const uint32_t pk = p_key(sc, R.M, R.thr, R.inv);
                        key = ((uint64_t)pk << 32) | (uint32_t)(~idx);
                        mine++;
                    }
                    buf[i] = key;
                }
                int n2 = 1;
                while (n2 < n) n2 <<= 1;
                for (int i = n + tid; i < n2; i += THREADS) buf[i] = 0ull;
                const int nk = block_sum_i(mine, s);
                if (nk > 0) {
                    bitonic_desc(buf, n2);
                    if (tid < 32) candidate_cuts(buf, nk, P, __fmul_rn(P.min_p, R.inv), u, s);
                    __syncthreads();
                    done = true;
                    path = QUASAR_PATH_CANDIDATE;
                }
            }
            if (!done) {
                __syncthreads();
                select_path(R, bits, H, P, u, s);
                path = QUASAR_PATH_SELECT;
            }
            if (tid == 0) a.rng[row] = st;
        }

        // ---- epilogue: clear the bitset, record, outputs ----
        const int chosen = s.res_id;
        if (R.use_pen) {
            for (int i = tid; i < len; i += THREADS) {
                const int id = ring[(head + i) % cap];
                if (id >= 0 && id < a.V) bits[id >> 5] = 0u;
            }
        }
        __syncthreads();
        if (tid == 0) {
            a.out[row] = chosen;
            if (a.diag) {
                quasar_pick_diag d;
                d.n_kept = s.res_nc;
                d.p_chosen = s.res_p;
                d.inv_sum = R.inv;
                d.path = path;
                a.diag[row] = d;
            }
            if (a.record && cap > 0 && a.hist_len && a.hist_head) {
                int32_t* wring = a.hist + (int64_t)row * cap;
                if (len < cap) {
                    wring[(head + len) % cap] = chosen;
                    a.hist_len[row] = len + 1;
                } else {
                    wring[head] = chosen;
                    a.hist_head[row] = (head + 1) % cap;
                }
            }
        }
        __syncthreads();
    }
}

}  // namespace rows

size_t rows_smem_bytes(int V) {
    const int nwords = ((V + 31) >> 5) + 1;
    return (size_t)rows::CAP * sizeof(uint64_t) + (size_t)nwords * sizeof(uint32_t);
}

int rows_threads() { return rows::THREADS; }

cudaError_t launch_sample_rows(const RowsArgs& args, int grid, cudaStream_t stream) {
    const size_t smem = rows_smem_bytes(args.V);
    static thread_local size_t configured[64] = {0};
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < 64 && configured[dev] < smem) {
        err = cudaFuncSetAttribute(rows::sample_rows_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (err != cudaSuccess) return err;
        configured[dev] = smem;
    }
    RowsArgs a = args;
    a.nwords = ((args.V + 31) >> 5) + 1;
    rows::sample_rows_kernel<<<grid, rows::THREADS, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace qs
