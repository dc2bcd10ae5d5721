// sample_rows.cu - batched token sampler for sm_100a.
//
// Replaces franzvill/quasar sample.c:111-178 (quasar_sampler_pick), batched:
// every row of a [B, V] fp32 logits matrix is sampled exactly as sample.c
// samples one row, in sample.c's order, by two kernels.
//
// Kernel A (sample_rows_tma / sample_rows_ldg), one pass over each row:
//   1. history ring -> shared-memory bitset of penalized ids (sample.c:120);
//   2. the stream: penalized ids read as -inf, temperature scale (sample.c:
//      137,142), running max, online window sum of exp(sc - m_ref) with a
//      lagging reference m_ref, in fp32 per tile and double per row
//      (sample.c:147), and a one-byte bound of each thread-slot's max (16
//      contiguous elements) in a workspace table with six checkpoint anchors.
//      Elements more than 30 below the max contribute < e^-30 each to the sum
//      instead of being dropped (relative effect < V*e^-30 in the worst case);
//   3. the penalized ids (sample.c:124, exact IEEE divide / multiply) join the
//      max and sum and are listed for kernel B; block reductions give the row
//      max and inv = (float)(1/sum). Greedy rows (temperature <= 0) finish
//      here: penalized argmax, first index on ties, no PRNG step
//      (sample.c:130-134).
// Kernel B (sample_rows_finish), one CTA per stochastic row:
//   candidate path (min_p > 0 or top_k <= 256): the kept prefix lies above a
//   threshold known from the max (min-p floor, or the k-th largest per-thread
//   max); only thread-slots whose bound clears it are read again. Survivors
//   get exact p = (float)exp(sc - max) * inv, ordered by (p desc, id asc) (=
//   glibc's stable qsort, sample.c:151) through per-candidate ranks (<= 256
//   survivors) or a counting sort, then the top-k / top-p / min-p cuts and the
//   inverse-CDF draw with the row's xorshift64* state (sample.c:153-177);
//   select path (any parameters, or more than 4096 candidates): an exact radix
//   select over the p keys of the whole row, re-reading it.
//
//   sample_rows_tma  persistent CTAs of 8 consumer warps + 1 producer warp. The
//                    producer streams the rows' 16 KB chunks with cp.async.bulk
//                    (TMA, this GPU's own memory only, L2 evict-first) into a
//                    3-stage shared-memory ring guarded by mbarriers, running
//                    ahead into the next row while the consumers finish the
//                    current one. Needs rows that start 16-byte aligned and
//                    V % 4 == 0.
//   sample_rows_ldg  the same persistent CTAs without the ring: register loads
//                    with tiles in flight; any alignment and V.
// Every mbarrier wait is bounded (clock64); a timeout sets the abort flag, the
// rows report id -1 and the kernel runs to its end.
#include <float.h>
#include <math.h>

#include <atomic>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "ptx.cuh"
#include "sample_rows.cuh"

namespace qs {
namespace rows {

constexpr int CONSUMERS = 256;                 // consumer threads per CTA (8 warps)
constexpr int CWARPS = CONSUMERS / 32;
constexpr int OCT_TILE = 2 * CONSUMERS;        // 32-byte octets per tile
constexpr int TILE_ELEMS = 8 * OCT_TILE;       // 4096 elements per tile / chunk
constexpr int TILE_BYTES = 4 * TILE_ELEMS;     // 16 KB
constexpr int NSTAGE = 3;                      // ring depth of the TMA kernel
constexpr int CAP = 4096;                      // candidate entries per row
constexpr int TMAX_TILES = 40;                 // tile-max slots per thread (groups of tiles beyond)
constexpr int TMAX_BYTES = TMAX_TILES * CONSUMERS;  // one byte per slot
// Byte tables are laid out [slot / 4][thread][slot % 4]: a thread's four
// consecutive slots share one 32-bit word, so kernel B reads them with one
// coalesced load per four slots.
__host__ __device__ constexpr int tbl_off(int slot, int tid) { return ((slot >> 2) * 256 + tid) * 4 + (slot & 3); }
static_assert(TMAX_TILES % 4 == 0 && CONSUMERS == 256, "byte-table layout");
constexpr int NCK = 6;                         // running-max checkpoints per thread (slots: ck_slot)
constexpr int ANC_BYTES = (NCK + 3) / 4 * 4 * CONSUMERS;  // checkpoint table per row (tbl_off layout)
// Slot of checkpoint k: 1, 3, 7, 11, 19, 27. Slot j is bounded through the
// first checkpoint at or after it (slots past 27: the thread's final max);
// of the six-checkpoint sets whose later checkpoints close a 4-slot table
// word, this one leaves kernel B the fewest slots to re-read on N(0, s)
// rows (11 % fewer than 0, 1, 3, 7, 15, 31).
__host__ __device__ constexpr int ck_slot(int k) {
    return k == 0 ? 1 : k == 1 ? 3 : k == 2 ? 7 : k == 3 ? 11 : k == 4 ? 19 : 27;
}
constexpr int TOPK_MAX = CONSUMERS;            // largest top_k the candidate path takes
constexpr int QMAX = 4096;                     // qualifying thread-tiles re-read per row
// a list entry is slot * CONSUMERS + thread, slot < TMAX_TILES: 16 bits hold it
static_assert(TMAX_TILES * CONSUMERS <= 65536, "16-bit slot-list entries");
constexpr int NB = 1024;                       // radix bins per level (10 bits)
// Candidate key a vocab shard sends first when it has more min-p survivors
// than keys to send (no real key reaches it: p keys are at most 1.0f's bits)
constexpr uint64_t SHARD_OVERFLOW = ~0ull;
constexpr float REF_SLACK = 64.0f;             // kernel A: exp reference lag (nats), e^64 << FLT_MAX
#ifndef QS_LDG_DEPTH
#define QS_LDG_DEPTH 1
#endif
#ifndef QS_A_CTAS
#define QS_A_CTAS 3
#endif
constexpr int LDG_DEPTH = QS_LDG_DEPTH;        // tiles in flight per thread, row-load kernel

// The select path reuses the candidate storage as histograms.
struct Hist {
    uint32_t cnt1[NB];
    unsigned long long mass1[NB];
    uint32_t cnt2[NB];
    unsigned long long mass2[NB];
    int32_t minid2[NB];
};
// kernel B scratch: candidate keys [CAP]; the select path's histograms alias it
constexpr int FINISH_SCRATCH = (int)sizeof(Hist) > CAP * 8 ? (int)sizeof(Hist) : CAP * 8;

// Counting sort of the candidate keys (kernel B): NBK buckets of the p key's
// bits below the row's largest key, two per consumer thread.
constexpr int NBK = 512;
constexpr int BK_MAX = 256;  // largest bucket the in-bucket ranking takes
struct Buckets {
    uint32_t cnt[NBK];
    uint32_t start[NBK];
};
static_assert(sizeof(Buckets) >= CONSUMERS * sizeof(uint64_t), "topk_floor's scratch");

struct Shared {
    int abort;            // a bounded wait gave up
    int ncand;            // candidate keys appended
    int nq;               // qualifying thread-tiles listed
    int npen;             // penalized ids listed (kernel A)
    float tfmax[CONSUMERS];  // each consumer thread's final running max (scaled)
    float rf[CWARPS];
    double rd[CWARPS];
    int ri[CWARPS];
    // broadcast slots
    int bin_found, bin;
    unsigned long long bin_mass_above;
    unsigned int bin_cnt_above;
    float pf_lo, pf_hi;
    int res_id, res_nc, res_pos;
    float res_p;
    int cut_p, cut_m, cut_d;  // candidate cuts (atomicMin targets)
    int big_bucket;           // a bucket of the counting sort exceeds BK_MAX
    uint32_t bk_hi[CWARPS];   // per-warp maxima of the counting sort's keys
    double rsum;
};

// Kernel A's shared state: the common slots plus the penalty mask table.
struct SharedA : Shared {
    // the CTA's next row, copied during the current row's tail (stage_next_row):
    // parameters and ring position; its first CONSUMERS ring slots go to tfmax
    quasar_sample_params nxt_pr;
    int nxt_len, nxt_head;
};

// Barrier of the 256 consumer threads (warps 0-7); the TMA producer warp never
// takes part, so it can run ahead into the next row.
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ void lds4(uint32_t addr, float* v) {
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
                 : "r"(addr)
                 : "memory");
}
// Asynchronous 4-byte global -> shared copy (cp.async) and its wait.
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Mass fixed point: p * 2^62 truncated (p <= 1, row sums stay below 2^64).
__device__ __forceinline__ unsigned long long fixp(uint32_t pkey) {
    return __float2ull_rz(__fmul_rn(__uint_as_float(pkey), 4611686018427387904.0f));
}

// 256-bit streaming load of 8 floats (32-byte aligned address).
__device__ __forceinline__ void ld4(const float* p, float* v) {
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
                 : "l"(p));
}
__device__ __forceinline__ void ld8(const float* p, float* v) {
    asm volatile("ld.global.nc.L1::no_allocate.L2::evict_first.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]),
                   "=f"(v[7])
                 : "l"(p));
}

// One 32-byte octet of a row (elements 8o..8o+7) from global memory with the
// default cache policy: a single 256-bit load when the row is 32-byte aligned
// (sm_100 ld.global.v8), else masked scalar loads; elements past V read as -inf.
__device__ __forceinline__ void load_oct_keep(const float* row, int o, int V, bool vec, float* v) {
    const int e = o * 8;
    if (vec && e + 7 < V) {
        asm volatile("ld.global.nc.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]),
                       "=f"(v[6]), "=f"(v[7])
                     : "l"(row + e));
    } else {
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = (e + k < V) ? __ldg(row + e + k) : -INFINITY;
    }
}

// Penalty for the octet whose bitset byte is `m` (bit k = element 8o+k).
__device__ __forceinline__ void apply_pen_oct(float* v, uint32_t m, float rp) {
#pragma unroll
    for (int k = 0; k < 8; k++)
        if (m & (1u << k)) v[k] = penalize(v[k], rp);
}

__device__ float block_max_f(float v, Shared& s) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) s.rf[threadIdx.x >> 5] = v;
    csync();
    float r = s.rf[0];
#pragma unroll
    for (int i = 1; i < CWARPS; i++) r = fmaxf(r, s.rf[i]);
    csync();
    return r;
}

__device__ double block_sum_d(double v, Shared& s) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) s.rd[threadIdx.x >> 5] = v;
    csync();
    double r = 0.0;
#pragma unroll
    for (int i = 0; i < CWARPS; i++) r += s.rd[i];
    csync();
    return r;
}

__device__ int block_sum_i(int v, Shared& s) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) s.ri[threadIdx.x >> 5] = v;
    csync();
    int r = 0;
#pragma unroll
    for (int i = 0; i < CWARPS; i++) r += s.ri[i];
    csync();
    return r;
}

__device__ unsigned long long block_sum_u64(unsigned long long v, Shared& s) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) s.rd[threadIdx.x >> 5] = __longlong_as_double((long long)v);
    csync();
    unsigned long long r = 0ull;
#pragma unroll
    for (int i = 0; i < CWARPS; i++) r += (unsigned long long)__double_as_longlong(s.rd[i]);
    csync();
    return r;
}

// Descending bitonic sort of n (power of two) 64-bit keys in shared memory.
__device__ void bitonic_desc(uint64_t* a, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += CONSUMERS) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t x = a[i], y = a[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (x < y) : (x > y)) {
                        a[i] = y;
                        a[ixj] = x;
                    }
                }
            }
            csync();
        }
    }
}

// ---------------------------------------------------------------------------
// Row context shared by the passes.
struct Row {
    const float* ptr;
    int V, noct, ntiles;
    bool vec, use_pen;
    float rp, inv_t, M, thr, inv;
};

// Octets in flight per thread in the select path's passes over a row (2:
// more unrolling made the passes bound by instruction fetch).
#ifndef QS_SCAN_U
#define QS_SCAN_U 2
#endif
constexpr int SCAN_U = QS_SCAN_U;
// The select path's steps, inlined; select_path calls select_row from one
// loop, so the kernel holds one copy of each pass (its whole-row passes are
// bound by instruction fetch when the kernel's code outgrows the
// instruction cache).
#define QS_SELECT_FN __device__

// Calls f(sc, idx) for every in-range element whose scaled logit lies in
// [s_lo, s_hi], reading the row from global memory in coalesced octets,
// SCAN_U loads in flight per thread. The select path passes over the same
// row up to ten times, so the loads keep the default L2 policy: after the
// first pass the row is read from L2.
template <class F>
__device__ __forceinline__ void scan_row(const Row& R, const uint8_t* bits8, float s_lo, float s_hi,
                                         F&& f) {
    for (int ob = threadIdx.x; ob < R.noct; ob += SCAN_U * CONSUMERS) {
        float v[SCAN_U][8];
#pragma unroll
        for (int u = 0; u < SCAN_U; u++)
            if (ob + u * CONSUMERS < R.noct) load_oct_keep(R.ptr, ob + u * CONSUMERS, R.V, R.vec, v[u]);
#pragma unroll
        for (int u = 0; u < SCAN_U; u++) {
            const int o = ob + u * CONSUMERS;
            if (o < R.noct) {
                if (R.use_pen) apply_pen_oct(v[u], bits8[o], R.rp);
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const float sc = __fmul_rn(v[u][k], R.inv_t);
                    const int idx = 8 * o + k;
                    if (idx < R.V && sc >= s_lo && sc <= s_hi) f(sc, idx);
                }
            }
        }
    }
}

// Scaled-logit interval that can hold p keys in [klo, khi) (khi exclusive),
// computed by thread 0 in double with a slack far above every rounding step
// between sc and p (float subtraction, exp, product with inv).
__device__ void key_range_to_sc(const Row& R, uint32_t klo, uint64_t khi, Shared& s) {
    csync();  // earlier readers of pf_lo / pf_hi are done
    if (threadIdx.x == 0) {
        const double slack = 1e-4 + 1e-6 * fabs((double)R.M);
        const double M = (double)R.M, inv = (double)R.inv;
        float lo = -INFINITY, hi = INFINITY;
        if (klo > 0u) lo = (float)(M + log((double)__uint_as_float(klo) / inv) - slack);
        if (khi < 0x7F800000ull) hi = (float)(M + log((double)__uint_as_float((uint32_t)khi) / inv) + slack);
        s.pf_lo = lo;
        s.pf_hi = hi;
    }
    csync();
}

// Warp 0: first bin, scanning from the top bin down, where the running total
// (mass or count) reaches `target` (>= 1). Publishes the bin and the mass and
// count of all higher bins; bin_found = 0 when the total stays below target.
__device__ void find_bin(const uint32_t* cnt, const unsigned long long* mass, bool by_mass,
                         unsigned long long target, Shared& s) {
    csync();  // earlier readers of the bin_* slots are done
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const int hi = NB - 1 - 32 * lane;  // this lane owns bins hi, hi-1, ..., hi-31
        unsigned long long tm = 0;
        unsigned int tc = 0;
        for (int b = hi; b > hi - 32; b--) {
            tm += mass[b];
            tc += cnt[b];
        }
        const unsigned long long tv = by_mass ? tm : (unsigned long long)tc;
        const unsigned long long incl_v = warp_incl_scan(tv, lane);
        const unsigned long long incl_m = warp_incl_scan(tm, lane);
        const unsigned int incl_c = warp_incl_scan(tc, lane);
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
                    if (av + v >= target) {
                        found = b;
                        break;
                    }
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
    csync();
}

__device__ void zero_level2(Hist* H) {
    for (int i = threadIdx.x; i < NB; i += CONSUMERS) {
        H->cnt2[i] = 0u;
        H->mass2[i] = 0ull;
        H->minid2[i] = 0x7FFFFFFF;
    }
    csync();
}

// Histogram of key bits [shift, shift+10) over the elements whose key has
// prefix `prefix` above bit shift+10.
QS_SELECT_FN void refine(const Row& R, const uint8_t* bits8, Hist* H, uint32_t prefix, int shift,
                       Shared& s) {
    zero_level2(H);
    const uint32_t klo = prefix << (shift + 10);
    const uint64_t khi = (uint64_t)(prefix + 1) << (shift + 10);
    key_range_to_sc(R, klo, khi, s);
    const float s_lo = s.pf_lo, s_hi = s.pf_hi;
    scan_row(R, bits8, s_lo, s_hi, [&](float sc, int idx) {
        const uint32_t key = p_key(sc, R.M, R.thr, R.inv);
        if (key != 0u && (key >> (shift + 10)) == prefix) {
            const int b = (key >> shift) & (NB - 1);
            atomicAdd(&H->cnt2[b], 1u);
            atomicAdd(&H->mass2[b], fixp(key));
            atomicMin(&H->minid2[b], idx);
        }
    });
    csync();
}

struct Sel {
    int found;
    int rank;                    // position in (p desc, id asc) order
    uint32_t key;                // p key of that position
    int t;                       // index inside the group of equal keys (id order)
    int minid;                   // smallest id with this key
    unsigned long long m_above;  // mass of strictly larger keys
    unsigned int c_above;        // count of strictly larger keys
};

// Exact select over the row: by_mass -> smallest rank whose cumulative mass
// reaches target; otherwise the element of rank target-1 (target = rank + 1).
QS_SELECT_FN Sel select_row(const Row& R, const uint8_t* bits8, Hist* H, bool by_mass,
                          unsigned long long target, Shared& s) {
    Sel out = {};
    if (by_mass && target == 0ull) target = 1ull;  // every window element carries mass >= 1
    find_bin(H->cnt1, H->mass1, by_mass, target, s);
    if (!s.bin_found) return out;
    uint32_t prefix = (uint32_t)s.bin;
    unsigned long long m_above = s.bin_mass_above;
    unsigned int c_above = s.bin_cnt_above;
    int n_eq = 0, minid = 0;
#pragma unroll 1
    for (int level = 0; level < 2; level++) {
        const int shift = level == 0 ? 10 : 0;
        refine(R, bits8, H, prefix, shift, s);
        const unsigned long long rem = target - (by_mass ? m_above : (unsigned long long)c_above);
        find_bin(H->cnt2, H->mass2, by_mass, rem, s);
        if (!s.bin_found) return out;  // unreachable for consistent histograms
        prefix = (prefix << 10) | (uint32_t)s.bin;
        m_above += s.bin_mass_above;
        c_above += s.bin_cnt_above;
        n_eq = (int)H->cnt2[s.bin];
        minid = H->minid2[s.bin];
        csync();
    }
    out.found = 1;
    out.key = prefix;
    out.m_above = m_above;
    out.c_above = c_above;
    out.minid = minid;
    if (by_mass) {
        const unsigned long long pf = fixp(prefix);
        const unsigned long long rem = target - m_above;
        const long long t = pf ? (long long)((rem + pf - 1) / pf) - 1 : 0;
        out.t = (int)min(max(t, 0ll), (long long)(n_eq - 1));
    } else {
        out.t = (int)(target - 1 - c_above);
    }
    out.rank = (int)c_above + out.t;
    return out;
}

// Id of the t-th element (ascending id) whose key equals sel.key.
QS_SELECT_FN int resolve_id(const Row& R, const uint8_t* bits8, const Sel& sel, Shared& s) {
    if (sel.t == 0) return sel.minid;
    key_range_to_sc(R, sel.key, (uint64_t)sel.key + 1, s);
    const float s_lo = s.pf_lo, s_hi = s.pf_hi;
    // each thread owns a contiguous run of octets
    const int per = (R.noct + CONSUMERS - 1) / CONSUMERS;
    const int o0 = threadIdx.x * per, o1 = min(o0 + per, R.noct);
    auto match = [&](float l, int idx) {
        const float sc = __fmul_rn(l, R.inv_t);
        return idx < R.V && sc >= s_lo && sc <= s_hi && p_key(sc, R.M, R.thr, R.inv) == sel.key;
    };
    int mine = 0;
    for (int ob = o0; ob < o1; ob += SCAN_U) {  // SCAN_U loads in flight
        float v[SCAN_U][8];
#pragma unroll
        for (int u = 0; u < SCAN_U; u++)
            if (ob + u < o1) load_oct_keep(R.ptr, ob + u, R.V, R.vec, v[u]);
#pragma unroll
        for (int u = 0; u < SCAN_U; u++) {
            if (ob + u < o1) {
                if (R.use_pen) apply_pen_oct(v[u], bits8[ob + u], R.rp);
#pragma unroll
                for (int k = 0; k < 8; k++) mine += match(v[u][k], 8 * (ob + u) + k) ? 1 : 0;
            }
        }
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int incl = warp_incl_scan(mine, lane);
    if (lane == 31) s.ri[w] = incl;
    csync();
    int before = incl - mine;
    for (int i = 0; i < w; i++) before += s.ri[i];
    if (sel.t >= before && sel.t < before + mine) {
        int want = sel.t - before;
        for (int o = o0; o < o1 && want >= 0; o++) {
            float v[8];
            load_oct_keep(R.ptr, o, R.V, R.vec, v);
            if (R.use_pen) apply_pen_oct(v, bits8[o], R.rp);
            for (int k = 0; k < 8 && want >= 0; k++) {
                if (match(v[k], 8 * o + k)) {
                    if (want == 0) s.res_pos = 8 * o + k;
                    want--;
                }
            }
        }
    }
    csync();
    const int id = s.res_pos;
    csync();
    return id;
}

// Select path: exact cuts and draw over the whole row. Publishes res_id,
// res_nc, res_p.
QS_SELECT_FN void select_path(const Row& R, const uint8_t* bits8, Hist* H,
                                         const RowParams& P, double u, Shared& s) {
    for (int i = threadIdx.x; i < NB; i += CONSUMERS) {
        H->cnt1[i] = 0u;
        H->mass1[i] = 0ull;
    }
    csync();
    int nw_local = 0;
    scan_row(R, bits8, R.thr, INFINITY, [&](float sc, int) {
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
    // min-p (sample.c:162-167): keep = min(nc, max(1, #{p >= min_p * p_max}))
    int ge = 0x7FFFFFFF;
    if (P.min_p > 0.0f) {
        const float floor_p = __fmul_rn(P.min_p, R.inv);  // p_max = 1 * inv
        const uint32_t fk = __float_as_uint(floor_p);
        const uint32_t fb = fk >> 20;
        int above = 0;
        for (int b = threadIdx.x; b < NB; b += CONSUMERS)
            if ((uint32_t)b > fb) above += (int)H->cnt1[b];
        int in_bin = 0;
        if (fb < (uint32_t)NB) {
            key_range_to_sc(R, fk, (uint64_t)(fb + 1) << 20, s);
            const float s_lo = s.pf_lo, s_hi = s.pf_hi;
            scan_row(R, bits8, s_lo, s_hi, [&](float sc, int) {
                const uint32_t key = p_key(sc, R.M, R.thr, R.inv);
                if (key >= fk && (key >> 20) == fb) in_bin++;
            });
        }
        ge = max(1, block_sum_i(above + in_bin, s));
    }
    // Three exact selects, in one loop so that the select code exists once
    // in the kernel: 0 the top-p position (sample.c:156-160), 1 the last
    // kept element (its kept mass, sample.c:171-172), 2 the draw position
    // (sample.c:173-177). Step 1 is skipped when its answer is already
    // known: the top-p position itself, or every window element (rsum = the
    // histogram's whole mass).
    int nc2 = nc1, nc = nc1;
    Sel last = {}, d = {};
    double rsum = 0.0;
#pragma unroll 1
    for (int step = 0; step < 3; step++) {
        bool by_mass = true;
        unsigned long long tgt = 0ull;
        if (step == 0) {
            if (!(P.top_p < 1.0f)) continue;
            tgt = (unsigned long long)ceil((double)P.top_p * 4611686018427387904.0);
        } else if (step == 1) {
            nc = max(1, min(nc2, ge));
            if (nc == n_window && !last.found) {
                // every window element is kept: the kept mass is the whole histogram's
                unsigned long long m = 0ull;
                for (int b = threadIdx.x; b < NB; b += CONSUMERS) m += H->mass1[b];
                m = block_sum_u64(m, s);
                rsum = (double)m * (1.0 / 4611686018427387904.0);
                continue;
            }
            if (last.found && last.rank == nc - 1) {  // the top-p position is the last kept element
                rsum = (double)(last.m_above + (unsigned long long)(last.t + 1) * fixp(last.key)) *
                       (1.0 / 4611686018427387904.0);
                continue;
            }
            by_mass = false;
            tgt = (unsigned long long)nc;
        } else {
            tgt = (unsigned long long)ceil(u * rsum * 4611686018427387904.0);  // r = u * rsum
        }
        const Sel x = select_row(R, bits8, H, by_mass, tgt, s);
        if (step == 0) {
            if (x.found && x.rank < nc1) {
                nc2 = x.rank + 1;
                last = x;
            }
        } else if (step == 1) {
            last = x;
            rsum = (double)(last.m_above + (unsigned long long)(last.t + 1) * fixp(last.key)) *
                   (1.0 / 4611686018427387904.0);
        } else {
            d = x;
        }
    }
    if (!d.found || d.rank >= nc) {
        // the draw fell past the kept set (r at the very end): its last element
        if (!last.found || last.rank != nc - 1) last = select_row(R, bits8, H, false, (unsigned long long)nc, s);
        d = last;
    }
    const int id = resolve_id(R, bits8, d, s);
    if (threadIdx.x == 0) {
        s.res_id = id;
        s.res_nc = nc;
        s.res_p = __uint_as_float(d.key);
    }
    csync();
}

// Candidate path over the sorted list keys[0, nk): cuts and draw by all
// consumer threads. Thread t owns the contiguous positions [t*L, t*L + L);
// cumulative sums are per-thread double sums joined by a block scan (the
// reference's sequential double cumsum, regrouped: equal up to ~1e-16).
__device__ void candidate_cuts(const uint64_t* keys, int nk, const RowParams& P, float floor_p,
                               double u, Shared& s) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int BEYOND = 0x7FFFFFFF;
    auto pval = [&](int i) { return __uint_as_float((uint32_t)(keys[i] >> 32)); };
    const int L = (nk + CONSUMERS - 1) / CONSUMERS;
    const int i0 = min(tid * L, nk), i1 = min(i0 + L, nk);
    double seg = 0.0;
    for (int i = i0; i < i1; i++) seg += (double)pval(i);
    const double incl = warp_incl_scan(seg, lane);
    if (lane == 31) s.rd[w] = incl;
    if (tid == 0) {
        s.cut_p = BEYOND;
        s.cut_m = nk;
        s.cut_d = BEYOND;
    }
    csync();
    double excl = incl - seg;
    for (int k = 0; k < w; k++) excl += s.rd[k];
    // top-k (sample.c:154): a cut inside the list is exact; a larger k lies
    // beyond the list's own bound
    const int nc1 = (P.top_k > 0 && P.top_k < nk) ? P.top_k : BEYOND;
    const int lim = min(nc1, nk);
    // top-p (sample.c:156-160): first prefix whose cumsum reaches top_p
    if (P.top_p < 1.0f) {
        double c = excl;
        for (int i = i0; i < min(i1, lim); i++) {
            c += (double)pval(i);
            if (c >= (double)P.top_p) {
                atomicMin(&s.cut_p, i + 1);
                break;
            }
        }
    }
    // min-p (sample.c:162-167): first i >= 1 below the floor; every element
    // outside the list is below the floor, so "none" means nk
    for (int i = max(i0, 1); i < i1; i++)
        if (pval(i) < floor_p) {
            atomicMin(&s.cut_m, i);
            break;
        }
    csync();
    const int nc2 = s.cut_p != BEYOND ? s.cut_p : nc1;
    const int nc = max(1, min(nc2, s.cut_m));
    if (nc - 1 >= i0 && nc - 1 < i1) {  // the kept mass (sample.c:171-172)
        double c = excl;
        for (int i = i0; i < nc; i++) c += (double)pval(i);
        s.rsum = c;
    }
    csync();
    const double r = u * s.rsum;  // sample.c:173-175
    {
        double c = excl;
        for (int i = i0; i < min(i1, nc); i++) {
            c += (double)pval(i);
            if (c >= r) {
                atomicMin(&s.cut_d, i);
                break;
            }
        }
    }
    csync();
    if (tid == 0) {
        const int chosen = s.cut_d != BEYOND ? s.cut_d : nc - 1;
        s.res_id = (int)(~(uint32_t)keys[chosen]);
        s.res_nc = nc;
        s.res_p = pval(chosen);
    }
    csync();
}

// Cuts and draw for a short candidate list (nk <= RANK_MAX), without sorting
// and with four barriers: thread t < nk takes raw entry t (at buf[CAP - nk,
// CAP)), finds its rank in (p desc, id asc) order and the mass above it by
// scanning all nk keys, so every cumsum of candidate_cuts is known at its
// rank. Masses are exact integer sums of p * 2^54 (each p <= 1, nk <= 256:
// no overflow), so the cumsums agree with the reference's double sums far
// inside the CDF tolerance. A vocab shard (cand != nullptr) writes its first
// shard_k keys in order instead, ids made global.
constexpr int RANK_MAX = CONSUMERS;
__device__ void rank_cuts(uint64_t* buf, int nk, const Row& R, const RowParams& P, float floor_p, double u,
                          Shared& s, uint64_t* cand, int shard_k, int64_t col0) {
    const int tid = threadIdx.x;
    const int BEYOND = 0x7FFFFFFF;
    ulonglong2* E = reinterpret_cast<ulonglong2*>(buf);  // {key, p * 2^54}, buf[0, 2 nk): below the raw entries
    uint64_t key = 0ull;
    float p = 0.0f;
    unsigned long long fix = 0ull;
    if (tid < nk) {
        const uint64_t en = buf[CAP - nk + tid];
        const uint32_t pk = p_key(__uint_as_float((uint32_t)(en >> 32)), R.M, R.thr, R.inv);
        key = ((uint64_t)pk << 32) | (uint32_t)(~(uint32_t)en);
        p = __uint_as_float(pk);
        fix = __float2ull_rz(p * 18014398509481984.0f);  // p * 2^54, exact
    }
    if (tid == 0) {
        s.cut_p = BEYOND;
        s.cut_m = nk;
        s.cut_d = BEYOND;
    }
    csync();  // every raw entry is read
    if (tid < nk) E[tid] = make_ulonglong2(key, fix);
    csync();
    int rank = 0;
    unsigned long long above = 0ull;
    if (tid < nk) {
#pragma unroll 4
        for (int j = 0; j < nk; j++) {
            const ulonglong2 e = E[j];
            const bool gt = e.x > key;
            rank += gt ? 1 : 0;
            above += gt ? e.y : 0ull;
        }
    }
    if (cand) {
        if (tid < nk && rank < shard_k)
            cand[rank] = (key & 0xFFFFFFFF00000000ull) | (uint32_t)(~(uint32_t)(col0 + (int64_t)(~(uint32_t)key)));
        for (int i = nk + tid; i < shard_k; i += CONSUMERS) cand[i] = 0ull;
        return;
    }
    const double cum = (double)(above + fix) * 0x1p-54;  // inclusive cumsum at this rank
    const int nc1 = (P.top_k > 0 && P.top_k < nk) ? P.top_k : BEYOND;
    if (tid < nk) {
        // top-k (sample.c:154); top-p (sample.c:156-160): first prefix whose
        // cumsum reaches top_p; min-p (sample.c:162-167): first i >= 1 below
        // the floor (none: nk)
        if (P.top_p < 1.0f && rank < min(nc1, nk) && cum >= (double)P.top_p) atomicMin(&s.cut_p, rank + 1);
        if (rank >= 1 && p < floor_p) atomicMin(&s.cut_m, rank);
    }
    csync();
    const int nc2 = s.cut_p != BEYOND ? s.cut_p : nc1;
    const int nc = max(1, min(nc2, s.cut_m));
    if (tid < nk && rank == nc - 1) s.rsum = cum;  // the kept mass (sample.c:171-172)
    csync();
    const double r = u * s.rsum;  // sample.c:173-175: first kept i with r <= cumsum
    if (tid < nk && rank < nc && cum >= r) atomicMin(&s.cut_d, rank);
    csync();
    const int chosen = s.cut_d != BEYOND ? s.cut_d : nc - 1;
    if (tid < nk && rank == chosen) {
        s.res_id = (int)(~(uint32_t)key);
        s.res_nc = nc;
        s.res_p = p;
    }
    csync();
}

// Tile-max table entry: how far (in 1/8 nat, rounded down, saturating at 255)
// a slot's max lies below the thread's running max m at the slot's end. Since
// m only grows, slot max <= (thread's final max) - d/8 holds at the end.
__device__ __forceinline__ uint8_t tile_deficit(float m, float slotmax) {
    const float d = __fmul_rd(__fsub_rd(m, slotmax), 8.0f);  // never above the true deficit
    return !(d < 255.0f) ? (uint8_t)255 : (uint8_t)(int)d;   // NaN / +inf -> 255
}
// tile_deficit as a 32-bit value, for packing four slots into one store
// (fminf maps NaN to 255, like tile_deficit).
__device__ __forceinline__ uint32_t deficit_byte(float m, float slotmax) {
    return __float2uint_rd(fminf(__fmul_rd(__fsub_rd(m, slotmax), 8.0f), 255.0f));
}
// Lower bound of the k-th largest scaled logit of the row (k <= 256): the
// k-th largest of the 256 per-thread maxima (256 distinct elements), lowered by
// a margin that covers ties in p. Rank by (value desc, thread asc).
// Each warp sorts its 32 maxima (keys ord_key(max) << 32 | (255 - thread):
// value desc, thread asc) with a shuffle bitonic network and publishes the
// sorted run in `scratch` (CONSUMERS keys); every thread then ranks the key it
// holds against the other runs by binary search, and the holder of rank k-1
// publishes its value.
__device__ float topk_floor(int k, Shared& s, uint64_t* scratch) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    uint64_t key = ((uint64_t)ord_key(s.tfmax[tid]) << 32) | (uint32_t)(CONSUMERS - 1 - tid);
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
            const uint64_t other = __shfl_xor_sync(FULL, key, j);
            const bool up = (lane & size) != 0;  // size 32: descending over the warp
            key = (((lane & j) == 0) != up) ? max(key, other) : min(key, other);
        }
    }
    scratch[tid] = key;  // lane L holds its warp's L-th largest key
    csync();
    int rank = lane;
#pragma unroll
    for (int v = 0; v < CWARPS; v++) {
        if (v == w) continue;
        const uint64_t* run = scratch + 32 * v;
        int lo = 0, hi = 32;  // keys of run v greater than this one
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (run[mid] > key) lo = mid + 1;
            else hi = mid;
        }
        rank += lo;
    }
    if (rank == k - 1) s.pf_lo = ord_key_inv((uint32_t)(key >> 32));
    csync();
    const float t = s.pf_lo;
    csync();
    if (!(t > -INFINITY)) return -INFINITY;
    return t - (1e-5f + 1e-5f * fabsf(t));
}

// Lower bound of the kept prefix of a row cut by top-p alone (sample.c:
// 155-160), from the 256 per-thread maxima: sorted descending (warp sorts,
// then ranks, as topk_floor), with their exact p (p_key) summed in double
// down the order, the first maximum where the sum reaches top_p (with a
// 1e-9 safety margin) bounds the prefix - every element at or above it
// carries at least that mass, so the top-p cut falls among them. Returns
// that value less topk_floor's tie margin, or -inf when the maxima do not
// carry top_p. Uses `scratch` (2 KB) and s.tfmax; all consumer threads.
__device__ float topp_floor(float top_p, const Row& R, Shared& s, uint64_t* scratch) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    uint64_t key = ((uint64_t)ord_key(s.tfmax[tid]) << 32) | (uint32_t)(CONSUMERS - 1 - tid);
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
            const uint64_t other = __shfl_xor_sync(FULL, key, j);
            const bool up = (lane & size) != 0;
            key = (((lane & j) == 0) != up) ? max(key, other) : min(key, other);
        }
    }
    scratch[tid] = key;
    csync();
    int rank = lane;
#pragma unroll
    for (int v = 0; v < CWARPS; v++) {
        if (v == w) continue;
        const uint64_t* run = scratch + 32 * v;
        int lo = 0, hi = 32;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (run[mid] > key) lo = mid + 1;
            else hi = mid;
        }
        rank += lo;
    }
    csync();  // every run is read
    // the values in rank order (the thread holding rank r writes slot r)
    float* sorted = reinterpret_cast<float*>(scratch);
    const float val = ord_key_inv((uint32_t)(key >> 32));
    sorted[rank] = val;
    if (tid == 0) s.cut_p = 0x7FFFFFFF;
    csync();
    // this thread takes rank tid: its p and the double sum down to it
    const float mv = sorted[tid];
    const double pv = (double)__uint_as_float(p_key(mv, R.M, R.thr, R.inv));
    const double incl = warp_incl_scan(pv, lane);
    if (lane == 31) s.rd[w] = incl;
    csync();
    double cum = incl;
    for (int v = 0; v < w; v++) cum += s.rd[v];
    if (cum >= (double)top_p + 1e-9) atomicMin(&s.cut_p, tid);
    csync();
    const int j = s.cut_p;
    const float t = j < CONSUMERS ? sorted[j] : -INFINITY;
    csync();  // sorted and cut_p are read before any later use
    if (!(t > -INFINITY)) return -INFINITY;
    return t - (1e-5f + 1e-5f * fabsf(t));
}

// Minimum and maximum of an unsigned value over the consumer threads.
__device__ void block_minmax_u(uint32_t& lo, uint32_t& hi, Shared& s) {
    lo = __reduce_min_sync(FULL, lo);
    hi = __reduce_max_sync(FULL, hi);
    if ((threadIdx.x & 31) == 0) {
        s.ri[threadIdx.x >> 5] = (int)lo;
        s.bk_hi[threadIdx.x >> 5] = hi;
    }
    csync();
    lo = (uint32_t)s.ri[0];
    hi = s.bk_hi[0];
#pragma unroll
    for (int i = 1; i < CWARPS; i++) {
        lo = min(lo, (uint32_t)s.ri[i]);
        hi = max(hi, s.bk_hi[i]);
    }
    csync();
}

// Converts the nk raw (sc, id) entries at buf[CAP - nk, CAP) into (p, ~id)
// keys and sorts them descending (requires nk <= CAP / 2): a counting sort
// over NBK buckets of (largest key - key) >> sh, sh the smallest shift that
// fits the row's key range (bucket order is key order; equal p share a
// bucket), scattered to buf[0, nk); then every key finds its place inside its
// bucket by counting the larger keys there, and lands at buf[CAP - nk + rank].
// Returns the sorted keys, or nullptr when a bucket holds more than BK_MAX
// keys (the converted keys are then left unsorted at buf[CAP - nk, CAP)).
__device__ const uint64_t* bucket_sort_keys(uint64_t* buf, int nk, const Row& R, Buckets* bk, Shared& s) {
    const int tid = threadIdx.x;
    uint64_t* src = buf + CAP - nk;
    uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
    for (int i = tid; i < nk; i += CONSUMERS) {
        const uint64_t en = src[i];
        const uint32_t pk = p_key(__uint_as_float((uint32_t)(en >> 32)), R.M, R.thr, R.inv);
        src[i] = ((uint64_t)pk << 32) | (uint32_t)(~(uint32_t)en);
        kmin = min(kmin, pk);
        kmax = max(kmax, pk);
    }
    for (int b = tid; b < NBK; b += CONSUMERS) bk->cnt[b] = 0u;
    if (tid == 0) s.big_bucket = 0;
    // every key lies in [kmin, kmax], so every bucket index is in [0, NBK)
    block_minmax_u(kmin, kmax, s);
    int sh = 0;
    while (((kmax - kmin) >> sh) >= (uint32_t)NBK) sh++;
    for (int i = tid; i < nk; i += CONSUMERS)
        atomicAdd(&bk->cnt[(kmax - (uint32_t)(src[i] >> 32)) >> sh], 1u);
    csync();
    {
        // exclusive scan of the counts: thread t owns buckets PER*t .. PER*t+PER-1
        constexpr int PER = NBK / CONSUMERS;
        uint32_t c[PER], tot = 0u;
#pragma unroll
        for (int k = 0; k < PER; k++) {
            c[k] = bk->cnt[PER * tid + k];
            tot += c[k];
            if (c[k] > (uint32_t)BK_MAX) s.big_bucket = 1;
        }
        const int lane = tid & 31, w = tid >> 5;
        const uint32_t incl = warp_incl_scan(tot, lane);
        if (lane == 31) s.ri[w] = (int)incl;
        csync();
        uint32_t start = incl - tot;
        for (int k = 0; k < w; k++) start += (uint32_t)s.ri[k];
#pragma unroll
        for (int k = 0; k < PER; k++) {
            bk->start[PER * tid + k] = start;  // the scatter's cursor
            start += c[k];
        }
    }
    csync();
    if (s.big_bucket) return nullptr;
    for (int i = tid; i < nk; i += CONSUMERS) {
        const uint64_t key = src[i];
        buf[atomicAdd(&bk->start[(kmax - (uint32_t)(key >> 32)) >> sh], 1u)] = key;
    }
    csync();
    // bucket b now spans [start[b] - cnt[b], start[b]) of buf
    for (int i = tid; i < nk; i += CONSUMERS) {
        const uint64_t key = buf[i];
        const int b = (int)((kmax - (uint32_t)(key >> 32)) >> sh);
        const int e = (int)bk->start[b], b0 = e - (int)bk->cnt[b];
        int rank = b0;
        for (int q = b0; q < e; q++) rank += buf[q] > key ? 1 : 0;
        src[rank] = key;
    }
    csync();
    return src;
}

// ---------------------------------------------------------------------------
// Tile sources: where the consumers' 16 elements per tile come from. Thread
// tid owns the 16 contiguous elements 16*tid .. 16*tid+15 of each tile
// (octets it*OCT_TILE + 2*tid and + 1), so a slot of kernel B's re-read is
// one 64-byte span. In registers its four 4-element chunks sit in XOR order:
// register chunk k holds chunk k ^ chunk_swz(tid). In the ring that makes the
// 128-bit shared loads of eight neighbouring threads hit eight different
// 16-byte bank groups; max and sum do not care about the order, and kernel
// A's penalty bitset stores each id at pen_bit(id), the same permutation, so a
// thread's 16 bits come out in register order.
__device__ __forceinline__ int chunk_swz(int tid) { return (tid >> 1) & 3; }
// Bit of id in kernel A's penalty bitset: chunk bits 2-3 flipped by the owner
// thread's chunk_swz (bits 5-6 of id). Same 32-bit word as id.
__device__ __forceinline__ int pen_bit(int id) { return id ^ (((id >> 5) & 3) << 2); }
// Element index of register j of thread tid in tile it.
__device__ __forceinline__ int reg_elem(int it, int tid, int j) {
    return it * TILE_ELEMS + 16 * tid + 4 * ((j >> 2) ^ chunk_swz(tid)) + (j & 3);
}

struct LdgSource {
    static constexpr bool kRegs = true;
    static constexpr bool kPick = false;  // penalized values are claimed at the row's end
    float nxt[LDG_DEPTH][16];  // tiles it+1 .. it+LDG_DEPTH in flight
    __device__ __forceinline__ void begin(const Row& R) {
#pragma unroll
        for (int d = 0; d < LDG_DEPTH; d++)
            if (d < R.ntiles) load(R, d, nxt[d]);
    }
    __device__ __forceinline__ static void load(const Row& R, int it, float* v) {
        const int tid = threadIdx.x, sw = chunk_swz(tid);
        const float* p = R.ptr + (int64_t)it * TILE_ELEMS + 16 * tid;
        if (R.vec && it + 1 < R.ntiles) {  // a full tile of a 32-byte aligned row
#pragma unroll
            for (int k = 0; k < 4; k++) ld4(p + 4 * (k ^ sw), v + 4 * k);
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int e = reg_elem(it, tid, j);
                v[j] = e < R.V ? __ldcs(R.ptr + e) : -INFINITY;
            }
        }
    }
    // tile `it` into v; the loads of tile it+LDG_DEPTH are issued before returning
    __device__ __forceinline__ void get(const Row& R, int it, float (&v)[16], Shared&) {
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] = nxt[0][j];
#pragma unroll
        for (int d = 0; d + 1 < LDG_DEPTH; d++)
#pragma unroll
            for (int j = 0; j < 16; j++) nxt[d][j] = nxt[d + 1][j];
        if (it + LDG_DEPTH < R.ntiles) load(R, it + LDG_DEPTH, nxt[LDG_DEPTH - 1]);
    }
    __device__ __forceinline__ void release() {}
    __device__ __forceinline__ uint32_t stage_addr() const { return 0u; }  // no ring (never picks up)
};

// The slow side of a ring wait: the chunk has not landed yet. Gives up at
// once after an abort, else waits (bounded) and records a timeout as one.
__device__ __noinline__ bool ring_wait_slow(uint32_t bar, uint32_t par, int* abort_flag) {
    if (*reinterpret_cast<volatile int*>(abort_flag)) return false;
    if (mbar_wait(bar, par)) return true;
    *reinterpret_cast<volatile int*>(abort_flag) = 1;
    return false;
}

// kPickable: stochastic rows with long histories pick their penalized values
// up from the ring (a separate kernel instance, so the common case's code is
// not affected by it).
template <bool kPickable>
struct TmaSource {
    static constexpr bool kRegs = false;
    static constexpr bool kPick = kPickable;
    uint32_t ring_u32;  // NSTAGE tiles (shared-window address)
    uint32_t thr_off;   // 64 * tid + 16 * chunk_swz(tid)
    uint32_t full0, empty0;
    uint32_t g;  // chunks consumed by this CTA so far
    __device__ __forceinline__ void begin(const Row&) {}
    // kMaybeLast = false: the caller knows `it` is not the row's last chunk
    // (the only partial one), so no bounds mask is needed
    template <bool kMaybeLast = true>
    __device__ __forceinline__ void get(const Row& R, int it, float (&v)[16], Shared& s) {
        const int st = (int)(g % NSTAGE);
        const uint32_t par = (g / NSTAGE) & 1u;
        // a landed chunk is valid whatever else happened; only a chunk that
        // has not landed consults the abort flag
        const bool ok = mbar_try_wait(full0 + 8u * st, par) || ring_wait_slow(full0 + 8u * st, par, &s.abort);
        const int tid = threadIdx.x;
        if (ok) {
            // chunk k ^ sw of the thread's 64 bytes: the address's bits 4-5
            // start at sw (thr_off) and are flipped by k
            const uint32_t base = ring_u32 + (uint32_t)st * TILE_BYTES + thr_off;
#pragma unroll
            for (int k = 0; k < 4; k++) lds4(base ^ (16u * k), v + 4 * k);
        }
        if (!ok || (kMaybeLast && it == R.ntiles - 1)) {  // only the last chunk of a row is partial
#pragma unroll
            for (int j = 0; j < 16; j++)
                if (!ok || reg_elem(it, tid, j) >= R.V) v[j] = -INFINITY;
        }
    }
    __device__ __forceinline__ void release() {
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(empty0 + 8u * (g % NSTAGE));
        g++;
    }
    // shared address of this thread's 64 bytes in the chunk last taken by
    // get() (valid until release())
    __device__ __forceinline__ uint32_t stage_addr() const {
        return ring_u32 + (uint32_t)(g % NSTAGE) * TILE_BYTES + thr_off;
    }
};

// ---------------------------------------------------------------------------
// Per-row set-up and finish shared by the kernels.

struct RowCtx {
    RowParams P;
    int cap, len, head;
    const int32_t* ring;
    int64_t col0;  // global id of column 0 (vocab shards; 0 otherwise)
};

// History entry i of the row as a column index of this matrix (negative or
// >= V when the id is not one of its columns).
__device__ __forceinline__ int ring_id(const RowCtx& c, int i) {
    const int64_t id = (int64_t)c.ring[(c.head + i) % c.cap] - c.col0;
    return (id >= 0 && id < 0x7FFFFFFF) ? (int)id : -1;
}

// Row parameters and history ring of `row` (no shared-memory work).
// len_raw / head_raw: the row's hist_len / hist_head entries as stored (or
// the defaults of ring_len_raw / ring_head_raw).
__device__ __forceinline__ RowCtx row_ctx_raw(const RowsArgs& a, int row, const quasar_sample_params& pr,
                                              int len_raw, int head_raw, Row& R) {
    RowCtx c;
    c.P = clamp_params(pr);
    c.cap = a.hist ? a.hist_cap : 0;
    c.len = 0;
    c.head = 0;
    c.ring = nullptr;
    c.col0 = a.col0;
    if (c.cap > 0) {
        c.ring = a.hist + (int64_t)row * c.cap;
        c.len = min(max(len_raw, 0), c.cap);
        c.head = ((head_raw % c.cap) + c.cap) % c.cap;
    }
    R.ptr = a.logits + (int64_t)row * a.ld;
    R.V = a.V;
    R.noct = (a.V + 7) >> 3;
    R.ntiles = (R.noct + OCT_TILE - 1) / OCT_TILE;
    R.vec = a.vec != 0;
    R.use_pen = c.P.rp > 1.0f && c.len > 0;
    R.rp = c.P.rp;
    R.inv_t = c.P.T > 0.0f ? __fdiv_rn(1.0f, c.P.T) : 0.0f;  // sample.c:137
    R.M = R.thr = R.inv = 0.0f;
    return c;
}

__device__ __forceinline__ bool has_len(const RowsArgs& a) { return a.hist && a.hist_cap > 0 && a.hist_len; }
__device__ __forceinline__ bool has_head(const RowsArgs& a) { return a.hist && a.hist_cap > 0 && a.hist_head; }
__device__ __forceinline__ int ring_len_raw(const RowsArgs& a, int row) { return has_len(a) ? a.hist_len[row] : a.hist_cap; }
__device__ __forceinline__ int ring_head_raw(const RowsArgs& a, int row) { return has_head(a) ? a.hist_head[row] : 0; }
__device__ __forceinline__ RowCtx row_ctx(const RowsArgs& a, int row, const quasar_sample_params& pr, Row& R) {
    return row_ctx_raw(a, row, pr, ring_len_raw(a, row), ring_head_raw(a, row), R);
}

// row_ctx plus the penalty bitset of the row's history ids (consumer threads).
// my_id: this thread's ring entry (threadIdx.x) when it is a column id, else
// -1; its logit is copied into s.tfmax[threadIdx.x] (idle in kernel A) while
// the row streams, for claim_penalized.
// Ring slot p (a raw position) holds a history entry when it is one of the
// len slots from head on.
__device__ __forceinline__ bool ring_slot_used(const RowCtx& c, int p) {
    return p - c.head + (p < c.head ? c.cap : 0) < c.len;
}
// Copies the inputs row_setup needs for `row` into shared memory (cp.async,
// one group): parameters, ring length and head, ring slots 0..CONSUMERS-1
// (raw positions, into tfmax). Rows past B are skipped.
__device__ __forceinline__ void stage_next_row(const RowsArgs& a, int row, SharedA& s) {
    const int tid = threadIdx.x;
    if (row < a.B) {
        if (a.d_params && tid < (int)(sizeof(quasar_sample_params) / 4))
            cp_async4(smem_u32(&s.nxt_pr) + 4u * tid, reinterpret_cast<const char*>(a.d_params + row) + 4 * tid);
        if (tid == 32 && has_len(a)) cp_async4(smem_u32(&s.nxt_len), a.hist_len + row);
        if (tid == 64 && has_head(a)) cp_async4(smem_u32(&s.nxt_head), a.hist_head + row);
        if (a.hist && tid < a.hist_cap)
            cp_async4(smem_u32(&s.tfmax[tid]), a.hist + (int64_t)row * a.hist_cap + tid);
    }
    cp_async_commit();
}
// A stochastic row whose history ring has more slots than there are consumer
// threads: its penalized values are picked up in the stream (from the ring
// of the bulk-copy kernel), not claimed and gathered at the row's end, where
// the stream has already pushed those logits out of L2.
__device__ __forceinline__ bool picks_in_stream(const RowCtx& c, const Row& R) {
    return R.use_pen && c.P.T > 0.0f && c.cap > CONSUMERS;
}

// staged: stage_next_row ran for this row. my_id: the column id in this
// thread's ring slot (threadIdx.x) when that slot holds an entry, else -1;
// its logit is copied into s.tfmax[threadIdx.x] (idle in kernel A) while the
// row streams, for claim_penalized.
// pick_tma: the row is streamed through the bulk-copy ring, so a stochastic
// row with a long history (more ring slots than consumer threads) picks its
// penalized values up from the ring while it streams (pick_penalized) and
// needs no staged logit.
template <bool kPickTma>
__device__ __forceinline__ RowCtx row_setup(const RowsArgs& a, int row, Row& R, uint32_t* bits, SharedA& s,
                                            int& my_id, bool staged) {
    const int tid = threadIdx.x;
    if (staged) {
        cp_async_wait_all();
        csync();  // every thread's copies have landed
    }
    const quasar_sample_params pr = a.d_params ? (staged ? s.nxt_pr : a.d_params[row]) : a.h_params;
    const int len_raw = staged ? (has_len(a) ? s.nxt_len : a.hist_cap) : ring_len_raw(a, row);
    const int head_raw = staged ? (has_head(a) ? s.nxt_head : 0) : ring_head_raw(a, row);
    const RowCtx c = row_ctx_raw(a, row, pr, len_raw, head_raw, R);
    my_id = -1;
    if (R.use_pen) {
        for (int p = tid; p < c.cap; p += CONSUMERS) {
            if (!ring_slot_used(c, p)) continue;
            const int raw = (staged && p == tid) ? __float_as_int(s.tfmax[tid]) : c.ring[p];
            const int64_t id64 = (int64_t)raw - c.col0;
            const int id = (id64 >= 0 && id64 < a.V) ? (int)id64 : -1;
            if (id >= 0) {
                atomicOr(&bits[id >> 5], 1u << (pen_bit(id) & 31));
                if (p == tid && !(kPickTma && picks_in_stream(c, R))) {
                    my_id = id;
                    cp_async4(smem_u32(&s.tfmax[tid]), R.ptr + id);
                }
            }
        }
        cp_async_commit();
    }
    if (threadIdx.x == 0) s.npen = 0;
    csync();
    return c;
}

__device__ __forceinline__ void clear_bits(const RowsArgs& a, const RowCtx& c, const Row& R, uint32_t* bits) {
    if (R.use_pen) {
        for (int i = threadIdx.x; i < c.len; i += CONSUMERS) {
            const int id = ring_id(c, i);
            if (id >= 0 && id < a.V) bits[id >> 5] = 0u;
        }
    }
}

// The row's id, report, PRNG state and ring append (one thread).
__device__ __forceinline__ void write_row(const RowsArgs& a, int row, const RowCtx& c, int chosen, int nkept,
                                          float p, float inv, int path, uint64_t st_rng) {
    if (c.P.T > 0.0f) a.rng[row] = st_rng;
    a.out[row] = chosen;
    if (a.diag) {
        quasar_pick_diag d;
        d.n_kept = nkept;
        d.p_chosen = p;
        d.inv_sum = inv;
        d.path = path;
        a.diag[row] = d;
    }
    if (a.record && c.cap > 0 && a.hist_len && a.hist_head && chosen >= 0) {
        int32_t* wring = a.hist + (int64_t)row * c.cap;
        if (c.len < c.cap) {  // sample.c:85-87
            wring[(c.head + c.len) % c.cap] = chosen;
            a.hist_len[row] = c.len + 1;
        } else {              // sample.c:88-90
            wring[c.head] = chosen;
            a.hist_head[row] = (c.head + 1) % c.cap;
        }
    }
}

// Clears the bitset and writes the row's outputs from the result slots.
__device__ __forceinline__ void row_finish(const RowsArgs& a, int row, const RowCtx& c, const Row& R,
                                           uint32_t* bits, int path, uint64_t st_rng, Shared& s) {
    const int chosen = *reinterpret_cast<volatile int*>(&s.abort) ? -1 : s.res_id;
    clear_bits(a, c, R, bits);
    csync();
    if (threadIdx.x == 0) write_row(a, row, c, chosen, s.res_nc, s.res_p, R.inv, path, st_rng);
    csync();
}

// Runs body(v, it) over every tile of the row. Register loads: two buffers
// alternate, the next tile's loads in flight while one is processed, with
// unchecked 256-bit loads for every tile but the last. Ring: tiles come from
// shared memory and the stage is released as soon as it is in registers.
// kBodyReleases: the body releases each ring chunk itself (after reading
// more of it than the registers get() filled).
template <bool kBodyReleases = false, class Src, class F>
__device__ __forceinline__ void stream_tiles(const Row& R, Src& src, Shared& s, F& body) {
    if constexpr (Src::kRegs) {
        float va[16], vb[16];
        Src::load(R, 0, va);
        for (int it = 0; it < R.ntiles; it += 2) {
            if (it + 1 < R.ntiles) Src::load(R, it + 1, vb);
            body(va, it, std::true_type());
            if (it + 2 < R.ntiles) Src::load(R, it + 2, va);
            if (it + 1 < R.ntiles) body(vb, it + 1, std::true_type());
        }
    } else {
        // every chunk but the last is full: its checks are compile-time
        for (int it = 0; it + 1 < R.ntiles; it++) {
            float v[16];
            src.template get<false>(R, it, v, s);
            if constexpr (!kBodyReleases) src.release();
            body(v, it, std::false_type());
        }
        float v[16];
        src.template get<true>(R, R.ntiles - 1, v, s);
        if constexpr (!kBodyReleases) src.release();
        body(v, R.ntiles - 1, std::true_type());
    }
}

// Streaming form of exclude_penalized: the thread's 16 bitset bits select
// -inf for its penalized elements (one select per element; a 16-entry table
// of float4 {0, -inf} added per nibble cost four 16-byte shared loads per
// thread and was slower: config 3 0.526 -> 0.521 ms, config 5 2.54 -> 2.52
// ms); warps with no penalized element in the tile skip it.
// kCheck = false: tile it is not the row's last, so its octets are in range
template <bool kCheck = true>
__device__ __forceinline__ void mask_penalized(const Row& R, const uint8_t* bits8, float* v, int it) {
    // the thread's 16 bits (pen_bit order = register order), one 16-bit load
    const int o0 = it * OCT_TILE + 2 * (int)threadIdx.x;
    const uint32_t m = (!kCheck || o0 < R.noct) ? *reinterpret_cast<const uint16_t*>(bits8 + o0) : 0u;
    if (__any_sync(FULL, m != 0u)) {
#pragma unroll
        for (int j = 0; j < 16; j++)
            if ((m >> j) & 1u) v[j] = -INFINITY;
    }
}

// mask_penalized plus the pick-up of the penalized values (sample.c:118-128)
// from the ring chunk the tile came from (`stage`: this thread's 64 bytes,
// chunk k of register chunk k at stage ^ 16k, see TmaSource::get): each
// penalized element's raw logit is listed with its column; the list is
// penalized, scaled and summed at the row's end by every thread together
// (finish_picked), not here, where only the lanes holding a penalized element
// would do the work (about 7 of 32 at 2048 history ids: the arithmetic in
// this loop cost 0.9 ms of a 2.7 ms config-5 call). The thread's 16 bitset
// bits are cleared once read, so the bitset is all zero at the row's end.
// Every column is streamed once, so every distinct history id is picked up
// once.
template <bool kCheck>
__device__ __forceinline__ void pick_penalized(const Row& R, uint8_t* bits8, float* v, int it, uint32_t stage,
                                               int2* pen, int* npen) {
    const int o0 = it * OCT_TILE + 2 * (int)threadIdx.x;
    const uint32_t mb = (!kCheck || o0 < R.noct) ? *reinterpret_cast<const uint16_t*>(bits8 + o0) : 0u;
    if (__any_sync(FULL, mb != 0u)) {
        // a select per element, as mask_penalized (with 2048 history ids
        // nearly every warp takes this branch on every tile)
#pragma unroll
        for (int j = 0; j < 16; j++)
            if ((mb >> j) & 1u) v[j] = -INFINITY;
        // list positions: one shared atomic per warp for all of its picks
        // (the whole warp is here: the branch condition is warp-uniform)
        const int cnt = __popc(mb);
        const int incl = warp_incl_scan(cnt, (int)threadIdx.x & 31);
        int pos = 0;
        if ((threadIdx.x & 31) == 31) pos = atomicAdd(npen, incl);
        pos = __shfl_sync(FULL, pos, 31) + incl - cnt;
        if (mb) {
            *reinterpret_cast<uint16_t*>(bits8 + o0) = 0;
            uint32_t b = mb;
            do {
                const int j = __ffs(b) - 1;
                b &= b - 1u;
                float x;
                asm volatile("ld.shared.f32 %0, [%1];" : "=f"(x) : "r"((stage ^ (16u * (uint32_t)(j >> 2))) + 4u * (uint32_t)(j & 3)));
                pen[pos++] = make_int2(reg_elem(it, (int)threadIdx.x, j), __float_as_int(x));  // raw logit
            } while (b);
        }
    }
}

// Penalized elements are left out of the stream (read as -inf); their
// penalized values re-enter through claim_penalized.
__device__ __forceinline__ void exclude_penalized(const Row& R, const uint8_t* bits8, float* v, int o0, int o1) {
    const uint32_t m0 = o0 < R.noct ? bits8[o0] : 0u;
    const uint32_t m1 = o1 < R.noct ? bits8[o1] : 0u;
    if (m0 | m1) {
#pragma unroll
        for (int k = 0; k < 8; k++) {
            if (m0 & (1u << k)) v[k] = -INFINITY;
            if (m1 & (1u << k)) v[8 + k] = -INFINITY;
        }
    }
}

// Hands every distinct in-range history id of the row to f(id, penalized
// logit) (sample.c:118-128) exactly once: the thread whose atomic clears the
// id's bit owns it. Leaves the bitset all zero. Callers synchronise first so
// that no thread still reads the bitset.
// Ring slot threadIdx.x comes from row_setup (my_id, logit staged in
// s.tfmax); slots past the first CONSUMERS are read here.
template <class F>
__device__ __forceinline__ void claim_penalized(const RowCtx& c, const Row& R, uint32_t* bits, int my_id,
                                                const Shared& s, F&& f) {
    cp_async_wait_all();  // this thread's staged logit
    for (int p = threadIdx.x; p < c.cap; p += CONSUMERS) {
        const bool first = p == (int)threadIdx.x;
        int id = my_id;
        if (!first) {
            if (!ring_slot_used(c, p)) continue;
            const int64_t id64 = (int64_t)c.ring[p] - c.col0;
            id = (id64 >= 0 && id64 < R.V) ? (int)id64 : -1;
        }
        if (id >= 0 && id < R.V) {
            const uint32_t bit = 1u << (pen_bit(id) & 31);
            if (atomicAnd(&bits[id >> 5], ~bit) & bit)
                f(id, penalize(first ? s.tfmax[threadIdx.x] : __ldg(R.ptr + id), R.rp));
        }
    }
}

// ---------------------------------------------------------------------------
// Kernel A, one row: greedy rows are finished here; a stochastic row is
// streamed once and leaves its summary in the workspace for kernel B: max M,
// 1/sum, the per-thread maxima, the tile-max table with its checkpoint
// anchors, and the list of penalized ids with their scaled logits.
//
// Tile-max table: one byte per thread and slot (a slot is g consecutive
// tiles, g = 1 up to 40 tiles), the slot max's deficit below the thread's
// running max m_j at the slot's end. The running max at the checkpoint slots
// (ck_slot, kept in anc_s) is stored as a deficit below the thread's
// final max, so slot j's max is bounded by final - (anchor deficit of the
// first checkpoint >= j + slot deficit)/8: tight for early slots too.
template <class Src>
__device__ __forceinline__ void stream_row(const RowsArgs& a, int row, Src& src, uint32_t* bits, float* anc_s,
                                           SharedA& s, bool staged) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint8_t* bits8 = reinterpret_cast<const uint8_t*>(bits);
    Row R;
    int my_id;
    const RowCtx c = row_setup<Src::kPick>(a, row, R, bits, s, my_id, staged);
    const bool pick = Src::kPick && picks_in_stream(c, R);
    const RowParams& P = c.P;
    src.begin(R);

    if (P.T <= 0.0f) {
        // ---- greedy: penalized argmax, first index on ties ----
        float bv = -INFINITY;
        int bi = 0x7FFFFFFF;
        for (int it = 0; it < R.ntiles; it++) {
            float v[16];
            src.get(R, it, v, s);
            if (R.use_pen) mask_penalized(R, bits8, v, it);
            src.release();
            float mt = v[0];
#pragma unroll
            for (int j = 1; j < 16; j++) mt = fmaxf(mt, v[j]);
            if (mt > bv) {  // strictly larger: the first index holding mt wins
                int e = 0x7FFFFFFF;  // registers are not in index order
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (v[j] == mt) e = min(e, reg_elem(it, tid, j));
                bv = mt;
                bi = e;
            }
        }
        if (R.use_pen) {
            csync();
            // penalized ids compete by (value desc, id asc); -inf never wins,
            // so an all -inf row still gives id 0 (sample.c:130-134)
            claim_penalized(c, R, bits, my_id, s, [&](int id, float l) {
                if (l > bv || (l == bv && id < bi && l > -INFINITY)) {
                    bv = l;
                    bi = id;
                }
            });
        }
        stage_next_row(a, row + (int)gridDim.x, s);  // s.tfmax is free again
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(FULL, bv, o);
            const int oi = __shfl_xor_sync(FULL, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            s.rf[warp] = bv;
            s.ri[warp] = bi;
        }
        csync();
        if (tid == 0) {
            float best = s.rf[0];
            int besti = s.ri[0];
            for (int w = 1; w < CWARPS; w++)
                if (s.rf[w] > best || (s.rf[w] == best && s.ri[w] < besti)) {
                    best = s.rf[w];
                    besti = s.ri[w];
                }
            s.res_id = (besti == 0x7FFFFFFF || besti >= a.V) ? 0 : besti;
            s.res_nc = 0;
            s.res_p = 1.0f;
            // a vocab shard: its best (value, column) joins the merge; -1 when
            // every value is -inf (the merge then falls back to id 0)
            if (a.shard_stats)
                a.shard_stats[row] = quasar_shard_stat{best, (besti == 0x7FFFFFFF || besti >= a.V) ? -1 : besti,
                                                       0.0};
        }
        csync();
        if (a.shard_stats) {
            clear_bits(a, c, R, bits);
            csync();
            return;
        }
        row_finish(a, row, c, R, bits, QUASAR_PATH_GREEDY, 0, s);
        return;
    }

    // ---- one streaming pass: max, online window sum, tile maxima ----
    const int g = (R.ntiles + TMAX_TILES - 1) / TMAX_TILES;  // tiles per table slot
    uint32_t* tmax32 = reinterpret_cast<uint32_t*>(a.work_tmax + (int64_t)row * TMAX_BYTES);
    uint32_t tword = 0u;  // four slot bytes of this thread, stored together (tbl_off layout)
    float slotmax = -INFINITY;
    const f32x2 inv_t2 = pack2(R.inv_t, R.inv_t);
    // m: the thread's running max (tile table, anchors, kernel B). S sums
    // exp(sc - m_ref) against a reference that moves only when a tile max
    // passes it by more than REF_SLACK nats, so the double-precision rescale
    // runs about once per row instead of at every new max; terms stay below
    // e^REF_SLACK, far inside fp32 range. Both start finite (an all -inf
    // stretch adds exp(-inf) = 0).
    float m = -FLT_MAX, m_ref = -FLT_MAX;
    double S = 0.0;
    int next_ck = ck_slot(0), ck = 0;  // next checkpoint slot and its index
    // g1: one tile per table slot (compile-time); last: std::true_type when
    // `it` may be the row's last tile
    // pen: the row has penalized ids (compile-time, like g1)
    // pen: 0 no penalized ids, 1 masked in the stream and claimed at the
    // row's end, 2 masked and picked up in the stream (ring kernel only)
    auto run = [&](auto g1, auto pen) {
        constexpr bool kG1 = decltype(g1)::value;
        constexpr bool kPen = decltype(pen)::value == 1;
        constexpr bool kPick = decltype(pen)::value == 2;
        auto body = [&](float (&v)[16], int it, auto last) {
            constexpr bool kMaybeLast = decltype(last)::value;
            if constexpr (kPen) mask_penalized<kMaybeLast>(R, bits8, v, it);
            if constexpr (kPick) {
                pick_penalized<kMaybeLast>(R, reinterpret_cast<uint8_t*>(bits), v, it, src.stage_addr(),
                                           a.work_pen + (int64_t)row * a.hist_cap, &s.npen);
                src.release();
            }
            // sample.c:142: sc = l * inv_t, rounded exactly like the reference
            // (packed pairs: each lane is the same IEEE multiply)
            f32x2 sc2[8];
            float sc[16];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                sc2[j] = mul2(pack2(v[2 * j], v[2 * j + 1]), inv_t2);
                unpack2(sc2[j], sc[2 * j], sc[2 * j + 1]);
            }
            const float mt = fmaxf(max3(max3(sc[0], sc[1], sc[2]), max3(sc[3], sc[4], sc[5]),
                                        max3(sc[6], sc[7], sc[8])),
                                   max3(max3(sc[9], sc[10], sc[11]), max3(sc[12], sc[13], sc[14]), sc[15]));
            m = fmaxf(m, mt);
            if (mt > m_ref + REF_SLACK) {
                S *= exp((double)m_ref - (double)mt);
                m_ref = mt;
            }
            {
                // sample.c:148 against the reference: x = sc - m_ref, then the term
                f32x2 e[8];
                const f32x2 nm2 = pack2(-m_ref, -m_ref);
#pragma unroll
                for (int j = 0; j < 8; j++) {
#if QS_SUM_EXP == 3
                    e[j] = exp_fast2(add2(sc2[j], nm2));
#elif QS_SUM_EXP == 2 || QS_SUM_EXP == 4
                    if (QS_SUM_EXP == 4 && (j & 1) == 0) {
                        e[j] = exp_fast2(add2(sc2[j], nm2));
                    } else {
                        float x0, x1;
                        unpack2(add2(sc2[j], nm2), x0, x1);
                        e[j] = exp_poly2(x0, x1);
                    }
#else
                    e[j] = pack2(sum_term_exp(__fsub_rn(sc[2 * j], m_ref)),
                                 sum_term_exp(__fsub_rn(sc[2 * j + 1], m_ref)));
#endif
                }
#pragma unroll
                for (int w = 4; w > 0; w >>= 1)
#pragma unroll
                    for (int j = 0; j < w; j++) e[j] = add2(e[j], e[j + w]);
                float e0, e1;
                unpack2(e[0], e0, e1);
                S += (double)(e0 + e1);
            }
            if constexpr (kG1) {
                tword |= deficit_byte(m, mt) << (8 * (it & 3));
                if ((it & 3) == 3 || (kMaybeLast && it == R.ntiles - 1)) {
                    tmax32[(it >> 2) * CONSUMERS + tid] = tword;
                    tword = 0u;
                }
                if (it == next_ck) {
                    anc_s[ck * CONSUMERS + tid] = m;
                    next_ck = ++ck < NCK ? ck_slot(ck) : -1;
                }
            } else {
                slotmax = fmaxf(slotmax, mt);
                if (it % g == g - 1 || (kMaybeLast && it == R.ntiles - 1)) {
                    const int sl = it / g;
                    tword |= deficit_byte(m, slotmax) << (8 * (sl & 3));
                    if ((sl & 3) == 3 || (kMaybeLast && it == R.ntiles - 1)) {
                        tmax32[(sl >> 2) * CONSUMERS + tid] = tword;
                        tword = 0u;
                    }
                    if (sl == next_ck) {
                        anc_s[ck * CONSUMERS + tid] = m;
                        next_ck = ++ck < NCK ? ck_slot(ck) : -1;
                    }
                    slotmax = -INFINITY;
                }
            }
        };
        stream_tiles<kPick>(R, src, s, body);
    };
    using P0 = std::integral_constant<int, 0>;
    using P1 = std::integral_constant<int, 1>;
    using P2 = std::integral_constant<int, Src::kPick ? 2 : 1>;  // (pick is false without a pickable ring)
    if (g == 1) {
        if (pick) run(std::true_type(), P2());
        else if (R.use_pen) run(std::true_type(), P1());
        else run(std::true_type(), P0());
    } else {
        if (pick) run(std::false_type(), P2());
        else if (R.use_pen) run(std::false_type(), P1());
        else run(std::false_type(), P0());
    }
    if (pick) {
        csync();  // the picked list is complete
        // its raw logits penalized exactly (IEEE divide / multiply) and
        // scaled, joining the running max and sum (against m_ref, as the
        // streamed terms do); the list keeps the scaled values for kernel B
        int2* pen = a.work_pen + (int64_t)row * a.hist_cap;
        const int np = min(s.npen, a.hist_cap);
        for (int i = tid; i < np; i += CONSUMERS) {
            const int2 e = pen[i];
            const float sc = __fmul_rn(penalize(__int_as_float(e.y), R.rp), R.inv_t);
            pen[i].y = __float_as_int(sc);
            m = fmaxf(m, sc);
            if (sc > m_ref + REF_SLACK) {
                S = S * exp((double)m_ref - (double)sc) + 1.0;
                m_ref = sc;
            } else if (sc > -INFINITY) {
                S += (double)exp_fast(__fsub_rn(sc, m_ref));  // like the streamed terms
            }
        }
    }
    if (R.use_pen && !pick) {
        csync();
        // the penalized elements join the running max and sum exactly, and
        // are listed for kernel B
        int2* pen = a.work_pen + (int64_t)row * a.hist_cap;
        claim_penalized(c, R, bits, my_id, s, [&](int id, float l) {
            const float sc = __fmul_rn(l, R.inv_t);
            pen[atomicAdd(&s.npen, 1)] = make_int2(id, __float_as_int(sc));
            m = fmaxf(m, sc);
            if (sc > m_ref + REF_SLACK) {
                S = S * exp((double)m_ref - (double)sc) + 1.0;
                m_ref = sc;
            } else if (sc > -INFINITY) {
                S += (double)exp_fast(__fsub_rn(sc, m_ref));  // like the streamed terms
            }
        });
    }
    stage_next_row(a, row + (int)gridDim.x, s);  // s.tfmax is free again
    a.work_tfmax[(int64_t)row * CONSUMERS + tid] = m;
    {
        // anchor deficits, four per word (tbl_off), stored as whole words;
        // checkpoints past the last slot stay 0 (kernel B ignores them)
        const int nsl = (R.ntiles + g - 1) / g;
        uint32_t* anc = reinterpret_cast<uint32_t*>(a.work_anc + (int64_t)row * ANC_BYTES);
        uint32_t w[(NCK + 3) / 4] = {};
#pragma unroll
        for (int k = 0; k < NCK; k++)
            if (ck_slot(k) < nsl) w[k >> 2] |= (uint32_t)tile_deficit(m, anc_s[k * CONSUMERS + tid]) << (8 * (k & 3));
#pragma unroll
        for (int q = 0; q < (NCK + 3) / 4; q++) anc[q * CONSUMERS + tid] = w[q];
    }
    const float M = block_max_f(m, s);
    const double contrib = S > 0.0 ? S * exp((double)m_ref - (double)M) : 0.0;
    const double Stot = block_sum_d(contrib, s);
    if (tid == 0) {
        a.work_info[row] = make_float4(M, __double2float_rn(1.0 / Stot), __int_as_float(s.npen), 0.0f);
        if (a.shard_stats) a.shard_stats[row] = quasar_shard_stat{M, -1, Stot};
    }
}

// ---------------------------------------------------------------------------
// Kernel B, one stochastic row: cuts and draw from the row summary.
//
// Candidate path. The kept prefix lies above a threshold known once M is:
// min_p -> sc >= M + ln(min_p) - 0.01 (every p >= min_p * p_max clears it);
// top_k -> the k-th largest per-thread max less a tie margin (k distinct
// elements reach it). Only thread-slots whose bound clears the threshold are
// read again; penalized ids come from kernel A's list. Rows it cannot bound
// take the exact select path.

// Global max M and inv = (float)(1/sum) of a row split into vocab shards,
// from the shards' (max, sum against that max) pairs - the same combination
// as the one over threads inside a shard. nb: rows per shard in all_stats
// ([G][nb]). Called by whole warps: the lanes read the shards' pairs
// together and combine them by butterfly reductions, which leave the same
// bits in every lane (each step adds the same two values), so every kernel
// and rank that combines a row's pairs gets the same M and inv.
__device__ __forceinline__ void shard_norm(const RowsArgs& a, int row, int nb, float& M, float& inv) {
    const int lane = threadIdx.x & 31;
    float mx = -INFINITY;
    for (int g = lane; g < a.shard_G; g += 32) mx = fmaxf(mx, a.all_stats[(int64_t)g * nb + row].max);
    mx = warp_max(mx);
    double S = 0.0;
    for (int g = lane; g < a.shard_G; g += 32) {
        const quasar_shard_stat st = a.all_stats[(int64_t)g * nb + row];
        if (st.max > -INFINITY) S += st.sum * exp((double)st.max - (double)mx);
    }
    S = warp_sum(S);
    M = mx;
    inv = __double2float_rn(1.0 / S);
}

// The exact top-k of a vocab shard, for a row whose bound let more elements
// through than its candidate buffer holds (the k-th largest per-thread
// maximum bounds the shard's top k loosely when k is near the thread count,
// or when many elements tie): the k-th largest key (p desc, global id asc)
// over every element of the shard's 30-nat window is found by a radix
// select (eight passes of 8 bits over the 64-bit keys, p recomputed in each
// pass), and the n = min(k, window elements) elements whose keys reach it
// are written as (scaled value bits, column) entries, unordered, to
// raw[0, n) (end = 0) or raw[end - n, end). Returns n. One warp; hist: 256
// words of shared memory apart from raw. Rare (a slow path of one warp over
// the whole shard).
__device__ __noinline__ int shard_topk_exact(const Row& R, const uint32_t* bits, const int2* pen, int npen,
                                             int64_t col0, int k, uint64_t* raw, int end, uint32_t* hist) {
    const int lane = threadIdx.x & 31;
    // every window element once: penalized columns with their listed values
    auto each = [&](auto&& f) {
        for (int e = lane; e < R.V; e += 32) {
            if ((bits[e >> 5] >> (e & 31)) & 1u) continue;
            const float sc = __fmul_rn(__ldg(R.ptr + e), R.inv_t);  // sample.c:142
            if (sc >= R.thr) f(sc, e);
        }
        for (int i = lane; i < npen; i += 32) {
            const int2 pe = pen[i];
            const float sc = __int_as_float(pe.y);
            if (pe.x >= 0 && pe.x < R.V && sc >= R.thr) f(sc, pe.x);
        }
    };
    auto key_of = [&](float sc, int e) {
        return ((uint64_t)p_key(sc, R.M, R.thr, R.inv) << 32) | (uint32_t)(~(uint32_t)(col0 + e));
    };
    uint64_t prefix = 0ull;
    uint32_t need = (uint32_t)k;  // rank of the wanted key among those matching prefix
    int n = k;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int i = lane; i < 256; i += 32) hist[i] = 0u;
        __syncwarp();
        const uint64_t hi = shift == 56 ? 0ull : ~0ull << (shift + 8);
        each([&](float sc, int e) {
            const uint64_t key = key_of(sc, e);
            if ((key & hi) == prefix) atomicAdd(&hist[(uint32_t)(key >> shift) & 255u], 1u);
        });
        __syncwarp();
        // bins in descending order, eight per lane: lane l holds 255 - 8l - j
        uint32_t c[8], t = 0u;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            c[j] = hist[255 - 8 * lane - j];
            t += c[j];
        }
        const uint32_t incl = warp_incl_scan(t, lane), excl = incl - t;
        if (shift == 56) {
            const int total = (int)__shfl_sync(FULL, incl, 31);  // window elements
            if (total <= k) {  // all of them (prefix 0: every key)
                n = total;
                __syncwarp();
                break;
            }
        }
        const bool mine = excl < need && incl >= need;
        int bin = 0;
        uint32_t above = 0u;
        if (mine) {
            uint32_t acc = excl;
            for (int j = 0; j < 8; j++) {
                if (acc + c[j] >= need) {
                    bin = 255 - 8 * lane - j;
                    above = acc;
                    break;
                }
                acc += c[j];
            }
        }
        const int src = max(__ffs(__ballot_sync(FULL, mine)) - 1, 0);
        bin = __shfl_sync(FULL, bin, src);
        above = __shfl_sync(FULL, above, src);
        prefix |= (uint64_t)bin << shift;
        need -= above;
        __syncwarp();
    }
    // the keys at or above the k-th (keys are distinct: exactly n)
    uint64_t* out = raw + (end > 0 ? end - n : 0);
    if (lane == 0) hist[0] = 0u;
    __syncwarp();
    each([&](float sc, int e) {
        if (key_of(sc, e) >= prefix) {
            const uint32_t pos = atomicAdd(&hist[0], 1u);
            if (pos < (uint32_t)n) out[pos] = ((uint64_t)__float_as_uint(sc) << 32) | (uint32_t)e;
        }
    });
    __syncwarp();
    return n;
}

// kLongPen: histories longer than CONSUMERS slots (a separate kernel
// instance: the penalized list is staged in shared memory).
// kShard: the candidate kernel of a vocab shard (quasar_shard_candidates),
// also an instance of its own.
template <bool kLongPen, bool kShard>
__device__ __forceinline__ void finish_row(const RowsArgs& a, int row, uint64_t* buf, uint32_t* bits,
                                           Buckets* bk, uint16_t* qlist, Shared& s) {
    const int tid = threadIdx.x, lane = tid & 31;
    const uint8_t* bits8 = reinterpret_cast<const uint8_t*>(bits);
    // every global load of the row - parameters, ring state and kernel A's
    // summary - issued together (a greedy row's summary loads go unused)
    const quasar_sample_params pr = a.d_params ? a.d_params[row] : a.h_params;
    Row R;
    const RowCtx c = row_ctx(a, row, pr, R);
    const RowParams& P = c.P;
    const float4 info = a.work_info[row];
    const float m = a.work_tfmax[(int64_t)row * CONSUMERS + tid];  // this thread's max in kernel A
    const int g = (R.ntiles + TMAX_TILES - 1) / TMAX_TILES;
    const int nsl = (R.ntiles + g - 1) / g;
    const uint8_t* tmax = a.work_tmax + (int64_t)row * TMAX_BYTES;
    const uint8_t* anc = a.work_anc + (int64_t)row * ANC_BYTES;
    constexpr int DW = TMAX_TILES / 4, EW = (NCK + 3) / 4;
    uint32_t dw[DW], ew[EW];  // four slots per word (tbl_off)
#pragma unroll
    for (int q = 0; q < DW; q++)
        dw[q] = 4 * q < nsl ? reinterpret_cast<const uint32_t*>(tmax)[q * CONSUMERS + tid] : 0xFFFFFFFFu;
#pragma unroll
    for (int q = 0; q < EW; q++) ew[q] = reinterpret_cast<const uint32_t*>(anc)[q * CONSUMERS + tid];
    const int2* pen = a.work_pen + (int64_t)row * a.hist_cap;
    const int2 pen0 = tid < a.hist_cap ? pen[tid] : make_int2(0, 0);  // used only if tid < npen
    uint64_t st_rng = a.rng ? a.rng[row] : 0ull;
    // kernel A's abort word (read where the row is written)
    const int aborted = tid == 0 ? *reinterpret_cast<volatile int*>(a.work_abort) : 0;
    constexpr bool shard = kShard;  // a vocab shard: emit candidates, no draw
    uint64_t* cand = shard ? a.shard_cand + (int64_t)row * a.shard_k : nullptr;
    if (!(pr.temperature > 0.0f)) {
        // greedy: finished by kernel A; a shard contributes its best column
        if (shard && tid == 0) {
            const quasar_shard_stat st = a.all_stats[(int64_t)a.shard_rank * a.B + row];
            cand[0] = aborted ? SHARD_OVERFLOW
                    : st.best >= 0 ? ((uint64_t)ord_key(st.max) << 32) | (uint32_t)(~(uint32_t)(a.col0 + st.best))
                                   : 0ull;
            for (int i = 1; i < a.shard_k; i++) cand[i] = 0ull;
        }
        return;
    }
    // the bitset starts empty (shared memory is not cleared between CTAs);
    // the loads above are in flight meanwhile
    for (int i = tid; i < a.nwords; i += CONSUMERS) bits[i] = 0u;
    R.M = info.x;
    R.inv = info.y;
    if (shard) shard_norm(a, row, a.B, R.M, R.inv);  // the row's global max and 1/sum
    R.thr = __fsub_rn(R.M, 30.0f);
    // (an aborted kernel A leaves stale summaries: keep every index in range)
    const int npen = min(max(__float_as_int(info.z), 0), a.hist_cap);
    R.use_pen = npen > 0;
    // A list longer than one entry per thread (and at most half of buf) is
    // read twice below: it is copied once into the bottom of buf
    // (asynchronous copies, all in flight together), where the candidates
    // appended from the top never reach it.
    const bool pen_staged = kLongPen && npen > CONSUMERS && npen <= CAP / 2;
    const int2* pen_s = reinterpret_cast<const int2*>(buf);
    if (pen_staged) {
        for (int i = tid; i < npen; i += CONSUMERS) cp_async8(smem_u32(buf + i), pen + i);
        cp_async_commit();
    }
    s.tfmax[tid] = m;
    if (tid == 0) s.ncand = 0;
    if (pen_staged) cp_async_wait_all();
    csync();  // the bitset is clear (and the staged list has landed)
    // bitset of the penalized ids: re-reads leave them out, the select path
    // penalizes them (both come after barriers below)
    for (int i = tid; i < npen; i += CONSUMERS) {
        const int id = (pen_staged ? pen_s[i] : (i == tid ? pen0 : pen[i])).x;
        if (id >= 0 && id < R.V) atomicOr(&bits[id >> 5], 1u << (id & 31));
    }

    const double u = rng_unit(&st_rng);  // sample.c:173: one step per stochastic row
    int path = QUASAR_PATH_SELECT;
    bool done = false;
    const bool by_minp = P.min_p > 0.0f;
    const bool by_topk = P.top_k > 0 && P.top_k <= TOPK_MAX;
    // (a shard emits k candidates per row: its rows need 1 <= top_k <= k)
    // A vocab shard can stand for its part of a row when its k best keys
    // cover the row's top_k (top_k <= k), or when it sends every key at or
    // above the min-p threshold of the global max (at most k of them: more
    // are reported as an overflow, see below).
    const bool shard_topk = by_topk && P.top_k <= a.shard_k;
    // A row cut by top-p alone: when the per-thread maxima (each a real
    // element) above some value already carry the top-p mass, the kept
    // prefix lies above that value and the candidate path takes the row
    // (topp_floor); otherwise the select path.
    float tau_p = -INFINITY;
    bool by_topp = false;
    if (!kShard && !by_minp && !by_topk && P.top_p < 1.0f && !(a.flags & QUASAR_FLAG_EXACT_SELECT)) {
        csync();  // every thread's max is in s.tfmax
        tau_p = topp_floor(P.top_p, R, s, reinterpret_cast<uint64_t*>(bk));
        by_topp = tau_p > -INFINITY;
    }
    if (!(a.flags & QUASAR_FLAG_EXACT_SELECT) && (by_minp || by_topk || by_topp) &&
        (!shard || shard_topk || by_minp)) {
        float tau = tau_p;
        // (logf is within a few ulp: far inside the 0.01 margin)
        if (by_minp) tau = __fadd_rn(R.M, logf(fminf(P.min_p, 1.0f)) - 0.01f);
        if (by_topk) {
            csync();  // every thread's max is in s.tfmax
            tau = fmaxf(tau, topk_floor(P.top_k, s, reinterpret_cast<uint64_t*>(bk)));  // bk is free until the sort
        }
        const float lo = fmaxf(tau, R.thr);
        // qualifying thread-slots -> a shared list (its own area), so the
        // re-reads spread over all threads; positions from a block scan
        // A slot qualifies when thread max - (anchor + slot deficit)/8 >= lo,
        // i.e. anchor + deficit <= X = floor(8 (max - lo)) (+1 of slack, so
        // no qualifying slot is missed); four slots per byte-SIMD compare.
        // Anchors of checkpoints past the last slot were never written: the
        // thread's final max is the anchor there (deficit 0).
        uint32_t keep0 = 0u, keep1 = 0u;
#pragma unroll
        for (int k = 0; k < NCK; k++)
            if (ck_slot(k) < nsl) (k < 4 ? keep0 : keep1) |= 255u << (8 * (k & 3));
        const uint32_t ea = ew[0] & keep0, eb = ew[1] & keep1;
        const float xd = __fmul_ru(__fsub_ru(m, lo), 8.0f);
        const int X = !(xd < 1000.0f) ? 1000 : (xd < -1.0f ? -1 : (int)floorf(xd) + 1);  // NaN -> 1000
        auto thr = [&](uint32_t ek) {  // slot bytes <= X - ek qualify; -1: none
            const int tq = X - (int)ek;
            return tq < 0 ? -1 : (tq > 255 ? 255 : tq);
        };
        uint64_t qmask = 0ull;
#pragma unroll
        for (int q = 0; q < DW; q++) {
            const uint32_t d4 = dw[q];
            uint32_t r;
            if (q == 0) {  // slots 0-1: checkpoint 0 (slot 1); slots 2-3: checkpoint 1 (slot 3)
                const int t0 = thr(ea & 255u), t1 = thr((ea >> 8) & 255u);
                r = (t0 >= 0 && (d4 & 255u) <= (uint32_t)t0 ? 1u : 0u) |
                    (t0 >= 0 && ((d4 >> 8) & 255u) <= (uint32_t)t0 ? 2u : 0u) |
                    (t1 >= 0 && ((d4 >> 16) & 255u) <= (uint32_t)t1 ? 4u : 0u) |
                    (t1 >= 0 && (d4 >> 24) <= (uint32_t)t1 ? 8u : 0u);
            } else {
                // checkpoint of slots 4q..4q+3: 2 (q=1, slot 7), 3 (q=2, slot 11),
                // 4 (q<=4, slot 19), 5 (q<=6, slot 27), none (the final max)
                const uint32_t ek = q == 1 ? ((ea >> 16) & 255u) : q == 2 ? (ea >> 24) : q <= 4 ? (eb & 255u)
                                  : q <= 6 ? ((eb >> 8) & 255u) : 0u;
                const int tq = thr(ek);
                const uint32_t cmp = __vcmpleu4(d4, (uint32_t)max(tq, 0) * 0x01010101u);  // 0xFF per slot <= tq
                r = tq < 0 ? 0u : (((cmp >> 7) & 1u) | ((cmp >> 14) & 2u) | ((cmp >> 21) & 4u) | ((cmp >> 28) & 8u));
            }
            qmask |= (uint64_t)r << (4 * q);
        }
        if (nsl < 64) qmask &= (1ull << nsl) - 1ull;
        const int cnt = __popcll(qmask);
        const int incl = warp_incl_scan(cnt, lane);
        if (lane == 31) s.ri[tid >> 5] = incl;
        csync();
        int off = incl - cnt, nq_all = 0;
#pragma unroll
        for (int w = 0; w < CWARPS; w++) {
            if (w < (tid >> 5)) off += s.ri[w];
            nq_all += s.ri[w];
        }
        for (; qmask; qmask &= qmask - 1ull, off++)
            if (off < QMAX) qlist[off] = (uint16_t)((__ffsll((long long)qmask) - 1) * CONSUMERS + tid);
        const int nq = min(nq_all, QMAX);
        // the slot list has its own area: every candidate entry above a
        // staged penalized list is free
        const int room = pen_staged ? CAP - npen : CAP;
        // raw survivors are appended from the top of buf downwards: first the
        // penalized ids that clear the threshold
        for (int i = tid; i < npen; i += CONSUMERS) {
            const int2 pe = pen_staged ? pen_s[i] : (i == tid ? pen0 : pen[i]);
            const float sc = __int_as_float(pe.y);
            if (sc >= lo && pe.x >= 0 && pe.x < R.V) {
                const int pos = atomicAdd(&s.ncand, 1);
                if (pos < room) buf[CAP - 1 - pos] = ((uint64_t)__float_as_uint(sc) << 32) | (uint32_t)pe.x;
            }
        }
        csync();  // the list is complete
        // two list entries per thread in flight per round
        for (int base = 0; base < nq; base += 2 * CONSUMERS) {
            for (int t = 0; t < g; t++) {
                float sc[2][16];
                uint32_t mask[2] = {0u, 0u};
                int o0[2], o1[2];
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int i = base + h * CONSUMERS + tid;
                    const uint32_t entry = i < nq ? qlist[i] : 0u;
                    const int sl = (int)(entry / CONSUMERS), owner = (int)(entry % CONSUMERS);
                    const int it = sl * g + t;
                    o0[h] = it * OCT_TILE + 2 * owner;  // the slot's 64 contiguous bytes
                    o1[h] = o0[h] + 1;
                    if (i < nq && it < R.ntiles) {
                        load_oct_keep(R.ptr, o0[h], R.V, R.vec, sc[h]);
                        load_oct_keep(R.ptr, o1[h], R.V, R.vec, sc[h] + 8);
                        mask[h] = 0xFFFFu;
                    }
                }
                int cnt2 = 0;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    if (mask[h]) {
                        // the tile bounds leave penalized elements out; they
                        // came from the list above
                        if (R.use_pen) exclude_penalized(R, bits8, sc[h], o0[h], o1[h]);
                        uint32_t mk = 0u;
#pragma unroll
                        for (int j = 0; j < 16; j++) {
                            sc[h][j] = __fmul_rn(sc[h][j], R.inv_t);
                            mk |= (sc[h][j] >= lo ? 1u : 0u) << j;
                        }
                        // elements 8*o0 + j (contiguous); only the row's last slot is partial
                        const int left = R.V - 8 * o0[h];
                        mask[h] = left >= 16 ? mk : mk & ((1u << max(left, 0)) - 1u);
                    }
                    cnt2 += __popc(mask[h]);
                }
                // one shared atomic per warp reserves the slots
                const int incl2 = warp_incl_scan(cnt2, lane);
                int pos = 0;
                if (lane == 31 && incl2 > 0) pos = atomicAdd(&s.ncand, incl2);
                pos = __shfl_sync(FULL, pos, 31) + incl2 - cnt2;
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const uint32_t mh = mask[h];
#pragma unroll
                    for (int nb = 0; nb < 4; nb++) {
                        if (mh & (15u << (4 * nb))) {  // most survivors come one or two per slot
#pragma unroll
                            for (int k = 0; k < 4; k++) {
                                const int j = 4 * nb + k;
                                if (mh & (1u << j)) {
                                    if (pos < room)
                                        buf[CAP - 1 - pos] =
                                            ((uint64_t)__float_as_uint(sc[h][j]) << 32) | (uint32_t)(8 * o0[h] + j);
                                    pos++;
                                }
                            }
                        }
                    }
                }
            }
        }
        csync();
        const int nk = nq_all <= QMAX ? s.ncand : CAP + 1;
        if (shard && !shard_topk && nk > a.shard_k) {
            // a min-p row with more survivors in this shard than it may send:
            // the all-ones key tells the merge (the row then gets id -1)
            for (int i = tid; i < a.shard_k; i += CONSUMERS) cand[i] = i == 0 ? SHARD_OVERFLOW : 0ull;
            done = true;
        } else if (nk > 0 && nk <= RANK_MAX) {
            rank_cuts(buf, nk, R, P, by_minp ? __fmul_rn(P.min_p, R.inv) : 0.0f, u, s, cand, a.shard_k, a.col0);
            done = true;
            path = QUASAR_PATH_CANDIDATE;
        } else if (shard && shard_topk && nk > room) {
            // more survivors than the buffer holds: the shard's exact top_k
            // (warp 0; raw entries at the top of buf, where rank_cuts reads them)
            if (tid < 32) {
                const int n = shard_topk_exact(R, bits, pen_staged ? pen_s : pen, npen, a.col0, P.top_k, buf, CAP,
                                               reinterpret_cast<uint32_t*>(bk));
                if (tid == 0) s.ncand = n;
            }
            csync();
            rank_cuts(buf, s.ncand, R, P, 0.0f, u, s, cand, a.shard_k, a.col0);
            done = true;
            path = QUASAR_PATH_CANDIDATE;
        } else if (nk > 0 && nk <= room) {
            const uint64_t* keys = buf;
            // raw entries live in buf[CAP - nk, CAP)
            // counting sort; a full bitonic sort for very large or clustered lists
            const uint64_t* sorted = nk <= CAP / 2 ? bucket_sort_keys(buf, nk, R, bk, s) : nullptr;
            const bool converted = nk <= CAP / 2 && !sorted;
            if (sorted) keys = sorted;
            if (nk > CAP / 2 || converted) {
                int n2 = 32;
                while (n2 < nk) n2 <<= 1;
                uint64_t* area = buf + CAP - n2;  // n2 <= CAP: in place, padded below
                for (int i = tid; i < n2 - nk; i += CONSUMERS) area[i] = 0ull;
                if (!converted) {
                    for (int i = n2 - nk + tid; i < n2; i += CONSUMERS) {
                        const uint64_t en = area[i];
                        const float v = __uint_as_float((uint32_t)(en >> 32));
                        area[i] = ((uint64_t)p_key(v, R.M, R.thr, R.inv) << 32) | (uint32_t)(~(uint32_t)en);
                    }
                }
                csync();
                bitonic_desc(area, n2);
                keys = area;
            }
            if (shard) {
                // the shard's first k keys in (p desc, id asc) order, ids made global
                for (int i = tid; i < a.shard_k; i += CONSUMERS) {
                    uint64_t key = 0ull;
                    if (i < nk) {
                        const uint64_t k0 = keys[i];
                        key = (k0 & 0xFFFFFFFF00000000ull) | (uint32_t)(~(uint32_t)(a.col0 + (int64_t)(~(uint32_t)k0)));
                    }
                    cand[i] = key;
                }
            } else {
                candidate_cuts(keys, nk, P, by_minp ? __fmul_rn(P.min_p, R.inv) : 0.0f, u, s);
            }
            done = true;
            path = QUASAR_PATH_CANDIDATE;
        }
        csync();
    }
    if (shard) {
        // a shard row the candidate path could not bound: no candidates (the
        // merge reports id -1 for it)
        if (!done)
            for (int i = tid; i < a.shard_k; i += CONSUMERS) cand[i] = 0ull;
        if (aborted) cand[0] = SHARD_OVERFLOW;  // (tid 0) stale summaries: the merge reports id -1
        return;
    }
    if (!done) {
        csync();
        select_path(R, bits8, reinterpret_cast<Hist*>(buf), P, u, s);
    }
    if (tid == 0) write_row(a, row, c, aborted ? -1 : s.res_id, s.res_nc, s.res_p, R.inv, path, st_rng);
}

// ---------------------------------------------------------------------------
// Kernels. Dynamic shared memory: kernel A row-load variant [bits]; kernel A
// ring variant [to 64 B][ring NSTAGE x 16 KB][bits][full bars][empty bars]; kernel B
// [scratch: candidate keys / select histograms][bits][counting-sort buckets]
// [qualifying-slot list: QMAX 16-bit entries].

__global__ void __launch_bounds__(CONSUMERS, QS_A_CTAS) sample_rows_ldg(RowsArgs a) {
    extern __shared__ __align__(128) unsigned char dyn[];
    uint32_t* bits = reinterpret_cast<uint32_t*>(dyn);
    __shared__ SharedA s;
    __shared__ float anc_s[NCK * CONSUMERS];
    for (int i = threadIdx.x; i < a.nwords; i += CONSUMERS) bits[i] = 0u;
    if (threadIdx.x == 0) s.abort = 0;
    csync();
    LdgSource src;
    for (int row = blockIdx.x; row < a.B; row += gridDim.x) stream_row(a, row, src, bits, anc_s, s, row != (int)blockIdx.x);
}

template <bool kPickable>
__global__ void __launch_bounds__(CONSUMERS + 32, 3) sample_rows_tma(RowsArgs a) {
    extern __shared__ __align__(128) unsigned char dyn[];
    // the ring starts on a 64-byte boundary (the chunk swizzle flips address
    // bits 4-5 inside each thread's 64 bytes)
    unsigned char* dyn64 = dyn + ((64u - (smem_u32(dyn) & 63u)) & 63u);
    float* ring = reinterpret_cast<float*>(dyn64);
    uint32_t* bits = reinterpret_cast<uint32_t*>(dyn64 + NSTAGE * TILE_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(dyn64 + NSTAGE * TILE_BYTES + ((a.nwords * 4 + 7) & ~7));
    __shared__ SharedA s;
    __shared__ float anc_s[NCK * CONSUMERS];
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + NSTAGE);
    if (threadIdx.x == 0) {
        for (int i = 0; i < NSTAGE; i++) {
            mbar_init(full0 + 8u * i, 1);          // producer's arrive.expect_tx
            mbar_init(empty0 + 8u * i, CWARPS);   // one arrival per consumer warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s.abort = 0;
    }
    for (int i = threadIdx.x; i < a.nwords; i += blockDim.x) bits[i] = 0u;
    __syncthreads();

    if (threadIdx.x >= CONSUMERS) {
        // ---- producer warp: lane 0 streams every chunk of this CTA's rows ----
        if (threadIdx.x != CONSUMERS) return;
        const int ntiles = ((a.V + 7) / 8 + OCT_TILE - 1) / OCT_TILE;
        const int64_t row_bytes = (int64_t)a.V * 4;
        uint32_t g = 0;
        for (int row = blockIdx.x; row < a.B; row += gridDim.x) {
            const char* src = reinterpret_cast<const char*>(a.logits + (int64_t)row * a.ld);
            for (int c = 0; c < ntiles; c++, g++) {
                const int st = (int)(g % NSTAGE);
                if (g >= (uint32_t)NSTAGE) {
                    const uint32_t par = ((g / NSTAGE) - 1u) & 1u;
                    if (!mbar_wait(empty0 + 8u * st, par)) {
                        s.abort = 1;
                        return;  // consumers time out on the missing chunk and finish
                    }
                }
                const int64_t off = (int64_t)c * TILE_BYTES;
                const uint32_t bytes = (uint32_t)min((int64_t)TILE_BYTES, row_bytes - off);
                mbar_arrive_tx(full0 + 8u * st, bytes);
                bulk_g2s(smem_u32(ring + st * TILE_ELEMS), src + off, bytes, full0 + 8u * st);
            }
        }
        return;
    }
    TmaSource<kPickable> src;
    src.ring_u32 = smem_u32(ring);
    src.thr_off = 64u * threadIdx.x + 16u * chunk_swz(threadIdx.x);
    src.full0 = full0;
    src.empty0 = empty0;
    src.g = 0;
    for (int row = blockIdx.x; row < a.B; row += gridDim.x) stream_row(a, row, src, bits, anc_s, s, row != (int)blockIdx.x);
    // After an abort, give chunks still in flight a bounded chance to land
    // before the CTA (and its shared memory) goes away; the rows of this CTA
    // are marked failed (id -1) by kernel B through the abort word.
    if (threadIdx.x == 0 && *reinterpret_cast<volatile int*>(&s.abort)) {
        atomicExch(a.work_abort, 1);
        for (int k = 1; k <= NSTAGE && (uint32_t)k <= src.g; k++) {
            const uint32_t g = src.g - k;
            mbar_wait(full0 + 8u * (g % NSTAGE), (g / NSTAGE) & 1u);
        }
    }
}

template <bool kLongPen, bool kShard>
__global__ void __launch_bounds__(CONSUMERS, 3) sample_rows_finish(RowsArgs a) {
    extern __shared__ __align__(128) unsigned char dyn[];
    uint64_t* buf = reinterpret_cast<uint64_t*>(dyn);
    uint32_t* bits = reinterpret_cast<uint32_t*>(dyn + FINISH_SCRATCH);
    Buckets* bk = reinterpret_cast<Buckets*>(dyn + FINISH_SCRATCH + (((size_t)a.nwords * 4 + 15) & ~(size_t)15));
    __shared__ Shared s;
    uint16_t* qlist = reinterpret_cast<uint16_t*>(reinterpret_cast<unsigned char*>(bk) + sizeof(Buckets));
    if ((int)blockIdx.x < a.B) finish_row<kLongPen, kShard>(a, blockIdx.x, buf, bits, bk, qlist, s);  // one row per CTA
}

// Descending bitonic sort of n2 (a power of two) keys in shared memory by one warp.
__device__ void warp_bitonic_desc(uint64_t* a, int n2, int lane) {
    for (int size = 2; size <= n2; size <<= 1) {
        for (int j = size >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < n2; i += 32) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t x = a[i], y = a[ixj];
                    const bool desc = (i & size) == 0;
                    if (desc ? (x < y) : (x > y)) {
                        a[i] = y;
                        a[ixj] = x;
                    }
                }
            }
            __syncwarp();
        }
    }
}

// Vocab shards, phase 2, one warp per row (shards of up to SW_MAX_COLS
// columns; a CTA holds SW_WARPS rows, no block barriers). The same cuts as
// the CTA kernel's candidate mode, found without the tile tables: the row's
// threshold lo (min-p floor of the global max, the k-th largest per-thread
// max less its tie margin, the 30-nat window) leaves out every thread of
// kernel A whose final max is below it, so only the thread-tiles of the
// other threads (each 16 contiguous columns) are read again; their elements
// at or above lo, minus the penalized columns, plus the penalized list's
// entries at or above lo, are the candidates. They are sorted by (p desc,
// global id asc) and the first k are sent - or, for a min-p row without a
// top_k <= k, all of them (more than k: the overflow key).
constexpr int SW_WARPS = 4;
constexpr int SW_CAP = 512;           // candidates per row
// shard columns the warp kernel takes: a warp re-reads every tile of the
// listed threads, so wider shards (the 2-way split of V = 151936: 19 tiles
// per thread, 342 us per 8192 rows against 208 us for the CTA kernel) keep
// the CTA kernel; 4- and 8-way splits (10 and 5 tiles) are faster per warp
constexpr int SW_MAX_COLS = 12 * TILE_ELEMS;
// Shared memory of one warp: [candidates SW_CAP x 8][listed threads
// CONSUMERS x 2][penalty bitset over the shard's columns].
__host__ __device__ inline size_t sw_warp_bytes(int V) {
    return (size_t)SW_CAP * 8 + CONSUMERS * 2 + (((size_t)(V + 31) / 32 * 4 + 15) & ~(size_t)15);
}
struct ShardWarpSmem {
    uint64_t* cand;
    uint16_t* thr;
    uint32_t* bits;
};

__global__ void __launch_bounds__(32 * SW_WARPS) sample_rows_shard_cand_warp(RowsArgs a) {
    extern __shared__ __align__(128) unsigned char dyn[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    unsigned char* base = dyn + (size_t)w * sw_warp_bytes(a.V);
    ShardWarpSmem sm;
    sm.cand = reinterpret_cast<uint64_t*>(base);
    sm.thr = reinterpret_cast<uint16_t*>(base + (size_t)SW_CAP * 8);
    sm.bits = reinterpret_cast<uint32_t*>(base + (size_t)SW_CAP * 8 + CONSUMERS * 2);
    const int k = a.shard_k;
    // an aborted kernel A (bulk-copy ring timeout) left stale summaries: every
    // row sends the overflow mark, so the merge reports id -1
    const bool aborted = *reinterpret_cast<volatile int*>(a.work_abort) != 0;
    for (int row = blockIdx.x * SW_WARPS + w; row < a.B; row += gridDim.x * SW_WARPS) {
        const quasar_sample_params pr = a.d_params ? a.d_params[row] : a.h_params;
        Row R;
        const RowCtx c = row_ctx(a, row, pr, R);
        const int64_t col0 = c.col0;
        const RowParams& P = c.P;
        uint64_t* out = a.shard_cand + (int64_t)row * k;
        if (aborted) {
            for (int i = lane; i < k; i += 32) out[i] = i == 0 ? SHARD_OVERFLOW : 0ull;
            __syncwarp();
            continue;
        }
        if (!(pr.temperature > 0.0f)) {
            // greedy: this shard's best column (kernel A), as in the CTA kernel
            if (lane == 0) {
                const quasar_shard_stat st = a.all_stats[(int64_t)a.shard_rank * a.B + row];
                out[0] = st.best >= 0 ? ((uint64_t)ord_key(st.max) << 32) | (uint32_t)(~(uint32_t)(col0 + st.best))
                                      : 0ull;
            }
            for (int i = 1 + lane; i < k; i += 32) out[i] = 0ull;
            __syncwarp();
            continue;
        }
        const bool by_minp = P.min_p > 0.0f;
        const bool by_topk = P.top_k > 0 && P.top_k <= TOPK_MAX;
        const bool shard_topk = by_topk && P.top_k <= k;
        if (!(by_minp || shard_topk)) {
            // no bound this shard can stand for: no candidates (the merge reports -1)
            for (int i = lane; i < k; i += 32) out[i] = 0ull;
            __syncwarp();
            continue;
        }
        const float4 info = a.work_info[row];
        const int npen = min(max(__float_as_int(info.z), 0), a.hist_cap);
        shard_norm(a, row, a.B, R.M, R.inv);  // the row's global max and 1/sum
        R.thr = __fsub_rn(R.M, 30.0f);
        const float* tf = a.work_tfmax + (int64_t)row * CONSUMERS;
        float lo = -INFINITY;
        if (by_minp) lo = __fadd_rn(R.M, logf(fminf(P.min_p, 1.0f)) - 0.01f);
        if (by_topk) {
            // the k-th largest per-thread max (topk_floor's value), by a radix
            // select over the order-preserving keys, 8 per lane, bit by bit
            uint32_t key8[CONSUMERS / 32];
#pragma unroll
            for (int q = 0; q < CONSUMERS / 32; q++) key8[q] = ord_key(tf[q * 32 + lane]);
            uint32_t prefix = 0u;
            int need = P.top_k;  // rank (1-based) of the wanted key among those matching prefix
#pragma unroll 1
            for (int b = 31; b >= 0; b--) {
                const uint32_t want = (prefix << 1) | 1u;  // the bit-b-set half sorts first
                int c = 0;
#pragma unroll
                for (int q = 0; q < CONSUMERS / 32; q++) c += ((key8[q] >> b) == want) ? 1 : 0;
                c = __reduce_add_sync(FULL, c);
                if (c >= need) {
                    prefix = want;
                } else {
                    prefix = want - 1u;
                    need -= c;
                }
            }
            const float t = ord_key_inv(prefix);
            lo = fmaxf(lo, !(t > -INFINITY) ? -INFINITY : t - (1e-5f + 1e-5f * fabsf(t)));
        }
        lo = fmaxf(lo, R.thr);
        // the penalized columns of this shard (their re-read values are raw)
        const int nwords = (R.V + 31) >> 5;
        for (int i = lane; i < nwords; i += 32) sm.bits[i] = 0u;
        __syncwarp();
        const int2* pen = a.work_pen + (int64_t)row * a.hist_cap;
        for (int i = lane; i < npen; i += 32) {
            const int id = pen[i].x;
            if (id >= 0 && id < R.V) atomicOr(&sm.bits[id >> 5], 1u << (id & 31));
        }
        // kernel A threads whose final max reaches lo
        int nthr = 0;
        for (int base = 0; base < CONSUMERS; base += 32) {
            const bool q = tf[base + lane] >= lo;
            const unsigned bal = __ballot_sync(FULL, q);
            if (q) sm.thr[nthr + __popc(bal & ((1u << lane) - 1u))] = (uint16_t)(base + lane);
            nthr += __popc(bal);
        }
        __syncwarp();
        // their thread-tiles (16 contiguous columns each), two per lane per
        // round with all four loads in flight
        const int nitems = nthr * R.ntiles;
        int ncand = 0;
        for (int base = 0; base < nitems; base += 64) {
            uint32_t mk[2] = {0u, 0u};
            float v[2][16];
            int e0[2] = {0, 0};
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int i = base + h * 32 + lane;
                if (i < nitems) {
                    const int t = sm.thr[i / R.ntiles], it = i - (i / R.ntiles) * R.ntiles;
                    const int o0 = it * OCT_TILE + 2 * t;
                    e0[h] = 8 * o0;
                    load_oct_keep(R.ptr, o0, R.V, R.vec, v[h]);
                    load_oct_keep(R.ptr, o0 + 1, R.V, R.vec, v[h] + 8);
                    mk[h] = 0xFFFFu;
                }
            }
            int cnt = 0;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                if (mk[h]) {
                    uint32_t m = 0u;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int idx = e0[h] + j;
                        v[h][j] = __fmul_rn(v[h][j], R.inv_t);  // sample.c:142
                        const bool pen_col = idx < R.V && ((sm.bits[idx >> 5] >> (idx & 31)) & 1u);
                        m |= (idx < R.V && !pen_col && v[h][j] >= lo ? 1u : 0u) << j;
                    }
                    mk[h] = m;
                }
                cnt += __popc(mk[h]);
            }
            const int incl = warp_incl_scan(cnt, lane);
            int pos = ncand + incl - cnt;
            ncand += __shfl_sync(FULL, incl, 31);
#pragma unroll
            for (int h = 0; h < 2; h++) {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    if (mk[h] & (1u << j)) {
                        if (pos < SW_CAP)
                            sm.cand[pos] = ((uint64_t)__float_as_uint(v[h][j]) << 32) | (uint32_t)(e0[h] + j);
                        pos++;
                    }
                }
            }
        }
        // the penalized columns at or above lo, with their penalized values
        for (int base = 0; base < npen; base += 32) {
            const int i = base + lane;
            bool keep = false;
            int2 pe = make_int2(0, 0);
            if (i < npen) {
                pe = pen[i];
                keep = pe.x >= 0 && pe.x < R.V && __int_as_float(pe.y) >= lo;
            }
            const unsigned bal = __ballot_sync(FULL, keep);
            const int pos = ncand + __popc(bal & ((1u << lane) - 1u));
            if (keep && pos < SW_CAP) sm.cand[pos] = ((uint64_t)(uint32_t)pe.y << 32) | (uint32_t)pe.x;
            ncand += __popc(bal);
        }
        __syncwarp();
        if (shard_topk && ncand > SW_CAP)  // the bound let too many through: the shard's exact top_k
            ncand = shard_topk_exact(R, sm.bits, pen, npen, col0, P.top_k, sm.cand, 0,
                                     reinterpret_cast<uint32_t*>(sm.cand + SW_CAP / 2));
        if (ncand > SW_CAP || (!shard_topk && ncand > k)) {
            // more candidates than this shard can hold or send
            for (int i = lane; i < k; i += 32) out[i] = i == 0 ? SHARD_OVERFLOW : 0ull;
            __syncwarp();
            continue;
        }
        // keys (p desc, global id asc); each key's rank is the number of
        // larger keys (all distinct: the id is part of the key), and the
        // first k by rank go out in order
        for (int i = lane; i < ncand; i += 32) {
            const uint64_t en = sm.cand[i];
            const uint32_t pk = p_key(__uint_as_float((uint32_t)(en >> 32)), R.M, R.thr, R.inv);
            sm.cand[i] = ((uint64_t)pk << 32) | (uint32_t)(~(uint32_t)(col0 + (int64_t)(uint32_t)en));
        }
        __syncwarp();
        constexpr int PER = 4;  // keys a lane ranks per sweep
        for (int b0 = 0; b0 < ncand; b0 += 32 * PER) {
            uint64_t mine[PER];
            int rank[PER];
#pragma unroll
            for (int q = 0; q < PER; q++) {
                const int i = b0 + q * 32 + lane;
                mine[q] = i < ncand ? sm.cand[i] : 0ull;
                rank[q] = 0;
            }
            for (int j = 0; j < ncand; j++) {
                const uint64_t o = sm.cand[j];  // the same j for every lane: one broadcast read
#pragma unroll
                for (int q = 0; q < PER; q++) rank[q] += o > mine[q] ? 1 : 0;
            }
#pragma unroll
            for (int q = 0; q < PER; q++)
                if (b0 + q * 32 + lane < ncand && rank[q] < k) out[rank[q]] = mine[q];
        }
        for (int i = ncand + lane; i < k; i += 32) out[i] = 0ull;
        __syncwarp();
    }
}

// Merge of the vocab shards' candidates, one warp per row (a CTA holds
// several rows, no block barriers): every shard's k keys arrive sorted (p
// desc, global id asc, 0-padded), so each key's place in the merged order is
// its place in its own list plus, per other list, the number of keys greater
// than it (a binary search). The keys that fall inside the row's kept bound
// are placed into a warp-private sorted array, and the candidate path's cuts
// (top-k, top-p, min-p) and draw run over it with warp scans and ballots -
// the cumulative sums per lane in double, joined by a warp scan, as
// candidate_cuts does. Greedy rows take the largest key. Shared memory per
// warp: the G*k gathered keys and the sorted prefix.
__global__ void __launch_bounds__(256) sample_rows_merge_warp(RowsArgs a) {
    extern __shared__ __align__(128) unsigned char dyn[];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int G = a.shard_G, k = a.shard_k, n = G * k;
    uint64_t* keys = reinterpret_cast<uint64_t*>(dyn) + (size_t)w * 2 * n;  // [G][k] gathered
    uint64_t* sorted = keys + n;                                             // merged prefix
    const int BEYOND = 0x7FFFFFFF;
    for (int row = blockIdx.x * nw + w; row < a.B; row += gridDim.x * nw) {
        const quasar_sample_params pr = a.d_params ? a.d_params[row] : a.h_params;
        Row R;
        const RowCtx c = row_ctx(a, row, pr, R);
        for (int i = lane; i < n; i += 32) {
            const int g = i / k, j = i - g * k;
            keys[i] = a.shard_cand[((int64_t)g * a.B + row) * k + j];
        }
        __syncwarp();
        // keys per list (each list is descending, zeros last) and the overflow mark
        int nk = 0, overflow = 0;
        uint64_t best = 0ull;
        for (int i = lane; i < n; i += 32) {
            const uint64_t key = keys[i];
            nk += (key >> 32) != 0ull ? 1 : 0;  // real keys carry a nonzero p (or ord_key) part
            overflow |= key == SHARD_OVERFLOW ? 1 : 0;
            best = max(best, key);
        }
        nk = warp_sum(nk);
        overflow = __any_sync(FULL, overflow);
        best = warp_max(best);
        if (!(pr.temperature > 0.0f)) {
            // greedy: the largest penalized logit over the shards, lowest
            // global id on ties (sample.c:130-134)
            // (overflow: a shard's streaming pass aborted - id -1)
            if (lane == 0)
                write_row(a, row, c, overflow ? -1 : nk > 0 ? (int)(~(uint32_t)best) : 0, 0, 1.0f, 0.0f,
                          QUASAR_PATH_GREEDY, 0ull);
            __syncwarp();
            continue;
        }
        float M = 0.0f, inv = 0.0f;
        shard_norm(a, row, a.B, M, inv);
        uint64_t st_rng = a.rng[row];
        const double u = rng_unit(&st_rng);  // sample.c:173: one step per stochastic row
        int id = -1, nc = 0;
        float pch = 0.0f;
        if (nk > 0 && !overflow) {
            const RowParams& P = c.P;
            // the merged prefix that can hold the kept set: top_k keys at most
            const int L = (P.top_k > 0 && P.top_k < nk) ? P.top_k : nk;
            for (int i = lane; i < n; i += 32) {
                const uint64_t key = keys[i];
                if ((key >> 32) == 0ull) continue;
                const int g = i / k;
                int rank = i - g * k;  // keys of its own list above it
                for (int h = 0; h < G; h++) {
                    if (h == g) continue;
                    const uint64_t* lst = keys + h * k;
                    int lo = 0, hi = k;  // first position whose key is not greater
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        if (lst[mid] > key) lo = mid + 1;
                        else hi = mid;
                    }
                    rank += lo;
                }
                if (rank < L) sorted[rank] = key;
            }
            __syncwarp();
            auto pval = [&](int i) { return __uint_as_float((uint32_t)(sorted[i] >> 32)); };
            const int S = (L + 31) / 32;
            const int i0 = min(lane * S, L), i1 = min(i0 + S, L);
            double seg = 0.0;
            for (int i = i0; i < i1; i++) seg += (double)pval(i);
            const double incl = warp_incl_scan(seg, lane);
            const double excl = incl - seg;
            // top-k (sample.c:154), top-p (sample.c:156-160), min-p (sample.c:162-167)
            const int nc1 = (P.top_k > 0 && P.top_k < nk) ? P.top_k : BEYOND;
            const int lim = min(nc1, nk);
            const float floor_p = P.min_p > 0.0f ? __fmul_rn(P.min_p, inv) : 0.0f;
            int cut_p = BEYOND, cut_m = nk;
            double cum = excl;
            for (int i = i0; i < i1; i++) {
                cum += (double)pval(i);
                if (P.top_p < 1.0f && i < lim && cut_p == BEYOND && cum >= (double)P.top_p) cut_p = i + 1;
                if (i >= 1 && cut_m == nk && pval(i) < floor_p) cut_m = i;
            }
            cut_p = __reduce_min_sync(FULL, cut_p);
            cut_m = __reduce_min_sync(FULL, cut_m);
            const int nc2 = cut_p != BEYOND ? cut_p : nc1;
            nc = max(1, min(nc2, cut_m));
            // the kept mass (sample.c:171-172): the cumulative sum at nc - 1
            double rs = 0.0;
            if (nc - 1 >= i0 && nc - 1 < i1) {
                rs = excl;
                for (int i = i0; i < nc; i++) rs += (double)pval(i);
            }
            const int owner = max(__ffs(__ballot_sync(FULL, nc - 1 >= i0 && nc - 1 < i1)) - 1, 0);
            const double rsum = __shfl_sync(FULL, rs, owner);
            const double r = u * rsum;  // sample.c:173-175: first kept i with r <= cumsum
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
            const int chosen = cut_d != BEYOND ? cut_d : nc - 1;
            id = (int)(~(uint32_t)sorted[chosen]);
            pch = pval(chosen);
        }
        // (nk == 0: a shard could not bound its candidates; overflow: a shard
        // had more min-p survivors than keys to send - the row gets id -1)
        if (lane == 0) write_row(a, row, c, id, nc, pch, inv, QUASAR_PATH_CANDIDATE, st_rng);
        __syncwarp();
    }
}

// Merge of the vocab shards' candidates, one CTA per row: the G*k gathered
// keys ([G][B][k]) sorted descending, then greedy rows take the first (the
// largest penalized logit, lowest global id on ties) and stochastic rows the
// cuts and draw of the candidate path over the merged list, with the row's
// PRNG step and ring append. Every rank computes the same ids.
__global__ void __launch_bounds__(CONSUMERS, 3) sample_rows_merge(RowsArgs a) {
    extern __shared__ __align__(128) unsigned char dyn[];
    uint64_t* buf = reinterpret_cast<uint64_t*>(dyn);
    __shared__ Shared s;
    const int tid = threadIdx.x;
    const int n = a.shard_G * a.shard_k;
    int n2 = 32;
    while (n2 < n) n2 <<= 1;
    for (int row = blockIdx.x; row < a.B; row += gridDim.x) {
        const quasar_sample_params pr = a.d_params ? a.d_params[row] : a.h_params;
        Row R;
        const RowCtx c = row_ctx(a, row, pr, R);
        for (int i = tid; i < n2; i += CONSUMERS) {
            const int g = i / a.shard_k, j = i - g * a.shard_k;
            buf[i] = i < n ? a.shard_cand[((int64_t)g * a.B + row) * a.shard_k + j] : 0ull;
        }
        csync();
        bitonic_desc(buf, n2);
        int cnt = 0;
        for (int i = tid; i < n; i += CONSUMERS) cnt += (buf[i] >> 32) != 0ull ? 1 : 0;
        const int nk = block_sum_i(cnt, s);  // real keys sort first
        // a shard that overflowed its min-p keys (the largest key sorts first)
        const bool overflow = nk > 0 && buf[0] == SHARD_OVERFLOW;
        if (!(pr.temperature > 0.0f)) {
            if (tid == 0)  // (overflow: a shard's streaming pass aborted - id -1)
                write_row(a, row, c, overflow ? -1 : nk > 0 ? (int)(~(uint32_t)buf[0]) : 0, 0, 1.0f, 0.0f,
                          QUASAR_PATH_GREEDY, 0ull);
        } else {
            float M, inv;
            shard_norm(a, row, a.B, M, inv);
            uint64_t st_rng = a.rng[row];
            const double u = rng_unit(&st_rng);  // sample.c:173
            if (nk > 0 && !overflow) {
                candidate_cuts(buf, nk, c.P, c.P.min_p > 0.0f ? __fmul_rn(c.P.min_p, inv) : 0.0f, u, s);
            } else if (tid == 0) {
                s.res_id = -1;  // a shard could not bound (or send) its candidates
                s.res_nc = 0;
                s.res_p = 0.0f;
            }
            csync();
            if (tid == 0) write_row(a, row, c, s.res_id, s.res_nc, s.res_p, inv, QUASAR_PATH_CANDIDATE, st_rng);
        }
        csync();
    }
}

}  // namespace rows

static int nwords_for(int V) { return ((V + 31) >> 5) + 1; }

size_t rows_smem_bytes(int V) {  // kernel A, row-load variant
    return (size_t)nwords_for(V) * sizeof(uint32_t);
}

size_t rows_tma_smem_bytes(int V) {  // kernel A, ring variant (+64: ring alignment)
    return 64 + (size_t)rows::NSTAGE * rows::TILE_BYTES + (((size_t)nwords_for(V) * 4 + 7) & ~(size_t)7) +
           2 * rows::NSTAGE * sizeof(uint64_t);
}

size_t rows_finish_smem_bytes(int V) {  // kernel B: [scratch][bits][buckets][slot list]
    return (size_t)rows::FINISH_SCRATCH + (((size_t)nwords_for(V) * 4 + 15) & ~(size_t)15) + sizeof(rows::Buckets) +
           rows::QMAX * sizeof(uint16_t);
}

// [abort word][pad][info B x float4][tfmax B x 256 floats][penalized list B x
// hist_cap x int2][tmax B x TMAX_BYTES][anchors B x ANC_BYTES]
size_t rows_workspace_bytes(int B, int hist_cap) {
    const size_t per_row = 16 + 4 * rows::CONSUMERS + 8 * (size_t)(hist_cap > 0 ? hist_cap : 0) +
                           rows::TMAX_BYTES + rows::ANC_BYTES;
    return (size_t)256 + (size_t)B * per_row;
}

int rows_threads() { return rows::CONSUMERS; }

namespace {
// Per-device launch set-up of one kernel (dynamic shared-memory attribute and
// resident-CTA count), shared by every host thread of the process: the first
// launch on a device does it under the mutex, later launches read it.
struct KernelCfg {
    std::atomic<size_t> smem_set[64];
    std::atomic<int> grid[64];  // resident CTAs of the kernel on each device
};
KernelCfg g_ldg, g_tma, g_tma_pick, g_fin, g_fin_long, g_fin_shard, g_fin_shard_long, g_merge, g_merge_warp,
    g_shard_warp;
std::mutex g_cfg_mu;

cudaError_t configure(KernelCfg& cfg, const void* fn, int threads, size_t smem, int dev, int& grid) {
    grid = cfg.grid[dev].load(std::memory_order_acquire);
    if (grid > 0 && cfg.smem_set[dev].load(std::memory_order_acquire) >= smem) return cudaSuccess;
    std::lock_guard<std::mutex> lock(g_cfg_mu);
    cudaError_t err = cudaSuccess;
    if (cfg.smem_set[dev].load() < smem) {
        err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (err != cudaSuccess) return err;
        // the CTA count below is for the larger carve-out
        cfg.grid[dev].store(0);
        cfg.smem_set[dev].store(smem, std::memory_order_release);
    }
    if (cfg.grid[dev].load() == 0) {
        int per_sm = 0, sms = 0;
        err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, cfg.smem_set[dev].load());
        if (err != cudaSuccess) return err;
        err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (err != cudaSuccess) return err;
        cfg.grid[dev].store(max(1, per_sm) * sms, std::memory_order_release);
    }
    grid = cfg.grid[dev].load();
    return cudaSuccess;
}
}  // namespace

namespace {
// Points the workspace fields of a at the layout of rows_workspace_bytes.
void layout_workspace(RowsArgs& a, void* workspace) {
    a.nwords = nwords_for(a.V);
    char* ws = reinterpret_cast<char*>(workspace);
    const size_t B = (size_t)a.B, H = (size_t)(a.hist && a.hist_cap > 0 ? a.hist_cap : 0);
    a.hist_cap = (int)H;
    a.work_abort = reinterpret_cast<int*>(ws);
    ws += 256;
    a.work_info = reinterpret_cast<float4*>(ws);
    ws += B * 16;
    a.work_tfmax = reinterpret_cast<float*>(ws);
    ws += B * 4 * rows::CONSUMERS;
    a.work_pen = reinterpret_cast<int2*>(ws);
    ws += B * 8 * H;
    a.work_tmax = reinterpret_cast<uint8_t*>(ws);
    ws += B * rows::TMAX_BYTES;
    a.work_anc = reinterpret_cast<uint8_t*>(ws);
}

cudaError_t current_device(int& dev) {
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    return (dev < 0 || dev >= 64) ? cudaErrorInvalidDevice : cudaSuccess;
}

// Kernel A: clears the abort word, then streams every row once.
cudaError_t launch_stream(const RowsArgs& a, int dev, cudaStream_t stream) {
    cudaError_t err = cudaMemsetAsync(a.work_abort, 0, sizeof(int), stream);
    if (err != cudaSuccess) return err;
    if (a.tma) {
        const size_t smem = rows_tma_smem_bytes(a.V);
        int grid = 0;
        // long histories: penalized values picked up in the stream (an instance of its own)
        const bool pick = a.hist && a.hist_cap > rows::CONSUMERS;
        const void* fn = pick ? (const void*)rows::sample_rows_tma<true> : (const void*)rows::sample_rows_tma<false>;
        KernelCfg& cfg = pick ? g_tma_pick : g_tma;
        err = configure(cfg, fn, rows::CONSUMERS + 32, smem, dev, grid);
        if (err != cudaSuccess) return err;
        void* args[] = {const_cast<RowsArgs*>(&a)};
        err = cudaLaunchKernel(fn, dim3(min(a.B, grid)), dim3(rows::CONSUMERS + 32), args, smem, stream);
        if (err != cudaSuccess) return err;
    } else {
        const size_t smem = rows_smem_bytes(a.V);
        int grid = 0;
        err = configure(g_ldg, (const void*)rows::sample_rows_ldg, rows::CONSUMERS, smem, dev, grid);
        if (err != cudaSuccess) return err;
        rows::sample_rows_ldg<<<min(a.B, grid), rows::CONSUMERS, smem, stream>>>(a);
    }
    return cudaGetLastError();
}

// The vocab-shard candidate kernel with one warp per row (V <= SW_MAX_COLS).
cudaError_t launch_cand_warp(const RowsArgs& a, int dev, cudaStream_t stream) {
    const size_t smem = rows::SW_WARPS * rows::sw_warp_bytes(a.V);
    int grid = 0;
    cudaError_t err =
        configure(g_shard_warp, (const void*)rows::sample_rows_shard_cand_warp, 32 * rows::SW_WARPS, smem, dev, grid);
    if (err != cudaSuccess) return err;
    const int ctas = min((a.B + rows::SW_WARPS - 1) / rows::SW_WARPS, grid);
    rows::sample_rows_shard_cand_warp<<<ctas, 32 * rows::SW_WARPS, smem, stream>>>(a);
    return cudaGetLastError();
}

// Kernel B: one CTA per row.
cudaError_t launch_finish(const RowsArgs& a, int dev, cudaStream_t stream) {
    const size_t fsmem = rows_finish_smem_bytes(a.V);
    int grid = 0;  // unused: one CTA per row
    const bool long_pen = a.hist && a.hist_cap > rows::CONSUMERS;
    const bool shard = a.shard_cand != nullptr;
    // one instance per (long history, vocab shard) combination
    const void* fn = shard ? (long_pen ? (const void*)rows::sample_rows_finish<true, true>
                                       : (const void*)rows::sample_rows_finish<false, true>)
                           : (long_pen ? (const void*)rows::sample_rows_finish<true, false>
                                       : (const void*)rows::sample_rows_finish<false, false>);
    KernelCfg& cfg = shard ? (long_pen ? g_fin_shard_long : g_fin_shard) : (long_pen ? g_fin_long : g_fin);
    cudaError_t err = configure(cfg, fn, rows::CONSUMERS, fsmem, dev, grid);
    if (err != cudaSuccess) return err;
    void* args[] = {const_cast<RowsArgs*>(&a)};
    err = cudaLaunchKernel(fn, dim3(a.B), dim3(rows::CONSUMERS), args, fsmem, stream);
    if (err != cudaSuccess) return err;
    return cudaGetLastError();
}
}  // namespace

cudaError_t launch_sample_rows(const RowsArgs& args, void* workspace, cudaStream_t stream) {
    RowsArgs a = args;
    layout_workspace(a, workspace);
    int dev = 0;
    cudaError_t err = current_device(dev);
    if (err != cudaSuccess) return err;
    err = launch_stream(a, dev, stream);
    if (err != cudaSuccess) return err;
    return launch_finish(a, dev, stream);
}

cudaError_t launch_shard_stats(const RowsArgs& args, void* workspace, cudaStream_t stream) {
    RowsArgs a = args;
    layout_workspace(a, workspace);
    int dev = 0;
    cudaError_t err = current_device(dev);
    if (err != cudaSuccess) return err;
    return launch_stream(a, dev, stream);
}

cudaError_t launch_shard_candidates(const RowsArgs& args, void* workspace, cudaStream_t stream) {
    RowsArgs a = args;
    layout_workspace(a, workspace);
    int dev = 0;
    cudaError_t err = current_device(dev);
    if (err != cudaSuccess) return err;
    if (a.V <= rows::SW_MAX_COLS) return launch_cand_warp(a, dev, stream);  // one warp per row
    return launch_finish(a, dev, stream);
}

size_t rows_merge_smem_bytes(int G, int k) {
    size_t n2 = 32;
    while (n2 < (size_t)G * (size_t)k) n2 <<= 1;
    return n2 * sizeof(uint64_t);
}

constexpr int MERGE_WARP_MIN_ROWS = 256;

cudaError_t launch_shard_merge(const RowsArgs& args, cudaStream_t stream) {
    int dev = 0;
    cudaError_t err = current_device(dev);
    if (err != cudaSuccess) return err;
    // one warp per row while a warp's keys fit (up to 8 warps per CTA within
    // 96 KB of shared memory) and the batch is large enough to keep the SMs
    // busy with warps; a small batch gets one CTA per row (its sort has 8
    // times the threads of a warp's binary searches: a one-row merge of 32
    // shards' 20 keys took 213 us on one warp)
    const size_t per_warp = (size_t)16 * args.shard_G * args.shard_k;
    if (per_warp <= (size_t)96 * 1024 && args.B >= MERGE_WARP_MIN_ROWS) {
        int warps = (int)min((size_t)8, (size_t)96 * 1024 / per_warp);
        const size_t wsmem = per_warp * warps;
        int grid = 0;
        err = configure(g_merge_warp, (const void*)rows::sample_rows_merge_warp, 32 * warps, wsmem, dev, grid);
        if (err != cudaSuccess) return err;
        const int ctas = min((args.B + warps - 1) / warps, grid);
        rows::sample_rows_merge_warp<<<ctas, 32 * warps, wsmem, stream>>>(args);
        return cudaGetLastError();
    }
    const size_t smem = rows_merge_smem_bytes(args.shard_G, args.shard_k);
    int grid = 0;
    err = configure(g_merge, (const void*)rows::sample_rows_merge, rows::CONSUMERS, smem, dev, grid);
    if (err != cudaSuccess) return err;
    rows::sample_rows_merge<<<min(args.B, grid), rows::CONSUMERS, smem, stream>>>(args);
    return cudaGetLastError();
}

}  // namespace qs
