"""CPU stand-in for the three vocab-shard phases (TEST INFRASTRUCTURE ONLY).

Implements the protocol of quasar_shard_{stats,candidates,finish} (same
tensor layouts: 16-byte stat records, 64-bit candidate keys p_bits << 32 |
~global_id) in numpy, so the host orchestration of
quasar_b200.sharded.VocabShardedSampler - shard offsets, gather order,
record layouts, replicated state updates - runs under gloo ranks on a machine
without a GPU. The numerics follow sample.c:111-178 (penalty, float scale,
double sums, candidate cuts, xorshift64* draw); results are checked against
the unsharded oracle by the tests.
"""
from __future__ import annotations

import numpy as np

from oracle import oracle as O

STAT_DTYPE = np.dtype([("max", "<f4"), ("best", "<i4"), ("sum", "<f8")])
M64 = (1 << 64) - 1


def _params(hp, d_params, B):
    if d_params is not None:
        return d_params.numpy().view(O.PARAMS_DTYPE).reshape(B)
    p = np.zeros(B, dtype=O.PARAMS_DTYPE)
    p["temperature"], p["top_p"], p["min_p"] = hp.temperature, hp.top_p, hp.min_p
    p["repeat_penalty"], p["top_k"] = hp.repeat_penalty, hp.top_k
    return p


def _clamp(r):
    top_p = float(r["top_p"]) if 0.0 < r["top_p"] < 1.0 else 1.0
    return (np.float32(r["temperature"]), np.float32(top_p), max(int(r["top_k"]), 0),
            np.float32(r["min_p"]) if r["min_p"] > 0 else np.float32(0.0),
            np.float32(r["repeat_penalty"]) if r["repeat_penalty"] > 1 else np.float32(1.0))


def _ring(hist, hist_len, hist_head, r):
    if hist is None:
        return []
    cap = hist.shape[1]
    ln = cap if hist_len is None else min(max(int(hist_len[r]), 0), cap)
    hd = 0 if hist_head is None else int(hist_head[r]) % cap
    return [int(hist[r, (hd + i) % cap]) for i in range(ln)]


def _penalized(l, ids, col0, rp):
    l = l.astype(np.float32).copy()
    if rp > 1.0:
        for gid in set(ids):
            j = gid - col0
            if 0 <= j < l.size:
                l[j] = l[j] / rp if l[j] > 0 else l[j] * rp
    return l


def _ord_key(f):
    u = int(np.float32(f).view(np.uint32))
    return (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)


def _norm(st):
    M = np.float32(st["max"].max())
    S = 0.0
    for g in range(st.size):
        if st["max"][g] > -np.inf:
            S += float(st["sum"][g]) * np.exp(np.float64(st["max"][g]) - np.float64(M))
    return M, np.float32(1.0 / S)


def _rng_unit(state):
    x = state
    x ^= (x << 13) & M64
    x ^= x >> 7
    x ^= (x << 17) & M64
    return x, (((x * 0x2545F4914F6CDD1D) & M64) >> 11) * (1.0 / 9007199254740992.0)


class CpuShardPhases:
    def stats(self, logits, col0, hp, d_params, hist, hist_len, hist_head, stats, workspace, stream):
        L = logits.numpy()
        B = L.shape[0]
        prm = _params(hp, d_params, B)
        hn = None if hist is None else hist.numpy()
        ln = None if hist_len is None else hist_len.numpy()
        hh = None if hist_head is None else hist_head.numpy()
        st = np.zeros(B, dtype=STAT_DTYPE)
        for r in range(B):
            T, _, _, _, rp = _clamp(prm[r])
            l = _penalized(L[r], _ring(hn, ln, hh, r), col0, rp)
            if not T > 0:
                j = int(np.argmax(l))
                st[r] = (l[j], j if l[j] > -np.inf else -1, 0.0)
            else:
                sc = (l * (np.float32(1.0) / T)).astype(np.float32)
                M = sc.max()
                fin = sc[np.isfinite(sc)]
                st[r] = (M, -1, float(np.exp(fin.astype(np.float64) - np.float64(M)).sum()))
        stats.numpy()[:] = st.view(np.uint8)

    def candidates(self, logits, col0, hp, d_params, hist, hist_len, hist_head, all_stats, G, rank, k, cand,
                   workspace, stream):
        L = logits.numpy()
        B, Vs = L.shape
        prm = _params(hp, d_params, B)
        allst = all_stats.numpy().view(STAT_DTYPE).reshape(G, B)
        hn = None if hist is None else hist.numpy()
        ln = None if hist_len is None else hist_len.numpy()
        hh = None if hist_head is None else hist_head.numpy()
        out = np.zeros((B, k), dtype=np.uint64)
        for r in range(B):
            T, _, top_k, _, rp = _clamp(prm[r])
            if not T > 0:
                own = allst[rank, r]
                if own["best"] >= 0:
                    out[r, 0] = (_ord_key(own["max"]) << 32) | (~(col0 + int(own["best"])) & 0xFFFFFFFF)
                continue
            if not 1 <= top_k <= k:
                continue
            M, inv = _norm(allst[:, r])
            thr = np.float32(M - np.float32(30.0))
            l = _penalized(L[r], _ring(hn, ln, hh, r), col0, rp)
            sc = (l * (np.float32(1.0) / T)).astype(np.float32)
            j = np.nonzero(sc >= thr)[0]
            e = np.exp((sc[j] - M).astype(np.float32).astype(np.float64)).astype(np.float32)
            p = (e * inv).astype(np.float32)
            keys = (p.view(np.uint32).astype(np.uint64) << np.uint64(32)) | \
                   (~(j.astype(np.int64) + col0) & 0xFFFFFFFF).astype(np.uint64)
            keys = np.sort(keys)[::-1][:k]
            out[r, :keys.size] = keys
        cand.numpy()[:] = out.reshape(-1).view(np.int64)

    def finish(self, all_cand, all_stats, G, k, B, hp, d_params, rng, hist, hist_len, hist_head, record, out,
               diag, stream):
        prm = _params(hp, d_params, B)
        allc = all_cand.numpy().view(np.uint64).reshape(G, B, k)
        allst = all_stats.numpy().view(STAT_DTYPE).reshape(G, B)
        rn = rng.numpy().view(np.uint64)
        hn = None if hist is None else hist.numpy()
        ln = None if hist_len is None else hist_len.numpy()
        hh = None if hist_head is None else hist_head.numpy()
        o = out.numpy()
        dg = None if diag is None else diag.numpy().reshape(B, 4)
        for r in range(B):
            T, top_p, top_k, min_p, _ = _clamp(prm[r])
            keys = np.sort(allc[:, r, :].reshape(-1))[::-1]
            nk = int(((keys >> np.uint64(32)) != 0).sum())
            if not T > 0:
                chosen, nc, pc, inv, path = (int(~int(keys[0]) & 0xFFFFFFFF) if nk else 0), 0, 1.0, 0.0, 0
            else:
                M, inv = _norm(allst[:, r])
                state, u = _rng_unit(int(rn[r]))
                rn[r] = np.uint64(state)
                path = 1
                if nk == 0:
                    chosen, nc, pc = -1, 0, 0.0
                else:
                    p = (keys[:nk] >> np.uint64(32)).astype(np.uint32).view(np.float32)
                    nc1 = top_k if 0 < top_k < nk else None
                    lim = nk if nc1 is None else min(nc1, nk)
                    cut_p = None
                    if top_p < 1.0:
                        c = 0.0
                        for i in range(lim):
                            c += float(p[i])
                            if c >= float(top_p):
                                cut_p = i + 1
                                break
                    floor = np.float32(min_p * inv) if min_p > 0 else np.float32(0.0)
                    cut_m = nk
                    for i in range(1, nk):
                        if p[i] < floor:
                            cut_m = i
                            break
                    nc2 = cut_p if cut_p is not None else (nc1 if nc1 is not None else 1 << 30)
                    nc = max(1, min(nc2, cut_m))
                    rsum = float(np.sum(p[:nc].astype(np.float64)))
                    rr = u * rsum
                    c, pos = 0.0, nc - 1
                    for i in range(nc):
                        c += float(p[i])
                        if c >= rr:
                            pos = i
                            break
                    chosen, pc = int(~int(keys[pos]) & 0xFFFFFFFF), float(p[pos])
            o[r] = chosen
            if dg is not None:
                dg[r] = np.array([nc, np.float32(pc).view(np.int32), np.float32(inv).view(np.int32), path],
                                 dtype=np.int32)
            if record and hn is not None and ln is not None and hh is not None and chosen >= 0:
                cap = hn.shape[1]
                L0 = min(max(int(ln[r]), 0), cap)
                H0 = int(hh[r]) % cap
                if L0 < cap:
                    hn[r, (H0 + L0) % cap] = chosen
                    ln[r] = L0 + 1
                else:
                    hn[r, H0] = chosen
                    hh[r] = (H0 + 1) % cap
