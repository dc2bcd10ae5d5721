"""Shared parity machinery: run the CUDA sampler and the CPU oracle on the same
bits and compare them under the tolerance BASELINE.json states:
  * greedy and top_k=1: bit-exact ids;
  * stochastic: identical ids and kept-set sizes except where the oracle's own
    sorted order puts a draw, a cut or a tie within 1e-6 of its boundary;
    probabilities within 1e-5 relative;
  * PRNG states after the pick: bit-exact (one xorshift64* step per stochastic
    row, none for greedy rows).
"""
from __future__ import annotations

import numpy as np

from oracle import oracle as O

V_FULL = 151936
TOL_BOUNDARY = 1e-6
TOL_P_REL = 1e-5


def gpu_inputs(kind: int, seed: int, B: int, V: int, scale: float, H: int = 0, hist_seed: int = 0,
               row0: int = 0):
    import torch
    import quasar_b200 as q
    logits = torch.empty(B, V, dtype=torch.float32, device="cuda")
    q.synth_logits(kind, seed, row0, B, V, scale, logits)
    hist = None
    if H:
        hist = torch.empty(B, H, dtype=torch.int32, device="cuda")
        q.synth_hist(hist_seed, row0, B, H, V, hist)
    return logits, hist


def run_gpu(logits, params: np.ndarray, seeds: np.ndarray, hist=None, hist_len=None,
            hist_head=None, flags: int = 0, record: bool = False):
    """Returns (ids, diag records, rng after) as numpy arrays."""
    import torch
    import quasar_b200 as q
    B = logits.shape[0]
    dev = logits.device
    rng = torch.from_numpy(np.ascontiguousarray(seeds, dtype=np.uint64).view(np.int64).copy()).to(dev)
    diag = torch.zeros(B, 4, dtype=torch.int32, device=dev)
    kw = {}
    if len(params) == B and B > 1:
        kw["d_params"] = q.params_to_device(params, dev)
    else:
        kw["params"] = params[:1]
    out = q.pick_batch(logits, rng, hist=hist, hist_len=hist_len, hist_head=hist_head,
                       record=record, diag=diag, flags=flags, **kw)
    torch.cuda.synchronize()
    d = diag.cpu().numpy().view(q.DIAG_DTYPE).reshape(B)
    return out.cpu().numpy(), d, rng.cpu().numpy().view(np.uint64)


def run_oracle(logits, params, seeds, hist=None, hist_len=None, hist_head=None, backend=None):
    ln = logits.cpu().numpy() if hasattr(logits, "cpu") else logits
    hn = None if hist is None else (hist.cpu().numpy() if hasattr(hist, "cpu") else hist)
    ll = None if hist_len is None else (hist_len.cpu().numpy() if hasattr(hist_len, "cpu") else hist_len)
    hh = None if hist_head is None else (hist_head.cpu().numpy() if hasattr(hist_head, "cpu") else hist_head)
    return O.pick_rows(ln, params, seeds, hist=hn, hist_len=ll, hist_head=hh, backend=backend)


def assert_parity(ids, diag, rng_gpu, res, rng_ref, max_mismatch_frac: float = 0.01):
    """Check one batch; returns a small report dict."""
    ids = np.asarray(ids)
    greedy = res["greedy"] == 1
    assert np.array_equal(rng_gpu, rng_ref), "PRNG states differ"
    g_bad = np.nonzero(greedy & (ids != res["id"]))[0]
    assert g_bad.size == 0, f"greedy rows differ: {g_bad[:10]} gpu={ids[g_bad[:10]]} ref={res['id'][g_bad[:10]]}"
    st = ~greedy
    near = res["margin"] < TOL_BOUNDARY
    mism = st & (ids != res["id"])
    bad = np.nonzero(mism & ~near)[0]
    assert bad.size == 0, (f"stochastic rows differ away from any boundary: rows {bad[:10]} "
                           f"gpu={ids[bad[:10]]} ref={res['id'][bad[:10]]} margin={res['margin'][bad[:10]]}")
    nk_bad = np.nonzero(st & (diag["n_kept"] != res["n_kept"]) & ~near)[0]
    assert nk_bad.size == 0, (f"kept-set sizes differ: rows {nk_bad[:10]} gpu={diag['n_kept'][nk_bad[:10]]} "
                              f"ref={res['n_kept'][nk_bad[:10]]}")
    same = st & ~mism
    if same.any():
        rel = np.abs(diag["p_chosen"][same].astype(np.float64) - res["p_chosen"][same]) / res["p_chosen"][same]
        assert rel.max() <= TOL_P_REL, f"p_chosen off by {rel.max():.3g} relative"
    n_st = int(st.sum())
    frac = float(mism.sum()) / max(1, n_st)
    assert frac <= max_mismatch_frac, f"{mism.sum()} of {n_st} stochastic rows differ (all near boundaries)"
    return {"rows": int(ids.size), "stochastic": n_st, "mismatched_near_boundary": int(mism.sum())}
