"""The decode loop the benchmark runs, against the reference step by step.

Each of B rows at V=151936 keeps one set of logits and is re-sampled for many
steps with record on, so its history ring fills with its own recent choices
and the repeat penalty flattens the top of its distribution step after step
(the regime in which rows grow to thousands of candidates). The oracle side
is one reference sampler object per row (oracle/_ref: sample.c compiled
unmodified), given the same starting ring and seed and picked the same number
of times (sample.c:83-92 records each choice, sample.c:111-178 picks).

Per row, every step must match until the first step whose pick the reference
itself puts within 1e-6 of a CDF or tie boundary; from there on the two
sequences may legitimately diverge (different rings), so the row is compared
no further. PRNG states are compared after the loop: each stochastic step
advances them once, whatever was picked."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_BOUNDARY, TOL_P_REL, V_FULL

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not O.available("ref"):
        pytest.skip("reference build (oracle/_ref) absent")


def _decode(B, H, steps, prm, seeds, kind, scale, seed, hist_seed, hist_len0):
    import torch
    import quasar_b200 as q
    dev = torch.device("cuda")
    logits = torch.empty(B, V_FULL, dtype=torch.float32, device=dev)
    q.synth_logits(kind, seed, 0, B, V_FULL, scale, logits)
    hist = torch.empty(B, H, dtype=torch.int32, device=dev)
    q.synth_hist(hist_seed, 0, B, H, V_FULL, hist)
    head0 = (np.arange(B, dtype=np.int32) * 7) % H
    hist_np, len_np = hist.cpu().numpy(), hist_len0.copy()
    hist_len = torch.from_numpy(hist_len0.copy()).to(dev)
    hist_head = torch.from_numpy(head0.copy()).to(dev)
    rng = torch.from_numpy(seeds.view(np.int64).copy()).to(dev)
    d_params = q.params_to_device(prm, dev)
    ids = np.zeros((steps, B), np.int32)
    diags = np.zeros((steps, B), q.DIAG_DTYPE)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    diag = torch.zeros(B, 4, dtype=torch.int32, device=dev)
    for t in range(steps):
        q.pick_batch(logits, rng, d_params=d_params, hist=hist, hist_len=hist_len, hist_head=hist_head,
                     record=True, out=out, diag=diag)
        ids[t] = out.cpu().numpy()
        diags[t] = diag.cpu().numpy().view(q.DIAG_DTYPE).reshape(B)
    gpu = dict(ids=ids, diag=diags, rng=rng.cpu().numpy().view(np.uint64), hist=hist.cpu().numpy(),
               len=hist_len.cpu().numpy(), head=hist_head.cpu().numpy())
    ref, rng_ref, h_ref, l_ref, d_ref = O.ref_decode(logits.cpu().numpy(), prm, seeds, steps, hist_np, len_np,
                                                     head0)
    return gpu, dict(res=ref, rng=rng_ref, hist=h_ref, len=l_ref, head=d_ref)


def _compare(gpu, ref, prm):
    res = ref["res"]
    steps, B = res.shape
    diverged = np.full(B, steps, dtype=np.int64)  # first step a boundary case let the row diverge
    for r in range(B):
        stochastic = prm["temperature"][r] > 0
        for t in range(steps):
            g_id, e = gpu["ids"][t, r], res[t, r]
            near = e["margin"] < TOL_BOUNDARY
            if g_id != e["id"] or (stochastic and gpu["diag"]["n_kept"][t, r] != e["n_kept"]):
                assert stochastic and near, (f"row {r} step {t}: gpu id {g_id} kept {gpu['diag']['n_kept'][t, r]}, "
                                             f"ref id {e['id']} kept {e['n_kept']} margin {e['margin']}")
                diverged[r] = t
                break
            if stochastic:
                rel = abs(float(gpu["diag"]["p_chosen"][t, r]) - float(e["p_chosen"])) / float(e["p_chosen"])
                assert rel <= TOL_P_REL, f"row {r} step {t}: p_chosen off by {rel:.3g}"
    # PRNG: one step per stochastic pick on both sides, whatever was picked
    assert np.array_equal(gpu["rng"], ref["rng"]), "PRNG states differ after the loop"
    whole = diverged == steps
    assert np.array_equal(gpu["hist"][whole], ref["hist"][whole]), "history rings differ"
    assert np.array_equal(gpu["len"][whole], ref["len"][whole]) and np.array_equal(gpu["head"][whole],
                                                                                   ref["head"][whole])
    assert (~whole).sum() <= max(1, B // 16), f"{(~whole).sum()} of {B} rows hit a boundary case"
    return {"rows": B, "steps": steps, "rows_diverged_at_boundary": int((~whole).sum()),
            "max_kept": int(gpu["diag"]["n_kept"].max()), "paths": np.bincount(gpu["diag"]["path"].ravel()).tolist()}


def test_config3_decode_loop_matches_reference_objects():
    """64 config-3 rows (per-row T in [0.2, 1.5], top_p 0.95, min_p 0.05,
    repeat_penalty 1.1 over 256 ids), 128 steps of pick_batch with record on."""
    B, H, steps = 64, 256, 128
    temps = O.synth_uniform(3, 0, B, 0.2, 1.5)
    prm = O.make_params(B, temperature=temps, top_p=0.95, min_p=0.05, repeat_penalty=1.1)
    seeds = np.arange(B, dtype=np.uint64) + np.uint64(5000)
    gpu, ref = _decode(B, H, steps, prm, seeds, O.SYNTH_NORMAL, 3.0, 3, 33, np.full(B, H, np.int32))
    print(_compare(gpu, ref, prm))


def test_mixed_params_decode_loop_from_empty_rings():
    """Rings that start empty and fill up, with greedy, top-k, top-p-only and
    min-p rows side by side (the select path included), 96 steps."""
    B, H, steps = 40, 64, 96
    prm = O.make_params(B, temperature=0.9, top_p=0.9, top_k=0, min_p=0.0, repeat_penalty=1.3)
    prm["temperature"][::5] = 0.0
    prm["top_k"][1::5] = 40
    prm["min_p"][2::5] = 0.05
    prm["top_p"][3::5] = 1.0
    prm["min_p"][3::5] = 0.1
    seeds = np.arange(1, B + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    gpu, ref = _decode(B, H, steps, prm, seeds, O.SYNTH_NORMAL, 2.0, 41, 42, np.zeros(B, np.int32))
    print(_compare(gpu, ref, prm))


def test_long_history_decode_loop_picks_penalties_in_stream():
    """Rings of 512 slots (more than the streaming kernel's 256 threads: the
    instance that picks penalized values up from its ring while streaming)
    filling from empty, with greedy rows (which still claim) mixed in, 64
    steps under a strong repeat penalty."""
    B, H, steps = 24, 512, 64
    prm = O.make_params(B, temperature=1.0, top_p=1.0, min_p=0.1, repeat_penalty=1.5)
    prm["temperature"][::4] = 0.0
    prm["top_k"][1::4] = 20
    seeds = np.arange(3, B + 3, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    gpu, ref = _decode(B, H, steps, prm, seeds, O.SYNTH_ZIPF, 1.1, 71, 72, np.zeros(B, np.int32))
    print(_compare(gpu, ref, prm))
