"""GPU parity: the CUDA sampler (through the C ABI) against the CPU oracle
(the reference sample.c compiled unmodified when oracle/_ref is present, the
plain-C restatement otherwise) on identical seeded inputs.

Configs follow BASELINE.json; full-size batches are cut to row subsets the CPU
oracle finishes in seconds (the reference costs ~33 ms per full-vocab row).
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import V_FULL, assert_parity, gpu_inputs, run_gpu, run_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import quasar_b200  # noqa: F401  (fails loudly if the library is missing)


def _seeds(B, base=1000):
    return (np.arange(B, dtype=np.uint64) + np.uint64(base))


@pytest.mark.parametrize("kind,scale", [(O.SYNTH_NORMAL, 3.0), (O.SYNTH_GUMBEL_PEAK, 1.0),
                                        (O.SYNTH_ZIPF, 1.1)])
def test_synth_bits_match(kind, scale):
    logits, hist = gpu_inputs(kind, 77, 3, V_FULL, scale, H=64, hist_seed=5, row0=11)
    cpu = O.synth_logits(kind, 77, 11, 3, V_FULL, scale)
    assert np.array_equal(logits.cpu().numpy().view(np.uint32), cpu.view(np.uint32))
    assert np.array_equal(hist.cpu().numpy(), O.synth_hist(5, 11, 3, 64, V_FULL))


def test_config2_greedy_bit_exact():
    B = 256
    logits, hist = gpu_inputs(O.SYNTH_GUMBEL_PEAK, 2, B, V_FULL, 1.0, H=64, hist_seed=3)
    seeds = _seeds(B)
    for rp in (1.0, 1.1):
        prm = O.make_params(1, temperature=0.0, repeat_penalty=rp)
        ids, diag, rng = run_gpu(logits, prm, seeds, hist=hist)
        res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
        assert np.array_equal(ids, res["id"])
        assert np.array_equal(rng, seeds)  # greedy draws nothing
        assert (diag["path"] == 0).all()


def test_config2_topk1_bit_exact():
    B = 256
    logits, _ = gpu_inputs(O.SYNTH_GUMBEL_PEAK, 2, B, V_FULL, 1.0)
    seeds = _seeds(B)
    prm = O.make_params(1, temperature=1.0, top_k=1)
    ids, diag, rng = run_gpu(logits, prm, seeds)
    res, rng_ref = run_oracle(logits, prm, seeds)
    assert np.array_equal(ids, res["id"])
    assert np.array_equal(rng, rng_ref)  # top_k=1 still draws once
    assert (diag["n_kept"] == 1).all()


def test_config1_single_row():
    logits, hist = gpu_inputs(O.SYNTH_NORMAL, 42, 1, V_FULL, 3.0, H=64, hist_seed=42)
    seeds = np.array([42], dtype=np.uint64)
    prm = O.make_params(1, temperature=0.7, top_k=20, top_p=0.8, repeat_penalty=1.1)
    ids, diag, rng = run_gpu(logits, prm, seeds, hist=hist)
    res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
    assert_parity(ids, diag, rng, res, rng_ref)


def _config3(B, flags=0):
    import torch
    import quasar_b200 as q
    logits, hist = gpu_inputs(O.SYNTH_NORMAL, 3, B, V_FULL, 3.0, H=256, hist_seed=33)
    temps = torch.empty(B, dtype=torch.float32, device="cuda")
    q.synth_uniform(3, 0, B, 0.2, 1.5, temps)
    prm = O.make_params(B, temperature=temps.cpu().numpy(), top_p=0.95, min_p=0.05,
                        repeat_penalty=1.1)
    seeds = _seeds(B, 5000)
    return logits, hist, prm, seeds


def test_config3_subset_candidate_path():
    logits, hist, prm, seeds = _config3(256)
    ids, diag, rng = run_gpu(logits, prm, seeds, hist=hist)
    res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
    rep = assert_parity(ids, diag, rng, res, rng_ref)
    assert (diag["path"] == 1).all(), np.bincount(diag["path"])
    print(rep)


def test_config3_exact_select_agrees():
    logits, hist, prm, seeds = _config3(64)
    ids_c, diag_c, rng_c = run_gpu(logits, prm, seeds, hist=hist)
    ids_s, diag_s, rng_s = run_gpu(logits, prm, seeds, hist=hist, flags=1)
    assert (diag_s["path"] == 2).all()
    assert np.array_equal(ids_c, ids_s)
    assert np.array_equal(diag_c["n_kept"], diag_s["n_kept"])
    assert np.array_equal(diag_c["p_chosen"].view(np.uint32), diag_s["p_chosen"].view(np.uint32))
    res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
    assert_parity(ids_s, diag_s, rng_s, res, rng_ref)


def test_large_candidate_lists_stay_on_candidate_path():
    """Rows with 2200-3400 candidates spread over about as many thread-slots
    (the flat top a history full of recently chosen tokens gives under a
    repeat penalty): the candidate path takes every one of them, without the
    select path's whole-row passes, and matches the reference. Per-row min_p
    puts the min-p floor halfway between the k-th and (k+1)-th largest scaled
    logits, away from any tie."""
    B = 32
    T = 1.5
    logits, hist = gpu_inputs(O.SYNTH_NORMAL, 17, B, V_FULL, 3.0, H=64, hist_seed=18)
    sc = np.sort(logits.cpu().numpy() / np.float32(T), axis=1)[:, ::-1]
    k = np.linspace(2200, 3400, B).astype(np.int64)
    mid = 0.5 * (sc[np.arange(B), k - 1].astype(np.float64) + sc[np.arange(B), k])
    min_p = np.exp(mid - sc[:, 0]).astype(np.float32)
    prm = O.make_params(B, temperature=T, top_p=1.0, min_p=min_p, repeat_penalty=1.1)
    seeds = _seeds(B, 700)
    ids, diag, rng = run_gpu(logits, prm, seeds, hist=hist)
    res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
    # (a few of these rows draw within 1e-6 of a CDF or tie boundary)
    assert_parity(ids, diag, rng, res, rng_ref, max_mismatch_frac=0.1)
    assert (diag["path"] == 1).all(), np.bincount(diag["path"])
    assert (res["n_kept"] > 2048).all(), res["n_kept"]


def test_config5_subset_zipf():
    B = 96
    logits, hist = gpu_inputs(O.SYNTH_ZIPF, 5, B, V_FULL, 1.1, H=2048, hist_seed=55)
    prm = O.make_params(1, temperature=1.0, top_p=1.0, min_p=0.1, repeat_penalty=1.3)
    seeds = _seeds(B, 9000)
    ids, diag, rng = run_gpu(logits, prm, seeds, hist=hist)
    res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
    assert_parity(ids, diag, rng, res, rng_ref)


@pytest.mark.parametrize("prm_kw", [
    dict(temperature=0.8, top_k=40, top_p=0.9),                 # config 4's parameters
    dict(temperature=1.0),                                      # pure multinomial
    dict(temperature=0.7, top_p=0.95),                          # nucleus only
    dict(temperature=1.5, top_k=200, min_p=0.01),
    dict(temperature=0.05, top_p=0.5, min_p=0.2),
])
def test_select_path_params(prm_kw):
    B = 32
    logits, hist = gpu_inputs(O.SYNTH_NORMAL, 11, B, V_FULL, 3.0, H=64, hist_seed=12)
    prm = O.make_params(1, repeat_penalty=1.1, **prm_kw)
    seeds = _seeds(B, 100)
    ids, diag, rng = run_gpu(logits, prm, seeds, hist=hist)
    res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
    assert_parity(ids, diag, rng, res, rng_ref)


@pytest.mark.parametrize("V", [1, 2, 3, 31, 33, 1000, 4095])
@pytest.mark.parametrize("prm_kw", [dict(temperature=0.0, repeat_penalty=1.5),
                                    dict(temperature=0.9, min_p=0.05, repeat_penalty=1.2),
                                    dict(temperature=1.3, top_p=0.7, top_k=5),
                                    dict(temperature=2.0)])
def test_small_vocab_edges(V, prm_kw):
    B = 16
    H = min(8, V)
    logits, hist = gpu_inputs(O.SYNTH_NORMAL, 1234 + V, B, V, 2.0, H=H, hist_seed=V)
    prm = O.make_params(1, **prm_kw)
    seeds = _seeds(B, 77)
    ids, diag, rng = run_gpu(logits, prm, seeds, hist=hist)
    res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
    assert_parity(ids, diag, rng, res, rng_ref, max_mismatch_frac=0.1)


def test_ties_resolve_by_id():
    import torch
    B, V = 8, 5000
    # quantised logits: many exact ties in p, resolved by ascending id
    base = torch.randint(-3, 4, (B, V), generator=torch.Generator().manual_seed(0)).float()
    logits = base.cuda()
    seeds = _seeds(B, 31)
    for prm_kw in (dict(temperature=0.0), dict(temperature=1.0, top_k=7),
                   dict(temperature=1.0, top_p=0.3), dict(temperature=0.5, min_p=0.5),
                   dict(temperature=1.0)):
        prm = O.make_params(1, **prm_kw)
        ids, diag, rng = run_gpu(logits, prm, seeds)
        ids_s, diag_s, _ = run_gpu(logits, prm, seeds, flags=1)
        res, rng_ref = run_oracle(logits, prm, seeds)
        assert_parity(ids, diag, rng, res, rng_ref, max_mismatch_frac=0.0)
        assert_parity(ids_s, diag_s, rng, res, rng_ref, max_mismatch_frac=0.0)


def test_history_ring_edges():
    import torch
    B, V, H = 12, 9000, 16
    logits, _ = gpu_inputs(O.SYNTH_NORMAL, 8, B, V, 3.0)
    # put the top ids into the history (duplicates, out-of-range ids, partial rings)
    top = torch.topk(logits, 4, dim=1).indices.int()
    hist = torch.full((B, H), -5, dtype=torch.int32, device="cuda")
    hist[:, :4] = top
    hist[:, 4:8] = top
    hist[:, 8] = V + 10
    hist_len = torch.tensor([H, 0, 3, 9, 16, 1, 5, 16, 2, 7, 16, 12], dtype=torch.int32, device="cuda")
    hist_head = torch.tensor([0, 3, 15, 14, 7, 0, 2, 9, 11, 4, 1, 13], dtype=torch.int32, device="cuda")
    for prm_kw in (dict(temperature=0.0, repeat_penalty=2.0),
                   dict(temperature=0.6, min_p=0.02, repeat_penalty=1.7),
                   dict(temperature=0.6, top_k=10, repeat_penalty=1.7)):
        prm = O.make_params(1, **prm_kw)
        seeds = _seeds(B, 555)
        ids, diag, rng = run_gpu(logits, prm, seeds, hist=hist, hist_len=hist_len, hist_head=hist_head)
        res, rng_ref = run_oracle(logits, prm, seeds, hist=hist, hist_len=hist_len, hist_head=hist_head)
        assert_parity(ids, diag, rng, res, rng_ref, max_mismatch_frac=0.0)


def test_record_matches_reference_ring():
    """record=1 appends like sample.c:83-92 (fill, then overwrite the oldest)."""
    import torch
    B, V, H = 6, 3000, 4
    seeds = _seeds(B, 4242)
    hist = torch.zeros(B, H, dtype=torch.int32, device="cuda")
    hist_len = torch.zeros(B, dtype=torch.int32, device="cuda")
    hist_head = torch.zeros(B, dtype=torch.int32, device="cuda")
    rng = seeds.copy()
    ring = [[] for _ in range(B)]
    prm = O.make_params(1, temperature=0.8, min_p=0.01, repeat_penalty=1.3)
    for step in range(7):
        logits, _ = gpu_inputs(O.SYNTH_NORMAL, 900 + step, B, V, 2.0)
        ids, diag, rng_new = run_gpu(logits, prm, rng, hist=hist, hist_len=hist_len,
                                     hist_head=hist_head, record=True)
        for r in range(B):
            ring[r].append(int(ids[r]))
            ring[r] = ring[r][-H:]
        got_len = hist_len.cpu().numpy()
        assert (got_len == min(step + 1, H)).all()
        h = hist.cpu().numpy()
        hd = hist_head.cpu().numpy()
        for r in range(B):
            n = got_len[r]
            cur = [int(h[r][(hd[r] + i) % H]) for i in range(n)]
            assert cur == ring[r]
        rng = rng_new


def test_dropin_sequence_matches_reference():
    """The sample.h drop-in (host pointer in, id out) reproduces a reference
    sampler object's id sequence, history recording and PRNG included."""
    if not O.available("ref"):
        pytest.skip("reference build absent")
    import quasar_b200 as q
    V, n = 20000, 24
    steps = O.synth_logits(O.SYNTH_NORMAL, 31337, 0, n, V, 2.5)
    # feed back: plant a strong logit on a few ids so the repeat penalty matters
    steps[:, 7] += 6.0
    steps[:, 11] += 5.5
    for kw, last_n, seed in ((dict(temperature=0.9, top_p=0.95, top_k=40, min_p=0.05,
                                   repeat_penalty=1.3), 8, 99),
                             (dict(temperature=0.0, repeat_penalty=1.5), 3, 5),
                             (dict(temperature=1.2, repeat_penalty=1.1), 64, 7)):
        prm = O.make_params(1, **kw)
        ref_ids = O.ref_sequence(steps, prm, last_n, seed)
        s = q.Sampler()
        s.config(kw["temperature"], kw.get("top_p", 1.0), kw.get("top_k", 0), kw.get("min_p", 0.0),
                 kw["repeat_penalty"], last_n, seed)
        got = [s.pick(steps[t]) for t in range(n)]
        s.close()
        assert got == list(ref_ids), (got, list(ref_ids))


@pytest.mark.parametrize("prm_kw", [dict(temperature=0.0, repeat_penalty=1.3),
                                    dict(temperature=1.1, top_p=0.95, min_p=0.05, repeat_penalty=1.1),
                                    dict(temperature=0.7, top_k=20, top_p=0.8)])
def test_ring_kernel_equals_row_kernel(prm_kw):
    """The bulk-copy ring kernel and the one-CTA-per-row kernel give identical
    rows (ids, kept counts, p bits, PRNG), on the same seeded inputs."""
    B = 300
    logits, hist = gpu_inputs(O.SYNTH_NORMAL, 21, B, V_FULL, 3.0, H=128, hist_seed=22)
    prm = O.make_params(1, **prm_kw)
    seeds = _seeds(B, 808)
    a = run_gpu(logits, prm, seeds, hist=hist)
    b = run_gpu(logits, prm, seeds, hist=hist, flags=2)
    assert np.array_equal(a[0], b[0])
    assert np.array_equal(a[1]["n_kept"], b[1]["n_kept"])
    assert np.array_equal(a[1]["p_chosen"].view(np.uint32), b[1]["p_chosen"].view(np.uint32))
    assert np.array_equal(a[2], b[2])


@pytest.mark.parametrize("offset,extra", [(1, 0), (4, 3), (0, 5)])
def test_strided_and_unaligned_rows(offset, extra):
    """Row stride ld > V and a base pointer off the 16/32-byte grid take the
    scalar-load path and still match the oracle."""
    import torch
    B, V = 24, 20000
    ld = V + extra
    src, _ = gpu_inputs(O.SYNTH_NORMAL, 55, B, V, 2.5)
    store = torch.full((B * ld + offset + 8,), float("nan"), dtype=torch.float32, device="cuda")
    view = store[offset:offset + B * ld].view(B, ld)
    view[:, :V] = src
    logits = view[:, :V]
    prm = O.make_params(1, temperature=0.9, min_p=0.03, top_p=0.9)
    seeds = _seeds(B, 64)
    ids, diag, rng = run_gpu(logits, prm, seeds)
    res, rng_ref = run_oracle(src, prm, seeds)
    assert_parity(ids, diag, rng, res, rng_ref)


def test_top_p_only_rows_bounded_by_thread_maxima():
    """Rows cut by top-p alone: where the per-thread maxima above some value
    already carry the top-p mass (peaked rows: low temperature), the row
    takes the candidate path with that value as its threshold; flat rows
    (high temperature) keep the select path. Both match the reference, and
    the bounded rows match the exact select path bit for bit."""
    B = 64
    logits, hist = gpu_inputs(O.SYNTH_NORMAL, 61, B, V_FULL, 3.0, H=64, hist_seed=62)
    temps = np.linspace(0.15, 1.5, B).astype(np.float32)
    prm = O.make_params(B, temperature=temps, top_p=0.9, repeat_penalty=1.1)
    seeds = _seeds(B, 4242)
    ids, diag, rng = run_gpu(logits, prm, seeds, hist=hist)
    res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
    assert_parity(ids, diag, rng, res, rng_ref)
    paths = diag["path"]
    assert (paths[:8] == 1).all(), paths      # the coolest rows are bounded
    assert (paths[-8:] == 2).all(), paths     # the flattest are not
    ids_s, diag_s, rng_s = run_gpu(logits, prm, seeds, hist=hist, flags=1)
    bounded = paths == 1
    assert np.array_equal(ids[bounded], ids_s[bounded])
    assert np.array_equal(diag["n_kept"][bounded], diag_s["n_kept"][bounded])
    assert np.array_equal(diag["p_chosen"][bounded].view(np.uint32), diag_s["p_chosen"][bounded].view(np.uint32))
