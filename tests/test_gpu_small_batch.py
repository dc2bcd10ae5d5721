"""Small batches: rows with host parameters sampled by the fused cluster
kernel (a cluster of G CTAs per row, each holding V/G columns in shared
memory; quasar_sampler_split_shards > 0), against the reference
(oracle/_ref: sample.c compiled unmodified, sample.c:111-178) and against
the same calls on one CTA per row (QUASAR_FLAG_NO_SPLIT).

Greedy rows are bit-exact; stochastic rows follow the tolerance of every
parity test (ids equal away from the 1e-6 boundary band, p_chosen within
1e-5 relative, PRNG states bit-exact)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_BOUNDARY, TOL_P_REL, V_FULL, assert_parity, gpu_inputs, run_gpu, run_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not O.available("ref"):
        pytest.skip("reference build (oracle/_ref) absent")


def _seeds(B, base):
    return np.arange(B, dtype=np.uint64) + np.uint64(base)


def _shards(B, V, prm, H=0, flags=0):
    import quasar_b200 as q
    return q.split_shards(B, V, params=prm[:1], hist_cap=H, flags=flags)


def _same_as_unsplit(a, b, res):
    """Split (a) and one-CTA (b) results of one batch: ids and kept counts
    equal, p_chosen within 1e-5 (the row sums are added in another order),
    except on rows the reference puts within 1e-6 of a boundary (res)."""
    ids, diag, rng = a
    ids_n, diag_n, rng_n = b
    assert np.array_equal(rng, rng_n)
    far = res["margin"] >= TOL_BOUNDARY
    assert np.array_equal(ids[far], ids_n[far]), np.nonzero(ids != ids_n)
    assert np.array_equal(diag["n_kept"][far], diag_n["n_kept"][far])
    st = far & (diag["path"] != 0)
    if st.any():
        rel = np.abs(diag["p_chosen"][st].astype(np.float64) - diag_n["p_chosen"][st]) / diag_n["p_chosen"][st]
        assert rel.max() <= TOL_P_REL


def test_split_config1_rows():
    """Config 1's parameters (T 0.7, top_k 20, top_p 0.8, repeat_penalty 1.1
    over 64 ids): eight single rows, then the same rows as one batch of 8
    and of 16 (8 shards each)."""
    import quasar_b200 as q
    prm = O.make_params(1, temperature=0.7, top_k=20, top_p=0.8, repeat_penalty=1.1)
    for r in range(8):
        logits, hist = gpu_inputs(O.SYNTH_NORMAL, 42, 1, V_FULL, 3.0, H=64, hist_seed=42, row0=r)
        assert _shards(1, V_FULL, prm, 64) == 8
        seeds = _seeds(1, 42 + r)
        got = run_gpu(logits, prm, seeds, hist=hist)
        res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
        assert_parity(*got, res, rng_ref, max_mismatch_frac=0.0 if res["margin"][0] >= TOL_BOUNDARY else 1.0)
        _same_as_unsplit(got, run_gpu(logits, prm, seeds, hist=hist, flags=q.FLAG_NO_SPLIT), res)
    for B, G in ((8, 8), (16, 8)):
        logits, hist = gpu_inputs(O.SYNTH_NORMAL, 42, B, V_FULL, 3.0, H=64, hist_seed=42)
        assert _shards(B, V_FULL, prm, 64) == G
        seeds = _seeds(B, 4200)
        got = run_gpu(logits, prm, seeds, hist=hist)
        res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
        print(assert_parity(*got, res, rng_ref, max_mismatch_frac=1.0 / B))
        _same_as_unsplit(got, run_gpu(logits, prm, seeds, hist=hist, flags=q.FLAG_NO_SPLIT), res)


@pytest.mark.parametrize("kind,scale", [(O.SYNTH_GUMBEL_PEAK, 1.0), (O.SYNTH_NORMAL, 3.0)])
def test_split_greedy_bit_exact(kind, scale):
    """Greedy and top_k = 1 rows: the penalized argmax over the shards' best
    columns, lowest id on ties, no PRNG step for the greedy rows."""
    B = 12
    logits, hist = gpu_inputs(kind, 7, B, V_FULL, scale, H=96, hist_seed=8)
    # the rows' own top ids in their rings, so the penalty moves the argmax
    import torch
    hist[:, :4] = torch.topk(logits, 4, dim=1).indices.int()
    seeds = _seeds(B, 77)
    for prm in (O.make_params(1, temperature=0.0, repeat_penalty=1.3),
                O.make_params(1, temperature=0.8, top_k=1, repeat_penalty=1.3)):
        assert _shards(B, V_FULL, prm, 96) == 8
        ids, diag, rng = run_gpu(logits, prm, seeds, hist=hist)
        res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
        assert_parity(ids, diag, rng, res, rng_ref, max_mismatch_frac=0.0)
        assert np.array_equal(ids, res["id"])


def test_split_wide_top_k_with_top_p_and_min_p():
    """top_k 256 (the largest a shard sends) with top_p and min_p cuts and a
    256-id ring, at two temperatures."""
    import quasar_b200 as q
    B = 4
    logits, hist = gpu_inputs(O.SYNTH_NORMAL, 19, B, V_FULL, 2.0, H=256, hist_seed=20)
    seeds = _seeds(B, 1900)
    for T in (0.6, 1.4):
        prm = O.make_params(1, temperature=T, top_k=256, top_p=0.9, min_p=0.01, repeat_penalty=1.2)
        assert _shards(B, V_FULL, prm, 256) == 8
        got = run_gpu(logits, prm, seeds, hist=hist)
        res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
        print(assert_parity(*got, res, rng_ref, max_mismatch_frac=0.25))
        _same_as_unsplit(got, run_gpu(logits, prm, seeds, hist=hist, flags=q.FLAG_NO_SPLIT), res)


def test_split_tied_logits():
    """Logits quantised to 7 values: each shard of 18,992 columns holds ~2,700
    elements tied at the row maximum, more than a CTA lists, so the CTAs take
    their exact top k by a radix select over (p, id) keys; ties go to the
    lowest ids, as the reference's sort leaves them."""
    import torch
    B = 4
    base = torch.randint(-3, 4, (B, V_FULL), generator=torch.Generator().manual_seed(0)).float()
    logits = base.cuda()
    seeds = _seeds(B, 31)
    for prm in (O.make_params(1, temperature=1.0, top_k=7), O.make_params(1, temperature=0.5, top_k=40, top_p=0.5),
                O.make_params(1, temperature=0.0)):
        assert _shards(B, V_FULL, prm) == 8
        got = run_gpu(logits, prm, seeds)
        res, rng_ref = run_oracle(base.numpy(), prm, seeds)
        assert_parity(*got, res, rng_ref, max_mismatch_frac=0.0)


def test_split_long_history_rings():
    """Rings of 512 slots, partly filled, strong penalty (penalized columns
    in every shard)."""
    import torch
    B, H = 3, 512
    logits, hist = gpu_inputs(O.SYNTH_ZIPF, 5, B, V_FULL, 1.1, H=H, hist_seed=6)
    hist_len = torch.tensor([512, 300, 17], dtype=torch.int32, device="cuda")
    hist_head = torch.tensor([5, 500, 0], dtype=torch.int32, device="cuda")
    seeds = _seeds(B, 512)
    for prm in (O.make_params(1, temperature=1.0, top_k=50, repeat_penalty=1.5),
                O.make_params(1, temperature=0.0, repeat_penalty=1.5)):
        assert _shards(B, V_FULL, prm, H) == 8
        got = run_gpu(logits, prm, seeds, hist=hist, hist_len=hist_len, hist_head=hist_head)
        res, rng_ref = run_oracle(logits, prm, seeds, hist=hist, hist_len=hist_len, hist_head=hist_head)
        assert_parity(*got, res, rng_ref, max_mismatch_frac=0.34)


def test_split_uneven_vocab_and_unsplit_shapes():
    """V = 20000 splits into 8 shards of 2500; V = 20001 (no shard width that
    is a multiple of 4) and rows cut by min-p alone stay on one CTA per row.
    All match the reference."""
    import quasar_b200 as q
    B = 5
    cases = [(20000, O.make_params(1, temperature=0.9, top_k=40, top_p=0.95, repeat_penalty=1.2), 8),
             (20001, O.make_params(1, temperature=0.9, top_k=40, top_p=0.95, repeat_penalty=1.2), 0),
             (V_FULL, O.make_params(1, temperature=0.9, min_p=0.05, repeat_penalty=1.2), 0)]
    for V, prm, G in cases:
        logits, hist = gpu_inputs(O.SYNTH_NORMAL, 23, B, V, 2.5, H=32, hist_seed=24)
        assert _shards(B, V, prm, 32) == G, V
        seeds = _seeds(B, V)
        got = run_gpu(logits, prm, seeds, hist=hist)
        res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
        assert_parity(*got, res, rng_ref, max_mismatch_frac=0.2)
        assert q.split_shards(B, V, params=prm, hist_cap=32, flags=q.FLAG_NO_SPLIT) == 0


def test_small_batch_ignores_workspace_and_no_alloc_entry():
    """The fused kernel uses no workspace: a caller workspace of the one-CTA
    size, the library's own and the no-allocation entry give the same
    results, all matching the reference."""
    import torch
    import quasar_b200 as q
    B, H = 2, 64
    prm = O.make_params(1, temperature=0.7, top_k=20, top_p=0.8, repeat_penalty=1.1)
    logits, hist = gpu_inputs(O.SYNTH_NORMAL, 99, B, V_FULL, 3.0, H=H, hist_seed=98)
    seeds = _seeds(B, 9900)
    res, rng_ref = run_oracle(logits, prm, seeds, hist=hist)
    nbytes = q.workspace_bytes(B, H)
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device="cuda")
    ws = ws[(-ws.data_ptr()) % 256:][:nbytes]
    outs = []
    for mode in ("caller", "library", "noalloc"):
        rng = torch.from_numpy(seeds.view(np.int64).copy()).cuda()
        diag = torch.zeros(B, 4, dtype=torch.int32, device="cuda")
        out = torch.empty(B, dtype=torch.int32, device="cuda")
        if mode == "noalloc":
            hp = q.SampleParams(*(float(prm[0][f]) for f in ("temperature", "top_p", "min_p", "repeat_penalty")),
                                int(prm[0]["top_k"]), 0)
            import ctypes
            rc = q.lib().quasar_sampler_pick_batch_noalloc(
                ctypes.c_void_p(logits.data_ptr()), V_FULL, B, V_FULL, None, ctypes.byref(hp),
                ctypes.c_void_p(rng.data_ptr()), ctypes.c_void_p(hist.data_ptr()), H, None, None, 0,
                ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(diag.data_ptr()), 0,
                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            assert rc == 0
        else:
            q.pick_batch(logits, rng, params=prm[:1], hist=hist, diag=diag, out=out,
                         workspace=ws if mode == "caller" else None)
        torch.cuda.synchronize()
        got = (out.cpu().numpy(), diag.cpu().numpy().view(q.DIAG_DTYPE).reshape(B), rng.cpu().numpy().view(np.uint64))
        assert_parity(*got, res, rng_ref, max_mismatch_frac=0.5)
        outs.append(got)
    for o in outs[1:]:
        assert np.array_equal(o[0], outs[0][0]) and np.array_equal(o[2], outs[0][2])
        assert np.array_equal(o[1]["p_chosen"].view(np.uint32), outs[0][1]["p_chosen"].view(np.uint32))
