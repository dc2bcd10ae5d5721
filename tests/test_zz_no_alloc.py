"""quasar_sampler_pick_batch_noalloc (workspace in a fixed device array) against
quasar_sampler_pick_batch on the same inputs: two calls in a row from the same
starting state must give the same ids, reports, PRNG states and history
rings. Collected last so it also runs after every other GPU test in the same
process; it passes on its own as well."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import gpu_inputs

B, V, H = 512, 151936, 64


def _noalloc(lib, logits, d_params, rng, hist, hist_len, hist_head, out, diag, stream):
    P = ctypes.c_void_p
    return lib.quasar_sampler_pick_batch_noalloc(
        P(logits.data_ptr()), logits.stride(0), logits.shape[0], logits.shape[1], P(d_params.data_ptr()),
        None, P(rng.data_ptr()), P(hist.data_ptr()), hist.shape[1], P(hist_len.data_ptr()),
        P(hist_head.data_ptr()), 1, P(out.data_ptr()), P(diag.data_ptr()), 0, P(stream.cuda_stream))


def test_noalloc_rejects_oversize_without_gpu_work():
    import quasar_b200 as q
    lib = q.lib()
    limit = q.QUASAR_NOALLOC_WORKSPACE_BYTES
    rows = 1
    while lib.quasar_sampler_workspace_bytes(rows, 256) <= limit:
        rows *= 2
    P = ctypes.c_void_p
    rc = lib.quasar_sampler_pick_batch_noalloc(P(16), V, rows, V, P(16), None, P(16), P(16), 256, P(16),
                                               P(16), 1, P(16), None, 0, None)
    assert rc == -6  # QUASAR_EOVERFLOW, before any pointer is touched


@pytest.mark.gpu
def test_noalloc_matches_pick_batch_two_calls():
    import torch
    import quasar_b200 as q
    lib = q.lib()
    assert lib.quasar_sampler_workspace_bytes(B, H) <= q.QUASAR_NOALLOC_WORKSPACE_BYTES
    logits, hist0 = gpu_inputs(O.SYNTH_NORMAL, 21, B, V, 3.0, H=H, hist_seed=22)
    temps = O.synth_uniform(23, 0, B, 0.2, 1.5)
    prm = q.make_params(B, temperature=temps, top_p=0.95, min_p=0.05, repeat_penalty=1.1)
    prm["temperature"][::7] = 0.0          # some greedy rows
    prm["min_p"][3::11] = 0.0              # some rows on the exact-select path
    prm["top_p"][3::11] = 1.0              # (pure multinomial: no bound keeps them off it)
    d_params = q.params_to_device(prm, logits.device)
    seeds = np.arange(1, B + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    stream = torch.cuda.current_stream()

    def state():
        rng = torch.from_numpy(seeds.view(np.int64).copy()).cuda()
        hist = hist0.clone()
        hist_len = torch.full((B,), H - 3, dtype=torch.int32, device="cuda")  # two rows of growth
        hist_head = torch.arange(B, dtype=torch.int32, device="cuda") % H
        return rng, hist, hist_len, hist_head

    ra, ha, la, hda = state()
    rb, hb, lb, hdb = state()
    for call in range(2):
        out_a = torch.empty(B, dtype=torch.int32, device="cuda")
        out_b = torch.empty(B, dtype=torch.int32, device="cuda")
        diag_a = torch.zeros(B, 4, dtype=torch.int32, device="cuda")
        diag_b = torch.zeros(B, 4, dtype=torch.int32, device="cuda")
        q.pick_batch(logits, ra, d_params=d_params, hist=ha, hist_len=la, hist_head=hda, record=True,
                     out=out_a, diag=diag_a, stream=stream)
        assert _noalloc(lib, logits, d_params, rb, hb, lb, hdb, out_b, diag_b, stream) == 0
        torch.cuda.synchronize()
        ia, ib = out_a.cpu().numpy(), out_b.cpu().numpy()
        assert np.array_equal(ia, ib), f"call {call}: ids differ in rows {np.nonzero(ia != ib)[0][:10]}"
        da = diag_a.cpu().numpy().view(q.DIAG_DTYPE).reshape(B)
        db = diag_b.cpu().numpy().view(q.DIAG_DTYPE).reshape(B)
        assert np.array_equal(da["n_kept"], db["n_kept"]) and np.array_equal(da["path"], db["path"])
        # the same kernels on the same inputs: the reported floats agree bit for bit
        assert np.array_equal(db["p_chosen"].view(np.uint32), da["p_chosen"].view(np.uint32))
        assert np.array_equal(db["inv_sum"].view(np.uint32), da["inv_sum"].view(np.uint32))
        assert set(np.unique(da["path"])) >= {0, 1, 2}
        for x, y in ((ra, rb), (ha, hb), (la, lb), (hda, hdb)):
            assert torch.equal(x, y), f"call {call}: sampler state differs"


def test_noalloc_checks_arguments_before_size():
    """A call that is both oversize and malformed reports the malformed
    argument, as quasar_sampler_pick_batch would (no GPU work either way)."""
    import quasar_b200 as q
    lib = q.lib()
    P = ctypes.c_void_p
    rows = 1 << 20
    rc = lib.quasar_sampler_pick_batch_noalloc(P(16), V - 1, rows, V, P(16), None, P(16), P(16), 256, P(16),
                                               P(16), 1, P(16), None, 0, None)  # ld < V
    assert rc == -1  # QUASAR_EINVAL
    rc = lib.quasar_sampler_pick_batch_noalloc(P(16), V, rows, V, P(16), None, None, P(16), 256, P(16),
                                               P(16), 1, P(16), None, 0, None)  # no rng
    assert rc == -1


@pytest.mark.gpu
def test_noalloc_host_params_without_history_two_calls():
    """The other argument path: one host parameter record for every row and no
    history ring (hist_cap 0), two calls in a row against pick_batch."""
    import torch
    import quasar_b200 as q
    lib = q.lib()
    n = 256
    logits, _ = gpu_inputs(O.SYNTH_NORMAL, 31, n, V, 3.0)
    hp = q.SampleParams(0.9, 0.9, 0.05, 1.0, 0, 0)
    seeds = np.arange(7, n + 7, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    ra = torch.from_numpy(seeds.view(np.int64).copy()).cuda()
    rb = ra.clone()
    stream = torch.cuda.current_stream()
    P = ctypes.c_void_p
    for call in range(2):
        out_a = torch.empty(n, dtype=torch.int32, device="cuda")
        out_b = torch.empty(n, dtype=torch.int32, device="cuda")
        diag_a = torch.zeros(n, 4, dtype=torch.int32, device="cuda")
        diag_b = torch.zeros(n, 4, dtype=torch.int32, device="cuda")
        q.pick_batch(logits, ra, params=q.make_params(1, temperature=0.9, top_p=0.9, min_p=0.05),
                     out=out_a, diag=diag_a, stream=stream)
        rc = lib.quasar_sampler_pick_batch_noalloc(
            P(logits.data_ptr()), logits.stride(0), n, V, None, ctypes.byref(hp), P(rb.data_ptr()), None, 0,
            None, None, 0, P(out_b.data_ptr()), P(diag_b.data_ptr()), 0, P(stream.cuda_stream))
        assert rc == 0
        torch.cuda.synchronize()
        assert torch.equal(out_a, out_b), f"call {call}: ids differ"
        assert torch.equal(diag_a, diag_b), f"call {call}: reports differ"
        assert torch.equal(ra, rb), f"call {call}: PRNG states differ"
