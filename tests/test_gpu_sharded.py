"""Vocab-sharded sampling on the GPU (quasar_shard_* through
quasar_b200.VocabShardedSampler / CudaShardPhases), against the unsharded
reference sampler on the full rows.

* emulated shards: G column slices of one matrix on one GPU, the gathers done
  by placing each shard's output at its rank's offset;
* NCCL: two processes on two GPUs (skipped with fewer GPUs)."""
import datetime
import os
import socket

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import V_FULL, assert_parity

pytestmark = pytest.mark.gpu

B, H, K = 64, 64, 40


def _params(B):
    prm = O.make_params(B, temperature=0.8, top_k=K, top_p=0.9, repeat_penalty=1.1)
    prm["temperature"][::5] = 0.0     # greedy rows
    prm["top_k"][1::5] = 1            # top_k = 1: one PRNG step, bit-exact id
    prm["min_p"][2::5] = 0.05
    prm["top_p"][3::5] = 1.0
    return prm


def _state(B):
    seeds = np.arange(1, B + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    hist_len = np.full(B, H - 3, dtype=np.int32)
    hist_head = (np.arange(B, dtype=np.int32) * 5) % H
    return seeds, hist_len, hist_head


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _check(ids, diag, rng_after, hist_after, len_after, logits_np, hist_np, prm, seeds, hist_len, hist_head):
    import quasar_b200 as q
    ref, ref_rng = O.pick_rows(logits_np, prm, seeds, hist=hist_np.copy(), hist_len=hist_len.copy(),
                               hist_head=hist_head.copy())
    assert_parity(ids, diag.view(q.DIAG_DTYPE).reshape(-1), rng_after.view(np.uint64), ref, ref_rng)
    greedy = prm["temperature"] <= 0
    assert np.array_equal(ids[greedy], ref["id"][greedy])
    top1 = (prm["top_k"] == 1) & ~greedy
    assert np.array_equal(ids[top1], ref["id"][top1])
    for r in range(ids.size):
        slot = (hist_head[r] + hist_len[r]) % H
        assert hist_after[r, slot] == ids[r] and len_after[r] == hist_len[r] + 1


def _emulate(logits, hist, prm, seeds, hist_len, hist_head, G, k=K):
    """G column slices of one matrix on one GPU, the gathers done by placing
    each shard's output at its rank's offset. Returns the numpy results."""
    import torch
    import quasar_b200 as q
    from quasar_b200.sharded import STAT_BYTES, CudaShardPhases
    nb = logits.shape[0]
    Hh = 0 if hist is None else hist.shape[1]
    dev = logits.device
    d_params = q.params_to_device(prm, dev)
    rng = torch.from_numpy(seeds.view(np.int64).copy()).to(dev)
    th = None if hist is None else hist.clone()
    tl = None if hist is None else torch.from_numpy(hist_len).to(dev)
    thd = None if hist is None else torch.from_numpy(hist_head).to(dev)
    vs = V_FULL // G
    ph = CudaShardPhases()
    stream = torch.cuda.current_stream()
    wsb = q.workspace_bytes(nb, Hh)
    wss = [torch.empty(wsb + 256, dtype=torch.uint8, device=dev) for _ in range(G)]
    wss = [w[(-w.data_ptr()) % 256:][:wsb] for w in wss]
    all_stats = torch.empty(G * nb * STAT_BYTES, dtype=torch.uint8, device=dev)
    all_cand = torch.empty(G * nb * k, dtype=torch.int64, device=dev)
    for g in range(G):
        view = logits[:, g * vs:(g + 1) * vs]
        ph.stats(view, g * vs, None, d_params, th, tl, thd, all_stats[g * nb * STAT_BYTES:(g + 1) * nb * STAT_BYTES],
                 wss[g], stream)
    for g in range(G):
        view = logits[:, g * vs:(g + 1) * vs]
        ph.candidates(view, g * vs, None, d_params, th, tl, thd, all_stats, G, g, k,
                      all_cand[g * nb * k:(g + 1) * nb * k], wss[g], stream)
    out = torch.empty(nb, dtype=torch.int32, device=dev)
    diag = torch.zeros(nb, 4, dtype=torch.int32, device=dev)
    ph.finish(all_cand, all_stats, G, k, nb, None, d_params, rng, th, tl, thd, th is not None, out, diag, stream)
    torch.cuda.synchronize()
    return (out.cpu().numpy(), diag.cpu().numpy(), rng.cpu().numpy(),
            None if th is None else th.cpu().numpy(), None if tl is None else tl.cpu().numpy())


@pytest.mark.parametrize("G", [2, 4, 8])
def test_emulated_shards_match_unsharded(G):
    from tests.helpers import gpu_inputs
    logits, hist = gpu_inputs(O.SYNTH_NORMAL, 77, B, V_FULL, 3.0, H=H, hist_seed=78)
    prm = _params(B)
    seeds, hist_len, hist_head = _state(B)
    ids, diag, rng, th, tl = _emulate(logits, hist, prm, seeds, hist_len, hist_head, G)
    _check(ids, diag, rng, th, tl, logits.cpu().numpy(), hist.cpu().numpy(), prm, seeds, hist_len, hist_head)


def test_config4_emulated_full_batch():
    """BASELINE.json config 4 as stated: 8192 rows, 8 shards of 18,992
    columns, N(0,3), top_k 40, top_p 0.9, temperature 0.8, no history; every
    row against the unsharded reference."""
    import quasar_b200 as q
    from tests.helpers import gpu_inputs
    nb, G = 8192, 8
    logits, _ = gpu_inputs(O.SYNTH_NORMAL, 3, nb, V_FULL, 3.0)
    prm = O.make_params(nb, temperature=0.8, top_k=K, top_p=0.9)
    seeds = np.arange(nb, dtype=np.uint64) + np.uint64(5000)
    ids, diag, rng, _, _ = _emulate(logits, None, prm, seeds, None, None, G)
    reps = []
    for c0 in range(0, nb, 1024):
        sl = slice(c0, c0 + 1024)
        ref, ref_rng = O.pick_rows(logits[sl].cpu().numpy(), prm[sl], seeds[sl])
        reps.append(assert_parity(ids[sl], diag[sl].view(q.DIAG_DTYPE).reshape(-1), rng[sl].view(np.uint64),
                                  ref, ref_rng))
    assert sum(r["mismatched_near_boundary"] for r in reps) <= nb // 100


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _nccl_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        import quasar_b200 as qb
        vs = V_FULL // world
        logits = torch.empty(B, vs, dtype=torch.float32, device=dev)
        full = torch.empty(B, V_FULL, dtype=torch.float32, device=dev)
        qb.synth_logits(qb.SYNTH_NORMAL, 79, 0, B, V_FULL, 3.0, full)
        logits.copy_(full[:, rank * vs:(rank + 1) * vs])
        hist = torch.empty(B, H, dtype=torch.int32, device=dev)
        qb.synth_hist(80, 0, B, H, V_FULL, hist)
        prm = _params(B)
        seeds, hist_len, hist_head = _state(B)
        rng = torch.from_numpy(seeds.view(np.int64).copy()).to(dev)
        tl, thd = torch.from_numpy(hist_len).to(dev), torch.from_numpy(hist_head).to(dev)
        diag = torch.zeros(B, 4, dtype=torch.int32, device=dev)
        hist0 = hist.clone()
        out = qb.VocabShardedSampler(K).pick(logits, rank * vs, rng, d_params=qb.params_to_device(prm, dev),
                                             hist=hist, hist_len=tl, hist_head=thd, record=True, diag=diag)
        torch.cuda.synchronize()
        q.put((rank, out.cpu().numpy(), diag.cpu().numpy(), rng.cpu().numpy(), hist.cpu().numpy(),
               tl.cpu().numpy(), hist0.cpu().numpy(), full.cpu().numpy() if rank == 0 else None))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_nccl_matches_unsharded():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r = q.get(timeout=300)
        res[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for a, b in zip(res[0][:5], res[1][:5]):
        assert np.array_equal(a, b), "ranks disagree"
    ids, diag, rng_after, hist_after, len_after, hist0, full = res[0]
    seeds, hist_len, hist_head = _state(B)
    _check(ids, diag, rng_after, hist_after, len_after, full, hist0, _params(B), seeds, hist_len, hist_head)


@pytest.mark.parametrize("G", [2, 8])
def test_emulated_shards_min_p_rows_without_top_k(G):
    """Rows with top_k 0 and a min-p floor: every shard sends all of its keys
    at or above the floor of the global max, so the merge is exact; one row
    whose floor lets too many keys through a shard comes back as -1."""
    import quasar_b200 as q
    from tests.helpers import gpu_inputs
    nb = 48
    logits, hist = gpu_inputs(O.SYNTH_NORMAL, 91, nb, V_FULL, 3.0, H=H, hist_seed=92)
    prm = O.make_params(nb, temperature=0.9, top_k=0, top_p=0.95, min_p=0.2, repeat_penalty=1.1)
    prm["min_p"][1::4] = 0.1
    prm["top_p"][2::4] = 1.0
    prm["min_p"][nb - 1] = 1e-30   # this row's floor lets thousands of keys through every shard
    seeds, hist_len, hist_head = _state(nb)
    # k = 128 keys per shard: room for every min-p survivor of the other rows
    ids, diag, rng, th, tl = _emulate(logits, hist, prm, seeds, hist_len, hist_head, G, k=128)
    assert ids[nb - 1] == -1
    keep = np.arange(nb - 1)
    ref, ref_rng = O.pick_rows(logits.cpu().numpy()[keep], prm[keep], seeds[keep], hist=hist.cpu().numpy()[keep],
                               hist_len=hist_len[keep], hist_head=hist_head[keep])
    assert_parity(ids[keep], diag[keep].view(q.DIAG_DTYPE).reshape(-1), rng[keep].view(np.uint64), ref, ref_rng)
    assert (ids[keep] >= 0).all()


@pytest.mark.parametrize("G", [2, 8])
def test_emulated_shards_top_k_rows_whose_bound_overflows(G):
    """Top-k rows whose per-thread-maxima bound lets more elements through a
    shard than its candidate buffer holds (the one-warp kernel at G = 8 holds
    512, the CTA kernel at G = 2 holds 4096): logits quantised to 7 values,
    so every thread's maximum ties and a shard holds thousands of elements at
    the row maximum, and flat rows with top_k = 256. Each shard then finds
    its exact top k by a radix select over the whole shard; ties go to the
    lowest ids, as the reference's sort leaves them."""
    import torch
    import quasar_b200 as q
    nb = 8
    base = torch.randint(-3, 4, (nb, V_FULL), generator=torch.Generator().manual_seed(5)).float()
    logits = base.cuda()
    hist = torch.randint(0, V_FULL, (nb, H), generator=torch.Generator().manual_seed(6)).int().cuda()
    prm = O.make_params(nb, temperature=1.0, top_k=40, top_p=0.95, repeat_penalty=1.2)
    prm["top_k"][1::2] = 256
    prm["temperature"][1::2] = 3.0   # flat rows: the top 256 are ties and near-ties
    prm["min_p"][2::4] = 0.5
    seeds, hist_len, hist_head = _state(nb)
    ids, diag, rng, th, tl = _emulate(logits, hist, prm, seeds, hist_len, hist_head, G, k=256)
    ref, ref_rng = O.pick_rows(base.numpy(), prm, seeds, hist=hist.cpu().numpy(), hist_len=hist_len.copy(),
                               hist_head=hist_head.copy())
    assert (ids >= 0).all(), ids
    assert_parity(ids, diag.view(q.DIAG_DTYPE).reshape(-1), rng.view(np.uint64), ref, ref_rng, max_mismatch_frac=0.0)
