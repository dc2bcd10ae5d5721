"""Vocab-sharded sampling, host logic on CPU: two gloo ranks each hold half
of the vocab columns and run quasar_b200.VocabShardedSampler with the numpy
stand-in phases (tests/shard_cpu.py). Both ranks must end with the same ids,
PRNG states and history rings, and those must match the unsharded reference
sampler on the full rows (ids within the stochastic tolerance)."""
import datetime
import os
import socket

import numpy as np
import pytest

from oracle import oracle as O

V, B, H, K = 151936, 12, 64, 40


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _inputs():
    logits = O.synth_logits(O.SYNTH_NORMAL, 404, 0, B, V, 3.0)
    hist = O.synth_hist(405, 0, B, H, V)
    prm = O.make_params(B, temperature=0.8, top_k=K, top_p=0.9, repeat_penalty=1.1)
    prm["temperature"][::4] = 0.0                 # greedy rows
    prm["top_k"][1::4] = 20
    prm["min_p"][2::4] = 0.05
    seeds = np.arange(1, B + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    hist_len = np.full(B, H - 2, dtype=np.int32)
    hist_head = (np.arange(B, dtype=np.int32) * 7) % H
    return logits, hist, prm, seeds, hist_len, hist_head


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import quasar_b200 as qb
        from tests.shard_cpu import CpuShardPhases
        logits, hist, prm, seeds, hist_len, hist_head = _inputs()
        vs = V // world
        shard = torch.from_numpy(np.ascontiguousarray(logits[:, rank * vs:(rank + 1) * vs]))
        rng = torch.from_numpy(seeds.view(np.int64).copy())
        th, tl, thd = torch.from_numpy(hist.copy()), torch.from_numpy(hist_len.copy()), torch.from_numpy(hist_head.copy())
        d_params = torch.from_numpy(prm.view(np.uint8).copy())
        diag = torch.zeros(B, 4, dtype=torch.int32)
        smp = qb.VocabShardedSampler(K, phases=CpuShardPhases())
        out = smp.pick(shard, rank * vs, rng, d_params=d_params, hist=th, hist_len=tl, hist_head=thd, record=True,
                       diag=diag)
        q.put((rank, out.numpy().copy(), rng.numpy().copy(), th.numpy().copy(), tl.numpy().copy(),
               thd.numpy().copy(), diag.numpy().copy()))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_match_unsharded_reference():
    pytest.importorskip("torch")
    import torch.multiprocessing as mp
    from tests.helpers import assert_parity
    import quasar_b200 as qb
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r = q.get(timeout=300)
        res[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for a, b in zip(res[0], res[1]):
        assert np.array_equal(a, b), "ranks disagree"
    ids, rng_after, hist_after, len_after, head_after, diag = res[0]
    logits, hist, prm, seeds, hist_len, hist_head = _inputs()
    ref_hist, ref_len, ref_head = hist.copy(), hist_len.copy(), hist_head.copy()
    ref, ref_rng = O.pick_rows(logits, prm, seeds, hist=ref_hist, hist_len=ref_len, hist_head=ref_head)
    assert_parity(ids, diag.view(qb.DIAG_DTYPE).reshape(B), rng_after.view(np.uint64), ref, ref_rng)
    # the rings advanced the same way (the record of sample.c:83-92)
    for r in range(B):
        if ids[r] == ref["id"][r]:
            cap = H
            L0, H0 = hist_len[r], hist_head[r]
            slot = (H0 + L0) % cap if L0 < cap else H0
            assert hist_after[r, slot] == ids[r]
            assert len_after[r] == min(L0 + 1, cap)
