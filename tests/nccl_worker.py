"""Child processes of tests/test_gpu_nccl.py: each run is one rank of a
libquasar_cuda NCCL communicator (quasar_nccl_* / quasar_shard_pick), kept out
of the pytest process so that a communicator problem can only end a child.
NVLS is off (NCCL_NVLS_ENABLE=0), peers use plain NCCL transports.

  python -m tests.nccl_worker pick   RANK WORLD ID_FILE OUT_FILE   vocab-sharded batch, results to OUT_FILE
  python -m tests.nccl_worker nojoin OUT_FILE                      rank 0 of 2 whose peer never joins
  python -m tests.nccl_worker leave  RANK WORLD ID_FILE OUT_FILE   rank 1 leaves after step 1; rank 0 runs step 2
"""
from __future__ import annotations

import json
import os
import sys
import time

os.environ.setdefault("NCCL_NVLS_ENABLE", "0")

import numpy as np  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

V = 151936
B, H, K = 64, 64, 40


def params(n):
    """Config-4 parameters (top_k 40, top_p 0.9, T 0.8) with greedy, top_k=1,
    min-p-only and top-p-off rows mixed in, repeat penalty 1.1."""
    from oracle import oracle as O
    prm = O.make_params(n, temperature=0.8, top_k=K, top_p=0.9, repeat_penalty=1.1)
    prm["temperature"][::5] = 0.0      # greedy
    prm["top_k"][1::5] = 1             # top_k = 1
    prm["top_k"][2::5] = 0             # min-p only (the floor of the global max; ~10 survivors)
    prm["min_p"][2::5] = 0.2
    prm["top_p"][3::5] = 1.0
    return prm


def state(n):
    seeds = np.arange(1, n + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
    hist_len = np.full(n, H - 3, dtype=np.int32)
    hist_head = (np.arange(n, dtype=np.int32) * 5) % H
    return seeds, hist_len, hist_head


def read_id(path, timeout=60.0):
    t0 = time.time()
    while time.time() - t0 < timeout:
        if os.path.exists(path) and os.path.getsize(path) == 128:
            with open(path, "rb") as f:
                return f.read()
        time.sleep(0.05)
    raise TimeoutError("no communicator id")


def make_comm(rank, world, id_file, timeout_ms=30000):
    import quasar_b200 as q
    if rank == 0:
        uid = q.NcclCommunicator.unique_id()
        tmp = id_file + ".tmp"
        with open(tmp, "wb") as f:
            f.write(uid)
        os.replace(tmp, id_file)
    else:
        uid = read_id(id_file)
    return q.NcclCommunicator(world, rank, uid, timeout_ms=timeout_ms)


def inputs(rank, world, dev):
    import torch
    import quasar_b200 as q
    vs = V // world
    full = torch.empty(B, V, dtype=torch.float32, device=dev)
    q.synth_logits(q.SYNTH_NORMAL, 79, 0, B, V, 3.0, full)
    shard = full[:, rank * vs:(rank + 1) * vs].contiguous()
    hist = torch.empty(B, H, dtype=torch.int32, device=dev)
    q.synth_hist(80, 0, B, H, V, hist)
    return full, shard, hist, vs


def run_pick(rank, world, id_file, out_file):
    import torch
    import quasar_b200 as q
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    comm = make_comm(rank, world, id_file)
    full, shard, hist, vs = inputs(rank, world, dev)
    prm = params(B)
    seeds, hist_len, hist_head = state(B)
    rng = torch.from_numpy(seeds.view(np.int64).copy()).to(dev)
    tl, thd = torch.from_numpy(hist_len).to(dev), torch.from_numpy(hist_head).to(dev)
    hist0 = hist.clone()
    diag = torch.zeros(B, 4, dtype=torch.int32, device=dev)
    smp = q.NcclShardedSampler(comm, K)
    out = smp.pick(shard, rank * vs, rng, d_params=q.params_to_device(prm, dev), hist=hist, hist_len=tl,
                   hist_head=thd, record=True, diag=diag)
    comm.wait(timeout_ms=30000)
    np.savez(out_file, ids=out.cpu().numpy(), diag=diag.cpu().numpy(), rng=rng.cpu().numpy(),
             hist=hist.cpu().numpy(), len=tl.cpu().numpy(), hist0=hist0.cpu().numpy(),
             full=full.cpu().numpy() if rank == 0 else np.zeros(1, np.float32))
    comm.close()


def run_nojoin(out_file):
    """Rank 0 of a two-rank communicator whose rank 1 never starts: the join
    must end with QUASAR_ENCCL within its time limit, and the process's CUDA
    context must stay usable."""
    import torch
    import quasar_b200 as q
    torch.cuda.set_device(0)
    uid = q.NcclCommunicator.unique_id()
    t0 = time.time()
    status = 0
    try:
        q.NcclCommunicator(2, 0, uid, timeout_ms=3000)
    except q.QuasarError as e:
        status = e.status
    elapsed = time.time() - t0
    # the context still works: a small batch through the sampler
    logits = torch.empty(4, 1000, dtype=torch.float32, device="cuda")
    q.synth_logits(q.SYNTH_NORMAL, 1, 0, 4, 1000, 2.0, logits)
    rng = torch.arange(1, 5, dtype=torch.int64, device="cuda")
    ids = q.pick_batch(logits, rng, params=q.make_params(1, temperature=0.0)).cpu().numpy()
    ok = bool((ids == logits.argmax(dim=1).int().cpu().numpy()).all())
    with open(out_file, "w") as f:
        json.dump({"status": status, "elapsed": elapsed, "context_ok": ok}, f)


def run_leave(rank, world, id_file, out_file):
    """Two ranks sample one batch together; then rank 1 leaves (aborts its
    communicator and exits, with nothing of its own in flight) and rank 0
    samples the next batch: its wait must end with QUASAR_ENCCL, the abort
    must end its kernel still waiting for the peer, and its context must stay
    usable."""
    import torch
    import quasar_b200 as q
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    comm = make_comm(rank, world, id_file, timeout_ms=5000)
    full, shard, hist, vs = inputs(rank, world, dev)
    prm = params(B)
    seeds, hist_len, hist_head = state(B)
    rng = torch.from_numpy(seeds.view(np.int64).copy()).to(dev)
    smp = q.NcclShardedSampler(comm, K)
    dprm = q.params_to_device(prm, dev)
    smp.pick(shard, rank * vs, rng, d_params=dprm)
    comm.wait(timeout_ms=30000)
    res = {"step1": "ok"}
    if rank == 1:
        comm.abort()
        with open(out_file, "w") as f:
            json.dump(res, f)
        os._exit(0)
    time.sleep(1.0)  # rank 1 is gone
    t0 = time.time()
    status = 0
    try:
        smp.pick(shard, rank * vs, rng, d_params=dprm)
        comm.wait(timeout_ms=5000)
    except q.QuasarError as e:
        status = e.status
    res["status"] = status
    res["elapsed"] = time.time() - t0
    logits = torch.empty(4, 1000, dtype=torch.float32, device=dev)
    q.synth_logits(q.SYNTH_NORMAL, 1, 0, 4, 1000, 2.0, logits)
    r4 = torch.arange(1, 5, dtype=torch.int64, device=dev)
    ids = q.pick_batch(logits, r4, params=q.make_params(1, temperature=0.0)).cpu().numpy()
    res["context_ok"] = bool((ids == logits.argmax(dim=1).int().cpu().numpy()).all())
    with open(out_file, "w") as f:
        json.dump(res, f)
    os._exit(0)


if __name__ == "__main__":
    mode = sys.argv[1]
    if mode == "pick":
        run_pick(int(sys.argv[2]), int(sys.argv[3]), sys.argv[4], sys.argv[5])
    elif mode == "nojoin":
        run_nojoin(sys.argv[2])
    elif mode == "leave":
        run_leave(int(sys.argv[2]), int(sys.argv[3]), sys.argv[4], sys.argv[5])
    else:
        raise SystemExit("unknown mode " + mode)
