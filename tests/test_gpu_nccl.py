"""quasar_shard_pick over libquasar_cuda's own NCCL communicators
(quasar_nccl_*), through the C ABI, each rank a child process
(tests/nccl_worker.py, NVLS off):

* one rank: the C entry on a one-rank communicator equals the unsharded
  reference on every row (the exchanges degenerate to copies);
* a rank that never joins: the join ends with QUASAR_ENCCL inside its time
  limit and the CUDA context stays usable (no GPU work is involved);
* two ranks (skipped with fewer GPUs): the vocab split over two GPUs equals
  the unsharded reference, and a rank that leaves between steps ends the
  other's next batch with QUASAR_ENCCL through the time limit and abort."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle as O
from tests import nccl_worker as W
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import quasar_b200 as q
    if q.lib().quasar_nccl_available() != 0:
        pytest.skip("no NCCL library to load")


def _env():
    env = dict(os.environ)
    env["NCCL_NVLS_ENABLE"] = "0"
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    return env


def _spawn(*args):
    return subprocess.Popen([sys.executable, "-m", "tests.nccl_worker", *map(str, args)], cwd=ROOT, env=_env(),
                            stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)


def _finish(procs, timeout=240):
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
            raise AssertionError("rank timed out:\n" + out[-3000:])
        outs.append(out)
        assert p.returncode == 0, out[-3000:]
    return outs


def _check_against_reference(res):
    import quasar_b200 as q
    prm = W.params(W.B)
    seeds, hist_len, hist_head = W.state(W.B)
    ref, ref_rng = O.pick_rows(res["full"], prm, seeds, hist=res["hist0"].copy(), hist_len=hist_len.copy(),
                               hist_head=hist_head.copy())
    ids = res["ids"]
    assert_parity(ids, res["diag"].view(q.DIAG_DTYPE).reshape(-1), res["rng"].view(np.uint64), ref, ref_rng)
    greedy = prm["temperature"] <= 0
    assert np.array_equal(ids[greedy], ref["id"][greedy])
    assert (ids >= 0).all(), "a row the shards should cover came back -1"
    for r in range(W.B):
        slot = (hist_head[r] + hist_len[r]) % W.H
        assert res["hist"][r, slot] == ids[r] and res["len"][r] == hist_len[r] + 1


def test_single_rank_c_entry_matches_unsharded(tmp_path):
    idf, out = str(tmp_path / "id"), str(tmp_path / "r0.npz")
    _finish([_spawn("pick", 0, 1, idf, out)])
    _check_against_reference(dict(np.load(out)))


def test_rank_that_never_joins_ends_with_encl(tmp_path):
    out = str(tmp_path / "nojoin.json")
    _finish([_spawn("nojoin", out)], timeout=120)
    with open(out) as f:
        res = json.load(f)
    assert res["status"] == -5, res  # QUASAR_ENCCL
    assert res["elapsed"] < 30.0, res
    assert res["context_ok"], res


def _two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


def test_two_ranks_c_entry_matches_unsharded(tmp_path):
    _two_gpus()
    idf = str(tmp_path / "id")
    outs = [str(tmp_path / f"r{r}.npz") for r in range(2)]
    _finish([_spawn("pick", r, 2, idf, outs[r]) for r in range(2)])
    r0, r1 = dict(np.load(outs[0])), dict(np.load(outs[1]))
    for key in ("ids", "diag", "rng", "hist", "len"):
        assert np.array_equal(r0[key], r1[key]), "ranks disagree on " + key
    _check_against_reference(r0)


def test_rank_leaving_between_steps_ends_the_next_batch(tmp_path):
    _two_gpus()
    idf = str(tmp_path / "id")
    outs = [str(tmp_path / f"l{r}.json") for r in range(2)]
    _finish([_spawn("leave", r, 2, idf, outs[r]) for r in range(2)], timeout=180)
    with open(outs[0]) as f:
        res = json.load(f)
    assert res["step1"] == "ok"
    assert res["status"] == -5, res  # QUASAR_ENCCL
    assert res["elapsed"] < 60.0, res
    assert res["context_ok"], res
