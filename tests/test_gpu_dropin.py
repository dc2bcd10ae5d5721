"""The sample.h drop-in used the way separate sequences use it: one sampler
object per sequence, each driven from its own host thread at the same time.

In the reference every object owns its scratch (sample.c:94-104), so
objects are independent; here every object owns its device workspace and
stream, so two objects picking concurrently must each reproduce the id
sequence of their own reference object (oracle/_ref, sample.c compiled
unmodified, stepped through quasar_sampler_pick the same number of times)."""
import threading

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import V_FULL

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not O.available("ref"):
        pytest.skip("reference build (oracle/_ref) absent")


CASES = [  # (params, repeat_last_n, seed, logits seed)
    (dict(temperature=0.9, top_p=0.95, top_k=0, min_p=0.05, repeat_penalty=1.1), 64, 11, 101),
    (dict(temperature=0.7, top_p=0.8, top_k=20, min_p=0.0, repeat_penalty=1.3), 32, 12, 102),
    (dict(temperature=0.0, top_p=1.0, top_k=0, min_p=0.0, repeat_penalty=1.5), 16, 13, 103),
]


@pytest.mark.parametrize("device_logits", [False, True], ids=["host", "device"])
def test_objects_pick_concurrently_from_threads(device_logits):
    import torch
    import quasar_b200 as q
    n = 50
    steps = []
    for _, _, _, lseed in CASES:
        lg = O.synth_logits(O.SYNTH_NORMAL, lseed, 0, n, V_FULL, 3.0)
        lg[:, 5 * lseed] += 9.0  # a strong token that the repeat penalty then has to push down
        steps.append(lg)
    expect = [O.ref_sequence(steps[i], O.make_params(1, **kw), last_n, seed)
              for i, (kw, last_n, seed, _) in enumerate(CASES)]
    inputs = [torch.from_numpy(s).cuda() if device_logits else s for s in steps]
    torch.cuda.synchronize()
    got = [None] * len(CASES)
    errors = []
    start = threading.Barrier(len(CASES))

    def worker(i):
        try:
            kw, last_n, seed, _ = CASES[i]
            s = q.Sampler()
            s.config(kw["temperature"], kw["top_p"], kw["top_k"], kw["min_p"], kw["repeat_penalty"], last_n, seed)
            start.wait(timeout=60)
            got[i] = [s.pick(inputs[i][t]) for t in range(n)]
            s.close()
        except Exception as e:  # reported by the main thread
            errors.append(repr(e))

    th = [threading.Thread(target=worker, args=(i,)) for i in range(len(CASES))]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    assert not errors, errors
    for i in range(len(CASES)):
        assert got[i] == list(expect[i]), f"object {i}: {got[i]} vs {list(expect[i])}"
