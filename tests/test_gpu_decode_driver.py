"""The C batched decode driver (quasar_b200/batched_decode.c): B sequences
sampled together, one quasar_sampler_pick_batch call per step with the state
on the device, against one reference sampler object per sequence
(oracle/_ref: sample.c compiled unmodified, configured like server.c
configures a request, stepped through the same logits rows).

Every sequence must match its reference object step by step until the first
step the reference itself puts within 1e-6 of a CDF or tie boundary (after
which the two may legitimately diverge); greedy sequences match entirely.
A second run with a stop token ends each sequence at that token's first
occurrence and leaves everything before it unchanged."""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_BOUNDARY, TOL_P_REL, V_FULL

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DRIVER = os.path.join(ROOT, "quasar_b200", "batched_decode")
B, N, H, SEED = 30, 20, 16, 11


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not O.available("ref"):
        pytest.skip("reference build (oracle/_ref) absent")
    assert os.path.exists(DRIVER), "batched_decode is not built (quasar_b200/build.py builds it)"


def _params(r):
    """batched_decode.c row_params, restated."""
    t = 0.0 if r % 5 == 0 else np.float32(0.6) + np.float32(0.1) * np.float32(r % 7)
    return O.make_params(1, temperature=t, top_p=0.9, min_p=0.05 if r % 2 else 0.0, repeat_penalty=1.1,
                         top_k=40 if r % 3 == 1 else 0)


def _run(tmp_path, name, stop=None):
    out = str(tmp_path / name)
    cmd = [DRIVER, "--rows", str(B), "--steps", str(N), "--hist", str(H), "--seed", str(SEED), "--out", out]
    if stop is not None:
        cmd += ["--stop", str(stop)]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout + p.stderr
    raw = np.fromfile(out, dtype=np.int32)
    return raw[:B], raw[B:].reshape(B, N)


def test_driver_matches_reference_objects(tmp_path):
    lens, ids = _run(tmp_path, "free.bin")
    assert (lens == N).all()
    # step t's logits for every row, as the driver generates them
    steps = np.stack([O.synth_logits(O.SYNTH_NORMAL, SEED + t, 0, B, V_FULL, 3.0) for t in range(N)], axis=1)
    diverged = 0
    for r in range(B):
        prm = _params(r)
        ref = O.ref_sequence_diag(steps[r], prm, H, 1000 + r)
        for t in range(N):
            if ids[r, t] != ref["id"][t]:
                assert prm["temperature"][0] > 0 and ref["margin"][t] < TOL_BOUNDARY, \
                    f"row {r} step {t}: driver {ids[r, t]} reference {ref['id'][t]} margin {ref['margin'][t]}"
                diverged += 1
                break
    assert diverged <= 1, f"{diverged} sequences hit a boundary case"
    del steps


def test_driver_stop_token_ends_sequences(tmp_path):
    _, free = _run(tmp_path, "free.bin")
    stop = int(free[0, 6])  # row 0 is greedy: a token it certainly emits
    lens, ids = _run(tmp_path, "stop.bin", stop=stop)
    for r in range(B):
        hit = np.nonzero(free[r] == stop)[0]
        n = int(hit[0]) + 1 if hit.size else N
        assert lens[r] == n, (r, lens[r], n)
        assert np.array_equal(ids[r, :n], free[r, :n])
        assert (ids[r, n:] == -1).all()
