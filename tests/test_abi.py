"""CPU checks of the C ABI: the library loads, exports every function the
public headers declare, and rejects bad arguments before touching a GPU."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")


def declared_functions():
    names = []
    for f in sorted(os.listdir(INCLUDE)):
        if not f.endswith(".h"):
            continue
        text = open(os.path.join(INCLUDE, f)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"^\s*#.*$", "", text, flags=re.M)
        for m in re.finditer(r"\b(quasar_\w+)\s*\([^;{]*\)\s*;", text):
            names.append(m.group(1))
    return sorted(set(names))


def test_headers_declare_functions():
    names = declared_functions()
    for n in ("quasar_sampler_new", "quasar_sampler_free", "quasar_sampler_config",
              "quasar_sampler_reset", "quasar_sampler_pick", "quasar_sampler_pick_batch"):
        assert n in names


def test_library_exports_every_declared_symbol():
    import quasar_b200 as q
    out = subprocess.run(["nm", "-D", "--defined-only", q.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing


def test_python_signatures_cover_header():
    from quasar_b200._lib import SIGNATURES
    assert set(declared_functions()) <= set(SIGNATURES)


def test_status_strings():
    import quasar_b200 as q
    lib = q.lib()
    assert lib.quasar_status_string(0) == b"ok"
    assert lib.quasar_status_string(-1) == b"invalid argument"
    assert lib.quasar_status_string(-99) == b"unknown status"


@pytest.mark.parametrize("B,V,ld", [(1, 0, 0), (1, 10, 5), (-1, 10, 10), (1, (1 << 20) + 1, (1 << 20) + 1)])
def test_batch_rejects_bad_shapes(B, V, ld):
    import quasar_b200 as q
    lib = q.lib()
    rc = lib.quasar_sampler_pick_batch(ctypes.c_void_p(16), ld, B, V, None, None,
                                       ctypes.c_void_p(16), None, 0, None, None, 0,
                                       ctypes.c_void_p(16), None, None, 0, 0, None)
    assert rc == -1


def test_batch_rejects_missing_pointers():
    import quasar_b200 as q
    lib = q.lib()
    P = ctypes.c_void_p
    # no params at all
    assert lib.quasar_sampler_pick_batch(P(16), 10, 1, 10, None, None, P(16), None, 0, None, None,
                                         0, P(16), None, None, 0, 0, None) == -1
    prm = q.SampleParams(1.0, 1.0, 0.0, 1.0, 0, 0)
    # history capacity without a ring
    assert lib.quasar_sampler_pick_batch(P(16), 10, 1, 10, None, ctypes.byref(prm), P(16), None, 4,
                                         None, None, 0, P(16), None, None, 0, 0, None) == -1
    # record without len/head
    assert lib.quasar_sampler_pick_batch(P(16), 10, 1, 10, None, ctypes.byref(prm), P(16), P(16), 4,
                                         None, None, 1, P(16), None, None, 0, 0, None) == -1
    # B == 0 is a no-op
    assert lib.quasar_sampler_pick_batch(None, 10, 0, 10, None, None, None, None, 0, None, None, 0,
                                         None, None, None, 0, 0, None) == 0
    # an explicit workspace must be large enough and 256-byte aligned
    assert lib.quasar_sampler_pick_batch(P(16), 10, 1, 10, None, ctypes.byref(prm), P(16), None, 0,
                                         None, None, 0, P(16), None, P(256), 8, 0, None) == -1
    assert lib.quasar_sampler_workspace_bytes(4096, 256) >= 4096 * (256 * 8 + 12)
    assert lib.quasar_sampler_workspace_bytes(0, 256) == 0


def test_pick_guards_without_gpu():
    import quasar_b200 as q
    lib = q.lib()
    h = lib.quasar_sampler_new()
    assert h
    assert lib.quasar_sampler_pick(h, None, 0) == 0       # n_vocab <= 0 -> 0 (sample.c:112)
    assert lib.quasar_sampler_pick(h, None, -5) == 0
    assert lib.quasar_sampler_pick(h, None, 10) == -1     # NULL logits
    assert lib.quasar_sampler_last_error(h) == -1
    lib.quasar_sampler_free(h)
    lib.quasar_sampler_free(None)                         # NULL-safe (sample.c:42)


def test_params_layout_matches_oracle():
    import quasar_b200 as q
    from oracle import oracle as O
    assert ctypes.sizeof(q.SampleParams) == 24
    assert q.PARAMS_DTYPE == O.PARAMS_DTYPE


def test_small_batch_decision_without_gpu():
    """Which batches pick_batch samples with the fused cluster kernel (host
    arithmetic: at most 16 rows with host parameters, greedy or
    1 <= top_k <= 256, rows the bulk-copy ring can stream, V % 32 == 0 and
    V >= 8192), and that the workspace query is the one-CTA path's."""
    import quasar_b200 as q
    V = 151936
    cfg1 = dict(temperature=0.7, top_k=20, top_p=0.8, repeat_penalty=1.1)
    assert [q.split_shards(B, V, params=cfg1, hist_cap=64) for B in (1, 2, 8, 16, 17)] == [8, 8, 8, 8, 0]
    assert q.split_shards(1, V, params=dict(temperature=0.0)) == 8              # greedy
    assert q.split_shards(1, V, params=dict(temperature=1.0, top_k=256)) == 8
    assert q.split_shards(1, V, params=dict(temperature=1.0, top_k=257)) == 0   # beyond a shard's keys
    assert q.split_shards(1, V, params=dict(temperature=0.9, min_p=0.05)) == 0  # no per-shard bound
    assert q.split_shards(1, V, params=dict(temperature=0.9, top_p=0.9)) == 0
    assert q.split_shards(1, V, per_row_params=True) == 0                       # parameters on the device
    assert q.split_shards(1, V, params=cfg1, flags=q.FLAG_NO_SPLIT) == 0
    assert q.split_shards(1, V, params=cfg1, flags=q.FLAG_EXACT_SELECT) == 0
    assert q.split_shards(1, V, params=cfg1, flags=q.FLAG_NO_TMA) == 0
    assert q.split_shards(1, V, params=cfg1, ptr=260) == 0                      # not 16-byte aligned
    assert q.split_shards(1, V, params=cfg1, ld=V + 2) == 0                     # ld % 4 != 0
    assert q.split_shards(1, V, params=cfg1, ld=V + 4) == 8
    assert q.split_shards(1, 20000, params=cfg1) == 8                           # 8 x 2500
    assert q.split_shards(1, 20004, params=cfg1) == 0                           # 20004 / 8 not whole
    assert q.split_shards(1, 4000, params=cfg1) == 0                            # shards under 1024 columns
    assert q.split_shards(16, V, params=cfg1, hist_cap=100000) == 8             # no workspace involved
    for B, H in ((1, 0), (1, 64), (4, 256), (17, 64), (16, 100000)):
        assert q.workspace_bytes(B, H) == 256 + B * (16 + 4 * 256 + 8 * H + 40 * 256 + 8 * 256)
