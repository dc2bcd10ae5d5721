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
