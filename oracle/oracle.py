"""ctypes wrapper of the CPU checker libraries (TEST INFRASTRUCTURE ONLY).

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm import this module, as the checker or the timed CPU baseline;
the shipped sampler (``quasar_b200``) never does.

Two backends share one interface:
  * ``"ref"``    - oracle/_ref/libsample_ref.so: the reference sample.c compiled
                   unmodified (franzvill/quasar sample.c:111-178), one sampler
                   object per row;
  * ``"oracle"`` - oracle/_lib/liboracle.so: the plain-C restatement
                   (sample_oracle.c), used where the reference tree is absent.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "libsample_ref.so")
ORACLE_SO = os.path.join(HERE, "_lib", "liboracle.so")

SYNTH_NORMAL, SYNTH_GUMBEL_PEAK, SYNTH_ZIPF = 0, 1, 2

PARAMS_DTYPE = np.dtype([("temperature", "<f4"), ("top_p", "<f4"), ("min_p", "<f4"),
                         ("repeat_penalty", "<f4"), ("top_k", "<i4"), ("reserved", "<i4")])
RESULT_DTYPE = np.dtype([("id", "<i4"), ("n_window", "<i4"), ("n_kept", "<i4"),
                         ("greedy", "<i4"), ("p_chosen", "<f4"), ("inv_sum", "<f4"),
                         ("margin", "<f8"), ("rng_out", "<u8")])
assert PARAMS_DTYPE.itemsize == 24 and RESULT_DTYPE.itemsize == 40

_libs: dict[str, ctypes.CDLL] = {}


def reference_tree() -> str | None:
    """The franzvill/quasar checkout to build the reference from: the one
    QUASAR_REFERENCE names, else a checkout named ``reference`` beside this
    repository; None when neither holds sample.c."""
    for d in (os.environ.get("QUASAR_REFERENCE"), os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")):
        if d and os.path.isfile(os.path.join(d, "sample.c")):
            return d
    return None


def build() -> None:
    """Compile oracle/ (restatement always; reference build when its tree exists)."""
    ref = reference_tree()
    subprocess.run(["make", "-s", "-C", HERE] + ([f"REF={ref}"] if ref else []), check=True)


def available(backend: str) -> bool:
    return os.path.exists(REF_SO if backend == "ref" else ORACLE_SO)


def best_backend() -> str:
    return "ref" if available("ref") else "oracle"


def _lib(backend: str) -> ctypes.CDLL:
    if backend not in _libs:
        path = REF_SO if backend == "ref" else ORACLE_SO
        if not os.path.exists(path):
            build()
        lib = ctypes.CDLL(path)
        P = ctypes.c_void_p
        pick_args = [P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, P, ctypes.c_int,
                     P, ctypes.c_int, P, P, P, P, ctypes.c_int]
        fn = lib.qs_ref_pick_rows if backend == "ref" else lib.qs_oracle_pick_rows
        fn.argtypes, fn.restype = pick_args, ctypes.c_int
        lib.qs_synth_logits.argtypes = [ctypes.c_int, ctypes.c_uint64, ctypes.c_int64, ctypes.c_int,
                                        ctypes.c_int, ctypes.c_int64, ctypes.c_float, P]
        lib.qs_synth_hist.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, P]
        lib.qs_synth_uniform.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_int,
                                         ctypes.c_float, ctypes.c_float, P]
        lib.qs_det_log.argtypes, lib.qs_det_log.restype = [ctypes.c_double], ctypes.c_double
        if backend == "ref":
            lib.qs_ref_sequence.argtypes = [P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, P,
                                            ctypes.c_int, ctypes.c_uint64, P]
            lib.qs_ref_sequence.restype = ctypes.c_int
            lib.qs_ref_sequence_diag.argtypes = [P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, P,
                                                 ctypes.c_int, ctypes.c_uint64, P]
            lib.qs_ref_sequence_diag.restype = ctypes.c_int
            lib.qs_ref_decode.argtypes = [P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, P, ctypes.c_int,
                                          P, ctypes.c_int, P, P, P, ctypes.c_int, P, P, P, P, ctypes.c_int]
            lib.qs_ref_decode.restype = ctypes.c_int
        _libs[backend] = lib
    return _libs[backend]


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def make_params(B=1, temperature=0.0, top_p=1.0, top_k=0, min_p=0.0, repeat_penalty=1.0):
    """Array of B parameter records; any argument may be a scalar or a length-B array."""
    p = np.zeros(B, dtype=PARAMS_DTYPE)
    p["temperature"], p["top_p"], p["top_k"] = temperature, top_p, top_k
    p["min_p"], p["repeat_penalty"] = min_p, repeat_penalty
    return p


def pick_rows(logits: np.ndarray, params: np.ndarray, rng: np.ndarray,
              hist: np.ndarray | None = None, hist_len: np.ndarray | None = None,
              hist_head: np.ndarray | None = None, backend: str | None = None,
              nthreads: int | None = None):
    """Sample every row of logits[B, V] on the CPU. Returns (results, rng_after)."""
    backend = backend or best_backend()
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    if logits.ndim == 1:
        logits = logits[None, :]
    B, V = logits.shape
    params = np.ascontiguousarray(params, dtype=PARAMS_DTYPE)
    per_row = 1 if params.shape[0] == B and B > 1 else 0
    rng = np.array(rng, dtype=np.uint64).reshape(B).copy()
    cap = 0
    if hist is not None:
        hist = np.ascontiguousarray(hist, dtype=np.int32).reshape(B, -1)
        cap = hist.shape[1]
        if hist_len is not None:
            hist_len = np.ascontiguousarray(hist_len, dtype=np.int32).reshape(B)
        if hist_head is not None:
            hist_head = np.ascontiguousarray(hist_head, dtype=np.int32).reshape(B)
    res = np.zeros(B, dtype=RESULT_DTYPE)
    lib = _lib(backend)
    fn = lib.qs_ref_pick_rows if backend == "ref" else lib.qs_oracle_pick_rows
    rc = fn(_ptr(logits), V, B, V, _ptr(params), per_row, _ptr(hist), cap,
            _ptr(hist_len), _ptr(hist_head), _ptr(rng), _ptr(res),
            nthreads or os.cpu_count() or 1)
    if rc != 0:
        raise RuntimeError(f"{backend} pick_rows failed: {rc}")
    return res, rng


def ref_sequence(logits: np.ndarray, params: np.ndarray, repeat_last_n: int, seed: int):
    """Ids of len(logits) successive picks through one reference sampler object."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    n, V = logits.shape
    out = np.zeros(n, dtype=np.int32)
    params = np.ascontiguousarray(params, dtype=PARAMS_DTYPE)
    rc = _lib("ref").qs_ref_sequence(_ptr(logits), V, n, V, _ptr(params), repeat_last_n,
                                     seed, _ptr(out))
    if rc != 0:
        raise RuntimeError(f"ref_sequence failed: {rc}")
    return out


def ref_sequence_diag(logits: np.ndarray, params: np.ndarray, repeat_last_n: int, seed: int):
    """ref_sequence with each pick's full result (RESULT_DTYPE: id, kept count, p, margin)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    n, V = logits.shape
    res = np.zeros(n, dtype=RESULT_DTYPE)
    params = np.ascontiguousarray(params, dtype=PARAMS_DTYPE)
    rc = _lib("ref").qs_ref_sequence_diag(_ptr(logits), V, n, V, _ptr(params), repeat_last_n, seed, _ptr(res))
    if rc != 0:
        raise RuntimeError(f"ref_sequence_diag failed: {rc}")
    return res


def ref_decode(logits: np.ndarray, params: np.ndarray, rng: np.ndarray, n_steps: int,
               hist: np.ndarray, hist_len: np.ndarray, hist_head: np.ndarray,
               nthreads: int | None = None):
    """A decode loop through the reference: row r gets one sampler object with
    its own ring and seed, picked n_steps times on the same logits row with each
    choice recorded. Returns (results [n_steps, B], rng_after, hist, len, head)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    B, V = logits.shape
    params = np.ascontiguousarray(params, dtype=PARAMS_DTYPE)
    per_row = 1 if params.shape[0] == B and B > 1 else 0
    rng = np.array(rng, dtype=np.uint64).reshape(B).copy()
    hist = np.ascontiguousarray(hist, dtype=np.int32).reshape(B, -1)
    cap = hist.shape[1]
    hist_len = np.ascontiguousarray(hist_len, dtype=np.int32).reshape(B)
    hist_head = np.ascontiguousarray(hist_head, dtype=np.int32).reshape(B)
    res = np.zeros((n_steps, B), dtype=RESULT_DTYPE)
    h_out = np.zeros_like(hist)
    l_out = np.zeros(B, dtype=np.int32)
    d_out = np.zeros(B, dtype=np.int32)
    rc = _lib("ref").qs_ref_decode(_ptr(logits), V, B, V, _ptr(params), per_row, _ptr(hist), cap,
                                   _ptr(hist_len), _ptr(hist_head), _ptr(rng), int(n_steps), _ptr(res),
                                   _ptr(h_out), _ptr(l_out), _ptr(d_out), nthreads or os.cpu_count() or 1)
    if rc != 0:
        raise RuntimeError(f"ref_decode failed: {rc}")
    return res, rng, h_out, l_out, d_out


def synth_logits(kind: int, seed: int, row0: int, B: int, V: int, scale: float = 1.0,
                 backend: str | None = None) -> np.ndarray:
    out = np.empty((B, V), dtype=np.float32)
    _lib(backend or best_backend()).qs_synth_logits(kind, seed, row0, B, V, V, scale, _ptr(out))
    return out


def synth_hist(seed: int, row0: int, B: int, H: int, V: int, backend: str | None = None):
    out = np.empty((B, H), dtype=np.int32)
    _lib(backend or best_backend()).qs_synth_hist(seed, row0, B, H, V, _ptr(out))
    return out


def synth_uniform(seed: int, row0: int, B: int, lo: float, hi: float, backend: str | None = None):
    out = np.empty(B, dtype=np.float32)
    _lib(backend or best_backend()).qs_synth_uniform(seed, row0, B, lo, hi, _ptr(out))
    return out


def det_log(x: float, backend: str | None = None) -> float:
    return _lib(backend or best_backend()).qs_det_log(x)
