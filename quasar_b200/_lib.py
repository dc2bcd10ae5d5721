"""Loader of libquasar_cuda.so and its ctypes signatures.

The shared library is the product: every sampling call goes through it. There
is no Python or CPU fallback - if the library is missing or does not load, the
import fails with the reason.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libquasar_cuda.so")

QUASAR_OK = 0
STATUS = {0: "ok", -1: "invalid argument", -2: "unsupported shape", -3: "CUDA error",
          -4: "out of memory", -5: "NCCL error", -6: "buffer overflow"}

PATH_GREEDY, PATH_CANDIDATE, PATH_SELECT = 0, 1, 2
FLAG_EXACT_SELECT, FLAG_NO_TMA, FLAG_NO_SPLIT = 1, 2, 4
QUASAR_NOALLOC_WORKSPACE_BYTES = 32 << 20  # include/quasar_sampler.h
SYNTH_NORMAL, SYNTH_GUMBEL_PEAK, SYNTH_ZIPF = 0, 1, 2

# Every symbol include/quasar_sampler.h declares, with (argtypes, restype).
_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_U64 = ctypes.c_uint64
_F = ctypes.c_float
SIGNATURES = {
    "quasar_sampler_new": ([], _P),
    "quasar_sampler_free": ([_P], None),
    "quasar_sampler_config": ([_P, _F, _F, _I, _F, _F, _I, _U64], None),
    "quasar_sampler_reset": ([_P], None),
    "quasar_sampler_pick": ([_P, _P, _I], _I),
    "quasar_sampler_last_error": ([_P], _I),
    "quasar_status_string": ([_I], ctypes.c_char_p),
    "quasar_sampler_pick_batch": ([_P, _I64, _I, _I, _P, _P, _P, _P, _I, _P, _P, _I, _P, _P,
                                   _P, ctypes.c_size_t, _I, _P], _I),
    "quasar_sampler_pick_batch_launches": ([], _I),
    "quasar_sampler_split_shards": ([_P, _I64, _I, _I, _P, _P, _I, _I], _I),
    "quasar_sampler_pick_batch_noalloc": ([_P, _I64, _I, _I, _P, _P, _P, _P, _I, _P, _P, _I, _P, _P,
                                           _I, _P], _I),
    "quasar_sampler_workspace_bytes": ([_I, _I], ctypes.c_size_t),
    "quasar_shard_stats": ([_P, _I64, _I, _I, _I64, _P, _P, _P, _I, _P, _P, _P, _P, ctypes.c_size_t, _I, _P],
                           _I),
    "quasar_shard_candidates": ([_P, _I64, _I, _I, _I64, _P, _P, _P, _I, _P, _P, _P, _I, _I, _I, _P, _P,
                                 ctypes.c_size_t, _I, _P], _I),
    "quasar_shard_finish": ([_P, _P, _I, _I, _I, _P, _P, _P, _P, _I, _P, _P, _I, _P, _P, _P], _I),
    "quasar_nccl_available": ([], _I),
    "quasar_nccl_unique_id": ([_P], _I),
    "quasar_nccl_init": ([_P, _I, _I, _P, _I], _I),
    "quasar_nccl_wrap": ([_P, _P, _I, _I, _I], _I),
    "quasar_nccl_abort": ([_P], _I),
    "quasar_nccl_free": ([_P], _I),
    "quasar_nccl_wait": ([_P, _P, _I], _I),
    "quasar_shard_workspace_bytes": ([_I, _I, _I, _I], ctypes.c_size_t),
    "quasar_shard_pick": ([_P, _P, _I64, _I, _I, _I64, _P, _P, _P, _P, _I, _P, _P, _I, _P, _P, _I, _P,
                           ctypes.c_size_t, _I, _P], _I),
    "quasar_synth_logits": ([_I, _U64, _I64, _I, _I, _I64, _F, _P, _P], _I),
    "quasar_synth_hist": ([_U64, _I64, _I, _I, _I, _P, _P], _I),
    "quasar_synth_uniform": ([_U64, _I64, _I, _F, _F, _P, _P], _I),
    "quasar_selftest_exp": ([_P, _P, _I, _I, _P], _I),
}

_lib: ctypes.CDLL | None = None


class QuasarError(RuntimeError):
    def __init__(self, what: str, status: int):
        super().__init__(f"{what}: {STATUS.get(status, 'status %d' % status)} ({status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """The loaded library (loads it on first use; raises if it is missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; "
                f"g.build()'` (nvcc, sm_100a). There is no CPU fallback.")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes, fn.restype = args, res
        _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != QUASAR_OK:
        raise QuasarError(what, status)
