"""Host-side mirror of the reference sampler API on top of libquasar_cuda.

``Sampler`` mirrors franzvill/quasar sample.h:12-29 one to one (new / config /
reset / pick / free, same argument meaning, clamps and seeding), and
``pick_batch`` exposes the batched C entry (``quasar_sampler_pick_batch``) for
device-resident logits held in torch tensors. torch is used only for device
memory and streams; all sampling runs in the CUDA library.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import FLAG_EXACT_SELECT, QuasarError, check, lib

PARAMS_DTYPE = np.dtype([("temperature", "<f4"), ("top_p", "<f4"), ("min_p", "<f4"),
                         ("repeat_penalty", "<f4"), ("top_k", "<i4"), ("reserved", "<i4")])
DIAG_DTYPE = np.dtype([("n_kept", "<i4"), ("p_chosen", "<f4"), ("inv_sum", "<f4"),
                       ("path", "<i4")])


class SampleParams(ctypes.Structure):
    """ctypes twin of quasar_sample_params."""
    _fields_ = [("temperature", ctypes.c_float), ("top_p", ctypes.c_float),
                ("min_p", ctypes.c_float), ("repeat_penalty", ctypes.c_float),
                ("top_k", ctypes.c_int32), ("reserved", ctypes.c_int32)]


def make_params(B: int = 1, temperature=0.0, top_p=1.0, top_k=0, min_p=0.0,
                repeat_penalty=1.0) -> np.ndarray:
    """Structured array of B raw parameter records (scalars or length-B arrays)."""
    p = np.zeros(B, dtype=PARAMS_DTYPE)
    p["temperature"], p["top_p"], p["top_k"] = temperature, top_p, top_k
    p["min_p"], p["repeat_penalty"] = min_p, repeat_penalty
    return p


class Sampler:
    """The reference's stateful per-sequence sampler (sample.c:17-29), GPU-backed.

    ``pick`` accepts a host array (numpy / CPU tensor, copied to the device) or a
    CUDA tensor (read in place) and returns the token id, recording it in the
    history ring exactly like sample.c:83-92.
    """

    def __init__(self):
        self._lib = lib()
        self._h = self._lib.quasar_sampler_new()
        if not self._h:
            raise MemoryError("quasar_sampler_new failed")

    def config(self, temperature: float, top_p: float, top_k: int, min_p: float,
               repeat_penalty: float, repeat_last_n: int, seed: int) -> None:
        self._lib.quasar_sampler_config(self._h, temperature, top_p, int(top_k), min_p,
                                        repeat_penalty, int(repeat_last_n), int(seed) & (2**64 - 1))
        check(self._lib.quasar_sampler_last_error(self._h), "quasar_sampler_config")

    def reset(self) -> None:
        self._lib.quasar_sampler_reset(self._h)
        check(self._lib.quasar_sampler_last_error(self._h), "quasar_sampler_reset")

    def pick(self, logits) -> int:
        keep = logits
        if hasattr(logits, "data_ptr"):  # torch tensor
            if not logits.is_contiguous() or logits.dtype.itemsize != 4:
                raise ValueError("logits must be a contiguous float32 tensor")
            ptr, n = logits.data_ptr(), logits.numel()
        else:
            keep = np.ascontiguousarray(logits, dtype=np.float32)
            ptr, n = keep.ctypes.data, keep.size
        tok = self._lib.quasar_sampler_pick(self._h, ctypes.c_void_p(ptr), int(n))
        del keep
        if tok < 0:
            raise QuasarError("quasar_sampler_pick", self._lib.quasar_sampler_last_error(self._h))
        return tok

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.quasar_sampler_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _ptr(t) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def params_to_device(params: np.ndarray, device):
    """Upload a PARAMS_DTYPE array as raw bytes (a uint8 CUDA tensor)."""
    import torch
    raw = np.ascontiguousarray(params, dtype=PARAMS_DTYPE).view(np.uint8)
    return torch.from_numpy(raw.copy()).to(device)


def pick_batch(logits, rng, *, params=None, d_params=None, hist=None, hist_len=None,
               hist_head=None, record: bool = False, out=None, diag=None,
               workspace=None, flags: int = 0, stream=None):
    """Sample every row of ``logits`` ([B, V] float32 CUDA tensor, unit column stride).

    rng: [B] int64 CUDA tensor holding xorshift64* states (advanced in place).
    params: one PARAMS_DTYPE record (or a dict) shared by all rows; d_params: a
    uint8 CUDA tensor from ``params_to_device`` with one record per row.
    hist / hist_len / hist_head: int32 CUDA tensors [B, H] / [B] / [B].
    out: optional int32 [B] CUDA tensor; diag: optional int32 [B, 4] CUDA tensor
    (DIAG_DTYPE records). workspace: optional uint8 CUDA tensor of at least
    ``workspace_bytes(B, H)`` bytes (default: the library's per-device one).
    Returns ``out``. Launches on ``stream`` (a torch.cuda.Stream; default: the
    current stream).
    """
    import torch
    if logits.dim() != 2 or logits.dtype != torch.float32 or logits.stride(1) != 1:
        raise ValueError("logits must be a [B, V] float32 tensor with unit column stride")
    B, V = logits.shape
    if out is None:
        out = torch.empty(B, dtype=torch.int32, device=logits.device)
    hp = None
    if d_params is None:
        if params is None:
            raise ValueError("pass params or d_params")
        if isinstance(params, dict):
            params = make_params(1, **params)
        rec = np.asarray(params, dtype=PARAMS_DTYPE).reshape(-1)[0]
        hp = SampleParams(float(rec["temperature"]), float(rec["top_p"]), float(rec["min_p"]),
                          float(rec["repeat_penalty"]), int(rec["top_k"]), 0)
    H = 0 if hist is None else int(hist.shape[1])
    if stream is None:
        stream = torch.cuda.current_stream(logits.device)
    rc = lib().quasar_sampler_pick_batch(
        _ptr(logits), logits.stride(0), B, V, _ptr(d_params),
        None if hp is None else ctypes.byref(hp), _ptr(rng), _ptr(hist), H,
        _ptr(hist_len), _ptr(hist_head), 1 if record else 0, _ptr(out), _ptr(diag),
        _ptr(workspace), 0 if workspace is None else workspace.numel() * workspace.element_size(),
        int(flags), ctypes.c_void_p(stream.cuda_stream))
    check(rc, "quasar_sampler_pick_batch")
    return out


def split_shards(B: int, V: int, *, params=None, per_row_params: bool = False, hist_cap: int = 0, flags: int = 0,
                 ld: int = None, ptr: int = 256) -> int:
    """CTAs per row (cluster size) of the fused small-batch kernel pick_batch uses for
    a batch of B rows (0: the streaming and finishing kernels, one CTA per row).

    params: the record shared by all rows (as pick_batch's ``params``);
    per_row_params: the rows have device parameters instead (never split).
    ptr / ld: the logits address and row stride the call would get (the
    bulk-copy alignment conditions). Host arithmetic only, no GPU call."""
    hp = None
    if not per_row_params:
        if isinstance(params, dict):
            params = make_params(1, **params)
        rec = np.asarray(params, dtype=PARAMS_DTYPE).reshape(-1)[0]
        hp = SampleParams(float(rec["temperature"]), float(rec["top_p"]), float(rec["min_p"]),
                          float(rec["repeat_penalty"]), int(rec["top_k"]), 0)
    return int(lib().quasar_sampler_split_shards(
        ctypes.c_void_p(ptr), int(V if ld is None else ld), int(B), int(V),
        ctypes.c_void_p(16) if per_row_params else None, None if hp is None else ctypes.byref(hp),
        int(hist_cap), int(flags)))


def workspace_bytes(B: int, hist_cap: int = 0) -> int:
    """Bytes of device workspace one pick_batch call over B rows with history capacity hist_cap needs."""
    return int(lib().quasar_sampler_workspace_bytes(int(B), int(hist_cap)))


def synth_logits(kind: int, seed: int, row0: int, B: int, V: int, scale: float, out, stream=None):
    """Fill out[B, V] (float32 CUDA tensor) with the deterministic synthetic recipe."""
    import torch
    stream = stream or torch.cuda.current_stream(out.device)
    check(lib().quasar_synth_logits(kind, seed, row0, B, V, out.stride(0), scale, _ptr(out),
                                    ctypes.c_void_p(stream.cuda_stream)), "quasar_synth_logits")
    return out


def synth_hist(seed: int, row0: int, B: int, H: int, V: int, out, stream=None):
    import torch
    stream = stream or torch.cuda.current_stream(out.device)
    check(lib().quasar_synth_hist(seed, row0, B, H, V, _ptr(out),
                                  ctypes.c_void_p(stream.cuda_stream)), "quasar_synth_hist")
    return out


def synth_uniform(seed: int, row0: int, B: int, lo: float, hi: float, out, stream=None):
    import torch
    stream = stream or torch.cuda.current_stream(out.device)
    check(lib().quasar_synth_uniform(seed, row0, B, lo, hi, _ptr(out),
                                     ctypes.c_void_p(stream.cuda_stream)), "quasar_synth_uniform")
    return out


__all__ = ["Sampler", "SampleParams", "make_params", "params_to_device", "pick_batch", "workspace_bytes",
           "split_shards", "synth_logits", "synth_hist", "synth_uniform", "PARAMS_DTYPE", "DIAG_DTYPE",
           "FLAG_EXACT_SELECT"]
