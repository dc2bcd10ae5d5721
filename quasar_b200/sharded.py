"""Vocab-sharded sampling: rank g of a process group holds global columns
[col0, col0 + Vs) of every logits row (a tensor-parallel LM head), and the
batch is sampled with two all-gathers and no other exchange.

  1. every rank: per-row stats of its shard (max scaled logit and the window
     sum against it; the penalized argmax for greedy rows)      -> all-gather
  2. every rank: its k best candidates per row under the global max and sum
     (p desc, global id asc)                                     -> all-gather
  3. every rank: merge the G*k candidates, cut, draw with the row's PRNG and
     append to the row's history ring - the same ids on every rank.

The merge is exact because the global top-k lies in the union of the
shards' top-k, or, for min-p rows, because every shard sends all of its keys
at or above the min-p threshold of the global max; stochastic rows therefore
need 1 <= top_k <= k <= 256, or min_p > 0 with at most k such keys per shard.
``VocabShardedSampler`` does the orchestration through torch.distributed;
``NcclShardedSampler`` makes one C call per batch (quasar_shard_pick) that
runs the three phases (quasar_shard_{stats,candidates,finish}) and the two
all-gathers over a libquasar_cuda NCCL communicator (``NcclCommunicator``,
non-blocking, with a time limit and abort).
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import check, lib
from .sampler import PARAMS_DTYPE, SampleParams, make_params

STAT_BYTES = 16  # quasar_shard_stat: float max, int32 best, double sum


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _host_params(params):
    if isinstance(params, dict):
        params = make_params(1, **params)
    rec = np.asarray(params, dtype=PARAMS_DTYPE).reshape(-1)[0]
    return SampleParams(float(rec["temperature"]), float(rec["top_p"]), float(rec["min_p"]),
                        float(rec["repeat_penalty"]), int(rec["top_k"]), 0)


class CudaShardPhases:
    """The three phases on this rank's GPU (quasar_shard_* of libquasar_cuda)."""

    def __init__(self):
        self._lib = lib()

    def stats(self, logits, col0, hp, d_params, hist, hist_len, hist_head, stats, workspace, stream):
        B, Vs = logits.shape
        H = 0 if hist is None else int(hist.shape[1])
        check(self._lib.quasar_shard_stats(
            _ptr(logits), logits.stride(0), B, Vs, int(col0), _ptr(d_params),
            None if hp is None else ctypes.byref(hp), _ptr(hist), H, _ptr(hist_len), _ptr(hist_head),
            _ptr(stats), _ptr(workspace), workspace.numel(), 0, ctypes.c_void_p(stream.cuda_stream)),
            "quasar_shard_stats")

    def candidates(self, logits, col0, hp, d_params, hist, hist_len, hist_head, all_stats, G, rank, k, cand,
                   workspace, stream):
        B, Vs = logits.shape
        H = 0 if hist is None else int(hist.shape[1])
        check(self._lib.quasar_shard_candidates(
            _ptr(logits), logits.stride(0), B, Vs, int(col0), _ptr(d_params),
            None if hp is None else ctypes.byref(hp), _ptr(hist), H, _ptr(hist_len), _ptr(hist_head),
            _ptr(all_stats), G, rank, k, _ptr(cand), _ptr(workspace), workspace.numel(), 0,
            ctypes.c_void_p(stream.cuda_stream)), "quasar_shard_candidates")

    def finish(self, all_cand, all_stats, G, k, B, hp, d_params, rng, hist, hist_len, hist_head, record, out,
               diag, stream):
        H = 0 if hist is None else int(hist.shape[1])
        check(self._lib.quasar_shard_finish(
            _ptr(all_cand), _ptr(all_stats), G, k, B, _ptr(d_params),
            None if hp is None else ctypes.byref(hp), _ptr(rng), _ptr(hist), H, _ptr(hist_len),
            _ptr(hist_head), 1 if record else 0, _ptr(out), _ptr(diag), ctypes.c_void_p(stream.cuda_stream)),
            "quasar_shard_finish")


class VocabShardedSampler:
    """Samples row batches whose vocab is split over the ranks of ``group``.

    Every rank calls ``pick`` with its shard (``logits`` [B, Vs], global
    columns [col0, col0 + Vs)) and its replica of the per-row state (rng,
    history ring); all ranks get the same ids and the same state updates.
    Collectives go through torch.distributed (NCCL on GPUs; any backend whose
    all_gather_into_tensor handles the tensors ``phases`` produces).
    """

    def __init__(self, k: int, group=None, phases=None):
        if not 1 <= k <= 256:
            raise ValueError("k must be in [1, 256]")
        self.k = int(k)
        self.group = group
        self.phases = phases if phases is not None else CudaShardPhases()
        self._ws = {}

    def workspace(self, B: int, H: int, device):
        import torch
        key = (B, H, str(device))
        if key not in self._ws:
            n = int(lib().quasar_sampler_workspace_bytes(B, H))
            self._ws[key] = torch.empty(n + 256, dtype=torch.uint8, device=device)
        buf = self._ws[key]
        off = (-buf.data_ptr()) % 256  # 256-byte aligned view
        return buf[off:off + int(lib().quasar_sampler_workspace_bytes(B, H))]

    def pick(self, logits, col0: int, rng, *, params=None, d_params=None, hist=None, hist_len=None,
             hist_head=None, record: bool = False, out=None, diag=None, stream=None):
        import torch
        import torch.distributed as dist
        G = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        B = logits.shape[0]
        dev = logits.device
        hp = None if d_params is not None else _host_params(params)
        H = 0 if hist is None else int(hist.shape[1])
        if stream is None and dev.type == "cuda":
            stream = torch.cuda.current_stream(dev)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=dev)
        ws = self.workspace(B, H, dev)
        stats = torch.empty(B * STAT_BYTES, dtype=torch.uint8, device=dev)
        self.phases.stats(logits, col0, hp, d_params, hist, hist_len, hist_head, stats, ws, stream)
        all_stats = torch.empty(G * B * STAT_BYTES, dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(all_stats, stats, group=self.group)
        cand = torch.empty(B * self.k, dtype=torch.int64, device=dev)
        self.phases.candidates(logits, col0, hp, d_params, hist, hist_len, hist_head, all_stats, G, rank,
                               self.k, cand, ws, stream)
        all_cand = torch.empty(G * B * self.k, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(all_cand, cand, group=self.group)
        self.phases.finish(all_cand, all_stats, G, self.k, B, hp, d_params, rng, hist, hist_len, hist_head,
                           record, out, diag, stream)
        return out


class NcclCommunicator:
    """An NCCL communicator of libquasar_cuda (quasar_nccl_*): non-blocking,
    every NCCL call bounded by ``timeout_ms``; on an error or expiry it is
    aborted and the call raises QuasarError (QUASAR_ENCCL = -5).

    Rank 0 makes the id (``NcclCommunicator.unique_id()``) and hands it to the
    other ranks (any side channel: a store, a broadcast); every rank then
    constructs the communicator on its current CUDA device."""

    ID_BYTES = 128

    def __init__(self, nranks: int, rank: int, unique_id: bytes, timeout_ms: int = 60000):
        if len(unique_id) != self.ID_BYTES:
            raise ValueError("unique_id must be %d bytes" % self.ID_BYTES)
        self._lib = lib()
        self.nranks, self.rank = int(nranks), int(rank)
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(unique_id), self.ID_BYTES)
        check(self._lib.quasar_nccl_init(ctypes.byref(h), self.nranks, self.rank, buf, int(timeout_ms)),
              "quasar_nccl_init")
        self._h = h

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(NcclCommunicator.ID_BYTES)
        check(lib().quasar_nccl_unique_id(buf), "quasar_nccl_unique_id")
        return buf.raw

    @property
    def handle(self):
        return self._h

    def wait(self, stream=None, timeout_ms: int = 60000) -> None:
        """Block until the work queued on ``stream`` has completed, watching
        the communicator (QuasarError on an NCCL error or timeout)."""
        import torch
        stream = stream or torch.cuda.current_stream()
        check(self._lib.quasar_nccl_wait(self._h, ctypes.c_void_p(stream.cuda_stream), int(timeout_ms)),
              "quasar_nccl_wait")

    def abort(self) -> None:
        if self._h:
            self._lib.quasar_nccl_abort(self._h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            rc = self._lib.quasar_nccl_free(self._h)
            self._h = None
            check(rc, "quasar_nccl_free")

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class NcclShardedSampler:
    """Vocab-sharded sampling in one C call per batch (quasar_shard_pick):
    the three phases and their two NCCL all-gathers on the caller's stream,
    through a ``NcclCommunicator``. Same contract as ``VocabShardedSampler``."""

    def __init__(self, comm: NcclCommunicator, k: int):
        if not 1 <= k <= 256:
            raise ValueError("k must be in [1, 256]")
        self.comm, self.k = comm, int(k)
        self._lib = lib()
        self._ws = {}

    def workspace(self, B: int, H: int, device):
        import torch
        n = int(self._lib.quasar_shard_workspace_bytes(B, H, self.comm.nranks, self.k))
        key = (B, H, str(device))
        if key not in self._ws:
            self._ws[key] = torch.empty(n + 256, dtype=torch.uint8, device=device)
        buf = self._ws[key]
        off = (-buf.data_ptr()) % 256
        return buf[off:off + n]

    def pick(self, logits, col0: int, rng, *, params=None, d_params=None, hist=None, hist_len=None,
             hist_head=None, record: bool = False, out=None, diag=None, flags: int = 0, stream=None):
        import torch
        B, Vs = logits.shape
        dev = logits.device
        hp = None if d_params is not None else _host_params(params)
        H = 0 if hist is None else int(hist.shape[1])
        stream = stream or torch.cuda.current_stream(dev)
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=dev)
        ws = self.workspace(B, H, dev)
        check(self._lib.quasar_shard_pick(
            self.comm.handle, _ptr(logits), logits.stride(0), B, Vs, int(col0), _ptr(d_params),
            None if hp is None else ctypes.byref(hp), _ptr(rng), _ptr(hist), H, _ptr(hist_len), _ptr(hist_head),
            1 if record else 0, _ptr(out), _ptr(diag), self.k, _ptr(ws), ws.numel(), int(flags),
            ctypes.c_void_p(stream.cuda_stream)), "quasar_shard_pick")
        return out


__all__ = ["VocabShardedSampler", "CudaShardPhases", "STAT_BYTES", "NcclCommunicator", "NcclShardedSampler"]
