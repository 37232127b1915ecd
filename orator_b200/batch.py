"""Continuous-batching host API over the C ABI (orx_batch_*).

``BatchDecoder`` serves many independent sessions from one paged KV pool and
the weights of an ``AsrTextDecoder``; each ``step`` decodes one greedy token
for every listed session in a single batched pass (ragged KV lengths).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import call, lib
from .decoder import AsrTextDecoder, _stream


class BatchDecoder:
    def __init__(self, weights: AsrTextDecoder, max_sessions: int = 64, max_batch: int = 64,
                 pool_pages: int = 64 * 160, max_pages_per_session: int = 160):
        self.weights = weights  # keeps the model alive
        h = C.c_void_p()
        call("orx_batch_create", weights._h, max_sessions, max_batch, pool_pages,
             max_pages_per_session, C.byref(h))
        self._h = h

    def close(self):
        if getattr(self, "_h", None):
            lib().orx_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def create_session(self) -> int:
        v = C.c_int()
        call("orx_batch_session_create", self._h, C.byref(v))
        return v.value

    def free_session(self, sid: int):
        call("orx_batch_session_free", self._h, sid)

    def cache_len(self, sid: int) -> int:
        v = C.c_int()
        call("orx_batch_cache_len", self._h, sid, C.byref(v))
        return v.value

    def truncate(self, sid: int, n: int):
        call("orx_batch_truncate", self._h, sid, n)

    def free_pages(self) -> int:
        v = C.c_int()
        call("orx_batch_free_pages", self._h, C.byref(v))
        return v.value

    def prefill(self, sids, embeds_list, stream=None, lens=None):
        """Appends rows to each session: `embeds_list` is one [T_i, 2048] array
        per session, or (with `lens`) the rows of all sessions already
        concatenated (e.g. in pinned memory, copied as is)."""
        sids = np.ascontiguousarray(sids, np.int32)
        if lens is None:
            lens = np.array([len(e) for e in embeds_list], np.int32)
            x = np.ascontiguousarray(np.concatenate(embeds_list, 0), np.float32)
        else:
            lens = np.ascontiguousarray(lens, np.int32)
            x = embeds_list
            if x.dtype != np.float32 or not x.flags["C_CONTIGUOUS"] or len(x) != int(lens.sum()):
                raise ValueError("concatenated rows must be contiguous fp32 [sum(lens), 2048]")
        call("orx_batch_prefill", self._h, sids.ctypes.data_as(C.c_void_p),
             lens.ctypes.data_as(C.c_void_p), len(sids), x.ctypes.data_as(C.c_void_p),
             _stream(stream))

    def step(self, sids, stream=None) -> np.ndarray:
        sids = np.ascontiguousarray(sids, np.int32)
        out = np.zeros(max(len(sids), 1), np.int32)
        call("orx_batch_step", self._h, sids.ctypes.data_as(C.c_void_p), len(sids),
             out.ctypes.data_as(C.c_void_p), _stream(stream))
        return out[:len(sids)]

    def set_ban(self, sid: int, ban0: int, ban1: int, steps: int, stream=None):
        """The session's next `steps` argmaxes exclude ban0 / ban1 (DecodeGreedy's ban window)."""
        call("orx_batch_set_ban", self._h, sid, ban0, ban1, steps, _stream(stream))

    def next_tokens(self, sids, stream=None) -> np.ndarray:
        """Pending greedy token of each session (fed by its next step)."""
        sids = np.ascontiguousarray(sids, np.int32)
        out = np.zeros(max(len(sids), 1), np.int32)
        call("orx_batch_next_tokens", self._h, sids.ctypes.data_as(C.c_void_p), len(sids),
             out.ctypes.data_as(C.c_void_p), _stream(stream))
        return out[:len(sids)]

    def device_error(self) -> int:
        v = C.c_int()
        call("orx_batch_device_error", self._h, C.byref(v))
        return v.value
