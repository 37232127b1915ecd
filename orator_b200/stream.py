"""Multi-session streaming front door over the batched decoder (token level).

Restates the decoder side of the reference's streaming protocol,
``Qwen3Asr::StreamReset / StreamChunk / StreamDecodeStep``
(src/model/qwen3_asr.cc:269-304, 307-407, 503-557), for many sessions that
share one ``BatchDecoder``:

* ``open``: prefill the fixed prefix ``<|im_start|>system\\n{system}<|im_end|>\\n
  <|im_start|>user\\n<|audio_start|>`` at position 0; the checkpoint is its
  length.
* ``append_audio``: the encoder rows of new audio windows are prefilled after
  the checkpoint, which advances past them (the persistent [system][audio]
  cache).
* ``decode``: for every requested session, prefill the suffix
  ``<|audio_end|><|im_end|>\\n<|im_start|>assistant\\n{language}<asr_text>
  {committed}`` after the checkpoint, greedy-decode with the rules of
  ``AsrTextDecoder::DecodeGreedy`` (EOS ids banned for the first
  ``ban_steps`` argmaxes; stop at ``<|im_end|>`` / ``<|endoftext|>`` or six
  equal tokens; at most ``max_new``), then truncate back to the checkpoint.
  The sessions' decode steps run together, one batched step per token.

Text handling (tokenizer, the utf-8-safe rollback of committed text) stays
with the caller: ``language`` and ``committed`` arrive as token ids.
"""
from __future__ import annotations

import numpy as np

# Special token ids of Qwen3-ASR (include/model/qwen3_asr.h:193-203).
IM_START, IM_END, END_OF_TEXT = 151644, 151645, 151643
AUDIO_START, AUDIO_END, ASR_TEXT = 151669, 151670, 151704
SYSTEM, USER, ASSISTANT, NEWLINE = 8948, 872, 77091, 198


def prefix_ids(system_ids) -> list[int]:
    return [IM_START, SYSTEM, NEWLINE, *system_ids, IM_END, NEWLINE, IM_START, USER, NEWLINE,
            AUDIO_START]


def suffix_ids(language_ids=(), committed_ids=()) -> list[int]:
    return [AUDIO_END, IM_END, NEWLINE, IM_START, ASSISTANT, NEWLINE, *language_ids, ASR_TEXT,
            *committed_ids]


class GreedyHarvest:
    """DecodeGreedy's output rule applied token by token: an EOS id ends the
    output (not included); six equal tokens in a row end it (included)."""

    def __init__(self, eos0: int, eos1: int):
        self.eos = (eos0, eos1)
        self.out: list[int] = []
        self.done = False

    def push(self, t: int) -> bool:
        if self.done:
            return True
        if t in self.eos:
            self.done = True
            return True
        self.out.append(int(t))
        if len(self.out) >= 6 and all(x == self.out[-1] for x in self.out[-6:]):
            self.done = True
        return self.done


class AsrStreamPool:
    def __init__(self, weights, batch, max_new: int = 32, ban_steps: int = 3,
                 eos0: int = IM_END, eos1: int = END_OF_TEXT):
        """weights: AsrTextDecoder (for Embed), batch: BatchDecoder over it."""
        self.w, self.b = weights, batch
        self.max_new, self.ban_steps, self.eos0, self.eos1 = max_new, ban_steps, eos0, eos1
        self.ckpt: dict[int, int] = {}

    def _embed(self, ids) -> np.ndarray:
        return np.stack([self.w.Embed(int(t)) for t in ids]).astype(np.float32)

    def open(self, system_ids=()) -> int:
        sid = self.b.create_session()
        ids = prefix_ids(system_ids)
        self.b.prefill([sid], [self._embed(ids)])
        self.ckpt[sid] = len(ids)
        return sid

    def close(self, sid: int):
        self.b.free_session(sid)
        self.ckpt.pop(sid)

    def append_audio(self, sids, rows_list):
        """Encoder rows [T_i, 2048] of new audio windows, one array per session."""
        for sid in sids:
            self.b.truncate(sid, self.ckpt[sid])
        self.b.prefill(list(sids), [np.asarray(r, np.float32) for r in rows_list])
        for sid, r in zip(sids, rows_list):
            self.ckpt[sid] += len(r)

    def decode(self, requests: dict) -> dict:
        """requests: sid -> (language_ids, committed_ids). Returns sid -> the
        generated token ids (without EOS), as DecodeGreedy would."""
        sids = list(requests)
        if not sids:
            return {}
        for sid in sids:
            self.b.truncate(sid, self.ckpt[sid])
            self.b.set_ban(sid, self.eos0, self.eos1, self.ban_steps)
        self.b.prefill(sids, [self._embed(suffix_ids(*requests[s])) for s in sids])
        pending = dict(zip(sids, (int(t) for t in self.b.next_tokens(sids))))
        harvest = {s: GreedyHarvest(self.eos0, self.eos1) for s in sids}
        emitted = {s: 0 for s in sids}
        active = [s for s in sids if self.max_new > 0]
        while active:
            nxt = self.b.step(active)  # feeds each pending token, returns the next
            still = []
            for s, t in zip(active, nxt):
                emitted[s] += 1
                stop = harvest[s].push(pending[s])
                pending[s] = int(t)
                if not stop and emitted[s] < self.max_new:
                    still.append(s)
            active = still
        for sid in sids:
            self.b.truncate(sid, self.ckpt[sid])
            self.b.set_ban(sid, -1, -1, 0)
        return {s: harvest[s].out for s in sids}
