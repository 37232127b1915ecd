"""Streaming front door (orator_b200/stream.py) on the host, over a scripted
stand-in for the batched engine: prompt layout, checkpoints and truncation,
the ban window and DecodeGreedy's stop rules (EOS ends the output, six equal
tokens end it), several sessions decoding together."""
import numpy as np

from orator_b200 import stream as S


class FakeWeights:
    def Embed(self, t):
        v = np.zeros(8, np.float32)
        v[0] = t
        return v


class FakeBatch:
    """Each session's greedy sequence is scripted; a banned token is replaced
    by token + 1 while the session's ban window is open."""

    def __init__(self, scripts):
        self.scripts = scripts      # sid -> list of tokens the model would produce
        self.len, self.ids, self.ban, self.pend, self.k = {}, {}, {}, {}, {}
        self.next_sid = 0

    def create_session(self):
        s = self.next_sid
        self.next_sid += 1
        self.len[s], self.ids[s], self.ban[s] = 0, [], (-1, -1, 0)
        return s

    def free_session(self, s):
        del self.len[s]

    def truncate(self, s, n):
        assert 0 <= n <= self.len[s]
        self.len[s] = n
        self.ids[s] = self.ids[s][:n]

    def set_ban(self, s, b0, b1, steps):
        self.ban[s] = (b0, b1, steps)

    def _argmax(self, s):
        t = self.scripts[s][self.k[s]]
        self.k[s] += 1
        b0, b1, left = self.ban[s]
        if left > 0:
            if t in (b0, b1):
                t += 1
            self.ban[s] = (b0, b1, left - 1)
        return t

    def prefill(self, sids, rows):
        for s, r in zip(sids, rows):
            self.ids[s] += [int(x[0]) for x in r]
            self.len[s] += len(r)
            if s in self.scripts and self.ids[s][-1] == S.ASR_TEXT or (
                    s in self.scripts and S.ASR_TEXT in self.ids[s][-len(r):]):
                self.k[s] = 0
                self.pend[s] = self._argmax(s)

    def next_tokens(self, sids):
        return np.array([self.pend[s] for s in sids])

    def step(self, sids):
        out = []
        for s in sids:
            self.ids[s].append(self.pend[s])
            self.len[s] += 1
            self.pend[s] = self._argmax(s)
            out.append(self.pend[s])
        return np.array(out)


def test_prompt_layout_and_checkpoints():
    b = FakeBatch({0: [5] * 40})
    pool = S.AsrStreamPool(FakeWeights(), b, max_new=4)
    sid = pool.open([11, 12])
    assert b.ids[sid] == [S.IM_START, S.SYSTEM, S.NEWLINE, 11, 12, S.IM_END, S.NEWLINE,
                          S.IM_START, S.USER, S.NEWLINE, S.AUDIO_START]
    ckpt = pool.ckpt[sid]
    audio = np.zeros((3, 8), np.float32) + 7
    pool.append_audio([sid], [audio])
    assert pool.ckpt[sid] == ckpt + 3 == b.len[sid]
    pool.decode({sid: ([99], [42, 43])})
    assert b.len[sid] == pool.ckpt[sid]  # suffix and generated tokens dropped
    # the next decode prefills the suffix right after the audio block again
    pool.decode({sid: ((), ())})
    assert b.len[sid] == pool.ckpt[sid]


def test_greedy_rules_and_ban_several_sessions():
    eos = S.IM_END
    scripts = {
        0: [eos, 3, 4, eos, 9, 9, 9, 9, 9, 9, 9],  # t0 is banned -> eos+1; stops at the 2nd eos
        1: [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12],  # runs to max_new
        2: [7, 7, 7, 7, 7, 7, 7, 7, 7, 7, 7, 7],  # six equal tokens
    }
    b = FakeBatch(scripts)
    pool = S.AsrStreamPool(FakeWeights(), b, max_new=10, ban_steps=3)
    sids = [pool.open() for _ in range(3)]
    out = pool.decode({s: ((), ()) for s in sids})
    assert out[0] == [eos + 1, 3, 4]
    assert out[1] == [1, 2, 3, 4, 5, 6, 7, 8, 9, 10]
    assert out[2] == [7] * 6
    assert all(b.len[s] == pool.ckpt[s] for s in sids)
    assert all(b.ban[s][2] == 0 for s in sids)
