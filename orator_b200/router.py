"""Placement of independent decode sessions on the GPUs of one node.

One process per GPU; sessions never exchange data, so the decode path has no
collective. What the ranks share is the placement rule: a new session goes to
the rank with the least total KV length (sum of its sessions' cache lengths)
among the ranks whose page pool can still hold it; ties go to the lowest rank.
Every rank applies the rule to the same inputs, so all ranks agree on every
placement without messages. ``gather_loads`` (host side, any torch.distributed
backend) lets ranks replace the modelled loads by reported ones, e.g. when
sessions end early on one rank; it is the only exchange, and it runs between
decode steps.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class RankLoad:
    kv_tokens: int = 0            # sum of cache lengths of the rank's sessions
    free_pages: int = 0
    sessions: set = field(default_factory=set)


class SessionRouter:
    def __init__(self, world: int, pages_per_rank: int, page: int = 16):
        if world < 1 or pages_per_rank < 1:
            raise ValueError("world and pages_per_rank must be positive")
        self.world, self.page = world, page
        self.ranks = [RankLoad(0, pages_per_rank) for _ in range(world)]
        self.where: dict[int, int] = {}
        self.lens: dict[int, int] = {}

    def _pages(self, tokens: int) -> int:
        return (tokens + self.page - 1) // self.page

    def place(self, sid: int, kv_len: int, headroom: int = 0) -> int:
        """Rank for new session `sid` holding `kv_len` tokens, with room for
        `headroom` more; raises RuntimeError when no rank has the pages."""
        if sid in self.where:
            raise ValueError(f"session {sid} already placed")
        need = self._pages(kv_len + headroom)
        best = None
        for r, ld in enumerate(self.ranks):
            if ld.free_pages < need:
                continue
            if best is None or ld.kv_tokens < self.ranks[best].kv_tokens:
                best = r
        if best is None:
            raise RuntimeError("no rank has free pages for the session")
        ld = self.ranks[best]
        ld.kv_tokens += kv_len
        ld.free_pages -= self._pages(kv_len)
        ld.sessions.add(sid)
        self.where[sid] = best
        self.lens[sid] = kv_len
        return best

    def grow(self, sid: int, n: int = 1):
        """Session `sid` appended n tokens (new pages are taken as needed);
        raises RuntimeError, changing nothing, when its rank lacks the pages."""
        r = self.where[sid]
        old = self.lens[sid]
        extra = self._pages(old + n) - self._pages(old)
        if extra > self.ranks[r].free_pages:
            raise RuntimeError(f"rank {r} has no free page for session {sid}")
        self.ranks[r].free_pages -= extra
        self.ranks[r].kv_tokens += n
        self.lens[sid] = old + n

    def release(self, sid: int):
        r = self.where.pop(sid)
        n = self.lens.pop(sid)
        ld = self.ranks[r]
        ld.kv_tokens -= n
        ld.free_pages += self._pages(n)
        ld.sessions.discard(sid)

    def rank_of(self, sid: int) -> int:
        return self.where[sid]

    def sessions_on(self, rank: int) -> list[int]:
        return sorted(self.ranks[rank].sessions)

    def loads(self) -> list[int]:
        return [ld.kv_tokens for ld in self.ranks]

    def gather_loads(self, rank: int, kv_tokens: int, free_pages: int, lens=None, group=None):
        """Replace the modelled state of every rank by what the ranks report
        (collective over `group`; host only): (kv_tokens, free_pages) and, in
        `lens`, the measured cache length of each of the reporting rank's
        sessions (sid -> tokens). Reported lengths replace the modelled ones,
        so a later `release` returns what the rank actually held; sessions a
        rank does not report keep their modelled length."""
        import torch.distributed as dist
        got = [None] * self.world
        dist.all_gather_object(got, (rank, int(kv_tokens), int(free_pages),
                                     {int(k): int(v) for k, v in (lens or {}).items()}),
                               group=group)
        for r, kv, fp, ln in got:
            self.ranks[r].kv_tokens = kv
            self.ranks[r].free_pages = fp
            for sid, n in ln.items():
                if self.where.get(sid) == r:
                    self.lens[sid] = n
