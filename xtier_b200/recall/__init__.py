"""Recall: a persistent record of the token ids a server has read and written, and copy drafts from it for speculative
decoding (the target model verifies every copied token, so the output is the same with Recall on or off).

`Record` keeps token ids only: chunks of up to 2^20 int32 ids (on disk: `chunk-NNNNNNNN.ids` files, 0600, in a 0700
directory with an `identity.json` naming the tokenizer and a `lock` file; or in memory). A separator id (-1) ends
every added run, so no match crosses two unrelated texts. Every window of 16 consecutive ids is indexed by a 64-bit
hash (a polynomial over the ids, then the SplitMix64 finalizer of Steele, Lea and Flood, 2014): each chunk's index is
a few sorted runs of (hash, position) numpy arrays -- one per add, merged into one when the chunk fills -- searched with
binary search, so a lookup costs a few dozen `searchsorted` calls and no Python dictionary of millions of entries.
Adding a text skips stretches of 128 or more ids the record already holds (keeping 32 ids at each edge, so windows
across the cut stay indexed): a request sent twice adds nothing new. Past the id budget the oldest chunk goes first;
with less than `min_free_gib` on the record's file system nothing is added. One process holds the lock and writes;
the others open the record read-only and `refresh()` to see new chunks.

`RecallEngine` makes the copy decisions per stream: a stream's own context is asked first (a per-stream index) and
wins ties, then the record; a candidate is the continuation after the longest match (16 ids or more, extended back up
to 128) of the stream's last 16 ids. Expected landed tokens are kept per source and match tier (16-31, 32-63, 64+
ids) as decayed means with a prior; a copy is offered when its expectation reaches the stream's own draft yield (or
`min_n`). A stream whose copy landed nothing leaves copies alone for `cooldown` rounds; a source whose expectation
fell below the bar is only probed, rarer after every probe that misses.

(Reference parity: xtier/packs/deepseek_v4/recall/core.py -- RecallRecord (ids-only chunk files, identity, lock,
dedup of repeated runs, FIFO budget, min free space, read-only refresh) and RecallEngine (own context first, match tiers,
cooldown after a miss, probes, the heat-ordered eviction with its hot zone) and the proposal broadcast to the
tensor-parallel ranks (`sync_proposal`). The index layout, hash, expectation rule and heat bookkeeping here are this
project's own; the copies also feed multi-branch draft trees (`RecallEngine.candidates`, runtime/tree.py). The
prompt-hash reply store (a third source, asked first: the reply filed for the same prompt) is in replies.py. Not
built: the GPU-resident id store.)
"""
from __future__ import annotations

import dataclasses
import json
import math
import os
import shutil
from pathlib import Path

import numpy as np

from .replies import REALIGN_GRAM, ReplyStore, prompt_keys, realign

WINDOW = 16
SENTINEL = -1
CHUNK_IDS = 1 << 20
DEDUP_RUN = 128
OVERLAP = 32
MAX_BACK = 128
MAX_RUNS = 8            # sorted index runs per chunk before they are merged
HEAT_SEG = 256          # heat eviction: the record's segments by global position
HOT_PRE, HOT_POST = WINDOW, 64   # ids a promoted segment takes along before and after it
HOT_FLAG = 1 << 62      # positions at or above it name a hot-zone entry: HOT_FLAG + (uid << 20) + offset
_P = np.uint64(0x100000001B3)          # odd multiplier of the polynomial window hash
_M1 = np.uint64(0xBF58476D1CE4E5B9)    # SplitMix64 finalizer constants
_M2 = np.uint64(0x94D049BB133111EB)


def window_hashes(a: np.ndarray, w: int = WINDOW) -> tuple[np.ndarray, np.ndarray]:
    """(hashes uint64, start offsets) of every window of `w` ids of `a` that contains no separator."""
    a = np.asarray(a, dtype=np.int64)
    n = a.shape[0] - w + 1
    if n <= 0:
        return np.zeros(0, np.uint64), np.zeros(0, np.int64)
    with np.errstate(over='ignore'):
        v = (a & 0xFFFFFFFF).astype(np.uint64)
        h = np.zeros(n, np.uint64)
        for k in range(w):
            h = h * _P + v[k:k + n]
        h ^= h >> np.uint64(30)
        h *= _M1
        h ^= h >> np.uint64(27)
        h *= _M2
        h ^= h >> np.uint64(31)
    bad = np.convolve((a == SENTINEL).astype(np.int64), np.ones(w, np.int64), 'valid') > 0
    keep = ~bad
    return h[keep], np.nonzero(keep)[0].astype(np.int64)


class _Chunk:
    def __init__(self, seq: int, ids: np.ndarray | None = None):
        self.seq = seq
        self.ids = np.empty(CHUNK_IDS, np.int32)
        self.n = 0
        self.runs: list[tuple[np.ndarray, np.ndarray]] = []   # sorted (hashes, global window starts)
        if ids is not None:
            self.ids[:ids.shape[0]] = ids
            self.n = ids.shape[0]

    @property
    def base(self) -> int:
        return self.seq * CHUNK_IDS

    def index(self, lo: int, hi: int):
        """Indexes the windows starting in [lo, hi) (offsets in this chunk; a window may not leave the chunk)."""
        seg = self.ids[max(0, lo):min(self.n, hi + WINDOW - 1)]
        h, off = window_hashes(seg)
        if h.shape[0] == 0:
            return
        order = np.argsort(h, kind='stable')
        self.runs.append((h[order], off[order] + max(0, lo) + self.base))
        if len(self.runs) > MAX_RUNS:
            self.merge()

    def merge(self):
        if len(self.runs) > 1:
            h = np.concatenate([r[0] for r in self.runs])
            p = np.concatenate([r[1] for r in self.runs])
            order = np.argsort(h, kind='stable')
            self.runs = [(h[order], p[order])]

    def find(self, h: int) -> list[int]:
        key = np.uint64(h)
        out = []
        for hs, ps in self.runs:
            i = int(np.searchsorted(hs, key))
            while i < hs.shape[0] and hs[i] == key:
                out.append(int(ps[i]))
                i += 1
        return out

    def contains(self, hs: np.ndarray) -> np.ndarray:
        """For every hash of `hs`, whether this chunk indexes it."""
        found = np.zeros(hs.shape[0], bool)
        for rh, _ in self.runs:
            i = np.searchsorted(rh, hs)
            i = np.minimum(i, rh.shape[0] - 1)
            found |= rh[i] == hs
        return found


class _HotEntry:
    """A promoted stretch of the record: its ids, their sorted window index and its heat (log domain)."""

    def __init__(self, uid: int, ids: np.ndarray, heat: float, seg: int):
        self.uid, self.ids, self.heat, self.seg = uid, ids, heat, seg
        h, off = window_hashes(ids)
        order = np.argsort(h, kind='stable')
        self.h, self.off = h[order], off[order]

    def find(self, h: int) -> list[int]:
        key = np.uint64(h)
        i = int(np.searchsorted(self.h, key))
        out = []
        while i < self.h.shape[0] and self.h[i] == key:
            out.append(int(self.off[i]))
            i += 1
        return out


class Record:
    """Token ids with a 16-id window index; `path` None keeps everything in memory.

    Eviction (`evict`): 'fifo' drops the oldest chunk past the id budget. 'heat' (default) also keeps a decayed heat
    per 256-id segment of the record -- the copied tokens the target accepted from it, halving every
    `heat_halflife_ids` ids added -- and copies a segment whose heat reaches `promote` (with 16 ids before it and 64
    after) into a hot zone of `hot_frac` of the budget, which the chunks' FIFO eviction does not touch; a full hot zone
    drops its coldest entry first. Lookups search the chunks and the hot zone (the longer match wins, the hot one on
    ties). The hot zone lives in memory: after a restart it fills again as copies land."""

    def __init__(self, path=None, identity: dict | None = None, budget_ids: int = 1 << 24, min_free_gib: float = 1.0,
                 dedup: bool = True, evict: str = 'heat', hot_frac: float = 0.25,
                 heat_halflife_ids: float | None = None, promote: float = 24.0):
        self.path = Path(path) if path is not None else None
        self.identity = identity or {}
        self.budget_ids = max(CHUNK_IDS, int(budget_ids))
        if evict not in ('heat', 'fifo'):
            raise ValueError(f'evict must be heat or fifo, not {evict!r}')
        self.evict_mode = evict
        self.hot_cap = int(self.budget_ids * min(0.9, max(0.0, hot_frac))) if evict == 'heat' else 0
        self.cold_budget = max(CHUNK_IDS, self.budget_ids - self.hot_cap)
        self.halflife = float(heat_halflife_ids or max(1, self.cold_budget // 4))
        self.promote_at = float(promote)
        self.clock = 0.0           # ids added so far (the heat's time axis)
        self.heat: dict[int, float] = {}   # segment -> log2(score) + clock / halflife
        self.hot: dict[int, _HotEntry] = {}
        self.hot_segs: set[int] = set()
        self.hot_ids = 0
        self._uid = 0
        self.promoted = self.hot_dropped = 0
        self.min_free_gib = min_free_gib
        self.dedup = dedup
        self.chunks: list[_Chunk] = []
        self.writer = True
        self._lock = None
        self.added = self.skipped = self.evicted = 0
        if self.path is not None:
            self._open_dir()

    # ------------------------------------------------------------------ disk
    def _open_dir(self):
        p = self.path
        p.mkdir(parents=True, exist_ok=True)
        os.chmod(p, 0o700)
        ident = p / 'identity.json'
        if ident.exists():
            have = json.loads(ident.read_text())
            if self.identity and have != self.identity:
                raise RuntimeError(f'recall record {p} belongs to another tokenizer: {have} != {self.identity}')
            self.identity = have
        else:
            fd = os.open(ident, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o600)
            with os.fdopen(fd, 'w') as f:
                f.write(json.dumps(self.identity))
        import fcntl
        self._lock = open(p / 'lock', 'a+')
        try:
            fcntl.flock(self._lock.fileno(), fcntl.LOCK_EX | fcntl.LOCK_NB)
        except OSError:
            self.writer = False
        self.refresh()

    def _chunk_file(self, seq: int) -> Path:
        return self.path / f'chunk-{seq:08d}.ids'

    def refresh(self) -> int:
        """Reads chunks (and growth of the last one) other processes wrote; returns ids read."""
        if self.path is None:
            return 0
        seqs = sorted(int(f.name[6:14]) for f in self.path.glob('chunk-*.ids'))
        have = {c.seq: c for c in self.chunks}
        self.chunks = [have[s] for s in seqs if s in have]   # chunks evicted elsewhere go
        read = 0
        for s in seqs:
            data = np.fromfile(self._chunk_file(s), dtype='<i4')
            c = have.get(s)
            if c is None:
                c = _Chunk(s, data.astype(np.int32))
                c.index(0, c.n)
                c.merge()
                self.chunks.append(c)
                read += c.n
            elif data.shape[0] > c.n:
                lo = c.n
                c.ids[lo:data.shape[0]] = data[lo:]
                c.n = data.shape[0]
                c.index(lo - WINDOW + 1, c.n)
                read += c.n - lo
        self.chunks.sort(key=lambda c: c.seq)
        return read

    # ------------------------------------------------------------------ add
    @property
    def size(self) -> int:
        return sum(c.n for c in self.chunks)

    def _seen(self, a: np.ndarray) -> np.ndarray:
        """Per id of `a`: whether it lies in a run of >= DEDUP_RUN ids whose windows the record already indexes,
        keeping OVERLAP ids at each edge of the run."""
        h, off = window_hashes(a)
        if h.shape[0] == 0 or not self.chunks:
            return np.zeros(a.shape[0], bool)
        known = np.zeros(h.shape[0], bool)
        for c in self.chunks:
            known |= c.contains(h)
        win = np.zeros(a.shape[0] - WINDOW + 1, bool)
        win[off] = known
        skip = np.zeros(a.shape[0], bool)
        i, n = 0, win.shape[0]
        while i < n:
            if not win[i]:
                i += 1
                continue
            j = i
            while j < n and win[j]:
                j += 1
            lo, hi = i, j - 1 + WINDOW          # ids [lo, hi) are covered by known windows
            if hi - lo >= DEDUP_RUN:            # keep OVERLAP ids where the run meets new text, none at the ends
                skip[lo + (OVERLAP if lo > 0 else 0):hi - (OVERLAP if hi < a.shape[0] else 0)] = True
            i = j
        return skip

    def _append(self, seg: np.ndarray, sep: bool = True):
        seg = np.asarray(seg, np.int32)
        if sep:
            seg = np.concatenate([seg, np.array([SENTINEL], np.int32)])
        while seg.shape[0]:
            if not self.chunks or self.chunks[-1].n == CHUNK_IDS:
                if self.chunks:
                    self.chunks[-1].merge()
                self.chunks.append(_Chunk(self.chunks[-1].seq + 1 if self.chunks else 0))
            c = self.chunks[-1]
            k = min(seg.shape[0], CHUNK_IDS - c.n)
            lo = c.n
            c.ids[lo:lo + k] = seg[:k]
            c.n += k
            if self.path is not None:
                fd = os.open(self._chunk_file(c.seq), os.O_WRONLY | os.O_CREAT | os.O_APPEND, 0o600)
                with os.fdopen(fd, 'ab') as f:
                    f.write(seg[:k].astype('<i4').tobytes())
            c.index(lo - WINDOW + 1, c.n)
            seg = seg[k:]

    def _evict(self):
        while len(self.chunks) > 1 and self.size > self.cold_budget:
            c = self.chunks.pop(0)
            self.evicted += c.n
            if self.path is not None:
                self._chunk_file(c.seq).unlink(missing_ok=True)
        if self.heat and self.chunks:   # the heat of segments no longer held
            first = self.chunks[0].base // HEAT_SEG
            for seg in [g for g in self.heat if g < first]:
                del self.heat[seg]

    # ------------------------------------------------------------------ heat
    def _score(self, L: float) -> float:
        """A log-domain heat as the decayed score now."""
        return 2.0 ** (L - self.clock / self.halflife)

    def _bump(self, L: float | None, x: float) -> float:
        now = self.clock / self.halflife
        score = (2.0 ** (L - now) if L is not None else 0.0) + x
        return math.log2(max(score, 1e-30)) + now

    def credit(self, pos: int, n: int):
        """The target accepted `n` copied tokens read from position `pos` (a record or hot-zone position)."""
        if self.evict_mode != 'heat' or n <= 0:
            return
        if pos >= HOT_FLAG:
            e = self.hot.get((pos - HOT_FLAG) >> 20)
            if e is not None:
                e.heat = self._bump(e.heat, n)
            return
        for seg in range(pos // HEAT_SEG, (pos + n - 1) // HEAT_SEG + 1):
            lo, hi = max(pos, seg * HEAT_SEG), min(pos + n, (seg + 1) * HEAT_SEG)
            self.heat[seg] = self._bump(self.heat.get(seg), hi - lo)
            if seg not in self.hot_segs and self._score(self.heat[seg]) >= self.promote_at:
                self._promote(seg)

    def _promote(self, seg: int):
        if not self.chunks:
            return
        g_lo, g_hi = self.chunks[0].base, self.chunks[-1].base + self.chunks[-1].n
        g0, g1 = max(g_lo, seg * HEAT_SEG - HOT_PRE), min(g_hi, (seg + 1) * HEAT_SEG + HOT_POST)
        ids = self._ids(g0, g1) if g0 < g1 else None
        if ids is None or ids.shape[0] < WINDOW or ids.shape[0] > self.hot_cap:
            return
        L = self.heat[seg]
        while self.hot_ids + ids.shape[0] > self.hot_cap:   # the coldest entries make room, if colder than this one
            cold = min(self.hot.values(), key=lambda e: e.heat)
            if cold.heat >= L:
                return
            del self.hot[cold.uid]
            self.hot_segs.discard(cold.seg)
            self.hot_ids -= cold.ids.shape[0]
            self.hot_dropped += 1
        self._uid += 1
        e = _HotEntry(self._uid, np.array(ids, np.int32), L, seg)
        self.hot[e.uid] = e
        self.hot_segs.add(seg)
        self.hot_ids += e.ids.shape[0]
        self.promoted += 1

    def add(self, ids) -> int:
        """Adds a text; returns the ids stored (0 when read-only, short of disk space, or all already held)."""
        if not self.writer:
            return 0
        if self.path is not None and shutil.disk_usage(self.path).free < self.min_free_gib * (1 << 30):
            return 0
        a = np.asarray(ids, dtype=np.int64)
        a = a[a >= 0]
        if a.shape[0] < WINDOW:
            return 0
        skip = self._seen(a) if self.dedup else np.zeros(a.shape[0], bool)
        stored = 0
        i = 0
        while i < a.shape[0]:     # the kept stretches, each ended by a separator
            if skip[i]:
                i += 1
                continue
            j = i
            while j < a.shape[0] and not skip[j]:
                j += 1
            if j - i >= WINDOW:
                self._append(a[i:j])
                stored += j - i
            i = j
        self.added += stored
        self.clock += stored
        self.skipped += int(skip.sum())
        self._evict()
        return stored

    # ------------------------------------------------------------------ lookup
    def _ids(self, g0: int, g1: int) -> np.ndarray | None:
        """Ids of global positions [g0, g1) if they are still held (one chunk or two)."""
        out = []
        for c in self.chunks:
            lo, hi = max(g0, c.base), min(g1, c.base + c.n)
            if lo < hi:
                out.append(c.ids[lo - c.base:hi - c.base])
        if not out:
            return None
        r = np.concatenate(out)
        return r if r.shape[0] == g1 - g0 else None

    def lookup(self, tail, max_back: int = MAX_BACK):
        """(match length, position after the match) of the longest match of `tail`'s last ids (>= WINDOW), newest
        first on ties; None without one."""
        t = np.asarray(tail, dtype=np.int64)
        if t.shape[0] < WINDOW:
            return None
        h, off = window_hashes(t[-WINDOW:])
        if h.shape[0] == 0:
            return None
        best = None
        for c in reversed(self.chunks):
            for p in sorted(c.find(int(h[0])), reverse=True):
                w = self._ids(p, p + WINDOW)
                if w is None or not np.array_equal(w, t[-WINDOW:]):
                    continue                              # a hash collision
                back = 0
                lim = min(max_back, t.shape[0] - WINDOW)
                if lim > 0:
                    g0 = max(self.chunks[0].base, p - lim)
                    prev = self._ids(g0, p)
                    if prev is not None:
                        mine = t[-WINDOW - (p - g0):-WINDOW] if p > g0 else t[:0]
                        eq = prev[::-1] == mine[::-1]
                        back = int(np.argmin(eq)) if not eq.all() else eq.shape[0]
                m = WINDOW + back
                if best is None or m > best[0]:
                    best = (m, p + WINDOW)
        for e in self.hot.values():   # the hot zone: the longer match wins, the hot one on ties
            for o in e.find(int(h[0])):
                if not np.array_equal(e.ids[o:o + WINDOW], t[-WINDOW:]):
                    continue
                lim = min(max_back, t.shape[0] - WINDOW, o)
                back = 0
                if lim > 0:
                    eq = e.ids[o - lim:o][::-1] == t[-WINDOW - lim:-WINDOW][::-1]
                    back = int(np.argmin(eq)) if not eq.all() else lim
                m = WINDOW + back
                if best is None or m >= best[0]:
                    best = (m, HOT_FLAG + (e.uid << 20) + o + WINDOW)
        return best

    def continuation(self, pos: int, n: int) -> np.ndarray:
        """Up to n ids from global position `pos` (or a hot-zone position), stopping at a separator."""
        if pos >= HOT_FLAG:
            e = self.hot.get((pos - HOT_FLAG) >> 20)
            if e is None:
                return np.zeros(0, np.int32)
            o = (pos - HOT_FLAG) & ((1 << 20) - 1)
            ids = e.ids[o:o + n]
            stop = np.nonzero(ids == SENTINEL)[0]
            return ids[:stop[0]] if stop.shape[0] else ids
        ids = self._ids(pos, pos + n)
        if ids is None:
            for k in range(n - 1, 0, -1):
                ids = self._ids(pos, pos + k)
                if ids is not None:
                    break
            else:
                return np.zeros(0, np.int32)
        stop = np.nonzero(ids == SENTINEL)[0]
        return ids[:stop[0]] if stop.shape[0] else ids

    def stats(self) -> dict:
        return dict(ids=self.size, chunks=len(self.chunks), added=self.added, skipped=self.skipped,
                    evicted=self.evicted, writer=self.writer, evict=self.evict_mode, hot_entries=len(self.hot),
                    hot_ids=self.hot_ids, promoted=self.promoted, hot_dropped=self.hot_dropped,
                    heat_segments=len(self.heat))

    def clear(self):
        if not self.writer:
            return
        for c in self.chunks:
            if self.path is not None:
                self._chunk_file(c.seq).unlink(missing_ok=True)
        self.chunks = []
        self.heat, self.hot, self.hot_segs, self.hot_ids = {}, {}, set(), 0

    def close(self):
        if self._lock is not None:
            self._lock.close()
            self._lock = None


def tier_of(match: int) -> int:
    return 0 if match < 32 else (1 if match < 64 else 2)


@dataclasses.dataclass
class Proposal:
    source: str          # 'own', 'record' or 'reply'
    ids: list[int]
    match: int
    tier: int
    probe: bool = False
    pos: int = -1        # record position of the copy (heat credit)


class _Stream:
    def __init__(self, prompt, reply_from: int | None = None):
        self.own = Record(None, dedup=False)
        self.ids: list[int] = list(prompt)
        self.indexed = 0
        self.cooldown = 0
        self.own_yield = 0.0     # tokens the stream's own draft model lands per round (0: none)
        self.last: Proposal | None = None
        self.prompt_len = len(prompt) if reply_from is None else int(reply_from)
        self.reply_keys: list[str] = []
        self.reply: np.ndarray | None = None   # a filed reply to the same prompt
        self.rpos = -1           # where in `reply` the stream's next id is expected (-1: not lined up)
        self.run = 0             # ids the stream agreed with `reply` since it lined up

    def follow(self, ids):
        """Moves the reply position along the stream's new ids; a mismatch leaves the reply (-1)."""
        if self.reply is None:
            return
        for t in ids:
            if 0 <= self.rpos < self.reply.shape[0] and int(self.reply[self.rpos]) == t:
                self.rpos += 1
                self.run += 1
            else:
                self.rpos, self.run = -1, 0


class RecallEngine:
    SOURCES = ('own', 'record', 'reply')

    def __init__(self, record: Record | None, gamma: int = 16, min_n: float = 2.0, cooldown: int = 4,
                 prior: float = 0.5, prior_weight: float = 2.0, decay: float = 0.98, probe_start: int = 16,
                 probe_max: int = 4096, replies=True):
        """`replies`: a `ReplyStore`, True (the default: one beside the record -- `<record>/replies` for a record on
        disk, written only by the process that writes the record -- or in memory), or None / False (off)."""
        self.record = record
        if replies is True:
            on_disk = record is not None and record.path is not None
            replies = ReplyStore(record.path / 'replies' if on_disk else None,
                                 writer=record.writer if on_disk else True)
        self.replies = replies or None
        self.reply_hits = self.realigns = 0
        self.gamma = gamma
        self.min_n = min_n
        self.cooldown = cooldown
        self.prior, self.prior_w, self.decay = prior * gamma, prior_weight, decay
        self.sums = {(s, t): [0.0, 0.0] for s in self.SOURCES for t in range(3)}   # decayed (landed, offers)
        self.probe_iv = {s: probe_start for s in self.SOURCES}
        self.probe_left = {s: probe_start for s in self.SOURCES}
        self.probe_start, self.probe_max = probe_start, probe_max
        self.streams: dict = {}
        self.offers = self.probes = self.landed = 0

    # ------------------------------------------------------------------ streams
    def begin_stream(self, rid, prompt_ids, reply_from: int | None = None):
        """A new stream; `reply_from` is where its reply starts in `prompt_ids` (default: after all of them -- a
        caller that already sampled the first reply id passes the prompt's length)."""
        st = self.streams[rid] = _Stream([int(t) for t in prompt_ids], reply_from)
        if self.replies is not None and st.prompt_len > 0:
            st.reply_keys = prompt_keys(st.ids[:st.prompt_len])
            ans = self.replies.get(st.reply_keys)
            if ans is not None:
                st.reply, st.rpos, st.run = ans, 0, 64     # a prompt hit ranks as a long match
                self.reply_hits += 1
                st.follow(st.ids[st.prompt_len:])

    def extend_stream(self, rid, ids):
        st = self.streams[rid]
        ids = [int(t) for t in ids]
        st.ids += ids
        st.follow(ids)

    def end_stream(self, rid, add: bool = True):
        st = self.streams.pop(rid)
        if add and self.record is not None:
            self.record.add(st.ids)
        if add and self.replies is not None and st.reply_keys:
            self.replies.put(st.reply_keys, st.ids[st.prompt_len:])

    def observe_own(self, rid, landed: float, alpha: float = 0.25):
        """The stream's own draft model landed `landed` tokens this round (the bar a copy must reach)."""
        st = self.streams[rid]
        st.own_yield = (1 - alpha) * st.own_yield + alpha * landed

    # ------------------------------------------------------------------ decisions
    def expect(self, source: str, tier: int) -> float:
        landed, offers = self.sums[(source, tier)]
        return (self.prior * self.prior_w + landed) / (self.prior_w + offers)

    def _own_candidate(self, st: _Stream):
        if len(st.ids) - st.indexed >= WINDOW:    # index the stream's history except its last window
            hi = len(st.ids) - 1
            st.own._append(np.asarray(st.ids[st.indexed:hi], np.int64), sep=False)   # one continuous text
            st.indexed = hi
        m = st.own.lookup(st.ids)
        if m is None:
            return None
        cont = st.own.continuation(m[1], self.gamma)
        return (m[0], cont) if cont.shape[0] else None

    def _record_candidate(self, st: _Stream):
        if self.record is None:
            return None
        m = self.record.lookup(st.ids)
        if m is None:
            return None
        cont = self.record.continuation(m[1], self.gamma)
        return (m[0], cont, m[1]) if cont.shape[0] else None

    def _reply_candidate(self, st: _Stream):
        if st.reply is None:
            return None
        out = st.ids[st.prompt_len:]
        if st.rpos < 0:
            st.rpos = realign(st.reply, out, len(out))
            if st.rpos < 0:
                return None
            st.run = REALIGN_GRAM
            self.realigns += 1
        cont = st.reply[st.rpos:st.rpos + self.gamma]
        return (max(st.run, WINDOW), cont) if cont.shape[0] else None

    def _sources(self, st: _Stream):
        return (('reply', self._reply_candidate(st)), ('own', self._own_candidate(st)),
                ('record', self._record_candidate(st)))

    def propose(self, rid) -> Proposal | None:
        st = self.streams[rid]
        if st.cooldown > 0:
            st.cooldown -= 1
            return None
        cands = []
        for src, cand in self._sources(st):
            if cand is not None:
                cands.append((self.expect(src, tier_of(cand[0])), src == 'own', src, cand))
        if not cands:
            return None
        cands.sort(key=lambda c: (c[0], c[1]), reverse=True)    # best expectation, own context on ties
        e, _, src, cand = cands[0]
        match, cont = cand[0], cand[1]
        bar = max(self.min_n, st.own_yield)
        probe = False
        if e < bar:                    # below the bar: only a probe now and then
            self.probe_left[src] -= 1
            if self.probe_left[src] > 0:
                return None
            probe = True
            self.probe_left[src] = self.probe_iv[src]
        p = Proposal(src, [int(t) for t in cont], match, tier_of(match), probe,
                     cand[2] if src == 'record' else -1)
        st.last = p
        self.offers += 1
        self.probes += probe
        return p

    def candidates(self, rid) -> list[Proposal]:
        """Every available copy of the stream (a filed reply's, its own context's and the record's), without the
        offer rule: the branches of a draft tree, which the target verifies in the same forward as the other drafts."""
        st = self.streams[rid]
        out = []
        for src, cand in self._sources(st):
            if cand is not None:
                out.append(Proposal(src, [int(t) for t in cand[1]], cand[0], tier_of(cand[0]), False,
                                    cand[2] if src == 'record' else -1))
        return out

    def note(self, p: Proposal, landed: int):
        """`landed` tokens of copy `p` were accepted: the expectation of its source and tier, and the record's heat."""
        for k in self.sums:
            self.sums[k][0] *= self.decay
            self.sums[k][1] *= self.decay
        s = self.sums[(p.source, p.tier)]
        s[0] += landed
        s[1] += 1
        self.landed += landed
        if p.source == 'record' and p.pos >= 0 and self.record is not None:
            self.record.credit(p.pos, landed)

    def feedback(self, rid, landed: int):
        """The target accepted `landed` tokens of the last proposal."""
        st = self.streams[rid]
        p, st.last = st.last, None
        if p is None:
            return
        self.note(p, landed)
        if landed == 0:
            st.cooldown = self.cooldown
        if p.probe:
            self.probe_iv[p.source] = (self.probe_start if landed > 0 else
                                       min(self.probe_max, self.probe_iv[p.source] * 2))

    def stats(self) -> dict:
        return dict(offers=self.offers, probes=self.probes, landed=self.landed,
                    expect={f'{s}/{t}': round(self.expect(s, t), 3) for s, t in self.sums},
                    record=self.record.stats() if self.record is not None else None,
                    replies=(dict(self.replies.stats(), prompt_hits=self.reply_hits, realigns=self.realigns)
                             if self.replies is not None else None))


_SOURCE_CODE = {s: i for i, s in enumerate(RecallEngine.SOURCES)}


def sync_proposal(prop: Proposal | None, group=None, src: int = 0) -> Proposal | None:
    """Every rank of `group` takes rank `src`'s proposal (tensor-parallel ranks must verify the same drafts; only
    `src` keeps a record and an engine). One broadcast of a small int64 tensor: [count, match, tier, probe, source,
    ids...] padded to a fixed length; the source is its index in `RecallEngine.SOURCES`."""
    import torch
    import torch.distributed as dist
    cap = 64
    buf = torch.full((5 + cap,), -1, dtype=torch.int64)
    if dist.get_rank(group) == src if group is not None else dist.get_rank() == src:
        if prop is not None and prop.ids:
            ids = prop.ids[:cap]
            buf[:5] = torch.tensor([len(ids), prop.match, prop.tier, int(prop.probe), _SOURCE_CODE[prop.source]])
            buf[5:5 + len(ids)] = torch.tensor(ids)
        else:
            buf[0] = 0
    dist.broadcast(buf, src=src if group is None else dist.get_global_rank(group, src), group=group)
    n = int(buf[0])
    if n <= 0:
        return None
    return Proposal(RecallEngine.SOURCES[int(buf[4])], buf[5:5 + n].tolist(), int(buf[1]), int(buf[2]),
                    bool(buf[3]))


def tokenizer_identity(tokenizer, model_name: str = '') -> dict:
    """What a record's ids mean: the tokenizer's class, vocabulary size and a digest of its vocabulary."""
    import hashlib
    vocab = tokenizer.get_vocab() if hasattr(tokenizer, 'get_vocab') else {}
    digest = hashlib.sha256(json.dumps(sorted(vocab.items())).encode()).hexdigest()[:16] if vocab else ''
    return dict(tokenizer=type(tokenizer).__name__, vocab=len(vocab), digest=digest, model=model_name)
