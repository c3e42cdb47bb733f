"""Prompt-hash reply store: the reply a server gave to a prompt, found again when the same prompt comes back.

A finished stream files its reply (the ids generated after the prompt) under a few keys of its prompt: a digest of the
whole prompt and of its last 1024, 256 and 64 ids, so a prompt that differs only near its head (a date or a session id
in a system part) still finds the reply. A new stream whose prompt hits a key copies from that reply from its first
generated id; after a divergence it lines up again inside the same reply on its last 4 generated ids (the occurrence
nearest to where the reply would be by now). The target verifies every copied id, so a stale or wrong reply costs one
forward and changes no output.

Layout: replies are content-addressed -- one `r-<digest>.ids` file (little-endian int32) per distinct reply -- and each
key is a small `k-<key>` file that names its reply's digest, so the four keys of one prompt share one reply file.
Both are written to a temporary name and renamed (atomic on POSIX), so readers in other processes never see half a
file; lookups read the files every time, so every process sharing the directory sees new replies and they survive a
restart. Past `cap` keys the least recently written keys go, and reply files no key names any more are removed. With
no directory the same maps live in memory.

Reference parity: xtier/packs/deepseek_v4/recall/core.py:1926-2060 (prompt-hash keys over the whole prompt and its
tails, a reply store on disk or in memory, the shortest and longest reply filed) and 2346-2391 (following the reply and
lining up again after a divergence). Content-addressed reply files, the key lengths and the realignment rule here are
this project's own.
"""
from __future__ import annotations

import collections
import hashlib
import os
import threading
from pathlib import Path

import numpy as np

KEY_TAILS = (0, 1024, 256, 64)   # 0: the whole prompt
REALIGN_GRAM = 4
MIN_REPLY = 8
MAX_REPLY = 16384
CAP = 8192                        # keys kept


def prompt_keys(prompt) -> list[str]:
    """The keys of a prompt, most specific first: the whole prompt, then tails shorter than it."""
    p = np.ascontiguousarray(np.asarray(prompt, dtype='<i8').ravel())
    out = []
    for k in KEY_TAILS:
        if k and p.shape[0] <= k:
            continue
        part = p if k == 0 else p[-k:]
        h = hashlib.blake2b(part.tobytes(), digest_size=16, key=b'xtier-reply-%d' % k).hexdigest()
        out.append(f't{k}-{h}')
    return out


def _digest(a32: np.ndarray) -> str:
    return hashlib.blake2b(a32.tobytes(), digest_size=16).hexdigest()


class ReplyStore:
    """key -> reply ids (int64 arrays); `path` None keeps the maps in memory. `writer` False never writes (a process
    that does not hold the record's lock)."""

    def __init__(self, path=None, cap: int = CAP, writer: bool = True):
        self.path = Path(path) if path is not None else None
        self.cap = max(4, int(cap))
        self.writer = bool(writer)
        self._keys: collections.OrderedDict = collections.OrderedDict()   # memory: key -> digest (oldest first)
        self._replies: dict = {}                                          # memory: digest -> int32 array
        self._lock = threading.Lock()
        self.puts = self.hits = self.misses = self.dropped = 0
        if self.path is not None and self.writer:
            self.path.mkdir(parents=True, exist_ok=True)
            os.chmod(self.path, 0o700)

    # ------------------------------------------------------------------ files
    def _write(self, name: str, data: bytes):
        tmp = self.path / f'.{name}.{os.getpid()}.{threading.get_ident()}'
        fd = os.open(tmp, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o600)
        with os.fdopen(fd, 'wb') as f:
            f.write(data)
        os.replace(tmp, self.path / name)

    def _read(self, name: str) -> bytes | None:
        try:
            with open(self.path / name, 'rb') as f:
                return f.read()
        except OSError:
            return None

    # ------------------------------------------------------------------ api
    def get(self, keys) -> np.ndarray | None:
        """The reply filed under the first key that has one (keys most specific first), or None."""
        for k in keys:
            if self.path is None:
                with self._lock:
                    d = self._keys.get(k)
                    a = self._replies.get(d) if d is not None else None
            else:
                d = self._read(f'k-{k}')
                raw = self._read(f'r-{d.decode()}.ids') if d else None
                a = np.frombuffer(raw[:len(raw) // 4 * 4], dtype='<i4') if raw else None
            if a is not None and a.shape[0] >= MIN_REPLY:
                self.hits += 1
                return a.astype(np.int64)
        self.misses += 1
        return None

    def put(self, keys, reply) -> bool:
        """Files `reply` under `keys` (replacing what they named); False when not written (read-only, too short, or
        ids outside int32)."""
        a = np.asarray(reply, dtype=np.int64).ravel()[:MAX_REPLY]
        if not self.writer or not keys or a.shape[0] < MIN_REPLY or a.min() < 0 or a.max() > 0x7FFFFFFF:
            return False
        a32 = a.astype('<i4')
        d = _digest(a32)
        with self._lock:
            self.puts += 1
            if self.path is None:
                self._replies[d] = a32
                for k in keys:
                    self._keys.pop(k, None)
                    self._keys[k] = d
                while len(self._keys) > self.cap:
                    self._keys.popitem(last=False)
                    self.dropped += 1
                if len(self._replies) > len(self._keys):
                    live = set(self._keys.values())
                    self._replies = {x: v for x, v in self._replies.items() if x in live}
                return True
            if not (self.path / f'r-{d}.ids').exists():
                self._write(f'r-{d}.ids', a32.tobytes())
            for k in keys:
                self._write(f'k-{k}', d.encode())
            if self.puts % max(1, self.cap // 16) == 0:
                self._trim()
        return True

    def _trim(self):
        """Drops the least recently written keys past `cap` and the reply files no key names."""
        ks = []
        for f in self.path.glob('k-*'):
            try:
                ks.append((f.stat().st_mtime_ns, f))
            except OSError:
                pass
        ks.sort()
        for _, f in ks[:max(0, len(ks) - self.cap)]:
            f.unlink(missing_ok=True)
            self.dropped += 1
        live = set()
        for _, f in ks[max(0, len(ks) - self.cap):]:
            try:
                live.add(f.read_text())
            except OSError:
                pass
        for f in self.path.glob('r-*.ids'):
            if f.name[2:-4] not in live:
                f.unlink(missing_ok=True)

    def count(self) -> int:
        if self.path is None:
            return len(self._keys)
        return sum(1 for _ in self.path.glob('k-*')) if self.path.is_dir() else 0

    def stats(self) -> dict:
        return dict(entries=self.count(), puts=self.puts, hits=self.hits, misses=self.misses, dropped=self.dropped)


def realign(reply: np.ndarray, out, expected: int, gram: int = REALIGN_GRAM) -> int:
    """Where in `reply` the id after `out` (the stream's generated ids) would come: just past an occurrence of
    `out`'s last `gram` ids, the one nearest to `expected`; -1 when there is none."""
    if len(out) < gram or reply.shape[0] <= gram:
        return -1
    tail = np.asarray(out[-gram:], np.int64)
    win = np.lib.stride_tricks.sliding_window_view(reply[:-1], gram)    # leaves at least one id to copy
    hits = np.nonzero((win == tail).all(axis=1))[0]
    if hits.shape[0] == 0:
        return -1
    ends = hits + gram
    return int(ends[np.argmin(np.abs(ends - expected))])
