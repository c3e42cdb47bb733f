"""Recall on the CPU: the record's lookup / dedup / budget / persistence / lock, the engine's copy decisions, and
speculative decoding with copy drafts against a stand-in target (greedy output unchanged, copies land)."""
import os
import stat

import numpy as np
import pytest
import torch

from xtier_b200 import recall
from xtier_b200.runtime.speculative import SpeculativeDecoder


def _text(n, seed, vocab=5000):
    return np.random.default_rng(seed).integers(0, vocab, n).tolist()


def test_lookup_continuation_and_match_length():
    r = recall.Record()
    a = _text(500, 1)
    assert r.add(a) == 500
    m = r.lookup(a[100:140])                        # the last 16 ids match, and 24 more before them
    assert m is not None and m[0] == 40
    assert r.continuation(m[1], 10).tolist() == a[140:150]
    assert r.continuation(m[1], 1000).tolist() == a[140:]          # stops at the end of the added text
    m = r.lookup([7, 7, 7] + a[200:216])            # only the window matches
    assert m[0] == 16 and r.continuation(m[1], 3).tolist() == a[216:219]
    assert r.lookup(_text(40, 2)) is None
    assert r.lookup(a[:10]) is None                 # shorter than a window


def test_dedup_budget_and_free_space(tmp_path):
    r = recall.Record()
    a = _text(2000, 3)
    assert r.add(a) == 2000
    assert r.add(a) == 0                            # the same text again adds nothing
    b = _text(300, 4)
    mixed = a[:1000] + b + a[1000:]
    stored = r.add(mixed)
    assert stored == 300 + 2 * recall.OVERLAP        # the new part and an overlap on each side of it
    m = r.lookup(mixed[1000 - 20:1000 + 30])        # a window across the old / new boundary is found
    assert m is not None and r.continuation(m[1], 5).tolist() == mixed[1030:1035]
    big = recall.Record(budget_ids=recall.CHUNK_IDS)
    for s in range(3):
        big.add(_text(700_000, 10 + s))
    assert big.stats()['ids'] <= recall.CHUNK_IDS + 700_001 and big.evicted > 0
    assert big.lookup(_text(700_000, 10)[:64]) is None      # the oldest text went first
    t3 = _text(700_000, 12)       # whole chunks go: only the tail of the newest text is left in the budget
    m = big.lookup(t3[-300:-200])
    assert m is not None and big.continuation(m[1], 4).tolist() == t3[-200:-196]
    full = recall.Record(tmp_path / 'full', min_free_gib=1e9)
    assert full.add(_text(100, 5)) == 0
    full.close()


def test_heat_eviction_keeps_landed_copies():
    """A segment whose copies the target accepted is promoted to the hot zone and outlives the FIFO eviction of its
    chunk; with FIFO eviction alone it goes with the chunk. A full hot zone drops its coldest entry."""
    a = _text(3000, 21)
    results = {}
    for mode in ('heat', 'fifo'):
        r = recall.Record(budget_ids=2 * recall.CHUNK_IDS, evict=mode, hot_frac=0.25, promote=8)
        r.add(a)
        m = r.lookup(a[1000:1040])
        assert m is not None and m[1] < recall.HOT_FLAG
        r.credit(m[1], 12)                               # 12 copied ids landed from segment m[1] // 256
        for s in range(4):                                # enough new text to evict a's chunk
            r.add(_text(700_000, 30 + s))
        assert r.evicted > 0
        results[mode] = (r.lookup(a[1030:1070]), r)   # inside the promoted stretch [1008, 1344)
    m, r = results['heat']
    assert m is not None and m[1] >= recall.HOT_FLAG and m[0] == 40
    assert r.continuation(m[1], 8).tolist() == a[1070:1078]
    st = r.stats()
    assert st['promoted'] == 1 and st['hot_entries'] == 1 and st['hot_ids'] <= r.hot_cap
    assert results['fifo'][0] is None and results['fifo'][1].stats()['hot_entries'] == 0
    # hot-zone capacity: promotions beyond it drop the coldest entries
    small = recall.Record(budget_ids=recall.CHUNK_IDS, hot_frac=0.0004, promote=4)   # room for one entry
    b = _text(5000, 40)
    small.add(b)
    for i, seg in enumerate((2, 6, 10)):
        small.credit(seg * recall.HEAT_SEG + 30, 5 + i)   # later segments hotter
    st = small.stats()
    assert st['promoted'] == 3 and st['hot_dropped'] == 2 and st['hot_entries'] == 1
    assert next(iter(small.hot.values())).seg == 10
    small.credit(2 * recall.HEAT_SEG + 30, 1)            # colder than the entry held: not promoted again
    assert small.stats()['promoted'] == 3


def test_engine_feedback_credits_the_record():
    r = recall.Record(promote=4)
    a = _text(600, 22)
    r.add(a)
    eng = recall.RecallEngine(r, gamma=8, min_n=0.0)
    eng.begin_stream(1, a[:300])
    p = eng.propose(1)
    assert p is not None and p.source == 'record' and p.ids == a[300:308] and p.pos >= 0
    eng.feedback(1, 6)
    assert r.stats()['heat_segments'] >= 1 and r.stats()['promoted'] == 1


def test_disk_record_persistence_identity_and_lock(tmp_path):
    d = tmp_path / 'rec'
    ident = {'tokenizer': 'T', 'vocab': 5000, 'digest': 'x'}
    r = recall.Record(d, identity=ident)
    a = _text(3000, 6)
    r.add(a)
    assert stat.S_IMODE(os.stat(d).st_mode) == 0o700
    files = list(d.glob('chunk-*.ids'))
    assert files and all(stat.S_IMODE(os.stat(f).st_mode) == 0o600 for f in files)
    ro = recall.Record(d, identity=ident)           # another opener: read-only while r holds the lock
    assert not ro.writer and ro.add(_text(100, 7)) == 0
    m = ro.lookup(a[1000:1050])
    assert m is not None and ro.continuation(m[1], 3).tolist() == a[1050:1053]
    b = _text(400, 8)
    r.add(b)
    assert ro.lookup(b[100:140]) is None
    assert ro.refresh() > 0 and ro.lookup(b[100:140]) is not None
    ro.close()
    r.close()
    again = recall.Record(d, identity=ident)        # reopened: the index is rebuilt from the chunk files
    assert again.writer and again.lookup(a[2000:2040])[0] == 40
    again.close()
    with pytest.raises(RuntimeError):
        recall.Record(d, identity={'tokenizer': 'other'})


def test_engine_own_context_cooldown_and_probes():
    eng = recall.RecallEngine(recall.Record(), gamma=8, min_n=1.0, cooldown=2, prior=0.5)
    period = _text(40, 9)
    eng.begin_stream('s', period * 2 + period[:20])            # the stream repeats itself
    p = eng.propose('s')
    assert p is not None and p.source == 'own' and p.ids == (period * 3)[60:68]
    eng.feedback('s', 8)
    assert eng.expect('own', p.tier) > 4
    eng.extend_stream('s', p.ids)
    p = eng.propose('s')
    assert p is not None and p.source == 'own'
    eng.feedback('s', 0)                                          # a miss: two rounds without copies
    assert eng.propose('s') is None and eng.propose('s') is None
    assert eng.propose('s') is not None
    eng.end_stream('s')
    assert eng.record.stats()['ids'] == 108 + 1                 # the stream's ids and a separator
    # a source whose expectation fell below the bar is only probed now and then
    low = recall.RecallEngine(recall.Record(), gamma=8, min_n=4.0, prior=0.1, probe_start=3)
    low.begin_stream('t', period * 3)
    got = [low.propose('t') for _ in range(6)]
    offered = [g for g in got if g is not None]
    assert len(offered) == 2 and all(g.probe for g in offered)


class Bigram:
    """A stand-in target: the logits of a position depend on its token only."""

    def __init__(self, V=64, seed=0):
        g = torch.Generator().manual_seed(seed)
        self.W = torch.randn(V, V, generator=g) * 4
        self.vocab = V
        self.device = torch.device('cpu')
        self.calls = 0

    def alloc_state(self, b, n):
        return {}

    def prefill(self, st, tokens, start=0, return_logits=False, all_logits=False, active=None):
        self.calls += 1
        lg = self.W[tokens.long()]
        nxt = torch.argmax(lg, -1)
        if all_logits:
            return nxt, lg
        return (nxt[-1:], lg[-1]) if return_logits else nxt[-1:]


def _greedy(target, prompt, n):
    seq = list(prompt)
    for _ in range(n):
        seq.append(int(torch.argmax(target.W[seq[-1]])))
    return seq[len(prompt):]


def test_speculative_with_copy_drafts_is_lossless():
    tgt = Bigram()
    prompt = torch.tensor(_text(20, 11, 64))
    want = _greedy(tgt, prompt.tolist(), 60)
    eng = recall.RecallEngine(recall.Record(), gamma=8, min_n=1.0)
    dec = SpeculativeDecoder(tgt, None, temperature=0.0, recall=eng)
    assert dec.generate(prompt, 60) == want                 # greedy: exactly the target's tokens
    first = dict(dec.stats)
    assert first['copy_landed'] > 0                          # a bigram's greedy path cycles: its own context copies
    # a second run of the same prompt copies from the record from the start
    tgt.calls = 0
    dec2 = SpeculativeDecoder(tgt, None, temperature=0.0, recall=eng)
    assert dec2.generate(prompt, 60) == want
    assert tgt.calls < 30 and dec2.stats['copy_landed'] > first['copy_landed']
    # sampling: the same seed gives the same tokens, every one a valid id
    s1 = SpeculativeDecoder(Bigram(), None, temperature=1.0, seed=3, recall=recall.RecallEngine(recall.Record()))
    s2 = SpeculativeDecoder(Bigram(), None, temperature=1.0, seed=3, recall=recall.RecallEngine(recall.Record()))
    a, b = s1.generate(prompt, 40), s2.generate(prompt, 40)
    assert a == b and all(0 <= t < 64 for t in a)
    with pytest.raises(ValueError):
        SpeculativeDecoder(tgt, None)


def _sync_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    mine = recall.Proposal('own', [5, 6, 7], 40, 1, False) if rank == 0 else None
    got = recall.sync_proposal(mine)
    none = recall.sync_proposal(None if rank == 0 else recall.Proposal('record', [1], 16, 0))
    q.put((rank, got, none))
    dist.destroy_process_group()


def test_proposal_broadcast_two_ranks():
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    ps = [ctx.Process(target=_sync_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=120) for _ in ps], key=lambda x: x[0])
    for p in ps:
        p.join(timeout=30)
    want = recall.Proposal('own', [5, 6, 7], 40, 1, False)
    assert res[0][1] == want and res[1][1] == want          # rank 1 takes rank 0's drafts
    assert res[0][2] is None and res[1][2] is None          # rank 0 had none: nobody copies


def test_reply_store_keys_disk_memory_and_cap(tmp_path):
    from xtier_b200.recall import replies
    p = _text(2000, 21)
    ks = replies.prompt_keys(p)
    assert len(ks) == 4 and len(set(ks)) == 4
    assert len(replies.prompt_keys(p[:100])) == 2                       # only the tails shorter than the prompt
    other_head = _text(50, 22) + p[50:]                                 # the same prompt with another head
    assert set(replies.prompt_keys(other_head)) & set(ks)
    reply = _text(300, 23)
    for path in (None, tmp_path / 'rs'):
        st = replies.ReplyStore(path)
        assert st.get(ks) is None
        assert not st.put(ks, reply[:replies.MIN_REPLY - 1])           # too short
        assert st.put(ks, reply)
        assert st.get(ks).tolist() == reply
        assert st.get(replies.prompt_keys(other_head)).tolist() == reply   # found through a tail key
        assert st.count() == 4
    # on disk: one reply file for the four keys, 0600 files, seen by another process's store, survives a restart
    files = sorted(f.name[:2] for f in (tmp_path / 'rs').iterdir())
    assert files.count('r-') == 1 and files.count('k-') == 4
    assert all(stat.S_IMODE(f.stat().st_mode) == 0o600 for f in (tmp_path / 'rs').iterdir())
    ro = replies.ReplyStore(tmp_path / 'rs', writer=False)
    assert ro.get(ks).tolist() == reply and not ro.put(ks, reply[::-1])
    # past the cap the oldest keys go, and their reply files with them
    st = replies.ReplyStore(tmp_path / 'cap', cap=16)
    for i in range(40):
        st.put([f'key{i}'], _text(20, 100 + i))
    st._trim()
    assert st.count() == 16 and st.get(['key39']) is not None and st.get(['key0']) is None
    assert sum(1 for _ in (tmp_path / 'cap').glob('r-*')) == 16
    mem = replies.ReplyStore(None, cap=8)
    for i in range(20):
        mem.put([f'k{i}'], _text(20, 200 + i))
    assert mem.count() == 8 and len(mem._replies) == 8 and mem.get(['k0']) is None


def test_reply_realign():
    from xtier_b200.recall import replies
    r = np.asarray([1, 2, 3, 4, 9, 9, 1, 2, 3, 4, 7, 7, 8], np.int64)
    assert replies.realign(r, [5, 1, 2, 3, 4], 4) == 4                 # nearest occurrence to the expected spot
    assert replies.realign(r, [5, 1, 2, 3, 4], 11) == 10
    assert replies.realign(r, [6, 6, 6, 6], 3) == -1
    assert replies.realign(r, [3], 3) == -1                            # shorter than the gram


def test_engine_drafts_a_filed_reply_and_realigns(tmp_path):
    rec = recall.Record(tmp_path / 'rec')
    eng = recall.RecallEngine(rec, gamma=8, min_n=1.0)
    prompt, reply = _text(200, 31), _text(120, 32)
    eng.begin_stream('a', prompt)
    assert eng.propose('a') is None
    eng.extend_stream('a', reply)
    eng.end_stream('a')
    assert (tmp_path / 'rec' / 'replies').is_dir()
    eng2 = recall.RecallEngine(recall.Record(tmp_path / 'rec2'), replies=eng.replies, gamma=8, min_n=1.0)
    eng2.begin_stream('b', prompt + reply[:1], reply_from=len(prompt))   # the first reply id already sampled
    p = eng2.propose('b')
    assert p.source == 'reply' and p.ids == reply[1:9] and p.tier == 2
    eng2.extend_stream('b', reply[1:4])
    eng2.feedback('b', 3)
    p = eng2.propose('b')
    assert p.source == 'reply' and p.ids == reply[4:12]
    # a divergence, then 4 ids of the reply again: the copy lines up after them
    eng2.extend_stream('b', [99999] + reply[60:64])
    eng2.feedback('b', 0)
    eng2.streams['b'].cooldown = 0
    p = eng2.propose('b')
    assert p.source == 'reply' and p.ids == reply[64:72] and p.tier == 0
    assert eng2.stats()['replies']['prompt_hits'] == 1 and eng2.realigns == 1
    off = recall.RecallEngine(recall.Record(), replies=None)
    off.begin_stream('c', prompt)
    assert off.stats()['replies'] is None


def test_speculative_second_run_copies_the_reply():
    """A sampled-free bigram target whose greedy path never cycles inside 40 tokens: the record has nothing to copy
    on the first run, and the second run of the same prompt copies the filed reply from its first token."""
    tgt = Bigram(V=4096, seed=5)
    prompt = torch.tensor(_text(24, 41, 4096))
    want = _greedy(tgt, prompt.tolist(), 40)
    eng = recall.RecallEngine(None, gamma=16, min_n=1.0)
    dec = SpeculativeDecoder(tgt, None, temperature=0.0, recall=eng)
    assert dec.generate(prompt, 40) == want
    dec.end()
    tgt.calls = 0
    dec2 = SpeculativeDecoder(tgt, None, temperature=0.0, recall=eng)
    assert dec2.generate(prompt, 40) == want
    assert eng.stats()['replies']['prompt_hits'] == 1
    assert tgt.calls <= 5 and dec2.stats['copy_landed'] >= 35
