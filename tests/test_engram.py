"""Hashed bigram rows: the device hash against a Python-integer oracle, and the prefill lookup against the table."""
import numpy as np
import torch

from xtier_b200.tables import RowStore, write_table
from xtier_b200.tables.engram import BigramTable, bigram_rows, bigram_rows_reference


def test_hash_matches_oracle_and_spreads():
    g = torch.Generator().manual_seed(0)
    p = torch.randint(0, 2 ** 31 - 1, (4000,), generator=g)
    c = torch.randint(0, 2 ** 31 - 1, (4000,), generator=g)
    for rows, seed in ((4_000_000, 0), (1000, 12345)):
        a = bigram_rows(p, c, rows, seed).numpy()
        assert np.array_equal(a, bigram_rows_reference(p.numpy(), c.numpy(), rows, seed))
        assert a.min() >= 0 and a.max() < rows
    counts = np.bincount(bigram_rows(p, c, 64).numpy(), minlength=64)
    assert counts.min() > 30 and counts.max() < 100          # 4000 keys over 64 rows: about 62 each


def test_prefill_rows_from_the_table(tmp_path):
    rows, dim = 3000, 64
    data = (np.random.default_rng(1).standard_normal((rows, dim)) * 0.02).astype(np.float32)
    bf = torch.from_numpy(data).bfloat16()
    segs = write_table(tmp_path / 'bigram', bf.view(torch.uint8).numpy().reshape(rows, dim * 2), None, segments=2)
    store = RowStore(segs, dim * 2, 0, io_threads=2, cache_rows=64)
    t = BigramTable.__new__(BigramTable)          # host-side parts only (no GPU lookup object)
    t.store, t.rows, t.dim, t.hidden, t.seed, t.proj = store, rows, dim, dim, 5, None
    tokens = torch.tensor([11, 22, 33, 44])
    prev = torch.tensor([0, 11, 22, 33])
    got = t.rows_host(prev, tokens)
    ids = bigram_rows_reference(prev.numpy(), tokens.numpy(), rows, 5)
    assert torch.equal(got, bf[torch.from_numpy(ids)])
    x = torch.zeros(4, dim, dtype=torch.bfloat16)
    t.add_prefill(x, tokens)
    assert torch.equal(x, bf[torch.from_numpy(ids)])
    store.close()


def test_chunk_look_ahead_rows_match_direct_lookup(tmp_path):
    """prefetch_rows (a chunked prefill's read-ahead of the next chunk) gives the rows add_prefill would read."""
    from xtier_b200.tables.engram import BigramTable
    rows, dim = 4096, 64
    bf = (torch.arange(rows * dim, dtype=torch.float32).reshape(rows, dim) % 251 / 251.0).bfloat16()
    segs = write_table(tmp_path / 'bigram', bf.view(torch.uint8).numpy().reshape(rows, dim * 2), None, segments=2)
    store = RowStore(segs, dim * 2, 0, io_threads=2, cache_rows=64)
    bt = BigramTable.__new__(BigramTable)
    bt.store, bt.rows, bt.dim, bt.hidden, bt.seed, bt.proj = store, rows, dim, dim, 0, None
    toks = torch.randint(0, 1000, (300,), generator=torch.Generator().manual_seed(1))
    fut = bt.prefetch_rows(toks[100:], int(toks[99]))
    direct = bt.rows_host(toks[99:-1], toks[100:])
    assert torch.equal(fut.result(), direct)
    x = torch.zeros(200, dim, dtype=torch.bfloat16)
    bt.add_prefill(x, toks[100:], prev0=int(toks[99]), rows=fut.result())
    assert torch.equal(x, direct)
    store.close()
