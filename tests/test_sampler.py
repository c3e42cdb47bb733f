"""Vocabulary-parallel token choice on 2 CPU ranks (gloo): the global argmax equals torch.argmax of the full row
(ties to the lowest id), the Gumbel-max sample is identical on every rank and distributed as softmax(logits / T), and
the token-id sync broadcasts rank 0's ids."""
import os
import socket

import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from xtier_b200.parallel.sampler import sync_token_ids, vocab_parallel_argmax, vocab_parallel_sample
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    g = torch.Generator().manual_seed(0)
    full = torch.randn(6, 40, generator=g)
    full[2, 5] = full[2, 31] = 100.0                       # a tie across the two ranks' slices: lowest id wins
    V = 40 // world
    local = full[:, rank * V:(rank + 1) * V]
    top = vocab_parallel_argmax(local, rank * V)
    ok_argmax = torch.equal(top, torch.argmax(full, -1))
    logits = torch.tensor([[1.0, 0.0, -1.0, 0.5] * 5])     # one row, 20 ids
    Vl = 20 // world
    counts = torch.zeros(20)
    draws = []
    for step in range(3000):
        t = vocab_parallel_sample(logits[:, rank * Vl:(rank + 1) * Vl], rank * Vl, 0.7, seed=5, step=step)
        counts[int(t)] += 1
        draws.append(int(t))
    ids = torch.tensor([rank * 10 + 1, rank * 10 + 2])
    sync_token_ids(ids)
    q.put((rank, ok_argmax, counts, draws, ids.tolist()))
    dist.destroy_process_group()


def test_vocab_parallel_sampling_two_ranks():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=120) for _ in ps])
    for p in ps:
        p.join(timeout=30)
    (_, ok0, c0, d0, ids0), (_, ok1, c1, d1, ids1) = res
    assert ok0 and ok1
    assert d0 == d1                                         # every rank draws the same token
    p = torch.softmax(torch.tensor([1.0, 0.0, -1.0, 0.5] * 5) / 0.7, -1)
    assert float((c0 / c0.sum() - p).abs().max()) < 0.02
    assert ids0 == ids1 == [1, 2]
