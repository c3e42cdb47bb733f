"""DSA selection on the GPU against fp32 PyTorch: FP8 index-key cache round trip, indexer scores (ReLU head sum over
64 heads, per-query lengths), top-k sets and their ascending order (with -1 padding on short rows), and the whole
sparse decode chain (indexer -> top-k -> MLA over the selected latent rows)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_index_scores_and_topk(cuda_ops):
    from xtier_b200.attention import dsa
    g = torch.Generator(device='cuda').manual_seed(3)
    rows, max_len = 3, 3000
    cache = dsa.IndexCache(rows, max_len)
    k = torch.randn(rows * max_len, 128, device='cuda', generator=g).bfloat16()
    cache.write(k, torch.arange(rows * max_len, device='cuda'))
    back = cache.dequant(torch.arange(rows * max_len, device='cuda'))
    assert float((back - k.float()).norm() / k.float().norm()) < 0.05   # E4M3: 3 mantissa bits
    Q = 4
    q = torch.randn(Q, 64, 128, device='cuda', generator=g).bfloat16()
    w = torch.rand(Q, 64, device='cuda', generator=g)
    qrows = torch.tensor([0, 1, 2, 1], device='cuda')
    lens = torch.tensor([3000, 1500, 700, 2999], device='cuda', dtype=torch.int32)
    ref = dsa.reference_scores(q, w, cache, qrows, lens)
    fin = torch.isfinite(ref)
    sc_cc = dsa.index_scores(q, w, cache, qrows, lens, tensor_cores=False)       # CUDA cores, BF16 queries
    assert torch.equal(fin, torch.isfinite(sc_cc))
    assert float((sc_cc[fin] - ref[fin]).abs().max() / ref[fin].abs().max()) < 1e-3
    err = torch.zeros(1, dtype=torch.int32, device='cuda')
    sc = dsa.index_scores(q, w, cache, qrows, lens, err=err)                      # tcgen05, FP8 queries
    ref8 = dsa.reference_scores(q, w, cache, qrows, lens, fp8_queries=True)
    assert int(err) == 0 and torch.equal(fin, torch.isfinite(sc))
    assert float((sc[fin] - ref8[fin]).abs().max() / ref8[fin].abs().max()) < 1e-3
    # two queries of one cache row per CTA (prefill layout)
    q2rows = torch.tensor([1, 1, 2, 2], device='cuda')
    lens2 = torch.tensor([1500, 900, 700, 3000], device='cuda', dtype=torch.int32)
    sc2 = dsa.index_scores(q, w, cache, q2rows, lens2, err=err, per_cta=2)
    ref2 = dsa.reference_scores(q, w, cache, q2rows, lens2, fp8_queries=True)
    fin2 = torch.isfinite(ref2)
    assert int(err) == 0 and torch.equal(fin2, torch.isfinite(sc2))
    assert float((sc2[fin2] - ref2[fin2]).abs().max() / ref2[fin2].abs().max()) < 1e-3
    K = 1024
    idx = dsa.topk(sc, K)
    want = dsa.reference_topk(sc, K)
    for r in range(Q):
        row = idx[r].tolist()
        got = [i for i in row if i >= 0]
        assert got == sorted(got)                       # ascending
        assert set(got) == want[r], r
        assert all(i == -1 for i in row[len(got):])     # padding at the end only
    assert (idx[2] >= 0).sum() == 700                  # short row: every finite score, then -1


@pytest.mark.parametrize('Q,splits', [(6, 1), (9, 3), (64, 0)])
def test_prefill_indexer_and_length_topk(cuda_ops, Q, splits):
    """Pipelined prefill indexer (4 queries per CTA, key splits, a partial last group) against the FP8-query oracle
    over each query's causal length, and top-k that reads each row only up to its length."""
    from xtier_b200.attention import dsa
    g = torch.Generator(device='cuda').manual_seed(11 + Q)
    rows, max_len = 2, 5000
    cache = dsa.IndexCache(rows, max_len)
    cache.write(torch.randn(rows * max_len, 128, device='cuda', generator=g).bfloat16(),
                torch.arange(rows * max_len, device='cuda'))
    q = torch.randn(Q, 64, 128, device='cuda', generator=g).bfloat16()
    w = torch.rand(Q, 64, device='cuda', generator=g)
    lens = torch.randint(1, max_len + 1, (Q,), device='cuda', generator=g).int()
    lens[0] = max_len
    err = torch.zeros(1, dtype=torch.int32, device='cuda')
    out = torch.full((Q, max_len), float('nan'), device='cuda')
    sc = dsa.index_scores_prefill(q, w, cache, 1, lens, out=out, err=err, splits=splits)
    ref = dsa.reference_scores(q, w, cache, torch.ones(Q, dtype=torch.long, device='cuda'), lens, fp8_queries=True)
    assert int(err) == 0
    for i in range(Q):
        n = int(lens[i])
        assert float((sc[i, :n] - ref[i, :n]).abs().max() / ref[i, :n].abs().max()) < 1e-3, i
        end = min(max_len, (n + 127) // 128 * 128)
        assert bool(torch.isneginf(sc[i, n:end]).all()), i
    K = 2048
    idx = dsa.topk(sc, K, lengths=lens)
    masked = sc.clone()
    for i in range(Q):
        masked[i, int(lens[i]):] = float('-inf')
    want = dsa.reference_topk(masked, K)
    for i in range(Q):
        row = idx[i].tolist()
        got = [j for j in row if j >= 0]
        assert got == sorted(got) and set(got) == want[i], i
        assert len(got) == min(K, int(lens[i])), i
        assert all(j == -1 for j in row[len(got):]), i


def test_sparse_decode_chain(cuda_ops):
    from xtier_b200.attention import dsa
    from xtier_b200.attention.mla import LatentCache, MlaWorkspace, default_scale, mla_decode, reference_decode
    g = torch.Generator(device='cuda').manual_seed(5)
    rows, max_len, K = 2, 4096, 2048
    icache, lcache = dsa.IndexCache(rows, max_len), LatentCache(rows, max_len)
    n = rows * max_len
    icache.write(torch.randn(n, 128, device='cuda', generator=g).bfloat16(), torch.arange(n, device='cuda'))
    lcache.write(torch.randn(n, 576, device='cuda', generator=g).bfloat16(), torch.arange(n, device='cuda'))
    qrows = torch.tensor([0, 1], device='cuda')
    lens = torch.tensor([4000, 1800], device='cuda', dtype=torch.int32)
    sc = dsa.index_scores(torch.randn(2, 64, 128, device='cuda', generator=g).bfloat16(),
                          torch.rand(2, 64, device='cuda', generator=g), icache, qrows, lens)
    slots = dsa.select_slots(sc, qrows, K, max_len)
    assert int((slots[1] >= 0).sum()) == 1800
    q = (torch.randn(2, 128, 576, device='cuda', generator=g) * 0.5).bfloat16()
    ws = MlaWorkspace(2, K)
    out = mla_decode(q, slots, lcache, ws, default_scale())
    ref = reference_decode(q, slots, lcache, default_scale())
    assert float((out.float() - ref).norm() / ref.norm()) < 2e-2
