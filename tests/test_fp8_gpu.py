"""FP8 kernels against plain PyTorch fp32 references: Engram-style FP8 rows with E8M0 block scales (gather by id with
a row range, and the decode of rows the graph lookup brought in), the W8A16 decode GEMV with per-row x 128-column
scales, the dequant + tcgen05 GEMM prefill path and the W8A8 (MXFP8) prefill path."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _e4m3_bytes(shape, gen):
    x = torch.randn(*shape, generator=gen) * 3.0
    return x.to(torch.float8_e4m3fn).view(torch.uint8)


def _rows_ref(tab, sc, blk):
    v = tab.view(torch.float8_e4m3fn).float()
    e = sc.int()
    s = torch.where(e == 0, torch.tensor(2.0 ** -127), torch.pow(2.0, (e - 127).float()))
    return (v * s.repeat_interleave(blk, dim=-1)).bfloat16()


@pytest.mark.parametrize('dim,blk', [(512, 128), (256, 32), (64, 16)])
def test_fp8_rows_gather_and_decode(cuda_ops, dim, blk):
    g = torch.Generator().manual_seed(dim + blk)
    R = 300
    tab = _e4m3_bytes((R, dim), g)
    sc = torch.randint(100, 140, (R, dim // blk), generator=g, dtype=torch.int64).to(torch.uint8)
    sc[0, 0] = 0                                           # E8M0 zero: 2^-127
    ref = _rows_ref(tab, sc, blk)
    lo, hi = 1000, 1000 + R
    ids = torch.tensor([1000, 1299, 5, 1100, 2000, 1000 + 17], dtype=torch.int64)
    out = torch.empty(len(ids), dim, dtype=torch.bfloat16, device='cuda')
    cuda_ops.fp8_rows(tab.cuda(), sc.cuda(), out, ids=ids.cuda(), block=blk, lo=lo, hi=hi)
    torch.cuda.synchronize()
    for i, idx in enumerate(ids.tolist()):
        want = ref[idx - lo] if lo <= idx < hi else torch.zeros(dim, dtype=torch.bfloat16)
        assert torch.equal(out[i].cpu(), want), idx
    dec = torch.empty(R, dim, dtype=torch.bfloat16, device='cuda')
    cuda_ops.fp8_rows(tab.cuda(), sc.cuda(), dec, block=blk)
    torch.cuda.synchronize()
    assert torch.equal(dec.cpu(), ref)


@pytest.mark.parametrize('m,N,K', [(1, 4096, 7168), (4, 1536, 2048), (16, 300, 1024)])
def test_gemv_fp8_vs_fp32(cuda_ops, m, N, K):
    g = torch.Generator().manual_seed(m * N)
    w = _e4m3_bytes((N, K), g)
    s = torch.rand(N, K // 128, generator=g) * 0.01 + 0.001
    x = torch.randn(m, K, generator=g).bfloat16()
    add = torch.randn(m, N, generator=g).bfloat16()
    wf = w.view(torch.float8_e4m3fn).float() * s.repeat_interleave(128, dim=1)
    ref = x.float() @ wf.T + add.float()
    out = torch.empty(m, N, dtype=torch.bfloat16, device='cuda')
    cuda_ops.gemv_fp8(x.cuda(), w.cuda(), s.cuda(), out, add=add.cuda())
    torch.cuda.synchronize()
    rel = float((out.cpu().float() - ref).norm() / ref.norm())
    assert rel < 5e-3, rel


def test_linear_fp8_prefill_path(cuda_ops):
    g = torch.Generator().manual_seed(3)
    N, K, m = 1024, 2048, 512
    w = _e4m3_bytes((N, K), g)
    s = torch.rand(N, K // 128, generator=g) * 0.01 + 0.001
    x = torch.randn(m, K, generator=g).bfloat16()
    wf = w.view(torch.float8_e4m3fn).float() * s.repeat_interleave(128, dim=1)
    deq = cuda_ops.fp8_dequant(w.cuda(), s.cuda())
    torch.cuda.synchronize()
    assert torch.equal(deq.cpu(), wf.bfloat16())
    out = cuda_ops.linear_fp8(x.cuda(), w.cuda(), s.cuda())
    torch.cuda.synchronize()
    ref = x.float() @ wf.bfloat16().float().T
    rel = float((out.cpu().float() - ref).norm() / ref.norm())
    assert rel < 1e-2, rel


def test_linear_fp8_w8a8_prefill(cuda_ops):
    """The W8A8 path: the FP8 weight requantized to MXFP8 once, activations quantized per call, block-scaled tcgen05
    GEMM; within E4M3 error of the fp32 product of the BF16 activations and the FP8 weight."""
    g = torch.Generator().manual_seed(4)
    N, K, m = 1024, 2048, 700
    w = _e4m3_bytes((N, K), g)
    s = torch.rand(N, K // 128, generator=g) * 0.01 + 0.001
    x = torch.randn(m, K, generator=g).bfloat16()
    wf = w.view(torch.float8_e4m3fn).float() * s.repeat_interleave(128, dim=1)
    mx8 = cuda_ops.fp8_weight_to_mx8(w.cuda(), s.cuda())
    out = cuda_ops.linear_fp8(x.cuda(), w.cuda(), s.cuda(), mx8=mx8)
    torch.cuda.synchronize()
    ref = x.float() @ wf.T
    rel = float((out.cpu().float() - ref).norm() / ref.norm())
    assert rel < 8e-2, rel


def test_graph_lookup_fp8_rows(cuda_ops, tmp_path):
    """Engram-shaped: FP8 rows and E8M0 scales on the drive, looked up inside a CUDA graph and decoded to BF16."""
    from xtier_b200.tables import RowStore, write_table
    from xtier_b200.tables.lookup import GraphLookup
    g = torch.Generator().manual_seed(9)
    R, dim, blk = 3000, 512, 128
    tab = _e4m3_bytes((R, dim), g)
    sc = torch.randint(110, 135, (R, dim // blk), generator=g, dtype=torch.int64).to(torch.uint8)
    segs = write_table(tmp_path / 'engram', tab.numpy(), sc.numpy(), segments=2)
    st = RowStore(segs, dim, dim // blk, io_threads=2, cache_rows=64)
    gl = GraphLookup(st, 32, fp8_block=blk)
    ids = torch.zeros(32, dtype=torch.int64, device='cuda')
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        gl.fetch(ids)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        rows = gl.fetch(ids)
    ref = _rows_ref(tab, sc, blk)
    for seed in range(2):
        want = np.random.default_rng(seed).integers(0, R, size=32)
        ids.copy_(torch.from_numpy(want))
        graph.replay()
        torch.cuda.synchronize()
        gl.check()
        assert torch.equal(rows.cpu(), ref[torch.from_numpy(want)])
    del graph
    st.close()
