"""Row-table lookups captured in a CUDA graph (device->host ids, host-function node with the C++ lookup, host->device
rows), replayed with new ids written into the same device tensor between replays."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_graph_lookup_replays(cuda_ops, tmp_path):
    from xtier_b200.tables import RowStore, write_table
    from xtier_b200.tables.lookup import GraphLookup
    rng = np.random.default_rng(1)
    data = rng.integers(0, 256, size=(5000, 256), dtype=np.uint8)
    segs = write_table(tmp_path / 'rows', data, None, segments=2)
    st = RowStore(segs, 256, 0, io_threads=2, cache_rows=128)
    gl = GraphLookup(st, 64)
    ids = torch.zeros(64, dtype=torch.int64, device='cuda')
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        gl.fetch(ids)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        rows = gl.fetch(ids)
    for seed in range(3):
        want = np.random.default_rng(seed).integers(0, 5000, size=64)
        ids.copy_(torch.from_numpy(want))
        g.replay()
        torch.cuda.synchronize()
        gl.check()
        assert np.array_equal(rows.cpu().numpy(), data[want])
    del g
    st.close()
