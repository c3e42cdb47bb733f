"""NVMe row tables on the CPU: every segment boundary byte for byte against the source array, cache hits, TP range,
RAM mode, and a bad id failing the lookup."""
import numpy as np
import pytest

from xtier_b200.tables import RowStore, write_table


@pytest.fixture()
def table(tmp_path):
    rng = np.random.default_rng(0)
    data = rng.integers(0, 256, size=(1000, 96), dtype=np.uint8)   # 96-byte rows straddle 4 KiB pages
    scales = rng.integers(0, 256, size=(1000, 3), dtype=np.uint8)
    segs = write_table(tmp_path / 'tab', data, scales, segments=3)
    return data, scales, segs


@pytest.mark.parametrize('mode', ['direct', 'ram'])
def test_lookup_every_boundary(table, mode):
    data, scales, segs = table
    st = RowStore(segs, 96, 3, io_threads=4, cache_rows=64, mode=mode)
    edges = sorted({0, 999} | {s.first for s in segs} | {s.first + s.count - 1 for s in segs} |
                   {s.first + 1 for s in segs})
    ids = np.array(edges + list(range(0, 1000, 37)) + [5, 5, 5], dtype=np.int64)
    rows, sc = st.lookup(ids)
    assert np.array_equal(rows, data[ids])
    assert np.array_equal(sc, scales[ids])
    rows2, _ = st.lookup(ids)   # second time from the cache (direct mode)
    assert np.array_equal(rows2, data[ids])
    if mode == 'direct':
        assert st.stats()['hits'] > 0
    st.close()


def test_tp_range_and_bad_id(table):
    data, scales, segs = table
    st = RowStore(segs, 96, 3, io_threads=2, cache_rows=0)
    st.set_range(100, 200)
    rows, _ = st.lookup(np.array([50, 150, 250]))
    assert not rows[0].any() and not rows[2].any()
    assert np.array_equal(rows[1], data[150])
    with pytest.raises(IndexError, match='outside'):
        st.lookup(np.array([1000]))
    st.close()


def test_host_function_callback(table):
    """The graph lookup's host node, called directly: rows for the context's ids, error word on a bad id."""
    import ctypes as C
    from xtier_b200.tables import lib
    from xtier_b200.tables.lookup import _Ctx
    data, scales, segs = table
    st = RowStore(segs, 96, 3, io_threads=2, cache_rows=16)
    ids = np.array([3, 999, 400, 3], dtype=np.int64)
    rows = np.zeros((4, 96), dtype=np.uint8)
    sc = np.zeros((4, 3), dtype=np.uint8)
    ctx = _Ctx(st.handle, ids.ctypes.data, 4, rows.ctypes.data, sc.ctypes.data, 0)
    fn = C.CFUNCTYPE(None, C.c_void_p)(C.cast(lib().xt_rows_host_fn, C.c_void_p).value)
    fn(C.addressof(ctx))
    assert ctx.error == 0 and np.array_equal(rows, data[ids]) and np.array_equal(sc, scales[ids])
    ids[1] = 5000
    fn(C.addressof(ctx))
    assert ctx.error == 1
    st.close()
