"""Cold experts on drives: record layout against the engine's slots, manifest reuse and CRC checks, an engine whose
misses come from the store (per-expert global scales follow the expert into its slot), start-up fill from the store,
relayout to other drives / weights / node counts, and punching the checkpoint's copy (compare, marker, restore)."""
import json
import os

import numpy as np
import pytest
import torch

from xtier_b200 import checkpoint, formats
from xtier_b200.cache import cold
from xtier_b200.engine import CpuEngine

H, I, E = 256, 128, 8


def _experts(fmt=formats.NVFP4, seed=0):
    ew = formats.random_experts(E, H, I, fmt, seed=seed)
    # distinct global scales per expert, so a slot holding the wrong expert's scales shows up
    ew.g13 = (torch.rand(E, 2, generator=torch.Generator().manual_seed(seed)) + 0.5) * ew.g13.float()
    ew.g2 = (torch.rand(E, generator=torch.Generator().manual_seed(seed + 1)) + 0.5) * ew.g2.float()
    return ew


def _routes(m, k, seed):
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(m)]).int()
    w = torch.rand(m, k, generator=g)
    x = torch.randn(m, H, generator=g).bfloat16()
    return x, ids, w


@pytest.mark.parametrize('fmt', [formats.NVFP4, formats.MXFP4])
def test_record_layout_matches_engine_slots(fmt):
    ew = _experts(fmt)
    eng = CpuEngine(ew, threads=2)
    N = eng.nodes()
    sizes = [eng.slot_pieces(0, n)[1] for n in range(N)]
    for n in range(N):
        assert sizes[n] == cold.piece_bytes(H, I, fmt, N)
        ptrs, sz = eng.slot_pieces(3, n)
        pieces = cold.shard_pieces(ew, 3, n, N)
        for p, q, b in zip(ptrs, pieces, sz):   # the engine slot holds exactly these bytes
            got = np.ctypeslib.as_array((np.ctypeslib.ctypes.c_uint8 * b).from_address(p))
            assert np.array_equal(got, q)
    eng.close()


def test_manifest_reuse_crc_and_source(tmp_path):
    ew = _experts()
    d = tmp_path / 'd0'
    pool = cold.ColdPool([d])
    src = [['layer0.safetensors', 123, 456]]
    assert pool.ensure_layer(0, ew, 1, src) is False        # written
    assert pool.ensure_layer(0, ew, 1, src) is True         # reused
    pool.close()
    pool = cold.ColdPool([d])                                # restart: the manifest is read back
    assert pool.layer_ok(0, H, I, ew.fmt, 1, E, src)
    assert not pool.layer_ok(0, H, I, ew.fmt, 1, E, [['layer0.safetensors', 123, 999]])   # source changed
    # corrupt the last 4 KiB of record 5
    ent = pool.entry(0)
    dr, off = ent['loc'][5]
    with open(pool.files[dr], 'r+b') as f:
        f.seek(off + ent['record'] - 10)
        f.write(b'\xff' * 4)
    assert pool.check_layer(0) == [5]
    assert pool.ensure_layer(0, ew, 1, src) is False        # rewritten
    assert pool.check_layer(0) == []
    back = pool.load_layer(0)
    for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):
        assert torch.equal(getattr(back, f), getattr(ew, f).float() if f in ('g13', 'g2') else getattr(ew, f)), f
    pool.close()


@pytest.mark.parametrize('fmt', [formats.NVFP4, formats.MXFP4])
def test_engine_reads_misses_from_the_store(tmp_path, fmt):
    ew = _experts(fmt, seed=4)
    full = CpuEngine(ew, threads=2)
    pool = cold.ColdPool([tmp_path / 'a', tmp_path / 'b'], parts='3:1')
    eng = cold.cold_engine(0, ew, pool, 0.5, popularity=torch.arange(E, 0, -1).float(), gpu_hot=[0], threads=2)
    assert eng.shape()['slots'] == E // 2
    drives = [dd for dd, _ in pool.entry(0)['loc']]
    assert drives.count(0) == 3 * drives.count(1)            # dealt 3:1
    for i in range(6):                                        # different expert sets: misses and evictions
        x, ids, w = _routes(1, 4, seed=10 + i)
        assert torch.equal(eng.forward(x, ids, w), full.forward(x, ids, w)), i
    for i in range(3):     # more distinct experts than RAM slots: batches of experts, summed in batch order
        x, ids, w = _routes(4, 4, seed=20 + i)
        want = full.forward(x, ids, w)
        got = eng.forward(x, ids, w)
        assert torch.allclose(got, want, rtol=1e-5, atol=1e-6), i
        ref = formats.reference_moe(x, ids, w, ew)
        assert torch.allclose(got, ref, rtol=2e-2, atol=2e-3)
    st = eng.cold_stats()
    assert st['reads'] > 0 and pool.stats()['bytes_read'] > 0
    eng.close()
    full.close()
    pool.close()


def test_three_unit_records_dealt_by_bytes(tmp_path):
    """Records cut into gate / up / rest units: each unit is dealt to a drive on its own, the engine reads the pieces
    of one record from several drives, and start-up fill, CRC checks and relayout work per unit."""
    from xtier_b200.tools.cold_relayout import relayout
    ew = _experts(formats.NVFP4, seed=9)
    full = CpuEngine(ew, threads=2)
    N = full.nodes()
    dirs = [tmp_path / 'a', tmp_path / 'b', tmp_path / 'c']
    pool = cold.ColdPool(dirs, units=3)
    pool.write_layer(0, ew, N)
    ent = pool.entry(0)
    assert ent['units'] == 3 and len(ent['loc']) == E * N * 3
    assert sum(ent['unit_bytes']) == ent['record']
    per_drive = [0, 0, 0]
    for i, (d, _) in enumerate(ent['loc']):
        per_drive[d] += ent['unit_bytes'][i % 3]
    assert max(per_drive) - min(per_drive) <= max(ent['unit_bytes'])          # bytes dealt evenly
    assert any(len({ent['loc'][r * 3 + u][0] for u in range(3)}) > 1 for r in range(E * N))   # records span drives
    assert pool.layer_ok(0, H, I, ew.fmt, N, E)
    assert not cold.ColdPool(dirs, units=1).layer_ok(0, H, I, ew.fmt, N, E)   # another unit count: rewrite
    back = pool.load_layer(0)
    assert torch.equal(back.w13, ew.w13) and torch.equal(back.s13, ew.s13) and torch.equal(back.w2, ew.w2)
    assert torch.equal(back.s2, ew.s2)
    # a bad unit is reported by its own index
    d, off = ent['loc'][7]
    with open(pool.files[d], 'r+b') as f:
        f.seek(off + 3)
        f.write(b'\x5a' * 2)
    assert pool.check_layer(0) == [7]
    pool.write_layer(0, ew, N)
    assert pool.check_layer(0) == []
    # misses come from three drives; start-up fill reads per piece
    eng = CpuEngine(ew, threads=2, slots=4, fill=False)
    pool.fill_engine(eng, 0, [1, 4, -1, -1])
    pool.attach(eng, 0)
    for i in range(4):
        x, ids, w = _routes(1, 3, seed=30 + i)
        assert torch.equal(eng.forward(x, ids, w), full.forward(x, ids, w)), i
    assert eng.cold_stats()['reads'] > 0
    eng.close()
    full.close()
    pool.close()
    # relayout back to whole-shard records on one drive, and to 3 units again
    rep = relayout(','.join(map(str, dirs)), str(tmp_path / 'one'), units=1, log=lambda s: None)
    assert rep[0]['units'] == E * N
    rep = relayout(str(tmp_path / 'one'), str(tmp_path / 'three'), units=3, log=lambda s: None)
    assert rep[0]['units'] == E * N * 3
    p3 = cold.ColdPool(tmp_path / 'three', units=3)
    assert torch.equal(p3.load_layer(0).w13, ew.w13)
    p3.close()


def _offset_stage(n, fmt, shift):
    """Host staging tensors whose rows start `shift` bytes past a 4 KiB boundary (exercises the bounce reads)."""
    bs = 16 if fmt == formats.NVFP4 else 32
    shapes = [(n, 2 * I, H // 2), (n, H, I // 2), (n, 2 * I, H // bs), (n, H, I // bs)]
    out = []
    for sh in shapes:
        raw = cold._aligned(int(np.prod(sh)) + 8192)
        out.append(torch.from_numpy(raw[shift:shift + int(np.prod(sh))]).view(sh))
    return formats.ExpertWeights(fmt, *out, torch.empty(n, 2), torch.empty(n))


@pytest.mark.parametrize('units', [1, 3])
def test_cold_prefill_staging_from_ram_and_drives(tmp_path, units):
    """The GPU prefill's host staging of a cold-backed layer: experts in the engine's RAM slots are copied from the
    slots, the others read from the drives; bytes and global scales equal the layer's; a threaded fill waits for the
    previous upload out of the same buffer."""
    ew = _experts(formats.NVFP4, seed=11)
    pool = cold.ColdPool([tmp_path / 'a', tmp_path / 'b'], units=units)
    gpu_hot = [0, 5]
    eng = cold.cold_engine(2, ew, pool, 0.5, popularity=torch.arange(E, 0, -1).float(), gpu_hot=gpu_hot, threads=2)
    non_gpu = [e for e in range(E) if e not in gpu_hot]
    cp = cold.ColdPrefill(pool, 2, eng, non_gpu)
    want = ew.select(torch.tensor(non_gpu))
    st = cp.stage()                                        # no read-ahead started: fills now
    for f in ('w13', 'w2', 's13', 's2'):
        assert torch.equal(getattr(st, f), getattr(want, f)), f
    assert torch.equal(st.g13, want.g13.float()) and torch.equal(st.g2, want.g2.float())
    assert cp.stats['from_ram'] > 0 and cp.stats['from_drive'] > 0
    assert cp.stats['from_ram'] + cp.stats['from_drive'] == len(non_gpu)

    class Ev:          # the upload out of the buffer: the next fill of the same parity must wait for it
        done = False

        def synchronize(self):
            Ev.done = True
    cp.uploaded(Ev())
    st.w13.zero_()
    cp.start()
    st = cp.stage()
    assert Ev.done and torch.equal(st.w13, want.w13)
    # unaligned destinations go through bounce buffers; a subset in any order
    sub = [non_gpu[3], non_gpu[0]]
    st2 = _offset_stage(2, formats.NVFP4, 64)
    cp.fill(st2, sub)
    got = cp.read_experts(sub)
    ref = ew.select(torch.tensor(sub))
    for f in ('w13', 'w2', 's13', 's2'):
        assert torch.equal(getattr(st2, f), getattr(ref, f)) and torch.equal(getattr(got, f), getattr(ref, f)), f
    eng.close()
    pool.close()


def test_cold_mode_swap_sources_the_store(tmp_path):
    """A GPU-slot swap in cold mode (no host copy of the layer): the incoming expert comes from the engine or the
    drives, and the victim takes the incoming expert's place in the prefill staging."""
    from xtier_b200.cache.pool import TieredMoE
    ew = _experts(formats.NVFP4, seed=12)
    pool = cold.ColdPool([tmp_path / 'a'])
    hot = [1, 2]
    eng = cold.cold_engine(0, ew, pool, 0.5, popularity=torch.arange(E, 0, -1).float(), gpu_hot=hot, threads=2)
    router = torch.randn(E, H)
    moe = TieredMoE(0, router, ew, 2, hot=hot, engine=eng, device='cpu', host_experts=None)
    assert not moe.can_refill
    moe.attach_cold_prefill(cold.ColdPrefill(pool, 0, eng, [e for e in range(E) if e not in hot]))
    assert moe.can_refill
    incoming, victim = 6, 2
    idx = int(moe._cold_index[incoming])
    moe.swap(incoming, victim)
    slot = int(moe.table_host[incoming])
    assert slot == 1 and int(moe.table_host[victim]) == -1
    for f in ('w13', 'w2', 's13', 's2'):
        assert torch.equal(getattr(moe.pool, f)[slot], getattr(ew, f)[incoming]), f
    assert float(moe.pool.g2[slot]) == float(ew.g2[incoming])
    assert int(moe._cold_index[victim]) == idx and int(moe._cold_index[incoming]) == -1
    st = moe.cold_prefill.stage()
    assert torch.equal(st.w13[idx], ew.w13[victim])
    eng.close()
    pool.close()


def test_fill_engine_from_store(tmp_path):
    ew = _experts(seed=7)
    pool = cold.ColdPool([tmp_path / 'a'])
    eng0 = CpuEngine(ew, threads=2)
    N = eng0.nodes()
    pool.write_layer(3, ew, N)
    resident = [6, 2, 5, -1]
    eng = CpuEngine(ew, threads=2, slots=4, fill=False)      # no expert bytes from the checkpoint
    pool.fill_engine(eng, 3, resident)
    pool.attach(eng, 3)
    assert list(eng.slot_table()[[6, 2, 5]]) == [0, 1, 2]
    x, ids, w = _routes(2, 3, seed=1)
    assert torch.equal(eng.forward(x, ids, w), eng0.forward(x, ids, w))
    eng.close()
    eng0.close()
    pool.close()


def test_relayout_to_other_drives_and_nodes(tmp_path):
    from xtier_b200.tools.cold_relayout import relayout
    ew = _experts(formats.MXFP4, seed=2)
    src = cold.ColdPool([tmp_path / 's'])
    src.write_layer(0, ew, 1, [['f', 1, 2]])
    src.write_layer(1, _experts(formats.MXFP4, seed=3), 1)
    src.close()
    dst_dirs = f'{tmp_path / "x"},{tmp_path / "y"}'
    rep = relayout(str(tmp_path / 's'), dst_dirs, parts='1:1', nodes=2, log=lambda s: None)
    assert sorted(rep) == [0, 1]
    dst = cold.ColdPool(dst_dirs)
    assert dst.entry(0)['shape'][3] == 2 and dst.entry(0)['source'] == [['f', 1, 2]]
    back = dst.load_layer(0)
    assert torch.equal(back.w13, ew.w13) and torch.equal(back.s2, ew.s2) and torch.equal(back.g2, ew.g2.float())
    dst.close()
    with pytest.raises(SystemExit):        # a store onto itself is refused
        relayout(str(tmp_path / 's'), str(tmp_path / 's'), log=lambda s: None)


def test_punch_compare_marker_restore(tmp_path):
    from xtier_b200.tools import cold_punch
    ew = _experts(seed=9)
    ck = tmp_path / 'model'
    ck.mkdir()
    path = ck / 'layer0.safetensors'
    checkpoint.save_experts(path, ew)
    original = path.read_bytes()
    mtime = os.stat(path).st_mtime_ns
    pool = cold.ColdPool([tmp_path / 'c'])
    got = cold.open_layer(pool, 0, path, nodes=1)
    assert torch.equal(got.w13, ew.w13)
    assert cold_punch.compare(pool, pool.ranges()) == []
    try:
        cold_punch.punch(pool, pool.ranges(), log=lambda s: None)
    except OSError as e:        # a filesystem without hole punching
        pytest.skip(f'fallocate punch unsupported here: {e}')
    assert (ck / checkpoint.MARKER).exists() and os.stat(path).st_mtime_ns == mtime
    assert path.stat().st_size == len(original)
    with pytest.raises(RuntimeError):
        checkpoint.load_experts(path)
    ranges = json.loads(pool.ranges_path.read_text())['0']['tensors']
    data = path.read_bytes()
    off, stride = ranges['w13']
    lo = (off + 4095) // 4096 * 4096
    assert data[lo:lo + 4096] == bytes(4096)                 # the tensor's inner blocks are gone
    assert data[:off] == original[:off]                      # the header and what precedes are untouched
    rebuilt = cold.open_layer(pool, 0, path, nodes=1)        # from the store alone
    assert torch.equal(rebuilt.w2, ew.w2)
    cold_punch.restore(pool, pool.ranges(), log=lambda s: None)
    assert path.read_bytes() == original and not (ck / checkpoint.MARKER).exists()
    assert os.stat(path).st_mtime_ns == mtime
    pool.close()
