"""PCIe staging on the CPU: the engine mapping declines (no half-registered state) when CUDA refuses the registration
or when the engine's shards do not split rows evenly, and the model sizes its staging slots from the share of the
CPU-tier experts a call is expected to touch."""
import logging
import math

import torch

from xtier_b200 import formats
from xtier_b200.parallel import ep


class _Engine:
    def __init__(self, H=256, I=128, nodes=1, fmt=formats.NVFP4, bad=False):
        self.H, self.I, self.fmt, self._nodes, self.bad = H, I, fmt, nodes, bad

    def nodes(self):
        return self._nodes

    def shard(self, node):
        N, H, I = self._nodes, self.H, self.I
        sizes = [I // N * (H // 2)] * 2 + [I // N * (H // 16)] * 2 + [H // N * (I // 2), H // N * (I // 16)]
        if self.bad:
            sizes[0] += 16
        offs, o = [], 0
        for sz in sizes:
            offs.append(o)
            o += (sz + 4095) // 4096 * 4096
        return dict(base=0x7f0000000000 + node * (1 << 30), bytes=o * 4, stride=o, piece_off=offs, piece_bytes=sizes)


class _Lib:
    def __init__(self, rc):
        self.rc, self.registered, self.unregistered = rc, [], []

        class _F:
            def __init__(s, fn):
                s.fn, s.argtypes = fn, None

            def __call__(s, *a):
                return s.fn(*a)

        def reg(ptr, size, dev):
            if self.rc:
                return self.rc
            self.registered.append(ptr.value)
            dev._obj.value = ptr.value
            return 0

        self.xt_host_register_mapped = _F(reg)
        self.xt_host_unregister = _F(lambda ptr: self.unregistered.append(ptr.value) or 0)


def test_map_engine_declines_cleanly(monkeypatch, caplog):
    g13, g2 = torch.ones(4, 2), torch.ones(4)
    lib = _Lib(rc=0)
    monkeypatch.setattr(ep.ops, 'cdll', lambda: lib)
    stage, regs = ep.map_engine(_Engine(nodes=2), [5, 9, 11, 2], 16, g13, g2)
    assert len(regs) == 2 and stage['bases'] == regs and stage['cold_index'].tolist()[5] == 0
    assert stage['cold_index'].tolist()[2] == 3 and int((stage['cold_index'] >= 0).sum()) == 4
    with caplog.at_level(logging.WARNING, logger='xtier_b200'):
        lib2 = _Lib(rc=0)
        monkeypatch.setattr(ep.ops, 'cdll', lambda: lib2)
        assert ep.map_engine(_Engine(bad=True), [0], 16, g13, g2) == (None, [])
        assert lib2.unregistered == lib2.registered and lib2.registered   # nothing left registered
        lib3 = _Lib(rc=1)
        monkeypatch.setattr(ep.ops, 'cdll', lambda: lib3)
        assert ep.map_engine(_Engine(), [0], 16, g13, g2) == (None, [])
    assert 'PCIe staging off' in caplog.text


def test_auto_staging_slots_formula():
    # the share of the CPU-tier experts one call touches: 32 tokens x top-8 of 256 with 112 in HBM (config 3, 1 GPU)
    n_cpu, E, k, T = 256 - 112, 256, 8, 32
    touched = n_cpu * (1 - (1 - k / E) ** T)
    assert 90 < touched < 95 and math.ceil(0.37 * touched) == 34
