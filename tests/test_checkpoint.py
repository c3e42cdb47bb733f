"""Expert checkpoints: safetensors round trip through the plain reader and through the O_DIRECT fast loader (tensor
windows not aligned to 512 bytes, several read pieces), and the scale sanity check."""
import json
import struct

import torch

from xtier_b200 import checkpoint, formats


def test_safetensors_roundtrip_direct_and_plain(tmp_path, monkeypatch):
    monkeypatch.setattr(checkpoint, 'PIECE', 1 << 16)   # several pieces per tensor
    for fmt in (formats.NVFP4, formats.MXFP4):
        ew = formats.random_experts(6, 256, 128, fmt, seed=3)
        p = tmp_path / f'layer_{fmt}.safetensors'
        checkpoint.save_experts(p, ew)
        hdr, data0 = checkpoint.read_header(p)
        assert hdr['__metadata__']['xtier.fmt'] == fmt and data0 % 8 == 0
        with open(p, 'rb') as f:   # a standard safetensors file: 8-byte length, JSON header
            n = struct.unpack('<Q', f.read(8))[0]
            assert 'experts.w13' in json.loads(f.read(n))
        for direct in (False, True):
            back = checkpoint.load_experts(p, direct=direct, threads=3)
            for name in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):
                assert torch.equal(getattr(back, name), getattr(ew, name).cpu()), (fmt, direct, name)
            assert back.fmt == fmt and checkpoint.check_scales(back)
