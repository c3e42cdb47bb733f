"""The allocation-free decode attention entry point (xt_attn_decode_noalloc), called through its exported C symbol.

It serves callers that cannot call cudaMalloc (a host framework that owns all device memory, a plugin that may not
allocate after start-up, a serving loop that must never enter the driver's allocator): its split workspace is a fixed
device array inside the library. The test checks it against the regular entry point (torch.ops.xtier.attn_decode,
whose workspace the caller allocates) on two calls in a row, and that an oversized call is refused. This file is
collected last on purpose, so a run that stops at its first failure has run every other test before this one.
"""
import ctypes as C
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _lib():
    from xtier_b200 import ops
    L = ops.cdll()
    L.xt_attn_decode_noalloc.restype = C.c_int
    L.xt_attn_decode_noalloc.argtypes = [C.c_void_p] * 5 + [C.c_int] * 5 + [C.c_float, C.c_void_p]
    L.xt_attn_decode_noalloc_error.restype = C.c_char_p
    return L


def _call(L, q, kc, vc, lens, out, splits, scale):
    B, Hq, _ = q.shape
    Hkv, Lmax = kc.shape[1], kc.shape[2]
    return L.xt_attn_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), out.data_ptr(), B,
                                    Hq, Hkv, Lmax, splits, scale, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize('B,Hq,Hkv,Lmax,lens', [(1, 32, 4, 2304, [2100]), (2, 16, 2, 1024, [700, 33])])
def test_noalloc_matches_regular_entry_point(cuda_ops, B, Hq, Hkv, Lmax, lens):
    L = _lib()
    torch.manual_seed(7)
    D = 128
    G = Hq // Hkv
    kc = torch.randn(B, Hkv, Lmax, D, device='cuda').bfloat16()
    vc = torch.randn(B, Hkv, Lmax, D, device='cuda').bfloat16()
    seq = torch.tensor(lens, dtype=torch.int32, device='cuda')
    splits = cuda_ops.attn_decode_splits(B, Hkv, Lmax)
    scale = 1 / math.sqrt(D)
    ws_o = torch.empty(B * Hkv * splits * G * D, device='cuda')
    ws_ml = torch.empty(B * Hkv * splits * G * 2, device='cuda')
    cnt = torch.zeros(B * Hkv, dtype=torch.int32, device='cuda')
    for call in range(2):   # two calls in a row: the shared array keeps the previous call's contents
        q = torch.randn(B, Hq, D, device='cuda').bfloat16()
        ref = torch.empty_like(q)
        cuda_ops.attn_decode(q, kc, vc, seq, ref, ws_o, ws_ml, cnt, splits, scale)
        out = torch.full_like(q, float('nan'))
        rc = _call(L, q, kc, vc, seq, out, splits, scale)
        assert rc == 0, L.xt_attn_decode_noalloc_error().decode()
        torch.cuda.synchronize()
        assert _rel(out, ref) < 1e-2, (call, _rel(out, ref))
        assert torch.isfinite(out.float()).all()


def test_noalloc_rejects_oversized_workspace(cuda_ops):
    L = _lib()
    B, Hq, Hkv, Lmax, D = 64, 128, 8, 512, 128   # 64 * 8 * 2 splits * 16 * 130 floats > 512 Ki
    q = torch.zeros(B, Hq, D, device='cuda').bfloat16()
    kc = torch.zeros(B, Hkv, Lmax, D, device='cuda').bfloat16()
    seq = torch.full((B,), 4, dtype=torch.int32, device='cuda')
    out = torch.empty_like(q)
    rc = _call(L, q, kc, kc, seq, out, 2, 0.1)
    assert rc == -6
    assert 'exceeds the fixed workspace' in L.xt_attn_decode_noalloc_error().decode()
