"""Block-scaled grouped expert GEMM (MXFP4 weights x MXFP8 activations, tcgen05 kind::mxf8f6f4 with scales in TMEM):
the MXFP8 row quantizer's bytes and scale atoms, the kernel against the product of its exactly dequantized operands
(which checks the scale-atom layout and per-MMA scale selection to FP32 rounding), and the whole grouped MoE against
the fp32 reference within the activation quantization's error."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _atom_scales(sfx: torch.Tensor, R: int, K: int) -> torch.Tensor:
    """Scale atoms [R/128][K/128][512] -> UE8M0 exponent bytes [R, K/32]."""
    r = torch.arange(R)
    b = torch.arange(K // 32)
    rr = (r % 128)[:, None]
    idx = ((r // 128)[:, None] * (K // 128) + (b // 4)[None]) * 512 + (rr % 32) * 16 + (rr // 32) * 4 + (b % 4)[None]
    return sfx.cpu()[idx].long()


def _dequant_x8(x8: torch.Tensor, sfx: torch.Tensor) -> torch.Tensor:
    R, K = x8.shape
    e = _atom_scales(sfx, R, K)
    vals = x8.cpu().view(torch.float8_e4m3fn).float()
    return vals * torch.pow(2.0, (e - 127).float()).repeat_interleave(32, 1)


def test_mx_quant_rows_bytes_and_atoms(cuda_ops):
    g = torch.Generator().manual_seed(1)
    R, K, n = 256, 512, 300
    x = torch.randn(n, K, generator=g) * torch.pow(10.0, torch.empty(n, 1).uniform_(-3, 3, generator=g))
    x[5, 64:96] = 0.0                                       # an all-zero block
    x = x.bfloat16()
    src = torch.randperm(n, generator=g)[:R].int()
    src[::17] = -1                                          # padding rows
    x8 = torch.empty(R, K, dtype=torch.uint8, device='cuda')
    sfx = torch.empty(R * K // 32, dtype=torch.uint8, device='cuda')
    torch.ops.xtier.mx_quant_rows(x.cuda(), src.cuda(), x8, sfx)
    torch.cuda.synchronize()
    want = torch.where(src[:, None] >= 0, x.float()[src.clamp_min(0).long()], torch.zeros(R, K))
    e = _atom_scales(sfx, R, K) - 127
    amax = want.abs().unflatten(1, (-1, 32)).amax(-1)
    nz = amax > 0
    assert bool((amax[nz] / torch.pow(2.0, e[nz].float()) <= 448).all())        # no value saturates
    assert bool((amax[nz] / torch.pow(2.0, e[nz].float() - 1) > 448).all())     # the smallest such power of two
    dq = _dequant_x8(x8, sfx)
    bound = torch.maximum(want.abs() * 2 ** -4, torch.pow(2.0, e.float() - 10).repeat_interleave(32, 1))
    assert bool(((dq - want).abs() <= bound * 1.0001).all())
    assert bool((dq[~nz.repeat_interleave(32, 1)] == 0).all())


def _setup(E, H, I, m, k, seed):
    from xtier_b200 import formats
    from xtier_b200.cache.prefill import plan
    g = torch.Generator().manual_seed(seed)
    ex = formats.random_experts(E, H, I, formats.MXFP4, seed=seed, std=0.05).to('cuda')
    x = torch.randn(m, H, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(m)]).int()
    ids[: m // 2, 0] = 0                                    # a run longer than one 128-row tile
    w = torch.rand(m, k, generator=g)
    return ex, x, ids, w, plan


def test_grouped_mx_kernel_matches_dequantized_operands(cuda_ops):
    from xtier_b200 import formats
    from xtier_b200.cache.prefill import TILE, _tiles
    E, H, I, m, k = 8, 512, 256, 300, 4
    ex, x, ids, w, plan = _setup(E, H, I, m, k, 7)
    order, rows, R, runs = plan(ids.cuda())
    src = torch.full((R,), -1, dtype=torch.int32, device='cuda')
    src[rows] = (order // k).int()
    err = torch.zeros(1, dtype=torch.int32, device='cuda')
    x8 = torch.empty(R, H, dtype=torch.uint8, device='cuda')
    sfx = torch.empty(R * H // 32, dtype=torch.uint8, device='cuda')
    torch.ops.xtier.mx_quant_rows(x.cuda(), src, x8, sfx)
    mid = torch.zeros(R, I, dtype=torch.bfloat16, device='cuda')
    torch.ops.xtier.moe_grouped_mx(x8, sfx, ex.w13, ex.s13, ex.g13.float().contiguous(),
                                   _tiles(runs, I // 64, 'cuda', TILE), True, I, None, mid, err)
    m8 = torch.empty(R, I, dtype=torch.uint8, device='cuda')
    sfm = torch.empty(R * I // 32, dtype=torch.uint8, device='cuda')
    torch.ops.xtier.mx_quant_rows(mid, None, m8, sfm)
    rw = torch.zeros(R, dtype=torch.float32, device='cuda')
    rw[rows] = w.cuda().flatten()[order]
    y = torch.zeros(R, H, dtype=torch.float32, device='cuda')
    torch.ops.xtier.moe_grouped_mx(m8, sfm, ex.w2, ex.s2, ex.g2.float().contiguous(),
                                   _tiles(runs, H // 128, 'cuda', TILE), False, I, rw, y, err)
    torch.cuda.synchronize()
    assert int(err) == 0
    xd, md = _dequant_x8(x8, sfx), _dequant_x8(m8, sfm)
    slot_of_row = torch.full((R,), -1, dtype=torch.long)
    for s, first, count in runs.tolist():
        slot_of_row[first:first + count] = s
    mid_c, y_c, rw_c = mid.cpu().float(), y.cpu(), rw.cpu()
    gate_err = up_ref_n = down_err = down_n = 0.0
    for s in slot_of_row.unique().tolist():
        if s < 0:
            continue
        r = slot_of_row == s
        w1, w3, w2 = ex.to('cpu').dequant(s)
        gt, ut = xd[r] @ w1.t(), xd[r] @ w3.t()
        ref_mid = torch.nn.functional.silu(gt) * ut
        gate_err += float((mid_c[r] - ref_mid).norm() ** 2)
        up_ref_n += float(ref_mid.norm() ** 2)
        ref_y = (md[r] @ w2.t()) * rw_c[r][:, None]
        down_err += float((y_c[r] - ref_y).norm() ** 2)
        down_n += float(ref_y.norm() ** 2)
    assert (gate_err / up_ref_n) ** 0.5 < 5e-3      # BF16 rounding of mid
    assert (down_err / down_n) ** 0.5 < 1e-4        # FP32 accumulation order only


def test_grouped_experts_mx_vs_reference(cuda_ops, monkeypatch):
    from xtier_b200 import formats
    from xtier_b200.cache.prefill import grouped_experts
    monkeypatch.setenv('XTIER_PREFILL_MX', '1')
    E, H, I, m, k = 16, 1024, 512, 200, 8
    ex, x, ids, w, _ = _setup(E, H, I, m, k, 21)
    slots = ids.clone()
    slots[torch.rand(m, k, generator=torch.Generator().manual_seed(3)) < 0.2] = -1
    err = torch.zeros(1, dtype=torch.int32, device='cuda')
    out = grouped_experts(x.cuda(), slots.cuda(), w.cuda(), ex, err)
    torch.cuda.synchronize()
    assert int(err) == 0
    ids_ref = torch.where(slots >= 0, ids, torch.full_like(ids, -1))
    ref = formats.reference_moe(x, ids_ref, w, ex.to('cpu'))
    rel = float((out.cpu() - ref).norm() / ref.norm())
    assert rel < 6e-2, rel                          # MXFP8 activations (E4M3, power-of-two block scales)
