"""Python entry to the sm_100a kernels (libxt_cuda.so, registered as torch.ops.xtier.*).

The library is built in-tree (xtier_b200/_build.py) and loaded once. On a machine with a CUDA device a missing or
unloadable library is an error, never a silent fallback: every op here runs the native kernel or raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import torch

_LIB = Path(__file__).resolve().parent.parent / '_lib' / 'libxt_cuda.so'
_loaded = False
_cdll = None


def lib_path() -> Path:
    return _LIB


def load():
    """Loads the op library (building it first if it is missing)."""
    global _loaded, _cdll
    if _loaded:
        return
    if not _LIB.exists():
        from .. import _build
        _build.build(verbose=False)
    if not _LIB.exists():
        raise RuntimeError(f'xtier_b200: {_LIB} is missing; run python -m xtier_b200._build')
    torch.ops.load_library(str(_LIB))
    _cdll = C.CDLL(str(_LIB))
    _loaded = True


def cdll():
    load()
    return _cdll


def _ops():
    load()
    return torch.ops.xtier


def add_rmsnorm(x, residual, w, out, eps: float):
    _ops().add_rmsnorm(x, residual, w, out, eps)
    return out


def rmsnorm(x, w, eps: float, out=None):
    out = torch.empty_like(x) if out is None else out
    _ops().add_rmsnorm(x, None, w, out, eps)
    return out


def qk_norm_rope_kv(qkv, q_norm, k_norm, pos, batch, q_out, k_cache, v_cache, hq: int, hkv: int, theta: float,
                    eps: float, slots=None):
    """slots (int32 [T], optional): the cache position each token's K / V goes to (default: its RoPE position)."""
    _ops().qk_norm_rope_kv(qkv, q_norm, k_norm, pos, batch, q_out, k_cache, v_cache, hq, hkv, theta, eps, slots)


def attn_decode(q, k_cache, v_cache, seqlens, out, ws_o, ws_ml, counters, splits: int, scale: float):
    _ops().attn_decode(q, k_cache, v_cache, seqlens, out, ws_o, ws_ml, counters, splits, scale)


def attn_prefill(q, k_cache, v_cache, row: int, start: int, scale: float, out=None, tree_mask=None):
    """Causal GQA attention of q [T, Hq, 128] (a view with unit stride along the last dim) at positions
    start .. start + T - 1 over row `row` of the caches [B, Hkv, max_len, 128] (tcgen05 flash kernel): query t sees keys
    0 .. start + t. Returns out [T, Hq, 128] (or writes the given view). A wait that runs out sets the shared error
    word (gemm_error_word); the caller's check() raises. tree_mask (int64 [T], T <= 64): a draft tree in cache slots
    start .. start + T - 1; query t then sees the keys before `start` and the tree slots whose bit is set in
    tree_mask[t] (its ancestors and itself) instead of the causal range."""
    if out is None:
        out = torch.empty(q.shape[0], q.shape[1], 128, dtype=torch.bfloat16, device=q.device)
    _ops().attn_prefill(q, k_cache, v_cache, out, row, start, scale, gemm_error_word(q.device), tree_mask)
    return out


def moe_route(x, wr, bias, corr, table, shared_slots, ids, w, slots, ws_logits, ws_count, k: int, mode: int = 0,
              n_group: int = 1, topk_group: int = 1, renorm: bool = True, scale: float = 1.0, layer: int = 0,
              mailbox: int = 0, active=None, logits_in=None, cold_index=None, share_min: int = 0,
              host_base: int = 0, claim=None, claim_list=None, claim_count=None, stage_max: int = 0,
              stage_slot0: int = 0):
    """`active` (int32 [m], optional): token flags; a token with flag 0 skips its routed experts (GPU and CPU),
    e.g. a verify token after a truncated draft. `logits_in` (fp32 [m, E], prefill): precomputed router logits; the
    kernel only selects (one CTA per token). `stage_max` > 0 (expert parallelism): a CPU-tier route whose expert has an
    engine slot (`cold_index` >= 0) claims one of stage_max PCIe staging slots (`claim` / `claim_list` / `claim_count`,
    reset by `ep_stage`) and becomes GPU slot stage_slot0 + index."""
    _ops().moe_route(x, wr, bias, corr, table, shared_slots, ids, w, slots, ws_logits, ws_count, k, mode, n_group,
                     topk_group, renorm, scale, layer, mailbox, active, logits_in, cold_index, share_min, host_base,
                     claim, claim_list, claim_count, stage_max, stage_slot0)


def gemm_f32(a, b, out=None):
    """a [M, K] . b [N, K]^T on the tensor cores with an FP32 result (BF16 operands)."""
    M = a.numel() // a.shape[-1]
    out = torch.empty(M, b.shape[0], dtype=torch.float32, device=a.device) if out is None else out
    _ops().gemm_tc_f32(a, b, out, gemm_error_word(a.device))
    return out


def gemv(x, w, out, add=None):
    """out[m, N] = x[m, K] . w[N, K]^T (+ add), m <= 16, BF16 (the decode projections)."""
    _ops().gemv(x, w, add, out)
    return out


def fp8_rows(table, scales, out, ids=None, block: int = 128, lo: int = 0, hi: int = 2 ** 62):
    """BF16 rows of an FP8 (E4M3) table with E8M0 block scales: out[r] = e4m3(row) * 2^(e - 127). With `ids`
    (int64, device) rows ids - lo of `table` are gathered and ids outside [lo, hi) give zeros; without, `table` holds
    the rows already gathered."""
    _ops().fp8_rows(table, scales, ids, lo, hi, block, out)
    return out


def gemv_fp8(x, w, s, out, add=None):
    """out[m, N] = x[m, K] . (w[N, K] E4M3 * s[N, K/128])^T (+ add), m <= 16 (W8A16 decode)."""
    _ops().gemv_fp8(x, w, s, add, out)
    return out


def fp8_quantize(w):
    """BF16 w [N, K] (K % 128 == 0) -> (E4M3 bytes [N, K], FP32 scales [N, K / 128]): one scale per row and 128
    columns, amax / 448 (the layout gemv_fp8, fp8_dequant and linear_fp8 read)."""
    N, K = w.shape
    g = w.float().view(N, K // 128, 128)
    s = (g.abs().amax(-1) / 448.0).clamp_min(1e-12)
    q = (g / s.unsqueeze(-1)).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8).view(N, K)
    return q.contiguous(), s.contiguous()


def fp8_dequant(w, s, out=None):
    """w[N, K] E4M3 * s[N, K/128] -> BF16 [N, K]."""
    out = torch.empty(w.shape, dtype=torch.bfloat16, device=w.device) if out is None else out
    _ops().fp8_dequant(w, s, out)
    return out


def spec_truncate(q, tokens, flags, threshold: float, topk=None):
    """Chain-draft truncation in place: q [B, S, V] draft probabilities (fp32, zeroed at the first dropped draft),
    tokens [B, S + 1] verify input, flags [B * (S + 1)] int32 out (1: the token is computed)."""
    _ops().spec_truncate(q, tokens, topk, flags, threshold)


_FP8_SCRATCH: dict = {}


def linear_fp8(x, w, s, out=None, mx8=None):
    """x @ (w * s)^T with FP8 weights (per row x 128-column scales): the W8A16 GEMV for decode-sized inputs; larger
    inputs through the W8A8 block-scaled GEMM when `mx8` (fp8_weight_to_mx8 of the same weight) is given (activations
    quantized to MXFP8 per call, as the reference's W8A8 prefill quantizes them to E4M3 per 128 columns), else a
    dequant pass into a per-device scratch and the tcgen05 BF16 GEMM (prefill is compute-bound)."""
    m = x.numel() // x.shape[-1]
    K = x.shape[-1]
    if m <= 16 and K * m * 2 <= 200 * 1024:
        out = torch.empty(*x.shape[:-1], w.shape[0], dtype=torch.bfloat16, device=x.device) if out is None else out
        return gemv_fp8(x, w, s, out)
    if mx8 is not None:
        return linear_mx8(x, mx8, out=out)
    key = (x.device, w.numel())
    buf = _FP8_SCRATCH.get(key)
    if buf is None:
        buf = _FP8_SCRATCH[key] = torch.empty(w.numel(), dtype=torch.bfloat16, device=x.device)
    wb = fp8_dequant(w, s, buf.view(w.shape))
    return linear(x.reshape(m, K), wb, out)


class MX8Weight:
    """A BF16 weight [N, K] quantized once to MXFP8 for `linear_mx8`: E4M3 codes [N, K] and UE8M0 scales per 32 values
    along K, laid out as the 512-byte scale atoms the block-scaled MMA reads (N and K multiples of 128)."""

    def __init__(self, w: torch.Tensor):
        N, K = w.shape
        if N % 128 or K % 128:
            raise ValueError('MX8Weight: N and K must be multiples of 128')
        self.N, self.K = N, K
        self.w8 = torch.empty(N, K, dtype=torch.uint8, device=w.device)
        self.sf = torch.empty(N * K // 32, dtype=torch.uint8, device=w.device)
        _ops().mx_quant_rows(w.to(torch.bfloat16).contiguous(), None, self.w8, self.sf)


def fp8_weight_to_mx8(w, s) -> MX8Weight:
    """An FP8 weight with per-row x 128-column FP32 scales as MXFP8 (dequantized to BF16, then requantized with one
    power-of-two scale per 32 values): the operand of linear_fp8's W8A8 path."""
    return MX8Weight(fp8_dequant(w, s, torch.empty(w.shape, dtype=torch.bfloat16, device=w.device)))


_MX_PAD: dict = {}


def linear_mx8(x, wq: MX8Weight, residual=None, out=None):
    """x [..., K] BF16 . wq^T (+ residual) -> [..., N] BF16 through the block-scaled FP8 tensor cores: x quantized to
    MXFP8 per call (E4M3, one power-of-two scale per 32 values), FP32 accumulation (csrc/cuda/gemm_mx8.cu)."""
    K = x.shape[-1]
    M = x.numel() // K
    Mp = (M + 127) // 128 * 128
    dev = x.device
    x8 = torch.empty(Mp, K, dtype=torch.uint8, device=dev)
    sfx = torch.empty(Mp * K // 32, dtype=torch.uint8, device=dev)
    src = None
    if Mp != M:   # rows past M quantize zeros
        key = (M, Mp, dev)
        src = _MX_PAD.get(key)
        if src is None:
            src = torch.cat([torch.arange(M, dtype=torch.int32), torch.full((Mp - M,), -1, dtype=torch.int32)]).to(dev)
            if len(_MX_PAD) < 64:
                _MX_PAD[key] = src
    _ops().mx_quant_rows(x.reshape(M, K).contiguous(), src, x8, sfx)
    out = torch.empty(*x.shape[:-1], wq.N, dtype=torch.bfloat16, device=dev) if out is None else out
    _ops().gemm_mx8(x8, sfx, M, wq.w8, wq.sf, None if residual is None else residual.reshape(M, wq.N), out,
                    gemm_error_word(dev))
    return out


# ------------------------------------------------------------------ model-pack ops (csrc/cuda/packs.cu)
def mhc_post(x, res, post, comb, out=None):
    """DeepSeek V4 manifold hyper-connection post-mix: out[m, i] = BF16(post[m, i] x[m] + sum_j comb[m, j, i] res[m, j])
    summed in the fixed order ((j0 + j1) + j2) + j3 without fused multiply-adds (bit-identical to PyTorch's FP32
    evaluation of that expression). x [M, H], res [M, 4, H] BF16; post [M, 4], comb [M, 4, 4] FP32."""
    out = torch.empty_like(res) if out is None else out
    _ops().mhc_post(x.contiguous(), res.contiguous(), post.float().contiguous(), comb.float().contiguous(), out)
    return out


def wo_a(o, w, scale=None, out=None):
    """DeepSeek V4 grouped low-rank output projection at decode sizes: out[t, g, r] = sum_h o[t, g, h] w[g, r, h], with
    w FP8 E4M3 (uint8 bytes or float8_e4m3fn) and FP32 scales per 32 x 32 block of [G R, D], or w BF16."""
    if w.dtype == torch.float8_e4m3fn:
        w = w.view(torch.uint8)
    T, G = o.shape[0], o.shape[1]
    out = torch.empty(T, G, w.shape[1], dtype=torch.bfloat16, device=o.device) if out is None else out
    _ops().wo_a(o, w, None if scale is None else scale.float(), out)
    return out


_HC_ACC: dict = {}


def hc_mix(x, w_down, w_up, hc: int, out=None):
    """Qwen4-exp hyper-connection low-rank mix: acc = x . w_down^T, t = BF16(silu(acc / hc)), gate = sigmoid(t . w_up^T)
    [rows, hc, hs], out[m, j] = sum_g gate[m, g, j] x[m, g hs + j] / hc. x [rows, hc hs] BF16 -> out [rows, hs]."""
    rows, K = x.shape
    L = w_down.shape[0]
    key = (x.device, L)
    acc = _HC_ACC.get(key)
    if acc is None:
        acc = _HC_ACC[key] = torch.empty(16 * L, dtype=torch.float32, device=x.device)
    out = torch.empty(rows, K // hc, dtype=torch.bfloat16, device=x.device) if out is None else out
    _ops().hc_mix(x.contiguous(), w_down.contiguous(), w_up.contiguous(), acc, out, hc)
    return out


_gemm_err: dict = {}


def gemm_error_word(device) -> torch.Tensor:
    """The tcgen05 GEMM's error word of `device` (non-zero after a bounded wait in the kernel ran out)."""
    key = torch.device(device)
    if key not in _gemm_err:
        _gemm_err[key] = torch.zeros(1, dtype=torch.int32, device=key)
    return _gemm_err[key]


def gemm(a, b, out=None, residual=None):
    """out[M, N] = a[M, K] . b[N, K]^T (+ residual) on the tcgen05 tensor cores (TMA, TMEM, persistent)."""
    M, N = a.numel() // a.shape[-1], b.shape[0]
    out = torch.empty(*a.shape[:-1], N, dtype=a.dtype, device=a.device) if out is None else out
    _ops().gemm_tc(a, b, residual, out, gemm_error_word(a.device))
    return out


_SMS: dict = {}


def _sms(device) -> int:
    key = torch.device(device)
    if key not in _SMS:
        _SMS[key] = torch.cuda.get_device_properties(key).multi_processor_count
    return _SMS[key]


def skinny_splits(N: int, K: int, sms: int) -> int:
    """K splits of skinny_gemm for (N, K): about two CTAs per SM, at least 4 k-blocks of 64 per CTA."""
    nblk = -(-N // 128)
    return max(1, min(-(-2 * sms // nblk), (K // 64) // 4))


def skinny_gemm(x, w, out=None, add=None):
    """out[M, N] = x[M, K] . w[N, K]^T (+ add) for M <= 32, K % 64 == 0, on the tcgen05 tensor cores with the weights
    as the MMA's 128-row operand (csrc/cuda/gemm_skinny.cu); K split over CTAs with FP32 partials reduced in order."""
    K = x.shape[-1]
    M, N = x.numel() // K, w.shape[0]
    out = torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device) if out is None else out
    splits = skinny_splits(N, K, _sms(x.device))
    part = torch.empty(splits, M, N, dtype=torch.float32, device=x.device) if splits > 1 else None
    _ops().skinny_gemm(x, w, add, out, part, splits, gemm_error_word(x.device))
    return out


def linear(x, w, out=None):
    """x @ w^T in BF16. Decode-sized inputs (<= 32 rows): the tcgen05 skinny GEMM when K % 64 == 0 and there are three
    rows or more, else the weight-streaming GEMV (at most two passes over the weights, each of <= 16 rows whose
    activations fit the kernel's shared memory). Larger inputs: the tcgen05 GEMM (cuBLAS only for shapes TMA cannot
    describe: K not a multiple of 8 or unaligned rows)."""
    m = x.numel() // x.shape[-1]
    K = x.shape[-1]
    # the skinny GEMM from 3 rows on (measured faster than the GEMV on every decode projection from 4 rows: the
    # GEMV's FP32 FMA issue grows with the rows), the GEMV for one or two rows
    if (3 <= m <= 32 and K % 64 == 0 and x.is_cuda and x.is_contiguous() and w.is_contiguous()
            and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.data_ptr() % 16 == 0
            and w.data_ptr() % 16 == 0 and (out is None or out.is_contiguous())):
        return skinny_gemm(x, w, out)
    per = min(16, (200 * 1024) // (K * 2))
    if per >= 1 and m <= 2 * per and x.is_contiguous() and x.dtype == torch.bfloat16:
        out = torch.empty(*x.shape[:-1], w.shape[0], dtype=x.dtype, device=x.device) if out is None else out
        if m <= per:
            _ops().gemv(x, w, None, out)
            return out
        x2, o2 = x.reshape(m, K), out.view(m, w.shape[0])
        _ops().gemv(x2[:per], w, None, o2[:per])
        _ops().gemv(x2[per:], w, None, o2[per:])
        return out
    if (x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.is_contiguous() and w.is_contiguous()
            and K % 8 == 0 and x.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0 and x.is_cuda):
        return gemm(x, w, out)
    return torch.matmul(x, w.t(), out=out) if out is not None else torch.matmul(x, w.t())


def mla_prep(inp, q_lora: int, q_norm, kv_norm, pos, slot, eps: float, theta: float, q_out, codes, scales, rope,
             lat_out=None):
    """The fused [q_a | kv_a] projection rows inp [T, >= q_lora + 576] -> q_out [T, q_lora] = RMSNorm(q_a) and the
    NVFP4 latent cache at `slot` (int64 [T]): RMSNorm of the compressed KV and RoPE of the rotary key at `pos`
    (int32 [T]); lat_out [T, 576] (optional) receives the BF16 latent rows."""
    _ops().mla_prep(inp, q_lora, q_norm, kv_norm, pos, slot, eps, theta, q_out, codes, scales, rope, lat_out)
    return q_out


def head_gemm(x, w, y, pos=None, rope_x: int = 0, rope_y: int = 0, rope_dims: int = 0, theta: float = 0.0):
    """Per head h: y[t, h, :N] = x[t, h, :K] . w[h] (w [heads, K, N]); with rope_dims, also
    y[t, h, rope_y:rope_y + rope_dims] = NeoX RoPE of x[t, h, rope_x:rope_x + rope_dims] at pos[t]."""
    _ops().head_gemm(x, w, y, pos, rope_x, rope_y, rope_dims, theta)
    return y


def rope_heads(x, pos, theta: float, out):
    """out[t, h, :] = NeoX RoPE of x[t, h, :] at pos[t] (int32): x and out [T, H, d] BF16 views with unit stride along
    d (any token and head strides)."""
    _ops().rope_heads(x, pos, float(theta), out)
    return out


def silu_mul(inp, out):
    """inp [T, 2I] (gate then up) -> out [T, I] = SiLU(gate) * up."""
    _ops().silu_mul(inp, out)
    return out


def l2_prefetch(ptrs, sizes, ctas: int = 16):
    """Bulk-prefetch the device ranges (int64 address and byte tensors on the device) into L2."""
    _ops().l2_prefetch(ptrs, sizes, ctas)


def moe_gate_up(x, slots, w13, s13, g13, mid, fmt: int, limit: float = 0.0, alpha: float = 1.0, beta: float = 0.0,
                peer=None, spr: int = 0, host=None, host_base: int = 0):
    """`peer` (int64 [W * 6] on the device, with `spr` slots per rank): every rank's pool base addresses; slots then
    name (rank, local slot) and a peer's slot is read over NVLink. `host` (int64 [6]): the pinned host pool of the CPU
    tier's experts; a slot >= host_base names one of them (read over PCIe, the miss share)."""
    _ops().moe_gate_up(x, slots, w13, s13, g13, mid, fmt, limit, alpha, beta, peer, spr, host, host_base)


def moe_down(mid, slots, w, w2, s2, g2, add, out, out_f32=None, fmt: int = 0, mailbox: int = 0, gpu_part=None,
             peer=None, spr: int = 0, host=None, host_base: int = 0):
    _ops().moe_down(mid, slots, w, w2, s2, g2, add, out, out_f32, gpu_part, fmt, mailbox, peer, spr, host, host_base)


def attn_decode_splits(batch: int, kv_heads: int, max_len: int, sms: int = 148) -> int:
    """Key splits of the decode attention: about 192 keys of the cache per split (measured on B200 with the tensor-core
    kernel: fewer, longer splits lose to the load latency, more lose to the merge), at most enough CTAs (splits x batch
    x kv_heads) to cover every SM once, at most 64 (the merge reads every split's partial). The kernel cuts the splits
    from the actual sequence length, so all of them have work."""
    want = max(1, (sms + batch * kv_heads - 1) // (batch * kv_heads))
    return max(1, min(64, want, (max_len + 191) // 192))
