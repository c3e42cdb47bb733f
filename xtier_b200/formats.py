"""Expert weight formats: NVFP4 and MXFP4 encode / decode and the checkpoint adapters.

Both formats store E2M1 (FP4) codes two per byte, the even element of a row in the low nibble, with a block scale
per 16 (NVFP4: E4M3 bytes, plus an FP32 global scale per expert and projection) or per 32 elements (MXFP4: UE8M0
bytes, 2^(e-127), no global scale). The expert tensors every tier of this framework consumes are

    w13 [E, 2I, H/2] uint8   gate rows then up rows      s13 [E, 2I, H/bs] uint8
    w2  [E, H, I/2]  uint8                               s2  [E, H, I/bs]  uint8
    g13 [E, 2] float32 (gate, up multipliers)            g2  [E] float32

which is the layout of ModelOpt NVFP4 and DeepSeek MXFP4 checkpoints, so a checkpoint is consumed byte for byte
(reference: xtier/backend/formats.py:1-5, :117-128 for the ModelOpt encoding rule, :74-90 for UE8M0 bytes).

Everything here is plain torch and runs on the CPU; it is the oracle the CUDA kernels and the C++ engine are
tested against.
"""
from __future__ import annotations

import dataclasses

import torch

# E2M1 magnitudes of codes 0..7; bit 3 is the sign.
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
# Rounding boundaries between consecutive magnitudes. A value equal to a boundary takes the smaller magnitude
# (torch.bucketize with right=False puts it in the lower bucket).
_E2M1_MIDPOINTS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)

NVFP4 = 'nvfp4'
MXFP4 = 'mxfp4'
BLOCK = {NVFP4: 16, MXFP4: 32}


def e2m1_table(device=None, dtype=torch.float32) -> torch.Tensor:
    """All 16 codes as values: [0, .5, 1, 1.5, 2, 3, 4, 6, -0, -.5, ..., -6]."""
    pos = torch.tensor(E2M1_VALUES, dtype=dtype, device=device)
    return torch.cat([pos, -pos])


def unpack_e2m1(packed: torch.Tensor) -> torch.Tensor:
    """uint8 [..., K/2] -> float32 [..., K] (low nibble = even element)."""
    lo = (packed & 0x0F).long()
    hi = (packed >> 4).long()
    codes = torch.stack([lo, hi], dim=-1).flatten(-2)
    return e2m1_table(packed.device)[codes]


def e4m3_to_float(b: torch.Tensor) -> torch.Tensor:
    return b.contiguous().view(torch.float8_e4m3fn).float()


def ue8m0_to_float(b: torch.Tensor) -> torch.Tensor:
    """UE8M0 bytes -> 2^(e-127); e=0 is 2^-127 (not zero), 255 is NaN in OCP MX and never produced here."""
    return torch.pow(2.0, b.float() - 127.0)


def _e2m1_codes(q: torch.Tensor) -> torch.Tensor:
    """Nearest E2M1 code of q (saturating at 6), sign in bit 3, -0 encoded as +0."""
    bounds = torch.tensor(_E2M1_MIDPOINTS, device=q.device)
    code = torch.bucketize(q.abs().clamp(max=6.0), bounds).to(torch.uint8)
    code |= ((q < 0) & (code > 0)).to(torch.uint8) << 3
    return code


def _pack_codes(code: torch.Tensor) -> torch.Tensor:
    return code[..., 0::2] | (code[..., 1::2] << 4)


def nvfp4_encode(w: torch.Tensor):
    """ModelOpt NVFP4 of w [rows, K] (K % 16 == 0): (codes [rows, K/2], E4M3 scales [rows, K/16] as bytes, FP32 global
    scale g = amax / (6 * 448)) with w ~ e2m1 * scale * g. The global scale keeps every block scale <= 448 (E4M3 max);
    each element rounds to the nearest E2M1 value of w / (scale * g). This is the checkpoint format's own rule, so it
    is kept exactly (reference xtier/backend/formats.py:117-128)."""
    w = w.float()
    g = (w.abs().amax() / (6.0 * 448.0)).clamp_min(1e-12)
    blocks = w.unflatten(-1, (-1, 16))
    s = (blocks.abs().amax(-1) / (6.0 * g)).to(torch.float8_e4m3fn)
    q = (blocks / (s.float() * g).clamp_min(1e-30).unsqueeze(-1)).flatten(-2)
    return _pack_codes(_e2m1_codes(q)), s.view(torch.uint8), g


def mxfp4_encode(w: torch.Tensor):
    """OCP MXFP4 of w [rows, K] (K % 32 == 0): (codes [rows, K/2], UE8M0 scales [rows, K/32]). The shared exponent is
    floor(log2(amax)) - 2 (E2M1's largest exponent), so the block's largest magnitude lands in [4, 8) before
    rounding, saturating at 6 (OCP Microscaling Formats spec v1.0, section 6.3)."""
    w = w.float()
    blocks = w.unflatten(-1, (-1, 32))
    amax = blocks.abs().amax(-1)
    e = torch.floor(torch.log2(amax.clamp_min(2.0 ** -125))) - 2.0
    e = e.clamp(-127, 127)
    scale = torch.pow(2.0, e)
    q = (blocks / scale.unsqueeze(-1)).flatten(-2)
    return _pack_codes(_e2m1_codes(q)), (e + 127).to(torch.uint8)


def dequant(packed: torch.Tensor, scales: torch.Tensor, fmt: str, global_scale=None) -> torch.Tensor:
    """codes [..., K/2] + block scales [..., K/bs] (+ global) -> float32 [..., K]."""
    vals = unpack_e2m1(packed)
    bs = BLOCK[fmt]
    sf = e4m3_to_float(scales) if fmt == NVFP4 else ue8m0_to_float(scales)
    out = (vals.unflatten(-1, (-1, bs)) * sf.unsqueeze(-1)).flatten(-2)
    if global_scale is not None:
        out = out * global_scale
    return out


@dataclasses.dataclass
class ExpertWeights:
    """Quantized experts of one MoE layer in the engine layout (module docstring). `fmt` is NVFP4 or MXFP4."""
    fmt: str
    w13: torch.Tensor
    w2: torch.Tensor
    s13: torch.Tensor
    s2: torch.Tensor
    g13: torch.Tensor
    g2: torch.Tensor

    @property
    def experts(self) -> int:
        return self.w13.shape[0]

    @property
    def hidden(self) -> int:
        return self.w2.shape[1]

    @property
    def inter(self) -> int:
        return self.w13.shape[1] // 2

    def to(self, device) -> 'ExpertWeights':
        return ExpertWeights(self.fmt, *(getattr(self, f).to(device) for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2')))

    def select(self, idx) -> 'ExpertWeights':
        return ExpertWeights(self.fmt, *(getattr(self, f)[idx] for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2')))

    def contiguous(self) -> 'ExpertWeights':
        return ExpertWeights(self.fmt, *(getattr(self, f).contiguous()
                                         for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2')))

    def tp_slice(self, rank: int, world: int) -> 'ExpertWeights':
        """This tensor-parallel rank's share of every expert: intermediate units [rank * I / world, (rank + 1) * I /
        world) -- those gate and up rows, the same columns of the down projection (codes and block scales), the global
        scales unchanged. SwiGLU acts per intermediate unit and the down projection is linear in them, so the ranks'
        outputs sum to the whole expert's. I / world must be a multiple of the block size."""
        I, bs = self.inter, BLOCK[self.fmt]
        if I % world or (I // world) % bs:
            raise ValueError(f'tp_slice: {I} intermediate units do not split into {world} shares of whole '
                             f'{bs}-blocks')
        n = I // world
        a, b = rank * n, (rank + 1) * n
        w13 = torch.cat([self.w13[:, a:b], self.w13[:, I + a:I + b]], 1).contiguous()
        s13 = torch.cat([self.s13[:, a:b], self.s13[:, I + a:I + b]], 1).contiguous()
        w2 = self.w2[:, :, a // 2:b // 2].contiguous()
        s2 = self.s2[:, :, a // bs:b // bs].contiguous()
        return ExpertWeights(self.fmt, w13, w2, s13, s2, self.g13.clone(), self.g2.clone())

    def dequant(self, e: int):
        """(w1 [I,H], w3 [I,H], w2 [H,I]) float32 of expert e."""
        I = self.inter
        g13 = self.g13[e].float()
        w13 = dequant(self.w13[e], self.s13[e], self.fmt)
        w1 = w13[:I] * g13[0]
        w3 = w13[I:] * g13[1]
        w2 = dequant(self.w2[e], self.s2[e], self.fmt) * self.g2[e].float()
        return w1, w3, w2

    def nbytes_per_expert(self) -> int:
        return sum(getattr(self, f)[0].numel() * getattr(self, f).element_size() for f in ('w13', 'w2', 's13', 's2'))


def quantize_experts(w1: torch.Tensor, w3: torch.Tensor, w2: torch.Tensor, fmt: str) -> ExpertWeights:
    """fp32 experts w1/w3 [E, I, H], w2 [E, H, I] -> ExpertWeights. NVFP4 takes a global scale per expert and
    projection (gate and up separately, as ModelOpt does)."""
    E, I, H = w1.shape
    w13_l, s13_l, w2_l, s2_l = [], [], [], []
    g13 = torch.ones(E, 2)
    g2 = torch.ones(E)
    for e in range(E):
        if fmt == NVFP4:
            qg, sg, gg = nvfp4_encode(w1[e])
            qu, su, gu = nvfp4_encode(w3[e])
            qd, sd, gd = nvfp4_encode(w2[e])
            g13[e, 0], g13[e, 1], g2[e] = gg, gu, gd
        else:
            qg, sg = mxfp4_encode(w1[e])
            qu, su = mxfp4_encode(w3[e])
            qd, sd = mxfp4_encode(w2[e])
        w13_l.append(torch.cat([qg, qu]))
        s13_l.append(torch.cat([sg, su]))
        w2_l.append(qd)
        s2_l.append(sd)
    return ExpertWeights(fmt, torch.stack(w13_l), torch.stack(w2_l), torch.stack(s13_l), torch.stack(s2_l),
                         g13.float(), g2.float())


def random_experts(E: int, H: int, I: int, fmt: str, std: float = 0.02, seed: int = 0,
                   device='cpu') -> ExpertWeights:
    """Random-init N(0, std) experts quantized to `fmt`, generated in chunks so that big layers fit in memory."""
    gen = torch.Generator(device='cpu').manual_seed(seed)
    w1 = torch.randn(E, I, H, generator=gen) * std
    w3 = torch.randn(E, I, H, generator=gen) * std
    w2 = torch.randn(E, H, I, generator=gen) * std
    return quantize_experts(w1, w3, w2, fmt).to(device)


def synthetic_experts(E: int, H: int, I: int, fmt: str, device, seed: int = 0, std: float = 0.02) -> ExpertWeights:
    """Random experts for benchmarks, generated on `device` without an fp32 round trip: uniform random E2M1 codes
    and block scales that give roughly N(0, std)-sized weights. Same bytes per expert as a quantized checkpoint."""
    g = torch.Generator(device=device).manual_seed(seed)
    bs = BLOCK[fmt]
    w13 = torch.randint(0, 256, (E, 2 * I, H // 2), dtype=torch.uint8, device=device, generator=g)
    w2 = torch.randint(0, 256, (E, H, I // 2), dtype=torch.uint8, device=device, generator=g)
    if fmt == NVFP4:
        # block scale ~ amax/6 of N(0, std) blocks with g = 1: e4m3 of ~ 2.5*std/6 ~ 0.0083 at std 0.02
        sv = torch.tensor([std * 2.5 / 6.0], device=device).to(torch.float8_e4m3fn).view(torch.uint8)
    else:
        sv = torch.tensor([127 + round(torch.log2(torch.tensor(std * 2.5 / 4.0)).item())],
                          dtype=torch.uint8, device=device)
    s13 = sv.expand(E, 2 * I, H // bs).contiguous()
    s2 = sv.expand(E, H, I // bs).contiguous()
    g13 = torch.ones(E, 2, device=device)
    g2 = torch.ones(E, device=device)
    return ExpertWeights(fmt, w13, w2, s13, s2, g13, g2)


def reference_moe(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, experts: ExpertWeights,
                  limit: float = 0.0, alpha: float = 1.0, beta: float = 0.0, shared: ExpertWeights | None = None):
    """FP32 dequant reference of the routed experts: y[t] = sum_k w[t,k] * down(swiglu(gate x, up x)) (+ shared
    experts with weight 1). ids < 0 are skipped. swiglu with limit L > 0 clamps up to [-L, L] and gate to (-inf, L];
    alpha / beta give the GPT-OSS form gate*sigmoid(alpha*gate)*(up+beta)."""
    x = x.float().cpu()
    m, k = ids.shape
    y = torch.zeros(m, experts.hidden)
    cache = {}

    def run(ew, e, xt):
        key = (id(ew), e)
        if key not in cache:
            cache[key] = ew.dequant(e)
        w1, w3, w2 = cache[key]
        g = xt @ w1.T
        u = xt @ w3.T
        if limit > 0:
            g = g.clamp(max=limit)
            u = u.clamp(-limit, limit)
        if alpha == 1.0 and beta == 0.0:
            h = torch.nn.functional.silu(g) * u
        else:
            h = g * torch.sigmoid(alpha * g) * (u + beta)
        return h @ w2.T

    cpu_experts = experts.to('cpu')
    for t in range(m):
        for j in range(k):
            e = int(ids[t, j])
            if e < 0:
                continue
            y[t] += float(weights[t, j]) * run(cpu_experts, e, x[t])
        if shared is not None:
            sh = shared.to('cpu')
            for e in range(sh.experts):
                y[t] += run(sh, e, x[t])
    return y
