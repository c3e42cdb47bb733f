"""Hugging Face checkpoints of Qwen3-MoE models: `config.json`, safetensors shards, and the expert formats they come in.

    model = Qwen3MoeModel.from_pretrained('/models/Qwen3-30B-A3B-NVFP4', device='cuda', hot_fraction=0.4, ...)

`SafeTensors` reads a checkpoint directory (a `model.safetensors.index.json` weight map, or every `*.safetensors` file
in it) from the files' own headers: 8-byte little-endian header length, JSON of dtype / shape / data offsets, tensor
bytes. Tensors are copied out of a read-only memory map one at a time, so a checkpoint larger than RAM loads layer by
layer.

`HFWeights` is the weight source `Qwen3MoeModel` builds from: the dense weights as BF16 (BF16 / FP16 / FP32 as
stored; FP8 weights times their `weight_scale`; NVFP4-packed weights dequantized), the router, and each layer's
routed experts in the framework's expert layout (formats.py), taken from the checkpoint's own format:

    ModelOpt NVFP4         experts.<e>.<proj>.weight U8 [rows, K/2], .weight_scale F8_E4M3 [rows, K/16],
                           .weight_scale_2 F32 (the global multiplier)                     -> bytes as stored
    compressed-tensors     .weight_packed, .weight_scale, .weight_global_scale (a divisor) -> g = 1 / global scale
    MXFP4                  .weight U8/I8 packed, .weight_scale_inv or .weight_scale as UE8M0 bytes, F8_E8M0 or FP32
                           powers of two                                                   -> bytes as stored, g = 1
    BF16 / FP16 / FP32     experts.<e>.<proj>.weight, or fused experts.gate_up_proj [E, 2I, H] + experts.down_proj
                           [E, H, I]                                                       -> quantized at load to
                           XTIER_CKPT_FORMAT (nvfp4 by default; ModelOpt's rounding rule, formats.nvfp4_encode)

with <proj> gate_proj / up_proj / down_proj. Gate rows come first in w13, and gate and up keep their own global scale.
(Reference parity: xtier/backend/formats.py:40-175 -- ModelOptNvFp4, CompressedTensorsNvFp4 (reciprocal global scale),
Fp8Fp4Experts (UE8M0 bytes from FP32 powers of two), Bf16AsNvFp4 (BF16 experts quantized at hand-off); the reference
takes these tensors from SGLang's loader, this module reads the checkpoint files itself.)
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np
import torch

from .. import formats
from ..formats import MXFP4, NVFP4, ExpertWeights

_DTYPES = {
    'BF16': torch.bfloat16, 'F16': torch.float16, 'F32': torch.float32, 'F64': torch.float64,
    'U8': torch.uint8, 'I8': torch.int8, 'I16': torch.int16, 'I32': torch.int32, 'I64': torch.int64,
    'BOOL': torch.bool, 'F8_E4M3': torch.float8_e4m3fn, 'F8_E5M2': torch.float8_e5m2,
    'F8_E8M0': torch.float8_e8m0fnu,
}


class SafeTensors:
    """Read-only view of the tensors of a safetensors file or checkpoint directory."""

    def __init__(self, path):
        p = Path(path)
        files = [p] if p.is_file() else None
        if files is None:
            index = p / 'model.safetensors.index.json'
            if index.exists():
                files = sorted({p / f for f in json.loads(index.read_text())['weight_map'].values()})
            else:
                files = sorted(p.glob('*.safetensors'))
        if not files:
            raise FileNotFoundError(f'{path}: no safetensors files')
        self.entries: dict[str, tuple[int, dict, int]] = {}
        self._maps: list = [None] * len(files)
        self.files = [str(f) for f in files]
        for i, f in enumerate(files):
            with open(f, 'rb') as fh:
                n = struct.unpack('<Q', fh.read(8))[0]
                header = json.loads(fh.read(n))
            for name, h in header.items():
                if name != '__metadata__':
                    self.entries[name] = (i, h, 8 + n)

    def __contains__(self, name: str) -> bool:
        return name in self.entries

    def names(self):
        return self.entries.keys()

    def dtype(self, name: str) -> str:
        return self.entries[name][1]['dtype']

    def shape(self, name: str) -> list[int]:
        return list(self.entries[name][1]['shape'])

    def get(self, name: str) -> torch.Tensor:
        """The tensor, copied into a new CPU tensor of its dtype."""
        if name not in self.entries:
            raise KeyError(f'checkpoint has no tensor {name!r}')
        i, h, data0 = self.entries[name]
        if self._maps[i] is None:
            from ..utils.platform import read_ahead
            read_ahead(self.files[i])
            self._maps[i] = np.memmap(self.files[i], dtype=np.uint8, mode='r')
        a, b = h['data_offsets']
        raw = torch.from_numpy(np.array(self._maps[i][data0 + a:data0 + b]))
        dt = _DTYPES.get(h['dtype'])
        if dt is None:
            raise TypeError(f'{name}: safetensors dtype {h["dtype"]} is not supported')
        return raw.view(dt).reshape(h['shape'])

    def close(self, drop_cache: bool = True):
        """Unmaps the files; drop_cache also evicts their pages from the page cache (the tensors were copied out)."""
        used = [f for f, m in zip(self.files, self._maps) if m is not None]
        self._maps = [None] * len(self._maps)
        if drop_cache and used:
            from ..utils.platform import drop_file_cache
            drop_file_cache(used)


def save_safetensors(path, tensors: dict, metadata: dict | None = None):
    """Writes `tensors` (name -> CPU tensor) as one safetensors file (the format `SafeTensors` reads)."""
    rev = {v: k for k, v in _DTYPES.items()}
    header, off, blobs = {}, 0, []
    if metadata:
        header['__metadata__'] = {k: str(v) for k, v in metadata.items()}
    for name, t in tensors.items():
        t = t.detach().to('cpu').contiguous()
        b = t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b''
        header[name] = dict(dtype=rev[t.dtype], shape=list(t.shape), data_offsets=[off, off + len(b)])
        off += len(b)
        blobs.append(b)
    h = json.dumps(header).encode()
    h += b' ' * ((-len(h)) % 8)
    with open(path, 'wb') as f:
        f.write(struct.pack('<Q', len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


# ---------------------------------------------------------------------------------------------------- config
def config_from_hf(cfg: dict, fmt: str | None = None):
    """Qwen3MoeConfig of a Hugging Face `config.json` (qwen3_moe), plus (tie_word_embeddings, norm_topk_prob)."""
    from .qwen3_moe import Qwen3MoeConfig
    mt = cfg.get('model_type', 'qwen3_moe')
    if mt != 'qwen3_moe':
        raise NotImplementedError(f'model_type {mt!r}: this loader reads qwen3_moe checkpoints')
    if cfg.get('mlp_only_layers') or cfg.get('decoder_sparse_step', 1) != 1:
        raise NotImplementedError('qwen3_moe with dense-MLP layers (mlp_only_layers / decoder_sparse_step) is not '
                                  'supported: every layer must be MoE')
    if cfg.get('attention_bias'):
        raise NotImplementedError('qwen3_moe with attention biases is not supported')
    rope = cfg.get('rope_parameters') or cfg.get('rope_scaling') or {}
    if rope.get('rope_type', 'default') not in ('default', None):
        raise NotImplementedError(f'RoPE type {rope.get("rope_type")!r} is not supported')
    theta = cfg.get('rope_theta', rope.get('rope_theta', 1e6))
    heads = cfg['num_attention_heads']
    out = Qwen3MoeConfig(
        hidden=cfg['hidden_size'], layers=cfg['num_hidden_layers'], heads=heads,
        kv_heads=cfg.get('num_key_value_heads', heads), head_dim=cfg.get('head_dim', cfg['hidden_size'] // heads),
        experts=cfg.get('num_experts', cfg.get('num_local_experts')), top_k=cfg['num_experts_per_tok'],
        inter=cfg['moe_intermediate_size'], vocab=cfg['vocab_size'], rope_theta=float(theta),
        eps=float(cfg.get('rms_norm_eps', 1e-6)), fmt=fmt or NVFP4, norm_topk=bool(cfg.get('norm_topk_prob', True)))
    return out, bool(cfg.get('tie_word_embeddings', False))


# ---------------------------------------------------------------------------------------------------- tensors
def _ue8m0(t: torch.Tensor) -> torch.Tensor:
    """UE8M0 block scales as bytes from U8, F8_E8M0 or FP32 powers of two."""
    if t.dtype == torch.uint8:
        return t.contiguous()
    if t.dtype == torch.float8_e8m0fnu:
        return t.contiguous().view(torch.uint8)
    if t.dtype == torch.float32:
        bits = t.contiguous().view(torch.int32)
        if bool(((bits & 0x7FFFFF) != 0).logical_and((bits >> 23) != 0).any()):
            raise ValueError('an MXFP4 block scale is not a power of two')
        return ((bits >> 23) & 0xFF).to(torch.uint8)
    raise TypeError(f'MXFP4 block scales of dtype {t.dtype}')


def _scalar(t: torch.Tensor) -> float:
    return float(t.float().reshape(-1)[0])


def dense(st: SafeTensors, prefix: str) -> torch.Tensor:
    """`<prefix>.weight` as BF16 (dequantized when stored as FP8 or NVFP4)."""
    name = prefix + '.weight'
    w = st.get(name)
    if w.dtype in (torch.bfloat16, torch.float16, torch.float32):
        return w.to(torch.bfloat16)
    if w.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
        s = st.get(prefix + '.weight_scale').float() if prefix + '.weight_scale' in st else torch.ones(())
        if s.dim() == 1 and s.numel() == w.shape[0]:
            s = s[:, None]
        return (w.float() * s).to(torch.bfloat16)
    if w.dtype == torch.uint8 and prefix + '.weight_scale_2' in st:      # ModelOpt NVFP4
        out = formats.dequant(w, st.get(prefix + '.weight_scale').view(torch.uint8), NVFP4,
                              _scalar(st.get(prefix + '.weight_scale_2')))
        return out.to(torch.bfloat16)
    raise TypeError(f'{name}: dense weight of dtype {st.dtype(name)} is not supported')


def expert_format(st: SafeTensors, prefix: str) -> str:
    """'modelopt', 'ct' (compressed-tensors), 'mxfp4', 'dense' (per-expert BF16/FP16/FP32) or 'fused' for the
    experts under `prefix` (e.g. 'model.layers.0.mlp')."""
    e0 = f'{prefix}.experts.0.gate_proj'
    if f'{prefix}.experts.gate_up_proj' in st:
        return 'fused'
    if e0 + '.weight_packed' in st:
        return 'ct'
    if e0 + '.weight' not in st:
        raise KeyError(f'no experts under {prefix}')
    if e0 + '.weight_scale_2' in st:
        return 'modelopt'
    if st.dtype(e0 + '.weight') in ('U8', 'I8'):
        return 'mxfp4'
    return 'dense'


def load_experts(st: SafeTensors, prefix: str, E: int, H: int, I: int, fmt: str = NVFP4,
                 device='cpu') -> ExpertWeights:
    """The routed experts under `prefix` as ExpertWeights (CPU). `fmt` applies to unquantized checkpoints; a
    quantized one keeps its own (NVFP4 or MXFP4). `device` is where unquantized experts are quantized."""
    kind = expert_format(st, prefix)
    projs = ('gate_proj', 'up_proj', 'down_proj')
    if kind in ('dense', 'fused'):
        if kind == 'fused':
            gu = st.get(f'{prefix}.experts.gate_up_proj')
            if list(gu.shape) != [E, 2 * I, H] and list(gu.shape) == [E, H, 2 * I]:   # the transposed layout
                gu = gu.transpose(1, 2)
            w1, w3 = gu[:, :I], gu[:, I:]
            w2 = st.get(f'{prefix}.experts.down_proj')
            if list(w2.shape) != [E, H, I] and list(w2.shape) == [E, I, H]:
                w2 = w2.transpose(1, 2)
        else:
            w1 = torch.stack([st.get(f'{prefix}.experts.{e}.gate_proj.weight') for e in range(E)])
            w3 = torch.stack([st.get(f'{prefix}.experts.{e}.up_proj.weight') for e in range(E)])
            w2 = torch.stack([st.get(f'{prefix}.experts.{e}.down_proj.weight') for e in range(E)])
        dev = torch.device(device)
        out = formats.quantize_experts(w1.to(dev).float(), w3.to(dev).float(), w2.to(dev).float(), fmt)
        return out.to('cpu')
    bs = 16 if kind in ('modelopt', 'ct') else 32
    efmt = NVFP4 if bs == 16 else MXFP4
    w13 = torch.empty(E, 2 * I, H // 2, dtype=torch.uint8)
    s13 = torch.empty(E, 2 * I, H // bs, dtype=torch.uint8)
    w2 = torch.empty(E, H, I // 2, dtype=torch.uint8)
    s2 = torch.empty(E, H, I // bs, dtype=torch.uint8)
    g13 = torch.ones(E, 2)
    g2 = torch.ones(E)
    wname = {'modelopt': 'weight', 'ct': 'weight_packed', 'mxfp4': 'weight'}[kind]
    for e in range(E):
        for j, p in enumerate(projs):
            base = f'{prefix}.experts.{e}.{p}'
            w = st.get(f'{base}.{wname}').view(torch.uint8)
            if kind == 'mxfp4':
                sname = base + ('.weight_scale_inv' if base + '.weight_scale_inv' in st else '.weight_scale')
                s = _ue8m0(st.get(sname))
                g = 1.0
            else:
                s = st.get(base + '.weight_scale').view(torch.uint8)
                g = (_scalar(st.get(base + '.weight_scale_2')) if kind == 'modelopt'
                     else 1.0 / _scalar(st.get(base + '.weight_global_scale')))
            if j < 2:
                rows = slice(j * I, (j + 1) * I)
                w13[e, rows], s13[e, rows] = w, s
                g13[e, j] = g
            else:
                w2[e], s2[e] = w, s
                g2[e] = g
    return ExpertWeights(efmt, w13, w2, s13, s2, g13, g2)


class HFWeights:
    """Weight source of `Qwen3MoeModel` for a Hugging Face qwen3_moe checkpoint directory."""

    def __init__(self, path, fmt: str | None = None, quant_device='cpu'):
        from .. import config as xconfig
        self.path = Path(path)
        raw = json.loads((self.path / 'config.json').read_text())
        self.cfg, self.tied = config_from_hf(raw, fmt or xconfig.get('XTIER_CKPT_FORMAT'))
        self.st = SafeTensors(self.path)
        self.quant_device = quant_device
        p = self.prefix = 'model.' if 'model.embed_tokens.weight' in self.st else ''
        if p + 'embed_tokens.weight' not in self.st:
            raise KeyError(f'{path}: no embed_tokens.weight')
        first = expert_format(self.st, f'{p}layers.0.mlp')
        if first in ('modelopt', 'ct'):
            self.cfg.fmt = NVFP4
        elif first == 'mxfp4':
            self.cfg.fmt = MXFP4

    def embed(self) -> torch.Tensor:
        return self.st.get(self.prefix + 'embed_tokens.weight').to(torch.bfloat16)

    def lm_head(self) -> torch.Tensor:
        if self.tied or 'lm_head.weight' not in self.st:
            return self.embed()
        return dense(self.st, 'lm_head')

    def final_norm(self) -> torch.Tensor:
        return self.st.get(self.prefix + 'norm.weight').to(torch.bfloat16)

    def layer(self, li: int) -> dict:
        c, st = self.cfg, self.st
        p = f'{self.prefix}layers.{li}'
        a = f'{p}.self_attn'
        qkv = torch.cat([dense(st, f'{a}.q_proj'), dense(st, f'{a}.k_proj'), dense(st, f'{a}.v_proj')])
        return dict(
            in_norm=st.get(f'{p}.input_layernorm.weight').to(torch.bfloat16),
            post_norm=st.get(f'{p}.post_attention_layernorm.weight').to(torch.bfloat16),
            qkv=qkv, q_norm=st.get(f'{a}.q_norm.weight').to(torch.bfloat16),
            k_norm=st.get(f'{a}.k_norm.weight').to(torch.bfloat16), o=dense(st, f'{a}.o_proj'),
            router=dense(st, f'{p}.mlp.gate'),
            experts=load_experts(st, f'{p}.mlp', c.experts, c.hidden, c.inter, c.fmt, self.quant_device))

    def close(self):
        self.st.close()
