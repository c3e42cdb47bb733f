"""Hugging Face qwen3_moe checkpoints: the loader's name mapping and expert formats, and a model built from a
checkpoint against transformers' own Qwen3-MoE forward (fp32, on the CPU, experts set to the loaded FP4 values)."""
import json

import pytest
import torch

from xtier_b200 import formats
from xtier_b200.models import hf
from xtier_b200.models.qwen3_moe import Qwen3MoeModel

transformers = pytest.importorskip('transformers')

E, H, I, L = 8, 256, 128, 2


def _hf_model(seed=0, tie=False):
    cfg = transformers.Qwen3MoeConfig(
        vocab_size=512, hidden_size=H, intermediate_size=512, moe_intermediate_size=I, num_hidden_layers=L,
        num_attention_heads=4, num_key_value_heads=2, head_dim=128, num_experts=E, num_experts_per_tok=2,
        norm_topk_prob=True, max_position_embeddings=4096, rope_theta=1e6, rms_norm_eps=1e-6,
        tie_word_embeddings=tie, decoder_sparse_step=1, mlp_only_layers=[])
    torch.manual_seed(seed)
    m = transformers.Qwen3MoeForCausalLM(cfg)
    with torch.no_grad():
        for n, p in m.named_parameters():   # norms away from 1 too, so a swapped norm shows up
            p.copy_(1.0 + 0.2 * torch.randn_like(p) if 'norm' in n else 0.05 * torch.randn_like(p))
    return m.to(torch.bfloat16)


def _fp32(m):
    """The transformers model in fp32, its RoPE frequencies rebuilt (the BF16 round trip rounded the buffer)."""
    m = m.float()
    m.model.rotary_emb = type(m.model.rotary_emb)(config=m.config)
    return m


def _set_experts(m, model):
    """Puts the loaded model's dequantized experts into the transformers model (so both compute the same thing)."""
    with torch.no_grad():
        for li, layer in enumerate(m.model.layers):
            pool = model.layers[li]['moe'].pool
            for e in range(E):
                w1, w3, w2 = pool.dequant(e)
                layer.mlp.experts.gate_up_proj[e].copy_(torch.cat([w1, w3]))
                layer.mlp.experts.down_proj[e].copy_(w2)


@pytest.mark.parametrize('tie', [False, True])
def test_model_from_checkpoint_matches_transformers(tmp_path, tie):
    m = _hf_model(seed=1, tie=tie)
    m.save_pretrained(tmp_path)
    model = Qwen3MoeModel.from_pretrained(tmp_path, device='cpu', hot_fraction=1.0)
    cfg = model.cfg
    assert (cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.experts, cfg.top_k, cfg.inter) == (H, L, 4, 2, E, 2, I)
    assert model.layers[0]['moe'].router_bias is None and cfg.norm_topk
    m = _fp32(m)
    _set_experts(m, model)
    tokens = torch.randint(0, 512, (9,), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        want = m(input_ids=tokens[None]).logits[0, -1]
    got = model.reference_logits(tokens)
    rel = float((got - want).norm() / want.norm())
    assert rel < 1e-4, rel


def _quantized_checkpoint(tmp_path, m, kind):
    """The transformers model's checkpoint with its experts stored in a quantized format: (dir, ExpertWeights per
    layer as written)."""
    m.save_pretrained(tmp_path / 'bf16')
    src = hf.SafeTensors(tmp_path / 'bf16')
    out, written = {}, []
    for name in src.names():
        if '.mlp.experts.' not in name:
            out[name] = src.get(name)
    fmt = formats.MXFP4 if kind == 'mxfp4' else formats.NVFP4
    for li in range(L):
        p = f'model.layers.{li}.mlp.experts'
        w1 = torch.stack([src.get(f'{p}.{e}.gate_proj.weight') for e in range(E)]).float()
        w3 = torch.stack([src.get(f'{p}.{e}.up_proj.weight') for e in range(E)]).float()
        w2 = torch.stack([src.get(f'{p}.{e}.down_proj.weight') for e in range(E)]).float()
        ew = formats.quantize_experts(w1, w3, w2, fmt)
        written.append(ew)
        for e in range(E):
            parts = {'gate_proj': (ew.w13[e, :I], ew.s13[e, :I], ew.g13[e, 0]),
                     'up_proj': (ew.w13[e, I:], ew.s13[e, I:], ew.g13[e, 1]),
                     'down_proj': (ew.w2[e], ew.s2[e], ew.g2[e])}
            for proj, (w, s, g) in parts.items():
                b = f'{p}.{e}.{proj}'
                if kind == 'modelopt':
                    out[b + '.weight'] = w.clone()
                    out[b + '.weight_scale'] = s.clone().view(torch.float8_e4m3fn)
                    out[b + '.weight_scale_2'] = torch.tensor(float(g))
                    out[b + '.input_scale'] = torch.tensor(1.0)
                elif kind == 'ct':
                    out[b + '.weight_packed'] = w.clone()
                    out[b + '.weight_scale'] = s.clone().view(torch.float8_e4m3fn)
                    out[b + '.weight_global_scale'] = torch.tensor([1.0 / float(g)])
                else:   # MXFP4: int8 codes, scales as FP32 powers of two in one projection, E8M0 in the others
                    out[b + '.weight'] = w.clone().view(torch.int8)
                    out[b + '.weight_scale_inv'] = (torch.pow(2.0, s.float() - 127.0) if proj == 'up_proj'
                                                    else s.clone().view(torch.float8_e8m0fnu))
    d = tmp_path / kind
    d.mkdir()
    hf.save_safetensors(d / 'model.safetensors', out)
    (d / 'config.json').write_text((tmp_path / 'bf16' / 'config.json').read_text())
    return d, written


@pytest.mark.parametrize('kind', ['modelopt', 'ct', 'mxfp4'])
def test_quantized_expert_formats_load_byte_exact(tmp_path, kind):
    m = _hf_model(seed=3)
    d, written = _quantized_checkpoint(tmp_path, m, kind)
    w = hf.HFWeights(d)
    assert w.cfg.fmt == (formats.MXFP4 if kind == 'mxfp4' else formats.NVFP4)
    for li in range(L):
        got = w.layer(li)['experts']
        want = written[li]
        for f in ('w13', 'w2', 's13', 's2'):
            assert torch.equal(getattr(got, f), getattr(want, f)), (li, f)
        assert torch.allclose(got.g13, want.g13.float(), rtol=1e-6) and torch.allclose(got.g2, want.g2.float(),
                                                                                        rtol=1e-6)
    w.close()
    model = Qwen3MoeModel.from_pretrained(d, device='cpu', hot_fraction=1.0)
    m = _fp32(m)
    _set_experts(m, model)
    tokens = torch.randint(0, 512, (6,), generator=torch.Generator().manual_seed(4))
    with torch.no_grad():
        want = m(input_ids=tokens[None]).logits[0, -1]
    rel = float((model.reference_logits(tokens) - want).norm() / want.norm())
    assert rel < 1e-4, rel


def test_fused_bf16_experts_and_fp8_dense(tmp_path):
    """Fused gate_up_proj / down_proj tensors quantize like the per-expert ones; an FP8 dense weight is scaled."""
    m = _hf_model(seed=5)
    m.save_pretrained(tmp_path / 'a')
    src = hf.SafeTensors(tmp_path / 'a')
    out = {n: src.get(n) for n in src.names() if '.mlp.experts.' not in n}
    for li in range(L):
        p = f'model.layers.{li}.mlp.experts'
        out[f'{p}.gate_up_proj'] = torch.stack([torch.cat([src.get(f'{p}.{e}.gate_proj.weight'),
                                                           src.get(f'{p}.{e}.up_proj.weight')]) for e in range(E)])
        out[f'{p}.down_proj'] = torch.stack([src.get(f'{p}.{e}.down_proj.weight') for e in range(E)])
    o = out['model.layers.0.self_attn.o_proj.weight'].float()
    scale = o.abs().amax() / 448.0
    out['model.layers.0.self_attn.o_proj.weight'] = (o / scale).to(torch.float8_e4m3fn)
    out['model.layers.0.self_attn.o_proj.weight_scale'] = scale.reshape(())
    d = tmp_path / 'b'
    d.mkdir()
    hf.save_safetensors(d / 'model.safetensors', out)
    (d / 'config.json').write_text((tmp_path / 'a' / 'config.json').read_text())
    a, b = hf.HFWeights(tmp_path / 'a'), hf.HFWeights(d)
    assert hf.expert_format(b.st, 'model.layers.0.mlp') == 'fused'
    la, lb = a.layer(0), b.layer(0)
    for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):
        assert torch.equal(getattr(la['experts'], f), getattr(lb['experts'], f)), f
    fp8 = out['model.layers.0.self_attn.o_proj.weight'].float() * scale
    assert torch.equal(lb['o'], fp8.to(torch.bfloat16))
    rel = float((lb['o'].float() - o).norm() / o.norm())
    assert rel < 0.05
    a.close()
    b.close()


def test_config_mapping_and_refusals():
    base = dict(model_type='qwen3_moe', hidden_size=2048, num_hidden_layers=48, num_attention_heads=32,
                num_key_value_heads=4, head_dim=128, num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768,
                vocab_size=151936, rope_theta=1e6, rms_norm_eps=1e-6, norm_topk_prob=True, tie_word_embeddings=False)
    cfg, tied = hf.config_from_hf(base)
    assert (cfg.hidden, cfg.layers, cfg.experts, cfg.inter, cfg.rope_theta, tied) == (2048, 48, 128, 768, 1e6, False)
    v5 = dict(base, num_local_experts=64, rope_parameters={'rope_theta': 5e5, 'rope_type': 'default'})
    del v5['num_experts'], v5['rope_theta']
    cfg, _ = hf.config_from_hf(v5)
    assert cfg.experts == 64 and cfg.rope_theta == 5e5
    for bad in (dict(base, mlp_only_layers=[0]), dict(base, model_type='llama'),
                dict(base, rope_scaling={'rope_type': 'yarn', 'factor': 4.0})):
        with pytest.raises(NotImplementedError):
            hf.config_from_hf(bad)
    json.dumps(base)


def test_bf16_experts_quantized_to_the_chosen_format(tmp_path):
    """Unquantized experts follow `fmt` (XTIER_CKPT_FORMAT): MXFP4 here, dequantizing close to the BF16 weights."""
    m = _hf_model(seed=6)
    m.save_pretrained(tmp_path)
    w = hf.HFWeights(tmp_path, fmt=formats.MXFP4)
    ew = w.layer(1)['experts']
    assert ew.fmt == formats.MXFP4 and ew.s13.shape[-1] == H // 32
    src = w.st.get('model.layers.1.mlp.experts.2.gate_proj.weight').float()
    w1, _, _ = ew.dequant(2)
    assert float((w1 - src).norm() / src.norm()) < 0.2
    w.close()
