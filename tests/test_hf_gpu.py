"""A model built from a Hugging Face qwen3_moe checkpoint runs the GPU paths (tiered decode through the mailbox,
grouped prefill) and matches its fp32 reference forward (which tests/test_hf.py checks against transformers)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

transformers = pytest.importorskip('transformers')


def _checkpoint(path):
    cfg = transformers.Qwen3MoeConfig(
        vocab_size=512, hidden_size=256, intermediate_size=512, moe_intermediate_size=128, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=128, num_experts=8, num_experts_per_tok=2,
        norm_topk_prob=True, max_position_embeddings=4096, rope_theta=1e6, rms_norm_eps=1e-6,
        tie_word_embeddings=False, decoder_sparse_step=1, mlp_only_layers=[])
    torch.manual_seed(0)
    m = transformers.Qwen3MoeForCausalLM(cfg)
    with torch.no_grad():
        for n, p in m.named_parameters():
            p.copy_(1.0 + 0.2 * torch.randn_like(p) if 'norm' in n else 0.05 * torch.randn_like(p))
    m.to(torch.bfloat16).save_pretrained(path)


@pytest.mark.parametrize('tokens', [12, 40])
def test_loaded_checkpoint_on_the_gpu(cuda_ops, tmp_path, monkeypatch, tokens):
    from xtier_b200.engine.mailbox import Mailbox
    from xtier_b200.models.qwen3_moe import Qwen3MoeModel
    monkeypatch.setenv('XTIER_GPU_PREFILL_MIN', '16')     # 40 tokens: the grouped prefill; 12: the decode path
    _checkpoint(tmp_path)
    mb = Mailbox(256, timeout_s=20.0)
    model = Qwen3MoeModel.from_pretrained(tmp_path, device='cuda', hot_fraction=0.5, engine_threads=2, mailbox=mb)
    assert model.layers[0]['moe'].router_bias is None
    mb.start()
    try:
        prompt = torch.randint(0, 512, (tokens,), generator=torch.Generator().manual_seed(1)).cuda()
        st = model.alloc_state(1, 64)
        _, lp = model.prefill(st, prompt, return_logits=True)
        torch.cuda.synchronize()
        mb.check()
        ref = model.reference_logits(prompt)
        rel = float((lp.float() - ref.float()).norm() / ref.float().norm())
        assert rel < 3e-2, rel
    finally:
        mb.stop()
