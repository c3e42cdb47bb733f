"""Cold experts in the model: XTIER_COLD with half of each layer's CPU-tier experts kept only in the drive store; the
CPU engine reads its misses from the store inside mailbox calls; logits match the fp32 reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_model_with_cold_store(cuda_ops, tmp_path, monkeypatch):
    from xtier_b200.engine.mailbox import Mailbox
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    monkeypatch.setenv('XTIER_COLD', '1')
    monkeypatch.setenv('XTIER_COLD_DIR', f'{tmp_path / "d0"},{tmp_path / "d1"}')
    monkeypatch.setenv('XTIER_COLD_FRACTION', '0.5')
    cfg = Qwen3MoeConfig.tiny(std=0.05, hidden=256, inter=128, experts=16, top_k=4)
    mb = Mailbox(cfg.hidden, timeout_s=20.0)
    model = Qwen3MoeModel(cfg, device='cuda', seed=6, hot_fraction=0.25, synthetic_experts=False,
                          engine_threads=2, mailbox=mb)
    assert model.cold is not None and model.engines and model.engines[0].shape()['slots'] == 8
    mb.start()
    try:
        prompt = torch.randint(0, cfg.vocab, (12,), generator=torch.Generator().manual_seed(7)).cuda()
        st = model.alloc_state(1, 32)
        _, lp = model.prefill(st, prompt, return_logits=True)   # 12 tokens: the decode path and the mailbox
        torch.cuda.synchronize()
        mb.check()
        ref = model.reference_logits(prompt)
        rel = float((lp.float() - ref.float()).norm() / ref.float().norm())
        assert rel < 3e-2, rel
        assert sum(e.cold_stats()['reads'] for e in model.engines) > 0
        assert model.cold.stats()['bytes_read'] > 0
    finally:
        mb.stop()
        model.cold.close()
